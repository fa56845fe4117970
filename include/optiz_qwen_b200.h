/*
 * optiz_qwen_b200 -- C ABI of the B200 decode hot path for the Qwen3.5 hybrid LM.
 *
 * Every entry point takes plain device pointers, sizes, element strides and a
 * cudaStream_t (passed as void*), enqueues its kernels on that stream and
 * returns an oq_status code.  Nothing here allocates device memory, frees it or
 * synchronises the stream; scratch comes from caller-provided workspaces.  No
 * entry point aborts the process.  All pointers are device pointers unless a
 * comment says otherwise.
 *
 * Storage of the paged INT4 KV cache (one pool per attention layer):
 *   kv_codes  uint8   [num_pages, num_kv_heads, 2, page_size, head_dim/2]
 *             index 2: 0 = keys, 1 = values; byte j of a token row holds
 *             dimension 2j in its low nibble and 2j+1 in its high nibble.
 *             The 8-bit cache (the *_int8 entry points) has rows of head_dim
 *             bytes, one code per dimension, and the same meta.
 *   kv_meta   fp16    [num_pages, num_kv_heads, 4, page_size]
 *             index 4: 0 = key scale, 1 = key min, 2 = value scale, 3 = value min.
 *   block_table int32 [batch, block_table_stride]  physical page of each logical page.
 *   seq_lens  int32   [batch]  tokens held by each sequence.
 * Dequantised value = min + code * scale (the reference's asymmetric "zero" is
 * an additive minimum).
 */
#ifndef OPTIZ_QWEN_B200_H
#define OPTIZ_QWEN_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ------------------------------------------------------------------ status */
enum oq_status {
  OQ_OK = 0,
  OQ_ERR_INVALID_ARGUMENT = 1,  /* null pointer, negative size, bad stride */
  OQ_ERR_UNSUPPORTED = 2,       /* shape / dtype / bit width this build does not implement */
  OQ_ERR_MISALIGNED = 3,        /* pointer or stride breaks a 16-byte vector / TMA rule */
  OQ_ERR_WORKSPACE = 4,         /* workspace missing or too small */
  OQ_ERR_CUDA = 5               /* a CUDA runtime / driver call failed (see oq_last_error) */
};

/* Element types for the dtype arguments. */
enum oq_dtype { OQ_F32 = 0, OQ_F16 = 1, OQ_BF16 = 2 };

/* Bits a kernel ORs into the optional device status word when it meets bad data. */
enum oq_device_status {
  OQ_DEV_BAD_PAGE = 1,     /* block_table entry outside [0, num_pages): page skipped */
  OQ_DEV_OVERFLOW = 2,     /* position beyond max_pages_per_seq * page_size: token skipped */
  OQ_DEV_TIMEOUT = 4       /* a bounded wait on a copy ran out: the CTA gave up */
};

/* Flags of oq_gdn_recurrent. */
enum oq_gdn_flags {
  /* Launch with programmatic stream serialisation and read the state before the
   * preceding kernel in the stream has finished: set only when no kernel still
   * running ahead of this call writes initial_state (in a decode step the state of
   * layer l is written only by layer l's previous step).  q/k/v/g/beta are always
   * read after the preceding kernel finishes.  Pays off when the preceding kernel
   * is another GDN step. */
  OQ_GDN_STATE_PREFETCH = 1
};

/* Flags of oq_decode_attn_paged_ex and oq_decode_attn_int4_paged_xrank. */
enum oq_attn_flags {
  /* Launch with programmatic stream serialisation and read seq_lens, the block table and the
   * cached pages (all but the page that receives an appended token) before the kernel ahead
   * in the stream has finished: set only when that kernel writes none of them (in a decode
   * step: the previous layer's kernels).  The query, the appended key / value and the gate
   * are always read after it finishes, and every write comes after that too. */
  OQ_ATTN_EARLY = 1
};

/* Static description of an oq_status value. */
const char* oq_status_string(int status);
/* Detail of the last failing call on this host thread ("" when none). */
const char* oq_last_error(void);
/* ABI version: bumped when a signature changes. */
int oq_abi_version(void);

/* Test hook (no reference counterpart): sets how many times a kernel polls a copy's
 * mbarrier before it gives up, reports OQ_DEV_TIMEOUT in the device status word and
 * winds down (each poll sleeps up to ~20 us; the default, 100000, is about 2 s).  It
 * applies to launches made after the call, process-wide.  0 makes every bounded wait
 * run out at once while the copies themselves still land, which is how the tests drive
 * the timeout path without faulting or hanging a GPU.  Before a CTA exits it waits for
 * its own copies with the default limit, whatever this setting.  polls < 0 restores the
 * default.  Returns the previous value. */
int oq_debug_set_wait_polls(int polls);

/* ------------------------------------------------------------------ append-quantize
 * Replaces QServeAttentionLayer._append_keys/_append_values/_quantize_and_append_*
 * + _quantize_groupwise + _pack_uint4
 * (optiz_qwen/compression/qserve_kv_cache.py:210-232, 278-292, 313-335, 356-362)
 * with group_size = head_dim, fp16 scale/min, paged storage and no dense window.
 *
 * key/value: [batch, num_kv_heads, num_new, head_dim] in `dtype` (F32/F16/BF16),
 * last dimension contiguous, other strides in elements.  Token t of sequence b
 * is written at position seq_lens[b] + t.  Codes use the fp32 scale/min
 * (round-half-even of (x - min) / scale, clamped to [0, 15]); the stored
 * scale/min are the fp32 values rounded to fp16.  When advance_seq_lens != 0
 * seq_lens[b] += num_new on exit (stream-ordered).  device_status may be NULL.
 */
int oq_append_quant_int4(
    const void* key, const void* value, int dtype,
    int64_t batch, int64_t num_kv_heads, int64_t num_new, int64_t head_dim,
    int64_t key_stride_b, int64_t key_stride_h, int64_t key_stride_t,
    int64_t value_stride_b, int64_t value_stride_h, int64_t value_stride_t,
    uint8_t* kv_codes, uint16_t* kv_meta, int64_t num_pages, int64_t page_size,
    const int32_t* block_table, int64_t block_table_stride, int64_t max_pages_per_seq,
    int32_t* seq_lens, int advance_seq_lens,
    int32_t* device_status, void* stream);

/* The 8-bit cache format (the reference's k_bits = v_bits = 8 path, _quantize_groupwise with
 * bits = 8): codes [num_pages, num_kv_heads, 2, page_size, head_dim] one byte per element,
 * 255 levels (round-half-even of (x - min) / scale clamped to [0, 255], scale = (max - min) / 255),
 * same fp16 scale/min, same arguments and contract as oq_append_quant_int4. */
int oq_append_quant_int8(
    const void* key, const void* value, int dtype,
    int64_t batch, int64_t num_kv_heads, int64_t num_new, int64_t head_dim,
    int64_t key_stride_b, int64_t key_stride_h, int64_t key_stride_t,
    int64_t value_stride_b, int64_t value_stride_h, int64_t value_stride_t,
    uint8_t* kv_codes, uint16_t* kv_meta, int64_t num_pages, int64_t page_size,
    const int32_t* block_table, int64_t block_table_stride, int64_t max_pages_per_seq,
    int32_t* seq_lens, int advance_seq_lens,
    int32_t* device_status, void* stream);

/* seq_lens[b] += delta for b < batch (cache bookkeeping between steps). */
int oq_advance_seq_lens(int32_t* seq_lens, int64_t batch, int32_t delta, void* stream);

/* ------------------------------------------------------------------ decode attention
 * Replaces qserve_int4_decode_attention / qserve_int4_split_decode_attention
 * (optiz_qwen/kernels/qserve_int4_attention.py:520-545, 576-620) and their
 * Triton kernels (:112-205, :209-261, :328-395).
 *
 * One query token per sequence: query [batch, num_heads, head_dim] (BF16 or
 * F16, element strides for batch and head, last dim contiguous) attends over
 * seq_lens[b] cached tokens of KV head h / (num_heads / num_kv_heads); scores
 * are scaling * q.k.  head_dim must be 256 and num_heads / num_kv_heads <= 8
 * in this build.  The KV range of each (sequence, KV head) is cut into
 * num_splits page ranges (num_splits <= 0: chosen from the grid size); the
 * partial (max, sum, acc) of each range are merged by log-sum-exp inside the
 * same launch.
 *
 * Outputs (each may be NULL, at least one must be given):
 *   out      [batch, num_heads, head_dim] in the query dtype, strides in elements;
 *   out_f32  [batch, num_heads, head_dim] fp32, contiguous;
 *   out_lse  [batch, num_heads] fp32 natural-log log-sum-exp of the scores
 *            (-inf for an empty sequence, whose output row is 0).
 * workspace: oq_decode_attn_workspace_bytes(...) bytes, zero-filled once before
 * its first use; every launch leaves its counters at zero again.  Launches that
 * share a workspace must be ordered on one stream.
 */
size_t oq_decode_attn_workspace_bytes(int64_t batch, int64_t num_heads, int64_t num_kv_heads,
                                      int64_t head_dim, int64_t max_splits);

int oq_decode_attn_int4_paged(
    const void* query, int dtype, int64_t query_stride_b, int64_t query_stride_h,
    const uint8_t* kv_codes, const uint16_t* kv_meta, int64_t num_pages, int64_t page_size,
    const int32_t* block_table, int64_t block_table_stride, int64_t max_pages_per_seq,
    const int32_t* seq_lens,
    int64_t batch, int64_t num_heads, int64_t num_kv_heads, int64_t head_dim,
    float scaling,
    void* out, int64_t out_stride_b, int64_t out_stride_h,
    float* out_f32, float* out_lse,
    void* workspace, size_t workspace_bytes, int num_splits,
    int32_t* device_status, void* stream);

/* The same attention over the 8-bit cache of oq_append_quant_int8 (codes
 * [num_pages, num_kv_heads, 2, page_size, head_dim], one byte per element): replaces
 * qserve_int8_decode_attention and its Triton kernel (qserve_int4_attention.py:18-109,
 * 548-573).  Same arguments and contract as oq_decode_attn_int4_paged. */
int oq_decode_attn_int8_paged(
    const void* query, int dtype, int64_t query_stride_b, int64_t query_stride_h,
    const uint8_t* kv_codes, const uint16_t* kv_meta, int64_t num_pages, int64_t page_size,
    const int32_t* block_table, int64_t block_table_stride, int64_t max_pages_per_seq,
    const int32_t* seq_lens,
    int64_t batch, int64_t num_heads, int64_t num_kv_heads, int64_t head_dim,
    float scaling,
    void* out, int64_t out_stride_b, int64_t out_stride_h,
    float* out_f32, float* out_lse,
    void* workspace, size_t workspace_bytes, int num_splits,
    int32_t* device_status, void* stream);

/* Same attention with the decode forward's output gate fused into the store:
 * out = rnd(rnd(o) * rnd(sigmoid(gate))) in the query dtype (rnd = rounding to it),
 * replacing ``attn_output * torch.sigmoid(gate)`` after the kernel
 * (optiz_qwen/kernels/qwen35_fused_attention.py:96-97).  gate [batch, num_heads, head_dim]
 * in the query dtype with element strides (b, h), the half of q_proj's output that is
 * not the query.  out is required; no fp32 / lse outputs (they feed merges, which
 * must see the ungated values). */
int oq_decode_attn_int4_paged_gated(
    const void* query, int dtype, int64_t query_stride_b, int64_t query_stride_h,
    const uint8_t* kv_codes, const uint16_t* kv_meta, int64_t num_pages, int64_t page_size,
    const int32_t* block_table, int64_t block_table_stride, int64_t max_pages_per_seq,
    const int32_t* seq_lens,
    int64_t batch, int64_t num_heads, int64_t num_kv_heads, int64_t head_dim,
    float scaling,
    const void* gate, int64_t gate_stride_b, int64_t gate_stride_h,
    void* out, int64_t out_stride_b, int64_t out_stride_h,
    void* workspace, size_t workspace_bytes, int num_splits,
    int32_t* device_status, void* stream);

/* The gated attention over the 8-bit cache; same arguments and contract as
 * oq_decode_attn_int4_paged_gated. */
int oq_decode_attn_int8_paged_gated(
    const void* query, int dtype, int64_t query_stride_b, int64_t query_stride_h,
    const uint8_t* kv_codes, const uint16_t* kv_meta, int64_t num_pages, int64_t page_size,
    const int32_t* block_table, int64_t block_table_stride, int64_t max_pages_per_seq,
    const int32_t* seq_lens,
    int64_t batch, int64_t num_heads, int64_t num_kv_heads, int64_t head_dim,
    float scaling,
    const void* gate, int64_t gate_stride_b, int64_t gate_stride_h,
    void* out, int64_t out_stride_b, int64_t out_stride_h,
    void* workspace, size_t workspace_bytes, int num_splits,
    int32_t* device_status, void* stream);

/* Decode attention with the options of a decode step: an appended token, a gate and launch
 * flags, over the `bits`-bit cache (4 or 8).  With new_key / new_value [batch, num_kv_heads,
 * head_dim] (query dtype, last dim contiguous, rows 16-byte aligned) the launch is append +
 * attend in one (no reference counterpart as one call: it fuses the cache layer's update --
 * QServeAttentionLayer._append_decode_token / _quantize_groupwise, qserve_kv_cache.py:200-232,
 * 313-335 -- with the decode attention that follows it, qserve_int4_attention.py:520-545,
 * 576-620): the token is quantised into the cache at position seq_lens[b], with the same codes
 * and fp16 scale / min as oq_append_quant_int4 / _int8, and the query attends over the
 * seq_lens[b] + 1 tokens.  seq_lens is not modified (advance it with oq_advance_seq_lens, or
 * keep it to hold the context).  Both NULL: no token is appended.  gate may be NULL (else as
 * oq_decode_attn_int4_paged_gated: out only); other arguments as oq_decode_attn_int4_paged;
 * flags: OQ_ATTN_EARLY or 0. */
int oq_decode_attn_paged_ex(
    int bits, const void* query, int dtype, int64_t query_stride_b, int64_t query_stride_h,
    const void* new_key, int64_t key_stride_b, int64_t key_stride_h,
    const void* new_value, int64_t value_stride_b, int64_t value_stride_h,
    uint8_t* kv_codes, uint16_t* kv_meta, int64_t num_pages, int64_t page_size,
    const int32_t* block_table, int64_t block_table_stride, int64_t max_pages_per_seq,
    const int32_t* seq_lens,
    int64_t batch, int64_t num_heads, int64_t num_kv_heads, int64_t head_dim,
    float scaling,
    const void* gate, int64_t gate_stride_b, int64_t gate_stride_h,
    void* out, int64_t out_stride_b, int64_t out_stride_h,
    float* out_f32, float* out_lse,
    void* workspace, size_t workspace_bytes, int num_splits, int flags,
    int32_t* device_status, void* stream);

/* Same attention, for callers that cannot allocate device memory (no counterpart
 * in the reference, which only runs inside PyTorch's allocator).  A decode loop
 * embedded in a host runtime whose arena owns all device memory, or a
 * foreign-language caller holding only buffers allocated by someone else, has
 * no way to provide the workspace above.  This variant takes its split-KV
 * scratch from a fixed 8 MiB array compiled into the library (held on every
 * GPU that loads it until exit) and calls no allocator.  The caller still
 * passes inputs and outputs.  An explicit num_splits whose scratch exceeds
 * 8 MiB is rejected with OQ_ERR_WORKSPACE; num_splits <= 0 picks the usual
 * split count capped to fit.  All calls share the array: its merge counters are
 * cleared on `stream` at the start of each call, and calls that overlap on the
 * GPU race.  The first call on a device looks up the array's address with that
 * device current; make it before any stream capture. */
int oq_decode_attn_int4_paged_noalloc(
    const void* query, int dtype, int64_t query_stride_b, int64_t query_stride_h,
    const uint8_t* kv_codes, const uint16_t* kv_meta, int64_t num_pages, int64_t page_size,
    const int32_t* block_table, int64_t block_table_stride, int64_t max_pages_per_seq,
    const int32_t* seq_lens,
    int64_t batch, int64_t num_heads, int64_t num_kv_heads, int64_t head_dim,
    float scaling,
    void* out, int64_t out_stride_b, int64_t out_stride_h,
    float* out_f32, float* out_lse,
    int num_splits, int32_t* device_status, void* stream);

/* ------------------------------------------------------------------ log-sum-exp merge
 * Combines attention partials computed over disjoint KV ranges (another GPU's
 * slice of a long context, gathered over NVLink):
 *   out = sum_i exp(lse_i - L) * part_out_i,  L = log sum_i exp(lse_i).
 * part_out [num_parts, rows, head_dim] fp32, part_lse [num_parts, rows] fp32;
 * out [rows, head_dim] in `dtype`; out_lse [rows] fp32 or NULL.
 * No reference counterpart (the reference runs on one GPU).
 */
int oq_lse_merge(const float* part_out, const float* part_lse,
                 int64_t num_parts, int64_t rows, int64_t head_dim,
                 void* out, int dtype, float* out_lse, void* stream);

/* ------------------------------------------------------------------ exchange over NVLink
 * The long-context exchange of (out, lse) partials without NCCL: each rank stores its
 * merged rows straight into every other rank's receive buffer over NVLink (plain stores,
 * CUDA IPC mappings, no multicast object), raises a per-row flag there, waits (bounded)
 * for every rank's flag in its own buffer and merges with the arithmetic of oq_lse_merge,
 * in the same order, so the result is bit-identical to the all-gather + oq_lse_merge path.
 * No reference counterpart (the reference runs on one GPU).
 *
 * Set-up, once per rank and buffer:
 *   oq_xrank_buffer_bytes(rows, head_dim, world): bytes of one call site's receive buffer
 *     (0 for bad sizes).  Allocate one per call site (e.g. per attention layer), zeroed; it
 *     also holds this rank's per-row call counters, so a CUDA graph replay works.
 *   oq_ipc_export(ptr, handle, &offset): writes oq_ipc_handle_bytes() bytes of IPC handle
 *     for the device allocation holding ptr, and ptr's offset in it.  Exchange handles and
 *     offsets between the ranks by any host channel.
 *   oq_ipc_import(handle, offset, &ptr): maps a peer's allocation into this process.
 *   oq_ipc_close(ptr, offset): unmaps it (after every rank's last exchange).
 * Per call (peer_buffers: device array [world] of every rank's buffer for this call site,
 * this rank's own at [rank]; every rank calls each call site the same number of times, in
 * the same order, and calls at one call site are ordered on one stream; a rank whose peers
 * do not arrive within ~2 s sets OQ_DEV_TIMEOUT in device_status and merges what it has):
 *   oq_xrank_lse_merge: part_out [rows, head_dim] fp32, part_lse [rows] fp32 (an earlier
 *     kernel's partial) -> out [rows, head_dim] in `dtype`, out_lse [rows] or NULL.
 *   oq_decode_attn_int4_paged_xrank: oq_decode_attn_int4_paged over this rank's KV range
 *     whose split merge exchanges every merged row in the same launch (no fp32 partial round
 *     trip, no separate exchange kernel); `out` / out_f32 / out_lse receive the merge over
 *     all ranks (rows = batch x num_heads).  The workspace is required (its size for
 *     `num_splits` as for oq_decode_attn_int4_paged, at least one split). */
size_t oq_xrank_buffer_bytes(int64_t rows, int64_t head_dim, int64_t world);
size_t oq_ipc_handle_bytes(void);
int oq_ipc_export(const void* ptr, void* handle, int64_t* offset);
int oq_ipc_import(const void* handle, int64_t offset, void** ptr);
int oq_ipc_close(void* ptr, int64_t offset);
int oq_xrank_lse_merge(const float* part_out, const float* part_lse, int64_t rows, int64_t head_dim,
                       float* const* peer_buffers, int rank, int world,
                       void* out, int dtype, float* out_lse, int32_t* device_status, void* stream);
int oq_decode_attn_int4_paged_xrank(
    const void* query, int dtype, int64_t query_stride_b, int64_t query_stride_h,
    const uint8_t* kv_codes, const uint16_t* kv_meta, int64_t num_pages, int64_t page_size,
    const int32_t* block_table, int64_t block_table_stride, int64_t max_pages_per_seq,
    const int32_t* seq_lens,
    int64_t batch, int64_t num_heads, int64_t num_kv_heads, int64_t head_dim,
    float scaling,
    void* out, int64_t out_stride_b, int64_t out_stride_h,
    float* out_f32, float* out_lse,
    void* workspace, size_t workspace_bytes, int num_splits,
    float* const* peer_buffers, int rank, int world, int flags,
    int32_t* device_status, void* stream);

/* ------------------------------------------------------------------ paged gather
 * Replaces QServeAttentionLayer.materialize / _dequantize_groupwise / _unpack_uint4
 * (qserve_kv_cache.py:126-135, 294-353, 365-372): writes the dequantised cache
 * of every sequence, positions [0, length) with length = min(seq_lens[b], max_len),
 * into keys/values [batch, num_kv_heads, max_len, head_dim] (`dtype`, contiguous).
 * Rows at or beyond a sequence's length are left untouched.
 */
int oq_gather_dequant_int4(
    const uint8_t* kv_codes, const uint16_t* kv_meta, int64_t num_pages, int64_t page_size,
    const int32_t* block_table, int64_t block_table_stride, int64_t max_pages_per_seq,
    const int32_t* seq_lens, int64_t batch, int64_t num_kv_heads, int64_t head_dim,
    int64_t max_len, void* keys, void* values, int dtype,
    int32_t* device_status, void* stream);

/* The same gather over the 8-bit cache of oq_append_quant_int8 (the reference's
 * _dequantize_groupwise with bits = 8, qserve_kv_cache.py:337-353, 126-135). */
int oq_gather_dequant_int8(
    const uint8_t* kv_codes, const uint16_t* kv_meta, int64_t num_pages, int64_t page_size,
    const int32_t* block_table, int64_t block_table_stride, int64_t max_pages_per_seq,
    const int32_t* seq_lens, int64_t batch, int64_t num_kv_heads, int64_t head_dim,
    int64_t max_len, void* keys, void* values, int dtype,
    int32_t* device_status, void* stream);

/* ------------------------------------------------------------------ gated delta rule: recurrent
 * Replaces the GDN hook `recurrent_gated_delta_rule` = fla 0.5.1
 * fused_recurrent_gated_delta_rule (fla/ops/gated_delta_rule/fused_recurrent.py:291)
 * or transformers torch_recurrent_gated_delta_rule
 * (models/qwen3_5/modeling_qwen3_5.py:314-353), called from the decode branch
 * of Qwen3_5GatedDeltaNet.forward (:511-520).
 *
 * q, k [batch, seq_len, num_heads, k_dim]; v [batch, seq_len, num_heads, v_dim]
 * in qkv_dtype, element strides (b, t, h), last dim contiguous.
 * g, beta [batch, seq_len, num_heads] contiguous, in g_dtype / beta_dtype.
 * initial_state [batch, num_heads, k_dim, v_dim] fp32 or NULL (zeros);
 * final_state same shape or NULL; it may alias initial_state (in place).
 * out [batch, seq_len, num_heads, v_dim] contiguous in qkv_dtype.
 * Per token: S *= exp(g); kv = S^T k; delta = beta (v - kv); S += k delta^T;
 * o = S^T (scale q).  With use_qk_l2norm, q and k are first scaled by
 * 1/sqrt(sum(x^2) + 1e-6).  k_dim = v_dim = 128 in this build.
 * flags: OQ_GDN_STATE_PREFETCH or 0.  device_status (nullable) gets OQ_DEV_TIMEOUT if the
 * bounded wait on a state copy gives up; that slice's state and outputs are then left
 * untouched.
 */
int oq_gdn_recurrent(
    const void* q, const void* k, const void* v, int qkv_dtype,
    int64_t q_stride_b, int64_t q_stride_t, int64_t q_stride_h,
    int64_t k_stride_b, int64_t k_stride_t, int64_t k_stride_h,
    int64_t v_stride_b, int64_t v_stride_t, int64_t v_stride_h,
    const void* g, int g_dtype, const void* beta, int beta_dtype,
    const float* initial_state, float* final_state, void* out,
    int64_t batch, int64_t seq_len, int64_t num_heads, int64_t k_dim, int64_t v_dim,
    float scale, int use_qk_l2norm, int flags, int32_t* device_status, void* stream);

/* oq_gdn_recurrent with the layer's gate arithmetic fused in: instead of g and beta it
 * takes the raw projections a, b [batch, seq_len, num_heads] (contiguous, ab_dtype) and the
 * layer's A_log and dt_bias [num_heads] (their own dtypes), and computes per token, as the
 * decode branch of Qwen3_5GatedDeltaNet.forward does before calling the hook (transformers
 * models/qwen3_5/modeling_qwen3_5.py:492-493): beta = sigmoid(b) rounded to ab_dtype, and in
 * fp32 g = -exp(A_log) * softplus(a + dt_bias) (softplus(x) = x for x > 20).  The rest of
 * the contract is oq_gdn_recurrent's. */
int oq_gdn_recurrent_gates(
    const void* q, const void* k, const void* v, int qkv_dtype,
    int64_t q_stride_b, int64_t q_stride_t, int64_t q_stride_h,
    int64_t k_stride_b, int64_t k_stride_t, int64_t k_stride_h,
    int64_t v_stride_b, int64_t v_stride_t, int64_t v_stride_h,
    const void* a, const void* b, int ab_dtype, const void* a_log, int a_log_dtype, const void* dt_bias,
    int dt_bias_dtype,
    const float* initial_state, float* final_state, void* out,
    int64_t batch, int64_t seq_len, int64_t num_heads, int64_t k_dim, int64_t v_dim,
    float scale, int use_qk_l2norm, int flags, int32_t* device_status, void* stream);

/* oq_gdn_recurrent with the GDN layer's output norm fused in:
 * out = Qwen3_5RMSNormGated(o, z) per head (transformers models/qwen3_5/modeling_qwen3_5.py:175-190,
 * applied at :527-529) = rnd(rnd(rnd(o * rsqrt(mean(o^2) + norm_eps)) * w) * silu(z)), with o
 * first rounded to qkv_dtype as the unfused layer hands it on.  z [batch, seq_len, num_heads,
 * v_dim] in qkv_dtype (element strides b, t, h; unit stride along v_dim), norm_weight [v_dim]
 * in qkv_dtype.  norm_workspace: oq_gdn_norm_workspace_bytes(batch, num_heads) bytes,
 * zero-filled once before first use; every launch leaves it zero (launches sharing one must
 * be ordered on a stream).  The last of a head's four column-slice CTAs to finish normalises
 * the head's outputs, so none waits for another. */
size_t oq_gdn_norm_workspace_bytes(int64_t batch, int64_t num_heads);

int oq_gdn_recurrent_norm(
    const void* q, const void* k, const void* v, int qkv_dtype,
    int64_t q_stride_b, int64_t q_stride_t, int64_t q_stride_h,
    int64_t k_stride_b, int64_t k_stride_t, int64_t k_stride_h,
    int64_t v_stride_b, int64_t v_stride_t, int64_t v_stride_h,
    const void* g, int g_dtype, const void* beta, int beta_dtype,
    const float* initial_state, float* final_state, void* out,
    int64_t batch, int64_t seq_len, int64_t num_heads, int64_t k_dim, int64_t v_dim,
    float scale, int use_qk_l2norm,
    const void* z, int64_t z_stride_b, int64_t z_stride_t, int64_t z_stride_h,
    const void* norm_weight, float norm_eps, void* norm_workspace, size_t norm_workspace_bytes,
    int flags, void* stream);

/* One GDN decode token with the layer's causal conv1d update fused in front of it.
 * Replaces, for the decode branch of Qwen3_5GatedDeltaNet.forward
 * (transformers models/qwen3_5/modeling_qwen3_5.py:454-520), the pair
 * causal_conv1d_update (:210-225) + recurrent_gated_delta_rule, reading the
 * projection output directly.
 * qkv [batch, C] in qkv_dtype (row stride qkv_stride_b, channels contiguous), with
 * C = num_heads * (2 k_dim + v_dim) ordered q heads | k heads | v heads;
 * conv_state [batch, C, conv_width] contiguous in qkv_dtype, updated in place;
 * conv_weight [C, conv_kernel_size], conv_bias [C] or NULL, in conv_w_dtype; this fused
 * form needs conv_kernel_size = conv_width = 4 and conv_w_dtype = qkv_dtype.
 * q, k, v = silu(conv) rounded to qkv_dtype, then the recurrent step of
 * oq_gdn_recurrent (same state / out / flags contract, seq_len = 1). */
int oq_gdn_conv_step(
    const void* qkv, int qkv_dtype, int64_t qkv_stride_b,
    void* conv_state, const void* conv_weight, const void* conv_bias, int conv_w_dtype,
    int64_t conv_width, int64_t conv_kernel_size,
    const void* g, int g_dtype, const void* beta, int beta_dtype,
    const float* initial_state, float* final_state, void* out,
    int64_t batch, int64_t num_heads, int64_t k_dim, int64_t v_dim,
    float scale, int use_qk_l2norm, int flags, void* stream);

/* oq_gdn_conv_step with the output norm of oq_gdn_recurrent_norm (z [batch, num_heads,
 * v_dim] with element strides b, h): conv update, recurrent step and gated RMSNorm of
 * the decode branch (modeling_qwen3_5.py:454-529) in one launch. */
int oq_gdn_conv_step_norm(
    const void* qkv, int qkv_dtype, int64_t qkv_stride_b,
    void* conv_state, const void* conv_weight, const void* conv_bias, int conv_w_dtype,
    int64_t conv_width, int64_t conv_kernel_size,
    const void* g, int g_dtype, const void* beta, int beta_dtype,
    const float* initial_state, float* final_state, void* out,
    int64_t batch, int64_t num_heads, int64_t k_dim, int64_t v_dim,
    float scale, int use_qk_l2norm,
    const void* z, int64_t z_stride_b, int64_t z_stride_h, const void* norm_weight, float norm_eps,
    void* norm_workspace, size_t norm_workspace_bytes, int flags, void* stream);

/* Gated RMSNorm as a standalone op: replaces Qwen3_5RMSNormGated.forward
 * (transformers models/qwen3_5/modeling_qwen3_5.py:175-190) for callers that keep the
 * norm a separate module.  rows of dim elements: x, z, out with row strides (elements,
 * rows contiguous along dim), weight [dim]; all in dtype.  dim <= 1024.
 * out = rnd(rnd(rnd(x * rsqrt(mean(x^2) + eps)) * weight) * silu(z)). */
int oq_rmsnorm_gated(const void* x, int64_t x_stride, const void* z, int64_t z_stride, const void* weight,
                     void* out, int64_t out_stride, int dtype, int64_t rows, int64_t dim, float eps,
                     void* stream);

/* Causal depthwise conv1d update (the GDN layer's short convolution).
 * Replaces the hook causal_conv1d_update (transformers torch_causal_conv1d_update,
 * models/qwen3_5/modeling_qwen3_5.py:210-225; causal-conv1d 1.6.2).
 * x [batch, channels, seq_len] with element strides (b, c, t), in dtype;
 * conv_state [batch, channels, state_width] contiguous in dtype, updated in place to
 * the last state_width inputs of [state | x]; weight [channels, kernel_size] and bias
 * [channels] (or NULL) in w_dtype; out [batch, channels, seq_len] contiguous in dtype:
 * out[t] = act(bias + sum_k weight[k] * [state | x][state_width + t - kernel_size + 1 + k]),
 * act = silu when silu != 0.  kernel_size 2..4 with state_width kernel_size - 1 or
 * kernel_size; w_dtype is dtype or OQ_F32. */
int oq_causal_conv1d_update(const void* x, int dtype, int64_t x_stride_b, int64_t x_stride_c, int64_t x_stride_t,
                            void* conv_state, const void* weight, const void* bias, int w_dtype, void* out,
                            int64_t batch, int64_t channels, int64_t seq_len, int64_t state_width,
                            int64_t kernel_size, int silu, void* stream);

/* Chunked gated delta rule (GDN prefill) on the tensor cores (tcgen05 / TMEM).
 * Replaces the hook chunk_gated_delta_rule (transformers models/qwen3_5/modeling_qwen3_5.py:466-476;
 * torch_chunk_gated_delta_rule :234-311; fla chunk_gated_delta_rule, fla/ops/gated_delta_rule/chunk.py:365).
 * q, k, v: bf16 [B, T, H, 128], element strides per (b, t, h), unit stride along the head dim,
 * every stride a multiple of 16 bytes and the pointers 16-byte aligned.  g, beta: [B, T, H]
 * contiguous (f32 / f16 / bf16).  out: bf16 [B, T, H, 128] contiguous.  States fp32
 * [B, H, 128, 128] contiguous; initial_state NULL = zeros, final_state may be NULL.
 * chunk_size must be 64.  One CTA per (sequence, head).  device_status (nullable) gets
 * OQ_DEV_TIMEOUT if an internal wait gives up. */
int oq_gdn_chunk_fwd(
    const void* q, const void* k, const void* v, int qkv_dtype,
    int64_t q_stride_b, int64_t q_stride_t, int64_t q_stride_h,
    int64_t k_stride_b, int64_t k_stride_t, int64_t k_stride_h,
    int64_t v_stride_b, int64_t v_stride_t, int64_t v_stride_h,
    const void* g, int g_dtype, const void* beta, int beta_dtype,
    const float* initial_state, float* final_state, void* out,
    int64_t batch, int64_t seq_len, int64_t num_heads, int64_t k_dim, int64_t v_dim,
    float scale, int use_qk_l2norm, int64_t chunk_size, int32_t* device_status, void* stream);

/* The same chunked recurrence in two launches (the same reference hook; same arguments
 * and results as oq_gdn_chunk_fwd, to the last bit).  The first launch does, for all
 * chunks of all (sequence, head) at once, the work that does not depend on the state
 * (norms, decays, the Gram matrix, the triangular solve, the P and W / U factors) and
 * writes it to `workspace`.  The second walks each (sequence, head)'s chunks in order
 * and only does the state products.  workspace: oq_gdn_chunk_workspace_bytes(batch,
 * seq_len, num_heads) bytes (about 49 KB per 64-token chunk and head), 128-byte aligned,
 * no initialisation needed; launches that share it must be ordered on one stream. */
size_t oq_gdn_chunk_workspace_bytes(int64_t batch, int64_t seq_len, int64_t num_heads);

int oq_gdn_chunk_fwd_ws(
    const void* q, const void* k, const void* v, int qkv_dtype,
    int64_t q_stride_b, int64_t q_stride_t, int64_t q_stride_h,
    int64_t k_stride_b, int64_t k_stride_t, int64_t k_stride_h,
    int64_t v_stride_b, int64_t v_stride_t, int64_t v_stride_h,
    const void* g, int g_dtype, const void* beta, int beta_dtype,
    const float* initial_state, float* final_state, void* out,
    int64_t batch, int64_t seq_len, int64_t num_heads, int64_t k_dim, int64_t v_dim,
    float scale, int use_qk_l2norm, int64_t chunk_size, void* workspace, size_t workspace_bytes,
    int32_t* device_status, void* stream);

#ifdef __cplusplus
}  /* extern "C" */
#endif

#endif  /* OPTIZ_QWEN_B200_H */
