// Decode-attention definitions shared by the kernel and its split-KV merge: the paged
// INT4 layout, the launch parameters, the output store, and the merge done by the last
// CTA of a (sequence, KV head), written over a named barrier so that a kernel may run it
// with a subset of its warps.
#pragma once

#include <cudaTypedefs.h>

#include "common.cuh"
#include "xrank.cuh"

namespace oq {

constexpr int kHeadDim = 256;
constexpr int kPage = 64;
constexpr int kRowBytes = kHeadDim / 2;                // 128 bytes of codes per token
constexpr int kStageCodeBytes = 2 * kPage * kRowBytes;  // K rows then V rows of a page: 16 KB
constexpr int kStageMetaBytes = 4 * kPage * 2;          // 512 B of fp16 k_scale, k_min, v_scale, v_min
constexpr int kMaxGroup = 8;
constexpr int kMaxSplits = 512;
constexpr int kMinPagesPerSplit = 4;  // (context 16384: 64 ranges of 4 pages 12.8 us, 32 of 8 13.3 us)
constexpr int kInLaunchMergeSplits = 8;

struct AttnParams {
  const void* query;
  int64_t q_sb, q_sh;
  const uint16_t* kv_meta;
  int64_t num_pages, num_kv_heads;
  const int32_t* block_table;
  int64_t bt_stride, max_pages;
  const int32_t* seq_lens;
  int group;
  float scale_log2;  // scaling * log2(e)
  void* out;
  int64_t o_sb, o_sh;
  float* out_f32;
  float* out_lse;
  float* partials;
  int* counters;
  int max_splits;
  int pages_per_split;
  int defer_merge;  // 1: write partials only, a separate merge kernel combines them
  int32_t* status;
  // optional output gate: out = o * sigmoid(gate), gate [B, Hq, 256] in the query dtype
  const void* gate;
  int64_t g_sb, g_sh;
  int wait_polls;  // polls of a bounded wait on a page copy (wait_polls() at launch)
  // optional appended token (append = 1): new_k / new_v [B, Hkv, 256] in the query dtype, written
  // at position seq_lens[b] and attended with the seq_lens[b] cached tokens (see the kernel)
  int append;
  const void* new_k;
  const void* new_v;
  int64_t nk_sb, nk_sh, nv_sb, nv_sh;
  uint8_t* kv_codes;     // the cache, for the appended token's writes
  uint16_t* kv_meta_w;
  int early;             // 1: launched early (programmatic stream serialisation), see the kernel
  // optional cross-GPU exchange (xr.world > 0): the split merge publishes each merged row to
  // every rank over NVLink, waits for theirs and writes the merge of all ranks (xrank.cuh)
  XrankArgs xr;
  XrankLayout xl;
};

// The partition a decode-attention launch uses (host side): the number of KV ranges per
// (sequence, KV head) for `num_splits` (<= 0: ~7/8 of a wave of resident CTAs, at least
// kMinPagesPerSplit pages per range), clamped to the pages and to kMaxSplits and rounded
// to whole pages per range; *pages_per_split (may be null) receives the range length.
int decode_attn_plan(int bits, int dtype, int64_t group, int64_t batch, int64_t num_kv_heads,
                     int64_t max_pages_per_seq, int num_splits, int* pages_per_split);

// Bounded wait for a stage: the thread sleeps in try_wait (up to 20 us per poll) and
// gives up after `polls` polls (kDefaultWaitPolls: ~2 s, after which a copy that has not
// landed never will).
constexpr uint32_t kWaitHintNs = 20000;
__device__ __forceinline__ bool wait_stage(uint64_t* bar, uint32_t parity, int polls) {
  for (int i = 0; i < polls; ++i) {
    if (mbar_try_wait_suspend(bar, parity, kWaitHintNs)) return true;
  }
  return false;
}

// A split CTA that leaves without merging still counts itself in on its unit's merge
// counter, so that the counter is back at zero after every launch; the last to arrive
// resets it (the unit's output is then not written, and the status word says why).
__device__ __forceinline__ void merge_arrive_only(const AttnParams& p, int64_t unit, int nsplit_b) {
  const int done = atomicAdd(&p.counters[unit], 1);
  if (done == nsplit_b - 1) p.counters[unit] = 0;
}

__device__ __forceinline__ float lse_nat(float m_log2, float l) {
  return l > 0.0f ? (m_log2 + log2f(l)) * 0.69314718055994531f : -INFINITY;
}

// Gate element of output (b, hq, d), 0 without a gate.
template <typename T>
__device__ __forceinline__ float gate_value(const AttnParams& p, int64_t b, int64_t hq, int d) {
  return p.gate ? to_float<T>(static_cast<const T*>(p.gate)[b * p.g_sb + hq * p.g_sh + d]) : 0.0f;
}

// The model-dtype output, gated if asked (g = the gate element, loaded ahead): the decode
// forward's ``attn_output * torch.sigmoid(gate)``
// (optiz_qwen/kernels/qwen35_fused_attention.py:96-97) with each operand rounded to the
// model dtype as the unfused ops leave it.
template <typename T>
__device__ __forceinline__ void store_out_g(const AttnParams& p, int64_t b, int64_t hq, int d, float o, float m,
                                            float l, float g) {
  const int64_t hq_total = p.num_kv_heads * p.group;
  if (p.out) {
    T y = from_float<T>(o);
    if (p.gate) {
      const float sg = to_float<T>(from_float<T>(1.0f / (1.0f + expf(-g))));
      y = from_float<T>(to_float<T>(y) * sg);
    }
    static_cast<T*>(p.out)[b * p.o_sb + hq * p.o_sh + d] = y;
  }
  if (p.out_f32) p.out_f32[(b * hq_total + hq) * kHeadDim + d] = o;
  if (p.out_lse && d == 0) p.out_lse[b * hq_total + hq] = lse_nat(m, l);
}

template <typename T>
__device__ __forceinline__ void store_out(const AttnParams& p, int64_t b, int64_t hq, int d, float o, float m,
                                          float l) {
  store_out_g<T>(p, b, hq, d, o, m, l, gate_value<T>(p, b, hq, d));
}

// Split-KV merge, run by the kNT threads [0, kNT) of every CTA of a (sequence, KV head)
// after each has written its partial record (numerators [G][256], then M[G], L[G]):
// the last CTA to arrive combines the records by log-sum-exp and writes the outputs.
// `scratch` holds at least 2 * nsplit * G + 2 * kMaxGroup floats of shared memory;
// `flag` is one int of shared memory.  Barriers are the named barrier `bar_id` over kNT
// threads, so other warps of the CTA may be busy or gone.
template <typename T, int kNT>
__device__ void merge_splits_last_cta(const AttnParams& p, int64_t b, int kvh, int nsplit_b, int tid, float* scratch,
                                      int* flag, int bar_id) {
  const int G = p.group;
  const int outputs = G * kHeadDim;
  const int64_t unit = b * p.num_kv_heads + kvh;
  const int rec_floats = G * (kHeadDim + 2);
  // this thread's outputs: e = tid + j * kNT < outputs (kNT need not divide them)
  constexpr int kMaxPer = (kMaxGroup * kHeadDim + kNT - 1) / kNT;
  float gv[kMaxPer];  // gate elements of this thread's outputs, in flight across the atomic
#pragma unroll
  for (int j = 0; j < kMaxPer; ++j) {
    const int e = tid + j * kNT;
    gv[j] = e < outputs ? gate_value<T>(p, b, int64_t(kvh) * G + e / kHeadDim, e % kHeadDim) : 0.0f;
  }
  __threadfence();
  named_bar_sync(bar_id, kNT);
  if (tid == 0) {
    const int done = atomicAdd(&p.counters[unit], 1);
    *flag = done == nsplit_b - 1;
  }
  named_bar_sync(bar_id, kNT);
  if (!*flag) return;
  __threadfence();
  const float* recs = p.partials + unit * p.max_splits * rec_floats;
  // stage every split's (M, L) in shared memory, then turn M into merge weights
  float* wm = scratch;                // [nsplit_b][G]
  float* wl = wm + nsplit_b * G;      // [nsplit_b][G]
  float* head_m = wl + nsplit_b * G;  // [G]
  float* head_l = head_m + kMaxGroup;  // [G]
  for (int idx = tid; idx < nsplit_b * G; idx += kNT) {
    const int s = idx / G, h = idx - (idx / G) * G;
    wm[idx] = __ldcg(recs + s * rec_floats + outputs + h);
    wl[idx] = __ldcg(recs + s * rec_floats + outputs + G + h);
  }
  named_bar_sync(bar_id, kNT);
  if (tid < G) {
    float M = -INFINITY;
    for (int s = 0; s < nsplit_b; ++s) M = fmaxf(M, wm[s * G + tid]);
    float L = 0.0f;
    if (M != -INFINITY) {
      for (int s = 0; s < nsplit_b; ++s) L += wl[s * G + tid] * exp2f(wm[s * G + tid] - M);
    }
    head_m[tid] = M;
    head_l[tid] = L;
  }
  named_bar_sync(bar_id, kNT);
  for (int idx = tid; idx < nsplit_b * G; idx += kNT) {
    const int h = idx - (idx / G) * G;
    const float M = head_m[h];
    wm[idx] = M == -INFINITY ? 0.0f : exp2f(wm[idx] - M);
  }
  named_bar_sync(bar_id, kNT);
  float num[kMaxPer];
#pragma unroll
  for (int j = 0; j < kMaxPer; ++j) num[j] = 0.0f;
  for (int s = 0; s < nsplit_b; ++s) {
    const float* rec = recs + s * rec_floats;
#pragma unroll
    for (int j = 0; j < kMaxPer; ++j) {
      const int e = tid + j * kNT;
      if (e < outputs) num[j] = fmaf(wm[s * G + e / kHeadDim], __ldcg(rec + e), num[j]);
    }
  }
#pragma unroll
  for (int j = 0; j < kMaxPer; ++j) {
    const int e = tid + j * kNT;
    if (e < outputs) {
      const int h = e / kHeadDim;
      const float L = head_l[h];
      store_out_g<T>(p, b, int64_t(kvh) * G + h, e - h * kHeadDim, L > 0.0f ? num[j] / L : 0.0f, head_m[h], L,
                     gv[j]);
    }
  }
  if (tid == 0) p.counters[unit] = 0;  // ready for the next launch
}

}  // namespace oq
