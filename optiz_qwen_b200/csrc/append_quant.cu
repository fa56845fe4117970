// Fused append-quantize into the paged INT4 (or INT8) KV cache.
//
// Replaces the reference's per-token torch.cat into a dense residual window and
// its periodic groupwise quantise + torch.cat of the whole code tensor
// (optiz_qwen/compression/qserve_kv_cache.py:210-232, 278-292, 313-335, 356-362).
// Here every appended token is quantised at once into its page slot: one warp
// per (token, KV head, K-or-V) row of head_dim values, min/max by warp shuffles,
// codes from the fp32 scale/min with IEEE division and round-half-even exactly
// as the reference computes them, then one 4-byte store per lane.  The 8-bit variant
// (the reference's bits=8 path: 255 levels, one code per byte) shares the kernel.
#include <algorithm>

#include "quant_row.cuh"

namespace oq {
namespace {

constexpr int kWarps = 4;

struct AppendParams {
  const void* key;
  const void* value;
  int64_t stride[2][3];  // [K/V][b, h, t] in elements
  int64_t num_kv_heads, num_new;
  uint8_t* kv_codes;
  uint16_t* kv_meta;
  int64_t num_pages, page_size;
  const int32_t* block_table;
  int64_t block_table_stride, max_pages_per_seq;
  int32_t* seq_lens;
  int advance;
  int32_t* status;
};

// One (token, head, K|V) row per warp; head_dim = 32 * EPL; codes of kBits bits.
template <typename T, int EPL, bool VEC, int kBits>
__global__ void __launch_bounds__(kWarps * 32) append_quant_kernel(AppendParams p) {
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int64_t b = blockIdx.y;
  pdl_wait();
  pdl_allow_next();
  const int32_t start = p.seq_lens[b];
  const int64_t jobs = p.num_kv_heads * p.num_new * 2;
  constexpr int kHeadDim = EPL * 32;
  constexpr int kRowBytes = kHeadDim * kBits / 8;

  for (int64_t job = int64_t(blockIdx.x) * kWarps + warp; job < jobs; job += int64_t(gridDim.x) * kWarps) {
    const int kv = int(job & 1);
    const int64_t th = job >> 1;
    const int64_t t = th % p.num_new;
    const int64_t h = th / p.num_new;
    const int64_t pos = int64_t(start) + t;
    const int64_t logical_page = pos / p.page_size;
    const int64_t slot = pos - logical_page * p.page_size;
    if (logical_page >= p.max_pages_per_seq) {
      if (lane == 0) report(p.status, OQ_DEV_OVERFLOW);
      continue;
    }
    const int64_t page = p.block_table[b * p.block_table_stride + logical_page];
    if (page < 0 || page >= p.num_pages) {
      if (lane == 0) report(p.status, OQ_DEV_BAD_PAGE);
      continue;
    }

    const T* src = static_cast<const T*>(kv ? p.value : p.key) + b * p.stride[kv][0] + h * p.stride[kv][1] +
                   t * p.stride[kv][2];
    const int64_t block = (page * p.num_kv_heads + h) * 2 + kv;
    quantize_row<T, EPL, VEC, kBits>(src, lane, p.kv_codes + (block * p.page_size + slot) * kRowBytes,
                                     p.kv_meta + ((page * p.num_kv_heads + h) * 4 + kv * 2) * p.page_size + slot,
                                     p.page_size);
  }
  if (p.advance) {
    __syncthreads();  // every warp has read seq_lens[b]
    if (threadIdx.x == 0) p.seq_lens[b] = start + int32_t(p.num_new);
  }
}

__global__ void advance_kernel(int32_t* seq_lens, int64_t batch, int32_t delta) {
  pdl_wait();
  pdl_allow_next();
  int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i < batch) seq_lens[i] += delta;
}

template <typename T, int EPL, int kBits>
void launch_append(const AppendParams& p, bool vec, dim3 grid, cudaStream_t s) {
  if (vec) {
    launch_plain(append_quant_kernel<T, EPL, true, kBits>, grid, dim3(kWarps * 32), 0, s, p);
  } else {
    launch_plain(append_quant_kernel<T, EPL, false, kBits>, grid, dim3(kWarps * 32), 0, s, p);
  }
}

template <typename T, int kBits>
void launch_dim(const AppendParams& p, int64_t head_dim, bool vec, dim3 grid, cudaStream_t s) {
  switch (head_dim) {
    case 64: launch_append<T, 2, kBits>(p, vec, grid, s); break;
    case 128: launch_append<T, 4, kBits>(p, vec, grid, s); break;
    case 256: launch_append<T, 8, kBits>(p, vec, grid, s); break;
    default: launch_append<T, 16, kBits>(p, vec, grid, s); break;  // 512
  }
}

}  // namespace
}  // namespace oq

extern "C" int oq_advance_seq_lens(int32_t* seq_lens, int64_t batch, int32_t delta, void* stream) {
  using namespace oq;
  if (seq_lens == nullptr || batch < 0) return fail(OQ_ERR_INVALID_ARGUMENT, "advance_seq_lens: bad arguments");
  if (batch == 0) return ok();
  const int threads = 256;
  launch_plain(advance_kernel, dim3(unsigned((batch + threads - 1) / threads)), dim3(threads), 0,
             static_cast<cudaStream_t>(stream), seq_lens, batch, int32_t(delta));
  return check_launch("advance_seq_lens");
}

namespace oq {
namespace {

int append_quant_impl(
    int bits, const void* key, const void* value, int dtype,
    int64_t batch, int64_t num_kv_heads, int64_t num_new, int64_t head_dim,
    int64_t key_stride_b, int64_t key_stride_h, int64_t key_stride_t,
    int64_t value_stride_b, int64_t value_stride_h, int64_t value_stride_t,
    uint8_t* kv_codes, uint16_t* kv_meta, int64_t num_pages, int64_t page_size,
    const int32_t* block_table, int64_t block_table_stride, int64_t max_pages_per_seq,
    int32_t* seq_lens, int advance_seq_lens,
    int32_t* device_status, void* stream) {
  if (!valid_dtype(dtype)) return fail(OQ_ERR_UNSUPPORTED, "append_quant: unknown dtype %d", dtype);
  if (batch < 0 || num_kv_heads <= 0 || num_new < 0 || num_pages <= 0 || page_size <= 0 ||
      max_pages_per_seq <= 0 || block_table_stride < max_pages_per_seq) {
    return fail(OQ_ERR_INVALID_ARGUMENT, "append_quant: bad sizes");
  }
  if (head_dim != 64 && head_dim != 128 && head_dim != 256 && head_dim != 512) {
    return fail(OQ_ERR_UNSUPPORTED, "append_quant: head_dim %lld not in {64,128,256,512}",
                (long long)head_dim);
  }
  if (batch == 0 || num_new == 0) return ok();
  if (!key || !value || !kv_codes || !kv_meta || !block_table || !seq_lens) {
    return fail(OQ_ERR_INVALID_ARGUMENT, "append_quant: null pointer");
  }
  const int64_t esize = dtype == OQ_F32 ? 4 : 2;
  const int64_t strides[6] = {key_stride_b, key_stride_h, key_stride_t, value_stride_b, value_stride_h, value_stride_t};
  bool vec = (reinterpret_cast<uintptr_t>(key) % 16 == 0) && (reinterpret_cast<uintptr_t>(value) % 16 == 0) &&
             ((head_dim / 32) * esize % 16 == 0);
  for (int64_t s : strides) {
    if (s < 0) return fail(OQ_ERR_INVALID_ARGUMENT, "append_quant: negative stride");
    vec = vec && ((s * esize) % 16 == 0);
  }

  AppendParams p;
  p.key = key;
  p.value = value;
  for (int i = 0; i < 3; ++i) {
    p.stride[0][i] = strides[i];
    p.stride[1][i] = strides[3 + i];
  }
  p.num_kv_heads = num_kv_heads;
  p.num_new = num_new;
  p.kv_codes = kv_codes;
  p.kv_meta = kv_meta;
  p.num_pages = num_pages;
  p.page_size = page_size;
  p.block_table = block_table;
  p.block_table_stride = block_table_stride;
  p.max_pages_per_seq = max_pages_per_seq;
  p.seq_lens = seq_lens;
  p.status = device_status;

  // Decode appends (a few rows per sequence) run one CTA per sequence and bump
  // seq_lens in the same launch; bulk appends (prefill adoption) spread over
  // more CTAs and bump seq_lens with a follow-up launch on the same stream.
  const int64_t jobs = num_kv_heads * num_new * 2;
  const int64_t blocks_x = std::min<int64_t>((jobs + kWarps - 1) / kWarps, 1024);
  const bool fused_advance = blocks_x == 1;
  p.advance = (advance_seq_lens && fused_advance) ? 1 : 0;
  if (batch > 65535) return fail(OQ_ERR_UNSUPPORTED, "append_quant: batch > 65535");
  dim3 grid((unsigned)blocks_x, (unsigned)batch);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (bits == 8) {
    switch (dtype) {
      case OQ_F32: launch_dim<float, 8>(p, head_dim, vec, grid, s); break;
      case OQ_F16: launch_dim<__half, 8>(p, head_dim, vec, grid, s); break;
      default: launch_dim<__nv_bfloat16, 8>(p, head_dim, vec, grid, s); break;
    }
  } else {
    switch (dtype) {
      case OQ_F32: launch_dim<float, 4>(p, head_dim, vec, grid, s); break;
      case OQ_F16: launch_dim<__half, 4>(p, head_dim, vec, grid, s); break;
      default: launch_dim<__nv_bfloat16, 4>(p, head_dim, vec, grid, s); break;
    }
  }
  int st = check_launch(bits == 8 ? "append_quant_int8" : "append_quant_int4");
  if (st != OQ_OK) return st;
  if (advance_seq_lens && !fused_advance) {
    return oq_advance_seq_lens(seq_lens, batch, int32_t(num_new), stream);
  }
  return ok();
}

}  // namespace
}  // namespace oq

extern "C" int oq_append_quant_int4(
    const void* key, const void* value, int dtype,
    int64_t batch, int64_t num_kv_heads, int64_t num_new, int64_t head_dim,
    int64_t key_stride_b, int64_t key_stride_h, int64_t key_stride_t,
    int64_t value_stride_b, int64_t value_stride_h, int64_t value_stride_t,
    uint8_t* kv_codes, uint16_t* kv_meta, int64_t num_pages, int64_t page_size,
    const int32_t* block_table, int64_t block_table_stride, int64_t max_pages_per_seq,
    int32_t* seq_lens, int advance_seq_lens,
    int32_t* device_status, void* stream) {
  return oq::append_quant_impl(4, key, value, dtype, batch, num_kv_heads, num_new, head_dim, key_stride_b,
                               key_stride_h, key_stride_t, value_stride_b, value_stride_h, value_stride_t, kv_codes,
                               kv_meta, num_pages, page_size, block_table, block_table_stride, max_pages_per_seq,
                               seq_lens, advance_seq_lens, device_status, stream);
}

extern "C" int oq_append_quant_int8(
    const void* key, const void* value, int dtype,
    int64_t batch, int64_t num_kv_heads, int64_t num_new, int64_t head_dim,
    int64_t key_stride_b, int64_t key_stride_h, int64_t key_stride_t,
    int64_t value_stride_b, int64_t value_stride_h, int64_t value_stride_t,
    uint8_t* kv_codes, uint16_t* kv_meta, int64_t num_pages, int64_t page_size,
    const int32_t* block_table, int64_t block_table_stride, int64_t max_pages_per_seq,
    int32_t* seq_lens, int advance_seq_lens,
    int32_t* device_status, void* stream) {
  return oq::append_quant_impl(8, key, value, dtype, batch, num_kv_heads, num_new, head_dim, key_stride_b,
                               key_stride_h, key_stride_t, value_stride_b, value_stride_h, value_stride_t, kv_codes,
                               kv_meta, num_pages, page_size, block_table, block_table_stride, max_pages_per_seq,
                               seq_lens, advance_seq_lens, device_status, stream);
}
