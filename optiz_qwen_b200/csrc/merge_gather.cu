// Log-sum-exp merge of attention partials, and the paged gather + dequantise
// that backs the cache layer's materialize().
#include <algorithm>
#include <cmath>

#include "common.cuh"

namespace oq {
namespace {

// One warp per output row; lanes stride over head_dim.
template <typename T>
__global__ void lse_merge_kernel(const float* __restrict__ part_out, const float* __restrict__ part_lse,
                                 int64_t num_parts, int64_t rows, int64_t head_dim, T* __restrict__ out,
                                 float* __restrict__ out_lse) {
  const int lane = threadIdx.x & 31;
  const int64_t row = int64_t(blockIdx.x) * (blockDim.x / 32) + (threadIdx.x >> 5);
  pdl_wait();
  pdl_allow_next();
  if (row >= rows) return;
  float m = -INFINITY;
  for (int64_t i = 0; i < num_parts; ++i) m = fmaxf(m, part_lse[i * rows + row]);
  float denom = 0.0f;
  for (int64_t i = 0; i < num_parts; ++i) {
    const float l = part_lse[i * rows + row];
    denom += (m == -INFINITY || l == -INFINITY) ? 0.0f : expf(l - m);
  }
  for (int64_t d = lane; d < head_dim; d += 32) {
    float acc = 0.0f;
    for (int64_t i = 0; i < num_parts; ++i) {
      const float l = part_lse[i * rows + row];
      if (m == -INFINITY || l == -INFINITY) continue;
      acc += expf(l - m) * part_out[(i * rows + row) * head_dim + d];
    }
    out[row * head_dim + d] = from_float<T>(denom > 0.0f ? acc / denom : 0.0f);
  }
  if (out_lse != nullptr && lane == 0) out_lse[row] = denom > 0.0f ? m + logf(denom) : -INFINITY;
}

// One warp per (token, KV head, K|V) row: 32 lanes x head_dim/32 values.  kBits = 4: two
// codes per byte, low nibble first; kBits = 8: one code per byte.
template <typename T, int kBits>
__global__ void gather_dequant_kernel(const uint8_t* __restrict__ kv_codes, const uint16_t* __restrict__ kv_meta,
                                      int64_t num_pages, int64_t page_size, const int32_t* __restrict__ block_table,
                                      int64_t bt_stride, int64_t max_pages, const int32_t* __restrict__ seq_lens,
                                      int64_t batch, int64_t num_kv_heads, int64_t head_dim, int64_t max_len,
                                      T* __restrict__ keys, T* __restrict__ values, int32_t* status) {
  const int lane = threadIdx.x & 31;
  const int64_t row = int64_t(blockIdx.x) * (blockDim.x / 32) + (threadIdx.x >> 5);
  const int64_t total = batch * num_kv_heads * max_len * 2;
  pdl_wait();
  pdl_allow_next();
  if (row >= total) return;
  const int kv = int(row & 1);
  int64_t rest = row >> 1;
  const int64_t t = rest % max_len;
  rest /= max_len;
  const int64_t h = rest % num_kv_heads;
  const int64_t b = rest / num_kv_heads;
  const int64_t len = std::min<int64_t>(std::max(seq_lens[b], 0), max_len);
  if (t >= len) return;
  const int64_t lp = t / page_size;
  if (lp >= max_pages) {
    if (lane == 0) report(status, OQ_DEV_OVERFLOW);
    return;
  }
  const int64_t page = block_table[b * bt_stride + lp];
  if (page < 0 || page >= num_pages) {
    if (lane == 0) report(status, OQ_DEV_BAD_PAGE);
    return;
  }
  const int64_t slot = t - lp * page_size;
  const int64_t blk = page * num_kv_heads + h;
  const int64_t row_bytes = head_dim * kBits / 8;
  const uint8_t* src = kv_codes + ((blk * 2 + kv) * page_size + slot) * row_bytes;
  const uint16_t* meta = kv_meta + (blk * 4 + 2 * kv) * page_size + slot;
  const float scale = __half2float(__ushort_as_half(meta[0]));
  const float mn = __half2float(__ushort_as_half(meta[page_size]));
  T* dst = (kv ? values : keys) + ((b * num_kv_heads + h) * max_len + t) * head_dim;
  for (int64_t j = lane; j < row_bytes; j += 32) {
    const uint8_t byte = src[j];
    if constexpr (kBits == 8) {
      dst[j] = from_float<T>(__fadd_rn(mn, __fmul_rn(float(byte), scale)));
    } else {
      dst[2 * j] = from_float<T>(__fadd_rn(mn, __fmul_rn(float(byte & 15), scale)));
      dst[2 * j + 1] = from_float<T>(__fadd_rn(mn, __fmul_rn(float(byte >> 4), scale)));
    }
  }
}

template <int kBits>
int gather_dequant_impl(const uint8_t* kv_codes, const uint16_t* kv_meta, int64_t num_pages, int64_t page_size,
                        const int32_t* block_table, int64_t block_table_stride, int64_t max_pages_per_seq,
                        const int32_t* seq_lens, int64_t batch, int64_t num_kv_heads, int64_t head_dim,
                        int64_t max_len, void* keys, void* values, int dtype, int32_t* device_status, void* stream) {
  const char* name = kBits == 8 ? "gather_dequant_int8" : "gather_dequant_int4";
  if (!valid_dtype(dtype)) return fail(OQ_ERR_UNSUPPORTED, "%s: unknown dtype %d", name, dtype);
  if (batch < 0 || num_kv_heads <= 0 || head_dim <= 0 || head_dim % 2 || max_len < 0 || num_pages <= 0 ||
      page_size <= 0 || max_pages_per_seq <= 0 || block_table_stride < max_pages_per_seq) {
    return fail(OQ_ERR_INVALID_ARGUMENT, "%s: bad sizes", name);
  }
  if (batch == 0 || max_len == 0) return ok();
  if (!kv_codes || !kv_meta || !block_table || !seq_lens || !keys || !values) {
    return fail(OQ_ERR_INVALID_ARGUMENT, "%s: null pointer", name);
  }
  const int64_t rows = batch * num_kv_heads * max_len * 2;
  const int warps = 8;
  const int64_t blocks = (rows + warps - 1) / warps;
  if (blocks > 0x7fffffff) return fail(OQ_ERR_UNSUPPORTED, "%s: too many rows", name);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
#define OQ_GATHER(T)                                                                                              \
  launch_plain(gather_dequant_kernel<T, kBits>, dim3(unsigned(blocks)), dim3(warps * 32), 0, s, kv_codes, kv_meta, \
               num_pages, page_size, block_table, block_table_stride, max_pages_per_seq, seq_lens, batch,         \
               num_kv_heads, head_dim, max_len, static_cast<T*>(keys), static_cast<T*>(values), device_status)
  switch (dtype) {
    case OQ_F32: OQ_GATHER(float); break;
    case OQ_F16: OQ_GATHER(__half); break;
    default: OQ_GATHER(__nv_bfloat16); break;
  }
#undef OQ_GATHER
  return check_launch(name);
}

}  // namespace
}  // namespace oq

extern "C" int oq_lse_merge(const float* part_out, const float* part_lse, int64_t num_parts, int64_t rows,
                            int64_t head_dim, void* out, int dtype, float* out_lse, void* stream) {
  using namespace oq;
  if (!valid_dtype(dtype)) return fail(OQ_ERR_UNSUPPORTED, "lse_merge: unknown dtype %d", dtype);
  if (num_parts <= 0 || rows < 0 || head_dim <= 0) return fail(OQ_ERR_INVALID_ARGUMENT, "lse_merge: bad sizes");
  if (rows == 0) return ok();
  if (!part_out || !part_lse || !out) return fail(OQ_ERR_INVALID_ARGUMENT, "lse_merge: null pointer");
  const int warps = 8;
  const unsigned blocks = unsigned((rows + warps - 1) / warps);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  switch (dtype) {
    case OQ_F32:
      launch_plain(lse_merge_kernel<float>, dim3(blocks), dim3(warps * 32), 0, s, part_out, part_lse, num_parts, rows,
                 head_dim, static_cast<float*>(out), out_lse);
      break;
    case OQ_F16:
      launch_plain(lse_merge_kernel<__half>, dim3(blocks), dim3(warps * 32), 0, s, part_out, part_lse, num_parts, rows,
                 head_dim, static_cast<__half*>(out), out_lse);
      break;
    default:
      launch_plain(lse_merge_kernel<__nv_bfloat16>, dim3(blocks), dim3(warps * 32), 0, s, part_out, part_lse, num_parts,
                 rows, head_dim, static_cast<__nv_bfloat16*>(out), out_lse);
  }
  return check_launch("lse_merge");
}

extern "C" int oq_gather_dequant_int4(
    const uint8_t* kv_codes, const uint16_t* kv_meta, int64_t num_pages, int64_t page_size,
    const int32_t* block_table, int64_t block_table_stride, int64_t max_pages_per_seq,
    const int32_t* seq_lens, int64_t batch, int64_t num_kv_heads, int64_t head_dim,
    int64_t max_len, void* keys, void* values, int dtype,
    int32_t* device_status, void* stream) {
  return oq::gather_dequant_impl<4>(kv_codes, kv_meta, num_pages, page_size, block_table, block_table_stride,
                                    max_pages_per_seq, seq_lens, batch, num_kv_heads, head_dim, max_len, keys, values,
                                    dtype, device_status, stream);
}

extern "C" int oq_gather_dequant_int8(
    const uint8_t* kv_codes, const uint16_t* kv_meta, int64_t num_pages, int64_t page_size,
    const int32_t* block_table, int64_t block_table_stride, int64_t max_pages_per_seq,
    const int32_t* seq_lens, int64_t batch, int64_t num_kv_heads, int64_t head_dim,
    int64_t max_len, void* keys, void* values, int dtype,
    int32_t* device_status, void* stream) {
  return oq::gather_dequant_impl<8>(kv_codes, kv_meta, num_pages, page_size, block_table, block_table_stride,
                                    max_pages_per_seq, seq_lens, batch, num_kv_heads, head_dim, max_len, keys, values,
                                    dtype, device_status, stream);
}
