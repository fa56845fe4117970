// Gated RMSNorm as a standalone kernel: transformers' Qwen3_5RMSNormGated.forward
// (models/qwen3_5/modeling_qwen3_5.py:175-190), the GDN layer's output norm with the z
// projection as gate (:527-529), for callers that keep the norm a separate module (the
// decode step fuses the same epilogue into the GDN kernel: oq_gdn_recurrent_norm).
//
//   y = rnd(rnd(rnd(x * rsqrt(mean(x^2) + eps)) * w) * silu(z))
//
// rnd = rounding to the model dtype, as the module's .to(input_dtype) steps do; the
// variance, the normalisation and the gate are fp32.  One warp per row.
#include "common.cuh"

namespace oq {
namespace {

constexpr int kNormWarps = 8;
constexpr int kNormMaxDim = 1024;
constexpr int kPerLane = kNormMaxDim / 32;

template <typename T>
__global__ void __launch_bounds__(kNormWarps * 32) rmsnorm_gated_kernel(const T* x, int64_t xs, const T* z, int64_t zs,
                                                                        const T* w, T* out, int64_t os, int64_t rows,
                                                                        int dim, float eps) {
  const int64_t row = int64_t(blockIdx.x) * kNormWarps + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  pdl_wait();        // x comes from the preceding kernel
  pdl_allow_next();  // the successor may launch: this kernel is a few microseconds of tail
  if (row >= rows) return;
  const T* xr = x + row * xs;
  const T* zr = z + row * zs;
  float xv[kPerLane];
  float ss = 0.0f;
#pragma unroll
  for (int i = 0; i < kPerLane; ++i) {
    const int d = lane + 32 * i;
    xv[i] = d < dim ? to_float<T>(xr[d]) : 0.0f;
    ss = fmaf(xv[i], xv[i], ss);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  const float inv = 1.0f / sqrtf(ss / float(dim) + eps);
  T* orow = out + row * os;
#pragma unroll
  for (int i = 0; i < kPerLane; ++i) {
    const int d = lane + 32 * i;
    if (d < dim) {
      const float nrm = to_float<T>(from_float<T>(xv[i] * inv));
      const float y = to_float<T>(from_float<T>(to_float<T>(w[d]) * nrm));
      const float zv = to_float<T>(zr[d]);
      orow[d] = from_float<T>(y * (zv / (1.0f + expf(-zv))));
    }
  }
}

template <typename T>
void launch_norm(const void* x, int64_t xs, const void* z, int64_t zs, const void* w, void* out, int64_t os,
                 int64_t rows, int64_t dim, float eps, cudaStream_t s) {
  const dim3 grid(unsigned((rows + kNormWarps - 1) / kNormWarps));
  launch_pdl(rmsnorm_gated_kernel<T>, grid, dim3(kNormWarps * 32), 0, s, static_cast<const T*>(x), xs,
               static_cast<const T*>(z), zs, static_cast<const T*>(w), static_cast<T*>(out), os, rows, int(dim), eps);
}

}  // namespace
}  // namespace oq

extern "C" int oq_rmsnorm_gated(const void* x, int64_t x_stride, const void* z, int64_t z_stride, const void* weight,
                                void* out, int64_t out_stride, int dtype, int64_t rows, int64_t dim, float eps,
                                void* stream) {
  using namespace oq;
  if (!valid_dtype(dtype)) return fail(OQ_ERR_UNSUPPORTED, "rmsnorm_gated: unknown dtype");
  if (rows < 0 || dim <= 0 || !(eps >= 0.0f)) return fail(OQ_ERR_INVALID_ARGUMENT, "rmsnorm_gated: bad sizes");
  if (dim > kNormMaxDim) return fail(OQ_ERR_UNSUPPORTED, "rmsnorm_gated: dim above %d", kNormMaxDim);
  if (rows == 0) return ok();
  if (rows > int64_t(kNormWarps) * 2147483647LL) return fail(OQ_ERR_UNSUPPORTED, "rmsnorm_gated: too many rows");
  if (!x || !z || !weight || !out) return fail(OQ_ERR_INVALID_ARGUMENT, "rmsnorm_gated: null pointer");
  if (x_stride < dim || z_stride < dim || out_stride < dim) {
    return fail(OQ_ERR_INVALID_ARGUMENT, "rmsnorm_gated: row strides must cover a row");
  }
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  switch (dtype) {
    case OQ_F32: launch_norm<float>(x, x_stride, z, z_stride, weight, out, out_stride, rows, dim, eps, s); break;
    case OQ_F16: launch_norm<__half>(x, x_stride, z, z_stride, weight, out, out_stride, rows, dim, eps, s); break;
    default: launch_norm<__nv_bfloat16>(x, x_stride, z, z_stride, weight, out, out_stride, rows, dim, eps, s); break;
  }
  return check_launch("rmsnorm_gated");
}
