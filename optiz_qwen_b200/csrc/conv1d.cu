// Causal depthwise conv1d update (the GDN layer's short convolution over q/k/v).
//
// Replaces the hook `causal_conv1d_update` of Qwen3_5GatedDeltaNet (decode call
// transformers models/qwen3_5/modeling_qwen3_5.py:454; torch fallback
// torch_causal_conv1d_update :210-225; causal-conv1d 1.6.2 causal_conv1d_update).
// For every (sequence, channel): full = [conv_state (W) | x (T)];
// out[t] = act(bias + sum_k w[k] * full[W + t - K + 1 + k]); conv_state <- last W of full.
// One thread per (sequence, channel); arithmetic in fp32, state copied bit-exactly.
#include "common.cuh"

namespace oq {
namespace {

constexpr int kMaxWidth = 8;
constexpr int kMaxKernel = 8;
constexpr int kThreads = 256;

struct ConvParams {
  const void* x;
  int64_t xs[3];  // strides (b, c, t) of x, elements
  void* state;    // [B, C, W] contiguous, in x's dtype
  const void* weight;
  const void* bias;
  int w_dtype;
  void* out;      // [B, C, T] contiguous, in x's dtype
  int64_t batch, channels, seq_len;
  int width, ksize, silu;
};

__device__ __forceinline__ float silu(float v) { return v / (1.0f + expf(-v)); }

template <typename T>
__global__ void __launch_bounds__(kThreads) conv1d_update_kernel(ConvParams p) {
  const int64_t i = int64_t(blockIdx.x) * kThreads + threadIdx.x;
  pdl_wait();
  pdl_allow_next();
  if (i >= p.batch * p.channels) return;
  const int64_t b = i / p.channels, c = i - b * p.channels;
  const int W = p.width, K = p.ksize;
  T* st = static_cast<T*>(p.state) + i * W;
  float hist[kMaxWidth], w[kMaxKernel];
#pragma unroll
  for (int j = 0; j < kMaxWidth; ++j) hist[j] = j < W ? to_float<T>(st[j]) : 0.0f;
#pragma unroll
  for (int k = 0; k < kMaxKernel; ++k) w[k] = k < K ? load_as_float(p.weight, p.w_dtype, c * K + k) : 0.0f;
  const float bias = p.bias != nullptr ? load_as_float(p.bias, p.w_dtype, c) : 0.0f;
  const T* xr = static_cast<const T*>(p.x) + b * p.xs[0] + c * p.xs[1];
  T* orow = static_cast<T*>(p.out) + i * p.seq_len;
  for (int64_t t = 0; t < p.seq_len; ++t) {
    const float xt = to_float<T>(xr[t * p.xs[2]]);
    // slide the window: hist holds the W most recent inputs, oldest first
#pragma unroll
    for (int j = 0; j < kMaxWidth; ++j) {
      const float nxt = j + 1 < kMaxWidth ? hist[j + 1] : 0.0f;
      if (j < W - 1) hist[j] = nxt;
      if (j == W - 1) hist[j] = xt;
    }
    float acc = bias;
#pragma unroll
    for (int j = 0; j < kMaxWidth; ++j) {
      // tap k = j - (W - K) multiplies hist[j] (the K most recent inputs)
#pragma unroll
      for (int k = 0; k < kMaxKernel; ++k) {
        if (k < K && j == W - K + k) acc = fmaf(w[k], hist[j], acc);
      }
    }
    orow[t] = from_float<T>(p.silu ? silu(acc) : acc);
  }
  // the window is the last W of [state | x]: the new state (exact: values round-trip through fp32)
#pragma unroll
  for (int j = 0; j < kMaxWidth; ++j) {
    if (j < W) st[j] = from_float<T>(hist[j]);
  }
}

}  // namespace
}  // namespace oq

extern "C" int oq_causal_conv1d_update(const void* x, int dtype, int64_t x_stride_b, int64_t x_stride_c,
                                       int64_t x_stride_t, void* conv_state, const void* weight, const void* bias,
                                       int w_dtype, void* out, int64_t batch, int64_t channels, int64_t seq_len,
                                       int64_t state_width, int64_t kernel_size, int silu, void* stream) {
  using namespace oq;
  if (!valid_dtype(dtype) || !valid_dtype(w_dtype)) return fail(OQ_ERR_UNSUPPORTED, "causal_conv1d_update: unknown dtype");
  if (batch < 0 || channels <= 0 || seq_len < 0) return fail(OQ_ERR_INVALID_ARGUMENT, "causal_conv1d_update: bad sizes");
  if (kernel_size < 1 || kernel_size > kMaxKernel || state_width < kernel_size - 1 || state_width < 1 ||
      state_width > kMaxWidth) {
    return fail(OQ_ERR_UNSUPPORTED, "causal_conv1d_update: need 1 <= kernel_size - 1 <= state_width <= %d", kMaxWidth);
  }
  if (batch == 0 || seq_len == 0) return ok();
  if (!x || !conv_state || !weight || !out) return fail(OQ_ERR_INVALID_ARGUMENT, "causal_conv1d_update: null pointer");
  ConvParams p;
  p.x = x;
  p.xs[0] = x_stride_b;
  p.xs[1] = x_stride_c;
  p.xs[2] = x_stride_t;
  p.state = conv_state;
  p.weight = weight;
  p.bias = bias;
  p.w_dtype = w_dtype;
  p.out = out;
  p.batch = batch;
  p.channels = channels;
  p.seq_len = seq_len;
  p.width = int(state_width);
  p.ksize = int(kernel_size);
  p.silu = silu;
  const int64_t blocks = (batch * channels + kThreads - 1) / kThreads;
  if (blocks > 0x7fffffff) return fail(OQ_ERR_UNSUPPORTED, "causal_conv1d_update: too many channels");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  switch (dtype) {
    case OQ_F32: launch_plain(conv1d_update_kernel<float>, dim3(unsigned(blocks)), dim3(kThreads), 0, s, p); break;
    case OQ_F16: launch_plain(conv1d_update_kernel<__half>, dim3(unsigned(blocks)), dim3(kThreads), 0, s, p); break;
    default: launch_plain(conv1d_update_kernel<__nv_bfloat16>, dim3(unsigned(blocks)), dim3(kThreads), 0, s, p); break;
  }
  return check_launch("causal_conv1d_update");
}
