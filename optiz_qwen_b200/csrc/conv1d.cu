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

constexpr int kThreads = 256;

struct ConvParams {
  const void* x;
  int64_t xs[3];  // strides (b, c, t) of x, elements
  void* state;    // [B, C, W] contiguous, in x's dtype
  const void* weight;
  const void* bias;
  void* out;      // [B, C, T] contiguous, in x's dtype
  int64_t batch, channels, seq_len;
  int silu;
};

__device__ __forceinline__ float silu(float v) { return v / (1.0f + expf(-v)); }

// Window W and kernel size K are compile-time so that every load of a thread is
// unconditional and all of them are in flight together.
template <typename T, typename TW, int W, int K>
__global__ void __launch_bounds__(kThreads) conv1d_update_kernel(ConvParams p) {
  static_assert(K >= 1 && W >= K - 1 && W >= 1, "window must hold K - 1 past inputs");
  const int64_t i = int64_t(blockIdx.x) * kThreads + threadIdx.x;
  pdl_wait();
  pdl_allow_next();
  if (i >= p.batch * p.channels) return;
  const int64_t b = i / p.channels, c = i - b * p.channels;
  T* st = static_cast<T*>(p.state) + i * W;
  const TW* wr = static_cast<const TW*>(p.weight) + c * K;
  float hist[W], w[K];
#pragma unroll
  for (int j = 0; j < W; ++j) hist[j] = to_float<T>(st[j]);
#pragma unroll
  for (int k = 0; k < K; ++k) w[k] = to_float<TW>(wr[k]);
  const float bias = p.bias != nullptr ? to_float<TW>(static_cast<const TW*>(p.bias)[c]) : 0.0f;
  const T* xr = static_cast<const T*>(p.x) + b * p.xs[0] + c * p.xs[1];
  T* orow = static_cast<T*>(p.out) + i * p.seq_len;
  for (int64_t t = 0; t < p.seq_len; ++t) {
    // slide the window: hist holds the W most recent inputs, oldest first
#pragma unroll
    for (int j = 0; j + 1 < W; ++j) hist[j] = hist[j + 1];
    hist[W - 1] = to_float<T>(xr[t * p.xs[2]]);
    float acc = bias;
#pragma unroll
    for (int k = 0; k < K; ++k) acc = fmaf(w[k], hist[W - K + k], acc);
    orow[t] = from_float<T>(p.silu ? silu(acc) : acc);
  }
  // the window is the last W of [state | x]: the new state (exact: values round-trip through fp32)
#pragma unroll
  for (int j = 0; j < W; ++j) st[j] = from_float<T>(hist[j]);
}

template <typename T, typename TW>
int launch_conv(const ConvParams& p, int64_t width, int64_t ksize, dim3 grid, cudaStream_t s) {
#define OQ_CONV(W, K)                                                                          \
  if (width == W && ksize == K) {                                                              \
    launch_plain(conv1d_update_kernel<T, TW, W, K>, grid, dim3(kThreads), 0, s, p);           \
    return OQ_OK;                                                                              \
  }
  OQ_CONV(4, 4) OQ_CONV(3, 4) OQ_CONV(3, 3) OQ_CONV(2, 3) OQ_CONV(2, 2) OQ_CONV(1, 2)
#undef OQ_CONV
  return fail(OQ_ERR_UNSUPPORTED, "causal_conv1d_update: kernel_size must be 2..4 with state_width kernel_size - 1 "
              "or kernel_size (got %lld, %lld)", (long long)ksize, (long long)width);
}

}  // namespace
}  // namespace oq

extern "C" int oq_causal_conv1d_update(const void* x, int dtype, int64_t x_stride_b, int64_t x_stride_c,
                                       int64_t x_stride_t, void* conv_state, const void* weight, const void* bias,
                                       int w_dtype, void* out, int64_t batch, int64_t channels, int64_t seq_len,
                                       int64_t state_width, int64_t kernel_size, int silu, void* stream) {
  using namespace oq;
  if (!valid_dtype(dtype) || !valid_dtype(w_dtype)) return fail(OQ_ERR_UNSUPPORTED, "causal_conv1d_update: unknown dtype");
  if (w_dtype != dtype && w_dtype != OQ_F32) {
    return fail(OQ_ERR_UNSUPPORTED, "causal_conv1d_update: weight/bias must be fp32 or x's dtype");
  }
  if (batch < 0 || channels <= 0 || seq_len < 0) return fail(OQ_ERR_INVALID_ARGUMENT, "causal_conv1d_update: bad sizes");
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
  p.out = out;
  p.batch = batch;
  p.channels = channels;
  p.seq_len = seq_len;
  p.silu = silu;
  const int64_t blocks = (batch * channels + kThreads - 1) / kThreads;
  if (blocks > 0x7fffffff) return fail(OQ_ERR_UNSUPPORTED, "causal_conv1d_update: too many channels");
  const dim3 grid((unsigned)blocks);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int st;
  const bool wf = w_dtype == OQ_F32;
  switch (dtype) {
    case OQ_F32: st = launch_conv<float, float>(p, state_width, kernel_size, grid, s); break;
    case OQ_F16:
      st = wf ? launch_conv<__half, float>(p, state_width, kernel_size, grid, s)
              : launch_conv<__half, __half>(p, state_width, kernel_size, grid, s);
      break;
    default:
      st = wf ? launch_conv<__nv_bfloat16, float>(p, state_width, kernel_size, grid, s)
              : launch_conv<__nv_bfloat16, __nv_bfloat16>(p, state_width, kernel_size, grid, s);
  }
  if (st != OQ_OK) return st;
  return check_launch("causal_conv1d_update");
}
