// Gated delta rule, recurrent form (the GDN decode step).
//
// Replaces the hook `recurrent_gated_delta_rule` of Qwen3_5GatedDeltaNet
// (transformers models/qwen3_5/modeling_qwen3_5.py:511-520; fla 0.5.1
// fused_recurrent_gated_delta_rule, fla/ops/gated_delta_rule/fused_recurrent.py:291;
// torch fallback modeling_qwen3_5.py:314-353).  The fp32 state of one head is
// 128 x 128 = 64 KiB; a CTA owns a 128 x 32 column slice of it in registers
// (32 floats per thread), so every state byte crosses HBM exactly once per
// launch in each direction, however many tokens the launch steps through:
//   S *= exp(g);  kv = S^T k;  delta = beta (v - kv);  S += k delta^T;  o = S^T q.
// Column sums over the 128 state rows are reduced with warp shuffles and a
// 4-warp shared-memory step.  The plain step with a given initial state (the decode
// step) keeps the slice in shared memory instead (gdn_smem_kernel below), which lets twice
// as many slices be in flight per SM.  The fused conv / norm variants
// and the zero-initial-state case hold the slice in registers.
//
// Optional gated RMSNorm epilogue: the GDN layer's Qwen3_5RMSNormGated(o, z)
// (modeling_qwen3_5.py:175-190, call site :527-529) over each head's 128 outputs.  The
// four column-slice CTAs of a head store their outputs as usual and count themselves in
// on a per-(sequence, head) counter; the last to arrive reads the head's outputs back
// (from L2) and rewrites them normalised.  No CTA waits for another (a cluster-wide
// exchange measured ~8 us slower per launch on B200).
#include <algorithm>
#include <cmath>

#include "common.cuh"

namespace oq {
namespace {

constexpr int kDk = 128;
constexpr int kDv = 128;
constexpr int kCols = 32;               // state columns per CTA
constexpr int kThreads = 128;           // = kDk: one q/k element per thread when loading
constexpr int kRowsPerThread = kDk / 16;  // 16 row groups x 8 rows

struct GdnParams {
  const void *q, *k, *v;
  int64_t qs[3], ks[3], vs[3];  // strides (b, t, h) in elements
  const void *g, *beta;
  int g_dtype, beta_dtype;
  const float* s_in;
  float* s_out;
  void* out;
  int64_t seq_len, num_heads;
  float scale;
  int l2norm;
  int prefetch_state;  // read the state before waiting for the preceding kernel
  // fused causal conv1d update (decode, T = 1): q, k, v = silu(conv(state | x)) of the
  // projection output x = qkv [B, C] (channels: q heads, k heads, v heads)
  const void* qkv;
  int64_t qkv_sb;
  void* conv_state;  // [B, C, W] in T
  const void* conv_w;  // [C, K]
  const void* conv_b;  // [C] or null, in T
  int64_t conv_channels;
  // gated RMSNorm epilogue: out = rnd(rnd(rnd(o * rsqrt(mean(o^2) + eps)) * w) * silu(z))
  const void* z;       // [B, T, H, Dv] gate in T (strides b, t, h)
  int64_t zs[3];
  const void* norm_w;  // [Dv] in T
  float norm_eps;
  int* norm_counters;  // [B * H] zeroed; every launch leaves them zero
  int32_t* status_word;  // OQ_DEV_* bits of the shared-memory kernel's bounded wait (may be null)
  int wait_polls;        // polls of that wait (wait_polls() at launch)
  // raw gate inputs (oq_gdn_recurrent_gates; null: g and beta are given): a, b [B, T, H] in
  // ab_dtype, A_log and dt_bias [H]
  const void *gate_a, *gate_b, *a_log, *dt_bias;
  int ab_dtype, a_log_dtype, dt_bias_dtype;
};

__device__ __forceinline__ float round_to(int dtype, float x) {
  if (dtype == OQ_BF16) return __bfloat162float(__float2bfloat16_rn(x));
  if (dtype == OQ_F16) return __half2float(__float2half_rn(x));
  return x;
}

// The token's decay exponent g and write strength beta.  Given directly, or from the layer's
// raw projections as Qwen3_5GatedDeltaNet.forward computes them (transformers
// models/qwen3_5/modeling_qwen3_5.py:492-493): beta = sigmoid(b) in b's dtype, and in fp32
// g = -exp(A_log) * softplus(a + dt_bias), softplus(x) = x above 20 (torch's threshold),
// else log(1 + exp(x)).
template <int kRaw = -1>  // 1: raw projections, 0: g and beta given, -1: decided from p at run time
__device__ __forceinline__ void step_gates(const GdnParams& p, int64_t gi, int64_t h, float& g, float& beta) {
  if (kRaw == 0 || (kRaw < 0 && p.gate_a == nullptr)) {
    g = load_as_float(p.g, p.g_dtype, gi);
    beta = load_as_float(p.beta, p.beta_dtype, gi);
    return;
  }
  const float bv = load_as_float(p.gate_b, p.ab_dtype, gi);
  const float x = load_as_float(p.gate_a, p.ab_dtype, gi) + load_as_float(p.dt_bias, p.dt_bias_dtype, h);
  const float a_log = load_as_float(p.a_log, p.a_log_dtype, h);
  beta = round_to(p.ab_dtype, 1.0f / (1.0f + expf(-bv)));
  const float softplus = x > 20.0f ? x : log1pf(expf(x));
  g = -expf(a_log) * softplus;
}

constexpr int kConvWidth = 4;  // state width = kernel size = 4 (Qwen3.5's conv_kernel_size)

// One channel of the causal conv1d update for the single new token: the output
// (rounded to the input dtype, as the unfused layer hands it on) and the shifted
// window [state[1..3], x], which becomes the channel's new state.  Every load is
// unconditional, so all of them are in flight together.
template <typename T>
__device__ __forceinline__ float conv_channel(const GdnParams& p, int64_t b, int64_t c, float (&hist)[kConvWidth]) {
  const T* st = static_cast<const T*>(p.conv_state) + (b * p.conv_channels + c) * kConvWidth;
  const T* wr = static_cast<const T*>(p.conv_w) + c * kConvWidth;
#pragma unroll
  for (int j = 0; j + 1 < kConvWidth; ++j) hist[j] = to_float<T>(st[j + 1]);
  hist[kConvWidth - 1] = to_float<T>(static_cast<const T*>(p.qkv)[b * p.qkv_sb + c]);
  float acc = p.conv_b != nullptr ? to_float<T>(static_cast<const T*>(p.conv_b)[c]) : 0.0f;
#pragma unroll
  for (int k = 0; k < kConvWidth; ++k) acc = fmaf(to_float<T>(wr[k]), hist[k], acc);
  return to_float<T>(from_float<T>(acc / (1.0f + expf(-acc))));
}

template <typename T>
__device__ __forceinline__ void conv_store(const GdnParams& p, int64_t b, int64_t c, const float (&hist)[kConvWidth]) {
  T* st = static_cast<T*>(p.conv_state) + (b * p.conv_channels + c) * kConvWidth;
#pragma unroll
  for (int j = 0; j < kConvWidth; ++j) st[j] = from_float<T>(hist[j]);
}

__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.aligned;\nbarrier.cluster.wait.aligned;\n" ::: "memory");
}

template <typename T, bool kConv, bool kNorm>
__global__ void __launch_bounds__(kThreads) gdn_recurrent_kernel(GdnParams p) {
  __shared__ float q_s[kDk], k_s[kDk], v_s[kCols];
  __shared__ float red_kv[4][kCols], red_o[4][kCols];
  __shared__ float norm_q[4], norm_k[4];
  __shared__ float norm_red[4];
  __shared__ int norm_last;

  const int tid = threadIdx.x;
  const int lane = tid & 31;
  const int warp = tid >> 5;
  const int cg = lane & 7;                 // column group: columns 4cg .. 4cg+3 of the slice
  const int rg = (lane >> 3) + 4 * warp;   // row group: rows rg + 16 i
  const int v0 = blockIdx.x * kCols;
  const int64_t h = blockIdx.y;
  const int64_t b = blockIdx.z;
  const int64_t H = p.num_heads;

  float S[kRowsPerThread][4];
  const int64_t state_off = ((b * H + h) * kDk) * kDv + v0 + 4 * cg;
  // The state is the dominant traffic.  With prefetch_state the caller guarantees no
  // kernel still running ahead of this one writes it, so its loads are issued before
  // the dependency wait and overlap the previous kernel's tail.
  if (!p.prefetch_state) pdl_wait();
  if (p.s_in != nullptr) {
#pragma unroll
    for (int i = 0; i < kRowsPerThread; ++i) {
      const float4 x = *reinterpret_cast<const float4*>(p.s_in + state_off + int64_t(rg + 16 * i) * kDv);
      S[i][0] = x.x;
      S[i][1] = x.y;
      S[i][2] = x.z;
      S[i][3] = x.w;
    }
  } else {
#pragma unroll
    for (int i = 0; i < kRowsPerThread; ++i) S[i][0] = S[i][1] = S[i][2] = S[i][3] = 0.0f;
  }
  if (p.prefetch_state) pdl_wait();
  pdl_allow_next();

  for (int64_t t = 0; t < p.seq_len; ++t) {
    const T* qrow = static_cast<const T*>(p.q) + b * p.qs[0] + t * p.qs[1] + h * p.qs[2];
    const T* krow = static_cast<const T*>(p.k) + b * p.ks[0] + t * p.ks[1] + h * p.ks[2];
    const T* vrow = static_cast<const T*>(p.v) + b * p.vs[0] + t * p.vs[1] + h * p.vs[2];
    float qv, kvv;
    if constexpr (kConv) {
      // q / k channels of this head and v channels of this slice through the conv; the
      // four slice CTAs of a head form a cluster: all read the old state, then rank 0
      // writes the q / k state and every CTA its own v channels.
      float hq[kConvWidth], hk[kConvWidth], hv[kConvWidth];
      const int64_t ch_q = h * kDk + tid, ch_k = H * kDk + h * kDk + tid, ch_v = 2 * H * kDk + h * kDv + v0 + tid;
      qv = conv_channel<T>(p, b, ch_q, hq);
      kvv = conv_channel<T>(p, b, ch_k, hk);
      float vv = 0.0f;
      if (tid < kCols) vv = conv_channel<T>(p, b, ch_v, hv);
      if (tid < kCols) v_s[tid] = vv;
      cluster_sync();
      if (blockIdx.x == 0) {
        conv_store<T>(p, b, ch_q, hq);
        conv_store<T>(p, b, ch_k, hk);
      }
      if (tid < kCols) conv_store<T>(p, b, ch_v, hv);
    } else {
      qv = to_float<T>(qrow[tid]);
      kvv = to_float<T>(krow[tid]);
      if (tid < kCols) v_s[tid] = to_float<T>(vrow[v0 + tid]);
    }
    q_s[tid] = qv;
    k_s[tid] = kvv;
    if (p.l2norm) {
      float sq = qv * qv, sk = kvv * kvv;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        sq += __shfl_xor_sync(0xffffffffu, sq, o);
        sk += __shfl_xor_sync(0xffffffffu, sk, o);
      }
      if (lane == 0) {
        norm_q[warp] = sq;
        norm_k[warp] = sk;
      }
    }
    const int64_t gi = (b * p.seq_len + t) * H + h;
    float gt, bt;
    step_gates(p, gi, h, gt, bt);
    __syncthreads();

    float inv_q = 1.0f, inv_k = 1.0f;
    if (p.l2norm) {
      // l2norm: x * rsqrt(sum(x*x) + 1e-6)  (modeling_qwen3_5.py:228-231)
      inv_q = 1.0f / sqrtf((norm_q[0] + norm_q[1]) + (norm_q[2] + norm_q[3]) + 1e-6f);
      inv_k = 1.0f / sqrtf((norm_k[0] + norm_k[1]) + (norm_k[2] + norm_k[3]) + 1e-6f);
    }
    const float decay = expf(gt);

    // S *= exp(g); partial kv = sum_rows S * k
    float kv[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    float kr[kRowsPerThread];
#pragma unroll
    for (int i = 0; i < kRowsPerThread; ++i) {
      kr[i] = __fmul_rn(k_s[rg + 16 * i], inv_k);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        S[i][j] = __fmul_rn(S[i][j], decay);
        kv[j] = fmaf(S[i][j], kr[i], kv[j]);
      }
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      kv[j] += __shfl_xor_sync(0xffffffffu, kv[j], 8);
      kv[j] += __shfl_xor_sync(0xffffffffu, kv[j], 16);
    }
    if (lane < 8) {
#pragma unroll
      for (int j = 0; j < 4; ++j) red_kv[warp][4 * cg + j] = kv[j];
    }
    __syncthreads();

    // delta = beta (v - kv); S += k delta^T; partial o = sum_rows S * q
    float delta[4], o[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int col = 4 * cg + j;
      const float kvs = (red_kv[0][col] + red_kv[1][col]) + (red_kv[2][col] + red_kv[3][col]);
      delta[j] = __fmul_rn(__fsub_rn(v_s[col], kvs), bt);
    }
#pragma unroll
    for (int i = 0; i < kRowsPerThread; ++i) {
      const float qr = __fmul_rn(__fmul_rn(q_s[rg + 16 * i], inv_q), p.scale);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        S[i][j] = fmaf(kr[i], delta[j], S[i][j]);
        o[j] = fmaf(S[i][j], qr, o[j]);
      }
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      o[j] += __shfl_xor_sync(0xffffffffu, o[j], 8);
      o[j] += __shfl_xor_sync(0xffffffffu, o[j], 16);
    }
    if (lane < 8) {
#pragma unroll
      for (int j = 0; j < 4; ++j) red_o[warp][4 * cg + j] = o[j];
    }
    __syncthreads();
    if (tid < kCols) {
      const float ov = (red_o[0][tid] + red_o[1][tid]) + (red_o[2][tid] + red_o[3][tid]);
      static_cast<T*>(p.out)[((b * p.seq_len + t) * H + h) * kDv + v0 + tid] = from_float<T>(ov);
    }
  }

  if constexpr (kNorm) {
    // ---- gated RMSNorm by the last of the head's four slice CTAs: its outputs, in the model
    // dtype as the unfused layer hands them to the norm, are read back for every token
    __threadfence();
    __syncthreads();
    if (tid == 0) {
      const int done = atomicAdd(&p.norm_counters[b * H + h], 1);
      norm_last = done == kDv / kCols - 1;
    }
    __syncthreads();
    if (norm_last) {
      __threadfence();
      const float wv = to_float<T>(static_cast<const T*>(p.norm_w)[tid]);
      for (int64_t t = 0; t < p.seq_len; ++t) {
        T* orow = static_cast<T*>(p.out) + ((b * p.seq_len + t) * H + h) * kDv;
        const float zv = to_float<T>(static_cast<const T*>(p.z)[b * p.zs[0] + t * p.zs[1] + h * p.zs[2] + tid]);
        const float ov = to_float<T>(__ldcg(orow + tid));
        float ss = ov * ov;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
        if (lane == 0) norm_red[warp] = ss;
        __syncthreads();
        const float tot = (norm_red[0] + norm_red[1]) + (norm_red[2] + norm_red[3]);
        const float inv = 1.0f / sqrtf(tot * (1.0f / kDv) + p.norm_eps);
        const float nrm = to_float<T>(from_float<T>(ov * inv));
        const float y = to_float<T>(from_float<T>(wv * nrm));
        orow[tid] = from_float<T>(y * (zv / (1.0f + expf(-zv))));
        __syncthreads();  // norm_red is reused by the next token
      }
      if (tid == 0) p.norm_counters[b * H + h] = 0;  // ready for the next launch
    }
  }

  if (p.s_out != nullptr) {
#pragma unroll
    for (int i = 0; i < kRowsPerThread; ++i) {
      *reinterpret_cast<float4*>(p.s_out + state_off + int64_t(rg + 16 * i) * kDv) =
          make_float4(S[i][0], S[i][1], S[i][2], S[i][3]);
    }
  }
}

// ---- Shared-memory form of the plain step (no fused conv or norm; an initial state is
// given): one CTA per (sequence, head, 32-column slice) as above, but the slice lives in
// shared memory instead of registers.  One TMA copy brings it in; phase 1 reads it
// (decayed on the fly) for kv, phase 2 reads it again, applies the decay and the rank-1
// update and writes it back for the next token; the final values go straight to global
// memory.  Without 32 state floats per thread the CTA needs about half the registers, so
// twice as many slices are in flight per SM.  The arithmetic is that of
// gdn_recurrent_kernel, operation for operation (the decay product is recomputed in
// phase 2 with the same rounding).
constexpr int kSliceFloats = kDk * kCols;  // 16 KB
constexpr size_t kSmemSlice = size_t(kSliceFloats) * 4 + 128;

// Bounded wait on a copy's mbarrier (sleeping in try_wait up to 20 us per poll; the default
// kDefaultWaitPolls is ~2 s in all); false if it ran out.
__device__ __forceinline__ bool wait_bar_bounded(uint64_t* bar, uint32_t parity, int polls) {
  for (int i = 0; i < polls; ++i) {
    if (mbar_try_wait_suspend(bar, parity, 20000)) return true;
  }
  return false;
}

// The slice copy did not land within the caller's limit: report it, and let thread 0 wait for
// the copy (at the default limit) so that the CTA, whose shared memory the copy writes, does
// not end while it is in flight.  Nothing has been written to global memory yet, so the
// state and the outputs of this slice are left as they were.  (This kernel has no fused norm,
// so no norm counter is involved.)
__device__ __forceinline__ void slice_timeout(const GdnParams& p, uint64_t* bar, int tid) {
  if (tid == 0) {
    report(p.status_word, OQ_DEV_TIMEOUT);
    wait_bar_bounded(bar, 0, kDefaultWaitPolls);
  }
}

// 10 CTAs per SM (48 registers, no spill): at B = 64 x 16 heads x 4 slices = 4096 CTAs the
// grid is 2.77 waves of 1480 slots, where 9 per SM (55 registers) left a last wave of 100
// CTAs that cannot keep HBM busy; 11 per SM (2.52 waves) measured slower than 10.
template <typename T, bool kRaw>
__global__ void __launch_bounds__(kThreads, 10) gdn_smem_kernel(const __grid_constant__ CUtensorMap tmap, GdnParams p) {
  extern __shared__ uint8_t slice_raw[];
  float* sl = reinterpret_cast<float*>((reinterpret_cast<uintptr_t>(slice_raw) + 127) & ~uintptr_t(127));
  __shared__ uint64_t full;
  __shared__ float q_s[kDk], k_s[kDk], v_s[kCols];
  __shared__ float red_kv[4][kCols], red_o[4][kCols];
  __shared__ float norm_q[4], norm_k[4];

  const int tid = threadIdx.x;
  const int lane = tid & 31;
  const int warp = tid >> 5;
  const int cg = lane & 7;                // column group: columns 4cg .. 4cg+3 of the slice
  const int rg = (lane >> 3) + 4 * warp;  // row group: rows rg + 16 i
  const int v0 = blockIdx.x * kCols;
  const int64_t h = blockIdx.y;
  const int64_t b = blockIdx.z;
  const int64_t H = p.num_heads;

  if (tid == 0) {
    mbar_init(&full, 1);
    fence_mbar_init();
  }
  // The state is the dominant traffic.  With prefetch_state the caller guarantees no
  // kernel still running ahead of this one writes it, so its copy goes out before the
  // dependency wait and overlaps the previous kernel's tail.
  if (!p.prefetch_state) pdl_wait();
  if (tid == 0) {
    mbar_arrive_expect_tx(&full, kSliceFloats * 4);
    tma_load_2d(sl, &tmap, v0, int32_t((b * H + h) * kDk), &full);
  }
  if (p.prefetch_state) pdl_wait();
  pdl_allow_next();

  // this thread's elements: rows rg + 16 i, columns 4cg .. 4cg+3 of the slice
  auto elem = [&](int i) { return reinterpret_cast<float4*>(sl + (rg + 16 * i) * kCols + 4 * cg); };
  bool landed = false;  // the copy is waited for once, after the first token's inputs are loaded

  for (int64_t t = 0; t < p.seq_len; ++t) {
    const T* qrow = static_cast<const T*>(p.q) + b * p.qs[0] + t * p.qs[1] + h * p.qs[2];
    const T* krow = static_cast<const T*>(p.k) + b * p.ks[0] + t * p.ks[1] + h * p.ks[2];
    const T* vrow = static_cast<const T*>(p.v) + b * p.vs[0] + t * p.vs[1] + h * p.vs[2];
    const float qv = to_float<T>(qrow[tid]);
    const float kvv = to_float<T>(krow[tid]);
    if (tid < kCols) v_s[tid] = to_float<T>(vrow[v0 + tid]);
    q_s[tid] = qv;
    k_s[tid] = kvv;
    if (p.l2norm) {
      float sq = qv * qv, sk = kvv * kvv;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        sq += __shfl_xor_sync(0xffffffffu, sq, o);
        sk += __shfl_xor_sync(0xffffffffu, sk, o);
      }
      if (lane == 0) {
        norm_q[warp] = sq;
        norm_k[warp] = sk;
      }
    }
    const int64_t gi = (b * p.seq_len + t) * H + h;
    float gt, bt;
    step_gates<kRaw ? 1 : 0>(p, gi, h, gt, bt);
    if (!landed) {
      // thread 0 initialised the barrier; every thread sees that before it polls it
      __syncthreads();
      const bool ok = wait_bar_bounded(&full, 0, p.wait_polls);
      if (__syncthreads_or(!ok)) {
        slice_timeout(p, &full, tid);
        return;
      }
      landed = true;
    } else {
      __syncthreads();
    }

    float inv_q = 1.0f, inv_k = 1.0f;
    if (p.l2norm) {
      // l2norm: x * rsqrt(sum(x*x) + 1e-6)  (modeling_qwen3_5.py:228-231)
      inv_q = 1.0f / sqrtf((norm_q[0] + norm_q[1]) + (norm_q[2] + norm_q[3]) + 1e-6f);
      inv_k = 1.0f / sqrtf((norm_k[0] + norm_k[1]) + (norm_k[2] + norm_k[3]) + 1e-6f);
    }
    const float decay = expf(gt);

    // phase 1: partial kv = sum_rows (S * exp(g)) * k
    float kv[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    float kr[kRowsPerThread];
#pragma unroll
    for (int i = 0; i < kRowsPerThread; ++i) {
      kr[i] = __fmul_rn(k_s[rg + 16 * i], inv_k);
      const float4 x = *elem(i);
      kv[0] = fmaf(__fmul_rn(x.x, decay), kr[i], kv[0]);
      kv[1] = fmaf(__fmul_rn(x.y, decay), kr[i], kv[1]);
      kv[2] = fmaf(__fmul_rn(x.z, decay), kr[i], kv[2]);
      kv[3] = fmaf(__fmul_rn(x.w, decay), kr[i], kv[3]);
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      kv[j] += __shfl_xor_sync(0xffffffffu, kv[j], 8);
      kv[j] += __shfl_xor_sync(0xffffffffu, kv[j], 16);
    }
    if (lane < 8) {
#pragma unroll
      for (int j = 0; j < 4; ++j) red_kv[warp][4 * cg + j] = kv[j];
    }
    __syncthreads();

    // phase 2: delta = beta (v - kv); S = S exp(g) + k delta^T; partial o = sum_rows S * q
    float delta[4], o[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int col = 4 * cg + j;
      const float kvs = (red_kv[0][col] + red_kv[1][col]) + (red_kv[2][col] + red_kv[3][col]);
      delta[j] = __fmul_rn(__fsub_rn(v_s[col], kvs), bt);
    }
    const bool last = t + 1 == p.seq_len;
    const int64_t state_off = ((b * H + h) * kDk) * kDv + v0 + 4 * cg;
#pragma unroll
    for (int i = 0; i < kRowsPerThread; ++i) {
      const float qr = __fmul_rn(__fmul_rn(q_s[rg + 16 * i], inv_q), p.scale);
      float4 x = *elem(i);
      x.x = fmaf(kr[i], delta[0], __fmul_rn(x.x, decay));
      x.y = fmaf(kr[i], delta[1], __fmul_rn(x.y, decay));
      x.z = fmaf(kr[i], delta[2], __fmul_rn(x.z, decay));
      x.w = fmaf(kr[i], delta[3], __fmul_rn(x.w, decay));
      o[0] = fmaf(x.x, qr, o[0]);
      o[1] = fmaf(x.y, qr, o[1]);
      o[2] = fmaf(x.z, qr, o[2]);
      o[3] = fmaf(x.w, qr, o[3]);
      if (last) {
        if (p.s_out != nullptr) *reinterpret_cast<float4*>(p.s_out + state_off + int64_t(rg + 16 * i) * kDv) = x;
      } else {
        *elem(i) = x;
      }
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      o[j] += __shfl_xor_sync(0xffffffffu, o[j], 8);
      o[j] += __shfl_xor_sync(0xffffffffu, o[j], 16);
    }
    if (lane < 8) {
#pragma unroll
      for (int j = 0; j < 4; ++j) red_o[warp][4 * cg + j] = o[j];
    }
    __syncthreads();
    if (tid < kCols) {
      const float ov = (red_o[0][tid] + red_o[1][tid]) + (red_o[2][tid] + red_o[3][tid]);
      static_cast<T*>(p.out)[((b * p.seq_len + t) * H + h) * kDv + v0 + tid] = from_float<T>(ov);
    }
  }
  if (p.seq_len == 0) {
    // no token: the state passes through unchanged
    __syncthreads();  // (the barrier's initialisation, as above)
    const bool ok = wait_bar_bounded(&full, 0, p.wait_polls);
    if (__syncthreads_or(!ok)) {
      slice_timeout(p, &full, tid);
      return;
    }
    if (p.s_out != nullptr) {
      const int64_t state_off = ((b * H + h) * kDk) * kDv + v0 + 4 * cg;
#pragma unroll
      for (int i = 0; i < kRowsPerThread; ++i) {
        *reinterpret_cast<float4*>(p.s_out + state_off + int64_t(rg + 16 * i) * kDv) = *elem(i);
      }
    }
  }
}

// Early (programmatic) launch only when the caller allows the state prefetch.
void launch_gdn(void (*kernel)(GdnParams), dim3 grid, cudaStream_t s, const GdnParams& p) {
  if (p.prefetch_state) {
    launch_pdl(kernel, grid, dim3(kThreads), 0, s, p);
  } else {
    launch_plain(kernel, grid, dim3(kThreads), 0, s, p);
  }
}

// The fused conv variant runs the four column slices of a head as one cluster.
cudaError_t launch_gdn_cluster(void (*kernel)(GdnParams), dim3 grid, cudaStream_t s, const GdnParams& p) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(kThreads);
  cfg.stream = s;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = kDv / kCols;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = p.prefetch_state ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  return cudaLaunchKernelEx(&cfg, kernel, p);
}

// Raw gate inputs of oq_gdn_recurrent_gates (null: g and beta are given).
struct RawGates {
  const void *a, *b;
  int ab_dtype;
  const void* a_log;
  int a_log_dtype;
  const void* dt_bias;
  int dt_bias_dtype;
};

// Gated RMSNorm epilogue arguments (null: plain output).
struct NormArgs {
  const void* z;
  int64_t zs[3];
  const void* weight;
  float eps;
  int* counters;
  size_t counter_bytes;
};

template <bool kConv>
void (*gdn_kernel_for(int dtype, bool norm))(GdnParams) {
  if (norm) {
    switch (dtype) {
      case OQ_F32: return gdn_recurrent_kernel<float, kConv, true>;
      case OQ_F16: return gdn_recurrent_kernel<__half, kConv, true>;
      default: return gdn_recurrent_kernel<__nv_bfloat16, kConv, true>;
    }
  }
  switch (dtype) {
    case OQ_F32: return gdn_recurrent_kernel<float, kConv, false>;
    case OQ_F16: return gdn_recurrent_kernel<__half, kConv, false>;
    default: return gdn_recurrent_kernel<__nv_bfloat16, kConv, false>;
  }
}

int check_norm(const NormArgs* norm, int64_t batch, int64_t num_heads, const char* what) {
  if (norm && (!norm->z || !norm->weight)) return fail(OQ_ERR_INVALID_ARGUMENT, "%s: null gate or norm weight", what);
  if (norm && (!norm->counters || norm->counter_bytes < size_t(batch * num_heads) * sizeof(int))) {
    return fail(OQ_ERR_WORKSPACE, "%s: norm workspace of %zu bytes needed", what,
                size_t(batch * num_heads) * sizeof(int));
  }
  if (norm && !(norm->eps >= 0.0f)) return fail(OQ_ERR_INVALID_ARGUMENT, "%s: norm eps must be >= 0", what);
  return OQ_OK;
}

void set_norm(GdnParams& p, const NormArgs* norm) {
  p.z = norm ? norm->z : nullptr;
  p.zs[0] = norm ? norm->zs[0] : 0;
  p.zs[1] = norm ? norm->zs[1] : 0;
  p.zs[2] = norm ? norm->zs[2] : 0;
  p.norm_w = norm ? norm->weight : nullptr;
  p.norm_eps = norm ? norm->eps : 0.0f;
  p.norm_counters = norm ? norm->counters : nullptr;
}

// 2-D map over the fp32 state [B * H * 128 rows, 128 columns]: box = one 32-column slice
// of a head's 128 rows (16 KB, no swizzle).
int encode_state_map(CUtensorMap* map, const float* state, int64_t rows) {
  auto fn = tensor_map_encoder();
  if (fn == nullptr) return fail(OQ_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
  const cuuint64_t dims[2] = {cuuint64_t(kDv), cuuint64_t(rows)};
  const cuuint64_t strides[1] = {cuuint64_t(kDv) * 4};
  const cuuint32_t box[2] = {cuuint32_t(kCols), cuuint32_t(kDk)};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult res = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(state), dims, strides, box, estr,
                          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (res != CUDA_SUCCESS) return fail(OQ_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", int(res));
  return OQ_OK;
}

template <typename T, bool kRaw>
int launch_smem_as(const GdnParams& p, int64_t batch, cudaStream_t s) {
  CUtensorMap tmap;
  if (int st = encode_state_map(&tmap, p.s_in, batch * p.num_heads * kDk); st != OQ_OK) return st;
  cudaFuncSetAttribute(gdn_smem_kernel<T, kRaw>, cudaFuncAttributeMaxDynamicSharedMemorySize, int(kSmemSlice));
  const dim3 grid(unsigned(kDv / kCols), unsigned(p.num_heads), unsigned(batch));
  if (p.prefetch_state) {
    launch_pdl(gdn_smem_kernel<T, kRaw>, grid, dim3(kThreads), kSmemSlice, s, tmap, p);
  } else {
    launch_plain(gdn_smem_kernel<T, kRaw>, grid, dim3(kThreads), kSmemSlice, s, tmap, p);
  }
  return OQ_OK;
}

// (the raw-gate form is a separate instance: the given-gates step keeps no branch for it)
template <typename T>
int launch_smem(const GdnParams& p, int64_t batch, cudaStream_t s) {
  return p.gate_a != nullptr ? launch_smem_as<T, true>(p, batch, s) : launch_smem_as<T, false>(p, batch, s);
}

int gdn_recurrent_impl(
    const void* q, const void* k, const void* v, int qkv_dtype,
    int64_t q_stride_b, int64_t q_stride_t, int64_t q_stride_h,
    int64_t k_stride_b, int64_t k_stride_t, int64_t k_stride_h,
    int64_t v_stride_b, int64_t v_stride_t, int64_t v_stride_h,
    const void* g, int g_dtype, const void* beta, int beta_dtype,
    const float* initial_state, float* final_state, void* out,
    int64_t batch, int64_t seq_len, int64_t num_heads, int64_t k_dim, int64_t v_dim,
    float scale, int use_qk_l2norm, const NormArgs* norm, int flags, int32_t* device_status, void* stream,
    const RawGates* raw = nullptr) {
  if (int st = check_norm(norm, batch, num_heads, "gdn_recurrent"); st != OQ_OK) return st;
  if (raw) {
    if (!valid_dtype(raw->ab_dtype) || !valid_dtype(raw->a_log_dtype) || !valid_dtype(raw->dt_bias_dtype)) {
      return fail(OQ_ERR_UNSUPPORTED, "gdn_recurrent_gates: unknown dtype");
    }
    if (!raw->a || !raw->b || !raw->a_log || !raw->dt_bias) {
      return fail(OQ_ERR_INVALID_ARGUMENT, "gdn_recurrent_gates: null gate input");
    }
    g_dtype = beta_dtype = OQ_F32;  // (unused)
  }
  if (!valid_dtype(qkv_dtype) || !valid_dtype(g_dtype) || !valid_dtype(beta_dtype)) {
    return fail(OQ_ERR_UNSUPPORTED, "gdn_recurrent: unknown dtype");
  }
  if (k_dim != kDk || v_dim != kDv) return fail(OQ_ERR_UNSUPPORTED, "gdn_recurrent: k_dim = v_dim = 128 required");
  if (batch < 0 || seq_len < 0 || num_heads <= 0) return fail(OQ_ERR_INVALID_ARGUMENT, "gdn_recurrent: bad sizes");
  if (batch == 0) return ok();
  if (batch > 65535 || num_heads > 65535) return fail(OQ_ERR_UNSUPPORTED, "gdn_recurrent: grid too large");
  if ((!raw && (!g || !beta)) || (seq_len > 0 && (!q || !k || !v || !out))) {
    return fail(OQ_ERR_INVALID_ARGUMENT, "gdn_recurrent: null pointer");
  }
  if ((initial_state && reinterpret_cast<uintptr_t>(initial_state) % 16) ||
      (final_state && reinterpret_cast<uintptr_t>(final_state) % 16)) {
    return fail(OQ_ERR_MISALIGNED, "gdn_recurrent: state must be 16-byte aligned");
  }
  GdnParams p = {};
  p.q = q;
  p.k = k;
  p.v = v;
  p.qs[0] = q_stride_b; p.qs[1] = q_stride_t; p.qs[2] = q_stride_h;
  p.ks[0] = k_stride_b; p.ks[1] = k_stride_t; p.ks[2] = k_stride_h;
  p.vs[0] = v_stride_b; p.vs[1] = v_stride_t; p.vs[2] = v_stride_h;
  p.g = g;
  p.beta = beta;
  p.g_dtype = g_dtype;
  p.beta_dtype = beta_dtype;
  p.s_in = initial_state;
  p.s_out = final_state;
  p.out = out;
  p.seq_len = seq_len;
  p.num_heads = num_heads;
  p.scale = scale;
  p.l2norm = use_qk_l2norm;
  p.prefetch_state = (flags & OQ_GDN_STATE_PREFETCH) != 0;
  p.status_word = device_status;
  p.wait_polls = wait_polls();
  if (raw) {
    p.gate_a = raw->a;
    p.gate_b = raw->b;
    p.ab_dtype = raw->ab_dtype;
    p.a_log = raw->a_log;
    p.a_log_dtype = raw->a_log_dtype;
    p.dt_bias = raw->dt_bias;
    p.dt_bias_dtype = raw->dt_bias_dtype;
  }
  set_norm(p, norm);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (norm == nullptr && initial_state != nullptr && batch * num_heads * kDk < (int64_t(1) << 31)) {
    // the plain step keeps the state slice in shared memory (the decode step's form)
    int st = OQ_OK;
    switch (qkv_dtype) {
      case OQ_F32: st = launch_smem<float>(p, batch, s); break;
      case OQ_F16: st = launch_smem<__half>(p, batch, s); break;
      default: st = launch_smem<__nv_bfloat16>(p, batch, s); break;
    }
    if (st != OQ_OK) return st;
    return check_launch("gdn_recurrent");
  }
  dim3 grid((unsigned)(kDv / kCols), (unsigned)num_heads, (unsigned)batch);
  launch_gdn(gdn_kernel_for<false>(qkv_dtype, norm != nullptr), grid, s, p);
  return check_launch("gdn_recurrent");
}

int gdn_conv_step_impl(
    const void* qkv, int qkv_dtype, int64_t qkv_stride_b,
    void* conv_state, const void* conv_weight, const void* conv_bias, int conv_w_dtype,
    int64_t conv_width, int64_t conv_kernel_size,
    const void* g, int g_dtype, const void* beta, int beta_dtype,
    const float* initial_state, float* final_state, void* out,
    int64_t batch, int64_t num_heads, int64_t k_dim, int64_t v_dim,
    float scale, int use_qk_l2norm, const NormArgs* norm, int flags, void* stream) {
  if (int st = check_norm(norm, batch, num_heads, "gdn_conv_step"); st != OQ_OK) return st;
  if (!valid_dtype(qkv_dtype) || !valid_dtype(g_dtype) || !valid_dtype(beta_dtype) || !valid_dtype(conv_w_dtype)) {
    return fail(OQ_ERR_UNSUPPORTED, "gdn_conv_step: unknown dtype");
  }
  if (k_dim != kDk || v_dim != kDv) return fail(OQ_ERR_UNSUPPORTED, "gdn_conv_step: k_dim = v_dim = 128 required");
  if (conv_kernel_size != kConvWidth || conv_width != kConvWidth || conv_w_dtype != qkv_dtype) {
    return fail(OQ_ERR_UNSUPPORTED, "gdn_conv_step: fused conv needs kernel_size = state width = 4 and weights in "
                "the qkv dtype (use oq_causal_conv1d_update + oq_gdn_recurrent otherwise)");
  }
  if (batch < 0 || num_heads <= 0) return fail(OQ_ERR_INVALID_ARGUMENT, "gdn_conv_step: bad sizes");
  if (batch == 0) return ok();
  if (batch > 65535 || num_heads > 65535) return fail(OQ_ERR_UNSUPPORTED, "gdn_conv_step: grid too large");
  if (!qkv || !conv_state || !conv_weight || !g || !beta || !out) {
    return fail(OQ_ERR_INVALID_ARGUMENT, "gdn_conv_step: null pointer");
  }
  if ((initial_state && reinterpret_cast<uintptr_t>(initial_state) % 16) ||
      (final_state && reinterpret_cast<uintptr_t>(final_state) % 16)) {
    return fail(OQ_ERR_MISALIGNED, "gdn_conv_step: state must be 16-byte aligned");
  }
  GdnParams p = {};
  p.g = g;
  p.beta = beta;
  p.g_dtype = g_dtype;
  p.beta_dtype = beta_dtype;
  p.s_in = initial_state;
  p.s_out = final_state;
  p.out = out;
  p.seq_len = 1;
  p.num_heads = num_heads;
  p.scale = scale;
  p.l2norm = use_qk_l2norm;
  p.prefetch_state = (flags & OQ_GDN_STATE_PREFETCH) != 0;
  p.qkv = qkv;
  p.qkv_sb = qkv_stride_b;
  p.conv_state = conv_state;
  p.conv_w = conv_weight;
  p.conv_b = conv_bias;
  p.conv_channels = num_heads * (2 * kDk + kDv);
  set_norm(p, norm);
  dim3 grid((unsigned)(kDv / kCols), (unsigned)num_heads, (unsigned)batch);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  launch_gdn_cluster(gdn_kernel_for<true>(qkv_dtype, norm != nullptr), grid, s, p);
  return check_launch("gdn_conv_step");
}

}  // namespace
}  // namespace oq

extern "C" int oq_gdn_recurrent(
    const void* q, const void* k, const void* v, int qkv_dtype,
    int64_t q_stride_b, int64_t q_stride_t, int64_t q_stride_h,
    int64_t k_stride_b, int64_t k_stride_t, int64_t k_stride_h,
    int64_t v_stride_b, int64_t v_stride_t, int64_t v_stride_h,
    const void* g, int g_dtype, const void* beta, int beta_dtype,
    const float* initial_state, float* final_state, void* out,
    int64_t batch, int64_t seq_len, int64_t num_heads, int64_t k_dim, int64_t v_dim,
    float scale, int use_qk_l2norm, int flags, int32_t* device_status, void* stream) {
  return oq::gdn_recurrent_impl(q, k, v, qkv_dtype, q_stride_b, q_stride_t, q_stride_h, k_stride_b, k_stride_t,
                                k_stride_h, v_stride_b, v_stride_t, v_stride_h, g, g_dtype, beta, beta_dtype,
                                initial_state, final_state, out, batch, seq_len, num_heads, k_dim, v_dim, scale,
                                use_qk_l2norm, nullptr, flags, device_status, stream);
}

extern "C" int oq_gdn_recurrent_gates(
    const void* q, const void* k, const void* v, int qkv_dtype,
    int64_t q_stride_b, int64_t q_stride_t, int64_t q_stride_h,
    int64_t k_stride_b, int64_t k_stride_t, int64_t k_stride_h,
    int64_t v_stride_b, int64_t v_stride_t, int64_t v_stride_h,
    const void* a, const void* b, int ab_dtype, const void* a_log, int a_log_dtype, const void* dt_bias,
    int dt_bias_dtype,
    const float* initial_state, float* final_state, void* out,
    int64_t batch, int64_t seq_len, int64_t num_heads, int64_t k_dim, int64_t v_dim,
    float scale, int use_qk_l2norm, int flags, int32_t* device_status, void* stream) {
  const oq::RawGates raw = {a, b, ab_dtype, a_log, a_log_dtype, dt_bias, dt_bias_dtype};
  return oq::gdn_recurrent_impl(q, k, v, qkv_dtype, q_stride_b, q_stride_t, q_stride_h, k_stride_b, k_stride_t,
                                k_stride_h, v_stride_b, v_stride_t, v_stride_h, nullptr, OQ_F32, nullptr, OQ_F32,
                                initial_state, final_state, out, batch, seq_len, num_heads, k_dim, v_dim, scale,
                                use_qk_l2norm, nullptr, flags, device_status, stream, &raw);
}

extern "C" int oq_gdn_recurrent_norm(
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
    int flags, void* stream) {
  const oq::NormArgs norm = {z, {z_stride_b, z_stride_t, z_stride_h}, norm_weight, norm_eps,
                             static_cast<int*>(norm_workspace), norm_workspace_bytes};
  return oq::gdn_recurrent_impl(q, k, v, qkv_dtype, q_stride_b, q_stride_t, q_stride_h, k_stride_b, k_stride_t,
                                k_stride_h, v_stride_b, v_stride_t, v_stride_h, g, g_dtype, beta, beta_dtype,
                                initial_state, final_state, out, batch, seq_len, num_heads, k_dim, v_dim, scale,
                                use_qk_l2norm, &norm, flags, nullptr, stream);
}

extern "C" int oq_gdn_conv_step(
    const void* qkv, int qkv_dtype, int64_t qkv_stride_b,
    void* conv_state, const void* conv_weight, const void* conv_bias, int conv_w_dtype,
    int64_t conv_width, int64_t conv_kernel_size,
    const void* g, int g_dtype, const void* beta, int beta_dtype,
    const float* initial_state, float* final_state, void* out,
    int64_t batch, int64_t num_heads, int64_t k_dim, int64_t v_dim,
    float scale, int use_qk_l2norm, int flags, void* stream) {
  return oq::gdn_conv_step_impl(qkv, qkv_dtype, qkv_stride_b, conv_state, conv_weight, conv_bias, conv_w_dtype,
                                conv_width, conv_kernel_size, g, g_dtype, beta, beta_dtype, initial_state,
                                final_state, out, batch, num_heads, k_dim, v_dim, scale, use_qk_l2norm, nullptr,
                                flags, stream);
}

extern "C" int oq_gdn_conv_step_norm(
    const void* qkv, int qkv_dtype, int64_t qkv_stride_b,
    void* conv_state, const void* conv_weight, const void* conv_bias, int conv_w_dtype,
    int64_t conv_width, int64_t conv_kernel_size,
    const void* g, int g_dtype, const void* beta, int beta_dtype,
    const float* initial_state, float* final_state, void* out,
    int64_t batch, int64_t num_heads, int64_t k_dim, int64_t v_dim,
    float scale, int use_qk_l2norm,
    const void* z, int64_t z_stride_b, int64_t z_stride_h, const void* norm_weight, float norm_eps,
    void* norm_workspace, size_t norm_workspace_bytes, int flags, void* stream) {
  const oq::NormArgs norm = {z, {z_stride_b, 0, z_stride_h}, norm_weight, norm_eps,
                             static_cast<int*>(norm_workspace), norm_workspace_bytes};
  return oq::gdn_conv_step_impl(qkv, qkv_dtype, qkv_stride_b, conv_state, conv_weight, conv_bias, conv_w_dtype,
                                conv_width, conv_kernel_size, g, g_dtype, beta, beta_dtype, initial_state,
                                final_state, out, batch, num_heads, k_dim, v_dim, scale, use_qk_l2norm, &norm, flags,
                                stream);
}

extern "C" size_t oq_gdn_norm_workspace_bytes(int64_t batch, int64_t num_heads) {
  if (batch <= 0 || num_heads <= 0) return 0;
  return size_t((batch * num_heads * int64_t(sizeof(int)) + 255) / 256 * 256);
}
