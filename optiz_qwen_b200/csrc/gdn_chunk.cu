// Gated delta rule, chunked form (GDN prefill) on the sm_100a tensor cores.
//
// Replaces the hook `chunk_gated_delta_rule` of Qwen3_5GatedDeltaNet (transformers
// models/qwen3_5/modeling_qwen3_5.py:466-476; torch fallback torch_chunk_gated_delta_rule
// :234-311; fla 0.5.1 chunk_gated_delta_rule, fla/ops/gated_delta_rule/chunk.py:365).
//
// One CTA owns one (sequence, head) and walks its 64-token chunks in order; the fp32
// state S [dk=128, dv=128] stays in tensor memory (TMEM) for the whole prompt.  All
// products are written with dv (the state column) on the 128 TMEM lanes, so every
// tcgen05.mma is M = 128.  Per chunk, with the raw bf16 rows Q, K, V [64 x 128] as TMA
// loads them, the L2 norms dq, dk, beta and the decays applied as diagonal factors:
//
//   G   = [K; Q] K^T                                              (exact bf16 products)
//   N   = -(beta_i dk_i dk_j G_kk[i][j] e^{gc_i - gc_j})_{j<i};  X = (I - N)^-1  (CUDA cores)
//   P   = (scale dq_i dk_j G_qk[i][j] e^{gc_i - gc_j})_{j<=i}
//   W^T = K^T (X diag(beta e^gc dk))^T,   U^T = V^T (X diag(beta))^T
//   (WS)^T = S^T W^T,   (QS)^T = S^T Q^T
//   Vn^T = U^T - (WS)^T
//   O^T = (QS)^T diag(scale dq e^gc) + Vn^T P^T,   dS^T = (Vn diag(dk e^{gc_last - gc}))^T K
//   S^T <- e^{gc_last} S^T + dS^T
//
// which is the WY form of the reference (u = value, w = k_cumdecay, attn_inter, v_new).
// fp32 operands (S, X, W, P, Vn) enter the bf16 tensor cores split into hi + lo bf16
// parts (x = hi + lo to about 2^-17 relative); a product of two such operands uses
// hi*hi + hi*lo + lo*hi, a product with a raw bf16 input uses hi*raw + lo*raw, so the
// fp32 results stay within the 1e-4 relative tolerance of the fp32 reference.
// Accumulation is fp32 in TMEM.  Operand tiles use the 128-byte swizzle, both as TMA
// writes them and as this kernel writes its own split tiles.
#include <cmath>
#include <cstring>

#include "common.cuh"

namespace oq {
namespace {

constexpr int kC = 64;          // chunk length
constexpr int kD = 128;         // dk = dv
constexpr int kThreads = 128;   // one thread per TMEM lane
constexpr uint32_t kTmemCols = 512;

// TMEM columns (fp32 accumulators, lane = dv row unless noted)
constexpr uint32_t kColG = 0;     // [K;Q]K^T (lane = token), then W^T (lane = dk), then Vn^T P^T
constexpr uint32_t kColU = 64;    // U^T
constexpr uint32_t kColWS = 128;  // (W S)^T
constexpr uint32_t kColQS = 192;  // (Q S)^T
constexpr uint32_t kColDS = 256;  // dS^T, 128 columns
constexpr uint32_t kColS = 384;   // S^T, 128 columns: the state

// Shared memory (byte offsets from a 1024-aligned base).  A "tile" is 64 rows x 128 B.
constexpr uint32_t kTile = 8192;
constexpr uint32_t kKQBytes = 4 * kTile;           // one input stage: K d<64 | Q d<64 | K d>=64 | Q d>=64
constexpr uint32_t kOffV = 2 * kKQBytes;           // V d<64 | V d>=64
constexpr uint32_t kOffS = kOffV + 2 * kTile;      // S^T hi (2 x 16 KB) | S^T lo; later Vn hi|Vn lo|Vs hi|Vs lo
constexpr uint32_t kOffW = kOffS + 65536;          // W hi | W lo (16 KB each); before that N, then Ar/Ab tiles
constexpr uint32_t kOffX = kOffW + 32768;          // X fp32 [64][65]
constexpr uint32_t kOffP = kOffX + 17408;          // P hi | P lo
constexpr uint32_t kOffSmall = kOffP + 2 * kTile;
constexpr int kXStride = 65;
constexpr int kTStride = 17;
// small area: 8 per-token float arrays, the off-diagonal solve scratch, barriers
constexpr uint32_t kSmallFloats = 8 * kC + 3 * 16 * kTStride;
constexpr uint32_t kOffBars = kOffSmall + kSmallFloats * 4;
constexpr uint32_t kSmemBytes = kOffBars + 64 + 1024;  // + alignment slack

constexpr uint32_t kWaitHintNs = 20000;
constexpr int kWaitPolls = 100000;  // ~2 s

constexpr uint32_t kIdescN64 = idesc_bf16_f32(128, 64, false, false);
constexpr uint32_t kIdescN64BMn = idesc_bf16_f32(128, 64, false, true);
constexpr uint32_t kIdescN64AMn = idesc_bf16_f32(128, 64, true, false);
constexpr uint32_t kIdescN128BMn = idesc_bf16_f32(128, 128, false, true);

struct ChunkParams {
  const void *g, *beta;
  int g_dtype, beta_dtype;
  const float* s_in;
  float* s_out;
  __nv_bfloat16* out;
  int64_t seq_len;
  int num_heads;
  float scale;
  int l2norm;
  int32_t* status;
};

struct Bars {
  uint64_t kq[2];
  uint64_t v;
  uint64_t mma;
  uint64_t drain;
  uint32_t tmem_base;
};

__device__ __forceinline__ bool wait_bar(uint64_t* bar, uint32_t parity) {
  for (int i = 0; i < kWaitPolls; ++i) {
    if (mbar_try_wait_suspend(bar, parity, kWaitHintNs)) return true;
  }
  return false;
}

// Byte offset of 16-byte chunk `chunk` of row `row` in a 128B-swizzled tile.
__device__ __forceinline__ uint32_t swz(uint32_t row, uint32_t chunk) {
  return (row >> 3) * 1024u + (row & 7u) * 128u + ((chunk ^ (row & 7u)) << 4);
}

__device__ __forceinline__ uint32_t bf16x2_bits(__nv_bfloat162 v) { return *reinterpret_cast<uint32_t*>(&v); }

// Splits 8 fp32 values into bf16 hi + lo parts and stores one 16-byte chunk of each.
__device__ __forceinline__ void store_split8(uint8_t* hi, uint8_t* lo, uint32_t off, const float* x) {
  uint32_t h[4], l[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const __nv_bfloat162 hh = __floats2bfloat162_rn(x[2 * i], x[2 * i + 1]);
    const float2 hf = __bfloat1622float2(hh);
    h[i] = bf16x2_bits(hh);
    l[i] = bf16x2_bits(__floats2bfloat162_rn(x[2 * i] - hf.x, x[2 * i + 1] - hf.y));
  }
  *reinterpret_cast<uint4*>(hi + off) = make_uint4(h[0], h[1], h[2], h[3]);
  *reinterpret_cast<uint4*>(lo + off) = make_uint4(l[0], l[1], l[2], l[3]);
}

// Stores 32 consecutive fp32 values of row `row` (chunks c0 .. c0+3) as split tiles.
__device__ __forceinline__ void store_split32(uint8_t* hi, uint8_t* lo, uint32_t row, uint32_t c0, const float* x) {
#pragma unroll
  for (int c = 0; c < 4; ++c) store_split8(hi, lo, swz(row, c0 + c), x + 8 * c);
}

// Sum of squares of one 128-element bf16 row held as two swizzled 64-element halves.
__device__ __forceinline__ float row_sumsq(const uint8_t* lo_half, const uint8_t* hi_half, uint32_t row) {
  float ss = 0.0f;
#pragma unroll
  for (int half = 0; half < 2; ++half) {
    const uint8_t* base = half ? hi_half : lo_half;
#pragma unroll
    for (int c = 0; c < 8; ++c) {
      const uint4 w = *reinterpret_cast<const uint4*>(base + swz(row, c));
      const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&ws[i]));
        ss = fmaf(f.x, f.x, ss);
        ss = fmaf(f.y, f.y, ss);
      }
    }
  }
  return ss;
}

__global__ void __launch_bounds__(kThreads, 1)
    gdn_chunk_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                     const __grid_constant__ CUtensorMap tm_v, ChunkParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sa = smem_addr(sm);
  float* f_small = reinterpret_cast<float*>(sm + kOffSmall);
  float* s_graw = f_small;
  float* s_gc = f_small + kC;
  float* s_beta = f_small + 2 * kC;
  float* s_dk = f_small + 3 * kC;
  float* s_dq = f_small + 4 * kC;
  float* s_sfac = f_small + 5 * kC;  // dk e^{gc_last - gc}
  float* s_cq = f_small + 6 * kC;    // scale dq e^{gc}
  float* s_rfac = f_small + 7 * kC;  // beta e^{gc} dk
  float* s_T = f_small + 8 * kC;     // [3][16][17]
  float* s_N = reinterpret_cast<float*>(sm + kOffW);
  float* s_X = reinterpret_cast<float*>(sm + kOffX);
  Bars* bars = reinterpret_cast<Bars*>(sm + kOffBars);

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int h = blockIdx.x;
  const int b = blockIdx.y;
  const int H = p.num_heads;
  const int64_t T = p.seq_len;
  const int n_chunks = int((T + kC - 1) / kC);

  if (tid == 0) {
    mbar_init(&bars->kq[0], 1);
    mbar_init(&bars->kq[1], 1);
    mbar_init(&bars->v, 1);
    mbar_init(&bars->mma, 1);
    mbar_init(&bars->drain, 1);
    fence_mbar_init();
  }
  __syncwarp();
  if (warp == 0) {
    tmem_alloc(&bars->tmem_base, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bars->tmem_base;
  const uint32_t lane_base = tmem + (uint32_t(warp * 32) << 16);

  // Load schedule (identical in every thread; only thread 0 issues).
  int kq_issued[2] = {0, 0}, kq_waited[2] = {0, 0}, v_issued = 0, v_waited = 0;
  auto issue_kq = [&](int chunk, int stage) {
    if (tid == 0) {
      uint64_t* bar = &bars->kq[stage];
      uint8_t* dst = sm + stage * kKQBytes;
      mbar_arrive_expect_tx(bar, kKQBytes);
      const int t0 = chunk * kC;
      tma_load_4d(dst, &tm_k, 0, h, t0, b, bar);
      tma_load_4d(dst + kTile, &tm_q, 0, h, t0, b, bar);
      tma_load_4d(dst + 2 * kTile, &tm_k, 64, h, t0, b, bar);
      tma_load_4d(dst + 3 * kTile, &tm_q, 64, h, t0, b, bar);
    }
    ++kq_issued[stage];
  };
  auto issue_v = [&](int chunk) {
    if (tid == 0) {
      mbar_arrive_expect_tx(&bars->v, 2 * kTile);
      tma_load_4d(sm + kOffV, &tm_v, 0, h, chunk * kC, b, &bars->v);
      tma_load_4d(sm + kOffV + kTile, &tm_v, 64, h, chunk * kC, b, &bars->v);
    }
    ++v_issued;
  };
  if (n_chunks > 0) {
    issue_kq(0, 0);
    issue_v(0);
  }
  if (n_chunks > 1) issue_kq(1, 1);
  __syncwarp();  // tcgen05.ld / st below are warp-collective

  // Initial state -> TMEM (S^T, lane = dv column l = tid) and the split S^T operand tiles.
  uint8_t* st_hi = sm + kOffS;
  uint8_t* st_lo = sm + kOffS + 32768;
  const int64_t state_base = (int64_t(b) * H + h) * kD * kD;
#pragma unroll 1
  for (int q4 = 0; q4 < 4; ++q4) {
    float sv[32];
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      sv[j] = p.s_in != nullptr ? p.s_in[state_base + int64_t(32 * q4 + j) * kD + tid] : 0.0f;
    }
    tmem_st32(lane_base + kColS + 32 * q4, sv);
    store_split32(st_hi + (q4 >> 1) * 16384, st_lo + (q4 >> 1) * 16384, tid, (q4 & 1) * 4, sv);
  }
  tmem_wait_st();
  fence_proxy_async_smem();
  tc_fence_before();
  __syncthreads();

  uint32_t mma_phase = 0;
  bool aborted = false;
  // Waits on `bar` in every thread; true (in every thread) if any thread gave up.
  auto wait_all = [&](uint64_t* bar, uint32_t parity) {
    const bool ok = wait_bar(bar, parity);
    return __syncthreads_or(!ok) != 0;
  };
  auto mma_done = [&]() {
    const bool bad = wait_all(&bars->mma, mma_phase);
    mma_phase ^= 1u;
    if (!bad) tc_fence_after();
    return bad;
  };

#pragma unroll 1
  for (int c = 0; c < n_chunks; ++c) {
    const int st = c & 1;
    uint8_t* kq = sm + st * kKQBytes;
    const uint32_t kq_a = sa + st * kKQBytes;
    const int64_t t0 = int64_t(c) * kC;

    if (wait_all(&bars->kq[st], kq_waited[st] & 1)) { aborted = true; break; }
    ++kq_waited[st];
    if (wait_all(&bars->v, v_waited & 1)) { aborted = true; break; }
    ++v_waited;

    // ---- G = [K; Q] K^T  (M = 128 rows: 64 keys then 64 queries; N = 64 keys; K = d)
    if (tid == 0) {
      tc_fence_after();
#pragma unroll
      for (int kk = 0; kk < 8; ++kk) {
        const uint32_t off = kq_a + (kk >> 2) * 2 * kTile + (kk & 3) * 32;
        umma_bf16(tmem + kColG, smem_desc_sw128(off, 16, 1024), smem_desc_sw128(off, 16, 1024), kIdescN64, kk > 0);
      }
      umma_commit(&bars->mma);
    }

    // ---- per-token scalars: g, beta, norms
    if (tid < kC) {
      float gv = 0.0f, bv = 0.0f;
      if (t0 + tid < T) {
        const int64_t gi = (int64_t(b) * T + t0 + tid) * H + h;
        gv = load_as_float(p.g, p.g_dtype, gi);
        bv = load_as_float(p.beta, p.beta_dtype, gi);
      }
      s_graw[tid] = gv;
      s_beta[tid] = bv;
      s_dk[tid] = p.l2norm ? 1.0f / sqrtf(row_sumsq(kq, kq + 2 * kTile, tid) + 1e-6f) : 1.0f;
    } else {
      const int r = tid - kC;
      s_dq[r] = p.l2norm ? 1.0f / sqrtf(row_sumsq(kq + kTile, kq + 3 * kTile, r) + 1e-6f) : 1.0f;
    }
    __syncthreads();
    if (tid == 0) {  // in-chunk cumulative decay, sequential like the reference's cumsum
      float acc = 0.0f;
#pragma unroll 8
      for (int t = 0; t < kC; ++t) {
        acc += s_graw[t];
        s_gc[t] = acc;
      }
    }
    __syncthreads();
    if (tid < kC) {
      const float gt = s_gc[tid];
      s_sfac[tid] = s_dk[tid] * expf(s_gc[kC - 1] - gt);
      s_cq[tid] = p.scale * s_dq[tid] * expf(gt);
      s_rfac[tid] = s_beta[tid] * expf(gt) * s_dk[tid];
    }
    if (mma_done()) { aborted = true; break; }

    // ---- rows of N (threads 0..63) and P (threads 64..127) from the Gram lanes
    {
      float g0[32], g1[32];
      tmem_ld32(lane_base + kColG, g0);
      tmem_ld32(lane_base + kColG + 32, g1);
      if (tid < kC) {
        const int i = tid;
        const float fi = -s_beta[i] * s_dk[i];
        const float gci = s_gc[i];
        float* nrow = s_N + i * kXStride;
#pragma unroll
        for (int j = 0; j < kC; ++j) {
          const float gij = j < 32 ? g0[j] : g1[j - 32];
          nrow[j] = j < i ? fi * s_dk[j] * gij * expf(gci - s_gc[j]) : 0.0f;
        }
      } else {
        const int i = tid - kC;
        const float fi = p.scale * s_dq[i];
        const float gci = s_gc[i];
#pragma unroll
        for (int c8 = 0; c8 < 8; ++c8) {
          float pv[8];
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            const int j = 8 * c8 + e;
            const float gij = j < 32 ? g0[j] : g1[j - 32];
            pv[e] = j <= i ? fi * s_dk[j] * gij * expf(gci - s_gc[j]) : 0.0f;
          }
          store_split8(sm + kOffP, sm + kOffP + kTile, swz(i, c8), pv);
        }
      }
    }
    tc_fence_before();
    __syncthreads();

    // ---- X = (I - N)^-1: 16x16 diagonal blocks by forward substitution ...
    if (tid < kC) {
      const int o = 16 * (tid >> 4), jj = tid & 15;
      float x[16];
#pragma unroll
      for (int m = 0; m < 16; ++m) x[m] = m == jj ? 1.0f : 0.0f;
#pragma unroll
      for (int ii = 1; ii < 16; ++ii) {
        float acc = 0.0f;
#pragma unroll
        for (int m = 0; m < ii; ++m) acc = fmaf(s_N[(o + ii) * kXStride + o + m], x[m], acc);
        if (ii > jj) x[ii] = acc;
      }
#pragma unroll
      for (int ii = 0; ii < 16; ++ii) s_X[(o + ii) * kXStride + o + jj] = x[ii];
    }
    __syncthreads();
    // ... then the blocks below the diagonal, nearest first: X_IJ = X_II sum_{M=J}^{I-1} N_IM X_MJ.
#pragma unroll 1
    for (int dist = 1; dist <= 3; ++dist) {
      const int n_el = (4 - dist) * 256;
      for (int e = tid; e < n_el; e += kThreads) {
        const int J = e >> 8, I = J + dist, ii = (e >> 4) & 15, jj = e & 15;
        float acc = 0.0f;
        for (int M = J; M < I; ++M) {
#pragma unroll
          for (int m = 0; m < 16; ++m) {
            acc = fmaf(s_N[(16 * I + ii) * kXStride + 16 * M + m], s_X[(16 * M + m) * kXStride + 16 * J + jj], acc);
          }
        }
        s_T[(J * 16 + ii) * kTStride + jj] = acc;
      }
      __syncthreads();
      for (int e = tid; e < n_el; e += kThreads) {
        const int J = e >> 8, I = J + dist, ii = (e >> 4) & 15, jj = e & 15;
        float acc = 0.0f;
        for (int m = 0; m <= ii; ++m) {
          acc = fmaf(s_X[(16 * I + ii) * kXStride + 16 * I + m], s_T[(J * 16 + m) * kTStride + jj], acc);
        }
        s_X[(16 * I + ii) * kXStride + 16 * J + jj] = acc;
      }
      __syncthreads();
    }

    // ---- Ar = X diag(beta e^gc dk), Ab = X diag(beta): split K-major tiles [t][m] (over N)
    {
      const int t = tid >> 1, half = tid & 1;
#pragma unroll
      for (int cc = 0; cc < 4; ++cc) {
        const int c8 = 4 * half + cc;
        float ar[8], ab[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const int m = 8 * c8 + e;
          const float xv = m > t ? 0.0f : (m == t ? 1.0f : s_X[t * kXStride + m]);
          ar[e] = xv * s_rfac[m];
          ab[e] = xv * s_beta[m];
        }
        store_split8(sm + kOffW, sm + kOffW + kTile, swz(t, c8), ar);
        store_split8(sm + kOffW + 2 * kTile, sm + kOffW + 3 * kTile, swz(t, c8), ab);
      }
    }
    fence_proxy_async_smem();
    __syncthreads();

    // ---- W^T = K^T Ar^T (lanes = dk), U^T = V^T Ab^T (lanes = dv)
    if (tid == 0) {
      tc_fence_after();
#pragma unroll
      for (int part = 0; part < 2; ++part) {
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
          const uint64_t a_k = smem_desc_sw128(kq_a + kk * 2048, 2 * kTile, 1024);
          const uint64_t b_r = smem_desc_sw128(sa + kOffW + part * kTile + kk * 32, 16, 1024);
          umma_bf16(tmem + kColG, a_k, b_r, kIdescN64AMn, part | kk);
          const uint64_t a_v = smem_desc_sw128(sa + kOffV + kk * 2048, kTile, 1024);
          const uint64_t b_b = smem_desc_sw128(sa + kOffW + (2 + part) * kTile + kk * 32, 16, 1024);
          umma_bf16(tmem + kColU, a_v, b_b, kIdescN64AMn, part | kk);
        }
      }
      umma_commit(&bars->mma);
    }
    if (mma_done()) { aborted = true; break; }
    if (c + 1 < n_chunks) issue_v(c + 1);
    __syncwarp();

    // ---- W tiles: MN-major [d][t] (row d = this thread's lane)
    {
      float w0[32], w1[32];
      tmem_ld32(lane_base + kColG, w0);
      tmem_ld32(lane_base + kColG + 32, w1);
      store_split32(sm + kOffW, sm + kOffW + 16384, tid, 0, w0);
      store_split32(sm + kOffW, sm + kOffW + 16384, tid, 4, w1);
    }
    fence_proxy_async_smem();
    tc_fence_before();
    __syncthreads();

    // ---- (WS)^T = S^T W^T (3 products), (QS)^T = S^T Q^T (2 products)
    if (tid == 0) {
      tc_fence_after();
      const uint32_t sh = sa + kOffS, sl = sa + kOffS + 32768;
#pragma unroll
      for (int kk = 0; kk < 8; ++kk) {
        const uint32_t aoff = (kk >> 2) * 16384 + (kk & 3) * 32;
        const uint64_t a_hi = smem_desc_sw128(sh + aoff, 16, 1024);
        const uint64_t a_lo = smem_desc_sw128(sl + aoff, 16, 1024);
        const uint64_t b_whi = smem_desc_sw128(sa + kOffW + kk * 2048, 16384, 1024);
        const uint64_t b_wlo = smem_desc_sw128(sa + kOffW + 16384 + kk * 2048, 16384, 1024);
        const uint64_t b_q = smem_desc_sw128(kq_a + kTile + (kk >> 2) * 2 * kTile + (kk & 3) * 32, 16, 1024);
        umma_bf16(tmem + kColWS, a_hi, b_whi, kIdescN64BMn, kk > 0);
        umma_bf16(tmem + kColWS, a_lo, b_whi, kIdescN64BMn, true);
        umma_bf16(tmem + kColWS, a_hi, b_wlo, kIdescN64BMn, true);
        umma_bf16(tmem + kColQS, a_hi, b_q, kIdescN64, kk > 0);
        umma_bf16(tmem + kColQS, a_lo, b_q, kIdescN64, true);
      }
      umma_commit(&bars->mma);
    }
    if (mma_done()) { aborted = true; break; }

    // ---- Vn^T = U^T - (WS)^T; Vs^T = Vn^T diag(sfac): split K-major tiles [l][t] over S^T's tiles
    {
      uint8_t* vn_hi = sm + kOffS;
      uint8_t* vn_lo = sm + kOffS + 16384;
      uint8_t* vs_hi = sm + kOffS + 32768;
      uint8_t* vs_lo = sm + kOffS + 49152;
#pragma unroll 1
      for (int half = 0; half < 2; ++half) {
        float ws[32], u[32];
        tmem_ld32(lane_base + kColWS + 32 * half, ws);
        tmem_ld32(lane_base + kColU + 32 * half, u);
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          ws[j] = u[j] - ws[j];                   // v_new
          u[j] = ws[j] * s_sfac[32 * half + j];  // v_new scaled for the state update
        }
        store_split32(vn_hi, vn_lo, tid, 4 * half, ws);
        store_split32(vs_hi, vs_lo, tid, 4 * half, u);
      }
    }
    fence_proxy_async_smem();
    tc_fence_before();
    __syncthreads();

    // ---- Vn^T P^T (3 products) and dS^T = Vs^T K (2 products)
    if (tid == 0) {
      tc_fence_after();
      const uint32_t vnh = sa + kOffS, vnl = vnh + 16384, vsh = vnh + 32768, vsl = vnh + 49152;
      const uint32_t ph = sa + kOffP, pl = ph + kTile;
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
        const uint64_t a_nh = smem_desc_sw128(vnh + kk * 32, 16, 1024);
        const uint64_t a_nl = smem_desc_sw128(vnl + kk * 32, 16, 1024);
        const uint64_t b_ph = smem_desc_sw128(ph + kk * 32, 16, 1024);
        const uint64_t b_pl = smem_desc_sw128(pl + kk * 32, 16, 1024);
        umma_bf16(tmem + kColG, a_nh, b_ph, kIdescN64, kk > 0);
        umma_bf16(tmem + kColG, a_nh, b_pl, kIdescN64, true);
        umma_bf16(tmem + kColG, a_nl, b_ph, kIdescN64, true);
        const uint64_t a_sh = smem_desc_sw128(vsh + kk * 32, 16, 1024);
        const uint64_t a_sl = smem_desc_sw128(vsl + kk * 32, 16, 1024);
        const uint64_t b_k = smem_desc_sw128(kq_a + kk * 2048, 2 * kTile, 1024);
        umma_bf16(tmem + kColDS, a_sh, b_k, kIdescN128BMn, kk > 0);
        umma_bf16(tmem + kColDS, a_sl, b_k, kIdescN128BMn, true);
      }
      umma_commit(&bars->mma);
    }
    if (mma_done()) { aborted = true; break; }
    if (c + 2 < n_chunks) issue_kq(c + 2, st);
    __syncwarp();

    // ---- outputs: o[t][l] = cq_t (QS)^T[l][t] + (Vn^T P^T)[l][t]
    {
#pragma unroll 1
      for (int half = 0; half < 2; ++half) {
        float qs[32], pv[32];
        tmem_ld32(lane_base + kColQS + 32 * half, qs);
        tmem_ld32(lane_base + kColG + 32 * half, pv);
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          const int t = 32 * half + j;
          if (t0 + t < T) {
            p.out[((int64_t(b) * T + t0 + t) * H + h) * kD + tid] = __float2bfloat16_rn(fmaf(s_cq[t], qs[j], pv[j]));
          }
        }
      }
    }
    // ---- state: S^T <- e^{gc_last} S^T + dS^T, and the split operand for the next chunk
    {
      const float gamma = expf(s_gc[kC - 1]);
      const bool last = c + 1 == n_chunks;
#pragma unroll 1
      for (int q4 = 0; q4 < 4; ++q4) {
        float sv[32], ds[32];
        tmem_ld32(lane_base + kColS + 32 * q4, sv);
        tmem_ld32(lane_base + kColDS + 32 * q4, ds);
#pragma unroll
        for (int j = 0; j < 32; ++j) sv[j] = fmaf(gamma, sv[j], ds[j]);
        tmem_st32(lane_base + kColS + 32 * q4, sv);
        if (!last) store_split32(st_hi + (q4 >> 1) * 16384, st_lo + (q4 >> 1) * 16384, tid, (q4 & 1) * 4, sv);
      }
      tmem_wait_st();
    }
    fence_proxy_async_smem();
    tc_fence_before();
    __syncthreads();
  }

  if (aborted) {
    if (tid == 0) report(p.status, OQ_DEV_TIMEOUT);
    // Let every issued MMA and copy land before TMEM and shared memory go away.
    if (tid == 0) umma_commit(&bars->drain);
    wait_bar(&bars->drain, 0);
    for (int s = 0; s < 2; ++s) {
      while (kq_waited[s] < kq_issued[s]) wait_bar(&bars->kq[s], (kq_waited[s]++) & 1);
    }
    while (v_waited < v_issued) wait_bar(&bars->v, (v_waited++) & 1);
  } else if (p.s_out != nullptr) {
    tc_fence_after();
#pragma unroll 1
    for (int q4 = 0; q4 < 4; ++q4) {
      float sv[32];
      tmem_ld32(lane_base + kColS + 32 * q4, sv);
#pragma unroll
      for (int j = 0; j < 32; ++j) p.s_out[state_base + int64_t(32 * q4 + j) * kD + tid] = sv[j];
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, kTmemCols);
}

// 4-D map over a [B, T, H, 128] bf16 tensor: box = 64 head-dim elements x 1 head x 64 tokens x 1 sequence.
int encode_qkv_map(CUtensorMap* map, const void* base, int64_t B, int64_t T, int64_t H, int64_t sb, int64_t st,
                   int64_t sh) {
  auto fn = tensor_map_encoder();
  if (fn == nullptr) return fail(OQ_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
  const cuuint64_t dims[4] = {cuuint64_t(kD), cuuint64_t(H), cuuint64_t(T), cuuint64_t(B)};
  const cuuint64_t strides[3] = {cuuint64_t(sh * 2), cuuint64_t(st * 2), cuuint64_t(sb * 2)};
  const cuuint32_t box[4] = {64, 1, cuuint32_t(kC), 1};
  const cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult res = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(base), dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (res != CUDA_SUCCESS) return fail(OQ_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", int(res));
  return OQ_OK;
}

bool stride_ok(int64_t s) { return s > 0 && (s * 2) % 16 == 0 && s * 2 < (int64_t(1) << 40); }

}  // namespace
}  // namespace oq

extern "C" int oq_gdn_chunk_fwd(
    const void* q, const void* k, const void* v, int qkv_dtype,
    int64_t q_stride_b, int64_t q_stride_t, int64_t q_stride_h,
    int64_t k_stride_b, int64_t k_stride_t, int64_t k_stride_h,
    int64_t v_stride_b, int64_t v_stride_t, int64_t v_stride_h,
    const void* g, int g_dtype, const void* beta, int beta_dtype,
    const float* initial_state, float* final_state, void* out,
    int64_t batch, int64_t seq_len, int64_t num_heads, int64_t k_dim, int64_t v_dim,
    float scale, int use_qk_l2norm, int64_t chunk_size, int32_t* device_status, void* stream) {
  using namespace oq;
  if (qkv_dtype != OQ_BF16) return fail(OQ_ERR_UNSUPPORTED, "gdn_chunk_fwd: q, k, v must be bf16");
  if (!valid_dtype(g_dtype) || !valid_dtype(beta_dtype)) return fail(OQ_ERR_UNSUPPORTED, "gdn_chunk_fwd: unknown dtype");
  if (k_dim != kD || v_dim != kD) return fail(OQ_ERR_UNSUPPORTED, "gdn_chunk_fwd: k_dim = v_dim = 128 required");
  if (chunk_size != kC) return fail(OQ_ERR_UNSUPPORTED, "gdn_chunk_fwd: chunk_size must be 64");
  if (batch < 0 || seq_len < 0 || num_heads <= 0) return fail(OQ_ERR_INVALID_ARGUMENT, "gdn_chunk_fwd: bad sizes");
  if (batch == 0) return ok();
  if (batch > 65535 || num_heads > 65535 || seq_len > (int64_t(1) << 31) - kC) {
    return fail(OQ_ERR_UNSUPPORTED, "gdn_chunk_fwd: sizes too large");
  }
  if (seq_len > 0 && (!g || !beta || !q || !k || !v || !out)) {
    return fail(OQ_ERR_INVALID_ARGUMENT, "gdn_chunk_fwd: null pointer");
  }
  if (seq_len > 0) {
    const int64_t strides[9] = {q_stride_b, q_stride_t, q_stride_h, k_stride_b, k_stride_t,
                                k_stride_h, v_stride_b, v_stride_t, v_stride_h};
    for (int64_t s : strides) {
      if (!stride_ok(s)) return fail(OQ_ERR_MISALIGNED, "gdn_chunk_fwd: strides must be positive multiples of 16 bytes");
    }
    for (const void* ptr : {q, k, v, static_cast<const void*>(out)}) {
      if (reinterpret_cast<uintptr_t>(ptr) % 16) return fail(OQ_ERR_MISALIGNED, "gdn_chunk_fwd: q/k/v/out must be 16-byte aligned");
    }
  }
  CUtensorMap maps[3];
  if (seq_len > 0) {
    int st = encode_qkv_map(&maps[0], q, batch, seq_len, num_heads, q_stride_b, q_stride_t, q_stride_h);
    if (st == OQ_OK) st = encode_qkv_map(&maps[1], k, batch, seq_len, num_heads, k_stride_b, k_stride_t, k_stride_h);
    if (st == OQ_OK) st = encode_qkv_map(&maps[2], v, batch, seq_len, num_heads, v_stride_b, v_stride_t, v_stride_h);
    if (st != OQ_OK) return st;
  } else {
    memset(maps, 0, sizeof(maps));
  }
  static bool attr_set[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !attr_set[dev]) {
    if (cudaFuncSetAttribute(gdn_chunk_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(kSmemBytes)) !=
        cudaSuccess) {
      return check_launch("gdn_chunk_fwd: shared memory attribute");
    }
    attr_set[dev] = true;
  }
  ChunkParams p;
  p.g = g;
  p.beta = beta;
  p.g_dtype = g_dtype;
  p.beta_dtype = beta_dtype;
  p.s_in = initial_state;
  p.s_out = final_state;
  p.out = static_cast<__nv_bfloat16*>(out);
  p.seq_len = seq_len;
  p.num_heads = int(num_heads);
  p.scale = scale;
  p.l2norm = use_qk_l2norm;
  p.status = device_status;
  dim3 grid((unsigned)num_heads, (unsigned)batch);
  gdn_chunk_kernel<<<grid, kThreads, kSmemBytes, static_cast<cudaStream_t>(stream)>>>(maps[0], maps[1], maps[2], p);
  return check_launch("gdn_chunk_fwd");
}
