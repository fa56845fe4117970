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
constexpr int kThreads = 256;   // two threads per TMEM lane (warps w and w + 4), splitting the columns
constexpr uint32_t kTmemCols = 512;

// TMEM columns (fp32 accumulators, lane = dv row unless noted)
// Products of a raw operand with a split (hi | lo) one are one N = 128 MMA over the two split
// tiles, which lie next to each other as K-major tiles; the two 64-column halves of the
// accumulator are added when read.
constexpr uint32_t kColG = 0;     // [K;Q]K^T (lane = token)
constexpr uint32_t kColW = 0;     // W^T (lane = dk), 128 columns: the Ar hi | Ar lo halves (after G is read)
constexpr uint32_t kColQS = 64;   // (Q S)^T (after W is read; the next chunk's G takes columns 0-63 only)
constexpr uint32_t kColWS = 128;  // (W S)^T, 128 columns: S_hi W_hi + S_lo W_hi | S_hi W_lo
constexpr uint32_t kColU = 256;   // U^T, 128 columns: the Ab hi | Ab lo halves
constexpr uint32_t kColPV = 256;  // Vn^T P^T, 128 columns: Vn_hi P_hi + Vn_lo P_hi | Vn_hi P_lo (after U is read)
constexpr uint32_t kColS = 384;   // S^T, 128 columns: the state (dS^T accumulates onto e^{gc_last} S^T)

// Shared memory (byte offsets from a 1024-aligned base).  A "tile" is 64 rows x 128 B.
constexpr uint32_t kTile = 8192;
constexpr uint32_t kKQBytes = 4 * kTile;           // one input stage: K d<64 | Q d<64 | K d>=64 | Q d>=64
constexpr uint32_t kOffV = 2 * kKQBytes;           // V d<64 | V d>=64
constexpr uint32_t kOffS = kOffV + 2 * kTile;      // S^T hi (2 x 16 KB) | S^T lo; later Vn hi|Vn lo|Vs hi|Vs lo
constexpr uint32_t kOffW = kOffS + 65536;          // W hi | W lo (16 KB each); before that N, then Ar/Ab tiles
constexpr uint32_t kOffX = kOffW + 32768;          // X fp32 [64][68]
constexpr uint32_t kOffP = kOffX + 17408;          // P hi | P lo
constexpr uint32_t kOffSmall = kOffP + 2 * kTile;
constexpr int kNStride = 65;                       // N rows (written one row per thread)
constexpr int kXStride = 68;                       // X rows (read as float4)
constexpr uint32_t kOffTmp = kOffW + 16896;        // solve scratch after N: [2][16][20] then [32][36]
constexpr int kT2Stride = 20;
constexpr int kT3Stride = 36;
// small area: two buffers (this chunk, next chunk) of 9 per-token float arrays, barriers
constexpr int kTokArrays = 9;
constexpr uint32_t kSmallFloats = 2 * kTokArrays * kC;
constexpr uint32_t kOffBars = kOffSmall + kSmallFloats * 4;
constexpr uint32_t kSmemBytes = kOffBars + 64 + 1024;  // + alignment slack

constexpr uint32_t kWaitHintNs = 20000;

constexpr uint32_t kIdescN64 = idesc_bf16_f32(128, 64, false, false);
constexpr uint32_t kIdescN64BMn = idesc_bf16_f32(128, 64, false, true);
constexpr uint32_t kIdescN128BMn = idesc_bf16_f32(128, 128, false, true);
constexpr uint32_t kIdescN128AMn = idesc_bf16_f32(128, 128, true, false);
constexpr uint32_t kIdescN128 = idesc_bf16_f32(128, 128, false, false);

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
  int wait_polls;  // polls of a bounded wait on a copy or an MMA (wait_polls() at launch)
};

struct Bars {
  uint64_t kq[2];
  uint64_t v;
  uint64_t mma;
  uint64_t drain;
  uint64_t ab;  // two-phase form: a chunk's Ar / Ab tiles and scalars
  uint64_t pp;  // two-phase form: its P tiles
  uint32_t tmem_base;
};

// Workspace image of one (sequence, head, chunk) in the two-phase form (see below).
constexpr uint32_t kImgP = 4 * kTile;                   // P hi | P lo after the Ar / Ab tiles
constexpr uint32_t kImgScal = 6 * kTile;                // sfac[64], cq[64], gamma, padding
constexpr uint32_t kImgScalBytes = 160 * 4;
constexpr uint32_t kImgBytes = 6 * kTile + 1024;        // per (sequence, head, chunk)

// Bounded wait (sleeping in try_wait up to 20 us per poll); false if `polls` polls pass.  Waits
// that drain copies and MMAs before a CTA exits use kDefaultWaitPolls (~2 s).
__device__ __forceinline__ bool wait_bar(uint64_t* bar, uint32_t parity, int polls) {
  for (int i = 0; i < polls; ++i) {
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
  float ss[4] = {0.0f, 0.0f, 0.0f, 0.0f};
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
        ss[i] = fmaf(f.x, f.x, ss[i]);
        ss[i] = fmaf(f.y, f.y, ss[i]);
      }
    }
  }
  return (ss[0] + ss[1]) + (ss[2] + ss[3]);
}

// kPre: the two-phase form's second phase, reading the state-independent per-chunk tiles
// from `images` (written by gdn_chunk_prep_kernel) instead of computing them.
template <bool kPre>
__global__ void __launch_bounds__(kThreads, 1)
    gdn_chunk_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                     const __grid_constant__ CUtensorMap tm_v, ChunkParams p, const uint8_t* images) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sa = smem_addr(sm);
  // per-token arrays of chunk c live in buffer c & 1:
  // 0 g, 1 gc (in-chunk cumulative g), 2 beta, 3 dk, 4 dq (inverse L2 norms), 5 sfac = dk e^{gc_last - gc},
  // 6 cq = scale dq e^{gc}, 7 rfac = beta e^{gc} dk, 8 gcl = gc log2(e)
  float* f_small = reinterpret_cast<float*>(sm + kOffSmall);
  auto tok = [&](int buf, int k) { return f_small + (buf * kTokArrays + k) * kC; };
  float* s_T = reinterpret_cast<float*>(sm + kOffTmp);
  float* s_N = reinterpret_cast<float*>(sm + kOffW);
  float* s_X = reinterpret_cast<float*>(sm + kOffX);
  Bars* bars = reinterpret_cast<Bars*>(sm + kOffBars);

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 127;  // TMEM lane served by this thread
  const int half = tid >> 7;   // which half of the columns it takes
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
    mbar_init(&bars->ab, 1);
    mbar_init(&bars->pp, 1);
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
  const uint32_t lane_base = tmem + (uint32_t((warp & 3) * 32) << 16);
  pdl_wait();  // (one long wave: the successor is allowed to launch only after the chunk loop)

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
  int ab_issued = 0, ab_waited = 0, p_issued = 0, p_waited = 0;
  auto img_of = [&](int cc) {
    return images + ((int64_t(b) * H + h) * n_chunks + cc) * int64_t(kImgBytes);
  };
  // (thread 0; the regions it refills were last touched by the generic proxy or the MMAs,
  // both finished at the block barrier before each call)
  auto issue_ab = [&](int cc) {
    if (tid == 0) {
      fence_proxy_async_smem();
      mbar_arrive_expect_tx(&bars->ab, 4 * kTile + kImgScalBytes);
      bulk_load(sm + kOffW, img_of(cc), 4 * kTile, &bars->ab);
      bulk_load(tok(cc & 1, 5), img_of(cc) + kImgScal, kImgScalBytes, &bars->ab);
    }
    ++ab_issued;
  };
  auto issue_p = [&](int cc) {
    if (tid == 0) {
      fence_proxy_async_smem();
      mbar_arrive_expect_tx(&bars->pp, 2 * kTile);
      bulk_load(sm + kOffP, img_of(cc) + kImgP, 2 * kTile, &bars->pp);
    }
    ++p_issued;
  };
  if (n_chunks > 0) {
    issue_kq(0, 0);
    issue_v(0);
    if constexpr (kPre) {
      issue_ab(0);
      issue_p(0);
    }
  }
  if (n_chunks > 1) issue_kq(1, 1);
  __syncwarp();  // tcgen05.ld / st below are warp-collective

  // Initial state -> TMEM (S^T, lane = dv column l) and the split S^T operand tiles.
  uint8_t* st_hi = sm + kOffS;
  uint8_t* st_lo = sm + kOffS + 32768;
  const int64_t state_base = (int64_t(b) * H + h) * kD * kD;
#pragma unroll 1
  for (int q4 = 2 * half; q4 < 2 * half + 2; ++q4) {
    float sv[32];
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      sv[j] = p.s_in != nullptr ? p.s_in[state_base + int64_t(32 * q4 + j) * kD + lane] : 0.0f;
    }
    tmem_st32(lane_base + kColS + 32 * q4, sv);
    store_split32(st_hi + (q4 >> 1) * 16384, st_lo + (q4 >> 1) * 16384, lane, (q4 & 1) * 4, sv);
  }
  tmem_wait_st();
  fence_proxy_async_smem();
  tc_fence_before();
  __syncthreads();

  uint32_t mma_phase = 0;
  bool aborted = false;
  // Waits on `bar` in every thread; true (in every thread) if any thread gave up.
  auto wait_all = [&](uint64_t* bar, uint32_t parity) {
    const bool ok = wait_bar(bar, parity, p.wait_polls);
    return __syncthreads_or(!ok) != 0;
  };
  auto mma_done = [&]() {
    const bool bad = wait_all(&bars->mma, mma_phase);
    mma_phase ^= 1u;
    if (!bad) tc_fence_after();
    return bad;
  };
  // G = [K; Q] K^T of chunk cc (M = 128 rows: 64 keys then 64 queries; N = 64 keys; K = d); thread 0.
  auto issue_gram = [&](int cc) {
    const uint32_t kq_a = sa + (cc & 1) * kKQBytes;
    tc_fence_after();
#pragma unroll
    for (int kk = 0; kk < 8; ++kk) {
      const uint32_t off = kq_a + (kk >> 2) * 2 * kTile + (kk & 3) * 32;
      umma_bf16(tmem + kColG, smem_desc_sw128(off, 16, 1024), smem_desc_sw128(off, 16, 1024), kIdescN64, kk > 0);
    }
  };
  // Per-token scalars of chunk cc (its inputs have landed): g, beta, norms, then the in-chunk
  // cumulative decay (warp scan, two tokens per lane) and the derived factors.  Ends without a
  // barrier after the scan; callers synchronise before reading.
  // g and beta of token `t` of chunk cc (zero past the end), loaded ahead of use.
  auto load_gb = [&](int cc, float& gv, float& bv) {
    gv = 0.0f;
    bv = 0.0f;
    const int64_t t = int64_t(cc) * kC + tid;
    if (tid < kC && t < T) {
      const int64_t gi = (int64_t(b) * T + t) * H + h;
      gv = load_as_float(p.g, p.g_dtype, gi);
      bv = load_as_float(p.beta, p.beta_dtype, gi);
    }
  };
  auto prep_scalars = [&](int cc, float gv, float bv) {
    const uint8_t* kqc = sm + (cc & 1) * kKQBytes;
    const int buf = cc & 1;
    if (tid < kC) {
      tok(buf, 0)[tid] = gv;
      tok(buf, 2)[tid] = bv;
      tok(buf, 3)[tid] = p.l2norm ? 1.0f / sqrtf(row_sumsq(kqc, kqc + 2 * kTile, tid) + 1e-6f) : 1.0f;
    } else if (tid < 2 * kC) {
      const int r = tid - kC;
      tok(buf, 4)[r] = p.l2norm ? 1.0f / sqrtf(row_sumsq(kqc + kTile, kqc + 3 * kTile, r) + 1e-6f) : 1.0f;
    }
    __syncthreads();
    if (warp == 0) {
      const float a0 = tok(buf, 0)[2 * tid], a1 = tok(buf, 0)[2 * tid + 1];
      float incl = a0 + a1;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const float y = __shfl_up_sync(0xffffffffu, incl, o);
        if (tid >= o) incl += y;
      }
      float excl = __shfl_up_sync(0xffffffffu, incl, 1);
      if (tid == 0) excl = 0.0f;
      const float gc[2] = {excl + a0, (excl + a0) + a1};
      const float gl = __shfl_sync(0xffffffffu, gc[1], 31);
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int t = 2 * tid + e;
        const float dk = tok(buf, 3)[t];
        tok(buf, 1)[t] = gc[e];
        tok(buf, 8)[t] = gc[e] * 1.4426950408889634f;
        tok(buf, 5)[t] = dk * expf(gl - gc[e]);
        tok(buf, 6)[t] = p.scale * tok(buf, 4)[t] * expf(gc[e]);
        tok(buf, 7)[t] = tok(buf, 2)[t] * expf(gc[e]) * dk;
      }
    }
  };

  if (!kPre && n_chunks > 0) {
    if (wait_all(&bars->kq[0], 0)) {
      aborted = true;
    } else {
      ++kq_waited[0];
      if (tid == 0) {
        issue_gram(0);
        umma_commit(&bars->mma);
      }
      float gv, bv;
      load_gb(0, gv, bv);
      prep_scalars(0, gv, bv);
      aborted = mma_done();
    }
  }

#pragma unroll 1
  for (int c = 0; c < n_chunks && !aborted; ++c) {
    const int st = c & 1;
    const uint32_t kq_a = sa + st * kKQBytes;
    const int64_t t0 = int64_t(c) * kC;
    const float* s_gc = tok(st, 1);
    const float* s_beta = tok(st, 2);
    const float* s_dk = tok(st, 3);
    const float* s_dq = tok(st, 4);
    const float* s_sfac = tok(st, 5);
    const float* s_cq = tok(st, 6);
    const float* s_rfac = tok(st, 7);
    const float* s_gcl = tok(st, 8);
    const bool last = c + 1 == n_chunks;
    float g_next = 0.0f, b_next = 0.0f;
    if constexpr (kPre) {
      // this chunk's K / Q tiles, and its Ar / Ab tiles and scalars from the first phase
      if (wait_all(&bars->kq[st], kq_waited[st] & 1)) { aborted = true; break; }
      ++kq_waited[st];
      if (wait_all(&bars->ab, ab_waited & 1)) { aborted = true; break; }
      ++ab_waited;
    } else {
    load_gb(c + 1, g_next, b_next);

    // (G of this chunk and its per-token scalars are ready.)
    // ---- rows of N (lanes 0..63) and P (lanes 64..127) from the Gram lanes; each thread
    // takes 32 of the 64 columns
    {
      float gr[32];
      tmem_ld32(lane_base + kColG + 32 * half, gr);
      const int j0 = 32 * half;
      if (lane < kC) {
        const int i = lane;
        const float fi = -s_beta[i] * s_dk[i];
        const float gli = s_gcl[i];
        float* nrow = s_N + i * kNStride + j0;
#pragma unroll
        for (int jj = 0; jj < 32; ++jj) {
          const int j = j0 + jj;
          nrow[jj] = j < i ? fi * s_dk[j] * gr[jj] * exp2f(gli - s_gcl[j]) : 0.0f;
        }
      } else {
        const int i = lane - kC;
        const float fi = p.scale * s_dq[i];
        const float gli = s_gcl[i];
#pragma unroll
        for (int cc = 0; cc < 4; ++cc) {
          float pv[8];
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            const int j = j0 + 8 * cc + e;
            pv[e] = j <= i ? fi * s_dk[j] * gr[8 * cc + e] * exp2f(gli - s_gcl[j]) : 0.0f;
          }
          store_split8(sm + kOffP, sm + kOffP + kTile, swz(i, 4 * half + cc), pv);
        }
      }
    }
    tc_fence_before();
    __syncthreads();

    // ---- X = (I - N)^-1 by doubling.  16x16 diagonal blocks by forward substitution
    // (one column per thread), zeroing the blocks right of blocks 0 and 2 ...
    if (tid < kC) {
      const int o = 16 * (tid >> 4), jj = tid & 15;
      float x[16];
#pragma unroll
      for (int m = 0; m < 16; ++m) x[m] = m == jj ? 1.0f : 0.0f;
#pragma unroll
      for (int ii = 1; ii < 16; ++ii) {
        float acc = 0.0f;
#pragma unroll
        for (int m = 0; m < ii; ++m) acc = fmaf(s_N[(o + ii) * kNStride + o + m], x[m], acc);
        if (ii > jj) x[ii] = acc;
      }
#pragma unroll
      for (int ii = 0; ii < 16; ++ii) s_X[(o + ii) * kXStride + o + jj] = x[ii];
      if ((o & 16) == 0) {
#pragma unroll
        for (int ii = 0; ii < 16; ++ii) s_X[(o + ii) * kXStride + o + 16 + jj] = 0.0f;
      }
    }
    __syncthreads();
    // ... then the 32x32 diagonal blocks: X_10 = X_11 N_10 X_00 and X_32 = X_33 N_32 X_22
    // (1x2 outputs per thread) ...
    {
      const int blk = tid >> 7, I = 16 * (1 + 2 * blk), J = 32 * blk;
      const int r = (tid & 127) >> 3, c0 = (tid & 7) * 2;
      float* tb = s_T + blk * 16 * kT2Stride;
      float a0 = 0.0f, a1 = 0.0f;
#pragma unroll
      for (int m = 0; m < 16; ++m) {
        const float n = s_N[(I + r) * kNStride + J + m];
        const float2 x = *reinterpret_cast<const float2*>(&s_X[(J + m) * kXStride + J + c0]);
        a0 = fmaf(n, x.x, a0);
        a1 = fmaf(n, x.y, a1);
      }
      *reinterpret_cast<float2*>(&tb[r * kT2Stride + c0]) = make_float2(a0, a1);
      __syncthreads();
      a0 = a1 = 0.0f;
#pragma unroll
      for (int m = 0; m < 16; ++m) {
        const float x = s_X[(I + r) * kXStride + I + m];
        const float2 t = *reinterpret_cast<const float2*>(&tb[m * kT2Stride + c0]);
        a0 = fmaf(x, t.x, a0);
        a1 = fmaf(x, t.y, a1);
      }
      *reinterpret_cast<float2*>(&s_X[(I + r) * kXStride + J + c0]) = make_float2(a0, a1);
    }
    __syncthreads();
    // ... and the lower-left 32x32 block: X[32:, :32] = X[32:, 32:] N[32:, :32] X[:32, :32]
    // Warp w computes columns 4w..4w+3 of T = N[32:, :32] X[:32, :32] (lane = row; X[m][c] = 0
    // for m < c), then rows 4w..4w+3 of X[32:, 32:] T (lane = column; X[32 + r][32 + m] = 0 for m > r).
    {
      const int c0 = 4 * warp, r = tid & 31;
      float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll 4
      for (int m = c0; m < 32; ++m) {
        const float n = s_N[(32 + r) * kNStride + m];
        const float4 x = *reinterpret_cast<const float4*>(&s_X[m * kXStride + c0]);
        acc[0] = fmaf(n, x.x, acc[0]);
        acc[1] = fmaf(n, x.y, acc[1]);
        acc[2] = fmaf(n, x.z, acc[2]);
        acc[3] = fmaf(n, x.w, acc[3]);
      }
      *reinterpret_cast<float4*>(&s_T[r * kT3Stride + c0]) = make_float4(acc[0], acc[1], acc[2], acc[3]);
      __syncthreads();
      const int r0 = 4 * warp, col = tid & 31;
      float o[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll 1
      for (int m0 = 0; m0 < r0 + 4; m0 += 4) {
        float tcol[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) tcol[i] = s_T[(m0 + i) * kT3Stride + col];
#pragma unroll
        for (int a = 0; a < 4; ++a) {
          const float4 x = *reinterpret_cast<const float4*>(&s_X[(32 + r0 + a) * kXStride + 32 + m0]);
          o[a] = fmaf(x.x, tcol[0], o[a]);
          o[a] = fmaf(x.y, tcol[1], o[a]);
          o[a] = fmaf(x.z, tcol[2], o[a]);
          o[a] = fmaf(x.w, tcol[3], o[a]);
        }
      }
#pragma unroll
      for (int a = 0; a < 4; ++a) s_X[(32 + r0 + a) * kXStride + col] = o[a];
    }
    __syncthreads();

    // ---- Ar = X diag(beta e^gc dk), Ab = X diag(beta): split K-major tiles [t][m] (over N)
    {
      const int t = tid >> 2, qq = tid & 3;
#pragma unroll
      for (int cc = 0; cc < 2; ++cc) {
        const int c8 = 2 * qq + cc;
        float xr[8], ar[8], ab[8];
        *reinterpret_cast<float4*>(xr) = *reinterpret_cast<const float4*>(&s_X[t * kXStride + 8 * c8]);
        *reinterpret_cast<float4*>(xr + 4) = *reinterpret_cast<const float4*>(&s_X[t * kXStride + 8 * c8 + 4]);
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const int m = 8 * c8 + e;
          const float xv = m > t ? 0.0f : (m == t ? 1.0f : xr[e]);
          ar[e] = xv * s_rfac[m];
          ab[e] = xv * s_beta[m];
        }
        store_split8(sm + kOffW, sm + kOffW + kTile, swz(t, c8), ar);
        store_split8(sm + kOffW + 2 * kTile, sm + kOffW + 3 * kTile, swz(t, c8), ab);
      }
    }
    fence_proxy_async_smem();
    __syncthreads();
    }  // (kPre: copied in by the first phase)

    // ---- W^T = K^T Ar^T (lanes = dk), U^T = V^T Ab^T (lanes = dv)
    if (wait_all(&bars->v, v_waited & 1)) { aborted = true; break; }
    ++v_waited;
    if (tid == 0) {
      tc_fence_after();
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {  // B = the hi and lo tiles together (N = 128)
        const uint64_t a_k = smem_desc_sw128(kq_a + kk * 2048, 2 * kTile, 1024);
        const uint64_t b_r = smem_desc_sw128(sa + kOffW + kk * 32, 16, 1024);
        umma_bf16(tmem + kColW, a_k, b_r, kIdescN128AMn, kk > 0);
        const uint64_t a_v = smem_desc_sw128(sa + kOffV + kk * 2048, kTile, 1024);
        const uint64_t b_b = smem_desc_sw128(sa + kOffW + 2 * kTile + kk * 32, 16, 1024);
        umma_bf16(tmem + kColU, a_v, b_b, kIdescN128AMn, kk > 0);
      }
      umma_commit(&bars->mma);
    }
    if (mma_done()) { aborted = true; break; }
    if (c + 1 < n_chunks) issue_v(c + 1);
    __syncwarp();

    // ---- W tiles: MN-major [d][t] (row d = this thread's lane)
    {
      float w[32], wl[32];
      tmem_ld32(lane_base + kColW + 32 * half, w);
      tmem_ld32(lane_base + kColW + 64 + 32 * half, wl);
#pragma unroll
      for (int j = 0; j < 32; ++j) w[j] += wl[j];
      store_split32(sm + kOffW, sm + kOffW + 16384, lane, 4 * half, w);
    }
    fence_proxy_async_smem();
    tc_fence_before();
    __syncthreads();

    // ---- (WS)^T = S^T W^T (3 products), (QS)^T = S^T Q^T (2 products); meanwhile the state
    // in TMEM is scaled by e^{gc_last} so that dS^T can accumulate onto it.
    if (tid == 0) {
      tc_fence_after();
      const uint32_t sh = sa + kOffS, sl = sa + kOffS + 32768;
#pragma unroll
      for (int kk = 0; kk < 8; ++kk) {
        const uint32_t aoff = (kk >> 2) * 16384 + (kk & 3) * 32;
        const uint64_t a_hi = smem_desc_sw128(sh + aoff, 16, 1024);
        const uint64_t a_lo = smem_desc_sw128(sl + aoff, 16, 1024);
        const uint64_t b_whi = smem_desc_sw128(sa + kOffW + kk * 2048, 16384, 1024);
        const uint64_t b_q = smem_desc_sw128(kq_a + kTile + (kk >> 2) * 2 * kTile + (kk & 3) * 32, 16, 1024);
        umma_bf16(tmem + kColWS, a_hi, b_whi, kIdescN128BMn, kk > 0);  // S_hi [W_hi | W_lo] (W_lo at the LBO)
        umma_bf16(tmem + kColWS, a_lo, b_whi, kIdescN64BMn, true);      // + S_lo W_hi
        umma_bf16(tmem + kColQS, a_hi, b_q, kIdescN64, kk > 0);
        umma_bf16(tmem + kColQS, a_lo, b_q, kIdescN64, true);
      }
      umma_commit(&bars->mma);
    }
    __syncwarp();
    {
      const float gamma = kPre ? tok(st, 7)[0] : expf(s_gc[kC - 1]);  // (the image holds e^{gc_last} there)
#pragma unroll 1
      for (int q4 = 2 * half; q4 < 2 * half + 2; ++q4) {
        float sv[32];
        tmem_ld32(lane_base + kColS + 32 * q4, sv);
#pragma unroll
        for (int j = 0; j < 32; ++j) sv[j] *= gamma;
        tmem_st32(lane_base + kColS + 32 * q4, sv);
      }
      tmem_wait_st();
    }
    tc_fence_before();
    if (mma_done()) { aborted = true; break; }
    if constexpr (kPre) {
      if (!last) issue_ab(c + 1);  // the W tiles are consumed: the region takes the next chunk's tiles
    }

    // ---- Vn^T = U^T - (WS)^T; Vs^T = Vn^T diag(sfac): split K-major tiles [l][t] over S^T's tiles
    {
      uint8_t* vn_hi = sm + kOffS;
      uint8_t* vn_lo = sm + kOffS + 16384;
      uint8_t* vs_hi = sm + kOffS + 32768;
      uint8_t* vs_lo = sm + kOffS + 49152;
      float ws[32], u[32];
      tmem_ld32(lane_base + kColU + 64 + 32 * half, ws);  // (the lo half of U first)
      tmem_ld32(lane_base + kColU + 32 * half, u);
#pragma unroll
      for (int j = 0; j < 32; ++j) u[j] += ws[j];
      tmem_ld32(lane_base + kColWS + 64 + 32 * half, ws);  // (the S_hi W_lo half)
#pragma unroll
      for (int j = 0; j < 32; ++j) u[j] -= ws[j];
      tmem_ld32(lane_base + kColWS + 32 * half, ws);
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        ws[j] = u[j] - ws[j];                   // v_new
        u[j] = ws[j] * s_sfac[32 * half + j];  // v_new scaled for the state update
      }
      store_split32(vn_hi, vn_lo, lane, 4 * half, ws);
      store_split32(vs_hi, vs_lo, lane, 4 * half, u);
    }
    fence_proxy_async_smem();
    tc_fence_before();
    __syncthreads();

    // ---- Vn^T P^T (3 products) and S^T += Vs^T K (2 products); then the next chunk's G, whose
    // per-token scalars are computed while the tensor cores run.
    if constexpr (kPre) {
      if (wait_all(&bars->pp, p_waited & 1)) { aborted = true; break; }
      ++p_waited;
    }
    if (tid == 0) {
      tc_fence_after();
      const uint32_t vnh = sa + kOffS, vnl = vnh + 16384, vsh = vnh + 32768, vsl = vnh + 49152;
      const uint32_t ph = sa + kOffP;  // P_hi, with P_lo the next tile
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
        const uint64_t a_nh = smem_desc_sw128(vnh + kk * 32, 16, 1024);
        const uint64_t a_nl = smem_desc_sw128(vnl + kk * 32, 16, 1024);
        const uint64_t b_ph = smem_desc_sw128(ph + kk * 32, 16, 1024);
        umma_bf16(tmem + kColPV, a_nh, b_ph, kIdescN128, kk > 0);  // Vn_hi [P_hi | P_lo]
        umma_bf16(tmem + kColPV, a_nl, b_ph, kIdescN64, true);     // + Vn_lo P_hi
        const uint64_t a_sh = smem_desc_sw128(vsh + kk * 32, 16, 1024);
        const uint64_t a_sl = smem_desc_sw128(vsl + kk * 32, 16, 1024);
        const uint64_t b_k = smem_desc_sw128(kq_a + kk * 2048, 2 * kTile, 1024);
        umma_bf16(tmem + kColS, a_sh, b_k, kIdescN128BMn, true);
        umma_bf16(tmem + kColS, a_sl, b_k, kIdescN128BMn, true);
      }
    }
    if (!kPre && !last) {
      if (wait_all(&bars->kq[st ^ 1], kq_waited[st ^ 1] & 1)) {
        if (tid == 0) umma_commit(&bars->mma);
        aborted = true;
        break;
      }
      ++kq_waited[st ^ 1];
      if (tid == 0) issue_gram(c + 1);
    }
    if (tid == 0) umma_commit(&bars->mma);
    if (!kPre && !last) prep_scalars(c + 1, g_next, b_next);
    if (mma_done()) { aborted = true; break; }
    if (c + 2 < n_chunks) issue_kq(c + 2, st);
    __syncwarp();

    // ---- outputs: o[t][l] = cq_t (QS)^T[l][t] + (Vn^T P^T)[l][t]
    // (staged as [64][128] bf16 over the consumed P tiles, then written as 16-byte row pieces)
    {
      __nv_bfloat16* ostage = reinterpret_cast<__nv_bfloat16*>(sm + kOffP);
      float qs[32], pv[32];
      tmem_ld32(lane_base + kColPV + 64 + 32 * half, qs);  // (the Vn_hi P_lo half first)
      tmem_ld32(lane_base + kColPV + 32 * half, pv);
#pragma unroll
      for (int j = 0; j < 32; ++j) pv[j] += qs[j];
      tmem_ld32(lane_base + kColQS + 32 * half, qs);
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        const int t = 32 * half + j;
        ostage[t * kD + lane] = __float2bfloat16_rn(fmaf(s_cq[t], qs[j], pv[j]));
      }
      // ---- the updated state as the split S^T operand of the next chunk
      if (!last) {
#pragma unroll 1
        for (int q4 = 2 * half; q4 < 2 * half + 2; ++q4) {
          float sv[32];
          tmem_ld32(lane_base + kColS + 32 * q4, sv);
          store_split32(st_hi + (q4 >> 1) * 16384, st_lo + (q4 >> 1) * 16384, lane, (q4 & 1) * 4, sv);
        }
      }
      __syncthreads();
#pragma unroll
      for (int e = tid; e < kC * (kD / 8); e += kThreads) {
        const int row = e >> 4, ch = e & 15;
        if (t0 + row < T) {
          *reinterpret_cast<uint4*>(p.out + ((int64_t(b) * T + t0 + row) * H + h) * kD + 8 * ch) =
              *reinterpret_cast<const uint4*>(ostage + row * kD + 8 * ch);
        }
      }
    }
    fence_proxy_async_smem();
    tc_fence_before();
    __syncthreads();
    if constexpr (kPre) {
      if (!last) issue_p(c + 1);  // the output staging in the P region has been read
    }
  }

  pdl_allow_next();
  if (aborted) {
    if (tid == 0) report(p.status, OQ_DEV_TIMEOUT);
    // Let every issued MMA and copy land before TMEM and shared memory go away.
    if (tid == 0) umma_commit(&bars->drain);
    wait_bar(&bars->drain, 0, kDefaultWaitPolls);
    for (int s = 0; s < 2; ++s) {
      while (kq_waited[s] < kq_issued[s]) wait_bar(&bars->kq[s], (kq_waited[s]++) & 1, kDefaultWaitPolls);
    }
    while (v_waited < v_issued) wait_bar(&bars->v, (v_waited++) & 1, kDefaultWaitPolls);
    while (ab_waited < ab_issued) wait_bar(&bars->ab, (ab_waited++) & 1, kDefaultWaitPolls);
    while (p_waited < p_issued) wait_bar(&bars->pp, (p_waited++) & 1, kDefaultWaitPolls);
  } else if (p.s_out != nullptr) {
    tc_fence_after();
#pragma unroll 1
    for (int q4 = 2 * half; q4 < 2 * half + 2; ++q4) {
      float sv[32];
      tmem_ld32(lane_base + kColS + 32 * q4, sv);
#pragma unroll
      for (int j = 0; j < 32; ++j) p.s_out[state_base + int64_t(32 * q4 + j) * kD + lane] = sv[j];
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, kTmemCols);
}

// ---------------------------------------------------------------- two-phase form
// Phase 1 (gdn_chunk_prep_kernel) does, for every chunk of every (sequence, head) at once,
// the part of a chunk's work that does not depend on the state: the norms and decays, the
// Gram matrix, N and P, X = (I - N)^-1 and the split Ar / Ab tiles.  It writes them to a
// workspace as the exact shared-memory images phase 2 uses (per chunk: Ar hi | Ar lo |
// Ab hi | Ab lo, then P hi | P lo, 8 KB each in the 128-byte swizzle, then sfac[64], cq[64],
// e^{gc_last}).  Phase 2 (gdn_chunk_kernel<true>) walks the chunks of a (sequence, head) in
// order as before, but copies those images in instead of computing them, so its per-chunk
// chain keeps only the state products.  The arithmetic is the single-kernel form's.
// phase-1 shared memory (1024-aligned base): the K / Q tiles of the chunk; once the Gram MMA
// and the norms are done, X and the solve scratch reuse them
constexpr uint32_t kP1OffX = 0;                         // [64][68] fp32
constexpr uint32_t kP1OffT = 17408;                     // solve scratch, up to [32][36] fp32
constexpr uint32_t kP1OffN = kKQBytes;                  // [64][65] fp32
constexpr uint32_t kP1OffTok = kP1OffN + 16640;         // 9 per-token arrays of 64 floats
constexpr uint32_t kP1OffBars = kP1OffTok + kTokArrays * kC * 4;
constexpr uint32_t kP1Smem = kP1OffBars + 64 + 1024;
constexpr uint32_t kP1TmemCols = 64;

struct PrepBars {
  uint64_t kq;
  uint64_t mma;
  uint32_t tmem_base;
};

__global__ void __launch_bounds__(kThreads)
    gdn_chunk_prep_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                          ChunkParams p, uint8_t* workspace) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sa = smem_addr(sm);
  float* f_small = reinterpret_cast<float*>(sm + kP1OffTok);
  auto tok = [&](int, int k) { return f_small + k * kC; };  // one buffer
  float* s_T = reinterpret_cast<float*>(sm + kP1OffT);
  float* s_N = reinterpret_cast<float*>(sm + kP1OffN);
  float* s_X = reinterpret_cast<float*>(sm + kP1OffX);
  PrepBars* bars = reinterpret_cast<PrepBars*>(sm + kP1OffBars);

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 127;
  const int half = tid >> 7;
  const int c = blockIdx.x;
  const int h = blockIdx.y;
  const int b = blockIdx.z;
  const int H = p.num_heads;
  const int64_t T = p.seq_len;
  const int n_chunks = int((T + kC - 1) / kC);
  uint8_t* img = workspace + ((int64_t(b) * H + h) * n_chunks + c) * int64_t(kImgBytes);

  if (tid == 0) {
    mbar_init(&bars->kq, 1);
    mbar_init(&bars->mma, 1);
    fence_mbar_init();
  }
  __syncwarp();
  if (warp == 0) {
    tmem_alloc(&bars->tmem_base, kP1TmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bars->tmem_base;
  const uint32_t lane_base = tmem + (uint32_t((warp & 3) * 32) << 16);
  pdl_wait();
  if (tid == 0) {
    mbar_arrive_expect_tx(&bars->kq, kKQBytes);
    const int t0 = c * kC;
    tma_load_4d(sm, &tm_k, 0, h, t0, b, &bars->kq);
    tma_load_4d(sm + kTile, &tm_q, 0, h, t0, b, &bars->kq);
    tma_load_4d(sm + 2 * kTile, &tm_k, 64, h, t0, b, &bars->kq);
    tma_load_4d(sm + 3 * kTile, &tm_q, 64, h, t0, b, &bars->kq);
  }
  float gv = 0.0f, bv = 0.0f;
  {
    const int64_t t = int64_t(c) * kC + tid;
    if (tid < kC && t < T) {
      const int64_t gi = (int64_t(b) * T + t) * H + h;
      gv = load_as_float(p.g, p.g_dtype, gi);
      bv = load_as_float(p.beta, p.beta_dtype, gi);
    }
  }
  bool issued_mma = false;
  bool ok = wait_bar(&bars->kq, 0, p.wait_polls);
  if (__syncthreads_or(!ok) == 0) {
    // G = [K; Q] K^T (M = 128: 64 keys then 64 queries; N = 64 keys; K = d)
    if (tid == 0) {
      tc_fence_after();
#pragma unroll
      for (int kk = 0; kk < 8; ++kk) {
        const uint32_t off = sa + (kk >> 2) * 2 * kTile + (kk & 3) * 32;
        umma_bf16(tmem + kColG, smem_desc_sw128(off, 16, 1024), smem_desc_sw128(off, 16, 1024), kIdescN64, kk > 0);
      }
      umma_commit(&bars->mma);
    }
    issued_mma = true;
    // per-token scalars: g, beta, inverse norms, in-chunk cumulative decay and the factors
    const uint8_t* kqc = sm;
    if (tid < kC) {
      tok(0, 0)[tid] = gv;
      tok(0, 2)[tid] = bv;
      tok(0, 3)[tid] = p.l2norm ? 1.0f / sqrtf(row_sumsq(kqc, kqc + 2 * kTile, tid) + 1e-6f) : 1.0f;
    } else if (tid < 2 * kC) {
      const int r = tid - kC;
      tok(0, 4)[r] = p.l2norm ? 1.0f / sqrtf(row_sumsq(kqc + kTile, kqc + 3 * kTile, r) + 1e-6f) : 1.0f;
    }
    __syncthreads();
    if (warp == 0) {
      const float a0 = tok(0, 0)[2 * tid], a1 = tok(0, 0)[2 * tid + 1];
      float incl = a0 + a1;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const float y = __shfl_up_sync(0xffffffffu, incl, o);
        if (tid >= o) incl += y;
      }
      float excl = __shfl_up_sync(0xffffffffu, incl, 1);
      if (tid == 0) excl = 0.0f;
      const float gc[2] = {excl + a0, (excl + a0) + a1};
      const float gl = __shfl_sync(0xffffffffu, gc[1], 31);
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int t = 2 * tid + e;
        const float dk = tok(0, 3)[t];
        tok(0, 1)[t] = gc[e];
        tok(0, 8)[t] = gc[e] * 1.4426950408889634f;
        tok(0, 5)[t] = dk * expf(gl - gc[e]);
        tok(0, 6)[t] = p.scale * tok(0, 4)[t] * expf(gc[e]);
        tok(0, 7)[t] = tok(0, 2)[t] * expf(gc[e]) * dk;
      }
    }
    ok = wait_bar(&bars->mma, 0, p.wait_polls);
    if (__syncthreads_or(!ok) == 0) {
      tc_fence_after();
      const float* s_gc = tok(0, 1);
      const float* s_beta = tok(0, 2);
      const float* s_dk = tok(0, 3);
      const float* s_dq = tok(0, 4);
      const float* s_rfac = tok(0, 7);
      const float* s_gcl = tok(0, 8);
      (void)s_gc;
    // ---- rows of N (lanes 0..63) and P (lanes 64..127) from the Gram lanes; each thread
    // takes 32 of the 64 columns
    {
      float gr[32];
      tmem_ld32(lane_base + kColG + 32 * half, gr);
      const int j0 = 32 * half;
      if (lane < kC) {
        const int i = lane;
        const float fi = -s_beta[i] * s_dk[i];
        const float gli = s_gcl[i];
        float* nrow = s_N + i * kNStride + j0;
#pragma unroll
        for (int jj = 0; jj < 32; ++jj) {
          const int j = j0 + jj;
          nrow[jj] = j < i ? fi * s_dk[j] * gr[jj] * exp2f(gli - s_gcl[j]) : 0.0f;
        }
      } else {
        const int i = lane - kC;
        const float fi = p.scale * s_dq[i];
        const float gli = s_gcl[i];
#pragma unroll
        for (int cc = 0; cc < 4; ++cc) {
          float pv[8];
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            const int j = j0 + 8 * cc + e;
            pv[e] = j <= i ? fi * s_dk[j] * gr[8 * cc + e] * exp2f(gli - s_gcl[j]) : 0.0f;
          }
          store_split8(img + kImgP, img + kImgP + kTile, swz(i, 4 * half + cc), pv);
        }
      }
    }
    tc_fence_before();
    __syncthreads();

    // ---- X = (I - N)^-1 by doubling.  16x16 diagonal blocks by forward substitution
    // (one column per thread), zeroing the blocks right of blocks 0 and 2 ...
    if (tid < kC) {
      const int o = 16 * (tid >> 4), jj = tid & 15;
      float x[16];
#pragma unroll
      for (int m = 0; m < 16; ++m) x[m] = m == jj ? 1.0f : 0.0f;
#pragma unroll
      for (int ii = 1; ii < 16; ++ii) {
        float acc = 0.0f;
#pragma unroll
        for (int m = 0; m < ii; ++m) acc = fmaf(s_N[(o + ii) * kNStride + o + m], x[m], acc);
        if (ii > jj) x[ii] = acc;
      }
#pragma unroll
      for (int ii = 0; ii < 16; ++ii) s_X[(o + ii) * kXStride + o + jj] = x[ii];
      if ((o & 16) == 0) {
#pragma unroll
        for (int ii = 0; ii < 16; ++ii) s_X[(o + ii) * kXStride + o + 16 + jj] = 0.0f;
      }
    }
    __syncthreads();
    // ... then the 32x32 diagonal blocks: X_10 = X_11 N_10 X_00 and X_32 = X_33 N_32 X_22
    // (1x2 outputs per thread) ...
    {
      const int blk = tid >> 7, I = 16 * (1 + 2 * blk), J = 32 * blk;
      const int r = (tid & 127) >> 3, c0 = (tid & 7) * 2;
      float* tb = s_T + blk * 16 * kT2Stride;
      float a0 = 0.0f, a1 = 0.0f;
#pragma unroll
      for (int m = 0; m < 16; ++m) {
        const float n = s_N[(I + r) * kNStride + J + m];
        const float2 x = *reinterpret_cast<const float2*>(&s_X[(J + m) * kXStride + J + c0]);
        a0 = fmaf(n, x.x, a0);
        a1 = fmaf(n, x.y, a1);
      }
      *reinterpret_cast<float2*>(&tb[r * kT2Stride + c0]) = make_float2(a0, a1);
      __syncthreads();
      a0 = a1 = 0.0f;
#pragma unroll
      for (int m = 0; m < 16; ++m) {
        const float x = s_X[(I + r) * kXStride + I + m];
        const float2 t = *reinterpret_cast<const float2*>(&tb[m * kT2Stride + c0]);
        a0 = fmaf(x, t.x, a0);
        a1 = fmaf(x, t.y, a1);
      }
      *reinterpret_cast<float2*>(&s_X[(I + r) * kXStride + J + c0]) = make_float2(a0, a1);
    }
    __syncthreads();
    // ... and the lower-left 32x32 block: X[32:, :32] = X[32:, 32:] N[32:, :32] X[:32, :32]
    // Warp w computes columns 4w..4w+3 of T = N[32:, :32] X[:32, :32] (lane = row; X[m][c] = 0
    // for m < c), then rows 4w..4w+3 of X[32:, 32:] T (lane = column; X[32 + r][32 + m] = 0 for m > r).
    {
      const int c0 = 4 * warp, r = tid & 31;
      float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll 4
      for (int m = c0; m < 32; ++m) {
        const float n = s_N[(32 + r) * kNStride + m];
        const float4 x = *reinterpret_cast<const float4*>(&s_X[m * kXStride + c0]);
        acc[0] = fmaf(n, x.x, acc[0]);
        acc[1] = fmaf(n, x.y, acc[1]);
        acc[2] = fmaf(n, x.z, acc[2]);
        acc[3] = fmaf(n, x.w, acc[3]);
      }
      *reinterpret_cast<float4*>(&s_T[r * kT3Stride + c0]) = make_float4(acc[0], acc[1], acc[2], acc[3]);
      __syncthreads();
      const int r0 = 4 * warp, col = tid & 31;
      float o[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll 1
      for (int m0 = 0; m0 < r0 + 4; m0 += 4) {
        float tcol[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) tcol[i] = s_T[(m0 + i) * kT3Stride + col];
#pragma unroll
        for (int a = 0; a < 4; ++a) {
          const float4 x = *reinterpret_cast<const float4*>(&s_X[(32 + r0 + a) * kXStride + 32 + m0]);
          o[a] = fmaf(x.x, tcol[0], o[a]);
          o[a] = fmaf(x.y, tcol[1], o[a]);
          o[a] = fmaf(x.z, tcol[2], o[a]);
          o[a] = fmaf(x.w, tcol[3], o[a]);
        }
      }
#pragma unroll
      for (int a = 0; a < 4; ++a) s_X[(32 + r0 + a) * kXStride + col] = o[a];
    }
    __syncthreads();

    // ---- Ar = X diag(beta e^gc dk), Ab = X diag(beta): split K-major tiles [t][m] (over N)
    {
      const int t = tid >> 2, qq = tid & 3;
#pragma unroll
      for (int cc = 0; cc < 2; ++cc) {
        const int c8 = 2 * qq + cc;
        float xr[8], ar[8], ab[8];
        *reinterpret_cast<float4*>(xr) = *reinterpret_cast<const float4*>(&s_X[t * kXStride + 8 * c8]);
        *reinterpret_cast<float4*>(xr + 4) = *reinterpret_cast<const float4*>(&s_X[t * kXStride + 8 * c8 + 4]);
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const int m = 8 * c8 + e;
          const float xv = m > t ? 0.0f : (m == t ? 1.0f : xr[e]);
          ar[e] = xv * s_rfac[m];
          ab[e] = xv * s_beta[m];
        }
        store_split8(img, img + kTile, swz(t, c8), ar);
        store_split8(img + 2 * kTile, img + 3 * kTile, swz(t, c8), ab);
      }
    }


      // the scalars phase 2 needs: sfac, cq and e^{gc_last}
      float* scal = reinterpret_cast<float*>(img + kImgScal);
      if (tid < kC) {
        scal[tid] = tok(0, 5)[tid];
      } else if (tid < 2 * kC) {
        scal[tid] = tok(0, 6)[tid - kC];
      } else if (tid == 2 * kC) {
        scal[tid] = expf(tok(0, 1)[kC - 1]);
      }
    }
  }
  pdl_allow_next();
  if (!ok) {
    if (tid == 0) report(p.status, OQ_DEV_TIMEOUT);
    // let the copy and the MMA land before shared and tensor memory go away
    if (tid == 0) wait_bar(&bars->kq, 0, kDefaultWaitPolls);
    if (issued_mma && tid == 0) wait_bar(&bars->mma, 0, kDefaultWaitPolls);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, kP1TmemCols);
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

namespace oq {
namespace {

// workspace == nullptr: the single-kernel form; otherwise the two-phase form with the
// per-chunk images in `workspace` (gdn_chunk_workspace_bytes).
int gdn_chunk_impl(
    const void* q, const void* k, const void* v, int qkv_dtype,
    int64_t q_stride_b, int64_t q_stride_t, int64_t q_stride_h,
    int64_t k_stride_b, int64_t k_stride_t, int64_t k_stride_h,
    int64_t v_stride_b, int64_t v_stride_t, int64_t v_stride_h,
    const void* g, int g_dtype, const void* beta, int beta_dtype,
    const float* initial_state, float* final_state, void* out,
    int64_t batch, int64_t seq_len, int64_t num_heads, int64_t k_dim, int64_t v_dim,
    float scale, int use_qk_l2norm, int64_t chunk_size, void* workspace, size_t workspace_bytes,
    int32_t* device_status, void* stream) {
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
  const int64_t n_chunks = (seq_len + kC - 1) / kC;
  const bool two_phase = workspace != nullptr;
  if (two_phase) {
    const size_t need = size_t(batch * num_heads * n_chunks) * kImgBytes;
    if (workspace_bytes < need) {
      return fail(OQ_ERR_WORKSPACE, "gdn_chunk_fwd: workspace of %zu bytes needed", need);
    }
    if (reinterpret_cast<uintptr_t>(workspace) % 128) {
      return fail(OQ_ERR_MISALIGNED, "gdn_chunk_fwd: workspace must be 128-byte aligned");
    }
    if (n_chunks > 65535) return fail(OQ_ERR_UNSUPPORTED, "gdn_chunk_fwd: more than 65535 chunks");
  }
  static bool attr_set[64][2] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !attr_set[dev][two_phase]) {
    cudaError_t e = two_phase
                        ? cudaFuncSetAttribute(gdn_chunk_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                               int(kSmemBytes))
                        : cudaFuncSetAttribute(gdn_chunk_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                               int(kSmemBytes));
    if (e == cudaSuccess && two_phase) {
      e = cudaFuncSetAttribute(gdn_chunk_prep_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(kP1Smem));
    }
    if (e != cudaSuccess) return check_launch("gdn_chunk_fwd: shared memory attribute");
    attr_set[dev][two_phase] = true;
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
  p.wait_polls = wait_polls();
  dim3 grid((unsigned)num_heads, (unsigned)batch);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (two_phase) {
    if (n_chunks > 0) {
      const dim3 pgrid((unsigned)n_chunks, (unsigned)num_heads, (unsigned)batch);
      launch_plain(gdn_chunk_prep_kernel, pgrid, dim3(kThreads), kP1Smem, s, maps[0], maps[1], p,
                   static_cast<uint8_t*>(workspace));
    }
    launch_plain(gdn_chunk_kernel<true>, grid, dim3(kThreads), kSmemBytes, s, maps[0], maps[1], maps[2], p,
                 static_cast<const uint8_t*>(workspace));
  } else {
    launch_plain(gdn_chunk_kernel<false>, grid, dim3(kThreads), kSmemBytes, s, maps[0], maps[1], maps[2], p,
                 static_cast<const uint8_t*>(nullptr));
  }
  return check_launch("gdn_chunk_fwd");
}

}  // namespace
}  // namespace oq

extern "C" size_t oq_gdn_chunk_workspace_bytes(int64_t batch, int64_t seq_len, int64_t num_heads) {
  if (batch <= 0 || seq_len <= 0 || num_heads <= 0) return 0;
  return size_t(batch * num_heads * ((seq_len + oq::kC - 1) / oq::kC)) * oq::kImgBytes;
}

extern "C" int oq_gdn_chunk_fwd(
    const void* q, const void* k, const void* v, int qkv_dtype,
    int64_t q_stride_b, int64_t q_stride_t, int64_t q_stride_h,
    int64_t k_stride_b, int64_t k_stride_t, int64_t k_stride_h,
    int64_t v_stride_b, int64_t v_stride_t, int64_t v_stride_h,
    const void* g, int g_dtype, const void* beta, int beta_dtype,
    const float* initial_state, float* final_state, void* out,
    int64_t batch, int64_t seq_len, int64_t num_heads, int64_t k_dim, int64_t v_dim,
    float scale, int use_qk_l2norm, int64_t chunk_size, int32_t* device_status, void* stream) {
  return oq::gdn_chunk_impl(q, k, v, qkv_dtype, q_stride_b, q_stride_t, q_stride_h, k_stride_b, k_stride_t,
                            k_stride_h, v_stride_b, v_stride_t, v_stride_h, g, g_dtype, beta, beta_dtype,
                            initial_state, final_state, out, batch, seq_len, num_heads, k_dim, v_dim, scale,
                            use_qk_l2norm, chunk_size, nullptr, 0, device_status, stream);
}

extern "C" int oq_gdn_chunk_fwd_ws(
    const void* q, const void* k, const void* v, int qkv_dtype,
    int64_t q_stride_b, int64_t q_stride_t, int64_t q_stride_h,
    int64_t k_stride_b, int64_t k_stride_t, int64_t k_stride_h,
    int64_t v_stride_b, int64_t v_stride_t, int64_t v_stride_h,
    const void* g, int g_dtype, const void* beta, int beta_dtype,
    const float* initial_state, float* final_state, void* out,
    int64_t batch, int64_t seq_len, int64_t num_heads, int64_t k_dim, int64_t v_dim,
    float scale, int use_qk_l2norm, int64_t chunk_size, void* workspace, size_t workspace_bytes,
    int32_t* device_status, void* stream) {
  if (workspace == nullptr) return oq::fail(OQ_ERR_WORKSPACE, "gdn_chunk_fwd_ws: null workspace");
  return oq::gdn_chunk_impl(q, k, v, qkv_dtype, q_stride_b, q_stride_t, q_stride_h, k_stride_b, k_stride_t,
                            k_stride_h, v_stride_b, v_stride_t, v_stride_h, g, g_dtype, beta, beta_dtype,
                            initial_state, final_state, out, batch, seq_len, num_heads, k_dim, v_dim, scale,
                            use_qk_l2norm, chunk_size, workspace, workspace_bytes, device_status, stream);
}
