// Split-KV INT4 paged decode attention (one query token per sequence).
//
// Replaces qserve_int4_decode_attention / qserve_int4_split_decode_attention and
// their Triton kernels (optiz_qwen/kernels/qserve_int4_attention.py:112-205,
// 209-261, 328-395, launchers :520-545, :576-620).  Differences from the
// reference design, chosen for B200:
//   * the cache is paged (page = 64 tokens) and every token is already INT4;
//   * one CTA serves all query heads of a KV head (GQA), so each K/V byte is
//     read from HBM once instead of once per query head;
//   * a page of K+V codes (16 KB) plus its scale/min (512 B) is staged into
//     shared memory by one TMA tensor copy (128-byte swizzle) and one bulk copy,
//     four pages in flight per CTA, completion tracked by mbarriers with
//     bounded waits;
//   * nibbles are turned into bf16/fp16 in registers (lop3 with an exponent
//     bias, then an exact subtract) and both q.k and p.v run on the tensor
//     cores (mma.sync m16n8k16, the GQA heads as the N=8 dimension);
//     scale/min are applied after the dot products:
//       q.k = scale * sum(q*code) + min * sum(q),  p.v = sum((p*scale)*code) + sum(p*min);
//   * the KV range is split across CTAs and the partial (max, sum, acc) are
//     merged by log-sum-exp by the last CTA of each (sequence, KV head).
#include <cudaTypedefs.h>

#include <algorithm>
#include <cmath>
#include <mutex>

#include "common.cuh"

namespace oq {
namespace {

constexpr int kHeadDim = 256;
constexpr int kPage = 64;
constexpr int kRowBytes = kHeadDim / 2;                // 128 bytes of codes per token
constexpr int kStageCodeBytes = 2 * kPage * kRowBytes;  // K rows then V rows: 16 KB
constexpr int kStageMetaBytes = 4 * kPage * 2;          // 512 B of fp16 scale/min
constexpr int kStages = 4;
constexpr int kWarps = 4;
constexpr int kThreads = kWarps * 32;
constexpr int kMaxGroup = 8;
constexpr int kMaxSplits = 512;
constexpr long long kWaitCycles = 4000000000LL;  // ~2 s at 2 GHz: a copy that has not landed by then never will

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
  int32_t* status;
};

struct __align__(16) SmemTail {
  uint64_t full[kStages];
  int stage_ok[kStages];
  float warp_m[kWarps][kMaxGroup];
  float warp_l[kWarps][kMaxGroup];
  int is_last;
};

constexpr size_t kSmemBytes =
    1024 /*alignment slack*/ + kStages * (kStageCodeBytes + kStageMetaBytes) + sizeof(SmemTail);

// Nibble -> 16-bit float conversion.  lop3 puts codes c0 (bits 0-3) and c4
// (bits 16-19) of a word into the mantissa of an exponent-biased constant, giving
// (bias + c) exactly; callers either fold the bias into the epilogue or subtract it.
template <typename T> struct QkTraits;
template <> struct QkTraits<__nv_bfloat16> {
  // q.k runs on bf16 operands: codes become 128 + c; the 128 * sum(q) term is
  // removed in the score epilogue.
  static constexpr float kBias = 128.0f;
  static __device__ __forceinline__ uint32_t codes(uint32_t x) { return lop3_and_or(x, 0x000F000Fu, 0x43004300u); }
  static __device__ __forceinline__ void mma(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    mma_bf16_16816(d, a, b0, b1);
  }
};
template <> struct QkTraits<__half> {
  // fp16 queries: exact codes (1024 + c) - 1024.
  static constexpr float kBias = 0.0f;
  static __device__ __forceinline__ uint32_t codes(uint32_t x) {
    uint32_t v = lop3_and_or(x, 0x000F000Fu, 0x64006400u);
    __half2 h = *reinterpret_cast<__half2*>(&v);
    __half2 r = __hsub2(h, __floats2half2_rn(1024.0f, 1024.0f));
    return *reinterpret_cast<uint32_t*>(&r);
  }
  static __device__ __forceinline__ void mma(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    mma_f16_16816(d, a, b0, b1);
  }
};

// p.v runs on fp16 operands: codes become 1024 + c, removed with 1024 * sum(P').
constexpr float kVBias = 1024.0f;
__device__ __forceinline__ uint32_t v_codes(uint32_t x) { return lop3_and_or(x, 0x000F000Fu, 0x64006400u); }

// Lazy softmax rescale: the running max only moves when a tile's max exceeds it
// by more than kTau (log2 units), so p <= 2^kTau; P' = p * v_scale * 2^-kTau
// therefore stays inside the fp16 range whatever the stored fp16 scale.
constexpr float kTau = 4.0f;
constexpr float kPScale = 0.0625f;  // 2^-kTau
constexpr float kPUnscale = 16.0f;

// Shared-memory address of 16-byte chunk `chunk` of row `row` in a 128B-swizzled stage.
__device__ __forceinline__ const uint4* swz(const uint8_t* base, int row, int chunk) {
  return reinterpret_cast<const uint4*>(base + row * kRowBytes + ((chunk ^ (row & 7)) << 4));
}

__device__ __forceinline__ bool wait_stage(uint64_t* bar, uint32_t parity) {
  if (mbar_try_wait(bar, parity)) return true;
  const long long t0 = clock64();
  while (!mbar_try_wait(bar, parity)) {
    if (clock64() - t0 > kWaitCycles) return false;
  }
  return true;
}

__device__ __forceinline__ float lse_nat(float m_log2, float l) {
  return l > 0.0f ? (m_log2 + log2f(l)) * 0.69314718055994531f : -INFINITY;
}

template <typename T>
__device__ __forceinline__ void store_out(const AttnParams& p, int64_t b, int64_t hq, int d, float o, float m,
                                          float l) {
  const int64_t hq_total = p.num_kv_heads * p.group;
  if (p.out) static_cast<T*>(p.out)[b * p.o_sb + hq * p.o_sh + d] = from_float<T>(o);
  if (p.out_f32) p.out_f32[(b * hq_total + hq) * kHeadDim + d] = o;
  if (p.out_lse && d == 0) p.out_lse[b * hq_total + hq] = lse_nat(m, l);
}

template <typename T>
__global__ void __launch_bounds__(kThreads) decode_attn_kernel(const __grid_constant__ CUtensorMap tmap,
                                                               AttnParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* codes = smem;                                       // kStages x 16 KB, 1024-aligned
  uint8_t* metas = smem + kStages * kStageCodeBytes;           // kStages x 512 B
  SmemTail* tail = reinterpret_cast<SmemTail*>(metas + kStages * kStageMetaBytes);

  const int tid = threadIdx.x;
  const int lane = tid & 31;
  const int warp = tid >> 5;
  const int r = lane >> 2;  // mma groupID
  const int c = lane & 3;   // mma thread-in-group
  const int split = blockIdx.x;
  const int kvh = blockIdx.y;
  const int64_t b = blockIdx.z;
  const int G = p.group;

  const int len = max(p.seq_lens[b], 0);
  const int len_pages = (len + kPage - 1) / kPage;
  const int npages_b = int(min(int64_t(len_pages), p.max_pages));
  const int nsplit_b = max(1, (npages_b + p.pages_per_split - 1) / p.pages_per_split);
  if (split >= nsplit_b) return;
  if (len_pages > p.max_pages && tid == 0 && split == 0) report(p.status, OQ_DEV_OVERFLOW);
  const int page_begin = split * p.pages_per_split;
  const int n = max(0, min(npages_b, page_begin + p.pages_per_split) - page_begin);

  if (tid == 0) {
    for (int s = 0; s < kStages; ++s) mbar_init(&tail->full[s], 1);
    fence_mbar_init();
  }
  __syncthreads();

  const int32_t* bt_row = p.block_table + b * p.bt_stride;
  auto issue = [&](int i, int s) {
    const int64_t page = bt_row[page_begin + i];
    if (page < 0 || page >= p.num_pages) {
      tail->stage_ok[s] = 0;
      report(p.status, OQ_DEV_BAD_PAGE);
      mbar_arrive(&tail->full[s]);
      return;
    }
    tail->stage_ok[s] = 1;
    const int64_t blk = page * p.num_kv_heads + kvh;
    mbar_arrive_expect_tx(&tail->full[s], kStageCodeBytes + kStageMetaBytes);
    tma_load_2d(codes + s * kStageCodeBytes, &tmap, 0, int32_t(blk * 2 * kPage), &tail->full[s]);
    bulk_load(metas + s * kStageMetaBytes, p.kv_meta + blk * 4 * kPage, kStageMetaBytes, &tail->full[s]);
  };
  int issued = 0;
  if (tid == 0) {
    for (; issued < min(n, kStages); ++issued) issue(issued, issued);
  }

  // ---- query fragments (B operand of q.k): head r, dims 64c + 8i + {0..7}
  using Q = QkTraits<T>;
  uint32_t qb[16][2];
  float qsum = 0.0f;
  {
    const bool has = r < G;
    const T* qrow = static_cast<const T*>(p.query) + b * p.q_sb + int64_t(kvh * G + (has ? r : 0)) * p.q_sh + 64 * c;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      uint4 w = has ? __ldg(reinterpret_cast<const uint4*>(qrow + 8 * i)) : make_uint4(0, 0, 0, 0);
      qb[2 * i][0] = prmt(w.x, w.z, 0x5410);
      qb[2 * i][1] = prmt(w.x, w.z, 0x7632);
      qb[2 * i + 1][0] = prmt(w.y, w.w, 0x5410);
      qb[2 * i + 1][1] = prmt(w.y, w.w, 0x7632);
      const T* e = reinterpret_cast<const T*>(&w);
#pragma unroll
      for (int j = 0; j < 8; ++j) qsum += to_float<T>(e[j]);
    }
    qsum += __shfl_xor_sync(0xffffffffu, qsum, 1);
    qsum += __shfl_xor_sync(0xffffffffu, qsum, 2);
  }
  // sum(q) of the two heads (2c, 2c+1) whose scores this lane holds
  const float qs_a = __shfl_sync(0xffffffffu, qsum, (2 * c) * 4);
  const float qs_b = __shfl_sync(0xffffffffu, qsum, (2 * c + 1) * 4);

  float acc[16][4];
#pragma unroll
  for (int j = 0; j < 16; ++j) acc[j][0] = acc[j][1] = acc[j][2] = acc[j][3] = 0.0f;
  float m_a = -INFINITY, m_b = -INFINITY;  // reference max (log2 units) of heads 2c, 2c+1
  float l_a = 0.0f, l_b = 0.0f;            // this lane's share of sum(p)
  float mp_a = 0.0f, mp_b = 0.0f;          // ... of sum(p * v_min)
  float sp_a = 0.0f, sp_b = 0.0f;          // ... of sum(P') with P' as rounded to fp16

  const int tok0 = warp * 16 + r;  // token rows of this lane in the page (A rows r and r+8)
  const int tok1 = tok0 + 8;
  bool aborted = false;

  for (int i = 0; i < n; ++i) {
    const int s = i % kStages;
    const uint32_t parity = (i / kStages) & 1;
    bool ready = wait_stage(&tail->full[s], parity);
    ready = __all_sync(0xffffffffu, ready);
    const int page_tokens = min(kPage, len - (page_begin + i) * kPage);
    if (ready && tail->stage_ok[s] && warp * 16 < page_tokens) {
      const uint8_t* st = codes + s * kStageCodeBytes;
      const __half* meta = reinterpret_cast<const __half*>(metas + s * kStageMetaBytes);
      const int tb = warp * 16 + kPage;  // V rows follow the 64 K rows
      const uint4 k00 = *swz(st, tok0, 2 * c), k01 = *swz(st, tok0, 2 * c + 1);
      const uint4 k10 = *swz(st, tok1, 2 * c), k11 = *swz(st, tok1, 2 * c + 1);
      const uint4 va = *swz(st, tb + 2 * c, r), vb = *swz(st, tb + 2 * c + 1, r);
      const uint4 vc = *swz(st, tb + 2 * c + 8, r), vd = *swz(st, tb + 2 * c + 9, r);

      // ---------------- scores: A = K codes (16 tokens x 16 dims), B = q (16 dims x 8 heads);
      // two independent accumulator chains
      float sc0[4] = {0.0f, 0.0f, 0.0f, 0.0f}, sc1[4] = {0.0f, 0.0f, 0.0f, 0.0f};
      {
        const uint32_t w0[8] = {k00.x, k00.y, k00.z, k00.w, k01.x, k01.y, k01.z, k01.w};
        const uint32_t w1[8] = {k10.x, k10.y, k10.z, k10.w, k11.x, k11.y, k11.z, k11.w};
#pragma unroll
        for (int wi = 0; wi < 8; ++wi) {
          float(&sc)[4] = (wi & 1) ? sc1 : sc0;
          uint32_t a[4];
          a[0] = Q::codes(w0[wi]);
          a[1] = Q::codes(w1[wi]);
          a[2] = Q::codes(w0[wi] >> 4);
          a[3] = Q::codes(w1[wi] >> 4);
          Q::mma(sc, a, qb[2 * wi][0], qb[2 * wi][1]);
          a[0] = Q::codes(w0[wi] >> 8);
          a[1] = Q::codes(w1[wi] >> 8);
          a[2] = Q::codes(w0[wi] >> 12);
          a[3] = Q::codes(w1[wi] >> 12);
          Q::mma(sc, a, qb[2 * wi + 1][0], qb[2 * wi + 1][1]);
        }
      }
      const bool v0 = tok0 < page_tokens, v1 = tok1 < page_tokens;
      const float ks0 = __half2float(meta[tok0]), km0 = __half2float(meta[kPage + tok0]);
      const float ks1 = __half2float(meta[tok1]), km1 = __half2float(meta[kPage + tok1]);
      const float vs0 = __half2float(meta[2 * kPage + tok0]), vm0 = __half2float(meta[3 * kPage + tok0]);
      const float vs1 = __half2float(meta[2 * kPage + tok1]), vm1 = __half2float(meta[3 * kPage + tok1]);
      // q.k = scale * sum(q * (bias + c)) + (min - bias * scale) * sum(q)
      const float kb0 = fmaf(-Q::kBias, ks0, km0), kb1 = fmaf(-Q::kBias, ks1, km1);
      const float s0a = v0 ? fmaf(ks0, sc0[0] + sc1[0], kb0 * qs_a) * p.scale_log2 : -INFINITY;
      const float s0b = v0 ? fmaf(ks0, sc0[1] + sc1[1], kb0 * qs_b) * p.scale_log2 : -INFINITY;
      const float s1a = v1 ? fmaf(ks1, sc0[2] + sc1[2], kb1 * qs_a) * p.scale_log2 : -INFINITY;
      const float s1b = v1 ? fmaf(ks1, sc0[3] + sc1[3], kb1 * qs_b) * p.scale_log2 : -INFINITY;

      // ---------------- online softmax with a lazily moved reference max
      float tm_a = fmaxf(s0a, s1a), tm_b = fmaxf(s0b, s1b);
#pragma unroll
      for (int o = 4; o < 32; o <<= 1) {
        tm_a = fmaxf(tm_a, __shfl_xor_sync(0xffffffffu, tm_a, o));
        tm_b = fmaxf(tm_b, __shfl_xor_sync(0xffffffffu, tm_b, o));
      }
      if (__any_sync(0xffffffffu, tm_a > m_a + kTau || tm_b > m_b + kTau)) {
        const float nm_a = fmaxf(m_a, tm_a), nm_b = fmaxf(m_b, tm_b);
        const float corr_a = nm_a == -INFINITY ? 1.0f : exp2f(m_a - nm_a);
        const float corr_b = nm_b == -INFINITY ? 1.0f : exp2f(m_b - nm_b);
        m_a = nm_a;
        m_b = nm_b;
        l_a *= corr_a;
        l_b *= corr_b;
        mp_a *= corr_a;
        mp_b *= corr_b;
        sp_a *= corr_a;
        sp_b *= corr_b;
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          acc[j][0] *= corr_a;
          acc[j][2] *= corr_a;
          acc[j][1] *= corr_b;
          acc[j][3] *= corr_b;
        }
      }
      const float p0a = v0 ? exp2f(s0a - m_a) : 0.0f, p0b = v0 ? exp2f(s0b - m_b) : 0.0f;
      const float p1a = v1 ? exp2f(s1a - m_a) : 0.0f, p1b = v1 ? exp2f(s1b - m_b) : 0.0f;
      l_a += p0a + p1a;
      l_b += p0b + p1b;
      mp_a += (v0 ? p0a * vm0 : 0.0f) + (v1 ? p1a * vm1 : 0.0f);
      mp_b += (v0 ? p0b * vm0 : 0.0f) + (v1 ? p1b * vm1 : 0.0f);
      // P' = p * v_scale * 2^-kTau in fp16, rows = tokens, cols = heads
      const float ps0 = v0 ? vs0 * kPScale : 0.0f, ps1 = v1 ? vs1 * kPScale : 0.0f;
      const uint32_t blk0 = pack_half2(p0a * ps0, p0b * ps0);
      const uint32_t blk1 = pack_half2(p1a * ps1, p1b * ps1);
      {
        const float2 r0 = __half22float2(*reinterpret_cast<const __half2*>(&blk0));
        const float2 r1 = __half22float2(*reinterpret_cast<const __half2*>(&blk1));
        sp_a += r0.x + r1.x;
        sp_b += r0.y + r1.y;
      }
      // transpose into the B operand of p.v
      const uint32_t pb0 = movmatrix_trans(blk0);
      const uint32_t pb1 = movmatrix_trans(blk1);

      // ---------------- values: A = V^T codes (16 dims x 16 tokens), B = P' (16 tokens x 8 heads)
      {
        const uint32_t wa[4] = {va.x, va.y, va.z, va.w}, wb[4] = {vb.x, vb.y, vb.z, vb.w};
        const uint32_t wc[4] = {vc.x, vc.y, vc.z, vc.w}, wd[4] = {vd.x, vd.y, vd.z, vd.w};
#pragma unroll
        for (int wi = 0; wi < 4; ++wi) {
          const uint32_t x_lo = prmt(wa[wi], wb[wi], 0x5410), x_hi = prmt(wa[wi], wb[wi], 0x7632);
          const uint32_t y_lo = prmt(wc[wi], wd[wi], 0x5410), y_hi = prmt(wc[wi], wd[wi], 0x7632);
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            const uint32_t x = u < 2 ? x_lo : x_hi;
            const uint32_t y = u < 2 ? y_lo : y_hi;
            const int sh = (u & 1) * 8;
            uint32_t a[4];
            a[0] = v_codes(x >> sh);
            a[1] = v_codes(x >> (sh + 4));
            a[2] = v_codes(y >> sh);
            a[3] = v_codes(y >> (sh + 4));
            mma_f16_16816(acc[4 * wi + u], a, pb0, pb1);
          }
        }
      }
    }
    const bool stop = __syncthreads_or(!ready);
    if (stop) {
      aborted = true;
      break;
    }
    if (tid == 0 && i + kStages < n) {
      issue(i + kStages, s);
      ++issued;
    }
  }

  if (aborted) {
    // Leave no copy in flight before the CTA exits: wait (bounded) for every issued stage.
    if (tid == 0) {
      report(p.status, OQ_DEV_TIMEOUT);
      for (int i = max(0, issued - kStages); i < issued; ++i) {
        wait_stage(&tail->full[i % kStages], (i / kStages) & 1);
      }
    }
    return;
  }

  // ---- reduce this warp's per-lane sums over the 8 token rows
#pragma unroll
  for (int o = 4; o < 32; o <<= 1) {
    l_a += __shfl_xor_sync(0xffffffffu, l_a, o);
    l_b += __shfl_xor_sync(0xffffffffu, l_b, o);
    mp_a += __shfl_xor_sync(0xffffffffu, mp_a, o);
    mp_b += __shfl_xor_sync(0xffffffffu, mp_b, o);
    sp_a += __shfl_xor_sync(0xffffffffu, sp_a, o);
    sp_b += __shfl_xor_sync(0xffffffffu, sp_b, o);
  }
  if (r == 0) {
    tail->warp_m[warp][2 * c] = m_a;
    tail->warp_m[warp][2 * c + 1] = m_b;
    tail->warp_l[warp][2 * c] = l_a;
    tail->warp_l[warp][2 * c + 1] = l_b;
  }
  __syncthreads();  // also: every stage has been consumed, codes[] is free for reuse

  // ---- merge the 4 warps: red[w][h][d] = numerator_w * 2^(m_w - M),
  //      numerator = 2^kTau * (acc - 1024 * sum(P')) + sum(p * v_min)
  float* red = reinterpret_cast<float*>(codes);  // kWarps * kMaxGroup * 256 floats = 32 KB
  {
    const int ha = 2 * c, hb = 2 * c + 1;
    float fa = 0.0f, fb = 0.0f;
    if (ha < G) {
      float M = -INFINITY;
      for (int w = 0; w < kWarps; ++w) M = fmaxf(M, tail->warp_m[w][ha]);
      fa = M == -INFINITY ? 0.0f : exp2f(m_a - M);
    }
    if (hb < G) {
      float M = -INFINITY;
      for (int w = 0; w < kWarps; ++w) M = fmaxf(M, tail->warp_m[w][hb]);
      fb = M == -INFINITY ? 0.0f : exp2f(m_b - M);
    }
    const float off_a = -kVBias * sp_a, off_b = -kVBias * sp_b;
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const int d0 = 32 * r + 2 * j;
      if (ha < G) {
        red[(warp * kMaxGroup + ha) * kHeadDim + d0] = fmaf(acc[j][0] + off_a, kPUnscale, mp_a) * fa;
        red[(warp * kMaxGroup + ha) * kHeadDim + d0 + 1] = fmaf(acc[j][2] + off_a, kPUnscale, mp_a) * fa;
      }
      if (hb < G) {
        red[(warp * kMaxGroup + hb) * kHeadDim + d0] = fmaf(acc[j][1] + off_b, kPUnscale, mp_b) * fb;
        red[(warp * kMaxGroup + hb) * kHeadDim + d0 + 1] = fmaf(acc[j][3] + off_b, kPUnscale, mp_b) * fb;
      }
    }
  }
  __syncthreads();

  const int outputs = G * kHeadDim;
  const int64_t unit = b * p.num_kv_heads + kvh;
  const bool single = nsplit_b == 1;
  const int rec_floats = G * (kHeadDim + 2);
  float* my_rec = p.partials + (unit * p.max_splits + split) * rec_floats;

  for (int e = tid; e < outputs; e += kThreads) {
    const int h = e / kHeadDim;
    const int d = e - h * kHeadDim;
    float M = -INFINITY;
    for (int w = 0; w < kWarps; ++w) M = fmaxf(M, tail->warp_m[w][h]);
    float L = 0.0f, num = 0.0f;
    for (int w = 0; w < kWarps; ++w) {
      const float f = M == -INFINITY ? 0.0f : exp2f(tail->warp_m[w][h] - M);
      L += tail->warp_l[w][h] * f;
      num += red[(w * kMaxGroup + h) * kHeadDim + d];
    }
    if (single) {
      store_out<T>(p, b, int64_t(kvh) * G + h, d, L > 0.0f ? num / L : 0.0f, M, L);
    } else {
      my_rec[e] = num;
      if (d == 0) {
        my_rec[outputs + h] = M;
        my_rec[outputs + G + h] = L;
      }
    }
  }
  if (single) return;

  // ---- split-KV merge by the last CTA of this (sequence, KV head)
  __threadfence();
  __syncthreads();
  if (tid == 0) {
    const int done = atomicAdd(&p.counters[unit], 1);
    tail->is_last = done == nsplit_b - 1;
  }
  __syncthreads();
  if (!tail->is_last) return;
  __threadfence();
  const float* recs = p.partials + unit * p.max_splits * rec_floats;
  // stage every split's (M, L) in shared memory, then turn M into merge weights
  float* wm = reinterpret_cast<float*>(codes);  // [nsplit_b][G]
  float* wl = wm + nsplit_b * G;                // [nsplit_b][G]
  float* head_m = wl + nsplit_b * G;            // [G]
  float* head_l = head_m + kMaxGroup;           // [G]
  for (int idx = tid; idx < nsplit_b * G; idx += kThreads) {
    const int s = idx / G, h = idx - (idx / G) * G;
    wm[idx] = __ldcg(recs + s * rec_floats + outputs + h);
    wl[idx] = __ldcg(recs + s * rec_floats + outputs + G + h);
  }
  __syncthreads();
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
  __syncthreads();
  for (int idx = tid; idx < nsplit_b * G; idx += kThreads) {
    const int h = idx - (idx / G) * G;
    const float M = head_m[h];
    wm[idx] = M == -INFINITY ? 0.0f : exp2f(wm[idx] - M);
  }
  __syncthreads();
  constexpr int kMaxPer = kMaxGroup * kHeadDim / kThreads;  // 16 outputs per thread at most
  const int per = outputs / kThreads;
  float num[kMaxPer];
#pragma unroll
  for (int j = 0; j < kMaxPer; ++j) num[j] = 0.0f;
  for (int s = 0; s < nsplit_b; ++s) {
    const float* rec = recs + s * rec_floats;
#pragma unroll
    for (int j = 0; j < kMaxPer; ++j) {
      if (j < per) {
        const int e = tid + j * kThreads;
        num[j] = fmaf(wm[s * G + e / kHeadDim], __ldcg(rec + e), num[j]);
      }
    }
  }
#pragma unroll
  for (int j = 0; j < kMaxPer; ++j) {
    if (j < per) {
      const int e = tid + j * kThreads;
      const int h = e / kHeadDim;
      const float L = head_l[h];
      store_out<T>(p, b, int64_t(kvh) * G + h, e - h * kHeadDim, L > 0.0f ? num[j] / L : 0.0f, head_m[h], L);
    }
  }
  if (tid == 0) p.counters[unit] = 0;  // ready for the next launch
}

// ---------------------------------------------------------------- host side
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess) {
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
    }
  });
  return fn;
}

size_t counters_bytes(int64_t units) { return size_t((units * sizeof(int) + 255) / 256 * 256); }

}  // namespace

int encode_codes_map(CUtensorMap* map, const uint8_t* kv_codes, int64_t num_pages, int64_t num_kv_heads) {
  auto fn = encode_fn();
  if (fn == nullptr) return fail(OQ_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
  const cuuint64_t dims[2] = {cuuint64_t(kRowBytes), cuuint64_t(num_pages * num_kv_heads * 2 * kPage)};
  const cuuint64_t strides[1] = {cuuint64_t(kRowBytes)};
  const cuuint32_t box[2] = {cuuint32_t(kRowBytes), cuuint32_t(2 * kPage)};
  const cuuint32_t estr[2] = {1, 1};
  CUresult res = fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<uint8_t*>(kv_codes), dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (res != CUDA_SUCCESS) return fail(OQ_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", int(res));
  return OQ_OK;
}

}  // namespace oq

extern "C" size_t oq_decode_attn_workspace_bytes(int64_t batch, int64_t num_heads, int64_t num_kv_heads,
                                                 int64_t head_dim, int64_t max_splits) {
  if (batch <= 0 || num_kv_heads <= 0 || num_heads <= 0 || head_dim <= 0 || max_splits <= 0) return 0;
  const int64_t units = batch * num_kv_heads;
  const int64_t group = num_heads / num_kv_heads;
  return oq::counters_bytes(units) + size_t(units * max_splits * group * (head_dim + 2) * sizeof(float));
}

extern "C" int oq_decode_attn_int4_paged(
    const void* query, int dtype, int64_t query_stride_b, int64_t query_stride_h,
    const uint8_t* kv_codes, const uint16_t* kv_meta, int64_t num_pages, int64_t page_size,
    const int32_t* block_table, int64_t block_table_stride, int64_t max_pages_per_seq,
    const int32_t* seq_lens,
    int64_t batch, int64_t num_heads, int64_t num_kv_heads, int64_t head_dim,
    float scaling,
    void* out, int64_t out_stride_b, int64_t out_stride_h,
    float* out_f32, float* out_lse,
    void* workspace, size_t workspace_bytes, int num_splits,
    int32_t* device_status, void* stream) {
  using namespace oq;
  if (dtype != OQ_BF16 && dtype != OQ_F16) {
    return fail(OQ_ERR_UNSUPPORTED, "decode_attn_int4_paged: query dtype must be bf16 or fp16");
  }
  if (head_dim != kHeadDim) return fail(OQ_ERR_UNSUPPORTED, "decode_attn_int4_paged: head_dim must be 256");
  if (page_size != kPage) return fail(OQ_ERR_UNSUPPORTED, "decode_attn_int4_paged: page_size must be 64");
  if (batch < 0 || num_kv_heads <= 0 || num_heads <= 0 || num_heads % num_kv_heads != 0 || num_pages <= 0 ||
      max_pages_per_seq <= 0 || block_table_stride < max_pages_per_seq) {
    return fail(OQ_ERR_INVALID_ARGUMENT, "decode_attn_int4_paged: bad sizes");
  }
  const int64_t group = num_heads / num_kv_heads;
  if (group > kMaxGroup) return fail(OQ_ERR_UNSUPPORTED, "decode_attn_int4_paged: more than 8 query heads per KV head");
  if (batch == 0) return ok();
  if (batch > 65535 || num_kv_heads > 65535) return fail(OQ_ERR_UNSUPPORTED, "decode_attn_int4_paged: grid too large");
  if (!query || !kv_codes || !kv_meta || !block_table || !seq_lens || (!out && !out_f32 && !out_lse)) {
    return fail(OQ_ERR_INVALID_ARGUMENT, "decode_attn_int4_paged: null pointer");
  }
  if (reinterpret_cast<uintptr_t>(query) % 16 || (query_stride_b * 2) % 16 || (query_stride_h * 2) % 16 ||
      reinterpret_cast<uintptr_t>(kv_codes) % 128 || reinterpret_cast<uintptr_t>(kv_meta) % 16) {
    return fail(OQ_ERR_MISALIGNED,
                "decode_attn_int4_paged: query rows need 16-byte alignment, kv_codes 128 bytes, kv_meta 16 bytes");
  }
  if (num_pages * num_kv_heads * 2 * kPage >= (int64_t(1) << 31)) {
    return fail(OQ_ERR_UNSUPPORTED, "decode_attn_int4_paged: page pool too large for 32-bit TMA rows");
  }

  // Split heuristic: enough CTAs for ~6 per SM of 148, at least one page each.
  const int64_t units = batch * num_kv_heads;
  int splits = num_splits;
  if (splits <= 0) {
    const int64_t target = 148 * 6;
    splits = int(std::min<int64_t>(std::max<int64_t>(1, (target + units - 1) / units), max_pages_per_seq));
  }
  // the merging CTA stages (max, sum) of every split in 64 KB of shared memory
  splits = int(std::min<int64_t>(std::min<int64_t>(splits, max_pages_per_seq), kMaxSplits));
  const int pps = int((max_pages_per_seq + splits - 1) / splits);
  splits = int((max_pages_per_seq + pps - 1) / pps);

  if (splits > 1 || workspace) {
    const size_t need = oq_decode_attn_workspace_bytes(batch, num_heads, num_kv_heads, head_dim, splits);
    if (splits > 1 && (workspace == nullptr || workspace_bytes < need)) {
      return fail(OQ_ERR_WORKSPACE, "decode_attn_int4_paged: workspace of %zu bytes needed for %d splits", need,
                  splits);
    }
  }
  const int64_t max_splits_ws =
      workspace ? std::max<int64_t>(1, (int64_t(workspace_bytes) - int64_t(counters_bytes(units))) /
                                           int64_t(units * group * (head_dim + 2) * sizeof(float)))
                : 1;

  CUtensorMap tmap;
  int st = encode_codes_map(&tmap, kv_codes, num_pages, num_kv_heads);
  if (st != OQ_OK) return st;

  AttnParams p;
  p.query = query;
  p.q_sb = query_stride_b;
  p.q_sh = query_stride_h;
  p.kv_meta = kv_meta;
  p.num_pages = num_pages;
  p.num_kv_heads = num_kv_heads;
  p.block_table = block_table;
  p.bt_stride = block_table_stride;
  p.max_pages = max_pages_per_seq;
  p.seq_lens = seq_lens;
  p.group = int(group);
  p.scale_log2 = scaling * 1.4426950408889634f;
  p.out = out;
  p.o_sb = out_stride_b;
  p.o_sh = out_stride_h;
  p.out_f32 = out_f32;
  p.out_lse = out_lse;
  p.counters = workspace ? static_cast<int*>(workspace) : nullptr;
  p.partials = workspace ? reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) + counters_bytes(units)) : nullptr;
  p.max_splits = int(std::min<int64_t>(max_splits_ws, 1 << 20));
  p.pages_per_split = pps;
  p.status = device_status;

  dim3 grid((unsigned)splits, (unsigned)num_kv_heads, (unsigned)batch);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (dtype == OQ_BF16) {
    cudaFuncSetAttribute(decode_attn_kernel<__nv_bfloat16>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         int(kSmemBytes));
    decode_attn_kernel<__nv_bfloat16><<<grid, kThreads, kSmemBytes, s>>>(tmap, p);
  } else {
    cudaFuncSetAttribute(decode_attn_kernel<__half>, cudaFuncAttributeMaxDynamicSharedMemorySize, int(kSmemBytes));
    decode_attn_kernel<__half><<<grid, kThreads, kSmemBytes, s>>>(tmap, p);
  }
  return check_launch("decode_attn_int4_paged");
}
