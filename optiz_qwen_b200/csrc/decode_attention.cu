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
//   * q.k runs on the integer tensor cores: q is per-head 21-bit fixed point split
//     into three 8-bit digits, the codes are u8 (nibbles masked in place, no shifts),
//     mma.sync m16n8k32 gives exact int32 dot products; p.v runs on fp16 tensor
//     cores with the nibbles as exact fp16 subnormals (masked in place);
//     scale/min are applied after the dot products:
//       q.k = scale * sum(q*code) + min * sum(q),  p.v = sum((p*scale)*code) + sum(p*min);
//   * the KV range is split across CTAs and the partial (max, sum, acc) are
//     merged by log-sum-exp by the last CTA of each (sequence, KV head).
#include <cudaTypedefs.h>

#include <algorithm>
#include <cmath>
#include <mutex>

#include "decode_attention.cuh"
#include "quant_row.cuh"

namespace oq {
namespace {

constexpr int kStages = 4;
constexpr int kWarps = 4;
constexpr int kThreads = kWarps * 32;

struct __align__(16) SmemTail {
  uint32_t qfrag[4][32][12];  // per k-step, per lane: B-operand digit fragments of up to 3 MMA sets
  uint64_t full[kStages];
  int stage_ok[kStages];
  float warp_m[kWarps][kMaxGroup];
  float warp_l[kWarps][kMaxGroup];
  float warp_f[kWarps][kMaxGroup];  // 2^(m_w - M) merge factor of each warp
  float head_m[kMaxGroup];
  float head_l[kMaxGroup];
  int is_last;
};

// Page formats: INT4 (two codes per byte, 16 KB of codes per page and KV head, 4 stages)
// and INT8 (one code per byte, 32 KB, 2 stages).  A CTA holds 3 warp groups of 4 warps,
// each with its own stage ring, barriers and share of the CTA's pages, one CTA per SM (the
// shared memory of the rings and the registers of 384 threads at up to 168 per thread).
// For INT8, 3 groups x 2 stages beat 2 groups x 3 stages (the same 6 pages in flight per
// SM, 12 warps instead of 8 to cover the page loop's latencies).
template <int kBits, int kGroups = 3>
struct PageFormat {
  static constexpr int kCodeBytes = 2 * kPage * kHeadDim * kBits / 8;
  static constexpr int kStagesN = kBits == 8 ? 2 : kStages;
  static constexpr int kWG = kGroups;
  // one warp group's region, 1024-aligned: stage codes | stage metas | tail
  static constexpr size_t kWgBytes =
      (size_t(kStagesN) * (kCodeBytes + kStageMetaBytes) + sizeof(SmemTail) + 1023) / 1024 * 1024;
  static constexpr size_t kSmem = 1024 /*alignment slack*/ + kWG * kWgBytes;
};

// ---- q.k on integer tensor cores.
// Each query head is turned into 21-bit fixed point, q ~ q_int * 2^-e_h with
// |q_int| <= 2^21 - 1, split into three 8-bit digits q_int = 16384 d2 + 128 d1 + d0
// (d2 signed, d1 and d0 in [0, 127]).  mma.sync m16n8k32 u8 x s8 -> s32 then gives
// exact integer dot products of the codes with each digit, combined in fp32.  With
// 21 bits every bf16 (fp16) element within 2^-13 (2^-10) of the head's largest is
// represented exactly, so q.k is as exact as fp32 arithmetic on the codes.  With at
// most 4 query heads per KV head two MMAs per 32 dims cover every head ("packed"): the
// columns of set 0 are (d2, d1) of heads 0, 1, 2, 3 in turn and those of set 1 (d0, 0),
// so the lane holding columns 2h, 2h+1 of both sets has all three digit products of head
// h and assembles its dot products without exchanging anything.  With 5-8 heads each
// digit takes one MMA ("dual": sets d2, d1, d0; columns = heads).  The fragments live in
// shared memory and are read per k-step.
//
// Code unpacking needs no shifts: w & 0x0F0F0F0F gives the even dims' codes as
// bytes, w & 0xF0F0F0F0 the odd dims' codes times 16; the two are accumulated
// in separate MMA chains and the second is divided by 16 (exactly) at the end.
constexpr uint32_t kLowNibbles = 0x0F0F0F0Fu;
constexpr uint32_t kHighNibbles = 0xF0F0F0F0u;
constexpr int kQMax = (1 << 21) - 1;

// q_int = 16384 d2 + 128 d1 + d0 with d2 in [-128, 127] and d1, d0 in [0, 127].
__device__ __forceinline__ void split_digits(int q, int& d2, int& d1, int& d0) {
  d2 = q >> 14;
  const int rem = q - (d2 << 14);
  d1 = rem >> 7;
  d0 = rem & 127;
}

// Dot products of the three digits combined: 16384 D2 + (128 D1 + D0), the last sum exact in
// int32 (|128 D1 + D0| < 2^31 for 256 dims of 8-bit codes), the whole rounded once to fp32.
__device__ __forceinline__ float combine_digits(int d2, int d1, int d0) {
  return fmaf(16384.0f, float(d2), float(128 * d1 + d0));
}

// ---- p.v on fp16 tensor cores.  prmt pairs byte b of two tokens' words into
// the two 16-bit lanes; masking then leaves a nibble as the mantissa of an fp16
// subnormal: mask 0x000F000F gives c * 2^-24 (even dim), mask 0x00F000F0 gives
// 16 c * 2^-24 (odd dim), both exact.  The tensor cores multiply these exactly by
// P' and accumulate in fp32 with no bias to remove afterwards (a 1024 + c encoding
// would cost the accumulator ~7 bits); the epilogue scales by 2^24 (2^20 for the
// odd dims), which is exact.
constexpr float kVCodeUnscale = 16777216.0f;  // 2^24
__device__ __forceinline__ uint32_t byte_pair_sel(int b) { return uint32_t(b) | (uint32_t(4 + b) << 8); }

// Lazy softmax rescale: the running max only moves when a tile's max exceeds it
// by more than kTau (log2 units), so p <= 2^kTau; P' = p * v_scale * 2^-kTau
// therefore stays inside the fp16 range whatever the stored fp16 scale.
constexpr float kTau = 4.0f;
// 2^x by the MUFU instruction (ex2.approx.ftz: ~2 ulp, results below 2^-126 flush to zero).  The
// page loop's p = 2^(s - m) lie in (0, 2^kTau]; one that flushes is < 2^-126 of the head's largest.
__device__ __forceinline__ float ex2_ftz(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
constexpr float kPScale = 0.0625f;  // 2^-kTau
constexpr float kPUnscale = 16.0f;

// Cross-warp reduction buffer: row (warp, head) of 256 dims, padded so that the
// 32 lanes' stores of one MMA tile fall in 32 different banks.
constexpr int kRedStride = 268;
__device__ __forceinline__ int red_index(int w, int h, int d) { return (w * kMaxGroup + h) * kRedStride + d + (d >> 5); }

// Shared-memory address of 16-byte chunk `chunk` of row `row` in a 128B-swizzled stage.
__device__ __forceinline__ const uint4* swz(const uint8_t* base, int row, int chunk) {
  return reinterpret_cast<const uint4*>(base + row * kRowBytes + ((chunk ^ (row & 7)) << 4));
}
// INT8 stage: each 256-byte row is two 128-byte lines (line = 2 row + chunk / 8), swizzled per line.
__device__ __forceinline__ const uint4* swz8(const uint8_t* base, int row, int chunk) {
  const int line = 2 * row + (chunk >> 3);
  return reinterpret_cast<const uint4*>(base + line * 128 + (((chunk & 7) ^ (line & 7)) << 4));
}

__device__ __forceinline__ uint32_t pack_s8x4(int a, int b, int c, int d) {
  return (uint32_t(a) & 0xFFu) | ((uint32_t(b) & 0xFFu) << 8) | ((uint32_t(c) & 0xFFu) << 16) |
         ((uint32_t(d) & 0xFFu) << 24);
}

template <typename T, bool kDual, int kBits, int kGroups>
__global__ void __launch_bounds__(kGroups * kThreads, kGroups == 3 ? 1 : 3)
    decode_attn_kernel(const __grid_constant__ CUtensorMap tmap, AttnParams p) {
  using PF = PageFormat<kBits, kGroups>;
  constexpr int kSt = PF::kStagesN;
  constexpr int kCB = PF::kCodeBytes;
  constexpr int kWG = PF::kWG;
  constexpr int kNT = kWG * kThreads;  // threads of the CTA
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  // Warp group wg runs the page loop below on its own region; `tid`, `warp` and every
  // barrier of the loop are local to the group (named barrier 1 + wg over its 128 threads).
  const int ctid = threadIdx.x;
  const int wg = ctid / kThreads;
  const int bar_wg = 1 + wg;
  uint8_t* codes = smem + wg * PF::kWgBytes;  // kSt x kCB bytes, 1024-aligned
  uint8_t* metas = codes + kSt * kCB;                           // kSt x 512 B
  SmemTail* tail = reinterpret_cast<SmemTail*>(metas + kSt * kStageMetaBytes);
  auto tail_of = [&](int g) {
    return reinterpret_cast<SmemTail*>(smem + g * PF::kWgBytes + kSt * (kCB + kStageMetaBytes));
  };

  const int tid = ctid - wg * kThreads;
  const int lane = tid & 31;
  if (tid == 0) prefetch_tensormap(&tmap);  // the first copies are issued in a few microseconds
  const int warp = tid >> 5;
  const int r = lane >> 2;  // mma groupID
  const int c = lane & 3;   // mma thread-in-group
  const int split = blockIdx.x;
  const int kvh = blockIdx.y;
  const int64_t b = blockIdx.z;
  const int G = p.group;

  // ---- every independent global load of the prologue is issued first, so their latencies
  // overlap.  Group wg takes pages cta_begin + wg + kWG * i of the CTA's range (round robin,
  // so the groups' shares differ by at most one page), which makes the page ids of its first
  // kSt pages known before the sequence length is: they go out with the length and the 64
  // query elements this lane needs.
  constexpr int kSets = kDual ? 3 : 2;  // MMA column sets of the q digits (see split_digits)
  const int cta_begin = split * p.pages_per_split;
  auto page_at = [&](int i) { return cta_begin + wg + kWG * i; };  // sequence page of this group's page i
  const int32_t* bt_row = p.block_table + b * p.bt_stride;
  const bool pre_ok = warp == 0 && lane < kSt && int64_t(page_at(lane)) < p.max_pages;
  // This lane feeds q.k MMA column r: (packed) head r >> 1, digits d2 / d0 for even r and d1
  // for odd r; (dual) head r, every digit.  It holds dims 64c .. 64c+63 of that head, so the
  // four lanes (r, 0..3) hold the whole head.
  const int f_head = kDual ? r : (r >> 1);
  const bool f_has = f_head < G;
  uint4 qv[8];
  auto load_q = [&]() {
    const T* qrow = static_cast<const T*>(p.query) + b * p.q_sb + int64_t(kvh * G + (f_has ? f_head : 0)) * p.q_sh +
                    64 * c;
#pragma unroll
    for (int i = 0; i < 8; ++i) qv[i] = f_has ? __ldg(reinterpret_cast<const uint4*>(qrow + 8 * i)) : make_uint4(0, 0, 0, 0);
  };
  // Early launch (p.early): this CTA may run while the kernel ahead of it in the stream still
  // does, which by the caller's contract writes neither the cache, the block table nor
  // seq_lens.  Everything up to the first page copies then happens before the dependency wait;
  // the query, the appended token and every write come after it.  A plain launch waits first
  // (a no-op) and loads the query with the lengths.  (One long wave: the successor is allowed
  // to launch only after the page loop.)
  if (!p.early) {
    pdl_wait();
    load_q();
  }
  const int32_t len_raw = p.seq_lens[b];
  const int first_pre = pre_ok ? bt_row[page_at(lane)] : -1;
  if (tid == 0) {
    for (int s2 = 0; s2 < kSt; ++s2) mbar_init(&tail->full[s2], 1);
    fence_mbar_init();
  }

  // With an appended token (p.append) the sequence holds len_raw + 1 tokens: the new one, at
  // position len_raw of logical page lp_new, is quantised into the cache by this launch (warps 0
  // and 1 of the group that owns that page) before any copy of that page is issued.
  const int len = max(len_raw, 0) + (p.append ? 1 : 0);
  const int len_pages = (len + kPage - 1) / kPage;
  const int npages_b = int(min(int64_t(len_pages), p.max_pages));
  const int nsplit_b = max(1, (npages_b + p.pages_per_split - 1) / p.pages_per_split);
  if (split >= nsplit_b) {
    pdl_allow_next();
    return;
  }
  const bool overflow = len_pages > p.max_pages;
  const int cta_n = max(0, min(npages_b, cta_begin + p.pages_per_split) - cta_begin);
  // this group's share of the CTA's pages (an empty share is fine: m = -inf, l = 0)
  const int n = cta_n > wg ? (cta_n - wg + kWG - 1) / kWG : 0;
  const int lp_new = p.append ? (len - 1) / kPage : -1;
  const int rel_new = lp_new - cta_begin;
  // this group's index of the appended token's page, or -1
  const int i_new = (p.append && lp_new < npages_b && rel_new >= 0 && rel_new < cta_n && rel_new % kWG == wg)
                        ? rel_new / kWG : -1;
  const int pid_new = (i_new >= 0 && warp < 2) ? bt_row[lp_new] : -1;
  const int first_page = (warp == 0 && lane < min(n, kSt) && lane != i_new) ? first_pre : -1;
  // thread 0 loads the page id of the page it issues next one loop iteration ahead
  int next_pid = (tid == 0 && kSt < n) ? bt_row[page_at(kSt)] : 0;

  auto issue = [&](int i, int s, int64_t page) {
    if (page < 0 || page >= p.num_pages) {
      tail->stage_ok[s] = 0;
      report(p.status, OQ_DEV_BAD_PAGE);
      mbar_arrive(&tail->full[s]);
      return;
    }
    tail->stage_ok[s] = 1;
    const int64_t blk = page * p.num_kv_heads + kvh;
    mbar_arrive_expect_tx(&tail->full[s], kCB + kStageMetaBytes);
    if constexpr (kBits == 8) {  // box {128 B, 2 halves, 128 rows}
      tma_load_3d(codes + s * kCB, &tmap, 0, 0, int32_t(blk * 2 * kPage), &tail->full[s]);
    } else {
      tma_load_2d(codes + s * kCB, &tmap, 0, int32_t(blk * 2 * kPage), &tail->full[s]);
    }
    bulk_load(metas + s * kStageMetaBytes, p.kv_meta + blk * 4 * kPage, kStageMetaBytes, &tail->full[s]);
  };
  // warp 0: the first copies (thread 0 initialised the barriers above; the other threads
  // first wait on them after the group barrier at the end of the prologue)
  int issued = 0;
  if (warp == 0) {
#pragma unroll
    for (int i = 0; i < kSt; ++i) {
      const int page = __shfl_sync(0xffffffffu, first_page, i);
      if (lane == 0 && i < n && i != i_new) issue(i, i, page);  // (the appended token's page: below)
    }
    issued = min(n, kSt);
  }
  if (p.early) {
    pdl_wait();
    load_q();
  }
  if (overflow && ctid == 0 && split == 0) report(p.status, OQ_DEV_OVERFLOW);
  if (i_new >= 0 && warp < 2) {
    // the appended token: warp 0 quantises its K row, warp 1 its V row, into page pid_new
    if (pid_new < 0 || pid_new >= p.num_pages) {
      if (lane == 0) report(p.status, OQ_DEV_BAD_PAGE);
    } else {
      const int slot = (len - 1) - lp_new * kPage;
      const int64_t blk = int64_t(pid_new) * p.num_kv_heads + kvh;
      const T* src = static_cast<const T*>(warp == 0 ? p.new_k : p.new_v) + b * (warp == 0 ? p.nk_sb : p.nv_sb) +
                     int64_t(kvh) * (warp == 0 ? p.nk_sh : p.nv_sh);
      quantize_row<T, kHeadDim / 32, true, kBits>(src, lane, p.kv_codes + ((blk * 2 + warp) * kPage + slot) *
                                                                               (kHeadDim * kBits / 8),
                                                  p.kv_meta_w + (blk * 4 + 2 * warp) * kPage + slot, kPage);
      asm volatile("fence.proxy.async.global;\n" ::: "memory");  // the page copy below reads these bytes
    }
  }

  // ---- query digits (B operand of q.k).
  // Per head: 21-bit fixed point with exponent e (2^e <= kQMax / max|q|), from the
  // largest element of the head (the four lanes of the head reduce by shuffles), and
  // sum(q).  k-step s covers dims 64c + 16s + {0..15}: the even dims in the "low
  // nibble" MMA, the odd dims in the "high nibble" MMA.  INT8: the same 16 dims feed
  // two MMAs, 2s (dims 64c + 16s + 0..7) and 2s + 1 (+ 8..15), each taking 4 dims per
  // word: words (b0, b1) of MMA 2s, then of MMA 2s + 1.
  float amax = 0.0f, qsum = 0.0f;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const T* e = reinterpret_cast<const T*>(&qv[i]);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float v = to_float<T>(e[j]);
      amax = fmaxf(amax, fabsf(v));
      qsum += v;
    }
  }
  amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
  amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
  qsum += __shfl_xor_sync(0xffffffffu, qsum, 1);
  qsum += __shfl_xor_sync(0xffffffffu, qsum, 2);
  int q_exp = 0;
  if (amax > 0.0f) {
    frexpf(float(kQMax) / fmaxf(amax, 1e-30f), &q_exp);  // kQMax / amax = f * 2^e, f in [0.5, 1)
    q_exp -= 1;                                           // 2^e <= kQMax / amax
  }
  const float q_scale = ldexpf(1.0f, -q_exp);
  // warp w builds k-step w for all 32 lanes; the fragments are exchanged in shared memory
  // as words [set][nibble MMA (lo, hi)][b0, b1] per (k-step, lane)
  {
    const float up = f_has ? ldexpf(1.0f, q_exp) : 0.0f;
    uint4 qw[2] = {qv[0], qv[1]};  // the 16 dims of k-step `warp` (selected with constant indices)
#pragma unroll
    for (int w = 1; w < 4; ++w) {
      if (warp == w) {
        qw[0] = qv[2 * w];
        qw[1] = qv[2 * w + 1];
      }
    }
    uint32_t* dst = tail->qfrag[warp][lane];
#pragma unroll
    for (int half = 0; half < 2; ++half) {  // word 2s (b0) and word 2s+1 (b1) of the step
      const T* e = reinterpret_cast<const T*>(&qw[half]);
      int de[3][4], dodd[3][4];  // digit 2, 1, 0 -> [0], [1], [2] of the even / odd dims
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int q_e = max(-kQMax, min(kQMax, __float2int_rn(to_float<T>(e[2 * j]) * up)));
        const int q_o = max(-kQMax, min(kQMax, __float2int_rn(to_float<T>(e[2 * j + 1]) * up)));
        split_digits(q_e, de[0][j], de[1][j], de[2][j]);
        split_digits(q_o, dodd[0][j], dodd[1][j], dodd[2][j]);
      }
      uint32_t wa[3], wb[3];  // per digit: the lo-nibble and hi-nibble MMA words of this half
#pragma unroll
      for (int d = 0; d < 3; ++d) {
        if constexpr (kBits == 8) {  // a: dims +0..3 (b0), b: dims +4..7 (b1) of MMA 2w + half
          wa[d] = pack_s8x4(de[d][0], dodd[d][0], de[d][1], dodd[d][1]);
          wb[d] = pack_s8x4(de[d][2], dodd[d][2], de[d][3], dodd[d][3]);
        } else {
          wa[d] = pack_s8x4(de[d][0], de[d][1], de[d][2], de[d][3]);
          wb[d] = pack_s8x4(dodd[d][0], dodd[d][1], dodd[d][2], dodd[d][3]);
        }
      }
      if constexpr (kDual) {
#pragma unroll
        for (int k = 0; k < kSets; ++k) {  // set k = digit 2 - k of head r
          dst[4 * k + half] = wa[k];
          dst[4 * k + 2 + half] = wb[k];
        }
      } else {  // column r of head r >> 1: set 0 = d2 (even r) | d1 (odd r); set 1 = d0 (even r) | 0
        const bool odd = r & 1;
        dst[half] = odd ? wa[1] : wa[0];
        dst[2 + half] = odd ? wb[1] : wb[0];
        dst[4 + half] = odd ? 0u : wa[2];
        dst[6 + half] = odd ? 0u : wb[2];
      }
    }
  }
  named_bar_sync(bar_wg, kThreads);  // fragments written; the stage barriers are initialised
  // Packed layout (<= 4 query heads per KV head): this lane's fragments of all four k-steps
  // stay in registers (32 words) instead of being read from shared memory for every page
  // (B = 64, context 4096: 41.0 -> 39.5 us per INT4 launch, and the register spill of that
  // instance is gone; one-group CTAs at B = 384: 191 -> 187 us; INT8: 48.7 -> 48.3 us)
  constexpr bool kQReg = !kDual;
  uint4 qreg[4][2];
  if constexpr (kQReg) {
#pragma unroll
    for (int st4 = 0; st4 < 4; ++st4) {
#pragma unroll
      for (int k = 0; k < 2; ++k) qreg[st4][k] = reinterpret_cast<const uint4*>(tail->qfrag[st4][lane])[k];
    }
  }
  // the appended token's page, now that warps 0 and 1 have written its new row
  if (tid == 0 && i_new >= 0 && i_new < kSt) issue(i_new, i_new, pid_new);
  // Heads of this lane's scores: (packed) head c, from columns 2c (d2 / d0) and 2c+1 (d1);
  // (dual) heads 2c and 2c+1.  Lane 8c (r = 2c) holds sum(q) and 2^-e of head c (packed) or
  // 2c (dual), lane 8c + 4 those of head 2c + 1 (dual).
  constexpr int kNH = kDual ? 2 : 1;
  const int h0 = kDual ? 2 * c : c;
  float qs[kNH], qx[kNH];
  bool h_ok[kNH];
#pragma unroll
  for (int e = 0; e < kNH; ++e) {
    qs[e] = __shfl_sync(0xffffffffu, qsum, 8 * c + 4 * e);
    qx[e] = __shfl_sync(0xffffffffu, q_scale, 8 * c + 4 * e);
    h_ok[e] = h0 + e < G;
  }
  // The digit products of this lane's accumulators -> its q_int . codes, dot[tok][e] for tokens
  // r, r + 8 (accumulator rows) and heads h0 + e.
  auto digit_dots = [&](const int (&tot)[kSets][4], float (&dot)[2][kNH]) {
#pragma unroll
    for (int t = 0; t < 2; ++t) {
      if constexpr (kDual) {
#pragma unroll
        for (int e = 0; e < 2; ++e) dot[t][e] = combine_digits(tot[0][2 * t + e], tot[1][2 * t + e], tot[2][2 * t + e]);
      } else {
        dot[t][0] = combine_digits(tot[0][2 * t], tot[0][2 * t + 1], tot[1][2 * t]);
      }
    }
  };

  float acc[16][4];
#pragma unroll
  for (int j = 0; j < 16; ++j) acc[j][0] = acc[j][1] = acc[j][2] = acc[j][3] = 0.0f;
  float m[kNH], l[kNH], mp[kNH];  // per head: reference max (log2 units); this lane's sum(p), sum(p v_min)
#pragma unroll
  for (int e = 0; e < kNH; ++e) {
    m[e] = -INFINITY;
    l[e] = 0.0f;
    mp[e] = 0.0f;
  }

  const int tok0 = warp * 16 + r;  // token rows of this lane in the page (A rows r and r+8)
  const int tok1 = tok0 + 8;
  bool aborted = false;

  // p.v of one page: acc += V^T P' with the V codes of stage `stv` and P' (B operand) pv0, pv1
  auto pv_page = [&](const uint8_t* stv, uint32_t pv0, uint32_t pv1) {
    const int tb = warp * 16 + kPage;  // V rows follow the 64 K rows
    // ---------------- values: A = V^T codes (16 dims x 16 tokens), B = P' (16 tokens x 8 heads)
    if constexpr (kBits == 8) {
      // half hf, lane r: 16-byte chunk 8 hf + r of the four token rows; MMA 8 hf + k has
      // row r = dim 128 hf + 16 r + 2k, row r + 8 = that dim + 1, each code as the fp16
      // subnormal c * 2^-24 (the byte under a zero high byte)
#pragma unroll
      for (int hf = 0; hf < 2; ++hf) {
        const uint4 xa = *swz8(stv, tb + 2 * c, 8 * hf + r), xb = *swz8(stv, tb + 2 * c + 1, 8 * hf + r);
        const uint4 xc = *swz8(stv, tb + 2 * c + 8, 8 * hf + r), xd = *swz8(stv, tb + 2 * c + 9, 8 * hf + r);
        const uint32_t wa[4] = {xa.x, xa.y, xa.z, xa.w}, wb[4] = {xb.x, xb.y, xb.z, xb.w};
        const uint32_t wc[4] = {xc.x, xc.y, xc.z, xc.w}, wd[4] = {xd.x, xd.y, xd.z, xd.w};
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          const uint32_t pb = 2u * uint32_t(k & 1);  // bytes pb, pb + 1 of word k / 2
          const uint32_t sel = pb | ((4u + pb) << 4) | ((pb + 1u) << 8) | ((5u + pb) << 12);
          const uint32_t x = prmt(wa[k >> 1], wb[k >> 1], sel);  // tokens 2c, 2c+1: dims 2k, 2k+1 of the chunk
          const uint32_t y = prmt(wc[k >> 1], wd[k >> 1], sel);  // tokens 2c+8, 2c+9
          uint32_t a[4];
          a[0] = prmt(x, 0u, 0x4140u);  // row r: dim 2k, c * 2^-24
          a[1] = prmt(x, 0u, 0x4342u);  // row r+8: dim 2k + 1
          a[2] = prmt(y, 0u, 0x4140u);
          a[3] = prmt(y, 0u, 0x4342u);
          mma_f16_16816(acc[8 * hf + k], a, pv0, pv1);
        }
      }
    } else {
      const uint4 va = *swz(stv, tb + 2 * c, r), vb = *swz(stv, tb + 2 * c + 1, r);
      const uint4 vc = *swz(stv, tb + 2 * c + 8, r), vd = *swz(stv, tb + 2 * c + 9, r);
      const uint32_t wa[4] = {va.x, va.y, va.z, va.w}, wb[4] = {vb.x, vb.y, vb.z, vb.w};
      const uint32_t wc[4] = {vc.x, vc.y, vc.z, vc.w}, wd[4] = {vd.x, vd.y, vd.z, vd.w};
#pragma unroll
      for (int wi = 0; wi < 4; ++wi) {
#pragma unroll
        for (int bs = 0; bs < 4; ++bs) {
          const uint32_t x = prmt(wa[wi], wb[wi], byte_pair_sel(bs));  // tokens 2c, 2c+1: dims 2bs, 2bs+1
          const uint32_t y = prmt(wc[wi], wd[wi], byte_pair_sel(bs));  // tokens 2c+8, 2c+9
          uint32_t a[4];
          a[0] = x & 0x000F000Fu;  // row r: even dim, c * 2^-24
          a[1] = x & 0x00F000F0u;  // row r+8: odd dim, 16 c * 2^-24
          a[2] = y & 0x000F000Fu;
          a[3] = y & 0x00F000F0u;
          mma_f16_16816(acc[4 * wi + bs], a, pv0, pv1);
        }
      }
    }
    
  };

  // Page i: q.k, softmax and p.v; then the stage is refilled with page i + kSt.  (Running
  // the p.v of page i - 1 in the same block as the q.k of page i was measured: no faster.)
  for (int i = 0; i < n; ++i) {
    const int s = i % kSt;
    bool ready = wait_stage(&tail->full[s], (i / kSt) & 1, p.wait_polls);
    ready = __all_sync(0xffffffffu, ready);
    // tokens of page i (0 when its copy failed: every score is masked)
    const int page_tokens = (ready && tail->stage_ok[s]) ? min(kPage, len - page_at(i) * kPage) : 0;
    if (warp * 16 < page_tokens) {
      const uint8_t* st = codes + s * kCB;
      const __half* meta = reinterpret_cast<const __half*>(metas + s * kStageMetaBytes);

      // ---------------- integer q.k: A = K codes (16 tokens x 32 dims, u8), B = q digits (s8)
      float dot[2][kNH];  // q_int . codes of (token r / r + 8, head h0 + e)
      if constexpr (kBits == 8) {
        // lane c holds dims 64c .. 64c + 63 of both token rows (16 words each); MMA "lo" of
        // step s takes words 4s (b0 dims) and 4s + 2, MMA "hi" words 4s + 1 and 4s + 3,
        // both into one accumulator (codes are whole bytes)
        uint32_t w0[16], w1[16];
#pragma unroll
        for (int q4 = 0; q4 < 4; ++q4) {
          const uint4 x0 = *swz8(st, tok0, 4 * c + q4), x1 = *swz8(st, tok1, 4 * c + q4);
          w0[4 * q4] = x0.x; w0[4 * q4 + 1] = x0.y; w0[4 * q4 + 2] = x0.z; w0[4 * q4 + 3] = x0.w;
          w1[4 * q4] = x1.x; w1[4 * q4 + 1] = x1.y; w1[4 * q4 + 2] = x1.z; w1[4 * q4 + 3] = x1.w;
        }
        int tot[kSets][4];
#pragma unroll
        for (int k = 0; k < kSets; ++k) {
#pragma unroll
          for (int j = 0; j < 4; ++j) tot[k][j] = 0;
        }
#pragma unroll
        for (int st4 = 0; st4 < 4; ++st4) {
          const uint32_t al[4] = {w0[4 * st4], w1[4 * st4], w0[4 * st4 + 2], w1[4 * st4 + 2]};
          const uint32_t ah[4] = {w0[4 * st4 + 1], w1[4 * st4 + 1], w0[4 * st4 + 3], w1[4 * st4 + 3]};
          const uint4* qf = reinterpret_cast<const uint4*>(tail->qfrag[st4][lane]);
#pragma unroll
          for (int k = 0; k < kSets; ++k) {
            const uint4 f = kQReg ? qreg[st4][k] : qf[k];
            imma_u8s8_16832(tot[k], al, f.x, f.y);
            imma_u8s8_16832(tot[k], ah, f.z, f.w);
          }
        }
        digit_dots(tot, dot);
      } else {
        const uint4 k00 = *swz(st, tok0, 2 * c), k01 = *swz(st, tok0, 2 * c + 1);
        const uint4 k10 = *swz(st, tok1, 2 * c), k11 = *swz(st, tok1, 2 * c + 1);
        const uint32_t w0[8] = {k00.x, k00.y, k00.z, k00.w, k01.x, k01.y, k01.z, k01.w};
        const uint32_t w1[8] = {k10.x, k10.y, k10.z, k10.w, k11.x, k11.y, k11.z, k11.w};
        int lo[kSets][4], hi[kSets][4];
#pragma unroll
        for (int k = 0; k < kSets; ++k) {
#pragma unroll
          for (int j = 0; j < 4; ++j) lo[k][j] = hi[k][j] = 0;
        }
#pragma unroll
        for (int st4 = 0; st4 < 4; ++st4) {
          const uint32_t al[4] = {w0[2 * st4] & kLowNibbles, w1[2 * st4] & kLowNibbles,
                                  w0[2 * st4 + 1] & kLowNibbles, w1[2 * st4 + 1] & kLowNibbles};
          const uint32_t ah[4] = {w0[2 * st4] & kHighNibbles, w1[2 * st4] & kHighNibbles,
                                  w0[2 * st4 + 1] & kHighNibbles, w1[2 * st4 + 1] & kHighNibbles};
          const uint4* qf = reinterpret_cast<const uint4*>(tail->qfrag[st4][lane]);
#pragma unroll
          for (int k = 0; k < kSets; ++k) {
            const uint4 f = kQReg ? qreg[st4][k] : qf[k];
            imma_u8s8_16832(lo[k], al, f.x, f.y);
            imma_u8s8_16832(hi[k], ah, f.z, f.w);
          }
        }
        int tot[kSets][4];
#pragma unroll
        for (int k = 0; k < kSets; ++k) {
#pragma unroll
          for (int j = 0; j < 4; ++j) tot[k][j] = lo[k][j] + (hi[k][j] >> 4);  // (hi is a multiple of 16)
        }
        digit_dots(tot, dot);
      }
      const bool tv[2] = {tok0 < page_tokens, tok1 < page_tokens};
      const int tk[2] = {tok0, tok1};
      float vs[2], vm[2], sc[2][kNH];
#pragma unroll
      for (int t = 0; t < 2; ++t) {
        const float ks = __half2float(meta[tk[t]]), km = __half2float(meta[kPage + tk[t]]);
        vs[t] = __half2float(meta[2 * kPage + tk[t]]);
        vm[t] = __half2float(meta[3 * kPage + tk[t]]);
        // q.k = scale * 2^-e * sum(code * q_int) + min * sum(q), in log2 units
#pragma unroll
        for (int e = 0; e < kNH; ++e) {
          sc[t][e] = tv[t] && h_ok[e] ? fmaf(ks * qx[e], dot[t][e], km * qs[e]) * p.scale_log2 : -INFINITY;
        }
      }

      // ---------------- online softmax with a lazily moved reference max
      float tm[kNH];
      bool move = false;
#pragma unroll
      for (int e = 0; e < kNH; ++e) {
        tm[e] = fmaxf(sc[0][e], sc[1][e]);
#pragma unroll
        for (int o = 4; o < 32; o <<= 1) tm[e] = fmaxf(tm[e], __shfl_xor_sync(0xffffffffu, tm[e], o));
        move = move || tm[e] > m[e] + kTau;
      }
      if (__any_sync(0xffffffffu, move)) {
        float corr[kNH];
#pragma unroll
        for (int e = 0; e < kNH; ++e) {
          const float nm = fmaxf(m[e], tm[e]);
          corr[e] = nm == -INFINITY ? 1.0f : exp2f(m[e] - nm);
          m[e] = nm;
          l[e] *= corr[e];
          mp[e] *= corr[e];
        }
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          if constexpr (kDual) {  // columns 2c, 2c+1 = heads h0, h0 + 1
            acc[j][0] *= corr[0];
            acc[j][2] *= corr[0];
            acc[j][1] *= corr[kNH - 1];
            acc[j][3] *= corr[kNH - 1];
          } else {  // columns 2c, 2c+1 = the fp16 part and the remainder of head c
#pragma unroll
            for (int q4 = 0; q4 < 4; ++q4) acc[j][q4] *= corr[0];
          }
        }
      }
      float pp[2][kNH];
#pragma unroll
      for (int t = 0; t < 2; ++t) {
#pragma unroll
        for (int e = 0; e < kNH; ++e) {
          pp[t][e] = tv[t] && h_ok[e] ? ex2_ftz(sc[t][e] - m[e]) : 0.0f;
          l[e] += pp[t][e];
          mp[e] = fmaf(pp[t][e], tv[t] ? vm[t] : 0.0f, mp[e]);
        }
      }
      // P' = p * v_scale * 2^-kTau, rows = tokens.  Packed: columns 2c, 2c+1 = P' rounded to fp16
      // and its fp16 remainder (P' to ~22 bits); dual: columns = heads 2c, 2c+1 in fp16.
      uint32_t blk[2];
#pragma unroll
      for (int t = 0; t < 2; ++t) {
        const float ps = tv[t] ? vs[t] * kPScale : 0.0f;
        if constexpr (kDual) {
          blk[t] = pack_half2(pp[t][0] * ps, pp[t][kNH - 1] * ps);
        } else {
          const float x = pp[t][0] * ps;
          const float hi = __half2float(__float2half_rn(x));
          blk[t] = pack_half2(hi, x - hi);
        }
      }
      const uint32_t blk0 = blk[0], blk1 = blk[1];
      // transpose into the B operand of p.v
      pv_page(st, movmatrix_trans(blk0), movmatrix_trans(blk1));
    }
    const bool stop = named_bar_or(bar_wg, kThreads, !ready);
    if (stop) {
      aborted = true;
      break;
    }
    if (tid == 0 && i + kSt < n) {
      const int nxt = i + kSt;
      issue(nxt, s, next_pid);
      ++issued;
      if (nxt + 1 < n) next_pid = bt_row[page_at(nxt + 1)];
    }
  }

  pdl_allow_next();
  bool drained = true;
  if (aborted && tid == 0) {
    // A wait gave up.  The pages issued from this group's last refill on, [issued - kSt,
    // issued), are still unconsumed; let every one of them land (bounded, at the default
    // limit) before this shared memory is reused below or released at exit.  The
    // group's sums cover the pages it finished; the status word marks the result.
    report(p.status, OQ_DEV_TIMEOUT);
    for (int i = max(0, issued - kSt); i < issued; ++i) {
      drained = wait_stage(&tail->full[i % kSt], (i / kSt) & 1, kDefaultWaitPolls) && drained;
    }
  }
  // The groups finish their page loops at different times; from here on the whole CTA
  // works together (every stage of every group has been consumed).
  if (__syncthreads_or(!drained)) {
    // a copy never landed: shared memory may still be written, so the CTA leaves without
    // using it, keeping the merge counter consistent for the next launch
    if (ctid == 0 && nsplit_b > 1 && !p.defer_merge) merge_arrive_only(p, b * p.num_kv_heads + kvh, nsplit_b);
    return;
  }

  // ---- reduce this warp's per-lane sums over the 8 token rows
#pragma unroll
  for (int o = 4; o < 32; o <<= 1) {
#pragma unroll
    for (int e = 0; e < kNH; ++e) {
      l[e] += __shfl_xor_sync(0xffffffffu, l[e], o);
      mp[e] += __shfl_xor_sync(0xffffffffu, mp[e], o);
    }
  }
  if (r == 0) {
#pragma unroll
    for (int e = 0; e < kNH; ++e) {
      if (h_ok[e]) {
        tail->warp_m[warp][h0 + e] = m[e];
        tail->warp_l[warp][h0 + e] = l[e];
      }
    }
  }
  const int outputs = G * kHeadDim;
  const bool single = nsplit_b == 1 && p.xr.world == 0;  // (an exchange always goes through the merge kernel)
  __syncthreads();

  // per head, over every warp of every group: M = the largest reference max, L = the sums at
  // M, and each warp's factor 2^(m_w - M)
  if (ctid < G) {
    float M = -INFINITY;
#pragma unroll
    for (int g = 0; g < kWG; ++g) {
      for (int w = 0; w < kWarps; ++w) M = fmaxf(M, tail_of(g)->warp_m[w][ctid]);
    }
    float L = 0.0f;
#pragma unroll
    for (int g = 0; g < kWG; ++g) {
      SmemTail* tg = tail_of(g);
      for (int w = 0; w < kWarps; ++w) {
        const float f = M == -INFINITY ? 0.0f : exp2f(tg->warp_m[w][ctid] - M);
        tg->warp_f[w][ctid] = f;
        L = fmaf(tg->warp_l[w][ctid], f, L);
      }
    }
    tail_of(0)->head_m[ctid] = M;
    tail_of(0)->head_l[ctid] = L;
  }
  __syncthreads();

  // ---- each warp's numerators at the common max: red[w][h][d] = numerator_w * 2^(m_w - M),
  //      numerator = 2^kTau * 2^24 * acc / (1 or 16) + sum(p * v_min)
  float* red = reinterpret_cast<float*>(codes);  // this group's kWarps * kMaxGroup rows of kRedStride floats
  {
    float f[kNH];
#pragma unroll
    for (int e = 0; e < kNH; ++e) f[e] = h_ok[e] ? tail->warp_f[warp][h0 + e] : 0.0f;
    // INT4: row r = even dim 32r + 2j (codes x 1), row r + 8 = odd dim (codes x 16);
    // INT8: MMA j = 8 hf + k, row r = dim 128 hf + 16r + 2k, row r + 8 = the next dim (x 1)
    constexpr float kEvenUnscale = kPUnscale * kVCodeUnscale;
    constexpr float kOddUnscale = kBits == 8 ? kEvenUnscale : kEvenUnscale / 16.0f;
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const int d0 = kBits == 8 ? 128 * (j >> 3) + 16 * r + 2 * (j & 7) : 32 * r + 2 * j;
      // per head of this lane: the even-row (d0) and odd-row (d0 + 1) sums; packed: the fp16
      // part (column 2c) plus the remainder (column 2c + 1) of head c
      float ev[kNH], od[kNH];
      if constexpr (kDual) {
        ev[0] = acc[j][0];
        od[0] = acc[j][2];
        ev[kNH - 1] = acc[j][1];
        od[kNH - 1] = acc[j][3];
      } else {
        ev[0] = acc[j][0] + acc[j][1];
        od[0] = acc[j][2] + acc[j][3];
      }
#pragma unroll
      for (int e = 0; e < kNH; ++e) {
        if (h_ok[e]) {
          red[red_index(warp, h0 + e, d0)] = fmaf(ev[e], kEvenUnscale, mp[e]) * f[e];
          red[red_index(warp, h0 + e, d0 + 1)] = fmaf(od[e], kOddUnscale, mp[e]) * f[e];
        }
      }
    }
  }
  // this thread's outputs are e = ctid + j * kNT; their gate elements go out before the barrier
  constexpr int kPerThread = (kMaxGroup * kHeadDim + kNT - 1) / kNT;
  float gv[kPerThread];
#pragma unroll
  for (int j = 0; j < kPerThread; ++j) {
    const int e = ctid + j * kNT;
    gv[j] = single && e < outputs ? gate_value<T>(p, b, int64_t(kvh) * G + e / kHeadDim, e % kHeadDim) : 0.0f;
  }
  __syncthreads();

  // ---- sum the warps of every group: the CTA's output (one split) or its partial record
  const int64_t unit = b * p.num_kv_heads + kvh;
  const int rec_floats = G * (kHeadDim + 2);
  float* my_rec = p.partials + (unit * p.max_splits + split) * rec_floats;
#pragma unroll
  for (int j = 0; j < kPerThread; ++j) {
    const int e = ctid + j * kNT;
    if (e < outputs) {
      const int h = e / kHeadDim;
      const int d = e - h * kHeadDim;
      float num = 0.0f;
#pragma unroll
      for (int g = 0; g < kWG; ++g) {
        const float* rg = reinterpret_cast<const float*>(smem + g * PF::kWgBytes);
#pragma unroll
        for (int w = 0; w < kWarps; ++w) num += rg[red_index(w, h, d)];
      }
      const float M = tail_of(0)->head_m[h], L = tail_of(0)->head_l[h];
      if (single) {
        store_out_g<T>(p, b, int64_t(kvh) * G + h, d, L > 0.0f ? num / L : 0.0f, M, L, gv[j]);
      } else {
        my_rec[e] = num;
        if (d == 0) {
          my_rec[outputs + h] = M;
          my_rec[outputs + G + h] = L;
        }
      }
    }
  }
  if (single || p.defer_merge) return;

  // ---- split-KV merge by the last CTA of this (sequence, KV head); its scratch is group
  // 0's reduction buffer, free once every thread is past the loop above (the helper's first
  // barrier)
  merge_splits_last_cta<T, kNT>(p, b, kvh, nsplit_b, ctid, reinterpret_cast<float*>(smem), &tail_of(0)->is_last,
                                1 + kWG);
}

// ---- split-KV merge for many splits: one CTA per (sequence x KV head, query head),
// one thread per output dim; the (max, sum) of every split are staged in shared
// memory and each thread reduces its dim over the splits with coalesced loads.
constexpr int kMergeThreads = kHeadDim;

template <typename T>
__global__ void __launch_bounds__(kMergeThreads) split_merge_kernel(AttnParams p) {
  __shared__ float sm_w[kMaxSplits];
  __shared__ float sm_l[kMaxSplits];
  __shared__ float red_buf[kMergeThreads / 32];
  const int h = blockIdx.y;
  const int64_t unit = blockIdx.x;
  const int G = p.group;
  const int64_t b = unit / p.num_kv_heads;
  const int kvh = int(unit - b * p.num_kv_heads);
  // the exchange's epoch of this CTA's row: written by this call site's previous merge launch,
  // which is at least two launches back (the attention kernel of this call runs in between)
  const uint32_t e = p.xr.world > 0 ? xrank_epoch(p.xl, p.xr, int(unit) * G + h) : 0u;
  pdl_wait();
  pdl_allow_next();
  const int len = max(p.seq_lens[b], 0) + (p.append ? 1 : 0);  // (the attention kernel's length)
  const int npages_b = int(min(int64_t((len + kPage - 1) / kPage), p.max_pages));
  const int nsplit = max(1, (npages_b + p.pages_per_split - 1) / p.pages_per_split);
  if (nsplit == 1 && p.xr.world == 0) return;  // the attention kernel wrote this unit's output itself
  const int tid = threadIdx.x;
  const int rec_floats = G * (kHeadDim + 2);
  const int outputs = G * kHeadDim;
  const float* recs = p.partials + unit * p.max_splits * rec_floats;
  float mloc = -INFINITY;
  for (int s = tid; s < nsplit; s += kMergeThreads) {
    const float m = recs[s * rec_floats + outputs + h];
    sm_w[s] = m;
    sm_l[s] = recs[s * rec_floats + outputs + G + h];
    mloc = fmaxf(mloc, m);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mloc = fmaxf(mloc, __shfl_xor_sync(0xffffffffu, mloc, o));
  if ((tid & 31) == 0) red_buf[tid >> 5] = mloc;
  __syncthreads();
  float M = -INFINITY;
  for (int w = 0; w < kMergeThreads / 32; ++w) M = fmaxf(M, red_buf[w]);
  __syncthreads();
  float lloc = 0.0f;
  for (int s = tid; s < nsplit; s += kMergeThreads) {
    const float w = M == -INFINITY ? 0.0f : exp2f(sm_w[s] - M);
    sm_w[s] = w;
    lloc += sm_l[s] * w;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) lloc += __shfl_xor_sync(0xffffffffu, lloc, o);
  if ((tid & 31) == 0) red_buf[tid >> 5] = lloc;
  __syncthreads();
  float L = 0.0f;
  for (int w = 0; w < kMergeThreads / 32; ++w) L += red_buf[w];
  const int d = tid;
  const float* col = recs + h * kHeadDim + d;
  float n0 = 0.0f, n1 = 0.0f, n2 = 0.0f, n3 = 0.0f;
  int s = 0;
  for (; s + 4 <= nsplit; s += 4) {
    n0 = fmaf(sm_w[s], col[(s + 0) * rec_floats], n0);
    n1 = fmaf(sm_w[s + 1], col[(s + 1) * rec_floats], n1);
    n2 = fmaf(sm_w[s + 2], col[(s + 2) * rec_floats], n2);
    n3 = fmaf(sm_w[s + 3], col[(s + 3) * rec_floats], n3);
  }
  for (; s < nsplit; ++s) n0 = fmaf(sm_w[s], col[s * rec_floats], n0);
  const float num = (n0 + n1) + (n2 + n3);
  const int64_t hq = int64_t(kvh) * G + h;
  if (p.xr.world == 0) {
    store_out<T>(p, b, hq, d, L > 0.0f ? num / L : 0.0f, M, L);
    return;
  }
  // ---- exchange this rank's merged row with every rank's over NVLink, then merge them: the
  // values are those store_out would write to out_f32 / out_lse, merged as oq_lse_merge does
  const int row = int(b * p.num_kv_heads * G + hq);
  xrank_put(p.xl, p.xr, row, e, d, L > 0.0f ? num / L : 0.0f);
  if (tid == 0) xrank_put(p.xl, p.xr, row, e, kHeadDim, lse_nat(M, L));
  float lse_all;
  const float y = xrank_merge(p.xl, p.xr, row, e, d, p.status, &lse_all);
  if (p.out) static_cast<T*>(p.out)[b * p.o_sb + hq * p.o_sh + d] = from_float<T>(y);
  if (p.out_f32) p.out_f32[(b * p.num_kv_heads * G + hq) * kHeadDim + d] = y;
  if (p.out_lse && d == 0) p.out_lse[b * p.num_kv_heads * G + hq] = lse_all;
}

// ---------------------------------------------------------------- host side
size_t counters_bytes(int64_t units) { return size_t((units * sizeof(int) + 255) / 256 * 256); }

// SMs x resident CTAs per SM of `kernel` on the current device (cached per device and kernel).
// (Every decode_attn_kernel instance -- 2 widths x 2 query dtypes x 2 MMA layouts x 2 group counts --
// fits the table; an unexpected kernel is computed uncached.)
int64_t resident_slots(const void* kernel, int threads, size_t smem) {
  constexpr int kKernels = 32;
  static std::mutex mu;
  static int64_t cache[64][kKernels] = {};
  static const void* kernels[kKernels] = {};
  auto compute = [&](int dev) {
    int sms = 0, per_sm = 0;
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, threads, smem);
    return int64_t(std::max(1, sms)) * std::max(1, per_sm);
  };
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0) return 148;
  if (dev >= 64) return compute(dev);
  std::lock_guard<std::mutex> lock(mu);
  int k = 0;
  for (; k < kKernels && kernels[k] != nullptr && kernels[k] != kernel; ++k) {
  }
  if (k == kKernels) return compute(dev);
  kernels[k] = kernel;
  if (cache[dev][k] == 0) cache[dev][k] = compute(dev);
  return cache[dev][k];
}

using Kernel = void (*)(const CUtensorMap, AttnParams);

// A launchable form of the kernel: instance, dynamic shared memory and threads per CTA.
struct KernelChoice {
  Kernel kernel;
  size_t smem;
  int threads;
};

template <int kBits, int kG>
KernelChoice kernel_choice(int dtype, int64_t group) {
  const Kernel k = dtype == OQ_BF16 ? (group > 4 ? decode_attn_kernel<__nv_bfloat16, true, kBits, kG>
                                                 : decode_attn_kernel<__nv_bfloat16, false, kBits, kG>)
                                    : (group > 4 ? decode_attn_kernel<__half, true, kBits, kG>
                                                 : decode_attn_kernel<__half, false, kBits, kG>);
  return {k, PageFormat<kBits, kG>::kSmem, kG * kThreads};
}

// groups = 3: one CTA of three warp groups per SM (few units: long ranges, one wave);
// groups = 1: one warp group per CTA, three CTAs per SM, so that a CTA's prologue and
// epilogue run under its neighbours' page loops (many units in many waves, e.g. serving).
KernelChoice pick_kernel(int bits, int dtype, int64_t group, int groups = 3) {
  KernelChoice c = bits == 8 ? (groups == 1 ? kernel_choice<8, 1>(dtype, group) : kernel_choice<8, 3>(dtype, group))
                             : (groups == 1 ? kernel_choice<4, 1>(dtype, group) : kernel_choice<4, 3>(dtype, group));
  cudaFuncSetAttribute(c.kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(c.smem));
  return c;
}

// Which form a one-range-per-unit launch takes: the one with the shorter estimate of
//   waves x (pages per warp group + fixed cost),
// waves = ceil(units / resident CTAs), pages = the longest sequence's.  The fixed cost (prologue
// and epilogue, in pages of loop time) is ~5 pages for the three-group CTA, alone on its SM, and
// ~2 for the one-group CTA, whose neighbours' loops run under it.  Measured at context 4096:
// 160, 192 and 384 sequences faster with one group (100 / 101 / 195 us against 114 / 116 / 225),
// 256 slower (171 against 152); ragged U[256, 8192]: 1024 sequences faster (512 against 549 us),
// 256 and 512 slower or level.
bool prefer_one_group(int64_t units, int64_t max_pages, const KernelChoice& three, const KernelChoice& one) {
  const int64_t s3 = resident_slots(reinterpret_cast<const void*>(three.kernel), three.threads, three.smem);
  const int64_t s1 = resident_slots(reinterpret_cast<const void*>(one.kernel), one.threads, one.smem);
  const double p = double(max_pages);
  const double t3 = double((units + s3 - 1) / s3) * (p / 3.0 + 5.0);
  const double t1 = double((units + s1 - 1) / s1) * (p + 2.0);
  return t1 <= t3;
}

}  // namespace

int decode_attn_plan(int bits, int dtype, int64_t group, int64_t batch, int64_t num_kv_heads,
                     int64_t max_pages_per_seq, int num_splits, int* pages_per_split) {
  // Split heuristic: as many KV ranges per (sequence, KV head) as fill about 7/8 of one wave
  // of resident CTAs (SMs x CTAs per SM), so that no CTA waits for a second wave; slightly
  // fewer, longer ranges than a full wave measured faster for one long sequence (context
  // 131072 on 148 SMs: 64 ranges of 32 pages 26.7 us per layer, 74 of 28 pages 27.5 us).
  const int64_t units = std::max<int64_t>(1, batch * num_kv_heads);
  int splits = num_splits;
  if (splits <= 0) {
    const KernelChoice kc = pick_kernel(bits, dtype, group);
    const int64_t slots = resident_slots(reinterpret_cast<const void*>(kc.kernel), kc.threads, kc.smem);
    // ... but at least kMinPagesPerSplit pages per range: merging many short ranges costs more than it saves
    splits = int(std::min<int64_t>(std::max<int64_t>(1, slots * 7 / 8 / units),
                                   std::max<int64_t>(1, max_pages_per_seq / kMinPagesPerSplit)));
  }
  // the merging CTA stages (max, sum) of every split in 64 KB of shared memory
  splits = int(std::min<int64_t>(std::min<int64_t>(splits, max_pages_per_seq), kMaxSplits));
  const int pps = int((max_pages_per_seq + splits - 1) / splits);
  if (pages_per_split) *pages_per_split = pps;
  return int((max_pages_per_seq + pps - 1) / pps);
}

// INT4: rows of 128 B, one box = the 128 K + V rows of a (page, KV head).  INT8: rows of
// 256 B seen as {128 B, 2 halves, rows} (the 128-byte swizzle caps a box line at 128 B).
int encode_codes_map(CUtensorMap* map, const uint8_t* kv_codes, int64_t num_pages, int64_t num_kv_heads, int bits) {
  auto fn = tensor_map_encoder();
  if (fn == nullptr) return fail(OQ_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
  const cuuint64_t rows = cuuint64_t(num_pages * num_kv_heads * 2 * kPage);
  CUresult res;
  if (bits == 8) {
    const cuuint64_t dims[3] = {128, 2, rows};
    const cuuint64_t strides[2] = {128, 256};
    const cuuint32_t box[3] = {128, 2, cuuint32_t(2 * kPage)};
    const cuuint32_t estr[3] = {1, 1, 1};
    res = fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<uint8_t*>(kv_codes), dims, strides, box, estr,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  } else {
    const cuuint64_t dims[2] = {cuuint64_t(kRowBytes), rows};
    const cuuint64_t strides[1] = {cuuint64_t(kRowBytes)};
    const cuuint32_t box[2] = {cuuint32_t(kRowBytes), cuuint32_t(2 * kPage)};
    const cuuint32_t estr[2] = {1, 1};
    res = fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<uint8_t*>(kv_codes), dims, strides, box, estr,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  }
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

namespace oq {
namespace {

// Options of the extended entry points: an appended token and launch flags.
struct AttnExtras {
  const void* new_k;
  const void* new_v;
  int64_t nk_sb, nk_sh, nv_sb, nv_sh;
  int flags;
};

int decode_attn_impl(
    int bits, const void* query, int dtype, int64_t query_stride_b, int64_t query_stride_h,
    const uint8_t* kv_codes, const uint16_t* kv_meta, int64_t num_pages, int64_t page_size,
    const int32_t* block_table, int64_t block_table_stride, int64_t max_pages_per_seq,
    const int32_t* seq_lens,
    int64_t batch, int64_t num_heads, int64_t num_kv_heads, int64_t head_dim,
    float scaling,
    void* out, int64_t out_stride_b, int64_t out_stride_h,
    float* out_f32, float* out_lse,
    void* workspace, size_t workspace_bytes, int num_splits,
    const void* gate, int64_t gate_stride_b, int64_t gate_stride_h,
    int32_t* device_status, void* stream, const XrankArgs* xr = nullptr, const AttnExtras* ex = nullptr) {
  const char* name = bits == 8 ? "decode_attn_int8_paged" : "decode_attn_int4_paged";
  if (ex && ex->new_k) {
    if (!ex->new_v) return fail(OQ_ERR_INVALID_ARGUMENT, "%s: an appended token needs both key and value", name);
    if (reinterpret_cast<uintptr_t>(ex->new_k) % 16 || reinterpret_cast<uintptr_t>(ex->new_v) % 16 ||
        (ex->nk_sb * 2) % 16 || (ex->nk_sh * 2) % 16 || (ex->nv_sb * 2) % 16 || (ex->nv_sh * 2) % 16) {
      return fail(OQ_ERR_MISALIGNED, "%s: appended key / value rows need 16-byte alignment", name);
    }
  }
  if (gate && !out) return fail(OQ_ERR_INVALID_ARGUMENT, "%s: a gate needs the model-dtype output", name);
  if (dtype != OQ_BF16 && dtype != OQ_F16) {
    return fail(OQ_ERR_UNSUPPORTED, "%s: query dtype must be bf16 or fp16", name);
  }
  if (head_dim != kHeadDim) return fail(OQ_ERR_UNSUPPORTED, "%s: head_dim must be 256", name);
  if (page_size != kPage) return fail(OQ_ERR_UNSUPPORTED, "%s: page_size must be 64", name);
  if (batch < 0 || num_kv_heads <= 0 || num_heads <= 0 || num_heads % num_kv_heads != 0 || num_pages <= 0 ||
      max_pages_per_seq <= 0 || block_table_stride < max_pages_per_seq) {
    return fail(OQ_ERR_INVALID_ARGUMENT, "%s: bad sizes", name);
  }
  const int64_t group = num_heads / num_kv_heads;
  if (group > kMaxGroup) return fail(OQ_ERR_UNSUPPORTED, "%s: more than 8 query heads per KV head", name);
  if (batch == 0) return ok();
  if (batch > 65535 || num_kv_heads > 65535) return fail(OQ_ERR_UNSUPPORTED, "%s: grid too large", name);
  if (!query || !kv_codes || !kv_meta || !block_table || !seq_lens || (!out && !out_f32 && !out_lse)) {
    return fail(OQ_ERR_INVALID_ARGUMENT, "%s: null pointer", name);
  }
  if (reinterpret_cast<uintptr_t>(query) % 16 || (query_stride_b * 2) % 16 || (query_stride_h * 2) % 16 ||
      reinterpret_cast<uintptr_t>(kv_codes) % 128 || reinterpret_cast<uintptr_t>(kv_meta) % 16) {
    return fail(OQ_ERR_MISALIGNED, "%s: query rows need 16-byte alignment, kv_codes 128 bytes, kv_meta 16 bytes", name);
  }
  if (num_pages * num_kv_heads * 2 * kPage >= (int64_t(1) << 31)) {
    return fail(OQ_ERR_UNSUPPORTED, "%s: page pool too large for 32-bit TMA rows", name);
  }

  const int64_t units = batch * num_kv_heads;
  int pps = 0;
  int splits = decode_attn_plan(bits, dtype, group, batch, num_kv_heads, max_pages_per_seq, num_splits, &pps);
  KernelChoice kc = pick_kernel(bits, dtype, group);
  if (splits == 1) {
    const KernelChoice one = pick_kernel(bits, dtype, group, 1);
    if (prefer_one_group(units, max_pages_per_seq, kc, one)) kc = one;
  }
  const Kernel kernel = kc.kernel;
  const size_t smem_bytes = kc.smem;
  const int threads = kc.threads;
  if (xr) {
    if (gate) return fail(OQ_ERR_UNSUPPORTED, "%s: no gate with the cross-GPU exchange", name);
    if (!xr->peers || xr->world <= 0 || xr->rank < 0 || xr->rank >= xr->world || xr->world > kXrankMaxWorld) {
      return fail(OQ_ERR_INVALID_ARGUMENT, "%s: bad exchange rank / world / buffers", name);
    }
    if (batch * num_heads > (1 << 20)) return fail(OQ_ERR_UNSUPPORTED, "%s: too many rows to exchange", name);
    if (!workspace) return fail(OQ_ERR_WORKSPACE, "%s: the exchange needs the split workspace", name);
  }

  if (splits > 1 || workspace || xr) {
    const size_t need = oq_decode_attn_workspace_bytes(batch, num_heads, num_kv_heads, head_dim, splits);
    if ((splits > 1 || xr) && (workspace == nullptr || workspace_bytes < need)) {
      return fail(OQ_ERR_WORKSPACE, "%s: workspace of %zu bytes needed for %d splits", name, need,
                  splits);
    }
  }
  const int64_t max_splits_ws =
      workspace ? std::max<int64_t>(1, (int64_t(workspace_bytes) - int64_t(counters_bytes(units))) /
                                           int64_t(units * group * (head_dim + 2) * sizeof(float)))
                : 1;

  CUtensorMap tmap;
  int st = encode_codes_map(&tmap, kv_codes, num_pages, num_kv_heads, bits);
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
  // few splits: the last CTA of each (sequence, KV head) merges in-launch; many: a merge kernel
  p.defer_merge = (splits > kInLaunchMergeSplits || xr) ? 1 : 0;
  p.status = device_status;
  p.gate = gate;
  p.g_sb = gate_stride_b;
  p.g_sh = gate_stride_h;
  p.wait_polls = wait_polls();
  p.append = (ex && ex->new_k) ? 1 : 0;
  p.new_k = ex ? ex->new_k : nullptr;
  p.new_v = ex ? ex->new_v : nullptr;
  p.nk_sb = ex ? ex->nk_sb : 0;
  p.nk_sh = ex ? ex->nk_sh : 0;
  p.nv_sb = ex ? ex->nv_sb : 0;
  p.nv_sh = ex ? ex->nv_sh : 0;
  p.kv_codes = const_cast<uint8_t*>(kv_codes);
  p.kv_meta_w = const_cast<uint16_t*>(kv_meta);
  p.early = (ex && (ex->flags & OQ_ATTN_EARLY)) ? 1 : 0;
  p.xr = xr ? *xr : XrankArgs{nullptr, 0, 0, 0};
  p.xl = XrankLayout{int(batch * num_heads), int(head_dim), xr ? xr->world : 0};

  dim3 grid((unsigned)splits, (unsigned)num_kv_heads, (unsigned)batch);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (p.early) {
    launch_pdl(kernel, grid, dim3(threads), smem_bytes, s, tmap, p);
  } else {
    launch_plain(kernel, grid, dim3(threads), smem_bytes, s, tmap, p);
  }
  if (p.defer_merge) {
    // early launch: the merge waits (griddepcontrol.wait) for the whole attention grid before
    // it reads a partial, and its launch gap overlaps the attention's epilogue
    const dim3 mgrid((unsigned)units, (unsigned)group);
    if (dtype == OQ_BF16) {
      launch_pdl(split_merge_kernel<__nv_bfloat16>, mgrid, dim3(kMergeThreads), 0, s, p);
    } else {
      launch_pdl(split_merge_kernel<__half>, mgrid, dim3(kMergeThreads), 0, s, p);
    }
  }
  return check_launch(name);
}

}  // namespace
}  // namespace oq

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
  return oq::decode_attn_impl(4, query, dtype, query_stride_b, query_stride_h, kv_codes, kv_meta, num_pages,
                              page_size, block_table, block_table_stride, max_pages_per_seq, seq_lens, batch,
                              num_heads, num_kv_heads, head_dim, scaling, out, out_stride_b, out_stride_h, out_f32,
                              out_lse, workspace, workspace_bytes, num_splits, nullptr, 0, 0, device_status, stream);
}

extern "C" int oq_decode_attn_int8_paged(
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
  return oq::decode_attn_impl(8, query, dtype, query_stride_b, query_stride_h, kv_codes, kv_meta, num_pages,
                              page_size, block_table, block_table_stride, max_pages_per_seq, seq_lens, batch,
                              num_heads, num_kv_heads, head_dim, scaling, out, out_stride_b, out_stride_h, out_f32,
                              out_lse, workspace, workspace_bytes, num_splits, nullptr, 0, 0, device_status, stream);
}

extern "C" int oq_decode_attn_int4_paged_gated(
    const void* query, int dtype, int64_t query_stride_b, int64_t query_stride_h,
    const uint8_t* kv_codes, const uint16_t* kv_meta, int64_t num_pages, int64_t page_size,
    const int32_t* block_table, int64_t block_table_stride, int64_t max_pages_per_seq,
    const int32_t* seq_lens,
    int64_t batch, int64_t num_heads, int64_t num_kv_heads, int64_t head_dim,
    float scaling,
    const void* gate, int64_t gate_stride_b, int64_t gate_stride_h,
    void* out, int64_t out_stride_b, int64_t out_stride_h,
    void* workspace, size_t workspace_bytes, int num_splits,
    int32_t* device_status, void* stream) {
  if (gate == nullptr) return oq::fail(OQ_ERR_INVALID_ARGUMENT, "decode_attn_int4_paged_gated: null gate");
  return oq::decode_attn_impl(4, query, dtype, query_stride_b, query_stride_h, kv_codes, kv_meta, num_pages,
                              page_size, block_table, block_table_stride, max_pages_per_seq, seq_lens, batch,
                              num_heads, num_kv_heads, head_dim, scaling, out, out_stride_b, out_stride_h, nullptr,
                              nullptr,
                              workspace, workspace_bytes, num_splits, gate, gate_stride_b, gate_stride_h,
                              device_status, stream);
}

extern "C" int oq_decode_attn_int8_paged_gated(
    const void* query, int dtype, int64_t query_stride_b, int64_t query_stride_h,
    const uint8_t* kv_codes, const uint16_t* kv_meta, int64_t num_pages, int64_t page_size,
    const int32_t* block_table, int64_t block_table_stride, int64_t max_pages_per_seq,
    const int32_t* seq_lens,
    int64_t batch, int64_t num_heads, int64_t num_kv_heads, int64_t head_dim,
    float scaling,
    const void* gate, int64_t gate_stride_b, int64_t gate_stride_h,
    void* out, int64_t out_stride_b, int64_t out_stride_h,
    void* workspace, size_t workspace_bytes, int num_splits,
    int32_t* device_status, void* stream) {
  if (gate == nullptr) return oq::fail(OQ_ERR_INVALID_ARGUMENT, "decode_attn_int8_paged_gated: null gate");
  return oq::decode_attn_impl(8, query, dtype, query_stride_b, query_stride_h, kv_codes, kv_meta, num_pages,
                              page_size, block_table, block_table_stride, max_pages_per_seq, seq_lens, batch,
                              num_heads, num_kv_heads, head_dim, scaling, out, out_stride_b, out_stride_h, nullptr,
                              nullptr, workspace, workspace_bytes, num_splits, gate, gate_stride_b, gate_stride_h,
                              device_status, stream);
}

extern "C" int oq_decode_attn_int4_paged_xrank(
    const void* query, int dtype, int64_t query_stride_b, int64_t query_stride_h,
    const uint8_t* kv_codes, const uint16_t* kv_meta, int64_t num_pages, int64_t page_size,
    const int32_t* block_table, int64_t block_table_stride, int64_t max_pages_per_seq,
    const int32_t* seq_lens,
    int64_t batch, int64_t num_heads, int64_t num_kv_heads, int64_t head_dim,
    float scaling,
    void* out, int64_t out_stride_b, int64_t out_stride_h,
    float* out_f32, float* out_lse,
    void* workspace, size_t workspace_bytes, int num_splits,
    float* const* peer_buffers, int rank, int world, int flags,
    int32_t* device_status, void* stream) {
  const oq::XrankArgs xr{peer_buffers, rank, world, oq::xrank_polls()};
  const oq::AttnExtras ex{nullptr, nullptr, 0, 0, 0, 0, flags};
  return oq::decode_attn_impl(4, query, dtype, query_stride_b, query_stride_h, kv_codes, kv_meta, num_pages,
                              page_size, block_table, block_table_stride, max_pages_per_seq, seq_lens, batch,
                              num_heads, num_kv_heads, head_dim, scaling, out, out_stride_b, out_stride_h, out_f32,
                              out_lse, workspace, workspace_bytes, num_splits, nullptr, 0, 0, device_status, stream,
                              &xr, &ex);
}

extern "C" int oq_decode_attn_paged_ex(
    int bits, const void* query, int dtype, int64_t query_stride_b, int64_t query_stride_h,
    const void* new_key, int64_t key_stride_b, int64_t key_stride_h,
    const void* new_value, int64_t value_stride_b, int64_t value_stride_h,
    uint8_t* kv_codes, uint16_t* kv_meta, int64_t num_pages, int64_t page_size,
    const int32_t* block_table, int64_t block_table_stride, int64_t max_pages_per_seq,
    const int32_t* seq_lens,
    int64_t batch, int64_t num_heads, int64_t num_kv_heads, int64_t head_dim,
    float scaling,
    const void* gate, int64_t gate_stride_b, int64_t gate_stride_h,
    void* out, int64_t out_stride_b, int64_t out_stride_h,
    float* out_f32, float* out_lse,
    void* workspace, size_t workspace_bytes, int num_splits, int flags,
    int32_t* device_status, void* stream) {
  if (bits != 4 && bits != 8) return oq::fail(OQ_ERR_UNSUPPORTED, "decode_attn_paged_ex: bits must be 4 or 8");
  if (!new_key != !new_value) return oq::fail(OQ_ERR_INVALID_ARGUMENT, "decode_attn_paged_ex: key without value");
  if (gate && (out_f32 || out_lse)) {
    return oq::fail(OQ_ERR_INVALID_ARGUMENT, "decode_attn_paged_ex: a gated call writes the query-dtype output only");
  }
  const oq::AttnExtras ex{new_key, new_value, key_stride_b, key_stride_h, value_stride_b, value_stride_h, flags};
  return oq::decode_attn_impl(bits, query, dtype, query_stride_b, query_stride_h, kv_codes, kv_meta, num_pages,
                              page_size, block_table, block_table_stride, max_pages_per_seq, seq_lens, batch,
                              num_heads, num_kv_heads, head_dim, scaling, out, out_stride_b, out_stride_h, out_f32,
                              out_lse, workspace, workspace_bytes, num_splits, gate, gate_stride_b, gate_stride_h,
                              device_status, stream, nullptr, &ex);
}
