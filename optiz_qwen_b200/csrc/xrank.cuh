// Exchange of log-sum-exp attention partials between the GPUs of one box over NVLink, one
// output row at a time, shared by the standalone exchange kernel (xrank.cu) and the split-KV
// merge of the long-context attention (decode_attention.cu), which exchanges each row as
// soon as it has merged it.
//
// Every rank owns one receive buffer per call site in its own HBM; the other ranks see it
// through CUDA IPC mappings (no multicast object).  Each element travels with its call's
// epoch in one 8-byte store, {value bits, epoch}, so a reader that sees the epoch sees the
// value: no fence and no separate flag (the low-latency scheme NCCL calls LL).  Layout, for
// `rows` rows of `head_dim` floats and `world` ranks:
//   slots  [2 parities][world][rows][head_dim + 1] x {uint32 value bits, uint32 epoch}
//          (element head_dim of a row is its LSE);
//   epochs [rows] uint32, this rank's own call counter per row (never read by a peer).
// A call of row r: e = epochs[r] + 1; this rank's elements go into slot [e & 1][rank][r] of
// every rank, tagged e; the rank then polls (bounded) the words of slot [e & 1][q][r] in its
// own buffer until each carries e, merges, and stores epochs[r] = e.  A rank is at most one
// call ahead of another on a row (it cannot finish call e before every rank has written
// call e, and a rank writes call e only after finishing call e - 1, i.e. after reading
// parity (e - 1) & 1), so the parity double buffer is never overwritten while it is read.
// Peer memory is touched by plain loads and stores only (no TMA, no bulk copy, no multicast).
#pragma once

#include "common.cuh"

namespace oq {

__device__ __forceinline__ void st_tagged(uint2* p, float v, uint32_t e) {
  asm volatile("st.volatile.global.v2.u32 [%0], {%1, %2};\n" ::"l"(p), "r"(__float_as_uint(v)), "r"(e) : "memory");
}
__device__ __forceinline__ uint2 ld_tagged(const uint2* p) {
  uint2 w;
  asm volatile("ld.volatile.global.v2.u32 {%0, %1}, [%2];\n" : "=r"(w.x), "=r"(w.y) : "l"(p) : "memory");
  return w;
}

struct XrankLayout {
  int rows, head_dim, world;
  __host__ __device__ int64_t row_words() const { return int64_t(head_dim) + 1; }  // uint2 words
  __host__ __device__ int64_t slot_words() const { return int64_t(rows) * row_words(); }
  __host__ __device__ int64_t total_bytes() const {
    return 2 * int64_t(world) * slot_words() * 8 + int64_t(rows) * 4;
  }
  // element d (d == head_dim: the LSE) of row `row` in slot [par][q] of buffer `base`
  __device__ uint2* word(float* base, int par, int q, int row, int d) const {
    return reinterpret_cast<uint2*>(base) + (int64_t(par) * world + q) * slot_words() + int64_t(row) * row_words() + d;
  }
  __device__ uint32_t* epoch(float* base, int row) const {
    return reinterpret_cast<uint32_t*>(reinterpret_cast<uint2*>(base) + 2 * int64_t(world) * slot_words()) + row;
  }
};

struct XrankArgs {
  float* const* peers;  // [world] every rank's buffer of this call site ([rank] = this rank's)
  int rank, world;
  int64_t polls;        // polls of a word before OQ_DEV_TIMEOUT (~1 us each after the first 256)
};

// Polls of a launch: ~1 us each after the first 256, so the default copy-wait limit
// (wait_polls(), ~2 s) gives the same ~2 s bound, and the test hook shortens both.
inline int64_t xrank_polls() { return int64_t(wait_polls()) * 20; }

// This call's epoch of `row`; every thread reads it.  The word is written at the end of this
// call site's previous call: a kernel may read it before its dependency wait only when that
// call is at least two launches back in the stream (not the immediately preceding kernel).
__device__ __forceinline__ uint32_t xrank_epoch(const XrankLayout& L, const XrankArgs& x, int row) {
  return *reinterpret_cast<volatile uint32_t*>(L.epoch(x.peers[x.rank], row)) + 1;
}

// Element d of this rank's row into every rank's slot.
__device__ __forceinline__ void xrank_put(const XrankLayout& L, const XrankArgs& x, int row, uint32_t e, int d,
                                          float v) {
  const int par = int(e & 1);
  for (int q = 0; q < x.world; ++q) st_tagged(L.word(x.peers[q], par, x.rank, row, d), v, e);
}

// Element d of rank q's row from this rank's own buffer, once it carries epoch e; `ok` turns
// false when it does not arrive within the poll limit (later calls then do not wait).
__device__ __forceinline__ float xrank_get(const XrankLayout& L, const XrankArgs& x, int row, uint32_t e, int q,
                                           int d, bool& ok) {
  const uint2* w = L.word(x.peers[x.rank], int(e & 1), q, row, d);
  uint2 v = ld_tagged(w);
  if (x.polls == 0) ok = false;  // (the test hook: every wait runs out at once)
  if (v.y == e || !ok) return __uint_as_float(v.x);
  for (int64_t i = 0; i < x.polls; ++i) {
    if (i >= 256) __nanosleep(1000);
    v = ld_tagged(w);
    if (v.y == e) return __uint_as_float(v.x);
  }
  ok = false;
  return __uint_as_float(v.x);
}

// Every thread of the CTA that owns `row`: the merged element d over all ranks, out = sum_q
// exp(lse_q - m) o_q / sum_q exp(lse_q - m), m = max_q lse_q, q in rank order --
// oq_lse_merge's arithmetic and order; *lse_out receives the merged LSE.  Then the CTA
// agrees on the outcome (OQ_DEV_TIMEOUT into `status` if a word never arrived) and thread 0
// advances the row's epoch.  d may be out of range (d >= head_dim) for threads that only
// take part in the agreement.  world <= kXrankMaxWorld.
constexpr int kXrankMaxWorld = 8;  // ranks of one box

__device__ __forceinline__ float xrank_merge(const XrankLayout& L, const XrankArgs& x, int row, uint32_t e, int d,
                                             int32_t* status, float* lse_out) {
  bool ok = true;
  float y = 0.0f, lse = -INFINITY;
  if (d < L.head_dim) {
    float lq[kXrankMaxWorld], oq[kXrankMaxWorld];
    float m = -INFINITY;
#pragma unroll
    for (int q = 0; q < kXrankMaxWorld; ++q) {
      if (q < x.world) {
        lq[q] = xrank_get(L, x, row, e, q, L.head_dim, ok);
        oq[q] = xrank_get(L, x, row, e, q, d, ok);
        m = fmaxf(m, lq[q]);
      }
    }
    float denom = 0.0f;
#pragma unroll
    for (int q = 0; q < kXrankMaxWorld; ++q) {
      if (q < x.world) denom += (m == -INFINITY || lq[q] == -INFINITY) ? 0.0f : expf(lq[q] - m);
    }
    float acc = 0.0f;
#pragma unroll
    for (int q = 0; q < kXrankMaxWorld; ++q) {
      if (q < x.world && m != -INFINITY && lq[q] != -INFINITY) acc += expf(lq[q] - m) * oq[q];
    }
    lse = denom > 0.0f ? m + logf(denom) : -INFINITY;
    y = denom > 0.0f ? acc / denom : 0.0f;
  }
  const bool timed_out = __syncthreads_or(!ok);
  if (threadIdx.x == 0) {
    if (timed_out) report(status, OQ_DEV_TIMEOUT);
    *L.epoch(x.peers[x.rank], row) = e;
  }
  *lse_out = lse;
  return y;
}

}  // namespace oq
