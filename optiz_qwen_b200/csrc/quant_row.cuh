// Quantisation of one cache row (one token's K or V of one KV head) by one warp, shared by the
// append-quantize kernel and the decode attention that appends its step's token itself.
//
// The reference's _quantize_groupwise with group = head_dim (optiz_qwen/compression/
// qserve_kv_cache.py:313-335) and _pack_uint4 (:356-362): min and max of the row, scale =
// (max - min) / (2^bits - 1) in fp32 (1 where it is not positive), code = round-half-even of
// (x - min) / scale with IEEE division, clamped to [0, 2^bits - 1]; two codes per byte for 4
// bits (low nibble first).  The stored scale and min are the fp32 values rounded to fp16.
#pragma once

#include "common.cuh"

namespace oq {

template <typename T, int EPL, bool VEC>
__device__ __forceinline__ void load_row(const T* row, int lane, float (&x)[EPL]) {
  const T* p = row + lane * EPL;
  if constexpr (VEC && (EPL * sizeof(T)) % 16 == 0) {
    constexpr int kVecs = EPL * sizeof(T) / 16;
    constexpr int kPer = 16 / sizeof(T);
#pragma unroll
    for (int v = 0; v < kVecs; ++v) {
      uint4 u = __ldg(reinterpret_cast<const uint4*>(p) + v);
      const T* e = reinterpret_cast<const T*>(&u);
#pragma unroll
      for (int i = 0; i < kPer; ++i) x[v * kPer + i] = to_float<T>(e[i]);
    }
  } else {
#pragma unroll
    for (int i = 0; i < EPL; ++i) x[i] = to_float<T>(p[i]);
  }
}

// The warp's row `src` (head_dim = 32 * EPL values) into the codes row `row` (head_dim * kBits / 8
// bytes; lane l writes its EPL codes at byte l * EPL * kBits / 8) and the fp16 scale / min into
// meta[0] / meta[meta_stride] (lane 0).  Every lane of the warp calls it.
template <typename T, int EPL, bool VEC, int kBits>
__device__ __forceinline__ void quantize_row(const T* src, int lane, uint8_t* row, uint16_t* meta,
                                             int64_t meta_stride) {
  constexpr float kLevels = float((1 << kBits) - 1);
  constexpr int kLaneBytes = EPL * kBits / 8;
  float x[EPL];
  load_row<T, EPL, VEC>(src, lane, x);

  float mn = x[0], mx = x[0];
#pragma unroll
  for (int i = 1; i < EPL; ++i) {
    mn = fminf(mn, x[i]);
    mx = fmaxf(mx, x[i]);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    mn = fminf(mn, __shfl_xor_sync(0xffffffffu, mn, o));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  }
  // scale = (max - min) / levels in fp32; 1 where it is not positive (qserve_kv_cache.py:326-328)
  float scale = __fdiv_rn(__fsub_rn(mx, mn), kLevels);
  if (!(scale > 0.0f)) scale = 1.0f;

  constexpr int kWords = kLaneBytes / 4 > 0 ? kLaneBytes / 4 : 1;
  constexpr int kPerWord = 32 / kBits;
  uint32_t packed[kWords] = {};
#pragma unroll
  for (int i = 0; i < EPL; ++i) {
    float c = rintf(__fdiv_rn(__fsub_rn(x[i], mn), scale));
    c = fminf(fmaxf(c, 0.0f), kLevels);
    packed[i / kPerWord] |= static_cast<uint32_t>(c) << (kBits * (i % kPerWord));
  }

  uint8_t* dst = row + lane * kLaneBytes;
  if constexpr (kLaneBytes >= 4) {
#pragma unroll
    for (int w = 0; w < kLaneBytes / 4; ++w) reinterpret_cast<uint32_t*>(dst)[w] = packed[w];
  } else if constexpr (kLaneBytes == 2) {
    *reinterpret_cast<uint16_t*>(dst) = static_cast<uint16_t>(packed[0]);
  } else {
    *dst = static_cast<uint8_t>(packed[0]);
  }
  if (lane == 0) {
    meta[0] = __half_as_ushort(__float2half_rn(scale));
    meta[meta_stride] = __half_as_ushort(__float2half_rn(mn));
  }
}

}  // namespace oq
