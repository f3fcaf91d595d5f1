// Shared device helpers for the restricted output head kernels (sm_100a).
//
// Selection rule (include/marketforge/cuda/greedy.hpp:23-42, reference
// kernel src/cuda/greedy.cu:133-212): the highest FP32 score wins, equal
// scores go to the lowest token id, NaN never wins, an all-NaN row selects
// its lowest candidate.  Every kernel here encodes a (score, id) pair as one
// 64-bit key whose unsigned order IS that rule, so an argmax is a plain
// integer max — order-independent, so merges across lanes, warps and thread
// blocks (atomicMax) give the same answer however they are scheduled:
//
//   key = (ordered(score) << 32) | (0xFFFFFFFF - id)
//   ordered(x) = x >= +0 ? bits | 0x80000000 : ~bits   (-0 folded to +0)
//   ordered(NaN) = 0     -> a NaN key only beats "no candidate" (key 0),
//                           and among NaN keys the lowest id wins
//   key 0                -> no candidate was seen
//   key ~0               -> the row holds an invalid candidate (poisons it:
//                           no real key reaches ~0 because ordered() never
//                           returns 0xFFFFFFFF for a non-NaN float)
#pragma once

#include <cuda_fp16.h>
#include <stdint.h>

#include "mf_head.h"

namespace mfb {

constexpr unsigned long long kKeyNone = 0ull;
constexpr unsigned long long kKeyPoison = ~0ull;
constexpr uint32_t kInvalid = MF_INVALID_TOKEN;

__device__ __forceinline__ uint32_t ordered_score(float s) {
  uint32_t b = __float_as_uint(s);
  if ((b & 0x7FFFFFFFu) > 0x7F800000u) return 0u;  // NaN
  if (b == 0x80000000u) b = 0u;                     // -0 ties with +0
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

__device__ __forceinline__ float score_from_ordered(uint32_t o) {
  if (o == 0u) return __uint_as_float(0x7FC00000u);  // NaN
  const uint32_t b = (o & 0x80000000u) ? (o & 0x7FFFFFFFu) : ~o;
  return __uint_as_float(b);
}

__device__ __forceinline__ unsigned long long make_key(float s, uint32_t id) {
  return ((unsigned long long)ordered_score(s) << 32) | (unsigned long long)(~id);
}

__device__ __forceinline__ bool key_is_result(unsigned long long k) {
  return k != kKeyNone && k != kKeyPoison;
}
__device__ __forceinline__ uint32_t key_id(unsigned long long k) { return ~(uint32_t)k; }
__device__ __forceinline__ float key_score(unsigned long long k) {
  return score_from_ordered((uint32_t)(k >> 32));
}

__device__ __forceinline__ unsigned long long umax64(unsigned long long a,
                                                     unsigned long long b) {
  return a > b ? a : b;
}

// Programmatic dependent launch.  `pdl_trigger` lets the next kernel on the
// stream (launched with programmatic stream serialization) start while this
// one is still running; `pdl_wait` blocks until the previous kernel on the
// stream has completed and its memory is visible.  Both are no-ops for a
// kernel launched without the attribute.
__device__ __forceinline__ void pdl_trigger() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// 16-byte streaming load through the read-only path that does not allocate
// in L1: embedding rows are touched once per candidate.
__device__ __forceinline__ uint4 ld_stream_v4(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

__device__ __forceinline__ uint4 ld_v4(const void* p) {
  return *reinterpret_cast<const uint4*>(p);
}

// acc_lo += lo(h) * lo(e), acc_hi += hi(h) * hi(e): Blackwell's mixed
// precision FMA (f16 sources, f32 accumulator, one rounding), which is
// fmaf(float(h), float(e), acc) without separate conversions.
__device__ __forceinline__ void fma2_f16_f32(float& acc_lo, float& acc_hi, uint32_t h,
                                             uint32_t e) {
  asm("{\n\t.reg .f16 h0, h1, e0, e1;\n\t"
      "mov.b32 {h0, h1}, %2;\n\t"
      "mov.b32 {e0, e1}, %3;\n\t"
      "fma.rn.f32.f16 %0, h0, e0, %0;\n\t"
      "fma.rn.f32.f16 %1, h1, e1, %1;\n\t}"
      : "+f"(acc_lo), "+f"(acc_hi)
      : "r"(h), "r"(e));
}

__device__ __forceinline__ void dot_v4(float& a0, float& a1, const uint4& h, const uint4& e) {
  fma2_f16_f32(a0, a1, h.x, e.x);
  fma2_f16_f32(a0, a1, h.y, e.y);
  fma2_f16_f32(a0, a1, h.z, e.z);
  fma2_f16_f32(a0, a1, h.w, e.w);
}

// Sum across the 8 lanes of an aligned lane group (xor 4, 2, 1).
__device__ __forceinline__ float group8_sum(float v, unsigned mask) {
  v += __shfl_xor_sync(mask, v, 4);
  v += __shfl_xor_sync(mask, v, 2);
  v += __shfl_xor_sync(mask, v, 1);
  return v;
}

__device__ __forceinline__ unsigned long long warp_max_key(unsigned long long k) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) k = umax64(k, __shfl_xor_sync(0xFFFFFFFFu, k, o));
  return k;
}

// SmolLM2-135M hidden width: 576 fp16 = 1152 B = 72 x 16 B, so each of the
// 8 lanes of a group owns 9 16-byte chunks (chunk j = lane + 8 k).
constexpr int kFastHidden = 576;
constexpr int kFastChunksPerLane = kFastHidden / 8 / 8;  // 9

}  // namespace mfb
