// Row-level helpers shared by the decoder's kernels: vector loads, Snake and
// the depthwise k=7 tap sum on four channels, and the history pool's slots,
// head tables and ring rows.
#pragma once
#include "fav_device.cuh"
#include "fav_internal.h"

namespace fav {

__device__ __forceinline__ float2 ldg2(const float* p) { return __ldg(reinterpret_cast<const float2*>(p)); }
__device__ __forceinline__ float4 lds4(const float* p) { return *reinterpret_cast<const float4*>(p); }
__device__ __forceinline__ float4 ldg4(const float* p) { return __ldg(reinterpret_cast<const float4*>(p)); }

__device__ __forceinline__ float2 lo2(float4 v) { return make_float2(v.x, v.y); }
__device__ __forceinline__ float2 hi2(float4 v) { return make_float2(v.z, v.w); }
__device__ __forceinline__ float4 cat4(float2 a, float2 b) { return make_float4(a.x, a.y, b.x, b.y); }

// Snake of four channels: the bf16 path as two packed-fp32 lane pairs (or,
// with PACKED false, four scalar lanes: the same roundings, fewer registers),
// the int8 path (EXACT) in its fixed scalar operation order.
template <bool EXACT = false, bool PACKED = true>
__device__ __forceinline__ float4 snake4(float4 v, float4 al, float4 rc) {
  if constexpr (EXACT)
    return make_float4(snake_exact(v.x, al.x, rc.x), snake_exact(v.y, al.y, rc.y), snake_exact(v.z, al.z, rc.z),
                       snake_exact(v.w, al.w, rc.w));
  if constexpr (!PACKED)
    return make_float4(snake(v.x, al.x, rc.x), snake(v.y, al.y, rc.y), snake(v.z, al.z, rc.z), snake(v.w, al.w, rc.w));
  return cat4(snake2(lo2(v), lo2(al), lo2(rc)), snake2(hi2(v), hi2(al), hi2(rc)));
}

// Depthwise k=7 tap sum of four channels, oldest tap first, plus bias. The
// int8 path (EXACT) rounds every product and sum (the oracle's order); the
// bf16 path chains fused multiply-adds as two packed-fp32 lane pairs (PACKED)
// or four scalar lanes (the same roundings, fewer registers).
template <bool EXACT, bool PACKED = true>
__device__ __forceinline__ float4 dw7(const float4 (&w)[7], const float4 (&win)[7], float4 bias) {
  if constexpr (EXACT) {
    float4 h = make_float4(__fmul_rn(w[0].x, win[0].x), __fmul_rn(w[0].y, win[0].y), __fmul_rn(w[0].z, win[0].z),
                           __fmul_rn(w[0].w, win[0].w));
#pragma unroll
    for (int j = 1; j < 7; ++j) {
      h.x = __fadd_rn(h.x, __fmul_rn(w[j].x, win[j].x));
      h.y = __fadd_rn(h.y, __fmul_rn(w[j].y, win[j].y));
      h.z = __fadd_rn(h.z, __fmul_rn(w[j].z, win[j].z));
      h.w = __fadd_rn(h.w, __fmul_rn(w[j].w, win[j].w));
    }
    return make_float4(__fadd_rn(h.x, bias.x), __fadd_rn(h.y, bias.y), __fadd_rn(h.z, bias.z), __fadd_rn(h.w, bias.w));
  }
  if constexpr (!PACKED) {
    float4 h = make_float4(w[0].x * win[0].x, w[0].y * win[0].y, w[0].z * win[0].z, w[0].w * win[0].w);
#pragma unroll
    for (int j = 1; j < 7; ++j) {
      h.x = fmaf(w[j].x, win[j].x, h.x);
      h.y = fmaf(w[j].y, win[j].y, h.y);
      h.z = fmaf(w[j].z, win[j].z, h.z);
      h.w = fmaf(w[j].w, win[j].w, h.w);
    }
    return make_float4(h.x + bias.x, h.y + bias.y, h.z + bias.z, h.w + bias.w);
  }
  float2 h0 = f2mul(lo2(w[0]), lo2(win[0])), h1 = f2mul(hi2(w[0]), hi2(win[0]));
#pragma unroll
  for (int j = 1; j < 7; ++j) {
    h0 = f2fma(lo2(w[j]), lo2(win[j]), h0);
    h1 = f2fma(hi2(w[j]), hi2(win[j]), h1);
  }
  return cat4(f2add(h0, lo2(bias)), f2add(h1, hi2(bias)));
}

// ----------------------------------------------------------- history rings
// A stream's slot in the pool: every layer's ring, then two head tables.
__device__ __forceinline__ float* slot_base(const StateRef& st, int code) {
  return st.pool + (size_t)(code >> 2) * kSlotStride;
}
__device__ __forceinline__ int* head_table(float* slot, int parity) {
  return reinterpret_cast<int*>(slot + kRingFloats) + parity * kHeadInts;
}

// Ring row that receives chunk row tp (tp >= max(0, N - H)).
__device__ __forceinline__ float* hist_new_row(const StateRef& st, const HistRef& h, int code, int head, int tp,
                                               int N) {
  const int H = h.rows;
  int row = head + H + tp - (N > H ? N - H : 0);
  row %= 2 * H;
  return slot_base(st, code) + h.ring + row * h.width;
}

// Advanced head of the history, written to the other head table.
__device__ __forceinline__ void hist_commit_head(const StateRef& st, const HistRef& h, int code, int head, int N) {
  const int H = h.rows;
  head_table(slot_base(st, code), (code & 1) ^ 1)[h.index] = (head + (N < H ? N : H)) % (2 * H);
}

}  // namespace fav
