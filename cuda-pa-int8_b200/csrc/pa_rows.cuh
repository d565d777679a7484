// Token-row cache writes shared by the cache-write kernels (quant.cu) and the fused new-token
// write of the decode step (decode.cu).
//
// Quantisation is bit-exact with the reference quantizer quantize_per_token
// (tests/paged_decode_attn.py:106-112):
//   amax  = max_d |x_d|                     (exact in the input dtype)
//   amax' = max(amax, T(1e-8))              (T = input dtype; T(1e-8) is 0 for fp16)
//   scale = float(T(float(amax') / 127))    (IEEE fp32 divide, round-to-nearest-even into T)
//   q_d   = clamp(rint(float(x_d) / scale), -127, 127)   (IEEE divide, half-to-even)
// A zero scale (all-zero or tiny fp16 rows) gives x/0 = +-inf -> +-127 and 0/0 = NaN -> 0,
// which is what the reference produces on the CPU. The FP8 (e4m3) rows use scale = amax / 448
// and round-to-nearest-even with saturation. The files including this are built without
// fast-math, and the divides are explicit __fdiv_rn.
#pragma once

#include "pa_common.cuh"
#include "pa_internal.h"

namespace pa {

template <typename T> struct In;
template <> struct In<__half> {
  static __device__ __forceinline__ float ld(const __half* p) { return __half2float(*p); }
  static __device__ __forceinline__ float clamp_floor() { return 0.f; }  // half(1e-8) == 0
  static __device__ __forceinline__ float round_t(float v) {
    return __half2float(__float2half_rn(v));
  }
};
template <> struct In<__nv_bfloat16> {
  static __device__ __forceinline__ float ld(const __nv_bfloat16* p) {
    return __bfloat162float(*p);
  }
  static __device__ __forceinline__ float clamp_floor() {
    return __bfloat162float(__float2bfloat16_rn(1e-8f));
  }
  static __device__ __forceinline__ float round_t(float v) {
    return __bfloat162float(__float2bfloat16_rn(v));
  }
};
template <> struct In<float> {
  static __device__ __forceinline__ float ld(const float* p) { return *p; }
  static __device__ __forceinline__ float clamp_floor() { return 1e-8f; }
  static __device__ __forceinline__ float round_t(float v) { return v; }
};

// Per-token scale from the row absmax (quantize_per_token, tests/paged_decode_attn.py:109-110).
template <typename T>
__device__ __forceinline__ float token_scale(float amax) {
  return In<T>::round_t(__fdiv_rn(fmaxf(amax, In<T>::clamp_floor()), 127.f));
}

__device__ __forceinline__ int8_t quant1(float x, float s) {
  int q = __float2int_rn(__fdiv_rn(x, s));
  q = q < -127 ? -127 : (q > 127 ? 127 : q);
  return (int8_t)q;
}

// Load DPL consecutive input values starting at src (src aligned to DPL elements).
template <typename T, int DPL>
__device__ __forceinline__ void load_vals(const T* src, float (&x)[DPL]) {
#pragma unroll
  for (int e = 0; e < DPL; ++e) x[e] = In<T>::ld(src + e);
}

// One warp writes one row (K or V) of one (token, kv head) into the paged cache: page row
// `page` (= block * kv_heads + kv_head), token offset `off` inside the block. Lane l owns the
// D/32 consecutive values starting at src + l * D/32. KIND: kRowsF16 (fp16 copy), kRowsI8
// (per-token int8, or the fixed per-tensor scale *fix when fix is non-null), kRowsFP8
// (per-token e4m3). Lane 0 writes the scale slot.
//   K page [D/8][bs][8]: a lane's values lie inside one 8-wide chunk (one store);
//   V page [D][bs]:      one element per head_dim row.
template <typename T, int KIND, int D>
__device__ __forceinline__ void warp_write_row(const T* src, int lane, bool is_v, void* cache,
                                               float* scales, size_t page, int off, int bs,
                                               const float* fix) {
  constexpr int DPL = D / 32;
  float x[DPL];
  load_vals<T, DPL>(src + lane * DPL, x);
  const int d0 = lane * DPL;
  if constexpr (KIND == kRowsF16) {
    __half hv[DPL];
#pragma unroll
    for (int e = 0; e < DPL; ++e) hv[e] = __float2half_rn(x[e]);
    __half* c = reinterpret_cast<__half*>(cache);
    if (!is_v) {
      __half* dst = c + (page * (D / 8) + d0 / 8) * bs * 8 + (size_t)off * 8 + (d0 & 7);
      if constexpr (DPL == 4) {
        *reinterpret_cast<uint2*>(dst) = *reinterpret_cast<const uint2*>(hv);
      } else {
#pragma unroll
        for (int e = 0; e < DPL; ++e) dst[e] = hv[e];
      }
    } else {
#pragma unroll
      for (int e = 0; e < DPL; ++e) c[(page * D + d0 + e) * bs + off] = hv[e];
    }
  } else {
    float s;
    uint8_t qv[DPL];
    if (KIND == kRowsI8 && fix != nullptr) {
      s = __ldg(fix);
    } else {
      float am = 0.f;
#pragma unroll
      for (int e = 0; e < DPL; ++e) am = fmaxf(am, fabsf(x[e]));
      am = warp_max(am);
      s = (KIND == kRowsI8) ? token_scale<T>(am) : __fdiv_rn(am, 448.f);
    }
    if constexpr (KIND == kRowsI8) {
#pragma unroll
      for (int e = 0; e < DPL; ++e) qv[e] = (uint8_t)quant1(x[e], s);
    } else {
#pragma unroll
      for (int e = 0; e < DPL; ++e)
        qv[e] = s > 0.f ? (uint8_t)__nv_cvt_float_to_fp8(__fdiv_rn(x[e], s), __NV_SATFINITE,
                                                         __NV_E4M3)
                        : (uint8_t)0;
    }
    uint8_t* c = reinterpret_cast<uint8_t*>(cache);
    if (!is_v) {
      uint8_t* dst = c + (page * (D / 8) + d0 / 8) * bs * 8 + (size_t)off * 8 + (d0 & 7);
      if constexpr (DPL == 4) {
        *reinterpret_cast<uint32_t*>(dst) = *reinterpret_cast<const uint32_t*>(qv);
      } else {
#pragma unroll
        for (int e = 0; e < DPL; ++e) dst[e] = qv[e];
      }
    } else {
#pragma unroll
      for (int e = 0; e < DPL; ++e) c[(page * D + d0 + e) * bs + off] = qv[e];
    }
    if (lane == 0) scales[page * bs + off] = s;
  }
}

}  // namespace pa
