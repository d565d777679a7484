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

// quant1(x, s) without the division where that is provably the same: inv = 1/s rounded to
// nearest, y = x * inv rounded to nearest, so |y - x/s| <= 2^-23 |x/s| < 2^-15 for
// |y| < 256. When y is farther than 2^-14 from a half-integer, x/s rounds to the same integer
// as y, which the 1.5 * 2^23 add-and-subtract rounding gives (ties to even, exact for
// |y| < 2^22); the sum's low bits hold that integer. Everything else (values near a
// half-integer, s = 0 or non-finite, |y| >= 256) takes the division.
__device__ __forceinline__ int quant_fast(float x, float s, float inv) {
  constexpr float kRound = 12582912.f;
  const float y = __fmul_rn(x, inv);
  const float s1 = __fadd_rn(y, kRound);
  const float d = __fsub_rn(y, __fsub_rn(s1, kRound));
  if (fabsf(d) < 0.5f - 0x1p-14f && fabsf(y) < 256.f) {  // false for NaN
    const int q = __float_as_int(s1) - 0x4B400000;
    return q < -127 ? -127 : (q > 127 ? 127 : q);
  }
  return quant1(x, s);
}

// Load DPL consecutive input values starting at src (src aligned to DPL elements).
template <typename T, int DPL>
__device__ __forceinline__ void load_vals(const T* src, float (&x)[DPL]) {
#pragma unroll
  for (int e = 0; e < DPL; ++e) x[e] = In<T>::ld(src + e);
}

// One row of one (token, kv head), quantised by one warp: lane l's D/32 consecutive values
// (from src + l * D/32) packed in storage order -- DPL bytes (int8 or e4m3) or DPL fp16
// halves -- and the row's scale. KIND: kRowsF16 (fp16 copy), kRowsI8 (per-token int8, or the
// fixed per-tensor scale *fix when fix is non-null), kRowsFP8 (per-token e4m3).
template <int KIND, int D>
struct RowQ {
  static constexpr int DPL = D / 32;
  static constexpr int WORDS = KIND == kRowsF16 ? DPL / 2 : DPL / 4;
  uint32_t w[WORDS];
  float s;
};

// The row quantiser on values already loaded: each lane holds x = its D/32 consecutive values
// of the row (T is the input dtype, which the per-token scale is rounded to).
template <typename T, int KIND, int D>
__device__ __forceinline__ RowQ<KIND, D> warp_quantize_vals(const float (&x)[D / 32],
                                                            const float* fix) {
  constexpr int DPL = D / 32;
  static_assert(DPL % 4 == 0, "a lane packs whole 32-bit words");
  RowQ<KIND, D> r;
  if constexpr (KIND == kRowsF16) {
    r.s = 0.f;
#pragma unroll
    for (int e = 0; e < DPL; e += 2) {
      const __half2 h = __floats2half2_rn(x[e], x[e + 1]);
      r.w[e / 2] = *reinterpret_cast<const uint32_t*>(&h);
    }
  } else {
    float s;
    if (KIND == kRowsI8 && fix != nullptr) {
      s = __ldg(fix);
    } else {
      float am = 0.f;
#pragma unroll
      for (int e = 0; e < DPL; ++e) am = fmaxf(am, fabsf(x[e]));
      am = warp_max(am);
      s = (KIND == kRowsI8) ? token_scale<T>(am) : __fdiv_rn(am, 448.f);
    }
    uint8_t qv[DPL];
    if constexpr (KIND == kRowsI8) {
      const float inv = __frcp_rn(s);
#pragma unroll
      for (int e = 0; e < DPL; ++e) qv[e] = (uint8_t)quant_fast(x[e], s, inv);
    } else {
#pragma unroll
      for (int e = 0; e < DPL; ++e)
        qv[e] = s > 0.f ? (uint8_t)__nv_cvt_float_to_fp8(__fdiv_rn(x[e], s), __NV_SATFINITE,
                                                         __NV_E4M3)
                        : (uint8_t)0;
    }
#pragma unroll
    for (int e = 0; e < DPL; e += 4)
      r.w[e / 4] = (uint32_t)qv[e] | ((uint32_t)qv[e + 1] << 8) | ((uint32_t)qv[e + 2] << 16) |
                   ((uint32_t)qv[e + 3] << 24);
    r.s = s;
  }
  return r;
}

template <typename T, int KIND, int D>
__device__ __forceinline__ RowQ<KIND, D> warp_quantize_row(const T* src, int lane,
                                                           const float* fix) {
  float x[D / 32];
  load_vals<T, D / 32>(src + lane * (D / 32), x);
  return warp_quantize_vals<T, KIND, D>(x, fix);
}

// Element e (0 <= e < D/32) of lane `lane`'s part of a quantised row, as stored.
template <int KIND, int D>
__device__ __forceinline__ uint32_t row_elem(const RowQ<KIND, D>& r, int e) {
  if constexpr (KIND == kRowsF16) {
    return (r.w[e / 2] >> (16 * (e & 1))) & 0xffffu;
  } else {
    return (r.w[e / 4] >> (8 * (e & 3))) & 0xffu;
  }
}

// Store lane `lane`'s part of a quantised row into the paged cache: page row `page`
// (= block * kv_heads + kv_head), token offset `off` inside the block. Lane 0 writes the
// scale slot (one-byte caches).
//   K page [D/8][bs][8]: a lane's values lie inside one 8-wide chunk (one store);
//   V page [D][bs]:      one element per head_dim row.
template <int KIND, int D>
__device__ __forceinline__ void store_row(const RowQ<KIND, D>& r, int lane, bool is_v,
                                          void* cache, float* scales, size_t page, int off,
                                          int bs) {
  constexpr int DPL = D / 32;
  const int d0 = lane * DPL;
  constexpr int ES = KIND == kRowsF16 ? 2 : 1;
  uint8_t* c = reinterpret_cast<uint8_t*>(cache);
  if (!is_v) {
    uint8_t* dst = c + ((page * (D / 8) + d0 / 8) * bs * 8 + (size_t)off * 8 + (d0 & 7)) * ES;
    if constexpr (KIND == kRowsF16 && DPL == 4) {
      *reinterpret_cast<uint2*>(dst) = make_uint2(r.w[0], r.w[1]);
    } else if constexpr (KIND != kRowsF16 && DPL == 4) {
      *reinterpret_cast<uint32_t*>(dst) = r.w[0];
    } else {
#pragma unroll
      for (int e = 0; e < DPL; ++e) {
        if constexpr (ES == 2) {
          reinterpret_cast<uint16_t*>(dst)[e] = (uint16_t)row_elem<KIND, D>(r, e);
        } else {
          dst[e] = (uint8_t)row_elem<KIND, D>(r, e);
        }
      }
    }
  } else {
#pragma unroll
    for (int e = 0; e < DPL; ++e) {
      const size_t i = (page * D + d0 + e) * bs + off;
      if constexpr (ES == 2) {
        reinterpret_cast<uint16_t*>(c)[i] = (uint16_t)row_elem<KIND, D>(r, e);
      } else {
        c[i] = (uint8_t)row_elem<KIND, D>(r, e);
      }
    }
  }
  if (KIND != kRowsF16 && lane == 0) scales[page * bs + off] = r.s;
}

// One warp writes one row (K or V) of one (token, kv head) into the paged cache.
template <typename T, int KIND, int D>
__device__ __forceinline__ void warp_write_row(const T* src, int lane, bool is_v, void* cache,
                                               float* scales, size_t page, int off, int bs,
                                               const float* fix) {
  const RowQ<KIND, D> r = warp_quantize_row<T, KIND, D>(src, lane, fix);
  store_row<KIND, D>(r, lane, is_v, cache, scales, page, off, bs);
}

}  // namespace pa
