// Cache-write kernels for B200: per-token symmetric INT8 quantize-into-cache, FP16
// copy-into-cache, block-granular prefill scatter, and the per-tensor absmax scale.
//
// The per-row quantisation (bit-exact with the reference's quantize_per_token,
// tests/paged_decode_attn.py:106-112) lives in pa_rows.cuh, shared with the decode step's fused
// new-token write. These kernels are built without fast-math so the divides stay IEEE.

#include "pa_common.cuh"
#include "pa_internal.h"
#include "pa_rows.cuh"

#include <algorithm>

namespace pa {
namespace {

// ---------------------------------------------------------------------------------------
// Token-granular write: one warp per (token, kv-head, K|V) row.
// ---------------------------------------------------------------------------------------
template <typename T, int KIND, int D>
__global__ void __launch_bounds__(256) write_rows_kernel(
    const T* __restrict__ k, const T* __restrict__ v, long long token_stride,
    const int* __restrict__ slot_mapping, int N, int KVH, void* __restrict__ k_cache,
    void* __restrict__ v_cache, float* __restrict__ k_scales, float* __restrict__ v_scales,
    int NB, int bs, const float* __restrict__ kfix, const float* __restrict__ vfix,
    int* status) {
  const long long gw = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (gw >= (long long)N * KVH * 2) return;
  const int which = (int)(gw & 1);  // 0: K, 1: V
  const long long row = gw >> 1;
  const int n = (int)(row / KVH);
  const int kvh = (int)(row - (long long)n * KVH);
  const int slot = __ldg(slot_mapping + n);
  if (slot < 0) return;  // padding token
  const int blk = slot / bs;
  const int off = slot - blk * bs;
  if (blk >= NB) {
    if (lane == 0) flag_error(status, PA_ERR_SLOT);
    return;
  }
  const T* src = (which ? v : k) + (size_t)n * token_stride + (size_t)kvh * D;
  warp_write_row<T, KIND, D>(src, lane, which != 0, which ? v_cache : k_cache,
                             which ? v_scales : k_scales, (size_t)blk * KVH + kvh, off, bs,
                             which ? vfix : kfix);
}

// ---------------------------------------------------------------------------------------
// The decode step's new-token write: one warp per (sequence, kv-head, K|V) row; the token goes
// to position context_lens[b] - 1 of sequence b, through its block table.
// ---------------------------------------------------------------------------------------
template <typename T, int KIND, int D>
__global__ void __launch_bounds__(256) step_rows_kernel(
    const T* __restrict__ k, const T* __restrict__ v, long long token_stride,
    const int* __restrict__ block_table, const int* __restrict__ context_lens, int max_blocks,
    int B, int KVH, void* __restrict__ k_cache, void* __restrict__ v_cache,
    float* __restrict__ k_scales, float* __restrict__ v_scales, int NB, int bs,
    const float* __restrict__ kfix, const float* __restrict__ vfix, int* status) {
  const long long gw = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (gw >= (long long)B * KVH * 2) return;
  const int which = (int)(gw & 1);  // 0: K, 1: V
  const long long row = gw >> 1;
  const int b = (int)(row / KVH);
  const int kvh = (int)(row - (long long)b * KVH);
  const int ctx = __ldg(context_lens + b);
  if (ctx < 1 || ctx > max_blocks * bs) return;  // the decode flags the length
  const int pos = ctx - 1;
  const int blk = __ldg(block_table + (size_t)b * max_blocks + pos / bs);
  if (blk < 0 || blk >= NB) {
    if (lane == 0) flag_error(status, PA_ERR_BLOCK_ID);
    return;
  }
  const T* src = (which ? v : k) + (size_t)b * token_stride + (size_t)kvh * D;
  warp_write_row<T, KIND, D>(src, lane, which != 0, which ? v_cache : k_cache,
                             which ? v_scales : k_scales, (size_t)blk * KVH + kvh, pos % bs, bs,
                             which ? vfix : kfix);
}

// ---------------------------------------------------------------------------------------
// Group writes (the block-granular prefill scatter and the runs of the windowed token write):
// a warp holds the 16 rows of one 16-token group of one page, each lane four consecutive
// head_dim values of every row, loaded straight into registers; the warp reduces the 16 row
// maxima together and the lane writes the quantised (or fp16) values into the page layout with
// 16-byte stores (store_group below).
// ---------------------------------------------------------------------------------------
// CTA shape of the group-write kernels (prefill_kernel, write_slots_kernel): threads, and the
// CTAs per SM their register budget is compiled for. Both kernels are bound by the latency of
// a group's dependent steps, so resident warps count: five CTAs of four warps (96 registers)
// measured 17 % faster on the windowed write than two CTAs of eight warps (116 registers);
// six CTAs spill.
#ifndef PA_GROUP_THREADS
#define PA_GROUP_THREADS 128
#endif
#ifndef PA_GROUP_MIN_CTAS
#define PA_GROUP_MIN_CTAS 5
#endif
constexpr int kGroupThreads = PA_GROUP_THREADS;
constexpr int kGroupWarps = kGroupThreads / 32;

// A lane's four consecutive input values as loaded (8 bytes for 16-bit inputs, 16 for fp32).
template <typename T> struct Raw4 { using type = uint2; };
template <> struct Raw4<float> { using type = float4; };

template <typename T>
__device__ __forceinline__ typename Raw4<T>::type load_raw4(const T* p) {
  return __ldg(reinterpret_cast<const typename Raw4<T>::type*>(p));
}
__device__ __forceinline__ void unpack4(uint2 u, const __half*, float (&x)[4]) {
  const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&u.x));
  const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&u.y));
  x[0] = a.x; x[1] = a.y; x[2] = b.x; x[3] = b.y;
}
__device__ __forceinline__ void unpack4(uint2 u, const __nv_bfloat16*, float (&x)[4]) {
  const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u.x));
  const float2 b = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u.y));
  x[0] = a.x; x[1] = a.y; x[2] = b.x; x[3] = b.y;
}
__device__ __forceinline__ void unpack4(float4 u, const float*, float (&x)[4]) {
  x[0] = u.x; x[1] = u.y; x[2] = u.z; x[3] = u.w;
}

__device__ __forceinline__ uint32_t half2_bits(float a, float b) {
  const __half2 h = __floats2half2_rn(a, b);
  return *reinterpret_cast<const uint32_t*>(&h);
}

// Packed fp32 pairs (sm_100's two-wide fp32 instructions; each half rounds as the scalar op).
__device__ __forceinline__ uint64_t f2_pack(float a, float b) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
  return r;
}
__device__ __forceinline__ void f2_unpack(uint64_t r, float& a, float& b) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(r));
}
__device__ __forceinline__ uint64_t f2_mul(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ uint64_t f2_add(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ uint64_t f2_sub(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}

// One token's four int8 bytes, quant1(x[e], s) each, as one word (element 0 in the low byte).
// y = x * inv is rounded to an integer by adding and subtracting 1.5 * 2^23, whose sum's low
// byte is the int8 byte; that is quant1 unless some y lies within 2^-14 of a half-integer
// (|y - x/s| < 2^-15 for |y| < 256, see quant_fast), or s is 0 or infinite, where the division
// decides for the whole token. With `ranged` the token also takes the division when some
// |y| >= 127.5 (the clamp); rows need that only with a fixed scale or a scale below 2^-14,
// since otherwise s = T(amax / 127) keeps every |x / s| below 127.5. The arithmetic runs on
// value pairs.
template <bool kRanged>
__device__ __forceinline__ uint32_t quant4(const float (&x)[4], float s, uint64_t inv2,
                                           bool ranged) {
  const uint64_t kr = f2_pack(12582912.f, 12582912.f);
  float dmax = 0.f, ymax = 0.f;
  uint32_t bits[4];
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const uint64_t y = f2_mul(f2_pack(x[2 * h], x[2 * h + 1]), inv2);
    const uint64_t s1 = f2_add(y, kr);
    const uint64_t d = f2_sub(y, f2_sub(s1, kr));
    float d0, d1, y0, y1, b0, b1;
    f2_unpack(d, d0, d1);
    f2_unpack(s1, b0, b1);
    dmax = fmaxf(dmax, fmaxf(fabsf(d0), fabsf(d1)));
    if (kRanged || ranged) {
      f2_unpack(y, y0, y1);
      ymax = fmaxf(ymax, fmaxf(fabsf(y0), fabsf(y1)));
    }
    bits[2 * h] = __float_as_uint(b0);
    bits[2 * h + 1] = __float_as_uint(b1);
  }
  // fmaxf drops NaN, so the scales that can produce NaN quotients (0: 0/0, and infinite: an
  // infinite element over an infinite scale) take the division explicitly; ymax stays 0 unless
  // checked.
  if (dmax < 0.5f - 0x1p-14f && ymax < 127.5f && s != 0.f && s < __int_as_float(0x7f800000))
    return __byte_perm(__byte_perm(bits[0], bits[1], 0x0040), __byte_perm(bits[2], bits[3], 0x0040),
                       0x5410);
  return ((uint32_t)(uint8_t)quant1(x[0], s)) | ((uint32_t)(uint8_t)quant1(x[1], s) << 8) |
         ((uint32_t)(uint8_t)quant1(x[2], s) << 16) | ((uint32_t)(uint8_t)quant1(x[3], s) << 24);
}

// Quantise (or round to fp16) one page's 16-token group and store it into the page layout.
// raw[t]: the lane's four consecutive input values (head_dim 4 lane .. 4 lane + 3) of token t of
// the group, zero at and past `valid`; the group starts at token offset g0 (a multiple of 16)
// of page row `page` (= block * kv_heads + kv_head). One-byte caches (I8) get per-token int8
// (or, with kfix / vfix, the fixed scales) or, with F8, per-token e4m3 (scale = amax / 448, as
// the row quantiser), and their scales; otherwise the values are rounded to fp16. Rows at and
// past `valid` are written as zeros (one-byte caches: scale 0).
//   K page [D/8][bs][8]: the lane pair (2c, 2c+1) owns 8-wide chunk c; after the pair swaps
//     half of its words, lane 2c writes the group's tokens 0-7 and lane 2c+1 tokens 8-15;
//   V page [D][bs]: lane l owns head_dim rows 4l..4l+3, 16 consecutive tokens each.
template <typename T, bool I8, int D, bool F8 = false>
__device__ __forceinline__ void store_group(const typename Raw4<T>::type (&raw)[16], bool is_v,
                                            int valid, size_t page, int g0, int bs,
                                            void* k_cache, void* v_cache, float* k_scales,
                                            float* v_scales, const float* kfix,
                                            const float* vfix, int lane) {
  static_assert(D == 128, "a lane holds four consecutive head_dim values");
  constexpr unsigned kAll = 0xffffffffu;
  constexpr int ELEM = I8 ? 1 : 2;
  constexpr int KW = I8 ? 1 : 2;  // words of a lane's four values: int8 one, fp16 two
  const int c = lane >> 1;   // K: the lane pair's 8-wide chunk
  const int hlf = lane & 1;  // K: which half of the chunk the lane holds
  uint8_t* pg =
      reinterpret_cast<uint8_t*>(is_v ? v_cache : k_cache) + page * (size_t)D * bs * ELEM;
  // Per token, the lane's four values as stored: int8 bytes (zero past the context) or fp16.
  uint32_t kw[16][KW];
  if constexpr (I8) {
    // Row maxima, reduced together: after the steps over lane masks 16, 8, 4, 2 lane l holds
    // the maximum of row (l >> 1) over its half of the lanes; mask 1 completes it.
    float m[16];
#pragma unroll
    for (int t = 0; t < 16; ++t) {
      float x[4];
      unpack4(raw[t], static_cast<const T*>(nullptr), x);
      m[t] = fmaxf(fmaxf(fabsf(x[0]), fabsf(x[1])), fmaxf(fabsf(x[2]), fabsf(x[3])));
    }
#pragma unroll
    for (int h = 8, msk = 16; h >= 1; h >>= 1, msk >>= 1) {
      const bool up = (lane & msk) != 0;
#pragma unroll
      for (int i = 0; i < h; ++i) {
        const float send = up ? m[i] : m[i + h];
        const float keep = up ? m[i + h] : m[i];
        m[i] = fmaxf(keep, __shfl_xor_sync(kAll, send, msk));
      }
    }
    const float am = fmaxf(m[0], __shfl_xor_sync(kAll, m[0], 1));
    const int row = lane >> 1;
    if constexpr (F8) {
      const float s = row < valid ? __fdiv_rn(am, 448.f) : 0.f;
      if (hlf == 0) (is_v ? v_scales : k_scales)[page * bs + g0 + row] = s;
#pragma unroll
      for (int t = 0; t < 16; ++t) {
        const float st = __shfl_sync(kAll, s, 2 * t);
        float x[4];
        unpack4(raw[t], static_cast<const T*>(nullptr), x);
        uint32_t w = 0u;
        if (st > 0.f) {
#pragma unroll
          for (int e = 0; e < 4; ++e)
            w |= (uint32_t)(uint8_t)__nv_cvt_float_to_fp8(__fdiv_rn(x[e], st), __NV_SATFINITE,
                                                          __NV_E4M3)
                 << (8 * e);
        }
        kw[t][0] = w;
      }
    } else {
      const float* fix = is_v ? vfix : kfix;
      float s = 0.f;
      if (row < valid) s = fix != nullptr ? __ldg(fix) : token_scale<T>(am);
      const float inv = __frcp_rn(s);
      if (hlf == 0) (is_v ? v_scales : k_scales)[page * bs + g0 + row] = s;
      // The clamp can bind only with a fixed scale or a scale below 2^-14 (fp16 subnormal).
      const bool ranged = __any_sync(kAll, fix != nullptr || (s > 0.f && s < 0x1p-14f));
#pragma unroll
      for (int t = 0; t < 16; ++t) {
        const float st = __shfl_sync(kAll, s, 2 * t);
        const float it = __shfl_sync(kAll, inv, 2 * t);
        float x[4];
        unpack4(raw[t], static_cast<const T*>(nullptr), x);
        kw[t][0] = t < valid ? quant4<false>(x, st, f2_pack(it, it), ranged) : 0u;
      }
    }
  } else {
#pragma unroll
    for (int t = 0; t < 16; ++t) {
      float x[4];
      unpack4(raw[t], static_cast<const T*>(nullptr), x);
      kw[t][0] = half2_bits(x[0], x[1]);
      kw[t][1] = half2_bits(x[2], x[3]);
    }
  }
  if (!is_v) {
    // The pair swaps half of its words: lane 2c keeps tokens 0-7 and receives its partner's
    // words for them, lane 2c+1 the same for tokens 8-15.
    uint32_t pw[8][KW];
#pragma unroll
    for (int i = 0; i < 8; ++i)
#pragma unroll
      for (int w = 0; w < KW; ++w)
        pw[i][w] = __shfl_xor_sync(kAll, hlf ? kw[i][w] : kw[8 + i][w], 1);
    uint8_t* dst = pg + ((size_t)c * bs + g0 + 8 * hlf) * 8 * ELEM;
#pragma unroll
    for (int i = 0; i < 8; i += (I8 ? 2 : 1)) {
      if constexpr (I8) {
        // Two tokens of 8 bytes: lane 2c's half of the chunk, then lane 2c+1's.
        const uint32_t a0 = hlf ? pw[i][0] : kw[i][0], a1 = hlf ? kw[8 + i][0] : pw[i][0];
        const uint32_t b0 = hlf ? pw[i + 1][0] : kw[i + 1][0];
        const uint32_t b1 = hlf ? kw[9 + i][0] : pw[i + 1][0];
        *reinterpret_cast<uint4*>(dst + i * 8) = make_uint4(a0, a1, b0, b1);
      } else {
        // One token of 16 bytes.
        const uint32_t l0 = hlf ? pw[i][0] : kw[i][0], l1 = hlf ? pw[i][1] : kw[i][1];
        const uint32_t h0 = hlf ? kw[8 + i][0] : pw[i][0], h1 = hlf ? kw[8 + i][1] : pw[i][1];
        *reinterpret_cast<uint4*>(dst + i * 16) = make_uint4(l0, l1, h0, h1);
      }
    }
  } else {
    // Per head_dim row 4 * lane + e, the group's 16 tokens: byte (int8) or half (fp16) e of
    // every token's word.
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      uint32_t vw[4 * KW];
#pragma unroll
      for (int u = 0; u < 4 * KW; ++u) {
        if constexpr (I8) {
          const uint32_t sel = (uint32_t)e | ((uint32_t)(4 + e) << 4);
          vw[u] = __byte_perm(__byte_perm(kw[4 * u][0], kw[4 * u + 1][0], sel),
                              __byte_perm(kw[4 * u + 2][0], kw[4 * u + 3][0], sel), 0x5410);
        } else {
          // Halves e of tokens 2u and 2u + 1.
          const uint32_t sel = (e & 1) ? 0x7632u : 0x5410u;
          vw[u] = __byte_perm(kw[2 * u][e >> 1], kw[2 * u + 1][e >> 1], sel);
        }
      }
      uint8_t* dst = pg + ((size_t)(4 * lane + e) * bs + g0) * ELEM;
#pragma unroll
      for (int u = 0; u < KW; ++u)
        *reinterpret_cast<uint4*>(dst + 16 * u) =
            make_uint4(vw[4 * u], vw[4 * u + 1], vw[4 * u + 2], vw[4 * u + 3]);
    }
  }
}

// ---------------------------------------------------------------------------------------
// Block-granular prefill over the work items (sequence, block, 16-token group of the block,
// kv head, K|V): an item inside the context writes that group of its sequence's block; tokens
// past the context in a sequence's last block are written as zeros (INT8: scale 0); items of
// blocks past the context are skipped. CTAs are persistent (as many as fit on the GPU) and
// warps stride over the items; a warp that reaches a sequence's items past its context moves
// straight on to the next sequence, so block tables sized for long contexts cost little. An
// item's rows inside the context are all requested before the first is processed.
// ---------------------------------------------------------------------------------------
template <typename T, bool I8, int D>
__global__ void __launch_bounds__(kGroupThreads, PA_GROUP_MIN_CTAS) prefill_kernel(
    const T* __restrict__ k, const T* __restrict__ v, int S, int L, int KVH,
    const int* __restrict__ block_table, const int* __restrict__ context_lens, int max_blocks,
    void* __restrict__ k_cache, void* __restrict__ v_cache, float* __restrict__ k_scales,
    float* __restrict__ v_scales, int NB, int bs, const float* __restrict__ kfix,
    const float* __restrict__ vfix, int* status) {
  using R = typename Raw4<T>::type;
  const int lane = threadIdx.x & 31;
  const int gpb = bs / 16;  // groups per block
  // A sequence's items, in the order (block, group, kv head, K|V): those of blocks inside the
  // context come first.
  const long long per_seq = (long long)max_blocks * gpb * KVH * 2;
  const long long total = (long long)S * per_seq;
  const long long first = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const long long nw = ((long long)gridDim.x * blockDim.x) >> 5;
  const int cap = min(L, max_blocks * bs);
  const size_t tstride = (size_t)KVH * D;
  const bool narrow = total <= 0xffffffffLL;  // 32-bit division suffices
  for (long long gw = first; gw < total; gw += nw) {
    const int b = narrow ? (int)((unsigned)gw / (unsigned)per_seq) : (int)(gw / per_seq);
    const int item = (int)(gw - (long long)b * per_seq);
    int ctx = __ldg(context_lens + b);
    if (ctx > cap) {
      if (lane == 0 && item == 0) flag_error(status, PA_ERR_CONTEXT_RANGE);
      ctx = cap;
    }
    if (ctx < 0) ctx = 0;
    if (item >= (ctx + bs - 1) / bs * gpb * KVH * 2) {
      // Past the sequence's last block: on to this warp's first item of the next sequence
      // (the items a warp takes are those congruent to `first` modulo nw).
      const long long next = (long long)(b + 1) * per_seq;
      gw = next + (((first - next) % nw) + nw) % nw - nw;
      continue;
    }
    const int which = item & 1;  // 0: K, 1: V
    const int kvh = (item >> 1) % KVH;
    const int jg = (item >> 1) / KVH;
    const int j = jg / gpb;
    const int t0 = j * bs + (jg - j * gpb) * 16;
    const int valid = min(16, ctx - t0);
    const int blk = __ldg(block_table + (size_t)b * max_blocks + j);
    if (blk < 0 || blk >= NB) {
      if (lane == 0) flag_error(status, PA_ERR_BLOCK_ID);
      continue;
    }
    const T* src = (which ? v : k) + ((size_t)b * L * KVH + kvh) * D + lane * 4;
    R raw[16];
#pragma unroll
    for (int t = 0; t < 16; ++t)
      raw[t] = t < valid ? load_raw4(src + (size_t)(t0 + t) * tstride) : R{};
    store_group<T, I8, D>(raw, which != 0, valid, (size_t)blk * KVH + kvh, t0 % bs, bs, k_cache,
                          v_cache, k_scales, v_scales, kfix, vfix, lane);
  }
}

// ---------------------------------------------------------------------------------------
// Token-granular write of many tokens (a prefill through slot_mapping). Tokens whose slots
// form an aligned run of 16 (slots s, s+1, ..., s+15 with s a multiple of 16, so all in one
// block when the block size is a multiple of 16) are written as one group with the prefill's
// 16-byte page stores; the other tokens row by row. Warp (window, kv head, K|V) takes the
// 16 tokens [t0, t0 + 16) of its window: from the slots of tokens t0 - 16 .. t0 + 47 it marks
// the tokens that head a run (heads are at least 16 tokens apart, so at most one lies in the
// window), writes the run headed inside its window, and writes the rows of its window's
// tokens that no run covers (token t is covered when t - slot % 16 heads a run). Those rows
// are all requested before the first is quantised.
// ---------------------------------------------------------------------------------------
template <typename T, int KIND, int D>
__global__ void __launch_bounds__(kGroupThreads, PA_GROUP_MIN_CTAS) write_slots_kernel(
    const T* __restrict__ k, const T* __restrict__ v, long long token_stride,
    const int* __restrict__ slot_mapping, int N, int KVH, void* __restrict__ k_cache,
    void* __restrict__ v_cache, float* __restrict__ k_scales, float* __restrict__ v_scales,
    int NB, int bs, const float* __restrict__ kfix, const float* __restrict__ vfix,
    int* status) {
  using R = typename Raw4<T>::type;
  constexpr bool BYTE = KIND != kRowsF16;  // one-byte cache with scales
  constexpr unsigned kAll = 0xffffffffu;
  const long long gw = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  const long long nwin = ((long long)N + 15) >> 4;
  if (gw >= nwin * KVH * 2) return;
  const int which = (int)(gw & 1);  // 0: K, 1: V
  const long long wk = gw >> 1;
  const int kvh = (int)(wk % KVH);
  const long long t0 = (wk / KVH) << 4;
  auto slot_at = [&](long long u) -> int {
    return (u >= 0 && u < N) ? __ldg(slot_mapping + u) : -1;
  };
  // a: slot of token t0 - 16 + lane; b: slot of token t0 + 16 + lane.
  const int a = slot_at(t0 - 16 + lane);
  const int b = slot_at(t0 + 16 + lane);
  int a1 = __shfl_down_sync(kAll, a, 1);
  const int b0 = __shfl_sync(kAll, b, 0);
  if (lane == 31) a1 = b0;
  const int b1 = __shfl_down_sync(kAll, b, 1);
  // Bit j of links: token t0 - 16 + j's slot is followed by the next slot.
  const unsigned la = __ballot_sync(kAll, a >= 0 && a1 == a + 1);
  const unsigned lb = __ballot_sync(kAll, lane < 31 && b >= 0 && b1 == b + 1);
  const unsigned long long links = (unsigned long long)la | ((unsigned long long)lb << 32);
  // Bit j of heads: token t0 - 16 + j heads an aligned run of 16.
  const bool head = a >= 0 && (a & 15) == 0 && ((links >> lane) & 0x7fffull) == 0x7fffull;
  const unsigned heads = __ballot_sync(kAll, head);
  // Bit i of covered: window token t0 + i lies in a run (its head among t0 + i - 15 .. t0 + i).
  const unsigned covered =
      __ballot_sync(kAll, lane < 16 && ((heads >> (lane + 1)) & 0xffffu) != 0u);
  const T* src = (which ? v : k) + (size_t)kvh * D + lane * 4;

  const unsigned own = heads >> 16;
  if (own != 0u) {
    const int i = __ffs(own) - 1;
    const int s0 = __shfl_sync(kAll, a, 16 + i);
    const int blk = s0 / bs;
    if (blk >= NB) {
      if (lane == 0) flag_error(status, PA_ERR_SLOT);
    } else {
      R raw[16];
      const T* p = src + (t0 + i) * token_stride;
#pragma unroll
      for (int t = 0; t < 16; ++t) raw[t] = load_raw4(p + t * token_stride);
      store_group<T, BYTE, D, KIND == kRowsFP8>(raw, which != 0, 16, (size_t)blk * KVH + kvh,
                                                s0 - blk * bs, bs, k_cache, v_cache, k_scales,
                                                v_scales, kfix, vfix, lane);
    }
  }

  unsigned todo = ~covered & 0xffffu;
  const long long left = (long long)N - t0;
  if (left < 16) todo &= (1u << left) - 1u;
  if (todo == 0u) return;
  R raw[16];
#pragma unroll
  for (int t = 0; t < 16; ++t)
    raw[t] = ((todo >> t) & 1u) ? load_raw4(src + (t0 + t) * token_stride) : R{};
  void* cache = which ? v_cache : k_cache;
  float* scales = which ? v_scales : k_scales;
  const float* fix = which ? vfix : kfix;
#pragma unroll
  for (int t = 0; t < 16; ++t) {
    if (!((todo >> t) & 1u)) continue;
    const int s = __shfl_sync(kAll, a, 16 + t);
    if (s < 0) continue;  // padding token
    const int blk = s / bs;
    if (blk >= NB) {
      if (lane == 0) flag_error(status, PA_ERR_SLOT);
      continue;
    }
    float x[4];
    unpack4(raw[t], static_cast<const T*>(nullptr), x);
    const RowQ<KIND, D> q = warp_quantize_vals<T, KIND, D>(x, fix);
    store_row<KIND, D>(q, lane, which != 0, cache, scales, (size_t)blk * KVH + kvh,
                       s - blk * bs, bs);
  }
}

// ---------------------------------------------------------------------------------------
// Per-tensor absmax -> scale.
// ---------------------------------------------------------------------------------------
template <typename T>
__global__ void absmax_kernel(const T* __restrict__ x, long long n, unsigned int* out) {
  float m = 0.f;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (long long)gridDim.x * blockDim.x) {
    const float a = fabsf(In<T>::ld(x + i));
    m = (a > m || a != a) ? a : m;  // keep NaN
  }
  m = warp_max(m);
  if ((threadIdx.x & 31) == 0) atomicMax(out, __float_as_uint(m));
}

template <typename T>
__global__ void scale_finalize_kernel(const unsigned int* amax_bits, float* scale_out,
                                      int semantics) {
  const float amax = __uint_as_float(*amax_bits);
  float s;
  if (semantics == PA_SCALE_CLAMP_THEN_DIVIDE) {
    s = token_scale<T>(amax);
  } else {
    s = fmaxf(In<T>::round_t(__fdiv_rn(amax, 127.f)), 1e-8f);
  }
  *scale_out = s;
}

// Token-granular writes use the windowed kernel when it has at least this many warps per SM
// (a warp walks up to 16 rows that no run covers one after another, so fewer warps would leave
// scattered writes, a decode step's appends, waiting on that walk); smaller writes take one
// warp per row.
constexpr int kSlotWindowMinWarpsPerSm = 32;

template <typename T>
cudaError_t launch_rows_t(int kind, int D, const void* k, const void* v, long long ts,
                          const int* slots, int N, int KVH, void* kc, void* vc, float* ks,
                          float* vs, int NB, int bs, const float* kf, const float* vf,
                          int* status, cudaStream_t st) {
  const long long warps = (long long)N * KVH * 2;
  const int grid = (int)((warps + 7) / 8);
  if (grid == 0) return cudaSuccess;
  const T* kk = static_cast<const T*>(k);
  const T* vv = static_cast<const T*>(v);
  if (D != 128) return cudaErrorInvalidValue;
  // Many tokens, block size a multiple of 16 and rows aligned for the lanes' vector loads: the
  // windowed write, whose aligned runs of 16 slots take the page-group stores.
  constexpr size_t kRaw = sizeof(typename Raw4<T>::type);
  const bool aligned = reinterpret_cast<uintptr_t>(k) % kRaw == 0 &&
                       reinterpret_cast<uintptr_t>(v) % kRaw == 0 &&
                       ((size_t)ts * sizeof(T)) % kRaw == 0;
  const long long wwarps = ((long long)N + 15) / 16 * KVH * 2;
  int dev = 0, sms = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e == cudaSuccess) e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (e != cudaSuccess) return e;
  if (wwarps >= (long long)sms * kSlotWindowMinWarpsPerSm && bs % 16 == 0 && aligned) {
    const int wgrid = (int)((wwarps + kGroupWarps - 1) / kGroupWarps);
    if (kind == kRowsFP8) {
      write_slots_kernel<T, kRowsFP8, 128><<<wgrid, kGroupThreads, 0, st>>>(
          kk, vv, ts, slots, N, KVH, kc, vc, ks, vs, NB, bs, nullptr, nullptr, status);
    } else if (kind == kRowsI8) {
      write_slots_kernel<T, kRowsI8, 128><<<wgrid, kGroupThreads, 0, st>>>(
          kk, vv, ts, slots, N, KVH, kc, vc, ks, vs, NB, bs, kf, vf, status);
    } else {
      write_slots_kernel<T, kRowsF16, 128><<<wgrid, kGroupThreads, 0, st>>>(
          kk, vv, ts, slots, N, KVH, kc, vc, ks, vs, NB, bs, kf, vf, status);
    }
    return cudaGetLastError();
  }
  if (kind == kRowsFP8) {
    write_rows_kernel<T, kRowsFP8, 128><<<grid, 256, 0, st>>>(kk, vv, ts, slots, N, KVH, kc, vc,
                                                              ks, vs, NB, bs, nullptr, nullptr,
                                                              status);
  } else if (kind == kRowsI8) {
    write_rows_kernel<T, kRowsI8, 128><<<grid, 256, 0, st>>>(kk, vv, ts, slots, N, KVH, kc, vc,
                                                             ks, vs, NB, bs, kf, vf, status);
  } else {
    write_rows_kernel<T, kRowsF16, 128><<<grid, 256, 0, st>>>(kk, vv, ts, slots, N, KVH, kc, vc,
                                                              ks, vs, NB, bs, kf, vf, status);
  }
  return cudaGetLastError();
}

template <typename T>
cudaError_t launch_step_rows_t(int kind, const void* k, const void* v, long long ts,
                               const int* bt, const int* cl, int max_blocks, int B, int KVH,
                               void* kc, void* vc, float* ks, float* vs, int NB, int bs,
                               const float* kf, const float* vf, int* status, cudaStream_t st) {
  const long long warps = (long long)B * KVH * 2;
  const int grid = (int)((warps + 7) / 8);
  if (grid == 0) return cudaSuccess;
  const T* kk = static_cast<const T*>(k);
  const T* vv = static_cast<const T*>(v);
  if (kind == kRowsFP8) {
    step_rows_kernel<T, kRowsFP8, 128><<<grid, 256, 0, st>>>(
        kk, vv, ts, bt, cl, max_blocks, B, KVH, kc, vc, ks, vs, NB, bs, nullptr, nullptr, status);
  } else if (kind == kRowsI8) {
    step_rows_kernel<T, kRowsI8, 128><<<grid, 256, 0, st>>>(
        kk, vv, ts, bt, cl, max_blocks, B, KVH, kc, vc, ks, vs, NB, bs, kf, vf, status);
  } else {
    step_rows_kernel<T, kRowsF16, 128><<<grid, 256, 0, st>>>(
        kk, vv, ts, bt, cl, max_blocks, B, KVH, kc, vc, ks, vs, NB, bs, nullptr, nullptr, status);
  }
  return cudaGetLastError();
}

template <typename T>
cudaError_t launch_prefill_t(bool i8, const void* k, const void* v, int S, int L, int KVH,
                             const int* bt, const int* cl, int max_blocks, void* kc, void* vc,
                             float* ks, float* vs, int NB, int bs, const float* kf,
                             const float* vf, int* status, cudaStream_t st) {
  if (S == 0 || max_blocks == 0) return cudaSuccess;
  const T* kk = static_cast<const T*>(k);
  const T* vv = static_cast<const T*>(v);
  auto kern = i8 ? prefill_kernel<T, true, 128> : prefill_kernel<T, false, 128>;
  // Persistent CTAs: as many as fit on the GPU, never more than the work items need.
  int dev = 0, sms = 0, per_sm = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e == cudaSuccess) e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (e == cudaSuccess)
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kGroupThreads, 0);
  if (e != cudaSuccess) return e;
  const long long per_seq = (long long)max_blocks * (bs / 16) * KVH * 2;
  if (per_seq > 0x7fffffffLL) return cudaErrorInvalidValue;  // items of a sequence are ints
  const long long items = (long long)S * per_seq;
  const int grid = (int)std::min<long long>((items + kGroupWarps - 1) / kGroupWarps,
                                             (long long)sms * std::max(per_sm, 1));
  kern<<<grid, kGroupThreads, 0, st>>>(kk, vv, S, L, KVH, bt, cl, max_blocks, kc, vc, ks, vs, NB,
                                       bs, kf, vf, status);
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_write_rows(int in_dtype, int kind, int D, const void* k, const void* v,
                              long long ts, const int* slots, int N, int KVH, void* kc,
                              void* vc, float* ks, float* vs, int NB, int bs, const float* kf,
                              const float* vf, int* status, cudaStream_t st) {
  switch (in_dtype) {
    case PA_DTYPE_F16:
      return launch_rows_t<__half>(kind, D, k, v, ts, slots, N, KVH, kc, vc, ks, vs, NB, bs, kf,
                                   vf, status, st);
    case PA_DTYPE_BF16:
      return launch_rows_t<__nv_bfloat16>(kind, D, k, v, ts, slots, N, KVH, kc, vc, ks, vs, NB,
                                          bs, kf, vf, status, st);
    case PA_DTYPE_F32:
      return launch_rows_t<float>(kind, D, k, v, ts, slots, N, KVH, kc, vc, ks, vs, NB, bs, kf,
                                  vf, status, st);
    default:
      return cudaErrorInvalidValue;
  }
}

cudaError_t launch_step_rows(int in_dtype, int kind, const void* k, const void* v,
                             long long ts, const int* bt, const int* cl, int max_blocks, int B,
                             int KVH, void* kc, void* vc, float* ks, float* vs, int NB, int bs,
                             const float* kf, const float* vf, int* status, cudaStream_t st) {
  switch (in_dtype) {
    case PA_DTYPE_F16:
      return launch_step_rows_t<__half>(kind, k, v, ts, bt, cl, max_blocks, B, KVH, kc, vc, ks,
                                        vs, NB, bs, kf, vf, status, st);
    case PA_DTYPE_BF16:
      return launch_step_rows_t<__nv_bfloat16>(kind, k, v, ts, bt, cl, max_blocks, B, KVH, kc,
                                               vc, ks, vs, NB, bs, kf, vf, status, st);
    case PA_DTYPE_F32:
      return launch_step_rows_t<float>(kind, k, v, ts, bt, cl, max_blocks, B, KVH, kc, vc, ks,
                                       vs, NB, bs, kf, vf, status, st);
    default:
      return cudaErrorInvalidValue;
  }
}

cudaError_t launch_prefill(int in_dtype, bool i8, const void* k, const void* v, int S, int L,
                           int KVH, const int* bt, const int* cl, int max_blocks, void* kc,
                           void* vc, float* ks, float* vs, int NB, int bs, const float* kf,
                           const float* vf, int* status, cudaStream_t st) {
  switch (in_dtype) {
    case PA_DTYPE_F16:
      return launch_prefill_t<__half>(i8, k, v, S, L, KVH, bt, cl, max_blocks, kc, vc, ks, vs,
                                      NB, bs, kf, vf, status, st);
    case PA_DTYPE_BF16:
      return launch_prefill_t<__nv_bfloat16>(i8, k, v, S, L, KVH, bt, cl, max_blocks, kc, vc,
                                             ks, vs, NB, bs, kf, vf, status, st);
    case PA_DTYPE_F32:
      return launch_prefill_t<float>(i8, k, v, S, L, KVH, bt, cl, max_blocks, kc, vc, ks, vs,
                                     NB, bs, kf, vf, status, st);
    default:
      return cudaErrorInvalidValue;
  }
}

cudaError_t launch_absmax_scale(int in_dtype, const void* x, long long n, float* scale_out,
                                int semantics, unsigned int* scratch, int num_sms,
                                cudaStream_t st) {
  cudaError_t e = cudaMemsetAsync(scratch, 0, sizeof(unsigned int), st);
  if (e != cudaSuccess) return e;
  const int grid = num_sms * 4;
  switch (in_dtype) {
    case PA_DTYPE_F16:
      if (n > 0)
        absmax_kernel<__half><<<grid, 256, 0, st>>>(static_cast<const __half*>(x), n, scratch);
      scale_finalize_kernel<__half><<<1, 1, 0, st>>>(scratch, scale_out, semantics);
      break;
    case PA_DTYPE_BF16:
      if (n > 0)
        absmax_kernel<__nv_bfloat16>
            <<<grid, 256, 0, st>>>(static_cast<const __nv_bfloat16*>(x), n, scratch);
      scale_finalize_kernel<__nv_bfloat16><<<1, 1, 0, st>>>(scratch, scale_out, semantics);
      break;
    case PA_DTYPE_F32:
      if (n > 0)
        absmax_kernel<float><<<grid, 256, 0, st>>>(static_cast<const float*>(x), n, scratch);
      scale_finalize_kernel<float><<<1, 1, 0, st>>>(scratch, scale_out, semantics);
      break;
    default:
      return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

// ---------------------------------------------------------------------------------------
// bf16 <-> fp16 activation conversions around the decode (BF16-q entry point). A bf16 value
// whose magnitude is inside the fp16 normal range converts exactly (8 significant bits fit
// in fp16's 11); larger magnitudes saturate to +-65504 and set PA_ERR_Q_RANGE; smaller ones
// round to fp16 subnormals. The fp16 decode output converts to bf16 with one rounding.
// ---------------------------------------------------------------------------------------
__global__ void bf16_to_f16_kernel(const uint4* __restrict__ in, uint4* __restrict__ out,
                                   long long n8, int* status) {
  bool bad = false;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n8;
       i += (long long)gridDim.x * blockDim.x) {
    const uint4 w = in[i];
    const uint32_t src[4] = {w.x, w.y, w.z, w.w};
    uint32_t dst[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&src[e]));
      float a = f.x, b = f.y;
      if (fabsf(a) > 65504.f) {
        bad = true;
        a = copysignf(65504.f, a);
      }
      if (fabsf(b) > 65504.f) {
        bad = true;
        b = copysignf(65504.f, b);
      }
      const __half2 h = __floats2half2_rn(a, b);
      dst[e] = *reinterpret_cast<const uint32_t*>(&h);
    }
    out[i] = make_uint4(dst[0], dst[1], dst[2], dst[3]);
  }
  if (bad) flag_error(status, PA_ERR_Q_RANGE);
}

__global__ void f16_to_bf16_kernel(const uint4* __restrict__ in, uint4* __restrict__ out,
                                   long long n8) {
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n8;
       i += (long long)gridDim.x * blockDim.x) {
    const uint4 w = in[i];
    const uint32_t src[4] = {w.x, w.y, w.z, w.w};
    uint32_t dst[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&src[e]));
      const __nv_bfloat162 h = __floats2bfloat162_rn(f.x, f.y);
      dst[e] = *reinterpret_cast<const uint32_t*>(&h);
    }
    out[i] = make_uint4(dst[0], dst[1], dst[2], dst[3]);
  }
}

cudaError_t launch_bf16_to_f16(const void* in, void* out, long long n, int* status, int num_sms,
                               cudaStream_t st) {
  const long long n8 = n / 8;
  if (n8 == 0) return cudaSuccess;
  long long want = (n8 + 255) / 256;
  const int grid = (int)(want < num_sms * 4LL ? want : num_sms * 4LL);
  bf16_to_f16_kernel<<<grid, 256, 0, st>>>(static_cast<const uint4*>(in),
                                           static_cast<uint4*>(out), n8, status);
  return cudaGetLastError();
}

cudaError_t launch_f16_to_bf16(const void* in, void* out, long long n, int num_sms,
                               cudaStream_t st) {
  const long long n8 = n / 8;
  if (n8 == 0) return cudaSuccess;
  long long want = (n8 + 255) / 256;
  const int grid = (int)(want < num_sms * 4LL ? want : num_sms * 4LL);
  f16_to_bf16_kernel<<<grid, 256, 0, st>>>(static_cast<const uint4*>(in),
                                           static_cast<uint4*>(out), n8);
  return cudaGetLastError();
}

}  // namespace pa
