// Cache-write kernels for B200: per-token symmetric INT8 quantize-into-cache, FP16
// copy-into-cache, block-granular prefill scatter, and the per-tensor absmax scale.
//
// The per-row quantisation (bit-exact with the reference's quantize_per_token,
// tests/paged_decode_attn.py:106-112) lives in pa_rows.cuh, shared with the decode step's fused
// new-token write. These kernels are built without fast-math so the divides stay IEEE.

#include "pa_common.cuh"
#include "pa_internal.h"
#include "pa_rows.cuh"

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
// Block-granular prefill: one CTA per (block j, kv-head, sequence). The block's K and V rows
// are loaded with one vector load per lane and row, several rows in flight per warp, quantised
// (or rounded) into shared memory, and written as whole K and V pages with 16-byte stores,
// then the scales. Tokens past the context are written as zeros with scale 0.
// ---------------------------------------------------------------------------------------
constexpr int kPrefillThreads = 256;

// The four consecutive input values of one lane (8 bytes for 16-bit inputs, 16 for fp32).
__device__ __forceinline__ void load4(const __half* p, float (&x)[4]) {
  const uint2 u = __ldg(reinterpret_cast<const uint2*>(p));
  const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&u.x));
  const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&u.y));
  x[0] = a.x; x[1] = a.y; x[2] = b.x; x[3] = b.y;
}
__device__ __forceinline__ void load4(const __nv_bfloat16* p, float (&x)[4]) {
  const uint2 u = __ldg(reinterpret_cast<const uint2*>(p));
  const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u.x));
  const float2 b = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u.y));
  x[0] = a.x; x[1] = a.y; x[2] = b.x; x[3] = b.y;
}
__device__ __forceinline__ void load4(const float* p, float (&x)[4]) {
  const float4 u = __ldg(reinterpret_cast<const float4*>(p));
  x[0] = u.x; x[1] = u.y; x[2] = u.z; x[3] = u.w;
}

template <typename T, bool I8, int D>
__global__ void __launch_bounds__(kPrefillThreads) prefill_kernel(
    const T* __restrict__ k, const T* __restrict__ v, int L, int KVH,
    const int* __restrict__ block_table, const int* __restrict__ context_lens, int max_blocks,
    void* __restrict__ k_cache, void* __restrict__ v_cache, float* __restrict__ k_scales,
    float* __restrict__ v_scales, int NB, int bs, const float* __restrict__ kfix,
    const float* __restrict__ vfix, int* status) {
  static_assert(D == 128, "a lane loads four consecutive head_dim values");
  using OutT = typename std::conditional<I8, int8_t, __half>::type;
  constexpr int ELEM = sizeof(OutT);
  constexpr int NW = kPrefillThreads / 32;
  constexpr int RB = 4;  // rows per warp whose loads are in flight together
  extern __shared__ __align__(16) uint8_t sm[];
  OutT* kq = reinterpret_cast<OutT*>(sm);                              // [bs][D]
  OutT* vq = kq + (size_t)bs * D;                                      // [bs][D]
  float* ksm = reinterpret_cast<float*>(sm + 2 * (size_t)bs * D * ELEM);  // [bs]
  float* vsm = ksm + bs;                                               // [bs]

  const int j = blockIdx.x;
  const int kvh = blockIdx.y;
  const int b = blockIdx.z;
  int ctx = __ldg(context_lens + b);
  const int cap = min(L, max_blocks * bs);
  if (ctx > cap) {
    if (threadIdx.x == 0 && j == 0 && kvh == 0) flag_error(status, PA_ERR_CONTEXT_RANGE);
    ctx = cap;
  }
  if (ctx < 0) ctx = 0;
  const int nblk = (ctx + bs - 1) / bs;
  if (j >= nblk) return;
  const int blk = __ldg(block_table + (size_t)b * max_blocks + j);
  if (blk < 0 || blk >= NB) {
    if (threadIdx.x == 0) flag_error(status, PA_ERR_BLOCK_ID);
    return;
  }
  const int t0 = j * bs;
  const int valid = min(bs, ctx - t0);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const size_t page = (size_t)blk * KVH + kvh;

  // Rows 0 .. bs-1 are K rows, bs .. 2bs-1 V rows; warp w takes rows w, w + NW, ...
  for (int r0 = warp; r0 < 2 * bs; r0 += NW * RB) {
    float x[RB][4];
#pragma unroll
    for (int rb = 0; rb < RB; ++rb) {
      const int r = r0 + rb * NW;
      const int i = r < bs ? r : r - bs;
      if (r < 2 * bs && i < valid) {
        load4((r < bs ? k : v) + (((size_t)b * L + t0 + i) * KVH + kvh) * D + lane * 4, x[rb]);
      } else {
#pragma unroll
        for (int e = 0; e < 4; ++e) x[rb][e] = 0.f;
      }
    }
#pragma unroll
    for (int rb = 0; rb < RB; ++rb) {
      const int r = r0 + rb * NW;
      if (r >= 2 * bs) break;  // uniform across the warp
      const bool is_v = r >= bs;
      const int i = is_v ? r - bs : r;
      OutT* q = (is_v ? vq : kq) + (size_t)i * D + lane * 4;
      if constexpr (I8) {
        const float* fix = is_v ? vfix : kfix;
        float s;
        if (i >= valid) {
          s = 0.f;
        } else if (fix != nullptr) {
          s = __ldg(fix);
        } else {
          float am = 0.f;
#pragma unroll
          for (int e = 0; e < 4; ++e) am = fmaxf(am, fabsf(x[rb][e]));
          am = warp_max(am);
          s = token_scale<T>(am);
        }
        int8_t qv[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) qv[e] = (i < valid) ? quant1(x[rb][e], s) : (int8_t)0;
        *reinterpret_cast<uint32_t*>(q) = *reinterpret_cast<const uint32_t*>(qv);
        if (lane == 0) (is_v ? vsm : ksm)[i] = s;
      } else {
        const __half2 h0 = __floats2half2_rn(x[rb][0], x[rb][1]);
        const __half2 h1 = __floats2half2_rn(x[rb][2], x[rb][3]);
        *reinterpret_cast<uint2*>(q) = make_uint2(*reinterpret_cast<const uint32_t*>(&h0),
                                                  *reinterpret_cast<const uint32_t*>(&h1));
      }
    }
  }
  __syncthreads();

  constexpr int PER16 = 16 / ELEM;  // elements per 16-byte store
  const int units = D * bs / PER16;
  for (int which = 0; which < 2; ++which) {
    const OutT* q_sm = which ? vq : kq;
    OutT* pg = reinterpret_cast<OutT*>(which ? v_cache : k_cache) + page * (size_t)D * bs;
    for (int u = threadIdx.x; u < units; u += blockDim.x) {
      alignas(16) OutT tmp[PER16];
      const int e0 = u * PER16;  // element offset inside the page
      if (which == 0) {
        // K page [D/8][bs][8]: element e0 -> chunk c, token t, lane-in-chunk w
#pragma unroll
        for (int e = 0; e < PER16; ++e) {
          const int el = e0 + e;
          const int c = el / (bs * 8);
          const int rem = el - c * bs * 8;
          const int t = rem >> 3;
          const int w = rem & 7;
          tmp[e] = q_sm[t * D + c * 8 + w];
        }
      } else {
        // V page [D][bs]
#pragma unroll
        for (int e = 0; e < PER16; ++e) {
          const int el = e0 + e;
          const int d = el / bs;
          const int t = el - d * bs;
          tmp[e] = q_sm[t * D + d];
        }
      }
      *reinterpret_cast<uint4*>(pg + e0) = *reinterpret_cast<const uint4*>(tmp);
    }
  }
  if constexpr (I8) {
    for (int t = threadIdx.x; t < 2 * bs; t += blockDim.x) {
      if (t < bs) k_scales[page * bs + t] = ksm[t];
      else v_scales[page * bs + t - bs] = vsm[t - bs];
    }
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
  const dim3 grid(max_blocks, KVH, S);
  const T* kk = static_cast<const T*>(k);
  const T* vv = static_cast<const T*>(v);
  // Shared memory: the quantised K and V rows of one block plus their scales.
  const size_t smem = 2 * (size_t)bs * 128 * (i8 ? 1 : 2) + 2 * (size_t)bs * 4;
  auto kern = i8 ? prefill_kernel<T, true, 128> : prefill_kernel<T, false, 128>;
  if (smem > 48 * 1024) {
    const cudaError_t e =
        cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
  }
  kern<<<grid, kPrefillThreads, smem, st>>>(kk, vv, L, KVH, bt, cl, max_blocks, kc, vc, ks, vs,
                                            NB, bs, kf, vf, status);
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
