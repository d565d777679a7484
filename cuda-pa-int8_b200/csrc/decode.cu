// Paged-attention decode kernels for B200 (sm_100a): FP16, per-token INT8 and per-token FP8
// (e4m3) KV caches.
//
// Design (one kernel family, three modes, see pa_internal.h):
//  * A warp is an independent decode engine. It owns a DEPTH-deep ring of shared-memory
//    stages; its lane 0 fills them with TMA copies (the K tile through a tensor map with the
//    128-byte swizzle, V and the per-token scales through 1-D bulk copies or tensor maps) and
//    the whole warp consumes them. A stage holds one 16-token "subpage" of one
//    (block, kv-head) page: K and V tiles plus, for INT8 and FP8, 16 K scales and 16 V
//    scales. The ranges are walked piece by piece (a warp's pages inside one segment).
//  * Every CTA first scans context_lens (all sequences, kept in shared memory) and then the
//    flattened work list "sequence x kv-head x head-tile x subpage" is cut into equal page
//    ranges, one per warp (stream mode), so ragged batches and long contexts are balanced.
//    A warp whose range cuts a segment (one sequence x kv-head) writes an un-normalised
//    partial (O, m, l); the last warp to finish a segment (atomic arrival counter) merges the
//    partials with the log-sum-exp rule and writes the fp16 output. Split mode instead snaps
//    the ranges to 512-token splits and writes one partial per split for the reduce kernel
//    (the split-K pair); partial mode writes one merged partial per segment (cross-GPU).
//  * All q heads of a GQA group share one pass over the K/V page: QK^T and PV run on the
//    tensor cores (mma.sync m16n8k16, f16 in / f32 accumulate) with heads on the MMA rows
//    (QK) or columns (PV), so K and V are read from HBM once per kv-head. INT8: QK runs on
//    the integer tensor cores (m16n8k32) on the raw K bytes against q written exactly enough
//    as three int8 parts over a power-of-two scale; V bytes unpack to exact fp16 integers in
//    registers. FP8: K and V bytes convert to fp16 exactly (hardware e4m3x2 -> f16x2). The
//    per-token K scale multiplies the dot product and the per-token V scale is folded into
//    the softmax weight (the dequant
//    fusion of kernels/paged_attention_v5_warp_int8.cu:82-85,101-108); the weights enter the
//    PV MMA as two fp16 parts (hi + lo), so the output tracks the reference's fp32 arithmetic
//    to about 1e-5 even where attention concentrates on a few large V entries.
//
// Arithmetic follows the reference decode (tests/paged_decode_attn.py:4-49 and the split-K
// pair kernels/paged_attention_v4_splitk.cu:28-187): softmax(scale * q.k) v over the tokens
// of each sequence gathered through block_table, with online (running max) softmax and the
// split merge  m = max m_s,  l = sum l_s e^{m_s - m},  o = sum o_s e^{m_s - m} / l.
// Scores are kept in log2 units (scale * log2 e) so the exponentials are exp2.

#include "pa_common.cuh"
#include "pa_internal.h"
#include "pa_rows.cuh"

#include <atomic>
#include <cstdio>

namespace pa {
namespace {

// Per-lane chunk (8 head-dim values) used by load `si` of lane group position r.
// INT8 K tiles (128-byte rows = one chunk, 16 tokens x 8 bytes) and FP16 K tiles (two
// 128-byte rows per chunk) are stored with the TMA 128-byte swizzle; these chunk orders make
// every shared-memory K load of a warp hit 32 distinct banks.
__device__ __forceinline__ int chunk_i8(int r, int si) {
  return ((r & 1) | ((r & 2) << 1)) + ((si >> 1) << 3) + ((si & 1) << 1);
}
__device__ __forceinline__ int chunk_f16(int r, int si) { return r + 4 * si; }

// Offset of the 16 V scales inside an INT8 stage's scale tile (K scales sit at 0).
constexpr int kVsOff = 128;

// log2 of the factor by which the decode loop forms its softmax weights (2^6): large enough
// to keep the hi/lo fp16 parts of the weights normal, small enough that weight x V scale stays
// below the fp16 maximum for any fp16-derived scale (V scale <= 65504 / 127).
constexpr float kPExp = 6.f;

template <int KVK, int D, int GT, int DEPTH, int WARPS>
struct Tile {
  static constexpr bool I8 = KVK == 1;    // int8 values, per-token scales
  static constexpr bool F8 = KVK == 2;    // fp8 e4m3 values, per-token scales
  static constexpr bool BYTE = KVK != 0;  // one-byte elements (the INT8 page layout)
  static constexpr int ELEM = BYTE ? 1 : 2;
  static constexpr int KT = D * kSubTokens * ELEM;  // K tile bytes
  static constexpr int VT = D * kSubTokens * ELEM;  // V tile bytes
  // Scale tiles: 16 K scales at +0 and 16 V scales at +128 (tensor-copy destinations are
  // kept 128-byte aligned); 128 bytes of them are transferred per stage.
  static constexpr int ST = BYTE ? 256 : 0;
  static constexpr uint32_t TX = KT + VT + (BYTE ? 128 : 0);  // bytes delivered per stage
  static constexpr int NS = D / 32;                 // 8-value K loads per token per lane
  static constexpr int MT = D / 16;                 // PV m-tiles (head_dim rows)
  static constexpr int NT = GT / 8;                 // PV n-tiles (heads)
  static constexpr int SLOT = (D + 2) * GT;         // partial slot floats
  static constexpr size_t SMEM = 1024 + (size_t)WARPS * DEPTH * (KT + VT + ST) +
                                 (size_t)WARPS * DEPTH * 8;
  // Decode step launches: per stage, the new token's K and V rows (16-bit) when the stage's
  // page holds a sequence's new token.
  static constexpr int NR = 2 * D * 2;
  static constexpr size_t SMEM_STEP = SMEM + 16 + (size_t)WARPS * DEPTH * NR;
};

// ---------------------------------------------------------------------------------------
// Log-sum-exp merge of `np` partial slots by one warp, from copies of the slots in shared
// memory: the lanes bulk-copy the slots into `stage` (np * SLOT floats) on the warp's
// mbarrier `bar`, so a merge waits for one L2 round trip however many pieces it has. Sums
// run in piece order (k = 0, 1, ...): the arithmetic, and the output's bits, are the same
// whichever CTA performs the merge. Piece k of the segment is warp (wf + k)'s slot: slot
// 2 (wf + k) + 1 for the first piece (it starts the segment), 2 (wf + k) for the others.
// Returns false (status flagged) if the copies did not arrive within the wait limit; the
// caller then stops using the staging memory. Out of line: it runs a few times per CTA at
// the end of the launch and should not add to the page loop's registers.
// ---------------------------------------------------------------------------------------
template <int D, int GT>
__device__ __noinline__ bool staged_combine(const float* part, int wf, int np, int lane,
                                            int hcnt, __half* out_rows, float* out_slot,
                                            int* status, float* stage, uint64_t* bar,
                                            uint32_t parity) {
  constexpr int SLOT = (D + 2) * GT;
  constexpr uint32_t SB = SLOT * sizeof(float);
  constexpr int O4 = D * GT / 4 / 32;  // float4 outputs per lane
  static_assert(D * GT / 4 % 32 == 0, "outputs must tile the warp");
  // Earlier generic accesses (the ring's last reads, a previous merge's use of the staging
  // memory, the acquire that made the slots visible) come before the copies.
  fence_proxy_async_all();
  if (lane == 0) mbar_arrive_expect_tx(bar, (uint32_t)np * SB);
  __syncwarp();
  for (int k = lane; k < np; k += 32)
    bulk_g2s(stage + (size_t)k * SLOT, part + ((size_t)(wf + k) * 2 + (k == 0 ? 1 : 0)) * SLOT,
             SB, bar);
  if (!mbar_wait_bounded(bar, parity, status)) return false;

  // Weights: lane h < GT takes head h, M = max_k m_k, w_k = 2^(m_k - M) (written over m_k in
  // the staged slot), L = sum_k w_k l_k.
  float Lh = 0.f, Mh = neg_inf();
  if (lane < GT) {
    for (int k = 0; k < np; ++k) Mh = fmaxf(Mh, stage[(size_t)k * SLOT + D * GT + lane]);
    for (int k = 0; k < np; ++k) {
      float* mk = stage + (size_t)k * SLOT + D * GT + lane;
      const float w = (Mh == neg_inf()) ? 0.f : ex2(*mk - Mh);
      *mk = w;
      Lh = fmaf(w, mk[GT], Lh);
    }
  }
  __syncwarp();

  // O = sum_k w_k O_k. Slots hold O as [D][GT]; float4 o covers row o / (GT/4), heads
  // h0..h0+3 with h0 = 4 (o % (GT/4)), which is the same for all of a lane's outputs.
  const int h0 = 4 * (lane % (GT / 4));
  float4 acc[O4];
#pragma unroll
  for (int i = 0; i < O4; ++i) acc[i] = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int k = 0; k < np; ++k) {
    const float* sk = stage + (size_t)k * SLOT;
    const float4 w4 = *reinterpret_cast<const float4*>(sk + D * GT + h0);
#pragma unroll
    for (int i = 0; i < O4; ++i) {
      const float4 v = reinterpret_cast<const float4*>(sk)[lane + 32 * i];
      acc[i].x = fmaf(w4.x, v.x, acc[i].x);
      acc[i].y = fmaf(w4.y, v.y, acc[i].y);
      acc[i].z = fmaf(w4.z, v.z, acc[i].z);
      acc[i].w = fmaf(w4.w, v.w, acc[i].w);
    }
  }
  if (out_rows != nullptr) {
    float inv[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float L = __shfl_sync(0xffffffffu, Lh, h0 + e);
      inv[e] = L > 0.f ? 1.f / L : 0.f;
    }
    if (lane < hcnt && !(Lh > 0.f)) flag_error(status, PA_ERR_EMPTY_CONTEXT);
#pragma unroll
    for (int i = 0; i < O4; ++i) {
      const int d = (lane + 32 * i) / (GT / 4);
      const float a4[4] = {acc[i].x, acc[i].y, acc[i].z, acc[i].w};
#pragma unroll
      for (int e = 0; e < 4; ++e)
        if (h0 + e < hcnt) out_rows[(size_t)(h0 + e) * D + d] = __float2half_rn(a4[e] * inv[e]);
    }
  } else {
#pragma unroll
    for (int i = 0; i < O4; ++i) reinterpret_cast<float4*>(out_slot)[lane + 32 * i] = acc[i];
    if (lane < GT) {
      out_slot[D * GT + lane] = Mh;
      out_slot[D * GT + GT + lane] = Lh;
    }
  }
  return true;
}

// ---------------------------------------------------------------------------------------
// CTA-cooperative log-sum-exp merge of `np` partial slots (all NTHR threads of the block take
// part; scratch is shared memory). Pass 1 forms the maxima, the per-piece weights (kept in
// shared memory) and the denominators with every thread reading a different piece; pass 2
// gives each thread one float4 of the [D][GT] output and U pieces' loads in flight per step,
// so a merge costs a handful of dependent L2 round trips however many pieces there are.
// ---------------------------------------------------------------------------------------
template <int D, int GT, int NTHR, int U>
struct Coop {
  static constexpr int OUT4 = D * GT / 4;                        // float4 outputs
  static constexpr int PG = NTHR >= OUT4 ? NTHR / OUT4 : 1;      // piece groups
  static constexpr int OPT = NTHR >= OUT4 ? 1 : OUT4 / NTHR;     // outputs per thread
  static constexpr int NW = NTHR / 32;
  // Scratch floats needed for np pieces.
  __host__ __device__ static constexpr size_t floats(int np) {
    return 2 * GT + NW * GT + ((size_t)np * GT + 3) / 4 * 4 + (size_t)PG * OUT4 * 4;
  }
};

template <int D, int GT, int NTHR, int U, typename PieceFn>
__device__ __forceinline__ void coop_combine(PieceFn piece, int np, int hcnt, __half* out_rows,
                                             float* out_slot, int* status, float* sm) {
  using CC = Coop<D, GT, NTHR, U>;
  static_assert(NTHR >= CC::OUT4 || CC::OUT4 % NTHR == 0, "outputs must tile the block");
  const int tid = threadIdx.x;
  const int lane = tid & 31, warp = tid >> 5;
  float* sM = sm;
  float* sL = sm + GT;
  float* sRed = sm + 2 * GT;
  float* sW = sRed + CC::NW * GT;
  float4* sAcc = reinterpret_cast<float4*>(sW + ((size_t)np * GT + 3) / 4 * 4);

  float mx[GT];
#pragma unroll
  for (int h = 0; h < GT; ++h) mx[h] = neg_inf();
  for (int k = tid; k < np; k += NTHR) {
    const float4* mk = reinterpret_cast<const float4*>(piece(k) + D * GT);
#pragma unroll
    for (int h4 = 0; h4 < GT / 4; ++h4) {
      const float4 v = __ldcg(mk + h4);
      mx[4 * h4 + 0] = fmaxf(mx[4 * h4 + 0], v.x);
      mx[4 * h4 + 1] = fmaxf(mx[4 * h4 + 1], v.y);
      mx[4 * h4 + 2] = fmaxf(mx[4 * h4 + 2], v.z);
      mx[4 * h4 + 3] = fmaxf(mx[4 * h4 + 3], v.w);
    }
  }
#pragma unroll
  for (int h = 0; h < GT; ++h) {
    const float v = warp_max(mx[h]);
    if (lane == 0) sRed[warp * GT + h] = v;
  }
  __syncthreads();
  if (tid < GT) {
    float v = neg_inf();
    for (int w = 0; w < CC::NW; ++w) v = fmaxf(v, sRed[w * GT + tid]);
    sM[tid] = v;
  }
  __syncthreads();
  float ls[GT];
#pragma unroll
  for (int h = 0; h < GT; ++h) ls[h] = 0.f;
  for (int k = tid; k < np; k += NTHR) {
    const float4* mk = reinterpret_cast<const float4*>(piece(k) + D * GT);
#pragma unroll
    for (int h4 = 0; h4 < GT / 4; ++h4) {
      const float4 m4 = __ldcg(mk + h4);
      const float4 l4 = __ldcg(mk + GT / 4 + h4);
      const float mm[4] = {m4.x, m4.y, m4.z, m4.w};
      const float ll[4] = {l4.x, l4.y, l4.z, l4.w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int h = 4 * h4 + e;
        const float M = sM[h];
        const float w = (M == neg_inf()) ? 0.f : ex2(mm[e] - M);
        sW[(size_t)k * GT + h] = w;
        ls[h] += w * ll[e];
      }
    }
  }
#pragma unroll
  for (int h = 0; h < GT; ++h) {
    float v = ls[h];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    if (lane == 0) sRed[warp * GT + h] = v;
  }
  __syncthreads();
  if (tid < GT) {
    float v = 0.f;
    for (int w = 0; w < CC::NW; ++w) v += sRed[w * GT + tid];
    sL[tid] = v;
  }
  __syncthreads();

  const int pg = (NTHR >= CC::OUT4) ? tid / CC::OUT4 : 0;
  float4 acc[CC::OPT];
#pragma unroll
  for (int i = 0; i < CC::OPT; ++i) acc[i] = make_float4(0.f, 0.f, 0.f, 0.f);
  if (pg < CC::PG) {
#pragma unroll
    for (int i = 0; i < CC::OPT; ++i) {
      const int o = (NTHR >= CC::OUT4) ? tid % CC::OUT4 : tid + i * NTHR;
      const int h0 = (o % (GT / 4)) * 4;
      for (int k0 = pg; k0 < np; k0 += CC::PG * U) {
        float4 v[U];
#pragma unroll
        for (int u = 0; u < U; ++u) {
          const int k = k0 + u * CC::PG;
          v[u] = (k < np) ? __ldcg(reinterpret_cast<const float4*>(piece(k)) + o)
                          : make_float4(0.f, 0.f, 0.f, 0.f);
        }
#pragma unroll
        for (int u = 0; u < U; ++u) {
          const int k = k0 + u * CC::PG;
          if (k < np) {
            const float* w = sW + (size_t)k * GT + h0;
            acc[i].x += w[0] * v[u].x;
            acc[i].y += w[1] * v[u].y;
            acc[i].z += w[2] * v[u].z;
            acc[i].w += w[3] * v[u].w;
          }
        }
      }
    }
  }
  if constexpr (CC::PG > 1) {
    if (pg < CC::PG) sAcc[pg * CC::OUT4 + tid % CC::OUT4] = acc[0];
    __syncthreads();
    if (pg == 0) {
      for (int g2 = 1; g2 < CC::PG; ++g2) {
        const float4 t = sAcc[g2 * CC::OUT4 + tid];
        acc[0].x += t.x;
        acc[0].y += t.y;
        acc[0].z += t.z;
        acc[0].w += t.w;
      }
    }
  }
  if (pg == 0) {
#pragma unroll
    for (int i = 0; i < CC::OPT; ++i) {
      const int o = (NTHR >= CC::OUT4) ? tid : tid + i * NTHR;
      const int d = o / (GT / 4);
      const int h0 = (o % (GT / 4)) * 4;
      const float a4[4] = {acc[i].x, acc[i].y, acc[i].z, acc[i].w};
      if (out_rows != nullptr) {
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int h = h0 + e;
          if (h < hcnt) {
            const float L = sL[h];
            out_rows[(size_t)h * D + d] = __float2half_rn(L > 0.f ? a4[e] / L : 0.f);
          }
        }
      } else {
        reinterpret_cast<float4*>(out_slot)[o] = acc[i];
      }
    }
  }
  if (tid < GT) {
    if (out_slot != nullptr) {
      out_slot[D * GT + tid] = sM[tid];
      out_slot[D * GT + GT + tid] = sL[tid];
    } else if (tid < hcnt && !(sL[tid] > 0.f)) {
      flag_error(status, PA_ERR_EMPTY_CONTEXT);
    }
  }
  __syncthreads();
}

// ---------------------------------------------------------------------------------------
// Decode step: the new token's rows in a stage (bulk-copied with the page, rk = K row then V
// row, 16-bit) are quantised like the cache writes, placed into the staged page at token t of
// the subpage (the copy brought the slot's previous contents), and stored into the cache at
// page row `row`, offset `off` for later steps. Only the calling warp reads the page, so
// nothing orders the global stores against the copies. Kept out of line: it runs once per
// segment, and inlined into the page loop it made every page slower.
// ---------------------------------------------------------------------------------------
template <int KVK, int D>
__device__ __noinline__ void stage_new_token(const uint8_t* rk, uint8_t* kt, uint8_t* vt,
                                             uint8_t* sd, int lane, int row, int t, int off,
                                             int new_dtype, const float* kfix,
                                             const float* vfix, void* kc, void* vc, float* ks,
                                             float* vs, int bs) {
  static_assert(D == 128, "one lane per four head_dim values");
  constexpr bool BYTE = KVK != 0;
  constexpr int KIND = KVK == 1 ? kRowsI8 : (KVK == 2 ? kRowsFP8 : kRowsF16);
  RowQ<KIND, D> qk, qv;
  if (new_dtype == PA_DTYPE_BF16) {
    qk = warp_quantize_row<__nv_bfloat16, KIND, D>(reinterpret_cast<const __nv_bfloat16*>(rk),
                                                   lane, kfix);
    qv = warp_quantize_row<__nv_bfloat16, KIND, D>(
        reinterpret_cast<const __nv_bfloat16*>(rk + D * 2), lane, vfix);
  } else {
    qk = warp_quantize_row<__half, KIND, D>(reinterpret_cast<const __half*>(rk), lane, kfix);
    qv = warp_quantize_row<__half, KIND, D>(reinterpret_cast<const __half*>(rk + D * 2), lane,
                                            vfix);
  }
  const int c = lane >> 1;  // the 8-wide head_dim chunk of this lane's four values
  if constexpr (BYTE) {
    const int o = c * 128 + ((((t >> 1) ^ (c & 7)) << 4) | ((t & 1) << 3)) + 4 * (lane & 1);
    *reinterpret_cast<uint32_t*>(kt + o) = qk.w[0];
#pragma unroll
    for (int e = 0; e < 4; ++e) vt[(4 * lane + e) * kSubTokens + t] = (uint8_t)row_elem(qv, e);
    if (lane == 0) {
      reinterpret_cast<float*>(sd)[t] = qk.s;
      reinterpret_cast<float*>(sd + kVsOff)[t] = qv.s;
    }
  } else {
    const int rr = 2 * c + (t >> 3);
    const int o = rr * 128 + (((t & 7) ^ (rr & 7)) << 4) + 8 * (lane & 1);
    *reinterpret_cast<uint2*>(kt + o) = make_uint2(qk.w[0], qk.w[1]);
#pragma unroll
    for (int e = 0; e < 4; ++e)
      reinterpret_cast<uint16_t*>(vt)[(4 * lane + e) * kSubTokens + t] =
          (uint16_t)row_elem(qv, e);
  }
  store_row(qk, lane, false, kc, ks, (size_t)row, off, bs);
  store_row(qv, lane, true, vc, vs, (size_t)row, off, bs);
  __syncwarp();
}

// ---------------------------------------------------------------------------------------
// The decode kernel.
// ---------------------------------------------------------------------------------------
template <int KVK, int D, int GT, int DEPTH, int WARPS>
__global__ void __launch_bounds__(WARPS * 32, 1)
    decode_kernel(const DecodeArgs a, const __grid_constant__ CUtensorMap tm_k,
                  const __grid_constant__ CUtensorMap tm_v,
                  const __grid_constant__ CUtensorMap tm_ks,
                  const __grid_constant__ CUtensorMap tm_vs) {
  using C = Tile<KVK, D, GT, DEPTH, WARPS>;
  constexpr bool I8 = C::I8;
  constexpr bool F8 = C::F8;
  constexpr bool BYTE = C::BYTE;
  constexpr int NS = C::NS;
  constexpr int MT = C::MT;
  constexpr int NT = C::NT;
  constexpr int SLOT = C::SLOT;
  constexpr int NTHR = WARPS * 32;

  __shared__ int s_pre[kBMax + 1];
  __shared__ int s_ctx[kBMax];
  __shared__ int s_tmp[32];
  __shared__ int s_empty;
  __shared__ unsigned s_over[kBMax / 32];  // sequences whose context exceeds the table
  __shared__ int s_pend[WARPS][2][6];
  __shared__ int s_npend[WARPS];
  __shared__ int s_wrow[WARPS][DEPTH];  // decode step: page row whose new token a stage holds
  __shared__ uint64_t s_mmb[WARPS];     // per-warp barrier of the end-of-launch merges
  __shared__ int s_nblk[WARPS][32];     // block ids of a warp's next batch of pages
  __shared__ int s_nmeta[WARPS][32];    // their (kv_head << 3) | subpage
  __shared__ int s_nwr[WARPS][32];      // their decode-step new-token sequence, or -1
  extern __shared__ __align__(16) uint8_t dsm_raw[];

  uint8_t* dsm = dsm_raw + ((1024u - (smem_u32(dsm_raw) & 1023u)) & 1023u);
  uint8_t* k_tiles = dsm;
  uint8_t* v_tiles = k_tiles + WARPS * DEPTH * C::KT;
  uint8_t* s_tiles = v_tiles + WARPS * DEPTH * C::VT;
  uint64_t* bars = reinterpret_cast<uint64_t*>(s_tiles + WARPS * DEPTH * C::ST);
  // New-token rows of a decode step (allocated only for step launches).
  uint8_t* r_tiles = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(bars + WARPS * DEPTH) + 15) & ~uintptr_t(15));

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int g = lane >> 2;  // MMA group (row / column index)
  const int r = lane & 3;   // position inside the group
  uint64_t* wbar = bars + warp * DEPTH;

  if (lane == 0) {
#pragma unroll
    for (int s = 0; s < DEPTH; ++s) mbar_init(&wbar[s], 1);
    mbar_init(&s_mmb[warp], 1);
    fence_mbar_init();
  }
  if (threadIdx.x == 0) {
    s_empty = 0;
    // This CTA's share of the block tables and q rows into L2, so the first block-id and q
    // reads after the scan do not each wait for DRAM.
    prefetch_l2_share(a.block_table, (size_t)a.B * a.max_blocks * sizeof(int), blockIdx.x,
                      gridDim.x);
    prefetch_l2_share(a.q, (size_t)a.B * a.H * D * sizeof(__half), blockIdx.x, gridDim.x);
    if (a.new_k != nullptr) {
      const size_t nb = (size_t)a.B * a.new_stride * (a.new_dtype == PA_DTYPE_F32 ? 4 : 2);
      prefetch_l2_share(a.new_k, nb, blockIdx.x, gridDim.x);
      prefetch_l2_share(a.new_v, nb, blockIdx.x, gridDim.x);
    }
    prefetch_tensormap(&tm_k);
    if (!a.bulk) {
      prefetch_tensormap(&tm_v);
      if constexpr (BYTE) {
        prefetch_tensormap(&tm_ks);
        prefetch_tensormap(&tm_vs);
      }
    }
  }

  // ---- 1. Scan of per-sequence page counts (all CTAs, identical result) -------------------
  const int SEGS = a.KVH * a.HT;
  const int cap = a.max_blocks * a.bs;
  int carry = 0;
  for (int i = threadIdx.x; i < kBMax / 32; i += NTHR) s_over[i] = 0u;
  __syncthreads();
  for (int base = 0; base < a.B; base += NTHR) {
    const int b = base + threadIdx.x;
    int w = 0;
    if (b < a.B) {
      int c = __ldg(a.context_lens + b);
      if (c < 1) {
        if (blockIdx.x == 0 && a.mode != kModePartial) flag_error(a.status, PA_ERR_EMPTY_CONTEXT);
        if (blockIdx.x == 0 && c < 0) flag_error(a.status, PA_ERR_CONTEXT_RANGE);
        s_empty = 1;
        c = 0;
      }
      if (c > cap) {
        if (blockIdx.x == 0) flag_error(a.status, PA_ERR_CONTEXT_RANGE);
        atomicOr(&s_over[b >> 5], 1u << (b & 31));
        c = cap;
      }
      s_ctx[b] = c;
      w = ((c + kSubTokens - 1) / kSubTokens) * SEGS;
    }
    int v = w;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int t = __shfl_up_sync(0xffffffffu, v, o);
      if (lane >= o) v += t;
    }
    if (lane == 31) s_tmp[warp] = v;
    __syncthreads();
    if (warp == 0) {
      int t = (lane < WARPS) ? s_tmp[lane] : 0;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int u = __shfl_up_sync(0xffffffffu, t, o);
        if (lane >= o) t += u;
      }
      if (lane < WARPS) s_tmp[lane] = t;
    }
    __syncthreads();
    if (b < a.B) s_pre[b] = carry + (warp ? s_tmp[warp - 1] : 0) + v - w;
    carry += s_tmp[WARPS - 1];
    __syncthreads();
  }
  if (threadIdx.x == 0) s_pre[a.B] = carry;
  __syncthreads();
  const int T = carry;

  // Sequences with no tokens: zero output (stream) or an empty partial (partial mode).
  if (blockIdx.x == 0 && s_empty) {
    if (a.mode == kModeStream) {
      const int per_b = a.H * D / 8;
      for (int i = threadIdx.x; i < a.B * per_b; i += NTHR) {
        const int b = i / per_b;
        if (s_ctx[b] == 0)
          reinterpret_cast<uint4*>(a.out + (size_t)b * a.H * D)[i - b * per_b] =
              make_uint4(0u, 0u, 0u, 0u);
      }
    } else if (a.mode == kModePartial) {
      for (int i = threadIdx.x; i < a.B * SEGS * SLOT; i += NTHR) {
        const int segid = i / SLOT;
        const int b = segid / SEGS;
        if (s_ctx[b] == 0) {
          const int k = i - segid * SLOT;
          a.part_out[i] = (k >= D * GT && k < D * GT + GT) ? neg_inf() : 0.f;
        }
      }
    }
  }
  if (T == 0) return;

  auto pages_of = [&](int b) { return (s_ctx[b] + kSubTokens - 1) / kSubTokens; };
  // Flattened page index -> (sequence, segment inside the sequence, subpage).
  auto locate = [&](int p, int& b, int& seg, int& sp) {
    int lo = 0, hi = a.B - 1;
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (s_pre[mid] <= p) lo = mid; else hi = mid - 1;
    }
    b = lo;
    const int rel = p - s_pre[b];
    const int pg = pages_of(b);
    seg = rel / pg;
    sp = rel - seg * pg;
  };
  // Smallest split start >= p (split mode).
  auto snap = [&](long long p) -> long long {
    if (p >= T) return T;
    int b, seg, sp;
    locate((int)p, b, seg, sp);
    const int pg = pages_of(b);
    const int sp2 = (sp + kSplitPages - 1) / kSplitPages * kSplitPages;
    if (sp2 >= pg) return (long long)s_pre[b] + (long long)(seg + 1) * pg;
    return (long long)s_pre[b] + (long long)seg * pg + sp2;
  };

  // ---- 2. This warp's page range ------------------------------------------------------------
  const long long Wt = min((long long)a.total_warps, (long long)T);
  const int wg = blockIdx.x * WARPS + warp;
  long long p0 = 0, p1 = 0;
  if (wg < Wt) {
    p0 = (long long)wg * T / Wt;
    p1 = (long long)(wg + 1) * T / Wt;
    if (a.mode == kModeSplit) {
      p0 = snap(p0);
      p1 = snap(p1);
    }
  }
  const int n = (int)(p1 - p0);
  int nrec = 0;              // shared segments whose arrival this warp recorded
  int old0 = 0, old1 = 0;    // lane 0: the arrival counters' values before those arrivals
  if (n > 0) {

  // ---- 3. Consumer position and the first piece's q rows --------------------------------------
  int cb, cseg, csp;
  locate((int)p0, cb, cseg, csp);
  int cpg = pages_of(cb);
  int cctx = s_ctx[cb];
  const float qs = a.qk_scale_log2;

  // Q fragments, loaded in the chunk order of the cache's K tile layout (qa rows g, qb rows
  // g+8 of the MMA).
  // FP16 and FP8 caches: fp16 A fragments of the m16n8k16 MMA; e4m3 K bytes convert to fp16
  // exactly, so every QK product is exact and sums in fp32.
  // INT8 cache: the integer tensor cores (m16n8k32) take the raw K bytes, against q written as
  // three int8 parts over a power-of-two scale s_q = 2^(e-6), 2^e > max|q|:
  //   t = q / s_q (exact, |t| < 64), q1 = rint(t), q2 = rint(128 (t - q1)),
  //   q3 = rint(128 (128 (t - q1) - q2))          (every product and difference exact),
  // q = s_q (q1 + q2/128 + q3/16384) to within 2^-15 s_q, which is exact for every entry within
  // a factor 2^10 of max|q| and below 1e-6 max|q| for the rest; the three integer dot
  // products are exact. qa = {q1 lo, q1 hi, q2 lo, q2 hi}, qc / qd = {q3 lo, q3 hi}.
  uint4 qa[NS], qb[NS];
  uint2 qc[NS], qd[NS];
  uint4 ra[NS], rb[NS];  // q rows fetched ahead of the piece that uses them
  float qsc0 = 0.f, qsc1 = 0.f;
  // Per-token logit factors besides the K scale: scale * log2 e, times s_q for INT8.
  float qks0 = qs, qks1 = qs;
  int q_b = -1, q_seg = -1;

  auto fetch_q = [&](int b, int seg) {
    const int kvh = seg / a.HT;
    const int ht = seg - kvh * a.HT;
    const int hl = ht * GT + g;
    const __half* qrow = a.q + ((size_t)b * a.H + (size_t)kvh * a.G + hl) * D;
#pragma unroll
    for (int si = 0; si < NS; ++si) {
      const int c = BYTE ? chunk_i8(r, si) : chunk_f16(r, si);
      ra[si] = (hl < a.G) ? __ldg(reinterpret_cast<const uint4*>(qrow + 8 * c))
                          : make_uint4(0u, 0u, 0u, 0u);
      if constexpr (GT == 16) {
        rb[si] = (hl + 8 < a.G) ? __ldg(reinterpret_cast<const uint4*>(qrow + 8 * D + 8 * c))
                                : make_uint4(0u, 0u, 0u, 0u);
      } else {
        rb[si] = make_uint4(0u, 0u, 0u, 0u);
      }
    }
  };
  auto split_row = [&](const uint4 (&src)[NS], uint4 (&dst)[NS], uint2 (&dst3)[NS],
                       float& qsc) {
    float amax = 0.f;
#pragma unroll
    for (int si = 0; si < NS; ++si) {
      const uint32_t w4[4] = {src[si].x, src[si].y, src[si].z, src[si].w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w4[e]));
        amax = fmaxf(amax, fmaxf(fabsf(f.x), fabsf(f.y)));
      }
    }
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
    // 2^e > amax (e from amax's exponent field); s_q = 2^(e-6), inv = 2^(6-e). A zero row
    // keeps s_q = 1 and all-zero parts.
    const int e2 = amax > 0.f ? ((__float_as_int(amax) >> 23) & 0xff) - 126 : 6;
    qsc = __int_as_float((127 + e2 - 6) << 23);
    const float inv = __int_as_float((127 + 6 - e2) << 23);
    // Rounding to the nearest integer (ties to even) by adding and subtracting 1.5 * 2^23:
    // exact for |x| < 2^22 (here |x| <= 64), two full-rate adds instead of the conversion
    // pipe, which all warps of an SM need at once when a launch starts. The sum's low byte is
    // the int8 two's-complement byte of the rounded value.
    constexpr float kRound = 12582912.f;
#pragma unroll
    for (int si = 0; si < NS; ++si) {
      const uint32_t w4[4] = {src[si].x, src[si].y, src[si].z, src[si].w};
      int q1[8], q2[8], q3[8];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w4[e]));
        const float tt[2] = {f.x * inv, f.y * inv};
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const float t = tt[h];
          const float s1 = __fadd_rn(t, kRound);
          const float r1 = (t - __fsub_rn(s1, kRound)) * 128.f;
          const float s2 = __fadd_rn(r1, kRound);
          const float s3 = __fadd_rn((r1 - __fsub_rn(s2, kRound)) * 128.f, kRound);
          q1[2 * e + h] = __float_as_int(s1);
          q2[2 * e + h] = __float_as_int(s2);
          q3[2 * e + h] = __float_as_int(s3);
        }
      }
      dst[si] = make_uint4(pack_s8x4(q1[0], q1[1], q1[2], q1[3]),
                           pack_s8x4(q1[4], q1[5], q1[6], q1[7]),
                           pack_s8x4(q2[0], q2[1], q2[2], q2[3]),
                           pack_s8x4(q2[4], q2[5], q2[6], q2[7]));
      dst3[si] = make_uint2(pack_s8x4(q3[0], q3[1], q3[2], q3[3]),
                            pack_s8x4(q3[4], q3[5], q3[6], q3[7]));
    }
  };

  auto convert_q = [&]() {
    if constexpr (I8) {
      split_row(ra, qa, qc, qsc0);
      qks0 = qs * qsc0;  // s_q is a power of two: exact
      if constexpr (GT == 16) {
        split_row(rb, qb, qd, qsc1);
        qks1 = qs * qsc1;
      } else {
#pragma unroll
        for (int si = 0; si < NS; ++si) {
          qb[si] = make_uint4(0u, 0u, 0u, 0u);
          qd[si] = make_uint2(0u, 0u);
        }
      }
    } else {
#pragma unroll
      for (int si = 0; si < NS; ++si) {
        qa[si] = ra[si];
        qb[si] = rb[si];
      }
    }
  };
  // The first piece's q rows are requested before the page copies, so their latency overlaps
  // the block-table reads and the first copies rather than queueing behind them.
  fetch_q(cb, cseg);
  q_b = cb;
  q_seg = cseg;

  // ---- 4. Producer: the copies of 32 upcoming pages, one per lane, as (row << 3) | subpage,
  // where row = block * kv_heads + kv_head indexes [num_blocks * kv_heads] page rows.
  // With a decode step, wr receives the sequence whose new token lies in the page (the last
  // page of a segment whose context and block id are valid), else -1.
  const bool step_write = a.new_k != nullptr;
  const uint64_t pol = l2_policy_evict_first();
  // Page jbase + lane of the range: the address of its block id, its (kv_head << 3) | subpage
  // and, for a decode step, the sequence whose new token it holds (else -1).
  auto page_ref = [&](int jbase, int& meta, int& wr) -> const int* {
    meta = 0;
    wr = -1;
    const int jj = jbase + lane;
    if (jj >= n) return nullptr;
    int b, seg, sp;
    locate((int)(p0 + jj), b, seg, sp);
    const int bi = sp / a.subs;
    meta = ((seg / a.HT) << 3) | (sp - bi * a.subs);
    if (step_write && sp == pages_of(b) - 1 && !((s_over[b >> 5] >> (b & 31)) & 1u)) wr = b;
    return a.block_table + (size_t)b * a.max_blocks + bi;
  };
  // Copy descriptor (row << 3) | subpage; a block id outside the cache is flagged and read as
  // block 0, and its new token (if any) is not written.
  auto pack_page = [&](int blk, int meta, int& wr) -> int {
    if (blk < 0 || blk >= a.NB) {
      flag_error(a.status, PA_ERR_BLOCK_ID);
      blk = 0;
      wr = -1;
    }
    return ((blk * a.KVH + (meta >> 3)) << 3) | (meta & 7);
  };
  // The block ids of the next 32 pages are copied into shared memory in the background
  // (cp.async) a batch ahead, so no block-table load ever stalls the page loop.
  auto prefetch_batch = [&](int jbase) {
    int meta, wr;
    const int* p = page_ref(jbase, meta, wr);
    s_nmeta[warp][lane] = meta;
    s_nwr[warp][lane] = wr;
    if (p != nullptr) {
      cp_async_4(&s_nblk[warp][lane], p);
    } else {
      s_nblk[warp][lane] = 0;
    }
    cp_async_commit();
  };
  auto take_batch = [&](int& wr) -> int {
    cp_async_wait_all();
    wr = s_nwr[warp][lane];
    return pack_page(s_nblk[warp][lane], s_nmeta[warp][lane], wr);
  };
  int curw, meta0;
  const int* bref0 = page_ref(0, meta0, curw);
  const int blk0 = bref0 != nullptr ? __ldg(bref0) : 0;
  prefetch_batch(32);  // requested before the first batch's ids are waited for
  int cur = pack_page(blk0, meta0, curw);

  auto issue = [&](int j, int s) {
    if (j > 0 && (j & 31) == 0) {
      cur = take_batch(curw);
      prefetch_batch(j + 32);
    }
    const int pk = __shfl_sync(0xffffffffu, cur, j & 31);
    // Decode step: the page holding sequence wb's new token also brings the token's K and V
    // rows (bulk copies on the same barrier); the consumer quantises them into the stage.
    const int wb = step_write ? __shfl_sync(0xffffffffu, curw, j & 31) : -1;
    if (lane == 0) {
      const int row = pk >> 3;
      const int sub = pk & 7;
      uint64_t* bar = &wbar[s];
      uint8_t* kd = k_tiles + (warp * DEPTH + s) * C::KT;
      uint8_t* vd = v_tiles + (warp * DEPTH + s) * C::VT;
      // Recorded before the arrival, whose release the consumer's wait acquires.
      if (step_write) s_wrow[warp][s] = wb >= 0 ? row : -1;
      mbar_arrive_expect_tx(bar, C::TX + (wb >= 0 ? (uint32_t)C::NR : 0u));
      if (step_write) {
        if (wb >= 0) {
          const size_t so = ((size_t)wb * a.new_stride + (size_t)(row % a.KVH) * D) * 2;
          uint8_t* rd = r_tiles + (warp * DEPTH + s) * C::NR;
          bulk_g2s(rd, static_cast<const uint8_t*>(a.new_k) + so, D * 2, bar);
          bulk_g2s(rd + D * 2, static_cast<const uint8_t*>(a.new_v) + so, D * 2, bar);
        }
      }
      // The cache pages stream through L2 marked evict-first.
      if constexpr (BYTE) {
        tma_load_3d_hint(kd, &tm_k, bar, sub * 128, 0, row, pol);
      } else {
        tma_load_4d_hint(kd, &tm_k, bar, 0, sub * 2, 0, row, pol);
      }
      if (a.bulk) {
        bulk_g2s_hint(vd, a.v_base + (size_t)row * C::VT, C::VT, bar, pol);
        if constexpr (BYTE) {
          uint8_t* sd = s_tiles + (warp * DEPTH + s) * C::ST;
          bulk_g2s_hint(sd, a.ks_base + (size_t)row * kSubTokens, 64, bar, pol);
          bulk_g2s_hint(sd + kVsOff, a.vs_base + (size_t)row * kSubTokens, 64, bar, pol);
        }
      } else {
        tma_load_3d_hint(vd, &tm_v, bar, sub * kSubTokens, 0, row, pol);
        if constexpr (BYTE) {
          uint8_t* sd = s_tiles + (warp * DEPTH + s) * C::ST;
          tma_load_2d_hint(sd, &tm_ks, bar, sub * kSubTokens, row, pol);
          tma_load_2d_hint(sd + kVsOff, &tm_vs, bar, sub * kSubTokens, row, pol);
        }
      }
    }
  };

  static_assert(DEPTH < 32, "the prologue copies must come from the first batch of block ids");
  const int npro = n < DEPTH ? n : DEPTH;
  __syncwarp();
  for (int j = 0; j < npro; ++j) issue(j, j);
  int issued = npro;
  convert_q();

  // Shared-memory offsets of the K cells this lane reads (chunk of load si, token of n-tile
  // jt), fixed for the whole kernel.
  uint32_t koff[NS][2];
#pragma unroll
  for (int si = 0; si < NS; ++si) {
#pragma unroll
    for (int jt = 0; jt < 2; ++jt) {
      const int tau = 4 * (g >> 1) + (g & 1) + 2 * jt;
      if constexpr (BYTE) {
        const int c = chunk_i8(r, si);
        koff[si][jt] = c * 128 + ((((tau >> 1) ^ (c & 7)) << 4) | ((tau & 1) << 3));
      } else {
        const int c = chunk_f16(r, si);
        const int row = 2 * c + (tau >> 3);
        koff[si][jt] = row * 128 + (((tau & 7) ^ (row & 7)) << 4);
      }
    }
  }
  const uint32_t voff = BYTE ? (uint32_t)(g * 16 + 4 * r) : (uint32_t)((g * 16 + 4 * r) * 2);
  const uint32_t kbase = smem_u32(k_tiles) + warp * DEPTH * C::KT;
  const uint32_t vbase = smem_u32(v_tiles) + warp * DEPTH * C::VT;
  const uint32_t sbase = BYTE ? smem_u32(s_tiles) + warp * DEPTH * C::ST : 0u;

  // Decode step: the new token held in stage st goes into the staged page and the cache.
  auto merge_new_token = [&](int st, int row, int t, int off) {
    stage_new_token<KVK, D>(r_tiles + (warp * DEPTH + st) * C::NR,
                            k_tiles + (warp * DEPTH + st) * C::KT,
                            v_tiles + (warp * DEPTH + st) * C::VT,
                            BYTE ? s_tiles + (warp * DEPTH + st) * C::ST : nullptr, lane, row, t,
                            off, a.new_dtype, a.new_kfix, a.new_vfix, a.kc_w, a.vc_w, a.ks_w,
                            a.vs_w, a.bs);
  };

  float m0 = neg_inf(), l0 = 0.f, m1 = neg_inf(), l1 = 0.f;
  float oacc[MT][NT][4];

  int jfail = -1;
  int s = 0;        // ring stage of page j
  uint32_t ph = 0;  // its mbarrier phase parity
  const bool split = (a.mode == kModeSplit);
  int j = 0;
  while (j < n) {
    // ---- one piece: the pages of this warp's range inside one segment (one split in split
    // mode), subpages [csp, csp + len) of sequence cb, segment cseg.
    const int piece_sp0 = csp;
    int len = cpg - csp;
    if (split) len = min(len, kSplitPages - csp % kSplitPages);
    len = min(len, n - j);
    if (q_b != cb || q_seg != cseg) {
      fetch_q(cb, cseg);
      convert_q();
      q_b = cb;
      q_seg = cseg;
    }
    // When this piece ends its segment and the range goes on, the next segment's q rows are
    // brought into L1 while this piece runs, so the next piece's q fetch does not wait on L2.
    if (csp + len == cpg && j + len < n) {
      int nb = cb, ns = cseg + 1;
      if (ns == SEGS) {
        ns = 0;
        do { ++nb; } while (pages_of(nb) == 0);
      }
      const int kvh = ns / a.HT;
      const int hl = (ns - kvh * a.HT) * GT + (lane >> 1);
      if (lane < 2 * GT && hl < a.G)
        prefetch_l1(a.q + ((size_t)nb * a.H + (size_t)kvh * a.G + hl) * D + (lane & 1) * (D / 2));
    }
    m0 = neg_inf();
    l0 = 0.f;
    m1 = neg_inf();
    l1 = 0.f;
#pragma unroll
    for (int i = 0; i < MT; ++i)
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) oacc[i][nt][e] = 0.f;

    for (int k = 0; k < len; ++k) {
    if (!mbar_wait_bounded(&wbar[s], ph, a.status)) {
      jfail = j;
      break;
    }

    // ---- stage -> registers, then hand the stage back to the TMA right away -------------------
    const int valid = min(kSubTokens, cctx - (csp + k) * kSubTokens);
    // Decode step: only a segment's last page can hold a sequence's new token, so no other
    // page reads the stage's record.
    if (step_write && csp + k == cpg - 1) {
      const int wrow = s_wrow[warp][s];
      if (wrow >= 0) merge_new_token(s, wrow, valid - 1, (cctx - 1) % a.bs);
    }
    const uint32_t kb = kbase + s * C::KT;
    const uint32_t vb = vbase + s * C::VT;
    const uint32_t sb = sbase + s * C::ST;
    uint2 k8[NS][2];
    uint4 k16[NS][2];
    uint32_t v8[MT][2];
    uint2 v16[MT][2];
    float4 ksv = make_float4(0.f, 0.f, 0.f, 0.f), vsv = ksv;
#pragma unroll
    for (int si = 0; si < NS; ++si) {
#pragma unroll
      for (int jt = 0; jt < 2; ++jt) {
        if constexpr (BYTE) k8[si][jt] = lds64(kb + koff[si][jt]);
        else k16[si][jt] = lds128(kb + koff[si][jt]);
      }
    }
#pragma unroll
    for (int i = 0; i < MT; ++i) {
      if constexpr (BYTE) {
        v8[i][0] = lds32(vb + voff + i * 256);
        v8[i][1] = lds32(vb + voff + i * 256 + 128);
      } else {
        v16[i][0] = lds64(vb + voff + i * 512);
        v16[i][1] = lds64(vb + voff + i * 512 + 256);
      }
    }
    if constexpr (BYTE) {
      ksv = lds128f(sb + 16 * r);
      vsv = lds128f(sb + kVsOff + 16 * r);
    }
    __syncwarp();
    if (j + DEPTH < n) {
      if (lane == 0) fence_proxy_async_smem();
      issue(j + DEPTH, s);
      ++issued;
    }

    // ---- one 16-token subpage from registers ---------------------------------------------------
    {
      // S = Q K^T : rows = heads (g, g+8), columns = tokens tok(jt, n); tokens 4r..4r+3 of
      // head g end up in x[0..3] (and of head g+8 in y[0..3]).
      float x[4], y[4];
      if constexpr (I8) {
        // Three exact integer dot products per (head, token) on the raw K bytes, combined as
        // p1 + (128 p2 + p3) / 16384 (|q2|, |q3| <= 64, so |128 p2 + p3| < 2^28 is exact in
        // int32; s_q multiplies in with the K scale below).
        constexpr float k3 = 1.f / 16384.f;
        if constexpr (NT == 1) {
          // Eight heads leave the MMA's rows 8-15 free: they take q's second part, so one MMA
          // gives p1 (rows g) and p2 (rows g+8) and a second one p3.
          int s12[2][4], s3[2][4];
#pragma unroll
          for (int jt = 0; jt < 2; ++jt)
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              s12[jt][e] = 0;
              s3[jt][e] = 0;
            }
#pragma unroll
          for (int si = 0; si < NS; ++si) {
#pragma unroll
            for (int jt = 0; jt < 2; ++jt) {
              imma_16832(s12[jt], qa[si].x, qa[si].z, qa[si].y, qa[si].w, k8[si][jt].x,
                         k8[si][jt].y);
              imma_16832(s3[jt], qc[si].x, 0u, qc[si].y, 0u, k8[si][jt].x, k8[si][jt].y);
            }
          }
#pragma unroll
          for (int jt = 0; jt < 2; ++jt)
#pragma unroll
            for (int e = 0; e < 2; ++e)
              x[2 * jt + e] = fmaf((float)(s12[jt][2 + e] * 128 + s3[jt][e]), k3,
                                   (float)s12[jt][e]);
          y[0] = y[1] = y[2] = y[3] = 0.f;
        } else {
          int sa[2][4], sb2[2][4], sc3[2][4];
#pragma unroll
          for (int jt = 0; jt < 2; ++jt)
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              sa[jt][e] = 0;
              sb2[jt][e] = 0;
              sc3[jt][e] = 0;
            }
#pragma unroll
          for (int si = 0; si < NS; ++si) {
#pragma unroll
            for (int jt = 0; jt < 2; ++jt) {
              imma_16832(sa[jt], qa[si].x, qb[si].x, qa[si].y, qb[si].y, k8[si][jt].x,
                         k8[si][jt].y);
              imma_16832(sb2[jt], qa[si].z, qb[si].z, qa[si].w, qb[si].w, k8[si][jt].x,
                         k8[si][jt].y);
              imma_16832(sc3[jt], qc[si].x, qd[si].x, qc[si].y, qd[si].y, k8[si][jt].x,
                         k8[si][jt].y);
            }
          }
          auto comb = [&](int jt, int e) {
            return fmaf((float)(sb2[jt][e] * 128 + sc3[jt][e]), k3, (float)sa[jt][e]);
          };
          x[0] = comb(0, 0);
          x[1] = comb(0, 1);
          x[2] = comb(1, 0);
          x[3] = comb(1, 1);
          y[0] = comb(0, 2);
          y[1] = comb(0, 3);
          y[2] = comb(1, 2);
          y[3] = comb(1, 3);
        }
      } else {
        if constexpr (F8) {
          // e4m3 K bytes -> exact fp16.
#pragma unroll
          for (int si = 0; si < NS; ++si)
#pragma unroll
            for (int jt = 0; jt < 2; ++jt) {
              e4m3x4_to_f16x2x2(k8[si][jt].x, k16[si][jt].x, k16[si][jt].y);
              e4m3x4_to_f16x2x2(k8[si][jt].y, k16[si][jt].z, k16[si][jt].w);
            }
        }
        // Two accumulation chains per n-tile (even / odd si) shorten the MMA dependency.
        float sacc[2][2][4];
#pragma unroll
        for (int jt = 0; jt < 2; ++jt)
#pragma unroll
          for (int hh = 0; hh < 2; ++hh)
#pragma unroll
            for (int e = 0; e < 4; ++e) sacc[jt][hh][e] = 0.f;
#pragma unroll
        for (int si = 0; si < NS; ++si) {
#pragma unroll
          for (int jt = 0; jt < 2; ++jt) {
            float (&acc)[4] = sacc[jt][si & 1];
            mma_16816(acc, qa[si].x, qb[si].x, qa[si].y, qb[si].y, k16[si][jt].x,
                      k16[si][jt].y);
            mma_16816(acc, qa[si].z, qb[si].z, qa[si].w, qb[si].w, k16[si][jt].z,
                      k16[si][jt].w);
          }
        }
        x[0] = sacc[0][0][0] + sacc[0][1][0];
        x[1] = sacc[0][0][1] + sacc[0][1][1];
        x[2] = sacc[1][0][0] + sacc[1][1][0];
        x[3] = sacc[1][0][1] + sacc[1][1][1];
        y[0] = sacc[0][0][2] + sacc[0][1][2];
        y[1] = sacc[0][0][3] + sacc[0][1][3];
        y[2] = sacc[1][0][2] + sacc[1][1][2];
        y[3] = sacc[1][0][3] + sacc[1][1][3];
      }
      // Logits in log2 units: per token, the K scale times scale * log2 e (and, INT8, times
      // the q part scale s_q of the row's head, qks0 / qks1).
      {
        const float kx[4] = {ksv.x, ksv.y, ksv.z, ksv.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          if constexpr (BYTE) {
            x[e] *= kx[e] * qks0;
            if constexpr (NT == 2) y[e] *= kx[e] * qks1;
          } else {
            x[e] *= qs;
            if constexpr (NT == 2) y[e] *= qs;
          }
        }
      }
      if (valid < kSubTokens) {
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          if (4 * r + e >= valid) {
            x[e] = neg_inf();
            y[e] = neg_inf();
          }
        }
      }
      float tm0 = fmaxf(fmaxf(x[0], x[1]), fmaxf(x[2], x[3]));
      tm0 = fmaxf(tm0, __shfl_xor_sync(0xffffffffu, tm0, 1));
      tm0 = fmaxf(tm0, __shfl_xor_sync(0xffffffffu, tm0, 2));
      const float mn0 = fmaxf(m0, tm0);
      float mn1 = m1;
      if constexpr (NT == 2) {
        float tm1 = fmaxf(fmaxf(y[0], y[1]), fmaxf(y[2], y[3]));
        tm1 = fmaxf(tm1, __shfl_xor_sync(0xffffffffu, tm1, 1));
        tm1 = fmaxf(tm1, __shfl_xor_sync(0xffffffffu, tm1, 2));
        mn1 = fmaxf(m1, tm1);
      }
      if (__any_sync(0xffffffffu, (mn0 > m0) || (mn1 > m1))) {
        const float c0 = ex2(m0 - mn0);
        l0 *= c0;
        m0 = mn0;
        const float ca = __shfl_sync(0xffffffffu, c0, 8 * r);
        const float cb2 = __shfl_sync(0xffffffffu, c0, 8 * r + 4);
#pragma unroll
        for (int i = 0; i < MT; ++i) {
          oacc[i][0][0] *= ca;
          oacc[i][0][1] *= cb2;
          oacc[i][0][2] *= ca;
          oacc[i][0][3] *= cb2;
        }
        if constexpr (NT == 2) {
          const float c1 = ex2(m1 - mn1);
          l1 *= c1;
          m1 = mn1;
          const float cc = __shfl_sync(0xffffffffu, c1, 8 * r);
          const float cd = __shfl_sync(0xffffffffu, c1, 8 * r + 4);
#pragma unroll
          for (int i = 0; i < MT; ++i) {
            oacc[i][1][0] *= cc;
            oacc[i][1][1] *= cd;
            oacc[i][1][2] *= cc;
            oacc[i][1][3] *= cd;
          }
        }
      }
      // Weights are formed 2^kPExp times larger than p (the exponent is shifted), so that the
      // fp16 hi/lo split of P' below stays clear of the fp16 subnormal range while P' (at most
      // 2^kPExp times a V scale) stays below the fp16 maximum. O and l carry the same factor:
      // it cancels in O / l and is taken out when a partial slot is written.
      const float mb0 = m0 - kPExp;
      const float mb1 = m1 - kPExp;
      float p[4], pv[4], py[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        p[e] = ex2(x[e] - mb0);
        l0 += p[e];
        pv[e] = p[e];
        if constexpr (NT == 2) {
          py[e] = ex2(y[e] - mb1);
          l1 += py[e];
        } else {
          py[e] = 0.f;
        }
      }
      if constexpr (BYTE) {
        const float vsc[4] = {vsv.x, vsv.y, vsv.z, vsv.w};
        if (valid < kSubTokens) {
          // Scales of slots past the context may hold anything: keep them out of P'.
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const bool ok = (4 * r + e) < valid;
            pv[e] = ok ? p[e] * vsc[e] : 0.f;
            if constexpr (NT == 2) py[e] = ok ? py[e] * vsc[e] : 0.f;
          }
        } else {
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            pv[e] = p[e] * vsc[e];
            if constexpr (NT == 2) py[e] *= vsc[e];
          }
        }
      }
      // P' as two fp16 parts, hi + lo (about 22 significant bits), each multiplied by V: one
      // fp16 rounding of the weights alone can exceed the output tolerance when attention is
      // concentrated on a few tokens with large V entries.
      uint32_t pb0, pb1, pl0, pl1, pc0 = 0u, pc1 = 0u, pm0 = 0u, pm1 = 0u;
      split_f16x2(pv[0], pv[1], pb0, pl0);
      split_f16x2(pv[2], pv[3], pb1, pl1);
      if constexpr (NT == 2) {
        split_f16x2(py[0], py[1], pc0, pm0);
        split_f16x2(py[2], py[3], pc1, pm1);
      }

      // O^T += V^T P^T : rows = head_dim (16 per m-tile), columns = heads.
      uint32_t mlo = 0xffffffffu, mhi = 0xffffffffu;
      if (!I8 && valid < kSubTokens) {
        mlo = ((4 * r < valid) ? 0x0000ffffu : 0u) | ((4 * r + 1 < valid) ? 0xffff0000u : 0u);
        mhi = ((4 * r + 2 < valid) ? 0x0000ffffu : 0u) | ((4 * r + 3 < valid) ? 0xffff0000u : 0u);
      }
#pragma unroll
      for (int i = 0; i < MT; ++i) {
        uint32_t a0, a1, a2, a3;
        if constexpr (I8) {
          i8x4_to_f16x2x2(v8[i][0], a0, a2);
          i8x4_to_f16x2x2(v8[i][1], a1, a3);
        } else if constexpr (F8) {
          // e4m3 bytes past the context may be NaN encodings: masked like fp16 V.
          e4m3x4_to_f16x2x2(v8[i][0], a0, a2);
          e4m3x4_to_f16x2x2(v8[i][1], a1, a3);
          a0 &= mlo;
          a2 &= mhi;
          a1 &= mlo;
          a3 &= mhi;
        } else {
          a0 = v16[i][0].x & mlo;
          a2 = v16[i][0].y & mhi;
          a1 = v16[i][1].x & mlo;
          a3 = v16[i][1].y & mhi;
        }
        mma_16816(oacc[i][0], a0, a1, a2, a3, pb0, pb1);
        mma_16816(oacc[i][0], a0, a1, a2, a3, pl0, pl1);
        if constexpr (NT == 2) {
          mma_16816(oacc[i][1], a0, a1, a2, a3, pc0, pc1);
          mma_16816(oacc[i][1], a0, a1, a2, a3, pm0, pm1);
        }
      }
    }

    ++j;
    if (++s == DEPTH) {
      s = 0;
      ph ^= 1u;
    }
    }  // pages of the piece
    if (jfail >= 0) break;
    csp += len;

    {
      // ---- piece epilogue ---------------------------------------------------------------------
      float lt0 = l0 + __shfl_xor_sync(0xffffffffu, l0, 1);
      lt0 += __shfl_xor_sync(0xffffffffu, lt0, 2);
      float lt1 = 0.f;
      if constexpr (NT == 2) {
        lt1 = l1 + __shfl_xor_sync(0xffffffffu, l1, 1);
        lt1 += __shfl_xor_sync(0xffffffffu, lt1, 2);
      }
      const int segid = cb * SEGS + cseg;
      const int kvh = cseg / a.HT;
      const int ht = cseg - kvh * a.HT;
      const int hbase = kvh * a.G + ht * GT;
      const int hcnt = min(GT, a.G - ht * GT);

      // Partial slots hold O and l without the 2^kPExp weight factor (an exact rescale).
      auto write_slot = [&](float* slot) {
        constexpr float kUnscale = 1.f / (float)(1 << (int)kPExp);
#pragma unroll
        for (int i = 0; i < MT; ++i) {
#pragma unroll
          for (int nt = 0; nt < NT; ++nt) {
            *reinterpret_cast<float2*>(slot + (16 * i + g) * GT + nt * 8 + 2 * r) =
                make_float2(oacc[i][nt][0] * kUnscale, oacc[i][nt][1] * kUnscale);
            *reinterpret_cast<float2*>(slot + (16 * i + g + 8) * GT + nt * 8 + 2 * r) =
                make_float2(oacc[i][nt][2] * kUnscale, oacc[i][nt][3] * kUnscale);
          }
        }
        if (r == 0) {
          slot[D * GT + g] = m0;
          slot[D * GT + GT + g] = lt0 * kUnscale;
          if constexpr (NT == 2) {
            slot[D * GT + 8 + g] = m1;
            slot[D * GT + GT + 8 + g] = lt1 * kUnscale;
          }
        }
      };

      if (split) {
        write_slot(a.part + ((size_t)segid * a.s_max + piece_sp0 / kSplitPages) * SLOT);
      } else if (piece_sp0 == 0 && csp == cpg) {
        // The whole segment was this warp's: normalise and store directly.
        if (a.mode == kModeStream) {
          const float inv0 = 1.f / lt0;
          const float ia = __shfl_sync(0xffffffffu, inv0, 8 * r);
          const float ib = __shfl_sync(0xffffffffu, inv0, 8 * r + 4);
          float ic = 0.f, id = 0.f;
          if constexpr (NT == 2) {
            const float inv1 = 1.f / lt1;
            ic = __shfl_sync(0xffffffffu, inv1, 8 * r);
            id = __shfl_sync(0xffffffffu, inv1, 8 * r + 4);
          }
          __half* ob = a.out + ((size_t)cb * a.H + hbase) * D;
#pragma unroll
          for (int i = 0; i < MT; ++i) {
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) {
              const int h = nt * 8 + 2 * r;
              const float fa = nt ? ic : ia;
              const float fb = nt ? id : ib;
              if (h < hcnt) {
                ob[(size_t)h * D + 16 * i + g] = __float2half_rn(oacc[i][nt][0] * fa);
                ob[(size_t)h * D + 16 * i + g + 8] = __float2half_rn(oacc[i][nt][2] * fa);
              }
              if (h + 1 < hcnt) {
                ob[(size_t)(h + 1) * D + 16 * i + g] = __float2half_rn(oacc[i][nt][1] * fb);
                ob[(size_t)(h + 1) * D + 16 * i + g + 8] = __float2half_rn(oacc[i][nt][3] * fb);
              }
            }
          }
        } else {
          write_slot(a.part_out + (size_t)segid * SLOT);
        }
      } else {
        // A piece of a segment shared with neighbouring warps.
        write_slot(a.part + ((size_t)wg * 2 + (piece_sp0 == 0 ? 1 : 0)) * SLOT);
        __syncwarp();
        const long long s_start = (long long)s_pre[cb] + (long long)cseg * cpg;
        const long long s_end = s_start + cpg;
        const int wf = (int)(((s_start + 1) * Wt - 1) / T);
        const int wl = (int)((s_end * Wt - 1) / T);
        const int np = wl - wf + 1;
        // Release this piece; the arrival that completes the count acquires all of them and
        // owes the merge, which runs after the page loop, when the registers are free. The
        // merge is recorded now and kept if the atomic's old value shows the last arrival;
        // that value is first read after the loop, so the loop does not wait for the atomic.
        // A warp shares at most two segments (its first and its last).
        if (lane == 0 && nrec < 2) {
          if (nrec == 0) {
            old0 = atom_add_acq_rel_gpu(a.counters + segid, 1);
          } else {
            old1 = atom_add_acq_rel_gpu(a.counters + segid, 1);
          }
          int* pe = s_pend[warp][nrec];
          pe[0] = segid;
          pe[1] = wf;
          pe[2] = np;
          pe[3] = cb;
          pe[4] = hbase;
          pe[5] = hcnt;
        }
        ++nrec;
      }
    }

    // ---- next segment
    if (csp == cpg) {
      csp = 0;
      if (++cseg == SEGS) {
        cseg = 0;
        if (j < n) {
          do { ++cb; } while (pages_of(cb) == 0);
          cctx = s_ctx[cb];
        }
      }
      if (j < n) cpg = pages_of(cb);
    }
  }

  if (jfail >= 0) {
    // Let copies still in flight land before the CTA's shared memory is released.
    for (int jj = jfail; jj < issued; ++jj) {
      (void)mbar_wait_bounded(&wbar[jj % DEPTH], (uint32_t)(jj / DEPTH) & 1u, nullptr);
    }
  }
  }  // n > 0

  // ---- 5. Merges of the segments whose last piece this CTA's warps finished ------------------
  // The pieces of a recorded merge are visible: the recording arrival acquired them, and the
  // barrier below orders that arrival before every warp's reads.
  // Each merge of up to kStageCap pieces is one warp's: it bulk-copies the pieces into the
  // (now idle) ring memory and merges them from there, side by side with the CTA's other
  // merges; merges are packed into the ring memory in a fixed order, in waves when they do not
  // all fit at once. Only a merge of more pieces than the ring memory holds runs on the whole
  // CTA, reading the pieces from L2.
  if (lane == 0) {
    // The recorded merges this warp owes: those whose arrival completed the count.
    int k = 0;
    for (int e = 0; e < min(nrec, 2); ++e) {
      const int* pe = s_pend[warp][e];
      if ((e == 0 ? old0 : old1) == pe[2] - 1) {
        if (k != e)
          for (int f = 0; f < 6; ++f) s_pend[warp][k][f] = pe[f];
        ++k;
      }
    }
    s_npend[warp] = k;
  }
  __syncthreads();  // every warp is past its page loop: the ring memory is free
  constexpr size_t kRing = (size_t)WARPS * DEPTH * (C::KT + C::VT + C::ST);
  constexpr int kStageCap = (int)(kRing / (SLOT * sizeof(float)));
  float* scratch = reinterpret_cast<float*>(k_tiles);
  const bool stream = (a.mode == kModeStream);
  int used = 0, inwave = 0;
  uint32_t mph = 0;  // phase parity of this warp's merge barrier
  bool any_big = false;
  for (int w = 0; w < WARPS; ++w) {
    for (int e = 0; e < s_npend[w]; ++e) {
      const int* pe = s_pend[w][e];
      const int np = pe[2];
      if (np > kStageCap) {
        any_big = true;
        continue;
      }
      if (used + np > kStageCap || inwave == WARPS) {
        __syncthreads();  // the wave's merges are done with the ring memory
        used = 0;
        inwave = 0;
      }
      if (inwave == warp) {
        const int segid = pe[0], wf = pe[1], b = pe[3], hbase = pe[4], hcnt = pe[5];
        if (!staged_combine<D, GT>(a.part, wf, np, lane, hcnt,
                                   stream ? a.out + ((size_t)b * a.H + hbase) * D : nullptr,
                                   stream ? nullptr : a.part_out + (size_t)segid * SLOT,
                                   a.status, scratch + (size_t)used * SLOT, &s_mmb[warp], mph)) {
          // Timed out: let the copies land before the memory is used again.
          (void)mbar_wait_bounded(&s_mmb[warp], mph, nullptr);
        }
        mph ^= 1u;
        if (lane == 0) a.counters[segid] = 0;
      }
      used += np;
      ++inwave;
    }
  }
  if (!any_big) return;
  __syncthreads();  // the staged merges are done with the ring memory
  for (int w = 0; w < WARPS; ++w) {
    for (int e = 0; e < s_npend[w]; ++e) {
      const int* pe = s_pend[w][e];
      const int segid = pe[0], wf = pe[1], np = pe[2], b = pe[3], hbase = pe[4], hcnt = pe[5];
      if (np <= kStageCap) continue;
      if (Coop<D, GT, NTHR, 8>::floats(np) * sizeof(float) > kRing) {
        if (threadIdx.x == 0) {
          flag_error(a.status, PA_ERR_WORKSPACE);
          a.counters[segid] = 0;  // leave the counter ready for the next call
        }
        continue;
      }
      auto piece = [&](int k) -> const float* {
        return a.part + ((size_t)(wf + k) * 2 + (k == 0 ? 1 : 0)) * SLOT;
      };
      if (stream) {
        coop_combine<D, GT, NTHR, 8>(piece, np, hcnt, a.out + ((size_t)b * a.H + hbase) * D,
                                     nullptr, a.status, scratch);
      } else {
        coop_combine<D, GT, NTHR, 8>(piece, np, hcnt, nullptr,
                                     a.part_out + (size_t)segid * SLOT, a.status, scratch);
      }
      if (threadIdx.x == 0) a.counters[segid] = 0;
    }
  }
}

// ---------------------------------------------------------------------------------------
// LSE reduce of the split-K pair (and of partials gathered across GPUs): one CTA of
// kReduceThreads threads per (sequence, kv-head, head tile) segment, merged cooperatively.
// ---------------------------------------------------------------------------------------
constexpr int kReduceThreads = 512;

template <int D, int GT>
__global__ void __launch_bounds__(kReduceThreads, 1) reduce_kernel(const ReduceArgs a) {
  extern __shared__ __align__(16) float rsm[];
  const int SEGS = a.KVH * a.HT;
  const int segid = blockIdx.x;
  const int b = segid / SEGS;
  const int seg = segid - b * SEGS;
  const int kvh = seg / a.HT;
  const int ht = seg - kvh * a.HT;
  const int hbase = kvh * a.G + ht * GT;
  const int hcnt = min(GT, a.G - ht * GT);
  int np = a.num_parts;
  if (np <= 0) {
    int c = __ldg(a.context_lens + b);
    const int cap = a.max_blocks * a.bs;
    c = c < 0 ? 0 : (c > cap ? cap : c);
    const int pages = (c + kSubTokens - 1) / kSubTokens;
    np = (pages + kSplitPages - 1) / kSplitPages;
  }
  __half* orow = a.out + ((size_t)b * a.H + hbase) * D;
  if (np == 0) {
    for (int i = threadIdx.x; i < hcnt * D; i += blockDim.x) orow[i] = __float2half_rn(0.f);
    if (threadIdx.x == 0 && seg == 0) flag_error(a.status, PA_ERR_EMPTY_CONTEXT);
    return;
  }
  const float* base = a.part + (size_t)segid * a.seg_stride;
  coop_combine<D, GT, kReduceThreads, 16>(
      [&](int k) { return base + (size_t)k * a.piece_stride; }, np, hcnt, orow, nullptr,
      a.status, rsm);
}

// Launch shapes per (cache dtype, head tile): warps per CTA (one CTA per SM) and ring depth
// per warp. A stage is held only while its bytes are read into registers, so all DEPTH
// stages of a warp are in flight while it computes.
#ifndef PA_I8_WARPS
#define PA_I8_WARPS 12
#endif
#ifndef PA_I8_DEPTH
#define PA_I8_DEPTH 3
#endif
#ifndef PA_F16_WARPS
#define PA_F16_WARPS 8
#endif
#ifndef PA_F16_DEPTH
#define PA_F16_DEPTH 2
#endif
template <int KVK, int GT> struct Shape;
template <> struct Shape<1, 8> { static constexpr int W = PA_I8_WARPS, DP = PA_I8_DEPTH; };
template <> struct Shape<0, 8> { static constexpr int W = PA_F16_WARPS, DP = PA_F16_DEPTH; };
template <> struct Shape<1, 16> { static constexpr int W = 8, DP = 4; };
template <> struct Shape<0, 16> { static constexpr int W = 8, DP = 3; };
template <> struct Shape<2, 8> { static constexpr int W = 12, DP = 3; };
template <> struct Shape<2, 16> { static constexpr int W = 8, DP = 4; };

template <int KVK, int GT>
cudaError_t launch_one(const DecodeArgs& a, const CUtensorMap* maps, int grid,
                       cudaStream_t stream) {
  constexpr int W = Shape<KVK, GT>::W;
  constexpr int DP = Shape<KVK, GT>::DP;
  using C = Tile<KVK, 128, GT, DP, W>;
  static_assert(C::SMEM_STEP + 14 * 1024 <= 227 * 1024, "shared memory of a step launch");
  auto kern = decode_kernel<KVK, 128, GT, DP, W>;
  // The shared-memory opt-in is a per-device function attribute: set it once per device, to
  // the larger size of a decode step launch.
  static std::atomic<uint64_t> configured{0};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  const uint64_t bit = 1ull << (dev & 63);
  if (!(configured.load(std::memory_order_acquire) & bit)) {
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)C::SMEM_STEP);
    if (e != cudaSuccess) return e;
    configured.fetch_or(bit, std::memory_order_acq_rel);
  }
  const size_t smem = a.new_k != nullptr ? C::SMEM_STEP : C::SMEM;
  kern<<<grid, W * 32, smem, stream>>>(a, maps[0], maps[1], maps[2], maps[3]);
  return cudaGetLastError();
}

}  // namespace

int decode_warps_per_cta(int kv_i8, int gt) {
  if (kv_i8 == 2) return gt == 8 ? Shape<2, 8>::W : Shape<2, 16>::W;
  if (kv_i8) return gt == 8 ? Shape<1, 8>::W : Shape<1, 16>::W;
  return gt == 8 ? Shape<0, 8>::W : Shape<0, 16>::W;
}

cudaError_t launch_decode(int kv_i8, int gt, const DecodeArgs& a, const CUtensorMap* maps,
                          int grid, cudaStream_t stream) {
  if (kv_i8 == 2) {
    return gt == 8 ? launch_one<2, 8>(a, maps, grid, stream)
                   : launch_one<2, 16>(a, maps, grid, stream);
  }
  if (kv_i8) {
    return gt == 8 ? launch_one<1, 8>(a, maps, grid, stream)
                   : launch_one<1, 16>(a, maps, grid, stream);
  }
  return gt == 8 ? launch_one<0, 8>(a, maps, grid, stream)
                 : launch_one<0, 16>(a, maps, grid, stream);
}

namespace {
__global__ void selftest_wait_kernel(int* status) {
  __shared__ uint64_t bar;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    fence_mbar_init();
  }
  __syncwarp();
  // Nothing arrives on the barrier: phase 0 never completes, so the bounded wait gives up.
  (void)mbar_wait_bounded(&bar, 0u, status);
}
}  // namespace

cudaError_t launch_selftest_wait(int* status, cudaStream_t st) {
  selftest_wait_kernel<<<1, 32, 0, st>>>(status);
  return cudaGetLastError();
}

cudaError_t launch_reduce(int gt, const ReduceArgs& a, int max_pieces, cudaStream_t stream) {
  const int segs = a.B * a.KVH * a.HT;
  if (segs == 0) return cudaSuccess;
  size_t smem;
  cudaError_t e;
  if (Coop<128, 16, kReduceThreads, 16>::floats(max_pieces) * sizeof(float) > 200 * 1024)
    return cudaErrorInvalidValue;  // more splits than one CTA can merge (contexts > ~3M tokens)
  if (gt == 8) {
    smem = Coop<128, 8, kReduceThreads, 16>::floats(max_pieces) * sizeof(float);
    e = cudaFuncSetAttribute(reduce_kernel<128, 8>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)smem);
    if (e != cudaSuccess) return e;
    reduce_kernel<128, 8><<<segs, kReduceThreads, smem, stream>>>(a);
  } else {
    smem = Coop<128, 16, kReduceThreads, 16>::floats(max_pieces) * sizeof(float);
    e = cudaFuncSetAttribute(reduce_kernel<128, 16>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)smem);
    if (e != cudaSuccess) return e;
    reduce_kernel<128, 16><<<segs, kReduceThreads, smem, stream>>>(a);
  }
  return cudaGetLastError();
}

}  // namespace pa
