// Internal host/device interface between the C-ABI layer (capi.cu) and the kernels.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <stddef.h>
#include <stdint.h>

#include "pa_status.h"

namespace pa {

constexpr int kBMax = 1024;       // sequences per decode launch (the host splits larger batches)
constexpr int kSubTokens = 16;    // tokens per tensor-core tile ("subpage")
constexpr int kSplitPages = 32;   // split-K partition: 512 tokens = 32 subpages
constexpr int kWsHeader = 256;    // workspace bytes before the counters (status word first)
// Arrival counters occupy a fixed region right after the header, whatever the call shape, so
// a workspace reused across shapes always presents zeroed counters (each launch leaves the
// counters it used at zero). Batches are split so that sequences x segments fit.
constexpr int kCounterCap = 1 << 18;
constexpr size_t kWsPartOffset = kWsHeader + sizeof(int) * (size_t)kCounterCap;

enum DecodeMode : int {
  kModeStream = 0,    // single pass: page-balanced ranges, fused LSE combine, fp16 out
  kModeSplit = 1,     // split-K partition: one partial per 512-token split
  kModePartial = 2,   // per-(sequence, kv-head) partial for cross-GPU merging
};

struct DecodeArgs {
  __half* out;                 // [B, H, D] (stream mode)
  const __half* q;             // [B, H, D]
  const int* block_table;      // [B, max_blocks]
  const int* context_lens;     // [B]
  const uint8_t* v_base;       // V cache base (1-D bulk path when block_size == 16)
  const float* ks_base;        // K scales base (int8, block_size == 16)
  const float* vs_base;        // V scales base
  float* part;                 // partial slots
  int* counters;               // per-segment arrival counters (stream mode)
  int* status;                 // device status word
  float* part_out;             // per-segment partial output (partial mode)
  int B, H, KVH, G, HT, max_blocks, bs, subs, NB;
  int mode;
  int s_max;                   // split mode: splits per segment slot stride
  int total_warps;
  int bulk;                    // 1: V and scales via 1-D bulk copies (block_size == 16)
  float qk_scale_log2;         // scale * log2(e)
  // Decode step (new_k non-null): every sequence's new token, at position context_lens[b] - 1,
  // is quantised by the warp that reads the page holding it (its rows arrive with the page's
  // copy), placed into the staged page and stored into the cache (only when one head tile
  // covers each kv head, so that exactly one warp reads the page).
  const void* new_k;           // [B, KVH, D] 16-bit rows (16-byte aligned), new_stride elements
  const void* new_v;           //   per token (a multiple of 8)
  int new_dtype;               // PA_DTYPE_F16 or PA_DTYPE_BF16
  long long new_stride;
  const float* new_kfix;       // int8 per-tensor scales (null: per-token)
  const float* new_vfix;
  void* kc_w;                  // cache and scale bases the write stores into
  void* vc_w;
  float* ks_w;
  float* vs_w;
};

struct ReduceArgs {
  __half* out;
  const float* part;
  const int* context_lens;     // split mode: number of splits from the context length
  int* status;
  int B, H, KVH, G, HT, max_blocks, bs;
  int num_parts;               // > 0: fixed number of pieces per segment (cross-GPU merge)
  long long piece_stride;      // floats between consecutive pieces of one segment
  long long seg_stride;        // floats between consecutive segments
};

// Launch helpers implemented in decode.cu. They return a cudaError_t.
cudaError_t launch_decode(int kv_i8, int gt, const DecodeArgs& a, const CUtensorMap* maps,
                          int grid, cudaStream_t stream);
cudaError_t launch_reduce(int gt, const ReduceArgs& a, int max_pieces, cudaStream_t stream);
int decode_warps_per_cta(int kv_i8, int gt);
// Token-granular cache writes; kind selects the cache type.
enum RowKind {
  kRowsF16 = 0,  // fp16 copy
  kRowsI8 = 1,   // int8, per-token or fixed scale
  kRowsFP8 = 2,  // fp8 e4m3, per-token scale
};
cudaError_t launch_write_rows(int in_dtype, int kind, int D, const void* k, const void* v,
                              long long token_stride, const int* slots, int N, int KVH,
                              void* kc, void* vc, float* ks, float* vs, int NB, int bs,
                              const float* kfix, const float* vfix, int* status,
                              cudaStream_t st);
// The decode step's new-token write as its own kernel (one warp per sequence x kv head x K|V;
// slot from block_table and context_lens), for shapes where the fused write does not apply.
cudaError_t launch_step_rows(int in_dtype, int kind, const void* k, const void* v,
                             long long token_stride, const int* block_table,
                             const int* context_lens, int max_blocks, int B, int KVH, void* kc,
                             void* vc, float* ks, float* vs, int NB, int bs, const float* kfix,
                             const float* vfix, int* status, cudaStream_t st);
cudaError_t launch_prefill(int in_dtype, bool i8, const void* k, const void* v, int S, int L,
                           int KVH, const int* bt, const int* cl, int max_blocks, void* kc,
                           void* vc, float* ks, float* vs, int NB, int bs, const float* kfix,
                           const float* vfix, int* status, cudaStream_t st);
cudaError_t launch_absmax_scale(int in_dtype, const void* x, long long n, float* scale_out,
                                int semantics, unsigned int* scratch, int num_sms,
                                cudaStream_t st);

// bf16 <-> fp16 activation conversions (n a multiple of 8, 16-byte aligned buffers).
cudaError_t launch_bf16_to_f16(const void* in, void* out, long long n, int* status, int num_sms,
                               cudaStream_t st);
cudaError_t launch_f16_to_bf16(const void* in, void* out, long long n, int num_sms,
                               cudaStream_t st);
// One warp waits on an mbarrier that nothing completes; the bounded wait must give up after
// about a second and set PA_ERR_TIMEOUT in *status (exercises the failure path).
cudaError_t launch_selftest_wait(int* status, cudaStream_t st);

// Record a message for pa_last_error() and return `code` (defined in capi.cu).
int fail_status(int code, const char* fmt, ...);

// Partial slot size in floats: O[D][GT] + m[GT] + l[GT].
inline int slot_floats(int head_dim, int gt) { return (head_dim + 2) * gt; }

}  // namespace pa
