/*
 * pa_b200.h -- C ABI of the B200-native paged-attention decode library (libpa_b200.so).
 *
 * Plain pointers and sizes only: every tensor argument is a raw device pointer to a
 * contiguous buffer, every size is an int, the stream is a cudaStream_t passed as void*.
 * Each entry point validates its arguments on the host, launches asynchronously on `stream`
 * and returns PA_OK (0) or a PA_ERR_* code; pa_last_error() gives the message. Nothing here
 * aborts, traps or synchronises the device, except pa_read_status().
 *
 * Paged KV layout (the reference's, tests/paged_decode_attn.py:6-7,76-81,156-164):
 *   k_cache  [num_blocks, num_kv_heads, head_dim/8, block_size, 8]   fp16, int8 or fp8 e4m3
 *   v_cache  [num_blocks, num_kv_heads, head_dim,   block_size]      fp16, int8 or fp8 e4m3
 *   k_scales [num_blocks, num_kv_heads, block_size] fp32  (int8 and fp8 caches)
 *   v_scales [num_blocks, num_kv_heads, block_size] fp32
 *   block_table  [num_seqs, max_blocks_per_seq] int32
 *   context_lens [num_seqs] int32
 *   q, out [num_seqs, num_heads, head_dim] fp16 (bf16 with pa_decode_bf16q)
 * Supported: head_dim 128, block_size a multiple of 16 dividing 128, x = 8, num_heads a
 * multiple of num_kv_heads, num_blocks * num_kv_heads below 2^28 page rows.
 *
 * Workspace: the decode entry points need a device workspace of
 * pa_decode_workspace_bytes(...) bytes, zero-filled once before its first use (for example
 * with cudaMemset). The kernels leave it ready for the next call. Calls that share one
 * workspace must be ordered on one stream. Word 0 of the workspace is the device status
 * word: kernels OR PA_ERR_* bits into it (bad context length, bad block id, a wait that gave
 * up); pa_read_status() reads and clears it.
 */
#ifndef PA_B200_H
#define PA_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes (host return values and device status bits) ---- */
#define PA_OK 0
#define PA_ERR_INVALID_ARG 1    /* a host-side argument check failed */
#define PA_ERR_UNSUPPORTED 2    /* shape or dtype outside what this build implements */
#define PA_ERR_CUDA 4           /* a CUDA runtime or driver call failed */
#define PA_ERR_WORKSPACE 8      /* workspace missing or smaller than required */
#define PA_ERR_EMPTY_CONTEXT 16 /* device: a context length was < 1 */
#define PA_ERR_CONTEXT_RANGE 32 /* device: context length > max_blocks_per_seq * block_size */
#define PA_ERR_BLOCK_ID 64      /* device: a block_table entry outside [0, num_blocks) */
#define PA_ERR_TIMEOUT 128      /* device: a bounded wait gave up (about one second) */
#define PA_ERR_SLOT 256         /* device: a slot_mapping entry outside the cache */
#define PA_ERR_Q_RANGE 512      /* device: a bf16 q value outside the fp16 range (saturated) */

/* ---- dtype codes ---- */
#define PA_DTYPE_F16 0
#define PA_DTYPE_BF16 1
#define PA_DTYPE_F32 2
#define PA_DTYPE_I8 3
#define PA_DTYPE_FP8E4M3 4 /* fp8 e4m3 cache values with per-token fp32 scales */

/* ---- per-tensor scale semantics for pa_absmax_scale ---- */
/* quantize_per_tensor (tests/paged_decode_attn.py:115-121): clamp_min(1e-8) in the input
 * dtype, then amax/127 rounded to the input dtype. */
#define PA_SCALE_CLAMP_THEN_DIVIDE 0
/* PagedKVCache.prefill per-tensor (benchmarks/int8_bridge/paged_cache.py:101-102): amax/127
 * rounded to the input dtype, widened to fp32, then clamp_min(1e-8) in fp32. */
#define PA_SCALE_DIVIDE_THEN_CLAMP 1

int pa_version(void);
const char* pa_last_error(void);
const char* pa_status_string(int status);

/* ------------------------------------------------------------------------------------
 * Decode workspace size for one call shape on the current device (0 for an unsupported
 * shape). kv_dtype is PA_DTYPE_F16, PA_DTYPE_I8 or PA_DTYPE_FP8E4M3; splitk selects the
 * split-K partition/reduce pair (nonzero) or the single-pass op (zero).
 * ---------------------------------------------------------------------------------- */
size_t pa_decode_workspace_bytes(int num_seqs, int num_heads, int num_kv_heads, int head_dim,
                                 int max_blocks_per_seq, int block_size, int kv_dtype,
                                 int splitk);

/* Read the device status word of a workspace (synchronises `stream`), then clear it. */
int pa_read_status(void* workspace, int* status_out, void* stream);

/* Zero a workspace's status word and arrival counters (its first min(workspace_bytes,
 * 256 B + 1 MiB) bytes) on `stream`. A decode that stopped part-way on a device error (a
 * wait that gave up) can leave counters set, so after pa_read_status reports a nonzero status
 * call this before the next decode on that workspace. The reference has no workspace. */
int pa_reset_workspace(void* workspace, size_t workspace_bytes, void* stream);

/* ------------------------------------------------------------------------------------
 * Single-pass decode, FP16 KV cache: one launch, fused cross-split log-sum-exp combine.
 * Replaces the launchers behind paged_decode_attention / paged_decode_attn_{vec,online,warp}
 * (kernels/paged_attention_naive.cu:125-167, paged_attention_v1_vectorized.cu:112-151,
 * paged_attention_v2_online.cu:145-184, paged_attention_v3_warp.cu:137-176; registered in
 * kernels/bindings.cpp:45-50).
 * ---------------------------------------------------------------------------------- */
int pa_decode_f16(void* out, const void* q, const void* k_cache, const void* v_cache,
                  const int32_t* block_table, const int32_t* context_lens, int num_seqs,
                  int num_heads, int num_kv_heads, int head_dim, int num_blocks, int block_size,
                  int max_blocks_per_seq, float scale, void* workspace, size_t workspace_bytes,
                  void* stream);

/* Single-pass decode, INT8 KV cache with per-token fp32 scales (dequant fused).
 * Replaces paged_decode_attn_warp_int8 (kernels/paged_attention_v5_warp_int8.cu:150-197;
 * kernels/bindings.cpp:54). */
int pa_decode_i8(void* out, const void* q, const void* k_cache, const void* v_cache,
                 const float* k_scales, const float* v_scales, const int32_t* block_table,
                 const int32_t* context_lens, int num_seqs, int num_heads, int num_kv_heads,
                 int head_dim, int num_blocks, int block_size, int max_blocks_per_seq,
                 float scale, void* workspace, size_t workspace_bytes, void* stream);

/* Split-K flash-decoding, FP16 KV: partition kernel over 512-token splits, then the LSE
 * reduce kernel. Replaces paged_decode_attn_splitk (kernels/paged_attention_v4_splitk.cu:
 * 191-248; kernels/bindings.cpp:52). */
int pa_splitk_f16(void* out, const void* q, const void* k_cache, const void* v_cache,
                  const int32_t* block_table, const int32_t* context_lens, int num_seqs,
                  int num_heads, int num_kv_heads, int head_dim, int num_blocks, int block_size,
                  int max_blocks_per_seq, float scale, void* workspace, size_t workspace_bytes,
                  void* stream);

/* Split-K flash-decoding, INT8 KV. Replaces paged_decode_attn_splitk_int8
 * (kernels/paged_attention_v6_splitk_int8.cu:194-259; kernels/bindings.cpp:56). */
int pa_splitk_i8(void* out, const void* q, const void* k_cache, const void* v_cache,
                 const float* k_scales, const float* v_scales, const int32_t* block_table,
                 const int32_t* context_lens, int num_seqs, int num_heads, int num_kv_heads,
                 int head_dim, int num_blocks, int block_size, int max_blocks_per_seq,
                 float scale, void* workspace, size_t workspace_bytes, void* stream);

/* FP8 (e4m3) KV cache: the INT8 page layout with e4m3 bytes and per-token fp32 scales
 * (value = e4m3 * scale; see pa_quantize_into_cache_fp8). Same arguments as pa_decode_i8 /
 * pa_splitk_i8. The reference lists an FP8 KV variant as future work
 * (report/benchmark_report.md:196-197) and has no kernel for it. */
int pa_decode_fp8(void* out, const void* q, const void* k_cache, const void* v_cache,
                  const float* k_scales, const float* v_scales, const int32_t* block_table,
                  const int32_t* context_lens, int num_seqs, int num_heads, int num_kv_heads,
                  int head_dim, int num_blocks, int block_size, int max_blocks_per_seq,
                  float scale, void* workspace, size_t workspace_bytes, void* stream);
int pa_splitk_fp8(void* out, const void* q, const void* k_cache, const void* v_cache,
                  const float* k_scales, const float* v_scales, const int32_t* block_table,
                  const int32_t* context_lens, int num_seqs, int num_heads, int num_kv_heads,
                  int head_dim, int num_blocks, int block_size, int max_blocks_per_seq,
                  float scale, void* workspace, size_t workspace_bytes, void* stream);

/* ------------------------------------------------------------------------------------
 * Decode step: append every sequence's new token to the cache, then decode over the whole
 * context, in one call. context_lens[b] already counts the new token; new_k / new_v
 * [num_seqs, num_kv_heads, head_dim] (new_dtype F16, BF16 or F32, token stride
 * new_token_stride elements) are written at position context_lens[b] - 1 of sequence b through
 * block_table, quantised like pa_quantize_into_cache (int8; with k_fixed_scale / v_fixed_scale
 * the per-tensor scales), like pa_quantize_into_cache_fp8 (fp8) or copied (fp16), and the
 * decode (splitk: the split-K pair) reads them. With fused nonzero and at most 16 q heads per
 * kv head, the decode kernel writes each token itself, in the warp that reads the token's
 * page, just before that page's copy: no extra launch. Otherwise (fused zero, or larger
 * groups) a write kernel runs first. Both give bit-identical caches and outputs.
 * Replaces the reference bridge's decode step, PagedKVCache.decode_append
 * (benchmarks/int8_bridge/paged_cache.py:132-156) followed by the split-K op
 * (benchmarks/int8_bridge/qwen_paged_attn.py:61-73), for a whole batch.
 * ---------------------------------------------------------------------------------- */
int pa_decode_step(int kv_dtype, void* out, const void* q, const void* new_k,
                   const void* new_v, int new_dtype, int64_t new_token_stride, void* k_cache,
                   void* v_cache, float* k_scales, float* v_scales, const float* k_fixed_scale,
                   const float* v_fixed_scale, const int32_t* block_table,
                   const int32_t* context_lens, int num_seqs, int num_heads, int num_kv_heads,
                   int head_dim, int num_blocks, int block_size, int max_blocks_per_seq,
                   float scale, int splitk, int fused, void* workspace, size_t workspace_bytes,
                   void* stream);

/* FP16 single-pass decode that allocates nothing and takes no workspace, for callers that
 * cannot allocate device memory when they run attention: plugins whose host framework owns
 * all device memory, and serving loops that must stay out of any allocator. Its scratch is a
 * 12 MiB static device array that every GPU loading this code keeps until the process exits;
 * shapes whose scratch exceeds it (more than 8 q heads per kv head) are rejected with
 * PA_ERR_WORKSPACE. The first call on a device looks up the array's address and should come
 * before any stream capture. Calls share the array: calls that overlap on the GPU race, so
 * order them on one stream. Device-side errors (bad context length, bad block id, a wait
 * that gave up) accumulate in the array's status word until
 * pa_decode_f16_noalloc_read_status reads and clears them. This entry point has no
 * counterpart in the reference. */
int pa_decode_f16_noalloc(void* out, const void* q, const void* k_cache, const void* v_cache,
                          const int32_t* block_table, const int32_t* context_lens, int num_seqs,
                          int num_heads, int num_kv_heads, int head_dim, int num_blocks,
                          int block_size, int max_blocks_per_seq, float scale, void* stream);

/* Read the device status word of pa_decode_f16_noalloc's static scratch on the current
 * device (synchronises `stream`), then clear it; the PA_ERR_* bits of every call since the
 * last read. No counterpart in the reference. */
int pa_decode_f16_noalloc_read_status(int* status_out, void* stream);

/* Decode with bf16 activations: q and out are bf16 [num_seqs, num_heads, head_dim]; the cache
 * is fp16 (kv_dtype PA_DTYPE_F16), per-token int8 (PA_DTYPE_I8) or per-token fp8 e4m3
 * (PA_DTYPE_FP8E4M3), the last two with k_scales/v_scales; splitk selects the split-K pair.
 * q is converted to fp16 on the device (exact for magnitudes in the fp16 normal range; larger
 * values saturate and set PA_ERR_Q_RANGE in the status word), the fp16 decode runs, and its
 * output is rounded once to bf16. The workspace holds the decode workspace followed by the
 * fp16 copies: size it with pa_decode_bf16q_workspace_bytes. This is the BF16-q support the
 * reference lists as future work (report/benchmark_report.md:196-197); the reference's own
 * ops take fp16 q only. */
size_t pa_decode_bf16q_workspace_bytes(int num_seqs, int num_heads, int num_kv_heads,
                                       int head_dim, int max_blocks_per_seq, int block_size,
                                       int kv_dtype, int splitk);
int pa_decode_bf16q(void* out, const void* q, const void* k_cache, const void* v_cache,
                    const float* k_scales, const float* v_scales, const int32_t* block_table,
                    const int32_t* context_lens, int num_seqs, int num_heads, int num_kv_heads,
                    int head_dim, int num_blocks, int block_size, int max_blocks_per_seq,
                    int kv_dtype, int splitk, float scale, void* workspace,
                    size_t workspace_bytes, void* stream);

/* Failure-path self-test: one warp waits on a barrier that nothing completes; the bounded wait
 * gives up after about a second and ORs PA_ERR_TIMEOUT into the status word at workspace[0].
 * The context stays usable. No counterpart in the reference. */
int pa_selftest_bounded_wait(void* workspace, void* stream);

/* ------------------------------------------------------------------------------------
 * Per-sequence partial decode for split-K across GPUs: like pa_decode_*, but instead of
 * the normalised fp16 output it writes, per (sequence, kv-head), an un-normalised partial
 * to `partials` (layout: [num_seqs*num_kv_heads][pa_partial_floats(...)] fp32; within a
 * slot O[head_dim][heads_per_slot] then m[heads_per_slot] then l[heads_per_slot], m in
 * log2 units). A sequence with context 0 yields an empty partial (m=-inf, l=0).
 * Generalises the partition kernel of kernels/paged_attention_v4_splitk.cu:28-153 from a
 * token split inside one GPU to a token range owned by one GPU.
 * ---------------------------------------------------------------------------------- */
int pa_partial_floats(int num_heads, int num_kv_heads, int head_dim);
int pa_decode_partial(int kv_dtype, float* partials, const void* q, const void* k_cache,
                      const void* v_cache, const float* k_scales, const float* v_scales,
                      const int32_t* block_table, const int32_t* context_lens, int num_seqs,
                      int num_heads, int num_kv_heads, int head_dim, int num_blocks,
                      int block_size, int max_blocks_per_seq, float scale, void* workspace,
                      size_t workspace_bytes, void* stream);

/* LSE merge of `num_parts` partial buffers laid out [num_parts][num_seqs*num_kv_heads][slot]
 * (as gathered from pa_decode_partial on num_parts GPUs) into out [num_seqs, num_heads,
 * head_dim] fp16. The arithmetic of kernels/paged_attention_v4_splitk.cu:156-187. */
int pa_merge_partials(void* out, const float* partials, int num_parts, int num_seqs,
                      int num_heads, int num_kv_heads, int head_dim, int* status, void* stream);

/* ------------------------------------------------------------------------------------
 * Quantize-into-cache write (per-token symmetric INT8), one row per (token, kv-head):
 *   scale = round_to_in_dtype(max(amax, in_dtype(1e-8)) / 127)   (fp32 afterwards)
 *   q     = clamp(round_half_even(x / scale), -127, 127)
 * bit-exact with quantize_per_token (tests/paged_decode_attn.py:106-112) and the decode-step
 * write of PagedKVCache.decode_append (benchmarks/int8_bridge/paged_cache.py:132-156).
 * k, v: [num_tokens, num_kv_heads, head_dim] in in_dtype (F16, BF16 or F32), rows contiguous,
 * token stride `token_stride` elements. slot_mapping[i] = block*block_size + offset; a
 * negative slot skips the token. If k_fixed_scale / v_fixed_scale are non-null they point to
 * one device fp32 scale each (per-tensor mode, paged_cache.py:143-145) and that scale is
 * written into the scale slots instead. status (nullable) receives PA_ERR_SLOT bits.
 * Large writes (about 19 K tokens x 2 kv heads and up on a B200) write every run of 16
 * consecutive tokens whose slots are 16 consecutive slots starting at a multiple of 16 (a
 * prefill's full 16-token groups, block_size a multiple of 16) with whole-group stores, several
 * times faster than the row-by-row write that the other tokens, and small writes, take; the
 * result is the same either way.
 * ---------------------------------------------------------------------------------- */
int pa_quantize_into_cache(const void* k, const void* v, int in_dtype, int64_t token_stride,
                           const int32_t* slot_mapping, int num_tokens, int num_kv_heads,
                           int head_dim, void* k_cache, void* v_cache, float* k_scales,
                           float* v_scales, int num_blocks, int block_size,
                           const float* k_fixed_scale, const float* v_fixed_scale, int* status,
                           void* stream);

/* Per-token FP8 (e4m3) write, same rows and slots as pa_quantize_into_cache:
 *   scale = amax / 448 (fp32 IEEE divide; 448 is the largest finite e4m3)
 *   q     = e4m3(x / scale), round-to-nearest-even, saturating to +-448; a zero row gives
 *           scale 0 and zeros. */
int pa_quantize_into_cache_fp8(const void* k, const void* v, int in_dtype, int64_t token_stride,
                               const int32_t* slot_mapping, int num_tokens, int num_kv_heads,
                               int head_dim, void* k_cache, void* v_cache, float* k_scales,
                               float* v_scales, int num_blocks, int block_size, int* status,
                               void* stream);

/* FP16 copy-into-cache (no quantisation), same slot semantics: the fp16 cache write of
 * PagedKVCache.decode_append / build_paged_kv_cache (paged_cache.py:147-150,
 * tests/paged_decode_attn.py:96-99). in_dtype F16, BF16 or F32 (rounded to fp16). */
int pa_write_into_cache_f16(const void* k, const void* v, int in_dtype, int64_t token_stride,
                            const int32_t* slot_mapping, int num_tokens, int num_kv_heads,
                            int head_dim, void* k_cache, void* v_cache, int num_blocks,
                            int block_size, int* status, void* stream);

/* Block-granular bulk write (prefill scatter): k, v [num_seqs, max_len, num_kv_heads,
 * head_dim]; every block j < ceil(context_lens[b]/block_size) of sequence b is written in
 * full into physical block block_table[b, j], tokens past the context as zeros (scale 0).
 * cache_dtype PA_DTYPE_I8 quantises per token (or with the fixed scales), PA_DTYPE_F16
 * copies. Replaces the scatter loops of build_paged_kv_cache{,_int8}
 * (tests/paged_decode_attn.py:84-99,178-197) and PagedKVCache.prefill (paged_cache.py:88-130).
 */
int pa_prefill_into_cache(const void* k, const void* v, int in_dtype, int num_seqs,
                          int max_len, int num_kv_heads, int head_dim,
                          const int32_t* block_table, const int32_t* context_lens,
                          int max_blocks_per_seq, int cache_dtype, void* k_cache, void* v_cache,
                          float* k_scales, float* v_scales, int num_blocks, int block_size,
                          const float* k_fixed_scale, const float* v_fixed_scale, int* status,
                          void* stream);

/* Per-tensor absmax scale of n elements of x (in_dtype F16, BF16 or F32) into *scale_out
 * (device fp32), with the rounding of `semantics` (PA_SCALE_*). scratch: 4 device bytes. */
int pa_absmax_scale(const void* x, int in_dtype, int64_t n, float* scale_out, int semantics,
                    void* scratch, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* PA_B200_H */
