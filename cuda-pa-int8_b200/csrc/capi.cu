// C-ABI entry points of libpa_b200.so (declared in include/pa_b200.h).
//
// Host-side responsibilities: argument validation with the reference's error conditions
// (kernels/paged_attention_v6_splitk_int8.cu:201-221 and siblings), TMA tensor-map
// construction (cached per cache pointer/shape), workspace layout, grid sizing from the SM
// count, and splitting batches larger than one launch handles. No call here allocates device
// memory or synchronises the device, except pa_read_status().

#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>

#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>

#include <nvtx3/nvToolsExt.h>

#include "pa_internal.h"

namespace {

thread_local std::string g_err;

int vfail(int code, const char* fmt, va_list ap) {
  char buf[512];
  vsnprintf(buf, sizeof(buf), fmt, ap);
  g_err = buf;
  return code;
}

int fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vfail(code, fmt, ap);
  va_end(ap);
  return code;
}

int cuda_fail(cudaError_t e, const char* what) {
  return fail(PA_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

bool aligned(const void* p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

// An NVTX range named after the entry point, around its host work and launches, so profiler
// timelines (nsys, ncu's NVTX filters) show which library call issued which kernels. Without
// an attached tool the NVTX calls return immediately.
struct NvtxRange {
  explicit NvtxRange(const char* name) { nvtxRangePushA(name); }
  ~NvtxRange() { nvtxRangePop(); }
  NvtxRange(const NvtxRange&) = delete;
  NvtxRange& operator=(const NvtxRange&) = delete;
};

// ---- device properties ------------------------------------------------------------------
int num_sms_current(int* dev_out) {
  static int cache[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return -1;
  if (dev_out) *dev_out = dev;
  if (dev < 0 || dev >= 64) return -1;
  if (cache[dev] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return -1;
    cache[dev] = n;
  }
  return cache[dev];
}

// ---- tensor maps ----------------------------------------------------------------------------
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess) {
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    }
  });
  return fn;
}

enum MapKind { kMapKI8 = 0, kMapKF16 = 1, kMapVI8 = 2, kMapVF16 = 3, kMapScale = 4 };

struct MapKey {
  const void* ptr;
  int kind, nb, kvh, bs, d;
  bool operator==(const MapKey& o) const {
    return ptr == o.ptr && kind == o.kind && nb == o.nb && kvh == o.kvh && bs == o.bs &&
           d == o.d;
  }
};

struct MapEntry {
  MapKey key;
  CUtensorMap map;
  bool used;
};

constexpr int kMapCache = 64;
MapEntry g_maps[kMapCache];
int g_map_next = 0;
std::mutex g_map_mu;

int build_map(const MapKey& k, CUtensorMap* out) {
  auto enc = encode_fn();
  if (enc == nullptr) return fail(PA_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
  const cuuint64_t pages = (cuuint64_t)k.nb * (cuuint64_t)k.kvh;
  const cuuint64_t bs = (cuuint64_t)k.bs;
  const cuuint64_t D = (cuuint64_t)k.d;
  cuuint64_t dims[4];
  cuuint64_t strides[3];
  cuuint32_t box[4];
  cuuint32_t estr[4] = {1, 1, 1, 1};
  cuuint32_t rank = 0;
  CUtensorMapDataType dt = CU_TENSOR_MAP_DATA_TYPE_UINT8;
  CUtensorMapSwizzle sw = CU_TENSOR_MAP_SWIZZLE_NONE;
  switch (k.kind) {
    case kMapKI8:  // [pages][D/8][bs*8 bytes], box = 16 tokens x all chunks, 128B swizzle
      rank = 3;
      dims[0] = bs * 8; dims[1] = D / 8; dims[2] = pages;
      strides[0] = bs * 8; strides[1] = D * bs;
      box[0] = 128; box[1] = (cuuint32_t)(D / 8); box[2] = 1;
      sw = CU_TENSOR_MAP_SWIZZLE_128B;
      break;
    case kMapKF16:  // [pages][D/8][bs/8 octets][64 halves], box {64, 2, D/8, 1}, 128B swizzle
      rank = 4;
      dt = CU_TENSOR_MAP_DATA_TYPE_UINT16;
      dims[0] = 64; dims[1] = bs / 8; dims[2] = D / 8; dims[3] = pages;
      strides[0] = 128; strides[1] = bs * 16; strides[2] = D * bs * 2;
      box[0] = 64; box[1] = 2; box[2] = (cuuint32_t)(D / 8); box[3] = 1;
      sw = CU_TENSOR_MAP_SWIZZLE_128B;
      break;
    case kMapVI8:  // [pages][D][bs], box {16, D, 1}
      rank = 3;
      dims[0] = bs; dims[1] = D; dims[2] = pages;
      strides[0] = bs; strides[1] = D * bs;
      box[0] = 16; box[1] = (cuuint32_t)D; box[2] = 1;
      break;
    case kMapVF16:
      rank = 3;
      dt = CU_TENSOR_MAP_DATA_TYPE_UINT16;
      dims[0] = bs; dims[1] = D; dims[2] = pages;
      strides[0] = bs * 2; strides[1] = D * bs * 2;
      box[0] = 16; box[1] = (cuuint32_t)D; box[2] = 1;
      break;
    case kMapScale:  // [pages][bs] fp32, box {16, 1}
      rank = 2;
      dt = CU_TENSOR_MAP_DATA_TYPE_FLOAT32;
      dims[0] = bs; dims[1] = pages;
      strides[0] = bs * 4;
      box[0] = 16; box[1] = 1;
      break;
    default:
      return fail(PA_ERR_INVALID_ARG, "bad tensor map kind");
  }
  CUresult r = enc(out, dt, rank, const_cast<void*>(k.ptr), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(PA_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return PA_OK;
}

int get_map(const MapKey& k, CUtensorMap* out) {
  std::lock_guard<std::mutex> lock(g_map_mu);
  for (int i = 0; i < kMapCache; ++i) {
    if (g_maps[i].used && g_maps[i].key == k) {
      *out = g_maps[i].map;
      return PA_OK;
    }
  }
  CUtensorMap m;
  int rc = build_map(k, &m);
  if (rc != PA_OK) return rc;
  MapEntry& e = g_maps[g_map_next];
  g_map_next = (g_map_next + 1) % kMapCache;
  e.key = k;
  e.map = m;
  e.used = true;
  *out = m;
  return PA_OK;
}

// ---- decode shapes and workspace -------------------------------------------------------
struct Shape {
  int G, GT, HT, SEGS, SLOT, s_max, warps_per_cta, sms, chunk_b;
};

int check_common(int B, int H, int KVH, int D, int NB, int bs, int max_blocks) {
  if (B < 0 || H <= 0 || KVH <= 0 || NB <= 0 || max_blocks <= 0)
    return fail(PA_ERR_INVALID_ARG,
                "invalid sizes (num_seqs=%d num_heads=%d num_kv_heads=%d num_blocks=%d "
                "max_blocks_per_seq=%d)",
                B, H, KVH, NB, max_blocks);
  if (H % KVH != 0)
    return fail(PA_ERR_INVALID_ARG, "num_heads (%d) must be a multiple of num_kv_heads (%d)", H,
                KVH);
  if (D != 128) return fail(PA_ERR_UNSUPPORTED, "head_dim %d unsupported (this build: 128)", D);
  // The kernel's copy producer packs (page row << 3 | subpage) into an int, where
  // page row = block * num_kv_heads + kv_head: 2^28 page rows (1 TB of fp16 K pages).
  if ((long long)NB * KVH >= (1LL << 28))
    return fail(PA_ERR_UNSUPPORTED,
                "num_blocks * num_kv_heads = %lld page rows; this build addresses fewer than "
                "2^28",
                (long long)NB * KVH);
  if (bs % 16 != 0 || 128 % bs != 0)
    return fail(PA_ERR_INVALID_ARG,
                "block_size must divide TILE (multiple of 16); got %d (supported: 16, 32, 64, "
                "128)",
                bs);
  return PA_OK;
}

int make_shape(int kv_i8, int mode, int B, int H, int KVH, int D, int bs, int max_blocks,
               Shape* s) {
  s->G = H / KVH;
  s->GT = s->G <= 8 ? 8 : 16;
  s->HT = (s->G + s->GT - 1) / s->GT;
  s->SEGS = KVH * s->HT;
  s->SLOT = pa::slot_floats(D, s->GT);
  const long long subpages = ((long long)max_blocks * bs + pa::kSubTokens - 1) / pa::kSubTokens;
  s->s_max = (int)((subpages + pa::kSplitPages - 1) / pa::kSplitPages);
  s->warps_per_cta = pa::decode_warps_per_cta(kv_i8, s->GT);
  s->sms = num_sms_current(nullptr);
  if (s->sms <= 0) return fail(PA_ERR_CUDA, "cannot query the current device");
  // Sequences per launch: the in-kernel scan holds kBMax, and the flattened page count must
  // stay below 2^31.
  long long per_seq = subpages * s->SEGS;
  long long cb = pa::kBMax;
  if (s->SEGS > pa::kCounterCap)
    return fail(PA_ERR_UNSUPPORTED, "too many kv-head segments per sequence (%d)", s->SEGS);
  if (cb * s->SEGS > pa::kCounterCap) cb = pa::kCounterCap / s->SEGS;
  while (cb > 1 && cb * per_seq >= (1LL << 31)) cb >>= 1;
  if (per_seq >= (1LL << 31)) return fail(PA_ERR_UNSUPPORTED, "context too long for one launch");
  s->chunk_b = (int)cb;
  (void)mode;
  (void)B;
  return PA_OK;
}

size_t ws_bytes_for(const Shape& s, int mode, int B) {
  const long long cb = B < s.chunk_b ? B : s.chunk_b;
  const size_t off = pa::kWsPartOffset;
  size_t parts;
  if (mode == pa::kModeSplit) {
    parts = (size_t)(cb > 0 ? cb : 1) * s.SEGS * s.s_max * s.SLOT * sizeof(float);
  } else {
    parts = (size_t)s.sms * s.warps_per_cta * 2 * s.SLOT * sizeof(float);
  }
  return off + parts;
}

// The new token of a decode step (pa_decode_step): rows, their dtype, the optional per-tensor
// scales, and whether the decode kernel may write it itself.
struct StepWrite {
  const void* k;
  const void* v;
  int dtype;
  long long stride;  // elements per token
  const float* kfix;
  const float* vfix;
  bool fused;
};

int decode_impl(int mode, int kv_i8, void* out, float* part_out, const void* q,
                const void* k_cache, const void* v_cache, const float* k_scales,
                const float* v_scales, const int32_t* block_table, const int32_t* context_lens,
                int B, int H, int KVH, int D, int NB, int bs, int max_blocks, float scale,
                void* workspace, size_t workspace_bytes, void* stream,
                const StepWrite* sw = nullptr) {
  int rc = check_common(B, H, KVH, D, NB, bs, max_blocks);
  if (rc != PA_OK) return rc;
  if (B == 0) return PA_OK;
  if (q == nullptr || k_cache == nullptr || v_cache == nullptr || block_table == nullptr ||
      context_lens == nullptr || workspace == nullptr)
    return fail(PA_ERR_INVALID_ARG, "null pointer argument");
  if (mode == pa::kModePartial ? part_out == nullptr : out == nullptr)
    return fail(PA_ERR_INVALID_ARG, "null output pointer");
  if (kv_i8 && (k_scales == nullptr || v_scales == nullptr))
    return fail(PA_ERR_INVALID_ARG, "int8 cache needs k_scales and v_scales");
  if (!aligned(q, 16) || (out && !aligned(out, 16)) || !aligned(k_cache, 16) ||
      !aligned(v_cache, 16) || (kv_i8 && (!aligned(k_scales, 16) || !aligned(v_scales, 16))) ||
      !aligned(workspace, 256) || (part_out && !aligned(part_out, 16)))
    return fail(PA_ERR_INVALID_ARG, "tensors must be 16-byte aligned (workspace 256-byte)");
  if (!(scale == scale)) return fail(PA_ERR_INVALID_ARG, "scale is NaN");

  Shape s;
  rc = make_shape(kv_i8, mode, B, H, KVH, D, bs, max_blocks, &s);
  if (rc != PA_OK) return rc;
  const size_t need = ws_bytes_for(s, mode, B);
  if (workspace_bytes < need)
    return fail(PA_ERR_WORKSPACE, "workspace too small: %zu < %zu bytes", workspace_bytes, need);

  CUtensorMap maps[4];
  memset(maps, 0, sizeof(maps));
  rc = get_map({k_cache, kv_i8 ? kMapKI8 : kMapKF16, NB, KVH, bs, D}, &maps[0]);
  if (rc != PA_OK) return rc;
  const bool bulk = (bs == pa::kSubTokens);
  if (!bulk) {
    rc = get_map({v_cache, kv_i8 ? kMapVI8 : kMapVF16, NB, KVH, bs, D}, &maps[1]);
    if (rc != PA_OK) return rc;
    if (kv_i8) {
      rc = get_map({k_scales, kMapScale, NB, KVH, bs, D}, &maps[2]);
      if (rc != PA_OK) return rc;
      rc = get_map({v_scales, kMapScale, NB, KVH, bs, D}, &maps[3]);
      if (rc != PA_OK) return rc;
    }
  }

  uint8_t* ws = static_cast<uint8_t*>(workspace);
  int* status = reinterpret_cast<int*>(ws);
  int* counters = reinterpret_cast<int*>(ws + pa::kWsHeader);
  float* part = reinterpret_cast<float*>(ws + pa::kWsPartOffset);
  cudaStream_t st = static_cast<cudaStream_t>(stream);

  // A decode step writes its new tokens first: inside the decode kernel when exactly one warp
  // reads each page (one head tile per kv head) and the rows can be bulk-copied (16-bit rows,
  // 16-byte aligned), else as its own launch before the decode.
  const int row_kind = kv_i8 == 1 ? pa::kRowsI8 : (kv_i8 == 2 ? pa::kRowsFP8 : pa::kRowsF16);
  const bool fuse = sw != nullptr && sw->fused && s.HT == 1 && sw->dtype != PA_DTYPE_F32 &&
                    aligned(sw->k, 16) && aligned(sw->v, 16) && (sw->stride * 2) % 16 == 0;
  if (sw != nullptr && !fuse) {
    cudaError_t e = pa::launch_step_rows(
        sw->dtype, row_kind, sw->k, sw->v, sw->stride, block_table, context_lens, max_blocks, B,
        KVH, const_cast<void*>(k_cache), const_cast<void*>(v_cache),
        const_cast<float*>(k_scales), const_cast<float*>(v_scales), NB, bs, sw->kfix, sw->vfix,
        status, st);
    if (e != cudaSuccess) return cuda_fail(e, "step write launch");
  }
  const size_t new_es = sw == nullptr ? 0 : (sw->dtype == PA_DTYPE_F32 ? 4 : 2);

  for (int c0 = 0; c0 < B; c0 += s.chunk_b) {
    const int nb = (B - c0) < s.chunk_b ? (B - c0) : s.chunk_b;
    pa::DecodeArgs a;
    memset(&a, 0, sizeof(a));
    a.out = out ? static_cast<__half*>(out) + (size_t)c0 * H * D : nullptr;
    a.q = static_cast<const __half*>(q) + (size_t)c0 * H * D;
    a.block_table = block_table + (size_t)c0 * max_blocks;
    a.context_lens = context_lens + c0;
    a.v_base = static_cast<const uint8_t*>(v_cache);
    a.ks_base = k_scales;
    a.vs_base = v_scales;
    a.part = part;
    a.counters = counters;
    a.status = status;
    a.part_out = part_out ? part_out + (size_t)c0 * s.SEGS * s.SLOT : nullptr;
    a.B = nb;
    a.H = H;
    a.KVH = KVH;
    a.G = s.G;
    a.HT = s.HT;
    a.max_blocks = max_blocks;
    a.bs = bs;
    a.subs = bs / pa::kSubTokens;
    a.NB = NB;
    a.mode = mode;
    a.s_max = s.s_max;
    a.bulk = bulk ? 1 : 0;
    a.qk_scale_log2 = scale * 1.4426950408889634f;
    if (fuse) {
      a.new_k = static_cast<const uint8_t*>(sw->k) + (size_t)c0 * sw->stride * new_es;
      a.new_v = static_cast<const uint8_t*>(sw->v) + (size_t)c0 * sw->stride * new_es;
      a.new_dtype = sw->dtype;
      a.new_stride = sw->stride;
      a.new_kfix = sw->kfix;
      a.new_vfix = sw->vfix;
      a.kc_w = const_cast<void*>(k_cache);
      a.vc_w = const_cast<void*>(v_cache);
      a.ks_w = const_cast<float*>(k_scales);
      a.vs_w = const_cast<float*>(v_scales);
    }
    // Grid: one CTA per SM; fewer only when there are fewer subpages than warps.
    const long long subpages = ((long long)max_blocks * bs + pa::kSubTokens - 1) / pa::kSubTokens;
    const long long t_max = (long long)nb * s.SEGS * subpages;
    long long want = (t_max + s.warps_per_cta - 1) / s.warps_per_cta;
    if (want < 1) want = 1;
    const int grid = (int)(want < s.sms ? want : s.sms);
    a.total_warps = grid * s.warps_per_cta;
    cudaError_t e = pa::launch_decode(kv_i8, s.GT, a, maps, grid, st);
    if (e != cudaSuccess) return cuda_fail(e, "decode launch");
    if (mode == pa::kModeSplit) {
      pa::ReduceArgs ra;
      memset(&ra, 0, sizeof(ra));
      ra.out = a.out;
      ra.part = part;
      ra.context_lens = a.context_lens;
      ra.status = status;
      ra.B = nb;
      ra.H = H;
      ra.KVH = KVH;
      ra.G = s.G;
      ra.HT = s.HT;
      ra.max_blocks = max_blocks;
      ra.bs = bs;
      ra.num_parts = 0;
      ra.piece_stride = s.SLOT;
      ra.seg_stride = (long long)s.s_max * s.SLOT;
      e = pa::launch_reduce(s.GT, ra, s.s_max, st);
      if (e != cudaSuccess) return cuda_fail(e, "reduce launch");
    }
  }
  return PA_OK;
}

int check_in_dtype(int dt) {
  if (dt != PA_DTYPE_F16 && dt != PA_DTYPE_BF16 && dt != PA_DTYPE_F32)
    return fail(PA_ERR_UNSUPPORTED, "input dtype code %d unsupported (fp16, bf16, fp32)", dt);
  return PA_OK;
}

int elem_size(int dt) { return dt == PA_DTYPE_F32 ? 4 : (dt == PA_DTYPE_I8 ? 1 : 2); }

// Checks shared by the token-granular cache writes, in the order they are reported. scales:
// whether k_scales / v_scales are required; cache_align: byte alignment of the kernel's cache
// stores (4 for one-byte caches, 8 for fp16).
int check_row_write(int in_dtype, const void* k, const void* v, int64_t token_stride,
                    const int32_t* slot_mapping, int num_tokens, int num_kv_heads, int head_dim,
                    const void* k_cache, const void* v_cache, bool scales, const float* k_scales,
                    const float* v_scales, int num_blocks, int block_size, size_t cache_align) {
  if (num_tokens < 0 || num_kv_heads <= 0 || num_blocks <= 0 || block_size <= 0)
    return fail(PA_ERR_INVALID_ARG, "invalid sizes");
  if (head_dim != 128) return fail(PA_ERR_UNSUPPORTED, "head_dim %d unsupported", head_dim);
  if (k == nullptr || v == nullptr || slot_mapping == nullptr || k_cache == nullptr ||
      v_cache == nullptr || (scales && (k_scales == nullptr || v_scales == nullptr)))
    return fail(PA_ERR_INVALID_ARG, "null pointer argument");
  if (token_stride < (int64_t)num_kv_heads * head_dim)
    return fail(PA_ERR_INVALID_ARG, "token_stride smaller than num_kv_heads*head_dim");
  const size_t es = (size_t)elem_size(in_dtype);
  if (!aligned(k, es * 4) || !aligned(v, es * 4) || token_stride % 4 != 0 ||
      !aligned(k_cache, cache_align) || !aligned(v_cache, cache_align))
    return fail(PA_ERR_INVALID_ARG, "misaligned input or cache pointer");
  return PA_OK;
}
// Cache kind of the decode kernels: 0 fp16, 1 int8, 2 fp8 e4m3 (-1: not a cache dtype).
int kv_kind(int kv_dtype) {
  return kv_dtype == PA_DTYPE_F16 ? 0
         : kv_dtype == PA_DTYPE_I8 ? 1
         : kv_dtype == PA_DTYPE_FP8E4M3 ? 2 : -1;
}

}  // namespace

namespace pa {
int fail_status(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vfail(code, fmt, ap);
  va_end(ap);
  return code;
}
}  // namespace pa

extern "C" {

int pa_version(void) { return 100; }

const char* pa_last_error(void) { return g_err.c_str(); }

const char* pa_status_string(int status) {
  if (status == PA_OK) return "ok";
  if (status & PA_ERR_INVALID_ARG) return "invalid argument";
  if (status & PA_ERR_UNSUPPORTED) return "unsupported shape or dtype";
  if (status & PA_ERR_CUDA) return "CUDA error";
  if (status & PA_ERR_WORKSPACE) return "workspace too small";
  if (status & PA_ERR_EMPTY_CONTEXT)
    return "context_lens must be >= 1 (empty sequences unsupported)";
  if (status & PA_ERR_CONTEXT_RANGE)
    return "context length exceeds max_blocks_per_seq * block_size";
  if (status & PA_ERR_BLOCK_ID) return "block_table entry outside [0, num_blocks)";
  if (status & PA_ERR_TIMEOUT) return "device wait timed out";
  if (status & PA_ERR_SLOT) return "slot_mapping entry outside the cache";
  if (status & PA_ERR_Q_RANGE) return "bf16 q value outside the fp16 range (saturated)";
  return "unknown status";
}

size_t pa_decode_workspace_bytes(int num_seqs, int num_heads, int num_kv_heads, int head_dim,
                                 int max_blocks_per_seq, int block_size, int kv_dtype,
                                 int splitk) {
  if (check_common(num_seqs, num_heads, num_kv_heads, head_dim, 1, block_size,
                   max_blocks_per_seq) != PA_OK)
    return 0;
  Shape s;
  const int kv_i8 = kv_kind(kv_dtype);
  if (kv_i8 < 0) return 0;
  const int mode = splitk ? pa::kModeSplit : pa::kModeStream;
  if (make_shape(kv_i8, mode, num_seqs, num_heads, num_kv_heads, head_dim, block_size,
                 max_blocks_per_seq, &s) != PA_OK)
    return 0;
  return ws_bytes_for(s, mode, num_seqs);
}

int pa_read_status(void* workspace, int* status_out, void* stream) {
  if (workspace == nullptr || status_out == nullptr)
    return fail(PA_ERR_INVALID_ARG, "null pointer argument");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int h = 0;
  cudaError_t e = cudaMemcpyAsync(&h, workspace, sizeof(int), cudaMemcpyDeviceToHost, st);
  if (e == cudaSuccess) e = cudaStreamSynchronize(st);
  if (e == cudaSuccess) e = cudaMemsetAsync(workspace, 0, sizeof(int), st);
  if (e != cudaSuccess) return cuda_fail(e, "status read");
  *status_out = h;
  return PA_OK;
}

int pa_reset_workspace(void* workspace, size_t workspace_bytes, void* stream) {
  if (workspace == nullptr || workspace_bytes < sizeof(int))
    return fail(PA_ERR_INVALID_ARG, "null or empty workspace");
  const size_t n = workspace_bytes < pa::kWsPartOffset ? workspace_bytes : pa::kWsPartOffset;
  cudaError_t e = cudaMemsetAsync(workspace, 0, n, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "workspace reset");
  return PA_OK;
}

int pa_decode_f16(void* out, const void* q, const void* k_cache, const void* v_cache,
                  const int32_t* block_table, const int32_t* context_lens, int num_seqs,
                  int num_heads, int num_kv_heads, int head_dim, int num_blocks, int block_size,
                  int max_blocks_per_seq, float scale, void* workspace, size_t workspace_bytes,
                  void* stream) {
  const NvtxRange nvtx_range("pa_decode_f16");
  return decode_impl(pa::kModeStream, 0, out, nullptr, q, k_cache, v_cache, nullptr, nullptr,
                     block_table, context_lens, num_seqs, num_heads, num_kv_heads, head_dim,
                     num_blocks, block_size, max_blocks_per_seq, scale, workspace,
                     workspace_bytes, stream);
}

int pa_decode_i8(void* out, const void* q, const void* k_cache, const void* v_cache,
                 const float* k_scales, const float* v_scales, const int32_t* block_table,
                 const int32_t* context_lens, int num_seqs, int num_heads, int num_kv_heads,
                 int head_dim, int num_blocks, int block_size, int max_blocks_per_seq,
                 float scale, void* workspace, size_t workspace_bytes, void* stream) {
  const NvtxRange nvtx_range("pa_decode_i8");
  return decode_impl(pa::kModeStream, 1, out, nullptr, q, k_cache, v_cache, k_scales, v_scales,
                     block_table, context_lens, num_seqs, num_heads, num_kv_heads, head_dim,
                     num_blocks, block_size, max_blocks_per_seq, scale, workspace,
                     workspace_bytes, stream);
}

int pa_splitk_f16(void* out, const void* q, const void* k_cache, const void* v_cache,
                  const int32_t* block_table, const int32_t* context_lens, int num_seqs,
                  int num_heads, int num_kv_heads, int head_dim, int num_blocks, int block_size,
                  int max_blocks_per_seq, float scale, void* workspace, size_t workspace_bytes,
                  void* stream) {
  const NvtxRange nvtx_range("pa_splitk_f16");
  return decode_impl(pa::kModeSplit, 0, out, nullptr, q, k_cache, v_cache, nullptr, nullptr,
                     block_table, context_lens, num_seqs, num_heads, num_kv_heads, head_dim,
                     num_blocks, block_size, max_blocks_per_seq, scale, workspace,
                     workspace_bytes, stream);
}

int pa_splitk_i8(void* out, const void* q, const void* k_cache, const void* v_cache,
                 const float* k_scales, const float* v_scales, const int32_t* block_table,
                 const int32_t* context_lens, int num_seqs, int num_heads, int num_kv_heads,
                 int head_dim, int num_blocks, int block_size, int max_blocks_per_seq,
                 float scale, void* workspace, size_t workspace_bytes, void* stream) {
  const NvtxRange nvtx_range("pa_splitk_i8");
  return decode_impl(pa::kModeSplit, 1, out, nullptr, q, k_cache, v_cache, k_scales, v_scales,
                     block_table, context_lens, num_seqs, num_heads, num_kv_heads, head_dim,
                     num_blocks, block_size, max_blocks_per_seq, scale, workspace,
                     workspace_bytes, stream);
}

// BF16 activations: q (bf16) -> fp16 copy in the workspace, the fp16-q decode into an fp16
// output in the workspace, then -> bf16 out. Layout: [decode workspace | q fp16 | out fp16],
// each part 256-byte aligned.
static size_t round256(size_t x) { return (x + 255) & ~(size_t)255; }

size_t pa_decode_bf16q_workspace_bytes(int num_seqs, int num_heads, int num_kv_heads,
                                       int head_dim, int max_blocks_per_seq, int block_size,
                                       int kv_dtype, int splitk) {
  const size_t base = pa_decode_workspace_bytes(num_seqs, num_heads, num_kv_heads, head_dim,
                                                max_blocks_per_seq, block_size, kv_dtype, splitk);
  if (base == 0 || num_seqs < 0) return 0;
  const size_t act = round256((size_t)num_seqs * num_heads * head_dim * 2);
  return round256(base) + 2 * act;
}

int pa_decode_bf16q(void* out, const void* q, const void* k_cache, const void* v_cache,
                    const float* k_scales, const float* v_scales, const int32_t* block_table,
                    const int32_t* context_lens, int num_seqs, int num_heads, int num_kv_heads,
                    int head_dim, int num_blocks, int block_size, int max_blocks_per_seq,
                    int kv_dtype, int splitk, float scale, void* workspace,
                    size_t workspace_bytes, void* stream) {
  const NvtxRange nvtx_range("pa_decode_bf16q");
  if (kv_kind(kv_dtype) < 0)
    return fail(PA_ERR_UNSUPPORTED,
                "kv_dtype must be PA_DTYPE_F16, PA_DTYPE_I8 or PA_DTYPE_FP8E4M3");
  int rc = check_common(num_seqs, num_heads, num_kv_heads, head_dim, num_blocks, block_size,
                        max_blocks_per_seq);
  if (rc != PA_OK) return rc;
  if (num_seqs == 0) return PA_OK;
  if (out == nullptr || q == nullptr || workspace == nullptr)
    return fail(PA_ERR_INVALID_ARG, "null pointer argument");
  if (!aligned(out, 16) || !aligned(q, 16) || !aligned(workspace, 256))
    return fail(PA_ERR_INVALID_ARG, "tensors must be 16-byte aligned (workspace 256-byte)");
  const size_t need = pa_decode_bf16q_workspace_bytes(num_seqs, num_heads, num_kv_heads,
                                                      head_dim, max_blocks_per_seq, block_size,
                                                      kv_dtype, splitk);
  if (need == 0) return fail(PA_ERR_UNSUPPORTED, "unsupported decode shape");
  if (workspace_bytes < need)
    return fail(PA_ERR_WORKSPACE, "workspace too small: %zu < %zu bytes", workspace_bytes, need);
  const size_t base = round256(pa_decode_workspace_bytes(num_seqs, num_heads, num_kv_heads,
                                                         head_dim, max_blocks_per_seq,
                                                         block_size, kv_dtype, splitk));
  const long long n = (long long)num_seqs * num_heads * head_dim;
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  void* q16 = ws + base;
  void* o16 = ws + base + round256((size_t)n * 2);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int sms = num_sms_current(nullptr);
  if (sms <= 0) return fail(PA_ERR_CUDA, "cannot query the current device");
  cudaError_t e = pa::launch_bf16_to_f16(q, q16, n, reinterpret_cast<int*>(ws), sms, st);
  if (e != cudaSuccess) return cuda_fail(e, "q conversion launch");
  const int mode = splitk ? pa::kModeSplit : pa::kModeStream;
  rc = decode_impl(mode, kv_kind(kv_dtype), o16, nullptr, q16, k_cache, v_cache, k_scales, v_scales,
                   block_table, context_lens, num_seqs, num_heads, num_kv_heads, head_dim,
                   num_blocks, block_size, max_blocks_per_seq, scale, workspace, base, stream);
  if (rc != PA_OK) return rc;
  e = pa::launch_f16_to_bf16(o16, out, n, sms, st);
  if (e != cudaSuccess) return cuda_fail(e, "output conversion launch");
  return PA_OK;
}

int pa_selftest_bounded_wait(void* workspace, void* stream) {
  if (workspace == nullptr || !aligned(workspace, 4))
    return fail(PA_ERR_INVALID_ARG, "workspace must be a non-null, 4-byte aligned pointer");
  cudaError_t e = pa::launch_selftest_wait(static_cast<int*>(workspace),
                                           static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "self-test launch");
  return PA_OK;
}

int pa_decode_fp8(void* out, const void* q, const void* k_cache, const void* v_cache,
                  const float* k_scales, const float* v_scales, const int32_t* block_table,
                  const int32_t* context_lens, int num_seqs, int num_heads, int num_kv_heads,
                  int head_dim, int num_blocks, int block_size, int max_blocks_per_seq,
                  float scale, void* workspace, size_t workspace_bytes, void* stream) {
  const NvtxRange nvtx_range("pa_decode_fp8");
  return decode_impl(pa::kModeStream, 2, out, nullptr, q, k_cache, v_cache, k_scales, v_scales,
                     block_table, context_lens, num_seqs, num_heads, num_kv_heads, head_dim,
                     num_blocks, block_size, max_blocks_per_seq, scale, workspace,
                     workspace_bytes, stream);
}

int pa_splitk_fp8(void* out, const void* q, const void* k_cache, const void* v_cache,
                  const float* k_scales, const float* v_scales, const int32_t* block_table,
                  const int32_t* context_lens, int num_seqs, int num_heads, int num_kv_heads,
                  int head_dim, int num_blocks, int block_size, int max_blocks_per_seq,
                  float scale, void* workspace, size_t workspace_bytes, void* stream) {
  const NvtxRange nvtx_range("pa_splitk_fp8");
  return decode_impl(pa::kModeSplit, 2, out, nullptr, q, k_cache, v_cache, k_scales, v_scales,
                     block_table, context_lens, num_seqs, num_heads, num_kv_heads, head_dim,
                     num_blocks, block_size, max_blocks_per_seq, scale, workspace,
                     workspace_bytes, stream);
}

int pa_decode_step(int kv_dtype, void* out, const void* q, const void* new_k,
                   const void* new_v, int new_dtype, int64_t new_token_stride, void* k_cache,
                   void* v_cache, float* k_scales, float* v_scales, const float* k_fixed_scale,
                   const float* v_fixed_scale, const int32_t* block_table,
                   const int32_t* context_lens, int num_seqs, int num_heads, int num_kv_heads,
                   int head_dim, int num_blocks, int block_size, int max_blocks_per_seq,
                   float scale, int splitk, int fused, void* workspace, size_t workspace_bytes,
                   void* stream) {
  const NvtxRange nvtx_range("pa_decode_step");
  const int kind = kv_kind(kv_dtype);
  if (kind < 0)
    return fail(PA_ERR_UNSUPPORTED,
                "kv_dtype must be PA_DTYPE_F16, PA_DTYPE_I8 or PA_DTYPE_FP8E4M3");
  int rc = check_in_dtype(new_dtype);
  if (rc != PA_OK) return rc;
  if (num_seqs == 0) return PA_OK;
  if (new_k == nullptr || new_v == nullptr)
    return fail(PA_ERR_INVALID_ARG, "null new-token pointer");
  if (num_kv_heads <= 0 || new_token_stride < (int64_t)num_kv_heads * head_dim)
    return fail(PA_ERR_INVALID_ARG, "new_token_stride smaller than num_kv_heads*head_dim");
  const size_t es = (size_t)elem_size(new_dtype);
  if (!aligned(new_k, es * 4) || !aligned(new_v, es * 4) || new_token_stride % 4 != 0)
    return fail(PA_ERR_INVALID_ARG, "misaligned new-token rows");
  if ((k_fixed_scale != nullptr || v_fixed_scale != nullptr) &&
      (kind != 1 || k_fixed_scale == nullptr || v_fixed_scale == nullptr))
    return fail(PA_ERR_INVALID_ARG, "fixed scales need an int8 cache and both of k and v");
  StepWrite sw{new_k, new_v, new_dtype, (long long)new_token_stride, k_fixed_scale,
               v_fixed_scale, fused != 0};
  return decode_impl(splitk ? pa::kModeSplit : pa::kModeStream, kind, out, nullptr, q, k_cache,
                     v_cache, k_scales, v_scales, block_table, context_lens, num_seqs,
                     num_heads, num_kv_heads, head_dim, num_blocks, block_size,
                     max_blocks_per_seq, scale, workspace, workspace_bytes, stream, &sw);
}

int pa_partial_floats(int num_heads, int num_kv_heads, int head_dim) {
  if (num_kv_heads <= 0 || num_heads % num_kv_heads != 0) return 0;
  const int G = num_heads / num_kv_heads;
  const int GT = G <= 8 ? 8 : 16;
  return pa::slot_floats(head_dim, GT) * ((G + GT - 1) / GT);
}

int pa_decode_partial(int kv_dtype, float* partials, const void* q, const void* k_cache,
                      const void* v_cache, const float* k_scales, const float* v_scales,
                      const int32_t* block_table, const int32_t* context_lens, int num_seqs,
                      int num_heads, int num_kv_heads, int head_dim, int num_blocks,
                      int block_size, int max_blocks_per_seq, float scale, void* workspace,
                      size_t workspace_bytes, void* stream) {
  const NvtxRange nvtx_range("pa_decode_partial");
  if (kv_kind(kv_dtype) < 0)
    return fail(PA_ERR_UNSUPPORTED, "kv dtype must be fp16, int8 or fp8 e4m3");
  return decode_impl(pa::kModePartial, kv_kind(kv_dtype), nullptr, partials, q,
                     k_cache, v_cache, k_scales, v_scales, block_table, context_lens, num_seqs,
                     num_heads, num_kv_heads, head_dim, num_blocks, block_size,
                     max_blocks_per_seq, scale, workspace, workspace_bytes, stream);
}

int pa_merge_partials(void* out, const float* partials, int num_parts, int num_seqs,
                      int num_heads, int num_kv_heads, int head_dim, int* status,
                      void* stream) {
  const NvtxRange nvtx_range("pa_merge_partials");
  if (num_seqs == 0) return PA_OK;
  if (out == nullptr || partials == nullptr || num_parts <= 0 || num_seqs < 0 ||
      num_kv_heads <= 0 || num_heads % num_kv_heads != 0)
    return fail(PA_ERR_INVALID_ARG, "invalid merge arguments");
  if (head_dim != 128) return fail(PA_ERR_UNSUPPORTED, "head_dim %d unsupported", head_dim);
  if (!aligned(out, 16) || !aligned(partials, 16))
    return fail(PA_ERR_INVALID_ARG, "tensors must be 16-byte aligned");
  const int G = num_heads / num_kv_heads;
  const int GT = G <= 8 ? 8 : 16;
  const int HT = (G + GT - 1) / GT;
  const int SLOT = pa::slot_floats(head_dim, GT);
  pa::ReduceArgs ra;
  memset(&ra, 0, sizeof(ra));
  ra.out = static_cast<__half*>(out);
  ra.part = partials;
  ra.status = status;
  ra.B = num_seqs;
  ra.H = num_heads;
  ra.KVH = num_kv_heads;
  ra.G = G;
  ra.HT = HT;
  ra.num_parts = num_parts;
  ra.piece_stride = (long long)num_seqs * num_kv_heads * HT * SLOT;
  ra.seg_stride = SLOT;
  cudaError_t e = pa::launch_reduce(GT, ra, num_parts, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "merge launch");
  return PA_OK;
}

int pa_quantize_into_cache(const void* k, const void* v, int in_dtype, int64_t token_stride,
                           const int32_t* slot_mapping, int num_tokens, int num_kv_heads,
                           int head_dim, void* k_cache, void* v_cache, float* k_scales,
                           float* v_scales, int num_blocks, int block_size,
                           const float* k_fixed_scale, const float* v_fixed_scale, int* status,
                           void* stream) {
  const NvtxRange nvtx_range("pa_quantize_into_cache");
  int rc = check_in_dtype(in_dtype);
  if (rc != PA_OK) return rc;
  if (num_tokens == 0) return PA_OK;
  rc = check_row_write(in_dtype, k, v, token_stride, slot_mapping, num_tokens, num_kv_heads,
                       head_dim, k_cache, v_cache, true, k_scales, v_scales, num_blocks,
                       block_size, 4);
  if (rc != PA_OK) return rc;
  cudaError_t e = pa::launch_write_rows(in_dtype, pa::kRowsI8, head_dim, k, v, token_stride,
                                        slot_mapping, num_tokens, num_kv_heads, k_cache, v_cache,
                                        k_scales, v_scales, num_blocks, block_size,
                                        k_fixed_scale, v_fixed_scale, status,
                                        static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "quantize launch");
  return PA_OK;
}

int pa_quantize_into_cache_fp8(const void* k, const void* v, int in_dtype, int64_t token_stride,
                               const int32_t* slot_mapping, int num_tokens, int num_kv_heads,
                               int head_dim, void* k_cache, void* v_cache, float* k_scales,
                               float* v_scales, int num_blocks, int block_size, int* status,
                               void* stream) {
  const NvtxRange nvtx_range("pa_quantize_into_cache_fp8");
  int rc = check_in_dtype(in_dtype);
  if (rc != PA_OK) return rc;
  if (num_tokens == 0) return PA_OK;
  rc = check_row_write(in_dtype, k, v, token_stride, slot_mapping, num_tokens, num_kv_heads,
                       head_dim, k_cache, v_cache, true, k_scales, v_scales, num_blocks,
                       block_size, 4);
  if (rc != PA_OK) return rc;
  cudaError_t e = pa::launch_write_rows(in_dtype, pa::kRowsFP8, head_dim, k, v, token_stride,
                                        slot_mapping, num_tokens, num_kv_heads, k_cache, v_cache,
                                        k_scales, v_scales, num_blocks, block_size, nullptr,
                                        nullptr, status, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "fp8 quantize launch");
  return PA_OK;
}

int pa_write_into_cache_f16(const void* k, const void* v, int in_dtype, int64_t token_stride,
                            const int32_t* slot_mapping, int num_tokens, int num_kv_heads,
                            int head_dim, void* k_cache, void* v_cache, int num_blocks,
                            int block_size, int* status, void* stream) {
  const NvtxRange nvtx_range("pa_write_into_cache_f16");
  int rc = check_in_dtype(in_dtype);
  if (rc != PA_OK) return rc;
  if (num_tokens == 0) return PA_OK;
  rc = check_row_write(in_dtype, k, v, token_stride, slot_mapping, num_tokens, num_kv_heads,
                       head_dim, k_cache, v_cache, false, nullptr, nullptr, num_blocks,
                       block_size, 8);
  if (rc != PA_OK) return rc;
  cudaError_t e = pa::launch_write_rows(in_dtype, pa::kRowsF16, head_dim, k, v, token_stride,
                                        slot_mapping, num_tokens, num_kv_heads, k_cache, v_cache,
                                        nullptr, nullptr, num_blocks, block_size, nullptr,
                                        nullptr, status, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "cache write launch");
  return PA_OK;
}

int pa_prefill_into_cache(const void* k, const void* v, int in_dtype, int num_seqs,
                          int max_len, int num_kv_heads, int head_dim,
                          const int32_t* block_table, const int32_t* context_lens,
                          int max_blocks_per_seq, int cache_dtype, void* k_cache, void* v_cache,
                          float* k_scales, float* v_scales, int num_blocks, int block_size,
                          const float* k_fixed_scale, const float* v_fixed_scale, int* status,
                          void* stream) {
  const NvtxRange nvtx_range("pa_prefill_into_cache");
  int rc = check_in_dtype(in_dtype);
  if (rc != PA_OK) return rc;
  if (cache_dtype != PA_DTYPE_I8 && cache_dtype != PA_DTYPE_F16)
    return fail(PA_ERR_UNSUPPORTED, "cache dtype must be int8 or fp16");
  if (num_seqs == 0) return PA_OK;
  if (num_seqs < 0 || max_len < 0 || num_kv_heads <= 0 || num_blocks <= 0 ||
      max_blocks_per_seq <= 0)
    return fail(PA_ERR_INVALID_ARG, "invalid sizes");
  if (num_kv_heads > 65535 || num_seqs > 65535)
    return fail(PA_ERR_UNSUPPORTED, "num_seqs and num_kv_heads must be <= 65535");
  if (head_dim != 128) return fail(PA_ERR_UNSUPPORTED, "head_dim %d unsupported", head_dim);
  if (block_size % 16 != 0 || block_size > 128)
    return fail(PA_ERR_INVALID_ARG, "block_size must be a multiple of 16 up to 128");
  const bool i8 = cache_dtype == PA_DTYPE_I8;
  if (k == nullptr || v == nullptr || block_table == nullptr || context_lens == nullptr ||
      k_cache == nullptr || v_cache == nullptr ||
      (i8 && (k_scales == nullptr || v_scales == nullptr)))
    return fail(PA_ERR_INVALID_ARG, "null pointer argument");
  const size_t es = (size_t)elem_size(in_dtype);
  if (!aligned(k, es * 4) || !aligned(v, es * 4) || !aligned(k_cache, 16) || !aligned(v_cache, 16))
    return fail(PA_ERR_INVALID_ARG, "misaligned input or cache pointer");
  cudaError_t e = pa::launch_prefill(in_dtype, i8, k, v, num_seqs, max_len, num_kv_heads,
                                     block_table, context_lens, max_blocks_per_seq, k_cache,
                                     v_cache, k_scales, v_scales, num_blocks, block_size,
                                     k_fixed_scale, v_fixed_scale, status,
                                     static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "prefill launch");
  return PA_OK;
}

int pa_absmax_scale(const void* x, int in_dtype, int64_t n, float* scale_out, int semantics,
                    void* scratch, void* stream) {
  const NvtxRange nvtx_range("pa_absmax_scale");
  int rc = check_in_dtype(in_dtype);
  if (rc != PA_OK) return rc;
  if (scale_out == nullptr || scratch == nullptr || (n > 0 && x == nullptr) || n < 0)
    return fail(PA_ERR_INVALID_ARG, "invalid absmax arguments");
  if (semantics != PA_SCALE_CLAMP_THEN_DIVIDE && semantics != PA_SCALE_DIVIDE_THEN_CLAMP)
    return fail(PA_ERR_INVALID_ARG, "unknown scale semantics %d", semantics);
  const int sms = num_sms_current(nullptr);
  if (sms <= 0) return fail(PA_ERR_CUDA, "cannot query the current device");
  cudaError_t e = pa::launch_absmax_scale(in_dtype, x, n, scale_out, semantics,
                                          static_cast<unsigned int*>(scratch), sms,
                                          static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "absmax launch");
  return PA_OK;
}

}  // extern "C"
