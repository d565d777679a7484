// pa_decode_f16_noalloc: the FP16 single-pass decode without a caller-provided workspace.
//
// Some callers cannot allocate device memory at the moment they run attention: plugins
// whose host framework owns every device allocation and hands out only tensor pointers
// (the plugin has no allocator of its own to call), and latency-critical serving loops that
// must never enter an allocator (it can synchronise the device or fail when memory is
// fragmented, mid-step). This entry point serves them: its scratch (status word, arrival
// counters, partial slots) lives in one statically sized device array that belongs to this
// file.
//
// The array holds kNoAllocScratchBytes (12 MiB) on every GPU whose context loads this code,
// until the process exits. Every call on a device shares it and it keeps the last call's
// contents, so calls that overlap on the GPU (two streams, or two threads) race with each
// other; order them on one stream. Each call clears the whole arrival-counter region before
// launching, because the counters must start at zero (a call that stopped early on a device
// error can leave some set). The status word is not cleared: the kernels OR error bits into
// it, and they stay there until pa_decode_f16_noalloc_read_status reads and clears them.
//
// The first call on a device (and the first after that device's context was destroyed and
// created again) looks up the array's device address with cudaGetSymbolAddress, with that
// device current; make that first call before any stream capture. Later calls only launch
// asynchronous work (one memset and the decode kernel) and allocate nothing.

#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdio>
#include <mutex>

#include "pa_internal.h"

namespace {

constexpr size_t kNoAllocScratchBytes = 12u << 20;

// The scratch itself. In host code this name is only a stand-in for the symbol: its device
// address comes from cudaGetSymbolAddress below and is what the kernel receives.
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

// Per device: the context the address was looked up in, and the address.
struct ScratchSlot {
  CUcontext ctx;
  void* ptr;
};
std::mutex g_mu;
ScratchSlot g_slots[64] = {};

using CtxGetCurrentFn = CUresult (*)(CUcontext*);

CtxGetCurrentFn ctx_get_current() {
  static CtxGetCurrentFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<CtxGetCurrentFn>(p);
  });
  return fn;
}

// Device address of the scratch on the current device. It is looked up once per device and
// again whenever the device's current context differs from the one it was looked up in
// (after cudaDeviceReset, say), so a stale address is never handed to a kernel.
cudaError_t scratch_for_current_device(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  auto get = ctx_get_current();
  if (get == nullptr) return cudaErrorDeviceUninitialized;
  CUcontext ctx = nullptr;
  if (get(&ctx) != CUDA_SUCCESS) return cudaErrorDeviceUninitialized;
  std::lock_guard<std::mutex> lock(g_mu);
  ScratchSlot& slot = g_slots[dev];
  if (ctx == nullptr || slot.ptr == nullptr || slot.ctx != ctx) {
    // The lookup also makes the device's primary context current when no runtime call has
    // done so yet, so the context is read again after it.
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess) return e;
    if (get(&ctx) != CUDA_SUCCESS || ctx == nullptr) return cudaErrorDeviceUninitialized;
    slot.ctx = ctx;
    slot.ptr = p;
  }
  *out = slot.ptr;
  return cudaSuccess;
}

}  // namespace

extern "C" int pa_decode_f16_noalloc(void* out, const void* q, const void* k_cache,
                                     const void* v_cache, const int32_t* block_table,
                                     const int32_t* context_lens, int num_seqs, int num_heads,
                                     int num_kv_heads, int head_dim, int num_blocks,
                                     int block_size, int max_blocks_per_seq, float scale,
                                     void* stream) {
  const size_t need = pa_decode_workspace_bytes(num_seqs, num_heads, num_kv_heads, head_dim,
                                                max_blocks_per_seq, block_size, PA_DTYPE_F16, 0);
  if (need == 0) {
    // Unsupported shape or no device: let the regular entry point report the reason.
    return pa_decode_f16(out, q, k_cache, v_cache, block_table, context_lens, num_seqs,
                         num_heads, num_kv_heads, head_dim, num_blocks, block_size,
                         max_blocks_per_seq, scale, nullptr, 0, stream);
  }
  if (need > kNoAllocScratchBytes) {
    return pa::fail_status(PA_ERR_WORKSPACE,
                           "pa_decode_f16_noalloc: this shape needs %zu bytes of scratch but the "
                           "static scratch holds %zu (shapes with more than 8 q heads per kv "
                           "head exceed it)",
                           need, kNoAllocScratchBytes);
  }
  void* ws = nullptr;
  cudaError_t e = scratch_for_current_device(&ws);
  if (e != cudaSuccess)
    return pa::fail_status(PA_ERR_CUDA, "pa_decode_f16_noalloc: scratch lookup failed: %s",
                           cudaGetErrorString(e));
  // The arrival counters must start at zero. The whole fixed counter region is cleared, so
  // counters left set by any earlier call, of any shape, are covered; the status word in
  // front of it is kept until it is read.
  e = cudaMemsetAsync(static_cast<unsigned char*>(ws) + pa::kWsHeader, 0,
                      pa::kWsPartOffset - pa::kWsHeader, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess)
    return pa::fail_status(PA_ERR_CUDA, "pa_decode_f16_noalloc: clearing scratch failed: %s",
                           cudaGetErrorString(e));
  return pa_decode_f16(out, q, k_cache, v_cache, block_table, context_lens, num_seqs,
                       num_heads, num_kv_heads, head_dim, num_blocks, block_size,
                       max_blocks_per_seq, scale, ws, kNoAllocScratchBytes, stream);
}

extern "C" int pa_decode_f16_noalloc_read_status(int* status_out, void* stream) {
  if (status_out == nullptr)
    return pa::fail_status(PA_ERR_INVALID_ARG, "pa_decode_f16_noalloc_read_status: null output");
  void* ws = nullptr;
  cudaError_t e = scratch_for_current_device(&ws);
  if (e != cudaSuccess)
    return pa::fail_status(PA_ERR_CUDA,
                           "pa_decode_f16_noalloc_read_status: scratch lookup failed: %s",
                           cudaGetErrorString(e));
  return pa_read_status(ws, status_out, stream);
}
