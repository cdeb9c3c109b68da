// mb_adamw_step_noalloc: the fused AdamW step without any device allocation.
//
// Who needs it. mb_adamw_step takes a caller-allocated workspace (per-CTA FP64
// partial sums, a ticket counter, per-segment step scalars). Some callers cannot
// allocate device memory: a host framework whose pool allocator has already
// reserved the whole GPU (a second cudaMalloc would fail), a plugin or
// foreign-language binding that is handed fixed device buffers and has no
// allocator of its own, or code running where allocation is forbidden. This
// entry point runs the same kernels with that workspace replaced by one fixed
// array inside the library's device image.
//
// The array. g_noalloc_scratch is a file-scope __device__ array of
// kNoallocBytes (= 64 KiB of partials + 256 B ticket + 64 KiB of scalars for at
// most kNoallocMaxSegments = 8192 segments, about 129 KiB). Every GPU on which
// this library's device code is loaded holds it until the process exits. Plans
// with more segments are rejected with MB_ERR_TOO_LARGE before anything runs.
//
// Host code may not use the array's name as a device address (on the host it
// names a stand-in object). The first call on each device, with that device
// current, looks the address up with cudaGetSymbolAddress and caches it for the
// current CUDA context; make that first call before any stream capture on that
// device. A new context on the device (after cudaDeviceReset, say) reloads the
// library's device image, so the next call looks the address up again.
//
// Sharing. All calls on a device share the one array and it keeps the last
// call's contents. Each call clears the ticket counter on its stream before
// kernel 2 (the partials and scalars are fully rewritten by every call). Calls
// that can overlap on the GPU (different streams without ordering between them)
// race on the array and give wrong results: issue them in order.
#include <cuda.h>

#include <mutex>

#include "mb_common.cuh"

namespace {

constexpr int kNoallocMaxSegments = 8192;
constexpr size_t kNoallocBytes = mb::kSegScalOffset + sizeof(float2) * kNoallocMaxSegments;
constexpr int kMaxDevices = 64;

__device__ __align__(256) unsigned char g_noalloc_scratch[kNoallocBytes];

struct ScratchEntry {
  unsigned long long ctx_id;  // unique id of the context the address was looked up in
  void* addr;
};

std::mutex g_mu;
ScratchEntry g_scratch[kMaxDevices] = {};

using CtxGetCurrentFn = CUresult (*)(CUcontext*);
using CtxGetIdFn = CUresult (*)(CUcontext, unsigned long long*);

template <class Fn>
Fn driver_fn(const char* name) {
  void* p = nullptr;
  cudaDriverEntryPointQueryResult q;
  if (cudaGetDriverEntryPoint(name, &p, cudaEnableDefault, &q) != cudaSuccess || q != cudaDriverEntryPointSuccess)
    return nullptr;
  return reinterpret_cast<Fn>(p);
}

// Process-unique id of the calling thread's current context (through the
// runtime's driver entry points, so the library needs no link against
// libcuda). Ids are never reused, unlike context handles.
int current_context_id(unsigned long long* out) {
  static CtxGetCurrentFn get_current = driver_fn<CtxGetCurrentFn>("cuCtxGetCurrent");
  static CtxGetIdFn get_id = driver_fn<CtxGetIdFn>("cuCtxGetId");
  CUcontext ctx = nullptr;
  if (!get_current || !get_id || get_current(&ctx) != CUDA_SUCCESS || ctx == nullptr) return MB_ERR_CUDA;
  return get_id(ctx, out) == CUDA_SUCCESS ? MB_OK : MB_ERR_CUDA;
}

// Device address of g_noalloc_scratch on the current device and context
// (looked up once per context).
int scratch_address(void** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return MB_ERR_CUDA;
  unsigned long long ctx = 0;
  if (current_context_id(&ctx) != MB_OK) {
    // no context yet: the runtime's first call creates the device's primary one
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess || p == nullptr) return MB_ERR_CUDA;
    int rc = current_context_id(&ctx);
    if (rc) return rc;
  }
  std::lock_guard<std::mutex> lock(g_mu);
  ScratchEntry& e = g_scratch[dev];
  if (e.addr == nullptr || e.ctx_id != ctx) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess || p == nullptr) return MB_ERR_CUDA;
    e.ctx_id = ctx;
    e.addr = p;
  }
  *out = e.addr;
  return MB_OK;
}

}  // namespace

extern "C" MB_API int mb_adamw_step_noalloc(const mb_adamw_plan* plan, const mb_finalize_opts* fin,
                                            mb_stream_t stream) {
  if (!plan || !fin) return MB_ERR_ARG;
  if (plan->n_segs > kNoallocMaxSegments) return MB_ERR_TOO_LARGE;
  void* scratch = nullptr;
  int rc = scratch_address(&scratch);
  if (rc) return rc;
  mb_adamw_plan p = *plan;
  p.workspace = scratch;
  // validate everything before queueing any work on the stream
  if ((rc = mb::check_plan(&p)) || (rc = mb::check_fin(fin))) return rc;
  // Kernel 2 resets the ticket at the end of every launch; this clear only
  // matters after a launch that never finished (an aborted context or stream).
  if (cudaMemsetAsync(static_cast<char*>(scratch) + mb::kTicketOffset, 0, 16, (cudaStream_t)stream) != cudaSuccess)
    return MB_ERR_CUDA;
  return mb_adamw_step(&p, fin, stream);
}
