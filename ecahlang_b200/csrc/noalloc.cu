// ecah_sampler_launch_noalloc: the sampler for callers that cannot allocate
// device memory.
//
// Some hosts of this library have no device allocator they may call at
// sampling time: an inference runtime that owns every byte of device memory
// through its own pool and forbids cudaMalloc after start-up, a C or FFI
// caller linking the library without a CUDA memory manager of its own, or a
// decode loop that must not allocate between steps.  ecah_sampler_launch needs
// a caller-provided workspace; this entry point instead uses a fixed scratch
// array in the library's own device memory, so the caller passes only its
// inputs and outputs.
//
// The scratch is a file-scope __device__ array of kNoAllocScratchBytes; every
// GPU that loads the library holds it until the process exits.  Its device
// address is looked up on every call, with the calling device current
// (cudaGetSymbolAddress, which allocates nothing), so it stays right after a
// cudaDeviceReset; the first call on a device may load the module, so make it
// outside any stream capture.  Every call shares the array: it is cleared on
// the caller's stream before each launch, and calls whose work overlaps on
// the GPU (two streams at once) race on it.  The scratch holds what the
// cluster kernel needs, so every launch through this entry point runs the
// cluster kernel.

#include <cuda_runtime.h>

#include "../../include/ecah_sampler.h"

// sampler.cu: the least workspace ecah_sampler_launch accepts (not exported)
extern "C" size_t ecah_internal_min_workspace_bytes(void);

namespace {

constexpr size_t kNoAllocScratchBytes = 256;
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

// Device address of the scratch array on the current device (host code sees
// only a host-side stand-in for the symbol, never usable as a device pointer).
void* scratch_for_current_device() {
  void* p = nullptr;
  if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess) {
    cudaGetLastError();
    return nullptr;
  }
  return p;
}

}  // namespace

extern "C" {

size_t ecah_sampler_noalloc_scratch_bytes(void) { return kNoAllocScratchBytes; }

int ecah_sampler_launch_noalloc(const ecah_sampler_args* a, void* stream) {
  if (!a) return ECAH_ERR_NULL;
  if (a->abi_version != ECAH_SAMPLER_ABI_VERSION) return ECAH_ERR_ABI;
  if (a->dtype < ECAH_DTYPE_F16 || a->dtype > ECAH_DTYPE_F32) return ECAH_ERR_DTYPE;
  if (a->batch < 0 || a->vocab < 1) return ECAH_ERR_SHAPE;
  if (ecah_internal_min_workspace_bytes() > kNoAllocScratchBytes)
    return ECAH_ERR_WORKSPACE;  // the launch needs more scratch than the library holds
  if (a->batch == 0) return ECAH_OK;
  void* scratch = scratch_for_current_device();
  if (!scratch) return ECAH_ERR_LAUNCH;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (cudaMemsetAsync(scratch, 0, kNoAllocScratchBytes, s) != cudaSuccess) return ECAH_ERR_LAUNCH;
  ecah_sampler_args b = *a;
  b.workspace = scratch;
  b.workspace_bytes = kNoAllocScratchBytes;
  return ecah_sampler_launch(&b, stream);
}

}  // extern "C"
