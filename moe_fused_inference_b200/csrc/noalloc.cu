// noalloc.cu — mfi_mxfp4_linear_noalloc: the mxfp4_linear operation for
// callers that cannot allocate device memory.
//
// Who needs it: code that drives the GPU but owns no device allocator — a
// plugin loaded by a host program that has handed all GPU memory to its own
// pool, an FFI caller (JNI, ctypes, cgo) with no access to the framework's
// caching allocator, or a caller that must not call cudaMalloc on its hot path
// because the allocation would synchronise the device.  mfi_mxfp4_linear asks
// such callers for a workspace they cannot provide; this entry point instead
// carves the same scratch (quantised activations and re-laid-out scale
// factors) out of one file-scope device array that the library owns.
//
// Properties of that array, which callers must respect:
//  * size kNoAllocScratchBytes (4 MiB) on every GPU that loads the library,
//    held until the process exits;
//  * its device address is looked up once per device (cudaGetSymbolAddress,
//    with that device current) by the first call made on that device, so the
//    first call on each device should happen before any stream capture;
//  * every call on a device uses the same array and leaves its contents
//    behind; nothing in it has to start at zero because each call writes
//    every byte it later reads;
//  * calls that overlap on the GPU (different streams, or host threads
//    launching concurrently on one device) race on the array — serialise them;
//  * the looked-up address is kept for the life of the process: after
//    cudaDeviceReset() on a device the array lives at a new address, so the
//    entry point must not be called on that device again.  (Host threads may
//    make first calls concurrently: the cache is atomic, and two threads that
//    both look the address up store the same value.)
#include <cuda_runtime.h>

#include <atomic>

#include "../../include/moe_fp4.h"
#include "work.cuh"

namespace {

constexpr size_t kNoAllocScratchBytes = size_t(4) << 20;  // 4 MiB per device

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

// Device address of g_noalloc_scratch for the current device.  In host code
// the symbol names a host-side stand-in, never a device address, so kernels
// must be given this address, not the symbol.
void* scratch_address(int* status) {
  static std::atomic<void*> addr[64];  // zero-initialised (static storage)
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) {
    *status = MFI_ERR_CUDA;
    return nullptr;
  }
  void* p = addr[dev].load(std::memory_order_acquire);
  if (!p) {
    const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || p == nullptr) {
      *status = MFI_ERR_CUDA;
      return nullptr;
    }
    addr[dev].store(p, std::memory_order_release);
  }
  *status = MFI_OK;
  return p;
}

}  // namespace

extern "C" int mfi_mxfp4_linear_noalloc(const void* x, int dtype, int ld_x, const uint8_t* wp,
                                        const uint8_t* wsc, float* y, int M, int N, int Kp,
                                        void* stream) {
  if (M < 0 || N < 0 || Kp <= 0 || Kp % 32 != 0)
    return mfi::set_last_error(MFI_ERR_ARG, "M, N must be >= 0 and Kp a positive multiple of 32");
  if (M == 0 || N == 0) return MFI_OK;
  const size_t need = mfi_linear_workspace_bytes(M, N, Kp);
  if (need > kNoAllocScratchBytes)
    return mfi::set_last_error(
        MFI_ERR_WORKSPACE,
        "mxfp4_linear_noalloc: this shape needs more scratch than the library's 4 MiB static "
        "array; call mfi_mxfp4_linear with a workspace of mfi_linear_workspace_bytes(M, N, Kp)");
  int st = MFI_OK;
  void* ws = scratch_address(&st);
  if (st != MFI_OK)
    return mfi::set_last_error(st, "mxfp4_linear_noalloc: cudaGetSymbolAddress of the static "
                                   "scratch failed on the current device");
  return mfi_mxfp4_linear(x, dtype, ld_x, wp, wsc, y, M, N, Kp, ws, kNoAllocScratchBytes, stream);
}
