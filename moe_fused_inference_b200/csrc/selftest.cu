// selftest.cu — exhaustive device self-check of the library's own float
// arithmetic against CUDA's.
//
// Two functions of one fp32 value are computed by the library in its own way
// for speed, and each must equal a reference definition bit for bit:
//   * the SwiGLU quotient g / (1 + expf(-g)) (swiglu_quotient, Markstein's
//     division) against CUDA's correctly rounded __fdiv_rn of the same
//     operands, the arithmetic of the reference kernel's build
//     (src/ext/mxfp4_decode.cu:258);
//   * the E2M1 magnitude index read from the bits of |x| (e2m1_mag) against
//     the threshold definition of quant/fp4_format.py:24-46 (midpoints
//     .25 .75 1.25 1.75 2.5 3.5 5, ties up, NaN -> 7).
// Both are checked on all 2^32 bit patterns; NaN results compare equal to any
// NaN (only NaN-ness is observable downstream: the quantiser maps every NaN
// to the same code).
#include "mx_common.cuh"
#include "work.cuh"

#include "../../include/moe_fp4.h"

namespace mfi {
namespace {

__device__ __forceinline__ uint32_t e2m1_mag_thresholds(float a) {
  uint32_t c = 0;
  c += (a >= 0.25f);
  c += (a >= 0.75f);
  c += (a >= 1.25f);
  c += (a >= 1.75f);
  c += (a >= 2.5f);
  c += (a >= 3.5f);
  c += (a >= 5.0f);
  return (a != a) ? 7u : c;
}

// out[0], out[1]: mismatch counts (quotient, E2M1); out[2], out[3]: the
// smallest mismatching bit pattern of each (0xFFFFFFFF... when none).
__global__ void __launch_bounds__(256) selftest_kernel(unsigned long long* out) {
  unsigned long long bad_q = 0, bad_m = 0;
  unsigned long long first_q = ~0ull, first_m = ~0ull;
  const unsigned long long stride = (unsigned long long)gridDim.x * blockDim.x;
  for (unsigned long long i = (unsigned long long)blockIdx.x * blockDim.x + threadIdx.x;
       i < (1ull << 32); i += stride) {
    const float g = __uint_as_float(uint32_t(i));
    const float q = swiglu_quotient(g);
    const float r = __fdiv_rn(g, __fadd_rn(1.0f, expf(-g)));
    if (!(__float_as_uint(q) == __float_as_uint(r) || (q != q && r != r))) {
      ++bad_q;
      first_q = min(first_q, i);
    }
    const float a = fabsf(g);
    if (e2m1_mag(a) != e2m1_mag_thresholds(a)) {
      ++bad_m;
      first_m = min(first_m, i);
    }
  }
  if (bad_q) {
    atomicAdd(&out[0], bad_q);
    atomicMin(&out[2], first_q);
  }
  if (bad_m) {
    atomicAdd(&out[1], bad_m);
    atomicMin(&out[3], first_m);
  }
}

__global__ void selftest_init_kernel(unsigned long long* out) {
  if (threadIdx.x < 4) out[threadIdx.x] = threadIdx.x < 2 ? 0ull : ~0ull;
}

}  // namespace
}  // namespace mfi

extern "C" int mfi_selftest_numerics(unsigned long long* out, void* stream) {
  if (!out) return mfi::set_last_error(MFI_ERR_ARG, "null pointer");
  if (reinterpret_cast<uintptr_t>(out) & 7)
    return mfi::set_last_error(MFI_ERR_ARG, "selftest: out must be 8-byte aligned");
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  mfi::selftest_init_kernel<<<1, 32, 0, st>>>(out);
  mfi::selftest_kernel<<<148 * 8, 256, 0, st>>>(out);
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? MFI_OK : mfi::set_last_error(MFI_ERR_CUDA, cudaGetErrorString(e));
}
