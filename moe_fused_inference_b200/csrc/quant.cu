// quant.cu — MXFP4 row quantiser (activations and weights).
//
// Replaces the reference's activation quantiser prequant_kernel
// (src/ext/mxfp4_decode.cu:24-50) and the in-kernel activation quantisation of
// mxfp4_linear_kernel (src/ext/mxfp4_linear.cu:128-144), and is a bit-exact
// device version of the weight quantiser quantize_expert_tensor
// (quant/quantize_mxfp4.py:110-160).
//
// Mapping: one thread per 8 consecutive elements, a quad of threads per
// 32-element block (amax by two xor-shuffles), one 32-bit nibble word per
// thread.  Rows are independent, so the grid is a flat 1-D range over
// M * Kp/8 threads; the HBM traffic is the minimum (read x once, write
// Kp/2 + Kp/32 bytes per row).
#include "mx_common.cuh"
#include "work.cuh"
#include "tc_ptx.cuh"

namespace mfi {

template <bool kVec>
__global__ void __launch_bounds__(256) quant_rows_kernel(QuantArgs a) {
  const long tid = long(blockIdx.x) * blockDim.x + threadIdx.x;
  const int per_row = a.Kp >> 3;
  const long total = long(a.M) * per_row;
  // Threads past the end still take part in the quad shuffles (full-warp
  // mask); they hold zeros and store nothing.
  const bool live = tid < total;
  const int row = live ? int(tid / per_row) : 0;
  const int c8 = live ? int(tid % per_row) : 0;
  const int k0 = c8 << 3;

  float v[8];
  if (kVec && live && k0 + 8 <= a.K) {
    const uint4 raw = *reinterpret_cast<const uint4*>(
        reinterpret_cast<const uint8_t*>(a.x) + (row * a.ld_x + k0) * (a.dtype == kF32 ? 4 : 2));
    if (a.dtype == kBF16) {
      const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&raw);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        float2 f = __bfloat1622float2(h[i]);
        v[2 * i] = f.x;
        v[2 * i + 1] = f.y;
      }
    } else {
      const __half2* h = reinterpret_cast<const __half2*>(&raw);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        float2 f = __half22float2(h[i]);
        v[2 * i] = f.x;
        v[2 * i + 1] = f.y;
      }
    }
  } else {
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int k = k0 + i;
      v[i] = (live && k < a.K) ? load_elem(a.x, row * a.ld_x + k, a.dtype) : 0.0f;
    }
  }
  if (a.half_rt) {
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = __half2float(__float2half_rn(v[i]));
  }
  BlockScale bs;
  const uint32_t word = quant_group8(v, bs);
  if (!live) return;
  *reinterpret_cast<uint32_t*>(a.xq + long(row) * (a.Kp >> 1) + (k0 >> 1)) = word;
  if ((c8 & 3) == 0) a.xsc[long(row) * (a.Kp >> 5) + (c8 >> 2)] = bs.code;
}

cudaError_t launch_quant_rows(const QuantArgs& a, cudaStream_t stream) {
  const long total = long(a.M) * (a.Kp >> 3);
  if (total == 0) return cudaSuccess;
  const int threads = 256;
  const long blocks = (total + threads - 1) / threads;
  const int esz = a.dtype == kF32 ? 4 : 2;
  const bool vec = a.dtype != kF32 && (a.K % 8 == 0) && (a.ld_x % 8 == 0) &&
                   (reinterpret_cast<uintptr_t>(a.x) % 16 == 0) && esz == 2;
  if (vec)
    quant_rows_kernel<true><<<unsigned(blocks), threads, 0, stream>>>(a);
  else
    quant_rows_kernel<false><<<unsigned(blocks), threads, 0, stream>>>(a);
  return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// SwiGLU + requantisation of the gate/up output (decode semantics).
// h = g / (1 + exp(-g)) * u in fp32 (reference src/ext/mxfp4_decode.cu:252-272),
// then the same row quantiser.  gu rows are (g[0:K] | u[0:K]).
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256) swiglu_quant_kernel(const float* __restrict__ gu, long ld_gu,
                                                           const int* __restrict__ rows, int n_rows,
                                                           const int* __restrict__ n_rows_dev,
                                                           uint8_t* __restrict__ hq,
                                                           uint8_t* __restrict__ hsc, int K, int Kp) {
  tc::grid_dep_wait();  // gu (and the row list) come from the kernel before
  tc::grid_dep_launch();
  const int nr = n_rows_dev ? *n_rows_dev : n_rows;
  const int per_row = Kp >> 3;
  const long total = long(nr) * per_row;
  for (long base = long(blockIdx.x) * blockDim.x; base < total; base += long(gridDim.x) * blockDim.x) {
    const long tid = base + threadIdx.x;
    const bool live = tid < total;
    const int r = live ? int(tid / per_row) : 0;
    const int c8 = live ? int(tid % per_row) : 0;
    const int row = rows ? (live ? rows[r] : 0) : r;
    const int k0 = c8 << 3;
    float v[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int k = k0 + i;
      float h = 0.0f;
      if (live && k < K) {
        const float g = gu[row * ld_gu + k];
        const float u = gu[row * ld_gu + K + k];
        h = swiglu(g, u);
      }
      v[i] = h;
    }
    float am = 0.0f;
    bool has_nan = false;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      am = fmaxf(am, fabsf(v[i]));
      has_nan |= (v[i] != v[i]);
    }
    am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, 1));
    am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, 2));
    has_nan |= __shfl_xor_sync(0xffffffffu, int(has_nan), 1) != 0;
    has_nan |= __shfl_xor_sync(0xffffffffu, int(has_nan), 2) != 0;
    const BlockScale bs = block_scale(has_nan ? __uint_as_float(0x7fc00000u) : am);
    uint32_t word = 0;
#pragma unroll
    for (int i = 0; i < 8; ++i) word |= quant_nibble(v[i], bs.inv) << (4 * i);
    if (live) {
      *reinterpret_cast<uint32_t*>(hq + long(row) * (Kp >> 1) + (k0 >> 1)) = word;
      if ((c8 & 3) == 0) hsc[long(row) * (Kp >> 5) + (c8 >> 2)] = bs.code;
    }
  }
}

cudaError_t launch_swiglu_quant(const float* gu, long ld_gu, const int* rows, int n_rows,
                                const int* n_rows_dev, uint8_t* hq, uint8_t* hsc, int K, int Kp,
                                cudaStream_t stream, bool pdl) {
  const long total = long(n_rows) * (Kp >> 3);
  if (total == 0) return cudaSuccess;
  const int threads = 256;
  long blocks = (total + threads - 1) / threads;
  if (blocks > 148 * 16) blocks = 148 * 16;
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(unsigned(blocks));
  cfg.blockDim = dim3(threads);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, swiglu_quant_kernel, gu, ld_gu, rows, n_rows, n_rows_dev, hq, hsc,
                            K, Kp);
}

}  // namespace mfi
