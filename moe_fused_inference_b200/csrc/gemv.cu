// gemv.cu — grouped MXFP4 GEMV for decode-sized problems (CUDA cores).
//
// Replaces the reference's per-(token, slot, projection) kernels
// gateup_kernel / down_silu_kernel / lin_pq_kernel
// (src/ext/mxfp4_decode.cu:135-279), which re-stream an expert's weights once
// for every (token, slot) pair that selects it.  Here the work is described
// by a device-side list of weight groups: each group is one weight matrix
// (wp, wsc) and the list of activation rows that multiply it.  A work item is
// (group, tile of 32 weight rows); the weight tile is streamed from HBM once
// and applied to every row of the group, 8 activation rows at a time.
//
// Arithmetic: each 32-element block product is an exact integer (dp4a over
// nibbles expanded to int8 = 2*e2m1), scaled by 2^(sa+sb-256) and summed in
// fp32 — lane-local over the blocks b = lane, lane+32, ... then by a fixed
// xor-butterfly across the warp.  The result is deterministic run to run.
#include "mx_common.cuh"
#include "work.cuh"
#include "tc_ptx.cuh"

namespace mfi {

constexpr int kRowsPerWarp = 4;
constexpr int kWarps = 8;
constexpr int kTileRows = kRowsPerWarp * kWarps;  // 32
constexpr int kTG = 8;                              // activation rows per pass

// Warp reduce-scatter of 32 per-lane values: afterwards lane l holds the sum
// over the warp of v[l].
__device__ __forceinline__ float butterfly32(float (&v)[32], int lane) {
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) {
    const bool upper = (lane & off) != 0;
#pragma unroll
    for (int i = 0; i < off; ++i) {
      const float send = upper ? v[i] : v[i + off];
      const float keep = upper ? v[i + off] : v[i];
      v[i] = keep + __shfl_xor_sync(0xffffffffu, send, off);
    }
  }
  return v[0];
}

// Dense form (groups == nullptr): one weight (dense.wp, dense.wsc) applied to
// activation rows 0..M-1, output row m at m*ldy, split into groups of
// kDenseChunk rows so large M spreads over the grid.
constexpr int kDenseChunk = 64;

struct DenseDesc {
  const uint8_t* wp;
  const uint8_t* wsc;
  int M;
  long long ldy;
};

__device__ __forceinline__ GroupDesc get_group(const GroupDesc* groups, const DenseDesc& d, int g) {
  if (groups) return groups[g];
  GroupDesc gd;
  gd.wp = d.wp;
  gd.wsc = d.wsc;
  gd.first = g * kDenseChunk;
  gd.count = min(kDenseChunk, d.M - g * kDenseChunk);
  return gd;
}

__device__ __forceinline__ EntryDesc get_entry(const EntryDesc* entries, const DenseDesc& d, int i) {
  if (entries) return entries[i];
  EntryDesc e;
  e.act_row = i;
  e.pad = 0;
  e.out_off = (long long)i * d.ldy;
  return e;
}

__global__ void __launch_bounds__(256) grouped_gemv_kernel(
    const GroupDesc* __restrict__ groups, const int* __restrict__ n_groups_dev, int n_groups_host,
    const EntryDesc* __restrict__ entries, DenseDesc dense, const uint8_t* __restrict__ xq,
    const uint8_t* __restrict__ xsc, float* __restrict__ y, int N, int Kp) {
  extern __shared__ __align__(16) uint8_t smem[];
  uint8_t* s_act = smem;                   // kTG x Kp int8
  uint8_t* s_sc = smem + kTG * Kp;         // kTG x nb codes
  const int nb = Kp >> 5;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int n_groups = n_groups_dev ? *n_groups_dev : n_groups_host;
  const int n_tiles = (N + kTileRows - 1) / kTileRows;
  const long n_items = long(n_groups) * n_tiles;

  for (long item = blockIdx.x; item < n_items; item += gridDim.x) {
    const int g = int(item / n_tiles), tile = int(item % n_tiles);
    const GroupDesc gd = get_group(groups, dense, g);
    const int row0 = tile * kTileRows + warp * kRowsPerWarp;
    for (int c0 = 0; c0 < gd.count; c0 += kTG) {
      const int tg = min(kTG, gd.count - c0);
      __syncthreads();
      // stage activation rows: nibbles -> int8
      for (int idx = threadIdx.x; idx < tg * (Kp >> 3); idx += blockDim.x) {
        const int j = idx / (Kp >> 3), w = idx % (Kp >> 3);
        const int ar = get_entry(entries, dense, gd.first + c0 + j).act_row;
        const uint32_t p = *reinterpret_cast<const uint32_t*>(xq + long(ar) * (Kp >> 1) + w * 4);
        uint32_t lo, hi;
        nib8_to_i8(p, lo, hi);
        reinterpret_cast<uint2*>(s_act + j * Kp)[w] = make_uint2(lo, hi);
      }
      for (int idx = threadIdx.x; idx < tg * nb; idx += blockDim.x) {
        const int j = idx / nb, b = idx % nb;
        const int ar = get_entry(entries, dense, gd.first + c0 + j).act_row;
        s_sc[j * nb + b] = xsc[long(ar) * nb + b];
      }
      __syncthreads();

      float acc[32];
#pragma unroll
      for (int i = 0; i < 32; ++i) acc[i] = 0.0f;
      for (int kb = lane; kb < nb; kb += 32) {
        uint4 wv[kRowsPerWarp];
        int sw[kRowsPerWarp];
#pragma unroll
        for (int i = 0; i < kRowsPerWarp; ++i) {
          const int n = row0 + i;
          if (n < N) {
            wv[i] = ldg_u4(gd.wp + long(n) * (Kp >> 1) + kb * 16);
            sw[i] = gd.wsc[long(n) * nb + kb];
          } else {
            wv[i] = make_uint4(0, 0, 0, 0);
            sw[i] = 127;
          }
        }
        uint32_t w8[kRowsPerWarp][8];
#pragma unroll
        for (int i = 0; i < kRowsPerWarp; ++i) {
          nib8_to_i8(wv[i].x, w8[i][0], w8[i][1]);
          nib8_to_i8(wv[i].y, w8[i][2], w8[i][3]);
          nib8_to_i8(wv[i].z, w8[i][4], w8[i][5]);
          nib8_to_i8(wv[i].w, w8[i][6], w8[i][7]);
        }
#pragma unroll
        for (int j = 0; j < kTG; ++j) {
          if (j < tg) {
            const uint4* a4 = reinterpret_cast<const uint4*>(s_act + j * Kp + kb * 32);
            const uint4 a0 = a4[0], a1 = a4[1];
            const uint32_t a8[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
            const int sa = s_sc[j * nb + kb];
#pragma unroll
            for (int i = 0; i < kRowsPerWarp; ++i) {
              const int s = dot_i8x32(w8[i], a8);
              acc[i * kTG + j] += block_value(s, sw[i], sa);
            }
          }
        }
      }
      const float v = butterfly32(acc, lane);
      const int i = lane >> 3, j = lane & 7;
      const int n = row0 + i;
      if (j < tg && n < N) y[get_entry(entries, dense, gd.first + c0 + j).out_off + n] = v;
    }
  }
}

size_t gemv_smem_bytes(int Kp) { return size_t(kTG) * (Kp + (Kp >> 5)); }

static cudaError_t launch_gemv_impl(const GroupDesc* groups, const int* n_groups_dev,
                                    int n_groups_host, const EntryDesc* entries,
                                    const DenseDesc& dense, const uint8_t* xq, const uint8_t* xsc,
                                    float* y, int N, int Kp, int max_ctas, cudaStream_t stream) {
  const size_t smem = gemv_smem_bytes(Kp);
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(grouped_gemv_kernel,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
    if (e != cudaSuccess) return e;
  }
  const int n_tiles = (N + kTileRows - 1) / kTileRows;
  long items = long(n_groups_host) * n_tiles;
  long grid = items < max_ctas ? items : max_ctas;
  if (grid <= 0) return cudaSuccess;
  grouped_gemv_kernel<<<unsigned(grid), kWarps * 32, smem, stream>>>(
      groups, n_groups_dev, n_groups_host, entries, dense, xq, xsc, y, N, Kp);
  return cudaGetLastError();
}

cudaError_t launch_grouped_gemv(const GroupDesc* groups, const int* n_groups_dev, int n_groups_host,
                                const EntryDesc* entries, const uint8_t* xq, const uint8_t* xsc,
                                float* y, int N, int Kp, int max_ctas, cudaStream_t stream) {
  DenseDesc d{nullptr, nullptr, 0, 0};
  return launch_gemv_impl(groups, n_groups_dev, n_groups_host, entries, d, xq, xsc, y, N, Kp,
                          max_ctas, stream);
}

cudaError_t launch_dense_gemv(const uint8_t* xq, const uint8_t* xsc, const uint8_t* wp,
                              const uint8_t* wsc, float* y, long long ldy, int M, int N, int Kp,
                              cudaStream_t stream) {
  // a long weight stream, or enough rows to keep the CUDA cores busy: the
  // tensor-core form (~100 KB in flight per SM) is faster; short matrices at
  // one to a few rows stay on the GEMV (one tile per CTA, lower latency)
  if ((N >= 16384 || M >= 6) && lin_tc_supported(xq, xsc, wp, wsc, M, Kp))
    return launch_lin_tc(xq, xsc, wp, wsc, y, ldy, M, N, Kp, stream);
  DenseDesc d{wp, wsc, M, ldy};
  const int ng = (M + kDenseChunk - 1) / kDenseChunk;
  return launch_gemv_impl(nullptr, nullptr, ng, nullptr, d, xq, xsc, y, N, Kp, 1 << 30, stream);
}

// ---------------------------------------------------------------------------
// Pointer-table grouping (drop-in moe_gateup / moe_down / *_tab).
// Entry z of a table of length P is (wp_tab[z], wsc_tab[z]); entries with the
// same (wp, wsc) pair form one group, in order of first appearance, and keep
// ascending z inside the group.  The caller's table order (reference
// src/ext/mxfp4_decode.cu:193-195 for gate/up, :233 for down) decides the
// activation row and output row of each entry:
//   mode 0 (gate/up): z = m*2E + proj*E + e -> act row m, out row (m*E+e)*2N + proj*N
//   mode 1 (down):    z = m*E + e           -> act row z, out row z*N
// One CTA of 1024 threads; P <= 4096 (the table is staged in shared memory).
// Every step is spread over the block: each entry finds its group's first
// entry (its lead) and its rank among the group's entries by one pass over
// the entries before it, and the group numbering and the group offsets are
// block-wide prefix sums.
// ---------------------------------------------------------------------------
constexpr int kBgThreads = 1024;

// Exclusive prefix sum of v[0..n) in place (n <= 4 * kBgThreads), returns the
// total.  Each thread sums four consecutive elements, warps scan by shuffles,
// the 32 warp totals are scanned by warp 0.
__device__ int block_exclusive_scan(int* v, int n, int* s_warp) {
  const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
  int a[4], sum = 0;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int k = 4 * t + i;
    a[i] = k < n ? v[k] : 0;
    sum += a[i];
  }
  int inc = sum;
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) {
    const int u = __shfl_up_sync(0xffffffffu, inc, off);
    if (lane >= off) inc += u;
  }
  if (lane == 31) s_warp[warp] = inc;
  __syncthreads();
  if (warp == 0) {
    int w = s_warp[lane];
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const int u = __shfl_up_sync(0xffffffffu, w, off);
      if (lane >= off) w += u;
    }
    s_warp[lane] = w;  // inclusive
  }
  __syncthreads();
  int run = inc - sum + (warp > 0 ? s_warp[warp - 1] : 0);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int k = 4 * t + i;
    if (k < n) v[k] = run;
    run += a[i];
  }
  const int total = s_warp[31];
  __syncthreads();
  return total;
}

__global__ void __launch_bounds__(kBgThreads) build_groups_kernel(
    const uint8_t* const* __restrict__ wp_tab, const uint8_t* const* __restrict__ wsc_tab, int P,
    int mode, int E, int N, GroupDesc* __restrict__ groups, int* __restrict__ n_groups,
    EntryDesc* __restrict__ entries) {
  tc::grid_dep_wait();  // the tables may come from the kernel before
  tc::grid_dep_launch();
  extern __shared__ __align__(16) unsigned char shraw[];
  const uint8_t** s_wp = reinterpret_cast<const uint8_t**>(shraw);  // P
  const uint8_t** s_ws = s_wp + P;                                    // P
  int* lead = reinterpret_cast<int*>(s_ws + P);  // P: first entry of the entry's group
  int* rank = lead + P;                          // P: place among its group's entries
  int* gidx = lead + 2 * P;                      // P: is-lead flags, then group index of a lead
  int* cnt = lead + 3 * P;                       // P: entries per group, then group offsets
  __shared__ int s_warp[32];
  for (int z = threadIdx.x; z < P; z += blockDim.x) {
    s_wp[z] = wp_tab[z];
    s_ws[z] = wsc_tab[z];
    cnt[z] = 0;
  }
  __syncthreads();
  for (int z = threadIdx.x; z < P; z += blockDim.x) {
    const uint8_t* a = s_wp[z];
    const uint8_t* b = s_ws[z];
    int l = z, r = 0;
    for (int j = 0; j < z; ++j) {
      const bool same = s_wp[j] == a && s_ws[j] == b;
      if (same && l == z) l = j;
      r += same;
    }
    lead[z] = l;
    rank[z] = r;
    gidx[z] = l == z;
  }
  __syncthreads();
  const int ng = block_exclusive_scan(gidx, P, s_warp);  // gidx[lead] = its group's index
  for (int z = threadIdx.x; z < P; z += blockDim.x) atomicAdd(&cnt[gidx[lead[z]]], 1);
  __syncthreads();
  block_exclusive_scan(cnt, ng, s_warp);  // cnt[g] = first entry of group g
  for (int z = threadIdx.x; z < P; z += blockDim.x) {
    if (lead[z] == z) {
      const int g = gidx[z];
      GroupDesc gd;
      gd.wp = s_wp[z];
      gd.wsc = s_ws[z];
      gd.first = cnt[g];
      gd.count = (g + 1 < ng ? cnt[g + 1] : P) - cnt[g];
      groups[g] = gd;
    }
  }
  for (int z = threadIdx.x; z < P; z += blockDim.x) {
    const int g = gidx[lead[z]];
    EntryDesc ed;
    ed.pad = 0;
    if (mode == 0) {
      const int m = z / (2 * E), pair = z % (2 * E), proj = pair / E, e = pair % E;
      ed.act_row = m;
      ed.out_off = (long long)(m * E + e) * 2 * N + (long long)proj * N;
    } else {
      ed.act_row = z;
      ed.out_off = (long long)z * N;
    }
    entries[cnt[g] + rank[z]] = ed;
  }
  if (threadIdx.x == 0) *n_groups = ng;
}

cudaError_t launch_build_groups(const uint8_t* const* wp_tab, const uint8_t* const* wsc_tab, int P,
                                int mode, int E, int N, GroupDesc* groups, int* n_groups,
                                EntryDesc* entries, cudaStream_t stream, bool pdl) {
  if (P <= 0 || P > 4 * kBgThreads) return cudaErrorInvalidValue;
  const size_t smem = size_t(P) * (2 * sizeof(void*) + 4 * sizeof(int));
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(build_groups_kernel,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
    if (e != cudaSuccess) return e;
  }
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(1);
  cfg.blockDim = dim3(kBgThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, build_groups_kernel, wp_tab, wsc_tab, P, mode, E, N, groups,
                            n_groups, entries);
}

// ---------------------------------------------------------------------------
// Top-k combine: out[m, c] = sum_{e<E} w[m, e] * yd[m*E + e, c], sequential in
// e, separate multiply and add (no FMA contraction) so the fp32 result is
// reproducible on the host (reference src/ext/mxfp4_decode.cu:285-299).
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256) combine_kernel(const float* __restrict__ yd, long ystride,
                                                      const float* __restrict__ w, int E, int E_sum,
                                                      float* __restrict__ out, int M, int N,
                                                      unsigned* __restrict__ clear, int n_clear) {
  tc::grid_dep_wait();  // yd comes from the previous kernel
  // the layer's per-call counters: every kernel that used them has completed
  if (clear && blockIdx.x == 0 && blockIdx.y == 0)
    for (int i = threadIdx.x; i < n_clear; i += blockDim.x) clear[i] = 0u;
  const int m = blockIdx.y;
  const int c4 = (blockIdx.x * blockDim.x + threadIdx.x) * 4;
  if (m >= M || c4 >= N) return;
  const float* yb = yd + long(m) * E * ystride;
  const float* wb = w + long(m) * E;
  if (c4 + 4 <= N && (ystride % 4) == 0 && (N % 4) == 0) {
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    if (E_sum == 8) {
      // the usual top-8: every slot's row and weight is loaded before the
      // (unchanged, sequential) sums, so the loads overlap
      float we[8];
      float4 v[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        we[e] = wb[e];
        v[e] = *reinterpret_cast<const float4*>(yb + long(e) * ystride + c4);
      }
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        acc.x = __fadd_rn(acc.x, __fmul_rn(we[e], v[e].x));
        acc.y = __fadd_rn(acc.y, __fmul_rn(we[e], v[e].y));
        acc.z = __fadd_rn(acc.z, __fmul_rn(we[e], v[e].z));
        acc.w = __fadd_rn(acc.w, __fmul_rn(we[e], v[e].w));
      }
    } else {
      for (int e = 0; e < E_sum; ++e) {
        const float we = wb[e];
        const float4 v = *reinterpret_cast<const float4*>(yb + long(e) * ystride + c4);
        acc.x = __fadd_rn(acc.x, __fmul_rn(we, v.x));
        acc.y = __fadd_rn(acc.y, __fmul_rn(we, v.y));
        acc.z = __fadd_rn(acc.z, __fmul_rn(we, v.z));
        acc.w = __fadd_rn(acc.w, __fmul_rn(we, v.w));
      }
    }
    *reinterpret_cast<float4*>(out + long(m) * N + c4) = acc;
  } else {
    for (int c = c4; c < c4 + 4 && c < N; ++c) {
      float acc = 0.f;
      for (int e = 0; e < E_sum; ++e) acc = __fadd_rn(acc, __fmul_rn(wb[e], yb[long(e) * ystride + c]));
      out[long(m) * N + c] = acc;
    }
  }
}

// Prefill: bf16 rows, 8 columns per thread, the same fp32 arithmetic.
__global__ void __launch_bounds__(256) combine_bf16_kernel(const __nv_bfloat16* __restrict__ yd,
                                                           const float* __restrict__ w, int k,
                                                           float* __restrict__ out, int M, int N) {
  tc::grid_dep_wait();  // yd comes from the previous kernel
  const int m = blockIdx.y;
  const int c8 = (blockIdx.x * blockDim.x + threadIdx.x) * 8;
  if (m >= M || c8 >= N) return;
  const __nv_bfloat16* yb = yd + long(m) * k * N + c8;
  const float* wb = w + long(m) * k;
  float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  for (int e = 0; e < k; ++e) {
    const float we = wb[e];
    const uint4 v = *reinterpret_cast<const uint4*>(yb + long(e) * N);
    const __nv_bfloat162* h2 = reinterpret_cast<const __nv_bfloat162*>(&v);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 f = __bfloat1622float2(h2[i]);
      acc[2 * i] = __fadd_rn(acc[2 * i], __fmul_rn(we, f.x));
      acc[2 * i + 1] = __fadd_rn(acc[2 * i + 1], __fmul_rn(we, f.y));
    }
  }
  float4* o = reinterpret_cast<float4*>(out + long(m) * N + c8);
  o[0] = make_float4(acc[0], acc[1], acc[2], acc[3]);
  o[1] = make_float4(acc[4], acc[5], acc[6], acc[7]);
}

cudaError_t launch_combine_bf16(const __nv_bfloat16* yd, const float* w, int k, float* out, int M,
                                int N, cudaStream_t stream, bool pdl) {
  if (M == 0 || N == 0) return cudaSuccess;
  if (N % 8 != 0) return cudaErrorInvalidValue;
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3((N / 8 + 255) / 256, M);
  cfg.blockDim = dim3(256);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, combine_bf16_kernel, yd, w, k, out, M, N);
}

cudaError_t launch_combine(const float* yd, long ystride, const float* w, int E, int E_sum,
                           float* out, int M, int N, cudaStream_t stream, bool pdl,
                           unsigned* clear, int n_clear) {
  if (M == 0 || N == 0) return cudaSuccess;
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3((N / 4 + 255) / 256 + 1, M);
  cfg.blockDim = dim3(256);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, combine_kernel, yd, ystride, w, E, E_sum, out, M, N, clear,
                            n_clear);
}

}  // namespace mfi
