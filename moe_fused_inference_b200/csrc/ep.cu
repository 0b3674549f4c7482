// ep.cu — expert-parallel plumbing around the expert GEMMs.
//
// The reference is single-GPU (no collective anywhere); expert parallelism
// is this library's addition.  128/N experts live on each
// of N ranks; every rank routes its own tokens, then
//   pack      one row per (token, destination rank) that the token routes to:
//             its MXFP4 row and scales plus the token's expert ids local to
//             that rank and their weights (quantising before dispatch is
//             identical to quantising after: the quantiser works per row);
//   dispatch  one all_to_all_single of fixed-size blocks (capacity C = T rows
//             + a header row holding the count) — no host synchronisation;
//   experts   mfi_moe_experts on every received row (invalid rows masked);
//   return    one all_to_all_single of the fp32 per-row partial sums;
//   unpack    out[t] = sum over ranks in rank order of the returned rows.
//
// Row layout (RB bytes, a multiple of 16):
//   [0, H/2) packed nibbles | [H/2, H/2+H/32) E8M0 codes | int32 token, 3 x pad |
//   k x int32 local expert id (-1 = none) | k x f32 weight | padding
#include "mx_common.cuh"
#include "work.cuh"
#include "tc_ptx.cuh"

namespace mfi {

int ep_row_bytes(int H, int k) {
  const int b = H / 2 + H / 32 + 16 + 8 * k;
  return (b + 15) / 16 * 16;
}

namespace {

struct RowLayout {
  int H, k, rb;
  __host__ __device__ int sc_off() const { return H / 2; }
  __host__ __device__ int meta_off() const { return H / 2 + H / 32; }
  __host__ __device__ int sel_off() const { return meta_off() + 16; }
  __host__ __device__ int w_off() const { return sel_off() + 4 * k; }
};

// One CTA per token: for each destination rank that owns one of the token's
// experts, claim a row in that rank's block and write row + metadata.
__global__ void __launch_bounds__(128) ep_pack_kernel(const uint8_t* __restrict__ xq,
                                                      const uint8_t* __restrict__ xsc,
                                                      const int* __restrict__ topi,
                                                      const float* __restrict__ topw, int T,
                                                      int n_ranks, int e_local, int C, RowLayout L,
                                                      int* __restrict__ counts,
                                                      uint8_t* __restrict__ send,
                                                      int* __restrict__ pack_pos) {
  const int t = blockIdx.x;
  __shared__ int s_pos[64];
  if (threadIdx.x < n_ranks) {
    const int d = threadIdx.x;
    bool any = false;
    for (int j = 0; j < L.k; ++j) any |= (topi[t * L.k + j] / e_local) == d;
    int pos = -1;
    if (any) pos = atomicAdd(counts + d, 1);
    s_pos[d] = pos;
    pack_pos[t * n_ranks + d] = pos;
  }
  __syncthreads();
  for (int d = 0; d < n_ranks; ++d) {
    const int pos = s_pos[d];
    if (pos < 0) continue;
    uint8_t* row = send + (size_t(d) * (C + 1) + 1 + pos) * L.rb;
    for (int i = threadIdx.x; i < L.H / 32; i += blockDim.x)
      reinterpret_cast<uint4*>(row)[i] = reinterpret_cast<const uint4*>(xq + size_t(t) * (L.H / 2))[i];
    for (int i = threadIdx.x; i < L.H / 128; i += blockDim.x)
      reinterpret_cast<uint32_t*>(row + L.sc_off())[i] =
          reinterpret_cast<const uint32_t*>(xsc + size_t(t) * (L.H / 32))[i];
    if (threadIdx.x == 0) reinterpret_cast<int*>(row + L.meta_off())[0] = t;
    if (threadIdx.x < L.k) {
      const int e = topi[t * L.k + threadIdx.x];
      reinterpret_cast<int*>(row + L.sel_off())[threadIdx.x] = (e / e_local) == d ? e % e_local : -1;
      reinterpret_cast<float*>(row + L.w_off())[threadIdx.x] = topw[t * L.k + threadIdx.x];
    }
  }
}

// Header rows carry the counts; after the exchange every row past its
// block's count (and every header row) gets all expert ids set to -1.
__global__ void ep_write_headers_kernel(const int* __restrict__ counts, int n_ranks, int C,
                                        RowLayout L, uint8_t* __restrict__ send) {
  const int d = threadIdx.x;
  if (d < n_ranks) reinterpret_cast<int*>(send + size_t(d) * (C + 1) * L.rb)[0] = counts[d];
}

__global__ void ep_mask_recv_kernel(int n_ranks, int C, RowLayout L, uint8_t* __restrict__ recv) {
  const long long rows = (long long)n_ranks * (C + 1);
  for (long long g = blockIdx.x * (long long)blockDim.x + threadIdx.x; g < rows;
       g += (long long)gridDim.x * blockDim.x) {
    const int s = int(g / (C + 1)), r = int(g % (C + 1));
    const int count = reinterpret_cast<const int*>(recv + size_t(s) * (C + 1) * L.rb)[0];
    if (r == 0 || r - 1 >= count) {
      int* sel = reinterpret_cast<int*>(recv + size_t(g) * L.rb + L.sel_off());
      for (int j = 0; j < L.k; ++j) sel[j] = -1;
    }
  }
}

// out[t] = sum over ranks d (in rank order) of the row returned for (t, d).
__global__ void ep_unpack_kernel(const float* __restrict__ ret, const int* __restrict__ pack_pos,
                                 int T, int n_ranks, int C, int H, float* __restrict__ out) {
  const int t = blockIdx.y;
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= H) return;
  float acc = 0.0f;
  for (int d = 0; d < n_ranks; ++d) {
    const int pos = pack_pos[t * n_ranks + d];
    if (pos >= 0) acc = __fadd_rn(acc, ret[(size_t(d) * (C + 1) + 1 + pos) * H + c]);
  }
  out[size_t(t) * H + c] = acc;
}

// Expert-region scatter for pre-routed rows: row r's expert list sel[r][j]
// (-1 = none) claims rows in the per-expert regions like route.cu does.
__global__ void __launch_bounds__(128) scatter_sel_kernel(
    const uint8_t* __restrict__ xq, long long xq_ld, const uint8_t* __restrict__ xsc,
    long long xsc_ld, const int* __restrict__ sel, long long sel_ld, int R, int k, int H, int E,
    int T_pad, int* __restrict__ cursor, int* __restrict__ perm, uint8_t* __restrict__ xp,
    uint8_t* __restrict__ xp_atoms, int* __restrict__ status) {
  tc::grid_dep_launch();
  const int r = blockIdx.x;
  __shared__ int s_row[32];
  if (threadIdx.x < k) {
    const int e = sel[size_t(r) * sel_ld + threadIdx.x];
    int row = -1;
    if (e >= E) {
      atomicCAS(status, 0, 4);  // expert id out of range
    } else if (e >= 0) {
      const int pos = atomicAdd(cursor + e, 1);
      if (pos < T_pad) {
        row = e * T_pad + pos;
        perm[row] = r * k + threadIdx.x;
      } else {
        atomicCAS(status, 0, 5);  // an expert listed twice in one row overfills its region
      }
    }
    s_row[threadIdx.x] = row;
  }
  __syncthreads();
  const int q16 = H / 32, kc = H / 128;
  for (int j = 0; j < k; ++j) {
    const int row = s_row[j];
    if (row < 0) continue;
    for (int i = threadIdx.x; i < q16; i += blockDim.x)
      reinterpret_cast<uint4*>(xp + size_t(row) * (H / 2))[i] =
          reinterpret_cast<const uint4*>(xq + size_t(r) * xq_ld)[i];
    for (int i = threadIdx.x; i < kc; i += blockDim.x)
      *reinterpret_cast<uint32_t*>(xp_atoms + (size_t(row >> 5) * kc + i) * 512 + (row & 31) * 16) =
          reinterpret_cast<const uint32_t*>(xsc + size_t(r) * xsc_ld)[i];
  }
}

// Combine with a slot mask: out[m] = sum over slots j with 0 <= sel < E of
// w[m][j] * yd[m*k + j], sequential in j (unfused multiply and add).
__global__ void combine_sel_kernel(const float* __restrict__ yd, const int* __restrict__ sel,
                                   long long sel_ld, const float* __restrict__ w, long long w_ld,
                                   int k, int E, int H, float* __restrict__ out, long long out_ld) {
  tc::grid_dep_wait();  // yd comes from the previous kernel
  const int m = blockIdx.y;
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= H) return;
  float acc = 0.0f;
  for (int j = 0; j < k; ++j)
    if (unsigned(sel[size_t(m) * sel_ld + j]) < unsigned(E))
      acc = __fadd_rn(acc, __fmul_rn(w[size_t(m) * w_ld + j], yd[(size_t(m) * k + j) * H + c]));
  out[size_t(m) * out_ld + c] = acc;
}

}  // namespace

cudaError_t launch_ep_pack(const uint8_t* xq, const uint8_t* xsc, const int* topi,
                           const float* topw, int T, int H, int k, int n_ranks, int e_local, int C,
                           int* counts, uint8_t* send, int* pack_pos, cudaStream_t stream) {
  RowLayout L{H, k, ep_row_bytes(H, k)};
  cudaError_t e = cudaMemsetAsync(counts, 0, sizeof(int) * n_ranks, stream);
  if (e != cudaSuccess) return e;
  if (T > 0) {
    ep_pack_kernel<<<T, 128, 0, stream>>>(xq, xsc, topi, topw, T, n_ranks, e_local, C, L, counts,
                                          send, pack_pos);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
  }
  ep_write_headers_kernel<<<1, 64, 0, stream>>>(counts, n_ranks, C, L, send);
  return cudaGetLastError();
}

cudaError_t launch_ep_mask_recv(int n_ranks, int C, int H, int k, uint8_t* recv,
                                cudaStream_t stream) {
  RowLayout L{H, k, ep_row_bytes(H, k)};
  const long long rows = (long long)n_ranks * (C + 1);
  int blocks = int((rows + 255) / 256);
  if (blocks < 1) blocks = 1;
  ep_mask_recv_kernel<<<blocks, 256, 0, stream>>>(n_ranks, C, L, recv);
  return cudaGetLastError();
}

cudaError_t launch_ep_unpack(const float* ret, const int* pack_pos, int T, int n_ranks, int C,
                             int H, float* out, cudaStream_t stream) {
  if (T == 0) return cudaSuccess;
  dim3 grid((H + 255) / 256, T);
  ep_unpack_kernel<<<grid, 256, 0, stream>>>(ret, pack_pos, T, n_ranks, C, H, out);
  return cudaGetLastError();
}

cudaError_t launch_scatter_sel(const uint8_t* xq, long long xq_ld, const uint8_t* xsc,
                               long long xsc_ld, const int* sel, long long sel_ld, int R, int k,
                               int H, int E, int T_pad, int* cursor, int* perm, uint8_t* xp,
                               uint8_t* xp_atoms, int* status, cudaStream_t stream) {
  if (R == 0) return cudaSuccess;
  scatter_sel_kernel<<<R, 128, 0, stream>>>(xq, xq_ld, xsc, xsc_ld, sel, sel_ld, R, k, H, E, T_pad,
                                            cursor, perm, xp, xp_atoms, status);
  return cudaGetLastError();
}

cudaError_t launch_combine_sel(const float* yd, const int* sel, long long sel_ld, const float* w,
                               long long w_ld, int R, int k, int E, int H, float* out,
                               long long out_ld, cudaStream_t stream) {
  if (R == 0) return cudaSuccess;
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3((H + 255) / 256, R);
  cfg.blockDim = dim3(256);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, combine_sel_kernel, yd, sel, sel_ld, w, w_ld, k, E, H, out,
                            out_ld);
}

}  // namespace mfi
