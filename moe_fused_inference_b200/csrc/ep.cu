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

// sum over i < m, in order, of w[i] * rows[i][off .. off+3] (w == null: the
// plain sum) with unfused fp32 multiply and add.  All loads of a group of 8
// rows are issued before the first add, so the sum is latency-bound once per
// group, not once per row.  kCg: load through L2 only (rows a peer wrote).
template <bool kCg>
__device__ __forceinline__ float4 ordered_sum4(const float* const* rows, const float* w, int m,
                                               size_t off) {
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int i0 = 0; i0 < m; i0 += 8) {
    float4 v[8];
#pragma unroll
    for (int i = 0; i < 8; ++i)
      if (i0 + i < m) {
        const float4* src = reinterpret_cast<const float4*>(rows[i0 + i] + off);
        v[i] = kCg ? __ldcg(src) : *src;
      }
#pragma unroll
    for (int i = 0; i < 8; ++i)
      if (i0 + i < m) {
        if (w) {
          const float wi = w[i0 + i];
          acc.x = __fadd_rn(acc.x, __fmul_rn(wi, v[i].x));
          acc.y = __fadd_rn(acc.y, __fmul_rn(wi, v[i].y));
          acc.z = __fadd_rn(acc.z, __fmul_rn(wi, v[i].z));
          acc.w = __fadd_rn(acc.w, __fmul_rn(wi, v[i].w));
        } else {
          acc.x = __fadd_rn(acc.x, v[i].x);
          acc.y = __fadd_rn(acc.y, v[i].y);
          acc.z = __fadd_rn(acc.z, v[i].z);
          acc.w = __fadd_rn(acc.w, v[i].w);
        }
      }
  }
  return acc;
}

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

// A block whose count lies outside [0, C] (a corrupted header) is reported
// (device error 9) and treated as empty.
__global__ void ep_mask_recv_kernel(int n_ranks, int C, RowLayout L, uint8_t* __restrict__ recv,
                                    int* __restrict__ err) {
  const long long rows = (long long)n_ranks * (C + 1);
  for (long long g = blockIdx.x * (long long)blockDim.x + threadIdx.x; g < rows;
       g += (long long)gridDim.x * blockDim.x) {
    const int s = int(g / (C + 1)), r = int(g % (C + 1));
    int count = reinterpret_cast<const int*>(recv + size_t(s) * (C + 1) * L.rb)[0];
    if (count < 0 || count > C) {
      if (r == 0 && err) atomicCAS(err, 0, 9);
      count = 0;
    }
    if (r == 0 || r - 1 >= count) {
      int* sel = reinterpret_cast<int*>(recv + size_t(g) * L.rb + L.sel_off());
      for (int j = 0; j < L.k; ++j) sel[j] = -1;
    }
  }
}

// out[t] = sum over ranks d (in rank order) of the row returned for (t, d).
// One CTA per token, 4 columns per thread.
__global__ void __launch_bounds__(128) ep_unpack_kernel(const float* __restrict__ ret,
                                                        const int* __restrict__ pack_pos, int T,
                                                        int n_ranks, int C, int H,
                                                        float* __restrict__ out) {
  const int t = blockIdx.x;
  __shared__ const float* s_rows[kEpMaxRanks];
  __shared__ int s_m;
  if (threadIdx.x < 32) {
    // lanes look at ranks d, d+32 (n <= 64); rows compacted in rank order
    int base = 0;
    for (int d0 = 0; d0 < n_ranks; d0 += 32) {
      const int d = d0 + threadIdx.x;
      const int pos = d < n_ranks ? pack_pos[t * n_ranks + d] : -1;
      const unsigned mask = __ballot_sync(0xffffffffu, pos >= 0);
      if (pos >= 0)
        s_rows[base + __popc(mask & ((1u << threadIdx.x) - 1u))] = ret + (size_t(d) * (C + 1) + 1 + pos) * H;
      base += __popc(mask);
    }
    if (threadIdx.x == 0) s_m = base;
  }
  __syncthreads();
  for (int c4 = threadIdx.x * 4; c4 < H; c4 += blockDim.x * 4)
    *reinterpret_cast<float4*>(out + size_t(t) * H + c4) = ordered_sum4<false>(s_rows, nullptr, s_m, c4);
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
// w[m][j] * yd[m*k + j], sequential in j (unfused multiply and add).  One CTA
// per row, 4 columns per thread.
__global__ void __launch_bounds__(128) combine_sel_kernel(
    const float* __restrict__ yd, const int* __restrict__ sel, long long sel_ld,
    const float* __restrict__ w, long long w_ld, int k, int E, int H, float* __restrict__ out,
    long long out_ld) {
  tc::grid_dep_wait();  // yd comes from the previous kernel
  const int m = blockIdx.x;
  __shared__ const float* s_rows[32];
  __shared__ float s_w[32];
  __shared__ int s_m;
  if (threadIdx.x < 32) {
    // lane j looks at slot j; valid slots are compacted in slot order
    const int j = threadIdx.x;
    const bool valid = j < k && unsigned(sel[size_t(m) * sel_ld + j]) < unsigned(E);
    const unsigned mask = __ballot_sync(0xffffffffu, valid);
    if (valid) {
      const int pos = __popc(mask & ((1u << j) - 1u));
      s_rows[pos] = yd + (size_t(m) * k + j) * H;
      s_w[pos] = w[size_t(m) * w_ld + j];
    }
    if (j == 0) s_m = __popc(mask);
  }
  __syncthreads();
  for (int c4 = threadIdx.x * 4; c4 < H; c4 += blockDim.x * 4)
    *reinterpret_cast<float4*>(out + size_t(m) * out_ld + c4) = ordered_sum4<false>(s_rows, s_w, s_m, c4);
}

// combine_sel_kernel on bf16 rows: the same slot order and unfused fp32
// multiply and add, 8 columns per thread.
__global__ void __launch_bounds__(128) combine_sel_bf16_kernel(
    const __nv_bfloat16* __restrict__ yd, const int* __restrict__ sel, long long sel_ld,
    const float* __restrict__ w, long long w_ld, int k, int E, int H, float* __restrict__ out,
    long long out_ld) {
  tc::grid_dep_wait();  // yd comes from the previous kernel
  const int m = blockIdx.x;
  __shared__ const __nv_bfloat16* s_rows[32];
  __shared__ float s_w[32];
  __shared__ int s_m;
  if (threadIdx.x < 32) {
    const int j = threadIdx.x;
    const bool valid = j < k && unsigned(sel[size_t(m) * sel_ld + j]) < unsigned(E);
    const unsigned mask = __ballot_sync(0xffffffffu, valid);
    if (valid) {
      const int pos = __popc(mask & ((1u << j) - 1u));
      s_rows[pos] = yd + (size_t(m) * k + j) * H;
      s_w[pos] = w[size_t(m) * w_ld + j];
    }
    if (j == 0) s_m = __popc(mask);
  }
  __syncthreads();
  const int n = s_m;
  for (int c8 = threadIdx.x * 8; c8 < H; c8 += blockDim.x * 8) {
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    for (int i = 0; i < n; ++i) {
      const float wi = s_w[i];
      const uint4 v = *reinterpret_cast<const uint4*>(s_rows[i] + c8);
      const __nv_bfloat162* h2 = reinterpret_cast<const __nv_bfloat162*>(&v);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float2 f = __bfloat1622float2(h2[q]);
        acc[2 * q] = __fadd_rn(acc[2 * q], __fmul_rn(wi, f.x));
        acc[2 * q + 1] = __fadd_rn(acc[2 * q + 1], __fmul_rn(wi, f.y));
      }
    }
    float4* o = reinterpret_cast<float4*>(out + size_t(m) * out_ld + c8);
    o[0] = make_float4(acc[0], acc[1], acc[2], acc[3]);
    o[1] = make_float4(acc[4], acc[5], acc[6], acc[7]);
  }
}

// ---------------------------------------------------------------------------
// Peer-memory exchange: the router writes rows straight into the owning
// ranks' receive buffers and raises a per-source flag to the call id
// (route.cu); the kernels below consume and answer them.  Every wait polls a
// flag in this rank's own memory with acquire semantics at system scope and
// gives up after kWaitLimitNs (error flag, the block is then treated as
// empty), so no launch can hang on a peer that never writes.

__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
// Spin (one thread) until every flag[i], i < count, is >= call; each poll is
// an acquire load at system scope.  Bounded: returns false after the limit.
__device__ bool wait_flags(const unsigned* flag, int count, unsigned call, int* err, int code) {
  int i = 0;
  const uint64_t t0 = tc::globaltimer_ns();
  for (uint32_t spins = 0; i < count; ++spins) {
    if (ld_acquire_sys(flag + i) >= call) {
      ++i;
      continue;
    }
    __nanosleep(64);
    if ((spins & 255u) == 255u && tc::globaltimer_ns() - t0 > tc::kWaitLimitNs) {
      atomicCAS(err, 0, code);
      return false;
    }
  }
  return true;
}
__device__ __forceinline__ unsigned current_call(const unsigned* flags) {
  return *reinterpret_cast<const volatile unsigned*>(flags + kFlagEpoch) + 1u;
}

// One CTA per received row: wait for the source block's dispatch flag, then
// either mask the row (header / past the block's count: all ids -1) or claim
// its rows in the local experts' regions (scatter_sel_kernel's work).
__global__ void __launch_bounds__(128) ep_scatter_wait_kernel(
    unsigned* __restrict__ flags, uint8_t* __restrict__ recv, int n, int C, RowLayout L, int E,
    int T_pad, int* __restrict__ cursor, int* __restrict__ perm, uint8_t* __restrict__ xp,
    uint8_t* __restrict__ xp_atoms, int* __restrict__ err) {
  tc::grid_dep_launch();
  const int r = blockIdx.x;
  const int src = r / (C + 1), rr = r % (C + 1);
  __shared__ int s_valid;
  __shared__ int s_row[32];
  const unsigned call = current_call(flags);
  if (threadIdx.x == 0) {
    const bool ok = wait_flags(flags + kFlagDispatch + src, 1, call, err, 7);
    int count =
        ok ? *reinterpret_cast<const volatile int*>(recv + size_t(src) * (C + 1) * L.rb) : 0;
    if (count < 0 || count > C) {  // corrupted header: report, treat the block as empty
      if (rr == 0) atomicCAS(err, 0, 9);
      count = 0;
    }
    s_valid = rr >= 1 && rr - 1 < count;
  }
  __syncthreads();
  uint8_t* row = recv + size_t(r) * L.rb;
  int* sel = reinterpret_cast<int*>(row + L.sel_off());
  if (!s_valid) {
    if (threadIdx.x < L.k) sel[threadIdx.x] = -1;
    return;
  }
  if (threadIdx.x < L.k) {
    const int e = sel[threadIdx.x];
    int dst = -1;
    if (e >= E) {
      atomicCAS(err, 0, 4);
    } else if (e >= 0) {
      const int pos = atomicAdd(cursor + e, 1);
      if (pos < T_pad) {
        dst = e * T_pad + pos;
        perm[dst] = r * L.k + threadIdx.x;
      } else {
        atomicCAS(err, 0, 5);
      }
    }
    s_row[threadIdx.x] = dst;
  }
  __syncthreads();
  const int q16 = L.H / 32, kc = L.H / 128;
  for (int j = 0; j < L.k; ++j) {
    const int dst = s_row[j];
    if (dst < 0) continue;
    for (int i = threadIdx.x; i < q16; i += blockDim.x)
      reinterpret_cast<uint4*>(xp + size_t(dst) * (L.H / 2))[i] = reinterpret_cast<const uint4*>(row)[i];
    for (int i = threadIdx.x; i < kc; i += blockDim.x)
      *reinterpret_cast<uint32_t*>(xp_atoms + (size_t(dst >> 5) * kc + i) * 512 + (dst & 31) * 16) =
          reinterpret_cast<const uint32_t*>(row + L.sc_off())[i];
  }
}

// Weighted sum of each valid received row's local slots (combine_sel_kernel's
// arithmetic) written straight into the source rank's return buffer; the
// last CTA raises this rank's return flag at every source.
__global__ void __launch_bounds__(128) ep_combine_return_kernel(
    const EpTable* __restrict__ table, unsigned* __restrict__ flags, const float* __restrict__ yd,
    const uint8_t* __restrict__ recv, int rank, int n, int C, RowLayout L, int E,
    int* __restrict__ ws_counters, int n_counters, int* __restrict__ err) {
  tc::grid_dep_wait();  // yd comes from the expert kernel
  const unsigned call = current_call(flags);
  const int R = n * (C + 1);
  __shared__ const float* s_rows[32];
  __shared__ float s_w[32];
  __shared__ int s_m;
  for (int r = blockIdx.x; r < R; r += gridDim.x) {
    if (threadIdx.x < 32) {
      const uint8_t* row = recv + size_t(r) * L.rb;
      const int j = threadIdx.x;
      const bool valid =
          j < L.k && unsigned(reinterpret_cast<const int*>(row + L.sel_off())[j]) < unsigned(E);
      const unsigned mask = __ballot_sync(0xffffffffu, valid);
      if (valid) {
        const int pos = __popc(mask & ((1u << j) - 1u));
        s_rows[pos] = yd + (size_t(r) * L.k + j) * L.H;
        s_w[pos] = reinterpret_cast<const float*>(row + L.w_off())[j];
      }
      if (j == 0) s_m = __popc(mask);
    }
    __syncthreads();
    const int m = s_m;
    if (m > 0) {  // header, unused or not-for-us rows send nothing
      const int src = r / (C + 1), rr = r % (C + 1);
      float* dst = table->ret[src] + (size_t(rank) * (C + 1) + rr) * L.H;
      for (int c4 = threadIdx.x * 4; c4 < L.H; c4 += blockDim.x * 4)
        *reinterpret_cast<float4*>(dst + c4) = ordered_sum4<false>(s_rows, s_w, m, c4);
    }
    __syncthreads();
  }
  // Release: every thread's stores precede thread 0's fence (bar.sync); a
  // GPU-scope fence orders them before this CTA's count, and the last CTA's
  // system-scope fence (cumulative over everything that happened before it on
  // this GPU) orders them all before the flags the peers poll.  One system
  // fence per call instead of one per CTA.
  if (threadIdx.x != 0) return;
  __threadfence();
  if (atomicAdd(flags + kFlagDone + 1, 1u) != gridDim.x - 1) return;
  // the expert launch and the scatter are complete (programmatic wait at the
  // top): their counters start the next call at zero
  for (int i = 0; i < n_counters; ++i) ws_counters[i] = 0;
  __threadfence_system();
  for (int d = 0; d < n; ++d) tc::st_relaxed_sys(table->flags[d] + kFlagReturn + rank, call);
}

// out[t] = sum over ranks d (ascending) of the row that rank d returned for
// token t; waits for every rank's return flag first.  The last CTA closes the
// call: epoch + 1.
__global__ void __launch_bounds__(128) ep_unpack_wait_kernel(
    unsigned* __restrict__ flags, const float* __restrict__ ret, const int* __restrict__ pack_pos,
    int T, int n, int C, int H, float* __restrict__ out, int* __restrict__ err) {
  const unsigned call = current_call(flags);
  __shared__ const float* s_rows[kEpMaxRanks];
  __shared__ int s_m;
  const int t = blockIdx.x;
  // thread d waits for rank d's return (in parallel), then lanes compact rows
  const bool ok = __syncthreads_and(
      threadIdx.x >= n || wait_flags(flags + kFlagReturn + threadIdx.x, 1, call, err, 8));
  if (threadIdx.x < 32) {
    int base = 0;
    for (int d0 = 0; d0 < n; d0 += 32) {
      const int d = d0 + threadIdx.x;
      const int pos = (ok && t < T && d < n) ? pack_pos[t * n + d] : -1;
      const unsigned mask = __ballot_sync(0xffffffffu, pos >= 0);
      if (pos >= 0)
        s_rows[base + __popc(mask & ((1u << threadIdx.x) - 1u))] = ret + (size_t(d) * (C + 1) + 1 + pos) * H;
      base += __popc(mask);
    }
    if (threadIdx.x == 0) s_m = base;
  }
  __syncthreads();
  if (t < T)
    for (int c4 = threadIdx.x * 4; c4 < H; c4 += blockDim.x * 4)
      *reinterpret_cast<float4*>(out + size_t(t) * H + c4) = ordered_sum4<true>(s_rows, nullptr, s_m, c4);
  __syncthreads();
  if (threadIdx.x == 0 && atomicAdd(flags + kFlagDone + 2, 1u) == gridDim.x - 1) {
    // last CTA of the call's last kernel: clear the per-call counters for the
    // next call (nothing of this call reads them any more), then close it
    for (int i = kFlagZeroFirst; i < kFlagWords; ++i) flags[i] = 0u;
    __threadfence();
    atomicAdd(flags + kFlagEpoch, 1u);
  }
}

}  // namespace

cudaError_t launch_ep_scatter_wait(const EpTable* table, unsigned* flags, uint8_t* recv, int rank,
                                   int n, int C, int H, int k, int E, int T_pad, int* cursor,
                                   int* perm, uint8_t* xp, uint8_t* xp_atoms, int* err,
                                   cudaStream_t stream) {
  (void)table;
  (void)rank;
  RowLayout L{H, k, ep_row_bytes(H, k)};
  ep_scatter_wait_kernel<<<n * (C + 1), 128, 0, stream>>>(flags, recv, n, C, L, E, T_pad, cursor,
                                                          perm, xp, xp_atoms, err);
  return cudaGetLastError();
}

cudaError_t launch_ep_combine_return(const EpTable* table, unsigned* flags, const float* yd,
                                     const uint8_t* recv, int rank, int n, int C, int H, int k,
                                     int E, int* ws_counters, int n_counters, int* err,
                                     cudaStream_t stream) {
  RowLayout L{H, k, ep_row_bytes(H, k)};
  const int R = n * (C + 1);
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(R);  // one received row per CTA
  cfg.blockDim = dim3(128);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, ep_combine_return_kernel, table, flags, yd, recv, rank, n, C, L,
                            E, ws_counters, n_counters, err);
}

cudaError_t launch_ep_unpack_wait(unsigned* flags, const float* ret, const int* pack_pos, int T,
                                  int n, int C, int H, float* out, int* err, cudaStream_t stream) {
  ep_unpack_wait_kernel<<<T > 0 ? T : 1, 128, 0, stream>>>(flags, ret, pack_pos, T, n, C, H, out,
                                                           err);
  return cudaGetLastError();
}

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

cudaError_t launch_ep_mask_recv(int n_ranks, int C, int H, int k, uint8_t* recv, int* err,
                                cudaStream_t stream) {
  RowLayout L{H, k, ep_row_bytes(H, k)};
  const long long rows = (long long)n_ranks * (C + 1);
  int blocks = int((rows + 255) / 256);
  if (blocks < 1) blocks = 1;
  ep_mask_recv_kernel<<<blocks, 256, 0, stream>>>(n_ranks, C, L, recv, err);
  return cudaGetLastError();
}

cudaError_t launch_ep_unpack(const float* ret, const int* pack_pos, int T, int n_ranks, int C,
                             int H, float* out, cudaStream_t stream) {
  if (T == 0) return cudaSuccess;
  ep_unpack_kernel<<<T, 128, 0, stream>>>(ret, pack_pos, T, n_ranks, C, H, out);
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

cudaError_t launch_combine_sel_bf16(const __nv_bfloat16* yd, const int* sel, long long sel_ld,
                                    const float* w, long long w_ld, int R, int k, int E, int H,
                                    float* out, long long out_ld, cudaStream_t stream) {
  if (R == 0) return cudaSuccess;
  if (H % 8 != 0) return cudaErrorInvalidValue;
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(R);
  cfg.blockDim = dim3(128);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, combine_sel_bf16_kernel, yd, sel, sel_ld, w, w_ld, k, E, H, out,
                            out_ld);
}

cudaError_t launch_combine_sel(const float* yd, const int* sel, long long sel_ld, const float* w,
                               long long w_ld, int R, int k, int E, int H, float* out,
                               long long out_ld, cudaStream_t stream) {
  if (R == 0) return cudaSuccess;
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(R);
  cfg.blockDim = dim3(128);
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
