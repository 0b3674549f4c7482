// route.cu — device-side router for the fused decode MoE layer.
//
// Fulfils the reference's unimplemented K1 stub (src/kernels/k1_router_topk_sort.cu)
// and replaces the host round trip of model_runner_v2 (router GEMM
// runtime/model_runner_v2.py:186-188, softmax/top-k/renorm :189-192,
// ``topi.view(-1).tolist()`` :194 and the per-(token, slot) pointer lists
// :197-202): logits, top-k, weights and the per-expert work lists all stay on
// the device, so gate -> experts needs no host synchronisation.
//
// Logits are bit-reproducible: every 32-element block product is an exact
// integer times a power of two, accumulated in fp64 in a fixed order (lane l
// sums blocks l, l+32, ... ascending; then an xor-butterfly 16,8,4,2,1) and
// rounded once to fp32.  oracle/mxfp4.py:router_logits uses the same order,
// so the top-k indices match the oracle bit for bit.  Ties between equal
// logits go to the lower expert index.
#include "mx_common.cuh"
#include "work.cuh"
#include "tc_ptx.cuh"
#include "tmap.cuh"
#include "route_common.cuh"

namespace mfi {

constexpr int kRouteThreads = 512;
constexpr int kMaxE = kRouteMaxE;

template <int kMaxBlk>
__global__ void __launch_bounds__(kRouteThreads) route_kernel(RouteArgs a) {
  __shared__ float s_logit[kMaxE];
  __shared__ unsigned s_last;
  __shared__ __align__(16) uint8_t s_xq[kMaxBlk * 32 * 16];
  __shared__ __align__(16) uint8_t s_xsc[kMaxBlk * 32];
  // the expert kernels after this one may start their prologue now
  tc::grid_dep_launch();
  const int t = blockIdx.x;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int nwarp = kRouteThreads / 32;
  const int nb = a.H >> 5;

  // ---- quantise token t (the reference's prequant, fused) -------------------
  // one thread per 8 elements, a quad per 32-element block (quant_group8);
  // with a norm weight every warp first computes the row's RMS factor (the
  // same value in every warp)
  const float rms_r = a.norm_w ? warp_rms_inv(a, t, lane) : 1.0f;
  for (int base = warp * 32; base < (a.H >> 3); base += kRouteThreads) {
    const int c8 = base + lane;
    const bool live = c8 < (a.H >> 3);
    float v[8];
    if (live) {
      const uint4 raw = *reinterpret_cast<const uint4*>(
          reinterpret_cast<const __nv_bfloat16*>(a.x) + long(t) * a.H + c8 * 8);
      const __nv_bfloat162* h2 = reinterpret_cast<const __nv_bfloat162*>(&raw);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 f = __bfloat1622float2(h2[i]);
        v[2 * i] = f.x;
        v[2 * i + 1] = f.y;
      }
      if (a.norm_w) rms_apply8(a, c8 * 8, rms_r, v);
    } else {
#pragma unroll
      for (int i = 0; i < 8; ++i) v[i] = 0.0f;
    }
    BlockScale bs;
    const uint32_t word = quant_group8(v, bs);
    if (live) {
      reinterpret_cast<uint32_t*>(s_xq)[c8] = word;
      if ((c8 & 3) == 0) s_xsc[c8 >> 2] = bs.code;
    }
  }
  __syncthreads();
  for (int i = threadIdx.x; i < (a.H >> 3); i += kRouteThreads)
    reinterpret_cast<uint32_t*>(a.xq + long(t) * (a.H >> 1))[i] = reinterpret_cast<uint32_t*>(s_xq)[i];
  for (int i = threadIdx.x; i < nb; i += kRouteThreads) a.xsc[long(t) * nb + i] = s_xsc[i];

  // ---- logits for token t --------------------------------------------------
  // Each lane owns blocks b = lane + 32*j: the token's nibbles for them are
  // expanded to int8 once; the router rows of 4 experts per warp are in
  // flight together.
  uint32_t xa8[kMaxBlk][8];
  int xs[kMaxBlk];
#pragma unroll
  for (int j = 0; j < kMaxBlk; ++j) {
    const int b = lane + 32 * j;
    if (b < nb) {
      const uint4 q = reinterpret_cast<const uint4*>(s_xq)[b];
      nib8_to_i8(q.x, xa8[j][0], xa8[j][1]);
      nib8_to_i8(q.y, xa8[j][2], xa8[j][3]);
      nib8_to_i8(q.z, xa8[j][4], xa8[j][5]);
      nib8_to_i8(q.w, xa8[j][6], xa8[j][7]);
      xs[j] = s_xsc[b];
    }
  }
  constexpr int kU = kMaxBlk <= 2 ? 8 : 4;  // experts in flight per warp
  for (int e0 = warp; e0 < a.E; e0 += kU * nwarp) {
    uint4 wv[kU][kMaxBlk];
    int ws[kU][kMaxBlk];
#pragma unroll
    for (int u = 0; u < kU; ++u) {
      const int e = e0 + u * nwarp;
#pragma unroll
      for (int j = 0; j < kMaxBlk; ++j) {
        const int b = lane + 32 * j;
        if (e < a.E && b < nb) {
          wv[u][j] = ldg_u4(a.wr + long(e) * (a.H >> 1) + b * 16);
          ws[u][j] = a.sr[long(e) * nb + b];
        }
      }
    }
    double acc[kU];
#pragma unroll
    for (int u = 0; u < kU; ++u) {
      const int e = e0 + u * nwarp;
      acc[u] = 0.0;
#pragma unroll
      for (int j = 0; j < kMaxBlk; ++j) {
        const int b = lane + 32 * j;
        if (e < a.E && b < nb) {
          const int s = block_dot_pre(wv[u][j], xa8[j]);
          acc[u] += double(s) * exp2i_d(xs[j] + ws[u][j] - 256);
        }
      }
    }
    // xor-butterfly over the warp for all kU experts at once: at offset `off`
    // each lane keeps half of its values and adds the partner's copy, so every
    // value is the same pairwise sum as a per-expert butterfly 16,8,4,2,1
    // (bit-identical), with kU-1 + 5 - log2(kU) shuffles instead of 5 kU.
    int n = kU;
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) {
      if (n > 1) {
        const bool upper = (lane & off) != 0;
        const int h = n >> 1;
#pragma unroll
        for (int i = 0; i < kU / 2; ++i) {
          if (i < h) {
            const double send = upper ? acc[i] : acc[i + h];
            const double keep = upper ? acc[i + h] : acc[i];
            acc[i] = keep + __shfl_xor_sync(0xffffffffu, send, off);
          }
        }
        n = h;
      } else {
        acc[0] += __shfl_xor_sync(0xffffffffu, acc[0], off);
      }
    }
    // after log2(kU) halving steps lane l holds expert index (l >> (5 - log2 kU))
    constexpr int kLog = kU == 8 ? 3 : (kU == 4 ? 2 : (kU == 2 ? 1 : 0));
    if ((lane & ((32 >> kLog) - 1)) == 0) {
      const int u = lane >> (5 - kLog);
      const int e = e0 + u * nwarp;
      if (e < a.E) s_logit[e] = float(acc[0]);
    }
  }
  __syncthreads();
  if (a.logit_bias) {
    for (int e = threadIdx.x; e < a.E; e += blockDim.x)
      s_logit[e] = __fadd_rn(s_logit[e], a.logit_bias[e]);
    __syncthreads();
  }
  if (a.logits)
    for (int e = threadIdx.x; e < a.E; e += blockDim.x) a.logits[long(t) * a.E + e] = s_logit[e];

  // ---- top-k ----------------------------------------------------------------
  // Thread e computes the rank of expert e under the order (logit desc,
  // index asc); rank < k places it in the top-k at that position.
  __shared__ int s_sel[32];
  __shared__ float s_selv[32];
  for (int e = threadIdx.x; e < a.E; e += kRouteThreads) {
    const float v = s_logit[e];
    int rank = 0;
    for (int j = 0; j < a.E; ++j) rank += better(s_logit[j], j, v, e) ? 1 : 0;
    if (rank < a.k) {
      s_sel[rank] = e;
      s_selv[rank] = v;
    }
  }
  __syncthreads();
  __shared__ int s_row[32];
  if (warp == 0) {
    // weights: exp(l - max) over the selected, normalised by their sum
    const float mx = s_selv[0];
    const float p = (lane < a.k) ? expf(s_selv[lane < a.k ? lane : 0] - mx) : 0.f;
    float sum = 0.f;
    for (int j = 0; j < a.k; ++j) sum = __fadd_rn(sum, __shfl_sync(0xffffffffu, p, j));
    if (lane < a.k) {
      a.topi[long(t) * a.k + lane] = s_sel[lane];
      a.topw[long(t) * a.k + lane] = __fdiv_rn(p, sum);
      if (a.xp) {
        // claim a row in each selected expert's region
        const int e = s_sel[lane];
        const int pos = atomicAdd(a.cursor + e, 1);
        int row = -1;
        if (pos < a.T_pad) {
          row = e * a.T_pad + pos;
          a.perm[row] = t * a.k + lane;
        } else if (a.err) {
          atomicCAS(a.err, 0, 5);  // cursors not zero at entry
        }
        s_row[lane] = row;
      }
    }
  }
  if (a.xp) {
    // copy the quantised row into each claimed row, scales into the atoms
    __syncthreads();
    const int q16 = a.H >> 5;  // uint4 per row
    for (int i = threadIdx.x; i < a.k * q16; i += kRouteThreads) {
      const int j = i / q16, c = i % q16;
      if (s_row[j] < 0) continue;
      reinterpret_cast<uint4*>(a.xp + size_t(s_row[j]) * (a.H >> 1))[c] =
          reinterpret_cast<const uint4*>(s_xq)[c];
    }
    const int kc = a.H >> 7;  // atoms per row
    for (int i = threadIdx.x; i < a.k * kc; i += kRouteThreads) {
      const int j = i / kc, c = i % kc;
      const int row = s_row[j];
      if (row < 0) continue;
      *reinterpret_cast<uint32_t*>(a.xp_atoms + (size_t(row >> 5) * kc + c) * 512 + (row & 31) * 16) =
          reinterpret_cast<const uint32_t*>(s_xsc)[c];
    }
  }

  // ---- last CTA builds the per-expert work lists ----------------------------
  // (CUDA-core path only; the tensor-core kernels rebuild their chunk table
  // from the per-expert cursors themselves)
  if (!a.g_gu) return;
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) s_last = (atomicAdd(a.done, 1u) == unsigned(gridDim.x) - 1u);
  __syncthreads();
  if (!s_last) return;
  __threadfence();

  // Work lists: per active expert one gate group, one up group and one down
  // group.  The position of an entry inside its expert's list comes from a
  // shared-memory cursor; the order does not affect any result because every
  // entry owns its output row.
  __shared__ int s_cnt[kMaxE];
  __shared__ int s_off[kMaxE];
  __shared__ int s_act[kMaxE];  // active index of expert e, or -1
  __shared__ int s_cur[kMaxE];
  __shared__ int s_cbase[kMaxE];  // first chunk of expert e
  const int P = a.T * a.k;
  for (int e = threadIdx.x; e < a.E; e += blockDim.x) { s_cnt[e] = 0; s_cur[e] = 0; }
  __syncthreads();
  for (int i = threadIdx.x; i < P; i += blockDim.x) atomicAdd(&s_cnt[__ldcg(a.topi + i)], 1);
  __syncthreads();
  if (warp == 0) {
    // exclusive scans of counts and of "active" flags over E <= 256 experts
    int run_off = 0, run_act = 0, run_ch = 0;
    for (int e0 = 0; e0 < a.E; e0 += 32) {
      const int e = e0 + lane;
      const int c = e < a.E ? s_cnt[e] : 0;
      const int nch = (c + 31) / 32;
      int inc = c, act = c > 0 ? 1 : 0, ch = nch;
#pragma unroll
      for (int off = 1; off < 32; off <<= 1) {
        const int v = __shfl_up_sync(0xffffffffu, inc, off);
        const int w = __shfl_up_sync(0xffffffffu, act, off);
        const int x = __shfl_up_sync(0xffffffffu, ch, off);
        if (lane >= off) { inc += v; act += w; ch += x; }
      }
      if (e < a.E) {
        s_off[e] = run_off + inc - c;
        s_act[e] = c > 0 ? run_act + act - 1 : -1;
        s_cbase[e] = run_ch + ch - nch;
      }
      run_off += __shfl_sync(0xffffffffu, inc, 31);
      run_act += __shfl_sync(0xffffffffu, act, 31);
      run_ch += __shfl_sync(0xffffffffu, ch, 31);
    }
    if (lane == 0) {
      *a.n_gu = 2 * run_act;
      *a.n_dn = run_act;
      *a.n_active = run_act;
      if (a.n_chunks) *a.n_chunks = run_ch;
      *a.done = 0u;  // ready for the next call
    }
  }
  __syncthreads();
  if (a.cursor)
    for (int e = threadIdx.x; e < a.E; e += kRouteThreads) a.cursor[e] = 0;  // ready for next call
  const long gstride = long(a.Mi) * (a.H >> 1), gsstride = long(a.Mi) * (a.H >> 5);
  const long dstride = long(a.H) * (a.Mi >> 1), dsstride = long(a.H) * (a.Mi >> 5);
  for (int e = threadIdx.x; e < a.E; e += blockDim.x) {
    const int ai = s_act[e];
    if (ai < 0) continue;
    const int first = s_off[e], cnt = s_cnt[e];
    if (a.g_gu) {
      GroupDesc g;
      g.first = first; g.count = cnt;
      g.wp = a.gate_wp + e * gstride; g.wsc = a.gate_sc + e * gsstride;
      a.g_gu[2 * ai] = g;
      g.first = P + first;
      g.wp = a.up_wp + e * gstride; g.wsc = a.up_sc + e * gsstride;
      a.g_gu[2 * ai + 1] = g;
      g.first = first;
      g.wp = a.down_wp + e * dstride; g.wsc = a.down_sc + e * dsstride;
      a.g_dn[ai] = g;
    }
    if (a.chunks) {
      for (int c = 0; c * 32 < cnt; ++c) {
        ChunkDesc cd;
        cd.expert = e;
        cd.count = min(32, cnt - 32 * c);
        cd.row0 = e * a.T_pad + 32 * c;
        cd.pad = 0;
        a.chunks[s_cbase[e] + c] = cd;
        for (int r = cd.count; r < 32; ++r) a.perm[cd.row0 + r] = -1;
      }
    }
  }
  for (int i = threadIdx.x; i < P; i += blockDim.x) {
    if (!a.e_gu) continue;
    const int e = __ldcg(a.topi + i);
    const int pil = atomicAdd(&s_cur[e], 1);  // position in expert e's list
    const int pos = s_off[e] + pil;
    EntryDesc d;
    d.pad = 0;
    d.act_row = i / a.k;
    d.out_off = (long long)i * 2 * a.Mi;
    a.e_gu[pos] = d;
    d.out_off += a.Mi;
    a.e_gu[P + pos] = d;
    d.act_row = i;
    d.out_off = (long long)i * a.H;
    a.e_dn[pos] = d;
  }
}

// ---------------------------------------------------------------------------
// Cluster router (no work lists): one thread-block cluster per token, CTA r
// of the cluster owns experts [32r, 32r + 32).  Each CTA stages its 32 router
// rows in shared memory with one bulk copy issued at entry (before the expert
// launches that start under programmatic dependent launch begin streaming
// their weights), quantises the token (redundantly: 4 KB of input), computes
// its 32 logits with the same per-lane order and butterfly as route_kernel,
// and stores them into the leader CTA's shared memory through distributed
// shared memory.  The leader then runs top-k, the weights and the expert-row
// claims.  Logits are bit-identical to route_kernel's.
constexpr int kClusterThreads = 256;
constexpr int kExpertsPerCta = 32;  // most experts per CTA (clusters of <= 8 for 256 experts)

__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ void cluster_arrive_release() {
  asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait_acquire() {
  asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// Store a float into CTA `rank`'s shared memory at the address of `local`.
__device__ __forceinline__ void st_cluster_f32(const void* local, uint32_t rank, float v) {
  uint32_t remote;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;"
               : "=r"(remote)
               : "r"(tc::smem_u32(local)), "r"(rank));
  asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(remote), "f"(v) : "memory");
}

__device__ __forceinline__ int ep_row_bytes_dev(int H, int k) {
  return (H / 2 + H / 32 + 16 + 8 * k + 15) / 16 * 16;
}

// Completion of an expert-parallel dispatch, run by every thread of each
// cluster leader after its rows are written: the last leader writes each
// destination block's header (row count) and raises this rank's dispatch
// flag at every destination to the call id.
__device__ void ep_finish_dispatch(const EpDispatch& ep, int H, int k, int n_leaders,
                                   unsigned call) {
  __shared__ int s_last;
  __syncthreads();  // every thread's row stores precede thread 0's fence
  if (threadIdx.x == 0) {
    // GPU-scope release per leader; the last leader's system-scope fences
    // below are cumulative over every leader's rows
    __threadfence();
    s_last = atomicAdd(ep.flags + kFlagDone + 0, 1u) == unsigned(n_leaders - 1);
    if (s_last) __threadfence_system();  // the other leaders' rows and counts
  }
  __syncthreads();
  if (!s_last) return;
  if (threadIdx.x < ep.n) {
    const int d = threadIdx.x;
    const int rb = ep_row_bytes_dev(H, k);
    const int cnt = int(*reinterpret_cast<volatile unsigned*>(ep.flags + kFlagCounts + d));
    *reinterpret_cast<volatile int*>(ep.table->recv[d] + size_t(ep.rank) * (ep.C + 1) * rb) = cnt;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence_system();  // headers (all threads) before the flags
    for (int d = 0; d < ep.n; ++d)
      tc::st_relaxed_sys(ep.table->flags[d] + kFlagDispatch + ep.rank, call);
  }
}

// kEPC experts per CTA: 16 (8-CTA clusters for 128 experts: each CTA loads
// and reduces half as many router rows) or 32 (4-CTA clusters).
template <int kMaxBlk, int kEPC>
__global__ void __launch_bounds__(kClusterThreads) route_cluster_kernel(RouteArgs a, int n_split) {
  tc::grid_dep_launch();
  extern __shared__ __align__(128) uint8_t s_w[];  // [32][H/2] router rows of this CTA
  __shared__ float s_logit[kMaxE];
  __shared__ __align__(16) uint8_t s_xq[kMaxBlk * 32 * 16];
  __shared__ __align__(16) uint8_t s_xsc[kMaxBlk * 32];
  __shared__ __align__(16) uint8_t s_ws[kEPC * kMaxBlk * 32];
  __shared__ __align__(8) uint64_t s_bar;
  const uint32_t crank = cluster_ctarank();
  const int t = blockIdx.x / n_split;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  // expert parallelism: the call id this dispatch belongs to (the epoch only
  // moves at the end of the call); a launch for T = 0 tokens has one cluster
  // that only joins the completion
  const unsigned ep_call =
      a.ep.table ? *reinterpret_cast<volatile unsigned*>(a.ep.flags + kFlagEpoch) + 1u : 0u;
  if (a.ep.table && t >= a.ep.T) {
    if (crank == 0) ep_finish_dispatch(a.ep, a.H, a.k, int(gridDim.x) / n_split, ep_call);
    return;
  }
  const int nb = a.H >> 5;
  const int e_begin = int(crank) * kEPC;
  const int n_e = min(kEPC, a.E - e_begin);
  const uint32_t w_bytes = uint32_t(n_e) * uint32_t(a.H >> 1);

  // router rows first: their loads should not queue behind the weight
  // prefetch of the expert kernels
  const uint32_t sc_bytes = uint32_t(n_e) * uint32_t(nb);
  const uint8_t* sc_src = a.sr + size_t(e_begin) * nb;
  const bool sc_bulk = (sc_bytes % 16) == 0 && (reinterpret_cast<uintptr_t>(sc_src) % 16) == 0;
  if (threadIdx.x == 0) {
    tc::mbar_init(&s_bar, 1);
    tc::fence_mbar_init();
    tc::cta_abort_init();
    if (n_e > 0) {
      tc::mbar_expect_tx(&s_bar, w_bytes + (sc_bulk ? sc_bytes : 0u));
      tc::bulk_load(s_w, a.wr + size_t(e_begin) * (a.H >> 1), w_bytes, &s_bar);
      if (sc_bulk) tc::bulk_load(s_ws, sc_src, sc_bytes, &s_bar);
    }
  }
  if (!sc_bulk)
    for (int i = threadIdx.x; i < n_e * nb; i += kClusterThreads) s_ws[i] = sc_src[i];
  // the leader's logits start at 0 so that a failed peer leaves finite values
  if (crank == 0)
    for (int e = threadIdx.x; e < a.E; e += kClusterThreads) s_logit[e] = 0.0f;
  cluster_arrive_release();  // every CTA of the cluster has started (and the init is ordered)

  // ---- quantise token t (RMS-normalised first when a.norm_w is set) --------
  const float rms_r = a.norm_w ? warp_rms_inv(a, t, lane) : 1.0f;
  for (int base = warp * 32; base < (a.H >> 3); base += kClusterThreads) {
    const int c8 = base + lane;
    const bool live = c8 < (a.H >> 3);
    float v[8];
    if (live) {
      const uint4 raw = *reinterpret_cast<const uint4*>(
          reinterpret_cast<const __nv_bfloat16*>(a.x) + long(t) * a.H + c8 * 8);
      const __nv_bfloat162* h2 = reinterpret_cast<const __nv_bfloat162*>(&raw);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 f = __bfloat1622float2(h2[i]);
        v[2 * i] = f.x;
        v[2 * i + 1] = f.y;
      }
      if (a.norm_w) rms_apply8(a, c8 * 8, rms_r, v);
    } else {
#pragma unroll
      for (int i = 0; i < 8; ++i) v[i] = 0.0f;
    }
    BlockScale bs;
    const uint32_t word = quant_group8(v, bs);
    if (live) {
      reinterpret_cast<uint32_t*>(s_xq)[c8] = word;
      if ((c8 & 3) == 0) s_xsc[c8 >> 2] = bs.code;
    }
  }
  __syncthreads();
  if (crank == 0 && a.xq) {
    for (int i = threadIdx.x; i < (a.H >> 3); i += kClusterThreads)
      reinterpret_cast<uint32_t*>(a.xq + long(t) * (a.H >> 1))[i] = reinterpret_cast<uint32_t*>(s_xq)[i];
    for (int i = threadIdx.x; i < nb; i += kClusterThreads) a.xsc[long(t) * nb + i] = s_xsc[i];
  }

  // ---- 32 logits: warp w owns local experts w, w+8, w+16, w+24 --------------
  const bool have_w = n_e > 0 && tc::mbar_wait(&s_bar, 0, a.err, 6);
  // failed: the router rows may still be landing; wait for them before exit
  if (n_e > 0 && !have_w && threadIdx.x == 0) tc::mbar_wait(&s_bar, 0, nullptr, 0);
  if (warp == 0 && a.pf_bytes) {
    // this token's inputs are in: start streaming the expert weights that the
    // next kernel reads first into L2 (speculative: the routing is not known)
    const unsigned long long per = ((a.pf_bytes + gridDim.x - 1) / gridDim.x + 4095) & ~4095ull;
    const unsigned long long lo = per * blockIdx.x;
    const unsigned long long hi = min(lo + per, a.pf_bytes);
    for (unsigned long long off = lo + lane * 32768ull; off < hi; off += 32 * 32768ull)
      tc::prefetch_l2(a.pf_base + off, uint32_t(min(32768ull, hi - off)));
  }
  uint32_t xa8[kMaxBlk][8];
  int xs[kMaxBlk];
#pragma unroll
  for (int j = 0; j < kMaxBlk; ++j) {
    const int b = lane + 32 * j;
    if (b < nb) {
      const uint4 q = reinterpret_cast<const uint4*>(s_xq)[b];
      nib8_to_i8(q.x, xa8[j][0], xa8[j][1]);
      nib8_to_i8(q.y, xa8[j][2], xa8[j][3]);
      nib8_to_i8(q.z, xa8[j][4], xa8[j][5]);
      nib8_to_i8(q.w, xa8[j][6], xa8[j][7]);
      xs[j] = s_xsc[b];
    }
  }
  constexpr int kWarps = kClusterThreads / 32;
  constexpr int kU = kEPC / kWarps;  // experts per warp
  static_assert(kU == 2 || kU == 4, "experts per warp");
  constexpr int kLog = kU == 4 ? 2 : 1;
  double acc[kU];
#pragma unroll
  for (int u = 0; u < kU; ++u) {
    const int el = warp + u * kWarps;
    acc[u] = 0.0;
#pragma unroll
    for (int j = 0; j < kMaxBlk; ++j) {
      const int b = lane + 32 * j;
      if (have_w && el < n_e && b < nb) {
        const uint4 wv = *reinterpret_cast<const uint4*>(s_w + size_t(el) * (a.H >> 1) + b * 16);
        const int sc = s_ws[el * nb + b];
        const int sdot = block_dot_pre(wv, xa8[j]);
        acc[u] += double(sdot) * exp2i_d(xs[j] + sc - 256);
      }
    }
  }
  // reduce-scatter butterfly (same pairwise sums as route_kernel)
  int n = kU;
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) {
    if (n > 1) {
      const bool upper = (lane & off) != 0;
      const int h = n >> 1;
#pragma unroll
      for (int i = 0; i < kU / 2; ++i) {
        if (i < h) {
          const double send = upper ? acc[i] : acc[i + h];
          const double keep = upper ? acc[i + h] : acc[i];
          acc[i] = keep + __shfl_xor_sync(0xffffffffu, send, off);
        }
      }
      n = h;
    } else {
      acc[0] += __shfl_xor_sync(0xffffffffu, acc[0], off);
    }
  }
  cluster_wait_acquire();  // the leader has started (its shared memory exists)
  // after kLog halving steps lane l holds value l >> (5 - kLog)
  if ((lane & ((32 >> kLog) - 1)) == 0) {
    const int el = warp + (lane >> (5 - kLog)) * kWarps;
    if (have_w && el < n_e) st_cluster_f32(&s_logit[e_begin + el], 0, float(acc[0]));
  }
  cluster_arrive_release();
  cluster_wait_acquire();
  if (crank != 0) return;

  if (a.logit_bias) {
    for (int e = threadIdx.x; e < a.E; e += kClusterThreads)
      s_logit[e] = __fadd_rn(s_logit[e], a.logit_bias[e]);
    __syncthreads();
  }
  if (a.logits)
    for (int e = threadIdx.x; e < a.E; e += kClusterThreads) a.logits[long(t) * a.E + e] = s_logit[e];


  // ---- top-k, weights, expert-row claims (leader) ----------------------------
  __shared__ int s_sel[32];
  __shared__ float s_selv[32];
  for (int e = threadIdx.x; e < a.E; e += kClusterThreads) {
    const float v = s_logit[e];
    int rank = 0;
    for (int j = 0; j < a.E; ++j) rank += better(s_logit[j], j, v, e) ? 1 : 0;
    if (rank < a.k) {
      s_sel[rank] = e;
      s_selv[rank] = v;
    }
  }
  __syncthreads();
  __shared__ int s_row[32];
  __shared__ float s_tw[32];
  if (warp == 0) {
    const float mx = s_selv[0];
    const float p = (lane < a.k) ? expf(s_selv[lane < a.k ? lane : 0] - mx) : 0.f;
    float sum = 0.f;
    for (int j = 0; j < a.k; ++j) sum = __fadd_rn(sum, __shfl_sync(0xffffffffu, p, j));
    if (lane < a.k) {
      const float wgt = __fdiv_rn(p, sum);
      a.topi[long(t) * a.k + lane] = s_sel[lane];
      a.topw[long(t) * a.k + lane] = wgt;
      s_tw[lane] = wgt;
      if (a.slot_pos) a.slot_pos[long(t) * a.k + lane] = atomicAdd(a.cursor + s_sel[lane], 1);
      if (a.xp) {
        const int e = s_sel[lane];
        const int pos = atomicAdd(a.cursor + e, 1);
        int row = -1;
        if (pos < a.T_pad) {
          row = e * a.T_pad + pos;
          a.perm[row] = t * a.k + lane;
        } else if (a.err) {
          atomicCAS(a.err, 0, 5);  // cursors not zero at entry
        }
        s_row[lane] = row;
      }
    }
  }
  if (a.ep.table) {
    // ---- expert parallelism: send the token to every rank owning one of its
    // experts, straight into that rank's receive buffer (peer memory) --------
    const EpDispatch& ep = a.ep;
    __shared__ int s_dpos[kEpMaxRanks];
    __syncthreads();
    if (threadIdx.x < ep.n) {
      const int d = threadIdx.x;
      bool any = false;
      for (int j = 0; j < a.k; ++j) any |= (s_sel[j] / ep.el) == d;
      const int pos = any ? int(atomicAdd(ep.flags + kFlagCounts + d, 1u)) : -1;
      s_dpos[d] = pos;
      ep.pack_pos[long(t) * ep.n + d] = pos;
    }
    __syncthreads();
    const int rb = ep_row_bytes_dev(a.H, a.k);
    const int meta = (a.H >> 1) + nb;
    for (int d = 0; d < ep.n; ++d) {
      const int pos = s_dpos[d];
      if (pos < 0) continue;
      uint8_t* row = ep.table->recv[d] + (size_t(ep.rank) * (ep.C + 1) + 1 + pos) * rb;
      for (int i = threadIdx.x; i < (a.H >> 5); i += kClusterThreads)
        reinterpret_cast<uint4*>(row)[i] = reinterpret_cast<const uint4*>(s_xq)[i];
      for (int i = threadIdx.x; i < (a.H >> 7); i += kClusterThreads)
        reinterpret_cast<uint32_t*>(row + (a.H >> 1))[i] = reinterpret_cast<const uint32_t*>(s_xsc)[i];
      if (threadIdx.x == 0) reinterpret_cast<int*>(row + meta)[0] = t;
      if (threadIdx.x < a.k) {
        const int e = s_sel[threadIdx.x];
        reinterpret_cast<int*>(row + meta + 16)[threadIdx.x] = (e / ep.el) == d ? e % ep.el : -1;
        reinterpret_cast<float*>(row + meta + 16 + 4 * a.k)[threadIdx.x] = s_tw[threadIdx.x];
      }
    }
    ep_finish_dispatch(ep, a.H, a.k, int(gridDim.x) / n_split, ep_call);
    return;
  }
  if (a.xp) {
    __syncthreads();
    const int q16 = a.H >> 5;
    for (int i = threadIdx.x; i < a.k * q16; i += kClusterThreads) {
      const int j = i / q16, c = i % q16;
      if (s_row[j] < 0) continue;
      reinterpret_cast<uint4*>(a.xp + size_t(s_row[j]) * (a.H >> 1))[c] =
          reinterpret_cast<const uint4*>(s_xq)[c];
    }
    const int kc = a.H >> 7;
    for (int i = threadIdx.x; i < a.k * kc; i += kClusterThreads) {
      const int j = i / kc, c = i % kc;
      const int row = s_row[j];
      if (row < 0) continue;
      *reinterpret_cast<uint32_t*>(a.xp_atoms + (size_t(row >> 5) * kc + c) * 512 + (row & 31) * 16) =
          reinterpret_cast<const uint32_t*>(s_xsc)[c];
    }
  }
}

// ---------------------------------------------------------------------------
// Batch router for prefill sizes (many tokens): the whole router (E rows and
// their scales) is staged once per CTA in shared memory and every warp routes
// one token at a time — quantise, 128 logits with route_kernel's per-lane
// order and butterfly (bit-identical), top-k by 8 rounds of warp arg-max
// (value descending, lower index on ties: the same order as the rank method),
// weights, and the per-expert position claim of the prefill placement.
constexpr int kBatchThreads = 512;
constexpr int kBatchWarps = kBatchThreads / 32;

// Each warp routes kBatchTok tokens together, so every router block is
// expanded from nibbles to int8 once for all of them.
#ifndef MFI_BATCH_TOK
#define MFI_BATCH_TOK 2
#endif
#ifndef MFI_BATCH_U
#define MFI_BATCH_U 4
#endif
constexpr int kBatchTok = MFI_BATCH_TOK;

// per (warp, token): the quantised row (H/2 B, reused for the E logits once
// the row is in registers) and its scales
__host__ __device__ inline size_t route_batch_slot(int E, int H) {
  const size_t row = size_t(H / 2) > size_t(E) * sizeof(float) ? size_t(H / 2) : size_t(E) * sizeof(float);
  return (row + size_t(H / 32) + 15) / 16 * 16;
}
size_t route_batch_smem(int E, int H) {
  return size_t(E) * (H / 2) + size_t(E) * (H / 32) +
         size_t(kBatchWarps) * kBatchTok * route_batch_slot(E, H) + 64;
}

// Quantise token t into (s_xq, s_xsc) with the whole warp (quads of lanes per
// 32-element block); t < 0: zeros.
template <int kMaxBlk>
__global__ void __launch_bounds__(kBatchThreads) route_batch_kernel(RouteArgs a) {
  extern __shared__ __align__(128) uint8_t smem[];
  const int nb = a.H >> 5;
  uint8_t* s_w = smem;                                          // [E][H/2]
  uint8_t* s_ws = s_w + size_t(a.E) * (a.H >> 1);               // [E][H/32]
  uint8_t* s_slots = s_ws + size_t(a.E) * nb;                   // [warps][tok][slot]
  const size_t slot = route_batch_slot(a.E, a.H);
  const size_t row_bytes = a.H / 2 > a.E * 4 ? size_t(a.H / 2) : size_t(a.E) * 4;
  __shared__ __align__(8) uint64_t s_bar;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;

  const uint32_t w_bytes = uint32_t(a.E) * uint32_t(a.H >> 1);
  const uint32_t sc_bytes = uint32_t(a.E) * uint32_t(nb);
  const bool sc_bulk = (sc_bytes % 16) == 0 && (reinterpret_cast<uintptr_t>(a.sr) % 16) == 0;
  if (threadIdx.x == 0) {
    tc::mbar_init(&s_bar, 1);
    tc::fence_mbar_init();
    tc::cta_abort_init();
    tc::mbar_expect_tx(&s_bar, w_bytes + (sc_bulk ? sc_bytes : 0u));
    tc::bulk_load(s_w, a.wr, w_bytes, &s_bar);
    if (sc_bulk) tc::bulk_load(s_ws, a.sr, sc_bytes, &s_bar);
  }
  if (!sc_bulk)
    for (uint32_t i = threadIdx.x; i < sc_bytes; i += kBatchThreads) s_ws[i] = a.sr[i];
  __syncthreads();
  const bool have_w = tc::mbar_wait(&s_bar, 0, a.err, 6);
  // failed: the router rows may still be landing; wait for them before exit
  if (!have_w && threadIdx.x == 0) tc::mbar_wait(&s_bar, 0, nullptr, 0);
  __syncthreads();

  const int groups = (a.T + kBatchTok - 1) / kBatchTok;
  for (int grp = blockIdx.x * kBatchWarps + warp; grp < groups; grp += gridDim.x * kBatchWarps) {
    int tok[kBatchTok];
    uint32_t xa8[kBatchTok][kMaxBlk][8];
    int xs[kBatchTok][kMaxBlk];
#pragma unroll
    for (int q = 0; q < kBatchTok; ++q) {
      const int t = grp * kBatchTok + q;
      tok[q] = t < a.T ? t : -1;
      uint8_t* s_xq = s_slots + size_t(warp * kBatchTok + q) * slot;
      uint8_t* s_xsc = s_xq + row_bytes;
      warp_quant_token(a, tok[q], s_xq, s_xsc, lane);
      __syncwarp();
      if (a.xq && tok[q] >= 0) {
        for (int i = lane; i < (a.H >> 5); i += 32)
          reinterpret_cast<uint4*>(a.xq + long(tok[q]) * (a.H >> 1))[i] =
              reinterpret_cast<const uint4*>(s_xq)[i];
        for (int i = lane; i < nb; i += 32) a.xsc[long(tok[q]) * nb + i] = s_xsc[i];
      }
#pragma unroll
      for (int j = 0; j < kMaxBlk; ++j) {
        const int bl = lane + 32 * j;
        if (bl < nb) {
          const uint4 qv = reinterpret_cast<const uint4*>(s_xq)[bl];
          nib8_to_i8(qv.x, xa8[q][j][0], xa8[q][j][1]);
          nib8_to_i8(qv.y, xa8[q][j][2], xa8[q][j][3]);
          nib8_to_i8(qv.z, xa8[q][j][4], xa8[q][j][5]);
          nib8_to_i8(qv.w, xa8[q][j][6], xa8[q][j][7]);
          xs[q][j] = s_xsc[bl];
        }
      }
    }
    __syncwarp();  // the rows are in registers: their slots now take the logits
    // ---- logits: kU experts x kBatchTok tokens per pass ---------------------
    constexpr int kU = MFI_BATCH_U;
    constexpr int kV = kU * kBatchTok;  // values reduced together, index q * kU + u
    for (int e0 = 0; e0 < a.E; e0 += kU) {
      double acc[kV];
#pragma unroll
      for (int v = 0; v < kV; ++v) acc[v] = 0.0;
#pragma unroll
      for (int u = 0; u < kU; ++u) {
        const int e = e0 + u;
#pragma unroll
        for (int j = 0; j < kMaxBlk; ++j) {
          const int bl = lane + 32 * j;
          if (have_w && e < a.E && bl < nb) {
            const uint4 wv = *reinterpret_cast<const uint4*>(s_w + size_t(e) * (a.H >> 1) + bl * 16);
            uint32_t w8[8];
            nib8_to_i8(wv.x, w8[0], w8[1]);
            nib8_to_i8(wv.y, w8[2], w8[3]);
            nib8_to_i8(wv.z, w8[4], w8[5]);
            nib8_to_i8(wv.w, w8[6], w8[7]);
            const int sc = int(s_ws[e * nb + bl]);
#pragma unroll
            for (int q = 0; q < kBatchTok; ++q) {
              // two independent dp4a chains, then one add (exact integers)
              int d0 = 0, d1 = 0;
#pragma unroll
              for (int i = 0; i < 8; i += 2) {
                d0 = __dp4a(int(xa8[q][j][i]), int(w8[i]), d0);
                d1 = __dp4a(int(xa8[q][j][i + 1]), int(w8[i + 1]), d1);
              }
              const int sdot = d0 + d1;
              acc[q * kU + u] += double(sdot) * exp2i_d(xs[q][j] + sc - 256);
            }
          }
        }
      }
      // reduce-scatter butterfly over the kV values (same pairwise sums per
      // value as a full butterfly 16, 8, 4, 2, 1)
      int n = kV;
#pragma unroll
      for (int off = 16; off >= 1; off >>= 1) {
        if (n > 1) {
          const bool upper = (lane & off) != 0;
          const int h = n >> 1;
#pragma unroll
          for (int i = 0; i < kV / 2; ++i) {
            if (i < h) {
              const double send = upper ? acc[i] : acc[i + h];
              const double keep = upper ? acc[i + h] : acc[i];
              acc[i] = keep + __shfl_xor_sync(0xffffffffu, send, off);
            }
          }
          n = h;
        } else {
          acc[0] += __shfl_xor_sync(0xffffffffu, acc[0], off);
        }
      }
      // after log2(kV) halving steps lane l holds value l >> (5 - log2 kV)
      constexpr int kLog = kV == 16 ? 4 : (kV == 8 ? 3 : (kV == 4 ? 2 : 1));
      static_assert(kV == 2 || kV == 4 || kV == 8 || kV == 16, "values per pass");
      if ((lane & ((32 >> kLog) - 1)) == 0) {
        const int v = lane >> (5 - kLog);
        const int q = v / kU, e = e0 + v % kU;
        if (e < a.E)
          reinterpret_cast<float*>(s_slots + size_t(warp * kBatchTok + q) * slot)[e] = float(acc[0]);
      }
    }
    __syncwarp();
    // ---- per token: bias, logits out, top-k, weights, position claims -------
#pragma unroll 1
    for (int q = 0; q < kBatchTok; ++q) {
      const int t = tok[q];
      if (t < 0) continue;
      finish_token(a, t, reinterpret_cast<float*>(s_slots + size_t(warp * kBatchTok + q) * slot),
                   lane);
    }
  }
}

template <int kMaxBlk>
static cudaError_t launch_route_batch(const RouteArgs& a, cudaStream_t stream) {
  const size_t smem = route_batch_smem(a.E, a.H);
  {
    cudaError_t e = ensure_dynamic_smem(reinterpret_cast<const void*>(route_batch_kernel<kMaxBlk>), smem);
    if (e != cudaSuccess) return e;
  }
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int need = (a.T + kBatchWarps * kBatchTok - 1) / (kBatchWarps * kBatchTok);
  route_batch_kernel<kMaxBlk><<<need < sms ? need : sms, kBatchThreads, smem, stream>>>(a);
  return cudaGetLastError();
}

template <int kMaxBlk, int kEPC>
static cudaError_t launch_route_cluster_n(const RouteArgs& a, cudaStream_t stream) {
  const int n_split = (a.E + kEPC - 1) / kEPC;  // <= 8
  const size_t smem = size_t(kEPC) * (a.H >> 1);
  {
    cudaError_t e =
        ensure_dynamic_smem(reinterpret_cast<const void*>(route_cluster_kernel<kMaxBlk, kEPC>), smem);
    if (e != cudaSuccess) return e;
  }
  cudaLaunchConfig_t cfg{};
  const int clusters = a.ep.table ? (a.T > 0 ? a.T : 1) : a.T;
  cfg.gridDim = dim3(clusters * n_split);
  cfg.blockDim = dim3(kClusterThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = n_split;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, route_cluster_kernel<kMaxBlk, kEPC>, a, n_split);
}

template <int kMaxBlk>
static cudaError_t launch_route_cluster(const RouteArgs& a, cudaStream_t stream) {
  // small batches: 8-CTA clusters halve each CTA's router rows (the latency
  // of a few tokens); at T = 32/64 the 4-CTA clusters measured faster
  return a.E <= 8 * 16 && a.T <= 16 ? launch_route_cluster_n<kMaxBlk, 16>(a, stream)
                                    : launch_route_cluster_n<kMaxBlk, kExpertsPerCta>(a, stream);
}

cudaError_t launch_route(const RouteArgs& a, cudaStream_t stream) {
  if (a.T < 0 || (a.T == 0 && !a.ep.table)) return cudaSuccess;
  if (a.H > 4096) return cudaErrorInvalidValue;
  if (!a.g_gu) {
    // prefill sizes, Qwen-shaped router: the tensor-core router
    if (route_tc_applies(a)) return launch_route_tc(a, stream);
    // many tokens, placement by position claims, router fits in shared
    // memory: one router copy per CTA, one token per warp
    if (a.batch && !a.xp && !a.ep.table && route_batch_smem(a.E, a.H) <= 220 * 1024 &&
        (size_t(a.E) * (a.H >> 5)) % 16 == 0 && (reinterpret_cast<uintptr_t>(a.wr) & 15) == 0)
      return a.H <= 2048 ? launch_route_batch<2>(a, stream) : launch_route_batch<4>(a, stream);
    // routing alone, or routing + expert regions for the tensor-core kernels
    return a.H <= 2048 ? launch_route_cluster<2>(a, stream) : launch_route_cluster<4>(a, stream);
  }
  if (a.H <= 2048)
    route_kernel<2><<<a.T, kRouteThreads, 0, stream>>>(a);
  else
    route_kernel<4><<<a.T, kRouteThreads, 0, stream>>>(a);
  return cudaGetLastError();
}

}  // namespace mfi
