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

namespace mfi {

constexpr int kRouteThreads = 512;
constexpr int kMaxE = kRouteMaxE;

__device__ __forceinline__ bool better(float v, int i, float w, int j) {
  return v > w || (v == w && i < j);
}

template <int kMaxBlk>
__global__ void __launch_bounds__(kRouteThreads) route_kernel(RouteArgs a) {
  __shared__ float s_logit[kMaxE];
  __shared__ unsigned s_last;
  const int t = blockIdx.x;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int nwarp = kRouteThreads / 32;
  const int nb = a.H >> 5;

  // ---- logits for token t --------------------------------------------------
  // Each lane owns blocks b = lane + 32*j; the token's blocks are loaded once,
  // the router rows of all experts of this warp are in flight together.
  uint4 xa[kMaxBlk];
  int xs[kMaxBlk];
#pragma unroll
  for (int j = 0; j < kMaxBlk; ++j) {
    const int b = lane + 32 * j;
    if (b < nb) {
      xa[j] = ldg_u4(a.xq + long(t) * (a.H >> 1) + b * 16);
      xs[j] = a.xsc[long(t) * nb + b];
    }
  }
  for (int e0 = warp; e0 < a.E; e0 += 4 * nwarp) {
    uint4 wv[4][kMaxBlk];
    int ws[4][kMaxBlk];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
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
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int e = e0 + u * nwarp;
      double acc = 0.0;
#pragma unroll
      for (int j = 0; j < kMaxBlk; ++j) {
        const int b = lane + 32 * j;
        if (e < a.E && b < nb) {
          const int s = block_dot_i(xa[j], wv[u][j]);
          acc += double(s) * exp2i_d(xs[j] + ws[u][j] - 256);
        }
      }
#pragma unroll
      for (int off = 16; off >= 1; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
      if (lane == 0 && e < a.E) s_logit[e] = float(acc);
    }
  }
  __syncthreads();
  if (a.logits)
    for (int e = threadIdx.x; e < a.E; e += blockDim.x) a.logits[long(t) * a.E + e] = s_logit[e];

  // ---- top-k (warp 0) --------------------------------------------------------
  if (warp == 0) {
    unsigned long long taken = 0ull;  // bit i: expert lane + 32*i already selected
    float selv = 0.f;
    int seli = 0;
    for (int j = 0; j < a.k; ++j) {
      float bv = -INFINITY;
      int bi = 0x7fffffff;
      for (int i = 0; lane + 32 * i < a.E; ++i) {
        const int e = lane + 32 * i;
        if ((taken >> i) & 1ull) continue;
        const float v = s_logit[e];
        if (bi == 0x7fffffff || better(v, e, bv, bi)) { bv = v; bi = e; }
      }
#pragma unroll
      for (int off = 16; off >= 1; off >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, off);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, off);
        if (oi != 0x7fffffff && (bi == 0x7fffffff || better(ov, oi, bv, bi))) { bv = ov; bi = oi; }
      }
      if ((bi & 31) == lane && bi != 0x7fffffff) taken |= 1ull << (bi >> 5);
      if (lane == j) { selv = bv; seli = bi; }
    }
    // weights: exp(l - max) over the selected, normalised by their sum
    const float mx = __shfl_sync(0xffffffffu, selv, 0);
    const float p = (lane < a.k) ? expf(selv - mx) : 0.f;
    float sum = 0.f;
    for (int j = 0; j < a.k; ++j) sum = __fadd_rn(sum, __shfl_sync(0xffffffffu, p, j));
    if (lane < a.k) {
      a.topi[long(t) * a.k + lane] = seli;
      a.topw[long(t) * a.k + lane] = __fdiv_rn(p, sum);
    }
  }

  // ---- last CTA builds the per-expert work lists ----------------------------
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
  const long gstride = long(a.Mi) * (a.H >> 1), gsstride = long(a.Mi) * (a.H >> 5);
  const long dstride = long(a.H) * (a.Mi >> 1), dsstride = long(a.H) * (a.Mi >> 5);
  for (int e = threadIdx.x; e < a.E; e += blockDim.x) {
    const int ai = s_act[e];
    if (ai < 0) continue;
    const int first = s_off[e], cnt = s_cnt[e];
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
    if (a.chunks) {
      for (int c = 0; c * 32 < cnt; ++c) {
        ChunkDesc cd;
        cd.expert = e;
        cd.count = min(32, cnt - 32 * c);
        a.chunks[s_cbase[e] + c] = cd;
        for (int r = cd.count; r < 32; ++r) a.perm[(s_cbase[e] + c) * 32 + r] = -1;
      }
    }
  }
  for (int i = threadIdx.x; i < P; i += blockDim.x) {
    const int e = __ldcg(a.topi + i);
    const int pil = atomicAdd(&s_cur[e], 1);  // position in expert e's list
    const int pos = s_off[e] + pil;
    if (a.perm) a.perm[(s_cbase[e] + pil / 32) * 32 + pil % 32] = i;
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

cudaError_t launch_route(const RouteArgs& a, cudaStream_t stream) {
  if (a.T <= 0) return cudaSuccess;
  if (a.H <= 2048)
    route_kernel<2><<<a.T, kRouteThreads, 0, stream>>>(a);
  else if (a.H <= 4096)
    route_kernel<4><<<a.T, kRouteThreads, 0, stream>>>(a);
  else
    return cudaErrorInvalidValue;
  return cudaGetLastError();
}

}  // namespace mfi
