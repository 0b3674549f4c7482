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

__global__ void __launch_bounds__(kRouteThreads) route_kernel(RouteArgs a) {
  __shared__ float s_logit[kMaxE];
  __shared__ unsigned s_last;
  const int t = blockIdx.x;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int nwarp = kRouteThreads / 32;
  const int nb = a.H >> 5;

  // ---- logits for token t --------------------------------------------------
  for (int e = warp; e < a.E; e += nwarp) {
    double acc = 0.0;
    for (int b = lane; b < nb; b += 32) {
      const uint4 xa = ldg_u4(a.xq + long(t) * (a.H >> 1) + b * 16);
      const uint4 wb = ldg_u4(a.wr + long(e) * (a.H >> 1) + b * 16);
      const int s = block_dot_i(xa, wb);
      const int ex = int(a.xsc[long(t) * nb + b]) + int(a.sr[long(e) * nb + b]) - 256;
      acc += double(s) * exp2i_d(ex);
    }
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
    if (lane == 0) s_logit[e] = float(acc);
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

  __shared__ int s_cnt[kMaxE];
  __shared__ int s_off[kMaxE];
  __shared__ int s_act[kMaxE];  // active index of expert e, or -1
  const int P = a.T * a.k;
  for (int e = threadIdx.x; e < a.E; e += blockDim.x) s_cnt[e] = 0;
  __syncthreads();
  for (int i = threadIdx.x; i < P; i += blockDim.x) atomicAdd(&s_cnt[__ldcg(a.topi + i)], 1);
  __syncthreads();
  if (threadIdx.x == 0) {
    int off = 0, na = 0;
    for (int e = 0; e < a.E; ++e) {
      s_off[e] = off;
      off += s_cnt[e];
      s_act[e] = s_cnt[e] > 0 ? na++ : -1;
    }
    *a.n_gu = 2 * na;
    *a.n_dn = na;
    *a.n_active = na;
    *a.done = 0u;  // ready for the next call
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
    // entries of expert e in (token, slot) order
    int pos = first;
    for (int i = 0; i < P; ++i) {
      if (__ldcg(a.topi + i) != e) continue;
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
      ++pos;
    }
  }
}

cudaError_t launch_route(const RouteArgs& a, cudaStream_t stream) {
  if (a.T <= 0) return cudaSuccess;
  route_kernel<<<a.T, kRouteThreads, 0, stream>>>(a);
  return cudaGetLastError();
}

}  // namespace mfi
