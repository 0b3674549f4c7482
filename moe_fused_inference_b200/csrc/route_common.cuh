// route_common.cuh — pieces shared by the router kernels (route.cu,
// route_tc.cu): the fused bf16 -> MXFP4 quantiser of one token, the
// deterministic expert order, and the per-token tail (bias, logits out,
// top-k, weights, placement claims).
#pragma once
#include "mx_common.cuh"
#include "work.cuh"

namespace mfi {

// Expert order of the top-k: larger logit first, ties to the lower index.
__device__ __forceinline__ bool better(float v, int i, float w, int j) {
  return v > w || (v == w && i < j);
}

// RMSNorm of a token row before quantisation — the MoE block's
// post-attention layernorm (reference runtime/model_runner.py:20-25, called at
// runtime/model_runner_v2.py:183):
//   r = 1 / sqrt(float(ss) / H + eps),  ss = sum of x_i^2,
//   y_i = bf16(bf16(x_i * r) * w_i)
// (the reference normalises in fp32, casts to the activation type, then
// multiplies by the bf16 weight).  ss is accumulated in fp64: every square of
// a bf16 value is exact there, so the sum is exact, whatever the order, for
// any row whose magnitudes span less than 2^13, and rounded to fp32 once.
// One warp computes r for row t (every lane returns it).
__device__ __forceinline__ float warp_rms_inv(const RouteArgs& a, int t, int lane) {
  const __nv_bfloat16* row = reinterpret_cast<const __nv_bfloat16*>(a.x) + long(t) * a.H;
  double ss = 0.0;
  for (int c8 = lane; c8 < (a.H >> 3); c8 += 32) {
    const uint4 raw = *reinterpret_cast<const uint4*>(row + c8 * 8);
    const __nv_bfloat162* h2 = reinterpret_cast<const __nv_bfloat162*>(&raw);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 f = __bfloat1622float2(h2[i]);
      ss += double(f.x) * double(f.x);
      ss += double(f.y) * double(f.y);
    }
  }
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
  const float var = __fdiv_rn(__double2float_rn(ss), float(a.H));
  return __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(var, a.norm_eps)));
}

// Elements c .. c+7 of a normalised row (see warp_rms_inv), in place.
__device__ __forceinline__ void rms_apply8(const RouteArgs& a, int c, float r, float (&v)[8]) {
  const uint4 wr = *reinterpret_cast<const uint4*>(a.norm_w + c);
  const __nv_bfloat162* w2 = reinterpret_cast<const __nv_bfloat162*>(&wr);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 w = __bfloat1622float2(w2[i]);
    const float y0 = __bfloat162float(__float2bfloat16_rn(__fmul_rn(v[2 * i], r)));
    const float y1 = __bfloat162float(__float2bfloat16_rn(__fmul_rn(v[2 * i + 1], r)));
    v[2 * i] = __bfloat162float(__float2bfloat16_rn(__fmul_rn(y0, w.x)));
    v[2 * i + 1] = __bfloat162float(__float2bfloat16_rn(__fmul_rn(y1, w.y)));
  }
}

// One warp quantises token t (bf16 row of a.x, RMS-normalised first when
// a.norm_w is set) into s_xq (H/2 packed bytes) and s_xsc (H/32 E8M0 codes);
// t < 0 gives an all-zero row (codes 127).
__device__ __forceinline__ void warp_quant_token(const RouteArgs& a, int t, uint8_t* s_xq,
                                                 uint8_t* s_xsc, int lane) {
  const float r = (a.norm_w && t >= 0) ? warp_rms_inv(a, t, lane) : 1.0f;
  for (int base = 0; base < (a.H >> 3); base += 32) {
    const int c8 = base + lane;
    const bool live = c8 < (a.H >> 3);
    float v[8];
    if (live && t >= 0) {
      const uint4 raw = *reinterpret_cast<const uint4*>(
          reinterpret_cast<const __nv_bfloat16*>(a.x) + long(t) * a.H + c8 * 8);
      const __nv_bfloat162* h2 = reinterpret_cast<const __nv_bfloat162*>(&raw);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 f = __bfloat1622float2(h2[i]);
        v[2 * i] = f.x;
        v[2 * i + 1] = f.y;
      }
      if (a.norm_w) rms_apply8(a, c8 * 8, r, v);
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
}

// One warp finishes token t from its fp32 logits in s_lg[0..E): adds the
// logit bias, writes the logits, selects the top-k (larger first, ties to
// the lower expert), computes the weights exp(l - max) / sum in slot order
// and, for prefill placement, claims each slot's position in its expert —
// unless sel_out is given: then the selected experts go to sel_out[0..k) and
// the caller claims positions itself.
// Reference: runtime/model_runner_v2.py:100-106 (softmax, top-k, renorm).
__device__ __forceinline__ void finish_token(const RouteArgs& a, int t, float* s_lg, int lane,
                                             int* sel_out = nullptr) {
  if (a.logit_bias)
    for (int e = lane; e < a.E; e += 32) s_lg[e] = __fadd_rn(s_lg[e], a.logit_bias[e]);
  __syncwarp();
  if (a.logits)
    for (int e = lane; e < a.E; e += 32) a.logits[long(t) * a.E + e] = s_lg[e];
  constexpr int kPer = kRouteMaxE / 32;
  float v[kPer];
  uint32_t taken = 0;
#pragma unroll
  for (int i = 0; i < kPer; ++i) v[i] = (lane + 32 * i < a.E) ? s_lg[lane + 32 * i] : 0.0f;
  int my_sel = -1;
  float my_val = 0.0f;
  for (int j = 0; j < a.k; ++j) {
    float bv = 0.0f;
    int bi = -1;
#pragma unroll
    for (int i = 0; i < kPer; ++i) {
      const int e = lane + 32 * i;
      if (e < a.E && !((taken >> i) & 1u) && (bi < 0 || better(v[i], e, bv, bi))) {
        bv = v[i];
        bi = e;
      }
    }
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, off);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, off);
      if (oi >= 0 && (bi < 0 || better(ov, oi, bv, bi))) {
        bv = ov;
        bi = oi;
      }
    }
    if ((bi & 31) == lane) taken |= 1u << (bi >> 5);
    if (lane == j) {
      my_sel = bi;
      my_val = bv;
    }
  }
  const float mx = __shfl_sync(0xffffffffu, my_val, 0);
  const float pj = lane < a.k ? expf(my_val - mx) : 0.0f;
  float sum = 0.0f;
  for (int j = 0; j < a.k; ++j) sum = __fadd_rn(sum, __shfl_sync(0xffffffffu, pj, j));
  if (lane < a.k) {
    a.topi[long(t) * a.k + lane] = my_sel;
    a.topw[long(t) * a.k + lane] = __fdiv_rn(pj, sum);
    if (sel_out)
      sel_out[lane] = my_sel;
    else if (a.slot_pos)
      a.slot_pos[long(t) * a.k + lane] = atomicAdd(a.cursor + my_sel, 1);
  }
  __syncwarp();
}

}  // namespace mfi
