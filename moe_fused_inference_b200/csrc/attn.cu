// attn.cu — FP8 (E4M3) KV-cache write and single-sequence decode attention.
//
// Replaces the reference's graph-friendly decode attention and KV write
// (src/ext/mxfp4_decode.cu:352-490, bound as attn_decode / kv_write by
// src/ext/mxfp4_decode_binding.cpp:161-173, 213-230): the model runner's
// attention of M query rows of one sequence (runtime/model_runner_v2.py:
// 244-262) over an FP8 K/V cache laid out (max_pos, Hkv, D), the base
// position read from device memory so the calls can be replayed in a graph.
//
// The reference computes, per (query head, row), all scores in one warp and
// then one online-softmax pass over every position in one 128-thread block:
// Hq x M blocks stream the whole cache serially.  Here the positions are
// split over the grid (flash-decoding):
//   attn_partial_kernel  CTA (split j, KV head g): decodes a 32-position tile
//                        of K and V to fp32 in shared memory once and serves
//                        every query head of the group and every query row
//                        from it — scores, running max / sum, weighted V —
//                        writing one partial (max, sum, D accumulators) per
//                        (row, head, split) to the workspace;
//   attn_merge_kernel    per (row, head): log-sum-exp merge of the splits.
// Splits are sized from max_pos (the host does not know the device-side base
// position); CTAs past the live positions write empty partials.
//
// Two FP8 formats:
//  * scale == NULL: the reference's own codec, bit for bit.  Its encoder
//    (f32_to_e4m3, mxfp4_decode.cu:447-466) rounds the 3-bit mantissa half
//    away from zero, encodes values below 2^-6 as round(a * 64) (0 or 1) and
//    saturates anything that rounds to 2^8 or more to 0x7F; its decoder
//    (e4m3_to_f32, :362-371) reads exponent 0 as m * 2^-6 and exponent 15 as
//    448 * (1 + m/8).  The decode table below restates that decoder.
//  * per-KV-head fp32 scales: the standard E4M3 (e4m3fn) encoding of x/scale,
//    round to nearest even with saturation to +-448 (cvt.rn.satfinite), and
//    its exact decoding times the scale — the per-head scale the model
//    configuration asks for (the reference has none,
//    runtime/model_runner_v2.py:39).
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp8.h>

#include <cmath>

#include "../../include/moe_fp4.h"
#include "tmap.cuh"
#include "work.cuh"

namespace mfi {
namespace {

constexpr int kD = 128;          // head dimension (the reference kernels assume 128)
constexpr int kTile = 32;        // positions per shared-memory tile
constexpr int kWarps = 8;
constexpr int kThreads = kWarps * 32;
constexpr int kMaxGroup = 16;    // query heads per KV head
constexpr int kRowsPerPass = 4;  // query rows held in registers per pass
constexpr int kKStride = kD + 4; // padded fp32 row of the K tile (conflict-free float4 reads)
// one split's partial result: D accumulators, then max and sum, padded so
// every row starts on a 16-byte boundary (the accumulators go out as float4)
constexpr int kPartStride = kD + 4;
static_assert((kPartStride * 4) % 16 == 0, "partial rows must stay 16-byte aligned");

// ---- FP8 codecs --------------------------------------------------------------
// The reference encoder, restated: sign from v < 0; frexp exponent e of |v|;
// 3-bit mantissa round((|v| / 2^(e-1) - 1) * 8) half away from zero, carry
// into the exponent; exponent field e + 6, values with field <= 0 encoded as
// round(|v| * 64); field >= 15 saturates to 0x7F.  Non-finite inputs (left
// undefined by the reference's lroundf) saturate to 0x7F.
__device__ __forceinline__ uint8_t e4m3_ref_encode(float v) {
  const uint32_t sign = v < 0.0f ? 0x80u : 0u;
  const float a = fabsf(v);
  if (a == 0.0f) return uint8_t(sign);
  if (!(a <= 3.402823466e38f)) return uint8_t(sign | 0x7Fu);
  int e;
  frexpf(a, &e);
  int eb = e + 6;
  const float man = ldexpf(a, 1 - e);                 // [1, 2), exact
  int q = int(lroundf((man - 1.0f) * 8.0f));          // exact product, half away from zero
  if (q == 8) {
    q = 0;
    ++eb;
  }
  if (eb <= 0) {
    int s = int(lroundf(a * 64.0f));
    s = s < 0 ? 0 : (s > 7 ? 7 : s);
    return uint8_t(sign | uint32_t(s));
  }
  if (eb >= 15) {
    eb = 15;
    q = 7;
  }
  return uint8_t(sign | (uint32_t(eb) << 3) | uint32_t(q));
}

// Standard e4m3fn of v (round to nearest even, saturating; NaN -> 0x7F).
__device__ __forceinline__ uint8_t e4m3_std_encode(float v) {
  const __nv_fp8_e4m3 f(v);  // __NV_SATFINITE conversion
  return *reinterpret_cast<const uint8_t*>(&f);
}

// Decoded value of byte b: the reference's decoder or the standard format.
__device__ __forceinline__ float e4m3_decode(uint32_t b, bool ref) {
  const int m = int(b & 7u), e = int((b >> 3) & 15u);
  float v;
  if (ref) {
    if (e == 0) v = float(m) * 0.015625f;                       // m * 2^-6
    else if (e == 15) v = 448.0f * (float(m) * 0.125f + 1.0f);
    else v = (float(m) * 0.125f + 1.0f) * __uint_as_float(uint32_t(e - 7 + 127) << 23);
  } else {
    if (e == 0) v = float(m) * 0.001953125f;                    // m * 2^-9
    else if (e == 15 && m == 7) v = __uint_as_float(0x7fc00000u);
    else v = (float(m) * 0.125f + 1.0f) * __uint_as_float(uint32_t(e - 7 + 127) << 23);
  }
  return (b & 0x80u) ? -v : v;
}

// ---- KV write ----------------------------------------------------------------
// One thread per 8 elements of one (row, head): k and v bf16 (M, Hkv, D) ->
// kvk, kvv at position *dpos + m.
__global__ void __launch_bounds__(256) kv_write_kernel(
    const __nv_bfloat16* __restrict__ k, const __nv_bfloat16* __restrict__ v,
    uint8_t* __restrict__ kvk, uint8_t* __restrict__ kvv, const int* __restrict__ dpos, int M,
    int Hkv, int D, int max_pos, const float* __restrict__ k_scale,
    const float* __restrict__ v_scale) {
  const long long per_row = (long long)Hkv * D;
  const long long n8 = (long long)M * per_row / 8;
  const long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x;
  if (i >= n8) return;
  const int base = *dpos;
  const long long e0 = i * 8;
  const int m = int(e0 / per_row);
  const long long t = e0 % per_row;
  const int pos = base + m;
  if (base < 0 || pos >= max_pos) return;
  const int g = int(t / D);
  const uint4 kr = *reinterpret_cast<const uint4*>(k + e0);
  const uint4 vr = *reinterpret_cast<const uint4*>(v + e0);
  const __nv_bfloat16* kb = reinterpret_cast<const __nv_bfloat16*>(&kr);
  const __nv_bfloat16* vb = reinterpret_cast<const __nv_bfloat16*>(&vr);
  uint32_t ko[2] = {0u, 0u}, vo[2] = {0u, 0u};
  if (k_scale == nullptr) {
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      ko[j >> 2] |= uint32_t(e4m3_ref_encode(__bfloat162float(kb[j]))) << (8 * (j & 3));
      vo[j >> 2] |= uint32_t(e4m3_ref_encode(__bfloat162float(vb[j]))) << (8 * (j & 3));
    }
  } else {
    const float ks = k_scale[g], vs = v_scale[g];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      ko[j >> 2] |= uint32_t(e4m3_std_encode(__fdiv_rn(__bfloat162float(kb[j]), ks))) << (8 * (j & 3));
      vo[j >> 2] |= uint32_t(e4m3_std_encode(__fdiv_rn(__bfloat162float(vb[j]), vs))) << (8 * (j & 3));
    }
  }
  const long long off = (long long)pos * per_row + t;
  *reinterpret_cast<uint2*>(kvk + off) = make_uint2(ko[0], ko[1]);
  *reinterpret_cast<uint2*>(kvv + off) = make_uint2(vo[0], vo[1]);
}

// ---- decode attention ----------------------------------------------------------
struct AttnArgs {
  const __nv_bfloat16* q;   // (M, Hq, D)
  const uint8_t* kvk;       // (max_pos, Hkv, D)
  const uint8_t* kvv;
  const int* dpos;
  const float* k_scale;     // (Hkv) or null (reference codec)
  const float* v_scale;
  float* part;              // [M][Hq][nsplit][kPartStride]: acc[D], max, sum, pad
  float* o;                 // (M, Hq, D)
  int M, Hq, Hkv, max_pos, nsplit, chunk;
  float inv_sqrt_d;
  long long kv_seq_stride;  // bytes between consecutive sequences' caches
};

// The arguments of sequence `seq` of a batched call: sequence s owns rows
// [s*M, (s+1)*M) of q, o and the partials, and the cache at s*kv_seq_stride.
__device__ __forceinline__ AttnArgs for_sequence(AttnArgs a, int seq) {
  const size_t rows = size_t(seq) * a.M * a.Hq;
  a.q += rows * kD;
  a.o += rows * kD;
  a.part += rows * size_t(a.nsplit) * kPartStride;
  a.kvk += size_t(seq) * a.kv_seq_stride;
  a.kvv += size_t(seq) * a.kv_seq_stride;
  return a;
}

// dynamic shared memory: decode table, K tile (padded rows), V tile, queries
constexpr size_t kSmemLut = 256 * sizeof(float);
constexpr size_t kSmemK = size_t(kTile) * kKStride * sizeof(float);
constexpr size_t kSmemV = size_t(kTile) * kD * sizeof(float);
constexpr size_t kSmemQ = size_t(kMaxGroup) * kRowsPerPass * kD * sizeof(float);
constexpr size_t kAttnSmem = kSmemLut + kSmemK + kSmemV + kSmemQ;

__global__ void __launch_bounds__(kThreads) attn_partial_kernel(AttnArgs a_all) {
  const AttnArgs a = for_sequence(a_all, blockIdx.z);
  extern __shared__ __align__(16) float smem_f[];
  float* lut = smem_f;
  float* s_k = lut + 256;
  float* s_v = s_k + kTile * kKStride;
  float* s_q = s_v + kTile * kD;
  const int split = blockIdx.x, g = blockIdx.y;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int G = a.Hq / a.Hkv;
  const bool ref = a.k_scale == nullptr;
  lut[threadIdx.x] = e4m3_decode(threadIdx.x, ref);
  const float ks = ref ? 1.0f : a.k_scale[g];
  const float vs = ref ? 1.0f : a.v_scale[g];
  const float qscale = a.inv_sqrt_d * ks;  // softmax scale and the K scale, per score
  const int base = *a.dpos;
  const int p_lo = split * a.chunk;
  // positions a row m may see: [0, base + m]
  const int live_hi = min(base + a.M, a.max_pos);  // exclusive bound over all rows
  const int p_hi = min(p_lo + a.chunk, live_hi);
  const size_t part_stride = size_t(kPartStride);
  __syncthreads();

  for (int m0 = 0; m0 < a.M; m0 += kRowsPerPass) {
    const int mr = min(kRowsPerPass, a.M - m0);
    // this pass's queries of the group's heads, fp32
    for (int i = threadIdx.x; i < G * mr * kD; i += kThreads) {
      const int h = i / (mr * kD), r = (i / kD) % mr, d = i % kD;
      s_q[(h * kRowsPerPass + r) * kD + d] =
          __bfloat162float(a.q[(size_t(m0 + r) * a.Hq + g * G + h) * kD + d]);
    }
    // per (head of this warp, row): running max, sum and D/32 accumulators
    // (lane owns dims 4*lane .. 4*lane + 3); warp w serves heads w, w + 8
    float mx[2][kRowsPerPass], sm[2][kRowsPerPass], acc[2][kRowsPerPass][4];
#pragma unroll
    for (int hh = 0; hh < 2; ++hh)
#pragma unroll
      for (int r = 0; r < kRowsPerPass; ++r) {
        mx[hh][r] = -INFINITY;
        sm[hh][r] = 0.0f;
#pragma unroll
        for (int c = 0; c < 4; ++c) acc[hh][r][c] = 0.0f;
      }
    for (int p0 = p_lo; p0 < p_hi; p0 += kTile) {
      __syncthreads();  // previous tile consumed; s_q written
      // decode the tile: 32 positions x 128 bytes of K and of V
      for (int i = threadIdx.x; i < kTile * (kD / 4); i += kThreads) {
        const int p = i / (kD / 4), c4 = i % (kD / 4);
        const int pos = p0 + p;
        uint32_t kw = 0u, vw = 0u;
        if (pos < p_hi) {
          const size_t off = (size_t(pos) * a.Hkv + g) * kD + c4 * 4;
          kw = *reinterpret_cast<const uint32_t*>(a.kvk + off);
          vw = *reinterpret_cast<const uint32_t*>(a.kvv + off);
        }
        *reinterpret_cast<float4*>(s_k + p * kKStride + c4 * 4) =
            make_float4(lut[kw & 255u], lut[(kw >> 8) & 255u], lut[(kw >> 16) & 255u], lut[kw >> 24]);
        *reinterpret_cast<float4*>(s_v + p * kD + c4 * 4) =
            make_float4(lut[vw & 255u], lut[(vw >> 8) & 255u], lut[(vw >> 16) & 255u], lut[vw >> 24]);
      }
      __syncthreads();
      const int pos = p0 + lane;  // the position this lane scores
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        const int h = warp + hh * kWarps;
        if (h >= G) break;
#pragma unroll
        for (int r = 0; r < kRowsPerPass; ++r) {
          if (r >= mr) break;
          const float* qv = s_q + (h * kRowsPerPass + r) * kD;
          const float* kv = s_k + lane * kKStride;
          float s = 0.0f;
#pragma unroll 8
          for (int d = 0; d < kD; d += 4) {
            const float4 q4 = *reinterpret_cast<const float4*>(qv + d);
            const float4 k4 = *reinterpret_cast<const float4*>(kv + d);
            s = fmaf(q4.x, k4.x, s);
            s = fmaf(q4.y, k4.y, s);
            s = fmaf(q4.z, k4.z, s);
            s = fmaf(q4.w, k4.w, s);
          }
          // a row whose own position lies outside the cache attends to nothing
          // (the reference skips it), so it merges to zeros
          const int row_pos = base + m0 + r;
          const bool live = pos < p_hi && pos <= row_pos && row_pos < a.max_pos && base >= 0;
          const float x = live ? s * qscale : -INFINITY;
          float tmax = x;
#pragma unroll
          for (int off = 16; off >= 1; off >>= 1) tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, off));
          if (tmax == -INFINITY) continue;  // no live position in this tile for the row
          const float nmax = fmaxf(mx[hh][r], tmax);
          const float corr = expf(mx[hh][r] - nmax);   // 0 on the first live tile
          const float w = live ? expf(x - nmax) : 0.0f;
          float wsum = w;
#pragma unroll
          for (int off = 16; off >= 1; off >>= 1) wsum += __shfl_xor_sync(0xffffffffu, wsum, off);
          sm[hh][r] = sm[hh][r] * corr + wsum;
          mx[hh][r] = nmax;
          float a0 = acc[hh][r][0] * corr, a1 = acc[hh][r][1] * corr;
          float a2 = acc[hh][r][2] * corr, a3 = acc[hh][r][3] * corr;
#pragma unroll 8
          for (int p = 0; p < kTile; ++p) {
            const float wp = __shfl_sync(0xffffffffu, w, p);
            const float4 v4 = *reinterpret_cast<const float4*>(s_v + p * kD + lane * 4);
            a0 = fmaf(wp, v4.x, a0);
            a1 = fmaf(wp, v4.y, a1);
            a2 = fmaf(wp, v4.z, a2);
            a3 = fmaf(wp, v4.w, a3);
          }
          acc[hh][r][0] = a0;
          acc[hh][r][1] = a1;
          acc[hh][r][2] = a2;
          acc[hh][r][3] = a3;
        }
      }
    }
    // partials of this split (empty ones too: max -inf, sum 0)
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
      const int h = warp + hh * kWarps;
      if (h >= G) break;
      for (int r = 0; r < mr; ++r) {
        float* pp = a.part + ((size_t(m0 + r) * a.Hq + g * G + h) * a.nsplit + split) * part_stride;
        *reinterpret_cast<float4*>(pp + lane * 4) =
            make_float4(acc[hh][r][0] * vs, acc[hh][r][1] * vs, acc[hh][r][2] * vs,
                        acc[hh][r][3] * vs);
        if (lane == 0) {
          pp[kD] = mx[hh][r];
          pp[kD + 1] = sm[hh][r];
        }
      }
    }
    __syncthreads();  // s_q is rewritten by the next pass
  }
}

// One CTA of D threads per (row, head): o = sum_j acc_j e^(max_j - M) /
// sum_j sum_j e^(max_j - M), M the largest split maximum.  A row whose base
// position lies outside the cache has no live position and gets zeros.
constexpr int kMaxSplits = 1024;

__global__ void __launch_bounds__(kD) attn_merge_kernel(AttnArgs a_all) {
  const AttnArgs a = for_sequence(a_all, blockIdx.z);
  const int m = blockIdx.x, h = blockIdx.y, d = threadIdx.x;
  const float* pp = a.part + (size_t(m) * a.Hq + h) * a.nsplit * size_t(kPartStride);
  // every split's (max, sum) staged in shared memory by the whole block, the
  // largest maximum by a block reduction, then each split's weight
  // e^(max_j - M); the accumulators are read with independent loads
  __shared__ float s_c[kMaxSplits], s_den[kMaxSplits];
  __shared__ float s_red[kD / 32];
  float lmax = -INFINITY;
  for (int j = d; j < a.nsplit; j += kD) {
    s_c[j] = pp[j * kPartStride + kD];
    s_den[j] = pp[j * kPartStride + kD + 1];
    lmax = fmaxf(lmax, s_c[j]);
  }
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) lmax = fmaxf(lmax, __shfl_xor_sync(0xffffffffu, lmax, off));
  if ((d & 31) == 0) s_red[d >> 5] = lmax;
  __syncthreads();
  float gmax = s_red[0];
#pragma unroll
  for (int w = 1; w < kD / 32; ++w) gmax = fmaxf(gmax, s_red[w]);
  for (int j = d; j < a.nsplit; j += kD)
    s_c[j] = (gmax == -INFINITY || s_c[j] == -INFINITY) ? 0.0f : expf(s_c[j] - gmax);
  __syncthreads();
  float num = 0.0f, den = 0.0f;
#pragma unroll 8
  for (int j = 0; j < a.nsplit; ++j) {
    const float c = s_c[j];
    num = fmaf(pp[j * kPartStride + d], c, num);
    den = fmaf(s_den[j], c, den);
  }
  a.o[(size_t(m) * a.Hq + h) * kD + d] = den > 0.0f ? num / den : 0.0f;
}

// Split layout from max_pos: about two CTAs per SM over the KV heads, at
// least one 32-position tile per split.
void split_layout(int max_pos, int Hkv, int n_seq, int& nsplit, int& chunk) {
  const int per = Hkv * n_seq;  // CTAs per split
  const int target = (2 * 148 + per - 1) / per;
  chunk = (max_pos + target - 1) / target;
  chunk = (chunk + kTile - 1) / kTile * kTile;
  if (chunk < kTile) chunk = kTile;
  nsplit = (max_pos + chunk - 1) / chunk;
}

int check_shapes(int M, int Hq, int Hkv, int D, int max_pos) {
  if (M <= 0 || Hq <= 0 || Hkv <= 0 || max_pos <= 0)
    return set_last_error(MFI_ERR_ARG, "M, Hq, Hkv and max_pos must be positive");
  if (D != kD) return set_last_error(MFI_ERR_ARG, "head_dim must be 128 (as the reference kernels)");
  if (Hq % Hkv != 0 || Hq / Hkv > kMaxGroup)
    return set_last_error(MFI_ERR_ARG, "Hq must be a multiple of Hkv, at most 16 query heads per KV head");
  return MFI_OK;
}

}  // namespace
}  // namespace mfi

extern "C" int mfi_kv_write(const void* k, const void* v, uint8_t* kvk, uint8_t* kvv,
                            const int32_t* dpos, int M, int Hkv, int D, int max_pos,
                            const float* k_scale, const float* v_scale, void* stream) {
  if (M < 0 || Hkv <= 0 || D <= 0 || D % 8 != 0 || max_pos <= 0)
    return mfi::set_last_error(MFI_ERR_ARG, "kv_write: M >= 0, Hkv, max_pos > 0 and D a multiple of 8");
  if (!k || !v || !kvk || !kvv || !dpos) return mfi::set_last_error(MFI_ERR_ARG, "null pointer");
  if ((k_scale == nullptr) != (v_scale == nullptr))
    return mfi::set_last_error(MFI_ERR_ARG, "kv_write: give both scales or neither");
  if ((reinterpret_cast<uintptr_t>(k) & 15) || (reinterpret_cast<uintptr_t>(v) & 15) ||
      (reinterpret_cast<uintptr_t>(kvk) & 7) || (reinterpret_cast<uintptr_t>(kvv) & 7))
    return mfi::set_last_error(MFI_ERR_ARG, "kv_write: k, v 16-byte and kvk, kvv 8-byte aligned");
  if (M == 0) return MFI_OK;
  const long long n8 = (long long)M * Hkv * D / 8;
  mfi::kv_write_kernel<<<unsigned((n8 + 255) / 256), 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      reinterpret_cast<const __nv_bfloat16*>(k), reinterpret_cast<const __nv_bfloat16*>(v), kvk, kvv,
      dpos, M, Hkv, D, max_pos, k_scale, v_scale);
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? MFI_OK
                          : mfi::set_last_error(MFI_ERR_CUDA, cudaGetErrorString(e));
}

extern "C" size_t mfi_attn_decode_batched_workspace_bytes(int n_seq, int M, int Hq, int Hkv,
                                                         int D, int max_pos) {
  if (n_seq <= 0 || M <= 0 || Hq <= 0 || Hkv <= 0 || D <= 0 || max_pos <= 0) return 0;
  int nsplit, chunk;
  mfi::split_layout(max_pos, Hkv, n_seq, nsplit, chunk);
  return size_t(n_seq) * M * Hq * nsplit * mfi::kPartStride * sizeof(float);
}

extern "C" size_t mfi_attn_decode_workspace_bytes(int M, int Hq, int Hkv, int D, int max_pos) {
  return mfi_attn_decode_batched_workspace_bytes(1, M, Hq, Hkv, D, max_pos);
}

extern "C" int mfi_attn_decode_batched(const void* q, const uint8_t* kvk, const uint8_t* kvv,
                                       long long kv_seq_stride, const int32_t* dpos, float* o,
                                       int n_seq, int M, int Hq, int Hkv, int D, int max_pos,
                                       const float* k_scale, const float* v_scale,
                                       void* workspace, size_t workspace_bytes, void* stream) {
  int rc = mfi::check_shapes(M, Hq, Hkv, D, max_pos);
  if (rc != MFI_OK) return rc;
  if (n_seq <= 0 || n_seq > 65535) return mfi::set_last_error(MFI_ERR_ARG, "n_seq must be in [1, 65535]");
  if (!q || !kvk || !kvv || !dpos || !o || !workspace)
    return mfi::set_last_error(MFI_ERR_ARG, "null pointer");
  if ((k_scale == nullptr) != (v_scale == nullptr))
    return mfi::set_last_error(MFI_ERR_ARG, "attn_decode: give both scales or neither");
  if ((reinterpret_cast<uintptr_t>(kvk) & 3) || (reinterpret_cast<uintptr_t>(kvv) & 3) ||
      (kv_seq_stride & 3) || (reinterpret_cast<uintptr_t>(o) & 15) ||
      (reinterpret_cast<uintptr_t>(workspace) & 15))
    return mfi::set_last_error(MFI_ERR_ARG,
                               "attn_decode: kvk, kvv and the sequence stride 4-byte, o and the "
                               "workspace 16-byte aligned");
  if (n_seq > 1 && kv_seq_stride < (long long)max_pos * Hkv * D)
    return mfi::set_last_error(MFI_ERR_ARG, "attn_decode: sequence caches overlap");
  if (workspace_bytes < mfi_attn_decode_batched_workspace_bytes(n_seq, M, Hq, Hkv, D, max_pos))
    return mfi::set_last_error(MFI_ERR_WORKSPACE, "workspace smaller than the attn_decode workspace query");
  mfi::AttnArgs a{};
  a.q = reinterpret_cast<const __nv_bfloat16*>(q);
  a.kvk = kvk;
  a.kvv = kvv;
  a.kv_seq_stride = kv_seq_stride;
  a.dpos = dpos;
  a.k_scale = k_scale;
  a.v_scale = v_scale;
  a.part = static_cast<float*>(workspace);
  a.o = o;
  a.M = M;
  a.Hq = Hq;
  a.Hkv = Hkv;
  a.max_pos = max_pos;
  mfi::split_layout(max_pos, Hkv, n_seq, a.nsplit, a.chunk);
  a.inv_sqrt_d = 1.0f / sqrtf(float(D));
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  cudaError_t e = mfi::ensure_dynamic_smem(reinterpret_cast<const void*>(mfi::attn_partial_kernel),
                                           mfi::kAttnSmem);
  if (e != cudaSuccess) return mfi::set_last_error(MFI_ERR_CUDA, cudaGetErrorString(e));
  mfi::attn_partial_kernel<<<dim3(a.nsplit, Hkv, n_seq), mfi::kThreads, mfi::kAttnSmem, st>>>(a);
  e = cudaGetLastError();
  if (e == cudaSuccess) {
    mfi::attn_merge_kernel<<<dim3(M, Hq, n_seq), mfi::kD, 0, st>>>(a);
    e = cudaGetLastError();
  }
  return e == cudaSuccess ? MFI_OK
                          : mfi::set_last_error(MFI_ERR_CUDA, cudaGetErrorString(e));
}

extern "C" int mfi_attn_decode(const void* q, const uint8_t* kvk, const uint8_t* kvv,
                               const int32_t* dpos, float* o, int M, int Hq, int Hkv, int D,
                               int max_pos, const float* k_scale, const float* v_scale,
                               void* workspace, size_t workspace_bytes, void* stream) {
  return mfi_attn_decode_batched(q, kvk, kvv, 0, dpos, o, 1, M, Hq, Hkv, D, max_pos, k_scale,
                                 v_scale, workspace, workspace_bytes, stream);
}
