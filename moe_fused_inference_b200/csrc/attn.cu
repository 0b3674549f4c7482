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
//   attn_partial_kernel  CTA (split j, KV head g, sequence): decodes its
//                        positions tile by tile (128 at a time) to fp16 in
//                        shared memory once and serves every query head of
//                        the group and every query row from it on the tensor
//                        cores (mma.sync m16n8k16: scores Q.K^T, then P.V,
//                        per warp 16 positions with an online softmax), the
//                        warps merged in shared memory, one partial (max,
//                        sum, D accumulators) per (row, head, split) written
//                        to the workspace;
//   attn_merge_kernel    per (row, head): log-sum-exp merge of the splits,
//                        launched with programmatic serialization.
// Splits are sized from max_pos (the host does not know the device-side base
// position); CTAs past the live positions write empty partials.
//
// Two FP8 formats:
//  * scale == NULL: the reference's own codec, bit for bit.  Its encoder
//    (f32_to_e4m3, mxfp4_decode.cu:447-466) rounds the 3-bit mantissa half
//    away from zero, encodes values below 2^-6 as round(a * 64) (0 or 1) and
//    saturates anything that rounds to 2^8 or more to 0x7F; its decoder
//    (e4m3_to_f32, :362-371) reads exponent 0 as m * 2^-6 and exponent 15 as
//    448 * (1 + m/8).  ref_e4m3x2_f16x2 restates that decoder (bit shift
//    and one exact fp16 multiply per pair).
//  * per-KV-head fp32 scales: the standard E4M3 (e4m3fn) encoding of x/scale,
//    round to nearest even with saturation to +-448 (cvt.rn.satfinite), and
//    its exact decoding times the scale — the per-head scale the model
//    configuration asks for (the reference has none,
//    runtime/model_runner_v2.py:39).
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>

#include <cmath>

#include "../../include/moe_fp4.h"
#include "tc_ptx.cuh"
#include "tmap.cuh"
#include "work.cuh"

namespace mfi {
namespace {

constexpr int kD = 128;          // head dimension (the reference kernels assume 128)
constexpr int kMaxGroup = 16;    // query heads per KV head
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

// ---- tensor-core partial kernel ----------------------------------------------
// CTA (split j, KV head g, sequence s), 8 warps.  Positions [p_lo, p_hi) of the
// split go through shared memory in tiles of kAT = 128: the FP8 bytes are
// decoded to fp16 (exact for both codecs: every E4M3 value, the reference's
// 448 (1 + m/8) and m 2^-6 included, has at most 7 significant bits and lies in
// the fp16 range) into rows of 256 bytes whose 16-byte chunk c of row r sits at
// chunk c ^ (r & 7), so that ldmatrix reads 8 rows without bank conflicts.
// The query vectors of the group (vector v = m * G + h: row m of head g*G + h)
// are taken 16 at a time as the M = 16 side of mma.m16n8k16:
//   S (16 vectors x 16 positions) = Q . K^T     per warp: its 16 positions
//   O (16 vectors x 128 dims)    += P . V       of each tile
// fp16 operands and fp32 accumulation.  Q (bf16) and P (fp32 in [0, 1]) are
// split into fp16 high and low parts, x = hi + lo with |x - hi - lo| <= 2^-22 |x|
// (|q| below 65504), and multiplied twice, so the products are those of fp32
// operands to about 2^-22; K and V are exact.  Each warp keeps its own running
// maximum / sum (online softmax over its tiles); the 8 warps are merged in
// shared memory in warp order and the CTA writes one partial per vector.
constexpr int kAT = 128;               // positions per tile (16 per warp)
constexpr int kAWarps = 8;
constexpr int kAThreads = kAWarps * 32;
constexpr int kRowBytes = kD * 2;      // one fp16 row
constexpr size_t kSmK = size_t(kAT) * kRowBytes;     // 32 KB
constexpr size_t kSmV = kSmK;                        // 32 KB
// the warps' accumulators for the merge reuse the tiles' memory; rows padded
// to 136 floats so the fragment stores spread over the banks
constexpr int kAccStride = kD + 8;
constexpr size_t kSmAcc = size_t(kAWarps) * 16 * kAccStride * sizeof(float);
constexpr size_t kSmTiles = kSmK + kSmV > kSmAcc ? kSmK + kSmV : kSmAcc;
constexpr size_t kSmQ = size_t(16) * kRowBytes;      // 4 KB (x2: hi, lo)
constexpr size_t kSmML = size_t(kAWarps) * 16 * 2 * sizeof(float);
constexpr size_t kAttnSmem = kSmTiles + 2 * kSmQ + kSmML;

// byte offset of 16-byte chunk c of fp16 row r
__device__ __forceinline__ uint32_t sw_off(int r, int c) {
  return uint32_t(r) * kRowBytes + (uint32_t(c ^ (r & 7)) << 4);
}

// Two E4M3 bytes (low byte -> low half) to fp16x2, standard decoding.
__device__ __forceinline__ uint32_t e4m3x2_f16x2(uint32_t two) {
  uint32_t r;
  asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(r) : "h"(uint16_t(two & 0xFFFFu)));
  return r;
}

// Two bytes b0 (low) and b1 of the reference codec to fp16x2, branch-free:
// the 7 magnitude bits shifted into an fp16's exponent and mantissa fields
// (exponent field = the byte's 4-bit exponent e, mantissa = its 3 bits) read
// 2^(e-15) (1 + m/8), or m/8 2^-14 at e = 0; one fp16 multiply then gives the
// reference's value exactly: x 2^8 for 1 <= e <= 14 ((1 + m/8) 2^(e-7)),
// x 2^11 at e = 0 (m 2^-6), x 448 at e = 15 (448 (1 + m/8)).
__device__ __forceinline__ uint32_t ref_e4m3x2_f16x2(uint32_t two) {
  const uint32_t mag = __byte_perm(two & 0x7F7Fu, 0u, 0x4140u) << 7;  // [b0 & 0x7F, b1 & 0x7F] << 7
  const uint32_t sgn = __byte_perm(two & 0x8080u, 0u, 0x1404u);       // sign bits to 15 and 31
  const uint32_t ef = mag & 0x3C003C00u;                                // exponent fields
  const uint32_t is0 = __vcmpeq2(ef, 0u), is15 = __vcmpeq2(ef, 0x3C003C00u);
  const uint32_t mul = (0x5C005C00u & ~(is0 | is15)) | (0x68006800u & is0) | (0x5F005F00u & is15);
  const __half2 r = __hmul2(*reinterpret_cast<const __half2*>(&mag),
                            *reinterpret_cast<const __half2*>(&mul));
  return *reinterpret_cast<const uint32_t*>(&r) | sgn;
}

// 16 FP8 bytes -> 16 fp16 values (two 16-byte chunks).
__device__ __forceinline__ void decode16(const uint4 raw, bool ref, uint4& lo, uint4& hi) {
  const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
  uint32_t o[8];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    o[2 * i] = ref ? ref_e4m3x2_f16x2(w[i]) : e4m3x2_f16x2(w[i]);
    o[2 * i + 1] = ref ? ref_e4m3x2_f16x2(w[i] >> 16) : e4m3x2_f16x2(w[i] >> 16);
  }
  lo = make_uint4(o[0], o[1], o[2], o[3]);
  hi = make_uint4(o[4], o[5], o[6], o[7]);
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t (&r)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t (&r)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
// D (16x8 fp32) += A (16x16 fp16, row) . B (16x8 fp16, col)
__device__ __forceinline__ void mma_f16(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                        uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint32_t pack_f16x2(float lo, float hi) {
  const __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&h);
}
// x = hi + lo in fp16, hi = fp16(x), lo = fp16(x - hi)
__device__ __forceinline__ void split_f16x2(float x0, float x1, uint32_t& hi, uint32_t& lo) {
  const __half2 h = __floats2half2_rn(x0, x1);
  const float2 hf = __half22float2(h);
  hi = *reinterpret_cast<const uint32_t*>(&h);
  lo = pack_f16x2(x0 - hf.x, x1 - hf.y);
}

__global__ void __launch_bounds__(kAThreads, 1) attn_partial_kernel(AttnArgs a_all) {
  const AttnArgs a = for_sequence(a_all, blockIdx.z);
  extern __shared__ __align__(128) uint8_t smem_b[];
  uint8_t* s_k = smem_b;
  uint8_t* s_v = s_k + kSmK;
  uint8_t* s_qh = smem_b + kSmTiles;
  uint8_t* s_ql = s_qh + kSmQ;
  float* s_ml = reinterpret_cast<float*>(s_ql + kSmQ);  // [warp][16 rows][max, sum]
  float* s_acc = reinterpret_cast<float*>(smem_b);      // [warp][16 rows][kD], after the tiles
  const int split = blockIdx.x, g = blockIdx.y;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int gid = lane >> 2, tig = lane & 3;
  const int G = a.Hq / a.Hkv;
  const int NV = G * a.M;
  const bool ref = a.k_scale == nullptr;
  const float ks = ref ? 1.0f : a.k_scale[g];
  const float vs = ref ? 1.0f : a.v_scale[g];
  const float qscale = a.inv_sqrt_d * ks;
  const int base = *a.dpos;
  const int p_lo = split * a.chunk;
  const int live_hi = min(base + a.M, a.max_pos);  // exclusive bound over all rows
  const int p_hi = min(p_lo + a.chunk, live_hi);
  const uint32_t k_base = tc::smem_u32(s_k), v_base = tc::smem_u32(s_v);
  const uint32_t qh_base = tc::smem_u32(s_qh), ql_base = tc::smem_u32(s_ql);

  for (int v0 = 0; v0 < NV; v0 += 16) {
    // the 16 query vectors of this pass as fp16 hi / lo rows (zero rows past NV)
    for (int i = threadIdx.x; i < 16 * (kD / 8); i += kAThreads) {
      const int r = i / (kD / 8), c = i % (kD / 8);  // row, 16-byte chunk (8 dims)
      const int v = v0 + r;
      uint32_t hi[4] = {0u, 0u, 0u, 0u}, lo[4] = {0u, 0u, 0u, 0u};
      if (v < NV) {
        const int m = v / G, h = v % G;
        const uint4 qr = *reinterpret_cast<const uint4*>(
            a.q + (size_t(m) * a.Hq + size_t(g) * G + h) * kD + c * 8);
        const __nv_bfloat162* q2 = reinterpret_cast<const __nv_bfloat162*>(&qr);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float2 f = __bfloat1622float2(q2[j]);
          split_f16x2(f.x, f.y, hi[j], lo[j]);
        }
      }
      *reinterpret_cast<uint4*>(s_qh + sw_off(r, c)) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
      *reinterpret_cast<uint4*>(s_ql + sw_off(r, c)) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
    }
    // this thread's two rows of the C fragments: vectors v0 + gid and v0 + gid + 8
    int row_pos[2];
#pragma unroll
    for (int hr = 0; hr < 2; ++hr) {
      const int v = v0 + gid + 8 * hr;
      const int m = v / G;
      const int rp = base + m;
      // a row whose own position lies outside the cache attends to nothing
      row_pos[hr] = (v < NV && base >= 0 && rp < a.max_pos) ? rp : -1;
    }
    float mx[2] = {-INFINITY, -INFINITY}, sm[2] = {0.0f, 0.0f};
    float o[16][4];
#pragma unroll
    for (int n = 0; n < 16; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.0f;

    for (int t0 = p_lo; t0 < p_hi; t0 += kAT) {
      __syncthreads();  // the previous tile is consumed (and the queries written)
      // decode: 128 positions x 8 raw chunks of 16 bytes, for K and for V
      {
        uint4 rk[4], rv[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int i = threadIdx.x + u * kAThreads;
          const int p = i >> 3, c = i & 7;
          const int pos = t0 + p;
          rk[u] = rv[u] = make_uint4(0u, 0u, 0u, 0u);
          if (pos < p_hi) {
            const size_t off = (size_t(pos) * a.Hkv + g) * kD + c * 16;
            rk[u] = __ldg(reinterpret_cast<const uint4*>(a.kvk + off));
            rv[u] = __ldg(reinterpret_cast<const uint4*>(a.kvv + off));
          }
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int i = threadIdx.x + u * kAThreads;
          const int p = i >> 3, c = i & 7;
          uint4 lo, hi;
          decode16(rk[u], ref, lo, hi);
          *reinterpret_cast<uint4*>(s_k + sw_off(p, 2 * c)) = lo;
          *reinterpret_cast<uint4*>(s_k + sw_off(p, 2 * c + 1)) = hi;
          decode16(rv[u], ref, lo, hi);
          *reinterpret_cast<uint4*>(s_v + sw_off(p, 2 * c)) = lo;
          *reinterpret_cast<uint4*>(s_v + sw_off(p, 2 * c + 1)) = hi;
        }
      }
      __syncthreads();
      const int wp0 = warp * 16;  // this warp's 16 positions inside the tile
      if (t0 + wp0 >= p_hi) continue;
      // S = Q . K^T for 16 vectors x 16 positions
      float s[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll
      for (int kk = 0; kk < kD / 16; ++kk) {
        uint32_t qa[4], ql[4], kb[4];
        const int qr = (lane & 7) + ((lane >> 3) & 1) * 8, qc = 2 * kk + (lane >> 4);
        ldsm_x4(qh_base + sw_off(qr, qc), qa);
        ldsm_x4(ql_base + sw_off(qr, qc), ql);
        const int kr = wp0 + (lane & 7) + (lane >> 4) * 8, kc = 2 * kk + ((lane >> 3) & 1);
        ldsm_x4(k_base + sw_off(kr, kc), kb);
        mma_f16(s[0], qa, kb[0], kb[1]);
        mma_f16(s[0], ql, kb[0], kb[1]);
        mma_f16(s[1], qa, kb[2], kb[3]);
        mma_f16(s[1], ql, kb[2], kb[3]);
      }
      // scale, mask, online softmax per row (the 4 lanes of a quad share a row)
      float p[2][4];
#pragma unroll
      for (int hr = 0; hr < 2; ++hr) {
        float x[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int pos = t0 + wp0 + (j >> 1) * 8 + 2 * tig + (j & 1);
          const bool live = pos < p_hi && pos <= row_pos[hr];
          x[j] = live ? s[j >> 1][2 * hr + (j & 1)] * qscale : -INFINITY;
        }
        float tmax = fmaxf(fmaxf(x[0], x[1]), fmaxf(x[2], x[3]));
        tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, 1));
        tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, 2));
        const float nmax = fmaxf(mx[hr], tmax);
        float corr = 1.0f, psum = 0.0f;
        if (nmax == -INFINITY) {
#pragma unroll
          for (int j = 0; j < 4; ++j) p[hr][j] = 0.0f;
        } else {
          corr = expf(mx[hr] - nmax);  // 0 on the row's first live tile
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            p[hr][j] = x[j] == -INFINITY ? 0.0f : expf(x[j] - nmax);
            psum += p[hr][j];
          }
          mx[hr] = nmax;
        }
        psum += __shfl_xor_sync(0xffffffffu, psum, 1);
        psum += __shfl_xor_sync(0xffffffffu, psum, 2);
        sm[hr] = sm[hr] * corr + psum;
#pragma unroll
        for (int n = 0; n < 16; ++n) {
          o[n][2 * hr] *= corr;
          o[n][2 * hr + 1] *= corr;
        }
      }
      // P as the A operand (rows = vectors, k = the 16 positions), hi and lo
      uint32_t ph[4], pl[4];
      split_f16x2(p[0][0], p[0][1], ph[0], pl[0]);  // row gid,     positions 2tig..
      split_f16x2(p[1][0], p[1][1], ph[1], pl[1]);  // row gid + 8
      split_f16x2(p[0][2], p[0][3], ph[2], pl[2]);  // row gid,     positions 8 + 2tig..
      split_f16x2(p[1][2], p[1][3], ph[3], pl[3]);  // row gid + 8
      // O += P . V, 16 dims (two n-tiles) per ldmatrix
#pragma unroll
      for (int q = 0; q < kD / 16; ++q) {
        uint32_t vb[4];
        const int vr = wp0 + (lane & 7) + ((lane >> 3) & 1) * 8, vc = 2 * q + (lane >> 4);
        ldsm_x4_t(v_base + sw_off(vr, vc), vb);
        mma_f16(o[2 * q], ph, vb[0], vb[1]);
        mma_f16(o[2 * q], pl, vb[0], vb[1]);
        mma_f16(o[2 * q + 1], ph, vb[2], vb[3]);
        mma_f16(o[2 * q + 1], pl, vb[2], vb[3]);
      }
    }
    // merge the 8 warps' running states (warp order) and write this split's
    // partial of every vector of the pass
    __syncthreads();  // the tiles are consumed: their memory holds the merge
    if (tig == 0) {
      s_ml[(warp * 16 + gid) * 2] = mx[0];
      s_ml[(warp * 16 + gid) * 2 + 1] = sm[0];
      s_ml[(warp * 16 + gid + 8) * 2] = mx[1];
      s_ml[(warp * 16 + gid + 8) * 2 + 1] = sm[1];
    }
#pragma unroll
    for (int n = 0; n < 16; ++n) {
      *reinterpret_cast<float2*>(s_acc + (warp * 16 + gid) * kAccStride + 8 * n + 2 * tig) =
          make_float2(o[n][0], o[n][1]);
      *reinterpret_cast<float2*>(s_acc + (warp * 16 + gid + 8) * kAccStride + 8 * n + 2 * tig) =
          make_float2(o[n][2], o[n][3]);
    }
    __syncthreads();
    {
      const int r = threadIdx.x >> 4, d0 = (threadIdx.x & 15) * 8;
      float gmax = -INFINITY;
#pragma unroll
      for (int w = 0; w < kAWarps; ++w) gmax = fmaxf(gmax, s_ml[(w * 16 + r) * 2]);
      float den = 0.0f, acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int w = 0; w < kAWarps; ++w) {
        const float mw = s_ml[(w * 16 + r) * 2];
        const float c = (gmax == -INFINITY || mw == -INFINITY) ? 0.0f : expf(mw - gmax);
        den = fmaf(c, s_ml[(w * 16 + r) * 2 + 1], den);
        const float* src = s_acc + (w * 16 + r) * kAccStride + d0;
#pragma unroll
        for (int i = 0; i < 8; ++i) acc[i] = fmaf(c, src[i], acc[i]);
      }
      const int v = v0 + r;
      if (v < NV) {
        const int m = v / G, h = v % G;
        float* pp = a.part + ((size_t(m) * a.Hq + size_t(g) * G + h) * a.nsplit + split) * kPartStride;
        *reinterpret_cast<float4*>(pp + d0) =
            make_float4(acc[0] * vs, acc[1] * vs, acc[2] * vs, acc[3] * vs);
        *reinterpret_cast<float4*>(pp + d0 + 4) =
            make_float4(acc[4] * vs, acc[5] * vs, acc[6] * vs, acc[7] * vs);
        if (d0 == 0) {
          pp[kD] = gmax;
          pp[kD + 1] = den;
        }
      }
    }
  }
  // the merge kernel (launched with programmatic serialization) may start
  // its prologue; it waits for this grid's memory before reading partials
  tc::grid_dep_launch();
}

// One CTA of 256 threads per (row, head): o = sum_j acc_j e^(max_j - M) /
// sum_j sum_j e^(max_j - M), M the largest split maximum.  A row whose base
// position lies outside the cache has no live position and gets zeros.  The
// 8 warps take every 8th split (each lane 4 dims), so each thread issues its
// few accumulator loads at once; the 8 partial sums are added in warp order.
constexpr int kMaxSplits = 1024;
constexpr int kMergeThreads = 256;

__global__ void __launch_bounds__(kMergeThreads) attn_merge_kernel(AttnArgs a_all) {
  tc::grid_dep_wait();  // the partials come from the previous kernel
  const AttnArgs a = for_sequence(a_all, blockIdx.z);
  const int m = blockIdx.x, h = blockIdx.y;
  const int t = threadIdx.x, warp = t >> 5, lane = t & 31;
  const float* pp = a.part + (size_t(m) * a.Hq + h) * a.nsplit * size_t(kPartStride);
  __shared__ float s_c[kMaxSplits], s_den[kMaxSplits];
  __shared__ float s_red[kMergeThreads / 32];
  __shared__ __align__(16) float s_acc[kMergeThreads / 32][kD];
  float lmax = -INFINITY;
  for (int j = t; j < a.nsplit; j += kMergeThreads) {
    s_c[j] = pp[j * kPartStride + kD];
    s_den[j] = pp[j * kPartStride + kD + 1];
    lmax = fmaxf(lmax, s_c[j]);
  }
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) lmax = fmaxf(lmax, __shfl_xor_sync(0xffffffffu, lmax, off));
  if (lane == 0) s_red[warp] = lmax;
  __syncthreads();
  float gmax = s_red[0];
#pragma unroll
  for (int w = 1; w < kMergeThreads / 32; ++w) gmax = fmaxf(gmax, s_red[w]);
  for (int j = t; j < a.nsplit; j += kMergeThreads)
    s_c[j] = (gmax == -INFINITY || s_c[j] == -INFINITY) ? 0.0f : expf(s_c[j] - gmax);
  __syncthreads();
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll 4
  for (int j = warp; j < a.nsplit; j += kMergeThreads / 32) {
    const float c = s_c[j];
    const float4 v = *reinterpret_cast<const float4*>(pp + j * kPartStride + 4 * lane);
    acc.x = fmaf(v.x, c, acc.x);
    acc.y = fmaf(v.y, c, acc.y);
    acc.z = fmaf(v.z, c, acc.z);
    acc.w = fmaf(v.w, c, acc.w);
  }
  *reinterpret_cast<float4*>(&s_acc[warp][4 * lane]) = acc;
  __syncthreads();
  if (t < kD) {
    float num = 0.0f, den = 0.0f;
#pragma unroll
    for (int w = 0; w < kMergeThreads / 32; ++w) num += s_acc[w][t];
    for (int j = 0; j < a.nsplit; ++j) den = fmaf(s_den[j], s_c[j], den);
    a.o[(size_t(m) * a.Hq + h) * kD + t] = den > 0.0f ? num / den : 0.0f;
  }
}

// Split layout from max_pos: about one CTA per SM over the KV heads and
// sequences (one wave), splits a multiple of 16 positions (one warp's share of
// a tile).
void split_layout(int max_pos, int Hkv, int n_seq, int& nsplit, int& chunk) {
  const int per = Hkv * n_seq;  // CTAs per split
  const int target = (148 + per - 1) / per;
  chunk = (max_pos + target - 1) / target;
  chunk = (chunk + 15) / 16 * 16;
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
  // the partial kernel reads q, K and V rows in 16-byte loads
  if ((reinterpret_cast<uintptr_t>(q) & 15) || (reinterpret_cast<uintptr_t>(kvk) & 15) ||
      (reinterpret_cast<uintptr_t>(kvv) & 15) || (kv_seq_stride & 15) ||
      (reinterpret_cast<uintptr_t>(o) & 15) || (reinterpret_cast<uintptr_t>(workspace) & 15))
    return mfi::set_last_error(MFI_ERR_ARG,
                               "attn_decode: q, kvk, kvv, o, the workspace and the sequence "
                               "stride must be 16-byte aligned");
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
  mfi::attn_partial_kernel<<<dim3(a.nsplit, Hkv, n_seq), mfi::kAThreads, mfi::kAttnSmem, st>>>(a);
  e = cudaGetLastError();
  if (e == cudaSuccess) {
    // programmatic serialization: the merge grid is scheduled while the
    // partial kernel finishes and waits (griddepcontrol) for its memory
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(M, Hq, n_seq);
    cfg.blockDim = dim3(mfi::kMergeThreads);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    e = cudaLaunchKernelEx(&cfg, mfi::attn_merge_kernel, a);
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
