// route_tc.cu — the prefill router on the tensor cores.
//
// Same contract as the other routers (route.cu, reference
// runtime/model_runner_v2.py:100-106 with the router GEMM of
// src/ext/mxfp4_linear.cu): the logit of (token t, expert e) is
//
//   sum over 32-element blocks b of  S(t,e,b) * 2^(sx(t,b) + sw(e,b) - 256)
//
// where S is the exact integer dot product of the doubled E2M1 values
// (2 * e2m1 in [-12, 12]) and sx, sw are the E8M0 codes, rounded once to
// fp32.  The other routers add the terms in fp64 in a fixed order (lane l
// sums blocks l, l+32, ..., then an xor butterfly).  Every term is an integer
// below 2^13 times a power of two, so when the exponents of a (t, e) pair
// span at most 34 binades every partial sum of any subset of its 64 terms is
// exact in fp64 (|sum| < 64 * 4608 * 2^34 < 2^53 units of the smallest term):
// the order does not matter and the result is the exact sum rounded to fp32,
// bit for bit what the fixed order gives.
//
// Fast path.  When the codes of a row (a token's 64 blocks, or an expert's)
// span at most 3 binades, its int8 operand carries each block's scale
// relative to the row minimum: 2 * e2m1 * 2^(code - min) stays within
// [-96, 96].  If every token of a CTA's tile and every expert qualify, one
// s32 accumulator sums all 64 blocks inside the tensor core:
//   D(t,e) = sum_b S(t,e,b) * 2^(sx - minx(t) + sw - minw(e)),  |D| < 2^31,
// and logit = float(D) * 2^(minx(t) + minw(e) - 256) is the exact sum
// rounded once to fp32 (int -> fp32 rounds to nearest; the power of two is
// exact while the result is a normal number, which the CTA checks).
//
// Otherwise each block gets its own accumulator (four in TMEM, reused) and
// the epilogue adds D(t,e,b) * 2^(ex + ew - 256) in fp64, with ex, ew the
// effective codes (the row minimum for a scaled row, the block code else).
// |D(t,e,b)| < 2^19, so that sum is order-free while the effective span of a
// pair is at most 28 binades; a token beyond that is recomputed in the fixed
// order (ref_token_logits).  The logits therefore match the other routers
// for every input.
//
//   quant_x8_kernel  one warp per token: bf16 -> E2M1 + E8M0 (xq, xsc, for the
//                    expert kernels) and the int8 operand (scaled as above
//                    when the token qualifies) in the 128-token x
//                    128-element SW128 blocks the MMA reads; extra CTAs
//                    expand the router rows the same way (r8)
//   route_tc_kernel  one CTA per 128 tokens, all 128 experts:
//     warp 0       producer: per 128-element chunk two bulk copies (token
//                  block, router block)
//     warp 1       MMA issue: four tcgen05.mma kind::i8 per chunk (M = N =
//                  128, K = 32, one per 32-element block) into one s32
//                  accumulator (fast path) or four (one per block)
//     warps 2-17   epilogue: warp w holds TMEM lane quadrant w % 4 (32
//                  tokens) and 32 experts
//                  and, for k <= 8, sorts the best k of its 32 logits
//     tail         one thread per token merges its four sorted lists into
//                  the top-k and computes the weights (one warp per token
//                  for k > 8 or a recomputed token); then the CTA claims
//                  each expert's positions with one global atomic per expert
//                  (per-token claims on hot experts would serialise)
#include "mx_common.cuh"
#include "tc_ptx.cuh"
#include "tmap.cuh"
#include "work.cuh"
#include "route_common.cuh"

namespace mfi {

using namespace tc;

namespace {

constexpr int kRtTile = 128;                       // tokens per CTA (MMA M)
constexpr int kRtE = 128;                          // experts (MMA N)
constexpr int kRtMaxBlk = 64;                      // H <= 2048
constexpr int kRtStages = 4;
constexpr int kRtBlock = 128 * 128;                // int8 rows of one 128-element chunk
constexpr int kRtStageBytes = 2 * kRtBlock;        // token block + router block
constexpr int kRtEpiWarps = 16;
constexpr int kRtWarps = 2 + kRtEpiWarps;
constexpr int kRtThreads = 32 * kRtWarps;          // 576
constexpr int kRtLgStride = kRtE + 1;              // fp32 logits rows in the tail
constexpr int kRtXscStride = kRtMaxBlk + 4;        // token codes rows (conflict-free reads)
constexpr int kRtMaxK = 8;                         // per-thread top-k lists; larger k: warp top-k
constexpr int kShiftMax = 3;                       // row code span folded into int8
constexpr int kExactSpreadEff = 28;                // per-block fp64: order-free span
constexpr uint32_t kRtTmemCols = 512;              // four 128-column accumulators

constexpr size_t kRtOffSel = size_t(kRtTile) * kRtLgStride * 4;      // int [128][32] (tail)
constexpr size_t kRtOffLoc = kRtOffSel + size_t(kRtTile) * 32 * 4;  // int [128][32] (tail)
constexpr size_t kRtOffCv = kRtOffLoc + size_t(kRtTile) * 32 * 4;   // float [128][4][8] (tail)
constexpr size_t kRtOffCi = kRtOffCv + size_t(kRtTile) * 4 * kRtMaxK * 4;  // uint8 [128][4][8]
constexpr size_t kRtOffSwh = size_t(kRtStages) * kRtStageBytes;     // int32 [64][128]
constexpr size_t kRtOffXsc = kRtOffSwh + size_t(kRtMaxBlk) * kRtE * 4;
constexpr size_t kRtOffBar = kRtOffXsc + size_t(kRtTile) * kRtXscStride;
constexpr size_t kRtSmem = 1024 + kRtOffBar + 8 * (2 * kRtStages + 8) + 16;
static_assert(kRtOffCi + size_t(kRtTile) * 4 * kRtMaxK <= kRtOffSwh, "tail arrays alias the ring");

constexpr int kQxThreads = 256;                    // quant_x8_kernel: one warp per token
constexpr int kQxTok = kQxThreads / 32;
constexpr int kQxRouterCtas = 16;

// Byte offset of 16-byte chunk q of row r inside a 128-row SW128 block.
__device__ __forceinline__ uint32_t sw128_off(int r, int q) {
  return uint32_t(r >> 3) * 1024u + uint32_t(r & 7) * 128u + uint32_t((q ^ (r & 7)) * 16);
}

// 8 nibbles -> two words of 4 int8 each, value 2 * e2m1 * 2^sh, sh in
// [0, kShiftMax] (magnitudes up to 96: the byte tables shift without carry).
__device__ __forceinline__ void nib8_to_i8_shift(uint32_t w, int sh, uint32_t& lo, uint32_t& hi) {
  const uint32_t P0 = 0x03020100u << sh, P1 = 0x0C080604u << sh;  // 0 1 2 3 | 4 6 8 12
  const uint32_t N0 = __vneg4(P0), N1 = __vneg4(P1);
  const uint32_t m = w & 0x77777777u;         // magnitude selectors
  const uint32_t s = (w >> 1) & 0x44444444u;  // sign bit -> selector bit 2
  const uint32_t pl = __byte_perm(P0, P1, m & 0xFFFFu);
  const uint32_t nl = __byte_perm(N0, N1, m & 0xFFFFu);
  lo = __byte_perm(pl, nl, 0x3210u | (s & 0xFFFFu));
  const uint32_t ph = __byte_perm(P0, P1, m >> 16);
  const uint32_t nh = __byte_perm(N0, N1, m >> 16);
  hi = __byte_perm(ph, nh, 0x3210u | (s >> 16));
}

// 32 packed E2M1 values (16 bytes) -> their int8 operand values, stored as
// chunks 2u and 2u + 1 of row r of an SW128 block.
__device__ __forceinline__ void store_i8_row_part(uint8_t* block, int r, int u, const uint4& q,
                                                  int sh) {
  uint32_t w[8];
  nib8_to_i8_shift(q.x, sh, w[0], w[1]);
  nib8_to_i8_shift(q.y, sh, w[2], w[3]);
  nib8_to_i8_shift(q.z, sh, w[4], w[5]);
  nib8_to_i8_shift(q.w, sh, w[6], w[7]);
  *reinterpret_cast<uint4*>(block + sw128_off(r, 2 * u)) = make_uint4(w[0], w[1], w[2], w[3]);
  *reinterpret_cast<uint4*>(block + sw128_off(r, 2 * u + 1)) = make_uint4(w[4], w[5], w[6], w[7]);
}

// Smallest / largest byte of the 16 codes in v.
__device__ __forceinline__ int min_code(const uint4& v) {
  const uint32_t m = __vminu4(__vminu4(v.x, v.y), __vminu4(v.z, v.w));
  return min(min(int(m & 255u), int((m >> 8) & 255u)), min(int((m >> 16) & 255u), int(m >> 24)));
}
__device__ __forceinline__ int max_code(const uint4& v) {
  const uint32_t m = __vmaxu4(__vmaxu4(v.x, v.y), __vmaxu4(v.z, v.w));
  return max(max(int(m & 255u), int((m >> 8) & 255u)), max(int((m >> 16) & 255u), int(m >> 24)));
}

// ---------------------------------------------------------------------------
// Quantise the tokens (rows [T, ceil(T/128)*128) of x8 become zeros) and
// expand the router rows.
__global__ void __launch_bounds__(kQxThreads) quant_x8_kernel(RouteArgs a, int n_tok_ctas) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nb = a.H >> 5, nchunk = a.H >> 7;
  if (int(blockIdx.x) < n_tok_ctas) {
    // lane l quantises blocks l and l + 32 whole (the arithmetic of
    // quant_group8: block maximum, NaN -> code 127, nibbles at 2^-e)
    const int t = blockIdx.x * kQxTok + warp;  // < ceil(T/128) * 128
    const int tt = t < a.T ? t : -1;
    // RMSNorm factor of the row when a norm weight is given (route_common.cuh)
    const float rms_r = (a.norm_w && tt >= 0) ? warp_rms_inv(a, tt, lane) : 1.0f;
    uint4 packed[kRtMaxBlk / 32];
    int code[kRtMaxBlk / 32];
    int lo = 255, hi = 0;
#pragma unroll
    for (int jb = 0; jb < kRtMaxBlk / 32; ++jb) {
      const int b = lane + 32 * jb;
      code[jb] = 127;
      packed[jb] = make_uint4(0u, 0u, 0u, 0u);
      if (b >= nb) continue;
      float v[32];
      if (tt >= 0) {
        const uint4* src = reinterpret_cast<const uint4*>(
            reinterpret_cast<const __nv_bfloat16*>(a.x) + long(tt) * a.H + b * 32);
        uint4 raw[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) raw[q] = src[q];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const __nv_bfloat162* h2 = reinterpret_cast<const __nv_bfloat162*>(&raw[q]);
          float u[8];
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const float2 f = __bfloat1622float2(h2[i]);
            u[2 * i] = f.x;
            u[2 * i + 1] = f.y;
          }
          if (a.norm_w) rms_apply8(a, b * 32 + q * 8, rms_r, u);
#pragma unroll
          for (int i = 0; i < 8; ++i) v[q * 8 + i] = u[i];
        }
      } else {
#pragma unroll
        for (int i = 0; i < 32; ++i) v[i] = 0.0f;
      }
      float am = 0.0f;
      bool nan = false;
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        am = fmaxf(am, fabsf(v[i]));
        nan |= (v[i] != v[i]);
      }
      const BlockScale bs = block_scale(nan ? __uint_as_float(0x7fc00000u) : am);
      uint32_t w[4] = {0u, 0u, 0u, 0u};
#pragma unroll
      for (int i = 0; i < 32; ++i) w[i >> 3] |= quant_nibble(v[i], bs.inv) << (4 * (i & 7));
      packed[jb] = make_uint4(w[0], w[1], w[2], w[3]);
      code[jb] = bs.code;
      lo = min(lo, int(bs.code));
      hi = max(hi, int(bs.code));
    }
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) {
      lo = min(lo, __shfl_xor_sync(0xffffffffu, lo, off));
      hi = max(hi, __shfl_xor_sync(0xffffffffu, hi, off));
    }
    const bool scaled = hi - lo <= kShiftMax;
    uint8_t* x8t = a.x8 + size_t(t / kRtTile) * nchunk * kRtBlock;
#pragma unroll
    for (int jb = 0; jb < kRtMaxBlk / 32; ++jb) {
      const int b = lane + 32 * jb;
      if (b >= nb) continue;
      if (tt >= 0) {
        reinterpret_cast<uint4*>(a.xq + long(tt) * (a.H >> 1))[b] = packed[jb];
        a.xsc[long(tt) * nb + b] = uint8_t(code[jb]);
      }
      store_i8_row_part(x8t + size_t(b >> 2) * kRtBlock, t % kRtTile, b & 3, packed[jb],
                        scaled ? code[jb] - lo : 0);
    }
  } else {
    // one warp per expert
    for (int e = (blockIdx.x - n_tok_ctas) * kQxTok + warp; e < a.E; e += kQxRouterCtas * kQxTok) {
      int lo = 255, hi = 0;
      for (int b = lane; b < nb; b += 32) {
        lo = min(lo, int(a.sr[long(e) * nb + b]));
        hi = max(hi, int(a.sr[long(e) * nb + b]));
      }
#pragma unroll
      for (int off = 16; off >= 1; off >>= 1) {
        lo = min(lo, __shfl_xor_sync(0xffffffffu, lo, off));
        hi = max(hi, __shfl_xor_sync(0xffffffffu, hi, off));
      }
      const bool scaled = hi - lo <= kShiftMax;
      for (int u = lane; u < nb; u += 32)
        store_i8_row_part(a.r8 + size_t(u >> 2) * kRtBlock, e, u & 3,
                          ldg_u4(a.wr + long(e) * (a.H >> 1) + u * 16),
                          scaled ? int(a.sr[long(e) * nb + u]) - lo : 0);
    }
  }
}

// Compare-exchange: after it, (va, ia) is the better of the two in the
// routers' order (larger value, ties to the lower index).
__device__ __forceinline__ void cex(float& va, int& ia, float& vb, int& ib) {
  const bool sw = better(vb, ib, va, ia);
  const float t = va;
  const int u = ia;
  va = sw ? vb : va;
  ia = sw ? ib : ia;
  vb = sw ? t : vb;
  ib = sw ? u : ib;
}

// Sort 8 entries best first (an optimal 19-comparator network, depth 6).
__device__ __forceinline__ void sort8(float (&v)[8], int (&i)[8]) {
#define MFI_CX(a, b) cex(v[a], i[a], v[b], i[b])
  MFI_CX(0, 2); MFI_CX(1, 3); MFI_CX(4, 6); MFI_CX(5, 7);
  MFI_CX(0, 4); MFI_CX(1, 5); MFI_CX(2, 6); MFI_CX(3, 7);
  MFI_CX(0, 1); MFI_CX(2, 3); MFI_CX(4, 5); MFI_CX(6, 7);
  MFI_CX(2, 4); MFI_CX(3, 5);
  MFI_CX(1, 4); MFI_CX(3, 6);
  MFI_CX(1, 2); MFI_CX(3, 4); MFI_CX(5, 6);
#undef MFI_CX
}

// (v, i) <- the best 8 of two sorted runs, sorted: pairing a[m] with
// b[7 - m] keeps the 8 best as a bitonic sequence, three half-cleaner
// layers sort it.
__device__ __forceinline__ void merge8(float (&v)[8], int (&i)[8], const float (&bv)[8],
                                       const int (&bi)[8]) {
#pragma unroll
  for (int m = 0; m < 8; ++m) {
    const bool sw = better(bv[7 - m], bi[7 - m], v[m], i[m]);
    v[m] = sw ? bv[7 - m] : v[m];
    i[m] = sw ? bi[7 - m] : i[m];
  }
#pragma unroll
  for (int d = 4; d >= 1; d >>= 1)
#pragma unroll
    for (int m = 0; m < 8; ++m)
      if ((m & d) == 0) cex(v[m], i[m], v[m + d], i[m + d]);
}

// Logits of token t in the routers' fixed order (lane l sums blocks l, l+32,
// ... ascending, then the xor butterfly 16..1), plus the logit bias.  One
// warp; used only when the scale span of the token could make the order
// matter.
__device__ void ref_token_logits(const RouteArgs& a, int t, float* s_lg, int lane) {
  const int nb = a.H >> 5;
  const uint8_t* xrow = a.xq + long(t) * (a.H >> 1);
  const uint8_t* xs = a.xsc + long(t) * nb;
  for (int e = 0; e < a.E; ++e) {
    double acc = 0.0;
    for (int bl = lane; bl < nb; bl += 32) {
      const uint4 xv = ldg_u4(xrow + bl * 16);
      const uint4 wv = ldg_u4(a.wr + long(e) * (a.H >> 1) + bl * 16);
      const int s = block_dot_i(xv, wv);
      acc += double(s) * exp2i_d(int(xs[bl]) + int(a.sr[long(e) * nb + bl]) - 256);
    }
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
    if (lane == 0) s_lg[e] = a.logit_bias ? __fadd_rn(float(acc), a.logit_bias[e]) : float(acc);
  }
  __syncwarp();
}

__global__ void __launch_bounds__(kRtThreads, 1) route_tc_kernel(RouteArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* ring = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  int* s_swh = reinterpret_cast<int*>(ring + kRtOffSwh);  // [b][e] = ew(e, b) << 20
  uint8_t* s_xsc = ring + kRtOffXsc;                      // [r][b] effective token codes
  uint64_t* full = reinterpret_cast<uint64_t*>(ring + kRtOffBar);
  uint64_t* empty = full + kRtStages;
  uint64_t* acc_full = empty + kRtStages;
  uint64_t* acc_empty = acc_full + 4;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 4);
  __shared__ int s_xspread[kRtTile];  // effective code span of each token
  __shared__ int s_xminc[kRtTile], s_wminc[kRtE];
  __shared__ int s_wspread, s_unscaled, s_xlo, s_xhi, s_wlo, s_whi, s_failed;
  __shared__ int s_cnt[kRtE], s_base[kRtE];
  __shared__ uint64_t drain[1];  // the MMA issuer's error-path drain

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tile = blockIdx.x, t0 = tile * kRtTile;
  const int nb = a.H >> 5, nchunk = a.H >> 7;
  const int n_tok = min(kRtTile, a.T - t0);

  if (threadIdx.x == 0) {
    for (int s = 0; s < kRtStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 4; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], kRtEpiWarps);
    }
    mbar_init(drain, 1);
    fence_mbar_init();
    cta_abort_init();
    s_wspread = 0;
    s_unscaled = 0;
    s_xlo = 255;
    s_xhi = 0;
    s_wlo = 255;
    s_whi = 0;
  }
  for (int e = threadIdx.x; e < kRtE; e += kRtThreads) s_cnt[e] = 0;
  if (warp == 1) tmem_alloc(tmem_slot, kRtTmemCols);
  __syncthreads();

  // ---- codes: the rows' minima and effective codes -----------------------------
  // 16 codes per thread; the nb / 16 threads of a row are adjacent lanes.  A
  // row whose codes span <= kShiftMax was scaled into its int8 operand
  // (quant_x8_kernel): its effective code is its minimum.
  const int per_row = nb / 16;
  for (int p = threadIdx.x; p < kRtE * per_row; p += kRtThreads) {
    const int e = p / per_row, q = p - e * per_row;
    const uint4 v = ldg_u4(a.sr + long(e) * nb + q * 16);
    int l = min_code(v), h = max_code(v);
    for (int off = 1; off < per_row; off <<= 1) {
      l = min(l, __shfl_xor_sync(0xffffffffu, l, off));
      h = max(h, __shfl_xor_sync(0xffffffffu, h, off));
    }
    const bool scaled = h - l <= kShiftMax;
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int i = 0; i < 16; ++i)
      s_swh[(q * 16 + i) * kRtE + e] = (scaled ? l : int((w[i >> 2] >> (8 * (i & 3))) & 255u)) << 20;
    if (q == 0) {
      s_wminc[e] = l;
      if (!scaled) {
        atomicAdd(&s_unscaled, 1);
        atomicMax(&s_wspread, h - l);
      }
      atomicMin(&s_wlo, l);
      atomicMax(&s_whi, l);
    }
  }
  for (int p = threadIdx.x; p < kRtTile * per_row; p += kRtThreads) {
    const int r = p / per_row, q = p - r * per_row;
    // padding rows (t >= T) are zeros: code 127
    const uint4 v = r < n_tok ? ldg_u4(a.xsc + long(t0 + r) * nb + q * 16)
                              : make_uint4(0x7F7F7F7Fu, 0x7F7F7F7Fu, 0x7F7F7F7Fu, 0x7F7F7F7Fu);
    int l = min_code(v), h = max_code(v);
    for (int off = 1; off < per_row; off <<= 1) {
      l = min(l, __shfl_xor_sync(0xffffffffu, l, off));
      h = max(h, __shfl_xor_sync(0xffffffffu, h, off));
    }
    const bool scaled = h - l <= kShiftMax;
    const uint32_t lb = uint32_t(l) * 0x01010101u;
    uint32_t* dst = reinterpret_cast<uint32_t*>(s_xsc + r * kRtXscStride + q * 16);
    dst[0] = scaled ? lb : v.x;
    dst[1] = scaled ? lb : v.y;
    dst[2] = scaled ? lb : v.z;
    dst[3] = scaled ? lb : v.w;
    if (q == 0) {
      s_xminc[r] = l;
      s_xspread[r] = scaled ? 0 : h - l;
      if (!scaled) atomicAdd(&s_unscaled, 1);
      atomicMin(&s_xlo, l);
      atomicMax(&s_xhi, l);
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  // one accumulator for all blocks: every row scaled, every logit a normal
  // fp32 number (float(D) * 2^k with 1 <= |D| < 2^31)
  const bool fast = s_unscaled == 0 && s_xlo + s_wlo - 256 >= -126 && s_xhi + s_whi - 256 <= 96;

  if (warp == 0) {
    // ---- producer -------------------------------------------------------------
    if (elect_one()) {
      const uint8_t* x8t = a.x8 + size_t(tile) * nchunk * kRtBlock;
      int c = 0;
      for (; c < nchunk; ++c) {
        const int s = c % kRtStages;
        if (!mbar_wait(&empty[s], ((c / kRtStages) & 1) ^ 1, a.err, 6)) break;
        uint8_t* st = ring + s * kRtStageBytes;
        mbar_expect_tx(&full[s], kRtStageBytes);
        bulk_load(st, x8t + size_t(c) * kRtBlock, kRtBlock, &full[s]);
        bulk_load(st + kRtBlock, a.r8 + size_t(c) * kRtBlock, kRtBlock, &full[s]);
      }
      if (c < nchunk) drain_ring(full, kRtStages, uint32_t(c));  // failed: drain our copies
    }
  } else if (warp == 1) {
    // ---- MMA issue --------------------------------------------------------------
    if (elect_one()) {
      const uint32_t idesc = make_idesc_i8(kRtTile, kRtE);
      bool ok = true;
      for (int c = 0; c < nchunk && ok; ++c) {
        const int s = c % kRtStages;
        if (!mbar_wait(&full[s], (c / kRtStages) & 1, a.err, 6)) { ok = false; break; }
        tc_fence_after();
        const uint32_t base = smem_u32(ring + s * kRtStageBytes);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const uint64_t ad = make_sdesc(base + i * 32, 16, 1024, kLayoutSW128);
          const uint64_t bd = make_sdesc(base + kRtBlock + i * 32, 16, 1024, kLayoutSW128);
          if (fast) {
            mma_i8(tmem, ad, bd, idesc, (c | i) != 0 ? 1u : 0u);
          } else {
            // accumulator i takes block 4c + i; its previous use was chunk c - 1
            if (!mbar_wait(&acc_empty[i], (c & 1) ^ 1, a.err, 6)) {
              ok = false;
              break;
            }
            tc_fence_after();
            mma_i8(tmem + i * 128, ad, bd, idesc, 0u);
            tc_commit(&acc_full[i]);
          }
        }
        if (ok) tc_commit(&empty[s]);
      }
      if (ok && fast) tc_commit(&acc_full[0]);
      if (!ok) drain_mma(drain);
    }
  }

  // ---- epilogue ----------------------------------------------------------------
  const int quad = warp & 3, eg = (warp - 2) >> 2;
  const int r = quad * 32 + lane;
  const uint32_t tq = tmem + (uint32_t(quad * 32) << 16) + uint32_t(eg * 32);
  float* s_lg = reinterpret_cast<float*>(ring);
  float lg[32];
  if (warp >= 2 && fast) {
    if (mbar_wait(&acc_full[0], 0, a.err, 6)) {
      tc_fence_after();
      uint32_t d[32];
      tmem_ld_32x32b_x32(tq, d);
      tmem_ld_wait();
      const int kx = s_xminc[r] - 256 + 127;
#pragma unroll
      for (int j = 0; j < 32; ++j)
        lg[j] = __fmul_rn(__int2float_rn(int(d[j])),
                          __int_as_float((kx + s_wminc[eg * 32 + j]) << 23));
    }
  } else if (warp >= 2) {
    // one accumulator per block, added in fp64 (order-free within the span)
    double acc[32];
#pragma unroll
    for (int j = 0; j < 32; ++j) acc[j] = 0.0;
    const uint8_t* my_codes = s_xsc + r * kRtXscStride;
    for (int b = 0; b < nb; ++b) {
      const int buf = b & 3;
      if (!mbar_wait(&acc_full[buf], (b >> 2) & 1, a.err, 6)) break;
      tc_fence_after();
      // 2^(ex + ew - 256) as the high word of a double: (ex + ew + 767) << 20
      const int hx = (int(my_codes[b]) + 767) << 20;
      const int4* sw4 = reinterpret_cast<const int4*>(s_swh + b * kRtE + eg * 32);
      uint32_t d[16];
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        tmem_ld_32x32b_x16(tq + buf * 128 + h * 16, d);
        tmem_ld_wait();
        if (h == 1) {
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&acc_empty[buf]);
        }
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const int4 w = sw4[h * 4 + q];
          const int sc[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
          for (int m = 0; m < 4; ++m)
            acc[h * 16 + q * 4 + m] = fma(double(int(d[q * 4 + m])),
                                          __hiloint2double(hx + sc[m], 0), acc[h * 16 + q * 4 + m]);
        }
      }
    }
#pragma unroll
    for (int j = 0; j < 32; ++j) lg[j] = float(acc[j]);
  }
  tc_fence_before();
  if (threadIdx.x == 0) s_failed = cta_aborted() ? 1 : 0;
  __syncthreads();  // every MMA has been consumed: the ring is free
  float* s_cv = reinterpret_cast<float*>(ring + kRtOffCv);
  uint8_t* s_ci = ring + kRtOffCi;
  if (warp >= 2) {
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      const int e = eg * 32 + j;
      if (a.logit_bias) lg[j] = __fadd_rn(lg[j], a.logit_bias[e]);
      s_lg[r * kRtLgStride + e] = lg[j];
    }
    if (a.k <= kRtMaxK) {
      // the best 8 of this thread's 32 experts in the routers' order (larger
      // first, ties to the lower expert): each run of 8 sorted by a
      // 19-comparator network, runs merged two at a time keeping the top 8
      // (bitonic merge); branch-free, so the warp stays converged
      float tv[8], gv[8];
      int ti[8], gi[8];
#pragma unroll
      for (int m = 0; m < 8; ++m) {
        tv[m] = lg[m];
        ti[m] = eg * 32 + m;
      }
      sort8(tv, ti);
#pragma unroll
      for (int g = 1; g < 4; ++g) {
#pragma unroll
        for (int m = 0; m < 8; ++m) {
          gv[m] = lg[g * 8 + m];
          gi[m] = eg * 32 + g * 8 + m;
        }
        sort8(gv, gi);
        merge8(tv, ti, gv, gi);
      }
#pragma unroll
      for (int m = 0; m < kRtMaxK; ++m)
        if (m < a.k) {
          s_cv[(r * 4 + eg) * kRtMaxK + m] = tv[m];
          s_ci[(r * 4 + eg) * kRtMaxK + m] = uint8_t(ti[m]);
        }
    }
  }
  __syncthreads();
  const bool failed = s_failed != 0;  // uniform over the CTA

  // ---- tail -------------------------------------------------------------------
  int* s_sel = reinterpret_cast<int*>(ring + kRtOffSel);  // [i][j] selected expert
  int* s_loc = reinterpret_cast<int*>(ring + kRtOffLoc);  // [i][j] rank among the CTA's
  if (!failed) {
    if (!fast)
      for (int i = warp; i < n_tok; i += kRtWarps)
        if (s_xspread[i] + s_wspread > kExactSpreadEff)
          ref_token_logits(a, t0 + i, s_lg + i * kRtLgStride, lane);
    __syncthreads();
    if (a.logits)
      for (int p = threadIdx.x; p < n_tok * kRtE; p += kRtThreads)
        a.logits[long(t0) * kRtE + p] = s_lg[(p >> 7) * kRtLgStride + (p & (kRtE - 1))];
    auto recomputed = [&](int i) { return !fast && s_xspread[i] + s_wspread > kExactSpreadEff; };
    if (a.k <= kRtMaxK && int(threadIdx.x) < n_tok && !recomputed(threadIdx.x)) {
      // merge the four sorted lists of the token
      const int i = threadIdx.x, t = t0 + i;
      const float* cv = s_cv + i * 4 * kRtMaxK;
      const uint8_t* ci = s_ci + i * 4 * kRtMaxK;
      int head[4] = {0, 0, 0, 0};
      float pv[kRtMaxK];
      float sum = 0.0f, mx = 0.0f;
#pragma unroll
      for (int j = 0; j < kRtMaxK; ++j) {
        if (j >= a.k) break;
        float bv = 0.0f;
        int be = -1, bg = 0;
#pragma unroll
        for (int g = 0; g < 4; ++g) {
          if (head[g] >= a.k) continue;
          const float v = cv[g * kRtMaxK + head[g]];
          const int e = ci[g * kRtMaxK + head[g]];
          if (be < 0 || better(v, e, bv, be)) {
            bv = v;
            be = e;
            bg = g;
          }
        }
#pragma unroll
        for (int g = 0; g < 4; ++g) head[g] += (g == bg);
        if (j == 0) mx = bv;
        pv[j] = expf(bv - mx);
        sum = __fadd_rn(sum, pv[j]);
        a.topi[long(t) * a.k + j] = be;
        s_sel[i * 32 + j] = be;
      }
#pragma unroll
      for (int j = 0; j < kRtMaxK; ++j)
        if (j < a.k) a.topw[long(t) * a.k + j] = __fdiv_rn(pv[j], sum);
    }
    {
      // one warp per token (bias and logits are done) for k > 8 and for the
      // recomputed tokens
      RouteArgs b = a;
      b.logit_bias = nullptr;
      b.logits = nullptr;
      for (int i = warp; i < n_tok; i += kRtWarps)
        if (a.k > kRtMaxK || recomputed(i))
          finish_token(b, t0 + i, s_lg + i * kRtLgStride, lane, s_sel + i * 32);
    }
    if (a.slot_pos) {
      // positions: rank inside the CTA (shared-memory atomics), then one
      // global claim per expert for the CTA's block of positions
      __syncthreads();
      for (int p = threadIdx.x; p < n_tok * a.k; p += kRtThreads) {
        const int i = p / a.k, j = p - i * a.k;
        s_loc[i * 32 + j] = atomicAdd(&s_cnt[s_sel[i * 32 + j]], 1);
      }
      __syncthreads();
      for (int e = threadIdx.x; e < kRtE; e += kRtThreads)
        if (s_cnt[e] > 0) s_base[e] = atomicAdd(a.cursor + e, s_cnt[e]);
      __syncthreads();
      for (int p = threadIdx.x; p < n_tok * a.k; p += kRtThreads) {
        const int i = p / a.k, j = p - i * a.k;
        a.slot_pos[long(t0 + i) * a.k + j] = s_base[s_sel[i * 32 + j]] + s_loc[i * 32 + j];
      }
    }
  }
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kRtTmemCols);
  }
}

}  // namespace

bool route_tc_applies(const RouteArgs& a) {
  return a.x8 && a.r8 && a.batch && !a.xp && !a.ep.table && a.T > 0 && a.E == kRtE &&
         a.H >= 128 && a.H % 128 == 0 && a.H <= 32 * kRtMaxBlk && a.k <= 32 &&
         (reinterpret_cast<uintptr_t>(a.wr) & 15) == 0 &&
         (reinterpret_cast<uintptr_t>(a.sr) & 15) == 0 &&
         (reinterpret_cast<uintptr_t>(a.xsc) & 15) == 0 &&
         (reinterpret_cast<uintptr_t>(a.x8) & 15) == 0 &&
         (reinterpret_cast<uintptr_t>(a.r8) & 15) == 0;
}

cudaError_t launch_route_tc(const RouteArgs& a, cudaStream_t stream) {
  if (!route_tc_applies(a)) return cudaErrorInvalidValue;
  const int tiles = (a.T + kRtTile - 1) / kRtTile;
  const int n_tok_ctas = tiles * kRtTile / kQxTok;
  quant_x8_kernel<<<n_tok_ctas + kQxRouterCtas, kQxThreads, 0, stream>>>(a, n_tok_ctas);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  e = ensure_dynamic_smem(reinterpret_cast<const void*>(route_tc_kernel), kRtSmem);
  if (e != cudaSuccess) return e;
  route_tc_kernel<<<tiles, kRtThreads, kRtSmem, stream>>>(a);
  return cudaGetLastError();
}

}  // namespace mfi
