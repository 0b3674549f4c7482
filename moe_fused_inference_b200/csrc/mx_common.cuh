// mx_common.cuh — MXFP4 arithmetic shared by every kernel of the library.
//
// Format (reference quant/fp4_format.py:17-148, src/ext/mxfp4_common.cuh:24-54):
//   E2M1 nibble  bit3 = sign, bits0-2 index {0,.5,1,1.5,2,3,4,6}
//   E8M0 code    scale 2^(code-127), one per 32 consecutive K elements
//   packing      LSB-first: element 2k in the low nibble of byte k
//
// Quantiser contract = reference quant/quantize_mxfp4.py:110-160 (Python), not
// the reference kernel: t = max(fl32(amax/6), 1e-30f); e = ceil(log2 t) taken
// exactly from the float32 bits of t; code = clamp(e+127, 0, 255) (127 when
// amax == 0); nibbles use the unclamped scale 2^e.  Because t >= 1e-30 the
// exponent lies in [-99, 126] for finite inputs, so 2^-e is a normal float
// and x * 2^-e rounds exactly like the reference's x / 2^e.
//
// This file must be compiled WITHOUT flush-to-zero (no --use_fast_math): the
// sign bit of a tiny negative value that rounds to zero magnitude depends on
// subnormal arithmetic.
#pragma once
#include <cstdint>
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>

namespace mfi {

constexpr int kBlock = 32;

// Element dtypes accepted by the quantiser (mirrors torch dtypes the
// reference binding sees: bf16 in prequant, half/bf16/f32 in forward).
enum DType : int { kF32 = 0, kF16 = 1, kBF16 = 2 };

__device__ __forceinline__ float load_elem(const void* p, long i, int dtype) {
  if (dtype == kBF16) return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p)[i]);
  if (dtype == kF16) return __half2float(reinterpret_cast<const __half*>(p)[i]);
  return reinterpret_cast<const float*>(p)[i];
}

// Nearest E2M1 magnitude index of |x| (x already divided by the block scale),
// ties toward the larger magnitude, clamp at 6 (index 7); NaN gives 7, as in
// the reference.  Read from the bits of a = |x|: at a >= 1 the grid {1, 1.5,
// 2, 3, 4, 6} keeps one mantissa bit, so adding half of that bit's weight
// (bit 21) and keeping exponent + top mantissa bit (bits >> 22) rounds half
// up, and 1.0 (bits >> 22 = 254) is index 2; below 1 the grid is {0, .5, 1}
// with midpoints .25 and .75.  Infinities and NaNs (exponent field 255) land
// above index 7 and clamp to it.
__device__ __forceinline__ uint32_t e2m1_mag(float a) {
  const uint32_t b = __float_as_uint(a) & 0x7FFFFFFFu;
  const uint32_t hi = min(((b + 0x200000u) >> 22) - 252u, 7u);
  const uint32_t lo = uint32_t(b >= 0x3E800000u) + uint32_t(b >= 0x3F400000u);  // .25, .75
  return b >= 0x3F800000u ? hi : lo;
}

// Unclamped block exponent e (see header).  amax must be >= 0 or NaN.
__device__ __forceinline__ int block_exp(float amax) {
  float t = fmaxf(__fdiv_rn(amax, 6.0f), 1e-30f);
  uint32_t b = __float_as_uint(t);
  int ex = int((b >> 23) & 0xFF) - 127;
  return ex + ((b & 0x7FFFFF) != 0u ? 1 : 0);
}

struct BlockScale {
  uint8_t code;   // E8M0 code stored with the block
  float inv;      // 2^-e, multiplier applied to elements before rounding
};

__device__ __forceinline__ BlockScale block_scale(float amax) {
  BlockScale s;
  if (!(amax > 0.0f)) {  // zero or NaN block: code 127, scale 1
    s.code = 127;
    s.inv = 1.0f;
    return s;
  }
  int e = block_exp(amax);
  int c = e + 127;
  s.code = uint8_t(c < 0 ? 0 : (c > 255 ? 255 : c));
  int ee = e > 126 ? 126 : e;  // only non-finite inputs reach e > 126
  s.inv = __uint_as_float(uint32_t(127 - ee) << 23);
  return s;
}

__device__ __forceinline__ uint32_t quant_nibble(float v, float inv) {
  float x = __fmul_rn(v, inv);
  uint32_t c = e2m1_mag(fabsf(x));
  return c | (x < 0.0f ? 8u : 0u);
}

// Quantise 8 consecutive elements of a 32-element block held by a quad of
// lanes (lanes 4q..4q+3 hold the block's 4 groups of 8).  All 32 lanes must
// call it (full-mask shuffles); `live` = false lanes contribute zeros.
// Returns the 8 nibbles packed LSB-first and the block's scale.
__device__ __forceinline__ uint32_t quant_group8(const float (&v)[8], BlockScale& bs);

// 8 nibbles -> two words of 4 signed int8 each, value = 2*e2m1 in [-12, 12].
// lo holds elements 0-3, hi elements 4-7 (element order kept).
__device__ __forceinline__ void nib8_to_i8(uint32_t w, uint32_t& lo, uint32_t& hi) {
  const uint32_t P0 = 0x03020100u, P1 = 0x0C080604u;  // 0 1 2 3 | 4 6 8 12
  const uint32_t N0 = 0xFDFEFF00u, N1 = 0xF4F8FAFCu;  // 0 -1 -2 -3 | -4 -6 -8 -12
  const uint32_t m = w & 0x77777777u;                  // magnitude selectors
  const uint32_t s = (w >> 1) & 0x44444444u;           // sign bit -> selector bit 2
  uint32_t pl = __byte_perm(P0, P1, m & 0xFFFFu);
  uint32_t nl = __byte_perm(N0, N1, m & 0xFFFFu);
  lo = __byte_perm(pl, nl, 0x3210u | (s & 0xFFFFu));
  uint32_t ph = __byte_perm(P0, P1, m >> 16);
  uint32_t nh = __byte_perm(N0, N1, m >> 16);
  hi = __byte_perm(ph, nh, 0x3210u | (s >> 16));
}

// Correctly rounded a / b by Markstein's method (P. Markstein, "Computation
// of elementary functions on the IBM RISC System/6000 processor", IBM J. Res.
// Dev. 34(1), 1990): an approximate reciprocal y0, one Newton step
// y1 = y0 + y0 (1 - b y0), the quotient q0 = a y1, its exact remainder
// r = a - b q0 (one FMA) and the correction q0 + r y1, which is a / b rounded
// to nearest even as long as b, 1/b, a and the quotient are normal numbers.
__device__ __forceinline__ float div_markstein(float a, float b) {
  float y0;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y0) : "f"(b));
  const float e = __fmaf_rn(-b, y0, 1.0f);
  const float y1 = __fmaf_rn(y0, e, y0);
  const float q0 = __fmul_rn(a, y1);
  const float r = __fmaf_rn(-b, q0, a);
  return __fmaf_rn(r, y1, q0);
}

// g / b for b = 1 + expf(-g) where the plain Markstein division does not
// apply (|g| < 2^-100 or > 80, infinities, NaN); the exact IEEE quotient.
static __device__ __noinline__ float swiglu_quotient_edge(float g, float b) {
  if (g != g || b != b) return __uint_as_float(0x7FFFFFFFu);
  if (isinf(g)) return b == 1.0f ? g : __uint_as_float(0x7FFFFFFFu);  // +inf / 1, -inf / inf
  if (isinf(b)) return copysignf(0.0f, g);  // g < -88.7: e^-g overflows
  if (b == 1.0f) return g;                  // g > 80: e^-g is below half an ulp of 1
  if (b == 2.0f) return __fmul_rn(g, 0.5f); // |g| < 2^-100 (zeros, subnormals)
  // -88.7 < g < -80: b is up to 2^128 and 1/b may be subnormal, the quotient
  // is normal: divide by b 2^-32 and scale back (both exact powers of two)
  return __fmul_rn(div_markstein(g, __fmul_rn(b, 0x1p-32f)), 0x1p-32f);
}

// SwiGLU, h = (g / (1 + e^-g)) * u in fp32, the one form every kernel of the
// library uses (the moe_down operator and the fused decode / prefill
// epilogues).  It is the reference kernel's expression
// (src/ext/mxfp4_decode.cu:258) as its build compiles it: runtime/fp4_ext.py
// builds the extension with -O3 and no fast-math flag, so expf is CUDA's
// expf and '/' a correctly rounded division; nothing in it can be contracted
// into an FMA.  The division is div_markstein, which for |g| in [2^-100, 80]
// (b in [1, 1 + e^80], quotient normal) is the correctly rounded quotient;
// the rest goes to swiglu_quotient_edge.  mfi_selftest_numerics compares the
// quotient with CUDA's __fdiv_rn for all 2^32 values of g.
__device__ __forceinline__ float swiglu_quotient(float g) {
  const float b = __fadd_rn(1.0f, expf(-g));
  const float ag = fabsf(g);
  if (ag >= 0x1p-100f && ag <= 80.0f) return div_markstein(g, b);
  return swiglu_quotient_edge(g, b);
}
__device__ __forceinline__ float swiglu(float g, float u) {
  return __fmul_rn(swiglu_quotient(g), u);
}

// max(a, b) that returns NaN when either is NaN (PTX max.NaN).
__device__ __forceinline__ float fmax_nan(float a, float b) {
  float r;
  asm("max.NaN.f32 %0, %1, %2;" : "=f"(r) : "f"(a), "f"(b));
  return r;
}

// 2^e as float for e in the normal range; ldexpf outside it.
__device__ __forceinline__ float exp2i(int e) {
  if (e >= -126 && e <= 127) return __uint_as_float(uint32_t(e + 127) << 23);
  return ldexpf(1.0f, e);
}

// 2^e as double (e well inside the double range for any pair of E8M0 codes).
__device__ __forceinline__ double exp2i_d(int e) {
  return __longlong_as_double((long long)(e + 1023) << 52);
}

// Dot product of one 32-element block given as 16 packed bytes on each side;
// returns the exact integer sum of (2a)(2b).
__device__ __forceinline__ int block_dot_i(const uint4& a, const uint4& b) {
  int acc = 0;
  uint32_t al, ah, bl, bh;
  nib8_to_i8(a.x, al, ah); nib8_to_i8(b.x, bl, bh);
  acc = __dp4a(int(al), int(bl), acc); acc = __dp4a(int(ah), int(bh), acc);
  nib8_to_i8(a.y, al, ah); nib8_to_i8(b.y, bl, bh);
  acc = __dp4a(int(al), int(bl), acc); acc = __dp4a(int(ah), int(bh), acc);
  nib8_to_i8(a.z, al, ah); nib8_to_i8(b.z, bl, bh);
  acc = __dp4a(int(al), int(bl), acc); acc = __dp4a(int(ah), int(bh), acc);
  nib8_to_i8(a.w, al, ah); nib8_to_i8(b.w, bl, bh);
  acc = __dp4a(int(al), int(bl), acc); acc = __dp4a(int(ah), int(bh), acc);
  return acc;
}

// Same with b already expanded to int8 (8 words).
__device__ __forceinline__ int block_dot_pre(const uint4& a, const uint32_t* b8) {
  int acc = 0;
  uint32_t l, h;
  nib8_to_i8(a.x, l, h); acc = __dp4a(int(l), int(b8[0]), acc); acc = __dp4a(int(h), int(b8[1]), acc);
  nib8_to_i8(a.y, l, h); acc = __dp4a(int(l), int(b8[2]), acc); acc = __dp4a(int(h), int(b8[3]), acc);
  nib8_to_i8(a.z, l, h); acc = __dp4a(int(l), int(b8[4]), acc); acc = __dp4a(int(h), int(b8[5]), acc);
  nib8_to_i8(a.w, l, h); acc = __dp4a(int(l), int(b8[6]), acc); acc = __dp4a(int(h), int(b8[7]), acc);
  return acc;
}

__device__ __forceinline__ int dot_i8x32(const uint32_t* a8, const uint32_t* b8) {
  int acc = 0;
#pragma unroll
  for (int i = 0; i < 8; ++i) acc = __dp4a(int(a8[i]), int(b8[i]), acc);
  return acc;
}

// Value of one block partial: S * 2^(sa + sb - 256) (the 2 x 2 of the int
// encoding folded into the exponent).
__device__ __forceinline__ float block_value(int s, int sa, int sb) {
  return __fmul_rn(float(s), exp2i(sa + sb - 256));
}

__device__ __forceinline__ uint32_t quant_group8(const float (&v)[8], BlockScale& bs) {
  float am = 0.0f;
  bool has_nan = false;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    am = fmaxf(am, fabsf(v[i]));
    has_nan |= (v[i] != v[i]);
  }
  am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, 1));
  am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, 2));
  has_nan |= __shfl_xor_sync(0xffffffffu, int(has_nan), 1) != 0;
  has_nan |= __shfl_xor_sync(0xffffffffu, int(has_nan), 2) != 0;
  // a NaN anywhere in the block gives code 127, like the reference's NaN max
  bs = block_scale(has_nan ? __uint_as_float(0x7fc00000u) : am);
  uint32_t word = 0;
#pragma unroll
  for (int i = 0; i < 8; ++i) word |= quant_nibble(v[i], bs.inv) << (4 * i);
  return word;
}

__device__ __forceinline__ uint4 ldg_u4(const void* p) {
  return __ldg(reinterpret_cast<const uint4*>(p));
}

}  // namespace mfi
