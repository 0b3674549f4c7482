// tc_gemm.cu — tcgen05 block-scaled MXFP4 GEMM, y (M, N) fp32 = A . B^T.
//
// Replaces the reference's prefill GEMM mxfp4_linear_kernel
// (src/ext/mxfp4_linear.cu:106-198: mma.sync m16n8k64 block_scale, sm_120a
// only, one 16x32 output tile per CTA with scalar nibble gathers) with the
// sm_100a tensor-core path:
//
//   * tile 128 (M) x 256 (N) x 256 (K) per stage, 4 stages in shared memory;
//   * warp 0 (one elected thread): TMA 2-D loads of the A and B tiles
//     (128-byte swizzle, zero fill outside the tensor) and bulk copies of the
//     scale-factor atoms, all completing on the stage's mbarrier;
//   * warp 1: allocates 512 TMEM columns, copies the stage's scale factors
//     into TMEM (tcgen05.cp 32x128b.warpx4) and issues 4
//     tcgen05.mma.kind::mxf4.block_scale (M=128, N=256, K=64) per stage, the
//     fp32 accumulator living in TMEM columns [0, 256); tcgen05.commit frees
//     the smem stage and, after the last stage, signals the epilogue;
//   * warps 2-5: tcgen05.ld the accumulator (one row per thread) and store it.
//
// Operands are the reference's packed formats: rows of Kp/2 bytes (two E2M1
// per byte, low nibble first — the K-major FP4 operand order), plus E8M0
// scales re-laid out once into 512-byte atoms (see sf_atoms_kernel).
// Every wait is bounded (2 s); on timeout the kernel records an error code in
// the caller's flag, drains its own loads and frees TMEM before returning.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <atomic>

#include "tc_ptx.cuh"
#include "tmap.cuh"
#include "work.cuh"

namespace mfi {

using namespace tc;

constexpr int kBM = 128, kBN = 256, kBK = 256;  // BK in elements (128 bytes of FP4)
constexpr int kStages = 4;
constexpr int kABytes = kBM * kBK / 2;                       // 16 KB
constexpr int kBBytes = kBN * kBK / 2;                       // 32 KB
constexpr int kSFABytes = (kBM / 128) * (kBK / 128) * 512;   // 1 KB
constexpr int kSFBBytes = (kBN / 128) * (kBK / 128) * 512;   // 2 KB
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kTmemSFA = 256;      // 2 chunks x 4 columns
constexpr uint32_t kTmemSFB = 256 + 8;  // 2 chunks x 2 row blocks x 4 columns
constexpr int kGemmThreads = 192;

size_t tc_gemm_smem_bytes() {
  return 1024 + size_t(kStages) * (kABytes + kBBytes + kSFABytes + kSFBBytes) +
         8 * (2 * kStages + 1) + 16;
}

struct TcGemmArgs {
  int M, N, Kp;
  int kc_pad;              // scale atoms per 128-row block along K (even)
  const uint8_t* sfa;      // (ceil(M/128)) x kc_pad x 512
  const uint8_t* sfb;      // (ceil(N/256)*2) x kc_pad x 512
  float* y;
  long long ldy;
  int* err;
};

__global__ void __launch_bounds__(kGemmThreads, 1)
    tc_gemm_mxf4_kernel(const __grid_constant__ CUtensorMap tma_a,
                        const __grid_constant__ CUtensorMap tma_b, TcGemmArgs p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = sA + kStages * kABytes;
  uint8_t* sSFA = sB + kStages * kBBytes;
  uint8_t* sSFB = sSFA + kStages * kSFABytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(sSFB + kStages * kSFBBytes);
  uint64_t* empty = full + kStages;
  uint64_t* accb = empty + kStages;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(accb + 1);
  __shared__ uint64_t drain[1];  // the MMA issuer's error-path drain

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_tile = blockIdx.x, m_tile = blockIdx.y;
  const int k_tiles = (p.Kp + kBK - 1) / kBK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(accb, 1);
    mbar_init(drain, 1);
    fence_mbar_init();
    cta_abort_init();
  }
  if (warp == 1) tmem_alloc(tmem_slot, kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (elect_one()) {
      prefetch_tmap(&tma_a);
      prefetch_tmap(&tma_b);
      int issued = 0;
      bool ok = true;
      for (int kt = 0; kt < k_tiles; ++kt) {
        const int s = kt % kStages;
        const uint32_t ph = (kt / kStages) & 1;
        if (!mbar_wait(&empty[s], ph ^ 1, p.err, 1)) { ok = false; break; }
        mbar_expect_tx(&full[s], kABytes + kBBytes + kSFABytes + kSFBBytes);
        tma_load_2d(sA + s * kABytes, &tma_a, kt * (kBK / 2), m_tile * kBM, &full[s]);
        tma_load_2d(sB + s * kBBytes, &tma_b, kt * (kBK / 2), n_tile * kBN, &full[s]);
        bulk_load(sSFA + s * kSFABytes, p.sfa + (size_t(m_tile) * p.kc_pad + 2 * kt) * 512, 1024,
                  &full[s]);
        bulk_load(sSFB + s * kSFBBytes, p.sfb + (size_t(2 * n_tile) * p.kc_pad + 2 * kt) * 512,
                  1024, &full[s]);
        bulk_load(sSFB + s * kSFBBytes + 1024,
                  p.sfb + (size_t(2 * n_tile + 1) * p.kc_pad + 2 * kt) * 512, 1024, &full[s]);
        issued = kt + 1;
      }
      if (!ok) {
        // drain our own copies before the CTA can exit
        for (int kt = (issued > kStages ? issued - kStages : 0); kt < issued; ++kt)
          mbar_wait(&full[kt % kStages], (kt / kStages) & 1, nullptr, 0);
      }
    }
  } else if (warp == 1) {
    if (elect_one()) {
      bool ok = true;
      for (int kt = 0; kt < k_tiles; ++kt) {
        const int s = kt % kStages;
        const uint32_t ph = (kt / kStages) & 1;
        if (!mbar_wait(&full[s], ph, p.err, 2)) { ok = false; break; }
        tc_fence_after();
        const uint32_t a_base = smem_u32(sA + s * kABytes);
        const uint32_t b_base = smem_u32(sB + s * kBBytes);
        const uint32_t sfa_base = smem_u32(sSFA + s * kSFABytes);
        const uint32_t sfb_base = smem_u32(sSFB + s * kSFBBytes);
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          tmem_cp_sf(tmem + kTmemSFA + 4 * c, make_sdesc(sfa_base + c * 512, 0, 128, kLayoutNone));
#pragma unroll
          for (int rb = 0; rb < 2; ++rb)
            tmem_cp_sf(tmem + kTmemSFB + 8 * c + 4 * rb,
                       make_sdesc(sfb_base + rb * 1024 + c * 512, 0, 128, kLayoutNone));
        }
#pragma unroll
        for (int kb = 0; kb < 4; ++kb) {
          const int c = kb >> 1;
          const uint32_t byte = uint32_t(kb & 1) * 2;
          const uint64_t adesc = make_sdesc(a_base + kb * 32, 16, 1024, kLayoutSW128);
          const uint64_t bdesc = make_sdesc(b_base + kb * 32, 16, 1024, kLayoutSW128);
          const uint32_t idesc = make_idesc_mxf4(kBM, kBN, int(byte), int(byte));
          const uint32_t tsfa = (tmem + kTmemSFA + 4 * c) | (byte << 30);
          const uint32_t tsfb = (tmem + kTmemSFB + 8 * c) | (byte << 30);
          mma_mxf4(tmem, adesc, bdesc, idesc, (kt | kb) != 0 ? 1u : 0u, tsfa, tsfb);
        }
        tc_commit(&empty[s]);
      }
      if (ok) tc_commit(accb);
      else drain_mma(drain);
    }
  } else {
    const bool ok = mbar_wait(accb, 0, p.err, 3);
    tc_fence_after();
    if (ok) {
      const int lane_base = (warp & 3) * 32;
      const int row = m_tile * kBM + lane_base + lane;
      float* yrow = p.y + (long long)row * p.ldy;
      const bool vec = (p.ldy % 4 == 0) && ((reinterpret_cast<uintptr_t>(p.y) & 15) == 0);
#pragma unroll 1
      for (int c0 = 0; c0 < kBN; c0 += 32) {
        uint32_t r[32];
        tmem_ld_32x32b_x32(tmem + (uint32_t(lane_base) << 16) + uint32_t(c0), r);
        tmem_ld_wait();
        const int col0 = n_tile * kBN + c0;
        if (row < p.M && col0 < p.N) {
          if (vec && col0 + 32 <= p.N) {
#pragma unroll
            for (int j = 0; j < 32; j += 4)
              *reinterpret_cast<float4*>(yrow + col0 + j) =
                  make_float4(__uint_as_float(r[j]), __uint_as_float(r[j + 1]),
                              __uint_as_float(r[j + 2]), __uint_as_float(r[j + 3]));
          } else {
#pragma unroll
            for (int j = 0; j < 32; ++j)
              if (col0 + j < p.N) yrow[col0 + j] = __uint_as_float(r[j]);
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

// ---------------------------------------------------------------------------
// Persistent form for N a multiple of 4 (the dense projections at prefill
// sizes; weight rows past N read as zeros through the tensor map and their
// columns are not stored): one CTA per SM walks tiles of 128 x 128 (consecutive tiles share
// the weight tile: m inner, n outer), 6-stage ring (226 KB of shared memory), three rotating
// 128-column accumulators, so a tile's epilogue overlaps the next tiles'
// MMAs.  The epilogue takes the tile's 128 columns into registers, releases
// the accumulator, and stores through a per-warp shared-memory transpose so
// every store instruction writes whole 128-byte row segments.
// ---------------------------------------------------------------------------
constexpr int kPBN = 128;
#ifndef MFI_PG_STAGES
#define MFI_PG_STAGES 6
#endif
constexpr int kPStagesG = MFI_PG_STAGES;
constexpr int kPStageG = kABytes + kBM * kBK / 2 + 2 * 1024;  // A 16 KB, B 16 KB, SFA 1 KB, SFB 1 KB
constexpr int kPAccG = 3;
constexpr uint32_t kPTmemSFG = kPAccG * 128;                  // + 16 per ring slot
static_assert(kPTmemSFG + 16 * kPStagesG <= 512, "scale columns exceed the allocation");
constexpr int kPOutStageG = 32 * 32 * 4;                       // per epilogue warp

constexpr size_t tc_gemm_p_smem_bytes() {
  return 1024 + size_t(kPStagesG) * kPStageG + 4 * size_t(kPOutStageG) +
         8 * (2 * kPStagesG + 2 * kPAccG) + 16;
}
// dynamic shared memory per CTA on sm_100 is at most 227 KB (232,448 B)
static_assert(tc_gemm_p_smem_bytes() + 64 <= 232448, "ring stages exceed the shared memory of a CTA");

__global__ void __launch_bounds__(kGemmThreads, 1)
    tc_gemm_p_kernel(const __grid_constant__ CUtensorMap tma_a,
                     const __grid_constant__ CUtensorMap tma_b, TcGemmArgs p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* ring = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint8_t* out_stage = ring + size_t(kPStagesG) * kPStageG;
  uint64_t* full = reinterpret_cast<uint64_t*>(out_stage + 4 * kPOutStageG);
  uint64_t* empty = full + kPStagesG;
  uint64_t* acc_full = empty + kPStagesG;
  uint64_t* acc_empty = acc_full + kPAccG;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + kPAccG);
  __shared__ uint64_t drain[1];  // the MMA issuer's error-path drain
  constexpr int kOffB = kABytes, kOffSFA = kABytes + kBM * kBK / 2, kOffSFB = kOffSFA + 1024;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int k_tiles = (p.Kp + kBK - 1) / kBK;
  const int n_m = (p.M + kBM - 1) / kBM, n_n = (p.N + kPBN - 1) / kPBN;
  const int n_tiles = n_m * n_n;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kPStagesG; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < kPAccG; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 4);
    }
    mbar_init(drain, 1);
    fence_mbar_init();
    cta_abort_init();
  }
  if (warp == 1) tmem_alloc(tmem_slot, kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (elect_one()) {
      prefetch_tmap(&tma_a);
      prefetch_tmap(&tma_b);
      uint32_t it = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < n_tiles && ok; t += gridDim.x) {
        const int m = t % n_m, n = t / n_m;
        for (int kt = 0; kt < k_tiles; ++kt, ++it) {
          const int s = int(it % kPStagesG);
          if (!mbar_wait(&empty[s], ((it / kPStagesG) & 1) ^ 1, p.err, 1)) { ok = false; break; }
          uint8_t* st = ring + size_t(s) * kPStageG;
          mbar_expect_tx(&full[s], kPStageG);
          tma_load_2d(st, &tma_a, kt * (kBK / 2), m * kBM, &full[s]);
          tma_load_2d(st + kOffB, &tma_b, kt * (kBK / 2), n * kPBN, &full[s]);
          bulk_load(st + kOffSFA, p.sfa + (size_t(m) * p.kc_pad + 2 * kt) * 512, 1024, &full[s]);
          bulk_load(st + kOffSFB, p.sfb + (size_t(n) * p.kc_pad + 2 * kt) * 512, 1024, &full[s]);
        }
      }
      if (!ok) {
        // drain our own copies before the CTA can exit
        for (uint32_t j = (it > uint32_t(kPStagesG) ? it - kPStagesG : 0); j < it; ++j)
          mbar_wait(&full[j % kPStagesG], (j / kPStagesG) & 1, nullptr, 0);
      }
    }
  } else if (warp == 1) {
    if (elect_one()) {
      uint32_t it = 0, ti = 0;
      bool ok = true;
      const uint32_t idesc0 = make_idesc_mxf4(kBM, kPBN, 0, 0);
      const uint32_t idesc2 = make_idesc_mxf4(kBM, kPBN, 2, 2);
      for (int t = blockIdx.x; t < n_tiles && ok; t += gridDim.x, ++ti) {
        const uint32_t buf = ti % kPAccG;
        if (!mbar_wait(&acc_empty[buf], ((ti / kPAccG) & 1) ^ 1, p.err, 2)) { ok = false; break; }
        tc_fence_after();
        const uint32_t d = tmem + buf * 128;
        for (int kt = 0; kt < k_tiles; ++kt, ++it) {
          const int s = int(it % kPStagesG);
          if (!mbar_wait(&full[s], (it / kPStagesG) & 1, p.err, 2)) { ok = false; break; }
          tc_fence_after();
          const uint32_t base = smem_u32(ring + size_t(s) * kPStageG);
          const uint32_t sfa = tmem + kPTmemSFG + 16 * s, sfb = sfa + 8;
#pragma unroll
          for (int c = 0; c < 2; ++c) {
            tmem_cp_sf(sfa + 4 * c, make_sdesc(base + kOffSFA + c * 512, 0, 128, kLayoutNone));
            tmem_cp_sf(sfb + 4 * c, make_sdesc(base + kOffSFB + c * 512, 0, 128, kLayoutNone));
          }
#pragma unroll
          for (int kb = 0; kb < 4; ++kb) {
            const int c = kb >> 1;
            const uint32_t byte = uint32_t(kb & 1) * 2;
            mma_mxf4(d, make_sdesc(base + kb * 32, 16, 1024, kLayoutSW128),
                     make_sdesc(base + kOffB + kb * 32, 16, 1024, kLayoutSW128),
                     byte ? idesc2 : idesc0, (kt | kb) != 0 ? 1u : 0u,
                     (sfa + 4 * c) | (byte << 30), (sfb + 4 * c) | (byte << 30));
          }
          tc_commit(&empty[s]);
        }
        if (ok) tc_commit(&acc_full[buf]);
      }
      if (!ok) drain_mma(drain);
    }
  } else {
    const int quad = warp & 3;
    uint4* stg = reinterpret_cast<uint4*>(out_stage + (warp - 2) * kPOutStageG);
    uint32_t ti = 0;
    for (int t = blockIdx.x; t < n_tiles; t += gridDim.x, ++ti) {
      const int m = t % n_m, n = t / n_m;
      const uint32_t buf = ti % kPAccG;
      if (!mbar_wait(&acc_full[buf], (ti / kPAccG) & 1, p.err, 3)) break;
      tc_fence_after();
      uint32_t r[4][32];
      const uint32_t ta = tmem + (uint32_t(quad * 32) << 16) + buf * 128;
#pragma unroll
      for (int c = 0; c < 4; ++c) tmem_ld_32x32b_x32(ta + c * 32, r[c]);
      tmem_ld_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[buf]);
      // lane l holds row row0 + l; 16-byte chunk q of row l sits at q ^ (l & 7)
      const int row0 = m * kBM + quad * 32;
      const int sub = lane >> 3, ch = lane & 7;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
#pragma unroll
        for (int q = 0; q < 8; ++q)
          stg[lane * 8 + (q ^ (lane & 7))] =
              make_uint4(r[c][4 * q], r[c][4 * q + 1], r[c][4 * q + 2], r[c][4 * q + 3]);
        __syncwarp();
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const int rr = 4 * i + sub;
          const int row = row0 + rr;
          const int col = n * kPBN + c * 32 + ch * 4;
          const uint4 v = stg[rr * 8 + (ch ^ (rr & 7))];
          if (row < p.M && col < p.N)
            *reinterpret_cast<uint4*>(p.y + (long long)row * p.ldy + col) = v;
        }
        __syncwarp();
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

// ---------------------------------------------------------------------------
// Row-major E8M0 codes (R, nb) -> 512-byte atoms.  Atom (rb, kc) holds rows
// rb*128 .. rb*128+127 and K blocks kc*4 .. kc*4+3; inside it byte
// (r % 32)*16 + ((r % 128) / 32)*4 + (k % 4).  This is the layout that one
// tcgen05.cp 32x128b.warpx4 moves into the 4 TMEM columns the MMA reads for a
// 128-row operand.  Rows >= R and blocks >= nb are filled with code 127 (1.0).
// ---------------------------------------------------------------------------
__global__ void sf_atoms_kernel(const uint8_t* __restrict__ src, long long src_ld, int R, int nb,
                                int row_blocks, int kc_pad, uint8_t* __restrict__ dst) {
  const long long total = (long long)row_blocks * kc_pad * 512;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const int within = int(i & 511);
    const long long atom = i >> 9;
    const int kc = int(atom % kc_pad);
    const int rb = int(atom / kc_pad);
    const int r = rb * 128 + (within >> 4) + 32 * ((within & 15) >> 2);
    const int k = kc * 4 + (within & 3);
    dst[i] = (r < R && k < nb) ? src[(long long)r * src_ld + k] : uint8_t(127);
  }
}

size_t sf_atoms_bytes(int R, int Kp, int row_align) {
  const int rb = (R + row_align - 1) / row_align * (row_align / 128);
  const int kc_pad = 2 * ((Kp + kBK - 1) / kBK);
  return size_t(rb) * kc_pad * 512;
}

cudaError_t launch_sf_atoms(const uint8_t* src, long long src_ld, int R, int Kp, int row_align,
                            uint8_t* dst, cudaStream_t stream) {
  const int rb = (R + row_align - 1) / row_align * (row_align / 128);
  const int kc_pad = 2 * ((Kp + kBK - 1) / kBK);
  const long long total = (long long)rb * kc_pad * 512;
  if (total == 0) return cudaSuccess;
  long long blocks = (total + 255) / 256;
  if (blocks > 148 * 32) blocks = 148 * 32;
  sf_atoms_kernel<<<unsigned(blocks), 256, 0, stream>>>(src, src_ld, R, Kp / 32, rb, kc_pad, dst);
  return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// Device-wide error flag: 0 while healthy; the first failure of any kernel
// stores its code (a bounded wait that timed out, or invalid data).  It only
// reports to the host (mfi_device_error); a set flag does not stop later
// kernels (their waits stop on their own CTA's abort word, tc_ptx.cuh).
__device__ int g_device_error;

int* device_error_flag() {
  static std::atomic<int*> addr[64];  // zero-initialised; racing first lookups store one value
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return nullptr;
  int* a = addr[dev].load(std::memory_order_acquire);
  if (!a) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_device_error) != cudaSuccess) return nullptr;
    a = static_cast<int*>(p);
    addr[dev].store(a, std::memory_order_release);
  }
  return a;
}

bool tc_gemm_supported(const void* a, const void* b, int Kp) {
  return (reinterpret_cast<uintptr_t>(a) % 16 == 0) && (reinterpret_cast<uintptr_t>(b) % 16 == 0) &&
         (Kp % 32 == 0) && Kp > 0;
}

cudaError_t launch_tc_gemm(const uint8_t* a, const uint8_t* sfa_atoms, const uint8_t* b,
                           const uint8_t* sfb_atoms, float* y, long long ldy, int M, int N, int Kp,
                           int* err, cudaStream_t stream) {
  if (M == 0 || N == 0) return cudaSuccess;
  CUtensorMap ta, tb;
  if (!make_tmap(&ta, a, uint64_t(Kp / 2), uint64_t(M), kBM) ||
      !make_tmap(&tb, b, uint64_t(Kp / 2), uint64_t(N), kBN))
    return cudaErrorInvalidValue;
  const size_t smem = tc_gemm_smem_bytes();
  {
    cudaError_t e = ensure_dynamic_smem(reinterpret_cast<const void*>(tc_gemm_mxf4_kernel), smem);
    if (e != cudaSuccess) return e;
  }
  TcGemmArgs p;
  p.M = M; p.N = N; p.Kp = Kp;
  p.kc_pad = 2 * ((Kp + kBK - 1) / kBK);
  p.sfa = sfa_atoms; p.sfb = sfb_atoms; p.y = y; p.ldy = ldy; p.err = err;
  if (N % 4 == 0 && ldy % 4 == 0 && (reinterpret_cast<uintptr_t>(y) & 15) == 0) {
    CUtensorMap tb2;
    if (!make_tmap(&tb2, b, uint64_t(Kp / 2), uint64_t(N), kPBN)) return cudaErrorInvalidValue;
    const size_t smem2 = tc_gemm_p_smem_bytes();
    cudaError_t e = ensure_dynamic_smem(reinterpret_cast<const void*>(tc_gemm_p_kernel), smem2);
    if (e != cudaSuccess) return e;
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const int tiles = (M + kBM - 1) / kBM * ((N + kPBN - 1) / kPBN);
    tc_gemm_p_kernel<<<tiles < sms ? tiles : sms, kGemmThreads, smem2, stream>>>(ta, tb2, p);
    return cudaGetLastError();
  }
  dim3 grid((N + kBN - 1) / kBN, (M + kBM - 1) / kBM);
  tc_gemm_mxf4_kernel<<<grid, kGemmThreads, smem, stream>>>(ta, tb, p);
  return cudaGetLastError();
}

}  // namespace mfi
