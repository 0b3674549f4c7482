// lin_tc.cu — decode-sized dense MXFP4 GEMM (lin_pq / mxfp4_linear with at
// most 32 activation rows: the static projections and the lm_head of a decode
// step) on the tcgen05 tensor cores.
//
// Replaces, for M <= 32, the reference's lin_pq_kernel and
// mxfp4_linear_kernel (src/ext/mxfp4_decode.cu:135-170,
// src/ext/mxfp4_linear.cu:106-198).  The problem is a weight stream (the
// lm_head alone is 165 MB), so it runs "swap AB" like the decode expert
// kernel (moe_tc.cu):
//
//   D^T (128 weight rows x 32 tokens) += W_tile (128 x 256 K) . X^T,
//   tcgen05.mma.kind::mxf4.block_scale, M = 128, N = 32, K = 64,
//
// with fp32 accumulators in TMEM.  Per CTA (persistent, one per SM; weight
// tile t of 128 rows goes to CTA t % grid):
//   warp 0     TMA of each 128-row x 256-K stage of the raw row-major weights
//              through a 128-byte-swizzled tensor map (rows past N read as
//              zeros) into a ring, and one bulk copy per tile of the tile's
//              raw E8M0 codes
//   warp 6     rearranges those codes into the 512-byte scale atoms that
//              tcgen05.cp reads, once per tile (double-buffered)
//   warp 1     per stage: tcgen05.cp of the scales, 4 MMAs into one of four
//              32-column accumulators
//   warps 2-5  epilogue: tcgen05.ld, out[m][n] for the M real tokens
// The activation rows (zero-padded to 32) and their scale atoms are staged
// once per CTA.  Every wait is bounded (tc_ptx.cuh).
#include "mx_common.cuh"
#include "tc_ptx.cuh"
#include "tmap.cuh"
#include "work.cuh"

namespace mfi {

using namespace tc;

namespace {

constexpr int kLtRows = 128;           // weight rows per tile (MMA M)
constexpr int kLtTok = 32;             // activation rows (MMA N)
constexpr int kLtA = 16384;            // 128 rows x 128 B per K-stage of 256
constexpr int kLtB = 4096;             // 32 rows x 128 B per K-stage
constexpr int kLtAtom = 512;
constexpr int kLtThreads = 224;        // 7 warps
constexpr int kLtAccBufs = 4;
constexpr uint32_t kLtTmemCols = 256;
constexpr uint32_t kLtTmemSF = kLtAccBufs * 32;  // + 16 per ring slot: SFA 8, SFB 8
constexpr int kLtMaxStages = 6;
constexpr size_t kLtSmemBudget = 200 * 1024;
static_assert(kLtTmemSF + 16 * kLtMaxStages <= kLtTmemCols, "scale columns exceed the allocation");

// Shared-memory layout (offsets from the 1024-aligned base).
struct LtLayout {
  int nks, stages;
  size_t off_b, off_sfb, off_raw, off_sfa, off_bar, bytes;
};

__host__ __device__ inline LtLayout lt_layout(int Kp, int stages) {
  LtLayout L;
  L.nks = Kp / 256;
  L.stages = stages;
  const size_t nb = size_t(Kp) / 32;
  L.off_b = size_t(stages) * kLtA;                       // B: nks x 4 KB (SW128)
  L.off_sfb = L.off_b + size_t(L.nks) * kLtB;            // SFB atoms: nks x 2 x 512
  L.off_raw = L.off_sfb + size_t(L.nks) * 2 * kLtAtom;   // raw codes: 2 x 128 x nb
  L.off_sfa = L.off_raw + 2 * kLtRows * nb;              // SFA atoms: 2 x nks x 2 x 512
  L.off_bar = L.off_sfa + 2 * size_t(L.nks) * 2 * kLtAtom;
  L.bytes = 1024 + L.off_bar + 8 * (2 * kLtMaxStages + 2 * kLtAccBufs + 9) + 16;
  return L;
}

int lt_stages(int Kp) {
  const size_t fixed = lt_layout(Kp, 0).bytes;
  if (fixed >= kLtSmemBudget) return 0;
  const size_t st = (kLtSmemBudget - fixed) / kLtA;
  return st > size_t(kLtMaxStages) ? kLtMaxStages : int(st);
}

__global__ void __launch_bounds__(kLtThreads, 1)
    lin_tc_kernel(const __grid_constant__ CUtensorMap tma_w, const __grid_constant__ CUtensorMap tma_x,
                  const uint8_t* __restrict__ xsc, const uint8_t* __restrict__ wsc,
                  float* __restrict__ y, long long ldy, int M, int N, int Kp, int stages, int* err) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  const LtLayout L = lt_layout(Kp, stages);
  const int nb = Kp >> 5, nks = L.nks;
  uint8_t* ring = base;
  uint8_t* s_b = base + L.off_b;
  uint8_t* s_sfb = base + L.off_sfb;
  uint8_t* s_raw = base + L.off_raw;
  uint8_t* s_sfa = base + L.off_sfa;
  uint64_t* full = reinterpret_cast<uint64_t*>(base + L.off_bar);
  uint64_t* empty = full + kLtMaxStages;
  uint64_t* acc_full = empty + kLtMaxStages;
  uint64_t* acc_empty = acc_full + kLtAccBufs;
  uint64_t* raw_full = acc_empty + kLtAccBufs;   // [2]
  uint64_t* raw_empty = raw_full + 2;            // [2]
  uint64_t* sfa_full = raw_empty + 2;            // [2]
  uint64_t* sfa_empty = sfa_full + 2;            // [2]
  uint64_t* b_bar = sfa_empty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(b_bar + 1);
  __shared__ uint64_t drain[1];  // the MMA issuer's error-path drain
  const size_t raw_bytes = size_t(kLtRows) * nb;
  const size_t sfa_bytes = size_t(nks) * 2 * kLtAtom;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_tiles = (N + kLtRows - 1) / kLtRows;

  if (threadIdx.x == 0) {
    for (int s = 0; s < stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < kLtAccBufs; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 4);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&raw_full[b], 1);
      mbar_init(&raw_empty[b], 1);
      mbar_init(&sfa_full[b], 1);
      mbar_init(&sfa_empty[b], 1);
    }
    mbar_init(b_bar, 2);  // the activation TMA + the activation scale atoms
    mbar_init(drain, 1);
    fence_mbar_init();
    cta_abort_init();
  }
  if (warp == 1) tmem_alloc(tmem_slot, kLtTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ---- producer ---------------------------------------------------------------
    if (elect_one()) {
      prefetch_tmap(&tma_w);
      prefetch_tmap(&tma_x);
      mbar_expect_tx(b_bar, uint32_t(nks) * kLtB);
      for (int ks = 0; ks < nks; ++ks) tma_load_2d(s_b + ks * kLtB, &tma_x, ks * 128, 0, b_bar);
      // the raw codes of a tile go out one tile ahead of its weights, so the
      // scale atoms are ready when its first stage lands
      uint32_t n_raw = 0;  // raw-code copies issued (copy j: buffer j & 1, phase j >> 1)
      auto issue_raw = [&](int t, uint32_t ti) {
        const int ib = int(ti & 1);
        if (!mbar_wait(&raw_empty[ib], ((ti >> 1) & 1) ^ 1, err, 1)) return false;
        const int rows = min(kLtRows, N - t * kLtRows);
        mbar_expect_tx(&raw_full[ib], uint32_t(rows * nb));
        bulk_load(s_raw + ib * raw_bytes, wsc + size_t(t) * kLtRows * nb, uint32_t(rows * nb),
                  &raw_full[ib]);
        n_raw = ti + 1;
        return true;
      };
      uint32_t it = 0, ti = 0;
      bool ok = int(blockIdx.x) < n_tiles ? issue_raw(blockIdx.x, 0) : true;
      for (int t = blockIdx.x; t < n_tiles && ok; t += gridDim.x, ++ti) {
        if (t + int(gridDim.x) < n_tiles && !issue_raw(t + gridDim.x, ti + 1)) { ok = false; break; }
        for (int ks = 0; ks < nks; ++ks, ++it) {
          const int s = int(it % uint32_t(stages));
          if (!mbar_wait(&empty[s], ((it / stages) & 1) ^ 1, err, 1)) { ok = false; break; }
          mbar_expect_tx(&full[s], kLtA);
          tma_load_2d(ring + s * kLtA, &tma_w, ks * 128, t * kLtRows, &full[s]);
        }
      }
      if (!ok) {
        // drain our own copies before the CTA can exit: the activation rows,
        // the last two raw-code copies and the ring stages
        mbar_wait(b_bar, 0, nullptr, 0);
        drain_ring(raw_full, 2, n_raw);
        drain_ring(full, uint32_t(stages), it);
      }
    }
  } else if (warp == 6) {
    // ---- scale atoms ----------------------------------------------------------
    // activations: 32 rows, 4 codes per row and 128-K chunk, line r of the atom
    for (int q = 0; q < nks * 2; ++q) {
      uint32_t* atom = reinterpret_cast<uint32_t*>(s_sfb + q * kLtAtom);
      uint32_t v = 0x7F7F7F7Fu;  // padding rows are zeros; any finite scale
      if (lane < M) v = *reinterpret_cast<const uint32_t*>(xsc + size_t(lane) * nb + 4 * q);
      atom[lane * 4] = v;
      atom[lane * 4 + 1] = 0u;
      atom[lane * 4 + 2] = 0u;
      atom[lane * 4 + 3] = 0u;
    }
    fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0) mbar_arrive(b_bar);
    // weights: byte (r % 32) * 16 + (r / 32) * 4 + (k % 4) of the chunk's atom
    uint32_t ti = 0;
    for (int t = blockIdx.x; t < n_tiles; t += gridDim.x, ++ti) {
      const int ib = int(ti & 1);
      const uint32_t par = (ti >> 1) & 1;
      if (!__all_sync(0xffffffffu, mbar_wait(&raw_full[ib], par, err, 5))) break;
      if (!__all_sync(0xffffffffu, mbar_wait(&sfa_empty[ib], par ^ 1, err, 5))) break;
      const int rows = min(kLtRows, N - t * kLtRows);
      const uint8_t* raw = s_raw + ib * raw_bytes;
      uint8_t* atoms = s_sfa + ib * sfa_bytes;
#pragma unroll
      for (int g = 0; g < 4; ++g) {
        const int r = g * 32 + lane;
        for (int q = 0; q < nks * 2; ++q) {
          const uint32_t v = r < rows ? *reinterpret_cast<const uint32_t*>(raw + size_t(r) * nb + 4 * q)
                                      : 0x7F7F7F7Fu;
          *reinterpret_cast<uint32_t*>(atoms + q * kLtAtom + lane * 16 + g * 4) = v;
        }
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&sfa_full[ib]);
        mbar_arrive(&raw_empty[ib]);
      }
    }
  } else if (warp == 1) {
    // ---- MMA issue --------------------------------------------------------------
    if (elect_one()) {
      bool ok = mbar_wait(b_bar, 0, err, 2);
      uint32_t it = 0, ti = 0;
      for (int t = blockIdx.x; t < n_tiles && ok; t += gridDim.x, ++ti) {
        const uint32_t buf = ti % kLtAccBufs;
        const int ib = int(ti & 1);
        if (!mbar_wait(&acc_empty[buf], ((ti / kLtAccBufs) & 1) ^ 1, err, 2)) { ok = false; break; }
        if (!mbar_wait(&sfa_full[ib], (ti >> 1) & 1, err, 2)) { ok = false; break; }
        tc_fence_after();
        const uint32_t d = tmem + buf * 32;
        const uint32_t atoms = smem_u32(s_sfa + ib * sfa_bytes);
        for (int ks = 0; ks < nks; ++ks, ++it) {
          const int s = int(it % uint32_t(stages));
          if (!mbar_wait(&full[s], (it / stages) & 1, err, 2)) { ok = false; break; }
          tc_fence_after();
          const uint32_t a = smem_u32(ring + s * kLtA);
          const uint32_t b = smem_u32(s_b + ks * kLtB);
          const uint32_t sfa = tmem + kLtTmemSF + 16 * s, sfb = sfa + 8;
#pragma unroll
          for (int c = 0; c < 2; ++c) {
            tmem_cp_sf(sfa + 4 * c,
                       make_sdesc(atoms + (ks * 2 + c) * kLtAtom, 0, 128, kLayoutNone));
            tmem_cp_sf(sfb + 4 * c,
                       make_sdesc(smem_u32(s_sfb) + (ks * 2 + c) * kLtAtom, 0, 128, kLayoutNone));
          }
#pragma unroll
          for (int kb = 0; kb < 4; ++kb) {
            const int c = kb >> 1;
            const uint32_t byte = uint32_t(kb & 1) * 2;
            mma_mxf4(d, make_sdesc(a + kb * 32, 16, 1024, kLayoutSW128),
                     make_sdesc(b + kb * 32, 16, 1024, kLayoutSW128),
                     make_idesc_mxf4(kLtRows, kLtTok, int(byte), int(byte)),
                     (ks | kb) != 0 ? 1u : 0u, (sfa + 4 * c) | (byte << 30),
                     (sfb + 4 * c) | (byte << 30));
          }
          tc_commit(&empty[s]);
        }
        if (!ok) break;
        tc_commit(&acc_full[buf]);
        tc_commit(&sfa_empty[ib]);
      }
      if (!ok) drain_mma(drain);
    }
  } else {
    // ---- epilogue (warps 2-5, TMEM lane quadrant warp % 4) ----------------------
    const int quad = warp & 3;
    uint32_t ti = 0;
    for (int t = blockIdx.x; t < n_tiles; t += gridDim.x, ++ti) {
      const uint32_t buf = ti % kLtAccBufs;
      if (!mbar_wait(&acc_full[buf], (ti / kLtAccBufs) & 1, err, 3)) break;
      tc_fence_after();
      uint32_t r[32];
      tmem_ld_32x32b_x32(tmem + (uint32_t(quad * 32) << 16) + buf * 32, r);
      tmem_ld_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[buf]);
      const int n = t * kLtRows + quad * 32 + lane;
      if (n < N) {
#pragma unroll
        for (int j = 0; j < kLtTok; ++j)
          if (j < M) y[long(j) * ldy + n] = __uint_as_float(r[j]);
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kLtTmemCols);
  }
}

}  // namespace

bool lin_tc_supported(const void* xq, const uint8_t* xsc, const void* wp, const uint8_t* wsc, int M,
                      int Kp) {
  return M >= 1 && M <= kLtTok && Kp >= 512 && Kp % 512 == 0 && lt_stages(Kp) >= 2 &&
         (reinterpret_cast<uintptr_t>(xq) & 15) == 0 && (reinterpret_cast<uintptr_t>(wp) & 15) == 0 &&
         (reinterpret_cast<uintptr_t>(wsc) & 15) == 0 && (reinterpret_cast<uintptr_t>(xsc) & 3) == 0;
}

cudaError_t launch_lin_tc(const uint8_t* xq, const uint8_t* xsc, const uint8_t* wp,
                          const uint8_t* wsc, float* y, long long ldy, int M, int N, int Kp,
                          cudaStream_t stream) {
  if (!lin_tc_supported(xq, xsc, wp, wsc, M, Kp)) return cudaErrorNotSupported;
  if (N <= 0) return cudaSuccess;
  CUtensorMap tw, tx;
  if (!get_tmap(&tw, wp, uint64_t(Kp / 2), uint64_t(N), kLtRows) ||
      !get_tmap(&tx, xq, uint64_t(Kp / 2), uint64_t(M), kLtTok))
    return cudaErrorInvalidValue;
  const int stages = lt_stages(Kp);
  const LtLayout L = lt_layout(Kp, stages);
  cudaError_t e = ensure_dynamic_smem(reinterpret_cast<const void*>(lin_tc_kernel), L.bytes);
  if (e != cudaSuccess) return e;
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int n_tiles = (N + kLtRows - 1) / kLtRows;
  const int grid = n_tiles < sms ? n_tiles : sms;
  lin_tc_kernel<<<grid, kLtThreads, L.bytes, stream>>>(tw, tx, xsc, wsc, y, ldy, M, N, Kp, stages,
                                                       device_error_flag());
  return cudaGetLastError();
}

}  // namespace mfi
