// moe_tc.cu — decode-sized grouped expert GEMMs on the tcgen05 tensor cores.
//
// Replaces, inside the fused layer, the reference's per-(token, slot) kernels
// gateup_kernel and down_silu_kernel (src/ext/mxfp4_decode.cu:177-279), which
// re-read an expert's weights for every (token, slot) pair that picks it and
// use 1/16 of each m16 MMA tile.  Here decode is a weight-streaming problem
// and the tensor core does the FP4 decode for free ("swap AB"):
//
//   D^T (128 weight rows x 32 tokens) += W_tile (128 x 256 K) . X_chunk^T,
//   tcgen05.mma.kind::mxf4.block_scale, M = 128, N = 32, K = 64 per instruction.
//
// Tokens routed to one expert are packed in chunks of up to 32 rows
// (route.cu builds the chunk table; gather_chunks_kernel packs the rows and
// their scale atoms).  A persistent CTA per SM walks work items
// (chunk, weight tile) with
//   warp 0     TMA loads of the weight tile (A), the chunk tile (B) and bulk
//              copies of both scale-factor atoms into an 8-stage ring,
//   warp 1     tcgen05.cp of the scales into TMEM + 4 MMAs per stage into one
//              of two TMEM accumulators (32 fp32 columns each),
//   warps 2-5  epilogue of the previous item while the next one streams.
//
// gate/up items take 64 gate rows and the same 64 up rows as one 128-row A
// tile (two TMA boxes), so the epilogue has g and u for the same outputs: it
// computes h = g / (1 + exp(-g)) * u in fp32 (src/ext/mxfp4_decode.cu:258),
// requantises each 32-element block of h with the library's quantiser and
// writes the packed h rows plus their scale atoms — the B operand of the down
// items.  down items write per-(token, slot) rows of y for the deterministic
// combine.  Every wait is bounded (see tc_ptx.cuh).
#include "mx_common.cuh"
#include "tc_ptx.cuh"
#include "tmap.cuh"
#include "work.cuh"

namespace mfi {

using namespace tc;

namespace {

constexpr int kStages = 8;
constexpr int kA = 16384;      // 128 rows x 128 B
constexpr int kB = 4096;       // 32 rows x 128 B
constexpr int kSF = 1024;      // two 512-byte atoms (2 x 128 K)
constexpr int kStageBytes = kA + kB + 2 * kSF;
constexpr int kThreads = 192;
constexpr uint32_t kTmemCols = 128;
constexpr uint32_t kTmemSFA = 64;
constexpr uint32_t kTmemSFB = 72;
constexpr int kChunk = 32;     // tokens per chunk (MMA N)

struct MoeTcArgs {
  const ChunkDesc* chunks;
  const int* n_chunks;
  const int* perm;             // chunk row -> (token * k + slot), -1 for padding
  const uint8_t* sfa;          // weight scale atoms
  const uint8_t* sfb;          // chunk scale atoms [chunk][kc_pad][512]
  int K;                       // reduction length (hidden or inter), multiple of 256
  int tiles;                   // weight tiles per chunk
  int kc_pad;                  // atoms per 128-row block along K (= K / 128)
  // gate/up
  int inter;
  uint8_t* hp;                 // (rows, inter/2)
  uint8_t* hp_atoms;           // [chunk][inter/128][512]
  // down
  int hidden;
  float* yd;                   // (T*k, hidden)
  int* err;
};

__device__ __forceinline__ void named_bar_sync(int id, int n) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n) : "memory");
}

template <bool kGateUp>
__global__ void __launch_bounds__(kThreads, 1)
    moe_tc_kernel(const __grid_constant__ CUtensorMap tma_a0,
                  const __grid_constant__ CUtensorMap tma_a1,
                  const __grid_constant__ CUtensorMap tma_b, MoeTcArgs p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint8_t* ring = smem;
  float* su = reinterpret_cast<float*>(ring + kStages * kStageBytes);  // [64][33]
  float* sh = su + 64 * 33;                                           // [32][65]
  uint64_t* full = reinterpret_cast<uint64_t*>(sh + 32 * 65);
  uint64_t* empty = full + kStages;
  uint64_t* acc_full = empty + kStages;
  uint64_t* acc_empty = acc_full + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int k_stages = p.K / 256;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 4);
    }
    fence_mbar_init();
  }
  if (warp == 1) tmem_alloc(tmem_slot, kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const int n_items = *p.n_chunks * p.tiles;

  if (warp == 0) {
    if (elect_one()) {
      prefetch_tmap(&tma_a0);
      if (kGateUp) prefetch_tmap(&tma_a1);
      prefetch_tmap(&tma_b);
      uint32_t it = 0;
      bool ok = true;
      for (int item = blockIdx.x; ok && item < n_items; item += gridDim.x) {
        const int chunk = item / p.tiles, tile = item % p.tiles;
        const int e = p.chunks[chunk].expert;
        for (int ks = 0; ks < k_stages; ++ks, ++it) {
          const int s = it % kStages;
          if (!mbar_wait(&empty[s], ((it / kStages) & 1) ^ 1, p.err, 1)) { ok = false; break; }
          uint8_t* st = ring + s * kStageBytes;
          mbar_expect_tx(&full[s], kStageBytes);
          if (kGateUp) {
            const int row = e * p.inter + tile * 64;
            tma_load_2d(st, &tma_a0, ks * 128, row, &full[s]);
            tma_load_2d(st + kA / 2, &tma_a1, ks * 128, row, &full[s]);
          } else {
            tma_load_2d(st, &tma_a0, ks * 128, e * p.hidden + tile * 128, &full[s]);
          }
          tma_load_2d(st + kA, &tma_b, ks * 128, chunk * kChunk, &full[s]);
          const size_t arow = kGateUp ? size_t(e) * p.tiles + tile
                                      : (size_t(e) * p.hidden + size_t(tile) * 128) / 128;
          bulk_load(st + kA + kB, p.sfa + (arow * p.kc_pad + 2 * ks) * 512, kSF, &full[s]);
          bulk_load(st + kA + kB + kSF, p.sfb + (size_t(chunk) * p.kc_pad + 2 * ks) * 512, kSF,
                    &full[s]);
        }
      }
    }
  } else if (warp == 1) {
    if (elect_one()) {
      uint32_t it = 0, acc_it = 0;
      bool ok = true;
      for (int item = blockIdx.x; ok && item < n_items; item += gridDim.x, ++acc_it) {
        const uint32_t buf = acc_it & 1;
        if (!mbar_wait(&acc_empty[buf], ((acc_it >> 1) & 1) ^ 1, p.err, 2)) { ok = false; break; }
        tc_fence_after();
        const uint32_t d = tmem + buf * 32;
        for (int ks = 0; ks < k_stages; ++ks, ++it) {
          const int s = it % kStages;
          if (!mbar_wait(&full[s], (it / kStages) & 1, p.err, 2)) { ok = false; break; }
          tc_fence_after();
          const uint32_t base = smem_u32(ring + s * kStageBytes);
#pragma unroll
          for (int c = 0; c < 2; ++c) {
            tmem_cp_sf(tmem + kTmemSFA + 4 * c, make_sdesc(base + kA + kB + c * 512, 0, 128, kLayoutNone));
            tmem_cp_sf(tmem + kTmemSFB + 4 * c,
                       make_sdesc(base + kA + kB + kSF + c * 512, 0, 128, kLayoutNone));
          }
#pragma unroll
          for (int kb = 0; kb < 4; ++kb) {
            const int c = kb >> 1;
            const uint32_t byte = uint32_t(kb & 1) * 2;
            mma_mxf4(d, make_sdesc(base + kb * 32, 16, 1024, kLayoutSW128),
                     make_sdesc(base + kA + kb * 32, 16, 1024, kLayoutSW128),
                     make_idesc_mxf4(128, kChunk, int(byte), int(byte)), (ks | kb) != 0 ? 1u : 0u,
                     (tmem + kTmemSFA + 4 * c) | (byte << 30), (tmem + kTmemSFB + 4 * c) | (byte << 30));
          }
          tc_commit(&empty[s]);
        }
        if (ok) tc_commit(&acc_full[buf]);
      }
    }
  } else {
    const int lane_base = (warp & 3) * 32;
    const int et = threadIdx.x - 64;  // 0..127
    uint32_t acc_it = 0;
    for (int item = blockIdx.x; item < n_items; item += gridDim.x, ++acc_it) {
      const uint32_t buf = acc_it & 1;
      if (!mbar_wait(&acc_full[buf], (acc_it >> 1) & 1, p.err, 3)) break;
      tc_fence_after();
      uint32_t r[32];
      tmem_ld_32x32b_x32(tmem + (uint32_t(lane_base) << 16) + buf * 32, r);
      tmem_ld_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[buf]);
      const int chunk = item / p.tiles, tile = item % p.tiles;
      const int count = p.chunks[chunk].count;
      if (kGateUp) {
        if (lane_base >= 64) {
          float* row = su + (lane_base - 64 + lane) * 33;
#pragma unroll
          for (int n = 0; n < 32; ++n) row[n] = __uint_as_float(r[n]);
        }
        named_bar_sync(1, 128);
        if (lane_base < 64) {
          const int j = lane_base + lane;
          const float* urow = su + j * 33;
#pragma unroll
          for (int n = 0; n < 32; ++n) {
            const float g = __uint_as_float(r[n]);
            sh[n * 65 + j] = __fmul_rn(__fdiv_rn(g, __fadd_rn(1.0f, expf(-g))), urow[n]);
          }
        }
        named_bar_sync(1, 128);
        if (et < 64) {
          const int n = et >> 1, b = et & 1;
          if (n < count) {
            const float* hv = sh + n * 65 + b * 32;
            float am = 0.0f;
            bool nan = false;
#pragma unroll
            for (int i = 0; i < 32; ++i) {
              am = fmaxf(am, fabsf(hv[i]));
              nan |= (hv[i] != hv[i]);
            }
            const BlockScale bs = block_scale(nan ? __uint_as_float(0x7fc00000u) : am);
            uint32_t w[4] = {0, 0, 0, 0};
#pragma unroll
            for (int i = 0; i < 32; ++i) w[i >> 3] |= quant_nibble(hv[i], bs.inv) << (4 * (i & 7));
            const int prow = chunk * kChunk + n;
            *reinterpret_cast<uint4*>(p.hp + size_t(prow) * (p.inter / 2) + tile * 32 + b * 16) =
                make_uint4(w[0], w[1], w[2], w[3]);
            const int kb = tile * 2 + b;
            p.hp_atoms[(size_t(chunk) * (p.inter / 128) + kb / 4) * 512 + n * 16 + (kb & 3)] = bs.code;
          }
        }
        named_bar_sync(1, 128);
      } else {
        const int o = tile * 128 + lane_base + lane;
#pragma unroll
        for (int n = 0; n < kChunk; ++n) {
          if (n < count) {
            const int pair = p.perm[chunk * kChunk + n];
            p.yd[size_t(pair) * p.hidden + o] = __uint_as_float(r[n]);
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

size_t moe_tc_smem() {
  return 1024 + size_t(kStages) * kStageBytes + (64 * 33 + 32 * 65) * 4 +
         8 * (2 * kStages + 4) + 16;
}

// ---------------------------------------------------------------------------
// Pack each chunk's token rows (packed activations) and scale atoms.
// One warp per chunk row: 16 bytes per lane per pass.
__global__ void __launch_bounds__(256) gather_chunks_kernel(const uint8_t* __restrict__ xq,
                                                            const uint8_t* __restrict__ xsc,
                                                            const int* __restrict__ perm,
                                                            const int* __restrict__ n_chunks,
                                                            int k, int H, uint8_t* __restrict__ xp,
                                                            uint8_t* __restrict__ xp_atoms) {
  const int rows = *n_chunks * kChunk;
  const int lane = threadIdx.x & 31;
  const int nb = H / 32, kc = H / 128;
  for (int r = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; r < rows;
       r += (gridDim.x * blockDim.x) >> 5) {
    const int pair = perm[r];
    const int tok = pair >= 0 ? pair / k : -1;
    uint4* dst = reinterpret_cast<uint4*>(xp + size_t(r) * (H / 2));
    const uint4* src = reinterpret_cast<const uint4*>(xq + size_t(tok < 0 ? 0 : tok) * (H / 2));
    for (int i = lane; i < H / 32; i += 32) dst[i] = tok >= 0 ? src[i] : make_uint4(0, 0, 0, 0);
    const int chunk = r / kChunk, i = r % kChunk;
    for (int a = lane; a < kc; a += 32) {
      uint32_t v = 0x7f7f7f7fu;
      if (tok >= 0) v = *reinterpret_cast<const uint32_t*>(xsc + size_t(tok) * nb + 4 * a);
      *reinterpret_cast<uint32_t*>(xp_atoms + (size_t(chunk) * kc + a) * 512 + i * 16) = v;
    }
  }
}

// Gate/up scale atoms for 128-row tiles made of 64 gate rows and the same 64
// up rows: atom (e, tile, kc), rows 0-63 from gate, 64-127 from up.
__global__ void gu_atoms_kernel(const uint8_t* __restrict__ gsc, const uint8_t* __restrict__ usc,
                                int E, int Mi, int H, uint8_t* __restrict__ dst) {
  const int tiles = Mi / 64, kc = H / 128, nb = H / 32;
  const long long total = (long long)E * tiles * kc * 512;
  for (long long q = blockIdx.x * (long long)blockDim.x + threadIdx.x; q < total;
       q += (long long)gridDim.x * blockDim.x) {
    const int within = int(q & 511);
    const long long atom = q >> 9;
    const int a = int(atom % kc);
    const long long et = atom / kc;
    const int tile = int(et % tiles), e = int(et / tiles);
    const int r = (within >> 4) + 32 * ((within & 15) >> 2);
    const int kb = a * 4 + (within & 3);
    const uint8_t* src = r < 64 ? gsc : usc;
    const int row = e * Mi + tile * 64 + (r & 63);
    dst[q] = src[size_t(row) * nb + kb];
  }
}

}  // namespace

// ---------------------------------------------------------------------------
size_t moe_prepared_bytes(int E, int H, int Mi) {
  return size_t(E) * (Mi / 64) * (H / 128) * 512 + size_t(E) * (H / 128) * (Mi / 128) * 512;
}

cudaError_t launch_moe_prepare(const uint8_t* gate_sc, const uint8_t* up_sc,
                               const uint8_t* down_sc, int E, int H, int Mi, uint8_t* prepared,
                               cudaStream_t stream) {
  uint8_t* gu = prepared;
  uint8_t* dn = prepared + size_t(E) * (Mi / 64) * (H / 128) * 512;
  gu_atoms_kernel<<<148 * 8, 256, 0, stream>>>(gate_sc, up_sc, E, Mi, H, gu);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  return launch_sf_atoms(down_sc, Mi / 32, E * H, Mi, 128, dn, stream);
}

cudaError_t launch_gather_chunks(const uint8_t* xq, const uint8_t* xsc, const int* perm,
                                 const int* n_chunks, int max_chunks, int k, int H, uint8_t* xp,
                                 uint8_t* xp_atoms, cudaStream_t stream) {
  const int rows = max_chunks * kChunk;
  int blocks = (rows * 32 + 255) / 256;
  if (blocks > 148 * 8) blocks = 148 * 8;
  if (blocks < 1) blocks = 1;
  gather_chunks_kernel<<<blocks, 256, 0, stream>>>(xq, xsc, perm, n_chunks, k, H, xp, xp_atoms);
  return cudaGetLastError();
}

static cudaError_t set_smem_once(const void* fn, bool* done) {
  if (*done) return cudaSuccess;
  cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       int(moe_tc_smem()));
  if (e == cudaSuccess) *done = true;
  return e;
}

cudaError_t launch_moe_tc(const MoeTcLaunch& L, cudaStream_t stream) {
  static bool smem_gu = false, smem_dn = false;
  const int E = L.E, H = L.H, Mi = L.Mi;
  const uint8_t* prep_gu = L.prepared;
  const uint8_t* prep_dn = L.prepared + size_t(E) * (Mi / 64) * (H / 128) * 512;
  CUtensorMap a0, a1, b;
  MoeTcArgs p{};
  p.chunks = L.chunks;
  p.n_chunks = L.n_chunks;
  p.perm = L.perm;
  p.inter = Mi;
  p.hidden = H;
  p.hp = L.hp;
  p.hp_atoms = L.hp_atoms;
  p.yd = L.yd;
  p.err = L.err;
  const int grid = L.grid;
  if (L.gate_up) {
    if (!get_tmap(&a0, L.gate_wp, H / 2, uint64_t(E) * Mi, 64) ||
        !get_tmap(&a1, L.up_wp, H / 2, uint64_t(E) * Mi, 64) ||
        !get_tmap(&b, L.xp, H / 2, uint64_t(L.max_chunks) * kChunk, kChunk))
      return cudaErrorInvalidValue;
    p.sfa = prep_gu;
    p.sfb = L.xp_atoms;
    p.K = H;
    p.tiles = Mi / 64;
    p.kc_pad = H / 128;
    cudaError_t e = set_smem_once(reinterpret_cast<const void*>(moe_tc_kernel<true>), &smem_gu);
    if (e != cudaSuccess) return e;
    moe_tc_kernel<true><<<grid, kThreads, moe_tc_smem(), stream>>>(a0, a1, b, p);
  } else {
    if (!get_tmap(&a0, L.down_wp, Mi / 2, uint64_t(E) * H, 128) ||
        !get_tmap(&b, L.hp, Mi / 2, uint64_t(L.max_chunks) * kChunk, kChunk))
      return cudaErrorInvalidValue;
    p.sfa = prep_dn;
    p.sfb = L.hp_atoms;
    p.K = Mi;
    p.tiles = H / 128;
    p.kc_pad = Mi / 128;
    cudaError_t e = set_smem_once(reinterpret_cast<const void*>(moe_tc_kernel<false>), &smem_dn);
    if (e != cudaSuccess) return e;
    moe_tc_kernel<false><<<grid, kThreads, moe_tc_smem(), stream>>>(a0, a0, b, p);
  }
  return cudaGetLastError();
}

}  // namespace mfi
