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

// 2 CTAs per SM x 3 stages measured faster than 1 x 8 (two epilogues and two
// load streams per SM; the ring depth is not the limit)
#ifndef MFI_TC_STAGES
#define MFI_TC_STAGES 3
#endif
#ifndef MFI_TC_CTAS_PER_SM
#define MFI_TC_CTAS_PER_SM 2
#endif
constexpr int kStages = MFI_TC_STAGES;
constexpr int kCtasPerSm = MFI_TC_CTAS_PER_SM;
constexpr int kA = 16384;      // 128 rows x 128 B
constexpr int kB = 4096;       // 32 rows x 128 B
constexpr int kSF = 1024;      // two 512-byte atoms (2 x 128 K)
constexpr int kStageBytes = kA + kB + 2 * kSF;
// stage layout in shared memory: A (16 KB) | SFA (1 KB) | SFB (1 KB) | B (4 KB)
constexpr int kOffSFA = kA, kOffSFB = kA + kSF, kOffB = kA + 2 * kSF;
// prepared weight block in HBM: the A tile of one k-stage, already in the
// 128-byte-swizzled shared-memory order, followed by its two scale atoms
constexpr int kWBlock = kA + kSF;
constexpr int kThreads = 192;
constexpr int kAccBufs = 4;     // TMEM accumulators (32 fp32 columns each)
constexpr uint32_t kTmemCols = 256;
constexpr uint32_t kTmemSFA = kAccBufs * 32;
constexpr uint32_t kTmemSFB = kTmemSFA + 8;
constexpr int kChunk = 32;     // tokens per chunk (MMA N)

constexpr int kMaxExperts = 256;
// pairs (token, expert) per launch: T * top_k <= 4096 from the fused layer,
// rows * top_k <= 16384 from mfi_moe_experts
constexpr int kMaxPairs = 16384;
constexpr int kMaxChunks = kMaxExperts + kMaxPairs / kChunk;

struct MoeTcArgs {
  const int* counts;           // tokens routed to each expert (route.cu cursors)
  int E, T_pad;
  const int* perm;             // row -> (token * k + slot) for the rows of each expert region
  const uint8_t* wblocks;      // prepared weight blocks [expert][tile][k-stage][kWBlock]
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
  // speculative L2 prefetch, issued before the wait on the upstream kernels:
  // the first pf_bytes of this launch's weight blocks (storage order = item
  // order when every expert has one chunk), split evenly over the CTAs
  unsigned long long pf_bytes;
};

__device__ __forceinline__ void named_bar_sync(int id, int n) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n) : "memory");
}

template <bool kGateUp>
__global__ void __launch_bounds__(kThreads, kCtasPerSm)
    moe_tc_kernel(const __grid_constant__ CUtensorMap tma_b, MoeTcArgs p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint8_t* ring = smem;
  float* s_gu = reinterpret_cast<float*>(ring + kStages * kStageBytes);  // [2][128][33]
  uint64_t* full = reinterpret_cast<uint64_t*>(s_gu + 2 * 128 * 33);
  uint64_t* empty = full + kStages;
  uint64_t* acc_full = empty + kStages;
  uint64_t* acc_empty = acc_full + kAccBufs;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + kAccBufs);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int k_stages = p.K / 256;

  // prologue independent of the upstream kernels: barriers, TMEM, tensor map
  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < kAccBufs; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 4);
    }
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) prefetch_tmap(&tma_b);
  if (warp == 0 && p.pf_bytes) {
    // weights do not depend on the routing: stream the first blocks into L2
    // while the router (or the previous expert launch) is still running
    const unsigned long long per =
        ((p.pf_bytes + gridDim.x - 1) / gridDim.x + 4095) & ~4095ull;
    const unsigned long long lo = per * blockIdx.x;
    const unsigned long long hi = min(lo + per, p.pf_bytes);
    for (unsigned long long off = lo + lane * 32768ull; off < hi; off += 32 * 32768ull)
      prefetch_l2(p.wblocks + off, uint32_t(min(32768ull, hi - off)));
  }
  if (warp == 1) tmem_alloc(tmem_slot, kTmemCols);
  // counts, rows and activations come from the kernels before this one
  grid_dep_wait();
  grid_dep_launch();

  // chunk table from the per-expert token counts: chunk -> (expert, c), expert
  // e's tokens fill rows [e*T_pad, e*T_pad + count) in chunks of 32
  __shared__ int s_cnt[kMaxExperts];
  __shared__ int s_chunk[kMaxChunks];
  __shared__ int s_nchunks;
  for (int e = threadIdx.x; e < p.E; e += blockDim.x) s_cnt[e] = min(p.counts[e], p.T_pad);
  __syncthreads();
  if (warp == 0) {
    int run = 0;
    for (int e0 = 0; e0 < p.E; e0 += 32) {
      const int e = e0 + lane;
      const int nch = e < p.E ? (s_cnt[e] + kChunk - 1) / kChunk : 0;
      int inc = nch;
#pragma unroll
      for (int off = 1; off < 32; off <<= 1) {
        const int v = __shfl_up_sync(0xffffffffu, inc, off);
        if (lane >= off) inc += v;
      }
      for (int c = 0; c < nch; ++c)
        if (run + inc - nch + c < kMaxChunks) s_chunk[run + inc - nch + c] = e | (c << 16);
      run += __shfl_sync(0xffffffffu, inc, 31);
    }
    if (lane == 0) s_nchunks = min(run, kMaxChunks);
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const int n_items = s_nchunks * p.tiles;
  auto chunk_desc = [&](int chunk) {
    ChunkDesc cd;
    const int v = s_chunk[chunk];
    cd.expert = v & 0xffff;
    const int c = v >> 16;
    cd.count = min(kChunk, s_cnt[cd.expert] - kChunk * c);
    cd.row0 = cd.expert * p.T_pad + kChunk * c;
    cd.pad = 0;
    return cd;
  };

  if (warp == 0) {
    if (elect_one()) {
      uint32_t it = 0;
      bool ok = true;
      for (int item = blockIdx.x; ok && item < n_items; item += gridDim.x) {
        const int tile = item % p.tiles;
        const ChunkDesc cd = chunk_desc(item / p.tiles);
        const int e = cd.expert;
        for (int ks = 0; ks < k_stages; ++ks, ++it) {
          const int s = it % kStages;
          if (!mbar_wait(&empty[s], ((it / kStages) & 1) ^ 1, p.err, 1)) { ok = false; break; }
          uint8_t* st = ring + s * kStageBytes;
          mbar_expect_tx(&full[s], kStageBytes);
          const size_t blk = (size_t(e) * p.tiles + tile) * k_stages + ks;
          bulk_load(st, p.wblocks + blk * kWBlock, kWBlock, &full[s]);
          tma_load_2d(st + kOffB, &tma_b, ks * 128, cd.row0, &full[s]);
          bulk_load(st + kOffSFB, p.sfb + (size_t(cd.row0 / kChunk) * p.kc_pad + 2 * ks) * 512, kSF,
                    &full[s]);
        }
      }
    }
  } else if (warp == 1) {
    if (elect_one()) {
      uint32_t it = 0, acc_it = 0;
      bool ok = true;
      for (int item = blockIdx.x; ok && item < n_items; item += gridDim.x, ++acc_it) {
        const uint32_t buf = acc_it % kAccBufs;
        if (!mbar_wait(&acc_empty[buf], ((acc_it / kAccBufs) & 1) ^ 1, p.err, 2)) { ok = false; break; }
        tc_fence_after();
        const uint32_t d = tmem + buf * 32;
        for (int ks = 0; ks < k_stages; ++ks, ++it) {
          const int s = it % kStages;
          if (!mbar_wait(&full[s], (it / kStages) & 1, p.err, 2)) { ok = false; break; }
          tc_fence_after();
          const uint32_t base = smem_u32(ring + s * kStageBytes);
#pragma unroll
          for (int c = 0; c < 2; ++c) {
            tmem_cp_sf(tmem + kTmemSFA + 4 * c, make_sdesc(base + kOffSFA + c * 512, 0, 128, kLayoutNone));
            tmem_cp_sf(tmem + kTmemSFB + 4 * c, make_sdesc(base + kOffSFB + c * 512, 0, 128, kLayoutNone));
          }
#pragma unroll
          for (int kb = 0; kb < 4; ++kb) {
            const int c = kb >> 1;
            const uint32_t byte = uint32_t(kb & 1) * 2;
            mma_mxf4(d, make_sdesc(base + kb * 32, 16, 1024, kLayoutSW128),
                     make_sdesc(base + kOffB + kb * 32, 16, 1024, kLayoutSW128),
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
      const uint32_t buf = acc_it % kAccBufs;
      const int chunk = item / p.tiles, tile = item % p.tiles;
      // metadata loads issued before the wait so their latency overlaps it
      const ChunkDesc cd = chunk_desc(chunk);
      const int count = cd.count;
      const int row0 = cd.row0;
      const int my_pair = kGateUp ? 0 : p.perm[row0 + lane];
      if (!mbar_wait(&acc_full[buf], (acc_it / kAccBufs) & 1, p.err, 3)) break;
      tc_fence_after();
      uint32_t r[32];
      tmem_ld_32x32b_x32(tmem + (uint32_t(lane_base) << 16) + buf * 32, r);
      tmem_ld_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[buf]);
      if (kGateUp) {
        // rows 0-63 of the accumulator are gate outputs, rows 64-127 the up
        // outputs of the same 64 columns; columns are the chunk's tokens
        float* sg = s_gu + (acc_it & 1) * (128 * 33);
        float* row = sg + (lane_base + lane) * 33;
#pragma unroll
        for (int n = 0; n < 32; ++n)
          if (n < count) row[n] = __uint_as_float(r[n]);
        named_bar_sync(1, 128);
        // Only the chunk's `count` token columns are real: spread their
        // count x 2 blocks of 32 outputs over the 128 threads, G threads per
        // block (G a power of two in [2, 32]), q = 32 / G outputs per thread.
        int G = 32;
        while (G > 2 && 2 * count * G > 128) G >>= 1;
        const int q = 32 / G;
        const int task = et / G, sub = et % G;  // task = (token n, block b)
        const int n = task >> 1, b = task & 1;
        const bool active = n < count;          // uniform within each group of G
        const int j0 = b * 32 + sub * q;
        float h[16];
        float am = 0.0f;
        bool nan = false;
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          h[i] = 0.0f;
          if (active && i < q) {
            const float g = sg[(j0 + i) * 33 + n];
            const float u = sg[(64 + j0 + i) * 33 + n];
            h[i] = __fmul_rn(__fdiv_rn(g, __fadd_rn(1.0f, expf(-g))), u);
            am = fmaxf(am, fabsf(h[i]));
            nan |= (h[i] != h[i]);
          }
        }
        for (int off = 1; off < G; off <<= 1) {
          am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, off));
          nan |= __shfl_xor_sync(0xffffffffu, int(nan), off) != 0;
        }
        const BlockScale bs = block_scale(nan ? __uint_as_float(0x7fc00000u) : am);
        uint32_t w0 = 0, w1 = 0;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          if (i < q) w0 |= quant_nibble(h[i], bs.inv) << (4 * i);
          if (8 + i < q) w1 |= quant_nibble(h[8 + i], bs.inv) << (4 * i);
        }
        // q = 1: pair the nibbles of neighbouring threads into one byte
        const uint32_t nb_other = __shfl_xor_sync(0xffffffffu, w0, 1);
        if (active) {
          const int prow = row0 + n;
          uint8_t* dst = p.hp + size_t(prow) * (p.inter / 2) + tile * 32 + b * 16 + (sub * q) / 2;
          if (q == 16) *reinterpret_cast<uint2*>(dst) = make_uint2(w0, w1);
          else if (q == 8) *reinterpret_cast<uint32_t*>(dst) = w0;
          else if (q == 4) *reinterpret_cast<uint16_t*>(dst) = uint16_t(w0);
          else if (q == 2) *dst = uint8_t(w0);
          else if ((sub & 1) == 0) *dst = uint8_t(w0 | (nb_other << 4));
          if (sub == 0) {
            const int kb = tile * 2 + b;
            p.hp_atoms[(size_t(row0 / kChunk) * (p.inter / 128) + kb / 4) * 512 + n * 16 + (kb & 3)] =
                bs.code;
          }
        }
      } else {
        const int o = tile * 128 + lane_base + lane;
#pragma unroll
        for (int n = 0; n < kChunk; ++n) {
          if (n < count) {  // warp-uniform: columns past the chunk's tokens are skipped
            const int pair = __shfl_sync(0xffffffffu, my_pair, n);
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
  return 1024 + size_t(kStages) * kStageBytes + 2 * 128 * 33 * 4 + 8 * (2 * kStages + 2 * kAccBufs) +
         16;
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

// Prepared weight blocks.  Block (e, tile, ks) holds rows r = 0..127 of the
// tile (gate/up: rows 0-63 = gate rows tile*64 + r, rows 64-127 = the same up
// rows; down: rows tile*128 + r) restricted to K elements [ks*256, ks*256+256),
// i.e. 128 bytes per row, stored in the 128-byte-swizzle order TMA would
// produce (16-byte chunk c of row r at r*128 + ((c ^ (r % 8)) * 16)), followed
// by the two 512-byte scale atoms of those rows and K blocks.  One bulk copy
// then moves a whole stage's weights and scales from contiguous HBM.
__global__ void prepare_blocks_kernel(const uint8_t* __restrict__ wa, const uint8_t* __restrict__ sa,
                                      const uint8_t* __restrict__ wb, const uint8_t* __restrict__ sb,
                                      int E, int rows_per_e, int tile_rows, int K, bool paired,
                                      uint8_t* __restrict__ dst) {
  const int tiles = rows_per_e / tile_rows;
  const int k_stages = K / 256;
  const int nb = K / 32;
  const long long n_blocks = (long long)E * tiles * k_stages;
  const long long total = n_blocks * (kWBlock / 16);
  for (long long q = blockIdx.x * (long long)blockDim.x + threadIdx.x; q < total;
       q += (long long)gridDim.x * blockDim.x) {
    const long long blk = q / (kWBlock / 16);
    const int within = int(q % (kWBlock / 16)) * 16;  // byte offset inside the block
    const int ks = int(blk % k_stages);
    const long long et = blk / k_stages;
    const int tile = int(et % tiles), e = int(et / tiles);
    uint8_t* out = dst + blk * kWBlock + within;
    if (within < kA) {
      const int r = within >> 7;               // row inside the tile
      const int cpos = (within >> 4) & 7;      // swizzled chunk position
      const int c = cpos ^ (r & 7);            // logical 16-byte chunk
      const uint8_t* w = wa;
      int row;
      if (paired) {
        w = r < 64 ? wa : wb;
        row = e * rows_per_e + tile * 64 + (r & 63);
      } else {
        row = e * rows_per_e + tile * 128 + r;
      }
      *reinterpret_cast<uint4*>(out) =
          *reinterpret_cast<const uint4*>(w + size_t(row) * (K / 2) + ks * 128 + c * 16);
    } else {
      uint8_t v[16];
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const int off = within - kA + i;       // 0..1023 in the two atoms
        const int atom = off >> 9, ob = off & 511;
        const int r = (ob >> 4) + 32 * ((ob & 15) >> 2);
        const int kb = (2 * ks + atom) * 4 + (ob & 3);
        const uint8_t* sc = sa;
        int row;
        if (paired) {
          sc = r < 64 ? sa : sb;
          row = e * rows_per_e + tile * 64 + (r & 63);
        } else {
          row = e * rows_per_e + tile * 128 + r;
        }
        v[i] = sc[size_t(row) * nb + kb];
      }
      *reinterpret_cast<uint4*>(out) = *reinterpret_cast<const uint4*>(v);
    }
  }
}

}  // namespace

// ---------------------------------------------------------------------------
size_t moe_prepared_bytes(int E, int H, int Mi) {
  const size_t gu = size_t(E) * (Mi / 64) * (H / 256);
  const size_t dn = size_t(E) * (H / 128) * (Mi / 256);
  return (gu + dn) * kWBlock;
}

cudaError_t launch_moe_prepare(const uint8_t* gate_wp, const uint8_t* gate_sc,
                               const uint8_t* up_wp, const uint8_t* up_sc,
                               const uint8_t* down_wp, const uint8_t* down_sc, int E, int H, int Mi,
                               uint8_t* prepared, cudaStream_t stream) {
  uint8_t* gu = prepared;
  uint8_t* dn = prepared + size_t(E) * (Mi / 64) * (H / 256) * kWBlock;
  prepare_blocks_kernel<<<148 * 8, 256, 0, stream>>>(gate_wp, gate_sc, up_wp, up_sc, E, Mi, 64, H,
                                                     true, gu);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  prepare_blocks_kernel<<<148 * 8, 256, 0, stream>>>(down_wp, down_sc, nullptr, nullptr, E, H, 128,
                                                     Mi, false, dn);
  return cudaGetLastError();
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

static unsigned long long cap_prefetch(size_t want, size_t region) {
  return (unsigned long long)(want < region ? want : region) & ~15ull;
}

// Launch with programmatic stream serialisation when `pdl`: the kernel may
// start while the previous kernel in the stream drains (it waits with
// grid_dep_wait before reading that kernel's outputs).
template <class Kern>
static cudaError_t launch_ex(Kern kern, int grid, bool pdl, cudaStream_t stream,
                             const CUtensorMap& b, const MoeTcArgs& p) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = moe_tc_smem();
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kern, b, p);
}

cudaError_t launch_moe_tc(const MoeTcLaunch& L, cudaStream_t stream) {
  static bool smem_gu = false, smem_dn = false;
  const int E = L.E, H = L.H, Mi = L.Mi;
  CUtensorMap b;
  MoeTcArgs p{};
  p.counts = L.counts;
  p.E = L.E;
  p.T_pad = L.rows / L.E;
  p.perm = L.perm;
  p.inter = Mi;
  p.hidden = H;
  p.hp = L.hp;
  p.hp_atoms = L.hp_atoms;
  p.yd = L.yd;
  p.err = L.err;
  const int grid = L.grid * kCtasPerSm;
  if (L.gate_up) {
    if (!get_tmap(&b, L.xp, H / 2, uint64_t(L.rows), kChunk))
      return cudaErrorInvalidValue;
    p.wblocks = L.prepared;
    p.sfb = L.xp_atoms;
    p.K = H;
    p.tiles = Mi / 64;
    p.kc_pad = H / 128;
    p.pf_bytes = cap_prefetch(L.pf_bytes, size_t(E) * (Mi / 64) * (H / 256) * kWBlock);
    cudaError_t e = set_smem_once(reinterpret_cast<const void*>(moe_tc_kernel<true>), &smem_gu);
    if (e != cudaSuccess) return e;
    e = launch_ex(moe_tc_kernel<true>, grid, L.pdl, stream, b, p);
    if (e != cudaSuccess) return e;
  } else {
    if (!get_tmap(&b, L.hp, Mi / 2, uint64_t(L.rows), kChunk))
      return cudaErrorInvalidValue;
    p.wblocks = L.prepared + size_t(E) * (Mi / 64) * (H / 256) * kWBlock;
    p.sfb = L.hp_atoms;
    p.K = Mi;
    p.tiles = H / 128;
    p.kc_pad = Mi / 128;
    p.pf_bytes = cap_prefetch(L.pf_bytes, size_t(E) * (H / 128) * (Mi / 256) * kWBlock);
    cudaError_t e = set_smem_once(reinterpret_cast<const void*>(moe_tc_kernel<false>), &smem_dn);
    if (e != cudaSuccess) return e;
    e = launch_ex(moe_tc_kernel<false>, grid, L.pdl, stream, b, p);
    if (e != cudaSuccess) return e;
  }
  return cudaGetLastError();
}

}  // namespace mfi
