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
// The router (route.cu) writes each token's quantised row into per-expert
// regions; tokens of one expert form chunks of up to 32 rows.  One persistent
// launch (2 CTAs per SM) runs gate/up and down: work items (chunk, weight
// tile) come from a global counter in order — all gate/up items first, then
// the down items, each of which waits (bounded) until the gate/up items of
// its chunk have published the chunk's requantised h rows.  Per CTA
//   warp 0     bulk copies of the pre-swizzled weight block (A + its scale
//              atoms, one contiguous copy per stage), TMA of the chunk's rows
//              (B) and a bulk copy of their scale atoms into a 3-stage ring,
//   warp 1     tcgen05.cp of the scales into TMEM + 4 MMAs per stage into one
//              of four TMEM accumulators (32 fp32 columns each),
//   warps 2-5  epilogue of earlier items while the next ones stream.
//
// gate/up items take 64 gate rows and the same 64 up rows as one 128-row A
// tile, so the epilogue has g and u for the same outputs: it computes
// h = g / (1 + exp(-g)) * u in fp32 (src/ext/mxfp4_decode.cu:258), requantises
// each 32-element block of h with the library's quantiser and writes the
// packed h rows plus their scale atoms — the B operand of the down items.
// down items write per-(token, slot) rows of y for the deterministic combine.
// Every wait is bounded (see tc_ptx.cuh).
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
constexpr uint32_t kTmemSFA = kAccBufs * 32;   // + 16 per ring slot: SFA 8 columns, SFB 8
constexpr uint32_t kTmemSFB = kTmemSFA + 8;
static_assert(kTmemSFA + 16 * kStages <= kTmemCols, "scale-factor columns exceed the allocation");
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
  const uint8_t* w_gu;         // prepared gate/up blocks [expert][Mi/64][H/256][kWBlock]
  const uint8_t* w_dn;         // prepared down blocks [expert][H/128][Mi/256][kWBlock]
  const uint8_t* sfb_x;        // token-row scale atoms [chunk][H/128][512]
  uint8_t* hp;                 // requantised h rows (rows, inter/2)
  uint8_t* hp_atoms;           // their scale atoms [chunk][inter/128][512]
  int hidden, inter;
  float* yd;                   // (pairs, hidden) per-(token, slot) down outputs
  int* err;
  int* queue;                  // work-item counter, zero before the launch
  unsigned* ready;             // per chunk: finished gate/up items, zero before the launch
  // speculative L2 prefetch, issued before the wait on the upstream kernels:
  // the first pf_bytes of the gate/up blocks (storage order = item order when
  // every expert has one chunk), split evenly over the CTAs
  unsigned long long pf_bytes;
};

__device__ __forceinline__ void named_bar_sync(int id, int n) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n) : "memory");
}
// Order this thread's generic-proxy global accesses with its async-proxy
// (TMA / bulk copy) accesses.
__device__ __forceinline__ void fence_proxy_async_global() {
  asm volatile("fence.proxy.async.global;" ::: "memory");
}
__device__ __forceinline__ unsigned ld_acquire_u32(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// One persistent launch runs both expert GEMMs of the layer.  Work items,
// handed out in order by a global counter:
//   [0, n_gu)          gate/up items (chunk, 64-row gate+up tile), K = hidden
//   [n_gu, n_items)    down items (chunk, 128-row output tile), K = inter
// A down item's B operand (the chunk's requantised h rows) is complete once
// all inter/64 gate/up items of its chunk have published it: their epilogues
// bump ready[chunk] (release), the down producer polls it (acquire, bounded)
// and then reads h through the async proxy.  Items are only ever taken by
// running CTAs and every down item follows all gate/up items in the queue, so
// the wait always ends (no assumption that the grid is co-resident).
__global__ void __launch_bounds__(kThreads, kCtasPerSm)
    moe_experts_kernel(const __grid_constant__ CUtensorMap tma_x,
                       const __grid_constant__ CUtensorMap tma_h, MoeTcArgs p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint8_t* ring = smem;
  float* s_gu = reinterpret_cast<float*>(ring + kStages * kStageBytes);  // [2][128][33]
  uint64_t* full = reinterpret_cast<uint64_t*>(s_gu + 2 * 128 * 33);
  uint64_t* empty = full + kStages;
  uint64_t* acc_full = empty + kStages;
  uint64_t* acc_empty = acc_full + kAccBufs;
  uint64_t* item_full = acc_empty + kAccBufs;
  uint64_t* item_empty = item_full + kAccBufs;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(item_empty + kAccBufs);
  __shared__ int s_item[kAccBufs];  // work item of each accumulator slot (-1: no more work)
  __shared__ uint64_t drain[1];     // the MMA issuer's error-path drain

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tiles_gu = p.inter / 64, tiles_dn = p.hidden / 128;
  const int ks_gu = p.hidden / 256, ks_dn = p.inter / 256;
  const int kc_gu = p.hidden / 128, kc_dn = p.inter / 128;

  // prologue independent of the upstream kernels: barriers, TMEM, tensor maps
  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < kAccBufs; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 4);
      mbar_init(&item_full[b], 1);
      mbar_init(&item_empty[b], 5);  // the MMA thread + the 4 epilogue warps
    }
    mbar_init(drain, 1);
    fence_mbar_init();
    cta_abort_init();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&tma_x);
    prefetch_tmap(&tma_h);
  }
  if (warp == 0 && p.pf_bytes) {
    // weights do not depend on the routing: stream the first blocks into L2
    // while the router is still running
    const unsigned long long per =
        ((p.pf_bytes + gridDim.x - 1) / gridDim.x + 4095) & ~4095ull;
    const unsigned long long lo = per * blockIdx.x;
    const unsigned long long hi = min(lo + per, p.pf_bytes);
    for (unsigned long long off = lo + lane * 32768ull; off < hi; off += 32 * 32768ull)
      prefetch_l2(p.w_gu + off, uint32_t(min(32768ull, hi - off)));
  }
  if (warp == 1) tmem_alloc(tmem_slot, kTmemCols);
  // the counter was zeroed before the kernel ahead of this one started, so
  // the first claim may overlap the wait
  int first_item = 0;
  if (warp == 0 && lane == 0) first_item = atomicAdd(p.queue, 1);
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
  const int n_gu = s_nchunks * tiles_gu;
  const int n_items = n_gu + s_nchunks * tiles_dn;
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
  // item -> (gate/up?, chunk, tile)
  auto decode = [&](int item, bool& gu, int& chunk, int& tile) {
    gu = item < n_gu;
    const int i = gu ? item : item - n_gu;
    const int tiles = gu ? tiles_gu : tiles_dn;
    chunk = i / tiles;
    tile = i % tiles;
  };

  if (warp == 0) {
    first_item = __shfl_sync(0xffffffffu, first_item, 0);
    if (elect_one()) {
      uint32_t it = 0;
      bool ok = true;
      int item = first_item;
      for (uint32_t qi = 0; ok; ++qi) {
        const uint32_t slot = qi % kAccBufs;
        if (!mbar_wait(&item_empty[slot], ((qi / kAccBufs) & 1) ^ 1, p.err, 1)) { ok = false; break; }
        if (item >= n_items) item = -1;
        s_item[slot] = item;
        mbar_arrive(&item_full[slot]);
        if (item < 0) break;
        // claim the next item now; its value is needed only after this
        // item's loads are issued
        const int next = atomicAdd(p.queue, 1);
        bool gu;
        int chunk, tile;
        decode(item, gu, chunk, tile);
        const ChunkDesc cd = chunk_desc(chunk);
        const int ksn = gu ? ks_gu : ks_dn;
        const uint8_t* wb;
        // a down item's weight blocks do not depend on the h rows it waits
        // for: the first ring-full of them goes out before the wait, so their
        // latency overlaps it (each stage's barrier completes once the h rows
        // of the stage have landed too)
        const int pre = gu ? 0 : min(ksn, kStages);
        int pre_issued = 0;
        if (gu) {
          wb = p.w_gu + (size_t(cd.expert) * tiles_gu + tile) * ks_gu * size_t(kWBlock);
        } else {
          wb = p.w_dn + (size_t(cd.expert) * tiles_dn + tile) * ks_dn * size_t(kWBlock);
          for (; pre_issued < pre; ++pre_issued) {
            const uint32_t j = it + uint32_t(pre_issued);
            const int s = int(j % kStages);
            if (!mbar_wait(&empty[s], ((j / kStages) & 1) ^ 1, p.err, 1)) { ok = false; break; }
            mbar_expect_tx(&full[s], kStageBytes);
            bulk_load_stream(ring + s * kStageBytes, wb + size_t(pre_issued) * kWBlock, kWBlock,
                             &full[s]);
          }
          if (!ok) {
            it += uint32_t(pre_issued);  // the drain covers the copies already issued
            break;
          }
          // the chunk's h rows: published by its tiles_gu gate/up items
          if (ld_acquire_u32(p.ready + chunk) < unsigned(tiles_gu)) {
            const uint64_t t0 = globaltimer_ns();
            for (uint32_t i = 1;; ++i) {
              __nanosleep(64);
              if (ld_acquire_u32(p.ready + chunk) >= unsigned(tiles_gu)) break;
              if ((i & 255u) == 0) {
                if (cta_aborted()) { ok = false; break; }
                if (globaltimer_ns() - t0 > kWaitLimitNs) {
                  cta_fail(p.err, 4);
                  ok = false;
                  break;
                }
              }
            }
            if (!ok) {
              it += uint32_t(pre_issued);
              break;
            }
          }
          fence_proxy_async_global();
        }
        const int kc = gu ? kc_gu : kc_dn;
        const uint8_t* sfb = gu ? p.sfb_x : p.hp_atoms;
        const CUtensorMap* tb = gu ? &tma_x : &tma_h;
        for (int ks = 0; ks < ksn; ++ks, ++it) {
          const int s = it % kStages;
          uint8_t* st = ring + s * kStageBytes;
          if (ks >= pre_issued) {
            if (!mbar_wait(&empty[s], ((it / kStages) & 1) ^ 1, p.err, 1)) { ok = false; break; }
            mbar_expect_tx(&full[s], kStageBytes);
            bulk_load_stream(st, wb + size_t(ks) * kWBlock, kWBlock, &full[s]);
          }
          tma_load_2d(st + kOffB, tb, ks * 128, cd.row0, &full[s]);
          bulk_load(st + kOffSFB, sfb + (size_t(cd.row0 / kChunk) * kc + 2 * ks) * 512, kSF,
                    &full[s]);
        }
        item = next;
      }
      if (!ok) drain_ring(full, kStages, it);
    }
  } else if (warp == 1) {
    if (elect_one()) {
      uint32_t it = 0;
      bool ok = true;
      for (uint32_t acc_it = 0; ok; ++acc_it) {
        const uint32_t buf = acc_it % kAccBufs;
        if (!mbar_wait(&item_full[buf], (acc_it / kAccBufs) & 1, p.err, 2)) { ok = false; break; }
        const int item = s_item[buf];
        mbar_arrive(&item_empty[buf]);
        if (!mbar_wait(&acc_empty[buf], ((acc_it / kAccBufs) & 1) ^ 1, p.err, 2)) { ok = false; break; }
        if (item < 0) {
          mbar_arrive(&acc_full[buf]);  // tells the epilogue there is no more work
          break;
        }
        const int ksn = item < n_gu ? ks_gu : ks_dn;
        tc_fence_after();
        const uint32_t d = tmem + buf * 32;
        for (int ks = 0; ks < ksn; ++ks, ++it) {
          const int s = it % kStages;
          if (!mbar_wait(&full[s], (it / kStages) & 1, p.err, 2)) { ok = false; break; }
          tc_fence_after();
          const uint32_t base = smem_u32(ring + s * kStageBytes);
          // each ring slot has its own scale-factor columns, so the copy for
          // this stage need not wait for the MMAs of the previous one
          const uint32_t sfa = tmem + kTmemSFA + 16 * s, sfb = tmem + kTmemSFB + 16 * s;
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
                     make_idesc_mxf4(128, kChunk, int(byte), int(byte)), (ks | kb) != 0 ? 1u : 0u,
                     (sfa + 4 * c) | (byte << 30), (sfb + 4 * c) | (byte << 30));
          }
          tc_commit(&empty[s]);
        }
        if (ok) tc_commit(&acc_full[buf]);
      }
      if (!ok) drain_mma(drain);
    }
  } else {
    const int lane_base = (warp & 3) * 32;
    const int et = threadIdx.x - 64;  // 0..127
    for (uint32_t acc_it = 0;; ++acc_it) {
      const uint32_t buf = acc_it % kAccBufs;
      if (!mbar_wait(&item_full[buf], (acc_it / kAccBufs) & 1, p.err, 3)) break;
      const int item = s_item[buf];
      __syncwarp();
      if (lane == 0) mbar_arrive(&item_empty[buf]);
      if (item < 0) {
        // consume the final acc_full phase so the barrier is left in order
        mbar_wait(&acc_full[buf], (acc_it / kAccBufs) & 1, p.err, 3);
        break;
      }
      bool gu;
      int chunk, tile;
      decode(item, gu, chunk, tile);
      // metadata loads issued before the wait so their latency overlaps it
      const ChunkDesc cd = chunk_desc(chunk);
      const int count = cd.count;
      const int row0 = cd.row0;
      const int my_pair = gu ? 0 : p.perm[row0 + lane];
      if (!mbar_wait(&acc_full[buf], (acc_it / kAccBufs) & 1, p.err, 3)) break;
      tc_fence_after();
      uint32_t r[32];
      tmem_ld_32x32b_x32(tmem + (uint32_t(lane_base) << 16) + buf * 32, r);
      tmem_ld_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[buf]);
      if (gu) {
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
            h[i] = swiglu(g, u);
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
            p.hp_atoms[(size_t(row0 / kChunk) * kc_dn + kb / 4) * 512 + n * 16 + (kb & 3)] =
                bs.code;
          }
        }
        // publish this tile of the chunk's h rows to the down items (the
        // barrier also frees s_gu for reuse)
        named_bar_sync(1, 128);
        if (et == 0) {
          fence_proxy_async_global();
          __threadfence();
          atomicAdd(p.ready + chunk, 1u);
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
  return 1024 + size_t(kStages) * kStageBytes + 2 * 128 * 33 * 4 + 8 * (2 * kStages + 4 * kAccBufs) +
         16;
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

static unsigned long long cap_prefetch(size_t want, size_t region) {
  return (unsigned long long)(want < region ? want : region) & ~15ull;
}

cudaError_t launch_moe_tc(const MoeTcLaunch& L, cudaStream_t stream) {
  if (L.queue == nullptr || L.ready == nullptr) return cudaErrorInvalidValue;
  {
    cudaError_t e = ensure_dynamic_smem(reinterpret_cast<const void*>(moe_experts_kernel),
                                        moe_tc_smem());
    if (e != cudaSuccess) return e;
  }
  const int E = L.E, H = L.H, Mi = L.Mi;
  CUtensorMap tx, th;
  if (!get_tmap(&tx, L.xp, H / 2, uint64_t(L.rows), kChunk) ||
      !get_tmap(&th, L.hp, Mi / 2, uint64_t(L.rows), kChunk))
    return cudaErrorInvalidValue;
  MoeTcArgs p{};
  p.counts = L.counts;
  p.E = E;
  p.T_pad = L.rows / E;
  p.perm = L.perm;
  p.w_gu = L.prepared;
  p.w_dn = L.prepared + size_t(E) * (Mi / 64) * (H / 256) * kWBlock;
  p.sfb_x = L.xp_atoms;
  p.hp = L.hp;
  p.hp_atoms = L.hp_atoms;
  p.hidden = H;
  p.inter = Mi;
  p.yd = L.yd;
  p.err = L.err;
  p.queue = L.queue;
  p.ready = L.ready;
  p.pf_bytes = cap_prefetch(L.pf_bytes, size_t(E) * (Mi / 64) * (H / 256) * kWBlock);
  // programmatic stream serialisation when `pdl`: the kernel may start while
  // the previous kernel in the stream drains (it waits with grid_dep_wait
  // before reading that kernel's outputs)
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(L.grid * kCtasPerSm);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = moe_tc_smem();
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = L.pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, moe_experts_kernel, tx, th, p);
}

}  // namespace mfi
