// moe_prefill.cu — prefill-sized grouped expert GEMMs on the tcgen05 tensor
// cores (many tokens per expert).
//
// Replaces the reference's prefill MoE (runtime/model_runner_v2.py:108-122:
// per expert, gather its tokens on the host and call mxfp4_linear three
// times) with one routed pass and no host synchronisation:
//
//   quant_x8_kernel,       quantise the tokens, route them on the tensor
//   route_tc_kernel        cores (route_tc.cu; route_batch_kernel for other
//                          router shapes), count tokens per expert and give
//                          each (token, slot) its position among its
//                          expert's tokens
//   prefill_scatter_kernel place each token's quantised row (and its scale
//                          atoms) at expert base + position, where the bases
//                          are the prefix sum of the per-expert counts rounded
//                          up to 128-row tiles (computed once per CTA)
//   moe_prefill_kernel     one persistent launch: gate/up items
//                          (128-token tile, 64 gate + 64 up weight rows) with
//                          SwiGLU + requantisation of h in the epilogue, then
//                          down items (128-token tile, 128 output rows) whose
//                          epilogue stores each (token, slot) row of y in bf16
//   combine_bf16_kernel    the top-k combine (slot order, unfused fp32
//                          multiply and add of the bf16 rows)
//
//   D (128 tokens x 128 weight rows) += X_tile (128 x 256 K) . W_tile^T,
//   tcgen05.mma.cta_group::1.kind::mxf4.block_scale, M = N = 128, K = 64.
//
// The weight operand is the decode path's prepared block (pre-swizzled rows +
// scale atoms, one bulk copy per stage); the token operand comes by TMA from
// the compact rows.  The down items of a tile wait (bounded) for the 12
// gate/up items of the same tile, as in moe_tc.cu.
#include "mx_common.cuh"
#include "tc_ptx.cuh"
#include "tmap.cuh"
#include "work.cuh"

namespace mfi {

using namespace tc;

namespace {

#ifndef MFI_PF_STAGES
#define MFI_PF_STAGES 4
#endif
constexpr int kPStages = MFI_PF_STAGES;
// warp 0 loads, warp 1 issues MMAs, warps 2-17 run the epilogue in two
// independent groups of eight: group g takes the accumulators of items
// g, g + 2, g + 4, ... of the CTA, so one group's SwiGLU overlaps the other's
// (no CTA-wide barrier between items).  Inside a group two warps share each
// TMEM lane quadrant, each taking one 32-element block of h (gate/up) or 64
// output columns (down) of its 32 token rows.  The last warp publishes the
// finished h slices of each gate/up item to the down items of every CTA: the
// epilogue warps hand it each accumulator use through an mbarrier and go on
// to their next item, so the fences that make h visible at GPU scope (and to
// the async proxy that reads it) stay off the epilogue's path.
constexpr int kPEpiWarps = 16;
constexpr int kPGroups = 2;
constexpr int kPGroupWarps = kPEpiWarps / kPGroups;
constexpr int kPPubWarp = 2 + kPEpiWarps;
constexpr int kPThreads = 64 + 32 * kPEpiWarps + 32;
// publisher hand-off markers (besides a gate/up item's tile index)
constexpr int kPubDown = -1, kPubStop = -2;
constexpr int kPTile = 128;                    // token rows per tile (MMA M)
constexpr int kPA = 16384;                     // 128 token rows x 128 B
constexpr int kPSF = 1024;                     // two scale atoms
constexpr int kPW = 16384 + 1024;              // prepared weight block (tile + atoms)
constexpr int kPOffSFA = kPA;
constexpr int kPOffW = kPA + kPSF;             // 1024-byte aligned
constexpr int kPOffSFB = kPOffW + 16384;
constexpr int kPStageBytes = kPA + kPSF + kPW; // 34816
// down epilogue: per warp a 32-row x 32-column fp32 staging tile, so that each
// global store instruction writes whole 128-byte row segments (four rows per
// instruction) instead of 16 bytes of 32 different rows
constexpr int kPOutStage = 32 * 32 * 4;
constexpr int kPAccBufs = 3;                   // 128 fp32 columns each
constexpr uint32_t kPTmemCols = 512;
constexpr uint32_t kPTmemSFA = kPAccBufs * 128;  // + 16 per ring slot: SFA 8 columns, SFB 8
constexpr uint32_t kPTmemSFB = kPTmemSFA + 8;
static_assert(kPTmemSFA + 16 * kPStages <= kPTmemCols, "scale-factor columns exceed the allocation");
constexpr int kPMaxExperts = 256;
constexpr int kPMaxChunks = kPMaxExperts + kPrefillMaxPairs / kPTile;

struct PrefillArgs {
  const int* counts;           // tokens per expert (router cursors)
  int E;
  const int* perm;             // row -> pair (token * k + slot)
  const uint8_t* w_gu;         // prepared gate/up blocks [expert][Mi/64][H/256][block]
  const uint8_t* w_dn;         // prepared down blocks [expert][H/128][Mi/256][block]
  const uint8_t* xa;           // token-row scale atoms [row/128][H/128][512]
  uint8_t* hp;                 // requantised h rows (rows, inter/2)
  uint8_t* ha;                 // their scale atoms [row/128][inter/128][512]
  __nv_bfloat16* yd;           // (pairs, hidden) bf16 per-(token, slot) down rows
  int hidden, inter, top_k;
  int* err;
  int* queue;                  // work-item counter, zero before the launch
  unsigned* gu_done;           // finished gate/up warp slices in all, zero before the launch
  unsigned* ready;             // per tile: finished gate/up warp slices, zero before the launch
};

__device__ __forceinline__ void fence_proxy_async_global() {
  asm volatile("fence.proxy.async.global;" ::: "memory");
}
// Two fp32 values (as bits) -> packed bf16 pair, round to nearest even.
__device__ __forceinline__ uint32_t bf16x2_bits(uint32_t lo, uint32_t hi) {
  const __nv_bfloat162 v = __floats2bfloat162_rn(__uint_as_float(lo), __uint_as_float(hi));
  return *reinterpret_cast<const uint32_t*>(&v);
}
__device__ __forceinline__ unsigned ld_acquire_u32(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Rows of expert e start at base[e] = sum over e' < e of counts rounded up to
// 128.  Warp 0 of the calling CTA fills s_base[0..E) and returns the total.
__device__ int expert_bases(const int* s_cnt, int E, int* s_base) {
  const int lane = threadIdx.x & 31;
  int run = 0;
  for (int e0 = 0; e0 < E; e0 += 32) {
    const int e = e0 + lane;
    const int v = e < E ? (s_cnt[e] + kPTile - 1) / kPTile * kPTile : 0;
    int inc = v;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const int u = __shfl_up_sync(0xffffffffu, inc, off);
      if (lane >= off) inc += u;
    }
    if (e < E) s_base[e] = run + inc - v;
    run += __shfl_sync(0xffffffffu, inc, 31);
  }
  return run;
}

// One CTA per kScTok tokens: copy each token's quantised row and scale atoms
// to its k expert rows (the expert bases are computed once per CTA).  Row t's
// expert list is topi[t * sel_ld + j]; entries outside [0, E) (slots of
// received rows that name no local expert) are skipped.
constexpr int kScTok = 4;
constexpr int kScThreads = 256;
__global__ void __launch_bounds__(kScThreads) prefill_scatter_kernel(
    const uint8_t* __restrict__ xq, long long xq_ld, const uint8_t* __restrict__ xsc,
    long long xsc_ld, const int* __restrict__ topi, long long sel_ld,
    const int* __restrict__ slot_pos, const int* __restrict__ counts, int T, int E, int k, int H,
    int* __restrict__ perm, uint8_t* __restrict__ xp, uint8_t* __restrict__ xa) {
  const int tok0 = blockIdx.x * kScTok;
  const int nt = min(kScTok, T - tok0);
  __shared__ int s_cnt[kPMaxExperts];
  __shared__ int s_base[kPMaxExperts];
  __shared__ int s_row[kScTok * 32];
  for (int e = threadIdx.x; e < E; e += blockDim.x) s_cnt[e] = counts[e];
  __syncthreads();
  if (threadIdx.x < 32) expert_bases(s_cnt, E, s_base);
  __syncthreads();
  for (int p = threadIdx.x; p < nt * k; p += blockDim.x) {
    const int t = tok0 + p / k, j = p % k;
    const long pair = long(t) * k + j;
    const int e = topi[size_t(t) * sel_ld + j];
    int row = -1;
    if (unsigned(e) < unsigned(E)) {
      row = s_base[e] + slot_pos[pair];
      perm[row] = int(pair);
    }
    s_row[p] = row;
  }
  __syncthreads();
  const int q16 = H / 32, kc = H / 128;
  for (int p = threadIdx.x; p < nt * k * q16; p += blockDim.x) {
    const int pj = p / q16, c = p - pj * q16;  // pair (token i = pj / k), 16-byte chunk c
    if (s_row[pj] < 0) continue;
    reinterpret_cast<uint4*>(xp + size_t(s_row[pj]) * (H / 2))[c] =
        reinterpret_cast<const uint4*>(xq + size_t(tok0 + pj / k) * xq_ld)[c];
  }
  for (int p = threadIdx.x; p < nt * k * kc; p += blockDim.x) {
    const int pj = p / kc, c = p - pj * kc;
    const int row = s_row[pj];
    if (row < 0) continue;
    *reinterpret_cast<uint32_t*>(xa + (size_t(row / kPTile) * kc + c) * 512 + (row % 32) * 16 +
                                 ((row % kPTile) / 32) * 4) =
        reinterpret_cast<const uint32_t*>(xsc + size_t(tok0 + pj / k) * xsc_ld)[c];
  }
}

// Positions of pre-routed (row, slot) pairs among their expert's rows, for
// rows that arrive already routed (expert parallelism): slot_pos[r * k + j] =
// the count of expert sel[r][j] before it (atomic claim, so the order of the
// rows inside a region varies between runs; every row's result does not
// depend on it).  Slots naming no local expert (outside [0, E)) are skipped;
// ids >= E are reported as error 4.
__global__ void __launch_bounds__(256) prefill_count_sel_kernel(
    const int* __restrict__ sel, long long sel_ld, int R, int k, int E, int* __restrict__ counts,
    int* __restrict__ slot_pos, int* __restrict__ status) {
  const long i = long(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= long(R) * k) return;
  const int r = int(i / k), j = int(i % k);
  const int e = sel[size_t(r) * sel_ld + j];
  if (e >= E) atomicCAS(status, 0, 4);
  slot_pos[i] = unsigned(e) < unsigned(E) ? atomicAdd(counts + e, 1) : -1;
}

__global__ void __launch_bounds__(kPThreads, 1)
    moe_prefill_kernel(const __grid_constant__ CUtensorMap tma_x,
                       const __grid_constant__ CUtensorMap tma_h, PrefillArgs p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* ring = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint8_t* out_stage = ring + kPStages * kPStageBytes;  // [kPEpiWarps][32 rows][128 B]
  uint64_t* full = reinterpret_cast<uint64_t*>(out_stage + kPEpiWarps * kPOutStage);
  uint64_t* empty = full + kPStages;
  uint64_t* acc_full = empty + kPStages;
  uint64_t* acc_empty = acc_full + kPAccBufs;
  uint64_t* item_full = acc_empty + kPAccBufs;
  uint64_t* item_empty = item_full + kPAccBufs;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(item_empty + kPAccBufs);
  __shared__ int s_item[kPAccBufs];
  __shared__ uint64_t drain[1];  // the MMA issuer's error-path drain
  // epilogue group -> publisher, one slot per accumulator buffer
  __shared__ uint64_t pub_full[kPAccBufs], pub_empty[kPAccBufs];
  __shared__ int pub_tl[kPAccBufs];

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tiles_gu = p.inter / 64, tiles_dn = p.hidden / 128;
  const int ks_gu = p.hidden / 256, ks_dn = p.inter / 256;
  const int kc_gu = p.hidden / 128, kc_dn = p.inter / 128;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kPStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < kPAccBufs; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], kPGroupWarps);
      mbar_init(&item_full[b], 1);
      mbar_init(&item_empty[b], 1 + kPGroupWarps);  // the MMA thread + one epilogue group
      mbar_init(&pub_full[b], kPGroupWarps);
      mbar_init(&pub_empty[b], 1);
    }
    mbar_init(drain, 1);
    fence_mbar_init();
    cta_abort_init();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&tma_x);
    prefetch_tmap(&tma_h);
  }
  if (warp == 1) tmem_alloc(tmem_slot, kPTmemCols);
  int first_item = 0;
  if (warp == 0 && lane == 0) first_item = atomicAdd(p.queue, 1);
  grid_dep_wait();
  grid_dep_launch();

  // tile table: tile -> (expert, m) with rows [base[e] + 128 m, + count)
  __shared__ int s_cnt[kPMaxExperts];
  __shared__ int s_base[kPMaxExperts];
  __shared__ int s_tile[kPMaxChunks];
  __shared__ int s_ntiles;
  for (int e = threadIdx.x; e < p.E; e += blockDim.x) s_cnt[e] = p.counts[e];
  __syncthreads();
  if (warp == 0) {
    expert_bases(s_cnt, p.E, s_base);
    int run = 0;
    for (int e0 = 0; e0 < p.E; e0 += 32) {
      const int e = e0 + lane;
      const int nt = e < p.E ? (s_cnt[e] + kPTile - 1) / kPTile : 0;
      int inc = nt;
#pragma unroll
      for (int off = 1; off < 32; off <<= 1) {
        const int v = __shfl_up_sync(0xffffffffu, inc, off);
        if (lane >= off) inc += v;
      }
      for (int m = 0; m < nt; ++m)
        if (run + inc - nt + m < kPMaxChunks) s_tile[run + inc - nt + m] = e | (m << 16);
      run += __shfl_sync(0xffffffffu, inc, 31);
    }
    if (lane == 0) s_ntiles = min(run, kPMaxChunks);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const int n_gu = s_ntiles * tiles_gu;
  const int n_items = n_gu + s_ntiles * tiles_dn;
  auto tile_of = [&](int tl, int& expert, int& row0, int& count) {
    const int v = s_tile[tl];
    expert = v & 0xffff;
    const int m = v >> 16;
    row0 = s_base[expert] + kPTile * m;
    count = min(kPTile, s_cnt[expert] - kPTile * m);
  };
  auto decode = [&](int item, bool& gu, int& tl, int& tile) {
    gu = item < n_gu;
    const int i = gu ? item : item - n_gu;
    const int tiles = gu ? tiles_gu : tiles_dn;
    tl = i / tiles;
    tile = i % tiles;
  };

  if (warp == 0) {
    first_item = __shfl_sync(0xffffffffu, first_item, 0);
    if (elect_one()) {
      uint32_t it = 0;
      bool ok = true;
      bool all_ready = false;  // every gate/up item has published its h rows
      int item = first_item;
      int next = atomicAdd(p.queue, 1);  // items are claimed two ahead
      int stops = 0;
      for (uint32_t qi = 0; ok; ++qi) {
        const uint32_t slot = qi % kPAccBufs;
        if (!mbar_wait(&item_empty[slot], ((qi / kPAccBufs) & 1) ^ 1, p.err, 1)) { ok = false; break; }
        if (item >= n_items) item = -1;
        s_item[slot] = item;
        mbar_arrive(&item_full[slot]);
        if (item < 0) {
          // one end marker per epilogue group (consecutive slots)
          if (++stops == kPGroups) break;
          continue;
        }
        const int next2 = atomicAdd(p.queue, 1);
        bool gu;
        int tl, tile, e, row0, count;
        decode(item, gu, tl, tile);
        tile_of(tl, e, row0, count);
        const uint8_t* wb;
        if (gu) {
          wb = p.w_gu + (size_t(e) * tiles_gu + tile) * ks_gu * size_t(kPW);
        } else {
          wb = p.w_dn + (size_t(e) * tiles_dn + tile) * ks_dn * size_t(kPW);
          const unsigned tile_slices = unsigned(tiles_gu) * kPGroupWarps;
          if (!all_ready && ld_acquire_u32(p.gu_done) >= unsigned(n_gu) * kPGroupWarps)
            all_ready = true;
          if (!all_ready && ld_acquire_u32(p.ready + tl) < tile_slices) {
            const uint64_t t0 = globaltimer_ns();
            for (uint32_t i = 1;; ++i) {
              __nanosleep(64);
              if (ld_acquire_u32(p.ready + tl) >= tile_slices) break;
              if ((i & 255u) == 0) {
                if (cta_aborted()) { ok = false; break; }
                if (globaltimer_ns() - t0 > kWaitLimitNs) {
                  cta_fail(p.err, 4);
                  ok = false;
                  break;
                }
              }
            }
            if (!ok) break;
          }
          fence_proxy_async_global();
        }
        const int ksn = gu ? ks_gu : ks_dn;
        const int kc = gu ? kc_gu : kc_dn;
        const uint8_t* sfa = gu ? p.xa : p.ha;
        const CUtensorMap* ta = gu ? &tma_x : &tma_h;
        for (int ks = 0; ks < ksn; ++ks, ++it) {
          const int s = it % kPStages;
          if (!mbar_wait(&empty[s], ((it / kPStages) & 1) ^ 1, p.err, 1)) { ok = false; break; }
          uint8_t* st = ring + s * kPStageBytes;
          mbar_expect_tx(&full[s], kPStageBytes);
          tma_load_2d(st, ta, ks * 128, row0, &full[s]);
          bulk_load(st + kPOffSFA, sfa + (size_t(row0 / kPTile) * kc + 2 * ks) * 512, kPSF, &full[s]);
          bulk_load(st + kPOffW, wb + size_t(ks) * kPW, kPW, &full[s]);
        }
        item = next;
        next = next2;
      }
      if (!ok) drain_ring(full, kPStages, it);
    }
  } else if (warp == 1) {
    if (elect_one()) {
      uint32_t it = 0;
      bool ok = true;
      int stops = 0;
      for (uint32_t acc_it = 0; ok; ++acc_it) {
        const uint32_t buf = acc_it % kPAccBufs;
        if (!mbar_wait(&item_full[buf], (acc_it / kPAccBufs) & 1, p.err, 2)) { ok = false; break; }
        const int item = s_item[buf];
        mbar_arrive(&item_empty[buf]);
        if (!mbar_wait(&acc_empty[buf], ((acc_it / kPAccBufs) & 1) ^ 1, p.err, 2)) { ok = false; break; }
        if (item < 0) {
          mbar_arrive(&acc_full[buf]);
          if (++stops == kPGroups) break;
          continue;
        }
        const int ksn = item < n_gu ? ks_gu : ks_dn;
        tc_fence_after();
        const uint32_t d = tmem + buf * 128;
        for (int ks = 0; ks < ksn; ++ks, ++it) {
          const int s = it % kPStages;
          if (!mbar_wait(&full[s], (it / kPStages) & 1, p.err, 2)) { ok = false; break; }
          tc_fence_after();
          const uint32_t base = smem_u32(ring + s * kPStageBytes);
          // each ring slot has its own scale-factor columns, so the copy for
          // this stage need not wait for the MMAs of the previous one
          const uint32_t sfa = tmem + kPTmemSFA + 16 * s, sfb = tmem + kPTmemSFB + 16 * s;
#pragma unroll
          for (int c = 0; c < 2; ++c) {
            tmem_cp_sf(sfa + 4 * c, make_sdesc(base + kPOffSFA + c * 512, 0, 128, kLayoutNone));
            tmem_cp_sf(sfb + 4 * c, make_sdesc(base + kPOffSFB + c * 512, 0, 128, kLayoutNone));
          }
#pragma unroll
          for (int kb = 0; kb < 4; ++kb) {
            const int c = kb >> 1;
            const uint32_t byte = uint32_t(kb & 1) * 2;
            mma_mxf4(d, make_sdesc(base + kb * 32, 16, 1024, kLayoutSW128),
                     make_sdesc(base + kPOffW + kb * 32, 16, 1024, kLayoutSW128),
                     make_idesc_mxf4(128, 128, int(byte), int(byte)), (ks | kb) != 0 ? 1u : 0u,
                     (sfa + 4 * c) | (byte << 30), (sfb + 4 * c) | (byte << 30));
          }
          tc_commit(&empty[s]);
        }
        if (ok) tc_commit(&acc_full[buf]);
      }
      if (!ok) drain_mma(drain);
    }
  } else if (warp == kPPubWarp) {
    if (lane == 0) {
      int stops = 0;
      for (uint32_t acc_it = 0;; ++acc_it) {
        const uint32_t buf = acc_it % kPAccBufs;
        if (!mbar_wait(&pub_full[buf], (acc_it / kPAccBufs) & 1, p.err, 3)) break;
        const int tl = pub_tl[buf];
        mbar_arrive(&pub_empty[buf]);
        if (tl == kPubStop) {
          if (++stops == kPGroups) break;
          continue;
        }
        if (tl >= 0) {
          // the group's 8 warps wrote their h slices (and released them to
          // this thread through the barrier): make them visible to the
          // down items' producers, which read h with TMA
          fence_proxy_async_global();
          __threadfence();
          atomicAdd(p.ready + tl, unsigned(kPGroupWarps));
          atomicAdd(p.gu_done, unsigned(kPGroupWarps));
        }
      }
    }
  } else {
    const int ew = warp - 2;             // 0..15
    const int quad = warp & 3;           // TMEM lane quadrant of this warp
    const int grp = ew / kPGroupWarps;   // epilogue group
    const int half = (ew >> 2) & 1;      // which half of the tile's columns
    const int r = quad * 32 + lane;      // token row inside the tile
    // lane 0 hands accumulator use acc_it to the publisher (after the warp's
    // stores: the __syncwarp before the call orders them)
    auto hand_off = [&](uint32_t acc_it, int tl) -> bool {
      const uint32_t buf = acc_it % kPAccBufs;
      if (!mbar_wait(&pub_empty[buf], ((acc_it / kPAccBufs) & 1) ^ 1, p.err, 3)) return false;
      pub_tl[buf] = tl;
      mbar_arrive(&pub_full[buf]);
      return true;
    };
    for (uint32_t acc_it = grp;; acc_it += kPGroups) {
      const uint32_t buf = acc_it % kPAccBufs;
      if (!mbar_wait(&item_full[buf], (acc_it / kPAccBufs) & 1, p.err, 3)) break;
      const int item = s_item[buf];
      __syncwarp();
      if (lane == 0) mbar_arrive(&item_empty[buf]);
      if (item < 0) {
        mbar_wait(&acc_full[buf], (acc_it / kPAccBufs) & 1, p.err, 3);
        if (lane == 0) hand_off(acc_it, kPubStop);
        break;
      }
      bool gu;
      int tl, tile, e, row0, count;
      decode(item, gu, tl, tile);
      tile_of(tl, e, row0, count);
      const bool valid = r < count;
      const int row = row0 + r;
      const int pair = (!gu && valid) ? p.perm[row] : 0;
      if (!mbar_wait(&acc_full[buf], (acc_it / kPAccBufs) & 1, p.err, 3)) break;
      tc_fence_after();
      const uint32_t tbase = tmem + (uint32_t(quad * 32) << 16) + buf * 128;
      if (gu) {
        // columns 0-63: gate outputs tile*64 + c, 64-127: the same up outputs;
        // this warp takes h block `half` (outputs half*32 .. +31) whole, so
        // the block maximum needs no exchange with another warp
        // h goes through this warp's staging tile in shared memory (lane l
        // keeps its 32 values in its own 128-byte row, 16-byte chunk c at
        // chunk c ^ (l & 7), so the 16-byte stores and loads of both passes
        // are free of bank conflicts), and gate / up come in loads of 4 TMEM
        // columns: the SwiGLU pass and the quantisation pass each hold only a
        // few values, and the warp stays within the 96 registers a thread of
        // this 18-warp block has, without spilling.  The block maximum uses a
        // NaN-propagating max, so a NaN anywhere in the block gives code 127
        // (scale 1), like quant_group8.
        float4* hs4 = reinterpret_cast<float4*>(out_stage + ew * kPOutStage) + lane * 8;
        float am = 0.0f;
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          uint32_t gq[4], u[4];
          tmem_ld_32x32b_x4(tbase + half * 32 + q * 4, gq);
          tmem_ld_32x32b_x4(tbase + 64 + half * 32 + q * 4, u);
          tmem_ld_wait();
          if (q == 7) {
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&acc_empty[buf]);
          }
          float h[4];
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            h[i] = swiglu(__uint_as_float(gq[i]), __uint_as_float(u[i]));
            am = fmax_nan(am, fabsf(h[i]));
          }
          hs4[q ^ (lane & 7)] = make_float4(h[0], h[1], h[2], h[3]);
        }
        const BlockScale bs = block_scale(am);
        uint32_t w[4] = {0u, 0u, 0u, 0u};
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          const float4 v = hs4[c ^ (lane & 7)];
          const int i = 4 * c;
          w[i >> 3] |= (quant_nibble(v.x, bs.inv) << (4 * (i & 7))) |
                       (quant_nibble(v.y, bs.inv) << (4 * ((i + 1) & 7))) |
                       (quant_nibble(v.z, bs.inv) << (4 * ((i + 2) & 7))) |
                       (quant_nibble(v.w, bs.inv) << (4 * ((i + 3) & 7)));
        }
        if (valid) {
          *reinterpret_cast<uint4*>(p.hp + size_t(row) * (p.inter / 2) + tile * 32 + half * 16) =
              make_uint4(w[0], w[1], w[2], w[3]);
          const int kb = tile * 2 + half;  // 32-element block of h along inter
          p.ha[(size_t(row / kPTile) * kc_dn + kb / 4) * 512 + (row % 32) * 16 +
               ((row % kPTile) / 32) * 4 + (kb & 3)] = bs.code;
        }
        // this warp's slice (32 rows x one block) of the tile's h rows goes
        // to the publisher
        __syncwarp();
        int handed = 1;
        if (lane == 0) handed = hand_off(acc_it, tl) ? 1 : 0;
        if (__shfl_sync(0xffffffffu, handed, 0) == 0) break;
      } else {
        // this warp stores output columns half*64 .. +63 of its token rows in
        // bf16 (each expert's output row is rounded to the activation type,
        // as the reference's prefill does with y, runtime/model_runner_v2.py
        // :119), transposed through shared memory: lane r holds row r (128
        // bytes); the stores go out as 4 rows x 8 lanes x 16 B.  16-byte
        // chunk q of row r sits at chunk q ^ (r & 7), so both phases are free
        // of bank conflicts.
        uint4* stg = reinterpret_cast<uint4*>(out_stage + ew * kPOutStage);
        uint32_t y[32], pk[32];
        tmem_ld_32x32b_x32(tbase + half * 64, y);
        tmem_ld_wait();
#pragma unroll
        for (int i = 0; i < 16; ++i) pk[i] = bf16x2_bits(y[2 * i], y[2 * i + 1]);
        tmem_ld_32x32b_x32(tbase + half * 64 + 32, y);
        tmem_ld_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&acc_empty[buf]);
#pragma unroll
        for (int i = 0; i < 16; ++i) pk[16 + i] = bf16x2_bits(y[2 * i], y[2 * i + 1]);
#pragma unroll
        for (int q = 0; q < 8; ++q)
          stg[lane * 8 + (q ^ (lane & 7))] =
              make_uint4(pk[4 * q], pk[4 * q + 1], pk[4 * q + 2], pk[4 * q + 3]);
        __syncwarp();
        const int sub_row = lane >> 3, chunk = lane & 7;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const int rr = 4 * i + sub_row;  // row of this lane's store
          const int pr = __shfl_sync(0xffffffffu, pair, rr);
          const bool ok_row = __shfl_sync(0xffffffffu, int(valid), rr) != 0;
          const uint4 v = stg[rr * 8 + (chunk ^ (rr & 7))];
          if (ok_row)
            *reinterpret_cast<uint4*>(p.yd + size_t(pr) * p.hidden + tile * 128 + half * 64 +
                                      chunk * 8) = v;
        }
        __syncwarp();
        int handed = 1;
        if (lane == 0) handed = hand_off(acc_it, kPubDown) ? 1 : 0;
        if (__shfl_sync(0xffffffffu, handed, 0) == 0) break;
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kPTmemCols);
  }
}

size_t prefill_smem() {
  return 1024 + size_t(kPStages) * kPStageBytes + size_t(kPEpiWarps) * kPOutStage +
         8 * (2 * kPStages + 4 * kPAccBufs) + 16;
}

}  // namespace

// ---------------------------------------------------------------------------
size_t prefill_rows(int pairs, int E) {
  // every expert's rows rounded up to a whole tile
  const size_t active = size_t(pairs < E ? pairs : E);
  return (size_t(pairs) + kPTile - 1) / kPTile * kPTile + active * kPTile;
}

cudaError_t launch_prefill_scatter(const uint8_t* xq, long long xq_ld, const uint8_t* xsc,
                                   long long xsc_ld, const int* topi, long long sel_ld,
                                   const int* slot_pos, const int* counts, int T, int E, int k,
                                   int H, int* perm, uint8_t* xp, uint8_t* xa,
                                   cudaStream_t stream) {
  if (T == 0) return cudaSuccess;
  prefill_scatter_kernel<<<(T + kScTok - 1) / kScTok, kScThreads, 0, stream>>>(
      xq, xq_ld, xsc, xsc_ld, topi, sel_ld, slot_pos, counts, T, E, k, H, perm, xp, xa);
  return cudaGetLastError();
}

cudaError_t launch_prefill_count_sel(const int* sel, long long sel_ld, int R, int k, int E,
                                     int* counts, int* slot_pos, int* status,
                                     cudaStream_t stream) {
  const long n = long(R) * k;
  if (n == 0) return cudaSuccess;
  prefill_count_sel_kernel<<<unsigned((n + 255) / 256), 256, 0, stream>>>(sel, sel_ld, R, k, E,
                                                                           counts, slot_pos, status);
  return cudaGetLastError();
}

cudaError_t launch_moe_prefill(const PrefillLaunch& L, cudaStream_t stream) {
  if (L.queue == nullptr || L.ready == nullptr || L.gu_done == nullptr) return cudaErrorInvalidValue;
  {
    cudaError_t e = ensure_dynamic_smem(reinterpret_cast<const void*>(moe_prefill_kernel),
                                        prefill_smem());
    if (e != cudaSuccess) return e;
  }
  const int E = L.E, H = L.H, Mi = L.Mi;
  CUtensorMap tx, th;
  if (!get_tmap(&tx, L.xp, H / 2, uint64_t(L.rows), kPTile) ||
      !get_tmap(&th, L.hp, Mi / 2, uint64_t(L.rows), kPTile))
    return cudaErrorInvalidValue;
  PrefillArgs p{};
  p.counts = L.counts;
  p.E = E;
  p.perm = L.perm;
  p.w_gu = L.prepared;
  p.w_dn = L.prepared + size_t(E) * (Mi / 64) * (H / 256) * kPW;
  p.xa = L.xa;
  p.hp = L.hp;
  p.ha = L.ha;
  p.yd = L.yd;
  p.hidden = H;
  p.inter = Mi;
  p.top_k = L.top_k;
  p.err = L.err;
  p.queue = L.queue;
  p.gu_done = L.gu_done;
  p.ready = L.ready;
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(L.grid);
  cfg.blockDim = dim3(kPThreads);
  cfg.dynamicSmemBytes = prefill_smem();
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = L.pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, moe_prefill_kernel, tx, th, p);
}

}  // namespace mfi
