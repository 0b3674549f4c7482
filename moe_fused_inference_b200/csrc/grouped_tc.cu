// grouped_tc.cu — the drop-in grouped operators (moe_gateup, moe_down and
// their _tab forms) on the tcgen05 tensor cores.
//
// Replaces, for the operators the reference's model runner calls unchanged
// (runtime/model_runner_v2.py:195-207, 279-289), the reference's
// per-(token, slot, projection) kernels gateup_kernel / down_silu_kernel
// (src/ext/mxfp4_decode.cu:177-279).  The caller's pointer tables are grouped
// on the device (gemv.cu build_groups_kernel): one group per distinct weight
// matrix, listing the activation rows that multiply it.  A work item is
// (group, chunk of up to 32 of its rows, tile of 128 weight rows), computed
// "swap AB" like the decode expert kernel:
//
//   D^T (128 weight rows x 32 rows) += W_tile (128 x 256 K) . X_chunk^T,
//   tcgen05.mma.kind::mxf4.block_scale, M = 128, N = 32, K = 64,
//
// each weight tile streamed from HBM once per chunk.  The weights are the
// caller's raw row-major tensors at arbitrary (16-byte aligned) addresses, so
// there is no tensor map per weight: four producer warps copy each stage with
// 16-byte cp.async into the 128-byte-swizzled layout the MMA reads (chunk c of
// row r at r*128 + (c ^ r%8)*16), gather the chunk's activation rows the same
// way, and write both operands' E8M0 codes as the 512-byte scale atoms
// tcgen05.cp moves into TMEM.  Completion: each producer waits for its own
// copies of a stage (cp.async.wait_group with several stages in flight),
// fences the generic-proxy writes against the tensor core's async-proxy
// reads, and arrives on the stage's barrier.
//   warps 0-3  producers            warp 4     MMA issue (one thread)
//   warps 5-8  epilogue: tcgen05.ld of the 128 x 32 accumulator, stores of
//              each real row's 128 outputs to its entry's output offset
// Items are taken round-robin by a persistent grid (items are of equal cost).
// Every wait is bounded (tc_ptx.cuh).
#include "mx_common.cuh"
#include "tc_ptx.cuh"
#include "tmap.cuh"
#include "work.cuh"

namespace mfi {

using namespace tc;

namespace {

constexpr int kGtRows = 128;          // weight rows per tile (MMA M)
constexpr int kGtTok = 32;            // activation rows per chunk (MMA N)
constexpr int kGtA = 16384;           // 128 rows x 128 B per 256-K stage
constexpr int kGtB = 4096;            // 32 rows x 128 B
constexpr int kGtSF = 1024;           // two 512-byte atoms per operand and stage
constexpr int kGtOffB = kGtA, kGtOffSFA = kGtA + kGtB, kGtOffSFB = kGtOffSFA + kGtSF;
constexpr int kGtStage = kGtOffSFB + kGtSF;  // 22528, a multiple of 1024
constexpr int kGtStages = 6;
constexpr int kGtLag = kGtStages - 2;        // stages a producer keeps in flight
constexpr int kGtProducers = 128;
constexpr int kGtThreads = 32 * 9;
constexpr int kGtAccBufs = 4;
constexpr uint32_t kGtTmemCols = 256;
constexpr uint32_t kGtTmemSF = kGtAccBufs * 32;  // + 16 per ring slot
static_assert(kGtTmemSF + 16 * kGtStages <= kGtTmemCols, "scale columns exceed the allocation");
constexpr int kGtMaxChunks = kBuildGroupsMaxP + kBuildGroupsMaxP / kGtTok;
// tables of at most this many entries are grouped inside the kernel (one
// warp, shared memory) instead of by build_groups_kernel before it
constexpr int kGtLocalP = 64;

struct GtArgs {
  const GroupDesc* groups;
  const int* n_groups;
  const EntryDesc* entries;
  const uint8_t* xq;     // activation rows (rows, Kp/2)
  const uint8_t* xsc;    // (rows, Kp/32)
  float* y;
  int N, Kp;
  int* err;
  // in-kernel grouping (wp_tab non-null, P <= kGtLocalP): the caller's
  // pointer tables and their layout (mode 0: gate/up, 2·E entries per
  // activation row; mode 1: down, one entry per row), as build_groups_kernel
  // takes them; groups / n_groups / entries are then unused
  const uint8_t* const* wp_tab;
  const uint8_t* const* wsc_tab;
  int P, mode, E;
};

// Group the P <= 64 entries of the caller's tables with one warp, exactly as
// build_groups_kernel does (gemv.cu): entries with the same (weights, codes)
// pair form one group, groups in order of first appearance, entries of a
// group in table order; lane l handles entries l and l + 32.
__device__ void group_tables_warp(const GtArgs& p, GroupDesc* s_groups, EntryDesc* s_entries,
                                  int* s_cnt, int* s_ng) {
  const int lane = threadIdx.x & 31;
  const unsigned full = 0xffffffffu;
  const int P = p.P;
  const uint8_t* wa[2];
  const uint8_t* sa[2];
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const int z = lane + 32 * i;
    wa[i] = z < P ? p.wp_tab[z] : nullptr;
    sa[i] = z < P ? p.wsc_tab[z] : nullptr;
  }
  int lead[2] = {lane, lane + 32}, rank[2] = {0, 0};
  for (int j = 0; j < P; ++j) {
    const unsigned long long wj =
        __shfl_sync(full, reinterpret_cast<unsigned long long>(j < 32 ? wa[0] : wa[1]), j & 31);
    const unsigned long long sj =
        __shfl_sync(full, reinterpret_cast<unsigned long long>(j < 32 ? sa[0] : sa[1]), j & 31);
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const int z = lane + 32 * i;
      if (j < z && z < P && wj == reinterpret_cast<unsigned long long>(wa[i]) &&
          sj == reinterpret_cast<unsigned long long>(sa[i])) {
        if (lead[i] == z) lead[i] = j;
        ++rank[i];
      }
    }
  }
  const bool is0 = lane < P && lead[0] == lane;
  const bool is1 = lane + 32 < P && lead[1] == lane + 32;
  const unsigned b0 = __ballot_sync(full, is0), b1 = __ballot_sync(full, is1);
  const unsigned lt = (1u << lane) - 1u;
  const int g0 = __popc(b0 & lt), g1 = __popc(b0) + __popc(b1 & lt);
  const int ng = __popc(b0) + __popc(b1);
  // group of each entry: the index of its lead
  int g[2];
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const int v0 = __shfl_sync(full, g0, lead[i] & 31);
    const int v1 = __shfl_sync(full, g1, lead[i] & 31);
    g[i] = lead[i] < 32 ? v0 : v1;
  }
  s_cnt[lane] = 0;
  s_cnt[lane + 32] = 0;
  __syncwarp();
#pragma unroll
  for (int i = 0; i < 2; ++i)
    if (lane + 32 * i < P) atomicAdd(&s_cnt[g[i]], 1);
  __syncwarp();
  // exclusive scan of the counts: lane l owns groups 2l and 2l + 1
  const int c0 = s_cnt[2 * lane], c1 = s_cnt[2 * lane + 1];
  int inc = c0 + c1;
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) {
    const int u = __shfl_up_sync(full, inc, off);
    if (lane >= off) inc += u;
  }
  const int first0 = inc - c0 - c1;
  __syncwarp();
  s_cnt[2 * lane] = first0;
  s_cnt[2 * lane + 1] = first0 + c0;
  __syncwarp();
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const int z = lane + 32 * i;
    if (z >= P) continue;
    const int first = s_cnt[g[i]];
    if (lead[i] == z) {
      GroupDesc gd;
      gd.wp = wa[i];
      gd.wsc = sa[i];
      gd.first = first;
      gd.count = (g[i] + 1 < ng ? s_cnt[g[i] + 1] : P) - first;
      s_groups[g[i]] = gd;
    }
    EntryDesc ed;
    ed.pad = 0;
    if (p.mode == 0) {
      const int m = z / (2 * p.E), pair = z % (2 * p.E), proj = pair / p.E, e = pair % p.E;
      ed.act_row = m;
      ed.out_off = (long long)(m * p.E + e) * 2 * p.N + (long long)proj * p.N;
    } else {
      ed.act_row = z;
      ed.out_off = (long long)z * p.N;
    }
    s_entries[first + rank[i]] = ed;
  }
  if (lane == 0) *s_ng = ng;
  __syncwarp();
}

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, uint32_t src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(src_bytes)
               : "memory");
}
__device__ __forceinline__ void cp_async4(uint32_t dst, const void* src, uint32_t src_bytes) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(dst), "l"(src), "r"(src_bytes)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;" ::: "memory");
}
template <int kN>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(kN) : "memory");
}

__global__ void __launch_bounds__(kGtThreads, 1) grouped_tc_kernel(GtArgs p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* ring = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(ring + kGtStages * kGtStage);
  uint64_t* empty = full + kGtStages;
  uint64_t* acc_full = empty + kGtStages;
  uint64_t* acc_empty = acc_full + kGtAccBufs;
  uint64_t* drain = acc_empty + kGtAccBufs;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  __shared__ int s_chunk[kGtMaxChunks];  // (group << 8) | chunk index within the group
  __shared__ int s_nchunks;
  __shared__ GroupDesc s_groups[kGtLocalP];
  __shared__ EntryDesc s_entries[kGtLocalP];
  __shared__ int s_gcnt[kGtLocalP];
  __shared__ int s_ng;
  const bool local = p.wp_tab != nullptr;
  const GroupDesc* groups = local ? s_groups : p.groups;
  const EntryDesc* entries = local ? s_entries : p.entries;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nks = p.Kp / 256, nb = p.Kp / 32;
  const int n_tiles = (p.N + kGtRows - 1) / kGtRows;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kGtStages; ++s) {
      mbar_init(&full[s], kGtProducers);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < kGtAccBufs; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 4);
    }
    mbar_init(drain, 1);
    fence_mbar_init();
    cta_abort_init();
  }
  if (warp == 4) tmem_alloc(tmem_slot, kGtTmemCols);
  // the groups, entries and activation rows come from the kernels before
  grid_dep_wait();
  grid_dep_launch();
  // chunk table: every group's rows in chunks of 32, groups in order
  if (warp == 5) {
    if (local) group_tables_warp(p, s_groups, s_entries, s_gcnt, &s_ng);
    const int ng = local ? s_ng : *p.n_groups;
    int run = 0;
    for (int g0 = 0; g0 < ng; g0 += 32) {
      const int g = g0 + lane;
      const int nch = g < ng ? (groups[g].count + kGtTok - 1) / kGtTok : 0;
      int inc = nch;
#pragma unroll
      for (int off = 1; off < 32; off <<= 1) {
        const int v = __shfl_up_sync(0xffffffffu, inc, off);
        if (lane >= off) inc += v;
      }
      for (int c = 0; c < nch; ++c)
        if (run + inc - nch + c < kGtMaxChunks) s_chunk[run + inc - nch + c] = (g << 8) | c;
      run += __shfl_sync(0xffffffffu, inc, 31);
    }
    if (lane == 0) s_nchunks = min(run, kGtMaxChunks);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const int n_items = s_nchunks * n_tiles;

  if (warp < 4) {
    // ---- producers ------------------------------------------------------------
    // Every copy of a stage — weight and activation rows, both operands' E8M0
    // codes — is a cp.async, so no producer ever waits on a global load
    // inside the loop; an item's descriptors are loaded one item ahead.
    const int t = threadIdx.x;  // 0..127: weight row t of the tile for the codes
    const int j0 = t >> 3, j1 = 16 + (t >> 3);  // this thread's activation rows
    struct ItemDesc {
      const uint8_t* wp;
      const uint8_t* wsc;
      int tile, n_live, ar0, ar1, ar_sf;
    };
    auto load_item = [&](int item) {
      ItemDesc d;
      const int cv = s_chunk[item / n_tiles];
      d.tile = item % n_tiles;
      const GroupDesc gd = groups[cv >> 8];
      const int c0 = (cv & 255) * kGtTok;
      const int cnt = min(kGtTok, gd.count - c0);
      // the caller's weight pointers come from device tables: a tensor not
      // 16-byte (packed) / 8-byte (codes) aligned is reported (device error
      // 10) and read as zeros instead of faulting
      const bool w_ok = ((reinterpret_cast<uintptr_t>(gd.wp) & 15) == 0) &&
                        ((reinterpret_cast<uintptr_t>(gd.wsc) & 7) == 0);
      if (!w_ok && t == 0 && d.tile == 0) atomicCAS(p.err, 0, 10);
      d.wp = gd.wp;
      d.wsc = gd.wsc;
      d.n_live = w_ok ? p.N : 0;
      d.ar0 = j0 < cnt ? entries[gd.first + c0 + j0].act_row : -1;
      d.ar1 = j1 < cnt ? entries[gd.first + c0 + j1].act_row : -1;
      d.ar_sf = t < cnt ? entries[gd.first + c0 + t].act_row : -1;
      return d;
    };
    // the activation atoms' unused words (words 1-3 of each row line) stay zero
    for (int s = 0; s < kGtStages; ++s) {
      uint4* sfb = reinterpret_cast<uint4*>(ring + size_t(s) * kGtStage + kGtOffSFB);
      if (t < 64) sfb[t] = make_uint4(0u, 0u, 0u, 0u);
    }
    uint32_t it = 0, arrived = 0;
    bool ok = true;
    ItemDesc cur{};
    if (int(blockIdx.x) < n_items) cur = load_item(blockIdx.x);
    for (int item = blockIdx.x; item < n_items && ok; item += gridDim.x) {
      const ItemDesc d = cur;
      if (item + int(gridDim.x) < n_items) cur = load_item(item + gridDim.x);
      const int wrow = d.tile * kGtRows + t;
      for (int ks = 0; ks < nks; ++ks, ++it) {
        const int s = int(it % kGtStages);
        if (!mbar_wait(&empty[s], ((it / kGtStages) & 1) ^ 1, p.err, 1)) { ok = false; break; }
        uint8_t* st = ring + size_t(s) * kGtStage;
        const uint32_t sa = smem_u32(st), sb = smem_u32(st + kGtOffB);
        // A: 128 rows x 8 chunks; thread t copies chunk (t % 8) of rows t/8 + 16 i
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const int r = (t >> 3) + 16 * i, c = t & 7;
          const int n = d.tile * kGtRows + r;
          const bool live = n < d.n_live;
          // a dead row is zero-filled; its source address (not read) is the
          // host-checked, 16-byte aligned activation base
          const uint8_t* src = live ? d.wp + size_t(n) * (p.Kp / 2) + ks * 128 + c * 16 : p.xq;
          cp_async16(sa + r * 128 + ((c ^ (r & 7)) << 4), src, live ? 16u : 0u);
        }
        // B: 32 rows x 8 chunks; thread t copies chunk (t % 8) of rows t/8, 16 + t/8
        {
          const int c = t & 7;
          const uint8_t* s0 = p.xq + (d.ar0 >= 0 ? size_t(d.ar0) * (p.Kp / 2) + ks * 128 + c * 16 : 0);
          const uint8_t* s1 = p.xq + (d.ar1 >= 0 ? size_t(d.ar1) * (p.Kp / 2) + ks * 128 + c * 16 : 0);
          cp_async16(sb + j0 * 128 + ((c ^ (j0 & 7)) << 4), s0, d.ar0 >= 0 ? 16u : 0u);
          cp_async16(sb + j1 * 128 + ((c ^ (j1 & 7)) << 4), s1, d.ar1 >= 0 ? 16u : 0u);
        }
        // scale atoms: weight row t -> byte (t%32)*16 + (t/32)*4 + k%4 of atom
        // k/4; activation row t < 32 -> word 4t of each atom.  Dead rows get
        // code 0 (their operand bytes are zero, so the product is zero).
        {
          const uint32_t sfa = smem_u32(st + kGtOffSFA) + (t & 31) * 16 + (t >> 5) * 4;
          const bool wl = wrow < d.n_live;
          const uint8_t* wsrc = wl ? d.wsc + size_t(wrow) * nb + ks * 8 : p.xsc;
          cp_async4(sfa, wsrc, wl ? 4u : 0u);
          cp_async4(sfa + 512, wsrc + (wl ? 4 : 0), wl ? 4u : 0u);
          if (t < 32) {
            const uint32_t sfb = smem_u32(st + kGtOffSFB) + t * 16;
            const bool xl = d.ar_sf >= 0;
            const uint8_t* xsrc = xl ? p.xsc + size_t(d.ar_sf) * nb + ks * 8 : p.xsc;
            cp_async4(sfb, xsrc, xl ? 4u : 0u);
            cp_async4(sfb + 512, xsrc + (xl ? 4 : 0), xl ? 4u : 0u);
          }
        }
        cp_async_commit();
        if (it >= uint32_t(kGtLag)) {
          cp_async_wait<kGtLag>();
          fence_proxy_async_smem();
          mbar_arrive(&full[(it - kGtLag) % kGtStages]);
          arrived = it - kGtLag + 1;
        }
      }
    }
    // the last stages (and everything, on the error path)
    cp_async_wait<0>();
    fence_proxy_async_smem();
    for (uint32_t j = arrived; j < it; ++j) mbar_arrive(&full[j % kGtStages]);
  } else if (warp == 4) {
    // ---- MMA issue ------------------------------------------------------------
    if (elect_one()) {
      uint32_t it = 0, ti = 0;
      bool ok = true;
      const uint32_t idesc0 = make_idesc_mxf4(kGtRows, kGtTok, 0, 0);
      const uint32_t idesc2 = make_idesc_mxf4(kGtRows, kGtTok, 2, 2);
      for (int item = blockIdx.x; item < n_items && ok; item += gridDim.x, ++ti) {
        const uint32_t buf = ti % kGtAccBufs;
        if (!mbar_wait(&acc_empty[buf], ((ti / kGtAccBufs) & 1) ^ 1, p.err, 2)) { ok = false; break; }
        tc_fence_after();
        const uint32_t d = tmem + buf * 32;
        for (int ks = 0; ks < nks; ++ks, ++it) {
          const int s = int(it % kGtStages);
          if (!mbar_wait(&full[s], (it / kGtStages) & 1, p.err, 2)) { ok = false; break; }
          tc_fence_after();
          const uint32_t base = smem_u32(ring + size_t(s) * kGtStage);
          const uint32_t sfa = tmem + kGtTmemSF + 16 * s, sfb = sfa + 8;
#pragma unroll
          for (int c = 0; c < 2; ++c) {
            tmem_cp_sf(sfa + 4 * c, make_sdesc(base + kGtOffSFA + c * 512, 0, 128, kLayoutNone));
            tmem_cp_sf(sfb + 4 * c, make_sdesc(base + kGtOffSFB + c * 512, 0, 128, kLayoutNone));
          }
#pragma unroll
          for (int kb = 0; kb < 4; ++kb) {
            const int c = kb >> 1;
            const uint32_t byte = uint32_t(kb & 1) * 2;
            mma_mxf4(d, make_sdesc(base + kb * 32, 16, 1024, kLayoutSW128),
                     make_sdesc(base + kGtOffB + kb * 32, 16, 1024, kLayoutSW128),
                     byte ? idesc2 : idesc0, (ks | kb) != 0 ? 1u : 0u,
                     (sfa + 4 * c) | (byte << 30), (sfb + 4 * c) | (byte << 30));
          }
          tc_commit(&empty[s]);
        }
        if (ok) tc_commit(&acc_full[buf]);
      }
      if (!ok) drain_mma(drain);
    }
  } else {
    // ---- epilogue (warps 5-8, TMEM lane quadrant warp % 4) ---------------------
    const int quad = warp & 3;
    uint32_t ti = 0;
    for (int item = blockIdx.x; item < n_items; item += gridDim.x, ++ti) {
      const int cv = s_chunk[item / n_tiles];
      const int tile = item % n_tiles;
      const GroupDesc gd = groups[cv >> 8];
      const int c0 = (cv & 255) * kGtTok;
      const int cnt = min(kGtTok, gd.count - c0);
      const long long my_off = lane < cnt ? entries[gd.first + c0 + lane].out_off : 0;
      const uint32_t buf = ti % kGtAccBufs;
      if (!mbar_wait(&acc_full[buf], (ti / kGtAccBufs) & 1, p.err, 3)) break;
      tc_fence_after();
      uint32_t r[32];
      tmem_ld_32x32b_x32(tmem + (uint32_t(quad * 32) << 16) + buf * 32, r);
      tmem_ld_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[buf]);
      const int n = tile * kGtRows + quad * 32 + lane;
#pragma unroll
      for (int j = 0; j < kGtTok; ++j) {
        if (j < cnt) {  // warp-uniform
          const long long off = __shfl_sync(0xffffffffu, my_off, j);
          if (n < p.N) p.y[off + n] = __uint_as_float(r[j]);
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 4) {
    tc_fence_after();
    tmem_dealloc(tmem, kGtTmemCols);
  }
}

constexpr size_t grouped_tc_smem() {
  return 1024 + size_t(kGtStages) * kGtStage + 8 * (2 * kGtStages + 2 * kGtAccBufs + 1) + 16;
}
static_assert(grouped_tc_smem() + kGtMaxChunks * 4 + 64 <= 232448, "shared memory of a CTA");

}  // namespace

bool grouped_tc_supported(int N, int Kp) { return Kp % 256 == 0 && Kp >= 256 && N > 0; }
int grouped_tc_local_max() { return kGtLocalP; }

cudaError_t launch_grouped_tc(const GroupDesc* groups, const int* n_groups, int max_items,
                              const EntryDesc* entries, const uint8_t* xq, const uint8_t* xsc,
                              float* y, int N, int Kp, int* err, cudaStream_t stream, bool pdl,
                              const GtTables* tables) {
  if (!grouped_tc_supported(N, Kp)) return cudaErrorNotSupported;
  cudaError_t e = ensure_dynamic_smem(reinterpret_cast<const void*>(grouped_tc_kernel),
                                      grouped_tc_smem());
  if (e != cudaSuccess) return e;
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int grid = max_items < sms ? (max_items > 0 ? max_items : 1) : sms;
  GtArgs a{};
  a.groups = groups; a.n_groups = n_groups; a.entries = entries;
  a.xq = xq; a.xsc = xsc; a.y = y; a.N = N; a.Kp = Kp; a.err = err;
  a.wp_tab = tables ? tables->wp_tab : nullptr;
  a.wsc_tab = tables ? tables->wsc_tab : nullptr;
  a.P = tables ? tables->P : 0;
  a.mode = tables ? tables->mode : 0;
  a.E = tables ? tables->E : 0;
  if (tables && (tables->P <= 0 || tables->P > kGtLocalP)) return cudaErrorInvalidValue;
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kGtThreads);
  cfg.dynamicSmemBytes = grouped_tc_smem();
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, grouped_tc_kernel, a);
}

}  // namespace mfi
