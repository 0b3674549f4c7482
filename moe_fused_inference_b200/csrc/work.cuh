// work.cuh — work-list types and launch entry points shared by the kernels
// and the C ABI (capi.cu).  Host-visible only through include/moe_fp4.h.
#pragma once
#include <cstdint>
#include <cuda_runtime.h>
#include <cuda_bf16.h>

namespace mfi {

// One weight matrix and the activation rows that multiply it.
struct GroupDesc {
  const uint8_t* wp;   // (N, Kp/2) packed nibbles
  const uint8_t* wsc;  // (N, Kp/32) E8M0 codes
  int first;           // index of the group's first EntryDesc
  int count;           // number of entries
};

// One activation row of a group and where its output row goes.
struct EntryDesc {
  int act_row;         // row of the packed activations
  int pad;
  long long out_off;   // element offset of the output row (column n adds n)
};

struct QuantArgs {
  const void* x;
  long ld_x;          // row stride of x in elements
  int dtype;          // DType (mx_common.cuh)
  int half_rt;        // 1: round each element through fp16 first (mxfp4_linear semantics)
  uint8_t* xq;        // (M, Kp/2)
  uint8_t* xsc;       // (M, Kp/32)
  int M, K, Kp;
};

// Up to 32 tokens routed to one expert (one MMA N-tile of the decode path).
struct ChunkDesc {
  int expert;
  int count;
  int row0;   // first row of the chunk in the per-expert activation regions
  int pad;
};

// ---- expert parallelism over peer memory (ep.cu, route.cu) -----------------
// Per-rank flag area (32-bit words), in memory every peer maps:
constexpr int kEpMaxRanks = 64;
constexpr int kFlagDispatch = 0;    // [s]: call id of the last dispatch received from rank s
constexpr int kFlagReturn = 64;     // [d]: call id of the last return received from rank d
constexpr int kFlagEpoch = 128;     // calls completed by this rank
constexpr int kFlagCounts = 160;    // [d]: rows sent to rank d in this call (zeroed per call)
constexpr int kFlagDone = 224;      // completion counters of this call's launches (zeroed per call)
constexpr int kFlagWords = 256;
constexpr int kFlagZeroFirst = kFlagCounts;  // per-call zeroed range [kFlagCounts, kFlagWords)

// Peer pointers of one exchange, as seen from this rank (device copy).
struct EpTable {
  uint8_t* recv[kEpMaxRanks];   // rank d's receive buffer [n][C+1][row bytes]
  float* ret[kEpMaxRanks];      // rank d's return buffer [n][C+1][hidden]
  unsigned* flags[kEpMaxRanks]; // rank d's flag area
};

struct EpDispatch {            // route_cluster_kernel: send each routed token to its ranks
  const EpTable* table;
  unsigned* flags;             // this rank's flag area
  int* pack_pos;               // (T, n): row of token t in its block at rank d, or -1
  int rank, n, C, el;          // rank, ranks, capacity, experts per rank
  int T;                       // real tokens (clusters past T only join the completion)
};

struct RouteArgs {
  const void* x;       // bf16 (T, H): quantised inside the kernel into xq/xsc
  uint8_t* xq;         // (T, H/2)
  uint8_t* xsc;        // (T, H/32)
  const uint8_t* wr;   // (E, H/2)
  const uint8_t* sr;   // (E, H/32)
  int T, H, E, k;
  float* logits;       // (T, E) or null
  int* topi;           // (T, k)
  float* topw;         // (T, k)
  unsigned* done;      // completion counter, zero before the launch
  const uint8_t* gate_wp; const uint8_t* gate_sc;
  const uint8_t* up_wp; const uint8_t* up_sc;
  const uint8_t* down_wp; const uint8_t* down_sc;
  int Mi;
  GroupDesc* g_gu; EntryDesc* e_gu; int* n_gu;   // 2 groups per active expert
  GroupDesc* g_dn; EntryDesc* e_dn; int* n_dn;   // 1 group per active expert
  int* n_active;
  // tensor-core decode path: 32-token chunks per expert.  Expert e owns rows
  // [e*T_pad, (e+1)*T_pad) of xp / perm (T_pad = ceil32(T)); a token's row in
  // its expert's region comes from the atomic cursor[e].
  ChunkDesc* chunks;   // [max_chunks]
  int* n_chunks;
  int* perm;           // [E * T_pad]: row -> pair index (token * k + slot), -1 padding
  int* cursor;         // [E], zero before the launch; reset by the kernel
  uint8_t* xp;         // [E * T_pad][H/2] quantised rows per expert region
  uint8_t* xp_atoms;   // [E * T_pad / 32][H/128][512] their scale atoms
  int T_pad;
  int* err;            // device error flag (bounded waits)
  // speculative L2 prefetch of the first pf_bytes at pf_base (expert weights
  // in the order the next kernel reads them), issued once the inputs are in
  const uint8_t* pf_base;
  unsigned long long pf_bytes;
  EpDispatch ep;       // ep.table == null: no expert-parallel dispatch
  const float* logit_bias;  // [E] added to the logits before top-k, or null
  // RMSNorm of each token row before quantisation (route_common.cuh), or null
  const __nv_bfloat16* norm_w;  // [H] bf16 weight
  float norm_eps;
  // prefill placement: slot_pos[t*k + j] = the pair's position among the
  // tokens of its expert (cursor claim, no row copy)
  int* slot_pos;
  bool batch;          // prefer the one-token-per-warp batch router (many tokens)
  // scratch of the tensor-core router (route_tc.cu): ceil(T/128)*128 x H
  // bytes of int8 token rows and E x H bytes of int8 router rows; null: that
  // router is not used
  uint8_t* x8;
  uint8_t* r8;
};

constexpr int kRouteMaxE = 256;
constexpr int kRouteMaxPairs = 4096;
constexpr int kBuildGroupsMaxP = 4096;

cudaError_t launch_quant_rows(const QuantArgs& a, cudaStream_t stream);
// Decode-sized dense GEMM on the tensor cores (lin_tc.cu): M <= 32
// activation rows, Kp a multiple of 512 up to 4096; launch_dense_gemv uses it
// when it applies.
bool lin_tc_supported(const void* xq, const uint8_t* xsc, const void* wp, const uint8_t* wsc, int M,
                      int Kp);
cudaError_t launch_lin_tc(const uint8_t* xq, const uint8_t* xsc, const uint8_t* wp,
                          const uint8_t* wsc, float* y, long long ldy, int M, int N, int Kp,
                          cudaStream_t stream);

// Prefill router on the tensor cores (E = 128, H a multiple of 128, <= 2048,
// a.x8 set); launch_route picks it when it applies.
bool route_tc_applies(const RouteArgs& a);
cudaError_t launch_route_tc(const RouteArgs& a, cudaStream_t stream);

cudaError_t launch_swiglu_quant(const float* gu, long ld_gu, const int* rows, int n_rows,
                                const int* n_rows_dev, uint8_t* hq, uint8_t* hsc, int K, int Kp,
                                cudaStream_t stream, bool pdl = false);
size_t gemv_smem_bytes(int Kp);
cudaError_t launch_grouped_gemv(const GroupDesc* groups, const int* n_groups_dev, int n_groups_host,
                                const EntryDesc* entries, const uint8_t* xq, const uint8_t* xsc,
                                float* y, int N, int Kp, int max_ctas, cudaStream_t stream);
cudaError_t launch_dense_gemv(const uint8_t* xq, const uint8_t* xsc, const uint8_t* wp,
                              const uint8_t* wsc, float* y, long long ldy, int M, int N, int Kp,
                              cudaStream_t stream);
// The grouped tensor-core form of launch_grouped_gemv (grouped_tc.cu): Kp a
// multiple of 256, xq rows 16-byte and xsc rows 8-byte aligned; max_items
// bounds (groups' 32-row chunks) x (128-row tiles) for the grid size.
bool grouped_tc_supported(int N, int Kp);
// The caller's pointer tables, for a grouped_tc launch that groups them
// itself (P <= grouped_tc_local_max()); groups / n_groups / entries are then
// not read.
struct GtTables {
  const uint8_t* const* wp_tab;
  const uint8_t* const* wsc_tab;
  int P, mode, E;
};
int grouped_tc_local_max();
cudaError_t launch_grouped_tc(const GroupDesc* groups, const int* n_groups, int max_items,
                              const EntryDesc* entries, const uint8_t* xq, const uint8_t* xsc,
                              float* y, int N, int Kp, int* err, cudaStream_t stream,
                              bool pdl = false, const GtTables* tables = nullptr);
cudaError_t launch_build_groups(const uint8_t* const* wp_tab, const uint8_t* const* wsc_tab, int P,
                                int mode, int E, int N, GroupDesc* groups, int* n_groups,
                                EntryDesc* entries, cudaStream_t stream, bool pdl = false);
// pdl (the three launchers above): programmatic dependent launch.  Each of
// these kernels waits for the kernel before it before it reads or writes
// global memory, so only its launch and prologue overlap that kernel's tail.

// clear/n_clear: counters zeroed by the launch once the previous kernel is
// complete (the fused layer's per-call counters), or null
// Prefill combine: out[m] = sum over slots e (ascending) of w[m][e] * y[m][e],
// y rows in bf16, products and sums in fp32 as in combine_kernel.
cudaError_t launch_combine_bf16(const __nv_bfloat16* yd, const float* w, int k, float* out, int M,
                                int N, cudaStream_t stream, bool pdl);
cudaError_t launch_combine(const float* yd, long ystride, const float* w, int E, int E_sum,
                           float* out, int M, int N, cudaStream_t stream, bool pdl = false,
                           unsigned* clear = nullptr, int n_clear = 0);
cudaError_t launch_route(const RouteArgs& a, cudaStream_t stream);

// tcgen05 MXFP4 GEMM (tc_gemm.cu)
size_t tc_gemm_smem_bytes();
bool tc_gemm_supported(const void* a, const void* b, int Kp);
size_t sf_atoms_bytes(int R, int Kp, int row_align);
cudaError_t launch_sf_atoms(const uint8_t* src, long long src_ld, int R, int Kp, int row_align,
                            uint8_t* dst, cudaStream_t stream);
cudaError_t launch_tc_gemm(const uint8_t* a, const uint8_t* sfa_atoms, const uint8_t* b,
                           const uint8_t* sfb_atoms, float* y, long long ldy, int M, int N, int Kp,
                           int* err, cudaStream_t stream);

// Decode expert GEMMs on tensor cores (moe_tc.cu): gate/up and down in one
// persistent launch.
struct MoeTcLaunch {
  int E, H, Mi, max_chunks, grid;
  const uint8_t* prepared;           // weight blocks from launch_moe_prepare
  const int* counts;                            // tokens per expert (route cursors)
  const int* perm;
  int rows;                                     // E * T_pad rows in xp / hp / perm
  const uint8_t* xp; const uint8_t* xp_atoms;   // per-expert token rows (route.cu)
  uint8_t* hp; uint8_t* hp_atoms;               // requantised h (gate/up output)
  float* yd;                                    // per-pair down output
  int* err;
  bool pdl;                                     // programmatic dependent launch
  size_t pf_bytes;                              // speculative L2 prefetch of weights
  int* queue;                                   // work-item counter, zeroed before the launch
  unsigned* ready;                              // [max_chunks], zeroed before the launch
};
size_t moe_prepared_bytes(int E, int H, int Mi);
cudaError_t launch_moe_prepare(const uint8_t* gate_wp, const uint8_t* gate_sc,
                               const uint8_t* up_wp, const uint8_t* up_sc,
                               const uint8_t* down_wp, const uint8_t* down_sc, int E, int H, int Mi,
                               uint8_t* prepared, cudaStream_t stream);
cudaError_t launch_moe_tc(const MoeTcLaunch& L, cudaStream_t stream);

// Expert parallelism and pre-routed rows (ep.cu).
int ep_row_bytes(int H, int k);
cudaError_t launch_ep_pack(const uint8_t* xq, const uint8_t* xsc, const int* topi,
                           const float* topw, int T, int H, int k, int n_ranks, int e_local, int C,
                           int* counts, uint8_t* send, int* pack_pos, cudaStream_t stream);
cudaError_t launch_ep_mask_recv(int n_ranks, int C, int H, int k, uint8_t* recv, int* err,
                                cudaStream_t stream);
cudaError_t launch_ep_unpack(const float* ret, const int* pack_pos, int T, int n_ranks, int C,
                             int H, float* out, cudaStream_t stream);
cudaError_t launch_scatter_sel(const uint8_t* xq, long long xq_ld, const uint8_t* xsc,
                               long long xsc_ld, const int* sel, long long sel_ld, int R, int k,
                               int H, int E, int T_pad, int* cursor, int* perm, uint8_t* xp,
                               uint8_t* xp_atoms, int* status, cudaStream_t stream);
// combine_sel on bf16 rows (the prefill kernel's y).
cudaError_t launch_combine_sel_bf16(const __nv_bfloat16* yd, const int* sel, long long sel_ld,
                                    const float* w, long long w_ld, int R, int k, int E, int H,
                                    float* out, long long out_ld, cudaStream_t stream);
cudaError_t launch_combine_sel(const float* yd, const int* sel, long long sel_ld, const float* w,
                               long long w_ld, int R, int k, int E, int H, float* out,
                               long long out_ld, cudaStream_t stream);

// Prefill-sized expert GEMMs (moe_prefill.cu).
constexpr int kPrefillMaxPairs = 262144;   // T * top_k per call
struct PrefillLaunch {
  int E, H, Mi, top_k, grid;
  const uint8_t* prepared;       // weight blocks from launch_moe_prepare
  const int* counts;             // tokens per expert
  const int* perm;               // row -> pair
  int rows;                      // rows of xp / hp (prefill_rows)
  const uint8_t* xp; const uint8_t* xa;   // token rows and their 128-row scale atoms
  uint8_t* hp; uint8_t* ha;               // requantised h rows and atoms
  __nv_bfloat16* yd;             // (pairs, H) per-(token, slot) down rows, bf16
  int* err; int* queue; unsigned* gu_done; unsigned* ready;
  bool pdl;
};
size_t prefill_rows(int pairs, int E);
// Rows t < T with expert lists topi[t * sel_ld + j] (entries outside [0, E)
// skipped) into the per-expert regions; xq / xsc rows at strides xq_ld /
// xsc_ld bytes.
cudaError_t launch_prefill_scatter(const uint8_t* xq, long long xq_ld, const uint8_t* xsc,
                                   long long xsc_ld, const int* topi, long long sel_ld,
                                   const int* slot_pos, const int* counts, int T, int E, int k,
                                   int H, int* perm, uint8_t* xp, uint8_t* xa,
                                   cudaStream_t stream);
// Per-expert counts and slot positions of pre-routed rows (counts zeroed).
cudaError_t launch_prefill_count_sel(const int* sel, long long sel_ld, int R, int k, int E,
                                     int* counts, int* slot_pos, int* status,
                                     cudaStream_t stream);
cudaError_t launch_moe_prefill(const PrefillLaunch& L, cudaStream_t stream);

// Peer-memory exchange (ep.cu).
cudaError_t launch_ep_scatter_wait(const EpTable* table, unsigned* flags, uint8_t* recv, int rank,
                                   int n, int C, int H, int k, int E, int T_pad, int* cursor,
                                   int* perm, uint8_t* xp, uint8_t* xp_atoms, int* err,
                                   cudaStream_t stream);
cudaError_t launch_ep_combine_return(const EpTable* table, unsigned* flags, const float* yd,
                                     const uint8_t* recv, int rank, int n, int C, int H, int k,
                                     int E, int* ws_counters, int n_counters, int* err,
                                     cudaStream_t stream);
cudaError_t launch_ep_unpack_wait(unsigned* flags, const float* ret, const int* pack_pos, int T,
                                  int n, int C, int H, float* out, int* err, cudaStream_t stream);

// Device-wide error flag written by kernels whose bounded waits time out.
int* device_error_flag();

// Record a message for mfi_last_error() on this host thread; returns code.
int set_last_error(int code, const char* msg);

}  // namespace mfi
