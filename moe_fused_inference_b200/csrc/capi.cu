// capi.cu — the extern "C" surface of libmoe_fp4.so (declared in include/moe_fp4.h).
//
// Each entry point validates its arguments (messages follow the reference
// binding's TORCH_CHECK wording, src/ext/mxfp4_decode_binding.cpp and
// src/ext/mxfp4_binding.cpp), carves its scratch out of the caller's
// workspace, launches on the caller's stream and checks the launch — the
// reference launches never call cudaGetLastError.
#include <cstdio>
#include <cstring>
#include <string>

#include "../../include/moe_fp4.h"
#include "mx_common.cuh"
#include "work.cuh"

namespace {

thread_local std::string g_err;

int fail(int code, const std::string& msg) {
  g_err = msg;
  return code;
}

int cuda_status(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return MFI_OK;
  return fail(MFI_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
}

// The library links the shared CUDA runtime, so it shares the caller's current
// device; the stream must belong to that device (as with any torch extension).
inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }
inline int ceil32(int k) { return (k + 31) / 32 * 32; }

// Bump allocator over a caller-owned workspace (256-byte aligned pieces).
struct Carve {
  uint8_t* base;
  size_t used = 0;
  explicit Carve(void* p) : base(static_cast<uint8_t*>(p)) {}
  template <class T>
  T* take(size_t count) {
    used = (used + 255) & ~size_t(255);
    T* p = reinterpret_cast<T*>(base ? base + used : nullptr);
    used += count * sizeof(T);
    return p;
  }
};

constexpr int kGemvMaxCtas = 148 * 4;
// Rows of activations from which the tcgen05 tensor-core GEMM replaces the
// CUDA-core GEMV (one 128-row MMA tile is then at least half used).
constexpr int kTcMinM = 64;

bool bad_ptr(const void* p) { return p == nullptr; }

// Speculative L2 prefetch of expert weights by the tensor-core expert launches
// (issued while the kernel before them runs).  Only when routing is dense
// enough that nearly every expert is active (pairs >= 2 x experts), so the
// blocks fetched in storage order are the ones the launch reads first.
#ifndef MFI_PF_GATEUP_MB
#define MFI_PF_GATEUP_MB 64
#endif
#ifndef MFI_PF_DOWN_MB
#define MFI_PF_DOWN_MB 32
#endif
size_t prefetch_bytes(long long pairs, int E, bool gate_up) {
  if (pairs < 2LL * E) return 0;
  return size_t(gate_up ? MFI_PF_GATEUP_MB : MFI_PF_DOWN_MB) << 20;
}

}  // namespace

namespace mfi {
int set_last_error(int code, const char* msg) { return fail(code, msg); }
}  // namespace mfi

extern "C" {

const char* mfi_last_error(void) { return g_err.c_str(); }

int mfi_version(void) { return 3; }  // 3: mfi_moe_weights gained norm_weight / norm_eps

// ---------------------------------------------------------------------------
int mfi_quantize_rows(const void* x, int dtype, long long ld_x, int half_roundtrip, uint8_t* xq,
                      uint8_t* xsc, int M, int K, int Kp, void* stream) {
  if (M < 0 || K < 0) return fail(MFI_ERR_ARG, "M and K must be non-negative");
  if (Kp < K || Kp % 32 != 0) return fail(MFI_ERR_ARG, "Kp must be a multiple of 32 and >= K");
  if (dtype != MFI_F32 && dtype != MFI_F16 && dtype != MFI_BF16)
    return fail(MFI_ERR_ARG, "dtype must be MFI_F32, MFI_F16 or MFI_BF16");
  if (M == 0 || K == 0) return MFI_OK;
  if (bad_ptr(x) || bad_ptr(xq) || bad_ptr(xsc)) return fail(MFI_ERR_ARG, "null pointer");
  if (ld_x < K) return fail(MFI_ERR_ARG, "ld_x must be >= K");
  mfi::QuantArgs a{x, long(ld_x), dtype, half_roundtrip ? 1 : 0, xq, xsc, M, K, Kp};
  return cuda_status(mfi::launch_quant_rows(a, as_stream(stream)), "quantize_rows launch");
}

int mfi_prequant(const void* x_bf16, uint8_t* xq, uint8_t* xsc, int M, int K, int Kp,
                 void* stream) {
  return mfi_quantize_rows(x_bf16, MFI_BF16, K, 0, xq, xsc, M, K, Kp, stream);
}

// ---------------------------------------------------------------------------
size_t mfi_lin_pq_workspace_bytes(int M, int N, int Kp) {
  if (M < kTcMinM) return 0;
  Carve c(nullptr);
  c.take<uint8_t>(mfi::sf_atoms_bytes(M, Kp, 128));
  c.take<uint8_t>(mfi::sf_atoms_bytes(N, Kp, 256));
  return c.used + 256;
}

// Tensor-core GEMM of pre-quantised operands: scale factors re-laid out into
// atoms in the workspace, then one tcgen05 kernel.
static int tc_linear(const uint8_t* xq, const uint8_t* xsc, const uint8_t* wp, const uint8_t* wsc,
                     float* y, int M, int N, int Kp, Carve& c, cudaStream_t s) {
  uint8_t* sfa = c.take<uint8_t>(mfi::sf_atoms_bytes(M, Kp, 128));
  uint8_t* sfb = c.take<uint8_t>(mfi::sf_atoms_bytes(N, Kp, 256));
  int st = cuda_status(mfi::launch_sf_atoms(xsc, Kp / 32, M, Kp, 128, sfa, s), "sf atoms (A)");
  if (st != MFI_OK) return st;
  st = cuda_status(mfi::launch_sf_atoms(wsc, Kp / 32, N, Kp, 256, sfb, s), "sf atoms (B)");
  if (st != MFI_OK) return st;
  return cuda_status(mfi::launch_tc_gemm(xq, sfa, wp, sfb, y, N, M, N, Kp,
                                         mfi::device_error_flag(), s),
                     "tcgen05 gemm launch");
}

int mfi_lin_pq(const uint8_t* xq, const uint8_t* xsc, const uint8_t* wp, const uint8_t* wsc,
               float* y, int M, int N, int K, int Kp, void* workspace, size_t workspace_bytes,
               void* stream) {
  if (M < 0 || N < 0 || K < 0) return fail(MFI_ERR_ARG, "M, N, K must be non-negative");
  if (Kp <= 0 || Kp % 32 != 0) return fail(MFI_ERR_ARG, "Kp must be a positive multiple of 32");
  if (M == 0 || N == 0) return MFI_OK;
  if (bad_ptr(xq) || bad_ptr(xsc) || bad_ptr(wp) || bad_ptr(wsc) || bad_ptr(y))
    return fail(MFI_ERR_ARG, "null pointer");
  cudaStream_t s = as_stream(stream);
  if (M >= kTcMinM && mfi::tc_gemm_supported(xq, wp, Kp)) {
    if (bad_ptr(workspace) || workspace_bytes < mfi_lin_pq_workspace_bytes(M, N, Kp))
      return fail(MFI_ERR_WORKSPACE, "workspace too small for lin_pq");
    Carve c(workspace);
    return tc_linear(xq, xsc, wp, wsc, y, M, N, Kp, c, s);
  }
  return cuda_status(mfi::launch_dense_gemv(xq, xsc, wp, wsc, y, N, M, N, Kp, s), "lin_pq launch");
}

size_t mfi_linear_workspace_bytes(int M, int N, int Kp) {
  Carve c(nullptr);
  c.take<uint8_t>(size_t(M) * (Kp / 2));
  c.take<uint8_t>(size_t(M) * (Kp / 32));
  return c.used + mfi_lin_pq_workspace_bytes(M, N, Kp) + 256;
}

int mfi_mxfp4_linear(const void* x, int dtype, int ld_x, const uint8_t* wp, const uint8_t* wsc,
                     float* y, int M, int N, int Kp, void* workspace, size_t workspace_bytes,
                     void* stream) {
  if (M < 0 || N < 0 || ld_x <= 0) return fail(MFI_ERR_ARG, "M, N must be >= 0 and K > 0");
  if (Kp <= 0 || Kp % 32 != 0) return fail(MFI_ERR_ARG, "Kp must be a positive multiple of 32");
  if (M == 0 || N == 0) return MFI_OK;
  if (bad_ptr(x) || bad_ptr(wp) || bad_ptr(wsc) || bad_ptr(y) || bad_ptr(workspace))
    return fail(MFI_ERR_ARG, "null pointer");
  if (workspace_bytes < mfi_linear_workspace_bytes(M, N, Kp))
    return fail(MFI_ERR_WORKSPACE, "workspace too small for mxfp4_linear");
  Carve c(workspace);
  uint8_t* xq = c.take<uint8_t>(size_t(M) * (Kp / 2));
  uint8_t* xsc = c.take<uint8_t>(size_t(M) * (Kp / 32));
  // the reference kernel reads x columns [0, min(K, Kp)) and treats the rest as zero
  const int k_eff = ld_x < Kp ? ld_x : Kp;
  const int half_rt = dtype == MFI_F16 ? 0 : 1;
  int st = mfi_quantize_rows(x, dtype, ld_x, half_rt, xq, xsc, M, k_eff, Kp, stream);
  if (st != MFI_OK) return st;
  cudaStream_t s = as_stream(stream);
  if (M >= kTcMinM && mfi::tc_gemm_supported(xq, wp, Kp))
    return tc_linear(xq, xsc, wp, wsc, y, M, N, Kp, c, s);
  return cuda_status(mfi::launch_dense_gemv(xq, xsc, wp, wsc, y, N, M, N, Kp, s),
                     "mxfp4_linear gemm launch");
}

int mfi_device_error(int clear) {
  int v = 0;
  if (cudaMemcpy(&v, mfi::device_error_flag(), sizeof(int), cudaMemcpyDeviceToHost) != cudaSuccess)
    return -1;
  if (clear && v) {
    const int z = 0;
    cudaMemcpy(mfi::device_error_flag(), &z, sizeof(int), cudaMemcpyHostToDevice);
  }
  return v;
}

// ---------------------------------------------------------------------------
namespace {
// The grouped GEMM of the drop-in operators over the caller's pointer
// tables: the tcgen05 kernel when K tiles by 256 and the activations are
// aligned for 16-byte copies (every Qwen3-MoE expert shape), else the
// CUDA-core GEMV.  The tables are grouped by build_groups_kernel first,
// except for the tensor-core kernel at decode sizes (at most
// grouped_tc_local_max() entries), which groups them itself.
int grouped_launch(const uint8_t* const* wp_tab, const uint8_t* const* wsc_tab, int mode, int E,
                   mfi::GroupDesc* groups, int* ng, int P, mfi::EntryDesc* entries,
                   const uint8_t* xq, const uint8_t* xsc, float* y, int N, int Kp, cudaStream_t s,
                   const char* what) {
  const std::string w = std::string(what) + " grouped GEMM launch";
  const bool tc = mfi::grouped_tc_supported(N, Kp) && (reinterpret_cast<uintptr_t>(xq) & 15) == 0 &&
                  (reinterpret_cast<uintptr_t>(xsc) & 7) == 0;
  const long long items = (long long)P * ((N + 127) / 128);
  const int max_items = items > (1 << 30) ? (1 << 30) : int(items);
  if (tc && P <= mfi::grouped_tc_local_max()) {
    const mfi::GtTables tab{wp_tab, wsc_tab, P, mode, E};
    return cuda_status(mfi::launch_grouped_tc(groups, ng, max_items, entries, xq, xsc, y, N, Kp,
                                              mfi::device_error_flag(), s, true, &tab),
                       w.c_str());
  }
  const std::string wg = std::string(what) + " grouping launch";
  int st = cuda_status(mfi::launch_build_groups(wp_tab, wsc_tab, P, mode, E, N, groups, ng, entries,
                                                s, true),
                       wg.c_str());
  if (st != MFI_OK) return st;
  if (tc)
    return cuda_status(mfi::launch_grouped_tc(groups, ng, max_items, entries, xq, xsc, y, N, Kp,
                                              mfi::device_error_flag(), s, true),
                       w.c_str());
  return cuda_status(mfi::launch_grouped_gemv(groups, ng, P, entries, xq, xsc, y, N, Kp,
                                              kGemvMaxCtas, s),
                     w.c_str());
}
}  // namespace

size_t mfi_moe_gateup_workspace_bytes(int E, int M) {
  const size_t P = size_t(2) * E * M;
  Carve c(nullptr);
  c.take<int>(1);
  c.take<mfi::GroupDesc>(P);
  c.take<mfi::EntryDesc>(P);
  return c.used + 256;
}

int mfi_moe_gateup(const uint8_t* xq, const uint8_t* xsc, const uint8_t* const* wp_tab,
                   const uint8_t* const* wsc_tab, float* gu, int E, int M, int N, int K, int Kp,
                   void* workspace, size_t workspace_bytes, void* stream) {
  (void)K;
  if (E <= 0 || M <= 0 || N <= 0) return fail(MFI_ERR_ARG, "E, M, N must be positive");
  if (Kp <= 0 || Kp % 32 != 0) return fail(MFI_ERR_ARG, "Kp must be a positive multiple of 32");
  const long long P = 2LL * E * M;
  if (P > mfi::kBuildGroupsMaxP) return fail(MFI_ERR_ARG, "pointer table longer than 4096 entries");
  if (bad_ptr(xq) || bad_ptr(xsc) || bad_ptr(wp_tab) || bad_ptr(wsc_tab) || bad_ptr(gu) ||
      bad_ptr(workspace))
    return fail(MFI_ERR_ARG, "null pointer");
  if (workspace_bytes < mfi_moe_gateup_workspace_bytes(E, M))
    return fail(MFI_ERR_WORKSPACE, "workspace too small for moe_gateup");
  Carve c(workspace);
  int* ng = c.take<int>(1);
  auto* groups = c.take<mfi::GroupDesc>(P);
  auto* entries = c.take<mfi::EntryDesc>(P);
  cudaStream_t s = as_stream(stream);
  return grouped_launch(wp_tab, wsc_tab, 0, E, groups, ng, int(P), entries, xq, xsc, gu, N, Kp, s,
                        "moe_gateup");
}

size_t mfi_moe_down_workspace_bytes(int E, int M, int K) {
  const size_t P = size_t(E) * M;
  const int Kp = ceil32(K);
  Carve c(nullptr);
  c.take<int>(1);
  c.take<mfi::GroupDesc>(P);
  c.take<mfi::EntryDesc>(P);
  c.take<uint8_t>(P * (Kp / 2));
  c.take<uint8_t>(P * (Kp / 32));
  return c.used + 256;
}

int mfi_moe_down(const float* gu, const uint8_t* const* wp_tab, const uint8_t* const* wsc_tab,
                 float* yd, int E, int M, int N, int K, int Kp, void* workspace,
                 size_t workspace_bytes, void* stream) {
  if (E <= 0 || M <= 0 || N <= 0 || K <= 0) return fail(MFI_ERR_ARG, "E, M, N, K must be positive");
  if (Kp != ceil32(K)) return fail(MFI_ERR_ARG, "Kp must equal ceil32(K)");
  const long long P = 1LL * E * M;
  if (P > mfi::kBuildGroupsMaxP) return fail(MFI_ERR_ARG, "pointer table longer than 4096 entries");
  if (bad_ptr(gu) || bad_ptr(wp_tab) || bad_ptr(wsc_tab) || bad_ptr(yd) || bad_ptr(workspace))
    return fail(MFI_ERR_ARG, "null pointer");
  if (workspace_bytes < mfi_moe_down_workspace_bytes(E, M, K))
    return fail(MFI_ERR_WORKSPACE, "workspace too small for moe_down");
  Carve c(workspace);
  int* ng = c.take<int>(1);
  auto* groups = c.take<mfi::GroupDesc>(P);
  auto* entries = c.take<mfi::EntryDesc>(P);
  uint8_t* hq = c.take<uint8_t>(P * (Kp / 2));
  uint8_t* hsc = c.take<uint8_t>(P * (Kp / 32));
  cudaStream_t s = as_stream(stream);
  int st = cuda_status(mfi::launch_swiglu_quant(gu, 2L * K, nullptr, int(P), nullptr, hq, hsc, K,
                                                Kp, s, true),
                       "moe_down swiglu launch");
  if (st != MFI_OK) return st;
  return grouped_launch(wp_tab, wsc_tab, 1, E, groups, ng, int(P), entries, hq, hsc, yd, N, Kp, s,
                        "moe_down");
}

int mfi_moe_combine(const float* yd, int ystride, const float* w, int E, float* out, int M, int N,
                    void* stream) {
  if (E <= 0 || M < 0 || N < 0) return fail(MFI_ERR_ARG, "E must be positive, M and N non-negative");
  if (ystride < N) return fail(MFI_ERR_ARG, "ystride must be >= N");
  if (M == 0 || N == 0) return MFI_OK;
  if (bad_ptr(yd) || bad_ptr(w) || bad_ptr(out)) return fail(MFI_ERR_ARG, "null pointer");
  const int e_sum = E < 8 ? E : 8;
  return cuda_status(mfi::launch_combine(yd, ystride, w, E, e_sum, out, M, N, as_stream(stream)),
                     "moe_combine launch");
}

// ---------------------------------------------------------------------------
namespace {
// completion counter, per-expert cursors, the expert launch's work-item
// counter and per-chunk readiness counters
inline size_t layer_zero_words(int E, int max_chunks) { return 1 + size_t(E) + 1 + size_t(max_chunks); }

struct LayerScratch {
  unsigned* done;
  int* queue;
  unsigned* ready;
  size_t zero_words;
  int* n_gu;
  int* n_dn;
  int* n_active;
  int* n_chunks;
  int* cursor;
  uint8_t* xq;
  uint8_t* xsc;
  float* logits;
  mfi::GroupDesc* g_gu;
  mfi::EntryDesc* e_gu;
  mfi::GroupDesc* g_dn;
  mfi::EntryDesc* e_dn;
  mfi::ChunkDesc* chunks;
  int* perm;
  float* gu;
  uint8_t* hq;
  uint8_t* hsc;
  uint8_t* xp;
  uint8_t* xp_atoms;
  uint8_t* hp;
  uint8_t* hp_atoms;
  float* yd;
  int max_chunks;
  int T_pad;
  size_t bytes;
};

// Expert GEMMs on tensor cores when the tile shapes divide the layer.
bool layer_uses_tc(int H, int Mi) { return H % 256 == 0 && Mi % 256 == 0; }

LayerScratch carve_layer(void* ws, int T, int H, int Mi, int E, int k) {
  Carve c(ws);
  LayerScratch s;
  const size_t P = size_t(T) * k;
  const bool tc = layer_uses_tc(H, Mi);
  s.max_chunks = int((size_t(E) < P ? size_t(E) : P) + (P + 31) / 32);
  s.T_pad = (T + 31) / 32 * 32;
  const size_t rows = size_t(E) * s.T_pad;  // per-expert regions of T_pad rows
  // counters of the call, one region zeroed by one memset per call
  s.zero_words = layer_zero_words(E, s.max_chunks);
  s.done = c.take<unsigned>(s.zero_words);
  s.cursor = reinterpret_cast<int*>(s.done + 1);
  s.queue = s.cursor + E;
  s.ready = s.done + 1 + E + 1;
  s.n_gu = c.take<int>(1);
  s.n_dn = c.take<int>(1);
  s.n_active = c.take<int>(1);
  s.n_chunks = c.take<int>(1);
  s.xq = c.take<uint8_t>(size_t(T) * (H / 2));
  s.xsc = c.take<uint8_t>(size_t(T) * (H / 32));
  s.logits = c.take<float>(size_t(T) * E);
  s.g_gu = c.take<mfi::GroupDesc>(size_t(2) * E);
  s.e_gu = c.take<mfi::EntryDesc>(2 * P);
  s.g_dn = c.take<mfi::GroupDesc>(size_t(E));
  s.e_dn = c.take<mfi::EntryDesc>(P);
  s.chunks = c.take<mfi::ChunkDesc>(size_t(s.max_chunks));
  s.perm = c.take<int>(rows);
  if (tc) {
    s.gu = nullptr;
    s.hq = s.hsc = nullptr;
    s.xp = c.take<uint8_t>(rows * (H / 2));
    s.xp_atoms = c.take<uint8_t>(rows / 32 * (H / 128) * 512);
    s.hp = c.take<uint8_t>(rows * (Mi / 2));
    s.hp_atoms = c.take<uint8_t>(rows / 32 * (Mi / 128) * 512);
  } else {
    s.gu = c.take<float>(P * 2 * Mi);
    s.hq = c.take<uint8_t>(P * (Mi / 2));
    s.hsc = c.take<uint8_t>(P * (Mi / 32));
    s.xp = s.xp_atoms = s.hp = s.hp_atoms = nullptr;
  }
  s.yd = c.take<float>(P * H);
  s.bytes = c.used + 256;
  return s;
}
}  // namespace

namespace {
// Prefill workspace: per-call counters (zeroed), routing scratch, compact
// expert rows of the quantised tokens and of h with their 128-row atoms.
struct PrefillScratch {
  int* counts;          // [E] tokens per expert (router cursors)
  int* queue;           // work-item counter
  unsigned* gu_done;    // finished gate/up items
  unsigned* ready;      // [max tiles]
  size_t zero_words;
  int* slot_pos;        // [T*k]
  uint8_t* xq; uint8_t* xsc;
  int* perm;
  uint8_t* xp; uint8_t* xa; uint8_t* hp; uint8_t* ha;
  __nv_bfloat16* yd;    // (T*k, H) per-(token, slot) down rows, bf16
  uint8_t* x8;          // tensor-core router scratch (aliases yd: used before it)
  uint8_t* r8;          // the router rows as int8 blocks (E x H bytes)
  int rows;
  size_t bytes;
};

PrefillScratch carve_prefill(void* ws, int T, int H, int Mi, int E, int k) {
  Carve c(ws);
  PrefillScratch s;
  const int P = T * k;
  const size_t max_tiles = size_t(E) + size_t(P) / 128 + 1;
  s.zero_words = size_t(E) + 2 + max_tiles;
  s.counts = c.take<int>(s.zero_words);
  s.queue = s.counts + E;
  s.gu_done = reinterpret_cast<unsigned*>(s.counts + E + 1);
  s.ready = reinterpret_cast<unsigned*>(s.counts + E + 2);
  s.slot_pos = c.take<int>(size_t(P));
  s.xq = c.take<uint8_t>(size_t(T) * (H / 2));
  s.xsc = c.take<uint8_t>(size_t(T) * (H / 32));
  s.rows = int(mfi::prefill_rows(P, E));
  s.perm = c.take<int>(size_t(s.rows));
  s.xp = c.take<uint8_t>(size_t(s.rows) * (H / 2));
  s.xa = c.take<uint8_t>(size_t(s.rows) / 128 * (H / 128) * 512);
  s.hp = c.take<uint8_t>(size_t(s.rows) * (Mi / 2));
  s.ha = c.take<uint8_t>(size_t(s.rows) / 128 * (Mi / 128) * 512);
  // the router's int8 token rows (ceil(T/128)*128 x H bytes) live in the
  // yd region: the router finishes before the expert kernel writes yd
  const size_t x8_bytes = (size_t(T) + 127) / 128 * 128 * size_t(H);
  const size_t yd_elems = size_t(P) * H;
  s.yd = c.take<__nv_bfloat16>(yd_elems * 2 >= x8_bytes ? yd_elems : (x8_bytes + 1) / 2);
  s.x8 = reinterpret_cast<uint8_t*>(s.yd);
  s.r8 = c.take<uint8_t>(size_t(E) * H);
  s.bytes = c.used + 256;
  return s;
}

// Decode kernels up to this many (token, slot) pairs, prefill beyond.
constexpr long long kDecodeMaxPairs = 4096;

bool use_prefill(int T, int H, int Mi, int k) {
  return layer_uses_tc(H, Mi) && (long long)T * k > kDecodeMaxPairs;
}

// events (optional, 6 cudaEvent_t): [0] start, [1] after quantise + route,
// [2] after the scatter, [3] = [4] after the expert GEMMs, [5] after the combine.
int run_prefill(const mfi_moe_weights* w, const void* x_bf16, int T, float* out, int32_t* topi,
                float* topw, float* logits, void* workspace, size_t workspace_bytes,
                cudaStream_t st, void* const* events = nullptr) {
  const int E = w->n_experts, H = w->hidden, Mi = w->inter, k = w->top_k;
  auto rec = [&](int i) -> int {
    if (!events) return MFI_OK;
    // while the stream is being captured an external record becomes an event node
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    cudaStreamIsCapturing(st, &cs);
    const unsigned flags = cs == cudaStreamCaptureStatusActive ? cudaEventRecordExternal : 0u;
    return cuda_status(cudaEventRecordWithFlags(reinterpret_cast<cudaEvent_t>(events[i]), st, flags),
                       "moe_layer event record");
  };
  if (!layer_uses_tc(H, Mi))
    return fail(MFI_ERR_ARG, "the prefill path needs hidden and inter to be multiples of 256");
  if ((long long)T * k > mfi::kPrefillMaxPairs) return fail(MFI_ERR_ARG, "T * top_k must be <= 262144");
  if (bad_ptr(w->prepared)) return fail(MFI_ERR_ARG, "weights.prepared is null (mfi_moe_prepare)");
  PrefillScratch s = carve_prefill(workspace, T, H, Mi, E, k);
  if (workspace_bytes < s.bytes) return fail(MFI_ERR_WORKSPACE, "workspace too small for the prefill layer");
  int rc = rec(0);
  if (rc != MFI_OK) return rc;
  rc = cuda_status(cudaMemsetAsync(s.counts, 0, sizeof(int) * s.zero_words, st),
                   "moe_layer prefill memset");
  if (rc != MFI_OK) return rc;
  mfi::RouteArgs ra{};
  ra.x = x_bf16; ra.xq = s.xq; ra.xsc = s.xsc; ra.wr = w->router_wp; ra.sr = w->router_sc;
  ra.T = T; ra.H = H; ra.E = E; ra.k = k;
  ra.logits = logits; ra.topi = topi; ra.topw = topw;
  ra.cursor = s.counts; ra.slot_pos = s.slot_pos;
  ra.batch = T >= 512;  // enough tokens to fill the GPU one per warp
  ra.x8 = s.x8;
  ra.r8 = s.r8;
  ra.logit_bias = w->logit_bias;
  ra.norm_w = static_cast<const __nv_bfloat16*>(w->norm_weight);
  ra.norm_eps = w->norm_eps;
  ra.err = mfi::device_error_flag();
  rc = cuda_status(mfi::launch_route(ra, st), "moe_layer prefill route launch");
  if (rc == MFI_OK) rc = rec(1);
  if (rc != MFI_OK) return rc;
  rc = cuda_status(mfi::launch_prefill_scatter(s.xq, H / 2, s.xsc, H / 32, topi, k, s.slot_pos,
                                               s.counts, T, E, k, H,
                                               s.perm, s.xp, s.xa, st),
                   "moe_layer prefill scatter launch");
  if (rc == MFI_OK) rc = rec(2);
  if (rc != MFI_OK) return rc;
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  mfi::PrefillLaunch L{};
  L.E = E; L.H = H; L.Mi = Mi; L.top_k = k; L.grid = sms;
  L.prepared = static_cast<const uint8_t*>(w->prepared);
  L.counts = s.counts; L.perm = s.perm; L.rows = s.rows;
  L.xp = s.xp; L.xa = s.xa; L.hp = s.hp; L.ha = s.ha;
  L.yd = s.yd;
  L.err = mfi::device_error_flag(); L.queue = s.queue; L.gu_done = s.gu_done; L.ready = s.ready;
  L.pdl = events == nullptr;  // an event record between the kernels breaks the overlap anyway
  rc = cuda_status(mfi::launch_moe_prefill(L, st), "moe_layer prefill experts launch");
  if (rc == MFI_OK) rc = rec(3);
  if (rc == MFI_OK) rc = rec(4);
  if (rc != MFI_OK) return rc;
  // the decode combine's arithmetic on bf16 rows
  rc = cuda_status(mfi::launch_combine_bf16(s.yd, topw, k, out, T, H, st, events == nullptr),
                   "moe_layer prefill combine launch");
  if (rc == MFI_OK) rc = rec(5);
  return rc;
}

int layer_common_checks(const mfi_moe_weights* w, int T) {
  if (!w) return fail(MFI_ERR_ARG, "null weights");
  const int E = w->n_experts, H = w->hidden, Mi = w->inter, k = w->top_k;
  if (E <= 0 || E > mfi::kRouteMaxE) return fail(MFI_ERR_ARG, "n_experts must be in [1, 256]");
  if (H <= 0 || H % 32 != 0 || Mi <= 0 || Mi % 32 != 0 || H > 4096)
    return fail(MFI_ERR_ARG, "hidden and inter must be positive multiples of 32, hidden <= 4096");
  if (k <= 0 || k > E || k > 32) return fail(MFI_ERR_ARG, "top_k must be in [1, min(E, 32)]");
  if (T < 0) return fail(MFI_ERR_ARG, "T must be >= 0");
  return MFI_OK;
}

bool layer_ptrs_bad(const mfi_moe_weights* w, const void* x, const float* out, const int32_t* topi,
                    const float* topw, const void* ws) {
  return bad_ptr(x) || bad_ptr(out) || bad_ptr(topi) || bad_ptr(topw) || bad_ptr(ws) ||
         bad_ptr(w->gate_wp) || bad_ptr(w->gate_sc) || bad_ptr(w->up_wp) || bad_ptr(w->up_sc) ||
         bad_ptr(w->down_wp) || bad_ptr(w->down_sc) || bad_ptr(w->router_wp) ||
         bad_ptr(w->router_sc);
}
}  // namespace

size_t mfi_moe_layer_prefill_workspace_bytes(int T, int hidden, int inter, int n_experts,
                                             int top_k) {
  if (T <= 0 || hidden <= 0 || inter <= 0 || n_experts <= 0 || top_k <= 0) return 0;
  return carve_prefill(nullptr, T, hidden, inter, n_experts, top_k).bytes;
}

int mfi_moe_layer_prefill(const mfi_moe_weights* w, const void* x_bf16, int T, float* out,
                          int32_t* topi, float* topw, float* logits, void* workspace,
                          size_t workspace_bytes, void* stream) {
  int rc = layer_common_checks(w, T);
  if (rc != MFI_OK) return rc;
  if (T == 0) return MFI_OK;
  if (layer_ptrs_bad(w, x_bf16, out, topi, topw, workspace)) return fail(MFI_ERR_ARG, "null pointer");
  if ((reinterpret_cast<uintptr_t>(x_bf16) & 15) != 0 ||
      (reinterpret_cast<uintptr_t>(w->router_wp) & 15) != 0)
    return fail(MFI_ERR_ARG, "x and router_wp must be 16-byte aligned");
  return run_prefill(w, x_bf16, T, out, topi, topw, logits, workspace, workspace_bytes,
                     as_stream(stream));
}

size_t mfi_moe_prepared_bytes(int n_experts, int hidden, int inter) {
  if (!layer_uses_tc(hidden, inter)) return 0;
  return mfi::moe_prepared_bytes(n_experts, hidden, inter);
}

int mfi_moe_prepare(const mfi_moe_weights* w, void* prepared, size_t prepared_bytes,
                    void* stream) {
  if (!w) return fail(MFI_ERR_ARG, "null weights");
  const int E = w->n_experts, H = w->hidden, Mi = w->inter;
  if (!layer_uses_tc(H, Mi)) return MFI_OK;
  if (bad_ptr(prepared) || bad_ptr(w->gate_wp) || bad_ptr(w->gate_sc) || bad_ptr(w->up_wp) ||
      bad_ptr(w->up_sc) || bad_ptr(w->down_wp) || bad_ptr(w->down_sc))
    return fail(MFI_ERR_ARG, "null pointer");
  if (prepared_bytes < mfi::moe_prepared_bytes(E, H, Mi))
    return fail(MFI_ERR_WORKSPACE, "prepared buffer smaller than mfi_moe_prepared_bytes()");
  return cuda_status(mfi::launch_moe_prepare(w->gate_wp, w->gate_sc, w->up_wp, w->up_sc,
                                             w->down_wp, w->down_sc, E, H, Mi,
                                             static_cast<uint8_t*>(prepared), as_stream(stream)),
                     "moe_prepare launch");
}

size_t mfi_moe_layer_workspace_bytes(int T, int hidden, int inter, int n_experts, int top_k) {
  if (use_prefill(T, hidden, inter, top_k))
    return mfi_moe_layer_prefill_workspace_bytes(T, hidden, inter, n_experts, top_k);
  return carve_layer(nullptr, T, hidden, inter, n_experts, top_k).bytes;
}

int mfi_moe_layer_init_workspace(void* workspace, size_t workspace_bytes, int T, int hidden,
                                 int inter, int n_experts, int top_k, void* stream) {
  if (bad_ptr(workspace)) return fail(MFI_ERR_ARG, "null pointer");
  if (T <= 0 || hidden <= 0 || inter <= 0 || n_experts <= 0 || top_k <= 0)
    return fail(MFI_ERR_ARG, "invalid shape");
  if (workspace_bytes < mfi_moe_layer_workspace_bytes(T, hidden, inter, n_experts, top_k))
    return fail(MFI_ERR_WORKSPACE, "workspace too small for moe_layer");
  if (use_prefill(T, hidden, inter, top_k)) return MFI_OK;  // zeroed per call
  LayerScratch s = carve_layer(workspace, T, hidden, inter, n_experts, top_k);
  return cuda_status(cudaMemsetAsync(s.done, 0, sizeof(unsigned) * s.zero_words, as_stream(stream)),
                     "moe_layer_init_workspace memset");
}

int mfi_moe_layer(const mfi_moe_weights* w, const void* x_bf16, int T, float* out, int32_t* topi,
                  float* topw, float* logits, void* workspace, size_t workspace_bytes,
                  void* stream) {
  return mfi_moe_layer_ex(w, x_bf16, T, out, topi, topw, logits, workspace, workspace_bytes,
                          nullptr, 0, stream);
}

int mfi_moe_layer_ex(const mfi_moe_weights* w, const void* x_bf16, int T, float* out,
                     int32_t* topi, float* topw, float* logits, void* workspace,
                     size_t workspace_bytes, void* const* events, int n_events, void* stream) {
  if (events && n_events < 6) return fail(MFI_ERR_ARG, "events must hold 6 cudaEvent_t handles");
  int rc0 = layer_common_checks(w, T);
  if (rc0 != MFI_OK) return rc0;
  const int E = w->n_experts, H = w->hidden, Mi = w->inter, k = w->top_k;
  const bool prefill = use_prefill(T, H, Mi, k);
  if (!prefill && (long long)T * k > mfi::kRouteMaxPairs)
    return fail(MFI_ERR_ARG, "T * top_k must be <= 4096 unless hidden and inter are multiples of 256");
  if (T == 0) return MFI_OK;
  if (layer_ptrs_bad(w, x_bf16, out, topi, topw, workspace)) return fail(MFI_ERR_ARG, "null pointer");
  if (prefill) {
    if ((reinterpret_cast<uintptr_t>(x_bf16) & 15) != 0 ||
        (reinterpret_cast<uintptr_t>(w->router_wp) & 15) != 0)
      return fail(MFI_ERR_ARG, "x and router_wp must be 16-byte aligned");
    return run_prefill(w, x_bf16, T, out, topi, topw, logits, workspace, workspace_bytes,
                       as_stream(stream), events);
  }
  if (workspace_bytes < mfi_moe_layer_workspace_bytes(T, H, Mi, E, k))
    return fail(MFI_ERR_WORKSPACE, "workspace too small for moe_layer");
  LayerScratch s = carve_layer(workspace, T, H, Mi, E, k);
  cudaStream_t st = as_stream(stream);
  auto mark = [&](int i) -> int {
    if (!events) return MFI_OK;
    // While the stream is being captured into a CUDA graph an external record
    // becomes an event node, so the stage times stay measurable on replay.
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    cudaStreamIsCapturing(st, &cs);
    const unsigned flags = cs == cudaStreamCaptureStatusActive ? cudaEventRecordExternal : 0u;
    return cuda_status(cudaEventRecordWithFlags(reinterpret_cast<cudaEvent_t>(events[i]), st, flags),
                       "moe_layer event record");
  };
  int rc = mark(0);
  if (rc != MFI_OK) return rc;
  const bool tc = layer_uses_tc(H, Mi);
  if (!tc) {
    // CUDA-core path: counters zeroed per call
    rc = cuda_status(cudaMemsetAsync(s.done, 0, sizeof(unsigned) * s.zero_words, st),
                     "moe_layer memset");
    if (rc != MFI_OK) return rc;
  }
  // tensor-core path: the counters were zeroed by mfi_moe_layer_init_workspace
  // and every call's combine clears them again (no memset node per layer)
  if ((reinterpret_cast<uintptr_t>(x_bf16) & 15) != 0 ||
      (reinterpret_cast<uintptr_t>(w->router_wp) & 15) != 0)
    return fail(MFI_ERR_ARG, "x and router_wp must be 16-byte aligned");
  mfi::RouteArgs ra{};
  ra.x = x_bf16;
  ra.xq = s.xq; ra.xsc = s.xsc; ra.wr = w->router_wp; ra.sr = w->router_sc;
  ra.T = T; ra.H = H; ra.E = E; ra.k = k;
  ra.logits = logits ? logits : s.logits;
  ra.topi = topi; ra.topw = topw; ra.done = s.done;
  ra.gate_wp = w->gate_wp; ra.gate_sc = w->gate_sc; ra.up_wp = w->up_wp; ra.up_sc = w->up_sc;
  ra.down_wp = w->down_wp; ra.down_sc = w->down_sc; ra.Mi = Mi;
  ra.g_gu = tc ? nullptr : s.g_gu; ra.e_gu = tc ? nullptr : s.e_gu; ra.n_gu = s.n_gu;
  ra.g_dn = tc ? nullptr : s.g_dn; ra.e_dn = tc ? nullptr : s.e_dn; ra.n_dn = s.n_dn;
  ra.n_active = s.n_active;
  ra.chunks = s.chunks; ra.n_chunks = s.n_chunks; ra.perm = s.perm;
  ra.cursor = tc ? s.cursor : nullptr;
  ra.xp = tc ? s.xp : nullptr;
  ra.xp_atoms = tc ? s.xp_atoms : nullptr;
  ra.T_pad = s.T_pad;
  ra.err = mfi::device_error_flag();
  ra.logit_bias = w->logit_bias;
  ra.norm_w = static_cast<const __nv_bfloat16*>(w->norm_weight);
  ra.norm_eps = w->norm_eps;
  if (tc && w->prepared && (reinterpret_cast<uintptr_t>(w->prepared) & 15) == 0) {
    // the router issues the gate/up weight prefetch after its own loads
    ra.pf_base = static_cast<const uint8_t*>(w->prepared);
    ra.pf_bytes = prefetch_bytes((long long)T * k, E, true) & ~size_t(15);
    const size_t gu_bytes = mfi::moe_prepared_bytes(E, H, Mi) / 3 * 2;
    if (ra.pf_bytes > gu_bytes) ra.pf_bytes = gu_bytes & ~size_t(15);
  }
  rc = cuda_status(mfi::launch_route(ra, st), "moe_layer route launch");
  if (rc != MFI_OK || (rc = mark(1)) != MFI_OK) return rc;
  const int P = T * k;
  if (tc) {
    if (bad_ptr(w->prepared)) return fail(MFI_ERR_ARG, "weights.prepared is null (mfi_moe_prepare)");
    if ((rc = mark(2)) != MFI_OK) return rc;  // the chunk rows were written by the route kernel
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    mfi::MoeTcLaunch L{};
    L.E = E; L.H = H; L.Mi = Mi; L.max_chunks = s.max_chunks; L.grid = sms;
    L.prepared = static_cast<const uint8_t*>(w->prepared);
    L.counts = s.cursor; L.perm = s.perm;
    L.rows = E * s.T_pad;
    L.xp = s.xp; L.xp_atoms = s.xp_atoms; L.hp = s.hp; L.hp_atoms = s.hp_atoms; L.yd = s.yd;
    L.err = mfi::device_error_flag();
    // kernels overlap their prologue with the previous kernel's tail, except
    // when stage events sit between them
    L.pdl = events == nullptr;
    L.pf_bytes = 0;  // issued by the router
    L.queue = s.queue;
    L.ready = s.ready;
    rc = cuda_status(mfi::launch_moe_tc(L, st), "moe_layer experts (tensor cores) launch");
    if (rc != MFI_OK || (rc = mark(3)) != MFI_OK || (rc = mark(4)) != MFI_OK) return rc;
  } else {
    const int max_groups = E < P ? E : P;
    rc = cuda_status(mfi::launch_grouped_gemv(s.g_gu, s.n_gu, 2 * max_groups, s.e_gu, s.xq, s.xsc,
                                              s.gu, Mi, H, kGemvMaxCtas, st),
                     "moe_layer gate/up launch");
    if (rc != MFI_OK || (rc = mark(2)) != MFI_OK) return rc;
    rc = cuda_status(mfi::launch_swiglu_quant(s.gu, 2L * Mi, nullptr, P, nullptr, s.hq, s.hsc, Mi,
                                              Mi, st),
                     "moe_layer swiglu launch");
    if (rc != MFI_OK || (rc = mark(3)) != MFI_OK) return rc;
    rc = cuda_status(mfi::launch_grouped_gemv(s.g_dn, s.n_dn, max_groups, s.e_dn, s.hq, s.hsc,
                                              s.yd, H, Mi, kGemvMaxCtas, st),
                     "moe_layer down launch");
    if (rc != MFI_OK || (rc = mark(4)) != MFI_OK) return rc;
  }
  rc = cuda_status(mfi::launch_combine(s.yd, H, topw, k, k, out, T, H, st, tc && !events,
                                       tc ? s.done : nullptr, tc ? int(s.zero_words) : 0),
                   "moe_layer combine launch");
  if (rc != MFI_OK) return rc;
  return mark(5);
}

// ---------------------------------------------------------------------------
// Routing alone and expert compute on pre-routed rows: the two halves of
// mfi_moe_layer that expert parallelism puts a token exchange between.

namespace {
// Scratch of the tensor-core router (route_tc.cu) for T tokens: the int8 token
// tiles (T rounded up to 128 rows x hidden bytes) and the int8 router blocks
// (n_experts x hidden bytes); 0 where that router does not apply.
size_t route_tc_scratch(int T, int H, int E) {
  if (T < 512 || E != 128 || H < 128 || H % 128 != 0) return 0;
  return (size_t(T) + 127) / 128 * 128 * size_t(H) + size_t(E) * H + 512;
}
}  // namespace

size_t mfi_moe_route_workspace_bytes(int T, int hidden, int n_experts) {
  if (T < 0 || hidden <= 0 || n_experts <= 0) return 0;
  return route_tc_scratch(T, hidden, n_experts);
}

int mfi_moe_route(const mfi_moe_weights* w, const void* x_bf16, int T, uint8_t* xq, uint8_t* xsc,
                  int32_t* topi, float* topw, float* logits, void* stream) {
  return mfi_moe_route_ex(w, x_bf16, T, xq, xsc, topi, topw, logits, nullptr, 0, stream);
}

int mfi_moe_route_ex(const mfi_moe_weights* w, const void* x_bf16, int T, uint8_t* xq,
                     uint8_t* xsc, int32_t* topi, float* topw, float* logits, void* workspace,
                     size_t workspace_bytes, void* stream) {
  if (!w) return fail(MFI_ERR_ARG, "null weights");
  const int E = w->n_experts, H = w->hidden, k = w->top_k;
  if (E <= 0 || E > mfi::kRouteMaxE) return fail(MFI_ERR_ARG, "n_experts must be in [1, 256]");
  if (H <= 0 || H % 32 != 0 || H > 4096)
    return fail(MFI_ERR_ARG, "hidden must be a positive multiple of 32, <= 4096");
  if (k <= 0 || k > E || k > 32) return fail(MFI_ERR_ARG, "top_k must be in [1, min(E, 32)]");
  if (T < 0) return fail(MFI_ERR_ARG, "T must be >= 0");
  if (T == 0) return MFI_OK;
  if (bad_ptr(x_bf16) || bad_ptr(xq) || bad_ptr(xsc) || bad_ptr(topi) || bad_ptr(topw) ||
      bad_ptr(w->router_wp) || bad_ptr(w->router_sc))
    return fail(MFI_ERR_ARG, "null pointer");
  if ((reinterpret_cast<uintptr_t>(x_bf16) & 15) != 0 || (reinterpret_cast<uintptr_t>(xq) & 15) != 0 ||
      (reinterpret_cast<uintptr_t>(xsc) & 3) != 0 ||
      (reinterpret_cast<uintptr_t>(w->router_wp) & 15) != 0)
    return fail(MFI_ERR_ARG, "x, xq and router_wp must be 16-byte aligned, xsc 4-byte aligned");
  mfi::RouteArgs ra{};
  ra.x = x_bf16; ra.xq = xq; ra.xsc = xsc; ra.wr = w->router_wp; ra.sr = w->router_sc;
  ra.T = T; ra.H = H; ra.E = E; ra.k = k;
  ra.logits = logits; ra.topi = topi; ra.topw = topw;
  ra.err = mfi::device_error_flag();
  ra.logit_bias = w->logit_bias;
  ra.norm_w = static_cast<const __nv_bfloat16*>(w->norm_weight);
  ra.norm_eps = w->norm_eps;
  // many tokens: one token per warp, or the tensor-core router when the
  // caller gave its scratch
  ra.batch = T >= 512;
  const size_t need = route_tc_scratch(T, H, E);
  if (need && workspace && workspace_bytes >= need &&
      (reinterpret_cast<uintptr_t>(workspace) & 255) == 0) {
    ra.x8 = static_cast<uint8_t*>(workspace);
    ra.r8 = ra.x8 + (size_t(T) + 127) / 128 * 128 * size_t(H);
  }
  // no work lists, no expert regions: the kernel stops after the routing
  return cuda_status(mfi::launch_route(ra, as_stream(stream)), "moe_route launch");
}

namespace {
struct ExpertScratch {
  int* cursor;
  int max_chunks;
  size_t zero_words;
  int* perm;
  uint8_t* xp;
  uint8_t* xp_atoms;
  uint8_t* hp;
  uint8_t* hp_atoms;
  float* yd;
  int T_pad;
  size_t bytes;
};

ExpertScratch carve_experts(void* ws, int R, int H, int Mi, int E, int k) {
  Carve c(ws);
  ExpertScratch s;
  s.T_pad = (R + 31) / 32 * 32;
  const size_t rows = size_t(E) * s.T_pad;
  s.max_chunks = int((size_t(E) < size_t(R) * k ? size_t(E) : size_t(R) * k) +
                     (size_t(R) * k + 31) / 32);
  // per-expert cursors, the work-item counter, per-chunk readiness: zeroed per call
  s.zero_words = size_t(E) + 1 + size_t(s.max_chunks);
  s.cursor = c.take<int>(s.zero_words);
  s.perm = c.take<int>(rows);
  s.xp = c.take<uint8_t>(rows * (H / 2));
  s.xp_atoms = c.take<uint8_t>(rows / 32 * (H / 128) * 512);
  s.hp = c.take<uint8_t>(rows * (Mi / 2));
  s.hp_atoms = c.take<uint8_t>(rows / 32 * (Mi / 128) * 512);
  s.yd = c.take<float>(size_t(R) * k * H);
  s.bytes = c.used + 256;
  return s;
}

// Pre-routed rows whose pairs exceed the decode kernel's 16384 go through the
// prefill kernel (per-expert regions of 128-row tiles, bf16 rows of y).
constexpr long long kExpertsDecodeMaxPairs = 16384;

struct ExpertPrefillScratch {
  int* counts;          // [E] rows per expert
  int* queue;           // work-item counter
  unsigned* gu_done;    // finished gate/up items
  unsigned* ready;      // [max tiles]
  size_t zero_words;
  int* slot_pos;        // [R*k]
  int* perm;
  uint8_t* xp; uint8_t* xa; uint8_t* hp; uint8_t* ha;
  __nv_bfloat16* yd;    // (R*k, H)
  int rows;
  size_t bytes;
};

ExpertPrefillScratch carve_experts_prefill(void* ws, int R, int H, int Mi, int E, int k) {
  Carve c(ws);
  ExpertPrefillScratch s;
  const long long P = (long long)R * k;
  const size_t max_tiles = size_t(E) + size_t(P) / 128 + 1;
  s.zero_words = size_t(E) + 2 + max_tiles;
  s.counts = c.take<int>(s.zero_words);
  s.queue = s.counts + E;
  s.gu_done = reinterpret_cast<unsigned*>(s.counts + E + 1);
  s.ready = reinterpret_cast<unsigned*>(s.counts + E + 2);
  s.slot_pos = c.take<int>(size_t(P));
  s.rows = int(mfi::prefill_rows(int(P), E));
  s.perm = c.take<int>(size_t(s.rows));
  s.xp = c.take<uint8_t>(size_t(s.rows) * (H / 2));
  s.xa = c.take<uint8_t>(size_t(s.rows) / 128 * (H / 128) * 512);
  s.hp = c.take<uint8_t>(size_t(s.rows) * (Mi / 2));
  s.ha = c.take<uint8_t>(size_t(s.rows) / 128 * (Mi / 128) * 512);
  s.yd = c.take<__nv_bfloat16>(size_t(P) * H);
  s.bytes = c.used + 256;
  return s;
}

bool experts_use_prefill(int R, int k) { return (long long)R * k > kExpertsDecodeMaxPairs; }
}  // namespace

size_t mfi_moe_experts_workspace_bytes(int R, int hidden, int inter, int n_experts, int top_k) {
  if (R < 0 || hidden <= 0 || inter <= 0 || n_experts <= 0 || top_k <= 0) return 0;
  if ((long long)R * top_k > mfi::kPrefillMaxPairs) return 0;
  if (experts_use_prefill(R, top_k))
    return carve_experts_prefill(nullptr, R, hidden, inter, n_experts, top_k).bytes;
  return carve_experts(nullptr, R, hidden, inter, n_experts, top_k).bytes;
}

int mfi_moe_experts(const mfi_moe_weights* w, const uint8_t* xq, long long xq_ld,
                    const uint8_t* xsc, long long xsc_ld, const int32_t* sel, long long sel_ld,
                    const float* selw, long long selw_ld, int R, float* out, long long out_ld,
                    void* workspace, size_t workspace_bytes, void* stream) {
  if (!w) return fail(MFI_ERR_ARG, "null weights");
  const int E = w->n_experts, H = w->hidden, Mi = w->inter, k = w->top_k;
  if (E <= 0 || E > mfi::kRouteMaxE) return fail(MFI_ERR_ARG, "n_experts must be in [1, 256]");
  if (!layer_uses_tc(H, Mi))
    return fail(MFI_ERR_ARG, "moe_experts needs hidden and inter to be multiples of 256");
  if (k <= 0 || k > 32) return fail(MFI_ERR_ARG, "top_k must be in [1, 32]");
  if (R < 0 || (long long)R * k > mfi::kPrefillMaxPairs)
    return fail(MFI_ERR_ARG, "rows * top_k must be <= 262144");
  if (R == 0) return MFI_OK;
  if (bad_ptr(xq) || bad_ptr(xsc) || bad_ptr(sel) || bad_ptr(selw) || bad_ptr(out) ||
      bad_ptr(workspace) || bad_ptr(w->prepared))
    return fail(MFI_ERR_ARG, "null pointer (weights.prepared comes from mfi_moe_prepare)");
  if (xq_ld < H / 2 || xsc_ld < H / 32 || sel_ld < k || selw_ld < k || out_ld < H)
    return fail(MFI_ERR_ARG, "row strides must cover one row");
  if ((reinterpret_cast<uintptr_t>(xq) & 15) != 0 || xq_ld % 16 != 0 ||
      (reinterpret_cast<uintptr_t>(xsc) & 3) != 0 || xsc_ld % 4 != 0 ||
      (reinterpret_cast<uintptr_t>(out) & 15) != 0 || out_ld % 4 != 0)
    return fail(MFI_ERR_ARG,
                "xq and out rows must be 16-byte aligned, xsc rows 4-byte aligned");
  if (workspace_bytes < mfi_moe_experts_workspace_bytes(R, H, Mi, E, k))
    return fail(MFI_ERR_WORKSPACE, "workspace too small for moe_experts");
  cudaStream_t st = as_stream(stream);
  if (experts_use_prefill(R, k)) {
    // many rows (expert-parallel prefill): count the pairs per local expert,
    // place the rows in 128-row tiles, the prefill tcgen05 kernel, then the
    // masked combine of the bf16 rows
    if (H % 8 != 0) return fail(MFI_ERR_ARG, "hidden must be a multiple of 8");
    ExpertPrefillScratch s = carve_experts_prefill(workspace, R, H, Mi, E, k);
    int rc = cuda_status(cudaMemsetAsync(s.counts, 0, sizeof(int) * s.zero_words, st),
                         "moe_experts memset");
    if (rc != MFI_OK) return rc;
    rc = cuda_status(mfi::launch_prefill_count_sel(sel, sel_ld, R, k, E, s.counts, s.slot_pos,
                                                   mfi::device_error_flag(), st),
                     "moe_experts count launch");
    if (rc != MFI_OK) return rc;
    rc = cuda_status(mfi::launch_prefill_scatter(xq, xq_ld, xsc, xsc_ld, sel, sel_ld, s.slot_pos,
                                                 s.counts, R, E, k, H, s.perm, s.xp, s.xa, st),
                     "moe_experts scatter launch");
    if (rc != MFI_OK) return rc;
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    mfi::PrefillLaunch L{};
    L.E = E; L.H = H; L.Mi = Mi; L.top_k = k; L.grid = sms;
    L.prepared = static_cast<const uint8_t*>(w->prepared);
    L.counts = s.counts; L.perm = s.perm; L.rows = s.rows;
    L.xp = s.xp; L.xa = s.xa; L.hp = s.hp; L.ha = s.ha;
    L.yd = s.yd;
    L.err = mfi::device_error_flag(); L.queue = s.queue; L.gu_done = s.gu_done; L.ready = s.ready;
    L.pdl = true;
    rc = cuda_status(mfi::launch_moe_prefill(L, st), "moe_experts prefill launch");
    if (rc != MFI_OK) return rc;
    return cuda_status(mfi::launch_combine_sel_bf16(s.yd, sel, sel_ld, selw, selw_ld, R, k, E, H,
                                                    out, out_ld, st),
                       "moe_experts combine launch");
  }
  ExpertScratch s = carve_experts(workspace, R, H, Mi, E, k);
  int rc = cuda_status(cudaMemsetAsync(s.cursor, 0, sizeof(int) * s.zero_words, st),
                       "moe_experts memset");
  if (rc != MFI_OK) return rc;
  rc = cuda_status(mfi::launch_scatter_sel(xq, xq_ld, xsc, xsc_ld, sel, sel_ld, R, k, H, E, s.T_pad,
                                           s.cursor, s.perm, s.xp, s.xp_atoms,
                                           mfi::device_error_flag(), st),
                   "moe_experts scatter launch");
  if (rc != MFI_OK) return rc;
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  mfi::MoeTcLaunch L{};
  L.E = E; L.H = H; L.Mi = Mi; L.grid = sms;
  L.max_chunks = s.max_chunks;
  L.prepared = static_cast<const uint8_t*>(w->prepared);
  L.counts = s.cursor; L.perm = s.perm;
  L.rows = E * s.T_pad;
  L.xp = s.xp; L.xp_atoms = s.xp_atoms; L.hp = s.hp; L.hp_atoms = s.hp_atoms; L.yd = s.yd;
  L.err = mfi::device_error_flag();
  L.pdl = true;
  L.pf_bytes = prefetch_bytes((long long)R * k, E, true);
  L.queue = s.cursor + E;
  L.ready = reinterpret_cast<unsigned*>(s.cursor + E + 1);
  rc = cuda_status(mfi::launch_moe_tc(L, st), "moe_experts launch");
  if (rc != MFI_OK) return rc;
  return cuda_status(mfi::launch_combine_sel(s.yd, sel, sel_ld, selw, selw_ld, R, k, E, H, out,
                                             out_ld, st),
                     "moe_experts combine launch");
}

// ---------------------------------------------------------------------------
// Expert-parallel exchange buffers.

int mfi_ep_row_bytes(int hidden, int top_k) {
  if (hidden <= 0 || hidden % 128 != 0 || top_k <= 0 || top_k > 32) return 0;
  return mfi::ep_row_bytes(hidden, top_k);
}

namespace {
int ep_check(int T, int H, int k, int n_ranks, int C) {
  if (H <= 0 || H % 128 != 0 || H > 4096)
    return fail(MFI_ERR_ARG, "hidden must be a positive multiple of 128, <= 4096");
  if (k <= 0 || k > 32) return fail(MFI_ERR_ARG, "top_k must be in [1, 32]");
  if (n_ranks <= 0 || n_ranks > 64) return fail(MFI_ERR_ARG, "n_ranks must be in [1, 64]");
  if (T < 0 || C < T) return fail(MFI_ERR_ARG, "capacity must be >= T >= 0");
  return MFI_OK;
}
}  // namespace

int mfi_ep_pack(const uint8_t* xq, const uint8_t* xsc, const int32_t* topi, const float* topw,
                int T, int hidden, int top_k, int n_ranks, int experts_per_rank, int capacity,
                int32_t* counts, uint8_t* send, int32_t* pack_pos, void* stream) {
  int rc = ep_check(T, hidden, top_k, n_ranks, capacity);
  if (rc != MFI_OK) return rc;
  if (experts_per_rank <= 0) return fail(MFI_ERR_ARG, "experts_per_rank must be positive");
  if (bad_ptr(counts) || bad_ptr(send) || (T > 0 && (bad_ptr(xq) || bad_ptr(xsc) ||
                                                      bad_ptr(topi) || bad_ptr(topw) ||
                                                      bad_ptr(pack_pos))))
    return fail(MFI_ERR_ARG, "null pointer");
  if ((reinterpret_cast<uintptr_t>(send) & 15) != 0 || (reinterpret_cast<uintptr_t>(xq) & 15) != 0 ||
      (reinterpret_cast<uintptr_t>(xsc) & 3) != 0)
    return fail(MFI_ERR_ARG, "send and xq must be 16-byte aligned, xsc 4-byte aligned");
  return cuda_status(mfi::launch_ep_pack(xq, xsc, topi, topw, T, hidden, top_k, n_ranks,
                                         experts_per_rank, capacity, counts, send, pack_pos,
                                         as_stream(stream)),
                     "ep_pack launch");
}

int mfi_ep_mask_recv(uint8_t* recv, int n_ranks, int capacity, int hidden, int top_k,
                     void* stream) {
  int rc = ep_check(0, hidden, top_k, n_ranks, capacity);
  if (rc != MFI_OK) return rc;
  if (bad_ptr(recv)) return fail(MFI_ERR_ARG, "null pointer");
  if ((reinterpret_cast<uintptr_t>(recv) & 15) != 0)
    return fail(MFI_ERR_ARG, "recv must be 16-byte aligned");
  return cuda_status(mfi::launch_ep_mask_recv(n_ranks, capacity, hidden, top_k, recv,
                                              mfi::device_error_flag(),
                                              as_stream(stream)),
                     "ep_mask_recv launch");
}

int mfi_ep_unpack(const float* ret, const int32_t* pack_pos, int T, int n_ranks, int capacity,
                  int hidden, float* out, void* stream) {
  int rc = ep_check(T, hidden, 1, n_ranks, capacity);
  if (rc != MFI_OK) return rc;
  if (T == 0) return MFI_OK;
  if (bad_ptr(ret) || bad_ptr(pack_pos) || bad_ptr(out)) return fail(MFI_ERR_ARG, "null pointer");
  if ((reinterpret_cast<uintptr_t>(ret) & 15) || (reinterpret_cast<uintptr_t>(out) & 15))
    return fail(MFI_ERR_ARG, "ret and out must be 16-byte aligned");
  return cuda_status(mfi::launch_ep_unpack(ret, pack_pos, T, n_ranks, capacity, hidden, out,
                                           as_stream(stream)),
                     "ep_unpack launch");
}

// ---------------------------------------------------------------------------
// Expert parallelism over peer memory (CUDA IPC + NVLink stores).

int mfi_ipc_alloc(size_t bytes, void** ptr) {
  if (!ptr || bytes == 0) return fail(MFI_ERR_ARG, "ipc_alloc: null out pointer or zero size");
  *ptr = nullptr;
  void* p = nullptr;
  int rc = cuda_status(cudaMalloc(&p, bytes), "ipc_alloc cudaMalloc");
  if (rc != MFI_OK) return rc;
  rc = cuda_status(cudaMemset(p, 0, bytes), "ipc_alloc cudaMemset");
  if (rc != MFI_OK) {
    cudaFree(p);
    return rc;
  }
  *ptr = p;
  return MFI_OK;
}

int mfi_ipc_free(void* ptr) {
  if (!ptr) return MFI_OK;
  return cuda_status(cudaFree(ptr), "ipc_free");
}

int mfi_ipc_handle(const void* ptr, void* handle) {
  if (!ptr || !handle) return fail(MFI_ERR_ARG, "null pointer");
  cudaIpcMemHandle_t h;
  int rc = cuda_status(cudaIpcGetMemHandle(&h, const_cast<void*>(ptr)), "cudaIpcGetMemHandle");
  if (rc == MFI_OK) memcpy(handle, &h, sizeof(h));
  return rc;
}

int mfi_ipc_open(const void* handle, void** ptr) {
  if (!handle || !ptr) return fail(MFI_ERR_ARG, "null pointer");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  return cuda_status(cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess),
                     "cudaIpcOpenMemHandle");
}

int mfi_ipc_close(void* ptr) {
  if (!ptr) return MFI_OK;
  return cuda_status(cudaIpcCloseMemHandle(ptr), "cudaIpcCloseMemHandle");
}

int mfi_copy_async(void* dst, const void* src, size_t bytes, void* stream) {
  if (bytes == 0) return MFI_OK;
  if (!dst || !src) return fail(MFI_ERR_ARG, "null pointer");
  return cuda_status(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDefault, as_stream(stream)),
                     "copy_async");
}

size_t mfi_ep_flag_bytes(void) { return sizeof(unsigned) * mfi::kFlagWords; }

size_t mfi_ep_recv_bytes(int n_ranks, int capacity, int hidden, int top_k) {
  if (n_ranks <= 0 || capacity < 0 || hidden <= 0 || hidden % 128 || top_k <= 0 || top_k > 32)
    return 0;
  return size_t(n_ranks) * (capacity + 1) * mfi::ep_row_bytes(hidden, top_k);
}

size_t mfi_ep_ret_bytes(int n_ranks, int capacity, int hidden) {
  if (n_ranks <= 0 || capacity < 0 || hidden <= 0) return 0;
  return size_t(n_ranks) * (capacity + 1) * hidden * sizeof(float);
}

size_t mfi_ep_table_bytes(void) { return sizeof(mfi::EpTable); }

int mfi_ep_table_set(void* table, int n_ranks, void* const* recv, void* const* ret,
                     void* const* flags) {
  if (!table || !recv || !ret || !flags) return fail(MFI_ERR_ARG, "null pointer");
  if (n_ranks <= 0 || n_ranks > mfi::kEpMaxRanks) return fail(MFI_ERR_ARG, "n_ranks must be in [1, 64]");
  mfi::EpTable t{};
  for (int d = 0; d < n_ranks; ++d) {
    if (!recv[d] || !ret[d] || !flags[d]) return fail(MFI_ERR_ARG, "null peer pointer");
    if ((reinterpret_cast<uintptr_t>(recv[d]) & 15) || (reinterpret_cast<uintptr_t>(ret[d]) & 15) ||
        (reinterpret_cast<uintptr_t>(flags[d]) & 15))
      return fail(MFI_ERR_ARG, "peer buffers must be 16-byte aligned");
    t.recv[d] = static_cast<uint8_t*>(recv[d]);
    t.ret[d] = static_cast<float*>(ret[d]);
    t.flags[d] = static_cast<unsigned*>(flags[d]);
  }
  return cuda_status(cudaMemcpy(table, &t, sizeof(t), cudaMemcpyHostToDevice), "ep_table_set");
}

namespace {
int ep_p2p_check(int rank, int n, int C, int H, int k) {
  if (n <= 0 || n > mfi::kEpMaxRanks) return fail(MFI_ERR_ARG, "n_ranks must be in [1, 64]");
  if (rank < 0 || rank >= n) return fail(MFI_ERR_ARG, "rank out of range");
  if (C < 0) return fail(MFI_ERR_ARG, "capacity must be >= 0");
  if (H <= 0 || H % 256 != 0 || H > 4096)
    return fail(MFI_ERR_ARG, "hidden must be a positive multiple of 256, <= 4096");
  if (k <= 0 || k > 32) return fail(MFI_ERR_ARG, "top_k must be in [1, 32]");
  return MFI_OK;
}
}  // namespace

int mfi_ep_route_dispatch(const mfi_moe_weights* w, const void* x_bf16, int T, int rank,
                          int n_ranks, int capacity, const void* table, void* flags,
                          int32_t* topi, float* topw, int32_t* pack_pos, void* stream) {
  if (!w) return fail(MFI_ERR_ARG, "null weights");
  const int E = w->n_experts, H = w->hidden, k = w->top_k;
  int rc = ep_p2p_check(rank, n_ranks, capacity, H, k);
  if (rc != MFI_OK) return rc;
  if (E <= 0 || E > mfi::kRouteMaxE || E % n_ranks != 0)
    return fail(MFI_ERR_ARG, "n_experts must be in [1, 256] and divisible by n_ranks");
  if (k > E) return fail(MFI_ERR_ARG, "top_k must be <= n_experts");
  if (T < 0 || T > capacity) return fail(MFI_ERR_ARG, "T must be in [0, capacity]");
  if (bad_ptr(table) || bad_ptr(flags) || bad_ptr(w->router_wp) || bad_ptr(w->router_sc) ||
      (T > 0 && (bad_ptr(x_bf16) || bad_ptr(topi) || bad_ptr(topw) || bad_ptr(pack_pos))))
    return fail(MFI_ERR_ARG, "null pointer");
  if ((reinterpret_cast<uintptr_t>(x_bf16) & 15) || (reinterpret_cast<uintptr_t>(w->router_wp) & 15))
    return fail(MFI_ERR_ARG, "x and router_wp must be 16-byte aligned");
  cudaStream_t st = as_stream(stream);
  unsigned* fl = static_cast<unsigned*>(flags);
  // the per-call counters are zero: mfi_ipc_alloc zeroes the flag area and
  // every call's mfi_ep_unpack_wait clears them again
  mfi::RouteArgs ra{};
  ra.x = x_bf16; ra.wr = w->router_wp; ra.sr = w->router_sc;
  ra.T = T; ra.H = H; ra.E = E; ra.k = k;
  ra.topi = topi; ra.topw = topw;
  ra.err = mfi::device_error_flag();
  ra.logit_bias = w->logit_bias;
  ra.norm_w = static_cast<const __nv_bfloat16*>(w->norm_weight);
  ra.norm_eps = w->norm_eps;
  ra.ep.table = static_cast<const mfi::EpTable*>(table);
  ra.ep.flags = fl;
  ra.ep.pack_pos = pack_pos;
  ra.ep.rank = rank; ra.ep.n = n_ranks; ra.ep.C = capacity; ra.ep.el = E / n_ranks; ra.ep.T = T;
  return cuda_status(mfi::launch_route(ra, st), "ep_route_dispatch launch");
}

size_t mfi_ep_experts_workspace_bytes(int n_ranks, int capacity, int hidden, int inter,
                                      int local_experts, int top_k) {
  if (n_ranks <= 0 || capacity < 0) return 0;
  return mfi_moe_experts_workspace_bytes(n_ranks * (capacity + 1), hidden, inter, local_experts,
                                         top_k);
}

int mfi_ep_experts_return(const mfi_moe_weights* w, int rank, int n_ranks, int capacity,
                          const void* table, void* flags, uint8_t* recv, void* workspace,
                          size_t workspace_bytes, void* stream) {
  if (!w) return fail(MFI_ERR_ARG, "null weights");
  const int E = w->n_experts, H = w->hidden, Mi = w->inter, k = w->top_k;
  int rc = ep_p2p_check(rank, n_ranks, capacity, H, k);
  if (rc != MFI_OK) return rc;
  if (E <= 0 || E > mfi::kRouteMaxE) return fail(MFI_ERR_ARG, "n_experts must be in [1, 256]");
  if (!layer_uses_tc(H, Mi)) return fail(MFI_ERR_ARG, "hidden and inter must be multiples of 256");
  const int R = n_ranks * (capacity + 1);
  if ((long long)R * k > 16384) return fail(MFI_ERR_ARG, "n_ranks * (capacity + 1) * top_k must be <= 16384");
  if (bad_ptr(table) || bad_ptr(flags) || bad_ptr(recv) || bad_ptr(workspace) || bad_ptr(w->prepared))
    return fail(MFI_ERR_ARG, "null pointer (weights.prepared comes from mfi_moe_prepare)");
  if (reinterpret_cast<uintptr_t>(recv) & 15) return fail(MFI_ERR_ARG, "recv must be 16-byte aligned");
  if (workspace_bytes < mfi_moe_experts_workspace_bytes(R, H, Mi, E, k))
    return fail(MFI_ERR_WORKSPACE, "workspace too small for ep_experts_return");
  ExpertScratch s = carve_experts(workspace, R, H, Mi, E, k);
  cudaStream_t st = as_stream(stream);
  const mfi::EpTable* tb = static_cast<const mfi::EpTable*>(table);
  unsigned* fl = static_cast<unsigned*>(flags);
  // cursors, work counter and readiness counters are zero (workspace zeroed
  // before the first call; each call's combine/return kernel clears them)
  rc = cuda_status(mfi::launch_ep_scatter_wait(tb, fl, recv, rank, n_ranks, capacity, H, k, E,
                                               s.T_pad, s.cursor, s.perm, s.xp, s.xp_atoms,
                                               mfi::device_error_flag(), st),
                   "ep_experts_return scatter launch");
  if (rc != MFI_OK) return rc;
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  mfi::MoeTcLaunch L{};
  L.E = E; L.H = H; L.Mi = Mi; L.grid = sms;
  L.max_chunks = s.max_chunks;
  L.prepared = static_cast<const uint8_t*>(w->prepared);
  L.counts = s.cursor; L.perm = s.perm;
  L.rows = E * s.T_pad;
  L.xp = s.xp; L.xp_atoms = s.xp_atoms; L.hp = s.hp; L.hp_atoms = s.hp_atoms; L.yd = s.yd;
  L.err = mfi::device_error_flag();
  L.pdl = true;
  L.pf_bytes = prefetch_bytes((long long)R * k, E, true);
  L.queue = s.cursor + E;
  L.ready = reinterpret_cast<unsigned*>(s.cursor + E + 1);
  rc = cuda_status(mfi::launch_moe_tc(L, st), "ep_experts_return experts launch");
  if (rc != MFI_OK) return rc;
  return cuda_status(mfi::launch_ep_combine_return(tb, fl, s.yd, recv, rank, n_ranks, capacity, H,
                                                   k, E, s.cursor, int(s.zero_words),
                                                   mfi::device_error_flag(), st),
                     "ep_experts_return combine launch");
}

int mfi_ep_unpack_wait(int n_ranks, int capacity, int hidden, int T, void* flags, const float* ret,
                       const int32_t* pack_pos, float* out, void* stream) {
  if (n_ranks <= 0 || n_ranks > mfi::kEpMaxRanks) return fail(MFI_ERR_ARG, "n_ranks must be in [1, 64]");
  if (capacity < 0 || T < 0 || T > capacity) return fail(MFI_ERR_ARG, "T must be in [0, capacity]");
  if (hidden <= 0) return fail(MFI_ERR_ARG, "hidden must be positive");
  if (bad_ptr(flags) || bad_ptr(ret) || (T > 0 && (bad_ptr(pack_pos) || bad_ptr(out))))
    return fail(MFI_ERR_ARG, "null pointer");
  if (hidden % 4 || (reinterpret_cast<uintptr_t>(ret) & 15) || (reinterpret_cast<uintptr_t>(out) & 15))
    return fail(MFI_ERR_ARG, "ret and out must be 16-byte aligned, hidden a multiple of 4");
  return cuda_status(mfi::launch_ep_unpack_wait(static_cast<unsigned*>(flags), ret, pack_pos, T,
                                                n_ranks, capacity, hidden, out,
                                                mfi::device_error_flag(), as_stream(stream)),
                     "ep_unpack_wait launch");
}

}  // extern "C"
