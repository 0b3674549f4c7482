/*
 * moe_fp4.h — C ABI of libmoe_fp4.so, the B200 (sm_100a) MXFP4 grouped-MoE
 * expert path.
 *
 * Every entry point takes plain device pointers, sizes and a CUDA stream
 * (cudaStream_t / CUstream passed as void*), launches asynchronously on that
 * stream and returns an MFI_* status code.  On failure the message of
 * mfi_last_error() (per thread) says what was wrong; argument errors use the
 * reference binding's TORCH_CHECK wording where one exists.  Nothing here
 * allocates device memory: operations that need scratch take a caller-owned
 * workspace whose size the matching *_workspace_bytes() function returns.
 *
 * Data formats (reference quant/fp4_format.py:17-148,
 * quant/quantize_mxfp4.py:110-160):
 *   packed  uint8 (rows, Kp/2)  two E2M1 nibbles per byte, element 2k in the
 *                               low nibble of byte k
 *   scales  uint8 (rows, Kp/32) E8M0 codes, value 2^(code-127)
 *   Kp = ceil(K/32)*32; padding elements are zero nibbles.
 *
 * Citations are paths inside the reference project
 * (shuimenwang/moe_fused_inference).
 */
#ifndef MOE_FP4_H
#define MOE_FP4_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum mfi_status {
  MFI_OK = 0,
  MFI_ERR_ARG = 1,        /* invalid argument (shape, pointer, size)          */
  MFI_ERR_CUDA = 2,       /* a CUDA call or kernel launch failed               */
  MFI_ERR_WORKSPACE = 3,  /* caller workspace smaller than *_workspace_bytes() */
};

/* Element type codes for activation inputs. */
enum mfi_dtype { MFI_F32 = 0, MFI_F16 = 1, MFI_BF16 = 2 };

/* Message describing the last failed call on this host thread ("" if none). */
const char* mfi_last_error(void);

/* Library ABI version (bumped when a signature changes). */
int mfi_version(void);

/* Device error flag of the current device: 0 while healthy, else the code of
 * the first failure any kernel reported since it was last cleared — a bounded
 * wait (2 s) that timed out, after which that kernel's CTA stopped early and
 * its outputs are incomplete (1 load producer, 2 MMA issuer, 3 epilogue,
 * 4 down item waiting for its h rows, 6 router rows, 7 missing dispatch from
 * a peer, 8 missing return from a peer), or invalid data (4 expert id out of
 * range, 5 expert region overflow: a repeated id or counters not zeroed,
 * 9 a received exchange block whose row count lies outside [0, capacity],
 * treated as empty).
 * The flag only reports: a set flag does not stop later calls.  Synchronous;
 * clear != 0 resets it.  Returns -1 if the flag cannot be read. */
int mfi_device_error(int clear);

/* Exhaustive self-check of the library's own fp32 arithmetic on the current
 * device, over all 2^32 bit patterns: the SwiGLU quotient g / (1 + expf(-g))
 * (computed by Markstein's division) against CUDA's correctly rounded
 * division, and the E2M1 rounding of |x| read from its bits against the
 * threshold definition (quant/fp4_format.py:24-46).  Asynchronous on
 * `stream`; out (device, 4 words, 8-byte aligned) receives the mismatch
 * counts of the two checks and the smallest mismatching bit pattern of each
 * (all ones when there is none).  A few milliseconds on a B200. */
int mfi_selftest_numerics(unsigned long long* out, void* stream);

/* ------------------------------------------------------------------------
 * Quantisers
 * ------------------------------------------------------------------------ */

/* Activation quantiser: bf16 x (M, K) row-major -> xq (M, Kp/2), xsc (M, Kp/32).
 * Replaces mxfp4v2::launch_prequant_v2 (src/ext/mxfp4_decode.cu:304-309), bound
 * by prequant() (src/ext/mxfp4_decode_binding.cpp:65-81).  Every byte of xq
 * and xsc is written (padding included), so no zero-fill is needed.  Bit-exact
 * with quantize_expert_tensor (quant/quantize_mxfp4.py:110-160). */
int mfi_prequant(const void* x_bf16, uint8_t* xq, uint8_t* xsc, int M, int K, int Kp,
                 void* stream);

/* General row quantiser: x of dtype MFI_* with row stride ld_x elements.
 * half_roundtrip = 1 rounds every element through fp16 first, the cast the
 * reference's mxfp4_linear binding applies to non-half inputs
 * (src/ext/mxfp4_binding.cpp:31).  Columns [K, Kp) are zero padding (Kp a
 * multiple of 32, Kp >= K).  Also the bit-exact device form of the weight
 * quantiser quantize_expert_tensor (quant/quantize_mxfp4.py:110-160). */
int mfi_quantize_rows(const void* x, int dtype, long long ld_x, int half_roundtrip,
                      uint8_t* xq, uint8_t* xsc, int M, int K, int Kp, void* stream);

/* ------------------------------------------------------------------------
 * GEMMs (y = A . W^T, fp32 out)
 * ------------------------------------------------------------------------ */

/* Pre-quantised linear: y (M, N) fp32 = Q(x) . W^T.  M >= 64 runs on the
 * tcgen05 tensor cores and needs mfi_lin_pq_workspace_bytes() of workspace
 * (0 below that, where a CUDA-core GEMV runs and workspace may be NULL).
 * Replaces mxfp4v2::launch_lin_pq_v2 (src/ext/mxfp4_decode.cu:311-318), bound
 * by lin_pq() (src/ext/mxfp4_decode_binding.cpp:84-98). */
size_t mfi_lin_pq_workspace_bytes(int M, int N, int Kp);
int mfi_lin_pq(const uint8_t* xq, const uint8_t* xsc, const uint8_t* wp, const uint8_t* wsc,
               float* y, int M, int N, int K, int Kp, void* workspace, size_t workspace_bytes,
               void* stream);

/* Linear with on-the-fly activation quantisation: x (M, ld_x) of dtype
 * MFI_* (non-half inputs rounded through fp16 like the reference binding),
 * columns [0, min(ld_x, Kp)) quantised per 32 block and the rest zero,
 * multiplied by the packed W (N, Kp/2)/(N, Kp/32) -> y (M, N) fp32.
 * Replaces mxfp4::launch_mxfp4_linear (src/ext/mxfp4_linear.cu:200-206),
 * bound by forward() (src/ext/mxfp4_binding.cpp:21-45). */
size_t mfi_linear_workspace_bytes(int M, int N, int Kp);
int mfi_mxfp4_linear(const void* x, int dtype, int ld_x, const uint8_t* wp, const uint8_t* wsc,
                     float* y, int M, int N, int Kp, void* workspace, size_t workspace_bytes,
                     void* stream);

/* Allocation-free mxfp4_linear (no counterpart in the reference: its
 * bindings always allocate through torch).  For callers that cannot allocate
 * device memory — a plugin whose host program owns all GPU memory, an FFI
 * caller without the framework's allocator, a hot path that must not call
 * cudaMalloc — the scratch of mfi_mxfp4_linear comes from a 4 MiB static
 * device array inside the library instead of a caller workspace.  Same
 * arguments and results as mfi_mxfp4_linear minus the workspace.  Shapes with
 * mfi_linear_workspace_bytes(M, N, Kp) > 4 MiB are rejected with
 * MFI_ERR_WORKSPACE.  The first call on each device looks up the array's
 * device address and should happen before any stream capture; the address is
 * kept for the process, so after cudaDeviceReset() on a device this entry
 * point must not be called there again.  All calls on
 * a device share the array (it keeps the last call's contents; nothing needs
 * to start at zero), so calls that overlap on the GPU race: serialise them.
 * Allocates nothing (no cudaMalloc, cudaFree or allocating library call). */
int mfi_mxfp4_linear_noalloc(const void* x, int dtype, int ld_x, const uint8_t* wp,
                             const uint8_t* wsc, float* y, int M, int N, int Kp, void* stream);

/* ------------------------------------------------------------------------
 * Grouped MoE operators behind device pointer tables
 * ------------------------------------------------------------------------ */

/* Grouped gate/up.  wp_tab/wsc_tab: device arrays of 2*E*M pointers in the
 * reference order [token m: gate e0..e(E-1), up e0..e(E-1)]; gu (M*E, 2N) fp32
 * with gate in columns [0,N) and up in [N,2N).  Entries that point at the
 * same weight share one pass over it.
 * Replaces mxfp4v2::launch_gateup_v2 (src/ext/mxfp4_decode.cu:320-328), bound
 * by moe_gateup()/moe_gateup_tab() (src/ext/mxfp4_decode_binding.cpp:101-120,
 * 177-192). */
size_t mfi_moe_gateup_workspace_bytes(int E, int M);
int mfi_moe_gateup(const uint8_t* xq, const uint8_t* xsc, const uint8_t* const* wp_tab,
                   const uint8_t* const* wsc_tab, float* gu, int E, int M, int N, int K, int Kp,
                   void* workspace, size_t workspace_bytes, void* stream);

/* Fused SwiGLU + down.  gu (M*E, 2K) fp32 from mfi_moe_gateup; h = silu(g)*u
 * in fp32, requantised per 32 block; yd (M*E, N) fp32 = Q(h) . Wd^T with
 * wp_tab/wsc_tab of E*M pointers in order m*E + e.
 * Replaces mxfp4v2::launch_down_silu_v2 (src/ext/mxfp4_decode.cu:330-338),
 * bound by moe_down()/moe_down_tab() (src/ext/mxfp4_decode_binding.cpp:123-142,
 * 194-209). */
size_t mfi_moe_down_workspace_bytes(int E, int M, int K);
int mfi_moe_down(const float* gu, const uint8_t* const* wp_tab, const uint8_t* const* wsc_tab,
                 float* yd, int E, int M, int N, int K, int Kp, void* workspace,
                 size_t workspace_bytes, void* stream);

/* Top-k combine: out[m, c] = sum_{e < min(E, 8)} w[m, e] * yd[(m*E + e)*ystride + c]
 * in fp32, sequential in e (the reference kernel sums at most 8 slots).
 * Replaces mxfp4v2::launch_combine_v2 (src/ext/mxfp4_decode.cu:340-344), bound
 * by moe_combine() (src/ext/mxfp4_decode_binding.cpp:145-158). */
int mfi_moe_combine(const float* yd, int ystride, const float* w, int E, float* out, int M, int N,
                    void* stream);

/* ------------------------------------------------------------------------
 * FP8 (E4M3) KV cache and single-sequence decode attention (head_dim 128)
 * ------------------------------------------------------------------------ */

/* KV write: k, v bf16 (M, Hkv, D) -> one byte per element at position
 * *dpos + m of kvk, kvv (max_pos, Hkv, D); dpos is a device int32 read by the
 * kernel (graph replay with a moving position), rows past max_pos or a
 * negative base are skipped.  k_scale = v_scale = NULL: the reference's own
 * encoder bit for bit (half-away-from-zero mantissa rounding, values below
 * 2^-6 as round(|x| * 64), saturation to 0x7F).  Per-KV-head fp32 scales
 * (Hkv each): the standard e4m3fn encoding of x / scale (round to nearest
 * even, saturating at +-448).  k, v 16-byte, kvk, kvv 8-byte aligned; D a
 * multiple of 8.
 * Replaces mxfp4v2::launch_kvwrite_v2 (src/ext/mxfp4_decode.cu:485-490), bound
 * by kv_write() (src/ext/mxfp4_decode_binding.cpp:161-173). */
int mfi_kv_write(const void* k, const void* v, uint8_t* kvk, uint8_t* kvv, const int32_t* dpos,
                 int M, int Hkv, int D, int max_pos, const float* k_scale, const float* v_scale,
                 void* stream);

/* Decode attention of M query rows of one sequence: q bf16 (M, Hq, D) (RoPE
 * applied), row m attending to positions [0, *dpos + m] of the FP8 cache
 * kvk, kvv (max_pos, Hkv, D), query head h reading KV head h / (Hq / Hkv);
 * o fp32 (M, Hq, D) = softmax(q k^T / sqrt(D)) v with the cache decoded by the
 * reference's decoder (scales NULL) or as standard e4m3fn times the per-head
 * scales.  A row with no live position gets zeros.  D must be 128 and
 * Hq / Hkv <= 16.  q, kvk, kvv, o and the workspace must be 16-byte
 * aligned.  The positions are split over the grid; the partial results need
 * mfi_attn_decode_workspace_bytes() of workspace.
 * Replaces mxfp4v2::launch_attn_decode_v2 (src/ext/mxfp4_decode.cu:424-437),
 * bound by attn_decode() (src/ext/mxfp4_decode_binding.cpp:213-230), whose
 * score buffer `sc` this library does not need. */
size_t mfi_attn_decode_workspace_bytes(int M, int Hq, int Hkv, int D, int max_pos);
int mfi_attn_decode(const void* q, const uint8_t* kvk, const uint8_t* kvv, const int32_t* dpos,
                    float* o, int M, int Hq, int Hkv, int D, int max_pos, const float* k_scale,
                    const float* v_scale, void* workspace, size_t workspace_bytes, void* stream);

/* The same for n_seq sequences at the same base position in one launch (no
 * reference counterpart: the reference decodes one sequence per call):
 * sequence s has q rows [s*M, (s+1)*M) of q (n_seq*M, Hq, D), its cache at
 * kvk/kvv + s * kv_seq_stride bytes (kv_seq_stride >= max_pos*Hkv*D, a
 * multiple of 16) and o rows [s*M, (s+1)*M). */
size_t mfi_attn_decode_batched_workspace_bytes(int n_seq, int M, int Hq, int Hkv, int D,
                                               int max_pos);
int mfi_attn_decode_batched(const void* q, const uint8_t* kvk, const uint8_t* kvv,
                            long long kv_seq_stride, const int32_t* dpos, float* o, int n_seq,
                            int M, int Hq, int Hkv, int D, int max_pos, const float* k_scale,
                            const float* v_scale, void* workspace, size_t workspace_bytes,
                            void* stream);

/* ------------------------------------------------------------------------
 * Fused device-routed MoE layer (no reference counterpart as a single call:
 * it fulfils the reference's unimplemented K1/K2/K3 stubs
 * src/kernels/k1_router_topk_sort.cu, k2_mxfp4_grouped_gemm.cu,
 * k3_deterministic_combine.cu, and performs model_runner_v2's MoE block
 * runtime/model_runner_v2.py:183-208 / :266-290 without host round trips).
 * ------------------------------------------------------------------------ */
typedef struct mfi_moe_weights {
  const uint8_t* gate_wp;   /* (E, inter, hidden/2)  */
  const uint8_t* gate_sc;   /* (E, inter, hidden/32) */
  const uint8_t* up_wp;     /* (E, inter, hidden/2)  */
  const uint8_t* up_sc;     /* (E, inter, hidden/32) */
  const uint8_t* down_wp;   /* (E, hidden, inter/2)  */
  const uint8_t* down_sc;   /* (E, hidden, inter/32) */
  const uint8_t* router_wp; /* (E, hidden/2)         */
  const uint8_t* router_sc; /* (E, hidden/32)        */
  int n_experts;            /* E <= 256                               */
  int hidden;               /* multiple of 32, <= 4096                */
  int inter;                /* multiple of 32                         */
  int top_k;                /* 1..min(E, 32)                          */
  const void* prepared;     /* blocks from mfi_moe_prepare, or NULL       */
  const float* logit_bias;  /* [E] fp32 added to the router logits before
                               top-k (e.g. a synthetic load skew), or NULL */
  /* RMSNorm fused into the router (the MoE block's post-attention layernorm,
   * reference runtime/model_runner.py:20-25 called at
   * runtime/model_runner_v2.py:183): with norm_weight (bf16 [hidden]) set,
   * x is the residual stream and every token row is normalised before it is
   * quantised: r = 1 / sqrt(float(ss) / hidden + norm_eps), ss the row's sum
   * of squares accumulated in fp64, each element bf16(bf16(x * r) * weight).
   * NULL: x is quantised as given. */
  const void* norm_weight;
  float norm_eps;
} mfi_moe_weights;

/* Tensor-core form of the layer's expert weights.  When hidden and inter are
 * multiples of 256, mfi_moe_layer runs its expert GEMMs on the tcgen05 tensor
 * cores and needs `prepared`: a caller-owned buffer of
 * mfi_moe_prepared_bytes() (the size of the packed expert weights and scales)
 * filled once per weight set by mfi_moe_prepare — the weights cut into
 * per-stage 128-row x 256-K blocks stored in shared-memory order with their
 * E8M0 scale atoms, so each pipeline stage is one contiguous bulk copy.
 * Other shapes use a CUDA-core path and ignore it. */
size_t mfi_moe_prepared_bytes(int n_experts, int hidden, int inter);
int mfi_moe_prepare(const mfi_moe_weights* w, void* prepared, size_t prepared_bytes, void* stream);

/* x: bf16 (T, hidden) -> out fp32 (T, hidden); topi int32 (T, top_k) and
 * topw fp32 (T, top_k) receive the routing; logits fp32 (T, E) may be NULL
 * (with logit_bias set they hold the biased logits top-k ranked).
 * Decode sizes (T * top_k <= 4096) run the decode kernels; larger T, up to
 * T * top_k <= 262144, runs the prefill path of mfi_moe_layer_prefill
 * (needs hidden and inter multiples of 256).  Both combine a token's slots
 * in slot order with unfused fp32 multiply and add. */
size_t mfi_moe_layer_workspace_bytes(int T, int hidden, int inter, int n_experts, int top_k);
/* The decode tensor-core path keeps per-call counters in the workspace (so a
 * layer call needs no memset node): initialise a workspace once with
 * mfi_moe_layer_init_workspace for its (T, shape) and pass it unchanged to
 * every call with that T; each call leaves the counters zeroed.  A workspace
 * that was not initialised gives wrong results and device error 5, never an
 * out-of-bounds write. */
int mfi_moe_layer_init_workspace(void* workspace, size_t workspace_bytes, int T, int hidden,
                                 int inter, int n_experts, int top_k, void* stream);
int mfi_moe_layer(const mfi_moe_weights* w, const void* x_bf16, int T, float* out, int32_t* topi,
                  float* topw, float* logits, void* workspace, size_t workspace_bytes,
                  void* stream);

/* As mfi_moe_layer, recording six caller-created cudaEvent_t (passed as void*)
 * on the stream at the stage boundaries, for per-kernel timing:
 * tensor-core decode shapes: [0] start, [1] after quantise + route (which
 * also writes each token's row into its experts' regions), [2] = [1],
 * [3] = [4] after the expert GEMMs (gate/up, SwiGLU requant and down run as
 * one persistent launch), [5] after the combine; the prefill path: [0]
 * start, [1] after quantise + route, [2] after the row scatter, [3] = [4]
 * after the expert GEMMs, [5] after the combine; other shapes: [2] after the
 * gate/up GEMV, [3] after SwiGLU requantisation, [4] after the down GEMV. */
int mfi_moe_layer_ex(const mfi_moe_weights* w, const void* x_bf16, int T, float* out,
                     int32_t* topi, float* topw, float* logits, void* workspace,
                     size_t workspace_bytes, void* const* events, int n_events, void* stream);

/* Prefill path for any T >= 1 (T * top_k <= 262144): router with count-based
 * compact placement (per-expert rows rounded up to 128-token tiles), then one
 * persistent tcgen05 launch of 128-token x 128-row tiles — gate/up with the
 * SwiGLU requantisation in the epilogue, down storing per-(token, slot) rows
 * — and the top-k combine.  Needs `prepared`. */
size_t mfi_moe_layer_prefill_workspace_bytes(int T, int hidden, int inter, int n_experts,
                                             int top_k);
int mfi_moe_layer_prefill(const mfi_moe_weights* w, const void* x_bf16, int T, float* out,
                          int32_t* topi, float* topw, float* logits, void* workspace,
                          size_t workspace_bytes, void* stream);

/* ------------------------------------------------------------------------
 * The layer in two halves, for expert parallelism (no reference counterpart:
 * the reference runs on one GPU; the halves are its route step
 * runtime/model_runner_v2.py:183-194 and its expert step :195-208).
 * ------------------------------------------------------------------------ */

/* Quantise bf16 x (T, hidden) into xq (T, hidden/2) / xsc (T, hidden/32)
 * (16- and 4-byte aligned) and route it with the router of `w`: topi int32
 * (T, top_k), topw fp32 (T, top_k), logits fp32 (T, E) or NULL.  Bit-identical
 * to the routing of mfi_moe_layer.  Only router_wp/router_sc, n_experts,
 * hidden and top_k of `w` are read. */
int mfi_moe_route(const mfi_moe_weights* w, const void* x_bf16, int T, uint8_t* xq, uint8_t* xsc,
                  int32_t* topi, float* topw, float* logits, void* stream);
/* mfi_moe_route with scratch for the tensor-core router that prefill-sized
 * batches use (T >= 512 tokens, 128 experts); mfi_moe_route_workspace_bytes
 * gives its size (0 when it does not apply; the workspace, 256-byte aligned,
 * may then be NULL).  Same results as mfi_moe_route. */
size_t mfi_moe_route_workspace_bytes(int T, int hidden, int n_experts);
int mfi_moe_route_ex(const mfi_moe_weights* w, const void* x_bf16, int T, uint8_t* xq,
                     uint8_t* xsc, int32_t* topi, float* topw, float* logits, void* workspace,
                     size_t workspace_bytes, void* stream);

/* Expert compute on R pre-quantised, pre-routed rows:
 *   out[r] = sum over j < top_k with sel[r][j] >= 0, in slot order, of
 *            selw[r][j] * down_e(swiglu(gate_e(x_r), up_e(x_r))),  e = sel[r][j]
 * with each product and partial sum rounded to fp32 (the combine of
 * mfi_moe_combine).  Row r of xq / xsc / sel / selw / out starts at r * *_ld
 * (bytes for xq and xsc, elements otherwise); xq and out rows 16-byte
 * aligned, xsc rows 4-byte aligned.  sel entries are expert ids of `w` (0..n_experts-1) or
 * -1; an id must not repeat within a row (the device error flag then reads 5;
 * an id >= n_experts reads 4 and is skipped).  Needs hidden and inter to be
 * multiples of 256 and `w->prepared`; router fields are not read.
 * R * top_k <= 262144.  Up to 16384 pairs the decode kernels run (fp32 rows
 * of y); beyond, the prefill kernels of mfi_moe_layer (128-row expert tiles,
 * each expert's output row rounded to bf16 before the combine, as the
 * reference's prefill does, runtime/model_runner_v2.py:119) — the expert-
 * parallel prefill.  Rows whose slots are all -1 get zeros. */
size_t mfi_moe_experts_workspace_bytes(int R, int hidden, int inter, int n_experts, int top_k);
int mfi_moe_experts(const mfi_moe_weights* w, const uint8_t* xq, long long xq_ld,
                    const uint8_t* xsc, long long xsc_ld, const int32_t* sel, long long sel_ld,
                    const float* selw, long long selw_ld, int R, float* out, long long out_ld,
                    void* workspace, size_t workspace_bytes, void* stream);

/* ------------------------------------------------------------------------
 * Expert-parallel exchange (no reference counterpart).  N ranks each own
 * experts_per_rank consecutive experts (global expert e lives on rank
 * e / experts_per_rank).  A send buffer holds one block per destination rank
 * of (capacity + 1) rows of mfi_ep_row_bytes() bytes: a header row whose
 * first int32 is the block's row count, then one row per (token,
 * destination) pair:
 *   [0, hidden/2) packed nibbles | [hidden/2, +hidden/32) E8M0 codes |
 *   int32 token, 3 pad | top_k int32 local expert ids (-1 = other rank) |
 *   top_k fp32 routing weights | zero padding to a multiple of 16 bytes
 * Exchanging the blocks with an equal-split all-to-all needs no host
 * synchronisation; the receiver runs mfi_ep_mask_recv and then
 * mfi_moe_experts over all n_ranks * (capacity + 1) rows (xq at row offset 0,
 * xsc at hidden/2, sel and selw at the offsets above, all with stride
 * row_bytes), returns the fp32 rows with a second all-to-all, and the source
 * sums them with mfi_ep_unpack.
 * ------------------------------------------------------------------------ */

/* Row size in bytes (0 for invalid arguments: hidden % 128, top_k 1..32). */
int mfi_ep_row_bytes(int hidden, int top_k);

/* Pack routed tokens (xq/xsc/topi/topw of mfi_moe_route) into `send`.
 * counts: int32 device scratch [n_ranks]; pack_pos: int32 (T, n_ranks)
 * receives each pair's row in its destination block (-1: none).
 * capacity >= T; n_ranks <= 64. */
int mfi_ep_pack(const uint8_t* xq, const uint8_t* xsc, const int32_t* topi, const float* topw,
                int T, int hidden, int top_k, int n_ranks, int experts_per_rank, int capacity,
                int32_t* counts, uint8_t* send, int32_t* pack_pos, void* stream);

/* Mark the header row and the unused rows of every received block as having
 * no local expert (all ids -1), reading each block's count from its header. */
int mfi_ep_mask_recv(uint8_t* recv, int n_ranks, int capacity, int hidden, int top_k,
                     void* stream);

/* out[t] (fp32, hidden) = sum over ranks d = 0..n_ranks-1 in order, where
 * pack_pos[t][d] >= 0, of row 1 + pack_pos[t][d] of returned block d
 * (ret: fp32 [n_ranks][capacity + 1][hidden]). */
int mfi_ep_unpack(const float* ret, const int32_t* pack_pos, int T, int n_ranks, int capacity,
                  int hidden, float* out, void* stream);

/* ------------------------------------------------------------------------
 * Expert parallelism over peer memory (no reference counterpart).  Instead of
 * two all-to-alls, the router stores each token's row straight into the
 * receive buffer of every rank that owns one of its experts (NVLink stores
 * through CUDA IPC mappings) and raises a flag there; the expert side answers
 * with the weighted sums of its slots stored straight into the source's
 * return buffer.  Flags carry a call id (the rank's completed-call epoch + 1,
 * kept in its flag area), so no flag is ever reset and the whole exchange can
 * be captured in a CUDA graph.  Every wait is bounded (2 s; the device error
 * flag then reads 7 for a missing dispatch, 8 for a missing return).
 *
 * Per rank, in memory the peers map (e.g. one mfi_ipc_alloc block):
 *   recv   mfi_ep_recv_bytes()  block s = rows from rank s, same row layout
 *                               as the all-to-all exchange above
 *   ret    mfi_ep_ret_bytes()   block d = fp32 rows returned by rank d
 *   flags  mfi_ep_flag_bytes()  zero before the first call
 * Each rank calls, in order on one stream, for every layer call:
 *   mfi_ep_route_dispatch, mfi_ep_experts_return, mfi_ep_unpack_wait.
 * All ranks must make the same sequence of calls with the same capacity.
 * ------------------------------------------------------------------------ */

/* Device memory for peer mapping: cudaMalloc'd and zeroed (synchronous).
 * These, with mfi_ep_table_set, are the only calls that allocate or copy
 * synchronously; they are meant for setup. */
int mfi_ipc_alloc(size_t bytes, void** ptr);
int mfi_ipc_free(void* ptr);
/* 64-byte CUDA IPC handle of an mfi_ipc_alloc block / open a peer's handle. */
int mfi_ipc_handle(const void* ptr, void* handle);
int mfi_ipc_open(const void* handle, void** ptr);
int mfi_ipc_close(void* ptr);
/* Stream-ordered copy between device (or host) buffers (cudaMemcpyDefault),
 * for inspecting exchange buffers that have no torch tensor. */
int mfi_copy_async(void* dst, const void* src, size_t bytes, void* stream);

size_t mfi_ep_flag_bytes(void);
size_t mfi_ep_recv_bytes(int n_ranks, int capacity, int hidden, int top_k);
size_t mfi_ep_ret_bytes(int n_ranks, int capacity, int hidden);
/* Peer table: device buffer of mfi_ep_table_bytes() holding, for d < n_ranks,
 * rank d's recv, ret and flags addresses as seen from this rank (this rank's
 * own at d = rank).  Written synchronously. */
size_t mfi_ep_table_bytes(void);
int mfi_ep_table_set(void* table, int n_ranks, void* const* recv, void* const* ret,
                     void* const* flags);

/* Route T <= capacity tokens (x bf16 (T, hidden)) with the router of `w`
 * (n_experts divisible by n_ranks; rank d owns experts [d*E/n, (d+1)*E/n))
 * and send them: topi/topw as mfi_moe_route, pack_pos int32 (T, n_ranks) =
 * each token's row in its block at rank d, or -1. */
int mfi_ep_route_dispatch(const mfi_moe_weights* w, const void* x_bf16, int T, int rank,
                          int n_ranks, int capacity, const void* table, void* flags,
                          int32_t* topi, float* topw, int32_t* pack_pos, void* stream);

/* Wait for every rank's dispatch, run the local experts (`w`: this rank's
 * E/n experts, prepared) on the received rows and send each row's weighted
 * slot sum back to its source.  n_ranks * (capacity + 1) * top_k <= 16384.
 * The workspace keeps counters between calls: zero it before the first call
 * and pass the same one, unchanged, to every call of this exchange (each call
 * leaves its counters at zero, as mfi_ep_unpack_wait does for the flags). */
size_t mfi_ep_experts_workspace_bytes(int n_ranks, int capacity, int hidden, int inter,
                                      int local_experts, int top_k);
int mfi_ep_experts_return(const mfi_moe_weights* w, int rank, int n_ranks, int capacity,
                          const void* table, void* flags, uint8_t* recv, void* workspace,
                          size_t workspace_bytes, void* stream);

/* Wait for every rank's return and sum, in rank order, out[t] (fp32
 * (T, hidden)) from this rank's ret buffer; closes the call. */
int mfi_ep_unpack_wait(int n_ranks, int capacity, int hidden, int T, void* flags, const float* ret,
                       const int32_t* pack_pos, float* out, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* MOE_FP4_H */
