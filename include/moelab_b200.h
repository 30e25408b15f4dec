/*
 * moelab_b200 - C ABI of the B200-native (sm_100a) quantized MoE-layer forward.
 *
 * Drop-in boundary for moe-lab's hot path. moe-lab (Tigerly1/moe-lab) has no native library: its boundary is
 * the Python variant contract `prepare / run(state, x, idx, wts[, act]) / dequant` driven by
 * moelab/torch_backend.py:103-126 and moelab/worker.py:33-43, plus the layer composition of
 * moelab/e2e.py:51-69 (router -> run -> shared experts). Each entry point below names the reference interface
 * it replaces. All pointers are device pointers unless stated; every call is asynchronous on `stream`,
 * allocates nothing and returns MOEB_OK (0) or an error code with a message from moeb_last_error().
 *
 * Weight layout (the B200 layout, produced by moeb_quantize_* or by moeb_*_from_mlx from mlx's layout; the same
 * byte counts as mlx's [E][N][K/8] codes): each projection is a sequence of 16-row blocks (the E*N rows of all
 * experts, expert-major, N a multiple of 16), each block a sequence of its K/64 groups of 64 inputs, so one
 * (row block, group) is a contiguous unit. For weight row r (0 <= r < E*N) and input k (0 <= k < K), with
 * rb = r / 16, rr = r % 16, g = k / 64, j = (k % 64) / 8 (the 8-input word inside the group), e = k % 8:
 *   int4 codes q (uint32): word ((rb*(K/64) + g)*32 + lane)*4 + (rr/8)*2 + j%2, lane = (rr%8)*4 + j/2 (the lane of a
 *       warp whose m16n8k16 A fragment holds it); inside the word, input e sits at nibble e/2 if e is even and at
 *       nibble 4 + e/2 if odd (low nibble first);
 *   int4 scale|bias sb (uint32: bf16 scale in bits 0-15, bf16 bias in bits 16-31; w = scale * q + bias):
 *       word ((rb*(K/64) + g)*8 + rr%8)*2 + rr/8;
 *   MXFP4 codes q: as int4 (E2M1 codes: sign bit 3, magnitude {0, .5, 1, 1.5, 2, 3, 4, 6} in bits 0-2);
 *   MXFP4 scales sc (uint8 E8M0, one per 32 inputs, h = k / 32): byte (((rb*(K/64) + h/2)*8 + rr%8)*2 + rr/8)*2 + h%2.
 *   gate/up: N = f, K = d; down: N = d, K = f. Row counts (E*N) and K are multiples of 16 and 64 (MOEB_EINVAL
 *   otherwise). Activations x, y, residual: bf16 [T][d], row-major.
 */
#ifndef MOELAB_B200_H
#define MOELAB_B200_H

#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

#ifndef __CUDA_RUNTIME_H__
typedef struct CUstream_st *cudaStream_t;
#endif

#define MOEB_VERSION 1

/* status codes */
#define MOEB_OK 0
#define MOEB_EINVAL 1   /* bad shape or argument */
#define MOEB_ELAUNCH 2  /* CUDA launch / runtime error */
#define MOEB_ETIMEOUT 3 /* a bounded device wait gave up */
#define MOEB_EUNSUP 4   /* unsupported format / configuration */

/* dispatcher policies (reference: custom_wins / load_max, moelab/variants/mlx/metal_q4_moe.py:42-46,
 * metal_mxfp4_moe.py:468-471) */
#define MOEB_POLICY_AUTO 0    /* choose by load = T*k/E */
#define MOEB_POLICY_SLOTS 1   /* one tile per slot, no routing step (decode) */
#define MOEB_POLICY_TILES8 2  /* slots grouped by expert, tiles of <= 8 slots */
#define MOEB_POLICY_TILES16 3 /* tiles of <= 16 slots */
#define MOEB_POLICY_TILES8_RING 4  /* tiles of <= 8 slots, weights streamed by TMA into a per-warp ring */
#define MOEB_POLICY_TILES16_RING 5 /* tiles of <= 16 slots, TMA ring */
#define MOEB_POLICY_TC 6 /* tiles of 32 / 64 / 128 / 192 / 256 slots on tcgen05 tensor cores (d and f multiples of
                            128) */
#define MOEB_POLICY_TILES24_RING 8 /* tiles of <= 24 slots, TMA ring */
#define MOEB_POLICY_DECODE 7 /* decode (<= 16 slots) as ONE cooperative kernel, one CTA per SM: router, gate/up,
                                down and combine, every CTA's expert weights issued by bulk copies right after
                                routing (opt-in: 24.5 vs 20.7 us for the three decode launches at T=1; SLOTS where
                                its plan does not fit an SM) */

/* device error bits readable with moeb_read_error */
#define MOEB_DEVERR_EXPERT_ID 1u /* an expert id outside [0, E) was given; that slot contributed nothing */
#define MOEB_DEVERR_TIMEOUT 2u

int moeb_version(void);
const char *moeb_last_error(void); /* thread-local message of the last failing call */

/* Scratch for one layer call of up to T tokens (h, per-slot partials, routing tables, counters). The buffer
 * must be zeroed once with moeb_workspace_init before its first use; calls leave the counters zero again.
 * One workspace serves one stream at a time. (Reference: the variant caches its scratch per shape in
 * `state`, moelab/variants/mlx/metal_q4_tiles_v2.py:432-448; here the caller owns it.) */
size_t moeb_workspace_bytes(int T, int d, int f, int E, int k);
int moeb_workspace_init(void *ws, size_t ws_bytes, cudaStream_t stream);
/* Copies the sticky device error word to *out (host) and clears it. Synchronises `stream`. */
int moeb_read_error(void *ws, unsigned *out, cudaStream_t stream);
/* Policy the dispatcher picks for AUTO (host-only, no device work) for a layer whose d and f are multiples of 128:
 * SLOTS up to 16 slots, then by load = T*k/E: TILES8_RING below 8, TILES16_RING below 14, TC from 14. Other
 * shapes get TILES16_RING below 16 and TILES24_RING from 16 where this returns MOEB_POLICY_TC. */
int moeb_policy(int T, int E, int k);

/* --- quantizers: w bf16 [rows][K] -> B200 layout. Replace mx.quantize(w, group_size=64, bits=4) and
 * mx.quantize(w, mode="mxfp4") in prepare() (metal_q4_moe.py:32-35, metal_mxfp4_moe.py:448-451). */
int moeb_quantize_q4(const void *w, long rows, long K, void *q, void *sb, cudaStream_t stream);
int moeb_quantize_mxfp4(const void *w, long rows, long K, void *q, void *sc, cudaStream_t stream);
/* --- fp32 dequantisation in natural element order (the weights the kernels multiply). Replace
 * mx.dequantize in dequant() (metal_q4_moe.py:38-39, metal_mxfp4_moe.py:454-455). */
int moeb_dequant_q4(const void *q, const void *sb, long rows, long K, float *out, cudaStream_t stream);
int moeb_dequant_mxfp4(const void *q, const void *sc, long rows, long K, float *out, cudaStream_t stream);
/* --- mlx state (weight uint32 natural nibble order, bf16 scales / biases or uint8 scales) -> B200 layout.
 * Replaces the state construction from mlx-lm modules (e2e.py:48-49, metal_mxfp4_gptoss.py:100-107). */
int moeb_q4_from_mlx(const void *wq, const void *scales, const void *biases, long rows, long K, void *q,
                     void *sb, cudaStream_t stream);
int moeb_mxfp4_from_mlx(const void *wq, const void *scales, long rows, long K, void *q, void *sc,
                        cudaStream_t stream);

/* --- router: logits = x . gate_w^T (+ gate_b), fp32, fixed summation order; top-k (ties -> lowest id,
 * NaN -> -inf); norm=1: softmax over the top-k, norm=0: full-softmax probabilities; times `scale`.
 * Replaces moelab/router.py:71-80 topk_norm and the stock sequence of e2e.py:56-63 / :171-176 / :136-140.
 * idx int32 [T][k], wts fp32 [T][k], logits fp32 [T][E] (may be NULL). ws: a workspace from
 * moeb_workspace_bytes(T, d, 64, E, k) used by this router alone. */
int moeb_router(const void *x, const void *gate_w, const void *gate_b, int T, int d, int E, int k, int norm,
                float scale, int *idx, float *wts, float *logits, void *ws, size_t ws_bytes, cudaStream_t stream);

/* --- the routing step alone (the tile builder every tiled call runs), for bit-exact checks of its integer work:
 * stable counting sort of the T*k slots (idx int32 [T*k]) by expert. Writes counts[E] (slots per expert; may be
 * NULL), offsets[E] (their exclusive prefix sums; may be NULL), sorted[T*k] (slot ids grouped by expert, each
 * expert's slots in increasing order), tiles[ntiles][4] int32 {expert, start in sorted, n <= nt, 0} (each
 * expert's run cut every nt slots, experts in increasing order; room for T*k + E entries) and *ntiles. Ids
 * outside [0, E) set MOEB_DEVERR_EXPERT_ID and are grouped under expert 0. Replaces the map kernel of
 * moelab/variants/mlx/metal_q4_tiles_v2.py:362-373 (tiles of <= VT consecutive same-expert slots). ws: a workspace
 * of moeb_workspace_bytes(T, 64, 64, E, k) bytes (its counters and error word). */
int moeb_route_tables(const int *idx, int T, int k, int E, int nt, int *counts, int *offsets, int *sorted, int *tiles,
                      int *ntiles, void *ws, size_t ws_bytes, cudaStream_t stream);

/* --- expert forward with given routing: y = sum_j wts[t,j] * (Wd act(Wg x + bg, Wu x + bu) + bd) (+ residual).
 * Replaces the variant run(state, x, idx, wts, act) (metal_q4_moe.py:54-64 dispatcher; contract
 * problem.py:3-10). act: 0 SwiGLU, 1 tanh-GELU GLU, 2 gpt-oss clamped SwiGLU (alpha 1.702, limit 7, up+1).
 * Biases (fp32, NULL = none): bg, bu [E][f], bd [E][d]. residual bf16 [T][d] or NULL. */
int moeb_experts_q4(const void *x, const void *qg, const void *sbg, const void *qu, const void *sbu,
                    const void *qd, const void *sbd, const float *bg, const float *bu, const float *bd,
                    const int *idx, const float *wts, int T, int d, int f, int E, int k, int act, int policy,
                    const void *residual, void *y, void *ws, size_t ws_bytes, cudaStream_t stream);

/* --- the same for MXFP4 experts (E2M1 codes + E8M0 scales; replaces metal_mxfp4_moe.py:474-512 run and, with
 * act = 2 and biases, metal_mxfp4_gptoss.py:128-167 run). The E8M0 scale is folded exactly into bf16 operands. */
int moeb_experts_mxfp4(const void *x, const void *qg, const void *scg, const void *qu, const void *scu,
                       const void *qd, const void *scd, const float *bg, const float *bu, const float *bd,
                       const int *idx, const float *wts, int T, int d, int f, int E, int k, int act, int policy,
                       const void *residual, void *y, void *ws, size_t ws_bytes, cudaStream_t stream);

/* --- full layer call (x, gate weights, packed expert weights + scales + biases, k) -> y: router, routing
 * step, grouped experts and the weighted combine in one stream-ordered sequence: 3 launches for decode calls
 * (router, gate/up, down with the combine), 4 for tiled calls (router with the routing step, gate/up, down, combine),
 * 5 on the tensor-core path (+ the expert-sorted activation gather), 1 with MOEB_POLICY_DECODE.
 * Replaces the patched MoE block call of moelab/e2e.py:51-69 (router + mod.run). idx_out / wts_out may be
 * NULL (then they live in the workspace). stage_events: NULL, or 4 cudaEvent_t recorded before the router,
 * after the router, after gate/up and after down (per-kernel timing; recording them serialises the stages). */
int moeb_layer_q4(const void *x, const void *gate_w, const void *gate_b, int norm, float rscale, const void *qg,
                  const void *sbg, const void *qu, const void *sbu, const void *qd, const void *sbd,
                  const float *bg, const float *bu, const float *bd, int T, int d, int f, int E, int k, int act,
                  int policy, const void *residual, void *y, int *idx_out, float *wts_out,
                  void *const *stage_events, void *ws, size_t ws_bytes, cudaStream_t stream);
/* DeepSeek layer with always-on shared experts (replaces the MoE block of moelab/e2e.py:130-148: routed experts
 * + shared_experts(x), :146-147). The weight arrays hold E routed experts followed by n_shared shared experts of
 * the same width f (a shared MLP of width n*f split along f into n experts). The router picks k of the E routed
 * experts (DeepSeek-V2 greedy: norm = 0, rscale = routed_scaling_factor) and appends the shared ones with weight
 * 1, so the grouped kernels run them with the routed slots and the combine adds them last. idx_out / wts_out
 * are [T][k + n_shared]. k + n_shared <= 32. Workspace: moeb_workspace_bytes(T, d, f, E + n_shared, k + n_shared). */
int moeb_layer_q4_shared(const void *x, const void *gate_w, const void *gate_b, int norm, float rscale, int n_shared,
                         const void *qg, const void *sbg, const void *qu, const void *sbu, const void *qd,
                         const void *sbd, const float *bg, const float *bu, const float *bd, int T, int d, int f, int E,
                         int k, int act, int policy, const void *residual, void *y, int *idx_out, float *wts_out,
                         void *const *stage_events, void *ws, size_t ws_bytes, cudaStream_t stream);
/* MXFP4 layer (gpt-oss: gate_b = router bias, act = 2, expert biases bg/bu/bd). */
int moeb_layer_mxfp4(const void *x, const void *gate_w, const void *gate_b, int norm, float rscale, const void *qg,
                     const void *scg, const void *qu, const void *scu, const void *qd, const void *scd,
                     const float *bg, const float *bu, const float *bd, int T, int d, int f, int E, int k, int act,
                     int policy, const void *residual, void *y, int *idx_out, float *wts_out,
                     void *const *stage_events, void *ws, size_t ws_bytes, cudaStream_t stream);

/* --- expert parallelism over P ranks (one process per GPU; rank r owns experts [r*E/P, (r+1)*E/P)).
 * No counterpart in the reference (moe-lab runs one device); the exchange follows the usual two all-to-all-v
 * steps, done by the caller with NCCL between these calls:
 *   1. moeb_ep_dispatch: stable counting sort of the T*k slots (ids from the router) by owning rank. Writes
 *      send_counts[P], slot_pos[T*k] (send row of each slot, -1 for an invalid id, which also sets
 *      MOEB_DEVERR_EXPERT_ID in ws) and send_rows[T*k][d + 8] bf16: the slot's token row followed by a 16-byte
 *      tail {int32 local expert id, fp32 weight, 0, 0}. Rows for rank p are rows [sum(counts[<p]), +counts[p]).
 *   2. caller: all-to-all of the counts, then all-to-all-v of the rows (row size (d + 8) * 2 bytes).
 *   3. moeb_ep_experts_q4 / _mxfp4 on the R received rows: yp[R][d] fp32 = weight * (W_down h + b_down), the
 *      same per-slot value the single-GPU down kernel produces (workspace: moeb_ep_workspace_bytes).
 *   4. caller: all-to-all-v of yp back to the owners (reverse counts), into back[sum(send_counts)][d].
 *   5. moeb_ep_combine: y[t] = sum over j of back[slot_pos[t*k + j]] in j order, + residual, rounded to bf16
 *      (the single-GPU combine's order and rounding).
 * P <= 32, E % P == 0. */
int moeb_ep_dispatch(const void *x, const int *idx, const float *wts, int T, int d, int k, int E, int P,
                     void *send_rows, int *send_counts, int *slot_pos, void *ws, size_t ws_bytes,
                     cudaStream_t stream);
size_t moeb_ep_workspace_bytes(int R, int d, int f, int E_local);
int moeb_ep_experts_q4(const void *rows, int R, int d, int f, int E_local, const void *qg, const void *sbg,
                       const void *qu, const void *sbu, const void *qd, const void *sbd, const float *bg,
                       const float *bu, const float *bd, int act, int policy, float *yp, void *ws, size_t ws_bytes,
                       cudaStream_t stream);
int moeb_ep_experts_mxfp4(const void *rows, int R, int d, int f, int E_local, const void *qg, const void *scg,
                          const void *qu, const void *scu, const void *qd, const void *scd, const float *bg,
                          const float *bu, const float *bd, int act, int policy, float *yp, void *ws,
                          size_t ws_bytes, cudaStream_t stream);
int moeb_ep_combine(const float *back, const int *slot_pos, int T, int d, int k, const void *residual, void *y,
                    cudaStream_t stream);

/* --- expert parallelism over NVLink peer memory (no host synchronisation, CUDA-graph capturable).
 * Every rank owns one exchange buffer of moeb_ep_p2p_bytes(P, C, d) bytes (C = rows per (source, owner) block,
 * at least the largest T*k of a call), allocated with moeb_ep_ipc_alloc and mapped into every other rank with
 * moeb_ep_ipc_handle / moeb_ep_ipc_open (CUDA IPC, plain peer mappings, no multicast). `peers` is a DEVICE array
 * of the P buffer addresses as seen by this rank (its own included), `self` its own buffer. Per layer call,
 * every rank issues, in this order on one stream (Cs = this call's rows per source block, 0 < Cs <= C, the same
 * on every rank and at least every rank's T*k; Cs = 0 means C: a small Cs keeps the owners' scan of the blocks
 * short for small calls):
 *   1. moeb_ep_p2p_dispatch: plan as moeb_ep_dispatch, then each slot's row + tail is stored straight into its
 *      owner's buffer (block `me`, row slot_pos % C); the owner's flag for this source is released with the
 *      call's epoch (a per-buffer counter every rank advances once per call). slot_pos [T*k] is in capacity
 *      layout (owner * C + row).
 *   2. moeb_ep_p2p_experts_q4: waits (bounded, ~2 s, then MOEB_DEVERR_TIMEOUT) for each source's flag, runs the
 *      grouped kernels on the valid rows (tile mode; padding rows are skipped) and stores each weighted fp32 row
 *      straight into its owner's return block, then releases the owners' return flags.
 *      Workspace: moeb_ep_workspace_bytes(P * C, d, f, E_local). policy: AUTO picks the decode kernels for small
 *      calls, the tcgen05 kernels from 24 rows per local expert (Cs >= 24 * E_local; d, f multiples of 128) and
 *      the warp-specialized tiles in between; moeb_ep_experts_* picks from its R rows as a layer call does.
 *   3. moeb_ep_p2p_combine: waits for the return flags of all P ranks, then y as moeb_ep_combine.
 * The buffers are reused every call without extra synchronisation: a rank sends call n + 1 only after its
 * combine of call n saw every rank's return flag, i.e. after every rank finished reading call n's rows. */
size_t moeb_ep_p2p_bytes(int P, int C, int d);
int moeb_ep_ipc_alloc(size_t bytes, void **ptr);
int moeb_ep_ipc_free(void *ptr);
int moeb_ep_ipc_handle(void *ptr, void *handle /* 64 bytes */);
int moeb_ep_ipc_open(const void *handle, void **ptr);
int moeb_ep_ipc_close(void *ptr);
int moeb_ep_p2p_dispatch(const void *x, const int *idx, const float *wts, int T, int d, int k, int E, int P, int me,
                         int C, int Cs, void *const *peers, void *self, int *send_counts, int *slot_pos,
                         cudaStream_t stream);
int moeb_ep_p2p_experts_q4(void *const *peers, void *self, int P, int me, int C, int Cs, int d, int f, int E_local,
                           const void *qg, const void *sbg, const void *qu, const void *sbu, const void *qd,
                           const void *sbd, const float *bg, const float *bu, const float *bd, int act, int policy,
                           void *ws, size_t ws_bytes, cudaStream_t stream);
int moeb_ep_p2p_combine(void *self, const int *slot_pos, int P, int C, int T, int d, int k, const void *residual,
                        void *y, cudaStream_t stream);
/* Limit of every bounded wait on this rank's exchange buffer (for a peer's dispatch flag or return flag), in
 * seconds; 0 restores the default of 2 s. After the limit a wait records MOEB_DEVERR_TIMEOUT and the call goes on
 * without that peer's rows. Synchronises the stream. */
int moeb_ep_p2p_set_wait_limit(void *self, int P, int C, int d, double seconds, cudaStream_t stream);
/* Sticky error bits of the exchange buffer (a wait that gave up); synchronises the stream, clears them. */
int moeb_ep_p2p_read_error(void *self, int P, int C, int d, unsigned *out, cudaStream_t stream);

/* --- Measurement probes (no counterpart in the reference; not on any layer path; they allocate and synchronise).
 * moeb_probe_tc_issue: one CTA per SM; `issuers` (1..4) warps each issue back-to-back tcgen05.mma of M = 128,
 * K = 16, N = n (16..256, multiple of 16; 4 issuers need n <= 64, 3 need n <= 128, n > 128 allows one), A in TMEM,
 * into their own accumulators, `per_stage` (4, 8 or 16) MMAs between waits (wait != 0) on an already completed
 * mbarrier phase, `mmas_per_issuer` MMAs each; operands zero, or random bf16 (data != 0); side 1 / 2 / 3: four
 * more warps meanwhile keep storing to / loading from other TMEM columns (tcgen05.st 16x256b.x4 / tcgen05.ld
 * 32x32b.x16, each followed by its wait) or run integer ALU chains. Out: clock cycles per MMA per SM (all issuers' MMAs together), TFLOP/s
 * over the GPU from CUDA events, and cycles per side operation per side warp (may be null). moeb_probe_mma_sync:
 * the same for mma.sync m16n8k16 bf16 over independent chains, warps_per_sm warps per SM. */
int moeb_probe_tc_issue(int n, int issuers, int per_stage, int wait, int data, int side, int mmas_per_issuer,
                        double *cycles_per_mma, double *tflops, double *side_cycles_per_op);
int moeb_probe_mma_sync(int warps_per_sm, int iters, double *tflops);

/* --- moeb_experts_q4 for callers that cannot allocate device memory. No counterpart in the reference (moe-lab
 * always lets the variant allocate its scratch). The scratch lives in a static 16 MiB device array inside the
 * library (held by every GPU that loads it until exit), so the caller passes only inputs and the output. T is
 * limited to what fits: moeb_workspace_bytes(T, d, f, E, k) <= MOEB_STATIC_SCRATCH_BYTES, else MOEB_EINVAL.
 * The first call on a device looks up the array's device address; make it before any stream capture. `stream`
 * must belong to the current device (the address is looked up for the current device). All
 * calls share the array: calls that overlap on the GPU (two streams, two threads) race. Device error bits are
 * cleared on entry; moeb_experts_q4_static_read_error returns the last call's. Nothing is allocated. */
#define MOEB_STATIC_SCRATCH_BYTES (16u << 20)
int moeb_experts_q4_static(const void *x, const void *qg, const void *sbg, const void *qu, const void *sbu,
                           const void *qd, const void *sbd, const float *bg, const float *bu, const float *bd,
                           const int *idx, const float *wts, int T, int d, int f, int E, int k, int act, int policy,
                           const void *residual, void *y, cudaStream_t stream);
/* The device error bits (MOEB_DEVERR_*) the last moeb_experts_q4_static call on the current device recorded, read
 * from the static array and cleared (synchronises `stream`). No counterpart in the reference. Allocates nothing. */
int moeb_experts_q4_static_read_error(unsigned *out, cudaStream_t stream);

#ifdef __cplusplus
}
#endif
#endif /* MOELAB_B200_H */
