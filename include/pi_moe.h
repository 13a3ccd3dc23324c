/*
 * pi_moe.h — C ABI of the B200 (sm_100a) MoE feed-forward and hot-neuron
 * sparse-FFN path for PowerInfer_x64.
 *
 * The entry points replace, one for one, the reference's Rust operator
 * functions on this path (citations: file:line in the reference project).
 * The Rust side keeps its `quant`, `moe` and `predictor` signatures and calls
 * these through a thin `extern "C"` block on the Rust side.
 *
 * Conventions
 *   - Every function returns an int status: PI_OK (0) or one of PI_ERR_*.
 *     pi_last_error(ctx) gives a human-readable message for the last failure.
 *   - Pointers to activations, outputs and index lists are DEVICE pointers
 *     (caller-owned) unless a parameter says otherwise. Weight sources passed
 *     to the *_create functions may be host or device memory (src_on_host).
 *   - `stream` is a cudaStream_t (NULL = legacy default stream). Calls are
 *     asynchronous on it; results are valid after the stream synchronises.
 *   - Device-side index validation (an out-of-range index in a device list)
 *     is reported through pi_ctx_check(), which synchronises the stream.
 *   - There is no CPU fallback: every call runs CUDA kernels for sm_100a.
 *   - A context may be used from several host threads; concurrent calls on
 *     DIFFERENT streams each get their own scratch arena.
 */
#ifndef PI_MOE_H
#define PI_MOE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#pragma GCC visibility push(default)
#endif

/* status codes */
#define PI_OK 0
#define PI_ERR_ARG 1     /* bad argument: null pointer, bad size, unsupported type */
#define PI_ERR_INDEX 2   /* an index is out of range (reference: anyhow Err)        */
#define PI_ERR_SHORT 3   /* raw buffer shorter than the shape needs                 */
#define PI_ERR_OOM 4     /* device allocation failed                                */
#define PI_ERR_CUDA 5    /* a CUDA runtime call or kernel launch failed             */
#define PI_ERR_TIMEOUT 6 /* a bounded device-side wait gave up                      */

/* GGML tensor type ids (numbering of ggml_type; reference quant/mod.rs:12-40) */
#define PI_QT_F32 0
#define PI_QT_F16 1
#define PI_QT_Q4_0 2
#define PI_QT_Q8_0 8

/* pi_moe_forward flags */
#define PI_FWD_RMSNORM 1  /* apply RMSNorm (unit weight) before routing: model/mod.rs:1239 */
#define PI_FWD_RESIDUAL 2 /* out = x + ffn(x): model/mod.rs:1627-1633                     */
#define PI_FWD_FORCE_GEMV 4 /* expert products on the decode GEMV kernels                */
#define PI_FWD_FORCE_GEMM 8 /* expert products on the tcgen05 prefill GEMM                 */
/* Q8_0 prefill GEMM: each block term is added with one fused multiply-add
 * (acc + sumi * (d_w * d_x) rounded once) instead of the reference's separate
 * multiply and add. Results stay within the parity tolerance (rel-L2 1e-3)
 * but are no longer bit-identical to the reference's f32 sums. */
#define PI_FWD_FAST_SUM 16

typedef struct pi_ctx pi_ctx;
typedef struct pi_moe_layer pi_moe_layer;
typedef struct pi_sparse_ffn pi_sparse_ffn;
typedef struct pi_ep_comm pi_ep_comm;

#define PI_EP_MAX_WORLD 64    /* ranks of one expert-parallel group          */
#define PI_EP_HANDLE_BYTES 64 /* bytes of one rank's exported memory handle  */

/* ---- context ----------------------------------------------------------
 * Replaces GpuDevice::new / GpuResources::init (src/cuda/mod.rs:193-218,
 * :387-460): binds one CUDA device; owns per-stream scratch. */
int pi_ctx_create(int device, pi_ctx** out);
void pi_ctx_destroy(pi_ctx* ctx);
const char* pi_last_error(const pi_ctx* ctx);
/* Synchronises `stream`, then reports (and clears) device-side errors. */
int pi_ctx_check(pi_ctx* ctx, void* stream);
/* Pre-sizes the scratch arena of `stream` for `bytes` (0 = no-op), so later
 * calls on that stream allocate nothing (e.g. before CUDA-graph capture). */
int pi_ctx_reserve(pi_ctx* ctx, void* stream, uint64_t bytes);

/* Kernel timing (no reference counterpart; the reference has no GPU
 * profiler hook). enable != 0 starts recording a CUDA event pair around each
 * kernel launch of the layer path on its stream; pi_ctx_profile(ctx, 0) stops
 * and clears. pi_ctx_profile_read synchronises the device and writes up to
 * max_entries kernel names (32 chars each), accumulated milliseconds and
 * launch counts; it returns the number of distinct kernels timed. */
int pi_ctx_profile(pi_ctx* ctx, int enable);
int pi_ctx_profile_read(pi_ctx* ctx, int max_entries, char* names, double* total_ms, int64_t* launches);

/* ---- quant drop-ins (raw GGUF bytes in device memory) ------------------ */

/* quant::dequantize (src/quant/mod.rs:110-143): raw -> f32 [rows*cols].
 * Types F32, F16, Q4_0 (reference nibble order, :180-204), Q8_0 (:320-339).
 * raw_len < needed -> PI_ERR_SHORT (the reference's Err at :122-128). */
int pi_dequantize(pi_ctx* ctx, const void* raw, uint64_t raw_len, int qtype, int64_t rows, int64_t cols,
                  float* out, void* stream);

/* The reference's Q8_0 quantiser quantize_f32_to_q8_0 (src/quant/mod.rs:698-736)
 * emitted as GGUF Q8_0 blocks (34 B: f16 d, 32 x int8). n % 32 == 0. */
int pi_quantize_q8_0(pi_ctx* ctx, const float* x, int64_t n, void* out_raw, void* stream);

/* GGUF Q4_0 blocks (18 B) with the ggml-style quantiser (d = max/-8,
 * q = min(15, trunc(x/d + 8.5))), nibbles packed in the order the reference's
 * decoder reads them (src/quant/mod.rs:193-199). No reference counterpart
 * (the reference only reads Q4_0); used to build synthetic weights. */
int pi_quantize_q4_0(pi_ctx* ctx, const float* x, int64_t n, void* out_raw, void* stream);

/* quant::matvec_col_major (src/quant/mod.rs:939-970): y[j] = x . W[:,j],
 * W = [ne0=n_in, ne1=n_out]. Q8_0 quantises x (:698-736) and uses the
 * integer block dot (:652-689); F32 / Q4_0 use f32 x. */
int pi_matvec_col_major(pi_ctx* ctx, float* y, const float* x, const void* raw, int qtype, int64_t n_in,
                        int64_t n_out, void* stream);

/* Allocation-free variant of pi_matvec_col_major for Q8_0 weights (no
 * counterpart in the reference). For callers that cannot allocate device
 * memory when they call -- e.g. a host whose allocator owns all device memory
 * and forbids cudaMalloc on its hot path -- it needs no pi_ctx and calls no
 * cudaMalloc/cudaFree: the quantised copy of x lives in a fixed device array
 * that every GPU loading this library keeps until exit. Limit: n_in <= 16384
 * (larger n_in returns PI_ERR_ARG); n_in % 32 == 0. Runs on the current
 * device; its first call on a device looks up the array's address
 * (cudaGetSymbolAddress), so make that first call before any stream capture.
 * All calls share the one array: calls that overlap on the GPU (other streams
 * or threads) race and must be serialised by the caller. The looked-up address
 * is kept per device ordinal for the life of the process, so the entry point
 * must not be used after a cudaDeviceReset of that device. Returns PI_OK,
 * PI_ERR_ARG or PI_ERR_CUDA (no error string: there is no context). */
int pi_matvec_col_major_q8_0_noalloc(float* y, const float* x, const void* raw, int64_t n_in, int64_t n_out,
                                     void* stream);

/* quant::matvec_col_major_select (src/quant/mod.rs:974-1068): y[s] = x . W[:, idx[s]].
 * idx: int64 device array. Out-of-range -> device error (pi_ctx_check -> PI_ERR_INDEX). */
int pi_matvec_col_major_select(pi_ctx* ctx, float* y, const float* x, const void* raw, int qtype, int64_t n_in,
                               int64_t n_out, const int64_t* idx, int64_t n_idx, void* stream);

/* quant::matvec_col_major_sparse_input (src/quant/mod.rs:1073-1169):
 * y = W @ x_sparse, x[s] is the value at input row idx[s]. n_idx == 0 -> y = 0. */
int pi_matvec_col_major_sparse_input(pi_ctx* ctx, float* y, const float* x, const int64_t* idx, int64_t n_idx,
                                     const void* raw, int qtype, int64_t n_in, int64_t n_out, void* stream);

/* quant::ffn_swiglu_q (src/quant/mod.rs:1179-1204). */
int pi_ffn_swiglu_q(pi_ctx* ctx, float* out, const float* x, const void* gate_raw, const void* up_raw,
                    const void* down_raw, int qtype, int64_t n_embd, int64_t n_ff, void* stream);

/* quant::ffn_swiglu_q_selected (src/quant/mod.rs:1208-1249): empty idx -> zeros,
 * n_idx >= n_ff -> dense pi_ffn_swiglu_q. */
int pi_ffn_swiglu_q_selected(pi_ctx* ctx, float* out, const float* x, const void* gate_raw, const void* up_raw,
                             const void* down_raw, int qtype, int64_t n_embd, int64_t n_ff, const int64_t* idx,
                             int64_t n_idx, void* stream);

/* ---- MoE layer (weights repacked once into an HBM-resident layout) ----- */

typedef struct pi_moe_layer_desc {
    int64_t n_embd;         /* d: Q8_0 1024 or 2048; Q4_0 1024, 2048 or 4096         */
    int64_t n_ff_exp;       /* expert SwiGLU width f: 128, 256, 512 or 1024         */
    int64_t n_ff_shexp;     /* shared-expert width; the reference uses n_ff_exp    */
    int32_t n_expert;       /* E                                                   */
    int32_t n_expert_used;  /* k                                                   */
    int32_t qtype;          /* PI_QT_Q8_0 or PI_QT_Q4_0 (experts and shared expert) */
    int32_t src_on_host;    /* 1: the pointers below are host memory               */
    const float* router;         /* ffn_gate_inp   f32 [ne0=d, ne1=E]                 */
    const float* router_bias;    /* optional f32 [E], added to the logits (not in the reference) */
    const void* gate_exps;       /* ffn_gate_exps  GGUF bytes [ne0=d, ne1=f, ne2=E]   */
    const void* up_exps;         /* ffn_up_exps    GGUF bytes [ne0=d, ne1=f, ne2=E]   */
    const void* down_exps;       /* ffn_down_exps  GGUF bytes [ne0=f, ne1=d, ne2=E]   */
    const void* gate_shexp;      /* optional ffn_gate_shexp [ne0=d, ne1=f_sh]         */
    const void* up_shexp;        /* optional ffn_up_shexp                             */
    const void* down_shexp;      /* optional ffn_down_shexp [ne0=f_sh, ne1=d]         */
    const float* gate_inp_shexp; /* optional ffn_gate_inp_shexp f32 [d]               */
} pi_moe_layer_desc;

/* Builds the device layer: repacks each expert slice (weights.rs:78-113
 * expert_raw_slice) from GGUF array-of-blocks to structure-of-arrays. */
int pi_moe_layer_create(pi_ctx* ctx, const pi_moe_layer_desc* desc, pi_moe_layer** out);
void pi_moe_layer_destroy(pi_moe_layer* layer);

/* Routing only: model/mod.rs:1254-1312 for T tokens x [T][d] (f32, device, 16-byte
 * aligned: the kernels read token rows with 16-byte loads; PI_ERR_ARG otherwise).
 * idx/gates [T][k] (ascending expert per token; renormalised gates),
 * counts/offsets [E], perm [T*k] (perm[offsets[e]+r] = r-th token routed to e,
 * tokens ascending). Any output pointer may be NULL. */
int pi_moe_route(pi_ctx* ctx, pi_moe_layer* layer, const float* x, int64_t T, int32_t* idx, float* gates,
                 int32_t* counts, int32_t* offsets, int32_t* perm, void* stream);

/* Full MoE FFN for T tokens: router -> top-k -> dispatch -> expert SwiGLU ->
 * gate-weighted combine + sigmoid-gated shared expert
 * (model/mod.rs:1245-1571). out [T][d] f32. x and out 16-byte aligned. flags: PI_FWD_*. */
int pi_moe_forward(pi_ctx* ctx, pi_moe_layer* layer, const float* x, int64_t T, float* out, int32_t flags,
                   void* stream);

/* pi_moe_forward that also returns the routing the forward used (after the
 * optional RMSNorm): idx/gates [T][k], counts/offsets [E], perm [T*k], as
 * pi_moe_route documents; any of them may be NULL. Same reference lines as
 * pi_moe_forward (model/mod.rs:1239-1633); the reference has no separate
 * call, its routing lives inside the token loop (:1254-1312). */
int pi_moe_forward_routed(pi_ctx* ctx, pi_moe_layer* layer, const float* x, int64_t T, float* out, int32_t flags,
                          int32_t* idx, float* gates, int32_t* counts, int32_t* offsets, int32_t* perm, void* stream);

/* ---- Expert parallelism (config 5: experts sharded over the GPUs of a box) ----
 * No reference counterpart: the reference runs the whole layer in one process
 * (model/mod.rs:1245-1571). These calls split pi_moe_forward into the stages
 * around the two exchanges, which the caller performs (NCCL all-to-all-v, or
 * any transport); the result equals pi_moe_forward on the same tokens bit for
 * bit, because every expert row and the combine order are unchanged.
 *
 * A layer for rank r of `world` holds experts [first_expert, first_expert +
 * n_local) with n_local = E / world and first_expert = r * n_local; desc->
 * gate/up/down_exps then hold those n_local experts (GGUF bytes), the router,
 * bias and shared expert are the full ones. Q8_0 experts only. */
int pi_moe_layer_create_ep(pi_ctx* ctx, const pi_moe_layer_desc* desc, int32_t first_expert, int32_t n_local,
                           pi_moe_layer** out);

/* Stage 1, on every rank for its home tokens x [T][d]: RMSNorm (flags), Q8_0
 * quantisation and routing, then the send layout. Slot (t, j) (expert idx[t][j])
 * goes to rank idx / n_local as one row: send_xq [T*k][d] int8, send_xs
 * [T*k][d/32] f32 (token t's Q8_0 activations), send_eid [T*k] (expert id local
 * to the destination); rows are grouped by destination rank (ascending), slot
 * order within a rank; send_counts [world] rows per rank; slot_row [T*k] the row
 * of each slot. Also idx/gates [T][k], shscale [T] (shared-expert gate) and the
 * home tokens' own Q8_0 activations xq [T][d], xs [T][d/32] (for the shared
 * expert). All device pointers, caller-allocated. */
int pi_moe_ep_route(pi_ctx* ctx, pi_moe_layer* layer, const float* x, int64_t T, int32_t flags, int32_t world,
                    int32_t* idx, float* gates, float* shscale, int8_t* xq, float* xs, int32_t* send_counts,
                    int8_t* send_xq, float* send_xs, int32_t* send_eid, int32_t* slot_row, void* stream);

/* Stage 2: expert SwiGLU products of n_rows Q8_0 rows (xq [n][d], xs [n][d/32]):
 * y [n][d] f32, row i through the held expert eid[i] (local id), or through the
 * shared expert for every row when eid == NULL. Prefill-sized row counts use the
 * tensor-core GEMM, others the GEMV kernels. */
int pi_moe_experts_q8(pi_ctx* ctx, pi_moe_layer* layer, int64_t n_rows, const int8_t* xq, const float* xs,
                      const int32_t* eid, float* y, void* stream);

/* Stage 3, on the home rank: out [T][d] = sum over j (ascending expert) of
 * gates[t][j] * y_back[slot_row[t*k + j]] + shscale[t] * y_shared[t] (y_shared may
 * be NULL: no shared expert) + x (PI_FWD_RESIDUAL), in the reference's order
 * (model/mod.rs:1525-1534, :1627-1633). y_back [T*k][d] are the stage-2 rows sent back. */
int pi_moe_ep_combine(pi_ctx* ctx, pi_moe_layer* layer, const float* x, int64_t T, int32_t flags, const float* gates,
                      const float* shscale, const int32_t* slot_row, const float* y_back, const float* y_shared,
                      float* out, void* stream);

/* ---- expert parallelism over NVLink peer memory --------------------------
 * No counterpart in the reference, which runs one process (model/mod.rs:
 * 1245-1571); multi-GPU is only planned there. One rank per GPU; each holds
 * E / world experts (pi_moe_layer_create_ep with first_expert = rank * E / world).
 *
 * pi_ep_comm_create allocates this rank's exchange memory (about
 * world * max_tokens * (3 + 2 * n_embd) * 2 bytes, plus local scratch);
 * pi_ep_comm_ipc_handle exports it (PI_EP_HANDLE_BYTES bytes); the host
 * gathers every rank's handle in rank order (any host collective) and passes
 * them to pi_ep_comm_open, which maps the peers. One comm serves every layer of
 * the group; the ranks must call pi_moe_ep_forward the same number of times, in
 * the same order. */
int pi_ep_comm_create(pi_ctx* ctx, int32_t rank, int32_t world, int64_t max_tokens, int64_t n_embd, int32_t top_k,
                      pi_ep_comm** out);
int pi_ep_comm_ipc_handle(pi_ep_comm* comm, void* handle_out);
int pi_ep_comm_open(pi_ep_comm* comm, const void* handles);
void pi_ep_comm_destroy(pi_ep_comm* comm);

/* One expert-parallel MoE layer forward of this rank's T home tokens (T <= the
 * comm's max_tokens): routing, one Q8_0 row per (token, rank holding one of its
 * experts) stored into that rank's memory, the held experts over every row
 * received, the shared expert over the home tokens, one gate-weighted partial
 * row per (token, rank) stored back, and the combine in ascending rank order
 * (= ascending expert order), then the shared expert and x (PI_FWD_RESIDUAL).
 * Outputs match pi_moe_forward to f32 rounding: the partial rows regroup the
 * reference's left-to-right combine sum (model/mod.rs:1525-1534) by rank.
 * Waits between ranks give up after about a second: pi_ctx_check then reports
 * PI_ERR_TIMEOUT. flags: PI_FWD_RMSNORM | PI_FWD_RESIDUAL | PI_FWD_FAST_SUM. */
int pi_moe_ep_forward(pi_ctx* ctx, pi_moe_layer* layer, pi_ep_comm* comm, const float* x, int64_t T, float* out,
                      int32_t flags, void* stream);

/* Test hook (no reference counterpart): advances the comm's epoch by n with no
 * exchange, so the next pi_moe_ep_forward waits for acknowledgements that never
 * arrive. Its waits give up after about a second each and pi_ctx_check returns
 * PI_ERR_TIMEOUT; nothing faults. The comm is out of step afterwards. */
int pi_ep_comm_debug_skip(pi_ep_comm* comm, int32_t n);

/* MoeRouter::route of the standalone operator API (src/moe/mod.rs:69-108)
 * for T tokens: router f32 expert-major [E][d] (row e = column e of the
 * reference's row-major [d, E] gate), logits summed sequentially, top-k by
 * logit (ties to the lowest index) in descending-logit order, softmax over
 * the selected k (ops::softmax, src/ops.rs:160-180). idx/weights [T][k]. */
int pi_router_topk_softmax(pi_ctx* ctx, const float* x, int64_t T, const float* router, int64_t d, int32_t E,
                           int32_t k, int32_t* idx, float* weights, void* stream);

/* ---- device hot-neuron lists (CSR) for the sparse FFN ------------------
 * Predictor::predict_hot (src/predictor/mod.rs:87-95) turned into the lists the
 * sparse FFN takes, on the device: for token t the blocks b with
 * probs[t][b] >= threshold, ascending, block b = neurons [b*block, (b+1)*block)
 * clipped to n_ff (the predictor's output is blocks of 64 neurons,
 * src/predictor/mod.rs:15). ptr [T+1], idx int64 with room for T * n_ff. */
int pi_hot_lists_from_probs(pi_ctx* ctx, const float* probs, int64_t T, int64_t n_blocks, float threshold,
                            int64_t block, int64_t n_ff, int64_t* ptr, int64_t* idx, void* stream);
/* One static hot list (a HotNeuronIndex layer after Model::set_hot_index's sort
 * and dedup, src/model/mod.rs:1743-1761) for each of T tokens: ptr [T+1],
 * idx [T*n]. */
int pi_hot_lists_broadcast(pi_ctx* ctx, const int64_t* list, int64_t n, int64_t T, int64_t* ptr, int64_t* idx,
                           void* stream);

/* ---- hot-neuron sparse dense FFN --------------------------------------- */

/* Dense SwiGLU FFN weights for the sparse path (model/mod.rs:1573-1612):
 * gate/up GGUF [ne0=n_embd, ne1=n_ff], down [ne0=n_ff, ne1=n_embd]. The down
 * projection is repacked neuron-major so active neurons are contiguous. */
int pi_sparse_ffn_create(pi_ctx* ctx, const void* gate_raw, const void* up_raw, const void* down_raw, int32_t qtype,
                         int64_t n_embd, int64_t n_ff, int32_t src_on_host, pi_sparse_ffn** out);
void pi_sparse_ffn_destroy(pi_sparse_ffn* ffn);

/* ffn_swiglu_q_selected per token (quant/mod.rs:1208-1249, called per token at
 * model/mod.rs:1601-1612) for T tokens, token t using the ascending neuron
 * list idx[ptr[t] .. ptr[t+1]) (CSR, int64 device arrays, ptr has T+1 entries).
 * out [T][n_embd]. An empty list gives zeros; a list of n_ff or more neurons
 * gives the dense FFN. */
int pi_sparse_ffn_forward(pi_ctx* ctx, pi_sparse_ffn* ffn, const float* x, int64_t T, const int64_t* ptr,
                          const int64_t* idx, float* out, void* stream);

/* Predictor::predict (src/predictor/mod.rs:63-84): probs = sigmoid(W2 relu(W1 a + b1) + b2)
 * for T inputs a [T][n_in]; W1 [n_hidden][n_in], W2 [n_out][n_hidden] row-major f32. */
int pi_predictor_forward(pi_ctx* ctx, const float* a, int64_t T, const float* W1, const float* b1, const float* W2,
                         const float* b2, int64_t n_in, int64_t n_hidden, int64_t n_out, float* probs, void* stream);

/* ---- synthetic inputs (benchmarks and tests; no reference counterpart) --
 * out[i] = std * N(0,1) from SplitMix64 (model/mod.rs:2041-2061) + Box-Muller,
 * element i of stream `seed` (i = 2m, 2m+1 take the cos / sin halves of pair m). */
int pi_synth_normal(pi_ctx* ctx, uint64_t seed, uint64_t offset, int64_t n, float std, float* out, void* stream);
/* The same values computed on the host (x86 libm), for fixtures. */
int pi_synth_normal_host(uint64_t seed, uint64_t offset, int64_t n, float std, float* out);

#if defined(__GNUC__)
#pragma GCC visibility pop
#endif

#ifdef __cplusplus
}
#endif
#endif /* PI_MOE_H */
