/*
 * concord_b200.h — C ABI of the B200-native Concord packed-word hot path.
 *
 * Every entry point takes plain device pointers, element counts / strides
 * (in elements), and a `cudaStream_t` passed as `void*` (NULL = legacy
 * default stream).  Nothing here allocates device memory: scratch space is
 * passed in by the caller and its size is reported by the matching
 * `*_workspace_bytes` query.  Every entry point returns 0 on success or a
 * negative `CONCORD_E*` code; `concord_last_error()` gives a one-line
 * message for the calling thread.  bf16 tensors are passed as `uint16_t*`
 * (the raw bf16 bit patterns).
 *
 * Packed word layout (one int32 per parameter):
 *   bits 31:16  s_fast  int16   fast accumulator, mantissa units
 *   bits 15:8   s_slow  int8    slow position, x128 mantissa units
 *   bits  7:0   v_slow  int8    anchor,        x128 mantissa units
 *   weight = (128*s_slow + s_fast + 128*v_slow) * 2^(row_exp + col_exp - 15)
 *
 * Reference interfaces replaced (Theophite/Concord, concord/packed_b.py):
 *   concord_step          <- apply_packed_adamw / _apply_packed_adamw_kernel
 *                            (packed_b.py:863-951, 422-703) and
 *                            apply_packed_sgd / _apply_packed_sgd_kernel
 *                            (packed_b.py:362-394, 173-312)
 *   concord_vhat_update   <- the Adafactor v_row/v_col EMA + 1/sum(v_row)
 *                            in FusedConcordLinearPackedB.backward
 *                            (packed_b.py:1278-1303), plus the row/col max
 *                            zeroing (1281-1283) and the step-counter bump
 *                            (910-911)
 *   concord_salt_bump     <- _get_step_counter(...).add_(1) (packed_b.py:376-377, 910-911)
 *   concord_rebalance     <- rebalance_packed / _rebalance_packed_decide_kernel
 *                            (packed_b.py:1129-1190, 959-1095) and the
 *                            high-watermark fold + seed bump of
 *                            ConcordLinearPackedB.rebalance (1792-1814)
 *   concord_rebalance_gated <- GatedRebalance.__call__
 *                            (notebook/src/concord_winner.py:206-262)
 *   concord_materialize   <- materialize_packed_bf16 (packed_b.py:120-170),
 *                            consolidated_weight (1632-1649)
 *   concord_quantize      <- ConcordLinearPackedB.load_weights (1570-1603),
 *                            load_weights_finetune (1816-1856)
 *   concord_garbage_fraction <- get_garbage_fraction_stats (packed_b.py:1676-1730)
 *   concord_coherence     <- measure_coherence / gate_coherence_from_fields
 *                            (packed_b.py:2081-2106)
 *   concord_gemm_fwd/dx/dw <- F.linear / grad_y @ W / grad_y^T @ x
 *                            (packed_b.py:1219, 1263, 1271-1277)
 *   concord_gemm_dw_vhat  <- grad_y^T @ x followed by the v-hat update
 *                            (packed_b.py:1271-1303) in one call
 *   concord_im2col / concord_col2im / concord_transpose_bf16
 *                         <- the data movement inside torch's
 *                            conv2d / conv2d_input used by the conv layer
 *                            (packed_b.py:2024-2065); with them the conv
 *                            runs on concord_gemm_*
 * The peer-memory entry points (concord_peer_*, concord_ipc_*,
 * concord_step_sharded) have no counterpart: the reference is single-GPU.
 */
#ifndef CONCORD_B200_H
#define CONCORD_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define CONCORD_ABI_VERSION 4

/* status codes */
#define CONCORD_OK            0
#define CONCORD_EINVAL       -1  /* bad argument: null pointer, negative size */
#define CONCORD_ESHAPE       -2  /* shape / stride not supported              */
#define CONCORD_EALIGN       -3  /* pointer alignment not supported           */
#define CONCORD_EWORKSPACE   -4  /* workspace missing or too small            */
#define CONCORD_ELAUNCH      -5  /* CUDA launch / runtime error               */
#define CONCORD_ENODEVICE    -6  /* no usable CUDA device                      */
#define CONCORD_ETOOBIG      -7  /* size above a fixed maximum                */
#define CONCORD_ETIMEOUT     -8  /* a cross-GPU wait ran out (peer transport)  */

/* step-kernel flag bits (the reference's Triton constexprs, packed_b.py:451-458) */
#define CONCORD_F_MASS_PRESERVE   (1u << 0)
#define CONCORD_F_APPLY_CHASE     (1u << 1)
#define CONCORD_F_TRACK_REBALANCE (1u << 2)
#define CONCORD_F_GF_TRUST        (1u << 3)
#define CONCORD_F_GF_CONSOL       (1u << 4)
#define CONCORD_F_COHPRE          (1u << 5)
#define CONCORD_F_FIXED_COH       (1u << 6)
#define CONCORD_F_RATIO_COH       (1u << 7)

#define CONCORD_KIND_ADAMW 0
#define CONCORD_KIND_SGD   1

/*
 * fp32 arithmetic of the step (concord_step_params.arith).
 *   CONCORD_ARITH_GPU (default): the reference's kernel as compiled by Triton
 *     for NVIDIA GPUs: tl.exp2 = ex2.approx.f32, tl.log2 = CUDA log2f, `/` =
 *     div.full.f32, min/max drop NaN, and multiply-add contracted to fma where
 *     the compiled reference contracts it.  Scalars the kernel combines
 *     (1 - alpha_v_fast, 1 - floors, alpha * gate_gain) are combined in fp32
 *     in the kernel, as the compiled reference does.  Words bit-identical to
 *     the reference running on a B200.
 *   CONCORD_ARITH_CR: every fp32 operation rounded once, exp2/log2 correctly
 *     rounded, IEEE division, numpy NaN semantics: the model the CPU oracle
 *     restates (and the reference under its CPU interpreter with correctly
 *     rounded exp2/log2); the one_minus_* / alpha_gate_gain fields are used.
 */
#define CONCORD_ARITH_GPU 0
#define CONCORD_ARITH_CR  1

/*
 * Launch-time scalars of one packed step.  Every float is the fp32 value
 * the kernel multiplies with.  Where the reference combines two host
 * scalars before they meet a tensor (e.g. `1.0 - alpha_v_fast`), the
 * combined value is computed on the host in double and rounded once to
 * fp32 — the `one_minus_*` and `alpha_gate_gain` fields carry those.
 */
typedef struct concord_step_params {
    int32_t  kind;                  /* CONCORD_KIND_ADAMW / CONCORD_KIND_SGD */
    int32_t  mantissa_bias;         /* 15 */
    uint32_t flags;                 /* CONCORD_F_* */
    float alpha;                    /* chase rate */
    float beta1;
    float weight_decay;
    float step_cap;
    float v_scale;
    float precond_p;
    float gf_consol;                /* evaporation kappa */
    float drift_cancel_C;
    float alpha_v_fast;
    float one_minus_alpha_v_fast;   /* fp32(1.0 - alpha_v_fast), double-folded */
    float wd_sv;
    float wd_sf;
    float gf_trust_delta_sq;
    float gate_gain;
    float chase_floor;
    float one_minus_chase_floor;    /* fp32(1.0 - chase_floor) */
    float leak_floor;
    float one_minus_leak_floor;     /* fp32(1.0 - leak_floor) */
    float alpha_gate_gain;          /* fp32(alpha * 1.0 * gate_gain): chase gain when no gate tensor */
    /*
     * Optional device scalars, read by the kernel at run time (so a captured
     * CUDA graph follows their current values); NULL = not used.
     *   consolidate: gradient accumulation gate of the reference's prototype
     *     kernel (notebook/src/prototype_packed_b.py:481-515, 661-780).  The
     *     SR tick of s_fast always applies; the beta1 and evaporation terms of
     *     the tick, the chase, the v_slow leak and both weight decays are
     *     multiplied by float(*consolidate); the bf16 weight and the row/col
     *     maxima are written only when *consolidate == 1 (the weight stays
     *     frozen during accumulation).  coh_pre is updated either way.
     *     AdamW only.
     *   ratio_floors: [chase_floor, leak_floor] for the ratio-coherence gate,
     *     replacing chase_floor / leak_floor and their one_minus_* (then
     *     1 - floor in fp32, as the prototype kernel computes it).
     */
    const int32_t* consolidate;
    const float* ratio_floors;
    int32_t arith;                  /* CONCORD_ARITH_GPU (0) or CONCORD_ARITH_CR (1) */
} concord_step_params;

int         concord_abi_version(void);
const char* concord_last_error(void);

/* *salt += 1 on the stream (the reference's per-device step counter). */
int concord_salt_bump(int32_t* salt, void* stream);

/*
 * Adafactor second-moment update from a bf16 gradient [N,K] (row stride ldg):
 *   v_row = b2*v_row + (1-b2)*sum_k g^2,  v_col likewise over n,
 *   sum_v_inv = 1 / max(sum_n v_row, 1e-30).
 * Sums run in a fixed order (deterministic).  Also zeroes row_max[N] and
 * col_max[K] when they are non-NULL, and bumps *salt when it is non-NULL,
 * so that a following concord_step sees the reference's pre-launch state.
 * `workspace` must hold concord_vhat_workspace_bytes(N, K) bytes and be
 * zero-filled before its first use (the kernel leaves it reusable).
 */
size_t concord_vhat_workspace_bytes(int64_t N, int64_t K);
int concord_vhat_update(const uint16_t* grad, int64_t ldg, int64_t N, int64_t K,
                        float* v_row, float* v_col, float* sum_v_inv,
                        float beta2, float one_minus_beta2,
                        int32_t* row_max, int32_t* col_max, int32_t* salt,
                        void* workspace, size_t workspace_bytes, void* stream);

/*
 * concord_vhat_update without a caller-provided workspace.  No counterpart in
 * the reference.  For callers that may not allocate device memory (a host
 * framework that owns all device memory behind a fixed budget, or a
 * latency-critical caller that cannot afford cudaMalloc's implicit device
 * synchronisation): the scratch is a fixed 4 MiB array inside this library
 * (concord_vhat_noalloc_max_scratch_bytes()), held by every GPU that loads
 * the library until the process exits.  Sizes whose
 * concord_vhat_workspace_bytes(N, K) exceed it are rejected with
 * CONCORD_ETOOBIG.  Every call looks up the array's device address for the
 * current device (a host-side query); the first call on a device, and the
 * first call after that address changes (a new CUDA context on the device,
 * e.g. after cudaDeviceReset), clears the array on `stream`: make that first
 * call before any stream capture.  All calls on a device share the one
 * array: calls that may overlap on the GPU (different streams without
 * ordering) race and must be serialised by the caller.  Nothing else differs
 * from concord_vhat_update: same results, bit for bit.
 */
size_t concord_vhat_noalloc_max_scratch_bytes(void);
int concord_vhat_update_noalloc(const uint16_t* grad, int64_t ldg, int64_t N, int64_t K,
                                float* v_row, float* v_col, float* sum_v_inv,
                                float beta2, float one_minus_beta2,
                                int32_t* row_max, int32_t* col_max, int32_t* salt,
                                void* stream);

/*
 * Row-sharded form of concord_vhat_update for data-parallel training
 * (the reference has no multi-GPU code; this splits its v-hat update,
 * packed_b.py:1288-1303, at the one point that needs all rows).  On this
 * rank's shard grad [N,K]: v_row is updated in place; col_sum_out[K]
 * receives the shard's column sums of g^2 and *vsum_out the sum of the
 * shard's updated v_row.  The caller all-reduces (col_sum_out, vsum_out)
 * over ranks, then concord_vhat_finish applies v_col = b2*v_col +
 * (1-b2)*col_sum and sum_v_inv = 1/max(vsum, 1e-30).
 */
int concord_vhat_partial(const uint16_t* grad, int64_t ldg, int64_t N, int64_t K, float* v_row,
                         float beta2, float one_minus_beta2, int32_t* row_max, int32_t* col_max,
                         int32_t* salt, float* col_sum_out, float* vsum_out,
                         void* workspace, size_t workspace_bytes, void* stream);
int concord_vhat_finish(const float* col_sum, const float* vsum, float* v_col, float* sum_v_inv,
                        int64_t K, float beta2, float one_minus_beta2, void* stream);

/*
 * One packed optimizer step over rows [0,N) of a (row-)shard whose first
 * row is global row `row0` (0 when unsharded).  Mutates packed (and
 * coh_pre when CONCORD_F_COHPRE) in place, writes the new bf16 weight to
 * wbuf, and atomic-maxes |m_eff| into row_max[N]/col_max[K] when
 * CONCORD_F_TRACK_REBALANCE.  v_row/v_col/sum_v_inv are read only when a
 * flag needs them.  lr, eps and salt are device scalars.  coh_stats, when
 * non-NULL, receives (sum of coh, element count) as two doubles added
 * atomically (the fused coherence meter); it is only written when the
 * flags compute coh.
 */
int concord_step(const concord_step_params* p,
                 int32_t* packed, int64_t ldp,
                 const uint16_t* grad, int64_t ldg,
                 uint16_t* wbuf, int64_t ldw,
                 const int8_t* row_exp, const int8_t* col_exp,
                 int32_t* row_max, int32_t* col_max,
                 const float* v_row, const float* v_col, const float* sum_v_inv,
                 float* coh_pre, int64_t ldc,
                 const float* lr, const float* eps, const int32_t* salt,
                 int64_t N, int64_t K, int64_t row0,
                 double* coh_stats, void* stream);

/*
 * concord_step for a row shard in a data-parallel job whose ranks share
 * memory over NVLink (no reference counterpart).  Identical to concord_step,
 * and in addition every bf16 weight the step writes to wbuf (rows [0,N) of
 * the shard) is also stored to row row0 + n of each of the n_peers other
 * ranks' full forward-weight buffers: wbuf_peers is a DEVICE array of their
 * base addresses (opened with concord_ipc_open), each with row stride ldw.
 * This is the all-gather of the forward weight, overlapped with the step.
 */
int concord_step_sharded(const concord_step_params* p,
                         int32_t* packed, int64_t ldp,
                         const uint16_t* grad, int64_t ldg,
                         uint16_t* wbuf, int64_t ldw,
                         const int8_t* row_exp, const int8_t* col_exp,
                         int32_t* row_max, int32_t* col_max,
                         const float* v_row, const float* v_col, const float* sum_v_inv,
                         float* coh_pre, int64_t ldc,
                         const float* lr, const float* eps, const int32_t* salt,
                         int64_t N, int64_t K, int64_t row0,
                         double* coh_stats, const uint64_t* wbuf_peers, int32_t n_peers,
                         void* stream);

/*
 * Gated rebalance of many layers (the trainer-side GatedRebalance of the
 * reference, notebook/src/concord_winner.py:206-262): if any value of
 * row_max_all[0..n_rows_all) or col_max_all[0..n_cols_all) (every layer's
 * maxima, held in two shared arrays) exceeds gate_max_m, every layer runs
 * its rebalance -- seed bump, high-watermark fold, tick-up decisions from
 * the pre-launch exponents, SR shift of the ticked words (as
 * concord_rebalance with allow_tickdown 0) -- otherwise none does.  The
 * decision stays on the device: three launches, no host synchronisation.
 * `layers` is a DEVICE array of n_layers descriptors; layer l's decide
 * entries are [decide_off, decide_off + N + K) of [0, total_decide), in
 * increasing order.  Each layer's rt/ct/fired/rowlist/collist point into a
 * zero-filled workspace of concord_rebalance_gated_layer_workspace_bytes(N, K)
 * bytes (concord_rebalance_gated_layer_layout fills those five fields).
 * gate: device int32[2], zero-filled before the first call (the call leaves
 * it zeroed).  fired_out (optional): 1 if the layers ran, else 0.
 */
typedef struct concord_reb_layer {
    int32_t* packed; int64_t ldp;
    int8_t* row_exp; int8_t* col_exp;
    const int32_t* row_max; const int32_t* col_max;
    int32_t* row_hwm; int32_t* col_hwm;      /* may be NULL */
    int32_t* seed;
    int32_t max_m, exp_max, exp_min, pad0;
    int64_t N, K, row0, N_total;
    int64_t decide_off;
    int8_t* rt; int8_t* ct; int32_t* fired; int32_t* rowlist; int32_t* collist;
} concord_reb_layer;

size_t concord_rebalance_gated_layer_workspace_bytes(int64_t N, int64_t K);
int concord_rebalance_gated_layer_layout(int64_t N, int64_t K, void* workspace, concord_reb_layer* layer);
int concord_rebalance_gated(const concord_reb_layer* layers, int32_t n_layers, int64_t total_decide,
                            const int32_t* row_max_all, int64_t n_rows_all, const int32_t* col_max_all,
                            int64_t n_cols_all, int32_t gate_max_m, int32_t* gate, int32_t* fired_out,
                            void* stream);

/*
 * Peer memory for the data-parallel step over NVLink (no reference
 * counterpart).  concord_peer_alloc / concord_peer_free: plain device
 * allocations of the current device (zero-filled), exportable whole with
 * concord_ipc_export into a concord_ipc_handle_bytes()-byte handle that
 * another process on the same node maps with concord_ipc_open (and unmaps
 * with concord_ipc_close).
 */
size_t concord_ipc_handle_bytes(void);
int concord_peer_alloc(size_t bytes, void** dev_ptr);
int concord_peer_free(void* dev_ptr);
int concord_ipc_export(void* dev_ptr, void* handle_out);
int concord_ipc_open(const void* handle, void** dev_ptr);
int concord_ipc_close(void* dev_ptr);

/*
 * Cross-GPU rendezvous state of one peer-memory exchange (device memory):
 *   flags      this rank's flag array [n_ranks] in peer memory; rank q
 *              stores its epoch into flags[q]
 *   peer_flags DEVICE array [n_ranks] of every rank's flag array (own included)
 *   state      this rank's int32[4]: [0] epoch, [1] finished-block count,
 *              [2] error word (non-zero after a wait ran out; sticky until
 *              the caller clears it), [3] unused; zero-filled at creation
 * Every wait polls with a limit of timeout_ns of GPU time; when it runs out
 * the kernel sets state[2], skips its work and returns, so the context
 * stays usable and the host sees the error word.
 */
typedef struct concord_peer_sync {
    int32_t* flags;
    const uint64_t* peer_flags;
    int32_t* state;
    int32_t rank;
    int32_t n_ranks;
    int64_t timeout_ns;
} concord_peer_sync;

/*
 * Reduce-scatter of the bf16 dW over peer memory, in two launches.  Ranks own
 * row shards [q*S, min(N, (q+1)*S)) of an [N, K] gradient (S * n_ranks >= N).
 *
 * concord_peer_push_rows: for every q != rank, the rows of q's shard of this
 * rank's dW (grad, [N, K], row stride K) are stored into q's receive buffer at
 * block `rank` (recv_q + rank * S * K, row stride K); recv is a DEVICE array
 * [n_ranks] of every rank's receive buffer (n_ranks * S * K bf16 each).  It
 * never waits: when all its stores have landed it announces a new epoch to
 * every rank.
 *
 * concord_peer_reduce_vhat: waits until every rank has announced that epoch
 * (its pushes into this rank's receive buffer have landed), then
 *   grad_out[n, k] = bf16_rne( sum over q = 0..n_ranks-1, in rank order, in
 *                    fp32, of src_q[n * K + k] ),   n < n_rows, k < K,
 * src_rank = own_rows (this rank's rows of its own shard), src_q = recv + q*S*K
 * (the local receive buffer) otherwise, and in the same pass the v-hat
 * partials of concord_vhat_partial on grad_out, in the same fixed order: every
 * output (grad_out, v_row, row_max/col_max zeroing, salt bump, col_sum_out,
 * vsum_out) is bit-identical to the two steps run separately.  n_rows may be
 * 0 (a rank without rows: zero partials).  workspace: at least
 * concord_vhat_workspace_bytes(max(n_rows, 1), K) bytes, zero-filled before
 * first use.  After a wait ran out nothing is written.  K a multiple of 8;
 * every buffer 16-byte aligned; n_ranks <= 8.
 */
int concord_peer_push_rows(const uint16_t* grad, int64_t N, int64_t K, int64_t S, const uint64_t* recv,
                           const concord_peer_sync* sync, void* stream);
int concord_peer_reduce_vhat(const uint16_t* own_rows, const uint16_t* recv, int64_t S, int64_t K,
                             int64_t n_rows, uint16_t* grad_out, float* v_row, float beta2,
                             float one_minus_beta2, int32_t* row_max, int32_t* col_max, int32_t* salt,
                             float* col_sum_out, float* vsum_out, void* workspace, size_t workspace_bytes,
                             const concord_peer_sync* sync, void* stream);

/*
 * All-reduce of `count` 32-bit values over the ranks of `sync` through peer
 * slots (count 0: a pure rendezvous).  op CONCORD_PEER_SUM_F32: fp32 sum in
 * rank order (the same bits on every rank for any rank count);
 * CONCORD_PEER_MAX_I32: int32 max.  slots: DEVICE array [n_ranks] of every
 * rank's slot buffer of 2 * n_ranks * slot_count 32-bit values (concord_peer_alloc,
 * opened with concord_ipc_open); count <= slot_count.  out may alias in.
 */
#define CONCORD_PEER_SUM_F32 0
#define CONCORD_PEER_MAX_I32 1
int concord_peer_allreduce(const void* in, void* out, int64_t count, int32_t op, const uint64_t* slots,
                           int64_t slot_count, const concord_peer_sync* sync, void* stream);

/*
 * Rebalance ratchet.  Folds row_max/col_max into the high-watermarks (when
 * non-NULL), bumps *seed, decides per-row/col exponent ticks from the
 * PRE-launch exponents, SR-right-shifts the three fields where a tick-up
 * fires (Philox4x32-10 uniforms keyed by (seed, n*K+k + {0,NK,2NK})), and
 * left-shifts where a tick-down fires (allow_tickdown only).  N_total is
 * the global row count and row0 the first global row (Philox offsets use
 * global indices).  fired_out (nullable, device int32) is set to 1 when any
 * exponent moved, else 0.  stats (nullable, device uint64[3]) accumulates
 * the reference's optional rebalance instrumentation (packed_b.py:1161-1179):
 * [0] += rows+columns ticked up, [1] += rows+columns ticked down, [2] += words
 * whose larger int8 field exceeds 127 once the tick-down left shift is
 * applied (one extra read pass over the words, only when stats != NULL).
 * Workspace: concord_rebalance_workspace_bytes(N, K), zero-filled before
 * first use.
 */
size_t concord_rebalance_workspace_bytes(int64_t N, int64_t K);
int concord_rebalance(int32_t* packed, int64_t ldp,
                      int8_t* row_exp, int8_t* col_exp,
                      const int32_t* row_max, const int32_t* col_max,
                      int32_t* row_hwm, int32_t* col_hwm,
                      int32_t* seed, int32_t max_m, int32_t exp_max, int32_t exp_min,
                      int32_t allow_tickdown,
                      int64_t N, int64_t K, int64_t row0, int64_t N_total,
                      int32_t* fired_out, unsigned long long* stats,
                      void* workspace, size_t workspace_bytes, void* stream);

/* bf16 weight = (m_eff or the slow part only) * 2^(row_exp+col_exp-bias), RNE. */
int concord_materialize(const int32_t* packed, int64_t ldp,
                        const int8_t* row_exp, const int8_t* col_exp,
                        uint16_t* out, int64_t ldo, int64_t N, int64_t K,
                        int32_t mantissa_bias, int32_t consolidated, void* stream);

/*
 * fp32 W [N,K] -> packed words + row_exp (col_exp zeroed).  finetune=0:
 * whole mantissa in s_fast (load_weights); finetune=1: split half to
 * v_slow, rest to s_slow, residual to s_fast (load_weights_finetune).
 */
int concord_quantize(const float* W, int64_t ldw, int32_t* packed, int64_t ldp,
                     int8_t* row_exp, int8_t* col_exp, int64_t N, int64_t K,
                     int32_t mantissa_bias, int32_t exp_min, int32_t exp_max,
                     int32_t finetune, void* stream);

/*
 * Wiener coherence of the packed state (measure_coherence):
 * out[0] += sum of coh (double), out[1] += element count.  The caller
 * zeroes out[] first.
 */
int concord_coherence(const int32_t* packed, int64_t ldp, int64_t N, int64_t K,
                      float drift_cancel_C, double* out, void* stream);

/*
 * Garbage-fraction diagnostic of the packed state
 * (ConcordLinearPackedB.get_garbage_fraction_stats, packed_b.py:1676-1730):
 * gf = clamp((noise * 2^(row_exp+col_exp-bias))^2 / (v_hat + 1e-30), 0, 1),
 * noise = s_fast - C * 128 * (s_slow - v_slow), v_hat = v_row v_col / *sum_v.
 * gf_out (nullable, contiguous [N,K] fp32) receives gf; acc (device double[3],
 * zeroed by the caller) += sum of gf, count of gf < 0.1, count of gf > 0.9.
 */
int concord_garbage_fraction(const int32_t* packed, int64_t ldp, const int8_t* row_exp,
                             const int8_t* col_exp, const float* v_row, const float* v_col,
                             const float* sum_v, int64_t N, int64_t K, int32_t mantissa_bias,
                             float drift_cancel_C, float* gf_out, double* acc, void* stream);

/*
 * The layer's dense GEMMs on the tensor cores (tcgen05/TMEM, TMA-fed), bf16
 * in, fp32 accumulate, bf16 out (round to nearest even).  Row-major,
 * contiguous operands; every extent a multiple of 8 and 16-byte aligned
 * pointers (else CONCORD_ESHAPE / CONCORD_EALIGN).
 *   concord_gemm_fwd: y[M,N]  = x[M,K] * w[N,K]^T        (F.linear without bias)
 *   concord_gemm_dx:  dx[M,K] = dy[M,N] * w[N,K]
 *   concord_gemm_dw:  dw[N,K] = dy[M,N]^T * x[M,K]
 * Workspace: concord_gemm_workspace_bytes(M, N, K) (may be 0).
 */
size_t concord_gemm_workspace_bytes(int64_t M, int64_t N, int64_t K);
int concord_gemm_fwd(const uint16_t* x, const uint16_t* w, uint16_t* y, int64_t M, int64_t N, int64_t K,
                     void* workspace, size_t workspace_bytes, void* stream);
int concord_gemm_dx(const uint16_t* dy, const uint16_t* w, uint16_t* dx, int64_t M, int64_t N, int64_t K,
                    void* workspace, size_t workspace_bytes, void* stream);
int concord_gemm_dw(const uint16_t* dy, const uint16_t* x, uint16_t* dw, int64_t M, int64_t N, int64_t K,
                    void* workspace, size_t workspace_bytes, void* stream);

/*
 * dW = dY^T X (as concord_gemm_dw) together with the v-hat update of
 * concord_vhat_update on that dW (row/col max zeroing and salt bump
 * included): the backward's dW GEMM (packed_b.py:1271-1277) and its
 * Adafactor update (1278-1303) in one call.  When the N x K output has at
 * least 148 tiles of 128 x 256 (one per SM of a B200), the squared bf16
 * outputs are summed per tile in the GEMM's epilogue and one fold launch
 * finishes, so dW is not read again; the dW written is bit-identical to
 * concord_gemm_dw's, and v_row / v_col / sum_v_inv agree with
 * concord_vhat_update's to fp32 rounding (same tiles and fold order; the
 * in-tile order is the epilogue's).  Smaller layers run concord_gemm_dw and
 * then concord_vhat_update (bit-identical to calling them).  `workspace`: at least
 * concord_gemm_dw_vhat_workspace_bytes(M, N, K) bytes, 16-byte aligned,
 * zero-filled before its first use (the call leaves it reusable).
 */
size_t concord_gemm_dw_vhat_workspace_bytes(int64_t M, int64_t N, int64_t K);
int concord_gemm_dw_vhat(const uint16_t* dy, const uint16_t* x, uint16_t* dw, int64_t M, int64_t N, int64_t K,
                         float* v_row, float* v_col, float* sum_v_inv, float beta2, float one_minus_beta2,
                         int32_t* row_max, int32_t* col_max, int32_t* salt,
                         void* workspace, size_t workspace_bytes, void* stream);

/*
 * Convolution as GEMMs (bf16, NCHW input x [B, C, H, W], kernel kh x kw,
 * stride sh/sw, zero padding ph/pw; Ho = (H + 2ph - kh)/sh + 1, likewise Wo).
 * im2col: cols [B*Ho*Wo, C*kh*kw] row-major, column c*kh*kw + i*kw + j
 * (the order of the packed [O, C*kh*kw] weight); C*kh*kw % 8 == 0, cols
 * 16-byte aligned.  col2im: dx [B, C, H, W] from the transposed column
 * gradient dcols_t [C*kh*kw, B*Ho*Wo], each pixel summed in fp32 over
 * (i, j) in order and rounded once to bf16.
 */
int concord_im2col(const uint16_t* x, int64_t B, int64_t C, int64_t H, int64_t W,
                   int32_t kh, int32_t kw, int32_t sh, int32_t sw, int32_t ph, int32_t pw,
                   uint16_t* cols, void* stream);
int concord_col2im(const uint16_t* dcols_t, int64_t B, int64_t C, int64_t H, int64_t W,
                   int32_t kh, int32_t kw, int32_t sh, int32_t sw, int32_t ph, int32_t pw,
                   uint16_t* dx, void* stream);
/* bf16 out[b][c][r] = in[b][r][c] for in [batches, R, C] (the NCHW
 * convolution gradient as the [B*Ho*Wo, O] rows of the dW GEMM); batches
 * <= 65535. */
int concord_transpose_bf16(const uint16_t* in, int64_t batches, int64_t R, int64_t C, uint16_t* out,
                           void* stream);

/*
 * 2-SM tcgen05 GEMM written in this package (no CUTLASS): D[M,N] (bf16,
 * row-major, row stride ldd) = sum_k A(m,k) B(n,k), fp32 accumulation, one
 * RNE rounding.  a_mn = 0: A is K-major, the row-major [M, K] matrix (row
 * stride lda); a_mn = 1: A is MN-major, the row-major [K, M] matrix.  B
 * likewise with N.  Extents and strides multiples of 8, 16-byte aligned.
 * The layer's three GEMMs (packed_b.py:1219, 1263, 1273) are
 *   fwd (x K-major, w K-major), dX (dY K-major, w MN-major),
 *   dW (dY MN-major, x MN-major).
 * concord_gemm2sm_error(reset): the device's error word (non-zero when a
 * barrier wait inside the kernel ran out; 2 s of GPU time per wait).
 */
/* Kernels behind concord_gemm_fwd / _dx / _dw (process-wide; the split-K dW
 * and concord_gemm_dw_vhat always run the CUTLASS kernels):
 * CONCORD_GEMM_2SM (default) or CONCORD_GEMM_CUTLASS. */
#define CONCORD_GEMM_2SM 0
#define CONCORD_GEMM_CUTLASS 1
int concord_gemm_set_impl(int32_t impl);
int concord_gemm_get_impl(void);
int concord_gemm2sm(const uint16_t* a, int32_t a_mn, int64_t lda, const uint16_t* b, int32_t b_mn, int64_t ldb,
                    uint16_t* d, int64_t ldd, int64_t M, int64_t N, int64_t K, void* stream);
int concord_gemm2sm_error(int32_t reset);
/* CTA pairs the 2-SM GEMM keeps resident (its persistent grid). */
int concord_gemm2sm_pairs(void);

/*
 * Implicit-GEMM convolutions on channels-last (NHWC) bf16 tensors
 * (fp32 accumulation, one round-to-nearest-even per output element), with
 * no column matrix: the activation is read by TMA in im2col mode.  They
 * replace the reference conv layer's cuDNN calls, F.conv2d
 * (concord/packed_b.py:1890) and torch.nn.grad.conv2d_input /
 * conv2d_weight (packed_b.py:1939-1947).
 *   x  [B, H, W, C]      dx the same;  y / dy [B, Ho, Wo, O]
 *   w  [O, kh, kw, C]    (KRSC: the packed [O, C*kh*kw] weight permuted)
 *   dw [O, kh, kw, C]    (wgrad writes KRSC; the packed step reads KCRS)
 * C % 8 == 0, O % 8 == 0, every tensor 16-byte aligned; dgrad needs stride
 * 1.  Workspace: concord_conv_nhwc_workspace_bytes(op, ...) bytes (wgrad
 * splits its B*Ho*Wo reduction when the output has few tiles; its
 * split-ordered fixup is deterministic).
 */
#define CONCORD_CONV_FPROP 0
#define CONCORD_CONV_DGRAD 1
#define CONCORD_CONV_WGRAD 2
size_t concord_conv_nhwc_workspace_bytes(int op, int64_t B, int64_t H, int64_t W, int64_t C, int64_t O,
                                         int64_t kh, int64_t kw, int64_t sh, int64_t sw, int64_t ph, int64_t pw);
int concord_conv_fprop_nhwc(const uint16_t* x, const uint16_t* w, uint16_t* y, int64_t B, int64_t H, int64_t W,
                            int64_t C, int64_t O, int64_t kh, int64_t kw, int64_t sh, int64_t sw, int64_t ph,
                            int64_t pw, void* workspace, size_t workspace_bytes, void* stream);
int concord_conv_dgrad_nhwc(const uint16_t* dy, const uint16_t* w, uint16_t* dx, int64_t B, int64_t H, int64_t W,
                            int64_t C, int64_t O, int64_t kh, int64_t kw, int64_t sh, int64_t sw, int64_t ph,
                            int64_t pw, void* workspace, size_t workspace_bytes, void* stream);
int concord_conv_wgrad_nhwc(const uint16_t* dy, const uint16_t* x, uint16_t* dw, int64_t B, int64_t H, int64_t W,
                            int64_t C, int64_t O, int64_t kh, int64_t kw, int64_t sh, int64_t sw, int64_t ph,
                            int64_t pw, void* workspace, size_t workspace_bytes, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* CONCORD_B200_H */
