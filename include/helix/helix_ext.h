/* helix_ext.h -- entry points beyond the reference ABI.
 *
 * The reference (a single-device Metal encoder) has no counterpart to these;
 * each comment says why it exists on B200.
 */
#ifndef HELIX_EXT_H
#define HELIX_EXT_H

#include "helix/helix.h"

#ifdef __cplusplus
extern "C" {
#endif

/* Reads and clears the device-side fault word of the tensor-core kernels on
 * ctx's device.  Every wait inside those kernels (TMA arrival, tcgen05
 * completion) is bounded; when one expires the kernel releases its tensor
 * memory, returns, and records a nonzero code here instead of hanging the
 * GPU.  *code is 0 when nothing was recorded.  Codes: 1, 2 a wait of the
 * output kernels (copy arrival; MMA or hand-off), 3, 4 the same in the state
 * kernel, 5 an s0 row selected by ids overlapped the s1 rows being written
 * (that sequence's outputs are NaN), 6 the test hook HELIX_TEST_STALL_CYCLES.
 * Synchronous (it copies one word). */
helix_status helix_device_fault(helix_ctx* ctx, uint32_t* code);

/* No counterpart in the reference.  The multipass scan for callers that
 * cannot allocate device memory: hosts that give an op only its input and
 * output buffers (graph executors with a fixed memory plan and no per-op
 * workspace, plugins inside a process that owns all device memory, code that
 * may not allocate after start-up).  Same arguments and results as
 * helix_scan_encode with multipass forced on, minus `scratch`: the run
 * scratch lives in a 32 MiB array inside the library.
 *   - The first call on a device loads the array (CUDA reserves its 32 MiB
 *     then, with lazy module loading) and the device keeps it until the
 *     process exits.  Make that first call at start-up, before any stream
 *     capture; if the device has no room for the array the call fails with
 *     HELIX_ERR_PIPELINE and nothing is enqueued.
 *   - Descriptors needing more than 32 MiB of run scratch are rejected with
 *     HELIX_ERR_SCRATCH_TOO_SMALL (message in helix_ctx_last_error);
 *     nothing is enqueued.
 *   - All calls on a device share the array: calls that can overlap on the
 *     GPU race and must be serialised by the caller.  Nothing in it needs to
 *     start at zero (each call writes what it later reads).
 *   - Never calls cudaMalloc, cudaFree or any allocating routine. */
helix_status helix_scan_encode_static(helix_ctx*             ctx,
                                      void*                  stream,
                                      const helix_scan_desc* d,
                                      helix_tensor           s0,
                                      helix_tensor           x,
                                      helix_tensor           dt,
                                      helix_tensor           A,
                                      helix_tensor           B,
                                      helix_tensor           C,
                                      helix_tensor           ids,
                                      helix_tensor           y,
                                      helix_tensor           s1);

/* No counterpart in the reference.  How a descriptor will run: the kernel
 * family, the chunk the output kernel walks in, and the run cut of the
 * multipass decomposition (runs of whole 128-token blocks; the output kernel
 * gives each CTA a span of runs_per_span consecutive runs; the state pass
 * reduces the state_runs runs before the last span).  For profiling and
 * capacity planning; host only, nothing is enqueued.  Returns
 * HELIX_ERR_UNSUPPORTED_SHAPE (and fills nothing) for a descriptor
 * helix_scan_supported rejects. */
typedef struct helix_plan_info {
    int32_t  family;         /* 0: exact fp32 CUDA-core kernels, 1: tcgen05 bf16,
                                2: tcgen05 three-product (fp32-class),
                                3: diagonal-A recurrence (CUDA cores, fp32) */
    int32_t  chunk;          /* tokens per chunk of the output kernel */
    int32_t  run_tokens;     /* tokens per run */
    int32_t  n_runs;         /* runs per sequence */
    int32_t  runs_per_span;  /* runs per output CTA */
    int32_t  n_spans;        /* output spans per sequence */
    int32_t  state_runs;     /* runs the state pass reduces, per (sequence, head) */
    int32_t  reserved;
    uint64_t scratch_bytes;  /* helix_scan_scratch_size() of the descriptor */
} helix_plan_info;

helix_status helix_scan_plan_info(helix_ctx* ctx, const helix_scan_desc* d, helix_plan_info* out);

/* No counterpart in the reference (one Metal device, one encoder).  Support
 * for cutting every sequence's tokens into contiguous shards, one per GPU
 * ("L-split"): rank k holds tokens [l_k, l_{k+1}) of x, dt, B and C, with d
 * describing its shard (d->n_tok = shard length).  Per rank:
 *
 *   1. helix_scan_shard_state: the state the shard leaves from a zero start,
 *      state[seq][h][p][n] = sum_t exp(sum_{t'>t} A_h dt_t') dt_t x_t[p] B_t[n]
 *      (state strides s_s / seq_s of d, innermost 1), and its log-decay
 *      log_decay[seq * n_head + h] = sum_t A_h dt_t (natural log; f32).
 *   2. The caller gathers (state, log_decay) of ranks 0..k-1 (e.g. an
 *      all-gather over the ranks sharing the same heads) into dense arrays
 *      states[j][seq][h][p][n] and log_decays[j][seq][h], j = 0..n_prev-1.
 *   3. helix_scan_carry_combine: carry = the fold over j of
 *      S <- exp(log_decays[j]) S + states[j], starting from s0[ids[seq]]
 *      (ids may be null: s0[seq]); carry uses the state strides of d and
 *      must not overlap s0.
 *   4. helix_scan_encode on the shard with s0 = carry and ids = null.  The
 *      last shard's s1 is every sequence's final state.
 *
 * helix_scan_shard_state computes in d's precision path (compute_dtype,
 * backend) and needs helix_scan_shard_state_scratch_size() bytes of
 * 256-byte-aligned scratch (multipass is implied).  Both are enqueued on
 * `stream` and never synchronise or allocate.  The token-shard entry points
 * need scalar A (a_form HELIX_A_SCALAR_PER_HEAD): with a rate per state a
 * shard's decay is not one scalar per (seq, head), and they return
 * HELIX_ERR_UNSUPPORTED_SHAPE. */
size_t helix_scan_shard_state_scratch_size(helix_ctx* ctx, const helix_scan_desc* d);

helix_status helix_scan_shard_state(helix_ctx*             ctx,
                                    void*                  stream,
                                    const helix_scan_desc* d,
                                    helix_tensor           x,
                                    helix_tensor           dt,
                                    helix_tensor           A,
                                    helix_tensor           B,
                                    helix_tensor           C,
                                    helix_tensor           state,
                                    helix_tensor           log_decay,
                                    helix_tensor           scratch);

/* No counterpart in the reference.  Step 4 of the L-split above without a
 * second state pass: the scan of the shard (same d, x, dt, A, B, C as the
 * helix_scan_shard_state call) starting from `carry`, reading the run states
 * that call left in `scratch` (the same buffer, untouched since; its
 * contents are consumed, so call this once per shard-state call).  Writes y
 * and s1 like helix_scan_encode with s0 = carry and no ids. */
helix_status helix_scan_encode_shard(helix_ctx*             ctx,
                                     void*                  stream,
                                     const helix_scan_desc* d,
                                     helix_tensor           carry,
                                     helix_tensor           x,
                                     helix_tensor           dt,
                                     helix_tensor           A,
                                     helix_tensor           B,
                                     helix_tensor           C,
                                     helix_tensor           y,
                                     helix_tensor           s1,
                                     helix_tensor           scratch);

helix_status helix_scan_carry_combine(helix_ctx*             ctx,
                                      void*                  stream,
                                      const helix_scan_desc* d,
                                      helix_tensor           s0,
                                      helix_tensor           ids,
                                      helix_tensor           states,
                                      helix_tensor           log_decays,
                                      uint32_t               n_prev,
                                      helix_tensor           carry);

#ifdef __cplusplus
}
#endif

#endif /* HELIX_EXT_H */
