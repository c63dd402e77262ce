/* helix.h -- public C ABI of the B200 (sm_100a) SSD scan library.
 *
 * This header is a source-compatible replacement for the HELIX C ABI
 * (reference include/helix/helix.h:1-224): the enums keep their values, the
 * two structs keep their field order and types, and the ten entry points keep
 * their names and argument lists, so a host that was written against HELIX
 * recompiles unchanged.  What changes is what the opaque handles mean:
 *
 *   helix_tensor.buf      a CUDA device pointer (any allocation the device can
 *                         address); .offset is still a byte offset from it.
 *   cmd_buffer / encoder  a cudaStream_t.  Work is enqueued on that stream and
 *                         ordered by it; the library never synchronises,
 *                         never allocates device memory and never frees it.
 *   device                NULL for the current device, else a pointer to an
 *                         int holding a CUDA device ordinal.
 *   metallib_path         ignored (kernels are compiled into the library).
 *
 * The op is the Mamba-2 / SSD selective-state-space scan over a prefill slice
 * (ggml's SSM_SCAN with a scalar decay per head).  Per (sequence, head,
 * channel p) with state s[n]:
 *
 *     dt_t = clamp(softplus(dt_raw[t,h]), dt_min, dt_max)
 *     s[n] = exp(A[h] * dt_t) * s[n] + dt_t * B[t,g,n] * x[t,h,p]
 *     y[t,h,p] = sum_n C[t,g,n] * s[n]          with g = h / (n_head/n_group)
 *
 * Tensor layouts (fastest dimension last):
 *   s0, s1 : (n_seq, n_head, head_dim, d_state)  f32
 *   x      : (n_seq, n_tok,  n_head,   head_dim) io_dtype
 *   dt     : (n_seq, n_tok,  n_head)             f32, bias already folded in
 *   A      : (n_head)                            f32
 *   B, C   : (n_seq, n_tok,  n_group,  d_state)  io_dtype
 *   y      : (n_seq, n_tok,  n_head,   head_dim) f32
 *   ids    : (n_seq) int32, optional: s0 row read for output sequence i
 *
 * y and the states are always f32 (ggml's SSM_SCAN destination is f32);
 * io_dtype only selects the storage type of the x, B and C operands.  The D
 * skip connection is not applied; that stays with the caller.
 */
#ifndef HELIX_H
#define HELIX_H

#include <stdbool.h>
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define HELIX_ABI_VERSION 1

/* ------------------------------------------------------------------------ */
/* Enums (values identical to reference helix.h:42-70)                      */
/* ------------------------------------------------------------------------ */

typedef enum {
    HELIX_OK = 0,
    HELIX_ERR_UNSUPPORTED_SHAPE = 1,  /* helix_scan_supported() is false     */
    HELIX_ERR_NO_DEVICE         = 2,  /* no sm_100 CUDA device               */
    HELIX_ERR_SCRATCH_TOO_SMALL = 3,
    HELIX_ERR_INVALID_ARG       = 4,
    HELIX_ERR_PIPELINE          = 5,  /* kernel configuration/launch failed  */
} helix_status;

typedef enum {
    HELIX_F32  = 0,
    HELIX_F16  = 1,
    HELIX_BF16 = 2,
} helix_dtype;

typedef enum {
    /* One decay scalar per head: Mamba-2 / SSD (the chunked tensor-core
     * families). */
    HELIX_A_SCALAR_PER_HEAD = 0,
    /* One decay per (head, state), A[h * s_a + n]: Mamba-1.  The reference
     * declines it; here it runs the per-state recurrence on the CUDA cores in
     * fp32 whatever the backend and compute_dtype (d_state <= 256), and the
     * token-shard entry points of helix_ext.h decline it. */
    HELIX_A_DIAG_PER_CHANNEL = 1,
} helix_a_form;

typedef enum {
    /* The names are kept for ABI compatibility.  On B200:
     *   MPP, or AUTO with compute_dtype BF16
     *       -> tcgen05 kernels, bf16 operands (F32-stored x, B, C rounded
     *          once), fp32 accumulators and carried state
     *   SGMMA, or AUTO with compute_dtype F32
     *       -> tcgen05 kernels at fp32-class accuracy: every fp32 operand as
     *          a bf16 pair hi + lo, each product as hi.hi + hi.lo + lo.hi,
     *          fp32 accumulators and carried state (F32-stored x, B, C,
     *          multipass; otherwise the exact kernels below run)
     *   REF -> exact fp32 CUDA-core kernels, for differential testing
     * (also the family for single pass with F32-stored x, B, C). */
    HELIX_BACKEND_AUTO  = 0,
    HELIX_BACKEND_SGMMA = 1,
    HELIX_BACKEND_MPP   = 2,
    HELIX_BACKEND_REF   = 3,
} helix_backend;

/* ------------------------------------------------------------------------ */
/* Tensors (reference helix.h:79-84)                                        */
/* ------------------------------------------------------------------------ */

/* A view into caller-owned device memory: `buf` is a device pointer and
 * `offset` a byte offset from it.  The library never frees either. */
typedef struct {
    void*    buf;
    uint64_t offset;
} helix_tensor;

#ifdef __cplusplus
#define HELIX_TENSOR_NULL (helix_tensor{ NULL, 0 })
#else
#define HELIX_TENSOR_NULL ((helix_tensor){ NULL, 0 })
#endif

static inline bool helix_tensor_is_null(helix_tensor t) { return t.buf == NULL; }

/* ------------------------------------------------------------------------ */
/* Descriptor (reference helix.h:95-131)                                    */
/* ------------------------------------------------------------------------ */

/* All strides are in ELEMENTS of the tensor's own storage type. */
typedef struct {
    int32_t n_tok;     /* L: tokens in this slice                          */
    int32_t n_seq;     /* independent sequences                            */
    int32_t n_head;    /* H                                                */
    int32_t head_dim;  /* P                                                */
    int32_t d_state;   /* N                                                */
    int32_t n_group;   /* G, must divide n_head                            */

    int64_t s_x[3];    /* (tok, head, chan)                                */
    int64_t s_b[3];    /* (tok, group, state)                              */
    int64_t s_c[3];    /* (tok, group, state)                              */
    int64_t s_dt[2];   /* (tok, head)                                      */
    int64_t s_s[3];    /* (head, chan, state) within one sequence          */
    int64_t s_y[3];    /* (tok, head, chan)                                */
    int64_t s_a;       /* stride between heads in A                        */
    int64_t seq_x;     /* per-sequence strides                             */
    int64_t seq_b;
    int64_t seq_c;
    int64_t seq_dt;
    int64_t seq_s;
    int64_t seq_y;

    int32_t       chunk;          /* 0 = library choice; the scan is exact for
                                     any chunk, so this is a hint          */
    helix_a_form  a_form;
    helix_dtype   io_dtype;       /* storage of x, B, C                    */
    helix_dtype   compute_dtype;  /* tensor-core operand precision         */
    helix_backend backend;
    bool          multipass;      /* false: one CTA per (seq, head, slab)
                                     walks the whole slice, zero scratch.
                                     true: the slice is cut into runs that
                                     are processed in parallel, with run
                                     states carried through scratch.       */

    float dt_min;                 /* softplus(dt) clamp; 0 / +inf = off    */
    float dt_max;
} helix_scan_desc;

/* Fills defaults and dense strides (reference src/runtime/desc.cpp:9-46). */
void helix_scan_desc_init(helix_scan_desc* d,
                          int32_t n_tok, int32_t n_seq, int32_t n_head,
                          int32_t head_dim, int32_t d_state, int32_t n_group);

/* ------------------------------------------------------------------------ */
/* Context (reference helix.h:148-164, src/runtime/device.mm:7-85)          */
/* ------------------------------------------------------------------------ */

typedef struct helix_ctx helix_ctx;

/* Binds to a CUDA device (`device` = NULL or int* ordinal), checks that it is
 * sm_100, and configures every kernel up front so that later calls mutate no
 * shared state.  Returns HELIX_ERR_NO_DEVICE when no suitable device exists. */
helix_status helix_ctx_create(helix_ctx** out, void* device, const char* metallib_path);
void         helix_ctx_free(helix_ctx* ctx);

/* Last error recorded on this context by the calling thread.  Never NULL. */
const char*  helix_ctx_last_error(const helix_ctx* ctx);

/* Backend AUTO resolves to for this descriptor (see helix_backend). */
helix_backend helix_ctx_select_backend(helix_ctx* ctx, const helix_scan_desc* d);

/* Static, human-readable name of the kernel variant the descriptor resolves
 * to, e.g. "tcgen05 (bf16 operands, fp32 state)".  Never NULL. */
const char* helix_ctx_backend_desc(helix_ctx* ctx, const helix_scan_desc* d);

/* ------------------------------------------------------------------------ */
/* Scan (reference helix.h:172-218)                                         */
/* ------------------------------------------------------------------------ */

/* True when a kernel exists for this descriptor on this device.  When false
 * the caller keeps its own implementation. */
bool helix_scan_supported(helix_ctx* ctx, const helix_scan_desc* d);

/* Bytes of device scratch the encode call needs (0 when multipass is false).
 * A pure function of (ctx, d); encode computes the identical plan. */
size_t helix_scan_scratch_size(helix_ctx* ctx, const helix_scan_desc* d);

/* Enqueues the scan on `cmd_buffer` (a cudaStream_t; NULL = legacy default
 * stream).  Never synchronises, never allocates.  `ids` may be
 * HELIX_TENSOR_NULL (identity).  `scratch` may be HELIX_TENSOR_NULL when
 * helix_scan_scratch_size() is 0.  On any error nothing is enqueued.
 * s0 and s1 must not overlap. */
helix_status helix_scan_encode(helix_ctx*             ctx,
                               void*                  cmd_buffer,
                               const helix_scan_desc* d,
                               helix_tensor           s0,
                               helix_tensor           x,
                               helix_tensor           dt,
                               helix_tensor           A,
                               helix_tensor           B,
                               helix_tensor           C,
                               helix_tensor           ids,
                               helix_tensor           y,
                               helix_tensor           s1,
                               helix_tensor           scratch);

/* Same as helix_scan_encode.  In Metal this form appended to an encoder the
 * caller already had open; a CUDA stream has no such distinction, so
 * `encoder` is the cudaStream_t a graph executor (ggml-cuda included) is
 * currently filling. */
helix_status helix_scan_encode_into(helix_ctx*             ctx,
                                    void*                  encoder,
                                    const helix_scan_desc* d,
                                    helix_tensor           s0,
                                    helix_tensor           x,
                                    helix_tensor           dt,
                                    helix_tensor           A,
                                    helix_tensor           B,
                                    helix_tensor           C,
                                    helix_tensor           ids,
                                    helix_tensor           y,
                                    helix_tensor           s1,
                                    helix_tensor           scratch);

#ifdef __cplusplus
}  /* extern "C" */
#endif

#endif  /* HELIX_H */
