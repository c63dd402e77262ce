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
 * GPU.  *code is 0 when no wait expired.  Synchronous (it copies one word). */
helix_status helix_device_fault(helix_ctx* ctx, uint32_t* code);

/* No counterpart in the reference.  The multipass scan for callers that
 * cannot allocate device memory: hosts that give an op only its input and
 * output buffers (graph executors with a fixed memory plan and no per-op
 * workspace, plugins inside a process that owns all device memory, code that
 * may not allocate after start-up).  Same arguments and results as
 * helix_scan_encode with multipass forced on, minus `scratch`: the run
 * scratch lives in a 32 MiB array inside the library, present on every GPU
 * that loads the library until the process exits.
 *   - Descriptors needing more than 32 MiB of run scratch are rejected with
 *     HELIX_ERR_SCRATCH_TOO_SMALL (message in helix_ctx_last_error);
 *     nothing is enqueued.
 *   - The first call on a device looks up the array's address
 *     (cudaGetSymbolAddress); make that first call before any stream capture.
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

#ifdef __cplusplus
}
#endif

#endif /* HELIX_EXT_H */
