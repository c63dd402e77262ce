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

#ifdef __cplusplus
}
#endif

#endif /* HELIX_EXT_H */
