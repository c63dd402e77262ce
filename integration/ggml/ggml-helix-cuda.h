// ggml-helix-cuda.h -- HELIX interception point for ggml-cuda's SSM_SCAN.
//
// The CUDA counterpart of the reference's ggml-metal hook
// (reference integration/ggml/ggml-helix.h:1-30): one entry point, called
// from a single #ifdef at the top of ggml-cuda's SSM_SCAN op.  It returns
// false for anything HELIX cannot or should not serve, and the caller then
// runs its own kernel unchanged, so HELIX is never a regression.

#pragma once

#include <stdbool.h>

#ifdef __cplusplus
extern "C" {
#endif

struct ggml_tensor;

// `stream` is the cudaStream_t the op runs on and `device` its CUDA ordinal
// (the backend context's stream() and device at the call site).  Returns
// true if HELIX enqueued the op on `stream`; then y and the final state are
// in dst exactly where ggml's own kernel puts them.
bool ggml_cuda_op_ssm_scan_helix(void * stream, int device, const struct ggml_tensor * dst);

#ifdef __cplusplus
}
#endif
