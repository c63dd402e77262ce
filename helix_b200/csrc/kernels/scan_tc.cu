// scan_tc.cu -- tcgen05 (bf16 operand) kernel family.  Placeholder until the
// tensor-core kernels land: reports "not configured" so helix_scan_supported()
// declines the bf16 path instead of running anything.
#include <cuda_runtime.h>

#include "common.cuh"

namespace hx {
int configure_tc(const helix_ctx*) { return cudaErrorNotSupported; }
int launch_tc(const helix_ctx*, const Plan&, const ScanParams&, void*) { return cudaErrorNotSupported; }
}  // namespace hx
