// scan_static.cu -- helix_scan_encode_static: the multipass scan with its run
// scratch in a fixed device array owned by this library, for callers that
// cannot allocate device memory.
//
// Who needs it: hosts that hand an op nothing but its input and output
// buffers -- graph executors with a fixed memory plan and no per-op workspace,
// plugins loaded into a process whose device memory is owned by someone else,
// and code that runs where device allocation is forbidden after start-up.
// helix_scan_encode wants a caller-provided scratch buffer; those callers have
// no way to provide one.
//
// What it costs: the array below, kStaticScratchBytes (32 MiB) on each device.
// CUDA loads the code module that holds it (and reserves the 32 MiB) when the
// first call on a device asks for the array's address -- with lazy module
// loading, CUDA's default, not before.  From then on the device keeps it
// until the process exits.
//
// Rules for callers:
//   * Make the first call on each device at start-up, before any stream
//     capture: it loads the array.  If the device has no room left for it,
//     that call fails with HELIX_ERR_PIPELINE and says so, and nothing is
//     enqueued.
//   * Every call on a device uses the same array.  Two calls whose work can
//     overlap on the GPU (other streams, other threads, other contexts on the
//     same device) race on it and produce wrong results; serialise them.
//   * The array keeps whatever the last call left in it.  No part of it needs
//     to start at zero: each call's state kernel writes every run state, run
//     decay and run decay span, and its fast output kernel every tile flag,
//     before the same call's later kernels read them.
//   * A descriptor whose multipass scratch (helix_scan_scratch_size with
//     multipass = true) exceeds kStaticScratchBytes is rejected with
//     HELIX_ERR_SCRATCH_TOO_SMALL and a message; nothing is enqueued.
//   * Nothing here calls cudaMalloc, cudaFree or any allocating routine.
#include <cuda_runtime.h>

#include <string>

#include "../runtime/internal.h"
#include "helix/helix_ext.h"

namespace hx {
namespace {

constexpr size_t kStaticScratchBytes = (size_t)32 << 20;

static __device__ __align__(256) unsigned char g_static_scratch[kStaticScratchBytes];

}  // namespace
}  // namespace hx

extern "C" helix_status helix_scan_encode_static(helix_ctx* ctx, void* stream, const helix_scan_desc* desc,
                                                 helix_tensor s0, helix_tensor x, helix_tensor dt,
                                                 helix_tensor A, helix_tensor B, helix_tensor C,
                                                 helix_tensor ids, helix_tensor y, helix_tensor s1) {
    using namespace hx;
    if (!ctx || !desc) return HELIX_ERR_INVALID_ARG;
    if (!s0.buf || !x.buf || !dt.buf || !A.buf || !B.buf || !C.buf || !y.buf || !s1.buf) {
        set_error(ctx, "null tensor");
        return HELIX_ERR_INVALID_ARG;
    }
    // Always the multipass decomposition: that is the variant that needs scratch.
    helix_scan_desc d = *desc;
    d.multipass = true;
    std::string why;
    if (!supported_impl(ctx, d, &why)) {
        set_error(ctx, why);
        return HELIX_ERR_UNSUPPORTED_SHAPE;
    }
    const Plan pl = make_plan(ctx, d);
    if (pl.total > kStaticScratchBytes) {
        set_error(ctx, "helix_scan_encode_static: this descriptor needs " + std::to_string(pl.total) +
                           " bytes of run scratch; the built-in array holds " +
                           std::to_string(kStaticScratchBytes) +
                           " (use helix_scan_encode with caller scratch)");
        return HELIX_ERR_SCRATCH_TOO_SMALL;
    }
    ScanParams p{};
    const CallTensors t{s0, x, dt, A, B, C, ids, y, s1};
    const helix_status st = bind_call(ctx, d, pl, t, &p);
    if (st != HELIX_OK) return st;

    // The array's device address on ctx's device, looked up on every call
    // (cheap once the module is loaded; a cached address would dangle after
    // a device reset reloads the module elsewhere).  The lookup needs the
    // device current.
    int prev = -1;
    cudaGetDevice(&prev);
    if (prev != ctx->device) cudaSetDevice(ctx->device);
    void* scratch = nullptr;
    const cudaError_t se = cudaGetSymbolAddress(&scratch, g_static_scratch);
    if (prev >= 0 && prev != ctx->device) cudaSetDevice(prev);
    if (se != cudaSuccess) {
        cudaGetLastError();
        set_error(ctx, se == cudaErrorMemoryAllocation
                           ? std::string("helix_scan_encode_static: out of device memory loading its ") +
                                 std::to_string(kStaticScratchBytes >> 20) +
                                 " MiB scratch array (make the first call at start-up)"
                           : std::string("cudaGetSymbolAddress failed: ") + cudaGetErrorString(se));
        return HELIX_ERR_PIPELINE;
    }
    bind_scratch(pl, static_cast<char*>(scratch), &p);
    return run_call(ctx, pl, p, stream);
}
