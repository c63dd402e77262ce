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
// What it costs: the array below, kStaticScratchBytes (32 MiB), lives on every
// GPU that loads this library until the process exits, whether or not the
// entry point is ever called.
//
// Rules for callers:
//   * The first call on a device looks up the array's device address with
//     cudaGetSymbolAddress (with that device current).  Make that first call
//     before any stream capture.
//   * Every call on a device uses the same array.  Two calls whose work can
//     overlap on the GPU (other streams, other threads, other contexts on the
//     same device) race on it and produce wrong results; serialise them.
//   * The array keeps whatever the last call left in it.  No part of it needs
//     to start at zero: each call's state kernel writes every run state and
//     run decay before the same call's output kernel reads them.
//   * A descriptor whose multipass scratch (helix_scan_scratch_size with
//     multipass = true) exceeds kStaticScratchBytes is rejected with
//     HELIX_ERR_SCRATCH_TOO_SMALL and a message; nothing is enqueued.
//   * Nothing here calls cudaMalloc, cudaFree or any allocating routine.
#include <cuda_runtime.h>

#include <mutex>
#include <string>

#include "../runtime/internal.h"
#include "helix/helix_ext.h"

namespace hx {
namespace {

constexpr size_t kStaticScratchBytes = (size_t)32 << 20;
constexpr int kMaxDevices = 64;

static __device__ __align__(256) unsigned char g_static_scratch[kStaticScratchBytes];

std::mutex g_static_mu;
void* g_static_ptr[kMaxDevices] = {};

// Device address of g_static_scratch on `dev` (which must be current).
// Looked up once per device.
cudaError_t static_scratch_on(int dev, void** out) {
    if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
    std::lock_guard<std::mutex> lk(g_static_mu);
    if (!g_static_ptr[dev]) {
        void* ptr = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&ptr, g_static_scratch);
        if (e != cudaSuccess) return e;
        g_static_ptr[dev] = ptr;
    }
    *out = g_static_ptr[dev];
    return cudaSuccess;
}

template <class T>
T* at(helix_tensor t) {
    return reinterpret_cast<T*>(static_cast<char*>(t.buf) + t.offset);
}

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
    {
        const uintptr_t a0 = reinterpret_cast<uintptr_t>(at<char>(s0));
        const uintptr_t b0 = reinterpret_cast<uintptr_t>(at<char>(s1));
        const int64_t last = (int64_t)(d.n_seq - 1) * d.seq_s + (int64_t)(d.n_head - 1) * d.s_s[0] +
                             (int64_t)(d.head_dim - 1) * d.s_s[1] + (int64_t)(d.d_state - 1);
        const uintptr_t span = (uintptr_t)(last + 1) * sizeof(float);
        if (a0 < b0 + span && b0 < a0 + span) {
            set_error(ctx, "s0 and s1 overlap");
            return HELIX_ERR_INVALID_ARG;
        }
    }
    if (pl.path == kPathTcBf16) {
        const uintptr_t m = reinterpret_cast<uintptr_t>(at<char>(x)) | reinterpret_cast<uintptr_t>(at<char>(B)) |
                            reinterpret_cast<uintptr_t>(at<char>(C));
        if (m & 15) {
            set_error(ctx, "x, B and C must be 16-byte aligned for the tensor-core path");
            return HELIX_ERR_UNSUPPORTED_SHAPE;
        }
    }

    int prev = -1;
    cudaGetDevice(&prev);
    if (prev != ctx->device) cudaSetDevice(ctx->device);
    void* scratch = nullptr;
    const cudaError_t se = static_scratch_on(ctx->device, &scratch);
    if (se != cudaSuccess) {
        if (prev >= 0 && prev != ctx->device) cudaSetDevice(prev);
        set_error(ctx, std::string("cudaGetSymbolAddress failed: ") + cudaGetErrorString(se));
        return HELIX_ERR_PIPELINE;
    }

    ScanParams p{};
    fill_params(p, d, pl);
    p.has_ids = ids.buf ? 1 : 0;
    p.x = at<void>(x);
    p.dt = at<float>(dt);
    p.A = at<float>(A);
    p.B = at<void>(B);
    p.C = at<void>(C);
    p.ids = ids.buf ? at<int32_t>(ids) : nullptr;
    p.s0 = at<float>(s0);
    p.y = at<float>(y);
    p.s1 = at<float>(s1);
    p.agg = reinterpret_cast<float*>(static_cast<char*>(scratch) + pl.off_agg);
    p.lam = reinterpret_cast<float*>(static_cast<char*>(scratch) + pl.off_lam);
    p.tile_flag = pl.has_flags ? reinterpret_cast<int32_t*>(static_cast<char*>(scratch) + pl.off_flag) : nullptr;
    p.run_span = pl.has_span ? reinterpret_cast<float*>(static_cast<char*>(scratch) + pl.off_span) : nullptr;

    const int rc = pl.path == kPathTcBf16 ? launch_tc(ctx, pl, p, stream) : launch_simt(ctx, pl, p, stream);
    if (prev >= 0 && prev != ctx->device) cudaSetDevice(prev);
    if (rc != cudaSuccess) {
        set_error(ctx, std::string("kernel launch failed: ") + cudaGetErrorString(static_cast<cudaError_t>(rc)));
        return HELIX_ERR_PIPELINE;
    }
    return HELIX_OK;
}
