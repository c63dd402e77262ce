// dispatch.cpp -- the encoder.
//
// Replaces reference src/runtime/dispatch.mm:55-287.  Validates the call,
// resolves the plan, fills the kernel parameter block and enqueues one or two
// kernels on the caller's stream.  It never synchronises and never allocates;
// stream order replaces the reference's inter-pass Metal barriers.
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdlib>
#include <string>

#include "internal.h"

namespace {

template <class T>
T* at(helix_tensor t) {
    return reinterpret_cast<T*>(static_cast<char*>(t.buf) + t.offset);
}

// Byte extent [lo, hi) touched by a state tensor of this descriptor.
void state_extent(const helix_scan_desc& d, helix_tensor t, int64_t n_rows, uintptr_t* lo,
                  uintptr_t* hi) {
    const int64_t last = (n_rows - 1) * d.seq_s + (int64_t)(d.n_head - 1) * d.s_s[0] +
                         (int64_t)(d.head_dim - 1) * d.s_s[1] + (int64_t)(d.d_state - 1);
    *lo = reinterpret_cast<uintptr_t>(at<char>(t));
    *hi = *lo + (uintptr_t)(last + 1) * sizeof(float);
}

// Best-effort size check of the caller's scratch: when the driver knows the
// allocation containing it, the plan must fit inside that allocation.
bool scratch_fits(helix_tensor s, size_t need) {
    using range_fn = CUresult (*)(CUdeviceptr*, size_t*, CUdeviceptr);
    static range_fn fn = [] {
        void* f = nullptr;
        cudaDriverEntryPointQueryResult q{};
        if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &f, cudaEnableDefault, &q) !=
                cudaSuccess ||
            q != cudaDriverEntryPointSuccess) {
            cudaGetLastError();
            return (range_fn) nullptr;
        }
        return reinterpret_cast<range_fn>(f);
    }();
    if (!fn) return true;
    CUdeviceptr base = 0;
    size_t size = 0;
    const CUdeviceptr p = reinterpret_cast<CUdeviceptr>(at<char>(s));
    if (fn(&base, &size, p) != CUDA_SUCCESS) return true;  // unknown: cannot check
    return p + need <= base + size;
}

helix_status encode_core(helix_ctx* ctx, void* stream, const helix_scan_desc* d, helix_tensor s0,
                         helix_tensor x, helix_tensor dt, helix_tensor A, helix_tensor B,
                         helix_tensor C, helix_tensor ids, helix_tensor y, helix_tensor s1,
                         helix_tensor scratch) {
    if (!ctx || !d) return HELIX_ERR_INVALID_ARG;
    if (!s0.buf || !x.buf || !dt.buf || !A.buf || !B.buf || !C.buf || !y.buf || !s1.buf) {
        hx::set_error(ctx, "null tensor");
        return HELIX_ERR_INVALID_ARG;
    }
    std::string why;
    if (!hx::supported_impl(ctx, *d, &why)) {
        hx::set_error(ctx, why);
        return HELIX_ERR_UNSUPPORTED_SHAPE;
    }

    const hx::Plan pl = hx::make_plan(ctx, *d);
    if (pl.total > 0) {
        if (!scratch.buf) {
            hx::set_error(ctx, "multipass requires a scratch buffer");
            return HELIX_ERR_SCRATCH_TOO_SMALL;
        }
        if ((reinterpret_cast<uintptr_t>(at<char>(scratch)) & 255) != 0) {
            hx::set_error(ctx, "scratch must be 256-byte aligned");
            return HELIX_ERR_INVALID_ARG;
        }
        if (!scratch_fits(scratch, pl.total)) {
            hx::set_error(ctx, "scratch allocation smaller than helix_scan_scratch_size()");
            return HELIX_ERR_SCRATCH_TOO_SMALL;
        }
    }

    // s0 is read while s1 is written by other CTAs of the same launch.
    {
        uintptr_t a0, a1, b0, b1;
        int64_t src_rows = d->n_seq;
        state_extent(*d, s0, src_rows, &a0, &a1);
        state_extent(*d, s1, d->n_seq, &b0, &b1);
        if (a0 < b1 && b0 < a1) {
            hx::set_error(ctx, "s0 and s1 overlap");
            return HELIX_ERR_INVALID_ARG;
        }
    }

    hx::ScanParams p{};
    hx::fill_params(p, *d, pl);
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
    if (pl.total > 0) {
        p.agg = reinterpret_cast<float*>(at<char>(scratch) + pl.off_agg);
        p.lam = reinterpret_cast<float*>(at<char>(scratch) + pl.off_lam);
        p.tile_flag = pl.has_flags ? reinterpret_cast<int32_t*>(at<char>(scratch) + pl.off_flag) : nullptr;
        p.run_span = pl.has_span ? reinterpret_cast<float*>(at<char>(scratch) + pl.off_span) : nullptr;
    }

    if (pl.path == hx::kPathTcBf16) {
        // TMA needs 16-byte aligned global bases.
        const uintptr_t m = reinterpret_cast<uintptr_t>(p.x) | reinterpret_cast<uintptr_t>(p.B) |
                            reinterpret_cast<uintptr_t>(p.C);
        if (m & 15) {
            hx::set_error(ctx, "x, B and C must be 16-byte aligned for the tensor-core path");
            return HELIX_ERR_UNSUPPORTED_SHAPE;
        }
    }

    int dev_prev = -1;
    cudaGetDevice(&dev_prev);
    if (dev_prev != ctx->device) cudaSetDevice(ctx->device);
    const int rc = pl.path == hx::kPathTcBf16 ? hx::launch_tc(ctx, pl, p, stream)
                                               : hx::launch_simt(ctx, pl, p, stream);
    if (dev_prev >= 0 && dev_prev != ctx->device) cudaSetDevice(dev_prev);
    if (rc != cudaSuccess) {
        hx::set_error(ctx, std::string("kernel launch failed: ") +
                               cudaGetErrorString(static_cast<cudaError_t>(rc)));
        return HELIX_ERR_PIPELINE;
    }
    return HELIX_OK;
}

}  // namespace

namespace hx {

void fill_params(ScanParams& p, const helix_scan_desc& d, const Plan& pl) {
    p.S = d.n_seq;
    p.L = d.n_tok;
    p.H = d.n_head;
    p.P = d.head_dim;
    p.N = d.d_state;
    p.G = d.n_group;
    p.hpg = d.n_head / d.n_group;
    p.n_pslab = pl.n_pslab;
    p.run_tok = pl.run_tok;
    p.n_runs = pl.n_runs;
    p.out_k = pl.out_k;
    p.n_out = pl.n_out;
    p.state_runs = pl.state_runs;
    p.run_slots = pl.run_slots;
    {
        const int units = p.hpg * p.n_pslab;
        p.n_pair = (units + 1) / 2;
    }
    p.io_bf16 = d.io_dtype == HELIX_BF16 ? 1 : 0;
    p.dt_min = d.dt_min;
    p.dt_max = d.dt_max;
    p.s_x0 = d.s_x[0]; p.s_x1 = d.s_x[1]; p.s_x2 = d.s_x[2]; p.seq_x = d.seq_x;
    p.s_b0 = d.s_b[0]; p.s_b1 = d.s_b[1]; p.seq_b = d.seq_b;
    p.s_c0 = d.s_c[0]; p.s_c1 = d.s_c[1]; p.seq_c = d.seq_c;
    p.s_dt0 = d.s_dt[0]; p.s_dt1 = d.s_dt[1]; p.seq_dt = d.seq_dt;
    p.s_s0 = d.s_s[0]; p.s_s1 = d.s_s[1]; p.seq_s = d.seq_s;
    p.s_y0 = d.s_y[0]; p.s_y1 = d.s_y[1]; p.s_y2 = d.s_y[2]; p.seq_y = d.seq_y;
    p.s_a = d.s_a;
}

}  // namespace hx

extern "C" helix_status helix_scan_encode(helix_ctx* ctx, void* cmd_buffer,
                                          const helix_scan_desc* d, helix_tensor s0,
                                          helix_tensor x, helix_tensor dt, helix_tensor A,
                                          helix_tensor B, helix_tensor C, helix_tensor ids,
                                          helix_tensor y, helix_tensor s1, helix_tensor scratch) {
    return encode_core(ctx, cmd_buffer, d, s0, x, dt, A, B, C, ids, y, s1, scratch);
}

extern "C" helix_status helix_scan_encode_into(helix_ctx* ctx, void* encoder,
                                               const helix_scan_desc* d, helix_tensor s0,
                                               helix_tensor x, helix_tensor dt, helix_tensor A,
                                               helix_tensor B, helix_tensor C, helix_tensor ids,
                                               helix_tensor y, helix_tensor s1,
                                               helix_tensor scratch) {
    return encode_core(ctx, encoder, d, s0, x, dt, A, B, C, ids, y, s1, scratch);
}
