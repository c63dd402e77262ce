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

// Byte extent [lo, hi) touched by n_rows rows of a state tensor of d.
void state_extent(const helix_scan_desc& d, const void* base, int64_t n_rows, uintptr_t* lo, uintptr_t* hi) {
    const int64_t last = (n_rows - 1) * d.seq_s + (int64_t)(d.n_head - 1) * d.s_s[0] +
                         (int64_t)(d.head_dim - 1) * d.s_s[1] + (int64_t)(d.d_state - 1);
    *lo = reinterpret_cast<uintptr_t>(base);
    *hi = *lo + (uintptr_t)(last + 1) * sizeof(float);
}

using range_fn = CUresult (*)(CUdeviceptr*, size_t*, CUdeviceptr);

range_fn address_range_fn() {
    static range_fn fn = [] {
        void* f = nullptr;
        cudaDriverEntryPointQueryResult q{};
        if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &f, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess) {
            cudaGetLastError();
            return (range_fn) nullptr;
        }
        return reinterpret_cast<range_fn>(f);
    }();
    return fn;
}

// [base, end) of the driver allocation holding p; false when the driver does
// not know p (host memory, or no driver entry point).
bool allocation_of(const void* p, uintptr_t* base, uintptr_t* end) {
    const range_fn fn = address_range_fn();
    if (!fn) return false;
    CUdeviceptr b = 0;
    size_t size = 0;
    if (fn(&b, &size, reinterpret_cast<CUdeviceptr>(p)) != CUDA_SUCCESS) return false;
    *base = (uintptr_t)b;
    *end = (uintptr_t)b + size;
    return true;
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
        if (!hx::scratch_fits(at<char>(scratch), pl.total)) {
            hx::set_error(ctx, "scratch allocation smaller than helix_scan_scratch_size()");
            return HELIX_ERR_SCRATCH_TOO_SMALL;
        }
    }
    hx::ScanParams p{};
    const hx::CallTensors t{s0, x, dt, A, B, C, ids, y, s1};
    const helix_status st = hx::bind_call(ctx, *d, pl, t, &p);
    if (st != HELIX_OK) return st;
    if (pl.total > 0) hx::bind_scratch(pl, at<char>(scratch), &p);
    return hx::run_call(ctx, pl, p, stream);
}

}  // namespace

namespace hx {

bool scratch_fits(const void* s, size_t need) {
    uintptr_t base = 0, end = 0;
    if (!allocation_of(s, &base, &end)) return true;  // unknown: cannot check
    return reinterpret_cast<uintptr_t>(s) + need <= end;
}

bool states_overlap(const helix_scan_desc& d, const void* s0, const void* s1) {
    uintptr_t a0, a1, b0, b1;
    state_extent(d, s0, d.n_seq, &a0, &a1);
    state_extent(d, s1, d.n_seq, &b0, &b1);
    return a0 < b1 && b0 < a1;
}

helix_status bind_call(helix_ctx* ctx, const helix_scan_desc& d, const Plan& pl, const CallTensors& t,
                       ScanParams* out) {
    if (!t.s0.buf || !t.x.buf || !t.dt.buf || !t.A.buf || !t.B.buf || !t.C.buf || !t.y.buf || !t.s1.buf) {
        set_error(ctx, "null tensor");
        return HELIX_ERR_INVALID_ARG;
    }
    // s0 is read while s1 is written by other CTAs of the same launch.  Rows
    // that only ids reaches are checked by the kernels that read them
    // (kFaultIdsOverlap: that sequence comes out NaN).
    if (states_overlap(d, at<char>(t.s0), at<char>(t.s1))) {
        set_error(ctx, "s0 and s1 overlap");
        return HELIX_ERR_INVALID_ARG;
    }
    ScanParams& p = *out;
    p = ScanParams{};
    fill_params(p, d, pl);
    p.has_ids = t.ids.buf ? 1 : 0;
    p.x = at<void>(t.x);
    p.dt = at<float>(t.dt);
    p.A = at<float>(t.A);
    p.B = at<void>(t.B);
    p.C = at<void>(t.C);
    p.ids = t.ids.buf ? at<int32_t>(t.ids) : nullptr;
    p.s0 = at<float>(t.s0);
    p.y = at<float>(t.y);
    p.s1 = at<float>(t.s1);
    p.fault = ctx->fault_word;
    if (pl.path == kPathTcBf16 && !pl.cast) {
        // TMA needs 16-byte aligned global bases.
        const uintptr_t m = reinterpret_cast<uintptr_t>(p.x) | reinterpret_cast<uintptr_t>(p.B) |
                            reinterpret_cast<uintptr_t>(p.C);
        if (m & 15) {
            set_error(ctx, "x, B and C must be 16-byte aligned for the tensor-core path");
            return HELIX_ERR_UNSUPPORTED_SHAPE;
        }
    }
    if (pl.path == kPathTcX3 && pl.x_copy == 0 && (reinterpret_cast<uintptr_t>(p.x) & 15) != 0) {
        // TMA reads x in place
        set_error(ctx, "x must be 16-byte aligned for the tensor-core fp32 path");
        return HELIX_ERR_UNSUPPORTED_SHAPE;
    }
    return HELIX_OK;
}

void bind_scratch(const Plan& pl, char* base, ScanParams* p) {
    p->agg = reinterpret_cast<float*>(base + pl.off_agg);
    p->lam = reinterpret_cast<float*>(base + pl.off_lam);
    p->tile_flag = pl.has_flags ? reinterpret_cast<int32_t*>(base + pl.off_flag) : nullptr;
    p->run_span = pl.has_span ? reinterpret_cast<float*>(base + pl.off_span) : nullptr;
    if (pl.cast) {
        p->cast_x = base + pl.off_xc;
        p->cast_b = base + pl.off_bc;
        p->cast_c = base + pl.off_cc;
    }
    if (pl.cast_lo) {
        p->cast_bl = base + pl.off_bl;
        p->cast_cl = base + pl.off_cl;
    }
}

helix_status run_call(helix_ctx* ctx, const Plan& pl, const ScanParams& p, void* stream) {
    int dev_prev = -1;
    cudaGetDevice(&dev_prev);
    if (dev_prev != ctx->device) cudaSetDevice(ctx->device);
    const int rc = pl.path == kPathTcBf16 ? launch_tc(ctx, pl, p, stream)
                   : pl.path == kPathTcX3 ? launch_tc3(ctx, pl, p, stream)
                   : pl.path == kPathDiag ? launch_diag(ctx, pl, p, stream)
                                          : launch_simt(ctx, pl, p, stream);
    if (dev_prev >= 0 && dev_prev != ctx->device) cudaSetDevice(dev_prev);
    if (rc != cudaSuccess) {
        set_error(ctx, std::string("kernel launch failed: ") + cudaGetErrorString(static_cast<cudaError_t>(rc)));
        return HELIX_ERR_PIPELINE;
    }
    return HELIX_OK;
}

}  // namespace hx

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
    p.n_half = (d.d_state + 127) / 128;
    p.n_base = 0;
    p.y_add = 0;
    p.dt_min = d.dt_min;
    p.dt_max = d.dt_max;
    p.s_x0 = d.s_x[0]; p.s_x1 = d.s_x[1]; p.s_x2 = d.s_x[2]; p.seq_x = d.seq_x;
    p.s_b0 = d.s_b[0]; p.s_b1 = d.s_b[1]; p.seq_b = d.seq_b;
    p.s_c0 = d.s_c[0]; p.s_c1 = d.s_c[1]; p.seq_c = d.seq_c;
    p.s_dt0 = d.s_dt[0]; p.s_dt1 = d.s_dt[1]; p.seq_dt = d.seq_dt;
    p.s_s0 = d.s_s[0]; p.s_s1 = d.s_s[1]; p.seq_s = d.seq_s;
    p.s_y0 = d.s_y[0]; p.s_y1 = d.s_y[1]; p.s_y2 = d.s_y[2]; p.seq_y = d.seq_y;
    p.s_a = d.s_a;
    p.x_copy = pl.x_copy;
    const int64_t row = (int64_t)(d.n_head - 1) * d.s_s[0] + (int64_t)(d.head_dim - 1) * d.s_s[1] + d.d_state;
    p.s_row_bytes = row * (int64_t)sizeof(float);
    p.s1_bytes = ((int64_t)(d.n_seq - 1) * d.seq_s + row) * (int64_t)sizeof(float);
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
