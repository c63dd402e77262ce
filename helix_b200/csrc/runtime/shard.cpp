// shard.cpp -- entry points of the sequence-split (L-split) scan.
//
// No reference counterpart: HELIX encodes one scan on one Metal device.  On
// B200 one sequence's tokens can be cut into contiguous shards, one per GPU.
// Rank k then
//   1. reduces its shard to the state it would leave from a zero start and
//      the shard's total log-decay (helix_scan_shard_state),
//   2. receives those pairs from ranks 0..k-1 (an all-gather in the caller's
//      communicator) and folds them, starting from the sequence's initial
//      state, into the state entering its shard (helix_scan_carry_combine),
//   3. runs the ordinary scan on its shard with that carry as s0.
// The last shard's s1 is the sequence's final state.  Step 3 is exact by
// definition of s0; steps 1-2 reassociate the state recurrence over shards.
#include <cuda_runtime.h>

#include <string>

#include "helix/helix_ext.h"
#include "internal.h"

namespace {

template <class T>
T* at(helix_tensor t) {
    return reinterpret_cast<T*>(static_cast<char*>(t.buf) + t.offset);
}

struct DeviceScope {
    int prev = -1;
    explicit DeviceScope(int dev) {
        cudaGetDevice(&prev);
        if (prev != dev) cudaSetDevice(dev);
    }
    ~DeviceScope() {
        int cur = -1;
        cudaGetDevice(&cur);
        if (prev >= 0 && cur != prev) cudaSetDevice(prev);
    }
};

helix_status launch_error(helix_ctx* ctx, int rc) {
    hx::set_error(ctx, std::string("kernel launch failed: ") + cudaGetErrorString(static_cast<cudaError_t>(rc)));
    return HELIX_ERR_PIPELINE;
}

}  // namespace

extern "C" size_t helix_scan_shard_state_scratch_size(helix_ctx* ctx, const helix_scan_desc* d) {
    if (!d) return 0;
    return hx::make_shard_plan(ctx, *d).total;
}

extern "C" helix_status helix_scan_shard_state(helix_ctx* ctx, void* stream, const helix_scan_desc* d,
                                               helix_tensor x, helix_tensor dt, helix_tensor A, helix_tensor B,
                                               helix_tensor C, helix_tensor state, helix_tensor log_decay,
                                               helix_tensor scratch) {
    if (!ctx || !d) return HELIX_ERR_INVALID_ARG;
    if (!x.buf || !dt.buf || !A.buf || !B.buf || !C.buf || !state.buf || !log_decay.buf || !scratch.buf) {
        hx::set_error(ctx, "null tensor");
        return HELIX_ERR_INVALID_ARG;
    }
    helix_scan_desc m = *d;
    m.multipass = true;
    std::string why;
    if (!hx::supported_impl(ctx, m, &why)) {
        hx::set_error(ctx, why);
        return HELIX_ERR_UNSUPPORTED_SHAPE;
    }
    if (m.a_form != HELIX_A_SCALAR_PER_HEAD) {
        // a shard's decay is one scalar per (seq, head) only for scalar A
        hx::set_error(ctx, "token sharding needs scalar A");
        return HELIX_ERR_UNSUPPORTED_SHAPE;
    }
    const hx::Plan pl = hx::make_shard_plan(ctx, m);
    if ((reinterpret_cast<uintptr_t>(at<char>(scratch)) & 255) != 0) {
        hx::set_error(ctx, "scratch must be 256-byte aligned");
        return HELIX_ERR_INVALID_ARG;
    }
    if (!hx::scratch_fits(at<char>(scratch), pl.total)) {
        hx::set_error(ctx, "scratch allocation smaller than helix_scan_shard_state_scratch_size()");
        return HELIX_ERR_SCRATCH_TOO_SMALL;
    }
    hx::ScanParams p{};
    hx::fill_params(p, m, pl);
    p.x = at<void>(x);
    p.dt = at<float>(dt);
    p.A = at<float>(A);
    p.B = at<void>(B);
    p.C = at<void>(C);
    hx::bind_scratch(pl, at<char>(scratch), &p);
    p.fault = ctx->fault_word;
    if (pl.path == hx::kPathTcBf16 && !pl.cast) {
        const uintptr_t a = reinterpret_cast<uintptr_t>(p.x) | reinterpret_cast<uintptr_t>(p.B) |
                            reinterpret_cast<uintptr_t>(p.C);
        if (a & 15) {
            hx::set_error(ctx, "x, B and C must be 16-byte aligned for the tensor-core path");
            return HELIX_ERR_UNSUPPORTED_SHAPE;
        }
    }
    if (pl.path == hx::kPathTcX3 && pl.x_copy == 0 && (reinterpret_cast<uintptr_t>(p.x) & 15) != 0) {
        hx::set_error(ctx, "x must be 16-byte aligned for the tensor-core fp32 path");
        return HELIX_ERR_UNSUPPORTED_SHAPE;
    }
    DeviceScope ds(ctx->device);
    int rc = pl.path == hx::kPathTcBf16 ? hx::launch_tc_states(ctx, pl, p, stream)
             : pl.path == hx::kPathTcX3 ? hx::launch_tc3_states(ctx, pl, p, stream)
                                        : hx::launch_simt_states(ctx, pl, p, stream);
    if (rc == cudaSuccess) rc = hx::launch_shard_fold(p, at<float>(state), at<float>(log_decay), stream);
    if (rc != cudaSuccess) return launch_error(ctx, rc);
    return HELIX_OK;
}

extern "C" helix_status helix_scan_carry_combine(helix_ctx* ctx, void* stream, const helix_scan_desc* d,
                                                 helix_tensor s0, helix_tensor ids, helix_tensor states,
                                                 helix_tensor log_decays, uint32_t n_prev, helix_tensor carry) {
    if (!ctx || !d) return HELIX_ERR_INVALID_ARG;
    if (!s0.buf || !carry.buf || (n_prev > 0 && (!states.buf || !log_decays.buf))) {
        hx::set_error(ctx, "null tensor");
        return HELIX_ERR_INVALID_ARG;
    }
    if (d->n_seq <= 0 || d->n_head <= 0 || d->head_dim <= 0 || d->d_state <= 0 || d->s_s[2] != 1) {
        hx::set_error(ctx, "bad state shape or innermost state stride != 1");
        return HELIX_ERR_UNSUPPORTED_SHAPE;
    }
    if (d->a_form != HELIX_A_SCALAR_PER_HEAD) {
        hx::set_error(ctx, "token sharding needs scalar A");
        return HELIX_ERR_UNSUPPORTED_SHAPE;
    }
    if (hx::states_overlap(*d, at<char>(s0), at<char>(carry))) {
        hx::set_error(ctx, "s0 and carry overlap");
        return HELIX_ERR_INVALID_ARG;
    }
    hx::Plan pl{};
    hx::ScanParams p{};
    hx::fill_params(p, *d, pl);
    p.has_ids = ids.buf ? 1 : 0;
    p.ids = ids.buf ? at<int32_t>(ids) : nullptr;
    p.s0 = at<float>(s0);
    p.s1 = at<float>(carry);  // the rows written, for the device-side ids check
    p.fault = ctx->fault_word;
    DeviceScope ds(ctx->device);
    const int rc = hx::launch_carry_combine(p, n_prev ? at<float>(states) : nullptr,
                                            n_prev ? at<float>(log_decays) : nullptr, (int)n_prev,
                                            at<float>(carry), stream);
    if (rc != cudaSuccess) return launch_error(ctx, rc);
    return HELIX_OK;
}

extern "C" helix_status helix_scan_encode_shard(helix_ctx* ctx, void* stream, const helix_scan_desc* d,
                                                helix_tensor carry, helix_tensor x, helix_tensor dt, helix_tensor A,
                                                helix_tensor B, helix_tensor C, helix_tensor y, helix_tensor s1,
                                                helix_tensor scratch) {
    if (!ctx || !d) return HELIX_ERR_INVALID_ARG;
    if (!carry.buf || !x.buf || !dt.buf || !A.buf || !B.buf || !C.buf || !y.buf || !s1.buf || !scratch.buf) {
        hx::set_error(ctx, "null tensor");
        return HELIX_ERR_INVALID_ARG;
    }
    helix_scan_desc m = *d;
    m.multipass = true;
    std::string why;
    if (!hx::supported_impl(ctx, m, &why)) {
        hx::set_error(ctx, why);
        return HELIX_ERR_UNSUPPORTED_SHAPE;
    }
    if (m.a_form != HELIX_A_SCALAR_PER_HEAD) {
        // a shard's decay is one scalar per (seq, head) only for scalar A
        hx::set_error(ctx, "token sharding needs scalar A");
        return HELIX_ERR_UNSUPPORTED_SHAPE;
    }
    hx::Plan pl = hx::make_plan(ctx, m);
    const hx::Plan sp = hx::make_shard_plan(ctx, m);
    if ((reinterpret_cast<uintptr_t>(at<char>(scratch)) & 255) != 0) {
        hx::set_error(ctx, "scratch must be 256-byte aligned");
        return HELIX_ERR_INVALID_ARG;
    }
    if (!hx::scratch_fits(at<char>(scratch), sp.total)) {
        hx::set_error(ctx, "scratch allocation smaller than helix_scan_shard_state_scratch_size()");
        return HELIX_ERR_SCRATCH_TOO_SMALL;
    }
    hx::ScanParams p{};
    const hx::CallTensors t{carry, x, dt, A, B, C, helix_tensor{nullptr, 0}, y, s1};
    const helix_status st = hx::bind_call(ctx, m, pl, t, &p);
    if (st != HELIX_OK) return st;
    // the shard-state call's layout: a state, decay and decay span for every
    // run, of which the scan's carry reads the runs before its last span
    hx::bind_scratch(sp, at<char>(scratch), &p);
    p.run_slots = sp.run_slots;
    pl.states_ready = true;
    return hx::run_call(ctx, pl, p, stream);
}
