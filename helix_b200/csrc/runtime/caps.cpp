// caps.cpp -- which descriptors run, on which kernel family, with what plan.
//
// Replaces reference src/runtime/caps.mm:18-304.  helix_scan_supported() is
// still the contract with the host: false means "keep your own kernel", and
// nothing is ever enqueued for a descriptor it rejects.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdlib>
#include <string>

#include "helix/helix_ext.h"
#include "internal.h"

namespace hx {

namespace {

bool positive_dims(const helix_scan_desc& d) {
    return d.n_tok > 0 && d.n_seq > 0 && d.n_head > 0 && d.head_dim > 0 && d.d_state > 0 &&
           d.n_group > 0;
}

// Scratch budget for run states, MiB.  Plays the role of the reference's
// HELIX_SCRATCH_MB (src/runtime/caps.mm:166-176): a smaller budget means
// fewer runs (less parallelism), never a wrong answer.
size_t scratch_budget() {
    if (const char* e = std::getenv("HELIX_SCRATCH_MB")) {
        const long mb = std::strtol(e, nullptr, 10);
        if (mb > 0) return (size_t)mb << 20;
    }
    return (size_t)512 << 20;
}

// Test and tuning hook: force the run length (tokens, rounded up to a
// multiple of kRunQuantum).  Small values put many runs in flight, which is
// what exercises the run-to-run state carry.
int forced_run_tokens() {
    if (const char* e = std::getenv("HELIX_RUN_TOKENS")) {
        const long v = std::strtol(e, nullptr, 10);
        if (v > 0) return (int)((v + kRunQuantum - 1) / kRunQuantum * kRunQuantum);
    }
    return 0;
}

size_t align256(size_t v) { return (v + 255) & ~(size_t)255; }

}  // namespace

// Precision selects the kernel family:
//   backend REF                   -> exact fp32 on CUDA cores (the reference's
//                                    scalar path for differential testing)
//   backend SGMMA, or AUTO with   -> tcgen05 three-product family: fp32
//   compute_dtype F32                operands as bf16 hi + lo pairs, products
//                                    hi.hi + hi.lo + lo.hi, fp32 accumulators
//                                    and state (the reference's fp32 matrix
//                                    path, src/runtime/caps.mm:19, 97-102)
//   backend MPP, or AUTO with     -> tcgen05 bf16 (the reference's bf16 path)
//   compute_dtype BF16
// The tcgen05 families read F32-stored x, B, C through copies in the scratch,
// so single pass (no scratch) takes the exact fp32 family, as does the
// three-product family's request with bf16-stored x, B, C (the reference's
// bf16 Pass C needs its multipass staging too, src/runtime/caps.mm:59-72).
// Diagonal A (declined by the reference, caps.mm:121-123) takes the
// recurrence kernels of kernels/scan_diag.cu whatever the backend and
// precision asked for: they compute in fp32.
Path select_path(const helix_scan_desc& d) {
    if (d.a_form == HELIX_A_DIAG_PER_CHANNEL) return kPathDiag;  // every backend
    if (d.backend == HELIX_BACKEND_REF) return kPathSimtF32;
    const bool bf16 = d.backend == HELIX_BACKEND_MPP || (d.backend != HELIX_BACKEND_SGMMA && d.compute_dtype == HELIX_BF16);
    if (bf16) return d.io_dtype == HELIX_F32 && !d.multipass ? kPathSimtF32 : kPathTcBf16;
    return d.io_dtype == HELIX_F32 && d.multipass ? kPathTcX3 : kPathSimtF32;
}

bool supported_impl(helix_ctx* ctx, const helix_scan_desc& d, std::string* why) {
    auto no = [&](const char* m) {
        if (why) *why = m;
        return false;
    };
    if (!ctx) return no("null context");
    if (!positive_dims(d)) return no("non-positive dimension");
    if (d.n_head % d.n_group != 0) return no("n_head not a multiple of n_group");
    // Only the scalar decay admits the chunked reassociation (reference
    // src/runtime/caps.mm:121-123); diagonal A runs the recurrence itself.
    if (d.a_form != HELIX_A_SCALAR_PER_HEAD && d.a_form != HELIX_A_DIAG_PER_CHANNEL) return no("unknown a_form");
    if (d.io_dtype != HELIX_F32 && d.io_dtype != HELIX_BF16) return no("io_dtype must be F32 or BF16");
    if (d.compute_dtype != HELIX_F32 && d.compute_dtype != HELIX_BF16)
        return no("compute_dtype must be F32 or BF16");
    if (d.backend < HELIX_BACKEND_AUTO || d.backend > HELIX_BACKEND_REF) return no("unknown backend");
    // The kernels read B, C and the states with unit innermost stride
    // (reference src/runtime/caps.mm:136-139).
    if (d.s_b[2] != 1 || d.s_c[2] != 1 || d.s_s[2] != 1) return no("innermost B/C/state stride must be 1");
    if (d.chunk != 0 && d.chunk != 64 && d.chunk != 128) return no("chunk must be 0, 64 or 128");
    // Run bookkeeping and grid sizes are int32.
    if ((int64_t)d.n_seq * d.n_head * ((d.head_dim + kSlab - 1) / kSlab) *
            ((d.n_tok + kRunQuantum - 1) / kRunQuantum) > (int64_t)INT32_MAX)
        return no("problem too large for one launch");

    if (select_path(d) == kPathDiag) {
        // four state groups of up to 64 states per thread
        if (d.d_state > 256) return no("diagonal-A path needs d_state <= 256");
        return true;
    }
    if (select_path(d) == kPathSimtF32) {
        if (d.d_state % 8 != 0 || d.d_state > 256) return no("fp32 path needs d_state % 8 == 0 and <= 256");
        return true;
    }

    // tcgen05 paths.
    if (!ctx->tc_ready) return no("tensor-core kernels unavailable on this device");
    if (select_path(d) == kPathTcX3) {
        // 128 states per pass (two passes above 128), B and C read through
        // their bf16 copies by TMA: rows of d_state * 2 bytes, multiple of 16
        if (d.d_state % 8 != 0 || d.d_state > 256)
            return no("tensor-core fp32 path needs d_state % 8 == 0 and <= 256");
        return true;
    }
    // 128 states per pass of the kernels (two passes above 128); rows of B
    // and C are TMA-loaded, so d_state * 2 bytes must be a multiple of 16.
    if (d.d_state % 8 != 0 || d.d_state > 256)
        return no("bf16 tensor-core path needs d_state % 8 == 0 and <= 256");
    if (d.io_dtype == HELIX_F32) return true;  // read through dense bf16 copies
    if (d.s_x[2] != 1) return no("x innermost stride must be 1 for TMA");
    // TMA: every non-innermost global stride must be a multiple of 16 bytes.
    const int64_t tma[] = {d.s_x[0], d.s_x[1], d.seq_x, d.s_b[0], d.s_b[1], d.seq_b,
                           d.s_c[0], d.s_c[1], d.seq_c};
    for (int64_t s : tma)
        if (s <= 0 || (s * 2) % 16 != 0) return no("x/B/C strides must be positive multiples of 16 bytes");
    return true;
}

namespace {

// Run cut of the tensor-core families.  Their output kernels give a CTA
// slabs_per_cta 64-channel slabs of one group (bf16: a "pair" of two; the
// three-product family: one) over a span of consecutive runs, so the span
// length is picked first: the one that minimises (waves of
// CTAs) x (blocks per span + half a block of start-up).  The span is then
// cut into runs fine enough that the state kernel (state_ctas CTAs per SM)
// has enough CTAs to spread over.
void tc_split(const helix_scan_desc& d, int blocks, int n_sm, int max_runs, int slabs_per_cta, int state_ctas,
              int steps_per_block, int* run_blocks, int* out_k) {
    const int64_t units = (int64_t)(d.n_head / d.n_group) * ((d.head_dim + kSlab - 1) / kSlab);
    const int64_t pairs = (int64_t)d.n_seq * d.n_group * ((units + slabs_per_cta - 1) / slabs_per_cta);
    double best = 1e300;
    int sb = blocks;
    for (int n = 1; n <= blocks; ++n) {
        const int b = (blocks + n - 1) / n;
        if ((blocks + b - 1) / b != n) continue;  // same span length as a smaller n
        const int64_t waves = (pairs * n + n_sm - 1) / n_sm;
        const double cost = (double)waves * (b + 0.5);
        if (cost < best) {
            best = cost;
            sb = b;
        }
    }
    const int n_out = (blocks + sb - 1) / sb;
    int k = 1;
    if (n_out > 1) {
        // Runs per span for the state kernel: each CTA reduces one run of one
        // slab, state_ctas CTAs share an SM, and a CTA costs about
        // kStateStartSteps steps of set-up on top of steps_per_block steps per
        // 128-token block.  Pick the divisor of the span that minimises
        // waves x per-CTA steps, within the run-slot budget.
        const int64_t st_units = (int64_t)d.n_seq * d.n_head * ((d.head_dim + kSlab - 1) / kSlab) * (n_out - 1);
        const int64_t slots = (int64_t)state_ctas * n_sm;
        double kbest = 1e300;
        for (int c = 1; c <= sb; ++c) {
            if (sb % c != 0) continue;
            if ((int64_t)(blocks + sb / c - 1) / (sb / c) > max_runs) break;
            const int64_t waves = (st_units * c + slots - 1) / slots;
            const double cost = (double)waves * (kStateStartSteps + (double)steps_per_block * (sb / c));
            if (cost < kbest) {
                kbest = cost;
                k = c;
            }
        }
    }
    *run_blocks = sb / k;
    *out_k = k;
}

void add_cast_regions(const helix_scan_desc& d, Plan* pl);

// Scratch regions, each 256-byte aligned: run states and run decays
// (run_slots per head), per-tile path records, per-run decay spans, then the
// bf16 copies of F32-stored inputs.
void lay_out_scratch(const helix_scan_desc& d, Plan* pl) {
    pl->total = 0;
    if (!(pl->run_slots > 0 || pl->has_flags || pl->cast)) return;
    const size_t agg = (size_t)d.n_seq * d.n_head * pl->run_slots * d.head_dim * d.d_state;
    const size_t lam = (size_t)d.n_seq * d.n_head * pl->run_slots;
    const int64_t units = (int64_t)(d.n_head / d.n_group) * pl->n_pslab;
    const size_t tiles = pl->has_flags ? (size_t)d.n_seq * d.n_group * ((units + 1) / 2) * pl->n_out : 0;
    pl->off_agg = 0;
    pl->off_lam = align256(agg * sizeof(float));
    pl->off_flag = pl->off_lam + align256(lam * sizeof(float));
    const size_t spans = pl->has_span ? (size_t)d.n_seq * d.n_head * pl->n_runs : 0;
    pl->off_span = pl->off_flag + align256(tiles * sizeof(int32_t));
    pl->total = pl->off_span + align256(spans * sizeof(float));
    add_cast_regions(d, pl);
}

// Whether TMA can read x as stored (fp32, innermost stride 1, the other
// strides multiples of 16 bytes): the three-product family then reads it in
// place.  The base address is checked when the call binds its tensors.
bool x_tma_f32(const helix_scan_desc& d) {
    return d.s_x[2] == 1 && d.s_x[0] > 0 && d.s_x[1] > 0 && d.seq_x > 0 && (d.s_x[0] * 4) % 16 == 0 &&
           (d.s_x[1] * 4) % 16 == 0 && (d.seq_x * 4) % 16 == 0;
}

// The copies of F32-stored inputs at the end of the scratch: bf16 x, B, C for
// the bf16 family; bf16 hi and lo halves of B and C (and, only where TMA cannot
// read x as stored, a dense fp32 copy of x) for the three-product family.
void add_cast_regions(const helix_scan_desc& d, Plan* pl) {
    if (!pl->cast) return;
    const bool x3 = pl->path == kPathTcX3;
    pl->x_copy = x3 ? (x_tma_f32(d) ? 0 : 2) : 1;
    pl->x_pitch = pl->x_copy == 2 ? (d.head_dim + 3) / 4 * 4 : (d.head_dim + 7) / 8 * 8;
    const size_t rows = (size_t)d.n_seq * d.n_tok;
    const size_t x_bytes = pl->x_copy == 0 ? 0 : rows * d.n_head * pl->x_pitch * (pl->x_copy == 2 ? 4 : 2);
    const size_t bc_bytes = rows * d.n_group * d.d_state * 2;
    pl->off_xc = pl->total;
    pl->off_bc = pl->off_xc + align256(x_bytes);
    pl->off_cc = pl->off_bc + align256(bc_bytes);
    pl->total = pl->off_cc + align256(bc_bytes);
    if (!pl->cast_lo) return;
    pl->off_bl = pl->total;
    pl->off_cl = pl->off_bl + align256(bc_bytes);
    pl->total = pl->off_cl + align256(bc_bytes);
}

}  // namespace

Plan make_plan(const helix_ctx* ctx, const helix_scan_desc& d) {
    Plan pl;
    pl.path = select_path(d);
    const bool tc = pl.path == kPathTcBf16 || pl.path == kPathTcX3;
    const bool diag = pl.path == kPathDiag;
    // chunk: the output kernel's token block (diagonal A: tokens staged per tile)
    pl.cs = tc ? 128 : diag ? 32 : (d.d_state <= 128 ? 64 : 32);
    pl.n_pslab = (d.head_dim + kSlab - 1) / kSlab;

    const int blocks = (d.n_tok + kRunQuantum - 1) / kRunQuantum;  // 128-token blocks
    const int n_sm = ctx ? std::max(ctx->n_sm, 1) : 148;
    const size_t per_run = (size_t)d.n_seq * d.n_head * d.head_dim * d.d_state * sizeof(float);
    const int max_runs = (int)std::min<size_t>((size_t)kMaxRuns,
                                               std::max<size_t>(1, scratch_budget() / std::max<size_t>(per_run, 1)));
    int run_blocks = blocks, out_k = 1;
    if (d.multipass) {
        if (const int f = forced_run_tokens()) {
            run_blocks = std::max(1, f / kRunQuantum);
        } else if (pl.path == kPathTcBf16) {
            tc_split(d, blocks, n_sm, max_runs, 2, kStateCtasPerSm, 2, &run_blocks, &out_k);
        } else if (pl.path == kPathTcX3) {
            tc_split(d, blocks, n_sm, max_runs, 1, kStateCtasPerSmX3, 4, &run_blocks, &out_k);
        } else {
            // Enough CTAs in the output kernel to cover every SM a few times
            // (diagonal A: one CTA per 64 (head, channel) rows of a group).
            const int64_t units = diag ? (int64_t)d.n_seq * d.n_group *
                                             (((int64_t)(d.n_head / d.n_group) * d.head_dim + 63) / 64)
                                       : (int64_t)d.n_seq * d.n_head * pl.n_pslab;
            const int64_t target = 4 * (int64_t)n_sm;
            int n_runs = (int)std::min<int64_t>(blocks, std::max<int64_t>(1, (target + units - 1) / units));
            n_runs = std::min(n_runs, max_runs);
            run_blocks = (blocks + n_runs - 1) / n_runs;
        }
    }
    run_blocks = std::max(run_blocks, (blocks + kMaxRuns - 1) / kMaxRuns);
    pl.run_tok = run_blocks * kRunQuantum;
    pl.n_runs = (blocks + run_blocks - 1) / run_blocks;
    pl.out_k = std::max(1, std::min(out_k, pl.n_runs));
    pl.n_out = (pl.n_runs + pl.out_k - 1) / pl.out_k;
    pl.state_runs = pl.out_k * (pl.n_out - 1);
    pl.run_slots = pl.state_runs;
    pl.need_state_kernel = pl.state_runs > 0;

    // The tensor-core output kernels record per tile which path ran, so the
    // general-path kernel need not re-measure the decay spans.
    pl.has_flags = d.multipass && pl.path == kPathTcBf16;
    // ... and, when a state pass runs, the largest decay span of every run's
    // chunks, measured there, so the output kernel need not read dt for it.
    pl.has_span = pl.has_flags && pl.need_state_kernel;
    pl.cast = d.multipass && ((pl.path == kPathTcBf16 && d.io_dtype == HELIX_F32) || pl.path == kPathTcX3);
    pl.cast_lo = pl.path == kPathTcX3;
    lay_out_scratch(d, &pl);
    return pl;
}

Plan make_shard_plan(const helix_ctx* ctx, const helix_scan_desc& d) {
    helix_scan_desc m = d;
    m.multipass = true;
    Plan pl = make_plan(ctx, m);
    // every run's state is reduced (the fold needs them all), each run's
    // decay span measured (tensor-core family): the same scratch then serves
    // the shard's scan (helix_scan_encode_shard) without a second state pass
    pl.state_runs = pl.n_runs;
    pl.run_slots = pl.n_runs;
    pl.need_state_kernel = true;
    pl.has_span = pl.has_flags;
    lay_out_scratch(m, &pl);
    return pl;
}

}  // namespace hx

extern "C" bool helix_scan_supported(helix_ctx* ctx, const helix_scan_desc* d) {
    if (!ctx || !d) return false;
    std::string why;
    const bool ok = hx::supported_impl(ctx, *d, &why);
    if (!ok) hx::set_error(ctx, why);
    return ok;
}

extern "C" size_t helix_scan_scratch_size(helix_ctx* ctx, const helix_scan_desc* d) {
    if (!d || !d->multipass) return 0;
    return hx::make_plan(ctx, *d).total;
}

extern "C" helix_backend helix_ctx_select_backend(helix_ctx* ctx, const helix_scan_desc* d) {
    if (!ctx || !d) return HELIX_BACKEND_REF;
    if (d->backend == HELIX_BACKEND_REF) return HELIX_BACKEND_REF;
    if (!hx::supported_impl(ctx, *d, nullptr)) return HELIX_BACKEND_REF;
    const hx::Path path = hx::select_path(*d);
    return path == hx::kPathTcBf16 ? HELIX_BACKEND_MPP : path == hx::kPathTcX3 ? HELIX_BACKEND_SGMMA : HELIX_BACKEND_REF;
}

extern "C" const char* helix_ctx_backend_desc(helix_ctx* ctx, const helix_scan_desc* d) {
    if (!ctx || !d) return "unavailable (null context)";
    if (!hx::supported_impl(ctx, *d, nullptr)) return "declined (shape unsupported)";
    switch (hx::select_path(*d)) {
        case hx::kPathTcBf16: return "tcgen05 (bf16 operands, fp32 accumulators and state)";
        case hx::kPathTcX3: return "tcgen05 (fp32 operands as bf16 hi+lo, three products, fp32 accumulators and state)";
        case hx::kPathDiag: return "cuda-core (diagonal A: per-state decay recurrence, fp32)";
        default: return "cuda-core (exact fp32)";
    }
}

extern "C" helix_status helix_scan_plan_info(helix_ctx* ctx, const helix_scan_desc* d, helix_plan_info* out) {
    if (!ctx || !d || !out) return HELIX_ERR_INVALID_ARG;
    std::string why;
    if (!hx::supported_impl(ctx, *d, &why)) {
        hx::set_error(ctx, why);
        return HELIX_ERR_UNSUPPORTED_SHAPE;
    }
    const hx::Plan pl = hx::make_plan(ctx, *d);
    out->family = (int32_t)pl.path;
    out->chunk = pl.cs;
    out->run_tokens = pl.run_tok;
    out->n_runs = pl.n_runs;
    out->runs_per_span = pl.out_k;
    out->n_spans = pl.n_out;
    out->state_runs = pl.state_runs;
    out->reserved = 0;
    out->scratch_bytes = d->multipass ? (uint64_t)pl.total : 0;
    return HELIX_OK;
}
