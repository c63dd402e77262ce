// internal.h -- runtime internals shared by the C++ runtime and the CUDA
// kernels.  Not installed, not part of the ABI.
//
// Replaces the reference's Objective-C++ runtime internals
// (src/runtime/helix_internal.h:12-110) and its shared Metal parameter block
// (src/kernels/helix_params.h:45-110).  Differences that matter:
//   * every stride is 64-bit: config 5 (n_seq=8, L=131072, H=128, P=64) puts
//     n_seq*seq_x at 8.6e9, beyond the int32 fields the reference validates
//     against (src/runtime/caps.mm:243-257);
//   * the sequence is cut into "runs" of whole 128-token blocks.  The state
//     kernel reduces each run to one fp32 state (its contribution from a zero
//     start) plus one log-decay; the output kernel rebuilds the state entering
//     its run from those and walks the run's chunks.  Scratch therefore holds
//     one state per run instead of the reference's one state per chunk
//     (src/kernels/helix_params.h:101-109).
#pragma once

#include <cstddef>
#include <cstdint>
#include <map>
#include <mutex>
#include <string>
#include <thread>

#include "helix/helix.h"

namespace hx {

// Token granularity of runs.  Both kernel families cut runs on this boundary
// so the scratch plan does not depend on which family runs.
constexpr int kRunQuantum = 128;
// Head-dim slab handled by one CTA (reference HELIX_HD, helix_params.h:19).
constexpr int kSlab = 64;
// Upper bound on runs per sequence (the output kernels stage per-run decays
// and carry weights in shared memory).
constexpr int kMaxRuns = 256;
// Tensor-core state kernel: CTAs resident per SM, and its fixed cost per CTA
// (first loads, first decay weights, drain) in 64-token steps, as measured.
constexpr int kStateCtasPerSm = 3;
constexpr int kStateCtasPerSmX3 = 3;  // three-product family (32-token steps)
constexpr double kStateStartSteps = 3.5;

enum Path : int {
    kPathSimtF32 = 0,   // exact fp32 CUDA-core kernels
    kPathTcBf16  = 1,   // tcgen05 kernels, bf16 operands, fp32 state
    kPathTcX3    = 2,   // tcgen05 kernels, three-product bf16 split of fp32
                        // operands (hi.hi + hi.lo + lo.hi), fp32 state
    kPathDiag    = 3,   // diagonal A: the per-state recurrence on CUDA cores, fp32
};

// How one descriptor is executed.  A pure function of (ctx, desc, env):
// helix_scan_scratch_size() and the encoder both call make_plan().
struct Plan {
    Path   path     = kPathSimtF32;
    int    cs       = 64;   // chunk length inside the output kernel
    int    run_tok  = 0;    // tokens per run (multiple of kRunQuantum)
    int    n_runs   = 1;
    int    n_pslab  = 1;
    // The output kernel gives each CTA out_k consecutive runs (a "span"):
    // n_out spans per sequence.  The state kernel reduces the runs before the
    // last span (state_runs of them); their states sit in run_slots slots
    // per (seq, head).
    int    out_k      = 1;
    int    n_out      = 1;
    int    state_runs = 0;
    int    run_slots  = 0;
    bool   need_state_kernel = false;  // state_runs > 0
    size_t off_agg  = 0;    // f32 [seq][head][run_slots][head_dim][d_state]
    size_t off_lam  = 0;    // f32 [seq][head][run_slots]
    size_t off_flag = 0;    // i32 [output tiles] (tensor-core family, multipass): fast path taken
    bool   has_flags = false;
    size_t off_span = 0;    // f32 [seq][head][n_runs]: largest decay span of a run's chunks
    bool   has_span = false; // written by the state kernel (tensor-core family with a state pass)
    // Tensor-core family with x, B, C stored F32: dense bf16 copies made by a
    // cast kernel first (multipass only; single pass takes the fp32 family).
    bool   cast     = false;
    // x: 1 = bf16 copy (bf16 family); for the three-product family, which
    // reads fp32 x by TMA and splits it on chip, 0 = none (x read in place)
    // or 2 = dense fp32 copy (x strides TMA cannot describe).
    int    x_copy   = 0;
    int    x_pitch  = 0;    // channels per row of the x copy (bf16: head_dim rounded up to 8; fp32: to 4)
    size_t off_xc   = 0;    // [seq][tok][head][x_pitch]
    size_t off_bc   = 0;    // bf16 [seq][tok][group][d_state]
    size_t off_cc   = 0;    // bf16 [seq][tok][group][d_state]
    // Three-product family: the low halves of the B and C copies, same layouts.
    bool   cast_lo  = false;
    size_t off_bl   = 0;
    size_t off_cl   = 0;
    size_t total    = 0;    // scratch bytes
    // The run states (and bf16 copies) are already in the scratch, left by
    // helix_scan_shard_state: no cast and no state kernel run.
    bool   states_ready = false;
};

// Kernel parameter block (passed by value).
struct ScanParams {
    int32_t S, L, H, P, N, G, hpg;
    int32_t n_pslab, run_tok, n_runs;
    int32_t out_k, n_out, state_runs, run_slots;   // see Plan
    int32_t n_pair;         // two-slab tiles per group: ceil(hpg * n_pslab / 2)
    int32_t has_ids;
    int32_t io_bf16;        // x, B, C stored as bf16
    // Tensor-core family: the kernels cover 128 states at a time.  A d_state
    // above 128 runs as two halves (n_half = 2): the state kernel covers both
    // in one grid, the output kernels run once per half with n_base = 0, 128;
    // the second half adds its share of y to the first's (y_add = 1).
    int32_t n_half, n_base, y_add;
    // Test hook (0 = off): the fast output kernel's CTAs first wait this many
    // cycles on a barrier nothing arrives on, record kFaultTestStall and return.
    int64_t test_stall;
    float   dt_min, dt_max;

    int64_t s_x0, s_x1, s_x2, seq_x;
    int64_t s_b0, s_b1, seq_b;        // innermost B stride is 1
    int64_t s_c0, s_c1, seq_c;        // innermost C stride is 1
    int64_t s_dt0, s_dt1, seq_dt;
    int64_t s_s0, s_s1, seq_s;        // innermost state stride is 1
    int64_t s_y0, s_y1, s_y2, seq_y;
    int64_t s_a;

    const void*    x;
    const float*   dt;
    const float*   A;
    const void*    B;
    const void*    C;
    const int32_t* ids;
    const float*   s0;
    float*         y;
    float*         s1;
    float*         agg;     // scratch, see Plan
    float*         lam;
    int32_t*       tile_flag;  // scratch or null, see Plan
    float*         run_span;   // scratch or null, see Plan

    void*          cast_x;      // scratch: bf16 copies (Plan::cast), else null
    void*          cast_b;
    void*          cast_c;
    void*          cast_bl;     // scratch: low halves of the B and C copies (Plan::cast_lo), else null
    void*          cast_cl;
    int32_t        x_copy;      // Plan::x_copy

    unsigned*      fault;       // the device fault word (helix_device_fault)
    int64_t        s_row_bytes; // bytes one s0 / s1 row spans
    int64_t        s1_bytes;    // bytes the n_seq rows of s1 span
};

}  // namespace hx

struct helix_ctx {
    // Last error per calling thread (helix_ctx_last_error); freed with the
    // context.  Only error paths touch it.
    std::mutex err_mu;
    std::map<std::thread::id, std::string> errors;

    int    device      = 0;
    int    n_sm        = 0;
    int    cc_major    = 0;
    int    cc_minor    = 0;
    size_t max_smem_optin = 0;
    bool   tc_ready    = false;   // tensor-core kernels configured
    unsigned* fault_word = nullptr; // device address of the fault word
    void*  encode_tiled = nullptr; // cuTensorMapEncodeTiled entry point
};

namespace hx {

// Per-thread, per-context last error (helix_ctx_last_error).
void        set_error(const helix_ctx* ctx, const std::string& msg);
const char* get_error(const helix_ctx* ctx);

// caps.cpp
bool supported_impl(helix_ctx* ctx, const helix_scan_desc& d, std::string* why);
Plan make_plan(const helix_ctx* ctx, const helix_scan_desc& d);
// Plan of helix_scan_shard_state: the multipass run cut, with one state slot
// and one log-decay per run for every run (the last one included).
Plan make_shard_plan(const helix_ctx* ctx, const helix_scan_desc& d);
Path select_path(const helix_scan_desc& d);

// dispatch.cpp: fills everything but the tensor pointers.
void fill_params(ScanParams& p, const helix_scan_desc& d, const Plan& pl);

// The tensors of one scan call, as the caller passed them.
struct CallTensors {
    helix_tensor s0, x, dt, A, B, C, ids, y, s1;
};
// Checks the call's tensors (none null, s1 clear of every s0 row the call
// may read, TMA alignment on the tensor-core path) and fills *p from d, the
// plan and the tensors; scratch pointers are left null.  Shared by every
// entry point that runs a scan, so each check exists once.
helix_status bind_call(helix_ctx* ctx, const helix_scan_desc& d, const Plan& pl, const CallTensors& t,
                       ScanParams* p);
// Points the plan's scratch regions of *p into base.
void bind_scratch(const Plan& pl, char* base, ScanParams* p);
// Enqueues the plan's kernels on stream, on ctx's device.
helix_status run_call(helix_ctx* ctx, const Plan& pl, const ScanParams& p, void* stream);
// Whether the driver allocation holding s has need bytes from s on (true
// when the driver does not know s: a raw pointer carries no length).
bool scratch_fits(const void* s, size_t need);
// Whether the n_seq rows of s1 overlap the first n_seq rows of s0.  (Rows
// that only ids reaches are checked on the device; see s0_row.)
bool states_overlap(const helix_scan_desc& d, const void* s0, const void* s1);

// Kernel launchers (kernels/*.cu).  Return cudaSuccess or the launch error.
int launch_simt(const helix_ctx* ctx, const Plan& pl, const ScanParams& p, void* stream);
int launch_tc(const helix_ctx* ctx, const Plan& pl, const ScanParams& p, void* stream);
int launch_tc3(const helix_ctx* ctx, const Plan& pl, const ScanParams& p, void* stream);
int launch_diag(const helix_ctx* ctx, const Plan& pl, const ScanParams& p, void* stream);
// State kernel over every run of the plan (p.agg / p.lam for all n_runs).
int launch_simt_states(const helix_ctx* ctx, const Plan& pl, const ScanParams& p, void* stream);
int launch_tc_states(const helix_ctx* ctx, const Plan& pl, const ScanParams& p, void* stream);
int launch_tc3_states(const helix_ctx* ctx, const Plan& pl, const ScanParams& p, void* stream);
// kernels/scan_tc.cu, shared with scan_tc3.cu: the tcgen05 state kernel over
// `runs` runs (x3: the three-product mode, reading fp32 x and the low halves
// of B from p.cast_bl; a programmatic dependent of the cast kernel when
// after_cast), and the carry kernel (programmatic dependent of the previous
// kernel when after_ours).
int launch_tc_state_pass(const helix_ctx* ctx, const ScanParams& p, int runs, bool x3, bool after_cast,
                         void* stream);
int launch_tc_carry(const ScanParams& p, bool after_ours, void* stream);
// kernels/scan_cast.cu: when `run`, enqueues the copies of x (Plan::x_copy),
// B and C into p->cast_*; then points *p at the copies (dense strides).
int launch_cast(const helix_ctx* ctx, const Plan& pl, ScanParams* p, void* stream, bool run);
// kernels/scan_shard.cu
// state[seq][h] = fold over runs of (exp(lam_r) S + agg_r) from zero, written
// with the state strides of p (s_s0, s_s1, seq_s); log_decay[seq * H + h] =
// sum_r lam_r.
int launch_shard_fold(const ScanParams& p, float* state, float* log_decay, void* stream);
// carry[seq][h] = fold over j < n_prev of (exp(ld_j) S + states_j) from
// s0[ids[seq]]; s0 and carry use the state strides of p, states and ld are
// dense [n_prev][S][H][P][N] and [n_prev][S][H].
int launch_carry_combine(const ScanParams& p, const float* states, const float* log_decays, int n_prev,
                         float* carry, void* stream);
int configure_simt(const helix_ctx* ctx);
int configure_tc(const helix_ctx* ctx);
int configure_tc3(const helix_ctx* ctx);
int configure_diag(const helix_ctx* ctx);
int read_tc_fault(unsigned* code);
// Device address of the fault word on the current device.
int fault_word_address(unsigned** out);

}  // namespace hx
