// scan_diag.cu -- diagonal A (a_form HELIX_A_DIAG_PER_CHANNEL: one decay
// rate per (head, state), Mamba-1's selective scan) on the CUDA cores.
//
// With a decay that differs per state the masked C.B^T reassociation of the
// scalar-A families does not exist (reference src/runtime/caps.mm:121-123),
// so these kernels run the recurrence itself, the fp64 oracle's arithmetic
// in fp32 (reference src/reference/scan_ref.cpp:27-29, :61-65):
//     s[c][n] = exp(dt_t A[h][n]) s[c][n] + dt_t B_t[n] x_t[c]
//     y_t[c]  = sum_n C_t[n] s[c][n]
// in parallel over (sequence, run, group, 64-row tile, state group) and
// sequentially over the tokens of a run.  A row is one (head, channel) of a
// group, so a tile of head_dim-1 heads (Mamba-1) is as full as one of a
// 64-channel head.  The run cut is the scalar families' (runtime/internal.h):
//   state kernel  per run but the last: the run's state from a zero start
//                 (agg) and its dt sum D (lam); the run's decay of state n
//                 is exp(A[h][n] D), since A is constant over the run;
//   output kernel per run: S = s0[ids[seq]], then for earlier runs r
//                 S = exp(A[h][n] D_r) S + agg_r, then the run's tokens,
//                 writing y; the last run writes s1.
//
// Thread layout: 256 threads, 64 rows per CTA.  A lane holds NS states of R
// consecutive rows; the NG lanes of a lane group cover d_state (NS x NG >=
// d_state), so each B, C and decay value a lane reads from shared memory
// serves R rows, and a row's y is the sum over its lane group, taken with
// shuffles (a reduce-scatter: one lane of the group ends with each row).
#include <cuda_runtime.h>

#include <cstdlib>

#include "common.cuh"

namespace hx {
namespace {

constexpr int kDThreads = 256;
constexpr int kDRows = 64;  // rows of a tile
constexpr int kDTok = 32;   // tokens staged per tile

// NS states of R rows per lane, NG lanes per row group: (32 / NG) lane
// groups per warp x R rows x 8 warps = 64 rows.
template <int NS, int NG, int R>
struct DiagCfg {
    static_assert((32 / NG) * R * (kDThreads / 32) == kDRows, "64 rows per CTA");
    static constexpr int NP = NS * NG;                    // staged states per token (padded)
    static constexpr size_t kB = (size_t)kDTok * NP;      // B [t][n]
    static constexpr size_t kC = kB;                      // C [t][n]
    static constexpr size_t kA = kB;                      // exp(dt_t A[h][n]) [t][n] (one-head tiles)
    static constexpr size_t kR = (size_t)kDTok * kDRows;  // per row: dt, dt x, y [t][row]
    static constexpr size_t bytes = (kB + kC + kA + 3 * kR) * sizeof(float);
};

// CTA -> (seq, run, group, first row); tiles fastest, then group, so the CTAs
// that read one group's B and C run side by side.
struct DTile {
    int seq, run, g, r0, rows;
};
__device__ __forceinline__ DTile diag_tile(const ScanParams& p, int runs) {
    const int gr = p.hpg * p.P;
    const int n_rt = (gr + kDRows - 1) / kDRows;
    int b = (int)blockIdx.x;
    DTile t;
    const int rt = b % n_rt;
    b /= n_rt;
    t.g = b % p.G;
    b /= p.G;
    t.run = b % runs;
    t.seq = b / runs;
    t.r0 = rt * kDRows;
    t.rows = min(kDRows, gr - t.r0);
    return t;
}

template <int R>
__device__ __forceinline__ void ld_rows(const float* src, float (&o)[R]) {
    if constexpr (R == 4) {
        const float4 v = *reinterpret_cast<const float4*>(src);
        o[0] = v.x, o[1] = v.y, o[2] = v.z, o[3] = v.w;
    } else if constexpr (R == 2) {
        const float2 v = *reinterpret_cast<const float2*>(src);
        o[0] = v.x, o[1] = v.y;
    } else {
        o[0] = src[0];
    }
}

// Sums v[0..R) over the NG lanes of a lane group.  Each halving step trades
// half the rows with the lane NG/2, NG/4, .. away; the remaining steps sum
// the one row left.  Returns the total of row *sel of the group's rows.
template <int NG, int R>
__device__ __forceinline__ float reduce_rows(float (&v)[R], int lane, int* sel) {
    int row = 0;
#pragma unroll
    for (int lv = 0; (R >> lv) > 1; ++lv) {
        const int half = (R >> lv) / 2;
        const int o = NG >> (lv + 1);
        const bool up = (lane & o) != 0;
#pragma unroll
        for (int i = 0; i < half; ++i) {
            const float send = up ? v[i] : v[i + half];
            const float keep = up ? v[i + half] : v[i];
            v[i] = keep + __shfl_xor_sync(0xffffffffu, send, o);
        }
        if (up) row += half;
    }
    constexpr int kLog2R = R == 1 ? 0 : R == 2 ? 1 : 2;
#pragma unroll
    for (int o = (NG >> kLog2R) / 2; o >= 1; o >>= 1) v[0] += __shfl_xor_sync(0xffffffffu, v[0], o);
    *sel = row;
    return v[0];
}

// OUT: output kernel (entry state, y, s1), else state kernel (agg, lam).
// UNI: every tile lies in one head (head_dim % 64 == 0), so the decays of a
// token are shared by the tile's rows and staged once; otherwise each lane
// evaluates its own from its rows' rates.
template <bool OUT, bool BF16, int NS, int NG, int R, bool UNI>
__global__ void __launch_bounds__(kDThreads, NS * R <= 32 ? 2 : 1) diag_kernel(ScanParams p, int runs_in_grid) {
    using CF = DiagCfg<NS, NG, R>;
    constexpr int NP = CF::NP;
    constexpr int RS = 32 / NG;  // lane groups per warp
    extern __shared__ float4 dsm4[];
    float* Bs = reinterpret_cast<float*>(dsm4);
    float* Cs = Bs + CF::kB;
    float* As = Cs + CF::kC;
    float* dts = As + CF::kA;
    float* dxs = dts + CF::kR;
    float* ys = dxs + CF::kR;

    const DTile tl = diag_tile(p, runs_in_grid);
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int grp = lane % NG;
    const int rbase = (warp * RS + lane / NG) * R;  // this lane's first row of the tile
    const int n0 = grp * NS;
    const int N = p.N;

    // this lane's row r: whether it exists, its head and channel (recomputed
    // where needed rather than held in registers across the token loop)
    auto row_live = [&](int r) { return rbase + r < tl.rows; };
    auto row_at = [&](int r) { return tl.r0 + (rbase + r < tl.rows ? rbase + r : 0); };
    auto head_of = [&](int r) { return tl.g * p.hpg + row_at(r) / p.P; };
    auto chan_of = [&](int r) { return row_at(r) % p.P; };
    const float* Ah0 = p.A + (int64_t)(tl.g * p.hpg + tl.r0 / p.P) * p.s_a;  // the tile's head (UNI)

    // decay rates of this lane's states (per-lane path), 0 past d_state
    float ar[UNI ? 1 : R][UNI ? 1 : NS];
    if constexpr (!UNI) {
#pragma unroll
        for (int r = 0; r < R; ++r)
#pragma unroll
            for (int k = 0; k < NS; ++k) ar[r][k] = n0 + k < N ? p.A[(int64_t)head_of(r) * p.s_a + n0 + k] : 0.0f;
    }

    float s[R][NS];
    if constexpr (OUT) {
        int src;
        const bool clear = s0_row(p, tl.seq, &src);
#pragma unroll
        for (int r = 0; r < R; ++r) {
            const float* s0r =
                p.s0 + (int64_t)src * p.seq_s + (int64_t)head_of(r) * p.s_s0 + (int64_t)chan_of(r) * p.s_s1;
#pragma unroll
            for (int k = 0; k < NS; ++k) {
                const int n = n0 + k;
                s[r][k] = (row_live(r) && n < N) ? (clear ? s0r[n] : kNaN) : 0.0f;
            }
        }
        // carry over the earlier runs: S = exp(A_n D_r) S + agg_r
        for (int q = 0; q < tl.run; ++q) {
#pragma unroll
            for (int r = 0; r < R; ++r) {
                const int h = head_of(r);
                const int64_t unit = ((int64_t)tl.seq * p.H + h) * p.run_slots + q;
                const float D = p.lam[unit];
                const float* ag = p.agg + unit * (int64_t)p.P * N + (int64_t)chan_of(r) * N;
                const float* Ar = p.A + (int64_t)h * p.s_a;
#pragma unroll
                for (int k = 0; k < NS; ++k) {
                    const int n = n0 + k;
                    if (row_live(r) && n < N) s[r][k] = fmaf(expf(Ar[n] * D), s[r][k], ag[n]);
                }
            }
        }
    } else {
#pragma unroll
        for (int r = 0; r < R; ++r)
#pragma unroll
            for (int k = 0; k < NS; ++k) s[r][k] = 0.0f;
    }

    const int t_begin = tl.run * p.run_tok;
    const int t_end = min(p.L, t_begin + p.run_tok);
    const int64_t bb = (int64_t)tl.seq * p.seq_b + (int64_t)tl.g * p.s_b1;
    const int64_t cb = (int64_t)tl.seq * p.seq_c + (int64_t)tl.g * p.s_c1;
    float dsum[R];  // dt summed over the run per row (state kernel: lam)
#pragma unroll
    for (int r = 0; r < R; ++r) dsum[r] = 0.0f;

    // staging: this thread's share of a tile, every load of a round issued
    // before its first store, so a tile costs a few memory latencies rather
    // than one per element
    constexpr int kPerBC = kDTok * NP / kDThreads;       // B (and C) elements
    constexpr int kPerRow = kDTok * kDRows / kDThreads;  // (token, row) pairs
    constexpr int kRound = kPerBC < 8 ? kPerBC : 8;
    // the (token, row) pairs this thread stages: row rw, tokens tq + 4 j
    const int rw = tid % kDRows, tq = tid / kDRows;
    const bool rw_live = rw < tl.rows;
    const int r2 = tl.r0 + (rw_live ? rw : 0);
    const int h2 = tl.g * p.hpg + r2 / p.P, c2 = r2 % p.P;
    const float* dt2 = p.dt + (int64_t)tl.seq * p.seq_dt + (int64_t)h2 * p.s_dt1;
    const int64_t x2 = (int64_t)tl.seq * p.seq_x + (int64_t)h2 * p.s_x1 + (int64_t)c2 * p.s_x2;
    const int64_t y2 = (int64_t)tl.seq * p.seq_y + (int64_t)h2 * p.s_y1 + (int64_t)c2 * p.s_y2;

    for (int t0 = t_begin; t0 < t_end; t0 += kDTok) {
        const int tlen = min(kDTok, t_end - t0);
        // ---- stage the tile: B, C (zero past the run or d_state), dt, dt x
#pragma unroll
        for (int j0 = 0; j0 < kPerBC; j0 += kRound) {
            float bv[kRound], cv[OUT ? kRound : 1];
#pragma unroll
            for (int j = 0; j < kRound; ++j) {
                const int i = tid + (j0 + j) * kDThreads, t = i / NP, n = i - t * NP;
                const bool ok = t < tlen && n < N;
                bv[j] = ok ? ld_io<BF16>(p.B, bb + (int64_t)(t0 + t) * p.s_b0 + n) : 0.0f;
                if constexpr (OUT) cv[j] = ok ? ld_io<BF16>(p.C, cb + (int64_t)(t0 + t) * p.s_c0 + n) : 0.0f;
            }
#pragma unroll
            for (int j = 0; j < kRound; ++j) {
                Bs[tid + (j0 + j) * kDThreads] = bv[j];
                if constexpr (OUT) Cs[tid + (j0 + j) * kDThreads] = cv[j];
            }
        }
        {
            float dv[kPerRow], xv[kPerRow];
#pragma unroll
            for (int j = 0; j < kPerRow; ++j) {
                const int t = tq + j * (kDThreads / kDRows);
                const bool ok = t < tlen && rw_live;
                dv[j] = ok ? dt2[(int64_t)(t0 + t) * p.s_dt0] : 0.0f;
                xv[j] = ok ? ld_io<BF16>(p.x, x2 + (int64_t)(t0 + t) * p.s_x0) : 0.0f;
            }
#pragma unroll
            for (int j = 0; j < kPerRow; ++j) {
                const int t = tq + j * (kDThreads / kDRows);
                const float v = t < tlen && rw_live ? dt_of(dv[j], p.dt_min, p.dt_max) : 0.0f;
                dts[t * kDRows + rw] = v;
                dxs[t * kDRows + rw] = v * xv[j];
            }
        }
        __syncthreads();
        if constexpr (UNI) {
            // row 0's head is every row's head
            for (int i = tid; i < kDTok * NP; i += kDThreads) {
                const int t = i / NP, n = i - t * NP;
                As[i] = n < N ? expf(dts[t * kDRows] * Ah0[n]) : 1.0f;
            }
            __syncthreads();
        }

        // ---- the recurrence over the tile's tokens (two per iteration: one
        // token's y shuffles overlap the next token's loads and arithmetic)
#pragma unroll 2
        for (int t = 0; t < tlen; ++t) {
            float v[R];
            {
                float bx[R], d[R];
                ld_rows<R>(dxs + t * kDRows + rbase, bx);
                if constexpr (!UNI || !OUT) ld_rows<R>(dts + t * kDRows + rbase, d);
                const float4* b4 = reinterpret_cast<const float4*>(Bs + t * NP + n0);
                const float4* c4 = reinterpret_cast<const float4*>(Cs + t * NP + n0);
                const float4* a4 = reinterpret_cast<const float4*>(As + t * NP + n0);
#pragma unroll
                for (int r = 0; r < R; ++r) v[r] = 0.0f;
#pragma unroll
                for (int k4 = 0; k4 < NS / 4; ++k4) {
                    const float4 b = b4[k4];
                    float4 cv = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
                    if constexpr (OUT) cv = c4[k4];
                    float4 au = make_float4(1.0f, 1.0f, 1.0f, 1.0f);
                    if constexpr (UNI) au = a4[k4];
#pragma unroll
                    for (int r = 0; r < R; ++r) {
                        float4 a = au;
                        if constexpr (!UNI)
                            a = make_float4(expf(d[r] * ar[r][4 * k4]), expf(d[r] * ar[r][4 * k4 + 1]),
                                            expf(d[r] * ar[r][4 * k4 + 2]), expf(d[r] * ar[r][4 * k4 + 3]));
                        float* sr = s[r] + 4 * k4;
                        sr[0] = fmaf(a.x, sr[0], b.x * bx[r]);
                        sr[1] = fmaf(a.y, sr[1], b.y * bx[r]);
                        sr[2] = fmaf(a.z, sr[2], b.z * bx[r]);
                        sr[3] = fmaf(a.w, sr[3], b.w * bx[r]);
                        if constexpr (OUT) {
                            v[r] = fmaf(cv.x, sr[0], v[r]);
                            v[r] = fmaf(cv.y, sr[1], v[r]);
                            v[r] = fmaf(cv.z, sr[2], v[r]);
                            v[r] = fmaf(cv.w, sr[3], v[r]);
                        }
                    }
                }
                if constexpr (!OUT) {
#pragma unroll
                    for (int r = 0; r < R; ++r) dsum[r] += d[r];
                }
            }
            if constexpr (OUT) {
                int sel;
                const float yt = reduce_rows<NG, R>(v, lane, &sel);
                if (lane % (NG / R) == 0) ys[t * kDRows + rbase + sel] = yt;
            }
        }
        __syncthreads();

        // ---- y of the tile, row-contiguous
        if constexpr (OUT) {
#pragma unroll
            for (int j = 0; j < kPerRow; ++j) {
                const int t = tq + j * (kDThreads / kDRows);
                if (t < tlen && rw_live) p.y[y2 + (int64_t)(t0 + t) * p.s_y0] = ys[t * kDRows + rw];
            }
            // the next tile's staging touches only Bs .. dxs, and its
            // barrier orders these reads of ys before the next writes
        }
    }

    if constexpr (!OUT) {
#pragma unroll
        for (int r = 0; r < R; ++r) {
            if (!row_live(r)) continue;
            const int64_t unit = ((int64_t)tl.seq * p.H + head_of(r)) * p.run_slots + tl.run;
            float* out = p.agg + unit * (int64_t)p.P * N + (int64_t)chan_of(r) * N;
#pragma unroll
            for (int k = 0; k < NS; ++k)
                if (n0 + k < N) out[n0 + k] = s[r][k];
            if (grp == 0 && chan_of(r) == 0) p.lam[unit] = dsum[r];
        }
    } else if (tl.run == p.n_runs - 1) {
#pragma unroll
        for (int r = 0; r < R; ++r) {
            if (!row_live(r)) continue;
            float* s1r =
                p.s1 + (int64_t)tl.seq * p.seq_s + (int64_t)head_of(r) * p.s_s0 + (int64_t)chan_of(r) * p.s_s1;
#pragma unroll
            for (int k = 0; k < NS; ++k)
                if (n0 + k < N) s1r[n0 + k] = s[r][k];
        }
    }
}

template <bool OUT, bool BF16, int NS, int NG, int R, bool UNI>
int launch_one(const ScanParams& p, int runs, cudaStream_t st) {
    const int64_t n_rt = ((int64_t)p.hpg * p.P + kDRows - 1) / kDRows;
    const int64_t grid = (int64_t)p.S * runs * p.G * n_rt;
    diag_kernel<OUT, BF16, NS, NG, R, UNI>
        <<<(unsigned)grid, kDThreads, DiagCfg<NS, NG, R>::bytes, st>>>(p, runs);
    return cudaGetLastError();
}

template <bool OUT, bool BF16, int NS, int NG, int R, bool UNI>
int configure_one() {
    return cudaFuncSetAttribute(diag_kernel<OUT, BF16, NS, NG, R, UNI>,
                                cudaFuncAttributeMaxDynamicSharedMemorySize, (int)DiagCfg<NS, NG, R>::bytes);
}

// Lane shapes by d_state: (states per lane, lanes per row group, rows per lane).
template <bool OUT, bool BF16, bool UNI>
int launch_ns(const ScanParams& p, int runs, cudaStream_t st) {
    if (p.N <= 16) return launch_one<OUT, BF16, 4, 4, 1, UNI>(p, runs, st);
    if (p.N <= 32) return launch_one<OUT, BF16, 4, 8, 2, UNI>(p, runs, st);
    if (p.N <= 64) return launch_one<OUT, BF16, 4, 16, 4, UNI>(p, runs, st);
    if (p.N <= 128) return launch_one<OUT, BF16, 8, 16, 4, UNI>(p, runs, st);
    return launch_one<OUT, BF16, 16, 16, 4, UNI>(p, runs, st);
}

template <bool OUT, bool BF16, bool UNI>
int configure_ns() {
    int e;
    if ((e = configure_one<OUT, BF16, 4, 4, 1, UNI>()) != cudaSuccess) return e;
    if ((e = configure_one<OUT, BF16, 4, 8, 2, UNI>()) != cudaSuccess) return e;
    if ((e = configure_one<OUT, BF16, 4, 16, 4, UNI>()) != cudaSuccess) return e;
    if ((e = configure_one<OUT, BF16, 8, 16, 4, UNI>()) != cudaSuccess) return e;
    return configure_one<OUT, BF16, 16, 16, 4, UNI>();
}

template <bool OUT>
int launch_pass(const ScanParams& p, int runs, cudaStream_t st) {
    const bool uni = p.P % kDRows == 0;
    if (p.io_bf16) return uni ? launch_ns<OUT, true, true>(p, runs, st) : launch_ns<OUT, true, false>(p, runs, st);
    return uni ? launch_ns<OUT, false, true>(p, runs, st) : launch_ns<OUT, false, false>(p, runs, st);
}

template <bool OUT>
int configure_pass() {
    int e;
    if ((e = configure_ns<OUT, false, false>()) != cudaSuccess) return e;
    if ((e = configure_ns<OUT, false, true>()) != cudaSuccess) return e;
    if ((e = configure_ns<OUT, true, false>()) != cudaSuccess) return e;
    return configure_ns<OUT, true, true>();
}

}  // namespace

int configure_diag(const helix_ctx*) {
    const int e = configure_pass<false>();
    return e != cudaSuccess ? e : configure_pass<true>();
}

int launch_diag(const helix_ctx*, const Plan& pl, const ScanParams& p, void* stream) {
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const char* only = std::getenv("HELIX_ONLY_PASS");
    if (pl.need_state_kernel && (!only || *only == 'A')) {
        const int e = launch_pass<false>(p, pl.state_runs, st);
        if (e != cudaSuccess) return e;
    }
    if (!only || *only == 'C') return launch_pass<true>(p, pl.n_runs, st);
    return cudaSuccess;
}

}  // namespace hx
