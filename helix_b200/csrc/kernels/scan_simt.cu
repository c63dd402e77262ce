// scan_simt.cu -- exact fp32 kernels on the CUDA cores (backend REF/SGMMA,
// compute_dtype F32).  They serve the fp32 configurations at fp32 accuracy
// and are the differential baseline for the tensor-core kernels.
//
// Decomposition (same as the tensor-core family, see runtime/internal.h):
//   state kernel  per (seq, run, head, slab), runs 0..n_runs-2:
//                 agg[n][c] = sum_{j in run} B[j][n] * dt_j * exp(sum_{i>j, i in run} A dt_i) * x[j][c]
//                 lam       = sum_{j in run} A dt_j
//   output kernel per (seq, run, head, slab):
//                 S = s0[ids[seq]]; for earlier runs r: S = exp(lam_r) S + agg_r
//                 then, per chunk of CS tokens (reference chunked algebra,
//                 src/reference/scan_chunked_ref.cpp:81-128):
//                   M[t][j] = (C_t . B_j) exp(Lc_t - Lc_j) dt_j        (j <= t)
//                   y[t][c] = sum_j M[t][j] x[j][c] + exp(Lc_t) sum_n C[t][n] S[n][c]
//                   S[n][c] = exp(Lc_end) S[n][c] + sum_j B[j][n] dt_j exp(Lc_end - Lc_j) x[j][c]
//                 the last run writes s1.
// 256 threads; one CTA per SM is the design point (large smem tiles).
#include <cuda_runtime.h>

#include <cstdlib>

#include "common.cuh"

namespace hx {
namespace {

constexpr int kThreads = 256;
constexpr int kXs = kSlab + 4;  // padded row of x / state tiles (floats)

template <int CS, int NMAX>
struct SimtSmem {
    static constexpr int kRow = NMAX + 4;  // padded row of B / C tiles
    static constexpr size_t kS = (size_t)NMAX * kXs;
    static constexpr size_t kC = (size_t)CS * kRow;
    static constexpr size_t kB = (size_t)CS * kRow;
    static constexpr size_t kX = (size_t)CS * kXs;
    static constexpr size_t kM = (size_t)CS * (CS + 4);
    static constexpr size_t kVec = 4 * CS + 32;
    static constexpr size_t out_bytes = (kS + kC + kB + kX + kM + kVec) * sizeof(float);
    static constexpr size_t state_bytes =
        (kB + kX + kVec) * sizeof(float) > (size_t)kSlab * (NMAX + 1) * sizeof(float)
            ? (kB + kX + kVec) * sizeof(float)
            : (size_t)kSlab * (NMAX + 1) * sizeof(float) + kVec * sizeof(float);
};

// Rows [0, tlen) of a (token, state) operand of one group into smem; rows
// beyond are zero so padded tokens contribute nothing.
template <bool BF16, int ROW>
__device__ __forceinline__ void load_bc(float* dst, const void* src, int64_t base, int64_t s_tok,
                                        int t0, int tlen, int cs, int N) {
    for (int i = threadIdx.x; i < cs * N; i += kThreads) {
        const int r = i / N, n = i - r * N;
        dst[r * ROW + n] = r < tlen ? ld_io<BF16>(src, base + (int64_t)(t0 + r) * s_tok + n) : 0.0f;
    }
}

template <bool BF16>
__device__ __forceinline__ void load_x(float* dst, const ScanParams& p, int64_t base, int t0,
                                       int tlen, int cs, int pw) {
    for (int i = threadIdx.x; i < cs * kSlab; i += kThreads) {
        const int r = i / kSlab, c = i - r * kSlab;
        dst[r * kXs + c] = (r < tlen && c < pw)
                               ? ld_io<BF16>(p.x, base + (int64_t)(t0 + r) * p.s_x0 + (int64_t)c * p.s_x2)
                               : 0.0f;
    }
}

// ---------------------------------------------------------------------------
// State kernel: one run's contribution from a zero start, plus its log-decay.
// ---------------------------------------------------------------------------
template <int CS, int NMAX, bool BF16>
__global__ void __launch_bounds__(kThreads, 1) simt_state_kernel(ScanParams p, int runs_in_grid) {
    using SM = SimtSmem<CS, NMAX>;
    extern __shared__ float4 smem4[];
    float* sm = reinterpret_cast<float*>(smem4);
    float* Bs = sm;
    float* Xs = Bs + SM::kB;
    float* dtv = Xs + SM::kX;
    float* Lc = dtv + CS;
    float* wv = Lc + CS;
    float* tot = wv + CS;

    const Tile tl = decode_tile(blockIdx.x, p.n_pslab, p.H, runs_in_grid);
    const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
    const int p0 = tl.slab * kSlab, pw = min(kSlab, p.P - p0);
    const int g = tl.h / p.hpg;
    const float Ah = p.A[(int64_t)tl.h * p.s_a];
    const int t_begin = tl.run * p.run_tok;
    const int t_end = min(p.L, t_begin + p.run_tok);
    const int n_chunks = (t_end - t_begin + CS - 1) / CS;

    const int64_t xb = (int64_t)tl.seq * p.seq_x + (int64_t)tl.h * p.s_x1 + (int64_t)p0 * p.s_x2;
    const int64_t bb = (int64_t)tl.seq * p.seq_b + (int64_t)g * p.s_b1;
    const int64_t db = (int64_t)tl.seq * p.seq_dt + (int64_t)tl.h * p.s_dt1;

    constexpr int NI = NMAX / 16;
    float acc[NI][4];
#pragma unroll
    for (int i = 0; i < NI; ++i)
#pragma unroll
        for (int k = 0; k < 4; ++k) acc[i][k] = 0.0f;

    // Chunks are visited last to first so the decay from token j to the end
    // of the run is a sum of same-sign terms (no cancellation).
    float later = 0.0f;
    for (int ci = n_chunks - 1; ci >= 0; --ci) {
        const int t0 = t_begin + ci * CS;
        const int tlen = min(CS, t_end - t0);
        float v = 0.0f;
        if (tid < tlen) v = dt_of(p.dt[db + (int64_t)(t0 + tid) * p.s_dt0], p.dt_min, p.dt_max);
        const float pre = block_prefix(Ah * v, CS, tot);
        if (tid < CS) {
            dtv[tid] = v;
            Lc[tid] = pre;
        }
        load_bc<BF16, SM::kRow>(Bs, p.B, bb, p.s_b0, t0, tlen, CS, p.N);
        load_x<BF16>(Xs, p, xb, t0, tlen, CS, pw);
        __syncthreads();
        const float Lend = Lc[CS - 1];
        if (tid < CS) wv[tid] = dtv[tid] * expf(later + (Lend - Lc[tid]));
        __syncthreads();
        later += Lend;

        for (int j = 0; j < tlen; ++j) {
            const float w = wv[j];
            const float4 xv = *reinterpret_cast<const float4*>(Xs + j * kXs + 4 * tx);
            const float xw[4] = {xv.x * w, xv.y * w, xv.z * w, xv.w * w};
#pragma unroll
            for (int i = 0; i < NI; ++i) {
                const int n = ty + 16 * i;
                const float b = n < p.N ? Bs[j * SM::kRow + n] : 0.0f;
#pragma unroll
                for (int k = 0; k < 4; ++k) acc[i][k] = fmaf(b, xw[k], acc[i][k]);
            }
        }
        __syncthreads();
    }

    const int64_t unit = ((int64_t)tl.seq * p.H + tl.h) * p.run_slots + tl.run;
    if (tl.slab == 0 && tid == 0) p.lam[unit] = later;

    // Transpose through smem so the (chan, state) rows go out coalesced.
    float* T = sm;  // [kSlab][NMAX + 1]
#pragma unroll
    for (int i = 0; i < NI; ++i)
#pragma unroll
        for (int k = 0; k < 4; ++k) T[(4 * tx + k) * (NMAX + 1) + ty + 16 * i] = acc[i][k];
    __syncthreads();
    float* out = p.agg + unit * (int64_t)p.P * p.N;
    for (int i = tid; i < pw * p.N; i += kThreads) {
        const int c = i / p.N, n = i - c * p.N;
        out[(int64_t)(p0 + c) * p.N + n] = T[c * (NMAX + 1) + n];
    }
}

// ---------------------------------------------------------------------------
// Output kernel.
// ---------------------------------------------------------------------------
template <int CS, int NMAX, bool BF16>
__global__ void __launch_bounds__(kThreads, 1) simt_out_kernel(ScanParams p) {
    using SM = SimtSmem<CS, NMAX>;
    constexpr int ROW = SM::kRow;
    constexpr int MR = CS + 4;
    extern __shared__ float4 smem4[];
    float* sm = reinterpret_cast<float*>(smem4);
    float* Ss = sm;             // [NMAX][kXs]   state S[n][c]
    float* Cs = Ss + SM::kS;    // [CS][ROW]
    float* Bs = Cs + SM::kC;    // [CS][ROW]
    float* Xs = Bs + SM::kB;    // [CS][kXs]     raw x
    float* Ms = Xs + SM::kX;    // [CS][MR]      masked, decayed C.B^T times dt_j
    float* dtv = Ms + SM::kM;
    float* Lc = dtv + CS;
    float* ev = Lc + CS;
    float* wv = ev + CS;
    float* tot = wv + CS;

    const Tile tl = decode_tile(blockIdx.x, p.n_pslab, p.H, p.n_runs);
    const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
    const int p0 = tl.slab * kSlab, pw = min(kSlab, p.P - p0);
    const int N = p.N;
    const int g = tl.h / p.hpg;
    const float Ah = p.A[(int64_t)tl.h * p.s_a];
    const int t_begin = tl.run * p.run_tok;
    const int t_end = min(p.L, t_begin + p.run_tok);

    const int64_t xb = (int64_t)tl.seq * p.seq_x + (int64_t)tl.h * p.s_x1 + (int64_t)p0 * p.s_x2;
    const int64_t bb = (int64_t)tl.seq * p.seq_b + (int64_t)g * p.s_b1;
    const int64_t cb = (int64_t)tl.seq * p.seq_c + (int64_t)g * p.s_c1;
    const int64_t db = (int64_t)tl.seq * p.seq_dt + (int64_t)tl.h * p.s_dt1;
    const int64_t yb = (int64_t)tl.seq * p.seq_y + (int64_t)tl.h * p.s_y1 + (int64_t)p0 * p.s_y2;

    // ---- state entering this run --------------------------------------
    {
        int src;
        const bool clear = s0_row(p, tl.seq, &src);
        const float* s0 = p.s0 + (int64_t)src * p.seq_s + (int64_t)tl.h * p.s_s0 + (int64_t)p0 * p.s_s1;
        for (int i = tid; i < NMAX * kSlab; i += kThreads) {
            const int c = i / NMAX, n = i - c * NMAX;
            Ss[n * kXs + c] = (c < pw && n < N) ? (clear ? s0[(int64_t)c * p.s_s1 + n] : kNaN) : 0.0f;
        }
        // The carry loop below maps threads to (c, n) differently when
        // N < NMAX, so the fill must be complete first.
        __syncthreads();
        const int64_t unit0 = ((int64_t)tl.seq * p.H + tl.h) * p.run_slots;
        for (int r = 0; r < tl.run; ++r) {
            const float a = expf(p.lam[unit0 + r]);
            const float* ag = p.agg + (unit0 + r) * (int64_t)p.P * N + (int64_t)p0 * N;
            for (int i = tid; i < pw * N; i += kThreads) {
                const int c = i / N, n = i - c * N;
                Ss[n * kXs + c] = fmaf(a, Ss[n * kXs + c], ag[(int64_t)c * N + n]);
            }
        }
    }

    constexpr int RI = CS / 16;   // rows per thread in G1/G2/G3
    constexpr int NI = NMAX / 16; // state rows per thread in G4

    for (int t0 = t_begin; t0 < t_end; t0 += CS) {
        const int tlen = min(CS, t_end - t0);
        float v = 0.0f;
        if (tid < tlen) v = dt_of(p.dt[db + (int64_t)(t0 + tid) * p.s_dt0], p.dt_min, p.dt_max);
        // Padded tokens carry dt = 0, so Lc stays at its last live value and
        // every exponent below is <= 0 (reference helix_common.h:110-120).
        const float pre = block_prefix(Ah * v, CS, tot);
        if (tid < CS) {
            dtv[tid] = v;
            Lc[tid] = pre;
        }
        load_bc<BF16, ROW>(Cs, p.C, cb, p.s_c0, t0, tlen, CS, N);
        load_bc<BF16, ROW>(Bs, p.B, bb, p.s_b0, t0, tlen, CS, N);
        load_x<BF16>(Xs, p, xb, t0, tlen, CS, pw);
        __syncthreads();
        const float Lend = Lc[CS - 1];
        if (tid < CS) {
            ev[tid] = expf(Lc[tid]);
            wv[tid] = dtv[tid] * expf(Lend - Lc[tid]);
        }

        // ---- G1: M = tril(C B^T) * exp(Lc_t - Lc_j) * dt_j ----------------
        {
            float m[RI][RI];
#pragma unroll
            for (int i = 0; i < RI; ++i)
#pragma unroll
                for (int k = 0; k < RI; ++k) m[i][k] = 0.0f;
            for (int n = 0; n < N; n += 4) {
                float4 a[RI], b[RI];
#pragma unroll
                for (int i = 0; i < RI; ++i)
                    a[i] = *reinterpret_cast<const float4*>(Cs + (ty + 16 * i) * ROW + n);
#pragma unroll
                for (int k = 0; k < RI; ++k)
                    b[k] = *reinterpret_cast<const float4*>(Bs + (tx + 16 * k) * ROW + n);
#pragma unroll
                for (int i = 0; i < RI; ++i)
#pragma unroll
                    for (int k = 0; k < RI; ++k) {
                        m[i][k] = fmaf(a[i].x, b[k].x, m[i][k]);
                        m[i][k] = fmaf(a[i].y, b[k].y, m[i][k]);
                        m[i][k] = fmaf(a[i].z, b[k].z, m[i][k]);
                        m[i][k] = fmaf(a[i].w, b[k].w, m[i][k]);
                    }
            }
#pragma unroll
            for (int i = 0; i < RI; ++i)
#pragma unroll
                for (int k = 0; k < RI; ++k) {
                    const int t = ty + 16 * i, j = tx + 16 * k;
                    Ms[t * MR + j] = j <= t ? m[i][k] * expf(Lc[t] - Lc[j]) * dtv[j] : 0.0f;
                }
        }
        __syncthreads();

        // ---- G2 + G3: y = M x + exp(Lc_t) C S -----------------------------
        {
            float yi[RI][4], ye[RI][4];
#pragma unroll
            for (int i = 0; i < RI; ++i)
#pragma unroll
                for (int k = 0; k < 4; ++k) yi[i][k] = ye[i][k] = 0.0f;
            for (int j = 0; j < CS; ++j) {
                const float4 xv = *reinterpret_cast<const float4*>(Xs + j * kXs + 4 * tx);
#pragma unroll
                for (int i = 0; i < RI; ++i) {
                    const float mv = Ms[(ty + 16 * i) * MR + j];
                    yi[i][0] = fmaf(mv, xv.x, yi[i][0]);
                    yi[i][1] = fmaf(mv, xv.y, yi[i][1]);
                    yi[i][2] = fmaf(mv, xv.z, yi[i][2]);
                    yi[i][3] = fmaf(mv, xv.w, yi[i][3]);
                }
            }
            for (int n = 0; n < N; ++n) {
                const float4 sv = *reinterpret_cast<const float4*>(Ss + n * kXs + 4 * tx);
#pragma unroll
                for (int i = 0; i < RI; ++i) {
                    const float cv = Cs[(ty + 16 * i) * ROW + n];
                    ye[i][0] = fmaf(cv, sv.x, ye[i][0]);
                    ye[i][1] = fmaf(cv, sv.y, ye[i][1]);
                    ye[i][2] = fmaf(cv, sv.z, ye[i][2]);
                    ye[i][3] = fmaf(cv, sv.w, ye[i][3]);
                }
            }
#pragma unroll
            for (int i = 0; i < RI; ++i) {
                const int t = ty + 16 * i;
                if (t >= tlen) continue;
                const float e = ev[t];
                float* yr = p.y + yb + (int64_t)(t0 + t) * p.s_y0;
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    const int c = 4 * tx + k;
                    if (c < pw) yr[(int64_t)c * p.s_y2] = fmaf(e, ye[i][k], yi[i][k]);
                }
            }
        }
        __syncthreads();

        // ---- G4 + carry: S = exp(Lend) S + B^T diag(w) x ------------------
        {
            const float cd = expf(Lend);
            float a4[NI][4];
#pragma unroll
            for (int i = 0; i < NI; ++i)
#pragma unroll
                for (int k = 0; k < 4; ++k) a4[i][k] = 0.0f;
            for (int j = 0; j < tlen; ++j) {
                const float w = wv[j];
                const float4 xv = *reinterpret_cast<const float4*>(Xs + j * kXs + 4 * tx);
                const float xw[4] = {xv.x * w, xv.y * w, xv.z * w, xv.w * w};
#pragma unroll
                for (int i = 0; i < NI; ++i) {
                    const int n = ty + 16 * i;
                    const float b = n < N ? Bs[j * ROW + n] : 0.0f;
#pragma unroll
                    for (int k = 0; k < 4; ++k) a4[i][k] = fmaf(b, xw[k], a4[i][k]);
                }
            }
#pragma unroll
            for (int i = 0; i < NI; ++i) {
                const int n = ty + 16 * i;
                if (n >= N) continue;
                float4* sp = reinterpret_cast<float4*>(Ss + n * kXs + 4 * tx);
                float4 s = *sp;
                s.x = fmaf(cd, s.x, a4[i][0]);
                s.y = fmaf(cd, s.y, a4[i][1]);
                s.z = fmaf(cd, s.z, a4[i][2]);
                s.w = fmaf(cd, s.w, a4[i][3]);
                *sp = s;
            }
        }
        __syncthreads();
    }

    if (tl.run == p.n_runs - 1) {
        float* s1 = p.s1 + (int64_t)tl.seq * p.seq_s + (int64_t)tl.h * p.s_s0 + (int64_t)p0 * p.s_s1;
        for (int i = tid; i < pw * N; i += kThreads) {
            const int c = i / N, n = i - c * N;
            s1[(int64_t)c * p.s_s1 + n] = Ss[n * kXs + c];
        }
    }
}

template <int CS, int NMAX, bool BF16>
int configure_one() {
    using SM = SimtSmem<CS, NMAX>;
    cudaError_t e = cudaFuncSetAttribute(simt_out_kernel<CS, NMAX, BF16>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)SM::out_bytes);
    if (e != cudaSuccess) return e;
    return cudaFuncSetAttribute(simt_state_kernel<CS, NMAX, BF16>,
                                cudaFuncAttributeMaxDynamicSharedMemorySize, (int)SM::state_bytes);
}

}  // namespace

int configure_simt(const helix_ctx*) {
    int e;
    if ((e = configure_one<64, 128, false>()) != cudaSuccess) return e;
    if ((e = configure_one<64, 128, true>()) != cudaSuccess) return e;
    if ((e = configure_one<32, 256, false>()) != cudaSuccess) return e;
    return configure_one<32, 256, true>();
}

namespace {
template <int CS, int NMAX, bool BF16>
int launch_simt_t(const Plan& pl, const ScanParams& p, int n_seq, cudaStream_t st) {
    using SM = SimtSmem<CS, NMAX>;
    const char* only = std::getenv("HELIX_ONLY_PASS");
    const bool do_a = !only || *only == 'A';
    const bool do_c = !only || *only == 'C';
    const int64_t per_run = (int64_t)p.n_pslab * p.H;
    if (pl.need_state_kernel && do_a && !pl.states_ready) {
        const int runs = pl.state_runs;
        simt_state_kernel<CS, NMAX, BF16>
            <<<(unsigned)(per_run * runs * n_seq), kThreads, SM::state_bytes, st>>>(p, runs);
        const cudaError_t e = cudaGetLastError();
        if (e != cudaSuccess) return e;
    }
    if (do_c) {
        simt_out_kernel<CS, NMAX, BF16>
            <<<(unsigned)(per_run * pl.n_runs * n_seq), kThreads, SM::out_bytes, st>>>(p);
        const cudaError_t e = cudaGetLastError();
        if (e != cudaSuccess) return e;
    }
    return cudaSuccess;
}
}  // namespace

template <int CS, int NMAX, bool BF16>
int launch_simt_states_t(const Plan& pl, const ScanParams& p, cudaStream_t st) {
    using SM = SimtSmem<CS, NMAX>;
    const int64_t per_run = (int64_t)p.n_pslab * p.H;
    simt_state_kernel<CS, NMAX, BF16>
        <<<(unsigned)(per_run * pl.state_runs * p.S), kThreads, SM::state_bytes, st>>>(p, pl.state_runs);
    return cudaGetLastError();
}

int launch_simt_states(const helix_ctx*, const Plan& pl, const ScanParams& p, void* stream) {
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (p.N <= 128)
        return p.io_bf16 ? launch_simt_states_t<64, 128, true>(pl, p, st) : launch_simt_states_t<64, 128, false>(pl, p, st);
    return p.io_bf16 ? launch_simt_states_t<32, 256, true>(pl, p, st) : launch_simt_states_t<32, 256, false>(pl, p, st);
}

int launch_simt(const helix_ctx*, const Plan& pl, const ScanParams& p, void* stream) {
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const int n_seq = p.S;
    if (p.N <= 128)
        return p.io_bf16 ? launch_simt_t<64, 128, true>(pl, p, n_seq, st)
                         : launch_simt_t<64, 128, false>(pl, p, n_seq, st);
    return p.io_bf16 ? launch_simt_t<32, 256, true>(pl, p, n_seq, st)
                     : launch_simt_t<32, 256, false>(pl, p, n_seq, st);
}

}  // namespace hx
