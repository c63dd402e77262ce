/* helix_oracle.c -- TEST INFRASTRUCTURE ONLY.
 *
 * CPU restatement, in plain C with fp64 arithmetic, of the HELIX reference's
 * ground truth for the SSD scan.  Only tests/, __graft_entry__.smoke() and
 * bench.py's CPU-baseline leg load this library, and only as the checker or
 * the timed CPU baseline; the shipped library never links or calls it.
 *
 * Parity pin: tests/test_oracle.py checks every function here against the
 * reference's own fp64 oracle compiled from its sources (oracle/_ref, built by
 * oracle/Makefile) and against the committed golden vectors in tests/golden/.
 *
 * Semantics followed (reference file:line):
 *   softplus with the v > 20 shortcut      src/reference/scan_ref.cpp:13-17
 *   clamp to [dt_min, dt_max] after it     src/reference/scan_ref.cpp:19-24
 *   A[h*s_a] (+n for diagonal A)           src/reference/scan_ref.cpp:27-29
 *   group g = h / (n_head / n_group)       src/reference/scan_ref.cpp:38, :47
 *   ids selects the s0 row, s1 written at seq   src/reference/scan_ref.cpp:43, :49, :71
 *   sequential recurrence, f32 store only  src/reference/scan_ref.cpp:33-76
 *   chunk-boundary snapshots               src/reference/scan_ref.cpp:80-143
 *   chunked G1..G4 reassociation           src/reference/scan_chunked_ref.cpp:30-137
 */
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#include "helix/helix.h"

#define OR_EXPORT __attribute__((visibility("default")))

static double or_softplus(double v) { return v > 20.0 ? v : log1p(exp(v)); }

static double or_dt(const helix_scan_desc* d, const float* dt, int64_t seq, int64_t t, int64_t h) {
    double v = or_softplus((double)dt[seq * d->seq_dt + t * d->s_dt[0] + h * d->s_dt[1]]);
    if (v < (double)d->dt_min) v = (double)d->dt_min;
    if (v > (double)d->dt_max) v = (double)d->dt_max;
    return v;
}

/* Dense-stride defaults, restating reference src/runtime/desc.cpp:9-46. */
OR_EXPORT void oracle_desc_init(helix_scan_desc* d, int32_t L, int32_t S, int32_t H,
                                int32_t P, int32_t N, int32_t G) {
    memset(d, 0, sizeof(*d));
    d->n_tok = L; d->n_seq = S; d->n_head = H; d->head_dim = P; d->d_state = N; d->n_group = G;
    const int64_t l = L, h = H, p = P, n = N, g = G;
    d->s_x[0] = h * p; d->s_x[1] = p; d->s_x[2] = 1; d->seq_x = l * h * p;
    d->s_y[0] = h * p; d->s_y[1] = p; d->s_y[2] = 1; d->seq_y = l * h * p;
    d->s_b[0] = g * n; d->s_b[1] = n; d->s_b[2] = 1; d->seq_b = l * g * n;
    d->s_c[0] = g * n; d->s_c[1] = n; d->s_c[2] = 1; d->seq_c = l * g * n;
    d->s_dt[0] = h;    d->s_dt[1] = 1;                d->seq_dt = l * h;
    d->s_s[0] = p * n; d->s_s[1] = n; d->s_s[2] = 1; d->seq_s = h * p * n;
    d->s_a = 1;
    d->chunk = 0;
    d->a_form = HELIX_A_SCALAR_PER_HEAD;
    d->io_dtype = HELIX_F32;
    d->compute_dtype = HELIX_F32;
    d->backend = HELIX_BACKEND_AUTO;
    d->multipass = false;
    d->dt_min = 0.0f;
    d->dt_max = INFINITY;
}

/* One (seq, head) slice of the sequential recurrence.  `snap` (optional)
 * receives the state after every `chunk`-th token and after the last token,
 * in the caller's state layout, as n_chunks blocks of n_seq*seq_s doubles. */
static void scan_slice(const helix_scan_desc* d, int64_t seq, int64_t h,
                       const float* s0, const float* x, const float* dt, const float* A,
                       const float* B, const float* C, const int32_t* ids,
                       float* y, float* s1, int32_t chunk, double* snap, int64_t snap_stride,
                       double* s /* N scratch */, double* dA /* N scratch */) {
    const int64_t P = d->head_dim, N = d->d_state;
    const int64_t g = h / (d->n_head / d->n_group);
    const int64_t src = ids ? (int64_t)ids[seq] : seq;
    const int diag = d->a_form == HELIX_A_DIAG_PER_CHANNEL;

    for (int64_t p = 0; p < P; ++p) {
        const float* si = s0 + src * d->seq_s + h * d->s_s[0] + p * d->s_s[1];
        for (int64_t n = 0; n < N; ++n) s[n] = (double)si[n * d->s_s[2]];

        for (int64_t t = 0; t < d->n_tok; ++t) {
            const double dtt = or_dt(d, dt, seq, t, h);
            const double xt = (double)x[seq * d->seq_x + t * d->s_x[0] + h * d->s_x[1] + p * d->s_x[2]];
            const float* Bt = B + seq * d->seq_b + t * d->s_b[0] + g * d->s_b[1];
            const float* Ct = C + seq * d->seq_c + t * d->s_c[0] + g * d->s_c[1];
            if (diag) {
                for (int64_t n = 0; n < N; ++n) dA[n] = exp((double)A[h * d->s_a + n] * dtt);
            } else {
                const double a = exp((double)A[h * d->s_a] * dtt);
                for (int64_t n = 0; n < N; ++n) dA[n] = a;
            }
            double acc = 0.0;
            for (int64_t n = 0; n < N; ++n) {
                s[n] = dA[n] * s[n] + dtt * (double)Bt[n * d->s_b[2]] * xt;
                acc += (double)Ct[n * d->s_c[2]] * s[n];
            }
            y[seq * d->seq_y + t * d->s_y[0] + h * d->s_y[1] + p * d->s_y[2]] = (float)acc;

            if (snap && chunk > 0 && ((t + 1) % chunk == 0 || t + 1 == d->n_tok)) {
                double* dst = snap + (t / chunk) * snap_stride + seq * d->seq_s + h * d->s_s[0] +
                              p * d->s_s[1];
                for (int64_t n = 0; n < N; ++n) dst[n * d->s_s[2]] = s[n];
            }
        }
        float* so = s1 + seq * d->seq_s + h * d->s_s[0] + p * d->s_s[1];
        for (int64_t n = 0; n < N; ++n) so[n * d->s_s[2]] = (float)s[n];
    }
}

/* Sequential fp64 recurrence over every (seq, head); reference scan_ref.cpp:33-76. */
OR_EXPORT void oracle_scan(const helix_scan_desc* d, const float* s0, const float* x,
                           const float* dt, const float* A, const float* B, const float* C,
                           const int32_t* ids, float* y, float* s1) {
    double* s = (double*)malloc(sizeof(double) * 2 * (size_t)d->d_state);
    for (int64_t seq = 0; seq < d->n_seq; ++seq)
        for (int64_t h = 0; h < d->n_head; ++h)
            scan_slice(d, seq, h, s0, x, dt, A, B, C, ids, y, s1, 0, NULL, 0, s, s + d->d_state);
    free(s);
}

/* As oracle_scan, also writing the state at every chunk boundary (and after
 * the last token) into `snap`: n_chunks blocks of n_seq*seq_s doubles.
 * Reference scan_ref.cpp:80-143. */
OR_EXPORT void oracle_scan_snapshots(const helix_scan_desc* d, const float* s0, const float* x,
                                     const float* dt, const float* A, const float* B,
                                     const float* C, const int32_t* ids, float* y, float* s1,
                                     int32_t chunk, double* snap) {
    double* s = (double*)malloc(sizeof(double) * 2 * (size_t)d->d_state);
    const int64_t stride = (int64_t)d->n_seq * d->seq_s;
    for (int64_t seq = 0; seq < d->n_seq; ++seq)
        for (int64_t h = 0; h < d->n_head; ++h)
            scan_slice(d, seq, h, s0, x, dt, A, B, C, ids, y, s1, chunk, snap, stride, s,
                       s + d->d_state);
    free(s);
}

/* ---- threaded driver: (seq, head) slices are independent ---------------- */

typedef struct {
    const helix_scan_desc* d;
    const float *s0, *x, *dt, *A, *B, *C;
    const int32_t* ids;
    float *y, *s1;
    int64_t first, last; /* flattened (seq*H + h) range */
} mt_job;

static void* mt_worker(void* arg) {
    mt_job* j = (mt_job*)arg;
    double* s = (double*)malloc(sizeof(double) * 2 * (size_t)j->d->d_state);
    for (int64_t i = j->first; i < j->last; ++i)
        scan_slice(j->d, i / j->d->n_head, i % j->d->n_head, j->s0, j->x, j->dt, j->A, j->B, j->C,
                   j->ids, j->y, j->s1, 0, NULL, 0, s, s + j->d->d_state);
    free(s);
    return NULL;
}

/* oracle_scan split across `nthreads` POSIX threads by (seq, head) slice.
 * Bit-identical to oracle_scan: each slice runs the same code in the same
 * order, only on another thread. */
OR_EXPORT void oracle_scan_mt(const helix_scan_desc* d, const float* s0, const float* x,
                              const float* dt, const float* A, const float* B, const float* C,
                              const int32_t* ids, float* y, float* s1, int32_t nthreads) {
    const int64_t total = (int64_t)d->n_seq * d->n_head;
    if (nthreads < 1) nthreads = 1;
    if (nthreads > total) nthreads = (int32_t)total;
    pthread_t* th = (pthread_t*)malloc(sizeof(pthread_t) * (size_t)nthreads);
    mt_job* jobs = (mt_job*)malloc(sizeof(mt_job) * (size_t)nthreads);
    for (int32_t k = 0; k < nthreads; ++k) {
        mt_job j = {d, s0, x, dt, A, B, C, ids, y, s1, total * k / nthreads,
                    total * (k + 1) / nthreads};
        jobs[k] = j;
        pthread_create(&th[k], NULL, mt_worker, &jobs[k]);
    }
    for (int32_t k = 0; k < nthreads; ++k) pthread_join(th[k], NULL);
    free(th);
    free(jobs);
}

/* ---- chunked reassociation (scalar A only) ------------------------------- */
/* Restates reference scan_chunked_ref.cpp:30-137: per chunk,
 *   G1  M[t][j] = (C_t . B_j) exp(Lcum_t - Lcum_j), j <= t
 *   G2  y_intra = M . dtX
 *   G3  y_inter = exp(Lcum_t) C_t . S
 *   G4  S      <- exp(L_end) S + sum_j exp(L_end - Lcum_j) B_j dtX_j
 * Returns -1 (and writes nothing) for diagonal A, which has no such form. */
OR_EXPORT int oracle_scan_chunked(const helix_scan_desc* d, const float* s0, const float* x,
                                  const float* dt, const float* A, const float* B, const float* C,
                                  const int32_t* ids, float* y, float* s1) {
    if (d->a_form != HELIX_A_SCALAR_PER_HEAD) return -1;
    const int64_t H = d->n_head, P = d->head_dim, N = d->d_state, L = d->n_tok;
    const int64_t K = d->chunk > 0 ? d->chunk : 64;
    const int64_t hpg = d->n_head / d->n_group;

    double* S = (double*)malloc(sizeof(double) * (size_t)(P * N));
    double* dtX = (double*)malloc(sizeof(double) * (size_t)(K * P));
    double* M = (double*)malloc(sizeof(double) * (size_t)(K * K));
    double* Lc = (double*)malloc(sizeof(double) * (size_t)K);

    for (int64_t seq = 0; seq < d->n_seq; ++seq) {
        const int64_t src = ids ? (int64_t)ids[seq] : seq;
        for (int64_t h = 0; h < H; ++h) {
            const int64_t g = h / hpg;
            const double Ah = (double)A[h * d->s_a];
            const float* si = s0 + src * d->seq_s + h * d->s_s[0];
            for (int64_t p = 0; p < P; ++p)
                for (int64_t n = 0; n < N; ++n)
                    S[p * N + n] = (double)si[p * d->s_s[1] + n * d->s_s[2]];

            for (int64_t t0 = 0; t0 < L; t0 += K) {
                const int64_t tl = (L - t0) < K ? (L - t0) : K;
                double run = 0.0;
                for (int64_t j = 0; j < tl; ++j) {
                    const double v = or_dt(d, dt, seq, t0 + j, h);
                    run += Ah * v;
                    Lc[j] = run;
                    for (int64_t p = 0; p < P; ++p)
                        dtX[j * P + p] =
                            v * (double)x[seq * d->seq_x + (t0 + j) * d->s_x[0] + h * d->s_x[1] +
                                          p * d->s_x[2]];
                }
                const double Lend = Lc[tl - 1];
                for (int64_t t = 0; t < tl; ++t) {
                    const float* Ct = C + seq * d->seq_c + (t0 + t) * d->s_c[0] + g * d->s_c[1];
                    for (int64_t j = 0; j < tl; ++j) {
                        double cb = 0.0;
                        if (j <= t) {
                            const float* Bj = B + seq * d->seq_b + (t0 + j) * d->s_b[0] + g * d->s_b[1];
                            for (int64_t n = 0; n < N; ++n)
                                cb += (double)Ct[n * d->s_c[2]] * (double)Bj[n * d->s_b[2]];
                            cb *= exp(Lc[t] - Lc[j]);
                        }
                        M[t * K + j] = cb;
                    }
                }
                for (int64_t t = 0; t < tl; ++t) {
                    const float* Ct = C + seq * d->seq_c + (t0 + t) * d->s_c[0] + g * d->s_c[1];
                    const double eL = exp(Lc[t]);
                    for (int64_t p = 0; p < P; ++p) {
                        double intra = 0.0, inter = 0.0;
                        for (int64_t j = 0; j <= t; ++j) intra += M[t * K + j] * dtX[j * P + p];
                        for (int64_t n = 0; n < N; ++n) inter += (double)Ct[n * d->s_c[2]] * S[p * N + n];
                        y[seq * d->seq_y + (t0 + t) * d->s_y[0] + h * d->s_y[1] + p * d->s_y[2]] =
                            (float)(intra + eL * inter);
                    }
                }
                const double cd = exp(Lend);
                for (int64_t p = 0; p < P; ++p)
                    for (int64_t n = 0; n < N; ++n) {
                        double ds = 0.0;
                        for (int64_t j = 0; j < tl; ++j) {
                            const float* Bj = B + seq * d->seq_b + (t0 + j) * d->s_b[0] + g * d->s_b[1];
                            ds += exp(Lend - Lc[j]) * (double)Bj[n * d->s_b[2]] * dtX[j * P + p];
                        }
                        S[p * N + n] = cd * S[p * N + n] + ds;
                    }
            }
            float* so = s1 + seq * d->seq_s + h * d->s_s[0];
            for (int64_t p = 0; p < P; ++p)
                for (int64_t n = 0; n < N; ++n) so[p * d->s_s[1] + n * d->s_s[2]] = (float)S[p * N + n];
        }
    }
    free(S); free(dtX); free(M); free(Lc);
    return 0;
}

/* ---- run-state carry (the combine the library's runs and the multi-GPU
 * L-split rely on) ---------------------------------------------------------
 * State after a slice that starts from s_in:  exp(lam) * s_in + agg, where
 * agg is the slice's state from a zero start and lam = sum_t A*dt_t.  This is
 * the associative operator (a1,b1).(a2,b2) = (a1 a2, a2 b1 + b2) of reference
 * src/kernels/helix_scan_multipass.metal:10-15 applied to a whole slice.
 * Given K slices in order, writes carry[k] = state entering slice k:
 *   carry[0] = s0;  carry[k+1] = exp(lam[k]) * carry[k] + agg[k].
 * Arrays are [K][n_elem] (agg, carry) and [K] (lam), all fp64. */
OR_EXPORT void oracle_carry_chain(int32_t K, int64_t n_elem, const double* s0, const double* agg,
                                  const double* lam, double* carry) {
    for (int64_t i = 0; i < n_elem; ++i) carry[i] = s0[i];
    for (int32_t k = 0; k + 1 < K; ++k) {
        const double a = exp(lam[k]);
        for (int64_t i = 0; i < n_elem; ++i)
            carry[(k + 1) * n_elem + i] = a * carry[k * n_elem + i] + agg[k * n_elem + i];
    }
}

/* ---- the reference test harness's input generator -----------------------
 * Restates reference tests/harness.hpp:22-34 (xorshift64, uniform from the top
 * 24 bits, float arithmetic) and :151-186 (fill order s0, x, dt, A, B, C and
 * the SHORT/LONG memory regimes), so that fixtures built here use exactly the
 * inputs the reference's own tests use for a given seed. */
typedef struct { uint64_t s; } or_rng;

static uint64_t or_next(or_rng* r) {
    r->s ^= r->s << 13;
    r->s ^= r->s >> 7;
    r->s ^= r->s << 17;
    return r->s;
}

static float or_uniform(or_rng* r, float lo, float hi) {
    const float u = (float)(or_next(r) >> 40) / 16777216.0f;
    return lo + u * (hi - lo);
}

OR_EXPORT void oracle_harness_fill(int32_t L, int32_t S, int32_t H, int32_t P, int32_t N,
                                   int32_t G, uint64_t seed, int32_t long_memory, float* s0,
                                   float* x, float* dt, float* A, float* B, float* C) {
    or_rng r = {seed ? seed : 1};
    const size_t ns = (size_t)S * H * P * N, nx = (size_t)S * L * H * P, nd = (size_t)S * L * H;
    const size_t nb = (size_t)S * L * G * N;
    for (size_t i = 0; i < ns; ++i) s0[i] = or_uniform(&r, -0.5f, 0.5f);
    for (size_t i = 0; i < nx; ++i) x[i] = or_uniform(&r, -1.0f, 1.0f);
    if (long_memory) {
        for (size_t i = 0; i < nd; ++i) dt[i] = or_uniform(&r, -7.0f, -4.5f);
        for (int32_t h = 0; h < H; ++h) A[h] = -expf(or_uniform(&r, -0.5f, 1.0f));
    } else {
        for (size_t i = 0; i < nd; ++i) dt[i] = or_uniform(&r, -4.0f, 2.0f);
        for (int32_t h = 0; h < H; ++h) A[h] = -expf(or_uniform(&r, -2.0f, 0.5f));
    }
    const float sc = 1.0f / sqrtf((float)N);
    for (size_t i = 0; i < nb; ++i) B[i] = or_uniform(&r, -sc, sc);
    for (size_t i = 0; i < nb; ++i) C[i] = or_uniform(&r, -sc, sc);
}
