// scan_shard.cu -- the two small kernels of the sequence-split (L-split)
// scan: folding one shard's run states into its final state, and combining
// the final states of earlier shards into a shard's carried-in state.
//
// Both are elementwise over a (seq, head) state of P x N floats: one thread
// per element, runs (or shards) visited in order, a handful of independent
// loads kept in flight.  They move a few MB and sit far off the hot path; the
// combine is the associative operator (a1, b1) o (a2, b2) = (a1 a2, a2 b1 + b2)
// over (decay, state) pairs.
#include <cuda_runtime.h>

#include "../runtime/internal.h"
#include "common.cuh"

namespace hx {
namespace {

constexpr int kThreads = 256;

// state[seq][h][p][n] = fold_r (exp(lam_r) S + agg_r), S from 0.
__global__ void __launch_bounds__(kThreads) shard_fold_kernel(ScanParams p, float* state, float* log_decay) {
    const int64_t per_head = (int64_t)p.P * p.N;
    const int64_t gid = (int64_t)blockIdx.x * kThreads + threadIdx.x;
    const int64_t head_lin = gid / per_head;  // seq * H + h
    if (head_lin >= (int64_t)p.S * p.H) return;
    const int64_t e = gid - head_lin * per_head;
    const int seq = (int)(head_lin / p.H), h = (int)(head_lin % p.H);
    const int c = (int)(e / p.N), n = (int)(e % p.N);
    const int64_t unit0 = head_lin * p.run_slots;
    float S = 0.0f, total = 0.0f;
    int r = 0;
    for (; r + 4 <= p.state_runs; r += 4) {
        float a[4], v[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            a[k] = p.lam[unit0 + r + k];
            v[k] = p.agg[(unit0 + r + k) * per_head + e];
        }
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            S = fmaf(expf(a[k]), S, v[k]);
            total += a[k];
        }
    }
    for (; r < p.state_runs; ++r) {
        const float a = p.lam[unit0 + r];
        S = fmaf(expf(a), S, p.agg[(unit0 + r) * per_head + e]);
        total += a;
    }
    state[(int64_t)seq * p.seq_s + (int64_t)h * p.s_s0 + (int64_t)c * p.s_s1 + n] = S;
    if (e == 0) log_decay[head_lin] = total;
}

// carry = fold_{j < n_prev} (exp(ld_j) S + states_j), S from s0[ids[seq]].
__global__ void __launch_bounds__(kThreads)
    carry_combine_kernel(ScanParams p, const float* states, const float* ld, int n_prev, float* carry) {
    const int64_t per_head = (int64_t)p.P * p.N;
    const int64_t n_state = (int64_t)p.S * p.H * per_head;
    const int64_t gid = (int64_t)blockIdx.x * kThreads + threadIdx.x;
    if (gid >= n_state) return;
    const int64_t head_lin = gid / per_head;
    const int64_t e = gid - head_lin * per_head;
    const int seq = (int)(head_lin / p.H), h = (int)(head_lin % p.H);
    const int c = (int)(e / p.N), n = (int)(e % p.N);
    int src;
    float S = s0_row(p, seq, &src) ? p.s0[(int64_t)src * p.seq_s + (int64_t)h * p.s_s0 + (int64_t)c * p.s_s1 + n]
                                   : kNaN;
    const int64_t n_heads = (int64_t)p.S * p.H;
    for (int j = 0; j < n_prev; ++j)
        S = fmaf(expf(ld[(int64_t)j * n_heads + head_lin]), S, states[(int64_t)j * n_state + gid]);
    carry[(int64_t)seq * p.seq_s + (int64_t)h * p.s_s0 + (int64_t)c * p.s_s1 + n] = S;
}

unsigned grid_for(int64_t n) { return (unsigned)((n + kThreads - 1) / kThreads); }

}  // namespace

int launch_shard_fold(const ScanParams& p, float* state, float* log_decay, void* stream) {
    const int64_t n = (int64_t)p.S * p.H * p.P * p.N;
    shard_fold_kernel<<<grid_for(n), kThreads, 0, static_cast<cudaStream_t>(stream)>>>(p, state, log_decay);
    return cudaGetLastError();
}

int launch_carry_combine(const ScanParams& p, const float* states, const float* log_decays, int n_prev,
                         float* carry, void* stream) {
    const int64_t n = (int64_t)p.S * p.H * p.P * p.N;
    carry_combine_kernel<<<grid_for(n), kThreads, 0, static_cast<cudaStream_t>(stream)>>>(p, states, log_decays,
                                                                                         n_prev, carry);
    return cudaGetLastError();
}

}  // namespace hx
