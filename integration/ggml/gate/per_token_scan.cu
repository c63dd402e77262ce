// per_token_scan.cu -- MEASUREMENT BASELINE for the bridge's length gate.
//
// A plain per-token SSM scan of the kind a host framework runs for SSM_SCAN
// when HELIX declines: one CTA per (sequence, head), P x 4 threads, each
// thread holding d_state / 4 states of one channel in registers and walking
// the tokens in order (state update, then its share of y, reduced over the
// channel's four threads).  It is not part of the library; measure_gate.py
// times it against helix_scan_encode to find where the chunked scan starts
// to win, and checks it against the fp64 oracle first.
//
// Layouts are helix.h's dense ones: x, y (S, L, H, P); dt (S, L, H);
// B, C (S, L, G, N); A (H,); s0, s1 (S, H, P, N).  Scalar A; no dt clamp
// (softplus only), as the bridge's descriptor.
#include <cuda_runtime.h>

namespace {

template <int NPT>  // states per thread (d_state / 4)
__global__ void per_token_scan_kernel(int L, int H, int P, int N, int G, const float* x, const float* dt,
                                      const float* A, const float* B, const float* C, const float* s0, float* y,
                                      float* s1) {
    const int seq = blockIdx.x / H, h = blockIdx.x % H;
    const int c = threadIdx.x >> 2, part = threadIdx.x & 3;  // channel, quarter of the states
    const int g = h / (H / G);
    const int n0 = part * NPT;
    const bool live = c < P;
    float s[NPT];
    const float* s0p = s0 + (((size_t)seq * H + h) * P + (live ? c : 0)) * N + n0;
#pragma unroll
    for (int k = 0; k < NPT; ++k) s[k] = live ? s0p[k] : 0.0f;
    const float a_h = A[h];
    for (int t = 0; t < L; ++t) {
        const size_t tok = (size_t)seq * L + t;
        const float raw = dt[tok * H + h];
        const float d = raw > 20.0f ? raw : log1pf(expf(raw));
        const float decay = expf(a_h * d);
        const float xv = live ? x[(tok * H + h) * P + c] * d : 0.0f;
        const float* bt = B + (tok * G + g) * N + n0;
        const float* ct = C + (tok * G + g) * N + n0;
        float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
        for (int k = 0; k < NPT; k += 4) {
            const float4 b4 = *reinterpret_cast<const float4*>(bt + k);
            const float4 c4 = *reinterpret_cast<const float4*>(ct + k);
            s[k] = fmaf(decay, s[k], xv * b4.x);
            s[k + 1] = fmaf(decay, s[k + 1], xv * b4.y);
            s[k + 2] = fmaf(decay, s[k + 2], xv * b4.z);
            s[k + 3] = fmaf(decay, s[k + 3], xv * b4.w);
            acc[0] = fmaf(c4.x, s[k], acc[0]);
            acc[1] = fmaf(c4.y, s[k + 1], acc[1]);
            acc[2] = fmaf(c4.z, s[k + 2], acc[2]);
            acc[3] = fmaf(c4.w, s[k + 3], acc[3]);
        }
        float yv = (acc[0] + acc[1]) + (acc[2] + acc[3]);
        yv += __shfl_xor_sync(0xffffffffu, yv, 1);
        yv += __shfl_xor_sync(0xffffffffu, yv, 2);
        if (live && part == 0) y[(tok * H + h) * P + c] = yv;
    }
    if (live) {
        float* s1p = s1 + (((size_t)seq * H + h) * P + c) * N + n0;
#pragma unroll
        for (int k = 0; k < NPT; ++k) s1p[k] = s[k];
    }
}

}  // namespace

// Enqueues the per-token scan on `stream`; d_state must be 64, 128 or 256,
// head_dim at most 256.  Returns the launch status.
extern "C" int per_token_scan(int S, int L, int H, int P, int N, int G, const float* x, const float* dt,
                              const float* A, const float* B, const float* C, const float* s0, float* y, float* s1,
                              void* stream) {
    const dim3 grid(S * H), block(((P + 7) / 8) * 32);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (N == 64)
        per_token_scan_kernel<16><<<grid, block, 0, st>>>(L, H, P, N, G, x, dt, A, B, C, s0, y, s1);
    else if (N == 128)
        per_token_scan_kernel<32><<<grid, block, 0, st>>>(L, H, P, N, G, x, dt, A, B, C, s0, y, s1);
    else if (N == 256)
        per_token_scan_kernel<64><<<grid, block, 0, st>>>(L, H, P, N, G, x, dt, A, B, C, s0, y, s1);
    else
        return (int)cudaErrorInvalidValue;
    return (int)cudaGetLastError();
}
