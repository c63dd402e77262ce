// common.cuh -- device helpers shared by both kernel families.
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include "../runtime/internal.h"

namespace hx {

// Codes of the device fault word (helix_device_fault): the first event
// recorded since the word was last read.
enum : unsigned {
    kFaultTmaOut = 1,      // output kernel: a TMA arrival wait ran out
    kFaultMmaOut = 2,      // output kernel: an MMA / hand-off wait ran out
    kFaultTmaState = 3,    // state kernel: a TMA arrival wait ran out
    kFaultMmaState = 4,    // state kernel: an MMA / hand-off wait ran out
    kFaultIdsOverlap = 5,  // an s0 row selected by ids overlaps the s1 rows written
    kFaultTestStall = 6,   // test hook HELIX_TEST_STALL_CYCLES: a wait nothing ends ran out
};

constexpr float kNaN = __builtin_nanf("");

// Row of s0 that sequence seq starts from: ids[seq], or seq without ids.
// Returns false, and records kFaultIdsOverlap, when ids selects a row whose
// bytes overlap the s1 rows this call writes (other CTAs may be writing
// them while it is read); the caller then starts the sequence from NaN, so
// its outputs come out NaN instead of silently wrong.  Overlap with the
// first n_seq rows of s0 is rejected on the host before anything runs; this
// covers the rows only ids reaches.
__device__ __forceinline__ bool s0_row(const ScanParams& p, int seq, int* src) {
    const int r = p.has_ids ? p.ids[seq] : seq;
    *src = r;
    if (!p.has_ids) return true;
    const char* a = reinterpret_cast<const char*>(p.s0 + (int64_t)r * p.seq_s);
    const char* w = reinterpret_cast<const char*>(p.s1);
    if (a < w + p.s1_bytes && w < a + p.s_row_bytes) {
        if (p.fault) atomicCAS(p.fault, 0u, kFaultIdsOverlap);
        return false;
    }
    return true;
}

// log(1 + e^v) for v <= 20 as max(v, 0) + log1p(u), u = e^-|v| in (0, 1],
// with log1p(u) = 2 atanh(s) = 2 (s + s^3/3 + s^5/5 + ... + s^15/15),
// s = u / (2 + u) <= 1/3 (the Taylor series of atanh; the first omitted term
// is below 2e-9 of the sum).  One exp2 and one fast divide: a few ulp from
// the correctly rounded value, against two full library calls on the chain
// of every chunk's decay vectors.
__device__ __forceinline__ float softplus_le20(float v) {
    float u;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(u) : "f"(-fabsf(v) * 1.4426950408889634f));
    const float s = __fdividef(u, 2.0f + u);
    const float s2 = s * s;
    float t = 1.0f / 15.0f;
    t = fmaf(t, s2, 1.0f / 13.0f);
    t = fmaf(t, s2, 1.0f / 11.0f);
    t = fmaf(t, s2, 1.0f / 9.0f);
    t = fmaf(t, s2, 1.0f / 7.0f);
    t = fmaf(t, s2, 1.0f / 5.0f);
    t = fmaf(t, s2, 1.0f / 3.0f);
    t = fmaf(t, s2, 1.0f);
    return fmaxf(v, 0.0f) + 2.0f * s * t;
}

// softplus with the v > 20 shortcut, then the clamp
// (reference src/kernels/helix_common.h:14-20, src/reference/scan_ref.cpp:13-24).
__device__ __forceinline__ float dt_of(float raw, float lo, float hi) {
    float v = raw > 20.0f ? raw : softplus_le20(raw);
    v = v < lo ? lo : v;
    v = v > hi ? hi : v;
    return v;
}

template <bool BF16>
__device__ __forceinline__ float ld_io(const void* base, int64_t i) {
    if constexpr (BF16)
        return __bfloat162float(static_cast<const __nv_bfloat16*>(base)[i]);
    else
        return static_cast<const float*>(base)[i];
}

// Inclusive prefix sum over the first `n` threads of the block (n <= 32 *
// warps).  Every thread of the block must call it.  `tot` holds one float per
// warp.  Returns the prefix for threads < n (others get an unspecified value).
__device__ __forceinline__ float block_prefix(float v, int n, float* tot) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const float u = __shfl_up_sync(0xffffffffu, v, o);
        if (lane >= o) v += u;
    }
    if (lane == 31) tot[warp] = v;
    __syncthreads();
    const int nw = (n + 31) >> 5;
    float add = 0.0f;
    for (int w = 0; w < warp && w < nw; ++w) add += tot[w];
    __syncthreads();
    return v + add;
}

// Flattened CTA index -> (seq, run, head, slab), slab fastest, then head, so
// the CTAs of one group's heads run next to each other and share B/C in L2.
struct Tile {
    int seq, run, h, slab;
};
__device__ __forceinline__ Tile decode_tile(int b, int n_pslab, int H, int n_runs) {
    Tile t;
    t.slab = b % n_pslab;
    b /= n_pslab;
    t.h = b % H;
    b /= H;
    t.run = b % n_runs;
    t.seq = b / n_runs;
    return t;
}

}  // namespace hx
