// scan_cast.cu -- bf16 copies of F32-stored x, B and C for the tensor-core
// family (reference src/kernels/helix_cast.metal:19-46 and its use in
// src/runtime/dispatch.mm:232-245, which densify B and C to bf16 for the
// bf16 Pass C; here x is copied too, because the tensor-core kernels load
// all three with TMA from bf16 tiles).
//
// The copies are dense, in the caller's scratch (Plan::cast regions):
//   x  -> [S][L][H][Pp]  bf16 (bf16 family), Pp = head_dim rounded up to 8
//                        (TMA strides must be multiples of 16 bytes), or fp32
//                        (three-product family, only when TMA cannot read x
//                        as stored), Pp = head_dim rounded up to 4; channels
//                        P..Pp-1 hold 0
//   B, C -> [S][L][G][N] bf16 (d_state is a multiple of 8)
// Rounding is to nearest even, the same as the checkers' bf16 widening.
// For the three-product family (scan_tc3.cu) the kernel also writes the low
// halves of B and C, lo = bf16(v - hi), into copies of the same layout:
// hi + lo carries v to about 16 significant bits.
// HBM-bound: 4 bytes read and 2 (4 with the low halves) written per element,
// 16-byte loads where the source rows are contiguous and aligned.
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstdlib>

#include "../runtime/internal.h"
#include "common.cuh"

namespace hx {
namespace {

constexpr int kCastThreads = 256;

struct CastDst {
    __nv_bfloat16 *x, *b, *c;     // x: null when x is not copied
    __nv_bfloat16 *bl, *cl;       // low halves (three-product family), else null
    float* xf;                    // fp32 copy of x (three-product family), else null
    int pp;  // padded head_dim of the x copy
};

__device__ __forceinline__ uint2 bf16x4(float a, float b, float c, float e) {
    __nv_bfloat162 lo = __floats2bfloat162_rn(a, b), hi = __floats2bfloat162_rn(c, e);
    uint2 v;
    v.x = *reinterpret_cast<uint32_t*>(&lo);
    v.y = *reinterpret_cast<uint32_t*>(&hi);
    return v;
}

// v rounded to bf16 at d; with dl, also the rounding residual v - hi at dl.
__device__ __forceinline__ void put4(__nv_bfloat16* d, __nv_bfloat16* dl, const float (&v)[4]) {
    const uint2 h = bf16x4(v[0], v[1], v[2], v[3]);
    *reinterpret_cast<uint2*>(d) = h;
    if (dl) {
        const float h0 = __uint_as_float(h.x << 16), h1 = __uint_as_float(h.x & 0xffff0000u);
        const float h2 = __uint_as_float(h.y << 16), h3 = __uint_as_float(h.y & 0xffff0000u);
        *reinterpret_cast<uint2*>(dl) = bf16x4(v[0] - h0, v[1] - h1, v[2] - h2, v[3] - h3);
    }
}

// Four elements cols k..k+3 of one row (elements past `width` are zero).
__device__ __forceinline__ void cast_quad(const float* row, int64_t stride, int k, int width, __nv_bfloat16* dst,
                                          __nv_bfloat16* dst_lo) {
    float v[4];
    if (stride == 1 && k + 4 <= width && (reinterpret_cast<uintptr_t>(row + k) & 15) == 0) {
        const float4 f = __ldg(reinterpret_cast<const float4*>(row + k));
        v[0] = f.x;
        v[1] = f.y;
        v[2] = f.z;
        v[3] = f.w;
    } else {
#pragma unroll
        for (int e = 0; e < 4; ++e) v[e] = k + e < width ? __ldg(row + (int64_t)(k + e) * stride) : 0.0f;
    }
    put4(dst, dst_lo, v);
}

// x quad k..k+3 of one row as fp32 (elements past `width` are zero).
__device__ __forceinline__ void copy_quad(const float* row, int64_t stride, int k, int width, float* dst) {
    float4 v;
    v.x = k < width ? __ldg(row + (int64_t)k * stride) : 0.0f;
    v.y = k + 1 < width ? __ldg(row + (int64_t)(k + 1) * stride) : 0.0f;
    v.z = k + 2 < width ? __ldg(row + (int64_t)(k + 2) * stride) : 0.0f;
    v.w = k + 3 < width ? __ldg(row + (int64_t)(k + 3) * stride) : 0.0f;
    *reinterpret_cast<float4*>(dst) = v;
}

// The state kernel, launched behind this one as a programmatic dependent,
// may start at once: it waits (griddepcontrol.wait) before reading a copy.
__device__ __forceinline__ void allow_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

__global__ void __launch_bounds__(kCastThreads) cast_bf16_kernel(ScanParams p, CastDst d) {
    allow_dependents();
    const int64_t qx = (d.x || d.xf) ? (int64_t)p.S * p.L * p.H * (d.pp / 4) : 0;  // quads of x
    const int64_t qb = (int64_t)p.S * p.L * p.G * (p.N / 4);   // quads of B (and of C)
    const int64_t total = qx + 2 * qb;
    const float* x = static_cast<const float*>(p.x);
    const float* B = static_cast<const float*>(p.B);
    const float* C = static_cast<const float*>(p.C);
    for (int64_t q = (int64_t)blockIdx.x * kCastThreads + threadIdx.x; q < total;
         q += (int64_t)gridDim.x * kCastThreads) {
        if (q < qx) {
            const int64_t r = q / (d.pp / 4);  // (seq, tok, head) row
            const int k = 4 * (int)(q - r * (d.pp / 4));
            const int h = (int)(r % p.H);
            const int64_t st = r / p.H;
            const int t = (int)(st % p.L), seq = (int)(st / p.L);
            const float* row = x + (int64_t)seq * p.seq_x + (int64_t)t * p.s_x0 + (int64_t)h * p.s_x1;
            if (d.xf)
                copy_quad(row, p.s_x2, k, p.P, d.xf + r * d.pp + k);
            else
                cast_quad(row, p.s_x2, k, p.P, d.x + r * d.pp + k, nullptr);
        } else {
            const bool isc = q >= qx + qb;
            const int64_t u = q - qx - (isc ? qb : 0);
            const int64_t r = u / (p.N / 4);  // (seq, tok, group) row
            const int k = 4 * (int)(u - r * (p.N / 4));
            const int g = (int)(r % p.G);
            const int64_t st = r / p.G;
            const int t = (int)(st % p.L), seq = (int)(st / p.L);
            const float* row = isc ? C + (int64_t)seq * p.seq_c + (int64_t)t * p.s_c0 + (int64_t)g * p.s_c1
                                   : B + (int64_t)seq * p.seq_b + (int64_t)t * p.s_b0 + (int64_t)g * p.s_b1;
            __nv_bfloat16* lo = isc ? d.cl : d.bl;
            cast_quad(row, 1, k, p.N, (isc ? d.c : d.b) + r * p.N + k, lo ? lo + r * p.N + k : nullptr);
        }
    }
}

// Dense sources (the common case): x, B and C as flat arrays whose copies
// have the same element order.  Eight elements per thread step, two steps in
// flight per thread: the kernel is a stream of 16-byte loads and stores.
struct FlatSeg {
    const float* src;
    __nv_bfloat16* hi;
    __nv_bfloat16* lo;  // null: no low halves
    int64_t n8;         // groups of eight elements
};
struct FlatCast {
    FlatSeg seg[3];
};

__device__ __forceinline__ void cast8(const FlatSeg& g, int64_t k) {
    const float4 a = __ldg(reinterpret_cast<const float4*>(g.src) + 2 * k);
    const float4 b = __ldg(reinterpret_cast<const float4*>(g.src) + 2 * k + 1);
    const uint2 h0 = bf16x4(a.x, a.y, a.z, a.w), h1 = bf16x4(b.x, b.y, b.z, b.w);
    reinterpret_cast<uint4*>(g.hi)[k] = make_uint4(h0.x, h0.y, h1.x, h1.y);
    if (g.lo) {
        auto res = [](float v, uint32_t w, bool high) { return v - __uint_as_float(high ? (w & 0xffff0000u) : (w << 16)); };
        const uint2 l0 = bf16x4(res(a.x, h0.x, false), res(a.y, h0.x, true), res(a.z, h0.y, false), res(a.w, h0.y, true));
        const uint2 l1 = bf16x4(res(b.x, h1.x, false), res(b.y, h1.x, true), res(b.z, h1.y, false), res(b.w, h1.y, true));
        reinterpret_cast<uint4*>(g.lo)[k] = make_uint4(l0.x, l0.y, l1.x, l1.y);
    }
}

__global__ void __launch_bounds__(kCastThreads) cast_flat_kernel(FlatCast f) {
    allow_dependents();
    const int64_t n0 = f.seg[0].n8, n1 = n0 + f.seg[1].n8, total = n1 + f.seg[2].n8;
    const int64_t stride = (int64_t)gridDim.x * kCastThreads;
    for (int64_t q = (int64_t)blockIdx.x * kCastThreads + threadIdx.x; q < total; q += 2 * stride) {
#pragma unroll
        for (int u = 0; u < 2; ++u) {
            const int64_t k = q + u * stride;
            if (k >= total) break;
            if (k < n0)
                cast8(f.seg[0], k);
            else if (k < n1)
                cast8(f.seg[1], k - n0);
            else
                cast8(f.seg[2], k - n1);
        }
    }
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

}  // namespace

int launch_cast(const helix_ctx* ctx, const Plan& pl, ScanParams* p, void* stream, bool run) {
    CastDst d;
    d.x = pl.x_copy == 1 ? static_cast<__nv_bfloat16*>(p->cast_x) : nullptr;
    d.xf = pl.x_copy == 2 ? static_cast<float*>(p->cast_x) : nullptr;
    d.b = static_cast<__nv_bfloat16*>(p->cast_b);
    d.c = static_cast<__nv_bfloat16*>(p->cast_c);
    d.bl = static_cast<__nv_bfloat16*>(p->cast_bl);
    d.cl = static_cast<__nv_bfloat16*>(p->cast_cl);
    d.pp = pl.x_pitch;
    // dense x (bf16 copy, pitch = head_dim) or no x copy, dense B and C, all
    // 16-byte aligned: flat copies
    const bool x_dense = p->s_x2 == 1 && d.pp == p->P && p->s_x1 == p->P && p->s_x0 == (int64_t)p->H * p->P &&
                         p->seq_x == (int64_t)p->L * p->H * p->P && aligned16(p->x);
    const bool x_flat = pl.x_copy == 0 || (pl.x_copy == 1 && x_dense);
    const int64_t row_bc = (int64_t)p->G * p->N;
    const bool bc_flat = p->s_b1 == p->N && p->s_b0 == row_bc && p->seq_b == (int64_t)p->L * row_bc &&
                         p->s_c1 == p->N && p->s_c0 == row_bc && p->seq_c == (int64_t)p->L * row_bc &&
                         aligned16(p->B) && aligned16(p->C);
    if (run && x_flat && bc_flat) {
        FlatCast f;
        f.seg[0] = {static_cast<const float*>(p->x), d.x, nullptr,
                    pl.x_copy == 1 ? (int64_t)p->S * p->L * p->H * p->P / 8 : 0};
        f.seg[1] = {static_cast<const float*>(p->B), d.b, d.bl, (int64_t)p->S * p->L * row_bc / 8};
        f.seg[2] = {static_cast<const float*>(p->C), d.c, d.cl, (int64_t)p->S * p->L * row_bc / 8};
        const int64_t groups = f.seg[0].n8 + f.seg[1].n8 + f.seg[2].n8;
        const int64_t want = (groups + 2 * kCastThreads - 1) / (2 * kCastThreads);
        const int64_t cap = (int64_t)(ctx ? ctx->n_sm : 148) * 8;
        const unsigned grid = (unsigned)(want < cap ? (want > 0 ? want : 1) : cap);
        cast_flat_kernel<<<grid, kCastThreads, 0, static_cast<cudaStream_t>(stream)>>>(f);
        const cudaError_t e = cudaGetLastError();
        if (e != cudaSuccess) return e;
    } else if (run) {
        const int64_t quads = (int64_t)p->S * p->L * ((pl.x_copy ? p->H * (d.pp / 4) : 0) + 2 * p->G * (p->N / 4));
        const int64_t want = (quads + kCastThreads - 1) / kCastThreads;
        const int64_t cap = (int64_t)(ctx ? ctx->n_sm : 148) * 8;  // grid-stride beyond 8 CTAs per SM
        const unsigned grid = (unsigned)(want < cap ? (want > 0 ? want : 1) : cap);
        cast_bf16_kernel<<<grid, kCastThreads, 0, static_cast<cudaStream_t>(stream)>>>(*p, d);
        const cudaError_t e = cudaGetLastError();
        if (e != cudaSuccess) return e;
    }
    // the kernels that follow read the dense copies (and the low halves of B
    // and C, with the same strides, from p->cast_bl / cast_cl)
    if (pl.x_copy) {
        p->x = pl.x_copy == 1 ? static_cast<const void*>(d.x) : static_cast<const void*>(d.xf);
        p->s_x0 = (int64_t)p->H * d.pp;
        p->s_x1 = d.pp;
        p->s_x2 = 1;
        p->seq_x = (int64_t)p->L * p->H * d.pp;
    }
    p->B = d.b;
    p->C = d.c;
    p->s_b0 = p->s_c0 = (int64_t)p->G * p->N;
    p->s_b1 = p->s_c1 = p->N;
    p->seq_b = p->seq_c = (int64_t)p->L * p->G * p->N;
    p->io_bf16 = 1;
    return cudaSuccess;
}

}  // namespace hx
