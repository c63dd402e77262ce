// umma.cuh -- thin inline-PTX wrappers for the sm_100a features the
// tensor-core kernels use: mbarriers, TMA tile loads, TMEM allocation,
// tcgen05.mma / commit / ld, and the shared-memory matrix descriptors.
//
// Layout conventions (bf16 operands, 128-byte swizzle):
//   * A "SW128 tile" is a run of rows of exactly 128 bytes (64 bf16), 1024-byte
//     aligned.  Row r sits at r*128; its 16-byte chunk c sits at chunk
//     c ^ (r & 7).  This is the pattern TMA writes with
//     CU_TENSOR_MAP_SWIZZLE_128B and the one tcgen05 reads with layout type
//     SWIZZLE_128B.
//   * K-major operand (rows = M or N index, K contiguous): one SW128 tile per
//     64 K-elements; an MMA step of K=16 advances the start address by 32 B
//     inside the tile; 8-row groups are 1024 B apart (SBO).
//   * MN-major operand (rows = K index, M/N contiguous): one SW128 tile per
//     64 M/N-elements, LBO = distance between those tiles; an MMA step of
//     K=16 advances the start address by 16 rows = 2048 B; 8-row groups are
//     1024 B apart (SBO).
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace hx {
namespace umma {

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---------------------------------------------------------------------------
// mbarrier
// ---------------------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Waits for the phase with parity `parity` to complete, for at most
// `budget` clock cycles.  Returns false when the budget ran out.
// The clock is read once per 32 polls: reading it on every poll doubles
// the wake-up latency of a hand-off between warps.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, long long budget) {
    if (mbar_try_wait(bar, parity)) return true;
    const long long t0 = clock64();
    for (;;) {
#pragma unroll 1
        for (int k = 0; k < 32; ++k)
            if (mbar_try_wait(bar, parity)) return true;
        if (clock64() - t0 > budget) return false;
    }
}

// ---------------------------------------------------------------------------
// TMA: every copy targets this CTA only (no cluster-wide copies anywhere in this library)
// ---------------------------------------------------------------------------
__device__ __forceinline__ void tma_load_4d(void* dst, const CUtensorMap* map, uint64_t* bar, int c0,
                                            int c1, int c2, int c3) {
    asm volatile(
        "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%2, %3, %4, %5}], [%6];" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(smem_u32(bar))
        : "memory");
}

// Shared -> global tile store (bulk async group of the issuing thread).
__device__ __forceinline__ void tma_store_4d(const CUtensorMap* map, const void* src, int c0, int c1, int c2,
                                             int c3) {
    asm volatile(
        "cp.async.bulk.tensor.4d.global.shared::cta.bulk_group [%0, {%2, %3, %4, %5}], [%1];" ::"l"(
            reinterpret_cast<uint64_t>(map)),
        "r"(smem_u32(src)), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
        : "memory");
}
// y += box: the same copy as tma_store_4d with an fp32 add at the destination.
__device__ __forceinline__ void tma_reduce_add_4d(const CUtensorMap* map, const void* src, int c0, int c1, int c2,
                                                  int c3) {
    asm volatile(
        "cp.reduce.async.bulk.tensor.4d.global.shared::cta.add.tile.bulk_group [%0, {%2, %3, %4, %5}], [%1];" ::"l"(
            reinterpret_cast<uint64_t>(map)),
        "r"(smem_u32(src)), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
        : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// Until the issuing thread's bulk stores have finished READING shared memory.
__device__ __forceinline__ void bulk_wait_read0() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
// Until the issuing thread's bulk stores are complete.
__device__ __forceinline__ void bulk_wait0() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

// Plain arrive (count 1) on an mbarrier.
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// Programmatic dependent launch: wait until the grids this one was launched
// behind have completed and their memory is visible (returns at once when it
// was launched normally); allow the grid launched behind this one to start.
__device__ __forceinline__ void grid_dep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void grid_dep_launch() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// Named barrier among `n` threads (id >= 1; id 0 is __syncthreads).
__device__ __forceinline__ void named_sync(uint32_t id, uint32_t n) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n) : "memory");
}
// Named barrier with an AND vote over the participating threads.
__device__ __forceinline__ bool named_and(uint32_t id, uint32_t n, bool v) {
    uint32_t r;
    asm volatile(
        "{\n\t.reg .pred p, q;\n\t"
        "setp.ne.u32 p, %1, 0;\n\t"
        "bar.red.and.pred q, %2, %3, p;\n\t"
        "selp.u32 %0, 1, 0, q;\n\t}"
        : "=r"(r)
        : "r"((uint32_t)v), "r"(id), "r"(n)
        : "memory");
    return r != 0;
}

__device__ __forceinline__ void prefetch_tmap(const CUtensorMap* map) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// Generic-proxy shared-memory writes -> visible to the async proxy (UMMA/TMA).
__device__ __forceinline__ void fence_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ---------------------------------------------------------------------------
// TMEM
// ---------------------------------------------------------------------------
// Whole-warp instructions.
__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
                 "r"(ncols)
                 : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// 32 lanes x 32 bit, 16 consecutive columns per thread.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
    uint32_t r[16];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, "
        "%13, %14, %15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]),
          "=r"(r[15])
        : "r"(taddr));
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}
// Same shape, 8 columns.
__device__ __forceinline__ void tmem_ld8(uint32_t taddr, float (&v)[8]) {
    uint32_t r[8];
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
                 : "r"(taddr));
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = __uint_as_float(r[i]);
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// 32 lanes x 32 bit, 16 consecutive columns per thread (this thread's lane).
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&v)[16]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, "
        "%14, %15, %16};" ::"r"(taddr),
        "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]), "r"(v[9]),
        "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15])
        : "memory");
}
__device__ __forceinline__ void tmem_st8(uint32_t taddr, const uint32_t (&v)[8]) {
    asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"r"(taddr),
                 "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7])
                 : "memory");
}
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// exp2 on the special-function unit (max rel. error ~2^-22 over the whole
// range; inputs below -126 flush to 0).
__device__ __forceinline__ float ex2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// ---------------------------------------------------------------------------
// tcgen05.mma (kind::f16, bf16 x bf16 -> f32 accumulator in TMEM)
// ---------------------------------------------------------------------------
__device__ __forceinline__ void mma_bf16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                         uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// A operand from TMEM (M = 128: row m in lane m, bf16 elements packed two per
// 32-bit column, element 2c in the low half of column c).
__device__ __forceinline__ void mma_bf16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                            uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
        "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// Arrives on `bar` once every previously issued tcgen05 operation of this
// thread has completed.
__device__ __forceinline__ void mma_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                     smem_u32(bar))
                 : "memory");
}

// Instruction descriptor, kind::f16: D f32, A and B bf16, dense.
//   bits [4,6) D format (1 = f32), [7,10) A format (1 = bf16),
//   [10,13) B format (1 = bf16), 15 A major (1 = MN), 16 B major (1 = MN),
//   [17,23) N >> 3, [24,29) M >> 4.
__host__ __device__ constexpr uint32_t idesc_bf16(int M, int N, bool a_mn, bool b_mn) {
    return (1u << 4) | (1u << 7) | (1u << 10) | ((a_mn ? 1u : 0u) << 15) | ((b_mn ? 1u : 0u) << 16) |
           ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

// Shared-memory matrix descriptor, SWIZZLE_128B:
//   [0,14) start >> 4, [16,30) LBO >> 4, [32,46) SBO >> 4, [46,48) version 1,
//   [49,52) base offset 0, [61,64) layout 2 (SWIZZLE_128B).
__device__ __forceinline__ uint64_t sdesc_sw128(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
    uint64_t d = 0;
    d |= (uint64_t)((saddr >> 4) & 0x3FFF);
    d |= (uint64_t)((lbo >> 4) & 0x3FFF) << 16;
    d |= (uint64_t)((sbo >> 4) & 0x3FFF) << 32;
    d |= (uint64_t)1 << 46;
    d |= (uint64_t)2 << 61;
    return d;
}

// Byte offset of 16-byte chunk `c` (0..7) of row `r` inside a SW128 tile.
__device__ __forceinline__ uint32_t sw128_off(uint32_t r, uint32_t c) {
    return r * 128u + (((c ^ (r & 7u)) & 7u) << 4);
}

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
    __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&v);
}

__device__ __forceinline__ void unpack_bf16x2(uint32_t w, float& lo, float& hi) {
    __nv_bfloat162 v = *reinterpret_cast<__nv_bfloat162*>(&w);
    float2 f = __bfloat1622float2(v);
    lo = f.x;
    hi = f.y;
}

// Two fp32 lanes in one 64-bit register pair: sm_100 multiplies or subtracts
// both with one instruction (mul/sub .f32x2).
__device__ __forceinline__ uint64_t f2_of(float lo, float hi) {
    uint64_t d;
    asm("mov.b64 %0, {%1, %2};" : "=l"(d) : "f"(lo), "f"(hi));
    return d;
}
__device__ __forceinline__ void f2_to(uint64_t d, float& lo, float& hi) {
    asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(d));
}
__device__ __forceinline__ uint64_t f2_mul(uint64_t a, uint64_t b) {
    uint64_t d;
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}
__device__ __forceinline__ uint64_t f2_add(uint64_t a, uint64_t b) {
    uint64_t d;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}
__device__ __forceinline__ uint64_t f2_sub(uint64_t a, uint64_t b) {
    uint64_t d;
    asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}
// bf16 pair -> fp32 pair (exact: a bf16 is the top half of its fp32)
__device__ __forceinline__ uint64_t f2_of_bf16x2(uint32_t w) {
    return f2_of(__uint_as_float(w << 16), __uint_as_float(w & 0xffff0000u));
}

// x w for 8 bf16 x and one fp32 w, as bf16 hi = round(x w) and
// lo = round(x w - hi): hi + lo carries x w to about 16 significant bits.
__device__ __forceinline__ void split_xw8(const uint4& x, uint64_t w2, uint4& hi, uint4& lo) {
    const uint32_t in[4] = {x.x, x.y, x.z, x.w};
    uint32_t h[4], l[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
        const uint64_t p = f2_mul(f2_of_bf16x2(in[e]), w2);
        float p0, p1;
        f2_to(p, p0, p1);
        h[e] = pack_bf16x2(p0, p1);
        float l0, l1;
        f2_to(f2_sub(p, f2_of_bf16x2(h[e])), l0, l1);
        l[e] = pack_bf16x2(l0, l1);
    }
    hi = make_uint4(h[0], h[1], h[2], h[3]);
    lo = make_uint4(l[0], l[1], l[2], l[3]);
}

// Same, with x given as a bf16 pair (hi + lo, about 16 significant bits):
// w (xh + xl) split into hi and lo again.
__device__ __forceinline__ void split_xw8_x3(const uint4& xh, const uint4& xl, uint64_t w2, uint4& hi, uint4& lo) {
    const uint32_t a[4] = {xh.x, xh.y, xh.z, xh.w};
    const uint32_t b[4] = {xl.x, xl.y, xl.z, xl.w};
    uint32_t h[4], l[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
        const uint64_t p = f2_mul(f2_add(f2_of_bf16x2(a[e]), f2_of_bf16x2(b[e])), w2);
        float p0, p1;
        f2_to(p, p0, p1);
        h[e] = pack_bf16x2(p0, p1);
        float l0, l1;
        f2_to(f2_sub(p, f2_of_bf16x2(h[e])), l0, l1);
        l[e] = pack_bf16x2(l0, l1);
    }
    hi = make_uint4(h[0], h[1], h[2], h[3]);
    lo = make_uint4(l[0], l[1], l[2], l[3]);
}

// Eight fp32 values (a, b) times w, as bf16 hi = round(v w) and
// lo = round(v w - hi).
__device__ __forceinline__ void split_xw8_f32(const float4& a, const float4& b, uint64_t w2, uint4& hi, uint4& lo) {
    const uint64_t in[4] = {f2_of(a.x, a.y), f2_of(a.z, a.w), f2_of(b.x, b.y), f2_of(b.z, b.w)};
    uint32_t h[4], l[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
        const uint64_t p = f2_mul(in[e], w2);
        float p0, p1;
        f2_to(p, p0, p1);
        h[e] = pack_bf16x2(p0, p1);
        float l0, l1;
        f2_to(f2_sub(p, f2_of_bf16x2(h[e])), l0, l1);
        l[e] = pack_bf16x2(l0, l1);
    }
    hi = make_uint4(h[0], h[1], h[2], h[3]);
    lo = make_uint4(l[0], l[1], l[2], l[3]);
}

// Eight fp32 values as bf16 hi = round(v) and lo = round(v - hi).
__device__ __forceinline__ void split8_f32(const float4& a, const float4& b, uint4& hi, uint4& lo) {
    const uint64_t in[4] = {f2_of(a.x, a.y), f2_of(a.z, a.w), f2_of(b.x, b.y), f2_of(b.z, b.w)};
    uint32_t h[4], l[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
        float v0, v1;
        f2_to(in[e], v0, v1);
        h[e] = pack_bf16x2(v0, v1);
        float l0, l1;
        f2_to(f2_sub(in[e], f2_of_bf16x2(h[e])), l0, l1);
        l[e] = pack_bf16x2(l0, l1);
    }
    hi = make_uint4(h[0], h[1], h[2], h[3]);
    lo = make_uint4(l[0], l[1], l[2], l[3]);
}

}  // namespace umma
}  // namespace hx
