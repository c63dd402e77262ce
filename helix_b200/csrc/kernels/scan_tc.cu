// scan_tc.cu -- tcgen05 kernel family: bf16 operands (x, B, C stored bf16),
// fp32 accumulators in TMEM, fp32 carried state.  compute_dtype BF16 /
// backend MPP (the reference's bf16 path, src/kernels/mpp/helix_scan_mpp.metal,
// which narrows only the GEMM operands and keeps the carry fp32).
//
// Same run decomposition as the fp32 family (runtime/internal.h).  Chunks are
// 128 tokens so every GEMM has M = 128 (one TMEM lane per row):
//
//   G1  D1[t][j] = C[t][:] . B[j][:]            A = C  (K-major, TMA)   B = B  (K-major, TMA)
//   G3  D3[t][p] = C[t][:] . S[:][p]            A = C                   B = S  (MN-major, threads)
//   G4  D4[n][p] = sum_j B[j][n] xw[j][p]       A = B  (MN-major, TMA)  B = xw (MN-major, threads)
//       xw = dt_j exp(Lc_end - Lc_j) x[j][p], split into bf16 hi + lo so the
//       state update keeps ~16 mantissa bits (two MMAs into D4)
//   M'[t][j] = D1[t][j] exp(Lc_t - Lc_j) dt_j for j <= t   (epilogue, bf16, K-major smem)
//   G2  D2[t][p] = M'[t][:] . x[:][p]           A = M' (K-major)        B = x  (MN-major, TMA)
//   y = D2 + exp(Lc_t) D3;   S <- exp(Lc_end) S + D4   (S kept fp32 in registers)
//
// Threads: 256 = two warpgroups; warp w reads TMEM lanes 32*(w%4).., and the
// two warpgroups split the accumulator columns in halves.  Thread 0 issues
// TMA and MMA.  Every mbarrier wait is bounded: on expiry the block agrees
// (vote), records a fault code readable with helix_device_fault(), releases
// its TMEM and returns.
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdlib>

#include "common.cuh"
#include "umma.cuh"

namespace hx {

// Device-side fault word: 0 = none, else the code of the first bounded wait
// that expired (see tc_fault_*).
__device__ unsigned int g_tc_fault = 0;

namespace {

using namespace umma;

constexpr int kTcThreads = 256;
constexpr int kCS = 128;
constexpr long long kWaitBudget = 1ll << 31;  // clock cycles, ~1 s

enum : unsigned { kFaultTmaOut = 1, kFaultMmaOut = 2, kFaultTmaState = 3, kFaultMmaState = 4 };

struct TcMaps {
    CUtensorMap x, b, c;
};

// Output-kernel shared memory (byte offsets from a 1024-aligned base).
constexpr uint32_t OFF_C = 0;         // 2 x 16 KB  C chunk, K tiles n 0-63 / 64-127
constexpr uint32_t OFF_B = 32768;     // 2 x 16 KB  B chunk
constexpr uint32_t OFF_X = 65536;     // 16 KB      x chunk [j][p]
constexpr uint32_t OFF_M = 81920;     // 2 x 16 KB  M' [t][j], K tiles j 0-63 / 64-127
constexpr uint32_t OFF_XH = 114688;   // 16 KB      xw hi [j][p]
constexpr uint32_t OFF_XL = 131072;   // 16 KB      xw lo [j][p]
constexpr uint32_t OFF_S = 147456;    // 16 KB      state bf16 [n][p]
constexpr uint32_t OFF_VEC = 163840;  // dt, Lc, w, e (4 x 128 floats) + warp totals
constexpr uint32_t SMEM_OUT = OFF_VEC + 4 * 512 + 64 + 1024;

// State-kernel shared memory.
constexpr uint32_t SOFF_B = 0;
constexpr uint32_t SOFF_X = 32768;
constexpr uint32_t SOFF_XH = 49152;
constexpr uint32_t SOFF_XL = 65536;
constexpr uint32_t SOFF_VEC = 81920;
constexpr uint32_t SMEM_STATE = SOFF_VEC + 4 * 512 + 64 + 1024;

// TMEM columns.
constexpr uint32_t TM_D1 = 0, TM_D2 = 128, TM_D3 = 192, TM_D4 = 256;

constexpr uint32_t ID_G1 = idesc_bf16(128, 128, false, false);
constexpr uint32_t ID_G2 = idesc_bf16(128, 64, false, true);
constexpr uint32_t ID_G3 = idesc_bf16(128, 64, false, true);
constexpr uint32_t ID_G4 = idesc_bf16(128, 64, true, true);

__device__ __forceinline__ uint8_t* align1024(uint8_t* p) {
    return reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(p) + 1023) & ~uintptr_t(1023));
}

// K-major operand: K step ks (16 elements) of a 2-tile (K = 128) operand.
__device__ __forceinline__ uint64_t desc_kmajor(uint32_t base, int ks) {
    return sdesc_sw128(base + (uint32_t)(ks >> 2) * 16384u + (uint32_t)(ks & 3) * 32u, 16, 1024);
}
// MN-major operand: K step ks = 16 rows of 128 B; M/N tiles 16 KB apart.
__device__ __forceinline__ uint64_t desc_mnmajor(uint32_t base, int ks) {
    return sdesc_sw128(base + (uint32_t)ks * 2048u, 16384, 1024);
}

// Per-chunk scalars: dt (0 past the end), inclusive prefix of A*dt.
__device__ __forceinline__ float chunk_prefix(const ScanParams& p, int64_t db, int t0, int tlen, float Ah,
                                              float* dtv, float* Lc, float* tot, float* v_out) {
    const int tid = threadIdx.x;
    float v = 0.0f;
    if (tid < tlen) v = dt_of(p.dt[db + (int64_t)(t0 + tid) * p.s_dt0], p.dt_min, p.dt_max);
    const float pre = block_prefix(Ah * v, kCS, tot);
    if (tid < kCS) {
        dtv[tid] = v;
        Lc[tid] = pre;
    }
    *v_out = v;
    return pre;
}

// xw = w_j * x[j][p] as bf16 hi and lo tiles (same SW128 layout as x).
__device__ __forceinline__ void build_xw(const uint8_t* sX, uint8_t* sXH, uint8_t* sXL, const float* wv) {
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        const int i = threadIdx.x + kTcThreads * k;
        const int j = i >> 3, c = i & 7;
        const uint32_t off = sw128_off(j, c);
        const uint4 raw = *reinterpret_cast<const uint4*>(sX + off);
        const float w = wv[j];
        const uint32_t in[4] = {raw.x, raw.y, raw.z, raw.w};
        uint32_t hi[4], lo[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            float a, b;
            unpack_bf16x2(in[q], a, b);
            a *= w;
            b *= w;
            const __nv_bfloat16 ah = __float2bfloat16_rn(a), bh = __float2bfloat16_rn(b);
            hi[q] = pack_bf16x2(__bfloat162float(ah), __bfloat162float(bh));
            lo[q] = pack_bf16x2(a - __bfloat162float(ah), b - __bfloat162float(bh));
        }
        *reinterpret_cast<uint4*>(sXH + off) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
        *reinterpret_cast<uint4*>(sXL + off) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
    }
}

// The 32 state values this thread owns (row n, channels 32*wg..+32) -> bf16
// row n of the MN-major state tile.
__device__ __forceinline__ void store_state_bf16(uint8_t* sS, int n, int wg, const float (&S)[32]) {
#pragma unroll
    for (int cc = 0; cc < 4; ++cc) {
        uint32_t w[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) w[q] = pack_bf16x2(S[8 * cc + 2 * q], S[8 * cc + 2 * q + 1]);
        *reinterpret_cast<uint4*>(sS + sw128_off(n, 4 * wg + cc)) = make_uint4(w[0], w[1], w[2], w[3]);
    }
}

// Block-wide agreement on a bounded wait.
__device__ __forceinline__ bool wait_all(uint64_t* bar, uint32_t parity, unsigned code) {
    const bool ok = mbar_wait(bar, parity, kWaitBudget);
    const bool all = __syncthreads_and(ok) != 0;
    if (!all && threadIdx.x == 0) atomicCAS(&g_tc_fault, 0u, code);
    return all;
}

// ---------------------------------------------------------------------------
// Output kernel
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(kTcThreads, 1) tc_out_kernel(const __grid_constant__ TcMaps maps, ScanParams p) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* sm = align1024(smem_raw);
    uint8_t* sC = sm + OFF_C;
    uint8_t* sB = sm + OFF_B;
    uint8_t* sX = sm + OFF_X;
    uint8_t* sM = sm + OFF_M;
    uint8_t* sXH = sm + OFF_XH;
    uint8_t* sXL = sm + OFF_XL;
    uint8_t* sS = sm + OFF_S;
    float* dtv = reinterpret_cast<float*>(sm + OFF_VEC);
    float* Lc = dtv + kCS;
    float* wv = Lc + kCS;
    float* ev = wv + kCS;
    float* tot = ev + kCS;
    __shared__ uint64_t bar_tma, bar_mma;
    __shared__ uint32_t tmem_base;

    const int tid = threadIdx.x, warp = tid >> 5;
    const int wg = warp >> 2;                    // column half
    const int row = 32 * (warp & 3) + (tid & 31);  // TMEM lane / tile row
    const uint32_t lane_off = (uint32_t)(32 * (warp & 3)) << 16;

    const Tile tl = decode_tile(blockIdx.x, p.n_pslab, p.H, p.n_runs);
    const int p0 = tl.slab * kSlab, pw = min(kSlab, p.P - p0);
    const int g = tl.h / p.hpg;
    const float Ah = p.A[(int64_t)tl.h * p.s_a];
    const int t_begin = tl.run * p.run_tok;
    const int t_end = min(p.L, t_begin + p.run_tok);
    const int64_t db = (int64_t)tl.seq * p.seq_dt + (int64_t)tl.h * p.s_dt1;

    if (tid == 0) {
        mbar_init(&bar_tma, 1);
        mbar_init(&bar_mma, 1);
        fence_mbar_init();
        prefetch_tmap(&maps.x);
        prefetch_tmap(&maps.b);
        prefetch_tmap(&maps.c);
    }
    if (warp == 0) {
        tmem_alloc(&tmem_base, 512);
        tmem_relinquish();
    }

    // ---- state entering this run: thread (wg, row = n) owns S[n][32wg..] --
    float S[32];
    {
        const int src = p.has_ids ? p.ids[tl.seq] : tl.seq;
        const float* s0 = p.s0 + (int64_t)src * p.seq_s + (int64_t)tl.h * p.s_s0 + row;
#pragma unroll
        for (int i = 0; i < 32; ++i) {
            const int c = 32 * wg + i;
            S[i] = c < pw ? s0[(int64_t)(p0 + c) * p.s_s1] : 0.0f;
        }
        const int64_t unit0 = ((int64_t)tl.seq * p.H + tl.h) * p.n_runs;
        for (int r = 0; r < tl.run; ++r) {
            const float a = expf(p.lam[unit0 + r]);
            const float* ag = p.agg + (unit0 + r) * (int64_t)p.P * p.N + (int64_t)p0 * p.N + row;
#pragma unroll
            for (int i = 0; i < 32; ++i) {
                const int c = 32 * wg + i;
                if (c < pw) S[i] = fmaf(a, S[i], ag[(int64_t)c * p.N]);
            }
        }
        store_state_bf16(sS, row, wg, S);
    }
    __syncthreads();
    tc_fence_after();
    const uint32_t tm = tmem_base;
    const uint32_t aC = smem_u32(sC), aB = smem_u32(sB), aX = smem_u32(sX), aM = smem_u32(sM);
    const uint32_t aXH = smem_u32(sXH), aXL = smem_u32(sXL), aS = smem_u32(sS);

    uint32_t ph_tma = 0, ph_mma = 0;
    bool ok = true;
    for (int t0 = t_begin; t0 < t_end && ok; t0 += kCS) {
        const int tlen = min(kCS, t_end - t0);
        if (tid == 0) {
            mbar_expect_tx(&bar_tma, 5 * 16384);
            tma_load_4d(sC, &maps.c, &bar_tma, 0, g, t0, tl.seq);
            tma_load_4d(sC + 16384, &maps.c, &bar_tma, 64, g, t0, tl.seq);
            tma_load_4d(sB, &maps.b, &bar_tma, 0, g, t0, tl.seq);
            tma_load_4d(sB + 16384, &maps.b, &bar_tma, 64, g, t0, tl.seq);
            tma_load_4d(sX, &maps.x, &bar_tma, p0, tl.h, t0, tl.seq);
        }
        float v;
        const float pre = chunk_prefix(p, db, t0, tlen, Ah, dtv, Lc, tot, &v);
        __syncthreads();
        const float Lend = Lc[kCS - 1];
        if (tid < kCS) {
            wv[tid] = v * __expf(Lend - pre);
            ev[tid] = __expf(pre);
        }
        const float decay = __expf(Lend);
        if (!(ok = wait_all(&bar_tma, ph_tma, kFaultTmaOut))) break;
        ph_tma ^= 1;

        build_xw(sX, sXH, sXL, wv);
        fence_async_smem();
        tc_fence_before();
        __syncthreads();
        if (tid == 0) {
            tc_fence_after();
#pragma unroll
            for (int ks = 0; ks < 8; ++ks)
                mma_bf16(tm + TM_D1, desc_kmajor(aC, ks), desc_kmajor(aB, ks), ID_G1, ks > 0);
#pragma unroll
            for (int ks = 0; ks < 8; ++ks)
                mma_bf16(tm + TM_D3, desc_kmajor(aC, ks), desc_mnmajor(aS, ks), ID_G3, ks > 0);
#pragma unroll
            for (int ks = 0; ks < 8; ++ks)
                mma_bf16(tm + TM_D4, desc_mnmajor(aB, ks), desc_mnmajor(aXH, ks), ID_G4, ks > 0);
#pragma unroll
            for (int ks = 0; ks < 8; ++ks)
                mma_bf16(tm + TM_D4, desc_mnmajor(aB, ks), desc_mnmajor(aXL, ks), ID_G4, 1);
            mma_commit(&bar_mma);
        }
        if (!(ok = wait_all(&bar_mma, ph_mma, kFaultMmaOut))) break;
        ph_mma ^= 1;
        tc_fence_after();

        // ---- epilogue 1: M' (row t, columns j of this half) -> bf16 smem --
        {
            const float Lt = Lc[row];
#pragma unroll
            for (int cb = 0; cb < 4; ++cb) {
                float d[16];
                tmem_ld16(tm + lane_off + TM_D1 + 64 * wg + 16 * cb, d);
                tmem_wait_ld();
                uint32_t w[8];
#pragma unroll
                for (int e = 0; e < 16; e += 2) {
                    const int j0 = 64 * wg + 16 * cb + e;
                    const float m0 = j0 <= row ? d[e] * __expf(Lt - Lc[j0]) * dtv[j0] : 0.0f;
                    const float m1 = j0 + 1 <= row ? d[e + 1] * __expf(Lt - Lc[j0 + 1]) * dtv[j0 + 1] : 0.0f;
                    w[e >> 1] = pack_bf16x2(m0, m1);
                }
                uint8_t* tile = sM + 16384 * wg;
                *reinterpret_cast<uint4*>(tile + sw128_off(row, 2 * cb)) = make_uint4(w[0], w[1], w[2], w[3]);
                *reinterpret_cast<uint4*>(tile + sw128_off(row, 2 * cb + 1)) = make_uint4(w[4], w[5], w[6], w[7]);
            }
        }
        // ---- carry: S <- exp(Lend) S + D4 (row n, channels of this half) --
#pragma unroll
        for (int cb = 0; cb < 2; ++cb) {
            float d[16];
            tmem_ld16(tm + lane_off + TM_D4 + 32 * wg + 16 * cb, d);
            tmem_wait_ld();
#pragma unroll
            for (int e = 0; e < 16; ++e) S[16 * cb + e] = fmaf(decay, S[16 * cb + e], d[e]);
        }
        store_state_bf16(sS, row, wg, S);
        fence_async_smem();
        tc_fence_before();
        __syncthreads();
        if (tid == 0) {
            tc_fence_after();
#pragma unroll
            for (int ks = 0; ks < 8; ++ks)
                mma_bf16(tm + TM_D2, desc_kmajor(aM, ks), desc_mnmajor(aX, ks), ID_G2, ks > 0);
            mma_commit(&bar_mma);
        }
        if (!(ok = wait_all(&bar_mma, ph_mma, kFaultMmaOut))) break;
        ph_mma ^= 1;
        tc_fence_after();

        // ---- epilogue 2: y = D2 + exp(Lc_t) D3 ----------------------------
        {
            const float e = ev[row];
            float* yr = p.y + (int64_t)tl.seq * p.seq_y + (int64_t)(t0 + row) * p.s_y0 + (int64_t)tl.h * p.s_y1 +
                        (int64_t)(p0 + 32 * wg) * p.s_y2;
            const bool vec = p.s_y2 == 1 && pw == kSlab && (reinterpret_cast<uintptr_t>(yr) & 15) == 0;
#pragma unroll
            for (int cb = 0; cb < 2; ++cb) {
                float a[16], b[16];
                tmem_ld16(tm + lane_off + TM_D2 + 32 * wg + 16 * cb, a);
                tmem_ld16(tm + lane_off + TM_D3 + 32 * wg + 16 * cb, b);
                tmem_wait_ld();
                if (row < tlen) {
                    if (vec) {
#pragma unroll
                        for (int q = 0; q < 4; ++q)
                            reinterpret_cast<float4*>(yr + 16 * cb)[q] =
                                make_float4(fmaf(e, b[4 * q], a[4 * q]), fmaf(e, b[4 * q + 1], a[4 * q + 1]),
                                            fmaf(e, b[4 * q + 2], a[4 * q + 2]), fmaf(e, b[4 * q + 3], a[4 * q + 3]));
                    } else {
#pragma unroll
                        for (int q = 0; q < 16; ++q) {
                            const int c = 32 * wg + 16 * cb + q;
                            if (c < pw) yr[(int64_t)(16 * cb + q) * p.s_y2] = fmaf(e, b[q], a[q]);
                        }
                    }
                }
            }
        }
        tc_fence_before();
        __syncthreads();
    }

    if (ok && tl.run == p.n_runs - 1) {
        float* s1 = p.s1 + (int64_t)tl.seq * p.seq_s + (int64_t)tl.h * p.s_s0 + row;
#pragma unroll
        for (int i = 0; i < 32; ++i) {
            const int c = 32 * wg + i;
            if (c < pw) s1[(int64_t)(p0 + c) * p.s_s1] = S[i];
        }
    }
    if (!ok) {
        // An expired wait: give in-flight async work one more bounded chance
        // to land before the TMEM it targets is released.
        mbar_wait(&bar_mma, ph_mma, kWaitBudget);
        mbar_wait(&bar_tma, ph_tma, kWaitBudget);
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) tmem_dealloc(tm, 512);
}

// ---------------------------------------------------------------------------
// State kernel: run contribution from a zero start (G4 accumulated over the
// whole run in one TMEM accumulator) and the run log-decay.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(kTcThreads, 1) tc_state_kernel(const __grid_constant__ TcMaps maps, ScanParams p,
                                                                 int runs_in_grid) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* sm = align1024(smem_raw);
    uint8_t* sB = sm + SOFF_B;
    uint8_t* sX = sm + SOFF_X;
    uint8_t* sXH = sm + SOFF_XH;
    uint8_t* sXL = sm + SOFF_XL;
    float* dtv = reinterpret_cast<float*>(sm + SOFF_VEC);
    float* Lc = dtv + kCS;
    float* wv = Lc + kCS;
    float* tot = wv + 2 * kCS;
    __shared__ uint64_t bar_tma, bar_mma;
    __shared__ uint32_t tmem_base;

    const int tid = threadIdx.x, warp = tid >> 5;
    const int wg = warp >> 2;
    const int row = 32 * (warp & 3) + (tid & 31);
    const uint32_t lane_off = (uint32_t)(32 * (warp & 3)) << 16;

    const Tile tl = decode_tile(blockIdx.x, p.n_pslab, p.H, runs_in_grid);
    const int p0 = tl.slab * kSlab, pw = min(kSlab, p.P - p0);
    const int g = tl.h / p.hpg;
    const float Ah = p.A[(int64_t)tl.h * p.s_a];
    const int t_begin = tl.run * p.run_tok;
    const int t_end = min(p.L, t_begin + p.run_tok);
    const int n_chunks = (t_end - t_begin + kCS - 1) / kCS;
    const int64_t db = (int64_t)tl.seq * p.seq_dt + (int64_t)tl.h * p.s_dt1;

    if (tid == 0) {
        mbar_init(&bar_tma, 1);
        mbar_init(&bar_mma, 1);
        fence_mbar_init();
        prefetch_tmap(&maps.x);
        prefetch_tmap(&maps.b);
    }
    if (warp == 0) {
        tmem_alloc(&tmem_base, 64);
        tmem_relinquish();
    }
    __syncthreads();
    tc_fence_after();
    const uint32_t tm = tmem_base;
    const uint32_t aB = smem_u32(sB), aXH = smem_u32(sXH), aXL = smem_u32(sXL);

    uint32_t ph_tma = 0, ph_mma = 0;
    bool ok = true;
    float later = 0.0f;  // sum of A*dt over the chunks after the current one
    for (int ci = n_chunks - 1; ci >= 0; --ci) {
        const int t0 = t_begin + ci * kCS;
        const int tlen = min(kCS, t_end - t0);
        if (tid == 0) {
            mbar_expect_tx(&bar_tma, 3 * 16384);
            tma_load_4d(sB, &maps.b, &bar_tma, 0, g, t0, tl.seq);
            tma_load_4d(sB + 16384, &maps.b, &bar_tma, 64, g, t0, tl.seq);
            tma_load_4d(sX, &maps.x, &bar_tma, p0, tl.h, t0, tl.seq);
        }
        float v;
        const float pre = chunk_prefix(p, db, t0, tlen, Ah, dtv, Lc, tot, &v);
        __syncthreads();
        const float Lend = Lc[kCS - 1];
        if (tid < kCS) wv[tid] = v * __expf(later + (Lend - pre));
        later += Lend;
        if (!(ok = wait_all(&bar_tma, ph_tma, kFaultTmaState))) break;
        ph_tma ^= 1;
        build_xw(sX, sXH, sXL, wv);
        fence_async_smem();
        tc_fence_before();
        __syncthreads();
        if (tid == 0) {
            tc_fence_after();
            const bool first = ci == n_chunks - 1;
#pragma unroll
            for (int ks = 0; ks < 8; ++ks)
                mma_bf16(tm, desc_mnmajor(aB, ks), desc_mnmajor(aXH, ks), ID_G4, (!first || ks > 0) ? 1u : 0u);
#pragma unroll
            for (int ks = 0; ks < 8; ++ks) mma_bf16(tm, desc_mnmajor(aB, ks), desc_mnmajor(aXL, ks), ID_G4, 1u);
            mma_commit(&bar_mma);
        }
        if (!(ok = wait_all(&bar_mma, ph_mma, kFaultMmaState))) break;
        ph_mma ^= 1;
    }
    tc_fence_after();
    if (ok) {
        const int64_t unit = ((int64_t)tl.seq * p.H + tl.h) * p.n_runs + tl.run;
        if (tl.slab == 0 && tid == 0) p.lam[unit] = later;
        float* out = p.agg + unit * (int64_t)p.P * p.N + (int64_t)p0 * p.N + row;
#pragma unroll
        for (int cb = 0; cb < 2; ++cb) {
            float d[16];
            tmem_ld16(tm + lane_off + 32 * wg + 16 * cb, d);
            tmem_wait_ld();
#pragma unroll
            for (int e = 0; e < 16; ++e) {
                const int c = 32 * wg + 16 * cb + e;
                if (c < pw) out[(int64_t)c * p.N] = d[e];
            }
        }
    } else {
        mbar_wait(&bar_mma, ph_mma, kWaitBudget);
        mbar_wait(&bar_tma, ph_tma, kWaitBudget);
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) tmem_dealloc(tm, 64);
}

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------
using EncodeFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                              const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                              CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

// 4-D bf16 map (inner, d1, tok, seq) with a 64 x 1 x 128 x 1 box, 128-byte
// swizzle.  Coordinates past the extents read as zero.
bool make_map(EncodeFn fn, CUtensorMap* m, const void* base, int64_t inner, int64_t d1, int64_t tok, int64_t seq,
              int64_t s1, int64_t s_tok, int64_t s_seq) {
    cuuint64_t dims[4] = {(cuuint64_t)inner, (cuuint64_t)d1, (cuuint64_t)tok, (cuuint64_t)seq};
    cuuint64_t strides[3] = {(cuuint64_t)(s1 * 2), (cuuint64_t)(s_tok * 2), (cuuint64_t)(s_seq * 2)};
    cuuint32_t box[4] = {64, 1, (cuuint32_t)kCS, 1};
    cuuint32_t es[4] = {1, 1, 1, 1};
    return fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(base), dims, strides, box, es,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace

int configure_tc(const helix_ctx*) {
    cudaError_t e = cudaFuncSetAttribute(tc_out_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)SMEM_OUT);
    if (e != cudaSuccess) return e;
    return cudaFuncSetAttribute(tc_state_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)SMEM_STATE);
}

int launch_tc(const helix_ctx* ctx, const Plan& pl, const ScanParams& p, void* stream) {
    auto fn = reinterpret_cast<EncodeFn>(ctx->encode_tiled);
    if (!fn) return cudaErrorNotSupported;
    TcMaps maps;
    const int64_t S = p.S;
    // A sequence extent of 1 makes every sequence's token range its own
    // bounded box, so rows past L read as zero; the sequence coordinate then
    // moves through the seq stride.
    if (!make_map(fn, &maps.x, p.x, p.P, p.H, p.L, S, p.s_x1, p.s_x0, p.seq_x) ||
        !make_map(fn, &maps.b, p.B, p.N, p.G, p.L, S, p.s_b1, p.s_b0, p.seq_b) ||
        !make_map(fn, &maps.c, p.C, p.N, p.G, p.L, S, p.s_c1, p.s_c0, p.seq_c))
        return cudaErrorInvalidValue;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const char* only = std::getenv("HELIX_ONLY_PASS");
    const bool do_a = !only || *only == 'A';
    const bool do_c = !only || *only == 'C';
    const int64_t per_run = (int64_t)p.n_pslab * p.H * S;
    if (pl.need_state_kernel && do_a) {
        const int runs = pl.n_runs - 1;
        tc_state_kernel<<<(unsigned)(per_run * runs), kTcThreads, SMEM_STATE, st>>>(maps, p, runs);
        const cudaError_t e = cudaGetLastError();
        if (e != cudaSuccess) return e;
    }
    if (do_c) {
        tc_out_kernel<<<(unsigned)(per_run * pl.n_runs), kTcThreads, SMEM_OUT, st>>>(maps, p);
        const cudaError_t e = cudaGetLastError();
        if (e != cudaSuccess) return e;
    }
    return cudaSuccess;
}

int read_tc_fault(unsigned* code) {
    unsigned v = 0, zero = 0;
    cudaError_t e = cudaMemcpyFromSymbol(&v, g_tc_fault, sizeof(v));
    if (e != cudaSuccess) return e;
    e = cudaMemcpyToSymbol(g_tc_fault, &zero, sizeof(zero));
    *code = v;
    return e;
}

}  // namespace hx
