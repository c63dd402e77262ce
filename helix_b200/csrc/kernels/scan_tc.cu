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
#include <cstring>

#include "common.cuh"
#include "umma.cuh"

// Phase markers for cycle attribution.  They expand to nothing in the
// library; a profiling build that defines HX_PHASE_PROFILE provides
// hx_phase_cycles[] and accumulates thread 0's SM cycles between markers.
#ifdef HX_PHASE_PROFILE
extern __device__ unsigned long long hx_phase_cycles[32];
#define HX_PHASE_START long long hx_phase_t = clock64()
#define HX_PHASE(k) HX_PHASE_T(k, 0)
#define HX_PHASE_T(k, who)                                            \
    do {                                                              \
        if (threadIdx.x == (who)) {                                   \
            const long long now_ = clock64();                         \
            atomicAdd(&hx_phase_cycles[k], (unsigned long long)(now_ - hx_phase_t)); \
            hx_phase_t = now_;                                        \
        }                                                             \
    } while (0)
#else
#define HX_PHASE_START do {} while (0)
#define HX_PHASE(k) do {} while (0)
#define HX_PHASE_T(k, who) do {} while (0)
#endif

namespace hx {

// Device-side fault word: 0 = none, else the code of the first bounded wait
// that expired (see tc_fault_*).
__device__ unsigned int g_tc_fault = 0;

namespace {

using namespace umma;

constexpr int kCS = 128;
constexpr long long kWaitBudget = 1ll << 31;  // clock cycles, ~1 s

enum : unsigned { kFaultTmaOut = 1, kFaultMmaOut = 2, kFaultTmaState = 3, kFaultMmaState = 4 };

struct TcMaps {
    CUtensorMap x, b, c;
};

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

// ---------------------------------------------------------------------------
// Output kernel: warp-specialised pipeline over the run's chunks.
//
//   warp 16 (lane 0)  TMA producer and MMA issuer
//   warps 0-15        epilogue: four warpgroups; warp w reads TMEM lanes
//                     32*(w%4).. (row = token or state index), warpgroup
//                     k = w/4 owns a quarter of every accumulator's columns
//
// Per chunk i the epilogue runs
//   B  xw(i) hi/lo                          -> arrive xw_ready
//   D  y(i-1) = D2 + e^Lc D3, TMA store     -> arrive d_free     (after g2(i-1))
//   E  dt prefix of chunk i+1
//   F  M'(i) from D1, carry S += D4         -> arrive m_ready    (after acc1(i))
//   H  S_{i+1} -> bf16 smem                                      (after g3(i))
// and the MMA warp runs
//   G1(i), G4(i)  -> commit acc1            (after C/B(i), x(i), xw_ready(i))
//   G3(i)         -> commit g3              (after d_free(i-1)); x(i+1) TMA
//   C/B(i+1) TMA                            (after g3(i): G1/G3/G4 done reading)
//   G2(i)         -> commit g2              (after m_ready(i))
// C and B are single-buffered (reloaded as soon as G3 retires), x is
// double-buffered, xw, M', the state tile and the y staging tiles each have
// their own buffer, so the only cross-chunk waits are the data dependences.
//
// The state entering the run comes from s0 (run 0) or from the carry
// kernel's run-entry states (run r > 0, scratch slot r - 1).
//
// Decay factors of M': exp(Lc_t - Lc_j) = exp(Lc_t - Lc_g) exp(Lc_g - Lc_j)
// with g the first token of j's 8-token group; the second factor (times dt_j)
// is a per-chunk vector, so each thread needs one exp per 8 columns.  When a
// group spans more than 20 nats of decay (where the split could lose a
// factor to underflow) the chunk takes the direct per-element exp.
// ---------------------------------------------------------------------------
constexpr uint32_t OO_C = 0;              // 32 KB  C chunk (2 K tiles)
constexpr uint32_t OO_B = 32768;          // 32 KB  B chunk
constexpr uint32_t OO_X = 65536;          // 2 x 16 KB  x chunks
constexpr uint32_t OO_XW = 98304;         // 32 KB  xw hi | lo
constexpr uint32_t OO_M = 131072;         // 32 KB  M' (2 K tiles)
constexpr uint32_t OO_S = 163840;         // 16 KB  state bf16 [n][p]
constexpr uint32_t OO_Y = 180224;         // 32 KB  y staging, 2 x [128][32] f32 SW128
constexpr uint32_t OO_V = 212992;         // 2 x per-chunk vectors (dt, Lc2, w, e, f) + scratch
constexpr int kVecStride = 5 * 128 + 16;  // floats per chunk parity
constexpr uint32_t SMEM_OUT = OO_V + (2 * kVecStride + 64) * 4 + 1024;
constexpr int kOutThreads = 544;
constexpr int kEpi = 512;                 // epilogue threads (named barrier 1)
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kSpanMax2 = 20.0f * kLog2e;  // largest 8-token decay span for the split

struct OutBars {
    uint64_t cb, x[2], xw_ready, acc1, d_free, g3, m_ready, g2;
};

__device__ __forceinline__ void epi_sync() { named_sync(1, kEpi); }
__device__ __forceinline__ bool epi_wait(uint64_t* bar, uint32_t parity, unsigned code) {
    const bool ok = mbar_wait(bar, parity, kWaitBudget);
    const bool all = named_and(1, kEpi, ok);
    if (!all && threadIdx.x == 0) atomicCAS(&g_tc_fault, 0u, code);
    return all;
}
// One arrival per epilogue warp on a count-16 barrier.
__device__ __forceinline__ void epi_arrive(uint64_t* bar) {
    __syncwarp();
    if ((threadIdx.x & 31) == 0) mbar_arrive(bar);
}

// Inclusive prefix over the first 128 threads (named barrier 1, all 512 call it).
__device__ __forceinline__ float epi_prefix(float v, float* tot) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const float u = __shfl_up_sync(0xffffffffu, v, o);
        if (lane >= o) v += u;
    }
    if (lane == 31 && warp < 4) tot[warp] = v;
    epi_sync();
    float add = 0.0f;
    for (int w = 0; w < warp && w < 4; ++w) add += tot[w];
    return v + add;
}

// bf16 state row n, channels 16*wg .. +16 -> 2 chunks of the MN-major state tile.
__device__ __forceinline__ void store_state16(uint8_t* sS, int n, int wg, const float (&S)[16]) {
#pragma unroll
    for (int cc = 0; cc < 2; ++cc)
        *reinterpret_cast<uint4*>(sS + sw128_off(n, 2 * wg + cc)) =
            make_uint4(pack_bf16x2(S[8 * cc + 0], S[8 * cc + 1]), pack_bf16x2(S[8 * cc + 2], S[8 * cc + 3]),
                       pack_bf16x2(S[8 * cc + 4], S[8 * cc + 5]), pack_bf16x2(S[8 * cc + 6], S[8 * cc + 7]));
}

// xw = w_j x[j][p] as bf16 hi + lo tiles; 512 threads, 2 chunks each.
__device__ __forceinline__ void build_xw512(const uint8_t* sX, uint8_t* sXH, uint8_t* sXL, const float* wv) {
#pragma unroll
    for (int k = 0; k < 2; ++k) {
        const int i = threadIdx.x + kEpi * k;
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
            hi[q] = pack_bf16x2(a, b);
            float ah, bh;
            unpack_bf16x2(hi[q], ah, bh);
            lo[q] = pack_bf16x2(a - ah, b - bh);
        }
        *reinterpret_cast<uint4*>(sXH + off) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
        *reinterpret_cast<uint4*>(sXL + off) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
    }
}

__global__ void __launch_bounds__(kOutThreads, 1)
    tc_out_kernel(const __grid_constant__ TcMaps maps, const __grid_constant__ CUtensorMap ymap, ScanParams p,
                  int y_tma) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* sm = align1024(smem_raw);
    float* vec = reinterpret_cast<float*>(sm + OO_V);
    float* scr = vec + 2 * kVecStride;  // 64 floats: warp totals, Lend
    __shared__ OutBars bars;
    __shared__ uint32_t tmem_base;

    HX_PHASE_START;
    const int tid = threadIdx.x, warp = tid >> 5;
    const bool is_mma = warp == 16;
    const int wg = (warp >> 2) & 3;
    const int row = 32 * (warp & 3) + (tid & 31);
    const uint32_t lane_off = (uint32_t)(32 * (warp & 3)) << 16;

    const Tile tl = decode_tile(blockIdx.x, p.n_pslab, p.H, p.n_runs);
    const int p0 = tl.slab * kSlab, pw = min(kSlab, p.P - p0);
    const int g = tl.h / p.hpg;
    const float Ah = p.A[(int64_t)tl.h * p.s_a];
    const int t_begin = tl.run * p.run_tok;
    const int t_end = min(p.L, t_begin + p.run_tok);
    const int n_ch = (t_end - t_begin + kCS - 1) / kCS;
    const int64_t db = (int64_t)tl.seq * p.seq_dt + (int64_t)tl.h * p.s_dt1;
    const int64_t unit0 = ((int64_t)tl.seq * p.H + tl.h) * p.n_runs;

    uint8_t* sC = sm + OO_C;
    uint8_t* sB = sm + OO_B;
    uint8_t* sXW = sm + OO_XW;
    uint8_t* sM = sm + OO_M;
    uint8_t* sS = sm + OO_S;
    uint8_t* sY = sm + OO_Y;
    auto sX = [&](int i) { return sm + OO_X + (uint32_t)(i & 1) * 16384u; };
    // per chunk: [0] dt, [128] Lc*log2e, [256] w, [384] e^Lc, [512] f*dt, [640] flags
    auto vecs = [&](int i) { return vec + (i & 1) * kVecStride; };

    if (tid == 0) {
        mbar_init(&bars.cb, 1);
        mbar_init(&bars.x[0], 1);
        mbar_init(&bars.x[1], 1);
        mbar_init(&bars.xw_ready, kEpi / 32);
        mbar_init(&bars.acc1, 1);
        mbar_init(&bars.d_free, kEpi / 32);
        mbar_init(&bars.g3, 1);
        mbar_init(&bars.m_ready, kEpi / 32);
        mbar_init(&bars.g2, 1);
        fence_mbar_init();
    }
    if (is_mma) {
        tmem_alloc(&tmem_base, 512);
        tmem_relinquish();
    }
    __syncthreads();
    tc_fence_after();
    const uint32_t tm = tmem_base;

    auto load_cb = [&](int i) {
        const int t0 = t_begin + i * kCS;
        mbar_expect_tx(&bars.cb, 4 * 16384);
        tma_load_4d(sC, &maps.c, &bars.cb, 0, g, t0, tl.seq);
        tma_load_4d(sC + 16384, &maps.c, &bars.cb, 64, g, t0, tl.seq);
        tma_load_4d(sB, &maps.b, &bars.cb, 0, g, t0, tl.seq);
        tma_load_4d(sB + 16384, &maps.b, &bars.cb, 64, g, t0, tl.seq);
    };
    auto load_x = [&](int i) {
        mbar_expect_tx(&bars.x[i & 1], 16384);
        tma_load_4d(sX(i), &maps.x, &bars.x[i & 1], p0, tl.h, t_begin + i * kCS, tl.seq);
    };

    bool ok = true;
    if (is_mma) {
        // ================= TMA producer + MMA issuer (one thread) ==========
        if ((tid & 31) == 0) {
            prefetch_tmap(&maps.x);
            prefetch_tmap(&maps.b);
            prefetch_tmap(&maps.c);
            load_cb(0);
            load_x(0);
            if (n_ch > 1) load_x(1);
            const uint32_t aC = smem_u32(sC), aB = smem_u32(sB), aXH = smem_u32(sXW), aXL = aXH + 16384;
            const uint32_t aM = smem_u32(sM), aS = smem_u32(sS);
            for (int i = 0; i < n_ch && ok; ++i) {
                const uint32_t par = (uint32_t)(i & 1);
                if (!(ok = mbar_wait(&bars.cb, par, kWaitBudget))) break;
                if (!(ok = mbar_wait(&bars.x[i & 1], (uint32_t)((i >> 1) & 1), kWaitBudget))) break;
                if (!(ok = mbar_wait(&bars.xw_ready, par, kWaitBudget))) break;
                tc_fence_after();
#pragma unroll
                for (int ks = 0; ks < 8; ++ks)
                    mma_bf16(tm + TM_D1, desc_kmajor(aC, ks), desc_kmajor(aB, ks), ID_G1, ks > 0);
#pragma unroll
                for (int ks = 0; ks < 8; ++ks)
                    mma_bf16(tm + TM_D4, desc_mnmajor(aB, ks), desc_mnmajor(aXH, ks), ID_G4, ks > 0);
#pragma unroll
                for (int ks = 0; ks < 8; ++ks)
                    mma_bf16(tm + TM_D4, desc_mnmajor(aB, ks), desc_mnmajor(aXL, ks), ID_G4, 1);
                mma_commit(&bars.acc1);
                if (i > 0) {
                    if (!(ok = mbar_wait(&bars.d_free, par ^ 1u, kWaitBudget))) break;
                    tc_fence_after();
                    if (i + 1 < n_ch) load_x(i + 1);  // its buffer held x(i-1); G2(i-1) is done
                }
#pragma unroll
                for (int ks = 0; ks < 8; ++ks)
                    mma_bf16(tm + TM_D3, desc_kmajor(aC, ks), desc_mnmajor(aS, ks), ID_G3, ks > 0);
                mma_commit(&bars.g3);
                if (!(ok = mbar_wait(&bars.g3, par, kWaitBudget))) break;
                if (i + 1 < n_ch) load_cb(i + 1);  // G1, G3, G4 of chunk i are done with C and B
                if (!(ok = mbar_wait(&bars.m_ready, par, kWaitBudget))) break;
                tc_fence_after();
                const uint32_t aX = smem_u32(sX(i));
#pragma unroll
                for (int ks = 0; ks < 8; ++ks)
                    mma_bf16(tm + TM_D2, desc_kmajor(aM, ks), desc_mnmajor(aX, ks), ID_G2, ks > 0);
                mma_commit(&bars.g2);
            }
            if (!ok) {
                atomicCAS(&g_tc_fault, 0u, kFaultMmaOut);
                // let committed work land before the memory it targets goes away
                mbar_wait(&bars.g2, 0, kWaitBudget);
                mbar_wait(&bars.cb, 0, kWaitBudget);
            }
        }
        __syncwarp();
    } else {
        // ================= epilogue warpgroups ============================
        float S[16];
        {
            // run 0 starts from s0 (through ids); later runs from the carry
            // kernel's run-entry state in scratch slot run - 1
            const float* src;
            int64_t sc;
            if (tl.run == 0) {
                const int s = p.has_ids ? p.ids[tl.seq] : tl.seq;
                src = p.s0 + (int64_t)s * p.seq_s + (int64_t)tl.h * p.s_s0 + (int64_t)p0 * p.s_s1 + row;
                sc = p.s_s1;
            } else {
                src = p.agg + (unit0 + tl.run - 1) * (int64_t)p.P * p.N + (int64_t)p0 * p.N + row;
                sc = p.N;
            }
#pragma unroll
            for (int k = 0; k < 16; ++k) {
                const int c = 16 * wg + k;
                S[k] = c < pw ? src[(int64_t)c * sc] : 0.0f;
            }
            store_state16(sS, row, wg, S);
        }

        auto raw_dt = [&](int i) {
            const int t = t_begin + i * kCS + tid;
            return (i < n_ch && tid < kCS && t < t_end) ? p.dt[db + (int64_t)t * p.s_dt0] : 0.0f;
        };
        auto prefix = [&](int i, float raw) {
            const int tlen = min(kCS, t_end - (t_begin + i * kCS));
            float* v4 = vecs(i);
            const float v = tid < tlen ? dt_of(raw, p.dt_min, p.dt_max) : 0.0f;
            const float pre = epi_prefix(Ah * v, scr) * kLog2e;
            if (tid < kCS) v4[128 + tid] = pre;
            epi_sync();
            const float Lend = v4[128 + kCS - 1];
            bool span_ok = true;
            if (tid < kCS) {
                const float Lg = v4[128 + (tid & ~7)];
                v4[tid] = v;
                v4[256 + tid] = v * ex2(Lend - pre);
                v4[384 + tid] = ex2(pre);
                v4[512 + tid] = ex2(Lg - pre) * v;
                span_ok = Lg - pre <= kSpanMax2;
            }
            const bool all_ok = named_and(1, kEpi, span_ok);
            if (tid == 0) v4[640] = all_ok ? 1.0f : 0.0f;
        };
        float dt_next = raw_dt(1);
        prefix(0, raw_dt(0));
        fence_async_smem();
        epi_sync();
        HX_PHASE(1);

        // y(i) = D2 + e^Lc D3 for chunk i: TMA store from swizzled staging
        // tiles, or direct stores when y's layout does not allow TMA.
        auto emit_y = [&](int i) {
            const float* vp = vecs(i);
            const int tp = t_begin + i * kCS;
            const int tlen = t_end - tp;
            const float e = vp[384 + row];
            float a[16], b[16];
            tmem_ld16(tm + lane_off + TM_D2 + 16 * wg, a);
            tmem_ld16(tm + lane_off + TM_D3 + 16 * wg, b);
            tmem_wait_ld();
            tc_fence_before();
            if (y_tma) {
                if (tid == 0) bulk_wait_read0();  // previous chunk's store has left the staging tiles
                epi_sync();
                uint8_t* tile = sY + 16384 * (wg >> 1);
#pragma unroll
                for (int c = 0; c < 4; ++c)
                    *reinterpret_cast<float4*>(tile + sw128_off(row, 4 * (wg & 1) + c)) =
                        make_float4(fmaf(e, b[4 * c], a[4 * c]), fmaf(e, b[4 * c + 1], a[4 * c + 1]),
                                    fmaf(e, b[4 * c + 2], a[4 * c + 2]), fmaf(e, b[4 * c + 3], a[4 * c + 3]));
                fence_async_smem();
                epi_sync();
                if (tid == 0) {
                    tma_store_4d(&ymap, sY, p0, tl.h, tp, tl.seq);
                    tma_store_4d(&ymap, sY + 16384, p0 + 32, tl.h, tp, tl.seq);
                    bulk_commit();
                }
            } else if (row < tlen) {
                float* yr = p.y + (int64_t)tl.seq * p.seq_y + (int64_t)(tp + row) * p.s_y0 +
                            (int64_t)tl.h * p.s_y1 + (int64_t)(p0 + 16 * wg) * p.s_y2;
#pragma unroll
                for (int q = 0; q < 16; ++q) {
                    const int c = 16 * wg + q;
                    if (c < pw) yr[(int64_t)q * p.s_y2] = fmaf(e, b[q], a[q]);
                }
            }
        };

        for (int i = 0; i < n_ch; ++i) {
            const uint32_t par = (uint32_t)(i & 1);
            const float* v4 = vecs(i);

            // B: xw(i)
            if (!(ok = epi_wait(&bars.x[i & 1], (uint32_t)((i >> 1) & 1), kFaultTmaOut))) break;
            HX_PHASE(2);
            build_xw512(sX(i), sXW, sXW + 16384, v4 + 256);
            fence_async_smem();
            epi_arrive(&bars.xw_ready);
            HX_PHASE(5);

            // D: y(i-1)
            if (i > 0) {
                if (!(ok = epi_wait(&bars.g2, par ^ 1u, kFaultMmaOut))) break;
                HX_PHASE(3);
                tc_fence_after();
                emit_y(i - 1);
                epi_arrive(&bars.d_free);
                HX_PHASE(4);
            }

            // E: prefix of chunk i+1
            if (i + 1 < n_ch) {
                const float raw = dt_next;
                dt_next = raw_dt(i + 2);
                prefix(i + 1, raw);
            }
            HX_PHASE(7);

            // F: M'(i) (columns 32*wg .. +32) and the carry
            if (!(ok = epi_wait(&bars.acc1, par, kFaultMmaOut))) break;
            HX_PHASE(8);
            tc_fence_after();
            {
                const float* Lc2 = v4 + 128;
                float d[32], s4[16];
                tmem_ld16(tm + lane_off + TM_D1 + 32 * wg, *reinterpret_cast<float(*)[16]>(d));
                tmem_ld16(tm + lane_off + TM_D1 + 32 * wg + 16, *reinterpret_cast<float(*)[16]>(d + 16));
                tmem_ld16(tm + lane_off + TM_D4 + 16 * wg, s4);
                tmem_wait_ld();
                tc_fence_before();
                const float Lt = Lc2[row];
                const bool split = v4[640] != 0.0f;
                uint8_t* tile = sM + 16384 * (wg >> 1);
#pragma unroll
                for (int c = 0; c < 4; ++c) {
                    const int j0 = 32 * wg + 8 * c;
                    float m[8];
                    if (j0 > row) {
#pragma unroll
                        for (int e = 0; e < 8; ++e) m[e] = 0.0f;
                    } else if (split) {
                        const float4 fa = *reinterpret_cast<const float4*>(v4 + 512 + j0);
                        const float4 fb = *reinterpret_cast<const float4*>(v4 + 516 + j0);
                        const float F8[8] = {fa.x, fa.y, fa.z, fa.w, fb.x, fb.y, fb.z, fb.w};
                        const float eg = ex2(Lt - Lc2[j0]);
#pragma unroll
                        for (int e = 0; e < 8; ++e) m[e] = (j0 + e <= row) ? d[8 * c + e] * (eg * F8[e]) : 0.0f;
                    } else {
                        const float4 la = *reinterpret_cast<const float4*>(Lc2 + j0);
                        const float4 lb = *reinterpret_cast<const float4*>(Lc2 + j0 + 4);
                        const float4 da = *reinterpret_cast<const float4*>(v4 + j0);
                        const float4 dbv = *reinterpret_cast<const float4*>(v4 + j0 + 4);
                        const float L8[8] = {la.x, la.y, la.z, la.w, lb.x, lb.y, lb.z, lb.w};
                        const float T8[8] = {da.x, da.y, da.z, da.w, dbv.x, dbv.y, dbv.z, dbv.w};
#pragma unroll
                        for (int e = 0; e < 8; ++e)
                            m[e] = (j0 + e <= row) ? d[8 * c + e] * ex2(Lt - L8[e]) * T8[e] : 0.0f;
                    }
                    *reinterpret_cast<uint4*>(tile + sw128_off(row, 4 * (wg & 1) + c)) =
                        make_uint4(pack_bf16x2(m[0], m[1]), pack_bf16x2(m[2], m[3]), pack_bf16x2(m[4], m[5]),
                                   pack_bf16x2(m[6], m[7]));
                }
                const float decay = ex2(Lc2[kCS - 1]);
#pragma unroll
                for (int k = 0; k < 16; ++k) S[k] = fmaf(decay, S[k], s4[k]);
            }
            fence_async_smem();
            epi_arrive(&bars.m_ready);
            HX_PHASE(9);

            // H: S_{i+1} once G3(i) has read S_i
            if (!(ok = epi_wait(&bars.g3, par, kFaultMmaOut))) break;
            HX_PHASE(11);
            store_state16(sS, row, wg, S);
            fence_async_smem();
            HX_PHASE(12);
        }
        if (ok && n_ch > 0) {
            if ((ok = epi_wait(&bars.g2, (uint32_t)((n_ch - 1) & 1), kFaultMmaOut))) {
                tc_fence_after();
                emit_y(n_ch - 1);
            }
        }
        HX_PHASE(13);
        if (ok && tl.run == p.n_runs - 1) {
            float* s1 = p.s1 + (int64_t)tl.seq * p.seq_s + (int64_t)tl.h * p.s_s0 + (int64_t)p0 * p.s_s1 + row;
#pragma unroll
            for (int k = 0; k < 16; ++k) {
                const int c = 16 * wg + k;
                if (c < pw) s1[(int64_t)c * p.s_s1] = S[k];
            }
        }
        if (tid == 0 && y_tma) bulk_wait0();  // y stores complete before the CTA exits
    }
    tc_fence_before();
    __syncthreads();
    if (is_mma) tmem_dealloc(tm, 512);
    HX_PHASE(14);
}

// ---------------------------------------------------------------------------
// Carry kernel (the reference's Pass B, over runs instead of chunks): turns
// the run states from a zero start into run-entry states, in place:
//   S = s0[ids[seq]];  for r = 0 .. R-2:  S = exp(lam_r) S + agg_r;  agg_r <- S
// so afterwards slot r holds the state entering run r + 1.  One thread per
// float4 of one (seq, head)'s [P][N] state; the loads of successive runs are
// independent, so several are kept in flight.
// ---------------------------------------------------------------------------
constexpr int kCarryThreads = 256;

__global__ void __launch_bounds__(kCarryThreads) tc_carry_kernel(ScanParams p) {
    const int64_t per_head4 = (int64_t)p.P * p.N / 4;
    const int64_t gid = (int64_t)blockIdx.x * kCarryThreads + threadIdx.x;
    const int64_t head_lin = gid / per_head4;  // seq * H + h
    if (head_lin >= (int64_t)p.S * p.H) return;
    const int e4 = (int)(gid - head_lin * per_head4);
    const int seq = (int)(head_lin / p.H), h = (int)(head_lin % p.H);
    const int c = (4 * e4) / p.N, n = (4 * e4) % p.N;  // N % 4 == 0
    const int src = p.has_ids ? p.ids[seq] : seq;
    const float* s0 = p.s0 + (int64_t)src * p.seq_s + (int64_t)h * p.s_s0 + (int64_t)c * p.s_s1 + n;
    float4 S = make_float4(s0[0], s0[1], s0[2], s0[3]);
    const int64_t unit0 = head_lin * p.n_runs;
    float4* agg = reinterpret_cast<float4*>(p.agg + unit0 * (int64_t)p.P * p.N) + e4;
    const int R = p.n_runs - 1;
    int r = 0;
    for (; r + 4 <= R; r += 4) {
        float4 v[4];
        float a[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            v[k] = agg[(r + k) * per_head4];
            a[k] = expf(p.lam[unit0 + r + k]);
        }
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            S.x = fmaf(a[k], S.x, v[k].x);
            S.y = fmaf(a[k], S.y, v[k].y);
            S.z = fmaf(a[k], S.z, v[k].z);
            S.w = fmaf(a[k], S.w, v[k].w);
            agg[(r + k) * per_head4] = S;
        }
    }
    for (; r < R; ++r) {
        const float4 v = agg[r * per_head4];
        const float a = expf(p.lam[unit0 + r]);
        S.x = fmaf(a, S.x, v.x);
        S.y = fmaf(a, S.y, v.y);
        S.z = fmaf(a, S.z, v.z);
        S.w = fmaf(a, S.w, v.w);
        agg[r * per_head4] = S;
    }
}

// ---------------------------------------------------------------------------
// Chunk vectors computed by one warp (no block barriers): lane l owns the
// four tokens 4l..4l+3 of the 128-token chunk.  Returns, for those tokens,
// dt (0 past the chunk end) and the inclusive prefix of A*dt in log2 units;
// *total gets the chunk's sum of A*dt (log2 units).
// ---------------------------------------------------------------------------
__device__ __forceinline__ void warp_chunk_prefix(const ScanParams& p, int64_t db, int t0, int tlen, float Ah2,
                                                  const float (&raw)[4], float (&v)[4], float (&pre)[4],
                                                  float* total) {
    const int lane = threadIdx.x & 31;
    float run = 0.0f;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        v[k] = (4 * lane + k < tlen) ? dt_of(raw[k], p.dt_min, p.dt_max) : 0.0f;
        run += Ah2 * v[k];
        pre[k] = run;
    }
    float incl = run;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const float u = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += u;
    }
    const float excl = incl - run;
#pragma unroll
    for (int k = 0; k < 4; ++k) pre[k] += excl;
    *total = __shfl_sync(0xffffffffu, incl, 31);
}

__device__ __forceinline__ void warp_load_dt(const ScanParams& p, int64_t db, int t0, int t_end, float (&raw)[4]) {
    const int lane = threadIdx.x & 31;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        const int t = t0 + 4 * lane + k;
        raw[k] = t < t_end ? p.dt[db + (int64_t)t * p.s_dt0] : 0.0f;
    }
}

// ---------------------------------------------------------------------------
// State kernel: the run's state from a zero start, G4 accumulated over the
// whole run in one TMEM accumulator, plus the run's log-decay.
//
//   warps 0-7  (256)  xw hi/lo from x and the decay weights (2 buffers)
//   warp 8  (lane 0)  TMA producer (3-stage ring of B + x) and MMA issuer
//   warp 9            decay weights w_j = dt_j exp(sum_{i>j in run} A dt_i)
//                     into a 4-slot ring, running ahead of the builders
//
// Chunks are visited last to first so the decay from token j to the end of
// the run is a sum of same-sign terms.
// ---------------------------------------------------------------------------
constexpr int kStEpi = 256;
constexpr int kStThreads = kStEpi + 64;
constexpr int kStStages = 3;
constexpr int kStRing = 4;
constexpr uint32_t SO_STAGE = 49152;                   // B 32 KB | x 16 KB
constexpr uint32_t SO_XW = kStStages * SO_STAGE;       // 2 x (hi 16 KB | lo 16 KB)
constexpr uint32_t SO_W = SO_XW + 2 * 32768;           // kStRing x 128 weights
constexpr uint32_t SMEM_STATE = SO_W + kStRing * 512 + 1024;

struct StBars {
    uint64_t full[kStStages], b_done[kStStages], xw_full[2], xw_empty[2], w_full[kStRing], w_empty[kStRing];
};

__device__ __forceinline__ bool st_wait(uint64_t* bar, uint32_t parity, unsigned code) {
    const bool ok = mbar_wait(bar, parity, kWaitBudget);
    const bool all = named_and(1, kStEpi, ok);
    if (!all && threadIdx.x == 0) atomicCAS(&g_tc_fault, 0u, code);
    return all;
}

__global__ void __launch_bounds__(kStThreads, 1) tc_state_kernel(const __grid_constant__ TcMaps maps, ScanParams p,
                                                                 int runs_in_grid) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* sm = align1024(smem_raw);
    float* wring = reinterpret_cast<float*>(sm + SO_W);
    __shared__ StBars bars;
    __shared__ uint32_t tmem_base;
    __shared__ float lam_total;

    HX_PHASE_START;
    const int tid = threadIdx.x, warp = tid >> 5;
    const bool is_mma = warp == 8, is_vec = warp == 9;
    const int wg = (warp >> 2) & 1;
    const int row = 32 * (warp & 3) + (tid & 31);
    const uint32_t lane_off = (uint32_t)(32 * (warp & 3)) << 16;

    const Tile tl = decode_tile(blockIdx.x, p.n_pslab, p.H, runs_in_grid);
    const int p0 = tl.slab * kSlab, pw = min(kSlab, p.P - p0);
    const int g = tl.h / p.hpg;
    const float Ah = p.A[(int64_t)tl.h * p.s_a];
    const int t_begin = tl.run * p.run_tok;
    const int t_end = min(p.L, t_begin + p.run_tok);
    const int n_ch = (t_end - t_begin + kCS - 1) / kCS;
    const int64_t db = (int64_t)tl.seq * p.seq_dt + (int64_t)tl.h * p.s_dt1;
    auto stage = [&](int q) { return sm + (uint32_t)(q % kStStages) * SO_STAGE; };
    auto xwbuf = [&](int q) { return sm + SO_XW + (uint32_t)(q & 1) * 32768u; };
    auto t0_of = [&](int q) { return t_begin + (n_ch - 1 - q) * kCS; };  // visit order q -> chunk

    if (tid == 0) {
        for (int k = 0; k < kStStages; ++k) {
            mbar_init(&bars.full[k], 1);
            mbar_init(&bars.b_done[k], 1);
        }
        for (int k = 0; k < 2; ++k) {
            mbar_init(&bars.xw_full[k], kStEpi / 32);
            mbar_init(&bars.xw_empty[k], 1);
        }
        for (int k = 0; k < kStRing; ++k) {
            mbar_init(&bars.w_full[k], 1);
            mbar_init(&bars.w_empty[k], kStEpi / 32);
        }
        fence_mbar_init();
    }
    if (is_mma) {
        tmem_alloc(&tmem_base, 64);
        tmem_relinquish();
    }
    __syncthreads();
    tc_fence_after();
    const uint32_t tm = tmem_base;

    auto load = [&](int q) {
        uint8_t* st = stage(q);
        uint64_t* bar = &bars.full[q % kStStages];
        const int t0 = t0_of(q);
        mbar_expect_tx(bar, 3 * 16384);
        tma_load_4d(st, &maps.b, bar, 0, g, t0, tl.seq);
        tma_load_4d(st + 16384, &maps.b, bar, 64, g, t0, tl.seq);
        tma_load_4d(st + 32768, &maps.x, bar, p0, tl.h, t0, tl.seq);
    };

    bool ok = true;
    if (is_mma) {
        if ((tid & 31) == 0) {
            prefetch_tmap(&maps.x);
            prefetch_tmap(&maps.b);
            for (int q = 0; q < kStStages && q < n_ch; ++q) load(q);
            HX_PHASE_T(16, 256);
            for (int q = 0; q < n_ch && ok; ++q) {
                const int s = q % kStStages;
                const uint32_t pf = (uint32_t)((q / kStStages) & 1);
                if (!(ok = mbar_wait(&bars.full[s], pf, kWaitBudget))) break;
                HX_PHASE_T(17, 256);
                if (!(ok = mbar_wait(&bars.xw_full[q & 1], (uint32_t)((q >> 1) & 1), kWaitBudget))) break;
                HX_PHASE_T(18, 256);
                tc_fence_after();
                const uint32_t aB = smem_u32(stage(q)), aXH = smem_u32(xwbuf(q)), aXL = aXH + 16384;
#pragma unroll
                for (int ks = 0; ks < 8; ++ks)
                    mma_bf16(tm, desc_mnmajor(aB, ks), desc_mnmajor(aXH, ks), ID_G4, (q > 0 || ks > 0) ? 1u : 0u);
#pragma unroll
                for (int ks = 0; ks < 8; ++ks) mma_bf16(tm, desc_mnmajor(aB, ks), desc_mnmajor(aXL, ks), ID_G4, 1u);
                mma_commit(&bars.xw_empty[q & 1]);
                mma_commit(&bars.b_done[s]);
                HX_PHASE_T(19, 256);
                if (q + kStStages < n_ch) {
                    // the builders consumed this stage's x before xw_full; B is
                    // free once these MMAs retire
                    if (!(ok = mbar_wait(&bars.b_done[s], pf, kWaitBudget))) break;
                    load(q + kStStages);
                }
                HX_PHASE_T(20, 256);
            }
            if (!ok) {
                atomicCAS(&g_tc_fault, 0u, kFaultMmaState);
                mbar_wait(&bars.xw_empty[0], 0, kWaitBudget);
            }
        }
        __syncwarp();
    } else if (is_vec) {
        // ---- decay weights, ahead of the builders --------------------------
        const float Ah2 = Ah * kLog2e;
        float later = 0.0f;  // log2 units: sum of A*dt over chunks after this one
        float raw[4], raw_next[4];
        warp_load_dt(p, db, t0_of(0), t_end, raw);
        for (int q = 0; q < n_ch && ok; ++q) {
            const int t0 = t0_of(q);
            if (q + 1 < n_ch) warp_load_dt(p, db, t0_of(q + 1), t_end, raw_next);
            float v[4], pre[4], total;
            warp_chunk_prefix(p, db, t0, min(kCS, t_end - t0), Ah2, raw, v, pre, &total);
            const int slot = q % kStRing;
            if (q >= kStRing) {
                if (!(ok = mbar_wait(&bars.w_empty[slot], (uint32_t)(((q - kStRing) / kStRing) & 1), kWaitBudget)))
                    break;
            }
            float* w = wring + slot * 128;
            const int lane = tid & 31;
#pragma unroll
            for (int k = 0; k < 4; ++k) w[4 * lane + k] = v[k] * ex2(later + (total - pre[k]));
            later += total;
            __syncwarp();
            if (lane == 0) mbar_arrive(&bars.w_full[slot]);
#pragma unroll
            for (int k = 0; k < 4; ++k) raw[k] = raw_next[k];
        }
        if (!ok) atomicCAS(&g_tc_fault, 0u, kFaultMmaState);
        if ((tid & 31) == 0) lam_total = later / kLog2e;
        __syncwarp();
    } else {
        // ---- xw builders ----------------------------------------------------
        HX_PHASE(21);
        for (int q = 0; q < n_ch; ++q) {
            const int slot = q % kStRing;
            if (!(ok = st_wait(&bars.w_full[slot], (uint32_t)((q / kStRing) & 1), kFaultMmaState))) break;
            HX_PHASE(22);
            if (q >= 2) {
                if (!(ok = st_wait(&bars.xw_empty[q & 1], (uint32_t)(((q - 2) >> 1) & 1), kFaultMmaState))) break;
            }
            HX_PHASE(23);
            if (!(ok = st_wait(&bars.full[q % kStStages], (uint32_t)((q / kStStages) & 1), kFaultTmaState))) break;
            HX_PHASE(24);
            const float* wv = wring + slot * 128;
            const uint8_t* sX = stage(q) + 32768;
            uint8_t* sXH = xwbuf(q);
            uint8_t* sXL = sXH + 16384;
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const int i = tid + kStEpi * k;
                const int j = i >> 3, c = i & 7;
                const uint32_t off = sw128_off(j, c);
                const uint4 rw = *reinterpret_cast<const uint4*>(sX + off);
                const float wj = wv[j];
                const uint32_t in[4] = {rw.x, rw.y, rw.z, rw.w};
                uint32_t hi[4], lo[4];
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    float a, b;
                    unpack_bf16x2(in[e], a, b);
                    a *= wj;
                    b *= wj;
                    hi[e] = pack_bf16x2(a, b);
                    float ah, bh;
                    unpack_bf16x2(hi[e], ah, bh);
                    lo[e] = pack_bf16x2(a - ah, b - bh);
                }
                *reinterpret_cast<uint4*>(sXH + off) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
                *reinterpret_cast<uint4*>(sXL + off) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
            }
            fence_async_smem();
            __syncwarp();
            if ((tid & 31) == 0) {
                mbar_arrive(&bars.xw_full[q & 1]);
                mbar_arrive(&bars.w_empty[slot]);
            }
            HX_PHASE(25);
        }
        // all G4 MMAs retired: the last chunk's commit
        if (ok && n_ch > 0)
            ok = st_wait(&bars.xw_empty[(n_ch - 1) & 1], (uint32_t)(((n_ch - 1) >> 1) & 1), kFaultMmaState);
        tc_fence_after();
        if (ok) {
            const int64_t unit = ((int64_t)tl.seq * p.H + tl.h) * p.n_runs + tl.run;
            float* out = p.agg + unit * (int64_t)p.P * p.N + (int64_t)p0 * p.N + row;
            float d[32];
            tmem_ld16(tm + lane_off + 32 * wg, *reinterpret_cast<float(*)[16]>(d));
            tmem_ld16(tm + lane_off + 32 * wg + 16, *reinterpret_cast<float(*)[16]>(d + 16));
            tmem_wait_ld();
#pragma unroll
            for (int e = 0; e < 32; ++e) {
                const int c = 32 * wg + e;
                if (c < pw) out[(int64_t)c * p.N] = d[e];
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (ok && tid == 0 && tl.slab == 0)
        p.lam[((int64_t)tl.seq * p.H + tl.h) * p.n_runs + tl.run] = lam_total;
    if (is_mma) tmem_dealloc(tm, 64);
    HX_PHASE(26);
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

// 4-D f32 map (chan, head, tok, seq) for TMA stores of y, box 32 x 1 x 128 x 1.
bool make_ymap(EncodeFn fn, CUtensorMap* m, void* base, const ScanParams& p) {
    cuuint64_t dims[4] = {(cuuint64_t)p.P, (cuuint64_t)p.H, (cuuint64_t)p.L, (cuuint64_t)p.S};
    cuuint64_t strides[3] = {(cuuint64_t)(p.s_y1 * 4), (cuuint64_t)(p.s_y0 * 4), (cuuint64_t)(p.seq_y * 4)};
    cuuint32_t box[4] = {32, 1, (cuuint32_t)kCS, 1};
    cuuint32_t es[4] = {1, 1, 1, 1};
    return fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, base, dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
              CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool y_tma_ok(const ScanParams& p) {
    if (p.s_y2 != 1) return false;
    const int64_t st[3] = {p.s_y1, p.s_y0, p.seq_y};
    for (int64_t s : st)
        if (s <= 0 || (s * 4) % 16 != 0) return false;
    return (reinterpret_cast<uintptr_t>(p.y) & 15) == 0;
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
    CUtensorMap ymap;
    int y_tma = y_tma_ok(p) ? 1 : 0;
    if (y_tma && !make_ymap(fn, &ymap, p.y, p)) y_tma = 0;
    if (!y_tma) std::memset(&ymap, 0, sizeof(ymap));
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const char* only = std::getenv("HELIX_ONLY_PASS");
    const bool do_a = !only || *only == 'A';
    const bool do_c = !only || *only == 'C';
    const int64_t per_run = (int64_t)p.n_pslab * p.H * S;
    if (pl.need_state_kernel && do_a) {
        const int runs = pl.n_runs - 1;
        tc_state_kernel<<<(unsigned)(per_run * runs), kStThreads, SMEM_STATE, st>>>(maps, p, runs);
        const cudaError_t e = cudaGetLastError();
        if (e != cudaSuccess) return e;
    }
    const bool do_b = !only || *only == 'B';
    if (pl.need_state_kernel && do_b) {
        const int64_t n4 = (int64_t)S * p.H * p.P * p.N / 4;
        tc_carry_kernel<<<(unsigned)((n4 + kCarryThreads - 1) / kCarryThreads), kCarryThreads, 0, st>>>(p);
        const cudaError_t e = cudaGetLastError();
        if (e != cudaSuccess) return e;
    }
    if (do_c) {
        tc_out_kernel<<<(unsigned)(per_run * pl.n_runs), kOutThreads, SMEM_OUT, st>>>(maps, ymap, p, y_tma);
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
