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
// Timeline of one CTA (blockIdx.x == HX_TL_CTA): clock64 of event `ev` in
// chunk `i`.
extern __device__ long long hx_tl[32 * 64];
#define HX_TL_CTA 160
#define HX_TL(ev, i)                                                          \
    do {                                                                      \
        if (blockIdx.x == HX_TL_CTA && (i) < 64) hx_tl[(ev) * 64 + (i)] = clock64(); \
    } while (0)
#else
#define HX_TL(ev, i) do {} while (0)
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
constexpr uint32_t ID_G4W = idesc_bf16(128, 128, true, true);

constexpr uint32_t ID_G1 = idesc_bf16(128, 128, false, false);
constexpr uint32_t ID_G2 = idesc_bf16(128, 64, false, true);
constexpr uint32_t ID_G3 = idesc_bf16(128, 64, false, true);

__device__ __forceinline__ uint8_t* align1024(uint8_t* p) {
    return reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(p) + 1023) & ~uintptr_t(1023));
}

// Descriptor of a shared-memory address `off` bytes past the one `base`
// describes.  Shared addresses stay below 256 KB, so the 14-bit start field
// never carries into the next field and the offset simply adds.
__device__ __forceinline__ uint64_t desc_add(uint64_t base, uint32_t off) { return base + (uint64_t)(off >> 4); }
__device__ __forceinline__ uint32_t kmajor_off(int ks) { return (uint32_t)(ks >> 2) * 16384u + (uint32_t)(ks & 3) * 32u; }

// K-major operand: K step ks (16 elements) of a 2-tile (K = 128) operand.
__device__ __forceinline__ uint64_t desc_kmajor(uint32_t base, int ks) {
    return sdesc_sw128(base + (uint32_t)(ks >> 2) * 16384u + (uint32_t)(ks & 3) * 32u, 16, 1024);
}
// MN-major operand: K step ks = 16 rows of 128 B; M/N tiles 16 KB apart.
__device__ __forceinline__ uint64_t desc_mnmajor(uint32_t base, int ks) {
    return sdesc_sw128(base + (uint32_t)ks * 2048u, 16384, 1024);
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
// Output kernel: warp roles with the accumulators, M' and the carried state
// all in TMEM.
//
//   warps 0-3    W_y   y(i) = D2 + e^Lc D3 -> global (row per thread)
//   warps 4-11   W_m   M'(i) = D1 masked and decayed (x dt) -> bf16 into TMEM
//                      (two warps per lane quarter, 64 columns each)
//   warps 12-15  W_c   carry S_{i+1} = e^{Lc_end} S_i + D4 (fp32 in TMEM) and
//                      its bf16 copy in smem for G3
//   warps 16-17  W_xw  xw(i) = w x as bf16 hi | lo (no TMEM access)
//   warp 18      TMA producer and MMA issuer (lane 0)
//   warp 19      chunk vectors (dt, Lc, w, e^Lc, split decay) into a 3-slot
//                ring, running ahead
//
// MMA issue order, iteration i:
//   G1(i) C.B^T -> D1, G4(i) B^T.xw_hi + B^T.xw_lo -> D4     commit acc1, xw_free
//   G2(i-1) M'(i-1).x(i-1) -> D2 (A from TMEM)                commit g2; TMA x(i+1)
//   G3(i) C.S_i -> D3[i&1]                                    commit g3; TMA C/B(i+2)
// so M'(i-1) is built while G1/G4(i) run.  C/B and x are double-buffered.
//
// TMEM columns: D1 0-127 | M' 128-191 | D2 192-255 | D3 256-383 (x2) |
//               D4 384-447 | S 448-511.
//
// M' decay: exp(Lc_t - Lc_j) = exp(Lc_t - Lc_g) exp(Lc_g - Lc_j) with g the
// first token of j's 8-token group; the second factor times dt_j comes with
// the chunk vectors, so a row needs one exp per 8 columns.  A chunk in which
// some group spans more than 20 nats (where the split could lose a factor to
// underflow) takes the direct per-element exp.
// ---------------------------------------------------------------------------
constexpr uint32_t OO_CB = 0;             // 2 x (C 32 KB | B 32 KB)
constexpr uint32_t OO_X = 131072;         // 2 x 16 KB  x chunks
constexpr uint32_t OO_XW = 163840;        // 32 KB  xw hi | lo
constexpr uint32_t OO_S = 196608;         // 16 KB  state bf16 [n][p]
constexpr uint32_t OO_V = 212992;         // chunk-vector ring
constexpr int kRing = 3;
constexpr int kVec = 5 * 128 + 16;        // floats per ring slot: dt | Lc2 | w | e | f*dt | flag
constexpr uint32_t SMEM_OUT = OO_V + kRing * kVec * 4 + 1024;
constexpr int kOutThreads = 640;          // 20 warps: 96 registers per thread
constexpr uint32_t T_D1 = 0, T_M = 128, T_D2 = 192, T_D3 = 256, T_D4 = 384, T_S = 448;
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kSpanMax2 = 20.0f * kLog2e;
constexpr uint32_t ID_G4 = idesc_bf16(128, 64, true, true);

enum Role : int { kRoleY = 0, kRoleM = 1, kRoleC = 2, kRoleXW = 3 };
constexpr int kGWarpMma = 18, kGWarpVec = 19, kGXwThreads = 64;
__host__ __device__ constexpr int role_threads(int r) { return r == kRoleM ? 256 : r == kRoleXW ? kGXwThreads : 128; }

struct OutBars {
    uint64_t x[2], xw_ready, xw_free, acc1, d1_read, d4_read, m_ready, s_ready, g2, g3, g3y[2], d_free;
    uint64_t v_full[kRing], v_empty[kRing];
};

// Bounded wait by all threads of one role, agreed with a vote on the role's
// named barrier (ids 2..5).
__device__ __forceinline__ bool role_wait(uint64_t* bar, uint32_t parity, int role, unsigned code, bool leader) {
    const bool ok = mbar_wait(bar, parity, kWaitBudget);
    const bool all = named_and(2 + role, role_threads(role), ok);
    if (!all && leader) atomicCAS(&g_tc_fault, 0u, code);
    return all;
}
__device__ __forceinline__ void warp_arrive(uint64_t* bar) {
    __syncwarp();
    if ((threadIdx.x & 31) == 0) mbar_arrive(bar);
}

// One CTA's share of the output pass: (seq, head, 64-channel slab, run).
struct OutTile {
    Tile tl;
    int p0, pw, g;
    float Ah;
    int t_begin, t_end, n_ch;
    int64_t db, unit0;
};

__device__ __forceinline__ OutTile out_tile(const ScanParams& p) {
    OutTile o;
    o.tl = decode_tile(blockIdx.x, p.n_pslab, p.H, p.n_runs);
    o.p0 = o.tl.slab * kSlab;
    o.pw = min(kSlab, p.P - o.p0);
    o.g = o.tl.h / p.hpg;
    o.Ah = p.A[(int64_t)o.tl.h * p.s_a];
    o.t_begin = o.tl.run * p.run_tok;
    o.t_end = min(p.L, o.t_begin + p.run_tok);
    o.n_ch = (o.t_end - o.t_begin + kCS - 1) / kCS;
    o.db = (int64_t)o.tl.seq * p.seq_dt + (int64_t)o.tl.h * p.s_dt1;
    o.unit0 = ((int64_t)o.tl.seq * p.H + o.tl.h) * p.n_runs;
    return o;
}

// C and B of one chunk (128 tokens x 128 states each, two 64-state SW128
// tiles per operand) into st: C at +0, B at +32 KB.
__device__ __forceinline__ void load_cb_chunk(const TcMaps& maps, uint8_t* st, uint64_t* bar, int g, int t0, int seq) {
    mbar_expect_tx(bar, 4 * 16384);
    tma_load_4d(st, &maps.c, bar, 0, g, t0, seq);
    tma_load_4d(st + 16384, &maps.c, bar, 64, g, t0, seq);
    tma_load_4d(st + 32768, &maps.b, bar, 0, g, t0, seq);
    tma_load_4d(st + 49152, &maps.b, bar, 64, g, t0, seq);
}

__device__ __forceinline__ void out_general(const TcMaps& maps, const ScanParams& p, const OutTile& ot, uint8_t* sm,
                                            uint32_t tm, uint64_t* cb_bar) {
    float* ring = reinterpret_cast<float*>(sm + OO_V);
    __shared__ OutBars bars;

    HX_PHASE_START;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int role = warp < 4 ? kRoleY : warp < 12 ? kRoleM : warp < 16 ? kRoleC : kRoleXW;  // 16-17 XW
    const int row = 32 * (warp & 3) + lane;
    const uint32_t lane_off = (uint32_t)(32 * (warp & 3)) << 16;

    const Tile tl = ot.tl;
    const int p0 = ot.p0, pw = ot.pw, g = ot.g;
    const float Ah = ot.Ah;
    const int t_begin = ot.t_begin, t_end = ot.t_end, n_ch = ot.n_ch;
    const int64_t db = ot.db, unit0 = ot.unit0;

    uint8_t* sXW = sm + OO_XW;
    uint8_t* sS = sm + OO_S;
    auto sCB = [&](int i) { return sm + OO_CB + (uint32_t)(i & 1) * 65536u; };
    auto sX = [&](int i) { return sm + OO_X + (uint32_t)(i & 1) * 16384u; };
    auto slot = [&](int i) { return ring + (i % kRing) * kVec; };

    if (tid == 0) {
        for (int k = 0; k < 2; ++k) mbar_init(&bars.x[k], 1);
        mbar_init(&bars.xw_ready, kGXwThreads / 32);
        mbar_init(&bars.xw_free, 1);
        mbar_init(&bars.acc1, 1);
        mbar_init(&bars.d1_read, 8);
        mbar_init(&bars.d4_read, 4);
        mbar_init(&bars.m_ready, 8);
        mbar_init(&bars.s_ready, 4);
        mbar_init(&bars.g2, 1);
        mbar_init(&bars.g3, 1);
        mbar_init(&bars.g3y[0], 1);
        mbar_init(&bars.g3y[1], 1);
        mbar_init(&bars.d_free, 4);
        for (int k = 0; k < kRing; ++k) {
            mbar_init(&bars.v_full[k], 1);
            mbar_init(&bars.v_empty[k], 16 + kGXwThreads / 32);
        }
        fence_mbar_init();
    }
    __syncthreads();
    bool ok = true;

    if (warp == kGWarpMma) {
        // ================= TMA producer + MMA issuer ========================
        if (lane == 0) {
            auto load_cb = [&](int i) { load_cb_chunk(maps, sCB(i), &cb_bar[i & 1], g, t_begin + i * kCS, tl.seq); };
            auto load_x = [&](int i) {
                mbar_expect_tx(&bars.x[i & 1], 16384);
                tma_load_4d(sX(i), &maps.x, &bars.x[i & 1], p0, tl.h, t_begin + i * kCS, tl.seq);
            };
            // C/B of chunks 0 and 1 are already in flight (kernel prologue)
            for (int i = 0; i < 2 && i < n_ch; ++i) load_x(i);
            const uint32_t aXH = smem_u32(sXW), aXL = aXH + 16384, aS = smem_u32(sS);
            HX_PHASE_T(16, 32 * kGWarpMma);
            for (int i = 0; i <= n_ch && ok; ++i) {
                if (i < n_ch) {
                    const uint32_t par = (uint32_t)(i & 1), pf = (uint32_t)((i >> 1) & 1);
                    if (!(ok = mbar_wait(&cb_bar[i & 1], pf, kWaitBudget))) break;
                    if (!(ok = mbar_wait(&bars.x[i & 1], pf, kWaitBudget))) break;
                    if (!(ok = mbar_wait(&bars.xw_ready, par, kWaitBudget))) break;
                    if (i > 0) {
                        if (!(ok = mbar_wait(&bars.d1_read, par ^ 1u, kWaitBudget))) break;
                        if (!(ok = mbar_wait(&bars.d4_read, par ^ 1u, kWaitBudget))) break;
                    }
                    HX_PHASE_T(17, 32 * kGWarpMma);
                    tc_fence_after();
                    const uint32_t aC = smem_u32(sCB(i)), aB = aC + 32768;
#pragma unroll
                    for (int ks = 0; ks < 8; ++ks)
                        mma_bf16(tm + T_D1, desc_kmajor(aC, ks), desc_kmajor(aB, ks), ID_G1, ks > 0);
#pragma unroll
                    for (int ks = 0; ks < 8; ++ks)
                        mma_bf16(tm + T_D4, desc_mnmajor(aB, ks), desc_mnmajor(aXH, ks), ID_G4, ks > 0);
#pragma unroll
                    for (int ks = 0; ks < 8; ++ks)
                        mma_bf16(tm + T_D4, desc_mnmajor(aB, ks), desc_mnmajor(aXL, ks), ID_G4, 1);
                    mma_commit(&bars.acc1);
                    mma_commit(&bars.xw_free);
                    HX_PHASE_T(18, 32 * kGWarpMma);
                }
                if (i > 0) {
                    const int k = i - 1;  // G2 of the previous chunk
                    if (!(ok = mbar_wait(&bars.m_ready, (uint32_t)(k & 1), kWaitBudget))) break;
                    if (k > 0) {
                        if (!(ok = mbar_wait(&bars.d_free, (uint32_t)((k - 1) & 1), kWaitBudget))) break;
                    }
                    HX_PHASE_T(19, 32 * kGWarpMma);
                    tc_fence_after();
                    const uint32_t aX = smem_u32(sX(k));
#pragma unroll
                    for (int ks = 0; ks < 8; ++ks)
                        mma_bf16_ts(tm + T_D2, tm + T_M + 8 * ks, desc_mnmajor(aX, ks), ID_G2, ks > 0);
                    mma_commit(&bars.g2);
                    if (k + 2 < n_ch) {
                        // x(k)'s buffer is free once G2(k) retires
                        if (!(ok = mbar_wait(&bars.g2, (uint32_t)(k & 1), kWaitBudget))) break;
                        load_x(k + 2);
                    }
                }
                if (i < n_ch) {
                    const uint32_t par = (uint32_t)(i & 1);
                    if (!(ok = mbar_wait(&bars.s_ready, par, kWaitBudget))) break;  // S_i in smem
                    HX_PHASE_T(20, 32 * kGWarpMma);
                    tc_fence_after();
                    const uint32_t aC = smem_u32(sCB(i));
#pragma unroll
                    for (int ks = 0; ks < 8; ++ks)
                        mma_bf16(tm + T_D3 + 64 * (i & 1), desc_kmajor(aC, ks), desc_mnmajor(aS, ks), ID_G3, ks > 0);
                    mma_commit(&bars.g3);
                    mma_commit(&bars.g3y[i & 1]);
                    if (i + 2 < n_ch) {
                        // G1, G4, G3 of chunk i are the last readers of its C/B buffer
                        if (!(ok = mbar_wait(&bars.g3, par, kWaitBudget))) break;
                        load_cb(i + 2);
                    }
                    HX_PHASE_T(21, 32 * kGWarpMma);
                }
            }
            if (!ok) {
                atomicCAS(&g_tc_fault, 0u, kFaultMmaOut);
                mbar_wait(&bars.g2, 0, kWaitBudget);  // let committed work land
                mbar_wait(&bars.g3, 0, kWaitBudget);
            }
        }
        __syncwarp();
    } else if (warp == kGWarpVec) {
        // ================= chunk vectors ====================================
        const float Ah2 = Ah * kLog2e;
        float raw[4], raw_next[4];
        warp_load_dt(p, db, t_begin, t_end, raw);
        for (int i = 0; i < n_ch && ok; ++i) {
            const int t0 = t_begin + i * kCS;
            if (i + 1 < n_ch) warp_load_dt(p, db, t0 + kCS, t_end, raw_next);
            float v[4], pre[4], total;
            warp_chunk_prefix(p, db, t0, min(kCS, t_end - t0), Ah2, raw, v, pre, &total);
            if (i >= kRing) {
                if (!(ok = mbar_wait(&bars.v_empty[i % kRing], (uint32_t)(((i - kRing) / kRing) & 1), kWaitBudget)))
                    break;
            }
            float* vs = slot(i);
            const float Lg = __shfl_sync(0xffffffffu, pre[0], lane & ~1);
            bool span_ok = true;
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const int t = 4 * lane + k;
                vs[t] = v[k];
                vs[128 + t] = pre[k];
                vs[256 + t] = v[k] * ex2(total - pre[k]);
                vs[384 + t] = ex2(pre[k]);
                vs[512 + t] = ex2(Lg - pre[k]) * v[k];
                span_ok = span_ok && (Lg - pre[k] <= kSpanMax2);
            }
            const bool all_ok = __all_sync(0xffffffffu, span_ok);
            if (lane == 0) vs[640] = all_ok ? 1.0f : 0.0f;
            __syncwarp();
            if (lane == 0) mbar_arrive(&bars.v_full[i % kRing]);
#pragma unroll
            for (int k = 0; k < 4; ++k) raw[k] = raw_next[k];
        }
        if (!ok) atomicCAS(&g_tc_fault, 0u, kFaultMmaOut);
    } else if (role == kRoleXW) {
        // ================= W_xw =============================================
        const int r = tid - 512;  // warps 16-17
        const bool leader = r == 0;
        for (int i = 0; i < n_ch; ++i) {
            if (!(ok = role_wait(&bars.v_full[i % kRing], (uint32_t)((i / kRing) & 1), role, kFaultMmaOut, leader))) break;
            if (!(ok = role_wait(&bars.x[i & 1], (uint32_t)((i >> 1) & 1), role, kFaultTmaOut, leader))) break;
            if (i > 0) {
                if (!(ok = role_wait(&bars.xw_free, (uint32_t)((i - 1) & 1), role, kFaultMmaOut, leader))) break;
            }
            HX_PHASE_T(22, 512);
            const float* wv = slot(i) + 256;
            const uint8_t* x = sX(i);
#pragma unroll 4
            for (int k = 0; k < 1024 / kGXwThreads; ++k) {
                const int idx = r + kGXwThreads * k;
                const int j = idx >> 3, c = idx & 7;
                const uint32_t off = sw128_off(j, c);
                const uint4 rw = *reinterpret_cast<const uint4*>(x + off);
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
                *reinterpret_cast<uint4*>(sXW + off) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
                *reinterpret_cast<uint4*>(sXW + 16384 + off) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
            }
            fence_async_smem();
            __syncwarp();
            if (lane == 0) {
                mbar_arrive(&bars.xw_ready);
                mbar_arrive(&bars.v_empty[i % kRing]);
            }
            HX_PHASE_T(23, 512);
        }
    } else if (role == kRoleM) {
        // ================= W_m: M' into TMEM ================================
        const int half = (warp - 4) >> 2;  // columns 64*half .. +64 of D1
        const bool leader = tid == 128;
        for (int i = 0; i < n_ch; ++i) {
            if (!(ok = role_wait(&bars.acc1, (uint32_t)(i & 1), role, kFaultMmaOut, leader))) break;
            if (!(ok = role_wait(&bars.v_full[i % kRing], (uint32_t)((i / kRing) & 1), role, kFaultMmaOut, leader))) break;
            HX_PHASE_T(24, 128);
            tc_fence_after();
            const float* vs = slot(i);
            const float* Lc2 = vs + 128;
            const float Lt = Lc2[row];
            const bool split = vs[640] != 0.0f;
            uint32_t mp[32];
            // two passes of 32 columns keep 32 accumulators live, not 64
#pragma unroll
            for (int hh = 0; hh < 2; ++hh) {
                float d[32];
                tmem_ld16(tm + lane_off + T_D1 + 64 * half + 32 * hh, *reinterpret_cast<float(*)[16]>(d));
                tmem_ld16(tm + lane_off + T_D1 + 64 * half + 32 * hh + 16, *reinterpret_cast<float(*)[16]>(d + 16));
                tmem_wait_ld();
                if (hh == 1) {
                    tc_fence_before();
                    warp_arrive(&bars.d1_read);
                }
#pragma unroll
                for (int c = 0; c < 4; ++c) {
                    const int j0 = 64 * half + 32 * hh + 8 * c;
                    float m[8];
                    if (j0 > row) {
#pragma unroll
                        for (int e = 0; e < 8; ++e) m[e] = 0.0f;
                    } else if (split) {
                        const float eg = ex2(Lt - Lc2[j0]);
#pragma unroll
                        for (int e = 0; e < 8; ++e)
                            m[e] = (j0 + e <= row) ? d[8 * c + e] * (eg * vs[512 + j0 + e]) : 0.0f;
                    } else {
#pragma unroll
                        for (int e = 0; e < 8; ++e)
                            m[e] = (j0 + e <= row) ? d[8 * c + e] * ex2(Lt - Lc2[j0 + e]) * vs[j0 + e] : 0.0f;
                    }
#pragma unroll
                    for (int e = 0; e < 4; ++e) mp[16 * hh + 4 * c + e] = pack_bf16x2(m[2 * e], m[2 * e + 1]);
                }
            }
            // M'(i) overwrites M'(i-1): wait for G2(i-1) to retire
            if (i > 0) {
                if (!(ok = role_wait(&bars.g2, (uint32_t)((i - 1) & 1), role, kFaultMmaOut, leader))) break;
                tc_fence_after();
            }
            tmem_st16(tm + lane_off + T_M + 32 * half, *reinterpret_cast<const uint32_t(*)[16]>(mp));
            tmem_st16(tm + lane_off + T_M + 32 * half + 16, *reinterpret_cast<const uint32_t(*)[16]>(mp + 16));
            tmem_wait_st();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) {
                mbar_arrive(&bars.m_ready);
                mbar_arrive(&bars.v_empty[i % kRing]);
            }
            HX_PHASE_T(25, 128);
        }
    } else if (role == kRoleC) {
        // ================= W_c: the carry, fp32 state in TMEM ===============
        const bool leader = tid == 384;
        const uint32_t tS = tm + lane_off + T_S;
        {
            const float* src;
            int64_t sc;
            if (tl.run == 0) {
                const int sq = p.has_ids ? p.ids[tl.seq] : tl.seq;
                src = p.s0 + (int64_t)sq * p.seq_s + (int64_t)tl.h * p.s_s0 + (int64_t)p0 * p.s_s1 + row;
                sc = p.s_s1;
            } else {
                src = p.agg + (unit0 + tl.run - 1) * (int64_t)p.P * p.N + (int64_t)p0 * p.N + row;
                sc = p.N;
            }
#pragma unroll 1
            for (int q = 0; q < 8; ++q) {
                float v[8];
#pragma unroll
                for (int k = 0; k < 8; ++k) v[k] = (8 * q + k < pw) ? src[(int64_t)(8 * q + k) * sc] : 0.0f;
                tmem_st8(tS + 8 * q, *reinterpret_cast<const uint32_t(*)[8]>(v));
                *reinterpret_cast<uint4*>(sS + sw128_off(row, q)) =
                    make_uint4(pack_bf16x2(v[0], v[1]), pack_bf16x2(v[2], v[3]), pack_bf16x2(v[4], v[5]),
                               pack_bf16x2(v[6], v[7]));
            }
            tmem_wait_st();
            fence_async_smem();
            warp_arrive(&bars.s_ready);
        }
        for (int i = 0; i < n_ch; ++i) {
            if (!(ok = role_wait(&bars.acc1, (uint32_t)(i & 1), role, kFaultMmaOut, leader))) break;
            if (!(ok = role_wait(&bars.v_full[i % kRing], (uint32_t)((i / kRing) & 1), role, kFaultMmaOut, leader))) break;
            HX_PHASE_T(26, 384);
            tc_fence_after();
            const float decay = ex2(slot(i)[128 + kCS - 1]);
            // S_{i+1} = decay S_i + D4(i): fp32 in TMEM, bf16 copy kept in registers
            uint32_t sb[32];
#pragma unroll
            for (int q = 0; q < 8; ++q) {
                float sv[8], dv[8];
                tmem_ld8(tS + 8 * q, sv);
                tmem_ld8(tm + lane_off + T_D4 + 8 * q, dv);
                tmem_wait_ld();
#pragma unroll
                for (int k = 0; k < 8; ++k) sv[k] = fmaf(decay, sv[k], dv[k]);
                tmem_st8(tS + 8 * q, *reinterpret_cast<const uint32_t(*)[8]>(sv));
#pragma unroll
                for (int k = 0; k < 4; ++k) sb[4 * q + k] = pack_bf16x2(sv[2 * k], sv[2 * k + 1]);
            }
            tmem_wait_st();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) {
                mbar_arrive(&bars.d4_read);
                mbar_arrive(&bars.v_empty[i % kRing]);
            }
            // the bf16 S in smem is G3(i)'s operand: overwrite it once G3 retires
            if (!(ok = role_wait(&bars.g3, (uint32_t)(i & 1), role, kFaultMmaOut, leader))) break;
#pragma unroll
            for (int c = 0; c < 8; ++c)
                *reinterpret_cast<uint4*>(sS + sw128_off(row, c)) =
                    make_uint4(sb[4 * c], sb[4 * c + 1], sb[4 * c + 2], sb[4 * c + 3]);
            fence_async_smem();
            warp_arrive(&bars.s_ready);
            HX_PHASE_T(27, 384);
        }
        if (ok && tl.run == p.n_runs - 1) {
            float* s1 = p.s1 + (int64_t)tl.seq * p.seq_s + (int64_t)tl.h * p.s_s0 + (int64_t)p0 * p.s_s1 + row;
            tc_fence_after();
#pragma unroll 1
            for (int q = 0; q < 8; ++q) {
                float sv[8];
                tmem_ld8(tS + 8 * q, sv);
                tmem_wait_ld();
#pragma unroll
                for (int k = 0; k < 8; ++k)
                    if (8 * q + k < pw) s1[(int64_t)(8 * q + k) * p.s_s1] = sv[k];
            }
        }
    } else {
        // ================= W_y ==============================================
        const bool leader = tid == 0;
        for (int i = 0; i < n_ch; ++i) {
            if (!(ok = role_wait(&bars.g2, (uint32_t)(i & 1), role, kFaultMmaOut, leader))) break;
            // per-buffer barrier: G3(i+1) may retire before this wait, G3(i+2) may not
            if (!(ok = role_wait(&bars.g3y[i & 1], (uint32_t)((i >> 1) & 1), role, kFaultMmaOut, leader))) break;
            if (!(ok = role_wait(&bars.v_full[i % kRing], (uint32_t)((i / kRing) & 1), role, kFaultMmaOut, leader))) break;
            HX_PHASE(28);
            tc_fence_after();
            const int tp = t_begin + i * kCS;
            const int tlen = t_end - tp;
            const float e = slot(i)[384 + row];
            float* yr = p.y + (int64_t)tl.seq * p.seq_y + (int64_t)(tp + row) * p.s_y0 + (int64_t)tl.h * p.s_y1 +
                        (int64_t)p0 * p.s_y2;
            const bool vec = p.s_y2 == 1 && pw == kSlab && (reinterpret_cast<uintptr_t>(yr) & 15) == 0;
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                float a[16], b[16];
                tmem_ld16(tm + lane_off + T_D2 + 16 * q, a);
                tmem_ld16(tm + lane_off + T_D3 + 64 * (i & 1) + 16 * q, b);
                tmem_wait_ld();
                if (row < tlen) {
                    if (vec) {
#pragma unroll
                        for (int c = 0; c < 4; ++c)
                            reinterpret_cast<float4*>(yr + 16 * q)[c] =
                                make_float4(fmaf(e, b[4 * c], a[4 * c]), fmaf(e, b[4 * c + 1], a[4 * c + 1]),
                                            fmaf(e, b[4 * c + 2], a[4 * c + 2]), fmaf(e, b[4 * c + 3], a[4 * c + 3]));
                    } else {
#pragma unroll
                        for (int k = 0; k < 16; ++k)
                            if (16 * q + k < pw) yr[(int64_t)(16 * q + k) * p.s_y2] = fmaf(e, b[k], a[k]);
                    }
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) {
                mbar_arrive(&bars.d_free);
                mbar_arrive(&bars.v_empty[i % kRing]);
            }
            HX_PHASE(29);
        }
    }
}

// ---------------------------------------------------------------------------
// Output kernel, fast path.  With f_t = exp(Lc_t - Lc_end) and the G4 operand
// xw_j = dt_j exp(Lc_end - Lc_j) x_j, the chunk's output is
//
//   y_t = f_t [ C_t . S~ + sum_{j<=t} (C_t . B_j) xw_j ],   S~ = exp(Lc_end) S
//
// so G3 (C.S~) and G2 (masked D1 . xw_hi) share one accumulator, the masked
// D1 needs no exponentials, and x is only read to build xw.  It is exact
// algebra; the scaling factors stay inside fp32/bf16 range while no chunk of
// the run decays by more than kFastSpan2 (log2 units), which the kernel
// prologue checks (runs that fail take out_general).
//
// The carried state lives in the G4 accumulator itself: W_c writes S~_i
// there and G4(i) accumulates B^T.xw_hi and B^T.xw_lo onto it, leaving
// S_{i+1}.  One TMEM read per chunk per role: under concurrent MMA traffic a
// TMEM load round trip costs hundreds of cycles, so every role reads its
// whole accumulator slice at once.
//
//   warps 0-3    W_y   y = f_t D[i&1] -> smem (xw[i&1], free after G2) -> TMA store
//   warps 4-7    W_m   D1[i&1] -> causal mask -> bf16 pairs written over
//                      D1[i&1]'s first 64 columns (row per thread, 64 columns
//                      per TMEM read)
//   warps 8-11   W_c   S_{i+1} = D4 -> s1 (last chunk) / S~_{i+1} into D4 and,
//                      as bf16, into smem for G3(i+1)
//   warps 12-17  W_xw  x from global (one chunk prefetched in registers),
//                      xw = w x -> bf16 hi | lo, two buffers
//   warp 18      TMA producer and MMA issuer (lane 0)
//   warp 19      chunk vectors (w, f, exp(Lc_end)) into a 4-slot ring
//
// MMA issue order, chunk i (G1 runs a chunk ahead):
//   G4 B^T.xw_hi, B^T.xw_lo -> D4 (accumulating onto S~_i);  G3 C.S~ -> D[i&1];
//   G1(i+1) C.B^T -> D1[(i+1)&1];  G2 mask(i).xw_hi -> D[i&1] (A from TMEM);
//   C/B(i+2) once G3(i) retires.
//
// TMEM columns: D1 0-127 | D1' 128-255 (each holding its chunk's mask, packed
//               in place, once W_m has read it) | D4 256-319 | D 320-383 |
//               D' 384-447.
// smem: C/B 2 x 64 KB | xw 2 x 32 KB | S~ bf16 16 KB | vector ring.
// ---------------------------------------------------------------------------
constexpr uint32_t OF_XW = 131072;
constexpr uint32_t OF_S = 196608;
constexpr uint32_t OF_V = 212992;
constexpr int kFRing = 4;
constexpr int kFVec = 2 * 128 + 8;  // w | f | exp(Lc_end)
static_assert(OF_V + kFRing * kFVec * 4 + 1024 <= SMEM_OUT, "fast path fits the general path's allocation");
constexpr uint32_t TF_D4 = 256, TF_D = 320;
constexpr uint32_t ID_G4N = idesc_bf16(128, 64, true, true);
constexpr float kFastSpan2 = 86.0f;  // ~59.6 nats
// Warp w runs on SM sub-partition w % 4.  The MMA warp's sub-partition hosts
// only the light vector warp and one warp of each TMEM role: an ALU-heavy
// neighbour (the xw builders) slows its MMA issue by about a third.
constexpr int kWarpY = 0, kWarpM = 4, kWarpC = 8, kWarpXw = 12, kWarpMma = 14, kWarpVec = 18;
constexpr int kXwWarps = 6;  // warps 12, 13, 15, 16, 17, 19
__device__ __forceinline__ int xw_index(int warp) { return warp < 14 ? warp - 12 : warp < 18 ? warp - 13 : warp - 14; }
constexpr int kXwThreads = 32 * kXwWarps;
constexpr int kXwVec = (1024 + kXwThreads - 1) / kXwThreads;
constexpr int kMmaTid = 32 * kWarpMma;
static_assert(kOutThreads / 32 == 20, "warp map of the fast path assumes 20 warps");

struct FastBars {
    uint64_t xw_ready[2], xw_free[2], acc1[2], g2[2], d_free[2], m_ready, g4, d4_ready, s_ready, g3;
    uint64_t v_full[kFRing], v_empty[kFRing];
};

// Bounded wait agreed by one role's warps on named barrier `id`.
__device__ __forceinline__ bool group_wait(uint64_t* bar, uint32_t parity, int id, int nthreads, bool leader) {
    const bool ok = mbar_wait(bar, parity, kWaitBudget);
    const bool all = named_and(id, nthreads, ok);
    if (!all && leader) atomicCAS(&g_tc_fault, 0u, kFaultMmaOut);
    return all;
}

// x of chunk i for W_xw thread r (0..kXwThreads-1): up to kXwVec 16-byte
// vectors of 8 channels (vector idx = r + kXwThreads k of the chunk's 1024);
// tokens past the run and channels past P read as zero.
__device__ __forceinline__ void load_x_chunk(const ScanParams& p, const OutTile& ot, int r, int i,
                                             uint4 (&v)[kXwVec]) {
    const int64_t xb = (int64_t)ot.tl.seq * p.seq_x + (int64_t)ot.tl.h * p.s_x1 + ot.p0;
    const __nv_bfloat16* xg = static_cast<const __nv_bfloat16*>(p.x);
#pragma unroll
    for (int k = 0; k < kXwVec; ++k) {
        const int idx = r + kXwThreads * k, j = idx >> 3, c = idx & 7;
        const int t = ot.t_begin + i * kCS + j;
        v[k] = make_uint4(0u, 0u, 0u, 0u);
        if (idx < 1024 && t < ot.t_end) {
            const __nv_bfloat16* src = xg + xb + (int64_t)t * p.s_x0 + 8 * c;
            if (8 * c + 8 <= ot.pw) {
                v[k] = __ldg(reinterpret_cast<const uint4*>(src));
            } else if (8 * c < ot.pw) {
                uint16_t e[8];
#pragma unroll
                for (int q = 0; q < 8; ++q) e[q] = 8 * c + q < ot.pw ? __bfloat16_as_ushort(src[q]) : (uint16_t)0;
                v[k] = make_uint4(e[0] | (uint32_t)e[1] << 16, e[2] | (uint32_t)e[3] << 16, e[4] | (uint32_t)e[5] << 16,
                                  e[6] | (uint32_t)e[7] << 16);
            }
        }
    }
}

// Run-entry state for W_c thread `row` (state n): channels p0..p0+63 of
// s0[ids[seq]] (first run) or of the carry kernel's slot (later runs).
__device__ __forceinline__ void load_state_row(const ScanParams& p, const OutTile& ot, int row, float (&v)[64]) {
    const float* src;
    int64_t sc;
    if (ot.tl.run == 0) {
        const int sq = p.has_ids ? p.ids[ot.tl.seq] : ot.tl.seq;
        src = p.s0 + (int64_t)sq * p.seq_s + (int64_t)ot.tl.h * p.s_s0 + (int64_t)ot.p0 * p.s_s1 + row;
        sc = p.s_s1;
    } else {
        src = p.agg + (ot.unit0 + ot.tl.run - 1) * (int64_t)p.P * p.N + (int64_t)ot.p0 * p.N + row;
        sc = p.N;
    }
#pragma unroll
    for (int k = 0; k < 64; ++k) v[k] = k < ot.pw ? src[(int64_t)k * sc] : 0.0f;
}

__device__ __forceinline__ void out_fast(const TcMaps& maps, const CUtensorMap& ymap, int y_tma, const ScanParams& p,
                                         const OutTile& ot, uint8_t* sm, uint32_t tm, uint64_t* cb_bar,
                                         const float (&pre)[64]) {
    float* ring = reinterpret_cast<float*>(sm + OF_V);
    __shared__ FastBars bars;

    HX_PHASE_START;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int row = 32 * (warp & 3) + lane;
    const uint32_t lane_off = (uint32_t)(32 * (warp & 3)) << 16;
    const Tile tl = ot.tl;
    const int p0 = ot.p0, pw = ot.pw, n_ch = ot.n_ch;
    const int t_begin = ot.t_begin, t_end = ot.t_end;

    uint8_t* sS = sm + OF_S;
    auto sCB = [&](int i) { return sm + OO_CB + (uint32_t)(i & 1) * 65536u; };
    auto sXW = [&](int i) { return sm + OF_XW + (uint32_t)(i & 1) * 32768u; };
    auto slot = [&](int i) { return ring + (i % kFRing) * kFVec; };
    auto vpar = [&](int i) { return (uint32_t)((i / kFRing) & 1); };
    auto bpar = [&](int i) { return (uint32_t)((i >> 1) & 1); };  // per-buffer parity of chunk i

    if (tid == 0) {
        for (int k = 0; k < 2; ++k) {
            mbar_init(&bars.xw_ready[k], kXwWarps);
            mbar_init(&bars.xw_free[k], 1);
            mbar_init(&bars.acc1[k], 1);
            mbar_init(&bars.g2[k], 1);
            mbar_init(&bars.d_free[k], 4);
        }
        mbar_init(&bars.m_ready, 4);
        mbar_init(&bars.g4, 1);
        mbar_init(&bars.d4_ready, 4);
        mbar_init(&bars.s_ready, 4);
        mbar_init(&bars.g3, 1);
        for (int k = 0; k < kFRing; ++k) {
            mbar_init(&bars.v_full[k], 1);
            mbar_init(&bars.v_empty[k], 4 + 4 + kXwWarps);  // W_y, W_c, W_xw
        }
        fence_mbar_init();
    }
    __syncthreads();
    bool ok = true;

    if (warp == kWarpMma) {
        // ================= TMA producer + MMA issuer ========================
        if (lane == 0) {
            const uint32_t aS = smem_u32(sS);
            const uint64_t dSm = sdesc_sw128(aS, 16384, 1024);
            // G1 of chunk k -> D1[k & 1].  D1[k & 1] holds the mask of chunk
            // k-2 (W_m packs it in place), read by G2(k-2): wait for that first.
            auto issue_g1 = [&](int k) -> bool {
                if (!mbar_wait(&cb_bar[k & 1], bpar(k), kWaitBudget)) return false;
                if (k >= 2 && !mbar_wait(&bars.g2[k & 1], bpar(k - 2), kWaitBudget)) return false;
                HX_TL(0, k);
                tc_fence_after();
                const uint32_t aC = smem_u32(sCB(k)), aB = aC + 32768;
                const uint64_t dCk = sdesc_sw128(aC, 16, 1024), dBk = sdesc_sw128(aB, 16, 1024);
                const uint32_t tD1 = tm + 128u * (uint32_t)(k & 1);
#pragma unroll
                for (int ks = 0; ks < 8; ++ks)
                    mma_bf16(tD1, desc_add(dCk, kmajor_off(ks)), desc_add(dBk, kmajor_off(ks)), ID_G1, ks > 0);
                mma_commit(&bars.acc1[k & 1]);
                HX_TL(1, k);
                return true;
            };
            HX_PHASE_T(1, kMmaTid);
            if (n_ch > 0) ok = issue_g1(0);
            // Issue order for chunk i: G4(i), G3(i), G1(i+1), G2(i).  G1 runs a
            // chunk ahead so the tensor pipe has queued work while G2(i) waits
            // for the mask of chunk i, and W_m gets a chunk of slack.
            for (int i = 0; i < n_ch && ok; ++i) {
                const int b = i & 1;
                const uint32_t par = (uint32_t)(i & 1);
                const uint32_t aC = smem_u32(sCB(i)), aB = aC + 32768, aX = smem_u32(sXW(i));
                const uint32_t tD = tm + TF_D + 64u * (uint32_t)b;
                const uint64_t dCk = sdesc_sw128(aC, 16, 1024);
                const uint64_t dBm = sdesc_sw128(aB, 16384, 1024), dXm = sdesc_sw128(aX, 16384, 1024);
                // G4 accumulates onto S~_i, which W_c left in D4
                if (!(ok = mbar_wait(&bars.xw_ready[b], bpar(i), kWaitBudget))) break;
                if (!(ok = mbar_wait(&bars.d4_ready, par, kWaitBudget))) break;
                HX_TL(2, i);
                HX_PHASE_T(3, kMmaTid);
                tc_fence_after();
#pragma unroll
                for (int ks = 0; ks < 8; ++ks)
                    mma_bf16(tm + TF_D4, desc_add(dBm, 2048u * ks), desc_add(dXm, 2048u * ks), ID_G4N, 1u);
#pragma unroll
                for (int ks = 0; ks < 8; ++ks)
                    mma_bf16(tm + TF_D4, desc_add(dBm, 2048u * ks), desc_add(dXm, 16384u + 2048u * ks), ID_G4N, 1u);
                mma_commit(&bars.g4);
                HX_TL(3, i);
                if (!(ok = mbar_wait(&bars.s_ready, par, kWaitBudget))) break;
                if (i >= 2) {
                    if (!(ok = mbar_wait(&bars.d_free[b], bpar(i - 2), kWaitBudget))) break;
                }
                HX_TL(4, i);
                HX_PHASE_T(4, kMmaTid);
                tc_fence_after();
#pragma unroll
                for (int ks = 0; ks < 8; ++ks)
                    mma_bf16(tD, desc_add(dCk, kmajor_off(ks)), desc_add(dSm, 2048u * ks), ID_G3, ks > 0);
                mma_commit(&bars.g3);
                HX_TL(5, i);
                if (i + 1 < n_ch && !(ok = issue_g1(i + 1))) break;
                if (!(ok = mbar_wait(&bars.m_ready, par, kWaitBudget))) break;
                HX_TL(6, i);
                HX_PHASE_T(5, kMmaTid);
                tc_fence_after();
#pragma unroll
                for (int ks = 0; ks < 8; ++ks)
                    mma_bf16_ts(tD, tm + 128u * (uint32_t)b + 8u * (uint32_t)ks, desc_add(dXm, 2048u * ks), ID_G2, 1u);
                mma_commit(&bars.g2[b]);
                HX_TL(7, i);
                // G1(i), G4(i) and G3(i) were the last readers of C/B[b]
                if (!(ok = mbar_wait(&bars.g3, par, kWaitBudget))) break;
                if (i + 2 < n_ch) load_cb_chunk(maps, sCB(i + 2), &cb_bar[b], ot.g, t_begin + (i + 2) * kCS, tl.seq);
                HX_TL(8, i);
                HX_PHASE_T(6, kMmaTid);
            }
            if (!ok) {
                atomicCAS(&g_tc_fault, 0u, kFaultMmaOut);
                mbar_wait(&bars.g3, 0, kWaitBudget);
            }
        }
        __syncwarp();
    } else if (warp == kWarpVec) {
        // ================= chunk vectors ====================================
        const float Ah2 = ot.Ah * kLog2e;
        float raw[4] = {pre[0], pre[1], pre[2], pre[3]}, raw_next[4];  // chunk 0 prefetched
        for (int i = 0; i < n_ch && ok; ++i) {
            const int t0 = t_begin + i * kCS;
            if (i + 1 < n_ch) warp_load_dt(p, ot.db, t0 + kCS, t_end, raw_next);
            float v[4], lc[4], total;
            warp_chunk_prefix(p, ot.db, t0, min(kCS, t_end - t0), Ah2, raw, v, lc, &total);
            if (i >= kFRing) {
                if (!(ok = mbar_wait(&bars.v_empty[i % kFRing], vpar(i - kFRing), kWaitBudget))) break;
            }
            float* vs = slot(i);
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const int t = 4 * lane + k;
                vs[t] = v[k] * ex2(total - lc[k]);
                vs[128 + t] = ex2(lc[k] - total);
            }
            if (lane == 0) vs[256] = ex2(total);
            __syncwarp();
            if (lane == 0) mbar_arrive(&bars.v_full[i % kFRing]);
            if (lane == 0) HX_TL(20, i);
#pragma unroll
            for (int k = 0; k < 4; ++k) raw[k] = raw_next[k];
        }
        if (!ok) atomicCAS(&g_tc_fault, 0u, kFaultMmaOut);
    } else if (warp >= kWarpXw) {
        // ================= W_xw: xw = w x, hi | lo ===========================
        const int r = 32 * xw_index(warp) + lane;
        const bool leader = r == 0;
        uint4 cur[kXwVec], nxt[kXwVec];  // chunk 0 was prefetched by the kernel prologue
#pragma unroll
        for (int k = 0; k < kXwVec; ++k)
            cur[k] = make_uint4(__float_as_uint(pre[4 * k]), __float_as_uint(pre[4 * k + 1]),
                                __float_as_uint(pre[4 * k + 2]), __float_as_uint(pre[4 * k + 3]));
        for (int i = 0; i < n_ch; ++i) {
            if (i + 1 < n_ch) load_x_chunk(p, ot, r, i + 1, nxt);
            if (!(ok = group_wait(&bars.v_full[i % kFRing], vpar(i), 5, kXwThreads, leader))) break;
            if (i >= 2) {
                if (!(ok = group_wait(&bars.xw_free[i & 1], bpar(i - 2), 5, kXwThreads, leader))) break;
            }
            if (leader) HX_TL(18, i);
            HX_PHASE_T(7, 32 * 12);
            const float* wv = slot(i);
            uint8_t* xh = sXW(i);
#pragma unroll
            for (int k = 0; k < kXwVec; ++k) {
                const int idx = r + kXwThreads * k, j = idx >> 3, c = idx & 7;
                if (idx < 1024) {
                    const uint32_t off = sw128_off(j, c);
                    const float wj = wv[j];
                    const uint32_t in[4] = {cur[k].x, cur[k].y, cur[k].z, cur[k].w};
                    uint32_t hi[4], lo[4];
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        float a, bb;
                        unpack_bf16x2(in[e], a, bb);
                        a *= wj;
                        bb *= wj;
                        hi[e] = pack_bf16x2(a, bb);
                        float ah, bh;
                        unpack_bf16x2(hi[e], ah, bh);
                        lo[e] = pack_bf16x2(a - ah, bb - bh);
                    }
                    *reinterpret_cast<uint4*>(xh + off) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
                    *reinterpret_cast<uint4*>(xh + 16384 + off) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
                }
            }
            fence_async_smem();
            __syncwarp();
            if (lane == 0) {
                mbar_arrive(&bars.xw_ready[i & 1]);
                mbar_arrive(&bars.v_empty[i % kFRing]);
            }
            if (leader) HX_TL(19, i);
#pragma unroll
            for (int k = 0; k < kXwVec; ++k) cur[k] = nxt[k];
            HX_PHASE_T(8, 32 * 12);
        }
    } else if (warp >= kWarpC) {
        // ================= W_c: the carry, in the G4 accumulator ===========
        const bool leader = tid == 32 * kWarpC;
        const uint32_t tD4 = tm + lane_off + TF_D4;
        // S~ = decay S -> D4 (fp32) and bf16 pairs for the smem copy
        auto scale_store = [&](float (&v)[64], float decay, uint32_t (&sb)[32]) {
#pragma unroll
            for (int q = 0; q < 4; ++q) {
#pragma unroll
                for (int k = 0; k < 16; ++k) v[16 * q + k] *= decay;
                tmem_st16(tD4 + 16 * q, *reinterpret_cast<const uint32_t(*)[16]>(v + 16 * q));
#pragma unroll
                for (int k = 0; k < 8; ++k) sb[8 * q + k] = pack_bf16x2(v[16 * q + 2 * k], v[16 * q + 2 * k + 1]);
            }
            tmem_wait_st();
        };
        auto store_sbf = [&](const uint32_t (&sb)[32]) {
#pragma unroll
            for (int c = 0; c < 8; ++c)
                *reinterpret_cast<uint4*>(sS + sw128_off(row, c)) =
                    make_uint4(sb[4 * c], sb[4 * c + 1], sb[4 * c + 2], sb[4 * c + 3]);
            fence_async_smem();
        };
        // S~_0 from the prefetched run-entry state
        if (n_ch > 0 && (ok = group_wait(&bars.v_full[0], 0u, 4, 128, leader))) {
            float v[64];
#pragma unroll
            for (int k = 0; k < 64; ++k) v[k] = pre[k];
            uint32_t sb[32];
            scale_store(v, slot(0)[256], sb);
            store_sbf(sb);
            tc_fence_before();
            __syncwarp();
            if (lane == 0) {
                mbar_arrive(&bars.d4_ready);
                mbar_arrive(&bars.s_ready);
                mbar_arrive(&bars.v_empty[0]);
            }
        }
        for (int i = 0; i < n_ch && ok; ++i) {
            const bool last = i + 1 == n_ch;
            if (!(ok = group_wait(&bars.g4, (uint32_t)(i & 1), 4, 128, leader))) break;
            float decay = 1.0f;
            if (!last) {
                if (!(ok = group_wait(&bars.v_full[(i + 1) % kFRing], vpar(i + 1), 4, 128, leader))) break;
                decay = slot(i + 1)[256];
            }
            if (leader) HX_TL(11, i);
            HX_PHASE_T(9, 32 * kWarpC);
            tc_fence_after();
            float v[64];  // S_{i+1}
#pragma unroll
            for (int q = 0; q < 4; ++q) tmem_ld16(tD4 + 16 * q, *reinterpret_cast<float(*)[16]>(v + 16 * q));
            tmem_wait_ld();
            if (last) {
                if (tl.run == p.n_runs - 1) {
                    float* s1 = p.s1 + (int64_t)tl.seq * p.seq_s + (int64_t)tl.h * p.s_s0 + (int64_t)p0 * p.s_s1 + row;
#pragma unroll
                    for (int k = 0; k < 64; ++k)
                        if (k < pw) s1[(int64_t)k * p.s_s1] = v[k];
                }
                break;
            }
            uint32_t sb[32];
            scale_store(v, decay, sb);
            tc_fence_before();
            __syncwarp();
            if (lane == 0) {
                mbar_arrive(&bars.d4_ready);
                mbar_arrive(&bars.v_empty[(i + 1) % kFRing]);
            }
            if (leader) HX_TL(12, i);
            // smem S~ is G3(i)'s operand: overwrite it once G3(i) retires
            if (!(ok = group_wait(&bars.g3, (uint32_t)(i & 1), 4, 128, leader))) break;
            if (leader) HX_TL(13, i);
            store_sbf(sb);
            warp_arrive(&bars.s_ready);
            if (leader) HX_TL(14, i);
            HX_PHASE_T(10, 32 * kWarpC);
        }
    } else if (warp >= kWarpM) {
        // ================= W_m: causal mask, bf16 pairs into M =============
        const bool leader = tid == 32 * kWarpM;
        const int qw = warp & 3;
        const int rmax = 32 * qw + 31;  // last row of this lane quarter
        for (int i = 0; i < n_ch; ++i) {
            if (!(ok = group_wait(&bars.acc1[i & 1], bpar(i), 3, 128, leader))) break;
            if (leader) HX_TL(9, i);
            HX_PHASE_T(11, 32 * kWarpM);
            tc_fence_after();
            // The mask goes in place: packed pairs over D1[i&1]'s first 64
            // columns.  Each thread owns its row, and the columns a pass writes
            // (32 half .. +31) were read in this or the previous pass.  Columns
            // are read 64 at a time, and only where some row of this lane
            // quarter needs them.
            const uint32_t src = tm + lane_off + 128u * (uint32_t)(i & 1);
            const uint32_t dst = src;
#pragma unroll
            for (int half = 0; half < 2; ++half) {
                if (64 * half <= rmax) {
                    float d[64];
#pragma unroll
                    for (int g = 0; g < 4; ++g)
                        if (64 * half + 16 * g <= rmax)
                            tmem_ld16(src + 64 * half + 16 * g, *reinterpret_cast<float(*)[16]>(d + 16 * g));
                    tmem_wait_ld();
#pragma unroll
                    for (int h2 = 0; h2 < 2; ++h2) {
                        uint32_t mp[16];
#pragma unroll
                        for (int e2 = 0; e2 < 16; ++e2) {
                            const int e = 16 * h2 + e2;
                            const int j = 64 * half + 2 * e;
                            const bool need = 64 * half + 16 * (e >> 3) <= rmax;
                            mp[e2] = need ? pack_bf16x2(j <= row ? d[2 * e] : 0.0f, j + 1 <= row ? d[2 * e + 1] : 0.0f)
                                          : 0u;
                        }
                        tmem_st16(dst + 32 * half + 16 * h2, mp);
                    }
                } else {
                    const uint32_t z[16] = {};
                    tmem_st16(dst + 32 * half, z);
                    tmem_st16(dst + 32 * half + 16, z);
                }
            }
            tmem_wait_st();
            tc_fence_before();
            warp_arrive(&bars.m_ready);
            if (leader) HX_TL(10, i);
            HX_PHASE_T(12, 32 * kWarpM);
        }
    } else {
        // ================= W_y: y = f_t D ==================================
        // D[i&1] is read whole and released at once; y goes out through the
        // xw buffer of the same chunk (free once G2 retired) and two TMA
        // stores, after which the buffer is handed back to W_xw.
        const bool leader = tid == 0;
        for (int i = 0; i < n_ch; ++i) {
            if (!(ok = group_wait(&bars.g2[i & 1], bpar(i), 2, 128, leader))) break;
            if (!(ok = group_wait(&bars.v_full[i % kFRing], vpar(i), 2, 128, leader))) break;
            if (leader) HX_TL(15, i);
            HX_PHASE(13);
            tc_fence_after();
            const int tp = t_begin + i * kCS;
            const int tlen = t_end - tp;
            const float f = slot(i)[128 + row];
            float a[64];
#pragma unroll
            for (int q = 0; q < 4; ++q)
                tmem_ld16(tm + lane_off + TF_D + 64u * (uint32_t)(i & 1) + 16 * q, *reinterpret_cast<float(*)[16]>(a + 16 * q));
            tmem_wait_ld();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) {
                mbar_arrive(&bars.d_free[i & 1]);
                mbar_arrive(&bars.v_empty[i % kFRing]);
            }
            if (leader) HX_TL(16, i);
            if (y_tma) {
                uint8_t* stg = sXW(i);
#pragma unroll
                for (int c = 0; c < 16; ++c)
                    *reinterpret_cast<float4*>(stg + 16384 * (c >> 3) + sw128_off(row, c & 7)) =
                        make_float4(f * a[4 * c], f * a[4 * c + 1], f * a[4 * c + 2], f * a[4 * c + 3]);
                fence_async_smem();
                named_sync(2, 128);
                if (leader) {
                    tma_store_4d(&ymap, stg, p0, tl.h, tp, tl.seq);
                    if (p0 + 32 < p.P) tma_store_4d(&ymap, stg + 16384, p0 + 32, tl.h, tp, tl.seq);
                    bulk_commit();
                    bulk_wait_read0();  // the staging tiles have been read
                    mbar_arrive(&bars.xw_free[i & 1]);
                    HX_TL(17, i);
                }
            } else {
                if (row < tlen) {
                    float* yr = p.y + (int64_t)tl.seq * p.seq_y + (int64_t)(tp + row) * p.s_y0 +
                                (int64_t)tl.h * p.s_y1 + (int64_t)p0 * p.s_y2;
#pragma unroll
                    for (int k = 0; k < 64; ++k)
                        if (k < pw) yr[(int64_t)k * p.s_y2] = f * a[k];
                }
                if (leader) mbar_arrive(&bars.xw_free[i & 1]);
            }
            HX_PHASE(14);
        }
        if (leader && y_tma) bulk_wait0();  // y stores complete before the CTA exits
    }
}

// ---------------------------------------------------------------------------
// Output kernel entry: shared prologue, then one of the two paths for the
// whole CTA.  The prologue allocates TMEM, starts the C/B loads of chunks 0
// and 1 (same smem layout and barriers in both paths) and, while they fly,
// measures the largest per-chunk decay of the run.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(kOutThreads, 1)
    tc_out_kernel(const __grid_constant__ TcMaps maps, const __grid_constant__ CUtensorMap ymap, ScanParams p,
                  int y_tma, int force_general) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* sm = align1024(smem_raw);
    __shared__ uint64_t cb_bar[2];
    __shared__ uint32_t tmem_base;
    __shared__ unsigned span_bits;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const OutTile ot = out_tile(p);
    if (tid == 0) HX_TL(31, 0);
    if (tid == 0) {
        mbar_init(&cb_bar[0], 1);
        mbar_init(&cb_bar[1], 1);
        span_bits = 0u;
        fence_mbar_init();
    }
    if (warp == kWarpMma) {
        tmem_alloc(&tmem_base, 512);
        tmem_relinquish();
    }
    __syncthreads();
    tc_fence_after();
    if (tid == kMmaTid) {
        prefetch_tmap(&maps.x);
        prefetch_tmap(&maps.b);
        prefetch_tmap(&maps.c);
        if (y_tma) prefetch_tmap(&ymap);
        for (int i = 0; i < 2 && i < ot.n_ch; ++i)
            load_cb_chunk(maps, sm + OO_CB + (uint32_t)i * 65536u, &cb_bar[i], ot.g, ot.t_begin + i * kCS, ot.tl.seq);
    }
    // While the C/B loads fly: W_y and W_m warps measure each chunk's decay
    // span (|A| sum_t dt_t, log2 units, one warp per chunk) and the other
    // fast-path roles prefetch their first inputs into pre[]: the run-entry
    // state (W_c), x of chunk 0 (W_xw), dt of chunk 0 (vector warp).
    float pre[64];
    if (warp < kWarpC) {
        const float aa = fabsf(ot.Ah) * kLog2e;
        float mx = 0.0f;
        for (int c = warp; c < ot.n_ch; c += kWarpC) {
            const int t0 = ot.t_begin + c * kCS;
            float raw[4];
            warp_load_dt(p, ot.db, t0, ot.t_end, raw);
            float sum = 0.0f;
#pragma unroll
            for (int k = 0; k < 4; ++k)
                if (t0 + 4 * lane + k < ot.t_end) sum += dt_of(raw[k], p.dt_min, p.dt_max);
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
            mx = fmaxf(mx, sum * aa);
        }
        if (lane == 0 && mx > 0.0f) atomicMax(&span_bits, __float_as_uint(mx));
    } else if (warp < kWarpXw) {
        load_state_row(p, ot, 32 * (warp & 3) + lane, pre);
    } else if (warp != kWarpMma && warp != kWarpVec) {
        uint4 v[kXwVec];
        load_x_chunk(p, ot, 32 * xw_index(warp) + lane, 0, v);
#pragma unroll
        for (int k = 0; k < kXwVec; ++k) {
            pre[4 * k] = __uint_as_float(v[k].x);
            pre[4 * k + 1] = __uint_as_float(v[k].y);
            pre[4 * k + 2] = __uint_as_float(v[k].z);
            pre[4 * k + 3] = __uint_as_float(v[k].w);
        }
    } else if (warp == kWarpVec) {
        float raw[4];
        warp_load_dt(p, ot.db, ot.t_begin, ot.t_end, raw);
#pragma unroll
        for (int k = 0; k < 4; ++k) pre[k] = raw[k];
    }
    __syncthreads();
    if (tid == 0) HX_TL(31, 1);
    const uint32_t tm = tmem_base;
    if (!force_general && __uint_as_float(span_bits) <= kFastSpan2)
        out_fast(maps, ymap, y_tma, p, ot, sm, tm, cb_bar, pre);
    else
        out_general(maps, p, ot, sm, tm, cb_bar);
    tc_fence_before();
    __syncthreads();
    if (warp == kWarpMma) {
        tc_fence_after();
        tmem_dealloc(tm, 512);
    }
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
// State kernel: the run's state from a zero start, G4 accumulated over the
// whole run in one TMEM accumulator, plus the run's log-decay.  Sized for two
// CTAs per SM (107 KB of shared memory, 128 TMEM columns, 320 threads): the
// two CTAs hide each other's latencies.  It streams in 64-token steps (half
// chunks), which buys three-deep rings for B and x and two xw buffers within
// that budget, so no load latency sits on the MMA chain.
//
//   warps 0-7  (256)  xw = w x as bf16 hi | lo from the x ring
//   warp 8  (lane 0)  TMA producer (B and x, 3 stages each) and MMA issuer:
//                     per step four 128 x 128 x 16 MMAs, A = B (MN-major),
//                     B = [xw_hi | xw_lo] (MN-major)
//   warp 9            decay weights w_j = dt_j exp(sum_{i>j in run} A dt_i)
//                     per 128-token chunk into a 4-slot ring
//
// Chunks are visited last to first so the decay from token j to the end of
// the run is a sum of same-sign terms.
// ---------------------------------------------------------------------------
constexpr int kStEpi = 256;
constexpr int kStThreads = kStEpi + 64;
constexpr int kStHalf = 64;                            // tokens per step
constexpr int kStStages = 3;
constexpr int kStRing = 4;
constexpr uint32_t SO_B = 0;                           // 3 x 16 KB: B rows of one step, states 0-63 | 64-127
constexpr uint32_t SO_X = SO_B + kStStages * 16384;    // 3 x 8 KB: x rows of one step
constexpr uint32_t SO_XW = SO_X + kStStages * 8192;    // 2 x (hi 8 KB | lo 8 KB)
constexpr uint32_t SO_W = SO_XW + 2 * 16384;           // kStRing x 128 weights
constexpr uint32_t SMEM_STATE = SO_W + kStRing * 512 + 1024;

struct StBars {
    uint64_t b_full[kStStages], b_done[kStStages], x_full[kStStages], xw_full[2], xw_empty[2];
    uint64_t w_full[kStRing], w_empty[kStRing];
};

__device__ __forceinline__ bool st_wait(uint64_t* bar, uint32_t parity, unsigned code) {
    const bool ok = mbar_wait(bar, parity, kWaitBudget);
    const bool all = named_and(1, kStEpi, ok);
    if (!all && threadIdx.x == 0) atomicCAS(&g_tc_fault, 0u, code);
    return all;
}

__global__ void __launch_bounds__(kStThreads, 2) tc_state_kernel(const __grid_constant__ TcMaps maps, ScanParams p,
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
    const int n_st = 2 * n_ch;  // steps; a step past t_end reads zeros
    const int64_t db = (int64_t)tl.seq * p.seq_dt + (int64_t)tl.h * p.s_dt1;
    auto t0_of = [&](int q) { return t_begin + (n_ch - 1 - q) * kCS; };       // visit order q -> chunk
    auto ts_of = [&](int s) { return t0_of(s >> 1) + (s & 1) * kStHalf; };    // step s -> first token
    auto sB = [&](int s) { return sm + SO_B + (uint32_t)(s % kStStages) * 16384u; };
    auto sX = [&](int s) { return sm + SO_X + (uint32_t)(s % kStStages) * 8192u; };
    auto sXW = [&](int s) { return sm + SO_XW + (uint32_t)(s & 1) * 16384u; };

    if (tid == 0) {
        for (int k = 0; k < kStStages; ++k) {
            mbar_init(&bars.b_full[k], 1);
            mbar_init(&bars.b_done[k], 1);
            mbar_init(&bars.x_full[k], 1);
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
        tmem_alloc(&tmem_base, 128);
        tmem_relinquish();
    }
    __syncthreads();
    tc_fence_after();
    const uint32_t tm = tmem_base;

    auto load_b = [&](int s) {
        uint64_t* bar = &bars.b_full[s % kStStages];
        mbar_expect_tx(bar, 2 * 8192);
        tma_load_4d(sB(s), &maps.b, bar, 0, g, ts_of(s), tl.seq);
        tma_load_4d(sB(s) + 8192, &maps.b, bar, 64, g, ts_of(s), tl.seq);
    };
    auto load_x = [&](int s) {
        uint64_t* bar = &bars.x_full[s % kStStages];
        mbar_expect_tx(bar, 8192);
        tma_load_4d(sX(s), &maps.x, bar, p0, tl.h, ts_of(s), tl.seq);
    };

    bool ok = true;
    if (is_mma) {
        if ((tid & 31) == 0) {
            prefetch_tmap(&maps.b);
            prefetch_tmap(&maps.x);
            for (int s = 0; s < kStStages && s < n_st; ++s) {
                load_b(s);
                load_x(s);
            }
            HX_PHASE_T(16, 256);
            for (int s = 0; s < n_st && ok; ++s) {
                const int st = s % kStStages;
                const uint32_t pf = (uint32_t)((s / kStStages) & 1);
                if (!(ok = mbar_wait(&bars.b_full[st], pf, kWaitBudget))) break;
                HX_PHASE_T(17, 256);
                if (!(ok = mbar_wait(&bars.xw_full[s & 1], (uint32_t)((s >> 1) & 1), kWaitBudget))) break;
                HX_PHASE_T(18, 256);
                tc_fence_after();
                // A = B rows of the step (M = 128 states in two 64-state atoms),
                // B = [xw_hi | xw_lo] (N = 128 in two atoms), K = 64 tokens
                const uint64_t dA = sdesc_sw128(smem_u32(sB(s)), 8192, 1024);
                const uint64_t dX = sdesc_sw128(smem_u32(sXW(s)), 8192, 1024);
#pragma unroll
                for (int ks = 0; ks < 4; ++ks)
                    mma_bf16(tm, desc_add(dA, 2048u * ks), desc_add(dX, 2048u * ks), ID_G4W, (s > 0 || ks > 0) ? 1u : 0u);
                mma_commit(&bars.xw_empty[s & 1]);
                mma_commit(&bars.b_done[st]);
                HX_PHASE_T(19, 256);
                if (s + kStStages < n_st) {
                    // the builders consumed x(s) before xw_full; B(s) is free once
                    // these MMAs retire
                    load_x(s + kStStages);
                    if (!(ok = mbar_wait(&bars.b_done[st], pf, kWaitBudget))) break;
                    load_b(s + kStStages);
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
        // ---- xw builders: two 16-byte x vectors per thread per step -------
        HX_PHASE(21);
        for (int s = 0; s < n_st; ++s) {
            const int q = s >> 1, slot = q % kStRing;
            if ((s & 1) == 0) {
                if (!(ok = st_wait(&bars.w_full[slot], (uint32_t)((q / kStRing) & 1), kFaultMmaState))) break;
            }
            HX_PHASE(22);
            if (!(ok = st_wait(&bars.x_full[s % kStStages], (uint32_t)((s / kStStages) & 1), kFaultTmaState))) break;
            if (s >= 2) {  // xw buffer s & 1 was last read by step s - 2
                if (!(ok = st_wait(&bars.xw_empty[s & 1], (uint32_t)(((s - 2) >> 1) & 1), kFaultMmaState))) break;
            }
            HX_PHASE(23);
            const float* wv = wring + slot * 128 + (s & 1) * kStHalf;
            const uint8_t* x = sX(s);
            uint8_t* xh = sXW(s);
#pragma unroll
            for (int k = 0; k < 2; ++k) {
                const int i = tid + kStEpi * k;
                const int j = i >> 3, c = i & 7;
                const uint32_t off = sw128_off(j, c);
                const float wj = wv[j];
                const uint4 xr = *reinterpret_cast<const uint4*>(x + off);
                const uint32_t in[4] = {xr.x, xr.y, xr.z, xr.w};
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
                *reinterpret_cast<uint4*>(xh + off) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
                *reinterpret_cast<uint4*>(xh + 8192 + off) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
            }
            fence_async_smem();
            __syncwarp();
            if ((tid & 31) == 0) {
                mbar_arrive(&bars.xw_full[s & 1]);
                if (s & 1) mbar_arrive(&bars.w_empty[slot]);
            }
            HX_PHASE(25);
        }
        // all G4 MMAs retired: the last step's commit
        if (ok && n_st > 0)
            ok = st_wait(&bars.xw_empty[(n_st - 1) & 1], (uint32_t)(((n_st - 1) >> 1) & 1), kFaultMmaState);
        tc_fence_after();
        if (ok) {
            const int64_t unit = ((int64_t)tl.seq * p.H + tl.h) * p.n_runs + tl.run;
            float* out = p.agg + unit * (int64_t)p.P * p.N + (int64_t)p0 * p.N + row;
            // columns 0..63 hold the hi part, 64..127 the lo part
#pragma unroll
            for (int h2 = 0; h2 < 2; ++h2) {
                float hi[16], lo[16];
                tmem_ld16(tm + lane_off + 32 * wg + 16 * h2, hi);
                tmem_ld16(tm + lane_off + 64 + 32 * wg + 16 * h2, lo);
                tmem_wait_ld();
#pragma unroll
                for (int e = 0; e < 16; ++e) {
                    const int c = 32 * wg + 16 * h2 + e;
                    if (c < pw) out[(int64_t)c * p.N] = hi[e] + lo[e];
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (ok && tid == 0 && tl.slab == 0)
        p.lam[((int64_t)tl.seq * p.H + tl.h) * p.n_runs + tl.run] = lam_total;
    if (is_mma) {
        tc_fence_after();
        tmem_dealloc(tm, 128);
    }
    HX_PHASE(26);
}

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------
using EncodeFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                              const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                              CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

// 4-D bf16 map (inner, d1, tok, seq) with a 64 x 1 x box_tok x 1 box,
// 128-byte swizzle.  Coordinates past the extents read as zero.
bool make_map(EncodeFn fn, CUtensorMap* m, const void* base, int64_t inner, int64_t d1, int64_t tok, int64_t seq,
              int64_t s1, int64_t s_tok, int64_t s_seq, int box_tok = kCS) {
    cuuint64_t dims[4] = {(cuuint64_t)inner, (cuuint64_t)d1, (cuuint64_t)tok, (cuuint64_t)seq};
    cuuint64_t strides[3] = {(cuuint64_t)(s1 * 2), (cuuint64_t)(s_tok * 2), (cuuint64_t)(s_seq * 2)};
    cuuint32_t box[4] = {64, 1, (cuuint32_t)box_tok, 1};
    cuuint32_t es[4] = {1, 1, 1, 1};
    return fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(base), dims, strides, box, es,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// 4-D f32 map (chan, head, tok, seq) for TMA stores of y, box 32 x 1 x 128 x 1,
// 128-byte swizzle.  Rows past L and channels past P are not written.
bool make_ymap(EncodeFn fn, CUtensorMap* m, void* base, const ScanParams& p) {
    cuuint64_t dims[4] = {(cuuint64_t)p.P, (cuuint64_t)p.H, (cuuint64_t)p.L, (cuuint64_t)p.S};
    cuuint64_t strides[3] = {(cuuint64_t)(p.s_y1 * 4), (cuuint64_t)(p.s_y0 * 4), (cuuint64_t)(p.seq_y * 4)};
    cuuint32_t box[4] = {32, 1, (cuuint32_t)kCS, 1};
    cuuint32_t es[4] = {1, 1, 1, 1};
    return fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, base, dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
              CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// TMA stores of y need unit channel stride, 16-byte multiples for the other
// strides and a 16-byte aligned base.
// Maps of the state kernel: x and B in 64-token boxes (its step).
bool make_state_maps(EncodeFn fn, TcMaps* m, const ScanParams& p) {
    const int64_t S = p.S;
    std::memset(&m->c, 0, sizeof(m->c));
    return make_map(fn, &m->x, p.x, p.P, p.H, p.L, S, p.s_x1, p.s_x0, p.seq_x, kStHalf) &&
           make_map(fn, &m->b, p.B, p.N, p.G, p.L, S, p.s_b1, p.s_b0, p.seq_b, kStHalf);
}

bool y_tma_ok(const ScanParams& p) {
    if (p.s_y2 != 1) return false;
    const int64_t st[3] = {p.s_y1, p.s_y0, p.seq_y};
    for (int64_t s : st)
        if (s <= 0 || (s * 4) % 16 != 0) return false;
    return (reinterpret_cast<uintptr_t>(p.y) & 15) == 0;
}

// Test hook: HELIX_TC_GENERAL=1 sends every CTA of the output kernel down
// the general path, so tests can cover it on inputs the fast path accepts.
int force_general() {
    const char* e = std::getenv("HELIX_TC_GENERAL");
    return e && *e && *e != '0';
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
        TcMaps smaps;
        if (!make_state_maps(fn, &smaps, p)) return cudaErrorInvalidValue;
        tc_state_kernel<<<(unsigned)(per_run * runs), kStThreads, SMEM_STATE, st>>>(smaps, p, runs);
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
        tc_out_kernel<<<(unsigned)(per_run * pl.n_runs), kOutThreads, SMEM_OUT, st>>>(maps, ymap, p, y_tma, force_general());
        const cudaError_t e = cudaGetLastError();
        if (e != cudaSuccess) return e;
    }
    return cudaSuccess;
}

int launch_tc_states(const helix_ctx* ctx, const Plan& pl, const ScanParams& p, void* stream) {
    auto fn = reinterpret_cast<EncodeFn>(ctx->encode_tiled);
    if (!fn) return cudaErrorNotSupported;
    TcMaps maps;
    const int64_t S = p.S;
    if (!make_state_maps(fn, &maps, p)) return cudaErrorInvalidValue;
    const int64_t per_run = (int64_t)p.n_pslab * p.H * S;
    tc_state_kernel<<<(unsigned)(per_run * pl.n_runs), kStThreads, SMEM_STATE, static_cast<cudaStream_t>(stream)>>>(
        maps, p, pl.n_runs);
    return cudaGetLastError();
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
