// scan_tc3.cu -- tcgen05 kernel family at fp32-class accuracy for F32-stored
// x, B and C (compute_dtype F32, backend AUTO or SGMMA: the reference's fp32
// matrix path, src/kernels/helix_scan_multipass.metal:51-149, 225-361).
//
// Every fp32 operand u is carried as a pair of bf16, hi = bf16(u) and
// lo = bf16(u - hi) (hi + lo holds u to about 16 significant bits), and every
// product as three bf16 MMAs accumulated in fp32:
//
//   a . b  ~  a_hi . b_hi + a_hi . b_lo + a_lo . b_hi
//
// (the bf16x3 scheme of Henry, Tang and Heinecke, "Leveraging the bfloat16
// artificial intelligence datatype for higher-precision computations",
// ARITH 2019).  The dropped terms are of order 2^-16 of the product, so the
// scan lands near 1e-5 relative L2 against the fp64 oracle, an order below
// the 1e-4 bar of the fp32 path, at tensor-core speed.  B and C reach the
// kernels as hi and lo copies made by the cast kernel (scan_cast.cu); x is
// read as stored, fp32, by TMA and split on chip, like the mask, the carried
// state and the G4 operand.
//
// Same run/span decomposition as the bf16 family (runtime/internal.h): the
// state kernel (scan_tc.cu, tc_state_kernel<true>) reduces the runs before
// the last span, the carry kernel turns them into span-entry states, and
// tc3_out_kernel walks one span of one 64-channel slab per CTA.  Per chunk of
// 128 tokens, with Lc the inclusive prefix of A dt inside the chunk:
//
//   G1  D1[t][j]  = C_t . B_j                         A = C (K-major)    B = B (K-major)
//       M[t][j]   = D1 exp(Lc_t - Lc_j) dt_j, j <= t  (into TMEM, hi | lo)
//   G3  D3[t][p]  = C_t . S[:, p]                     A = C (K-major)    B = S (MN-major)
//   G4  D4[n][p]  = sum_j B'_j[n] x_j[p]              A = B'^T (MN-major) B = x (MN-major)
//       with B'_j = dt_j exp(Lc_end - Lc_j) B_j, made in place over B once G1 has read it
//   G2  D2[t][p]  = sum_j M[t][j] x_j[p]              A = M (TMEM)       B = x (MN-major)
//   y_t = D2 + exp(Lc_t) D3;   S_next = exp(Lc_end) S + D4
//
// Every exponent is <= 0 except the in-group factor of the split mask
// (bounded, see the vector warp), so no decay span needs a second path.
// Each GEMM is three passes of eight 128 x N x 16 MMAs.
//
// Warps (22, 88 registers per thread):
//   0-3    W_y   y = D2 + e^Lc D3 -> global (one token row per thread)
//   4-7    W_m   M from D1 -> TMEM, tokens j 0-63 of each row (one row per thread)
//   16-19  W_m   the same, tokens j 64-127
//   8-11   W_c   S_next in TMEM (fp32) and its hi | lo copy in smem for G3;
//                then x(i+1): fp32 through a 64-token staging buffer (its
//                own TMA loads) into the x hi | lo tiles
//   12-15  W_b   half of B' = w B (in place, re-split into hi | lo)
//   0-3    W_y   also the other half of B', before its y
//   20     TMA producer (C, B) and MMA issuer (lane 0)
//   21     chunk vectors (dt, Lc, w, split decays) into a 3-slot ring
// (two warps of every role but W_y's share each SM sub-partition with warps
// of other roles, so a role's work on the critical path is spread over all
// four issue units).
//
// MMA issue order per chunk: G1, G3, then G4 and G2 in whichever order their
// operands (B', M) are ready; C(i+1) loads once G3 retired, B(i+1) once G4
// retired, and x(i+1) is converted once G4 and G2 retired (one buffer each).
//
// TMEM columns: D1 0-127 | M hi 128-191 | M lo 192-255 | D2 256-319 |
//               D3 320-383 | D4 384-447 | S 448-511.
// smem: C hi|lo 64 KB | B hi|lo 64 KB | x hi|lo 32 KB | S hi|lo 32 KB |
//       x staging 16 KB | ring.
//
// Every wait is bounded; an expired wait records a fault code in the device
// word (helix_device_fault), the CTA lets issued MMAs land, frees its TMEM
// and returns.
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdlib>
#include <cstring>

#include "common.cuh"
#include "tc_shared.cuh"
#include "umma.cuh"

namespace hx {
namespace {

using namespace umma;
using namespace tc;

constexpr int k3Warps = 22;
constexpr int k3Threads = 32 * k3Warps;
constexpr int k3WarpMma = 20, k3WarpVec = 21;
enum Role3 : int { kR3Y = 0, kR3M = 1, kR3C = 2, kR3B = 3, kR3Other = 4 };
__host__ __device__ constexpr int role3_of(int warp) { return warp < 16 ? warp >> 2 : warp < 20 ? kR3M : kR3Other; }
__host__ __device__ constexpr int role3_threads(int role) { return role == kR3M ? 256 : 128; }
constexpr int k3BThreads = 256;  // W_b and W_c scale B' together

constexpr int k3Ring = 3;
constexpr int k3Vec = 4 * 128 + 16;  // floats per ring slot: dt | Lc | w | split dt | flag
constexpr uint32_t O3_C = 0;          // C hi (two 64-state atoms) | C lo
constexpr uint32_t O3_B = 65536;      // B hi | B lo (B' after the scaling)
constexpr uint32_t O3_X = 131072;     // x hi | x lo
constexpr uint32_t O3_S = 163840;     // S hi | S lo ([n][p])
constexpr uint32_t O3_XS = 196608;    // fp32 x staging, 64 tokens x 64 channels
constexpr uint32_t O3_V = 212992;     // chunk-vector ring
constexpr uint32_t O3_DT = O3_V + k3Ring * k3Vec * 4;  // vector warp's raw dt ring, 4 x 128 floats
constexpr uint32_t SMEM_3 = O3_DT + 4 * 512 + 1024;
static_assert(SMEM_3 <= 232448, "fits one CTA per SM");

constexpr uint32_t T3_D1 = 0, T3_MH = 128, T3_ML = 192, T3_D2 = 256, T3_D3 = 320, T3_D4 = 384, T3_S = 448;

constexpr uint32_t ID3_KK = idesc_bf16(128, 128, false, false);  // G1
constexpr uint32_t ID3_KM = idesc_bf16(128, 64, false, true);    // G3, G2 (A from TMEM is K-major)
constexpr uint32_t ID3_MM = idesc_bf16(128, 64, true, true);     // G4
constexpr float kSplitSpan2 = 20.0f * kLog2e;                    // in-group span of the split mask

struct Bars3 {
    uint64_t c_full, b_full;           // TMA arrivals, one phase per chunk
    uint64_t xs_full;                  // TMA arrivals, one phase per 64-token half of x
    uint64_t x_full;                   // W_c: x hi | lo tiles written
    uint64_t acc1, g3, g4, g2;         // MMA commits: G1, G3, G4, G2 of a chunk retired
    uint64_t d1_read, m_ready;         // W_m: D1 read, M written
    uint64_t b_ready;                  // W_b: B' written
    uint64_t s_ready, d4_read;         // W_c: S written to smem, D4 read
    uint64_t d_free;                   // W_y: D2, D3 read
    uint64_t fin;                      // drain after a fault
    uint64_t v_full[k3Ring], v_empty[k3Ring];
};

// Bounded wait by all threads of one role, agreed by a vote on the role's
// named barrier (ids 1-4), so the role leaves together.
__device__ __forceinline__ bool role3_wait(const ScanParams& p, uint64_t* bar, uint32_t parity, int role,
                                           unsigned code) {
    const bool ok = mbar_wait(bar, parity, kWaitBudget);
    const bool all = named_and(1 + role, role3_threads(role), ok);
    if (!all && p.fault && (threadIdx.x & 127) == 0 && (threadIdx.x >> 5) < 16) atomicCAS(p.fault, 0u, code);
    return all;
}

// B' = w B of one chunk, in place over the B stage (hi | lo, two 64-state
// atoms each): thread r of the 256 scaling threads takes every 256th of the
// 2048 sixteen-byte chunk positions (atom q >> 10, token row (q >> 3) & 127,
// chunk q & 7), so each quarter warp covers one 128-byte row.
__device__ __forceinline__ void scale_b(uint8_t* bh, const float* wv, int r) {
#pragma unroll 4
    for (int k = 0; k < 2048 / k3BThreads; ++k) {
        const int q = r + k3BThreads * k;
        const int j = (q >> 3) & 127;
        const uint32_t off = (uint32_t)(q >> 10) * 16384u + sw128_off(j, q & 7);
        const float wj = wv[j];
        uint4 hi, lo;
        split_xw8_x3(*reinterpret_cast<const uint4*>(bh + off), *reinterpret_cast<const uint4*>(bh + 32768 + off),
                     f2_of(wj, wj), hi, lo);
        *reinterpret_cast<uint4*>(bh + off) = hi;
        *reinterpret_cast<uint4*>(bh + 32768 + off) = lo;
    }
    fence_async_smem();
}
__device__ __forceinline__ void warp_arrive3(uint64_t* bar) {
    __syncwarp();
    if ((threadIdx.x & 31) == 0) mbar_arrive(bar);
}

// bf16 hi and lo of 2 x 8 floats, packed two per word (element 2c low).
__device__ __forceinline__ void split16(const float (&m)[16], uint32_t (&hi)[8], uint32_t (&lo)[8]) {
#pragma unroll
    for (int e = 0; e < 8; ++e) {
        hi[e] = pack_bf16x2(m[2 * e], m[2 * e + 1]);
        float h0, h1;
        unpack_bf16x2(hi[e], h0, h1);
        lo[e] = pack_bf16x2(m[2 * e] - h0, m[2 * e + 1] - h1);
    }
}

__global__ void __launch_bounds__(k3Threads, 1) tc3_out_kernel(const __grid_constant__ TcMaps maps, ScanParams p) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* sm = align1024(smem_raw);
    __shared__ Bars3 bars;
    __shared__ uint32_t tmem_base;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int role = role3_of(warp);
    const int row = 32 * (warp & 3) + lane;
    const uint32_t lane_off = (uint32_t)(32 * (warp & 3)) << 16;

    // tile: slab fastest, then head, span, sequence (the heads of a group
    // run side by side and share C and B in L2)
    const Tile tl = decode_tile((int)blockIdx.x, p.n_pslab, p.H, p.n_out);
    const int span = tl.run;
    const int p0 = tl.slab * kSlab, pw = min(kSlab, p.P - p0);
    const int g = tl.h / p.hpg;
    const float Ah = p.A[(int64_t)tl.h * p.s_a];
    const int run0 = span * p.out_k;
    const bool last = span == p.n_out - 1;
    const int t_begin = run0 * p.run_tok;
    const int t_end = min(p.L, t_begin + p.out_k * p.run_tok);
    const int n_ch = (t_end - t_begin + kCS - 1) / kCS;
    const int64_t db = (int64_t)tl.seq * p.seq_dt + (int64_t)tl.h * p.s_dt1;
    const int64_t unit0 = ((int64_t)tl.seq * p.H + tl.h) * p.run_slots;
    float* ring = reinterpret_cast<float*>(sm + O3_V);
    auto slot = [&](int i) { return ring + (i % k3Ring) * k3Vec; };

    grid_dep_launch();  // a second 128-state pass may start its prologue
    if (tid == 0) {
        mbar_init(&bars.c_full, 1);
        mbar_init(&bars.b_full, 1);
        mbar_init(&bars.xs_full, 1);
        mbar_init(&bars.x_full, 4);
        mbar_init(&bars.acc1, 1);
        mbar_init(&bars.g3, 1);
        mbar_init(&bars.g4, 1);
        mbar_init(&bars.g2, 1);
        mbar_init(&bars.fin, 1);
        mbar_init(&bars.d1_read, 8);
        mbar_init(&bars.m_ready, 8);
        mbar_init(&bars.b_ready, 8);
        mbar_init(&bars.s_ready, 4);
        mbar_init(&bars.d4_read, 4);
        mbar_init(&bars.d_free, 4);
        for (int k = 0; k < k3Ring; ++k) {
            mbar_init(&bars.v_full[k], 1);
            mbar_init(&bars.v_empty[k], 20);
        }
        fence_mbar_init();
    }
    if (warp == k3WarpMma) {
        tmem_alloc(&tmem_base, 512);
        tmem_relinquish();
    }
    __syncthreads();
    tc_fence_after();
    const uint32_t tm = tmem_base;
    bool ok = true;

    if (warp == k3WarpMma) {
        // ================= TMA producer + MMA issuer ========================
        if (lane == 0) {
            const int nb = p.n_base;
            auto load_c = [&](int i) {
                const int t0 = t_begin + i * kCS;
                mbar_expect_tx(&bars.c_full, 4 * 16384);
                tma_load_4d(sm + O3_C, &maps.c, &bars.c_full, nb, g, t0, tl.seq);
                tma_load_4d(sm + O3_C + 16384, &maps.c, &bars.c_full, nb + 64, g, t0, tl.seq);
                tma_load_4d(sm + O3_C + 32768, &maps.cl, &bars.c_full, nb, g, t0, tl.seq);
                tma_load_4d(sm + O3_C + 49152, &maps.cl, &bars.c_full, nb + 64, g, t0, tl.seq);
            };
            auto load_b = [&](int i) {
                const int t0 = t_begin + i * kCS;
                mbar_expect_tx(&bars.b_full, 4 * 16384);
                tma_load_4d(sm + O3_B, &maps.b, &bars.b_full, nb, g, t0, tl.seq);
                tma_load_4d(sm + O3_B + 16384, &maps.b, &bars.b_full, nb + 64, g, t0, tl.seq);
                tma_load_4d(sm + O3_B + 32768, &maps.bl, &bars.b_full, nb, g, t0, tl.seq);
                tma_load_4d(sm + O3_B + 49152, &maps.bl, &bars.b_full, nb + 64, g, t0, tl.seq);
            };
            prefetch_tmap(&maps.c);
            prefetch_tmap(&maps.cl);
            prefetch_tmap(&maps.b);
            prefetch_tmap(&maps.bl);
            if (n_ch > 0) {
                load_c(0);
                load_b(0);
            }
            const uint32_t aC = smem_u32(sm + O3_C), aB = smem_u32(sm + O3_B);
            const uint32_t aX = smem_u32(sm + O3_X), aS = smem_u32(sm + O3_S);
            auto wait = [&](uint64_t* bar, uint32_t par) { return mbar_wait(bar, par, kWaitBudget); };
            for (int i = 0; i < n_ch && ok; ++i) {
                const uint32_t par = (uint32_t)(i & 1);
                // ---- G1(i): D1 = C B^T -------------------------------------
                if (!(ok = wait(&bars.c_full, par) && wait(&bars.b_full, par))) break;
                if (i > 0 && !(ok = wait(&bars.d1_read, par ^ 1u))) break;
                tc_fence_after();
#pragma unroll
                for (int pass = 0; pass < 3; ++pass) {
                    const uint32_t a = aC + (pass == 2 ? 32768u : 0u), b = aB + (pass == 1 ? 32768u : 0u);
#pragma unroll
                    for (int ks = 0; ks < 8; ++ks)
                        mma_bf16(tm + T3_D1, desc_kmajor(a, ks), desc_kmajor(b, ks), ID3_KK, (pass | ks) != 0);
                }
                mma_commit(&bars.acc1);
                // ---- G3(i): D3 = C S_i -------------------------------------
                if (!(ok = wait(&bars.s_ready, par))) break;
                if (i > 0 && !(ok = wait(&bars.d_free, par ^ 1u))) break;
                tc_fence_after();
#pragma unroll
                for (int pass = 0; pass < 3; ++pass) {
                    const uint32_t a = aC + (pass == 2 ? 32768u : 0u), b = aS + (pass == 1 ? 16384u : 0u);
#pragma unroll
                    for (int ks = 0; ks < 8; ++ks)
                        mma_bf16(tm + T3_D3, desc_kmajor(a, ks), desc_mnmajor(b, ks), ID3_KM, (pass | ks) != 0);
                }
                mma_commit(&bars.g3);
                // ---- then, each as soon as it can go: G4(i) (B' ready), G2(i)
                // (M ready), and C(i+1) into the C stage once G3(i) retired
                if (!(ok = wait(&bars.x_full, par))) break;
                if (i > 0 && !(ok = wait(&bars.d4_read, par ^ 1u))) break;
                const bool more = i + 1 < n_ch;
                bool g4_done = false, g2_done = false, c_next = !more;
                const long long t_start = clock64();
                while (!(g4_done && g2_done && c_next)) {
                    if (!g4_done && mbar_try_wait(&bars.b_ready, par)) {
                        // D4 = B'^T x
                        tc_fence_after();
#pragma unroll
                        for (int pass = 0; pass < 3; ++pass) {
                            const uint32_t a = aB + (pass == 2 ? 32768u : 0u), b = aX + (pass == 1 ? 16384u : 0u);
#pragma unroll
                            for (int ks = 0; ks < 8; ++ks)
                                mma_bf16(tm + T3_D4, desc_mnmajor(a, ks), desc_mnmajor(b, ks), ID3_MM, (pass | ks) != 0);
                        }
                        mma_commit(&bars.g4);
                        g4_done = true;
                    }
                    if (!g2_done && mbar_try_wait(&bars.m_ready, par)) {
                        // D2 = M x
                        tc_fence_after();
#pragma unroll
                        for (int pass = 0; pass < 3; ++pass) {
                            const uint32_t a = tm + (pass == 2 ? T3_ML : T3_MH), b = aX + (pass == 1 ? 16384u : 0u);
#pragma unroll
                            for (int ks = 0; ks < 8; ++ks)
                                mma_bf16_ts(tm + T3_D2, a + 8 * ks, desc_mnmajor(b, ks), ID3_KM, (pass | ks) != 0);
                        }
                        mma_commit(&bars.g2);
                        g2_done = true;
                    }
                    if (!c_next && mbar_try_wait(&bars.g3, par)) {
                        load_c(i + 1);
                        c_next = true;
                    }
                    if (clock64() - t_start > kWaitBudget) break;
                }
                if (!(ok = g4_done && g2_done && c_next)) break;
                // ---- B(i+1) once G4(i) retired
                if (more) {
                    if (!(ok = wait(&bars.g4, par))) break;
                    load_b(i + 1);
                }
            }
            if (!ok) {
                if (p.fault) atomicCAS(p.fault, 0u, kFaultMmaOut);
                // every issued MMA retired before the tensor memory is freed
                mma_commit(&bars.fin);
                mbar_wait(&bars.fin, 0u, kWaitBudget);
            }
        }
        __syncwarp();
    } else if (warp == k3WarpVec) {
        // ================= chunk vectors ====================================
        // raw dt (token-major loads, far apart: several us under load) runs
        // three chunks ahead through a private shared-memory ring; the first
        // three chunks' loads go out together
        const float Ah2 = Ah * kLog2e;
        float* dtr = reinterpret_cast<float*>(sm + O3_DT);
        auto park = [&](int c, const float (&r)[4]) {
#pragma unroll
            for (int k = 0; k < 4; ++k) dtr[(c & 3) * 128 + 4 * lane + k] = r[k];
        };
        {
            float r[3][4];
#pragma unroll
            for (int c = 0; c < 3; ++c) warp_load_dt(p, db, t_begin + min(c, max(n_ch - 1, 0)) * kCS, t_end, r[c]);
#pragma unroll
            for (int c = 0; c < 3; ++c) park(c, r[c]);
        }
        __syncwarp();
        for (int i = 0; i < n_ch && ok; ++i) {
            const int t0 = t_begin + i * kCS;
            float nx[4];
            const bool more = i + 3 < n_ch;
            if (more) warp_load_dt(p, db, t0 + 3 * kCS, t_end, nx);
            const float raw[4] = {dtr[(i & 3) * 128 + 4 * lane], dtr[(i & 3) * 128 + 4 * lane + 1],
                                  dtr[(i & 3) * 128 + 4 * lane + 2], dtr[(i & 3) * 128 + 4 * lane + 3]};
            float v[4], pre[4], total;
            warp_chunk_prefix(p, db, t0, min(kCS, t_end - t0), Ah2, raw, v, pre, &total);
            if (i >= k3Ring) {
                const bool w = mbar_wait(&bars.v_empty[i % k3Ring], (uint32_t)(((i - k3Ring) / k3Ring) & 1), kWaitBudget);
                if (!(ok = __all_sync(0xffffffffu, w))) break;
            }
            float* vs = slot(i);
            // first token of this lane's 8-token group (lanes pair up)
            const float Lg = __shfl_sync(0xffffffffu, pre[0], lane & ~1);
            bool split_ok = true;
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const int t = 4 * lane + k;
                vs[t] = v[k];
                vs[128 + t] = pre[k];
                vs[256 + t] = v[k] * ex2(total - pre[k]);
                vs[384 + t] = ex2(Lg - pre[k]) * v[k];
                split_ok = split_ok && (Lg - pre[k] <= kSplitSpan2);
            }
            const bool all_ok = __all_sync(0xffffffffu, split_ok);
            if (lane == 0) vs[512] = all_ok ? 1.0f : 0.0f;
            __syncwarp();
            if (lane == 0) mbar_arrive(&bars.v_full[i % k3Ring]);
            if (more) park(i + 3, nx);
            __syncwarp();
        }
        if (!ok && lane == 0 && p.fault) atomicCAS(p.fault, 0u, kFaultMmaOut);
    } else if (role == kR3B) {
        // ================= W_b: half of B' = w B, in place ==================
        for (int i = 0; i < n_ch; ++i) {
            if (!(ok = role3_wait(p, &bars.acc1, (uint32_t)(i & 1), role, kFaultMmaOut))) break;
            if (!(ok = role3_wait(p, &bars.v_full[i % k3Ring], (uint32_t)((i / k3Ring) & 1), role, kFaultMmaOut)))
                break;
            scale_b(sm + O3_B, slot(i) + 256, tid - 32 * 12);
            warp_arrive3(&bars.b_ready);
            warp_arrive3(&bars.v_empty[i % k3Ring]);
        }
    } else if (role == kR3M) {
        // ================= W_m: M into TMEM =================================
        for (int i = 0; i < n_ch; ++i) {
            // G1(i) retired, and with it G2(i-1), the last reader of M(i-1)
            if (!(ok = role3_wait(p, &bars.acc1, (uint32_t)(i & 1), role, kFaultMmaOut))) break;
            if (!(ok = role3_wait(p, &bars.v_full[i % k3Ring], (uint32_t)((i / k3Ring) & 1), role, kFaultMmaOut)))
                break;
            tc_fence_after();
            const float* vs = slot(i);
            const float* Lc2 = vs + 128;
            const float Lt = Lc2[row];
            const bool split = vs[512] != 0.0f;
            const int mh = warp >= 16 ? 1 : 0;  // tokens j 64 mh .. 64 mh + 63
#pragma unroll
            for (int qq = 0; qq < 2; ++qq) {
                const int q = 2 * mh + qq;
                float d[32];
                tmem_ld16(tm + lane_off + T3_D1 + 32 * q, *reinterpret_cast<float(*)[16]>(d));
                tmem_ld16(tm + lane_off + T3_D1 + 32 * q + 16, *reinterpret_cast<float(*)[16]>(d + 16));
                tmem_wait_ld();
                if (qq == 1) {
                    tc_fence_before();
                    warp_arrive3(&bars.d1_read);
                }
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    float m[16];
#pragma unroll
                    for (int c = 0; c < 2; ++c) {
                        const int j0 = 32 * q + 16 * h + 8 * c;
                        const float* dd = d + 16 * h + 8 * c;
                        if (j0 > row) {
#pragma unroll
                            for (int e = 0; e < 8; ++e) m[8 * c + e] = 0.0f;
                        } else if (split) {
                            const float eg = ex2(Lt - Lc2[j0]);
#pragma unroll
                            for (int e = 0; e < 8; ++e)
                                m[8 * c + e] = (j0 + e <= row) ? dd[e] * (eg * vs[384 + j0 + e]) : 0.0f;
                        } else {
#pragma unroll
                            for (int e = 0; e < 8; ++e)
                                m[8 * c + e] = (j0 + e <= row) ? dd[e] * ex2(Lt - Lc2[j0 + e]) * vs[j0 + e] : 0.0f;
                        }
                    }
                    uint32_t hi[8], lo[8];
                    split16(m, hi, lo);
                    // columns 16 q + 8 h of the packed halves hold tokens 32 q + 16 h ..
                    tmem_st8(tm + lane_off + T3_MH + 16 * q + 8 * h, hi);
                    tmem_st8(tm + lane_off + T3_ML + 16 * q + 8 * h, lo);
                }
            }
            tmem_wait_st();
            tc_fence_before();
            warp_arrive3(&bars.m_ready);
            warp_arrive3(&bars.v_empty[i % k3Ring]);
        }
    } else if (role == kR3C) {
        // ================= W_c: the carried state ===========================
        const uint32_t tS = tm + lane_off + T3_S;
        const int n = p.n_base + row;  // this lane's state (zeros past d_state)
        uint8_t* sS = sm + O3_S;
        auto put_s = [&](int q, const float (&v)[8]) {
            uint32_t hi[4], lo[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                hi[e] = pack_bf16x2(v[2 * e], v[2 * e + 1]);
                float h0, h1;
                unpack_bf16x2(hi[e], h0, h1);
                lo[e] = pack_bf16x2(v[2 * e] - h0, v[2 * e + 1] - h1);
            }
            *reinterpret_cast<uint4*>(sS + sw128_off(row, q)) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
            *reinterpret_cast<uint4*>(sS + 16384 + sw128_off(row, q)) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
        };
        // x: fp32 halves of 64 tokens through the staging buffer; the role's
        // first thread issues each load once the whole role has read the
        // previous one out
        const bool xs_leader = tid == 32 * 8;
        uint32_t xs_phase = 0;
        auto xs_load = [&](int chunk, int half) {
            mbar_expect_tx(&bars.xs_full, 16384);
            tma_load_4d(sm + O3_XS, &maps.x, &bars.xs_full, p0, tl.h, t_begin + chunk * kCS + 64 * half, tl.seq);
        };
        // x(chunk) as bf16 hi | lo tiles (MN-major, token rows), then x_full
        auto convert_x = [&](int chunk) -> bool {
            const int r = tid - 32 * 8;
#pragma unroll 1
            for (int half = 0; half < 2; ++half) {
                if (!role3_wait(p, &bars.xs_full, xs_phase & 1u, role, kFaultTmaOut)) return false;
                ++xs_phase;
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    const int q = r + 128 * k;  // token row q >> 3 of the half, channel chunk q & 7
                    const int j = q >> 3, c = q & 7;
                    const float4* src = reinterpret_cast<const float4*>(sm + O3_XS + j * 256 + c * 32);
                    uint4 hi, lo;
                    split8_f32(src[0], src[1], hi, lo);
                    const uint32_t off = sw128_off(64 * half + j, c);
                    *reinterpret_cast<uint4*>(sm + O3_X + off) = hi;
                    *reinterpret_cast<uint4*>(sm + O3_X + 16384 + off) = lo;
                }
                named_sync(1 + role, 128);  // the staging buffer is read out
                if (xs_leader) {
                    fence_async_smem();
                    if (half == 0)
                        xs_load(chunk, 1);
                    else if (chunk + 1 < n_ch)
                        xs_load(chunk + 1, 0);  // lands while this chunk is computed
                }
            }
            fence_async_smem();
            warp_arrive3(&bars.x_full);
            return true;
        };
        if (xs_leader) {
            prefetch_tmap(&maps.x);
            if (n_ch > 0) xs_load(0, 0);
        }
        {
            grid_dep_wait();  // the carry kernel's span-entry states
            const float* src;
            int64_t sc;
            if (run0 == 0) {
                int sq;
                src = s0_row(p, tl.seq, &sq)
                          ? p.s0 + (int64_t)sq * p.seq_s + (int64_t)tl.h * p.s_s0 + (int64_t)p0 * p.s_s1 + n
                          : nullptr;
                sc = p.s_s1;
            } else {
                src = p.agg + (unit0 + run0 - 1) * (int64_t)p.P * p.N + (int64_t)p0 * p.N + n;
                sc = p.N;
            }
            const int pn = n < p.N ? pw : 0;
#pragma unroll 1
            for (int q = 0; q < 8; ++q) {
                float v[8];
#pragma unroll
                for (int k = 0; k < 8; ++k)
                    v[k] = (8 * q + k < pn) ? (src ? src[(int64_t)(8 * q + k) * sc] : kNaN) : 0.0f;
                tmem_st8(tS + 8 * q, *reinterpret_cast<const uint32_t(*)[8]>(v));
                put_s(q, v);
            }
            tmem_wait_st();
            fence_async_smem();
            warp_arrive3(&bars.s_ready);
        }
        if (n_ch > 0) ok = convert_x(0);
        for (int i = 0; i < n_ch && ok; ++i) {
            // G4(i) retired, and G3(i) before it: D4 is ready, S_i's copy free
            if (!(ok = role3_wait(p, &bars.g4, (uint32_t)(i & 1), role, kFaultMmaOut))) break;
            if (!(ok = role3_wait(p, &bars.v_full[i % k3Ring], (uint32_t)((i / k3Ring) & 1), role, kFaultMmaOut)))
                break;
            tc_fence_after();
            const float decay = ex2(slot(i)[128 + kCS - 1]);
            const bool more = i + 1 < n_ch;
#pragma unroll
            for (int q = 0; q < 8; ++q) {
                float sv[8], dv[8];
                tmem_ld8(tS + 8 * q, sv);
                tmem_ld8(tm + lane_off + T3_D4 + 8 * q, dv);
                tmem_wait_ld();
#pragma unroll
                for (int k = 0; k < 8; ++k) sv[k] = fmaf(decay, sv[k], dv[k]);
                tmem_st8(tS + 8 * q, *reinterpret_cast<const uint32_t(*)[8]>(sv));
                if (more) put_s(q, sv);
            }
            tmem_wait_st();
            tc_fence_before();
            warp_arrive3(&bars.d4_read);
            if (more) {
                fence_async_smem();
                warp_arrive3(&bars.s_ready);
            }
            warp_arrive3(&bars.v_empty[i % k3Ring]);
            // x(i+1) over x(i) once G2(i) retired too (G4(i) already has)
            if (more) {
                if (!(ok = role3_wait(p, &bars.g2, (uint32_t)(i & 1), role, kFaultMmaOut))) break;
                if (!(ok = convert_x(i + 1))) break;
            }
        }
        if (ok && last && n < p.N) {
            float* s1 = p.s1 + (int64_t)tl.seq * p.seq_s + (int64_t)tl.h * p.s_s0 + (int64_t)p0 * p.s_s1 + n;
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
        grid_dep_wait();  // y of the previous 128-state pass, when adding to it
        for (int i = 0; i < n_ch; ++i) {
            // first the other half of B'(i), once G1(i) has read B(i)
            if (!(ok = role3_wait(p, &bars.acc1, (uint32_t)(i & 1), role, kFaultMmaOut))) break;
            if (!(ok = role3_wait(p, &bars.v_full[i % k3Ring], (uint32_t)((i / k3Ring) & 1), role, kFaultMmaOut)))
                break;
            scale_b(sm + O3_B, slot(i) + 256, 128 + tid);
            warp_arrive3(&bars.b_ready);
            // G2(i) retired, and G3(i) before it
            if (!(ok = role3_wait(p, &bars.g2, (uint32_t)(i & 1), role, kFaultMmaOut))) break;
            tc_fence_after();
            const int tp = t_begin + i * kCS;
            const int tlen = t_end - tp;
            const float e = ex2(slot(i)[128 + row]);
            float* yr = p.y + (int64_t)tl.seq * p.seq_y + (int64_t)(tp + row) * p.s_y0 + (int64_t)tl.h * p.s_y1 +
                        (int64_t)p0 * p.s_y2;
            const bool vec = p.s_y2 == 1 && pw == kSlab && (reinterpret_cast<uintptr_t>(yr) & 15) == 0;
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                float a[16], b[16];
                tmem_ld16(tm + lane_off + T3_D2 + 16 * q, a);
                tmem_ld16(tm + lane_off + T3_D3 + 16 * q, b);
                tmem_wait_ld();
                if (row < tlen) {
                    if (vec) {
#pragma unroll
                        for (int c = 0; c < 4; ++c) {
                            float4 v = make_float4(fmaf(e, b[4 * c], a[4 * c]), fmaf(e, b[4 * c + 1], a[4 * c + 1]),
                                                   fmaf(e, b[4 * c + 2], a[4 * c + 2]),
                                                   fmaf(e, b[4 * c + 3], a[4 * c + 3]));
                            float4* dst = reinterpret_cast<float4*>(yr + 16 * q) + c;
                            if (p.y_add) {
                                const float4 o = *dst;
                                v.x += o.x;
                                v.y += o.y;
                                v.z += o.z;
                                v.w += o.w;
                            }
                            *dst = v;
                        }
                    } else {
#pragma unroll
                        for (int k = 0; k < 16; ++k)
                            if (16 * q + k < pw) {
                                float* dst = yr + (int64_t)(16 * q + k) * p.s_y2;
                                *dst = fmaf(e, b[k], a[k]) + (p.y_add ? *dst : 0.0f);
                            }
                    }
                }
            }
            tc_fence_before();
            warp_arrive3(&bars.d_free);
            warp_arrive3(&bars.v_empty[i % k3Ring]);
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == k3WarpMma) {
        tc_fence_after();
        tmem_dealloc(tm, 512);
    }
}

// Maps of the output kernel: fp32 x in 64-token boxes (the staging halves),
// B and C and their low halves in 128-token boxes.
bool make_tc3_maps(EncodeFn fn, TcMaps* m, const ScanParams& p) {
    const int64_t S = p.S;
    std::memset(m, 0, sizeof(*m));
    if (!p.cast_bl || !p.cast_cl) return false;
    return make_map_f32(fn, &m->x, p.x, p.P, p.H, p.L, S, p.s_x1, p.s_x0, p.seq_x, 64) &&
           make_map(fn, &m->b, p.B, p.N, p.G, p.L, S, p.s_b1, p.s_b0, p.seq_b) &&
           make_map(fn, &m->bl, p.cast_bl, p.N, p.G, p.L, S, p.s_b1, p.s_b0, p.seq_b) &&
           make_map(fn, &m->c, p.C, p.N, p.G, p.L, S, p.s_c1, p.s_c0, p.seq_c) &&
           make_map(fn, &m->cl, p.cast_cl, p.N, p.G, p.L, S, p.s_c1, p.s_c0, p.seq_c);
}

}  // namespace

int configure_tc3(const helix_ctx*) {
    return cudaFuncSetAttribute(tc3_out_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)SMEM_3);
}

int launch_tc3(const helix_ctx* ctx, const Plan& pl, const ScanParams& p_in, void* stream) {
    auto fn = reinterpret_cast<EncodeFn>(ctx->encode_tiled);
    if (!fn) return cudaErrorNotSupported;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const char* only = std::getenv("HELIX_ONLY_PASS");
    ScanParams p = p_in;
    // x, B, C as bf16 hi | lo copies (already in the scratch when the shard
    // state pass left them there)
    const bool cast_ran = !pl.states_ready && (!only || *only == 'X');
    int e = launch_cast(ctx, pl, &p, stream, cast_ran);
    if (e != cudaSuccess) return e;
    TcMaps maps;
    if (!make_tc3_maps(fn, &maps, p)) return cudaErrorInvalidValue;
    const bool do_a = (!only || *only == 'A') && !pl.states_ready;
    const bool do_b = !only || *only == 'B';
    const bool do_c = !only || *only == 'C';
    const bool state_ran = pl.need_state_kernel && do_a;
    const bool carry_ran = pl.need_state_kernel && do_b;
    if (state_ran) {
        e = launch_tc_state_pass(ctx, p, pl.state_runs, true, cast_ran, stream);
        if (e != cudaSuccess) return e;
    }
    if (carry_ran) {
        e = launch_tc_carry(p, state_ran, stream);
        if (e != cudaSuccess) return e;
    }
    if (do_c) {
        const int64_t ctas = (int64_t)p.S * p.H * p.n_pslab * p.n_out;
        for (int half = 0; half < p.n_half; ++half) {
            ScanParams ph = p;
            ph.n_base = 128 * half;
            ph.y_add = half > 0;
            cudaLaunchConfig_t cfg = {};
            cfg.gridDim = dim3((unsigned)ctas);
            cfg.blockDim = dim3(k3Threads);
            cfg.dynamicSmemBytes = SMEM_3;
            cfg.stream = st;
            cudaLaunchAttribute attr[1];
            attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
            attr[0].val.programmaticStreamSerializationAllowed = 1;
            cfg.attrs = attr;
            cfg.numAttrs = (carry_ran || half > 0) ? 1 : 0;
            const cudaError_t le = cudaLaunchKernelEx(&cfg, tc3_out_kernel, maps, ph);
            if (le != cudaSuccess) return le;
        }
    }
    return cudaSuccess;
}

int launch_tc3_states(const helix_ctx* ctx, const Plan& pl, const ScanParams& p_in, void* stream) {
    ScanParams p = p_in;
    const int e = launch_cast(ctx, pl, &p, stream, true);
    if (e != cudaSuccess) return e;
    return launch_tc_state_pass(ctx, p, pl.state_runs, true, true, stream);
}

}  // namespace hx
