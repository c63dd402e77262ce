// umma_probe.cu -- TEST INFRASTRUCTURE: checks the tcgen05 operand layouts the
// product kernels rely on, one GEMM per mode, in a single 128-thread CTA.
// P and Q are 128x128 bf16 row-major in global memory.
//   mode 0: D[128][128] = P Q^T    A K-major, B K-major, both loaded by TMA
//   mode 1: same, both operands written by threads with sw128_off()
//   mode 2: D[128][64]  = P Q[:, :64]    A K-major (threads), B MN-major (TMA)
//   mode 3: D[128][64]  = P^T Q[:, :64]  A MN-major, two 64-wide tiles (TMA),
//                                        B MN-major (threads)
//   mode 4: D[128][128] = P Q^T    A in TMEM (tcgen05.st: row m in lane m,
//                                  bf16 pairs per column), B K-major (TMA)
// Waits are bounded; on timeout the kernel records 1 in *status and returns
// after freeing its TMEM.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include "kernels/umma.cuh"

using namespace hx::umma;

namespace {

struct Maps {
    CUtensorMap p, q;
};

__global__ void __launch_bounds__(128, 1) probe_kernel(int mode, const __grid_constant__ Maps maps,
                                                       const __nv_bfloat16* P, const __nv_bfloat16* Q,
                                                       float* D, unsigned* status) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* a0 = sm;             // 16 KB
    uint8_t* a1 = sm + 16384;     // 16 KB
    uint8_t* b0 = sm + 32768;     // 16 KB
    uint8_t* b1 = sm + 49152;     // 16 KB
    __shared__ uint64_t bar_tma, bar_mma;
    __shared__ uint32_t tmem_base;
    __shared__ int abort_flag;
    const int tid = threadIdx.x, warp = tid >> 5;

    if (tid == 0) {
        mbar_init(&bar_tma, 1);
        mbar_init(&bar_mma, 1);
        fence_mbar_init();
        abort_flag = 0;
    }
    if (warp == 0) {
        tmem_alloc(&tmem_base, 256);
        tmem_relinquish();
    }
    __syncthreads();
    tc_fence_after();
    const uint32_t tm = tmem_base;

    // thread-written tiles: row r of a [rows][64] bf16 tile from global
    auto write_tile = [&](uint8_t* dst, const __nv_bfloat16* src, int ld, int col0, bool transpose) {
        for (int i = tid; i < 128 * 8; i += 128) {
            const int r = i >> 3, c = i & 7;
            uint32_t w[4];
            for (int k = 0; k < 4; ++k) {
                float lo, hi;
                const int e = col0 + c * 8 + 2 * k;
                if (!transpose) {
                    lo = __bfloat162float(src[r * ld + e]);
                    hi = __bfloat162float(src[r * ld + e + 1]);
                } else {
                    lo = __bfloat162float(src[e * ld + r]);
                    hi = __bfloat162float(src[(e + 1) * ld + r]);
                }
                w[k] = pack_bf16x2(lo, hi);
            }
            *reinterpret_cast<uint4*>(dst + sw128_off(r, c)) = make_uint4(w[0], w[1], w[2], w[3]);
        }
    };

    uint32_t tx_bytes = 0;
    if (mode == 0) tx_bytes = 65536;
    if (mode == 4) tx_bytes = 32768;
    if (mode == 2) tx_bytes = 16384;
    if (mode == 3) tx_bytes = 32768;
    if (tid == 0 && tx_bytes) {
        mbar_expect_tx(&bar_tma, tx_bytes);
        if (mode == 0) {
            tma_load_4d(a0, &maps.p, &bar_tma, 0, 0, 0, 0);
            tma_load_4d(a1, &maps.p, &bar_tma, 64, 0, 0, 0);
            tma_load_4d(b0, &maps.q, &bar_tma, 0, 0, 0, 0);
            tma_load_4d(b1, &maps.q, &bar_tma, 64, 0, 0, 0);
        } else if (mode == 2) {
            tma_load_4d(b0, &maps.q, &bar_tma, 0, 0, 0, 0);
        } else if (mode == 3) {
            tma_load_4d(a0, &maps.p, &bar_tma, 0, 0, 0, 0);
            tma_load_4d(a1, &maps.p, &bar_tma, 64, 0, 0, 0);
        } else if (mode == 4) {
            tma_load_4d(b0, &maps.q, &bar_tma, 0, 0, 0, 0);
            tma_load_4d(b1, &maps.q, &bar_tma, 64, 0, 0, 0);
        }
    }
    if (mode == 4) {
        // A = P into TMEM columns 128..191: this thread's row, 64 columns of
        // packed pairs (P[r][2c] low half, P[r][2c+1] high half).
        const int r = 32 * (warp & 3) + (tid & 31);
        for (int c0 = 0; c0 < 64; c0 += 16) {
            uint32_t w[16];
            for (int c = 0; c < 16; ++c)
                w[c] = pack_bf16x2(__bfloat162float(P[r * 128 + 2 * (c0 + c)]),
                                   __bfloat162float(P[r * 128 + 2 * (c0 + c) + 1]));
            tmem_st16(tm + ((uint32_t)(32 * (warp & 3)) << 16) + 128 + c0, w);
        }
        tmem_wait_st();
        tc_fence_before();
    }
    if (mode == 1) {
        write_tile(a0, P, 128, 0, false);
        write_tile(a1, P, 128, 64, false);
        write_tile(b0, Q, 128, 0, false);
        write_tile(b1, Q, 128, 64, false);
    } else if (mode == 2) {
        write_tile(a0, P, 128, 0, false);
        write_tile(a1, P, 128, 64, false);
    } else if (mode == 3) {
        write_tile(b0, Q, 128, 0, false);  // rows k, 64 n contiguous
    }
    fence_async_smem();
    __syncthreads();
    if (tx_bytes && !mbar_wait(&bar_tma, 0, 1ll << 31)) abort_flag = 1;
    __syncthreads();

    const int N = (mode <= 1 || mode == 4) ? 128 : 64;
    if (!abort_flag && tid == 0) {
        tc_fence_after();
        const uint32_t sa0 = smem_u32(a0), sb0 = smem_u32(b0);
        for (int ks = 0; ks < 8; ++ks) {
            uint64_t ad, bd;
            uint32_t id;
            if (mode <= 1) {  // K-major x K-major
                const uint32_t off = (ks >> 2) * 16384 + (ks & 3) * 32;
                ad = sdesc_sw128(sa0 + off, 16, 1024);
                bd = sdesc_sw128(sb0 + off, 16, 1024);
                id = idesc_bf16(128, 128, false, false);
            } else if (mode == 2) {  // K-major A, MN-major B
                ad = sdesc_sw128(sa0 + (ks >> 2) * 16384 + (ks & 3) * 32, 16, 1024);
                bd = sdesc_sw128(sb0 + ks * 2048, 16384, 1024);
                id = idesc_bf16(128, 64, false, true);
            } else if (mode == 3) {  // MN-major A (two tiles along M), MN-major B
                ad = sdesc_sw128(sa0 + ks * 2048, 16384, 1024);
                bd = sdesc_sw128(sb0 + ks * 2048, 16384, 1024);
                id = idesc_bf16(128, 64, true, true);
            } else {  // A from TMEM: K step ks = 8 columns
                bd = sdesc_sw128(sb0 + (ks >> 2) * 16384 + (ks & 3) * 32, 16, 1024);
                id = idesc_bf16(128, 128, false, false);
                mma_bf16_ts(tm, tm + 128 + 8 * ks, bd, id, ks > 0 ? 1u : 0u);
                continue;
            }
            mma_bf16(tm, ad, bd, id, ks > 0 ? 1u : 0u);
        }
        mma_commit(&bar_mma);
    }
    if (!abort_flag && !mbar_wait(&bar_mma, 0, 1ll << 31)) abort_flag = 1;
    tc_fence_after();
    __syncthreads();
    if (!abort_flag) {
        const int row = 32 * (warp & 3) + (tid & 31);
        for (int c0 = 0; c0 < N; c0 += 16) {
            float v[16];
            tmem_ld16(tm + ((uint32_t)(32 * (warp & 3)) << 16) + c0, v);
            tmem_wait_ld();
            for (int i = 0; i < 16; ++i) D[row * N + c0 + i] = v[i];
        }
    } else if (tid == 0) {
        *status = 1;
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) tmem_dealloc(tm, 256);
}

using EncodeFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                              const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                              CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

int make_map(CUtensorMap* m, const void* base) {
    static EncodeFn fn = nullptr;
    if (!fn) {
        cudaDriverEntryPointQueryResult q;
        void* f = nullptr;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) != cudaSuccess)
            return -1;
        fn = reinterpret_cast<EncodeFn>(f);
    }
    // 4-D view of a 128x128 bf16 row-major matrix: (col, 1, row, 1)
    cuuint64_t dims[4] = {128, 1, 128, 1};
    cuuint64_t strides[3] = {256, 256, 256 * 128};
    cuuint32_t box[4] = {64, 1, 128, 1};
    cuuint32_t es[4] = {1, 1, 1, 1};
    return fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(base), dims, strides, box, es,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS
               ? 0
               : -2;
}

}  // namespace

extern "C" int umma_probe(int mode, const void* P, const void* Q, float* D, unsigned* status) {
    Maps maps;
    if (make_map(&maps.p, P) || make_map(&maps.q, Q)) return -1;
    const int smem = 65536 + 1024;
    cudaFuncSetAttribute(probe_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    probe_kernel<<<1, 128, smem>>>(mode, maps, static_cast<const __nv_bfloat16*>(P),
                                   static_cast<const __nv_bfloat16*>(Q), D, status);
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return (int)e;
    return (int)cudaDeviceSynchronize();
}
