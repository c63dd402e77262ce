// tc_shared.cuh -- pieces shared by the two tcgen05 kernel files
// (scan_tc.cu: bf16 operands; scan_tc3.cu: three-product bf16 split):
// tensor maps, shared-memory descriptors of two-atom operands, the bounded
// wait budget, and the per-chunk decay vectors one warp computes.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <cstring>

#include "common.cuh"
#include "umma.cuh"

namespace hx {
namespace tc {

using namespace umma;

constexpr int kCS = 128;
constexpr long long kWaitBudget = 1ll << 31;  // clock cycles, ~1 s
constexpr float kLog2e = 1.4426950408889634f;

// Tensor maps of one scan.  x, b, c: bf16 (x, B, C or their bf16 copies);
// xl, bl, cl: the low halves of the three-product split (scan_tc3.cu only).
struct TcMaps {
    CUtensorMap x, b, c;
    CUtensorMap y;  // fp32 y in 32-channel x 64-token boxes (fast output path)
    CUtensorMap xl, bl, cl;
    int y_ok;       // y could be described by a tensor map
};

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

// Raw dt of tokens t0 + 4 lane .. +3.  Tokens at or past t_end read token
// t_end - 1 instead (every consumer masks them by the chunk length): the loads
// carry no condition, so nothing waits for them before their first use.
__device__ __forceinline__ void warp_load_dt(const ScanParams& p, int64_t db, int t0, int t_end, float (&raw)[4]) {
    const int lane = threadIdx.x & 31;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        const int t = min(t0 + 4 * lane + k, t_end - 1);
        raw[k] = __ldg(p.dt + db + (int64_t)t * p.s_dt0);
    }
}

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------
using EncodeFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                              const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                              CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

// 4-D bf16 map (inner, d1, tok, seq) with a 64 x 1 x box_tok x 1 box,
// 128-byte swizzle.  Coordinates past the extents read as zero.
inline bool make_map(EncodeFn fn, CUtensorMap* m, const void* base, int64_t inner, int64_t d1, int64_t tok, int64_t seq,
              int64_t s1, int64_t s_tok, int64_t s_seq, int box_tok = kCS) {
    cuuint64_t dims[4] = {(cuuint64_t)inner, (cuuint64_t)d1, (cuuint64_t)tok, (cuuint64_t)seq};
    cuuint64_t strides[3] = {(cuuint64_t)(s1 * 2), (cuuint64_t)(s_tok * 2), (cuuint64_t)(s_seq * 2)};
    cuuint32_t box[4] = {64, 1, (cuuint32_t)box_tok, 1};
    cuuint32_t es[4] = {1, 1, 1, 1};
    return fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(base), dims, strides, box, es,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// 4-D fp32 map (inner, d1, tok, seq) with a 64 x 1 x box_tok x 1 box and no
// swizzle (256-byte rows): fp32 x read in place by the three-product family.
inline bool make_map_f32(EncodeFn fn, CUtensorMap* m, const void* base, int64_t inner, int64_t d1, int64_t tok,
                         int64_t seq, int64_t s1, int64_t s_tok, int64_t s_seq, int box_tok) {
    cuuint64_t dims[4] = {(cuuint64_t)inner, (cuuint64_t)d1, (cuuint64_t)tok, (cuuint64_t)seq};
    cuuint64_t strides[3] = {(cuuint64_t)(s1 * 4), (cuuint64_t)(s_tok * 4), (cuuint64_t)(s_seq * 4)};
    cuuint32_t box[4] = {64, 1, (cuuint32_t)box_tok, 1};
    cuuint32_t es[4] = {1, 1, 1, 1};
    return fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, const_cast<void*>(base), dims, strides, box, es,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace tc
}  // namespace hx
