// ref_shim.cpp -- TEST INFRASTRUCTURE ONLY.
//
// extern "C" wrappers around the HELIX reference's own fp64 oracle
// (namespace helix::ref, reference include/helix/reference.hpp:31-52), so the
// Python tests can call the reference's code through ctypes.  This file is
// ours; the reference sources it links are compiled where they lie (see
// oracle/Makefile) into oracle/_ref/, which is git-ignored.
#include <cstring>
#include <vector>

#include "helix/reference.hpp"

extern "C" {

void ref_scan(const helix_scan_desc* d, const float* s0, const float* x, const float* dt,
              const float* A, const float* B, const float* C, const int32_t* ids, float* y,
              float* s1) {
    helix::ref::scan(*d, s0, x, dt, A, B, C, ids, y, s1);
}

void ref_scan_chunked(const helix_scan_desc* d, const float* s0, const float* x, const float* dt,
                      const float* A, const float* B, const float* C, const int32_t* ids,
                      float* y, float* s1) {
    helix::ref::scan_chunked(*d, s0, x, dt, A, B, C, ids, y, s1);
}

// snap: n_chunks blocks of n_seq*seq_s doubles (the reference's own layout).
void ref_scan_with_snapshots(const helix_scan_desc* d, const float* s0, const float* x,
                             const float* dt, const float* A, const float* B, const float* C,
                             const int32_t* ids, float* y, float* s1, int32_t chunk,
                             double* snap) {
    std::vector<std::vector<double>> st;
    helix::ref::scan_with_snapshots(*d, s0, x, dt, A, B, C, ids, y, s1, chunk, &st);
    size_t off = 0;
    for (const auto& v : st) {
        std::memcpy(snap + off, v.data(), v.size() * sizeof(double));
        off += v.size();
    }
}

void ref_desc_init(helix_scan_desc* d, int32_t L, int32_t S, int32_t H, int32_t P, int32_t N,
                   int32_t G) {
    helix_scan_desc_init(d, L, S, H, P, N, G);
}

int ref_desc_size(void) { return (int)sizeof(helix_scan_desc); }

}  // extern "C"
