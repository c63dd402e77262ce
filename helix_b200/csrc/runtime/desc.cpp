// desc.cpp -- descriptor defaults and dense strides.
// Same contract as reference src/runtime/desc.cpp:9-46: every field gets its
// documented default and the strides are the dense ones for the layouts in
// helix.h.  No CUDA in this file.
#include <cmath>
#include <cstring>

#include "helix/helix.h"

extern "C" void helix_scan_desc_init(helix_scan_desc* d, int32_t n_tok, int32_t n_seq,
                                     int32_t n_head, int32_t head_dim, int32_t d_state,
                                     int32_t n_group) {
    if (!d) return;
    std::memset(d, 0, sizeof(*d));
    d->n_tok = n_tok;
    d->n_seq = n_seq;
    d->n_head = n_head;
    d->head_dim = head_dim;
    d->d_state = d_state;
    d->n_group = n_group;

    const int64_t L = n_tok, H = n_head, P = head_dim, N = d_state, G = n_group;
    // x and y: (tok, head, chan); B and C: (tok, group, state);
    // dt: (tok, head); state: (head, chan, state).
    const int64_t xs[3] = {H * P, P, 1};
    for (int i = 0; i < 3; ++i) { d->s_x[i] = xs[i]; d->s_y[i] = xs[i]; }
    const int64_t bs[3] = {G * N, N, 1};
    for (int i = 0; i < 3; ++i) { d->s_b[i] = bs[i]; d->s_c[i] = bs[i]; }
    d->s_dt[0] = H;
    d->s_dt[1] = 1;
    d->s_s[0] = P * N;
    d->s_s[1] = N;
    d->s_s[2] = 1;
    d->seq_x = d->seq_y = L * H * P;
    d->seq_b = d->seq_c = L * G * N;
    d->seq_dt = L * H;
    d->seq_s = H * P * N;
    d->s_a = 1;

    d->chunk = 0;
    d->a_form = HELIX_A_SCALAR_PER_HEAD;
    d->io_dtype = HELIX_F32;
    d->compute_dtype = HELIX_F32;
    d->backend = HELIX_BACKEND_AUTO;
    d->multipass = false;
    d->dt_min = 0.0f;        // ggml applies no clamp
    d->dt_max = INFINITY;
}
