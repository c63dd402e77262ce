// ggml-helix-cuda.cpp -- the ggml-cuda <-> HELIX bridge.
//
// The CUDA counterpart of the reference's ggml-metal bridge
// (reference integration/ggml/ggml-helix.cpp:157-361).  Everything
// ggml-specific lives here so the upstream diff stays one #ifdef in
// ggml-cuda's SSM_SCAN:
//
//   #ifdef GGML_CUDA_USE_HELIX
//       if (ggml_cuda_op_ssm_scan_helix(ctx.stream(), ctx.device, dst)) return;
//   #endif
//
// Mapping.  ggml-cuda tensors are device pointers with byte strides nb[];
// helix_tensor is {device pointer, byte offset} and helix_scan_desc wants
// element strides, so the mapping is a divide, not a copy.  Layouts (ggml
// side, fastest dimension first):
//
//   src0  s     {d_state, head_dim, n_head, n_seqs}
//   src1  x     {head_dim, n_head, n_tokens, n_seqs}
//   src2  dt    {n_head, n_tokens, n_seqs}
//   src3  A     {1 | d_state, n_head}
//   src4  B     {d_state, n_group, n_tokens, n_seqs}
//   src5  C     {d_state, n_group, n_tokens, n_seqs}
//   src6  ids   {n_seqs}                                 int32
//   dst         y, then the final state at byte offset nelements(x) * 4
//
// Gates kept from the reference bridge: one snapshot (K == 1), all F32,
// n_head a multiple of n_group, and at least GGML_HELIX_MIN_TOKENS tokens.
// Unlike the reference's hook, a per-state A ({d_state, n_head}, Mamba-1)
// is passed on as HELIX_A_DIAG_PER_CHANNEL and served.  Below the token gate
// the fixed cost of the chunked scan's launches loses to ggml's own
// per-token kernel (the crossover is measured on B200 by measure_gate.py).
// ggml applies no clamp to softplus(dt), so neither does the descriptor.
//
// Precision.  By default the scan runs on HELIX's fp32-class tensor-core
// kernels (every fp32 operand as a bf16 hi + lo pair, three products per
// GEMM, fp32 accumulators and state: about 1e-5 relative L2 against fp64,
// far inside what ggml's op test accepts for fp32, which is why the
// reference bridge kept its bf16 path opt-in).  GGML_HELIX_BF16=1 opts into
// the bf16 tensor-core path (x, B, C rounded to bf16 once), the counterpart
// of the reference's GGML_HELIX_MPP=1; GGML_HELIX_EXACT=1 selects the exact
// fp32 CUDA-core kernels; GGML_HELIX_DISABLE=1 turns the hook off.
//
// Scratch.  helix never allocates; the bridge keeps one scratch buffer per
// (thread, device), grown with cudaMalloc outside stream capture.  While the
// stream is being captured into a CUDA graph, a call whose scratch does not
// fit the buffer already held is declined (ggml's own kernel runs), so
// nothing allocates inside a capture.

#include "ggml-helix-cuda.h"

#include <cuda_runtime.h>

#include <array>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <mutex>

#include "ggml.h"
#include "helix/helix.h"

namespace {

constexpr int kMaxDevices = 64;
// Below this many tokens the bridge declines.  Measured on B200 against a
// plain per-token scan kernel (measure_gate.py, 48 heads of 64 x 128): HELIX
// wins from 16 tokens on the fp32 kernels and from 8 on the tensor cores,
// and is twice as fast at 32; GGML_HELIX_MIN_TOKENS overrides.
constexpr int kDefaultMinTokens = 32;

struct Settings {
    bool disabled = false;
    bool bf16 = false;
    bool exact = false;
    int min_tokens = kDefaultMinTokens;
};

const Settings & settings() {
    static const Settings s = [] {
        Settings r;
        if (const char * e = std::getenv("GGML_HELIX_DISABLE"); e && e[0] == '1') r.disabled = true;
        if (const char * e = std::getenv("GGML_HELIX_BF16"); e && e[0] == '1') r.bf16 = true;
        if (const char * e = std::getenv("GGML_HELIX_EXACT"); e && e[0] == '1') r.exact = true;
        if (const char * e = std::getenv("GGML_HELIX_MIN_TOKENS")) r.min_tokens = std::atoi(e);
        return r;
    }();
    return s;
}

std::array<helix_ctx *, kMaxDevices> g_ctx{};
std::array<std::once_flag, kMaxDevices> g_once;

// One context per device, created on first use and shared by every thread
// (helix contexts are safe to share: encode keeps its error strings per
// thread and mutates nothing else).
helix_ctx * context_for(int device) {
    if (settings().disabled || device < 0 || device >= kMaxDevices) return nullptr;
    std::call_once(g_once[device], [device] {
        int dev = device;
        const helix_status st = helix_ctx_create(&g_ctx[device], &dev, nullptr);
        if (st != HELIX_OK) {
            g_ctx[device] = nullptr;
            std::fprintf(stderr, "ggml-helix-cuda: HELIX unavailable on device %d (status %d), using ggml kernels\n",
                         device, (int) st);
        }
    });
    return g_ctx[device];
}

// Per (thread, device) scratch: ggml may run several graphs from several
// threads; each thread's stream order then protects its own buffer.
struct Scratch {
    void * ptr = nullptr;
    size_t size = 0;
};
thread_local std::array<Scratch, kMaxDevices> t_scratch{};

void * scratch_for(int device, cudaStream_t stream, size_t bytes) {
    if (bytes == 0) return nullptr;
    Scratch & s = t_scratch[device];
    if (s.ptr && s.size >= bytes) return s.ptr;
    cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
    if (cudaStreamIsCapturing(stream, &cap) != cudaSuccess || cap != cudaStreamCaptureStatusNone) {
        cudaGetLastError();
        return nullptr;  // never allocate inside a capture
    }
    int prev = -1;
    cudaGetDevice(&prev);
    if (prev != device) cudaSetDevice(device);
    // the old buffer may still be in use by work on this thread's stream
    if (s.ptr) {
        cudaStreamSynchronize(stream);
        cudaFree(s.ptr);
        s = Scratch{};
    }
    void * p = nullptr;
    if (cudaMalloc(&p, bytes) == cudaSuccess) {
        s.ptr = p;
        s.size = bytes;
    } else {
        cudaGetLastError();
    }
    if (prev >= 0 && prev != device) cudaSetDevice(prev);
    return s.ptr;
}

inline int64_t elems(size_t nb, size_t type_size) { return (int64_t) (nb / type_size); }

inline helix_tensor to_helix(const ggml_tensor * t) {
    return t ? helix_tensor{ t->data, 0 } : HELIX_TENSOR_NULL;
}

bool build_desc(const ggml_tensor * op, helix_scan_desc * d) {
    const ggml_tensor * src0 = op->src[0];  // s
    const ggml_tensor * src1 = op->src[1];  // x
    const ggml_tensor * src2 = op->src[2];  // dt
    const ggml_tensor * src3 = op->src[3];  // A
    const ggml_tensor * src4 = op->src[4];  // B
    const ggml_tensor * src5 = op->src[5];  // C
    if (!src0 || !src1 || !src2 || !src3 || !src4 || !src5) return false;

    // One final state; K > 1 rollback snapshots are a different contract.
    if (ggml_get_op_params_i32(op, 0) != 1) return false;
    const ggml_tensor * all[] = { src0, src1, src2, src3, src4, src5, op };
    for (const ggml_tensor * t : all)
        if (t->type != GGML_TYPE_F32) return false;

    const int64_t d_state = src0->ne[0];
    const int64_t head_dim = src0->ne[1];
    const int64_t n_head = src0->ne[2];
    const int64_t n_group = src4->ne[1];
    const int64_t n_tok = src1->ne[2];
    const int64_t n_seq = src1->ne[3];
    if (n_head <= 0 || n_group <= 0 || n_head % n_group != 0) return false;
    if (n_tok < settings().min_tokens) return false;

    helix_scan_desc_init(d, (int32_t) n_tok, (int32_t) n_seq, (int32_t) n_head, (int32_t) head_dim,
                         (int32_t) d_state, (int32_t) n_group);
    const size_t ts = sizeof(float);
    d->s_s[0] = elems(src0->nb[2], ts);
    d->s_s[1] = elems(src0->nb[1], ts);
    d->s_s[2] = elems(src0->nb[0], ts);
    d->seq_s = elems(src0->nb[3], ts);
    d->s_x[0] = elems(src1->nb[2], ts);
    d->s_x[1] = elems(src1->nb[1], ts);
    d->s_x[2] = elems(src1->nb[0], ts);
    d->seq_x = elems(src1->nb[3], ts);
    d->s_dt[0] = elems(src2->nb[1], ts);
    d->s_dt[1] = elems(src2->nb[0], ts);
    d->seq_dt = elems(src2->nb[2], ts);
    d->s_b[0] = elems(src4->nb[2], ts);
    d->s_b[1] = elems(src4->nb[1], ts);
    d->s_b[2] = elems(src4->nb[0], ts);
    d->seq_b = elems(src4->nb[3], ts);
    d->s_c[0] = elems(src5->nb[2], ts);
    d->s_c[1] = elems(src5->nb[1], ts);
    d->s_c[2] = elems(src5->nb[0], ts);
    d->seq_c = elems(src5->nb[3], ts);
    if (src3->ne[0] == 1) {
        d->a_form = HELIX_A_SCALAR_PER_HEAD;
    } else if (src3->ne[0] == d_state) {
        d->a_form = HELIX_A_DIAG_PER_CHANNEL;  // the diagonal-A recurrence kernels
    } else {
        return false;
    }
    d->s_a = elems(src3->nb[1], ts);
    // y is the leading region of dst, dense like x
    d->s_y[0] = n_head * head_dim;
    d->s_y[1] = head_dim;
    d->s_y[2] = 1;
    d->seq_y = n_tok * n_head * head_dim;
    d->dt_min = 0.0f;
    d->dt_max = INFINITY;
    d->multipass = true;
    d->io_dtype = HELIX_F32;
    d->compute_dtype = settings().bf16 ? HELIX_BF16 : HELIX_F32;
    d->backend = settings().exact ? HELIX_BACKEND_REF : HELIX_BACKEND_AUTO;
    return true;
}

}  // namespace

extern "C" bool ggml_cuda_op_ssm_scan_helix(void * stream, int device, const struct ggml_tensor * op) {
    if (!op) return false;
    helix_ctx * ctx = context_for(device);
    if (!ctx) return false;
    helix_scan_desc d{};
    if (!build_desc(op, &d) || !helix_scan_supported(ctx, &d)) return false;

    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const size_t need = helix_scan_scratch_size(ctx, &d);
    void * scratch = scratch_for(device, st, need);
    if (need && !scratch) return false;

    // dst holds y first, then the final state
    char * dst = static_cast<char *>(op->data);
    const size_t s_off = (size_t) ggml_nelements(op->src[1]) * sizeof(float);
    const helix_tensor t_y{ dst, 0 };
    const helix_tensor t_s1{ dst, (uint64_t) s_off };
    const helix_tensor t_scratch = scratch ? helix_tensor{ scratch, 0 } : HELIX_TENSOR_NULL;

    // Announce the kernel family once: selection fails soft, so a declined or
    // differently served shape is otherwise invisible.
    static std::once_flag s_announced;
    std::call_once(s_announced, [&] {
        std::fprintf(stderr, "ggml-helix-cuda: kernel = %s (d_state=%d head_dim=%d n_head=%d)\n",
                     helix_ctx_backend_desc(ctx, &d), (int) d.d_state, (int) d.head_dim, (int) d.n_head);
    });

    const helix_status rc = helix_scan_encode(ctx, stream, &d, to_helix(op->src[0]), to_helix(op->src[1]),
                                              to_helix(op->src[2]), to_helix(op->src[3]), to_helix(op->src[4]),
                                              to_helix(op->src[5]), to_helix(op->src[6]), t_y, t_s1, t_scratch);
    if (rc != HELIX_OK) {
        // nothing was enqueued: ggml's own kernel runs instead
        std::fprintf(stderr, "ggml-helix-cuda: helix_scan_encode failed (%d): %s\n", (int) rc,
                     helix_ctx_last_error(ctx));
        return false;
    }
    return true;
}
