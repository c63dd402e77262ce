// device.cpp -- context lifetime, device capability probe, error strings.
// Replaces reference src/runtime/device.mm:7-85 (Metal device + metallib
// loading).  Everything a later encode call needs is resolved here, so encode
// mutates no shared state except the calling thread's error string.
#include <cuda.h>
#include <cuda_runtime.h>

#include <map>
#include <mutex>
#include <string>

#include "helix/helix_ext.h"
#include "internal.h"

namespace hx {

namespace {
// Errors raised before a context exists (helix_ctx_create), per thread.
thread_local std::string t_null_error;
}  // namespace

void set_error(const helix_ctx* ctx, const std::string& msg) {
    if (!ctx) {
        t_null_error = msg;
        return;
    }
    auto* c = const_cast<helix_ctx*>(ctx);
    std::lock_guard<std::mutex> lk(c->err_mu);
    c->errors[std::this_thread::get_id()] = msg;
}

// The string stays valid until this thread's next error on ctx, or until
// ctx is freed.
const char* get_error(const helix_ctx* ctx) {
    if (!ctx) return t_null_error.c_str();
    auto* c = const_cast<helix_ctx*>(ctx);
    std::lock_guard<std::mutex> lk(c->err_mu);
    auto it = c->errors.find(std::this_thread::get_id());
    return it == c->errors.end() ? "" : it->second.c_str();
}

}  // namespace hx

namespace {

// Restores the caller's current device on scope exit.
struct DeviceGuard {
    int prev = -1;
    explicit DeviceGuard(int dev) {
        if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
        if (prev != dev) cudaSetDevice(dev);
    }
    ~DeviceGuard() {
        int cur = -1;
        if (prev >= 0 && cudaGetDevice(&cur) == cudaSuccess && cur != prev) cudaSetDevice(prev);
    }
};

}  // namespace

extern "C" helix_status helix_ctx_create(helix_ctx** out, void* device, const char* /*path*/) {
    if (!out) return HELIX_ERR_INVALID_ARG;
    *out = nullptr;

    int count = 0;
    if (cudaGetDeviceCount(&count) != cudaSuccess || count <= 0) {
        cudaGetLastError();
        hx::set_error(nullptr, "no CUDA device");
        return HELIX_ERR_NO_DEVICE;
    }
    int dev = 0;
    if (device) {
        dev = *static_cast<const int*>(device);
    } else if (cudaGetDevice(&dev) != cudaSuccess) {
        cudaGetLastError();
        return HELIX_ERR_NO_DEVICE;
    }
    if (dev < 0 || dev >= count) {
        hx::set_error(nullptr, "device ordinal out of range");
        return HELIX_ERR_NO_DEVICE;
    }

    auto* ctx = new helix_ctx();
    ctx->device = dev;
    cudaDeviceGetAttribute(&ctx->cc_major, cudaDevAttrComputeCapabilityMajor, dev);
    cudaDeviceGetAttribute(&ctx->cc_minor, cudaDevAttrComputeCapabilityMinor, dev);
    cudaDeviceGetAttribute(&ctx->n_sm, cudaDevAttrMultiProcessorCount, dev);
    int smem = 0;
    cudaDeviceGetAttribute(&smem, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    ctx->max_smem_optin = (size_t)smem;

    // The kernels are compiled for sm_100a only (tcgen05, TMEM, TMA).
    if (ctx->cc_major != 10 || ctx->cc_minor != 0) {
        hx::set_error(nullptr, "device is not sm_100 (B200)");
        delete ctx;
        return HELIX_ERR_NO_DEVICE;
    }

    {
        DeviceGuard g(dev);
        if (hx::configure_simt(ctx) != cudaSuccess || hx::configure_diag(ctx) != cudaSuccess) {
            hx::set_error(nullptr, std::string("configuring fp32 kernels failed: ") +
                                       cudaGetErrorString(cudaGetLastError()));
            delete ctx;
            return HELIX_ERR_PIPELINE;
        }
        ctx->tc_ready = hx::configure_tc(ctx) == cudaSuccess && hx::configure_tc3(ctx) == cudaSuccess;
        if (!ctx->tc_ready) cudaGetLastError();
        if (hx::fault_word_address(&ctx->fault_word) != cudaSuccess) {
            cudaGetLastError();
            ctx->fault_word = nullptr;
        }

        cudaDriverEntryPointQueryResult q{};
        void* fn = nullptr;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            ctx->encode_tiled = fn;
        else
            cudaGetLastError();
        if (!ctx->encode_tiled) ctx->tc_ready = false;
    }

    *out = ctx;
    return HELIX_OK;
}

extern "C" void helix_ctx_free(helix_ctx* ctx) { delete ctx; }

extern "C" const char* helix_ctx_last_error(const helix_ctx* ctx) {
    if (!ctx) {
        const char* e = hx::get_error(nullptr);
        return *e ? e : "null context";
    }
    return hx::get_error(ctx);
}

extern "C" helix_status helix_device_fault(helix_ctx* ctx, uint32_t* code) {
    if (!ctx || !code) return HELIX_ERR_INVALID_ARG;
    DeviceGuard g(ctx->device);
    unsigned v = 0;
    if (hx::read_tc_fault(&v) != cudaSuccess) {
        hx::set_error(ctx, std::string("reading the fault word failed: ") +
                               cudaGetErrorString(cudaGetLastError()));
        return HELIX_ERR_PIPELINE;
    }
    *code = v;
    return HELIX_OK;
}
