// compat/ggml.h -- COMPILE-CHECK STAND-IN, not ggml.
//
// Declares only the tensor fields and helpers ggml-helix-cuda.cpp reads, so
// the bridge compiles and can be exercised in this repository without a
// llama.cpp checkout.  In a llama.cpp build the bridge includes ggml's own
// ggml.h instead (this directory is not on the include path there) and the
// real struct ggml_tensor is used; nothing here mirrors ggml's layout or
// values beyond the field names the bridge needs.

#pragma once

#include <stddef.h>
#include <stdint.h>

enum ggml_type {
    GGML_TYPE_F32 = 0,
    GGML_TYPE_I32 = 1,
    GGML_TYPE_OTHER = 2,
};

#define GGML_COMPAT_MAX_SRC 8

struct ggml_tensor {
    enum ggml_type       type;
    int64_t              ne[4];   // elements per dimension, fastest first
    size_t               nb[4];   // byte strides
    int32_t              op_params[16];
    struct ggml_tensor * src[GGML_COMPAT_MAX_SRC];
    void *               data;    // device pointer
};

static inline int32_t ggml_get_op_params_i32(const struct ggml_tensor * t, uint32_t i) { return t->op_params[i]; }

static inline int64_t ggml_nelements(const struct ggml_tensor * t) { return t->ne[0] * t->ne[1] * t->ne[2] * t->ne[3]; }
