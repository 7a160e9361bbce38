// ctx_internal.h — what other translation units of the library may ask of a
// context (oxg_ctx is defined in oxg_abi.cu). Not exported.
#pragma once

#include <cuda_runtime.h>

#include "kernels.h"

struct oxg_ctx;

namespace oxg {

// Device weights of uploaded layer `layer`, plus the context's device and
// stream. Returns false, with the context's last error set, when the layer
// has not been uploaded.
bool ctx_layer(oxg_ctx *ctx, int layer, MoeDeviceWeights *w, int *device, cudaStream_t *stream);

// Records `msg` as the context's last error and returns `status`.
int ctx_error(oxg_ctx *ctx, int status, const char *msg);

}  // namespace oxg
