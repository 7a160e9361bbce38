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
// Resident expert range [*begin, *begin + *count) of uploaded layer `layer`
// (all experts unless it was uploaded with oxg_moe_upload_shard); false when
// the layer has not been uploaded.
bool ctx_layer_experts(oxg_ctx *ctx, int layer, int *begin, int *count, int *n_experts);

// Records `msg` as the context's last error and returns `status`.
int ctx_error(oxg_ctx *ctx, int status, const char *msg);

// The context's device, stream and SM count.
int ctx_device(const oxg_ctx *ctx);
cudaStream_t ctx_stream(const oxg_ctx *ctx);
int ctx_n_sms(const oxg_ctx *ctx);

// One MoE-layer forward of T tokens (x [T, H] bf16 -> y [T, H] f32) on the
// context's stream with the library's automatic kernel choice, exactly as
// oxg_moe_forward; ctx_moe_reserve sizes the scratch for T tokens once.
int ctx_moe_forward(oxg_ctx *ctx, int layer, const uint16_t *x, int T, float *y);
// Expert parallelism: the hidden size of layer `layer` when it is a shard that
// the context's peer-memory exchange serves (0 otherwise), and its forward
// (oxg_moe_forward_ep; every process of the exchange must make the same calls).
int ctx_moe_ep_hidden(oxg_ctx *ctx, int layer);
int ctx_moe_forward_ep(oxg_ctx *ctx, int layer, const uint16_t *x, int T, float *y);
int ctx_moe_reserve(oxg_ctx *ctx, int layer, int T);
// Hidden size of uploaded MoE layer `layer` (0 when absent), its top-k, and
// the expert ids [T, k] the context's last MoE forward chose (device).
int ctx_moe_hidden(oxg_ctx *ctx, int layer);
int ctx_moe_topk(oxg_ctx *ctx, int layer);
const int32_t *ctx_moe_last_idx(oxg_ctx *ctx);

// Launch accounting: counts the launch and, with profiling on, brackets it
// with CUDA events on the context's stream under `name`.
void *ctx_prof_begin(oxg_ctx *ctx);
void ctx_prof_end(oxg_ctx *ctx, const char *name, void *begin, cudaError_t st);
template <class F>
cudaError_t ctx_launch(oxg_ctx *ctx, const char *name, F &&fn) {
  void *b = ctx_prof_begin(ctx);
  const cudaError_t st = fn();
  ctx_prof_end(ctx, name, b, st);
  return st;
}

// Changes whenever a device pointer a captured CUDA graph could hold goes
// stale: a layer (re)uploaded or released, the scratch reallocated.
unsigned long long ctx_epoch(const oxg_ctx *ctx);
// Profiling on/off flag (suspended while a graph is captured) and the launch
// counter (graph replays add their kernels to it).
bool &ctx_profile_flag(oxg_ctx *ctx);
void ctx_add_launches(oxg_ctx *ctx, long long n);
long long ctx_launch_count(const oxg_ctx *ctx);

// Full-model state (model_abi.cu), owned by the context.
struct ModelState;
ModelState *&ctx_model(oxg_ctx *ctx);
void model_free(oxg_ctx *ctx);
// Reads (and clears) the model kernels' error word after a synchronise.
int model_check_error(oxg_ctx *ctx);

}  // namespace oxg
