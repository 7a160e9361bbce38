// noalloc.cu — an MoE-layer forward that allocates no memory.
//
// oxg_moe_forward keeps its working buffers (routing, permutation, the
// SwiGLU intermediate and the per-slot expert outputs) in scratch memory the
// context allocates with cudaMalloc the first time a batch needs more. Some
// callers cannot let a library do that: a serving runtime that reserves the
// whole device for its own memory pool up front (a library cudaMalloc would
// fail or fragment the pool), a real-time decode loop that cannot afford the
// device-wide synchronisation cudaMalloc/cudaFree may imply, or an embedding
// runtime whose policy is that foreign code never allocates device memory.
// oxg_moe_forward_noalloc serves them: the same layer math (router, top-k,
// expert MLPs, weighted combine) on the library's per-expert decode kernels,
// with the scratch carved out of one fixed array compiled into this library.
// Its outputs agree with oxg_moe_forward's within the layer tolerance; they
// are not bit-identical, because oxg_moe_forward's small-batch path uses the
// fused router and the scheduled expert kernels, which sum in another order.
//
// The array is a file-scope __device__ variable, so every GPU that loads the
// library holds kNoAllocScratchBytes of it until the process exits. Its host
// name is only a stand-in for the device symbol, so the device address is
// looked up once per device with cudaGetSymbolAddress (with that device
// current) on the first call made there, and cached for the life of the
// process: a cudaDeviceReset (or anything else that tears down and recreates
// the device's primary context) invalidates it, so this entry point must not
// be used after one.
//
// The decode kernels used here stream their weights with cp.async, which has
// no bounded wait that could give up, so no error word is carved out: a call
// that returns OXG_OK has launched work that cannot report a timeout.
#include <cuda_runtime.h>

#include <cstdio>
#include <mutex>

#include "../../include/oxg_b200.h"
#include "ctx_internal.h"
#include "kernels.h"

namespace {

constexpr size_t kNoAllocScratchBytes = 4u << 20;  // 4 MiB
constexpr int kMaxDevices = 64;

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

std::mutex g_addr_mu;
void *g_addr[kMaxDevices] = {};

// Device address of g_noalloc_scratch on `device` (which must be current).
cudaError_t scratch_address(int device, void **out) {
  std::lock_guard<std::mutex> lock(g_addr_mu);
  if (!g_addr[device]) {
    void *p = nullptr;
    cudaError_t st = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (st != cudaSuccess) return st;
    g_addr[device] = p;
  }
  *out = g_addr[device];
  return cudaSuccess;
}

struct Carve {
  int32_t *idx, *sigma, *counts, *offsets, *perm, *slot_pos;
  float *wts, *logits, *h, *y_slot;
};

size_t up256(size_t v) { return (v + 255) / 256 * 256; }

// Bytes of scratch T tokens need (and, with base != nullptr, the carve-up).
size_t carve(const oxg::MoeDeviceWeights &w, int T, char *base, Carve *c) {
  const size_t S = (size_t)T * w.k;
  size_t off = 0;
  auto take = [&](size_t bytes) {
    char *p = base ? base + off : nullptr;
    off = up256(off + bytes);
    return p;
  };
  char *p_idx = take(S * 4), *p_wts = take(S * 4), *p_sigma = take((size_t)T * 4);
  char *p_logits = take((size_t)T * w.E * 4), *p_counts = take((size_t)w.E * 4);
  char *p_offsets = take(((size_t)w.E + 1) * 4), *p_perm = take(S * 4), *p_slot = take(S * 4);
  char *p_h = take(S * w.I * 4), *p_y = take(S * w.H * 4);
  if (c) {
    c->idx = (int32_t *)p_idx;
    c->wts = (float *)p_wts;
    c->sigma = (int32_t *)p_sigma;
    c->logits = (float *)p_logits;
    c->counts = (int32_t *)p_counts;
    c->offsets = (int32_t *)p_offsets;
    c->perm = (int32_t *)p_perm;
    c->slot_pos = (int32_t *)p_slot;
    c->h = (float *)p_h;
    c->y_slot = (float *)p_y;
  }
  return off;
}

int cuda_error(oxg_ctx *ctx, cudaError_t st, const char *what) {
  char msg[256];
  snprintf(msg, sizeof(msg), "%s: %s (%s)", what, cudaGetErrorName(st), cudaGetErrorString(st));
  return oxg::ctx_error(ctx, OXG_ERR_CUDA, msg);
}

}  // namespace

extern "C" int oxg_moe_forward_noalloc(oxg_ctx *ctx, int layer, const uint16_t *x, int n_tokens,
                                       float *y) {
  if (!ctx) return OXG_ERR_INVALID_ARG;
  oxg::MoeDeviceWeights w{};
  int device = 0;
  cudaStream_t stream = nullptr;
  if (!oxg::ctx_layer(ctx, layer, &w, &device, &stream)) return OXG_ERR_STATE;
  {
    // an expert-parallel shard holds only some experts' weights; the kernels
    // below index every expert of the layer, so refuse it before any launch
    // (oxg_moe_forward refuses it with the same message)
    int eb = 0, ec = 0, ne = 0;
    if (oxg::ctx_layer_experts(ctx, layer, &eb, &ec, &ne) && ec != ne) {
      char msg[256];
      snprintf(msg, sizeof(msg),
               "layer %d holds experts [%d, %d) only: use oxg_moe_dispatch / oxg_moe_experts / "
               "oxg_moe_combine",
               layer, eb, eb + ec);
      return oxg::ctx_error(ctx, OXG_ERR_STATE, msg);
    }
  }
  const int T = n_tokens;
  if (T < 0) return oxg::ctx_error(ctx, OXG_ERR_SHAPE, "n_tokens must be >= 0");
  if (T == 0) return OXG_OK;
  if (!x || !y) return oxg::ctx_error(ctx, OXG_ERR_INVALID_ARG, "x and y must be non-NULL");
  if (((uintptr_t)x & 15) || ((uintptr_t)y & 15))
    return oxg::ctx_error(ctx, OXG_ERR_INVALID_ARG, "x and y must be 16-byte aligned");
  if (device < 0 || device >= kMaxDevices)
    return oxg::ctx_error(ctx, OXG_ERR_UNSUPPORTED, "device index beyond the no-allocation table");
  const size_t need = carve(w, T, nullptr, nullptr);
  if (need > kNoAllocScratchBytes) {
    int lo = 0, hi = T;  // largest token count that fits, for the message
    while (lo < hi) {
      const int mid = (lo + hi + 1) / 2;
      if (carve(w, mid, nullptr, nullptr) <= kNoAllocScratchBytes) lo = mid; else hi = mid - 1;
    }
    char msg[256];
    snprintf(msg, sizeof(msg),
             "n_tokens=%d needs %zu bytes of scratch; oxg_moe_forward_noalloc has %zu, "
             "enough for %d tokens of this layer",
             T, need, kNoAllocScratchBytes, lo);
    return oxg::ctx_error(ctx, OXG_ERR_SHAPE, msg);
  }

  int prev = -1;
  if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
  if (prev != device && cudaSetDevice(device) != cudaSuccess)
    return oxg::ctx_error(ctx, OXG_ERR_CUDA, "cudaSetDevice failed");
  int rc = OXG_OK;
  do {
    void *base = nullptr;
    cudaError_t st = scratch_address(device, &base);
    if (st != cudaSuccess) { rc = cuda_error(ctx, st, "cudaGetSymbolAddress(no-allocation scratch)"); break; }
    Carve c{};
    carve(w, T, (char *)base, &c);
    // Every scratch buffer below is written in full before it is read within
    // this call, so nothing needs clearing between calls.
    const int S = T * w.k;
    if ((st = oxg::launch_router_topk(x, w.router_w, w.router_b, T, w.H, w.E, w.k, c.idx, c.wts,
                                      c.logits, c.sigma, stream)) != cudaSuccess) {
      rc = cuda_error(ctx, st, "router_topk launch");
      break;
    }
    if ((st = oxg::launch_permute(c.idx, S, w.E, c.counts, c.offsets, c.perm, c.slot_pos,
                                  stream)) != cudaSuccess) {
      rc = cuda_error(ctx, st, "permute launch");
      break;
    }
    if ((st = oxg::launch_moe_mlp1_decode(w, x, c.perm, c.sigma, c.counts, c.offsets, S, 0, w.E,
                                          c.h, nullptr, stream)) != cudaSuccess) {
      rc = cuda_error(ctx, st, "mlp1 launch");
      break;
    }
    if ((st = oxg::launch_moe_mlp2_decode(w, c.h, c.counts, c.offsets, S, 0, w.E, c.y_slot,
                                          nullptr, stream)) != cudaSuccess) {
      rc = cuda_error(ctx, st, "mlp2 launch");
      break;
    }
    if ((st = oxg::launch_combine(c.y_slot, c.slot_pos, c.wts, T, w.H, w.k, y, stream)) !=
        cudaSuccess) {
      rc = cuda_error(ctx, st, "combine launch");
      break;
    }
  } while (0);
  if (prev >= 0 && prev != device) cudaSetDevice(prev);
  return rc;
}
