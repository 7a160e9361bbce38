// oxg_abi.cu — the C ABI of liboxg_b200.so (declared in include/oxg_b200.h).
//
// Host-side runtime: contexts (device + stream + scratch), the per-layer weight
// registry, argument validation with the reference's error texts, and the
// launch sequence of one MoE layer. No entry point throws across the ABI.
#include <cuda_runtime.h>

#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <string>
#include <algorithm>
#include <cmath>
#include <vector>

#include "../../include/oxg_b200.h"
#include "ctx_internal.h"
#include "kernels.h"

namespace {

thread_local std::string g_tls_error = "";

struct Layer {
  bool present = false;
  oxg_moe_dims dims{};
  void *block = nullptr;  // one allocation holding everything below
  uint16_t *router_w = nullptr, *router_b = nullptr;
  uint8_t *w1 = nullptr, *w2 = nullptr;  // tile chunks (codes + scales) of mlp1 / mlp2
  uint16_t *b1 = nullptr, *b2 = nullptr;
  // Every E8M0 scale is 0 or in [104, 140], so scale * E2M1 is exact in f16
  // (0.5 * 2^-23 is the smallest f16 subnormal, 6 * 2^13 = 49152 stays below
  // the f16 maximum 65504 while 6 * 2^14 would not) and the tensor-core
  // prefill path applies (H and I multiples of 64 too).
  bool prefill_ok = false;
  unsigned scale_min = 0, scale_max = 0;
  // The block-scaled tensor-core copy: the checkpoint's packed codes as they
  // are and the scale atoms (moe_mxf.cu). Usable when H and I are multiples
  // of 64 (>= 128) and no scale is 255 (NaN as a UE8M0 scale; +inf in the
  // reference's dequantisation).
  uint8_t *q1 = nullptr, *a1 = nullptr, *q2 = nullptr, *a2 = nullptr;
  uint8_t *p1 = nullptr, *p2 = nullptr;  // scale atoms of the prefill GEMMs' 192-row weight tiles
  bool mxf_ok = false;
  // experts [expert_begin, expert_begin + expert_count) are resident (all of
  // them unless uploaded with oxg_moe_upload_shard); the router is complete
  int expert_begin = 0, expert_count = 0;
  bool sharded() const { return expert_count != dims.n_experts; }
};

// Completion counters at the start of the scratch: zeroed when the scratch is
// allocated and left at zero by every forward that uses them.
constexpr int kMaxBands = 1024;
// Tokens per chunk of a host-buffer forward (oxg_moe_forward_host) when the
// caller has not set one (a batch of T tokens runs in T / 1600 equal chunks).
// Measured on gpt-oss-20b, 8192 tokens: 5 chunks of 1639 tokens 2.67 M
// tokens/s, 4 of 2048 2.46 M, 8 of 1024 2.09 M — every chunk streams all the
// expert weights again and below ~200 tokens per expert the prefill GEMMs'
// 256-column tiles run half empty, while fewer chunks leave longer copies
// that cannot overlap.
constexpr int kHostChunkTokens = 1600;
// done, err, per-band counters, the flat-split decode kernels' counters
constexpr size_t kCounterBytes = (2 + kMaxBands + oxg::kFlatMaxWarps) * sizeof(uint32_t);

struct Scratch {
  void *base = nullptr;
  size_t bytes = 0;
  uint32_t *done = nullptr, *band_done = nullptr, *flat_cnt = nullptr;
  float4 *parts = nullptr;  // flat-split decode partial sums
  int *err = nullptr;  // prefill pipeline timeout code
  uint16_t *xp = nullptr, *h_hi = nullptr, *h_lo = nullptr;
  float *pos_scale = nullptr;
  int32_t *active = nullptr, *n_active = nullptr;
  int32_t *idx = nullptr, *sigma = nullptr, *counts = nullptr, *offsets = nullptr;
  int32_t *perm = nullptr, *slot_pos = nullptr;
  int32_t *cta_hist = nullptr, *local_rank = nullptr;  // batched router's counting-sort halves
  int32_t *v_expert = nullptr, *v_pos0 = nullptr, *v_count = nullptr, *n_virtual = nullptr;  // virtual experts
  float *wts = nullptr, *logits = nullptr, *h = nullptr, *y_slot = nullptr;
  uint16_t *x_stage = nullptr;
  float *y_stage = nullptr;
  // block-scaled decode operands: x and h as E4M3 terms and their scale
  // atoms; zeroed whenever the layout changes (no stale NaN scale bytes)
  uint8_t *xq = nullptr, *xsf = nullptr, *hq = nullptr, *hsf = nullptr;
  uint32_t *tok_mask = nullptr;
  size_t xq_bytes = 0, xsf_bytes = 0, hq_bytes = 0, hsf_bytes = 0;
  size_t layout_key = 0;
  // block-scaled prefill operands (padded positions, rows_cap rows per plane)
  uint8_t *pxq = nullptr, *pxsf = nullptr, *phq = nullptr, *phsf = nullptr;
  int rows_cap = 0;
};

// CUDA-event brackets around kernel launches, read back on demand.
struct Profiler {
  bool on = false;
  struct Rec {
    const char *name;
    cudaEvent_t start, stop;
  };
  std::vector<Rec> recs;       // pending brackets since the last read/reset
  std::vector<cudaEvent_t> pool;
  struct Sum {
    std::string name;
    double ms = 0.0;
    int launches = 0;
  };
  std::vector<Sum> sums;

  cudaEvent_t get() {
    if (!pool.empty()) {
      cudaEvent_t e = pool.back();
      pool.pop_back();
      return e;
    }
    cudaEvent_t e = nullptr;
    cudaEventCreate(&e);
    return e;
  }
  Sum &sum(const char *name) {
    for (Sum &s : sums)
      if (s.name == name) return s;
    sums.push_back(Sum{name, 0.0, 0});
    return sums.back();
  }
  // Folds finished brackets into the sums (the caller has synchronised).
  void drain() {
    for (Rec &r : recs) {
      float ms = 0.f;
      if (cudaEventElapsedTime(&ms, r.start, r.stop) == cudaSuccess) {
        Sum &s = sum(r.name);
        s.ms += ms;
        s.launches += 1;
      }
      pool.push_back(r.start);
      pool.push_back(r.stop);
    }
    recs.clear();
  }
  void destroy() {
    drain();
    for (cudaEvent_t e : pool) cudaEventDestroy(e);
    pool.clear();
  }
};

}  // namespace

struct oxg_ctx {
  int device = 0;
  cudaStream_t own_stream = nullptr;
  cudaStream_t stream = nullptr;
  std::string error;
  std::vector<Layer> layers;
  Scratch ws;
  int last_layer = -1;
  int ep_tokens = -1;  // tokens of the last oxg_moe_dispatch (its positions feed oxg_moe_combine)
  int n_sms = 148;
  long long launches = 0;
  bool prefill_pending = false;  // a prefill ran since the error word was last read
  Profiler prof;
  oxg::ModelState *model = nullptr;  // full-model state (model_abi.cu)
  unsigned long long epoch = 0;  // bumped when uploaded layers or the scratch move
  // Expert-parallel receive side (oxg_moe_experts): kept apart from ws so
  // that sizing it for the received rows never discards the dispatch's
  // slot positions and weights that oxg_moe_combine reads.
  struct {
    void *base = nullptr;
    size_t bytes = 0;
    uint16_t *h_hi = nullptr, *h_lo = nullptr;
    int32_t *seg = nullptr;  // counts [256] then offsets [257]
  } ep;
  std::vector<int32_t> seg_host;
  // Arrival counters of the prefill GEMM2's fused combine, one per (token,
  // 128-row tile of H): zero between calls (each call leaves them at zero;
  // cleared again after a failed call). Kept apart from ws, whose layout
  // moves with the batch size.
  uint32_t *comb_cnt = nullptr;
  size_t comb_cnt_n = 0;
  // Host-buffer forwards of large batches run in token chunks whose copies
  // overlap the neighbouring chunks' compute (oxg_moe_forward_host).
  struct {
    cudaStream_t h2d = nullptr, d2h = nullptr;
    cudaEvent_t x_ready[2] = {}, x_free[2] = {}, y_ready[2] = {}, y_free[2] = {};
    void *buf = nullptr;
    size_t bytes = 0;
    int chunk = 0;  // tokens per chunk; 0: automatic, < 0: never chunk
  } pipe;
  // Expert parallelism over peer memory (oxg_ep_init / oxg_ep_connect).
  struct {
    bool init = false, connected = false;
    int layer = -1;
    oxg::EpLayout lay{};
    oxg::EpPeers peers{};
    void *sym = nullptr;  // this rank's symmetric buffer (exported)
    void *local = nullptr;  // h hi/lo [max_recv, I] x 2, segment table + pointers, counters
    uint16_t *h_hi = nullptr, *h_lo = nullptr;
    int32_t *seg = nullptr;
    float **seg_ptr = nullptr;
    uint32_t *done_ctr = nullptr;
    int *ok_word = nullptr;
    uint32_t epoch = 0;
    int I = 0;  // intermediate size the h buffers were sized for
    // decode-sized exchanges: the received rows in groups of at most 8 run
    // through the grouped decode kernels instead of the prefill GEMMs
    oxg::EpVirtual virt{};
    bool decode = false;   // the grouped kernels fit these widths
    int decode_tokens = 0;  // forwards of at most this many tokens receive on them (oxg_ep_set_decode_tokens)
    float *h_f32 = nullptr;  // [max_recv, I] f32 SwiGLU output of the grouped kernels
  } p2p;
};

namespace {

// Unmaps the peers' buffers and frees this rank's (callers synchronise ranks
// first, so no peer still writes into it).
void p2p_release(oxg_ctx *ctx) {
  auto &q = ctx->p2p;
  if (q.connected)
    for (int r = 0; r < q.lay.W; ++r)
      if (r != q.lay.rank && q.peers.base[r]) cudaIpcCloseMemHandle(q.peers.base[r]);
  if (q.sym) cudaFree(q.sym);
  if (q.local) cudaFree(q.local);
  q = {};
}

struct DeviceGuard {
  int prev = -1;
  bool ok = true;
  explicit DeviceGuard(int dev) {
    if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
    if (prev != dev) ok = cudaSetDevice(dev) == cudaSuccess;
  }
  ~DeviceGuard() {
    if (prev >= 0) cudaSetDevice(prev);
  }
};

int fail(oxg_ctx *ctx, int status, const char *fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  if (ctx)
    ctx->error = buf;
  else
    g_tls_error = buf;
  return status;
}

int cuda_fail(oxg_ctx *ctx, cudaError_t st, const char *what) {
  return fail(ctx, st == cudaErrorMemoryAllocation ? OXG_ERR_OOM : OXG_ERR_CUDA, "%s: %s (%s)",
              what, cudaGetErrorName(st), cudaGetErrorString(st));
}

#define OXG_CUDA(ctx, call, what)                      \
  do {                                                 \
    cudaError_t st_ = (call);                          \
    if (st_ != cudaSuccess) return cuda_fail(ctx, st_, what); \
  } while (0)

size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

int check_dims(oxg_ctx *ctx, const oxg_moe_dims *d) {
  if (!d) return fail(ctx, OXG_ERR_INVALID_ARG, "dims is NULL");
  if (d->hidden <= 0 || d->hidden % 32)
    return fail(ctx, OXG_ERR_SHAPE, "hidden must be a positive multiple of 32, got %d", d->hidden);
  if (d->intermediate <= 0 || d->intermediate % 32)
    return fail(ctx, OXG_ERR_SHAPE, "intermediate must be a positive multiple of 32, got %d",
                d->intermediate);
  if (d->n_experts <= 0 || d->n_experts > 256)
    return fail(ctx, OXG_ERR_SHAPE, "n_experts must be in [1, 256], got %d", d->n_experts);
  if (d->top_k <= 0 || d->top_k > 16 || d->top_k > d->n_experts)
    return fail(ctx, OXG_ERR_SHAPE, "top_k must be in [1, min(16, n_experts)], got %d", d->top_k);
  if (!(d->swiglu_limit > 0.f) || d->swiglu_limit > 128.f)
    return fail(ctx, OXG_ERR_INVALID_ARG, "swiglu_limit must be in (0, 128], got %g",
                (double)d->swiglu_limit);
  return OXG_OK;
}

// Scratch layout for T tokens of a layer with dims d.
size_t scratch_bytes(const oxg_moe_dims &d, int T, int n_sms, Scratch *s, char *base) {
  const size_t S = (size_t)T * d.top_k;
  size_t off = 0;
  auto take = [&](size_t bytes) {
    size_t o = off;
    off = align_up(off + bytes, 256);
    return base ? base + o : nullptr;
  };
  char *p_cnt = take(kCounterBytes);
  char *p_parts = take(oxg::flat_parts_bytes(n_sms));
  char *p_active = take((size_t)d.n_experts * 4), *p_nactive = take(4);
  char *p_idx = take(S * 4), *p_wts = take(S * 4), *p_sigma = take((size_t)T * 4);
  char *p_logits = take((size_t)T * d.n_experts * 4);
  char *p_counts = take((size_t)d.n_experts * 4), *p_offsets = take(((size_t)d.n_experts + 1) * 4);
  // positions run up to rows_cap when each expert's first position is padded
  // to a multiple of 128 (block-scaled prefill)
  const int rows_cap = oxg::mxf_rows_cap((int)S, d.n_experts);
  char *p_perm = take(std::max(S, (size_t)rows_cap) * 4), *p_slot = take(S * 4);
  char *p_h = take(S * d.intermediate * 4), *p_y = take(std::max(S, (size_t)rows_cap) * d.hidden * 4);
  char *p_xs = take((size_t)T * d.hidden * 2), *p_ys = take((size_t)T * d.hidden * 4);
  char *p_xp = take(S * d.hidden * 2), *p_hhi = take(S * d.intermediate * 2);
  char *p_hlo = take(S * d.intermediate * 2), *p_psc = take(S * 4);
  char *p_hist = take((size_t)oxg::router_mma_ctas(T) * d.n_experts * 4), *p_rank = take(S * 4);
  const size_t n_virt = (size_t)oxg::max_virtual(d.n_experts, T, d.top_k) + 1;
  char *p_vexp = take(n_virt * 4), *p_vpos = take(n_virt * 4), *p_vcnt = take(n_virt * 4), *p_nvirt = take(4);
  const size_t xq_b = (size_t)2 * T * d.hidden, xsf_b = (size_t)(d.hidden + 127) / 128 * 512;
  const size_t hq_b = 4 * S * d.intermediate;
  const size_t hsf_b = (size_t)d.n_experts * ((d.intermediate + 127) / 128) * 512;
  char *p_xq = take(xq_b), *p_xsf = take(xsf_b), *p_hq = take(hq_b), *p_hsf = take(hsf_b);
  char *p_tmask = take((size_t)d.n_experts * 4);
  const size_t rt = (size_t)rows_cap / 128, kt1 = (d.hidden + 127) / 128, kt2 = (d.intermediate + 127) / 128;
  char *p_pxq = take(2 * (size_t)rows_cap * d.hidden), *p_pxsf = take(2 * rt * kt1 * 512);
  char *p_phq = take(4 * (size_t)rows_cap * d.intermediate), *p_phsf = take(4 * rt * kt2 * 512);
  if (s && base) {
    s->pxq = (uint8_t *)p_pxq;
    s->pxsf = (uint8_t *)p_pxsf;
    s->phq = (uint8_t *)p_phq;
    s->phsf = (uint8_t *)p_phsf;
    s->rows_cap = rows_cap;
    s->tok_mask = (uint32_t *)p_tmask;
    s->xq = (uint8_t *)p_xq;
    s->xsf = (uint8_t *)p_xsf;
    s->hq = (uint8_t *)p_hq;
    s->hsf = (uint8_t *)p_hsf;
    s->xq_bytes = xq_b;
    s->xsf_bytes = xsf_b;
    s->hq_bytes = hq_b;
    s->hsf_bytes = hsf_b;
    s->done = (uint32_t *)p_cnt;
    s->err = (int *)(s->done + 1);
    s->band_done = s->done + 2;
    s->flat_cnt = s->band_done + kMaxBands;
    s->parts = (float4 *)p_parts;
    s->xp = (uint16_t *)p_xp;
    s->h_hi = (uint16_t *)p_hhi;
    s->h_lo = (uint16_t *)p_hlo;
    s->pos_scale = (float *)p_psc;
    s->active = (int32_t *)p_active;
    s->n_active = (int32_t *)p_nactive;
    s->idx = (int32_t *)p_idx;
    s->wts = (float *)p_wts;
    s->sigma = (int32_t *)p_sigma;
    s->logits = (float *)p_logits;
    s->counts = (int32_t *)p_counts;
    s->offsets = (int32_t *)p_offsets;
    s->perm = (int32_t *)p_perm;
    s->slot_pos = (int32_t *)p_slot;
    s->cta_hist = (int32_t *)p_hist;
    s->local_rank = (int32_t *)p_rank;
    s->v_expert = (int32_t *)p_vexp;
    s->v_pos0 = (int32_t *)p_vpos;
    s->v_count = (int32_t *)p_vcnt;
    s->n_virtual = (int32_t *)p_nvirt;
    s->h = (float *)p_h;
    s->y_slot = (float *)p_y;
    s->x_stage = (uint16_t *)p_xs;
    s->y_stage = (float *)p_ys;
  }
  return off;
}

int ensure_scratch(oxg_ctx *ctx, const oxg_moe_dims &d, int T) {
  const int Tc = T < 1 ? 1 : T;
  const size_t need = scratch_bytes(d, Tc, ctx->n_sms, nullptr, nullptr);
  const size_t key = ((size_t)Tc * 1000003u + (size_t)d.hidden) * 1000003u +
                     ((size_t)d.intermediate * 4099u + (size_t)d.n_experts * 17u + (size_t)d.top_k);
  auto zero_terms = [&]() -> int {
    if (ctx->ws.layout_key == key) return OXG_OK;
    OXG_CUDA(ctx, cudaMemsetAsync(ctx->ws.xq, 0, ctx->ws.xq_bytes, ctx->stream), "cudaMemsetAsync(xq)");
    OXG_CUDA(ctx, cudaMemsetAsync(ctx->ws.xsf, 0, ctx->ws.xsf_bytes, ctx->stream), "cudaMemsetAsync(xsf)");
    OXG_CUDA(ctx, cudaMemsetAsync(ctx->ws.hq, 0, ctx->ws.hq_bytes, ctx->stream), "cudaMemsetAsync(hq)");
    OXG_CUDA(ctx, cudaMemsetAsync(ctx->ws.hsf, 0, ctx->ws.hsf_bytes, ctx->stream), "cudaMemsetAsync(hsf)");
    ctx->ws.layout_key = key;
    return OXG_OK;
  };
  if (need <= ctx->ws.bytes) {
    scratch_bytes(d, Tc, ctx->n_sms, &ctx->ws, (char *)ctx->ws.base);
    return zero_terms();
  }
  if (ctx->ws.base) {
    OXG_CUDA(ctx, cudaStreamSynchronize(ctx->stream), "cudaStreamSynchronize");
    cudaFree(ctx->ws.base);
    ctx->ws = Scratch{};
    ctx->epoch += 1;
  }
  void *p = nullptr;
  OXG_CUDA(ctx, cudaMalloc(&p, need), "cudaMalloc(scratch)");
  ctx->ws.base = p;
  ctx->ws.bytes = need;
  scratch_bytes(d, Tc, ctx->n_sms, &ctx->ws, (char *)p);
  OXG_CUDA(ctx, cudaMemsetAsync(p, 0, kCounterBytes, ctx->stream), "cudaMemsetAsync(counters)");
  return zero_terms();
}

Layer *get_layer(oxg_ctx *ctx, int layer) {
  if (layer < 0 || layer >= (int)ctx->layers.size() || !ctx->layers[layer].present) return nullptr;
  return &ctx->layers[layer];
}

void free_layer(Layer &L) {
  if (L.block) cudaFree(L.block);
  L = Layer{};
}

oxg::MoeDeviceWeights device_weights(const Layer &L) {
  oxg::MoeDeviceWeights w{};
  w.H = L.dims.hidden;
  w.I = L.dims.intermediate;
  w.E = L.dims.n_experts;
  w.k = L.dims.top_k;
  w.alpha = L.dims.swiglu_alpha;
  w.limit = L.dims.swiglu_limit;
  w.router_w = L.router_w;
  w.router_b = L.router_b;
  w.w1 = L.w1;
  w.b1 = L.b1;
  w.w2 = L.w2;
  w.b2 = L.b2;
  return w;
}

oxg::MxfWeights mxf_weights(const Layer &L) {
  oxg::MxfWeights w{};
  w.H = L.dims.hidden;
  w.I = L.dims.intermediate;
  w.E = L.dims.n_experts;
  w.k = L.dims.top_k;
  w.alpha = L.dims.swiglu_alpha;
  w.limit = L.dims.swiglu_limit;
  w.q1 = L.q1;
  w.a1 = L.a1;
  w.b1 = L.b1;
  w.q2 = L.q2;
  w.a2 = L.a2;
  w.b2 = L.b2;
  return w;
}

// Runs one kernel launcher, counting the launch and, when profiling is on,
// bracketing it with CUDA events on the context's stream.
template <class F>
cudaError_t launch(oxg_ctx *ctx, const char *name, F &&fn) {
  cudaEvent_t a = nullptr;
  if (ctx->prof.on) {
    a = ctx->prof.get();
    cudaEventRecord(a, ctx->stream);
  }
  cudaError_t st = fn();
  if (st == cudaSuccess) ctx->launches += 1;
  if (ctx->prof.on) {
    cudaEvent_t b = ctx->prof.get();
    cudaEventRecord(b, ctx->stream);
    ctx->prof.recs.push_back(Profiler::Rec{name, a, b});
  }
  return st;
}

// Routing of T tokens. Batches beyond the fused small-batch path go to the
// tensor-core router when the shape allows, which also leaves the first half
// of the counting sort in the scratch (*ranked = true) for scatter.
int route(oxg_ctx *ctx, Layer &L, const uint16_t *x, int T, int32_t *idx, float *wts,
          float *logits, bool *ranked = nullptr) {
  const oxg_moe_dims &d = L.dims;
  const bool mma = T > oxg::kMaxRouteTokens && oxg::router_mma_supported(d.hidden, d.n_experts, d.top_k);
  if (ranked) *ranked = mma;
  if (mma) {
    OXG_CUDA(ctx, launch(ctx, "router_mma", [&] {
               return oxg::launch_router_mma(x, L.router_w, L.router_b, T, d.hidden, d.n_experts,
                                             d.top_k, idx, wts, logits, ctx->ws.sigma,
                                             ctx->ws.cta_hist, ctx->ws.local_rank, ctx->stream, ctx->ws.err);
             }),
             "router_mma launch");
    ctx->prefill_pending = true;  // its bounded waits report a timeout in the error word
    return OXG_OK;
  }
  OXG_CUDA(ctx, launch(ctx, "router_topk", [&] {
             return oxg::launch_router_topk(x, L.router_w, L.router_b, T, d.hidden, d.n_experts,
                                            d.top_k, idx, wts, logits, ctx->ws.sigma, ctx->stream);
           }),
           "router_topk launch");
  return OXG_OK;
}

// Expert-sorted positions of the T * k slots (and, for prefill, the f16
// operand rows): from the router's ranks when it left them, else the
// single-CTA counting sort (and a separate gather).
int sort_slots(oxg_ctx *ctx, Layer &L, const uint16_t *x, int T, bool ranked, bool prefill,
               uint16_t *xp = nullptr, float *pos_scale = nullptr) {
  const oxg_moe_dims &d = L.dims;
  const int S = T * d.top_k;
  if (!xp) xp = ctx->ws.xp;
  if (!pos_scale) pos_scale = ctx->ws.pos_scale;
  if (ranked) {
    OXG_CUDA(ctx, launch(ctx, prefill ? "scatter_gather" : "scatter", [&] {
               return oxg::launch_scatter(ctx->ws.cta_hist, oxg::router_mma_ctas(T), ctx->ws.idx,
                                          ctx->ws.local_rank, T, d.top_k, d.n_experts,
                                          ctx->ws.counts, ctx->ws.offsets, ctx->ws.perm,
                                          ctx->ws.slot_pos, x, ctx->ws.sigma, d.hidden,
                                          prefill ? xp : nullptr, pos_scale, ctx->stream);
             }),
             "scatter launch");
    return OXG_OK;
  }
  OXG_CUDA(ctx, launch(ctx, "permute", [&] {
             return oxg::launch_permute(ctx->ws.idx, S, d.n_experts, ctx->ws.counts,
                                        ctx->ws.offsets, ctx->ws.perm, ctx->ws.slot_pos,
                                        ctx->stream);
           }),
           "permute launch");
  if (prefill)
    OXG_CUDA(ctx, launch(ctx, "gather_f16", [&] {
               return oxg::launch_gather_f16(x, ctx->ws.perm, ctx->ws.sigma, S, d.hidden, d.top_k,
                                             xp, pos_scale, ctx->ws.err, ctx->stream);
             }),
             "gather launch");
  return OXG_OK;
}

// Expected number of distinct experts T tokens route to with uniform routing:
// E * (1 - (1 - k/E)^T), at least 1 and at most min(E, T*k).
int expected_active(int E, int k, int T) {
  const double p = 1.0 - (double)k / (double)E;
  double v = (double)E * (1.0 - std::pow(p, (double)T));
  int n = (int)std::ceil(v - 1e-9);
  const int mx = std::min(E, T * k);
  return std::max(1, std::min(n, mx));
}

// Decode fast path (T <= kMaxRouteTokens): fused routing + permutation, then
// the two expert kernels, all chained with programmatic dependent launch; the
// weighted combine is done by the mlp2 kernel.
int forward_small(oxg_ctx *ctx, Layer &L, const uint16_t *x, int T, float *y, bool mxf) {
  const oxg_moe_dims &d = L.dims;
  const oxg::MoeDeviceWeights w = device_weights(L);
  const int exp_active = expected_active(d.n_experts, d.top_k, T);
  oxg::DecodeSched sched{};
  sched.active = ctx->ws.active;
  sched.n_active = ctx->ws.n_active;
  sched.max_active = std::min(d.n_experts, T * d.top_k);
  sched.bands1 = oxg::decode_bands(2 * d.intermediate, exp_active, ctx->n_sms);
  sched.bands2 = oxg::decode_bands(d.hidden, exp_active, ctx->n_sms);
  sched.n_sms = ctx->n_sms;
  sched.pdl = true;
  sched.err = ctx->ws.err;
  sched.parts = ctx->ws.parts;
  sched.flat_cnt = ctx->ws.flat_cnt;
  sched.exp_active = exp_active;
  sched.v_expert = ctx->ws.v_expert;
  sched.v_pos0 = ctx->ws.v_pos0;
  sched.v_count = ctx->ws.v_count;
  sched.n_virtual = ctx->ws.n_virtual;
  sched.max_virtual = oxg::max_virtual(d.n_experts, T, d.top_k);
  // counters the mlp2 kernel's fused combine uses (zeroed by route_small):
  // per 128-row band quarter (block-scaled), per band (f16 per-expert bands),
  // per 16-row tile (f16 flat split at most 8 tokens)
  const int n_bands = mxf ? 4 * ((d.hidden + 127) / 128)
                          : std::max(sched.bands2, d.hidden / 16);
  if (n_bands > kMaxBands) return fail(ctx, OXG_ERR_UNSUPPORTED, "too many row bands (%d)", n_bands);
  oxg::RouteSmallArgs ra{};
  ra.x = x;
  ra.router_w = L.router_w;
  ra.router_b = L.router_b;
  ra.T = T;
  ra.H = d.hidden;
  ra.E = d.n_experts;
  ra.k = d.top_k;
  ra.logits = ctx->ws.logits;
  ra.sigma = ctx->ws.sigma;
  ra.idx = ctx->ws.idx;
  ra.wts = ctx->ws.wts;
  ra.counts = ctx->ws.counts;
  ra.offsets = ctx->ws.offsets;
  ra.perm = ctx->ws.perm;
  ra.slot_pos = ctx->ws.slot_pos;
  ra.active = ctx->ws.active;
  ra.n_active = ctx->ws.n_active;
  ra.done = ctx->ws.done;
  ra.band_done = ctx->ws.band_done;
  ra.n_bands = n_bands;
  ra.v_expert = ctx->ws.v_expert;
  ra.v_pos0 = ctx->ws.v_pos0;
  ra.v_count = ctx->ws.v_count;
  ra.n_virtual = ctx->ws.n_virtual;
  if (mxf) {
    ra.xq = ctx->ws.xq;
    ra.xsf = ctx->ws.xsf;
    ra.tok_mask = ctx->ws.tok_mask;
  }
  OXG_CUDA(ctx, launch(ctx, "route_small", [&] { return oxg::launch_route_small(ra, ctx->stream, true); }),
           "route_small launch");
  if (mxf) {
    const oxg::MxfWeights mw = mxf_weights(L);
    oxg::MxfScratch ms{};
    ms.active = ctx->ws.active;
    ms.n_active = ctx->ws.n_active;
    ms.counts = ctx->ws.counts;
    ms.offsets = ctx->ws.offsets;
    ms.idx = ctx->ws.idx;
    ms.slot_pos = ctx->ws.slot_pos;
    ms.tok_mask = ctx->ws.tok_mask;
    ms.wts = ctx->ws.wts;
    ms.xq = ctx->ws.xq;
    ms.xsf = ctx->ws.xsf;
    ms.hq = ctx->ws.hq;
    ms.hsf = ctx->ws.hsf;
    ms.y_slot = ctx->ws.y_slot;
    ms.band_done = ctx->ws.band_done;
    ms.y = y;
    ms.err = ctx->ws.err;
    OXG_CUDA(ctx, launch(ctx, "mxf_mlp1", [&] {
               return oxg::launch_mxf_mlp1(mw, ms, T, ctx->n_sms, true, ctx->stream);
             }),
             "mxf mlp1 launch");
    OXG_CUDA(ctx, launch(ctx, "mxf_mlp2", [&] {
               return oxg::launch_mxf_mlp2(mw, ms, T, ctx->n_sms, true, ctx->stream);
             }),
             "mxf mlp2 launch");
    ctx->prefill_pending = true;  // the kernels report wait timeouts in the error word
    return OXG_OK;
  }
  OXG_CUDA(ctx, launch(ctx, "moe_mlp1_decode", [&] {
             return oxg::launch_moe_mlp1_sched(w, x, ctx->ws.perm, ctx->ws.sigma, ctx->ws.idx,
                                               ctx->ws.counts, ctx->ws.offsets, sched, T, ctx->ws.h,
                                               ctx->stream);
           }),
           "mlp1 launch");
  OXG_CUDA(ctx, launch(ctx, "moe_mlp2_decode", [&] {
             return oxg::launch_moe_mlp2_sched(w, ctx->ws.h, ctx->ws.counts, ctx->ws.offsets, sched,
                                               ctx->ws.band_done, T, ctx->ws.slot_pos,
                                               ctx->ws.wts, ctx->ws.y_slot, y, ctx->stream);
           }),
           "mlp2 launch");
  ctx->prefill_pending = true;  // the weight streams report wait timeouts in the error word
  return OXG_OK;
}

// Prefill path: routing and permutation, the slot-ordered f16 activations,
// the two tcgen05 grouped GEMMs and the weighted combine.
int forward_prefill(oxg_ctx *ctx, Layer &L, const uint16_t *x, int T, float *y, bool mxf) {
  const oxg_moe_dims &d = L.dims;
  const int S = T * d.top_k;
  bool ranked = false;
  int rc = route(ctx, L, x, T, ctx->ws.idx, ctx->ws.wts, ctx->ws.logits, &ranked);
  if (rc) return rc;
  if (mxf) {
    // block-scaled path: padded positions with the E4M3 x terms, the two
    // tcgen05 block-scaled GEMMs, the combine
    const oxg::ScatterTerms terms{ctx->ws.pxq, ctx->ws.pxsf, ctx->ws.rows_cap};
    if (ranked) {
      OXG_CUDA(ctx, launch(ctx, "scatter_e4m3", [&] {
                 return oxg::launch_scatter(ctx->ws.cta_hist, oxg::router_mma_ctas(T), ctx->ws.idx,
                                            ctx->ws.local_rank, T, d.top_k, d.n_experts, ctx->ws.counts,
                                            ctx->ws.offsets, ctx->ws.perm, ctx->ws.slot_pos, x, ctx->ws.sigma,
                                            d.hidden, nullptr, nullptr, ctx->stream, &terms);
               }),
               "scatter launch");
    } else {
      OXG_CUDA(ctx, launch(ctx, "permute", [&] {
                 return oxg::launch_permute(ctx->ws.idx, S, d.n_experts, ctx->ws.counts, ctx->ws.offsets,
                                            ctx->ws.perm, ctx->ws.slot_pos, ctx->stream, 128);
               }),
               "permute launch");
      OXG_CUDA(ctx, launch(ctx, "gather_e4m3", [&] {
                 return oxg::launch_gather_e4m3(x, ctx->ws.slot_pos, S, d.top_k, d.hidden, terms, ctx->stream);
               }),
               "gather launch");
    }
    oxg::MxfPrefillIO io{};
    io.counts = ctx->ws.counts;
    io.offsets = ctx->ws.offsets;
    io.xq = ctx->ws.pxq;
    io.xsf = ctx->ws.pxsf;
    io.hq = ctx->ws.phq;
    io.hsf = ctx->ws.phsf;
    io.rows_cap = ctx->ws.rows_cap;
    io.y_slot = ctx->ws.y_slot;
    io.err = ctx->ws.err;
    const oxg::MxfWeights mw = mxf_weights(L);
    OXG_CUDA(ctx, launch(ctx, "mxf_gemm1", [&] {
               return oxg::launch_mxf_prefill(mw, L.p1, io, 1, ctx->n_sms, ctx->stream);
             }),
             "mxf gemm1 launch");
    OXG_CUDA(ctx, launch(ctx, "mxf_gemm2", [&] {
               return oxg::launch_mxf_prefill(mw, L.p2, io, 2, ctx->n_sms, ctx->stream);
             }),
             "mxf gemm2 launch");
    OXG_CUDA(ctx, launch(ctx, "combine", [&] {
               return oxg::launch_combine(ctx->ws.y_slot, ctx->ws.slot_pos, ctx->ws.wts, T, d.hidden, d.top_k, y,
                                          ctx->stream);
             }),
             "combine launch");
    ctx->prefill_pending = true;
    return OXG_OK;
  }
  if ((rc = sort_slots(ctx, L, x, T, ranked, true))) return rc;
  // the fused combine's counters: T x (128-row tiles of H), zero on entry
  const size_t n_cnt = (size_t)T * oxg::prefill_comb_mtiles(d.hidden);
  if (ctx->comb_cnt_n < n_cnt) {
    OXG_CUDA(ctx, cudaStreamSynchronize(ctx->stream), "cudaStreamSynchronize");
    if (ctx->comb_cnt) cudaFree(ctx->comb_cnt);
    ctx->comb_cnt = nullptr;
    ctx->comb_cnt_n = 0;
    OXG_CUDA(ctx, cudaMalloc(&ctx->comb_cnt, n_cnt * sizeof(uint32_t)), "cudaMalloc(combine counters)");
    ctx->comb_cnt_n = n_cnt;
    OXG_CUDA(ctx, cudaMemsetAsync(ctx->comb_cnt, 0, n_cnt * sizeof(uint32_t), ctx->stream),
             "cudaMemsetAsync(combine counters)");
    ctx->epoch += 1;
  }
  const oxg::MoeDeviceWeights w = device_weights(L);
  oxg::PrefillIO io{};
  io.S = S;
  io.counts = ctx->ws.counts;
  io.offsets = ctx->ws.offsets;
  io.n_segments = d.n_experts;
  io.weight_mod = d.n_experts;
  io.xp = ctx->ws.xp;
  io.pos_scale = ctx->ws.pos_scale;
  io.h_hi = ctx->ws.h_hi;
  io.h_lo = ctx->ws.h_lo;
  io.y_slot = ctx->ws.y_slot;
  io.err = ctx->ws.err;
  const bool fused = d.top_k <= oxg::kPrefillCombineMaxK;
  if (fused) {  // GEMM2 sums each token's k rows (the weighted combine) itself
    io.y = y;
    io.perm = ctx->ws.perm;
    io.slot_pos = ctx->ws.slot_pos;
    io.wts = ctx->ws.wts;
    io.comb_cnt = ctx->comb_cnt;
    io.topk = d.top_k;
  }
  OXG_CUDA(ctx, launch(ctx, "moe_mlp1_prefill", [&] {
             return oxg::launch_prefill_mlp1(w, io, ctx->n_sms, ctx->stream);
           }),
           "prefill mlp1 launch");
  OXG_CUDA(ctx, launch(ctx, "moe_mlp2_prefill", [&] {
             return oxg::launch_prefill_mlp2(w, io, ctx->n_sms, ctx->stream);
           }),
           "prefill mlp2 launch");
  if (!fused)
    OXG_CUDA(ctx, launch(ctx, "combine", [&] {
               return oxg::launch_combine(ctx->ws.y_slot, ctx->ws.slot_pos, ctx->ws.wts, T, d.hidden, d.top_k, y,
                                          ctx->stream);
             }),
             "combine launch");
  ctx->prefill_pending = true;
  return OXG_OK;
}

int forward_device(oxg_ctx *ctx, Layer &L, const uint16_t *x, int T, float *y, int mode) {
  const oxg_moe_dims &d = L.dims;
  const int S = T * d.top_k;
  // AUTO: the measured-faster kernels first. Prefill: the f16 tcgen05 GEMMs
  // when every scale is f16-exact, else the block-scaled GEMMs (any scale).
  // Decode: the mma.sync kernels (the block-scaled decode kernels are
  // selected with OXG_MODE_MXF4).
  const bool mxf_prefill = L.mxf_ok && oxg::mxf_prefill_supported(d.hidden, d.intermediate, d.n_experts);
  if ((mode == OXG_MODE_MXF4 && T > oxg::kMaxMxfTokens) ||
      (mode == OXG_MODE_AUTO && T > oxg::kMaxRouteTokens && !L.prefill_ok && mxf_prefill))
    return forward_prefill(ctx, L, x, T, y, true);
  if (mode == OXG_MODE_PREFILL || (mode == OXG_MODE_AUTO && T > oxg::kMaxRouteTokens && L.prefill_ok))
    return forward_prefill(ctx, L, x, T, y, false);
  const bool mxf = mode == OXG_MODE_MXF4;
  if (T <= oxg::kMaxRouteTokens) return forward_small(ctx, L, x, T, y, mxf);
  bool ranked = false;
  int rc = route(ctx, L, x, T, ctx->ws.idx, ctx->ws.wts, ctx->ws.logits, &ranked);
  if (rc) return rc;
  if ((rc = sort_slots(ctx, L, x, T, ranked, false))) return rc;
  const oxg::MoeDeviceWeights w = device_weights(L);
  OXG_CUDA(ctx, launch(ctx, "moe_mlp1_decode", [&] {
             return oxg::launch_moe_mlp1_decode(w, x, ctx->ws.perm, ctx->ws.sigma, ctx->ws.counts,
                                                ctx->ws.offsets, S, 0, d.n_experts, ctx->ws.h,
                                                ctx->ws.err, ctx->stream);
           }),
           "mlp1 launch");
  OXG_CUDA(ctx, launch(ctx, "moe_mlp2_decode", [&] {
             return oxg::launch_moe_mlp2_decode(w, ctx->ws.h, ctx->ws.counts, ctx->ws.offsets, S,
                                                0, d.n_experts, ctx->ws.y_slot, ctx->ws.err, ctx->stream);
           }),
           "mlp2 launch");
  OXG_CUDA(ctx, launch(ctx, "combine", [&] {
             return oxg::launch_combine(ctx->ws.y_slot, ctx->ws.slot_pos, ctx->ws.wts, T,
                                        d.hidden, d.top_k, y, ctx->stream);
           }),
           "combine launch");
  ctx->prefill_pending = true;
  return OXG_OK;
}

// Reads (and clears) the prefill kernels' timeout code after the work has run.
int read_pipeline_error(oxg_ctx *ctx) {
  if (!ctx->prefill_pending || !ctx->ws.err) return OXG_OK;
  int h = 0;
  OXG_CUDA(ctx, cudaMemcpyAsync(&h, ctx->ws.err, sizeof(int), cudaMemcpyDeviceToHost, ctx->stream),
           "read pipeline status");
  OXG_CUDA(ctx, cudaStreamSynchronize(ctx->stream), "cudaStreamSynchronize");
  ctx->prefill_pending = false;
  if (h) {
    cudaMemsetAsync(ctx->ws.err, 0, sizeof(int), ctx->stream);
    // a pipeline that gave up may have left combine counters part-way
    if (ctx->comb_cnt) cudaMemsetAsync(ctx->comb_cnt, 0, ctx->comb_cnt_n * sizeof(uint32_t), ctx->stream);
    if (h == 50)
      return fail(ctx, OXG_ERR_STATE, "another rank reported a failed expert-parallel step");
    if (h == 51)
      return fail(ctx, OXG_ERR_SHAPE, "expert-parallel receive capacity exceeded (raise max_recv_rows)");
    return fail(ctx, h >= 100 ? OXG_ERR_CUDA : OXG_ERR_TIMEOUT,
                h >= 100 ? "prefill self-check failed (code %d)" : "pipeline wait timed out (stage %d)", h);
  }
  return OXG_OK;
}

int check_forward_args(oxg_ctx *ctx, int layer, const void *x, int T, const void *y, int mode,
                       int precision, Layer **out) {
  if (!ctx) return fail(nullptr, OXG_ERR_INVALID_ARG, "ctx is NULL");
  Layer *L = get_layer(ctx, layer);
  if (!L) return fail(ctx, OXG_ERR_STATE, "layer %d has not been uploaded", layer);
  if (L->sharded())
    return fail(ctx, OXG_ERR_STATE,
                "layer %d holds experts [%d, %d) only: use oxg_moe_dispatch / oxg_moe_experts / "
                "oxg_moe_combine",
                layer, L->expert_begin, L->expert_begin + L->expert_count);
  if (T < 0) return fail(ctx, OXG_ERR_SHAPE, "n_tokens must be >= 0, got %d", T);
  if (T > 0 && (!x || !y)) return fail(ctx, OXG_ERR_INVALID_ARG, "x and y must be non-NULL");
  if (mode != OXG_MODE_AUTO && mode != OXG_MODE_DECODE && mode != OXG_MODE_PREFILL &&
      mode != OXG_MODE_MXF4)
    return fail(ctx, OXG_ERR_INVALID_ARG, "unknown mode %d", mode);
  if (mode == OXG_MODE_MXF4 &&
      (!L->mxf_ok ||
       (T <= oxg::kMaxMxfTokens
            ? !oxg::mxf_decode_supported(L->dims.hidden, L->dims.intermediate, T, L->dims.top_k)
            : !oxg::mxf_prefill_supported(L->dims.hidden, L->dims.intermediate, L->dims.n_experts))))
    return fail(ctx, OXG_ERR_UNSUPPORTED,
                "MXF4 mode needs hidden and intermediate multiples of 64 (>= 128), at most 256 experts and no "
                "E8M0 scale 255; got n_tokens %d, scales in [%u, %u]",
                T, L->scale_min, L->scale_max);
  if (mode == OXG_MODE_PREFILL && !L->prefill_ok)
    return fail(ctx, OXG_ERR_UNSUPPORTED,
                "prefill mode needs hidden and intermediate multiples of 64 and E8M0 scales "
                "0 or in [104, 140]; this layer has scales in [%u, %u]",
                L->scale_min, L->scale_max);
  if (precision != OXG_PRECISION_PARITY)
    return fail(ctx, OXG_ERR_UNSUPPORTED, "unknown precision %d", precision);
  *out = L;
  return OXG_OK;
}

}  // namespace

namespace oxg {

bool ctx_layer(oxg_ctx *ctx, int layer, MoeDeviceWeights *w, int *device, cudaStream_t *stream) {
  Layer *L = get_layer(ctx, layer);
  if (!L) {
    fail(ctx, OXG_ERR_STATE, "layer %d has not been uploaded", layer);
    return false;
  }
  *w = device_weights(*L);
  *device = ctx->device;
  *stream = ctx->stream;
  return true;
}

bool ctx_layer_experts(oxg_ctx *ctx, int layer, int *begin, int *count, int *n_experts) {
  Layer *L = get_layer(ctx, layer);
  if (!L) return false;
  *begin = L->expert_begin;
  *count = L->expert_count;
  *n_experts = L->dims.n_experts;
  return true;
}

int ctx_error(oxg_ctx *ctx, int status, const char *msg) { return fail(ctx, status, "%s", msg); }

int ctx_device(const oxg_ctx *ctx) { return ctx->device; }
cudaStream_t ctx_stream(const oxg_ctx *ctx) { return ctx->stream; }
int ctx_n_sms(const oxg_ctx *ctx) { return ctx->n_sms; }

int ctx_moe_forward(oxg_ctx *ctx, int layer, const uint16_t *x, int T, float *y) {
  return oxg_moe_forward(ctx, layer, x, T, y, OXG_MODE_AUTO, OXG_PRECISION_PARITY);
}

int ctx_moe_reserve(oxg_ctx *ctx, int layer, int T) { return oxg_moe_reserve(ctx, layer, T); }

int ctx_moe_ep_hidden(oxg_ctx *ctx, int layer) {
  Layer *L = get_layer(ctx, layer);
  const auto &q = ctx->p2p;
  if (!L || !L->sharded() || !q.connected) return 0;
  if (L->expert_begin != q.lay.rank * q.lay.per || L->expert_count != q.lay.per || L->dims.n_experts != q.lay.E ||
      L->dims.hidden != q.lay.H || L->dims.intermediate != q.I || L->dims.top_k != q.lay.k)
    return 0;
  return L->dims.hidden;
}

int ctx_moe_forward_ep(oxg_ctx *ctx, int layer, const uint16_t *x, int T, float *y) {
  return oxg_moe_forward_ep(ctx, layer, x, T, y);
}

int ctx_moe_hidden(oxg_ctx *ctx, int layer) {
  Layer *L = get_layer(ctx, layer);
  return L && !L->sharded() ? L->dims.hidden : 0;
}

int ctx_moe_topk(oxg_ctx *ctx, int layer) {
  Layer *L = get_layer(ctx, layer);
  return L ? L->dims.top_k : 0;
}

const int32_t *ctx_moe_last_idx(oxg_ctx *ctx) { return ctx->ws.idx; }

void *ctx_prof_begin(oxg_ctx *ctx) {
  if (!ctx->prof.on) return nullptr;
  cudaEvent_t a = ctx->prof.get();
  cudaEventRecord(a, ctx->stream);
  return (void *)a;
}

void ctx_prof_end(oxg_ctx *ctx, const char *name, void *begin, cudaError_t st) {
  if (st == cudaSuccess) ctx->launches += 1;
  if (ctx->prof.on && begin) {
    cudaEvent_t b = ctx->prof.get();
    cudaEventRecord(b, ctx->stream);
    ctx->prof.recs.push_back(Profiler::Rec{name, (cudaEvent_t)begin, b});
  }
}

ModelState *&ctx_model(oxg_ctx *ctx) { return ctx->model; }
unsigned long long ctx_epoch(const oxg_ctx *ctx) { return ctx->epoch; }
bool &ctx_profile_flag(oxg_ctx *ctx) { return ctx->prof.on; }
void ctx_add_launches(oxg_ctx *ctx, long long n) { ctx->launches += n; }
long long ctx_launch_count(const oxg_ctx *ctx) { return ctx->launches; }

}  // namespace oxg

extern "C" {

int oxg_abi_version(void) { return OXG_ABI_VERSION; }

const char *oxg_status_string(int status) {
  switch (status) {
    case OXG_OK: return "ok";
    case OXG_ERR_INVALID_ARG: return "invalid argument";
    case OXG_ERR_SHAPE: return "shape mismatch";
    case OXG_ERR_CUDA: return "CUDA error";
    case OXG_ERR_NCCL: return "NCCL error";
    case OXG_ERR_TIMEOUT: return "timeout";
    case OXG_ERR_STATE: return "invalid state";
    case OXG_ERR_UNSUPPORTED: return "unsupported";
    case OXG_ERR_OOM: return "out of device memory";
    default: return "unknown status";
  }
}

int oxg_ctx_create(int device, oxg_ctx **out) {
  if (!out) return fail(nullptr, OXG_ERR_INVALID_ARG, "out is NULL");
  *out = nullptr;
  int n = 0;
  cudaError_t st = cudaGetDeviceCount(&n);
  if (st != cudaSuccess) return cuda_fail(nullptr, st, "cudaGetDeviceCount");
  if (device < 0 || device >= n)
    return fail(nullptr, OXG_ERR_INVALID_ARG, "device %d out of range (%d devices)", device, n);
  DeviceGuard g(device);
  if (!g.ok) return fail(nullptr, OXG_ERR_CUDA, "cudaSetDevice(%d) failed", device);
  cudaDeviceProp prop;
  st = cudaGetDeviceProperties(&prop, device);
  if (st != cudaSuccess) return cuda_fail(nullptr, st, "cudaGetDeviceProperties");
  if (prop.major != 10)
    return fail(nullptr, OXG_ERR_UNSUPPORTED,
                "device %d is sm_%d%d; this library is built for sm_100a (B200) only", device,
                prop.major, prop.minor);
  oxg_ctx *ctx = new (std::nothrow) oxg_ctx();
  if (!ctx) return fail(nullptr, OXG_ERR_OOM, "host allocation failed");
  ctx->device = device;
  ctx->n_sms = prop.multiProcessorCount;
  st = cudaStreamCreateWithFlags(&ctx->own_stream, cudaStreamNonBlocking);
  if (st != cudaSuccess) {
    delete ctx;
    return cuda_fail(nullptr, st, "cudaStreamCreate");
  }
  ctx->stream = ctx->own_stream;
  *out = ctx;
  return OXG_OK;
}

int oxg_ctx_destroy(oxg_ctx *ctx) {
  if (!ctx) return OXG_OK;
  DeviceGuard g(ctx->device);
  if (ctx->stream) cudaStreamSynchronize(ctx->stream);
  oxg::model_free(ctx);
  for (Layer &L : ctx->layers) free_layer(L);
  if (ctx->ws.base) cudaFree(ctx->ws.base);
  if (ctx->comb_cnt) cudaFree(ctx->comb_cnt);
  if (ctx->ep.base) cudaFree(ctx->ep.base);
  if (ctx->pipe.h2d) cudaStreamSynchronize(ctx->pipe.h2d);
  if (ctx->pipe.d2h) cudaStreamSynchronize(ctx->pipe.d2h);
  for (int b = 0; b < 2; ++b) {
    if (ctx->pipe.x_ready[b]) cudaEventDestroy(ctx->pipe.x_ready[b]);
    if (ctx->pipe.x_free[b]) cudaEventDestroy(ctx->pipe.x_free[b]);
    if (ctx->pipe.y_ready[b]) cudaEventDestroy(ctx->pipe.y_ready[b]);
    if (ctx->pipe.y_free[b]) cudaEventDestroy(ctx->pipe.y_free[b]);
  }
  if (ctx->pipe.h2d) cudaStreamDestroy(ctx->pipe.h2d);
  if (ctx->pipe.d2h) cudaStreamDestroy(ctx->pipe.d2h);
  if (ctx->pipe.buf) cudaFree(ctx->pipe.buf);
  p2p_release(ctx);
  ctx->prof.destroy();
  if (ctx->own_stream) cudaStreamDestroy(ctx->own_stream);
  delete ctx;
  return OXG_OK;
}

const char *oxg_last_error(const oxg_ctx *ctx) {
  return ctx ? ctx->error.c_str() : g_tls_error.c_str();
}

int oxg_ctx_set_stream(oxg_ctx *ctx, void *stream) {
  if (!ctx) return fail(nullptr, OXG_ERR_INVALID_ARG, "ctx is NULL");
  ctx->stream = (cudaStream_t)stream;  // NULL is the legacy default stream
  return OXG_OK;
}

void *oxg_ctx_get_stream(const oxg_ctx *ctx) { return ctx ? (void *)ctx->stream : nullptr; }

int oxg_sync(oxg_ctx *ctx) {
  if (!ctx) return fail(nullptr, OXG_ERR_INVALID_ARG, "ctx is NULL");
  DeviceGuard g(ctx->device);
  OXG_CUDA(ctx, cudaStreamSynchronize(ctx->stream), "cudaStreamSynchronize");
  const int rc = read_pipeline_error(ctx);
  if (rc) return rc;
  return oxg::model_check_error(ctx);
}

int oxg_dequant_mxfp4(oxg_ctx *ctx, const uint8_t *blocks, size_t n_block_bytes,
                      const void *scales, size_t n_scales, int scale_fmt, size_t rows, size_t cols,
                      uint16_t *out) {
  if (!ctx) return fail(nullptr, OXG_ERR_INVALID_ARG, "ctx is NULL");
  // Same checks, order and wording as src/mxfp4.rs:16-33.
  if (cols % 32 != 0) return fail(ctx, OXG_ERR_SHAPE, "cols must be divisible by 32, got %zu", cols);
  if (cols != 0 && rows > SIZE_MAX / cols)
    return fail(ctx, OXG_ERR_SHAPE, "rows * cols overflows: %zu x %zu", rows, cols);
  const size_t expected_blocks = rows * cols / 2;
  if (n_block_bytes != expected_blocks)
    return fail(ctx, OXG_ERR_SHAPE, "blocks length mismatch: expected %zu, got %zu",
                expected_blocks, n_block_bytes);
  const size_t expected_scales = rows * (cols / 32);
  if (n_scales != expected_scales)
    return fail(ctx, OXG_ERR_SHAPE, "scales length mismatch: expected %zu, got %zu",
                expected_scales, n_scales);
  if (scale_fmt != OXG_SCALE_E8M0 && scale_fmt != OXG_SCALE_BF16)
    return fail(ctx, OXG_ERR_INVALID_ARG, "unknown scale format %d", scale_fmt);
  if (expected_scales == 0) return OXG_OK;
  if (!blocks || !scales || !out)
    return fail(ctx, OXG_ERR_INVALID_ARG, "blocks, scales and out must be non-NULL");
  if (scale_fmt == OXG_SCALE_BF16 && ((uintptr_t)scales & 1))
    return fail(ctx, OXG_ERR_INVALID_ARG, "bf16 scales must be 2-byte aligned");
  if ((uintptr_t)out & 1) return fail(ctx, OXG_ERR_INVALID_ARG, "out must be 2-byte aligned");
  DeviceGuard g(ctx->device);
  OXG_CUDA(ctx, launch(ctx, "dequant_mxfp4", [&] {
             return oxg::launch_dequant_mxfp4(blocks, scales, scale_fmt, expected_scales, out,
                                              ctx->stream);
           }),
           "dequant launch");
  return OXG_OK;
}

int oxg_swiglu(oxg_ctx *ctx, const float *gate, const float *up, size_t n, float alpha,
               float limit, float *out) {
  if (!ctx) return fail(nullptr, OXG_ERR_INVALID_ARG, "ctx is NULL");
  if (n == 0) return OXG_OK;
  if (!gate || !up || !out) return fail(ctx, OXG_ERR_INVALID_ARG, "gate, up and out must be non-NULL");
  DeviceGuard g(ctx->device);
  OXG_CUDA(ctx, launch(ctx, "swiglu", [&] {
             return oxg::launch_swiglu(gate, up, n, alpha, limit, out, ctx->stream);
           }),
           "swiglu launch");
  return OXG_OK;
}

namespace {
int upload_impl(oxg_ctx *ctx, int layer, const oxg_moe_dims *dims, const oxg_moe_weights *w,
                int eb, int ec) {
  if (!ctx) return fail(nullptr, OXG_ERR_INVALID_ARG, "ctx is NULL");
  if (layer < 0 || layer > 4096) return fail(ctx, OXG_ERR_INVALID_ARG, "layer %d out of range", layer);
  int rc = check_dims(ctx, dims);
  if (rc) return rc;
  if (eb < 0 || ec < 1 || eb + ec > dims->n_experts)
    return fail(ctx, OXG_ERR_INVALID_ARG, "expert range [%d, %d) is not inside [0, %d)", eb, eb + ec,
                dims->n_experts);
  if (!w || !w->router_w || !w->w1_blocks || !w->w1_scales || !w->b1 || !w->w2_blocks ||
      !w->w2_scales || !w->b2)
    return fail(ctx, OXG_ERR_INVALID_ARG, "all weight pointers except router_b must be non-NULL");
  DeviceGuard g(ctx->device);
  const oxg_moe_dims d = *dims;
  // E: resident experts (the router below always has all d.n_experts rows)
  const size_t E = ec, H = d.hidden, I = d.intermediate, ER = d.n_experts;
  const size_t n_rw = ER * H * 2, n_rb = ER * 2;
  const size_t n_w1 = E * 2 * I * (H / 2), n_b1 = E * 2 * I * 2;
  const size_t n_w2 = E * H * (I / 2), n_b2 = E * H * 2;
  const size_t n_t1 = E * (2 * I / 16) * oxg::tile_item_bytes((int)H);  // tile chunks
  const size_t n_t2 = E * (H / 16) * oxg::tile_item_bytes((int)I);
  size_t off = 0;
  auto take = [&](size_t bytes) {
    size_t o = off;
    off = align_up(off + bytes, 256);
    return o;
  };
  const size_t o_rw = take(n_rw), o_rb = take(n_rb), o_w1 = take(n_t1), o_b1 = take(n_b1),
               o_w2 = take(n_t2), o_b2 = take(n_b2), o_mm = take(8);
  const size_t n_a1 = oxg::sf_atoms_bytes((int)E, (int)(2 * I), (int)H, 128);
  const size_t n_a2 = oxg::sf_atoms_bytes((int)E, (int)H, (int)I, 128);
  const size_t n_p1 = oxg::sf_atoms_bytes((int)E, (int)(2 * I), (int)H, oxg::kMxfPrefillTileN);
  const size_t n_p2 = oxg::sf_atoms_bytes((int)E, (int)H, (int)I, oxg::kMxfPrefillTileN);
  const size_t o_q1 = take(n_w1 + 64), o_a1 = take(n_a1), o_q2 = take(n_w2 + 64), o_a2 = take(n_a2);
  const size_t o_p1 = take(n_p1), o_p2 = take(n_p2);
  const size_t stage_bytes = n_w1 > n_w2 ? n_w1 : n_w2;

  if ((size_t)layer >= ctx->layers.size()) ctx->layers.resize(layer + 1);
  free_layer(ctx->layers[layer]);
  ctx->epoch += 1;
  Layer L;
  L.dims = d;
  void *block = nullptr, *stage = nullptr;
  OXG_CUDA(ctx, cudaMalloc(&block, off), "cudaMalloc(layer weights)");
  cudaError_t st = cudaMalloc(&stage, stage_bytes);
  if (st != cudaSuccess) {
    cudaFree(block);
    return cuda_fail(ctx, st, "cudaMalloc(upload staging)");
  }
  char *base = (char *)block;
  L.block = block;
  L.expert_begin = eb;
  L.expert_count = ec;
  L.router_w = (uint16_t *)(base + o_rw);
  L.router_b = w->router_b ? (uint16_t *)(base + o_rb) : nullptr;
  L.w1 = (uint8_t *)(base + o_w1);
  L.b1 = (uint16_t *)(base + o_b1);
  L.w2 = (uint8_t *)(base + o_w2);
  L.b2 = (uint16_t *)(base + o_b2);
  L.q1 = (uint8_t *)(base + o_q1);
  L.a1 = (uint8_t *)(base + o_a1);
  L.q2 = (uint8_t *)(base + o_q2);
  L.a2 = (uint8_t *)(base + o_a2);
  L.p1 = (uint8_t *)(base + o_p1);
  L.p2 = (uint8_t *)(base + o_p2);
  cudaStream_t s = ctx->stream;
  // the shard's slices of the caller's arrays (all experts, expert-major)
  const uint8_t *w1_src = (const uint8_t *)w->w1_blocks + (size_t)eb * 2 * I * (H / 2);
  const uint8_t *s1_src = (const uint8_t *)w->w1_scales + (size_t)eb * 2 * I * (H / 32);
  const uint16_t *b1_src = w->b1 + (size_t)eb * 2 * I;
  const uint8_t *w2_src = (const uint8_t *)w->w2_blocks + (size_t)eb * H * (I / 2);
  const uint8_t *s2_src = (const uint8_t *)w->w2_scales + (size_t)eb * H * (I / 32);
  const uint16_t *b2_src = w->b2 + (size_t)eb * H;
  auto body = [&]() -> cudaError_t {
    cudaError_t e;
    if ((e = cudaMemcpyAsync(L.router_w, w->router_w, n_rw, cudaMemcpyDefault, s))) return e;
    if (w->router_b && (e = cudaMemcpyAsync(L.router_b, w->router_b, n_rb, cudaMemcpyDefault, s)))
      return e;
    if ((e = cudaMemcpyAsync(L.b1, b1_src, n_b1, cudaMemcpyDefault, s))) return e;
    if ((e = cudaMemcpyAsync(L.b2, b2_src, n_b2, cudaMemcpyDefault, s))) return e;
    // scale range over both matrices (zero bytes are ignored)
    unsigned *mm_dev = (unsigned *)(base + o_mm);
    const unsigned init[2] = {255u, 0u};
    if ((e = cudaMemcpyAsync(mm_dev, init, sizeof(init), cudaMemcpyHostToDevice, s))) return e;
    if ((e = cudaMemcpyAsync(stage, w1_src, n_w1, cudaMemcpyDefault, s))) return e;
    if ((e = oxg::launch_tile_weights((const uint8_t *)stage, nullptr, L.w1, E * 2 * I, (int)H, 1, s))) return e;
    if ((e = cudaMemcpyAsync(L.q1, stage, n_w1, cudaMemcpyDeviceToDevice, s))) return e;
    if ((e = cudaMemsetAsync(L.q1 + n_w1, 0, 64, s))) return e;
    if ((e = cudaMemcpyAsync(stage, s1_src, E * 2 * I * (H / 32), cudaMemcpyDefault, s))) return e;
    if ((e = oxg::launch_tile_weights(nullptr, (const uint8_t *)stage, L.w1, E * 2 * I, (int)H, 1, s))) return e;
    if ((e = oxg::launch_scale_range((const uint8_t *)stage, E * 2 * I * (H / 32), mm_dev, s))) return e;
    if ((e = oxg::launch_sf_atoms((const uint8_t *)stage, (int)E, (int)(2 * I), (int)H, 128, L.a1, s))) return e;
    if ((e = oxg::launch_sf_atoms((const uint8_t *)stage, (int)E, (int)(2 * I), (int)H, oxg::kMxfPrefillTileN,
                                  L.p1, s)))
      return e;
    if ((e = cudaMemcpyAsync(stage, w2_src, n_w2, cudaMemcpyDefault, s))) return e;
    if ((e = oxg::launch_tile_weights((const uint8_t *)stage, nullptr, L.w2, E * H, (int)I, 0, s))) return e;
    if ((e = cudaMemcpyAsync(L.q2, stage, n_w2, cudaMemcpyDeviceToDevice, s))) return e;
    if ((e = cudaMemsetAsync(L.q2 + n_w2, 0, 64, s))) return e;
    if ((e = cudaMemcpyAsync(stage, s2_src, E * H * (I / 32), cudaMemcpyDefault, s))) return e;
    if ((e = oxg::launch_tile_weights(nullptr, (const uint8_t *)stage, L.w2, E * H, (int)I, 0, s))) return e;
    if ((e = oxg::launch_scale_range((const uint8_t *)stage, E * H * (I / 32), mm_dev, s))) return e;
    if ((e = oxg::launch_sf_atoms((const uint8_t *)stage, (int)E, (int)H, (int)I, 128, L.a2, s))) return e;
    if ((e = oxg::launch_sf_atoms((const uint8_t *)stage, (int)E, (int)H, (int)I, oxg::kMxfPrefillTileN, L.p2,
                                  s)))
      return e;
    unsigned mm[2] = {0u, 0u};
    if ((e = cudaMemcpyAsync(mm, mm_dev, sizeof(mm), cudaMemcpyDeviceToHost, s))) return e;
    if ((e = cudaStreamSynchronize(s))) return e;
    L.scale_min = mm[0];
    L.scale_max = mm[1];
    L.prefill_ok = H % 64 == 0 && I % 64 == 0 &&
                   (mm[1] == 0u || (mm[0] >= 104u && mm[1] <= 140u));
    L.mxf_ok = H % 64 == 0 && I % 64 == 0 && H >= 128 && I >= 128 && mm[1] <= 254u;
    return cudaSuccess;
  };
  st = body();
  cudaFree(stage);
  if (st != cudaSuccess) {
    cudaFree(block);
    return cuda_fail(ctx, st, "weight upload");
  }
  L.present = true;
  ctx->layers[layer] = L;
  return OXG_OK;
}
}  // namespace

int oxg_moe_upload(oxg_ctx *ctx, int layer, const oxg_moe_dims *dims, const oxg_moe_weights *w) {
  if (!dims) return fail(ctx, OXG_ERR_INVALID_ARG, "dims is NULL");
  return upload_impl(ctx, layer, dims, w, 0, dims->n_experts);
}

int oxg_moe_upload_shard(oxg_ctx *ctx, int layer, const oxg_moe_dims *dims,
                         const oxg_moe_weights *w, int expert_begin, int expert_count) {
  if (!dims) return fail(ctx, OXG_ERR_INVALID_ARG, "dims is NULL");
  return upload_impl(ctx, layer, dims, w, expert_begin, expert_count);
}

int oxg_moe_release(oxg_ctx *ctx, int layer) {
  if (!ctx) return fail(nullptr, OXG_ERR_INVALID_ARG, "ctx is NULL");
  Layer *L = get_layer(ctx, layer);
  if (!L) return fail(ctx, OXG_ERR_STATE, "layer %d has not been uploaded", layer);
  DeviceGuard g(ctx->device);
  OXG_CUDA(ctx, cudaStreamSynchronize(ctx->stream), "cudaStreamSynchronize");
  free_layer(*L);
  ctx->epoch += 1;
  return OXG_OK;
}

int oxg_moe_reserve(oxg_ctx *ctx, int layer, int n_tokens) {
  if (!ctx) return fail(nullptr, OXG_ERR_INVALID_ARG, "ctx is NULL");
  Layer *L = get_layer(ctx, layer);
  if (!L) return fail(ctx, OXG_ERR_STATE, "layer %d has not been uploaded", layer);
  if (n_tokens < 0) return fail(ctx, OXG_ERR_SHAPE, "n_tokens must be >= 0, got %d", n_tokens);
  DeviceGuard g(ctx->device);
  return ensure_scratch(ctx, L->dims, n_tokens);
}

int oxg_moe_forward(oxg_ctx *ctx, int layer, const uint16_t *x, int T, float *y, int mode,
                    int precision) {
  Layer *L = nullptr;
  int rc = check_forward_args(ctx, layer, x, T, y, mode, precision, &L);
  if (rc) return rc;
  if (T == 0) return OXG_OK;
  if (((uintptr_t)x & 15) || ((uintptr_t)y & 15))
    return fail(ctx, OXG_ERR_INVALID_ARG, "x and y must be 16-byte aligned");
  DeviceGuard g(ctx->device);
  rc = ensure_scratch(ctx, L->dims, T);
  if (rc) return rc;
  ctx->last_layer = layer;
  ctx->ep_tokens = -1;
  return forward_device(ctx, *L, x, T, y, mode);
}

namespace {
// Chunked host-buffer forward: chunk c's x copy (stream h2d), compute
// (ctx->stream) and y copy (stream d2h), with two staging buffers per
// direction, so chunk c+1's copy in and chunk c-1's copy out run during chunk
// c's kernels. Every token's result is the same as in one forward: routing,
// expert rows and combine are per token, and chunks stay on the prefill
// kernels (chunk > 64 tokens).
int forward_host_chunked(oxg_ctx *ctx, Layer &L, const uint16_t *x_host, int T, float *y_host, int mode,
                         int chunk) {
  auto &P = ctx->pipe;
  const size_t H = L.dims.hidden;
  // n chunks of floor or ceil(T / n) tokens, every one at least `chunk`
  const int n = T / chunk, Tc = (T + n - 1) / n;
  const size_t xb = align_up((size_t)Tc * H * 2, 256), yb = align_up((size_t)Tc * H * 4, 256);
  const size_t need = 2 * (xb + yb);
  if (!P.h2d) {
    OXG_CUDA(ctx, cudaStreamCreateWithFlags(&P.h2d, cudaStreamNonBlocking), "cudaStreamCreate(h2d)");
    OXG_CUDA(ctx, cudaStreamCreateWithFlags(&P.d2h, cudaStreamNonBlocking), "cudaStreamCreate(d2h)");
    for (int b = 0; b < 2; ++b) {
      OXG_CUDA(ctx, cudaEventCreateWithFlags(&P.x_ready[b], cudaEventDisableTiming), "cudaEventCreate");
      OXG_CUDA(ctx, cudaEventCreateWithFlags(&P.x_free[b], cudaEventDisableTiming), "cudaEventCreate");
      OXG_CUDA(ctx, cudaEventCreateWithFlags(&P.y_ready[b], cudaEventDisableTiming), "cudaEventCreate");
      OXG_CUDA(ctx, cudaEventCreateWithFlags(&P.y_free[b], cudaEventDisableTiming), "cudaEventCreate");
    }
  }
  if (P.bytes < need) {
    if (P.buf) cudaFree(P.buf);
    P.buf = nullptr;
    P.bytes = 0;
    OXG_CUDA(ctx, cudaMalloc(&P.buf, need), "cudaMalloc(host pipeline staging)");
    P.bytes = need;
  }
  char *base = (char *)P.buf;
  uint16_t *xs[2] = {(uint16_t *)base, (uint16_t *)(base + xb)};
  float *ys[2] = {(float *)(base + 2 * xb), (float *)(base + 2 * xb + yb)};
  int rc = ensure_scratch(ctx, L.dims, Tc);
  if (rc) return rc;
  // nothing earlier on the compute stream may still use the staging buffers
  OXG_CUDA(ctx, cudaEventRecord(P.y_ready[0], ctx->stream), "cudaEventRecord");
  OXG_CUDA(ctx, cudaStreamWaitEvent(P.h2d, P.y_ready[0], 0), "cudaStreamWaitEvent");
  for (int c = 0; c < n; ++c) {
    const int b = c & 1;
    const int t0 = (int)((long long)c * T / n), tc = (int)((long long)(c + 1) * T / n) - t0;
    if (c >= 2) OXG_CUDA(ctx, cudaStreamWaitEvent(P.h2d, P.x_free[b], 0), "cudaStreamWaitEvent");
    OXG_CUDA(ctx, cudaMemcpyAsync(xs[b], x_host + (size_t)t0 * H, (size_t)tc * H * 2, cudaMemcpyDefault, P.h2d),
             "copy x to device");
    OXG_CUDA(ctx, cudaEventRecord(P.x_ready[b], P.h2d), "cudaEventRecord");
    OXG_CUDA(ctx, cudaStreamWaitEvent(ctx->stream, P.x_ready[b], 0), "cudaStreamWaitEvent");
    if (c >= 2) OXG_CUDA(ctx, cudaStreamWaitEvent(ctx->stream, P.y_free[b], 0), "cudaStreamWaitEvent");
    rc = forward_device(ctx, L, xs[b], tc, ys[b], mode);
    if (rc) {
      cudaStreamSynchronize(P.h2d);
      cudaStreamSynchronize(P.d2h);
      return rc;
    }
    OXG_CUDA(ctx, cudaEventRecord(P.x_free[b], ctx->stream), "cudaEventRecord");
    OXG_CUDA(ctx, cudaEventRecord(P.y_ready[b], ctx->stream), "cudaEventRecord");
    OXG_CUDA(ctx, cudaStreamWaitEvent(P.d2h, P.y_ready[b], 0), "cudaStreamWaitEvent");
    OXG_CUDA(ctx, cudaMemcpyAsync(y_host + (size_t)t0 * H, ys[b], (size_t)tc * H * 4, cudaMemcpyDefault, P.d2h),
             "copy y to host");
    OXG_CUDA(ctx, cudaEventRecord(P.y_free[b], P.d2h), "cudaEventRecord");
  }
  OXG_CUDA(ctx, cudaStreamSynchronize(P.d2h), "cudaStreamSynchronize");
  OXG_CUDA(ctx, cudaStreamSynchronize(ctx->stream), "cudaStreamSynchronize");
  return read_pipeline_error(ctx);
}
}  // namespace

int oxg_ctx_set_host_chunk(oxg_ctx *ctx, int tokens) {
  if (!ctx) return fail(nullptr, OXG_ERR_INVALID_ARG, "ctx is NULL");
  if (tokens > 0 && tokens <= oxg::kMaxRouteTokens)
    return fail(ctx, OXG_ERR_INVALID_ARG, "host chunks must hold more than %d tokens (or 0: automatic, < 0: off)",
                oxg::kMaxRouteTokens);
  ctx->pipe.chunk = tokens;
  return OXG_OK;
}

int oxg_moe_forward_host(oxg_ctx *ctx, int layer, const uint16_t *x_host, int T, float *y_host,
                         int mode, int precision) {
  Layer *L = nullptr;
  int rc = check_forward_args(ctx, layer, x_host, T, y_host, mode, precision, &L);
  if (rc) return rc;
  if (T == 0) return OXG_OK;
  DeviceGuard g(ctx->device);
  {
    // large batches: chunked, copies overlapped
    const int Tc = ctx->pipe.chunk > 0 ? ctx->pipe.chunk : kHostChunkTokens;
    if (ctx->pipe.chunk >= 0 && T >= 2 * Tc) {
      ctx->last_layer = layer;
      ctx->ep_tokens = -1;
      return forward_host_chunked(ctx, *L, x_host, T, y_host, mode, Tc);
    }
  }
  rc = ensure_scratch(ctx, L->dims, T);
  if (rc) return rc;
  ctx->last_layer = layer;
  ctx->ep_tokens = -1;
  const size_t H = L->dims.hidden;
  OXG_CUDA(ctx, cudaMemcpyAsync(ctx->ws.x_stage, x_host, (size_t)T * H * 2, cudaMemcpyDefault, ctx->stream),
           "copy x to device");
  rc = forward_device(ctx, *L, ctx->ws.x_stage, T, ctx->ws.y_stage, mode);
  if (rc) return rc;
  OXG_CUDA(ctx, cudaMemcpyAsync(y_host, ctx->ws.y_stage, (size_t)T * H * 4, cudaMemcpyDefault, ctx->stream),
           "copy y to host");
  OXG_CUDA(ctx, cudaStreamSynchronize(ctx->stream), "cudaStreamSynchronize");
  return read_pipeline_error(ctx);
}

int oxg_moe_route(oxg_ctx *ctx, int layer, const uint16_t *x, int T, int32_t *idx, float *wts,
                  float *logits) {
  if (!ctx) return fail(nullptr, OXG_ERR_INVALID_ARG, "ctx is NULL");
  Layer *L = get_layer(ctx, layer);
  if (!L) return fail(ctx, OXG_ERR_STATE, "layer %d has not been uploaded", layer);
  if (T < 0) return fail(ctx, OXG_ERR_SHAPE, "n_tokens must be >= 0, got %d", T);
  if (T == 0) return OXG_OK;
  if (!x || !idx || !wts) return fail(ctx, OXG_ERR_INVALID_ARG, "x, idx and w must be non-NULL");
  if ((uintptr_t)x & 15) return fail(ctx, OXG_ERR_INVALID_ARG, "x must be 16-byte aligned");
  DeviceGuard g(ctx->device);
  int rc = ensure_scratch(ctx, L->dims, T);
  if (rc) return rc;
  return route(ctx, *L, x, T, idx, wts, logits);
}

int oxg_moe_last_counts(oxg_ctx *ctx, int32_t *counts_host, int n_experts) {
  if (!ctx) return fail(nullptr, OXG_ERR_INVALID_ARG, "ctx is NULL");
  Layer *L = get_layer(ctx, ctx->last_layer);
  if (!L || !ctx->ws.counts) return fail(ctx, OXG_ERR_STATE, "no forward has run on this context");
  if (!counts_host || n_experts != L->dims.n_experts)
    return fail(ctx, OXG_ERR_INVALID_ARG, "counts_host must hold n_experts = %d ints",
                L->dims.n_experts);
  DeviceGuard g(ctx->device);
  OXG_CUDA(ctx, cudaMemcpyAsync(counts_host, ctx->ws.counts, (size_t)n_experts * 4, cudaMemcpyDefault, ctx->stream),
           "copy counts");
  OXG_CUDA(ctx, cudaStreamSynchronize(ctx->stream), "cudaStreamSynchronize");
  return OXG_OK;
}

// ---- expert parallelism -------------------------------------------------------
namespace {

int check_ep_layer(oxg_ctx *ctx, int layer, Layer **out) {
  if (!ctx) return fail(nullptr, OXG_ERR_INVALID_ARG, "ctx is NULL");
  Layer *L = get_layer(ctx, layer);
  if (!L) return fail(ctx, OXG_ERR_STATE, "layer %d has not been uploaded", layer);
  if (!L->prefill_ok)
    return fail(ctx, OXG_ERR_UNSUPPORTED,
                "expert-parallel rows use the prefill kernels: hidden and intermediate must be "
                "multiples of 64 and E8M0 scales 0 or in [104, 140]; this layer has scales in "
                "[%u, %u]",
                L->scale_min, L->scale_max);
  *out = L;
  return OXG_OK;
}

// Receive-side scratch for R rows: SwiGLU output hi/lo and the segment table.
int ensure_ep_scratch(oxg_ctx *ctx, const oxg_moe_dims &d, size_t R) {
  const size_t hb = align_up(R * (size_t)d.intermediate * 2, 256);
  const size_t need = 2 * hb + align_up((256 + 257) * 4, 256);
  if (need > ctx->ep.bytes) {
    if (ctx->ep.base) {
      OXG_CUDA(ctx, cudaStreamSynchronize(ctx->stream), "cudaStreamSynchronize");
      cudaFree(ctx->ep.base);
      ctx->ep.base = nullptr;
      ctx->ep.bytes = 0;
    }
    void *p = nullptr;
    OXG_CUDA(ctx, cudaMalloc(&p, need), "cudaMalloc(expert-parallel scratch)");
    ctx->ep.base = p;
    ctx->ep.bytes = need;
  }
  char *b = (char *)ctx->ep.base;
  ctx->ep.h_hi = (uint16_t *)b;
  ctx->ep.h_lo = (uint16_t *)(b + hb);
  ctx->ep.seg = (int32_t *)(b + 2 * hb);
  return OXG_OK;
}

}  // namespace

int oxg_moe_dispatch(oxg_ctx *ctx, int layer, const uint16_t *x, int T, uint16_t *rows,
                     float *row_scale, int32_t *expert_counts) {
  Layer *L = nullptr;
  int rc = check_ep_layer(ctx, layer, &L);
  if (rc) return rc;
  if (T < 0) return fail(ctx, OXG_ERR_SHAPE, "n_tokens must be >= 0, got %d", T);
  if (!expert_counts) return fail(ctx, OXG_ERR_INVALID_ARG, "expert_counts must be non-NULL");
  if (T > 0 && (!x || !rows || !row_scale))
    return fail(ctx, OXG_ERR_INVALID_ARG, "x, rows and row_scale must be non-NULL");
  if (((uintptr_t)x & 15) || ((uintptr_t)rows & 15) || ((uintptr_t)row_scale & 3))
    return fail(ctx, OXG_ERR_INVALID_ARG, "x and rows must be 16-byte aligned, row_scale 4-byte");
  DeviceGuard g(ctx->device);
  const oxg_moe_dims &d = L->dims;
  if (T == 0) {
    OXG_CUDA(ctx, cudaMemsetAsync(expert_counts, 0, (size_t)d.n_experts * 4, ctx->stream),
             "cudaMemsetAsync(expert_counts)");
    return OXG_OK;
  }
  if ((rc = ensure_scratch(ctx, d, T))) return rc;
  bool ranked = false;
  if ((rc = route(ctx, *L, x, T, ctx->ws.idx, ctx->ws.wts, ctx->ws.logits, &ranked))) return rc;
  if ((rc = sort_slots(ctx, *L, x, T, ranked, true, rows, row_scale))) return rc;
  OXG_CUDA(ctx, cudaMemcpyAsync(expert_counts, ctx->ws.counts, (size_t)d.n_experts * 4,
                                cudaMemcpyDeviceToDevice, ctx->stream),
           "copy expert counts");
  ctx->last_layer = layer;
  ctx->ep_tokens = T;  // forward calls reset it: they reuse the same scratch
  return OXG_OK;
}

int oxg_moe_experts(oxg_ctx *ctx, int layer, const uint16_t *rows, const float *row_scale,
                    int n_src, const int32_t *seg_counts, float *y_rows) {
  Layer *L = nullptr;
  int rc = check_ep_layer(ctx, layer, &L);
  if (rc) return rc;
  const int ec = L->expert_count;
  if (n_src < 1 || (long long)n_src * ec > 256)
    return fail(ctx, OXG_ERR_INVALID_ARG,
                "n_src * resident experts must be in [1, 256], got %d * %d", n_src, ec);
  if (!seg_counts) return fail(ctx, OXG_ERR_INVALID_ARG, "seg_counts must be non-NULL");
  long long R = 0;
  for (int v = 0; v < n_src * ec; ++v) {
    if (seg_counts[v] < 0)
      return fail(ctx, OXG_ERR_INVALID_ARG, "seg_counts[%d] = %d is negative", v, seg_counts[v]);
    R += seg_counts[v];
  }
  if (R > (1LL << 30)) return fail(ctx, OXG_ERR_SHAPE, "%lld rows is too many", R);
  if (R == 0) return OXG_OK;
  if (!rows || !row_scale || !y_rows)
    return fail(ctx, OXG_ERR_INVALID_ARG, "rows, row_scale and y_rows must be non-NULL");
  if (((uintptr_t)rows & 15) || ((uintptr_t)row_scale & 3) || ((uintptr_t)y_rows & 15))
    return fail(ctx, OXG_ERR_INVALID_ARG,
                "rows and y_rows must be 16-byte aligned, row_scale 4-byte");
  DeviceGuard g(ctx->device);
  const oxg_moe_dims &d = L->dims;
  if (!ctx->ws.base && (rc = ensure_scratch(ctx, d, 1))) return rc;  // error word
  if ((rc = ensure_ep_scratch(ctx, d, (size_t)R))) return rc;
  // segment table: (source rank, resident expert) runs in row order
  const int nv = n_src * ec;
  ctx->seg_host.assign(256 + 257, 0);
  int run = 0;
  for (int v = 0; v < nv; ++v) {
    ctx->seg_host[v] = seg_counts[v];
    ctx->seg_host[256 + v] = run;
    run += seg_counts[v];
  }
  ctx->seg_host[256 + nv] = run;
  // from pageable memory: the call returns once the table is staged, so the
  // host vector may be rewritten by the next call
  OXG_CUDA(ctx, cudaMemcpyAsync(ctx->ep.seg, ctx->seg_host.data(), (256 + 257) * 4,
                                cudaMemcpyHostToDevice, ctx->stream),
           "copy segment table");
  const oxg::MoeDeviceWeights w = device_weights(*L);
  oxg::PrefillIO io{};
  io.S = (int)R;
  io.counts = ctx->ep.seg;
  io.offsets = ctx->ep.seg + 256;
  io.n_segments = nv;
  io.weight_mod = ec;
  io.xp = rows;
  io.pos_scale = row_scale;
  io.h_hi = ctx->ep.h_hi;
  io.h_lo = ctx->ep.h_lo;
  io.y_slot = y_rows;
  io.err = ctx->ws.err;
  OXG_CUDA(ctx, launch(ctx, "moe_mlp1_prefill", [&] {
             return oxg::launch_prefill_mlp1(w, io, ctx->n_sms, ctx->stream);
           }),
           "prefill mlp1 launch");
  OXG_CUDA(ctx, launch(ctx, "moe_mlp2_prefill", [&] {
             return oxg::launch_prefill_mlp2(w, io, ctx->n_sms, ctx->stream);
           }),
           "prefill mlp2 launch");
  ctx->prefill_pending = true;
  return OXG_OK;
}

int oxg_moe_combine(oxg_ctx *ctx, int layer, const float *y_rows, int T, float *y) {
  Layer *L = nullptr;
  int rc = check_ep_layer(ctx, layer, &L);
  if (rc) return rc;
  if (T < 0) return fail(ctx, OXG_ERR_SHAPE, "n_tokens must be >= 0, got %d", T);
  if (T == 0) return OXG_OK;
  if (!y_rows || !y) return fail(ctx, OXG_ERR_INVALID_ARG, "y_rows and y must be non-NULL");
  if (ctx->last_layer != layer || !ctx->ws.base || ctx->ep_tokens != T)
    return fail(ctx, OXG_ERR_STATE,
                "oxg_moe_combine needs the dispatch of the same %d tokens of layer %d first", T,
                layer);
  DeviceGuard g(ctx->device);
  const oxg_moe_dims &d = L->dims;
  OXG_CUDA(ctx, launch(ctx, "combine", [&] {
             return oxg::launch_combine(y_rows, ctx->ws.slot_pos, ctx->ws.wts, T, d.hidden,
                                        d.top_k, y, ctx->stream);
           }),
           "combine launch");
  return OXG_OK;
}

// ---- expert parallelism over peer memory -----------------------------------------
int oxg_ep_init(oxg_ctx *ctx, int layer, int rank, int world, int max_tokens, long long max_recv_rows,
                void *handle_out) {
  Layer *L = nullptr;
  int rc = check_ep_layer(ctx, layer, &L);
  if (rc) return rc;
  const oxg_moe_dims &d = L->dims;
  if (world < 1 || world > oxg::kEpMaxRanks || rank < 0 || rank >= world)
    return fail(ctx, OXG_ERR_INVALID_ARG, "rank %d of world %d: world must be in [1, %d]", rank, world,
                oxg::kEpMaxRanks);
  if (d.n_experts % world || d.n_experts > oxg::kEpMaxExperts ||
      !oxg::router_mma_supported(d.hidden, d.n_experts, d.top_k))
    return fail(ctx, OXG_ERR_UNSUPPORTED,
                "peer-memory expert parallelism needs n_experts (%d) a multiple of the world (%d) "
                "and of 16, at most %d, and hidden a multiple of 16",
                d.n_experts, world, oxg::kEpMaxExperts);
  const int per = d.n_experts / world;
  if (L->expert_begin != rank * per || L->expert_count != per)
    return fail(ctx, OXG_ERR_STATE, "rank %d must hold experts [%d, %d) of layer %d", rank, rank * per,
                rank * per + per, layer);
  if (max_tokens < 1) return fail(ctx, OXG_ERR_INVALID_ARG, "max_tokens must be >= 1");
  const long long worst = (long long)world * max_tokens * d.top_k;
  if (max_recv_rows <= 0) max_recv_rows = worst;
  if (max_recv_rows > worst) max_recv_rows = worst;
  if (!handle_out) return fail(ctx, OXG_ERR_INVALID_ARG, "handle_out must be non-NULL");
  DeviceGuard g(ctx->device);
  OXG_CUDA(ctx, cudaStreamSynchronize(ctx->stream), "cudaStreamSynchronize");
  p2p_release(ctx);
  auto &q = ctx->p2p;
  q.lay = oxg::ep_layout(world, d.n_experts, d.hidden, d.top_k, rank, max_tokens, max_recv_rows);
  OXG_CUDA(ctx, cudaMalloc(&q.sym, q.lay.bytes), "cudaMalloc(expert-parallel symmetric buffer)");
  OXG_CUDA(ctx, cudaMemset(q.sym, 0, q.lay.off_inbox), "zero the flags");
  const size_t hb = align_up((size_t)max_recv_rows * d.intermediate * 2, 256);
  // groups of at most 8 received rows: at most one per segment plus one per 8 rows
  const int vcap = q.lay.W * q.lay.per + (int)(max_recv_rows / oxg::kVirtualTokens) + 1;
  const size_t vb = align_up((size_t)vcap * 4, 256), vpb = align_up((size_t)vcap * sizeof(float *), 256);
  const size_t local_bytes = 2 * hb + align_up((oxg::kEpMaxSegments * 2 + 1) * 4, 256) +
                             align_up(oxg::kEpMaxSegments * sizeof(float *), 256) + 256 + 3 * vb + 256 + vpb;
  OXG_CUDA(ctx, cudaMalloc(&q.local, local_bytes), "cudaMalloc(expert-parallel scratch)");
  OXG_CUDA(ctx, cudaMemset(q.local, 0, local_bytes), "zero the expert-parallel scratch");
  char *b = (char *)q.local;
  q.h_hi = (uint16_t *)b;
  q.h_lo = (uint16_t *)(b + hb);
  q.seg = (int32_t *)(b + 2 * hb);
  q.seg_ptr = (float **)(b + 2 * hb + align_up((oxg::kEpMaxSegments * 2 + 1) * 4, 256));
  q.done_ctr = (uint32_t *)((char *)q.seg_ptr + align_up(oxg::kEpMaxSegments * sizeof(float *), 256));
  q.ok_word = (int *)(q.done_ctr + 1);
  {
    char *vbase = (char *)q.done_ctr + 256;
    q.virt.expert = (int32_t *)vbase;
    q.virt.row0 = (int32_t *)(vbase + vb);
    q.virt.count = (int32_t *)(vbase + 2 * vb);
    q.virt.n = (int32_t *)(vbase + 3 * vb);
    q.virt.out = (float **)(vbase + 3 * vb + 256);
    q.virt.cap = vcap;
  }
  q.decode = oxg::ep_decode_supported(d.hidden, d.intermediate, ctx->n_sms, vcap);
  if (q.decode) {
    // the grouped kernels keep h in f32: it takes the place of the f16 hi / lo pair
    if ((size_t)max_recv_rows * d.intermediate * 4 <= 2 * hb) q.h_f32 = (float *)q.h_hi;
    else q.decode = false;
  }
  cudaIpcMemHandle_t h;
  OXG_CUDA(ctx, cudaIpcGetMemHandle(&h, q.sym), "cudaIpcGetMemHandle");
  std::memcpy(handle_out, &h, sizeof(h));
  q.peers.base[rank] = (char *)q.sym;
  q.layer = layer;
  q.I = d.intermediate;
  q.init = true;
  return OXG_OK;
}

int oxg_ep_connect(oxg_ctx *ctx, const void *handles) {
  if (!ctx) return fail(nullptr, OXG_ERR_INVALID_ARG, "ctx is NULL");
  auto &q = ctx->p2p;
  if (!q.init) return fail(ctx, OXG_ERR_STATE, "oxg_ep_init first");
  if (!handles) return fail(ctx, OXG_ERR_INVALID_ARG, "handles must be non-NULL");
  DeviceGuard g(ctx->device);
  const char *hb = (const char *)handles;
  for (int r = 0; r < q.lay.W; ++r) {
    if (r == q.lay.rank) continue;
    cudaIpcMemHandle_t h;
    std::memcpy(&h, hb + (size_t)r * sizeof(h), sizeof(h));
    void *p = nullptr;
    OXG_CUDA(ctx, cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess),
             "cudaIpcOpenMemHandle (peer buffer)");
    q.peers.base[r] = (char *)p;
  }
  q.connected = true;
  return OXG_OK;
}

int oxg_ep_set_decode_tokens(oxg_ctx *ctx, int tokens) {
  if (!ctx) return fail(nullptr, OXG_ERR_INVALID_ARG, "ctx is NULL");
  auto &q = ctx->p2p;
  if (!q.init) return fail(ctx, OXG_ERR_STATE, "oxg_ep_init first");
  if (tokens < 0 || tokens > oxg::kMaxRouteTokens)
    return fail(ctx, OXG_ERR_INVALID_ARG, "tokens must be in [0, %d], got %d", oxg::kMaxRouteTokens, tokens);
  if (tokens > 0 && !q.decode)
    return fail(ctx, OXG_ERR_UNSUPPORTED, "the grouped decode kernels do not fit hidden %d / intermediate %d",
                q.lay.H, q.I);
  q.decode_tokens = tokens;
  return OXG_OK;
}

int oxg_ep_set_wait_budget(oxg_ctx *ctx, double seconds) {
  if (!ctx) return fail(nullptr, OXG_ERR_INVALID_ARG, "ctx is NULL");
  auto &q = ctx->p2p;
  if (!q.init) return fail(ctx, OXG_ERR_STATE, "oxg_ep_init first");
  if (!(seconds >= 1e-4) || seconds > 60.0)
    return fail(ctx, OXG_ERR_INVALID_ARG, "the wait budget must be in [1e-4, 60] seconds, got %g", seconds);
  int khz = 0;
  OXG_CUDA(ctx, cudaDeviceGetAttribute(&khz, cudaDevAttrClockRate, ctx->device), "cudaDeviceGetAttribute");
  q.lay.wait_cycles = (long long)(seconds * 1e3 * (double)(khz > 0 ? khz : 2000000));
  return OXG_OK;
}

int oxg_ep_close(oxg_ctx *ctx) {
  if (!ctx) return fail(nullptr, OXG_ERR_INVALID_ARG, "ctx is NULL");
  DeviceGuard g(ctx->device);
  OXG_CUDA(ctx, cudaStreamSynchronize(ctx->stream), "cudaStreamSynchronize");
  p2p_release(ctx);
  return OXG_OK;
}

int oxg_ep_last_received(oxg_ctx *ctx, long long *rows) {
  if (!ctx) return fail(nullptr, OXG_ERR_INVALID_ARG, "ctx is NULL");
  if (!rows) return fail(ctx, OXG_ERR_INVALID_ARG, "rows must be non-NULL");
  auto &q = ctx->p2p;
  if (!q.connected) return fail(ctx, OXG_ERR_STATE, "oxg_ep_init and oxg_ep_connect first");
  DeviceGuard g(ctx->device);
  int32_t total = 0;
  OXG_CUDA(ctx, cudaMemcpyAsync(&total, q.seg + oxg::kEpMaxSegments + q.lay.W * q.lay.per, sizeof(total),
                                cudaMemcpyDeviceToHost, ctx->stream),
           "read received rows");
  OXG_CUDA(ctx, cudaStreamSynchronize(ctx->stream), "cudaStreamSynchronize");
  *rows = total;
  return OXG_OK;
}

int oxg_moe_forward_ep(oxg_ctx *ctx, int layer, const uint16_t *x, int T, float *y) {
  Layer *L = nullptr;
  int rc = check_ep_layer(ctx, layer, &L);
  if (rc) return rc;
  auto &q = ctx->p2p;
  if (!q.connected) return fail(ctx, OXG_ERR_STATE, "oxg_ep_init and oxg_ep_connect first");
  if (L->expert_begin != q.lay.rank * q.lay.per || L->expert_count != q.lay.per ||
      L->dims.n_experts != q.lay.E || L->dims.hidden != q.lay.H || L->dims.intermediate != q.I ||
      L->dims.top_k != q.lay.k)
    return fail(ctx, OXG_ERR_STATE, "layer %d does not hold rank %d's experts of the connected layout",
                layer, q.lay.rank);
  if (T < 0 || T > q.lay.max_tokens)
    return fail(ctx, OXG_ERR_SHAPE, "n_tokens must be in [0, %lld], got %d", q.lay.max_tokens, T);
  if (T > 0 && (!x || !y)) return fail(ctx, OXG_ERR_INVALID_ARG, "x and y must be non-NULL");
  if (((uintptr_t)x & 15) || ((uintptr_t)y & 15))
    return fail(ctx, OXG_ERR_INVALID_ARG, "x and y must be 16-byte aligned");
  DeviceGuard g(ctx->device);
  const oxg_moe_dims &d = L->dims;
  if ((rc = ensure_scratch(ctx, d, T < 1 ? 1 : T))) return rc;
  ctx->last_layer = layer;
  ctx->ep_tokens = -1;
  // every rank takes every step, also with no tokens of its own: the others wait for its flags
  const uint32_t epoch = ++q.epoch;
  const oxg::EpLayout lay = q.lay;
  const oxg::EpPeers peers = q.peers;
  const int n_cta = oxg::router_mma_ctas(T);
  if (T > 0 && T <= oxg::kMaxRouteTokens) {
    // a decode-sized batch: the fused per-token router, which also gives the
    // one CTA's histogram and slot ranks the dispatch reads (and routes each
    // token as oxg_moe_forward does on one GPU)
    oxg::RouteSmallArgs ra{};
    ra.x = x;
    ra.router_w = L->router_w;
    ra.router_b = L->router_b;
    ra.T = T;
    ra.H = d.hidden;
    ra.E = d.n_experts;
    ra.k = d.top_k;
    ra.logits = ctx->ws.logits;
    ra.sigma = ctx->ws.sigma;
    ra.idx = ctx->ws.idx;
    ra.wts = ctx->ws.wts;
    ra.counts = ctx->ws.counts;
    ra.offsets = ctx->ws.offsets;
    ra.perm = ctx->ws.perm;
    ra.slot_pos = ctx->ws.slot_pos;
    ra.active = ctx->ws.active;
    ra.n_active = ctx->ws.n_active;
    ra.done = ctx->ws.done;
    ra.cta_hist = ctx->ws.cta_hist;
    ra.local_rank = ctx->ws.local_rank;
    OXG_CUDA(ctx, launch(ctx, "route_small", [&] { return oxg::launch_route_small(ra, ctx->stream, true); }),
             "route_small launch");
  } else if (T > 0) {
    OXG_CUDA(ctx, launch(ctx, "router_mma", [&] {
               return oxg::launch_router_mma(x, L->router_w, L->router_b, T, d.hidden, d.n_experts,
                                             d.top_k, ctx->ws.idx, ctx->ws.wts, ctx->ws.logits,
                                             ctx->ws.sigma, ctx->ws.cta_hist, ctx->ws.local_rank,
                                             ctx->stream, ctx->ws.err);
             }),
             "router_mma launch");
  }
  OXG_CUDA(ctx, launch(ctx, "ep_counts", [&] {
             return oxg::launch_ep_counts(lay, peers, ctx->ws.cta_hist, n_cta, ctx->ws.counts,
                                          ctx->ws.offsets, q.ok_word, epoch, ctx->ws.err, 11, ctx->stream);
           }),
           "ep_counts launch");
  if (T > 0) {
    OXG_CUDA(ctx, launch(ctx, "ep_scatter", [&] {
               return oxg::launch_ep_scatter(lay, peers, ctx->ws.cta_hist, n_cta, ctx->ws.idx,
                                             ctx->ws.local_rank, T, x, ctx->ws.sigma, ctx->ws.slot_pos,
                                             q.done_ctr, q.ok_word, ctx->ws.err, epoch, ctx->stream);
             }),
             "ep_scatter launch");
  } else {  // nothing to send: raise the rows flags at once
    OXG_CUDA(ctx, launch(ctx, "ep_signal", [&] {
               return oxg::launch_ep_signal(lay, peers, 1, epoch, q.ok_word, nullptr, 0, ctx->stream);
             }),
             "ep_signal launch");
  }
  // a decode-sized batch on this rank (the path is each receiver's own
  // choice: both handle whatever rows the others sent); off while the
  // decode size is 0, whatever this rank's batch
  const bool grouped = q.decode && q.decode_tokens > 0 && T <= q.decode_tokens;
  OXG_CUDA(ctx, launch(ctx, "ep_segments", [&] {
             return oxg::launch_ep_segments(lay, peers, epoch, ctx->ws.err, q.ok_word, q.seg,
                                            q.seg_ptr, grouped ? q.virt : oxg::EpVirtual{}, ctx->stream);
           }),
           "ep_segments launch");
  const oxg::MoeDeviceWeights w = device_weights(*L);
  if (grouped) {
    // the grouped decode kernels over the received rows, each group's output
    // rows stored straight into its source's return rows
    oxg::DecodeSched sched{};
    sched.n_sms = ctx->n_sms;
    sched.err = ctx->ws.err;
    sched.parts = ctx->ws.parts;
    sched.flat_cnt = ctx->ws.flat_cnt;
    OXG_CUDA(ctx, launch(ctx, "moe_ep_decode", [&] {
               return oxg::launch_ep_decode(w, (const uint16_t *)((char *)q.sym + lay.off_recv_rows),
                                            (const float *)((char *)q.sym + lay.off_recv_scale), q.h_f32, q.virt,
                                            sched, ctx->stream);
             }),
             "ep decode launch");
    ctx->launches += 1;  // two kernels
  } else {
  oxg::PrefillIO io{};
  io.S = (int)lay.max_recv;
  io.counts = q.seg;
  io.offsets = q.seg + oxg::kEpMaxSegments;
  io.n_segments = lay.W * lay.per;
  io.weight_mod = lay.per;
  io.xp = (const uint16_t *)((char *)q.sym + lay.off_recv_rows);
  io.pos_scale = (const float *)((char *)q.sym + lay.off_recv_scale);
  io.h_hi = q.h_hi;
  io.h_lo = q.h_lo;
  io.y_slot = nullptr;
  io.y_seg = q.seg_ptr;
  io.err = ctx->ws.err;
  OXG_CUDA(ctx, launch(ctx, "moe_mlp1_prefill", [&] {
             return oxg::launch_prefill_mlp1(w, io, ctx->n_sms, ctx->stream);
           }),
           "prefill mlp1 launch");
  OXG_CUDA(ctx, launch(ctx, "moe_mlp2_prefill", [&] {
             return oxg::launch_prefill_mlp2(w, io, ctx->n_sms, ctx->stream);
           }),
           "prefill mlp2 launch");
  }
  OXG_CUDA(ctx, launch(ctx, "ep_signal", [&] {
             return oxg::launch_ep_signal(lay, peers, 2, epoch, q.ok_word, ctx->ws.err, 13, ctx->stream);
           }),
           "ep_signal launch");
  ctx->prefill_pending = true;
  if (T == 0) return OXG_OK;
  OXG_CUDA(ctx, launch(ctx, "combine", [&] {
             return oxg::launch_combine((const float *)((char *)q.sym + lay.off_ret_rows),
                                        ctx->ws.slot_pos, ctx->ws.wts, T, d.hidden, d.top_k, y,
                                        ctx->stream);
           }),
           "combine launch");
  return OXG_OK;
}

int oxg_profile_enable(oxg_ctx *ctx, int on) {
  if (!ctx) return fail(nullptr, OXG_ERR_INVALID_ARG, "ctx is NULL");
  ctx->prof.on = on != 0;
  return OXG_OK;
}

int oxg_profile_read(oxg_ctx *ctx, const char *name, double *total_ms, int *launches) {
  if (!ctx) return fail(nullptr, OXG_ERR_INVALID_ARG, "ctx is NULL");
  if (!name || !total_ms || !launches)
    return fail(ctx, OXG_ERR_INVALID_ARG, "name, total_ms and launches must be non-NULL");
  DeviceGuard g(ctx->device);
  OXG_CUDA(ctx, cudaStreamSynchronize(ctx->stream), "cudaStreamSynchronize");
  ctx->prof.drain();
  *total_ms = 0.0;
  *launches = 0;
  for (const Profiler::Sum &s : ctx->prof.sums)
    if (s.name == name) {
      *total_ms = s.ms;
      *launches = s.launches;
    }
  return OXG_OK;
}

int oxg_profile_reset(oxg_ctx *ctx) {
  if (!ctx) return fail(nullptr, OXG_ERR_INVALID_ARG, "ctx is NULL");
  DeviceGuard g(ctx->device);
  OXG_CUDA(ctx, cudaStreamSynchronize(ctx->stream), "cudaStreamSynchronize");
  ctx->prof.drain();
  ctx->prof.sums.clear();
  return OXG_OK;
}

int oxg_kernel_launches(const oxg_ctx *ctx, long long *count) {
  if (!ctx || !count) return fail(nullptr, OXG_ERR_INVALID_ARG, "ctx and count must be non-NULL");
  *count = ctx->launches;
  return OXG_OK;
}

int oxg_measure_mma_rate(oxg_ctx *ctx, int kind, int iters, double *tflops) {
  if (!ctx || !tflops) return fail(ctx, OXG_ERR_INVALID_ARG, "ctx and tflops must be non-NULL");
  if (kind < 0 || kind > 2) return fail(ctx, OXG_ERR_INVALID_ARG, "kind must be 0, 1 or 2, got %d", kind);
  if (iters < 1 || iters > (1 << 22)) return fail(ctx, OXG_ERR_INVALID_ARG, "iters must be in [1, 2^22]");
  DeviceGuard g(ctx->device);
  int *err = nullptr;
  OXG_CUDA(ctx, cudaMalloc(&err, sizeof(int)), "cudaMalloc(error word)");
  cudaEvent_t a = nullptr, b = nullptr;
  int rc = OXG_OK, h = 0;
  float ms = 0.f;
  do {
    cudaError_t st;
    if ((st = cudaMemsetAsync(err, 0, sizeof(int), ctx->stream)) != cudaSuccess ||
        (st = cudaEventCreate(&a)) != cudaSuccess || (st = cudaEventCreate(&b)) != cudaSuccess ||
        (st = cudaEventRecord(a, ctx->stream)) != cudaSuccess ||
        (st = oxg::launch_mma_rate(kind, iters, ctx->n_sms, err, ctx->stream)) != cudaSuccess ||
        (st = cudaEventRecord(b, ctx->stream)) != cudaSuccess ||
        (st = cudaMemcpyAsync(&h, err, sizeof(int), cudaMemcpyDeviceToHost, ctx->stream)) != cudaSuccess ||
        (st = cudaStreamSynchronize(ctx->stream)) != cudaSuccess ||
        (st = cudaEventElapsedTime(&ms, a, b)) != cudaSuccess) {
      rc = fail(ctx, OXG_ERR_CUDA, "mma rate measurement: %s", cudaGetErrorString(st));
      break;
    }
    ctx->launches += 1;
    if (h) {
      rc = fail(ctx, OXG_ERR_TIMEOUT, "mma rate measurement: the final wait ran out");
      break;
    }
    *tflops = oxg::mma_flops_per_instr(kind) * iters * ctx->n_sms / (ms * 1e-3) / 1e12;
  } while (0);
  if (a) cudaEventDestroy(a);
  if (b) cudaEventDestroy(b);
  cudaFree(err);
  return rc;
}

}  // extern "C"
