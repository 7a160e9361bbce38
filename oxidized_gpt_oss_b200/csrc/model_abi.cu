// model_abi.cu — the full-decoder entry points (oxg_model_*): weights, KV
// cache and activations of a gpt-oss-20b-architecture decoder on one
// context, the launch sequence of one forward, and greedy generation.
//
// Layout in HBM (one allocation per part):
//   * per layer: attention norm [H], fused q/k/v rows [(nh + 2 nkv) 64, H]
//     (q rows, then k, then v, so one linear launch covers all three), their
//     bias, o projection [H, nh 64] + bias, sinks [nh], MoE norm [H];
//   * embeddings [V, H], LM head [V, H], final norm [H];
//   * KV cache [layer][K|V][nkv][pool rows][64] bf16, paged: the pool of a
//     kv head holds kv_pages pages of 64 rows; the page table [B][max_pages]
//     (device, with a host mirror) maps page p of sequence s (positions
//     64p .. 64p + 63) to a pool page, taken from a free list as the sequence
//     grows and returned by a reset. Every attention kernel reads and writes
//     rows through the table (a 64-key tile or split is one page). RoPE
//     cos/sin tables [max_seq][32] f32 (built on the host in double precision);
//   * activations for max_tokens tokens: residual f32, normed bf16, linear
//     partials f32, q and attention output bf16, MoE output f32, logits.
// Reference interfaces replaced: GPTModel::forward (src/model.rs:713-741),
// TransformerLayer::forward (src/model.rs:848-887), Attention::forward
// (src/model.rs:899-1084), reset_kv_cache (src/model.rs:743-747),
// InferenceEngine::generate_chat's greedy loop (src/inference.rs:62-97).
#include <cuda_runtime.h>

#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <vector>

#include "../../include/oxg_b200.h"
#include "ctx_internal.h"
#include "model.h"

namespace oxg {

struct ModelState {
  oxg_model_dims d{};
  int Nq = 0, Nkv = 0, Nqkv = 0, G = 0;
  void *emb_block = nullptr;
  uint16_t *embed = nullptr, *unembed = nullptr, *final_norm = nullptr;
  struct Attn {
    void *block = nullptr;
    uint16_t *norm1 = nullptr, *wqkv = nullptr, *bqkv = nullptr, *wo = nullptr, *bo = nullptr;
    uint16_t *sinks = nullptr, *norm2 = nullptr;
  };
  std::vector<Attn> layers;
  void *state = nullptr;
  uint16_t *kv = nullptr;
  // a tensor map (CUtensorMap) over the whole KV cache for the batched decode
  // attention's TMA loads; kv_map_ok false: the cache is too large for one
  alignas(64) unsigned char kv_map[128] = {};
  bool kv_map_ok = false;
  float *rope_cos = nullptr, *rope_sin = nullptr;
  float *res = nullptr, *part = nullptr, *y = nullptr, *apart = nullptr, *logits = nullptr;
  uint16_t *xn = nullptr, *qb = nullptr, *cb = nullptr;
  int32_t *tok = nullptr, *gen = nullptr;
  int32_t *dstate = nullptr;  // decode state {position, step, token} read by the captured step
  int32_t *first = nullptr;   // generate: the prompt's greedy token
  unsigned long long *am_keys = nullptr;  // fused LM-head argmax keys [8] (zero between uses)
  unsigned int *am_count = nullptr;       // its finished-CTA counter
  int *err = nullptr;
  int part_rows = 0, max_logits = 0, gen_cap = 0;
  int pos = 0;                 // sequence 0's position (the single-sequence API's)
  int B = 1;                   // sequences with a KV cache of their own
  size_t kv_stride = 0;        // cache rows per kv head: the page pool, n_pool * 64
  std::vector<int> seq_pos;    // positions of sequences 1 .. B-1 (index 0 unused)
  unsigned *merge_cnt = nullptr;  // tensor-core decode attention: per (sequence, kv head) arrivals
  int32_t *tok_pos = nullptr, *tok_seq = nullptr;  // batched step: [B] position; [B] sequence ids 0 .. B-1
  // paged KV cache: page table [B][max_pages] on the device and its host
  // mirror (-1: no page), the free pool pages, and each sequence's page count
  int32_t *pages = nullptr;
  int max_pages = 0, n_pool = 0;
  std::vector<int32_t> page_host;
  std::vector<int32_t> free_pages;
  std::vector<int> seq_npages;
  bool moe_reserved = false;
  bool state_ok = false;  // the device state holds the last forward's greedy token
  int32_t *route_tap = nullptr;  // oxg_model_route_tap: [n_layers][tap_tokens][k] expert ids
  int tap_tokens = 0;
  // One captured one-token decode step (oxg_model_decode): replayed per token.
  cudaGraphExec_t gexec = nullptr;
  cudaStream_t cap_stream = nullptr;
  unsigned long long g_epoch = 0;
  long long g_launches = 0;
};

namespace {

constexpr int kMaxLogits = 128;

int mfail(oxg_ctx *ctx, int status, const char *fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  return ctx_error(ctx, status, buf);
}

int mcuda(oxg_ctx *ctx, cudaError_t st, const char *what) {
  return mfail(ctx, st == cudaErrorMemoryAllocation ? OXG_ERR_OOM : OXG_ERR_CUDA, "%s: %s (%s)", what,
               cudaGetErrorName(st), cudaGetErrorString(st));
}

#define MCUDA(ctx, call, what)                             \
  do {                                                     \
    cudaError_t st_ = (call);                              \
    if (st_ != cudaSuccess) return ::oxg::mcuda(ctx, st_, what);  \
  } while (0)

struct DevGuard {
  int prev = -1;
  explicit DevGuard(int dev) {
    if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
    if (prev != dev) cudaSetDevice(dev);
  }
  ~DevGuard() {
    if (prev >= 0) cudaSetDevice(prev);
  }
};

size_t al(size_t v) { return (v + 255) / 256 * 256; }

void free_attn(ModelState::Attn &a) {
  if (a.block) cudaFree(a.block);
  a = ModelState::Attn{};
}

void free_model(ModelState *M) {
  if (!M) return;
  if (M->gexec) cudaGraphExecDestroy(M->gexec);
  if (M->cap_stream) cudaStreamDestroy(M->cap_stream);
  for (auto &a : M->layers) free_attn(a);
  if (M->emb_block) cudaFree(M->emb_block);
  if (M->state) cudaFree(M->state);
  delete M;
}

ModelState *get_model(oxg_ctx *ctx) { return ctx ? ctx_model(ctx) : nullptr; }

int check_model_dims(oxg_ctx *ctx, const oxg_model_dims *d) {
  if (!d) return mfail(ctx, OXG_ERR_INVALID_ARG, "dims is NULL");
  if (d->n_layers <= 0 || d->n_layers > 4096)
    return mfail(ctx, OXG_ERR_SHAPE, "n_layers must be in [1, 4096], got %d", d->n_layers);
  if (d->hidden <= 0 || d->hidden % 64)
    return mfail(ctx, OXG_ERR_SHAPE, "hidden must be a positive multiple of 64, got %d", d->hidden);
  if (d->head_dim != 64) return mfail(ctx, OXG_ERR_UNSUPPORTED, "head_dim must be 64, got %d", d->head_dim);
  if (d->n_heads <= 0 || d->n_kv_heads <= 0 || d->n_heads % d->n_kv_heads ||
      d->n_heads / d->n_kv_heads > attn_max_group())
    return mfail(ctx, OXG_ERR_SHAPE,
                 "n_heads (%d) must be a positive multiple of n_kv_heads (%d), at most %d times it",
                 d->n_heads, d->n_kv_heads, attn_max_group());
  if (d->vocab <= 0) return mfail(ctx, OXG_ERR_SHAPE, "vocab must be positive, got %d", d->vocab);
  if (d->sliding_window < 0)
    return mfail(ctx, OXG_ERR_SHAPE, "sliding_window must be >= 0, got %d", d->sliding_window);
  if (d->max_seq <= 0 || d->max_seq > (1 << 22))
    return mfail(ctx, OXG_ERR_SHAPE, "max_seq must be in [1, 2^22], got %d", d->max_seq);
  if (d->max_tokens <= 0 || d->max_tokens > d->max_seq)
    return mfail(ctx, OXG_ERR_SHAPE, "max_tokens must be in [1, max_seq], got %d", d->max_tokens);
  if (d->max_batch < 0 || d->max_batch > kMaxLogits || d->max_batch > d->max_tokens)
    return mfail(ctx, OXG_ERR_SHAPE, "max_batch must be in [0, min(%d, max_tokens)], got %d", kMaxLogits,
                 d->max_batch);
  if (d->kv_pages < 0 || d->kv_pages > (1 << 24))
    return mfail(ctx, OXG_ERR_SHAPE, "kv_pages must be in [0, 2^24], got %d", d->kv_pages);
  if (!(d->rope_theta > 0.f)) return mfail(ctx, OXG_ERR_INVALID_ARG, "rope_theta must be positive");
  if (!(d->rms_eps >= 0.f)) return mfail(ctx, OXG_ERR_INVALID_ARG, "rms_eps must be >= 0");
  return OXG_OK;
}

// The q/k/v weights of one layer as the fused [Nqkv, H] operand.
int upload_attn(oxg_ctx *ctx, ModelState &M, int layer, const oxg_attn_weights *w) {
  const oxg_model_dims &d = M.d;
  const size_t H = d.hidden, Nq = M.Nq, Nkv = M.Nkv, Nqkv = M.Nqkv;
  if (!w || !w->attn_norm || !w->wq || !w->wk || !w->wv || !w->wo || !w->mlp_norm)
    return mfail(ctx, OXG_ERR_INVALID_ARG,
                 "attention weights need attn_norm, wq, wk, wv, wo and mlp_norm (biases and sinks may be NULL)");
  ModelState::Attn a;
  size_t off = 0;
  auto take = [&](size_t bytes) {
    size_t o = off;
    off = al(off + bytes);
    return o;
  };
  const size_t o_n1 = take(H * 2), o_qkv = take(Nqkv * H * 2), o_bqkv = take(Nqkv * 2);
  const size_t o_wo = take(H * Nq * 2), o_bo = take(H * 2), o_sk = take((size_t)d.n_heads * 2);
  const size_t o_n2 = take(H * 2);
  MCUDA(ctx, cudaMalloc(&a.block, off), "cudaMalloc(attention weights)");
  char *b = (char *)a.block;
  a.norm1 = (uint16_t *)(b + o_n1);
  a.wqkv = (uint16_t *)(b + o_qkv);
  a.bqkv = (uint16_t *)(b + o_bqkv);
  a.wo = (uint16_t *)(b + o_wo);
  a.bo = (uint16_t *)(b + o_bo);
  a.sinks = (uint16_t *)(b + o_sk);
  a.norm2 = (uint16_t *)(b + o_n2);
  cudaStream_t s = ctx_stream(ctx);
  auto cp = [&](void *dst, const void *src, size_t bytes) -> cudaError_t {
    return cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDefault, s);
  };
  cudaError_t e = cudaSuccess;
  if (!e) e = cp(a.norm1, w->attn_norm, H * 2);
  if (!e) e = cp(a.wqkv, w->wq, Nq * H * 2);
  if (!e) e = cp(a.wqkv + Nq * H, w->wk, Nkv * H * 2);
  if (!e) e = cp(a.wqkv + (Nq + Nkv) * H, w->wv, Nkv * H * 2);
  if (!e) e = cudaMemsetAsync(a.bqkv, 0, Nqkv * 2, s);
  if (!e && w->bq) e = cp(a.bqkv, w->bq, Nq * 2);
  if (!e && w->bk) e = cp(a.bqkv + Nq, w->bk, Nkv * 2);
  if (!e && w->bv) e = cp(a.bqkv + Nq + Nkv, w->bv, Nkv * 2);
  if (!e) e = cp(a.wo, w->wo, H * Nq * 2);
  if (!e) e = cudaMemsetAsync(a.bo, 0, H * 2, s);
  if (!e && w->bo) e = cp(a.bo, w->bo, H * 2);
  if (!e && w->sinks) e = cp(a.sinks, w->sinks, (size_t)d.n_heads * 2);
  if (!e) e = cp(a.norm2, w->mlp_norm, H * 2);
  if (!e) e = cudaStreamSynchronize(s);
  if (e) {
    free_attn(a);
    return mcuda(ctx, e, "attention weight upload");
  }
  if (!w->sinks) a.sinks = nullptr;
  free_attn(M.layers[layer]);
  M.layers[layer] = a;
  return OXG_OK;
}

int &seq_pos_ref(ModelState &M, int seq) { return seq == 0 ? M.pos : M.seq_pos[seq]; }

// Gives sequence seq pool pages for every position up to last_pos and copies
// the new table entries to the device (stream order). Fails with OXG_ERR_OOM,
// changing nothing, when the pool has too few free pages.
int ensure_pages(oxg_ctx *ctx, ModelState &M, int seq, int last_pos) {
  if (last_pos < 0) return OXG_OK;
  const int need = (last_pos >> 6) + 1, have = M.seq_npages[seq];
  if (need <= have) return OXG_OK;
  if (need > M.max_pages)
    return mfail(ctx, OXG_ERR_SHAPE, "position %d of sequence %d exceeds max_seq %d", last_pos, seq, M.d.max_seq);
  if ((int)M.free_pages.size() < need - have)
    return mfail(ctx, OXG_ERR_OOM,
                 "KV-cache pool exhausted: sequence %d needs %d more pages of 64 positions, %d of %d are free",
                 seq, need - have, (int)M.free_pages.size(), M.n_pool);
  int32_t *row = M.page_host.data() + (size_t)seq * M.max_pages;
  for (int p = have; p < need; ++p) {
    row[p] = M.free_pages.back();
    M.free_pages.pop_back();
  }
  M.seq_npages[seq] = need;
  MCUDA(ctx, cudaMemcpyAsync(M.pages + (size_t)seq * M.max_pages + have, row + have, (size_t)(need - have) * 4,
                             cudaMemcpyHostToDevice, ctx_stream(ctx)),
        "page table update");
  return OXG_OK;
}

// Returns sequence seq's pages to the pool.
void release_pages(ModelState &M, int seq) {
  int32_t *row = M.page_host.data() + (size_t)seq * M.max_pages;
  for (int p = M.seq_npages[seq] - 1; p >= 0; --p) {
    M.free_pages.push_back(row[p]);
    row[p] = -1;
  }
  M.seq_npages[seq] = 0;
}

// One forward of T tokens of sequence seq at positions pos .. pos + T - 1.
// With dstate (the decode step a graph captures: sequence 0, T = 1,
// n_logits = 1) the token, position and output slot come from the device
// state instead, and the argmax advances it; otherwise a forward of sequence
// 0 that computes logits leaves the state at its end position and greedy
// token, ready for one-token steps. With batch, token t is the next token of
// sequence t (positions and sequences in M.tok_pos / M.tok_seq, max_splits
// the longest one's attention splits) and the caller advances the positions.
int forward(oxg_ctx *ctx, ModelState &M, const int32_t *tok, int T, int n_logits, float *logits_out,
            int32_t *next_out, int32_t *dstate = nullptr, int seq = 0, bool batch = false, int max_splits = 0) {
  const oxg_model_dims &d = M.d;
  const int H = d.hidden, L = d.n_layers;
  cudaStream_t s = ctx_stream(ctx);
  const int n_sms = ctx_n_sms(ctx);
  if (!M.embed) return mfail(ctx, OXG_ERR_STATE, "embeddings have not been uploaded");
  bool ep = false;  // the MoE blocks are expert-parallel shards (every process runs the same steps)
  for (int l = 0; l < L; ++l) {
    if (!M.layers[l].block) return mfail(ctx, OXG_ERR_STATE, "attention of layer %d has not been uploaded", l);
    int mh = ctx_moe_hidden(ctx, l);
    if (!mh && (mh = ctx_moe_ep_hidden(ctx, l)) != 0) ep = true;
    if (!mh)
      return mfail(ctx, OXG_ERR_STATE,
                   "MoE layer %d has not been uploaded (whole, or as this process's shard of a connected "
                   "expert-parallel exchange)", l);
    if (mh != H) return mfail(ctx, OXG_ERR_STATE, "MoE layer %d has hidden %d, the model %d", l, mh, H);
  }
  if (ep && dstate)
    return mfail(ctx, OXG_ERR_UNSUPPORTED,
                 "expert-parallel MoE blocks run eagerly (their exchange counts steps on the host): use "
                 "oxg_model_forward / oxg_model_step_batch");
  if (!M.moe_reserved) {
    for (int l = 0; l < L; ++l) {
      const int rc = ctx_moe_reserve(ctx, l, d.max_tokens);
      if (rc) return rc;
    }
    M.moe_reserved = true;
  }
  const bool own_state = !batch && seq == 0;  // the decode state follows sequence 0
  const int pos0 = batch ? 0 : seq_pos_ref(M, seq);
  if (!batch && !dstate) {  // pages for the positions this call writes (steps and batches: their callers)
    const int rcp = ensure_pages(ctx, M, seq, pos0 + T - 1);
    if (rcp) return rcp;
  }
  // embedding + layer 0's attention norm
  {
    NormArgs a;
    a.res = M.res;
    a.rows = T;
    a.H = H;
    a.tokens = dstate ? dstate + 2 : tok;
    a.embed = M.embed;
    a.V = d.vocab;
    a.gamma = M.layers[0].norm1;
    a.eps = d.rms_eps;
    a.out = M.xn;
    a.err = M.err;
    MCUDA(ctx, ctx_launch(ctx, "embed_norm", [&] { return launch_residual_norm(a, s); }), "embed launch");
  }
  const float scale = 1.0f / std::sqrt((float)d.head_dim);
  // A single query of one sequence runs the tensor-core decode attention of
  // the batched step, with its position read from the device (the decode
  // state, or M.tok_pos written here), so eager one-token forwards and graph
  // replays compute the same bits.
  const bool one_query = !batch && T == 1 && M.kv_map_ok && M.G == 8;
  if (one_query && !dstate)
    MCUDA(ctx, cudaMemcpyAsync(M.tok_pos, &pos0, 4, cudaMemcpyHostToDevice, s), "position copy");
  const size_t kv_layer = (size_t)2 * d.n_kv_heads * M.kv_stride * 64;
  const int32_t *tpos = batch ? M.tok_pos : nullptr, *tseq = batch ? M.tok_seq : nullptr;
  for (int l = 0; l < L; ++l) {
    const ModelState::Attn &A = M.layers[l];
    uint16_t *kc = M.kv + (size_t)l * kv_layer;
    uint16_t *vc = kc + kv_layer / 2;
    const int s_qkv = linear_splits(M.Nqkv, H, T, n_sms, M.part_rows);
    MCUDA(ctx, ctx_launch(ctx, "linear_qkv", [&] {
            return launch_linear(M.xn, T, H, A.wqkv, M.Nqkv, H, s_qkv, M.part, s);
          }),
          "qkv launch");
    MCUDA(ctx, ctx_launch(ctx, "qkv_rope", [&] {
            return launch_qkv_post(M.part, s_qkv, T, d.n_heads, d.n_kv_heads, A.bqkv, M.rope_cos, M.rope_sin,
                                   pos0, dstate, (int)M.kv_stride, M.pages, M.max_pages, seq, M.qb, kc, vc, s,
                                   tpos, tseq);
          }),
          "qkv epilogue launch");
    AttnArgs at;
    at.q = M.qb;
    at.kc = kc;
    at.vc = vc;
    at.T = T;
    at.nh = d.n_heads;
    at.nkv = d.n_kv_heads;
    at.max_seq = (int)M.kv_stride;
    at.split_rows = d.max_seq;
    at.tok_pos = tpos;
    at.tok_seq = tseq;
    at.pages = M.pages;
    at.max_pages = M.max_pages;
    at.seq = seq;
    at.max_splits = max_splits;
    at.pos0 = pos0;
    at.window = (l % 2 == 0) ? d.sliding_window : 0;
    at.scale = scale;
    at.sinks = A.sinks;
    at.part = M.apart;
    at.pos_dev = dstate;
    if (one_query) {  // one query of one sequence: the batched kernel, its position on the device
      at.tok_pos = dstate ? dstate : M.tok_pos;
      at.tok_seq = M.tok_seq + seq;
      at.max_splits = (d.max_seq + kKvPageRows - 1) / kKvPageRows;
    }
    if ((batch || one_query) && M.kv_map_ok) {
      at.kv_map = M.kv_map;
      at.k_row = (long long)l * 2 * d.n_kv_heads * (long long)M.kv_stride;
      at.v_row = at.k_row + (long long)d.n_kv_heads * (long long)M.kv_stride;
      at.n_sms = n_sms;
      at.err = M.err;
      if (one_query) at.merge_cnt = M.merge_cnt;
    }
    at.out = M.cb;
    MCUDA(ctx, ctx_launch(ctx, "attention", [&] { return launch_attention(at, s); }), "attention launch");
    const int s_o = linear_splits(H, M.Nq, T, n_sms, M.part_rows);
    MCUDA(ctx, ctx_launch(ctx, "linear_o", [&] { return launch_linear(M.cb, T, M.Nq, A.wo, H, M.Nq, s_o, M.part, s); }),
          "o projection launch");
    {
      NormArgs a;
      a.res = M.res;
      a.rows = T;
      a.H = H;
      a.add = M.part;
      a.S = s_o;
      a.add_stride = (size_t)T * H;
      a.add_bias = A.bo;
      a.gamma = A.norm2;
      a.eps = d.rms_eps;
      a.out = M.xn;
      a.err = M.err;
      MCUDA(ctx, ctx_launch(ctx, "residual_norm", [&] { return launch_residual_norm(a, s); }),
            "residual norm launch");
    }
    int rc = ctx_moe_hidden(ctx, l) ? ctx_moe_forward(ctx, l, M.xn, T, M.y) : ctx_moe_forward_ep(ctx, l, M.xn, T, M.y);
    if (rc) return rc;
    if (M.route_tap && !dstate && T <= M.tap_tokens) {
      const int k = ctx_moe_topk(ctx, l);
      MCUDA(ctx, cudaMemcpyAsync(M.route_tap + (size_t)l * M.tap_tokens * k, ctx_moe_last_idx(ctx),
                                 (size_t)T * k * sizeof(int32_t), cudaMemcpyDeviceToDevice, s),
            "route tap copy");
    }
    const bool last = l + 1 == L;
    const int rows = last ? n_logits : T;
    const int r0 = T - rows;
    if (rows > 0) {
      NormArgs a;
      a.res = M.res + (size_t)r0 * H;
      a.rows = rows;
      a.H = H;
      a.add = M.y + (size_t)r0 * H;
      a.S = 1;
      a.add_stride = 0;
      a.gamma = last ? M.final_norm : M.layers[l + 1].norm1;
      a.eps = d.rms_eps;
      a.out = M.xn;
      a.err = M.err;
      MCUDA(ctx, ctx_launch(ctx, "residual_norm", [&] { return launch_residual_norm(a, s); }),
            "residual norm launch");
    }
  }
  if (n_logits > 0 && n_logits <= 8) {
    // LM head with the greedy choice and the decode-state update in its epilogue
    float *lg = logits_out ? logits_out : M.logits;
    ArgmaxEpilogue am;
    am.keys = M.am_keys;
    am.count = M.am_count;
    am.next = dstate ? nullptr : (next_out ? next_out : M.tok);
    am.state = dstate ? dstate : M.dstate;
    am.out_seq = M.gen;
    am.state_mode = dstate ? 1 : (own_state ? 2 : 0);
    am.set_pos = pos0 + T;
    MCUDA(ctx, ctx_launch(ctx, "lm_head", [&] {
            return launch_linear(M.xn, n_logits, H, M.unembed, d.vocab, H, 1, lg, s, &am);
          }),
          "lm head launch");
    if (dstate) return OXG_OK;  // the caller advances the host position
  } else if (n_logits > 0) {
    float *lg = logits_out ? logits_out : M.logits;
    MCUDA(ctx, ctx_launch(ctx, "lm_head", [&] {
            return launch_linear(M.xn, n_logits, H, M.unembed, d.vocab, H, 1, lg, s);
          }),
          "lm head launch");
    if (dstate) {
      MCUDA(ctx, ctx_launch(ctx, "argmax", [&] {
              return launch_argmax(lg, 1, d.vocab, nullptr, dstate, M.gen, s);
            }),
            "argmax launch");
      return OXG_OK;  // the caller advances the host position
    }
    int32_t *nx = next_out ? next_out : M.tok;
    MCUDA(ctx, ctx_launch(ctx, "argmax", [&] {
            return launch_argmax(lg, n_logits, d.vocab, nx, nullptr, nullptr, s);
          }),
          "argmax launch");
    if (own_state) MCUDA(ctx, ctx_launch(ctx, "decode_state", [&] {
            return launch_set_state(M.dstate, pos0 + T, nx + n_logits - 1, s);
          }),
          "state launch");
  }
  if (batch) return OXG_OK;  // the caller advances every sequence's position
  if (own_state) M.state_ok = n_logits > 0;
  seq_pos_ref(M, seq) = pos0 + T;
  return OXG_OK;
}

// Captures one device-state decode step into M.gexec (on a private stream,
// so that a context bound to the legacy default stream can capture too).
int capture_step(oxg_ctx *ctx, ModelState &M) {
  if (M.gexec) {
    cudaGraphExecDestroy(M.gexec);
    M.gexec = nullptr;
  }
  if (!M.cap_stream)
    MCUDA(ctx, cudaStreamCreateWithFlags(&M.cap_stream, cudaStreamNonBlocking), "cudaStreamCreate(capture)");
  cudaStream_t orig = ctx_stream(ctx);
  const bool prof = ctx_profile_flag(ctx);
  ctx_profile_flag(ctx) = false;
  const long long l0 = ctx_launch_count(ctx);
  oxg_ctx_set_stream(ctx, M.cap_stream);
  cudaError_t st = cudaStreamBeginCapture(M.cap_stream, cudaStreamCaptureModeRelaxed);
  int rc = OXG_OK;
  cudaGraph_t graph = nullptr;
  if (st == cudaSuccess) {
    rc = forward(ctx, M, nullptr, 1, 1, nullptr, nullptr, M.dstate);
    st = cudaStreamEndCapture(M.cap_stream, &graph);
  }
  oxg_ctx_set_stream(ctx, orig);
  ctx_profile_flag(ctx) = prof;
  M.g_launches = ctx_launch_count(ctx) - l0;
  ctx_add_launches(ctx, -M.g_launches);  // captured, not launched
  if (rc) {
    if (graph) cudaGraphDestroy(graph);
    return rc;
  }
  if (st == cudaSuccess) st = cudaGraphInstantiate(&M.gexec, graph, 0);
  if (graph) cudaGraphDestroy(graph);
  if (st != cudaSuccess) {
    M.gexec = nullptr;
    return mcuda(ctx, st, "decode-step graph capture");
  }
  M.g_epoch = ctx_epoch(ctx);
  return OXG_OK;
}

// n greedy one-token steps from the state the last forward (or step) left:
// the first eagerly (it also settles the MoE scratch layout for one token),
// the rest as replays of the captured step. Tokens land in M.gen[0 .. n).
int decode_steps(oxg_ctx *ctx, ModelState &M, int n) {
  if (n <= 0) return OXG_OK;
  if (M.pos <= 0 || !M.state_ok)
    return mfail(ctx, OXG_ERR_STATE, "decoding continues from the greedy token of a forward with n_logits >= 1");
  if (M.pos + n > M.d.max_seq)
    return mfail(ctx, OXG_ERR_SHAPE, "KV cache full: position %d + %d steps exceeds max_seq %d", M.pos, n,
                 M.d.max_seq);
  // pages for every position the steps write (replays read the table on the device)
  int rcp = ensure_pages(ctx, M, 0, M.pos + n - 1);
  if (rcp) return rcp;
  // step counter back to 0 (tokens land in M.gen[0 ..)), position from the host
  MCUDA(ctx, ctx_launch(ctx, "decode_state", [&] {
          return launch_set_state(M.dstate, M.pos, M.dstate + 2, ctx_stream(ctx));
        }),
        "state launch");
  int rc = forward(ctx, M, nullptr, 1, 1, nullptr, nullptr, M.dstate);
  if (rc) return rc;
  if (n > 1 && (!M.gexec || M.g_epoch != ctx_epoch(ctx))) {
    rc = capture_step(ctx, M);
    if (rc) return rc;
  }
  cudaStream_t s = ctx_stream(ctx);
  for (int i = 1; i < n; ++i) {
    MCUDA(ctx, cudaGraphLaunch(M.gexec, s), "cudaGraphLaunch(decode step)");
    ctx_add_launches(ctx, M.g_launches);
  }
  M.pos += n;
  return OXG_OK;
}

int check_forward(oxg_ctx *ctx, ModelState *M, int T, int n_logits) {
  if (!M) return mfail(ctx, OXG_ERR_STATE, "oxg_model_init has not been called");
  if (T <= 0 || T > M->d.max_tokens)
    return mfail(ctx, OXG_ERR_SHAPE, "n_tokens must be in [1, max_tokens = %d], got %d", M->d.max_tokens, T);
  if (n_logits < 0 || n_logits > T || n_logits > M->max_logits)
    return mfail(ctx, OXG_ERR_SHAPE, "n_logits must be in [0, min(n_tokens, %d)], got %d", M->max_logits,
                 n_logits);
  if (M->pos + T > M->d.max_seq)
    return mfail(ctx, OXG_ERR_SHAPE, "KV cache full: position %d + %d tokens exceeds max_seq %d", M->pos, T,
                 M->d.max_seq);
  return OXG_OK;
}

}  // namespace

void model_free(oxg_ctx *ctx) {
  free_model(ctx_model(ctx));
  ctx_model(ctx) = nullptr;
}

int model_check_error(oxg_ctx *ctx) {
  ModelState *M = ctx_model(ctx);
  if (!M || !M->err) return OXG_OK;
  int h = 0;
  MCUDA(ctx, cudaMemcpy(&h, M->err, sizeof(int), cudaMemcpyDeviceToHost), "read model status");
  if (h) {
    MCUDA(ctx, cudaMemset(M->err, 0, sizeof(int)), "clear model status");
    // a split that stopped early never arrived: its counters start again at zero
    MCUDA(ctx, cudaMemset(M->merge_cnt, 0, (size_t)M->B * M->d.n_kv_heads * 4), "clear attention counters");
    if (h == 61)
      return mfail(ctx, OXG_ERR_TIMEOUT, "a KV tile load of the decode attention did not complete (code 61)");
    return mfail(ctx, OXG_ERR_INVALID_ARG, "a token id outside [0, vocab = %d) was given (code %d)", M->d.vocab, h);
  }
  return OXG_OK;
}

}  // namespace oxg

using oxg::ModelState;

extern "C" {

int oxg_model_init(oxg_ctx *ctx, const oxg_model_dims *dims) {
  if (!ctx) return oxg::ctx_error(nullptr, OXG_ERR_INVALID_ARG, "ctx is NULL");
  int rc = oxg::check_model_dims(ctx, dims);
  if (rc) return rc;
  oxg::DevGuard g(oxg::ctx_device(ctx));
  cudaStreamSynchronize(oxg::ctx_stream(ctx));
  oxg::model_free(ctx);
  ModelState *M = new (std::nothrow) ModelState();
  if (!M) return oxg::mfail(ctx, OXG_ERR_OOM, "host allocation failed");
  const oxg_model_dims &d = *dims;
  M->d = d;
  M->Nq = d.n_heads * 64;
  M->Nkv = d.n_kv_heads * 64;
  M->Nqkv = M->Nq + 2 * M->Nkv;
  M->G = d.n_heads / d.n_kv_heads;
  M->layers.resize(d.n_layers);
  M->max_logits = d.max_tokens < oxg::kMaxLogits ? d.max_tokens : oxg::kMaxLogits;
  M->part_rows = d.max_tokens > 1024 ? d.max_tokens : 1024;
  M->gen_cap = d.max_seq;
  M->B = d.max_batch > 1 ? d.max_batch : 1;
  M->max_pages = (d.max_seq + oxg::kKvPageRows - 1) / oxg::kKvPageRows;
  M->n_pool = d.kv_pages > 0 ? d.kv_pages : M->B * M->max_pages;
  M->kv_stride = (size_t)M->n_pool * oxg::kKvPageRows;
  M->seq_pos.assign(M->B, 0);
  M->page_host.assign((size_t)M->B * M->max_pages, -1);
  M->seq_npages.assign(M->B, 0);
  M->free_pages.resize(M->n_pool);
  for (int i = 0; i < M->n_pool; ++i) M->free_pages[i] = M->n_pool - 1 - i;  // page 0 is taken first
  const size_t H = d.hidden, Tm = d.max_tokens;
  const size_t nmax = (size_t)(M->Nqkv > d.hidden ? M->Nqkv : d.hidden);
  size_t off = 0;
  auto take = [&](size_t bytes) {
    size_t o = off;
    off = oxg::al(off + bytes);
    return o;
  };
  const size_t o_kv = take((size_t)d.n_layers * 2 * d.n_kv_heads * M->kv_stride * 64 * 2);
  const size_t o_cos = take((size_t)d.max_seq * 32 * 4), o_sin = take((size_t)d.max_seq * 32 * 4);
  const size_t o_res = take(Tm * H * 4), o_xn = take(Tm * H * 2), o_y = take(Tm * H * 4);
  const size_t o_part = take((size_t)M->part_rows * nmax * 4);
  const size_t o_qb = take(Tm * M->Nq * 2), o_cb = take(Tm * M->Nq * 2);
  const size_t o_ap = take(oxg::attn_part_floats(d.n_kv_heads, M->G, d.max_seq) * M->B * 4);
  const size_t o_lg = take((size_t)M->max_logits * d.vocab * 4);
  const size_t o_tok = take(Tm * 4), o_gen = take((size_t)M->gen_cap * 4), o_err = take(4);
  const size_t o_ds = take(4 * 4), o_first = take(4);
  const size_t o_amk = take(8 * 8), o_amc = take(4);
  const size_t o_tp = take((size_t)M->B * 4), o_tr = take((size_t)M->B * 4);
  const size_t o_pg = take((size_t)M->B * M->max_pages * 4);
  const size_t o_mc = take((size_t)M->B * d.n_kv_heads * 4);
  cudaError_t e = cudaMalloc(&M->state, off);
  if (e) {
    delete M;
    return oxg::mcuda(ctx, e, "cudaMalloc(model state)");
  }
  char *b = (char *)M->state;
  M->kv = (uint16_t *)(b + o_kv);
  M->rope_cos = (float *)(b + o_cos);
  M->rope_sin = (float *)(b + o_sin);
  M->res = (float *)(b + o_res);
  M->xn = (uint16_t *)(b + o_xn);
  M->y = (float *)(b + o_y);
  M->part = (float *)(b + o_part);
  M->qb = (uint16_t *)(b + o_qb);
  M->cb = (uint16_t *)(b + o_cb);
  M->apart = (float *)(b + o_ap);
  M->logits = (float *)(b + o_lg);
  M->tok = (int32_t *)(b + o_tok);
  M->gen = (int32_t *)(b + o_gen);
  M->err = (int *)(b + o_err);
  M->dstate = (int32_t *)(b + o_ds);
  M->first = (int32_t *)(b + o_first);
  M->am_keys = (unsigned long long *)(b + o_amk);
  M->am_count = (unsigned int *)(b + o_amc);
  M->tok_pos = (int32_t *)(b + o_tp);
  M->tok_seq = (int32_t *)(b + o_tr);
  M->pages = (int32_t *)(b + o_pg);
  M->merge_cnt = (unsigned *)(b + o_mc);
  // RoPE tables: angle(pos, i) = pos * theta^(-2i / head_dim), i < head_dim / 2,
  // evaluated in double and rounded once to f32.
  std::vector<float> cs((size_t)d.max_seq * 32), sn((size_t)d.max_seq * 32);
  for (int p = 0; p < d.max_seq; ++p)
    for (int i = 0; i < 32; ++i) {
      const double inv = std::pow((double)d.rope_theta, -2.0 * i / (double)d.head_dim);
      const double ang = (double)p * inv;
      cs[(size_t)p * 32 + i] = (float)std::cos(ang);
      sn[(size_t)p * 32 + i] = (float)std::sin(ang);
    }
  e = cudaMemcpy(M->rope_cos, cs.data(), cs.size() * 4, cudaMemcpyHostToDevice);
  if (!e) e = cudaMemcpy(M->rope_sin, sn.data(), sn.size() * 4, cudaMemcpyHostToDevice);
  if (!e) e = cudaMemset(M->err, 0, 4);
  if (!e) e = cudaMemset(M->dstate, 0, 16);
  if (!e) e = cudaMemset(M->am_keys, 0, 8 * 8);
  if (!e) e = cudaMemset(M->am_count, 0, 4);
  if (!e) e = cudaMemset(M->pages, 0, (size_t)M->B * M->max_pages * 4);
  if (!e) e = cudaMemset(M->merge_cnt, 0, (size_t)M->B * d.n_kv_heads * 4);
  if (!e) {  // sequence ids: entry i is i (a one-sequence call reads entry seq)
    std::vector<int32_t> ids((size_t)M->B);
    for (int i = 0; i < M->B; ++i) ids[(size_t)i] = i;
    e = cudaMemcpy(M->tok_seq, ids.data(), ids.size() * 4, cudaMemcpyHostToDevice);
  }
  if (e) {
    oxg::free_model(M);
    return oxg::mcuda(ctx, e, "model state initialisation");
  }
  M->kv_map_ok = oxg::make_kv_map(M->kv_map, M->kv,
                                  (long long)d.n_layers * 2 * d.n_kv_heads * (long long)M->kv_stride) == cudaSuccess;
  oxg::ctx_model(ctx) = M;
  return OXG_OK;
}

int oxg_model_upload_embeddings(oxg_ctx *ctx, const uint16_t *embed, const uint16_t *unembed,
                                const uint16_t *final_norm) {
  if (!ctx) return oxg::ctx_error(nullptr, OXG_ERR_INVALID_ARG, "ctx is NULL");
  ModelState *M = oxg::get_model(ctx);
  if (!M) return oxg::mfail(ctx, OXG_ERR_STATE, "oxg_model_init has not been called");
  if (!embed || !unembed || !final_norm)
    return oxg::mfail(ctx, OXG_ERR_INVALID_ARG, "embed, unembed and final_norm must be non-NULL");
  oxg::DevGuard g(oxg::ctx_device(ctx));
  const size_t VH = (size_t)M->d.vocab * M->d.hidden;
  void *blk = nullptr;
  const size_t o_u = oxg::al(VH * 2), o_n = o_u + oxg::al(VH * 2);
  MCUDA(ctx, cudaMalloc(&blk, o_n + oxg::al((size_t)M->d.hidden * 2)), "cudaMalloc(embeddings)");
  cudaStream_t s = oxg::ctx_stream(ctx);
  cudaError_t e = cudaMemcpyAsync(blk, embed, VH * 2, cudaMemcpyDefault, s);
  if (!e) e = cudaMemcpyAsync((char *)blk + o_u, unembed, VH * 2, cudaMemcpyDefault, s);
  if (!e) e = cudaMemcpyAsync((char *)blk + o_n, final_norm, (size_t)M->d.hidden * 2, cudaMemcpyDefault, s);
  if (!e) e = cudaStreamSynchronize(s);
  if (e) {
    cudaFree(blk);
    return oxg::mcuda(ctx, e, "embedding upload");
  }
  if (M->emb_block) cudaFree(M->emb_block);
  M->emb_block = blk;
  M->embed = (uint16_t *)blk;
  M->unembed = (uint16_t *)((char *)blk + o_u);
  M->final_norm = (uint16_t *)((char *)blk + o_n);
  return OXG_OK;
}

int oxg_model_upload_attention(oxg_ctx *ctx, int layer, const oxg_attn_weights *w) {
  if (!ctx) return oxg::ctx_error(nullptr, OXG_ERR_INVALID_ARG, "ctx is NULL");
  ModelState *M = oxg::get_model(ctx);
  if (!M) return oxg::mfail(ctx, OXG_ERR_STATE, "oxg_model_init has not been called");
  if (layer < 0 || layer >= M->d.n_layers)
    return oxg::mfail(ctx, OXG_ERR_INVALID_ARG, "layer %d out of range [0, %d)", layer, M->d.n_layers);
  oxg::DevGuard g(oxg::ctx_device(ctx));
  return oxg::upload_attn(ctx, *M, layer, w);
}

int oxg_model_reset(oxg_ctx *ctx) {
  if (!ctx) return oxg::ctx_error(nullptr, OXG_ERR_INVALID_ARG, "ctx is NULL");
  ModelState *M = oxg::get_model(ctx);
  if (!M) return oxg::mfail(ctx, OXG_ERR_STATE, "oxg_model_init has not been called");
  M->pos = 0;  // positions at or beyond pos are never read before they are written again
  for (int &p : M->seq_pos) p = 0;
  for (int q = 0; q < M->B; ++q) oxg::release_pages(*M, q);
  M->state_ok = false;
  return OXG_OK;
}

int oxg_model_reset_seq(oxg_ctx *ctx, int seq) {
  if (!ctx) return oxg::ctx_error(nullptr, OXG_ERR_INVALID_ARG, "ctx is NULL");
  ModelState *M = oxg::get_model(ctx);
  if (!M) return oxg::mfail(ctx, OXG_ERR_STATE, "oxg_model_init has not been called");
  if (seq < 0 || seq >= M->B)
    return oxg::mfail(ctx, OXG_ERR_INVALID_ARG, "seq %d out of range [0, max_batch = %d)", seq, M->B);
  oxg::seq_pos_ref(*M, seq) = 0;
  oxg::release_pages(*M, seq);
  if (seq == 0) M->state_ok = false;
  return OXG_OK;
}

int oxg_model_kv_pages(oxg_ctx *ctx, int *used, int *total) {
  if (!ctx) return oxg::ctx_error(nullptr, OXG_ERR_INVALID_ARG, "ctx is NULL");
  ModelState *M = oxg::get_model(ctx);
  if (!M) return oxg::mfail(ctx, OXG_ERR_STATE, "oxg_model_init has not been called");
  if (!used || !total) return oxg::mfail(ctx, OXG_ERR_INVALID_ARG, "used and total must be non-NULL");
  *total = M->n_pool;
  *used = M->n_pool - (int)M->free_pages.size();
  return OXG_OK;
}

int oxg_model_position(oxg_ctx *ctx, int *pos) {
  if (!ctx) return oxg::ctx_error(nullptr, OXG_ERR_INVALID_ARG, "ctx is NULL");
  if (!pos) return oxg::mfail(ctx, OXG_ERR_INVALID_ARG, "pos is NULL");
  ModelState *M = oxg::get_model(ctx);
  if (!M) return oxg::mfail(ctx, OXG_ERR_STATE, "oxg_model_init has not been called");
  *pos = M->pos;
  return OXG_OK;
}

int oxg_model_forward(oxg_ctx *ctx, const int32_t *tokens, int n_tokens, int n_logits, float *logits,
                      int32_t *next) {
  if (!ctx) return oxg::ctx_error(nullptr, OXG_ERR_INVALID_ARG, "ctx is NULL");
  ModelState *M = oxg::get_model(ctx);
  int rc = oxg::check_forward(ctx, M, n_tokens, n_logits);
  if (rc) return rc;
  if (!tokens) return oxg::mfail(ctx, OXG_ERR_INVALID_ARG, "tokens_dev is NULL");
  oxg::DevGuard g(oxg::ctx_device(ctx));
  return oxg::forward(ctx, *M, tokens, n_tokens, n_logits, logits, next);
}

int oxg_model_generate(oxg_ctx *ctx, const int32_t *prompt, int n_prompt, int n_new, int32_t *out) {
  if (!ctx) return oxg::ctx_error(nullptr, OXG_ERR_INVALID_ARG, "ctx is NULL");
  ModelState *M = oxg::get_model(ctx);
  if (!M) return oxg::mfail(ctx, OXG_ERR_STATE, "oxg_model_init has not been called");
  if (!prompt || !out) return oxg::mfail(ctx, OXG_ERR_INVALID_ARG, "prompt and tokens must be non-NULL");
  if (n_prompt <= 0 || n_new <= 0)
    return oxg::mfail(ctx, OXG_ERR_SHAPE, "n_prompt and n_new must be positive, got %d and %d", n_prompt, n_new);
  if ((long)n_prompt + n_new - 1 > M->d.max_seq)
    return oxg::mfail(ctx, OXG_ERR_SHAPE, "prompt %d + %d new tokens exceed max_seq %d", n_prompt, n_new,
                      M->d.max_seq);
  for (int i = 0; i < n_prompt; ++i)
    if (prompt[i] < 0 || prompt[i] >= M->d.vocab)
      return oxg::mfail(ctx, OXG_ERR_INVALID_ARG, "Token id %d out of bounds", prompt[i]);
  oxg::DevGuard g(oxg::ctx_device(ctx));
  cudaStream_t s = oxg::ctx_stream(ctx);
  M->pos = 0;
  const int chunk = M->d.max_tokens;
  for (int c0 = 0; c0 < n_prompt; c0 += chunk) {
    const int n = n_prompt - c0 < chunk ? n_prompt - c0 : chunk;
    MCUDA(ctx, cudaMemcpyAsync(M->tok, prompt + c0, (size_t)n * 4, cudaMemcpyHostToDevice, s), "prompt copy");
    const bool lastc = c0 + n == n_prompt;
    int rc = oxg::forward(ctx, *M, M->tok, n, lastc ? 1 : 0, nullptr, M->first);
    if (rc) return rc;
  }
  int rc = oxg::decode_steps(ctx, *M, n_new - 1);
  if (rc) return rc;
  MCUDA(ctx, cudaMemcpyAsync(out, M->first, 4, cudaMemcpyDeviceToHost, s), "token copy");
  if (n_new > 1)
    MCUDA(ctx, cudaMemcpyAsync(out + 1, M->gen, (size_t)(n_new - 1) * 4, cudaMemcpyDeviceToHost, s),
          "token copy");
  MCUDA(ctx, cudaStreamSynchronize(s), "cudaStreamSynchronize");
  return oxg_sync(ctx);
}

int oxg_model_decode(oxg_ctx *ctx, int n_steps, int32_t *tokens) {
  if (!ctx) return oxg::ctx_error(nullptr, OXG_ERR_INVALID_ARG, "ctx is NULL");
  ModelState *M = oxg::get_model(ctx);
  if (!M) return oxg::mfail(ctx, OXG_ERR_STATE, "oxg_model_init has not been called");
  if (n_steps < 0) return oxg::mfail(ctx, OXG_ERR_SHAPE, "n_steps must be >= 0, got %d", n_steps);
  if (n_steps > 0 && !tokens) return oxg::mfail(ctx, OXG_ERR_INVALID_ARG, "tokens_dev is NULL");
  oxg::DevGuard g(oxg::ctx_device(ctx));
  int rc = oxg::decode_steps(ctx, *M, n_steps);
  if (rc) return rc;
  if (n_steps > 0 && tokens != M->gen)
    MCUDA(ctx, cudaMemcpyAsync(tokens, M->gen, (size_t)n_steps * 4, cudaMemcpyDeviceToDevice, oxg::ctx_stream(ctx)),
          "token copy");
  return OXG_OK;
}

int oxg_model_route_tap(oxg_ctx *ctx, int32_t *idx_dev, int max_tokens) {
  if (!ctx) return oxg::ctx_error(nullptr, OXG_ERR_INVALID_ARG, "ctx is NULL");
  ModelState *M = oxg::get_model(ctx);
  if (!M) return oxg::mfail(ctx, OXG_ERR_STATE, "oxg_model_init has not been called");
  if (idx_dev && max_tokens <= 0)
    return oxg::mfail(ctx, OXG_ERR_SHAPE, "max_tokens must be positive, got %d", max_tokens);
  M->route_tap = idx_dev;
  M->tap_tokens = idx_dev ? max_tokens : 0;
  return OXG_OK;
}

int oxg_model_prefill_seq(oxg_ctx *ctx, int seq, const int32_t *tokens, int n_tokens, int32_t *next) {
  if (!ctx) return oxg::ctx_error(nullptr, OXG_ERR_INVALID_ARG, "ctx is NULL");
  ModelState *M = oxg::get_model(ctx);
  if (!M) return oxg::mfail(ctx, OXG_ERR_STATE, "oxg_model_init has not been called");
  if (seq < 0 || seq >= M->B)
    return oxg::mfail(ctx, OXG_ERR_INVALID_ARG, "seq %d out of range [0, max_batch = %d)", seq, M->B);
  if (n_tokens <= 0 || n_tokens > M->d.max_tokens)
    return oxg::mfail(ctx, OXG_ERR_SHAPE, "n_tokens must be in [1, max_tokens = %d], got %d", M->d.max_tokens,
                      n_tokens);
  if (!tokens) return oxg::mfail(ctx, OXG_ERR_INVALID_ARG, "tokens_dev is NULL");
  const int p = oxg::seq_pos_ref(*M, seq);
  if (p + n_tokens > M->d.max_seq)
    return oxg::mfail(ctx, OXG_ERR_SHAPE, "KV cache of sequence %d full: position %d + %d tokens exceeds max_seq %d",
                      seq, p, n_tokens, M->d.max_seq);
  oxg::DevGuard g(oxg::ctx_device(ctx));
  return oxg::forward(ctx, *M, tokens, n_tokens, 1, nullptr, next, nullptr, seq);
}

int oxg_model_step_batch(oxg_ctx *ctx, int n_seqs, const int32_t *tokens, int32_t *next, float *logits) {
  if (!ctx) return oxg::ctx_error(nullptr, OXG_ERR_INVALID_ARG, "ctx is NULL");
  ModelState *M = oxg::get_model(ctx);
  if (!M) return oxg::mfail(ctx, OXG_ERR_STATE, "oxg_model_init has not been called");
  if (n_seqs <= 0 || n_seqs > M->B)
    return oxg::mfail(ctx, OXG_ERR_SHAPE, "n_seqs must be in [1, max_batch = %d], got %d", M->B, n_seqs);
  if (!tokens || !next) return oxg::mfail(ctx, OXG_ERR_INVALID_ARG, "tokens_dev and next_dev must be non-NULL");
  std::vector<int32_t> hp(n_seqs);
  int max_splits = 1;
  for (int i = 0; i < n_seqs; ++i) {
    const int p = oxg::seq_pos_ref(*M, i);
    if (p + 1 > M->d.max_seq)
      return oxg::mfail(ctx, OXG_ERR_SHAPE, "KV cache of sequence %d full: position %d + 1 exceeds max_seq %d", i, p,
                        M->d.max_seq);
    hp[i] = p;
    const int sp = oxg::attn_page_splits(0, p);  // 64-key pages over positions 0 .. p
    if (sp > max_splits) max_splits = sp;
  }
  oxg::DevGuard g(oxg::ctx_device(ctx));
  for (int i = 0; i < n_seqs; ++i) {
    const int rc = oxg::ensure_pages(ctx, *M, i, hp[i]);
    if (rc) return rc;
  }
  cudaStream_t s = oxg::ctx_stream(ctx);
  // pageable sources: each copy is staged before the call returns
  MCUDA(ctx, cudaMemcpyAsync(M->tok_pos, hp.data(), (size_t)n_seqs * 4, cudaMemcpyHostToDevice, s), "position copy");
  int rc = oxg::forward(ctx, *M, tokens, n_seqs, n_seqs, logits, next, nullptr, 0, true, max_splits);
  if (rc) return rc;
  for (int i = 0; i < n_seqs; ++i) oxg::seq_pos_ref(*M, i) += 1;
  M->state_ok = false;  // sequence 0 moved without the one-token decode state
  return OXG_OK;
}

int oxg_model_release(oxg_ctx *ctx) {
  if (!ctx) return oxg::ctx_error(nullptr, OXG_ERR_INVALID_ARG, "ctx is NULL");
  oxg::DevGuard g(oxg::ctx_device(ctx));
  cudaStreamSynchronize(oxg::ctx_stream(ctx));
  oxg::model_free(ctx);
  return OXG_OK;
}

}  // extern "C"
