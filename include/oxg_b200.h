/*
 * oxg_b200.h — C ABI of liboxg_b200.so, the B200 (sm_100a) MXFP4
 * mixture-of-experts hot path of the gpt-oss runner cipher-rc5/oxidized_gpt_oss.
 *
 * The reference has no FFI: its "backend" is a compile-time module swap
 * (src/backend/mod.rs:5-10) between a Metal implementation and a host-memory
 * stub, and its hot path is host Rust (src/moe.rs, src/mxfp4.rs, src/ffn.rs,
 * src/model.rs:1088-1184). Each entry point below names the reference
 * interface it replaces. Conventions:
 *
 *  - Every function returns an int status: 0 (OXG_OK) or a negative
 *    oxg_status. Nothing aborts the process where the reference panics on a
 *    shape assert: the same condition returns OXG_ERR_SHAPE and
 *    oxg_last_error() holds the reference's message text.
 *  - Pointers named *_dev are device pointers (any CUDA allocation visible to
 *    the context's device); *_host are host pointers; upload accepts either.
 *  - Work is enqueued on the context's stream and is asynchronous unless the
 *    function says otherwise; oxg_sync() waits for it.
 *  - A context is used by one host thread at a time.
 *  - bf16 values travel as uint16_t bit patterns.
 */
#ifndef OXG_B200_H
#define OXG_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define OXG_ABI_VERSION 1

#if defined(__GNUC__)
#define OXG_API __attribute__((visibility("default")))
#else
#define OXG_API
#endif

typedef enum {
  OXG_OK = 0,
  OXG_ERR_INVALID_ARG = -1,
  OXG_ERR_SHAPE = -2,
  OXG_ERR_CUDA = -3,
  OXG_ERR_NCCL = -4,
  OXG_ERR_TIMEOUT = -5,
  OXG_ERR_STATE = -6,
  OXG_ERR_UNSUPPORTED = -7,
  OXG_ERR_OOM = -8
} oxg_status;

enum { OXG_SCALE_E8M0 = 0, OXG_SCALE_BF16 = 1 };
/* OXG_MODE_DECODE: the in-register-dequant mma.sync expert kernels;
 * OXG_MODE_MXF4: the block-scaled tcgen05 expert kernels (E2M1 weights and
 * E8M0 scales straight from HBM into the tensor cores: decode kernels for
 * T <= 8 tokens, CTA-pair GEMMs above; hidden and intermediate multiples of
 * 64, no scale byte 255). OXG_MODE_AUTO: DECODE for T <= 64; above, PREFILL
 * when every scale is 0 or in [104, 140], else MXF4. */
enum { OXG_MODE_AUTO = 0, OXG_MODE_DECODE = 1, OXG_MODE_PREFILL = 2, OXG_MODE_MXF4 = 3 };
enum { OXG_PRECISION_PARITY = 0 };

typedef struct oxg_ctx oxg_ctx;

/* ---- library / context --------------------------------------------------- */

OXG_API int oxg_abi_version(void);
OXG_API const char *oxg_status_string(int status);

/* Replaces MetalDevice::new + MetalCompute::new (src/backend/metal_stub.rs:31-34,
 * :92-95): binds a CUDA device and creates the context's stream. */
OXG_API int oxg_ctx_create(int device, oxg_ctx **out);
OXG_API int oxg_ctx_destroy(oxg_ctx *ctx);
/* Message of the last failing call on ctx (or of the last failing
 * context-less call on this thread when ctx is NULL). Never NULL. */
OXG_API const char *oxg_last_error(const oxg_ctx *ctx);
/* Runs the context's work on `stream` (a cudaStream_t) from now on, instead
 * of the stream the context created; NULL is CUDA's legacy default stream. */
OXG_API int oxg_ctx_set_stream(oxg_ctx *ctx, void *stream);
OXG_API void *oxg_ctx_get_stream(const oxg_ctx *ctx);
/* Replaces MetalDevice::synchronize (src/backend/metal_stub.rs:46-48). */
OXG_API int oxg_sync(oxg_ctx *ctx);

/* ---- MXFP4 dequantisation ------------------------------------------------ */

/* Replaces dequantize_mxfp4(blocks: &[u8], scales: &[u16], rows, cols) -> Vec<u16>
 * (src/mxfp4.rs:15-54, called from src/loader.rs:66). Device pointers;
 * n_block_bytes / n_scales are the slice lengths the reference asserts
 * (rows*cols/2 and rows*cols/32). scale_fmt OXG_SCALE_BF16 takes bf16 bit
 * patterns as the reference does; OXG_SCALE_E8M0 takes the checkpoint's
 * uint8 E8M0 bytes (2^(e-127), 0 -> 0.0 as F8E8M0::to_f32, src/dtype.rs:245-252).
 * out_dev receives rows*cols bf16 values, bit-exact with the reference. */
OXG_API int oxg_dequant_mxfp4(oxg_ctx *ctx, const uint8_t *blocks_dev, size_t n_block_bytes,
                              const void *scales_dev, size_t n_scales, int scale_fmt, size_t rows,
                              size_t cols, uint16_t *out_dev);

/* ---- SwiGLU -------------------------------------------------------------- */

/* Replaces ffn::swiglu(gate, up) (src/ffn.rs:5-13) with the clamped gpt-oss
 * form: g <- min(g, limit); u <- clamp(u, -limit, limit);
 * out = g * sigmoid(alpha * g) * (u + 1). Device f32 arrays of n elements. */
OXG_API int oxg_swiglu(oxg_ctx *ctx, const float *gate_dev, const float *up_dev, size_t n,
                       float alpha, float limit, float *out_dev);

/* ---- MoE layer ----------------------------------------------------------- */

typedef struct {
  int hidden;         /* H (2880 for gpt-oss-20b); multiple of 32 */
  int intermediate;   /* I (2880); multiple of 32; mlp1 has 2*I rows */
  int n_experts;      /* E (32); <= 256 */
  int top_k;          /* k (4; the reference hard-codes 4, src/moe.rs:56); <= 16 */
  float swiglu_alpha; /* 1.702 */
  float swiglu_limit; /* 7.0; 0 < limit <= 128 */
} oxg_moe_dims;

typedef struct {
  const uint16_t *router_w;  /* [E, H] bf16 ("mlp.router.weight", src/model.rs:239) */
  const uint16_t *router_b;  /* [E] bf16, or NULL for no bias */
  const uint8_t *w1_blocks;  /* [E, 2I, H/2] packed E2M1 ("mlp1_weight.blocks"), gate/up rows interleaved */
  const uint8_t *w1_scales;  /* [E, 2I, H/32] E8M0 */
  const uint16_t *b1;        /* [E, 2I] bf16 */
  const uint8_t *w2_blocks;  /* [E, H, I/2] */
  const uint8_t *w2_scales;  /* [E, H, I/32] */
  const uint16_t *b2;        /* [E, H] bf16 */
} oxg_moe_weights;

/* Replaces the MoE branch of load_transformer_layer (src/model.rs:238-359)
 * and the dequantising loader path (src/loader.rs:42-73): copies one layer's
 * packed weights (host or device pointers) into library-owned device memory,
 * still packed (no bf16 materialisation). Synchronous. Re-uploading a layer
 * replaces it. */
OXG_API int oxg_moe_upload(oxg_ctx *ctx, int layer, const oxg_moe_dims *dims,
                           const oxg_moe_weights *w);
OXG_API int oxg_moe_release(oxg_ctx *ctx, int layer);

/* Pre-sizes the context's scratch memory for n_tokens tokens of `layer`, so
 * that later forwards of at most that many tokens allocate nothing. */
OXG_API int oxg_moe_reserve(oxg_ctx *ctx, int layer, int n_tokens);

/* Replaces MoELayer::forward(&self, hidden: &MetalBuffer, compute) -> Result<MetalBuffer>
 * (src/moe.rs:16-100): router + top-k + softmax, permutation, expert MLPs
 * with clamped SwiGLU, weighted combine. x_dev: [n_tokens, H] bf16;
 * y_dev: [n_tokens, H] f32. mode: OXG_MODE_AUTO or OXG_MODE_DECODE (the
 * in-register-dequant tensor-core path); precision: OXG_PRECISION_PARITY. */
OXG_API int oxg_moe_forward(oxg_ctx *ctx, int layer, const uint16_t *x_dev, int n_tokens,
                            float *y_dev, int mode, int precision);

/* The same from host memory (pinned for full speed): copies x in, runs the
 * layer, copies y out and waits. This is the call a host-side runner makes. */
OXG_API int oxg_moe_forward_host(oxg_ctx *ctx, int layer, const uint16_t *x_host, int n_tokens,
                                 float *y_host, int mode, int precision);

/* Tokens per chunk for oxg_moe_forward_host on batches of at least twice
 * that many tokens: the chunks' host->device copies, kernels and
 * device->host copies overlap on three streams (results per token are the
 * same as one forward). 0: automatic (1600), < 0: never chunk, else > 64.
 * No counterpart in the reference (its forward runs on the host). */
OXG_API int oxg_ctx_set_host_chunk(oxg_ctx *ctx, int tokens);

/* Routing tap (src/moe.rs:40-73): idx_dev [n_tokens, k] int32 expert ids in
 * selection order, w_dev [n_tokens, k] f32 softmax weights; logits_dev
 * [n_tokens, E] f32 may be NULL. */
OXG_API int oxg_moe_route(oxg_ctx *ctx, int layer, const uint16_t *x_dev, int n_tokens,
                          int32_t *idx_dev, float *w_dev, float *logits_dev);

/* Per-expert token counts of the last forward on this context (host array of
 * E ints). Waits for the context's stream. */
OXG_API int oxg_moe_last_counts(oxg_ctx *ctx, int32_t *counts_host, int n_experts);

/* ---- Expert parallelism ------------------------------------------------------
 * No counterpart in the reference, which runs every expert of a layer in one
 * process (MoELayer::forward, src/moe.rs:76-97). With N processes, one per
 * GPU, each holding a contiguous range of a layer's experts:
 *   1. oxg_moe_dispatch routes the process's own tokens and writes their
 *      n_tokens * k slot rows expert-major (so also destination-process-major)
 *      into caller buffers, with the per-expert row counts;
 *   2. the caller exchanges the rows (an all-to-all) so that every process
 *      receives, source process by source process, the rows of its own
 *      experts in expert order;
 *   3. oxg_moe_experts runs the resident experts' MLPs over the received rows;
 *   4. the caller returns the output rows to their sources (the reverse
 *      all-to-all), which then lie in the order step 1 wrote;
 *   5. oxg_moe_combine forms y = sum_j w_j * row(t, j), as oxg_moe_forward does.
 * Rows are the prefill operand: f16 x * 2^-sigma (hidden halves per row) with a
 * per-row f32 2^sigma; all four calls need a layer the prefill kernels accept
 * (hidden and intermediate multiples of 64, E8M0 scales 0 or in [104, 140]). */

/* Uploads the router (all n_experts rows) and experts [expert_begin,
 * expert_begin + expert_count) of the given weights, whose arrays hold every
 * expert (oxg_moe_weights layout). oxg_moe_forward refuses such a layer
 * unless the range is all experts. */
OXG_API int oxg_moe_upload_shard(oxg_ctx *ctx, int layer, const oxg_moe_dims *dims,
                                 const oxg_moe_weights *weights, int expert_begin,
                                 int expert_count);

/* rows_dev [n_tokens*k, hidden] f16 and row_scale_dev [n_tokens*k] f32 (both
 * device, 16- and 4-byte aligned), expert_counts_dev [n_experts] int32. The
 * positions and routing weights stay on the context for oxg_moe_combine until
 * the next dispatch or forward on it. */
OXG_API int oxg_moe_dispatch(oxg_ctx *ctx, int layer, const uint16_t *x_dev, int n_tokens,
                             uint16_t *rows_dev, float *row_scale_dev, int32_t *expert_counts_dev);

/* rows_dev/row_scale_dev: the received rows, seg_counts_host [n_src *
 * expert_count] (host) the number from source s for resident expert e at
 * s * expert_count + e, in row order. Writes y_rows_dev [sum, hidden] f32
 * (16-byte aligned): each row's expert output with bias, before the routing
 * weight. n_src * expert_count must not exceed 256. */
OXG_API int oxg_moe_experts(oxg_ctx *ctx, int layer, const uint16_t *rows_dev,
                            const float *row_scale_dev, int n_src, const int32_t *seg_counts_host,
                            float *y_rows_dev);

/* y_rows_dev [n_tokens*k, hidden] f32 in the order oxg_moe_dispatch wrote
 * rows_dev; y_dev [n_tokens, hidden] f32. n_tokens must be the dispatch's. */
OXG_API int oxg_moe_combine(oxg_ctx *ctx, int layer, const float *y_rows_dev, int n_tokens,
                            float *y_dev);

/* The same exchange done by the library's own kernels over NVLink peer memory
 * (no host round trip per forward): every process allocates one buffer
 * (oxg_ep_init, which writes its 64-byte CUDA IPC handle to handle_out), the
 * processes exchange the handles, and each maps the others' (oxg_ep_connect,
 * handles: world x 64 bytes in rank order). oxg_moe_forward_ep then takes a
 * process's own n_tokens (<= max_tokens) to y_dev [n_tokens, hidden] f32:
 * rows are stored straight into the owner's receive buffer, output rows
 * straight back into the source's, and per-forward counts and completion
 * flags travel the same way; every wait is bounded and a failure on one
 * process is reported by all (oxg_sync returns it). All processes must call
 * oxg_moe_forward_ep the same number of times (n_tokens may be 0). The layer
 * must hold experts [rank * E / world, (rank + 1) * E / world); E a multiple
 * of 16 and of world, at most 64; world at most 8. max_recv_rows caps the rows
 * one process can receive per forward (<= 0: world * max_tokens * k, the
 * worst case). Call oxg_ep_close on every process after all of them have
 * finished their last forward. */
OXG_API int oxg_ep_init(oxg_ctx *ctx, int layer, int rank, int world, int max_tokens,
                        long long max_recv_rows, void *handle_out);
OXG_API int oxg_ep_connect(oxg_ctx *ctx, const void *handles);
OXG_API int oxg_moe_forward_ep(oxg_ctx *ctx, int layer, const uint16_t *x_dev, int n_tokens,
                               float *y_dev);
OXG_API int oxg_ep_close(oxg_ctx *ctx);
/* Decode-sized exchanges (no counterpart in the reference): forwards of at
 * most `tokens` tokens (<= 64; 0, the default: none) process the rows this
 * process receives with the grouped decode kernels (the rows of each resident
 * expert in groups of at most 8, each group an equal share of the GPU)
 * instead of the prefill GEMMs; outputs agree with oxg_moe_forward within the
 * layer tolerance instead of bit for bit. Set the same value on every process
 * after oxg_ep_connect. */
OXG_API int oxg_ep_set_decode_tokens(oxg_ctx *ctx, int tokens);
/* Failure detection (no counterpart in the reference): every wait of an
 * expert-parallel forward on another process's flag gives up after `seconds`
 * (default ~2 s of SM clock; at least 1e-4) and the forward then reports
 * OXG_ERR_TIMEOUT at the next oxg_sync, the context still usable. A process
 * that stops taking part (it left, or skips a step) is found this way. Set
 * after oxg_ep_init. */
OXG_API int oxg_ep_set_wait_budget(oxg_ctx *ctx, double seconds);
/* Rows this process received in its last oxg_moe_forward_ep (waits for it). */
OXG_API int oxg_ep_last_received(oxg_ctx *ctx, long long *rows);

/* Has no counterpart in the reference. The same layer math as
 * oxg_moe_forward (router, top-k, expert MLPs, weighted combine; outputs
 * within the layer tolerance of oxg_moe_forward's, not bit-identical: the
 * small-batch path of oxg_moe_forward sums in another order), for callers
 * that must not have the library allocate device memory during a forward: serving runtimes
 * that reserve the whole GPU for their own memory pool, decode loops that
 * cannot absorb the synchronisation a cudaMalloc/cudaFree may cause, and
 * embedders that forbid foreign code from allocating. This call allocates
 * nothing (no cudaMalloc, cudaFree or allocating library routine): its
 * working memory is one fixed 4 MiB array compiled into the library, which
 * every GPU that loads the library holds until the process exits. The layer
 * must have been uploaded before (the upload allocates, once); x_dev/y_dev are
 * as for oxg_moe_forward. Batches whose scratch exceeds 4 MiB are refused with
 * OXG_ERR_SHAPE and a message giving the largest token count that fits (45
 * tokens of a gpt-oss-20b layer). The first call on a device looks up the
 * array's device address (cudaGetSymbolAddress, done once per device), so make
 * that first call before any stream capture; the address is cached for the
 * life of the process, so do not use this call after a cudaDeviceReset. A
 * layer uploaded as an expert-parallel shard is refused (OXG_ERR_STATE). All
 * calls share the one array and
 * it keeps the last call's contents (every part is rewritten before it is read,
 * so nothing is cleared); calls that overlap on the GPU — concurrent streams,
 * contexts or threads on the same device — race on it and must be serialised
 * by the caller. */
OXG_API int oxg_moe_forward_noalloc(oxg_ctx *ctx, int layer, const uint16_t *x_dev,
                                    int n_tokens, float *y_dev);

/* ---- Full decoder (gpt-oss-20b architecture) --------------------------------
 * The transformer around the MoE block, for greedy generation on one GPU:
 * embedding, per layer RMSNorm -> q/k/v projections + RoPE -> attention
 * (GQA, sliding window on even layers, learned sinks) -> o projection +
 * residual -> RMSNorm -> MoE block (the layer's oxg_moe_upload) + residual,
 * final RMSNorm, LM head, argmax. Replaces GPTModel (src/model.rs:19-27,
 * 713-741), TransformerLayer::forward (src/model.rs:848-887),
 * Attention::forward (src/model.rs:899-1084) and InferenceEngine's greedy
 * loop (src/inference.rs:62-97). Activations are bf16 into every matrix
 * product and f32 in the residual stream; K/V are cached as bf16. */

typedef struct {
  int n_layers;        /* 24 */
  int hidden;          /* H = 2880; multiple of 64, equal to the MoE layers' hidden */
  int n_heads;         /* 64 query heads */
  int n_kv_heads;      /* 8; n_heads / n_kv_heads <= 16 */
  int head_dim;        /* 64 (the only supported value) */
  int vocab;           /* 201088 */
  int sliding_window;  /* 128: even-indexed layers see keys p-127..p (src/config.rs:93-101); 0: none */
  int max_seq;         /* KV-cache capacity in positions */
  int max_tokens;      /* largest n_tokens of one oxg_model_forward (prompts are chunked) */
  float rope_theta;    /* 150000 (src/config.rs:122) */
  float rms_eps;       /* 1e-5 (src/model.rs:433) */
  int max_batch;       /* sequences with a KV cache of their own (0 or 1: one), at most min(128, max_tokens) */
  int kv_pages;        /* paged KV cache: pages of 64 positions in the pool every sequence draws from as it
                          grows (per layer and kv head); 0: max_batch * ceil(max_seq / 64), room for every
                          sequence at max_seq. A step that needs a page when none is free fails with
                          OXG_ERR_OOM and changes nothing; oxg_model_reset / oxg_model_reset_seq free them. */
} oxg_model_dims;

/* One layer's attention weights (host or device pointers, bf16 unless noted;
 * checkpoint names of src/model.rs:148-412). */
typedef struct {
  const uint16_t *attn_norm;       /* [H] "input_layernorm.weight" */
  const uint16_t *wq, *wk, *wv;    /* [n_heads*64, H], [n_kv_heads*64, H] x 2 "self_attn.{q,k,v}_proj.weight" */
  const uint16_t *bq, *bk, *bv;    /* biases [rows] or NULL (zero) */
  const uint16_t *wo;              /* [H, n_heads*64] "self_attn.o_proj.weight" */
  const uint16_t *bo;              /* [H] or NULL */
  const uint16_t *sinks;           /* [n_heads] learned sink logits, or NULL for none */
  const uint16_t *mlp_norm;        /* [H] "post_attention_layernorm.weight" */
} oxg_attn_weights;

/* Allocates the KV cache, RoPE tables and activations for `dims` (replacing
 * any earlier model on the context). */
OXG_API int oxg_model_init(oxg_ctx *ctx, const oxg_model_dims *dims);
/* Token embedding [V, H], LM head [V, H] ("lm_head.weight"; pass the
 * embedding again for tied weights) and final norm [H] (src/model.rs:98-138). */
OXG_API int oxg_model_upload_embeddings(oxg_ctx *ctx, const uint16_t *embed, const uint16_t *unembed,
                                        const uint16_t *final_norm);
OXG_API int oxg_model_upload_attention(oxg_ctx *ctx, int layer, const oxg_attn_weights *w);
/* Empties the KV cache (GPTModel::reset_kv_cache, src/model.rs:743-747). */
OXG_API int oxg_model_reset(oxg_ctx *ctx);
/* Empties one sequence's KV cache and returns its pages to the pool (the
 * reference keeps one sequence per model: this is reset_kv_cache,
 * src/model.rs:743-747, for sequence `seq` of a batched model). */
OXG_API int oxg_model_reset_seq(oxg_ctx *ctx, int seq);
/* Pages of the KV-cache pool in use and in total. */
OXG_API int oxg_model_kv_pages(oxg_ctx *ctx, int *used, int *total);
/* Number of positions in the KV cache. */
OXG_API int oxg_model_position(oxg_ctx *ctx, int *pos);
/* GPTModel::forward (src/model.rs:713-741) on device data: appends n_tokens
 * tokens (int32 ids, device) at the current position, and for the last
 * n_logits of them (0 <= n_logits <= min(n_tokens, 128)) writes the logits
 * [n_logits, V] f32 to logits_dev and the greedy choice (argmax, ties to the
 * last index as src/sampler.rs:7-16) to next_dev [n_logits]; either output may
 * be NULL. Asynchronous on the context's stream; a token id outside [0, V)
 * is reported by the next oxg_sync. */
OXG_API int oxg_model_forward(oxg_ctx *ctx, const int32_t *tokens_dev, int n_tokens, int n_logits,
                              float *logits_dev, int32_t *next_dev);
/* The decode loop of src/inference.rs:77-92 at temperature 0 on the device:
 * n_steps one-token steps, each feeding the previous greedy token back,
 * starting from the greedy token of the last oxg_model_forward (which must
 * have had n_logits >= 1) or of the last step; tokens_dev [n_steps] receives
 * the new tokens. The step is captured once as a CUDA graph and replayed
 * (the first step of a call runs eagerly; the capture is redone when layers
 * or the scratch were reallocated). Asynchronous. */
OXG_API int oxg_model_decode(oxg_ctx *ctx, int n_steps, int32_t *tokens_dev);
/* InferenceEngine::generate_chat's loop at temperature 0 (src/inference.rs:62-97)
 * from host memory: empties the cache, runs the prompt (in chunks of
 * max_tokens), then n_new - 1 one-token steps that feed each greedy token back
 * on the device; writes the n_new generated ids to tokens_host. Synchronous. */
OXG_API int oxg_model_generate(oxg_ctx *ctx, const int32_t *prompt_host, int n_prompt, int n_new,
                               int32_t *tokens_host);
/* Routing tap (the expert ids src/moe.rs:51-73 chooses, per layer): while
 * set, every oxg_model_forward of at most max_tokens tokens copies each
 * layer's chosen experts [n_tokens, k] (int32, selection order) to
 * idx_dev + layer * max_tokens * k. NULL switches it off. Graph-replayed
 * decode steps do not record. */
OXG_API int oxg_model_route_tap(oxg_ctx *ctx, int32_t *idx_dev, int max_tokens);
/* Several sequences at once (the reference runs one sequence per GPTModel;
 * this is GPTModel::forward, src/model.rs:713-741, applied to max_batch
 * independent KV caches). Sequence 0 is the one oxg_model_forward, _decode
 * and _generate use; oxg_model_reset empties every sequence.
 * oxg_model_prefill_seq appends n_tokens tokens (device) to sequence seq's
 * cache and writes its greedy next token to next_dev [1] (may be NULL).
 * oxg_model_step_batch appends one token to each of sequences 0 .. n_seqs-1
 * (tokens_dev [n_seqs]; n_seqs <= max_batch) as one batch of n_seqs tokens
 * through every layer — each attends to its own cache only — and writes the
 * greedy next tokens to next_dev [n_seqs] and, if not NULL, the logits
 * [n_seqs, V] f32 to logits_dev. Both asynchronous on the context's stream. */
OXG_API int oxg_model_prefill_seq(oxg_ctx *ctx, int seq, const int32_t *tokens_dev, int n_tokens,
                                  int32_t *next_dev);
OXG_API int oxg_model_step_batch(oxg_ctx *ctx, int n_seqs, const int32_t *tokens_dev, int32_t *next_dev,
                                 float *logits_dev);
OXG_API int oxg_model_release(oxg_ctx *ctx);

/* ---- measurement (no reference counterpart: the reference's only timing is
 * the --bench wall clock of src/main.rs:159-164) --------------------------- */

/* When on, every kernel this context launches is bracketed by CUDA events on
 * the launching stream. */
OXG_API int oxg_profile_enable(oxg_ctx *ctx, int on);
/* Total device time (ms) and launch count of kernel `name` since the last
 * reset (names: router_topk, permute, moe_mlp1_decode, moe_mlp2_decode,
 * combine, dequant_mxfp4, swiglu). Waits for the context's stream. */
OXG_API int oxg_profile_read(oxg_ctx *ctx, const char *name, double *total_ms, int *launches);
OXG_API int oxg_profile_reset(oxg_ctx *ctx);
/* Number of kernels this context has launched since it was created. */
OXG_API int oxg_kernel_launches(const oxg_ctx *ctx, long long *count);
/* Tensor-core issue rate of one instruction kind, measured on this
 * context's device: one CTA per SM issues `iters` back-to-back MMAs of
 * M 128 x N 256 from shared memory into TMEM (no global traffic) and the
 * rate is the algorithmic FLOPs over the launch's CUDA-event time.
 * kind: 0 = kind::f16 (K 16), 1 = kind::mxf8f6f4.block_scale with E2M1 x
 * E4M3 (K 32, the block-scaled MoE kernels' instruction), 2 =
 * kind::mxf4.block_scale with E2M1 x E2M1 (K 64, the dense MXFP4 rate).
 * Synchronous; *tflops receives TFLOP/s. */
OXG_API int oxg_measure_mma_rate(oxg_ctx *ctx, int kind, int iters, double *tflops);

#ifdef __cplusplus
}
#endif
#endif /* OXG_B200_H */
