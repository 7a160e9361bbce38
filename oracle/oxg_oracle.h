/*
 * oxg_oracle.h — CPU oracle for the MXFP4 mixture-of-experts hot path.
 *
 * TEST INFRASTRUCTURE ONLY. This is a plain-C restatement of the reference
 * runner's (cipher-rc5/oxidized_gpt_oss) MoE hot path. It is the checker for
 * the CUDA library and the timed CPU baseline; it is never linked into the
 * product library and nothing in the product calls it. Only tests/,
 * __graft_entry__.smoke() and bench.py's CPU legs load it.
 *
 * Two variants of the MoE layer are provided:
 *
 *   SPEC           gpt-oss semantics: E8M0 block scales, router bias, top-4
 *                  then softmax over the 4, gate/up interleaved mlp1 (even rows
 *                  gate, odd rows up), clamped SwiGLU, fp32 output; optional
 *                  fp64 accumulation. This is the graded oracle.
 *   REF-FAITHFUL   the reference algorithm as written: every buffer stored as
 *                  IEEE f16, full expert weights converted f16->f32 on every
 *                  (token, expert) call, sequential f32 A*B^T loops, plain
 *                  SiLU, no router bias, f16 output. Documentary, and the
 *                  CPU baseline for timing.
 *
 * Pinning: the dequantisation is pinned bit-exactly by the reference's own
 * known-answer test (src/mxfp4.rs:63-95) and sanity test
 * (tests/integration.rs:30-48); see tests/golden/. Router, top-k, SwiGLU,
 * expert MLP and combine are NOT pinned by any reference test or fixture
 * ("parity unpinned"): they follow the reference source line by line where it
 * defines the behaviour, and the gpt-oss definition where it is silent.
 */
#ifndef OXG_ORACLE_H
#define OXG_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- scalar conversions (half 2.7.1 semantics: IEEE round-to-nearest-even) ---- */
uint16_t oxo_f32_to_bf16(float v);
float oxo_bf16_to_f32(uint16_t b);
uint16_t oxo_f32_to_f16(float v);
float oxo_f16_to_f32(uint16_t h);
/* F8E8M0::to_f32, src/dtype.rs:245-252: 0 -> 0.0, else 2^(e-127) (255 -> inf). */
float oxo_e8m0_to_f32(uint8_t e);
/* The E8M0 -> bf16-bits adapter used to feed E8M0 scales to the reference's
 * bf16-scale dequantiser: bits = e << 7 (exactly 2^(e-127); 0 -> +0.0; 255 -> +inf). */
uint16_t oxo_e8m0_to_bf16_bits(uint8_t e);
/* decode_e2m1, src/mxfp4.rs:9-13 (code 8 -> -0.0). */
float oxo_decode_e2m1(uint8_t nibble);

/* dequantize_mxfp4, src/mxfp4.rs:15-54. scales are bf16 bit patterns (u16),
 * one per 32 consecutive elements of a row. Returns 0, or -2 with a message
 * mirroring the reference's assert text. */
int oxo_dequantize_mxfp4(const uint8_t *blocks, size_t n_blocks, const uint16_t *scales,
                         size_t n_scales, size_t rows, size_t cols, uint16_t *out, char *err,
                         size_t err_len);
/* Same, with one E8M0 byte per block (adapter e << 7). */
int oxo_dequantize_mxfp4_e8m0(const uint8_t *blocks, size_t n_blocks, const uint8_t *scales,
                              size_t n_scales, size_t rows, size_t cols, uint16_t *out,
                              char *err, size_t err_len);

/* ---- MoE layer ---- */
typedef struct {
  int hidden;       /* H */
  int intermediate; /* I; mlp1 has 2*I rows */
  int n_experts;    /* E */
  int top_k;        /* k (the reference hard-codes 4, src/moe.rs:56) */
  float alpha;      /* SwiGLU alpha (1.702) */
  float limit;      /* SwiGLU clamp limit (7.0) */
  const uint16_t *router_w; /* [E, H] bf16 */
  const uint16_t *router_b; /* [E] bf16, may be NULL (no bias) */
  const uint8_t *w1_blocks; /* [E, 2I, H/2] packed E2M1, low nibble = even element */
  const uint8_t *w1_scales; /* [E, 2I, H/32] E8M0 */
  const uint16_t *b1;       /* [E, 2I] bf16 */
  const uint8_t *w2_blocks; /* [E, H, I/2] */
  const uint8_t *w2_scales; /* [E, H, I/32] */
  const uint16_t *b2;       /* [E, H] bf16 */
} oxo_moe_weights;

/* Router logits [T, E]: sequential f32 sum of x*W (mul then add, no FMA),
 * matmul src/utils.rs:77-87, plus the bf16 bias when router_b != NULL. */
void oxo_router_logits(const oxo_moe_weights *w, const uint16_t *x, int T, float *logits);
/* Stable descending sort (ties: lower expert index first), take k, softmax
 * over the k (src/moe.rs:51-73, src/utils.rs:91-111). */
void oxo_topk_softmax(const float *logits, int T, int E, int k, int32_t *idx, float *wts);
/* Clamped SwiGLU (gpt-oss): g <- min(g, limit); u <- clamp(u, -limit, limit);
 * out = g * sigmoid(alpha * g) * (u + 1). */
void oxo_swiglu_clamped(const float *gate, const float *up, size_t n, float alpha, float limit,
                        float *out);
/* ffn::swiglu, src/ffn.rs:5-13: silu(g) * u. */
void oxo_swiglu_plain(const float *gate, const float *up, size_t n, float *out);

/* SPEC forward. y: [T, H] fp32. If idx/wts are non-NULL they are used as the
 * routing (lets a test substitute a routing decided elsewhere on exact
 * near-ties); otherwise the layer routes itself. acc64 != 0 accumulates in
 * fp64. slot_y (optional, [T*k, H]) receives each (token, j) expert output
 * before weighting. nthreads <= 0 means all cores. Returns 0 or <0. */
int oxo_moe_forward_spec(const oxo_moe_weights *w, const uint16_t *x, int T, const int32_t *idx,
                         const float *wts, float *y, float *slot_y, int acc64, int nthreads);

/* REF-FAITHFUL forward: f16 in (x given as bf16 and rounded to f16 as the
 * reference's f16 buffers do), f16 out. Time-faithful to the reference:
 * converts the full f16 expert weights to f32 on every (token, expert) call.
 * nthreads <= 0 means all cores (parallel over tokens). */
int oxo_moe_forward_ref_faithful(const oxo_moe_weights *w, const uint16_t *x, int T,
                                 uint16_t *y_f16, int nthreads);

/* The same split at the reference's load/forward boundary, so that a timing
 * of the forward excludes load-time work: prepare does the load-time f16
 * materialisation (src/model.rs:238-359) of the router and of the experts
 * that x routes to; forward is MoELayer::forward (src/moe.rs:16-100) and
 * returns -4 if x routes to an expert that was not prepared. */
typedef struct oxo_ref_layer oxo_ref_layer;
oxo_ref_layer *oxo_ref_prepare(const oxo_moe_weights *w, const uint16_t *x, int T);
int oxo_ref_forward(const oxo_ref_layer *L, const uint16_t *x, int T, uint16_t *y_f16, int nthreads);
void oxo_ref_free(oxo_ref_layer *L);

/* Threads the oracle's OpenMP regions can use. */
int oxo_max_threads(void);

#ifdef __cplusplus
}
#endif
#endif
