/*
 * oxg_oracle.c — CPU oracle for the MXFP4 MoE hot path (TEST INFRASTRUCTURE
 * ONLY; see oxg_oracle.h for what it is and who may use it).
 *
 * Build with -O2 -ffp-contract=off so that every "sum += a * b" is a rounded
 * multiply followed by a rounded add, as in the reference's Rust loops.
 */
#include "oxg_oracle.h"

#include <math.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

/* ------------------------------------------------------------------------ */
/* scalar conversions                                                       */
/* ------------------------------------------------------------------------ */

static inline uint32_t f2u(float f) {
  uint32_t u;
  memcpy(&u, &f, 4);
  return u;
}
static inline float u2f(uint32_t u) {
  float f;
  memcpy(&f, &u, 4);
  return f;
}

/* bf16::from_f32 of half 2.7.1: NaN keeps its sign and top payload bits and
 * gets the quiet bit; everything else rounds to nearest, ties to even. */
uint16_t oxo_f32_to_bf16(float v) {
  uint32_t x = f2u(v);
  if ((x & 0x7FFFFFFFu) > 0x7F800000u) return (uint16_t)((x >> 16) | 0x0040u);
  uint32_t hi = x >> 16;
  uint32_t rest = x & 0xFFFFu;
  if (rest > 0x8000u || (rest == 0x8000u && (hi & 1u))) hi += 1;
  return (uint16_t)hi;
}

float oxo_bf16_to_f32(uint16_t b) { return u2f((uint32_t)b << 16); }

/* IEEE binary32 -> binary16, round to nearest even, overflow to inf,
 * gradual underflow; NaN stays NaN (quiet bit set). */
uint16_t oxo_f32_to_f16(float v) {
  uint32_t x = f2u(v);
  uint32_t sign = (x >> 16) & 0x8000u;
  uint32_t ex = (x >> 23) & 0xFFu;
  uint32_t man = x & 0x7FFFFFu;
  if (ex == 0xFFu) return (uint16_t)(sign | 0x7C00u | (man ? (0x200u | (man >> 13)) : 0u));
  int e = (int)ex - 127 + 15;
  if (e >= 31) return (uint16_t)(sign | 0x7C00u);
  if (e <= 0) {
    if (e < -10) return (uint16_t)sign; /* below half the smallest subnormal */
    uint32_t m = man | 0x800000u;       /* hidden bit */
    int shift = 14 - e;                 /* 14..24 */
    uint32_t hm = m >> shift;
    uint32_t rem = m & ((1u << shift) - 1u);
    uint32_t half = 1u << (shift - 1);
    if (rem > half || (rem == half && (hm & 1u))) hm += 1;
    return (uint16_t)(sign | hm);
  }
  uint32_t h = sign | ((uint32_t)e << 10) | (man >> 13);
  uint32_t rem = man & 0x1FFFu;
  if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) h += 1; /* may carry into inf: correct */
  return (uint16_t)h;
}

float oxo_f16_to_f32(uint16_t h) {
  uint32_t sign = ((uint32_t)h & 0x8000u) << 16;
  uint32_t ex = (h >> 10) & 0x1Fu;
  uint32_t man = h & 0x3FFu;
  if (ex == 0x1Fu) return u2f(sign | 0x7F800000u | (man << 13));
  if (ex == 0) {
    if (man == 0) return u2f(sign);
    /* subnormal: man * 2^-24, exact in f32 */
    float f = (float)man * (1.0f / 16777216.0f);
    return sign ? -f : f;
  }
  return u2f(sign | ((ex + 112u) << 23) | (man << 13));
}

float oxo_e8m0_to_f32(uint8_t e) {
  /* src/dtype.rs:245-252: 0 -> 0.0, else 2.0f32.powi(e - 127); powi(128) = inf. */
  if (e == 0) return 0.0f;
  if (e == 255) return INFINITY;
  return u2f((uint32_t)e << 23); /* exact 2^(e-127) for 1..254 */
}

uint16_t oxo_e8m0_to_bf16_bits(uint8_t e) { return (uint16_t)((uint16_t)e << 7); }

/* E2M1_MAGNITUDES, src/mxfp4.rs:7 */
static const float kE2M1[8] = {0.0f, 0.5f, 1.0f, 1.5f, 2.0f, 3.0f, 4.0f, 6.0f};

float oxo_decode_e2m1(uint8_t nibble) {
  float m = kE2M1[nibble & 7u];
  return (nibble & 8u) ? -m : m;
}

/* ------------------------------------------------------------------------ */
/* dequantize_mxfp4, src/mxfp4.rs:15-54                                      */
/* ------------------------------------------------------------------------ */

static int dequant_check(size_t n_blocks, size_t n_scales, size_t rows, size_t cols, char *err,
                         size_t err_len) {
  if (cols % 32 != 0) {
    if (err) snprintf(err, err_len, "cols must be divisible by 32, got %zu", cols);
    return -2;
  }
  if (n_blocks != rows * cols / 2) {
    if (err)
      snprintf(err, err_len, "blocks length mismatch: expected %zu, got %zu", rows * cols / 2,
               n_blocks);
    return -2;
  }
  if (n_scales != rows * (cols / 32)) {
    if (err)
      snprintf(err, err_len, "scales length mismatch: expected %zu, got %zu", rows * (cols / 32),
               n_scales);
    return -2;
  }
  return 0;
}

int oxo_dequantize_mxfp4(const uint8_t *blocks, size_t n_blocks, const uint16_t *scales,
                         size_t n_scales, size_t rows, size_t cols, uint16_t *out, char *err,
                         size_t err_len) {
  int rc = dequant_check(n_blocks, n_scales, rows, cols, err, err_len);
  if (rc) return rc;
  const size_t spr = cols / 32;
  for (size_t row = 0; row < rows; ++row) {
    for (size_t col = 0; col < cols; ++col) {
      size_t linear = row * cols + col;
      uint8_t packed = blocks[linear / 2];
      uint8_t nib = (linear % 2 == 0) ? (packed & 0x0F) : ((packed >> 4) & 0x0F);
      float scale = oxo_bf16_to_f32(scales[row * spr + col / 32]);
      float value = oxo_decode_e2m1(nib) * scale;
      out[linear] = oxo_f32_to_bf16(value);
    }
  }
  return 0;
}

int oxo_dequantize_mxfp4_e8m0(const uint8_t *blocks, size_t n_blocks, const uint8_t *scales,
                              size_t n_scales, size_t rows, size_t cols, uint16_t *out,
                              char *err, size_t err_len) {
  int rc = dequant_check(n_blocks, n_scales, rows, cols, err, err_len);
  if (rc) return rc;
  const size_t spr = cols / 32;
#pragma omp parallel for schedule(static)
  for (long long row = 0; row < (long long)rows; ++row) {
    for (size_t col = 0; col < cols; ++col) {
      size_t linear = (size_t)row * cols + col;
      uint8_t packed = blocks[linear / 2];
      uint8_t nib = (linear % 2 == 0) ? (packed & 0x0F) : ((packed >> 4) & 0x0F);
      float scale = oxo_bf16_to_f32(oxo_e8m0_to_bf16_bits(scales[(size_t)row * spr + col / 32]));
      out[linear] = oxo_f32_to_bf16(oxo_decode_e2m1(nib) * scale);
    }
  }
  return 0;
}

/* ------------------------------------------------------------------------ */
/* router, top-k, softmax                                                    */
/* ------------------------------------------------------------------------ */

void oxo_router_logits(const oxo_moe_weights *w, const uint16_t *x, int T, float *logits) {
  const int H = w->hidden, E = w->n_experts;
#pragma omp parallel for schedule(static)
  for (int t = 0; t < T; ++t) {
    for (int e = 0; e < E; ++e) {
      float sum = 0.0f; /* matmul, src/utils.rs:77-87 */
      for (int k = 0; k < H; ++k)
        sum += oxo_bf16_to_f32(x[(size_t)t * H + k]) * oxo_bf16_to_f32(w->router_w[(size_t)e * H + k]);
      if (w->router_b) sum += oxo_bf16_to_f32(w->router_b[e]);
      logits[(size_t)t * E + e] = sum;
    }
  }
}

/* softmax_inplace, src/utils.rs:91-111 */
static void softmax_inplace(float *v, int n) {
  if (n == 0) return;
  float mx = -INFINITY;
  for (int i = 0; i < n; ++i) mx = fmaxf(mx, v[i]);
  float sum = 0.0f;
  for (int i = 0; i < n; ++i) {
    v[i] = expf(v[i] - mx);
    sum += v[i];
  }
  if (sum == 0.0f) {
    for (int i = 0; i < n; ++i) v[i] = 1.0f / (float)n;
  } else {
    for (int i = 0; i < n; ++i) v[i] /= sum;
  }
}

void oxo_topk_softmax(const float *logits, int T, int E, int k, int32_t *idx, float *wts) {
  int kk = k < E ? k : E;
  for (int t = 0; t < T; ++t) {
    const float *l = logits + (size_t)t * E;
    /* Selection equivalent to a stable descending sort (src/moe.rs:53-54):
     * repeatedly take the largest remaining logit, lowest index on ties. */
    unsigned char used[1024];
    memset(used, 0, sizeof(used));
    float top[64];
    for (int j = 0; j < kk; ++j) {
      int best = -1;
      for (int e = 0; e < E; ++e) {
        if (used[e]) continue;
        if (best < 0 || l[e] > l[best]) best = e;
      }
      used[best] = 1;
      idx[(size_t)t * k + j] = best;
      top[j] = l[best];
    }
    softmax_inplace(top, kk);
    for (int j = 0; j < kk; ++j) wts[(size_t)t * k + j] = top[j];
  }
}

/* ------------------------------------------------------------------------ */
/* SwiGLU                                                                    */
/* ------------------------------------------------------------------------ */

/* Clamps written as comparisons so that NaN propagates, as torch.clamp does in
 * the gpt-oss definition. */
static inline float swiglu1(float g, float u, float alpha, float limit) {
  g = g > limit ? limit : g;
  u = u < -limit ? -limit : (u > limit ? limit : u);
  float sig = 1.0f / (1.0f + expf(-alpha * g));
  return g * sig * (u + 1.0f);
}

static inline double swiglu1_d(double g, double u, double alpha, double limit) {
  g = g > limit ? limit : g;
  u = u < -limit ? -limit : (u > limit ? limit : u);
  double sig = 1.0 / (1.0 + exp(-alpha * g));
  return g * sig * (u + 1.0);
}

void oxo_swiglu_clamped(const float *gate, const float *up, size_t n, float alpha, float limit,
                        float *out) {
  for (size_t i = 0; i < n; ++i) out[i] = swiglu1(gate[i], up[i], alpha, limit);
}

void oxo_swiglu_plain(const float *gate, const float *up, size_t n, float *out) {
  for (size_t i = 0; i < n; ++i) {
    float g = gate[i];
    float sig = 1.0f / (1.0f + expf(-g));
    out[i] = (g * sig) * up[i];
  }
}

/* ------------------------------------------------------------------------ */
/* SPEC MoE forward                                                          */
/* ------------------------------------------------------------------------ */

int oxo_max_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}

/* Decode one row of packed MXFP4 (cols elements) into floats. Exact. */
static void decode_row(const uint8_t *codes, const uint8_t *scales, int cols, float *dst) {
  for (int c = 0; c < cols; c += 2) {
    uint8_t b = codes[c / 2];
    float s = oxo_e8m0_to_f32(scales[c / 32]);
    dst[c] = oxo_decode_e2m1(b & 0x0F) * s;
    dst[c + 1] = oxo_decode_e2m1(b >> 4) * s;
  }
}

int oxo_moe_forward_spec(const oxo_moe_weights *w, const uint16_t *x, int T, const int32_t *idx_in,
                         const float *wts_in, float *y, float *slot_y, int acc64, int nthreads) {
  const int H = w->hidden, I = w->intermediate, E = w->n_experts, K = w->top_k;
  if (H % 32 || I % 32 || E <= 0 || K <= 0 || K > E || T < 0) return -1;
#ifdef _OPENMP
  if (nthreads > 0) omp_set_num_threads(nthreads);
#else
  (void)nthreads;
#endif
  if (T == 0) return 0;
  int32_t *idx = (int32_t *)malloc(sizeof(int32_t) * (size_t)T * K);
  float *wts = (float *)malloc(sizeof(float) * (size_t)T * K);
  float *xf = (float *)malloc(sizeof(float) * (size_t)T * H);
  double *h = (double *)malloc(sizeof(double) * (size_t)T * K * I); /* SwiGLU output per slot */
  double *ys = (double *)malloc(sizeof(double) * (size_t)T * K * H); /* expert output per slot */
  if (!idx || !wts || !xf || !h || !ys) {
    free(idx); free(wts); free(xf); free(h); free(ys);
    return -3;
  }
  for (size_t i = 0; i < (size_t)T * H; ++i) xf[i] = oxo_bf16_to_f32(x[i]);
  if (idx_in && wts_in) {
    memcpy(idx, idx_in, sizeof(int32_t) * (size_t)T * K);
    memcpy(wts, wts_in, sizeof(float) * (size_t)T * K);
  } else {
    float *logits = (float *)malloc(sizeof(float) * (size_t)T * E);
    oxo_router_logits(w, x, T, logits);
    oxo_topk_softmax(logits, T, E, K, idx, wts);
    free(logits);
  }

  /* For each expert, the (token, j) slots routed to it, in (t, j) order. */
  int *cnt = (int *)calloc((size_t)E, sizeof(int));
  int *off = (int *)calloc((size_t)E + 1, sizeof(int));
  int *slots = (int *)malloc(sizeof(int) * (size_t)T * K);
  for (int s = 0; s < T * K; ++s) cnt[idx[s]]++;
  for (int e = 0; e < E; ++e) off[e + 1] = off[e] + cnt[e];
  int *fill = (int *)calloc((size_t)E, sizeof(int));
  for (int s = 0; s < T * K; ++s) slots[off[idx[s]] + fill[idx[s]]++] = s;
  free(fill);

  const size_t r1 = (size_t)H / 2, s1 = (size_t)H / 32;
  const size_t r2 = (size_t)I / 2, s2 = (size_t)I / 32;
  for (int e = 0; e < E; ++e) {
    const int n = cnt[e];
    if (!n) continue;
    const int *es = slots + off[e];
    const uint8_t *c1 = w->w1_blocks + (size_t)e * 2 * I * r1;
    const uint8_t *sc1 = w->w1_scales + (size_t)e * 2 * I * s1;
    const uint8_t *c2 = w->w2_blocks + (size_t)e * H * r2;
    const uint8_t *sc2 = w->w2_scales + (size_t)e * H * s2;
    /* mlp1 (gate row 2p, up row 2p+1) + bias + clamped SwiGLU */
#pragma omp parallel
    {
      float *wg = (float *)malloc(sizeof(float) * (size_t)H);
      float *wu = (float *)malloc(sizeof(float) * (size_t)H);
#pragma omp for schedule(static)
      for (int p = 0; p < I; ++p) {
        decode_row(c1 + (size_t)(2 * p) * r1, sc1 + (size_t)(2 * p) * s1, H, wg);
        decode_row(c1 + (size_t)(2 * p + 1) * r1, sc1 + (size_t)(2 * p + 1) * s1, H, wu);
        const float bg = oxo_bf16_to_f32(w->b1[(size_t)e * 2 * I + 2 * p]);
        const float bu = oxo_bf16_to_f32(w->b1[(size_t)e * 2 * I + 2 * p + 1]);
        for (int q = 0; q < n; ++q) {
          const int s = es[q];
          const float *xr = xf + (size_t)(s / K) * H;
          if (acc64) {
            double ag = 0.0, au = 0.0;
            for (int k = 0; k < H; ++k) {
              ag += (double)xr[k] * (double)wg[k];
              au += (double)xr[k] * (double)wu[k];
            }
            h[(size_t)s * I + p] = swiglu1_d(ag + bg, au + bu, w->alpha, w->limit);
          } else {
            float ag = 0.0f, au = 0.0f;
            for (int k = 0; k < H; ++k) {
              ag += xr[k] * wg[k];
              au += xr[k] * wu[k];
            }
            h[(size_t)s * I + p] = swiglu1(ag + bg, au + bu, w->alpha, w->limit);
          }
        }
      }
      free(wg);
      free(wu);
    }
    /* mlp2 + bias */
#pragma omp parallel
    {
      float *wd = (float *)malloc(sizeof(float) * (size_t)I);
#pragma omp for schedule(static)
      for (int r = 0; r < H; ++r) {
        decode_row(c2 + (size_t)r * r2, sc2 + (size_t)r * s2, I, wd);
        const float bd = oxo_bf16_to_f32(w->b2[(size_t)e * H + r]);
        for (int q = 0; q < n; ++q) {
          const int s = es[q];
          const double *hr = h + (size_t)s * I;
          if (acc64) {
            double a = 0.0;
            for (int k = 0; k < I; ++k) a += hr[k] * (double)wd[k];
            ys[(size_t)s * H + r] = a + bd;
          } else {
            float a = 0.0f;
            for (int k = 0; k < I; ++k) a += (float)hr[k] * wd[k];
            ys[(size_t)s * H + r] = (double)(a + bd);
          }
        }
      }
      free(wd);
    }
  }
  /* weighted combine in j order, src/moe.rs:76-96 */
  for (int t = 0; t < T; ++t) {
    for (int c = 0; c < H; ++c) {
      if (acc64) {
        double a = 0.0;
        for (int j = 0; j < K; ++j) a += (double)wts[t * K + j] * ys[((size_t)t * K + j) * H + c];
        y[(size_t)t * H + c] = (float)a;
      } else {
        float a = 0.0f;
        for (int j = 0; j < K; ++j) a += wts[t * K + j] * (float)ys[((size_t)t * K + j) * H + c];
        y[(size_t)t * H + c] = a;
      }
    }
  }
  if (slot_y)
    for (size_t i = 0; i < (size_t)T * K * H; ++i) slot_y[i] = (float)ys[i];
  free(cnt); free(off); free(slots);
  free(idx); free(wts); free(xf); free(h); free(ys);
  return 0;
}

/* ------------------------------------------------------------------------ */
/* REF-FAITHFUL MoE forward                                                  */
/* ------------------------------------------------------------------------ */

/* matmul, src/utils.rs:34-89: A(m x k) * B^T, B stored (n x k), sequential f32. */
static void ref_matmul(const float *a, const float *b, int m, int k, int n, float *out) {
  for (int row = 0; row < m; ++row)
    for (int col = 0; col < n; ++col) {
      float sum = 0.0f;
      for (int inner = 0; inner < k; ++inner) sum += a[(size_t)row * k + inner] * b[(size_t)col * k + inner];
      out[(size_t)row * n + col] = sum;
    }
}

/* buffer_to_f32_vec, src/utils.rs:9-22: a fresh f32 copy of an f16 buffer. */
static float *f16_buffer_to_f32(const uint16_t *buf, size_t n) {
  float *o = (float *)malloc(sizeof(float) * n);
  for (size_t i = 0; i < n; ++i) o[i] = oxo_f16_to_f32(buf[i]);
  return o;
}

typedef struct {
  uint16_t *gate, *up, *down;   /* f16 buffers [I,H], [I,H], [H,I] */
  uint16_t *bg, *bu, *bd;       /* f16 biases */
} ref_expert;

struct oxo_ref_layer {
  int H, I, E, K;
  uint16_t *router;  /* f16 [E, H] */
  ref_expert *ex;    /* [E]; experts never prepared stay NULL */
};

/* Reference routing (src/moe.rs:22-73): f16 router buffer -> f32, sequential
 * matmul, no bias, stable top-k, softmax. */
static void ref_route(const oxo_ref_layer *L, const uint16_t *xh, int T, int32_t *idx, float *wts) {
  float *router = f16_buffer_to_f32(L->router, (size_t)L->E * L->H);
  float *hidden = f16_buffer_to_f32(xh, (size_t)T * L->H);
  float *logits = (float *)malloc(sizeof(float) * (size_t)T * L->E);
  ref_matmul(hidden, router, T, L->H, L->E, logits);
  oxo_topk_softmax(logits, T, L->E, L->K, idx, wts);
  free(logits); free(hidden); free(router);
}

static uint16_t *to_f16_buffer(const uint16_t *x_bf16, size_t n) {
  uint16_t *o = (uint16_t *)malloc(sizeof(uint16_t) * n);
  for (size_t i = 0; i < n; ++i) o[i] = oxo_f32_to_f16(oxo_bf16_to_f32(x_bf16[i]));
  return o;
}

oxo_ref_layer *oxo_ref_prepare(const oxo_moe_weights *w, const uint16_t *x, int T) {
  const int H = w->hidden, I = w->intermediate, E = w->n_experts;
  if (H % 32 || I % 32 || E <= 0 || T < 0) return NULL;
  oxo_ref_layer *L = (oxo_ref_layer *)calloc(1, sizeof(oxo_ref_layer));
  L->H = H; L->I = I; L->E = E; L->K = 4 < E ? 4 : E; /* hard-coded top-4, src/moe.rs:56 */
  L->router = to_f16_buffer(w->router_w, (size_t)E * H);
  L->ex = (ref_expert *)calloc((size_t)E, sizeof(ref_expert));
  /* Load-time materialisation (src/model.rs:238-359): f16 per-expert gate/up/down
   * buffers; gate = mlp1 even rows, up = mlp1 odd rows. Only the experts x routes to. */
  unsigned char *hit = (unsigned char *)calloc((size_t)E, 1);
  if (T > 0) {
    uint16_t *xh = to_f16_buffer(x, (size_t)T * H);
    int32_t *idx = (int32_t *)malloc(sizeof(int32_t) * (size_t)T * L->K);
    float *wts = (float *)malloc(sizeof(float) * (size_t)T * L->K);
    ref_route(L, xh, T, idx, wts);
    for (int s = 0; s < T * L->K; ++s) hit[idx[s]] = 1;
    free(idx); free(wts); free(xh);
  }
  const size_t r1 = (size_t)H / 2, s1 = (size_t)H / 32, r2 = (size_t)I / 2, s2 = (size_t)I / 32;
#pragma omp parallel for schedule(dynamic, 1)
  for (int e = 0; e < E; ++e) {
    if (!hit[e]) continue;
    ref_expert *xe = &L->ex[e];
    xe->gate = (uint16_t *)malloc(sizeof(uint16_t) * (size_t)I * H);
    xe->up = (uint16_t *)malloc(sizeof(uint16_t) * (size_t)I * H);
    xe->down = (uint16_t *)malloc(sizeof(uint16_t) * (size_t)H * I);
    xe->bg = (uint16_t *)malloc(sizeof(uint16_t) * (size_t)I);
    xe->bu = (uint16_t *)malloc(sizeof(uint16_t) * (size_t)I);
    xe->bd = (uint16_t *)malloc(sizeof(uint16_t) * (size_t)H);
    float *row = (float *)malloc(sizeof(float) * (size_t)(H > I ? H : I));
    for (int p = 0; p < I; ++p) {
      size_t rg = (size_t)e * 2 * I + 2 * p, ru = rg + 1;
      decode_row(w->w1_blocks + rg * r1, w->w1_scales + rg * s1, H, row);
      for (int k = 0; k < H; ++k) xe->gate[(size_t)p * H + k] = oxo_f32_to_f16(row[k]);
      decode_row(w->w1_blocks + ru * r1, w->w1_scales + ru * s1, H, row);
      for (int k = 0; k < H; ++k) xe->up[(size_t)p * H + k] = oxo_f32_to_f16(row[k]);
      xe->bg[p] = oxo_f32_to_f16(oxo_bf16_to_f32(w->b1[rg]));
      xe->bu[p] = oxo_f32_to_f16(oxo_bf16_to_f32(w->b1[ru]));
    }
    for (int r = 0; r < H; ++r) {
      size_t rr = (size_t)e * H + r;
      decode_row(w->w2_blocks + rr * r2, w->w2_scales + rr * s2, I, row);
      for (int k = 0; k < I; ++k) xe->down[(size_t)r * I + k] = oxo_f32_to_f16(row[k]);
      xe->bd[r] = oxo_f32_to_f16(oxo_bf16_to_f32(w->b2[rr]));
    }
    free(row);
  }
  free(hit);
  return L;
}

void oxo_ref_free(oxo_ref_layer *L) {
  if (!L) return;
  for (int e = 0; e < L->E; ++e) {
    free(L->ex[e].gate); free(L->ex[e].up); free(L->ex[e].down);
    free(L->ex[e].bg); free(L->ex[e].bu); free(L->ex[e].bd);
  }
  free(L->ex); free(L->router); free(L);
}

int oxo_ref_forward(const oxo_ref_layer *L, const uint16_t *x, int T, uint16_t *y_f16, int nthreads) {
  if (!L || T < 0) return -1;
#ifdef _OPENMP
  if (nthreads > 0) omp_set_num_threads(nthreads);
#else
  (void)nthreads;
#endif
  if (T == 0) return 0;
  const int H = L->H, I = L->I, K = L->K;
  /* The hidden states arrive as an f16 buffer (src/utils.rs:24-32). */
  uint16_t *xh = to_f16_buffer(x, (size_t)T * H);
  int32_t *idx = (int32_t *)malloc(sizeof(int32_t) * (size_t)T * K);
  float *wts = (float *)malloc(sizeof(float) * (size_t)T * K);
  ref_route(L, xh, T, idx, wts);
  for (int s = 0; s < T * K; ++s)
    if (!L->ex[idx[s]].gate) { free(idx); free(wts); free(xh); return -4; } /* not prepared */

  /* 3. per token, per selected expert (src/moe.rs:76-97) */
  float *final_h = (float *)calloc((size_t)T * H, sizeof(float));
#pragma omp parallel for schedule(dynamic, 1)
  for (int t = 0; t < T; ++t) {
    float *acc = final_h + (size_t)t * H;
    for (int j = 0; j < K; ++j) {
      const ref_expert *xp = &L->ex[idx[t * K + j]];
      const float weight = wts[t * K + j];
      /* token_buffer = buffer_from_f32(token) -> MLP::forward (src/model.rs:1088-1184) */
      float *tok = f16_buffer_to_f32(xh + (size_t)t * H, (size_t)H);
      float *gp = f16_buffer_to_f32(xp->gate, (size_t)I * H);
      float *g = (float *)malloc(sizeof(float) * (size_t)I);
      ref_matmul(tok, gp, 1, H, I, g);
      free(gp);
      float *bgf = f16_buffer_to_f32(xp->bg, (size_t)I);
      for (int i = 0; i < I; ++i) g[i] += bgf[i];
      free(bgf);
      for (int i = 0; i < I; ++i) g[i] = g[i] * (1.0f / (1.0f + expf(-g[i]))); /* silu */
      float *up = f16_buffer_to_f32(xp->up, (size_t)I * H);
      float *u = (float *)malloc(sizeof(float) * (size_t)I);
      ref_matmul(tok, up, 1, H, I, u);
      free(up);
      float *buf = f16_buffer_to_f32(xp->bu, (size_t)I);
      for (int i = 0; i < I; ++i) u[i] += buf[i];
      free(buf);
      for (int i = 0; i < I; ++i) g[i] = g[i] * u[i];
      float *dp = f16_buffer_to_f32(xp->down, (size_t)H * I);
      float *o = (float *)malloc(sizeof(float) * (size_t)H);
      ref_matmul(g, dp, 1, I, H, o);
      free(dp);
      float *bdf = f16_buffer_to_f32(xp->bd, (size_t)H);
      for (int c = 0; c < H; ++c) o[c] += bdf[c];
      free(bdf);
      /* buffer_from_f32(output) then buffer_to_f32_vec: f16 round trip */
      for (int c = 0; c < H; ++c) acc[c] += weight * oxo_f16_to_f32(oxo_f32_to_f16(o[c]));
      free(o); free(u); free(g); free(tok);
    }
  }
  for (size_t i = 0; i < (size_t)T * H; ++i) y_f16[i] = oxo_f32_to_f16(final_h[i]);
  free(final_h); free(idx); free(wts); free(xh);
  return 0;
}

int oxo_moe_forward_ref_faithful(const oxo_moe_weights *w, const uint16_t *x, int T,
                                 uint16_t *y_f16, int nthreads) {
  if (T == 0) return 0;
  oxo_ref_layer *L = oxo_ref_prepare(w, x, T);
  if (!L) return -1;
  int rc = oxo_ref_forward(L, x, T, y_f16, nthreads);
  oxo_ref_free(L);
  return rc;
}
