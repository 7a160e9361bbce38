// common.cuh — shared device helpers for the sm_100a MXFP4 MoE kernels.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace oxg {

// ----------------------------------------------------------------------------
// Scalar conversions. bf16 is carried as raw uint16 bits everywhere so that
// rounding is under our control.
// ----------------------------------------------------------------------------
__device__ __forceinline__ float bf16_to_f32(uint32_t b) { return __uint_as_float(b << 16); }

// f32 -> bf16 bits with the rounding of the reference's half 2.7.1
// bf16::from_f32: round to nearest, ties to even; NaN keeps sign and top
// payload bits and gets the quiet bit 0x0040.
__device__ __forceinline__ uint32_t f32_to_bf16_bits(float f) {
  uint32_t x = __float_as_uint(f);
  if ((x & 0x7FFFFFFFu) > 0x7F800000u) return (x >> 16) | 0x40u;
  return (x + 0x7FFFu + ((x >> 16) & 1u)) >> 16;
}

// E8M0 block scale -> f32, matching F8E8M0::to_f32 of the reference
// (src/dtype.rs:245-252): 0 -> 0.0, e -> 2^(e-127), 255 -> +inf.
__device__ __forceinline__ float e8m0_to_f32(uint32_t e) { return __uint_as_float((e & 0xFFu) << 23); }

// One E2M1 code (low 4 bits of n) -> exact f32. Bit pattern (m << 22) is the
// f32 with value e2m1(m) * 2^-126 (a subnormal for m < 2), so one exact
// multiply by 2^126 gives the E2M1 value; code 8 gives -0.0 (src/mxfp4.rs:9-13).
__device__ __forceinline__ float e2m1_to_f32(uint32_t n) {
  float v = __uint_as_float(((n & 7u) << 22) | ((n & 8u) << 28));
  return __fmul_rn(v, 0x1p126f);
}

// Two E2M1 codes in one byte -> f16x2 (low nibble in the low half), exact.
__device__ __forceinline__ uint32_t e2m1x2_to_f16x2(uint32_t byte) {
  uint32_t out;
  asm("{\n\t.reg .b8 b;\n\tcvt.u8.u32 b, %1;\n\tcvt.rn.f16x2.e2m1x2 %0, b;\n\t}"
      : "=r"(out)
      : "r"(byte));
  return out;
}

// Four bytes (8 codes) -> 4 x f16x2, element order preserved.
__device__ __forceinline__ void e2m1x8_to_f16x8(uint32_t w, uint32_t (&o)[4]) {
  asm("{\n\t.reg .b8 b0, b1, b2, b3;\n\t"
      "mov.b32 {b0, b1, b2, b3}, %4;\n\t"
      "cvt.rn.f16x2.e2m1x2 %0, b0;\n\t"
      "cvt.rn.f16x2.e2m1x2 %1, b1;\n\t"
      "cvt.rn.f16x2.e2m1x2 %2, b2;\n\t"
      "cvt.rn.f16x2.e2m1x2 %3, b3;\n\t}"
      : "=r"(o[0]), "=r"(o[1]), "=r"(o[2]), "=r"(o[3])
      : "r"(w));
}

// Clamped SwiGLU of gpt-oss: g <- min(g, limit); u <- clamp(u, -limit, limit);
// g * sigmoid(alpha * g) * (u + 1). Comparisons keep NaN, as torch.clamp does.
__device__ __forceinline__ float swiglu_clamped(float g, float u, float alpha, float limit) {
  g = g > limit ? limit : g;
  u = u < -limit ? -limit : (u > limit ? limit : u);
  const float sig = 1.0f / (1.0f + expf(-alpha * g));
  return g * sig * (u + 1.0f);
}
// The same function with the hardware exponential (__expf) and the
// approximate divide: a few ulp of error in the sigmoid for moderate
// arguments, growing to ~1e-5 relative only where the sigmoid is below 1e-30.
// For tensor-core epilogues, where the activation sits on the critical path.
__device__ __forceinline__ float swiglu_clamped_fast(float g, float u, float alpha, float limit) {
  g = g > limit ? limit : g;
  u = u < -limit ? -limit : (u > limit ? limit : u);
  const float sig = __fdividef(1.0f, 1.0f + __expf(-alpha * g));
  return g * sig * (u + 1.0f);
}

// ----------------------------------------------------------------------------
// Memory helpers
// ----------------------------------------------------------------------------
__device__ __forceinline__ uint4 ldg_stream_v4(const void *p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}
__device__ __forceinline__ uint32_t ldg_stream_u32(const void *p) {
  uint32_t r;
  asm volatile("ld.global.nc.L1::no_allocate.u32 %0, [%1];" : "=r"(r) : "l"(p));
  return r;
}
__device__ __forceinline__ void stg_stream_v4(void *p, uint4 v) {
  asm volatile("st.global.cs.v4.u32 [%0], {%1,%2,%3,%4};" ::"l"(p), "r"(v.x), "r"(v.y), "r"(v.z),
               "r"(v.w)
               : "memory");
}

// Asynchronous global -> shared copies (per thread; completion tracked per
// thread with commit/wait groups, no register staging).
__device__ __forceinline__ uint32_t smem_u32(const void *p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}
__device__ __forceinline__ void cp_async_16(void *smem, const void *gmem) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(smem)), "l"(gmem)
               : "memory");
}
__device__ __forceinline__ void cp_async_4(void *smem, const void *gmem) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_u32(smem)), "l"(gmem)
               : "memory");
}
// 16-byte copy reading src_bytes (0 or 16) bytes and zero-filling the rest.
__device__ __forceinline__ void cp_async_16_zfill(void *smem, const void *gmem, uint32_t src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(smem)), "l"(gmem),
               "r"(src_bytes)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// ----------------------------------------------------------------------------
// Warp MMA: D(16x8 f32) = A(16x16 f16, row) * B(16x8 f16, col) + C.
// ----------------------------------------------------------------------------
__device__ __forceinline__ void mma_f16_16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                              uint32_t b1, const float (&c)[4]) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%10,%11,%12,%13};"
      : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1), "f"(c[0]), "f"(c[1]),
        "f"(c[2]), "f"(c[3]));
}

// Same shape with bf16 operands.
__device__ __forceinline__ void mma_bf16_16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                               uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
// Four 8x8 b16 matrices from shared memory; lanes 8i..8i+7 give the row
// addresses of matrix i, register i receives it in the mma fragment layout.
__device__ __forceinline__ void ldmatrix_x4(uint32_t (&r)[4], const void *smem_row) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(smem_u32(smem_row)));
}

__device__ __forceinline__ uint32_t pack_f16x2(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}

__device__ __forceinline__ float2 unpack_f16x2(uint32_t v) {
  float2 r;
  asm("{\n\t.reg .f16 l, h;\n\tmov.b32 {l, h}, %2;\n\tcvt.f32.f16 %0, l;\n\tcvt.f32.f16 %1, h;\n\t}"
      : "=f"(r.x), "=f"(r.y)
      : "r"(v));
  return r;
}

// One bf16 activation row to f16 x * 2^-sigma (exact within the token's
// range, see router.cu) by one warp; H a multiple of 8, both rows 16-byte
// aligned. The lane's loads of up to 12 16-byte chunks (H <= 3072 in one
// pass) are all issued before the first conversion, so a row costs one
// memory round trip instead of one per chunk.
__device__ __forceinline__ void stage_row_f16(const uint16_t *__restrict__ src,
                                              uint16_t *__restrict__ dst, int H, int sigma,
                                              int lane) {
  constexpr int kPer = 12;
  const float inv = __uint_as_float((uint32_t)(127 - sigma) << 23);
  const uint4 *s4 = reinterpret_cast<const uint4 *>(src);
  uint4 *d4 = reinterpret_cast<uint4 *>(dst);
  const int nch = H / 8;
  for (int c0 = 0; c0 < nch; c0 += 32 * kPer) {
    uint4 v[kPer];
#pragma unroll
    for (int i = 0; i < kPer; ++i) {
      const int c = c0 + lane + 32 * i;
      v[i] = c < nch ? s4[c] : make_uint4(0u, 0u, 0u, 0u);
    }
#pragma unroll
    for (int i = 0; i < kPer; ++i) {
      const int c = c0 + lane + 32 * i;
      if (c < nch) {
        uint4 o;
        o.x = pack_f16x2(bf16_to_f32(v[i].x & 0xFFFFu) * inv, bf16_to_f32(v[i].x >> 16) * inv);
        o.y = pack_f16x2(bf16_to_f32(v[i].y & 0xFFFFu) * inv, bf16_to_f32(v[i].y >> 16) * inv);
        o.z = pack_f16x2(bf16_to_f32(v[i].z & 0xFFFFu) * inv, bf16_to_f32(v[i].z >> 16) * inv);
        o.w = pack_f16x2(bf16_to_f32(v[i].w & 0xFFFFu) * inv, bf16_to_f32(v[i].w >> 16) * inv);
        d4[c] = o;
      }
    }
  }
}

// Per expert e < E: the slots of e in router CTAs before CTA c (before_s[e])
// and in all n_cta CTAs (tot_s[e]), from the CTAs' histograms hist[cc, e].
// All THREADS threads of the block share the n_cta x E loads (independent
// loads, THREADS / E of them per expert) through part_s (2 x THREADS ints of
// shared memory); ends with the block synchronised.
template <int THREADS>
__device__ __forceinline__ void hist_prefix(const int32_t *__restrict__ hist, int n_cta, int E, int c,
                                            int *before_s, int *tot_s, int *part_s) {
  const int parts = THREADS / E;  // E <= THREADS
  const int tid = threadIdx.x;
  if (tid < parts * E) {
    const int e = tid % E, pt = tid / E;
    int tot = 0, before = 0;
#pragma unroll 4
    for (int cc = pt; cc < n_cta; cc += parts) {
      const int v = hist[(size_t)cc * E + e];
      tot += v;
      before += cc < c ? v : 0;
    }
    part_s[tid] = tot;
    part_s[THREADS + tid] = before;
  }
  __syncthreads();
  if (tid < E) {
    int tot = 0, before = 0;
    for (int pt = 0; pt < parts; ++pt) {
      tot += part_s[pt * E + tid];
      before += part_s[THREADS + pt * E + tid];
    }
    tot_s[tid] = tot;
    before_s[tid] = before;
  }
  __syncthreads();
}

// ----------------------------------------------------------------------------
// Top-k selection + softmax (MoELayer::forward, src/moe.rs:51-73, softmax_inplace
// src/utils.rs:91-111)
// ----------------------------------------------------------------------------
constexpr int kRankTopKMax = 16;  // k <= 16

// The k largest of the E <= 64 logits of one token (logit_s) in the order of
// a stable descending sort, by rank counting: the logit of expert e ranks
// #{e' : v' > v} + #{e' < e : v' == v} (a NaN logit counts as -inf). Lane l
// holds experts l and l + 32; the 64 comparisons per expert are independent,
// so the selection costs one pass of broadcasts instead of k rounds of
// dependent shuffle reductions. Lane 0 then forms the softmax over the k
// (max-subtracted, sum in j order, uniform if the sum is 0) exactly as
// select_topk_softmax does.
__device__ __forceinline__ void rank_topk_softmax(const float *logit_s, int E, int k, int lane,
                                                  int32_t *__restrict__ idx_out,
                                                  float *__restrict__ wts_out, int32_t *idx_smem,
                                                  float *top_v_s, int *top_e_s) {
  float v0 = lane < E ? logit_s[lane] : -INFINITY;
  float v1 = lane + 32 < E ? logit_s[lane + 32] : -INFINITY;
  if (v0 != v0) v0 = -INFINITY;
  if (v1 != v1) v1 = -INFINITY;
  int r0 = 0, r1 = 0;
#pragma unroll
  for (int l = 0; l < 32; ++l) {
    const float a = __shfl_sync(0xFFFFFFFFu, v0, l);   // expert l
    const float b = __shfl_sync(0xFFFFFFFFu, v1, l);   // expert l + 32
    r0 += (a > v0 || (a == v0 && l < lane)) ? 1 : 0;
    r0 += b > v0 ? 1 : 0;                               // l + 32 > lane: ties do not count
    r1 += (a > v1 || a == v1) ? 1 : 0;                  // l < lane + 32: ties count
    r1 += (b > v1 || (b == v1 && l < lane)) ? 1 : 0;
  }
  // experts beyond E (padding at -inf) rank after every real expert
  if (lane < E && r0 < k) {
    top_v_s[r0] = v0;
    top_e_s[r0] = lane;
  }
  if (lane + 32 < E && r1 < k) {
    top_v_s[r1] = v1;
    top_e_s[r1] = lane + 32;
  }
  __syncwarp();
  if (lane == 0) {
    float tv[kRankTopKMax];
    float mx = -INFINITY;
    for (int j = 0; j < k; ++j) {
      tv[j] = top_v_s[j];
      mx = fmaxf(mx, tv[j]);
    }
    float sum = 0.f;
    for (int j = 0; j < k; ++j) {
      tv[j] = expf(tv[j] - mx);
      sum += tv[j];
    }
    for (int j = 0; j < k; ++j) {
      const int e = top_e_s[j];
      idx_out[j] = e;
      wts_out[j] = sum == 0.f ? 1.0f / (float)k : tv[j] / sum;
      idx_smem[j] = e;
    }
  }
  __syncwarp();
}

}  // namespace oxg
