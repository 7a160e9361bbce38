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
// aligned.
__device__ __forceinline__ void stage_row_f16(const uint16_t *__restrict__ src,
                                              uint16_t *__restrict__ dst, int H, int sigma,
                                              int lane) {
  const float inv = __uint_as_float((uint32_t)(127 - sigma) << 23);
  const uint4 *s4 = reinterpret_cast<const uint4 *>(src);
  uint4 *d4 = reinterpret_cast<uint4 *>(dst);
  for (int c = lane; c < H / 8; c += 32) {
    const uint4 v = s4[c];
    uint4 o;
    o.x = pack_f16x2(bf16_to_f32(v.x & 0xFFFFu) * inv, bf16_to_f32(v.x >> 16) * inv);
    o.y = pack_f16x2(bf16_to_f32(v.y & 0xFFFFu) * inv, bf16_to_f32(v.y >> 16) * inv);
    o.z = pack_f16x2(bf16_to_f32(v.z & 0xFFFFu) * inv, bf16_to_f32(v.z >> 16) * inv);
    o.w = pack_f16x2(bf16_to_f32(v.w & 0xFFFFu) * inv, bf16_to_f32(v.w >> 16) * inv);
    d4[c] = o;
  }
}

}  // namespace oxg
