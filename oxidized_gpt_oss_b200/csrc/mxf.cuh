// mxf.cuh — the block-scaled tensor-core path for MXFP4 weights on sm_100a.
//
// tcgen05.mma.kind::mxf8f6f4.block_scale multiplies E2M1 weights (the MXFP4
// codes exactly as stored, 16 per 8 bytes; TMA's 16U4_ALIGN16B type spreads
// them to 16 bytes per 16 codes in shared memory) by E4M3 activations, each
// operand with one UE8M0 scale per 32 elements of K, accumulating in f32 in
// TMEM. K = 32 per instruction.
//
// Activations are not 4-bit numbers, so they enter as a short sum of E4M3
// terms that share one exponent per 32-element block:
//   v = t1 * S + t2 * S / 32 + t3 * S / 1024 + t4 * S / 32768 (+ remainder)
// with S = 2^(e - 7) for the block's largest exponent e, so |v| / S < 256 and
// every term stays inside E4M3's range (the residual after a round-to-nearest
// E4M3 step is at most 8 units of that step's scale). Two terms carry 8
// significant bits (exact for bf16 x down to 2^-14 of the block maximum, and
// within 2^-21 of it below), three carry 12 and four 16 (the f32 SwiGLU
// output between the two GEMMs).
//
// Scale factors reach TMEM with tcgen05.cp 32x128b.warpx4 from a 512-byte
// atom in shared memory: 128 rows x 4 consecutive 32-element blocks, row r's
// block j at byte 16 * (r % 32) + 4 * (r / 32) + j. The MMA's sf_id (and the
// two top bits of the scale TMEM address) selects j.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "sm100.cuh"

namespace oxg {
namespace mxf {

using namespace sm100;

constexpr int kAtomBytes = 512;   // scale atom: 128 rows x 4 blocks
constexpr int kTileK = 128;       // K elements per pipeline step (4 MMAs)
constexpr int kTileM = 128;       // weight rows per MMA (cta_group::1)
constexpr int kATileBytes = kTileM * kTileK;  // 16 KB in shared memory (8 KB of codes)
constexpr int kATileTx = kTileM * kTileK / 2; // bytes the TMA moves for it

__host__ __device__ __forceinline__ int atom_offset(int r, int j) {
  return 16 * (r & 31) + 4 * ((r >> 5) & 3) + (j & 3);
}

// Instruction descriptor: A = E2M1, B = E4M3, UE8M0 scales, both K-major,
// f32 accumulation; a_sf / b_sf pick the 32-element block inside the atom.
__host__ __device__ constexpr uint32_t idesc_e2m1_e4m3(int m, int n, int a_sf, int b_sf) {
  return ((uint32_t)b_sf << 4) | (5u << 7) | (0u << 10) | ((uint32_t)(n >> 3) << 17) | (1u << 23) |
         ((uint32_t)(m >> 4) << 24) | ((uint32_t)a_sf << 29);
}

__device__ __forceinline__ void umma_mxf(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                         uint32_t idesc, uint32_t sfa_tmem, uint32_t sfb_tmem,
                                         uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::mxf8f6f4.block_scale [%0], %1, %2, %3, [%5], [%6], p;\n\t}" ::"r"(
          d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate), "r"(sfa_tmem), "r"(sfb_tmem)
      : "memory");
}

// Copies a 512-byte scale atom from shared memory into 4 TMEM columns of all
// four lane quarters. Ordered with the MMAs the same thread issues.
__device__ __forceinline__ void utccp_atom(uint32_t taddr, uint32_t atom_saddr) {
  uint64_t d = 0;
  d |= (uint64_t)((atom_saddr >> 4) & 0x3FFFu);  // start address, 16-byte units
  d |= (uint64_t)1 << 16;                        // leading byte offset: one 16-byte core row
  d |= (uint64_t)(128 >> 4) << 32;               // 8-row core matrices 128 B apart
  d |= (uint64_t)1 << 46;                        // descriptor version (sm_100)
  asm volatile("tcgen05.cp.cta_group::1.32x128b.warpx4 [%0], %1;" ::"r"(taddr), "l"(d) : "memory");
}

// 1-D bulk copy global -> shared, completion counted on an mbarrier. Both
// addresses 16-byte aligned, bytes a multiple of 16.
__device__ __forceinline__ void bulk_load(void *smem_dst, const void *gsrc, uint32_t bytes, uint64_t *bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_addr(smem_dst)),
      "l"(gsrc), "r"(bytes), "r"(smem_addr(bar))
      : "memory");
}

// ---- E4M3 terms ---------------------------------------------------------------
// Two f32 -> two E4M3 bytes (round to nearest even, saturating), lo in the
// low byte.
__device__ __forceinline__ uint32_t f32x2_to_e4m3x2(float lo, float hi) {
  uint16_t r;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(r) : "f"(hi), "f"(lo));
  return r;
}
// One E4M3 byte -> its exact value: the exponent and mantissa bits placed
// at the top of an f32 (a subnormal f32 for E4M3's subnormals) are the value
// times 2^-120.
__device__ __forceinline__ float e4m3_to_f32(uint32_t byte) {
  return __uint_as_float(((byte & 0x7Fu) << 20) | ((byte & 0x80u) << 24)) * 0x1p120f;
}

// Block scale byte (UE8M0) of the first term from the block's largest |v|
// given as f32 bits: 2^(e-7) with e its exponent, at least 16 so that the
// fourth term's scale (byte - 15) is a normal f32.
__device__ __forceinline__ int term_scale_byte(uint32_t absmax_bits) {
  const int e = (int)(absmax_bits >> 23);
  return (e < 23 ? 23 : e) - 7;
}
__device__ __forceinline__ float pow2_from_byte(int b) { return __uint_as_float((uint32_t)b << 23); }
__device__ __forceinline__ float inv_pow2_from_byte(int b) {
  return __uint_as_float((uint32_t)(254 - b) << 23);
}

// Splits a pair of values into NT E4M3 terms with scale bytes sb, sb-5, sb-10, sb-15.
// out[i] receives the two bytes of term i (lo first).
template <int NT>
__device__ __forceinline__ void split_terms2(float v0, float v1, int sb, uint32_t (&out)[NT]) {
#pragma unroll
  for (int i = 0; i < NT; ++i) {
    const int b = sb - 5 * i;
    const uint32_t q = f32x2_to_e4m3x2(v0 * inv_pow2_from_byte(b), v1 * inv_pow2_from_byte(b));
    out[i] = q;
    if (i + 1 < NT) {
      const float s = pow2_from_byte(b);
      v0 = fmaf(-e4m3_to_f32(q & 0xFFu), s, v0);
      v1 = fmaf(-e4m3_to_f32(q >> 8), s, v1);
    }
  }
}

}  // namespace mxf
}  // namespace oxg
