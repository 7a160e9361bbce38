// dequant.cu — MXFP4 -> bf16 dequantisation (HBM-bound streaming kernel).
//
// Semantics follow dequantize_mxfp4 of the reference (src/mxfp4.rs:15-54):
// element i of the flattened [rows, cols] tensor is nibble i of the packed
// codes (low nibble = even index), decoded with the OCP E2M1 table
// (src/mxfp4.rs:7-13), multiplied in f32 by the scale of its 32-element block
// (block index = i / 32, because cols % 32 == 0) and rounded to bf16 with the
// half crate's round-to-nearest-even. The f32 product of an E2M1 value (2
// significant bits) and a bf16 or E8M0 scale (<= 8 bits) is exact, so bf16
// rounding is the only rounding, as in the reference: results are bit-exact.
//
// Work unit: a quarter block (8 elements = 4 code bytes -> 16 output bytes).
// Each thread streams UNR quarters per iteration so that enough loads are in
// flight to cover HBM latency; stores use the streaming (.cs) hint because the
// output is never re-read by this kernel.
#include "common.cuh"
#include "kernels.h"

namespace oxg {
namespace {

template <int FMT>
__device__ __forceinline__ float load_scale(const void *scales, size_t blk) {
  if (FMT == 0) return e8m0_to_f32(__ldg(static_cast<const uint8_t *>(scales) + blk));
  return bf16_to_f32(__ldg(static_cast<const uint16_t *>(scales) + blk));
}

// e2m1(n) * s in f32 with the NaN results of an x86-64 host (the reference's
// f32 multiply there): a NaN scale propagates quieted with its sign and
// payload; inf * 0 gives the default NaN 0xFFC00000. The GPU multiply alone
// returns the canonical 0x7FFFFFFF for both. (An AArch64 host agrees on the
// first rule and returns 0x7FC00000 for the second.)
__device__ __forceinline__ float scaled_code(uint32_t n, float s) {
  const float v = __fmul_rn(e2m1_to_f32(n), s);
  if (__builtin_expect(v != v, 0)) {
    const uint32_t sb = __float_as_uint(s);
    return __uint_as_float(s != s ? (sb | 0x00400000u) : 0xFFC00000u);
  }
  return v;
}

__device__ __forceinline__ uint4 decode8(uint32_t w, float s) {
  uint32_t o[4];
#pragma unroll
  for (int p = 0; p < 4; ++p) {
    const float lo = scaled_code(w >> (8 * p), s);
    const float hi = scaled_code(w >> (8 * p + 4), s);
    o[p] = f32_to_bf16_bits(lo) | (f32_to_bf16_bits(hi) << 16);
  }
  return make_uint4(o[0], o[1], o[2], o[3]);
}

// Fast path for one 32-element block whose scale is finite (E8M0 bytes 0..254,
// bf16 scales with exponent field below 0xFF): each code byte becomes two
// exact f16 values (cvt.rn.f16x2.e2m1x2), then two exact f32 values, one f32
// multiply each (the reference's f32 multiply; a finite scale times an E2M1
// value is never NaN) and one round-to-nearest-even pack of the pair to bf16
// (cvt.rn.bf16x2.f32, subnormals kept) — the same bits as scaled_code +
// f32_to_bf16_bits. A non-finite scale takes the exact slow path (NaN rules).
__device__ __forceinline__ uint32_t bf16x2_of(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}
__device__ __forceinline__ uint4 decode8_fast(uint32_t w, float s) {
  uint32_t f[4], o[4];
  e2m1x8_to_f16x8(w, f);
#pragma unroll
  for (int p = 0; p < 4; ++p) {
    const float2 v = unpack_f16x2(f[p]);
    o[p] = bf16x2_of(__fmul_rn(v.x, s), __fmul_rn(v.y, s));
  }
  return make_uint4(o[0], o[1], o[2], o[3]);
}
template <int FMT>
__device__ __forceinline__ bool scale_finite(float s) {
  return (__float_as_uint(s) & 0x7F800000u) != 0x7F800000u;
}

template <int FMT, int UNR>
__global__ void __launch_bounds__(256) dequant_vec_kernel(const uint32_t *__restrict__ codes,
                                                          const void *__restrict__ scales,
                                                          uint4 *__restrict__ out, size_t n_q) {
  const size_t stride = (size_t)gridDim.x * blockDim.x;
  size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  for (; i + (UNR - 1) * stride < n_q; i += UNR * stride) {
    uint32_t w[UNR];
    float s[UNR];
#pragma unroll
    for (int u = 0; u < UNR; ++u) {
      w[u] = ldg_stream_u32(codes + i + u * stride);
      s[u] = load_scale<FMT>(scales, (i + u * stride) >> 2);
    }
#pragma unroll
    for (int u = 0; u < UNR; ++u)
      stg_stream_v4(out + i + u * stride,
                    __builtin_expect(scale_finite<FMT>(s[u]), 1) ? decode8_fast(w[u], s[u]) : decode8(w[u], s[u]));
  }
  for (; i < n_q; i += stride) {
    const uint32_t w = ldg_stream_u32(codes + i);
    const float s = load_scale<FMT>(scales, i >> 2);
    stg_stream_v4(out + i, scale_finite<FMT>(s) ? decode8_fast(w, s) : decode8(w, s));
  }
}

// Any alignment: one thread per element pair (one code byte).
template <int FMT>
__global__ void __launch_bounds__(256) dequant_byte_kernel(const uint8_t *__restrict__ codes,
                                                           const void *__restrict__ scales,
                                                           uint16_t *__restrict__ out,
                                                           size_t n_bytes) {
  const size_t stride = (size_t)gridDim.x * blockDim.x;
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n_bytes; i += stride) {
    uint32_t b = __ldg(codes + i);
    float s = load_scale<FMT>(scales, i >> 4);
    out[2 * i] = (uint16_t)f32_to_bf16_bits(scaled_code(b, s));
    out[2 * i + 1] = (uint16_t)f32_to_bf16_bits(scaled_code(b >> 4, s));
  }
}

int num_sms() {
  static int sms = 0;
  if (!sms) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (sms <= 0) sms = 148;
  }
  return sms;
}

}  // namespace

cudaError_t launch_dequant_mxfp4(const uint8_t *codes, const void *scales, int scale_fmt,
                                 size_t n_blocks, uint16_t *out, cudaStream_t stream) {
  if (n_blocks == 0) return cudaSuccess;
  const int threads = 256;
  const bool aligned = ((uintptr_t)codes % 4 == 0) && ((uintptr_t)out % 16 == 0);
  if (aligned) {
    const size_t n_q = n_blocks * 4;
    constexpr int UNR = 8;
    size_t want = (n_q + (size_t)threads * UNR - 1) / ((size_t)threads * UNR);
    size_t cap = (size_t)num_sms() * 8;  // 8 x 256 threads = a full SM
    unsigned grid = (unsigned)(want < cap ? (want ? want : 1) : cap);
    if (scale_fmt == 0)
      dequant_vec_kernel<0, UNR><<<grid, threads, 0, stream>>>(
          reinterpret_cast<const uint32_t *>(codes), scales, reinterpret_cast<uint4 *>(out), n_q);
    else
      dequant_vec_kernel<1, UNR><<<grid, threads, 0, stream>>>(
          reinterpret_cast<const uint32_t *>(codes), scales, reinterpret_cast<uint4 *>(out), n_q);
  } else {
    const size_t n_bytes = n_blocks * 16;
    size_t want = (n_bytes + threads - 1) / threads;
    size_t cap = (size_t)num_sms() * 8;
    unsigned grid = (unsigned)(want < cap ? want : cap);
    if (scale_fmt == 0)
      dequant_byte_kernel<0><<<grid, threads, 0, stream>>>(codes, scales, out, n_bytes);
    else
      dequant_byte_kernel<1><<<grid, threads, 0, stream>>>(codes, scales, out, n_bytes);
  }
  return cudaGetLastError();
}

}  // namespace oxg
