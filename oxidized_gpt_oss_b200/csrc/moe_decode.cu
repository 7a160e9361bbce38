// moe_decode.cu — MoE expert kernels for small token counts (decode):
// in-register MXFP4 dequantisation feeding warp-level f16 tensor-core MMAs.
//
// Reference computation (MLP::forward, src/model.rs:1088-1184, called per
// (token, expert) from src/moe.rs:81-93), with the gpt-oss layout and
// activation (mlp1 rows interleaved gate/up, clamped SwiGLU):
//   h1 = x . W1^T + b1          W1 [2I, H]; gate = even rows, up = odd rows
//   h  = swiglu(gate, up)       alpha, limit
//   y  = h . W2^T + b2          W2 [H, I]
//
// Design (HBM-bound: every expert weight byte is read once per step):
//  * Each CTA owns one expert (blockIdx.y) and a band of 16-row tiles; a warp
//    computes a 16-row x 8-token tile with mma.m16n8k16 (f16 in, f32 out).
//  * Weight codes stream from HBM with 16-byte loads in the word-transposed
//    order of relayout.cu, so one load gives a lane the A-operand codes of all
//    four blocks of a 128-element group. cvt.rn.f16x2.e2m1x2 turns two codes
//    into two exact f16 values; the E8M0 scale of each 32-element block is
//    applied to the f32 MMA result of that block (exact power of two).
//  * The per-lane K order inside a block is permuted consistently on A (by the
//    byte order of the code word) and B (by the shared-memory "fragment order"
//    of the activations), so no shuffles are needed.
//  * mlp1: A rows g and g+8 of a tile are the gate and up rows of one
//    intermediate unit, so a lane holds both and applies bias + clamped SwiGLU
//    in registers; the activation is staged once per CTA as f16 x * 2^-sigma
//    (exact for bf16 input) and the products are scaled back by 2^sigma.
//  * mlp2: the f32 SwiGLU output is split into f16 hi + lo (h = hi + lo to
//    ~2^-22 relative), and each block takes two MMAs per operand half, so the
//    intermediate is not rounded to 16 bits.
#include "common.cuh"
#include "kernels.h"

namespace oxg {
namespace {

constexpr int kWarps = 8;
constexpr int kThreads = kWarps * 32;
constexpr int kTilesPerWarp = 2;
constexpr int kTilesPerCta = kWarps * kTilesPerWarp;

struct DecodeArgs {
  const uint8_t *codes;   // relaid codes [E, rows, K/2]
  const uint8_t *scales;  // padded scales [E, rows, kb_pad]
  const uint16_t *bias;   // [E, rows] bf16
  int K, rows, kb_pad;
  // mlp1 input: x [T, K] bf16, token of position p = perm[p] / topk
  const uint16_t *x;
  const int32_t *perm;
  const int32_t *sigma;
  int topk;
  // mlp2 input: h [n_slots, K] f32 in position order
  const float *h;
  const int32_t *counts, *offsets;
  int expert_base;
  float *out;  // mlp1: h [n_slots, I]; mlp2: y_slot [n_slots, H]
  int out_ld;
  float alpha, limit;
};

// Byte offset of the 8-element group (n-tile nt, block blk, half s, token g,
// lane-in-quad q) in the fragment-ordered activation buffer.
__device__ __forceinline__ int frag_off(int nt, int nb, int blk, int s, int g, int q, int bytes) {
  return ((((nt * nb + blk) * 2 + s) * 8 + g) * 4 + q) * bytes;
}

template <int MODE, int NT>
__global__ void __launch_bounds__(kThreads) moe_decode_kernel(const DecodeArgs a) {
  extern __shared__ __align__(16) uint8_t smem[];
  __shared__ float tok_scale[NT * 8];

  const int e = a.expert_base + blockIdx.y;
  const int n_e = a.counts[e];
  if (n_e == 0) return;
  const int pos0 = a.offsets[e];
  const int K = a.K, nb = K / 32, ngroups_full = nb / 4, tail = nb % 4;
  const int n_tiles = a.rows / 16;
  const int tile0 = blockIdx.x * kTilesPerCta;
  if (tile0 >= n_tiles) return;

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int g = lane >> 2, q = lane & 3;
  const size_t rbase = (size_t)e * a.rows;
  const float zero4[4] = {0.f, 0.f, 0.f, 0.f};

  for (int tok0 = 0; tok0 < n_e; tok0 += NT * 8) {
    // ---- stage this pass's activations in fragment order ----
    const int units = NT * 8 * (K / 8);
    for (int u = tid; u < units; u += kThreads) {
      const int tok = u / (K / 8), k0 = (u % (K / 8)) * 8;
      const int nt = tok >> 3, gg = tok & 7, blk = k0 >> 5, qq = (k0 & 31) >> 3;
      const bool valid = tok0 + tok < n_e;
      if (MODE == 1) {
        uint32_t o0 = 0, o1 = 0, o2 = 0, o3 = 0;
        if (valid) {
          const int t = a.perm[pos0 + tok0 + tok] / a.topk;
          const float inv = __uint_as_float((uint32_t)(127 - a.sigma[t]) << 23);
          const uint4 v = *reinterpret_cast<const uint4 *>(a.x + (size_t)t * K + k0);
          o0 = pack_f16x2(bf16_to_f32(v.x & 0xFFFFu) * inv, bf16_to_f32(v.x >> 16) * inv);
          o1 = pack_f16x2(bf16_to_f32(v.y & 0xFFFFu) * inv, bf16_to_f32(v.y >> 16) * inv);
          o2 = pack_f16x2(bf16_to_f32(v.z & 0xFFFFu) * inv, bf16_to_f32(v.z >> 16) * inv);
          o3 = pack_f16x2(bf16_to_f32(v.w & 0xFFFFu) * inv, bf16_to_f32(v.w >> 16) * inv);
        }
        *reinterpret_cast<uint2 *>(smem + frag_off(nt, nb, blk, 0, gg, qq, 8)) = make_uint2(o0, o1);
        *reinterpret_cast<uint2 *>(smem + frag_off(nt, nb, blk, 1, gg, qq, 8)) = make_uint2(o2, o3);
      } else {
        float f[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
        if (valid) {
          const float4 *src = reinterpret_cast<const float4 *>(a.h + (size_t)(pos0 + tok0 + tok) * K + k0);
          const float4 v0 = src[0], v1 = src[1];
          f[0] = v0.x; f[1] = v0.y; f[2] = v0.z; f[3] = v0.w;
          f[4] = v1.x; f[5] = v1.y; f[6] = v1.z; f[7] = v1.w;
        }
#pragma unroll
        for (int s = 0; s < 2; ++s) {
          const uint32_t h01 = pack_f16x2(f[4 * s], f[4 * s + 1]);
          const uint32_t h23 = pack_f16x2(f[4 * s + 2], f[4 * s + 3]);
          const float2 r01 = unpack_f16x2(h01), r23 = unpack_f16x2(h23);
          const uint32_t l01 = pack_f16x2(f[4 * s] - r01.x, f[4 * s + 1] - r01.y);
          const uint32_t l23 = pack_f16x2(f[4 * s + 2] - r23.x, f[4 * s + 3] - r23.y);
          *reinterpret_cast<uint4 *>(smem + frag_off(nt, nb, blk, s, gg, qq, 16)) =
              make_uint4(h01, h23, l01, l23);
        }
      }
    }
    if (MODE == 1 && tid < NT * 8) {
      float sc = 1.f;
      if (tok0 + tid < n_e) {
        const int t = a.perm[pos0 + tok0 + tid] / a.topk;
        sc = __uint_as_float((uint32_t)(127 + a.sigma[t]) << 23);
      }
      tok_scale[tid] = sc;
    }
    __syncthreads();

    // ---- tiles ----
    for (int ti = 0; ti < kTilesPerWarp; ++ti) {
      const int tile = tile0 + warp * kTilesPerWarp + ti;
      if (tile >= n_tiles) break;
      const int row_a = MODE == 1 ? 2 * (tile * 8 + g) : tile * 16 + g;
      const int row_b = MODE == 1 ? row_a + 1 : row_a + 8;
      const uint8_t *ca = a.codes + (rbase + row_a) * (size_t)(K / 2);
      const uint8_t *cb = a.codes + (rbase + row_b) * (size_t)(K / 2);
      const uint8_t *sa = a.scales + (rbase + row_a) * (size_t)a.kb_pad;
      const uint8_t *sb = a.scales + (rbase + row_b) * (size_t)a.kb_pad;

      float acc[NT][4];
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) acc[nt][0] = acc[nt][1] = acc[nt][2] = acc[nt][3] = 0.f;

      auto block_step = [&](uint32_t wa, uint32_t wb, float s_a, float s_b, int blk) {
        uint32_t fa[4], fb[4];
        e2m1x8_to_f16x8(wa, fa);
        e2m1x8_to_f16x8(wb, fb);
        const uint32_t A0[4] = {fa[0], fb[0], fa[1], fb[1]};
        const uint32_t A1[4] = {fa[2], fb[2], fa[3], fb[3]};
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
          float d[4];
          if (MODE == 1) {
            const uint2 b0 = *reinterpret_cast<const uint2 *>(smem + frag_off(nt, nb, blk, 0, g, q, 8));
            const uint2 b1 = *reinterpret_cast<const uint2 *>(smem + frag_off(nt, nb, blk, 1, g, q, 8));
            mma_f16_16816(d, A0, b0.x, b0.y, zero4);
            mma_f16_16816(d, A1, b1.x, b1.y, d);
          } else {
            const uint4 b0 = *reinterpret_cast<const uint4 *>(smem + frag_off(nt, nb, blk, 0, g, q, 16));
            const uint4 b1 = *reinterpret_cast<const uint4 *>(smem + frag_off(nt, nb, blk, 1, g, q, 16));
            mma_f16_16816(d, A0, b0.x, b0.y, zero4);
            mma_f16_16816(d, A0, b0.z, b0.w, d);
            mma_f16_16816(d, A1, b1.x, b1.y, d);
            mma_f16_16816(d, A1, b1.z, b1.w, d);
          }
          acc[nt][0] = fmaf(s_a, d[0], acc[nt][0]);
          acc[nt][1] = fmaf(s_a, d[1], acc[nt][1]);
          acc[nt][2] = fmaf(s_b, d[2], acc[nt][2]);
          acc[nt][3] = fmaf(s_b, d[3], acc[nt][3]);
        }
      };

      // full groups, one group of loads kept in flight ahead of the math
      if (ngroups_full > 0) {
        uint4 va = ldg_stream_v4(ca + q * 16);
        uint4 vb = ldg_stream_v4(cb + q * 16);
        uint32_t xa = ldg_stream_u32(sa);
        uint32_t xb = ldg_stream_u32(sb);
#pragma unroll 1
        for (int grp = 0; grp < ngroups_full; ++grp) {
          uint4 na = va, nb4 = vb;
          uint32_t nxa = xa, nxb = xb;
          if (grp + 1 < ngroups_full) {
            na = ldg_stream_v4(ca + (grp + 1) * 64 + q * 16);
            nb4 = ldg_stream_v4(cb + (grp + 1) * 64 + q * 16);
            nxa = ldg_stream_u32(sa + (grp + 1) * 4);
            nxb = ldg_stream_u32(sb + (grp + 1) * 4);
          }
          const uint32_t wa[4] = {va.x, va.y, va.z, va.w};
          const uint32_t wb[4] = {vb.x, vb.y, vb.z, vb.w};
#pragma unroll
          for (int b = 0; b < 4; ++b)
            block_step(wa[b], wb[b], e8m0_to_f32(xa >> (8 * b)), e8m0_to_f32(xb >> (8 * b)),
                       grp * 4 + b);
          va = na;
          vb = nb4;
          xa = nxa;
          xb = nxb;
        }
      }
      if (tail) {
        const int grp = ngroups_full;
        const uint32_t xa = ldg_stream_u32(sa + grp * 4);
        const uint32_t xb = ldg_stream_u32(sb + grp * 4);
        for (int b = 0; b < tail; ++b) {
          const uint32_t wa = ldg_stream_u32(ca + grp * 64 + (q * tail + b) * 4);
          const uint32_t wb = ldg_stream_u32(cb + grp * 64 + (q * tail + b) * 4);
          block_step(wa, wb, e8m0_to_f32(xa >> (8 * b)), e8m0_to_f32(xb >> (8 * b)), grp * 4 + b);
        }
      }

      // ---- epilogue ----
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          const int col = nt * 8 + 2 * q + c;
          const int tok = tok0 + col;
          if (tok >= n_e) continue;
          const size_t pos = (size_t)(pos0 + tok);
          if (MODE == 1) {
            const int p = tile * 8 + g;
            const float sc = tok_scale[col];
            const float gate = fmaf(acc[nt][c], sc, bf16_to_f32(a.bias[rbase + row_a]));
            const float up = fmaf(acc[nt][2 + c], sc, bf16_to_f32(a.bias[rbase + row_b]));
            a.out[pos * a.out_ld + p] = swiglu_clamped(gate, up, a.alpha, a.limit);
          } else {
            a.out[pos * a.out_ld + row_a] = acc[nt][c] + bf16_to_f32(a.bias[rbase + row_a]);
            a.out[pos * a.out_ld + row_b] = acc[nt][2 + c] + bf16_to_f32(a.bias[rbase + row_b]);
          }
        }
      }
    }
    __syncthreads();
  }
}

__global__ void __launch_bounds__(256) combine_kernel(const float *__restrict__ y_slot,
                                                      const int32_t *__restrict__ slot_pos,
                                                      const float *__restrict__ wts, int T, int H,
                                                      int k, float *__restrict__ out) {
  const int h4 = H / 4;
  const size_t n = (size_t)T * h4;
  const size_t stride = (size_t)gridDim.x * blockDim.x;
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
    const int t = (int)(i / h4), c = (int)(i % h4);
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int j = 0; j < k; ++j) {
      const int p = slot_pos[t * k + j];
      if (p < 0) continue;
      const float w = wts[t * k + j];
      const float4 v = reinterpret_cast<const float4 *>(y_slot + (size_t)p * H)[c];
      acc.x = fmaf(w, v.x, acc.x);
      acc.y = fmaf(w, v.y, acc.y);
      acc.z = fmaf(w, v.z, acc.z);
      acc.w = fmaf(w, v.w, acc.w);
    }
    reinterpret_cast<float4 *>(out + (size_t)t * H)[c] = acc;
  }
}

template <int MODE, int NT>
cudaError_t launch_decode(const DecodeArgs &a, int n_local_experts, cudaStream_t stream) {
  const int nb = a.K / 32;
  const size_t smem = (size_t)NT * nb * 2 * 32 * (MODE == 1 ? 8 : 16);
  auto fn = moe_decode_kernel<MODE, NT>;
  if (smem > 48 * 1024) {
    cudaError_t st = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (st != cudaSuccess) return st;
  }
  const int n_tiles = a.rows / 16;
  dim3 grid((n_tiles + kTilesPerCta - 1) / kTilesPerCta, n_local_experts);
  fn<<<grid, kThreads, smem, stream>>>(a);
  return cudaGetLastError();
}

}  // namespace

// Shared memory of the activation stage, per token n-tile: nb * 2 * 32 * 8 (mlp1)
// or * 16 (mlp2) bytes. One n-tile (8 tokens) per pass keeps several CTAs
// resident per SM; larger groups of tokens take several passes.
cudaError_t launch_moe_mlp1_decode(const MoeDeviceWeights &w, const uint16_t *x,
                                   const int32_t *perm, const int32_t *sigma,
                                   const int32_t *counts, const int32_t *offsets, int n_slots,
                                   int expert_base, int n_local_experts, float *h,
                                   cudaStream_t stream) {
  if (n_slots == 0 || n_local_experts == 0) return cudaSuccess;
  DecodeArgs a{};
  a.codes = w.w1;
  a.scales = w.s1;
  a.bias = w.b1;
  a.K = w.H;
  a.rows = 2 * w.I;
  a.kb_pad = (w.H / 32 + 3) / 4 * 4;
  a.x = x;
  a.perm = perm;
  a.sigma = sigma;
  a.topk = w.k;
  a.counts = counts;
  a.offsets = offsets;
  a.expert_base = expert_base;
  a.out = h;
  a.out_ld = w.I;
  a.alpha = w.alpha;
  a.limit = w.limit;
  return launch_decode<1, 1>(a, n_local_experts, stream);
}

cudaError_t launch_moe_mlp2_decode(const MoeDeviceWeights &w, const float *h,
                                   const int32_t *counts, const int32_t *offsets, int n_slots,
                                   int expert_base, int n_local_experts, float *y_slot,
                                   cudaStream_t stream) {
  if (n_slots == 0 || n_local_experts == 0) return cudaSuccess;
  DecodeArgs a{};
  a.codes = w.w2;
  a.scales = w.s2;
  a.bias = w.b2;
  a.K = w.I;
  a.rows = w.H;
  a.kb_pad = (w.I / 32 + 3) / 4 * 4;
  a.h = h;
  a.topk = w.k;
  a.counts = counts;
  a.offsets = offsets;
  a.expert_base = expert_base;
  a.out = y_slot;
  a.out_ld = w.H;
  return launch_decode<2, 1>(a, n_local_experts, stream);
}

cudaError_t launch_combine(const float *y_slot, const int32_t *slot_pos, const float *wts, int T,
                           int H, int k, float *out, cudaStream_t stream) {
  if (T == 0) return cudaSuccess;
  const size_t n = (size_t)T * (H / 4);
  size_t want = (n + 255) / 256;
  unsigned grid = (unsigned)(want < 148 * 8 ? want : 148 * 8);
  combine_kernel<<<grid, 256, 0, stream>>>(y_slot, slot_pos, wts, T, H, k, out);
  return cudaGetLastError();
}

}  // namespace oxg
