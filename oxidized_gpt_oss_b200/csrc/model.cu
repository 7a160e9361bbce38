// model.cu — the transformer around the MoE block (gpt-oss-20b architecture):
// token embedding + RMSNorm, bf16 linear layers on the tensor cores, RoPE and
// the KV cache, attention with a sliding window and learned sinks, the LM
// head and the greedy argmax. The MoE block itself is the library's MoE
// forward (moe_decode.cu / moe_prefill.cu).
//
// Reference behaviour followed (cipher-rc5/oxidized_gpt_oss):
//   * embedding gather: src/model.rs:749-798 (GPTModel::embed_tokens)
//   * RMS norm x * inv * gamma (+ beta): src/backend/metal_stub.rs:109-157
//   * q/k/v/o projections "A * B^T" + bias: src/model.rs:915-1071, src/utils.rs:34-89
//   * attention per head with GQA and a sliding window of `window` keys
//     (keys t+1-window .. t), scale 1/sqrt(head_dim): src/model.rs:1022-1057
//   * LM head on the last token: src/model.rs:800-844
//   * greedy argmax, ties to the LAST maximal index (Iterator::max_by):
//     src/sampler.rs:7-16
// Where the reference is incomplete (no RoPE, no sinks) the gpt-oss
// definitions apply: RoPE on the two halves of each head (x1 = d < 32,
// x2 = d >= 32) with angles pos * theta^(-2i/hd) from host-built tables;
// one learned sink logit per head that joins the softmax denominator only.
#include <cuda.h>
#include <cuda_runtime.h>

#include <math.h>

#include <algorithm>

#include <cooperative_groups.h>

#include "common.cuh"
#include "model.h"
#include "sm100.cuh"

namespace oxg {
namespace {

using namespace sm100;

// ---------------------------------------------------------------------------
// bf16 helpers local to this file
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}

__device__ __forceinline__ void ldmatrix_x2(uint32_t (&r)[2], const void *smem_row) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x2.shared.b16 {%0,%1}, [%2];"
               : "=r"(r[0]), "=r"(r[1])
               : "r"(smem_u32(smem_row)));
}

__device__ __forceinline__ void ldmatrix_x4_trans(uint32_t (&r)[4], const void *smem_row) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(smem_u32(smem_row)));
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// ---------------------------------------------------------------------------
// Embedding / residual update fused with the RMS norm. One CTA per row.
//   tokens != null: v = embed[tokens[t]] (a token id outside [0, V) sets
//                   *err = 60 and reads row 0), res[t] = v
//   add != null:    v = res[t] + (sum_s add[s][t] + bias), res[t] = v
//   otherwise:      v = res[t]
//   out[t] = bf16(v * (1 / sqrt(mean(v^2) + eps)) * gamma)
// ---------------------------------------------------------------------------
constexpr int kNormThreads = 512;
constexpr int kMaxSplits = 16;  // partial arrays a consumer sums (linear_splits caps at this)
constexpr int kNormClusterRows = 8;  // up to this many rows the norm runs as 8-CTA clusters

// 4 consecutive floats of row t: the residual (or embedding) plus the split
// partials and the bias; every load of an element is issued before the sums.
__device__ __forceinline__ float4 norm_value4(const float *__restrict__ r, const uint16_t *__restrict__ erow,
                                              const float *__restrict__ add, int S, size_t add_stride,
                                              size_t row_off, const uint16_t *__restrict__ add_bias, int i4) {
  if (erow) {
    const uint2 e = *reinterpret_cast<const uint2 *>(erow + 4 * i4);
    return make_float4(bf16_to_f32(e.x & 0xFFFFu), bf16_to_f32(e.x >> 16), bf16_to_f32(e.y & 0xFFFFu),
                       bf16_to_f32(e.y >> 16));
  }
  float4 v = reinterpret_cast<const float4 *>(r)[i4];
  if (add) {
    float4 a = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int s0 = 0; s0 < S; s0 += 8) {  // eight partials' loads in flight, summed in split order
      float4 p[8];
#pragma unroll
      for (int u = 0; u < 8; ++u)
        if (s0 + u < S) p[u] = reinterpret_cast<const float4 *>(add + (size_t)(s0 + u) * add_stride + row_off)[i4];
#pragma unroll
      for (int u = 0; u < 8; ++u)
        if (s0 + u < S) {
          a.x += p[u].x;
          a.y += p[u].y;
          a.z += p[u].z;
          a.w += p[u].w;
        }
    }
    if (add_bias) {
      const uint2 b = *reinterpret_cast<const uint2 *>(add_bias + 4 * i4);
      a.x += bf16_to_f32(b.x & 0xFFFFu);
      a.y += bf16_to_f32(b.x >> 16);
      a.z += bf16_to_f32(b.y & 0xFFFFu);
      a.w += bf16_to_f32(b.y >> 16);
    }
    v.x += a.x;
    v.y += a.y;
    v.z += a.z;
    v.w += a.w;
  }
  return v;
}

// The norm that feeds a MoE block lets the fused router (the only kernel of
// this file's successors launched as a programmatic dependent) start at once:
// it loads its read-only router rows, then waits for this kernel to complete
// before it reads anything this kernel writes. Launches without the
// programmatic attribute ignore the release.
__device__ __forceinline__ void release_router() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

__global__ void __launch_bounds__(kNormThreads)
    residual_norm_kernel(float *__restrict__ res, int H, const int32_t *__restrict__ tokens,
                         const uint16_t *__restrict__ embed, int V, const float *__restrict__ add, int S,
                         size_t add_stride, const uint16_t *__restrict__ add_bias,
                         const uint16_t *__restrict__ gamma, float eps, uint16_t *__restrict__ out,
                         int *__restrict__ err) {
  extern __shared__ float4 vs4[];
  __shared__ float red[kNormThreads / 32];
  release_router();
  const int t = blockIdx.x;
  float *r = res + (size_t)t * H;
  const uint16_t *erow = nullptr;
  if (tokens) {
    int tok = tokens[t];
    if (tok < 0 || tok >= V) {
      if (threadIdx.x == 0) atomicExch(err, 60);
      tok = 0;
    }
    erow = embed + (size_t)tok * H;
  }
  const bool write_res = erow || add;
  const int H4 = H >> 2;
  float ss = 0.f;
  for (int i4 = threadIdx.x; i4 < H4; i4 += kNormThreads) {
    const float4 v = norm_value4(r, erow, add, S, add_stride, (size_t)t * H, add_bias, i4);
    if (write_res) reinterpret_cast<float4 *>(r)[i4] = v;
    vs4[i4] = v;
    ss = fmaf(v.x, v.x, ss);
    ss = fmaf(v.y, v.y, ss);
    ss = fmaf(v.z, v.z, ss);
    ss = fmaf(v.w, v.w, ss);
  }
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  float tot = 0.f;
#pragma unroll
  for (int w = 0; w < kNormThreads / 32; ++w) tot += red[w];
  const float inv = 1.0f / sqrtf(tot / (float)H + eps);
  uint2 *o = reinterpret_cast<uint2 *>(out + (size_t)t * H);
  for (int i4 = threadIdx.x; i4 < H4; i4 += kNormThreads) {
    const float4 v = vs4[i4];
    const uint2 gm = *reinterpret_cast<const uint2 *>(gamma + 4 * i4);
    const uint32_t b0 = f32_to_bf16_bits(v.x * inv * bf16_to_f32(gm.x & 0xFFFFu));
    const uint32_t b1 = f32_to_bf16_bits(v.y * inv * bf16_to_f32(gm.x >> 16));
    const uint32_t b2 = f32_to_bf16_bits(v.z * inv * bf16_to_f32(gm.y & 0xFFFFu));
    const uint32_t b3 = f32_to_bf16_bits(v.w * inv * bf16_to_f32(gm.y >> 16));
    o[i4] = make_uint2(b0 | (b1 << 16), b2 | (b3 << 16));
  }
}

// The same for a few rows (decode): a cluster of kNormCl CTAs per row, each
// holding 1/kNormCl of the row, so every element's loads (residual, split
// partials, bias) are in flight at once across 8 SMs; the CTAs' partial sums
// of squares meet through distributed shared memory, added in rank order.
constexpr int kNormCl = 8;
constexpr int kNormClThreads = 128;

__global__ void __cluster_dims__(kNormCl, 1, 1) __launch_bounds__(kNormClThreads)
    residual_norm_cluster_kernel(float *__restrict__ res, int H, const int32_t *__restrict__ tokens,
                                 const uint16_t *__restrict__ embed, int V, const float *__restrict__ add, int S,
                                 size_t add_stride, const uint16_t *__restrict__ add_bias,
                                 const uint16_t *__restrict__ gamma, float eps, uint16_t *__restrict__ out,
                                 int *__restrict__ err) {
  namespace cg = cooperative_groups;
  cg::cluster_group cl = cg::this_cluster();
  extern __shared__ float4 vc4[];
  __shared__ float red[kNormClThreads / 32];
  __shared__ float part_ss;
  release_router();
  const int rank = (int)cl.block_rank();
  const int t = blockIdx.y;
  float *r = res + (size_t)t * H;
  const uint16_t *erow = nullptr;
  if (tokens) {
    int tok = tokens[t];
    if (tok < 0 || tok >= V) {
      if (threadIdx.x == 0 && rank == 0) atomicExch(err, 60);
      tok = 0;
    }
    erow = embed + (size_t)tok * H;
  }
  const bool write_res = erow || add;
  const int H4 = H >> 2, chunk = (H4 + kNormCl - 1) / kNormCl;
  const int i0 = rank * chunk, i1 = min(H4, i0 + chunk);
  float ss = 0.f;
  for (int i4 = i0 + threadIdx.x; i4 < i1; i4 += kNormClThreads) {
    const float4 v = norm_value4(r, erow, add, S, add_stride, (size_t)t * H, add_bias, i4);
    if (write_res) reinterpret_cast<float4 *>(r)[i4] = v;
    vc4[i4 - i0] = v;
    ss = fmaf(v.x, v.x, ss);
    ss = fmaf(v.y, v.y, ss);
    ss = fmaf(v.z, v.z, ss);
    ss = fmaf(v.w, v.w, ss);
  }
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  if (threadIdx.x == 0) {
    float p = 0.f;
#pragma unroll
    for (int w = 0; w < kNormClThreads / 32; ++w) p += red[w];
    part_ss = p;
  }
  cl.sync();
  float tot = 0.f;
#pragma unroll
  for (int q = 0; q < kNormCl; ++q) tot += *cl.map_shared_rank(&part_ss, q);
  const float inv = 1.0f / sqrtf(tot / (float)H + eps);
  uint2 *o = reinterpret_cast<uint2 *>(out + (size_t)t * H);
  for (int i4 = i0 + threadIdx.x; i4 < i1; i4 += kNormClThreads) {
    const float4 v = vc4[i4 - i0];
    const uint2 gm = *reinterpret_cast<const uint2 *>(gamma + 4 * i4);
    const uint32_t b0 = f32_to_bf16_bits(v.x * inv * bf16_to_f32(gm.x & 0xFFFFu));
    const uint32_t b1 = f32_to_bf16_bits(v.y * inv * bf16_to_f32(gm.x >> 16));
    const uint32_t b2 = f32_to_bf16_bits(v.z * inv * bf16_to_f32(gm.y & 0xFFFFu));
    const uint32_t b3 = f32_to_bf16_bits(v.w * inv * bf16_to_f32(gm.y >> 16));
    o[i4] = make_uint2(b0 | (b1 << 16), b2 | (b3 << 16));
  }
  cl.sync();  // no CTA leaves while another may still read its part_ss
}

// ---------------------------------------------------------------------------
// Linear layer: out[split][t][n] = sum_{k in split} x[t][k] * W[n][k]
// (bf16 operands, f32 accumulation, mma.sync m16n8k16). A CTA owns 64 weight
// rows (16 per warp) and NT tokens; the K range of its split streams through
// a cp.async ring of 64-wide stages (XOR-swizzled 16-byte chunks so every
// ldmatrix phase hits 32 distinct banks). Small batches split K across CTAs
// so that the weight stream covers every SM; the partial sums are added in
// split order by the consumer.
// ---------------------------------------------------------------------------
constexpr int kLinRows = 64;
constexpr int kLinK = 64;
constexpr int kLinThreads = 128;

template <int NT>
struct LinCfg {
  static constexpr int kStages = NT == 8 ? 8 : 4;
  static constexpr int kSmem = kStages * (kLinRows + NT) * kLinK * 2;
};

__device__ __forceinline__ int swz(int r, int c) { return r * 8 + (c ^ (r & 7)); }

// Orders (value, index) pairs as one 64-bit key: larger value wins, equal
// values go to the larger index (the reference's Iterator::max_by keeps the
// last maximum). 0 is below every key; NaN is never a candidate.
__device__ __forceinline__ unsigned long long argmax_key(float v, int i) {
  if (v != v) return 0ull;
  const uint32_t u = __float_as_uint(v);
  const uint32_t o = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
  return ((unsigned long long)o << 32) | (uint32_t)i;
}

template <int NT>
__global__ void __launch_bounds__(kLinThreads)
    linear_kernel(const uint16_t *__restrict__ x, int T, int ldx, const uint16_t *__restrict__ W, int N,
                  int K, int chunks_per_split, float *__restrict__ out, ArgmaxEpilogue am) {
  constexpr int ST = LinCfg<NT>::kStages;
  extern __shared__ __align__(128) uint8_t lin_smem[];
  uint4 *Ws = reinterpret_cast<uint4 *>(lin_smem);
  uint4 *Xs = Ws + ST * kLinRows * 8;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int row0 = blockIdx.x * kLinRows;
  const int t0 = blockIdx.y * NT;
  const int nck = K / kLinK;
  const int c_begin = blockIdx.z * chunks_per_split;
  const int n_local = min(nck, c_begin + chunks_per_split) - c_begin;

  auto load = [&](int slot, int c) {
    const int kofs = (c_begin + c) * kLinK;
    uint4 *ws = Ws + slot * kLinRows * 8;
#pragma unroll
    for (int i = 0; i < (kLinRows * 8) / kLinThreads; ++i) {
      const int id = tid + i * kLinThreads;
      const int r = id >> 3, ch = id & 7;
      const int gr = row0 + r;
      const bool ok = gr < N;
      cp_async_16_zfill(ws + swz(r, ch), W + (size_t)(ok ? gr : 0) * K + kofs + ch * 8, ok ? 16u : 0u);
    }
    uint4 *xs = Xs + slot * NT * 8;
    for (int id = tid; id < NT * 8; id += kLinThreads) {
      const int r = id >> 3, ch = id & 7;
      const int t = t0 + r;
      const bool ok = t < T;
      cp_async_16_zfill(xs + swz(r, ch), x + (size_t)(ok ? t : 0) * ldx + kofs + ch * 8, ok ? 16u : 0u);
    }
  };

  float acc[NT / 8][4];
#pragma unroll
  for (int j = 0; j < NT / 8; ++j) acc[j][0] = acc[j][1] = acc[j][2] = acc[j][3] = 0.f;

#pragma unroll
  for (int s = 0; s < ST - 1; ++s) {
    if (s < n_local) load(s, s);
    cp_async_commit();
  }
  for (int c = 0; c < n_local; ++c) {
    cp_async_wait<ST - 2>();
    __syncthreads();
    {
      const int nc = c + ST - 1;
      if (nc < n_local) load(nc % ST, nc);
      cp_async_commit();
    }
    const uint4 *ws = Ws + (c % ST) * kLinRows * 8;
    const uint4 *xs = Xs + (c % ST) * NT * 8;
#pragma unroll
    for (int ks = 0; ks < kLinK / 16; ++ks) {
      uint32_t a[4];
      {
        const int r = warp * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
        ldmatrix_x4(a, ws + swz(r, ks * 2 + (lane >> 4)));
      }
      if constexpr (NT == 8) {
        uint32_t b[2];
        ldmatrix_x2(b, xs + swz(lane & 7, ks * 2 + ((lane >> 3) & 1)));
        mma_bf16_16816(acc[0], a, b[0], b[1]);
      } else {
#pragma unroll
        for (int jp = 0; jp < NT / 16; ++jp) {
          uint32_t b[4];
          const int r = jp * 16 + (lane & 7) + (lane >> 4) * 8;
          ldmatrix_x4(b, xs + swz(r, ks * 2 + ((lane >> 3) & 1)));
          mma_bf16_16816(acc[2 * jp], a, b[0], b[1]);
          mma_bf16_16816(acc[2 * jp + 1], a, b[2], b[3]);
        }
      }
    }
  }
  cp_async_wait<0>();

  float *o = out + (size_t)blockIdx.z * T * N;
  const int g = lane >> 2, q = lane & 3;
  const int n_a = row0 + warp * 16 + g, n_b = n_a + 8;
#pragma unroll
  for (int j = 0; j < NT / 8; ++j) {
    const int ta = t0 + j * 8 + 2 * q, tb = ta + 1;
    if (ta < T) {
      if (n_a < N) o[(size_t)ta * N + n_a] = acc[j][0];
      if (n_b < N) o[(size_t)ta * N + n_b] = acc[j][2];
    }
    if (tb < T) {
      if (n_a < N) o[(size_t)tb * N + n_a] = acc[j][1];
      if (n_b < N) o[(size_t)tb * N + n_b] = acc[j][3];
    }
  }
  if constexpr (NT == 8) {
    if (am.keys) {
      // greedy choice per token: one 64-bit atomicMax per warp and token,
      // then the last CTA turns the keys into tokens (and resets them)
      __shared__ int am_last;
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        const int t = 2 * q + c;
        unsigned long long best = 0ull;
        if (n_a < N) best = argmax_key(acc[0][c], n_a);
        if (n_b < N) {
          const unsigned long long kb = argmax_key(acc[0][2 + c], n_b);
          best = kb > best ? kb : best;
        }
#pragma unroll
        for (int off = 4; off < 32; off <<= 1) {
          const unsigned long long ob = __shfl_xor_sync(0xffffffffu, best, off);
          best = ob > best ? ob : best;
        }
        if (g == 0 && t < T && best) atomicMax(am.keys + t, best);
      }
      __threadfence();
      __syncthreads();
      if (tid == 0)
        am_last = atomicAdd(am.count, 1u) == gridDim.x * gridDim.y * gridDim.z - 1;
      __syncthreads();
      if (am_last) {
        __threadfence();
        if (tid < T) {
          const unsigned long long key = atomicExch(am.keys + tid, 0ull);
          const int tok = key ? (int)(uint32_t)(key & 0xffffffffull) : 0;
          if (am.next) am.next[tid] = tok;
          if (am.state_mode == 1) {  // one-token decode step: feed back and advance
            am.out_seq[am.state[1]] = tok;
            am.state[2] = tok;
            am.state[0] += 1;
            am.state[1] += 1;
          } else if (am.state_mode == 2 && tid == T - 1) {
            am.state[0] = am.set_pos;
            am.state[1] = 0;
            am.state[2] = tok;
          }
        }
        if (tid == 0) *am.count = 0u;
      }
    }
  }
}

// ---------------------------------------------------------------------------
// q/k/v epilogue: sum of the split partials + bias, RoPE on q and k, bf16
// q rows and the K/V cache rows of positions pos0 .. pos0 + T - 1 of
// sequence seq, or, with tok_pos, token t at position tok_pos[t] of sequence
// tok_seq[t] (one token of each of T sequences); cache rows through the page
// table (kv_row). One CTA per token.
// ---------------------------------------------------------------------------
// Paged KV cache: a kv head's cache is a pool of pages of kKvPage rows;
// position pos of sequence seq lives in page pages[seq * max_pages + pos / 64]
// (the table the host fills as sequences grow), row pos % 64 of it.
constexpr int kKvPage = 64;
__device__ __forceinline__ long long kv_row(const int32_t *__restrict__ pages, int max_pages, int seq, int pos) {
  return (long long)__ldg(pages + (size_t)seq * max_pages + (pos >> 6)) * kKvPage + (pos & (kKvPage - 1));
}
// Splits of kKvPage keys (one page each) of the keys lo .. hi.
__host__ __device__ __forceinline__ int page_splits(int lo, int hi) { return (hi >> 6) - (lo >> 6) + 1; }

constexpr int kQkvThreads = 256;

__global__ void __launch_bounds__(kQkvThreads)
    qkv_post_kernel(const float *__restrict__ part, int S, int T, int nh, int nkv,
                    const uint16_t *__restrict__ bias, const float *__restrict__ rope_cos,
                    const float *__restrict__ rope_sin, int pos0, const int32_t *__restrict__ pos_dev,
                    const int32_t *__restrict__ tok_pos, const int32_t *__restrict__ tok_seq,
                    const int32_t *__restrict__ pages, int max_pages, int seq, int max_seq,
                    uint16_t *__restrict__ q_out, uint16_t *__restrict__ kc, uint16_t *__restrict__ vc) {
  const int t = blockIdx.x;
  const int Nq = nh * 64, Nkv = nkv * 64, N = Nq + 2 * Nkv;
  const int n_pairs = (nh + nkv) * 32;
  const int it = blockIdx.y * kQkvThreads + threadIdx.x;  // one RoPE pair or one v element
  if (it >= n_pairs + Nkv) return;
  const int pos = tok_pos ? tok_pos[t] : (pos_dev ? *pos_dev : pos0) + t;
  const long long row = kv_row(pages, max_pages, tok_pos ? tok_seq[t] : seq, pos);  // within a kv head's pool
  const float *pt = part + (size_t)t * N;
  const size_t ps = (size_t)T * N;
  if (it < n_pairs) {
    const int head = it >> 5, d = it & 31;
    const int n = head * 64 + d;  // q heads then k heads are contiguous in the fused rows
    float a1[kMaxSplits], a2[kMaxSplits];
#pragma unroll
    for (int s = 0; s < kMaxSplits; ++s)
      if (s < S) {
        a1[s] = pt[s * ps + n];
        a2[s] = pt[s * ps + n + 32];
      }
    float x1 = 0.f, x2 = 0.f;
#pragma unroll
    for (int s = 0; s < kMaxSplits; ++s)
      if (s < S) {
        x1 += a1[s];
        x2 += a2[s];
      }
    if (bias) {
      x1 += bf16_to_f32(bias[n]);
      x2 += bf16_to_f32(bias[n + 32]);
    }
    const float c = rope_cos[(size_t)pos * 32 + d], sn = rope_sin[(size_t)pos * 32 + d];
    const float o1 = x1 * c - x2 * sn;
    const float o2 = x2 * c + x1 * sn;
    uint16_t *dst = head < nh ? q_out + (size_t)t * Nq + head * 64
                              : kc + ((size_t)(head - nh) * max_seq + row) * 64;
    dst[d] = (uint16_t)f32_to_bf16_bits(o1);
    dst[d + 32] = (uint16_t)f32_to_bf16_bits(o2);
  } else {
    const int e = it - n_pairs;
    const int n = Nq + Nkv + e;
    float a[kMaxSplits];
#pragma unroll
    for (int s = 0; s < kMaxSplits; ++s)
      if (s < S) a[s] = pt[s * ps + n];
    float x = 0.f;
#pragma unroll
    for (int s = 0; s < kMaxSplits; ++s)
      if (s < S) x += a[s];
    if (bias) x += bf16_to_f32(bias[n]);
    vc[((size_t)(e >> 6) * max_seq + row) * 64 + (e & 63)] = (uint16_t)f32_to_bf16_bits(x);
  }
}

// ---------------------------------------------------------------------------
// Decode attention (one query token at position key_hi): CTA (kv head, split)
// handles the keys of [key_lo, key_hi] in one page of the cache (split sp:
// page key_lo / 64 + sp) for the G query heads sharing the kv head and
// writes (max, sum, unnormalised output) per head; the combine kernel merges
// the splits with the sink. With tok_pos, grid z runs over T tokens of T
// sequences: token t's keys are positions lo .. tok_pos[t] of sequence
// tok_seq[t], its q row t * Nq and its partials part_tok floats apart.
// ---------------------------------------------------------------------------
constexpr int kDecKeys = 64;
constexpr int kMaxGroup = 16;
constexpr int kDecThreads = 128;
constexpr int kKtPad = kDecKeys + 2;  // transposed-K row length (bf16 elements)

__global__ void __launch_bounds__(kDecThreads)
    attn_decode_kernel(const uint16_t *__restrict__ q, const uint16_t *__restrict__ kc,
                       const uint16_t *__restrict__ vc, int max_seq, int G, int key_lo, int key_hi,
                       float scale, int n_split, const int32_t *__restrict__ pos_dev, int window,
                       float *__restrict__ part, const int32_t *__restrict__ tok_pos,
                       const int32_t *__restrict__ tok_seq, const int32_t *__restrict__ pages, int max_pages,
                       int seq, int Nq, size_t part_tok) {
  __shared__ float qs[kMaxGroup][64];
  __shared__ __align__(16) uint16_t Kt[64][kKtPad];     // K transposed: [dim][key]
  __shared__ __align__(16) uint16_t Vs[kDecKeys][64];   // V as stored: [key][dim]
  __shared__ float ps[kMaxGroup][kDecKeys];
  __shared__ float ms[kMaxGroup], ls[kMaxGroup];
  const int kvh = blockIdx.x, sp = blockIdx.y;
  int sq = seq;
  if (pos_dev) {  // position from the device (graph replays): the grid covers the most splits
    key_hi = *pos_dev;
    key_lo = window > 0 ? max(0, key_hi - window + 1) : 0;
    n_split = page_splits(key_lo, key_hi);
    if (sp >= n_split) return;
  } else if (tok_pos) {  // one token per sequence: the grid covers the longest sequence
    const int t = blockIdx.z, p = tok_pos[t];
    const int lo = window > 0 ? max(0, p - window + 1) : 0;
    n_split = page_splits(lo, p);
    if (sp >= n_split) return;
    sq = tok_seq[t];
    key_lo = lo;
    key_hi = p;
    q += (size_t)t * Nq;
    part += (size_t)t * part_tok;
  }
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int kp = (key_lo >> 6) + sp;  // this split's page
  const int k0 = max(key_lo, kp * kKvPage);
  const int nk = min(key_hi, kp * kKvPage + kKvPage - 1) + 1 - k0;
  // stage q (pre-scaled), K transposed and V: every 16-byte load in flight at once
  for (int i = tid; i < G * 64; i += kDecThreads) qs[i >> 6][i & 63] = bf16_to_f32(q[(size_t)kvh * G * 64 + i]) * scale;
  const size_t base = ((size_t)kvh * max_seq + (size_t)kv_row(pages, max_pages, sq, k0)) * 64;  // nk rows of one page
#pragma unroll 4
  for (int c = tid; c < nk * 8; c += kDecThreads) {
    const int key = c >> 3, ch = c & 7;
    const uint4 kv = *reinterpret_cast<const uint4 *>(kc + base + (size_t)key * 64 + ch * 8);
    const uint4 vv = *reinterpret_cast<const uint4 *>(vc + base + (size_t)key * 64 + ch * 8);
    *reinterpret_cast<uint4 *>(&Vs[key][ch * 8]) = vv;
    const uint32_t w[4] = {kv.x, kv.y, kv.z, kv.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      Kt[ch * 8 + 2 * j][key] = (uint16_t)(w[j] & 0xFFFFu);
      Kt[ch * 8 + 2 * j + 1][key] = (uint16_t)(w[j] >> 16);
    }
  }
  __syncthreads();
  // scores: thread (key, head parity) for heads hp, hp + 2, ...
  {
    const int key = tid & (kDecKeys - 1), hp = tid >> 6;
    if (key < nk) {
      float acc[kMaxGroup / 2];
#pragma unroll
      for (int j = 0; j < kMaxGroup / 2; ++j) acc[j] = 0.f;
#pragma unroll 8
      for (int d = 0; d < 64; ++d) {
        const float kf = bf16_to_f32(Kt[d][key]);
#pragma unroll
        for (int j = 0; j < kMaxGroup / 2; ++j)
          if (hp + 2 * j < G) acc[j] = fmaf(qs[hp + 2 * j][d], kf, acc[j]);
      }
#pragma unroll
      for (int j = 0; j < kMaxGroup / 2; ++j)
        if (hp + 2 * j < G) ps[hp + 2 * j][key] = acc[j];
    }
  }
  __syncthreads();
  for (int h = warp; h < G; h += kDecThreads / 32) {
    const float s0 = lane < nk ? ps[h][lane] : -INFINITY;
    const float s1 = lane + 32 < nk ? ps[h][lane + 32] : -INFINITY;
    const float m = warp_max(fmaxf(s0, s1));
    const float p0 = lane < nk ? expf(s0 - m) : 0.f;
    const float p1 = lane + 32 < nk ? expf(s1 - m) : 0.f;
    if (lane < nk) ps[h][lane] = p0;
    if (lane + 32 < nk) ps[h][lane + 32] = p1;
    const float l = warp_sum(p0 + p1);
    if (lane == 0) {
      ms[h] = m;
      ls[h] = l;
    }
  }
  __syncthreads();
  // output: thread (head, 4 dims) accumulates the weighted V rows from shared memory
  float *dst = part + ((size_t)kvh * n_split + sp) * G * 66;
  for (int o = tid; o < G * 16; o += kDecThreads) {
    const int h = o >> 4, d0 = (o & 15) * 4;
    float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
#pragma unroll 4
    for (int j = 0; j < nk; ++j) {
      const float p = ps[h][j];
      const uint2 v = *reinterpret_cast<const uint2 *>(&Vs[j][d0]);
      a0 = fmaf(p, bf16_to_f32(v.x & 0xFFFFu), a0);
      a1 = fmaf(p, bf16_to_f32(v.x >> 16), a1);
      a2 = fmaf(p, bf16_to_f32(v.y & 0xFFFFu), a2);
      a3 = fmaf(p, bf16_to_f32(v.y >> 16), a3);
    }
    float *ph = dst + h * 66;
    ph[2 + d0] = a0;
    ph[3 + d0] = a1;
    ph[4 + d0] = a2;
    ph[5 + d0] = a3;
    if (d0 == 0) {
      ph[0] = ms[h];
      ph[1] = ls[h];
    }
  }
}

// ---------------------------------------------------------------------------
// Batched decode attention on the tensor cores: one query token of each of T
// sequences, G = 8 query heads per kv head. A work item is (token, kv head,
// split of kAdKeys keys); every warp streams its own items (item ids gw,
// gw + W, ... over the grid's W warps) through a ring of kAdStages K + V
// tiles of 64 keys, which its lane 0 loads by TMA from the KV cache's tensor
// map (128-byte swizzle, so the ldmatrix phases hit distinct banks) while the
// warp computes the previous tiles:
//   S^T (64 keys x 8 heads) = K Q^T    mma m16n8k16, keys as M, heads as N
//   online softmax per head (a column), P^T moved into the B-operand layout
//   with movmatrix, as a bf16 hi + lo pair (~16 significant bits, like the
//   prefill kernel)
//   O^T (64 dims x 8 heads) += V^T P^T
// Each item's per-head (max, sum, unnormalised output) go to the partials
// the combine kernel merges with kAdKeys keys per split. Keys past the
// item's end are masked in S, and their V rows zeroed in shared memory (the
// cache rows there may hold anything). Every wait is bounded: a timeout
// records code 61 in *err and the warp drains its loads and stops.
// ---------------------------------------------------------------------------
constexpr int kAdWarps = 4;
constexpr int kAdStages = 3;
constexpr int kAdTile = 64;
constexpr int kAdKeys = 4 * kAdTile;
constexpr uint32_t kAdTileBytes = kAdTile * 128;  // one K or V tile: 64 rows of 64 bf16
constexpr size_t kAdSmem = (size_t)kAdWarps * kAdStages * 2 * kAdTileBytes + 1024;

__device__ __forceinline__ uint32_t movmatrix_trans(uint32_t a) {
  uint32_t d;
  asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(d) : "r"(a));
  return d;
}

struct AdItem {
  int t, kvh, sp, n_split;
  int pg0, n_pages;  // the item's cache pages (tiles) of sequence t: pg0 .. pg0 + n_pages - 1
  int lo, hi;        // its token's keys
};
constexpr int kAdPages = kAdKeys / 64;  // pages per item

// Item idx = (t * max_split + sp) * nkv + kvh; false past sequence t's splits.
// Split sp covers pages lo / 64 + kAdPages sp .. (at most kAdPages of them).
__device__ __forceinline__ bool ad_item(int idx, int nkv, int max_split, const int32_t *tok_pos, int window,
                                        AdItem &it) {
  it.kvh = idx % nkv;
  const int r = idx / nkv;
  it.sp = r % max_split;
  it.t = r / max_split;
  const int p = tok_pos[it.t];
  const int lo = window > 0 ? max(0, p - window + 1) : 0;
  const int pages = page_splits(lo, p);
  it.n_split = (pages + kAdPages - 1) / kAdPages;
  if (it.sp >= it.n_split) return false;
  it.pg0 = (lo >> 6) + it.sp * kAdPages;
  it.n_pages = min(kAdPages, (p >> 6) - it.pg0 + 1);
  it.lo = lo;
  it.hi = p;
  return true;
}

struct AdCursor {
  int idx, tile, n_tiles;
  AdItem it;
};

// Moves c to the first tile of the next item at or after c.idx (stride W).
__device__ __forceinline__ bool ad_seek(AdCursor &c, int W, int n_items, int nkv, int max_split,
                                        const int32_t *tok_pos, int window) {
  for (; c.idx < n_items; c.idx += W)
    if (ad_item(c.idx, nkv, max_split, tok_pos, window, c.it)) {
      c.tile = 0;
      c.n_tiles = c.it.n_pages;
      return true;
    }
  return false;
}

// One warp merges the n_split partials (max, sum, unnormalised output) of
// the 8 query heads h0 .. h0 + 7 and their sinks into the bf16 output row:
// lane = (head lane / 4, 16 dims). Same arithmetic, in the same order, as
// attn_combine_kernel: the running max from the sink over the splits in
// order, then L and the outputs accumulated over the splits in order.
__device__ __forceinline__ void merge_splits(const float *p0, int n_split, int h0, const uint16_t *sinks,
                                             uint16_t *out_row, int lane) {
  const int h = lane >> 2, dq = lane & 3;
  const float *ph = p0 + h * 66;
  const size_t stride = (size_t)8 * 66;
  const float sink = sinks ? bf16_to_f32(sinks[h0 + h]) : -INFINITY;
  float M = sink;
#pragma unroll 8
  for (int s = 0; s < n_split; ++s) M = fmaxf(M, __ldcg(ph + s * stride));
  float L = sinks ? expf(sink - M) : 0.f;
  float acc[16];
#pragma unroll
  for (int j = 0; j < 16; ++j) acc[j] = 0.f;
#pragma unroll 4
  for (int s = 0; s < n_split; ++s) {
    const float *p = ph + s * stride;
    const float2 ml = __ldcg(reinterpret_cast<const float2 *>(p));
    float2 v[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) v[j] = __ldcg(reinterpret_cast<const float2 *>(p + 2 + dq * 16) + j);
    const float f = expf(ml.x - M);
    L = fmaf(ml.y, f, L);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      acc[2 * j] = fmaf(v[j].x, f, acc[2 * j]);
      acc[2 * j + 1] = fmaf(v[j].y, f, acc[2 * j + 1]);
    }
  }
  uint32_t w[8];
#pragma unroll
  for (int j = 0; j < 8; ++j)
    w[j] = f32_to_bf16_bits(acc[2 * j] / L) | (f32_to_bf16_bits(acc[2 * j + 1] / L) << 16);
  uint4 *o = reinterpret_cast<uint4 *>(out_row + (size_t)(h0 + h) * 64 + dq * 16);
  o[0] = make_uint4(w[0], w[1], w[2], w[3]);
  o[1] = make_uint4(w[4], w[5], w[6], w[7]);
}

__global__ void __launch_bounds__(kAdWarps * 32, 1)
    attn_decode_mma_kernel(const __grid_constant__ CUtensorMap kv_map, const uint16_t *__restrict__ q,
                           const int32_t *__restrict__ tok_pos, const int32_t *__restrict__ tok_seq,
                           const int32_t *__restrict__ pages, int max_pages,
                           long long k_row, long long v_row, long long kv_stride, int nkv, int Nq, int window,
                           float scale, int max_split, int n_items, float *__restrict__ part, size_t part_tok,
                           int *err, unsigned *__restrict__ merge_cnt, const uint16_t *__restrict__ sinks,
                           uint16_t *__restrict__ out) {
  extern __shared__ __align__(16) uint8_t ad_raw[];
  __shared__ __align__(8) uint64_t bars[kAdWarps][kAdStages];
  uint8_t *smem = ad_raw + ((1024 - (smem_addr(ad_raw) & 1023)) & 1023);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, qd = lane & 3;
  uint8_t *ring = smem + (size_t)warp * kAdStages * 2 * kAdTileBytes;
  uint64_t *bar = bars[warp];
  if (lane == 0) {
    for (int s = 0; s < kAdStages; ++s) mbar_init(&bar[s], 1);
    fence_mbar_init();
    prefetch_tmap(&kv_map);
  }
  __syncwarp();
  const int W = gridDim.x * kAdWarps, gw = blockIdx.x * kAdWarps + warp;

  // producer: lane 0 issues the K and V tiles at the producer cursor
  AdCursor pc;
  pc.idx = gw;
  bool p_ok = ad_seek(pc, W, n_items, nkv, max_split, tok_pos, window);
  int issued = 0;
  auto issue = [&]() {
    const int s = issued % kAdStages;
    if (lane == 0) {
      // tile = one whole cache page (64 rows)
      const long long r = (long long)pc.it.kvh * kv_stride +
                          kv_row(pages, max_pages, tok_seq[pc.it.t], (pc.it.pg0 + pc.tile) * kAdTile);
      uint8_t *ks = ring + (size_t)s * 2 * kAdTileBytes;
      mbar_arrive_expect_tx(&bar[s], 2 * kAdTileBytes);
      tma_load_2d(ks, &kv_map, &bar[s], 0, (int)(k_row + r));
      tma_load_2d(ks + kAdTileBytes, &kv_map, &bar[s], 0, (int)(v_row + r));
    }
    ++issued;
    if (++pc.tile == pc.n_tiles) {
      pc.idx += W;
      p_ok = ad_seek(pc, W, n_items, nkv, max_split, tok_pos, window);
    }
  };
  for (int i = 0; i < kAdStages && p_ok; ++i) issue();

  AdCursor cc;
  cc.idx = gw;
  bool c_ok = ad_seek(cc, W, n_items, nkv, max_split, tok_pos, window);
  int consumed = 0;
  bool failed = false;
  while (c_ok && !failed) {
    const AdItem it = cc.it;
    // Q^T as B operands: head g of the group, dims db * 16 + 2qd (+1) and + 8
    const uint16_t *qh = q + (size_t)it.t * Nq + (size_t)(it.kvh * 8 + g) * 64 + 2 * qd;
    uint32_t qf[4][2];
#pragma unroll
    for (int db = 0; db < 4; ++db) {
      qf[db][0] = *reinterpret_cast<const uint32_t *>(qh + db * 16);
      qf[db][1] = *reinterpret_cast<const uint32_t *>(qh + db * 16 + 8);
    }
    float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;  // heads 2qd, 2qd + 1
    float o[4][4];
#pragma unroll
    for (int mb = 0; mb < 4; ++mb) o[mb][0] = o[mb][1] = o[mb][2] = o[mb][3] = 0.f;

    for (; cc.tile < cc.n_tiles; ++cc.tile) {
      const int s = consumed % kAdStages;
      if (!mbar_wait(&bar[s], (uint32_t)(consumed / kAdStages) & 1u, err, 61)) {
        failed = true;
        break;
      }
      uint8_t *ks = ring + (size_t)s * 2 * kAdTileBytes;
      uint8_t *vs = ks + kAdTileBytes;
      // valid keys of this page: rows kf .. nkt - 1 (keys before the window
      // start are masked; their V rows hold earlier positions of the sequence)
      const int pbase = (it.pg0 + cc.tile) * kAdTile;
      const int kf = max(0, it.lo - pbase);
      const int nkt = min(kAdTile, it.hi + 1 - pbase);
      if (nkt < kAdTile) {  // zero the V rows past the end (whole 128-byte rows)
        for (int c = nkt * 8 + lane; c < kAdTile * 8; c += 32)
          *reinterpret_cast<uint4 *>(vs + c * 16) = make_uint4(0u, 0u, 0u, 0u);
        __syncwarp();
      }
      // S^T = K Q^T per block of 16 keys
      float sc[4][4];
#pragma unroll
      for (int kb = 0; kb < 4; ++kb) {
        sc[kb][0] = sc[kb][1] = sc[kb][2] = sc[kb][3] = 0.f;
#pragma unroll
        for (int db = 0; db < 4; ++db) {
          const int row = kb * 16 + (lane & 15), ch = db * 2 + (lane >> 4);
          uint32_t a[4];
          ldmatrix_x4(a, ks + row * 128 + ((ch ^ (row & 7)) << 4));
          mma_bf16_16816(sc[kb], a, qf[db][0], qf[db][1]);
        }
      }
      // scale, mask, running max per head
      float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
      for (int kb = 0; kb < 4; ++kb) {
        const int ka = kb * 16 + g, kb8 = ka + 8;
        const bool oka = ka >= kf && ka < nkt, okb = kb8 >= kf && kb8 < nkt;
        sc[kb][0] = oka ? sc[kb][0] * scale : -INFINITY;
        sc[kb][1] = oka ? sc[kb][1] * scale : -INFINITY;
        sc[kb][2] = okb ? sc[kb][2] * scale : -INFINITY;
        sc[kb][3] = okb ? sc[kb][3] * scale : -INFINITY;
        mx0 = fmaxf(mx0, fmaxf(sc[kb][0], sc[kb][2]));
        mx1 = fmaxf(mx1, fmaxf(sc[kb][1], sc[kb][3]));
      }
#pragma unroll
      for (int off = 4; off < 32; off <<= 1) {
        mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, off));
        mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, off));
      }
      const float mn0 = fmaxf(m0, mx0), mn1 = fmaxf(m1, mx1);  // finite: the tile has a key
      const float al0 = expf(m0 - mn0), al1 = expf(m1 - mn1);
      m0 = mn0;
      m1 = mn1;
      float rs0 = 0.f, rs1 = 0.f;
#pragma unroll
      for (int kb = 0; kb < 4; ++kb) {
        sc[kb][0] = expf(sc[kb][0] - mn0);
        sc[kb][1] = expf(sc[kb][1] - mn1);
        sc[kb][2] = expf(sc[kb][2] - mn0);
        sc[kb][3] = expf(sc[kb][3] - mn1);
        rs0 += sc[kb][0] + sc[kb][2];
        rs1 += sc[kb][1] + sc[kb][3];
      }
      l0 = l0 * al0 + rs0;
      l1 = l1 * al1 + rs1;
#pragma unroll
      for (int mb = 0; mb < 4; ++mb) {
        o[mb][0] *= al0;
        o[mb][1] *= al1;
        o[mb][2] *= al0;
        o[mb][3] *= al1;
      }
      // O^T += V^T P^T per block of 16 keys
#pragma unroll
      for (int kb = 0; kb < 4; ++kb) {
        const uint32_t x0 = pack_bf16x2(sc[kb][0], sc[kb][1]);  // key g: heads 2qd, 2qd + 1
        const uint32_t x1 = pack_bf16x2(sc[kb][2], sc[kb][3]);  // key g + 8
        const uint32_t y0 = pack_bf16x2(sc[kb][0] - __uint_as_float(x0 << 16),
                                        sc[kb][1] - __uint_as_float(x0 & 0xFFFF0000u));
        const uint32_t y1 = pack_bf16x2(sc[kb][2] - __uint_as_float(x1 << 16),
                                        sc[kb][3] - __uint_as_float(x1 & 0xFFFF0000u));
        const uint32_t b0h = movmatrix_trans(x0), b1h = movmatrix_trans(x1);  // head g: keys 2qd.., 2qd + 8..
        const uint32_t b0l = movmatrix_trans(y0), b1l = movmatrix_trans(y1);
#pragma unroll
        for (int mb = 0; mb < 4; ++mb) {
          const int key = kb * 16 + (lane & 7) + ((lane >> 4) << 3), ch = mb * 2 + ((lane >> 3) & 1);
          uint32_t a[4];
          ldmatrix_x4_trans(a, vs + key * 128 + ((ch ^ (key & 7)) << 4));
          mma_bf16_16816(o[mb], a, b0h, b1h);
          mma_bf16_16816(o[mb], a, b0l, b1l);
        }
      }
      // every lane is done with the stage (and its zeroed V rows are ordered
      // before the next TMA write into it)
      if (nkt < kAdTile) fence_proxy_async_smem();
      __syncwarp();
      ++consumed;
      if (p_ok) issue();
    }
    if (failed) break;
    // the item's partials: sums over the quad columns' eight key rows
#pragma unroll
    for (int off = 4; off < 32; off <<= 1) {
      l0 += __shfl_xor_sync(0xffffffffu, l0, off);
      l1 += __shfl_xor_sync(0xffffffffu, l1, off);
    }
    float *dst = part + (size_t)it.t * part_tok + (size_t)(it.kvh * it.n_split + it.sp) * 8 * 66;
    float *d0 = dst + (2 * qd) * 66, *d1 = d0 + 66;
#pragma unroll
    for (int mb = 0; mb < 4; ++mb) {
      d0[2 + mb * 16 + g] = o[mb][0];
      d1[2 + mb * 16 + g] = o[mb][1];
      d0[2 + mb * 16 + g + 8] = o[mb][2];
      d1[2 + mb * 16 + g + 8] = o[mb][3];
    }
    if (g == 0) {
      d0[0] = m0;
      d0[1] = l0;
      d1[0] = m1;
      d1[1] = l1;
    }
    // with merge_cnt: the last split of (token, kv head) to get here merges
    // them all (else attn_combine_kernel does)
    unsigned prev = 0u;
    if (merge_cnt) {
      __threadfence();
      __syncwarp();
      if (lane == 0) prev = atomicAdd(&merge_cnt[it.t * nkv + it.kvh], 1u);
    }
    if (merge_cnt && __shfl_sync(0xffffffffu, prev, 0) == (unsigned)it.n_split - 1u) {
      __threadfence();
      if (lane == 0) merge_cnt[it.t * nkv + it.kvh] = 0u;  // zero again for the next launch
      merge_splits(part + (size_t)it.t * part_tok + (size_t)it.kvh * it.n_split * 8 * 66, it.n_split,
                   it.kvh * 8, sinks, out + (size_t)it.t * Nq, lane);
    }
    cc.idx += W;
    c_ok = ad_seek(cc, W, n_items, nkv, max_split, tok_pos, window);
  }
  // after a timeout: the loads still in flight land before the CTA exits
  for (; consumed < issued; ++consumed)
    if (!mbar_wait(&bar[consumed % kAdStages], (uint32_t)(consumed / kAdStages) & 1u, err, 61)) break;
}

// One CTA of 64 threads per (query head, token): merges the decode splits and
// the sink.
__global__ void __launch_bounds__(64)
    attn_combine_kernel(const float *__restrict__ part, int G, int n_split, const int32_t *__restrict__ pos_dev,
                        int window, const uint16_t *__restrict__ sinks, uint16_t *__restrict__ out,
                        const int32_t *__restrict__ tok_pos, int Nq, size_t part_tok, int keys_per_split) {
  const int h = blockIdx.x, kvh = h / G, hl = h % G, d = threadIdx.x;
  if (pos_dev || tok_pos) {
    const int t = blockIdx.y;
    const int hi = tok_pos ? tok_pos[t] : *pos_dev, lo = window > 0 ? max(0, hi - window + 1) : 0;
    // splits of keys_per_split / 64 cache pages, from the page holding lo
    n_split = (page_splits(lo, hi) - 1) / (keys_per_split / kKvPage) + 1;
    if (tok_pos) {
      part += (size_t)t * part_tok;
      out += (size_t)t * Nq;
    }
  }
  const float sink = sinks ? bf16_to_f32(sinks[h]) : -INFINITY;
  const float *p0 = part + ((size_t)kvh * n_split * G + hl) * 66;
  const size_t stride = (size_t)G * 66;
  float M = sink;
#pragma unroll 8
  for (int s = 0; s < n_split; ++s) M = fmaxf(M, p0[s * stride]);
  float L = sinks ? expf(sink - M) : 0.f, acc = 0.f;
#pragma unroll 8
  for (int s = 0; s < n_split; ++s) {
    const float *p = p0 + s * stride;
    const float f = expf(p[0] - M);
    L = fmaf(p[1], f, L);
    acc = fmaf(p[2 + d], f, acc);
  }
  out[h * 64 + d] = (uint16_t)f32_to_bf16_bits(acc / L);
}

// ---------------------------------------------------------------------------
// Prefill attention (flash-attention style, mma.sync m16n8k16 bf16): CTA =
// 64 queries of one head, 4 warps x 16 rows; key tiles of 64 from the KV
// cache (cp.async, double-buffered, rows padded to 72 elements so ldmatrix
// is conflict-free); S = Q K^T in registers, online softmax seeded with the
// sink (max = sink, sum = 1), P rounded to bf16 as the A operand of P V.
// Causal and sliding-window masks per element; fully masked tiles leave the
// running state unchanged.
// ---------------------------------------------------------------------------
constexpr int kAttQ = 64, kAttK = 64, kAttPad = 72;

__global__ void __launch_bounds__(128)
    attn_prefill_kernel(const uint16_t *__restrict__ q, int T, int nh, int G, const uint16_t *__restrict__ kc,
                        const uint16_t *__restrict__ vc, int max_seq, const int32_t *__restrict__ pages,
                        int max_pages, int seq, int pos0, int window, float scale,
                        const uint16_t *__restrict__ sinks, uint16_t *__restrict__ out) {
  __shared__ __align__(16) uint16_t Ks[2][kAttK][kAttPad];
  __shared__ __align__(16) uint16_t Vs[2][kAttK][kAttPad];
  const int h = blockIdx.y, kvh = h / G;
  const int i0 = blockIdx.x * kAttQ;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, qd = lane & 3;
  const int ra = i0 + warp * 16 + g, rb = ra + 8;
  const int pa = pos0 + ra, pb = pos0 + rb;
  const size_t ld = (size_t)nh * 64;

  uint32_t qa[4][4];
#pragma unroll
  for (int ks = 0; ks < 4; ++ks) {
    const int c = h * 64 + ks * 16 + 2 * qd;
    qa[ks][0] = ra < T ? *reinterpret_cast<const uint32_t *>(q + ra * ld + c) : 0u;
    qa[ks][1] = rb < T ? *reinterpret_cast<const uint32_t *>(q + rb * ld + c) : 0u;
    qa[ks][2] = ra < T ? *reinterpret_cast<const uint32_t *>(q + ra * ld + c + 8) : 0u;
    qa[ks][3] = rb < T ? *reinterpret_cast<const uint32_t *>(q + rb * ld + c + 8) : 0u;
  }
  const int last = min(i0 + kAttQ, T) - 1;
  const int kmax = pos0 + last;
  const int kmin = window > 0 ? max(0, pos0 + i0 - window + 1) : 0;
  const int tb = kmin / kAttK, te = kmax / kAttK;
  const size_t kvbase = (size_t)kvh * max_seq;

  auto load_tile = [&](int buf, int tile) {
    const int kb = tile * kAttK;  // a key tile is one cache page
    const size_t prow = kvbase + (size_t)kv_row(pages, max_pages, seq, kb);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int id = tid + i * 128;
      const int r = id >> 3, ch = id & 7;
      const int key = kb + r;
      const bool ok = key <= kmax;
      const size_t off = (prow + (ok ? r : 0)) * 64 + ch * 8;
      cp_async_16_zfill(&Ks[buf][r][ch * 8], kc + off, ok ? 16u : 0u);
      cp_async_16_zfill(&Vs[buf][r][ch * 8], vc + off, ok ? 16u : 0u);
    }
  };

  const bool has_sink = sinks != nullptr;
  const float sink = has_sink ? bf16_to_f32(sinks[h]) : -INFINITY;
  float m[2] = {sink, sink};
  float l[2] = {has_sink ? 1.f : 0.f, has_sink ? 1.f : 0.f};
  float o[8][4];
#pragma unroll
  for (int j = 0; j < 8; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;

  load_tile(0, tb);
  cp_async_commit();
  for (int tile = tb; tile <= te; ++tile) {
    const int buf = (tile - tb) & 1;
    if (tile < te) load_tile(buf ^ 1, tile + 1);
    cp_async_commit();
    cp_async_wait<1>();
    __syncthreads();

    float s[8][4];
#pragma unroll
    for (int j = 0; j < 8; ++j) s[j][0] = s[j][1] = s[j][2] = s[j][3] = 0.f;
#pragma unroll
    for (int ks = 0; ks < 4; ++ks) {
#pragma unroll
      for (int jp = 0; jp < 4; ++jp) {
        uint32_t b[4];
        const int key = jp * 16 + (lane & 7) + (lane >> 4) * 8;
        ldmatrix_x4(b, &Ks[buf][key][(ks * 2 + ((lane >> 3) & 1)) * 8]);
        mma_bf16_16816(s[2 * jp], qa[ks], b[0], b[1]);
        mma_bf16_16816(s[2 * jp + 1], qa[ks], b[2], b[3]);
      }
    }
    const int kb = tile * kAttK;
#pragma unroll
    for (int j = 0; j < 8; ++j)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int key = kb + j * 8 + 2 * qd + (e & 1);
        const int p = e < 2 ? pa : pb;
        const bool ok = key <= p && (window <= 0 || key > p - window);
        s[j][e] = ok ? s[j][e] * scale : -INFINITY;
      }
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      float mx = -INFINITY;
#pragma unroll
      for (int j = 0; j < 8; ++j) mx = fmaxf(mx, fmaxf(s[j][2 * r], s[j][2 * r + 1]));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
      const float mn = fmaxf(m[r], mx);
      const float mu = mn == -INFINITY ? 0.f : mn;
      const float alpha = expf(m[r] - mu);
      m[r] = mn;
      float rs = 0.f;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float p0 = expf(s[j][2 * r] - mu), p1 = expf(s[j][2 * r + 1] - mu);
        s[j][2 * r] = p0;
        s[j][2 * r + 1] = p1;
        rs += p0 + p1;
      }
      rs += __shfl_xor_sync(0xffffffffu, rs, 1);
      rs += __shfl_xor_sync(0xffffffffu, rs, 2);
      l[r] = l[r] * alpha + rs;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        o[j][2 * r] *= alpha;
        o[j][2 * r + 1] *= alpha;
      }
    }
    // P as a bf16 hi + lo pair (~16 significant bits, as accurate as the
    // decode kernel's f32 weights): two MMAs per tile against the exact bf16 V
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      uint32_t ph[4], pl[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const float p0 = s[2 * kk + (u >> 1)][(u & 1) * 2], p1 = s[2 * kk + (u >> 1)][(u & 1) * 2 + 1];
        ph[u] = pack_bf16x2(p0, p1);
        pl[u] = pack_bf16x2(p0 - __uint_as_float(ph[u] << 16), p1 - __uint_as_float(ph[u] & 0xFFFF0000u));
      }
#pragma unroll
      for (int dp = 0; dp < 4; ++dp) {
        uint32_t b[4];
        const int key = kk * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
        ldmatrix_x4_trans(b, &Vs[buf][key][(dp * 2 + (lane >> 4)) * 8]);
        mma_bf16_16816(o[2 * dp], ph, b[0], b[1]);
        mma_bf16_16816(o[2 * dp + 1], ph, b[2], b[3]);
        mma_bf16_16816(o[2 * dp], pl, b[0], b[1]);
        mma_bf16_16816(o[2 * dp + 1], pl, b[2], b[3]);
      }
    }
    __syncthreads();
  }
  cp_async_wait<0>();
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    const int row = r ? rb : ra;
    if (row >= T) continue;
    const float inv = 1.0f / l[r];
    uint16_t *dst = out + row * ld + h * 64 + 2 * qd;
#pragma unroll
    for (int j = 0; j < 8; ++j)
      *reinterpret_cast<uint32_t *>(dst + j * 8) = pack_bf16x2(o[j][2 * r] * inv, o[j][2 * r + 1] * inv);
  }
}

// ---------------------------------------------------------------------------
// Greedy argmax per row of logits [rows, V]: the largest value, ties to the
// largest index (the reference's Iterator::max_by keeps the last maximum);
// NaN entries are skipped. next[row] receives the index.
// ---------------------------------------------------------------------------
constexpr int kArgThreads = 1024;

__device__ __forceinline__ bool arg_better(float v, int i, float bv, int bi) {
  return v > bv || (v == bv && i > bi);
}

__global__ void __launch_bounds__(kArgThreads)
    argmax_kernel(const float *__restrict__ logits, int V, int32_t *__restrict__ next,
                  int32_t *__restrict__ state, int32_t *__restrict__ out_seq) {
  __shared__ float sv[kArgThreads / 32];
  __shared__ int si[kArgThreads / 32];
  const float *x = logits + (size_t)blockIdx.x * V;
  float bv = -INFINITY;
  int bi = -1;
  for (int i = threadIdx.x; i < V; i += kArgThreads) {
    const float v = x[i];
    if (arg_better(v, i, bv, bi)) {
      bv = v;
      bi = i;
    }
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (oi >= 0 && (bi < 0 || arg_better(ov, oi, bv, bi))) {
      bv = ov;
      bi = oi;
    }
  }
  if ((threadIdx.x & 31) == 0) {
    sv[threadIdx.x >> 5] = bv;
    si[threadIdx.x >> 5] = bi;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    float v = sv[0];
    int ix = si[0];
    for (int w = 1; w < kArgThreads / 32; ++w)
      if (si[w] >= 0 && (ix < 0 || arg_better(sv[w], si[w], v, ix))) {
        v = sv[w];
        ix = si[w];
      }
    const int tok = ix < 0 ? 0 : ix;
    if (next) next[blockIdx.x] = tok;
    if (state) {  // one-token decode step: feed the token back and advance
      out_seq[state[1]] = tok;
      state[2] = tok;
      state[0] += 1;
      state[1] += 1;
    }
  }
}

// Decode state {position, step, current token} for the next one-token steps.
__global__ void set_state_kernel(int32_t *__restrict__ state, int pos, const int32_t *__restrict__ tok) {
  state[0] = pos;
  state[1] = 0;
  state[2] = *tok;
}

}  // namespace

// ---------------------------------------------------------------------------
// launchers
// ---------------------------------------------------------------------------
cudaError_t launch_residual_norm(const NormArgs &a, cudaStream_t stream) {
  if (a.rows <= 0) return cudaSuccess;
  if (a.S > kMaxSplits || a.H % 4) return cudaErrorInvalidValue;
  if (a.rows <= kNormClusterRows) {
    const int chunk = (a.H / 4 + kNormCl - 1) / kNormCl;
    residual_norm_cluster_kernel<<<dim3(kNormCl, a.rows), kNormClThreads, (size_t)chunk * sizeof(float4), stream>>>(
        a.res, a.H, a.tokens, a.embed, a.V, a.add, a.S, a.add_stride, a.add_bias, a.gamma, a.eps, a.out, a.err);
    return cudaGetLastError();
  }
  residual_norm_kernel<<<a.rows, kNormThreads, (size_t)a.H * sizeof(float), stream>>>(
      a.res, a.H, a.tokens, a.embed, a.V, a.add, a.S, a.add_stride, a.add_bias, a.gamma, a.eps, a.out,
      a.err);
  return cudaGetLastError();
}

int linear_splits(int N, int K, int T, int n_sms, int max_rows) {
  const int nt = T <= 8 ? 8 : 64;
  const long tiles = (long)((N + kLinRows - 1) / kLinRows) * ((T + nt - 1) / nt);
  const int nck = K / kLinK;
  long want = (2L * n_sms + tiles - 1) / tiles;
  if (want < 1) want = 1;
  if (want > nck) want = nck;
  const int tp = (T + nt - 1) / nt * nt;
  long cap = max_rows / tp;
  if (cap < 1) cap = 1;
  if (want > cap) want = cap;
  if (want > kMaxSplits) want = kMaxSplits;
  const int per = (nck + (int)want - 1) / (int)want;
  return (nck + per - 1) / per;
}

cudaError_t launch_linear(const uint16_t *x, int T, int ldx, const uint16_t *W, int N, int K, int splits,
                          float *out, cudaStream_t stream, const ArgmaxEpilogue *am) {
  if (T <= 0) return cudaSuccess;
  const int nck = K / kLinK;
  const int per = (nck + splits - 1) / splits;
  const ArgmaxEpilogue none{};
  if (T <= 8) {
    if (am && splits != 1) return cudaErrorInvalidValue;
    const dim3 grid((N + kLinRows - 1) / kLinRows, 1, splits);
    cudaError_t st = cudaFuncSetAttribute(linear_kernel<8>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          LinCfg<8>::kSmem);
    if (st != cudaSuccess) return st;
    linear_kernel<8><<<grid, kLinThreads, LinCfg<8>::kSmem, stream>>>(x, T, ldx, W, N, K, per, out,
                                                                       am ? *am : none);
  } else {
    if (am) return cudaErrorInvalidValue;
    const dim3 grid((N + kLinRows - 1) / kLinRows, (T + 63) / 64, splits);
    cudaError_t st = cudaFuncSetAttribute(linear_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          LinCfg<64>::kSmem);
    if (st != cudaSuccess) return st;
    linear_kernel<64><<<grid, kLinThreads, LinCfg<64>::kSmem, stream>>>(x, T, ldx, W, N, K, per, out, none);
  }
  return cudaGetLastError();
}

cudaError_t launch_qkv_post(const float *part, int S, int T, int nh, int nkv, const uint16_t *bias,
                            const float *rope_cos, const float *rope_sin, int pos0, const int32_t *pos_dev,
                            int kv_rows, const int32_t *pages, int max_pages, int seq, uint16_t *q_out,
                            uint16_t *kc, uint16_t *vc, cudaStream_t stream, const int32_t *tok_pos,
                            const int32_t *tok_seq) {
  if (T <= 0) return cudaSuccess;
  if (S > kMaxSplits || !pages || max_pages <= 0) return cudaErrorInvalidValue;
  const int items = (nh + nkv) * 32 + nkv * 64;
  qkv_post_kernel<<<dim3(T, (items + kQkvThreads - 1) / kQkvThreads), kQkvThreads, 0, stream>>>(
      part, S, T, nh, nkv, bias, rope_cos, rope_sin, pos0, pos_dev, tok_pos, tok_seq, pages, max_pages, seq,
      kv_rows, q_out, kc, vc);
  return cudaGetLastError();
}

int attn_decode_splits(int n_keys) { return (n_keys + kDecKeys - 1) / kDecKeys; }
// The most 64-key pages a window of `window` keys can touch.
int window_page_splits(int window) { return (window + 62) / kKvPage + 1; }

cudaError_t launch_attention(const AttnArgs &a, cudaStream_t stream) {
  if (a.T <= 0) return cudaSuccess;
  const int G = a.nh / a.nkv;
  const int Nq = a.nh * 64;
  const int rows = a.split_rows > 0 ? a.split_rows : a.max_seq;  // positions of one sequence
  if (!a.pages || a.max_pages <= 0) return cudaErrorInvalidValue;
  // the most pages one query's keys touch (full span: a.max_splits pages)
  const bool windowed = a.window > 0 && a.window < rows;
  if (a.tok_pos && a.kv_map && G == 8 && a.n_sms > 0) {  // one query of each of T sequences, tensor cores
    const size_t part_tok = attn_part_floats(a.nkv, G, rows);
    const int span_pages = windowed ? std::min(window_page_splits(a.window), a.max_splits) : a.max_splits;
    const int max_split = (span_pages + kAdPages - 1) / kAdPages;
    if (max_split <= 0 || a.max_splits > attn_decode_splits(rows)) return cudaErrorInvalidValue;
    const int n_items = a.T * max_split * a.nkv;
    const int grid = std::min((n_items + kAdWarps - 1) / kAdWarps, a.n_sms);
    cudaError_t st = cudaFuncSetAttribute(attn_decode_mma_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          (int)kAdSmem);
    if (st != cudaSuccess) return st;
    attn_decode_mma_kernel<<<grid, kAdWarps * 32, kAdSmem, stream>>>(
        *reinterpret_cast<const CUtensorMap *>(a.kv_map), a.q, a.tok_pos, a.tok_seq, a.pages, a.max_pages,
        a.k_row, a.v_row, (long long)a.max_seq, a.nkv, Nq, a.window, a.scale, max_split, n_items, a.part,
        part_tok, a.err, a.merge_cnt, a.sinks, a.out);
    if ((st = cudaGetLastError()) != cudaSuccess || a.merge_cnt) return st;
    attn_combine_kernel<<<dim3(a.nh, a.T), 64, 0, stream>>>(a.part, G, max_split, nullptr, a.window, a.sinks,
                                                           a.out, a.tok_pos, Nq, part_tok, kAdKeys);
    return cudaGetLastError();
  }
  if (a.tok_pos) {  // one query of each of T sequences
    const size_t part_tok = attn_part_floats(a.nkv, G, rows);
    const int grid_split = windowed ? std::min(window_page_splits(a.window), a.max_splits) : a.max_splits;
    if (grid_split <= 0 || grid_split > attn_decode_splits(rows)) return cudaErrorInvalidValue;
    attn_decode_kernel<<<dim3(a.nkv, grid_split, a.T), kDecThreads, 0, stream>>>(
        a.q, a.kc, a.vc, a.max_seq, G, 0, 0, a.scale, grid_split, nullptr, a.window, a.part, a.tok_pos,
        a.tok_seq, a.pages, a.max_pages, 0, Nq, part_tok);
    cudaError_t st = cudaGetLastError();
    if (st != cudaSuccess) return st;
    attn_combine_kernel<<<dim3(a.nh, a.T), 64, 0, stream>>>(a.part, G, grid_split, nullptr, a.window, a.sinks,
                                                           a.out, a.tok_pos, Nq, part_tok, kDecKeys);
    return cudaGetLastError();
  }
  if (a.T == 1) {
    const int pos = a.pos0;
    const int lo = a.window > 0 ? (pos - a.window + 1 > 0 ? pos - a.window + 1 : 0) : 0;
    // with the position on the device the grid covers the largest split count
    const int full = attn_decode_splits(rows);
    const int grid_split = a.pos_dev ? (windowed ? std::min(window_page_splits(a.window), full) : full)
                                     : page_splits(lo, pos);
    attn_decode_kernel<<<dim3(a.nkv, grid_split), kDecThreads, 0, stream>>>(
        a.q, a.kc, a.vc, a.max_seq, G, lo, pos, a.scale, grid_split, a.pos_dev, a.window, a.part, nullptr, nullptr,
        a.pages, a.max_pages, a.seq, Nq, 0);
    cudaError_t st = cudaGetLastError();
    if (st != cudaSuccess) return st;
    attn_combine_kernel<<<a.nh, 64, 0, stream>>>(a.part, G, grid_split, a.pos_dev, a.window, a.sinks, a.out,
                                                 nullptr, Nq, 0, kDecKeys);
    return cudaGetLastError();
  }
  attn_prefill_kernel<<<dim3((a.T + kAttQ - 1) / kAttQ, a.nh), 128, 0, stream>>>(
      a.q, a.T, a.nh, G, a.kc, a.vc, a.max_seq, a.pages, a.max_pages, a.seq, a.pos0, a.window, a.scale, a.sinks,
      a.out);
  return cudaGetLastError();
}

size_t attn_part_floats(int nkv, int G, int max_seq) {
  return (size_t)nkv * attn_decode_splits(max_seq) * G * 66;
}

int attn_max_group() { return kMaxGroup; }

typedef CUresult (*EncodeTiledFn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                  const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

cudaError_t make_kv_map(void *map, const uint16_t *kv, long long rows) {
  if (!map || !kv || ((uintptr_t)kv & 15) || rows <= 0 || rows >= (1LL << 31)) return cudaErrorInvalidValue;
  static EncodeTiledFn fn = nullptr;
  if (!fn) {
    void *p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return cudaErrorNotSupported;
    fn = reinterpret_cast<EncodeTiledFn>(p);
  }
  // rows of 64 bf16 (128 bytes); boxes of 64 rows with the 128-byte swizzle
  const cuuint64_t dims[2] = {64, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {128};
  const cuuint32_t box[2] = {64, (cuuint32_t)kAdTile};
  const cuuint32_t es[2] = {1u, 1u};
  CUresult r = fn(reinterpret_cast<CUtensorMap *>(map), CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2,
                  const_cast<uint16_t *>(kv), dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

cudaError_t launch_argmax(const float *logits, int rows, int V, int32_t *next, int32_t *state, int32_t *out_seq,
                          cudaStream_t stream) {
  if (rows <= 0) return cudaSuccess;
  argmax_kernel<<<rows, kArgThreads, 0, stream>>>(logits, V, next, state, out_seq);
  return cudaGetLastError();
}

cudaError_t launch_set_state(int32_t *state, int pos, const int32_t *tok, cudaStream_t stream) {
  set_state_kernel<<<1, 1, 0, stream>>>(state, pos, tok);
  return cudaGetLastError();
}

}  // namespace oxg
