// route_small.cu — router, top-k, softmax and permutation fused into one
// launch for decode-sized batches (T <= 64 tokens).
//
// Same semantics as router.cu + permute.cu (MoELayer::forward,
// src/moe.rs:40-93): logits = x . W^T (+ bias), the k largest with ties to
// the lower expert index, softmax over them with the sum taken in j order,
// and a stable grouping of the T*k (token, j) slots by expert.
//
// Phase 1 (one CTA per expert): the expert's router row is staged in shared
// memory and warp w computes the logits of tokens w, w+8, ... with 12
// independent 16-byte x loads per lane; the CTA of expert 0 also reduces
// each token's max|x| for the f16 staging exponent sigma.
// Phase 2 (the last CTA to finish, found with a completion counter): top-k
// and softmax per token (one warp per token), then the grouping of slots by
// expert (rank of each slot among the earlier slots of its expert), the
// active-expert list, and the reset of the per-band counters of the mlp2
// kernel. The counter is left at zero for the next call.
#include "common.cuh"
#include "kernels.h"
#include "mxf.cuh"

namespace oxg {
namespace {

constexpr int kWarpsPerCta = 8;
constexpr int kMaxChunks = 12;  // H <= 12 * 32 * 8 = 3072
constexpr int kMaxE = 256;

__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

__global__ void __launch_bounds__(kWarpsPerCta * 32) route_small_kernel(RouteSmallArgs a) {
  __shared__ int is_last;
  __shared__ int idx_s[kMaxRouteTokens * 16];
  __shared__ int cnt_s[kMaxE];
  __shared__ int off_s[kMaxE + 1];
  __shared__ __align__(16) uint4 w_s[kMaxChunks * 32];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int T = a.T, H = a.H, E = a.E, k = a.k;
  const int nch = H / 8;
  const int e = blockIdx.x;  // one CTA per expert

  // The previous kernel in the stream may still be reading this scratch.
  pdl_wait();

  // ---- phase 1 ----
  for (int c = tid; c < nch; c += blockDim.x)
    w_s[c] = __ldg(reinterpret_cast<const uint4 *>(a.router_w + (size_t)e * H) + c);
  __syncthreads();
  const float bias = a.router_b ? bf16_to_f32(a.router_b[e]) : 0.f;
  for (int t = warp; t < T; t += kWarpsPerCta) {
    const uint4 *xr = reinterpret_cast<const uint4 *>(a.x + (size_t)t * H);
    uint4 q[kMaxChunks];
#pragma unroll
    for (int i = 0; i < kMaxChunks; ++i) {
      const int c = lane + 32 * i;
      q[i] = c < nch ? __ldg(xr + c) : make_uint4(0, 0, 0, 0);
    }
    float acc = 0.f;
    uint32_t m = 0u;
#pragma unroll
    for (int i = 0; i < kMaxChunks; ++i) {
      const int c = lane + 32 * i;
      if (c < nch) {
        const uint4 w = w_s[c];
        acc = fmaf(bf16_to_f32(q[i].x & 0xFFFFu), bf16_to_f32(w.x & 0xFFFFu), acc);
        acc = fmaf(bf16_to_f32(q[i].x >> 16), bf16_to_f32(w.x >> 16), acc);
        acc = fmaf(bf16_to_f32(q[i].y & 0xFFFFu), bf16_to_f32(w.y & 0xFFFFu), acc);
        acc = fmaf(bf16_to_f32(q[i].y >> 16), bf16_to_f32(w.y >> 16), acc);
        acc = fmaf(bf16_to_f32(q[i].z & 0xFFFFu), bf16_to_f32(w.z & 0xFFFFu), acc);
        acc = fmaf(bf16_to_f32(q[i].z >> 16), bf16_to_f32(w.z >> 16), acc);
        acc = fmaf(bf16_to_f32(q[i].w & 0xFFFFu), bf16_to_f32(w.w & 0xFFFFu), acc);
        acc = fmaf(bf16_to_f32(q[i].w >> 16), bf16_to_f32(w.w >> 16), acc);
        if (e == 0) {
          const uint32_t m0 = max((q[i].x << 16) & 0x7FFFFFFFu, q[i].x & 0x7FFF0000u);
          const uint32_t m1 = max((q[i].y << 16) & 0x7FFFFFFFu, q[i].y & 0x7FFF0000u);
          const uint32_t m2 = max((q[i].z << 16) & 0x7FFFFFFFu, q[i].z & 0x7FFF0000u);
          const uint32_t m3 = max((q[i].w << 16) & 0x7FFFFFFFu, q[i].w & 0x7FFF0000u);
          m = max(m, max(max(m0, m1), max(m2, m3)));
        }
      }
    }
    // x as two E4M3 terms per 32-element block (4 lanes hold one block):
    // chunk iteration i of every token is done by the CTA of expert i mod E
    if (a.xq) {
#pragma unroll
      for (int i = 0; i < kMaxChunks; ++i) {
        if (i % (int)gridDim.x != e) continue;
        const int c = lane + 32 * i;
        const uint32_t w4[4] = {q[i].x, q[i].y, q[i].z, q[i].w};
        uint32_t mx = 0u;
#pragma unroll
        for (int u = 0; u < 4; ++u) mx = max(mx, max((w4[u] << 16) & 0x7FFFFFFFu, w4[u] & 0x7FFF0000u));
        mx = max(mx, __shfl_xor_sync(0xFFFFFFFFu, mx, 1));
        mx = max(mx, __shfl_xor_sync(0xFFFFFFFFu, mx, 2));
        if (c < nch) {
          const int sb = mxf::term_scale_byte(mx);
          uint32_t hi[2], lo[2];
#pragma unroll
          for (int u = 0; u < 4; u += 2) {
            uint32_t t0[2], t1[2];
            mxf::split_terms2<2>(bf16_to_f32(w4[u] & 0xFFFFu), bf16_to_f32(w4[u] >> 16), sb, t0);
            mxf::split_terms2<2>(bf16_to_f32(w4[u + 1] & 0xFFFFu), bf16_to_f32(w4[u + 1] >> 16), sb, t1);
            hi[u >> 1] = t0[0] | (t1[0] << 16);
            lo[u >> 1] = t0[1] | (t1[1] << 16);
          }
          *reinterpret_cast<uint2 *>(a.xq + (size_t)(2 * t) * H + 8 * c) = make_uint2(hi[0], hi[1]);
          *reinterpret_cast<uint2 *>(a.xq + (size_t)(2 * t + 1) * H + 8 * c) = make_uint2(lo[0], lo[1]);
          if ((c & 3) == 0) {
            const int kb = c >> 2;
            uint8_t *atom = a.xsf + (size_t)(kb >> 2) * mxf::kAtomBytes;
            atom[mxf::atom_offset(2 * t, kb & 3)] = (uint8_t)sb;
            atom[mxf::atom_offset(2 * t + 1, kb & 3)] = (uint8_t)(sb - 5);
          }
        }
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xFFFFFFFFu, acc, o);
    if (lane == 0) a.logits[(size_t)t * E + e] = acc + bias;
    if (e == 0) {
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) m = max(m, __shfl_xor_sync(0xFFFFFFFFu, m, o));
      if (lane == 0) {
        // per-token staging exponent sigma: max|x| * 2^-sigma in [2^14, 2^15)
        const int sg = (int)(m >> 23) - 141;
        a.sigma[t] = sg < -110 ? -110 : (sg > 100 ? 100 : sg);
      }
    }
  }

  // ---- hand over to the last CTA ----
  __threadfence();
  __syncthreads();
  if (tid == 0) is_last = atomicAdd(a.done, 1u) == gridDim.x - 1;
  __syncthreads();
  if (!is_last) return;
  __threadfence();

  // ---- phase 2a: top-k + softmax, one warp per token ----
  for (int t = warp; t < T; t += kWarpsPerCta) {
    constexpr int kPer = kMaxE / 32;
    float v[kPer];
    bool taken[kPer];
#pragma unroll
    for (int i = 0; i < kPer; ++i) {
      const int ex = lane + 32 * i;
      v[i] = ex < E ? __ldcg(a.logits + (size_t)t * E + ex) : -INFINITY;
      taken[i] = !(ex < E);
    }
    float top_v[16];
    int top_e[16];
    for (int j = 0; j < k; ++j) {
      float bv = 0.f;
      int be = 0x7FFFFFFF;
#pragma unroll
      for (int i = 0; i < kPer; ++i)
        if (!taken[i] && (be == 0x7FFFFFFF || v[i] > bv)) {
          bv = v[i];
          be = lane + 32 * i;
        }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xFFFFFFFFu, bv, o);
        const int oe = __shfl_xor_sync(0xFFFFFFFFu, be, o);
        if (oe != 0x7FFFFFFF && (be == 0x7FFFFFFF || ov > bv || (ov == bv && oe < be))) {
          bv = ov;
          be = oe;
        }
      }
      top_v[j] = bv;
      top_e[j] = be;
#pragma unroll
      for (int i = 0; i < kPer; ++i)
        if (lane + 32 * i == be) taken[i] = true;
    }
    if (lane == 0) {
      float mx = -INFINITY;
      for (int j = 0; j < k; ++j) mx = fmaxf(mx, top_v[j]);
      float sum = 0.f;
      for (int j = 0; j < k; ++j) {
        top_v[j] = expf(top_v[j] - mx);
        sum += top_v[j];
      }
      for (int j = 0; j < k; ++j) {
        idx_s[t * k + j] = top_e[j];
        a.idx[t * k + j] = top_e[j];
        a.wts[t * k + j] = sum == 0.f ? 1.0f / (float)k : top_v[j] / sum;
      }
    }
  }
  for (int x = tid; x < E; x += blockDim.x) cnt_s[x] = 0;
  __syncthreads();

  // ---- phase 2b: stable grouping of slots by expert ----
  const int S = T * k;
  for (int s = tid; s < S; s += blockDim.x) atomicAdd(&cnt_s[idx_s[s]], 1);
  __syncthreads();
  if (tid == 0) {
    int run = 0, n_active = 0;
    for (int x = 0; x < E; ++x) {
      off_s[x] = run;
      a.offsets[x] = run;
      a.counts[x] = cnt_s[x];
      if (cnt_s[x]) a.active[n_active++] = x;
      run += cnt_s[x];
    }
    off_s[E] = run;
    a.offsets[E] = run;
    a.n_active[0] = n_active;
    if (a.v_expert) {  // the active experts in groups of at most kVirtualTokens slots
      int nv = 0;
      for (int x = 0; x < E; ++x)
        for (int j = 0; j < cnt_s[x]; j += kVirtualTokens) {
          a.v_expert[nv] = x;
          a.v_pos0[nv] = off_s[x] + j;
          a.v_count[nv] = min(kVirtualTokens, cnt_s[x] - j);
          ++nv;
        }
      a.n_virtual[0] = nv;
    }
  }
  __syncthreads();
  for (int s = tid; s < S; s += blockDim.x) {
    const int ex = idx_s[s];
    int r = 0;
    for (int s2 = 0; s2 < s; ++s2) r += idx_s[s2] == ex;
    const int p = off_s[ex] + r;
    a.perm[p] = s;
    a.slot_pos[s] = p;
  }
  // per expert, the tokens routed to it as a bit mask (block-scaled path, T <= 32)
  if (a.tok_mask && T <= 32)
    for (int x = tid; x < E; x += blockDim.x) {
      uint32_t m = 0u;
      for (int s2 = 0; s2 < S; ++s2) m |= idx_s[s2] == x ? 1u << (s2 / k) : 0u;
      a.tok_mask[x] = m;
    }
  for (int b = tid; b < a.n_bands; b += blockDim.x) a.band_done[b] = 0u;
  if (tid == 0) *a.done = 0u;
  __threadfence();
  __syncthreads();
  pdl_launch();
}

}  // namespace

cudaError_t launch_route_small(const RouteSmallArgs &a, cudaStream_t stream, bool pdl) {
  if (a.T <= 0) return cudaSuccess;
  if (a.T > kMaxRouteTokens || a.E > kMaxE || a.k > 16 || a.k > a.E || a.H % 8 ||
      a.H > kMaxChunks * 32 * 8)
    return cudaErrorInvalidValue;
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(a.E);
  cfg.blockDim = dim3(kWarpsPerCta * 32);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, route_small_kernel, a);
}

}  // namespace oxg
