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
// and softmax per token (one warp per token; for E <= 64 by rank counting,
// rank_topk_softmax), then the grouping of slots by expert: offsets, the
// active-expert list and the virtual experts by warp prefix scans, the rank
// of each slot among the earlier slots of its expert, and the reset of the
// per-band counters of the mlp2 kernel. The counter is left at zero for the
// next call.
#include "common.cuh"
#include "kernels.h"
#include "mxf.cuh"
#include "sm100.cuh"

namespace oxg {
namespace {

constexpr int kWarpsPerCta = 8;
constexpr int kMaxChunks = 12;  // H <= 12 * 32 * 8 = 3072
constexpr int kMaxE = 256;

__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// Phase 2, run by one CTA of kWarpsPerCta warps once every logit exists:
// top-k and softmax per token (one warp per token; for E <= 64 by rank
// counting from logit_s [T][E], read from a.logits first unless
// logits_in_smem), then the grouping of slots by expert (offsets, the
// active-expert list and the virtual experts by warp prefix scans; each
// slot's rank among the earlier slots of its expert), the token masks of the
// block-scaled path, and leaves the block synchronised.
__device__ __forceinline__ void route_phase2(const RouteSmallArgs &a, float *logit_s, int *idx_s, int *cnt_s,
                                             int *off_s, float (*top_v_s)[kRankTopKMax],
                                             int (*top_e_s)[kRankTopKMax], bool logits_in_smem) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int T = a.T, E = a.E, k = a.k;
  // ---- phase 2a: top-k + softmax, one warp per token ----
  if (E <= 64) {
    // rank counting over the token's logits (rank_topk_softmax)
    if (!logits_in_smem) {
      for (int i = tid; i < T * E; i += blockDim.x) logit_s[i] = __ldcg(a.logits + i);
      __syncthreads();
    }
    for (int t = warp; t < T; t += kWarpsPerCta)
      rank_topk_softmax(logit_s + t * E, E, k, lane, a.idx + t * k, a.wts + t * k, idx_s + t * k,
                        top_v_s[warp], top_e_s[warp]);
  } else {
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
  }
  for (int x = tid; x < E; x += blockDim.x) cnt_s[x] = 0;
  __syncthreads();

  // ---- phase 2b: stable grouping of slots by expert ----
  const int S = T * k;
  for (int s = tid; s < S; s += blockDim.x) atomicAdd(&cnt_s[idx_s[s]], 1);
  __syncthreads();
  if (warp == 0) {
    // offsets, the active-expert list and the virtual experts by warp scans
    // over chunks of 32 experts (expert order, so the lists come out sorted)
    int run = 0, n_act = 0, n_v = 0;
    for (int x0 = 0; x0 < E; x0 += 32) {
      const int x = x0 + lane;
      const int c = x < E ? cnt_s[x] : 0;
      const int ng = (c + kVirtualTokens - 1) / kVirtualTokens;
      int cs = c, as = c > 0 ? 1 : 0, gs = ng;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int v1 = __shfl_up_sync(0xFFFFFFFFu, cs, o);
        const int v2 = __shfl_up_sync(0xFFFFFFFFu, as, o);
        const int v3 = __shfl_up_sync(0xFFFFFFFFu, gs, o);
        if (lane >= o) {
          cs += v1;
          as += v2;
          gs += v3;
        }
      }
      if (x < E) {
        const int off = run + cs - c;
        off_s[x] = off;
        a.offsets[x] = off;
        a.counts[x] = c;
        if (c) a.active[n_act + as - 1] = x;
        if (a.v_expert) {
          int gi = n_v + gs - ng;
          for (int j = 0; j < c; j += kVirtualTokens, ++gi) {
            a.v_expert[gi] = x;
            a.v_pos0[gi] = off + j;
            a.v_count[gi] = min(kVirtualTokens, c - j);
          }
        }
      }
      run += __shfl_sync(0xFFFFFFFFu, cs, 31);
      n_act += __shfl_sync(0xFFFFFFFFu, as, 31);
      n_v += __shfl_sync(0xFFFFFFFFu, gs, 31);
    }
    if (lane == 0) {
      off_s[E] = run;
      a.offsets[E] = run;
      a.n_active[0] = n_act;
      if (a.v_expert) a.n_virtual[0] = n_v;
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
}

__global__ void __launch_bounds__(kWarpsPerCta * 32) route_small_kernel(RouteSmallArgs a) {
  __shared__ int is_last;
  __shared__ int idx_s[kMaxRouteTokens * 16];
  __shared__ int cnt_s[kMaxE];
  __shared__ int off_s[kMaxE + 1];
  __shared__ __align__(16) uint4 w_s[kMaxChunks * 32];
  __shared__ float logit_s[kMaxRouteTokens * 64];  // phase 2a, E <= 64
  __shared__ float top_v_s[kWarpsPerCta][kRankTopKMax];
  __shared__ int top_e_s[kWarpsPerCta][kRankTopKMax];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int T = a.T, H = a.H, E = a.E;
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

  route_phase2(a, logit_s, idx_s, cnt_s, off_s, top_v_s, top_e_s, /*logits_in_smem=*/false);
  for (int b = tid; b < a.n_bands; b += blockDim.x) a.band_done[b] = 0u;
  if (tid == 0) *a.done = 0u;
  __threadfence();
  __syncthreads();
  pdl_launch();
}

// ---- cluster variant (T <= 16, E <= 64 and a multiple of 8, no E4M3 terms) ----
// One thread-block cluster of kRcCtas CTAs: CTA r stages the router rows of
// experts [r E/8, (r+1) E/8) in shared memory and computes their logits for
// every token (warp w: tokens w, w+8, ...; the same per-lane chunk order and
// xor reduction as route_small_kernel, so the logits are bit-identical);
// rank 0 also reduces max|x| per token. After a cluster barrier rank 0 reads
// all logits from its peers' shared memory (distributed shared memory), a
// second barrier lets the peers exit, and rank 0 runs phase 2. No global
// round trip of the logits, no threadfence or completion counter between the
// two phases.
constexpr int kRcCtas = 8;
constexpr int kRcMaxTokens = 16;
constexpr int kRcMaxPer = 8;  // experts per CTA (E <= 64)

__global__ void __launch_bounds__(kWarpsPerCta * 32) route_cluster_kernel(RouteSmallArgs a) {
  extern __shared__ __align__(16) uint4 rw_s[];  // [per][H / 8] router rows of this CTA
  __shared__ float my_logit[kRcMaxTokens * kRcMaxPer];
  __shared__ float logit_s[kRcMaxTokens * 64];
  __shared__ int idx_s[kRcMaxTokens * 16];
  __shared__ int cnt_s[64];
  __shared__ int off_s[65];
  __shared__ float top_v_s[kWarpsPerCta][kRankTopKMax];
  __shared__ int top_e_s[kWarpsPerCta][kRankTopKMax];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int T = a.T, H = a.H, E = a.E;
  const int nch = H / 8;
  const uint32_t r = sm100::cluster_ctarank();
  const int per = E / kRcCtas, e0 = (int)r * per;

  pdl_wait();
  for (int c = tid; c < per * nch; c += blockDim.x)
    rw_s[c] = __ldg(reinterpret_cast<const uint4 *>(a.router_w + (size_t)e0 * H) + c);
  __syncthreads();
  for (int t = warp; t < T; t += kWarpsPerCta) {
    const uint4 *xr = reinterpret_cast<const uint4 *>(a.x + (size_t)t * H);
    uint4 q[kMaxChunks];
#pragma unroll
    for (int i = 0; i < kMaxChunks; ++i) {
      const int c = lane + 32 * i;
      q[i] = c < nch ? __ldg(xr + c) : make_uint4(0, 0, 0, 0);
    }
    if (r == 0) {
      uint32_t m = 0u;
#pragma unroll
      for (int i = 0; i < kMaxChunks; ++i) {
        const uint32_t m0 = max((q[i].x << 16) & 0x7FFFFFFFu, q[i].x & 0x7FFF0000u);
        const uint32_t m1 = max((q[i].y << 16) & 0x7FFFFFFFu, q[i].y & 0x7FFF0000u);
        const uint32_t m2 = max((q[i].z << 16) & 0x7FFFFFFFu, q[i].z & 0x7FFF0000u);
        const uint32_t m3 = max((q[i].w << 16) & 0x7FFFFFFFu, q[i].w & 0x7FFF0000u);
        m = max(m, max(max(m0, m1), max(m2, m3)));
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) m = max(m, __shfl_xor_sync(0xFFFFFFFFu, m, o));
      if (lane == 0) {
        const int sg = (int)(m >> 23) - 141;  // max|x| * 2^-sigma in [2^14, 2^15)
        a.sigma[t] = sg < -110 ? -110 : (sg > 100 ? 100 : sg);
      }
    }
    for (int el = 0; el < per; ++el) {
      const uint4 *wr = rw_s + el * nch;
      float acc = 0.f;
#pragma unroll
      for (int i = 0; i < kMaxChunks; ++i) {
        const int c = lane + 32 * i;
        if (c < nch) {
          const uint4 w = wr[c];
          acc = fmaf(bf16_to_f32(q[i].x & 0xFFFFu), bf16_to_f32(w.x & 0xFFFFu), acc);
          acc = fmaf(bf16_to_f32(q[i].x >> 16), bf16_to_f32(w.x >> 16), acc);
          acc = fmaf(bf16_to_f32(q[i].y & 0xFFFFu), bf16_to_f32(w.y & 0xFFFFu), acc);
          acc = fmaf(bf16_to_f32(q[i].y >> 16), bf16_to_f32(w.y >> 16), acc);
          acc = fmaf(bf16_to_f32(q[i].z & 0xFFFFu), bf16_to_f32(w.z & 0xFFFFu), acc);
          acc = fmaf(bf16_to_f32(q[i].z >> 16), bf16_to_f32(w.z >> 16), acc);
          acc = fmaf(bf16_to_f32(q[i].w & 0xFFFFu), bf16_to_f32(w.w & 0xFFFFu), acc);
          acc = fmaf(bf16_to_f32(q[i].w >> 16), bf16_to_f32(w.w >> 16), acc);
        }
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xFFFFFFFFu, acc, o);
      if (lane == 0) {
        const float v = acc + (a.router_b ? bf16_to_f32(a.router_b[e0 + el]) : 0.f);
        my_logit[t * kRcMaxPer + el] = v;
        a.logits[(size_t)t * E + e0 + el] = v;
      }
    }
  }
  sm100::cluster_sync();  // every CTA's logits are in its shared memory
  if (r == 0) {
    const uint32_t base = sm100::smem_addr(my_logit);
    for (int i = tid; i < T * E; i += blockDim.x) {
      const int t = i / E, e = i % E;
      const uint32_t addr = sm100::mapa_shared(base + (uint32_t)(t * kRcMaxPer + e % per) * 4u, (uint32_t)(e / per));
      float v;
      asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(addr) : "memory");
      logit_s[i] = v;
    }
  }
  sm100::cluster_sync();  // rank 0 has read them: the other CTAs may exit
  if (r != 0) return;
  route_phase2(a, logit_s, idx_s, cnt_s, off_s, top_v_s, top_e_s, /*logits_in_smem=*/true);
  for (int b = tid; b < a.n_bands; b += blockDim.x) a.band_done[b] = 0u;
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
  if (a.T <= kRcMaxTokens && a.E % kRcCtas == 0 && a.E <= kRcCtas * kRcMaxPer && !a.xq && !a.tok_mask) {
    const size_t smem = (size_t)(a.E / kRcCtas) * a.H * 2;
    cudaError_t st = cudaFuncSetAttribute(route_cluster_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          (int)smem);
    if (st != cudaSuccess) return st;
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(kRcCtas);
    cfg.blockDim = dim3(kWarpsPerCta * 32);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = kRcCtas;
    attr[1].val.clusterDim.y = 1;
    attr[1].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    return cudaLaunchKernelEx(&cfg, route_cluster_kernel, a);
  }
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
