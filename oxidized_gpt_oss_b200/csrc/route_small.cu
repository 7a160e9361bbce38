// route_small.cu — router, top-k, softmax and permutation fused into one
// launch for decode-sized batches (T <= 64 tokens).
//
// Same semantics as router.cu + permute.cu (MoELayer::forward,
// src/moe.rs:40-93): logits = x . W^T (+ bias), the k largest with ties to
// the lower expert index, softmax over them with the sum taken in j order,
// and a stable grouping of the T*k (token, j) slots by expert.
//
// One thread-block cluster of C CTAs per token (C = min(8, ceil(E/8)), fewer
// for large T), so every phase but the last is local to a cluster:
//   1. warp w of cluster rank r computes the logits of experts r*8 + w,
//      r*8 + w + 8C, ... for the cluster's token: the router row sits in
//      registers (the next expert's row is loaded while the current one is
//      multiplied; the first is loaded before the programmatic-launch wait,
//      since the weights are never written), the token's x in registers, 12
//      independent 16-byte loads per lane each, and the logit is stored into
//      rank 0's shared memory (distributed shared memory); rank 0's warp 0
//      also reduces max|x| for the f16 staging exponent sigma, and the
//      cluster's warps split the E4M3 term split of x (block-scaled path).
//   2. after a cluster barrier, warp 0 of rank 0 picks the token's top-k and
//      its softmax (rank counting for E <= 64, rank_topk_softmax).
//   3. the last rank 0 to finish (completion counter) groups the T*k slots by
//      expert: counts, offsets, the active-expert list and the virtual
//      experts by warp prefix scans, each slot's rank among the earlier
//      slots of its expert by match_any over slot-ordered chunks of 32, the
//      token masks of the block-scaled path, the expert-parallel dispatch's
//      per-expert counts and slot ranks, and the reset of the mlp2 kernel's
//      per-band counters. The counter is left at zero.
// A token's logits come from the same per-lane chunk order and xor reduction
// whatever T is, so a token routes identically alone or in a batch.
#include "common.cuh"
#include "kernels.h"
#include "mxf.cuh"
#include "sm100.cuh"

namespace oxg {
namespace {

constexpr int kWarps = 8;
constexpr int kMaxChunks = 12;  // H <= 12 * 32 * 8 = 3072
constexpr int kMaxE = 256;

__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// Row r (H bf16 values, nch 16-byte chunks) into registers: chunk lane + 32 i.
__device__ __forceinline__ void load_row(uint4 (&v)[kMaxChunks], const uint16_t *row, int nch, int lane) {
  const uint4 *p = reinterpret_cast<const uint4 *>(row);
#pragma unroll
  for (int i = 0; i < kMaxChunks; ++i) {
    const int c = lane + 32 * i;
    v[i] = c < nch ? __ldg(p + c) : make_uint4(0, 0, 0, 0);
  }
}

// x . w over the lane's chunks (one fmaf chain in chunk then element order),
// summed over the warp by an xor butterfly.
__device__ __forceinline__ float row_dot(const uint4 (&q)[kMaxChunks], const uint4 (&w)[kMaxChunks], int nch,
                                         int lane) {
  float acc = 0.f;
#pragma unroll
  for (int i = 0; i < kMaxChunks; ++i) {
    if (lane + 32 * i < nch) {
      acc = fmaf(bf16_to_f32(q[i].x & 0xFFFFu), bf16_to_f32(w[i].x & 0xFFFFu), acc);
      acc = fmaf(bf16_to_f32(q[i].x >> 16), bf16_to_f32(w[i].x >> 16), acc);
      acc = fmaf(bf16_to_f32(q[i].y & 0xFFFFu), bf16_to_f32(w[i].y & 0xFFFFu), acc);
      acc = fmaf(bf16_to_f32(q[i].y >> 16), bf16_to_f32(w[i].y >> 16), acc);
      acc = fmaf(bf16_to_f32(q[i].z & 0xFFFFu), bf16_to_f32(w[i].z & 0xFFFFu), acc);
      acc = fmaf(bf16_to_f32(q[i].z >> 16), bf16_to_f32(w[i].z >> 16), acc);
      acc = fmaf(bf16_to_f32(q[i].w & 0xFFFFu), bf16_to_f32(w[i].w & 0xFFFFu), acc);
      acc = fmaf(bf16_to_f32(q[i].w >> 16), bf16_to_f32(w[i].w >> 16), acc);
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xFFFFFFFFu, acc, o);
  return acc;
}

// Largest |value| of two packed bf16 values as the bit pattern of a positive f32.
__device__ __forceinline__ uint32_t absmax2(uint32_t v) {
  return max((v << 16) & 0x7FFFFFFFu, v & 0x7FFF0000u);
}

// Top-k of one token's logits (logit_s, E of them) and the softmax over them
// by one warp, for E > 64: k rounds of a warp-wide arg-max (ties to the
// lower index), exp(v - max) summed in j order.
__device__ __forceinline__ void select_topk_softmax(const float *logit_s, int E, int k, int lane, int32_t *idx_out,
                                                    float *wts_out) {
  constexpr int kPer = kMaxE / 32;
  float v[kPer];
  bool taken[kPer];
#pragma unroll
  for (int i = 0; i < kPer; ++i) {
    const int ex = lane + 32 * i;
    v[i] = ex < E ? logit_s[ex] : -INFINITY;
    taken[i] = !(ex < E);
  }
  float top_v[kRankTopKMax];
  int top_e[kRankTopKMax];
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
      idx_out[j] = top_e[j];
      wts_out[j] = sum == 0.f ? 1.0f / (float)k : top_v[j] / sum;
    }
  }
}

// The x of token t as two E4M3 terms per element (rows 2t, 2t+1 of xq) with
// one UE8M0 byte per 32-element block in the scale atoms xsf; the chunk
// iterations are split over n_workers warps (4 lanes hold one block).
__device__ __forceinline__ void split_x_terms(const RouteSmallArgs &a, const uint4 (&q)[kMaxChunks], int t, int nch,
                                              int worker, int n_workers, int lane) {
  const int H = a.H;
#pragma unroll
  for (int i = 0; i < kMaxChunks; ++i) {
    if (i % n_workers != worker) continue;
    const int c = lane + 32 * i;
    const uint32_t w4[4] = {q[i].x, q[i].y, q[i].z, q[i].w};
    uint32_t mx = 0u;
#pragma unroll
    for (int u = 0; u < 4; ++u) mx = max(mx, absmax2(w4[u]));
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

// Grouping of the S = T*k slots by expert, run by the whole (last) CTA once
// every token's idx is in global memory (or, for one token, in idx_local):
// counts, offsets, the active-expert list and the virtual experts by warp
// scans over chunks of 32 experts (expert order, so the lists come out
// sorted), then perm / slot_pos with each slot's rank among the earlier
// slots of its expert (slot order), and the per-expert token masks of the
// block-scaled path (T <= 32).
__device__ __forceinline__ void group_slots(const RouteSmallArgs &a, const int *idx_local, int *idx_s,
                                            int *cnt_s, int *off_s, int *run_s, uint32_t *mask_s) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int E = a.E, k = a.k, S = a.T * a.k;
  for (int s = tid; s < S; s += blockDim.x) idx_s[s] = idx_local ? idx_local[s] : __ldcg(a.idx + s);
  for (int x = tid; x < E; x += blockDim.x) {
    cnt_s[x] = 0;
    run_s[x] = 0;
    mask_s[x] = 0u;
  }
  __syncthreads();
  const bool masks = a.tok_mask && a.T <= 32;
  for (int s = tid; s < S; s += blockDim.x) {
    atomicAdd(&cnt_s[idx_s[s]], 1);
    if (masks) atomicOr(&mask_s[idx_s[s]], 1u << (s / k));
  }
  __syncthreads();
  if (warp == 0) {
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
        if (masks) a.tok_mask[x] = mask_s[x];
        if (a.cta_hist) a.cta_hist[x] = c;
      }
      run += __shfl_sync(0xFFFFFFFFu, cs, 31);
      n_act += __shfl_sync(0xFFFFFFFFu, as, 31);
      n_v += __shfl_sync(0xFFFFFFFFu, gs, 31);
    }
    if (lane == 0) {
      a.offsets[E] = run;
      a.n_active[0] = n_act;
      if (a.v_expert) a.n_virtual[0] = n_v;
    }
    __syncwarp();
    // ranks: slots in chunks of 32 in slot order; a slot's rank is the count
    // of its expert in earlier chunks plus its lower-lane peers in this one
    const uint32_t lt = (1u << lane) - 1u;
    for (int s0 = 0; s0 < S; s0 += 32) {
      const int s = s0 + lane;
      const int ex = s < S ? idx_s[s] : -1;
      const uint32_t peers = __match_any_sync(0xFFFFFFFFu, ex);
      if (s < S) {
        const int r = run_s[ex] + __popc(peers & lt);
        const int p = off_s[ex] + r;
        a.perm[p] = s;
        a.slot_pos[s] = p;
        if (a.local_rank) a.local_rank[s] = r;
      }
      __syncwarp();
      if (s < S && lane == 31 - __clz(peers)) run_s[ex] += __popc(peers);
      __syncwarp();
    }
  }
}

__global__ void __launch_bounds__(kWarps * 32, 1) route_token_kernel(RouteSmallArgs a) {
  __shared__ int is_last;
  __shared__ float logit_s[kMaxE];  // rank 0: the token's logits, stored by every rank
  __shared__ int idx_s[kMaxRouteTokens * kRankTopKMax];
  __shared__ int cnt_s[kMaxE], off_s[kMaxE], run_s[kMaxE];
  __shared__ uint32_t mask_s[kMaxE];
  __shared__ float top_v_s[kRankTopKMax];
  __shared__ int top_e_s[kRankTopKMax], top_i_s[kRankTopKMax];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int H = a.H, E = a.E, k = a.k;
  const int nch = H / 8;
  const int t = blockIdx.y;  // one cluster per token
  const int C = (int)gridDim.x, r = (int)sm100::cluster_ctarank();
  const int e0 = r * kWarps + warp, step = C * kWarps;

  // the warp's first router row: read-only, so loaded before the wait
  uint4 w[kMaxChunks];
  if (e0 < E) load_row(w, a.router_w + (size_t)e0 * H, nch, lane);

  // The previous kernel in the stream may still be writing x or reading the
  // routing scratch this kernel writes.
  pdl_wait();

  uint4 q[kMaxChunks];
  load_row(q, a.x + (size_t)t * H, nch, lane);
  if (r == 0 && warp == 0) {
    uint32_t m = 0u;
#pragma unroll
    for (int i = 0; i < kMaxChunks; ++i)
      m = max(m, max(max(absmax2(q[i].x), absmax2(q[i].y)), max(absmax2(q[i].z), absmax2(q[i].w))));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = max(m, __shfl_xor_sync(0xFFFFFFFFu, m, o));
    if (lane == 0) {
      // per-token staging exponent sigma: max|x| * 2^-sigma in [2^14, 2^15)
      const int sg = (int)(m >> 23) - 141;
      a.sigma[t] = sg < -110 ? -110 : (sg > 100 ? 100 : sg);
    }
  }
  if (a.xq) split_x_terms(a, q, t, nch, e0, step, lane);

  const uint32_t logit0 = sm100::mapa_shared(sm100::smem_addr(logit_s), 0u);
  for (int e = e0; e < E; e += step) {
    uint4 wn[kMaxChunks];
    if (e + step < E) load_row(wn, a.router_w + (size_t)(e + step) * H, nch, lane);
    const float acc = row_dot(q, w, nch, lane);
    if (lane == 0) {
      const float v = acc + (a.router_b ? bf16_to_f32(a.router_b[e]) : 0.f);
      asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(logit0 + 4u * (uint32_t)e), "f"(v) : "memory");
      a.logits[(size_t)t * E + e] = v;
    }
    if (e + step < E) {
#pragma unroll
      for (int i = 0; i < kMaxChunks; ++i) w[i] = wn[i];
    }
  }
  sm100::cluster_sync();  // every logit is in rank 0's shared memory
  if (r != 0) return;
  if (warp == 0) {
    if (E <= 64)
      rank_topk_softmax(logit_s, E, k, lane, a.idx + t * k, a.wts + t * k, top_i_s, top_v_s, top_e_s);
    else
      select_topk_softmax(logit_s, E, k, lane, a.idx + t * k, a.wts + t * k);
  }

  // ---- hand over to the last token's rank 0 (one token: this CTA) ----
  const bool single = gridDim.y == 1;
  if (!single) {
    __threadfence();
    __syncthreads();
    if (tid == 0) is_last = atomicAdd(a.done, 1u) == gridDim.y - 1;
    __syncthreads();
    if (!is_last) return;
    __threadfence();
  } else {
    __syncthreads();
  }

  group_slots(a, single ? top_i_s : nullptr, idx_s, cnt_s, off_s, run_s, mask_s);
  for (int b = tid; b < a.n_bands; b += blockDim.x) a.band_done[b] = 0u;
  if (tid == 0 && !single) *a.done = 0u;
  // the dependents read all of this after their griddepcontrol.wait, which
  // waits for this grid to complete and its writes to be visible
  pdl_launch();
}

}  // namespace

cudaError_t launch_route_small(const RouteSmallArgs &a, cudaStream_t stream, bool pdl) {
  if (a.T <= 0) return cudaSuccess;
  if (a.T > kMaxRouteTokens || a.E > kMaxE || a.k > kRankTopKMax || a.k > a.E || a.H % 8 ||
      a.H > kMaxChunks * 32 * 8)
    return cudaErrorInvalidValue;
  // CTAs per token: enough for one expert per warp, at most 8, and about
  // 128 CTAs in all (more CTAs per token only queue behind each other)
  const int C = std::max(1, std::min(std::min(8, (a.E + kWarps - 1) / kWarps), 128 / a.T));
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(C, a.T);
  cfg.blockDim = dim3(kWarps * 32);
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
  attr[1].id = cudaLaunchAttributeClusterDimension;
  attr[1].val.clusterDim.x = C;
  attr[1].val.clusterDim.y = 1;
  attr[1].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  return cudaLaunchKernelEx(&cfg, route_token_kernel, a);
}

}  // namespace oxg
