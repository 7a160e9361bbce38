// permute.cu — token-to-expert permutation (stable counting sort of slots).
//
// The reference has no permutation: it runs every (token, j) pair through its
// expert one at a time (src/moe.rs:77-93). Grouping the T*k slots by expert is
// what lets one weight read serve every token routed to an expert. The sort is
// stable — within an expert, slots keep their (token, j) order — so results do
// not depend on scheduling: position p of expert e holds the
// (p - offsets[e])-th slot routed to e in slot order.
//
// Single CTA of 1024 threads: a shared-memory histogram, a serial scan over
// the experts, then chunks of 1024 slots ranked with __match_any_sync inside
// each warp and a per-expert prefix over the 32 warps.
#include "common.cuh"
#include "kernels.h"

namespace oxg {
namespace {

constexpr int kPermThreads = 1024;
constexpr int kPermMaxExperts = 256;

__global__ void __launch_bounds__(kPermThreads) permute_kernel(
    const int32_t *__restrict__ idx, int n_slots, int E, int32_t *__restrict__ counts,
    int32_t *__restrict__ offsets, int32_t *__restrict__ perm, int32_t *__restrict__ slot_pos) {
  __shared__ int hist[kPermMaxExperts];
  __shared__ int base[kPermMaxExperts];
  __shared__ int chunk_total[kPermMaxExperts];
  __shared__ int wcnt[kPermThreads / 32][kPermMaxExperts];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  for (int e = tid; e < E; e += kPermThreads) hist[e] = 0;
  __syncthreads();
  for (int s = tid; s < n_slots; s += kPermThreads) {
    const int e = idx[s];
    if (e >= 0 && e < E) atomicAdd(&hist[e], 1);
  }
  __syncthreads();
  if (tid == 0) {
    int run = 0;
    for (int e = 0; e < E; ++e) {
      offsets[e] = run;
      base[e] = run;
      counts[e] = hist[e];
      run += hist[e];
    }
    offsets[E] = run;
  }
  __syncthreads();
  const unsigned lt_mask = (1u << lane) - 1u;
  for (int c0 = 0; c0 < n_slots; c0 += kPermThreads) {
    for (int i = tid; i < (kPermThreads / 32) * E; i += kPermThreads) wcnt[i / E][i % E] = 0;
    __syncthreads();
    const int s = c0 + tid;
    int e = s < n_slots ? idx[s] : -1;
    if (e >= E) e = -1;
    const unsigned peers = __match_any_sync(0xFFFFFFFFu, e);
    const int rank = __popc(peers & lt_mask);
    if (e >= 0 && rank == 0) wcnt[warp][e] = __popc(peers);
    __syncthreads();
    for (int x = tid; x < E; x += kPermThreads) {
      int run = 0;
      for (int w = 0; w < kPermThreads / 32; ++w) {
        const int c = wcnt[w][x];
        wcnt[w][x] = run;
        run += c;
      }
      chunk_total[x] = run;
    }
    __syncthreads();
    if (e >= 0) {
      const int p = base[e] + wcnt[warp][e] + rank;
      perm[p] = s;
      slot_pos[s] = p;
    } else if (s < n_slots) {
      slot_pos[s] = -1;
    }
    __syncthreads();
    for (int x = tid; x < E; x += kPermThreads) base[x] += chunk_total[x];
    __syncthreads();
  }
}


// Second half of the counting sort for batches routed by router_mma_kernel:
// the router left, per CTA c of 64 tokens, the histogram cta_hist[c, e] and
// each slot's rank among CTA c's slots of its expert (slot order). The
// position of slot s (expert e, router CTA c) is
//   offsets[e] + sum_{c' < c} cta_hist[c', e] + local_rank[s],
// which is exactly the stable order permute_kernel produces. kScatterSub CTAs
// share each router CTA's slots; a warp per slot also copies the token's row
// into the prefill operand (f16 x * 2^-sigma) when xp is given.
constexpr int kScatterSub = 4;
constexpr int kScatterThreads = 256;
constexpr int kScatterTokens = 64;  // tokens per router CTA
constexpr int kScatterMaxE = 64;

__global__ void __launch_bounds__(kScatterThreads) scatter_kernel(
    const int32_t *__restrict__ cta_hist, int n_cta, const int32_t *__restrict__ idx,
    const int32_t *__restrict__ local_rank, int T, int k, int E, int32_t *__restrict__ counts,
    int32_t *__restrict__ offsets, int32_t *__restrict__ perm, int32_t *__restrict__ slot_pos,
    const uint16_t *__restrict__ x, const int32_t *__restrict__ sigma, int H,
    uint16_t *__restrict__ xp, float *__restrict__ pos_scale) {
  __shared__ int base_s[kScatterMaxE], tot_s[kScatterMaxE];
  const int c = blockIdx.x / kScatterSub, sub = blockIdx.x % kScatterSub;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (int e = threadIdx.x; e < E; e += kScatterThreads) {
    int tot = 0, before = 0;
    for (int cc = 0; cc < n_cta; ++cc) {
      const int v = cta_hist[(size_t)cc * E + e];
      tot += v;
      before += cc < c ? v : 0;
    }
    tot_s[e] = tot;
    base_s[e] = before;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    int run = 0;
    for (int e = 0; e < E; ++e) {
      base_s[e] += run;
      if (blockIdx.x == 0) {
        counts[e] = tot_s[e];
        offsets[e] = run;
      }
      run += tot_s[e];
    }
    if (blockIdx.x == 0) offsets[E] = run;
  }
  __syncthreads();
  const int s_begin = c * kScatterTokens * k;
  const int s_end = min(T, (c + 1) * kScatterTokens) * k;
  const int per = (kScatterTokens * k + kScatterSub - 1) / kScatterSub;
  const int my_begin = s_begin + sub * per, my_end = min(s_end, my_begin + per);
  for (int sl = my_begin + warp; sl < my_end; sl += kScatterThreads / 32) {
    const int e = idx[sl];
    const int p = base_s[e] + local_rank[sl];
    if (lane == 0) {
      perm[p] = sl;
      slot_pos[sl] = p;
    }
    if (xp) {
      const int t = sl / k, sg = sigma[t];
      if (lane == 0) pos_scale[p] = __uint_as_float((uint32_t)(127 + sg) << 23);
      stage_row_f16(x + (size_t)t * H, xp + (size_t)p * H, H, sg, lane);
    }
  }
}

}  // namespace

cudaError_t launch_permute(const int32_t *idx, int n_slots, int E, int32_t *counts,
                           int32_t *offsets, int32_t *perm, int32_t *slot_pos,
                           cudaStream_t stream) {
  if (E > kPermMaxExperts || E <= 0) return cudaErrorInvalidValue;
  permute_kernel<<<1, kPermThreads, 0, stream>>>(idx, n_slots, E, counts, offsets, perm, slot_pos);
  return cudaGetLastError();
}

cudaError_t launch_scatter(const int32_t *cta_hist, int n_cta, const int32_t *idx,
                           const int32_t *local_rank, int T, int k, int E, int32_t *counts,
                           int32_t *offsets, int32_t *perm, int32_t *slot_pos, const uint16_t *x,
                           const int32_t *sigma, int H, uint16_t *xp, float *pos_scale,
                           cudaStream_t stream) {
  if (T == 0) return cudaSuccess;
  if (E > kScatterMaxE || E <= 0 || n_cta != (T + kScatterTokens - 1) / kScatterTokens)
    return cudaErrorInvalidValue;
  if (xp && (H % 8 || ((uintptr_t)x & 15) || ((uintptr_t)xp & 15))) return cudaErrorInvalidValue;
  scatter_kernel<<<n_cta * kScatterSub, kScatterThreads, 0, stream>>>(
      cta_hist, n_cta, idx, local_rank, T, k, E, counts, offsets, perm, slot_pos, x, sigma, H, xp,
      pos_scale);
  return cudaGetLastError();
}

}  // namespace oxg
