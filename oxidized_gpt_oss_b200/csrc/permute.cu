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

}  // namespace

cudaError_t launch_permute(const int32_t *idx, int n_slots, int E, int32_t *counts,
                           int32_t *offsets, int32_t *perm, int32_t *slot_pos,
                           cudaStream_t stream) {
  if (E > kPermMaxExperts || E <= 0) return cudaErrorInvalidValue;
  permute_kernel<<<1, kPermThreads, 0, stream>>>(idx, n_slots, E, counts, offsets, perm, slot_pos);
  return cudaGetLastError();
}

}  // namespace oxg
