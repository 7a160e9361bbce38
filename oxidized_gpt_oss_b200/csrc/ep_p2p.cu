// ep_p2p.cu — the expert-parallel exchange over NVLink peer memory.
//
// The reference has no multi-device path (MoELayer::forward, src/moe.rs:16-100,
// runs every expert in one process). With one process per GPU and the experts
// split per rank, every rank owns one symmetric buffer (same layout on every
// rank, mapped into the others by CUDA IPC): flag words, a counts inbox, the
// receive rows and the return rows (EpLayout, kernels.h). One forward is:
//
//   router_mma_kernel        idx, weights, sigma, per-CTA histograms and ranks
//                            (route_token_kernel for batches of <= 64 tokens)
//   ep_counts_kernel         this rank's per-expert counts into every rank's
//                            inbox, then a counts flag to every rank; then it
//                            waits until all ranks' counts are here
//   ep_scatter_kernel        each slot's f16 operand row (x * 2^-sigma) and its
//                            2^sigma stored straight into the destination
//                            rank's receive rows; the last CTA raises a rows
//                            flag on every rank
//   ep_segments_kernel       waits for every rank's rows flag, then builds the
//                            segment table of the received rows (source-major,
//                            resident expert order) and, per segment, where its
//                            output rows go: the source rank's return rows
//   GEMM1, GEMM2             the resident experts (GEMM2's epilogue stores each
//                            row into its source's return rows)
//   ep_signal_kernel         a returns flag to every rank, then it waits
//                            until every rank has sent this rank's rows back
//   combine_kernel           as on one GPU, from the return rows
//
// Flags carry the forward's epoch (increasing per forward), so nothing is
// reset between forwards; a step that failed on a rank raises its flags with
// the poison bit, and waiting ranks then skip their work and report it. Every
// wait is bounded (~2 s of SM clock) and records a code in the error word.
// Stores only: no remote loads, no TMA or multicast on peer memory.
#include "common.cuh"
#include "kernels.h"

namespace oxg {
namespace {

constexpr uint32_t kPoison = 0x80000000u;
constexpr long long kEpWaitCycles = 4000000000LL;  // the default budget (~2 s of SM clock)

__device__ __forceinline__ void st_release_sys(uint32_t *p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t *p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ uint32_t *flag_ptr(const EpLayout &L, char *base, int kind, int from) {
  return reinterpret_cast<uint32_t *>(base + L.off_flags) + kind * kEpMaxRanks + from;
}
__device__ __forceinline__ const int32_t *inbox(const EpLayout &L, const EpPeers &P) {
  return reinterpret_cast<const int32_t *>(P.base[L.rank] + L.off_inbox);  // [W][E]
}

// Raises flag `kind` (from this rank) on every rank: epoch, or epoch | poison.
__device__ void raise_flags(const EpLayout &L, const EpPeers &P, int kind, uint32_t epoch, bool ok) {
  __threadfence_system();
  for (int d = 0; d < L.W; ++d)
    st_release_sys(flag_ptr(L, P.base[d], kind, L.rank), ok ? epoch : (epoch | kPoison));
}

// Lane s < W waits for flag `kind` from rank s; returns the warp's verdict.
__device__ bool wait_flags(const EpLayout &L, const EpPeers &P, int kind, uint32_t epoch, int *err,
                           int code) {
  const int lane = threadIdx.x & 31;
  bool ok = true;
  if (lane < L.W) {
    const uint32_t *f = flag_ptr(L, P.base[L.rank], kind, lane);
    const long long t0 = clock64();
    while (true) {
      const uint32_t v = ld_acquire_sys(f);
      if ((int)((v & ~kPoison) - epoch) >= 0) {
        if (v & kPoison) {
          ok = false;
          atomicCAS(err, 0, 50);
        }
        break;
      }
      if (clock64() - t0 > L.wait_cycles) {
        ok = false;
        atomicCAS(err, 0, code);
        break;
      }
    }
  }
  return __all_sync(0xFFFFFFFFu, ok);
}

// One CTA: totals per expert from the router's per-CTA histograms, local
// counts/offsets, then the counts into every rank's inbox row `rank`.
__global__ void __launch_bounds__(256) ep_counts_kernel(EpLayout L, EpPeers P,
                                                        const int32_t *__restrict__ cta_hist,
                                                        int n_cta, int32_t *counts, int32_t *offsets,
                                                        int *ok_word, uint32_t epoch, int *err, int code) {
  __shared__ int tot_s[kEpMaxExperts], before_s[kEpMaxExperts], part_s[2 * 256];
  if (threadIdx.x == 0) *ok_word = 1;
  hist_prefix<256>(cta_hist, n_cta, L.E, n_cta, before_s, tot_s, part_s);
  for (int e = threadIdx.x; e < L.E; e += blockDim.x) counts[e] = tot_s[e];
  if (threadIdx.x == 0) {
    int run = 0;
    for (int e = 0; e < L.E; ++e) {
      offsets[e] = run;
      run += tot_s[e];
    }
    offsets[L.E] = run;
  }
  for (int i = threadIdx.x; i < L.W * L.E; i += blockDim.x) {
    const int d = i / L.E, e = i % L.E;
    reinterpret_cast<int32_t *>(P.base[d] + L.off_inbox)[L.rank * L.E + e] = tot_s[e];
  }
  __threadfence_system();  // every writer orders its own stores before the flag
  __syncthreads();
  if (threadIdx.x == 0) raise_flags(L, P, 0, epoch, true);
  // then every rank's counts
  if (threadIdx.x < 32 && !wait_flags(L, P, 0, epoch, err, code) && threadIdx.x == 0) *ok_word = 0;
}

// As scatter_kernel (permute.cu) for the positions; rows go to the owner of
// their expert: row p of this rank's rows for rank d lands at d's receive row
// (rows of ranks < this one for d) + p.
constexpr int kEpSub = 4, kEpThreads = 256, kEpTokens = 64;

__global__ void __launch_bounds__(kEpThreads) ep_scatter_kernel(
    EpLayout L, EpPeers P, const int32_t *__restrict__ cta_hist, int n_cta,
    const int32_t *__restrict__ idx, const int32_t *__restrict__ local_rank, int T,
    const uint16_t *__restrict__ x, const int32_t *__restrict__ sigma, int32_t *__restrict__ slot_pos,
    uint32_t *done_ctr, int *ok_word, int *err, uint32_t epoch) {
  __shared__ int base_s[kEpMaxExperts];
  __shared__ long long dbase_s[kEpMaxRanks];
  __shared__ int doff_s[kEpMaxRanks];
  __shared__ int ok_s;
  const int c = blockIdx.x / kEpSub, sub = blockIdx.x % kEpSub;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int32_t *in = inbox(L, P);
  const int32_t *mine = in + (size_t)L.rank * L.E;
  __shared__ int before_s[kEpMaxExperts], tot_s[kEpMaxExperts], part_s[2 * kEpThreads];
  if (threadIdx.x == 0) ok_s = *(volatile int *)ok_word;
  hist_prefix<kEpThreads>(cta_hist, n_cta, L.E, c, before_s, tot_s, part_s);
  for (int e = threadIdx.x; e < L.E; e += blockDim.x) {
    int off = 0;
    for (int e2 = 0; e2 < e; ++e2) off += mine[e2];
    base_s[e] = off + before_s[e];
  }
  for (int d = threadIdx.x; d < L.W; d += blockDim.x) {
    long long b = 0;
    for (int s = 0; s < L.rank; ++s)
      for (int e = d * L.per; e < (d + 1) * L.per; ++e) b += in[(size_t)s * L.E + e];
    dbase_s[d] = b;
    int o = 0;
    for (int e = 0; e < d * L.per; ++e) o += mine[e];
    doff_s[d] = o;
  }
  __syncthreads();
  const bool ok = ok_s != 0;
  const int s_begin = c * kEpTokens * L.k;
  const int s_end = min(T, (c + 1) * kEpTokens) * L.k;
  const int per = (kEpTokens * L.k + kEpSub - 1) / kEpSub;
  const int my_begin = s_begin + sub * per, my_end = min(s_end, my_begin + per);
  bool overflow = false;
  // This warp's slots are my_begin + warp + W i (W warps): their positions,
  // destinations and sigma are fetched one slot per lane, all at once, then
  // the rows are stored one after another (one metadata round trip per 32
  // slots instead of three per slot).
  constexpr int W = kEpThreads / 32;
  const int n_mine = my_end - my_begin;
  const int n_w = n_mine > warp ? (n_mine - warp + W - 1) / W : 0;
  for (int i0 = 0; i0 < n_w; i0 += 32) {
    const int li = i0 + lane;
    const int sl_l = my_begin + warp + W * li;
    int d_l = -1, sg_l = 0;
    long long drow_l = 0;
    if (li < n_w) {
      const int e = idx[sl_l];
      const int p = base_s[e] + local_rank[sl_l];
      slot_pos[sl_l] = p;
      if (ok) {
        const int d = e / L.per;
        const long long drow = dbase_s[d] + (p - doff_s[d]);
        if (drow >= L.max_recv) {
          overflow = true;
        } else {
          d_l = d;
          drow_l = drow;
          sg_l = sigma[sl_l / L.k];
          reinterpret_cast<float *>(P.base[d] + L.off_recv_scale)[drow] =
              __uint_as_float((uint32_t)(127 + sg_l) << 23);
        }
      }
    }
    const int n_here = min(32, n_w - i0);
    for (int j = 0; j < n_here; ++j) {
      const int d = __shfl_sync(0xFFFFFFFFu, d_l, j);
      const long long drow = __shfl_sync(0xFFFFFFFFu, drow_l, j);
      const int sg = __shfl_sync(0xFFFFFFFFu, sg_l, j);
      if (d < 0) continue;  // the same for every lane of the warp
      const int t = (my_begin + warp + W * (i0 + j)) / L.k;
      stage_row_f16(x + (size_t)t * L.H,
                    reinterpret_cast<uint16_t *>(P.base[d] + L.off_recv_rows) + drow * L.H, L.H, sg, lane);
    }
  }
  if (overflow) {
    atomicCAS(err, 0, 51);
    atomicExch(ok_word, 0);
  }
  __threadfence_system();  // every writer orders its own stores before the count
  __syncthreads();
  if (threadIdx.x == 0) {
    const uint32_t prev = atomicAdd(done_ctr, 1u);
    if (prev == gridDim.x - 1) {  // the last CTA: every row of this rank is out
      *done_ctr = 0u;
      __threadfence_system();
      raise_flags(L, P, 1, epoch, *(volatile int *)ok_word != 0);
    }
  }
}

// Waits for every rank's rows, then the segment table: segment v = (source s,
// resident expert el) holds inbox[s][rank * per + el] rows; its output rows go
// to s's return rows from that expert's first position in s's dispatch order.
__global__ void __launch_bounds__(256) ep_segments_kernel(EpLayout L, EpPeers P, uint32_t epoch,
                                                          int *err, int *ok_word, int32_t *seg,
                                                          float **seg_ptr, EpVirtual virt) {
  __shared__ int ok_s;
  if (threadIdx.x < 32) {
    const bool ok = wait_flags(L, P, 1, epoch, err, 12);
    if (threadIdx.x == 0) {
      if (!ok) *ok_word = 0;
      ok_s = ok && *(volatile int *)ok_word != 0;
    }
  }
  __syncthreads();
  const int32_t *in = inbox(L, P);
  const int nv = L.W * L.per;
  for (int v = threadIdx.x; v < nv; v += blockDim.x) {
    const int s = v / L.per, e = L.rank * L.per + v % L.per;
    int off = 0;
    for (int e2 = 0; e2 < e; ++e2) off += in[(size_t)s * L.E + e2];
    seg[v] = ok_s ? in[(size_t)s * L.E + e] : 0;
    seg_ptr[v] = reinterpret_cast<float *>(P.base[s] + L.off_ret_rows) + (size_t)off * L.H;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    int run = 0;
    for (int v = 0; v < nv; ++v) {
      seg[kEpMaxSegments + v] = run;
      run += seg[v];
    }
    seg[kEpMaxSegments + nv] = run;
    if (virt.n) {  // each segment in groups of at most kVirtualTokens rows
      int g = 0;
      for (int v = 0; v < nv; ++v)
        for (int j = 0; j < seg[v] && g < virt.cap; j += kVirtualTokens) {
          virt.expert[g] = v % L.per;
          virt.row0[g] = seg[kEpMaxSegments + v] + j;
          virt.count[g] = min(kVirtualTokens, seg[v] - j);
          virt.out[g] = seg_ptr[v] + (size_t)j * L.H;
          ++g;
        }
      virt.n[0] = g;
    }
  }
}

__global__ void ep_signal_kernel(EpLayout L, EpPeers P, int kind, uint32_t epoch, int *ok_word, int *err,
                                 int code) {
  if (threadIdx.x == 0) raise_flags(L, P, kind, epoch, *(volatile const int *)ok_word != 0);
  __syncwarp();
  if (err && !wait_flags(L, P, kind, epoch, err, code) && threadIdx.x == 0) *ok_word = 0;
}

}  // namespace

EpLayout ep_layout(int W, int E, int H, int k, int rank, long long max_tokens, long long max_recv) {
  EpLayout L{};
  L.W = W;
  L.E = E;
  L.H = H;
  L.k = k;
  L.rank = rank;
  L.per = W > 0 ? E / W : 0;
  L.max_tokens = max_tokens;
  L.max_recv = max_recv;
  L.wait_cycles = kEpWaitCycles;
  auto up = [](size_t v) { return (v + 255) / 256 * 256; };
  size_t off = 0;
  L.off_flags = off;
  off = up(off + 3 * kEpMaxRanks * sizeof(uint32_t));
  L.off_inbox = off;
  off = up(off + (size_t)kEpMaxRanks * kEpMaxExperts * sizeof(int32_t));
  L.off_recv_scale = off;
  off = up(off + (size_t)max_recv * sizeof(float));
  L.off_recv_rows = off;
  off = up(off + (size_t)max_recv * H * 2);
  L.off_ret_rows = off;
  off = up(off + (size_t)max_tokens * k * H * sizeof(float));
  L.bytes = off;
  return L;
}

cudaError_t launch_ep_counts(const EpLayout &L, const EpPeers &P, const int32_t *cta_hist, int n_cta,
                             int32_t *counts, int32_t *offsets, int *ok_word, uint32_t epoch, int *err,
                             int code, cudaStream_t stream) {
  ep_counts_kernel<<<1, 256, 0, stream>>>(L, P, cta_hist, n_cta, counts, offsets, ok_word, epoch, err, code);
  return cudaGetLastError();
}

cudaError_t launch_ep_scatter(const EpLayout &L, const EpPeers &P, const int32_t *cta_hist, int n_cta,
                              const int32_t *idx, const int32_t *local_rank, int T, const uint16_t *x,
                              const int32_t *sigma, int32_t *slot_pos, uint32_t *done_ctr,
                              int *ok_word, int *err, uint32_t epoch, cudaStream_t stream) {
  if (T == 0) return cudaSuccess;
  if (n_cta != (T + kEpTokens - 1) / kEpTokens || L.H % 8 || ((uintptr_t)x & 15))
    return cudaErrorInvalidValue;
  ep_scatter_kernel<<<n_cta * kEpSub, kEpThreads, 0, stream>>>(L, P, cta_hist, n_cta, idx, local_rank,
                                                                T, x, sigma, slot_pos, done_ctr, ok_word,
                                                                err, epoch);
  return cudaGetLastError();
}

cudaError_t launch_ep_segments(const EpLayout &L, const EpPeers &P, uint32_t epoch, int *err,
                               int *ok_word, int32_t *seg, float **seg_ptr, const EpVirtual &virt,
                               cudaStream_t stream) {
  ep_segments_kernel<<<1, 256, 0, stream>>>(L, P, epoch, err, ok_word, seg, seg_ptr, virt);
  return cudaGetLastError();
}

cudaError_t launch_ep_signal(const EpLayout &L, const EpPeers &P, int kind, uint32_t epoch, int *ok_word,
                             int *err, int code, cudaStream_t stream) {
  ep_signal_kernel<<<1, 32, 0, stream>>>(L, P, kind, epoch, ok_word, err, code);
  return cudaGetLastError();
}

}  // namespace oxg
