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
#include "mxf.cuh"

namespace oxg {
namespace {

constexpr int kPermThreads = 1024;
constexpr int kPermMaxExperts = 256;

__global__ void __launch_bounds__(kPermThreads) permute_kernel(
    const int32_t *__restrict__ idx, int n_slots, int E, int32_t *__restrict__ counts,
    int32_t *__restrict__ offsets, int32_t *__restrict__ perm, int32_t *__restrict__ slot_pos, int pad) {
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
      run += (hist[e] + pad - 1) / pad * pad;
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
// One token row x (bf16, H elements, 16-byte aligned) as the block-scaled
// operand row p: two E4M3 terms in planes xq and xq + plane (row stride H)
// and their scale bytes in the atoms of row tile p / 128 (planes xsf and
// xsf + sf_plane); blocks past H in the last 128-wide k-tile get scale 0.
// One warp; a 32-element block is 4 lanes' 8-element chunks.
__device__ __forceinline__ void stage_row_e4m3(const uint16_t *__restrict__ src, uint8_t *__restrict__ xq,
                                               size_t plane, uint8_t *__restrict__ xsf, size_t sf_plane,
                                               int p, int H, int lane) {
  const int nch = H / 8, k_tiles = (H + mxf::kTileK - 1) / mxf::kTileK;
  const uint4 *s4 = reinterpret_cast<const uint4 *>(src);
  uint8_t *arow = xsf + (size_t)(p >> 7) * k_tiles * mxf::kAtomBytes;
  for (int c0 = 0; c0 < nch; c0 += 32) {
    const int c = c0 + lane;
    const bool ok = c < nch;
    const uint4 v = ok ? s4[c] : make_uint4(0u, 0u, 0u, 0u);
    const uint32_t w4[4] = {v.x, v.y, v.z, v.w};
    uint32_t mx = 0u;
#pragma unroll
    for (int u = 0; u < 4; ++u) mx = max(mx, max((w4[u] << 16) & 0x7FFFFFFFu, w4[u] & 0x7FFF0000u));
    mx = max(mx, __shfl_xor_sync(0xFFFFFFFFu, mx, 1));
    mx = max(mx, __shfl_xor_sync(0xFFFFFFFFu, mx, 2));
    if (!ok) continue;
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
    *reinterpret_cast<uint2 *>(xq + (size_t)p * H + 8 * c) = make_uint2(hi[0], hi[1]);
    *reinterpret_cast<uint2 *>(xq + plane + (size_t)p * H + 8 * c) = make_uint2(lo[0], lo[1]);
    if ((c & 3) == 0) {
      const int kb = c >> 2;
      const size_t o = (size_t)(kb >> 2) * mxf::kAtomBytes + mxf::atom_offset(p & 127, kb & 3);
      arow[o] = (uint8_t)sb;
      arow[sf_plane + o] = (uint8_t)(sb - 5);
    }
  }
  for (int kb = H / 32 + lane; kb < 4 * k_tiles; kb += 32) {
    const size_t o = (size_t)(kb >> 2) * mxf::kAtomBytes + mxf::atom_offset(p & 127, kb & 3);
    arow[o] = 0;
    arow[sf_plane + o] = 0;
  }
}

constexpr int kScatterSub = 4;
constexpr int kScatterThreads = 256;
constexpr int kScatterTokens = 64;  // tokens per router CTA
constexpr int kScatterMaxE = 64;

__global__ void __launch_bounds__(kScatterThreads) scatter_kernel(
    const int32_t *__restrict__ cta_hist, int n_cta, const int32_t *__restrict__ idx,
    const int32_t *__restrict__ local_rank, int T, int k, int E, int32_t *__restrict__ counts,
    int32_t *__restrict__ offsets, int32_t *__restrict__ perm, int32_t *__restrict__ slot_pos,
    const uint16_t *__restrict__ x, const int32_t *__restrict__ sigma, int H,
    uint16_t *__restrict__ xp, float *__restrict__ pos_scale, int pad, uint8_t *__restrict__ xq,
    uint8_t *__restrict__ xsf, int rows_cap) {
  __shared__ int base_s[kScatterMaxE], tot_s[kScatterMaxE];
  __shared__ int part_s[2 * kScatterThreads];
  const int c = blockIdx.x / kScatterSub, sub = blockIdx.x % kScatterSub;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  hist_prefix<kScatterThreads>(cta_hist, n_cta, E, c, base_s, tot_s, part_s);
  if (threadIdx.x == 0) {
    int run = 0;
    for (int e = 0; e < E; ++e) {
      base_s[e] += run;
      if (blockIdx.x == 0) {
        counts[e] = tot_s[e];
        offsets[e] = run;
      }
      run += (tot_s[e] + pad - 1) / pad * pad;
    }
    if (blockIdx.x == 0) offsets[E] = run;
  }
  __syncthreads();
  const int s_begin = c * kScatterTokens * k;
  const int s_end = min(T, (c + 1) * kScatterTokens) * k;
  const int per = (kScatterTokens * k + kScatterSub - 1) / kScatterSub;
  const int my_begin = s_begin + sub * per, my_end = min(s_end, my_begin + per);
  // This warp's slots are my_begin + warp + W i (W warps). Their positions (and the
  // tokens' sigma) are fetched one slot per lane, all at once, before the rows
  // are staged one after another: one memory round trip of metadata per 32
  // slots instead of three per slot.
  const int n_mine = my_end - my_begin;
  constexpr int W = kScatterThreads / 32;
  const int n_w = n_mine > warp ? (n_mine - warp + W - 1) / W : 0;
  for (int i0 = 0; i0 < n_w; i0 += 32) {
    const int li = i0 + lane;
    const int sl_l = my_begin + warp + W * li;
    int p_l = 0, sg_l = 0;
    if (li < n_w) {
      const int e = idx[sl_l];
      p_l = base_s[e] + local_rank[sl_l];
      perm[p_l] = sl_l;
      slot_pos[sl_l] = p_l;
      if (xp) {
        sg_l = sigma[sl_l / k];
        pos_scale[p_l] = __uint_as_float((uint32_t)(127 + sg_l) << 23);
      }
    }
    const int n_here = min(32, n_w - i0);
    for (int j = 0; j < n_here; ++j) {
      const int p = __shfl_sync(0xFFFFFFFFu, p_l, j);
      const int sg = __shfl_sync(0xFFFFFFFFu, sg_l, j);
      const int t = (my_begin + warp + W * (i0 + j)) / k;
      if (xp) stage_row_f16(x + (size_t)t * H, xp + (size_t)p * H, H, sg, lane);
      if (xq) {
        const size_t sf_plane = (size_t)(rows_cap / 128) * ((H + 127) / 128) * mxf::kAtomBytes;
        stage_row_e4m3(x + (size_t)t * H, xq, (size_t)rows_cap * H, xsf, sf_plane, p, H, lane);
      }
    }
  }
}

}  // namespace

cudaError_t launch_permute(const int32_t *idx, int n_slots, int E, int32_t *counts,
                           int32_t *offsets, int32_t *perm, int32_t *slot_pos,
                           cudaStream_t stream, int pad) {
  if (E > kPermMaxExperts || E <= 0 || pad < 1) return cudaErrorInvalidValue;
  permute_kernel<<<1, kPermThreads, 0, stream>>>(idx, n_slots, E, counts, offsets, perm, slot_pos, pad);
  return cudaGetLastError();
}

namespace {
// The block-scaled prefill operand for routings sorted by permute_kernel
// (padded positions): a warp per slot.
__global__ void __launch_bounds__(256) gather_e4m3_kernel(const uint16_t *__restrict__ x,
                                                          const int32_t *__restrict__ slot_pos, int S, int k,
                                                          int H, uint8_t *__restrict__ xq, uint8_t *__restrict__ xsf,
                                                          int rows_cap) {
  const int lane = threadIdx.x & 31;
  const size_t sf_plane = (size_t)(rows_cap / 128) * ((H + 127) / 128) * mxf::kAtomBytes;
  for (int sl = blockIdx.x * 8 + (threadIdx.x >> 5); sl < S; sl += gridDim.x * 8) {
    const int p = slot_pos[sl];
    if (p < 0) continue;
    stage_row_e4m3(x + (size_t)(sl / k) * H, xq, (size_t)rows_cap * H, xsf, sf_plane, p, H, lane);
  }
}
}  // namespace

cudaError_t launch_gather_e4m3(const uint16_t *x, const int32_t *slot_pos, int S, int k, int H,
                               const ScatterTerms &terms, cudaStream_t stream) {
  if (S <= 0) return cudaSuccess;
  if (H % 32 || ((uintptr_t)x & 15) || ((uintptr_t)terms.xq & 15) || terms.rows_cap % 128)
    return cudaErrorInvalidValue;
  const int blocks = (S + 7) / 8 < 4096 ? (S + 7) / 8 : 4096;
  gather_e4m3_kernel<<<blocks, 256, 0, stream>>>(x, slot_pos, S, k, H, terms.xq, terms.xsf, terms.rows_cap);
  return cudaGetLastError();
}

cudaError_t launch_scatter(const int32_t *cta_hist, int n_cta, const int32_t *idx,
                           const int32_t *local_rank, int T, int k, int E, int32_t *counts,
                           int32_t *offsets, int32_t *perm, int32_t *slot_pos, const uint16_t *x,
                           const int32_t *sigma, int H, uint16_t *xp, float *pos_scale,
                           cudaStream_t stream, const ScatterTerms *terms) {
  if (T == 0) return cudaSuccess;
  if (E > kScatterMaxE || E <= 0 || n_cta != (T + kScatterTokens - 1) / kScatterTokens)
    return cudaErrorInvalidValue;
  if (xp && (H % 8 || ((uintptr_t)x & 15) || ((uintptr_t)xp & 15))) return cudaErrorInvalidValue;
  const int pad = terms ? 128 : 1;
  if (terms && (H % 32 || ((uintptr_t)x & 15) || ((uintptr_t)terms->xq & 15) || terms->rows_cap % 128 ||
                (size_t)T * k + (size_t)E * 127 > (size_t)terms->rows_cap))
    return cudaErrorInvalidValue;
  scatter_kernel<<<n_cta * kScatterSub, kScatterThreads, 0, stream>>>(
      cta_hist, n_cta, idx, local_rank, T, k, E, counts, offsets, perm, slot_pos, x, sigma, H, xp,
      pos_scale, pad, terms ? terms->xq : nullptr, terms ? terms->xsf : nullptr, terms ? terms->rows_cap : 0);
  return cudaGetLastError();
}

}  // namespace oxg
