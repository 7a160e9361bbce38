// relayout.cu — upload-time re-layout of packed MXFP4 expert weights.
//
// Checkpoint order (gpt-oss "*.blocks"/"*.scales", the layout the reference's
// loader reads, src/loader.rs:42-73): row-major codes [rows, K/2] with the low
// nibble holding the even element, and E8M0 scales [rows, K/32].
//
// Device order used by the f16 MoE kernels ("tile chunks"): the rows are cut
// into tiles of 16 and each tile's K into groups of 4 blocks (128 elements);
// a trailing group of w = nb % 4 blocks is narrower. Every (tile, group) is one
// contiguous chunk, tiles one after another, so a 16-row tile streams as one
// run of item_bytes = full * 1088 + (w ? 256 w + 64 : 0) bytes:
//   codes: 2 parts x 32 lanes x (4 w) bytes. Tile row lr belongs to part p and
//          lane row g by the matrix's row pairing (gate/up interleaved mlp1:
//          lr = 2g + p; mlp2: lr = 8p + g). Lane (g, q) of part p holds word q
//          (elements 8q..8q+7) of each block b of its row at
//          p * 128 w + (4g + q) * 4 w + 4 b, so one 16-byte copy per lane and
//          part fetches exactly the operands of an m16n8k16 A fragment pair.
//   scales: after the codes, 64 bytes: the row's block scales at
//          p * 32 + 4 g + b (bytes b >= w of a narrow group are zero).
// Bytes are only moved (plus zero padding), never changed.
#include "common.cuh"
#include "kernels.h"

namespace oxg {
namespace {

__device__ __forceinline__ void tile_row(int lr, int pair_adj, int &p, int &g) {
  p = pair_adj ? (lr & 1) : (lr >> 3);
  g = pair_adj ? (lr >> 1) : (lr & 7);
}

__global__ void tile_codes_kernel(const uint32_t *__restrict__ src, uint8_t *__restrict__ dst,
                                  size_t rows, int K, int pair_adj) {
  const int words_per_row = K / 8, nb = K / 32, full = nb / 4, tail = nb % 4;
  const size_t item_bytes = tile_item_bytes(K);
  const size_t total = rows * (size_t)words_per_row;
  const size_t stride = (size_t)gridDim.x * blockDim.x;
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += stride) {
    const size_t row = i / words_per_row;
    const int wi = (int)(i % words_per_row);  // source word index in the row
    const int grp = wi / 16, inner = wi % 16;
    const int b = inner / 4, q = inner % 4;  // word q of block b
    const int w = grp < full ? 4 : tail;
    int p, g;
    tile_row((int)(row & 15), pair_adj, p, g);
    const size_t o = (row >> 4) * item_bytes + (size_t)grp * 1088 + p * 128 * w + (4 * g + q) * 4 * w + 4 * b;
    *reinterpret_cast<uint32_t *>(dst + o) = src[i];
  }
}

__global__ void tile_scales_kernel(const uint8_t *__restrict__ src, uint8_t *__restrict__ dst,
                                   size_t rows, int K, int pair_adj) {
  const int nb = K / 32, full = nb / 4, tail = nb % 4, nb_pad = (nb + 3) / 4 * 4;
  const size_t item_bytes = tile_item_bytes(K);
  const size_t total = rows * (size_t)nb_pad;
  const size_t stride = (size_t)gridDim.x * blockDim.x;
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += stride) {
    const size_t row = i / nb_pad;
    const int j = (int)(i % nb_pad), grp = j / 4, b = j % 4;
    const int w = grp < full ? 4 : tail;
    int p, g;
    tile_row((int)(row & 15), pair_adj, p, g);
    const size_t o = (row >> 4) * item_bytes + (size_t)grp * 1088 + 256 * w + p * 32 + 4 * g + b;
    dst[o] = j < nb ? src[row * nb + j] : (uint8_t)0;
  }
}

unsigned grid_for(size_t n) {
  size_t g = (n + 255) / 256;
  return (unsigned)(g < 148 * 32 ? (g ? g : 1) : 148 * 32);
}

}  // namespace

cudaError_t launch_tile_weights(const uint8_t *codes, const uint8_t *scales, uint8_t *dst,
                                size_t rows, int K, int pair_adj, cudaStream_t stream) {
  if (K % 32 || rows % 16) return cudaErrorInvalidValue;
  if (rows == 0) return cudaSuccess;
  if (codes)
    tile_codes_kernel<<<grid_for(rows * (K / 8)), 256, 0, stream>>>(
        reinterpret_cast<const uint32_t *>(codes), dst, rows, K, pair_adj);
  if (scales) {
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    tile_scales_kernel<<<grid_for(rows * ((K / 32 + 3) / 4 * 4)), 256, 0, stream>>>(scales, dst, rows, K,
                                                                                 pair_adj);
  }
  return cudaGetLastError();
}

}  // namespace oxg
