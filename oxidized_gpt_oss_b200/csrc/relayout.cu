// relayout.cu — upload-time re-layout of packed MXFP4 expert weights.
//
// Checkpoint order (gpt-oss "*.blocks"/"*.scales", the layout the reference's
// loader reads, src/loader.rs:42-73): row-major codes [rows, K/2] with the low
// nibble holding the even element, and E8M0 scales [rows, K/32].
//
// Device order used by the MoE kernels ("word-transposed"):
//   * codes: each row is cut into groups of 4 blocks (128 elements, 64 bytes,
//     16 four-byte words). Word q of block b inside a group moves to position
//     4*q + b, so the 16 bytes that tensor-core lane q of a quad needs from all
//     four blocks (elements 8q..8q+7 of each) are contiguous and one 16-byte
//     load fetches them. A trailing partial group of nb < 4 blocks uses
//     position nb*q + b. Element order inside a word is unchanged.
//   * scales: each row padded from K/32 to round_up(K/32, 4) bytes (zeros), so
//     the four scales of a group are one aligned 4-byte load.
// Bytes are only moved, never changed: the transform is exactly invertible.
#include "common.cuh"
#include "kernels.h"

namespace oxg {
namespace {

__global__ void relayout_codes_kernel(const uint32_t *__restrict__ src, uint32_t *__restrict__ dst,
                                      size_t rows, int words_per_row, int nb) {
  const size_t total = rows * (size_t)words_per_row;
  const size_t stride = (size_t)gridDim.x * blockDim.x;
  const int full_groups = nb / 4;
  const int tail = nb % 4;
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += stride) {
    const size_t row = i / words_per_row;
    const int wi = (int)(i % words_per_row);  // source word index in the row
    const int grp = wi / 16, inner = wi % 16;
    const int b = inner / 4, q = inner % 4;
    const int width = grp < full_groups ? 4 : tail;
    const int dpos = grp * 16 + q * width + b;
    dst[row * words_per_row + dpos] = src[i];
  }
}

__global__ void pad_scales_kernel(const uint8_t *__restrict__ src, uint8_t *__restrict__ dst,
                                  size_t rows, int nb, int nb_pad) {
  const size_t total = rows * (size_t)nb_pad;
  const size_t stride = (size_t)gridDim.x * blockDim.x;
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += stride) {
    const size_t row = i / nb_pad;
    const int c = (int)(i % nb_pad);
    dst[i] = c < nb ? src[row * nb + c] : (uint8_t)0;
  }
}

unsigned grid_for(size_t n) {
  size_t g = (n + 255) / 256;
  return (unsigned)(g < 148 * 32 ? (g ? g : 1) : 148 * 32);
}

}  // namespace

cudaError_t launch_relayout_codes(const uint8_t *src, uint8_t *dst, size_t rows, int K,
                                  cudaStream_t stream) {
  if (K % 32) return cudaErrorInvalidValue;
  if (rows == 0) return cudaSuccess;
  const int words_per_row = K / 8;
  relayout_codes_kernel<<<grid_for(rows * words_per_row), 256, 0, stream>>>(
      reinterpret_cast<const uint32_t *>(src), reinterpret_cast<uint32_t *>(dst), rows,
      words_per_row, K / 32);
  return cudaGetLastError();
}

cudaError_t launch_pad_scales(const uint8_t *src, uint8_t *dst, size_t rows, int K,
                              cudaStream_t stream) {
  if (K % 32) return cudaErrorInvalidValue;
  if (rows == 0) return cudaSuccess;
  const int nb = K / 32, nb_pad = (nb + 3) / 4 * 4;
  pad_scales_kernel<<<grid_for(rows * nb_pad), 256, 0, stream>>>(src, dst, rows, nb, nb_pad);
  return cudaGetLastError();
}

}  // namespace oxg
