// Weight layout converter: row-major bf16 [R, K] -> fragment-tiled bf16.
//
// Fragment-tiled ("FT") layout: the matrix is cut into units of 16 rows x 32 columns
// (1 KB).  Units are stored strip-major (16-row strip, then the 32-column tiles of that
// strip left to right), so each strip is one contiguous run that a single TMA bulk copy can
// move.  Inside a unit, the 16-byte word for (half h, lane l = 4*g + t) holds row
// 8*h + g, columns 8*t .. 8*t+7.  A warp then reads a unit with two conflict-free 128-bit
// shared loads per lane, and the two words are exactly the A fragments of two
// mma.m16n8k16 instructions once the k order inside each 32-column tile is permuted to
// {8t..8t+3} / {8t+4..8t+7} (the activation fragment uses the same permutation).
//
// NKM_PACK_GATE_UP: for Hugging Face experts gate_up [2I, K] (gate rows 0..I-1, up rows
// I..2I-1) strip s holds gate rows 8s..8s+7 in its first half and the matching up rows in
// its second half, so one thread of the mma owns gate and up of the same output.
#include <cuda_runtime.h>

#include <cstdint>

#include "nkimoe.h"

namespace {

__global__ void pack_ft_kernel(const uint4* __restrict__ src, uint4* __restrict__ dst, int64_t R, int64_t K,
                               int64_t count, int mode) {
  const int64_t per = R * K / 8;  // 16-byte words per matrix
  const int64_t total = per * count;
  const int64_t ktiles = K / 32;
  for (int64_t c = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; c < total;
       c += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t m = c / per, cu = c % per;
    const int64_t unit = cu / 64;
    const int inner = static_cast<int>(cu % 64);
    const int h = inner / 32, l = inner % 32, g = l / 4, t = l % 4;
    const int64_t rs = unit / ktiles, kt = unit % ktiles;
    int64_t row;
    if (mode == NKM_PACK_GATE_UP)
      row = (h == 0 ? 0 : R / 2) + 8 * rs + g;
    else
      row = 16 * rs + 8 * h + g;
    const int64_t col = 32 * kt + 8 * t;
    dst[c] = src[m * per + (row * K + col) / 8];
  }
}

}  // namespace

extern "C" int nkm_pack_ft(const void* src, void* dst, int64_t rows, int64_t cols, int64_t count, int32_t mode,
                           nkm_stream_t stream) {
  if (!src || !dst || rows <= 0 || cols <= 0 || count <= 0) return NKM_ERR_ARG;
  if (rows % 16 || cols % 32) return NKM_ERR_ARG;
  if (mode == NKM_PACK_GATE_UP && (rows / 2) % 8) return NKM_ERR_ARG;
  if (mode != NKM_PACK_PLAIN && mode != NKM_PACK_GATE_UP) return NKM_ERR_ARG;
  if ((reinterpret_cast<uintptr_t>(src) | reinterpret_cast<uintptr_t>(dst)) & 15u) return NKM_ERR_ARG;
  const int64_t total = rows * cols / 8 * count;
  int64_t blocks = (total + 255) / 256;
  if (blocks > 4096) blocks = 4096;
  pack_ft_kernel<<<static_cast<unsigned>(blocks), 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint4*>(src), static_cast<uint4*>(dst), rows, cols, count, mode);
  return cudaGetLastError() == cudaSuccess ? NKM_OK : NKM_ERR_CUDA;
}
