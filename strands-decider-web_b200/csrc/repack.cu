// Upload-time repack of MatMulNBits int4 weights into the B200 tiled layout.
//
// Input (convert/export_engine.py:24, kernels.js:1-3): packed[N][K/32][16] bytes, element 2i of
// a 32-block in the low nibble of byte i; scales[N][K/32] fp16.
//
// Output, per (n-block nb of 128 rows, k-tile kt of 64 K) "chunk", contiguous in nb-major order:
//   wq: 4096 bytes = [8 sub-tiles of 16 rows][32 lanes][4 u32]
//       lane L = 4g + t, word j = 2*blk + h holds row nb*128 + sub*16 + g + 8h,
//       K = kt*64 + blk*32 + 8t .. +8, nibble-shuffled (k0,k2,k4,k6 low; k1,k3,k5,k7 high)
//   ws:  512 bytes = [8 sub][8 g][4 halves] = scales of (g,blk0), (g+8,blk0), (g,blk1), (g+8,blk1)
// A warp of the decode GEMV reads one sub-tile as one coalesced 512-byte line whose 16-byte lane
// slices are exactly its mma.sync fragments; the tcgen05 GEMM reads whole 4 KB chunks with one
// bulk copy. Rows >= N and K >= K are padded with nibble 8 (weight 0) and scale 0. With wq == nullptr
// only the scale pass runs (the biases of an asymmetric format take the layout of the scales).
// glu_I > 0: the input is a fused gate|up weight of 2 * glu_I rows (gate rows, then up rows) and
// n-block b takes gate rows 64b .. 64b+63 followed by the up rows of the same features, so one
// 128-row tile holds both halves of 64 SiLU*mul outputs.
__device__ __forceinline__ int repack_src_row(int r, int glu_I) {
  if (glu_I <= 0) return r;
  const int b = r >> 7, i = r & 127;
  return i < 64 ? 64 * b + i : glu_I + 64 * b + (i - 64);
}
#include "common.cuh"

namespace s4 {

__device__ __forceinline__ uint32_t shuffle_nibbles(uint32_t w) {
  // nibble i of w is k_i; even k to nibbles 0..3, odd k to nibbles 4..7
  uint32_t out = 0;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const uint32_t nib = (w >> (4 * i)) & 15u;
    const int pos = (i & 1) ? 4 + (i >> 1) : (i >> 1);
    out |= nib << (4 * pos);
  }
  return out;
}

__global__ void repack_weights_kernel(const uint8_t* __restrict__ packed, const __half* __restrict__ scales,
                                      uint32_t* __restrict__ wq, __half* __restrict__ ws, int N, int K, int nblk,
                                      int ktiles, int glu_I) {
  const int64_t words = wq ? (int64_t)nblk * ktiles * 1024 : 0;  // 4096 B per chunk; none for a bias-only pass
  const int blocks_per_row = K / 32;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < words; i += (int64_t)gridDim.x * blockDim.x) {
    const int j = (int)(i & 3);
    const int lane = (int)((i >> 2) & 31);
    const int sub = (int)((i >> 7) & 7);
    const int64_t chunk = i >> 10;
    const int kt = (int)(chunk % ktiles);
    const int nb = (int)(chunk / ktiles);
    const int g = lane >> 2, t = lane & 3, blk = j >> 1, h = j & 1;
    const int r = nb * 128 + sub * 16 + g + 8 * h;
    const int k0 = kt * 64 + blk * 32 + 8 * t;
    uint32_t v = 0x88888888u;
    if (r < N && k0 < K) {
      const uint8_t* row = packed + (int64_t)repack_src_row(r, glu_I) * blocks_per_row * 16;
      v = *reinterpret_cast<const uint32_t*>(row + k0 / 2);
      v = shuffle_nibbles(v);
    }
    wq[i] = v;
  }
  const int64_t halves = (int64_t)nblk * ktiles * 256;  // 512 B per chunk
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < halves; i += (int64_t)gridDim.x * blockDim.x) {
    const int q = (int)(i & 3);
    const int g = (int)((i >> 2) & 7);
    const int sub = (int)((i >> 5) & 7);
    const int64_t chunk = i >> 8;
    const int kt = (int)(chunk % ktiles);
    const int nb = (int)(chunk / ktiles);
    const int blk = q >> 1, h = q & 1;
    const int r = nb * 128 + sub * 16 + g + 8 * h;
    const int b = kt * 2 + blk;
    __half s = __ushort_as_half((unsigned short)0);
    if (r < N && b < blocks_per_row) s = scales[(int64_t)repack_src_row(r, glu_I) * blocks_per_row + b];
    ws[i] = s;
  }
}

cudaError_t launch_repack(const uint8_t* packed, const __half* scales, uint32_t* wq, __half* ws, int N, int K,
                          int nblk, int ktiles, int sm_count, cudaStream_t stream, int glu_I) {
  const int64_t words = (int64_t)nblk * ktiles * 1024;
  int64_t want = (words + 255) / 256;
  int grid = (int)(want < (int64_t)sm_count * 16 ? want : (int64_t)sm_count * 16);
  if (grid < 1) grid = 1;
  repack_weights_kernel<<<grid, 256, 0, stream>>>(packed, scales, wq, ws, N, K, nblk, ktiles, glu_I);
  return cudaGetLastError();
}

}  // namespace s4
