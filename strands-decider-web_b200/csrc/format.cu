// Non-default weight formats and the online Hadamard rotation of `had` tensors.
//
// Formats (web/public/gemmbench/kernels.js:5-12, engine.js:36 fmtOf): a block of 32 consecutive K
// values of one output row takes `bits` u32 words --
//   4 bits: element e at bits 4(e%8) of word e/8 (MatMulNBits),
//   2 bits: element e at bits 2(e%16) of word e/16,
//   3 bits: words 0-1 hold the low two bits as in the 2-bit layout, bit e of word 2 is the high bit,
// with one fp16 scale per `group` (32 or 64) values, [N][K/group]. Symmetric: w = (q - 2^(bits-1)) s.
// A symmetric 2- or 3-bit value is an int4 one with the same scale (q4 = q - 2^(bits-1) + 8 in
// [4, 11]) and a group-64 scale is the scale of both of its 32-blocks, so upload rewrites those
// formats into MatMulNBits bytes and [N][K/32] scales exactly, and every kernel family runs them.
// Asymmetric (w = q s + b, fp16 bias per group): q is kept uncentered as a nibble in [0, 2^bits) and
// scales and biases are spread to [N][K/32]; the kernels dequantise fma(q, s, b) in fp16.
//
// FWHT (wgsl.js:94-110, engine.js:238): each contiguous n-block of the activations is replaced by
// its orthonormal Walsh-Hadamard transform, in place, in fp32: stages h = 1, 2, 4, ... < n turn the
// pair (i, i+h), i = (p / h) 2h + p % h, into (x + y, x - y); the result times 1/sqrt(n) (as a
// float) is rounded to fp16. The same operations in the same order as the reference's shader. Blocks
// of 32..1024 elements take one warp each (registers and shuffles); others one CTA (shared memory).
#include "common.cuh"

namespace s4 {

__global__ void transcode_kernel(const uint32_t* __restrict__ q, const __half* __restrict__ scales,
                                 const __half* __restrict__ bias, int N, int blocks, int bits, int gper,
                                 uint32_t* __restrict__ out4, __half* __restrict__ out_s, __half* __restrict__ out_b) {
  const int64_t total = (int64_t)N * blocks;
  const uint32_t zero = bias ? 8u : 1u << (bits - 1);  // asymmetric: q stays uncentered
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const uint32_t* w = q + i * bits;
    uint32_t o[4] = {0, 0, 0, 0};
    if (bits == 4) {
#pragma unroll
      for (int j = 0; j < 4; ++j) o[j] = w[j];
    } else {
      const uint32_t lo0 = w[0], lo1 = w[1], hi = bits == 3 ? w[2] : 0u;
#pragma unroll
      for (int e = 0; e < 32; ++e) {
        uint32_t v = ((e < 16 ? lo0 : lo1) >> (2 * (e & 15))) & 3u;
        if (bits == 3) v |= ((hi >> e) & 1u) << 2;
        o[e >> 3] |= (v + 8u - zero) << (4 * (e & 7));
      }
    }
    uint4 ov = make_uint4(o[0], o[1], o[2], o[3]);
    reinterpret_cast<uint4*>(out4)[i] = ov;
    const int64_t n = i / blocks;
    const int b = (int)(i - n * blocks);
    const int64_t gi = n * (blocks / gper) + b / gper;
    out_s[i] = scales[gi];
    if (bias) out_b[i] = bias[gi];
  }
}

// Native 2-bit decode layout (symmetric 2-bit weights): per (n-block, k-tile) chunk 2048 bytes =
// [8 sub-tiles][32 lanes][2 u32]. Lane L = 4g + t of sub-tile s holds word h (row nb*128 + 16s + g + 8h)
// for both 32-blocks of the k-tile: value i (K = kt*64 + 32*blk + 8t + i) of block blk sits at bits
// 8*blk + 2*(i/2) for even i and 16 + 8*blk + 2*(i/2) for odd i, so one shift and a 0x00030003-style
// mask put the pair (i, i + 1) in the two halves of a half2 (the GEMV's fragment order, as the int4
// layout's nibble shuffle does). Rows >= N and blocks >= K/32 hold 2, the zero weight.
__global__ void repack2_kernel(const uint32_t* __restrict__ q, int N, int blocks, int nblk, int ktiles,
                               uint32_t* __restrict__ out) {
  const int64_t words = (int64_t)nblk * ktiles * 512;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < words; i += (int64_t)gridDim.x * blockDim.x) {
    const int h = (int)(i & 1);
    const int lane = (int)((i >> 1) & 31);
    const int sub = (int)((i >> 6) & 7);
    const int64_t chunk = i >> 9;
    const int kt = (int)(chunk % ktiles);
    const int nb = (int)(chunk / ktiles);
    const int g = lane >> 2, t = lane & 3;
    const int r = nb * 128 + sub * 16 + g + 8 * h;
    uint32_t o = 0;
#pragma unroll
    for (int blk = 0; blk < 2; ++blk) {
      const int b = kt * 2 + blk;
      const bool in = r < N && b < blocks;
      const uint32_t w = in ? q[((int64_t)r * blocks + b) * 2 + (t >> 1)] : 0u;
#pragma unroll
      for (int v = 0; v < 8; ++v) {
        const int e = 8 * t + v;  // position in the 32-block
        const uint32_t val = in ? (w >> (2 * (e & 15))) & 3u : 2u;
        o |= val << ((v & 1) * 16 + 8 * blk + 2 * (v >> 1));
      }
    }
    out[i] = o;
  }
}

cudaError_t launch_repack2(const uint32_t* q, int N, int K, int nblk, int ktiles, uint8_t* out, int sm_count,
                           cudaStream_t stream) {
  const int64_t words = (int64_t)nblk * ktiles * 512;
  int64_t want = (words + 255) / 256;
  int grid = (int)(want < (int64_t)sm_count * 16 ? want : (int64_t)sm_count * 16);
  if (grid < 1) grid = 1;
  repack2_kernel<<<grid, 256, 0, stream>>>(q, N, K / 32, nblk, ktiles, reinterpret_cast<uint32_t*>(out));
  return cudaGetLastError();
}

cudaError_t launch_transcode(const uint32_t* q, const __half* scales, const __half* bias, int N, int K, int bits,
                             int group, uint8_t* packed4, __half* scales32, __half* bias32, int sm_count,
                             cudaStream_t stream) {
  const int blocks = K / 32;
  const int64_t total = (int64_t)N * blocks;
  const int64_t want = (total + 255) / 256;
  const int grid = (int)(want < (int64_t)sm_count * 8 ? (want < 1 ? 1 : want) : (int64_t)sm_count * 8);
  transcode_kernel<<<grid, 256, 0, stream>>>(q, scales, bias, N, blocks, bits, group / 32,
                                              reinterpret_cast<uint32_t*>(packed4), scales32, bias32);
  return cudaGetLastError();
}

__global__ void fwht_kernel(__half* __restrict__ a, int n, float c) {
  extern __shared__ float fw_sh[];
  pdl_wait();
  const int64_t o = (int64_t)blockIdx.x * n;
  for (int e = threadIdx.x; e < n; e += blockDim.x) fw_sh[e] = __half2float(a[o + e]);
  __syncwarp();  // each warp reaches the (warp-aligned) block barrier as a whole
  __syncthreads();
  for (int h = 1; h < n; h <<= 1) {
    for (int p = threadIdx.x; p < n / 2; p += blockDim.x) {
      const int i = (p / h) * 2 * h + p % h;
      const float x = fw_sh[i], y = fw_sh[i + h];
      fw_sh[i] = __fadd_rn(x, y);
      fw_sh[i + h] = __fsub_rn(x, y);
    }
    __syncwarp();
    __syncthreads();
  }
  pdl_launch_dependents();
  for (int e = threadIdx.x; e < n; e += blockDim.x) a[o + e] = __float2half_rn(__fmul_rn(fw_sh[e], c));
}

// n = 32 E (E = 1 .. 32): one warp per block, lane l holding elements [l E, l E + E) in registers.
// Stages h < E pair registers of one lane; stages h >= E pair lane l with lane l ^ (h / E), the
// lower lane keeping x + y and the upper x - y (its own value is y): the same operations on the
// same operands as the shared-memory form, so the same bits.
template <int E>
__global__ void fwht_warp_kernel(__half* __restrict__ a, int64_t blocks, float c) {
  const int lane = threadIdx.x & 31;
  const int64_t blk = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  pdl_wait();
  if (blk >= blocks) return;
  __half* p = a + blk * (32 * E) + lane * E;
  float v[E];
  if constexpr (E >= 8) {
#pragma unroll
    for (int q = 0; q < E / 8; ++q) {
      const uint4 u = reinterpret_cast<const uint4*>(p)[q];
      const __half2* h2 = reinterpret_cast<const __half2*>(&u);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 f = __half22float2(h2[j]);
        v[8 * q + 2 * j] = f.x;
        v[8 * q + 2 * j + 1] = f.y;
      }
    }
  } else {
#pragma unroll
    for (int e = 0; e < E; ++e) v[e] = __half2float(p[e]);
  }
#pragma unroll
  for (int h = 1; h < E; h <<= 1) {
#pragma unroll
    for (int i = 0; i < E; ++i)
      if ((i & h) == 0) {
        const float x = v[i], y = v[i + h];
        v[i] = __fadd_rn(x, y);
        v[i + h] = __fsub_rn(x, y);
      }
  }
#pragma unroll
  for (int m = 1; m < 32; m <<= 1) {
    const bool upper = (lane & m) != 0;
#pragma unroll
    for (int i = 0; i < E; ++i) {
      const float o = __shfl_xor_sync(0xffffffffu, v[i], m);
      v[i] = upper ? __fsub_rn(o, v[i]) : __fadd_rn(v[i], o);
    }
  }
  pdl_launch_dependents();
  if constexpr (E >= 8) {
#pragma unroll
    for (int q = 0; q < E / 8; ++q) {
      uint4 u;
      __half2* h2 = reinterpret_cast<__half2*>(&u);
#pragma unroll
      for (int j = 0; j < 4; ++j)
        h2[j] = __floats2half2_rn(__fmul_rn(v[8 * q + 2 * j], c), __fmul_rn(v[8 * q + 2 * j + 1], c));
      reinterpret_cast<uint4*>(p)[q] = u;
    }
  } else {
#pragma unroll
    for (int e = 0; e < E; ++e) p[e] = __float2half_rn(__fmul_rn(v[e], c));
  }
}

template <int E>
static cudaError_t launch_fwht_warp(__half* a, int64_t blocks, float c, cudaStream_t stream) {
  const int warps = 8;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)((blocks + warps - 1) / warps), 1, 1);
  cfg.blockDim = dim3(32 * warps, 1, 1);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, fwht_warp_kernel<E>, a, blocks, c);
}

cudaError_t launch_fwht(__half* a, int64_t blocks, int n, cudaStream_t stream) {
  const float c = (float)(1.0 / sqrt((double)n));
  const bool aligned16 = (reinterpret_cast<uintptr_t>(a) & 15) == 0;
  switch (n) {
    case 32: return launch_fwht_warp<1>(a, blocks, c, stream);
    case 64: return launch_fwht_warp<2>(a, blocks, c, stream);
    case 128: return launch_fwht_warp<4>(a, blocks, c, stream);
    case 256: if (aligned16) return launch_fwht_warp<8>(a, blocks, c, stream); break;
    case 512: if (aligned16) return launch_fwht_warp<16>(a, blocks, c, stream); break;
    case 1024: if (aligned16) return launch_fwht_warp<32>(a, blocks, c, stream); break;
    default: break;
  }
  const size_t smem = (size_t)n * sizeof(float);
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(fwht_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)blocks, 1, 1);
  cfg.blockDim = dim3(n / 2 < 256 ? (n / 2 < 32 ? 32 : n / 2) : 256, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, fwht_kernel, a, n, c);
}

}  // namespace s4
