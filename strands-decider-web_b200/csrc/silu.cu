// mid[t][j] = silu(big[t][j]) * big[t][I + j]  (web/public/engine/wgsl.js:81-90): fp16 in/out,
// fp32 math. Between the fused gate|up projection and the down projection of every layer
// (engine.js:279-280). HBM-bound elementwise pass: 6 bytes moved per output element.
#include "common.cuh"

namespace s4 {

__device__ __forceinline__ float silu_mul_f32(float g, float u) { return g / (1.0f + expf(-g)) * u; }

// Vector path: I % 8 == 0, one thread per 8 outputs (16-byte loads and stores).
__global__ void silu_mul_vec8_kernel(const __half* __restrict__ big, __half* __restrict__ mid, int M, int I) {
  pdl_wait();
  pdl_launch_dependents();
  const int per_row = I / 8;
  const int64_t total = (int64_t)M * per_row;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t t = i / per_row;
    const int j = (int)(i - t * per_row) * 8;
    const uint4 gv = *reinterpret_cast<const uint4*>(big + t * 2 * I + j);
    const uint4 uv = *reinterpret_cast<const uint4*>(big + t * 2 * I + I + j);
    const __half2* g2 = reinterpret_cast<const __half2*>(&gv);
    const __half2* u2 = reinterpret_cast<const __half2*>(&uv);
    uint4 ov;
    __half2* o2 = reinterpret_cast<__half2*>(&ov);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 g = __half22float2(g2[e]);
      const float2 u = __half22float2(u2[e]);
      o2[e] = __floats2half2_rn(silu_mul_f32(g.x, u.x), silu_mul_f32(g.y, u.y));
    }
    *reinterpret_cast<uint4*>(mid + t * I + j) = ov;
  }
}

__global__ void silu_mul_scalar_kernel(const __half* __restrict__ big, __half* __restrict__ mid, int M, int I) {
  pdl_wait();
  pdl_launch_dependents();
  const int64_t total = (int64_t)M * I;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t t = i / I;
    const int j = (int)(i - t * I);
    const float g = __half2float(big[t * 2 * I + j]);
    const float u = __half2float(big[t * 2 * I + I + j]);
    mid[i] = __float2half_rn(silu_mul_f32(g, u));
  }
}

cudaError_t launch_silu_mul(const __half* big, __half* mid, int M, int I, int sm_count, cudaStream_t stream) {
  const bool vec = (I % 8 == 0) && ((reinterpret_cast<uintptr_t>(big) & 15) == 0) &&
                   ((reinterpret_cast<uintptr_t>(mid) & 15) == 0);
  const int64_t work = vec ? (int64_t)M * (I / 8) : (int64_t)M * I;
  int64_t blocks = (work + 255) / 256;
  const int64_t cap = (int64_t)sm_count * 8;
  const int grid = (int)(blocks < 1 ? 1 : (blocks > cap ? cap : blocks));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid, 1, 1);
  cfg.blockDim = dim3(256, 1, 1);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (vec) return cudaLaunchKernelEx(&cfg, silu_mul_vec8_kernel, big, mid, M, I);
  return cudaLaunchKernelEx(&cfg, silu_mul_scalar_kernel, big, mid, M, I);
}

}  // namespace s4
