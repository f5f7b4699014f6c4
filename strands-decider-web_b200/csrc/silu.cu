// mid[t][j] = silu(big[t][j]) * big[t][I + j]  (web/public/engine/wgsl.js:81-90): fp16 in/out,
// fp32 math. Between the fused gate|up projection and the down projection of every layer
// (engine.js:279-280). HBM-bound elementwise pass: 6 bytes moved per output element.
#include "common.cuh"

namespace s4 {


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

namespace s4 {

// Column-sharded prefill: this GPU's gate|up slice big[M][2*Is] -> mid slice, written into every
// rank's gathered buffer dst[d][tok * ldd + col0 + j] (peer buffers over NVLink).
__device__ __forceinline__ void silu_mul_gather_body(const __half* __restrict__ big, int M, int Is,
                                                    __half* const* dsts, int ndst, int64_t ldd, int col0) {
  pdl_wait();
  pdl_launch_dependents();
  const int per_row = Is / 8;
  const int64_t total = (int64_t)M * per_row;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t t = i / per_row;
    const int j = (int)(i - t * per_row) * 8;
    const uint4 gv = *reinterpret_cast<const uint4*>(big + t * 2 * Is + j);
    const uint4 uv = *reinterpret_cast<const uint4*>(big + t * 2 * Is + Is + j);
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
    const int64_t off = t * ldd + col0 + j;
    for (int d = 0; d < ndst; ++d) *reinterpret_cast<uint4*>(dsts[d] + off) = ov;
  }
}

struct DstList {
  __half* p[8];
};

__global__ void silu_mul_gather_kernel_v(const __half* __restrict__ big, int M, int Is, DstList dsts, int ndst,
                                         int64_t ldd, int col0) {
  silu_mul_gather_body(big, M, Is, dsts.p, ndst, ldd, col0);
}

cudaError_t launch_silu_mul_gather(const __half* big, int M, int Is, __half* const* dst, int ndst, int64_t ldd, int col0,
                                   int sm_count, cudaStream_t stream) {
  if (Is % 8 || ldd % 8 || col0 % 8 || ndst < 1 || ndst > 8 || (reinterpret_cast<uintptr_t>(big) & 15))
    return cudaErrorInvalidValue;
  DstList dl = {};
  for (int d = 0; d < ndst; ++d) {
    if (reinterpret_cast<uintptr_t>(dst[d]) & 15) return cudaErrorInvalidValue;
    dl.p[d] = dst[d];
  }
  const int64_t work = (int64_t)M * (Is / 8);
  const int64_t blocks = (work + 255) / 256;
  const int64_t cap = (int64_t)sm_count * 8;
  const int grid = (int)(blocks < 1 ? 1 : (blocks > cap ? cap : blocks));
  silu_mul_gather_kernel_v<<<grid, 256, 0, stream>>>(big, M, Is, dl, ndst, ldd, col0);
  return cudaGetLastError();
}

}  // namespace s4
