// Residual add + zero-centred RMSNorm between the projections (ADD_NORM, web/public/engine/
// wgsl.js:55-78; called as in_norm / post_norm, engine.js:247, 255, 277): the residual stream x is
// fp32, y (the previous projection's output) fp16, the normalised h fp16:
//   x += y (optional);  h = f16(x * rsqrt(mean(x^2) + eps) * w)  (w is the stored 1 + weight)
// HBM-bound: one CTA per row, 256 threads, fp32 sum of squares reduced through shared memory.
// Algorithmic bytes per row: 4D read of x, 2D of y, 4D write of x (when y is given), 2D of h.
#include "common.cuh"

namespace s4 {

__device__ __forceinline__ float block_sum_256(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  float tot = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) tot += red[i];
  return tot;
}

// D % 1024 == 0, D <= 1024 * kNormMaxNV: the row stays in registers (NV float4 per thread, 16-byte x
// loads and stores, 8-byte y loads and h stores), so x is read once.
constexpr int kNormMaxNV = 8;

// wait_flags: y was gathered from wait_n ranks (column-sharded prefill): thread 0 waits for every
// rank's signal before the CTA reads y (a timeout sets err and the row is computed from what is there).
__device__ __forceinline__ void norm_peer_wait(const uint32_t* wait_flags, int wait_n, uint32_t* err) {
  if (!wait_flags) return;
  if (threadIdx.x == 0 && !peer_wait_all(wait_flags, wait_n)) set_error(err, kErrWaitTimeout);
  __syncthreads();
}

// y and h may be the same buffer (the projection's output normalised in place): every thread reads
// its elements of y before the block reduction and writes the same elements of h after it.
template <int NV>
__global__ void __launch_bounds__(256) add_rmsnorm_reg_kernel(float* __restrict__ x, const __half* y,
                                                              const float* __restrict__ w, int D, float eps,
                                                              __half* h, const uint32_t* wait_flags, int wait_n,
                                                              uint32_t* err) {
  pdl_wait();
  pdl_launch_dependents();
  norm_peer_wait(wait_flags, wait_n, err);
  __shared__ float red[8];
  const int64_t row = blockIdx.x;
  float4* xr = reinterpret_cast<float4*>(x + row * D);
  float4 v[NV];
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const int c4 = threadIdx.x + 256 * i;
    v[i] = xr[c4];
    if (y) {
      const uint2 yy = *reinterpret_cast<const uint2*>(y + row * D + 4 * c4);
      const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&yy.x));
      const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&yy.y));
      v[i].x += a.x;
      v[i].y += a.y;
      v[i].z += b.x;
      v[i].w += b.y;
      xr[c4] = v[i];
    }
    ss += v[i].x * v[i].x + v[i].y * v[i].y + v[i].z * v[i].z + v[i].w * v[i].w;
  }
  const float inv = rsqrtf(block_sum_256(ss, red) / (float)D + eps);
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const int c4 = threadIdx.x + 256 * i;
    const float4 g = w ? reinterpret_cast<const float4*>(w)[c4] : make_float4(1.f, 1.f, 1.f, 1.f);
    const __half2 lo = __floats2half2_rn(v[i].x * inv * g.x, v[i].y * inv * g.y);
    const __half2 hi = __floats2half2_rn(v[i].z * inv * g.z, v[i].w * inv * g.w);
    uint2 o;
    o.x = *reinterpret_cast<const uint32_t*>(&lo);
    o.y = *reinterpret_cast<const uint32_t*>(&hi);
    *reinterpret_cast<uint2*>(h + row * D + 4 * c4) = o;
  }
}

__global__ void __launch_bounds__(256) add_rmsnorm_kernel(float* __restrict__ x, const __half* y,
                                                          const float* __restrict__ w, int D, float eps, __half* h,
                                                          const uint32_t* wait_flags, int wait_n, uint32_t* err) {
  pdl_wait();
  pdl_launch_dependents();
  norm_peer_wait(wait_flags, wait_n, err);
  __shared__ float red[8];
  const int64_t row = blockIdx.x;
  float* xr = x + row * D;
  const __half* yr = y ? y + row * D : nullptr;
  float ss = 0.f;
  for (int c = threadIdx.x; c < D; c += 256) {
    float a = xr[c];
    if (yr) {
      a += __half2float(yr[c]);
      xr[c] = a;
    }
    ss += a * a;
  }
  const float inv = rsqrtf(block_sum_256(ss, red) / (float)D + eps);
  for (int c = threadIdx.x; c < D; c += 256) {
    const float a = xr[c];
    h[row * D + c] = __float2half_rn(a * inv * (w ? w[c] : 1.f));
  }
}

// The normalisation half of ADD_NORM when the residual add ran in the matmul's epilogue (the
// tcgen05 GEMM's residual mode): x already holds x + y, and ssp[g * ldss + row] the sum of squares of
// row's columns [32 g, 32 g + 32), g < D / 32. One CTA per row sums the groups (in a fixed order: the
// result does not depend on the GEMM's tile split beyond the per-group sums) and writes
// h = f16(x * rsqrt(sum / D + eps) * w). Algorithmic bytes per row: 4D read of x, 2D write of h.
__global__ void __launch_bounds__(256) rmsnorm_from_sums_kernel(const float* __restrict__ x,
                                                                const float* __restrict__ ssp, int64_t ldss,
                                                                const float* __restrict__ w, int D, float eps,
                                                                __half* __restrict__ h) {
  pdl_wait();
  pdl_launch_dependents();
  __shared__ float red[8];
  const int64_t row = blockIdx.x;
  float s = 0.f;
  for (int g = threadIdx.x; g < D / 32; g += 256) s += ssp[g * ldss + row];
  const float inv = rsqrtf(block_sum_256(s, red) / (float)D + eps);
  const float4* xr = reinterpret_cast<const float4*>(x + row * D);
  for (int c4 = threadIdx.x; c4 < D / 4; c4 += 256) {
    const float4 v = xr[c4];
    const float4 g = w ? reinterpret_cast<const float4*>(w)[c4] : make_float4(1.f, 1.f, 1.f, 1.f);
    const __half2 lo = __floats2half2_rn(v.x * inv * g.x, v.y * inv * g.y);
    const __half2 hi = __floats2half2_rn(v.z * inv * g.z, v.w * inv * g.w);
    uint2 o;
    o.x = *reinterpret_cast<const uint32_t*>(&lo);
    o.y = *reinterpret_cast<const uint32_t*>(&hi);
    *reinterpret_cast<uint2*>(h + row * D + 4 * c4) = o;
  }
}

// D % 32 == 0; x and w 16-byte aligned, h 8-byte aligned (checked by the caller)
cudaError_t launch_rmsnorm_from_sums(const float* x, const float* ssp, int64_t ldss, const float* w, int M, int D,
                                     float eps, __half* h, cudaStream_t stream, bool pdl) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(M, 1, 1);
  cfg.blockDim = dim3(256, 1, 1);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, rmsnorm_from_sums_kernel, x, ssp, ldss, w, D, eps, h);
}

cudaError_t launch_add_rmsnorm(float* x, const __half* y, const float* w, int M, int D, float eps, __half* h,
                               cudaStream_t stream, const uint32_t* wait_flags, int wait_n, uint32_t* err) {
  if (wait_flags && (wait_n < 1 || wait_n > 8)) return cudaErrorInvalidValue;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(M, 1, 1);
  cfg.blockDim = dim3(256, 1, 1);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const auto aligned = [](const void* p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) & (a - 1)) == 0; };
  const int nv = D / 1024;
  if (D % 1024 == 0 && nv <= kNormMaxNV && aligned(x, 16) && aligned(y, 8) && aligned(w, 16) && aligned(h, 8)) {
    switch (nv) {
      case 1: return cudaLaunchKernelEx(&cfg, add_rmsnorm_reg_kernel<1>, x, y, w, D, eps, h, wait_flags, wait_n, err);
      case 2: return cudaLaunchKernelEx(&cfg, add_rmsnorm_reg_kernel<2>, x, y, w, D, eps, h, wait_flags, wait_n, err);
      case 3: return cudaLaunchKernelEx(&cfg, add_rmsnorm_reg_kernel<3>, x, y, w, D, eps, h, wait_flags, wait_n, err);
      case 4: return cudaLaunchKernelEx(&cfg, add_rmsnorm_reg_kernel<4>, x, y, w, D, eps, h, wait_flags, wait_n, err);
      case 5: return cudaLaunchKernelEx(&cfg, add_rmsnorm_reg_kernel<5>, x, y, w, D, eps, h, wait_flags, wait_n, err);
      case 6: return cudaLaunchKernelEx(&cfg, add_rmsnorm_reg_kernel<6>, x, y, w, D, eps, h, wait_flags, wait_n, err);
      case 7: return cudaLaunchKernelEx(&cfg, add_rmsnorm_reg_kernel<7>, x, y, w, D, eps, h, wait_flags, wait_n, err);
      default: return cudaLaunchKernelEx(&cfg, add_rmsnorm_reg_kernel<8>, x, y, w, D, eps, h, wait_flags, wait_n, err);
    }
  }
  return cudaLaunchKernelEx(&cfg, add_rmsnorm_kernel, x, y, w, D, eps, h, wait_flags, wait_n, err);
}

}  // namespace s4
