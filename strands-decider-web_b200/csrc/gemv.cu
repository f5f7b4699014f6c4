// Decode GEMV family (M <= 32): y[M][N] = x[M][K] @ W^T for int4 block-32 weights.
//
// Replaces kernelV1 (web/public/gemmbench/kernels.js:40-81), which the engine uses for M <= 8
// (engine.js:25), and the small-M end of kernelV4 + REDUCE (kernels.js:269-353).
//
// Design (HBM-bound: ~0.53 byte of weight per multiply-add at M = 1):
//  * stream-K: the weight is a contiguous run of 4.5 KB chunks (one n-block of 128 rows x one
//    k-tile of 64 K). CTA b of G owns chunks [b*T/G, (b+1)*T/G): every SM streams the same number
//    of bytes whatever the shape. One producer thread issues 1-D bulk copies (TMA engine) of all
//    its chunks into a ring of shared-memory slots at kernel start, before waiting on the
//    previous kernel (programmatic dependent launch), so weight traffic overlaps the previous
//    kernel's tail.
//  * 8 compute warps; warp w owns rows w*16..w*16+15 of every chunk. Its 512-byte slice of a
//    chunk is its mma.sync A fragments (weights as the 16-row operand, tokens as the 8 columns);
//    int4 is converted to exact fp16 (q - 8) and the per-block scale is applied in fp32 to the
//    fp32 block partial, so the only roundings are fp32 accumulation and the final fp16 store.
//  * segments of an n-block split across CTAs are combined deterministically: each CTA writes
//    its fp32 partial to context scratch, the last CTA to arrive (atomic ticket, no waiting)
//    sums all partials in CTA order and writes fp16. Tickets reset themselves.
#include "common.cuh"

namespace s4 {

struct GemvParams {
  const uint8_t* wq;     // repacked int4, chunk c at wq + c*4096
  const uint8_t* ws;     // repacked scales, chunk c at ws + c*512
  const __half* x;       // [M][K]
  __half* y;             // [M][N]
  float4* partials;      // [G][2][MG][8 warps][32 lanes] float4
  uint32_t* tickets;     // [nblk], zero between calls
  uint32_t* err;         // device error word
  int M, N, K;
  int nblk, ktiles;
  int total;             // nblk * ktiles
  int grid;              // G
  int token0;            // first token of this launch (tokens token0 .. token0 + 8*MG - 1)
};

constexpr int kGemvComputeWarps = 8;
constexpr int kGemvMaxCtasPerSm = 4;  // scratch is sized for this many CTAs per SM
constexpr int kGemvThreads = (kGemvComputeWarps + 1) * 32;
constexpr int kGemvSlots = 12;
constexpr int kSlotBytes = kChunkWBytes + kChunkSBytes;
constexpr size_t kGemvSmem = (size_t)kGemvSlots * kSlotBytes + 2 * kGemvSlots * sizeof(uint64_t) + 16;

__device__ __forceinline__ int chunk_begin(int b, int total, int grid) {
  return (int)(((int64_t)b * total) / grid);
}
// CTA whose range contains chunk c.
__device__ __forceinline__ int cta_of_chunk(int c, int total, int grid) {
  return (int)((((int64_t)c + 1) * grid - 1) / total);
}

template <int MG>
__device__ __forceinline__ void store_tile(const GemvParams& p, int nb, int warp, int lane, const float (&v)[MG][4]) {
  const int g = lane >> 2, t = lane & 3;
  const int n0 = nb * 128 + warp * 16 + g;
#pragma unroll
  for (int mg = 0; mg < MG; ++mg) {
    const int tok = p.token0 + mg * 8 + 2 * t;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int m = tok + (e & 1);
      const int n = n0 + ((e >> 1) << 3);
      if (m < p.M && n < p.N) p.y[(int64_t)m * p.N + n] = __float2half_rn(v[mg][e]);
    }
  }
}

template <int MG>
__device__ __forceinline__ void flush_segment(const GemvParams& p, int nb, int s0, int s1, int c0, float (&acc)[MG][4],
                                              int warp, int lane, int* s_flag) {
  const int KT = p.ktiles;
  if (s0 == nb * KT && s1 - s0 == KT) {  // whole n-block inside this CTA
    store_tile<MG>(p, nb, warp, lane, acc);
    return;
  }
  const int bid = blockIdx.x;
  const int sel = (s0 == c0) ? 0 : 1;
  float4* mine = p.partials + ((((int64_t)bid * 2 + sel) * MG) * kGemvComputeWarps + warp) * 32 + lane;
#pragma unroll
  for (int mg = 0; mg < MG; ++mg)
    __stcg(mine + (int64_t)mg * kGemvComputeWarps * 32, make_float4(acc[mg][0], acc[mg][1], acc[mg][2], acc[mg][3]));
  __threadfence();
  named_bar_sync(1, kGemvComputeWarps * 32);
  const int first = cta_of_chunk(nb * KT, p.total, p.grid);
  const int last = cta_of_chunk(nb * KT + KT - 1, p.total, p.grid);
  if (threadIdx.x == 0) {
    const uint32_t prev = atomicAdd(p.tickets + nb, 1u);
    *s_flag = (prev == (uint32_t)(last - first)) ? 1 : 0;
  }
  named_bar_sync(1, kGemvComputeWarps * 32);
  if (*s_flag) {
    __threadfence();
    float sum[MG][4];
#pragma unroll
    for (int mg = 0; mg < MG; ++mg)
#pragma unroll
      for (int e = 0; e < 4; ++e) sum[mg][e] = 0.f;
    for (int b = first; b <= last; ++b) {
      if (b == bid) {
#pragma unroll
        for (int mg = 0; mg < MG; ++mg)
#pragma unroll
          for (int e = 0; e < 4; ++e) sum[mg][e] += acc[mg][e];
      } else {
        const int bsel = (chunk_begin(b, p.total, p.grid) >= nb * KT) ? 0 : 1;
        const float4* src = p.partials + ((((int64_t)b * 2 + bsel) * MG) * kGemvComputeWarps + warp) * 32 + lane;
#pragma unroll
        for (int mg = 0; mg < MG; ++mg) {
          const float4 v = ldcg_f4(src + (int64_t)mg * kGemvComputeWarps * 32);
          sum[mg][0] += v.x;
          sum[mg][1] += v.y;
          sum[mg][2] += v.z;
          sum[mg][3] += v.w;
        }
      }
    }
    store_tile<MG>(p, nb, warp, lane, sum);
    named_bar_sync(1, kGemvComputeWarps * 32);
    if (threadIdx.x == 0) atomicExch(p.tickets + nb, 0u);
  }
}

template <int MG>
__device__ __forceinline__ void load_x(uint4 (&xv)[MG][2], const __half* const (&xr)[MG], const bool (&xok)[MG],
                                       int kbase, int K, bool kfull) {
#pragma unroll
  for (int mg = 0; mg < MG; ++mg)
#pragma unroll
    for (int blk = 0; blk < 2; ++blk) {
      const bool ok = xok[mg] && (kfull || kbase + blk * 32 < K);
      xv[mg][blk] = ok ? __ldg(reinterpret_cast<const uint4*>(xr[mg] + kbase + blk * 32)) : make_uint4(0, 0, 0, 0);
    }
}

template <int MG>
__global__ void __launch_bounds__(kGemvThreads, (MG == 1 ? 3 : (MG == 2 ? 2 : 1))) gemv_streamk_kernel(const GemvParams p) {
  extern __shared__ __align__(128) uint8_t smem[];
  uint8_t* slots = smem;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + (size_t)kGemvSlots * kSlotBytes);
  uint64_t* empty = full + kGemvSlots;
  int* s_flag = reinterpret_cast<int*>(empty + kGemvSlots);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int c0 = chunk_begin(blockIdx.x, p.total, p.grid);
  const int c1 = chunk_begin(blockIdx.x + 1, p.total, p.grid);
  const int n = c1 - c0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kGemvSlots; ++s) {
      mbar_init(full + s, 1);
      mbar_init(empty + s, kGemvComputeWarps);
    }
    fence_mbar_init();
  }
  __syncthreads();
  pdl_launch_dependents();

  if (warp == kGemvComputeWarps) {
    // ---------------- producer: stream this CTA's weight bytes into the slot ring ----------------
    if (lane == 0) {
      const uint64_t pol = policy_evict_first();
      const uint8_t* wsrc = p.wq + (int64_t)c0 * kChunkWBytes;
      const uint8_t* ssrc = p.ws + (int64_t)c0 * kChunkSBytes;
      int issued = 0;
      bool ok = true;
      int s = 0;
      uint32_t ph = 0;  // phase of empty[s] to wait for (used once the ring wraps)
      for (int i = 0; i < n; ++i) {
        if (i >= kGemvSlots && !mbar_wait(empty + s, ph)) {
          set_error(p.err, kErrWaitTimeout);
          ok = false;
          break;
        }
        uint8_t* dst = slots + (size_t)s * kSlotBytes;
        mbar_arrive_expect_tx(full + s, kSlotBytes);
        bulk_g2s(dst, wsrc, kChunkWBytes, full + s, pol);
        bulk_g2s(dst + kChunkWBytes, ssrc, kChunkSBytes, full + s, pol);
        wsrc += kChunkWBytes;
        ssrc += kChunkSBytes;
        ++issued;
        if (++s == kGemvSlots) {
          s = 0;
          if (i >= kGemvSlots) ph ^= 1;
        }
      }
      if (!ok) {
        // drain: do not leave the CTA while copies into its shared memory are in flight
        const uint64_t deadline = globaltimer_ns() + kWaitTimeoutNs;
        for (int i = (issued > kGemvSlots ? issued - kGemvSlots : 0); i < issued; ++i)
          if (!mbar_wait_until(full + (i % kGemvSlots), (i / kGemvSlots) & 1, deadline)) break;
      }
    }
    return;
  }

  // ---------------- compute warps ----------------
  const int g = lane >> 2, t = lane & 3;
  const int KT = p.ktiles;
  const bool kfull = (p.K & 63) == 0;
  const __half* xr[MG];
  bool xok[MG];
#pragma unroll
  for (int mg = 0; mg < MG; ++mg) {
    const int m = p.token0 + mg * 8 + g;
    xok[mg] = m < p.M;
    xr[mg] = p.x + (int64_t)(xok[mg] ? m : 0) * p.K + 8 * t;
  }
  float acc[MG][4];
#pragma unroll
  for (int mg = 0; mg < MG; ++mg)
#pragma unroll
    for (int e = 0; e < 4; ++e) acc[mg][e] = 0.f;

  int nb = c0 / KT, kt = c0 - nb * KT;  // the only division: chunk indices advance incrementally
  int cur_nb = nb;
  int seg_start = c0;
  bool failed = false;
  int consumed = 0;  // chunks whose copies this warp has seen land
  int s = 0;
  uint32_t ph = 0;
  const uint8_t* my_w = slots + warp * 512 + lane * 16;
  const uint8_t* my_s = slots + kChunkWBytes + warp * 64 + g * 8;

  pdl_wait();  // x is written by the previous kernel in the stream
  uint4 xn[MG][2];
  if (n > 0) load_x<MG>(xn, xr, xok, kt * 64, p.K, kfull);
  for (int i = 0; i < n; ++i) {
    if (nb != cur_nb) {
      flush_segment<MG>(p, cur_nb, seg_start, c0 + i, c0, acc, warp, lane, s_flag);
#pragma unroll
      for (int mg = 0; mg < MG; ++mg)
#pragma unroll
        for (int e = 0; e < 4; ++e) acc[mg][e] = 0.f;
      cur_nb = nb;
      seg_start = c0 + i;
    }
    uint4 xv[MG][2];
#pragma unroll
    for (int mg = 0; mg < MG; ++mg) {
      xv[mg][0] = xn[mg][0];
      xv[mg][1] = xn[mg][1];
    }
    // prefetch the next chunk's activations while this one is computed
    const int kt_next = (kt + 1 == KT) ? 0 : kt + 1;
    if (i + 1 < n) load_x<MG>(xn, xr, xok, kt_next * 64, p.K, kfull);

    if (!failed && !mbar_wait(full + s, ph)) {
      set_error(p.err, kErrWaitTimeout);
      failed = true;  // keep walking the chunk list so every warp meets the same named barriers
    }
    if (!failed) {
      consumed = i + 1;
      const uint4 wv = *reinterpret_cast<const uint4*>(my_w + s * kSlotBytes);
      const uint2 sv = *reinterpret_cast<const uint2*>(my_s + s * kSlotBytes);
      __syncwarp();
      if (lane == 0) mbar_arrive(empty + s);

      const uint32_t wr[4] = {wv.x, wv.y, wv.z, wv.w};
      const float2 sb0 = __half22float2(*reinterpret_cast<const __half2*>(&sv.x));  // (row g, blk0), (row g+8, blk0)
      const float2 sb1 = __half22float2(*reinterpret_cast<const __half2*>(&sv.y));  // (row g, blk1), (row g+8, blk1)
#pragma unroll
      for (int blk = 0; blk < 2; ++blk) {
        uint32_t ha[4], hb[4];
        i4x8_to_h2x4_centered(wr[2 * blk + 0], ha);  // row g
        i4x8_to_h2x4_centered(wr[2 * blk + 1], hb);  // row g + 8
        const float sg = blk ? sb1.x : sb0.x;
        const float sg8 = blk ? sb1.y : sb0.y;
#pragma unroll
        for (int mg = 0; mg < MG; ++mg) {
          float d[4] = {0.f, 0.f, 0.f, 0.f};
          mma_16816(d, ha[0], hb[0], ha[1], hb[1], xv[mg][blk].x, xv[mg][blk].y);
          mma_16816(d, ha[2], hb[2], ha[3], hb[3], xv[mg][blk].z, xv[mg][blk].w);
          acc[mg][0] = fmaf(sg, d[0], acc[mg][0]);
          acc[mg][1] = fmaf(sg, d[1], acc[mg][1]);
          acc[mg][2] = fmaf(sg8, d[2], acc[mg][2]);
          acc[mg][3] = fmaf(sg8, d[3], acc[mg][3]);
        }
      }
    }
    if (++s == kGemvSlots) {
      s = 0;
      ph ^= 1;
    }
    if (++kt == KT) {
      kt = 0;
      ++nb;
    }
  }
  // Every compute warp walks the same chunk list (also after a failed wait, see above), so all of
  // them meet the named barriers in flush_segment the same number of times.
  if (n > 0) flush_segment<MG>(p, cur_nb, seg_start, c1, c0, acc, warp, lane, s_flag);
  if (failed && warp == 0 && lane == 0) {
    // drain copies the producer may still have in flight into this CTA's slots
    const uint64_t deadline = globaltimer_ns() + kWaitTimeoutNs;
    const int end = (consumed + kGemvSlots < n) ? consumed + kGemvSlots : n;
    for (int i = consumed; i < end; ++i)
      if (!mbar_wait_until(full + (i % kGemvSlots), (i / kGemvSlots) & 1, deadline)) break;
  }
}

// CTAs of one launch when the caller leaves the split to the kernel: every resident slot.
template <int MG>
static cudaError_t gemv_auto_grid(int sm_count, int* grid) {
  static int occ[64] = {};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  if (occ[dev] == 0) {
    e = cudaFuncSetAttribute(gemv_streamk_kernel<MG>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kGemvSmem);
    if (e != cudaSuccess) return e;
    int blocks = 0;
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&blocks, gemv_streamk_kernel<MG>, kGemvThreads, kGemvSmem);
    if (e != cudaSuccess) return e;
    occ[dev] = blocks < 1 ? 1 : (blocks > kGemvMaxCtasPerSm ? kGemvMaxCtasPerSm : blocks);
  }
  *grid = occ[dev] * sm_count;
  return cudaSuccess;
}

template <int MG>
static cudaError_t launch_gemv_mg(GemvParams p, int sm_count, cudaStream_t stream, bool pdl) {
  int auto_grid = 0;
  cudaError_t e = gemv_auto_grid<MG>(sm_count, &auto_grid);  // also sets the shared-memory attribute
  if (e != cudaSuccess) return e;
  if (p.grid <= 0) p.grid = auto_grid;
  if (p.grid > p.total) p.grid = p.total;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(p.grid, 1, 1);
  cfg.blockDim = dim3(kGemvThreads, 1, 1);
  cfg.dynamicSmemBytes = kGemvSmem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, gemv_streamk_kernel<MG>, p);
}

// Number of 8-token groups a single GEMV launch handles at most.
constexpr int kGemvMaxGroups = 4;

cudaError_t launch_gemv(const uint8_t* wq, const uint8_t* ws, const __half* x, __half* y, float* partials,
                        uint32_t* tickets, uint32_t* err, int M, int N, int K, int nblk, int ktiles, int token0,
                        int groups, int grid, int sm_count, cudaStream_t stream, bool pdl) {
  GemvParams p;
  p.wq = wq;
  p.ws = ws;
  p.x = x;
  p.y = y;
  p.partials = reinterpret_cast<float4*>(partials);
  p.tickets = tickets;
  p.err = err;
  p.M = M;
  p.N = N;
  p.K = K;
  p.nblk = nblk;
  p.ktiles = ktiles;
  p.total = nblk * ktiles;
  p.grid = grid;  // 0: one CTA per resident slot
  p.token0 = token0;
  switch (groups) {
    case 1: return launch_gemv_mg<1>(p, sm_count, stream, pdl);
    case 2: return launch_gemv_mg<2>(p, sm_count, stream, pdl);
    case 3: return launch_gemv_mg<3>(p, sm_count, stream, pdl);
    case 4: return launch_gemv_mg<4>(p, sm_count, stream, pdl);
    default: return cudaErrorInvalidValue;
  }
}

int gemv_max_grid(int sm_count) { return kGemvMaxCtasPerSm * sm_count; }

size_t gemv_partials_bytes(int sm_count) {
  return (size_t)gemv_max_grid(sm_count) * 2 * kGemvMaxGroups * kGemvComputeWarps * 32 * sizeof(float4);
}

}  // namespace s4
