// Decode GEMV family (M <= 16): y[M][N] = x[M][K] @ W^T for int4 block-32 weights.
//
// Replaces kernelV1 (web/public/gemmbench/kernels.js:40-81), which the engine uses for M <= 8
// (engine.js:25), and the small-M end of kernelV4 + REDUCE (kernels.js:269-353).
//
// Design (HBM-bound at ~0.53 byte of weight per multiply-add at M = 1; on B200 the int4 -> fp16
// conversion makes it nearly issue-bound too, so the loop carries no bookkeeping):
//  * one thread-block cluster of S CTAs per n-block of 128 output rows; CTA r of the cluster
//    takes k-tiles [r*KT/S, (r+1)*KT/S). S is chosen so that about two CTAs land on every SM,
//    leaving room for some of the next launch's CTAs (programmatic dependent launch).
//  * a CTA's weights and scales are one contiguous span of the repacked layout (its k-tiles of one
//    n-block). Thread 0 requests all of it at kernel start with 1-D bulk copies (TMA engine, no
//    multicast) into shared memory, in groups of four k-tiles with one mbarrier each, before the
//    wait on the previous kernel (weights do not depend on it): every byte of the launch is in
//    flight at once, so DRAM latency is paid once per launch instead of once per batch per warp.
//  * warp w of a CTA owns rows w*16 .. w*16+15. Each k-tile of its sub-tile is a 512-byte line
//    whose 16-byte lane slices are its mma.sync A fragments (weights as the 16-row operand, tokens
//    as the 8 columns), read from shared memory without bank conflicts.
//  * activations (<= 16 rows x the CTA's K range) are staged once into padded shared-memory rows.
//  * int4 is converted to exact fp16 (q - 8) and the block scale is applied in fp32 to the fp32
//    block partial, so the only roundings are fp32 accumulation and the final fp16 store.
//  * the S partials of an n-block are summed in rank order by rank 0 through distributed shared
//    memory between two cluster barriers: deterministic, no global scratch, no atomics.
#include "common.cuh"
#include "gemv_tile.cuh"

namespace s4 {

struct GemvParams {
  const uint8_t* wq;  // repacked int4: chunk (nb, kt) at wq + (nb*KT + kt)*4096, sub-tile s at +s*512
  const uint8_t* ws;  // repacked scales: chunk at ws + (nb*KT + kt)*512, sub-tile s at +s*64
  const uint8_t* wb;  // asymmetric formats: biases in the layout of ws (else unused)
  int glu;            // fused gate|up weight: y[M][N/2] = silu(gate) * up (see repack.cu)
  const __half* x;    // [M][K]
  __half* y;          // [M][N]
  uint32_t* err;      // device error word
  int M, N, K;
  int nblk, ktiles;
  int split;          // S: CTAs per cluster / k-splits per n-block
  int token0;         // first token of this launch (tokens token0 .. token0 + 8*MG - 1)
  // dynamic shared memory layout (bytes), from gemv_layout()
  int s_off, b_off, x_off, red_off, bar_off;
  int xrow;           // padded activation row: 128 bytes per k-tile + 64
};

constexpr int kChunkW2Bytes = 2048;  // native 2-bit decode layout: bytes of one chunk (format.cu)

constexpr int kGemvWarps = 8;                 // one per 16-row sub-tile of the n-block
constexpr int kGemvThreads = kGemvWarps * 32;
constexpr int kGemvMaxGroups = 2;             // GEMV serves M <= 16
constexpr int kGemvMaxKtPerCta = 16;          // activation staging: <= 16 k-tiles per CTA
constexpr int kGemvMaxSplit = 16;             // non-portable cluster size limit
constexpr int kGemvGroup = 4;                 // k-tiles per bulk-copy group (one mbarrier each)
constexpr int kGemvMaxCopyGroups = kGemvMaxKtPerCta / kGemvGroup;

// Shared memory of one CTA holding at most `nkt` k-tiles for MG token groups: weights, scales,
// biases (asymmetric formats only), activation rows (64 bytes of padding per row: consecutive rows start 16 banks apart),
// reduction partials, mbarriers.
struct GemvLayout {
  int s_off, b_off, x_off, red_off, bar_off, total, xrow;
};
static GemvLayout gemv_layout(int nkt, int MG, bool asym, int wbytes = kChunkWBytes) {
  GemvLayout L;
  L.xrow = nkt * 128 + 64;
  L.s_off = nkt * wbytes;
  L.b_off = L.s_off + nkt * kChunkSBytes;
  L.x_off = L.b_off + (asym ? nkt * kChunkSBytes : 0);
  L.red_off = L.x_off + 8 * MG * L.xrow;
  L.bar_off = L.red_off + kGemvWarps * 32 * 16 * MG;
  L.total = L.bar_off + kGemvMaxCopyGroups * 8;
  return L;
}

__device__ __forceinline__ uint32_t cluster_map(const void* p, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_u32(p)), "r"(rank));
  return r;
}
__device__ __forceinline__ float4 ld_cluster_f4(uint32_t addr) {
  float4 v;
  asm volatile("ld.shared::cluster.v4.f32 {%0,%1,%2,%3}, [%4];" : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w) : "r"(addr)
               : "memory");
  return v;
}
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
  asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// BITS: 4 (wq in the int4 layout) or 2 (wq in the native 2-bit decode layout; symmetric only)
template <int MG, bool ASYM, int BITS>
__global__ void __launch_bounds__(kGemvThreads, 3) gemv_cluster_kernel(const GemvParams p) {
  static_assert(BITS == 4 || (BITS == 2 && !ASYM), "2-bit decode layout: symmetric weights only");
  constexpr int WBYTES = BITS == 2 ? kChunkW2Bytes : kChunkWBytes;
  extern __shared__ __align__(128) uint8_t smem[];
  uint8_t* wsm = smem;
  uint8_t* ssm = smem + p.s_off;
  uint8_t* bsm = smem + p.b_off;
  uint8_t* xs = smem + p.x_off;
  float4* red = reinterpret_cast<float4*>(smem + p.red_off);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + p.bar_off);

  const int S = p.split, KT = p.ktiles;
  const int rank = blockIdx.x % S, nb = blockIdx.x / S;
  const int kt0 = (int)(((int64_t)rank * KT) / S), kt1 = (int)(((int64_t)(rank + 1) * KT) / S);
  const int nkt = kt1 - kt0;
  const int ngroups = (nkt + kGemvGroup - 1) / kGemvGroup;
  const int sub = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  const int rows = min(8 * MG, p.M - p.token0);

  if (threadIdx.x == 0) {
    // the CTA's whole weight and scale span, in groups of kGemvGroup k-tiles
    for (int q = 0; q < ngroups; ++q) mbar_init(bars + q, 1);
    fence_mbar_init();
    const uint64_t pol = policy_evict_first();  // streamed once
    const int64_t chunk0 = (int64_t)nb * KT + kt0;
    for (int q = 0; q < ngroups; ++q) {
      const int t0 = q * kGemvGroup, nt = min(kGemvGroup, nkt - t0);
      mbar_arrive_expect_tx(bars + q, (uint32_t)nt * (WBYTES + (ASYM ? 2 : 1) * kChunkSBytes));
      bulk_g2s(wsm + t0 * WBYTES, p.wq + (chunk0 + t0) * WBYTES, (uint32_t)nt * WBYTES, bars + q, pol);
      bulk_g2s(ssm + t0 * kChunkSBytes, p.ws + (chunk0 + t0) * kChunkSBytes, (uint32_t)nt * kChunkSBytes, bars + q, pol);
      if (ASYM)
        bulk_g2s(bsm + t0 * kChunkSBytes, p.wb + (chunk0 + t0) * kChunkSBytes, (uint32_t)nt * kChunkSBytes, bars + q, pol);
    }
  }
  pdl_launch_dependents();
  pdl_wait();  // activations are written by the previous kernel in the stream

  // stage activation rows [token0, token0 + rows) x K range [kt0*64, kt1*64) (zeros past K)
  {
    const int kbase = kt0 * 64;
    const int per_row = nkt * 8;  // 16-byte pieces per row
    for (int i = threadIdx.x; i < rows * per_row; i += kGemvThreads) {
      const int r = i / per_row, c = i - r * per_row;
      const int k = kbase + c * 8;
      uint4 v = make_uint4(0, 0, 0, 0);
      if (k < p.K) v = *reinterpret_cast<const uint4*>(p.x + (int64_t)(p.token0 + r) * p.K + k);
      *reinterpret_cast<uint4*>(xs + r * p.xrow + c * 16) = v;
    }
  }
  __syncwarp();  // each warp reaches the (warp-aligned) block barrier as a whole after its role code
  __syncthreads();  // also orders the mbarrier initialisation before the waits below

  bool xok[MG];
#pragma unroll
  for (int mg = 0; mg < MG; ++mg) xok[mg] = (mg * 8 + g) < rows;
  const int xgroup = 8 * p.xrow;
  const uint8_t* xl = xs + g * p.xrow + 16 * t;  // lane's row, k offset 8t (blk adds 64 bytes)
  // symmetric path: one row pointer per token group; a token past the staged rows reads the last
  // staged row (its outputs are never stored) and K past the end is staged as zeros, so no predicates
  const uint8_t* xr[MG];
#pragma unroll
  for (int mg = 0; mg < MG; ++mg) xr[mg] = xs + min(mg * 8 + g, rows - 1) * p.xrow + 16 * t;
  const uint8_t* wl = wsm + (BITS == 2 ? sub * 256 + lane * 8 : sub * 512 + lane * 16);
  const uint8_t* sl = ssm + sub * 64 + g * 8;
  float acc[MG][4];
#pragma unroll
  for (int mg = 0; mg < MG; ++mg)
#pragma unroll
    for (int e = 0; e < 4; ++e) acc[mg][e] = 0.f;

  for (int q = 0; q < ngroups; ++q) {
    if (!mbar_wait(bars + q, 0)) set_error(p.err, kErrWaitTimeout);  // results invalid; error reported
#pragma unroll
    for (int i = 0; i < kGemvGroup; ++i) {
      const int kk = q * kGemvGroup + i;
      if (kk < nkt) {
        const uint2 sc = *reinterpret_cast<const uint2*>(sl + kk * kChunkSBytes);
        if constexpr (BITS == 2) {
          const uint2 w2 = *reinterpret_cast<const uint2*>(wl + kk * WBYTES);
          const uint8_t* xj[MG];
#pragma unroll
          for (int mg = 0; mg < MG; ++mg) xj[mg] = xr[mg] + kk * 128;
          gemv_tile_rows2<MG>(w2, sc, xj, acc);
        } else if constexpr (ASYM) {
          const uint4 w = *reinterpret_cast<const uint4*>(wl + kk * WBYTES);
          const uint2 bi = *reinterpret_cast<const uint2*>(sl + (p.b_off - p.s_off) + kk * kChunkSBytes);
          gemv_tile_asym<MG>(w, sc, bi, xl + kk * 128, xgroup, (kt0 + kk) * 64 + 32 < p.K, xok, acc);
        } else {
          const uint4 w = *reinterpret_cast<const uint4*>(wl + kk * WBYTES);
          const uint8_t* xj[MG];
#pragma unroll
          for (int mg = 0; mg < MG; ++mg) xj[mg] = xr[mg] + kk * 128;
          gemv_tile_rows<MG>(w, sc, xj, acc);
        }
      }
    }
  }

  // ---- split-K reduction across the cluster (rank order, deterministic) ----
  float4* mine = red + sub * 32 + lane;
#pragma unroll
  for (int mg = 0; mg < MG; ++mg) mine[mg * kGemvWarps * 32] = make_float4(acc[mg][0], acc[mg][1], acc[mg][2], acc[mg][3]);
  if (S > 1) cluster_sync_all();
  if (rank == 0) {
    float sums[MG][4];
#pragma unroll
    for (int mg = 0; mg < MG; ++mg) {
      // every peer's partial requested at once (one round trip), then summed in rank order
      float4 v[kGemvMaxSplit];
#pragma unroll
      for (int q = 1; q < kGemvMaxSplit; ++q)
        if (q < S) v[q] = ld_cluster_f4(cluster_map(mine + mg * kGemvWarps * 32, (uint32_t)q));
      float4 sum = mine[mg * kGemvWarps * 32];
#pragma unroll
      for (int q = 1; q < kGemvMaxSplit; ++q)
        if (q < S) {
          sum.x += v[q].x;
          sum.y += v[q].y;
          sum.z += v[q].z;
          sum.w += v[q].w;
        }
      const float out[4] = {sum.x, sum.y, sum.z, sum.w};
      sums[mg][0] = sum.x;
      sums[mg][1] = sum.y;
      sums[mg][2] = sum.z;
      sums[mg][3] = sum.w;
      if (p.glu) continue;
      const int n0 = nb * 128 + sub * 16 + g;
      const int tok = p.token0 + mg * 8 + 2 * t;
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int m = tok + (e & 1);
        const int n = n0 + ((e >> 1) << 3);
        if (m < p.M && n < p.N) p.y[(int64_t)m * p.N + n] = __float2half_rn(out[e]);
      }
    }
    if (p.glu) {
      // sub-tiles 4..7 hold the up rows of sub-tiles 0..3 (see repack.cu): each up warp leaves its
      // sums in its own reduction slot (already consumed), the gate warps combine
      if (sub >= 4)
#pragma unroll
        for (int mg = 0; mg < MG; ++mg)
          mine[mg * kGemvWarps * 32] = make_float4(sums[mg][0], sums[mg][1], sums[mg][2], sums[mg][3]);
      __syncthreads();
      if (sub < 4) {
        const int I = p.N / 2;
#pragma unroll
        for (int mg = 0; mg < MG; ++mg) {
          const float4 uv = mine[4 * 32 + mg * kGemvWarps * 32];
          const float up[4] = {uv.x, uv.y, uv.z, uv.w};
          const int j0 = nb * 64 + sub * 16 + g;
          const int tok = p.token0 + mg * 8 + 2 * t;
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int m = tok + (e & 1);
            const float gf = __half2float(__float2half_rn(sums[mg][e])), uf = __half2float(__float2half_rn(up[e]));
            if (m < p.M) p.y[(int64_t)m * I + j0 + ((e >> 1) << 3)] = __float2half_rn(silu_mul_f32(gf, uf));
          }
        }
      }
    }
  }
  if (S > 1) cluster_sync_all();  // peers keep their shared memory until rank 0 has read it
}

// k-splits per n-block: about two CTAs per SM over the grid, at most kGemvMaxKtPerCta k-tiles per
// CTA (activation staging), at most KT and kGemvMaxSplit.
static int gemv_pick_split(int nblk, int KT, int sm_count) {
  int s = (2 * sm_count + nblk / 2) / nblk;
  const int min_s = (KT + kGemvMaxKtPerCta - 1) / kGemvMaxKtPerCta;
  if (s < min_s) s = min_s;
  if (s > KT) s = KT;
  if (s > kGemvMaxSplit) s = kGemvMaxSplit;
  if (s < 1) s = 1;
  return s;
}

template <int MG, bool ASYM, int BITS>
static cudaError_t launch_gemv_mg(GemvParams p, int sm_count, cudaStream_t stream, bool pdl) {
  constexpr int WBYTES = BITS == 2 ? kChunkW2Bytes : kChunkWBytes;
  static bool configured[64] = {};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  const GemvLayout L = gemv_layout((p.ktiles + p.split - 1) / p.split, MG, ASYM, WBYTES);
  p.s_off = L.s_off;
  p.b_off = L.b_off;
  p.x_off = L.x_off;
  p.red_off = L.red_off;
  p.bar_off = L.bar_off;
  p.xrow = L.xrow;
  if (!configured[dev]) {
    // the 2-bit layout keeps the int4 layout's shared-memory footprint: with a smaller one the block
    // scheduler packs three CTAs onto an SM where the int4 launch spreads them over more SMs, and the
    // call ran 20-40 % slower for all its halved bytes
    const int max_smem = gemv_layout(kGemvMaxKtPerCta, kGemvMaxGroups, ASYM, kChunkWBytes).total;
    e = cudaFuncSetAttribute(gemv_cluster_kernel<MG, ASYM, BITS>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             max_smem);
    if (e == cudaSuccess)
      e = cudaFuncSetAttribute(gemv_cluster_kernel<MG, ASYM, BITS>, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
    if (e != cudaSuccess) return e;
    configured[dev] = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(p.nblk * p.split, 1, 1);
  cfg.blockDim = dim3(kGemvThreads, 1, 1);
  cfg.dynamicSmemBytes = gemv_layout((p.ktiles + p.split - 1) / p.split, MG, ASYM, kChunkWBytes).total;
  cfg.stream = stream;
  cudaLaunchAttribute attr[3];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = p.split;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
  attr[2].id = cudaLaunchAttributeClusterSchedulingPolicyPreference;
  attr[2].val.clusterSchedulingPolicyPreference = cudaClusterSchedulingPolicySpread;
  cfg.attrs = attr;
  cfg.numAttrs = 3;
  return cudaLaunchKernelEx(&cfg, gemv_cluster_kernel<MG, ASYM, BITS>, p);
}

// k-splits per n-block for a single call: the fewest CTAs (each streaming the most weight bytes)
// that still give at least half the SMs a CTA and fit in one wave with 10 % to spare (a cluster must
// fit in one GPC). A sweep of the four decode shapes at M = 1, 8, 16 found these 14-36 % faster than
// about two CTAs per SM (gemv_pick_split), e.g. attn qkv M = 1 at S = 4: 4.1 us instead of 6.5 us.
static int gemv_pick_split_fit(int nblk, int KT, int sm_count, int MG, bool asym, int wbytes) {
  const int min_s = (KT + kGemvMaxKtPerCta - 1) / kGemvMaxKtPerCta;
  for (int S = min_s < 1 ? 1 : min_s; S <= kGemvMaxSplit && S <= KT; ++S) {
    const GemvLayout L = gemv_layout((KT + S - 1) / S, MG, asym, wbytes);
    int per_sm = (228 * 1024) / (L.total + 1024);  // 228 KB per SM, 1 KB reserved per CTA
    if (per_sm > 3) per_sm = 3;                     // __launch_bounds__ of the kernel
    const long long grid = (long long)nblk * S, cap = (long long)sm_count * per_sm;
    if (per_sm >= 1 && grid * 2 >= sm_count && grid * 10 <= cap * 9) return S;
  }
  return gemv_pick_split(nblk, KT, sm_count);
}

// wq2: the weight's native 2-bit decode layout (symmetric 2-bit formats), streamed instead of wq
cudaError_t launch_gemv(const uint8_t* wq, const uint8_t* ws, const uint8_t* wb, const __half* x, __half* y,
                        uint32_t* err, int M, int N, int K, int nblk, int ktiles, int token0, int groups, int split,
                        int sm_count, cudaStream_t stream, bool pdl, int glu, const uint8_t* wq2) {
  const bool two = wq2 != nullptr && wb == nullptr && !glu;
  GemvParams p;
  p.wq = two ? wq2 : wq;
  p.ws = ws;
  p.wb = wb;
  p.glu = glu;
  p.x = x;
  p.y = y;
  p.err = err;
  p.M = M;
  p.N = N;
  p.K = K;
  p.nblk = nblk;
  p.ktiles = ktiles;
  if (split > 0) {
    // a requested split is clamped to what the activation staging and cluster size allow
    const int min_s = (ktiles + kGemvMaxKtPerCta - 1) / kGemvMaxKtPerCta;
    if (split < min_s) split = min_s;
    if (split > ktiles) split = ktiles;
    if (split > kGemvMaxSplit) split = kGemvMaxSplit;
  } else {
    split = gemv_pick_split_fit(nblk, ktiles, sm_count, groups, wb != nullptr, kChunkWBytes);
  }
  p.split = split;
  if ((ktiles + p.split - 1) / p.split > kGemvMaxKtPerCta) return cudaErrorInvalidValue;  // K > 16384
  p.token0 = token0;
  switch (groups) {
    case 1:
      if (two) return launch_gemv_mg<1, false, 2>(p, sm_count, stream, pdl);
      return wb ? launch_gemv_mg<1, true, 4>(p, sm_count, stream, pdl) : launch_gemv_mg<1, false, 4>(p, sm_count, stream, pdl);
    case 2:
      if (two) return launch_gemv_mg<2, false, 2>(p, sm_count, stream, pdl);
      return wb ? launch_gemv_mg<2, true, 4>(p, sm_count, stream, pdl) : launch_gemv_mg<2, false, 4>(p, sm_count, stream, pdl);
    default: return cudaErrorInvalidValue;
  }
}

int gemv_max_split() { return kGemvMaxSplit; }
int gemv_max_tokens() { return 8 * kGemvMaxGroups; }
int gemv_split_for(int nblk, int ktiles, int sm_count) { return gemv_pick_split(nblk, ktiles, sm_count); }

}  // namespace s4
