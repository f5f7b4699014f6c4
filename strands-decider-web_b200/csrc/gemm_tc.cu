// tcgen05 GEMM family (M > 32): y[M][N] = x[M][K] @ W^T with int4 block-32 weights dequantised to
// fp16 in shared memory and fed to the 5th-generation tensor cores, fp32 accumulation in TMEM.
//
// Replaces kernelV4 (+ REDUCE) of web/public/gemmbench/kernels.js:269-353 and the portable
// kernelV6 (kernels.js:438-479) that the engine picks for M > 8 (engine.js:17-33). Unlike V4 it
// accumulates in fp32 end to end, split-K partials included.
//
// Shape of one MMA (swap-AB): A = 128 weight rows (output columns n) x 16 K, fp16, K-major in
// shared memory with the 128-byte swizzle; B = tn tokens x 16 K of the activations, loaded by TMA
// with the same swizzle; D = 128 x tn fp32 in TMEM (lane = n, column = token).
//
// Work: units (token block tb, n-block nb, k-tile kt) of 64 K, kt fastest; a (tb, nb) tile is KT
// units. The first floor(T/G)*G of the T tiles are dealt out whole, floor(T/G) per CTA, and the units
// of the remaining T mod G tiles are cut into G equal stream-K ranges, so every SM gets the same
// number of MMAs and only those last tiles can be split. A run of units of one tile is a segment; a
// segment that covers the whole K range is written as fp16 directly, otherwise its fp32 partial goes
// to scratch and either a fix-up kernel launched right after sums the partials of each split tile in
// CTA order (the automatic choice, and the allocation-free entry point's), or the last CTA to arrive
// at the tile does it in this kernel (atomic ticket; a dispatch-table choice).
//
// Warp roles (512 threads): warp 0 lane 0 streams raw int4 chunks (1-D bulk copies) into a
// kTcSlotsW-slot ring; warp 2 lane 0 loads activation tiles by TMA into a kTcStagesX-stage ring; warp 1 owns TMEM
// and lane 0 issues the MMAs; warps 4-11 dequantise int4 -> fp16 into the MMA's A stage; warps
// 12-15 drain TMEM (double-buffered accumulators) and write the output.
#include <cuda.h>

#include <atomic>
#include <cstdio>

#include "common.cuh"
#include "internal.h"

namespace s4 {

constexpr int kTcMaxTn = 256;
// Pipeline stages: stage s holds one k-tile's activations (TMA) and its dequantised weights (A). One
// "full" barrier per stage completes when the activation bytes have landed AND all dequant warps have
// arrived; one "empty" barrier per stage is signalled by a single tcgen05.commit once the stage's
// MMAs are done. The MMA thread thus waits once and commits once per k-tile (~370 cycles for four
// MMAs and the commit). Single-thread roles share their sub-partition's issue slots with two busy
// dequant warps and an epilogue warp, so their loops do their index math once per tile segment:
// a runtime division or two per k-tile kept the weight producer at ~850 cycles per chunk, one chunk
// ahead of the dequant warps, and paced the kernel (a per-role clock64 timeline showed it). With
// that gone the activation loads' round trip through the stage ring is on the critical loop: four
// stages, and six weight slots (the weight producer now keeps all six filled ahead of the dequant).
constexpr int kTcStages = 4;
constexpr int kTcStagesX = kTcStages;  // activation tiles (TMA)
constexpr int kTcStagesA = kTcStages;  // dequantised weight (MMA operand A)
constexpr int kTcSlotsW = 6;
constexpr int kTcThreads = 512;
constexpr int kTcDequantWarps = 8;  // warps 4..11
// The dequant warps form kTcDqGroups groups that take alternate chunks (group g: chunks i with
// i % kTcDqGroups == g), so that many chunks convert at once and each thread has
// kTcDqGroups independent 16-byte lane slots per chunk.
#ifndef S4_TC_DQ_GROUPS
#define S4_TC_DQ_GROUPS 2
#endif
constexpr int kTcDqGroups = S4_TC_DQ_GROUPS;
constexpr int kTcDqWarpsPerChunk = kTcDequantWarps / kTcDqGroups;
// Every stage wait is a parity wait, which cannot tell a phase from the one two back. A group reaching
// chunk j (stage j % kTcStages) waits for the MMAs of chunk j - kTcStages; that is safe only if chunk
// j - 2 * kTcStages is known to be consumed, which the group's own previous wait (chunk j - groups)
// guarantees when groups <= stages. With more groups than stages a group could write a stage that is
// still in use and over-arrive on its barrier.
static_assert(kTcDqGroups >= 1 && kTcDqGroups <= kTcStages && kTcDequantWarps % kTcDqGroups == 0,
              "dequant groups must not outnumber the pipeline stages");
constexpr int kTcEpiWarp0 = 12;     // warps 12..15 drain TMEM (lane quarter = warp % 4)
constexpr int kTcXStageBytes = kTcMaxTn * 128;  // tn rows x 64 fp16
constexpr int kTcAStageBytes = 128 * 128;       // 128 rows x 64 fp16
constexpr int kTcWSlotBytes = kChunkWBytes + kChunkSBytes;
// asymmetric formats: a slot also holds the chunk's biases; fewer slots fit the same region
constexpr int kTcWSlotBytesAsym = kChunkWBytes + 2 * kChunkSBytes;
constexpr int kTcSlotsWAsym = (kTcSlotsW * kTcWSlotBytes) / kTcWSlotBytesAsym;
constexpr int kTcOffX = 0;
constexpr int kTcOffA = kTcOffX + kTcStagesX * kTcXStageBytes;
constexpr int kTcOffW = kTcOffA + kTcStagesA * kTcAStageBytes;
constexpr int kTcOffBar = kTcOffW + kTcSlotsW * kTcWSlotBytes;
constexpr int kTcNumBars = 2 * kTcStages + 2 * kTcSlotsW + 2 + 2 + 1;
constexpr int kTcOffMisc = kTcOffBar + kTcNumBars * 8;
constexpr int kTcOffEpi = (kTcOffMisc + 64 + 127) & ~127;  // epilogue staging: 4 warps x 16 tokens x 32 n fp16
constexpr int kTcEpiStageBytes = 16 * 32 * 2;
constexpr size_t kTcSmem = (size_t)kTcOffEpi + 4 * kTcEpiStageBytes + 1024;  // + alignment slack
static_assert(kTcSmem <= 227 * 1024, "tcgen05 GEMM shared memory above the per-CTA limit");
constexpr uint32_t kTcTmemCols = 512;                       // two 256-column accumulators

constexpr int kTcMaxDst = 8;  // output copies one launch writes (this GPU + peers)

struct TcParams {
  const uint8_t* wq;
  const uint8_t* ws;
  const uint8_t* wb;  // asymmetric formats: biases in the layout of ws (else nullptr)
  int glu;            // fused gate|up weight: write silu(gate) * up, N / 2 columns (see repack.cu)
  __half* ydst[kTcMaxDst];  // output buffers: y[tok * ldy + ycol0 + n] is written to each
  int ndst;
  int64_t ldy;
  int ycol0;
  int vec;  // 16-byte output stores allowed: ldy and ycol0 multiples of 8, every ydst 16-byte aligned
  float* partials;    // [grid][2][tn][128] fp32
  uint32_t* tickets;  // [ntb * nblk]
  uint32_t* err;
  int M, N, K;
  int nblk, ktiles;
  int tn;     // tokens per tile = MMA N (multiple of 16, <= 256)
  int ntb;    // token blocks
  int total;  // units = ntb * nblk * ktiles
  int grid;
  int dpq;       // whole tiles per CTA (data-parallel part): CTA b takes tiles [b*dpq, (b+1)*dpq)
  int sk_base;   // first unit of the stream-K part (dpq * grid * ktiles)
  int sk_total;  // units of the stream-K part, split evenly over the grid
  // Residual add + RMSNorm epilogue (resid != nullptr): instead of storing y, each output adds
  // f16(y) to the fp32 residual stream resid[tok * ldr + n] in place and the squares of the updated
  // values are summed per 32-column group into ssp[(n / 32) * ldss + tok]; a row kernel then
  // normalises (ADD_NORM, web/public/engine/wgsl.js:55-78, after out_proj / down, engine.js:247, 277).
  float* resid;
  int64_t ldr;
  float* ssp;
  int64_t ldss;
  // Column-sharded prefill: the activations were gathered from wait_n ranks; the activation producer
  // waits for every rank's signal (peer_wait_all on this rank's flag array) before its first load.
  const uint32_t* wait_flags;
  int wait_n;
};

// Output stores. Each destination is the local buffer or, for the column-sharded prefill, a peer's
// gathered buffer over NVLink. Call sites branch on ndst == 1 once, outside their element loops:
// the epilogue runs 256 stores per thread per tile, and per-element guards for the other
// destinations (predicated code, issued even when off) made a K = 2048 GEMM's epilogue outlast the
// next tile's main loop.
__device__ __forceinline__ int64_t tc_out_off(const TcParams& p, int tok, int ncol) {
  return (int64_t)tok * p.ldy + p.ycol0 + ncol;
}

// resid[tok][n0 .. n0 + 8) = a, b + f16 outputs v (the projection's y, rounded to fp16 as the
// reference stores it; a, b the loaded residual); returns the sum of the updated values' squares, in
// column order
__device__ __forceinline__ float tc_add_resid8(const TcParams& p, int tok, int n0, float4 a, float4 b,
                                               const uint4& v) {
  float4* r = reinterpret_cast<float4*>(p.resid + (int64_t)tok * p.ldr + n0);
  const __half2* h2 = reinterpret_cast<const __half2*>(&v);
  const float2 y0 = __half22float2(h2[0]), y1 = __half22float2(h2[1]);
  const float2 y2 = __half22float2(h2[2]), y3 = __half22float2(h2[3]);
  a.x += y0.x;
  a.y += y0.y;
  a.z += y1.x;
  a.w += y1.y;
  b.x += y2.x;
  b.y += y2.y;
  b.z += y3.x;
  b.w += y3.y;
  r[0] = a;
  r[1] = b;
  float ss = a.x * a.x;
  ss += a.y * a.y;
  ss += a.z * a.z;
  ss += a.w * a.w;
  ss += b.x * b.x;
  ss += b.y * b.y;
  ss += b.z * b.z;
  ss += b.w * b.w;
  return ss;
}

// the residual values tc_add_resid8 needs for tokens tok .. tok + 16 of this lane (j = 0, 1: token
// tok + j * 8 + lane / 4); rows at or past M read nothing
__device__ __forceinline__ void tc_load_resid16(const TcParams& p, int tok, int n0, int lane, float4 (&r)[2][2]) {
#pragma unroll
  for (int j = 0; j < 2; ++j) {
    const int t = tok + j * 8 + (lane >> 2);
    if (t < p.M && n0 < p.N) {
      const float4* src = reinterpret_cast<const float4*>(p.resid + (int64_t)t * p.ldr + n0);
      r[j][0] = src[0];
      r[j][1] = src[1];
    } else {
      r[j][0] = r[j][1] = make_float4(0.f, 0.f, 0.f, 0.f);
    }
  }
}
__device__ __forceinline__ void tc_store_all(const TcParams& p, int64_t off, __half h) {
  for (int d = 0; d < p.ndst; ++d) p.ydst[d][off] = h;
}

// ---- tcgen05 / TMA wrappers -----------------------------------------------------------------------
__device__ __forceinline__ uint64_t sw128_kmajor_desc(uint32_t saddr) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFFu);  // start address
  d |= (uint64_t)1u << 16;                  // leading byte offset (unused with 128-byte swizzle)
  d |= (uint64_t)(1024u >> 4) << 32;        // stride byte offset: 8 rows x 128 bytes
  d |= (uint64_t)1u << 46;                  // descriptor version (sm_100)
  d |= (uint64_t)2u << 61;                  // 128-byte swizzle
  return d;
}
__device__ __forceinline__ uint32_t f16_f32_idesc(int n) {
  // dense, D f32 (bits 4-5 = 1), A/B f16 (0), both K-major, N >> 3 at 17, M >> 4 at 24
  return (1u << 4) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(128 >> 4) << 24);
}
__device__ __forceinline__ void tc_mma(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(acc)
      : "memory");
}
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_proxy_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}
__device__ __forceinline__ void bulk_g2s_plain(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   smem_u32(dst)),
               "l"(src), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}

// Work split: the first dpq * grid tiles go whole to the CTAs (dpq each, no partials); the units of
// the remaining tiles (fewer than grid tiles) are cut into grid equal stream-K ranges, so only those
// tiles can be split. tc_begin(b) is where CTA b's stream-K range starts; tc_cta_of(u) is the CTA
// whose stream-K range holds unit u.
__device__ __forceinline__ int tc_begin(int b, const TcParams& p) {
  return p.sk_base + (int)(((int64_t)b * p.sk_total) / p.grid);
}
__device__ __forceinline__ int tc_cta_of(int u, const TcParams& p) {
  return (int)((((int64_t)(u - p.sk_base) + 1) * p.grid - 1) / p.sk_total);
}
struct TcWork {
  int dp0, ndp;  // whole-tile units [dp0, dp0 + ndp)
  int sk0, sk1;  // stream-K units [sk0, sk1)
  __device__ __forceinline__ int count() const { return ndp + (sk1 - sk0); }
  __device__ __forceinline__ int unit(int i) const { return i < ndp ? dp0 + i : sk0 + (i - ndp); }
  __device__ __forceinline__ int range_end(int i) const { return i < ndp ? dp0 + ndp : sk1; }
};
__device__ __forceinline__ TcWork tc_work(int b, const TcParams& p) {
  TcWork w;
  w.ndp = p.dpq * p.ktiles;
  w.dp0 = b * w.ndp;
  w.sk0 = tc_begin(b, p);
  w.sk1 = tc_begin(b + 1, p);
  return w;
}

// kTicketFixup: split tiles are finished inside this kernel by the last CTA to arrive (atomic
// ticket); otherwise partials are only published and tc_fixup_kernel, launched next, sums them.
template <bool kTicketFixup, bool kAsym>
__global__ void __launch_bounds__(kTcThreads, 1) tc_gemm_kernel(const TcParams p, const __grid_constant__ CUtensorMap tmap_x) {
  constexpr int SW = kAsym ? kTcSlotsWAsym : kTcSlotsW;            // raw weight ring slots
  constexpr int WB = kAsym ? kTcWSlotBytesAsym : kTcWSlotBytes;    // bytes per slot
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + (((raw_addr + 1023u) & ~1023u) - raw_addr);
  uint8_t* xs = smem + kTcOffX;
  uint8_t* wa = smem + kTcOffA;
  uint8_t* wraw = smem + kTcOffW;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kTcOffBar);
  uint64_t* full = bars;                 // stage full: activation bytes + dequant warps
  uint64_t* empty = full + kTcStages;    // stage consumed by the MMAs (tcgen05.commit)
  uint64_t* full_w = empty + kTcStages;
  uint64_t* empty_w = full_w + kTcSlotsW;  // barrier arrays keep the symmetric layout's size
  uint64_t* accf = empty_w + kTcSlotsW;
  uint64_t* acce = accf + 2;
  uint64_t* drain = acce + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + kTcOffMisc);
  int* s_flag = reinterpret_cast<int*>(smem + kTcOffMisc + 16);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const TcWork wk = tc_work(blockIdx.x, p);
  const int n = wk.count();
  const int KT = p.ktiles;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kTcStages; ++s) {
      mbar_init(full + s, kTcDqWarpsPerChunk + 1);  // + the activation producer's expect-tx arrival
      mbar_init(empty + s, 1);
    }
    for (int s = 0; s < SW; ++s) {
      mbar_init(full_w + s, 1);
      mbar_init(empty_w + s, kTcDqWarpsPerChunk);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(accf + b, 1);
      mbar_init(acce + b, 128);
    }
    mbar_init(drain, 1);
    fence_mbar_init();
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(kTcTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  __syncwarp();  // each warp reaches the (warp-aligned) block barrier as a whole after its role code
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  pdl_launch_dependents();

  if (warp == 0) {
    // ------------- raw int4 chunks: producer -------------
    if (lane == 0) {
      int issued = 0;
      bool ok = true;
      // index math once per segment (a run of units of one tile): runtime divisions per unit cost
      // this single thread issue slots it shares with the dequant warps
      int slot = 0, round = 0;
      for (int i = 0; i < n && ok;) {
        const int u0 = wk.unit(i);
        const int tile = u0 / KT;
        const int seg_end = min(wk.range_end(i), (tile + 1) * KT);
        const int64_t chunk0 = (int64_t)(tile % p.nblk) * KT + (u0 - tile * KT);
        const uint8_t* srcq = p.wq + chunk0 * kChunkWBytes;
        const uint8_t* srcs = p.ws + chunk0 * kChunkSBytes;
        const uint8_t* srcb = kAsym ? p.wb + chunk0 * kChunkSBytes : nullptr;
        for (int u = u0; u < seg_end; ++u, ++i) {
          if (round > 0 && !mbar_wait(empty_w + slot, (round - 1) & 1)) {
            set_error(p.err, kErrWaitTimeout);
            ok = false;
            break;
          }
          uint8_t* dst = wraw + slot * WB;
          mbar_arrive_expect_tx(full_w + slot, WB);
          bulk_g2s_plain(dst, srcq, kChunkWBytes, full_w + slot);
          bulk_g2s_plain(dst + kChunkWBytes, srcs, kChunkSBytes, full_w + slot);
          if (kAsym) {
            bulk_g2s_plain(dst + kChunkWBytes + kChunkSBytes, srcb, kChunkSBytes, full_w + slot);
            srcb += kChunkSBytes;
          }
          srcq += kChunkWBytes;
          srcs += kChunkSBytes;
          ++issued;
          if (++slot == SW) {
            slot = 0;
            ++round;
          }
        }
      }
      if (!ok) {
        const uint64_t deadline = globaltimer_ns() + kWaitTimeoutNs;
        for (int i = (issued > SW ? issued - SW : 0); i < issued; ++i)
          if (!mbar_wait_until(full_w + (i % SW), (i / SW) & 1, deadline)) break;
      }
    }
  } else if (warp == 2) {
    // ------------- activation tiles: producer (TMA) -------------
    if (lane == 0) {
      pdl_wait();  // x is written by the previous kernel in the stream
      if (p.wait_flags) {
        // and by the peers: their generic stores, then this warp's TMA (async proxy) loads
        if (!peer_wait_all(p.wait_flags, p.wait_n)) set_error(p.err, kErrWaitTimeout);
        asm volatile("fence.proxy.async.global;" ::: "memory");
      }
      int issued = 0;
      bool ok = true;
      const uint32_t xbytes = (uint32_t)p.tn * 128u;
      int s = 0, round = 0;
      for (int i = 0; i < n && ok;) {
        const int u0 = wk.unit(i);
        const int tile = u0 / KT;
        const int seg_end = min(wk.range_end(i), (tile + 1) * KT);
        const int row0 = (tile / p.nblk) * p.tn;
        int kcol = (u0 - tile * KT) * 64;
        for (int u = u0; u < seg_end; ++u, ++i) {
          if (round > 0 && !mbar_wait(empty + s, (round - 1) & 1)) {
            set_error(p.err, kErrWaitTimeout);
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(full + s, xbytes);
          tma_load_2d(xs + s * kTcXStageBytes, &tmap_x, kcol, row0, full + s);
          kcol += 64;
          ++issued;
          if (++s == kTcStagesX) {
            s = 0;
            ++round;
          }
        }
      }
      if (!ok) {
        const uint64_t deadline = globaltimer_ns() + kWaitTimeoutNs;
        for (int i = (issued > kTcStagesX ? issued - kTcStagesX : 0); i < issued; ++i)
          if (!mbar_wait_until(full + (i % kTcStagesX), (i / kTcStagesX) & 1, deadline)) break;
      }
    }
  } else if (warp == 1) {
    // ------------- MMA issuer -------------
    if (lane == 0) {
      const uint32_t idesc = f16_f32_idesc(p.tn);
      // descriptors of stage 0; a stage adds its byte offset >> 4, each 16-K step 32 bytes >> 4 = 2
      const uint64_t adesc0 = sw128_kmajor_desc(smem_u32(wa)), bdesc0 = sw128_kmajor_desc(smem_u32(xs));
      bool ok = true;
      int si = 0;
      int i = 0;
      int s = 0;
      uint32_t ph = 0;
      while (ok && i < n) {
        const int u0 = wk.unit(i);
        const int tile = u0 / KT;
        const int seg_end = min(wk.range_end(i), (tile + 1) * KT);  // units [u0, seg_end) belong to this tile
        const int buf = si & 1;
        if (si >= 2 && !mbar_wait(acce + buf, ((si >> 1) - 1) & 1)) {
          set_error(p.err, kErrWaitTimeout);
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t dcol = tmem_base + (uint32_t)(buf * 256);
        for (int u = u0; u < seg_end; ++u, ++i) {
          if (!mbar_wait(full + s, ph)) {
            set_error(p.err, kErrWaitTimeout);
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t ad = adesc0 + (uint64_t)((s * kTcAStageBytes) >> 4);
          const uint64_t bd = bdesc0 + (uint64_t)((s * kTcXStageBytes) >> 4);
          tc_mma(dcol, ad, bd, idesc, u != u0 ? 1u : 0u);
          tc_mma(dcol, ad + 2, bd + 2, idesc, 1u);
          tc_mma(dcol, ad + 4, bd + 4, idesc, 1u);
          tc_mma(dcol, ad + 6, bd + 6, idesc, 1u);
          tc_commit(empty + s);
          if (++s == kTcStages) {
            s = 0;
            ph ^= 1u;
          }
        }
        if (!ok) break;
        tc_commit(accf + buf);
        ++si;
      }
      tc_commit(drain);  // completes when every MMA issued above has finished
      (void)mbar_wait(drain, 0);
    }
  } else if (warp >= 4 && warp < 4 + kTcDequantWarps) {
    // ------------- dequantisers: int4 chunk -> fp16 A stage (128-byte swizzled, K-major) -------------
    const int dg = (warp - 4) / kTcDqWarpsPerChunk;              // this warp's group
    const int d = threadIdx.x - 128 - dg * kTcDqWarpsPerChunk * 32;  // thread index within the group
    bool ok = true;
    for (int i = dg; i < n && ok; i += kTcDqGroups) {
      const int s = i % kTcStagesA, slot = i % SW;
      if (!mbar_wait(full_w + slot, (i / SW) & 1) ||
          (i >= kTcStagesA && !mbar_wait(empty + s, ((i / kTcStagesA) - 1) & 1))) {
        set_error(p.err, kErrWaitTimeout);
        ok = false;
        break;
      }
      const uint8_t* src = wraw + slot * WB;
      const uint32_t dst = smem_u32(wa + s * kTcAStageBytes);
#pragma unroll
      for (int rep = 0; rep < 256 / (32 * kTcDqWarpsPerChunk); ++rep) {
        const int L = d + rep * 32 * kTcDqWarpsPerChunk;  // 16-byte lane slot: sub-tile L / 32, lane L % 32
        const int sub = L >> 5, ln = L & 31, g = ln >> 2, t = ln & 3;
        const uint4 v = *reinterpret_cast<const uint4*>(src + L * 16);
        const uint2 sc = *reinterpret_cast<const uint2*>(src + kChunkWBytes + sub * 64 + g * 8);
        const uint32_t words[4] = {v.x, v.y, v.z, v.w};
        const uint32_t sh[4] = {sc.x & 0xFFFFu, sc.x >> 16, sc.y & 0xFFFFu, sc.y >> 16};  // (g,b0) (g+8,b0) (g,b1) (g+8,b1)
        const bool odd = (g & 1) != 0;
#pragma unroll
        for (int jj = 0; jj < 4; ++jj) {
          // odd rows store the other quant block first: the 8 lanes of a store phase then hit
          // 32 distinct banks
          const int j = odd ? (jj ^ 2) : jj;
          const uint32_t w = odd ? words[jj ^ 2] : words[jj];
          const uint32_t sbits = odd ? sh[jj ^ 2] : sh[jj];
          const int blk = j >> 1, h = j & 1;
          const int r = sub * 16 + g + 8 * h;
          const int c = blk * 4 + t;
          uint32_t hv[4];
          if constexpr (kAsym) {  // w = fma(q, scale, bias) in fp16 (kernels.js:36)
            const uint2 bi = *reinterpret_cast<const uint2*>(src + kChunkWBytes + kChunkSBytes + sub * 64 + g * 8);
            const uint32_t jb = odd ? (jj ^ 2) : jj;
            const uint32_t bbits = ((jb >> 1) ? bi.y : bi.x) >> (16 * (jb & 1)) & 0xFFFFu;
            i4x8_to_h2x4_raw(w, hv);
            h2x4_fma(hv, sbits, bbits);
          } else {
            i4x8_to_h2x4_centered(w, hv);
            const uint32_t s2 = sbits | (sbits << 16);
#pragma unroll
            for (int e = 0; e < 4; ++e) asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(hv[e]) : "r"(hv[e]), "r"(s2));
          }
          const uint32_t addr = dst + r * 128 + ((c ^ (r & 7)) << 4);
          asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(hv[0]), "r"(hv[1]), "r"(hv[2]),
                       "r"(hv[3])
                       : "memory");
        }
      }
      fence_proxy_async_smem();  // generic-proxy stores -> visible to the tensor core's async proxy
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(full + s);
        mbar_arrive(empty_w + slot);
      }
    }
  } else if (warp >= kTcEpiWarp0) {
    // ------------- epilogue: TMEM -> output (or fp32 partial + ticket fix-up) -------------
    const int q = warp - kTcEpiWarp0;  // TMEM lane quarter this warp may access (warp % 4)
    const int nl = q * 32 + lane;
    const int et = threadIdx.x - kTcEpiWarp0 * 32;
    uint8_t* epi_base = smem + kTcOffEpi;
    __half* epi_stage = reinterpret_cast<__half*>(epi_base + q * kTcEpiStageBytes);
    bool failed = false;
    int si = 0;
    for (int i = 0; i < n; ++si) {
      const int u0 = wk.unit(i);
      const int tile = u0 / KT;
      const int seg_end = min(wk.range_end(i), (tile + 1) * KT);
      const int ks = u0 - tile * KT, ke = seg_end - tile * KT;
      i += seg_end - u0;
      const int tb = tile / p.nblk, nb = tile - tb * p.nblk;
      const int buf = si & 1;
      const bool full = (ks == 0 && ke == KT);
      const int tok0 = tb * p.tn;
      const int ncol = nb * 128 + nl;
      const uint32_t taddr = tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(buf * 256);
      if (p.resid && full && !failed) {
        // the tile's residual rows go to L2 while its MMAs run, so the epilogue's loads hit L2
        const int nbytes = min(128, p.N - nb * 128) * 4;
        for (int t = et; t < p.tn && tok0 + t < p.M; t += 128)
          asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p.resid + (int64_t)(tok0 + t) * p.ldr +
                                                                          nb * 128),
                       "r"(nbytes)
                       : "memory");
      }
      if (!failed && !mbar_wait(accf + buf, (si >> 1) & 1)) {
        set_error(p.err, kErrWaitTimeout);
        failed = true;  // keep walking segments so the named barriers below stay matched
      }
      const int sel = (u0 == wk.sk0) ? 0 : 1;  // partial slot: first or last stream-K segment
      float* mine = p.partials + (((int64_t)blockIdx.x * 2 + sel) * p.tn) * 128 + nl;
      if (p.glu && full) {
        // SiLU*mul: lane quarters q and q + 2 hold the gate and up rows of the same 32 features; each
        // stages its fp16 values, then the pair computes the outputs, 8 tokens each. The pair's two
        // barriers run on every slab even after a failed wait (the partner still arrives).
        const int pq = q & 1;
        const __half* gs = reinterpret_cast<const __half*>(epi_base + pq * kTcEpiStageBytes);
        const __half* us = reinterpret_cast<const __half*>(epi_base + (pq + 2) * kTcEpiStageBytes);
        if (!failed) tc_fence_after();
        for (int cb = 0; cb < p.tn; cb += 16) {
          if (!failed) {
            float v[16];
            tmem_ld16(taddr + cb, v);
#pragma unroll
            for (int e = 0; e < 16; ++e) epi_stage[e * 32 + lane] = __float2half_rn(v[e]);
          }
          named_bar_sync(3 + pq, 64);
          if (!failed) {
            const int t = (q >> 1) * 8 + (lane >> 2), c = lane & 3;
            const uint4 gv = *reinterpret_cast<const uint4*>(gs + t * 32 + c * 8);
            const uint4 uv = *reinterpret_cast<const uint4*>(us + t * 32 + c * 8);
            const __half2* g2 = reinterpret_cast<const __half2*>(&gv);
            const __half2* u2 = reinterpret_cast<const __half2*>(&uv);
            uint4 ov;
            __half2* o2 = reinterpret_cast<__half2*>(&ov);
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const float2 g = __half22float2(g2[e]), u = __half22float2(u2[e]);
              o2[e] = __floats2half2_rn(silu_mul_f32(g.x, u.x), silu_mul_f32(g.y, u.y));
            }
            const int tok = tok0 + cb + t;
            if (tok < p.M) {
              const int64_t off = tc_out_off(p, tok, nb * 64 + pq * 32 + c * 8);
              for (int d = 0; d < p.ndst; ++d) *reinterpret_cast<uint4*>(p.ydst[d] + off) = ov;
            }
          }
          named_bar_sync(3 + pq, 64);
        }
        if (!failed) {
          tc_fence_before();
          mbar_arrive(acce + buf);
        }
      } else if (full) {
        if (!failed) {
          tc_fence_after();
          // residual mode: this lane's residual values of the next 16 tokens are loaded one chunk
          // ahead (t = j * 8 + lane / 4, columns n0 .. n0 + 8)
          const int n0r = nb * 128 + q * 32 + (lane & 3) * 8;
          float4 rnext[2][2];
          if (p.resid) tc_load_resid16(p, tok0, n0r, lane, rnext);
          for (int cb = 0; cb < p.tn; cb += 16) {
            float v[16];
            float4 rcur[2][2];
            if (p.resid) {
#pragma unroll
              for (int j = 0; j < 2; ++j) {
                rcur[j][0] = rnext[j][0];
                rcur[j][1] = rnext[j][1];
              }
              if (cb + 16 < p.tn) tc_load_resid16(p, tok0 + cb + 16, n0r, lane, rnext);
            }
            tmem_ld16(taddr + cb, v);
            if (p.vec) {
              // transpose 32 n x 16 tokens through shared memory, then 16-byte stores of 8 n
#pragma unroll
              for (int e = 0; e < 16; ++e) epi_stage[e * 32 + lane] = __float2half_rn(v[e]);
              __syncwarp();
#pragma unroll
              for (int j = 0; j < 2; ++j) {
                const int t = j * 8 + (lane >> 2), c = lane & 3;
                const uint4 val = *reinterpret_cast<const uint4*>(epi_stage + t * 32 + c * 8);
                const int tok = tok0 + cb + t;
                const int n0 = nb * 128 + q * 32 + c * 8;
                if (p.resid) {
                  // residual add; the four lanes of a token hold its 32 columns of this quarter
                  float ss = (tok < p.M && n0 < p.N) ? tc_add_resid8(p, tok, n0, rcur[j][0], rcur[j][1], val) : 0.f;
                  ss += __shfl_xor_sync(0xffffffffu, ss, 1);
                  ss += __shfl_xor_sync(0xffffffffu, ss, 2);
                  if (c == 0 && tok < p.M && n0 < p.N) p.ssp[(int64_t)(nb * 4 + q) * p.ldss + tok] = ss;
                } else if (tok < p.M && n0 < p.N) {
                  const int64_t off = tc_out_off(p, tok, n0);
                  if (n0 + 8 <= p.N) {
                    *reinterpret_cast<uint4*>(p.ydst[0] + off) = val;
                    for (int d = 1; d < p.ndst; ++d) *reinterpret_cast<uint4*>(p.ydst[d] + off) = val;
                  } else {
                    const __half* hv = reinterpret_cast<const __half*>(&val);
#pragma unroll
                    for (int k = 0; k < 8; ++k)
                      if (n0 + k < p.N) tc_store_all(p, off + k, hv[k]);
                  }
                }
              }
              __syncwarp();
            } else if (ncol < p.N) {
              const int64_t off0 = tc_out_off(p, tok0 + cb, ncol);
              if (p.ndst == 1) {
#pragma unroll
                for (int e = 0; e < 16; ++e)
                  if (tok0 + cb + e < p.M) p.ydst[0][off0 + e * p.ldy] = __float2half_rn(v[e]);
              } else {
#pragma unroll
                for (int e = 0; e < 16; ++e)
                  if (tok0 + cb + e < p.M) tc_store_all(p, off0 + e * p.ldy, __float2half_rn(v[e]));
              }
            }
          }
          tc_fence_before();
          mbar_arrive(acce + buf);
        }
      } else if (!kTicketFixup) {
        // split tile: publish the fp32 partial for tc_fixup_kernel
        if (!failed) {
          tc_fence_after();
          for (int cb = 0; cb < p.tn; cb += 16) {
            float v[16];
            tmem_ld16(taddr + cb, v);
#pragma unroll
            for (int e = 0; e < 16; ++e) __stcg(mine + (int64_t)(cb + e) * 128, v[e]);
          }
          tc_fence_before();
          mbar_arrive(acce + buf);
        }
      } else {
        // split tile finished in this kernel by the part that arrives last. A part that sees every
        // other part already published (acquire peek) adds them to its own sums straight from TMEM;
        // otherwise it publishes its partial and takes a ticket (release/acquire), and the part whose
        // ticket completes the count sums all published partials. Either way the parts are added in
        // part order (the CTAs' order), so the result does not depend on which part came last.
        const int first = tc_cta_of(tile * KT, p), last = tc_cta_of(tile * KT + KT - 1, p);
        const int nparts = last - first + 1;
        if (et == 0) s_flag[0] = (!failed && ld_acquire_gpu_u32(p.tickets + tile) == (uint32_t)(nparts - 1)) ? 1 : 0;
        named_bar_sync(2, 128);
        int mode = s_flag[0];  // 1: last, own sums in TMEM; 2: last, own sums published; 0: not last
        if (mode == 0) {
          if (!failed) {
            tc_fence_after();
            for (int cb = 0; cb < p.tn; cb += 16) {
              float v[16];
              tmem_ld16(taddr + cb, v);
#pragma unroll
              for (int e = 0; e < 16; ++e) __stcg(mine + (int64_t)(cb + e) * 128, v[e]);
            }
            tc_fence_before();
            mbar_arrive(acce + buf);
          }
          named_bar_sync(2, 128);  // every thread's partial is written before the ticket (release)
          if (et == 0)
            s_flag[1] = (!failed && atom_add_acq_rel_gpu(p.tickets + tile, 1u) == (uint32_t)(nparts - 1)) ? 2 : 0;
          named_bar_sync(2, 128);
          mode = s_flag[1];
        }
        if (mode != 0) {
          const int rows = min(p.tn, p.M - tok0);
          if (mode == 1) tc_fence_after();
          for (int t0 = 0; t0 < rows; t0 += 16) {
            float own[16], acc[16];
            if (mode == 1) tmem_ld16(taddr + t0, own);
#pragma unroll
            for (int e = 0; e < 16; ++e) acc[e] = 0.f;
            for (int b = first; b <= last; ++b) {
              float v[16];
              if (mode == 1 && b == (int)blockIdx.x) {
#pragma unroll
                for (int e = 0; e < 16; ++e) v[e] = own[e];
              } else {
                const int bsel = (tc_begin(b, p) >= tile * KT) ? 0 : 1;
                const float* src = p.partials + (((int64_t)b * 2 + bsel) * p.tn + t0) * 128 + nl;
#pragma unroll
                for (int e = 0; e < 16; ++e) v[e] = (t0 + e < rows) ? __ldcg(src + e * 128) : 0.f;
              }
#pragma unroll
              for (int e = 0; e < 16; ++e) acc[e] += v[e];
            }
            if (ncol < p.N) {
#pragma unroll
              for (int e = 0; e < 16; ++e)
                if (t0 + e < rows) tc_store_all(p, tc_out_off(p, tok0 + t0 + e, ncol), __float2half_rn(acc[e]));
            }
          }
          if (mode == 1) {
            tc_fence_before();
            mbar_arrive(acce + buf);
          }
          if (et == 0) atomicExch(p.tickets + tile, 0u);  // every part has arrived: ready for the next call
        }
        named_bar_sync(2, 128);  // the flags are read by every thread before the next segment writes them
      }
    }
  }

  __syncwarp();  // each warp reaches the (warp-aligned) block barrier as a whole after its role code
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(kTcTmemCols)
                 : "memory");
  }
}

// Sums the published fp32 partials of every split tile in CTA order and writes fp16 (the REDUCE step,
// kernels.js:269-282, fp32 throughout). CTA (b, row group) handles the tile that GEMM CTA b's range
// starts inside of, when b is that tile's second CTA, so every split tile is done exactly once.
__global__ void __launch_bounds__(128) tc_fixup_kernel(const TcParams p) {
  __shared__ float up_s[64][8];  // fused gate|up weight: the up rows' sums
  pdl_wait();  // the partials come from the GEMM launched just before
  // the next kernel may start its prologue and weight prefetch now; it reads this kernel's output
  // only after its own grid-dependency wait, which waits for this grid to complete
  pdl_launch_dependents();
  const int b = blockIdx.x, KT = p.ktiles;
  const int cb = tc_begin(b, p);
  if (b == 0 || cb % KT == 0) return;
  const int tile = cb / KT;
  if (tc_cta_of(tile * KT, p) != b - 1) return;
  const int first = b - 1, last = tc_cta_of(tile * KT + KT - 1, p);
  const int tb = tile / p.nblk, nb = tile - tb * p.nblk;
  const int tok0 = tb * p.tn;
  const int rows = min(p.tn, p.M - tok0);
  const int r0 = blockIdx.y * 8;
  if (r0 >= rows) return;
  const int nl = threadIdx.x, ncol = nb * 128 + nl;
  float acc[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) acc[e] = 0.f;
  for (int b0 = first; b0 <= last; b0 += 4) {
    float v[4][8];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int bb = b0 + j;
      if (bb <= last) {
        const int bsel = (tc_begin(bb, p) >= tile * KT) ? 0 : 1;
        const float* src = p.partials + (((int64_t)bb * 2 + bsel) * p.tn + r0) * 128 + nl;
#pragma unroll
        for (int e = 0; e < 8; ++e) v[j][e] = (r0 + e < rows) ? __ldcg(src + e * 128) : 0.f;
      }
    }
#pragma unroll
    for (int j = 0; j < 4; ++j)
      if (b0 + j <= last) {
#pragma unroll
        for (int e = 0; e < 8; ++e) acc[e] += v[j][e];
      }
  }
  if (p.glu) {  // rows 64.. are the up rows of rows 0..63 (see repack.cu): SiLU*mul, fp16 in between
    if (nl >= 64)
#pragma unroll
      for (int e = 0; e < 8; ++e) up_s[nl - 64][e] = acc[e];
    __syncthreads();
    if (nl < 64) {
      const int64_t off0 = tc_out_off(p, tok0 + r0, nb * 64 + nl);
#pragma unroll
      for (int e = 0; e < 8; ++e)
        if (r0 + e < rows) {
          const float g = __half2float(__float2half_rn(acc[e])), u = __half2float(__float2half_rn(up_s[nl][e]));
          tc_store_all(p, off0 + e * p.ldy, __float2half_rn(silu_mul_f32(g, u)));
        }
    }
    return;
  }
  if (p.resid) {  // residual add + per-group sums of squares (see TcParams)
    float ss[8], rv[8];
    float* rrow = p.resid + (int64_t)(tok0 + r0) * p.ldr + ncol;
#pragma unroll
    for (int e = 0; e < 8; ++e) rv[e] = (r0 + e < rows && ncol < p.N) ? rrow[(int64_t)e * p.ldr] : 0.f;
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      ss[e] = 0.f;
      if (r0 + e < rows && ncol < p.N) {
        const float a = rv[e] + __half2float(__float2half_rn(acc[e]));
        rrow[(int64_t)e * p.ldr] = a;
        ss[e] = a * a;
      }
    }
#pragma unroll
    for (int e = 0; e < 8; ++e)
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) ss[e] += __shfl_xor_sync(0xffffffffu, ss[e], o);
    if ((nl & 31) == 0 && ncol < p.N) {
      float* dst = p.ssp + (int64_t)(nb * 4 + (nl >> 5)) * p.ldss + tok0 + r0;
#pragma unroll
      for (int e = 0; e < 8; ++e)
        if (r0 + e < rows) dst[e] = ss[e];
    }
    return;
  }
  if (ncol < p.N) {
    const int64_t off0 = tc_out_off(p, tok0 + r0, ncol);
    if (p.ndst == 1) {
#pragma unroll
      for (int e = 0; e < 8; ++e)
        if (r0 + e < rows) p.ydst[0][off0 + e * p.ldy] = __float2half_rn(acc[e]);
    } else {
#pragma unroll
      for (int e = 0; e < 8; ++e)
        if (r0 + e < rows) tc_store_all(p, off0 + e * p.ldy, __float2half_rn(acc[e]));
    }
  }
}

// ---- host side -------------------------------------------------------------------------------------
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static bool tried = false;
  if (!tried) {
    tried = true;
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  }
  return fn;
}

bool tc_available() { return true; }

size_t tc_partials_bytes(int max_grid) { return (size_t)max_grid * 2 * kTcMaxTn * 128 * sizeof(float); }

// tile_n: requested tokens per tile (0 = automatic).
// General form: x has row stride ldx (elements); the output goes to ndst buffers with row stride ldy,
// starting at column ycol0 (a rank's slice of a gathered buffer).
cudaError_t launch_tc_gemm_ex(const uint8_t* wq, const uint8_t* ws, const uint8_t* wb, const __half* x, int64_t ldx,
                              __half* const* ydst,
                              int ndst, int64_t ldy, int ycol0, float* partials, uint32_t* tickets, int max_tickets,
                              uint32_t* err, int M, int N, int K, int nblk, int ktiles, int tile_n, int grid,
                              cudaStream_t stream, bool pdl, bool ticket_fixup, int glu, float* resid,
                              int64_t ldr, float* ssp, int64_t ldss, const uint32_t* wait_flags, int wait_n) {
  EncodeTiledFn enc = encode_fn();
  if (!enc) return cudaErrorNotSupported;
  int tn = tile_n > 0 ? tile_n : (M >= kTcMaxTn ? kTcMaxTn : ((M + 15) / 16) * 16);
  if (tn < 16 || tn > kTcMaxTn || tn % 16) return cudaErrorInvalidValue;
  if (ndst < 1 || ndst > kTcMaxDst || ldx < K || (ldx * 2) % 16 != 0) return cudaErrorInvalidValue;
  TcParams p;
  p.wq = wq;
  p.ws = ws;
  p.wb = wb;
  p.glu = glu;
  for (int d = 0; d < kTcMaxDst; ++d) p.ydst[d] = d < ndst ? ydst[d] : nullptr;
  p.ndst = ndst;
  p.ldy = ldy;
  p.ycol0 = ycol0;
  p.vec = (ldy % 8 == 0 && ycol0 % 8 == 0) ? 1 : 0;
  for (int d = 0; d < ndst; ++d)
    if (reinterpret_cast<uintptr_t>(ydst[d]) & 15) p.vec = 0;
  if (wait_flags && (wait_n < 1 || wait_n > 8)) return cudaErrorInvalidValue;
  p.wait_flags = wait_flags;
  p.wait_n = wait_n;
  p.resid = resid;
  p.ldr = ldr;
  p.ssp = ssp;
  p.ldss = ldss;
  p.partials = partials;
  p.tickets = tickets;
  p.err = err;
  p.M = M;
  p.N = N;
  p.K = K;
  p.nblk = nblk;
  p.ktiles = ktiles;
  p.tn = tn;
  p.ntb = (M + tn - 1) / tn;
  if ((int64_t)p.ntb * nblk > max_tickets) return cudaErrorInvalidValue;
  const int64_t total = (int64_t)p.ntb * nblk * ktiles;
  if (total > INT32_MAX) return cudaErrorInvalidValue;
  p.total = (int)total;
  if (grid < 1) return cudaErrorInvalidValue;
  p.grid = grid < p.total ? grid : p.total;
  const int tiles = p.ntb * nblk;
  // the fused SiLU*mul epilogue stores 8 outputs at a time and has no in-kernel ticket fix-up
  if (glu && (!p.vec || ticket_fixup || N % 128)) return cudaErrorInvalidValue;
  // the residual epilogue: 16-byte residual accesses of 8 columns, whole 32-column groups, the
  // fix-up kernel for split tiles, no fused gate|up
  if (resid && (!p.vec || ticket_fixup || glu || N % 32 || ldr % 4 || ldr < N || !ssp || ldss < M ||
                (reinterpret_cast<uintptr_t>(resid) & 15)))
    return cudaErrorInvalidValue;
  p.dpq = tiles / p.grid;
  // every CTA's stream-K range must hold at least one unit: an empty range inside a split tile's
  // CTA span would count as a part that never arrives. With fewer leftover units than CTAs, one wave
  // of whole tiles moves into the stream-K part.
  if (p.dpq > 0 && (int64_t)(tiles - p.dpq * p.grid) * ktiles < p.grid && tiles % p.grid != 0) --p.dpq;
  p.sk_base = p.dpq * p.grid * ktiles;
  p.sk_total = p.total - p.sk_base;

  CUtensorMap tmap;
  cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)M};
  cuuint64_t strides[1] = {(cuuint64_t)ldx * 2};
  cuuint32_t box[2] = {64u, (cuuint32_t)tn};
  cuuint32_t estr[2] = {1u, 1u};
  CUresult r = enc(&tmap, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<__half*>(x), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return cudaErrorInvalidValue;

  static std::atomic<bool> configured[64] = {};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  if (!configured[dev]) {
    e = cudaFuncSetAttribute(tc_gemm_kernel<true, false>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kTcSmem);
    if (e == cudaSuccess)
      e = cudaFuncSetAttribute(tc_gemm_kernel<false, false>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kTcSmem);
    if (e == cudaSuccess)
      e = cudaFuncSetAttribute(tc_gemm_kernel<true, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kTcSmem);
    if (e == cudaSuccess)
      e = cudaFuncSetAttribute(tc_gemm_kernel<false, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kTcSmem);
    if (e != cudaSuccess) return e;
    configured[dev] = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(p.grid, 1, 1);
  cfg.blockDim = dim3(kTcThreads, 1, 1);
  cfg.dynamicSmemBytes = kTcSmem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (ticket_fixup)
    return wb ? cudaLaunchKernelEx(&cfg, tc_gemm_kernel<true, true>, p, tmap)
              : cudaLaunchKernelEx(&cfg, tc_gemm_kernel<true, false>, p, tmap);
  e = wb ? cudaLaunchKernelEx(&cfg, tc_gemm_kernel<false, true>, p, tmap)
         : cudaLaunchKernelEx(&cfg, tc_gemm_kernel<false, false>, p, tmap);
  if (e != cudaSuccess) return e;
  // any CTA whose range starts inside a tile leaves that tile split
  bool split = false;
  for (int b = 1; b < p.grid && !split; ++b)
    split = ((p.sk_base + (((int64_t)b * p.sk_total) / p.grid)) % ktiles) != 0;
  if (!split) return cudaSuccess;
  cudaLaunchConfig_t fcfg = cfg;
  fcfg.gridDim = dim3(p.grid, (p.tn + 7) / 8, 1);
  fcfg.blockDim = dim3(128, 1, 1);
  fcfg.dynamicSmemBytes = 0;
  return cudaLaunchKernelEx(&fcfg, tc_fixup_kernel, p);
}

cudaError_t launch_tc_gemm(const uint8_t* wq, const uint8_t* ws, const uint8_t* wb, const __half* x, __half* y,
                           float* partials, uint32_t* tickets, int max_tickets, uint32_t* err, int M, int N, int K,
                           int nblk, int ktiles, int tile_n, int grid, cudaStream_t stream, bool pdl,
                           bool ticket_fixup, int glu) {
  __half* dst[1] = {y};
  return launch_tc_gemm_ex(wq, ws, wb, x, K, dst, 1, glu ? N / 2 : N, 0, partials, tickets, max_tickets, err, M, N, K,
                           nblk, ktiles, tile_n, grid, stream, pdl, ticket_fixup, glu, nullptr, 0, nullptr, 0,
                           nullptr, 0);
}

}  // namespace s4

// ---- allocation-free entry point ------------------------------------------------------------------
// Some callers cannot allocate device memory when they run a matmul: a host whose memory manager
// already owns the device's whole budget, or a serving loop that must not take cudaMalloc's implicit
// device-wide synchronisation. s4_matmul_noalloc gives them the tcgen05 split-K GEMM with its scratch
// (split-K partials, tile arrival counters, error word) in the static array below instead of context
// memory. Every GPU that loads this library holds the array until the process exits. All calls share
// it, so calls that overlap on the GPU (different streams, or concurrent host threads) race.
namespace {
constexpr size_t kStaticScratchBytes = 8u << 20;                         // 8 MiB
constexpr size_t kStaticTicketCount = 16384;                             // tile counters
constexpr size_t kStaticErrOffset = kStaticTicketCount * sizeof(uint32_t);
constexpr size_t kStaticPartialOffset = kStaticErrOffset + 256;
constexpr size_t kStaticPartialBytes = kStaticScratchBytes - kStaticPartialOffset;
}  // namespace

static __device__ __align__(256) unsigned char g_s4_static_scratch[kStaticScratchBytes];

// Device address of g_s4_static_scratch per device (the symbol itself names a host-side stand-in).
// Looked up by the first call on each device; concurrent first calls store the same address.
static std::atomic<void*> g_static_scratch_addr[64];

static int static_scratch(int dev, uint8_t** base) {
  void* ptr = g_static_scratch_addr[dev].load(std::memory_order_acquire);
  if (!ptr) {
    // set-up, once per device, with that device current
    const cudaError_t e = cudaGetSymbolAddress(&ptr, g_s4_static_scratch);
    if (e != cudaSuccess || !ptr)
      return s4::record_error(S4_ERR_CUDA, "s4_matmul_noalloc: cudaGetSymbolAddress of the static scratch failed");
    g_static_scratch_addr[dev].store(ptr, std::memory_order_release);
  }
  *base = static_cast<uint8_t*>(ptr);
  return S4_OK;
}

extern "C" int s4_matmul_noalloc(const s4_weight* w, const void* x, int M, void* y, void* stream) {
  using namespace s4;
  if (!w) return record_error(S4_ERR_INVALID, "s4_matmul_noalloc: NULL weight");
  if (M < 0) return record_error(S4_ERR_INVALID, "s4_matmul_noalloc: M must be >= 0");
  if (M == 0) return S4_OK;
  if (!x || !y) return record_error(S4_ERR_INVALID, "s4_matmul_noalloc: NULL x or y");
  if (w->glu) return record_error(S4_ERR_UNSUPPORTED, "s4_matmul_noalloc: fused gate|up weights run through s4_matmul");
  if ((reinterpret_cast<uintptr_t>(x) & 15) || (reinterpret_cast<uintptr_t>(y) & 15))
    return record_error(S4_ERR_INVALID, "s4_matmul_noalloc: x and y must be 16-byte aligned");
  // the weight records its own device and SM count: the call needs no live context
  const int dev = w->device;
  if (dev < 0 || dev >= 64) return record_error(S4_ERR_INVALID, "s4_matmul_noalloc: device ordinal out of range");
  const int tn = M >= kTcMaxTn ? kTcMaxTn : ((M + 15) / 16) * 16;
  const long long tiles = (long long)((M + tn - 1) / tn) * w->nblk;
  if (tiles > (long long)kStaticTicketCount) {
    char msg[256];
    snprintf(msg, sizeof(msg),
             "s4_matmul_noalloc: M=%d, N=%d needs %lld (token block, n-block) tiles; the static scratch holds "
             "%zu (ceil(M/256) * ceil(N/128) <= %zu)",
             M, w->N, tiles, kStaticTicketCount, kStaticTicketCount);
    return record_error(S4_ERR_INVALID, msg);
  }
  DeviceGuard guard(dev);
  if (!guard.ok) return record_error(S4_ERR_CUDA, "s4_matmul_noalloc: cudaSetDevice failed");
  uint8_t* base = nullptr;
  int rc = static_scratch(dev, &base);
  if (rc != S4_OK) return rc;
  uint32_t* tickets = reinterpret_cast<uint32_t*>(base);
  uint32_t* err = reinterpret_cast<uint32_t*>(base + kStaticErrOffset);
  float* partials = reinterpret_cast<float*>(base + kStaticPartialOffset);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  // Nothing needs clearing per call: split tiles are summed by the fix-up kernel, which uses no tile
  // counters, and the error word accumulates until s4_noalloc_check_errors clears it.
  // CTAs: whole tiles need no partials, so a CTA count that divides the tile count (at least half the
  // SMs) runs at any size; otherwise stream-K with two partial slots of tn x 128 fp32 per CTA, as many
  // CTAs as the array holds
  const int max_grid = (int)(kStaticPartialBytes / (2ull * tn * 128 * sizeof(float)));
  int grid = w->sm_count < max_grid ? w->sm_count : max_grid;
  for (int g = w->sm_count; g * 2 >= w->sm_count && g > grid; --g)
    if (tiles % g == 0) {
      grid = g;
      break;
    }
  // split tiles are summed by the fix-up kernel launched right after (it reads the partials from the
  // same static array); a second launch allocates nothing either
  const cudaError_t e = launch_tc_gemm(w->wq, w->ws, w->wb, static_cast<const __half*>(x), static_cast<__half*>(y), partials, tickets,
                     (int)kStaticTicketCount, err, M, w->N, w->K, w->nblk, w->ktiles, tn, grid, st, true, false, 0);
  if (e != cudaSuccess) return record_error(S4_ERR_CUDA, "s4_matmul_noalloc: tcgen05 GEMM launch failed");
  return S4_OK;
}

extern "C" int s4_noalloc_check_errors(int device, uint32_t* flags, int clear) {
  using namespace s4;
  if (!flags) return record_error(S4_ERR_INVALID, "s4_noalloc_check_errors: NULL flags");
  if (device < 0 || device >= 64) return record_error(S4_ERR_INVALID, "s4_noalloc_check_errors: bad device");
  DeviceGuard guard(device);
  if (!guard.ok) return record_error(S4_ERR_CUDA, "s4_noalloc_check_errors: cudaSetDevice failed");
  uint8_t* base = nullptr;
  int rc = static_scratch(device, &base);
  if (rc != S4_OK) return rc;
  cudaError_t e = cudaDeviceSynchronize();
  if (e == cudaSuccess) e = cudaMemcpy(flags, base + kStaticErrOffset, sizeof(uint32_t), cudaMemcpyDeviceToHost);
  if (e == cudaSuccess && clear) e = cudaMemset(base + kStaticErrOffset, 0, sizeof(uint32_t));
  if (e != cudaSuccess) return record_error(S4_ERR_CUDA, "s4_noalloc_check_errors: reading the error word failed");
  return S4_OK;
}
