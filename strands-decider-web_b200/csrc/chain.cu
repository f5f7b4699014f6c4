// Chained decode GEMV: a list of small-M int4 matmuls (M <= 16) run by ONE persistent launch.
//
// The engine records a forward pass as one list of steps bound to fixed buffers and submits it at
// once (plan() / forward, web/public/engine/engine.js:236-282); at decode every matmul step is a
// GEMV over a few MB of weights. Launched one by one, each GEMV pays a launch, a DRAM ramp and a
// split-K reduction in series (~4-8 us for 3.5-14 MB on B200, well below HBM speed). Here the whole
// list is one launch with one CTA per SM and five warp roles:
//
//  * producer (warp 8, one lane): streams the CTA's weight chunks (128 rows x 64 K: 4096 bytes of
//    nibbles + 512 bytes of scales, contiguous in the repacked layout) into a ring of shared-memory
//    slots, eight consecutive chunks per slot with two 1-D bulk copies (32 KB of nibbles, 4 KB of
//    scales; TMA engine, no multicast), op after op without a pause. Copy size matters: the bytes
//    an SM keeps in flight grow with it (4.6 KB copies streamed at under half the rate);
//  * stager (warp 9, one lane): per op, waits until the op it depends on is complete (if any), then
//    fetches the op's activation window into one of two shared-memory buffers with at most two bulk
//    copies per activation row, one op ahead of the consumers (16-byte pieces from every CTA at
//    once made the window of an 8-row op take ~4 us);
//  * consumers (warps 0-7, one 16-row sub-tile each): only the tile math of gemv_tile.cuh, one
//    ring slot (eight chunks) per batch. At the end of an n-block segment they leave their fp32 sums in shared memory
//    and move on: they never touch global memory, so they never wait for it;
//  * publisher (warp 10): writes the consumers' finished segments to global memory (fp16 outputs,
//    or fp32 partials of split n-blocks), then issues one gpu-scope fence for its own stores and
//    bumps the counters other CTAs wait on. It never waits on other CTAs;
//  * reducer (warp 11): finishes the split n-blocks whose part 0 this CTA holds (below). It waits
//    on other CTAs, which is why it is not the publisher.
//
// Work split: op i's chunks (n-block-major, k-tile-minor) are cut into G equal contiguous ranges,
// one per CTA (stream-K). A 16-row sub-tile that one CTA covers over the whole K range is written
// as fp16 by that CTA. A split sub-tile has parts 0..P-1 in CTA order. Parts 1..P-1 (the start of a
// later CTA's range) are published as fp32 partials with a release-increment of the sub-tile's
// counter. Part 0 belongs to the CTA whose range ends inside the n-block, which usually finishes it
// last: its reducer waits for the counter to reach P-1, adds the parts in order 0..P-1
// (deterministic), writes fp16 and resets the counter. Every final sub-tile increments the op's
// completion counter (release); a dependent op's stager waits for the full count (acquire). All
// waits are bounded (1 s) and report through the error word; a CTA whose wait expired stops.
//
// The launch is cooperative (all CTAs resident), so waiting on other CTAs of the grid cannot
// deadlock. The last CTA to finish resets the completion counters for the next run.
#include <utility>
#include <vector>

#include "common.cuh"
#include "gemv_tile.cuh"
#include "internal.h"

namespace s4 {

constexpr int kChainConsumers = 8;  // warps 0..7
constexpr int kChainProducerWarp = 8;
constexpr int kChainStagerWarp = 9;
constexpr int kChainPublisherWarp = 10;
constexpr int kChainReducerWarp = 11;
constexpr int kChainThreads = 12 * 32;
constexpr int kChainGroup = 8;  // chunks per ring slot (and per consumer batch: 8 independent tiles in
                                // flight per consumer warp; 4 left the warps waiting on dependencies)
constexpr int kChainSlotBytes = kChainGroup * (kChunkWBytes + kChunkSBytes);
constexpr int kChainSlotScales = kChainGroup * kChunkWBytes;  // scales follow the nibbles in a slot
constexpr int kChainMaxSlots = 16;
constexpr int kChainMinSlots = 2;
constexpr int kChainPreferSlots = 3;   // 110 KB of weights in flight per SM before more windows
constexpr int kChainMaxWindows = 8;
constexpr int kChainPhaseWindow = 36 * 1024;  // largest whole-K activation window of an op sharing a phase
constexpr int kChainCachedOps = 64;  // op descriptors kept in shared memory
constexpr int kChainSmemBudget = 216 * 1024;  // dynamic; the static part holds the op cache
constexpr int kChainSegBytes = kChainConsumers * 2 * 32 * 16;  // one segment's fp32 sums (MG <= 2)
constexpr int kChainEv = 2;  // part-0 buffers (the reducer may lag the consumers by this many)

struct ChainOp {
  const uint8_t* wq;
  const uint8_t* ws;
  const __half* x;    // [M][K]
  __half* y;          // [M][N]
  float* partials;    // [nblk][8][maxparts][2][32] float4 (part 0 unused), then the sub-tile
                      // tickets [nblk * 8] (arrivals of parts 1..), see chain_tickets
  int M, N, K, nblk, ktiles;
  int dep;            // op whose output this op reads (-1: none)
  int maxparts;
  int xrow;           // padded activation window row (bytes)
  int phase_base;     // first chunk of this op in its phase's concatenated chunk sequence
  int phase_U;        // chunks of the whole phase; -1 for the dynamic op (no static ranges)
};

__device__ __forceinline__ uint32_t* chain_tickets(const ChainOp& op) {
  return reinterpret_cast<uint32_t*>(reinterpret_cast<uint8_t*>(op.partials) +
                                     (size_t)op.nblk * 8 * op.maxparts * 2 * 32 * 16);
}

struct ChainParams {
  const ChainOp* ops;
  int nops;
  int slots;           // weight ring slots
  int x_off, x_bytes;  // nx activation windows of x_bytes each
  int nx;
  int ev_off;          // kChainEv part-0 buffers, then two publish buffers, kChainSegBytes each
  int bar_off;         // mbarriers: full[slots], empty[slots], xfull[nx], xempty[nx], evfull[kChainEv],
                       // evempty[kChainEv], pubfull[2], pubempty[2]
  uint32_t* op_done;   // [nops] finished sub-tiles
  uint32_t* exit_count;
  uint32_t* dyn_next;  // next unclaimed n-block of the dynamic op
  int dyn_op;          // index of the op whose n-blocks CTAs claim at run time, or -1
  uint32_t* err;
};

// A CTA's share of one op: op-local chunks [c0, c1). The chunks of a phase (consecutive ops none
// of which reads another's output) are concatenated and cut into min(G, U) equal contiguous
// ranges, U = the phase's chunk count, so an n-block is split only where a CTA's range ends.
//
// Only the first and the last n-block of a range can be shared with other CTAs: every n-block in
// between lies wholly inside the range and is written directly. The range and the kinds of its two
// end segments are computed once per launch (chain_range_make, one thread per op at kernel entry, into
// shared memory): they need 64-bit divisions, a slow software sequence, and the role warps that walk
// the op list every launch (skipping ops with empty ranges) used to recompute them per op and per
// segment, ~5 us per launch for a CTA whose range lies in the 14th op.
enum ChainSeg { kSegDirect = 0, kSegPart0 = 1, kSegPartial = 2 };
struct ChainRange {
  int c0, c1;           // op-local chunks [c0, c1)
  int nb0, nb1;         // first and last n-block of the range
  int kind0, part0, np0;  // segment kind, part index and part count of n-block nb0
  int kind1, part1, np1;  // the same for nb1
};
__device__ __forceinline__ int chain_begin(int b, int U, int G) { return (int)(((int64_t)b * U) / G); }
__device__ __forceinline__ int chain_cta_of(int u, int U, int G) { return (int)((((int64_t)u + 1) * G - 1) / U); }
__device__ __forceinline__ void chain_seg_calc(const ChainOp& op, int U, int G, int nb, int b, int* kind, int* part,
                                               int* nparts) {
  const int KT = op.ktiles, base = op.phase_base;
  const int first = chain_cta_of(base + nb * KT, U, G), last = chain_cta_of(base + nb * KT + KT - 1, U, G);
  *nparts = last - first + 1;
  *part = b - first;
  *kind = first == last ? kSegDirect : (*part == 0 ? kSegPart0 : kSegPartial);
}
__device__ __forceinline__ ChainRange chain_range_make(const ChainOp& op, int b, int grid) {
  ChainRange r;
  const int U = op.phase_U, G = min(grid, U);
  const int u0 = b < G ? chain_begin(b, U, G) : 0, u1 = b < G ? chain_begin(b + 1, U, G) : 0;
  const int n = op.nblk * op.ktiles;
  r.c0 = min(max(u0 - op.phase_base, 0), n);
  r.c1 = max(min(u1 - op.phase_base, n), r.c0);
  r.nb0 = r.nb1 = 0;
  r.kind0 = r.kind1 = kSegDirect;
  r.part0 = r.part1 = 0;
  r.np0 = r.np1 = 1;
  if (r.c0 < r.c1) {
    r.nb0 = r.c0 / op.ktiles;
    r.nb1 = (r.c1 - 1) / op.ktiles;
    chain_seg_calc(op, U, G, r.nb0, b, &r.kind0, &r.part0, &r.np0);
    chain_seg_calc(op, U, G, r.nb1, b, &r.kind1, &r.part1, &r.np1);
  }
  return r;
}
// Kind of the segment of n-block nb inside range r (nb within [r.nb0, r.nb1]).
__device__ __forceinline__ int chain_seg_kind(const ChainRange& r, int nb, int* part, int* nparts) {
  if (nb == r.nb0) {
    *part = r.part0;
    *nparts = r.np0;
    return r.kind0;
  }
  if (nb == r.nb1) {
    *part = r.part1;
    *nparts = r.np1;
    return r.kind1;
  }
  *part = 0;
  *nparts = 1;
  return kSegDirect;
}

__device__ __forceinline__ uint32_t ld_acquire_gpu(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void red_relaxed_gpu(uint32_t* p, uint32_t v) {
  asm volatile("red.relaxed.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ void fence_acq_rel_gpu() { asm volatile("fence.acq_rel.gpu;" ::: "memory"); }
// Bounded spin until *p >= target (acquire); false on expiry.
__device__ __forceinline__ bool wait_count(const uint32_t* p, uint32_t target) {
  if (ld_acquire_gpu(p) >= target) return true;
  const uint64_t deadline = globaltimer_ns() + kWaitTimeoutNs;
  while (ld_acquire_gpu(p) < target) {
    if (globaltimer_ns() > deadline) return false;
    __nanosleep(64);
  }
  return true;
}
// 16-byte global -> shared copy through L2 (no L1: the source may have been written by other CTAs
// of this launch), asynchronous until cp_async_wait_all.
__device__ __forceinline__ void cp_async_cg16(void* dst_smem, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst_smem)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

struct ChainSmem {
  int* slot_unit;  // [kChainMaxSlots] n-block of the dynamic op a ring slot holds (-1: no more)
  int* pub_nb;     // [2] n-block of a dynamic segment in a publish buffer (-1: no more)
  uint8_t* ring;
  uint8_t* xbuf;
  float4* ev;   // [2] part-0 sums for the reducer
  float4* pub;  // [2] finished segments for the publisher
  uint64_t *full, *empty, *xfull, *xempty, *evfull, *evempty, *pubfull, *pubempty;
  const ChainOp* ops;  // op descriptor cache (the first kChainCachedOps)
  const ChainRange* rng;  // this CTA's range of each cached op
  int* fail;
};
__device__ __forceinline__ ChainOp chain_op_at(const ChainParams& p, const ChainSmem& sm, int i) {
  return i < kChainCachedOps ? sm.ops[i] : p.ops[i];
}
__device__ __forceinline__ ChainRange chain_range_at(const ChainSmem& sm, const ChainOp& op, int i, int b, int G) {
  return i < kChainCachedOps ? sm.rng[i] : chain_range_make(op, b, G);
}

// fp32 sums of one 16-row sub-tile (lane layout of gemv_tile: rows g, g+8; tokens 2t, 2t+1 per
// 8-token group) -> fp16 y.
template <int MG>
__device__ __forceinline__ void chain_store_y(const ChainOp& op, int nb, int sub, const float (&v)[MG][4]) {
  const int lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  const int n0 = nb * 128 + sub * 16 + g;
#pragma unroll
  for (int mg = 0; mg < MG; ++mg) {
    const int tok = mg * 8 + 2 * t;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int m = tok + (e & 1);
      const int nn = n0 + ((e >> 1) << 3);
      if (m < op.M && nn < op.N) op.y[(int64_t)m * op.N + nn] = __float2half_rn(v[mg][e]);
    }
  }
}

// ---- consumers: end of an n-block segment -----------------------------------------------------------
template <int MG>
__device__ __forceinline__ bool chain_flush(const ChainOp& op, const ChainRange& r, const ChainParams& p,
                                            const ChainSmem& sm, int nb, float (&acc)[MG][4], int& evk, int& pubk) {
  const int sub = threadIdx.x >> 5, lane = threadIdx.x & 31;
  int part, nparts;
  const int kind = chain_seg_kind(r, nb, &part, &nparts);
  float4* dst;
  uint64_t* full;
  if (kind == kSegPart0) {
    const int e = evk % kChainEv;
    if (evk >= kChainEv && !mbar_wait(sm.evempty + e, (uint32_t)((evk / kChainEv) - 1) & 1u)) return false;
    dst = sm.ev + (size_t)e * (kChainSegBytes / 16);
    full = sm.evfull + e;
    ++evk;
  } else {
    const int e = pubk & 1;
    if (pubk >= 2 && !mbar_wait(sm.pubempty + e, (uint32_t)((pubk >> 1) - 1) & 1u)) return false;
    dst = sm.pub + (size_t)e * (kChainSegBytes / 16);
    full = sm.pubfull + e;
    ++pubk;
  }
  dst += (sub * MG) * 32 + lane;
#pragma unroll
  for (int mg = 0; mg < MG; ++mg) dst[mg * 32] = make_float4(acc[mg][0], acc[mg][1], acc[mg][2], acc[mg][3]);
  __syncwarp();
  if (lane == 0) mbar_arrive(full);
#pragma unroll
  for (int mg = 0; mg < MG; ++mg)
#pragma unroll
    for (int e = 0; e < 4; ++e) acc[mg][e] = 0.f;
  return true;
}

// ---- consumers: one op ------------------------------------------------------------------------
template <int MG>
__device__ bool chain_consume(const ChainOp& op, const ChainRange& r, const ChainParams& p, const ChainSmem& sm,
                              int& slot, uint32_t& phase, int xk, int& evk, int& pubk) {
  const int KT = op.ktiles;
  const int sub = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  const int xb = xk % p.nx;
  if (!mbar_wait(sm.xfull + xb, (uint32_t)(xk / p.nx) & 1u) || *(volatile int*)sm.fail) return false;
  const uint8_t* xs = sm.xbuf + xb * p.x_bytes;
  bool xok[MG];
#pragma unroll
  for (int mg = 0; mg < MG; ++mg) xok[mg] = (mg * 8 + g) < op.M;
  const int xgroup = 8 * op.xrow;
  const uint8_t* xl = xs + g * op.xrow + 16 * t;
  const uint8_t* xr[MG];  // per token group; a token past M reads row M - 1 (never stored)
#pragma unroll
  for (int mg = 0; mg < MG; ++mg) xr[mg] = xs + min(mg * 8 + g, op.M - 1) * op.xrow + 16 * t;

  float acc[MG][4];
#pragma unroll
  for (int mg = 0; mg < MG; ++mg)
#pragma unroll
    for (int e = 0; e < 4; ++e) acc[mg][e] = 0.f;
  int nb = r.c0 / KT, kt = r.c0 - nb * KT, wpos = 0;
  for (int g0 = r.c0; g0 < r.c1; g0 += kChainGroup) {
    const int n = min(kChainGroup, r.c1 - g0);
    if (!mbar_wait(sm.full + slot, phase)) return false;
    const uint8_t* ch = sm.ring + slot * kChainSlotBytes;
    uint4 wv[kChainGroup];
    uint2 sc[kChainGroup];
    const uint8_t* wl = ch + sub * 512 + lane * 16;
    const uint8_t* sl = ch + kChainSlotScales + sub * 64 + g * 8;
    if (n == kChainGroup) {
#pragma unroll
      for (int j = 0; j < kChainGroup; ++j) {
        wv[j] = *reinterpret_cast<const uint4*>(wl + j * kChunkWBytes);
        sc[j] = *reinterpret_cast<const uint2*>(sl + j * kChunkSBytes);
      }
    } else {
#pragma unroll
      for (int j = 0; j < kChainGroup; ++j)
        if (j < n) {
          wv[j] = *reinterpret_cast<const uint4*>(wl + j * kChunkWBytes);
          sc[j] = *reinterpret_cast<const uint2*>(sl + j * kChunkSBytes);
        }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(sm.empty + slot);
    if (++slot == p.slots) {
      slot = 0;
      phase ^= 1u;
    }
    if (n == kChainGroup && kt + n <= KT && wpos + n <= KT && (kt + n) * 64 <= op.K) {
      // fast path: a full slot in one n-block and one stretch of the window, all of K in range;
      // the tiles are independent, so the compiler can overlap their latencies
#pragma unroll
      for (int j = 0; j < kChainGroup; ++j) {
        const uint8_t* xj[MG];
#pragma unroll
        for (int mg = 0; mg < MG; ++mg) xj[mg] = xr[mg] + (wpos + j) * 128;
        gemv_tile_rows<MG>(wv[j], sc[j], xj, acc);
      }
      kt += n;
      wpos += n;
      if (wpos == KT) wpos = 0;
      if (kt == KT || g0 + n == r.c1) {
        if (!chain_flush<MG>(op, r, p, sm, nb, acc, evk, pubk)) return false;
      }
      if (kt == KT) {
        kt = 0;
        ++nb;
      }
    } else {
      // the group crosses an n-block boundary or wraps the window: one chunk at a time
      for (int j = 0; j < n; ++j) {
        const int c = g0 + j;
        gemv_tile<MG>(wv[j], sc[j], xl + wpos * 128, xgroup, kt * 64 + 32 < op.K, xok, acc);
        if (kt == KT - 1 || c == r.c1 - 1) {
          if (!chain_flush<MG>(op, r, p, sm, nb, acc, evk, pubk)) return false;
        }
        if (++kt == KT) {
          kt = 0;
          ++nb;
        }
        if (++wpos == KT) wpos = 0;  // window position of the next chunk: (c + 1 - c0) mod KT
      }
    }
  }
  __syncwarp();
  if (lane == 0) mbar_arrive(sm.xempty + xb);
  return true;
}

// ---- publisher: one op's direct and partial segments, in the consumers' order ------------------------
template <int MG>
__device__ bool chain_publish_op(const ChainOp& op, const ChainRange& r, const ChainParams& p, const ChainSmem& sm,
                                 int i, int& pubk) {
  const int lane = threadIdx.x & 31, KT = op.ktiles;
  for (int c = r.c0; c < r.c1;) {
    const int nb = c / KT;
    c = min(r.c1, (nb + 1) * KT);
    int part, nparts;
    const int kind = chain_seg_kind(r, nb, &part, &nparts);
    if (kind == kSegPart0) continue;  // the reducer's
    const int e = pubk & 1;
    if (!mbar_wait(sm.pubfull + e, (uint32_t)(pubk >> 1) & 1u)) return false;
    const float4* src = sm.pub + (size_t)e * (kChainSegBytes / 16) + lane;
    if (kind == kSegDirect) {
      for (int sub = 0; sub < 8; ++sub) {
        float v[MG][4];
#pragma unroll
        for (int mg = 0; mg < MG; ++mg) {
          const float4 f = src[(sub * MG + mg) * 32];
          v[mg][0] = f.x;
          v[mg][1] = f.y;
          v[mg][2] = f.z;
          v[mg][3] = f.w;
        }
        chain_store_y<MG>(op, nb, sub, v);
      }
    } else {
      float4* dst = reinterpret_cast<float4*>(op.partials) + lane;
      for (int sub = 0; sub < 8; ++sub) {
        const size_t base = ((((size_t)nb * 8 + sub) * op.maxparts) + part) * MG * 32;
#pragma unroll
        for (int mg = 0; mg < MG; ++mg) __stcg(dst + base + mg * 32, src[(sub * MG + mg) * 32]);
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(sm.pubempty + e);
    ++pubk;
    fence_acq_rel_gpu();  // this warp's stores above, then the counter bumps (release pattern)
    if (kind == kSegDirect) {
      if (lane == 0) red_relaxed_gpu(p.op_done + i, 8u);
    } else {
      if (lane < 8) red_relaxed_gpu(chain_tickets(op) + nb * 8 + lane, 1u);
    }
  }
  return true;
}

// ---- reducer: the split n-block whose part 0 this CTA holds ---------------------------------------
template <int MG>
__device__ bool chain_reduce(const ChainOp& op, const ChainRange& r, const ChainParams& p, const ChainSmem& sm, int i,
                             int nb, int nparts, int evk) {
  const int lane = threadIdx.x & 31;
  const int e = evk % kChainEv;
  if (!mbar_wait(sm.evfull + e, (uint32_t)(evk / kChainEv) & 1u)) return false;
  bool ok = true;
  if (lane < 8) ok = wait_count(chain_tickets(op) + nb * 8 + lane, (uint32_t)(nparts - 1));
  ok = __all_sync(0xffffffffu, ok);
  __syncwarp();  // lanes 0-7 acquired the counters; order the whole warp's loads after them
  if (!ok) return false;
  float out[8][MG][4];
  const float4* own = sm.ev + (size_t)e * (kChainSegBytes / 16) + lane;
#pragma unroll
  for (int sub = 0; sub < 8; ++sub)
#pragma unroll
    for (int mg = 0; mg < MG; ++mg) {
      const float4 v = own[(sub * MG + mg) * 32];
      out[sub][mg][0] = v.x;
      out[sub][mg][1] = v.y;
      out[sub][mg][2] = v.z;
      out[sub][mg][3] = v.w;
    }
  __syncwarp();
  if (lane == 0) mbar_arrive(sm.evempty + e);  // part 0 is in registers now
  const float4* src = reinterpret_cast<const float4*>(op.partials) + lane;
  for (int q = 1; q < nparts; ++q) {  // parts added in order 1, 2, ...: one round trip per part
    float4 v[8][MG];
#pragma unroll
    for (int sub = 0; sub < 8; ++sub)
#pragma unroll
      for (int mg = 0; mg < MG; ++mg) v[sub][mg] = __ldcg(src + ((((size_t)nb * 8 + sub) * op.maxparts + q) * MG + mg) * 32);
#pragma unroll
    for (int sub = 0; sub < 8; ++sub)
#pragma unroll
      for (int mg = 0; mg < MG; ++mg) {
        out[sub][mg][0] += v[sub][mg].x;
        out[sub][mg][1] += v[sub][mg].y;
        out[sub][mg][2] += v[sub][mg].z;
        out[sub][mg][3] += v[sub][mg].w;
      }
  }
#pragma unroll
  for (int sub = 0; sub < 8; ++sub) chain_store_y<MG>(op, nb, sub, out[sub]);
  if (lane < 8) chain_tickets(op)[nb * 8 + lane] = 0u;  // every part has arrived: ready for the next run
  fence_acq_rel_gpu();
  if (lane == 0) red_relaxed_gpu(p.op_done + i, 8u);
  return true;
}

// ---- the dynamic op -------------------------------------------------------------------------------
// When no op depends on another, the chain's last op is not cut into static ranges: each CTA's
// producer, once its static share is streamed, claims whole n-blocks of it (atomic counter) until
// none is left. A whole n-block needs no split-K partials, and the claims even out the CTAs' random
// speed differences, which otherwise leave every launch waiting for its slowest CTA.

// Producer: stream claimed n-blocks (all K, in groups of kChainGroup chunks) into the ring after
// `seq` slots; a slot whose unit is -1 ends the op.
__device__ bool chain_dyn_produce(const ChainOp& op, const ChainParams& p, const ChainSmem& sm, int& seq,
                                  uint64_t pol) {
  const int KT = op.ktiles;
  for (;;) {
    const int u = (int)atomicAdd(p.dyn_next, 1u);
    const bool last = u >= op.nblk;
    for (int k0 = 0; k0 < (last ? 1 : KT); k0 += kChainGroup, ++seq) {
      const int slot = seq % p.slots;
      if ((seq >= p.slots && !mbar_wait(sm.empty + slot, (uint32_t)((seq / p.slots) - 1) & 1u)) || *(volatile int*)sm.fail)
        return false;
      if (last) {
        sm.slot_unit[slot] = -1;
        mbar_arrive(sm.full + slot);  // no bytes: the sentinel completes the slot's phase by itself
        break;
      }
      sm.slot_unit[slot] = u;
      const int n = min(kChainGroup, KT - k0);
      const int64_t g0 = (int64_t)u * KT + k0;
      uint8_t* dst = sm.ring + slot * kChainSlotBytes;
      mbar_arrive_expect_tx(sm.full + slot, (uint32_t)n * (kChunkWBytes + kChunkSBytes));
      bulk_g2s(dst, op.wq + g0 * kChunkWBytes, (uint32_t)n * kChunkWBytes, sm.full + slot, pol);
      bulk_g2s(dst + kChainSlotScales, op.ws + g0 * kChunkSBytes, (uint32_t)n * kChunkSBytes, sm.full + slot, pol);
    }
    if (last) return true;
  }
}

// Consumers: whole n-blocks from the ring (window = all of K), each flushed as a direct segment
// tagged with its n-block; a publish buffer tagged -1 ends the op.
template <int MG>
__device__ bool chain_dyn_consume(const ChainOp& op, const ChainParams& p, const ChainSmem& sm, int& slot,
                                  uint32_t& phase, int xk, int& pubk) {
  const int KT = op.ktiles;
  const int sub = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  const int xb = xk % p.nx;
  if (!mbar_wait(sm.xfull + xb, (uint32_t)(xk / p.nx) & 1u) || *(volatile int*)sm.fail) return false;
  const uint8_t* xs = sm.xbuf + xb * p.x_bytes;
  const uint8_t* xl = xs + g * op.xrow + 16 * t;
  const int xgroup = 8 * op.xrow;
  bool xok[MG];
  const uint8_t* xr[MG];  // a token past M reads row M - 1 (never stored)
#pragma unroll
  for (int mg = 0; mg < MG; ++mg) {
    xok[mg] = (mg * 8 + g) < op.M;
    xr[mg] = xs + min(mg * 8 + g, op.M - 1) * op.xrow + 16 * t;
  }
  const bool kfull = (op.K % 64) == 0;
  float acc[MG][4];
  int kt = 0;
  for (;;) {
    if (!mbar_wait(sm.full + slot, phase)) return false;
    const int u = sm.slot_unit[slot];
    const uint8_t* ch = sm.ring + slot * kChainSlotBytes;
    if (u >= 0) {
      if (kt == 0) {
#pragma unroll
        for (int mg = 0; mg < MG; ++mg)
#pragma unroll
          for (int e = 0; e < 4; ++e) acc[mg][e] = 0.f;
      }
      const int n = min(kChainGroup, KT - kt);
      uint4 wv[kChainGroup];
      uint2 sc[kChainGroup];
#pragma unroll
      for (int j = 0; j < kChainGroup; ++j)
        if (j < n) {
          wv[j] = *reinterpret_cast<const uint4*>(ch + j * kChunkWBytes + sub * 512 + lane * 16);
          sc[j] = *reinterpret_cast<const uint2*>(ch + kChainSlotScales + j * kChunkSBytes + sub * 64 + g * 8);
        }
      __syncwarp();
      if (lane == 0) mbar_arrive(sm.empty + slot);
      if (n == kChainGroup && kfull) {
#pragma unroll
        for (int j = 0; j < kChainGroup; ++j) {
          const uint8_t* xj[MG];
#pragma unroll
          for (int mg = 0; mg < MG; ++mg) xj[mg] = xr[mg] + (kt + j) * 128;
          gemv_tile_rows<MG>(wv[j], sc[j], xj, acc);
        }
      } else {
#pragma unroll
        for (int j = 0; j < kChainGroup; ++j)
          if (j < n) gemv_tile<MG>(wv[j], sc[j], xl + (kt + j) * 128, xgroup, (kt + j) * 64 + 32 < op.K, xok, acc);
      }
      kt += n;
    }
    if (++slot == p.slots) {
      slot = 0;
      phase ^= 1u;
    }
    if (u >= 0 && kt < KT) continue;
    // an n-block is complete (or the op ended): hand it to the publisher
    const int e = pubk & 1;
    if (pubk >= 2 && !mbar_wait(sm.pubempty + e, (uint32_t)((pubk >> 1) - 1) & 1u)) return false;
    ++pubk;
    if (u >= 0) {
      float4* dst = sm.pub + (size_t)e * (kChainSegBytes / 16) + (sub * MG) * 32 + lane;
#pragma unroll
      for (int mg = 0; mg < MG; ++mg) dst[mg * 32] = make_float4(acc[mg][0], acc[mg][1], acc[mg][2], acc[mg][3]);
    }
    if (threadIdx.x == 0) sm.pub_nb[e] = u;
    __syncwarp();
    if (lane == 0) mbar_arrive(sm.pubfull + e);
    if (u < 0) break;
    kt = 0;
  }
  __syncwarp();
  if (lane == 0) mbar_arrive(sm.xempty + xb);
  return true;
}

// Publisher: the dynamic op's segments, in the consumers' order.
template <int MG>
__device__ bool chain_dyn_publish(const ChainOp& op, const ChainParams& p, const ChainSmem& sm, int& pubk) {
  const int lane = threadIdx.x & 31;
  for (;;) {
    const int e = pubk & 1;
    if (!mbar_wait(sm.pubfull + e, (uint32_t)(pubk >> 1) & 1u)) return false;
    ++pubk;
    const int nb = sm.pub_nb[e];
    if (nb < 0) return true;
    const float4* src = sm.pub + (size_t)e * (kChainSegBytes / 16) + lane;
    for (int sub = 0; sub < 8; ++sub) {
      float v[MG][4];
#pragma unroll
      for (int mg = 0; mg < MG; ++mg) {
        const float4 f = src[(sub * MG + mg) * 32];
        v[mg][0] = f.x;
        v[mg][1] = f.y;
        v[mg][2] = f.z;
        v[mg][3] = f.w;
      }
      chain_store_y<MG>(op, nb, sub, v);
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(sm.pubempty + e);
    fence_acq_rel_gpu();
    if (lane == 0) red_relaxed_gpu(p.op_done + p.dyn_op, 8u);
  }
}

// MG: 8-token groups of every op of the launch (1 if all ops have M <= 8, else 2). One MG per
// kernel keeps the code small enough for the instruction cache (five warp roles share it).
template <int MG>
__global__ void __launch_bounds__(kChainThreads, 1) chain_kernel(const ChainParams p) {
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ int s_fail;
  __shared__ int s_slot_unit[kChainMaxSlots];
  __shared__ int s_pub_nb[2];
  __shared__ __align__(16) ChainOp s_ops[kChainCachedOps];
  __shared__ ChainRange s_rng[kChainCachedOps];
  __shared__ int s_act[kChainCachedOps];  // ops with a range in this CTA (and the dynamic op), in order
  __shared__ int s_nact;                  // their count, or -1 when the op list is longer than the cache
  ChainSmem sm;
  sm.slot_unit = s_slot_unit;
  sm.pub_nb = s_pub_nb;
  sm.ring = smem;
  sm.xbuf = smem + p.x_off;
  sm.ev = reinterpret_cast<float4*>(smem + p.ev_off);
  sm.pub = sm.ev + kChainEv * (kChainSegBytes / 16);
  sm.full = reinterpret_cast<uint64_t*>(smem + p.bar_off);
  sm.empty = sm.full + p.slots;
  sm.xfull = sm.empty + p.slots;
  sm.xempty = sm.xfull + p.nx;
  sm.evfull = sm.xempty + p.nx;
  sm.evempty = sm.evfull + kChainEv;
  sm.pubfull = sm.evempty + kChainEv;
  sm.pubempty = sm.pubfull + 2;
  sm.ops = s_ops;
  sm.rng = s_rng;
  sm.fail = &s_fail;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int G = gridDim.x, b = blockIdx.x;
  {
    const int ncached = min(p.nops, kChainCachedOps) * (int)(sizeof(ChainOp) / 4);
    const uint32_t* src = reinterpret_cast<const uint32_t*>(p.ops);
    uint32_t* dst = reinterpret_cast<uint32_t*>(s_ops);
    for (int q = threadIdx.x; q < ncached; q += kChainThreads) dst[q] = src[q];
    // this CTA's range of every cached op, one thread per op (ordered before use by the barrier below)
    for (int i = threadIdx.x; i < min(p.nops, kChainCachedOps); i += kChainThreads)
      s_rng[i] = chain_range_make(p.ops[i], b, G);
  }
  if (threadIdx.x == 0) {
    for (int s = 0; s < p.slots; ++s) {
      mbar_init(sm.full + s, 1);
      mbar_init(sm.empty + s, kChainConsumers);
    }
    for (int k = 0; k < p.nx; ++k) {
      mbar_init(sm.xfull + k, 1);
      mbar_init(sm.xempty + k, kChainConsumers);
    }
    for (int k = 0; k < kChainEv; ++k) {
      mbar_init(sm.evfull + k, kChainConsumers);
      mbar_init(sm.evempty + k, 1);
    }
    for (int k = 0; k < 2; ++k) {
      mbar_init(sm.pubfull + k, kChainConsumers);
      mbar_init(sm.pubempty + k, 1);
    }
    fence_mbar_init();
    s_fail = 0;
  }
  __syncwarp();  // each warp reaches the (warp-aligned) block barrier as a whole after its role code
  __syncthreads();
  // the ops this CTA takes part in: every role walks only these (a walk over all ops cost each CTA
  // ~0.1 us per op it has no range in)
  if (threadIdx.x == 0) {
    int n = -1;
    if (p.nops <= kChainCachedOps) {
      n = 0;
      for (int i = 0; i < p.nops; ++i)
        if (s_rng[i].c0 < s_rng[i].c1 || i == p.dyn_op) s_act[n++] = i;
    }
    s_nact = n;
  }
  __syncthreads();
  const int nwalk = s_nact >= 0 ? s_nact : p.nops;
  // Launched with programmatic stream serialization, the next grid in the stream may start its
  // CTAs as ours exit. Only the producer runs before the previous grid has completed: it reads
  // nothing but the weights (immutable after upload) and fills this CTA's ring. Every other role
  // reads activations, completion counters or scratch the previous grid may write, so it waits.
  // (Both instructions are no-ops in a cooperative launch.)
  pdl_launch_dependents();
  if (warp != kChainProducerWarp) pdl_wait();

  bool ok = true;
  if (warp == kChainProducerWarp) {
    // ---------------- producer: the CTA's chunks of every op, in order ----------------
    if (lane == 0) {
      const uint64_t pol = policy_evict_first();
      int seq = 0;
      for (int ii = 0; ii < nwalk && ok; ++ii) {
        const int i = s_nact >= 0 ? s_act[ii] : ii;
        const ChainOp op = chain_op_at(p, sm, i);
        const ChainRange r = chain_range_at(sm, op, i, b, G);
        for (int g0 = r.c0; g0 < r.c1; g0 += kChainGroup, ++seq) {
          const int n = min(kChainGroup, r.c1 - g0);
          const int slot = seq % p.slots;
          if ((seq >= p.slots && !mbar_wait(sm.empty + slot, (uint32_t)((seq / p.slots) - 1) & 1u)) ||
              *(volatile int*)&s_fail) {
            ok = false;
            break;
          }
          uint8_t* dst = sm.ring + slot * kChainSlotBytes;
          mbar_arrive_expect_tx(sm.full + slot, (uint32_t)n * (kChunkWBytes + kChunkSBytes));
          bulk_g2s(dst, op.wq + (int64_t)g0 * kChunkWBytes, (uint32_t)n * kChunkWBytes, sm.full + slot, pol);
          bulk_g2s(dst + kChainSlotScales, op.ws + (int64_t)g0 * kChunkSBytes, (uint32_t)n * kChunkSBytes, sm.full + slot,
                   pol);
        }
      }
      if (ok && p.dyn_op >= 0) {
        pdl_wait();  // the claim counter is reset by the previous run's last CTA
        ok = chain_dyn_produce(chain_op_at(p, sm, p.dyn_op), p, sm, seq, pol);
      }
      if (!ok) {
        // copies still in flight land before the CTA exits (bounded)
        const uint64_t deadline = globaltimer_ns() + kWaitTimeoutNs;
        const int first = seq > p.slots ? seq - p.slots : 0;
        for (int q = first; q < seq; ++q)
          if (!mbar_wait_until(sm.full + (q % p.slots), (uint32_t)(q / p.slots) & 1u, deadline)) break;
      }
    }
  } else if (warp == kChainStagerWarp) {
    // ---------------- stager: dependency wait + activation window, one op ahead ----------------
    if (lane == 0) {
      int xk = 0;
      const uint64_t pol = policy_evict_last();  // every CTA reads the same activations
      for (int ii = 0; ii < nwalk && ok; ++ii) {
        const int i = s_nact >= 0 ? s_act[ii] : ii;
        const ChainOp op = chain_op_at(p, sm, i);
        ChainRange r = chain_range_at(sm, op, i, b, G);
        if (i == p.dyn_op) {  // the whole of K: any n-block may be claimed
          r.c0 = 0;
          r.c1 = op.ktiles;
        }
        if (r.c0 >= r.c1) continue;
        const int xb = xk % p.nx;
        ok = !(xk >= p.nx && !mbar_wait(sm.xempty + xb, (uint32_t)((xk / p.nx) - 1) & 1u));
        if (ok && op.dep >= 0) {
          const ChainOp d = chain_op_at(p, sm, op.dep);
          ok = wait_count(p.op_done + op.dep, (uint32_t)d.nblk * 8u);
          // the input was written by other CTAs through the generic proxy; the bulk copies below
          // read it through the async proxy
          asm volatile("fence.proxy.async.global;" ::: "memory");
        }
        if (!ok || *(volatile int*)&s_fail) {
          ok = false;
          break;
        }
        // window k-tiles kt_start, kt_start + 1, ... (mod KT): one or two contiguous pieces per row
        const int KT = op.ktiles;
        const int kt_start = r.c0 % KT;
        const int n_win = min(r.c1 - r.c0, KT);
        const int n1 = min(n_win, KT - kt_start);
        const uint32_t b1 = (uint32_t)(min((kt_start + n1) * 64, op.K) - kt_start * 64) * 2u;
        const uint32_t b2 = n_win > n1 ? (uint32_t)min((n_win - n1) * 64, op.K) * 2u : 0u;
        uint8_t* xs = sm.xbuf + xb * p.x_bytes;
        mbar_arrive_expect_tx(sm.xfull + xb, (uint32_t)op.M * (b1 + b2));
        for (int row = 0; row < op.M; ++row) {
          const __half* xr = op.x + (int64_t)row * op.K;
          bulk_g2s(xs + row * op.xrow, xr + kt_start * 64, b1, sm.xfull + xb, pol);
          if (b2) bulk_g2s(xs + row * op.xrow + n1 * 128, xr, b2, sm.xfull + xb, pol);
        }
        ++xk;
      }
      if (!ok) {
        // window copies still in flight land before the CTA exits (bounded)
        const uint64_t deadline = globaltimer_ns() + kWaitTimeoutNs;
        for (int q = (xk > p.nx ? xk - p.nx : 0); q < xk; ++q)
          if (!mbar_wait_until(sm.xfull + (q % p.nx), (uint32_t)(q / p.nx) & 1u, deadline)) break;
      }
    }
  } else if (warp == kChainPublisherWarp) {
    // ---------------- publisher ----------------
    int pubk = 0;
    for (int ii = 0; ii < nwalk && ok; ++ii) {
        const int i = s_nact >= 0 ? s_act[ii] : ii;
      const ChainOp op = chain_op_at(p, sm, i);
      const ChainRange r = chain_range_at(sm, op, i, b, G);
      if (r.c0 >= r.c1) continue;
      ok = chain_publish_op<MG>(op, r, p, sm, i, pubk);
    }
    if (ok && p.dyn_op >= 0) ok = chain_dyn_publish<MG>(chain_op_at(p, sm, p.dyn_op), p, sm, pubk);
  } else if (warp == kChainReducerWarp) {
    // ---------------- reducer ----------------
    int evk = 0;
    for (int ii = 0; ii < nwalk && ok; ++ii) {
        const int i = s_nact >= 0 ? s_act[ii] : ii;
      const ChainOp op = chain_op_at(p, sm, i);
      const ChainRange r = chain_range_at(sm, op, i, b, G);
      if (r.c0 >= r.c1) continue;
      const int nb = (r.c1 - 1) / op.ktiles;  // only the last segment of a range can be a part 0
      int part, nparts;
      if (chain_seg_kind(r, nb, &part, &nparts) != kSegPart0) continue;
      ok = chain_reduce<MG>(op, r, p, sm, i, nb, nparts, evk);
      ++evk;
    }
  } else {
    // ---------------- consumers ----------------
    int slot = 0, xk = 0, evk = 0, pubk = 0;
    uint32_t phase = 0;
    for (int ii = 0; ii < nwalk && ok; ++ii) {
        const int i = s_nact >= 0 ? s_act[ii] : ii;
      const ChainOp op = chain_op_at(p, sm, i);
      const ChainRange r = chain_range_at(sm, op, i, b, G);
      if (r.c0 >= r.c1) continue;
      ok = chain_consume<MG>(op, r, p, sm, slot, phase, xk, evk, pubk);
      ++xk;
    }
    if (ok && p.dyn_op >= 0) ok = chain_dyn_consume<MG>(chain_op_at(p, sm, p.dyn_op), p, sm, slot, phase, xk, pubk);
  }
  if (!ok && lane == 0) {
    set_error(p.err, kErrWaitTimeout);
    s_fail = 1;
  }
  __syncwarp();  // each warp reaches the (warp-aligned) block barrier as a whole after its role code
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    const uint32_t prev = atomicAdd(p.exit_count, 1u);
    if (prev == (uint32_t)(G - 1)) {  // last CTA of the run: completion counters back to zero
      __threadfence();
      for (int i = 0; i < p.nops; ++i) p.op_done[i] = 0u;
      *p.dyn_next = 0u;
      *p.exit_count = 0u;
      __threadfence();
    }
  }
}

}  // namespace s4

// ---- host side -------------------------------------------------------------------------------------
using s4::ChainOp;

struct s4_chain {
  s4_ctx* ctx;
  int device;  // the context's device (chain_destroy needs no live context)
  int nops;
  int grid;
  int slots;
  int x_off, x_bytes, nx, ev_off, bar_off, smem;
  int mg;  // token groups of the launch: 2 if any op has M > 8
  ChainOp* d_ops;
  uint8_t* d_scratch;  // partials, tickets, op_done, exit_count
  uint32_t* op_done;
  uint32_t* exit_count;
  uint32_t* dyn_next;
  int dyn_op;  // index of the dynamic op (the last), or -1
  std::vector<ChainOp> ops;
};

namespace s4 {

int chain_create(s4_ctx* ctx, int nops, const s4_weight* const* w, const void* const* x, void* const* y, const int* M,
                 const int* dep, s4_chain** out, const char** why) {
  *why = nullptr;
  const int G = ctx->sm_count;
  std::vector<ChainOp> ops(nops);
  size_t scratch = 0;
  int xmax = 0;
  std::vector<size_t> part_off(nops);
  for (int i = 0; i < nops; ++i) {
    const s4_weight* wi = w[i];
    ChainOp& o = ops[i];
    o.wq = wi->wq;
    o.ws = wi->ws;
    o.x = static_cast<const __half*>(x[i]);
    o.y = static_cast<__half*>(y[i]);
    o.M = M[i];
    o.N = wi->N;
    o.K = wi->K;
    o.nblk = wi->nblk;
    o.ktiles = wi->ktiles;
    o.dep = dep ? dep[i] : -1;
    if (wi->wb) return *why = "asymmetric-format weights run through s4_matmul, not a chain", S4_ERR_UNSUPPORTED;
    if (wi->glu) return *why = "fused gate|up (SiLU*mul) weights run through s4_matmul, not a chain", S4_ERR_UNSUPPORTED;
    if (o.M < 1 || o.M > 16) return *why = "every op needs 1 <= M <= 16", S4_ERR_INVALID;
    if (o.dep >= i || o.dep < -1) return *why = "dep must name an earlier op or be -1", S4_ERR_INVALID;
    if ((reinterpret_cast<uintptr_t>(x[i]) & 15) || (o.K * 2) % 16) return *why = "x must be 16-byte aligned", S4_ERR_INVALID;
  }
  // With no dependencies at all the ops may run in any order: the ops that need a phase of their own
  // (whole-K activation window above kChainPhaseWindow) go first, so their split-K reductions overlap
  // the streaming of the merged phase and the launch ends on a phase split at most twice per CTA.
  // The small op with the most n-blocks then becomes the dynamic op (claimed n-block by n-block at
  // run time, after every static range): it goes last and is left out of the phases.
  int dyn_op = -1;
  {
    bool any_dep = false;
    for (int i = 0; i < nops; ++i) any_dep |= ops[i].dep >= 0;
    if (!any_dep) {
      std::vector<ChainOp> big, small;
      for (int i = 0; i < nops; ++i)
        (ops[i].M * (ops[i].ktiles * 128 + 64) > kChainPhaseWindow ? big : small).push_back(ops[i]);
      long long total = 0;
      for (int i = 0; i < nops; ++i) total += (long long)ops[i].nblk * ops[i].ktiles;
      int pick = -1;
      for (int i = 0; i < (int)small.size(); ++i)
        if (pick < 0 || small[i].nblk > small[pick].nblk) pick = i;
      if (nops >= 2 && pick >= 0 && small[pick].nblk >= 16 &&
          (long long)small[pick].nblk * small[pick].ktiles * 100 <= total * 35) {
        const ChainOp d = small[pick];
        small.erase(small.begin() + pick);
        small.push_back(d);
        dyn_op = nops - 1;
      }
      ops = big;
      ops.insert(ops.end(), small.begin(), small.end());
    }
  }
  const int nstatic = dyn_op >= 0 ? nops - 1 : nops;
  // phases: runs of consecutive ops none of which reads another op of the run. An op whose whole-K
  // activation window would exceed kChainPhaseWindow ("big") never shares a phase with the others
  // (its range within a merged phase could span whole n-blocks, i.e. all of K); consecutive big ops
  // share one while every op's window for the phase's per-CTA range still fits: a CTA then streams
  // one longer range instead of one short range per op (fewer part-filled ring slots, windows and
  // split-K parts per n-block).
  std::vector<int> phase_start(nops);
  {
    auto is_big = [&](const ChainOp& o) { return o.M * (o.ktiles * 128 + 64) > kChainPhaseWindow; };
    int start = 0;
    long long U = 0;  // chunks of the current phase so far
    for (int i = 0; i < nstatic; ++i) {
      const ChainOp& o = ops[i];
      const long long Uo = (long long)o.nblk * o.ktiles;
      bool join = i > 0 && o.dep < start && is_big(o) == is_big(ops[i - 1]);
      if (join && is_big(o)) {
        const long long U2 = U + Uo;
        const long long Gp = U2 < G ? U2 : G;
        const long long per_cta = (U2 + Gp - 1) / Gp;
        for (int q = start; q <= i && join; ++q) {
          const long long n_win = per_cta < ops[q].ktiles ? per_cta : ops[q].ktiles;
          join = (long long)ops[q].M * (n_win * 128 + 64) <= kChainPhaseWindow;
        }
      }
      if (!join) {
        start = i;
        U = 0;
      }
      phase_start[i] = start;
      U += Uo;
    }
  }
  for (int i = 0; i < nstatic;) {
    int j = i, U = 0;
    while (j < nstatic && phase_start[j] == i) {
      ops[j].phase_base = U;
      U += ops[j].nblk * ops[j].ktiles;
      ++j;
    }
    for (int q = i; q < j; ++q) ops[q].phase_U = U;
    i = j;
  }
  if (dyn_op >= 0) {
    ops[dyn_op].phase_base = 0;
    ops[dyn_op].phase_U = -1;
  }
  for (int i = 0; i < nops; ++i) {
    ChainOp& o = ops[i];
    if (i == dyn_op) {  // whole n-blocks only: no partials, a window of all of K
      o.maxparts = 1;
      o.xrow = o.ktiles * 128 + 64;
    } else {
      const int U = o.nblk * o.ktiles;
      const int Gp = o.phase_U < G ? o.phase_U : G;
      const int per_cta = (o.phase_U + Gp - 1) / Gp;
      const int min_cta = o.phase_U / Gp;  // >= 1
      o.maxparts = (o.ktiles + min_cta - 1) / min_cta + 1;  // CTAs one n-block can span
      if (o.maxparts > Gp) o.maxparts = Gp;
      int n_win = per_cta < U ? per_cta : U;
      if (n_win > o.ktiles) n_win = o.ktiles;
      o.xrow = n_win * 128 + 64;
    }
    const int xb = o.M * o.xrow;
    if (xb > xmax) xmax = xb;
    part_off[i] = scratch;  // partials sized for MG = 2, the tickets right after (chain_tickets)
    scratch += (size_t)o.nblk * 8 * o.maxparts * 2 * 32 * 16;
    scratch += (size_t)o.nblk * 8 * 4;
    scratch = (scratch + 255) & ~(size_t)255;
  }
  xmax = (xmax + 127) & ~127;
  // shared memory: the weight ring first (at least kChainPreferSlots slots when possible), then as
  // many activation windows (2..kChainMaxWindows) as fit: more windows = more ops of lookahead for
  // the stager, which hides the activation fetch of small ops
  const int fixed = (kChainEv + 2) * kChainSegBytes + 2 * (2 * kChainMaxSlots + 2 * kChainMaxWindows + 12) * 8 + 256;
  const int avail = kChainSmemBudget - fixed;
  if (avail < 2 * xmax + kChainMinSlots * kChainSlotBytes)
    return *why = "activation window too large for shared memory (M * K range)", S4_ERR_UNSUPPORTED;
  int slots = (avail - 2 * xmax) / kChainSlotBytes;
  if (slots > kChainPreferSlots) slots = kChainPreferSlots;
  int nx = (avail - slots * kChainSlotBytes) / xmax;
  if (nx > kChainMaxWindows) nx = kChainMaxWindows;
  slots = (avail - nx * xmax) / kChainSlotBytes;
  if (slots > kChainMaxSlots) slots = kChainMaxSlots;

  s4_chain* c = new s4_chain();
  c->ctx = ctx;
  c->device = ctx->device;
  c->nops = nops;
  c->grid = G;
  c->slots = slots;
  c->nx = nx;
  c->mg = 1;
  for (int i = 0; i < nops; ++i)
    if (ops[i].M > 8) c->mg = 2;
  c->x_off = slots * kChainSlotBytes;
  c->x_bytes = xmax;
  c->ev_off = c->x_off + nx * xmax;
  c->bar_off = c->ev_off + (kChainEv + 2) * kChainSegBytes;
  c->smem = c->bar_off + (2 * slots + 2 * nx + 2 * kChainEv + 4) * 8;
  const size_t ctr_off = scratch;
  scratch += (size_t)(nops + 2) * 4;  // op_done[nops], exit_count, dyn_next
  cudaError_t e = cudaMalloc(&c->d_scratch, scratch);
  if (e == cudaSuccess) e = cudaMemset(c->d_scratch, 0, scratch);
  if (e == cudaSuccess) e = cudaMalloc(&c->d_ops, sizeof(ChainOp) * nops);
  if (e != cudaSuccess) {
    cudaFree(c->d_scratch);
    delete c;
    return *why = "device allocation failed", S4_ERR_NOMEM;
  }
  for (int i = 0; i < nops; ++i) ops[i].partials = reinterpret_cast<float*>(c->d_scratch + part_off[i]);
  c->op_done = reinterpret_cast<uint32_t*>(c->d_scratch + ctr_off);
  c->exit_count = c->op_done + nops;
  c->dyn_next = c->exit_count + 1;
  c->dyn_op = dyn_op;
  e = cudaMemcpy(c->d_ops, ops.data(), sizeof(ChainOp) * nops, cudaMemcpyHostToDevice);
  if (e != cudaSuccess) {
    cudaFree(c->d_ops);
    cudaFree(c->d_scratch);
    delete c;
    return *why = "op table upload failed", S4_ERR_CUDA;
  }
  c->ops = std::move(ops);  // no allocation after the device buffers exist
  *out = c;
  return S4_OK;
}

cudaError_t chain_launch(s4_chain* c, uint32_t* err, cudaStream_t stream, bool cooperative) {
  static bool configured[64] = {};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  if (!configured[dev]) {
    e = cudaFuncSetAttribute(chain_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, kChainSmemBudget);
    if (e == cudaSuccess)
      e = cudaFuncSetAttribute(chain_kernel<2>, cudaFuncAttributeMaxDynamicSharedMemorySize, kChainSmemBudget);
    if (e != cudaSuccess) return e;
    configured[dev] = true;
  }
  ChainParams p;
  p.ops = c->d_ops;
  p.nops = c->nops;
  p.slots = c->slots;
  p.x_off = c->x_off;
  p.x_bytes = c->x_bytes;
  p.nx = c->nx;
  p.ev_off = c->ev_off;
  p.bar_off = c->bar_off;
  p.op_done = c->op_done;
  p.exit_count = c->exit_count;
  p.dyn_next = c->dyn_next;
  p.dyn_op = c->dyn_op;
  p.err = err;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(c->grid, 1, 1);
  cfg.blockDim = dim3(kChainThreads, 1, 1);
  cfg.dynamicSmemBytes = c->smem;
  cfg.stream = stream;
  // Every CTA must be resident at once (CTAs wait on one another's counters). A cooperative launch
  // guarantees that on any stream. A programmatic-dependent launch does too when runs follow one
  // another on ONE stream: it begins only after every CTA of the previous grid has started (each
  // triggers at entry), and that grid finishes without ours, freeing every SM. Chained runs on other
  // streams must not overlap a programmatic one.
  cudaLaunchAttribute attr[1];
  if (cooperative) {
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
  } else {
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
  }
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return c->mg == 2 ? cudaLaunchKernelEx(&cfg, chain_kernel<2>, p) : cudaLaunchKernelEx(&cfg, chain_kernel<1>, p);
}

void chain_destroy(s4_chain* c) {
  DeviceGuard guard(c->device);
  cudaFree(c->d_ops);
  cudaFree(c->d_scratch);
  delete c;
}

int chain_info(const s4_chain* c, int* grid, int* slots, int* smem) {
  if (grid) *grid = c->grid;
  if (slots) *slots = c->slots;
  if (smem) *smem = c->smem;
  return S4_OK;
}

}  // namespace s4
