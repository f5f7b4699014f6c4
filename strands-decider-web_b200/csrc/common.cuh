// Shared device helpers for the s4mm kernels (sm_100a only).
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#if defined(__CUDA_ARCH__) && (__CUDA_ARCH__ < 1000)
#error "s4mm kernels are written for sm_100a (B200) only"
#endif

namespace s4 {

// Repacked layout constants (see repack.cu).
constexpr int kRowsPerBlock = 128;      // output rows per n-block
constexpr int kKPerTile = 64;           // K per k-tile = two quant blocks of 32
constexpr int kChunkWBytes = 4096;      // int4 bytes of one (n-block, k-tile) chunk
constexpr int kChunkSBytes = 512;       // fp16 scale bytes of one chunk

// Error bits written to the context's device error word.
constexpr uint32_t kErrWaitTimeout = 1u;   // a bounded mbarrier wait expired
constexpr uint32_t kErrBadShape = 2u;      // kernel saw arguments outside its contract
constexpr uint32_t kErrTmem = 4u;          // TMEM allocation returned an unusable address

// Bounded waits give up after this many nanoseconds of %globaltimer.
constexpr uint64_t kWaitTimeoutNs = 1000000000ull;

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// ---- mbarrier -------------------------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
// try_wait with a suspend-time hint: a warp whose phase is not complete sleeps (up to the hint)
// until the phase completes instead of spinning and taking issue slots from working warps.
constexpr uint32_t kSuspendHintNs = 1000000u;
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity), "r"(kSuspendHintNs)
      : "memory");
  return ok != 0;
}
// Non-blocking check of phase `parity` (no suspend): the fast path of a wait whose phase is usually
// complete already.
__device__ __forceinline__ bool mbar_test_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}
// Wait for phase `parity` of `bar` until %globaltimer passes `deadline`; false on expiry.
__device__ __forceinline__ bool mbar_wait_until(uint64_t* bar, uint32_t parity, uint64_t deadline) {
  const uint32_t a = smem_u32(bar);
  while (true) {
    if (mbar_try_wait(a, parity)) return true;
    if (globaltimer_ns() > deadline) return false;
  }
}
// Wait for phase `parity` of `bar` to complete; false if kWaitTimeoutNs passed first.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
  const uint32_t a = smem_u32(bar);
  if (mbar_test_wait(a, parity)) return true;
  if (mbar_try_wait(a, parity)) return true;
  const uint64_t deadline = globaltimer_ns() + kWaitTimeoutNs;
  while (true) {
    if (mbar_try_wait(a, parity)) return true;
    if (globaltimer_ns() > deadline) return false;
  }
}

// ---- bulk async copies (TMA engine, no multicast) ------------------------------------------------
// 1-D global -> shared copy of `bytes` (multiple of 16, both addresses 16-byte aligned),
// completing `bytes` transactions on `bar`.
__device__ __forceinline__ void bulk_g2s(void* dst_smem, const void* src_gmem, uint32_t bytes, uint64_t* bar,
                                         uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
          smem_u32(dst_smem)),
      "l"(src_gmem), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}
__device__ __forceinline__ uint64_t policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}
__device__ __forceinline__ uint64_t policy_evict_last() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
  return p;
}

// ---- programmatic dependent launch ----------------------------------------------------------------
// Wait until the previous kernel in the stream has completed and its writes are visible.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
// Allow the next kernel in the stream to start launching its CTAs.
__device__ __forceinline__ void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// ---- named barriers --------------------------------------------------------------------------------
__device__ __forceinline__ void named_bar_sync(int id, int nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// ---- global loads ----------------------------------------------------------------------------------
__device__ __forceinline__ uint4 ldg_nc_v4(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}
__device__ __forceinline__ float4 ldcg_f4(const float4* p) { return __ldcg(p); }

// ---- tensor-core mma (legacy warp-level path, used by the decode GEMV) -----------------------------
// D = A(16x16 f16, row) * B(16x8 f16, col) + C, f32 accumulate.
__device__ __forceinline__ void mma_16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                          uint32_t b0, uint32_t b1) {
  // not volatile: no side effects, so the compiler may interleave independent MMAs with other work
  asm(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// Same with C = 0: d = A * B (no registers to clear first).
__device__ __forceinline__ void mma_16816_zero(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                               uint32_t b0, uint32_t b1) {
  asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%10,%10,%10,%10};"
      : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "f"(0.0f));
}

// ---- int4 -> fp16 ---------------------------------------------------------------------------------
// Device word layout: nibbles 0-3 hold k0,k2,k4,k6 and nibbles 4-7 hold k1,k3,k5,k7 of eight
// consecutive K values of one row. Output h[i] = half2(k_{2i} - 8, k_{2i+1} - 8), exact.
// Method: OR-ing a nibble into the mantissa of fp16 1024.0 (bits 0x6400) gives 1024 + q exactly
// (Kim et al. 2022, "Who Says Elephants Can't Run"; FasterTransformer's int4 converter).
__device__ __forceinline__ uint32_t lop3_and_or(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t r;
  asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(r) : "r"(a), "r"(b), "r"(c));  // (a & b) | c
  return r;
}
__device__ __forceinline__ void i4x8_to_h2x4_centered(uint32_t w, uint32_t (&h)[4]) {
  const uint32_t kLo = 0x000f000fu, kHi = 0x00f000f0u, kMagic = 0x64006400u;
  const uint32_t sub1032 = 0x64086408u;  // half2(1032, 1032)
  const uint32_t mul16 = 0x2c002c00u;    // half2(1/16, 1/16)
  const uint32_t add72 = 0xd480d480u;    // half2(-72, -72)
  const uint32_t top = w >> 8;
  uint32_t t0 = lop3_and_or(w, kLo, kMagic);
  uint32_t t1 = lop3_and_or(w, kHi, kMagic);
  uint32_t t2 = lop3_and_or(top, kLo, kMagic);
  uint32_t t3 = lop3_and_or(top, kHi, kMagic);
  asm("sub.f16x2 %0, %1, %2;" : "=r"(h[0]) : "r"(t0), "r"(sub1032));
  asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(h[1]) : "r"(t1), "r"(mul16), "r"(add72));
  asm("sub.f16x2 %0, %1, %2;" : "=r"(h[2]) : "r"(t2), "r"(sub1032));
  asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(h[3]) : "r"(t3), "r"(mul16), "r"(add72));
}

// Symmetric 2-bit: the four half2 (q - 2) pairs of 32-block blk of a word in the native 2-bit decode
// layout (repack2_kernel in format.cu): h[j] = (value 2j, value 2j + 1) of the lane's 8 values, the
// same fragment order i4x8_to_h2x4_centered gives for an int4 word. Each 2-bit field lands in the
// mantissa of 1024 (times 1, 4, 16, 64) and one exact f16 subtract or fma removes the offset.
__device__ __forceinline__ void i2x8_to_h2x4_centered(uint32_t u, int blk, uint32_t (&h)[4]) {
  const uint32_t w = blk ? (u >> 8) : u;
  const uint32_t kMagic = 0x64006400u;
  const uint32_t sub1026 = 0x64026402u;  // half2(1026, 1026)
  const uint32_t mul4 = 0x34003400u;     // half2(1/4, 1/4)
  const uint32_t add258 = 0xdc08dc08u;   // half2(-258, -258)
  const uint32_t mul16 = 0x2c002c00u;    // half2(1/16, 1/16)
  const uint32_t add66 = 0xd420d420u;    // half2(-66, -66)
  const uint32_t mul64 = 0x24002400u;    // half2(1/64, 1/64)
  const uint32_t add18 = 0xcc80cc80u;    // half2(-18, -18)
  const uint32_t t0 = lop3_and_or(w, 0x00030003u, kMagic);
  const uint32_t t1 = lop3_and_or(w, 0x000c000cu, kMagic);
  const uint32_t t2 = lop3_and_or(w, 0x00300030u, kMagic);
  const uint32_t t3 = lop3_and_or(w, 0x00c000c0u, kMagic);
  asm("sub.f16x2 %0, %1, %2;" : "=r"(h[0]) : "r"(t0), "r"(sub1026));
  asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(h[1]) : "r"(t1), "r"(mul4), "r"(add258));
  asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(h[2]) : "r"(t2), "r"(mul16), "r"(add66));
  asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(h[3]) : "r"(t3), "r"(mul64), "r"(add18));
}

// silu(g) * u in fp32 (wgsl.js:81-90); every kernel that produces SiLU*mul outputs uses this one.
__device__ __forceinline__ float silu_mul_f32(float g, float u) { return g / (1.0f + expf(-g)) * u; }

// Same element order, uncentered: fp16 q in [0, 15] (asymmetric formats, w = q * scale + bias).
__device__ __forceinline__ void i4x8_to_h2x4_raw(uint32_t w, uint32_t (&h)[4]) {
  const uint32_t kLo = 0x000f000fu, kHi = 0x00f000f0u, kMagic = 0x64006400u;
  const uint32_t sub1024 = 0x64006400u;  // half2(1024, 1024)
  const uint32_t mul16 = 0x2c002c00u;    // half2(1/16, 1/16)
  const uint32_t add64 = 0xd400d400u;    // half2(-64, -64)
  const uint32_t top = w >> 8;
  uint32_t t0 = lop3_and_or(w, kLo, kMagic);
  uint32_t t1 = lop3_and_or(w, kHi, kMagic);
  uint32_t t2 = lop3_and_or(top, kLo, kMagic);
  uint32_t t3 = lop3_and_or(top, kHi, kMagic);
  asm("sub.f16x2 %0, %1, %2;" : "=r"(h[0]) : "r"(t0), "r"(sub1024));
  asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(h[1]) : "r"(t1), "r"(mul16), "r"(add64));
  asm("sub.f16x2 %0, %1, %2;" : "=r"(h[2]) : "r"(t2), "r"(sub1024));
  asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(h[3]) : "r"(t3), "r"(mul16), "r"(add64));
}

// h[e] = h[e] * s + b for four half2 words (one fp16 scale and bias broadcast to both halves).
__device__ __forceinline__ void h2x4_fma(uint32_t (&h)[4], uint32_t s16, uint32_t b16) {
  const uint32_t s2 = s16 | (s16 << 16), b2 = b16 | (b16 << 16);
#pragma unroll
  for (int e = 0; e < 4; ++e) asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(h[e]) : "r"(h[e]), "r"(s2), "r"(b2));
}

// Atomic add with release (orders this thread's, and by cumulativity its CTA's barrier-ordered,
// earlier writes) and acquire (orders later reads) semantics at GPU scope.
__device__ __forceinline__ uint32_t atom_add_acq_rel_gpu(uint32_t* p, uint32_t v) {
  uint32_t old;
  asm volatile("atom.add.acq_rel.gpu.global.u32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
  return old;
}

// Load with acquire semantics at GPU scope (pairs with a release by another CTA).
__device__ __forceinline__ uint32_t ld_acquire_gpu_u32(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void set_error(uint32_t* err, uint32_t bits) {
  if (err) atomicOr(err, bits);
}

// Cross-GPU flag arrays of the column-sharded prefill (peer.cu): slot q of a rank's own array holds
// the latest epoch rank q has signalled to it; slot kPeerCounterSlot counts the rank's own signals.
constexpr int kPeerCounterSlot = 8;

// Called by one thread of a consumer kernel after its grid-dependency wait: waits until every one
// of the nranks ranks has signalled at least this rank's latest epoch (the kernel before it in the
// stream was this rank's signal, so its counter slot is visible). Acquire at system scope: the
// peers' stores before their signals are then visible to this thread and, after a block barrier, to
// its CTA. Bounded: false after kWaitTimeoutNs.
__device__ __forceinline__ bool peer_wait_all(const uint32_t* own, int nranks) {
  const uint32_t epoch = *reinterpret_cast<const volatile uint32_t*>(own + kPeerCounterSlot);
  const uint64_t deadline = globaltimer_ns() + kWaitTimeoutNs;
  for (int q = 0; q < nranks; ++q) {
    while (true) {
      uint32_t v;
      asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(own + q) : "memory");
      if ((int32_t)(v - epoch) >= 0) break;
      if (globaltimer_ns() > deadline) return false;
      __nanosleep(32);
    }
  }
  return true;
}

}  // namespace s4
