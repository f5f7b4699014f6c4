// One 16-row x 64-K tile of the decode GEMV math, shared by the per-launch GEMV (gemv.cu) and the
// chained persistent GEMV (chain.cu). Weights are the 16-row mma.sync operand, tokens the 8 columns.
#pragma once
#include "common.cuh"

namespace s4 {

// One k-tile of one sub-tile: w = lane's 16 bytes (words (g,b0) (g+8,b0) (g,b1) (g+8,b1)),
// sc = scales in the same order, xrow = this lane's activation row at the k-tile.
template <int MG>
__device__ __forceinline__ void gemv_tile(const uint4 w, const uint2 sc, const uint8_t* xrow, int xgroup, bool kin1,
                                          const bool (&xok)[MG], float (&acc)[MG][4]) {
  const uint32_t wr[4] = {w.x, w.y, w.z, w.w};
  const float2 s0 = __half22float2(*reinterpret_cast<const __half2*>(&sc.x));
  const float2 s1 = __half22float2(*reinterpret_cast<const __half2*>(&sc.y));
#pragma unroll
  for (int blk = 0; blk < 2; ++blk) {
    uint32_t ha[4], hb[4];
    i4x8_to_h2x4_centered(wr[2 * blk + 0], ha);  // row g
    i4x8_to_h2x4_centered(wr[2 * blk + 1], hb);  // row g + 8
    const float sg = blk ? s1.x : s0.x, sg8 = blk ? s1.y : s0.y;
#pragma unroll
    for (int mg = 0; mg < MG; ++mg) {
      uint4 xv = make_uint4(0, 0, 0, 0);
      if (xok[mg] && (blk == 0 || kin1))
        xv = *reinterpret_cast<const uint4*>(xrow + mg * xgroup + blk * 64);
      float d[4];
      mma_16816_zero(d, ha[0], hb[0], ha[1], hb[1], xv.x, xv.y);
      mma_16816(d, ha[2], hb[2], ha[3], hb[3], xv.z, xv.w);
      acc[mg][0] = fmaf(sg, d[0], acc[mg][0]);
      acc[mg][1] = fmaf(sg, d[1], acc[mg][1]);
      acc[mg][2] = fmaf(sg8, d[2], acc[mg][2]);
      acc[mg][3] = fmaf(sg8, d[3], acc[mg][3]);
    }
  }
}

// The same tile with one activation row pointer per token group, already at this k-tile, and both
// 32-blocks inside K: no predicates. A lane whose token is past M reads a valid row instead
// (min(token, M - 1)): token columns of the MMA are independent and those outputs are never stored.
template <int MG>
__device__ __forceinline__ void gemv_tile_rows(const uint4 w, const uint2 sc, const uint8_t* const (&xr)[MG],
                                               float (&acc)[MG][4]) {
  const uint32_t wr[4] = {w.x, w.y, w.z, w.w};
  const float2 s0 = __half22float2(*reinterpret_cast<const __half2*>(&sc.x));
  const float2 s1 = __half22float2(*reinterpret_cast<const __half2*>(&sc.y));
  uint4 xv[MG][2];
#pragma unroll
  for (int mg = 0; mg < MG; ++mg)
#pragma unroll
    for (int blk = 0; blk < 2; ++blk) xv[mg][blk] = *reinterpret_cast<const uint4*>(xr[mg] + blk * 64);
#pragma unroll
  for (int blk = 0; blk < 2; ++blk) {
    uint32_t ha[4], hb[4];
    i4x8_to_h2x4_centered(wr[2 * blk + 0], ha);
    i4x8_to_h2x4_centered(wr[2 * blk + 1], hb);
    const float sg = blk ? s1.x : s0.x, sg8 = blk ? s1.y : s0.y;
#pragma unroll
    for (int mg = 0; mg < MG; ++mg) {
      float d[4];
      mma_16816_zero(d, ha[0], hb[0], ha[1], hb[1], xv[mg][blk].x, xv[mg][blk].y);
      mma_16816(d, ha[2], hb[2], ha[3], hb[3], xv[mg][blk].z, xv[mg][blk].w);
      acc[mg][0] = fmaf(sg, d[0], acc[mg][0]);
      acc[mg][1] = fmaf(sg, d[1], acc[mg][1]);
      acc[mg][2] = fmaf(sg8, d[2], acc[mg][2]);
      acc[mg][3] = fmaf(sg8, d[3], acc[mg][3]);
    }
  }
}

// The same tile from the native 2-bit decode layout: w = the lane's two words (rows g and g + 8, both
// 32-blocks of the k-tile), converted to the same fragments as the int4 form, then the same math.
template <int MG>
__device__ __forceinline__ void gemv_tile_rows2(const uint2 w, const uint2 sc, const uint8_t* const (&xr)[MG],
                                                float (&acc)[MG][4]) {
  const float2 s0 = __half22float2(*reinterpret_cast<const __half2*>(&sc.x));
  const float2 s1 = __half22float2(*reinterpret_cast<const __half2*>(&sc.y));
  uint4 xv[MG][2];
#pragma unroll
  for (int mg = 0; mg < MG; ++mg)
#pragma unroll
    for (int blk = 0; blk < 2; ++blk) xv[mg][blk] = *reinterpret_cast<const uint4*>(xr[mg] + blk * 64);
#pragma unroll
  for (int blk = 0; blk < 2; ++blk) {
    uint32_t ha[4], hb[4];
    i2x8_to_h2x4_centered(w.x, blk, ha);
    i2x8_to_h2x4_centered(w.y, blk, hb);
    const float sg = blk ? s1.x : s0.x, sg8 = blk ? s1.y : s0.y;
#pragma unroll
    for (int mg = 0; mg < MG; ++mg) {
      float d[4];
      mma_16816_zero(d, ha[0], hb[0], ha[1], hb[1], xv[mg][blk].x, xv[mg][blk].y);
      mma_16816(d, ha[2], hb[2], ha[3], hb[3], xv[mg][blk].z, xv[mg][blk].w);
      acc[mg][0] = fmaf(sg, d[0], acc[mg][0]);
      acc[mg][1] = fmaf(sg, d[1], acc[mg][1]);
      acc[mg][2] = fmaf(sg8, d[2], acc[mg][2]);
      acc[mg][3] = fmaf(sg8, d[3], acc[mg][3]);
    }
  }
}

// Asymmetric formats: the lane's weights dequantised to fp16 first, w = fma(q, scale, bias) per
// element (the f16 form of kernels.js:36), then one mma per 16 K; no per-block scaling after it.
// bi = biases in the order of sc.
template <int MG>
__device__ __forceinline__ void gemv_tile_asym(const uint4 w, const uint2 sc, const uint2 bi, const uint8_t* xrow,
                                               int xgroup, bool kin1, const bool (&xok)[MG], float (&acc)[MG][4]) {
  const uint32_t wr[4] = {w.x, w.y, w.z, w.w};
  const uint32_t sh[4] = {sc.x & 0xFFFFu, sc.x >> 16, sc.y & 0xFFFFu, sc.y >> 16};
  const uint32_t bh[4] = {bi.x & 0xFFFFu, bi.x >> 16, bi.y & 0xFFFFu, bi.y >> 16};
#pragma unroll
  for (int blk = 0; blk < 2; ++blk) {
    uint32_t ha[4], hb[4];
    i4x8_to_h2x4_raw(wr[2 * blk + 0], ha);  // row g
    i4x8_to_h2x4_raw(wr[2 * blk + 1], hb);  // row g + 8
    h2x4_fma(ha, sh[2 * blk + 0], bh[2 * blk + 0]);
    h2x4_fma(hb, sh[2 * blk + 1], bh[2 * blk + 1]);
#pragma unroll
    for (int mg = 0; mg < MG; ++mg) {
      uint4 xv = make_uint4(0, 0, 0, 0);
      if (xok[mg] && (blk == 0 || kin1))
        xv = *reinterpret_cast<const uint4*>(xrow + mg * xgroup + blk * 64);
      mma_16816(acc[mg], ha[0], hb[0], ha[1], hb[1], xv.x, xv.y);
      mma_16816(acc[mg], ha[2], hb[2], ha[3], hb[3], xv.z, xv.w);
    }
  }
}

}  // namespace s4
