// Download-format scale decode (wire.js:1-33): 8-bit log codes -> fp16 scales, on the device.
//
// A scale tensor [N][G] travels as N row headers of 4 bytes (m = fp16 bits of the row's largest
// magnitude, j = u16 step, little-endian) followed by N*G codes c = sign << 7 | k. A code decodes to
//   toHalf(fromHalf(m) * 2^(-k*j/4096)) | sign << 15
// with the product in double. fromHalf (wire.js:5) reads exponent 31 as a finite power of two;
// toHalf (wire.js:8-15) rounds to float32 and then builds the fp16 bits with integer steps, stored
// mod 2^16. Both are followed here bit for bit, so every header maps like the JS maps it.
//
// 2^(-i/4096) = 2^-(i >> 12) * pow_table[i & 4095], the table holding the correctly rounded
// 2^(-r/4096) (built on the host). The power-of-two factor is exact except where the double result
// is subnormal, and there |m * p| < 2^-1005, which every path rounds to an fp16 zero.
//
// The JS caches the 128 magnitudes of a row (a speed-up only); each thread here decodes one code.
// Reads are bytes, so the wire buffer needs no alignment; the output is 2-byte aligned fp16.
#include "common.cuh"

namespace s4 {

__device__ __forceinline__ double wire_from_half(uint32_t h) {
  const int e = (h >> 10) & 31, f = h & 1023;
  const double v = e ? ldexp((double)(1024 + f), e - 25) : ldexp((double)f, -24);
  return (h & 0x8000u) ? -v : v;
}

__device__ __forceinline__ uint32_t wire_to_half(double x) {
  const float F = __double2float_rn(x);
  const uint32_t b = __float_as_uint(F);
  const int e = (int)((b >> 23) & 255) - 112;
  const uint32_t rest = b & 0x1fffu;
  long long h;
  if (e > 0 && e < 31) {
    h = (e << 10) | ((b >> 13) & 1023);
    if (rest > 0x1000u || (rest == 0x1000u && (h & 1))) ++h;
  } else if (e >= 31) {
    h = 0x7c00;
  } else {  // subnormal fp16: units of 2^-24, rounded by floor arithmetic as the JS does
    const double u = __dmul_rn((double)F, 16777216.0);
    const double fl = floor(u);
    const double d = __dsub_rn(u, fl);
    h = (long long)fl;
    if (d > 0.5 || (d == 0.5 && (h & 1))) ++h;
  }
  return (uint32_t)h & 0xffffu;
}

__global__ void wire_scales_kernel(const uint8_t* __restrict__ wire, int N, int G, const double* __restrict__ pow_table,
                                   uint16_t* __restrict__ out) {
  const int64_t total = (int64_t)N * G;
  const uint8_t* codes = wire + 4 * (int64_t)N;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / G;
    const uint8_t* hdr = wire + 4 * r;
    const uint32_t hb = (uint32_t)__ldg(hdr) | ((uint32_t)__ldg(hdr + 1) << 8);
    const uint32_t j = (uint32_t)__ldg(hdr + 2) | ((uint32_t)__ldg(hdr + 3) << 8);
    const uint32_t c = __ldg(codes + i);
    const uint32_t ij = (c & 127u) * j;  // <= 127 * 65535
    const double p = ldexp(__ldg(pow_table + (ij & 4095u)), -(int)(ij >> 12));
    out[i] = (uint16_t)(wire_to_half(__dmul_rn(wire_from_half(hb), p)) | ((c & 128u) << 8));
  }
}

cudaError_t launch_wire_scales(const uint8_t* wire, int N, int G, const double* pow_table, uint16_t* out, int sms,
                               cudaStream_t stream) {
  const int64_t total = (int64_t)N * G;
  const int threads = 256;
  const int64_t need = (total + threads - 1) / threads;
  const int grid = (int)(need < (int64_t)sms * 8 ? need : (int64_t)sms * 8);
  wire_scales_kernel<<<grid, threads, 0, stream>>>(wire, N, G, pow_table, out);
  return cudaGetLastError();
}

}  // namespace s4
