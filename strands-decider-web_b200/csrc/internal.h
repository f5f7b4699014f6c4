// Internal definitions shared by the library's translation units (not part of the C ABI).
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include <vector>

#include "../../include/s4mm.h"

namespace s4 {
// Sets the calling thread's s4_last_error() message and returns `code`.
int record_error(int code, const char* msg);

// One entry of the dispatch table: calls with M <= max_m on a weight of K columns and N rows (0 =
// any) use `family`; for the tcgen05 GEMM, `tile` tokens per tile and `split` CTAs (0 = automatic),
// split tiles summed by a second kernel or by their last CTA (`fixup`, kFixup*).
struct Bucket {
  int max_m;
  int family;
  int tile;
  int split;
  int fixup = 0;
  int K = 0;
  int N = 0;
};
constexpr int kFixupAuto = 0;
constexpr int kFixupKernel = 1;
constexpr int kFixupCta = 2;

// Restores the caller's current device on scope exit.
struct DeviceGuard {
  int prev = -1;
  bool ok = false;
  explicit DeviceGuard(int dev) {
    if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
    ok = (prev == dev) || (cudaSetDevice(dev) == cudaSuccess);
  }
  ~DeviceGuard() {
    if (prev >= 0) cudaSetDevice(prev);
  }
};

}  // namespace s4

struct s4_ctx {
  int device = 0;
  int sm_count = 0;
  cudaStream_t stream = nullptr;  // used by the synchronous host-pointer calls
  float* partials = nullptr;      // tcgen05 split-K partials
  uint32_t* tickets = nullptr;    // tcgen05 tile arrival counters (self-resetting)
  uint32_t* err = nullptr;        // device error word
  float* norm_ss = nullptr;       // per-32-column sums of squares of s4_matmul_add_rmsnorm (kNormSums floats)
  void* dx = nullptr;             // staging for s4_matmul_host
  void* dy = nullptr;
  size_t dx_cap = 0, dy_cap = 0;
  double* wire_pow = nullptr;     // 2^(-r/4096) table of the wire scale decoder (first wire call)
  std::vector<s4::Bucket> table;
  s4::Bucket forced{0, S4_FAMILY_AUTO, 0, 0, 0, 0, 0};
  uint64_t launches = 0;
  bool pdl = true;    // launch with programmatic dependent launch (env S4_PDL=0 turns it off)
  int ticket_fixup = -1;  // split tcgen05 tiles: -1 by the table / automatic rule, 1 always summed by their
                          // last CTA in-kernel, 0 always by the fix-up kernel (env S4_TICKET_FIXUP=1 / 0)
};

struct s4_weight {
  s4_ctx* ctx = nullptr;
  int device = -1;  // the context's device: freeing or reading back the weight needs no live context
  int sm_count = 0;  // the device's SM count (the allocation-free matmul sizes its grid without a context)
  int N = 0, K = 0, nblk = 0, ktiles = 0;
  uint8_t* wq = nullptr;
  uint8_t* ws = nullptr;
  uint8_t* wb = nullptr;  // asymmetric formats: per-32-block fp16 biases in the layout of ws
  int glu = 0;            // fused gate|up weight (rows permuted, see repack.cu): matmuls write SiLU*mul, N / 2 wide
  size_t wq_bytes = 0, ws_bytes = 0;
  // symmetric 2-bit formats: the same weight in a 2-bit decode layout (2048 bytes per chunk, scales
  // shared with ws) that the decode GEMV streams instead of wq; nullptr for every other weight
  uint8_t* wq2 = nullptr;
  size_t wq2_bytes = 0;
};

