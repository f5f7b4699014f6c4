// Internal definitions shared by the library's translation units (not part of the C ABI).
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include <vector>

#include "../../include/s4mm.h"

namespace s4 {
// Sets the calling thread's s4_last_error() message and returns `code`.
int record_error(int code, const char* msg);

struct Bucket {
  int max_m;
  int family;
  int tile;
  int split;
};

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
  void* dx = nullptr;             // staging for s4_matmul_host
  void* dy = nullptr;
  size_t dx_cap = 0, dy_cap = 0;
  double* wire_pow = nullptr;     // 2^(-r/4096) table of the wire scale decoder (first wire call)
  std::vector<s4::Bucket> table;
  s4::Bucket forced{0, S4_FAMILY_AUTO, 0, 0};
  uint64_t launches = 0;
  bool pdl = true;    // launch with programmatic dependent launch (env S4_PDL=0 turns it off)
  bool ticket_fixup = false;  // split tcgen05 tiles summed by their last CTA in-kernel (env S4_TICKET_FIXUP=1)
};

struct s4_weight {
  s4_ctx* ctx = nullptr;
  int device = -1;  // the context's device: freeing or reading back the weight needs no live context
  int N = 0, K = 0, nblk = 0, ktiles = 0;
  uint8_t* wq = nullptr;
  uint8_t* ws = nullptr;
  uint8_t* wb = nullptr;  // asymmetric formats: per-32-block fp16 biases in the layout of ws
  int glu = 0;            // fused gate|up weight (rows permuted, see repack.cu): matmuls write SiLU*mul, N / 2 wide
  size_t wq_bytes = 0, ws_bytes = 0;
};

