// Cross-GPU barrier for the column-sharded prefill: after every rank's GEMM has written its output
// slice into all ranks' gathered buffers (NVLink peer stores), each rank signals every peer and
// waits until every peer has signalled it. Flags live in each rank's own memory and are mapped into
// the peers' address spaces (CUDA IPC, plain peer mappings). Waits are bounded: after
// kWaitTimeoutNs a rank stops waiting and sets the context's error word.
#include "common.cuh"

namespace s4 {

struct FlagList {
  uint32_t* p[8];  // flag array of rank q (kPeerMaxRanks slots), as mapped in this process
};

__global__ void peer_barrier_kernel(FlagList flags, int nranks, int rank, uint32_t epoch, uint32_t* err) {
  const int q = threadIdx.x;
  __shared__ uint32_t s_epoch;
  if (q == 0) {
    if (epoch == 0) {  // device-side epoch: this rank's barriers are ordered on its stream
      uint32_t* ctr = flags.p[rank] + kPeerCounterSlot;
      epoch = *ctr + 1;
      if (epoch == 0) epoch = 1;
      *ctr = epoch;
    }
    s_epoch = epoch;
  }
  __threadfence_system();  // this GPU's earlier peer stores (previous kernels) before the signal
  __syncwarp();  // each warp reaches the (warp-aligned) block barrier as a whole after its role code
  __syncthreads();
  epoch = s_epoch;
  if (q < nranks)
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(flags.p[q] + rank), "r"(epoch) : "memory");
  if (q < nranks) {
    const uint32_t* mine = flags.p[rank] + q;
    const uint64_t deadline = globaltimer_ns() + kWaitTimeoutNs;
    while (true) {
      uint32_t v;
      asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(mine) : "memory");
      if ((int32_t)(v - epoch) >= 0) break;
      if (globaltimer_ns() > deadline) {
        set_error(err, kErrWaitTimeout);
        break;
      }
      __nanosleep(64);
    }
  }
  __syncwarp();  // each warp reaches the (warp-aligned) block barrier as a whole after its role code
  __syncthreads();
}

// The signalling half of the barrier, for consumers that wait themselves (peer_wait_all at their
// start: the tcgen05 GEMM's activation producer, the ADD_NORM kernel): once the kernel before it in
// the stream has completed (grid-dependency wait), counts the next epoch on the device and stores
// it, with release semantics at system scope, into slot `rank` of every rank's flag array. Launched
// with programmatic dependent launch, so its own launch overlaps the previous kernel, and it lets
// the next kernel start its prologue (and its weight stream) while the peers catch up.
__global__ void peer_signal_kernel(FlagList flags, int nranks, int rank) {
  const int q = threadIdx.x;
  // the next kernel may launch now: it reads nothing of this one before its own grid-dependency
  // wait, which waits for this kernel (and so for the one before it) to complete
  pdl_launch_dependents();
  pdl_wait();
  __shared__ uint32_t s_epoch;
  if (q == 0) {
    uint32_t* ctr = flags.p[rank] + kPeerCounterSlot;
    uint32_t epoch = *ctr + 1;
    if (epoch == 0) epoch = 1;
    *ctr = epoch;
    s_epoch = epoch;
  }
  __threadfence_system();  // this GPU's peer stores of the previous kernel before the signal
  __syncwarp();
  const uint32_t epoch = s_epoch;
  if (q < nranks)
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(flags.p[q] + rank), "r"(epoch) : "memory");
}

cudaError_t launch_peer_signal(uint32_t* const* flags, int nranks, int rank, cudaStream_t stream, bool pdl) {
  if (nranks < 1 || nranks > 8 || rank < 0 || rank >= nranks) return cudaErrorInvalidValue;
  FlagList fl = {};
  for (int q = 0; q < nranks; ++q) fl.p[q] = flags[q];
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(1, 1, 1);
  cfg.blockDim = dim3(32, 1, 1);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, peer_signal_kernel, fl, nranks, rank);
}

cudaError_t launch_peer_barrier(uint32_t* const* flags, int nranks, int rank, uint32_t epoch, uint32_t* err,
                                cudaStream_t stream) {
  if (nranks < 1 || nranks > 8 || rank < 0 || rank >= nranks) return cudaErrorInvalidValue;
  FlagList fl = {};
  for (int q = 0; q < nranks; ++q) fl.p[q] = flags[q];
  peer_barrier_kernel<<<1, 32, 0, stream>>>(fl, nranks, rank, epoch, err);
  return cudaGetLastError();
}

}  // namespace s4
