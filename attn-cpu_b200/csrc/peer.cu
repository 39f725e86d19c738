// peer.cu -- cross-GPU synchronisation over peer memory (NVLink / NVSwitch).
//
// The sharded paths (row-sharded SGEMM, the MHA block's output rows, the
// decode step's output heads) let their kernels store results straight into
// the other GPUs' buffers.  A reader on another GPU may use those results only
// once every writer is done; a collective of the communication library costs
// tens of microseconds for that, which is most of a sharded decode step.  This
// is the same ordering done with one flag per rank pair:
//
//   rank r's flag array F_r holds one 64-bit epoch per rank, plus its own
//   barrier count, in device memory every rank has mapped (CUDA IPC).  At
//   each barrier rank r's kernel (one warp) advances its count to e, fences
//   its earlier stores system-wide, writes e into slot r of every other
//   rank's array with a release store, then waits until every slot of its own
//   array holds at least e (acquire loads).
//
// Every rank runs the same sequence of barriers, so the counts agree; they
// live on the device, so a captured CUDA graph replays correctly.  Epochs
// only grow, so no reset is needed between barriers.  The wait is bounded
// (ATTNB_WAIT_LIMIT_NS or the caller's limit): a rank that never arrives
// makes the others raise the device status word and return, and the host
// reports ATTNB_ERR_DEVICE_TIMEOUT instead of a hung GPU.
#include "common.cuh"
#include "kernels.h"
#include "runtime.h"

namespace attnb {
namespace {

__device__ __forceinline__ void store_release_sys(uint64_t* p, uint64_t v) {
  asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

__device__ __forceinline__ uint64_t load_acquire_sys(const uint64_t* p) {
  uint64_t v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

__global__ void peer_barrier_kernel(PeerFlags f, uint64_t limit_ns, int* status) {
  const int t = threadIdx.x;
  grid_dep_wait();  // launched behind the kernel whose stores this barrier publishes
  // This rank's barrier count (slot n of its own array, written only here).
  const uint64_t epoch = f.local[f.n] + 1;
  __syncwarp();
  if (t == 0) f.local[f.n] = epoch;
  // Earlier kernels on this stream fenced their peer stores before retiring;
  // this fence orders anything else this thread's stream made visible.
  __threadfence_system();
  if (t < f.n && t != f.rank) store_release_sys(f.peer[t] + f.rank, epoch);
  if (t < f.n && t != f.rank) {
    const uint64_t t0 = globaltimer();
    while (load_acquire_sys(f.local + t) < epoch) {
      if (globaltimer() - t0 > limit_ns) {
        raise_timeout(status);
        break;
      }
      __nanosleep(64);
    }
  }
  __syncwarp();
}

}  // namespace

void peer_barrier(const PeerFlags& f, uint64_t limit_ns, int* status, cudaStream_t s) {
  ATTNB_CUDA(launch_pdl(peer_barrier_kernel, dim3(1), dim3(32), 0, s, f, limit_ns, status));
}

}  // namespace attnb
