// runtime.h -- host runtime of libattnb: errors, per-device context (stream,
// status word, scratch arenas), TMA descriptor encoding, precision selection.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>
#include <mutex>
#include <string>

#include "../../include/attnb.h"

namespace attnb {

// Internal error type; the C ABI converts it into a status code + message.
struct Error {
  int code;
  std::string msg;
};
[[noreturn]] void fail(int code, const std::string& msg);
void check_cuda(cudaError_t e, const char* what, const char* file, int line);
#define ATTNB_CUDA(call) ::attnb::check_cuda((call), #call, __FILE__, __LINE__)

// An NVTX range around a host entry point: pushed on construction, popped on
// destruction (a no-op unless a profiling tool is attached).
class NvtxRange {
 public:
  explicit NvtxRange(const char* name);
  ~NvtxRange();
  NvtxRange(const NvtxRange&) = delete;
  NvtxRange& operator=(const NvtxRange&) = delete;
};

// Records `msg` as the calling thread's last error and returns `code`.
int set_last_error(int code, const std::string& msg);

// Grow-only device buffer.  Growing synchronises `stream` first, so a buffer
// that earlier work on the same stream still reads is never freed under it.
struct DeviceBuffer {
  void* ptr = nullptr;
  size_t bytes = 0;
  void* ensure(size_t need, cudaStream_t stream);
};

struct DeviceCtx {
  int device = -1;
  int num_sms = 0;
  cudaStream_t stream = nullptr;  // used by the host-pointer entry points
  int* status = nullptr;          // status word as kernels see it (1: a wait timed out)
  int* status_host = nullptr;     // the same word: page-locked host memory, mapped
  std::mutex status_mu;           // guards reading and clearing it
  std::mutex mu;                  // serialises host-pointer calls on this device
  DeviceBuffer io;                // device copies of host inputs/outputs
  DeviceBuffer scratch_host_path; // kernel scratch for host-pointer calls
  std::mutex scratch_mu;
  DeviceBuffer scratch_dev_path;  // kernel scratch for _dev calls (per device)
  // Host-pointer calls that overlap their copies in, kernels and copies out
  // over groups of rows use a copy-in and a copy-out stream besides `stream`,
  // and one event per group and stage (ensure_copy_streams, under `mu`).
  static constexpr int kMaxGroups = 8;
  cudaStream_t h2d = nullptr, d2h = nullptr;
  cudaEvent_t ev_start = nullptr, ev_out = nullptr;
  cudaEvent_t ev_in[kMaxGroups] = {}, ev_k[kMaxGroups] = {};
  struct ForkStreams* forks = nullptr;
};

// Creates ctx's copy streams and events on first use (hold ctx.mu).
void ensure_copy_streams(DeviceCtx& c);

// Streams that the batched MHA runs its per-sequence attention on, side by
// side (the tail of one sequence's CTAs overlaps the next one's), and the
// events that fork them from and join them back to the caller's stream.
struct ForkStreams {
  static constexpr int kForks = 4;
  std::mutex mu;  // held while a call enqueues on them
  cudaStream_t s[kForks] = {};
  cudaEvent_t fork = nullptr, join[kForks] = {};
};
// ctx's fork streams, created on first use (hold the returned object's mu).
ForkStreams& fork_streams(DeviceCtx& c);

// Context of the current CUDA device (created on first use).
DeviceCtx& current_ctx();

// Scratch for a _dev call on `stream`.  Calls on different streams of one
// device share this buffer, so concurrent _dev calls must use one stream or be
// ordered by the caller; the returned lock keeps other host threads out while
// the launch is enqueued.
void* dev_scratch(DeviceCtx& c, size_t bytes, cudaStream_t stream);

// Resolves ATTNB_PREC_DEFAULT via the ATTNB_PRECISION environment variable.
int resolve_precision(int precision);

// 2-D fp32 tensor map: rows x cols (cols contiguous, row pitch ld elements),
// box box_rows x box_cols, 128-byte swizzle, out-of-range elements read as 0.
CUtensorMap make_tmap_2d(const float* base, uint64_t rows, uint64_t cols, uint64_t ld,
                         uint32_t box_rows, uint32_t box_cols);

// 3-D fp32 tensor map over [depth, rows, cols] (cols contiguous, row pitch
// ld elements, depth pitch ld_depth elements), box 1 x box_rows x box_cols,
// 128-byte swizzle; out-of-range elements (per depth slice) read as 0.
CUtensorMap make_tmap_3d(const float* base, uint64_t depth, uint64_t rows, uint64_t cols,
                         uint64_t ld, uint64_t ld_depth, uint32_t box_rows, uint32_t box_cols);

// CUDA-event timing of the dominant kernel of each call (attnb_profile_*):
// construct before the launch, destroy after it, on the launching stream.
class ProfScope {
 public:
  ProfScope(const char* kernel, cudaStream_t s);
  ~ProfScope();
  ProfScope(const ProfScope&) = delete;
  ProfScope& operator=(const ProfScope&) = delete;

 private:
  const char* name_;
  cudaStream_t s_;
  cudaEvent_t a_ = nullptr, b_ = nullptr;
};

// Launches a kernel whose bounded wait expires after limit_us (see attnb.h).
void selftest_wait_timeout(DeviceCtx& c, int limit_us, cudaStream_t s);

// Reads and clears the device status word of ctx (synchronises `stream`).
int consume_status(DeviceCtx& c, cudaStream_t stream);

// Page-locked host blocks for results handed to callers (attnb_host_alloc):
// power-of-two size classes from 4 KiB, recycled on free, at most
// ATTNB_PINNED_POOL_MB (default 1024) MiB held.  host_pool_alloc returns
// nullptr when the cap would be exceeded.
void* host_pool_alloc(size_t bytes);
// Returns a block to its size class; false if `p` is not a live pool block.
bool host_pool_free(void* p);

}  // namespace attnb
