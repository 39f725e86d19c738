// runtime.cu -- host runtime of libattnb (see runtime.h).
#include "runtime.h"

#include "common.cuh"

#include <nvtx3/nvToolsExt.h>

#include <algorithm>
#include <cstdlib>
#include <cstring>
#include <atomic>
#include <map>
#include <memory>
#include <vector>

namespace attnb {

static thread_local std::string t_last_error;

[[noreturn]] void fail(int code, const std::string& msg) { throw Error{code, msg}; }

void check_cuda(cudaError_t e, const char* what, const char* file, int line) {
  if (e == cudaSuccess) return;
  fail(ATTNB_ERR_CUDA, std::string(what) + " failed: " + cudaGetErrorString(e) + " (" + file +
                           ":" + std::to_string(line) + ")");
}

NvtxRange::NvtxRange(const char* name) { nvtxRangePushA(name); }
NvtxRange::~NvtxRange() { nvtxRangePop(); }

int set_last_error(int code, const std::string& msg) {
  t_last_error = msg;
  return code;
}

const char* last_error_cstr() { return t_last_error.c_str(); }

// ATTNB_DEVICE_ARENA_CAP_MB: most bytes all arenas of the process may hold
// (0 = no cap).  Read once.
static size_t arena_cap() {
  static const size_t cap = [] {
    const char* e = std::getenv("ATTNB_DEVICE_ARENA_CAP_MB");
    const long mb = e ? std::atol(e) : 0;
    return (size_t)(mb > 0 ? mb : 0) << 20;
  }();
  return cap;
}
static std::atomic<size_t> g_arena_bytes{0};  // bytes held by all arenas

void* DeviceBuffer::ensure(size_t need, cudaStream_t stream) {
  if (need <= bytes && ptr) return ptr;
  size_t grow = need + need / 4 + 4096;
  const size_t cap = arena_cap();
  if (cap) {
    const size_t others = g_arena_bytes.load() - bytes;
    if (others + need > cap)
      fail(ATTNB_ERR_OUT_OF_MEMORY,
           "device scratch of " + std::to_string(need) + " bytes exceeds the arena cap of " +
               std::to_string(cap >> 20) + " MiB (ATTNB_DEVICE_ARENA_CAP_MB)");
    grow = std::min(grow, cap - others);
  }
  if (ptr) {
    ATTNB_CUDA(cudaStreamSynchronize(stream));
    ATTNB_CUDA(cudaFree(ptr));
    g_arena_bytes -= bytes;
    ptr = nullptr;
    bytes = 0;
  }
  const cudaError_t e = cudaMalloc(&ptr, grow);
  if (e == cudaErrorMemoryAllocation) {
    cudaGetLastError();
    ptr = nullptr;
    fail(ATTNB_ERR_OUT_OF_MEMORY, "cudaMalloc of " + std::to_string(grow) +
                                      " bytes of device scratch failed: out of memory");
  }
  ATTNB_CUDA(e);
  bytes = grow;
  g_arena_bytes += bytes;
  return ptr;
}

static std::mutex g_ctx_mu;
static std::map<int, std::unique_ptr<DeviceCtx>> g_ctx;

DeviceCtx& current_ctx() {
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) {
    cudaGetLastError();
    fail(ATTNB_ERR_CUDA, std::string("no CUDA device available: ") + cudaGetErrorString(e));
  }
  std::lock_guard<std::mutex> g(g_ctx_mu);
  auto it = g_ctx.find(dev);
  if (it != g_ctx.end()) return *it->second;
  auto c = std::make_unique<DeviceCtx>();
  c->device = dev;
  int major = 0, minor = 0;
  ATTNB_CUDA(cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev));
  ATTNB_CUDA(cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev));
  if (major != 10 || minor != 0)
    fail(ATTNB_ERR_RUNTIME, "libattnb is built for sm_100a (B200); device " + std::to_string(dev) +
                                " is sm_" + std::to_string(major) + std::to_string(minor));
  ATTNB_CUDA(cudaDeviceGetAttribute(&c->num_sms, cudaDevAttrMultiProcessorCount, dev));
  ATTNB_CUDA(cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking));
  // The status word lives in page-locked host memory mapped into the device's
  // address space: a kernel whose bounded wait expires stores 1 into it over
  // the bus, and the host reads it once the stream is synchronised -- no copy
  // on the normal path (a 4-byte device-to-host copy cost each host-pointer
  // call about 6 us).
  ATTNB_CUDA(cudaHostAlloc(&c->status_host, sizeof(int),
                           cudaHostAllocMapped | cudaHostAllocPortable));
  *c->status_host = 0;
  ATTNB_CUDA(cudaHostGetDevicePointer(reinterpret_cast<void**>(&c->status), c->status_host, 0));
  DeviceCtx& ref = *c;
  g_ctx.emplace(dev, std::move(c));
  return ref;
}

void ensure_copy_streams(DeviceCtx& c) {
  if (c.ev_out) return;
  ATTNB_CUDA(cudaStreamCreateWithFlags(&c.h2d, cudaStreamNonBlocking));
  ATTNB_CUDA(cudaStreamCreateWithFlags(&c.d2h, cudaStreamNonBlocking));
  for (int g = 0; g < DeviceCtx::kMaxGroups; ++g) {
    ATTNB_CUDA(cudaEventCreateWithFlags(&c.ev_in[g], cudaEventDisableTiming));
    ATTNB_CUDA(cudaEventCreateWithFlags(&c.ev_k[g], cudaEventDisableTiming));
  }
  ATTNB_CUDA(cudaEventCreateWithFlags(&c.ev_start, cudaEventDisableTiming));
  ATTNB_CUDA(cudaEventCreateWithFlags(&c.ev_out, cudaEventDisableTiming));  // last: the guard
}

ForkStreams& fork_streams(DeviceCtx& c) {
  static std::mutex create_mu;
  std::lock_guard<std::mutex> g(create_mu);
  if (!c.forks) {
    auto f = std::make_unique<ForkStreams>();
    for (int i = 0; i < ForkStreams::kForks; ++i) {
      ATTNB_CUDA(cudaStreamCreateWithFlags(&f->s[i], cudaStreamNonBlocking));
      ATTNB_CUDA(cudaEventCreateWithFlags(&f->join[i], cudaEventDisableTiming));
    }
    ATTNB_CUDA(cudaEventCreateWithFlags(&f->fork, cudaEventDisableTiming));
    c.forks = f.release();  // lives as long as the context
  }
  return *c.forks;
}

void* dev_scratch(DeviceCtx& c, size_t bytes, cudaStream_t stream) {
  if (bytes == 0) return nullptr;
  std::lock_guard<std::mutex> g(c.scratch_mu);
  return c.scratch_dev_path.ensure(bytes, stream);
}

int resolve_precision(int precision) {
  if (precision == ATTNB_PREC_3XTF32 || precision == ATTNB_PREC_TF32) return precision;
  if (precision != ATTNB_PREC_DEFAULT)
    fail(ATTNB_ERR_INVALID_ARGUMENT, "unknown precision " + std::to_string(precision));
  const char* e = std::getenv("ATTNB_PRECISION");
  if (e && (std::strcmp(e, "tf32") == 0 || std::strcmp(e, "TF32") == 0)) return ATTNB_PREC_TF32;
  return ATTNB_PREC_3XTF32;
}

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    cudaError_t e = cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000,
                                                     cudaEnableDefault, &q);
    if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || !p) return (EncodeTiledFn) nullptr;
    return reinterpret_cast<EncodeTiledFn>(p);
  }();
  if (!fn) fail(ATTNB_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable from the driver");
  return fn;
}

CUtensorMap make_tmap_2d(const float* base, uint64_t rows, uint64_t cols, uint64_t ld,
                         uint32_t box_rows, uint32_t box_cols) {
  if ((reinterpret_cast<uintptr_t>(base) & 15u) != 0)
    fail(ATTNB_ERR_RUNTIME, "TMA base address is not 16-byte aligned");
  if ((ld * sizeof(float)) % 16 != 0) fail(ATTNB_ERR_RUNTIME, "TMA row pitch is not 16-byte aligned");
  if (box_cols * sizeof(float) > 128 || box_rows > 256 || box_rows == 0 || box_cols == 0)
    fail(ATTNB_ERR_RUNTIME, "TMA box exceeds the 128-byte swizzle span");
  CUtensorMap m;
  std::memset(&m, 0, sizeof(m));
  const cuuint64_t dims[2] = {cols, rows};
  const cuuint64_t strides[1] = {ld * sizeof(float)};
  const cuuint32_t box[2] = {box_cols, box_rows};
  const cuuint32_t estr[2] = {1, 1};
  CUresult r = encode_fn()(&m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(base), dims,
                           strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                           CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    fail(ATTNB_ERR_CUDA, "cuTensorMapEncodeTiled failed (" + std::to_string((int)r) + ")");
  return m;
}

CUtensorMap make_tmap_3d(const float* base, uint64_t depth, uint64_t rows, uint64_t cols,
                         uint64_t ld, uint64_t ld_depth, uint32_t box_rows, uint32_t box_cols) {
  if ((reinterpret_cast<uintptr_t>(base) & 15u) != 0)
    fail(ATTNB_ERR_RUNTIME, "TMA base address is not 16-byte aligned");
  if ((ld * sizeof(float)) % 16 != 0 || (ld_depth * sizeof(float)) % 16 != 0)
    fail(ATTNB_ERR_RUNTIME, "TMA pitch is not 16-byte aligned");
  if (box_cols * sizeof(float) > 128 || box_rows > 256 || box_rows == 0 || box_cols == 0)
    fail(ATTNB_ERR_RUNTIME, "TMA box exceeds the 128-byte swizzle span");
  CUtensorMap m;
  std::memset(&m, 0, sizeof(m));
  const cuuint64_t dims[3] = {cols, rows, depth};
  const cuuint64_t strides[2] = {ld * sizeof(float), ld_depth * sizeof(float)};
  const cuuint32_t box[3] = {box_cols, box_rows, 1};
  const cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = encode_fn()(&m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, const_cast<float*>(base), dims,
                           strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                           CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    fail(ATTNB_ERR_CUDA, "cuTensorMapEncodeTiled (3-D) failed (" + std::to_string((int)r) + ")");
  return m;
}

static std::atomic<bool> g_prof_on{false};
static std::mutex g_prof_mu;
static std::map<std::string, std::vector<std::pair<cudaEvent_t, cudaEvent_t>>> g_prof;

ProfScope::ProfScope(const char* kernel, cudaStream_t s) : name_(kernel), s_(s) {
  if (!g_prof_on.load(std::memory_order_relaxed)) return;
  if (cudaEventCreate(&a_) != cudaSuccess || cudaEventCreate(&b_) != cudaSuccess ||
      cudaEventRecord(a_, s_) != cudaSuccess) {
    cudaGetLastError();
    a_ = b_ = nullptr;
  }
}

ProfScope::~ProfScope() {
  if (!a_) return;
  if (cudaEventRecord(b_, s_) != cudaSuccess) {
    cudaGetLastError();
    return;
  }
  std::lock_guard<std::mutex> g(g_prof_mu);
  g_prof[name_].emplace_back(a_, b_);
}

int profile_enable(int on) {
  g_prof_on.store(on != 0);
  return ATTNB_OK;
}

int profile_read(const char* kernel, double* total_ms, int* launches) {
  std::vector<std::pair<cudaEvent_t, cudaEvent_t>> ev;
  {
    std::lock_guard<std::mutex> g(g_prof_mu);
    auto it = g_prof.find(kernel ? kernel : "");
    if (it != g_prof.end()) ev.swap(it->second);
  }
  double ms = 0.0;
  int n = 0;
  for (auto& e : ev) {
    float t = 0.f;
    if (cudaEventSynchronize(e.second) == cudaSuccess &&
        cudaEventElapsedTime(&t, e.first, e.second) == cudaSuccess) {
      ms += t;
      ++n;
    }
    cudaEventDestroy(e.first);
    cudaEventDestroy(e.second);
  }
  cudaGetLastError();
  if (total_ms) *total_ms = ms;
  if (launches) *launches = n;
  return ATTNB_OK;
}

// Self-test of the bounded-wait machinery: one thread waits on an mbarrier
// that nothing arrives on; after `limit_ns` it raises the status word and the
// kernel returns normally (the context stays usable).
__global__ void wait_timeout_selftest_kernel(int* status, uint64_t limit_ns) {
  __shared__ __align__(8) uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    abort_flag = 0;
    mbar_init(smem_addr(&bar), 1);
    fence_barrier_init();
    mbar_wait_limit(smem_addr(&bar), 0, &abort_flag, status, limit_ns);
  }
}

void selftest_wait_timeout(DeviceCtx& c, int limit_us, cudaStream_t s) {
  wait_timeout_selftest_kernel<<<1, 32, 0, s>>>(c.status, (uint64_t)limit_us * 1000ull);
  ATTNB_CUDA(cudaGetLastError());
}

int consume_status(DeviceCtx& c, cudaStream_t stream) {
  ATTNB_CUDA(cudaStreamSynchronize(stream));
  std::lock_guard<std::mutex> g(c.status_mu);
  volatile int* word = c.status_host;
  if (*word) {
    *word = 0;
    return ATTNB_ERR_DEVICE_TIMEOUT;
  }
  return ATTNB_OK;
}

// ------------------------------------------------------ pinned host pool
namespace {
struct HostPool {
  std::mutex mu;
  std::vector<void*> free_list[64];
  std::map<void*, int> live;  // block -> size class (log2 bytes)
  size_t held = 0;            // bytes of all blocks, live or free
  size_t cap = 0;
  HostPool() {
    const char* e = std::getenv("ATTNB_PINNED_POOL_MB");
    const long mb = e ? std::atol(e) : 1024;
    cap = (size_t)(mb > 0 ? mb : 0) << 20;
  }
};
HostPool& host_pool() {
  static HostPool* p = new HostPool();  // never destroyed: blocks may outlive exit order
  return *p;
}
}  // namespace

void* host_pool_alloc(size_t bytes) {
  int cls = 12;
  while (((size_t)1 << cls) < bytes) ++cls;
  if (cls >= 63) return nullptr;
  HostPool& hp = host_pool();
  std::lock_guard<std::mutex> g(hp.mu);
  void* p = nullptr;
  if (!hp.free_list[cls].empty()) {
    p = hp.free_list[cls].back();
    hp.free_list[cls].pop_back();
  } else {
    const size_t sz = (size_t)1 << cls;
    if (hp.held + sz > hp.cap) return nullptr;
    ATTNB_CUDA(cudaHostAlloc(&p, sz, cudaHostAllocPortable));
    hp.held += sz;
  }
  hp.live.emplace(p, cls);
  return p;
}

bool host_pool_free(void* p) {
  HostPool& hp = host_pool();
  std::lock_guard<std::mutex> g(hp.mu);
  auto it = hp.live.find(p);
  if (it == hp.live.end()) return false;
  hp.free_list[it->second].push_back(p);
  hp.live.erase(it);
  return true;
}

}  // namespace attnb
