// capi.cu -- the C ABI (include/attnb.h): validation with the reference's
// messages, host<->device staging for the host-pointer entry points, and
// dispatch to the kernels.
#include <algorithm>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <initializer_list>
#include <memory>
#include <string>
#include <vector>

#include "kernels.h"
#include "runtime.h"

namespace attnb {
const char* last_error_cstr();
int profile_enable(int on);
int profile_read(const char* kernel, double* total_ms, int* launches);
}

using namespace attnb;

namespace {

// Runs an entry point's body inside an NVTX range named after the entry point
// (visible in Nsight timelines; free when no tool is attached) and turns its
// exceptions into a status code plus the thread's last-error message.
template <class F>
int guarded(const char* name, F&& f) {
  NvtxRange range(name);
  try {
    f();
    return ATTNB_OK;
  } catch (const Error& e) {
    return set_last_error(e.code, e.msg);
  } catch (const std::exception& e) {
    return set_last_error(ATTNB_ERR_RUNTIME, e.what());
  } catch (...) {
    return set_last_error(ATTNB_ERR_RUNTIME, "unknown error");
  }
}

cudaStream_t as_stream(void* s) { return static_cast<cudaStream_t>(s); }

// ------------------------------------------------------------- validation
// attn::validate_dense_shapes, include/attn.h:54-83 of the reference.
void validate_step(const attnb_tensor* Q, const attnb_tensor* K, const attnb_tensor* V,
                   const attnb_mtensor* O) {
  if (!Q || !K || !V || !O) fail(ATTNB_ERR_INVALID_ARGUMENT, "Null tensor descriptor");
  if (!Q->data || !K->data || !V->data || !O->data)
    fail(ATTNB_ERR_INVALID_ARGUMENT, "Null data pointer");
  if (Q->H <= 0 || Q->Dh <= 0) fail(ATTNB_ERR_INVALID_ARGUMENT, "Q has invalid H/Dh");
  if (K->H != Q->H || V->H != Q->H) fail(ATTNB_ERR_INVALID_ARGUMENT, "K/V H must match Q.H");
  if (K->Dh != Q->Dh || V->Dh != Q->Dh)
    fail(ATTNB_ERR_INVALID_ARGUMENT, "K/V Dh must match Q.Dh");
  if (K->T <= 0 || V->T != K->T)
    fail(ATTNB_ERR_INVALID_ARGUMENT, "K/V T must be positive and equal");
  if (O->H != Q->H || O->Dh != Q->Dh)
    fail(ATTNB_ERR_INVALID_ARGUMENT, "O must be [H, Dh] matching Q");
  if (Q->strideH == 0 || Q->strideDh == 0 || K->strideH == 0 || K->strideT == 0 ||
      K->strideDh == 0 || V->strideH == 0 || V->strideT == 0 || V->strideDh == 0 ||
      O->strideH == 0 || O->strideDh == 0)
    fail(ATTNB_ERR_INVALID_ARGUMENT, "Zero stride encountered");
}

// attn::attn_block_dense checks, src/attn_block.cpp:109-120 of the reference.
void validate_block(const attnb_tensor* Q, const attnb_tensor* K, const attnb_tensor* V,
                    const attnb_mtensor* O, int causal) {
  if (!Q || !K || !V || !O) fail(ATTNB_ERR_INVALID_ARGUMENT, "Null tensor descriptor");
  if (!Q->data || !K->data || !V->data || !O->data)
    fail(ATTNB_ERR_INVALID_ARGUMENT, "Null data pointer");
  if (Q->H <= 0 || Q->Dh <= 0 || K->H != Q->H || V->H != Q->H)
    fail(ATTNB_ERR_INVALID_ARGUMENT, "H mismatch");
  if (K->Dh != Q->Dh || V->Dh != Q->Dh) fail(ATTNB_ERR_INVALID_ARGUMENT, "Dh mismatch");
  if (K->T <= 0 || V->T != K->T) fail(ATTNB_ERR_INVALID_ARGUMENT, "K/V T mismatch");
  if (O->H != Q->H || O->Dh != Q->Dh || O->T != Q->T)
    fail(ATTNB_ERR_INVALID_ARGUMENT, "O must be [H,L,Dh] matching Q");
  if (causal && Q->T != K->T) fail(ATTNB_ERR_INVALID_ARGUMENT, "causal=true requires L==T");
  if (Q->T < 0) fail(ATTNB_ERR_INVALID_ARGUMENT, "H mismatch");
}

// attn::mha_block_dense checks, src/attn_dispatch.cpp:22,45,132 of the reference.
void validate_mha(const float* x, int T, int D, const float* W_in, const float* b_in,
                  const float* W_out, const float* b_out, int H, const float* y) {
  if (H <= 0) fail(ATTNB_ERR_INVALID_ARGUMENT, "num_heads must be positive");
  if (D % H != 0) fail(ATTNB_ERR_RUNTIME, "D must be divisible by H");
  if (D <= 0 || D % 16 != 0)
    fail(ATTNB_ERR_RUNTIME, "D not multiple of 16 fast path not implemented yet.");
  if (T < 0) fail(ATTNB_ERR_INVALID_ARGUMENT, "T must be non-negative");
  if (T > 0 && (!x || !W_in || !b_in || !W_out || !b_out || !y))
    fail(ATTNB_ERR_INVALID_ARGUMENT, "Null data pointer");
}

View3 view(const attnb_tensor* t, int T) {
  return View3{t->data, t->H, T, t->Dh, t->strideH, t->strideT, t->strideDh};
}
MView3 mview(const attnb_mtensor* t, int T) {
  return MView3{t->data, t->H, T, t->Dh, t->strideH, t->strideT, t->strideDh};
}

// ------------------------------------------------------------ host staging
// Element-offset range [lo, hi] a strided view touches.
struct Span {
  int64_t lo = 0, hi = 0;
  int64_t count() const { return hi - lo + 1; }
};
Span span_of(int H, int T, int Dh, int64_t sH, int64_t sT, int64_t sD) {
  Span s;
  auto add = [&](int n, int64_t st) {
    if (n <= 1) return;
    const int64_t e = (int64_t)(n - 1) * st;
    if (e < 0) s.lo += e;
    else s.hi += e;
  };
  add(H, sH);
  add(T, sT);
  add(Dh, sD);
  return s;
}

// Carves 256-byte-aligned pieces out of one device allocation.
struct Carver {
  size_t off = 0;
  size_t take(size_t bytes) {
    const size_t o = off;
    off += (bytes + 255) & ~size_t(255);
    return o;
  }
};

struct Staged {
  Span span;
  size_t off;
};

template <class Fn>
void with_host_ctx(Fn&& fn) {
  DeviceCtx& c = current_ctx();
  std::lock_guard<std::mutex> g(c.mu);
  fn(c);
}

void finish_host_call(DeviceCtx& c) {
  ATTNB_CUDA(cudaGetLastError());
  if (consume_status(c, c.stream) != ATTNB_OK)
    fail(ATTNB_ERR_DEVICE_TIMEOUT, "a bounded device wait expired");
}

// ------------------------------------------------------------------ decode
void step_dev(const attnb_tensor* Q, const attnb_tensor* K, const attnb_tensor* V,
              const attnb_mtensor* O, DeviceCtx& c, cudaStream_t s, void* scratch_override,
              size_t scratch_bytes, const PeerOut* peers = nullptr) {
  const View3 q = view(Q, 1), k = view(K, K->T), v = view(V, V->T);
  const MView3 o = mview(O, 1);
  const DecodePlan p = decode_plan(q, k, v, c.num_sms);
  const size_t need = decode_workspace_bytes(p, K->H, K->Dh);
  void* ws = scratch_override;
  if (!ws) ws = dev_scratch(c, need, s);
  else if (need > scratch_bytes) fail(ATTNB_ERR_RUNTIME, "scratch too small");
  decode_launch(p, q, k, v, o, ws, s, peers);
  ATTNB_CUDA(cudaGetLastError());
}

// ---------------------------------------------------------------- prefill
// Head sizes up to 128 take the tcgen05 kernel (any strides: operands are
// packed first); larger heads the CUDA-core kernel, which needs no scratch.
size_t block_scratch_bytes(int H, int L, int T, int Dh, bool causal, int prec, int num_sms) {
  if (L == 0 || !attn_tc_supported(Dh)) return 0;
  return attn_tc_plan(H, L, T, Dh, causal, prec, num_sms).ws_bytes;
}

void block_dev(const attnb_tensor* Q, const attnb_tensor* K, const attnb_tensor* V,
               const attnb_mtensor* O, int causal, int precision, DeviceCtx& c, cudaStream_t s,
               void* ws) {
  if (Q->T == 0) return;
  const View3 q = view(Q, Q->T), k = view(K, K->T), v = view(V, V->T);
  const MView3 o = mview(O, O->T);
  if (attn_tc_supported(Q->Dh)) {
    const AttnTcPlan p =
        attn_tc_plan(Q->H, Q->T, K->T, Q->Dh, causal != 0, precision, c.num_sms);
    attn_tc_run(p, q, k, v, o, causal != 0, ws, c.status, c.num_sms, s);
  } else {
    attn_block_simt_launch(q, k, v, o, causal != 0, s);
  }
  ATTNB_CUDA(cudaGetLastError());
}

// ------------------------------------------- overlapped host-pointer calls
bool page_locked(const void* p) {
  cudaPointerAttributes a;
  if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  return a.type == cudaMemoryTypeHost;
}

// Groups for a host-pointer call that overlaps copies in, kernels and copies
// out: ATTNB_HOST_GROUPS (default 4; 0 or 1 turns the overlap off), at most
// DeviceCtx::kMaxGroups and at most `units`, for calls that move at least
// ATTNB_HOST_OVERLAP_MB (default 32) MiB.  Each group adds a launch and two
// cross-stream waits, about 13 us: on a 4 MiB call (the [8,512,64] prefill)
// two groups took 135 us against 122 us for one, on a 64 MiB call four
// groups took 1.20 ms against 1.35 ms.  The overlap needs every host buffer
// page-locked: a copy from or to pageable memory returns only once it is
// staged, which would serialise the groups.
int host_groups(int units, size_t bytes, std::initializer_list<const void*> host) {
  static const int want = [] {
    const char* e = std::getenv("ATTNB_HOST_GROUPS");
    return e ? std::atoi(e) : 4;
  }();
  static const size_t min_bytes = [] {
    const char* e = std::getenv("ATTNB_HOST_OVERLAP_MB");
    const long mb = e ? std::atol(e) : 32;
    return (size_t)(mb > 0 ? mb : 0) << 20;
  }();
  const int g = std::min({want, units, DeviceCtx::kMaxGroups});
  if (g < 2 || bytes < min_bytes) return 1;
  for (const void* p : host)
    if (!page_locked(p)) return 1;
  return g;
}

bool dense_heads(const attnb_tensor& t) {
  return t.strideDh == 1 && t.strideT == t.Dh && t.strideH == (int64_t)t.T * t.Dh;
}

// Prefill host calls with dense [H,T,Dh] tensors in page-locked memory split
// their heads into groups: group g's kernel runs while group g+1 is copied in
// and group g-1 is copied out.
int block_host_groups(const attnb_tensor* Q, const attnb_tensor* K, const attnb_tensor* V,
                      const attnb_mtensor* O) {
  const attnb_tensor o{O->data, O->H, O->T, O->Dh, O->strideH, O->strideT, O->strideDh};
  if (!dense_heads(*Q) || !dense_heads(*K) || !dense_heads(*V) || !dense_heads(o)) return 1;
  const size_t bytes = 4 * ((size_t)Q->H * Q->T * Q->Dh * 2 + (size_t)K->H * K->T * K->Dh * 2);
  return host_groups(Q->H, bytes, {Q->data, K->data, V->data, O->data});
}

// Runs `body` and, if it throws, waits for what it left on the three streams
// before rethrowing, so that no copy still writes a caller's buffer.
template <class Fn>
void with_copy_streams(DeviceCtx& c, Fn&& body) {
  ensure_copy_streams(c);
  try {
    // Copies in wait for anything still queued on the context stream.
    ATTNB_CUDA(cudaEventRecord(c.ev_start, c.stream));
    ATTNB_CUDA(cudaStreamWaitEvent(c.h2d, c.ev_start, 0));
    body();
  } catch (...) {
    cudaStreamSynchronize(c.h2d);
    cudaStreamSynchronize(c.stream);
    cudaStreamSynchronize(c.d2h);
    cudaGetLastError();
    throw;
  }
}

void block_host_overlapped(const attnb_tensor* Q, const attnb_tensor* K, const attnb_tensor* V,
                           const attnb_mtensor* O, int causal, int prec, int groups,
                           DeviceCtx& c) {
  const int H = Q->H;
  const size_t qh = (size_t)Q->T * Q->Dh, kh = (size_t)K->T * K->Dh;  // floats per head
  Carver cv;
  const size_t oq = cv.take(H * qh * 4), ok = cv.take(H * kh * 4), ov = cv.take(H * kh * 4),
               oo = cv.take(H * qh * 4);
  char* base = static_cast<char*>(c.io.ensure(cv.take(0), c.stream));
  float* dq = reinterpret_cast<float*>(base + oq);
  float* dk = reinterpret_cast<float*>(base + ok);
  float* dv = reinterpret_cast<float*>(base + ov);
  float* dout = reinterpret_cast<float*>(base + oo);
  auto first = [&](int g) { return (int)((int64_t)H * g / groups); };
  int most = 0;
  for (int g = 0; g < groups; ++g) most = std::max(most, first(g + 1) - first(g));
  void* ws = c.scratch_host_path.ensure(
      block_scratch_bytes(most, Q->T, K->T, Q->Dh, causal != 0, prec, c.num_sms) + 256, c.stream);
  with_copy_streams(c, [&] {
    // Every copy in first, so the copy engine never waits for the host.
    for (int g = 0; g < groups; ++g) {
      const size_t h0 = first(g), n = first(g + 1) - h0;
      ATTNB_CUDA(cudaMemcpyAsync(dq + h0 * qh, Q->data + h0 * qh, n * qh * 4,
                                 cudaMemcpyHostToDevice, c.h2d));
      ATTNB_CUDA(cudaMemcpyAsync(dk + h0 * kh, K->data + h0 * kh, n * kh * 4,
                                 cudaMemcpyHostToDevice, c.h2d));
      ATTNB_CUDA(cudaMemcpyAsync(dv + h0 * kh, V->data + h0 * kh, n * kh * 4,
                                 cudaMemcpyHostToDevice, c.h2d));
      ATTNB_CUDA(cudaEventRecord(c.ev_in[g], c.h2d));
    }
    for (int g = 0; g < groups; ++g) {
      const int h0 = first(g), n = first(g + 1) - h0;
      attnb_tensor gq = *Q, gk = *K, gv = *V;
      attnb_mtensor go = *O;
      gq.H = gk.H = gv.H = go.H = n;
      gq.data = dq + h0 * qh;
      gk.data = dk + h0 * kh;
      gv.data = dv + h0 * kh;
      go.data = dout + h0 * qh;
      ATTNB_CUDA(cudaStreamWaitEvent(c.stream, c.ev_in[g], 0));
      block_dev(&gq, &gk, &gv, &go, causal, prec, c, c.stream, ws);
      ATTNB_CUDA(cudaEventRecord(c.ev_k[g], c.stream));
      ATTNB_CUDA(cudaStreamWaitEvent(c.d2h, c.ev_k[g], 0));
      ATTNB_CUDA(cudaMemcpyAsync(O->data + h0 * qh, go.data, n * qh * 4, cudaMemcpyDeviceToHost,
                                 c.d2h));
    }
    ATTNB_CUDA(cudaEventRecord(c.ev_out, c.d2h));
    ATTNB_CUDA(cudaStreamWaitEvent(c.stream, c.ev_out, 0));
    finish_host_call(c);
  });
}

// Runs attend(b, stream, scratch) for b in [0, batch): with one fork it runs
// on s with scratch ws; otherwise sequence b runs on fork b % nf with its own
// attn_ws-byte slice of ws, the forks start after the work already queued on
// s, and s waits for all of them.
template <class F>
void run_forked(DeviceCtx& c, cudaStream_t s, int batch, int nf, void* ws, size_t attn_ws,
                F&& attend) {
  if (nf == 1) {
    for (int b = 0; b < batch; ++b) attend(b, s, ws);
    return;
  }
  ForkStreams& f = fork_streams(c);
  std::lock_guard<std::mutex> g(f.mu);
  try {
    ATTNB_CUDA(cudaEventRecord(f.fork, s));
    for (int i = 0; i < nf; ++i) ATTNB_CUDA(cudaStreamWaitEvent(f.s[i], f.fork, 0));
    for (int b = 0; b < batch; ++b)
      attend(b, f.s[b % nf], static_cast<char*>(ws) + (b % nf) * attn_ws);
    for (int i = 0; i < nf; ++i) {
      ATTNB_CUDA(cudaEventRecord(f.join[i], f.s[i]));
      ATTNB_CUDA(cudaStreamWaitEvent(s, f.join[i], 0));
    }
  } catch (...) {
    // Nothing queued on a fork may still use the scratch after an error.
    for (int i = 0; i < nf; ++i) cudaStreamSynchronize(f.s[i]);
    cudaGetLastError();
    throw;
  }
}

// -------------------------------------------------------------------- MHA
void mha_dev(const float* x, int batch, int T, int D, const float* W_in, const float* b_in,
             const float* W_out, const float* b_out, int H, int causal, float* y, int prec,
             DeviceCtx& c, cudaStream_t s) {
  if (batch <= 0 || T <= 0) return;
  const int Dh = D / H;
  const int rows = batch * T;
  const GemmPlan p_in = gemm_plan(rows, 3 * D, D, prec);
  Carver cv;
  const size_t off_qkv = cv.take((size_t)rows * 3 * D * sizeof(float));
  const size_t off_ctx = cv.take((size_t)rows * D * sizeof(float));
  const size_t off_g = cv.take(0);
  // The projections and the attention run one after the other and share one
  // scratch region.  Several sequences' attention runs side by side on the
  // fork streams, each fork with its own slice of that region.
  const int nf = std::min(batch, ForkStreams::kForks);
  const size_t attn_ws =
      (block_scratch_bytes(H, T, T, Dh, causal != 0, prec, c.num_sms) + 255) & ~size_t(255);
  const size_t g_bytes =
      std::max({p_in.ws_bytes, gemm_workspace_bound(rows, D, D, prec), nf * attn_ws});
  char* w = static_cast<char*>(dev_scratch(c, off_g + g_bytes, s));
  float* qkv = reinterpret_cast<float*>(w + off_qkv);
  float* ctx = reinterpret_cast<float*>(w + off_ctx);
  void* gws = w + off_g;
  // 1) [Q|K|V] = x . W_in^T + b_in   (src/attn_dispatch.cpp:63-95)
  gemm_run(p_in, x, D, true, W_in, D, true, qkv, 3 * D, 1.f, 0.f, b_in, gws, c.status, c.num_sms, s);
  // 2) per-sequence attention over the head-strided projections (:98-107)
  auto attend = [&](int b, cudaStream_t st, void* ws) {
    const float* base = qkv + (size_t)b * T * 3 * D;
    attnb_tensor q{base, H, T, Dh, Dh, 3 * D, 1};
    attnb_tensor k{base + D, H, T, Dh, Dh, 3 * D, 1};
    attnb_tensor v{base + 2 * D, H, T, Dh, Dh, 3 * D, 1};
    attnb_mtensor o{ctx + (size_t)b * T * D, H, T, Dh, Dh, D, 1};
    block_dev(&q, &k, &v, &o, causal, prec, c, st, ws);
  };
  // Sequence b runs on fork b % nf, after the projection; the output
  // projection waits for every fork.
  run_forked(c, s, batch, nf, gws, attn_ws, attend);
  // 3) y = ctx . W_out^T + b_out   (:110-127)
  const GemmPlan p_out = gemm_plan(rows, D, D, prec);
  gemm_run(p_out, ctx, D, true, W_out, D, true, y, D, 1.f, 0.f, b_out, gws, c.status, c.num_sms, s);
}

}  // namespace

extern "C" {

const char* attnb_last_error(void) { return last_error_cstr(); }

const char* attnb_version(void) { return "attnb 0.1 sm_100a"; }

int attnb_profile_enable(int on) { return profile_enable(on); }

int attnb_selftest_wait_timeout(int limit_us, void* stream) {
  return guarded(__func__, [&] {
    if (limit_us <= 0 || limit_us > 10000000)
      fail(ATTNB_ERR_INVALID_ARGUMENT, "limit_us must be in (0, 1e7]");
    selftest_wait_timeout(current_ctx(), limit_us, as_stream(stream));
  });
}

int attnb_profile_read(const char* kernel, double* total_ms, int* launches) {
  return profile_read(kernel, total_ms, launches);
}

int attnb_host_alloc(size_t bytes, void** ptr) {
  return guarded(__func__, [&] {
    if (!ptr) fail(ATTNB_ERR_INVALID_ARGUMENT, "Null data pointer");
    *ptr = nullptr;
    if (bytes == 0) fail(ATTNB_ERR_INVALID_ARGUMENT, "bytes must be positive");
    *ptr = host_pool_alloc(bytes);
  });
}

int attnb_host_free(void* ptr) {
  return guarded(__func__, [&] {
    if (!host_pool_free(ptr))
      fail(ATTNB_ERR_INVALID_ARGUMENT, "pointer was not allocated by attnb_host_alloc");
  });
}

int attnb_stream_status(void* stream) {
  return guarded(__func__, [&] {
    DeviceCtx& c = current_ctx();
    if (consume_status(c, as_stream(stream)) != ATTNB_OK)
      fail(ATTNB_ERR_DEVICE_TIMEOUT, "a bounded device wait expired");
  });
}

// ------------------------------------------------------------------- SGEMM
int attnb_sgemm_dev(const float* A, int lda, const float* B, int ldb, float* C, int ldc, int M,
                    int N, int K, float alpha, float beta, int precision, void* stream) {
  return guarded(__func__, [&] {
    if (M <= 0 || N <= 0 || K <= 0) return;
    if (!A || !B || !C) fail(ATTNB_ERR_INVALID_ARGUMENT, "Null data pointer");
    if (lda < K || ldb < N || ldc < N)
      fail(ATTNB_ERR_INVALID_ARGUMENT, "leading dimension smaller than the row length");
    const int prec = resolve_precision(precision);
    DeviceCtx& c = current_ctx();
    cudaStream_t s = as_stream(stream);
    const GemmPlan p = gemm_plan(M, N, K, prec);
    void* ws = dev_scratch(c, p.ws_bytes, s);
    gemm_run(p, A, lda, true, B, ldb, false, C, ldc, alpha, beta, nullptr, ws, c.status,
             c.num_sms, s);
    ATTNB_CUDA(cudaGetLastError());
  });
}

int attnb_gemm_ex_dev(int trans_a, int trans_b, const float* A, int lda, const float* B, int ldb,
                      const float* bias, float* C, int ldc, int M, int N, int K, float alpha,
                      float beta, int precision, void* stream) {
  return guarded(__func__, [&] {
    if (K < 0) fail(ATTNB_ERR_INVALID_ARGUMENT, "K must be non-negative");
    if (M <= 0 || N <= 0) return;
    if (!C) fail(ATTNB_ERR_INVALID_ARGUMENT, "Null data pointer");
    if (K == 0) {
      // An empty product: C = beta * C + bias.
      if (ldc < N) fail(ATTNB_ERR_INVALID_ARGUMENT, "leading dimension smaller than the row length");
      DeviceCtx& c = current_ctx();
      gemm_scale_bias(C, ldc, M, N, beta, bias, c.num_sms, as_stream(stream));
      ATTNB_CUDA(cudaGetLastError());
      return;
    }
    if (!A || !B) fail(ATTNB_ERR_INVALID_ARGUMENT, "Null data pointer");
    if ((trans_a != 0 && trans_a != 1) || (trans_b != 0 && trans_b != 1))
      fail(ATTNB_ERR_INVALID_ARGUMENT, "trans_a and trans_b must be 0 or 1");
    if (lda < (trans_a ? M : K) || ldb < (trans_b ? K : N) || ldc < N)
      fail(ATTNB_ERR_INVALID_ARGUMENT, "leading dimension smaller than the row length");
    const int prec = resolve_precision(precision);
    DeviceCtx& c = current_ctx();
    cudaStream_t s = as_stream(stream);
    const GemmPlan p = gemm_plan(M, N, K, prec);
    void* ws = dev_scratch(c, p.ws_bytes, s);
    gemm_run(p, A, lda, trans_a == 0, B, ldb, trans_b == 1, C, ldc, alpha, beta, bias, ws,
             c.status, c.num_sms, s);
    ATTNB_CUDA(cudaGetLastError());
  });
}

int attnb_gemm_ex_bcast_dev(int trans_a, int trans_b, const float* A, int lda, const float* B,
                            int ldb, const float* bias, float* C, int ldc,
                            float* const* replicas, int nreplicas, int M, int N, int K,
                            float alpha, float beta, int precision, void* stream) {
  return guarded(__func__, [&] {
    if (nreplicas < 0 || nreplicas > kMaxPeerOut)
      fail(ATTNB_ERR_INVALID_ARGUMENT, "nreplicas must be in [0, 7]");
    if (nreplicas > 0 && !replicas) fail(ATTNB_ERR_INVALID_ARGUMENT, "Null replica list");
    PeerOut po{};
    po.n = nreplicas;
    for (int i = 0; i < nreplicas; ++i) {
      if (!replicas[i]) fail(ATTNB_ERR_INVALID_ARGUMENT, "Null replica pointer");
      // One vector-width decision serves C and every replica.
      if (((reinterpret_cast<uintptr_t>(replicas[i]) ^ reinterpret_cast<uintptr_t>(C)) & 15u) != 0)
        fail(ATTNB_ERR_INVALID_ARGUMENT, "replicas must have C's alignment modulo 16 bytes");
      po.dst[i] = replicas[i];
    }
    if (K < 0) fail(ATTNB_ERR_INVALID_ARGUMENT, "K must be non-negative");
    if (M <= 0 || N <= 0) return;
    if (!C) fail(ATTNB_ERR_INVALID_ARGUMENT, "Null data pointer");
    if (ldc < N) fail(ATTNB_ERR_INVALID_ARGUMENT, "leading dimension smaller than the row length");
    DeviceCtx& c = current_ctx();
    cudaStream_t s = as_stream(stream);
    if (K == 0) {
      gemm_scale_bias(C, ldc, M, N, beta, bias, c.num_sms, s);
      for (int i = 0; i < nreplicas; ++i)
        ATTNB_CUDA(cudaMemcpy2DAsync(po.dst[i], (size_t)ldc * sizeof(float), C,
                                     (size_t)ldc * sizeof(float), (size_t)N * sizeof(float), M,
                                     cudaMemcpyDeviceToDevice, s));
      ATTNB_CUDA(cudaGetLastError());
      return;
    }
    if (!A || !B) fail(ATTNB_ERR_INVALID_ARGUMENT, "Null data pointer");
    if ((trans_a != 0 && trans_a != 1) || (trans_b != 0 && trans_b != 1))
      fail(ATTNB_ERR_INVALID_ARGUMENT, "trans_a and trans_b must be 0 or 1");
    if (lda < (trans_a ? M : K) || ldb < (trans_b ? K : N))
      fail(ATTNB_ERR_INVALID_ARGUMENT, "leading dimension smaller than the row length");
    const int prec = resolve_precision(precision);
    const GemmPlan p = gemm_plan(M, N, K, prec);
    void* ws = dev_scratch(c, p.ws_bytes, s);
    gemm_run(p, A, lda, trans_a == 0, B, ldb, trans_b == 1, C, ldc, alpha, beta, bias, ws,
             c.status, c.num_sms, s, &po);
    ATTNB_CUDA(cudaGetLastError());
  });
}

// -------------------------------------------------------- packed weights
struct attnb_packed_weight {
  int device, N, K, precision;
  void* mem;  // hi, then lo in 3xTF32 (gemm_packed_bytes)
  float* hi;
  float* lo;
};

int attnb_weight_pack_dev(const float* W, int ldw, int N, int K, int precision,
                          attnb_packed_weight** out, void* stream) {
  return guarded(__func__, [&] {
    if (!out) fail(ATTNB_ERR_INVALID_ARGUMENT, "Null output handle");
    *out = nullptr;
    if (!W) fail(ATTNB_ERR_INVALID_ARGUMENT, "Null data pointer");
    if (N <= 0 || K <= 0) fail(ATTNB_ERR_INVALID_ARGUMENT, "N and K must be positive");
    if (ldw < K) fail(ATTNB_ERR_INVALID_ARGUMENT, "leading dimension smaller than the row length");
    const int prec = resolve_precision(precision);
    const bool split3 = prec != ATTNB_PREC_TF32;
    DeviceCtx& c = current_ctx();
    const size_t bytes = gemm_packed_bytes(N, K, split3);
    void* mem = nullptr;
    const cudaError_t e = cudaMalloc(&mem, bytes);
    if (e == cudaErrorMemoryAllocation) {
      cudaGetLastError();
      fail(ATTNB_ERR_OUT_OF_MEMORY, "cudaMalloc of a packed weight failed");
    }
    ATTNB_CUDA(e);
    std::unique_ptr<attnb_packed_weight> w(new attnb_packed_weight{c.device, N, K, prec, mem,
                                                                   nullptr, nullptr});
    w->hi = static_cast<float*>(mem);
    w->lo = split3 ? reinterpret_cast<float*>(static_cast<char*>(mem) + bytes / 2) : nullptr;
    gemm_pack_b(W, ldw, true, N, K, split3, w->hi, w->lo, c.num_sms, as_stream(stream));
    const cudaError_t le = cudaGetLastError();
    if (le != cudaSuccess) {
      cudaFree(mem);
      ATTNB_CUDA(le);
    }
    *out = w.release();
  });
}

int attnb_weight_free(attnb_packed_weight* w) {
  return guarded(__func__, [&] {
    if (!w) return;
    int dev = 0;
    ATTNB_CUDA(cudaGetDevice(&dev));
    if (dev != w->device) ATTNB_CUDA(cudaSetDevice(w->device));
    const cudaError_t e = cudaFree(w->mem);
    if (dev != w->device) cudaSetDevice(dev);
    delete w;
    ATTNB_CUDA(e);
  });
}

int attnb_linear_packed_dev(int trans_x, const float* x, int ldx, const attnb_packed_weight* W,
                            const float* b, float* y, int ldy, int M, float* const* replicas,
                            int nreplicas, void* stream) {
  return guarded(__func__, [&] {
    if (!W) fail(ATTNB_ERR_INVALID_ARGUMENT, "Null packed weight");
    if (M <= 0) return;
    if (!x || !y) fail(ATTNB_ERR_INVALID_ARGUMENT, "Null data pointer");
    if (trans_x != 0 && trans_x != 1) fail(ATTNB_ERR_INVALID_ARGUMENT, "trans_x must be 0 or 1");
    if (ldx < (trans_x ? M : W->K) || ldy < W->N)
      fail(ATTNB_ERR_INVALID_ARGUMENT, "leading dimension smaller than the row length");
    if (nreplicas < 0 || nreplicas > kMaxPeerOut)
      fail(ATTNB_ERR_INVALID_ARGUMENT, "nreplicas must be in [0, 7]");
    if (nreplicas > 0 && !replicas) fail(ATTNB_ERR_INVALID_ARGUMENT, "Null replica list");
    PeerOut po{};
    po.n = nreplicas;
    for (int i = 0; i < nreplicas; ++i) {
      if (!replicas[i]) fail(ATTNB_ERR_INVALID_ARGUMENT, "Null replica pointer");
      if (((reinterpret_cast<uintptr_t>(replicas[i]) ^ reinterpret_cast<uintptr_t>(y)) & 15u) != 0)
        fail(ATTNB_ERR_INVALID_ARGUMENT, "replicas must have y's alignment modulo 16 bytes");
      po.dst[i] = replicas[i];
    }
    DeviceCtx& c = current_ctx();
    if (c.device != W->device)
      fail(ATTNB_ERR_INVALID_ARGUMENT, "the packed weight lives on another device");
    cudaStream_t s = as_stream(stream);
    const GemmPlan p = gemm_plan(M, W->N, W->K, W->precision);
    void* ws = dev_scratch(c, p.ws_bytes, s);
    gemm_run(p, x, ldx, trans_x == 0, nullptr, 0, true, y, ldy, 1.f, 0.f, b, ws, c.status,
             c.num_sms, s, &po, W->hi, W->lo);
    ATTNB_CUDA(cudaGetLastError());
  });
}

// ------------------------------------------------------------ peer memory
namespace {
// Device memory of other processes opened in this one.  A handle can be
// opened once per context, so openings are shared and counted.
struct IpcOpening {
  std::string key;  // the handle's bytes
  int device;
  void* base;
  int refs;
};
std::mutex g_ipc_mu;
std::vector<IpcOpening> g_ipc;

using GetAddressRangeFn = CUresult (*)(CUdeviceptr*, size_t*, CUdeviceptr);
GetAddressRangeFn address_range_fn() {
  static GetAddressRangeFn fn = [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuMemGetAddressRange", &p, 12000, cudaEnableDefault,
                                         &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return (GetAddressRangeFn) nullptr;
    return reinterpret_cast<GetAddressRangeFn>(p);
  }();
  if (!fn) fail(ATTNB_ERR_CUDA, "cuMemGetAddressRange is unavailable from the driver");
  return fn;
}
}  // namespace

int attnb_ipc_alloc(size_t bytes, void** dptr) {
  return guarded(__func__, [&] {
    if (!dptr || bytes == 0) fail(ATTNB_ERR_INVALID_ARGUMENT, "need a size and an output pointer");
    *dptr = nullptr;
    const cudaError_t e = cudaMalloc(dptr, bytes);
    if (e == cudaErrorMemoryAllocation) {
      cudaGetLastError();
      fail(ATTNB_ERR_OUT_OF_MEMORY, "cudaMalloc of a shared buffer failed");
    }
    ATTNB_CUDA(e);
  });
}

int attnb_ipc_free(void* dptr) {
  return guarded(__func__, [&] {
    if (dptr) ATTNB_CUDA(cudaFree(dptr));
  });
}

int attnb_ipc_export(const void* dptr, void* handle, uint64_t* offset) {
  return guarded(__func__, [&] {
    if (!dptr || !handle || !offset) fail(ATTNB_ERR_INVALID_ARGUMENT, "Null pointer");
    CUdeviceptr base = 0;
    size_t size = 0;
    const CUresult r = address_range_fn()(&base, &size, reinterpret_cast<CUdeviceptr>(dptr));
    if (r != CUDA_SUCCESS)
      fail(ATTNB_ERR_INVALID_ARGUMENT, "not a device allocation of this process");
    cudaIpcMemHandle_t h;
    ATTNB_CUDA(cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base)));
    std::memcpy(handle, &h, sizeof(h));
    *offset = reinterpret_cast<uintptr_t>(dptr) - (uintptr_t)base;
  });
}

int attnb_ipc_import(const void* handle, uint64_t offset, void** dptr) {
  return guarded(__func__, [&] {
    if (!handle || !dptr) fail(ATTNB_ERR_INVALID_ARGUMENT, "Null pointer");
    int dev = 0;
    ATTNB_CUDA(cudaGetDevice(&dev));
    std::string key(static_cast<const char*>(handle), sizeof(cudaIpcMemHandle_t));
    std::lock_guard<std::mutex> lk(g_ipc_mu);
    for (auto& o : g_ipc)
      if (o.key == key && o.device == dev) {
        ++o.refs;
        *dptr = static_cast<char*>(o.base) + offset;
        return;
      }
    cudaIpcMemHandle_t h;
    std::memcpy(&h, handle, sizeof(h));
    void* base = nullptr;
    ATTNB_CUDA(cudaIpcOpenMemHandle(&base, h, cudaIpcMemLazyEnablePeerAccess));
    g_ipc.push_back({key, dev, base, 1});
    *dptr = static_cast<char*>(base) + offset;
  });
}

int attnb_ipc_close(void* dptr) {
  return guarded(__func__, [&] {
    if (!dptr) fail(ATTNB_ERR_INVALID_ARGUMENT, "Null pointer");
    std::lock_guard<std::mutex> lk(g_ipc_mu);
    int dev = 0;
    ATTNB_CUDA(cudaGetDevice(&dev));
    for (size_t i = 0; i < g_ipc.size(); ++i) {
      IpcOpening& o = g_ipc[i];
      if (o.device != dev) continue;
      CUdeviceptr base = 0;
      size_t size = 0;
      if (address_range_fn()(&base, &size, reinterpret_cast<CUdeviceptr>(o.base)) !=
          CUDA_SUCCESS)
        continue;
      const uintptr_t p = reinterpret_cast<uintptr_t>(dptr);
      if (p < (uintptr_t)base || p >= (uintptr_t)base + size) continue;
      if (--o.refs == 0) {
        ATTNB_CUDA(cudaIpcCloseMemHandle(o.base));
        g_ipc.erase(g_ipc.begin() + (std::ptrdiff_t)i);
      }
      return;
    }
    fail(ATTNB_ERR_INVALID_ARGUMENT, "pointer was not opened by attnb_ipc_import");
  });
}

int attnb_linear_dev(const float* x, int ldx, const float* W, int ldw, const float* b, float* y,
                     int ldy, int T, int N, int K, int precision, void* stream) {
  return guarded(__func__, [&] {
    if (T <= 0 || N <= 0 || K <= 0) return;
    if (!x || !W || !y) fail(ATTNB_ERR_INVALID_ARGUMENT, "Null data pointer");
    if (ldx < K || ldw < K || ldy < N)
      fail(ATTNB_ERR_INVALID_ARGUMENT, "leading dimension smaller than the row length");
    const int prec = resolve_precision(precision);
    DeviceCtx& c = current_ctx();
    cudaStream_t s = as_stream(stream);
    const GemmPlan p = gemm_plan(T, N, K, prec);
    void* ws = dev_scratch(c, p.ws_bytes, s);
    gemm_run(p, x, ldx, true, W, ldw, true, y, ldy, 1.f, 0.f, b, ws, c.status, c.num_sms, s);
    ATTNB_CUDA(cudaGetLastError());
  });
}

static int sgemm_host(const float* A, int M, int K, const float* B, int N, float* C, float alpha,
                      float beta, int precision) {
  return guarded(__func__, [&] {
    if (M <= 0 || N <= 0 || K <= 0) return;
    if (!A || !B || !C) fail(ATTNB_ERR_INVALID_ARGUMENT, "Null data pointer");
    const int prec = resolve_precision(precision);
    with_host_ctx([&](DeviceCtx& c) {
      cudaStream_t s = c.stream;
      const size_t a = (size_t)M * K, b = (size_t)K * N, cc = (size_t)M * N;
      const bool read_c = (beta != 0.f);
      Carver cv;
      const size_t oa = cv.take(a * 4), ob = cv.take(b * 4), oc = cv.take(cc * 4);
      const size_t io = cv.take(0);
      char* base = static_cast<char*>(c.io.ensure(io, s));
      float* dA = reinterpret_cast<float*>(base + oa);
      float* dB = reinterpret_cast<float*>(base + ob);
      float* dC = reinterpret_cast<float*>(base + oc);
      const GemmPlan p = gemm_plan(M, N, K, prec);
      void* ws = c.scratch_host_path.ensure(p.ws_bytes + 256, s);
      if (alpha != 0.f) {
        ATTNB_CUDA(cudaMemcpyAsync(dA, A, a * 4, cudaMemcpyHostToDevice, s));
        ATTNB_CUDA(cudaMemcpyAsync(dB, B, b * 4, cudaMemcpyHostToDevice, s));
      }
      if (read_c) ATTNB_CUDA(cudaMemcpyAsync(dC, C, cc * 4, cudaMemcpyHostToDevice, s));
      gemm_run(p, dA, K, true, dB, N, false, dC, N, alpha, beta, nullptr, ws, c.status,
               c.num_sms, s);
      ATTNB_CUDA(cudaMemcpyAsync(C, dC, cc * 4, cudaMemcpyDeviceToHost, s));
      finish_host_call(c);
    });
  });
}

int attnb_sgemm(const float* A, int M, int K, const float* B, int N, float* C, float alpha,
                float beta, int precision) {
  return sgemm_host(A, M, K, B, N, C, alpha, beta, precision);
}

int attnb_gemm_jit(const float* A, int M, int K, const float* B, int N, float* C, float alpha,
                   float beta, int precision) {
  return sgemm_host(A, M, K, B, N, C, alpha, beta, precision);
}

// --------------------------------------------------------------- decode step
int attnb_attn_step_dense_dev(const attnb_tensor* Q, const attnb_tensor* K, const attnb_tensor* V,
                              attnb_mtensor* O, void* stream) {
  return guarded(__func__, [&] {
    validate_step(Q, K, V, O);
    DeviceCtx& c = current_ctx();
    step_dev(Q, K, V, O, c, as_stream(stream), nullptr, 0);
  });
}

int attnb_attn_step_dense_bcast_dev(const attnb_tensor* Q, const attnb_tensor* K,
                                    const attnb_tensor* V, attnb_mtensor* O,
                                    float* const* replicas, int nreplicas, void* stream) {
  return guarded(__func__, [&] {
    validate_step(Q, K, V, O);
    if (nreplicas < 0 || nreplicas > kMaxPeerOut)
      fail(ATTNB_ERR_INVALID_ARGUMENT, "nreplicas must be in [0, 7]");
    if (nreplicas > 0 && !replicas) fail(ATTNB_ERR_INVALID_ARGUMENT, "Null replica list");
    if (nreplicas > 0 && O->strideDh != 1)
      fail(ATTNB_ERR_INVALID_ARGUMENT, "replicated O needs a unit head-dim stride");
    PeerOut po{};
    po.n = nreplicas;
    for (int i = 0; i < nreplicas; ++i) {
      if (!replicas[i]) fail(ATTNB_ERR_INVALID_ARGUMENT, "Null replica pointer");
      po.dst[i] = replicas[i];
    }
    DeviceCtx& c = current_ctx();
    step_dev(Q, K, V, O, c, as_stream(stream), nullptr, 0, &po);
  });
}

int attnb_peer_barrier_dev(uint64_t* flags, uint64_t* const* peer_flags, int nranks, int rank,
                           int limit_us, void* stream) {
  return guarded(__func__, [&] {
    if (nranks < 1 || nranks > kMaxRanks)
      fail(ATTNB_ERR_INVALID_ARGUMENT, "nranks must be in [1, 8]");
    if (rank < 0 || rank >= nranks) fail(ATTNB_ERR_INVALID_ARGUMENT, "rank out of range");
    if (!flags || (nranks > 1 && !peer_flags)) fail(ATTNB_ERR_INVALID_ARGUMENT, "Null pointer");
    if (limit_us < 0 || limit_us > 10000000)
      fail(ATTNB_ERR_INVALID_ARGUMENT, "limit_us must be in [0, 1e7] (0: the default 2 s)");
    PeerFlags f{};
    f.local = flags;
    f.n = nranks;
    f.rank = rank;
    for (int r = 0; r < nranks; ++r) {
      if (r == rank) continue;
      if (!peer_flags[r]) fail(ATTNB_ERR_INVALID_ARGUMENT, "Null peer flag array");
      f.peer[r] = peer_flags[r];
    }
    if (nranks == 1) return;
    DeviceCtx& c = current_ctx();
    // Default: the 2 s limit of the kernels' other bounded waits.
    const uint64_t limit_ns = limit_us ? (uint64_t)limit_us * 1000ull : 2000000000ull;
    peer_barrier(f, limit_ns, c.status, as_stream(stream));
    ATTNB_CUDA(cudaGetLastError());
  });
}

int attnb_attn_step_dense(const attnb_tensor* Q, const attnb_tensor* K, const attnb_tensor* V,
                          attnb_mtensor* O) {
  return guarded(__func__, [&] {
    validate_step(Q, K, V, O);
    with_host_ctx([&](DeviceCtx& c) {
      cudaStream_t s = c.stream;
      const Span sq = span_of(Q->H, 1, Q->Dh, Q->strideH, 0, Q->strideDh);
      const Span sk = span_of(K->H, K->T, K->Dh, K->strideH, K->strideT, K->strideDh);
      const Span sv = span_of(V->H, V->T, V->Dh, V->strideH, V->strideT, V->strideDh);
      const Span so = span_of(O->H, 1, O->Dh, O->strideH, 0, O->strideDh);
      Carver cv;
      const size_t oq = cv.take(sq.count() * 4), ok = cv.take(sk.count() * 4),
                   ov = cv.take(sv.count() * 4), oo = cv.take(so.count() * 4);
      char* base = static_cast<char*>(c.io.ensure(cv.take(0), s));
      auto put = [&](const float* host, const Span& sp, size_t off) {
        ATTNB_CUDA(cudaMemcpyAsync(base + off, host + sp.lo, sp.count() * 4,
                                   cudaMemcpyHostToDevice, s));
        return reinterpret_cast<float*>(base + off) - sp.lo;
      };
      attnb_tensor dq = *Q, dk = *K, dv = *V;
      attnb_mtensor dO = *O;
      dq.data = put(Q->data, sq, oq);
      dk.data = put(K->data, sk, ok);
      dv.data = put(V->data, sv, ov);
      // Strided outputs with holes keep the caller's bytes between elements.
      if (so.count() != (int64_t)O->H * O->Dh) put(O->data, so, oo);
      dO.data = reinterpret_cast<float*>(base + oo) - so.lo;
      const View3 q = view(&dq, 1), k = view(&dk, dk.T), v = view(&dv, dv.T);
      const DecodePlan p = decode_plan(q, k, v, c.num_sms);
      void* ws = c.scratch_host_path.ensure(decode_workspace_bytes(p, K->H, K->Dh) + 256, s);
      decode_launch(p, q, k, v, mview(&dO, 1), ws, s);
      ATTNB_CUDA(cudaMemcpyAsync(O->data + so.lo, base + oo, so.count() * 4,
                                 cudaMemcpyDeviceToHost, s));
      finish_host_call(c);
    });
  });
}

// --------------------------------------------------------- resident KV cache
}  // extern "C"

// K and V of every head, [H, capacity, Dh] each, on the device that was
// current at creation; `length` tokens are valid.  The length is host-side
// state, advanced when an append is enqueued.
struct attnb_kv_cache {
  int device, H, Dh, capacity, length;
  float* k;
  float* v;
};

namespace {

attnb_kv_cache* checked_cache(attnb_kv_cache* kc) {
  if (!kc) fail(ATTNB_ERR_INVALID_ARGUMENT, "Null KV cache");
  int dev = -1;
  ATTNB_CUDA(cudaGetDevice(&dev));
  if (dev != kc->device)
    fail(ATTNB_ERR_INVALID_ARGUMENT, "KV cache belongs to device " + std::to_string(kc->device) +
                                         ", current device is " + std::to_string(dev));
  return kc;
}

// Copies n tokens of k and v ([H, n, Dh], rows contiguous; host or device
// memory) behind the valid ones: one 2-D copy per tensor (H rows of n * Dh).
void cache_append(attnb_kv_cache* kc, const float* k, const float* v, int n, cudaStream_t s) {
  if (n < 0) fail(ATTNB_ERR_INVALID_ARGUMENT, "n must be non-negative");
  if (n == 0) return;
  if (!k || !v) fail(ATTNB_ERR_INVALID_ARGUMENT, "Null data pointer");
  if (n > kc->capacity - kc->length)
    fail(ATTNB_ERR_INVALID_ARGUMENT, "KV cache capacity exceeded (" + std::to_string(kc->length) +
                                         " + " + std::to_string(n) + " > " +
                                         std::to_string(kc->capacity) + ")");
  const size_t pitch = (size_t)kc->capacity * kc->Dh * sizeof(float);
  const size_t width = (size_t)n * kc->Dh * sizeof(float);
  const size_t off = (size_t)kc->length * kc->Dh;
  ATTNB_CUDA(cudaMemcpy2DAsync(kc->k + off, pitch, k, width, width, kc->H, cudaMemcpyDefault, s));
  ATTNB_CUDA(cudaMemcpy2DAsync(kc->v + off, pitch, v, width, width, kc->H, cudaMemcpyDefault, s));
  kc->length += n;
}

// Device views of the valid part of the cache.
void cache_views(const attnb_kv_cache* kc, attnb_tensor& K, attnb_tensor& V) {
  const int64_t sH = (int64_t)kc->capacity * kc->Dh;
  K = attnb_tensor{kc->k, kc->H, kc->length, kc->Dh, sH, kc->Dh, 1};
  V = attnb_tensor{kc->v, kc->H, kc->length, kc->Dh, sH, kc->Dh, 1};
}

}  // namespace

extern "C" {

int attnb_kv_cache_create(int H, int Dh, int capacity, attnb_kv_cache** cache) {
  return guarded(__func__, [&] {
    if (!cache) fail(ATTNB_ERR_INVALID_ARGUMENT, "Null data pointer");
    *cache = nullptr;
    if (H <= 0 || Dh <= 0 || capacity <= 0)
      fail(ATTNB_ERR_INVALID_ARGUMENT, "H, Dh and capacity must be positive");
    DeviceCtx& c = current_ctx();
    auto kc = std::make_unique<attnb_kv_cache>();
    kc->device = c.device;
    kc->H = H;
    kc->Dh = Dh;
    kc->capacity = capacity;
    kc->length = 0;
    kc->k = kc->v = nullptr;
    const size_t bytes = (size_t)H * capacity * Dh * sizeof(float);
    auto check_alloc = [&](cudaError_t e) {
      if (e == cudaSuccess) return;
      cudaGetLastError();
      if (kc->k) cudaFree(kc->k);
      if (e == cudaErrorMemoryAllocation)
        fail(ATTNB_ERR_OUT_OF_MEMORY, "cudaMalloc of the KV cache (2 x " + std::to_string(bytes) +
                                          " bytes) failed: out of memory");
      ATTNB_CUDA(e);
    };
    check_alloc(cudaMalloc(&kc->k, bytes));
    check_alloc(cudaMalloc(&kc->v, bytes));
    *cache = kc.release();
  });
}

int attnb_kv_cache_destroy(attnb_kv_cache* cache) {
  return guarded(__func__, [&] {
    if (!cache) return;
    int prev = -1;
    ATTNB_CUDA(cudaGetDevice(&prev));
    ATTNB_CUDA(cudaSetDevice(cache->device));
    // Work still queued on the cache's buffers finishes before they are freed.
    ATTNB_CUDA(cudaDeviceSynchronize());
    ATTNB_CUDA(cudaFree(cache->k));
    ATTNB_CUDA(cudaFree(cache->v));
    ATTNB_CUDA(cudaSetDevice(prev));
    delete cache;
  });
}

int attnb_kv_cache_length(const attnb_kv_cache* cache, int* length) {
  return guarded(__func__, [&] {
    if (!cache || !length) fail(ATTNB_ERR_INVALID_ARGUMENT, "Null data pointer");
    *length = cache->length;
  });
}

int attnb_kv_cache_truncate(attnb_kv_cache* cache, int length) {
  return guarded(__func__, [&] {
    if (!cache) fail(ATTNB_ERR_INVALID_ARGUMENT, "Null KV cache");
    if (length < 0 || length > cache->length)
      fail(ATTNB_ERR_INVALID_ARGUMENT, "length must be in [0, current length]");
    cache->length = length;
  });
}

int attnb_kv_cache_append(attnb_kv_cache* cache, const float* k, const float* v, int n,
                          void* stream) {
  return guarded(__func__, [&] { cache_append(checked_cache(cache), k, v, n, as_stream(stream)); });
}

int attnb_kv_cache_step_dev(attnb_kv_cache* cache, const float* q, const float* k_new,
                            const float* v_new, float* o, void* stream) {
  return guarded(__func__, [&] {
    attnb_kv_cache* kc = checked_cache(cache);
    if (!q || !o) fail(ATTNB_ERR_INVALID_ARGUMENT, "Null data pointer");
    if ((k_new == nullptr) != (v_new == nullptr))
      fail(ATTNB_ERR_INVALID_ARGUMENT, "k_new and v_new are given together");
    cudaStream_t s = as_stream(stream);
    if (k_new) cache_append(kc, k_new, v_new, 1, s);
    if (kc->length == 0) fail(ATTNB_ERR_INVALID_ARGUMENT, "K/V T must be positive and equal");
    attnb_tensor Q{q, kc->H, 1, kc->Dh, kc->Dh, 0, 1}, K, V;
    attnb_mtensor O{o, kc->H, 1, kc->Dh, kc->Dh, 0, 1};
    cache_views(kc, K, V);
    step_dev(&Q, &K, &V, &O, current_ctx(), s, nullptr, 0);
  });
}

int attnb_kv_cache_step(attnb_kv_cache* cache, const float* q, const float* k_new,
                        const float* v_new, float* o) {
  return guarded(__func__, [&] {
    attnb_kv_cache* kc = checked_cache(cache);
    if (!q || !o) fail(ATTNB_ERR_INVALID_ARGUMENT, "Null data pointer");
    if ((k_new == nullptr) != (v_new == nullptr))
      fail(ATTNB_ERR_INVALID_ARGUMENT, "k_new and v_new are given together");
    if (!k_new && kc->length == 0)
      fail(ATTNB_ERR_INVALID_ARGUMENT, "K/V T must be positive and equal");
    with_host_ctx([&](DeviceCtx& c) {
      cudaStream_t s = c.stream;
      const size_t hd = (size_t)kc->H * kc->Dh;
      Carver cv;
      const size_t oq = cv.take(hd * 4), oo = cv.take(hd * 4);
      char* base = static_cast<char*>(c.io.ensure(cv.take(0), s));
      float* dq = reinterpret_cast<float*>(base + oq);
      float* dout = reinterpret_cast<float*>(base + oo);
      if (k_new) cache_append(kc, k_new, v_new, 1, s);
      ATTNB_CUDA(cudaMemcpyAsync(dq, q, hd * 4, cudaMemcpyHostToDevice, s));
      attnb_tensor Q{dq, kc->H, 1, kc->Dh, kc->Dh, 0, 1}, K, V;
      attnb_mtensor O{dout, kc->H, 1, kc->Dh, kc->Dh, 0, 1};
      cache_views(kc, K, V);
      const View3 qv = view(&Q, 1), kv = view(&K, K.T), vv = view(&V, V.T);
      const DecodePlan p = decode_plan(qv, kv, vv, c.num_sms);
      void* ws = c.scratch_host_path.ensure(decode_workspace_bytes(p, kc->H, kc->Dh) + 256, s);
      decode_launch(p, qv, kv, vv, mview(&O, 1), ws, s);
      ATTNB_CUDA(cudaMemcpyAsync(o, dout, hd * 4, cudaMemcpyDeviceToHost, s));
      finish_host_call(c);
    });
  });
}

// ------------------------------------------------------------------- prefill
int attnb_attn_block_dense_dev(const attnb_tensor* Q, const attnb_tensor* K,
                               const attnb_tensor* V, attnb_mtensor* O, int causal, int precision,
                               void* stream) {
  return guarded(__func__, [&] {
    validate_block(Q, K, V, O, causal);
    const int prec = resolve_precision(precision);
    DeviceCtx& c = current_ctx();
    cudaStream_t s = as_stream(stream);
    void* ws = dev_scratch(c, block_scratch_bytes(Q->H, Q->T, K->T, Q->Dh, causal != 0, prec,
                                                  c.num_sms), s);
    block_dev(Q, K, V, O, causal, prec, c, s, ws);
  });
}

int attnb_attn_block_dense_batched_dev(const attnb_tensor* Q, const attnb_tensor* K,
                                       const attnb_tensor* V, attnb_mtensor* O, int batch,
                                       int64_t q_bs, int64_t k_bs, int64_t v_bs, int64_t o_bs,
                                       int causal, int precision, void* stream) {
  return guarded(__func__, [&] {
    if (batch < 0) fail(ATTNB_ERR_INVALID_ARGUMENT, "batch must be >= 0");
    validate_block(Q, K, V, O, causal);
    if (batch == 0) return;
    const int prec = resolve_precision(precision);
    DeviceCtx& c = current_ctx();
    cudaStream_t s = as_stream(stream);
    const int nf = std::min(batch, ForkStreams::kForks);
    const size_t attn_ws =
        (block_scratch_bytes(Q->H, Q->T, K->T, Q->Dh, causal != 0, prec, c.num_sms) + 255) &
        ~size_t(255);
    void* ws = dev_scratch(c, nf * attn_ws, s);
    run_forked(c, s, batch, nf, ws, attn_ws, [&](int b, cudaStream_t st, void* w) {
      attnb_tensor q = *Q, k = *K, v = *V;
      attnb_mtensor o = *O;
      q.data += b * q_bs;
      k.data += b * k_bs;
      v.data += b * v_bs;
      o.data += b * o_bs;
      block_dev(&q, &k, &v, &o, causal, prec, c, st, w);
    });
  });
}

int attnb_attn_block_dense(const attnb_tensor* Q, const attnb_tensor* K, const attnb_tensor* V,
                           attnb_mtensor* O, int causal, int precision) {
  return guarded(__func__, [&] {
    validate_block(Q, K, V, O, causal);
    const int prec = resolve_precision(precision);
    if (Q->T == 0) return;
    with_host_ctx([&](DeviceCtx& c) {
      const int groups = block_host_groups(Q, K, V, O);
      if (groups > 1) {
        block_host_overlapped(Q, K, V, O, causal, prec, groups, c);
        return;
      }
      cudaStream_t s = c.stream;
      const Span sq = span_of(Q->H, Q->T, Q->Dh, Q->strideH, Q->strideT, Q->strideDh);
      const Span sk = span_of(K->H, K->T, K->Dh, K->strideH, K->strideT, K->strideDh);
      const Span sv = span_of(V->H, V->T, V->Dh, V->strideH, V->strideT, V->strideDh);
      const Span so = span_of(O->H, O->T, O->Dh, O->strideH, O->strideT, O->strideDh);
      Carver cv;
      const size_t oq = cv.take(sq.count() * 4), ok = cv.take(sk.count() * 4),
                   ov = cv.take(sv.count() * 4), oo = cv.take(so.count() * 4);
      char* base = static_cast<char*>(c.io.ensure(cv.take(0), s));
      auto put = [&](const float* host, const Span& sp, size_t off) {
        ATTNB_CUDA(cudaMemcpyAsync(base + off, host + sp.lo, sp.count() * 4,
                                   cudaMemcpyHostToDevice, s));
        return reinterpret_cast<float*>(base + off) - sp.lo;
      };
      attnb_tensor dq = *Q, dk = *K, dv = *V;
      attnb_mtensor dO = *O;
      dq.data = put(Q->data, sq, oq);
      dk.data = put(K->data, sk, ok);
      dv.data = put(V->data, sv, ov);
      if (so.count() != (int64_t)O->H * O->T * O->Dh) put(O->data, so, oo);
      dO.data = reinterpret_cast<float*>(base + oo) - so.lo;
      void* ws = c.scratch_host_path.ensure(
          block_scratch_bytes(Q->H, Q->T, K->T, Q->Dh, causal != 0, prec, c.num_sms) + 256, s);
      block_dev(&dq, &dk, &dv, &dO, causal, prec, c, s, ws);
      ATTNB_CUDA(cudaMemcpyAsync(O->data + so.lo, base + oo, so.count() * 4,
                                 cudaMemcpyDeviceToHost, s));
      finish_host_call(c);
    });
  });
}

// ------------------------------------------------------------------------ MHA
int attnb_mha_block_dense_dev(const float* x, int batch, int T, int D, const float* W_in,
                              const float* b_in, const float* W_out, const float* b_out, int H,
                              int causal, float* y, int precision, void* stream) {
  return guarded(__func__, [&] {
    validate_mha(x, T, D, W_in, b_in, W_out, b_out, H, y);
    if (batch < 0) fail(ATTNB_ERR_INVALID_ARGUMENT, "batch must be non-negative");
    const int prec = resolve_precision(precision);
    DeviceCtx& c = current_ctx();
    mha_dev(x, batch, T, D, W_in, b_in, W_out, b_out, H, causal, y, prec, c, as_stream(stream));
    ATTNB_CUDA(cudaGetLastError());
  });
}

int attnb_mha_block_dense(const float* x, int T, int D, const float* W_in, const float* b_in,
                          const float* W_out, const float* b_out, int H, int causal, float* y,
                          int precision) {
  return guarded(__func__, [&] {
    validate_mha(x, T, D, W_in, b_in, W_out, b_out, H, y);
    const int prec = resolve_precision(precision);
    if (T == 0) return;
    with_host_ctx([&](DeviceCtx& c) {
      cudaStream_t s = c.stream;
      const size_t nx = (size_t)T * D, nwi = (size_t)3 * D * D, nbi = 3 * (size_t)D,
                   nwo = (size_t)D * D, nbo = D;
      Carver cv;
      const size_t ox = cv.take(nx * 4), owi = cv.take(nwi * 4), obi = cv.take(nbi * 4),
                   owo = cv.take(nwo * 4), obo = cv.take(nbo * 4), oy = cv.take(nx * 4);
      char* base = static_cast<char*>(c.io.ensure(cv.take(0), s));
      auto put = [&](const float* host, size_t n, size_t off) {
        ATTNB_CUDA(cudaMemcpyAsync(base + off, host, n * 4, cudaMemcpyHostToDevice, s));
        return reinterpret_cast<const float*>(base + off);
      };
      const float* dx = put(x, nx, ox);
      const float* dwi = put(W_in, nwi, owi);
      const float* dbi = put(b_in, nbi, obi);
      const float* dwo = put(W_out, nwo, owo);
      const float* dbo = put(b_out, nbo, obo);
      float* dy = reinterpret_cast<float*>(base + oy);
      mha_dev(dx, 1, T, D, dwi, dbi, dwo, dbo, H, causal, dy, prec, c, s);
      ATTNB_CUDA(cudaMemcpyAsync(y, dy, nx * 4, cudaMemcpyDeviceToHost, s));
      finish_host_call(c);
    });
  });
}

}  // extern "C"
