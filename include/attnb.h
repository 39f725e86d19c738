/*
 * attnb.h -- C ABI of the B200 attention/SGEMM library (libattnb.so).
 *
 * Plain pointers, sizes and status codes; no C++ or torch types.  Each entry
 * point replaces one reference interface, cited beside it.  The C++ headers
 * attn.h / attn_api.h / gemm.h in this directory keep the reference's own
 * signatures as thin shims over these calls.
 *
 * Host-pointer entry points (no suffix) follow the reference's contract: all
 * pointers are caller-owned row-major fp32 HOST memory, the call copies inputs
 * to the current CUDA device, computes there and copies the result back before
 * returning.  Pinned (page-locked) host buffers make those copies faster but
 * are not required.
 *
 * Device-pointer entry points (suffix _dev) take device pointers and a
 * cudaStream_t (passed as void*, NULL = legacy default stream); they enqueue
 * work and return without synchronising.  Kernel-side wait time-outs are
 * reported by attnb_stream_status().
 *
 * Every function returns ATTNB_OK (0) or an error code; attnb_last_error()
 * returns a message for the calling thread's last failure.
 */
#ifndef ATTNB_H
#define ATTNB_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define ATTNB_API __attribute__((visibility("default")))
#else
#define ATTNB_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define ATTNB_OK 0
#define ATTNB_ERR_INVALID_ARGUMENT 1 /* shape/null/stride problems: std::invalid_argument */
#define ATTNB_ERR_RUNTIME 2          /* unsupported configuration: std::runtime_error */
#define ATTNB_ERR_CUDA 3             /* a CUDA runtime/driver call failed */
#define ATTNB_ERR_DEVICE_TIMEOUT 4   /* a bounded in-kernel wait expired */
#define ATTNB_ERR_OUT_OF_MEMORY 5    /* device memory could not be had: std::bad_alloc */

/* Device memory.  Scratch (packed operands, split partials) and the device
 * copies of host-pointer calls' data live in per-device arenas that grow on
 * demand and are reused.  A growth that cudaMalloc refuses, or that would take
 * the arenas past ATTNB_DEVICE_ARENA_CAP_MB MiB (environment variable, read
 * once; unset or 0 = no cap), fails the call with ATTNB_ERR_OUT_OF_MEMORY
 * before any of its work is enqueued; the library stays usable for calls that
 * fit.  The reference allocates with std::vector, so its allocation failures
 * are std::bad_alloc (MemoryError in Python), which the shims and the Python
 * module raise for this code. */

/* Arithmetic used by the tensor-core contractions (SGEMM, projections,
 * prefill attention).  Decode is always plain fp32 FMA on CUDA cores.
 *   ATTNB_PREC_3XTF32: split fp32 operands into tf32 big+small parts and
 *     accumulate big*big + big*small + small*big in fp32 (fp32-level accuracy,
 *     max|y-r|/max|r| <= 1e-5 against the reference).
 *   ATTNB_PREC_TF32: one tf32 pass (<= 2e-3).
 *   ATTNB_PREC_DEFAULT: ATTNB_PREC_3XTF32 unless the environment variable
 *     ATTNB_PRECISION is "tf32". */
#define ATTNB_PREC_DEFAULT (-1)
#define ATTNB_PREC_3XTF32 0
#define ATTNB_PREC_TF32 1

/* Non-owning view of a 3-D fp32 tensor [H, T, Dh]; strides in elements.
 * Mirrors attn::TensorF32 / MutableTensor3F32 (include/attn.h:10-26 of the
 * reference).  For a 2-D [H, Dh] view set T = 1 and strideT = 0. */
typedef struct attnb_tensor {
  const float* data;
  int H, T, Dh;
  int64_t strideH, strideT, strideDh;
} attnb_tensor;

typedef struct attnb_mtensor {
  float* data;
  int H, T, Dh;
  int64_t strideH, strideT, strideDh;
} attnb_mtensor;

/* ---------------------------------------------------------------- errors */
ATTNB_API const char* attnb_last_error(void);
/* Library version string, e.g. "attnb 0.1 sm_100a". */
ATTNB_API const char* attnb_version(void);
/* Device status word of `stream`'s device: ATTNB_OK or ATTNB_ERR_DEVICE_TIMEOUT
 * (and clears it).  Synchronises the stream. */
ATTNB_API int attnb_stream_status(void* stream);
/* Self-test of the failure path (no counterpart in the reference): enqueues a
 * kernel whose bounded wait on a barrier that nothing arrives on expires after
 * limit_us microseconds (0 < limit_us <= 1e7).  The kernel then returns
 * normally, so a following attnb_stream_status() reports
 * ATTNB_ERR_DEVICE_TIMEOUT and the context stays usable. */
ATTNB_API int attnb_selftest_wait_timeout(int limit_us, void* stream);

/* Kernel timing for measurements (no counterpart in the reference).  While
 * enabled, every call records a CUDA event pair around its dominant kernel on
 * the launching stream: "attn_tc" (tensor-core prefill), "attn_simt" (CUDA-core
 * prefill), "gemm_tc" (SGEMM / projections), "decode" (decode step).
 * attnb_profile_read synchronises the recorded events, returns the summed
 * milliseconds and launch count for `kernel`, and forgets them. */
ATTNB_API int attnb_profile_enable(int on);
ATTNB_API int attnb_profile_read(const char* kernel, double* total_ms, int* launches);

/* Page-locked host memory for results (no counterpart in the reference).
 * Host-pointer calls move data by DMA at full PCIe rate only to and from
 * page-locked memory; these blocks come from a recycled pool (power-of-two
 * size classes, at most ATTNB_PINNED_POOL_MB MiB, default 1024).  The Python
 * module returns its result arrays in them.  attnb_host_alloc sets *ptr to
 * NULL (and returns ATTNB_OK) when the pool is full; attnb_host_free rejects
 * pointers it did not hand out with ATTNB_ERR_INVALID_ARGUMENT. */
ATTNB_API int attnb_host_alloc(size_t bytes, void** ptr);
ATTNB_API int attnb_host_free(void* ptr);

/* ---------------------------------------------------------------- SGEMM */
/* C[M,N] = alpha * A[M,K] . B[K,N] + beta * C.
 * Replaces gemm::sgemm_blocked (include/gemm.h:11-14; src/gemm.cpp:319-415).
 * M,N,K <= 0 return ATTNB_OK without touching C; alpha == 0 only scales C;
 * beta == 0 never reads C. */
ATTNB_API int attnb_sgemm(const float* A, int M, int K, const float* B, int N, float* C,
                float alpha, float beta, int precision);
/* Replaces gemm::gemm_blocked_jit (include/gemm.h:17-20; src/jit_gemm.cpp:740-754).
 * Same function as attnb_sgemm; there is no run-time autotune. */
ATTNB_API int attnb_gemm_jit(const float* A, int M, int K, const float* B, int N, float* C,
                   float alpha, float beta, int precision);
/* Device-pointer SGEMM with leading dimensions (elements): lda >= K, ldb >= N,
 * ldc >= N. */
ATTNB_API int attnb_sgemm_dev(const float* A, int lda, const float* B, int ldb, float* C, int ldc,
                    int M, int N, int K, float alpha, float beta, int precision,
                    void* stream);

/* C[M,N] = alpha * op(A) . op(B) + beta * C + bias[N] on device pointers.
 * op(A) is A stored [M,K] (trans_a = 0, lda >= K) or A^T with A stored [K,M]
 * (trans_a = 1, lda >= M); op(B) is B stored [K,N] (trans_b = 0, ldb >= N) or
 * B^T with B stored [N,K] (trans_b = 1, ldb >= K); ldc >= N; bias may be
 * NULL.  M <= 0 or N <= 0 leaves C untouched; K == 0 (an empty product; A and
 * B are not read and may be NULL) gives C = beta * C + bias, where beta == 0
 * never reads C; K < 0 is ATTNB_ERR_INVALID_ARGUMENT.
 * No reference counterpart: the reference's GEMMs take row-major
 * operands only (include/gemm.h:11-20).  The sharded MHA block uses it to read
 * the all-gathered context in its transposed layout. */
ATTNB_API int attnb_gemm_ex_dev(int trans_a, int trans_b, const float* A, int lda, const float* B,
                      int ldb, const float* bias, float* C, int ldc, int M, int N, int K,
                      float alpha, float beta, int precision, void* stream);

/* attnb_gemm_ex_dev whose epilogue also writes every element of C, at the
 * same offset (same ldc), into each of the `nreplicas` (0..7) buffers in
 * `replicas` -- typically the same rows of C's replicas on the other GPUs of
 * the node, opened with attnb_ipc_import -- so the product and its broadcast
 * over NVLink are one kernel: the stores leave tile by tile while the
 * remaining tiles are still being multiplied.  Each replica must have C's
 * alignment modulo 16 bytes.  Replicas are complete once the stream has
 * passed the call (the kernel fences its stores system-wide before it
 * retires); the caller orders the readers on the other GPUs after that, e.g.
 * with a collective.  No reference counterpart: the reference has no
 * multi-device code.  It assembles C on every rank for the row-sharded SGEMM
 * and the sharded MHA block's output rows. */
ATTNB_API int attnb_gemm_ex_bcast_dev(int trans_a, int trans_b, const float* A, int lda,
                                      const float* B, int ldb, const float* bias, float* C,
                                      int ldc, float* const* replicas, int nreplicas, int M,
                                      int N, int K, float alpha, float beta, int precision,
                                      void* stream);

/* Device memory shared between the processes of one node (no counterpart in
 * the reference).  attnb_ipc_export writes the 64-byte handle of the device
 * allocation that holds `dptr` and dptr's byte offset in it; another process
 * passes both to attnb_ipc_import, which maps the allocation into the
 * current device's context (once per handle; later imports share it) and
 * returns the address that corresponds to `dptr`.  attnb_ipc_close releases
 * one import (any address inside the mapping).  The exporting process keeps
 * the allocation alive until every importer has closed it. */
#define ATTNB_IPC_HANDLE_BYTES 64
/* A device allocation of its own (cudaMalloc on the current device) for
 * buffers that other processes will import; attnb_ipc_free releases it. */
ATTNB_API int attnb_ipc_alloc(size_t bytes, void** dptr);
ATTNB_API int attnb_ipc_free(void* dptr);
ATTNB_API int attnb_ipc_export(const void* dptr, void* handle, uint64_t* offset);
ATTNB_API int attnb_ipc_import(const void* handle, uint64_t offset, void** dptr);
ATTNB_API int attnb_ipc_close(void* dptr);

/* Barrier of `nranks` GPUs over peer memory (no counterpart in the
 * reference).  Every rank owns an array of nranks + 1 uint64 words, zeroed
 * before first use, that every other rank has mapped (attnb_ipc_import):
 * one epoch slot per rank and, last, this rank's own barrier count.
 * peer_flags[r] is rank r's array as mapped here (peer_flags[rank] is not
 * read).  The call enqueues one small kernel on `stream` that advances the
 * count to e, makes this stream's earlier stores visible system-wide, writes
 * e into slot `rank` of every other rank's array, and waits until every slot
 * of `flags` (its own array) holds at least e: work enqueued after it on any
 * rank sees everything every rank enqueued before it.  Every rank must make
 * the same sequence of barrier calls.  The count lives on the device, so a
 * CUDA graph that captured the call replays it correctly.  The wait is
 * bounded (limit_us microseconds, 0 = 2 s): a rank that never arrives makes
 * the others raise the device status word, reported by attnb_stream_status
 * as ATTNB_ERR_DEVICE_TIMEOUT, and return. */
ATTNB_API int attnb_peer_barrier_dev(uint64_t* flags, uint64_t* const* peer_flags, int nranks,
                                     int rank, int limit_us, void* stream);

/* A projection weight W [N, K] (the B operand of y = x W^T) packed once for
 * repeated products (no counterpart in the reference, whose projections
 * repack per call; its shape-keyed weight cache, src/attn_dispatch.cpp:46,
 * is not reproduced: a packed weight is tied to the handle, not to a shape).
 * attnb_weight_pack_dev allocates device memory on the current device
 * (released by attnb_weight_free) and enqueues the packing of W (device
 * pointer, ldw >= K) for `precision` on `stream`.
 * attnb_linear_packed_dev: y[M,N] = op(x) . W^T + b[N] (b may be NULL), op(x)
 * = x stored [M,K] (trans_x = 0, ldx >= K) or x^T with x stored [K,M]
 * (trans_x = 1, ldx >= M), ldy >= N, in the weight's precision; like
 * attnb_gemm_ex_bcast_dev it also stores y into the `nreplicas` (0..7)
 * replicas (same ldy, y's alignment modulo 16 bytes).  The sharded MHA block
 * packs its weights once and runs both projections through it. */
typedef struct attnb_packed_weight attnb_packed_weight;
ATTNB_API int attnb_weight_pack_dev(const float* W, int ldw, int N, int K, int precision,
                                    attnb_packed_weight** out, void* stream);
ATTNB_API int attnb_weight_free(attnb_packed_weight* w);
ATTNB_API int attnb_linear_packed_dev(int trans_x, const float* x, int ldx,
                                      const attnb_packed_weight* W, const float* b, float* y,
                                      int ldy, int M, float* const* replicas, int nreplicas,
                                      void* stream);

/* y[T,N] = x[T,K] . W[N,K]^T + b[N] on device pointers (b may be NULL).
 * The projection step of attn::mha_block_dense (src/attn_dispatch.cpp:45-95,
 * include/gemm_16x16.h:7-60, include/pack_16x16.h:9-25); ldx >= K, ldw >= K,
 * ldy >= N. */
ATTNB_API int attnb_linear_dev(const float* x, int ldx, const float* W, int ldw, const float* b,
                     float* y, int ldy, int T, int N, int K, int precision, void* stream);

/* ------------------------------------------------------------ attention */
/* Decode step: O[h,:] = softmax(Q[h,:] . K[h]^T / sqrt(Dh)) . V[h].
 * Q: [H, Dh] (T ignored), K/V: [H, T, Dh], O: [H, Dh].
 * Replaces attn::attn_step_dense (include/attn.h:35-38; src/attn_dense.cpp:21-73),
 * with the reference's validate_dense_shapes checks (include/attn.h:54-83). */
ATTNB_API int attnb_attn_step_dense(const attnb_tensor* Q, const attnb_tensor* K,
                          const attnb_tensor* V, attnb_mtensor* O);
ATTNB_API int attnb_attn_step_dense_dev(const attnb_tensor* Q, const attnb_tensor* K,
                              const attnb_tensor* V, attnb_mtensor* O, void* stream);
/* attnb_attn_step_dense_dev that also stores every element of O, at the same
 * offset (same strides), into each of the `nreplicas` (0..7) buffers in
 * `replicas` -- the same heads of O's replicas on the other GPUs (see
 * attnb_ipc_import); O needs a unit head-dim stride when nreplicas > 0.  The
 * stores are fenced system-wide before the kernel retires.  No reference
 * counterpart (the reference has no multi-device code): the head-sharded
 * decode step assembles O on every rank with it. */
ATTNB_API int attnb_attn_step_dense_bcast_dev(const attnb_tensor* Q, const attnb_tensor* K,
                                              const attnb_tensor* V, attnb_mtensor* O,
                                              float* const* replicas, int nreplicas,
                                              void* stream);
/* The decode step for callers that may not allocate device memory (a custom
 * allocator or pool that owns the device, a hot path where allocation is
 * forbidden, a fixed memory footprint).  No counterpart in the reference.
 * Same arguments, plan and kernels as attnb_attn_step_dense_dev, but the
 * split-KV scratch is a fixed 2 MiB file-scope device array, held by every
 * GPU that loads the library until exit; calls needing more are rejected with
 * ATTNB_ERR_INVALID_ARGUMENT.  All calls share that array: calls that overlap
 * on the GPU race.  The first call on a device looks up the array's address;
 * make it before any stream capture.  The address is cached per device and
 * CUDA context: the first call after the caller recreates the device's context
 * (e.g. cudaDeviceReset) looks it up again, and likewise belongs before any
 * capture.  Allocates nothing. */
ATTNB_API int attnb_attn_step_dense_noalloc(const attnb_tensor* Q, const attnb_tensor* K,
                                            const attnb_tensor* V, attnb_mtensor* O,
                                            void* stream);

/* ------------------------------------------------- resident KV cache */
/* Multi-step decode with K and V kept on the device between steps, for the
 * host<->device residency the reference's boundary cannot offer (its
 * attn::attn_step_dense, src/attn_dense.cpp:21-73, takes the whole cache
 * from host memory on every call).  A cache holds K and V as [H, capacity,
 * Dh] fp32 on the device that is current when it is created; calls must be
 * made with that device current.  `length` tokens are valid, advanced when
 * an append is enqueued: calls that use one cache from several streams must
 * be ordered by the caller.
 *   append: k and v are [H, n, Dh] with contiguous rows, in host or device
 *     memory; more than capacity - length tokens is ATTNB_ERR_INVALID_ARGUMENT.
 *   truncate: drops tokens from the end (0 <= length <= current length).
 *   step: optionally appends one token (k_new, v_new: [H, Dh], both or
 *     neither), then O[h,:] = softmax(Q[h,:] . K[h]^T / sqrt(Dh)) . V[h] over
 *     the valid tokens -- the function of attnb_attn_step_dense.
 *     attnb_kv_cache_step takes host pointers and returns when O is written;
 *     attnb_kv_cache_step_dev takes device pointers (k_new / v_new may also
 *     be host memory) and enqueues on `stream`.
 * destroy synchronises the cache's device before freeing it. */
typedef struct attnb_kv_cache attnb_kv_cache;
ATTNB_API int attnb_kv_cache_create(int H, int Dh, int capacity, attnb_kv_cache** cache);
ATTNB_API int attnb_kv_cache_destroy(attnb_kv_cache* cache);
ATTNB_API int attnb_kv_cache_length(const attnb_kv_cache* cache, int* length);
ATTNB_API int attnb_kv_cache_truncate(attnb_kv_cache* cache, int length);
ATTNB_API int attnb_kv_cache_append(attnb_kv_cache* cache, const float* k, const float* v, int n,
                                    void* stream);
ATTNB_API int attnb_kv_cache_step(attnb_kv_cache* cache, const float* q, const float* k_new,
                                  const float* v_new, float* o);
ATTNB_API int attnb_kv_cache_step_dev(attnb_kv_cache* cache, const float* q, const float* k_new,
                                      const float* v_new, float* o, void* stream);

/* Prefill with given Q/K/V: Q [H,L,Dh], K/V [H,T,Dh] -> O [H,L,Dh]; causal
 * needs L == T.  Replaces attn::attn_block_dense (include/attn.h:40-44;
 * src/attn_block.cpp:104-241). */
ATTNB_API int attnb_attn_block_dense(const attnb_tensor* Q, const attnb_tensor* K,
                           const attnb_tensor* V, attnb_mtensor* O, int causal,
                           int precision);
ATTNB_API int attnb_attn_block_dense_dev(const attnb_tensor* Q, const attnb_tensor* K,
                               const attnb_tensor* V, attnb_mtensor* O, int causal,
                               int precision, void* stream);
/* The same prefill for `batch` independent sequences of equal shape: sequence
 * b's views are Q, K, V, O with data advanced by b * {q,k,v,o}_bs elements.
 * The sequences run side by side on internal streams forked from `stream`
 * and joined back to it.  No reference counterpart: the reference's MHA block
 * loops over sequences (src/attn_dispatch.cpp:98-107); the sharded MHA block
 * uses this for its local heads. */
ATTNB_API int attnb_attn_block_dense_batched_dev(const attnb_tensor* Q, const attnb_tensor* K,
                                       const attnb_tensor* V, attnb_mtensor* O, int batch,
                                       int64_t q_bs, int64_t k_bs, int64_t v_bs, int64_t o_bs,
                                       int causal, int precision, void* stream);

/* Full MHA block, x[T,D] -> y[T,D] with W_in[3D,D], b_in[3D], W_out[D,D],
 * b_out[D] (PyTorch nn.MultiheadAttention packing), H heads.
 * Replaces attn::mha_block_dense (include/attn_api.h:4-7; src/attn_dispatch.cpp:17-133).
 * Errors: D % H != 0 or D % 16 != 0 -> ATTNB_ERR_RUNTIME, like the reference. */
ATTNB_API int attnb_mha_block_dense(const float* x, int T, int D, const float* W_in,
                          const float* b_in, const float* W_out, const float* b_out, int H,
                          int causal, float* y, int precision);
/* Device-pointer MHA block over `batch` independent sequences laid out as
 * x[batch, T, D] -> y[batch, T, D]. */
ATTNB_API int attnb_mha_block_dense_dev(const float* x, int batch, int T, int D, const float* W_in,
                              const float* b_in, const float* W_out, const float* b_out,
                              int H, int causal, float* y, int precision, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* ATTNB_H */
