// pymodule.cpp -- the `_attn_cpu` extension module with the reference's
// Python signatures (src/bindings.cpp:102-124 of the reference): arrays are
// force-cast to C-contiguous float32, shapes are checked with the same
// messages (src/bindings.cpp:17-39, 55-61), and a new output array is
// returned.  It adds attn_step_dense / attn_block_dense, which the
// reference's tests call (tests/test_attn_step.py:32, python/attn_cpu/mha_np.py:34)
// but its module never exported, and an optional `precision` argument
// (-1 default, 0 = 3xTF32, 1 = TF32).  Work runs on the current CUDA device
// through the C ABI in attnb.h, with the GIL released.
#include <pybind11/numpy.h>
#include <pybind11/pybind11.h>

#include <cmath>
#include <new>
#include <stdexcept>
#include <string>
#include <vector>

#include "../../include/attnb.h"

namespace py = pybind11;
using farray = py::array_t<float, py::array::c_style | py::array::forcecast>;

namespace {

void rethrow(int rc) {
  if (rc == ATTNB_OK) return;
  const std::string msg = attnb_last_error();
  if (rc == ATTNB_ERR_INVALID_ARGUMENT) throw std::invalid_argument(msg);
  if (rc == ATTNB_ERR_OUT_OF_MEMORY) throw std::bad_alloc();
  throw std::runtime_error(msg);
}

// A new, uninitialised result array in page-locked memory from the library's
// pool (the device-to-host copy of the result then runs by DMA at full rate
// and touches no fresh pages), or in ordinary memory when the pool is full.
// The block returns to the pool when the array is freed.
py::array_t<float> result_array(std::vector<py::ssize_t> shape) {
  size_t n = 1;
  for (py::ssize_t d : shape) n *= (size_t)d;
  void* p = nullptr;
  if (n > 0 && attnb_host_alloc(n * sizeof(float), &p) == ATTNB_OK && p) {
    py::capsule owner(p, [](void* q) { attnb_host_free(q); });
    return py::array_t<float>(shape, static_cast<float*>(p), owner);
  }
  return py::array_t<float>(shape);
}

py::array_t<float> mha_block_dense_py(farray x, farray W_in, farray b_in, farray W_out,
                                      farray b_out, int num_heads, bool causal, int precision) {
  if (x.ndim() != 2) throw std::invalid_argument("x must be [T,D]");
  if (W_in.ndim() != 2) throw std::invalid_argument("W_in must be [3D,D]");
  if (b_in.ndim() != 1) throw std::invalid_argument("b_in must be [3D]");
  if (W_out.ndim() != 2) throw std::invalid_argument("W_out must be [D,D]");
  if (b_out.ndim() != 1) throw std::invalid_argument("b_out must be [D]");
  const int T = (int)x.shape(0), D = (int)x.shape(1);
  if ((int)W_in.shape(0) != 3 * D || (int)W_in.shape(1) != D)
    throw std::invalid_argument("W_in shape must be [3D, D]");
  if ((int)b_in.shape(0) != 3 * D) throw std::invalid_argument("b_in shape must be [3D]");
  if ((int)W_out.shape(0) != D || (int)W_out.shape(1) != D)
    throw std::invalid_argument("W_out shape must be [D, D]");
  if ((int)b_out.shape(0) != D) throw std::invalid_argument("b_out shape must be [D]");
  if (num_heads <= 0 || (D % num_heads) != 0)
    throw std::invalid_argument("num_heads must divide D");
  py::array_t<float> y = result_array({T, D});
  const float *px = x.data(), *pwi = W_in.data(), *pbi = b_in.data(), *pwo = W_out.data(),
              *pbo = b_out.data();
  float* py_ = y.mutable_data();
  int rc;
  {
    py::gil_scoped_release nogil;
    rc = attnb_mha_block_dense(px, T, D, pwi, pbi, pwo, pbo, num_heads, causal ? 1 : 0, py_,
                               precision);
  }
  rethrow(rc);
  return y;
}

py::array_t<float> gemm_common(farray A, farray B, float alpha, float beta, int precision,
                               bool jit) {
  if (A.ndim() != 2 || B.ndim() != 2)
    throw std::invalid_argument("A and B must be 2D: A[M,K], B[K,N]");
  const int M = (int)A.shape(0), K = (int)A.shape(1), KB = (int)B.shape(0),
            N = (int)B.shape(1);
  if (K != KB) throw std::invalid_argument("Inner dim mismatch: A[M,K] x B[K,N]");
  // C starts as zeros, so beta * C contributes nothing for a finite beta and
  // the call runs with beta = 0 (C never read); a non-finite beta keeps its
  // NaN product with explicit zeros, and K = 0 (C left untouched) returns
  // them.  (The reference reads an uninitialised buffer there,
  // src/bindings.cpp:64-71.)
  py::array_t<float> C = result_array({M, N});
  if ((size_t)M * N && (K <= 0 || !std::isfinite(beta)))
    std::fill(C.mutable_data(), C.mutable_data() + (size_t)M * N, 0.f);
  if (std::isfinite(beta)) beta = 0.f;
  const float *pa = A.data(), *pb = B.data();
  float* pc = C.mutable_data();
  int rc;
  {
    py::gil_scoped_release nogil;
    rc = jit ? attnb_gemm_jit(pa, M, K, pb, N, pc, alpha, beta, precision)
             : attnb_sgemm(pa, M, K, pb, N, pc, alpha, beta, precision);
  }
  rethrow(rc);
  return C;
}

py::array_t<float> gemm_py(farray A, farray B, float alpha, float beta, int precision) {
  return gemm_common(A, B, alpha, beta, precision, false);
}
py::array_t<float> gemm_jit_py(farray A, farray B, float alpha, float beta, int precision) {
  return gemm_common(A, B, alpha, beta, precision, true);
}

py::array_t<float> attn_step_dense_py(farray Q, farray K, farray V) {
  if (Q.ndim() != 2) throw std::invalid_argument("Q must be [H,Dh]");
  if (K.ndim() != 3 || V.ndim() != 3) throw std::invalid_argument("K and V must be [H,T,Dh]");
  const int H = (int)Q.shape(0), Dh = (int)Q.shape(1);
  attnb_tensor q{Q.data(), H, 1, Dh, (int64_t)Dh, 0, 1};
  attnb_tensor k{K.data(), (int)K.shape(0), (int)K.shape(1), (int)K.shape(2),
                 (int64_t)K.shape(1) * K.shape(2), (int64_t)K.shape(2), 1};
  attnb_tensor v{V.data(), (int)V.shape(0), (int)V.shape(1), (int)V.shape(2),
                 (int64_t)V.shape(1) * V.shape(2), (int64_t)V.shape(2), 1};
  py::array_t<float> O = result_array({H, Dh});
  attnb_mtensor o{O.mutable_data(), H, 1, Dh, (int64_t)Dh, 0, 1};
  int rc;
  {
    py::gil_scoped_release nogil;
    rc = attnb_attn_step_dense(&q, &k, &v, &o);
  }
  rethrow(rc);
  return O;
}

py::array_t<float> attn_block_dense_py(farray Q, farray K, farray V, bool causal, int precision) {
  if (Q.ndim() != 3 || K.ndim() != 3 || V.ndim() != 3)
    throw std::invalid_argument("Q must be [H,L,Dh], K and V [H,T,Dh]");
  const int H = (int)Q.shape(0), L = (int)Q.shape(1), Dh = (int)Q.shape(2);
  attnb_tensor q{Q.data(), H, L, Dh, (int64_t)L * Dh, (int64_t)Dh, 1};
  attnb_tensor k{K.data(), (int)K.shape(0), (int)K.shape(1), (int)K.shape(2),
                 (int64_t)K.shape(1) * K.shape(2), (int64_t)K.shape(2), 1};
  attnb_tensor v{V.data(), (int)V.shape(0), (int)V.shape(1), (int)V.shape(2),
                 (int64_t)V.shape(1) * V.shape(2), (int64_t)V.shape(2), 1};
  py::array_t<float> O = result_array({H, L, Dh});
  attnb_mtensor o{O.mutable_data(), H, L, Dh, (int64_t)L * Dh, (int64_t)Dh, 1};
  int rc;
  {
    py::gil_scoped_release nogil;
    rc = attnb_attn_block_dense(&q, &k, &v, &o, causal ? 1 : 0, precision);
  }
  rethrow(rc);
  return O;
}

// Resident K/V cache for multi-step decode (attnb_kv_cache_*): K and V stay on
// the device between steps; a step moves only the new token and the query in
// and the output row out.
class KVCache {
 public:
  KVCache(int H, int Dh, int capacity) : H_(H), Dh_(Dh) {
    rethrow(attnb_kv_cache_create(H, Dh, capacity, &c_));
  }
  ~KVCache() {
    if (c_) attnb_kv_cache_destroy(c_);
  }
  KVCache(const KVCache&) = delete;
  KVCache& operator=(const KVCache&) = delete;

  int length() const {
    int n = 0;
    rethrow(attnb_kv_cache_length(c_, &n));
    return n;
  }
  void truncate(int n) { rethrow(attnb_kv_cache_truncate(c_, n)); }

  // k, v: [H, n, Dh]; returns once they are copied.
  void append(farray k, farray v) {
    if (k.ndim() != 3 || v.ndim() != 3) throw std::invalid_argument("k and v must be [H,n,Dh]");
    if (k.shape(0) != H_ || k.shape(2) != Dh_ || v.shape(0) != H_ || v.shape(1) != k.shape(1) ||
        v.shape(2) != Dh_)
      throw std::invalid_argument("k and v must both be [H,n,Dh] with the cache's H and Dh");
    const float *pk = k.data(), *pv = v.data();
    const int n = (int)k.shape(1);
    int rc;
    {
      py::gil_scoped_release nogil;
      rc = attnb_kv_cache_append(c_, pk, pv, n, nullptr);
      if (rc == ATTNB_OK) rc = attnb_stream_status(nullptr);  // the host arrays are read
    }
    rethrow(rc);
  }

  // q: [H, Dh]; k_new / v_new: [H, Dh] (both or neither) appended first.
  py::array_t<float> step(farray q, py::object k_new, py::object v_new) {
    auto row = [&](const farray& x, const char* what) {
      if (x.ndim() != 2 || x.shape(0) != H_ || x.shape(1) != Dh_)
        throw std::invalid_argument(std::string(what) + " must be [H,Dh] with the cache's H and Dh");
    };
    row(q, "q");
    if (k_new.is_none() != v_new.is_none())
      throw std::invalid_argument("k_new and v_new are given together");
    farray kn, vn;
    const float *pk = nullptr, *pv = nullptr;
    if (!k_new.is_none()) {
      kn = k_new.cast<farray>();
      vn = v_new.cast<farray>();
      row(kn, "k_new");
      row(vn, "v_new");
      pk = kn.data();
      pv = vn.data();
    }
    py::array_t<float> O = result_array({H_, Dh_});
    const float* pq = q.data();
    float* po = O.mutable_data();
    int rc;
    {
      py::gil_scoped_release nogil;
      rc = attnb_kv_cache_step(c_, pq, pk, pv, po);
    }
    rethrow(rc);
    return O;
  }

 private:
  attnb_kv_cache* c_ = nullptr;
  int H_, Dh_;
};

}  // namespace

PYBIND11_MODULE(_attn_cpu, m) {
  m.doc() = "Dense attention (step + block) and SGEMM on B200 (sm_100a)";
  m.def("mha_block_dense", &mha_block_dense_py, py::arg("x"), py::arg("W_in"), py::arg("b_in"),
        py::arg("W_out"), py::arg("b_out"), py::arg("num_heads"), py::arg("causal") = false,
        py::arg("precision") = -1,
        "Full MHA block: x:[T,D], W_in:[3D,D], b_in:[3D], W_out:[D,D], b_out:[D] -> y:[T,D]");
  m.def("gemm", &gemm_py, py::arg("A"), py::arg("B"), py::arg("alpha") = 1.0f,
        py::arg("beta") = 0.0f, py::arg("precision") = -1,
        "SGEMM: C = alpha * A@B + beta*C, A:[M,K], B:[K,N] -> C:[M,N]");
  m.def("gemm_jit", &gemm_jit_py, py::arg("A"), py::arg("B"), py::arg("alpha") = 1.0f,
        py::arg("beta") = 0.0f, py::arg("precision") = -1,
        "SGEMM (same kernel as gemm): C = alpha * A@B + beta*C -> C:[M,N]");
  m.def("attn_step_dense", &attn_step_dense_py, py::arg("Q"), py::arg("K"), py::arg("V"),
        "Decode step: Q:[H,Dh], K,V:[H,T,Dh] -> O:[H,Dh]");
  m.def("attn_block_dense", &attn_block_dense_py, py::arg("Q"), py::arg("K"), py::arg("V"),
        py::arg("causal") = false, py::arg("precision") = -1,
        "Prefill: Q:[H,L,Dh], K,V:[H,T,Dh] -> O:[H,L,Dh]");
  m.def("version", &attnb_version);
  py::class_<KVCache>(m, "KVCache",
                      "Resident K/V cache on the current device for multi-step decode")
      .def(py::init<int, int, int>(), py::arg("H"), py::arg("Dh"), py::arg("capacity"))
      .def("__len__", &KVCache::length)
      .def("truncate", &KVCache::truncate, py::arg("length"),
           "Drop tokens from the end: keep the first `length`.")
      .def("append", &KVCache::append, py::arg("k"), py::arg("v"),
           "Append k, v: [H, n, Dh] behind the valid tokens.")
      .def("step", &KVCache::step, py::arg("q"), py::arg("k_new") = py::none(),
           py::arg("v_new") = py::none(),
           "Append k_new, v_new ([H, Dh]) if given, then O[H, Dh] = attention of q over the "
           "cache (the function of attn_step_dense).");
}
