// pybind11 module `orchard_core`: the reference's operator surface (src/bindings.cpp:10-83)
// over the B200 backend.
//
// Same classes, methods, argument names and order: MetalBackend(initialize,
// is_available, get_device_name, run_*), DType{Float32, Float16, Int8}, Tensor(backend,
// shape, dtype) with copy_from_host/copy_to_host/shape/numel/size_bytes.
//
// The reference passes raw buffers to kernels that assume half activations regardless of
// the tensor's declared dtype, and its host declares Float32 activations
// (orchard/model.py:86-92). Here each op reads the Tensor's dtype and runs the kernel for
// it (Float16 is the Metal kernels' behaviour; Float32 is computed and stored in fp32),
// checks every extent against the tensor sizes, and raises RuntimeError instead of
// reading out of bounds or returning silently.
#include <pybind11/numpy.h>
#include <pybind11/pybind11.h>
#include <pybind11/stl.h>

#include <stdexcept>
#include <string>

#include "core_backend.h"
#include "orchard_b200.h"

namespace py = pybind11;
using orchard::platform::check_status;
using orchard::platform::MetalBackend;
using orchard::runtime::DType;
using orchard::runtime::Tensor;

namespace {

void need(const Tensor& t, size_t elems, const char* op, const char* arg) {
  const size_t have = t.numel();
  if (have < elems)
    throw std::runtime_error(std::string(op) + ": tensor '" + arg + "' has " + std::to_string(have) +
                             " elements, the op needs " + std::to_string(elems));
}

int act(const Tensor& t, const char* op, const char* arg) {
  if (t.dtype() == DType::Float32) return ORCH_F32;
  if (t.dtype() == DType::Float16) return ORCH_F16;
  throw std::runtime_error(std::string(op) + ": tensor '" + arg + "' must be Float16 or Float32");
}

void same(int a, int b, const char* op) {
  if (a != b) throw std::runtime_error(std::string(op) + ": tensors must share one dtype");
}

size_t sz(uint32_t a) { return (size_t)a; }

py::array to_numpy(const Tensor& t) {
  std::vector<py::ssize_t> shape;
  for (size_t s : t.shape()) shape.push_back((py::ssize_t)s);
  py::array out;
  switch (t.dtype()) {
    case DType::Float32: out = py::array_t<float>(shape); break;
    case DType::Float16: out = py::array(py::dtype("float16"), shape); break;
    default: out = py::array_t<int8_t>(shape); break;
  }
  py::buffer_info info = out.request();
  if (t.size_bytes()) t.copy_to_host(info.ptr, t.size_bytes());
  return out;
}

void require_contiguous(const py::buffer_info& info) {
  py::ssize_t expect = info.itemsize;
  for (py::ssize_t d = info.ndim - 1; d >= 0; --d) {
    if (info.shape[d] > 1 && info.strides[d] != expect)
      throw std::runtime_error("buffer must be C-contiguous");
    expect *= info.shape[d];
  }
}

}  // namespace

PYBIND11_MODULE(orchard_core, m) {
  m.doc() = "Orchard core runtime on NVIDIA B200 (sm_100a)";

  py::class_<MetalBackend>(m, "MetalBackend")
      .def(py::init<>())
      .def("initialize", &MetalBackend::initialize, py::arg("resource_path"))
      .def("is_available", &MetalBackend::is_available)
      .def("get_device_name", &MetalBackend::get_device_name)
      .def("synchronize", &MetalBackend::synchronize)
      .def("run_matmul",
           [](MetalBackend& self, Tensor& a, Tensor& b, Tensor& c, uint32_t M, uint32_t N, uint32_t K) {
             need(a, sz(M) * K, "run_matmul", "a");
             need(b, sz(K) * N, "run_matmul", "b");
             need(c, sz(M) * N, "run_matmul", "c");
             const int d = act(a, "run_matmul", "a");
             same(d, act(b, "run_matmul", "b"), "run_matmul");
             same(d, act(c, "run_matmul", "c"), "run_matmul");
             if (d == ORCH_F32)
               check_status(orch_matmul((const float*)a.data(), (const float*)b.data(), (float*)c.data(), M, N, K,
                                        self.stream()), "run_matmul");
             else
               check_status(orch_matmul_simd(a.data(), b.data(), c.data(), M, N, K, self.stream()), "run_matmul");
           })
      .def("run_matmul_simd",
           [](MetalBackend& self, Tensor& a, Tensor& b, Tensor& c, uint32_t M, uint32_t N, uint32_t K) {
             need(a, sz(M) * K, "run_matmul_simd", "a");
             need(b, sz(K) * N, "run_matmul_simd", "b");
             need(c, sz(M) * N, "run_matmul_simd", "c");
             const int d = act(a, "run_matmul_simd", "a");
             same(d, act(b, "run_matmul_simd", "b"), "run_matmul_simd");
             same(d, act(c, "run_matmul_simd", "c"), "run_matmul_simd");
             if (d == ORCH_F16)
               check_status(orch_matmul_simd(a.data(), b.data(), c.data(), M, N, K, self.stream()), "run_matmul_simd");
             else
               check_status(orch_matmul((const float*)a.data(), (const float*)b.data(), (float*)c.data(), M, N, K,
                                        self.stream()), "run_matmul_simd");
           })
      .def("run_rmsnorm",
           [](MetalBackend& self, Tensor& input, Tensor& weight, Tensor& output, float epsilon, uint32_t N,
              uint32_t count) {
             need(input, sz(N) * count, "run_rmsnorm", "input");
             need(weight, N, "run_rmsnorm", "weight");
             need(output, sz(N) * count, "run_rmsnorm", "output");
             check_status(orch_rmsnorm_ex(input.data(), act(input, "run_rmsnorm", "input"), weight.data(),
                                          act(weight, "run_rmsnorm", "weight"), output.data(),
                                          act(output, "run_rmsnorm", "output"), epsilon, N, count, self.stream()),
                          "run_rmsnorm");
           })
      .def("run_rope",
           [](MetalBackend& self, Tensor& input, Tensor& freqs_cos, Tensor& freqs_sin, Tensor& output,
              uint32_t head_dim, uint32_t num_heads, uint32_t seq_len) {
             if (head_dim % 2) throw std::runtime_error("run_rope: head_dim must be even");
             const size_t row = sz(num_heads) * head_dim;
             need(input, row * seq_len, "run_rope", "input");
             need(output, row * seq_len, "run_rope", "output");
             const int td = act(freqs_cos, "run_rope", "freqs_cos");
             same(td, act(freqs_sin, "run_rope", "freqs_sin"), "run_rope");
             const int id = act(input, "run_rope", "input"), od = act(output, "run_rope", "output");
             const size_t half = head_dim / 2;
             if (freqs_cos.numel() >= half * seq_len && freqs_sin.numel() >= half * seq_len) {
               check_status(orch_rope_ex(input.data(), id, freqs_cos.data(), freqs_sin.data(), td, output.data(), od,
                                         head_dim, num_heads, seq_len, self.stream()), "run_rope");
             } else {
               // One row of angles for every row (a [head_dim/2] table).
               need(freqs_cos, half, "run_rope", "freqs_cos");
               need(freqs_sin, half, "run_rope", "freqs_sin");
               const size_t ib = id == ORCH_F32 ? 4 : 2, ob = od == ORCH_F32 ? 4 : 2;
               for (uint32_t r = 0; r < seq_len; ++r)
                 check_status(orch_rope_ex((const char*)input.data() + r * row * ib, id, freqs_cos.data(),
                                           freqs_sin.data(), td, (char*)output.data() + r * row * ob, od, head_dim,
                                           num_heads, 1, self.stream()), "run_rope");
             }
           })
      .def("run_gemv_q8_0",
           [](MetalBackend& self, Tensor& weights, Tensor& scales, Tensor& input, Tensor& output, uint32_t K,
              uint32_t N) {
             need(weights, sz(N) * K, "run_gemv_q8_0", "weights");
             if (scales.dtype() != DType::Float16) throw std::runtime_error("run_gemv_q8_0: scales must be Float16");
             need(scales, sz(N) * (K / 32), "run_gemv_q8_0", "scales");
             need(input, K, "run_gemv_q8_0", "input");
             need(output, N, "run_gemv_q8_0", "output");
             check_status(orch_gemm_q8_0_ex(weights.data(), scales.data(), input.data(), act(input, "run_gemv_q8_0", "input"),
                                            output.data(), act(output, "run_gemv_q8_0", "output"), K, N, 1,
                                            self.stream()), "run_gemv_q8_0");
           })
      .def("run_gemv_q4_0",
           [](MetalBackend& self, Tensor& weights, Tensor& scales, Tensor& input, Tensor& output, uint32_t K,
              uint32_t N) {
             if (weights.dtype() != DType::Int8) throw std::runtime_error("run_gemv_q4_0: weights must be Int8");
             need(weights, sz(N) * (K / 2), "run_gemv_q4_0", "weights");
             if (scales.dtype() != DType::Float16) throw std::runtime_error("run_gemv_q4_0: scales must be Float16");
             need(scales, sz(N) * (K / 32), "run_gemv_q4_0", "scales");
             need(input, K, "run_gemv_q4_0", "input");
             need(output, N, "run_gemv_q4_0", "output");
             check_status(orch_gemm_q4_0_ex(weights.data(), scales.data(), input.data(), act(input, "run_gemv_q4_0", "input"),
                                            output.data(), act(output, "run_gemv_q4_0", "output"), K, N, 1,
                                            self.stream()), "run_gemv_q4_0");
           })
      .def("run_gemm_q4_0",
           [](MetalBackend& self, Tensor& weights, Tensor& scales, Tensor& input, Tensor& output, uint32_t K,
              uint32_t N, uint32_t B) {
             if (weights.dtype() != DType::Int8) throw std::runtime_error("run_gemm_q4_0: weights must be Int8");
             need(weights, sz(N) * (K / 2), "run_gemm_q4_0", "weights");
             if (scales.dtype() != DType::Float16) throw std::runtime_error("run_gemm_q4_0: scales must be Float16");
             need(scales, sz(N) * (K / 32), "run_gemm_q4_0", "scales");
             need(input, sz(B) * K, "run_gemm_q4_0", "input");
             need(output, sz(B) * N, "run_gemm_q4_0", "output");
             check_status(orch_gemm_q4_0_ex(weights.data(), scales.data(), input.data(), act(input, "run_gemm_q4_0", "input"),
                                            output.data(), act(output, "run_gemm_q4_0", "output"), K, N, B,
                                            self.stream()), "run_gemm_q4_0");
           })
      .def("run_add",
           [](MetalBackend& self, Tensor& a, Tensor& b, Tensor& c, uint32_t size) {
             need(a, size, "run_add", "a");
             need(b, size, "run_add", "b");
             need(c, size, "run_add", "c");
             const int d = act(a, "run_add", "a");
             same(d, act(b, "run_add", "b"), "run_add");
             same(d, act(c, "run_add", "c"), "run_add");
             check_status(orch_binary_ex(0, a.data(), b.data(), c.data(), d, size, self.stream()), "run_add");
           })
      .def("run_mul",
           [](MetalBackend& self, Tensor& a, Tensor& b, Tensor& c, uint32_t size) {
             need(a, size, "run_mul", "a");
             need(b, size, "run_mul", "b");
             need(c, size, "run_mul", "c");
             const int d = act(a, "run_mul", "a");
             same(d, act(b, "run_mul", "b"), "run_mul");
             same(d, act(c, "run_mul", "c"), "run_mul");
             check_status(orch_binary_ex(1, a.data(), b.data(), c.data(), d, size, self.stream()), "run_mul");
           })
      .def("run_silu",
           [](MetalBackend& self, Tensor& in, Tensor& out, uint32_t size) {
             need(in, size, "run_silu", "in");
             need(out, size, "run_silu", "out");
             const int d = act(in, "run_silu", "in");
             same(d, act(out, "run_silu", "out"), "run_silu");
             check_status(orch_silu_ex(in.data(), out.data(), d, size, self.stream()), "run_silu");
           })
      .def("run_softmax",
           [](MetalBackend& self, Tensor& input, Tensor& output, uint32_t rows, uint32_t cols) {
             need(input, sz(rows) * cols, "run_softmax", "input");
             need(output, sz(rows) * cols, "run_softmax", "output");
             check_status(orch_softmax_ex(input.data(), act(input, "run_softmax", "input"), output.data(),
                                          act(output, "run_softmax", "output"), rows, cols, self.stream()),
                          "run_softmax");
           })
      .def("run_embedding",
           [](MetalBackend& self, Tensor& input_ids, Tensor& weights, Tensor& output, uint32_t num_tokens,
              uint32_t hidden_dim) {
             // ids are int32 bits in any 4-byte container (examples/full_test.py:135 uses Float32)
             if (input_ids.size_bytes() < sz(num_tokens) * 4)
               throw std::runtime_error("run_embedding: input_ids holds fewer than num_tokens int32 values");
             if (hidden_dim == 0) throw std::runtime_error("run_embedding: hidden_dim must be positive");
             need(output, sz(num_tokens) * hidden_dim, "run_embedding", "output");
             const size_t vocab = weights.numel() / hidden_dim;
             check_status(orch_embedding_ex(input_ids.data(), weights.data(), act(weights, "run_embedding", "weights"),
                                            output.data(), act(output, "run_embedding", "output"), num_tokens,
                                            hidden_dim, (uint32_t)vocab, self.stream()), "run_embedding");
           });

  py::enum_<DType>(m, "DType")
      .value("Float32", DType::Float32)
      .value("Float16", DType::Float16)
      .value("Int8", DType::Int8)
      .export_values();

  py::class_<Tensor>(m, "Tensor")
      .def(py::init<MetalBackend&, const std::vector<size_t>&, DType>(), py::keep_alive<1, 2>())
      .def("copy_from_host",
           [](Tensor& self, py::buffer b) {
             py::buffer_info info = b.request();
             require_contiguous(info);
             self.copy_from_host(info.ptr, (size_t)(info.size * info.itemsize));
           })
      .def("copy_to_host",
           [](Tensor& self, py::buffer b) {
             py::buffer_info info = b.request(true);
             require_contiguous(info);
             const size_t expected = self.size_bytes();
             if ((size_t)(info.size * info.itemsize) < expected) throw std::runtime_error("Buffer too small");
             self.copy_to_host(info.ptr, expected);
           })
      // The reference's Python calls copy_to_host() without a destination
      // (orchard/model.py:113-115,358); that form returns a new array of the tensor's dtype.
      .def("copy_to_host", [](Tensor& self) { return to_numpy(self); })
      .def("shape", &Tensor::shape)
      .def("numel", &Tensor::numel)
      .def("size_bytes", &Tensor::size_bytes)
      .def("data_ptr", [](Tensor& self) { return (uintptr_t)self.data(); })
      .def("dtype", &Tensor::dtype);
}
