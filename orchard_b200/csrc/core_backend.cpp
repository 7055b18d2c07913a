// MetalBackend / Tensor over liborchard_b200 (see core_backend.h).
#include "core_backend.h"

#include <numeric>
#include <stdexcept>

#include "orchard_b200.h"

namespace orchard {
namespace platform {

void check_status(int status, const char* what) {
  if (status != ORCH_OK)
    throw std::runtime_error(std::string(what) + " failed (" + orch_status_string(status) +
                             "): " + orch_last_error());
}

MetalBackend::MetalBackend() {}
MetalBackend::~MetalBackend() {}

// Reference: metal_backend.mm:42-169 compiles the .metal sources under resource_path.
// The kernels here are compiled ahead of time; the path is only validated.
void MetalBackend::initialize(const std::string& resource_path) {
  check_status(orch_init(0, resource_path.empty() ? nullptr : resource_path.c_str()), "initialize");
  initialized_ = true;
}

bool MetalBackend::is_available() const { return orch_is_available() != 0; }

std::string MetalBackend::get_device_name() const {
  char buf[256];
  if (orch_device_name(buf, sizeof(buf)) != ORCH_OK) return "unavailable";
  return buf;
}

void* MetalBackend::create_buffer(size_t size) {
  void* p = nullptr;
  if (orch_alloc(size, &p) != ORCH_OK) return nullptr;
  return p;
}
void MetalBackend::copy_to_buffer(void* buffer, const void* data, size_t size) {
  check_status(orch_h2d(buffer, data, size, stream_), "copy_to_buffer");
}
void MetalBackend::copy_from_buffer(void* buffer, void* data, size_t size) {
  check_status(orch_d2h(data, buffer, size, stream_), "copy_from_buffer");
}
void MetalBackend::release_buffer(void* buffer) { orch_free(buffer); }
void MetalBackend::synchronize() { check_status(orch_sync(stream_), "synchronize"); }

void MetalBackend::run_matmul(void* a, void* b, void* c, uint32_t M, uint32_t N, uint32_t K) {
  check_status(orch_matmul((const float*)a, (const float*)b, (float*)c, M, N, K, stream_), "run_matmul");
}
void MetalBackend::run_matmul_simd(void* a, void* b, void* c, uint32_t M, uint32_t N, uint32_t K) {
  check_status(orch_matmul_simd(a, b, c, M, N, K, stream_), "run_matmul_simd");
}
void MetalBackend::run_rmsnorm(void* in, void* w, void* out, float eps, uint32_t N, uint32_t count) {
  check_status(orch_rmsnorm(in, w, out, eps, N, count, stream_), "run_rmsnorm");
}
void MetalBackend::run_rope(void* in, void* c, void* s, void* out, uint32_t hd, uint32_t nh, uint32_t sl) {
  check_status(orch_rope(in, c, s, out, hd, nh, sl, stream_), "run_rope");
}
void MetalBackend::run_gemv_q8_0(void* w, void* s, void* in, void* out, uint32_t K, uint32_t N) {
  check_status(orch_gemv_q8_0(w, s, in, out, K, N, stream_), "run_gemv_q8_0");
}
void MetalBackend::run_gemv_q4_0(void* w, void* s, void* in, void* out, uint32_t K, uint32_t N) {
  check_status(orch_gemv_q4_0(w, s, in, out, K, N, stream_), "run_gemv_q4_0");
}
void MetalBackend::run_gemm_q4_0(void* w, void* s, void* in, void* out, uint32_t K, uint32_t N, uint32_t B) {
  check_status(orch_gemm_q4_0(w, s, in, out, K, N, B, stream_), "run_gemm_q4_0");
}
void MetalBackend::run_add(void* a, void* b, void* c, uint32_t size) {
  check_status(orch_add(a, b, c, size, stream_), "run_add");
}
void MetalBackend::run_mul(void* a, void* b, void* c, uint32_t size) {
  check_status(orch_mul(a, b, c, size, stream_), "run_mul");
}
void MetalBackend::run_silu(void* in, void* out, uint32_t size) {
  check_status(orch_silu(in, out, size, stream_), "run_silu");
}
void MetalBackend::run_softmax(void* in, void* out, uint32_t rows, uint32_t cols) {
  check_status(orch_softmax(in, out, rows, cols, stream_), "run_softmax");
}
void MetalBackend::run_embedding(void* ids, void* w, void* out, uint32_t n, uint32_t hd, uint32_t vocab) {
  check_status(orch_embedding(ids, w, out, n, hd, vocab, stream_), "run_embedding");
}

}  // namespace platform

namespace runtime {

size_t dtype_size(DType dt) {
  switch (dt) {
    case DType::Float32: return 4;
    case DType::Float16: return 2;
    default: return 1;
  }
}

Tensor::Tensor(platform::MetalBackend& backend, const std::vector<size_t>& shape, DType dtype)
    : backend_(backend), shape_(shape), dtype_(dtype), buffer_(nullptr) {
  buffer_ = backend_.create_buffer(size_bytes());
  if (!buffer_) throw std::runtime_error(std::string("Failed to allocate tensor on GPU: ") + orch_last_error());
}

Tensor::~Tensor() {
  if (buffer_) backend_.release_buffer(buffer_);
}

Tensor::Tensor(Tensor&& o) noexcept : backend_(o.backend_), shape_(std::move(o.shape_)), dtype_(o.dtype_), buffer_(o.buffer_) {
  o.buffer_ = nullptr;
}

Tensor& Tensor::operator=(Tensor&& o) noexcept {
  if (this != &o) {
    if (buffer_) backend_.release_buffer(buffer_);
    shape_ = std::move(o.shape_);
    dtype_ = o.dtype_;
    buffer_ = o.buffer_;
    o.buffer_ = nullptr;
  }
  return *this;
}

// An empty shape has no elements, as in the reference (src/runtime/tensor.cpp:51-54).
size_t Tensor::numel() const {
  if (shape_.empty()) return 0;
  return std::accumulate(shape_.begin(), shape_.end(), (size_t)1, std::multiplies<size_t>());
}
size_t Tensor::size_bytes() const { return numel() * dtype_size(dtype_); }

void Tensor::copy_from_host(const void* data, size_t size) {
  if (size != size_bytes()) throw std::runtime_error("Size mismatch in copy_from_host");
  backend_.copy_to_buffer(buffer_, data, size);
}
void Tensor::copy_to_host(void* data, size_t size) const {
  if (size != size_bytes()) throw std::runtime_error("Size mismatch in copy_to_host");
  backend_.copy_from_buffer(buffer_, data, size);
}

}  // namespace runtime
}  // namespace orchard
