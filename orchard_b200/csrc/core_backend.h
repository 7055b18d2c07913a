// Host-side mirror of the reference's backend/runtime classes, implemented over the C ABI.
//
// The class keeps the reference's name `MetalBackend` and method set
// (src/platform/metal_backend.h:9-55) because it *is* the interface the operator surface
// binds to; `Tensor`/`DType` follow src/runtime/tensor.h:11-42. Differences, all
// deliberate: ops run asynchronously on one CUDA stream and copies to the host
// synchronise (observably the reference's synchronous behaviour, src/platform/
// metal_backend.mm:208-235); failures throw std::runtime_error instead of silently
// returning (metal_backend.mm:206).
#pragma once

#include <cstdint>
#include <string>
#include <vector>

namespace orchard {
namespace platform {

class MetalBackend {
 public:
  MetalBackend();
  ~MetalBackend();

  void initialize(const std::string& resource_path);
  bool is_available() const;
  std::string get_device_name() const;

  void* create_buffer(size_t size);
  void copy_to_buffer(void* buffer, const void* data, size_t size);
  void copy_from_buffer(void* buffer, void* data, size_t size);
  void release_buffer(void* buffer);

  // The reference's raw-pointer ops, with the Metal kernels' half activations.
  void run_matmul(void* a, void* b, void* c, uint32_t M, uint32_t N, uint32_t K);
  void run_matmul_simd(void* a, void* b, void* c, uint32_t M, uint32_t N, uint32_t K);
  void run_rmsnorm(void* input, void* weight, void* output, float epsilon, uint32_t N, uint32_t count);
  void run_rope(void* input, void* freqs_cos, void* freqs_sin, void* output, uint32_t head_dim,
                uint32_t num_heads, uint32_t seq_len);
  void run_gemv_q8_0(void* weights, void* scales, void* input, void* output, uint32_t K, uint32_t N);
  void run_gemv_q4_0(void* weights, void* scales, void* input, void* output, uint32_t K, uint32_t N);
  void run_gemm_q4_0(void* weights, void* scales, void* input, void* output, uint32_t K, uint32_t N,
                     uint32_t B);
  void run_add(void* a, void* b, void* c, uint32_t size);
  void run_mul(void* a, void* b, void* c, uint32_t size);
  void run_silu(void* in, void* out, uint32_t size);
  void run_softmax(void* input, void* output, uint32_t rows, uint32_t cols);
  void run_embedding(void* input_ids, void* weights, void* output, uint32_t num_tokens,
                     uint32_t hidden_dim, uint32_t vocab);

  void* stream() const { return stream_; }
  void synchronize();

 private:
  void* stream_ = nullptr;  // the legacy default stream: ordered with every copy
  bool initialized_ = false;
};

// Throws std::runtime_error carrying orch_last_error() when status != 0.
void check_status(int status, const char* what);

}  // namespace platform

namespace runtime {

enum class DType { Float32, Float16, Int8 };
size_t dtype_size(DType dt);

class Tensor {
 public:
  Tensor(platform::MetalBackend& backend, const std::vector<size_t>& shape, DType dtype);
  ~Tensor();
  Tensor(const Tensor&) = delete;
  Tensor& operator=(const Tensor&) = delete;
  Tensor(Tensor&& other) noexcept;
  Tensor& operator=(Tensor&& other) noexcept;

  void copy_from_host(const void* data, size_t size);
  void copy_to_host(void* data, size_t size) const;

  void* data() const { return buffer_; }
  const std::vector<size_t>& shape() const { return shape_; }
  DType dtype() const { return dtype_; }
  size_t numel() const;
  size_t size_bytes() const;
  platform::MetalBackend& backend() const { return backend_; }

 private:
  platform::MetalBackend& backend_;
  std::vector<size_t> shape_;
  DType dtype_;
  void* buffer_;
};

}  // namespace runtime
}  // namespace orchard
