// Shared device helpers and host-side status plumbing for liborchard_b200.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <string>
#include <utility>

#include "../../include/orchard_b200.h"

namespace orch {

// ------------------------------------------------------------------------------------
// host status plumbing
// ------------------------------------------------------------------------------------
void set_error(const std::string& msg);
int fail(int status, const std::string& msg);
int cuda_status(cudaError_t e, const char* what);
int check_launch(const char* what);
int num_sms();
int device_index();
uint32_t* device_check_word();  // per-device flag word, set by kernels' own bounds checks
// The allocation-free attention entry point's own flag word on device `dev` (null until that
// entry point has run on the device); orch_device_check reports it with the shared word.
uint32_t* noalloc_check_word(int dev);

inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }
bool pdl_enabled();  // ORCHARD_PDL=0 in the environment turns programmatic launch off

// Launch with an optional cluster shape, and programmatic stream serialization when allowed.
template <typename... KArgs, typename... Args>
cudaError_t launch_k_pdl(bool allow_pdl, void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem,
                         cudaStream_t st, dim3 cluster, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  int n = 0;
  if (cluster.x > 0) {  // dim3(0, 0, 0): no cluster
    attr[n].id = cudaLaunchAttributeClusterDimension;
    attr[n].val.clusterDim.x = cluster.x;
    attr[n].val.clusterDim.y = cluster.y;
    attr[n].val.clusterDim.z = cluster.z;
    ++n;
  }
  if (allow_pdl && pdl_enabled()) {
    attr[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[n].val.programmaticStreamSerializationAllowed = 1;
    ++n;
  }
  cfg.attrs = attr;
  cfg.numAttrs = n;
  return cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
}

// Launch with programmatic dependent launch (when enabled).
template <typename... KArgs, typename... Args>
cudaError_t launch_k(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st, dim3 cluster,
                     Args&&... args) {
  return launch_k_pdl(true, kern, grid, block, smem, st, cluster, std::forward<Args>(args)...);
}
// Launch fully serialised after the previous work in the stream.
template <typename... KArgs, typename... Args>
cudaError_t launch_k_serial(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                            dim3 cluster, Args&&... args) {
  return launch_k_pdl(false, kern, grid, block, smem, st, cluster, std::forward<Args>(args)...);
}

#define ORCH_REQUIRE(cond, msg)                                  \
  do {                                                           \
    if (!(cond)) return ::orch::fail(ORCH_ERR_INVALID, (msg));   \
  } while (0)

// dst = this device's check word, or return ORCH_ERR_NOT_INITIALIZED (kernels must never
// be handed a null flag pointer).
#define ORCH_CHECK_WORD(dst)                                                                    \
  do {                                                                                          \
    (dst) = ::orch::device_check_word();                                                        \
    if ((dst) == nullptr) return ::orch::fail(ORCH_ERR_NOT_INITIALIZED, "no device state for the current device"); \
  } while (0)

#define ORCH_CUDA(call)                                          \
  do {                                                           \
    cudaError_t e_ = (call);                                     \
    if (e_ != cudaSuccess) return ::orch::cuda_status(e_, #call); \
  } while (0)

// ------------------------------------------------------------------------------------
// device helpers
// ------------------------------------------------------------------------------------
template <typename T> __device__ __forceinline__ float to_f32(T v);
template <> __device__ __forceinline__ float to_f32<float>(float v) { return v; }
template <> __device__ __forceinline__ float to_f32<__half>(__half v) { return __half2float(v); }

template <typename T> __device__ __forceinline__ T from_f32(float v);
template <> __device__ __forceinline__ float from_f32<float>(float v) { return v; }
template <> __device__ __forceinline__ __half from_f32<__half>(float v) { return __float2half_rn(v); }

__device__ __forceinline__ uint32_t h2_bits(__half2 h) { return *reinterpret_cast<uint32_t*>(&h); }
__device__ __forceinline__ __half2 bits_h2(uint32_t u) { return *reinterpret_cast<__half2*>(&u); }

// (a & b) | c in one LOP3.
__device__ __forceinline__ uint32_t lop3_and_or(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t r;
  asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(r) : "r"(a), "r"(b), "r"(c));
  return r;
}

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t r;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(sel));
  return r;
}

// D += A(16x16 f16, row) * B(16x8 f16, col), fp32 accumulators.
__device__ __forceinline__ void mma_16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                          uint32_t a3, uint32_t b0, uint32_t b1) {
  asm(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 "
      "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// Streaming 16-byte load: read once, not kept in L1.
// fp32 -> TF32 (round to nearest, ties away), as the 32-bit pattern an m16n8k8 TF32 operand takes
__device__ __forceinline__ uint32_t to_tf32(float v) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(v));
  return r;
}
// d += a.b, m16n8k8, TF32 operands, fp32 accumulator
__device__ __forceinline__ void mma_tf32(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm("mma.sync.aligned.m16n8k8.row.col.f32.tf32.tf32.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint4 ld_stream16(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

// Programmatic dependent launch. A kernel launched with the programmatic-serialization
// attribute may start while the previous kernel on the stream is still running; it must
// call pdl_wait() before reading that kernel's output or writing anything the previous
// kernel reads. pdl_trigger() lets the next kernel start launching. Both are no-ops for a
// kernel launched without the attribute.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" :::); }

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Block-wide sum for blockDim.x a multiple of 32 (<= 1024); `red` holds >= 32 floats.
__device__ __forceinline__ float block_sum(float v, float* red) {
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = blockDim.x >> 5;
  v = warp_sum(v);
  __syncthreads();
  if (lane == 0) red[wid] = v;
  __syncthreads();
  float t = lane < nw ? red[lane] : 0.f;
  return warp_sum(t);
}
__device__ __forceinline__ float block_max(float v, float* red) {
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = blockDim.x >> 5;
  v = warp_max(v);
  __syncthreads();
  if (lane == 0) red[wid] = v;
  __syncthreads();
  float t = lane < nw ? red[lane] : -INFINITY;
  return warp_max(t);
}

}  // namespace orch
