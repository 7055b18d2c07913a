// On-device packers, bit-identical to the host rules.
//
// INT4 (orchard/quantizer.py:3-78): per 32-weight group, scale = fp16_rne(max|w| / 7)
// computed in fp32; a zero scale becomes fp16(1e-5) (subnormal 0x00A8);
// q = clip(int8(rint(w / scale + 8)), 0, 15) with every step correctly rounded in fp32
// (__fdiv_rn/__fadd_rn, so no contraction changes a bit); low nibble = even k.
// INT8 (src/main.cpp:35-64): scale = fp16_rne(max|w| / 127), zero -> 1.0,
// q = round-half-away(w / scale); group 32 or one group per output row.
#include "orch_common.cuh"

namespace orch {

template <typename T>
__device__ __forceinline__ void load32(const T* p, float (&v)[32]);

template <>
__device__ __forceinline__ void load32<float>(const float* p, float (&v)[32]) {
  const float4* q = reinterpret_cast<const float4*>(p);
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const float4 f = __ldg(q + i);
    v[4 * i] = f.x;
    v[4 * i + 1] = f.y;
    v[4 * i + 2] = f.z;
    v[4 * i + 3] = f.w;
  }
}

template <>
__device__ __forceinline__ void load32<__half>(const __half* p, float (&v)[32]) {
  const uint4* q = reinterpret_cast<const uint4*>(p);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const uint4 r = __ldg(q + i);
    const uint32_t w[4] = {r.x, r.y, r.z, r.w};
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 f = __half22float2(bits_h2(w[e]));
      v[8 * i + 2 * e] = f.x;
      v[8 * i + 2 * e + 1] = f.y;
    }
  }
}

template <typename T>
__global__ void quant_q4_kernel(const T* w, uint8_t* packed, __half* scales, size_t groups) {
  pdl_trigger();
  pdl_wait();
  for (size_t gi = blockIdx.x * (size_t)blockDim.x + threadIdx.x; gi < groups;
       gi += (size_t)gridDim.x * blockDim.x) {
    float v[32];
    load32<T>(w + gi * 32, v);
    float amax = 0.f;
#pragma unroll
    for (int i = 0; i < 32; ++i) amax = fmaxf(amax, fabsf(v[i]));
    __half sh = __float2half_rn(__fdiv_rn(amax, 7.0f));
    if (__half2float(sh) == 0.f) sh = __ushort_as_half((unsigned short)0x00A8u);
    const float s = __half2float(sh);
    uint32_t out[4] = {0, 0, 0, 0};
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      const float r = rintf(__fadd_rn(__fdiv_rn(v[i], s), 8.0f));
      int q = (int)(int8_t)(int)r;
      q = q < 0 ? 0 : (q > 15 ? 15 : q);
      out[i >> 3] |= (uint32_t)q << (4 * (i & 7));
    }
    reinterpret_cast<uint4*>(packed)[gi] = make_uint4(out[0], out[1], out[2], out[3]);
    scales[gi] = sh;
  }
}

// One group of `gs` consecutive weights per warp (gs = 32 or the row length).
template <typename T>
__global__ void quant_q8_kernel(const T* w, int8_t* q, __half* scales, size_t groups, int gs) {
  pdl_trigger();
  pdl_wait();
  const int lane = threadIdx.x & 31;
  const size_t warp = (blockIdx.x * (size_t)blockDim.x + threadIdx.x) >> 5;
  const size_t nwarps = ((size_t)gridDim.x * blockDim.x) >> 5;
  for (size_t gi = warp; gi < groups; gi += nwarps) {
    const T* src = w + gi * gs;
    float amax = 0.f;
    for (int i = lane; i < gs; i += 32) amax = fmaxf(amax, fabsf(to_f32(src[i])));
    amax = warp_max(amax);
    __half sh = __float2half_rn(__fdiv_rn(amax, 127.0f));
    if (__half2float(sh) == 0.f) sh = __float2half(1.0f);
    const float s = __half2float(sh);
    for (int i = lane; i < gs; i += 32) {
      float r = roundf(__fdiv_rn(to_f32(src[i]), s));
      r = fminf(127.f, fmaxf(-127.f, r));
      q[gi * gs + i] = (int8_t)(int)r;
    }
    if (lane == 0) scales[gi] = sh;
  }
}

static int qgrid(size_t work, int block) {
  size_t g = (work + block - 1) / block;
  const size_t cap = (size_t)num_sms() * 32;
  return (int)(g == 0 ? 1 : (g < cap ? g : cap));
}

}  // namespace orch

using namespace orch;

extern "C" int orch_quantize_q4_0(const void* w, int w_dt, void* packed, void* scales, uint32_t N,
                                  uint32_t K, void* stream) {
  if (N == 0 || K == 0) return ORCH_OK;
  ORCH_REQUIRE(w && packed && scales, "quantize_q4_0: null pointer");
  ORCH_REQUIRE(K % 32 == 0, "quantize_q4_0: K must be divisible by the group size 32");
  ORCH_REQUIRE(((uintptr_t)packed & 15) == 0 && ((uintptr_t)w & 15) == 0,
               "quantize_q4_0: buffers must be 16-byte aligned");
  const size_t groups = (size_t)N * (K / 32);
  cudaStream_t st = as_stream(stream);
  if (w_dt == ORCH_F32)
    ORCH_CUDA(launch_k(quant_q4_kernel<float>, dim3(qgrid(groups, 128)), dim3(128), 0, st, dim3(0, 0, 0), (const float*)w, (uint8_t*)packed,
                                                               (__half*)scales, groups));
  else if (w_dt == ORCH_F16)
    ORCH_CUDA(launch_k(quant_q4_kernel<__half>, dim3(qgrid(groups, 128)), dim3(128), 0, st, dim3(0, 0, 0), (const __half*)w, (uint8_t*)packed,
                                                                (__half*)scales, groups));
  else
    return fail(ORCH_ERR_INVALID, "quantize_q4_0: bad dtype");
  return check_launch("quantize_q4_0");
}

static int quant_q8(const void* w, int w_dt, void* q, void* scales, size_t groups, int gs, void* stream) {
  cudaStream_t st = as_stream(stream);
  const int g = qgrid(groups * 32, 256);
  if (w_dt == ORCH_F32)
    ORCH_CUDA(launch_k(quant_q8_kernel<float>, dim3(g), dim3(256), 0, st, dim3(0, 0, 0), (const float*)w, (int8_t*)q, (__half*)scales, groups, gs));
  else if (w_dt == ORCH_F16)
    ORCH_CUDA(launch_k(quant_q8_kernel<__half>, dim3(g), dim3(256), 0, st, dim3(0, 0, 0), (const __half*)w, (int8_t*)q, (__half*)scales, groups, gs));
  else
    return fail(ORCH_ERR_INVALID, "quantize_q8: bad dtype");
  return check_launch("quantize_q8");
}

extern "C" int orch_quantize_q8_0(const void* w, int w_dt, void* q, void* scales, uint32_t N, uint32_t K,
                                  void* stream) {
  if (N == 0 || K == 0) return ORCH_OK;
  ORCH_REQUIRE(w && q && scales, "quantize_q8_0: null pointer");
  ORCH_REQUIRE(K % 32 == 0, "quantize_q8_0: K must be divisible by 32");
  return quant_q8(w, w_dt, q, scales, (size_t)N * (K / 32), 32, stream);
}

extern "C" int orch_quantize_q8_pc(const void* w, int w_dt, void* q, void* scales, uint32_t N, uint32_t K,
                                   void* stream) {
  if (N == 0 || K == 0) return ORCH_OK;
  ORCH_REQUIRE(w && q && scales, "quantize_q8_pc: null pointer");
  return quant_q8(w, w_dt, q, scales, (size_t)N, (int)K, stream);
}
