// On-device packers, bit-identical to the host rules.
//
// INT4 (orchard/quantizer.py:3-78): per 32-weight group, scale = fp16_rne(max|w| / 7)
// computed in fp32; a zero scale becomes fp16(1e-5) (subnormal 0x00A8);
// q = clip(int8(rint(w / scale + 8)), 0, 15) with every step correctly rounded in fp32
// (__fdiv_rn/__fadd_rn, so no contraction changes a bit); low nibble = even k.
// INT8 (src/main.cpp:35-64): scale = fp16_rne(max|w| / 127), zero -> 1.0,
// q = round-half-away(w / scale); group 32 or one group per output row.
#include "qgemm.cuh"

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
  // No early griddepcontrol.launch_dependents here: the GEMMs start streaming weights
  // before their own griddepcontrol.wait, so a packer releases dependents only on exit.
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
  pdl_wait();  // releases dependents only on exit (see quant_q4_kernel)
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

// Standard packed INT4 -> tiled layout (qgemm.cuh). One thread per (tile, block, row):
// the row's 128 packed bytes of the block (8 x 16) and its 8 scales.
__device__ __forceinline__ uint32_t q4t_word(uint32_t w) {
  // nibble p of the result is nibble {0,2,4,6,1,3,5,7}[p] of w
  uint32_t o = 0;
#pragma unroll
  for (int p = 0; p < 8; ++p) {
    const int q = (p < 4) ? 2 * p : 2 * (p - 4) + 1;
    o |= ((w >> (4 * q)) & 0xFu) << (4 * p);
  }
  return o;
}

__global__ void q4t_pack_kernel(const uint8_t* __restrict__ w, const __half* __restrict__ sc, uint8_t* __restrict__ out,
                                int N, int K, int nblk, size_t units) {
  pdl_wait();
  const int G = K / 32;
  for (size_t u = blockIdx.x * (size_t)blockDim.x + threadIdx.x; u < units; u += (size_t)gridDim.x * blockDim.x) {
    const int r = (int)(u % kQ4tRows);
    const size_t tb = u / kQ4tRows;  // tile * nblk + block
    const int b = (int)(tb % nblk);
    const int row = (int)(tb / nblk) * kQ4tRows + r;
    uint8_t* blk = out + tb * kQ4tBlockBytes;
#pragma unroll 1
    for (int j = 0; j < 8; ++j) {  // 32-k halves of the block: stage j/2, half j%2
      const int g = b * 8 + j;      // scale group
      uint4 v = make_uint4(0x88888888u, 0x88888888u, 0x88888888u, 0x88888888u);
      __half s = __float2half(0.f);
      if (row < N && g < G) {
        v = *reinterpret_cast<const uint4*>(w + (size_t)row * (K / 2) + (size_t)g * 16);
        s = sc[(size_t)row * G + g];
        v.x = q4t_word(v.x);
        v.y = q4t_word(v.y);
        v.z = q4t_word(v.z);
        v.w = q4t_word(v.w);
      }
      *reinterpret_cast<uint4*>(blk + (j >> 1) * kQ4tStageBytes + (j & 1) * 2048 + r * 16) = v;
      reinterpret_cast<__half*>(blk + 4 * kQ4tStageBytes)[j * kQ4tRows + r] = s;
    }
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

extern "C" size_t orch_q4t_bytes(uint32_t N, uint32_t K) { return (N == 0 || K == 0) ? 0 : q4t_bytes(N, K); }

extern "C" int orch_q4t_pack(const void* packed, const void* scales, uint32_t N, uint32_t K, void* tiled,
                             void* stream) {
  if (N == 0 || K == 0) return ORCH_OK;
  ORCH_REQUIRE(packed && scales && tiled, "q4t_pack: null pointer");
  ORCH_REQUIRE(K % 32 == 0, "q4t_pack: K must be divisible by the group size 32");
  ORCH_REQUIRE(((uintptr_t)packed & 15) == 0 && ((uintptr_t)tiled & 15) == 0,
               "q4t_pack: buffers must be 16-byte aligned");
  const int nblk = (int)((K + kQ4tBlockK - 1) / kQ4tBlockK);
  const size_t units = (size_t)((N + kQ4tRows - 1) / kQ4tRows) * nblk * kQ4tRows;
  ORCH_CUDA(launch_k(q4t_pack_kernel, dim3(qgrid(units, 128)), dim3(128), 0, as_stream(stream), dim3(0, 0, 0),
                     (const uint8_t*)packed, (const __half*)scales, (uint8_t*)tiled, (int)N, (int)K, nblk, units));
  return check_launch("q4t_pack");
}
