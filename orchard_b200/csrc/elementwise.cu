// RMSNorm, RoPE, add/mul/SiLU, embedding gathers and the fp32/fp16 dense matmuls of the
// reference operator surface.
//
// Reference kernels: orchard/kernels/rmsnorm.metal:4-36 (one thread per row there; here
// one CTA per row with a warp-shuffle reduction), rope.metal:4-50 (interleaved pairs; here
// each row uses its own row of angles), elementwise.metal:4-30, embedding.metal:4-17,
// matmul.metal:4-23, matmul_simd.metal:4-40. All arithmetic is fp32; half tensors are
// converted on load and rounded once on store.
#include "orch_common.cuh"

namespace orch {

// ---- RMSNorm ---------------------------------------------------------------------------
template <typename TI, typename TW, typename TO>
__global__ void rmsnorm_kernel(const TI* in, const TW* w, TO* out, float eps, int N) {
  __shared__ float red[32];
  pdl_trigger();
  pdl_wait();
  const TI* r = in + (size_t)blockIdx.x * N;
  TO* o = out + (size_t)blockIdx.x * N;
  float ss = 0.f;
  for (int i = threadIdx.x; i < N; i += blockDim.x) {
    const float v = to_f32(r[i]);
    ss = fmaf(v, v, ss);
  }
  ss = block_sum(ss, red);
  const float inv = rsqrtf(ss / (float)N + eps);
  for (int i = threadIdx.x; i < N; i += blockDim.x) o[i] = from_f32<TO>(to_f32(r[i]) * inv * to_f32(w[i]));
}

// Vectorised form for N % 4 == 0, N <= 4 * V * blockDim.x: each thread holds its V
// four-element pieces of the row in registers, so the row is read once and every load is
// in flight at the same time (the generic loop above waits one memory latency per element
// it reads). The gamma pieces do not depend on the previous kernel and are requested first.
template <typename T> __device__ __forceinline__ float4 ld4(const T* p);
template <> __device__ __forceinline__ float4 ld4<float>(const float* p) {
  return *reinterpret_cast<const float4*>(p);
}
template <> __device__ __forceinline__ float4 ld4<__half>(const __half* p) {
  const uint2 u = *reinterpret_cast<const uint2*>(p);
  const float2 a = __half22float2(bits_h2(u.x)), b = __half22float2(bits_h2(u.y));
  return make_float4(a.x, a.y, b.x, b.y);
}
template <typename T> __device__ __forceinline__ void st4(T* p, float4 v);
template <> __device__ __forceinline__ void st4<float>(float* p, float4 v) { *reinterpret_cast<float4*>(p) = v; }
template <> __device__ __forceinline__ void st4<__half>(__half* p, float4 v) {
  uint2 u;
  u.x = h2_bits(__floats2half2_rn(v.x, v.y));
  u.y = h2_bits(__floats2half2_rn(v.z, v.w));
  *reinterpret_cast<uint2*>(p) = u;
}

template <typename TI, typename TW, typename TO, int V>
__global__ void rmsnorm_vec_kernel(const TI* in, const TW* w, TO* out, float eps, int N) {
  __shared__ float red[32];
  pdl_trigger();
  float4 g[V], v[V];
#pragma unroll
  for (int j = 0; j < V; ++j) {
    const int i = (j * blockDim.x + threadIdx.x) * 4;
    g[j] = i < N ? ld4(w + i) : make_float4(0.f, 0.f, 0.f, 0.f);
  }
  pdl_wait();
  const TI* r = in + (size_t)blockIdx.x * N;
  TO* o = out + (size_t)blockIdx.x * N;
#pragma unroll
  for (int j = 0; j < V; ++j) {
    const int i = (j * blockDim.x + threadIdx.x) * 4;
    v[j] = i < N ? ld4(r + i) : make_float4(0.f, 0.f, 0.f, 0.f);
  }
  float ss = 0.f;
#pragma unroll
  for (int j = 0; j < V; ++j) {
    ss = fmaf(v[j].x, v[j].x, ss);
    ss = fmaf(v[j].y, v[j].y, ss);
    ss = fmaf(v[j].z, v[j].z, ss);
    ss = fmaf(v[j].w, v[j].w, ss);
  }
  ss = block_sum(ss, red);
  const float inv = rsqrtf(ss / (float)N + eps);
#pragma unroll
  for (int j = 0; j < V; ++j) {
    const int i = (j * blockDim.x + threadIdx.x) * 4;
    if (i < N)
      st4(o + i, make_float4(v[j].x * inv * g[j].x, v[j].y * inv * g[j].y, v[j].z * inv * g[j].z,
                             v[j].w * inv * g[j].w));
  }
}

// ---- RoPE: in/out [rows, heads, hd], cos/sin [rows, hd/2] ---------------------------------
template <typename TI, typename TT, typename TO>
__global__ void rope_kernel(const TI* in, const TT* cs, const TT* sn, TO* out, int hd, int heads,
                            int rows) {
  pdl_trigger();
  pdl_wait();
  const int half = hd >> 1;
  const size_t total = (size_t)rows * heads * half;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
    const int pi = (int)(i % half);
    const size_t rh = i / half;
    const int row = (int)(rh / heads);
    const size_t b = rh * hd + 2 * pi;
    const float x0 = to_f32(in[b]), x1 = to_f32(in[b + 1]);
    const float c = to_f32(cs[(size_t)row * half + pi]), s = to_f32(sn[(size_t)row * half + pi]);
    const float o0 = x0 * c - x1 * s;
    const float o1 = x0 * s + x1 * c;
    out[b] = from_f32<TO>(o0);
    out[b + 1] = from_f32<TO>(o1);
  }
}

// ---- elementwise -------------------------------------------------------------------------
template <typename T, int OP>
__global__ void binary_kernel(const T* a, const T* b, T* c, size_t n) {
  pdl_trigger();
  pdl_wait();
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
    const float x = to_f32(a[i]), y = to_f32(b[i]);
    c[i] = from_f32<T>(OP == 0 ? x + y : x * y);
  }
}

template <typename T>
__global__ void silu_kernel(const T* in, T* out, size_t n) {
  pdl_trigger();
  pdl_wait();
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
    const float x = to_f32(in[i]);
    out[i] = from_f32<T>(x / (1.0f + expf(-x)));
  }
}

// ---- embedding gathers ---------------------------------------------------------------------
template <typename TW, typename TO>
__global__ void embedding_kernel(const int* ids, const TW* w, TO* out, int tokens, int hd, int vocab,
                                 uint32_t* check) {
  pdl_trigger();
  pdl_wait();
  const size_t total = (size_t)tokens * hd;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
    const int t = (int)(i / hd), d = (int)(i % hd);
    const int id = ids[t];
    if (id < 0 || id >= vocab) {
      out[i] = from_f32<TO>(0.f);
      if (d == 0) atomicOr(check, 4u);
      continue;
    }
    out[i] = from_f32<TO>(to_f32(w[(size_t)id * hd + d]));
  }
}

// ---- dense matmuls (surface): C[M,N] = A[M,K] B[K,N], 64x64 tiles, 4x4 per thread --------
template <typename T>
__global__ void __launch_bounds__(256) matmul_kernel(const T* A, const T* B, T* C, int M, int N, int K) {
  __shared__ float As[16][64 + 1];
  __shared__ float Bs[16][64 + 1];
  pdl_trigger();
  pdl_wait();
  const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
  const int m0 = blockIdx.y * 64, n0 = blockIdx.x * 64;
  float acc[4][4] = {};
  for (int k0 = 0; k0 < K; k0 += 16) {
    for (int i = threadIdx.x; i < 64 * 16; i += 256) {
      const int r = i / 16, kk = i % 16;  // A tile [64 rows][16 k]
      const int gm = m0 + r, gk = k0 + kk;
      As[kk][r] = (gm < M && gk < K) ? to_f32(A[(size_t)gm * K + gk]) : 0.f;
      const int kb = i / 64, cn = i % 64;  // B tile [16 k][64 cols]
      const int gk2 = k0 + kb, gn = n0 + cn;
      Bs[kb][cn] = (gk2 < K && gn < N) ? to_f32(B[(size_t)gk2 * N + gn]) : 0.f;
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < 16; ++kk) {
      float av[4], bv[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) av[i] = As[kk][ty * 4 + i];
#pragma unroll
      for (int j = 0; j < 4; ++j) bv[j] = Bs[kk][tx * 4 + j];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(av[i], bv[j], acc[i][j]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int gm = m0 + ty * 4 + i, gn = n0 + tx * 4 + j;
      if (gm < M && gn < N) C[(size_t)gm * N + gn] = from_f32<T>(acc[i][j]);
    }
}

static int grid_for(size_t n, int block) {
  const size_t g = (n + block - 1) / block;
  const size_t cap = (size_t)num_sms() * 16;
  return (int)(g < cap ? (g ? g : 1) : cap);
}

}  // namespace orch

using namespace orch;

#define DT_OK(dt) ((dt) == ORCH_F32 || (dt) == ORCH_F16)

extern "C" int orch_rmsnorm_ex(const void* in, int in_dt, const void* weight, int w_dt, void* out,
                               int out_dt, float eps, uint32_t N, uint32_t count, void* stream) {
  if (count == 0) return ORCH_OK;
  ORCH_REQUIRE(in && weight && out && N > 0, "rmsnorm: bad arguments");
  ORCH_REQUIRE(DT_OK(in_dt) && DT_OK(w_dt) && DT_OK(out_dt), "rmsnorm: bad dtype");
  cudaStream_t st = as_stream(stream);
  const int th = N >= 1024 ? 256 : 128;
  // vector path: 16-byte (fp32) / 8-byte (fp16) aligned rows of at most 4 * 8 * 256 elements
  const bool vec = (N % 4) == 0 && N <= 8192 && ((uintptr_t)in & 15) == 0 && ((uintptr_t)weight & 15) == 0 &&
                   ((uintptr_t)out & 15) == 0;
  const bool v4 = N <= 4096;
#define RMS_CASE(TI, TW, TO)                                                                                     \
  if (vec && v4)                                                                                                 \
    ORCH_CUDA(launch_k(rmsnorm_vec_kernel<TI, TW, TO, 4>, dim3(count), dim3(256), 0, st, dim3(0, 0, 0),          \
                       (const TI*)in, (const TW*)weight, (TO*)out, eps, (int)N));                                 \
  else if (vec)                                                                                                  \
    ORCH_CUDA(launch_k(rmsnorm_vec_kernel<TI, TW, TO, 8>, dim3(count), dim3(256), 0, st, dim3(0, 0, 0),          \
                       (const TI*)in, (const TW*)weight, (TO*)out, eps, (int)N));                                 \
  else                                                                                                           \
    ORCH_CUDA(launch_k(rmsnorm_kernel<TI, TW, TO>, dim3(count), dim3(th), 0, st, dim3(0, 0, 0), (const TI*)in,   \
                       (const TW*)weight, (TO*)out, eps, (int)N))
  const int key = in_dt * 4 + w_dt * 2 + out_dt;
  switch (key) {
    case 0: RMS_CASE(float, float, float); break;
    case 1: RMS_CASE(float, float, __half); break;
    case 2: RMS_CASE(float, __half, float); break;
    case 3: RMS_CASE(float, __half, __half); break;
    case 4: RMS_CASE(__half, float, float); break;
    case 5: RMS_CASE(__half, float, __half); break;
    case 6: RMS_CASE(__half, __half, float); break;
    default: RMS_CASE(__half, __half, __half); break;
  }
#undef RMS_CASE
  return check_launch("rmsnorm");
}

extern "C" int orch_rmsnorm(const void* in, const void* weight, void* out, float eps, uint32_t N,
                            uint32_t count, void* stream) {
  return orch_rmsnorm_ex(in, ORCH_F16, weight, ORCH_F16, out, ORCH_F16, eps, N, count, stream);
}

extern "C" int orch_rope_ex(const void* in, int in_dt, const void* cs, const void* sn, int tab_dt,
                            void* out, int out_dt, uint32_t head_dim, uint32_t num_heads,
                            uint32_t seq_len, void* stream) {
  if (seq_len == 0 || num_heads == 0) return ORCH_OK;
  ORCH_REQUIRE(in && cs && sn && out, "rope: null pointer");
  ORCH_REQUIRE(head_dim >= 2 && head_dim % 2 == 0, "rope: head_dim must be even");
  ORCH_REQUIRE(DT_OK(in_dt) && DT_OK(tab_dt) && DT_OK(out_dt), "rope: bad dtype");
  cudaStream_t st = as_stream(stream);
  const size_t n = (size_t)seq_len * num_heads * (head_dim / 2);
  const int g = grid_for(n, 256);
#define ROPE_CASE(TI, TT, TO)                                                                 \
  ORCH_CUDA(launch_k(rope_kernel<TI, TT, TO>, dim3(g), dim3(256), 0, st, dim3(0, 0, 0), (const TI*)in, \
                     (const TT*)cs, (const TT*)sn, (TO*)out, (int)head_dim, (int)num_heads, (int)seq_len))
  const int key = in_dt * 4 + tab_dt * 2 + out_dt;
  switch (key) {
    case 0: ROPE_CASE(float, float, float); break;
    case 1: ROPE_CASE(float, float, __half); break;
    case 2: ROPE_CASE(float, __half, float); break;
    case 3: ROPE_CASE(float, __half, __half); break;
    case 4: ROPE_CASE(__half, float, float); break;
    case 5: ROPE_CASE(__half, float, __half); break;
    case 6: ROPE_CASE(__half, __half, float); break;
    default: ROPE_CASE(__half, __half, __half); break;
  }
#undef ROPE_CASE
  return check_launch("rope");
}

extern "C" int orch_rope(const void* in, const void* cs, const void* sn, void* out, uint32_t head_dim,
                         uint32_t num_heads, uint32_t seq_len, void* stream) {
  return orch_rope_ex(in, ORCH_F16, cs, sn, ORCH_F16, out, ORCH_F16, head_dim, num_heads, seq_len, stream);
}

extern "C" int orch_binary_ex(int op, const void* a, const void* b, void* c, int dt, uint32_t size,
                              void* stream) {
  if (size == 0) return ORCH_OK;
  ORCH_REQUIRE(a && b && c, "binary: null pointer");
  ORCH_REQUIRE(op == 0 || op == 1, "binary: op must be 0 (add) or 1 (mul)");
  ORCH_REQUIRE(DT_OK(dt), "binary: bad dtype");
  cudaStream_t st = as_stream(stream);
  const int g = grid_for(size, 256);
  if (dt == ORCH_F16) {
    if (op == 0) ORCH_CUDA(launch_k(binary_kernel<__half, 0>, dim3(g), dim3(256), 0, st, dim3(0, 0, 0), (const __half*)a, (const __half*)b, (__half*)c, (size_t)size));
    else ORCH_CUDA(launch_k(binary_kernel<__half, 1>, dim3(g), dim3(256), 0, st, dim3(0, 0, 0), (const __half*)a, (const __half*)b, (__half*)c, (size_t)size));
  } else {
    if (op == 0) ORCH_CUDA(launch_k(binary_kernel<float, 0>, dim3(g), dim3(256), 0, st, dim3(0, 0, 0), (const float*)a, (const float*)b, (float*)c, (size_t)size));
    else ORCH_CUDA(launch_k(binary_kernel<float, 1>, dim3(g), dim3(256), 0, st, dim3(0, 0, 0), (const float*)a, (const float*)b, (float*)c, (size_t)size));
  }
  return check_launch("binary");
}

extern "C" int orch_add(const void* a, const void* b, void* c, uint32_t size, void* stream) {
  return orch_binary_ex(0, a, b, c, ORCH_F16, size, stream);
}
extern "C" int orch_mul(const void* a, const void* b, void* c, uint32_t size, void* stream) {
  return orch_binary_ex(1, a, b, c, ORCH_F16, size, stream);
}

extern "C" int orch_silu_ex(const void* in, void* out, int dt, uint32_t size, void* stream) {
  if (size == 0) return ORCH_OK;
  ORCH_REQUIRE(in && out, "silu: null pointer");
  ORCH_REQUIRE(DT_OK(dt), "silu: bad dtype");
  cudaStream_t st = as_stream(stream);
  const int g = grid_for(size, 256);
  if (dt == ORCH_F16) ORCH_CUDA(launch_k(silu_kernel<__half>, dim3(g), dim3(256), 0, st, dim3(0, 0, 0), (const __half*)in, (__half*)out, (size_t)size));
  else ORCH_CUDA(launch_k(silu_kernel<float>, dim3(g), dim3(256), 0, st, dim3(0, 0, 0), (const float*)in, (float*)out, (size_t)size));
  return check_launch("silu");
}
extern "C" int orch_silu(const void* in, void* out, uint32_t size, void* stream) {
  return orch_silu_ex(in, out, ORCH_F16, size, stream);
}

extern "C" int orch_embedding_ex(const void* ids, const void* weights, int w_dt, void* out, int out_dt,
                                 uint32_t num_tokens, uint32_t hidden_dim, uint32_t vocab, void* stream) {
  if (num_tokens == 0 || hidden_dim == 0) return ORCH_OK;
  ORCH_REQUIRE(ids && weights && out, "embedding: null pointer");
  ORCH_REQUIRE(vocab > 0, "embedding: vocab must be positive");
  ORCH_REQUIRE(DT_OK(w_dt) && DT_OK(out_dt), "embedding: bad dtype");
  cudaStream_t st = as_stream(stream);
  const size_t n = (size_t)num_tokens * hidden_dim;
  const int g = grid_for(n, 256);
  uint32_t* chk = device_check_word();
  const int* id = (const int*)ids;
  if (w_dt == ORCH_F16 && out_dt == ORCH_F16)
    ORCH_CUDA(launch_k(embedding_kernel<__half, __half>, dim3(g), dim3(256), 0, st, dim3(0, 0, 0), id, (const __half*)weights, (__half*)out, (int)num_tokens, (int)hidden_dim, (int)vocab, chk));
  else if (w_dt == ORCH_F16)
    ORCH_CUDA(launch_k(embedding_kernel<__half, float>, dim3(g), dim3(256), 0, st, dim3(0, 0, 0), id, (const __half*)weights, (float*)out, (int)num_tokens, (int)hidden_dim, (int)vocab, chk));
  else if (out_dt == ORCH_F16)
    ORCH_CUDA(launch_k(embedding_kernel<float, __half>, dim3(g), dim3(256), 0, st, dim3(0, 0, 0), id, (const float*)weights, (__half*)out, (int)num_tokens, (int)hidden_dim, (int)vocab, chk));
  else
    ORCH_CUDA(launch_k(embedding_kernel<float, float>, dim3(g), dim3(256), 0, st, dim3(0, 0, 0), id, (const float*)weights, (float*)out, (int)num_tokens, (int)hidden_dim, (int)vocab, chk));
  return check_launch("embedding");
}

extern "C" int orch_embedding(const void* ids, const void* weights, void* out, uint32_t num_tokens,
                              uint32_t hidden_dim, uint32_t vocab, void* stream) {
  return orch_embedding_ex(ids, weights, ORCH_F16, out, ORCH_F16, num_tokens, hidden_dim, vocab, stream);
}

extern "C" int orch_embed_rows(const int32_t* ids, const void* table, int table_dt, float* x, uint32_t M,
                               uint32_t H, uint32_t V, void* stream) {
  return orch_embedding_ex(ids, table, table_dt, x, ORCH_F32, M, H, V, stream);
}

extern "C" int orch_matmul(const float* a, const float* b, float* c, uint32_t M, uint32_t N, uint32_t K,
                           void* stream) {
  if (M == 0 || N == 0) return ORCH_OK;
  ORCH_REQUIRE(a && b && c, "matmul: null pointer");
  dim3 grid((N + 63) / 64, (M + 63) / 64);
  ORCH_CUDA(launch_k(matmul_kernel<float>, grid, dim3(256), 0, as_stream(stream), dim3(0, 0, 0), a, b, c, (int)M,
                     (int)N, (int)K));
  return check_launch("matmul");
}

extern "C" int orch_matmul_simd(const void* a, const void* b, void* c, uint32_t M, uint32_t N, uint32_t K,
                                void* stream) {
  if (M == 0 || N == 0) return ORCH_OK;
  ORCH_REQUIRE(a && b && c, "matmul_simd: null pointer");
  dim3 grid((N + 63) / 64, (M + 63) / 64);
  ORCH_CUDA(launch_k(matmul_kernel<__half>, grid, dim3(256), 0, as_stream(stream), dim3(0, 0, 0), (const __half*)a,
                     (const __half*)b, (__half*)c, (int)M, (int)N, (int)K));
  return check_launch("matmul_simd");
}

// ---- LoRA down-projection t[m, :] = x[m, :] . A   (x fp16 [M,K], A fp32 [K,R]) -------------
namespace orch {
__global__ void __launch_bounds__(256) lora_xa_kernel(const __half* x, const float* A, float* t, int K, int R) {
  __shared__ float part[8][33];
  pdl_trigger();
  pdl_wait();
  const int m = blockIdx.x;
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
  const __half* xr = x + (size_t)m * K;
  for (int j0 = 0; j0 < R; j0 += 32) {
    const int j = j0 + tx;
    float acc = 0.f;
    if (j < R)
      for (int k = ty; k < K; k += 8) acc = fmaf(__half2float(xr[k]), A[(size_t)k * R + j], acc);
    part[ty][tx] = acc;
    __syncthreads();
    if (ty == 0 && j < R) {
      float s = 0.f;
#pragma unroll
      for (int i = 0; i < 8; ++i) s += part[i][tx];
      t[(size_t)m * R + j] = s;
    }
    __syncthreads();
  }
}

// x.A for many rows (prefill): a CTA takes 32 rows and all R <= 64 columns, staging 64-k
// chunks of x (as fp32) and A in shared memory, so A is read once per 32 rows instead of once
// per row; the next chunk's loads are in flight (in registers) while the current one is
// multiplied. Thread (row, column group g) accumulates columns g, g + 8, ..., in fp32 over k
// in increasing order.
constexpr int kXaRows = 32, kXaK = 64, kXaCols = 64;
constexpr int kXaXPer = kXaRows * kXaK / 256, kXaAPer = kXaK * kXaCols / 256;  // loads per thread
__global__ void __launch_bounds__(256) lora_xa_tiled_kernel(const __half* x, const float* A, float* t, int M, int K,
                                                           int R) {
  __shared__ float xs[kXaRows][kXaK + 1];
  __shared__ float as[kXaK][kXaCols];
  pdl_trigger();
  pdl_wait();
  const int m0 = blockIdx.x * kXaRows;
  const int tid = threadIdx.x, row = tid >> 3, cgp = tid & 7;
  float xr[kXaXPer], ar[kXaAPer];
  auto gload = [&](int k0) {
#pragma unroll
    for (int u = 0; u < kXaXPer; ++u) {
      const int i = tid + 256 * u, r = i / kXaK, k = k0 + (i - r * kXaK), m = m0 + r;
      xr[u] = (m < M && k < K) ? __half2float(x[(size_t)m * K + k]) : 0.f;
    }
#pragma unroll
    for (int u = 0; u < kXaAPer; ++u) {
      const int i = tid + 256 * u, kk = i / kXaCols, j = i - kk * kXaCols, k = k0 + kk;
      ar[u] = (k < K && j < R) ? A[(size_t)k * R + j] : 0.f;
    }
  };
  float acc[kXaCols / 8];
#pragma unroll
  for (int i = 0; i < kXaCols / 8; ++i) acc[i] = 0.f;
  gload(0);
  for (int k0 = 0; k0 < K; k0 += kXaK) {
#pragma unroll
    for (int u = 0; u < kXaXPer; ++u) {
      const int i = tid + 256 * u, r = i / kXaK;
      xs[r][i - r * kXaK] = xr[u];
    }
#pragma unroll
    for (int u = 0; u < kXaAPer; ++u) {
      const int i = tid + 256 * u, kk = i / kXaCols;
      as[kk][i - kk * kXaCols] = ar[u];
    }
    __syncthreads();
    if (k0 + kXaK < K) gload(k0 + kXaK);
#pragma unroll 8
    for (int kk = 0; kk < kXaK; ++kk) {
      const float xv = xs[row][kk];
#pragma unroll
      for (int i = 0; i < kXaCols / 8; ++i) acc[i] = fmaf(xv, as[kk][cgp + 8 * i], acc[i]);
    }
    __syncthreads();
  }
  const int m = m0 + row;
#pragma unroll
  for (int i = 0; i < kXaCols / 8; ++i) {
    const int j = cgp + 8 * i;
    if (m < M && j < R) t[(size_t)m * R + j] = acc[i];
  }
}
}  // namespace orch

extern "C" int orch_lora_xa(const void* x, const float* a, float* t, uint32_t M, uint32_t K, uint32_t R,
                            void* stream) {
  if (M == 0 || R == 0) return ORCH_OK;
  ORCH_REQUIRE(x && a && t && K > 0, "lora_xa: bad arguments");
  if (M >= 256 && R <= (uint32_t)orch::kXaCols)  // many rows: A staged once per 32 rows
    ORCH_CUDA(orch::launch_k(orch::lora_xa_tiled_kernel, dim3((M + orch::kXaRows - 1) / orch::kXaRows), dim3(256), 0,
                             as_stream(stream), dim3(0, 0, 0), (const __half*)x, a, t, (int)M, (int)K, (int)R));
  else
    ORCH_CUDA(orch::launch_k(orch::lora_xa_kernel, dim3(M), dim3(256), 0, as_stream(stream), dim3(0, 0, 0),
                             (const __half*)x, a, t, (int)K, (int)R));
  return check_launch("lora_xa");
}
