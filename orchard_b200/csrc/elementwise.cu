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

// SwiGLU in one pass: out = silu(g) * u in fp32, rounded once (the fused gate/up epilogue's
// arithmetic; the reference runs silu_fp16 then mul_fp16, elementwise.metal:13-30).
template <typename T>
__global__ void swiglu_kernel(const T* g, const T* u, T* out, size_t n) {
  pdl_trigger();
  pdl_wait();
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
    const float x = to_f32(g[i]);
    out[i] = from_f32<T>(x / (1.0f + expf(-x)) * to_f32(u[i]));
  }
}
// fp16 with 16-byte accesses: eight elements of g and u per thread and step.
__global__ void swiglu_h8_kernel(const uint4* g, const uint4* u, uint4* out, size_t n8) {
  pdl_trigger();
  pdl_wait();
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n8; i += (size_t)gridDim.x * blockDim.x) {
    const uint4 a = ld_stream16(g + i), b = ld_stream16(u + i);
    const uint32_t aw[4] = {a.x, a.y, a.z, a.w}, bw[4] = {b.x, b.y, b.z, b.w};
    uint32_t o[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 x = __half22float2(bits_h2(aw[j])), y = __half22float2(bits_h2(bw[j]));
      o[j] = h2_bits(__floats2half2_rn(x.x / (1.0f + expf(-x.x)) * y.x, x.y / (1.0f + expf(-x.y)) * y.y));
    }
    out[i] = make_uint4(o[0], o[1], o[2], o[3]);
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

extern "C" int orch_swiglu_ex(const void* gate, const void* up, void* out, int dt, uint32_t size, void* stream) {
  if (size == 0) return ORCH_OK;
  ORCH_REQUIRE(gate && up && out, "swiglu: null pointer");
  ORCH_REQUIRE(DT_OK(dt), "swiglu: bad dtype");
  cudaStream_t st = as_stream(stream);
  const bool vec = dt == ORCH_F16 && size % 8 == 0 &&
                   (((uintptr_t)gate | (uintptr_t)up | (uintptr_t)out) & 15) == 0;
  if (vec) {
    const size_t n8 = size / 8;
    ORCH_CUDA(launch_k(swiglu_h8_kernel, dim3(grid_for(n8, 256)), dim3(256), 0, st, dim3(0, 0, 0),
                       (const uint4*)gate, (const uint4*)up, (uint4*)out, n8));
  } else if (dt == ORCH_F16) {
    ORCH_CUDA(launch_k(swiglu_kernel<__half>, dim3(grid_for(size, 256)), dim3(256), 0, st, dim3(0, 0, 0),
                       (const __half*)gate, (const __half*)up, (__half*)out, (size_t)size));
  } else {
    ORCH_CUDA(launch_k(swiglu_kernel<float>, dim3(grid_for(size, 256)), dim3(256), 0, st, dim3(0, 0, 0),
                       (const float*)gate, (const float*)up, (float*)out, (size_t)size));
  }
  return check_launch("swiglu");
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
  uint32_t* chk = nullptr;
  ORCH_CHECK_WORD(chk);
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

// x.A for many rows (prefill) on the tensor cores: mma.sync m16n8k8 with TF32 operands.
// x is fp16, exact in TF32; A (fp32) is split into two TF32 terms, big = round(A) and
// small = round(A - big), so x.A = x.big + x.small keeps ~22 bits of A with fp32's exponent
// range. The tensor core adds its products into the accumulator with less care than an fp32
// add (K = 4096 in one accumulator drifted 2e-5 of max|t|), so every 16 k start a fresh
// accumulator that is added into the running fp32 sums with a plain (round-to-nearest) add.
// A CTA takes 32 rows and NC >= R columns; its 8 warps are 2 row groups of 16 x 4 quarters
// of each 64-k chunk, the quarters summed in a fixed order at the end. x and A chunks stream
// through a 6-stage cp.async ring (5 chunks in flight while one is multiplied).
constexpr int kXaRows = 32, kXaK = 64, kXaStages = 6, kXaThreads = 256;
constexpr int kXaXP = kXaK + 8;  // x pitch (halves): 144-B rows, A fragments hit bank 4g + c/2
template <int NC>
struct XaCfg {
  static constexpr int AP = NC + 8;  // A pitch (floats): B fragments (k = c, n = g) hit bank 8c + g
  static constexpr int XBytes = kXaRows * kXaXP * 2, ABytes = kXaK * AP * 4;
  static constexpr int Smem = kXaStages * (XBytes + ABytes);
};

__device__ __forceinline__ void xa_cp16(void* dst, const void* src, bool ok) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(static_cast<uint32_t>(__cvta_generic_to_shared(dst))),
               "l"(src), "r"(ok ? 16 : 0)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit_xa() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait_xa() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// Requires K % 8 == 0, R % 4 == 0, R <= NC, x and A 16-byte aligned (whole 16-B copies).
template <int NC>
__global__ void __launch_bounds__(kXaThreads) lora_xa_tiled_kernel(const __half* x, const float* A, float* t, int M,
                                                                  int K, int R) {
  using C = XaCfg<NC>;
  extern __shared__ __align__(16) uint8_t xa_smem[];
  auto xs = reinterpret_cast<__half(*)[kXaRows][kXaXP]>(xa_smem);                       // [stage][row][k]
  auto as = reinterpret_cast<float(*)[kXaK][C::AP]>(xa_smem + kXaStages * C::XBytes);  // [stage][k][col]
  pdl_trigger();
  pdl_wait();
  const int m0 = blockIdx.x * kXaRows;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 2, c = lane & 3;
  const int rg = warp & 1, kq = warp >> 1;
  const int nchunks = (K + kXaK - 1) / kXaK;
  auto issue = [&](int ch) {
    const int st = ch % kXaStages, k0 = ch * kXaK;
    {  // x: 32 rows x 8 pieces of 8 k, one copy per thread
      const int r = tid >> 3, q = tid & 7, m = m0 + r, k = k0 + 8 * q;
      const bool ok = m < M && k < K;
      xa_cp16(&xs[st][r][8 * q], ok ? x + (size_t)m * K + k : x, ok);
    }
    constexpr int kSeg = NC / 4;  // 16-B pieces of an A row
#pragma unroll
    for (int i = tid; i < kXaK * kSeg; i += kXaThreads) {
      const int kk = i / kSeg, j = 4 * (i - kk * kSeg), k = k0 + kk;
      const bool ok = k < K && j < R;
      xa_cp16(&as[st][kk][j], ok ? A + (size_t)k * R + j : A, ok);
    }
  };
#pragma unroll
  for (int s = 0; s < kXaStages - 1; ++s) {
    if (s < nchunks) issue(s);
    cp_async_commit_xa();
  }
  float tot[NC / 8][4];
#pragma unroll
  for (int nt = 0; nt < NC / 8; ++nt) tot[nt][0] = tot[nt][1] = tot[nt][2] = tot[nt][3] = 0.f;
  const int r0 = 16 * rg + g;
  for (int ch = 0; ch < nchunks; ++ch) {
    cp_async_wait_xa<kXaStages - 2>();  // this thread's copies of chunk ch have landed
    __syncthreads();                    // everyone's; and chunk ch - 1's stage is free again
    if (ch + kXaStages - 1 < nchunks) issue(ch + kXaStages - 1);
    cp_async_commit_xa();  // empty groups keep the count uniform
    const int st = ch % kXaStages;
    uint32_t af[2][4];  // this warp's two 8-k steps of the chunk
#pragma unroll
    for (int q = 0; q < 2; ++q) {
      const int kb = 8 * (2 * kq + q);
      af[q][0] = __float_as_uint(__half2float(xs[st][r0][kb + c]));
      af[q][1] = __float_as_uint(__half2float(xs[st][r0 + 8][kb + c]));
      af[q][2] = __float_as_uint(__half2float(xs[st][r0][kb + c + 4]));
      af[q][3] = __float_as_uint(__half2float(xs[st][r0 + 8][kb + c + 4]));
    }
#pragma unroll
    for (int nt = 0; nt < NC / 8; ++nt) {
      float d[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int q = 0; q < 2; ++q) {
        const int kb = 8 * (2 * kq + q);
        const float v0 = as[st][kb + c][8 * nt + g], v1 = as[st][kb + c + 4][8 * nt + g];
        const uint32_t b0 = to_tf32(v0), b1 = to_tf32(v1);
        mma_tf32(d, af[q], b0, b1);
        mma_tf32(d, af[q], to_tf32(v0 - __uint_as_float(b0)), to_tf32(v1 - __uint_as_float(b1)));
      }
#pragma unroll
      for (int e = 0; e < 4; ++e) tot[nt][e] += d[e];
    }
  }
  cp_async_wait_xa<0>();
  __syncthreads();  // all fragment reads done: the A ring is reused for the quarters' sums
  float* red = reinterpret_cast<float*>(as);  // [quarter 1..3][row group][nt][e][lane]
  auto ridx = [&](int qq, int nt, int e) { return ((((qq - 1) * 2 + rg) * (NC / 8) + nt) * 4 + e) * 32 + lane; };
  if (kq > 0) {
#pragma unroll
    for (int nt = 0; nt < NC / 8; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) red[ridx(kq, nt, e)] = tot[nt][e];
  }
  __syncthreads();
  if (kq > 0) return;
#pragma unroll
  for (int nt = 0; nt < NC / 8; ++nt)
#pragma unroll
    for (int e = 0; e < 4; ++e) tot[nt][e] = ((tot[nt][e] + red[ridx(1, nt, e)]) + red[ridx(2, nt, e)]) + red[ridx(3, nt, e)];
  // C fragment: (row g, cols 2c, 2c + 1) and (row g + 8, same cols) of each 8-column tile
  const int ra = m0 + r0, rb = ra + 8;
#pragma unroll
  for (int nt = 0; nt < NC / 8; ++nt)
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const int j = 8 * nt + 2 * c + e;
      if (j < R) {
        if (ra < M) t[(size_t)ra * R + j] = tot[nt][e];
        if (rb < M) t[(size_t)rb * R + j] = tot[nt][2 + e];
      }
    }
}
}  // namespace orch

extern "C" int orch_lora_xa(const void* x, const float* a, float* t, uint32_t M, uint32_t K, uint32_t R,
                            void* stream) {
  if (M == 0 || R == 0) return ORCH_OK;
  ORCH_REQUIRE(x && a && t && K > 0, "lora_xa: bad arguments");
  const bool tiled = M >= 256 && R <= 64 && R % 4 == 0 && K % 8 == 0 && ((uintptr_t)x & 15) == 0 &&
                     ((uintptr_t)a & 15) == 0;  // many rows, whole 16-B copies
  if (tiled) {
    static bool attr_done[64] = {};
    const int dev = device_index();
    if (dev >= 0 && dev < 64 && !attr_done[dev]) {
      ORCH_CUDA(cudaFuncSetAttribute(orch::lora_xa_tiled_kernel<32>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     orch::XaCfg<32>::Smem));
      ORCH_CUDA(cudaFuncSetAttribute(orch::lora_xa_tiled_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     orch::XaCfg<64>::Smem));
      attr_done[dev] = true;
    }
    const dim3 grid((M + orch::kXaRows - 1) / orch::kXaRows);
    if (R <= 32)
      ORCH_CUDA(orch::launch_k(orch::lora_xa_tiled_kernel<32>, grid, dim3(orch::kXaThreads), orch::XaCfg<32>::Smem,
                               as_stream(stream), dim3(0, 0, 0), (const __half*)x, a, t, (int)M, (int)K, (int)R));
    else
      ORCH_CUDA(orch::launch_k(orch::lora_xa_tiled_kernel<64>, grid, dim3(orch::kXaThreads), orch::XaCfg<64>::Smem,
                               as_stream(stream), dim3(0, 0, 0), (const __half*)x, a, t, (int)M, (int)K, (int)R));
  } else {
    ORCH_CUDA(orch::launch_k(orch::lora_xa_kernel, dim3(M), dim3(256), 0, as_stream(stream), dim3(0, 0, 0),
                             (const __half*)x, a, t, (int)K, (int)R));
  }
  return check_launch("lora_xa");
}
