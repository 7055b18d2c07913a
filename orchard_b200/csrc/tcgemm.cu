// INT4 dequant GEMM on the 5th-generation tensor cores (tcgen05 + TMEM), for M >= 16
// activation rows: batched decode (M = 16..256) and prefill (M = thousands of tokens).
//
// Replaces the reference's batched kernel (orchard/kernels/gemm_int4.metal:10-68, one
// thread per output, weights re-read per row) for the same packed format
// (orchard/quantizer.py:3-78).
//
// D[128 weight rows, NT tokens] (fp32, TMEM) += A[128, 16] . B[NT, 16]^T per MMA, with
//  * A = dequantised weights: thread t of the CTA owns weight row R0 + t, streams its
//    packed nibbles (32 bytes per 64-k stage, four stages ahead in registers), turns them
//    into fp16 (q - 8) * scale with the magic-exponent trick and stores them into a
//    128B-swizzled K-major shared-memory tile (the canonical UMMA layout);
//  * B = activations [tokens, K] fp16, loaded by TMA (SWIZZLE_128B; rows past M and k
//    past K read as zero) into a four-stage ring guarded by mbarriers;
//  * one thread issues tcgen05.mma.kind::f16 and tcgen05.commit releases each stage.
// After the K loop the accumulator is read with tcgen05.ld into a shared-memory partial
// tile and handed to the same split-K (cluster / distributed shared memory) reduction and
// fused epilogues as the mma.sync kernel (qgemm.cuh). TMA loads never use multicast.
//
// Every mbarrier wait is bounded (~2 s of globaltimer); on expiry the CTA records
// ORCH device check bit 8, stops issuing, drains what it issued and frees its TMEM.
#include <cuda.h>

#include <algorithm>
#include <cstdlib>

#include "qgemm.cuh"

namespace orch {

constexpr int kTcThreads = 128;
constexpr int kTcRows = 128;
constexpr int kTcBK = 64;  // k per stage: one 128-byte swizzle row of fp16
constexpr int kTcStages = 4;
constexpr int kTcABytes = kTcRows * kTcBK * 2;  // 16 KB
constexpr unsigned long long kWaitNs = 2000000000ull;

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ unsigned long long gtimer() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ bool mbar_try(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded wait for the phase of `parity` to complete.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
  if (mbar_try(bar, parity)) return true;
  const unsigned long long t0 = gtimer();
  while (!mbar_try(bar, parity)) {
    if (gtimer() - t0 > kWaitNs) return false;
  }
  return true;
}
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(
          smem_u32(dst)),
      "l"(map), "r"(smem_u32(bar)), "r"(x), "r"(y)
      : "memory");
}
__device__ __forceinline__ void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void tmem_alloc(uint32_t* dst, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst)), "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void umma_f16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                         uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr)
      : "memory");
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// Shared-memory matrix descriptor: K-major, 128-byte swizzle, 8-row groups 1024 B apart.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFFu);  // start address
  d |= (uint64_t)1 << 16;                    // leading byte offset (unused: swizzled K-major)
  d |= (uint64_t)(1024 >> 4) << 32;          // stride byte offset
  d |= (uint64_t)1 << 46;                    // descriptor version
  d |= (uint64_t)2 << 61;                    // SWIZZLE_128B
  return d;
}

// Eight packed nibbles (k .. k+7) -> eight fp16 (q - 8) * scale in natural k order.
__device__ __forceinline__ uint4 dq8_natural(uint32_t w, uint32_t sc) {
  const __half2 s2 = bits_h2(sc);
  const __half2 magic_sub = bits_h2(0x64086408u);
  const __half2 p04 = __hmul2(__hsub2(bits_h2(lop3_and_or(w, 0x000F000Fu, 0x64006400u)), magic_sub), s2);
  const __half2 p15 = __hmul2(
      __hfma2(bits_h2(lop3_and_or(w, 0x00F000F0u, 0x64006400u)), bits_h2(0x2C002C00u), bits_h2(0xD480D480u)), s2);
  const uint32_t v = w >> 8;
  const __half2 p26 = __hmul2(__hsub2(bits_h2(lop3_and_or(v, 0x000F000Fu, 0x64006400u)), magic_sub), s2);
  const __half2 p37 = __hmul2(
      __hfma2(bits_h2(lop3_and_or(v, 0x00F000F0u, 0x64006400u)), bits_h2(0x2C002C00u), bits_h2(0xD480D480u)), s2);
  uint4 o;
  o.x = prmt(h2_bits(p04), h2_bits(p15), 0x5410);  // k0 k1
  o.y = prmt(h2_bits(p26), h2_bits(p37), 0x5410);  // k2 k3
  o.z = prmt(h2_bits(p04), h2_bits(p15), 0x7632);  // k4 k5
  o.w = prmt(h2_bits(p26), h2_bits(p37), 0x7632);  // k6 k7
  return o;
}

template <int EPI, int NTILE>
__global__ void __launch_bounds__(kTcThreads, 1) tc_qgemm_kernel(const __grid_constant__ CUtensorMap tmx,
                                                                 const QArgs a0) {
  extern __shared__ __align__(1024) uint8_t smraw[];
  constexpr int kBBytes = NTILE * kTcBK * 2;
  constexpr uint32_t kCols = NTILE < 32 ? 32 : NTILE;
  constexpr uint32_t kIdesc = (1u << 4) | ((uint32_t)(NTILE >> 3) << 17) | ((uint32_t)(kTcRows >> 4) << 24);

  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smraw) + 1023) & ~(uintptr_t)1023);
  uint8_t* sA = sm;
  uint8_t* sB = sm + kTcStages * kTcABytes;
  uint64_t* full_b = reinterpret_cast<uint64_t*>(sB + kTcStages * kBBytes);
  uint64_t* empty = full_b + kTcStages;
  uint64_t* done = empty + kTcStages;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
  volatile int* failed = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int tid = threadIdx.x, warp = tid >> 5;
  const int KS = gridDim.y, ks = blockIdx.y;
  const int R0 = blockIdx.x * kTcRows;
  const int tok0 = blockIdx.z * NTILE;
  const int nst_total = (a0.K + kTcBK - 1) / kTcBK;
  const int st0 = (ks * nst_total) / KS, st1 = ((ks + 1) * nst_total) / KS;
  const int nst = st1 - st0;
  const int row = R0 + tid;
  const bool row_ok = row < a0.N;
  const int G = a0.K >> 5;
  const uint8_t* wrow = a0.w + (size_t)(row_ok ? row : 0) * (size_t)(a0.K >> 1);
  const __half* srow = a0.s + (size_t)(row_ok ? row : 0) * G;

  // this row's packed weights for one stage: 2 x 16 bytes (64 k) + two group scales
  auto wload = [&](int s, uint4& w0, uint4& w1, uint32_t& s0, uint32_t& s1) {
    const int k0 = (st0 + s) * kTcBK;
    const uint4 fill = make_uint4(0x88888888u, 0x88888888u, 0x88888888u, 0x88888888u);
    w0 = fill;
    w1 = fill;
    s0 = 0;
    s1 = 0;
    if (s < nst && row_ok) {
      const uint8_t* p = wrow + (k0 >> 1);
      w0 = ld_stream16(p);
      s0 = h2_bits(__half2half2(srow[k0 >> 5]));
      if (k0 + 32 < a0.K) {
        w1 = ld_stream16(p + 16);
        s1 = h2_bits(__half2half2(srow[(k0 >> 5) + 1]));
      }
    }
  };

  uint4 wA[kTcStages], wB[kTcStages];
  uint32_t sc0[kTcStages], sc1[kTcStages];

  if (warp == 0) tmem_alloc(tmem_slot, kCols);
  if (tid == 0) {
    for (int i = 0; i < kTcStages; ++i) {
      mbar_init(&full_b[i], 1);
      mbar_init(&empty[i], 1);
    }
    mbar_init(done, 1);
    *failed = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    fence_proxy_async();
  }
  // Weights do not depend on the previous kernel: request the first stages before waiting.
#pragma unroll
  for (int u = 0; u < kTcStages; ++u) wload(u, wA[u], wB[u], sc0[u], sc1[u]);
  pdl_trigger();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_d = *tmem_slot;
  pdl_wait();

  int pend_slot = -1;  // thread 0: slot whose TMA load was issued but not yet waited for
  uint32_t pend_par = 0;
  for (int s0 = 0; s0 < nst; s0 += kTcStages) {
#pragma unroll
    for (int u = 0; u < kTcStages; ++u) {
      const int s = s0 + u;
      if (s >= nst) break;
      const uint32_t it = (uint32_t)(s / kTcStages);
      if (s >= kTcStages && !mbar_wait(&empty[u], (it - 1) & 1)) *failed = 1;
      if (tid == 0 && !*failed) {
        mbar_expect_tx(&full_b[u], kBBytes);
        tma_load_2d(sB + u * kBBytes, &tmx, &full_b[u], (st0 + s) * kTcBK, tok0);
        pend_slot = u;
        pend_par = it & 1;
      }
      // dequantise this row's 64 weights into the swizzled A tile
      {
        uint8_t* arow = sA + u * kTcABytes + (tid >> 3) * 1024 + (tid & 7) * 128;
        const uint32_t wv[8] = {wA[u].x, wA[u].y, wA[u].z, wA[u].w, wB[u].x, wB[u].y, wB[u].z, wB[u].w};
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          const uint4 v = dq8_natural(wv[c], c < 4 ? sc0[u] : sc1[u]);
          *reinterpret_cast<uint4*>(arow + ((c ^ (tid & 7)) << 4)) = v;
        }
      }
      wload(s + kTcStages, wA[u], wB[u], sc0[u], sc1[u]);
      fence_proxy_async();
      __syncthreads();
      if (*failed) break;
      if (tid == 0) {
        if (!mbar_wait(&full_b[u], it & 1)) {
          *failed = 1;
        } else {
          pend_slot = -1;
          tc_fence_after();
          const uint64_t ad = sw128_desc(smem_u32(sA + u * kTcABytes));
          const uint64_t bd = sw128_desc(smem_u32(sB + u * kBBytes));
#pragma unroll
          for (int kk = 0; kk < kTcBK / 16; ++kk)
            umma_f16(tmem_d, ad + 2 * kk, bd + 2 * kk, kIdesc, (s > 0 || kk > 0) ? 1u : 0u);
          umma_commit(&empty[u]);
        }
      }
    }
    __syncthreads();
    if (*failed) break;
  }
  // all MMAs issued by thread 0 -> done barrier; every thread waits (bounded)
  if (tid == 0) umma_commit(done);
  const bool done_ok = mbar_wait(done, 0);
  if (tid == 0 && pend_slot >= 0) mbar_wait(&full_b[pend_slot], pend_par);  // drain after a failure
  tc_fence_after();

  // accumulator -> shared-memory partial tile red[n][row] (the ring is no longer in use)
  float* red = reinterpret_cast<float*>(sm);
  constexpr int LDR = kTcRows + 4;
  const int mcount = min(NTILE, a0.M - tok0);
#pragma unroll 1
  for (int c = 0; c < NTILE; c += 16) {
    uint32_t r[16];
    tmem_ld16(tmem_d + ((uint32_t)(32 * warp) << 16) + (uint32_t)c, r);
#pragma unroll
    for (int j = 0; j < 16; ++j)
      if (c + j < mcount) red[(c + j) * LDR + tid] = (*failed || !done_ok) ? 0.f : __uint_as_float(r[j]);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem_d, kCols);
  if (tid == 0 && (*failed || !done_ok)) atomicOr(a0.check, 256u);

  QArgs a = a0;
  a.M = mcount;
  constexpr int LR = EPI == EPI_QKV ? 3 : (EPI == EPI_SWIGLU ? 2 : 1);
  if (a.lora_t) a.lora_t = a0.lora_t + (size_t)tok0 * LR * a0.lora_r;
  if (EPI == EPI_STORE || EPI == EPI_RESID) {
    const size_t os = (EPI == EPI_RESID || a0.out_f32) ? 4 : 2;
    a.out = static_cast<char*>(a0.out) + (size_t)tok0 * a0.ldo * os;
  } else if (EPI == EPI_SWIGLU) {
    a.out = static_cast<__half*>(a0.out) + (size_t)tok0 * (a0.N >> 1);
  } else {
    a.out = static_cast<__half*>(a0.out) + (size_t)tok0 * a0.H;
    a.pos = a0.pos + tok0;
    if (a0.slots) a.slots = a0.slots + tok0;
  }
  qgemm_epilogue<W_Q4, EPI, kTcRows>(a, red, KS, ks, R0);
}

// ------------------------------------------------------------------------------------------
// host side
// ------------------------------------------------------------------------------------------
namespace {

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return (EncodeTiledFn) nullptr;
    return reinterpret_cast<EncodeTiledFn>(p);
  }();
  return fn;
}

size_t tc_smem(int ntile) { return (size_t)kTcStages * (kTcABytes + ntile * kTcBK * 2) + 1024 + 256; }

template <int EPI, int NTILE>
int tc_launch(const CUtensorMap& map, const QArgs& a, int KS, cudaStream_t st) {
  static bool attr_done[64] = {};
  const int dev = device_index();
  auto kern = tc_qgemm_kernel<EPI, NTILE>;
  const size_t smem = tc_smem(NTILE);
  if (dev >= 0 && dev < 64 && !attr_done[dev]) {
    ORCH_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    attr_done[dev] = true;
  }
  const dim3 grid((a.N + kTcRows - 1) / kTcRows, KS, (a.M + NTILE - 1) / NTILE);
  ORCH_CUDA(launch_k(kern, grid, dim3(kTcThreads), smem, st, dim3(1, KS, 1), map, a));
  return ORCH_OK;
}

}  // namespace

static uint32_t g_tc_min_m = [] {
  const char* v = std::getenv("ORCHARD_TC_MIN_M");
  return v ? (uint32_t)std::atoi(v) : 17u;
}();

uint32_t tc_min_m() { return g_tc_min_m; }
void set_tc_min_m(uint32_t m) { g_tc_min_m = m; }

template <int EPI>
int tc_qgemm_run(QArgs a, cudaStream_t st) {
  if (a.x_f32 || a.M < 16 || (a.K % 32) != 0) return ORCH_ERR_UNSUPPORTED;
  EncodeTiledFn enc = encode_fn();
  if (!enc) return ORCH_ERR_UNSUPPORTED;
  if (((uintptr_t)a.x & 15) != 0) return ORCH_ERR_UNSUPPORTED;
  a.check = device_check_word();
  const int ntile = a.M <= 32 ? 32 : a.M <= 64 ? 64 : a.M <= 128 ? 128 : 256;
  CUtensorMap map;
  const cuuint64_t gdim[2] = {(cuuint64_t)a.K, (cuuint64_t)a.M};
  const cuuint64_t gstride[1] = {(cuuint64_t)a.K * 2};
  const cuuint32_t box[2] = {(cuuint32_t)kTcBK, (cuuint32_t)ntile};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult cr = enc(&map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(a.x), gdim, gstride, box, estr,
                          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                          CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (cr != CUDA_SUCCESS) return fail(ORCH_ERR_UNSUPPORTED, "tensor map encode failed");
  const int nst = (a.K + kTcBK - 1) / kTcBK;
  const int tiles = ((a.N + kTcRows - 1) / kTcRows) * ((a.M + ntile - 1) / ntile);
  const int per_sm = tc_smem(ntile) * 2 <= 227 * 1024 ? 2 : 1;
  int KS = 1;
  while (KS < 8 && tiles * KS < per_sm * num_sms() && nst >= 2 * kTcStages * KS) KS *= 2;
  int rc;
  switch (ntile) {
    case 32: rc = tc_launch<EPI, 32>(map, a, KS, st); break;
    case 64: rc = tc_launch<EPI, 64>(map, a, KS, st); break;
    case 128: rc = tc_launch<EPI, 128>(map, a, KS, st); break;
    default: rc = tc_launch<EPI, 256>(map, a, KS, st); break;
  }
  if (rc != ORCH_OK) return rc;
  return check_launch("tc_qgemm");
}

template int tc_qgemm_run<EPI_STORE>(QArgs, cudaStream_t);
template int tc_qgemm_run<EPI_RESID>(QArgs, cudaStream_t);
template int tc_qgemm_run<EPI_SWIGLU>(QArgs, cudaStream_t);
template int tc_qgemm_run<EPI_QKV>(QArgs, cudaStream_t);

}  // namespace orch

extern "C" int orch_set_tc_min_m(uint32_t m) {
  orch::set_tc_min_m(m);
  return ORCH_OK;
}
