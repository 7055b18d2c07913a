// tcgen05 / TMA building blocks shared by the tensor-core INT4 GEMMs (tcgemm.cu, the
// per-tile kernel; tcgemm_sk.cu, the persistent stream-K decode kernel): inline PTX for
// tensor-memory allocation, loads and stores, the kind::f16 MMA with A in tensor memory,
// commits, shared-memory matrix descriptors, 2-D TMA loads (never multicast), the INT4
// dequantisation of eight nibbles, and the host-side tensor-map encoder.
#pragma once

#include <cuda.h>

#include "async_copy.cuh"
#include "qgemm.cuh"

namespace orch {

constexpr int kTcRows = 128;                    // weight rows per tile (TMEM lanes)
constexpr int kTcBK = 128;                      // k per stage: two 128-byte swizzle atoms of fp16
constexpr int kSub = 64;                        // k per swizzle atom / tiled 64-k stage
constexpr int kWBytes = kTcRows * (kTcBK / 2);  // packed INT4 tile: 128 rows x 64 bytes
constexpr int kSBytes = kTcRows * 16;           // scales of a 256-k block: 128 rows x 8 fp16
constexpr int kWarpsDq = 8;                     // dequantisation warps

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(
          smem_u32(dst)),
      "l"(map), "r"(smem_u32(bar)), "r"(x), "r"(y)
      : "memory");
}
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
// D (TMEM) += A (TMEM, K-major: row i in lane i, two fp16 of consecutive k per column) . B (smem)
__device__ __forceinline__ void umma_f16_ta(uint32_t tmem_d, uint32_t tmem_a, uint64_t bdesc, uint32_t idesc,
                                            uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}\n" ::"r"(tmem_d),
      "r"(tmem_a), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Thirty-two consecutive 32-bit columns of this thread's TMEM lane; waits for completion.
// The store reads its source registers until tcgen05.wait::st, so both instructions sit in
// one asm statement: the compiler cannot reuse those registers in between.
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};\n\t"
      "tcgen05.wait::st.sync.aligned;" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]),
      "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]),
      "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}
// Sixteen consecutive 32-bit columns of this thread's TMEM lane; waits for completion. The
// destination registers are written until tcgen05.wait::ld, so the load and its wait are one
// asm statement: nothing can read them in between.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr)
      : "memory");
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

// Instruction descriptor of kind::f16: fp16 A and B, fp32 D, K-major operands, M = 128.
template <int NTILE>
__host__ __device__ constexpr uint32_t umma_idesc_f16() {
  return (1u << 4) | ((uint32_t)(NTILE >> 3) << 17) | ((uint32_t)(kTcRows >> 4) << 24);
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

// Eight nibbles of the tiled layout (stored k0 k2 k4 k6 k1 k3 k5 k7) -> eight fp16
// (q - 8) * scale in natural k order, with no byte permutes.
__device__ __forceinline__ uint4 dq8_tiled(uint32_t w, uint32_t sc) {
  const __half2 s2 = bits_h2(sc);
  const __half2 magic_sub = bits_h2(0x64086408u);
  const __half2 hi_mul = bits_h2(0x2C002C00u), hi_add = bits_h2(0xD480D480u);
  const uint32_t v = w >> 8;
  uint4 o;
  o.x = h2_bits(__hmul2(__hsub2(bits_h2(lop3_and_or(w, 0x000F000Fu, 0x64006400u)), magic_sub), s2));
  o.y = h2_bits(__hmul2(__hfma2(bits_h2(lop3_and_or(w, 0x00F000F0u, 0x64006400u)), hi_mul, hi_add), s2));
  o.z = h2_bits(__hmul2(__hsub2(bits_h2(lop3_and_or(v, 0x000F000Fu, 0x64006400u)), magic_sub), s2));
  o.w = h2_bits(__hmul2(__hfma2(bits_h2(lop3_and_or(v, 0x00F000F0u, 0x64006400u)), hi_mul, hi_add), s2));
  return o;
}

// The fused epilogue from registers, for activation rows n0 .. n0 + 15: the lane holds tile
// row rl = 32 quarter + lane of the tile starting at weight row R0, v[i] = sum_k
// W[R0 + rl][k] x[n0 + i][k]. Pairs of rows meet through shuffles: SwiGLU's gate row 32b + i
// and up row 32b + 16 + i (lanes i, i + 16 of one warp), a RoPE pair 2p, 2p + 1 (adjacent
// lanes); the arithmetic is epi_apply's.
template <int EPI>
__device__ __forceinline__ void tc_epilogue16(const QArgs& a, int R0, int quarter, int lane, const float (&v)[16],
                                              int n0) {
  const int rl = quarter * 32 + lane;
  const int M = a.M;
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    const int n = n0 + i;
    if (EPI == EPI_STORE || EPI == EPI_RESID) {
      const int row = R0 + rl;
      if (n < M && row < a.N) epi_apply<W_Q4, EPI>(a, n, row, v[i], 0.f);
    } else if (EPI == EPI_SWIGLU) {
      const int j = (R0 >> 1) + quarter * 16 + (lane & 15);
      const float up = __shfl_xor_sync(0xffffffffu, v[i], 16);
      if (n < M && lane < 16 && j < (a.N >> 1)) epi_apply<W_Q4, EPI>(a, n, j, v[i], up);
    } else {
      const int row = R0 + rl;
      const float v1 = __shfl_xor_sync(0xffffffffu, v[i], 1);
      if (n < M && (lane & 1) == 0 && row < a.N) epi_apply<W_Q4, EPI>(a, n, row, v[i], v1);
    }
  }
}

// ---- host: tensor maps ----------------------------------------------------------------
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

inline EncodeTiledFn encode_fn() {
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

// 2-D tensor map: `inner` elements per row, `outer` rows `row_bytes` apart; out-of-range
// boxes read as zero.
inline bool encode2d(CUtensorMap* map, CUtensorMapDataType dt, const void* base, uint64_t inner, uint64_t outer,
                     uint64_t row_bytes, uint32_t box_inner, uint32_t box_outer, CUtensorMapSwizzle sw) {
  const cuuint64_t gdim[2] = {inner, outer};
  const cuuint64_t gstride[1] = {row_bytes};
  const cuuint32_t box[2] = {box_inner, box_outer};
  const cuuint32_t estr[2] = {1, 1};
  return encode_fn()(map, dt, 2, const_cast<void*>(base), gdim, gstride, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                     sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace orch
