// INT4 decode GEMV on tiled weights, M <= 8 activation rows (batch-1..8 decode).
//
// Replaces the reference's one-thread-per-output-row kernel
// (orchard/kernels/gemv_int4.metal:10-74) for weights re-laid by orch_q4t_pack
// (qgemm.cuh: 128-row tiles, 64-k stages of [2 halves][128 rows][16 B], per-block scales).
//
// Design (sm_100a): every warp owns 16 weight rows of a 64-row CTA and streams them through
// its own ring of three 256-k blocks in shared memory with cp.async (16-byte copies: 512
// contiguous bytes of nibbles per 64-k stage + 256 bytes of scales per block), two blocks
// ahead, so 4-7 KB per warp are in flight without holding registers and no CTA-wide barrier
// sits in the loop. The loop body is unrolled over the four stages of a block, which keeps
// the instruction count per weight byte low (the kernel is issue-bound, not memory-bound,
// when each stage pays its own address arithmetic and waits). Lane (g, c) takes
// 8 bytes (16 k) of rows g and g + 8; the tiled nibble order makes the magic-exponent
// extraction yield (k, k+1) pairs, which are exactly the mma.sync m16n8k16 A fragments when
// each lane's 16 k are walked 4 at a time, so the activations (B fragments) are read in
// natural order from a per-CTA copy in shared memory. The CTAs of a cluster split K; their
// partial sums meet in the same distributed-shared-memory reduce-scatter and fused
// epilogues as the other GEMMs (qgemm.cuh).
#include <algorithm>
#include <cstdlib>

#include "qgemm.cuh"

namespace orch {

namespace {

constexpr int kGvWarps = 4;
constexpr int kGvThreads = kGvWarps * 32;
constexpr int kGvRows = kGvWarps * 16;    // rows per CTA
constexpr int kGvBlocks = 3;              // per-warp ring: 3 blocks of 4 stages (256 k)
constexpr int kGvBlockBytes = 4 * 512 + 256;  // nibbles of 16 rows x 256 k + their 8 scale groups
constexpr int kGvRingBytes = kGvWarps * kGvBlocks * kGvBlockBytes;

__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(static_cast<uint32_t>(__cvta_generic_to_shared(dst))),
               "l"(src)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// (q - 8) * scale for the nibble pairs at positions (0, 4) / (1, 5) of a word.
__device__ __forceinline__ uint32_t gv_lo(uint32_t w, uint32_t sc) {
  const __half2 v = bits_h2(lop3_and_or(w, 0x000F000Fu, 0x64006400u));
  return h2_bits(__hmul2(__hsub2(v, bits_h2(0x64086408u)), bits_h2(sc)));
}
__device__ __forceinline__ uint32_t gv_hi(uint32_t w, uint32_t sc) {
  const __half2 v = bits_h2(lop3_and_or(w, 0x00F000F0u, 0x64006400u));
  return h2_bits(__hmul2(__hfma2(v, bits_h2(0x2C002C00u), bits_h2(0xD480D480u)), bits_h2(sc)));
}

// Activation row pitch in shared memory: 64 k per stage plus 16 bytes, so the two rows a
// quarter-warp reads with one 16-byte load fall into distinct banks.
__host__ __device__ __forceinline__ int gv_xpitch(int nst) { return nst * 128 + 16; }

template <int EPI>
__global__ void __launch_bounds__(kGvThreads) gemv_tiled_kernel(const QArgs a) {
  extern __shared__ __align__(16) uint8_t smem[];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int g = lane >> 2, c = lane & 3;
  const int KS = gridDim.y, ks = blockIdx.y;
  const int R0 = blockIdx.x * kGvRows;
  const int nblk = (a.K + kQ4tBlockK - 1) / kQ4tBlockK;
  const int b0 = (ks * nblk) / KS, nb = ((ks + 1) * nblk) / KS - b0;  // this CTA's 256-k blocks
  const int xp = gv_xpitch(4 * nb);

  uint8_t* ring = smem + warp * kGvBlocks * kGvBlockBytes;
  uint8_t* xs = smem + kGvRingBytes;
  const int wrow = (R0 & 127) + warp * 16;  // first row of this warp inside its 128-row tile
  // this lane's copy sources inside a block: nibbles of stage j at + j * 4096, scales
  const uint8_t* src = a.w + ((size_t)(R0 >> 7) * nblk + b0) * kQ4tBlockBytes + (lane >> 4) * (kQ4tStageBytes / 2) +
                       (wrow + (lane & 15)) * 16;
  const uint8_t* ssrc = a.w + ((size_t)(R0 >> 7) * nblk + b0) * kQ4tBlockBytes + 4 * kQ4tStageBytes +
                        ((lane >> 1) * kQ4tRows + wrow) * 2 + (lane & 1) * 16;
  const int dst_off = (lane >> 4) * 256 + (lane & 15) * 16;
  const int sdst_off = 2048 + (lane >> 1) * 32 + (lane & 1) * 16;

  auto issue = [&](int bb) {  // block b0 + bb into ring slot bb % kGvBlocks
    if (bb < nb) {
      uint8_t* dst = ring + (bb % kGvBlocks) * kGvBlockBytes;
      const uint8_t* sp = src + (size_t)bb * kQ4tBlockBytes;
#pragma unroll
      for (int j = 0; j < 4; ++j) cp_async16(dst + j * 512 + dst_off, sp + j * kQ4tStageBytes);
      if (lane < 16) cp_async16(dst + sdst_off, ssrc + (size_t)bb * kQ4tBlockBytes);
    }
    cp_async_commit();  // empty groups keep the group count uniform
  };

  // A CTA may write a cluster peer's shared memory only once the peer runs. With the RMSNorm
  // prologue its cluster barrier establishes that; otherwise a split barrier does, arrived
  // here and waited on just before the push, when it has long completed.
  const bool norm_prologue = a.norm_w != nullptr;
  if (!norm_prologue) asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");
  // Weights do not depend on the previous kernel (the packers release dependents only on
  // exit): start the rings before griddepcontrol.wait.
  issue(0);
  issue(1);
  pdl_trigger();
  pdl_wait();

  // activations x[n][k] for n < M, k in this CTA's K range (zero past K), natural order
  const int kbeg = b0 * kQ4tBlockK, units = nb * 32;  // 8 halves per unit
  if (a.norm_w == nullptr) {
    for (int i = threadIdx.x; i < a.M * units; i += kGvThreads) {
      const int n = i / units, u = i - n * units;
      const int k = kbeg + u * 8;
      uint4 v = make_uint4(0, 0, 0, 0);
      if (k < a.K) v = __ldg(reinterpret_cast<const uint4*>(static_cast<const __half*>(a.x) + (size_t)n * a.K + k));
      *reinterpret_cast<uint4*>(xs + n * xp + u * 16) = v;
    }
  } else {
    // The RMSNorm of orchard/kernels/rmsnorm.metal:23-35 fused in front of the projection,
    // rsqrt(sum(x^2) / K + eps) per row of the fp32 residual, then fp16(x * rsqrt * gamma)
    // staged for this CTA's K slice -- the arithmetic of rmsnorm_vec_kernel, summed in another
    // order. The KS CTAs splitting K form one cluster: each sums the squares of its own slice
    // only (all rows in one pass, so M loads are in flight; per row a warp butterfly, then
    // the four warps as (w0 + w2) + (w1 + w3)), publishes the M partials in shared memory,
    // and after one cluster barrier every CTA adds the KS partials in rank order, so all of
    // them scale by the same factor. (Each CTA reading whole rows cost KS times the L2 reads:
    // 68 us instead of 21 us for the 8-row gate/up launch with its 8-way split.)
    static_assert(kGvWarps == 4, "the cross-warp sum below is written for four warps");
    __shared__ float red8[kGvWarps][8];
    __shared__ float ss_part[8];
    __shared__ float inv_s[8];
    const float* xr = static_cast<const float*>(a.x);
    const int kend = min(a.K, kbeg + nb * kQ4tBlockK);
    float ss[8];
#pragma unroll
    for (int n = 0; n < 8; ++n) ss[n] = 0.f;
    for (int k = kbeg + threadIdx.x * 4; k < kend; k += kGvThreads * 4) {
      float4 v[8];
#pragma unroll
      for (int n = 0; n < 8; ++n)
        if (n < a.M) v[n] = __ldg(reinterpret_cast<const float4*>(xr + (size_t)n * a.K + k));
#pragma unroll
      for (int n = 0; n < 8; ++n)
        if (n < a.M) {
          ss[n] = fmaf(v[n].x, v[n].x, ss[n]);
          ss[n] = fmaf(v[n].y, v[n].y, ss[n]);
          ss[n] = fmaf(v[n].z, v[n].z, ss[n]);
          ss[n] = fmaf(v[n].w, v[n].w, ss[n]);
        }
    }
#pragma unroll
    for (int n = 0; n < 8; ++n) {
      if (n < a.M) {
        const float t = warp_sum(ss[n]);
        if ((threadIdx.x & 31) == 0) red8[threadIdx.x >> 5][n] = t;
      }
    }
    __syncthreads();
    if (threadIdx.x < a.M) {
      const int n = threadIdx.x;
      ss_part[n] = (red8[0][n] + red8[2][n]) + (red8[1][n] + red8[3][n]);
    }
    // Every CTA of the cluster reaches this barrier and the one before the split-K exchange
    // below, so a peer's ss_part is read before that peer can exit.
    cg::cluster_group clu = cg::this_cluster();
    clu.sync();
    if (threadIdx.x < a.M) {
      const int n = threadIdx.x;
      float t = 0.f;
      for (int r = 0; r < KS; ++r) t += *clu.map_shared_rank(&ss_part[n], (unsigned)r);
      inv_s[n] = rsqrtf(t / (float)a.K + a.norm_eps);
    }
    __syncthreads();
    for (int i = threadIdx.x; i < a.M * units; i += kGvThreads) {
      const int n = i / units, u = i - n * units;
      const int k = kbeg + u * 8;
      uint4 v = make_uint4(0, 0, 0, 0);
      if (k < a.K) {
        const float inv = inv_s[n];
        const float4 x0 = __ldg(reinterpret_cast<const float4*>(xr + (size_t)n * a.K + k));
        const float4 x1 = __ldg(reinterpret_cast<const float4*>(xr + (size_t)n * a.K + k + 4));
        const float4 g0 = __ldg(reinterpret_cast<const float4*>(a.norm_w + k));
        const float4 g1 = __ldg(reinterpret_cast<const float4*>(a.norm_w + k + 4));
        v.x = h2_bits(__floats2half2_rn(x0.x * inv * g0.x, x0.y * inv * g0.y));
        v.y = h2_bits(__floats2half2_rn(x0.z * inv * g0.z, x0.w * inv * g0.w));
        v.z = h2_bits(__floats2half2_rn(x1.x * inv * g1.x, x1.y * inv * g1.y));
        v.w = h2_bits(__floats2half2_rn(x1.z * inv * g1.z, x1.w * inv * g1.w));
      }
      *reinterpret_cast<uint4*>(xs + n * xp + u * 16) = v;
    }
  }
  __syncthreads();

  // two accumulators (even / odd k-steps) halve the chain of dependent MMAs
  float acc[4] = {0.f, 0.f, 0.f, 0.f}, acc2[4] = {0.f, 0.f, 0.f, 0.f};
  const bool has_x = g < a.M;
  const uint8_t* xrow = xs + (has_x ? g : 0) * xp + c * 32;
  const int woff = (c >> 1) * 256 + g * 16 + (c & 1) * 8;  // row g; row g + 8 is 128 bytes on
  const int soff = 2048 + (c >> 1) * 32 + g * 2;           // group (c >> 1) of stage 0, row g
  for (int bb = 0; bb < nb; ++bb) {
    issue(bb + 2);
    cp_async_wait<2>();  // this lane's copies of block bb have landed
    __syncwarp();        // ... and so have the other lanes'
    const uint8_t* buf = ring + (bb % kGvBlocks) * kGvBlockBytes;
    const uint8_t* xb = xrow + bb * 512;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const uint2 w0 = *reinterpret_cast<const uint2*>(buf + j * 512 + woff);
      const uint2 w1 = *reinterpret_cast<const uint2*>(buf + j * 512 + woff + 128);
      const uint32_t s0 = h2_bits(__half2half2(*reinterpret_cast<const __half*>(buf + soff + j * 64)));
      const uint32_t s1 = h2_bits(__half2half2(*reinterpret_cast<const __half*>(buf + soff + j * 64 + 16)));
      uint4 x0 = make_uint4(0, 0, 0, 0), x1 = x0;
      if (has_x) {
        x0 = *reinterpret_cast<const uint4*>(xb + j * 128);
        x1 = *reinterpret_cast<const uint4*>(xb + j * 128 + 16);
      }
      const uint32_t u0[4] = {w0.x, w0.x >> 8, w0.y, w0.y >> 8};
      const uint32_t u1[4] = {w1.x, w1.x >> 8, w1.y, w1.y >> 8};
      const uint32_t bx[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
#pragma unroll
      for (int t = 0; t < 4; t += 2) {
        mma_16816(acc, gv_lo(u0[t], s0), gv_lo(u1[t], s1), gv_hi(u0[t], s0), gv_hi(u1[t], s1), bx[2 * t],
                  bx[2 * t + 1]);
        mma_16816(acc2, gv_lo(u0[t + 1], s0), gv_lo(u1[t + 1], s1), gv_hi(u0[t + 1], s0), gv_hi(u1[t + 1], s1),
                  bx[2 * t + 2], bx[2 * t + 3]);
      }
    }
    __syncwarp();  // slot bb is read: the copies issued next iteration may overwrite it
  }
  cp_async_wait<0>();
#pragma unroll
  for (int i = 0; i < 4; ++i) acc[i] += acc2[i];

  // ---- partials -> owners' receive buffers ----
  // The receive buffer has its own region past the rings and the largest K slice's
  // activations (the same offset in every CTA of the cluster), so partials are pushed as soon
  // as this CTA's loop ends: one cluster barrier, in qgemm_finish. (Aliased onto the rings it
  // needed a barrier before the push as well: 0.8 us of a ~4 us launch at one row.)
  cg::cluster_group cl = cg::this_cluster();
  if (!norm_prologue) asm volatile("barrier.cluster.wait.aligned;" ::: "memory");
  const int nb_max = (nblk + KS - 1) / KS;
  float* recv = reinterpret_cast<float*>(smem + kGvRingBytes + (size_t)a.M * gv_xpitch(4 * nb_max));
  const int Mp = epi_mp(a.M);
  const int n0 = 2 * c;
  if (n0 < Mp) {  // Mp is a multiple of 4, so n0 + 1 < Mp too
    const int rl = warp * 16 + g;
    const int pitch = epi_pitch<EPI, kGvRows>(KS);
    float* d0 = epi_dest<EPI, kGvRows>(cl, recv, Mp, KS, ks, rl, n0);
    float* d1 = epi_dest<EPI, kGvRows>(cl, recv, Mp, KS, ks, rl + 8, n0);
    d0[0] = acc[0];
    d0[pitch] = acc[1];
    d1[0] = acc[2];
    d1[pitch] = acc[3];
  }
  qgemm_finish<W_Q4, EPI, kGvRows>(a, recv, KS, ks, R0);
}

template <int EPI>
size_t gv_smem(int M, int nst) {  // rings, activations of the largest K slice, receive buffer
  return (size_t)kGvRingBytes + (size_t)M * gv_xpitch(nst) + (size_t)4 * epi_recv_floats<kGvRows>(M);
}

}  // namespace

uint32_t gemv_max_m() { return 8; }

template <int EPI>
int gemv_tiled_run(QArgs a, cudaStream_t st) {
  if (a.M < 1 || a.M > 8 || (a.x_f32 && a.norm_w == nullptr)) return ORCH_ERR_UNSUPPORTED;
  ORCH_CHECK_WORD(a.check);
  const int nblk = (a.K + kQ4tBlockK - 1) / kQ4tBlockK;
  const int ctas = (a.N + kGvRows - 1) / kGvRows;
  // Split K until there are a few CTAs per SM and each CTA's activations stay within 32 KB.
  // (A 16 KB bound split 8-row launches 8 ways, 4 ways being faster: 4096 x 11008 took 13.5
  // instead of 10.5 us, 4096 x 32000 31.5 instead of 27.2 us.)
  int KS = 1;
  static const int ks_force = [] {
    const char* e = std::getenv("ORCHARD_GEMV_KS");
    return e ? std::atoi(e) : 0;
  }();
  while (KS < 8 && nblk >= 2 * KS &&
         (ctas * KS < 4 * num_sms() || (size_t)a.M * gv_xpitch(((nblk + KS - 1) / KS) * 4) > 32768))
    KS *= 2;
  if (ks_force > 0) KS = std::min(ks_force, nblk);
  const int nst_max = ((nblk + KS - 1) / KS) * 4;  // stages of the largest K slice
  const size_t smem = gv_smem<EPI>(a.M, nst_max);
  static bool attr_done[64] = {};
  const int dev = device_index();
  auto kern = gemv_tiled_kernel<EPI>;
  if (dev >= 0 && dev < 64 && !attr_done[dev]) {
    ORCH_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024));
    attr_done[dev] = true;
  }
  if (smem > 200 * 1024) return ORCH_ERR_UNSUPPORTED;
  ORCH_CUDA(launch_k(kern, dim3(ctas, KS, 1), dim3(kGvThreads), smem, st, dim3(1, KS, 1), a));
  return check_launch("gemv_tiled");
}

template int gemv_tiled_run<EPI_STORE>(QArgs, cudaStream_t);
template int gemv_tiled_run<EPI_RESID>(QArgs, cudaStream_t);
template int gemv_tiled_run<EPI_SWIGLU>(QArgs, cudaStream_t);
template int gemv_tiled_run<EPI_QKV>(QArgs, cudaStream_t);

}  // namespace orch
