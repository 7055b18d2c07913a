// INT4 dequant GEMM on the 5th-generation tensor cores (tcgen05 + TMEM), for M >= 17
// activation rows: batched decode (M = 16..256) and prefill (M = thousands of tokens).
//
// Replaces the reference's batched kernel (orchard/kernels/gemm_int4.metal:10-68, one
// thread per output, weights re-read per row) for the same packed format
// (orchard/quantizer.py:3-78).
//
// D[128 weight rows, NTILE tokens] (fp32, TMEM) += A[128, 16] . B[NTILE, 16]^T per MMA, in
// stages of 128 k, with four warp roles per CTA:
//  * a weight producer (one thread) streams packed 128-row x 128-k tiles and their scales
//    (per stage an 8 KB and a 1 KB bulk copy from the tiled layout, or 2-D TMA boxes from
//    the reference layout) into a 6-stage ring, starting before griddepcontrol.wait;
//  * an activation producer (one thread) streams the [NTILE, 128] fp16 activation tiles
//    (two TMA boxes of 64 k, SWIZZLE_128B; rows past M and k past K read as zero);
//  * eight dequantisation warps turn each packed tile into fp16 (q - 8) * scale with the
//    magic-exponent trick and store it with tcgen05.st into a ring of A tiles in tensor
//    memory (3-4 stages deep), one weight row per TMEM lane. They form two groups of four
//    (one warp per TMEM lane quarter) that take alternate stages, so two stages' chains of
//    wait, dequantise, store and arrive run at once;
//  * one thread issues eight tcgen05.mma.kind::f16 per stage with A from tensor memory and
//    B (activations) from shared memory; tcgen05.commit releases the activation and A
//    slots. Each handshake is one elected arrival per warp.
// Decode tiles (NTILE <= 64) use half the tensor memory and ~105 KB of shared memory, so
// two CTAs share an SM. After the K loop the accumulator is read with tcgen05.ld: a decode
// CTA that holds the whole K range runs the fused epilogue straight from registers
// (tc_epilogue16); otherwise the partials go through the same distributed-shared-memory
// reduction and fused epilogues as the mma.sync kernel (qgemm.cuh). TMA loads never use
// multicast.
//
// Every mbarrier wait is bounded (~2 s of globaltimer); on expiry the CTA records
// ORCH device check bit 8, stops issuing, drains what it issued and frees its TMEM.
#include <algorithm>
#include <cstdlib>

#include "tcgen05.cuh"

namespace orch {

constexpr int kWarpProdW = kWarpsDq;              // TMA producer of weights and scales
constexpr int kWarpProdX = kWarpsDq + 1;          // TMA producer of activations
constexpr int kWarpMma = kWarpsDq + 2;            // MMA issuer
constexpr int kTcThreads2 = (kWarpsDq + 3) * 32;

// Shared-memory and tensor-memory plan for 128-k stages. Weights (from HBM) and activations
// (from L2) have separate shared-memory rings so the weight stream runs far ahead without
// holding activation tiles: a weight slot is released by the dequantisation warps, an
// activation slot by the MMA's commit. The dequantised A tiles live in tensor memory (64
// columns per stage, beside the accumulator). Decode tiles (NTILE <= 64) take half of the
// SM's tensor memory and ~105 KB of shared memory, so two CTAs share an SM; prefill tiles
// take the whole SM.
template <int NTILE>
struct TcCfg {
  static constexpr bool kDecode = NTILE <= 64;
  static constexpr int kMinBlocks = kDecode ? 2 : 1;  // CTAs per SM
  static constexpr uint32_t kTmemCols = kDecode ? 256 : 512;
  static constexpr uint32_t kAccCols = NTILE < 32 ? 32 : NTILE;
  static constexpr int AR = (kTmemCols - kAccCols) / 64 < 4 ? (int)((kTmemCols - kAccCols) / 64) : 4;
  static constexpr int SW = 6;  // weight ring (with each stage's scales)
  static constexpr int SX = NTILE <= 16 ? 6 : (NTILE <= 32 ? 4 : (NTILE <= 128 ? 3 : 2));
  static constexpr int XSub = NTILE * kSub * 2;  // one 64-k swizzle atom of activations
  static constexpr int XBytes = 2 * XSub;
  static constexpr int OffX = 0;
  static constexpr int OffW = OffX + SX * XBytes;
  static constexpr int OffS = OffW + SW * kWBytes;
  static constexpr int OffBar = OffS + SW * kSBytes;  // a scale slot per weight slot
  static constexpr int Bytes = OffBar + 512;
  static_assert(2 * SW + 2 * SX + 2 * AR + 1 <= 62, "barrier area");
  // the split-K receive buffer reuses the rings and must stay below the barriers
  static_assert((kTcRows + 16) * NTILE * 4 <= OffBar, "receive buffer");
  static_assert(AR >= 2, "A ring");
  static_assert(kMinBlocks * (Bytes + 2048) <= 228 * 1024, "shared memory per SM");
  static_assert(XSub % 1024 == 0, "swizzle atoms are 1024-byte aligned");
};

// LoRA terms of one prefill tile from shared memory: the tile's slice of t (the regions it
// touches, all its activation rows) and of B (those regions, its columns), staged once after
// the K loop instead of 2r global loads per output. Same FMA order as lora_delta_r.
struct LoraSmem {
  const float* ts;  // [region][Mp][r]
  const float* bs;  // [region][r][bp]: columns c0.. of B, row pitch bp
  int reg0, c0, bp, r, Mp;
  __device__ __forceinline__ float operator()(int n, int reg, int col, int width) const {
    const float* t = ts + ((size_t)(reg - reg0) * Mp + n) * r;
    const float* b = bs + (size_t)(reg - reg0) * r * bp + (col - c0);
    float v = 0.f;
    for (int q = 0; q < r; ++q) v = fmaf(t[q], b[q * bp], v);
    return v;
  }
  // Columns col and col + 1 of a RoPE pair (col - c0 even: 8-byte aligned in bs): t[n] is
  // read once for both and B as float2, a third of the shared-memory wavefronts of two calls
  // (a warp's t row is one broadcast address; its B pairs are 256 contiguous bytes).
  __device__ __forceinline__ void pair(int n, int reg, int col, int width, float& d0, float& d1) const {
    const float* t = ts + ((size_t)(reg - reg0) * Mp + n) * r;
    const float* b = bs + (size_t)(reg - reg0) * r * bp + (col - c0);
    float v0 = 0.f, v1 = 0.f;
    if ((r & 3) == 0) {  // t rows 16-byte aligned
      for (int q = 0; q < r; q += 4) {
        const float4 t4 = *reinterpret_cast<const float4*>(t + q);
        const float tv[4] = {t4.x, t4.y, t4.z, t4.w};
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const float2 bb = *reinterpret_cast<const float2*>(b + (q + u) * bp);
          v0 = fmaf(tv[u], bb.x, v0);
          v1 = fmaf(tv[u], bb.y, v1);
        }
      }
    } else {
      for (int q = 0; q < r; ++q) {
        const float tq = t[q];
        const float2 bb = *reinterpret_cast<const float2*>(b + q * bp);
        v0 = fmaf(tq, bb.x, v0);
        v1 = fmaf(tq, bb.y, v1);
      }
    }
    d0 = v0;
    d1 = v1;
  }
};

// LAY 0: weights in the reference layout, read by 2-D TMA boxes of 128 rows x 64 bytes.
// LAY 1: weights in the tiled layout (qgemm.cuh), read by contiguous 8 KB bulk copies.
// LoRA term of a prefill QKV tile whose K range this CTA holds alone, added into its receive
// buffer before the epilogue: D[n][c] = sum_q t[n][q] B[q][c] for tokens n < Mp and the
// tile's 128 columns (column c is item row c / 2, pair element c % 2). mma.sync m16n8k8 with
// both operands split into two TF32 terms and the three products big.big + big.small +
// small.big (the dropped small.small is below 2^-22 of the product); k zero-padded to a
// multiple of 8. A warp takes units of 16 tokens x 64 columns: the t fragments of up to 32 k
// stay in registers across the unit's eight 16 x 8 output tiles. B is staged with a row pitch
// bp = 8 (mod 32) floats, so a fragment load (k = c, column g) touches 32 distinct banks.
__device__ __forceinline__ void lora_qkv_tile_into_recv(float* recv, const float* ts, const float* bs, int bp, int Mp,
                                                        int r, int warp, int nwarps, int lane) {
  constexpr int IRL = kTcRows / 2, NTU = kTcRows / 16;  // output tiles of 8 columns per unit
  const int g = lane >> 2, c = lane & 3;
  const int units = ((Mp + 15) / 16) * 2;
  for (int u = warp; u < units; u += nwarps) {
    const int m0 = (u >> 1) * 16, cb = (u & 1) * (kTcRows / 2);
    for (int kc = 0; kc < r; kc += 32) {
      uint32_t tb[4][4], tl[4][4];  // t fragments of k steps kc + 8s: big, small terms
#pragma unroll
      for (int st = 0; st < 4; ++st) {
        const int qa = kc + 8 * st + c, qb = qa + 4;
        const float fa[4] = {m0 + g < Mp && qa < r ? ts[(m0 + g) * r + qa] : 0.f,
                             m0 + g + 8 < Mp && qa < r ? ts[(m0 + g + 8) * r + qa] : 0.f,
                             m0 + g < Mp && qb < r ? ts[(m0 + g) * r + qb] : 0.f,
                             m0 + g + 8 < Mp && qb < r ? ts[(m0 + g + 8) * r + qb] : 0.f};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          tb[st][i] = to_tf32(fa[i]);
          tl[st][i] = to_tf32(fa[i] - __uint_as_float(tb[st][i]));
        }
      }
#pragma unroll 2
      for (int j = 0; j < NTU; ++j) {
        const int n0 = cb + 8 * j;
        float d[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int st = 0; st < 4; ++st) {
          if (kc + 8 * st < r) {
            const int qa = kc + 8 * st + c, qb = qa + 4;
            const float fb0 = qa < r ? bs[qa * bp + n0 + g] : 0.f;
            const float fb1 = qb < r ? bs[qb * bp + n0 + g] : 0.f;
            const uint32_t bb0 = to_tf32(fb0), bb1 = to_tf32(fb1);
            mma_tf32(d, tl[st], bb0, bb1);  // small terms first
            mma_tf32(d, tb[st], to_tf32(fb0 - __uint_as_float(bb0)), to_tf32(fb1 - __uint_as_float(bb1)));
            mma_tf32(d, tb[st], bb0, bb1);
          }
        }
        // d[0], d[1]: token m0 + g, columns n0 + 2c, n0 + 2c + 1 (item n0 / 2 + c, elements 0,
        // 1); d[2], d[3]: token m0 + g + 8
        const int irl = (n0 >> 1) + c;
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int n = m0 + g + 8 * h;
          if (n < Mp) {
            recv[(size_t)n * (IRL + 1) + irl] += d[2 * h];
            recv[((size_t)Mp + n) * (IRL + 1) + irl] += d[2 * h + 1];
          }
        }
      }
    }
  }
}

template <int EPI, int NTILE, int LAY>
__global__ void __launch_bounds__(kTcThreads2, TcCfg<NTILE>::kMinBlocks)
    tc_qgemm_kernel(const __grid_constant__ CUtensorMap tmx, const __grid_constant__ CUtensorMap tmw,
                    const __grid_constant__ CUtensorMap tms, const QArgs a0) {
  using C = TcCfg<NTILE>;
  extern __shared__ __align__(1024) uint8_t smraw[];
  constexpr uint32_t kIdesc = umma_idesc_f16<NTILE>();

  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smraw) + 1023) & ~(uintptr_t)1023);
  uint8_t* sX = sm + C::OffX;
  uint8_t* sW = sm + C::OffW;
  uint8_t* sS = sm + C::OffS;
  uint64_t* fullW = reinterpret_cast<uint64_t*>(sm + C::OffBar);
  uint64_t* emptyW = fullW + C::SW;
  uint64_t* fullX = emptyW + C::SW;
  uint64_t* emptyX = fullX + C::SX;
  uint64_t* afull = emptyX + C::SX;
  uint64_t* aempty = afull + C::AR;
  uint64_t* done = aempty + C::AR;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
  volatile int* failed = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int KS = gridDim.y, ks = blockIdx.y;
  const int R0 = blockIdx.x * kTcRows;
  const int tok0 = blockIdx.z * NTILE;
  // K is split over the cluster in 256-k blocks (two stages, one scale tile)
  const int nblk = (a0.K + 2 * kTcBK - 1) / (2 * kTcBK);
  const int nst_total = LAY == 1 ? 2 * nblk : (a0.K + kTcBK - 1) / kTcBK;
  const int st0 = ((ks * nblk) / KS) * 2;
  const int st1 = min(nst_total, (((ks + 1) * nblk) / KS) * 2);
  const int nst = st1 - st0;

  if (warp == 0) tmem_alloc(tmem_slot, C::kTmemCols);
  if (tid == 0) {
    for (int i = 0; i < C::SW; ++i) {
      mbar_init(&fullW[i], 1);
      mbar_init(&emptyW[i], kWarpsDq / 2);  // one elected lane per warp of the stage's group
    }
    for (int i = 0; i < C::SX; ++i) {
      mbar_init(&fullX[i], 1);
      mbar_init(&emptyX[i], 1);
    }
    for (int i = 0; i < C::AR; ++i) {
      mbar_init(&afull[i], kWarpsDq / 2);
      mbar_init(&aempty[i], 1);
    }
    mbar_init(done, 1);
    *failed = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    fence_proxy_async();
  }
  pdl_trigger();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_d = *tmem_slot;
  const uint32_t tmem_a = tmem_d + C::kAccCols;  // A ring: slot i at columns 64 i

  bool done_ok = true;
  if (warp == kWarpProdW) {
    // ------------- weight producer: packed tiles + scales, up to SW stages ahead -------------
    // Weights are written only by the packers, which release dependents on exit, so this
    // stream starts before griddepcontrol.wait and overlaps the previous kernel's tail.
    if (lane == 0) {
      int issued = 0;
      for (int p = 0; p < nst && !*failed; ++p) {
        const int v = p % C::SW;
        if (p >= C::SW && !mbar_wait_f(&emptyW[v], (uint32_t)(p / C::SW - 1) & 1, failed)) {
          *failed = 1;
          break;
        }
        // Every stage brings its own scales into the scale slot beside its weight slot, under
        // the same full / empty barriers: the tiled layout's half of the block's [8 groups][128
        // rows] scales (1 KB), or the reference layout's [128 rows][8 groups] box of the block
        // (its x, a multiple of 8 fp16, keeps the copy 16-byte aligned).
        const int half = (st0 + p) & 1;
        mbar_expect_tx(&fullW[v], (uint32_t)(kWBytes + (LAY == 1 ? kSBytes / 2 : kSBytes)));
        if (LAY == 1) {
          const uint8_t* blk = a0.w + ((size_t)blockIdx.x * nblk + ((st0 + p) >> 1)) * kQ4tBlockBytes;
          bulk_load(sW + v * kWBytes, blk + half * kWBytes, kWBytes, &fullW[v]);
          bulk_load(sS + v * kSBytes, blk + 4 * kQ4tStageBytes + half * (kSBytes / 2), kSBytes / 2, &fullW[v]);
        } else {
          const int k0 = (st0 + p) * kTcBK;
          tma_load_2d(sW + v * kWBytes, &tmw, &fullW[v], k0 >> 1, R0);
          tma_load_2d(sS + v * kSBytes, &tms, &fullW[v], ((st0 + p) >> 1) * 8, R0);
        }
        issued = p + 1;
      }
      // loads still in flight when the consumers gave up: wait for them before exiting
      if (*failed)
        for (int p = max(0, issued - C::SW); p < issued; ++p) mbar_wait(&fullW[p % C::SW], (uint32_t)(p / C::SW) & 1);
    }
    // The other lanes wait here, inactive: spinning on an mbarrier beside the issuing lane
    // would take its issue slots (and a blocked try_wait stalls the whole warp).
    __syncwarp();
    pdl_wait();
  } else if (warp == kWarpProdX) {
    // ------------- activation producer: up to SX stages ahead of the MMA -------------
    pdl_wait();  // activations may come from the previous kernel
    if (lane == 0) {
      int issued = 0;
      for (int p = 0; p < nst && !*failed; ++p) {
        const int v = p % C::SX;
        if (p >= C::SX && !mbar_wait_f(&emptyX[v], (uint32_t)(p / C::SX - 1) & 1, failed)) {
          *failed = 1;
          break;
        }
        mbar_expect_tx(&fullX[v], (uint32_t)C::XBytes);
        const int k0 = (st0 + p) * kTcBK;
        tma_load_2d(sX + v * C::XBytes, &tmx, &fullX[v], k0, tok0);
        tma_load_2d(sX + v * C::XBytes + C::XSub, &tmx, &fullX[v], k0 + kSub, tok0);
        issued = p + 1;
      }
      if (*failed)
        for (int p = max(0, issued - C::SX); p < issued; ++p) mbar_wait(&fullX[p % C::SX], (uint32_t)(p / C::SX) & 1);
    }
    __syncwarp();
  } else if (warp == kWarpMma) {
    // ---------------- MMA issuer: one thread; A from tensor memory, B from shared ----------------
    pdl_wait();
    if (lane == 0) {
      for (int s = 0; s < nst && !*failed; ++s) {
        const int v = s % C::SX, ai = s % C::AR;
        if (!mbar_wait_f(&fullX[v], (uint32_t)(s / C::SX) & 1, failed) ||
            !mbar_wait_f(&afull[ai], (uint32_t)(s / C::AR) & 1, failed)) {
          *failed = 1;
          break;
        }
        tc_fence_after();
        const uint64_t bd0 = sw128_desc(smem_u32(sX + v * C::XBytes));
        const uint64_t bd1 = sw128_desc(smem_u32(sX + v * C::XBytes + C::XSub));
#pragma unroll
        for (int kk = 0; kk < kTcBK / 16; ++kk)
          umma_f16_ta(tmem_d, tmem_a + ai * 64 + kk * 8, (kk < 4 ? bd0 : bd1) + 2 * (kk & 3), kIdesc,
                      (s > 0 || kk > 0) ? 1u : 0u);
        umma_commit(&emptyX[v]);
        umma_commit(&aempty[ai]);
      }
      umma_commit(done);
    }
    __syncwarp();
  } else {
    // ------- dequantisation warps: packed tile -> fp16 A tile in tensor memory -------
    // Warp w owns TMEM lanes 32 (w % 4) .. + 31 (= weight rows); warps 0-3 take the even
    // stages and warps 4-7 the odd ones, each warp writing all 128 k of its rows (columns
    // 0..63 of the slot) in two 64-k halves.
    pdl_wait();
    const int grp = warp >> 2, r = (warp & 3) * 32 + lane;
    const uint32_t lane_base = (uint32_t)((warp & 3) * 32) << 16;
    for (int s = grp; s < nst; s += 2) {
      const int v = s % C::SW, ai = s % C::AR;
      bool ok = mbar_wait_f(&fullW[v], (uint32_t)(s / C::SW) & 1, failed);
      if (ok && s >= C::AR) ok = mbar_wait_f(&aempty[ai], (uint32_t)(s / C::AR - 1) & 1, failed);
      if (!__all_sync(0xffffffffu, ok)) {  // the warp leaves together (it synchronises below)
        *failed = 1;
        break;
      }
      const uint8_t* wt = sW + v * kWBytes;
      const __half* st = reinterpret_cast<const __half*>(sS + v * kSBytes);
      uint4 wa[2], wb[2];
      uint32_t sca[2], scb[2];
#pragma unroll
      for (int j2 = 0; j2 < 2; ++j2) {
        if (LAY == 1) {  // 64-k stages [2 halves][128 rows][16 B]; the stage's scales [4 groups][128 rows]
          wa[j2] = *reinterpret_cast<const uint4*>(wt + j2 * kQ4tStageBytes + r * 16);
          wb[j2] = *reinterpret_cast<const uint4*>(wt + j2 * kQ4tStageBytes + (kQ4tStageBytes / 2) + r * 16);
          sca[j2] = h2_bits(__half2half2(st[(2 * j2) * kTcRows + r]));
          scb[j2] = h2_bits(__half2half2(st[(2 * j2 + 1) * kTcRows + r]));
        } else {  // TMA boxes: [128 rows][64 B], the block's scales [128 rows][8 groups]
          const int g0 = ((s & 1) * 2 + j2) * 2;  // group of the half's first 32 k in the block
          wa[j2] = *reinterpret_cast<const uint4*>(wt + r * 64 + j2 * 32);
          wb[j2] = *reinterpret_cast<const uint4*>(wt + r * 64 + j2 * 32 + 16);
          sca[j2] = h2_bits(__half2half2(st[r * 8 + g0]));
          scb[j2] = h2_bits(__half2half2(st[r * 8 + g0 + 1]));
        }
      }
      // The slot is refilled by TMA, i.e. written through the async proxy: order this warp's
      // generic-proxy reads of it before that write. Without the fence, 2-D TMA refills of
      // reference-layout slots overwrote data still being read, once stages alternated
      // between the two groups.
      fence_proxy_async();
      __syncwarp();
      if (lane == 0) mbar_arrive(&emptyW[v]);  // the packed slot is in registers now
#pragma unroll
      for (int j2 = 0; j2 < 2; ++j2) {
        const uint32_t wv[8] = {wa[j2].x, wa[j2].y, wa[j2].z, wa[j2].w, wb[j2].x, wb[j2].y, wb[j2].z, wb[j2].w};
        uint32_t q[32];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const uint32_t sc = i < 4 ? sca[j2] : scb[j2];
          const uint4 o = LAY == 1 ? dq8_tiled(wv[i], sc) : dq8_natural(wv[i], sc);
          q[4 * i] = o.x;
          q[4 * i + 1] = o.y;
          q[4 * i + 2] = o.z;
          q[4 * i + 3] = o.w;
        }
        // the store's source registers stay live until its wait (tmem_st32 waits)
        tmem_st32(tmem_a + lane_base + ai * 64 + j2 * 32, q);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&afull[ai]);
    }
  }
  done_ok = mbar_wait(done, 0);
  tc_fence_after();

  const int mcount = min(NTILE, a0.M - tok0);
  const bool bad = *failed || !done_ok;
  const int Mp = epi_mp(mcount);
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
    else a.slot0 = a0.slot0 + tok0;
  }

  if (KS == 1 && C::kDecode) {
    // The CTA holds the whole sum of a decode tile: the fused epilogue straight from tensor
    // memory, 16 activation rows at a time (warp w owns TMEM lanes / weight rows 32w .. + 31).
    // Prefill tiles (128-256 rows) keep the receive-buffer path below, where all eleven warps
    // share the epilogue (with four warps the LoRA terms of 256 rows took 8x512-token prefill
    // from 162 to 264 ms).
    // Warps w and w + 4 share TMEM lane quarter w % 4 and take alternate groups of 16
    // activation rows (one warp per quarter ran this latency-bound code ~2x slower).
    if (warp < kWarpsDq && !bad) {
      const int quarter = warp & 3;
#pragma unroll 1
      for (int cc = (warp >> 2) * 16; cc < Mp; cc += 32) {
        uint32_t r[16];
        tmem_ld16(tmem_d + ((uint32_t)(32 * quarter) << 16) + (uint32_t)cc, r);
        float v[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
        tc_epilogue16<EPI>(a, R0, quarter, lane, v, cc);
      }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) tmem_dealloc(tmem_d, C::kTmemCols);
    if (tid == 0 && bad) atomicOr(a0.check, 256u);
    return;
  }

  // accumulator rows -> owners' receive buffers (they alias the rings: wait for the cluster)
  cg::cluster_group cl = cg::this_cluster();
  cl.sync();
  float* recv = reinterpret_cast<float*>(sm);
  if (warp < kWarpsDq) {  // TMEM lanes 32 (w % 4) .. + 31; warps w, w + 4 alternate row groups
    const int quarter = warp & 3;
#pragma unroll 1
    for (int cc = (warp >> 2) * 16; cc < Mp; cc += 32) {
      uint32_t r[16];
      tmem_ld16(tmem_d + ((uint32_t)(32 * quarter) << 16) + (uint32_t)cc, r);
      float* dst = epi_dest<EPI, kTcRows>(cl, recv, Mp, KS, ks, quarter * 32 + lane, cc);
      const int pitch = epi_pitch<EPI, kTcRows>(KS);
#pragma unroll
      for (int j = 0; j < 16; ++j)
        if (cc + j < Mp) dst[j * pitch] = bad ? 0.f : __uint_as_float(r[j]);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem_d, C::kTmemCols);
  if (tid == 0 && bad) atomicOr(a0.check, 256u);
  if (!C::kDecode && a.lora_t != nullptr) {
    // prefill tiles: stage the LoRA operands of this tile beyond the receive buffer
    constexpr int RR = EPI == EPI_QKV ? 3 : (EPI == EPI_SWIGLU ? 2 : 1);
    const int reg0 = EPI == EPI_QKV ? R0 / a.H : 0;
    const int nreg = EPI == EPI_SWIGLU ? 2 : 1;
    const int c0 = EPI == EPI_QKV ? R0 - reg0 * a.H : (EPI == EPI_SWIGLU ? R0 >> 1 : R0);
    const int cw = EPI == EPI_SWIGLU ? kTcRows / 2 : kTcRows;
    const int width = EPI == EPI_QKV ? a.H : (EPI == EPI_SWIGLU ? a.N >> 1 : a.N);
    const int r = a.lora_r;
    // both staged arrays start on 16-byte boundaries (the pair reads above)
    const int ts_off = (epi_recv_floats<kTcRows>(mcount) + 3) & ~3;
    const int bs_off = ts_off + ((nreg * Mp * r + 3) & ~3);
    const int bp = cw + 8;  // staged B pitch (floats; 8 mod 32 for cw = 128)
    const size_t need = (size_t)(bs_off + nreg * r * bp) * sizeof(float);
    if ((EPI != EPI_QKV || c0 + kTcRows <= a.H) && need <= (size_t)C::OffBar) {
      float* ts = recv + ts_off;
      float* bs = recv + bs_off;
      for (int i = tid; i < nreg * Mp * r; i += kTcThreads2) {
        const int g = i / (Mp * r), rem = i - g * Mp * r, n = rem / r, q = rem - n * r;
        ts[i] = n < mcount ? a.lora_t[((size_t)n * RR + reg0 + g) * r + q] : 0.f;
      }
      for (int i = tid; i < nreg * r * cw; i += kTcThreads2) {
        const int g = i / (r * cw), rem = i - g * r * cw, q = rem / cw, cl = rem - q * cw, col = c0 + cl;
        bs[(g * r + q) * bp + cl] = col < width ? a.lora_b[((size_t)(reg0 + g) * r + q) * width + col] : 0.f;
      }
      if (EPI == EPI_QKV && KS == 1) {
        // the receive buffer holds this CTA's whole sums: add the LoRA term there
        __syncthreads();
        lora_qkv_tile_into_recv(recv, ts, bs, bp, Mp, r, warp, kTcThreads2 / 32, lane);
        a.lora_t = nullptr;
        qgemm_finish<W_Q4, EPI, kTcRows>(a, recv, KS, ks, R0);
        return;
      }
      // qgemm_finish's cluster barrier orders these stores before the epilogue reads them
      qgemm_finish<W_Q4, EPI, kTcRows>(a, recv, KS, ks, R0, LoraSmem{ts, bs, reg0, c0, bp, r, Mp});
      return;
    }
  }
  qgemm_finish<W_Q4, EPI, kTcRows>(a, recv, KS, ks, R0);
}

// ------------------------------------------------------------------------------------------
// host side
// ------------------------------------------------------------------------------------------
namespace {

template <int EPI, int NTILE, int LAY>
int tc_launch(const CUtensorMap& mx, const CUtensorMap& mw, const CUtensorMap& ms, const QArgs& a, int KS,
              cudaStream_t st) {
  static bool attr_done[64] = {};
  const int dev = device_index();
  auto kern = tc_qgemm_kernel<EPI, NTILE, LAY>;
  const size_t smem = TcCfg<NTILE>::Bytes + 1024;
  if (dev >= 0 && dev < 64 && !attr_done[dev]) {
    ORCH_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    attr_done[dev] = true;
  }
  const dim3 grid((a.N + kTcRows - 1) / kTcRows, KS, (a.M + NTILE - 1) / NTILE);
  ORCH_CUDA(launch_k(kern, grid, dim3(kTcThreads2), smem, st, dim3(1, KS, 1), mx, mw, ms, a));
  return ORCH_OK;
}

}  // namespace

static uint32_t g_tc_min_m = [] {
  const char* v = std::getenv("ORCHARD_TC_MIN_M");
  return v ? (uint32_t)std::atoi(v) : 17u;
}();

uint32_t tc_min_m() { return g_tc_min_m; }
void set_tc_min_m(uint32_t m) { g_tc_min_m = m; }

template <int EPI, int LAY>
int tc_dispatch(const CUtensorMap& mx, const CUtensorMap& mw, const CUtensorMap& ms, const QArgs& a, int ntile,
                int KS, cudaStream_t st) {
  switch (ntile) {
    case 16: return tc_launch<EPI, 16, LAY>(mx, mw, ms, a, KS, st);
    case 32: return tc_launch<EPI, 32, LAY>(mx, mw, ms, a, KS, st);
    case 64: return tc_launch<EPI, 64, LAY>(mx, mw, ms, a, KS, st);
    case 128: return tc_launch<EPI, 128, LAY>(mx, mw, ms, a, KS, st);
    default: return tc_launch<EPI, 256, LAY>(mx, mw, ms, a, KS, st);
  }
}

template <int EPI>
int tc_qgemm_run(QArgs a, cudaStream_t st) {
  if (a.tiled && a.M <= 64) {  // batched decode: persistent stream-K kernel
    const int rc = tc_sk_run<EPI>(a, st);
    if (rc != ORCH_ERR_UNSUPPORTED) return rc;
  }
  // Reference layout: tensor maps need 16-byte row strides, so K % 256 == 0 for the scale
  // rows. Tiled layout: any K % 32 == 0 (the layout is padded to 256).
  const bool tiled = a.tiled != 0;
  if (a.x_f32 || a.M < 1 || (!tiled && (a.K % 256) != 0) || (a.K % 8) != 0 || !encode_fn())
    return ORCH_ERR_UNSUPPORTED;
  if (((uintptr_t)a.x & 15) != 0 || ((uintptr_t)a.w & 15) != 0 || (!tiled && ((uintptr_t)a.s & 15) != 0))
    return ORCH_ERR_UNSUPPORTED;
  ORCH_CHECK_WORD(a.check);
  const int ntile = a.M <= 16 ? 16 : a.M <= 32 ? 32 : a.M <= 64 ? 64 : a.M <= 128 ? 128 : 256;
  CUtensorMap mx, mw, ms;
  bool ok = encode2d(&mx, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, a.x, (uint64_t)a.K, (uint64_t)a.M, (uint64_t)a.K * 2,
                     kSub, ntile, CU_TENSOR_MAP_SWIZZLE_128B);
  if (ok && !tiled)
    ok = encode2d(&mw, CU_TENSOR_MAP_DATA_TYPE_UINT8, a.w, (uint64_t)(a.K / 2), (uint64_t)a.N, (uint64_t)(a.K / 2),
                  kTcBK / 2, kTcRows, CU_TENSOR_MAP_SWIZZLE_NONE) &&
         encode2d(&ms, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, a.s, (uint64_t)(a.K / 32), (uint64_t)a.N,
                  (uint64_t)(a.K / 32) * 2, 8, kTcRows, CU_TENSOR_MAP_SWIZZLE_NONE);
  if (!ok) return fail(ORCH_ERR_UNSUPPORTED, "tensor map encode failed");
  if (tiled) mw = ms = mx;  // unused by the tiled kernel
  const int nblk = (a.K + 2 * kTcBK - 1) / (2 * kTcBK);  // 256-k blocks
  const int tiles = ((a.N + kTcRows - 1) / kTcRows) * ((a.M + ntile - 1) / ntile);
  // split K only as far as one wave of CTAs covers the SMs
  const int slots = (ntile <= 64 ? 2 : 1) * num_sms();  // TcCfg::kMinBlocks
  int KS = 1;
  while (KS < 8 && tiles * KS * 2 <= slots && nblk >= KS * 4) KS *= 2;
  static const int ks_force = [] {  // ORCHARD_TC_KS=1/2/4/8 fixes the split (measurements)
    const char* e = std::getenv("ORCHARD_TC_KS");
    const int v = e ? std::atoi(e) : 0;
    return (v == 1 || v == 2 || v == 4 || v == 8) ? v : 0;
  }();
  if (ks_force > 0) KS = std::min(ks_force, std::max(1, nblk));
  const int rc = tiled ? tc_dispatch<EPI, 1>(mx, mw, ms, a, ntile, KS, st)
                       : tc_dispatch<EPI, 0>(mx, mw, ms, a, ntile, KS, st);
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
