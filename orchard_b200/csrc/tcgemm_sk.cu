// Batched-decode INT4 GEMM (M <= 64 activation rows, tiled weights) on the tensor cores as a
// persistent stream-K kernel: one CTA per SM, each owning a contiguous run of the
// (128-row tile, 256-k block) units of the weight matrix.
//
// Replaces the reference's batched kernel (orchard/kernels/gemm_int4.metal:10-68) for the
// engine's decode steps; same arithmetic as tcgemm.cu (fp16 (q - 8) * scale times fp16
// activations, fp32 accumulation in tensor memory) and the same fused epilogues (qgemm.cuh).
//
// Why persistent: a 128-row x 128-k tcgen05.mma step at N <= 64 costs ~210 ns of tensor pipe
// whatever N is, and each handshake of the dequant -> MMA -> release chain has a latency of
// several hundred ns, so a decode tile needs deep rings to stream weights at HBM speed; deep
// rings take a whole SM's tensor and shared memory, and one CTA per SM then needs balanced
// work: 172 tiles of the 7B gate/up projection on 148 SMs would leave 24 SMs with two.
// Units are dealt out evenly (CTA c takes units [c U / G, (c + 1) U / G)); in the tiled
// layout such a run is one contiguous byte range, streamed by one bulk copy per 128-k stage.
//
// Warp roles (480 threads):
//  * 0-7   dequantisation: packed stage -> fp16 A tile in a ring of tensor-memory slots
//          (tcgen05.st), one weight row per TMEM lane; warps 0-3 k 0..63, 4-7 k 64..127;
//  * 8     weight producer (one thread): 8 KB bulk copy per stage + the block's scales,
//          started before griddepcontrol.wait (weights are not written by earlier kernels);
//  * 9     activation producer (one thread): two 2-D TMA boxes per stage (SWIZZLE_128B,
//          rows past M and k past K read as zero; never multicast);
//  * 10    MMA issuer (one thread): eight tcgen05.mma.kind::f16 per stage into one of two
//          accumulators (alternating per tile), commits release the A and activation slots
//          and, at a tile's last stage, hand the accumulator to the epilogue;
//  * 11-14 epilogue: read the accumulator (tcgen05.ld), release it to the MMA, and either
//          run the fused epilogue (a tile this CTA summed alone) or store the partial sum to
//          the workspace and bump the tile's arrival counter; the CTA that arrives last
//          adds every partial of the tile in CTA order (deterministic) and runs the fused
//          epilogue, then zeroes the counter. Nobody waits on another CTA.
// Every mbarrier wait is bounded (~2 s); on expiry the CTA records device check bit 8 and
// winds down (waits give up once the failure flag is set), drains its copies and frees its
// tensor memory. The host zeroes the arrival counters when it reads that bit.
#include <algorithm>
#include <cstdlib>
#include <mutex>
#include <vector>

#include "tcgen05.cuh"

namespace orch {

constexpr int kSkCtasPerSm = 2;
constexpr int kSkDqWarps = 4;                // dequantisation warps (one TMEM lane quarter each)
constexpr int kSkWarpW = kSkDqWarps;         // weight producer
constexpr int kSkWarpX = kSkDqWarps + 1;     // activation producer
constexpr int kSkWarpMma = kSkDqWarps + 2;   // MMA issuer
constexpr int kSkWarpEpi = kSkDqWarps + 3;   // first of four epilogue warps (TMEM quarters 3, 0, 1, 2)
constexpr int kSkEpiThreads = 128;
constexpr int kSkThreads = (kSkDqWarps + 3) * 32 + kSkEpiThreads;
constexpr int kSkMaxTiles = 1 << 16;  // tiles per GEMM (N <= 8M rows)
constexpr int kSkMaxNtile = 64;
constexpr uint32_t kSkTmemCols = 256;  // half of the SM's tensor memory

// Shared and tensor memory of one CTA (two per SM). TMEM: the accumulator(s) of max(32, NTILE)
// columns (two, alternating per tile, when they fit), then three A stages of 64 columns.
template <int NTILE>
struct SkCfg {
  static constexpr uint32_t kAccCols = NTILE < 32 ? 32 : NTILE;
  static constexpr int kAccBufs = 2 * kAccCols + 3 * 64 <= kSkTmemCols ? 2 : 1;
  static constexpr int AR = (int)((kSkTmemCols - kAccBufs * kAccCols) / 64);
  static constexpr int SW = 6;                      // weight stages in flight
  static constexpr int SS = 4;                      // scale slots, one per 256-k block
  static constexpr int SX = NTILE <= 16 ? 8 : (NTILE <= 32 ? 5 : 3);
  static constexpr int XSub = NTILE * kSub * 2;     // one 64-k swizzle atom of activations
  static constexpr int XBytes = 2 * XSub;
  static constexpr int OffX = 0;
  static constexpr int OffW = OffX + SX * XBytes;
  static constexpr int OffS = OffW + SW * kWBytes;
  static constexpr int OffBar = OffS + SS * kSBytes;
  static constexpr int NBar = 2 * SW + 2 * SX + 2 * AR + 2 * kAccBufs + 1;
  static constexpr int Bytes = OffBar + NBar * 8 + 64;
  // The scale slot of block b is refilled with block b + SS, i.e. when the producer issues
  // stage 2 (b + SS), which needs stage 2 (b + SS) - SW consumed; its last reader is stage
  // 2 b + 1, so SW <= 2 SS - 1 keeps it live.
  static_assert(SW <= 2 * SS - 1, "scale ring reuse");
  static_assert(AR >= 3, "A ring");
  static_assert(XSub % 1024 == 0, "swizzle atoms are 1024-byte aligned");
  static_assert(kSkCtasPerSm * (Bytes + 1024 + 1024) <= 228 * 1024, "shared memory per SM");
};

struct SkWork {
  float* part;  // partial accumulators [2 G][NTILE][128]: slot 2c = CTA c's first tile, 2c + 1 its last
  int U;        // units = tiles x 256-k blocks
  int nblk;     // 256-k blocks per tile
};

__device__ __forceinline__ int sk_start(int c, int U, int G) { return (int)(((long long)c * U) / G); }
// The CTA whose unit range holds unit u (largest c with sk_start(c) <= u).
__device__ __forceinline__ int sk_cta_of(int u, int U, int G) { return (int)(((long long)(u + 1) * G - 1) / U); }

template <int EPI, int NTILE>
__global__ void __launch_bounds__(kSkThreads, kSkCtasPerSm)
    tc_sk_kernel(const __grid_constant__ CUtensorMap tmx, const QArgs a, const SkWork wk) {
  using C = SkCfg<NTILE>;
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
  uint64_t* accfull = aempty + C::AR;
  uint64_t* accempty = accfull + C::kAccBufs;
  uint64_t* done = accempty + C::kAccBufs;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
  volatile int* failed = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int G = gridDim.x, c = blockIdx.x;
  const int U = wk.U, nblk = wk.nblk;
  const int u0 = sk_start(c, U, G), u1 = sk_start(c + 1, U, G);  // u1 > u0: the host keeps G <= U
  const int nst = 2 * (u1 - u0);
  const int tile0 = u0 / nblk;
  const int nseg = (u1 - 1) / nblk - tile0 + 1;

  if (warp == 0) tmem_alloc(tmem_slot, kSkTmemCols);
  if (tid == 0) {
    for (int i = 0; i < C::SW; ++i) {
      mbar_init(&fullW[i], 1);
      mbar_init(&emptyW[i], kSkDqWarps);
    }
    for (int i = 0; i < C::SX; ++i) {
      mbar_init(&fullX[i], 1);
      mbar_init(&emptyX[i], 1);
    }
    for (int i = 0; i < C::AR; ++i) {
      mbar_init(&afull[i], kSkDqWarps);
      mbar_init(&aempty[i], 1);
    }
    for (int i = 0; i < C::kAccBufs; ++i) {
      mbar_init(&accfull[i], 1);
      mbar_init(&accempty[i], kSkEpiThreads / 32);
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
  const uint32_t tmem = *tmem_slot;
  const uint32_t tmem_a = tmem + C::kAccBufs * C::kAccCols;  // A ring slot i at columns 64 i

  if (warp == kSkWarpW) {
    // ------------- weight producer: one contiguous run of blocks, SW stages ahead -------------
    if (lane == 0) {
      const uint8_t* base = a.w + (size_t)u0 * kQ4tBlockBytes;
      int issued = 0;
      for (int p = 0; p < nst && !*failed; ++p) {
        const int v = p % C::SW;
        if (p >= C::SW && !mbar_wait_f(&emptyW[v], (uint32_t)(p / C::SW - 1) & 1, failed)) {
          *failed = 1;
          break;
        }
        const bool with_s = (p & 1) == 0;
        mbar_expect_tx(&fullW[v], (uint32_t)(kWBytes + (with_s ? kSBytes : 0)));
        const uint8_t* blk = base + (size_t)(p >> 1) * kQ4tBlockBytes;
        bulk_load(sW + v * kWBytes, blk + (p & 1) * kWBytes, kWBytes, &fullW[v]);
        if (with_s) bulk_load(sS + ((p >> 1) % C::SS) * kSBytes, blk + 4 * kQ4tStageBytes, kSBytes, &fullW[v]);
        issued = p + 1;
      }
      if (*failed)
        for (int p = max(0, issued - C::SW); p < issued; ++p) mbar_wait(&fullW[p % C::SW], (uint32_t)(p / C::SW) & 1);
    }
    __syncwarp();
  } else if (warp == kSkWarpX) {
    // ------------- activation producer: [NTILE, 128] tiles (two TMA boxes), SX stages ahead -------------
    pdl_wait();  // activations come from the previous kernel
    if (lane == 0) {
      int issued = 0;
      for (int p = 0; p < nst && !*failed; ++p) {
        const int v = p % C::SX;
        if (p >= C::SX && !mbar_wait_f(&emptyX[v], (uint32_t)(p / C::SX - 1) & 1, failed)) {
          *failed = 1;
          break;
        }
        mbar_expect_tx(&fullX[v], (uint32_t)C::XBytes);
        const int k0 = (((u0 + (p >> 1)) % nblk) * 2 + (p & 1)) * kTcBK;
        tma_load_2d(sX + v * C::XBytes, &tmx, &fullX[v], k0, 0);
        tma_load_2d(sX + v * C::XBytes + C::XSub, &tmx, &fullX[v], k0 + kSub, 0);
        issued = p + 1;
      }
      if (*failed)
        for (int p = max(0, issued - C::SX); p < issued; ++p) mbar_wait(&fullX[p % C::SX], (uint32_t)(p / C::SX) & 1);
    }
    __syncwarp();
  } else if (warp == kSkWarpMma) {
    // ------------- MMA issuer: A from tensor memory, activations from shared memory -------------
    if (lane == 0) {
      int seg = 0, seg_begin = 0;
      int seg_end = 2 * (min(u1, (tile0 + 1) * nblk) - u0);
      for (int p = 0; p < nst && !*failed; ++p) {
        const int ab = seg % C::kAccBufs;
        if (p == seg_begin && seg >= C::kAccBufs &&
            !mbar_wait_f(&accempty[ab], (uint32_t)(seg / C::kAccBufs - 1) & 1, failed)) {
          *failed = 1;
          break;
        }
        const int v = p % C::SX, ai = p % C::AR;
        if (!mbar_wait_f(&fullX[v], (uint32_t)(p / C::SX) & 1, failed) ||
            !mbar_wait_f(&afull[ai], (uint32_t)(p / C::AR) & 1, failed)) {
          *failed = 1;
          break;
        }
        tc_fence_after();
        const uint32_t td = tmem + (uint32_t)ab * C::kAccCols;
        const uint32_t ta = tmem_a + (uint32_t)ai * 64;
        const uint64_t bd0 = sw128_desc(smem_u32(sX + v * C::XBytes));
        const uint64_t bd1 = sw128_desc(smem_u32(sX + v * C::XBytes + C::XSub));
        const uint32_t acc0 = p > seg_begin ? 1u : 0u;
#pragma unroll
        for (int kk = 0; kk < kTcBK / 16; ++kk)
          umma_f16_ta(td, ta + kk * 8, (kk < 4 ? bd0 : bd1) + 2 * (kk & 3), kIdesc, kk > 0 ? 1u : acc0);
        umma_commit(&emptyX[v]);
        umma_commit(&aempty[ai]);
        if (p + 1 == seg_end) {
          umma_commit(&accfull[ab]);
          ++seg;
          seg_begin = seg_end;
          seg_end = 2 * (min(u1, (tile0 + seg + 1) * nblk) - u0);
        }
      }
      umma_commit(done);  // completes once every MMA issued above has
    }
    __syncwarp();
  } else if (warp < kSkDqWarps) {
    // ------- dequantisation warps: packed stage -> fp16 A tile in tensor memory -------
    // Warp w: weight rows (TMEM lanes) 32 w .. + 31, all 128 k of the stage.
    const int r = warp * 32 + lane;
    const uint32_t lane_base = (uint32_t)(warp * 32) << 16;
    for (int s = 0; s < nst; ++s) {
      const int v = s % C::SW, ai = s % C::AR;
      bool ok = mbar_wait_f(&fullW[v], (uint32_t)(s / C::SW) & 1, failed);
      if (ok && s >= C::AR) ok = mbar_wait_f(&aempty[ai], (uint32_t)(s / C::AR - 1) & 1, failed);
      if (!__all_sync(0xffffffffu, ok)) {
        *failed = 1;
        break;
      }
      // two 64-k stages [2 halves of 32 k][128 rows][16 B]; scales [8 groups][128 rows]
      const uint8_t* wt = sW + v * kWBytes;
      const __half* st = reinterpret_cast<const __half*>(sS + ((s >> 1) % C::SS) * kSBytes);
      const int g0 = (s & 1) * 4;  // scale group of the stage's first 32 k in the block
      uint4 w4[4];
      uint32_t sc[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        w4[i] = *reinterpret_cast<const uint4*>(wt + (i >> 1) * kQ4tStageBytes + (i & 1) * (kQ4tStageBytes / 2) + r * 16);
        sc[i] = h2_bits(__half2half2(st[(g0 + i) * kTcRows + r]));
      }
      fence_proxy_async();  // generic reads of the slot before its async-proxy (bulk copy) refill
      __syncwarp();
      if (lane == 0) mbar_arrive(&emptyW[v]);  // the packed slot is in registers now
#pragma unroll
      for (int j2 = 0; j2 < 2; ++j2) {
        const uint32_t wv[8] = {w4[2 * j2].x, w4[2 * j2].y, w4[2 * j2].z, w4[2 * j2].w,
                                w4[2 * j2 + 1].x, w4[2 * j2 + 1].y, w4[2 * j2 + 1].z, w4[2 * j2 + 1].w};
        uint32_t q[32];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const uint4 o = dq8_tiled(wv[i], sc[2 * j2 + (i >> 2)]);
          q[4 * i] = o.x;
          q[4 * i + 1] = o.y;
          q[4 * i + 2] = o.z;
          q[4 * i + 3] = o.w;
        }
        tmem_st32(tmem_a + lane_base + ai * 64 + j2 * 32, q);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&afull[ai]);
    }
  } else {
    // ---------------- epilogue warps: one tile (segment) at a time ----------------
    pdl_wait();  // outputs, the residual and the workspace are shared with earlier kernels
    const int quarter = warp & 3;  // TMEM lanes 32 quarter .. + 31
    const int rl = quarter * 32 + lane;
    const int Mp = epi_mp(a.M);
    for (int j = 0; j < nseg; ++j) {
      const int t = tile0 + j;
      const int ab = j % C::kAccBufs;
      const bool ok =
          __all_sync(0xffffffffu, mbar_wait_f(&accfull[ab], (uint32_t)(j / C::kAccBufs) & 1, failed));
      if (!ok) *failed = 1;
      const int ca = sk_cta_of(t * nblk, U, G), cb = sk_cta_of((t + 1) * nblk - 1, U, G);
      // a tile this CTA summed alone: the fused epilogue, 16 activation rows at a time; a
      // split tile: its partial sum to this CTA's slot (row index fastest: coalesced), for
      // sk_fixup_kernel
      float* mine = wk.part + (size_t)(2 * c + (t == tile0 ? 0 : 1)) * NTILE * kTcRows;
      if (ok) {
        tc_fence_after();
#pragma unroll 1
        for (int cc = 0; cc < Mp; cc += 16) {
          uint32_t rr[16];
          tmem_ld16(tmem + (uint32_t)ab * C::kAccCols + ((uint32_t)(32 * quarter) << 16) + (uint32_t)cc, rr);
          if (ca == cb) {
            float v[16];
#pragma unroll
            for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(rr[i]);
            tc_epilogue16<EPI>(a, t * kTcRows, quarter, lane, v, cc);
          } else {
#pragma unroll
            for (int i = 0; i < 16; ++i)
              if (cc + i < Mp) __stcg(mine + (cc + i) * kTcRows + rl, __uint_as_float(rr[i]));
          }
        }
        tc_fence_before();
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&accempty[ab]);  // the MMA may overwrite this accumulator
    }
  }

  const bool done_ok = mbar_wait(done, 0);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 0) tmem_dealloc(tmem, kSkTmemCols);
  if (tid == 0 && (*failed || !done_ok)) atomicOr(a.check, 256u);
}

// Split tiles: one thread per (activation row n, epilogue item) of a tile; the partials of
// the tile's CTAs are added in CTA order (deterministic) and the item gets the fused epilogue
// (epi_apply). Items are weight rows (STORE / RESID), SwiGLU outputs (gate row 32b + i, up
// row 32b + 16 + i) or RoPE pairs (rows 2p, 2p + 1). blockIdx.x = tile, blockIdx.y = a block
// of 256 (item, n); up to eight partials' loads are in flight per thread. Tiles one CTA
// summed alone are skipped (the GEMM kernel ran their epilogue).
template <int EPI, int NTILE>
__global__ void __launch_bounds__(256) sk_fixup_kernel(const QArgs a, const SkWork wk, int G) {
  pdl_wait();  // the GEMM kernel's partials
  pdl_trigger();
  const int t = blockIdx.x;
  const int U = wk.U, nblk = wk.nblk;
  const int ca = sk_cta_of(t * nblk, U, G), cb = sk_cta_of((t + 1) * nblk - 1, U, G);
  if (ca == cb) return;
  constexpr int E = epi_elems<EPI>();
  constexpr int IR = kTcRows / E;
  const int id = blockIdx.y * 256 + threadIdx.x;  // item + IR n
  if (id >= IR * a.M) return;
  const int item = id % IR, n = id / IR;
  const int r0 = E == 1 ? item : (EPI == EPI_SWIGLU ? (item >> 4) * 32 + (item & 15) : 2 * item);
  const int r1 = EPI == EPI_SWIGLU ? r0 + 16 : r0 + 1;
  float v0 = 0.f, v1 = 0.f;
  for (int c0 = ca; c0 <= cb; c0 += 8) {
    float p0[8], p1[8];
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      const int c2 = c0 + q;
      const bool live = c2 <= cb;
      const int slot = live ? 2 * c2 + (t == sk_start(c2, U, G) / nblk ? 0 : 1) : 0;
      const float* src = wk.part + ((size_t)slot * NTILE + n) * kTcRows;
      p0[q] = live ? __ldcg(src + r0) : 0.f;
      p1[q] = live && E == 2 ? __ldcg(src + r1) : 0.f;
    }
#pragma unroll
    for (int q = 0; q < 8; ++q)
      if (c0 + q <= cb) {
        v0 += p0[q];
        v1 += p1[q];
      }
  }
  const int R0 = t * kTcRows;
  if (EPI == EPI_SWIGLU) {
    const int j = (R0 >> 1) + item;
    if (j < (a.N >> 1)) epi_apply<W_Q4, EPI>(a, n, j, v0, v1);
  } else if (R0 + r0 < a.N) {
    epi_apply<W_Q4, EPI>(a, n, R0 + r0, v0, v1);
  }
}

// ------------------------------------------------------------------------------------------
// host side
// ------------------------------------------------------------------------------------------
namespace {

// Partial sums and arrival counters, one set per (device, stream): kernels on one stream run
// in order (and the epilogue touches the workspace only after griddepcontrol.wait), so calls
// on different streams never share one. Each device gets a pool of kSkPool sets when its
// state is created (so that a stream's first call may come inside a graph capture); more
// are allocated outside capture on demand. ~10 MB + 256 KB per set, kept for the process.
constexpr int kSkPool = 3;
struct SkWorkspace {
  int dev;
  bool used;
  cudaStream_t st;
  float* part;
};
std::mutex g_sk_mu;
std::vector<SkWorkspace> g_sk_ws;

bool sk_alloc(int dev, int sms, SkWorkspace* w) {
  *w = SkWorkspace{dev, false, nullptr, nullptr};
  const size_t part_bytes = (size_t)2 * kSkCtasPerSm * sms * kSkMaxNtile * kTcRows * sizeof(float);
  if (cudaMalloc(&w->part, part_bytes) != cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  return true;
}

int sk_workspace(cudaStream_t st, SkWorkspace* out) {
  const int dev = device_index();
  const int sms = num_sms();
  std::lock_guard<std::mutex> lock(g_sk_mu);
  for (const SkWorkspace& w : g_sk_ws)
    if (w.dev == dev && w.used && w.st == st) {
      *out = w;
      return ORCH_OK;
    }
  for (SkWorkspace& w : g_sk_ws)
    if (w.dev == dev && !w.used) {
      w.used = true;
      w.st = st;
      *out = w;
      return ORCH_OK;
    }
  cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
  if (cudaStreamIsCapturing(st, &cs) != cudaSuccess || cs != cudaStreamCaptureStatusNone) {
    cudaGetLastError();
    return ORCH_ERR_UNSUPPORTED;  // pool used up inside a capture: the per-tile kernel runs
  }
  SkWorkspace w;
  if (!sk_alloc(dev, sms, &w)) return ORCH_ERR_UNSUPPORTED;
  w.used = true;
  w.st = st;
  g_sk_ws.push_back(w);
  *out = w;
  return ORCH_OK;
}

// 0 never (default: in the 7B decode step the per-tile kernel measured faster overall, 9,876
// vs 9,616 tokens/s at batch 64), 1 whenever it applies, 2 when it pays (sk_pays);
// ORCHARD_TC_SK=0/1/2 sets the start.
int g_sk_mode = [] {
  const char* e = std::getenv("ORCHARD_TC_SK");
  return e ? (e[0] == '1' ? 1 : (e[0] == '2' ? 2 : 0)) : 0;
}();
int sk_mode() { return g_sk_mode; }

// The per-tile kernel runs tiles x KS CTAs, two per SM (tcgemm.cu). Between one and one and a
// half waves of SMs it leaves some SMs with two CTAs and the rest with one, and those SMs set
// the time; there the balanced stream-K split wins (7B gate/up: 172 tiles on 148 SMs,
// 36 -> 29 us at 64 rows). Elsewhere the per-tile kernel is as fast or faster (fewer, longer
// CTAs; no fix-up pass).
bool sk_pays(const QArgs& a, int sms) {
  const int tiles = (a.N + kTcRows - 1) / kTcRows;
  const int nblk = (a.K + 2 * kTcBK - 1) / (2 * kTcBK);
  int KS = 1;
  while (KS < 8 && tiles * KS * 2 <= 2 * sms && nblk >= KS * 4) KS *= 2;
  const int ctas = tiles * KS;
  return ctas > sms && 2 * ctas < 3 * sms;
}

template <int EPI, int NTILE>
int sk_launch(const CUtensorMap& mx, const QArgs& a, const SkWork& wk, int G, cudaStream_t st) {
  static bool attr_done[64] = {};
  const int dev = device_index();
  auto kern = tc_sk_kernel<EPI, NTILE>;
  const size_t smem = SkCfg<NTILE>::Bytes + 1024;
  if (dev >= 0 && dev < 64 && !attr_done[dev]) {
    ORCH_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    attr_done[dev] = true;
  }
  ORCH_CUDA(launch_k(kern, dim3(G), dim3(kSkThreads), smem, st, dim3(0, 0, 0), mx, a, wk));
  // split tiles exist unless every CTA's range is whole tiles
  bool split = false;
  for (int c = 0; c < G && !split; ++c) split = (int)(((long long)c * wk.U) / G) % wk.nblk != 0;
  if (split) {
    const int items = (kTcRows / epi_elems<EPI>()) * a.M;
    const dim3 fgrid(wk.U / wk.nblk, (items + 255) / 256);
    ORCH_CUDA(launch_k(sk_fixup_kernel<EPI, NTILE>, fgrid, dim3(256), 0, st, dim3(0, 0, 0), a, wk, G));
  }
  return ORCH_OK;
}

}  // namespace

// The pool of stream-K workspaces of device `dev` (best effort: on failure the per-tile
// kernel serves streams without one).
void sk_preallocate(int dev, int sms) {
  std::lock_guard<std::mutex> lock(g_sk_mu);
  int have = 0;
  for (const SkWorkspace& w : g_sk_ws) have += w.dev == dev;
  for (; have < kSkPool; ++have) {
    SkWorkspace w;
    if (!sk_alloc(dev, sms, &w)) return;
    g_sk_ws.push_back(w);
  }
}

template <int EPI>
int tc_sk_run(QArgs a, cudaStream_t st) {
  const int mode = sk_mode();
  if (mode == 0 || !a.tiled || a.x_f32 || a.M < 1 || a.M > kSkMaxNtile || (a.K % 8) != 0 || !encode_fn())
    return ORCH_ERR_UNSUPPORTED;
  if (mode == 2 && !sk_pays(a, num_sms())) return ORCH_ERR_UNSUPPORTED;
  if (((uintptr_t)a.x & 15) != 0 || ((uintptr_t)a.w & 15) != 0) return ORCH_ERR_UNSUPPORTED;
  const int tiles = (a.N + kTcRows - 1) / kTcRows;
  const int nblk = (a.K + 2 * kTcBK - 1) / (2 * kTcBK);
  if (tiles > kSkMaxTiles || (long long)tiles * nblk > (1LL << 30)) return ORCH_ERR_UNSUPPORTED;
  SkWorkspace ws;
  if (sk_workspace(st, &ws) != ORCH_OK) return ORCH_ERR_UNSUPPORTED;
  ORCH_CHECK_WORD(a.check);
  const int ntile = a.M <= 16 ? 16 : a.M <= 32 ? 32 : 64;
  CUtensorMap mx;
  if (!encode2d(&mx, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, a.x, (uint64_t)a.K, (uint64_t)a.M, (uint64_t)a.K * 2, kSub,
                ntile, CU_TENSOR_MAP_SWIZZLE_128B))
    return fail(ORCH_ERR_UNSUPPORTED, "tensor map encode failed");
  SkWork wk{ws.part, tiles * nblk, nblk};
  const int G = std::min(kSkCtasPerSm * num_sms(), wk.U);
  int rc;
  switch (ntile) {
    case 16: rc = sk_launch<EPI, 16>(mx, a, wk, G, st); break;
    case 32: rc = sk_launch<EPI, 32>(mx, a, wk, G, st); break;
    default: rc = sk_launch<EPI, 64>(mx, a, wk, G, st); break;
  }
  if (rc != ORCH_OK) return rc;
  return check_launch("tc_sk_qgemm");
}

template int tc_sk_run<EPI_STORE>(QArgs, cudaStream_t);
template int tc_sk_run<EPI_RESID>(QArgs, cudaStream_t);
template int tc_sk_run<EPI_SWIGLU>(QArgs, cudaStream_t);
template int tc_sk_run<EPI_QKV>(QArgs, cudaStream_t);

}  // namespace orch

extern "C" int orch_set_stream_k(int mode) {
  if (mode < 0 || mode > 2) return orch::fail(ORCH_ERR_INVALID, "stream-K mode must be 0, 1 or 2");
  orch::g_sk_mode = mode;
  return ORCH_OK;
}
