// Weight-only quantised skinny GEMM for decode: y[m, n] = sum_k W[n, k] x[m, k], M <= 64.
//
// Replaces the reference's one-thread-per-output-row Metal kernels
// (orchard/kernels/gemv_int4.metal:10-74, gemm_int4.metal:10-68, gemv_int8.metal:13-55).
//
// Design (sm_100a):
//  * The weight stream is the only large operand, so the kernel is built around reading
//    it once with 16-byte streaming loads: lane (g = lane/4, c = lane%4) of a warp loads
//    one 16-byte piece (one 32-weight INT4 group) of weight rows g and g+8 of a 16-row
//    tile per 128-k chunk; four lanes cover a row's 64-byte chunk, so every load
//    instruction reads whole 32-byte sectors.
//  * Nibbles become fp16 with the magic-exponent trick (one LOP3 per pair, exact), are
//    scaled by the group's fp16 scale, and feed mma.sync m16n8k16 directly as the A
//    operand. The reduction over k is a sum, so any fixed permutation of k applied to both
//    operands is exact; the kernel uses the permutation under which the extracted nibble
//    pairs (k, k+4) *are* the A fragment, and stages the activations in shared memory in
//    the same permuted, bank-swizzled order so each B fragment pair is one LDS.128.
//  * Activations (M <= 64 rows) are the B operand (N dimension of the MMA, 8 rows per
//    n-tile); the tensor pipe does all multiply-adds, CUDA cores only dequantise.
//  * Split-K across the CTAs of a thread-block cluster; partial tiles are reduced through
//    distributed shared memory, then the fused epilogue (store, residual add, SwiGLU,
//    RoPE + KV-cache append) runs on the full sums. No global scratch, no atomics.
#include <cooperative_groups.h>

#include <algorithm>
#include <cstdlib>

#include "qgemm.cuh"



namespace orch {

constexpr int kWarps = 4;
constexpr int kThreads = kWarps * 32;

template <int WF> struct WCfg;
template <> struct WCfg<W_Q4> { static constexpr int kPieces = 1; };   // 16 B per row per chunk per lane
template <> struct WCfg<W_Q8G> { static constexpr int kPieces = 2; };  // 32 B
template <> struct WCfg<W_Q8PC> { static constexpr int kPieces = 2; };

__device__ __forceinline__ int swz(int u) { return u ^ ((u >> 3) & 1); }

__device__ __forceinline__ uint32_t word_of(const uint4& v, int j) {
  return j == 0 ? v.x : j == 1 ? v.y : j == 2 ? v.z : v.w;
}

// Stage x[m, kbeg : kbeg + 8*nunits) into shared memory, 8 elements per 16-byte unit,
// permuted for the weight format (Q4: pairs (0,4)(1,5)(2,6)(3,7); Q8: (0,2)(1,3)(4,6)(5,7)).
template <int WF>
__device__ __forceinline__ void stage_x(uint4* sm, const QArgs& a, int kbeg, int nunits, int RS) {
  const int total = a.M * nunits;
  for (int idx = threadIdx.x; idx < total; idx += kThreads) {
    const int m = idx / nunits;
    const int u = idx - m * nunits;
    const int k = kbeg + u * 8;
    uint4 raw = make_uint4(0, 0, 0, 0);
    if (k < a.K) {
      if (a.x_f32) {
        const float4* p = reinterpret_cast<const float4*>(static_cast<const float*>(a.x) + (size_t)m * a.K + k);
        const float4 lo = __ldg(p), hi = __ldg(p + 1);
        raw.x = h2_bits(__floats2half2_rn(lo.x, lo.y));
        raw.y = h2_bits(__floats2half2_rn(lo.z, lo.w));
        raw.z = h2_bits(__floats2half2_rn(hi.x, hi.y));
        raw.w = h2_bits(__floats2half2_rn(hi.z, hi.w));
      } else {
        raw = __ldg(reinterpret_cast<const uint4*>(static_cast<const __half*>(a.x) + (size_t)m * a.K + k));
      }
    }
    uint4 o;
    if (WF == W_Q4) {
      o.x = prmt(raw.x, raw.z, 0x5410);  // (x0, x4)
      o.y = prmt(raw.x, raw.z, 0x7632);  // (x1, x5)
      o.z = prmt(raw.y, raw.w, 0x5410);  // (x2, x6)
      o.w = prmt(raw.y, raw.w, 0x7632);  // (x3, x7)
    } else {
      o.x = prmt(raw.x, raw.y, 0x5410);  // (x0, x2)
      o.y = prmt(raw.x, raw.y, 0x7632);  // (x1, x3)
      o.z = prmt(raw.z, raw.w, 0x5410);  // (x4, x6)
      o.w = prmt(raw.z, raw.w, 0x7632);  // (x5, x7)
    }
    sm[m * RS + swz(u)] = o;
  }
}

// INT4 pair extraction: nibbles (i, i+4) of a word -> fp16 (q-8) pair, scaled.
__device__ __forceinline__ uint32_t dq4_lo(uint32_t w, uint32_t sc) {
  const __half2 v = bits_h2(lop3_and_or(w, 0x000F000Fu, 0x64006400u));
  return h2_bits(__hmul2(__hsub2(v, bits_h2(0x64086408u)), bits_h2(sc)));
}
__device__ __forceinline__ uint32_t dq4_hi(uint32_t w, uint32_t sc) {
  const __half2 v = bits_h2(lop3_and_or(w, 0x00F000F0u, 0x64006400u));
  return h2_bits(__hmul2(__hfma2(v, bits_h2(0x2C002C00u), bits_h2(0xD480D480u)), bits_h2(sc)));
}
// INT8 pair extraction: bytes (0,2) or (1,3) of a word -> fp16 pair (exact).
__device__ __forceinline__ uint32_t dq8(uint32_t wx, uint32_t sel) {
  const __half2 v = bits_h2(prmt(wx, 0x64646464u, sel));
  return h2_bits(__hsub2(v, bits_h2(0x64806480u)));
}

template <int WF, int NT, int MT, int EPI>
__global__ void __launch_bounds__(kThreads) qgemm_kernel(const QArgs a) {
  extern __shared__ __align__(16) uint4 sm[];
  constexpr int ROWS = kWarps * 16 * MT;
  constexpr int P = WCfg<WF>::kPieces;
  // chunks per load batch; two batches are in flight (ping-pong registers)
  constexpr int U = (NT >= 8) ? 1 : ((MT * P >= 4) ? 1 : (MT * P == 2 ? 2 : 4));

  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int g = lane >> 2, c = lane & 3;
  const int KS = gridDim.y, ks = blockIdx.y;
  const int c0 = (ks * a.nchunk) / KS, c1 = ((ks + 1) * a.nchunk) / KS;
  const int nunits = (c1 - c0) * 16;
  const int RS = nunits + 2;

  const int R0 = blockIdx.x * ROWS;
  const int rowbase = R0 + warp * 16 * MT;
  const int G = a.K >> 5;  // 32-k groups
  const size_t rowbytes = (WF == W_Q4) ? (size_t)(a.K >> 1) : (size_t)a.K;

  float acc[MT][NT][4];
#pragma unroll
  for (int i = 0; i < MT; ++i)
#pragma unroll
    for (int j = 0; j < NT; ++j)
#pragma unroll
      for (int e = 0; e < 4; ++e) acc[i][j][e] = 0.f;

  uint4 wa[U][MT][2][P], wb[U][MT][2][P];
  uint32_t sa[U][MT][2], sb[U][MT][2];

  // Weight stream of chunks [ch, ch + U) into registers (independent of the activations).
  auto load = [&](int ch, uint4 (&wv)[U][MT][2][P], uint32_t (&sc)[U][MT][2]) {
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int grp = (ch + u) * 4 + c;
      const bool okk = (ch + u < c1) && (grp < G);
#pragma unroll
      for (int mt = 0; mt < MT; ++mt) {
#pragma unroll
        for (int hr = 0; hr < 2; ++hr) {
          const int r = rowbase + mt * 16 + g + hr * 8;
          const bool ok = okk && (r < a.N);
          const uint8_t* p = a.w + (size_t)r * rowbytes + (size_t)grp * 16 * P;
#pragma unroll
          for (int pc = 0; pc < P; ++pc) {
            const uint32_t fill = (WF == W_Q4) ? 0x88888888u : 0u;
            wv[u][mt][hr][pc] = ok ? ld_stream16(p + 16 * pc) : make_uint4(fill, fill, fill, fill);
          }
          if (WF != W_Q8PC) {
            const __half s = ok ? a.s[(size_t)r * G + grp] : __float2half(0.f);
            sc[u][mt][hr] = h2_bits(__half2half2(s));
          } else {
            sc[u][mt][hr] = 0;
          }
        }
      }
    }
  };

  auto compute = [&](int ch, const uint4 (&wv)[U][MT][2][P], const uint32_t (&sc)[U][MT][2]) {
#pragma unroll
    for (int u = 0; u < U; ++u) {
      if (ch + u >= c1) break;
      const int ubase = (ch + u - c0) * 16 + 4 * c;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int us = swz(ubase + j);
        uint4 bf[NT];
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
          const int n = nt * 8 + g;
          bf[nt] = (n < a.M) ? sm[n * RS + us] : make_uint4(0, 0, 0, 0);
        }
#pragma unroll
        for (int mt = 0; mt < MT; ++mt) {
          if (WF == W_Q4) {
            uint32_t w0 = word_of(wv[u][mt][0][0], j), w1 = word_of(wv[u][mt][1][0], j);
            const uint32_t s0 = sc[u][mt][0], s1 = sc[u][mt][1];
            {
              const uint32_t a0 = dq4_lo(w0, s0), a1 = dq4_lo(w1, s1);
              const uint32_t a2 = dq4_hi(w0, s0), a3 = dq4_hi(w1, s1);
#pragma unroll
              for (int nt = 0; nt < NT; ++nt) mma_16816(acc[mt][nt], a0, a1, a2, a3, bf[nt].x, bf[nt].y);
            }
            w0 >>= 8;
            w1 >>= 8;
            {
              const uint32_t a0 = dq4_lo(w0, s0), a1 = dq4_lo(w1, s1);
              const uint32_t a2 = dq4_hi(w0, s0), a3 = dq4_hi(w1, s1);
#pragma unroll
              for (int nt = 0; nt < NT; ++nt) mma_16816(acc[mt][nt], a0, a1, a2, a3, bf[nt].z, bf[nt].w);
            }
          } else {
            // unit j covers words 2j, 2j+1 of the 32-byte (8-word) per-lane span
#pragma unroll
            for (int hw = 0; hw < 2; ++hw) {
              const int wi = 2 * j + hw;
              const uint32_t w0 = word_of(wv[u][mt][0][wi >> 2], wi & 3) ^ 0x80808080u;
              const uint32_t w1 = word_of(wv[u][mt][1][wi >> 2], wi & 3) ^ 0x80808080u;
              uint32_t a0 = dq8(w0, 0x4240), a1 = dq8(w1, 0x4240);
              uint32_t a2 = dq8(w0, 0x4341), a3 = dq8(w1, 0x4341);
              if (WF == W_Q8G) {
                const __half2 s0 = bits_h2(sc[u][mt][0]), s1 = bits_h2(sc[u][mt][1]);
                a0 = h2_bits(__hmul2(bits_h2(a0), s0));
                a2 = h2_bits(__hmul2(bits_h2(a2), s0));
                a1 = h2_bits(__hmul2(bits_h2(a1), s1));
                a3 = h2_bits(__hmul2(bits_h2(a3), s1));
              }
#pragma unroll
              for (int nt = 0; nt < NT; ++nt) {
                const uint32_t b0 = hw ? bf[nt].z : bf[nt].x;
                const uint32_t b1 = hw ? bf[nt].w : bf[nt].y;
                mma_16816(acc[mt][nt], a0, a1, a2, a3, b0, b1);
              }
            }
          }
        }
      }
    }
  };

  // Prologue: the first weight batch is requested before waiting on the previous kernel,
  // so it streams while that kernel finishes.
  load(c0, wa, sa);
  pdl_trigger();
  pdl_wait();
  stage_x<WF>(sm, a, c0 * 128, nunits, RS);
  __syncthreads();

  for (int ch = c0; ch < c1; ch += 2 * U) {
    load(ch + U, wb, sb);
    compute(ch, wa, sa);
    load(ch + 2 * U, wa, sa);
    compute(ch + U, wb, sb);
  }

  // ---- partials -> owners' receive buffers (they alias the staged activations) ----------
  cg::cluster_group cl = cg::this_cluster();
  cl.sync();
  float* recv = reinterpret_cast<float*>(sm);
  const int Mp = epi_mp(a.M);
#pragma unroll
  for (int mt = 0; mt < MT; ++mt) {
    const int rl = warp * 16 * MT + mt * 16 + g;
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      const int n0 = nt * 8 + 2 * c;
      if (n0 < Mp) {  // Mp is a multiple of 4, so n0 + 1 < Mp too
        const int pitch = epi_pitch<EPI, ROWS>(KS);
        float* d0 = epi_dest<EPI, ROWS>(cl, recv, Mp, KS, ks, rl, n0);
        float* d1 = epi_dest<EPI, ROWS>(cl, recv, Mp, KS, ks, rl + 8, n0);
        d0[0] = acc[mt][nt][0];
        d0[pitch] = acc[mt][nt][1];
        d1[0] = acc[mt][nt][2];
        d1[pitch] = acc[mt][nt][3];
      }
    }
  }
  qgemm_finish<WF, EPI, ROWS>(a, recv, KS, ks, R0);
}

// ------------------------------------------------------------------------------------
// host launcher
// ------------------------------------------------------------------------------------
namespace {

constexpr int kSmemBudget = 110 * 1024;  // two CTAs per SM
constexpr int kSmemMax = 200 * 1024;     // one CTA per SM

template <int WF, int NT, int MT, int EPI>
int launch_cfg(QArgs a, int KS, size_t smem, cudaStream_t st) {
  static bool attr_done[64] = {};
  const int dev = device_index();
  auto kern = qgemm_kernel<WF, NT, MT, EPI>;
  if (dev >= 0 && dev < 64 && !attr_done[dev]) {
    ORCH_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 210 * 1024));
    attr_done[dev] = true;
  }
  constexpr int ROWS = kWarps * 16 * MT;
  ORCH_CUDA(launch_k(kern, dim3((a.N + ROWS - 1) / ROWS, KS, 1), dim3(kThreads, 1, 1), smem, st,
                     dim3(1, KS, 1), a));
  return ORCH_OK;
}

template <int WF, int EPI>
int dispatch_nt(const QArgs& a, int KS, size_t smem, cudaStream_t st) {
  const int nt = (a.M + 7) / 8;
  if (nt <= 1) return launch_cfg<WF, 1, 1, EPI>(a, KS, smem, st);
  if (nt <= 2) return launch_cfg<WF, 2, 1, EPI>(a, KS, smem, st);
  if (nt <= 4) return launch_cfg<WF, 4, 1, EPI>(a, KS, smem, st);
  return launch_cfg<WF, 8, 2, EPI>(a, KS, smem, st);
}

int rows_per_cta(int M) { return (M > 32) ? 128 : 64; }

// CTAs per SM the cluster K-split aims for (more resident warps keep more weight bytes in
// flight); ORCHARD_QGEMM_CTAS_PER_SM overrides.
int ks_target() {
  static const int v = [] {
    const char* e = std::getenv("ORCHARD_QGEMM_CTAS_PER_SM");
    return e ? std::max(1, std::atoi(e)) : 2;
  }();
  return v;
}

}  // namespace

// Rows up to which tiled INT4 GEMMs take the mma.sync GEMV (gemv.cu); ORCHARD_GEMV_MAX_M
// overrides (0: always the tensor-core kernel).
uint32_t gemv_tiled_limit() {
  static const uint32_t v = [] {
    const char* e = std::getenv("ORCHARD_GEMV_MAX_M");
    return e ? (uint32_t)std::max(0, std::atoi(e)) : gemv_max_m();
  }();
  return std::min(v, gemv_max_m());
}

// Splits M into blocks of <= 64 rows that fit shared memory, picks the cluster K-split,
// and launches. `advance` moves the per-row pointers of an args block by `m` rows.
template <int WF, int EPI>
int qgemm_run(QArgs a, cudaStream_t st) {
  if (a.M <= 0 || a.N <= 0) return ORCH_OK;
  if (a.K <= 0 || (a.K % 32) != 0) return fail(ORCH_ERR_UNSUPPORTED, "K must be a positive multiple of 32");
  if (a.tiled) {  // tiled INT4 weights: GEMV kernel for a few rows, tensor-core kernel above
    if (WF != W_Q4) return fail(ORCH_ERR_INVALID, "tiled weights are INT4 only");
    if (!a.x_f32 && a.M <= (int)gemv_tiled_limit()) {
      const int rc = gemv_tiled_run<EPI>(a, st);
      if (rc != ORCH_ERR_UNSUPPORTED) return rc;
    }
    const int rc = tc_qgemm_run<EPI>(a, st);
    if (rc == ORCH_ERR_UNSUPPORTED)
      return fail(ORCH_ERR_UNSUPPORTED, "tiled INT4 GEMM: needs fp16 activations and 16-byte aligned buffers");
    return rc;
  }
  if (WF == W_Q4 && !a.x_f32 && tc_min_m() > 0 && a.M >= (int)tc_min_m()) {
    const int rc = tc_qgemm_run<EPI>(a, st);
    if (rc != ORCH_ERR_UNSUPPORTED) return rc;
  }
  a.nchunk = (a.K + 127) / 128;
  ORCH_CHECK_WORD(a.check);
  const int total_M = a.M;
  int m0 = 0;
  while (m0 < total_M) {
    QArgs b = a;
    int mb = std::min(64, total_M - m0);
    const int rows = rows_per_cta(mb);
    const int tiles = (a.N + rows - 1) / rows;
    const int target = ks_target() * num_sms();
    int KS = 1;
    while (KS < 8 && tiles * KS < target && a.nchunk >= 4 * KS) KS *= 2;
    auto xbytes = [&](int ks, int m) {
      const int nunits = ((a.nchunk + ks - 1) / ks) * 16;
      return (size_t)m * (nunits + 2) * 16;
    };
    while (KS < 8 && xbytes(KS, mb) > (size_t)kSmemBudget && a.nchunk >= 2 * KS) KS *= 2;
    // a larger shared-memory slice (fewer CTAs per SM) beats splitting M, which re-reads weights
    while (mb > 8 && xbytes(KS, mb) > (size_t)kSmemMax) mb = (mb + 1) / 2;
    if (xbytes(KS, mb) > (size_t)kSmemMax) return fail(ORCH_ERR_UNSUPPORTED, "K too large for the decode GEMM");
    const size_t redb = (size_t)4 * (rows_per_cta(mb) == 128 ? epi_recv_floats<128>(mb) : epi_recv_floats<64>(mb));
    const size_t smem = std::max(xbytes(KS, mb), redb);
    b.M = mb;
    // advance per-row pointers
    const size_t xs = a.x_f32 ? 4 : 2;
    b.x = static_cast<const char*>(a.x) + (size_t)m0 * a.K * xs;
    constexpr int LR = EPI == EPI_QKV ? 3 : (EPI == EPI_SWIGLU ? 2 : 1);
    if (a.lora_t) b.lora_t = a.lora_t + (size_t)m0 * LR * a.lora_r;
    if (EPI == EPI_STORE || EPI == EPI_RESID) {
      const size_t os = (EPI == EPI_RESID || a.out_f32) ? 4 : 2;
      b.out = static_cast<char*>(a.out) + (size_t)m0 * a.ldo * os;
    } else if (EPI == EPI_SWIGLU) {
      b.out = static_cast<__half*>(a.out) + (size_t)m0 * (a.N >> 1);
    } else {
      b.out = static_cast<__half*>(a.out) + (size_t)m0 * a.H;
      b.pos = a.pos + m0;
      if (a.slots) b.slots = a.slots + m0;
      else b.slot0 = a.slot0 + m0;
    }
    const int rc = dispatch_nt<WF, EPI>(b, KS, smem, st);
    if (rc != ORCH_OK) return rc;
    m0 += mb;
  }
  return check_launch("qgemm");
}

template int qgemm_run<W_Q4, EPI_STORE>(QArgs, cudaStream_t);
template int qgemm_run<W_Q4, EPI_RESID>(QArgs, cudaStream_t);
template int qgemm_run<W_Q4, EPI_SWIGLU>(QArgs, cudaStream_t);
template int qgemm_run<W_Q4, EPI_QKV>(QArgs, cudaStream_t);
template int qgemm_run<W_Q8G, EPI_STORE>(QArgs, cudaStream_t);
template int qgemm_run<W_Q8PC, EPI_STORE>(QArgs, cudaStream_t);

}  // namespace orch
