// Arguments of the quantised skinny-GEMM kernel family (qgemm.cu).
#pragma once

#include <cooperative_groups.h>

#include "orch_common.cuh"

namespace orch {

enum { W_Q4 = 0, W_Q8G = 1, W_Q8PC = 2 };
enum { EPI_STORE = 0, EPI_RESID = 1, EPI_SWIGLU = 2, EPI_QKV = 3 };

// Tiled INT4 weight layout: the engine's device copy of a packed [N, K/2] + [N, K/32]
// weight, re-laid once at load so that the tensor-core GEMM streams every CTA's weights
// as one contiguous run (row-major rows read 32 bytes at a time leave HBM activation-bound).
// Rows come in tiles of 128, k in blocks of 256 (N and K are padded with zero weights:
// nibble 8, scale 0). Block (tile t, block b) sits at byte (t * nblk + b) * kQ4tBlockBytes:
//   4 stages of 64 k, each [2 halves of 32 k][128 rows][16 bytes];
//   then the block's scales [8 groups][128 rows] fp16.
// Inside each 32-bit word the nibbles of k0..k7 are stored in the order
// k0 k2 k4 k6 k1 k3 k5 k7 (low nibble first), so the magic-exponent extraction yields
// (k0,k1) (k2,k3) (k4,k5) (k6,k7) pairs directly.
constexpr int kQ4tRows = 128;
constexpr int kQ4tBlockK = 256;
constexpr int kQ4tStageBytes = 4096;
constexpr int kQ4tScaleBytes = 2048;
constexpr int kQ4tBlockBytes = 4 * kQ4tStageBytes + kQ4tScaleBytes;
inline size_t q4t_bytes(uint32_t N, uint32_t K) {
  return (size_t)((N + kQ4tRows - 1) / kQ4tRows) * ((K + kQ4tBlockK - 1) / kQ4tBlockK) * kQ4tBlockBytes;
}

struct QArgs {
  const uint8_t* w;   // packed weights [N, K/2] (INT4) or [N, K] (INT8)
  const __half* s;    // scales [N, K/32] or [N] (per channel)
  const void* x;      // activations [M, K], fp16 or fp32
  int x_f32;
  int M, N, K;
  int nchunk;         // ceil(K / 128), set by the launcher
  // STORE / RESID / SWIGLU / QKV(q) output
  void* out;
  int out_f32;
  int ldo;
  // QKV + RoPE + KV append
  int H, nh, hd, max_seq, max_pos;
  uint32_t hd_magic;  // ceil(2^32 / hd): rr / hd = umulhi(rr, hd_magic) for rr, hd < 2^16
  const int* pos;
  const int* slots;   // cache slot of each row; null: row index (slot0 + local row)
  int slot0;          // with null slots, the first row's index (row blocks advance it)
  int num_slots;      // slots in the caches: a row whose slot is outside [0, num_slots) is skipped
  const float* cos_tab;
  const float* sin_tab;
  __half* kc;
  __half* vc;
  const float* lora_t;
  const float* lora_b;
  int lora_r;
  uint32_t* check;
  int tiled;          // w is in the tiled INT4 layout (s unused); tensor-core path only
  // RMSNorm prologue (GEMV for M <= 8 only): x is the fp32 residual [M, K]; the kernel uses
  // fp16(x * rsqrt(sum(x^2) / K + norm_eps) * norm_w) as its activations
  const float* norm_w;
  float norm_eps;
};

template <int WF, int EPI>
int qgemm_run(QArgs a, cudaStream_t st);

// Tensor-core (tcgen05) path for INT4, M >= 16; returns ORCH_ERR_UNSUPPORTED when the
// shape is outside what it implements.
template <int EPI>
int tc_qgemm_run(QArgs a, cudaStream_t st);
// Persistent stream-K tensor-core path for tiled INT4 weights and M <= 64 (tcgemm_sk.cu);
// ORCH_ERR_UNSUPPORTED when it does not apply.
template <int EPI>
int tc_sk_run(QArgs a, cudaStream_t st);
// Allocates device `dev`'s pool of stream-K workspaces (called once per device).
void sk_preallocate(int dev, int sms);
// Activation-row count from which INT4 GEMMs take the tensor-core path (0 = never).
uint32_t tc_min_m();
// mma.sync GEMV on tiled weights for M <= gemv_max_m() (gemv.cu).
template <int EPI>
int gemv_tiled_run(QArgs a, cudaStream_t st);
uint32_t gemv_max_m();
// Rows up to which tiled INT4 GEMMs take that GEMV (ORCHARD_GEMV_MAX_M may lower it).
uint32_t gemv_tiled_limit();

namespace cg = cooperative_groups;

// LoRA term of output column `col` of region `reg` (R regions of width `width`):
// sum_q t[n, reg, q] * B[reg, q, col].
template <int R>
__device__ __forceinline__ float lora_delta_r(const QArgs& a, int n, int reg, int col, int width) {
  const float* t = a.lora_t + ((size_t)n * R + reg) * a.lora_r;
  const float* bm = a.lora_b + (size_t)reg * a.lora_r * width + col;
  float v = 0.f;
  for (int q = 0; q < a.lora_r; ++q) v = fmaf(t[q], bm[(size_t)q * width], v);
  return v;
}

// ---- split-K reduce-scatter over the cluster and the fused epilogue ----------------------
// An epilogue item row is one weight row (STORE/RESID), a rotation pair of rows 2p, 2p+1
// (QKV) or the gate and up rows of one output (SWIGLU, rows 32b+i and 32b+16+i). The ROWS/E
// item rows of a tile are owned in equal contiguous blocks of IRL = ROWS/E/KS by the KS
// CTAs of the cluster. Each CTA pushes its partial sums into the owners' receive buffers
// with distributed-shared-memory stores (no remote loads); after one cluster barrier every
// owner sums its KS slices locally and runs the epilogue, consecutive threads on
// consecutive rows. Receive buffer of an owner: [src][e][n][irl] floats, the row index
// fastest with a pitch of IRL + 1 per activation row n (n < Mp, M rounded up to 4), so the
// owner's sum loop and a warp pushing 32 consecutive rows of one n touch 32 consecutive
// words (no bank conflicts). Size Mp * (ROWS + E * KS) floats <= Mp * (ROWS + 16).
template <int EPI>
__host__ __device__ constexpr int epi_elems() { return (EPI == EPI_QKV || EPI == EPI_SWIGLU) ? 2 : 1; }

__host__ __device__ __forceinline__ int epi_mp(int M) { return (M + 3) & ~3; }

template <int ROWS>
__host__ __device__ __forceinline__ int epi_recv_floats(int M) { return (ROWS + 16) * epi_mp(M); }

template <int EPI>
__device__ __forceinline__ int epi_item_row(int rl, int& e) {
  if (EPI == EPI_QKV) {
    e = rl & 1;
    return rl >> 1;
  }
  if (EPI == EPI_SWIGLU) {
    const int w = rl & 31;
    e = w >> 4;
    return (rl >> 5) * 16 + (w & 15);
  }
  e = 0;
  return rl;
}

// Distance in floats between the partials of activation rows n and n + 1.
template <int EPI, int ROWS>
__device__ __forceinline__ int epi_pitch(int KS) { return ROWS / epi_elems<EPI>() / KS + 1; }

// Destination of the partial sum of tile row `rl` for activation row n; the partial of row
// n + j goes to the returned pointer + j * epi_pitch.
template <int EPI, int ROWS>
__device__ __forceinline__ float* epi_dest(cg::cluster_group& cl, float* recv, int Mp, int KS, int ks, int rl,
                                           int n) {
  constexpr int E = epi_elems<EPI>();
  constexpr int IR = ROWS / E;
  const int IRL = IR / KS;  // KS is a power of two <= IR
  int e;
  const int irow = epi_item_row<EPI>(rl, e);
  const int q = irow / IRL, irl = irow - q * IRL;
  float* base = (q == ks) ? recv : cl.map_shared_rank(recv, q);
  return base + ((ks * E + e) * Mp + n) * (IRL + 1) + irl;
}

// Receive-buffer slot of tile row `rl` for activation row n when one CTA holds the whole
// sum of the tile (KS = 1; same layout as epi_dest).
template <int EPI, int ROWS>
__device__ __forceinline__ float* epi_dest_local(float* recv, int Mp, int rl, int n) {
  constexpr int IR = ROWS / epi_elems<EPI>();
  int e;
  const int irow = epi_item_row<EPI>(rl, e);
  return recv + (e * Mp + n) * (IR + 1) + irow;
}

// The fused epilogue of one item for activation row n: idx is the weight row (STORE /
// RESID), the SwiGLU output column j (v0 = gate, v1 = up), or the even row of a RoPE pair
// (QKV: v0, v1 = rows idx, idx + 1). The caller checks idx against the output's extent.
// Every GEMM path ends here, so the epilogue arithmetic has one statement.
template <int EPI>
struct LoraGlobal {  // the LoRA term from the operands in global memory
  const QArgs& a;
  __device__ __forceinline__ float operator()(int n, int reg, int col, int width) const {
    constexpr int R = EPI == EPI_QKV ? 3 : (EPI == EPI_SWIGLU ? 2 : 1);
    return lora_delta_r<R>(a, n, reg, col, width);
  }
  // columns col and col + 1 (a RoPE pair)
  __device__ __forceinline__ void pair(int n, int reg, int col, int width, float& d0, float& d1) const {
    d0 = (*this)(n, reg, col, width);
    d1 = (*this)(n, reg, col + 1, width);
  }
};

// STORE / RESID: the value of output (n, row idx) before it is stored or added.
template <int WF, typename LoraF>
__device__ __forceinline__ float epi_value(const QArgs& a, int n, int idx, float v0, const LoraF& lora) {
  if (WF == W_Q8PC) v0 *= __half2float(a.s[idx]);
  if (a.lora_t != nullptr) v0 += lora(n, 0, idx, a.N);
  return v0;
}

template <int WF, int EPI, typename LoraF>
__device__ __forceinline__ void epi_apply(const QArgs& a, int n, int idx, float v0, float v1, const LoraF& lora) {
  if (EPI == EPI_STORE || EPI == EPI_RESID) {
    v0 = epi_value<WF>(a, n, idx, v0, lora);
    const size_t o = (size_t)n * a.ldo + idx;
    if (EPI == EPI_RESID) {
      float* y = static_cast<float*>(a.out);
      y[o] = y[o] + v0;
    } else if (a.out_f32) {
      static_cast<float*>(a.out)[o] = v0;
    } else {
      static_cast<__half*>(a.out)[o] = __float2half_rn(v0);
    }
  } else if (EPI == EPI_SWIGLU) {
    const int F = a.N >> 1;
    if (a.lora_t != nullptr) {
      v0 += lora(n, 0, idx, F);
      v1 += lora(n, 1, idx, F);
    }
    // silu(g) = g / (1 + e^-g); the fast divide is within 2 ulp (the IEEE divide is a
    // subroutine that dominated the decode epilogue); exp(-g) = inf gives 0, silu's limit
    const float si = __fdividef(v0, 1.0f + expf(-v0));
    static_cast<__half*>(a.out)[(size_t)n * F + idx] = __float2half_rn(si * v1);
  } else {  // EPI_QKV
    const int half_hd = a.hd >> 1;
    const int region = idx >= a.H ? (idx >= 2 * a.H ? 2 : 1) : 0;  // idx < 3H (the caller's check)
    const int rr = idx - region * a.H;
    // division by an invariant integer as a multiply-high (Granlund & Montgomery): with
    // m = ceil(2^32 / hd) = (2^32 + e) / hd, 0 <= e < hd, the error rr e / (hd 2^32) stays
    // below 1 / hd for rr < 2^16, so the floor is exact
    const int head = (int)__umulhi((uint32_t)rr, a.hd_magic);
    const int d = rr - head * a.hd;
    if (a.lora_t != nullptr) {
      float d0, d1;
      lora.pair(n, region, rr, a.H, d0, d1);
      v0 += d0;
      v1 += d1;
    }
    const int p = a.pos[n];
    if (p < 0 || p >= a.max_seq || p >= a.max_pos) {
      atomicOr(a.check, 1u);
      return;
    }
    if (region < 2) {
      const float cs = a.cos_tab[(size_t)p * half_hd + (d >> 1)];
      const float sn = a.sin_tab[(size_t)p * half_hd + (d >> 1)];
      const float r0 = v0 * cs - v1 * sn;
      const float r1 = v0 * sn + v1 * cs;
      v0 = r0;
      v1 = r1;
    }
    const __half2 hv = __floats2half2_rn(v0, v1);
    if (region == 0) {
      *reinterpret_cast<__half2*>(static_cast<__half*>(a.out) + (size_t)n * a.H + rr) = hv;
    } else {
      const int slot = a.slots ? a.slots[n] : a.slot0 + n;
      if (slot < 0 || slot >= a.num_slots) {
        atomicOr(a.check, 8u);
        return;
      }
      __half* cache = region == 1 ? a.kc : a.vc;
      const size_t off = (((size_t)slot * a.nh + head) * a.max_seq + p) * a.hd + d;
      *reinterpret_cast<__half2*>(cache + off) = hv;
    }
  }
}

template <int WF, int EPI>
__device__ __forceinline__ void epi_apply(const QArgs& a, int n, int idx, float v0, float v1) {
  epi_apply<WF, EPI>(a, n, idx, v0, v1, LoraGlobal<EPI>{a});
}

// The sums of this CTA's item rows over the KS partials in `recv` and the fused epilogue,
// by threads t0, t0 + nt, ... of the CTA (LoRA terms from `lora`).
template <int WF, int EPI, int ROWS, typename LoraF>
__device__ __forceinline__ void qgemm_epilogue(const QArgs& a, const float* recv, int KS, int ks, int R0, int t0,
                                               int nt, const LoraF& lora) {
  constexpr int E = epi_elems<EPI>();
  constexpr int IR = ROWS / E;
  const int IRL = IR / KS;
  const int IRL_LOG = __ffs(IRL) - 1;
  const int Mp = epi_mp(a.M);
  const int items = IRL * a.M;
  auto total = [&](int irl, int n, int e) {
    float v = 0.f;
    for (int r = 0; r < KS; ++r) v += recv[((r * E + e) * Mp + n) * (IRL + 1) + irl];
    return v;
  };
  if (EPI == EPI_RESID && items >= 8 * nt) {
    // prefill-sized tiles: residual read-modify-writes eight at a time, their loads issued
    // together instead of one dependent round trip per output (the compiler cannot tell the
    // stores from the loads); with a few items per thread (decode) the plain loop is faster
    float* y = static_cast<float*>(a.out);
    for (int i0 = t0; i0 < items; i0 += 8 * nt) {
      float v[8], yv[8];
      size_t o[8];
      bool live[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int i = i0 + u * nt;
        const int irl = i & (IRL - 1), n = i >> IRL_LOG;
        const int row = R0 + ks * IRL + irl;
        live[u] = i < items && row < a.N;
        o[u] = live[u] ? (size_t)n * a.ldo + row : 0;
        v[u] = live[u] ? epi_value<WF>(a, n, row, total(irl, n, 0), lora) : 0.f;
      }
#pragma unroll
      for (int u = 0; u < 8; ++u) yv[u] = live[u] ? y[o[u]] : 0.f;
#pragma unroll
      for (int u = 0; u < 8; ++u)
        if (live[u]) y[o[u]] = yv[u] + v[u];
    }
    return;
  }
  for (int i = t0; i < items; i += nt) {
    const int irl = i & (IRL - 1), n = i >> IRL_LOG;
    if (EPI == EPI_STORE || EPI == EPI_RESID) {
      const int row = R0 + ks * IRL + irl;
      if (row < a.N) epi_apply<WF, EPI>(a, n, row, total(irl, n, 0), 0.f, lora);
    } else if (EPI == EPI_SWIGLU) {
      const int j = (R0 >> 1) + ks * IRL + irl;
      if (j < (a.N >> 1)) epi_apply<WF, EPI>(a, n, j, total(irl, n, 0), total(irl, n, 1), lora);
    } else {
      const int row = R0 + 2 * (ks * IRL + irl);
      if (row < a.N) epi_apply<WF, EPI>(a, n, row, total(irl, n, 0), total(irl, n, 1), lora);
    }
  }
}

template <int WF, int EPI, int ROWS>
__device__ __forceinline__ void qgemm_epilogue(const QArgs& a, const float* recv, int KS, int ks, int R0, int t0,
                                               int nt) {
  qgemm_epilogue<WF, EPI, ROWS>(a, recv, KS, ks, R0, t0, nt, LoraGlobal<EPI>{a});
}

// After every CTA of the cluster pushed its partials: the cluster barrier, then the sums and
// the epilogue of this CTA's item rows.
template <int WF, int EPI, int ROWS>
__device__ __forceinline__ void qgemm_finish(const QArgs& a, const float* recv, int KS, int ks, int R0) {
  cg::this_cluster().sync();
  qgemm_epilogue<WF, EPI, ROWS>(a, recv, KS, ks, R0, threadIdx.x, blockDim.x);
}
template <int WF, int EPI, int ROWS, typename LoraF>
__device__ __forceinline__ void qgemm_finish(const QArgs& a, const float* recv, int KS, int ks, int R0,
                                             const LoraF& lora) {
  cg::this_cluster().sync();
  qgemm_epilogue<WF, EPI, ROWS>(a, recv, KS, ks, R0, threadIdx.x, blockDim.x, lora);
}

}  // namespace orch
