// Decode attention over the device KV cache, row softmax and row argmax.
//
// Reference: the host NumPy attention of orchard/model.py:112-144 (per sequence, per head,
// softmax(q.K / sqrt(hd)) . V over positions 0..pos, the current token appended first) and
// the Metal softmax of orchard/kernels/softmax.metal:4-56.
//
// Cache layout [slot][head][max_seq][head_dim] fp16: one (slot, head) pair is a contiguous
// run of pos+1 rows of head_dim halves, so both passes stream whole 32-byte sectors.
// A CTA owns one (row, head) and a range of positions; with few rows (B = 1) the positions
// are split over several CTAs and their (max, sum, acc) partials are merged by a second
// small kernel (flash-decoding). Split partials live in a caller-provided workspace.
#include <algorithm>
#include <mutex>

#include "orch_common.cuh"

namespace orch {

constexpr int kAttnThreads = 128;
constexpr int kAttnChunk = 1024;  // positions per CTA at most (scores live in shared memory)

struct AttnArgs {
  const __half* q;
  const __half* kc;
  const __half* vc;
  const int* pos;
  const int* slots;
  __half* out;
  float* ws;  // [M*nh][S][HD + 2]
  int M, nh, max_seq, S;
  int num_slots;  // slots in the caches; a row whose slot is outside [0, num_slots) is skipped
  uint32_t* check;
};

// Cache slot of row m, or -1 when it lies outside the caches (uniform per CTA).
__device__ __forceinline__ int attn_slot(const AttnArgs& a, int m) {
  const int slot = a.slots ? a.slots[m] : m;
  return (slot < 0 || slot >= a.num_slots) ? -1 : slot;
}

template <int HD>
__global__ void __launch_bounds__(kAttnThreads) attn_decode_kernel(const AttnArgs a) {
  __shared__ float sc[kAttnChunk];
  __shared__ float red[32];
  __shared__ float accs[kAttnThreads / 32][HD];
  pdl_trigger();
  pdl_wait();

  const int mh = blockIdx.x;
  const int m = mh / a.nh, h = mh - m * a.nh;
  const int split = blockIdx.y;
  const int p = a.pos[m];
  if (p < 0 || p >= a.max_seq) {  // uniform per CTA
    if (threadIdx.x == 0) atomicOr(a.check, 2u);
    return;
  }
  const int slot = attn_slot(a, m);
  if (slot < 0) {
    if (threadIdx.x == 0) atomicOr(a.check, 8u);
    return;
  }
  const int L = p + 1;
  const int per = (L + a.S - 1) / a.S;
  const int p0 = split * per;
  const int p1 = min(L, p0 + per);
  const size_t base = ((size_t)slot * a.nh + h) * a.max_seq * HD;
  const __half* K = a.kc + base;
  const __half* V = a.vc + base;
  const float scale = rsqrtf((float)HD);

  // pass 1: four lanes per position, each holding HD/4 dims of q (scaled) in registers; a
  // warp scores 8 positions per step (a two-step shuffle sums the four partial dots), two
  // steps' K rows are requested before either is used
  constexpr int DPL = HD / 4, CPL = DPL / 8;  // dims and 16-byte chunks per lane
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int sub = lane & 3;
  float qv[DPL];
  {
    const __half* qp = a.q + (size_t)m * a.nh * HD + h * HD + sub * DPL;
#pragma unroll
    for (int cidx = 0; cidx < CPL; ++cidx) {
      const uint4 raw = __ldg(reinterpret_cast<const uint4*>(qp) + cidx);
      const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 f = __half22float2(bits_h2(w[e]));
        qv[cidx * 8 + 2 * e] = f.x * scale;
        qv[cidx * 8 + 2 * e + 1] = f.y * scale;
      }
    }
  }
  auto dot = [&](const uint4 (&raw)[CPL]) {
    float sdot = 0.f;
#pragma unroll
    for (int cidx = 0; cidx < CPL; ++cidx) {
      const uint32_t w[4] = {raw[cidx].x, raw[cidx].y, raw[cidx].z, raw[cidx].w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 f = __half22float2(bits_h2(w[e]));
        sdot = fmaf(f.x, qv[cidx * 8 + 2 * e], sdot);
        sdot = fmaf(f.y, qv[cidx * 8 + 2 * e + 1], sdot);
      }
    }
    sdot += __shfl_xor_sync(0xffffffffu, sdot, 1);
    sdot += __shfl_xor_sync(0xffffffffu, sdot, 2);
    return sdot;
  };
  float lmax = -INFINITY;
  constexpr int kStep = (kAttnThreads / 32) * 8;  // positions per CTA step
  for (int tb = p0 + warp * 8; tb < p1; tb += 2 * kStep) {  // warp-uniform trip count
    const int t0 = tb + (lane >> 2), t1 = t0 + kStep;
    const bool v0 = t0 < p1, v1 = t1 < p1;
    uint4 r0[CPL], r1[CPL];
#pragma unroll
    for (int cidx = 0; cidx < CPL; ++cidx) {
      r0[cidx] = v0 ? ld_stream16(K + (size_t)t0 * HD + sub * DPL + cidx * 8) : make_uint4(0, 0, 0, 0);
      r1[cidx] = v1 ? ld_stream16(K + (size_t)t1 * HD + sub * DPL + cidx * 8) : make_uint4(0, 0, 0, 0);
    }
    const float s0 = dot(r0), s1 = dot(r1);
    if (v0) {
      if (sub == 0) sc[t0 - p0] = s0;
      lmax = fmaxf(lmax, s0);
    }
    if (v1) {
      if (sub == 0) sc[t1 - p0] = s1;
      lmax = fmaxf(lmax, s1);
    }
  }
  // pass 2's geometry: LPR lanes cover one position row in 16-byte pieces, so a warp load
  // instruction reads RPW whole rows; U such loads per lane are in flight before any is used
  constexpr int LPR = HD / 8, RPW = 32 / LPR, NW = kAttnThreads / 32, STR = NW * RPW, U = 8;
  const int vsub = lane / LPR, ci = lane - vsub * LPR;
  // A split that fits one batch of U loads per lane (the short splits of small batches):
  // its V rows are requested now, so their latency runs under the softmax reductions.
  const bool one_batch = p1 - p0 <= U * STR;  // uniform per CTA
  const int tv = p0 + warp * RPW + vsub;
  uint4 rawv[U];
  if (one_batch) {
#pragma unroll
    for (int u = 0; u < U; ++u)
      rawv[u] = tv + u * STR < p1 ? ld_stream16(V + (size_t)(tv + u * STR) * HD + ci * 8) : make_uint4(0, 0, 0, 0);
  }
  const float mx = block_max(lmax, red);
  float lsum = 0.f;
  for (int t = threadIdx.x; t < p1 - p0; t += kAttnThreads) {
    const float e = __expf(sc[t] - mx);
    sc[t] = e;
    lsum += e;
  }
  const float sum = block_sum(lsum, red);  // contains __syncthreads: sc[] complete

  // pass 2: P.V in ascending position order per lane
  float acc[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) acc[i] = 0.f;
  auto fma8 = [&](const uint4& raw, float w) {
    const float2 f0 = __half22float2(bits_h2(raw.x)), f1 = __half22float2(bits_h2(raw.y));
    const float2 f2 = __half22float2(bits_h2(raw.z)), f3 = __half22float2(bits_h2(raw.w));
    acc[0] = fmaf(w, f0.x, acc[0]);
    acc[1] = fmaf(w, f0.y, acc[1]);
    acc[2] = fmaf(w, f1.x, acc[2]);
    acc[3] = fmaf(w, f1.y, acc[3]);
    acc[4] = fmaf(w, f2.x, acc[4]);
    acc[5] = fmaf(w, f2.y, acc[5]);
    acc[6] = fmaf(w, f3.x, acc[6]);
    acc[7] = fmaf(w, f3.y, acc[7]);
  };
  if (one_batch) {
#pragma unroll
    for (int u = 0; u < U; ++u)
      if (tv + u * STR < p1) fma8(rawv[u], sc[tv + u * STR - p0]);
  } else {
    int t = tv;
    for (; t + (U - 1) * STR < p1; t += U * STR) {
      uint4 raw[U];
#pragma unroll
      for (int u = 0; u < U; ++u) raw[u] = ld_stream16(V + (size_t)(t + u * STR) * HD + ci * 8);
#pragma unroll
      for (int u = 0; u < U; ++u) fma8(raw[u], sc[t + u * STR - p0]);
    }
    for (; t < p1; t += STR) fma8(ld_stream16(V + (size_t)t * HD + ci * 8), sc[t - p0]);
  }
#pragma unroll
  for (int o = LPR; o < 32; o <<= 1)
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[i] += __shfl_xor_sync(0xffffffffu, acc[i], o);
  if (vsub == 0)
#pragma unroll
    for (int i = 0; i < 8; ++i) accs[warp][ci * 8 + i] = acc[i];
  __syncthreads();
  for (int d = threadIdx.x; d < HD; d += kAttnThreads) {
    float v = 0.f;
#pragma unroll
    for (int w2 = 0; w2 < kAttnThreads / 32; ++w2) v += accs[w2][d];
    if (a.S == 1) {
      a.out[(size_t)m * a.nh * HD + h * HD + d] = __float2half_rn(v / sum);
    } else {
      float* wp = a.ws + ((size_t)mh * a.S + split) * (HD + 2);
      wp[2 + d] = v;
      if (d == 0) {
        wp[0] = (p1 > p0) ? mx : -INFINITY;
        wp[1] = (p1 > p0) ? sum : 0.f;
      }
    }
  }
}

template <int HD>
__global__ void attn_combine_kernel(const AttnArgs a) {
  pdl_trigger();
  pdl_wait();
  const int mh = blockIdx.x;
  const int m = mh / a.nh, h = mh - m * a.nh;
  const int p = a.pos[m];
  if (p < 0 || p >= a.max_seq || attn_slot(a, m) < 0) return;  // flagged by attn_decode_kernel
  // One thread per output dimension (blockDim.x == HD). The splits are taken HD at a time: each
  // thread turns one split's running max into its weight f_s = exp(m_s - max) in shared memory,
  // then every thread sums that group's partials with the loads issued together. (A loop that
  // read m_s, then l_s, then the partial, split by split, waited one L2 round trip per split:
  // 11 us per layer at batch 1 with 19 splits.)
  __shared__ float fsh[HD];
  __shared__ float red[32];
  const int d = threadIdx.x;
  const float* wp = a.ws + (size_t)mh * a.S * (HD + 2);
  if (a.S <= 32) {
    // Up to 32 splits (batch 1 at the 7B shape has 19): every load is issued before the two
    // block reductions, so the kernel waits on L2 once instead of once per pass. The sums are
    // those of the general loop below (split d's weight by thread d, partials in split order).
    float pv[32];
#pragma unroll
    for (int j = 0; j < 32; ++j) pv[j] = j < a.S ? wp[j * (HD + 2) + 2 + d] : 0.f;
    const float ms = d < a.S ? wp[d * (HD + 2)] : -INFINITY;
    const float ls = d < a.S ? wp[d * (HD + 2) + 1] : 0.f;
    const float gmax = block_max(ms, red);
    const float f = ms == -INFINITY ? 0.f : __expf(ms - gmax);
    fsh[d] = f;
    const float den = block_sum(fmaf(f, ls, 0.f), red);  // its barriers also publish fsh
    float num = 0.f;
#pragma unroll
    for (int j = 0; j < 32; ++j)
      if (j < a.S) num = fmaf(fsh[j], pv[j], num);
    a.out[(size_t)m * a.nh * HD + h * HD + d] = __float2half_rn(num / den);
    return;
  }
  float lmax = -INFINITY;
  for (int s = d; s < a.S; s += HD) lmax = fmaxf(lmax, wp[s * (HD + 2)]);
  const float gmax = block_max(lmax, red);
  float lden = 0.f, num = 0.f;
  for (int s0 = 0; s0 < a.S; s0 += HD) {
    float f = 0.f;
    if (s0 + d < a.S) {
      const float ms = wp[(s0 + d) * (HD + 2)];
      f = ms == -INFINITY ? 0.f : __expf(ms - gmax);
      lden = fmaf(f, wp[(s0 + d) * (HD + 2) + 1], lden);
    }
    fsh[d] = f;
    __syncthreads();
    const int n = min(HD, a.S - s0);
    const float* part = wp + (size_t)s0 * (HD + 2) + 2 + d;
#pragma unroll 8
    for (int j = 0; j < n; ++j) num = fmaf(fsh[j], part[j * (HD + 2)], num);
    __syncthreads();
  }
  const float den = block_sum(lden, red);
  a.out[(size_t)m * a.nh * HD + h * HD + d] = __float2half_rn(num / den);
}

static int attn_splits(int M, int nh, int max_seq) {
  // enough CTAs to cover the SMs a few times; positions per CTA <= kAttnChunk
  const int pairs = M * nh;
  int S = std::max(1, (4 * num_sms() + pairs - 1) / pairs);
  S = std::max(S, (max_seq + kAttnChunk - 1) / kAttnChunk);
  return std::min(S, std::max(1, (max_seq + 31) / 32));
}

template <int HD>
static int attn_launch(AttnArgs a, cudaStream_t st) {
  dim3 grid(a.M * a.nh, a.S);
  const dim3 none(0, 0, 0);
  // Not a programmatic dependent: launched early (the QKV GEMM releases dependents at its
  // start), its many small CTAs occupy the SMs while the GEMM still runs; measured at batch
  // 64 (7B shape) that made the decode step 12.1 ms instead of 8.1 ms.
  ORCH_CUDA(launch_k_serial(attn_decode_kernel<HD>, grid, dim3(kAttnThreads), 0, st, none, a));
  if (a.S > 1) ORCH_CUDA(launch_k(attn_combine_kernel<HD>, dim3(a.M * a.nh), dim3(HD), 0, st, none, a));
  return check_launch("attention_decode");
}

// ---- row softmax (softmax.metal:4-56), any cols -------------------------------------------
template <typename TI, typename TO>
__global__ void softmax_rows_kernel(const TI* in, TO* out, int cols) {
  __shared__ float red[32];
  pdl_trigger();
  pdl_wait();
  const TI* r = in + (size_t)blockIdx.x * cols;
  TO* o = out + (size_t)blockIdx.x * cols;
  float mx = -INFINITY;
  for (int i = threadIdx.x; i < cols; i += blockDim.x) mx = fmaxf(mx, to_f32(r[i]));
  mx = block_max(mx, red);
  float s = 0.f;
  for (int i = threadIdx.x; i < cols; i += blockDim.x) s += __expf(to_f32(r[i]) - mx);
  s = block_sum(s, red);
  const float inv = 1.0f / s;
  for (int i = threadIdx.x; i < cols; i += blockDim.x) o[i] = from_f32<TO>(__expf(to_f32(r[i]) - mx) * inv);
}

// ---- row argmax (first index of the maximum, as np.argmax) ---------------------------------
// Whether candidate (v, i) beats (best, bi) in np.argmax order: a NaN beats any number, the
// larger value wins, equal values (or two NaNs) go to the lower index.
__device__ __forceinline__ bool argmax_better(float v, int i, float best, int bi) {
  const bool vn = v != v, bn = best != best;
  if (vn || bn) return vn && (!bn || i < bi);
  return v > best || (v == best && i < bi);
}

// PAIRS: also write the row's maximum (as float) and base + index (as float, exact below
// 2^24) to out_pairs[row] for the vocabulary-split merge.
template <bool PAIRS>
__global__ void argmax_rows_kernel(const float* logits, int V, int* out, float2* out_pairs, int base) {
  __shared__ float sv[32];
  __shared__ int si[32];
  pdl_trigger();
  pdl_wait();
  const float* r = logits + (size_t)blockIdx.x * V;
  float best = -INFINITY;
  int bi = 0x7fffffff;
  // Eight loads in flight per step, compared in ascending index order as one at a time would
  // (a dependent load per element was 31 L2 round trips: 18 us for one 32000-entry row).
  int i = threadIdx.x;
  const int step = blockDim.x;
  for (; i + 7 * step < V; i += 8 * step) {
    float v[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) v[u] = r[i + u * step];
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int j = i + u * step;
      if (v[u] > best || (v[u] == best && j < bi) || (v[u] != v[u] && best == best)) {  // NaN wins, as np.argmax
        best = v[u];
        bi = j;
      }
    }
  }
  for (; i < V; i += step) {
    const float v = r[i];
    if (v > best || (v == best && i < bi) || (v != v && best == best)) {
      best = v;
      bi = i;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, best, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (argmax_better(ov, oi, best, bi)) {
      best = ov;
      bi = oi;
    }
  }
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  if (lane == 0) {
    sv[wid] = best;
    si[wid] = bi;
  }
  __syncthreads();
  if (wid == 0) {
    const int nw = blockDim.x >> 5;
    best = lane < nw ? sv[lane] : -INFINITY;
    bi = lane < nw ? si[lane] : 0x7fffffff;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, best, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (argmax_better(ov, oi, best, bi)) {
        best = ov;
        bi = oi;
      }
    }
    if (lane == 0) {
      const int i = bi == 0x7fffffff ? 0 : bi;
      if (PAIRS)
        out_pairs[blockIdx.x] = make_float2(best, (float)(base + i));
      else
        out[blockIdx.x] = i;
    }
  }
}

}  // namespace orch

using namespace orch;

extern "C" size_t orch_attention_workspace_bytes(uint32_t M, uint32_t num_heads, uint32_t head_dim,
                                                 uint32_t max_seq) {
  if (M == 0 || num_heads == 0 || max_seq == 0) return 0;
  const int S = attn_splits((int)M, (int)num_heads, (int)max_seq);
  return S > 1 ? (size_t)M * num_heads * S * (head_dim + 2) * sizeof(float) : 0;
}

extern "C" int orch_attention_decode(const void* q, const void* k_cache, const void* v_cache,
                                     const int32_t* pos, const int32_t* slots, void* out, uint32_t M,
                                     uint32_t num_heads, uint32_t head_dim, uint32_t max_seq, uint32_t num_slots,
                                     void* workspace, size_t workspace_bytes, void* stream) {
  if (M == 0) return ORCH_OK;
  ORCH_REQUIRE(q && k_cache && v_cache && pos && out, "attention_decode: null pointer");
  ORCH_REQUIRE(num_heads > 0 && max_seq > 0 && num_slots > 0 && num_slots <= 0x7fffffffu,
               "attention_decode: empty shape");
  ORCH_REQUIRE(head_dim == 32 || head_dim == 64 || head_dim == 128,
               "attention_decode: head_dim must be 32, 64 or 128");
  AttnArgs a;
  a.q = static_cast<const __half*>(q);
  a.kc = static_cast<const __half*>(k_cache);
  a.vc = static_cast<const __half*>(v_cache);
  a.pos = pos;
  a.slots = slots;
  a.out = static_cast<__half*>(out);
  a.M = (int)M;
  a.nh = (int)num_heads;
  a.max_seq = (int)max_seq;
  a.num_slots = (int)num_slots;
  a.S = attn_splits(a.M, a.nh, a.max_seq);
  ORCH_CHECK_WORD(a.check);
  const size_t need = orch_attention_workspace_bytes(M, num_heads, head_dim, max_seq);
  ORCH_REQUIRE(workspace_bytes >= need && (need == 0 || workspace != nullptr),
               "attention_decode: workspace too small");
  a.ws = static_cast<float*>(workspace);
  cudaStream_t st = as_stream(stream);
  switch (head_dim) {
    case 32: return attn_launch<32>(a, st);
    case 64: return attn_launch<64>(a, st);
    default: return attn_launch<128>(a, st);
  }
}

extern "C" int orch_softmax_ex(const void* in, int in_dt, void* out, int out_dt, uint32_t rows,
                               uint32_t cols, void* stream) {
  if (rows == 0 || cols == 0) return ORCH_OK;
  ORCH_REQUIRE(in && out, "softmax: null pointer");
  cudaStream_t st = as_stream(stream);
  const int th = cols >= 1024 ? 1024 : cols >= 256 ? 256 : 128;
  if (in_dt == ORCH_F16 && out_dt == ORCH_F16)
    ORCH_CUDA(launch_k(softmax_rows_kernel<__half, __half>, dim3(rows), dim3(th), 0, st, dim3(0, 0, 0), (const __half*)in, (__half*)out, cols));
  else if (in_dt == ORCH_F32 && out_dt == ORCH_F32)
    ORCH_CUDA(launch_k(softmax_rows_kernel<float, float>, dim3(rows), dim3(th), 0, st, dim3(0, 0, 0), (const float*)in, (float*)out, cols));
  else if (in_dt == ORCH_F16 && out_dt == ORCH_F32)
    ORCH_CUDA(launch_k(softmax_rows_kernel<__half, float>, dim3(rows), dim3(th), 0, st, dim3(0, 0, 0), (const __half*)in, (float*)out, cols));
  else if (in_dt == ORCH_F32 && out_dt == ORCH_F16)
    ORCH_CUDA(launch_k(softmax_rows_kernel<float, __half>, dim3(rows), dim3(th), 0, st, dim3(0, 0, 0), (const float*)in, (__half*)out, cols));
  else
    return fail(ORCH_ERR_INVALID, "softmax: bad dtype");
  return check_launch("softmax");
}

extern "C" int orch_softmax(const void* in, void* out, uint32_t rows, uint32_t cols, void* stream) {
  return orch_softmax_ex(in, ORCH_F16, out, ORCH_F16, rows, cols, stream);
}

extern "C" int orch_argmax_rows(const float* logits, uint32_t M, uint32_t V, int32_t* out, void* stream) {
  if (M == 0) return ORCH_OK;
  ORCH_REQUIRE(logits && out && V > 0, "argmax_rows: bad arguments");
  ORCH_CUDA(launch_k(argmax_rows_kernel<false>, dim3(M), dim3(1024), 0, as_stream(stream), dim3(0, 0, 0), logits,
                     (int)V, (int*)out, (float2*)nullptr, 0));
  return check_launch("argmax_rows");
}

// (max, base + argmax) of each row of a vocabulary slice, as float pairs [M][2].
extern "C" int orch_argmax_pairs(const float* logits, uint32_t M, uint32_t V, uint32_t base, float* pairs,
                                 void* stream) {
  if (M == 0) return ORCH_OK;
  ORCH_REQUIRE(logits && pairs && V > 0 && base + V < (1u << 24), "argmax_pairs: bad arguments");
  ORCH_CUDA(launch_k(argmax_rows_kernel<true>, dim3(M), dim3(1024), 0, as_stream(stream), dim3(0, 0, 0), logits,
                     (int)V, (int*)nullptr, (float2*)pairs, (int)base));
  return check_launch("argmax_pairs");
}

namespace orch {
// Temperature sampling of one row per CTA (orchard/model.py:247-252 with np.random.choice):
// e_i = exp((l_i - max) / T) in fp32, then the first index whose running sum exceeds
// u * sum(e) for the row's uniform u (the inverse CDF np.random.choice evaluates). Each
// thread owns a contiguous chunk; chunk sums are scanned across the block, and the thread
// whose chunk holds the crossing walks it in order.
__global__ void __launch_bounds__(1024) sample_rows_kernel(const float* logits, int V, float temperature,
                                                           const float* uniforms, int* tok) {
  __shared__ float red[32];
  __shared__ float wsum[32];
  __shared__ int found;
  pdl_trigger();
  pdl_wait();
  const float* r = logits + (size_t)blockIdx.x * V;
  float mx = -INFINITY;
  for (int i = threadIdx.x; i < V; i += blockDim.x) mx = fmaxf(mx, r[i]);
  mx = block_max(mx, red);
  const int chunk = (V + blockDim.x - 1) / blockDim.x;
  const int c0 = min(V, (int)threadIdx.x * chunk), c1 = min(V, c0 + chunk);
  float local = 0.f;
  for (int i = c0; i < c1; ++i) local += expf((r[i] - mx) / temperature);
  // inclusive scan of the chunk sums over the block
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  float incl = local;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const float v = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += v;
  }
  if (lane == 31) wsum[w] = incl;
  if (threadIdx.x == 0) found = 0;
  __syncthreads();
  float wprefix = 0.f, total = 0.f;
  for (int j = 0; j < (int)(blockDim.x >> 5); ++j) {
    if (j < w) wprefix += wsum[j];
    total += wsum[j];
  }
  const float before = wprefix + incl - local;  // sum of all earlier chunks
  const float target = uniforms[blockIdx.x] * total;
  if (local > 0.f && before <= target && target < before + local) {
    float run = before;
    int pick = c1 - 1;
    for (int i = c0; i < c1; ++i) {
      run += expf((r[i] - mx) / temperature);
      if (run > target) {
        pick = i;
        break;
      }
    }
    if (atomicCAS(&found, 0, 1) == 0) tok[blockIdx.x] = pick;
  }
  __syncthreads();
  if (threadIdx.x == 0 && !found) {  // rounding put the target past the last sum: the argmax
    int best = 0;
    for (int i = 0; i < V; ++i)
      if (r[i] == mx) {
        best = i;
        break;
      }
    tok[blockIdx.x] = best;
  }
}

// One thread per row: the highest value over the ranks' pairs, the lowest id among equal
// values, a NaN wins (np.argmax over the whole vocabulary).
__global__ void argmax_merge_kernel(const float2* pairs, int world, int B, int row0, int rows, int* tok) {
  pdl_trigger();
  pdl_wait();
  const int r = blockIdx.x * blockDim.x + threadIdx.x;
  if (r >= rows) return;
  float2 best = pairs[row0 + r];
  for (int w = 1; w < world; ++w) {
    if (best.x != best.x) break;
    const float2 v = pairs[(size_t)w * B + row0 + r];
    if (v.x != v.x || v.x > best.x || (v.x == best.x && v.y < best.y)) best = v;
  }
  tok[r] = (int)best.y;
}
}  // namespace orch

extern "C" int orch_sample_rows(const float* logits, uint32_t M, uint32_t V, float temperature,
                                const float* uniforms, int32_t* tok, void* stream) {
  if (M == 0) return ORCH_OK;
  ORCH_REQUIRE(logits && uniforms && tok && V > 0, "sample_rows: bad arguments");
  ORCH_REQUIRE(temperature > 0.f, "sample_rows: temperature must be positive (0 is argmax)");
  ORCH_CUDA(launch_k(sample_rows_kernel, dim3(M), dim3(1024), 0, as_stream(stream), dim3(0, 0, 0), logits, (int)V,
                     temperature, uniforms, (int*)tok));
  return check_launch("sample_rows");
}

// Merge the all-gathered pairs [world][B][2] for rows row0 .. row0 + rows - 1 into tokens.
extern "C" int orch_argmax_merge(const float* pairs, uint32_t world, uint32_t B, uint32_t row0, uint32_t rows,
                                 int32_t* tok, void* stream) {
  if (rows == 0) return ORCH_OK;
  ORCH_REQUIRE(pairs && tok && world > 0 && row0 + rows <= B, "argmax_merge: bad arguments");
  ORCH_CUDA(launch_k(argmax_merge_kernel, dim3((rows + 127) / 128), dim3(128), 0, as_stream(stream),
                     dim3(0, 0, 0), (const float2*)pairs, (int)world, (int)B, (int)row0, (int)rows, (int*)tok));
  return check_launch("argmax_merge");
}

// ---------------------------------------------------------------------------------------------
// Allocation-free decode attention.
//
// For callers that must not allocate device memory at all: code that runs while a CUDA
// graph is being captured by someone else, real-time or embedded hosts whose memory is
// fixed at start-up, and plugin hosts that hand this library only the tensors of the call.
// The split-position partials live in a file-scope device array instead of a caller
// workspace. Every GPU that loads the library holds this array until the process exits.
// ---------------------------------------------------------------------------------------------
namespace orch {

// 1 MiB of partials: (row, head, split) records of head_dim + 2 floats.
constexpr size_t kNoAllocScratchFloats = 256 * 1024;
static __device__ __align__(256) float g_attn_scratch[kNoAllocScratchFloats];
static __device__ __align__(256) uint32_t g_attn_noalloc_check[64];

struct NoAllocState {
  float* scratch = nullptr;
  uint32_t* check = nullptr;
  int sms = 0;
};
static NoAllocState g_noalloc[64];
static std::mutex g_noalloc_mu;

// Host code may not use the arrays' names as addresses; fetch the device addresses once
// per device, with that device current.
static int noalloc_setup(int dev, NoAllocState** out) {
  if (dev < 0 || dev >= 64) return fail(ORCH_ERR_UNSUPPORTED, "attention_decode_noalloc: device index out of range");
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  NoAllocState& st = g_noalloc[dev];
  if (st.scratch == nullptr) {
    void* p = nullptr;
    ORCH_CUDA(cudaGetSymbolAddress(&p, g_attn_scratch));
    void* c = nullptr;
    ORCH_CUDA(cudaGetSymbolAddress(&c, g_attn_noalloc_check));
    int sms = 0;
    ORCH_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
    st.check = static_cast<uint32_t*>(c);
    st.sms = sms;
    st.scratch = static_cast<float*>(p);
  }
  *out = &st;
  return ORCH_OK;
}

uint32_t* noalloc_check_word(int dev) {
  if (dev < 0 || dev >= 64) return nullptr;
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  return g_noalloc[dev].check;
}

static int noalloc_splits(int M, int nh, int max_seq, int sms) {
  const int pairs = M * nh;
  int S = std::max(1, (4 * sms + pairs - 1) / pairs);
  S = std::max(S, (max_seq + kAttnChunk - 1) / kAttnChunk);
  return std::min(S, std::max(1, (max_seq + 31) / 32));
}

}  // namespace orch

extern "C" size_t orch_attention_noalloc_max_bytes(void) { return orch::kNoAllocScratchFloats * sizeof(float); }

extern "C" int orch_attention_decode_noalloc(const void* q, const void* k_cache, const void* v_cache,
                                             const int32_t* pos, const int32_t* slots, void* out, uint32_t M,
                                             uint32_t num_heads, uint32_t head_dim, uint32_t max_seq,
                                             uint32_t num_slots, void* stream) {
  if (M == 0) return ORCH_OK;
  ORCH_REQUIRE(q && k_cache && v_cache && pos && out, "attention_decode_noalloc: null pointer");
  ORCH_REQUIRE(num_heads > 0 && max_seq > 0 && num_slots > 0 && num_slots <= 0x7fffffffu,
               "attention_decode_noalloc: empty shape");
  ORCH_REQUIRE(head_dim == 32 || head_dim == 64 || head_dim == 128,
               "attention_decode_noalloc: head_dim must be 32, 64 or 128");
  int dev = 0;
  ORCH_CUDA(cudaGetDevice(&dev));
  orch::NoAllocState* st = nullptr;
  int rc = orch::noalloc_setup(dev, &st);
  if (rc != ORCH_OK) return rc;
  AttnArgs a;
  a.q = static_cast<const __half*>(q);
  a.kc = static_cast<const __half*>(k_cache);
  a.vc = static_cast<const __half*>(v_cache);
  a.pos = pos;
  a.slots = slots;
  a.out = static_cast<__half*>(out);
  a.M = (int)M;
  a.nh = (int)num_heads;
  a.max_seq = (int)max_seq;
  a.num_slots = (int)num_slots;
  a.S = orch::noalloc_splits(a.M, a.nh, a.max_seq, st->sms);
  a.check = st->check;
  a.ws = st->scratch;
  // every split record is written before the combine pass reads it: nothing needs clearing
  const size_t need = a.S > 1 ? (size_t)M * num_heads * a.S * (head_dim + 2) : 0;
  if (need > orch::kNoAllocScratchFloats)
    return fail(ORCH_ERR_UNSUPPORTED, "attention_decode_noalloc: rows x heads x splits exceed the 1 MiB scratch "
                                      "(use orch_attention_decode with a workspace)");
  cudaStream_t s = as_stream(stream);
  switch (head_dim) {
    case 32: return attn_launch<32>(a, s);
    case 64: return attn_launch<64>(a, s);
    default: return attn_launch<128>(a, s);
  }
}
