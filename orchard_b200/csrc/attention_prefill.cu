// Causal attention for prefill chunks on the tensor cores (mma.sync m16n8k16), over the same
// device KV cache as decode attention ([slot][head][max_seq][128] fp16).
//
// Reference: the host NumPy attention of orchard/model.py:112-144, run there once per prompt
// token (softmax(q.K / sqrt(hd)) . V over positions 0..pos). Decode attention (attention.cu)
// reads a row's whole prefix for each row; in a prefill chunk consecutive rows of a sequence
// share that prefix, so here a CTA takes up to 64 consecutive query rows of one sequence (a
// "unit": row0, count, slot, first position, listed by the host) for one head and streams the
// keys 0..last position once, 64 at a time, flash-attention style:
//  * S = Q K^T with fp16 MMAs and fp32 accumulation (the products of fp16 values are exact in
//    fp32), scaled by 1/sqrt(hd) in fp32, keys after a row's own position masked;
//  * an online softmax in fp32 (running max and sum per row);
//  * O += P V with P split into fp16 hi + lo terms (P - hi rounded to fp16), so the
//    probabilities keep ~22 bits and the result stays at fp32-level accuracy.
// Keys past the unit's last position are zero-filled in shared memory (never read from the
// cache), so stale cache contents cannot reach the output. K and V blocks are copied row-major
// with cp.async into a double buffer (the next block in flight while one is multiplied); the
// MMA operands come from ldmatrix (K rows as the B operand of Q K^T, V rows transposed by
// ldmatrix.trans as the B operand of P V), with a row pitch of 136 halves so the eight rows
// of each 8 x 8 matrix fall in distinct banks.
#include "orch_common.cuh"

namespace orch {

namespace {

constexpr int kPfRows = 64;            // query rows per CTA: 4 warps x 16
constexpr int kPfKeys = 64;            // keys per block
constexpr int kPfHD = 128;             // head dim
constexpr int kPfP = kPfHD + 8;        // Q / K / V smem row pitch (halves): 272 B, 16-byte aligned
constexpr int kPfTile = kPfKeys * kPfP;  // one K or V block (halves)
constexpr int kPfSmem = 4 * kPfTile * 2;  // double buffer of K and V blocks; Q staged in buffer 1

struct PfArgs {
  const __half* q;
  const __half* kc;
  const __half* vc;
  const int4* units;  // (row0, rows, slot, pos0)
  __half* out;
  int M, nh, max_seq;
  int num_slots;  // slots in the caches
  uint32_t* check;
};

__device__ __forceinline__ uint32_t ld_h2(const __half* p) { return *reinterpret_cast<const uint32_t*>(p); }
__device__ __forceinline__ uint32_t pack_h2(float lo, float hi) { return h2_bits(__floats2half2_rn(lo, hi)); }

__device__ __forceinline__ void pf_cp16(const void* dst, const void* src, bool ok) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(static_cast<uint32_t>(__cvta_generic_to_shared(dst))),
               "l"(src), "r"(ok ? 16 : 0)
               : "memory");
}
__device__ __forceinline__ void ldsm_x4(const __half* p, uint32_t (&r)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(static_cast<uint32_t>(__cvta_generic_to_shared(p))));
}
__device__ __forceinline__ void ldsm_x4_t(const __half* p, uint32_t (&r)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(static_cast<uint32_t>(__cvta_generic_to_shared(p))));
}

__global__ void __launch_bounds__(128, 3) attn_prefill_kernel(const PfArgs a) {
  extern __shared__ __align__(16) uint8_t pf_smem[];
  __half* kbuf = reinterpret_cast<__half*>(pf_smem);  // [buffer][K, V][key][dim], pitch kPfP
  pdl_trigger();
  pdl_wait();

  const int4 u = a.units[blockIdx.x];
  const int h = blockIdx.y;
  const int row0 = u.x, n = u.y, slot = u.z, p0 = u.w;
  const int plast = p0 + n - 1;
  if (n < 1 || n > kPfRows || row0 < 0 || row0 + n > a.M || p0 < 0 || plast >= a.max_seq) {
    if (threadIdx.x == 0) atomicOr(a.check, 2u);
    return;
  }
  if (slot < 0 || slot >= a.num_slots) {
    if (threadIdx.x == 0) atomicOr(a.check, 8u);
    return;
  }
  const int H = a.nh * kPfHD;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 2, c = lane & 3;
  const size_t base = ((size_t)slot * a.nh + h) * a.max_seq * kPfHD;
  const int nkb = plast / kPfKeys + 1;

  // K and V rows of block kb into buffer kb & 1 (keys past plast zero-filled, not read)
  auto issue = [&](int kb) {
    __half* kd = kbuf + (kb & 1) * 2 * kPfTile;
    __half* vd = kd + kPfTile;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int i = tid + 128 * j, r = i >> 4, d8 = (i & 15) * 8, key = kb * kPfKeys + r;
      const bool ok = key <= plast;
      const size_t off = ok ? base + (size_t)key * kPfHD + d8 : 0;
      pf_cp16(kd + r * kPfP + d8, a.kc + off, ok);
      pf_cp16(vd + r * kPfP + d8, a.vc + off, ok);
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
  };
  issue(0);

  // Q rows through buffer 1's K area, then into registers (A fragments of 16 rows x 16 dims)
  __half* qs = kbuf + 2 * kPfTile;
  for (int i = tid; i < kPfRows * (kPfHD / 8); i += 128) {
    const int r = i >> 4, d8 = (i & 15) * 8;
    uint4 v = make_uint4(0u, 0u, 0u, 0u);
    if (r < n) v = *reinterpret_cast<const uint4*>(a.q + (size_t)(row0 + r) * H + h * kPfHD + d8);
    *reinterpret_cast<uint4*>(qs + r * kPfP + d8) = v;
  }
  __syncthreads();
  const int qr = warp * 16 + g;  // this thread's rows: qr and qr + 8
  uint32_t qa[kPfHD / 16][4];
#pragma unroll
  for (int kk = 0; kk < kPfHD / 16; ++kk) {
    qa[kk][0] = ld_h2(qs + qr * kPfP + 16 * kk + 2 * c);
    qa[kk][1] = ld_h2(qs + (qr + 8) * kPfP + 16 * kk + 2 * c);
    qa[kk][2] = ld_h2(qs + qr * kPfP + 16 * kk + 8 + 2 * c);
    qa[kk][3] = ld_h2(qs + (qr + 8) * kPfP + 16 * kk + 8 + 2 * c);
  }
  __syncthreads();  // buffer 1 is free for block 1

  float o[kPfHD / 8][4];
#pragma unroll
  for (int d = 0; d < kPfHD / 8; ++d) o[d][0] = o[d][1] = o[d][2] = o[d][3] = 0.f;
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;
  const float scale = rsqrtf((float)kPfHD);
  const int qp0 = p0 + qr, qp1 = p0 + qr + 8;  // positions of the two rows
  // ldmatrix row addresses of this lane: matrix lane >> 3, row lane & 7
  const int lm = lane >> 3, lr = lane & 7;

  for (int kb = 0; kb < nkb; ++kb) {
    const int k0 = kb * kPfKeys;
    if (kb + 1 < nkb) {
      issue(kb + 1);
      asm volatile("cp.async.wait_group 1;" ::: "memory");
    } else {
      asm volatile("cp.async.wait_group 0;" ::: "memory");
    }
    __syncthreads();  // block kb's rows from every thread's copies
    const __half* ks = kbuf + (kb & 1) * 2 * kPfTile;
    const __half* vs = ks + kPfTile;

    // S = Q K^T for this warp's 16 rows x 64 keys (8 tiles of 8 keys). ldmatrix x4 per key
    // tile and dim pair kk, kk + 1: matrices (dims 16kk, +8, 16kk + 16, +24) of keys 8t..8t+7
    float sc[kPfKeys / 8][4];
#pragma unroll
    for (int t = 0; t < kPfKeys / 8; ++t) {
      sc[t][0] = sc[t][1] = sc[t][2] = sc[t][3] = 0.f;
#pragma unroll
      for (int kk = 0; kk < kPfHD / 16; kk += 2) {
        uint32_t b[4];
        ldsm_x4(ks + (8 * t + lr) * kPfP + 16 * kk + 8 * lm, b);
        mma_16816(sc[t], qa[kk][0], qa[kk][1], qa[kk][2], qa[kk][3], b[0], b[1]);
        mma_16816(sc[t], qa[kk + 1][0], qa[kk + 1][1], qa[kk + 1][2], qa[kk + 1][3], b[2], b[3]);
      }
    }
    // scale, causal mask, running max
    float bm0 = -INFINITY, bm1 = -INFINITY;
#pragma unroll
    for (int t = 0; t < kPfKeys / 8; ++t)
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int key = k0 + 8 * t + 2 * c + e;
        sc[t][e] = (key <= qp0 && key <= plast) ? sc[t][e] * scale : -INFINITY;
        sc[t][2 + e] = (key <= qp1 && key <= plast) ? sc[t][2 + e] * scale : -INFINITY;
        bm0 = fmaxf(bm0, sc[t][e]);
        bm1 = fmaxf(bm1, sc[t][2 + e]);
      }
#pragma unroll
    for (int o2 = 1; o2 <= 2; o2 <<= 1) {
      bm0 = fmaxf(bm0, __shfl_xor_sync(0xffffffffu, bm0, o2));
      bm1 = fmaxf(bm1, __shfl_xor_sync(0xffffffffu, bm1, o2));
    }
    // key 0 is in block 0 and valid for every row, so the running max is finite from here on
    const float mn0 = fmaxf(m0, bm0), mn1 = fmaxf(m1, bm1);
    const float al0 = expf(m0 - mn0), al1 = expf(m1 - mn1);
    m0 = mn0;
    m1 = mn1;
    float rs0 = 0.f, rs1 = 0.f;
#pragma unroll
    for (int t = 0; t < kPfKeys / 8; ++t) {
      sc[t][0] = expf(sc[t][0] - mn0);
      sc[t][1] = expf(sc[t][1] - mn0);
      sc[t][2] = expf(sc[t][2] - mn1);
      sc[t][3] = expf(sc[t][3] - mn1);
      rs0 += sc[t][0] + sc[t][1];
      rs1 += sc[t][2] + sc[t][3];
    }
    l0 = l0 * al0 + rs0;
    l1 = l1 * al1 + rs1;
#pragma unroll
    for (int d = 0; d < kPfHD / 8; ++d) {
      o[d][0] *= al0;
      o[d][1] *= al0;
      o[d][2] *= al1;
      o[d][3] *= al1;
    }
    // O += P V: keys 16 j .. 16 j + 15 per k-step; P from the score tiles 2 j, 2 j + 1. V by
    // ldmatrix.trans, x4 per dim pair d, d + 1: matrices (keys 16j, 16j + 8) x (dims 8d, 8d + 8)
#pragma unroll
    for (int j = 0; j < kPfKeys / 16; ++j) {
      const float* s0 = sc[2 * j];
      const float* s1 = sc[2 * j + 1];
      uint32_t hi[4], lo[4];
      {
        const float pv[8] = {s0[0], s0[1], s0[2], s0[3], s1[0], s1[1], s1[2], s1[3]};
        float ph[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) ph[e] = __half2float(__float2half_rn(pv[e]));
        hi[0] = pack_h2(ph[0], ph[1]);
        hi[1] = pack_h2(ph[2], ph[3]);
        hi[2] = pack_h2(ph[4], ph[5]);
        hi[3] = pack_h2(ph[6], ph[7]);
        lo[0] = pack_h2(pv[0] - ph[0], pv[1] - ph[1]);
        lo[1] = pack_h2(pv[2] - ph[2], pv[3] - ph[3]);
        lo[2] = pack_h2(pv[4] - ph[4], pv[5] - ph[5]);
        lo[3] = pack_h2(pv[6] - ph[6], pv[7] - ph[7]);
      }
#pragma unroll
      for (int d = 0; d < kPfHD / 8; d += 2) {
        uint32_t b[4];
        ldsm_x4_t(vs + (16 * j + 8 * (lm & 1) + lr) * kPfP + 8 * d + 8 * (lm >> 1), b);
        mma_16816(o[d], hi[0], hi[1], hi[2], hi[3], b[0], b[1]);
        mma_16816(o[d], lo[0], lo[1], lo[2], lo[3], b[0], b[1]);
        mma_16816(o[d + 1], hi[0], hi[1], hi[2], hi[3], b[2], b[3]);
        mma_16816(o[d + 1], lo[0], lo[1], lo[2], lo[3], b[2], b[3]);
      }
    }
    __syncthreads();  // every warp is done with buffer kb & 1 before block kb + 2 is copied in
  }

#pragma unroll
  for (int o2 = 1; o2 <= 2; o2 <<= 1) {
    l0 += __shfl_xor_sync(0xffffffffu, l0, o2);
    l1 += __shfl_xor_sync(0xffffffffu, l1, o2);
  }
  const float inv0 = 1.0f / l0, inv1 = 1.0f / l1;
#pragma unroll
  for (int d = 0; d < kPfHD / 8; ++d) {
    const int col = h * kPfHD + 8 * d + 2 * c;
    if (qr < n)
      *reinterpret_cast<__half2*>(a.out + (size_t)(row0 + qr) * H + col) = __floats2half2_rn(o[d][0] * inv0, o[d][1] * inv0);
    if (qr + 8 < n)
      *reinterpret_cast<__half2*>(a.out + (size_t)(row0 + qr + 8) * H + col) =
          __floats2half2_rn(o[d][2] * inv1, o[d][3] * inv1);
  }
}

}  // namespace

}  // namespace orch

using namespace orch;

// No counterpart in the reference (its prefill attention is the per-token host NumPy loop of
// orchard/model.py:112-144).
extern "C" int orch_attention_prefill(const void* q, const void* k_cache, const void* v_cache, const int32_t* units,
                                      uint32_t num_units, void* out, uint32_t M, uint32_t num_heads,
                                      uint32_t head_dim, uint32_t max_seq, uint32_t num_slots, void* stream) {
  if (num_units == 0 || M == 0) return ORCH_OK;
  ORCH_REQUIRE(q && k_cache && v_cache && units && out, "attention_prefill: null pointer");
  ORCH_REQUIRE(((uintptr_t)units & 15) == 0, "attention_prefill: units must be 16-byte aligned");
  ORCH_REQUIRE(num_heads > 0 && num_heads <= 65535 && max_seq > 0 && num_slots > 0 && num_slots <= 0x7fffffffu,
               "attention_prefill: bad shape");
  if (head_dim != (uint32_t)kPfHD) return fail(ORCH_ERR_UNSUPPORTED, "attention_prefill: head_dim must be 128");
  static bool attr_done[64] = {};
  const int dev = device_index();
  if (dev >= 0 && dev < 64 && !attr_done[dev]) {
    ORCH_CUDA(cudaFuncSetAttribute(attn_prefill_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kPfSmem));
    attr_done[dev] = true;
  }
  PfArgs a;
  a.q = static_cast<const __half*>(q);
  a.kc = static_cast<const __half*>(k_cache);
  a.vc = static_cast<const __half*>(v_cache);
  a.units = reinterpret_cast<const int4*>(units);
  a.out = static_cast<__half*>(out);
  a.M = (int)M;
  a.nh = (int)num_heads;
  a.max_seq = (int)max_seq;
  a.num_slots = (int)num_slots;
  ORCH_CHECK_WORD(a.check);
  ORCH_CUDA(launch_k_serial(attn_prefill_kernel, dim3(num_units, num_heads), dim3(128), kPfSmem, as_stream(stream),
                            dim3(0, 0, 0), a));
  return check_launch("attention_prefill");
}
