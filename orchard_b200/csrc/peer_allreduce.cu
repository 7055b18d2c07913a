// Sum of an fp32 buffer over the ranks of one box through peer memory (NVLink / NVSwitch),
// for the head split's two all-reduces of the residual per layer. One shot is described
// here; the two-shot form for larger buffers on more ranks is described at its kernel.
//
// The reference runs on one device and has no collective; the split's order of operations
// (orchard_b200/parallel.py) names an all-reduce after the O and the down projections. At
// decode sizes (16 KB per row) a library all-reduce is latency-bound, so this one takes a
// single launch and one NVLink crossing, with no fence and no separate flag:
//
//  * every rank owns a region (cudaMalloc'd by the caller, mapped by the other ranks through
//    CUDA IPC): a header (call counter, block counter) and two banks of receive slots
//    [2][world][cap] of 64-bit words, used on alternate calls;
//  * each word carries one fp32 value in its low half and the call number in its high half,
//    so one aligned 8-byte store delivers both at once (single-copy atomic);
//  * thread j of rank r stores its two values of x into slot r of bank (call & 1) on every
//    rank (16-byte relaxed system-scope stores over NVLink; no multicast), then polls the
//    same two words of every slot q in its own region (relaxed system-scope loads, all ranks'
//    loads in flight together, bounded by ~5 s of globaltimer) until they carry this call's
//    number, and writes x = sum over q, added in rank order: every rank computes the same bits.
//
// Two banks suffice: a rank can only start call k + 2 after it has read every rank's words
// of call k + 1, which each rank writes after its call k (the one reading bank k & 1) has
// ended. On a wait that runs out the thread sets device check bit 512 and sums what it has;
// the call counters still advance.
#include <algorithm>
#include <cstring>

#include "orch_common.cuh"

namespace orch {

constexpr int kArMaxRanks = 8;
constexpr int kArMaxBlocks = 296;  // two blocks per SM: always co-resident (launch bounds below)
constexpr int kArThreads = 256;
constexpr size_t kArSlotsOff = 4096;  // after the header: call counter, block counter

struct ArArgs {
  char* base[kArMaxRanks];  // every rank's region as mapped on this device (own included)
  float* x;
  uint32_t* check;
  int rank, world;
  int npairs;   // pairs of floats to reduce
  size_t cap2;  // pairs per receive slot
};

__device__ __forceinline__ void st_relaxed_sys_v2(uint64_t* p, uint64_t a, uint64_t b) {
  asm volatile("st.relaxed.sys.global.v2.u64 [%0], {%1, %2};" ::"l"(p), "l"(a), "l"(b) : "memory");
}
__device__ __forceinline__ void ld_relaxed_sys_v2(const uint64_t* p, uint64_t& a, uint64_t& b) {
  asm volatile("ld.relaxed.sys.global.v2.u64 {%0, %1}, [%2];" : "=l"(a), "=l"(b) : "l"(p) : "memory");
}
__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}
__device__ __forceinline__ uint64_t ll_word(float v, uint32_t e) {
  return ((uint64_t)e << 32) | (uint64_t)__float_as_uint(v);
}

// Polls the words of pair j from the slots of every rank q in `qmask` (slot q at
// base + 2 (q * qstride + j) 64-bit words) until they carry call number e, all loads in
// flight together; bounded by ~5 s of globaltimer (then check bit 512, and whatever arrived).
__device__ __forceinline__ void poll_pairs(const uint64_t* base, size_t qstride, size_t j, uint32_t qmask,
                                           uint32_t e, uint64_t (&w)[kArMaxRanks][2], uint32_t* check) {
  uint32_t pending = 0;
#pragma unroll
  for (int q = 0; q < kArMaxRanks; ++q)
    if (qmask & (1u << q)) {
      ld_relaxed_sys_v2(base + 2 * ((size_t)q * qstride + j), w[q][0], w[q][1]);
      if ((uint32_t)(w[q][0] >> 32) != e || (uint32_t)(w[q][1] >> 32) != e) pending |= 1u << q;
    }
  if (!pending) return;
  const uint64_t t0 = global_ns();
  while (pending) {
#pragma unroll
    for (int q = 0; q < kArMaxRanks; ++q)
      if (pending & (1u << q)) {
        ld_relaxed_sys_v2(base + 2 * ((size_t)q * qstride + j), w[q][0], w[q][1]);
        if ((uint32_t)(w[q][0] >> 32) == e && (uint32_t)(w[q][1] >> 32) == e) pending &= ~(1u << q);
      }
    if (pending && global_ns() - t0 > 5000000000ull) {
      atomicOr(check, 512u);
      return;
    }
  }
}

// Rank-ordered sum of the polled pairs of the ranks in qmask (bit 0 always set).
__device__ __forceinline__ float2 sum_pairs(const uint64_t (&w)[kArMaxRanks][2], uint32_t qmask) {
  float2 s = make_float2(__uint_as_float((uint32_t)w[0][0]), __uint_as_float((uint32_t)w[0][1]));
#pragma unroll
  for (int q = 1; q < kArMaxRanks; ++q)
    if (qmask & (1u << q)) {
      s.x += __uint_as_float((uint32_t)w[q][0]);
      s.y += __uint_as_float((uint32_t)w[q][1]);
    }
  return s;
}

// The last block to finish advances this rank's call counter (every block has read it).
__device__ __forceinline__ void advance_call(uint32_t* hdr, uint32_t e) {
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    const uint32_t done = atomicAdd(hdr + 1, 1u);
    if (done == gridDim.x - 1) {
      hdr[1] = 0u;
      *reinterpret_cast<volatile uint32_t*>(hdr) = e;
    }
  }
}

// One shot: every rank's whole buffer to every rank, each rank sums all of it.
__global__ void __launch_bounds__(kArThreads, 2) peer_allreduce_kernel(ArArgs a) {
  pdl_wait();  // x is the previous kernel's output
  char* own = a.base[a.rank];
  uint32_t* hdr = reinterpret_cast<uint32_t*>(own);
  const uint32_t e = *reinterpret_cast<volatile uint32_t*>(hdr) + 1u;  // this call's number
  const size_t bank = e & 1u;
  const int stride = gridDim.x * kArThreads;
  const float2* x2 = reinterpret_cast<const float2*>(a.x);
  float2* xo = reinterpret_cast<float2*>(a.x);
  const uint32_t all = (1u << a.world) - 1u;

  // 1. this rank's values into slot `rank` of the bank, on every rank
  const size_t my_slot = (bank * a.world + a.rank) * a.cap2;
  for (int j = blockIdx.x * kArThreads + threadIdx.x; j < a.npairs; j += stride) {
    const float2 v = x2[j];
    const uint64_t w0 = ll_word(v.x, e), w1 = ll_word(v.y, e);
#pragma unroll
    for (int q = 0; q < kArMaxRanks; ++q)
      if (q < a.world)
        st_relaxed_sys_v2(reinterpret_cast<uint64_t*>(a.base[q] + kArSlotsOff) + 2 * (my_slot + j), w0, w1);
  }
  // 2. every rank's values of the same pairs from this rank's region, summed in rank order
  const uint64_t* slots = reinterpret_cast<const uint64_t*>(own + kArSlotsOff) + 2 * bank * a.world * a.cap2;
  for (int j = blockIdx.x * kArThreads + threadIdx.x; j < a.npairs; j += stride) {
    uint64_t w[kArMaxRanks][2];
    poll_pairs(slots, a.cap2, j, all, e, w, a.check);
    xo[j] = sum_pairs(w, all);
  }
  advance_call(hdr, e);
}

// Two shots, for larger buffers on more ranks: the pairs are cut into `world` chunks of cp;
// rank r sums chunk r (reduce-scatter: chunk q of every rank goes to rank q only) and sends
// the sum to every rank (all-gather). Per rank 16 n (world - 1) / world bytes cross NVLink
// instead of 8 n (world - 1). In the bank of this call, slot q of the first half holds rank
// q's part of this rank's chunk, slot q of the second half rank q's summed chunk (cs pairs
// each). Thread j handles pair j of every chunk, so the ranks' threads j depend only on one
// another: their first stores come before any wait.
__global__ void __launch_bounds__(kArThreads, 2) peer_allreduce2_kernel(ArArgs a, int cp, int cs) {
  pdl_wait();
  char* own = a.base[a.rank];
  uint32_t* hdr = reinterpret_cast<uint32_t*>(own);
  const uint32_t e = *reinterpret_cast<volatile uint32_t*>(hdr) + 1u;
  const size_t bank0 = (size_t)(e & 1u) * a.world * a.cap2;  // pairs
  const int stride = gridDim.x * kArThreads;
  float2* x2 = reinterpret_cast<float2*>(a.x);
  const uint64_t* mine = reinterpret_cast<const uint64_t*>(own + kArSlotsOff);
  for (int j = blockIdx.x * kArThreads + threadIdx.x; j < cp; j += stride) {
    // 1. pair j of chunk q to rank q, first half, slot `rank`
#pragma unroll
    for (int q = 0; q < kArMaxRanks; ++q) {
      const int idx = q * cp + j;
      if (q < a.world && idx < a.npairs) {
        const float2 v = x2[idx];
        st_relaxed_sys_v2(reinterpret_cast<uint64_t*>(a.base[q] + kArSlotsOff) + 2 * (bank0 + (size_t)a.rank * cs + j),
                          ll_word(v.x, e), ll_word(v.y, e));
      }
    }
    // 2. this rank's chunk: every rank's part, summed in rank order, to every rank's second half
    const int idx_r = a.rank * cp + j;
    const uint32_t all = (1u << a.world) - 1u;
    uint64_t w[kArMaxRanks][2];
    if (idx_r < a.npairs) {
      poll_pairs(mine + 2 * bank0, cs, j, all, e, w, a.check);
      const float2 r = sum_pairs(w, all);
      const uint64_t w0 = ll_word(r.x, e), w1 = ll_word(r.y, e);
#pragma unroll
      for (int q = 0; q < kArMaxRanks; ++q)
        if (q < a.world)
          st_relaxed_sys_v2(reinterpret_cast<uint64_t*>(a.base[q] + kArSlotsOff) +
                                2 * (bank0 + (size_t)(a.world + a.rank) * cs + j),
                            w0, w1);
    }
    // 3. every chunk's sum: pair j of chunk q from slot q of the second half
    uint32_t have = 0;
#pragma unroll
    for (int q = 0; q < kArMaxRanks; ++q)
      if (q < a.world && q * cp + j < a.npairs) have |= 1u << q;
    poll_pairs(mine + 2 * (bank0 + (size_t)a.world * cs), cs, j, have, e, w, a.check);
#pragma unroll
    for (int q = 0; q < kArMaxRanks; ++q)
      if (have & (1u << q))
        x2[q * cp + j] = make_float2(__uint_as_float((uint32_t)w[q][0]), __uint_as_float((uint32_t)w[q][1]));
  }
  advance_call(hdr, e);
}

}  // namespace orch

using namespace orch;

extern "C" size_t orch_peer_region_bytes(uint32_t world, uint32_t max_floats) {
  if (world == 0 || world > (uint32_t)kArMaxRanks) return 0;
  const size_t cap = ((size_t)max_floats + 3) / 4 * 4;
  return kArSlotsOff + 2 * (size_t)world * cap * sizeof(uint64_t);  // a word per value
}

extern "C" int orch_ipc_handle(void* base, void* handle_out) {
  ORCH_REQUIRE(base && handle_out, "ipc_handle: null pointer");
  cudaIpcMemHandle_t h;
  ORCH_CUDA(cudaIpcGetMemHandle(&h, base));
  std::memcpy(handle_out, &h, sizeof(h));
  return ORCH_OK;
}

extern "C" int orch_ipc_open(const void* handle, void** base_out) {
  ORCH_REQUIRE(handle && base_out, "ipc_open: null pointer");
  *base_out = nullptr;
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  ORCH_CUDA(cudaIpcOpenMemHandle(base_out, h, cudaIpcMemLazyEnablePeerAccess));
  return ORCH_OK;
}

extern "C" int orch_ipc_close(void* base) {
  if (base) ORCH_CUDA(cudaIpcCloseMemHandle(base));
  return ORCH_OK;
}

extern "C" int orch_peer_allreduce(void* const* bases, uint32_t rank, uint32_t world, uint32_t max_floats,
                                   float* x, uint32_t n, int algo, void* stream) {
  if (n == 0) return ORCH_OK;
  ORCH_REQUIRE(bases && x, "peer_allreduce: null pointer");
  ORCH_REQUIRE(world >= 1 && world <= (uint32_t)kArMaxRanks && rank < world, "peer_allreduce: bad rank / world");
  ORCH_REQUIRE(n % 4 == 0 && max_floats % 4 == 0 && n <= max_floats,
               "peer_allreduce: n and max_floats must be multiples of 4, n <= max_floats");
  ORCH_REQUIRE(algo >= 0 && algo <= 2, "peer_allreduce: algo must be 0 (automatic), 1 or 2");
  ORCH_REQUIRE(((uintptr_t)x & 15) == 0, "peer_allreduce: x must be 16-byte aligned");
  ArArgs a = {};
  for (uint32_t q = 0; q < world; ++q) {
    ORCH_REQUIRE(bases[q] != nullptr && ((uintptr_t)bases[q] & 255) == 0,
                 "peer_allreduce: every rank's region must be non-null and 256-byte aligned");
    a.base[q] = static_cast<char*>(bases[q]);
  }
  ORCH_CHECK_WORD(a.check);
  a.x = x;
  a.rank = (int)rank;
  a.world = (int)world;
  a.npairs = (int)(n / 2);
  a.cap2 = max_floats / 2;
  // two shots' slots (2 world cs pairs per bank) must fit the bank of world cap2 pairs
  const int cs = (int)((a.cap2 + world - 1) / world);
  const bool fits2 = world > 1 && 2 * (size_t)cs <= a.cap2;
  if (algo == 0)  // one shot while what it sends stays small (and always on two ranks)
    algo = (world <= 2 || (size_t)8 * n * (world - 1) <= ((size_t)1 << 20) || !fits2) ? 1 : 2;
  if (algo == 2) {
    ORCH_REQUIRE(fits2, "peer_allreduce: max_floats too small for two shots");
    const int cp = (a.npairs + (int)world - 1) / (int)world;
    const int nb = std::min(kArMaxBlocks, std::max(1, (cp + kArThreads - 1) / kArThreads));
    ORCH_CUDA(launch_k(peer_allreduce2_kernel, dim3(nb), dim3(kArThreads), 0, as_stream(stream), dim3(0, 0, 0), a,
                       cp, cs));
    return check_launch("peer_allreduce");
  }
  // a thread per pair of values, at most two blocks per SM (larger buffers loop)
  const int nb = std::min(kArMaxBlocks, std::max(1, (a.npairs + kArThreads - 1) / kArThreads));
  ORCH_CUDA(launch_k(peer_allreduce_kernel, dim3(nb), dim3(kArThreads), 0, as_stream(stream), dim3(0, 0, 0), a));
  return check_launch("peer_allreduce");
}
