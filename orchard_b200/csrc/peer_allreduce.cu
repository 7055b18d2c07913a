// Sum of an fp32 buffer over the ranks of one box through peer memory (NVLink / NVSwitch),
// for the head split's two all-reduces of the residual per layer.
//
// The reference runs on one device and has no collective; the split's order of operations
// (orchard_b200/parallel.py) names an all-reduce after the O and the down projections. At
// decode sizes (16 KB per row) a library all-reduce is latency-bound, so this one takes a
// single launch and one NVLink crossing:
//
//  * every rank owns a region (cudaMalloc'd here, mapped by the other ranks through CUDA
//    IPC): a header (call counter, block counter), flags [8 ranks][64 blocks] and two
//    banks of receive slots [2][world][cap] fp32, used on alternate calls;
//  * block b of rank r stores its chunk of x into slot r of bank (call & 1) on every rank
//    (plain stores over NVLink; no multicast), then, after a system-scope fence, writes
//    the call number into flag [r][b] on every rank with a release store;
//  * it waits (acquire loads, bounded by ~5 s of globaltimer) until flag [q][b] of its own
//    region holds this call's number for every rank q, and writes x = sum over q of slot q,
//    added in rank order: every rank computes the same bits.
//
// Two banks suffice: a rank can only start call k + 2 after every rank's flags of call
// k + 1, which each rank writes after its call k (the one reading bank k & 1) has ended.
// On a wait that runs out the block sets device check bit 512, sums what it has and the
// call counters still advance.
#include <algorithm>
#include <cstring>

#include "orch_common.cuh"

namespace orch {

constexpr int kArMaxRanks = 8;
constexpr int kArMaxBlocks = 64;
constexpr int kArThreads = 256;
constexpr size_t kArFlagsOff = 256;   // after the header: epoch, block counter
constexpr size_t kArSlotsOff = 4096;  // flags take 8 x 64 x 4 = 2 KB

struct ArArgs {
  char* base[kArMaxRanks];  // every rank's region as mapped on this device (own included)
  float* x;
  uint32_t* check;
  int rank, world;
  int n4;       // float4s to reduce
  int per_blk;  // float4s per block
  size_t cap4;  // float4s per receive slot
};

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

__global__ void __launch_bounds__(kArThreads) peer_allreduce_kernel(ArArgs a) {
  pdl_wait();  // x is the previous kernel's output
  char* own = a.base[a.rank];
  uint32_t* hdr = reinterpret_cast<uint32_t*>(own);
  const uint32_t e = *reinterpret_cast<volatile uint32_t*>(hdr) + 1u;  // this call's number
  const size_t bank = e & 1u;
  const int b = blockIdx.x;
  const int i0 = b * a.per_blk;
  const int i1 = min(a.n4, i0 + a.per_blk);
  const float4* x4 = reinterpret_cast<const float4*>(a.x);

  // 1. this rank's chunk into slot `rank` of the bank, on every rank
  const size_t my_slot = (bank * a.world + a.rank) * a.cap4;
  for (int i = i0 + threadIdx.x; i < i1; i += kArThreads) {
    const float4 v = x4[i];
    for (int q = 0; q < a.world; ++q)
      reinterpret_cast<float4*>(a.base[q] + kArSlotsOff)[my_slot + i] = v;
  }
  __syncthreads();
  // 2. publish: flag [rank][b] = e on every rank, after a system-scope fence
  if (threadIdx.x < a.world) {
    __threadfence_system();
    uint32_t* f = reinterpret_cast<uint32_t*>(a.base[threadIdx.x] + kArFlagsOff) + a.rank * kArMaxBlocks + b;
    st_release_sys(f, e);
  }
  // 3. wait for every rank's chunk b in this rank's region (bounded)
  if (threadIdx.x < a.world) {
    const uint32_t* f = reinterpret_cast<const uint32_t*>(own + kArFlagsOff) + threadIdx.x * kArMaxBlocks + b;
    const uint64_t t0 = global_ns();
    while ((int32_t)(ld_acquire_sys(f) - e) < 0) {
      if (global_ns() - t0 > 5000000000ull) {
        atomicOr(a.check, 512u);
        break;
      }
      __nanosleep(32);
    }
  }
  __syncthreads();
  // 4. x = sum of the slots in rank order (L2 loads: peers wrote them over NVLink)
  const float4* slots = reinterpret_cast<const float4*>(own + kArSlotsOff) + bank * a.world * a.cap4;
  float4* xo = reinterpret_cast<float4*>(a.x);
  for (int i = i0 + threadIdx.x; i < i1; i += kArThreads) {
    float4 s = __ldcg(slots + i);
    for (int q = 1; q < a.world; ++q) {
      const float4 v = __ldcg(slots + (size_t)q * a.cap4 + i);
      s.x += v.x;
      s.y += v.y;
      s.z += v.z;
      s.w += v.w;
    }
    xo[i] = s;
  }
  // 5. the last block advances this rank's call counter (every block has read it)
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

}  // namespace orch

using namespace orch;

extern "C" size_t orch_peer_region_bytes(uint32_t world, uint32_t max_floats) {
  if (world == 0 || world > (uint32_t)kArMaxRanks) return 0;
  const size_t cap = ((size_t)max_floats + 3) / 4 * 4;
  return kArSlotsOff + 2 * (size_t)world * cap * sizeof(float);
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
                                   float* x, uint32_t n, void* stream) {
  if (n == 0) return ORCH_OK;
  ORCH_REQUIRE(bases && x, "peer_allreduce: null pointer");
  ORCH_REQUIRE(world >= 1 && world <= (uint32_t)kArMaxRanks && rank < world, "peer_allreduce: bad rank / world");
  ORCH_REQUIRE(n % 4 == 0 && max_floats % 4 == 0 && n <= max_floats,
               "peer_allreduce: n and max_floats must be multiples of 4, n <= max_floats");
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
  a.n4 = (int)(n / 4);
  a.cap4 = max_floats / 4;
  // a block per 1024 float4s (4 per thread), at most 64
  const int nb = std::min(kArMaxBlocks, std::max(1, (a.n4 + 1023) / 1024));
  a.per_blk = (a.n4 + nb - 1) / nb;
  ORCH_CUDA(launch_k(peer_allreduce_kernel, dim3(nb), dim3(kArThreads), 0, as_stream(stream), dim3(0, 0, 0), a));
  return check_launch("peer_allreduce");
}
