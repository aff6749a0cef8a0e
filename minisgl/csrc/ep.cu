// Expert-parallel token dispatch and return over NVLink peer memory.
//
// Every rank owns a heap (CUDA IPC, mapped by every peer):
//   [signals 4 KB][recv ids: world x cap int32][recv rows: world x cap x H
//   bf16][back rows: cap x H bf16]
// where cap is the pair capacity of one rank's step (tokens x k).
//
//   dispatch (on every rank, one warp per pair slot p < cap): the pair's
//     hidden row goes to its expert owner's recv rows [me][p] (peer stores)
//     and every rank's recv ids [me][p] gets the local expert id (owner) or
//     -1 (everyone else, and slots past this step's pairs); a grid barrier
//     then signals every peer and waits (bounded) for all peers' signals.
//   (the owner runs its experts over its recv rows; -1 rows are dropped by
//     the align kernel)
//   return (one warp per received slot): each valid result row goes back to
//     the source rank's back rows [p]; barrier again. The source then sums
//     each token's k back rows weighted by the router (the MoE combine).
//
// Single buffers are safe: a rank writes its peers' recv rows of step n + 1
// only after the return barrier of step n, which every peer passes only
// after its experts (the readers of recv rows) finished; and back rows of
// step n + 1 are written after the dispatch barrier of step n + 1, which a
// source reaches after its step-n combine. Waits give up after two seconds
// and record kErrPeerTimeout (no trap, no hang). No multicast objects.
#include <cuda_runtime.h>

#include <algorithm>
#include <stdexcept>

#include "common.cuh"
#include "launch.h"
#include "ops.h"

namespace minisgl {
namespace {

constexpr int kEpMaxRanks = 8;
// uint32 slots of the signal page
constexpr int kSigDispatch = 64, kSigReturn = 80, kCtaDone = 96;

__device__ __forceinline__ void st_release_sys_u32(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys_u32(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ uint8_t* heap(const EpArgs& a, int r) {
  return reinterpret_cast<uint8_t*>(a.bases[r]);
}
__device__ __forceinline__ int32_t* recv_ids(const EpArgs& a, int r) {
  return reinterpret_cast<int32_t*>(heap(a, r) + a.ids_off);
}
__device__ __forceinline__ uint4* recv_rows(const EpArgs& a, int r) {
  return reinterpret_cast<uint4*>(heap(a, r) + a.rows_off);
}
__device__ __forceinline__ uint4* back_rows(const EpArgs& a, int r) {
  return reinterpret_cast<uint4*>(heap(a, r) + a.back_off);
}

// The last CTA of the grid to finish signals every peer (slot `which` +
// rank) with this call's epoch and waits until every peer has signalled.
__device__ void grid_barrier_peers(const EpArgs& a, int which, int site) {
  __shared__ bool last;
  __threadfence_system();  // this CTA's peer stores are visible before the count
  __syncthreads();
  if (threadIdx.x == 0) {
    uint32_t* done = reinterpret_cast<uint32_t*>(heap(a, a.rank)) + kCtaDone + (which == kSigDispatch ? 0 : 1);
    last = atomicAdd(done, 1u) == gridDim.x - 1;
    if (last) *done = 0;  // ready for the next call (which starts after this kernel)
  }
  __syncthreads();
  if (!last) return;
  const uint32_t e = *a.epoch + 1;
  if (threadIdx.x < a.world) {
    __threadfence_system();
    st_release_sys_u32(reinterpret_cast<uint32_t*>(heap(a, threadIdx.x)) + which + a.rank, e);
    const uint32_t* mine = reinterpret_cast<const uint32_t*>(heap(a, a.rank)) + which + threadIdx.x;
    const uint64_t t0 = globaltimer_ns();
    uint32_t it = 0;
    while (static_cast<int32_t>(ld_acquire_sys_u32(mine) - e) < 0) {
      if (((++it) & 0xFFu) == 0 && globaltimer_ns() - t0 > kWaitBudgetNs) {
        ErrorSink{a.err}.report(kErrPeerTimeout, site + static_cast<int>(threadIdx.x));
        break;
      }
    }
  }
}

// one warp per pair slot of this rank
__global__ void __launch_bounds__(256) ep_dispatch_kernel(EpArgs a) {
  pdl_launch_dependents();
  pdl_wait();
  const int lane = threadIdx.x & 31;
  const int p = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (p < a.cap) {
    const int pairs = a.T * a.k;
    int owner = -1, le = -1;
    if (p < pairs) {
      const int id = a.topk_ids[p];
      owner = id / a.e_local;
      le = id - owner * a.e_local;
      if (owner < 0 || owner >= a.world) owner = -1;  // an id outside the model: dropped
    }
    if (lane < a.world) recv_ids(a, lane)[static_cast<int64_t>(a.rank) * a.cap + p] = lane == owner ? le : -1;
    if (owner >= 0) {
      const int vecs = a.H / 8;
      const uint4* src = reinterpret_cast<const uint4*>(a.x) + static_cast<int64_t>(p / a.k) * vecs;
      uint4* dst = recv_rows(a, owner) + (static_cast<int64_t>(a.rank) * a.cap + p) * vecs;
      for (int v = lane; v < vecs; v += 32) dst[v] = src[v];
    }
  }
  grid_barrier_peers(a, kSigDispatch, 500);
}

// one warp per received slot q = src * cap + p
__global__ void __launch_bounds__(256) ep_return_kernel(EpArgs a) {
  pdl_launch_dependents();
  pdl_wait();
  const int lane = threadIdx.x & 31;
  const int64_t q = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (q < static_cast<int64_t>(a.world) * a.cap && recv_ids(a, a.rank)[q] >= 0) {
    const int src = static_cast<int>(q / a.cap);
    const int p = static_cast<int>(q - static_cast<int64_t>(src) * a.cap);
    const int r = a.pair_pos[q];
    if (r >= 0) {
      const int vecs = a.H / 8;
      const uint4* from = reinterpret_cast<const uint4*>(a.ys) + static_cast<int64_t>(r) * vecs;
      uint4* to = back_rows(a, src) + static_cast<int64_t>(p) * vecs;
      for (int v = lane; v < vecs; v += 32) to[v] = from[v];
    }
  }
  grid_barrier_peers(a, kSigReturn, 520);
}

__global__ void ep_bump_kernel(uint32_t* epoch) {
  pdl_launch_dependents();
  pdl_wait();
  *epoch += 1;
}

}  // namespace

void launch_ep_dispatch(const EpArgs& a, cudaStream_t s) {
  if (a.world < 1 || a.world > kEpMaxRanks) throw std::runtime_error("minisgl.ep: 1..8 ranks");
  if (a.H % 8 != 0 || a.T * a.k > a.cap) throw std::runtime_error("minisgl.ep_dispatch: H % 8 == 0 and T * k <= cap");
  const int warps = 8;
  launch_pdl(ep_dispatch_kernel, dim3((a.cap + warps - 1) / warps), dim3(warps * 32), 0, s, a);
  launch_pdl(ep_bump_kernel, dim3(1), dim3(1), 0, s, a.epoch);
}

void launch_ep_return(const EpArgs& a, cudaStream_t s) {
  if (a.world < 1 || a.world > kEpMaxRanks) throw std::runtime_error("minisgl.ep: 1..8 ranks");
  const int warps = 8;
  const int64_t slots = static_cast<int64_t>(a.world) * a.cap;
  launch_pdl(ep_return_kernel, dim3(static_cast<unsigned>((slots + warps - 1) / warps)), dim3(warps * 32), 0, s, a);
  launch_pdl(ep_bump_kernel, dim3(1), dim3(1), 0, s, a.epoch);
}

}  // namespace minisgl
