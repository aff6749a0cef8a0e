// Tensor-parallel collectives over NVLink peer memory, issued from our own
// kernels (no NCCL on this path).
//
// Symmetric heap: every rank allocates the same-sized device buffer, exports a
// CUDA IPC handle, and maps every peer's buffer (handles are exchanged over
// the CPU process group by minisgl/parallel/symm.py). Layout of each heap:
//
//   [0, 4 KB)        uint32 slots: entry[src] at 0, exit[src] at 16,
//                    done-CTA counter at 32 (local)
//   [4 KB, 20 KB)    per-CTA flags of the GEMM with the all-reduce fused
//                    (gemm.cu, kEpiAllReduce)
//   [20 KB, +C)      collective data: this rank's partial, written before
//                    the call
//   [+C, +3C)        the fused GEMM's two partial halves (gemm.cu)
//
// A call with epoch e (a device counter, so CUDA-graph replays advance it):
//   1. entry barrier: CTA 0 stores e into entry[rank] of every peer
//      (system-scope release) and every CTA waits until its own entry slots
//      of all ranks reach e: all partials are complete;
//   2. every rank reads all partials over NVLink in rank order 0..R-1 (the
//      same order everywhere, so all ranks produce the same bits);
//   3. exit barrier: the last CTA of the rank to finish stores e into
//      exit[rank] of every peer and waits for all exit slots: no peer still
//      reads this rank's data once the kernel has completed, so the next
//      producer (which starts after griddepcontrol.wait) may overwrite it.
// Waits give up after two seconds, record kErrPeerTimeout in the error word
// and let the kernel finish (the result is then undefined but the GPU keeps
// running). No NVLS / multicast objects are created.
#include <cuda_runtime.h>

#include <algorithm>
#include <stdexcept>
#include <string>

#include "common.cuh"
#include "launch.h"
#include "ops.h"

namespace minisgl {
namespace {

constexpr int kMaxRanks = 8;
constexpr int64_t kSignalBytes = 4096;
constexpr int kEntry = 0, kExit = 16, kDone = 32;  // uint32 slot offsets

struct SymmArgs {
  const int64_t* bases;  // [world] heap base of every rank (own one included)
  const uint32_t* epoch; // this rank's call counter (the call uses epoch + 1)
  int rank, world;
  int n8;                // elements / 8 (16-byte vectors)
  __nv_bfloat16* out;
  const __nv_bfloat16* residual;  // all-reduce: added after the sum (may be nullptr)
  int rows_per_rank;     // all-gather: rows of each rank's slice
  int row_vecs;          // all-gather: 16-byte vectors per row
  ErrorSink err;
};

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Threads 0..world-1: store e into slot `which` + rank of every peer.
__device__ __forceinline__ void signal_peers(const SymmArgs& a, int which, uint32_t e) {
  if (threadIdx.x < a.world) {
    __threadfence_system();  // data written before the signal is visible to the peers
    st_release_sys(reinterpret_cast<uint32_t*>(a.bases[threadIdx.x]) + which + a.rank, e);
  }
}

// Threads 0..world-1 wait (bounded) until slot `which` + t of this rank
// reaches e.
__device__ __forceinline__ void wait_peers(const SymmArgs& a, int which, uint32_t e, int site) {
  if (threadIdx.x < a.world) {
    const uint32_t* mine = reinterpret_cast<const uint32_t*>(a.bases[a.rank]) + which + threadIdx.x;
    const uint64_t t0 = globaltimer_ns();
    uint32_t it = 0;
    while (static_cast<int32_t>(ld_acquire_sys(mine) - e) < 0) {
      if (((++it) & 0xFFu) == 0 && globaltimer_ns() - t0 > kWaitBudgetNs) {
        a.err.report(kErrPeerTimeout, site + static_cast<int>(threadIdx.x));
        break;
      }
    }
  }
}

// Entry barrier; returns the epoch of this call.
__device__ uint32_t symm_enter(const SymmArgs& a) {
  const uint32_t e = *a.epoch + 1;
  if (blockIdx.x == 0) signal_peers(a, kEntry, e);
  wait_peers(a, kEntry, e, 300);
  __syncthreads();
  return e;
}

// Exit barrier, run by the last CTA of this rank to finish reading. Kernels
// that stored into peer heaps pass sys_fence so those stores are visible to
// the peers before this rank's exit signal.
__device__ void symm_exit(const SymmArgs& a, uint32_t e, bool sys_fence = false) {
  __shared__ bool last;
  __syncthreads();
  if (threadIdx.x == 0) {
    if (sys_fence) __threadfence_system();
    else __threadfence();
    uint32_t* done = reinterpret_cast<uint32_t*>(a.bases[a.rank]) + kDone;
    last = atomicAdd(done, 1u) == gridDim.x - 1;
    if (last) *done = 0;  // ready for the next call (which starts after this kernel)
  }
  __syncthreads();
  if (!last) return;
  signal_peers(a, kExit, e);
  wait_peers(a, kExit, e, 310);
}

__device__ __forceinline__ const uint4* data_ptr(const SymmArgs& a, int r) {
  return reinterpret_cast<const uint4*>(reinterpret_cast<const uint8_t*>(a.bases[r]) + kSignalBytes +
                                        kSymmFlagBytes);
}

__global__ void symm_all_reduce_kernel(SymmArgs a) {
  pdl_launch_dependents();
  pdl_wait();
  const uint32_t e = symm_enter(a);
  const uint4* src[kMaxRanks];
#pragma unroll
  for (int r = 0; r < kMaxRanks; ++r) src[r] = r < a.world ? data_ptr(a, r) : nullptr;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < a.n8; i += gridDim.x * blockDim.x) {
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int r = 0; r < kMaxRanks; ++r) {
      if (r >= a.world) break;
      const uint4 raw = src[r][i];
      const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&raw);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float2 f = __bfloat1622float2(h[q]);
        acc[2 * q] += f.x;
        acc[2 * q + 1] += f.y;
      }
    }
    if (a.residual != nullptr) {
      // the sum as a bf16 all-reduce would return it, then the residual add
      const uint4 rr = reinterpret_cast<const uint4*>(a.residual)[i];
      const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&rr);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float2 f = __bfloat1622float2(h[q]);
        acc[2 * q] = __bfloat162float(__float2bfloat16_rn(acc[2 * q])) + f.x;
        acc[2 * q + 1] = __bfloat162float(__float2bfloat16_rn(acc[2 * q + 1])) + f.y;
      }
    }
    uint4 pk;
    pk.x = pack_bf16x2(acc[0], acc[1]);
    pk.y = pack_bf16x2(acc[2], acc[3]);
    pk.z = pack_bf16x2(acc[4], acc[5]);
    pk.w = pack_bf16x2(acc[6], acc[7]);
    reinterpret_cast<uint4*>(a.out)[i] = pk;
  }
  symm_exit(a, e);
}

// out [world * rows_per_rank, row] = concatenation of every rank's slice
__global__ void symm_all_gather_kernel(SymmArgs a) {
  pdl_launch_dependents();
  pdl_wait();
  const uint32_t e = symm_enter(a);
  const int per_rank = a.rows_per_rank * a.row_vecs;
  const int total = per_rank * a.world;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < total; i += gridDim.x * blockDim.x) {
    const int r = i / per_rank;
    reinterpret_cast<uint4*>(a.out)[i] = data_ptr(a, r)[i - r * per_rank];
  }
  symm_exit(a, e);
}

// ------------------------------------------- reduce-scatter + norm + gather
// The row-parallel projection's collective on a token-sharded residual
// stream. Each rank's heap data region holds its partial product [T, H]
// (T = rows * world); rank r owns rows [r * rows, (r + 1) * rows):
//   1. (entry barrier) sum the owned rows of every rank's partial, in rank
//      order, in fp32; round the sum to bf16 (what a bf16 all-reduce returns)
//      and add it to this rank's residual slice (or start the slice with it),
//      rounding the new residual to bf16 (the residual stream's dtype);
//   2. RMS-normalise each new residual row (times the norm weight, when one is
//      given; otherwise the weight is folded into the next GEMM) and store the
//      bf16 row into the gather region of EVERY rank's heap (peer stores);
//   3. (exit barrier, system-scope fences) every rank's gather region then
//      holds all T normalised rows, the input of the next column-parallel
//      GEMM, read from local memory.
// NVLink traffic per rank: (world - 1) / world of the partial in and the
// same of the normalised rows out, the bytes of a two-shot all-reduce,
// with the add and the norm of the next layer folded in.
struct RsnArgs {
  SymmArgs s;                   // bases, epoch, rank, world, err
  int rows;                     // rows of each rank's slice
  int vecs;                     // H / 8 (16-byte vectors per row)
  int64_t data_off;             // byte offset of the partial region in every heap
  int64_t gather_off;           // byte offset of the gather region in every heap
  __nv_bfloat16* resid;         // [rows, H] this rank's residual slice (in / out)
  int add_resid;                // 1: resid += sum, 0: resid = sum
  const __nv_bfloat16* norm_w;  // [H] or nullptr
  float eps;
};

template <int VPT>
__global__ void __launch_bounds__(1024) symm_rsn_kernel(RsnArgs a) {
  pdl_launch_dependents();
  pdl_wait();
  const uint32_t e = symm_enter(a.s);
  const int world = a.s.world;
  __shared__ float red[32];
  for (int row = blockIdx.x; row < a.rows; row += gridDim.x) {
    const int64_t grow = static_cast<int64_t>(a.s.rank) * a.rows + row;
    float v[VPT][8];
    float ss = 0.f;
#pragma unroll
    for (int j = 0; j < VPT; ++j) {
      const int c = threadIdx.x + j * blockDim.x;
      if (c >= a.vecs) continue;
      const int64_t idx = grow * a.vecs + c;
      uint4 raw[kMaxRanks];
#pragma unroll
      for (int r = 0; r < kMaxRanks; ++r)  // every load in flight before the adds
        if (r < world)
          raw[r] = reinterpret_cast<const uint4*>(reinterpret_cast<const uint8_t*>(a.s.bases[r]) + a.data_off)[idx];
      float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int r = 0; r < kMaxRanks; ++r) {
        if (r >= world) break;
        const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&raw[r]);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const float2 f = __bfloat1622float2(h[q]);
          acc[2 * q] += f.x;
          acc[2 * q + 1] += f.y;
        }
      }
      uint4* rp = reinterpret_cast<uint4*>(a.resid) + static_cast<int64_t>(row) * a.vecs + c;
      float old[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
      if (a.add_resid) {
        const uint4 rr = *rp;
        const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&rr);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const float2 f = __bfloat1622float2(h[q]);
          old[2 * q] = f.x;
          old[2 * q + 1] = f.y;
        }
      }
      uint4 pk;
      uint32_t* pw = reinterpret_cast<uint32_t*>(&pk);
#pragma unroll
      for (int q = 0; q < 4; ++q)
        pw[q] = pack_bf16x2(__bfloat162float(__float2bfloat16_rn(acc[2 * q])) + old[2 * q],
                            __bfloat162float(__float2bfloat16_rn(acc[2 * q + 1])) + old[2 * q + 1]);
      *rp = pk;
      const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&pk);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float2 f = __bfloat1622float2(h[q]);
        v[j][2 * q] = f.x;
        v[j][2 * q + 1] = f.y;
        ss += f.x * f.x + f.y * f.y;
      }
    }
    // block-wide sum of squares of the row
    ss = warp_sum(ss);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
    __syncthreads();
    float tot = (threadIdx.x & 31) < (blockDim.x >> 5) ? red[threadIdx.x & 31] : 0.f;
    tot = warp_sum(tot);
    __syncthreads();
    const float inv = rsqrtf(tot / static_cast<float>(a.vecs * 8) + a.eps);
#pragma unroll
    for (int j = 0; j < VPT; ++j) {
      const int c = threadIdx.x + j * blockDim.x;
      if (c >= a.vecs) continue;
      float wv[8] = {1.f, 1.f, 1.f, 1.f, 1.f, 1.f, 1.f, 1.f};
      if (a.norm_w != nullptr) {
        const uint4 ww = reinterpret_cast<const uint4*>(a.norm_w)[c];
        const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&ww);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const float2 f = __bfloat1622float2(h[q]);
          wv[2 * q] = f.x;
          wv[2 * q + 1] = f.y;
        }
      }
      uint4 pk;
      uint32_t* pw = reinterpret_cast<uint32_t*>(&pk);
#pragma unroll
      for (int q = 0; q < 4; ++q)
        pw[q] = pack_bf16x2(v[j][2 * q] * inv * wv[2 * q], v[j][2 * q + 1] * inv * wv[2 * q + 1]);
      const int64_t idx = grow * a.vecs + c;
#pragma unroll
      for (int r = 0; r < kMaxRanks; ++r)
        if (r < world)
          reinterpret_cast<uint4*>(reinterpret_cast<uint8_t*>(a.s.bases[r]) + a.gather_off)[idx] = pk;
    }
  }
  symm_exit(a.s, e, /*sys_fence=*/true);
}

__global__ void symm_bump_kernel(uint32_t* epoch) {
  pdl_launch_dependents();
  pdl_wait();  // every CTA of the collective has read the old value
  *epoch += 1;
}

}  // namespace

void launch_symm_rsn(const int64_t* bases, uint32_t* epoch, int rank, int world, int rows, int hidden,
                     int64_t data_off, int64_t gather_off, void* resid, bool add_resid, const void* norm_w, float eps,
                     int* err, cudaStream_t s) {
  if (world < 1 || world > kMaxRanks) throw std::runtime_error("minisgl.symm_rsn: 1..8 ranks");
  if (hidden % 8 != 0 || hidden > 8 * 1024 * 4) throw std::runtime_error("minisgl.symm_rsn: hidden % 8, <= 32768");
  if (rows <= 0) return;
  RsnArgs a{};
  a.s.bases = bases;
  a.s.epoch = epoch;
  a.s.rank = rank;
  a.s.world = world;
  a.s.err = ErrorSink{err};
  a.rows = rows;
  a.vecs = hidden / 8;
  a.data_off = data_off;
  a.gather_off = gather_off;
  a.resid = static_cast<__nv_bfloat16*>(resid);
  a.add_resid = add_resid ? 1 : 0;
  a.norm_w = static_cast<const __nv_bfloat16*>(norm_w);
  a.eps = eps;
  const int vpt = (a.vecs + 1023) / 1024;
  const int threads = ((a.vecs + vpt - 1) / vpt + 31) / 32 * 32;
  const int blocks = std::min(rows, 148 * 2);
  if (vpt == 1) launch_pdl(symm_rsn_kernel<1>, dim3(blocks), dim3(threads), 0, s, a);
  else if (vpt == 2) launch_pdl(symm_rsn_kernel<2>, dim3(blocks), dim3(threads), 0, s, a);
  else launch_pdl(symm_rsn_kernel<4>, dim3(blocks), dim3(threads), 0, s, a);
  launch_pdl(symm_bump_kernel, dim3(1), dim3(1), 0, s, epoch);
}

void launch_epoch_bump(uint32_t* epoch, cudaStream_t s) {
  launch_pdl(symm_bump_kernel, dim3(1), dim3(1), 0, s, epoch);
}

void launch_symm_collective(int kind, const int64_t* bases, uint32_t* epoch, int rank, int world, int64_t n_elems,
                            void* out, const void* residual, int rows_per_rank, int row_elems, int* err,
                            cudaStream_t s) {
  if (world < 1 || world > kMaxRanks) throw std::runtime_error("minisgl.symm: 1..8 ranks");
  if (n_elems % 8 != 0) throw std::runtime_error("minisgl.symm: element count must be a multiple of 8");
  SymmArgs a{};
  a.bases = bases;
  a.epoch = epoch;
  a.rank = rank;
  a.world = world;
  a.n8 = static_cast<int>(n_elems / 8);
  a.out = static_cast<__nv_bfloat16*>(out);
  a.residual = static_cast<const __nv_bfloat16*>(residual);
  a.rows_per_rank = rows_per_rank;
  a.row_vecs = row_elems / 8;
  a.err = ErrorSink{err};
  const int threads = 512;
  const int64_t work = kind == 0 ? a.n8 : static_cast<int64_t>(a.n8) * world;
  const int blocks = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>((work + threads - 1) / threads, 148 * 2)));
  if (kind == 0) launch_pdl(symm_all_reduce_kernel, dim3(blocks), dim3(threads), 0, s, a);
  else launch_pdl(symm_all_gather_kernel, dim3(blocks), dim3(threads), 0, s, a);
  launch_pdl(symm_bump_kernel, dim3(1), dim3(1), 0, s, epoch);
}

}  // namespace minisgl
