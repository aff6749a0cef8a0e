// Persistent tcgen05 GEMM for long token batches (prefill):
// out[M, N] = x[M, K] @ w[N, K]^T (+ bias), bf16 in, fp32 accumulate.
//
// One CTA per SM walks a static list of 128 x BN output tiles (grouped by
// 16 row blocks so a wave of CTAs shares its weight tiles in L2). Two TMEM
// accumulators of BN columns alternate between tiles, so the epilogue warps
// drain tile i (TMEM -> registers -> global) while the MMA thread already
// accumulates tile i + 1, and the TMA ring never stops between tiles: the
// per-tile prologue and epilogue of a one-tile-per-CTA launch are hidden.
//
// Warp roles (192 threads): warp 0 TMA producer, warp 1 MMA issuer (and
// TMEM owner), warps 2-5 epilogue (warp w reads TMEM lanes 32 (w % 4)..).
// Every wait is bounded; a timeout records an error, raises an abort flag
// that the other roles check, and the CTA drains its copies and returns.
//
// The reference calls cuBLAS / FlashInfer GEMMs through torch
// (python/minisgl/layers/linear.py); these kernels are the long-M paths of
// minisgl.ops.gemm (plan mode 3, one CTA per tile; plan mode 5, CTA pairs).
#include <cstdlib>
#include <stdexcept>
#include <string>

#include "common.cuh"
#include "launch.h"
#include "ops.h"
#include "tma_host.h"

namespace minisgl {
namespace {

constexpr int PBM = 128;
constexpr int PBK = 64;
constexpr int kPThreads = 192;
constexpr int kGroupRows = 16;  // row blocks per tile group (L2 reuse of weight tiles)

template <int BN>
struct PSmem {
  static constexpr int kA = PBM * PBK * 2;
  static constexpr int kB = BN * PBK * 2;
  static constexpr int kStage = kA + kB;
  static constexpr int kStages = BN == 256 ? 4 : 6;
  static constexpr int kBytes = 1024 + kStages * kStage + 256;
};

struct PParams {
  void* out;
  const __nv_bfloat16* bias;
  int M, N, K, ldo;
  int out_f32;
  int m_tiles, n_tiles;
  // measurement switches (MINISGL_GEMM_DEBUG; 0 in production): 1 skip the
  // global stores, 2 skip the accumulator read-out, 4 load only A each
  // k-block (B stays from an earlier stage), 8 issue no MMAs
  int debug;
  int prefetch;  // k-blocks ahead of the loads that the producer prefetches into L2 (0: none)
  ErrorSink err;
};

int gemm_prefetch_depth() {
  static const int d = [] {
    const char* v = std::getenv("MINISGL_GEMM_PREFETCH");
    return v == nullptr ? 0 : std::atoi(v);
  }();
  return d;
}

int gemm_debug_bits() {
  static const int bits = [] {
    const char* v = std::getenv("MINISGL_GEMM_DEBUG");
    return v == nullptr ? 0 : std::atoi(v);
  }();
  return bits;
}

__device__ __forceinline__ void tile_coords(int tile, int m_tiles, int n_tiles, int& mb, int& nb) {
  const int per_group = kGroupRows * n_tiles;
  const int group = tile / per_group;
  const int first = group * kGroupRows;
  const int rows = min(kGroupRows, m_tiles - first);
  const int in = tile - group * per_group;
  mb = first + in % rows;
  nb = in / rows;
}

template <int BN>
__global__ void __launch_bounds__(kPThreads, 1)
    gemm_persistent_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                           const PParams p) {
  using S = PSmem<BN>;
  constexpr int kStages = S::kStages;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kStages * S::kStage);
  uint64_t* empty = full + kStages;
  uint64_t* acc_full = empty + kStages;   // [2]
  uint64_t* acc_empty = acc_full + 2;     // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);
  int* s_abort = reinterpret_cast<int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int num_tiles = p.m_tiles * p.n_tiles;
  const int nkb = (p.K + PBK - 1) / PBK;
  pdl_launch_dependents();
  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&acc_full[i], 1);
      mbar_init(&acc_empty[i], 4);
    }
    *s_abort = 0;
    fence_barrier_init();
    prefetch_tmap(&tmA);
    prefetch_tmap(&tmB);
  }
  pdl_wait();  // x comes from the previous kernel; TMEM is taken after it
  if (warp == 1) {
    tmem_alloc(tmem_slot, 2 * BN);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  volatile int* abort_flag = s_abort;
  int issued = 0;  // stages whose copies the producer started

  if (warp == 0) {
    // ------------------------------------------------------------ TMA ----
    if (lane == 0) {
      int it = 0;
      for (int tile = blockIdx.x; tile < num_tiles && !*abort_flag; tile += gridDim.x) {
        int mb, nb;
        tile_coords(tile, p.m_tiles, p.n_tiles, mb, nb);
        for (int kb = 0; kb < nkb; ++kb, ++it) {
          const int s = it % kStages;
          if (it >= kStages && !mbar_wait(&empty[s], ((it / kStages) - 1) & 1, p.err, 301)) {
            *abort_flag = 1;
            break;
          }
          if (p.prefetch > 0) {
            // the tiles of the k-block `prefetch` iterations ahead (possibly
            // in this CTA's next output tile) into L2
            const int ahead = kb + p.prefetch;
            const int t2 = tile + (ahead / nkb) * static_cast<int>(gridDim.x);
            if (t2 < num_tiles) {
              int mb2, nb2;
              tile_coords(t2, p.m_tiles, p.n_tiles, mb2, nb2);
              tma_prefetch_2d(&tmA, (ahead % nkb) * PBK, mb2 * PBM);
              tma_prefetch_2d(&tmB, (ahead % nkb) * PBK, nb2 * BN);
            }
          }
          uint8_t* st = smem + s * S::kStage;
          const bool b_too = (p.debug & 4) == 0 || it < kStages;
          mbar_arrive_expect_tx(&full[s], b_too ? S::kStage : S::kA);
          tma_load_2d(st, &tmA, &full[s], kb * PBK, mb * PBM);
          if (b_too) tma_load_2d(st + S::kA, &tmB, &full[s], kb * PBK, nb * BN);
          issued = it + 1;
        }
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA ----
    constexpr uint32_t idesc = make_idesc_bf16(PBM, BN);
    const uint32_t base = smem_u32(smem);
    int it = 0, lt = 0;
    bool ok = true;
    for (int tile = blockIdx.x; ok && tile < num_tiles; tile += gridDim.x, ++lt) {
      const int acc = lt & 1;
      if (lt >= 2) ok = __all_sync(0xffffffffu, mbar_wait(&acc_empty[acc], ((lt >> 1) - 1) & 1, p.err, 302));
      if (!ok) break;
      tc_fence_after();
      const uint32_t d = tmem + acc * BN;
      for (int kb = 0; kb < nkb; ++kb, ++it) {
        const int s = it % kStages;
        ok = __all_sync(0xffffffffu, mbar_wait(&full[s], (it / kStages) & 1, p.err, 303));
        if (!ok) break;
        tc_fence_after();
        if (lane == 0) {
          const uint32_t a_addr = base + s * S::kStage;
          const uint32_t b_addr = a_addr + S::kA;
          if ((p.debug & 8) == 0) {
#pragma unroll
            for (int k = 0; k < PBK / 16; ++k)
              tc_mma_f16(d, make_sdesc_k_sw128(a_addr + k * 32), make_sdesc_k_sw128(b_addr + k * 32), idesc,
                         (kb > 0 || k > 0) ? 1u : 0u);
          }
          tc_commit(&empty[s]);
        }
        __syncwarp();
      }
      if (ok && lane == 0) tc_commit(&acc_full[acc]);
      __syncwarp();
    }
    if (!ok && lane == 0) *abort_flag = 1;
    __syncwarp();
  } else {
    // ------------------------------------------------------- epilogue ----
    const int quad = warp & 3;
    const int row = 32 * quad + lane;
    const uint32_t lane_base = tmem + (static_cast<uint32_t>(32 * quad) << 16);
    int lt = 0;
    bool ok = true;
    for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x, ++lt) {
      const int acc = lt & 1;
      ok = __all_sync(0xffffffffu, mbar_wait(&acc_full[acc], (lt >> 1) & 1, p.err, 304));
      if (!ok) break;
      tc_fence_after();
      int mb, nb;
      tile_coords(tile, p.m_tiles, p.n_tiles, mb, nb);
      const int m = mb * PBM + row;
      const int n_base = nb * BN;
      if (p.debug & 2) {
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&acc_empty[acc]);
        continue;
      }
#pragma unroll 1
      for (int c = 0; c < BN / 32; ++c) {
        uint32_t r[32];
        tmem_ld_32x32b_x32(lane_base + acc * BN + c * 32, r);
        tc_wait_ld();
        if (c == BN / 32 - 1) {
          // the accumulator is read out: the MMA thread may reuse it
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&acc_empty[acc]);
        }
        if (m >= p.M || (p.debug & 1)) continue;
        const int n0 = n_base + c * 32;
        float v[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          v[j] = __uint_as_float(r[j]);
          if (p.bias != nullptr && n0 + j < p.N) v[j] += __bfloat162float(p.bias[n0 + j]);
        }
        if (p.out_f32) {
          float* dst = reinterpret_cast<float*>(p.out) + static_cast<size_t>(m) * p.ldo;
#pragma unroll
          for (int j = 0; j < 32; j += 4) {
            const int n = n0 + j;
            if (n + 4 <= p.N) {
              *reinterpret_cast<float4*>(dst + n) = make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
            } else {
              for (int q = 0; q < 4 && n + q < p.N; ++q) dst[n + q] = v[j + q];
            }
          }
        } else {
          __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(p.out) + static_cast<size_t>(m) * p.ldo;
#pragma unroll
          for (int j = 0; j < 32; j += 8) {
            const int n = n0 + j;
            if (n + 8 <= p.N) {
              uint4 pk;
              pk.x = pack_bf16x2(v[j], v[j + 1]);
              pk.y = pack_bf16x2(v[j + 2], v[j + 3]);
              pk.z = pack_bf16x2(v[j + 4], v[j + 5]);
              pk.w = pack_bf16x2(v[j + 6], v[j + 7]);
              *reinterpret_cast<uint4*>(dst + n) = pk;
            } else {
              for (int q = 0; q < 8 && n + q < p.N; ++q) dst[n + q] = __float2bfloat16_rn(v[j + q]);
            }
          }
        }
      }
    }
    if (!ok && lane == 0) *abort_flag = 1;
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0 && lane == 0 && *abort_flag) {
    // after an abort, let the copies still in flight land (bounded)
    for (int it = max(0, issued - kStages); it < issued; ++it)
      mbar_wait(&full[it % kStages], (it / kStages) & 1, p.err, 305);
  }
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 2 * BN);
  }
}

// ------------------------------------------------------------- CTA pairs ----
// The same persistent schedule on 256 x 256 output tiles, each computed by a
// pair of CTAs (cluster of 2, cta_group::2 MMAs): CTA r of the pair loads its
// 128 rows of A and its 128 rows of B (half of the tile's N) per k-block, and
// holds rows 128 r .. 128 r + 127 of the tile (all 256 columns) in its tensor
// memory. Per SM and k-block that is 32 KB of operand traffic for a
// 128 x 256 x 64 product, against 48 KB for a one-SM 128 x 256 tile: the
// pair shares B, which halves what the weights cost in L2 and shared-memory
// bandwidth.
//
// Synchronisation (the even CTA, rank 0, issues every MMA):
//   full[s]      rank 0's: one arrive (rank 0's expect_tx of both halves'
//                bytes); both CTAs' TMA loads complete on it
//   empty[s]     each CTA's own: the MMA thread commits to both
//   acc_full[a]  each CTA's own: the MMA thread commits to both
//   acc_empty[a] rank 0's: the 4 epilogue warps of each CTA arrive (8)
constexpr int kPairStages = 6;
constexpr int kPairA = PBM * PBK * 2;              // 16 KB: this CTA's 128 rows of A
constexpr int kPairB = 128 * PBK * 2;              // 16 KB: this CTA's 128 rows of B
constexpr int kPairStage = kPairA + kPairB;
constexpr int kPairBytes = 1024 + kPairStages * kPairStage + 256;
constexpr int kPairN = 256;                        // tile columns (both halves of B)

__device__ __forceinline__ void pair_tile_coords(int tile, int m_tiles, int n_tiles, int& mb, int& nb) {
  tile_coords(tile, m_tiles, n_tiles, mb, nb);
}

__global__ void __launch_bounds__(kPThreads, 1)
    gemm_pair_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                     const PParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kPairStages * kPairStage);
  uint64_t* empty = full + kPairStages;
  uint64_t* acc_full = empty + kPairStages;  // [2]
  uint64_t* acc_empty = acc_full + 2;        // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);
  int* s_abort = reinterpret_cast<int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();  // 0: issues the MMAs
  const int pair = static_cast<int>(blockIdx.x) >> 1, pairs = static_cast<int>(gridDim.x) >> 1;
  const int num_tiles = p.m_tiles * p.n_tiles;
  const int nkb = p.K / PBK;
  pdl_launch_dependents();
  if (threadIdx.x == 0) {
    for (int s = 0; s < kPairStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&acc_full[i], 1);
      mbar_init(&acc_empty[i], 8);
    }
    *s_abort = 0;
    fence_barrier_init();
    prefetch_tmap(&tmA);
    prefetch_tmap(&tmB);
  }
  pdl_wait();  // x comes from the previous kernel; TMEM is taken after it
  if (warp == 1) {
    tmem_alloc_pair(tmem_slot, 2 * kPairN);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  // every barrier of both CTAs is initialised before either CTA signals one
  // of the other's
  __syncthreads();
  cluster_sync();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  volatile int* abort_flag = s_abort;
  int issued = 0;  // k-blocks whose copies this CTA's producer started

  if (warp == 0) {
    // ------------------------------------------------------------ TMA ----
    if (lane == 0) {
      int it = 0;
      for (int tile = pair; tile < num_tiles && !*abort_flag; tile += pairs) {
        int mb, nb;
        pair_tile_coords(tile, p.m_tiles, p.n_tiles, mb, nb);
        const int a_row = mb * 256 + static_cast<int>(rank) * PBM;
        const int b_row = nb * kPairN + static_cast<int>(rank) * 128;
        for (int kb = 0; kb < nkb; ++kb, ++it) {
          const int s = it % kPairStages;
          if (it >= kPairStages && !mbar_wait(&empty[s], ((it / kPairStages) - 1) & 1, p.err, 311)) {
            *abort_flag = 1;
            break;
          }
          if (p.prefetch > 0) {
            const int ahead = kb + p.prefetch;
            const int t2 = tile + (ahead / nkb) * pairs;
            if (t2 < num_tiles) {
              int mb2, nb2;
              pair_tile_coords(t2, p.m_tiles, p.n_tiles, mb2, nb2);
              tma_prefetch_2d(&tmA, (ahead % nkb) * PBK, mb2 * 256 + static_cast<int>(rank) * PBM);
              tma_prefetch_2d(&tmB, (ahead % nkb) * PBK, nb2 * kPairN + static_cast<int>(rank) * 128);
            }
          }
          uint8_t* st = smem + s * kPairStage;
          const bool b_too = (p.debug & 4) == 0 || it < kPairStages;
          // rank 0 expects the bytes of both CTAs' loads on its own barrier
          if (rank == 0) mbar_arrive_expect_tx(&full[s], 2 * (b_too ? kPairStage : kPairA));
          const uint32_t bar = map_shared_rank(smem_u32(&full[s]), 0);
          tma_load_2d_pair(st, &tmA, bar, kb * PBK, a_row);
          if (b_too) tma_load_2d_pair(st + kPairA, &tmB, bar, kb * PBK, b_row);
          issued = it + 1;
        }
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA ----
    if (rank == 0) {
      constexpr uint32_t idesc = make_idesc_bf16(256, kPairN);
      const uint32_t base = smem_u32(smem);
      int it = 0, lt = 0;
      bool ok = true;
      for (int tile = pair; ok && tile < num_tiles; tile += pairs, ++lt) {
        const int acc = lt & 1;
        if (lt >= 2) ok = __all_sync(0xffffffffu, mbar_wait(&acc_empty[acc], ((lt >> 1) - 1) & 1, p.err, 312));
        if (!ok) break;
        tc_fence_after();
        const uint32_t d = tmem + acc * kPairN;
        for (int kb = 0; kb < nkb; ++kb, ++it) {
          const int s = it % kPairStages;
          ok = __all_sync(0xffffffffu, mbar_wait(&full[s], (it / kPairStages) & 1, p.err, 313));
          if (!ok) break;
          tc_fence_after();
          if (lane == 0) {
            const uint32_t a_addr = base + s * kPairStage;
            const uint32_t b_addr = a_addr + kPairA;
            if ((p.debug & 8) == 0) {
#pragma unroll
              for (int k = 0; k < PBK / 16; ++k)
                tc_mma_f16_pair(d, make_sdesc_k_sw128(a_addr + k * 32), make_sdesc_k_sw128(b_addr + k * 32), idesc,
                                (kb > 0 || k > 0) ? 1u : 0u);
            }
            // stage s of both CTAs is free once these MMAs are done
            tc_commit_pair(smem_u32(&empty[s]));
            tc_commit_pair(map_shared_rank(smem_u32(&empty[s]), 1));
          }
          __syncwarp();
        }
        if (ok && lane == 0) {
          tc_commit_pair(smem_u32(&acc_full[acc]));
          tc_commit_pair(map_shared_rank(smem_u32(&acc_full[acc]), 1));
        }
        __syncwarp();
      }
      if (!ok && lane == 0) *abort_flag = 1;
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------- epilogue ----
    const int quad = warp & 3;
    const int row = 32 * quad + lane;
    const uint32_t lane_base = tmem + (static_cast<uint32_t>(32 * quad) << 16);
    const uint32_t acc_empty0 = map_shared_rank(smem_u32(acc_empty), 0);
    int lt = 0;
    bool ok = true;
    for (int tile = pair; tile < num_tiles; tile += pairs, ++lt) {
      const int acc = lt & 1;
      ok = __all_sync(0xffffffffu, mbar_wait(&acc_full[acc], (lt >> 1) & 1, p.err, 314));
      if (!ok) break;
      tc_fence_after();
      int mb, nb;
      pair_tile_coords(tile, p.m_tiles, p.n_tiles, mb, nb);
      const int m = mb * 256 + static_cast<int>(rank) * PBM + row;
      const int n_base = nb * kPairN;
      if (p.debug & 2) {
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive_cluster(acc_empty0 + static_cast<uint32_t>(acc) * 8u);
        continue;
      }
#pragma unroll 1
      for (int c = 0; c < kPairN / 32; ++c) {
        uint32_t r[32];
        tmem_ld_32x32b_x32(lane_base + acc * kPairN + c * 32, r);
        tc_wait_ld();
        if (c == kPairN / 32 - 1) {
          // the accumulator is read out: rank 0's MMA thread may reuse it
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive_cluster(acc_empty0 + static_cast<uint32_t>(acc) * 8u);
        }
        if (m >= p.M || (p.debug & 1)) continue;
        const int n0 = n_base + c * 32;
        float v[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          v[j] = __uint_as_float(r[j]);
          if (p.bias != nullptr && n0 + j < p.N) v[j] += __bfloat162float(p.bias[n0 + j]);
        }
        if (p.out_f32) {
          float* dst = reinterpret_cast<float*>(p.out) + static_cast<size_t>(m) * p.ldo;
#pragma unroll
          for (int j = 0; j < 32; j += 4) {
            const int n = n0 + j;
            if (n + 4 <= p.N) {
              *reinterpret_cast<float4*>(dst + n) = make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
            } else {
              for (int q = 0; q < 4 && n + q < p.N; ++q) dst[n + q] = v[j + q];
            }
          }
        } else {
          __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(p.out) + static_cast<size_t>(m) * p.ldo;
#pragma unroll
          for (int j = 0; j < 32; j += 8) {
            const int n = n0 + j;
            if (n + 8 <= p.N) {
              uint4 pk;
              pk.x = pack_bf16x2(v[j], v[j + 1]);
              pk.y = pack_bf16x2(v[j + 2], v[j + 3]);
              pk.z = pack_bf16x2(v[j + 4], v[j + 5]);
              pk.w = pack_bf16x2(v[j + 6], v[j + 7]);
              *reinterpret_cast<uint4*>(dst + n) = pk;
            } else {
              for (int q = 0; q < 8 && n + q < p.N; ++q) dst[n + q] = __float2bfloat16_rn(v[j + q]);
            }
          }
        }
      }
    }
    if (!ok && lane == 0) *abort_flag = 1;
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0 && lane == 0 && *abort_flag) {
    // after an abort, let the copies still in flight land before the pair
    // leaves: rank 0 waits for its stages (which count both CTAs' bytes);
    // rank 1 cannot wait on rank 0's barrier, so it gives its own copies a
    // fixed 200 us (copies of 16 KB take about a microsecond)
    if (rank == 0) {
      for (int it = max(0, issued - kPairStages); it < issued; ++it)
        mbar_wait(&full[it % kPairStages], (it / kPairStages) & 1, p.err, 315);
    } else {
      const uint64_t t0 = globaltimer_ns();
      while (globaltimer_ns() - t0 < 200000ull) {
      }
    }
  }
  // neither CTA leaves (or frees tensor memory) while the other may still
  // signal one of its barriers or read its shared memory
  tc_fence_before();
  __syncthreads();
  cluster_sync();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem, 2 * kPairN);
  }
}

int num_sms() {
  static int n = 0;
  if (n == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    if (n <= 0) n = 148;
  }
  return n;
}

template <int BN>
void launch_bn(const GemmArgs& a, cudaStream_t stream) {
  using S = PSmem<BN>;
  static bool attr = false;
  if (!attr) {
    cudaFuncSetAttribute(gemm_persistent_kernel<BN>, cudaFuncAttributeMaxDynamicSharedMemorySize, S::kBytes);
    attr = true;
  }
  CUtensorMap ta = make_tmap_bf16_2d_sw128(a.x, a.M, a.K, a.ldx, PBM);
  CUtensorMap tb = make_tmap_bf16_2d_sw128(a.w, a.N, a.K, a.ldw, BN);
  PParams p;
  p.out = a.out;
  p.bias = reinterpret_cast<const __nv_bfloat16*>(a.bias);
  p.M = a.M;
  p.N = a.N;
  p.K = a.K;
  p.ldo = a.ldo;
  p.out_f32 = a.out_f32 ? 1 : 0;
  p.m_tiles = (a.M + PBM - 1) / PBM;
  p.n_tiles = (a.N + BN - 1) / BN;
  p.debug = gemm_debug_bits();
  p.prefetch = gemm_prefetch_depth();
  p.err = ErrorSink{a.err};
  const int tiles = p.m_tiles * p.n_tiles;
  const int grid = tiles < num_sms() ? tiles : num_sms();
  launch_pdl(gemm_persistent_kernel<BN>, dim3(grid), dim3(kPThreads), S::kBytes, stream, ta, tb, p);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess)
    throw std::runtime_error(std::string("minisgl.gemm (persistent) launch failed: ") + cudaGetErrorString(e));
}

void launch_pair(const GemmArgs& a, cudaStream_t stream) {
  static bool attr[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (!attr[dev & 63]) {
    cudaFuncSetAttribute(gemm_pair_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kPairBytes);
    attr[dev & 63] = true;
  }
  CUtensorMap ta = make_tmap_bf16_2d_sw128(a.x, a.M, a.K, a.ldx, PBM);
  CUtensorMap tb = make_tmap_bf16_2d_sw128(a.w, a.N, a.K, a.ldw, 128);
  PParams p;
  p.out = a.out;
  p.bias = reinterpret_cast<const __nv_bfloat16*>(a.bias);
  p.M = a.M;
  p.N = a.N;
  p.K = a.K;
  p.ldo = a.ldo;
  p.out_f32 = a.out_f32 ? 1 : 0;
  p.m_tiles = (a.M + 255) / 256;
  p.n_tiles = (a.N + kPairN - 1) / kPairN;
  p.debug = gemm_debug_bits();
  p.prefetch = gemm_prefetch_depth();
  p.err = ErrorSink{a.err};
  const int tiles = p.m_tiles * p.n_tiles;
  const int max_pairs = num_sms() / 2;
  const int pairs = tiles < max_pairs ? tiles : max_pairs;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(2 * pairs, 1, 1);
  cfg.blockDim = dim3(kPThreads, 1, 1);
  cfg.dynamicSmemBytes = kPairBytes;
  cfg.stream = stream;
  cudaLaunchAttribute attrs[2];
  int n = 0;
  attrs[n].id = cudaLaunchAttributeClusterDimension;
  attrs[n].val.clusterDim.x = 2;
  attrs[n].val.clusterDim.y = 1;
  attrs[n].val.clusterDim.z = 1;
  ++n;
  if (pdl_enabled()) {
    attrs[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attrs[n].val.programmaticStreamSerializationAllowed = 1;
    ++n;
  }
  cfg.attrs = attrs;
  cfg.numAttrs = n;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, gemm_pair_kernel, ta, tb, p);
  if (e != cudaSuccess)
    throw std::runtime_error(std::string("minisgl.gemm (CTA pairs) launch failed: ") + cudaGetErrorString(e));
}

}  // namespace

bool gemm_pair_supported(const GemmArgs& a) {
  return a.epi.kind == 0 && a.g_num_tiles == nullptr && a.M > 0 && a.K % PBK == 0 && a.K > 0;
}

void launch_gemm_pair(const GemmArgs& a, cudaStream_t stream) {
  if (!gemm_pair_supported(a))
    throw std::runtime_error("minisgl.gemm: CTA-pair tiles take plain GEMMs with K % 64 == 0");
  launch_pair(a, stream);
}

bool gemm_persistent_supported(const GemmArgs& a) {
  return a.epi.kind == 0 && a.g_num_tiles == nullptr && a.M > 0 && a.K % PBK == 0 && a.K > 0 &&
         (a.force_bn == 0 || a.force_bn == 128 || a.force_bn == 256);
}

void launch_gemm_persistent(const GemmArgs& a, cudaStream_t stream) {
  if (!gemm_persistent_supported(a))
    throw std::runtime_error("minisgl.gemm: persistent tiles take plain GEMMs with K % 64 == 0 and an N tile of 128 "
                             "or 256");
  if (a.force_bn == 128) launch_bn<128>(a, stream);
  else launch_bn<256>(a, stream);
}

}  // namespace minisgl
