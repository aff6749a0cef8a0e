// Weight-streaming GEMM for decode batches (up to 256 tokens), stream-K over
// every SM.
//
//   out[M, N] = x[M, K] @ w[N, K]^T (+ bias)
//
// A decode projection reads each weight once and little else: at M <= 256
// its time is the weight stream plus how evenly the SMs share it. Tiles are
// weight-major (operand A = 128 * R weight rows, the R sub-tiles sharing one
// token tile of BN rows as operand B, so each x k-block is loaded once per
// 128 * R weight rows). The (tile, k-block) units of the whole GEMM are cut
// into one contiguous range per CTA, one CTA per SM (stream-K), so every SM
// streams the same number of weight bytes whatever N / 128 is.
//
// A CTA's range covers whole tiles plus at most a tail of one tile at its
// start and a head of one tile at its end:
//   * a whole tile is stored straight from TMEM;
//   * a range that starts inside tile t is a contributor: it writes its fp32
//     partial tile into its own workspace slot and sets its ready flag;
//   * the CTA whose range holds the first k-block of a split tile owns it:
//     it waits (bounded) for the contributors' flags, adds their partials in
//     CTA order (a fixed order, so results are deterministic), stores the
//     tile and clears the flags for the next launch.
// Contributors do their part of tile t first and owners last, so an owner
// rarely waits. Every CTA is resident (one per SM, grid <= SM count), and
// contributors never wait, so the waits always end.
//
// Warp roles (192 threads): warp 0 TMA producer (each stage is one 3-D box of
// kps k-blocks per operand), warp 1 TMEM allocation + single-thread
// tcgen05.mma issue, warps 2-5 epilogue (TMEM lane = weight row). The
// accumulator is double-buffered in TMEM when 2 * R * BN columns fit, so a
// segment's epilogue overlaps the next segment's mainloop.
//
// The producer streams the first stages of weights before
// griddepcontrol.wait (weights never depend on the previous kernel), and
// the kernel triggers its dependents at entry (programmatic dependent
// launch). Workspace and flags are only touched after griddepcontrol.wait, so
// back-to-back launches on one stream never overlap on them.
#include <algorithm>
#include <cstdlib>
#include <stdexcept>
#include <string>

#include "common.cuh"
#include "launch.h"
#include "ops.h"
#include "tma_host.h"

namespace minisgl {
namespace {

constexpr int kSkThreads = 192;
constexpr int kFlagStride = 32;  // int32 words between ready flags (one 128-byte line each)
constexpr int kStageLd = 132;    // floats per token row of the output staging tile (128 + pad)
constexpr uint32_t kStageBytes = 32 * kStageLd * 4;
constexpr int kSkSmemBudget = 196 * 1024;  // stage ring bytes (the output staging tile comes on top)

struct SkParams {
  void* out;
  const __nv_bfloat16* bias;
  int M, N, K;
  int ldo;
  int out_f32;
  int vec_ok;     // out and ldo allow 16-byte (bf16) / 32-byte (fp32) row stores
  int num_tiles;  // ceil(N / (128 R))
  int num_kb;     // K / 64
  int kps;        // k-blocks per stage
  int stages;
  int grid;       // CTAs (= workspace slots)
  float* ws;      // [grid][R * BN * 128] fp32 partial tiles
  int* flags;     // [grid * kFlagStride] ready flags (0 between launches)
  ErrorSink err;
  // optional per-CTA %globaltimer stamps, 8 slots per CTA: 0 entry, 1 set-up
  // done, 2 producer past griddepcontrol.wait, 3 first accumulator ready,
  // 4 last accumulator ready, 5 owner's contributors ready, 6 epilogue done
  unsigned long long* trace;
  // measurement switches (MINISGL_STREAMK_DEBUG): 1 skip global stores,
  // 2 skip the MMAs, 4 skip the x loads, 8 skip the weight loads
  int dbg;
};

__device__ __forceinline__ void sk_stamp(const SkParams& p, int slot) {
  if (p.trace != nullptr) p.trace[static_cast<size_t>(blockIdx.x) * 8 + slot] = globaltimer_ns();
}

__device__ __forceinline__ int64_t unit_start(int c, int64_t units, int grid) {
  return units * c / grid;
}

__device__ __forceinline__ void st_release_gpu(int* p, int v) {
  asm volatile("st.release.gpu.global.b32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ int ld_acquire_gpu(const int* p) {
  int v;
  asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Walks a CTA's stages: each stage holds up to kps k-blocks of one tile.
struct StageCursor {
  int64_t u, u1;
  int num_kb, kps;
  int tile, kb, left;  // current stage: tile, first k-block, k-blocks left in its segment
  __device__ void init(int64_t a, int64_t b, int nkb, int k) {
    u = a, u1 = b, num_kb = nkb, kps = k;
    load();
  }
  __device__ void load() {
    if (u >= u1) return;
    tile = static_cast<int>(u / num_kb);
    kb = static_cast<int>(u - static_cast<int64_t>(tile) * num_kb);
    left = static_cast<int>(min(u1, static_cast<int64_t>(tile + 1) * num_kb) - u);
  }
  __device__ bool valid() const { return u < u1; }
  __device__ int count() const { return min(kps, left); }  // k-blocks of the current stage
  __device__ void next() {
    const int n = count();
    u += n;
    kb += n;
    left -= n;
    if (left == 0) load();
  }
};

template <int BN, int R>
struct SkSmem {
  static constexpr uint32_t kA = R * 128 * 128;  // one k-block of weights: 128 R rows x 128 bytes
  static constexpr uint32_t kB = BN * 128;       // one k-block of tokens
  static constexpr int kBufCols = R * BN;        // TMEM columns of one accumulator
  static constexpr int kBufs = 2 * kBufCols <= 512 ? 2 : 1;
  static constexpr uint32_t kTmemCols = kBufs * kBufCols <= 32 ? 32
                                        : kBufs * kBufCols <= 64 ? 64
                                        : kBufs * kBufCols <= 128 ? 128
                                        : kBufs * kBufCols <= 256 ? 256 : 512;
  // ring, barriers (512 B), output staging tile, alignment slack
  static uint32_t bytes(int stages, int kps) { return stages * kps * (kA + kB) + 512 + kStageBytes + 1024; }
};

template <int BN, int R>
__global__ void __launch_bounds__(kSkThreads, 1)
    gemm_streamk_kernel(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmX, SkParams p) {
  using S = SkSmem<BN, R>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  const int stages = p.stages, kps = p.kps;
  const uint32_t stA = kps * S::kA, stB = kps * S::kB;
  uint8_t* sA = smem;
  uint8_t* sB = smem + stages * stA;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + stages * (stA + stB));
  uint64_t* empty = full + stages;
  uint64_t* acc_full = empty + stages;    // [2]
  uint64_t* acc_empty = acc_full + 2;     // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t units = static_cast<int64_t>(p.num_tiles) * p.num_kb;
  const int64_t u0 = unit_start(blockIdx.x, units, p.grid);
  const int64_t u1 = unit_start(blockIdx.x + 1, units, p.grid);

  pdl_launch_dependents();
  if (threadIdx.x == 0) sk_stamp(p, 0);
  if (threadIdx.x == 0) {
    for (int s = 0; s < stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 4);
    }
    fence_barrier_init();
    prefetch_tmap(&tmW);
    prefetch_tmap(&tmX);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, S::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  if (threadIdx.x == 0) sk_stamp(p, 1);

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    // 1. weights of the first ring's worth of stages (they do not depend on
    //    the previous kernel); 2. griddepcontrol.wait; 3. the x halves of
    //    those stages; 4. the remaining stages, both operands.
    const uint32_t stage_bytes = stA + stB;
    StageCursor cur;
    cur.init(u0, u1, p.num_kb, kps);
    int total = 0;
    for (StageCursor c2 = cur; c2.valid(); c2.next()) ++total;
    const int pre = min(total, stages);
    StageCursor c1 = cur;
    const bool do_x = (p.dbg & 4) == 0, do_w = (p.dbg & 8) == 0;
    const uint32_t tx_bytes = (do_w ? stA : 0u) + (do_x ? stB : 0u);
    for (int it = 0; it < pre; ++it, c1.next()) {
      if (lane == 0) {
        if (tx_bytes > 0) mbar_arrive_expect_tx(&full[it], tx_bytes);
        else mbar_arrive(&full[it]);
        if (do_w) tma_load_3d(sA + it * stA, &tmW, &full[it], 0, c1.tile * 128 * R, c1.kb);
      }
    }
    pdl_wait();
    if (lane == 0) sk_stamp(p, 2);
    c1 = cur;
    for (int it = 0; it < pre; ++it, c1.next())
      if (lane == 0 && do_x) tma_load_3d(sB + it * stB, &tmX, &full[it], 0, 0, c1.kb);
    __syncwarp();
    for (int it = pre; it < total; ++it, c1.next()) {
      const int s = it % stages;
      const uint32_t ph = (it / stages) & 1u;
      if (!__all_sync(0xffffffffu, mbar_wait(&empty[s], ph ^ 1u, p.err, 401))) break;
      if (lane == 0) {
        if (tx_bytes > 0) mbar_arrive_expect_tx(&full[s], tx_bytes);
        else mbar_arrive(&full[s]);
        if (do_w) tma_load_3d(sA + s * stA, &tmW, &full[s], 0, c1.tile * 128 * R, c1.kb);
        if (do_x) tma_load_3d(sB + s * stB, &tmX, &full[s], 0, 0, c1.kb);
      }
      __syncwarp();
    }
  } else if (warp == 1) {
    // ----------------------------------------------------------------- MMA
    constexpr uint32_t idesc = make_idesc_bf16(128, BN);
    int it = 0, seg = 0;
    for (int64_t u = u0; u < u1; ++seg) {
      const int tile = static_cast<int>(u / p.num_kb);
      const int64_t seg_end = min(u1, static_cast<int64_t>(tile + 1) * p.num_kb);
      const int nkb = static_cast<int>(seg_end - u);
      const int nst = (nkb + kps - 1) / kps;
      const int buf = S::kBufs == 2 ? (seg & 1) : 0;
      const int use = S::kBufs == 2 ? (seg >> 1) : seg;  // uses of this buffer before
      if (use > 0 && !__all_sync(0xffffffffu, mbar_wait(&acc_empty[buf], (use - 1) & 1u, p.err, 402))) break;
      tc_fence_after();
      const uint32_t dacc = tmem + buf * S::kBufCols;
      bool ok = true;
      for (int i = 0; i < nst; ++i, ++it) {
        const int s = it % stages;
        const uint32_t ph = (it / stages) & 1u;
        if (!__all_sync(0xffffffffu, mbar_wait(&full[s], ph, p.err, 403))) {
          ok = false;
          break;
        }
        tc_fence_after();
        if (lane == 0) {
          const int nj = (p.dbg & 2) ? 0 : min(kps, nkb - i * kps);
          for (int j = 0; j < nj; ++j) {
#pragma unroll
            for (int r = 0; r < R; ++r) {
              const uint32_t a_addr = smem_u32(sA + s * stA + j * S::kA + r * 128 * 128);
              const uint32_t b_addr = smem_u32(sB + s * stB + j * S::kB);
#pragma unroll
              for (int k = 0; k < 4; ++k)
                tc_mma_f16(dacc + r * BN, make_sdesc_k_sw128(a_addr + k * 32), make_sdesc_k_sw128(b_addr + k * 32),
                           idesc, (i > 0 || j > 0 || k > 0) ? 1u : 0u);
            }
          }
          tc_commit(&empty[s]);
        }
        __syncwarp();
      }
      if (!ok) break;
      if (lane == 0) tc_commit(&acc_full[buf]);
      __syncwarp();
      u = seg_end;
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int sub = warp & 3;
    const int row = sub * 32 + lane;  // TMEM lane == weight row within a 128-row sub-tile
    float* stage = reinterpret_cast<float*>(smem + stages * (stA + stB) + 512);  // [32][kStageLd] output staging
    const int et = threadIdx.x - 64;  // 0..127
    int seg = 0;
    for (int64_t u = u0; u < u1; ++seg) {
      const int tile = static_cast<int>(u / p.num_kb);
      const int64_t t_begin = static_cast<int64_t>(tile) * p.num_kb;
      const int64_t t_end = t_begin + p.num_kb;
      const int64_t seg_end = min(u1, t_end);
      const bool head = u == t_begin;       // this CTA holds the tile's first k-block
      const bool whole = head && seg_end == t_end && (blockIdx.x + 1 >= p.grid ||
                                                     unit_start(blockIdx.x + 1, units, p.grid) >= t_end);
      const int buf = S::kBufs == 2 ? (seg & 1) : 0;
      const int use = S::kBufs == 2 ? (seg >> 1) : seg;
      const bool ok = mbar_wait(&acc_full[buf], use & 1u, p.err, 404);
      tc_fence_after();
      if (et == 0) sk_stamp(p, seg == 0 ? 3 : 4);
      const uint32_t taddr = tmem + buf * S::kBufCols + (static_cast<uint32_t>(sub * 32) << 16);
      if (!head) {
        // contributor: park the partial tile in this CTA's slot
        float* slot = p.ws + static_cast<size_t>(blockIdx.x) * (R * BN * 128);
#pragma unroll 1
        for (int r = 0; r < R; ++r) {
#pragma unroll 1
          for (int c = 0; c < BN; c += (BN < 32 ? BN : 32)) {
            uint32_t v[32];
            if constexpr (BN < 32) {
              uint32_t v16[16];
              tmem_ld_32x32b_x16(taddr + r * BN + c, v16);
#pragma unroll
              for (int j = 0; j < 16; ++j) v[j] = v16[j];
            } else {
              tmem_ld_32x32b_x32(taddr + r * BN + c, v);
            }
            tc_wait_ld();
            if ((p.dbg & 1) == 0) {
              // layout [R][BN / 4][128 rows][4 tokens]: a warp's float4
              // stores cover 512 contiguous bytes
              float4* s4 = reinterpret_cast<float4*>(slot) + (static_cast<size_t>(r) * (BN / 4) + c / 4) * 128 + row;
#pragma unroll
              for (int q = 0; q < (BN < 32 ? BN : 32) / 4; ++q)
                s4[static_cast<size_t>(q) * 128] =
                    ok ? make_float4(__uint_as_float(v[4 * q]), __uint_as_float(v[4 * q + 1]),
                                     __uint_as_float(v[4 * q + 2]), __uint_as_float(v[4 * q + 3]))
                       : make_float4(0.f, 0.f, 0.f, 0.f);
            }
          }
        }
        // every epilogue thread's partial is written; one thread publishes
        // them (the barrier orders the other threads' stores before its
        // release store, which is cumulative at GPU scope)
        asm volatile("bar.sync 1, 128;" ::: "memory");
        if (et == 0) {
          __threadfence();
          st_release_gpu(p.flags + static_cast<size_t>(blockIdx.x) * kFlagStride, 1);
        }
      } else {
        // owner (or a whole tile): contributors are the CTAs that start inside this tile
        int c_last = blockIdx.x;
        if (!whole) {
          while (c_last + 1 < p.grid && unit_start(c_last + 1, units, p.grid) < t_end) ++c_last;
          // one thread polls the contributors' flags (bounded, backing off so
          // the flag lines are not hammered), then releases the others
          if (et == 0) {
            for (int c2 = blockIdx.x + 1; c2 <= c_last; ++c2) {
              const uint64_t t0 = globaltimer_ns();
              uint32_t spins = 0;
              while (ld_acquire_gpu(p.flags + static_cast<size_t>(c2) * kFlagStride) == 0) {
                __nanosleep(64);
                if (((++spins) & 0xFFu) == 0 && globaltimer_ns() - t0 > kWaitBudgetNs) {
                  p.err.report(kErrMbarTimeout, 405);
                  break;
                }
              }
            }
          }
          asm volatile("bar.sync 1, 128;" ::: "memory");
        }
        if (et == 0) sk_stamp(p, 5);
        const int tok_step = BN < 32 ? BN : 32;
#pragma unroll 1
        for (int r = 0; r < R; ++r) {
          const int f_row = tile * 128 * R + r * 128 + row;  // this thread's output feature
          const float b = (p.bias != nullptr && f_row < p.N) ? __bfloat162float(p.bias[f_row]) : 0.f;
#pragma unroll 1
          for (int c = 0; c < BN; c += tok_step) {
            uint32_t v[32];
            if constexpr (BN < 32) {
              uint32_t v16[16];
              tmem_ld_32x32b_x16(taddr + r * BN + c, v16);
#pragma unroll
              for (int j = 0; j < 16; ++j) v[j] = v16[j];
            } else {
              tmem_ld_32x32b_x32(taddr + r * BN + c, v);
            }
            tc_wait_ld();
            float acc[32];
#pragma unroll
            for (int j = 0; j < 32; ++j) acc[j] = j < tok_step ? __uint_as_float(v[j]) : 0.f;
            for (int c2 = blockIdx.x + 1; c2 <= c_last; ++c2) {
              const float4* s4 = reinterpret_cast<const float4*>(p.ws + static_cast<size_t>(c2) * (R * BN * 128)) +
                                 (static_cast<size_t>(r) * (BN / 4) + c / 4) * 128 + row;
              float4 pv[8];
#pragma unroll
              for (int q = 0; q < 8; ++q)  // every load in flight before the adds
                if (q < tok_step / 4) pv[q] = s4[static_cast<size_t>(q) * 128];
#pragma unroll
              for (int q = 0; q < 8; ++q)
                if (q < tok_step / 4) {
                  acc[4 * q] += pv[q].x;
                  acc[4 * q + 1] += pv[q].y;
                  acc[4 * q + 2] += pv[q].z;
                  acc[4 * q + 3] += pv[q].w;
                }
            }
            // stage the chunk token-major in shared memory, then store each
            // token's 128 features with 16-byte vectors (256 contiguous bytes
            // per half-warp) instead of one 2-byte store per element
#pragma unroll
            for (int j = 0; j < 32; ++j)
              if (j < tok_step) stage[j * kStageLd + row] = acc[j] + b;
            asm volatile("bar.sync 1, 128;" ::: "memory");
            if ((p.dbg & 1) == 0) {
              const int f0 = tile * 128 * R + r * 128;
              const int col = (lane & 15) * 8;  // 8 features per lane
#pragma unroll
              for (int i = 0; i < 4; ++i) {
                const int t = sub * 8 + i * 2 + (lane >> 4);  // token within the chunk
                const int m = c + t;
                if (t >= tok_step || m >= p.M) continue;
                const float* src = stage + t * kStageLd + col;
                const float4 lo = *reinterpret_cast<const float4*>(src);
                const float4 hi = *reinterpret_cast<const float4*>(src + 4);
                const int f = f0 + col;
                if (p.out_f32) {
                  float* dst = reinterpret_cast<float*>(p.out) + static_cast<size_t>(m) * p.ldo + f;
                  if (p.vec_ok && f + 8 <= p.N) {
                    *reinterpret_cast<float4*>(dst) = lo;
                    *reinterpret_cast<float4*>(dst + 4) = hi;
                  } else {
                    const float e8[8] = {lo.x, lo.y, lo.z, lo.w, hi.x, hi.y, hi.z, hi.w};
                    for (int q = 0; q < 8; ++q)
                      if (f + q < p.N) dst[q] = e8[q];
                  }
                } else {
                  __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(p.out) + static_cast<size_t>(m) * p.ldo + f;
                  if (p.vec_ok && f + 8 <= p.N) {
                    uint4 pk;
                    pk.x = pack_bf16x2(lo.x, lo.y);
                    pk.y = pack_bf16x2(lo.z, lo.w);
                    pk.z = pack_bf16x2(hi.x, hi.y);
                    pk.w = pack_bf16x2(hi.z, hi.w);
                    *reinterpret_cast<uint4*>(dst) = pk;
                  } else {
                    const float e8[8] = {lo.x, lo.y, lo.z, lo.w, hi.x, hi.y, hi.z, hi.w};
                    for (int q = 0; q < 8; ++q)
                      if (f + q < p.N) dst[q] = __float2bfloat16_rn(e8[q]);
                  }
                }
              }
            }
            asm volatile("bar.sync 1, 128;" ::: "memory");  // the stage is rewritten by the next chunk
          }
        }
        if (!whole) {
          asm volatile("bar.sync 1, 128;" ::: "memory");
          if (et == 0)  // ready for the next launch
            for (int c2 = blockIdx.x + 1; c2 <= c_last; ++c2) p.flags[static_cast<size_t>(c2) * kFlagStride] = 0;
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[buf]);
      u = seg_end;
    }
  }

  tc_fence_before();
  __syncthreads();
  if (threadIdx.x == 0) sk_stamp(p, 6);
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, S::kTmemCols);
  }
}

template <int BN, int R>
void launch_sk(const GemmStreamKArgs& a, SkParams p, cudaStream_t stream) {
  using S = SkSmem<BN, R>;
  // k-blocks per stage and ring depth from the byte budget: about eight
  // k-blocks in flight, at most four per stage
  const uint32_t per_kb = S::kA + S::kB;
  const int in_flight = std::max(2, std::min(8, static_cast<int>(kSkSmemBudget / per_kb)));
  int kps = a.kps > 0 ? a.kps : (in_flight >= 8 ? 2 : 1);
  kps = std::min(kps, std::max(1, in_flight / 2));
  const int stages = std::max(2, in_flight / kps);
  p.kps = kps;
  p.stages = stages;
  const CUtensorMap tw = make_tmap_bf16_kblocks(a.w, a.N, a.K, a.ldw, 128 * R, kps);
  const CUtensorMap tx = make_tmap_bf16_kblocks(a.x, a.M, a.K, a.ldx, BN, kps);
  auto kern = gemm_streamk_kernel<BN, R>;
  const uint32_t smem = S::bytes(stages, kps);
  static bool configured[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (!configured[dev & 63]) {
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
    configured[dev & 63] = true;
  }
  launch_pdl(kern, dim3(p.grid), dim3(kSkThreads), smem, stream, tw, tx, p);
}

template <int R>
void dispatch_bn(int bn, const GemmStreamKArgs& a, const SkParams& p, cudaStream_t s) {
  switch (bn) {
    case 16: return launch_sk<16, R>(a, p, s);
    case 32: return launch_sk<32, R>(a, p, s);
    case 64: return launch_sk<64, R>(a, p, s);
    case 128: return launch_sk<128, R>(a, p, s);
    default: return launch_sk<256, R>(a, p, s);
  }
}

}  // namespace

int gemm_streamk_grid(int M, int N, int K, int R, int sms) {
  const int tiles = (N + 128 * R - 1) / (128 * R);
  const int64_t units = static_cast<int64_t>(tiles) * (K / 64);
  // MINISGL_STREAMK_CTAS caps the grid (measurement switch)
  static const int cap = [] {
    const char* v = std::getenv("MINISGL_STREAMK_CTAS");
    return v != nullptr && v[0] != '\0' ? std::atoi(v) : 0;
  }();
  const int limit = cap > 0 ? std::min(cap, sms) : sms;
  // at least two k-blocks per CTA
  return static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(limit, units / 2)));
}

void launch_gemm_streamk(const GemmStreamKArgs& a, cudaStream_t stream) {
  if (a.M <= 0 || a.N <= 0) return;
  if (a.M > 256) throw std::runtime_error("minisgl.gemm_streamk: at most 256 tokens");
  if (a.K % 64 != 0 || a.K <= 0) throw std::runtime_error("minisgl.gemm_streamk: K must be a positive multiple of 64");
  if (a.ldx % 8 != 0 || a.ldw % 8 != 0) throw std::runtime_error("minisgl.gemm_streamk: row strides must be multiples of 8");
  if (a.R != 1 && a.R != 2) throw std::runtime_error("minisgl.gemm_streamk: R must be 1 or 2");
  const int bn = a.M <= 16 ? 16 : a.M <= 32 ? 32 : a.M <= 64 ? 64 : a.M <= 128 ? 128 : 256;
  SkParams p{};
  p.out = a.out;
  p.bias = static_cast<const __nv_bfloat16*>(a.bias);
  p.M = a.M;
  p.N = a.N;
  p.K = a.K;
  p.ldo = a.ldo;
  p.out_f32 = a.out_f32;
  p.vec_ok = (reinterpret_cast<uintptr_t>(a.out) % 16 == 0) && (a.ldo % (a.out_f32 ? 4 : 8) == 0);
  p.num_tiles = (a.N + 128 * a.R - 1) / (128 * a.R);
  p.num_kb = a.K / 64;
  p.grid = a.grid;
  p.ws = a.ws;
  p.flags = a.flags;
  p.err = ErrorSink{a.err};
  p.trace = static_cast<unsigned long long*>(a.trace);
  static const int dbg = [] {
    const char* v = std::getenv("MINISGL_STREAMK_DEBUG");
    return v != nullptr && v[0] != '\0' ? std::atoi(v) : 0;
  }();
  p.dbg = dbg;
  if (p.grid < 1 || p.grid > a.ws_slots) throw std::runtime_error("minisgl.gemm_streamk: grid exceeds the workspace");
  if (static_cast<int64_t>(a.R) * bn * 128 > a.ws_slot_floats)
    throw std::runtime_error("minisgl.gemm_streamk: workspace slot too small");
  if (a.R == 1) dispatch_bn<1>(bn, a, p, stream);
  else dispatch_bn<2>(bn, a, p, stream);
}

}  // namespace minisgl
