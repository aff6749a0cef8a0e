// Dense bf16 GEMM on 5th-generation tensor cores (tcgen05 + TMEM + TMA).
//
//   out[M, N] = x[M, K] @ w[N, K]^T (+ bias)        (the F.linear convention)
//
// Replaces the cuBLAS calls behind every dense projection in the reference
// (python/minisgl/layers/linear.py:31-32, layers/embedding.py:98).
//
// One CTA computes one 128 x BN output tile:
//   warp 0      TMA producer: streams 128x64 and BNx64 bf16 k-blocks into a
//               STAGES-deep ring of 128B-swizzled shared-memory buffers;
//   warp 1      allocates TMEM and issues tcgen05.mma (M=128, N=BN, K=16)
//               from a single thread, committing each stage back to the
//               producer through an mbarrier;
//   warps 2..5  epilogue: tcgen05.ld the fp32 accumulator (each warp owns
//               the 32 TMEM lanes of its sub-partition), add bias, convert
//               and store.
//
// Two tile orientations:
//   token-major   (A = x, B = w): rows of the tile are tokens. Used when M is
//                 large (prefill).
//   weight-major  (A = w, B = x): rows are output features and the token
//                 count becomes the MMA N dimension (16..256). Used for small
//                 M (decode) so the 128-row MMA is filled by weights rather
//                 than by padding rows.
// Split-K spreads the K loop over gridDim.z CTAs when there are too few tiles
// to cover the 148 SMs; partial sums go to an fp32 workspace and a small
// reduction kernel finishes the tile (bias, conversion).
#include <algorithm>
#include <stdexcept>
#include <string>

#include "common.cuh"
#include "ops.h"
#include "tma_host.h"

namespace minisgl {
namespace {

constexpr int BM = 128;
constexpr int BK = 64;
constexpr int kThreads = 192;

struct KParams {
  void* out;
  float* ws;
  const __nv_bfloat16* bias;
  int M, N;            // logical output is out[M, N] (M = tokens, N = features)
  int ldo;
  int kb_per_split;
  int num_kb;
  int out_f32;
  ErrorSink err;
};

template <int BN, int STAGES>
struct Smem {
  static constexpr uint32_t kA = BM * BK * 2;
  static constexpr uint32_t kB = BN * BK * 2;
  static constexpr uint32_t kBytes = STAGES * (kA + kB) + 1024 /*align*/ + 256 /*barriers*/;
};

template <int N>
struct TmemCols {
  static constexpr uint32_t value = N <= 32 ? 32 : (N <= 64 ? 64 : (N <= 128 ? 128 : 256));
};

// SWAP = weight-major tiles; SPLIT = write fp32 partials to the workspace.
template <int BN, int STAGES, bool SWAP, bool SPLIT>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                   KParams p) {
  using S = Smem<BN, STAGES>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * S::kA;
  uint64_t* full = reinterpret_cast<uint64_t*>(sB + STAGES * S::kB);
  uint64_t* empty = full + STAGES;
  uint64_t* done = empty + STAGES;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);

  constexpr uint32_t kCols = TmemCols<BN>::value;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int a_row0 = blockIdx.y * BM;
  const int b_row0 = blockIdx.x * BN;
  const int kb0 = blockIdx.z * p.kb_per_split;
  const int kb1 = min(p.num_kb, kb0 + p.kb_per_split);
  const int nkb = kb1 - kb0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(done, 1);
    fence_barrier_init();
    prefetch_tmap(&tmA);
    prefetch_tmap(&tmB);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, kCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      for (int i = 0; i < nkb; ++i) {
        const int s = i % STAGES;
        const uint32_t ph = (i / STAGES) & 1u;
        if (!mbar_wait(&empty[s], ph ^ 1u, p.err, 101)) break;
        mbar_arrive_expect_tx(&full[s], S::kA + S::kB);
        const int kc = (kb0 + i) * BK;
        tma_load_2d(sA + s * S::kA, &tmA, &full[s], kc, a_row0);
        tma_load_2d(sB + s * S::kB, &tmB, &full[s], kc, b_row0);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = make_idesc_bf16(BM, BN);
      for (int i = 0; i < nkb; ++i) {
        const int s = i % STAGES;
        const uint32_t ph = (i / STAGES) & 1u;
        if (!mbar_wait(&full[s], ph, p.err, 102)) break;
        tc_fence_after();
        const uint32_t a_addr = smem_u32(sA + s * S::kA);
        const uint32_t b_addr = smem_u32(sB + s * S::kB);
#pragma unroll
        for (int k = 0; k < BK / 16; ++k) {
          tc_mma_f16(tmem, make_sdesc_k_sw128(a_addr + k * 32), make_sdesc_k_sw128(b_addr + k * 32),
                     idesc, (i > 0 || k > 0) ? 1u : 0u);
        }
        tc_commit(&empty[s]);
      }
      tc_commit(done);
    }
  } else {
    // ------------------------------------------------------- epilogue ----
    const bool ok = mbar_wait(done, 0, p.err, 103);
    tc_fence_after();
    const int sub = warp & 3;
    const int row = sub * 32 + lane;  // TMEM lane == tile row
    const uint32_t taddr = tmem + (static_cast<uint32_t>(sub * 32) << 16);
    constexpr int CH = BN < 32 ? BN : 32;
#pragma unroll 1
    for (int c = 0; c < BN; c += CH) {
      uint32_t r[32];
      if constexpr (CH == 32) {
        tmem_ld_32x32b_x32(taddr + c, r);
      } else {
        uint32_t r16[16];
        tmem_ld_32x32b_x16(taddr + c, r16);
#pragma unroll
        for (int j = 0; j < 16; ++j) r[j] = r16[j];
      }
      tc_wait_ld();
      if (!ok) continue;
      if constexpr (!SWAP) {
        const int m = a_row0 + row;
        if (m >= p.M) continue;
        const int n0 = b_row0 + c;
        if constexpr (SPLIT) {
          float* dst = p.ws + (static_cast<size_t>(blockIdx.z) * p.M + m) * p.N;
#pragma unroll
          for (int j = 0; j < CH; j += 4) {
            const int n = n0 + j;
            if (n + 4 <= p.N) {
              *reinterpret_cast<float4*>(dst + n) =
                  make_float4(__uint_as_float(r[j]), __uint_as_float(r[j + 1]),
                              __uint_as_float(r[j + 2]), __uint_as_float(r[j + 3]));
            } else {
              for (int q = 0; q < 4 && n + q < p.N; ++q) dst[n + q] = __uint_as_float(r[j + q]);
            }
          }
        } else {
          float v[32];
#pragma unroll
          for (int j = 0; j < CH; ++j) {
            v[j] = __uint_as_float(r[j]);
            if (p.bias != nullptr && n0 + j < p.N) v[j] += __bfloat162float(p.bias[n0 + j]);
          }
          if (p.out_f32) {
            float* dst = reinterpret_cast<float*>(p.out) + static_cast<size_t>(m) * p.ldo;
#pragma unroll
            for (int j = 0; j < CH; j += 4) {
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
            for (int j = 0; j < CH; j += 8) {
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
      } else {
        // weight-major: this thread owns feature f; columns are tokens
        const int f = a_row0 + row;
        if (f >= p.N) continue;
        const float b = (!SPLIT && p.bias != nullptr) ? __bfloat162float(p.bias[f]) : 0.f;
#pragma unroll
        for (int j = 0; j < CH; ++j) {
          const int t = b_row0 + c + j;
          if (t >= p.M) break;
          const float v = __uint_as_float(r[j]);
          if constexpr (SPLIT) {
            p.ws[(static_cast<size_t>(blockIdx.z) * p.M + t) * p.N + f] = v;
          } else if (p.out_f32) {
            reinterpret_cast<float*>(p.out)[static_cast<size_t>(t) * p.ldo + f] = v + b;
          } else {
            reinterpret_cast<__nv_bfloat16*>(p.out)[static_cast<size_t>(t) * p.ldo + f] =
                __float2bfloat16_rn(v + b);
          }
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kCols);
  }
}

// out = sum over splits of ws (+ bias), converted to the output dtype.
__global__ void splitk_reduce_kernel(const float* __restrict__ ws, void* out,
                                     const __nv_bfloat16* __restrict__ bias, int M, int N, int ldo,
                                     int splits, int out_f32) {
  const int n4 = N / 4;
  const size_t total = static_cast<size_t>(M) * n4;
  const size_t stride_split = static_cast<size_t>(M) * N;
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<size_t>(gridDim.x) * blockDim.x) {
    const int m = static_cast<int>(i / n4);
    const int n = static_cast<int>(i % n4) * 4;
    const float* src = ws + static_cast<size_t>(m) * N + n;
    float4 acc = *reinterpret_cast<const float4*>(src);
    for (int s = 1; s < splits; ++s) {
      const float4 v = *reinterpret_cast<const float4*>(src + s * stride_split);
      acc.x += v.x, acc.y += v.y, acc.z += v.z, acc.w += v.w;
    }
    if (bias != nullptr) {
      acc.x += __bfloat162float(bias[n]);
      acc.y += __bfloat162float(bias[n + 1]);
      acc.z += __bfloat162float(bias[n + 2]);
      acc.w += __bfloat162float(bias[n + 3]);
    }
    if (out_f32) {
      *reinterpret_cast<float4*>(reinterpret_cast<float*>(out) + static_cast<size_t>(m) * ldo + n) = acc;
    } else {
      uint2 pk;
      pk.x = pack_bf16x2(acc.x, acc.y);
      pk.y = pack_bf16x2(acc.z, acc.w);
      *reinterpret_cast<uint2*>(reinterpret_cast<__nv_bfloat16*>(out) + static_cast<size_t>(m) * ldo + n) = pk;
    }
  }
}

template <int BN, int STAGES, bool SWAP, bool SPLIT>
void launch_tile(const CUtensorMap& ta, const CUtensorMap& tb, const KParams& kp, dim3 grid,
                 cudaStream_t stream) {
  auto kern = gemm_tc_kernel<BN, STAGES, SWAP, SPLIT>;
  constexpr uint32_t smem = Smem<BN, STAGES>::kBytes;
  static bool configured[64] = {};  // one attribute call per instantiation and device
  int dev = 0;
  cudaGetDevice(&dev);
  if (!configured[dev & 63]) {
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    configured[dev & 63] = true;
  }
  kern<<<grid, kThreads, smem, stream>>>(ta, tb, kp);
}

template <int BN, int STAGES, bool SWAP>
void dispatch_split(bool split, const CUtensorMap& ta, const CUtensorMap& tb, const KParams& kp,
                    dim3 grid, cudaStream_t stream) {
  if (split) launch_tile<BN, STAGES, SWAP, true>(ta, tb, kp, grid, stream);
  else launch_tile<BN, STAGES, SWAP, false>(ta, tb, kp, grid, stream);
}

constexpr int kNumSM = 148;

struct Plan {
  bool swap;
  int bn;
  int tiles;  // output tiles
  int splits;
  int kb_per_split;
};

Plan make_plan(int M, int N, int K, int force_mode, int force_splits) {
  Plan pl;
  const int num_kb = (K + BK - 1) / BK;
  pl.swap = force_mode == 2 || (force_mode == 0 && M <= 128);
  if (pl.swap) {
    pl.bn = M <= 16 ? 16 : (M <= 32 ? 32 : (M <= 64 ? 64 : 128));
    pl.tiles = ((N + BM - 1) / BM) * ((M + pl.bn - 1) / pl.bn);
  } else {
    pl.bn = N >= 256 ? 256 : 128;
    pl.tiles = ((M + BM - 1) / BM) * ((N + pl.bn - 1) / pl.bn);
  }
  int splits = 1;
  if (force_splits > 0) {
    splits = force_splits;
  } else if (pl.tiles < kNumSM) {
    // enough CTAs to cover the SMs, at least two k-blocks per split
    splits = std::max(1, std::min(kNumSM / pl.tiles, num_kb / 2));
  }
  splits = std::max(1, std::min(splits, num_kb));
  pl.kb_per_split = (num_kb + splits - 1) / splits;
  pl.splits = (num_kb + pl.kb_per_split - 1) / pl.kb_per_split;  // no empty split
  return pl;
}

}  // namespace

int64_t gemm_workspace_elems(int M, int N, int K) {
  Plan pl = make_plan(M, N, K, 0, 0);
  return pl.splits > 1 ? static_cast<int64_t>(pl.splits) * M * N : 0;
}

void launch_gemm(const GemmArgs& a, cudaStream_t stream) {
  if (a.M <= 0 || a.N <= 0) return;
  if (a.K % 8 != 0 || a.ldx % 8 != 0 || a.ldw % 8 != 0)
    throw std::runtime_error("minisgl.gemm: K and row strides must be multiples of 8 elements");
  if (a.N % 4 != 0) throw std::runtime_error("minisgl.gemm: N must be a multiple of 4");
  Plan pl = make_plan(a.M, a.N, a.K, a.force_mode, a.force_splits);
  if (pl.splits > 1) {
    const int64_t need = static_cast<int64_t>(pl.splits) * a.M * a.N;
    if (a.workspace == nullptr || a.workspace_elems < need) {
      // fall back to fewer splits that fit the workspace
      int fit = a.workspace == nullptr ? 1 : static_cast<int>(a.workspace_elems / (static_cast<int64_t>(a.M) * a.N));
      pl = make_plan(a.M, a.N, a.K, a.force_mode, std::max(1, fit));
    }
  }
  const bool split = pl.splits > 1;
  KParams kp;
  kp.out = a.out;
  kp.ws = a.workspace;
  kp.bias = reinterpret_cast<const __nv_bfloat16*>(a.bias);
  kp.M = a.M;
  kp.N = a.N;
  kp.ldo = a.ldo;
  kp.kb_per_split = pl.kb_per_split;
  kp.num_kb = (a.K + BK - 1) / BK;
  kp.out_f32 = a.out_f32 ? 1 : 0;
  kp.err = ErrorSink{a.err};

  if (pl.swap) {
    CUtensorMap ta = make_tmap_bf16_2d_sw128(a.w, a.N, a.K, a.ldw, BM);
    CUtensorMap tb = make_tmap_bf16_2d_sw128(a.x, a.M, a.K, a.ldx, pl.bn);
    dim3 grid((a.M + pl.bn - 1) / pl.bn, (a.N + BM - 1) / BM, pl.splits);
    switch (pl.bn) {
      case 16: dispatch_split<16, 8, true>(split, ta, tb, kp, grid, stream); break;
      case 32: dispatch_split<32, 8, true>(split, ta, tb, kp, grid, stream); break;
      case 64: dispatch_split<64, 8, true>(split, ta, tb, kp, grid, stream); break;
      default: dispatch_split<128, 6, true>(split, ta, tb, kp, grid, stream); break;
    }
  } else {
    CUtensorMap ta = make_tmap_bf16_2d_sw128(a.x, a.M, a.K, a.ldx, BM);
    CUtensorMap tb = make_tmap_bf16_2d_sw128(a.w, a.N, a.K, a.ldw, pl.bn);
    dim3 grid((a.N + pl.bn - 1) / pl.bn, (a.M + BM - 1) / BM, pl.splits);
    if (pl.bn == 256) dispatch_split<256, 4, false>(split, ta, tb, kp, grid, stream);
    else dispatch_split<128, 6, false>(split, ta, tb, kp, grid, stream);
  }
  if (split) {
    const size_t total = static_cast<size_t>(a.M) * (a.N / 4);
    const int threads = 256;
    const int blocks = static_cast<int>(std::min<size_t>((total + threads - 1) / threads, 148 * 8));
    splitk_reduce_kernel<<<blocks, threads, 0, stream>>>(a.workspace, a.out, kp.bias, a.M, a.N,
                                                         a.ldo, pl.splits, kp.out_f32);
  }
}

}  // namespace minisgl
