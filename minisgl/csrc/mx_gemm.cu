// Block-scaled MX grouped expert GEMM: MXFP4 weights x MXFP8 activations on
// the 5th-generation tensor cores (tcgen05.mma .kind::mxf8f6f4.block_scale),
// and the MXFP8 activation quantiser that feeds it. Replaces the bf16 Triton
// fused_moe kernel of the reference (python/minisgl/kernel/triton/fused_moe.py:50-193)
// for experts quantised with `--moe-quant mxfp4-a8`.
//
// Numbers (OCP microscaling v1.0):
//   weights      E2M1 elements, one E8M0 scale per 32 along K (minisgl.quant.mxfp4)
//   activations  E4M3 elements, one E8M0 scale per 32 along K:
//                e = ceil(log2(amax / 448)) (amax / 448 in fp32), scale byte
//                e + 127, elements x / 2^e rounded to nearest even (they fit
//                E4M3's +-448; satfinite guards the rounding of amax / 448);
//                an all-zero block gets scale byte 0 and zero elements. (The
//                OCP example rule floor(log2 amax) - 8 lets amax / 2^e reach
//                512 and clips up to 12 % off a block's largest element.)
//   product      sum_k (w_k 2^(sw - 127)) (x_k 2^(sx - 127)) accumulated in fp32
//                by the tensor core, which applies both scales per 32-wide block.
//
// Scale layout ("scale block", shared by weights and activations): the
// scales of 128 rows x 128 K elements (4 per row) are 512 bytes, byte
// (r % 32) * 16 + (r / 32) * 4 + j for row r and 32-block j. One
// tcgen05.cp .32x128b.warpx4 moves a block into 4 TMEM columns (lane r % 32
// of every lane quarter, column r / 32, byte j); the MMA of the j-th K=32
// step selects byte j through the scale-factor ids of its instruction
// descriptor. Storage:
//   weight scales      [E, N / 128, K / 128, 512]   (minisgl.quant.mxfp4.block_scales)
//   activation scales  [P / tile, K / 128, 512]     one block per token tile;
//                      a tile of fewer than 128 rows uses rows 0..tile-1,
//                      the rest of its block is zero
//
// Per k-block of 128 the producer moves (all single-CTA copies):
//   - 128 weight rows of packed E2M1 by TMA with the 16U4_ALIGN16B element
//     type: 8 KB from HBM, landing as 16 KB in shared memory (each 8-byte
//     group of 16 codes padded to 16 bytes, the operand layout the
//     mxf8f6f4 kind reads for 4-bit types), 128-byte swizzle;
//   - the tile's E4M3 token rows by TMA, 128-byte swizzle;
//   - the two 512-byte scale blocks by bulk copies.
// One thread copies the scale blocks to TMEM and issues the four K=32 MMAs
// (weights as the 128-row A operand, tokens as N); a commit frees the stage.
// The epilogue is the grouped GEMM's usual one: TMEM lane r is weight row
// n0 + r, columns are tokens; interleaved gate|up rows become
// silu(gate) * up.
#include <cuda_fp8.h>

#include <cstdlib>
#include <stdexcept>
#include <string>

#include "common.cuh"
#include "launch.h"
#include "ops.h"
#include "tma_host.h"

namespace minisgl {
namespace {

// ------------------------------------------------ MXFP8 quantiser ----
// One warp per (row, 128-wide k-block); lane l owns elements 4l..4l+3, so
// the 8 lanes of a 32-block reduce its amax with three shuffles.
__global__ void __launch_bounds__(256)
    mx8_quantize_rows_kernel(uint32_t* q, uint8_t* sf, const __nv_bfloat16* x, const int32_t* idx, int k,
                             int rows, int K, int tile, const int32_t* num_tiles) {
  pdl_launch_dependents();
  pdl_wait();  // the gather index and the rows come from earlier kernels
  const int nkb = K / 128;
  const int64_t w = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (w >= static_cast<int64_t>(rows) * nkb) return;
  const int p = static_cast<int>(w / nkb), kb = static_cast<int>(w % nkb);
  if (num_tiles != nullptr && p / tile >= *num_tiles) return;  // rows of tiles nobody reads
  const int lane = threadIdx.x & 31;
  int src = p;
  if (idx != nullptr) {
    const int s = idx[p];
    src = s >= 0 ? s / k : -1;  // -1: a padding row of the expert-sorted order
  }
  float v[4] = {0.f, 0.f, 0.f, 0.f};
  if (src >= 0) {
    const uint2 u = *reinterpret_cast<const uint2*>(x + static_cast<int64_t>(src) * K + kb * 128 + lane * 4);
    const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u.x));
    const float2 b = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u.y));
    v[0] = a.x, v[1] = a.y, v[2] = b.x, v[3] = b.y;
  }
  float amax = fmaxf(fmaxf(fabsf(v[0]), fabsf(v[1])), fmaxf(fabsf(v[2]), fabsf(v[3])));
#pragma unroll
  for (int o = 1; o < 8; o <<= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  // scale 2^e with e = ceil(log2(amax / 448)): the biased exponent of
  // amax / 448, one up unless that is an exact power of two
  const uint32_t sb = __float_as_uint(amax * (1.f / 448.f));
  const uint32_t sbyte = ((sb >> 23) & 0xFFu) + ((sb & 0x7FFFFFu) != 0u ? 1u : 0u);
  const float inv = sbyte != 0 ? __uint_as_float((254u - sbyte) << 23) : 0.f;  // 2^-(sbyte - 127)
  const __nv_fp8x2_storage_t lo = __nv_cvt_float2_to_fp8x2(make_float2(v[0] * inv, v[1] * inv), __NV_SATFINITE,
                                                           __NV_E4M3);
  const __nv_fp8x2_storage_t hi = __nv_cvt_float2_to_fp8x2(make_float2(v[2] * inv, v[3] * inv), __NV_SATFINITE,
                                                           __NV_E4M3);
  q[(static_cast<int64_t>(p) * K + kb * 128) / 4 + lane] =
      static_cast<uint32_t>(lo) | (static_cast<uint32_t>(hi) << 16);
  // the four scale bytes of this row's k-block sit in lanes 0, 8, 16, 24
  uint32_t word = 0;
#pragma unroll
  for (int j = 0; j < 4; ++j) word |= (__shfl_sync(0xffffffffu, sbyte, 8 * j) & 0xFFu) << (8 * j);
  const int t = p / tile, r = p % tile;
  uint8_t* blk = sf + (static_cast<int64_t>(t) * nkb + kb) * 512;
  if (lane == 0) *reinterpret_cast<uint32_t*>(blk + (r % 32) * 16 + (r / 32) * 4) = word;
  // a tile of fewer than 128 rows leaves rows tile..127 of its block unused: zero them
  if (tile < 128 && lane > 0 && lane < 128 / tile) {
    const int rr = r + lane * tile;
    *reinterpret_cast<uint32_t*>(blk + (rr % 32) * 16 + (rr / 32) * 4) = 0u;
  }
}

// ------------------------------------------- block-scaled grouped GEMM ----
constexpr int XBM = 128;                   // weight rows per tile (MMA M)
constexpr int XBK = 128;                   // K elements per k-block
constexpr int kXThreads = 192;             // warp 0 TMA, warp 1 TMEM + MMA, warps 2-5 epilogue
constexpr int kWTile = XBM * XBK;          // unpacked E2M1 tile in shared memory (16 KB)
constexpr int kWTx = XBM * XBK / 2;        // its transaction bytes: the packed size read from HBM
constexpr int kSfBlock = 512;

template <int BN, int STAGES>
struct XSmem {
  static constexpr int kAct = BN * XBK;  // E4M3 token tile
  static constexpr int kStage = (kWTile + kAct + 2 * kSfBlock + 1023) / 1024 * 1024;  // swizzle alignment
  static constexpr int kXchg = 64 * BN * 4;  // SiLU epilogue: up rows, fp32 (aliases the ring)
  static constexpr int kRing = STAGES * kStage > kXchg ? STAGES * kStage : kXchg;
  static constexpr int kBytes = 1024 + kRing + 256;
  static constexpr uint32_t kAccCols = BN < 32 ? 32 : BN;
  // accumulator columns, then 4 columns of weight scales and 4 of token scales
  static constexpr uint32_t kCols = kAccCols + 8 <= 64 ? 64 : (kAccCols + 8 <= 128 ? 128 : 256);
};

struct XParams {
  void* out;                // [P, ldo] bf16
  int ldo;
  const uint8_t* sfw;       // [E, N / 128, K / 128, 512]
  const uint8_t* sfx;       // [P / BN, K / 128, 512]
  int N, K;                 // per expert: N rows of K
  int silu;                 // interleaved gate|up rows: write silu(gate) * up (N / 2 features)
  const int32_t* tile_expert;
  const int32_t* tile_row;
  const int32_t* num_tiles;
  ErrorSink err;
};

// D[tmem] (+)= A[smem] * B[smem]^T with per-32 E8M0 scales of A and B read
// from TMEM (addresses carry the scale byte in their top two bits).
__device__ __forceinline__ void tc_mma_mx(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                          uint32_t sfa_tmem, uint32_t sfb_tmem, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::mxf8f6f4.block_scale [%0], %1, %2, %3, [%5], [%6], p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(sfa_tmem), "r"(sfb_tmem)
      : "memory");
}

// Shared memory -> TMEM: 32 rows of 16 bytes into 32 lanes x 4 columns,
// repeated in all four lane quarters. Issued by the MMA thread before the
// MMAs that read it (the two are ordered for one issuing thread).
__device__ __forceinline__ void tc_cp_32x128b_x4(uint32_t taddr, uint64_t sdesc) {
  asm volatile("tcgen05.cp.cta_group::1.32x128b.warpx4 [%0], %1;" ::"r"(taddr), "l"(sdesc) : "memory");
}

// Descriptor of a scale block as the copy's source: K-major without
// swizzle, 8-row core groups of 8 x 16 bytes, 128 bytes apart (SBO).
__device__ __forceinline__ uint64_t make_sdesc_scales(uint32_t smem_addr) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((smem_addr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>(128u >> 4) << 32;  // SBO
  d |= static_cast<uint64_t>(1u) << 46;          // descriptor version for sm_100
  return d;                                      // layout type 0: no swizzle
}

// Instruction descriptor of .kind::mxf8f6f4.block_scale: A E2M1 (5), B E4M3
// (0), both K-major, E8M0 scales (bit 23), scale byte `j` of A and of B.
// Bits: [4,6) B scale id | [7,10) A fmt | [10,13) B fmt | [17,23) N>>3
//       | 23 scale fmt | [24,29) M>>4 | [29,31) A scale id.
__host__ __device__ constexpr uint32_t make_idesc_mx(int M, int N, uint32_t j) {
  return (j << 4) | (5u << 7) | (0u << 10) | (static_cast<uint32_t>(N >> 3) << 17) | (1u << 23) |
         (static_cast<uint32_t>(M >> 4) << 24) | (j << 29);
}

template <int BN, int STAGES>
__global__ void __launch_bounds__(kXThreads, 1)
    moe_mx_gemm_kernel(const __grid_constant__ CUtensorMap tm_w, const __grid_constant__ CUtensorMap tm_x,
                       const XParams p) {
  using S = XSmem<BN, STAGES>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint8_t* ring = smem;  // stage s at ring + s * kStage: [weights 16 KB][tokens][weight scales][token scales]
  uint8_t* xchg = ring;  // epilogue only: after the last MMA completed
  uint64_t* full = reinterpret_cast<uint64_t*>(ring + S::kRing);  // [STAGES] copies landed
  uint64_t* empty = full + STAGES;                                  // [STAGES] MMAs done with the stage
  uint64_t* done = empty + STAGES;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  pdl_launch_dependents();
  pdl_wait();  // the tile tables, the token rows and their scales come from earlier kernels
  const int tile = blockIdx.x;
  if (tile >= *p.num_tiles) return;
  const int expert = p.tile_expert[tile];
  const int row0 = p.tile_row[tile];
  const int n0 = blockIdx.y * XBM;  // weight row block inside the expert
  const int nkb = p.K / XBK;
  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(done, 1);
    fence_barrier_init();
    prefetch_tmap(&tm_w);
    prefetch_tmap(&tm_x);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, S::kCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t sfa_tmem = tmem + S::kAccCols;      // lane 0, 4 columns of weight scales
  const uint32_t sfb_tmem = tmem + S::kAccCols + 4;  // lane 0, 4 columns of token scales
  bool ok = true;

  if (warp == 0) {
    // ------------------------------------------------------------ TMA ----
    if (lane == 0) {
      const uint8_t* sfw = p.sfw + (static_cast<int64_t>(expert) * (p.N / XBM) + n0 / XBM) * nkb * kSfBlock;
      const uint8_t* sfx = p.sfx + static_cast<int64_t>(row0 / BN) * nkb * kSfBlock;
      for (int kb = 0; kb < nkb; ++kb) {
        const int s = kb % STAGES;
        if (kb >= STAGES && !mbar_wait(&empty[s], ((kb / STAGES) - 1) & 1, p.err, 451)) break;
        uint8_t* st = ring + s * S::kStage;
        mbar_arrive_expect_tx(&full[s], kWTx + S::kAct + 2 * kSfBlock);
        tma_load_2d(st, &tm_w, &full[s], kb * XBK, expert * p.N + n0);  // x in E2M1 elements
        tma_load_2d(st + kWTile, &tm_x, &full[s], kb * XBK, row0);     // x in bytes (E4M3)
        bulk_load(st + kWTile + S::kAct, sfw + static_cast<int64_t>(kb) * kSfBlock, kSfBlock, &full[s]);
        bulk_load(st + kWTile + S::kAct + kSfBlock, sfx + static_cast<int64_t>(kb) * kSfBlock, kSfBlock,
                  &full[s]);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA ----
    for (int kb = 0; kb < nkb && ok; ++kb) {
      const int s = kb % STAGES;
      ok = __all_sync(0xffffffffu, mbar_wait(&full[s], (kb / STAGES) & 1, p.err, 452));
      if (!ok) break;
      tc_fence_after();
      if (lane == 0) {
        const uint32_t a = smem_u32(ring + s * S::kStage);
        const uint32_t b = a + kWTile;
        const uint32_t sa = b + S::kAct, sb = sa + kSfBlock;
        // the previous k-block's MMAs read these TMEM columns; copies and
        // MMAs issued by this thread run in order
        tc_cp_32x128b_x4(sfa_tmem, make_sdesc_scales(sa));
        tc_cp_32x128b_x4(sfb_tmem, make_sdesc_scales(sb));
#pragma unroll
        for (uint32_t j = 0; j < XBK / 32; ++j)
          tc_mma_mx(tmem, make_sdesc_k_sw128(a + j * 32), make_sdesc_k_sw128(b + j * 32), make_idesc_mx(XBM, BN, j),
                    sfa_tmem | (j << 30), sfb_tmem | (j << 30), (kb > 0 || j > 0) ? 1u : 0u);
        tc_commit(&empty[s]);  // also covers the scale copies' reads of the stage
      }
      __syncwarp();
    }
    if (lane == 0) tc_commit(done);
    __syncwarp();
  } else {
    // ------------------------------------------------------- epilogue ----
    // TMEM lane r holds weight row n0 + r for the BN tokens
    ok = __all_sync(0xffffffffu, mbar_wait(done, 0, p.err, 453));
    tc_fence_after();
    const int quad = warp & 3;  // TMEM lane quadrant of this warp
    const int lrow = 32 * quad + lane;
    const uint32_t lane_base = tmem + (static_cast<uint32_t>(32 * quad) << 16);
    __nv_bfloat16* out = reinterpret_cast<__nv_bfloat16*>(p.out);
    float* up = reinterpret_cast<float*>(xchg);
    constexpr int CH = BN < 32 ? BN : 32;
    for (int c = 0; c < BN; c += CH) {
      uint32_t v[32];
      if (CH == 32) {
        tmem_ld_32x32b_x32(lane_base + c, *reinterpret_cast<uint32_t(*)[32]>(v));
      } else {
        tmem_ld_32x32b_x16(lane_base + c, *reinterpret_cast<uint32_t(*)[16]>(v));
      }
      tc_wait_ld();
      // every epilogue warp reaches both named barriers (ok or not); only
      // the stores depend on ok
      if (ok && !p.silu) {
#pragma unroll
        for (int j = 0; j < CH; ++j)
          out[static_cast<int64_t>(row0 + c + j) * p.ldo + n0 + lrow] = __float2bfloat16_rn(__uint_as_float(v[j]));
      } else if (ok && lrow >= 64) {
#pragma unroll
        for (int j = 0; j < CH; ++j) up[(c + j) * 64 + (lrow - 64)] = __uint_as_float(v[j]);  // lanes contiguous
      }
      if (p.silu) {
        asm volatile("bar.sync 1, 128;" ::: "memory");  // up rows of this column block are parked
        if (ok && lrow < 64) {
          const int f = n0 / 2 + lrow;  // feature of the SiLU output
#pragma unroll
          for (int j = 0; j < CH; ++j) {
            const float g = __uint_as_float(v[j]);
            const float u = up[(c + j) * 64 + lrow];
            out[static_cast<int64_t>(row0 + c + j) * p.ldo + f] = __float2bfloat16_rn(g / (1.f + __expf(-g)) * u);
          }
        }
        asm volatile("bar.sync 1, 128;" ::: "memory");
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, S::kCols);
  }
}

template <int BN, int STAGES>
void launch_x(const MoeMxGemmArgs& a, cudaStream_t s) {
  using S = XSmem<BN, STAGES>;
  static bool attr = false;
  if (!attr) {
    cudaFuncSetAttribute(moe_mx_gemm_kernel<BN, STAGES>, cudaFuncAttributeMaxDynamicSharedMemorySize, S::kBytes);
    attr = true;
  }
  // packed E2M1 [E * N, K]: 16 codes per 8 bytes in HBM, 16 bytes in shared memory
  uint64_t wd[2] = {static_cast<uint64_t>(a.K), static_cast<uint64_t>(a.E) * a.N};
  uint64_t ws[1] = {static_cast<uint64_t>(a.K / 2)};
  uint32_t wb[2] = {XBK, XBM};
  CUtensorMap tw = make_tmap(a.packed, CU_TENSOR_MAP_DATA_TYPE_16U4_ALIGN16B, 1, 2, wd, ws, wb,
                             CU_TENSOR_MAP_SWIZZLE_128B);
  uint64_t xd[2] = {static_cast<uint64_t>(a.K), static_cast<uint64_t>(a.P)};
  uint64_t xs[1] = {static_cast<uint64_t>(a.K)};
  uint32_t xb[2] = {XBK, BN};
  CUtensorMap tx = make_tmap(a.xq, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, 2, xd, xs, xb, CU_TENSOR_MAP_SWIZZLE_128B);
  XParams p;
  p.out = a.out;
  p.ldo = a.ldo;
  p.sfw = static_cast<const uint8_t*>(a.sfw);
  p.sfx = static_cast<const uint8_t*>(a.sfx);
  p.N = a.N;
  p.K = a.K;
  p.silu = a.silu ? 1 : 0;
  p.tile_expert = a.tile_expert;
  p.tile_row = a.tile_row;
  p.num_tiles = a.num_tiles;
  p.err = ErrorSink{a.err};
  dim3 grid(a.P / BN, a.N / XBM);
  launch_pdl(moe_mx_gemm_kernel<BN, STAGES>, grid, dim3(kXThreads), S::kBytes, s, tw, tx, p);
}

}  // namespace

void launch_mx8_quantize_rows(void* q, void* sf, const void* x, const int32_t* idx, int k, int rows, int K, int tile,
                              const int32_t* num_tiles, cudaStream_t s) {
  if (K % 128 != 0) throw std::runtime_error("minisgl.mx8_quantize: K must be a multiple of 128");
  if (tile != 16 && tile != 32 && tile != 64 && tile != 128)
    throw std::runtime_error("minisgl.mx8_quantize: tile of 16, 32, 64 or 128 rows");
  if (rows % tile != 0) throw std::runtime_error("minisgl.mx8_quantize: rows must be a multiple of the tile");
  const int64_t warps = static_cast<int64_t>(rows) * (K / 128);
  if (warps == 0) return;
  launch_pdl(mx8_quantize_rows_kernel, dim3(static_cast<unsigned>((warps + 7) / 8)), dim3(256), 0, s,
             static_cast<uint32_t*>(q), static_cast<uint8_t*>(sf), static_cast<const __nv_bfloat16*>(x), idx, k,
             rows, K, tile, num_tiles);
}

void launch_moe_mx_gemm(const MoeMxGemmArgs& a, cudaStream_t s) {
  if (a.N % 128 != 0 || a.K % 128 != 0) throw std::runtime_error("minisgl.moe_mx: N % 128 == 0 and K % 128 == 0");
  if (a.P % a.tile != 0) throw std::runtime_error("minisgl.moe_mx: rows must be a multiple of the tile");
  // the 16U4_ALIGN16B weight map wants a 32-byte aligned base and row pitch
  if ((reinterpret_cast<uintptr_t>(a.packed) & 31) != 0)
    throw std::runtime_error("minisgl.moe_mx: packed weights must be 32-byte aligned");
  if ((reinterpret_cast<uintptr_t>(a.sfw) & 15) != 0 || (reinterpret_cast<uintptr_t>(a.sfx) & 15) != 0)
    throw std::runtime_error("minisgl.moe_mx: scale blocks must be 16-byte aligned");
  switch (a.tile) {
    // stage counts chosen so two CTAs share an SM (about 100 KB each)
    case 16: launch_x<16, 5>(a, s); break;
    case 32: launch_x<32, 4>(a, s); break;
    case 64: launch_x<64, 4>(a, s); break;
    case 128: launch_x<128, 3>(a, s); break;
    default: throw std::runtime_error("minisgl.moe_mx: tile of 16, 32, 64 or 128");
  }
}

}  // namespace minisgl
