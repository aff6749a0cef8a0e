// MXFP4 (OCP microscaling, E2M1 elements with one E8M0 scale per 32) for
// the routed experts: the quantiser and a W4A16 grouped tcgen05 GEMM.
//
// Storage of a quantised weight w [E, N, K]:
//   packed [E, N, K / 2] uint8: element 2i in the low nibble of byte i
//   scales [E, K / 64, N, 2] uint8: E8M0 exponents (bias 127) of the two
//          32-element blocks of every 64-wide k-block, row-contiguous so one
//          k-block of 128 rows is 256 consecutive bytes (one bulk copy)
//
// Quantisation (OCP MX v1.0 rules): per block of 32, e = floor(log2 amax) - 2
// (2 is the largest E2M1 exponent), scale byte = e + 127, elements
// round-to-nearest-even onto {0, 0.5, 1, 1.5, 2, 3, 4, 6} x 2^e, saturating at
// 6. Blocks with amax below 2^-124 (or zero) get scale byte 0 and zero
// elements.
//
// The GEMM keeps activations in bf16 (weight-only quantisation; the reference
// has no MXFP4 path, its experts run the bf16 Triton fused_moe kernel of
// python/minisgl/kernel/triton/fused_moe.py:50-193). Per k-block
// the producer moves the packed weights (TMA, 128 rows x 32 bytes), their
// scales (one 256-byte bulk copy) and the bf16 token tile (TMA, 128-byte
// swizzle) into a deep ring of small stages; four converter warps expand
// each stage's weights into one of two bf16 tiles in the swizzled
// K-major operand layout with register byte permutes (no shared-memory table)
// and one exact power-of-two multiply, and the MMA thread runs kind::f16 tcgen05 MMAs
// on the expanded tile. Weight bytes per token tile are 4.25 bits per weight,
// the quantity a decode step streams from HBM.
#include <cstdlib>
#include <stdexcept>
#include <string>

#include "common.cuh"
#include "launch.h"
#include "ops.h"
#include "tma_host.h"

namespace minisgl {
namespace {

// ---------------------------------------------------------- quantiser ----
// E2M1 code of |x| in units of the block scale, round to nearest even.
__device__ __forceinline__ uint32_t e2m1_code(float a) {
  return (a > 0.25f) + (a >= 0.75f) + (a > 1.25f) + (a >= 1.75f) + (a > 2.5f) + (a >= 3.5f) + (a > 5.f);
}

// One thread per 32-element block: grid over E * N * (K / 32) blocks.
__global__ void __launch_bounds__(256) mxfp4_quantize_kernel(uint8_t* packed, uint8_t* scales,
                                                            const __nv_bfloat16* w, int E, int N, int K) {
  const int64_t nblk = static_cast<int64_t>(K) / 32;
  const int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (idx >= static_cast<int64_t>(E) * N * nblk) return;
  const int64_t row = idx / nblk;  // e * N + n
  const int j = static_cast<int>(idx - row * nblk);
  const __nv_bfloat16* src = w + row * K + j * 32;
  float v[32];
  float amax = 0.f;
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const uint4 u = *reinterpret_cast<const uint4*>(src + q * 8);
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      v[q * 8 + 2 * e] = __bfloat162float(h[e].x);
      v[q * 8 + 2 * e + 1] = __bfloat162float(h[e].y);
    }
  }
#pragma unroll
  for (int i = 0; i < 32; ++i) amax = fmaxf(amax, fabsf(v[i]));
  const int ebits = (__float_as_uint(amax) >> 23) & 0xFF;  // biased exponent: floor(log2 amax) + 127
  uint32_t sbyte = 0;
  float inv = 0.f;
  if (ebits >= 3) {
    sbyte = static_cast<uint32_t>(ebits - 2);               // (floor(log2 amax) - 2) + 127
    inv = __uint_as_float(static_cast<uint32_t>(254 - static_cast<int>(sbyte)) << 23);  // 2^-(e)
  }
  const int64_t e_idx = row / N, n = row - e_idx * N;
  scales[((e_idx * (K / 64) + j / 2) * N + n) * 2 + (j & 1)] = static_cast<uint8_t>(sbyte);
  uint32_t out[4];
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    uint32_t word = 0;
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const float x = v[q * 8 + e] * inv;
      const uint32_t code = e2m1_code(fabsf(x)) | (x < 0.f && e2m1_code(fabsf(x)) != 0 ? 8u : 0u);
      word |= code << (4 * e);
    }
    out[q] = word;
  }
  *reinterpret_cast<uint4*>(packed + row * (K / 2) + j * 16) = make_uint4(out[0], out[1], out[2], out[3]);
}


// ------------------------------------------------------- grouped GEMM ----
constexpr int QBM = 128;             // weight rows per tile (MMA M)
constexpr int QBK = 64;
constexpr int kQThreads = 192;
constexpr int kPackedBytes = QBM * QBK / 2;   // 4 KB of E2M1 per k-block
constexpr int kScaleBytes = QBM * 2;          // 256 B of E8M0 per k-block
constexpr int kWideBytes = QBM * QBK * 2;     // 16 KB of expanded bf16

template <int BN, int STAGES>
struct QSmem {
  // [expanded bf16 weights: 2 x 16 KB][STAGES x (token tile | packed | scales)][barriers]; the SiLU
  // exchange of the epilogue reuses the ring (every copy has been consumed by then)
  // The copy ring is deep and cheap (6-13 KB a stage); only the two
  // expanded tiles the converter and the MMA hand back and forth are wide.
  static constexpr int kAct = BN * QBK * 2;
  static constexpr int kStage = (kAct + kPackedBytes + kScaleBytes + 1023) / 1024 * 1024;  // swizzle alignment
  static constexpr int kStages = STAGES;
  static constexpr int kWide = 2 * kWideBytes;
  static constexpr int kXchg = 64 * BN * 4;   // SiLU epilogue: the up rows, fp32, column-major (aliases the ring)
  static constexpr int kRing = kStages * kStage > kXchg ? kStages * kStage : kXchg;
  static constexpr int kBytes = 1024 + kWide + kRing + 256;
};

struct QParams {
  void* out;                  // [P, ldo] bf16
  int ldo;
  const uint8_t* scales;      // [E, K / 64, N, 2]
  int N, K;                   // per expert: N rows of K
  int silu;                   // interleaved gate|up rows: write silu(gate) * up (N / 2 features)
  const int32_t* tile_expert;
  const int32_t* tile_row;
  const int32_t* num_tiles;
  ErrorSink err;
};

// PTX byte permute in its default mode: selector nibble i picks byte
// (nibble & 7) of {a, b} for result byte i; with bit 3 of the nibble set the
// result byte is that byte's top bit replicated (0x00 or 0xFF).
__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t d;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
  return d;
}

// Eight E2M1 codes (one 32-bit word, code j in bits 4j..4j+3) -> four
// bf16x2 words (unscaled), in registers. The bf16 patterns of the eight
// magnitudes {0, 0.5, 1, 1.5, 2, 3, 4, 6} are 0x0000, 0x3F00, 0x3F80,
// 0x3FC0, 0x4000, 0x4040, 0x4080, 0x40C0: their high and low bytes form two
// 8-byte tables that a permute indexes with four 3-bit magnitudes at a
// time. Signs: byte k of w << 4 has code 2k's sign bit on top and byte k of
// w has code 2k + 1's, so a sign-replicating permute of the two gives a
// 0xFF / 0x00 mask per code for the high bytes (a negative zero stays -0,
// harmless in an MMA). Two more permutes interleave low and high bytes into
// bf16 pairs: 14 integer operations for eight weights.
__device__ __forceinline__ void e2m1x8_to_bf16x8(uint32_t w, uint32_t (&o)[4]) {
  constexpr uint32_t kHiA = 0x3F3F3F00u, kHiB = 0x40404040u;  // high bytes of magnitudes 0..3, 4..7
  constexpr uint32_t kLoA = 0xC0800000u, kLoB = 0xC0804000u;  // low bytes
  const uint32_t m = w & 0x77777777u;
  const uint32_t w4 = w << 4;
  const uint32_t hi03 = prmt(kHiA, kHiB, m) | (prmt(w4, w, 0xD9C8u) & 0x80808080u);
  const uint32_t hi47 = prmt(kHiA, kHiB, m >> 16) | (prmt(w4, w, 0xFBEAu) & 0x80808080u);
  const uint32_t lo03 = prmt(kLoA, kLoB, m), lo47 = prmt(kLoA, kLoB, m >> 16);
  o[0] = prmt(lo03, hi03, 0x5140u);
  o[1] = prmt(lo03, hi03, 0x7362u);
  o[2] = prmt(lo47, hi47, 0x5140u);
  o[3] = prmt(lo47, hi47, 0x7362u);
}

template <int BN, int STAGES>
__global__ void __launch_bounds__(kQThreads, 1)
    moe_mxfp4_gemm_kernel(const __grid_constant__ CUtensorMap tm_w, const __grid_constant__ CUtensorMap tm_x,
                          const QParams p) {
  using S = QSmem<BN, STAGES>;
  constexpr int kStages = S::kStages;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint8_t* wide_buf = smem;                         // two expanded 128 x 64 bf16 weight tiles
  uint8_t* ring = smem + S::kWide;                   // stage s at ring + s * kStage: [act][packed][scales]
  uint8_t* xchg = ring;                              // epilogue only: after the last MMA completed
  uint64_t* full = reinterpret_cast<uint64_t*>(ring + S::kRing);  // [kStages] copies landed
  uint64_t* empty = full + kStages;                                 // [kStages] MMA done with the stage
  uint64_t* wfull = empty + kStages;                                // [2] expanded tile written
  uint64_t* wempty = wfull + 2;                                     // [2] MMA done with the expanded tile
  uint64_t* done = wempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  pdl_launch_dependents();
  pdl_wait();  // the tile tables and the token rows come from earlier kernels
  const int tile = blockIdx.x;
  if (tile >= *p.num_tiles) return;
  const int expert = p.tile_expert[tile];
  const int row0 = p.tile_row[tile];
  const int n0 = blockIdx.y * QBM;        // weight row block inside the expert
  const int nkb = p.K / QBK;
  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int w = 0; w < 2; ++w) {
      mbar_init(&wfull[w], 4);
      mbar_init(&wempty[w], 1);
    }
    mbar_init(done, 1);
    fence_barrier_init();
    prefetch_tmap(&tm_w);
    prefetch_tmap(&tm_x);
  }
  constexpr uint32_t kCols = BN < 32 ? 32 : BN;
  if (warp == 1) {
    tmem_alloc(tmem_slot, kCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  bool ok = true;

  if (warp == 0) {
    // ------------------------------------------------------------ TMA ----
    if (lane == 0) {
      const uint8_t* sc = p.scales + (static_cast<int64_t>(expert) * nkb * p.N + n0) * 2;
      for (int kb = 0; kb < nkb; ++kb) {
        const int s = kb % kStages;
        if (kb >= kStages && !mbar_wait(&empty[s], ((kb / kStages) - 1) & 1, p.err, 401)) break;
        uint8_t* st = ring + s * S::kStage;
        mbar_arrive_expect_tx(&full[s], S::kAct + kPackedBytes + kScaleBytes);
        tma_load_2d(st, &tm_x, &full[s], kb * QBK, row0);
        tma_load_2d(st + S::kAct, &tm_w, &full[s], kb * (QBK / 2), expert * p.N + n0);
        bulk_load(st + S::kAct + kPackedBytes, sc + static_cast<int64_t>(kb) * p.N * 2, kScaleBytes, &full[s]);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA ----
    constexpr uint32_t idesc = make_idesc_bf16(QBM, BN);
    for (int kb = 0; kb < nkb && ok; ++kb) {
      const int s = kb % kStages, w = kb & 1;
      ok = __all_sync(0xffffffffu, mbar_wait(&wfull[w], (kb >> 1) & 1, p.err, 402) &&
                                       mbar_wait(&full[s], (kb / kStages) & 1, p.err, 405));
      if (!ok) break;
      tc_fence_after();
      if (lane == 0) {
        const uint32_t a = smem_u32(wide_buf + w * kWideBytes);
        const uint32_t b = smem_u32(ring + s * S::kStage);
#pragma unroll
        for (int k = 0; k < QBK / 16; ++k)
          tc_mma_f16(tmem, make_sdesc_k_sw128(a + k * 32), make_sdesc_k_sw128(b + k * 32), idesc,
                     (kb > 0 || k > 0) ? 1u : 0u);
        tc_commit(&empty[s]);
        tc_commit(&wempty[w]);
      }
      __syncwarp();
    }
    if (lane == 0) tc_commit(done);
    __syncwarp();
  } else {
    // --------------------------------------------------- expand + store ----
    const int r = threadIdx.x - 64;  // weight row of this thread (0..127)
    for (int kb = 0; kb < nkb && ok; ++kb) {
      const int s = kb % kStages, w = kb & 1;
      ok = __all_sync(0xffffffffu, mbar_wait(&full[s], (kb / kStages) & 1, p.err, 403) &&
                                       (kb < 2 || mbar_wait(&wempty[w], ((kb >> 1) - 1) & 1, p.err, 406)));
      if (!ok) break;
      uint8_t* st = ring + s * S::kStage;
      uint8_t* dst = wide_buf + w * kWideBytes;
      const uint4* src = reinterpret_cast<const uint4*>(st + S::kAct + r * 32);
      const uint8_t* scl = st + S::kAct + kPackedBytes + r * 2;
      // 2^(byte - 127) as a bf16x2 multiplier (exact: a power of two)
      uint32_t mul[2];
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const uint32_t eb = scl[h];
        const uint32_t bits = eb == 0 ? 0u : (eb << 7);  // bf16 exponent field = scale byte
        mul[h] = bits | (bits << 16);
      }
      const uint4 q0 = src[0], q1 = src[1];
      const uint32_t words[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
#pragma unroll
      for (int c = 0; c < 8; ++c) {  // 16-byte chunk c = elements 8c..8c+7 = bytes 4c..4c+3
        uint32_t o[4];
        e2m1x8_to_bf16x8(words[c], o);
#pragma unroll
        for (int b = 0; b < 4; ++b) {
          const __nv_bfloat162 v = __hmul2(*reinterpret_cast<const __nv_bfloat162*>(&o[b]),
                                           *reinterpret_cast<const __nv_bfloat162*>(&mul[c >> 2]));
          o[b] = *reinterpret_cast<const uint32_t*>(&v);
        }
        *reinterpret_cast<uint4*>(dst + r * 128 + ((c ^ (r & 7)) << 4)) = make_uint4(o[0], o[1], o[2], o[3]);
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(&wfull[w]);
    }
    // epilogue: TMEM lane r holds weight row n0 + r for the BN tokens
    ok = __all_sync(0xffffffffu, ok && mbar_wait(done, 0, p.err, 404));
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
    tmem_dealloc(tmem, kCols);
  }
}

template <int BN, int STAGES>
void launch_q(const MoeMxfp4GemmArgs& a, cudaStream_t s) {
  using S = QSmem<BN, STAGES>;
  static bool attr = false;
  if (!attr) {
    cudaFuncSetAttribute(moe_mxfp4_gemm_kernel<BN, STAGES>, cudaFuncAttributeMaxDynamicSharedMemorySize, S::kBytes);
    attr = true;
  }
  uint64_t wd[2] = {static_cast<uint64_t>(a.K / 2), static_cast<uint64_t>(a.E) * a.N};
  uint64_t ws[1] = {static_cast<uint64_t>(a.K / 2)};
  uint32_t wb[2] = {QBK / 2, QBM};
  CUtensorMap tw = make_tmap(a.packed, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, 2, wd, ws, wb, CU_TENSOR_MAP_SWIZZLE_NONE);
  CUtensorMap tx = make_tmap_bf16_2d_sw128(a.x, a.P, a.K, a.K, BN);
  QParams p;
  p.out = a.out;
  p.ldo = a.ldo;
  p.scales = static_cast<const uint8_t*>(a.scales);
  p.N = a.N;
  p.K = a.K;
  p.silu = a.silu ? 1 : 0;
  p.tile_expert = a.tile_expert;
  p.tile_row = a.tile_row;
  p.num_tiles = a.num_tiles;
  p.err = ErrorSink{a.err};
  dim3 grid(a.P / BN, a.N / QBM);
  launch_pdl(moe_mxfp4_gemm_kernel<BN, STAGES>, grid, dim3(kQThreads), S::kBytes, s, tw, tx, p);
}

}  // namespace

void launch_mxfp4_quantize(void* packed, void* scales, const void* w, int E, int N, int K, cudaStream_t s) {
  if (K % 64 != 0) throw std::runtime_error("minisgl.mxfp4_quantize: K must be a multiple of 64");
  const int64_t blocks = static_cast<int64_t>(E) * N * (K / 32);
  if (blocks == 0) return;
  const int64_t grid = (blocks + 255) / 256;
  launch_pdl(mxfp4_quantize_kernel, dim3(static_cast<unsigned>(grid)), dim3(256), 0, s,
             static_cast<uint8_t*>(packed), static_cast<uint8_t*>(scales), static_cast<const __nv_bfloat16*>(w), E,
             N, K);
}

}  // namespace minisgl

namespace minisgl {
void launch_moe_mxfp4_gemm(const MoeMxfp4GemmArgs& a, cudaStream_t s) {
  if (a.N % 128 != 0 || a.K % 64 != 0) throw std::runtime_error("minisgl.moe_mxfp4: N % 128 == 0 and K % 64 == 0");
  if (a.P % a.tile != 0) throw std::runtime_error("minisgl.moe_mxfp4: rows must be a multiple of the tile");
  switch (a.tile) {
    // copy-ring depths chosen so two CTAs share an SM (91-100 KB each)
    case 16: launch_q<16, 8>(a, s); break;
    case 32: launch_q<32, 6>(a, s); break;
    case 64: launch_q<64, 5>(a, s); break;
    case 128: launch_q<128, 3>(a, s); break;
    default: throw std::runtime_error("minisgl.moe_mxfp4: tile of 16, 32, 64 or 128");
  }
}
}  // namespace minisgl
