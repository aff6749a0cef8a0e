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
//   token-major   (A = x, B = w): rows of the tile are tokens (prefill).
//   weight-major  (A = w, B = x): rows are output features and the token
//                 count becomes the MMA N dimension (16..128). Used for small
//                 M (decode) so the 128-row MMA is filled by weights.
//
// Decode GEMMs are latency bound, so two launch-level features matter:
//   * programmatic dependent launch: the kernel lets its successor start
//     early, and its own producer streams the first weight stages before
//     griddepcontrol.wait (weights never depend on the previous kernel);
//   * split-K inside a thread-block cluster: the S CTAs that share an output
//     tile (cluster dims 1x1xS) each reduce a K range, park their fp32 tile
//     in shared memory and sum the S tiles through distributed shared memory
//     (mapa + ld.shared::cluster). No global workspace, no second kernel.
#include <algorithm>
#include <stdexcept>
#include <string>
#include <vector>

#include "common.cuh"
#include "launch.h"
#include "ops.h"
#include "sampling_rng.cuh"
#include "tma_host.h"

namespace minisgl {
namespace {

constexpr int BM = 128;
constexpr int BK = 64;
constexpr int kThreads = 192;

struct KParams {
  void* out;
  const __nv_bfloat16* bias;
  int M, N;            // logical output is out[M, N] (M = tokens, N = features)
  int ldo;
  int kb_per_split;
  int num_kb;
  int stages;          // ring depth used by this launch (<= the template maximum)
  int kps;             // k-blocks per stage: >1 loads them with one 3-D TMA box per operand
  int K;               // reduction length (the RMSNorm mean of kEpiNorm)
  // grouped weight-major GEMM (MoE experts): w holds the experts' [N, K]
  // matrices back to back; token tile i is rows [g_tile_row[i], + BN) of x
  const int32_t* g_tile_expert;
  const int32_t* g_tile_row;
  const int32_t* g_num_tiles;  // nullptr: plain GEMM
  int out_f32;
  GemmEpilogue epi;    // fused epilogue (weight-major split-K instantiations only)
  ErrorSink err;
  // optional per-CTA phase timestamps (%globaltimer ns), 8 slots per CTA:
  // 0 entry, 1 setup done, 2 producer past griddepcontrol.wait, 3 first
  // stage consumed by the MMA thread, 4 accumulator ready, 5 exit
  unsigned long long* trace;
};

__device__ __forceinline__ void trace_stamp(const KParams& p, int slot) {
  if (p.trace != nullptr) {
    const size_t cta = (static_cast<size_t>(blockIdx.z) * gridDim.y + blockIdx.y) * gridDim.x + blockIdx.x;
    p.trace[cta * 8 + slot] = globaltimer_ns();
  }
}

template <int BN, int STAGES>
struct Smem {
  static constexpr uint32_t kA = BM * BK * 2;
  static constexpr uint32_t kB = BN * BK * 2;
  static constexpr uint32_t kPipe = STAGES * (kA + kB);
  // split-K reduction tile, output-major: tokens x features fp32, each row
  // padded by 4 floats (weight-major tiles: BN tokens x 128 features)
  static constexpr uint32_t kRedLdSwap = BM + 4;
  static constexpr uint32_t kRedLdTok = BN + 4;
  static constexpr uint32_t kRed = (BN * kRedLdSwap > BM * kRedLdTok ? BN * kRedLdSwap : BM * kRedLdTok) * 4;
  static constexpr uint32_t kMain = kPipe > kRed ? kPipe : kRed;
  static constexpr uint32_t kBytes = kMain + 1024 /*align*/ + 256 /*barriers*/ + 2 * (BN > BM ? BN : BM) * 4;
  // bytes of a launch whose ring holds `stages` k-blocks: a CTA with fewer
  // k-blocks than the template depth asks for less shared memory, so more
  // CTAs (of this and of neighbouring kernels) stay resident together
  __host__ __device__ static constexpr uint32_t main_bytes(int stages, bool split, int kps = 1) {
    const uint32_t pipe = static_cast<uint32_t>(stages * kps) * (kA + kB);
    return split && kRed > pipe ? kRed : pipe;
  }
  // + per-token sum of squares and rstd arrays (kEpiNorm) after the barriers
  static constexpr int kRows = BN > BM ? BN : BM;
  static constexpr uint32_t bytes(int stages, bool split, int kps = 1) {
    return main_bytes(stages, split, kps) + 1024 + 256 + 2 * kRows * 4;
  }
};

template <int N>
struct TmemCols {
  static constexpr uint32_t value = N <= 32 ? 32 : (N <= 64 ? 64 : (N <= 128 ? 128 : 256));
};

__device__ __forceinline__ void store_out(const KParams& p, int m, int n, float v) {
  if (p.out_f32) {
    reinterpret_cast<float*>(p.out)[static_cast<size_t>(m) * p.ldo + n] = v;
  } else {
    reinterpret_cast<__nv_bfloat16*>(p.out)[static_cast<size_t>(m) * p.ldo + n] = __float2bfloat16_rn(v);
  }
}

__device__ __forceinline__ float round_bf16(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

__device__ __forceinline__ void store4_bf16(__nv_bfloat16* dst, const float (&v)[4]) {
  uint2 pk;
  pk.x = pack_bf16x2(v[0], v[1]);
  pk.y = pack_bf16x2(v[2], v[3]);
  *reinterpret_cast<uint2*>(dst) = pk;
}

// Sum of the float4 at byte offset `addr` of every cluster CTA's parked tile
// (one split: this CTA's own tile, read with a plain shared load).
__device__ __forceinline__ float4 reduce_parts(uint32_t addr, int nsplit) {
  if (nsplit == 1) {
    float4 v;
    asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];"
                 : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
                 : "r"(addr)
                 : "memory");
    return v;
  }
  constexpr int kMaxS = 16;
  float4 part[kMaxS];
#pragma unroll
  for (int q = 0; q < kMaxS; ++q)
    if (q < nsplit) part[q] = ld_shared_cluster_v4(map_shared_rank(addr, static_cast<uint32_t>(q)));
  float4 acc = part[0];
#pragma unroll
  for (int q = 1; q < kMaxS; ++q)
    if (q < nsplit) acc.x += part[q].x, acc.y += part[q].y, acc.z += part[q].z, acc.w += part[q].w;
  return acc;
}

// kEpiRope for one token row of one 128-feature head; the calling warp holds
// the whole row (lane l: features 4l..4l+3). Same steps and roundings as
// the unfused rope_store kernel: bf16 GEMM output, per-head RMSNorm rounded
// to bf16, NeoX rotation (feature j pairs with j + 64, held by lane l ^ 16).
__device__ __forceinline__ void rope_epilogue(const KParams& p, int head, int m, int ocol, float (&v)[4]) {
  const GemmEpilogue& e = p.epi;
  const int lane = threadIdx.x & 31;
  const bool is_q = head < e.hq;
  const bool is_k = !is_q && head < e.hq + e.hk;
#pragma unroll
  for (int q = 0; q < 4; ++q) v[q] = round_bf16(v[q]);
  if (is_q || is_k) {
    const __nv_bfloat16* nw = static_cast<const __nv_bfloat16*>(is_q ? e.q_norm_w : e.k_norm_w);
    if (nw != nullptr) {
      float ss = v[0] * v[0] + v[1] * v[1] + v[2] * v[2] + v[3] * v[3];
      ss = warp_sum(ss);
      const float inv = rsqrtf(ss / 128.f + e.head_eps);
#pragma unroll
      for (int q = 0; q < 4; ++q) v[q] = round_bf16(v[q] * inv * __bfloat162float(nw[ocol + q]));
    }
    const float* cs = e.cos_sin + static_cast<int64_t>(e.positions[m]) * 128;
    const bool first = lane < 16;
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const float other = __shfl_xor_sync(0xffffffffu, v[q], 16);
      const int j = (ocol + q) & 63;
      const float c = cs[j], sn = cs[64 + j];
      v[q] = first ? (v[q] * c - other * sn) : (v[q] * c + other * sn);
    }
  }
  if (is_q) {
    store4_bf16(reinterpret_cast<__nv_bfloat16*>(p.out) + static_cast<size_t>(m) * p.ldo + head * 128 + ocol, v);
    return;
  }
  const int kvh = is_k ? head - e.hq : head - e.hq - e.hk;
  const int slot = e.out_loc[m];
  if (e.kv_slots > 0 && (slot < 0 || slot >= e.kv_slots)) {  // uniform over the warp
    if (lane == 0) p.err.report(kErrBadIndex, 941);
    return;
  }
  const int page = slot / e.page_size, off = slot % e.page_size;
  __nv_bfloat16* cache = static_cast<__nv_bfloat16*>(is_k ? e.k_cache : e.v_cache);
  store4_bf16(cache + ((static_cast<int64_t>(page) * e.hk + kvh) * e.page_size + off) * 128 + ocol, v);
}

// kEpiAllReduce heap addressing: [signal 4 KB][flags 16 KB][collective data
// C][half 0 C][half 1 C], C = ar_half_bytes.
__device__ __forceinline__ __nv_bfloat16* ar_half(const KParams& p, int r, uint32_t e) {
  uint8_t* base = reinterpret_cast<uint8_t*>(p.epi.ar_bases[r]);
  return reinterpret_cast<__nv_bfloat16*>(base + kSymmSignalBytes + kSymmFlagBytes +
                                          (1 + (e & 1u)) * p.epi.ar_half_bytes);
}
__device__ __forceinline__ uint32_t* ar_flag(const KParams& p, int r, int cta) {
  return reinterpret_cast<uint32_t*>(reinterpret_cast<uint8_t*>(p.epi.ar_bases[r]) + kSymmSignalBytes) + cta;
}
__device__ __forceinline__ void ar_store_release(uint32_t* f, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(f), "r"(v) : "memory");
}
// bounded wait until a peer's flag reaches e (kErrPeerTimeout after 2 s)
__device__ __forceinline__ void ar_wait(const KParams& p, const uint32_t* f, uint32_t e) {
  const uint64_t t0 = globaltimer_ns();
  uint32_t it = 0;
  while (true) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(f) : "memory");
    if (static_cast<int32_t>(v - e) >= 0) return;
    if (((++it) & 0xFFu) == 0 && globaltimer_ns() - t0 > kWaitBudgetNs) {
      p.err.report(kErrPeerTimeout, 320);
      return;
    }
  }
}

// kEpiSample for one token row m of one 128-row vocabulary tile; the calling
// warp holds the row (lane l: vocabulary entries n .. n + 3, n = tile base +
// 4 l). Score and tie rule are the sampling kernel's: score = logit / max(T,
// 1e-6) + Gumbel(row_key(seed, step, m), index) when T > 0, else the logit;
// the larger score wins, ties go to the smaller index.
__device__ __forceinline__ void sample_epilogue(const KParams& p, int m, int n, float4 acc) {
  const GemmEpilogue& e = p.epi;
  const float T = e.temps != nullptr ? e.temps[m] : 0.f;
  const bool hot = T > 0.f;
  const float inv = 1.f / fmaxf(T, 1e-6f);
  const uint32_t key = hot ? row_key(e.seed, static_cast<uint64_t>(*e.step), m) : 0u;
  const float v[4] = {acc.x, acc.y, acc.z, acc.w};
  float bv = -INFINITY;
  int bi = 0x7fffffff;
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const int idx = n + q;
    if (idx >= p.N) break;
    float l = v[q];
    if (p.bias != nullptr) l += __bfloat162float(p.bias[idx]);
    const float sc = hot ? l * inv + gumbel(key, idx) : l;
    if (sc > bv || (sc == bv && idx < bi)) bv = sc, bi = idx;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (ov > bv || (ov == bv && oi < bi)) bv = ov, bi = oi;
  }
  if ((threadIdx.x & 31) == 0) {
    const int64_t o = static_cast<int64_t>(m) * e.ntiles + n / 128;
    e.part_val[o] = bv;
    e.part_idx[o] = bi;
  }
}

// Fused epilogue of a token-major tile without split-K, straight from TMEM:
// this thread owns token row m (its TMEM lane) and the tile's BN features
// [feat0, feat0 + BN). tcgen05.ld is warp-collective, so every lane loads
// and only `valid` lanes (row inside M, pipeline healthy) read or write
// global memory. Same arithmetic and roundings as the split-K path.
template <int BN>
__device__ __forceinline__ void rows_epilogue(const KParams& p, uint32_t taddr, int m, int feat0, float rstd,
                                              bool valid) {
  const GemmEpilogue& e = p.epi;
  const __nv_bfloat16* bias = p.bias;
  auto col = [&](const uint32_t (&r)[32], int j, int n) {
    float x = __uint_as_float(r[j]) * rstd;
    if (bias != nullptr) x += __bfloat162float(bias[n]);
    return x;
  };
  if ((e.kind & kEpiSiluMul) != 0) {
#pragma unroll 1
    for (int blk = 0; blk < BN / 128; ++blk) {
#pragma unroll 1
      for (int c = 0; c < 64; c += 32) {
        uint32_t g[32], u[32];
        tmem_ld_32x32b_x32(taddr + blk * 128 + c, g);
        tmem_ld_32x32b_x32(taddr + blk * 128 + 64 + c, u);
        tc_wait_ld();
        if (!valid) continue;
        const int n = feat0 + blk * 128 + c;
        float v[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          const float gq = round_bf16(col(g, j, n + j)), uq = round_bf16(col(u, j, n + 64 + j));
          v[j] = gq / (1.f + __expf(-gq)) * uq;
        }
        __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(p.out) + static_cast<size_t>(m) * p.ldo + feat0 / 2 +
                             blk * 64 + c;
#pragma unroll
        for (int j = 0; j < 32; j += 4) store4_bf16(dst + j, {v[j], v[j + 1], v[j + 2], v[j + 3]});
      }
    }
    return;
  }
  if ((e.kind & kEpiRope) != 0) {
    const float* cs = e.cos_sin + static_cast<int64_t>(valid ? e.positions[m] : 0) * 128;
#pragma unroll 1
    for (int hb = 0; hb < BN / 128; ++hb) {
      const int head = (feat0 + hb * 128) / 128;
      const bool is_q = head < e.hq, is_k = !is_q && head < e.hq + e.hk;
      const __nv_bfloat16* nw =
          static_cast<const __nv_bfloat16*>(is_q ? e.q_norm_w : (is_k ? e.k_norm_w : nullptr));
      const uint32_t ta = taddr + hb * 128;
      const int n0 = head * 128;
      // pass 1: per-head RMS of the bf16-rounded projection
      float inv = 1.f;
      if (nw != nullptr) {
        float ss = 0.f;
#pragma unroll 1
        for (int c = 0; c < 128; c += 32) {
          uint32_t r[32];
          tmem_ld_32x32b_x32(ta + c, r);
          tc_wait_ld();
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            const float x = round_bf16(col(r, j, n0 + c + j));
            ss += x * x;
          }
        }
        inv = rsqrtf(ss / 128.f + e.head_eps);
      }
      // pass 2: feature j (< 64) and its NeoX partner j + 64 together
      __nv_bfloat16* dst;
      if (is_q) {
        dst = reinterpret_cast<__nv_bfloat16*>(p.out) + static_cast<size_t>(m) * p.ldo + n0;
      } else {
        const int kvh = is_k ? head - e.hq : head - e.hq - e.hk;
        const int slot = valid ? e.out_loc[m] : 0;
        const int page = slot / e.page_size, off = slot % e.page_size;
        dst = static_cast<__nv_bfloat16*>(is_k ? e.k_cache : e.v_cache) +
              ((static_cast<int64_t>(page) * e.hk + kvh) * e.page_size + off) * 128;
      }
#pragma unroll 1
      for (int c = 0; c < 64; c += 32) {
        uint32_t lo[32], hi[32];
        tmem_ld_32x32b_x32(ta + c, lo);
        tmem_ld_32x32b_x32(ta + 64 + c, hi);
        tc_wait_ld();
        if (!valid) continue;
        float a[32], b[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          float xl = round_bf16(col(lo, j, n0 + c + j)), xh = round_bf16(col(hi, j, n0 + 64 + c + j));
          if (nw != nullptr) {
            xl = round_bf16(xl * inv * __bfloat162float(nw[c + j]));
            xh = round_bf16(xh * inv * __bfloat162float(nw[64 + c + j]));
          }
          if (is_q || is_k) {
            const float cj = cs[c + j], sj = cs[64 + c + j];
            a[j] = xl * cj - xh * sj;
            b[j] = xh * cj + xl * sj;
          } else {
            a[j] = xl, b[j] = xh;
          }
        }
#pragma unroll
        for (int j = 0; j < 32; j += 4) {
          store4_bf16(dst + c + j, {a[j], a[j + 1], a[j + 2], a[j + 3]});
          store4_bf16(dst + 64 + c + j, {b[j], b[j + 1], b[j + 2], b[j + 3]});
        }
      }
    }
    return;
  }
#pragma unroll 1
  for (int c = 0; c < BN; c += 32) {
    uint32_t r[32];
    tmem_ld_32x32b_x32(taddr + c, r);
    tc_wait_ld();
    if (!valid) continue;
    const int n = feat0 + c;
    float v[32];
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] = col(r, j, n + j);
    if ((e.kind & kEpiResidual) != 0) {
      const __nv_bfloat16* res = static_cast<const __nv_bfloat16*>(e.residual) + static_cast<size_t>(m) * e.ld_res + n;
#pragma unroll
      for (int j = 0; j < 32; j += 8) {
        const uint4 raw = *reinterpret_cast<const uint4*>(res + j);
        const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&raw);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const float2 f = __bfloat1622float2(h[q]);
          v[j + 2 * q] = round_bf16(v[j + 2 * q]) + f.x;
          v[j + 2 * q + 1] = round_bf16(v[j + 2 * q + 1]) + f.y;
        }
      }
    }
    __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(p.out) + static_cast<size_t>(m) * p.ldo + n;
#pragma unroll
    for (int j = 0; j < 32; j += 4) store4_bf16(dst + j, {v[j], v[j + 1], v[j + 2], v[j + 3]});
  }
}

// SWAP = weight-major tiles; SPLIT = cluster split-K (gridDim.z CTAs per tile).
template <int BN, int STAGES, bool SWAP, bool SPLIT>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                   KParams p) {
  using S = Smem<BN, STAGES>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  const int stages = p.stages;
  const int kps = p.kps;
  const uint32_t stA = kps * S::kA, stB = kps * S::kB;  // bytes of one stage per operand
  uint8_t* sA = smem;
  uint8_t* sB = smem + stages * stA;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + S::main_bytes(stages, SPLIT, kps));
  uint64_t* empty = full + stages;
  uint64_t* done = empty + stages;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
  float* s_ss = reinterpret_cast<float*>(smem + S::main_bytes(stages, SPLIT, kps) + 256);  // [token rows]
  float* s_rstd = s_ss + S::kRows;                                                     // [token rows]
  // kEpiNorm: the epilogue warps read every x tile of the ring too, so a
  // stage is free once the MMA commit and those four warps have released it
  const bool do_norm = (SPLIT || !SWAP) && (p.epi.kind & kEpiNorm) != 0;

  constexpr uint32_t kCols = TmemCols<BN>::value;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int a_row0 = blockIdx.y * BM;
  int b_row0 = blockIdx.x * BN;
  const int kb0 = blockIdx.z * p.kb_per_split;
  const int kb1 = min(p.num_kb, kb0 + p.kb_per_split);
  const int nkb = max(0, kb1 - kb0);
  // grouped (MoE) weight-major GEMM: token tile i of the expert-sorted rows
  // belongs to expert g_tile_expert[i]; the table comes from the previous
  // kernel, and tiles past the live count leave before any set-up
  int w_off = 0;
  if (SWAP && p.g_num_tiles != nullptr) {
    pdl_launch_dependents();
    pdl_wait();
    if (static_cast<int>(blockIdx.x) >= *p.g_num_tiles) return;
    b_row0 = p.g_tile_row[blockIdx.x];
    w_off = p.g_tile_expert[blockIdx.x] * p.N;
  }

  pdl_launch_dependents();
  if (threadIdx.x == 0) trace_stamp(p, 0);
  if (threadIdx.x == 0) {
    for (int s = 0; s < stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], do_norm ? 5 : 1);
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
  if (threadIdx.x == 0) trace_stamp(p, 1);

  // The producer and MMA warps stay converged: every lane walks the loop and
  // waits, lane 0 alone issues TMA / tcgen05 work (the cluster barrier of the
  // split-K epilogue is .aligned and needs converged warps).
  if (warp == 0) {
    // weights first: they do not depend on the previous kernel
    const CUtensorMap* tw = SWAP ? &tmA : &tmB;
    const CUtensorMap* tx = SWAP ? &tmB : &tmA;
    const int w_row = (SWAP ? a_row0 : b_row0) + w_off;
    const int x_row = SWAP ? b_row0 : a_row0;
    uint8_t* sW = SWAP ? sA : sB;
    uint8_t* sX = SWAP ? sB : sA;
    const uint32_t sw = SWAP ? stA : stB;
    const uint32_t sx = SWAP ? stB : stA;
    const uint32_t stage_bytes = stA + stB;
    const int nst = (nkb + kps - 1) / kps;  // stages of this CTA's K range
    // stage i holds k-blocks [kb0 + i * kps, + kps): one 2-D box per operand,
    // or one 3-D box of kps k-blocks
    auto load = [&](const CUtensorMap* tm, uint8_t* dst, int i, int row, uint64_t* bar) {
      if (kps == 1) tma_load_2d(dst, tm, bar, (kb0 + i) * BK, row);
      else tma_load_3d(dst, tm, bar, 0, row, kb0 + i * kps);
    };
    const int pre = min(nst, stages);
    if (lane == 0) {
      for (int i = 0; i < pre; ++i) {
        mbar_arrive_expect_tx(&full[i], stage_bytes);
        load(tw, sW + i * sw, i, w_row, &full[i]);
      }
    }
    pdl_wait();
    if (lane == 0) {
      trace_stamp(p, 2);
      for (int i = 0; i < pre; ++i) load(tx, sX + i * sx, i, x_row, &full[i]);
    }
    __syncwarp();
    for (int i = pre; i < nst; ++i) {
      const int s = i % stages;
      const uint32_t ph = (i / stages) & 1u;
      const bool ok = __all_sync(0xffffffffu, mbar_wait(&empty[s], ph ^ 1u, p.err, 101));
      if (!ok) break;
      if (lane == 0) {
        mbar_arrive_expect_tx(&full[s], stage_bytes);
        load(tw, sW + s * sw, i, w_row, &full[s]);
        load(tx, sX + s * sx, i, x_row, &full[s]);
      }
      __syncwarp();
    }
  } else if (warp == 1) {
    constexpr uint32_t idesc = make_idesc_bf16(BM, BN);
    const int nst = (nkb + kps - 1) / kps;
    for (int i = 0; i < nst; ++i) {
      const int s = i % stages;
      const uint32_t ph = (i / stages) & 1u;
      const bool ok = __all_sync(0xffffffffu, mbar_wait(&full[s], ph, p.err, 102));
      if (!ok) break;
      tc_fence_after();
      if (lane == 0) {
        if (i == 0) trace_stamp(p, 3);
        const int nj = min(kps, nkb - i * kps);
        for (int j = 0; j < nj; ++j) {
          const uint32_t a_addr = smem_u32(sA + s * stA + j * S::kA);
          const uint32_t b_addr = smem_u32(sB + s * stB + j * S::kB);
#pragma unroll
          for (int k = 0; k < BK / 16; ++k) {
            tc_mma_f16(tmem, make_sdesc_k_sw128(a_addr + k * 32), make_sdesc_k_sw128(b_addr + k * 32),
                       idesc, (i > 0 || j > 0 || k > 0) ? 1u : 0u);
          }
        }
        tc_commit(&empty[s]);
      }
      __syncwarp();
    }
    if (lane == 0) tc_commit(done);
    __syncwarp();
  }

  // --------------------------------------- kEpiNorm: per-token sum of x^2 ----
  if (do_norm && warp >= 2) {
    // x tile of a stage: token rows of 128 bytes (64 bf16 of K), BN of them
    // in weight-major tiles (operand B), BM in token-major ones (operand A);
    // the 128-byte swizzle only permutes 16-byte chunks inside a row, so a
    // row's sum is the sum over its 128-byte line. Thread et takes chunks
    // et, et + 128, ...; the 8 lanes of a row combine by shuffles at the end.
    constexpr int kChunks = (SWAP ? BN : BM) * 8;
    constexpr int kPer = (kChunks + 127) / 128;
    const int et = threadIdx.x - 64;
    float acc[kPer];
#pragma unroll
    for (int j = 0; j < kPer; ++j) acc[j] = 0.f;
    const int nst = (nkb + kps - 1) / kps;
    for (int i = 0; i < nst; ++i) {
      const int s = i % stages;
      const uint32_t ph = (i / stages) & 1u;
      if (!__all_sync(0xffffffffu, mbar_wait(&full[s], ph, p.err, 104))) break;
      const int nj = min(kps, nkb - i * kps);
      for (int kb = 0; kb < nj; ++kb) {
        const uint8_t* xs = SWAP ? sB + s * stB + kb * S::kB : sA + s * stA + kb * S::kA;
#pragma unroll
        for (int j = 0; j < kPer; ++j) {
          const int idx = et + j * 128;
          if (idx < kChunks) {
            const uint4 raw = *reinterpret_cast<const uint4*>(xs + idx * 16);
            const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&raw);
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              const float2 f = __bfloat1622float2(h[q]);
              acc[j] += f.x * f.x + f.y * f.y;
            }
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);
    }
#pragma unroll
    for (int j = 0; j < kPer; ++j) {
      float v = acc[j];
      v += __shfl_xor_sync(0xffffffffu, v, 1);
      v += __shfl_xor_sync(0xffffffffu, v, 2);
      v += __shfl_xor_sync(0xffffffffu, v, 4);
      const int idx = et + j * 128;
      if ((lane & 7) == 0 && idx < kChunks) s_ss[idx >> 3] = v;
    }
    // the parked split-K tile below overlaps the ring: no epilogue warp may
    // write it while another still reads x tiles
    asm volatile("bar.sync 2, 128;" ::: "memory");
  }

  // ------------------------------------------------------------ epilogue ----
  constexpr int CH = BN < 32 ? BN : 32;
  if (warp >= 2) {
    const bool ok = mbar_wait(done, 0, p.err, 103);
    if (threadIdx.x == 64) trace_stamp(p, 4);
    tc_fence_after();
    const int sub = warp & 3;
    const int row = sub * 32 + lane;  // TMEM lane == tile row
    const uint32_t taddr = tmem + (static_cast<uint32_t>(sub * 32) << 16);
    bool fused_done = false;
    if constexpr (!SWAP && !SPLIT && BN >= 32) {
      if (p.epi.kind != 0) {
        const int m = a_row0 + row;
        const bool valid = ok && m < p.M;
        const float rstd = do_norm ? rsqrtf(s_ss[row] / static_cast<float>(p.K) + p.epi.eps) : 1.f;
        rows_epilogue<BN>(p, taddr, m, b_row0, rstd, valid);
        fused_done = true;
      }
    }
    float* red = reinterpret_cast<float*>(smem);  // split-K parking tile (output-major)
#pragma unroll 1
    for (int c = 0; c < BN && !fused_done; c += CH) {
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
      if constexpr (SPLIT) {
        // park the partial tile output-major (zeros if the pipeline failed)
        const bool have = ok && nkb > 0;
        if constexpr (SWAP) {
#pragma unroll
          for (int j = 0; j < CH; ++j)
            red[(c + j) * S::kRedLdSwap + row] = have ? __uint_as_float(r[j]) : 0.f;
        } else {
#pragma unroll
          for (int j = 0; j < CH; j += 4) {
            float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
            if (have)
              v = make_float4(__uint_as_float(r[j]), __uint_as_float(r[j + 1]), __uint_as_float(r[j + 2]),
                              __uint_as_float(r[j + 3]));
            *reinterpret_cast<float4*>(red + row * S::kRedLdTok + c + j) = v;
          }
        }
        continue;
      }
      if (!ok) continue;
      if constexpr (!SWAP) {
        const int m = a_row0 + row;
        if (m >= p.M) continue;
        const int n0 = b_row0 + c;
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
      } else {
        // weight-major: this thread owns feature f; columns are tokens
        const int f = a_row0 + row;
        if (f >= p.N) continue;
        const float b = p.bias != nullptr ? __bfloat162float(p.bias[f]) : 0.f;
#pragma unroll
        for (int j = 0; j < CH; ++j) {
          const int t = b_row0 + c + j;
          if (t >= p.M) break;
          store_out(p, t, f, __uint_as_float(r[j]) + b);
        }
      }
    }
  }

  if constexpr (SPLIT) {
    // one split (a fused epilogue without split-K) runs without a cluster
    const bool clustered = gridDim.z > 1;
    if (clustered) cluster_sync();  // every CTA of the cluster has parked its partial tile
    else __syncthreads();
    // sum the cluster's partial tiles through distributed shared memory: CTA
    // rank r finalises output rows [r * R / S, (r + 1) * R / S) of the tile
    // (R = tokens in the tile), 4 consecutive features per thread and load
    constexpr int kOutRows = SWAP ? BN : BM;
    constexpr int kOutCols = SWAP ? BM : BN;
    constexpr int kLd = SWAP ? S::kRedLdSwap : S::kRedLdTok;
    const int nsplit = static_cast<int>(gridDim.z);  // == cluster size along z
    const int rank = static_cast<int>(cluster_ctarank());
    // rows [row_lo, row_lo + rows_per) of the tile; a split count that does
    // not divide the rows gives the ranks ragged shares
    const int row_lo = rank * kOutRows / nsplit;
    const int rows_per = (rank + 1) * kOutRows / nsplit - row_lo;
    const uint32_t red_base = smem_u32(smem);
    const int tok0 = SWAP ? b_row0 : a_row0;
    const int feat0 = SWAP ? a_row0 : b_row0;
    if (do_norm) {
      // rstd of this rank's rows from every CTA's partial sum of squares
      for (int r = threadIdx.x; r < rows_per; r += kThreads) {
        const int orow = row_lo + r;
        const uint32_t off = smem_u32(s_ss + orow);
        float ss = 0.f;
        if (nsplit == 1) ss = s_ss[orow];
        else
          for (int q = 0; q < nsplit; ++q) ss += ld_shared_cluster_f32(map_shared_rank(off, static_cast<uint32_t>(q)));
        s_rstd[orow] = rsqrtf(ss / static_cast<float>(p.K) + p.epi.eps);
      }
      __syncthreads();
    }
    if ((p.epi.kind & kEpiSiluMul) != 0) {
      // every 128 tile columns hold 64 gate features, then the matching 64 up
      // features; output feature = feat0 / 2 + block * 64 + column
      constexpr int kBlocks = kOutCols / 128;
      const int vecs = rows_per * kBlocks * 16;
      for (int e = threadIdx.x; e < vecs; e += kThreads) {
        const int orow = row_lo + e / (kBlocks * 16);
        const int blk = (e % (kBlocks * 16)) / 16;
        const int ocol = blk * 128 + (e % 16) * 4;
        const float4 g = reduce_parts(red_base + static_cast<uint32_t>((orow * kLd + ocol) * 4), nsplit);
        const float4 u = reduce_parts(red_base + static_cast<uint32_t>((orow * kLd + ocol + 64) * 4), nsplit);
        const int m = tok0 + orow;
        if (m >= p.M || feat0 + ocol >= p.N) continue;
        const float sc = do_norm ? s_rstd[orow] : 1.f;
        float gv[4] = {g.x * sc, g.y * sc, g.z * sc, g.w * sc};
        float uv[4] = {u.x * sc, u.y * sc, u.z * sc, u.w * sc};
        if (p.bias != nullptr) {
          for (int q = 0; q < 4; ++q) {
            gv[q] += __bfloat162float(p.bias[feat0 + ocol + q]);
            uv[q] += __bfloat162float(p.bias[feat0 + 64 + ocol + q]);
          }
        }
        float v[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          // the unfused path rounds the GEMM output to bf16 before the activation
          const float gq = round_bf16(gv[q]), uq = round_bf16(uv[q]);
          v[q] = gq / (1.f + __expf(-gq)) * uq;
        }
        store4_bf16(reinterpret_cast<__nv_bfloat16*>(p.out) + static_cast<size_t>(m) * p.ldo + feat0 / 2 + blk * 64 +
                        (e % 16) * 4,
                    v);
      }
    } else {
      const int vecs = rows_per * (kOutCols / 4);
      const bool rope = (p.epi.kind & kEpiRope) != 0;
      const bool allreduce = (p.epi.kind & kEpiAllReduce) != 0;
      const uint32_t ar_e = allreduce ? *p.epi.ar_epoch + 1 : 0u;  // after griddepcontrol.wait (see below)
      for (int e = threadIdx.x; e < vecs; e += kThreads) {
        // kEpiRope relies on one warp covering one 128-feature head of one
        // token row: kOutCols / 4 is a multiple of 32 vectors per row and
        // kThreads a multiple of 32 (the host asks for N tiles of >= 128)
        const int orow = row_lo + e / (kOutCols / 4);
        const int ocol = (e % (kOutCols / 4)) * 4;
        const float4 acc = reduce_parts(red_base + static_cast<uint32_t>((orow * kLd + ocol) * 4), nsplit);
        const int m = tok0 + orow;
        const int n = feat0 + ocol;
        if (SWAP && (p.epi.kind & kEpiSample) != 0) {
          if (m < p.M) sample_epilogue(p, m, n, acc);  // m is uniform per warp
          continue;
        }
        if (m >= p.M || n >= p.N) continue;  // uniform per warp for kEpiRope
        const float sc = do_norm ? s_rstd[orow] : 1.f;
        float v[4] = {acc.x * sc, acc.y * sc, acc.z * sc, acc.w * sc};
        if (p.bias != nullptr)
          for (int q = 0; q < 4; ++q) v[q] += n + q < p.N ? __bfloat162float(p.bias[n + q]) : 0.f;
        if (allreduce) {
          // this rank's partial, rounded as a bf16 GEMM output would be
          store4_bf16(ar_half(p, p.epi.ar_rank, ar_e) + static_cast<size_t>(m) * p.N + n, v);
          continue;
        }
        if (rope) {
          rope_epilogue(p, n / 128, m, n % 128, v);
          continue;
        }
        if ((p.epi.kind & kEpiResidual) != 0) {
          const uint2 rr = *reinterpret_cast<const uint2*>(
              reinterpret_cast<const __nv_bfloat16*>(p.epi.residual) + static_cast<size_t>(m) * p.epi.ld_res + n);
          const float2 r0 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&rr.x));
          const float2 r1 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&rr.y));
          // the residual stream is kept in bf16: round the projection first,
          // then the sum, as a separate add would
          v[0] = round_bf16(v[0]) + r0.x, v[1] = round_bf16(v[1]) + r0.y;
          v[2] = round_bf16(v[2]) + r1.x, v[3] = round_bf16(v[3]) + r1.y;
        }
        if (n + 4 <= p.N && (p.ldo & 3) == 0) {
          if (p.out_f32) {
            *reinterpret_cast<float4*>(reinterpret_cast<float*>(p.out) + static_cast<size_t>(m) * p.ldo + n) =
                make_float4(v[0], v[1], v[2], v[3]);
          } else {
            store4_bf16(reinterpret_cast<__nv_bfloat16*>(p.out) + static_cast<size_t>(m) * p.ldo + n, v);
          }
        } else {
          for (int q = 0; q < 4 && n + q < p.N; ++q) store_out(p, m, n + q, v[q]);
        }
      }
      if (allreduce) {
        // Exchange with the other ranks: every rank runs the same plan, so
        // CTA `cta` covers the same output elements everywhere. The epoch was
        // read after this CTA's producer passed griddepcontrol.wait, i.e.
        // after the previous call's counter bump completed.
        const int cta = static_cast<int>((blockIdx.z * gridDim.y + blockIdx.y) * gridDim.x + blockIdx.x);
        __syncthreads();
        if (threadIdx.x == 0) {
          __threadfence_system();
          ar_store_release(ar_flag(p, p.epi.ar_rank, cta), ar_e);
        }
        if (threadIdx.x < p.epi.ar_world) ar_wait(p, ar_flag(p, threadIdx.x, cta), ar_e);
        __syncthreads();
        for (int e = threadIdx.x; e < vecs; e += kThreads) {
          const int orow = row_lo + e / (kOutCols / 4);
          const int ocol = (e % (kOutCols / 4)) * 4;
          const int m = tok0 + orow;
          const int n = feat0 + ocol;
          if (m >= p.M || n >= p.N) continue;
          float v[4] = {0.f, 0.f, 0.f, 0.f};
          for (int r = 0; r < p.epi.ar_world; ++r) {  // rank order: the same bits on every rank
            const uint2 raw = *reinterpret_cast<const uint2*>(ar_half(p, r, ar_e) + static_cast<size_t>(m) * p.N + n);
            const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&raw.x));
            const float2 b = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&raw.y));
            v[0] += a.x, v[1] += a.y, v[2] += b.x, v[3] += b.y;
          }
          if ((p.epi.kind & kEpiResidual) != 0) {
            const uint2 rr = *reinterpret_cast<const uint2*>(
                reinterpret_cast<const __nv_bfloat16*>(p.epi.residual) + static_cast<size_t>(m) * p.epi.ld_res + n);
            const float2 r0 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&rr.x));
            const float2 r1 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&rr.y));
            v[0] = round_bf16(v[0]) + r0.x, v[1] = round_bf16(v[1]) + r0.y;
            v[2] = round_bf16(v[2]) + r1.x, v[3] = round_bf16(v[3]) + r1.y;
          }
          store4_bf16(reinterpret_cast<__nv_bfloat16*>(p.out) + static_cast<size_t>(m) * p.ldo + n, v);
        }
      }
    }
    if (clustered) cluster_sync();  // peers may still be reading this CTA's tile
  }

  tc_fence_before();
  __syncthreads();
  if (threadIdx.x == 0) trace_stamp(p, 5);
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kCols);
  }
}

// When set, launch_tile reports grid residency here instead of launching.
thread_local int* g_resident_query = nullptr;

template <int BN, int STAGES, bool SWAP, bool SPLIT>
void launch_tile(const CUtensorMap& ta, const CUtensorMap& tb, const KParams& kp, dim3 grid, int splits,
                 cudaStream_t stream) {
  auto kern = gemm_tc_kernel<BN, STAGES, SWAP, SPLIT>;
  const uint32_t smem = Smem<BN, STAGES>::bytes(kp.stages, SPLIT, kp.kps);
  static bool configured[64] = {};  // one attribute call per instantiation and device
  int dev = 0;
  cudaGetDevice(&dev);
  if (!configured[dev & 63]) {
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Smem<BN, STAGES>::kBytes);
    if (SPLIT) cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
    configured[dev & 63] = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attrs[2];
  int n = 0;
  if (pdl_enabled()) {
    attrs[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attrs[n].val.programmaticStreamSerializationAllowed = 1;
    ++n;
  }
  if (SPLIT && splits > 1) {
    attrs[n].id = cudaLaunchAttributeClusterDimension;
    attrs[n].val.clusterDim.x = 1;
    attrs[n].val.clusterDim.y = 1;
    attrs[n].val.clusterDim.z = static_cast<unsigned>(splits);
    ++n;
  }
  cfg.attrs = attrs;
  cfg.numAttrs = n;
  if (g_resident_query != nullptr) {
    // query only: can every CTA (cluster) of this grid be resident at once?
    int sms = 0;
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const int64_t ctas = static_cast<int64_t>(grid.x) * grid.y * grid.z;
    if (SPLIT && splits > 1) {
      int clusters = 0;
      const cudaError_t q = cudaOccupancyMaxActiveClusters(&clusters, kern, &cfg);
      *g_resident_query = q == cudaSuccess && static_cast<int64_t>(clusters) * splits >= ctas;
    } else {
      int per_sm = 0;
      const cudaError_t q = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kThreads, smem);
      *g_resident_query = q == cudaSuccess && static_cast<int64_t>(per_sm) * sms >= ctas;
    }
    if (ctas > kSymmFlagBytes / 4) *g_resident_query = 0;  // one flag slot per CTA
    return;
  }
  cudaError_t e = cudaLaunchKernelEx(&cfg, kern, ta, tb, kp);
  if (e != cudaSuccess) throw std::runtime_error(std::string("minisgl.gemm launch failed: ") + cudaGetErrorString(e));
}

template <int BN, int STAGES, bool SWAP>
void dispatch_split(int splits, const CUtensorMap& ta, const CUtensorMap& tb, KParams kp, dim3 grid,
                    cudaStream_t stream) {
  // the ring keeps its byte budget: STAGES k-blocks in stages of kps
  kp.stages = std::max(1, std::min(STAGES / kp.kps, (kp.kb_per_split + kp.kps - 1) / kp.kps));
  // fused epilogues of weight-major tiles live in the cluster (split-K) path
  // (one split = a cluster of one); token-major tiles without split-K apply
  // them straight from TMEM
  if (splits > 1 || (SWAP && kp.epi.kind != 0) || (kp.epi.kind & kEpiAllReduce) != 0)
    launch_tile<BN, STAGES, SWAP, true>(ta, tb, kp, grid, splits, stream);
  else launch_tile<BN, STAGES, SWAP, false>(ta, tb, kp, grid, 1, stream);
}

constexpr int kMaxSplits = 16;
constexpr int kTargetCtas = 148;

struct Plan {
  bool swap;
  int bn;
  int stages;
  int tiles;
  int splits;
  int kb_per_split;
};

int tiles_for(int M, int N, int bn, bool swap) {
  return swap ? ((N + BM - 1) / BM) * ((M + bn - 1) / bn) : ((M + BM - 1) / BM) * ((N + bn - 1) / bn);
}

int stages_for(int bn) { return bn <= 64 ? 8 : 4; }

// Default tile plan (autotuned plans from the Python side override it):
//   * weight-major tiles for up to 128 tokens, 16 or 32 tokens per tile;
//   * split K until each CTA's whole weight slice fits its stage ring (so it
//     is prefetched under PDL before griddepcontrol.wait), then keep
//     splitting while that still fits about one CTA per SM.
Plan make_plan(int M, int N, int K, int force_mode, int force_splits, int force_bn = 0) {
  Plan pl;
  const int num_kb = (K + BK - 1) / BK;
  pl.swap = force_mode == 2 || (force_mode == 0 && M <= 128);
  if (pl.swap) {
    pl.bn = M <= 16 ? 16 : 32;
  } else {
    pl.bn = M >= 1024 ? 256 : 64;
    if (M >= 1024 && tiles_for(M, N, 256, false) < 120) pl.bn = 128;
  }
  if (force_bn > 0) pl.bn = force_bn;
  pl.stages = stages_for(pl.bn);
  pl.tiles = tiles_for(M, N, pl.bn, pl.swap);
  const int out_rows = pl.swap ? pl.bn : BM;
  int splits = 1;
  if (force_splits > 0) {
    splits = force_splits;
  } else if (M < 1024) {
    while (splits < kMaxSplits && (num_kb + splits - 1) / splits > pl.stages) splits *= 2;
    while (splits < kMaxSplits && pl.tiles * splits * 2 <= kTargetCtas && num_kb / (splits * 2) >= 2) splits *= 2;
  }
  splits = std::max(1, std::min(splits, kMaxSplits));
  while (splits > 1 && (splits > num_kb || splits > out_rows)) splits /= 2;
  pl.kb_per_split = (num_kb + splits - 1) / splits;
  pl.splits = splits;
  return pl;
}

}  // namespace

int64_t gemm_workspace_elems(int, int, int) { return 0; }

// (swap, bn, splits, grid CTAs) of the heuristic plan, for tests and tools.
std::vector<int64_t> gemm_plan_desc(int64_t M, int64_t N, int64_t K) {
  const Plan pl = make_plan(static_cast<int>(M), static_cast<int>(N), static_cast<int>(K), 0, 0, 0);
  return {pl.swap ? 1 : 0, pl.bn, pl.splits, static_cast<int64_t>(pl.tiles) * pl.splits, pl.stages};
}

void launch_gemm(const GemmArgs& a, cudaStream_t stream) {
  if (a.M <= 0 || a.N <= 0) return;
  if (a.force_mode == 4) {
    // stream-K weight streaming (gemm_streamk.cu): force_bn = weight sub-tiles
    // per work tile (R), force_kps = k-blocks per stage (0: automatic); the
    // workspace holds one partial tile per SM followed by the ready flags
    int dev = 0, sms = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (a.workspace == nullptr || a.workspace_elems < static_cast<int64_t>(sms) * (kStreamKSlotFloats + kStreamKFlagWords))
      throw std::runtime_error("minisgl.gemm: the stream-K plan needs its workspace");
    GemmStreamKArgs k{};
    k.x = a.x;
    k.w = a.w;
    k.bias = a.bias;
    k.out = a.out;
    k.M = a.M;
    k.N = a.N;
    k.K = a.K;
    k.ldx = a.ldx;
    k.ldw = a.ldw;
    k.ldo = a.ldo;
    k.out_f32 = a.out_f32 ? 1 : 0;
    k.R = a.force_bn == 2 ? 2 : 1;
    k.kps = a.force_kps;
    k.grid = gemm_streamk_grid(a.M, a.N, a.K, k.R, sms);
    k.ws = a.workspace;
    k.flags = reinterpret_cast<int*>(a.workspace + static_cast<int64_t>(sms) * kStreamKSlotFloats);
    k.ws_slots = sms;
    k.ws_slot_floats = kStreamKSlotFloats;
    k.err = a.err;
    k.trace = a.trace;
    launch_gemm_streamk(k, stream);
    return;
  }
  if (a.K % 8 != 0 || a.ldx % 8 != 0 || a.ldw % 8 != 0)
    throw std::runtime_error("minisgl.gemm: K and row strides must be multiples of 8 elements");
  if (a.N % 4 != 0) throw std::runtime_error("minisgl.gemm: N must be a multiple of 4");
  if (a.force_bn != 0 && a.force_bn != 16 && a.force_bn != 32 && a.force_bn != 64 && a.force_bn != 128 &&
      a.force_bn != 256)
    throw std::runtime_error("minisgl.gemm: N tile must be 16, 32, 64, 128 or 256");
  // persistent tiles: asked for (plan mode 3), or the default for long
  // token batches of a plain GEMM (measured 1.7-2x faster than one tile per
  // CTA at 16k tokens on B200)
  if (a.force_mode == 5) {  // persistent CTA pairs (256 x 256 tiles, cta_group::2)
    launch_gemm_pair(a, stream);
    return;
  }
  if (a.force_mode == 3 ||
      (a.force_mode == 0 && a.force_splits <= 1 && a.M >= 1024 && gemm_persistent_supported(a))) {
    launch_gemm_persistent(a, stream);
    return;
  }
  if (a.force_bn == 16 && a.force_mode == 1)
    throw std::runtime_error("minisgl.gemm: token-major tiles need an N tile of at least 32");
  if (a.g_num_tiles != nullptr) {
    if (a.force_mode == 1 || a.force_bn <= 0 || a.force_splits > 1 || a.g_experts <= 0 || a.N % BM != 0)
      throw std::runtime_error("minisgl.gemm: grouped GEMMs use weight-major tiles of the align tile, no split-K, "
                               "and expert matrices of a multiple of 128 rows");
  }
  const int fused = a.epi.kind;
  if (fused != 0) {
    if (a.out_f32) throw std::runtime_error("minisgl.gemm: fused epilogues write bf16");
    // token-major tiles hold whole 128-feature heads / gate|up blocks only
    // when their N tile is a multiple of 128
    if ((fused & (kEpiSiluMul | kEpiRope)) != 0 && a.force_mode == 1 && a.force_bn % 128 != 0)
      throw std::runtime_error("minisgl.gemm: token-major silu / rope epilogues need an N tile of 128 or 256");
    if ((fused & kEpiResidual) != 0 && (a.epi.residual == nullptr || a.epi.ld_res % 4 != 0))
      throw std::runtime_error("minisgl.gemm: residual epilogue needs a residual with row stride % 4 == 0");
    if ((fused & kEpiSiluMul) != 0 && (a.N % 128 != 0 || (fused & (kEpiRope | kEpiResidual)) != 0))
      throw std::runtime_error("minisgl.gemm: silu epilogue needs N % 128 == 0 and no rope / residual");
    if ((fused & kEpiSample) != 0) {
      if (fused != kEpiSample || a.force_mode == 1 || a.epi.part_val == nullptr || a.epi.part_idx == nullptr ||
          a.epi.step == nullptr || a.epi.ntiles != (a.N + 127) / 128)
        throw std::runtime_error("minisgl.gemm: the sampling epilogue runs alone on weight-major tiles");
    }
    if ((fused & kEpiRope) != 0) {
      if (a.N != (a.epi.hq + 2 * a.epi.hk) * 128 || a.epi.cos_sin == nullptr || a.epi.positions == nullptr ||
          a.epi.out_loc == nullptr || a.epi.k_cache == nullptr || a.epi.v_cache == nullptr || a.epi.page_size <= 0 ||
          (fused & kEpiResidual) != 0)
        throw std::runtime_error("minisgl.gemm: rope epilogue needs head_dim 128 qkv weights and cache pointers");
    }
  }
  // fused and grouped calls default to weight-major tiles
  const bool default_swap = (fused != 0 || a.g_num_tiles != nullptr) && a.force_mode == 0;
  const Plan pl = make_plan(a.M, a.N, a.K, default_swap ? 2 : a.force_mode, a.force_splits, a.force_bn);
  KParams kp;
  kp.out = a.out;
  kp.bias = reinterpret_cast<const __nv_bfloat16*>(a.bias);
  kp.M = a.M;
  kp.N = a.N;
  kp.ldo = a.ldo;
  kp.kb_per_split = pl.kb_per_split;
  kp.num_kb = (a.K + BK - 1) / BK;
  // k-blocks per stage: one 3-D TMA box per operand moves kps k-blocks (a
  // TMA box costs about the same whatever its size, so bigger boxes stream
  // faster); needs whole k-blocks everywhere and at least two stages
  {
    const int max_stages = pl.bn >= 128 ? 4 : 8;
    const bool ok_k = a.K % BK == 0;
    auto fits = [&](int c) {
      return ok_k && kp.num_kb % c == 0 && kp.kb_per_split % c == 0 && max_stages / c >= 2;
    };
    if (a.force_kps > 0) {
      if (a.force_kps != 1 && !fits(a.force_kps))
        throw std::runtime_error("minisgl.gemm: k-blocks per stage must divide the K range of every split");
      kp.kps = a.force_kps;
    } else {
      kp.kps = fits(4) ? 4 : (fits(2) ? 2 : 1);
    }
  }
  kp.out_f32 = a.out_f32 ? 1 : 0;
  kp.K = a.K;
  kp.epi = a.epi;
  kp.g_tile_expert = a.g_tile_expert;
  kp.g_tile_row = a.g_tile_row;
  kp.g_num_tiles = a.g_num_tiles;
  kp.err = ErrorSink{a.err};
  kp.trace = reinterpret_cast<unsigned long long*>(a.trace);
  auto tmap = [&](const void* base, int rows, int ld, int box_rows) {
    return kp.kps > 1 ? make_tmap_bf16_kblocks(base, rows, a.K, ld, box_rows, kp.kps)
                      : make_tmap_bf16_2d_sw128(base, rows, a.K, ld, box_rows);
  };
  if (pl.swap) {
    CUtensorMap ta = tmap(a.w, a.g_num_tiles != nullptr ? a.N * a.g_experts : a.N, a.ldw, BM);
    CUtensorMap tb = tmap(a.x, a.M, a.ldx, pl.bn);
    dim3 grid((a.M + pl.bn - 1) / pl.bn, (a.N + BM - 1) / BM, pl.splits);
    switch (pl.bn) {
      case 16: dispatch_split<16, 8, true>(pl.splits, ta, tb, kp, grid, stream); break;
      case 32: dispatch_split<32, 8, true>(pl.splits, ta, tb, kp, grid, stream); break;
      case 64: dispatch_split<64, 8, true>(pl.splits, ta, tb, kp, grid, stream); break;
      case 128: dispatch_split<128, 4, true>(pl.splits, ta, tb, kp, grid, stream); break;
      default: dispatch_split<256, 4, true>(pl.splits, ta, tb, kp, grid, stream); break;
    }
  } else {
    CUtensorMap ta = tmap(a.x, a.M, a.ldx, BM);
    CUtensorMap tb = tmap(a.w, a.N, a.ldw, pl.bn);
    dim3 grid((a.N + pl.bn - 1) / pl.bn, (a.M + BM - 1) / BM, pl.splits);
    switch (pl.bn) {
      case 32: dispatch_split<32, 8, false>(pl.splits, ta, tb, kp, grid, stream); break;
      case 64: dispatch_split<64, 8, false>(pl.splits, ta, tb, kp, grid, stream); break;
      case 128: dispatch_split<128, 4, false>(pl.splits, ta, tb, kp, grid, stream); break;
      default: dispatch_split<256, 4, false>(pl.splits, ta, tb, kp, grid, stream); break;
    }
  }
}

// Row-parallel GEMM with the tensor-parallel all-reduce. When every CTA of
// the planned grid can be resident at once, one kernel computes, exchanges
// and reduces (kEpiAllReduce; CTAs wait on the same CTA of the other ranks,
// which is only deadlock-free if none of them waits for a slot). Otherwise
// the GEMM writes its partial into the heap's collective region and the
// collective kernel reduces it.
void launch_gemm_allreduce(const GemmArgs& a, const int64_t* bases, uint32_t* epoch, int64_t own_base, int rank,
                           int world, int64_t half_bytes, void* residual_out, cudaStream_t s) {
  if (static_cast<int64_t>(a.M) * a.N * 2 > half_bytes)
    throw std::runtime_error("minisgl.gemm_allreduce: output larger than the heap half");
  GemmArgs b = a;
  b.out = residual_out;
  b.ldo = a.N;
  b.epi.kind = kEpiAllReduce | kEpiResidual;
  b.epi.residual = residual_out;
  b.epi.ld_res = a.N;
  b.epi.ar_bases = bases;
  b.epi.ar_epoch = epoch;
  b.epi.ar_rank = rank;
  b.epi.ar_world = world;
  b.epi.ar_half_bytes = half_bytes;
  int resident = 0;
  g_resident_query = &resident;
  try {
    launch_gemm(b, s);
  } catch (...) {
    g_resident_query = nullptr;
    throw;
  }
  g_resident_query = nullptr;
  if (resident) {
    launch_gemm(b, s);
    launch_epoch_bump(epoch, s);
    return;
  }
  GemmArgs c = a;  // the partial into the collective region, then the collective kernel
  c.out = reinterpret_cast<void*>(own_base + kSymmSignalBytes + kSymmFlagBytes);
  c.ldo = a.N;
  c.epi.kind = 0;
  launch_gemm(c, s);
  launch_symm_collective(0, bases, epoch + 1, rank, world, static_cast<int64_t>(a.M) * a.N, residual_out,
                         residual_out, 0, 0, a.err, s);
}

}  // namespace minisgl
