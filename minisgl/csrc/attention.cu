// Paged GQA attention for sm_100a: decode (split-KV flash-decoding) and
// causal prefill/extend over a paged KV pool.
//
// Replaces the reference's attention backends (python/minisgl/attention/
// trtllm.py:49-89 TRT-LLM FMHA, attention/fi.py, attention/fa.py).
//
// KV tiles of 64 keys x head_dim (128) bf16 are moved by TMA (2-D tensor map
// over the whole pool, 128-byte swizzle, one box per page segment and
// 64-column half) into a multi-stage mbarrier ring. Prefill runs on tcgen05
// (prefill_attn_tc_kernel: 128 query rows per CTA, S / O / P in TMEM). Decode
// and the prefill kernel for q strides TMA cannot take use the warp-level
// bf16 MMA (m16n8k16) with ldmatrix fragments read from the swizzled tiles:
// decode has 1-16 query rows per KV head, too few for a 128-row tcgen05
// tile. Decode attention moves ~2 bytes per multiply-add
// pair (GQA group <= 16 query rows per key), so it is bound by HBM bandwidth,
// not by the tensor pipe; the design goal is to keep enough bytes in flight
// (3 stages x 32 KB per CTA, 2 CTAs per SM) to saturate HBM3e.
//
// Softmax runs in the exp2 domain: q is pre-scaled by scale * log2(e).
#include <algorithm>
#include <cstdlib>
#include <cstdarg>
#include <cstdio>
#include <mutex>
#include <stdexcept>
#include <string>
#include <utility>

#include "common.cuh"
#include "launch.h"
#include "noalloc.h"
#include "ops.h"
#include "tma_host.h"

namespace minisgl {
namespace {

constexpr int kD = 128;      // head_dim supported by the tensor-core path
constexpr int kTile = 64;    // keys per tile
constexpr int kStages = 3;
constexpr int kHalfBytes = kTile * 128;        // one 64-column half of a tile (8 KB)
constexpr int kTileBytes = 2 * kHalfBytes;     // K or V tile (16 KB)
constexpr int kStageBytes = 2 * kTileBytes;    // K + V (32 KB)
constexpr float kLog2e = 1.4426950408889634f;

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                        uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                          uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void mma_bf16(float (&c)[4], const uint32_t (&a)[4], uint32_t b0,
                                         uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// Byte offset of (row, 16-byte chunk 0..15) inside a 64-row tile stored as
// two 128B-swizzled halves (chunks 0..7 and 8..15).
__device__ __forceinline__ uint32_t tile_off(int row, int chunk) {
  const int half = chunk >> 3;
  const int c = chunk & 7;
  return half * kHalfBytes + row * 128 + ((c ^ (row & 7)) << 4);
}

// Issue the TMA loads of one 64-key tile (K and V) starting at position p0.
__device__ __forceinline__ void issue_kv_tile(uint8_t* stage, uint64_t* bar,
                                              const CUtensorMap* tm, const AttnArgs& a,
                                              const int32_t* pt_row, int L, int p0, int h) {
  mbar_arrive_expect_tx(bar, kStageBytes);
  const int P = a.page_size;
  const int seg = P < kTile ? P : kTile;
  for (int j = 0; j < kTile; j += seg) {
    const int pos = p0 + j;
    int page = 0;
    if (pos < L) page = pt_row[pos] / P;  // positions past the end read page 0 (masked later)
    const int64_t in_page = P < kTile ? 0 : (p0 % P);
    const int64_t row = (static_cast<int64_t>(page) * a.hk + h) * P + in_page;
    const int32_t rk = static_cast<int32_t>(a.k_row0 + row);
    const int32_t rv = static_cast<int32_t>(a.v_row0 + row);
    uint8_t* k = stage;
    uint8_t* v = stage + kTileBytes;
    tma_load_2d(k + j * 128, tm, bar, 0, rk);
    tma_load_2d(k + kHalfBytes + j * 128, tm, bar, 64, rk);
    tma_load_2d(v + j * 128, tm, bar, 0, rv);
    tma_load_2d(v + kHalfBytes + j * 128, tm, bar, 64, rv);
  }
}

// Load 16 query rows (rows >= nrows are zero) as m16n8k16 A fragments for the
// 8 k-steps of d = 128, pre-scaled by `mul`.
__device__ __forceinline__ void load_q_frags(uint32_t (&qa)[8][4], const __nv_bfloat16* q,
                                             int64_t row_stride, int nrows, float mul) {
  const int lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
#pragma unroll
  for (int ks = 0; ks < 8; ++ks) {
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      const int row = g + ((r & 1) ? 8 : 0);
      const int col = ks * 16 + 2 * t + ((r & 2) ? 8 : 0);
      float x0 = 0.f, x1 = 0.f;
      if (row < nrows) {
        const __nv_bfloat162 v =
            *reinterpret_cast<const __nv_bfloat162*>(q + row * row_stride + col);
        x0 = __bfloat162float(v.x) * mul;
        x1 = __bfloat162float(v.y) * mul;
      }
      qa[ks][r] = pack_bf16x2(x0, x1);
    }
  }
}

// ============================================================== decode ====
// grid (max_splits, hk, B); 5 warps. Warps 0-3 consume: warp w handles keys
// [16w, 16w+16) of each tile for all G = hq / hk query heads of this kv
// head. Warp 4 produces: it streams 64-key K/V tiles through a 3-stage ring
// (full barriers completed by TMA bytes, empty barriers by the 4 consumer
// warps), so no CTA-wide barrier sits in the loop. The four partial softmax
// states are merged at the end.
constexpr int kConsumers = 4;
constexpr int kDecodeThreads = (kConsumers + 1) * 32;
constexpr int kMergeLd = kD + 4;  // padded row of the merge buffer (floats)

__global__ void __launch_bounds__(kDecodeThreads, 2)
    decode_attn_kernel(const __grid_constant__ CUtensorMap tm, AttnArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kStages * kStageBytes);
  uint64_t* empty = full + kStages;
  const ErrorSink err{a.err};

  pdl_launch_dependents();
  const int split = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int G = a.hq / a.hk;
  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kConsumers);
    }
    fence_barrier_init();
    prefetch_tmap(&tm);
  }
  // q, the KV of the current token and the metadata come from earlier kernels
  pdl_wait();
  const int L = a.seq_lens[b];
  // chunk of keys for this split: a multiple of the tile, at least one tile
  int chunk = (L + a.max_splits - 1) / a.max_splits;
  chunk = max(kTile, (chunk + kTile - 1) / kTile * kTile);
  const int nsplit = max(1, (L + chunk - 1) / chunk);
  if (split >= nsplit) return;
  const int k_begin = split * chunk;
  const int k_end = min(L, k_begin + chunk);
  const int ntiles = k_end > k_begin ? (k_end - k_begin + kTile - 1) / kTile : 0;
  const int32_t* pt_row = a.page_table + static_cast<int64_t>(a.req_rows[b]) * a.ld_pt;
  if (a.pt_rows > 0 && (a.req_rows[b] < 0 || a.req_rows[b] >= a.pt_rows)) {  // uniform over the CTA
    if (threadIdx.x == 0) err.report(kErrBadIndex, 921);
    return;
  }
  __syncthreads();

  const int g = lane >> 2, t = lane & 3;
  float m_lo = -INFINITY, m_hi = -INFINITY;  // running max for rows g and g+8
  float l_lo = 0.f, l_hi = 0.f;
  float o[16][4];
#pragma unroll
  for (int n = 0; n < 16; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;

  if (warp == kConsumers) {
    // ------------------------------------------------------- producer ----
    if (lane == 0) {
      for (int i = 0; i < ntiles; ++i) {
        const int s = i % kStages;
        if (i >= kStages && !mbar_wait(&empty[s], ((i / kStages) & 1u) ^ 1u, err, 200)) break;
        issue_kv_tile(smem + s * kStageBytes, &full[s], &tm, a, pt_row, L, k_begin + i * kTile, h);
      }
    }
  } else {
    // ------------------------------------------------------- consumers ----
    const __nv_bfloat16* qb =
        reinterpret_cast<const __nv_bfloat16*>(a.q) + static_cast<int64_t>(b) * a.ld_q + h * G * kD;
    uint32_t qa[8][4];
    load_q_frags(qa, qb, kD, G, a.scale * kLog2e);
    bool ok = true;
    const int mi = lane >> 3, rr = lane & 7;
    const int tok0 = warp * 16;  // this warp's 16 keys inside the tile
    for (int i = 0; i < ntiles; ++i) {
      const int s = i % kStages;
      if (ok) ok = mbar_wait(&full[s], (i / kStages) & 1u, err, 201);
      const uint32_t kbase = smem_u32(smem + s * kStageBytes);
      const uint32_t vbase = kbase + kTileBytes;
      // S = Q K^T for 16 rows x 16 keys
      float sc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
      {
        const int tok = tok0 + (mi >> 1) * 8 + rr;
#pragma unroll
        for (int ks = 0; ks < 8; ++ks) {
          uint32_t b0, b1, b2, b3;
          ldsm_x4(kbase + tile_off(tok, ks * 2 + (mi & 1)), b0, b1, b2, b3);
          mma_bf16(sc[0], qa[ks], b0, b1);
          mma_bf16(sc[1], qa[ks], b2, b3);
        }
      }
      // mask keys past the end of this split
      const int pos0 = k_begin + i * kTile + tok0;
#pragma unroll
      for (int nt = 0; nt < 2; ++nt) {
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int pos = pos0 + nt * 8 + 2 * t + (e & 1);
          if (pos >= k_end) sc[nt][e] = -INFINITY;
        }
      }
      // online softmax (rows g: elements 0,1 ; rows g+8: elements 2,3)
      float mx_lo = fmaxf(fmaxf(sc[0][0], sc[0][1]), fmaxf(sc[1][0], sc[1][1]));
      float mx_hi = fmaxf(fmaxf(sc[0][2], sc[0][3]), fmaxf(sc[1][2], sc[1][3]));
      mx_lo = fmaxf(mx_lo, __shfl_xor_sync(0xffffffffu, mx_lo, 1));
      mx_lo = fmaxf(mx_lo, __shfl_xor_sync(0xffffffffu, mx_lo, 2));
      mx_hi = fmaxf(mx_hi, __shfl_xor_sync(0xffffffffu, mx_hi, 1));
      mx_hi = fmaxf(mx_hi, __shfl_xor_sync(0xffffffffu, mx_hi, 2));
      const float new_lo = fmaxf(m_lo, mx_lo), new_hi = fmaxf(m_hi, mx_hi);
      const float base_lo = new_lo == -INFINITY ? 0.f : new_lo;
      const float base_hi = new_hi == -INFINITY ? 0.f : new_hi;
      const float alpha_lo = exp2f(m_lo - base_lo), alpha_hi = exp2f(m_hi - base_hi);
      m_lo = new_lo, m_hi = new_hi;
      float p[2][4];
      float sum_lo = 0.f, sum_hi = 0.f;
#pragma unroll
      for (int nt = 0; nt < 2; ++nt) {
        p[nt][0] = exp2f(sc[nt][0] - base_lo);
        p[nt][1] = exp2f(sc[nt][1] - base_lo);
        p[nt][2] = exp2f(sc[nt][2] - base_hi);
        p[nt][3] = exp2f(sc[nt][3] - base_hi);
        sum_lo += p[nt][0] + p[nt][1];
        sum_hi += p[nt][2] + p[nt][3];
      }
      l_lo = l_lo * alpha_lo + sum_lo;
      l_hi = l_hi * alpha_hi + sum_hi;
#pragma unroll
      for (int n = 0; n < 16; ++n) {
        o[n][0] *= alpha_lo, o[n][1] *= alpha_lo;
        o[n][2] *= alpha_hi, o[n][3] *= alpha_hi;
      }
      uint32_t pa[4];
      pa[0] = pack_bf16x2(p[0][0], p[0][1]);
      pa[1] = pack_bf16x2(p[0][2], p[0][3]);
      pa[2] = pack_bf16x2(p[1][0], p[1][1]);
      pa[3] = pack_bf16x2(p[1][2], p[1][3]);
      // O += P V   (V rows tok0..tok0+15, all 128 columns)
      {
        const int tok = tok0 + (mi & 1) * 8 + rr;
#pragma unroll
        for (int nd = 0; nd < 16; nd += 2) {
          uint32_t b0, b1, b2, b3;
          ldsm_x4_t(vbase + tile_off(tok, nd + (mi >> 1)), b0, b1, b2, b3);
          mma_bf16(o[nd], pa, b0, b1);
          mma_bf16(o[nd + 1], pa, b2, b3);
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);  // this warp is done with stage s
    }
  }

  // ---- merge the four consumer warps' partial states (rows < G)
  l_lo += __shfl_xor_sync(0xffffffffu, l_lo, 1);
  l_lo += __shfl_xor_sync(0xffffffffu, l_lo, 2);
  l_hi += __shfl_xor_sync(0xffffffffu, l_hi, 1);
  l_hi += __shfl_xor_sync(0xffffffffu, l_hi, 2);
  __syncthreads();  // every tile consumed: the ring buffers are free now
  float* so = reinterpret_cast<float*>(smem);           // [4 warps][16 rows][kMergeLd]
  float* sm = so + kConsumers * 16 * kMergeLd;           // [4][16]
  float* sl = sm + kConsumers * 16;                      // [4][16]
  if (warp < kConsumers) {
#pragma unroll
    for (int n = 0; n < 16; ++n) {
      const int col = n * 8 + 2 * t;
      *reinterpret_cast<float2*>(so + (warp * 16 + g) * kMergeLd + col) = make_float2(o[n][0], o[n][1]);
      *reinterpret_cast<float2*>(so + (warp * 16 + g + 8) * kMergeLd + col) = make_float2(o[n][2], o[n][3]);
    }
    if (t == 0) {
      sm[warp * 16 + g] = m_lo;
      sm[warp * 16 + g + 8] = m_hi;
      sl[warp * 16 + g] = l_lo;
      sl[warp * 16 + g + 8] = l_hi;
    }
  }
  __syncthreads();
  // each consumer warp finishes rows warp, warp+4, ... (< G); lane covers 4 columns
  for (int r = warp; r < G && warp < kConsumers; r += kConsumers) {
    float mx = -INFINITY;
    for (int w = 0; w < kConsumers; ++w) mx = fmaxf(mx, sm[w * 16 + r]);
    const float base = mx == -INFINITY ? 0.f : mx;
    float lsum = 0.f, f[kConsumers];
    for (int w = 0; w < kConsumers; ++w) {
      f[w] = exp2f(sm[w * 16 + r] - base);
      lsum += sl[w * 16 + r] * f[w];
    }
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    for (int w = 0; w < kConsumers; ++w) {
      const float4 v = *reinterpret_cast<const float4*>(so + (w * 16 + r) * kMergeLd + lane * 4);
      acc[0] += v.x * f[w], acc[1] += v.y * f[w], acc[2] += v.z * f[w], acc[3] += v.w * f[w];
    }
    const float inv = lsum > 0.f ? 1.f / lsum : 0.f;
    const int qh = h * G + r;
    if (nsplit == 1) {
      __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(a.out) +
                           (static_cast<int64_t>(b) * a.hq + qh) * kD + lane * 4;
      uint2 pk;
      pk.x = pack_bf16x2(acc[0] * inv, acc[1] * inv);
      pk.y = pack_bf16x2(acc[2] * inv, acc[3] * inv);
      *reinterpret_cast<uint2*>(dst) = pk;
    } else {
      const int64_t slot = (static_cast<int64_t>(b) * a.hq + qh) * a.max_splits + split;
      float* dst = a.part_o + slot * kD + lane * 4;
      *reinterpret_cast<float4*>(dst) =
          make_float4(acc[0] * inv, acc[1] * inv, acc[2] * inv, acc[3] * inv);
      // log2-sum-exp of this split (in the scaled exp2 domain)
      if (lane == 0) a.part_lse[slot] = lsum > 0.f ? base + log2f(lsum) : -INFINITY;
    }
  }
}

// Merge split-KV partials: grid (B), block = 32 * 4 threads, warp per head.
__global__ void decode_combine_kernel(AttnArgs a) {
  pdl_launch_dependents();
  pdl_wait();
  const int b = blockIdx.y;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int qh = blockIdx.x * 4 + warp;
  if (qh >= a.hq) return;
  const int L = a.seq_lens[b];
  int chunk = (L + a.max_splits - 1) / a.max_splits;
  chunk = max(kTile, (chunk + kTile - 1) / kTile * kTile);
  const int nsplit = max(1, (L + chunk - 1) / chunk);
  if (nsplit == 1) return;  // written directly by the main kernel
  const int64_t base_slot = (static_cast<int64_t>(b) * a.hq + qh) * a.max_splits;
  float mx = -INFINITY;
  for (int s = 0; s < nsplit; ++s) mx = fmaxf(mx, a.part_lse[base_slot + s]);
  const float base = mx == -INFINITY ? 0.f : mx;
  float acc[4] = {0.f, 0.f, 0.f, 0.f}, wsum = 0.f;
  for (int s = 0; s < nsplit; ++s) {
    const float w = exp2f(a.part_lse[base_slot + s] - base);
    wsum += w;
    const float4 v = *reinterpret_cast<const float4*>(a.part_o + (base_slot + s) * kD + lane * 4);
    acc[0] += v.x * w, acc[1] += v.y * w, acc[2] += v.z * w, acc[3] += v.w * w;
  }
  const float inv = wsum > 0.f ? 1.f / wsum : 0.f;
  __nv_bfloat16* dst =
      reinterpret_cast<__nv_bfloat16*>(a.out) + (static_cast<int64_t>(b) * a.hq + qh) * kD + lane * 4;
  uint2 pk;
  pk.x = pack_bf16x2(acc[0] * inv, acc[1] * inv);
  pk.y = pack_bf16x2(acc[2] * inv, acc[3] * inv);
  *reinterpret_cast<uint2*>(dst) = pk;
}

// ============================================================= prefill ====
// grid (ceil(max_q / 64), hq, B); 4 warps, warp w owns query rows
// [16w, 16w + 16) of the 64-row query tile. Causal: query i of request b sits
// at position (L_b - q_len_b + i) and sees keys [0, position].
__global__ void __launch_bounds__(128, 2)
    prefill_attn_kernel(const __grid_constant__ CUtensorMap tm, AttnArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kStages * kStageBytes);
  const ErrorSink err{a.err};

  pdl_launch_dependents();
  pdl_wait();
  const int qt = blockIdx.x, qh = blockIdx.y, b = blockIdx.z;
  const int q_begin = a.cu_q[b];
  const int q_len = a.cu_q[b + 1] - q_begin;
  if (qt * 64 >= q_len) return;
  const int L = a.seq_lens[b];
  const int cached = L - q_len;
  const int G = a.hq / a.hk;
  const int h = qh / G;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  const int row0 = qt * 64;                       // first query row of this CTA
  const int last_pos = cached + min(q_len, row0 + 64) - 1;  // largest position in the tile
  const int ntiles = last_pos / kTile + 1;
  const int32_t* pt_row = a.page_table + static_cast<int64_t>(a.req_rows[b]) * a.ld_pt;
  if (a.pt_rows > 0 && (a.req_rows[b] < 0 || a.req_rows[b] >= a.pt_rows)) {  // uniform over the CTA
    if (threadIdx.x == 0) err.report(kErrBadIndex, 922);
    return;
  }

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) mbar_init(&bars[s], 1);
    fence_barrier_init();
    prefetch_tmap(&tm);
    for (int i = 0; i < kStages && i < ntiles; ++i)
      issue_kv_tile(smem + i * kStageBytes, &bars[i], &tm, a, pt_row, L, i * kTile, h);
  }
  __syncthreads();

  const int wrow0 = row0 + warp * 16;  // this warp's first query row
  const __nv_bfloat16* qb = reinterpret_cast<const __nv_bfloat16*>(a.q) +
                            static_cast<int64_t>(q_begin + wrow0) * a.ld_q + qh * kD;
  uint32_t qa[8][4];
  load_q_frags(qa, qb, a.ld_q, max(0, min(16, q_len - wrow0)), a.scale * kLog2e);
  const int pos_lo = cached + wrow0 + g;  // positions of rows g and g+8
  const int pos_hi = pos_lo + 8;

  float m_lo = -INFINITY, m_hi = -INFINITY, l_lo = 0.f, l_hi = 0.f;
  float o[16][4];
#pragma unroll
  for (int n = 0; n < 16; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;

  bool ok = true;
  const int warp_last = cached + min(q_len, wrow0 + 16) - 1;
  for (int i = 0; i < ntiles; ++i) {
    const int s = i % kStages;
    if (ok) ok = mbar_wait(&bars[s], (i / kStages) & 1u, err, 211);
    const uint32_t kbase = smem_u32(smem + s * kStageBytes);
    const uint32_t vbase = kbase + kTileBytes;
    const int kpos0 = i * kTile;
    if (wrow0 < q_len && kpos0 <= warp_last) {
      float sc[8][4];
#pragma unroll
      for (int nt = 0; nt < 8; ++nt) sc[nt][0] = sc[nt][1] = sc[nt][2] = sc[nt][3] = 0.f;
      const int mi = lane >> 3, rr = lane & 7;
#pragma unroll
      for (int ks = 0; ks < 8; ++ks) {
#pragma unroll
        for (int np = 0; np < 4; ++np) {  // pairs of 8-key n-tiles
          uint32_t b0, b1, b2, b3;
          ldsm_x4(kbase + tile_off(np * 16 + (mi >> 1) * 8 + rr, ks * 2 + (mi & 1)), b0, b1, b2, b3);
          mma_bf16(sc[2 * np], qa[ks], b0, b1);
          mma_bf16(sc[2 * np + 1], qa[ks], b2, b3);
        }
      }
      // causal + length mask
      if (kpos0 + kTile - 1 > pos_lo || kpos0 + kTile > L) {
#pragma unroll
        for (int nt = 0; nt < 8; ++nt) {
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int kp = kpos0 + nt * 8 + 2 * t + (e & 1);
            const int qp = (e & 2) ? pos_hi : pos_lo;
            if (kp > qp || kp >= L) sc[nt][e] = -INFINITY;
          }
        }
      }
      float mx_lo = -INFINITY, mx_hi = -INFINITY;
#pragma unroll
      for (int nt = 0; nt < 8; ++nt) {
        mx_lo = fmaxf(mx_lo, fmaxf(sc[nt][0], sc[nt][1]));
        mx_hi = fmaxf(mx_hi, fmaxf(sc[nt][2], sc[nt][3]));
      }
      mx_lo = fmaxf(mx_lo, __shfl_xor_sync(0xffffffffu, mx_lo, 1));
      mx_lo = fmaxf(mx_lo, __shfl_xor_sync(0xffffffffu, mx_lo, 2));
      mx_hi = fmaxf(mx_hi, __shfl_xor_sync(0xffffffffu, mx_hi, 1));
      mx_hi = fmaxf(mx_hi, __shfl_xor_sync(0xffffffffu, mx_hi, 2));
      const float new_lo = fmaxf(m_lo, mx_lo), new_hi = fmaxf(m_hi, mx_hi);
      const float base_lo = new_lo == -INFINITY ? 0.f : new_lo;
      const float base_hi = new_hi == -INFINITY ? 0.f : new_hi;
      const float alpha_lo = exp2f(m_lo - base_lo), alpha_hi = exp2f(m_hi - base_hi);
      m_lo = new_lo, m_hi = new_hi;
      float sum_lo = 0.f, sum_hi = 0.f;
      uint32_t pa[4][4];
#pragma unroll
      for (int nt = 0; nt < 8; ++nt) {
        const float p0 = exp2f(sc[nt][0] - base_lo), p1 = exp2f(sc[nt][1] - base_lo);
        const float p2 = exp2f(sc[nt][2] - base_hi), p3 = exp2f(sc[nt][3] - base_hi);
        sum_lo += p0 + p1;
        sum_hi += p2 + p3;
        // A fragment for k-step kk = nt / 2: (row g | g+8) x (keys 2t | 2t+8)
        pa[nt >> 1][(nt & 1) * 2 + 0] = pack_bf16x2(p0, p1);
        pa[nt >> 1][(nt & 1) * 2 + 1] = pack_bf16x2(p2, p3);
      }
      l_lo = l_lo * alpha_lo + sum_lo;
      l_hi = l_hi * alpha_hi + sum_hi;
#pragma unroll
      for (int n = 0; n < 16; ++n) {
        o[n][0] *= alpha_lo, o[n][1] *= alpha_lo;
        o[n][2] *= alpha_hi, o[n][3] *= alpha_hi;
      }
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
        const int tok = kk * 16 + (mi & 1) * 8 + rr;
#pragma unroll
        for (int nd = 0; nd < 16; nd += 2) {
          uint32_t b0, b1, b2, b3;
          ldsm_x4_t(vbase + tile_off(tok, nd + (mi >> 1)), b0, b1, b2, b3);
          mma_bf16(o[nd], pa[kk], b0, b1);
          mma_bf16(o[nd + 1], pa[kk], b2, b3);
        }
      }
    }
    __syncthreads();
    if (threadIdx.x == 0 && i + kStages < ntiles) {
      fence_proxy_async_smem();
      issue_kv_tile(smem + s * kStageBytes, &bars[s], &tm, a, pt_row, L, (i + kStages) * kTile, h);
    }
  }

  l_lo += __shfl_xor_sync(0xffffffffu, l_lo, 1);
  l_lo += __shfl_xor_sync(0xffffffffu, l_lo, 2);
  l_hi += __shfl_xor_sync(0xffffffffu, l_hi, 1);
  l_hi += __shfl_xor_sync(0xffffffffu, l_hi, 2);
  const float inv_lo = l_lo > 0.f ? 1.f / l_lo : 0.f;
  const float inv_hi = l_hi > 0.f ? 1.f / l_hi : 0.f;
  __nv_bfloat16* ob = reinterpret_cast<__nv_bfloat16*>(a.out);
  const int r_lo = wrow0 + g, r_hi = wrow0 + g + 8;
#pragma unroll
  for (int n = 0; n < 16; ++n) {
    const int col = n * 8 + 2 * t;
    if (r_lo < q_len)
      *reinterpret_cast<uint32_t*>(ob + (static_cast<int64_t>(q_begin + r_lo) * a.hq + qh) * kD + col) =
          pack_bf16x2(o[n][0] * inv_lo, o[n][1] * inv_lo);
    if (r_hi < q_len)
      *reinterpret_cast<uint32_t*>(ob + (static_cast<int64_t>(q_begin + r_hi) * a.hq + qh) * kD + col) =
          pack_bf16x2(o[n][2] * inv_hi, o[n][3] * inv_hi);
  }
}

// ================================================== prefill (tcgen05) ====
// grid (ceil(max_q / 128), hq, B); 320 threads. One CTA computes 128 query
// rows of one head (the MMA M) against the 64-key tiles of the same paged
// ring as above, with the products on the 5th-generation tensor cores:
//
//   S = Q . K^T   A = Q (K-major, two 64-dim chunks loaded once by TMA),
//                 B = K tile (K-major), M = 128, N = 64, K = 128
//   O += P . V    A = P in TMEM (bf16 pairs written by the softmax warps
//                 with tcgen05.st, two buffers), B = the V tile read
//                 MN-major, N = 128
//
// TMEM (512 columns, lane = query row): O in columns 0-127, the scores of
// tiles with j % 2 == 0 / 1 in columns 128-191 / 192-255, P of those tiles
// in columns 256-287 / 288-319. P never touches shared memory, which leaves
// its bandwidth to the TMA writes and the Q / K / V operand reads. Warps 0-7
// run the softmax (warps q and q + 4 share lane quadrant q, one half of each
// row's 64 keys per thread), warp 8 issues TMA (page ids read one tile
// ahead), warp 9 issues tcgen05.mma in whichever order their inputs arrive
// (QK(j) as soon as tile j and a free score buffer are there, PV(i) as soon
// as P_i is written).
// Softmax is in the exp2 domain with a lazy rescale: O and l are rescaled
// only when a row's running max grows by more than 8 (a factor of 256), so
// P stays below 256 in bf16 and most tiles never touch O.
constexpr int kTcRows = 128;                        // query rows per CTA
constexpr int kTcStages = 5;                        // K/V ring depth: copies start 4 tiles ahead
constexpr int kTcQChunk = kTcRows * 128;            // one 64-dim chunk of Q (16 KB)
constexpr int kTcSCol = 128;                        // first TMEM column of the score buffers
constexpr int kTcPCol = 256;                        // first TMEM column of the P buffers (32 each)
constexpr int kTcSoftmaxWarps = 8;                 // two per TMEM lane quadrant
constexpr int kTcProducer = kTcSoftmaxWarps, kTcIssuer = kTcSoftmaxWarps + 1;
constexpr int kTcThreads = 32 * (kTcSoftmaxWarps + 2);
constexpr int kTcRedBytes = 2 * 2 * kTcRows * 4;    // row-max exchange: [tile parity][half][row] fp32
constexpr int kTcSmem = 1024 + 2 * kTcQChunk + kTcStages * kStageBytes + 256 + kTcRedBytes;
static_assert(kTcSmem <= 227 * 1024, "prefill smem over the per-CTA limit");
// The rope variant (non-absorbed MLA prefill): a third 64-dim Q chunk (the
// rotated query rope part) and, per key tile, the keys' shared 64-dim rope
// rows next to K and V; one stage less to fit.
constexpr int kRopeTileBytes = kTile * 128;
constexpr int kTcRopeStages = kTcStages - 1;
constexpr int kTcRopeSmem = 1024 + 3 * kTcQChunk + kTcRopeStages * (kStageBytes + kRopeTileBytes) + 256 + kTcRedBytes;
static_assert(kTcRopeSmem <= 227 * 1024, "rope prefill smem over the per-CTA limit");
constexpr float kTcRescaleLog2 = 8.f;

// 2^x on the special-function unit (PTX ex2.approx.ftz: relative error of a
// few ulp, ex2(-inf) = +0).
__device__ __forceinline__ float ex2_fast(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Packed fp32 pairs (sm_100 f32x2 arithmetic: one instruction for two lanes
// of work) for the softmax inner loop.
__device__ __forceinline__ uint64_t f2_pack(float a, float b) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
  return r;
}
__device__ __forceinline__ void f2_unpack(uint64_t v, float& a, float& b) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(v));
}
__device__ __forceinline__ uint64_t f2_fma(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ uint64_t f2_add(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ float max3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

// 2^x for a pair of arguments on the FMA pipe, to take part of a softmax's
// exponentials off the special-function unit (which otherwise bounds it).
// Method: x = n + f with n = round(x) (adding and subtracting 1.5 * 2^23
// rounds to the nearest integer and leaves n in the low mantissa bits),
// f in [-1/2, 1/2]; 2^f by a cubic fitted here for minimal relative error
// on [-1/2, 1/2] (Lawson-weighted least squares; max relative error 7.5e-5,
// far below the 2^-8 of the bf16 P it feeds); 2^n added to the exponent
// field as n << 23. Arguments are clamped at -126 so that field stays in
// range: 2^-126 and below all come out as about 1e-38 instead of 0, which
// adds nothing measurable to a softmax whose largest term is at least 1.
__device__ __forceinline__ void exp2_poly_pair(uint64_t x2, float& y0, float& y1) {
  constexpr float kRound = 12582912.f;  // 1.5 * 2^23
  float x0, x1;
  f2_unpack(x2, x0, x1);
  x2 = f2_pack(fmaxf(x0, -126.f), fmaxf(x1, -126.f));
  const uint64_t t = f2_add(x2, f2_pack(kRound, kRound));
  const uint64_t r = f2_add(t, f2_pack(-kRound, -kRound));
  const uint64_t f = f2_fma(r, f2_pack(-1.f, -1.f), x2);
  uint64_t q = f2_fma(f, f2_pack(0.05517132f, 0.05517132f), f2_pack(0.24261054f, 0.24261054f));
  q = f2_fma(q, f, f2_pack(0.69326097f, 0.69326097f));
  q = f2_fma(q, f, f2_pack(0.99992812f, 0.99992812f));
  float q0, q1, t0, t1;
  f2_unpack(q, q0, q1);
  f2_unpack(t, t0, t1);
  y0 = __uint_as_float(__float_as_uint(q0) + (__float_as_uint(t0) << 23));
  y1 = __uint_as_float(__float_as_uint(q1) + (__float_as_uint(t1) << 23));
}

// kRope: the non-absorbed MLA prefill form. Scores are q_nope . k_nope (the
// two 64-dim chunks of the usual path, with q heads a.q_head_stride
// elements apart in a q row) plus q_rope . k_rope, the rotated 64-dim rope
// parts: the query's from its own [T, hq, 64] tensor (map tm_qr), the key's
// shared by every head and read per key tile from [slots, 64] rows at the
// same page-table slots as K and V (map tm_kr). V and the output keep 128
// dims.
template <bool kRope>
__global__ void __launch_bounds__(kTcThreads, 1)
    prefill_attn_tc_kernel(const __grid_constant__ CUtensorMap tm_kv, const __grid_constant__ CUtensorMap tm_q,
                           const __grid_constant__ CUtensorMap tm_qr, const __grid_constant__ CUtensorMap tm_kr,
                           AttnArgs a) {
  constexpr int kQC = kRope ? 3 : 2;                    // 64-dim Q chunks in shared memory
  constexpr int kSt = kRope ? kTcRopeStages : kTcStages;
  constexpr int kStage = kStageBytes + (kRope ? kRopeTileBytes : 0);
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint8_t* sQ = smem;
  uint8_t* sKV = sQ + kQC * kTcQChunk;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sKV + kSt * kStage);
  uint64_t* q_full = bars;
  uint64_t* kv_full = bars + 1;               // [kSt]
  uint64_t* kv_empty = kv_full + kSt;         // [kSt]
  uint64_t* s_full = kv_empty + kSt;          // [2] score buffers
  uint64_t* s_free = s_full + 2;              // [2]
  uint64_t* p_full = s_free + 2;              // [2] P of tiles with j % 2 == h written
  uint64_t* o_done = p_full + 2;              // [2] PV of tiles with j % 2 == h complete (P_h free)
  uint64_t* x_full = o_done + 2;              // [4 quadrants][2] partial row maxima written
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(x_full + 8);
  int* s_abort = reinterpret_cast<int*>(x_full + 9);
  float* red = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(bars) + 256);
  const ErrorSink err{a.err};
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  pdl_launch_dependents();
  pdl_wait();
  const int qt = static_cast<int>(gridDim.x) - 1 - static_cast<int>(blockIdx.x);  // longest key ranges first
  const int qh = blockIdx.y, b = blockIdx.z;
  const int q_begin = a.cu_q[b];
  const int q_len = a.cu_q[b + 1] - q_begin;
  const int row0 = qt * kTcRows;
  if (row0 >= q_len) return;  // uniform over the CTA, before any barrier or TMEM
  const int L = a.seq_lens[b];
  const int cached = L - q_len;
  const int h = qh / (a.hq / a.hk);
  const int n = (cached + min(q_len, row0 + kTcRows) - 1) / kTile + 1;  // key tiles up to the last row
  const int32_t* pt_row = a.page_table + static_cast<int64_t>(a.req_rows[b]) * a.ld_pt;
  if (a.pt_rows > 0 && (a.req_rows[b] < 0 || a.req_rows[b] >= a.pt_rows)) {  // uniform over the CTA
    if (threadIdx.x == 0) err.report(kErrBadIndex, 923);
    return;
  }
  unsigned long long* trace = (a.trace != nullptr && blockIdx.x == 0 && qh == 0 && b == 0) ? a.trace : nullptr;
  auto stamp = [&](int i, int slot) {
    if (trace != nullptr && i < 64) trace[i * 8 + slot] = globaltimer_ns();
  };

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < kSt; ++i) {
      mbar_init(&kv_full[i], 1);
      mbar_init(&kv_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&s_free[i], kTcSoftmaxWarps);
      mbar_init(&p_full[i], kTcSoftmaxWarps);
      mbar_init(&o_done[i], 1);
    }
    for (int i = 0; i < 8; ++i) mbar_init(&x_full[i], 2);
    *s_abort = 0;
    fence_barrier_init();
    prefetch_tmap(&tm_kv);
    prefetch_tmap(&tm_q);
    if (kRope) {
      prefetch_tmap(&tm_qr);
      prefetch_tmap(&tm_kr);
    }
  }
  if (warp == kTcIssuer) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  int issued = 0;  // key tiles whose copies the producer started

  if (warp == kTcProducer) {
    // ------------------------------------------------------------ TMA ----
    if (lane == 0) {
      mbar_arrive_expect_tx(q_full, kQC * kTcQChunk);
      // rows past the last query token read the next request's rows (or the
      // zero fill past the end); their results are never stored
      const int qx = qh * (a.q_head_stride > 0 ? a.q_head_stride : kD);
      tma_load_2d(sQ, &tm_q, q_full, qx, q_begin + row0);
      tma_load_2d(sQ + kTcQChunk, &tm_q, q_full, qx + 64, q_begin + row0);
      if (kRope) tma_load_2d(sQ + 2 * kTcQChunk, &tm_qr, q_full, qh * 64, q_begin + row0);
      // page ids of tile j + 1 are read while tile j waits for its stage, so
      // no copy waits on a page-table load
      const int P = a.page_size;
      const int seg = P < kTile ? P : kTile;
      int cur[kTile / 16], nxt[kTile / 16];
      auto read_pages = [&](int (&pg)[kTile / 16], int j) {
#pragma unroll
        for (int q = 0; q < kTile / 16; ++q) {
          const int pos = j * kTile + q * seg;
          pg[q] = (q * seg < kTile && pos < L) ? pt_row[pos] / P : 0;  // past the end: page 0, masked later
        }
      };
      read_pages(cur, 0);
      for (int j = 0; j < n; ++j) {
        const int s = j % kSt;
        read_pages(nxt, j + 1);
        if (j >= kSt && !mbar_wait(&kv_empty[s], ((j / kSt) - 1) & 1, err, 231)) {
          atomicExch(s_abort, 1);
          break;
        }
        if (*reinterpret_cast<volatile int*>(s_abort)) break;
        ++issued;
        stamp(j, 0);
        uint8_t* st = sKV + s * kStage;
        mbar_arrive_expect_tx(&kv_full[s], kStage);
        const int64_t in_page = P < kTile ? 0 : (j * kTile) % P;
#pragma unroll
        for (int q = 0; q < kTile / 16; ++q) {
          if (q * seg >= kTile) break;
          const int64_t row = (static_cast<int64_t>(cur[q]) * a.hk + h) * P + in_page;
          const int32_t rk = static_cast<int32_t>(a.k_row0 + row);
          const int32_t rv = static_cast<int32_t>(a.v_row0 + row);
          const int o = q * seg * 128;
          tma_load_2d(st + o, &tm_kv, &kv_full[s], 0, rk);
          tma_load_2d(st + kHalfBytes + o, &tm_kv, &kv_full[s], 64, rk);
          tma_load_2d(st + kTileBytes + o, &tm_kv, &kv_full[s], 0, rv);
          tma_load_2d(st + kTileBytes + kHalfBytes + o, &tm_kv, &kv_full[s], 64, rv);
          if (kRope)  // the keys' rope rows: one 64-dim row per slot
            tma_load_2d(st + kStageBytes + o, &tm_kr, &kv_full[s], 0,
                        static_cast<int32_t>(static_cast<int64_t>(cur[q]) * P + in_page));
        }
#pragma unroll
        for (int q = 0; q < kTile / 16; ++q) cur[q] = nxt[q];
      }
    }
    __syncwarp();
  } else if (warp == kTcIssuer) {
    // ------------------------------------------------------------ MMA ----
    constexpr uint32_t idesc_qk = make_idesc_bf16(kTcRows, kTile);
    constexpr uint32_t idesc_pv = make_idesc_bf16(kTcRows, kD, false, true);
    const uint32_t q_addr = smem_u32(sQ), kv_addr = smem_u32(sKV);
    bool ok = __all_sync(0xffffffffu, mbar_wait(q_full, 0, err, 232));
    auto qk = [&](int j) {  // S[j % 2] = Q . K_j^T
      const uint32_t st = kv_addr + (j % kSt) * kStage;
      const uint32_t d = tmem + kTcSCol + (j % 2) * kTile;
#pragma unroll
      for (int c = 0; c < 2; ++c)
#pragma unroll
        for (int k = 0; k < 4; ++k)
          tc_mma_f16(d, make_sdesc_k_sw128(q_addr + c * kTcQChunk + k * 32),
                     make_sdesc_k_sw128(st + c * kHalfBytes + k * 32), idesc_qk, (c | k) != 0 ? 1u : 0u);
      if (kRope) {  // + q_rope . k_rope
#pragma unroll
        for (int k = 0; k < 4; ++k)
          tc_mma_f16(d, make_sdesc_k_sw128(q_addr + 2 * kTcQChunk + k * 32),
                     make_sdesc_k_sw128(st + kStageBytes + k * 32), idesc_qk, 1u);
      }
      tc_commit(&s_full[j % 2]);
    };
    auto pv = [&](int i) {  // O += P_i . V_i
      const uint32_t v = kv_addr + (i % kSt) * kStage + kTileBytes;
#pragma unroll
      for (int kk = 0; kk < kTile / 16; ++kk)  // 16 keys = 8 TMEM columns of P per MMA
        tc_mma_f16_ta(tmem, tmem + kTcPCol + (i % 2) * (kTile / 2) + kk * 8,
                      make_sdesc_mn_sw128(v + kk * 2048, kHalfBytes), idesc_pv, (i > 0 || kk > 0) ? 1u : 0u);
      tc_commit(&kv_empty[i % kSt]);
      tc_commit(&o_done[i % 2]);
    };
    int qn = 0, pn = 0;  // next QK, next PV
    uint64_t t0 = globaltimer_ns();
    uint32_t spins = 0;
    while (ok && pn < n) {
      // lane 0 polls and decides; the warp follows its choice
      // QK first, tested without suspending: a try_wait on P_pn would sleep
      // until the softmax of tile pn ends, and QK(pn + 1) would then start
      // only after PV(pn), leaving the softmax of tile pn + 1 without scores
      int choice = 0;
      if (lane == 0) {
        if (qn < n && qn <= pn + 1 && mbar_test_wait(&kv_full[qn % kSt], (qn / kSt) & 1) &&
            (qn < 2 || mbar_test_wait(&s_free[qn % 2], ((qn / 2) - 1) & 1)))
          choice = 2;
        else if (pn < qn && mbar_try_wait(&p_full[pn % 2], (pn / 2) & 1)) choice = 1;
        else if (*reinterpret_cast<volatile int*>(s_abort) ||
                 (((++spins) & 0xFFu) == 0 && globaltimer_ns() - t0 > kWaitBudgetNs))
          choice = 3;
      }
      choice = __shfl_sync(0xffffffffu, choice, 0);
      if (choice == 3) {
        if (lane == 0 && !*reinterpret_cast<volatile int*>(s_abort)) err.report(kErrMbarTimeout, 236);
        ok = false;
      } else if (choice != 0) {
        tc_fence_after();
        if (lane == 0) {
          if (choice == 1) {
            pv(pn);
            stamp(pn, 6);
          } else {
            qk(qn);
            stamp(qn, 1);
          }
        }
        if (choice == 1) ++pn;
        else ++qn;
        __syncwarp();
        if (lane == 0) {
          t0 = globaltimer_ns();
          spins = 0;
        }
      }
    }
    if (!ok && lane == 0) atomicExch(s_abort, 1);
    __syncwarp();
  } else {
    // -------------------------------------------------------- softmax ----
    // warps q and q + 4 share TMEM lane quadrant q: thread (half, r) owns key
    // columns 32 half.. of row r, and output dims 64 half.. of that row. The
    // two halves swap partial row maxima through shared memory each tile
    // (x_full: one arrival per warp, bounded wait), so both apply the same
    // running max; their partial sums are added once at the end.
    const int quad = warp & 3, half = warp >> 2;
    const int r = 32 * quad + lane;  // this thread's query row (TMEM lane)
    const uint32_t lane_base = tmem + (static_cast<uint32_t>(32 * quad) << 16);
    const float sl2 = a.scale * kLog2e;
    const int pos = cached + row0 + r;  // position of this row's query token
    constexpr int kCols = kTile / 2;    // key columns per thread
    float m_run = -INFINITY, l_sum = 0.f;
    bool ok = true;
    auto exchange = [&](float v, int i, int where, float& other) {  // swap v with the other half of row r
      red[((i & 1) * 2 + half) * kTcRows + r] = v;
      __syncwarp();
      if (lane == 0) mbar_arrive(&x_full[quad * 2 + (i & 1)]);
      const bool got = __all_sync(0xffffffffu, mbar_wait(&x_full[quad * 2 + (i & 1)], (i >> 1) & 1, err, where));
      other = red[((i & 1) * 2 + (half ^ 1)) * kTcRows + r];
      return got;
    };
    for (int i = 0; i < n; ++i) {
      const int bf = i % 2;
      ok = __all_sync(0xffffffffu, mbar_wait(&s_full[bf], (i / 2) & 1, err, 233));
      if (!ok) break;
      const bool tr = warp == 0 && lane == 0;
      if (tr) stamp(i, 2);
      tc_fence_after();
      uint32_t sv[kCols];
      tmem_ld_32x32b_x32(lane_base + kTcSCol + bf * kTile + half * kCols, sv);
      tc_wait_ld();
      if (tr) stamp(i, 7);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&s_free[bf]);
      // causal and length mask: keys [0, lim) of this thread's columns are visible
      const int lim = min(pos + 1, L) - i * kTile - half * kCols;
      if (lim < kCols) {
#pragma unroll
        for (int j = 0; j < kCols; ++j)
          if (j >= lim) sv[j] = __float_as_uint(-INFINITY);
      }
      float m4[4];  // four independent chains
#pragma unroll
      for (int c = 0; c < 4; ++c) m4[c] = __uint_as_float(sv[c]);
#pragma unroll
      for (int j = 4; j < kCols; ++j) m4[j & 3] = fmaxf(m4[j & 3], __uint_as_float(sv[j]));
      float other;
      ok = exchange(fmaxf(fmaxf(m4[0], m4[1]), fmaxf(m4[2], m4[3])), i, 240, other);
      if (!ok) break;
      const float mt = fmaxf(fmaxf(fmaxf(m4[0], m4[1]), fmaxf(m4[2], m4[3])), other) * sl2;
      const bool grow = mt > m_run + kTcRescaleLog2;  // the same decision in both halves
      float alpha = 1.f;
      if (grow) {
        alpha = ex2_fast(m_run - mt);  // 0 on the first tile (m_run = -inf)
        l_sum *= alpha;
        m_run = mt;
      }
      const bool any_grow = __any_sync(0xffffffffu, grow) && i > 0;
      // P = 2^(s * scale * log2 e - m) as bf16 pairs
      uint32_t pk[kCols / 2];
      float ps[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int e = 0; e < kCols / 2; ++e) {
        const float lo = ex2_fast(fmaf(__uint_as_float(sv[2 * e]), sl2, -m_run));
        const float hi = ex2_fast(fmaf(__uint_as_float(sv[2 * e + 1]), sl2, -m_run));
        ps[e & 3] += lo + hi;
        pk[e] = pack_bf16x2(lo, hi);
      }
      l_sum += (ps[0] + ps[1]) + (ps[2] + ps[3]);
      if (tr) stamp(i, 3);
      // P buffer i % 2 was last read by PV(i - 2)
      if (i >= 2) {
        ok = __all_sync(0xffffffffu, mbar_wait(&o_done[bf], ((i - 2) / 2) & 1, err, 234));
        if (!ok) break;
      }
      if (tr) stamp(i, 4);
      if (any_grow) {  // rescale O once PV(i - 1) is complete
        ok = __all_sync(0xffffffffu, mbar_wait(&o_done[(i - 1) % 2], ((i - 1) / 2) & 1, err, 235));
        if (!ok) break;
        tc_fence_after();
#pragma unroll 1
        for (int c = 0; c < 2; ++c) {
          uint32_t ov[32];
          const uint32_t col = lane_base + half * 64 + c * 32;
          tmem_ld_32x32b_x32(col, ov);
          tc_wait_ld();
#pragma unroll
          for (int j = 0; j < 32; ++j) ov[j] = __float_as_uint(__uint_as_float(ov[j]) * alpha);
          tmem_st_32x32b_x32(col, ov);
        }
      }
      // keys 32 half.. of row r of P: 16 TMEM columns of bf16 pairs
      tmem_st_32x32b_x16(lane_base + kTcPCol + bf * (kTile / 2) + half * (kCols / 2), pk);
      tc_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_full[bf]);
      if (tr) stamp(i, 5);
    }
    // ------------------------------------------------------- epilogue ----
    if (!ok && lane == 0) atomicExch(s_abort, 1);
    float l_other = 0.f;
    if (ok) ok = exchange(l_sum, n, 241, l_other);
    if (ok) ok = __all_sync(0xffffffffu, mbar_wait(&o_done[(n - 1) % 2], ((n - 1) / 2) & 1, err, 237));
    tc_fence_after();
    const float l_row = l_sum + l_other;
    const float inv = ok && l_row > 0.f ? 1.f / l_row : 0.f;
    const bool store = row0 + r < q_len;
    __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(a.out) +
                         (static_cast<int64_t>(q_begin + row0 + r) * a.hq + qh) * kD + half * 64;
#pragma unroll 1
    for (int c = 0; c < 2; ++c) {
      uint32_t ov[32];
      if (ok) {
        tmem_ld_32x32b_x32(lane_base + half * 64 + c * 32, ov);
        tc_wait_ld();
      } else {
#pragma unroll
        for (int j = 0; j < 32; ++j) ov[j] = 0u;
      }
      if (!store) continue;
#pragma unroll
      for (int q4 = 0; q4 < 4; ++q4) {
        uint4 v;
        v.x = pack_bf16x2(__uint_as_float(ov[q4 * 8 + 0]) * inv, __uint_as_float(ov[q4 * 8 + 1]) * inv);
        v.y = pack_bf16x2(__uint_as_float(ov[q4 * 8 + 2]) * inv, __uint_as_float(ov[q4 * 8 + 3]) * inv);
        v.z = pack_bf16x2(__uint_as_float(ov[q4 * 8 + 4]) * inv, __uint_as_float(ov[q4 * 8 + 5]) * inv);
        v.w = pack_bf16x2(__uint_as_float(ov[q4 * 8 + 6]) * inv, __uint_as_float(ov[q4 * 8 + 7]) * inv);
        *reinterpret_cast<uint4*>(dst + c * 32 + q4 * 8) = v;
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == kTcProducer && lane == 0 && *reinterpret_cast<volatile int*>(s_abort)) {
    // after an abort, let the copies still in flight land before the CTA
    // leaves (bounded waits; the normal path never gets here)
    mbar_wait(q_full, 0, err, 238);
    for (int j = max(0, issued - kSt); j < issued; ++j)
      mbar_wait(&kv_full[j % kSt], (j / kSt) & 1, err, 239);
  }
  if (warp == kTcIssuer) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// ------------------------------------------------------ head-pair prefill ----
// Two query heads of one KV group per CTA (128 query rows each), sharing every
// K/V tile. Tensor memory: O of head h at columns [128 h, +128), scores S_h at
// [256 + 64 h, +64) with P_h (bf16 pairs) written over the first 32 of them.
// Both heads' Q tiles (64 KB) sit in shared memory, loaded once by TMA, as
// the A operand of Q.K^T (with A in tensor memory the MMA thread took twice
// as long to issue each Q.K^T MMA). The MMA thread ping-pongs the heads,
//   QK0(0) QK1(0) | PV0(i) QK0(i+1) PV1(i) QK1(i+1) | ...,
// so the softmax of one head runs while the tensor core works on the other.
// tcgen05 operations of one thread complete in order, which is what makes
// the single S/P buffer per head safe: QK_h(i+1) is issued after PV_h(i), and
// S_h(i+1) being ready implies PV_h(i) finished (the softmax may rescale O_h
// then without another wait). Warps 0-3 own the rows of head 0 and warps 4-7
// those of head 1 (one row per thread, the whole 64-key tile), so no row
// statistics cross warps.
constexpr int kPrStages = 5;
constexpr int kPrSCol = 256;
constexpr int kPrProducer = 8, kPrIssuer = 9;
constexpr int kPrThreads = 32 * 10;
constexpr int kPrPolyPairs = 3;  // of every 8 exponent pairs, computed on the FMA pipe
constexpr int kPrSmem = 1024 + 4 * kTcQChunk + kPrStages * kStageBytes + 256;
static_assert(kPrSmem <= 227 * 1024, "head-pair prefill smem over the per-CTA limit");

__global__ void __launch_bounds__(kPrThreads, 1)
    prefill_attn_pair_kernel(const __grid_constant__ CUtensorMap tm_kv, const __grid_constant__ CUtensorMap tm_q,
                             AttnArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint8_t* sQ = smem;                        // [head][64-dim chunk] of 128 rows x 128 B
  uint8_t* sKV = sQ + 4 * kTcQChunk;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sKV + kPrStages * kStageBytes);
  uint64_t* kv_full = bars;                  // [kPrStages]
  uint64_t* kv_empty = kv_full + kPrStages;  // [kPrStages]
  uint64_t* s_full = kv_empty + kPrStages;   // [2 heads]
  uint64_t* p_full = s_full + 2;             // [2 heads]
  uint64_t* o_done = p_full + 2;             // [2 heads]
  uint64_t* q_ready = o_done + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(q_ready + 1);
  int* s_abort = reinterpret_cast<int*>(tmem_slot + 1);
  const ErrorSink err{a.err};
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  pdl_launch_dependents();
  pdl_wait();
  const int qt = static_cast<int>(gridDim.x) - 1 - static_cast<int>(blockIdx.x);  // longest key ranges first
  const int qh0 = 2 * static_cast<int>(blockIdx.y), b = blockIdx.z;
  const int q_begin = a.cu_q[b];
  const int q_len = a.cu_q[b + 1] - q_begin;
  const int row0 = qt * kTcRows;
  if (row0 >= q_len) return;  // uniform over the CTA, before any barrier or TMEM
  const int L = a.seq_lens[b];
  const int cached = L - q_len;
  const int h = qh0 / (a.hq / a.hk);  // both heads of the pair share this KV head
  const int n = (cached + min(q_len, row0 + kTcRows) - 1) / kTile + 1;
  const int32_t* pt_row = a.page_table + static_cast<int64_t>(a.req_rows[b]) * a.ld_pt;
  if (a.pt_rows > 0 && (a.req_rows[b] < 0 || a.req_rows[b] >= a.pt_rows)) {  // uniform over the CTA
    if (threadIdx.x == 0) err.report(kErrBadIndex, 924);
    return;
  }
  // optional per-tile phase stamps of CTA (0, 0, 0) (the longest key range
  // of request 0's first head pair), 8 slots a tile: 0 scores seen by head
  // 0 (warp 0), 1-4 P handed over by head 0's warps 0-3, 5 the MMA thread
  // saw P of head 0, 6 PV of head 0 issued, 7 QK of head 0's next tile issued
  unsigned long long* trace = (a.trace != nullptr && blockIdx.x == 0 && blockIdx.y == 0 && b == 0) ? a.trace : nullptr;
  auto stamp = [&](int i, int slot) {
    if (trace != nullptr && i < 64) trace[i * 8 + slot] = globaltimer_ns();
  };

  if (threadIdx.x == 0) {
    for (int i = 0; i < kPrStages; ++i) {
      mbar_init(&kv_full[i], 1);
      mbar_init(&kv_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&p_full[i], 4);
      mbar_init(&o_done[i], 1);
    }
    mbar_init(q_ready, 1);
    *s_abort = 0;
    fence_barrier_init();
    prefetch_tmap(&tm_kv);
    prefetch_tmap(&tm_q);
  }
  if (warp == kPrIssuer) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  int issued = 0;  // key tiles whose copies the producer started

  if (warp == kPrProducer) {
    // ------------------------------------------------------------ TMA ----
    if (lane == 0) {
      // both heads' Q tiles; rows past the last query token read the next
      // request's rows (or the zero fill past the end), never stored
      mbar_arrive_expect_tx(q_ready, 4 * kTcQChunk);
#pragma unroll
      for (int hh = 0; hh < 2; ++hh)
#pragma unroll
        for (int c = 0; c < 2; ++c)
          tma_load_2d(sQ + (2 * hh + c) * kTcQChunk, &tm_q, q_ready, (qh0 + hh) * kD + 64 * c, q_begin + row0);
      const int P = a.page_size;
      const int seg = P < kTile ? P : kTile;
      int cur[kTile / 16], nxt[kTile / 16];
      auto read_pages = [&](int (&pg)[kTile / 16], int j) {
#pragma unroll
        for (int q = 0; q < kTile / 16; ++q) {
          const int pos = j * kTile + q * seg;
          pg[q] = (q * seg < kTile && pos < L) ? pt_row[pos] / P : 0;  // past the end: page 0, masked later
        }
      };
      read_pages(cur, 0);
      for (int j = 0; j < n; ++j) {
        const int s = j % kPrStages;
        read_pages(nxt, j + 1);
        if (j >= kPrStages && !mbar_wait(&kv_empty[s], ((j / kPrStages) - 1) & 1, err, 251)) {
          atomicExch(s_abort, 1);
          break;
        }
        if (*reinterpret_cast<volatile int*>(s_abort)) break;
        ++issued;
        uint8_t* st = sKV + s * kStageBytes;
        mbar_arrive_expect_tx(&kv_full[s], kStageBytes);
        const int64_t in_page = P < kTile ? 0 : (j * kTile) % P;
#pragma unroll
        for (int q = 0; q < kTile / 16; ++q) {
          if (q * seg >= kTile) break;
          const int64_t row = (static_cast<int64_t>(cur[q]) * a.hk + h) * P + in_page;
          const int32_t rk = static_cast<int32_t>(a.k_row0 + row);
          const int32_t rv = static_cast<int32_t>(a.v_row0 + row);
          const int o = q * seg * 128;
          tma_load_2d(st + o, &tm_kv, &kv_full[s], 0, rk);
          tma_load_2d(st + kHalfBytes + o, &tm_kv, &kv_full[s], 64, rk);
          tma_load_2d(st + kTileBytes + o, &tm_kv, &kv_full[s], 0, rv);
          tma_load_2d(st + kTileBytes + kHalfBytes + o, &tm_kv, &kv_full[s], 64, rv);
        }
#pragma unroll
        for (int q = 0; q < kTile / 16; ++q) cur[q] = nxt[q];
      }
    }
    __syncwarp();
  } else if (warp == kPrIssuer) {
    // ------------------------------------------------------------ MMA ----
    // (one MMA warp per head was measured slower: 2.2 vs 1.7 us per tile,
    // the second warp's issue competing with the softmax warps)
    constexpr uint32_t idesc_qk = make_idesc_bf16(kTcRows, kTile);
    constexpr uint32_t idesc_pv = make_idesc_bf16(kTcRows, kD, false, true);
    // descriptors of stage 0; a stage, head, half or k-step moves only the
    // start address field (bytes >> 4, well inside its 14 bits), so each MMA
    // adds a constant to a warp-uniform base instead of rebuilding one
    const uint32_t kv_addr = smem_u32(sKV);
    const uint64_t k_desc0 = make_sdesc_k_sw128(kv_addr);
    const uint64_t v_desc0 = make_sdesc_mn_sw128(kv_addr + kTileBytes, kHalfBytes);
    const uint64_t q_desc0 = make_sdesc_k_sw128(smem_u32(sQ));
    const uint32_t tm = __shfl_sync(0xffffffffu, tmem, 0);  // warp-uniform for the MMA operands
    auto qk = [&](int hh, int j) {  // S_hh = Q_hh . K_j^T
      const uint64_t st = k_desc0 + static_cast<uint64_t>((j % kPrStages) * (kStageBytes >> 4));
#pragma unroll
      for (int c = 0; c < 2; ++c)
#pragma unroll
        for (int k = 0; k < 4; ++k)
          tc_mma_f16(tm + kPrSCol + 64 * hh, q_desc0 + static_cast<uint64_t>(((2 * hh + c) * kTcQChunk + k * 32) >> 4),
                     st + static_cast<uint64_t>((c * kHalfBytes + k * 32) >> 4), idesc_qk, (c | k) != 0 ? 1u : 0u);
      tc_commit(&s_full[hh]);
    };
    auto pv = [&](int hh, int i) {  // O_hh += P_hh . V_i
      const uint64_t v = v_desc0 + static_cast<uint64_t>((i % kPrStages) * (kStageBytes >> 4));
#pragma unroll
      for (int kk = 0; kk < kTile / 16; ++kk)  // 16 keys = 8 TMEM columns of P per MMA
        tc_mma_f16_ta(tm + 128 * hh, tm + kPrSCol + 64 * hh + kk * 8, v + static_cast<uint64_t>(kk * (2048 >> 4)),
                      idesc_pv, (i > 0 || kk > 0) ? 1u : 0u);
      tc_commit(&o_done[hh]);
    };
    // every wait of this warp is bounded; lane 0 polls alone and the warp
    // follows its result
    auto wait = [&](uint64_t* bar, uint32_t parity, int where) {  // uniform over the warp
      int ok = 1;
      if (lane == 0) ok = mbar_wait(bar, parity, err, where) && !*reinterpret_cast<volatile int*>(s_abort);
      return __shfl_sync(0xffffffffu, ok, 0) != 0;
    };
    bool ok = wait(q_ready, 0, 252) && wait(&kv_full[0], 0, 253);
    tc_fence_after();
    if (ok && lane == 0) {
      qk(0, 0);
      qk(1, 0);
    }
    __syncwarp();
    for (int i = 0; ok && i < n; ++i) {
      const bool more = i + 1 < n;
      ok = wait(&p_full[0], i & 1, 254);
      if (!ok) break;
      if (lane == 0) stamp(i, 5);
      tc_fence_after();
      if (lane == 0) pv(0, i);
      if (lane == 0) stamp(i, 6);
      __syncwarp();
      if (more) {
        ok = wait(&kv_full[(i + 1) % kPrStages], ((i + 1) / kPrStages) & 1, 255);
        if (!ok) break;
        tc_fence_after();
        if (lane == 0) qk(0, i + 1);
        if (lane == 0) stamp(i, 7);
        __syncwarp();
      }
      ok = wait(&p_full[1], i & 1, 256);
      if (!ok) break;
      tc_fence_after();
      if (lane == 0) {
        pv(1, i);
        tc_commit(&kv_empty[i % kPrStages]);  // both heads have read tile i
        if (more) qk(1, i + 1);
      }
      __syncwarp();
    }
    if (!ok && lane == 0) atomicExch(s_abort, 1);
    __syncwarp();
  } else {
    // -------------------------------------------------------- softmax ----
    const int hh = warp >> 2, quad = warp & 3;
    const int r = 32 * quad + lane;  // this thread's query row (TMEM lane)
    const uint32_t lane_base = tmem + (static_cast<uint32_t>(32 * quad) << 16);
    const bool row_valid = row0 + r < q_len;
    const int64_t tok = q_begin + row0 + (row_valid ? r : 0);
    const float sl2 = a.scale * kLog2e;
    const int pos = cached + row0 + r;  // position of this row's query token
    const uint32_t s_col = lane_base + kPrSCol + 64 * hh;
    const uint32_t o_col = lane_base + 128 * hh;
    float m_run = -INFINITY, l_sum = 0.f;
    bool ok = true;
    for (int i = 0; i < n; ++i) {
      ok = __all_sync(0xffffffffu, mbar_wait(&s_full[hh], i & 1, err, 257) &&
                                       !*reinterpret_cast<volatile int*>(s_abort));  // uniform over the warp
      if (!ok) break;
      if (lane == 0 && quad == 0 && hh == 0) stamp(i, 0);
      tc_fence_after();
      uint32_t sv[kTile];
      tmem_ld_32x32b_x32(s_col, *reinterpret_cast<uint32_t(*)[32]>(sv));
      tmem_ld_32x32b_x32(s_col + 32, *reinterpret_cast<uint32_t(*)[32]>(sv + 32));
      tc_wait_ld();
      // causal and length mask: keys [0, lim) of the tile are visible to this row
      const int lim = min(pos + 1, L) - i * kTile;
      if (lim < kTile) {
#pragma unroll
        for (int j = 0; j < kTile; ++j)
          if (j >= lim) sv[j] = __float_as_uint(-INFINITY);
      }
      // row max: four independent chains of 3-input max
      float m4[4];
#pragma unroll
      for (int c = 0; c < 4; ++c) m4[c] = fmaxf(__uint_as_float(sv[2 * c]), __uint_as_float(sv[2 * c + 1]));
#pragma unroll
      for (int j = 8; j < kTile; j += 8) {
#pragma unroll
        for (int c = 0; c < 4; ++c)
          m4[c] = max3(m4[c], __uint_as_float(sv[j + 2 * c]), __uint_as_float(sv[j + 2 * c + 1]));
      }
      static_assert(kTile % 8 == 0, "row max reads the tile in groups of 8");
      const float mt = max3(m4[0], m4[1], fmaxf(m4[2], m4[3])) * sl2;
      // lazy rescale: the running max moves only when it grows by more than
      // 2^kTcRescaleLog2, so P stays below that bound in bf16
      const bool grow = mt > m_run + kTcRescaleLog2;
      float alpha = 1.f;
      if (grow) {
        alpha = ex2_fast(m_run - mt);  // 0 on the first tile (m_run = -inf)
        l_sum *= alpha;
        m_run = mt;
      }
      // tcgen05.ld / st are warp-collective: the whole warp rescales when any
      // of its rows grew (the others multiply by 1). O_hh holds PV_hh(0 .. i-1)
      // complete: S_hh(i) was committed after them.
      if (__any_sync(0xffffffffu, grow) && i > 0) {
#pragma unroll 1
        for (int c = 0; c < 4; ++c) {
          uint32_t ov[32];
          tmem_ld_32x32b_x32(o_col + 32 * c, ov);
          tc_wait_ld();
#pragma unroll
          for (int j = 0; j < 32; ++j) ov[j] = __float_as_uint(__uint_as_float(ov[j]) * alpha);
          tmem_st_32x32b_x32(o_col + 32 * c, ov);
        }
      }
      // P = 2^(s * scale * log2 e - m) as bf16 pairs over the first 32 score
      // columns; arguments and sums in packed pairs, and 3 pairs in 8 take
      // the FMA-pipe exponential so the special-function unit is not the
      // bound of the loop
      uint32_t pk[kTile / 2];
      const uint64_t sl2x2 = f2_pack(sl2, sl2), negm = f2_pack(-m_run, -m_run);
      uint64_t ps2[2] = {f2_pack(0.f, 0.f), f2_pack(0.f, 0.f)};
#pragma unroll
      for (int e = 0; e < kTile / 2; ++e) {
        const uint64_t x2 = f2_fma(f2_pack(__uint_as_float(sv[2 * e]), __uint_as_float(sv[2 * e + 1])), sl2x2, negm);
        float lo, hi;
        if (kPrPolyPairs > 0 && (e % 8) < kPrPolyPairs) {
          exp2_poly_pair(x2, lo, hi);
        } else {
          float x0, x1;
          f2_unpack(x2, x0, x1);
          lo = ex2_fast(x0);
          hi = ex2_fast(x1);
        }
        ps2[e & 1] = f2_add(ps2[e & 1], f2_pack(lo, hi));
        pk[e] = pack_bf16x2(lo, hi);
      }
      {
        float a0, a1;
        f2_unpack(f2_add(ps2[0], ps2[1]), a0, a1);
        l_sum += a0 + a1;
      }
      tmem_st_32x32b_x32(s_col, pk);
      tc_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_full[hh]);
      if (lane == 0 && hh == 0) stamp(i, 1 + quad);
    }
    // ------------------------------------------------------- epilogue ----
    if (!ok && lane == 0) atomicExch(s_abort, 1);
    if (ok) ok = __all_sync(0xffffffffu, mbar_wait(&o_done[hh], (n - 1) & 1, err, 258));
    tc_fence_after();
    const float inv = ok && l_sum > 0.f ? 1.f / l_sum : 0.f;
    __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(a.out) + (tok * a.hq + qh0 + hh) * kD;
#pragma unroll 1
    for (int c = 0; c < 4; ++c) {
      uint32_t ov[32];
      if (ok) {
        tmem_ld_32x32b_x32(o_col + 32 * c, ov);
        tc_wait_ld();
      } else {
#pragma unroll
        for (int j = 0; j < 32; ++j) ov[j] = 0u;
      }
      if (!row_valid) continue;
#pragma unroll
      for (int q4 = 0; q4 < 4; ++q4) {
        uint4 v;
        v.x = pack_bf16x2(__uint_as_float(ov[q4 * 8 + 0]) * inv, __uint_as_float(ov[q4 * 8 + 1]) * inv);
        v.y = pack_bf16x2(__uint_as_float(ov[q4 * 8 + 2]) * inv, __uint_as_float(ov[q4 * 8 + 3]) * inv);
        v.z = pack_bf16x2(__uint_as_float(ov[q4 * 8 + 4]) * inv, __uint_as_float(ov[q4 * 8 + 5]) * inv);
        v.w = pack_bf16x2(__uint_as_float(ov[q4 * 8 + 6]) * inv, __uint_as_float(ov[q4 * 8 + 7]) * inv);
        *reinterpret_cast<uint4*>(dst + c * 32 + q4 * 8) = v;
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == kPrProducer && lane == 0 && *reinterpret_cast<volatile int*>(s_abort)) {
    // after an abort, let the copies still in flight land before the CTA leaves
    mbar_wait(q_ready, 0, err, 260);
    for (int j = max(0, issued - kPrStages); j < issued; ++j)
      mbar_wait(&kv_full[j % kPrStages], (j / kPrStages) & 1, err, 259);
  }
  if (warp == kPrIssuer) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

constexpr int kAttnSmem = kStages * kStageBytes + 1024 + 128;
static_assert(kConsumers * 16 * kMergeLd * 4 + 2 * kConsumers * 16 * 4 <= kStages * kStageBytes,
              "merge buffer must fit in the ring");

CUtensorMap pool_map(const AttnArgs& a) {
  const uint32_t box_rows = a.page_size < kTile ? a.page_size : kTile;
  return make_tmap_bf16_2d_sw128(a.kv_pool, a.pool_rows, a.d, a.d, box_rows);
}

void check_args(const AttnArgs& a) {
  if (a.d != kD) throw std::runtime_error("minisgl.attention: head_dim must be 128");
  if (a.hq % a.hk != 0 || a.hq / a.hk > 16)
    throw std::runtime_error("minisgl.attention: need hq % hk == 0 and a GQA group of at most 16");
  if (a.page_size < 16 || (a.page_size & (a.page_size - 1)) != 0)
    throw std::runtime_error("minisgl.attention: page_size must be a power of two >= 16");
  if (a.pool_rows >= (int64_t(1) << 31)) throw std::runtime_error("minisgl.attention: KV pool too large for int32 rows");
}

template <int Tag, typename K>
void set_smem_once(K kern) {
  static bool done[64] = {};  // per kernel (Tag) and device
  int dev = 0;
  cudaGetDevice(&dev);
  if (!done[dev & 63]) {
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kAttnSmem);
    done[dev & 63] = true;
  }
}

}  // namespace

void launch_decode_attention(const AttnArgs& a, cudaStream_t s) {
  if (a.B <= 0) return;
  check_args(a);
  if (a.max_splits > 1 && (a.part_o == nullptr || a.part_lse == nullptr))
    throw std::runtime_error("minisgl.attention: split-KV decode needs scratch buffers");
  CUtensorMap tm = pool_map(a);
  set_smem_once<0>(decode_attn_kernel);
  dim3 grid(std::max(1, a.max_splits), a.hk, a.B);
  launch_pdl(decode_attn_kernel, grid, dim3(kDecodeThreads), kAttnSmem, s, tm, a);
  if (a.max_splits > 1) {
    dim3 g2((a.hq + 3) / 4, a.B);
    launch_pdl(decode_combine_kernel, g2, dim3(128), 0, s, a);
  }
}

void launch_prefill_attention(const AttnArgs& a, cudaStream_t s) {
  if (a.B <= 0 || a.max_q <= 0) return;
  check_args(a);
  CUtensorMap tm = pool_map(a);
  const bool q_aligned = reinterpret_cast<uintptr_t>(a.q) % 16 == 0 && a.ld_q % 8 == 0;
  // head pairs of one KV group share the K/V stream (MINISGL_PREFILL_PAIR=0
  // selects the one-head kernel instead, a measurement switch)
  static const bool pair_on = [] {
    const char* v = std::getenv("MINISGL_PREFILL_PAIR");
    return v == nullptr || v[0] != '0';
  }();
  if (pair_on && q_aligned && a.q_rows > 0 && (a.hq / a.hk) % 2 == 0) {
    static bool pair_attr[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (!pair_attr[dev & 63]) {
      cudaFuncSetAttribute(prefill_attn_pair_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kPrSmem);
      pair_attr[dev & 63] = true;
    }
    const CUtensorMap tq = make_tmap_bf16_2d_sw128(a.q, a.q_rows, static_cast<uint64_t>(a.hq) * kD, a.ld_q, kTcRows);
    dim3 grid((a.max_q + kTcRows - 1) / kTcRows, a.hq / 2, a.B);
    launch_pdl(prefill_attn_pair_kernel, grid, dim3(kPrThreads), kPrSmem, s, tm, tq, a);
    return;
  }
  // the tcgen05 kernel reads Q by TMA: a 16-byte aligned base and row stride
  if (a.q_rows > 0 && q_aligned) {
    static bool attr_set[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (!attr_set[dev & 63]) {
      cudaFuncSetAttribute(prefill_attn_tc_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, kTcSmem);
      attr_set[dev & 63] = true;
    }
    const CUtensorMap tq = make_tmap_bf16_2d_sw128(a.q, a.q_rows, static_cast<uint64_t>(a.hq) * kD, a.ld_q, kTcRows);
    dim3 grid((a.max_q + kTcRows - 1) / kTcRows, a.hq, a.B);
    // the rope maps are unused in this variant: the Q map stands in for them
    launch_pdl(prefill_attn_tc_kernel<false>, grid, dim3(kTcThreads), kTcSmem, s, tm, tq, tq, tq, a);
    return;
  }
  set_smem_once<1>(prefill_attn_kernel);
  dim3 grid((a.max_q + 63) / 64, a.hq, a.B);
  launch_pdl(prefill_attn_kernel, grid, dim3(128), kAttnSmem, s, tm, a);
}

void launch_mla_prefill_attention(const AttnArgs& a, cudaStream_t s) {
  if (a.B <= 0 || a.max_q <= 0) return;
  check_args(a);
  if (a.q_rope == nullptr || a.k_rope == nullptr || a.q_rows <= 0 || a.q_head_stride < kD ||
      a.q_head_stride % 8 != 0)
    throw std::runtime_error("minisgl.mla_prefill_attention: q heads of >= 128 values (multiple of 8), "
                             "q_rope and k_rope are required");
  if (reinterpret_cast<uintptr_t>(a.q) % 16 != 0 || a.ld_q % 8 != 0 ||
      reinterpret_cast<uintptr_t>(a.q_rope) % 16 != 0 || reinterpret_cast<uintptr_t>(a.k_rope) % 16 != 0)
    throw std::runtime_error("minisgl.mla_prefill_attention: 16-byte aligned q / q_rope / k_rope rows");
  static bool attr_set[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (!attr_set[dev & 63]) {
    cudaFuncSetAttribute(prefill_attn_tc_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, kTcRopeSmem);
    attr_set[dev & 63] = true;
  }
  const CUtensorMap tm = pool_map(a);
  const CUtensorMap tq =
      make_tmap_bf16_2d_sw128(a.q, a.q_rows, static_cast<uint64_t>(a.hq) * a.q_head_stride, a.ld_q, kTcRows);
  const CUtensorMap tqr = make_tmap_bf16_2d_sw128(a.q_rope, a.q_rows, static_cast<uint64_t>(a.hq) * 64,
                                                  static_cast<uint64_t>(a.hq) * 64, kTcRows);
  const uint32_t seg = a.page_size < kTile ? a.page_size : kTile;
  const CUtensorMap tkr = make_tmap_bf16_2d_sw128(a.k_rope, a.rope_rows, 64, 64, seg);
  dim3 grid((a.max_q + kTcRows - 1) / kTcRows, a.hq, a.B);
  launch_pdl(prefill_attn_tc_kernel<true>, grid, dim3(kTcThreads), kTcRopeSmem, s, tm, tq, tqr, tkr, a);
}

}  // namespace minisgl

// ====================================================== allocation-free ====
// minisgl_decode_attention_noalloc (declared in noalloc.h): the split-KV
// decode above with its scratch in a fixed device array instead of caller
// buffers. Nothing here allocates: argument errors are reported through the
// return code and a caller-owned message buffer, the tensor map is encoded on
// the stack, and launches go straight to cudaLaunchKernelEx.

namespace minisgl {
namespace {

constexpr size_t kNoAllocFloats = MINISGL_NOALLOC_SCRATCH_BYTES / sizeof(float);
static_assert(MINISGL_NOALLOC_SCRATCH_BYTES % 256 == 0, "scratch size must keep 256-byte alignment");

// Shared by every call on a device; see noalloc.h for the race rule.
static __device__ __align__(256) float g_decode_scratch[kNoAllocFloats];

constexpr int kNoAllocMaxDevices = 64;
constexpr int kNoAllocMaxSplits = 16;

struct NoAllocDeviceState {
  float* scratch = nullptr;  // device address of g_decode_scratch
  bool ready = false;
};
NoAllocDeviceState g_noalloc_state[kNoAllocMaxDevices];
std::mutex g_noalloc_mu;
PFN_cuTensorMapEncodeTiled_v12000 g_noalloc_encode = nullptr;

int noalloc_fail(char* msg, size_t msg_len, int code, const char* fmt, ...) {
  if (msg != nullptr && msg_len > 0) {
    va_list ap;
    va_start(ap, fmt);
    std::vsnprintf(msg, msg_len, fmt, ap);
    va_end(ap);
  }
  return code;
}

// Once per device, with that device current: look up the scratch array and
// the tensor-map encoder, and raise the kernel's shared-memory limit.
int noalloc_setup(int dev, float** scratch, char* msg, size_t msg_len) {
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  NoAllocDeviceState& st = g_noalloc_state[dev];
  if (st.ready) {
    *scratch = st.scratch;
    return MINISGL_NOALLOC_OK;
  }
  if (g_noalloc_encode == nullptr) {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    const cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q);
    if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || fn == nullptr)
      return noalloc_fail(msg, msg_len, MINISGL_NOALLOC_ECUDA,
                          "minisgl_decode_attention_noalloc: cuTensorMapEncodeTiled unavailable (%s)",
                          cudaGetErrorString(e));
    g_noalloc_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  }
  void* ptr = nullptr;
  cudaError_t e = cudaGetSymbolAddress(&ptr, g_decode_scratch);
  if (e != cudaSuccess || ptr == nullptr)
    return noalloc_fail(msg, msg_len, MINISGL_NOALLOC_ECUDA,
                        "minisgl_decode_attention_noalloc: cudaGetSymbolAddress failed on device %d: %s", dev,
                        cudaGetErrorString(e));
  if ((reinterpret_cast<uintptr_t>(ptr) & 255) != 0)
    return noalloc_fail(msg, msg_len, MINISGL_NOALLOC_ECUDA,
                        "minisgl_decode_attention_noalloc: scratch array is not 256-byte aligned");
  e = cudaFuncSetAttribute(decode_attn_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kAttnSmem);
  if (e != cudaSuccess)
    return noalloc_fail(msg, msg_len, MINISGL_NOALLOC_ECUDA,
                        "minisgl_decode_attention_noalloc: cannot set shared memory limit: %s",
                        cudaGetErrorString(e));
  st.scratch = static_cast<float*>(ptr);
  st.ready = true;
  *scratch = st.scratch;
  return MINISGL_NOALLOC_OK;
}

template <typename... KArgs, typename... Args>
cudaError_t noalloc_launch(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                           Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr;
  attr.id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr.val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = &attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
}

}  // namespace
}  // namespace minisgl

extern "C" __attribute__((visibility("default"))) int minisgl_decode_attention_noalloc(
    void* out, const void* q, int ld_q, const void* kv_pool, int num_layers, int num_pages, int layer,
    const int32_t* page_table, int ld_pt, const int32_t* req_rows, const int32_t* seq_lens, int B, int hq,
    int hk, int d, int page_size, float scale, int max_splits, int* err, void* stream, char* msg,
    size_t msg_len) {
  using namespace minisgl;
  constexpr const char* kName = "minisgl_decode_attention_noalloc";
  if (msg != nullptr && msg_len > 0) msg[0] = '\0';
  if (B <= 0) return MINISGL_NOALLOC_OK;
  // ---- argument checks (the same rules as the regular entry point)
  if (out == nullptr || q == nullptr || kv_pool == nullptr || page_table == nullptr || req_rows == nullptr ||
      seq_lens == nullptr)
    return noalloc_fail(msg, msg_len, MINISGL_NOALLOC_EINVAL, "%s: a required pointer is NULL", kName);
  if (d != kD) return noalloc_fail(msg, msg_len, MINISGL_NOALLOC_EINVAL, "%s: head_dim must be 128 (got %d)", kName, d);
  if (hk <= 0 || hq <= 0 || hq % hk != 0 || hq / hk > 16)
    return noalloc_fail(msg, msg_len, MINISGL_NOALLOC_EINVAL,
                        "%s: need hq %% hk == 0 and a GQA group of at most 16 (hq=%d hk=%d)", kName, hq, hk);
  if (page_size < 16 || (page_size & (page_size - 1)) != 0)
    return noalloc_fail(msg, msg_len, MINISGL_NOALLOC_EINVAL, "%s: page_size must be a power of two >= 16 (got %d)",
                        kName, page_size);
  if (num_layers <= 0 || num_pages <= 0 || layer < 0 || layer >= num_layers)
    return noalloc_fail(msg, msg_len, MINISGL_NOALLOC_EINVAL, "%s: layer %d out of range for %d layers", kName, layer,
                        num_layers);
  if (max_splits < 1 || max_splits > kNoAllocMaxSplits)
    return noalloc_fail(msg, msg_len, MINISGL_NOALLOC_EINVAL, "%s: max_splits must be in [1, %d] (got %d)", kName,
                        kNoAllocMaxSplits, max_splits);
  if (ld_pt < 1)
    return noalloc_fail(msg, msg_len, MINISGL_NOALLOC_EINVAL, "%s: ld_pt (page-table row stride) must be >= 1 (got %d)",
                        kName, ld_pt);
  if (ld_q < hq * d || (ld_q & 7) != 0)
    return noalloc_fail(msg, msg_len, MINISGL_NOALLOC_EINVAL, "%s: ld_q must be >= hq*d and a multiple of 8 (got %d)",
                        kName, ld_q);
  if (((reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(out) | reinterpret_cast<uintptr_t>(kv_pool)) &
       15) != 0)
    return noalloc_fail(msg, msg_len, MINISGL_NOALLOC_EINVAL, "%s: q, out and kv_pool must be 16-byte aligned", kName);
  const int64_t rows_per_layer = static_cast<int64_t>(num_pages) * hk * page_size;
  const int64_t pool_rows = 2 * static_cast<int64_t>(num_layers) * rows_per_layer;
  if (pool_rows >= (int64_t(1) << 31))
    return noalloc_fail(msg, msg_len, MINISGL_NOALLOC_EINVAL, "%s: KV pool too large for int32 rows", kName);
  // ---- scratch size against the fixed array
  const uint64_t lse_floats = static_cast<uint64_t>(B) * hq * max_splits;
  const uint64_t o_floats = lse_floats * d;
  const uint64_t o_padded = (o_floats + 63) / 64 * 64;  // part_lse starts on a 256-byte boundary
  const uint64_t need = max_splits > 1 ? o_padded + lse_floats : 0;
  if (need > kNoAllocFloats)
    return noalloc_fail(msg, msg_len, MINISGL_NOALLOC_ETOOLARGE,
                        "%s: split-KV scratch of %llu bytes exceeds the fixed %u-byte array "
                        "(B=%d hq=%d max_splits=%d); lower max_splits or split the batch",
                        kName, static_cast<unsigned long long>(need * sizeof(float)),
                        static_cast<unsigned>(MINISGL_NOALLOC_SCRATCH_BYTES), B, hq, max_splits);
  // ---- per-device set-up (first call on the device)
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess)
    return noalloc_fail(msg, msg_len, MINISGL_NOALLOC_ECUDA, "%s: cudaGetDevice failed: %s", kName,
                        cudaGetErrorString(e));
  if (dev < 0 || dev >= kNoAllocMaxDevices)
    return noalloc_fail(msg, msg_len, MINISGL_NOALLOC_ECUDA, "%s: device index %d not supported", kName, dev);
  float* scratch = nullptr;
  const int rc = noalloc_setup(dev, &scratch, msg, msg_len);
  if (rc != MINISGL_NOALLOC_OK) return rc;
  // ---- tensor map over the whole pool, encoded on the stack (no cache)
  CUtensorMap tm;
  {
    const uint32_t box_rows = page_size < kTile ? page_size : kTile;
    cuuint64_t gdim[2] = {static_cast<cuuint64_t>(d), static_cast<cuuint64_t>(pool_rows)};
    cuuint64_t gstride[1] = {static_cast<cuuint64_t>(d) * 2};
    cuuint32_t bdim[2] = {64, box_rows};
    cuuint32_t estride[2] = {1, 1};
    const CUresult r = g_noalloc_encode(&tm, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(kv_pool), gdim,
                                        gstride, bdim, estride, CU_TENSOR_MAP_INTERLEAVE_NONE,
                                        CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS)
      return noalloc_fail(msg, msg_len, MINISGL_NOALLOC_ECUDA, "%s: cuTensorMapEncodeTiled failed with code %d", kName,
                          static_cast<int>(r));
  }
  AttnArgs a{};
  a.q = q;
  a.ld_q = ld_q;
  a.out = out;
  a.kv_pool = kv_pool;
  a.pool_rows = pool_rows;
  a.k_row0 = layer * rows_per_layer;
  a.v_row0 = (static_cast<int64_t>(num_layers) + layer) * rows_per_layer;
  a.page_table = page_table;
  a.ld_pt = ld_pt;
  a.req_rows = req_rows;
  a.seq_lens = seq_lens;
  a.cu_q = nullptr;
  a.B = B;
  a.hq = hq;
  a.hk = hk;
  a.d = d;
  a.page_size = page_size;
  a.max_q = 1;
  a.scale = scale;
  a.max_splits = max_splits;
  a.part_o = max_splits > 1 ? scratch : nullptr;
  a.part_lse = max_splits > 1 ? scratch + o_padded : nullptr;
  a.err = err;
  const cudaStream_t s = static_cast<cudaStream_t>(stream);
  e = noalloc_launch(decode_attn_kernel, dim3(max_splits, hk, B), dim3(kDecodeThreads), kAttnSmem, s, tm, a);
  if (e == cudaSuccess && max_splits > 1)
    e = noalloc_launch(decode_combine_kernel, dim3((hq + 3) / 4, B), dim3(128), 0, s, a);
  if (e != cudaSuccess)
    return noalloc_fail(msg, msg_len, MINISGL_NOALLOC_ECUDA, "%s: launch failed: %s", kName, cudaGetErrorString(e));
  return MINISGL_NOALLOC_OK;
}
