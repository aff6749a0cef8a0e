// Multi-head latent attention (DeepSeek-V3 / Kimi-K2) for sm_100a.
//
// The reference has no MLA (its attention backends are MHA/GQA only:
// python/minisgl/attention/fi.py, trtllm.py). Layout of the absorbed form:
//
//   latent cache   [slots, 576] bf16: rmsnorm(c_kv) (512) | rope(k_pe) (64)
//   q_lat          [H, T_pad, 512]: q_nope absorbed through W_UK (a grouped
//                  GEMM with heads as groups, written head-major so each
//                  head's tokens are contiguous rows of the GEMM)
//   q_pe           [T, H, 64]: rotated positional part of the queries
//   o_lat          [H, T_pad, 512]: attention output in the latent space,
//                  head-major again so W_UV is another grouped GEMM
//
// mla_attn_kernel is a tcgen05 kernel. One CTA handles one query token, 64
// heads and a range of 32-key tiles streamed through a 4-stage ring. With
// M = 64 rows the accumulator fills half of each TMEM lane quadrant (rows
// 16q..16q+15 in lanes 32q..32q+15), so the 64 x 512 fp32 output is kept
// whole in TMEM: dims 0-255 in the lower half-quadrants and dims 256-511 in
// the upper ones (lane offset 16), both in columns 0-255; scores S (64 heads
// x 32 keys, two buffers) sit in columns 256-319 of the lower halves.
//
//   S = Q . K^T   A = Q (K-major, 9 chunks of 64 dims), B = latent tile
//                 (K-major), M = 64 heads, N = 32 keys, K = 576
//   O += P . V    A = P (K-major, written by the softmax warps; tile j uses
//                 keys 32 (j % 2).. of a 64-key buffer, so consecutive
//                 tiles never share a half), B = the first 512 dims of the
//                 same latent tile read MN-major, N = 256 per MMA (two MMAs
//                 for the two output halves)
//
// Warps 0-3 run the softmax (warp q owns heads 16q..16q+15 in lanes 0-15;
// lanes 16-31 own the upper output half of the same heads), warp 4 issues
// TMA, warp 5 issues tcgen05.mma. Softmax is in the exp2 domain with a
// lazy rescale: O and l are only rescaled when a row's running max grows
// by more than 8 (a factor of 256), which keeps P below 256 in bf16.
#include <algorithm>
#include <stdexcept>
#include <string>

#include "common.cuh"
#include "launch.h"
#include "ops.h"
#include "tma_host.h"

namespace minisgl {
namespace {

constexpr int kLora = 512;
constexpr int kRope = 64;
constexpr int kLat = kLora + kRope;          // 576
constexpr int kChunks = kLat / 64;           // 9 chunks of 64 dims
constexpr int kKeys = 64;                    // keys per tile (N of QK; smaller N runs the tensor pipe at a loss)
constexpr int kHeadsCta = 64;                // heads per CTA (MMA M)
constexpr int kQChunk = 64 * 128;            // one 64-dim chunk of Q: 64 heads x 128 bytes
constexpr int kKvChunk = kKeys * 128;        // one 64-dim chunk of a latent tile
constexpr int kQBytes = kChunks * kQChunk;
constexpr int kKvBytes = kChunks * kKvChunk;
constexpr int kPBytes = 64 * 128;            // P: 64 heads x 64 keys
constexpr int kPHalves = 64 / kKeys;         // tiles whose P the buffer holds at once
constexpr int kStages = 2;
constexpr int kSCol = 256;                   // first TMEM column of the score buffers
constexpr int kMlaThreads = 192;
constexpr int kMlaSmem = 1024 + kQBytes + kStages * kKvBytes + kPBytes + 256;
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kRescaleLog2 = 8.f;

// ------------------------------------------------------------ prepare ----
// One CTA per token: the latent row [rmsnorm(c_kv) * w | rope(k_pe)] into
// the cache slot, rope(q_pe) into q_pe [T, H, 64] and q_nope into the
// head-major GEMM input xs [H, T_pad, nope]. Interleaved (GPT-J) rotation:
// pairs (2i, 2i + 1) turn by frequency i; cos_sin [pos, 64] = 32 cos | 32 sin.
__global__ void __launch_bounds__(256) mla_prepare_kernel(MlaPrepareArgs a) {
  pdl_launch_dependents();
  pdl_wait();
  const int t = blockIdx.x;
  const int tid = threadIdx.x;
  const float* cs = a.cos_sin + static_cast<int64_t>(a.positions[t]) * kRope;
  // the two halves run alone when the key rows and the queries are of
  // different token sets (token-sharded context parallelism); both
  // conditions are uniform over the CTA
  if (a.latent != nullptr) {
    __shared__ float red[8];
    const __nv_bfloat16* kva = reinterpret_cast<const __nv_bfloat16*>(a.kv_a) + static_cast<int64_t>(t) * a.ld_kv_a;
    // rmsnorm over kv_lora (512): two values per thread
    float v0 = __bfloat162float(kva[2 * tid]), v1 = __bfloat162float(kva[2 * tid + 1]);
    float ss = warp_sum(v0 * v0 + v1 * v1);
    if ((tid & 31) == 0) red[tid >> 5] = ss;
    __syncthreads();
    float tot = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) tot += red[i];
    const float rstd = rsqrtf(tot / kLora + a.eps);
    int64_t slot = a.out_loc[t];
    // context parallelism: the row lives on the rank owning its 64-key tile,
    // in that rank's pool at local page (global page) / cp
    const bool store = a.cp_size <= 1 || (a.positions[t] / kKeys) % a.cp_size == a.cp_rank;
    if (a.cp_size > 1) slot = (slot / a.page_size / a.cp_size) * a.page_size + slot % a.page_size;
    if (store && a.num_slots > 0 && (slot < 0 || slot >= a.num_slots)) {  // uniform over the CTA
      if (tid == 0) ErrorSink{a.err}.report(kErrBadIndex, 951);
      return;
    }
    __nv_bfloat16* lat = reinterpret_cast<__nv_bfloat16*>(a.latent) + slot * kLat;
    const __nv_bfloat16* nw = reinterpret_cast<const __nv_bfloat16*>(a.norm_w);
    {
      __nv_bfloat162 o;  // x * rstd * w in fp32, one rounding
      o.x = __float2bfloat16_rn(v0 * rstd * __bfloat162float(nw[2 * tid]));
      o.y = __float2bfloat16_rn(v1 * rstd * __bfloat162float(nw[2 * tid + 1]));
      if (store) *reinterpret_cast<__nv_bfloat162*>(lat + 2 * tid) = o;
    }
    if (store && tid < kRope / 2) {
      const float c = cs[tid], s = cs[kRope / 2 + tid];
      const float x0 = __bfloat162float(kva[kLora + 2 * tid]), x1 = __bfloat162float(kva[kLora + 2 * tid + 1]);
      __nv_bfloat162 o;
      o.x = __float2bfloat16_rn(x0 * c - x1 * s);
      o.y = __float2bfloat16_rn(x1 * c + x0 * s);
      *reinterpret_cast<__nv_bfloat162*>(lat + kLora + 2 * tid) = o;
    }
  }
  if (a.q == nullptr) return;
  // queries: H heads of (nope + 64) values
  const int qk = a.nope + kRope;
  const __nv_bfloat16* q = reinterpret_cast<const __nv_bfloat16*>(a.q) + static_cast<int64_t>(t) * a.ld_q;
  __nv_bfloat16* qpe = reinterpret_cast<__nv_bfloat16*>(a.q_pe) + static_cast<int64_t>(t) * a.H * kRope;
  __nv_bfloat16* xs = reinterpret_cast<__nv_bfloat16*>(a.xs);
  const int pairs = a.H * (qk / 2);
  for (int i = tid; i < pairs; i += blockDim.x) {
    const int h = i / (qk / 2);
    const int j = 2 * (i - h * (qk / 2));  // even column inside the head
    const __nv_bfloat162 v = *reinterpret_cast<const __nv_bfloat162*>(q + h * qk + j);
    if (j < a.nope) {
      if (xs != nullptr)  // absent when only the rotated rope part is wanted
        *reinterpret_cast<__nv_bfloat162*>(xs + (static_cast<int64_t>(h) * a.T_pad + t) * a.nope + j) = v;
    } else {
      const int r = (j - a.nope) / 2;
      const float c = cs[r], s = cs[kRope / 2 + r];
      const float x0 = __bfloat162float(v.x), x1 = __bfloat162float(v.y);
      __nv_bfloat162 o;
      o.x = __float2bfloat16_rn(x0 * c - x1 * s);
      o.y = __float2bfloat16_rn(x1 * c + x0 * s);
      *reinterpret_cast<__nv_bfloat162*>(qpe + h * kRope + (j - a.nope)) = o;
    }
  }
}

// [H, T_pad, v] (the W_UV grouped GEMM output) -> [T, H * v] rows for o_proj;
// with a row map, token t lands in row row_map[t] of out_rows rows (the
// rank-major layout a reduce-scatter over context-parallel ranks takes).
__global__ void __launch_bounds__(128) mla_heads_to_rows_kernel(__nv_bfloat16* out, const __nv_bfloat16* in, int T,
                                                               int T_pad, int H, int v, const int32_t* row_map,
                                                               int out_rows, ErrorSink err) {
  pdl_launch_dependents();
  pdl_wait();
  const int t = blockIdx.x;
  const int row = row_map != nullptr ? row_map[t] : t;
  if (row < 0 || row >= out_rows) {
    if (threadIdx.x == 0) err.report(kErrBadIndex, 901);
    return;
  }
  const int n8 = H * v / 8;
  for (int i = threadIdx.x; i < n8; i += blockDim.x) {
    const int h = (i * 8) / v, c = i * 8 - h * v;
    *reinterpret_cast<uint4*>(out + static_cast<int64_t>(row) * H * v + h * v + c) =
        *reinterpret_cast<const uint4*>(in + (static_cast<int64_t>(h) * T_pad + t) * v + c);
  }
}

// ------------------------------------------------ non-absorbed prefill ----
// Latent rows of every key of a prefill batch in a compact page-aligned order:
// row r holds (request row_req[r], position row_pos[r]) and reads that key's
// cache slot (rows with row_req < 0 pad a request to whole pages and read
// slot 0; the attention masks them). c_kv (512) goes to x [R, 512], the kv_b
// GEMM input, and the rotated rope part (64) to k_rope [R, 64]. One warp per
// row.
__global__ void __launch_bounds__(256) mla_gather_keys_kernel(__nv_bfloat16* x, __nv_bfloat16* k_rope,
                                                             const __nv_bfloat16* latent, const int32_t* page_table,
                                                             int ld_pt, const int32_t* req_rows,
                                                             const int32_t* row_req, const int32_t* row_pos, int R,
                                                             int64_t num_slots, ErrorSink err) {
  pdl_launch_dependents();
  pdl_wait();
  const int r = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (r >= R) return;
  const int b = row_req[r];
  int64_t slot = b < 0 ? 0 : page_table[static_cast<int64_t>(req_rows[b]) * ld_pt + row_pos[r]];
  if (slot < 0 || slot >= num_slots) {
    if (lane == 0) err.report(kErrBadIndex, 911);
    slot = 0;
  }
  const uint4* src = reinterpret_cast<const uint4*>(latent + slot * kLat);
  uint4* dx = reinterpret_cast<uint4*>(x + static_cast<int64_t>(r) * kLora);
  dx[lane] = src[lane];
  dx[lane + 32] = src[lane + 32];
  if (lane < 8) reinterpret_cast<uint4*>(k_rope + static_cast<int64_t>(r) * kRope)[lane] = src[64 + lane];
}

// kv_b_proj output y [R, H * 256] (per head 128 k_nope values, then 128 v)
// into the prefill attention's pool layout [2, R / 64, H, 64, 128]: row r at
// page r / 64, position r % 64. One warp per (row, head).
__global__ void __launch_bounds__(256) mla_scatter_kv_kernel(__nv_bfloat16* pool, const __nv_bfloat16* y, int R,
                                                            int H) {
  pdl_launch_dependents();
  pdl_wait();
  const int64_t w = static_cast<int64_t>(blockIdx.x) * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (w >= static_cast<int64_t>(R) * H) return;
  const int r = static_cast<int>(w / H), h = static_cast<int>(w % H);
  const int64_t plane = static_cast<int64_t>(R) * H * 128;  // elements of the K plane
  const int64_t dst = ((static_cast<int64_t>(r / 64) * H + h) * 64 + r % 64) * 128;
  const uint4 v = reinterpret_cast<const uint4*>(y + (static_cast<int64_t>(r) * H + h) * 256)[lane];
  // lanes 0-15: k_nope (128 values), 16-31: v
  reinterpret_cast<uint4*>(pool + (lane < 16 ? 0 : plane) + dst)[lane & 15] = v;
}

// ---------------------------------------------------------- attention ----
__device__ __forceinline__ uint32_t f2u(float f) { return __float_as_uint(f); }
__device__ __forceinline__ float u2f(uint32_t u) { return __uint_as_float(u); }
// 2^x on the special-function unit (PTX ex2.approx.ftz: relative error of a
// few ulp, ex2(-inf) = +0), which is what a softmax needs.
__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// The request and causal key count of query token t: the last query token
// of a request sees all seq_lens[b] keys, the one before it one fewer.
__device__ __forceinline__ void mla_token(const MlaAttnArgs& a, int t, int& row, int& len) {
  int lo = 0, hi = a.B - 1;
  while (lo < hi) {  // largest b with cu_q[b] <= t
    const int mid = (lo + hi + 1) >> 1;
    if (a.cu_q[mid] <= t) lo = mid;
    else hi = mid - 1;
  }
  row = a.req_rows[lo];
  len = a.seq_lens[lo] - (a.cu_q[lo + 1] - 1 - t);
}

// grid (splits, T, head groups of 64); 192 threads.
__global__ void __launch_bounds__(kMlaThreads, 1)
    mla_attn_kernel(const __grid_constant__ CUtensorMap tm_qlat, const __grid_constant__ CUtensorMap tm_qpe,
                    const __grid_constant__ CUtensorMap tm_lat, const MlaAttnArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint8_t* sQ = smem;
  uint8_t* sKV = sQ + kQBytes;
  uint8_t* sP = sKV + kStages * kKvBytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sP + kPBytes);
  uint64_t* q_full = bars;
  uint64_t* kv_full = bars + 1;              // [kStages]
  uint64_t* kv_empty = kv_full + kStages;    // [kStages]
  uint64_t* s_full = kv_empty + kStages;     // [2] score buffers
  uint64_t* s_free = s_full + 2;             // [2]
  uint64_t* p_full = s_free + 2;             // [2] P of tiles with j % 2 == h written
  uint64_t* o_done = p_full + 2;             // [2] PV of tiles with j % 2 == h complete
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(o_done + 2);
  int* s_abort = reinterpret_cast<int*>(o_done + 3);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int split = blockIdx.x, t = blockIdx.y, g = blockIdx.z;
  pdl_launch_dependents();
  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < kStages; ++i) {
      mbar_init(&kv_full[i], 1);
      mbar_init(&kv_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&s_free[i], 4);
      mbar_init(&p_full[i], 4);
      mbar_init(&o_done[i], 1);
    }
    *s_abort = 0;
    fence_barrier_init();
    prefetch_tmap(&tm_qlat);
    prefetch_tmap(&tm_qpe);
    prefetch_tmap(&tm_lat);
  }
  // queries, cache rows and metadata come from earlier kernels; TMEM is
  // taken only after them, so an earlier kernel still waiting to allocate on
  // this SM is never blocked by this CTA
  pdl_wait();
  if (warp == 5) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  int row = 0, len = 0;
  mla_token(a, t, row, len);
  // context parallelism: this rank owns the 64-key tiles t with
  // t % cp_size == cp_rank; local tile j is global tile cp_rank + cp_size j
  const int cp = a.cp_size > 1 ? a.cp_size : 1, cpr = a.cp_size > 1 ? a.cp_rank : 0;
  const int ntiles_glob = (max(len, 0) + kKeys - 1) / kKeys;
  const int ntiles_all = ntiles_glob > cpr ? (ntiles_glob - cpr + cp - 1) / cp : 0;
  const int per = (ntiles_all + a.splits - 1) / a.splits;
  const int tile0 = split * per;
  const int n = max(0, min(ntiles_all, tile0 + per) - tile0);
  auto tile_pos = [&](int j) { return (cpr + cp * (tile0 + j)) * kKeys; };  // first key of local tile j
  const ErrorSink err{a.err};
  const bool traced = a.trace != nullptr && blockIdx.x == 0 && blockIdx.y == 0 && blockIdx.z == 0;
  int issued = 0;  // latent tiles whose copies the producer started

  if (warp == 4) {
    // ------------------------------------------------------------ TMA ----
    // The whole warp walks the loop: lane 0 waits and issues copies, and the
    // 32 lanes keep the page ids of the next 32 key segments in registers,
    // read one window ahead, so no copy waits on a page-table load.
    if (n > 0) {
      if (lane == 0) {
        mbar_arrive_expect_tx(q_full, kQBytes);
        for (int c = 0; c < kLora / 64; ++c)
          tma_load_3d(sQ + c * kQChunk, &tm_qlat, q_full, c * 64, t, g * kHeadsCta);
        tma_load_2d(sQ + (kChunks - 1) * kQChunk, &tm_qpe, q_full, 0, t * a.H + g * kHeadsCta);
      }
      const int32_t* pt = a.page_table + static_cast<int64_t>(row) * a.ld_pt;
      const int P = a.page_size;
      const int seg = P < kKeys ? P : kKeys;
      const int segs = kKeys / seg;  // segments per tile
      auto page_of = [&](int k) {  // page id of segment k (positions past the end: page 0, masked later)
        const int pos = tile_pos(k / segs) + (k % segs) * seg;
        return pos < len ? pt[pos] / P / cp : 0;  // context parallelism: local page (global page) / cp
      };
      int base = 0;
      int cur = page_of(lane), nxt = page_of(32 + lane);
      for (int j = 0; j < n; ++j) {
        const int s = j % kStages;
        int go = 1;
        if (lane == 0) {
          if (j >= kStages && !mbar_wait(&kv_empty[s], ((j / kStages) - 1) & 1, err, 201)) {
            atomicExch(s_abort, 1);
            go = 0;
          }
          if (*reinterpret_cast<volatile int*>(s_abort)) go = 0;
        }
        if (!__shfl_sync(0xffffffffu, go, 0)) break;
        if (lane == 0) {
          ++issued;
          mbar_arrive_expect_tx(&kv_full[s], kKvBytes);
          if (traced && j < 64) a.trace[j * 8 + 0] = globaltimer_ns();
        }
        uint8_t* st = sKV + s * kKvBytes;
        const int p0 = tile_pos(j);
        for (int q = 0; q < segs; ++q) {
          const int k = j * segs + q;
          if (k >= base + 32) {  // slide the window (warp-uniform)
            base += 32;
            cur = nxt;
            nxt = page_of(base + 32 + lane);
          }
          const int page = __shfl_sync(0xffffffffu, cur, k - base);
          if (lane == 0) {
            const int r = page * P + (P < kKeys ? 0 : p0 % P);
            if (seg == kKeys) {
              tma_load_3d(st, &tm_lat, &kv_full[s], 0, r, 0);  // all 9 chunks in one box
            } else {
              for (int c = 0; c < kChunks; ++c)
                tma_load_2d(st + c * kKvChunk + q * seg * 128, &tm_lat, &kv_full[s], c * 64, r);
            }
          }
        }
      }
    }
    __syncwarp();
  } else if (warp == 5) {
    // ------------------------------------------------------------ MMA ----
    constexpr uint32_t idesc_qk = make_idesc_bf16(64, kKeys);
    constexpr uint32_t idesc_pv = make_idesc_bf16(64, 256, false, true);
    const uint32_t q_addr = smem_u32(sQ), kv_addr = smem_u32(sKV), p_addr = smem_u32(sP);
    bool ok = n > 0 && __all_sync(0xffffffffu, mbar_wait(q_full, 0, err, 202));
    auto qk = [&](int j) {  // S[j % 2] = Q . K_j^T
      const uint32_t st = kv_addr + (j % kStages) * kKvBytes;
      const uint32_t d = tmem + kSCol + (j % 2) * kKeys;
      for (int c = 0; c < kChunks; ++c)
#pragma unroll
        for (int k = 0; k < 4; ++k)
          tc_mma_f16(d, make_sdesc_k_sw128(q_addr + c * kQChunk + k * 32),
                     make_sdesc_k_sw128(st + c * kKvChunk + k * 32), idesc_qk, (c | k) != 0 ? 1u : 0u);
      tc_commit(&s_full[j % 2]);
    };
    auto pv = [&](int i) {  // O += P_i . V_i (two N = 256 halves)
      const uint32_t st = kv_addr + (i % kStages) * kKvBytes;
#pragma unroll
      for (int kk = 0; kk < kKeys / 16; ++kk) {
        const uint64_t pa = make_sdesc_k_sw128(p_addr + ((i % kPHalves) * (kKeys / 16) + kk) * 32);
        const uint32_t acc = (i > 0 || kk > 0) ? 1u : 0u;
        tc_mma_f16(tmem, pa, make_sdesc_mn_sw128(st + kk * 2048, kKvChunk), idesc_pv, acc);
        tc_mma_f16(tmem + (16u << 16), pa, make_sdesc_mn_sw128(st + 4 * kKvChunk + kk * 2048, kKvChunk),
                   idesc_pv, acc);
      }
      tc_commit(&kv_empty[i % kStages]);
      tc_commit(&o_done[i % 2]);
    };
    // Issue QK(j) and PV(i) in whichever order their inputs arrive: QK(j)
    // needs latent tile j and a free score buffer (the softmax of tile j - 2
    // has read it), PV(i) needs P_i. Waiting for tile j before PV(i) would
    // chain every copy's latency into the loop.
    int qn = 0, pn = 0;  // next QK, next PV
    uint64_t t0 = globaltimer_ns();
    uint32_t spins = 0;
    while (ok && pn < n) {
      // lane 0 polls and decides; the warp follows its choice
      // QK first, tested without suspending (a try_wait on P_pn sleeps until
      // that softmax ends, which would start QK(pn + 1) only after PV(pn))
      int choice = 0;
      if (lane == 0) {
        if (qn < n && qn <= pn + 1 && mbar_test_wait(&kv_full[qn % kStages], (qn / kStages) & 1) &&
            (qn < 2 || mbar_test_wait(&s_free[qn % 2], ((qn / 2) - 1) & 1)))
          choice = 2;
        else if (pn < qn && mbar_try_wait(&p_full[pn % 2], (pn / 2) & 1)) choice = 1;
        else if (((++spins) & 0xFFu) == 0 && globaltimer_ns() - t0 > kWaitBudgetNs)
          choice = 3;
      }
      choice = __shfl_sync(0xffffffffu, choice, 0);
      if (choice == 3) {
        if (lane == 0) err.report(kErrMbarTimeout, 206);
        ok = false;
      } else if (choice != 0) {
        tc_fence_after();
        if (choice == 1) {
          if (lane == 0) {
            pv(pn);
            if (traced && pn < 64) a.trace[pn * 8 + 4] = globaltimer_ns();
          }
          ++pn;
        } else {
          if (lane == 0) {
            qk(qn);
            if (traced && qn < 64) a.trace[qn * 8 + 1] = globaltimer_ns();
          }
          ++qn;
        }
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
    const int r = 16 * warp + (lane & 15);  // head row of this lane (both halves)
    const bool lower = lane < 16;
    const uint32_t lane_base = tmem + (static_cast<uint32_t>(32 * warp) << 16);
    const float sl2 = a.scale * kLog2e;
    float m_run = -INFINITY, l_sum = 0.f;
    bool ok = true;
    for (int i = 0; i < n; ++i) {
      const int b = i % 2;
      ok = __all_sync(0xffffffffu, mbar_wait(&s_full[b], (i / 2) & 1, err, 211));
      if (!ok) break;
      tc_fence_after();
      const bool tr = traced && threadIdx.x == 0 && i < 64;
      if (tr) a.trace[i * 8 + 2] = globaltimer_ns();
      uint32_t sv[kKeys];
#pragma unroll
      for (int c = 0; c < kKeys / 32; ++c)
        tmem_ld_32x32b_x32(lane_base + kSCol + b * kKeys + 32 * c, *reinterpret_cast<uint32_t(*)[32]>(&sv[32 * c]));
      tc_wait_ld();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&s_free[b]);
      const int p0 = tile_pos(i);
      const int valid = min(kKeys, len - p0);
      if (valid < kKeys) {
#pragma unroll
        for (int j = 0; j < kKeys; ++j)
          if (j >= valid) sv[j] = f2u(-INFINITY);
      }
      float mr = u2f(sv[0]);
#pragma unroll
      for (int j = 1; j < kKeys; ++j) mr = fmaxf(mr, u2f(sv[j]));
      const float mt = mr * sl2;  // the scale is positive: max commutes with it
      // lazy rescale: only when the running max grows by more than 2^8
      const bool grow = lower && mt > m_run + kRescaleLog2;
      float alpha = 1.f;
      if (grow) {
        alpha = fast_exp2(m_run - mt);  // 0 on the first tile (m_run = -inf)
        l_sum *= alpha;
        m_run = mt;
      }
      const bool any_grow = __any_sync(0xffffffffu, grow) && i > 0;
      const float alpha_row = __shfl_sync(0xffffffffu, alpha, lane & 15);
      // P = 2^(s * scale * log2 e - m) packed to bf16 pairs, computed while
      // earlier P . V products may still be running
      uint32_t pk[kKeys / 2];
      if (lower) {
        float ps = 0.f;
#pragma unroll
        for (int e = 0; e < kKeys / 2; ++e) {
          const float lo = fast_exp2(fmaf(u2f(sv[2 * e]), sl2, -m_run));
          const float hi = fast_exp2(fmaf(u2f(sv[2 * e + 1]), sl2, -m_run));
          ps += lo + hi;
          const __nv_bfloat162 b2 = __floats2bfloat162_rn(lo, hi);
          pk[e] = *reinterpret_cast<const uint32_t*>(&b2);
        }
        l_sum += ps;
      }
      // this part of P was last read by PV(i - kPHalves); a rescale of O
      // needs PV(i - 1) finished as well
      if (i >= kPHalves) {
        const int prev = i - kPHalves;
        ok = __all_sync(0xffffffffu, mbar_wait(&o_done[prev % 2], (prev / 2) & 1, err, 212));
        if (!ok) break;
      }
      if (any_grow) {
        if (kPHalves > 1) {
          ok = __all_sync(0xffffffffu, mbar_wait(&o_done[(i - 1) % 2], ((i - 1) / 2) & 1, err, 214));
          if (!ok) break;
        }
        tc_fence_after();
        // O rows of this warp: lanes 0-15 the low 256 dims, 16-31 the high
#pragma unroll 1
        for (int c = 0; c < 8; ++c) {
          uint32_t ov[32];
          tmem_ld_32x32b_x32(lane_base + c * 32, ov);
          tc_wait_ld();
#pragma unroll
          for (int j = 0; j < 32; ++j) ov[j] = f2u(u2f(ov[j]) * alpha_row);
          tmem_st_32x32b_x32(lane_base + c * 32, ov);
        }
        tc_wait_st();
      }
      if (tr && i >= 1) a.trace[(i - 1) * 8 + 5] = globaltimer_ns();
      if (lower) {
        // keys 32 (i % 2).. of row r of P, 128-byte-swizzled K-major layout
        uint8_t* prow = sP + r * 128;
#pragma unroll
        for (int c = 0; c < kKeys / 8; ++c) {
          const int chunk = (i % kPHalves) * (kKeys / 8) + c;
          *reinterpret_cast<uint4*>(prow + ((chunk ^ (r & 7)) << 4)) =
              make_uint4(pk[4 * c], pk[4 * c + 1], pk[4 * c + 2], pk[4 * c + 3]);
        }
      }
      fence_proxy_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_full[i % 2]);
      if (tr) a.trace[i * 8 + 3] = globaltimer_ns();
    }
    // ------------------------------------------------------- epilogue ----
    if (!ok && lane == 0) atomicExch(s_abort, 1);
    if (ok && n > 0) ok = __all_sync(0xffffffffu, mbar_wait(&o_done[(n - 1) % 2], ((n - 1) / 2) & 1, err, 213));
    tc_fence_after();
    const float l_row = __shfl_sync(0xffffffffu, l_sum, lane & 15);
    const float m_row = __shfl_sync(0xffffffffu, m_run, lane & 15);
    const int h = g * kHeadsCta + r;
    const int half = lower ? 0 : 1;
    const bool live = ok && n > 0;
    const float inv = live && l_row > 0.f ? 1.f / l_row : 0.f;
#pragma unroll 1
    for (int c = 0; c < 8; ++c) {
      uint32_t ov[32];
      if (live) {
        tmem_ld_32x32b_x32(lane_base + c * 32, ov);
        tc_wait_ld();
      } else {
#pragma unroll
        for (int j = 0; j < 32; ++j) ov[j] = 0u;
      }
      if (h >= a.H) continue;
      const int d0 = half * 256 + c * 32;
      if (a.splits == 1 && cp == 1) {
        __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(a.out) + (static_cast<int64_t>(h) * a.T_pad + t) * kLora + d0;
#pragma unroll
        for (int q4 = 0; q4 < 4; ++q4) {
          uint4 v;
          v.x = pack_bf16x2(u2f(ov[q4 * 8 + 0]) * inv, u2f(ov[q4 * 8 + 1]) * inv);
          v.y = pack_bf16x2(u2f(ov[q4 * 8 + 2]) * inv, u2f(ov[q4 * 8 + 3]) * inv);
          v.z = pack_bf16x2(u2f(ov[q4 * 8 + 4]) * inv, u2f(ov[q4 * 8 + 5]) * inv);
          v.w = pack_bf16x2(u2f(ov[q4 * 8 + 6]) * inv, u2f(ov[q4 * 8 + 7]) * inv);
          *reinterpret_cast<uint4*>(dst + q4 * 8) = v;
        }
      } else {
        float* dst = a.part_o + ((static_cast<int64_t>(cpr * a.splits + split) * a.T + t) * a.H + h) * kLora + d0;
#pragma unroll
        for (int q4 = 0; q4 < 8; ++q4)
          *reinterpret_cast<float4*>(dst + q4 * 4) = make_float4(u2f(ov[q4 * 4]) * inv, u2f(ov[q4 * 4 + 1]) * inv,
                                                                 u2f(ov[q4 * 4 + 2]) * inv, u2f(ov[q4 * 4 + 3]) * inv);
      }
    }
    if ((a.splits > 1 || cp > 1) && lower && h < a.H)
      a.part_lse[(static_cast<int64_t>(cpr * a.splits + split) * a.T + t) * a.H + h] =
          live && l_row > 0.f ? m_row + log2f(l_row) : -INFINITY;
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 4 && lane == 0 && n > 0 && *reinterpret_cast<volatile int*>(s_abort)) {
    // after an abort, let the copies still in flight land before the CTA
    // leaves (bounded waits; the normal path never gets here)
    mbar_wait(q_full, 0, err, 207);
    for (int j = max(0, issued - kStages); j < issued; ++j)
      mbar_wait(&kv_full[j % kStages], (j / kStages) & 1, err, 208);
  }
  if (warp == 5) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// Merge the split-KV partials: grid (T, H), 128 threads x 4 dims. With
// own_only (token-sharded context parallelism) the normaliser runs over the
// log-sum-exps of every rank's splits but only this rank's partial outputs
// are summed: the result is this rank's share of the merged output, and the
// shares of all ranks add up to it (after any linear map, such as W_UV).
__global__ void __launch_bounds__(128) mla_combine_kernel(MlaAttnArgs a) {
  pdl_launch_dependents();
  pdl_wait();
  const int t = blockIdx.x, h = blockIdx.y;
  float mx = -INFINITY;
  const int parts = a.splits * (a.cp_size > 1 ? a.cp_size : 1);  // every rank's splits
  const int own_lo = a.own_only ? a.cp_rank * a.splits : 0;
  const int own_hi = a.own_only ? own_lo + a.splits : parts;
  for (int s = 0; s < parts; ++s) mx = fmaxf(mx, a.part_lse[(static_cast<int64_t>(s) * a.T + t) * a.H + h]);
  float acc[4] = {0.f, 0.f, 0.f, 0.f};
  float wsum = 0.f;
  for (int s = 0; s < parts; ++s) {
    const float lse = a.part_lse[(static_cast<int64_t>(s) * a.T + t) * a.H + h];
    if (lse == -INFINITY) continue;
    const float w = exp2f(lse - mx);
    wsum += w;
    if (s < own_lo || s >= own_hi) continue;
    const float4 v = *reinterpret_cast<const float4*>(a.part_o + ((static_cast<int64_t>(s) * a.T + t) * a.H + h) * kLora +
                                                      threadIdx.x * 4);
    acc[0] += w * v.x, acc[1] += w * v.y, acc[2] += w * v.z, acc[3] += w * v.w;
  }
  const float inv = wsum > 0.f ? 1.f / wsum : 0.f;
  __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(a.out) + (static_cast<int64_t>(h) * a.T_pad + t) * kLora +
                       threadIdx.x * 4;
  uint2 o;
  o.x = pack_bf16x2(acc[0] * inv, acc[1] * inv);
  o.y = pack_bf16x2(acc[2] * inv, acc[3] * inv);
  *reinterpret_cast<uint2*>(dst) = o;
}

}  // namespace

// ---------------------------------------------------------------- host ----
void launch_mla_prepare(const MlaPrepareArgs& a, cudaStream_t s) {
  if (a.T <= 0 || (a.latent == nullptr && a.q == nullptr)) return;
  if (a.kv_lora != kLora || a.rope != kRope)
    throw std::runtime_error("minisgl.mla_prepare: the sm_100a kernels take kv_lora_rank 512 and qk_rope_head_dim 64");
  if (a.nope % 2 != 0 || a.T_pad < a.T || a.H <= 0)
    throw std::runtime_error("minisgl.mla_prepare: bad head layout");
  launch_pdl(mla_prepare_kernel, dim3(a.T), dim3(256), 0, s, a);
}

void launch_mla_heads_to_rows(void* out, const void* in, int T, int T_pad, int H, int v, const int32_t* row_map,
                              int out_rows, int* err, cudaStream_t s) {
  if (T <= 0) return;
  if ((H * v) % 8 != 0 || v % 8 != 0) throw std::runtime_error("minisgl.mla_output: v must be a multiple of 8");
  launch_pdl(mla_heads_to_rows_kernel, dim3(T), dim3(128), 0, s, static_cast<__nv_bfloat16*>(out),
             static_cast<const __nv_bfloat16*>(in), T, T_pad, H, v, row_map, out_rows, ErrorSink{err});
}

void launch_mla_gather_keys(void* x, void* k_rope, const void* latent, int64_t num_slots, const int32_t* page_table,
                            int ld_pt, const int32_t* req_rows, const int32_t* row_req, const int32_t* row_pos, int R,
                            int* err, cudaStream_t s) {
  if (R <= 0) return;
  launch_pdl(mla_gather_keys_kernel, dim3((R + 7) / 8), dim3(256), 0, s, static_cast<__nv_bfloat16*>(x),
             static_cast<__nv_bfloat16*>(k_rope), static_cast<const __nv_bfloat16*>(latent), page_table, ld_pt,
             req_rows, row_req, row_pos, R, num_slots, ErrorSink{err});
}

void launch_mla_scatter_kv(void* pool, const void* y, int R, int H, cudaStream_t s) {
  if (R <= 0) return;
  if (R % 64 != 0) throw std::runtime_error("minisgl.mla_scatter_kv: rows must fill whole pages of 64");
  const int64_t warps = static_cast<int64_t>(R) * H;
  launch_pdl(mla_scatter_kv_kernel, dim3(static_cast<unsigned>((warps + 7) / 8)), dim3(256), 0, s,
             static_cast<__nv_bfloat16*>(pool), static_cast<const __nv_bfloat16*>(y), R, H);
}

int mla_num_splits(int T, int H) {
  const int ctas = T * ((H + kHeadsCta - 1) / kHeadsCta);
  return std::max(1, std::min(16, 148 / std::max(1, ctas)));
}

void launch_mla_attention(const MlaAttnArgs& a, cudaStream_t s) {
  if (a.T <= 0) return;
  const int P = a.page_size;
  if (!(P == 8 || P == 16 || (P > 0 && P % 32 == 0)))
    throw std::runtime_error("minisgl.mla_attention: page_size must be 8, 16 or a multiple of 32");
  const bool partials = a.splits > 1 || a.cp_size > 1;
  if (a.splits < 1 || a.splits > 16 || (partials && (a.part_o == nullptr || a.part_lse == nullptr)))
    throw std::runtime_error("minisgl.mla_attention: splits in [1, 16] with partial buffers");
  if (a.cp_size > 1 && (a.cp_rank < 0 || a.cp_rank >= a.cp_size))
    throw std::runtime_error("minisgl.mla_attention: cp_rank outside [0, cp_size)");
  if (a.T_pad < a.T || a.B <= 0 || a.H <= 0) throw std::runtime_error("minisgl.mla_attention: bad shapes");
  static bool smem_set = false;
  if (!smem_set) {
    cudaFuncSetAttribute(mla_attn_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kMlaSmem);
    smem_set = true;
  }
  uint64_t qd[3] = {static_cast<uint64_t>(kLora), static_cast<uint64_t>(a.T_pad), static_cast<uint64_t>(a.H)};
  uint64_t qs[2] = {kLora * 2ull, static_cast<uint64_t>(a.T_pad) * kLora * 2ull};
  uint32_t qb[3] = {64, 1, kHeadsCta};
  CUtensorMap tq = make_tmap(a.q_lat, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, 3, qd, qs, qb, CU_TENSOR_MAP_SWIZZLE_128B);
  CUtensorMap tp = make_tmap_bf16_2d_sw128(a.q_pe, static_cast<uint64_t>(a.T) * a.H, kRope, kRope, kHeadsCta);
  const int seg = P < kKeys ? P : kKeys;
  // pages of >= 32 keys: one 3-D box {64 dims, 32 keys, 9 chunks} per tile,
  // landing chunk-major as [9][32 keys][128 B]; smaller pages: 2-D boxes of
  // one page segment per chunk
  CUtensorMap tl = seg == kKeys ? make_tmap_bf16_kblocks(a.latent, static_cast<uint64_t>(a.num_slots), kLat, kLat,
                                                         kKeys, kChunks)
                                : make_tmap_bf16_2d_sw128(a.latent, static_cast<uint64_t>(a.num_slots), kLat, kLat, seg);
  dim3 grid(a.splits, a.T, (a.H + kHeadsCta - 1) / kHeadsCta);
  launch_pdl(mla_attn_kernel, grid, dim3(kMlaThreads), kMlaSmem, s, tq, tp, tl, a);
  // context parallelism: the partials of every rank are merged after the
  // caller has gathered them (launch_mla_combine)
  if (a.splits > 1 && a.cp_size <= 1) launch_pdl(mla_combine_kernel, dim3(a.T, a.H), dim3(128), 0, s, a);
}

void launch_mla_combine(const MlaAttnArgs& a, cudaStream_t s) {
  if (a.T <= 0) return;
  launch_pdl(mla_combine_kernel, dim3(a.T, a.H), dim3(128), 0, s, a);
}

}  // namespace minisgl
