// MoE router (top-k expert selection per token, one warp per token) and the
// data movement around the grouped expert GEMMs (align / gather / combine).
//
// scoring 0 (Qwen3-MoE): softmax over experts, top-k, optional
//   renormalisation of the k weights. Replaces sgl_kernel topk_softmax and
//   the renormalise step of the reference (python/minisgl/moe/fused.py:9-29).
// scoring 1 (DeepSeek-V3 / Kimi-K2 style): sigmoid scores, selection on
//   score + correction bias, optional group-limited routing (top-2 sum per
//   group, keep topk_group groups), weights are the unbiased sigmoid scores,
//   renormalised and multiplied by routed_scale.
#include <algorithm>
#include <stdexcept>

#include "common.cuh"
#include "launch.h"
#include "ops.h"

namespace minisgl {
namespace {

constexpr int kMaxPerLane = 16;  // E <= 512

__device__ __forceinline__ void warp_argmax(float& v, int& i) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, v, o);
    const int oi = __shfl_xor_sync(0xffffffffu, i, o);
    if (ov > v || (ov == v && oi < i)) v = ov, i = oi;
  }
}

__global__ void moe_route_kernel(MoeRouteArgs a) {
  pdl_launch_dependents();
  pdl_wait();  // router logits come from the previous kernel
  const int warps = blockDim.x >> 5;
  const int t = blockIdx.x * warps + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (t >= a.T) return;
  const float* lg = a.logits + static_cast<int64_t>(t) * a.E;
  const int per = (a.E + 31) / 32;
  float score[kMaxPerLane], choice[kMaxPerLane];
#pragma unroll
  for (int j = 0; j < kMaxPerLane; ++j) {
    const int e = j * 32 + lane;
    score[j] = -INFINITY;
    choice[j] = -INFINITY;
    if (j < per && e < a.E) {
      const float x = lg[e];
      if (a.scoring == 0) {
        score[j] = x;
      } else {
        score[j] = 1.f / (1.f + __expf(-x));
        choice[j] = score[j] + (a.bias != nullptr ? a.bias[e] : 0.f);
      }
    }
  }
  if (a.scoring == 0) {
    float mx = -INFINITY;
#pragma unroll
    for (int j = 0; j < kMaxPerLane; ++j) mx = fmaxf(mx, score[j]);
    mx = warp_max(mx);
    float sum = 0.f;
#pragma unroll
    for (int j = 0; j < kMaxPerLane; ++j) {
      score[j] = score[j] == -INFINITY ? 0.f : __expf(score[j] - mx);
      sum += score[j];
    }
    sum = warp_sum(sum);
    const float inv = 1.f / sum;
#pragma unroll
    for (int j = 0; j < kMaxPerLane; ++j) {
      const int e = j * 32 + lane;
      score[j] *= inv;
      choice[j] = (j < per && e < a.E) ? score[j] : -INFINITY;
    }
  } else if (a.n_group > 1 && a.topk_group < a.n_group) {
    // group-limited routing: keep the topk_group groups with the best top-2 sums
    const int gsize = a.E / a.n_group;
    __shared__ float gscore_s[8][64];
    float* gscore = gscore_s[threadIdx.x >> 5];
    for (int g = 0; g < a.n_group; ++g) {
      float b1 = -INFINITY, b2 = -INFINITY;
#pragma unroll
      for (int j = 0; j < kMaxPerLane; ++j) {
        const int e = j * 32 + lane;
        if (e < a.E && e / gsize == g) {
          const float c = choice[j];
          if (c > b1) b2 = b1, b1 = c;
          else if (c > b2) b2 = c;
        }
      }
      // warp top-2 merge
      for (int o = 16; o > 0; o >>= 1) {
        const float o1 = __shfl_xor_sync(0xffffffffu, b1, o);
        const float o2 = __shfl_xor_sync(0xffffffffu, b2, o);
        float n1 = fmaxf(b1, o1);
        float n2 = fmaxf(fminf(b1, o1), fmaxf(b2, o2));
        b1 = n1, b2 = n2;
      }
      if (lane == 0) gscore[g] = b1 + b2;
    }
    __syncwarp();
    // mark the kept groups
    unsigned long long keep = 0ull;
    for (int r = 0; r < a.topk_group; ++r) {
      int best = -1;
      float bv = -INFINITY;
      for (int g = 0; g < a.n_group; ++g)
        if (!((keep >> g) & 1ull) && gscore[g] > bv) bv = gscore[g], best = g;
      if (best >= 0) keep |= 1ull << best;
    }
#pragma unroll
    for (int j = 0; j < kMaxPerLane; ++j) {
      const int e = j * 32 + lane;
      if (e < a.E && !((keep >> (e / gsize)) & 1ull)) choice[j] = -INFINITY;
    }
  }
  // top-k by repeated warp argmax over `choice`
  float wsum = 0.f;
  float my_w = 0.f;
  int my_id = 0;
  for (int r = 0; r < a.k; ++r) {
    float v = -INFINITY;
    int idx = 0x7fffffff;
#pragma unroll
    for (int j = 0; j < kMaxPerLane; ++j) {
      const int e = j * 32 + lane;
      if (choice[j] > v) v = choice[j], idx = e;
    }
    warp_argmax(v, idx);
    // fetch the weight (unbiased score) of the winner from its owner lane
    float w = 0.f;
#pragma unroll
    for (int j = 0; j < kMaxPerLane; ++j) {
      const int e = j * 32 + lane;
      if (e == idx) {
        w = score[j];
        choice[j] = -INFINITY;
      }
    }
    w = warp_sum(w);  // exactly one lane contributed
    wsum += w;
    if (lane == r) my_w = w, my_id = idx;
  }
  float scale = a.routed_scale;
  if (a.renormalize) scale = scale / (wsum + 1e-20f);
  if (lane < a.k) {
    a.topk_w[static_cast<int64_t>(t) * a.k + lane] = my_w * scale;
    a.topk_ids[static_cast<int64_t>(t) * a.k + lane] = my_id;
  }
}

// One CTA: histogram of expert ids, padded exclusive scan, tile table,
// scatter of the pairs (order inside an expert segment follows atomics; the
// combine step sums a token's k rows in slot order, so results do not
// depend on it).
constexpr int kAlignThreads = 1024;
constexpr int kMaxExperts = 1024;

__global__ void __launch_bounds__(kAlignThreads) moe_align_kernel(MoeAlignArgs a) {
  pdl_launch_dependents();
  pdl_wait();
  __shared__ int cnt[kMaxExperts];
  __shared__ int off[kMaxExperts + 1];
  __shared__ int tiles_before[kMaxExperts + 1];
  const int n = a.T * a.k;
  const int P = n + a.E * (a.tile - 1);
  for (int e = threadIdx.x; e < a.E; e += blockDim.x) cnt[e] = 0;
  __syncthreads();
  // ids outside [0, E) (experts held by another rank under expert
  // parallelism) are dropped: no row, pair_pos -1, no share in the combine
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const int e = a.topk_ids[i];
    if (e >= 0 && e < a.E) atomicAdd(&cnt[e], 1);
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    int rows = 0, tiles = 0;
    for (int e = 0; e < a.E; ++e) {
      off[e] = rows;
      tiles_before[e] = tiles;
      const int t = (cnt[e] + a.tile - 1) / a.tile;
      rows += t * a.tile;
      tiles += t;
    }
    off[a.E] = rows;
    tiles_before[a.E] = tiles;
    *a.num_tiles = tiles;
  }
  __syncthreads();
  // tile table and padding rows
  for (int e = threadIdx.x; e < a.E; e += blockDim.x) {
    for (int t = tiles_before[e]; t < tiles_before[e + 1]; ++t) {
      a.tile_expert[t] = e;
      a.tile_row[t] = off[e] + (t - tiles_before[e]) * a.tile;
    }
    for (int r = off[e] + cnt[e]; r < off[e + 1]; ++r) a.sorted_pair[r] = -1;
  }
  for (int r = off[a.E] + threadIdx.x; r < P; r += blockDim.x) a.sorted_pair[r] = -1;
  __syncthreads();
  for (int e = threadIdx.x; e < a.E; e += blockDim.x) cnt[e] = 0;  // reused as cursors
  __syncthreads();
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const int e = a.topk_ids[i];
    if (e < 0 || e >= a.E) {
      a.pair_pos[i] = -1;
      continue;
    }
    const int r = off[e] + atomicAdd(&cnt[e], 1);
    a.sorted_pair[r] = i;
    a.pair_pos[i] = r;
  }
}

// one warp per sorted row, 16-byte vectors
__global__ void moe_gather_kernel(uint4* xs, const uint4* x, const int32_t* sorted_pair, int P, int k, int vecs) {
  pdl_launch_dependents();
  pdl_wait();
  const int r = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (r >= P) return;
  const int lane = threadIdx.x & 31;
  const int pair = sorted_pair[r];
  uint4* dst = xs + static_cast<int64_t>(r) * vecs;
  if (pair < 0) {
    for (int v = lane; v < vecs; v += 32) dst[v] = make_uint4(0, 0, 0, 0);
    return;
  }
  const uint4* src = x + static_cast<int64_t>(pair / k) * vecs;
  for (int v = lane; v < vecs; v += 32) dst[v] = src[v];
}

// one CTA per token; each thread owns 8 consecutive features
__global__ void moe_combine_kernel(__nv_bfloat16* out, const __nv_bfloat16* ys, const float* topk_w,
                                   const int32_t* pair_pos, int k, int H) {
  pdl_launch_dependents();
  pdl_wait();
  const int t = blockIdx.x;
  for (int c = threadIdx.x * 8; c < H; c += blockDim.x * 8) {
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    for (int j = 0; j < k; ++j) {
      const float w = topk_w[t * k + j];
      const int r = pair_pos[t * k + j];
      if (r < 0) continue;  // expert on another rank
      const uint4 raw = *reinterpret_cast<const uint4*>(ys + static_cast<int64_t>(r) * H + c);
      const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&raw);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float2 f = __bfloat1622float2(h[q]);
        acc[2 * q] += w * f.x;
        acc[2 * q + 1] += w * f.y;
      }
    }
    uint4 pk;
    pk.x = pack_bf16x2(acc[0], acc[1]);
    pk.y = pack_bf16x2(acc[2], acc[3]);
    pk.z = pack_bf16x2(acc[4], acc[5]);
    pk.w = pack_bf16x2(acc[6], acc[7]);
    *reinterpret_cast<uint4*>(out + static_cast<int64_t>(t) * H + c) = pk;
  }
}

}  // namespace

void launch_moe_align(const MoeAlignArgs& a, cudaStream_t s) {
  if (a.E > kMaxExperts) throw std::runtime_error("minisgl.moe_align: at most 1024 experts");
  if (a.tile <= 0) throw std::runtime_error("minisgl.moe_align: tile must be positive");
  launch_pdl(moe_align_kernel, dim3(1), dim3(kAlignThreads), 0, s, a);
}

void launch_moe_gather(void* xs, const void* x, const int32_t* sorted_pair, int P, int k, int H, cudaStream_t s) {
  if (P <= 0) return;
  if (H % 8 != 0) throw std::runtime_error("minisgl.moe_gather: hidden size must be a multiple of 8");
  const int warps = 8;
  launch_pdl(moe_gather_kernel, dim3((P + warps - 1) / warps), dim3(warps * 32), 0, s, static_cast<uint4*>(xs),
             static_cast<const uint4*>(x), sorted_pair, P, k, H / 8);
}

void launch_moe_combine(void* out, const void* ys, const float* topk_w, const int32_t* pair_pos, int T, int k, int H,
                        cudaStream_t s) {
  if (T <= 0) return;
  if (H % 8 != 0) throw std::runtime_error("minisgl.moe_combine: hidden size must be a multiple of 8");
  const int threads = std::min(256, std::max(32, (H / 8 + 31) / 32 * 32));
  launch_pdl(moe_combine_kernel, dim3(T), dim3(threads), 0, s, static_cast<__nv_bfloat16*>(out),
             static_cast<const __nv_bfloat16*>(ys), topk_w, pair_pos, k, H);
}

void launch_moe_route(const MoeRouteArgs& a, cudaStream_t s) {
  if (a.T <= 0) return;
  if (a.E > 32 * kMaxPerLane || a.k > 32 || a.n_group > 64)
    throw std::runtime_error("minisgl.moe_route: too many experts");
  const int warps = 8;
  launch_pdl(moe_route_kernel, dim3((a.T + warps - 1) / warps), dim3(warps * 32), 0, s, a);
}

}  // namespace minisgl
