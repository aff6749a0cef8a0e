// MoE router: top-k expert selection per token, one warp per token.
//
// scoring 0 (Qwen3-MoE): softmax over experts, top-k, optional
//   renormalisation of the k weights. Replaces sgl_kernel topk_softmax and
//   the renormalise step of the reference (python/minisgl/moe/fused.py:9-29).
// scoring 1 (DeepSeek-V3 / Kimi-K2 style): sigmoid scores, selection on
//   score + correction bias, optional group-limited routing (top-2 sum per
//   group, keep topk_group groups), weights are the unbiased sigmoid scores,
//   renormalised and multiplied by routed_scale.
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

}  // namespace

void launch_moe_route(const MoeRouteArgs& a, cudaStream_t s) {
  if (a.T <= 0) return;
  if (a.E > 32 * kMaxPerLane || a.k > 32 || a.n_group > 64)
    throw std::runtime_error("minisgl.moe_route: too many experts");
  const int warps = 8;
  launch_pdl(moe_route_kernel, dim3((a.T + warps - 1) / warps), dim3(warps * 32), 0, s, a);
}

}  // namespace minisgl
