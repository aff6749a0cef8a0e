// Token sampling over fp32 logits, one CTA per request row.
//
// Replaces torch.argmax and the flashinfer softmax / top-k / top-p sampling
// calls of the reference sampler (python/minisgl/engine/sample.py:24-75).
//
// Method (exact sampling, no sort):
//   * temperature only: Gumbel-max, argmax_i(l_i / T + G_i) with
//     G_i = -log(-log(U_i)) is an exact draw from softmax(l / T)
//     (Gumbel 1954; see Maddison et al., "A* Sampling", 2014). One pass.
//   * top-k / top-p: the kept set is {i : l_i >= tau}. tau is found by a
//     most-significant-digit radix select over the order-preserving uint32
//     image of the fp32 logits (4 passes of 8 bits). For top-k the histogram
//     counts elements; for top-p it accumulates exp((l - max) / T) mass and
//     stops at the bucket where the mass from the top reaches p * Z. Gumbel-max
//     restricted to the kept set then draws the token.
// Random numbers: counter based. A per-row key comes from the SplitMix64
// finaliser (Steele, Lea and Flood, "Fast splittable pseudorandom number
// generators", OOPSLA 2014) of (seed, step, row); each column's 24-bit
// uniform is the 32-bit MurmurHash3 finaliser (Appleby) of key ^ (column *
// golden ratio), two multiplies per element so the pass stays memory bound.
#include <stdexcept>

#include "common.cuh"
#include "launch.h"
#include "ops.h"
#include "sampling_rng.cuh"

namespace minisgl {
namespace {

constexpr int kThreads = 1024;

// order-preserving map of fp32 to uint32 (larger float -> larger key)
__device__ __forceinline__ uint32_t fkey(float f) {
  const uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

struct ArgMax {
  float v;
  int i;
};
__device__ __forceinline__ ArgMax better(ArgMax a, ArgMax b) {
  // larger value wins; ties -> smaller index (matches torch.argmax)
  if (b.v > a.v || (b.v == a.v && b.i < a.i)) return b;
  return a;
}
__device__ ArgMax block_argmax(ArgMax x) {
  __shared__ float sv[32];
  __shared__ int si[32];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    ArgMax y{__shfl_xor_sync(0xffffffffu, x.v, o), __shfl_xor_sync(0xffffffffu, x.i, o)};
    x = better(x, y);
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) sv[warp] = x.v, si[warp] = x.i;
  __syncthreads();
  const int nw = blockDim.x >> 5;
  x = lane < nw ? ArgMax{sv[lane], si[lane]} : ArgMax{-INFINITY, 0x7fffffff};
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    ArgMax y{__shfl_xor_sync(0xffffffffu, x.v, o), __shfl_xor_sync(0xffffffffu, x.i, o)};
    x = better(x, y);
  }
  __syncthreads();
  return x;
}

__device__ float block_reduce_sum(float v) {
  __shared__ float s[32];
  v = warp_sum(v);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) s[warp] = v;
  __syncthreads();
  v = lane < (blockDim.x >> 5) ? s[lane] : 0.f;
  v = warp_sum(v);
  __syncthreads();
  return v;
}

__global__ void argmax_kernel(int32_t* out, const float* logits, int V, int ld) {
  pdl_launch_dependents();
  pdl_wait();
  const float* row = logits + static_cast<int64_t>(blockIdx.x) * ld;
  ArgMax best{-INFINITY, 0x7fffffff};
  for (int i = threadIdx.x; i < V; i += blockDim.x) best = better(best, ArgMax{row[i], i});
  best = block_argmax(best);
  if (threadIdx.x == 0) out[blockIdx.x] = best.i == 0x7fffffff ? 0 : best.i;
}

// Radix select: find the largest key threshold `tau` such that the selected
// statistic over {key >= tau} reaches `target` (count for top-k, mass for
// top-p). Only elements with key >= floor_key take part.
template <bool MASS>
__device__ uint32_t radix_threshold(const float* row, int V, float target, uint32_t floor_key,
                                    float mx, float inv_t) {
  __shared__ float hist[256];
  __shared__ uint32_t s_prefix;
  __shared__ float s_above;
  uint32_t prefix = 0;   // decided high bits
  float above = 0.f;     // statistic of elements strictly above the current prefix range
  for (int shift = 24; shift >= 0; shift -= 8) {
    for (int i = threadIdx.x; i < 256; i += blockDim.x) hist[i] = 0.f;
    __syncthreads();
    const uint32_t hi_mask = shift == 24 ? 0u : (0xFFFFFFFFu << (shift + 8));
    for (int i = threadIdx.x; i < V; i += blockDim.x) {
      const float l = row[i];
      const uint32_t k = fkey(l);
      if (k < floor_key || (k & hi_mask) != prefix) continue;
      const float w = MASS ? __expf((l - mx) * inv_t) : 1.f;
      atomicAdd(&hist[(k >> shift) & 0xFFu], w);
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      float acc = above;
      int bucket = 0;
      for (int bkt = 255; bkt >= 0; --bkt) {
        if (acc + hist[bkt] >= target) {
          bucket = bkt;
          break;
        }
        acc += hist[bkt];
      }
      s_prefix = prefix | (static_cast<uint32_t>(bucket) << shift);
      s_above = acc;
    }
    __syncthreads();
    prefix = s_prefix;
    above = s_above;
  }
  return prefix;
}

__global__ void sample_kernel(SampleArgs a) {
  pdl_launch_dependents();
  pdl_wait();
  const int r = blockIdx.x;
  const float* row = a.logits + static_cast<int64_t>(r) * a.ld;
  const int V = a.V;
  const float T = fmaxf(a.temperature[r], 1e-6f);
  const float inv_t = 1.f / T;
  const uint64_t step = a.step != nullptr ? static_cast<uint64_t>(*a.step) : 0ull;
  int top_k = a.top_k != nullptr ? a.top_k[r] : 0;
  float top_p = a.top_p != nullptr ? a.top_p[r] : 1.f;
  const bool use_k = top_k > 0 && top_k < V;
  const bool use_p = top_p < 1.f;

  uint32_t floor_key = 0;
  if (use_k || use_p) {
    ArgMax m{-INFINITY, 0};
    for (int i = threadIdx.x; i < V; i += blockDim.x) m = better(m, ArgMax{row[i], i});
    const float mx = block_argmax(m).v;
    if (use_k) floor_key = radix_threshold<false>(row, V, static_cast<float>(top_k), 0u, mx, inv_t);
    if (use_p) {
      float z = 0.f;
      for (int i = threadIdx.x; i < V; i += blockDim.x) {
        const float l = row[i];
        if (fkey(l) >= floor_key) z += __expf((l - mx) * inv_t);
      }
      z = block_reduce_sum(z);
      floor_key = radix_threshold<true>(row, V, top_p * z, floor_key, mx, inv_t);
    }
  }
  ArgMax best{-INFINITY, 0x7fffffff};
  const uint32_t key = row_key(a.seed, step, r);
  if ((V & 3) == 0 && (a.ld & 3) == 0) {
    const float4* row4 = reinterpret_cast<const float4*>(row);
    for (int i4 = threadIdx.x; i4 < V / 4; i4 += blockDim.x) {
      const float4 l4 = row4[i4];
      const float ls[4] = {l4.x, l4.y, l4.z, l4.w};
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const int i = i4 * 4 + q;
        if (fkey(ls[q]) < floor_key) continue;
        best = better(best, ArgMax{ls[q] * inv_t + gumbel(key, i), i});
      }
    }
  } else {
    for (int i = threadIdx.x; i < V; i += blockDim.x) {
      const float l = row[i];
      if (fkey(l) < floor_key) continue;
      best = better(best, ArgMax{l * inv_t + gumbel(key, i), i});
    }
  }
  best = block_argmax(best);
  if (threadIdx.x == 0) a.out[r] = best.i == 0x7fffffff ? 0 : best.i;
}

// Token of each row from the LM-head epilogue's per-vocab-tile partials
// (best score, its vocabulary index): the same argmax (ties to the smaller
// index) the sampling kernel takes over the whole row. CTA 0 then advances
// the step counter when any row sampled with a temperature, as the sampling
// kernel does; every reader of the counter (the GEMM) finished before this
// kernel passed griddepcontrol.wait.
__global__ void lm_sample_reduce_kernel(int32_t* out, const float* part_val, const int32_t* part_idx, int ntiles,
                                        int B, const float* temps, int64_t* step) {
  pdl_launch_dependents();
  pdl_wait();
  const int r = blockIdx.x;
  ArgMax best{-INFINITY, 0x7fffffff};
  for (int t = threadIdx.x; t < ntiles; t += blockDim.x) {
    const int64_t o = static_cast<int64_t>(r) * ntiles + t;
    best = better(best, ArgMax{part_val[o], part_idx[o]});
  }
  best = block_argmax(best);
  if (threadIdx.x == 0) out[r] = best.i == 0x7fffffff ? 0 : best.i;
  if (r == 0 && step != nullptr && temps != nullptr) {
    int any = 0;
    for (int i = threadIdx.x; i < B; i += blockDim.x) any |= temps[i] > 0.f;
    if (__syncthreads_or(any) && threadIdx.x == 0) *step += 1;
  }
}

// Split rows: CTA (c, b) scans vocabulary chunk c of row b and writes its
// best (score, index): the plain logit without temperatures (greedy), else
// logit / T + Gumbel noise of the same counter-based stream the whole-row
// kernel draws. lm_sample_reduce_kernel then picks each row's winner with
// the same tie rule, so tokens equal the whole-row kernels' tokens; a row no
// longer occupies one SM for its whole vocabulary (64 rows kept 64 SMs busy).
constexpr int kPartThreads = 256;
constexpr int kPartChunk = 8192;  // 8 float4 per thread

__global__ void __launch_bounds__(kPartThreads) sample_part_kernel(SampleArgs a, float* part_val,
                                                                   int32_t* part_idx, int nchunks, int ld) {
  pdl_launch_dependents();
  pdl_wait();
  const int b = blockIdx.y, c = blockIdx.x;
  const float* row = a.logits + static_cast<int64_t>(b) * a.ld;
  const bool greedy = a.temperature == nullptr;
  const float inv_t = greedy ? 1.f : 1.f / fmaxf(a.temperature[b], 1e-6f);
  const uint64_t step = a.step != nullptr ? static_cast<uint64_t>(*a.step) : 0ull;
  const uint32_t key = row_key(a.seed, step, b);
  const int i0 = c * kPartChunk, i1 = min(a.V, i0 + kPartChunk);
  const int off = a.index_offset;  // global index = off + local column
  ArgMax best{-INFINITY, 0x7fffffff};
  if ((a.V & 3) == 0 && (a.ld & 3) == 0) {
    const float4* row4 = reinterpret_cast<const float4*>(row);
#pragma unroll 4
    for (int i4 = i0 / 4 + static_cast<int>(threadIdx.x); i4 < i1 / 4; i4 += kPartThreads) {
      const float4 l4 = row4[i4];
      const float ls[4] = {l4.x, l4.y, l4.z, l4.w};
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const int i = off + i4 * 4 + q;
        best = better(best, ArgMax{greedy ? ls[q] : ls[q] * inv_t + gumbel(key, i), i});
      }
    }
  } else {
    for (int j = i0 + static_cast<int>(threadIdx.x); j < i1; j += kPartThreads) {
      const float l = row[j];
      const int i = off + j;
      best = better(best, ArgMax{greedy ? l : l * inv_t + gumbel(key, i), i});
    }
  }
  best = block_argmax(best);
  if (threadIdx.x == 0) {
    part_val[static_cast<int64_t>(b) * ld + c] = best.v;
    part_idx[static_cast<int64_t>(b) * ld + c] = best.i;
  }
}

// Token of each row from the packed partials of every rank's vocabulary
// shard ([ranks][B][ld] int32: fp32 value bits, then indices); the same
// argmax and step advance as lm_sample_reduce_kernel.
__global__ void shard_sample_reduce_kernel(int32_t* out, const int32_t* packed, int chunks, int ld, int ranks, int B,
                                           const float* temps, int64_t* step) {
  pdl_launch_dependents();
  pdl_wait();
  const int r = blockIdx.x;
  ArgMax best{-INFINITY, 0x7fffffff};
  for (int t = threadIdx.x; t < ranks * chunks; t += blockDim.x) {
    const int32_t* row = packed + (static_cast<int64_t>(t / chunks) * B + r) * ld;
    best = better(best, ArgMax{__int_as_float(row[t % chunks]), row[chunks + t % chunks]});
  }
  best = block_argmax(best);
  if (threadIdx.x == 0) out[r] = best.i == 0x7fffffff ? 0 : best.i;
  if (r == 0 && step != nullptr && temps != nullptr) {
    int any = 0;
    for (int i = threadIdx.x; i < B; i += blockDim.x) any |= temps[i] > 0.f;
    if (__syncthreads_or(any) && threadIdx.x == 0) *step += 1;
  }
}

__global__ void bump_step_kernel(int64_t* step) {
  pdl_launch_dependents();
  pdl_wait();  // the sampling kernel reads the counter first
  *step += 1;
}

}  // namespace

void launch_argmax(int32_t* out, const float* logits, int B, int V, int ld, cudaStream_t s) {
  if (B <= 0) return;
  launch_pdl(argmax_kernel, dim3(B), dim3(kThreads), 0, s, out, logits, V, ld);
}

void launch_lm_sample_reduce(int32_t* out, const float* part_val, const int32_t* part_idx, int ntiles, int B,
                             const float* temps, int64_t* step, cudaStream_t s) {
  if (B <= 0) return;
  launch_pdl(lm_sample_reduce_kernel, dim3(B), dim3(256), 0, s, out, part_val, part_idx, ntiles, B, temps, step);
}

int sample_split_chunks(int V) { return (V + kPartChunk - 1) / kPartChunk; }

void launch_sample_split(const SampleArgs& a, float* part_val, int32_t* part_idx, cudaStream_t s) {
  if (a.B <= 0) return;
  if (a.top_k != nullptr || a.top_p != nullptr)
    throw std::runtime_error("minisgl.sample: split rows take greedy / temperature sampling only");
  const int nchunks = sample_split_chunks(a.V);
  launch_pdl(sample_part_kernel, dim3(nchunks, a.B), dim3(kPartThreads), 0, s, a, part_val, part_idx, nchunks,
             nchunks);
  launch_lm_sample_reduce(a.out, part_val, part_idx, nchunks, a.B, a.temperature, const_cast<int64_t*>(a.step), s);
}

void launch_sample_shard_partials(const SampleArgs& a, int32_t* packed, int ld, cudaStream_t s) {
  if (a.B <= 0) return;
  const int nchunks = sample_split_chunks(a.V);
  if (ld < 2 * nchunks) throw std::runtime_error("minisgl.sample_shard: packed row too short");
  launch_pdl(sample_part_kernel, dim3(nchunks, a.B), dim3(kPartThreads), 0, s, a,
             reinterpret_cast<float*>(packed), packed + nchunks, nchunks, ld);
}

void launch_sample_shard_reduce(int32_t* out, const int32_t* packed, int chunks, int ld, int ranks, int B,
                                const float* temps, int64_t* step, cudaStream_t s) {
  if (B <= 0) return;
  launch_pdl(shard_sample_reduce_kernel, dim3(B), dim3(256), 0, s, out, packed, chunks, ld, ranks, B, temps, step);
}

void launch_sample(const SampleArgs& a, cudaStream_t s) {
  if (a.B <= 0) return;
  launch_pdl(sample_kernel, dim3(a.B), dim3(kThreads), 0, s, a);
  if (a.step != nullptr) launch_pdl(bump_step_kernel, dim3(1), dim3(1), 0, s, const_cast<int64_t*>(a.step));
}

}  // namespace minisgl
