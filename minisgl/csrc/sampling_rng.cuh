// Counter-based random numbers of the sampler, shared by the sampling kernel
// and the LM-head GEMM epilogue that samples while it computes the logits
// (both must draw the same numbers for the same (seed, step, row, column)).
//
// Row key: the SplitMix64 finaliser (Steele, Lea and Flood, "Fast
// splittable pseudorandom number generators", OOPSLA 2014) of (seed, step,
// row). Column uniform: the 32-bit MurmurHash3 finaliser (Appleby) of
// key ^ (column * golden ratio), 24 bits, open interval (0, 1).
#pragma once

#include <cstdint>

namespace minisgl {

__device__ __forceinline__ uint64_t mix64(uint64_t z) {
  z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ull;
  z = (z ^ (z >> 27)) * 0x94d049bb133111ebull;
  return z ^ (z >> 31);
}

__device__ __forceinline__ uint32_t row_key(uint64_t seed, uint64_t step, int row) {
  return static_cast<uint32_t>(mix64(seed ^ mix64(step * 0x9e3779b97f4a7c15ull + static_cast<uint64_t>(row))));
}

__device__ __forceinline__ uint32_t fmix32(uint32_t h) {
  h ^= h >> 16;
  h *= 0x85ebca6bu;
  h ^= h >> 13;
  h *= 0xc2b2ae35u;
  h ^= h >> 16;
  return h;
}

// uniform in (0, 1)
__device__ __forceinline__ float uniform(uint32_t key, int col) {
  const uint32_t r = fmix32(key ^ (static_cast<uint32_t>(col) * 0x9e3779b9u));
  return (static_cast<float>(r >> 8) + 0.5f) * (1.0f / 16777216.0f);
}

// Gumbel(0, 1) noise of column `col` in the row stream `key`
__device__ __forceinline__ float gumbel(uint32_t key, int col) { return -__logf(-__logf(uniform(key, col))); }

}  // namespace minisgl
