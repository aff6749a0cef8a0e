// Memory-bound row kernels: RMSNorm, fused residual-add + RMSNorm, gated
// activations (SiLU / GELU times the up projection) and the vocab-sharded
// embedding gather.
//
// Replaces flashinfer rmsnorm / fused_add_rmsnorm (reference
// python/minisgl/layers/norm.py:8-38), silu_and_mul / gelu_and_mul
// (layers/activation.py:9-18) and the JIT index kernel
// (kernel/csrc/jit/index.cu:31-96, wrapper kernel/index.py:15-50).
//
// All kernels move 16-byte vectors and accumulate in fp32.
#include <algorithm>
#include <stdexcept>

#include "common.cuh"
#include "launch.h"
#include "ops.h"

namespace minisgl {
namespace {

template <typename T>
struct Vec {
  static constexpr int N = 16 / sizeof(T);
  using Raw = uint4;
};

template <typename T>
__device__ __forceinline__ void load_vec(const T* p, float (&v)[Vec<T>::N]) {
  const uint4 raw = *reinterpret_cast<const uint4*>(p);
  const T* e = reinterpret_cast<const T*>(&raw);
#pragma unroll
  for (int i = 0; i < Vec<T>::N; ++i) v[i] = to_f32<T>(e[i]);
}
template <typename T>
__device__ __forceinline__ void store_vec(T* p, const float (&v)[Vec<T>::N]) {
  uint4 raw;
  T* e = reinterpret_cast<T*>(&raw);
#pragma unroll
  for (int i = 0; i < Vec<T>::N; ++i) e[i] = from_f32<T>(v[i]);
  *reinterpret_cast<uint4*>(p) = raw;
}

__device__ __forceinline__ float block_sum(float v, float* red) {
  v = warp_sum(v);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) red[warp] = v;
  __syncthreads();
  const int nw = blockDim.x >> 5;
  float r = lane < nw ? red[lane] : 0.f;
  r = warp_sum(r);
  __syncthreads();
  return r;
}

// Rows up to kMaxVecs * blockDim * vec elements stay in registers (one read).
constexpr int kMaxVecs = 4;

template <typename T>
__global__ void rmsnorm_kernel(T* __restrict__ out, const T* __restrict__ x,
                               const T* __restrict__ w, int cols, int ld_x, int ld_out, float eps) {
  pdl_launch_dependents();  // let a following PDL kernel start its prologue
  pdl_wait();               // inputs come from the previous kernel
  constexpr int V = Vec<T>::N;
  __shared__ float red[32];
  const int row = blockIdx.x;
  const T* xr = x + static_cast<int64_t>(row) * ld_x;
  T* orow = out + static_cast<int64_t>(row) * ld_out;
  float v[kMaxVecs][V];
  float ss = 0.f;
#pragma unroll
  for (int k = 0; k < kMaxVecs; ++k) {
    const int c = (k * blockDim.x + threadIdx.x) * V;
    if (c < cols) {
      load_vec<T>(xr + c, v[k]);
#pragma unroll
      for (int i = 0; i < V; ++i) ss += v[k][i] * v[k][i];
    }
  }
  const float inv = rsqrtf(block_sum(ss, red) / cols + eps);
#pragma unroll
  for (int k = 0; k < kMaxVecs; ++k) {
    const int c = (k * blockDim.x + threadIdx.x) * V;
    if (c < cols) {
      float wv[V];
      if (w != nullptr) {
        load_vec<T>(w + c, wv);
      } else {
#pragma unroll
        for (int i = 0; i < V; ++i) wv[i] = 1.f;
      }
#pragma unroll
      for (int i = 0; i < V; ++i) v[k][i] = v[k][i] * inv * wv[i];
      store_vec<T>(orow + c, v[k]);
    }
  }
}

template <typename T>
__global__ void fused_add_rmsnorm_kernel(T* __restrict__ x, T* __restrict__ res,
                                         const T* __restrict__ w, int cols, float eps) {
  pdl_launch_dependents();  // let a following PDL kernel start its prologue
  pdl_wait();               // inputs come from the previous kernel
  constexpr int V = Vec<T>::N;
  __shared__ float red[32];
  const int row = blockIdx.x;
  T* xr = x + static_cast<int64_t>(row) * cols;
  T* rr = res + static_cast<int64_t>(row) * cols;
  float v[kMaxVecs][V];
  float ss = 0.f;
#pragma unroll
  for (int k = 0; k < kMaxVecs; ++k) {
    const int c = (k * blockDim.x + threadIdx.x) * V;
    if (c < cols) {
      float a[V], b[V];
      load_vec<T>(xr + c, a);
      load_vec<T>(rr + c, b);
#pragma unroll
      for (int i = 0; i < V; ++i) {
        // the residual stream is kept in the activation dtype, like the
        // reference's fused_add_rmsnorm: round the sum before normalising
        v[k][i] = to_f32<T>(from_f32<T>(a[i] + b[i]));
        ss += v[k][i] * v[k][i];
      }
      store_vec<T>(rr + c, v[k]);
    }
  }
  const float inv = rsqrtf(block_sum(ss, red) / cols + eps);
#pragma unroll
  for (int k = 0; k < kMaxVecs; ++k) {
    const int c = (k * blockDim.x + threadIdx.x) * V;
    if (c < cols) {
      float wv[V];
      if (w != nullptr) {
        load_vec<T>(w + c, wv);
      } else {
#pragma unroll
        for (int i = 0; i < V; ++i) wv[i] = 1.f;
      }
#pragma unroll
      for (int i = 0; i < V; ++i) v[k][i] = v[k][i] * inv * wv[i];
      store_vec<T>(xr + c, v[k]);
    }
  }
}

__device__ __forceinline__ float silu(float x) { return x / (1.f + __expf(-x)); }
__device__ __forceinline__ float gelu(float x) { return 0.5f * x * (1.f + erff(x * 0.7071067811865476f)); }

template <typename T, int ACT>
__global__ void act_and_mul_kernel(T* __restrict__ out, const T* __restrict__ x, int rows, int d, int interleaved) {
  pdl_launch_dependents();  // let a following PDL kernel start its prologue
  pdl_wait();               // inputs come from the previous kernel
  constexpr int V = Vec<T>::N;
  const int nvec = d / V;
  const int64_t total = static_cast<int64_t>(rows) * nvec;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = i / nvec;
    const int c = static_cast<int>(i % nvec) * V;
    float g[V], u[V], o[V];
    // interleaved rows: gate block c / 64 at column 128 * (c / 64), its up block 64 later
    const int64_t gc = interleaved ? (c / 64) * 128 + c % 64 : c;
    const int64_t uc = interleaved ? gc + 64 : d + c;
    load_vec<T>(x + r * 2 * d + gc, g);
    load_vec<T>(x + r * 2 * d + uc, u);
#pragma unroll
    for (int k = 0; k < V; ++k) o[k] = (ACT == 0 ? silu(g[k]) : gelu(g[k])) * u[k];
    store_vec<T>(out + r * d + c, o);
  }
}

template <typename T>
__global__ void embedding_kernel(T* __restrict__ out, const T* __restrict__ w,
                                 const int32_t* __restrict__ ids, int hidden, int lo, int n) {
  pdl_launch_dependents();  // let a following PDL kernel start its prologue
  pdl_wait();               // inputs come from the previous kernel
  constexpr int V = Vec<T>::N;
  const int row = blockIdx.x;
  const int id = ids[row] - lo;
  const bool inside = id >= 0 && id < n;
  T* dst = out + static_cast<int64_t>(row) * hidden;
  const T* src = w + static_cast<int64_t>(inside ? id : 0) * hidden;
  for (int c = threadIdx.x * V; c < hidden; c += blockDim.x * V) {
    uint4 v = make_uint4(0, 0, 0, 0);
    if (inside) v = *reinterpret_cast<const uint4*>(src + c);
    *reinterpret_cast<uint4*>(dst + c) = v;
  }
}

int norm_threads(int cols, int vec) {
  int t = (cols / vec + kMaxVecs - 1) / kMaxVecs;
  t = (t + 31) / 32 * 32;
  return std::max(32, std::min(1024, t));
}

template <typename F>
void by_dtype(DType dt, F&& f) {
  switch (dt) {
    case DType::kBF16: f(__nv_bfloat16{}); break;
    case DType::kF16: f(__half{}); break;
    default: f(float{}); break;
  }
}

}  // namespace

void launch_rmsnorm(void* out, const void* x, const void* w, int rows, int cols, int ld_x,
                    int ld_out, float eps, DType dt, cudaStream_t s) {
  if (rows <= 0) return;
  by_dtype(dt, [&](auto tag) {
    using T = decltype(tag);
    constexpr int V = Vec<T>::N;
    if (cols % V != 0 || cols > kMaxVecs * 1024 * V) throw std::runtime_error("minisgl.rmsnorm: unsupported width");
    launch_pdl(rmsnorm_kernel<T>, dim3(rows), dim3(norm_threads(cols, V)), 0, s, static_cast<T*>(out),
               static_cast<const T*>(x), static_cast<const T*>(w), cols, ld_x, ld_out, eps);
  });
}

void launch_fused_add_rmsnorm(void* x, void* residual, const void* w, int rows, int cols,
                              float eps, DType dt, cudaStream_t s) {
  if (rows <= 0) return;
  by_dtype(dt, [&](auto tag) {
    using T = decltype(tag);
    constexpr int V = Vec<T>::N;
    if (cols % V != 0 || cols > kMaxVecs * 1024 * V) throw std::runtime_error("minisgl.rmsnorm: unsupported width");
    launch_pdl(fused_add_rmsnorm_kernel<T>, dim3(rows), dim3(norm_threads(cols, V)), 0, s, static_cast<T*>(x),
               static_cast<T*>(residual), static_cast<const T*>(w), cols, eps);
  });
}

void launch_act_and_mul(void* out, const void* x, int rows, int d, int act, bool interleaved, DType dt,
                        cudaStream_t s) {
  if (rows <= 0) return;
  by_dtype(dt, [&](auto tag) {
    using T = decltype(tag);
    constexpr int V = Vec<T>::N;
    if (d % V != 0) throw std::runtime_error("minisgl.act_and_mul: width must be a multiple of 16 bytes");
    if (interleaved && d % 64 != 0) throw std::runtime_error("minisgl.act_and_mul: interleaved width must be a multiple of 64");
    const int64_t total = static_cast<int64_t>(rows) * (d / V);
    const int threads = 256;
    const int blocks = static_cast<int>(std::min<int64_t>((total + threads - 1) / threads, 148 * 16));
    if (act == 0)
      launch_pdl(act_and_mul_kernel<T, 0>, dim3(blocks), dim3(threads), 0, s, static_cast<T*>(out),
                 static_cast<const T*>(x), rows, d, interleaved ? 1 : 0);
    else
      launch_pdl(act_and_mul_kernel<T, 1>, dim3(blocks), dim3(threads), 0, s, static_cast<T*>(out),
                 static_cast<const T*>(x), rows, d, interleaved ? 1 : 0);
  });
}

void launch_embedding(void* out, const void* w, const int32_t* ids, int num_tokens, int hidden,
                      int vocab_lo, int vocab_n, DType dt, cudaStream_t s) {
  if (num_tokens <= 0) return;
  by_dtype(dt, [&](auto tag) {
    using T = decltype(tag);
    constexpr int V = Vec<T>::N;
    if (hidden % V != 0) throw std::runtime_error("minisgl.embedding: hidden must be a multiple of 16 bytes");
    const int threads = std::min(256, std::max(32, (hidden / V + 31) / 32 * 32));
    launch_pdl(embedding_kernel<T>, dim3(num_tokens), dim3(threads), 0, s, static_cast<T*>(out),
               static_cast<const T*>(w), ids, hidden, vocab_lo, vocab_n);
  });
}

}  // namespace minisgl
