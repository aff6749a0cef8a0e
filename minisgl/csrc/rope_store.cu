// Fused per-head RMSNorm (Qwen3 q_norm / k_norm) + NeoX rotary embedding +
// paged KV-cache store, one warp per (token, head).
//
// Replaces three reference launches per layer: flashinfer rmsnorm on q and k
// (python/minisgl/layers/attention.py:47-52), flashinfer
// apply_rope_with_cos_sin_cache_inplace (layers/rotary.py:35-52) and the
// store_kv_cache JIT kernel (kernel/csrc/jit/store.cu:25-53).
//
// q heads are rewritten in place inside the fused qkv activation; k heads are
// rotated and written, together with v, straight into the paged pool whose
// per-layer layout is [pages, hk, page_size, d] (token slot = page *
// page_size + offset).
#include <stdexcept>

#include "common.cuh"
#include "launch.h"
#include "ops.h"

namespace minisgl {
namespace {

template <typename T, int D>
__global__ void rope_store_kernel(RopeStoreArgs a) {
  pdl_launch_dependents();  // let a following PDL kernel start its prologue
  pdl_wait();               // qkv comes from the previous kernel
  constexpr int E = D / 32;  // elements per lane (contiguous)
  const int warps_per_block = blockDim.x >> 5;
  const int item = blockIdx.x * warps_per_block + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  const int heads = a.hq + 2 * a.hk;
  if (item >= a.T * heads) return;
  const int t = item / heads;
  const int head = item % heads;
  T* row = static_cast<T*>(a.qkv) + static_cast<int64_t>(t) * a.ld_qkv + head * D;
  float x[E];
  {
    const T* src = row + lane * E;
#pragma unroll
    for (int i = 0; i < E; ++i) x[i] = to_f32<T>(src[i]);
  }
  const bool is_q = head < a.hq;
  const bool is_k = !is_q && head < a.hq + a.hk;

  if (is_q || is_k) {
    const T* nw = static_cast<const T*>(is_q ? a.q_norm_w : a.k_norm_w);
    if (nw != nullptr) {
      float ss = 0.f;
#pragma unroll
      for (int i = 0; i < E; ++i) ss += x[i] * x[i];
      ss = warp_sum(ss);
      const float inv = rsqrtf(ss / D + a.eps);
#pragma unroll
      for (int i = 0; i < E; ++i) {
        // round to the activation dtype between norm and rotation, as two
        // separate kernels would
        x[i] = to_f32<T>(from_f32<T>(x[i] * inv * to_f32<T>(nw[lane * E + i])));
      }
    }
    // NeoX rotation over the full head: element j pairs with j + D/2, which
    // lives in lane ^ 16.
    const int pos = a.positions[t];
    const float* cs = a.cos_sin + static_cast<int64_t>(pos) * D;
    constexpr int H = D / 2;
    const bool first = lane < 16;
#pragma unroll
    for (int i = 0; i < E; ++i) {
      const float other = __shfl_xor_sync(0xffffffffu, x[i], 16);
      const int j = (lane * E + i) % H;
      const float c = cs[j], s = cs[H + j];
      x[i] = first ? (x[i] * c - other * s) : (x[i] * c + other * s);
    }
  }

  if (is_q) {
    T* dst = row + lane * E;
#pragma unroll
    for (int i = 0; i < E; ++i) dst[i] = from_f32<T>(x[i]);
    return;
  }
  const int kvh = is_k ? head - a.hq : head - a.hq - a.hk;
  const int slot = a.out_loc[t];
  if (a.kv_slots > 0 && (slot < 0 || slot >= a.kv_slots)) {  // uniform over the warp
    if (lane == 0) ErrorSink{a.err}.report(kErrBadIndex, 931);
    return;
  }
  const int page = slot / a.page_size, off = slot % a.page_size;
  T* cache = static_cast<T*>(is_k ? a.k_cache : a.v_cache);
  T* dst = cache + ((static_cast<int64_t>(page) * a.hk + kvh) * a.page_size + off) * D + lane * E;
#pragma unroll
  for (int i = 0; i < E; ++i) dst[i] = from_f32<T>(x[i]);
  if (is_k) {
    // keep the rotated key in the activation too (used by callers that read it)
    T* kd = row + lane * E;
#pragma unroll
    for (int i = 0; i < E; ++i) kd[i] = from_f32<T>(x[i]);
  }
}

template <typename T>
void launch_typed(const RopeStoreArgs& a, cudaStream_t s) {
  const int items = a.T * (a.hq + 2 * a.hk);
  const int warps = 4;
  const int blocks = (items + warps - 1) / warps;
  switch (a.d) {
    case 64: launch_pdl(rope_store_kernel<T, 64>, dim3(blocks), dim3(warps * 32), 0, s, a); break;
    case 128: launch_pdl(rope_store_kernel<T, 128>, dim3(blocks), dim3(warps * 32), 0, s, a); break;
    case 256: launch_pdl(rope_store_kernel<T, 256>, dim3(blocks), dim3(warps * 32), 0, s, a); break;
    default: throw std::runtime_error("minisgl.rope_store: head_dim must be 64, 128 or 256");
  }
}

}  // namespace

void launch_rope_store(const RopeStoreArgs& a, cudaStream_t s) {
  if (a.T <= 0) return;
  if (a.rot_dim != a.d) throw std::runtime_error("minisgl.rope_store: rotary_dim must equal head_dim");
  switch (a.dt) {
    case DType::kBF16: launch_typed<__nv_bfloat16>(a, s); break;
    case DType::kF16: launch_typed<__half>(a, s); break;
    default: launch_typed<float>(a, s); break;
  }
}

}  // namespace minisgl
