// Python bindings of the minisgl native library (module `minisgl._C`).
//
// Every entry point validates device, dtype, shape and contiguity of its
// tensor arguments on the host (the role of the reference's TensorMatcher,
// python/minisgl/kernel/csrc/include/minisgl/tensor.h) and then calls the
// plain launchers declared in ops.h on the current CUDA stream.
#include <cstring>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "ops.h"

namespace minisgl {
int64_t compare_key_raw(const void* a, int64_t na, int ea, const void* b, int64_t nb, int eb);
std::vector<int64_t> gemm_plan_desc(int64_t M, int64_t N, int64_t K);
}

using minisgl::DType;

namespace {

#define MSG_CHECK(cond, ...) TORCH_CHECK(cond, "minisgl: ", __VA_ARGS__)

DType dtype_of(const at::Tensor& t) {
  switch (t.scalar_type()) {
    case at::kBFloat16: return DType::kBF16;
    case at::kHalf: return DType::kF16;
    case at::kFloat: return DType::kF32;
    default: MSG_CHECK(false, "unsupported dtype ", t.scalar_type());
  }
  return DType::kF32;
}

void check_cuda(const at::Tensor& t, const char* name) {
  MSG_CHECK(t.is_cuda(), name, " must be a CUDA tensor");
}
void check_rowmajor(const at::Tensor& t, const char* name) {
  MSG_CHECK(t.dim() == 2 && t.stride(1) == 1, name, " must be a 2-D tensor with unit column stride");
}
void check_same_device(const at::Tensor& a, const at::Tensor& b) {
  MSG_CHECK(a.device() == b.device(), "tensors are on different devices");
}
void check_i32(const at::Tensor& t, const char* name) {
  check_cuda(t, name);
  MSG_CHECK(t.scalar_type() == at::kInt && t.is_contiguous(), name, " must be contiguous int32");
}
int* err_ptr(const c10::optional<at::Tensor>& err) {
  if (!err.has_value()) return nullptr;
  MSG_CHECK(err->scalar_type() == at::kInt && err->numel() >= 2 && err->is_cuda(),
            "error word must be a CUDA int32 tensor with 2 elements");
  return err->data_ptr<int>();
}
cudaStream_t stream_of(const at::Tensor& t) {
  return at::cuda::getCurrentCUDAStream(t.device().index()).stream();
}

// ------------------------------------------------------------------- GEMM
void gemm(at::Tensor out, const at::Tensor& x, const at::Tensor& w,
          const c10::optional<at::Tensor>& bias, const c10::optional<at::Tensor>& workspace,
          int64_t force_splits, int64_t force_mode, const c10::optional<at::Tensor>& err, int64_t force_bn,
          const c10::optional<at::Tensor>& trace, int64_t force_kps) {
  check_cuda(x, "x");
  check_cuda(w, "w");
  check_cuda(out, "out");
  check_same_device(x, w);
  check_same_device(x, out);
  check_rowmajor(x, "x");
  check_rowmajor(w, "w");
  check_rowmajor(out, "out");
  MSG_CHECK(x.scalar_type() == at::kBFloat16 && w.scalar_type() == at::kBFloat16,
            "gemm inputs must be bfloat16");
  MSG_CHECK(out.scalar_type() == at::kBFloat16 || out.scalar_type() == at::kFloat,
            "gemm output must be bfloat16 or float32");
  MSG_CHECK(x.size(1) == w.size(1), "gemm K mismatch: ", x.sizes(), " vs ", w.sizes());
  MSG_CHECK(out.size(0) == x.size(0) && out.size(1) == w.size(0), "gemm output shape mismatch");
  minisgl::GemmArgs a{};
  a.x = x.data_ptr();
  a.w = w.data_ptr();
  a.bias = nullptr;
  if (bias.has_value()) {
    MSG_CHECK(bias->is_cuda() && bias->scalar_type() == at::kBFloat16 && bias->is_contiguous() &&
                  bias->numel() == w.size(0),
              "bias must be a contiguous bf16 vector of N elements");
    a.bias = bias->data_ptr();
  }
  a.out = out.data_ptr();
  a.workspace = nullptr;
  a.workspace_elems = 0;
  if (workspace.has_value()) {
    MSG_CHECK(workspace->is_cuda() && workspace->scalar_type() == at::kFloat && workspace->is_contiguous(),
              "workspace must be contiguous float32");
    a.workspace = workspace->data_ptr<float>();
    a.workspace_elems = workspace->numel();
  }
  a.M = static_cast<int>(x.size(0));
  a.N = static_cast<int>(w.size(0));
  a.K = static_cast<int>(x.size(1));
  a.ldx = static_cast<int>(x.stride(0));
  a.ldw = static_cast<int>(w.stride(0));
  a.ldo = static_cast<int>(out.stride(0));
  a.out_f32 = out.scalar_type() == at::kFloat;
  a.force_splits = static_cast<int>(force_splits);
  a.force_mode = static_cast<int>(force_mode);
  a.force_bn = static_cast<int>(force_bn);
  a.force_kps = static_cast<int>(force_kps);
  a.trace = nullptr;
  if (trace.has_value()) {
    MSG_CHECK(trace->is_cuda() && trace->scalar_type() == at::kLong && trace->is_contiguous(), "trace must be CUDA int64");
    a.trace = trace->data_ptr();
  }
  a.err = err_ptr(err);
  const c10::cuda::CUDAGuard guard(x.device());
  minisgl::launch_gemm(a, stream_of(x));
}

// out = epilogue(x @ w^T (+ bias)) with the fused decode epilogues (see
// GemmEpilogue in ops.h); optional tensors are None when a kind is unused.
void gemm_fused(at::Tensor out, const at::Tensor& x, const at::Tensor& w, const c10::optional<at::Tensor>& bias,
                int64_t force_mode, int64_t force_splits, int64_t force_bn, const c10::optional<at::Tensor>& err,
                int64_t kind,
                double eps, const c10::optional<at::Tensor>& residual, const c10::optional<at::Tensor>& q_norm_w,
                const c10::optional<at::Tensor>& k_norm_w, double head_eps,
                const c10::optional<at::Tensor>& cos_sin, const c10::optional<at::Tensor>& positions,
                const c10::optional<at::Tensor>& out_loc, const c10::optional<at::Tensor>& k_cache,
                const c10::optional<at::Tensor>& v_cache, int64_t hq, int64_t hk, int64_t page_size) {
  check_cuda(x, "x");
  check_cuda(w, "w");
  check_cuda(out, "out");
  check_same_device(x, w);
  check_same_device(x, out);
  check_rowmajor(x, "x");
  check_rowmajor(w, "w");
  check_rowmajor(out, "out");
  MSG_CHECK(x.scalar_type() == at::kBFloat16 && w.scalar_type() == at::kBFloat16 &&
                out.scalar_type() == at::kBFloat16,
            "fused gemm: bf16 x, w and out");
  MSG_CHECK(x.size(1) == w.size(1), "gemm K mismatch: ", x.sizes(), " vs ", w.sizes());
  const int64_t M = x.size(0), N = w.size(0);
  MSG_CHECK(out.size(0) == M, "fused gemm: output rows");
  if (kind & minisgl::kEpiSiluMul) {
    MSG_CHECK(out.size(1) == N / 2, "silu epilogue: out must be [M, N / 2]");
  } else if (kind & minisgl::kEpiRope) {
    MSG_CHECK(out.size(1) >= hq * 128, "rope epilogue: out must hold the q heads");
  } else {
    MSG_CHECK(out.size(1) == N, "fused gemm: out must be [M, N]");
  }
  minisgl::GemmArgs a{};
  a.x = x.data_ptr();
  a.w = w.data_ptr();
  a.bias = nullptr;
  if (bias.has_value()) {
    MSG_CHECK(bias->is_cuda() && bias->scalar_type() == at::kBFloat16 && bias->is_contiguous() && bias->numel() == N,
              "bias must be a contiguous bf16 vector of N elements");
    a.bias = bias->data_ptr();
  }
  a.out = out.data_ptr();
  a.M = static_cast<int>(M);
  a.N = static_cast<int>(N);
  a.K = static_cast<int>(x.size(1));
  a.ldx = static_cast<int>(x.stride(0));
  a.ldw = static_cast<int>(w.stride(0));
  a.ldo = static_cast<int>(out.stride(0));
  a.out_f32 = false;
  a.force_splits = static_cast<int>(force_splits);
  a.force_mode = static_cast<int>(force_mode);
  a.force_bn = static_cast<int>(force_bn);
  a.err = err_ptr(err);
  minisgl::GemmEpilogue& e = a.epi;
  e.kind = static_cast<int>(kind);
  e.eps = static_cast<float>(eps);
  if (kind & minisgl::kEpiResidual) {
    MSG_CHECK(residual.has_value() && residual->is_cuda() && residual->scalar_type() == at::kBFloat16 &&
                  residual->dim() == 2 && residual->stride(1) == 1 && residual->size(0) == M &&
                  residual->size(1) == N,
              "residual epilogue: bf16 residual [M, N]");
    e.residual = residual->data_ptr();
    e.ld_res = static_cast<int>(residual->stride(0));
  }
  if (kind & minisgl::kEpiRope) {
    MSG_CHECK(cos_sin.has_value() && cos_sin->scalar_type() == at::kFloat && cos_sin->is_contiguous() &&
                  cos_sin->size(-1) == 128,
              "rope epilogue: float32 cos_sin [max_pos, 128]");
    MSG_CHECK(positions.has_value() && out_loc.has_value(), "rope epilogue: positions and out_loc");
    check_i32(*positions, "positions");
    check_i32(*out_loc, "out_loc");
    MSG_CHECK(positions->numel() == M && out_loc->numel() == M, "rope epilogue: positions / out_loc size");
    for (const auto* c : {&k_cache, &v_cache})
      MSG_CHECK(c->has_value() && (*c)->is_cuda() && (*c)->scalar_type() == at::kBFloat16 && (*c)->is_contiguous(),
                "rope epilogue: bf16 contiguous k / v cache");
    for (const auto* nw : {&q_norm_w, &k_norm_w})
      if (nw->has_value())
        MSG_CHECK((*nw)->scalar_type() == at::kBFloat16 && (*nw)->is_contiguous() && (*nw)->numel() == 128,
                  "rope epilogue: bf16 head norm weight of 128");
    e.q_norm_w = q_norm_w.has_value() ? q_norm_w->data_ptr() : nullptr;
    e.k_norm_w = k_norm_w.has_value() ? k_norm_w->data_ptr() : nullptr;
    e.head_eps = static_cast<float>(head_eps);
    e.cos_sin = cos_sin->data_ptr<float>();
    e.positions = positions->data_ptr<int32_t>();
    e.out_loc = out_loc->data_ptr<int32_t>();
    e.k_cache = k_cache->data_ptr();
    e.v_cache = v_cache->data_ptr();
    e.hq = static_cast<int>(hq);
    e.hk = static_cast<int>(hk);
    e.page_size = static_cast<int>(page_size);
    e.kv_slots = k_cache->size(0) * page_size;  // [pages, hk, page, 128]: a slot outside is reported
  }
  const c10::cuda::CUDAGuard guard(x.device());
  minisgl::launch_gemm(a, stream_of(x));
}

// Sampled tokens of the LM head without materialising logits: the GEMM's
// epilogue writes per-vocabulary-tile (best score, index) partials, a second
// kernel reduces them to one token per row (and advances the step counter
// when a row sampled with a temperature). temps = None: greedy argmax.
void gemm_sample(at::Tensor out_tokens, const at::Tensor& x, const at::Tensor& w, const c10::optional<at::Tensor>& bias,
                 const c10::optional<at::Tensor>& temps, int64_t seed, at::Tensor step, at::Tensor part_val,
                 at::Tensor part_idx, int64_t force_splits, int64_t force_bn, const c10::optional<at::Tensor>& err) {
  check_cuda(x, "x");
  check_cuda(w, "w");
  check_same_device(x, w);
  check_rowmajor(x, "x");
  check_rowmajor(w, "w");
  check_i32(out_tokens, "out_tokens");
  check_i32(part_idx, "part_idx");
  MSG_CHECK(x.scalar_type() == at::kBFloat16 && w.scalar_type() == at::kBFloat16, "gemm_sample: bf16 x and w");
  MSG_CHECK(x.size(1) == w.size(1), "gemm K mismatch");
  const int64_t M = x.size(0), N = w.size(0);
  const int64_t ntiles = (N + 127) / 128;
  MSG_CHECK(out_tokens.numel() == M, "gemm_sample: one token per row");
  MSG_CHECK(part_val.is_cuda() && part_val.scalar_type() == at::kFloat && part_val.is_contiguous() &&
                part_val.numel() >= M * ntiles && part_idx.numel() >= M * ntiles,
            "gemm_sample: partial buffers of M * ceil(N / 128) entries");
  MSG_CHECK(step.is_cuda() && step.scalar_type() == at::kLong && step.numel() == 1, "gemm_sample: int64 step counter");
  minisgl::GemmArgs a{};
  a.x = x.data_ptr();
  a.w = w.data_ptr();
  a.bias = nullptr;
  if (bias.has_value()) {
    MSG_CHECK(bias->is_cuda() && bias->scalar_type() == at::kBFloat16 && bias->is_contiguous() && bias->numel() == N,
              "bias must be a contiguous bf16 vector of N elements");
    a.bias = bias->data_ptr();
  }
  a.out = part_val.data_ptr();
  a.M = static_cast<int>(M);
  a.N = static_cast<int>(N);
  a.K = static_cast<int>(x.size(1));
  a.ldx = static_cast<int>(x.stride(0));
  a.ldw = static_cast<int>(w.stride(0));
  a.ldo = static_cast<int>(ntiles);
  a.force_splits = static_cast<int>(force_splits);
  a.force_mode = 2;
  a.force_bn = static_cast<int>(force_bn);
  a.err = err_ptr(err);
  minisgl::GemmEpilogue& e = a.epi;
  e.kind = minisgl::kEpiSample;
  const float* tp = nullptr;
  if (temps.has_value()) {
    MSG_CHECK(temps->is_cuda() && temps->scalar_type() == at::kFloat && temps->is_contiguous() && temps->numel() >= M,
              "gemm_sample: float32 temperatures per row");
    tp = temps->data_ptr<float>();
  }
  e.temps = tp;
  e.seed = static_cast<uint64_t>(seed);
  e.step = step.data_ptr<int64_t>();
  e.part_val = part_val.data_ptr<float>();
  e.part_idx = part_idx.data_ptr<int32_t>();
  e.ntiles = static_cast<int>(ntiles);
  const c10::cuda::CUDAGuard guard(x.device());
  minisgl::launch_gemm(a, stream_of(x));
  minisgl::launch_lm_sample_reduce(out_tokens.data_ptr<int32_t>(), e.part_val, e.part_idx, e.ntiles,
                                   static_cast<int>(M), tp, step.data_ptr<int64_t>(), stream_of(x));
}

// Routed experts on the expert-sorted layout: align -> gather -> grouped
// gate_up GEMM with SiLU x up in its epilogue (w1 rows interleaved in 64-row
// gate / up blocks per expert) -> grouped down GEMM -> weighted combine.
// Scratch tensors come from the caller (static shapes for CUDA graphs):
// P = T * k + E * (tile - 1) rows.
void moe_experts(at::Tensor out, const at::Tensor& x, const at::Tensor& w1, const at::Tensor& w2,
                 const at::Tensor& topk_w, const at::Tensor& topk_ids, int64_t tile, at::Tensor xs, at::Tensor h,
                 at::Tensor ys, at::Tensor sorted_pair, at::Tensor pair_pos, at::Tensor tile_expert,
                 at::Tensor tile_row, at::Tensor num_tiles, const c10::optional<at::Tensor>& err, bool combine) {
  check_cuda(x, "x");
  MSG_CHECK(x.scalar_type() == at::kBFloat16 && w1.scalar_type() == at::kBFloat16 && w2.scalar_type() == at::kBFloat16,
            "moe_experts: bf16 activations and expert weights");
  MSG_CHECK(x.is_contiguous() && w1.is_contiguous() && w2.is_contiguous() && out.is_contiguous(),
            "moe_experts: contiguous tensors");
  MSG_CHECK(w1.dim() == 3 && w2.dim() == 3 && w1.size(0) == w2.size(0) && w1.size(2) == x.size(1) &&
                w2.size(1) == x.size(1) && w1.size(1) == 2 * w2.size(2),
            "moe_experts: w1 [E, 2I, H], w2 [E, H, I]");
  const int64_t T = x.size(0), H = x.size(1), E = w1.size(0), I = w2.size(2), k = topk_ids.size(1);
  MSG_CHECK(topk_ids.scalar_type() == at::kInt && topk_ids.is_contiguous() && topk_ids.size(0) == T,
            "moe_experts: int32 topk_ids [T, k]");
  MSG_CHECK(topk_w.scalar_type() == at::kFloat && topk_w.is_contiguous() && topk_w.numel() == T * k,
            "moe_experts: float32 topk_w [T, k]");
  MSG_CHECK(I % 64 == 0 && H % 128 == 0, "moe_experts: I % 64 == 0 and H % 128 == 0");
  MSG_CHECK(tile == 16 || tile == 32 || tile == 64 || tile == 128, "moe_experts: tile of 16, 32, 64 or 128");
  const int64_t P = T * k + E * (tile - 1);
  MSG_CHECK(xs.numel() >= P * H && h.numel() >= P * I && ys.numel() >= P * H && sorted_pair.numel() >= P &&
                pair_pos.numel() >= T * k && tile_expert.numel() >= P / tile && tile_row.numel() >= P / tile &&
                num_tiles.numel() >= 1,
            "moe_experts: scratch too small");
  MSG_CHECK(!combine || (out.numel() == T * H && out.scalar_type() == at::kBFloat16), "moe_experts: out [T, H] bf16");
  const c10::cuda::CUDAGuard guard(x.device());
  cudaStream_t st = stream_of(x);
  minisgl::MoeAlignArgs al{};
  al.topk_ids = topk_ids.data_ptr<int32_t>();
  al.T = static_cast<int>(T);
  al.k = static_cast<int>(k);
  al.E = static_cast<int>(E);
  al.tile = static_cast<int>(tile);
  al.sorted_pair = sorted_pair.data_ptr<int32_t>();
  al.pair_pos = pair_pos.data_ptr<int32_t>();
  al.tile_expert = tile_expert.data_ptr<int32_t>();
  al.tile_row = tile_row.data_ptr<int32_t>();
  al.num_tiles = num_tiles.data_ptr<int32_t>();
  minisgl::launch_moe_align(al, st);
  minisgl::launch_moe_gather(xs.data_ptr(), x.data_ptr(), al.sorted_pair, static_cast<int>(P), static_cast<int>(k),
                             static_cast<int>(H), st);
  for (int pass = 0; pass < 2; ++pass) {
    minisgl::GemmArgs a{};
    a.x = pass == 0 ? xs.data_ptr() : h.data_ptr();
    a.w = pass == 0 ? w1.data_ptr() : w2.data_ptr();
    a.out = pass == 0 ? h.data_ptr() : ys.data_ptr();
    a.M = static_cast<int>(P);
    a.N = static_cast<int>(pass == 0 ? 2 * I : H);
    a.K = static_cast<int>(pass == 0 ? H : I);
    a.ldx = a.K;
    a.ldw = a.K;
    a.ldo = static_cast<int>(pass == 0 ? I : H);
    a.force_mode = 2;
    a.force_bn = static_cast<int>(tile);
    a.force_splits = 1;
    a.err = err_ptr(err);
    if (pass == 0) a.epi.kind = minisgl::kEpiSiluMul;
    a.g_tile_expert = al.tile_expert;
    a.g_tile_row = al.tile_row;
    a.g_num_tiles = al.num_tiles;
    a.g_experts = static_cast<int>(E);
    minisgl::launch_gemm(a, st);
  }
  if (combine)  // otherwise the caller reads the expert rows ys through pair_pos
    minisgl::launch_moe_combine(out.data_ptr(), ys.data_ptr(), topk_w.data_ptr<float>(), al.pair_pos,
                                static_cast<int>(T), static_cast<int>(k), static_cast<int>(H), st);
}

// -------------------------------------------------------------- MXFP4 ----
void mxfp4_quantize(at::Tensor packed, at::Tensor scales, const at::Tensor& w) {
  check_cuda(w, "w");
  MSG_CHECK(w.dim() == 3 && w.is_contiguous() && w.scalar_type() == at::kBFloat16, "mxfp4_quantize: w [E, N, K] bf16");
  const int64_t E = w.size(0), N = w.size(1), K = w.size(2);
  MSG_CHECK(K % 64 == 0, "mxfp4_quantize: K % 64 == 0");
  MSG_CHECK(packed.scalar_type() == at::kByte && packed.is_contiguous() && packed.numel() == E * N * K / 2,
            "mxfp4_quantize: packed uint8 [E, N, K / 2]");
  MSG_CHECK(scales.scalar_type() == at::kByte && scales.is_contiguous() && scales.numel() == E * N * K / 32,
            "mxfp4_quantize: scales uint8 [E, K / 64, N, 2]");
  const c10::cuda::CUDAGuard guard(w.device());
  minisgl::launch_mxfp4_quantize(packed.data_ptr(), scales.data_ptr(), w.data_ptr(), static_cast<int>(E),
                                 static_cast<int>(N), static_cast<int>(K), stream_of(w));
}

// MXFP4 routed experts: align -> gather -> gate_up (E2M1 weights expanded
// to bf16 in shared memory, SiLU x up epilogue) -> down -> weighted combine.
void moe_experts_mxfp4(at::Tensor out, const at::Tensor& x, const at::Tensor& w1q, const at::Tensor& w1s,
                       const at::Tensor& w2q, const at::Tensor& w2s, const at::Tensor& topk_w,
                       const at::Tensor& topk_ids, int64_t tile, at::Tensor xs, at::Tensor h, at::Tensor ys,
                       at::Tensor sorted_pair, at::Tensor pair_pos, at::Tensor tile_expert, at::Tensor tile_row,
                       at::Tensor num_tiles, const c10::optional<at::Tensor>& err, bool combine) {
  check_cuda(x, "x");
  MSG_CHECK(x.scalar_type() == at::kBFloat16 && x.is_contiguous(), "moe_experts_mxfp4: bf16 x");
  MSG_CHECK(w1q.scalar_type() == at::kByte && w2q.scalar_type() == at::kByte && w1s.scalar_type() == at::kByte &&
                w2s.scalar_type() == at::kByte && w1q.is_contiguous() && w2q.is_contiguous() && w1s.is_contiguous() &&
                w2s.is_contiguous(),
            "moe_experts_mxfp4: uint8 packed weights and scales");
  const int64_t T = x.size(0), H = x.size(1), E = w1q.size(0), I2 = w1q.size(1), I = I2 / 2, k = topk_ids.size(1);
  MSG_CHECK(w1q.dim() == 3 && w1q.size(2) * 2 == H && w2q.dim() == 3 && w2q.size(0) == E && w2q.size(1) == H &&
                w2q.size(2) * 2 == I && w1s.numel() == E * I2 * H / 32 && w2s.numel() == E * H * I / 32,
            "moe_experts_mxfp4: w1 packed [E, 2I, H / 2], w2 packed [E, H, I / 2] with their scales");
  MSG_CHECK(I % 64 == 0 && H % 128 == 0 && I2 % 128 == 0, "moe_experts_mxfp4: I % 64 == 0 and H % 128 == 0");
  MSG_CHECK(topk_ids.scalar_type() == at::kInt && topk_ids.is_contiguous() && topk_ids.size(0) == T,
            "moe_experts_mxfp4: int32 topk_ids [T, k]");
  MSG_CHECK(topk_w.scalar_type() == at::kFloat && topk_w.is_contiguous() && topk_w.numel() == T * k,
            "moe_experts_mxfp4: float32 topk_w [T, k]");
  MSG_CHECK(tile == 16 || tile == 32 || tile == 64 || tile == 128, "moe_experts_mxfp4: tile of 16, 32, 64 or 128");
  const int64_t P = T * k + E * (tile - 1);
  const int64_t Pp = (P + tile - 1) / tile * tile;
  MSG_CHECK(xs.numel() >= Pp * H && h.numel() >= Pp * I && ys.numel() >= Pp * H && sorted_pair.numel() >= P &&
                pair_pos.numel() >= T * k && tile_expert.numel() >= P / tile && tile_row.numel() >= P / tile &&
                num_tiles.numel() >= 1,
            "moe_experts_mxfp4: scratch too small");
  MSG_CHECK(!combine || (out.numel() == T * H && out.scalar_type() == at::kBFloat16),
            "moe_experts_mxfp4: out [T, H] bf16");
  const c10::cuda::CUDAGuard guard(x.device());
  cudaStream_t st = stream_of(x);
  minisgl::MoeAlignArgs al{};
  al.topk_ids = topk_ids.data_ptr<int32_t>();
  al.T = static_cast<int>(T);
  al.k = static_cast<int>(k);
  al.E = static_cast<int>(E);
  al.tile = static_cast<int>(tile);
  al.sorted_pair = sorted_pair.data_ptr<int32_t>();
  al.pair_pos = pair_pos.data_ptr<int32_t>();
  al.tile_expert = tile_expert.data_ptr<int32_t>();
  al.tile_row = tile_row.data_ptr<int32_t>();
  al.num_tiles = num_tiles.data_ptr<int32_t>();
  minisgl::launch_moe_align(al, st);
  minisgl::launch_moe_gather(xs.data_ptr(), x.data_ptr(), al.sorted_pair, static_cast<int>(P), static_cast<int>(k),
                             static_cast<int>(H), st);
  for (int pass = 0; pass < 2; ++pass) {
    minisgl::MoeMxfp4GemmArgs a{};
    a.x = pass == 0 ? xs.data_ptr() : h.data_ptr();
    a.packed = pass == 0 ? w1q.data_ptr() : w2q.data_ptr();
    a.scales = pass == 0 ? w1s.data_ptr() : w2s.data_ptr();
    a.out = pass == 0 ? h.data_ptr() : ys.data_ptr();
    a.P = static_cast<int>(Pp);
    a.E = static_cast<int>(E);
    a.N = static_cast<int>(pass == 0 ? I2 : H);
    a.K = static_cast<int>(pass == 0 ? H : I);
    a.ldo = static_cast<int>(pass == 0 ? I : H);
    a.tile = static_cast<int>(tile);
    a.silu = pass == 0;
    a.tile_expert = al.tile_expert;
    a.tile_row = al.tile_row;
    a.num_tiles = al.num_tiles;
    a.err = err_ptr(err);
    minisgl::launch_moe_mxfp4_gemm(a, st);
  }
  if (combine)
    minisgl::launch_moe_combine(out.data_ptr(), ys.data_ptr(), topk_w.data_ptr<float>(), al.pair_pos,
                                static_cast<int>(T), static_cast<int>(k), static_cast<int>(H), st);
}

// MXFP8 rows for the block-scaled expert GEMM: q [rows, K] E4M3 (uint8) and
// scale blocks sf [rows / tile, K / 128, 512] (E8M0), row p from x[idx[p] / k]
// (zeros where idx[p] < 0) or, without idx, from x[p].
void mx8_quantize(at::Tensor q, at::Tensor sf, const at::Tensor& x, const c10::optional<at::Tensor>& idx, int64_t k,
                  int64_t rows, int64_t tile) {
  check_cuda(x, "x");
  MSG_CHECK(x.dim() == 2 && x.is_contiguous() && x.scalar_type() == at::kBFloat16, "mx8_quantize: x [*, K] bf16");
  const int64_t K = x.size(1);
  MSG_CHECK(K % 128 == 0, "mx8_quantize: K % 128 == 0");
  MSG_CHECK(tile == 16 || tile == 32 || tile == 64 || tile == 128, "mx8_quantize: tile of 16, 32, 64 or 128");
  MSG_CHECK(rows % tile == 0, "mx8_quantize: rows must be a multiple of the tile");
  MSG_CHECK(q.scalar_type() == at::kByte && q.is_contiguous() && q.numel() >= rows * K,
            "mx8_quantize: q uint8 [rows, K]");
  MSG_CHECK(sf.scalar_type() == at::kByte && sf.is_contiguous() && sf.numel() >= rows / tile * (K / 128) * 512,
            "mx8_quantize: sf uint8 [rows / tile, K / 128, 512]");
  const int32_t* ip = nullptr;
  if (idx.has_value()) {
    check_i32(*idx, "idx");
    MSG_CHECK(idx->numel() >= rows, "mx8_quantize: idx [rows]");
    ip = idx->data_ptr<int32_t>();
  } else {
    MSG_CHECK(x.size(0) >= rows, "mx8_quantize: x has fewer than rows rows");
  }
  const c10::cuda::CUDAGuard guard(x.device());
  minisgl::launch_mx8_quantize_rows(q.data_ptr(), sf.data_ptr(), x.data_ptr(), ip, static_cast<int>(k),
                                    static_cast<int>(rows), static_cast<int>(K), static_cast<int>(tile), nullptr,
                                    stream_of(x));
}

// Block-scaled MX routed experts: align -> gather + MXFP8 quantise -> gate_up
// (tcgen05 kind::mxf8f6f4, E2M1 weights x E4M3 tokens, SiLU x up epilogue)
// -> MXFP8 quantise -> down -> weighted combine.
void moe_experts_mx(at::Tensor out, const at::Tensor& x, const at::Tensor& w1q, const at::Tensor& w1sb,
                    const at::Tensor& w2q, const at::Tensor& w2sb, const at::Tensor& topk_w, const at::Tensor& topk_ids,
                    int64_t tile, at::Tensor xq, at::Tensor xsf, at::Tensor h, at::Tensor hq, at::Tensor hsf,
                    at::Tensor ys, at::Tensor sorted_pair, at::Tensor pair_pos, at::Tensor tile_expert,
                    at::Tensor tile_row, at::Tensor num_tiles, const c10::optional<at::Tensor>& err, bool combine) {
  check_cuda(x, "x");
  MSG_CHECK(x.scalar_type() == at::kBFloat16 && x.is_contiguous(), "moe_experts_mx: bf16 x");
  for (const at::Tensor* t :
       std::initializer_list<const at::Tensor*>{&w1q, &w2q, &w1sb, &w2sb, &xq, &xsf, &hq, &hsf})
    MSG_CHECK(t->scalar_type() == at::kByte && t->is_contiguous(), "moe_experts_mx: uint8 weights, scales, rows");
  const int64_t T = x.size(0), H = x.size(1), E = w1q.size(0), I2 = w1q.size(1), I = I2 / 2, k = topk_ids.size(1);
  MSG_CHECK(w1q.dim() == 3 && w1q.size(2) * 2 == H && w2q.dim() == 3 && w2q.size(0) == E && w2q.size(1) == H &&
                w2q.size(2) * 2 == I,
            "moe_experts_mx: w1 packed [E, 2I, H / 2], w2 packed [E, H, I / 2]");
  MSG_CHECK(I % 128 == 0 && H % 128 == 0, "moe_experts_mx: I % 128 == 0 and H % 128 == 0");
  MSG_CHECK(w1sb.numel() == E * I2 * H / 32 && w2sb.numel() == E * H * I / 32,
            "moe_experts_mx: scale blocks [E, N / 128, K / 128, 512]");
  MSG_CHECK(topk_ids.scalar_type() == at::kInt && topk_ids.is_contiguous() && topk_ids.size(0) == T,
            "moe_experts_mx: int32 topk_ids [T, k]");
  MSG_CHECK(topk_w.scalar_type() == at::kFloat && topk_w.is_contiguous() && topk_w.numel() == T * k,
            "moe_experts_mx: float32 topk_w [T, k]");
  MSG_CHECK(tile == 16 || tile == 32 || tile == 64 || tile == 128, "moe_experts_mx: tile of 16, 32, 64 or 128");
  const int64_t P = T * k + E * (tile - 1);
  const int64_t Pp = (P + tile - 1) / tile * tile;
  MSG_CHECK(xq.numel() >= Pp * H && xsf.numel() >= Pp / tile * (H / 128) * 512 && h.numel() >= Pp * I &&
                hq.numel() >= Pp * I && hsf.numel() >= Pp / tile * (I / 128) * 512 && ys.numel() >= Pp * H &&
                sorted_pair.numel() >= P && pair_pos.numel() >= T * k && tile_expert.numel() >= P / tile &&
                tile_row.numel() >= P / tile && num_tiles.numel() >= 1,
            "moe_experts_mx: scratch too small");
  MSG_CHECK(h.scalar_type() == at::kBFloat16 && ys.scalar_type() == at::kBFloat16, "moe_experts_mx: bf16 h and ys");
  MSG_CHECK(!combine || (out.numel() == T * H && out.scalar_type() == at::kBFloat16),
            "moe_experts_mx: out [T, H] bf16");
  const c10::cuda::CUDAGuard guard(x.device());
  cudaStream_t st = stream_of(x);
  minisgl::MoeAlignArgs al{};
  al.topk_ids = topk_ids.data_ptr<int32_t>();
  al.T = static_cast<int>(T);
  al.k = static_cast<int>(k);
  al.E = static_cast<int>(E);
  al.tile = static_cast<int>(tile);
  al.sorted_pair = sorted_pair.data_ptr<int32_t>();
  al.pair_pos = pair_pos.data_ptr<int32_t>();
  al.tile_expert = tile_expert.data_ptr<int32_t>();
  al.tile_row = tile_row.data_ptr<int32_t>();
  al.num_tiles = num_tiles.data_ptr<int32_t>();
  minisgl::launch_moe_align(al, st);
  // rows of tiles at or beyond num_tiles are never read: only the tiles'
  // rows are gathered (P / tile tiles at most)
  const int rows = static_cast<int>(P / tile * tile);
  minisgl::launch_mx8_quantize_rows(xq.data_ptr(), xsf.data_ptr(), x.data_ptr(), al.sorted_pair, static_cast<int>(k),
                                    rows, static_cast<int>(H), static_cast<int>(tile), al.num_tiles, st);
  for (int pass = 0; pass < 2; ++pass) {
    if (pass == 1)
      minisgl::launch_mx8_quantize_rows(hq.data_ptr(), hsf.data_ptr(), h.data_ptr(), nullptr, 1, rows,
                                        static_cast<int>(I), static_cast<int>(tile), al.num_tiles, st);
    minisgl::MoeMxGemmArgs a{};
    a.xq = pass == 0 ? xq.data_ptr() : hq.data_ptr();
    a.sfx = pass == 0 ? xsf.data_ptr() : hsf.data_ptr();
    a.packed = pass == 0 ? w1q.data_ptr() : w2q.data_ptr();
    a.sfw = pass == 0 ? w1sb.data_ptr() : w2sb.data_ptr();
    a.out = pass == 0 ? h.data_ptr() : ys.data_ptr();
    a.P = static_cast<int>(Pp);
    a.E = static_cast<int>(E);
    a.N = static_cast<int>(pass == 0 ? I2 : H);
    a.K = static_cast<int>(pass == 0 ? H : I);
    a.ldo = static_cast<int>(pass == 0 ? I : H);
    a.tile = static_cast<int>(tile);
    a.silu = pass == 0;
    a.tile_expert = al.tile_expert;
    a.tile_row = al.tile_row;
    a.num_tiles = al.num_tiles;
    a.err = err_ptr(err);
    minisgl::launch_moe_mx_gemm(a, st);
  }
  if (combine)
    minisgl::launch_moe_combine(out.data_ptr(), ys.data_ptr(), topk_w.data_ptr<float>(), al.pair_pos,
                                static_cast<int>(T), static_cast<int>(k), static_cast<int>(H), st);
}

void moe_combine(at::Tensor out, const at::Tensor& ys, const at::Tensor& topk_w, const at::Tensor& pair_pos, int64_t T,
                 int64_t k) {
  check_cuda(ys, "ys");
  MSG_CHECK(ys.dim() == 2 && ys.is_contiguous() && ys.scalar_type() == at::kBFloat16 && out.is_contiguous() &&
                out.scalar_type() == at::kBFloat16 && out.numel() == T * ys.size(1),
            "moe_combine: ys [P, H] and out [T, H] bf16");
  MSG_CHECK(topk_w.scalar_type() == at::kFloat && topk_w.is_contiguous() && topk_w.numel() == T * k,
            "moe_combine: float32 topk_w [T, k]");
  check_i32(pair_pos, "pair_pos");
  MSG_CHECK(pair_pos.numel() >= T * k, "moe_combine: pair_pos [T * k]");
  const c10::cuda::CUDAGuard guard(ys.device());
  minisgl::launch_moe_combine(out.data_ptr(), ys.data_ptr(), topk_w.data_ptr<float>(), pair_pos.data_ptr<int32_t>(),
                              static_cast<int>(T), static_cast<int>(k), static_cast<int>(ys.size(1)), stream_of(ys));
}

// ------------------------------------------------ EP dispatch / return ----
minisgl::EpArgs ep_args(const at::Tensor& bases, at::Tensor epoch, int64_t rank, int64_t world, int64_t cap,
                        int64_t ids_off, int64_t rows_off, int64_t back_off, int64_t H,
                        const c10::optional<at::Tensor>& err) {
  check_cuda(bases, "bases");
  MSG_CHECK(bases.scalar_type() == at::kLong && bases.numel() == world && epoch.scalar_type() == at::kInt &&
                epoch.is_cuda(),
            "ep: int64 bases [world] and an int32 epoch on the device");
  MSG_CHECK(world >= 1 && world <= 8 && rank >= 0 && rank < world && H % 8 == 0 && cap > 0,
            "ep: 1..8 ranks, H % 8 == 0");
  MSG_CHECK(ids_off % 16 == 0 && rows_off % 16 == 0 && back_off % 16 == 0, "ep: 16-byte aligned heap regions");
  minisgl::EpArgs a{};
  a.bases = bases.data_ptr<int64_t>();
  a.epoch = reinterpret_cast<uint32_t*>(epoch.data_ptr<int32_t>());
  a.rank = static_cast<int>(rank);
  a.world = static_cast<int>(world);
  a.cap = static_cast<int>(cap);
  a.ids_off = ids_off;
  a.rows_off = rows_off;
  a.back_off = back_off;
  a.H = static_cast<int>(H);
  a.err = err_ptr(err);
  return a;
}

void ep_dispatch(const at::Tensor& bases, at::Tensor epoch, int64_t rank, int64_t world, int64_t cap, int64_t ids_off,
                 int64_t rows_off, int64_t back_off, const at::Tensor& x, const at::Tensor& topk_ids, int64_t e_local,
                 const c10::optional<at::Tensor>& err) {
  MSG_CHECK(x.is_cuda() && x.dim() == 2 && x.is_contiguous() && x.scalar_type() == at::kBFloat16,
            "ep_dispatch: x [T, H] bf16 contiguous");
  check_i32(topk_ids, "topk_ids");
  MSG_CHECK(topk_ids.dim() == 2 && topk_ids.size(0) == x.size(0), "ep_dispatch: topk_ids [T, k]");
  MSG_CHECK(topk_ids.numel() <= cap, "ep_dispatch: more pairs than the heap capacity");
  const c10::cuda::CUDAGuard guard(x.device());
  minisgl::EpArgs a = ep_args(bases, epoch, rank, world, cap, ids_off, rows_off, back_off, x.size(1), err);
  a.x = x.data_ptr();
  a.topk_ids = topk_ids.data_ptr<int32_t>();
  a.T = static_cast<int>(x.size(0));
  a.k = static_cast<int>(topk_ids.size(1));
  a.e_local = static_cast<int>(e_local);
  minisgl::launch_ep_dispatch(a, stream_of(x));
}

void ep_return(const at::Tensor& bases, at::Tensor epoch, int64_t rank, int64_t world, int64_t cap, int64_t ids_off,
               int64_t rows_off, int64_t back_off, const at::Tensor& ys, const at::Tensor& pair_pos,
               const c10::optional<at::Tensor>& err) {
  MSG_CHECK(ys.is_cuda() && ys.dim() == 2 && ys.is_contiguous() && ys.scalar_type() == at::kBFloat16,
            "ep_return: ys [P, H] bf16 contiguous");
  check_i32(pair_pos, "pair_pos");
  MSG_CHECK(pair_pos.numel() >= world * cap, "ep_return: pair_pos of world * cap slots");
  const c10::cuda::CUDAGuard guard(ys.device());
  minisgl::EpArgs a = ep_args(bases, epoch, rank, world, cap, ids_off, rows_off, back_off, ys.size(1), err);
  a.ys = ys.data_ptr();
  a.pair_pos = pair_pos.data_ptr<int32_t>();
  minisgl::launch_ep_return(a, stream_of(ys));
}

// ---------------------------------------------------------------- MLA ----
// Grouped GEMM over G uniform groups: out[g] = x[g] @ w[g]^T with x rows of
// group g at [g * rows_pad, + rows_pad) and w [G, N, K]; the tile tables map
// each token tile to its group (weight-major tiles of `tile` rows).
void grouped_gemm(at::Tensor out, const at::Tensor& x, const at::Tensor& w, int64_t tile,
                  const at::Tensor& tile_expert, const at::Tensor& tile_row, const at::Tensor& num_tiles,
                  const c10::optional<at::Tensor>& err) {
  check_cuda(x, "x");
  MSG_CHECK(x.scalar_type() == at::kBFloat16 && w.scalar_type() == at::kBFloat16 && out.scalar_type() == at::kBFloat16,
            "grouped_gemm: bf16 tensors");
  MSG_CHECK(x.dim() == 2 && out.dim() == 2 && w.dim() == 3 && x.is_contiguous() && w.is_contiguous() &&
                out.is_contiguous() && w.size(2) == x.size(1) && out.size(0) == x.size(0) && out.size(1) == w.size(1),
            "grouped_gemm: x [R, K], w [G, N, K], out [R, N] contiguous");
  MSG_CHECK(tile == 16 || tile == 32 || tile == 64 || tile == 128, "grouped_gemm: tile of 16, 32, 64 or 128");
  check_i32(tile_expert, "tile_expert");
  check_i32(tile_row, "tile_row");
  check_i32(num_tiles, "num_tiles");
  const c10::cuda::CUDAGuard guard(x.device());
  minisgl::GemmArgs a{};
  a.x = x.data_ptr();
  a.w = w.data_ptr();
  a.out = out.data_ptr();
  a.M = static_cast<int>(x.size(0));
  a.N = static_cast<int>(w.size(1));
  a.K = static_cast<int>(w.size(2));
  a.ldx = a.K;
  a.ldw = a.K;
  a.ldo = a.N;
  a.force_mode = 2;
  a.force_bn = static_cast<int>(tile);
  a.force_splits = 1;
  a.err = err_ptr(err);
  a.g_tile_expert = tile_expert.data_ptr<int32_t>();
  a.g_tile_row = tile_row.data_ptr<int32_t>();
  a.g_num_tiles = num_tiles.data_ptr<int32_t>();
  a.g_experts = static_cast<int>(w.size(0));
  minisgl::launch_gemm(a, stream_of(x));
}

void mla_prepare(at::Tensor q_pe, at::Tensor xs, const at::Tensor& q, const at::Tensor& kv_a, const at::Tensor& norm_w,
                 double eps, const at::Tensor& positions, const at::Tensor& cos_sin, at::Tensor latent,
                 const at::Tensor& out_loc, int64_t T_pad, const c10::optional<at::Tensor>& err, int64_t cp_size,
                 int64_t cp_rank) {
  check_cuda(q, "q");
  MSG_CHECK(q.dim() == 3 && q.stride(2) == 1 && q.stride(1) == q.size(2) && q.scalar_type() == at::kBFloat16,
            "mla_prepare: q [T, H, nope + rope] bf16 with packed heads");
  const int64_t T = q.size(0), H = q.size(1);
  MSG_CHECK(kv_a.dim() == 2 && kv_a.stride(1) == 1 && kv_a.size(0) == T && kv_a.scalar_type() == at::kBFloat16,
            "mla_prepare: kv_a [T, kv_lora + rope] bf16");
  MSG_CHECK(latent.dim() == 3 && latent.is_contiguous() && latent.size(2) == kv_a.size(1) &&
                latent.scalar_type() == at::kBFloat16,
            "mla_prepare: latent [pages, page, kv_lora + rope] bf16 contiguous");
  const int64_t rope = q_pe.size(2), kv_lora = kv_a.size(1) - rope, nope = q.size(2) - rope;
  MSG_CHECK(q_pe.is_contiguous() && q_pe.size(0) == T && q_pe.size(1) == H, "mla_prepare: q_pe [T, H, rope]");
  MSG_CHECK(xs.is_contiguous() && xs.numel() >= H * T_pad * nope && T_pad >= T, "mla_prepare: xs [H, T_pad, nope]");
  MSG_CHECK(norm_w.numel() == kv_lora && norm_w.scalar_type() == at::kBFloat16, "mla_prepare: bf16 norm weight");
  MSG_CHECK(cos_sin.scalar_type() == at::kFloat && cos_sin.is_contiguous() && cos_sin.size(1) == rope,
            "mla_prepare: fp32 cos_sin [max_pos, rope]");
  check_i32(positions, "positions");
  check_i32(out_loc, "out_loc");
  MSG_CHECK(positions.numel() >= T && out_loc.numel() >= T, "mla_prepare: positions / out_loc of T tokens");
  const c10::cuda::CUDAGuard guard(q.device());
  minisgl::MlaPrepareArgs a{};
  a.q = q.data_ptr();
  a.ld_q = static_cast<int>(q.stride(0));
  a.kv_a = kv_a.data_ptr();
  a.ld_kv_a = static_cast<int>(kv_a.stride(0));
  a.norm_w = norm_w.data_ptr();
  a.eps = static_cast<float>(eps);
  a.positions = positions.data_ptr<int32_t>();
  a.cos_sin = cos_sin.data_ptr<float>();
  a.latent = latent.data_ptr();
  a.out_loc = out_loc.data_ptr<int32_t>();
  a.q_pe = q_pe.data_ptr();
  a.xs = xs.data_ptr();
  a.T = static_cast<int>(T);
  a.T_pad = static_cast<int>(T_pad);
  a.H = static_cast<int>(H);
  a.nope = static_cast<int>(nope);
  a.kv_lora = static_cast<int>(kv_lora);
  a.rope = static_cast<int>(rope);
  a.cp_size = static_cast<int>(cp_size);
  a.cp_rank = static_cast<int>(cp_rank);
  a.page_size = static_cast<int>(latent.size(1));
  a.num_slots = latent.size(0) * latent.size(1);
  a.err = err_ptr(err);
  minisgl::launch_mla_prepare(a, stream_of(q));
}

// Key rows only: the normalised, rotated latent rows of T tokens into the
// cache (token-sharded context parallelism stores a rank's own tokens).
void mla_store_latent(const at::Tensor& kv_a, const at::Tensor& norm_w, double eps, const at::Tensor& positions,
                      const at::Tensor& cos_sin, at::Tensor latent, const at::Tensor& out_loc,
                      const c10::optional<at::Tensor>& err, int64_t cp_size, int64_t cp_rank) {
  check_cuda(kv_a, "kv_a");
  MSG_CHECK(kv_a.dim() == 2 && kv_a.stride(1) == 1 && kv_a.scalar_type() == at::kBFloat16,
            "mla_store_latent: kv_a [T, kv_lora + rope] bf16");
  MSG_CHECK(latent.dim() == 3 && latent.is_contiguous() && latent.size(2) == kv_a.size(1) &&
                latent.scalar_type() == at::kBFloat16,
            "mla_store_latent: latent [pages, page, kv_lora + rope] bf16 contiguous");
  const int64_t T = kv_a.size(0), rope = cos_sin.size(1), kv_lora = kv_a.size(1) - rope;
  MSG_CHECK(norm_w.numel() == kv_lora && norm_w.scalar_type() == at::kBFloat16, "mla_store_latent: bf16 norm weight");
  MSG_CHECK(cos_sin.scalar_type() == at::kFloat && cos_sin.is_contiguous(), "mla_store_latent: fp32 cos_sin");
  check_i32(positions, "positions");
  check_i32(out_loc, "out_loc");
  MSG_CHECK(positions.numel() >= T && out_loc.numel() >= T, "mla_store_latent: positions / out_loc of T tokens");
  MSG_CHECK(cp_size >= 1 && cp_rank >= 0 && cp_rank < cp_size, "mla_store_latent: cp_rank outside [0, cp_size)");
  const c10::cuda::CUDAGuard guard(kv_a.device());
  minisgl::MlaPrepareArgs a{};
  a.kv_a = kv_a.data_ptr();
  a.ld_kv_a = static_cast<int>(kv_a.stride(0));
  a.norm_w = norm_w.data_ptr();
  a.eps = static_cast<float>(eps);
  a.positions = positions.data_ptr<int32_t>();
  a.cos_sin = cos_sin.data_ptr<float>();
  a.latent = latent.data_ptr();
  a.out_loc = out_loc.data_ptr<int32_t>();
  a.T = static_cast<int>(T);
  a.T_pad = static_cast<int>(T);
  a.H = 1;
  a.kv_lora = static_cast<int>(kv_lora);
  a.rope = static_cast<int>(rope);
  a.cp_size = static_cast<int>(cp_size);
  a.cp_rank = static_cast<int>(cp_rank);
  a.page_size = static_cast<int>(latent.size(1));
  a.num_slots = latent.size(0) * latent.size(1);
  a.err = err_ptr(err);
  minisgl::launch_mla_prepare(a, stream_of(kv_a));
}

// Queries only: rotated q_pe [T, H, rope] and q_nope head-major into xs.
void mla_prepare_q(at::Tensor q_pe, at::Tensor xs, const at::Tensor& q, const at::Tensor& positions,
                   const at::Tensor& cos_sin, int64_t T_pad, const c10::optional<at::Tensor>& err) {
  check_cuda(q, "q");
  MSG_CHECK(q.dim() == 3 && q.stride(2) == 1 && q.stride(1) == q.size(2) && q.scalar_type() == at::kBFloat16,
            "mla_prepare_q: q [T, H, nope + rope] bf16 with packed heads");
  const int64_t T = q.size(0), H = q.size(1), rope = q_pe.size(2), nope = q.size(2) - rope;
  MSG_CHECK(q_pe.is_contiguous() && q_pe.size(0) == T && q_pe.size(1) == H, "mla_prepare_q: q_pe [T, H, rope]");
  MSG_CHECK(xs.is_contiguous() && xs.numel() >= H * T_pad * nope && T_pad >= T, "mla_prepare_q: xs [H, T_pad, nope]");
  MSG_CHECK(cos_sin.scalar_type() == at::kFloat && cos_sin.is_contiguous() && cos_sin.size(1) == rope,
            "mla_prepare_q: fp32 cos_sin [max_pos, rope]");
  check_i32(positions, "positions");
  MSG_CHECK(positions.numel() >= T, "mla_prepare_q: positions of T tokens");
  const c10::cuda::CUDAGuard guard(q.device());
  minisgl::MlaPrepareArgs a{};
  a.q = q.data_ptr();
  a.ld_q = static_cast<int>(q.stride(0));
  a.positions = positions.data_ptr<int32_t>();
  a.cos_sin = cos_sin.data_ptr<float>();
  a.q_pe = q_pe.data_ptr();
  a.xs = xs.data_ptr();
  a.T = static_cast<int>(T);
  a.T_pad = static_cast<int>(T_pad);
  a.H = static_cast<int>(H);
  a.nope = static_cast<int>(nope);
  a.kv_lora = 512;
  a.rope = static_cast<int>(rope);
  a.cp_size = 1;
  a.err = err_ptr(err);
  minisgl::launch_mla_prepare(a, stream_of(q));
}

void mla_attention(at::Tensor out, const at::Tensor& q_lat, const at::Tensor& q_pe, const at::Tensor& latent,
                   const at::Tensor& page_table, const at::Tensor& req_rows, const at::Tensor& seq_lens,
                   const at::Tensor& cu_q, int64_t page_size, double scale, int64_t splits,
                   const c10::optional<at::Tensor>& part_o, const c10::optional<at::Tensor>& part_lse,
                   const c10::optional<at::Tensor>& err, const c10::optional<at::Tensor>& trace, int64_t cp_size,
                   int64_t cp_rank, bool combine_only, bool own_only) {
  check_cuda(q_lat, "q_lat");
  MSG_CHECK(q_lat.dim() == 3 && q_lat.is_contiguous() && q_lat.scalar_type() == at::kBFloat16,
            "mla_attention: q_lat [H, T_pad, kv_lora] bf16 contiguous");
  MSG_CHECK(q_pe.dim() == 3 && q_pe.is_contiguous() && q_pe.scalar_type() == at::kBFloat16,
            "mla_attention: q_pe [T, H, rope] bf16 contiguous");
  const int64_t H = q_lat.size(0), T_pad = q_lat.size(1), T = q_pe.size(0);
  MSG_CHECK(q_pe.size(1) == H && out.sizes() == q_lat.sizes() && out.scalar_type() == at::kBFloat16 &&
                out.is_contiguous(),
            "mla_attention: out like q_lat");
  MSG_CHECK(latent.dim() == 3 && latent.is_contiguous() && latent.size(1) == page_size &&
                latent.size(2) == q_lat.size(2) + q_pe.size(2),
            "mla_attention: latent [pages, page_size, kv_lora + rope] contiguous");
  check_i32(req_rows, "req_rows");
  check_i32(seq_lens, "seq_lens");
  check_i32(cu_q, "cu_q");
  MSG_CHECK(page_table.scalar_type() == at::kInt && page_table.dim() == 2 && page_table.stride(1) == 1,
            "mla_attention: int32 page table");
  const c10::cuda::CUDAGuard guard(q_lat.device());
  minisgl::MlaAttnArgs a{};
  a.q_lat = q_lat.data_ptr();
  a.q_pe = q_pe.data_ptr();
  a.latent = latent.data_ptr();
  a.num_slots = latent.size(0) * latent.size(1);
  a.page_table = page_table.data_ptr<int32_t>();
  a.ld_pt = static_cast<int>(page_table.stride(0));
  a.req_rows = req_rows.data_ptr<int32_t>();
  a.seq_lens = seq_lens.data_ptr<int32_t>();
  a.cu_q = cu_q.data_ptr<int32_t>();
  a.out = out.data_ptr();
  a.B = static_cast<int>(req_rows.numel());
  a.T = static_cast<int>(T);
  a.T_pad = static_cast<int>(T_pad);
  a.H = static_cast<int>(H);
  a.page_size = static_cast<int>(page_size);
  a.splits = static_cast<int>(splits);
  a.scale = static_cast<float>(scale);
  a.cp_size = static_cast<int>(cp_size);
  a.cp_rank = static_cast<int>(cp_rank);
  a.own_only = own_only ? 1 : 0;
  MSG_CHECK(cp_size >= 1 && cp_rank >= 0 && cp_rank < cp_size, "mla_attention: cp_rank outside [0, cp_size)");
  MSG_CHECK(!own_only || (combine_only && cp_size > 1), "mla_attention: own_only is a context-parallel combine");
  if (splits > 1 || cp_size > 1) {
    const int64_t parts = splits * cp_size;
    MSG_CHECK(part_o.has_value() && part_lse.has_value() && part_o->scalar_type() == at::kFloat &&
                  part_lse->scalar_type() == at::kFloat && part_o->numel() >= parts * T * H * q_lat.size(2) &&
                  part_lse->numel() >= parts * T * H,
              "mla_attention: fp32 split-KV scratch too small");
    a.part_o = part_o->data_ptr<float>();
    a.part_lse = part_lse->data_ptr<float>();
  }
  a.err = err_ptr(err);
  if (trace.has_value()) {
    MSG_CHECK(trace->scalar_type() == at::kLong && trace->is_cuda() && trace->numel() >= 64 * 8,
              "mla_attention: trace must be a CUDA int64 tensor of 512 slots");
    a.trace = reinterpret_cast<unsigned long long*>(trace->data_ptr<int64_t>());
  }
  if (combine_only) minisgl::launch_mla_combine(a, stream_of(q_lat));
  else minisgl::launch_mla_attention(a, stream_of(q_lat));
}

void mla_heads_to_rows(at::Tensor out, const at::Tensor& in, int64_t T, const c10::optional<at::Tensor>& row_map,
                       const c10::optional<at::Tensor>& err) {
  check_cuda(in, "in");
  const int64_t hv = in.size(0) * in.size(2);
  MSG_CHECK(in.dim() == 3 && in.is_contiguous() && in.scalar_type() == at::kBFloat16 && out.is_contiguous() &&
                out.scalar_type() == at::kBFloat16 && in.size(1) >= T && out.numel() % hv == 0,
            "mla_heads_to_rows: in [H, T_pad, v] -> out [rows, H * v] bf16");
  const int64_t out_rows = out.numel() / hv;
  const int32_t* map = nullptr;
  if (row_map.has_value()) {
    check_i32(*row_map, "row_map");
    MSG_CHECK(row_map->numel() >= T, "mla_heads_to_rows: a row for each of T tokens");
    map = row_map->data_ptr<int32_t>();
  } else {
    MSG_CHECK(out_rows == T, "mla_heads_to_rows: out [T, H * v] without a row map");
  }
  const c10::cuda::CUDAGuard guard(in.device());
  minisgl::launch_mla_heads_to_rows(out.data_ptr(), in.data_ptr(), static_cast<int>(T), static_cast<int>(in.size(1)),
                                    static_cast<int>(in.size(0)), static_cast<int>(in.size(2)), map,
                                    static_cast<int>(out_rows), err_ptr(err), stream_of(in));
}

// ------------------------------------------------- symmetric heap (IPC) ----
// Allocate a heap of `bytes` on the current device with zeroed signal slots;
// returns (device address, CUDA IPC handle bytes) for the other ranks.
py::tuple symm_create(int64_t bytes) {
  MSG_CHECK(bytes > minisgl::kSymmSignalBytes, "symm_create: heap too small");
  void* p = nullptr;
  cudaError_t e = cudaMalloc(&p, static_cast<size_t>(bytes));
  MSG_CHECK(e == cudaSuccess, "symm_create: cudaMalloc failed: ", cudaGetErrorString(e));
  e = cudaMemset(p, 0, static_cast<size_t>(minisgl::kSymmSignalBytes));
  MSG_CHECK(e == cudaSuccess, "symm_create: cudaMemset failed: ", cudaGetErrorString(e));
  cudaIpcMemHandle_t h;
  e = cudaIpcGetMemHandle(&h, p);
  MSG_CHECK(e == cudaSuccess, "symm_create: cudaIpcGetMemHandle failed: ", cudaGetErrorString(e));
  return py::make_tuple(reinterpret_cast<int64_t>(p),
                        py::bytes(reinterpret_cast<const char*>(&h), sizeof(cudaIpcMemHandle_t)));
}

// Map a peer's heap (same node, P2P over NVLink); returns its device address here.
int64_t symm_open(py::bytes handle) {
  const std::string raw = handle;
  MSG_CHECK(raw.size() == sizeof(cudaIpcMemHandle_t), "symm_open: bad handle");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, raw.data(), sizeof(h));
  void* p = nullptr;
  const cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
  MSG_CHECK(e == cudaSuccess, "symm_open: cudaIpcOpenMemHandle failed: ", cudaGetErrorString(e));
  return reinterpret_cast<int64_t>(p);
}

void symm_close(int64_t ptr) { cudaIpcCloseMemHandle(reinterpret_cast<void*>(ptr)); }
void symm_free(int64_t ptr) { cudaFree(reinterpret_cast<void*>(ptr)); }

// kind 0: out = sum over ranks of the partials (+ residual); kind 1:
// out = concatenation of every rank's rows. bases: int64 CUDA tensor of the
// heap addresses of all ranks (in this process's address space).
void symm_collective(int64_t kind, at::Tensor out, const c10::optional<at::Tensor>& residual, const at::Tensor& bases,
                     at::Tensor epoch, int64_t rank, int64_t world, int64_t n_elems, int64_t rows_per_rank,
                     int64_t row_elems, const c10::optional<at::Tensor>& err) {
  check_cuda(out, "out");
  MSG_CHECK(out.scalar_type() == at::kBFloat16 && out.is_contiguous(),
            "symm_collective: contiguous bf16 out (other dtypes as bf16 views)");
  MSG_CHECK(bases.is_cuda() && bases.scalar_type() == at::kLong && bases.numel() == world, "symm_collective: bases");
  MSG_CHECK(epoch.is_cuda() && epoch.scalar_type() == at::kInt && epoch.numel() == 1, "symm_collective: epoch");
  const void* res = nullptr;
  if (residual.has_value()) {
    MSG_CHECK(residual->scalar_type() == at::kBFloat16 && residual->is_contiguous() && residual->numel() == n_elems,
              "symm_collective: residual");
    res = residual->data_ptr();
  }
  MSG_CHECK(kind == 0 ? out.numel() == n_elems : out.numel() == world * rows_per_rank * row_elems,
            "symm_collective: output size");
  const c10::cuda::CUDAGuard guard(out.device());
  minisgl::launch_symm_collective(static_cast<int>(kind), bases.data_ptr<int64_t>(),
                                  reinterpret_cast<uint32_t*>(epoch.data_ptr<int32_t>()), static_cast<int>(rank),
                                  static_cast<int>(world), n_elems, out.data_ptr(), res,
                                  static_cast<int>(rows_per_rank), static_cast<int>(row_elems), err_ptr(err),
                                  stream_of(out));
}

// Reduce-scatter + residual + RMSNorm + all-gather over the symmetric heaps
// (see symm.cu). resid: this rank's residual slice [rows, hidden] bf16.
void symm_rsn(at::Tensor resid, bool add_resid, const c10::optional<at::Tensor>& norm_w, double eps,
              const at::Tensor& bases, at::Tensor epoch, int64_t rank, int64_t world, int64_t data_off,
              int64_t gather_off, const c10::optional<at::Tensor>& err) {
  check_cuda(resid, "resid");
  MSG_CHECK(resid.scalar_type() == at::kBFloat16 && resid.is_contiguous() && resid.dim() == 2,
            "symm_rsn: resid must be a contiguous bf16 [rows, hidden] tensor");
  MSG_CHECK(bases.is_cuda() && bases.scalar_type() == at::kLong && bases.numel() == world, "symm_rsn: bases");
  MSG_CHECK(epoch.is_cuda() && epoch.scalar_type() == at::kInt && epoch.numel() == 1, "symm_rsn: epoch");
  MSG_CHECK(data_off % 16 == 0 && gather_off % 16 == 0, "symm_rsn: heap offsets must be 16-byte aligned");
  const void* w = nullptr;
  if (norm_w.has_value()) {
    MSG_CHECK(norm_w->scalar_type() == at::kBFloat16 && norm_w->is_contiguous() && norm_w->numel() == resid.size(1),
              "symm_rsn: norm weight must be bf16 [hidden]");
    w = norm_w->data_ptr();
  }
  const c10::cuda::CUDAGuard guard(resid.device());
  minisgl::launch_symm_rsn(bases.data_ptr<int64_t>(), reinterpret_cast<uint32_t*>(epoch.data_ptr<int32_t>()),
                           static_cast<int>(rank), static_cast<int>(world), static_cast<int>(resid.size(0)),
                           static_cast<int>(resid.size(1)), data_off, gather_off, resid.data_ptr(), add_resid, w,
                           static_cast<float>(eps), err_ptr(err), stream_of(resid));
}

// residual += all-reduce over ranks of x @ w^T (+ bias on the caller's rank
// 0): one fused kernel when the grid is resident (see gemm.cu). epoch: int32
// [2] device counters (fused GEMM, collective kernel).
void gemm_allreduce(at::Tensor residual, const at::Tensor& x, const at::Tensor& w,
                    const c10::optional<at::Tensor>& bias, const at::Tensor& bases, at::Tensor epoch,
                    int64_t own_base, int64_t rank, int64_t world, int64_t half_bytes, int64_t force_mode,
                    int64_t force_splits, int64_t force_bn, const c10::optional<at::Tensor>& err) {
  check_cuda(x, "x");
  check_rowmajor(x, "x");
  check_rowmajor(w, "w");
  MSG_CHECK(x.scalar_type() == at::kBFloat16 && w.scalar_type() == at::kBFloat16 &&
                residual.scalar_type() == at::kBFloat16 && residual.is_contiguous(),
            "gemm_allreduce: bf16 x, w and contiguous residual");
  MSG_CHECK(x.size(1) == w.size(1) && residual.size(0) == x.size(0) && residual.size(1) == w.size(0),
            "gemm_allreduce: shapes");
  MSG_CHECK(bases.is_cuda() && bases.scalar_type() == at::kLong && bases.numel() == world, "gemm_allreduce: bases");
  MSG_CHECK(epoch.is_cuda() && epoch.scalar_type() == at::kInt && epoch.numel() == 2, "gemm_allreduce: epoch [2]");
  minisgl::GemmArgs a{};
  a.x = x.data_ptr();
  a.w = w.data_ptr();
  a.bias = bias.has_value() ? bias->data_ptr() : nullptr;
  a.M = static_cast<int>(x.size(0));
  a.N = static_cast<int>(w.size(0));
  a.K = static_cast<int>(x.size(1));
  a.ldx = static_cast<int>(x.stride(0));
  a.ldw = static_cast<int>(w.stride(0));
  a.ldo = a.N;
  a.force_mode = static_cast<int>(force_mode);
  a.force_splits = static_cast<int>(force_splits);
  a.force_bn = static_cast<int>(force_bn);
  a.err = err_ptr(err);
  const c10::cuda::CUDAGuard guard(x.device());
  minisgl::launch_gemm_allreduce(a, bases.data_ptr<int64_t>(), reinterpret_cast<uint32_t*>(epoch.data_ptr<int32_t>()),
                                 own_base, static_cast<int>(rank), static_cast<int>(world), half_bytes,
                                 residual.data_ptr(), stream_of(x));
}

int64_t gemm_workspace_elems(int64_t M, int64_t N, int64_t K) {
  return minisgl::gemm_workspace_elems(static_cast<int>(M), static_cast<int>(N), static_cast<int>(K));
}

// ------------------------------------------------------------ elementwise
// w = None: the plain normalisation (its weight folded into the next GEMM)
void rmsnorm(at::Tensor out, const at::Tensor& x, const c10::optional<at::Tensor>& w, double eps) {
  check_cuda(x, "x");
  check_rowmajor(x, "x");
  check_rowmajor(out, "out");
  if (w.has_value())
    MSG_CHECK(w->is_contiguous() && w->numel() == x.size(1) && w->scalar_type() == x.scalar_type(),
              "rmsnorm weight shape / dtype");
  MSG_CHECK(out.sizes() == x.sizes() && out.scalar_type() == x.scalar_type(), "rmsnorm dtype/shape mismatch");
  const c10::cuda::CUDAGuard guard(x.device());
  minisgl::launch_rmsnorm(out.data_ptr(), x.data_ptr(), w.has_value() ? w->data_ptr() : nullptr,
                          static_cast<int>(x.size(0)),
                          static_cast<int>(x.size(1)), static_cast<int>(x.stride(0)),
                          static_cast<int>(out.stride(0)), static_cast<float>(eps), dtype_of(x),
                          stream_of(x));
}

void fused_add_rmsnorm(at::Tensor x, at::Tensor residual, const c10::optional<at::Tensor>& w, double eps) {
  check_cuda(x, "x");
  MSG_CHECK(x.is_contiguous() && residual.is_contiguous() && x.sizes() == residual.sizes() &&
                x.dim() == 2,
            "fused_add_rmsnorm needs contiguous 2-D x and residual of equal shape");
  MSG_CHECK(x.scalar_type() == residual.scalar_type(), "fused_add_rmsnorm dtype mismatch");
  if (w.has_value())
    MSG_CHECK(w->scalar_type() == x.scalar_type() && w->numel() == x.size(1) && w->is_contiguous(),
              "fused_add_rmsnorm weight shape / dtype");
  const c10::cuda::CUDAGuard guard(x.device());
  minisgl::launch_fused_add_rmsnorm(x.data_ptr(), residual.data_ptr(), w.has_value() ? w->data_ptr() : nullptr,
                                    static_cast<int>(x.size(0)), static_cast<int>(x.size(1)),
                                    static_cast<float>(eps), dtype_of(x), stream_of(x));
}

// interleaved: gate|up columns alternate in blocks of 64 (the layout the
// fused decode GEMM uses); otherwise all gate columns, then all up columns
void act_and_mul(at::Tensor out, const at::Tensor& x, int64_t act, bool interleaved) {
  check_cuda(x, "x");
  MSG_CHECK(x.is_contiguous() && out.is_contiguous() && x.dim() == 2 && out.dim() == 2 &&
                x.size(1) == 2 * out.size(1) && x.size(0) == out.size(0) &&
                x.scalar_type() == out.scalar_type(),
            "act_and_mul shape mismatch");
  const c10::cuda::CUDAGuard guard(x.device());
  minisgl::launch_act_and_mul(out.data_ptr(), x.data_ptr(), static_cast<int>(x.size(0)),
                              static_cast<int>(out.size(1)), static_cast<int>(act), interleaved, dtype_of(x),
                              stream_of(x));
}

void embedding(at::Tensor out, const at::Tensor& w, const at::Tensor& ids, int64_t vocab_lo,
               int64_t vocab_n) {
  check_cuda(w, "weight");
  check_i32(ids, "ids");
  MSG_CHECK(w.is_contiguous() && out.is_contiguous() && out.size(0) == ids.numel() &&
                out.size(1) == w.size(1) && out.scalar_type() == w.scalar_type(),
            "embedding shape mismatch");
  const c10::cuda::CUDAGuard guard(w.device());
  minisgl::launch_embedding(out.data_ptr(), w.data_ptr(), ids.data_ptr<int32_t>(),
                            static_cast<int>(ids.numel()), static_cast<int>(w.size(1)),
                            static_cast<int>(vocab_lo), static_cast<int>(vocab_n), dtype_of(w),
                            stream_of(w));
}

// ------------------------------------------------------ rope + KV store
void rope_store(at::Tensor qkv, const at::Tensor& positions, const at::Tensor& cos_sin,
                const c10::optional<at::Tensor>& q_norm_w, const c10::optional<at::Tensor>& k_norm_w,
                at::Tensor k_cache, at::Tensor v_cache, const at::Tensor& out_loc, int64_t hq,
                int64_t hk, int64_t d, int64_t page_size, double eps, const c10::optional<at::Tensor>& err) {
  check_cuda(qkv, "qkv");
  check_rowmajor(qkv, "qkv");
  check_i32(positions, "positions");
  check_i32(out_loc, "out_loc");
  MSG_CHECK(cos_sin.scalar_type() == at::kFloat && cos_sin.is_contiguous() && cos_sin.size(1) == d,
            "cos_sin cache must be float32 [max_pos, head_dim]");
  MSG_CHECK(qkv.size(1) >= (hq + 2 * hk) * d, "qkv too narrow");
  MSG_CHECK(positions.numel() == qkv.size(0) && out_loc.numel() == qkv.size(0), "token count mismatch");
  MSG_CHECK(k_cache.scalar_type() == qkv.scalar_type() && v_cache.scalar_type() == qkv.scalar_type(),
            "cache dtype mismatch");
  minisgl::RopeStoreArgs a{};
  a.qkv = qkv.data_ptr();
  a.ld_qkv = static_cast<int>(qkv.stride(0));
  a.positions = positions.data_ptr<int32_t>();
  a.cos_sin = cos_sin.data_ptr<float>();
  a.q_norm_w = q_norm_w.has_value() ? q_norm_w->data_ptr() : nullptr;
  a.k_norm_w = k_norm_w.has_value() ? k_norm_w->data_ptr() : nullptr;
  a.k_cache = k_cache.data_ptr();
  a.v_cache = v_cache.data_ptr();
  a.out_loc = out_loc.data_ptr<int32_t>();
  a.T = static_cast<int>(qkv.size(0));
  a.hq = static_cast<int>(hq);
  a.hk = static_cast<int>(hk);
  a.d = static_cast<int>(d);
  a.rot_dim = static_cast<int>(d);
  a.page_size = static_cast<int>(page_size);
  a.eps = static_cast<float>(eps);
  a.dt = dtype_of(qkv);
  // the cache's own extent: a slot outside it is reported and not written
  a.kv_slots = k_cache.dim() >= 1 ? k_cache.size(0) * page_size : 0;
  a.err = err_ptr(err);
  const c10::cuda::CUDAGuard guard(qkv.device());
  minisgl::launch_rope_store(a, stream_of(qkv));
}

// -------------------------------------------------------------- attention
minisgl::AttnArgs attn_common(const at::Tensor& q, at::Tensor& out, const at::Tensor& kv_pool,
                              int64_t layer, const at::Tensor& page_table, const at::Tensor& req_rows,
                              const at::Tensor& seq_lens, int64_t hq, int64_t hk, int64_t d,
                              int64_t page_size, double scale) {
  check_cuda(q, "q");
  check_cuda(kv_pool, "kv_pool");
  check_i32(page_table, "page_table");
  check_i32(req_rows, "req_rows");
  check_i32(seq_lens, "seq_lens");
  MSG_CHECK(q.scalar_type() == at::kBFloat16 && kv_pool.scalar_type() == at::kBFloat16,
            "attention needs bfloat16 q and KV pool");
  MSG_CHECK(q.dim() == 2 && q.stride(1) == 1 && q.size(1) >= hq * d, "q must be [T, >= hq*d] row-major");
  MSG_CHECK(out.is_contiguous() && out.numel() == q.size(0) * hq * d, "out must be contiguous [T, hq*d]");
  // pool: [2, layers, pages, hk, page_size, d]
  MSG_CHECK(kv_pool.dim() == 6 && kv_pool.is_contiguous() && kv_pool.size(0) == 2 &&
                kv_pool.size(3) == hk && kv_pool.size(4) == page_size && kv_pool.size(5) == d,
            "kv_pool must be [2, layers, pages, hk, page_size, d]");
  MSG_CHECK(layer >= 0 && layer < kv_pool.size(1), "layer out of range");
  minisgl::AttnArgs a{};
  a.q = q.data_ptr();
  a.ld_q = static_cast<int>(q.stride(0));
  a.out = out.data_ptr();
  a.kv_pool = kv_pool.data_ptr();
  const int64_t L = kv_pool.size(1), P = kv_pool.size(2);
  const int64_t rows_per_layer = P * hk * page_size;
  a.pool_rows = 2 * L * rows_per_layer;
  a.k_row0 = layer * rows_per_layer;
  a.v_row0 = (L + layer) * rows_per_layer;
  a.page_table = page_table.data_ptr<int32_t>();
  a.ld_pt = static_cast<int>(page_table.stride(0));
  a.req_rows = req_rows.data_ptr<int32_t>();
  a.seq_lens = seq_lens.data_ptr<int32_t>();
  a.B = static_cast<int>(req_rows.numel());
  a.hq = static_cast<int>(hq);
  a.hk = static_cast<int>(hk);
  a.d = static_cast<int>(d);
  a.page_size = static_cast<int>(page_size);
  a.scale = static_cast<float>(scale);
  a.pt_rows = static_cast<int>(page_table.size(0));
  return a;
}

void decode_attention(const at::Tensor& q, at::Tensor out, const at::Tensor& kv_pool, int64_t layer,
                      const at::Tensor& page_table, const at::Tensor& req_rows,
                      const at::Tensor& seq_lens, int64_t hq, int64_t hk, int64_t d,
                      int64_t page_size, double scale, const c10::optional<at::Tensor>& part_o,
                      const c10::optional<at::Tensor>& part_lse, int64_t max_splits,
                      const c10::optional<at::Tensor>& err) {
  auto a = attn_common(q, out, kv_pool, layer, page_table, req_rows, seq_lens, hq, hk, d, page_size, scale);
  MSG_CHECK(q.size(0) == a.B, "decode attention expects one query token per request");
  a.max_splits = static_cast<int>(std::max<int64_t>(1, max_splits));
  a.part_o = nullptr;
  a.part_lse = nullptr;
  if (a.max_splits > 1) {
    MSG_CHECK(part_o.has_value() && part_lse.has_value(), "split-KV decode needs part_o and part_lse");
    MSG_CHECK(part_o->scalar_type() == at::kFloat && part_o->is_contiguous() &&
                  part_o->numel() >= static_cast<int64_t>(a.B) * hq * a.max_splits * d,
              "part_o too small");
    MSG_CHECK(part_lse->scalar_type() == at::kFloat && part_lse->is_contiguous() &&
                  part_lse->numel() >= static_cast<int64_t>(a.B) * hq * a.max_splits,
              "part_lse too small");
    a.part_o = part_o->data_ptr<float>();
    a.part_lse = part_lse->data_ptr<float>();
  }
  a.err = err_ptr(err);
  const c10::cuda::CUDAGuard guard(q.device());
  minisgl::launch_decode_attention(a, stream_of(q));
}

void prefill_attention(const at::Tensor& q, at::Tensor out, const at::Tensor& kv_pool, int64_t layer,
                       const at::Tensor& page_table, const at::Tensor& req_rows,
                       const at::Tensor& seq_lens, const at::Tensor& cu_q, int64_t max_q,
                       int64_t hq, int64_t hk, int64_t d, int64_t page_size, double scale,
                       const c10::optional<at::Tensor>& err, const c10::optional<at::Tensor>& trace) {
  auto a = attn_common(q, out, kv_pool, layer, page_table, req_rows, seq_lens, hq, hk, d, page_size, scale);
  if (trace.has_value()) {
    MSG_CHECK(trace->scalar_type() == at::kLong && trace->is_cuda() && trace->numel() >= 64 * 8,
              "prefill_attention: trace must be a CUDA int64 tensor of 512 slots");
    a.trace = reinterpret_cast<unsigned long long*>(trace->data_ptr<int64_t>());
  }
  check_i32(cu_q, "cu_q");
  MSG_CHECK(cu_q.numel() == a.B + 1, "cu_q must have B + 1 entries");
  a.cu_q = cu_q.data_ptr<int32_t>();
  a.max_q = static_cast<int>(max_q);
  a.q_rows = static_cast<int>(q.size(0));
  a.err = err_ptr(err);
  const c10::cuda::CUDAGuard guard(q.device());
  minisgl::launch_prefill_attention(a, stream_of(q));
}

// Keys of a prefill batch gathered for the kv_b expansion (row_req / row_pos
// give each compact row's request and position; -1 pads).
void mla_gather_keys(at::Tensor x, at::Tensor k_rope, const at::Tensor& latent, const at::Tensor& page_table,
                     const at::Tensor& req_rows, const at::Tensor& row_req, const at::Tensor& row_pos,
                     const c10::optional<at::Tensor>& err) {
  check_cuda(latent, "latent");
  check_i32(page_table, "page_table");
  check_i32(req_rows, "req_rows");
  check_i32(row_req, "row_req");
  check_i32(row_pos, "row_pos");
  const int64_t R = row_req.numel();
  MSG_CHECK(latent.scalar_type() == at::kBFloat16 && latent.is_contiguous() && latent.size(-1) == 576,
            "mla_gather_keys: latent [pages, page, 576] bf16");
  MSG_CHECK(x.is_contiguous() && x.scalar_type() == at::kBFloat16 && x.numel() == R * 512,
            "mla_gather_keys: x [R, 512] bf16");
  MSG_CHECK(k_rope.is_contiguous() && k_rope.scalar_type() == at::kBFloat16 && k_rope.numel() == R * 64,
            "mla_gather_keys: k_rope [R, 64] bf16");
  MSG_CHECK(row_pos.numel() == R && page_table.dim() == 2 && page_table.stride(1) == 1,
            "mla_gather_keys: row_pos of R rows, int32 page table");
  const c10::cuda::CUDAGuard guard(latent.device());
  minisgl::launch_mla_gather_keys(x.data_ptr(), k_rope.data_ptr(), latent.data_ptr(), latent.numel() / 576,
                                  page_table.data_ptr<int32_t>(), static_cast<int>(page_table.stride(0)),
                                  req_rows.data_ptr<int32_t>(), row_req.data_ptr<int32_t>(),
                                  row_pos.data_ptr<int32_t>(), static_cast<int>(R), err_ptr(err), stream_of(latent));
}

void mla_scatter_kv(at::Tensor pool, const at::Tensor& y, int64_t H) {
  check_cuda(y, "y");
  MSG_CHECK(y.scalar_type() == at::kBFloat16 && y.is_contiguous() && y.dim() == 2 && y.size(1) == H * 256,
            "mla_scatter_kv: y [R, H * 256] bf16");
  const int64_t R = y.size(0);
  MSG_CHECK(pool.scalar_type() == at::kBFloat16 && pool.is_contiguous() && pool.numel() == 2 * R * H * 128,
            "mla_scatter_kv: pool [2, R / 64, H, 64, 128] bf16");
  const c10::cuda::CUDAGuard guard(y.device());
  minisgl::launch_mla_scatter_kv(pool.data_ptr(), y.data_ptr(), static_cast<int>(R), static_cast<int>(H),
                                 stream_of(y));
}

// Rotated query rope parts only: q_pe [T, H, rope] from q [T, H, nope + rope].
void mla_rope_q(at::Tensor q_pe, const at::Tensor& q, const at::Tensor& positions, const at::Tensor& cos_sin,
                const c10::optional<at::Tensor>& err) {
  check_cuda(q, "q");
  MSG_CHECK(q.dim() == 3 && q.stride(2) == 1 && q.stride(1) == q.size(2) && q.scalar_type() == at::kBFloat16,
            "mla_rope_q: q [T, H, nope + rope] bf16 with packed heads");
  const int64_t T = q.size(0), H = q.size(1), rope = q_pe.size(2), nope = q.size(2) - rope;
  MSG_CHECK(q_pe.is_contiguous() && q_pe.size(0) == T && q_pe.size(1) == H, "mla_rope_q: q_pe [T, H, rope]");
  MSG_CHECK(cos_sin.scalar_type() == at::kFloat && cos_sin.is_contiguous() && cos_sin.size(1) == rope,
            "mla_rope_q: fp32 cos_sin [max_pos, rope]");
  check_i32(positions, "positions");
  MSG_CHECK(positions.numel() >= T, "mla_rope_q: positions of T tokens");
  const c10::cuda::CUDAGuard guard(q.device());
  minisgl::MlaPrepareArgs a{};
  a.q = q.data_ptr();
  a.ld_q = static_cast<int>(q.stride(0));
  a.positions = positions.data_ptr<int32_t>();
  a.cos_sin = cos_sin.data_ptr<float>();
  a.q_pe = q_pe.data_ptr();
  a.T = static_cast<int>(T);
  a.T_pad = static_cast<int>(T);
  a.H = static_cast<int>(H);
  a.nope = static_cast<int>(nope);
  a.kv_lora = 512;
  a.rope = static_cast<int>(rope);
  a.cp_size = 1;
  a.err = err_ptr(err);
  minisgl::launch_mla_prepare(a, stream_of(q));
}

// Non-absorbed MLA prefill: q [T, hq * qk] (q_nope first in each head),
// q_rope [T, hq, 64] rotated, K_nope / V expanded into kv_pool
// [2, 1, pages, hq, page, 128] and the keys' rope rows k_rope [slots, 64],
// both at the slots of page_table; out [T, hq * 128].
void mla_prefill_attention(const at::Tensor& q, at::Tensor out, const at::Tensor& kv_pool,
                           const at::Tensor& page_table, const at::Tensor& req_rows, const at::Tensor& seq_lens,
                           const at::Tensor& cu_q, int64_t max_q, int64_t hq, int64_t qk, int64_t page_size,
                           double scale, const at::Tensor& q_rope, const at::Tensor& k_rope,
                           const c10::optional<at::Tensor>& err) {
  auto a = attn_common(q, out, kv_pool, 0, page_table, req_rows, seq_lens, hq, hq, 128, page_size, scale);
  MSG_CHECK(q.size(1) == hq * qk && qk >= 128 + 64, "mla_prefill_attention: q [T, hq * (nope + rope)]");
  check_cuda(q_rope, "q_rope");
  check_cuda(k_rope, "k_rope");
  MSG_CHECK(q_rope.scalar_type() == at::kBFloat16 && q_rope.is_contiguous() && q_rope.numel() == q.size(0) * hq * 64,
            "mla_prefill_attention: q_rope [T, hq, 64] bf16 contiguous");
  MSG_CHECK(k_rope.scalar_type() == at::kBFloat16 && k_rope.is_contiguous() && k_rope.dim() == 2 &&
                k_rope.size(1) == 64,
            "mla_prefill_attention: k_rope [slots, 64] bf16 contiguous");
  MSG_CHECK(k_rope.size(0) >= kv_pool.size(2) * page_size, "mla_prefill_attention: k_rope covers every slot");
  check_i32(cu_q, "cu_q");
  MSG_CHECK(cu_q.numel() == a.B + 1, "cu_q must have B + 1 entries");
  a.cu_q = cu_q.data_ptr<int32_t>();
  a.max_q = static_cast<int>(max_q);
  a.q_rows = static_cast<int>(q.size(0));
  a.q_head_stride = static_cast<int>(qk);
  a.q_rope = q_rope.data_ptr();
  a.k_rope = k_rope.data_ptr();
  a.rope_rows = k_rope.size(0);
  a.err = err_ptr(err);
  const c10::cuda::CUDAGuard guard(q.device());
  minisgl::launch_mla_prefill_attention(a, stream_of(q));
}

// --------------------------------------------------------------- sampling
void argmax(at::Tensor out, const at::Tensor& logits) {
  check_cuda(logits, "logits");
  check_i32(out, "out");
  MSG_CHECK(logits.scalar_type() == at::kFloat && logits.dim() == 2 && logits.stride(1) == 1,
            "logits must be float32 [B, V]");
  MSG_CHECK(out.numel() == logits.size(0), "argmax output size");
  const c10::cuda::CUDAGuard guard(logits.device());
  const int64_t B = logits.size(0);
  if (B == 0) return;
  // rows split over vocabulary chunks (partials from torch's allocator)
  const int64_t parts = B * minisgl::sample_split_chunks(static_cast<int>(logits.size(1)));
  at::Tensor pv = at::empty({parts}, logits.options());
  at::Tensor pi = at::empty({parts}, logits.options().dtype(at::kInt));
  minisgl::SampleArgs a{};
  a.out = out.data_ptr<int32_t>();
  a.logits = logits.data_ptr<float>();
  a.ld = static_cast<int>(logits.stride(0));
  a.B = static_cast<int>(B);
  a.V = static_cast<int>(logits.size(1));
  minisgl::launch_sample_split(a, pv.data_ptr<float>(), pi.data_ptr<int32_t>(), stream_of(logits));
}

void sample(at::Tensor out, const at::Tensor& logits, const at::Tensor& temperature,
            const c10::optional<at::Tensor>& top_k, const c10::optional<at::Tensor>& top_p,
            int64_t seed, const c10::optional<at::Tensor>& step) {
  check_cuda(logits, "logits");
  check_i32(out, "out");
  MSG_CHECK(logits.scalar_type() == at::kFloat && logits.dim() == 2 && logits.stride(1) == 1,
            "logits must be float32 [B, V]");
  const int64_t B = logits.size(0);
  MSG_CHECK(out.numel() == B && temperature.numel() == B && temperature.scalar_type() == at::kFloat &&
                temperature.is_contiguous(),
            "temperature must be float32 [B]");
  minisgl::SampleArgs a{};
  a.out = out.data_ptr<int32_t>();
  a.logits = logits.data_ptr<float>();
  a.ld = static_cast<int>(logits.stride(0));
  a.B = static_cast<int>(B);
  a.V = static_cast<int>(logits.size(1));
  a.temperature = temperature.data_ptr<float>();
  a.top_k = nullptr;
  a.top_p = nullptr;
  if (top_k.has_value()) {
    check_i32(*top_k, "top_k");
    MSG_CHECK(top_k->numel() == B, "top_k size");
    a.top_k = top_k->data_ptr<int32_t>();
  }
  if (top_p.has_value()) {
    MSG_CHECK(top_p->scalar_type() == at::kFloat && top_p->numel() == B && top_p->is_contiguous(),
              "top_p must be float32 [B]");
    a.top_p = top_p->data_ptr<float>();
  }
  a.seed = static_cast<uint64_t>(seed);
  a.step = nullptr;
  if (step.has_value()) {
    MSG_CHECK(step->scalar_type() == at::kLong && step->is_cuda(), "step must be a CUDA int64 scalar");
    a.step = step->data_ptr<int64_t>();
  }
  const c10::cuda::CUDAGuard guard(logits.device());
  if (a.top_k == nullptr && a.top_p == nullptr && B > 0) {
    // plain temperature sampling: rows split over vocabulary chunks (the
    // step counter advances in the reduce, as in the LM-head sampling path)
    const int64_t parts = B * minisgl::sample_split_chunks(a.V);
    at::Tensor pv = at::empty({parts}, logits.options());
    at::Tensor pi = at::empty({parts}, logits.options().dtype(at::kInt));
    minisgl::launch_sample_split(a, pv.data_ptr<float>(), pi.data_ptr<int32_t>(), stream_of(logits));
    return;
  }
  minisgl::launch_sample(a, stream_of(logits));
}

// Vocabulary-sharded sampling: packed partials of this rank's logits shard
// (global indices from `offset`), then (after an all-gather of the packed
// rows) the tokens. temperature None: greedy.
int64_t sample_shard_chunks(int64_t v_shard) { return minisgl::sample_split_chunks(static_cast<int>(v_shard)); }

void sample_shard_partials(at::Tensor packed, const at::Tensor& logits, const c10::optional<at::Tensor>& temperature,
                           int64_t seed, const c10::optional<at::Tensor>& step, int64_t offset) {
  check_cuda(logits, "logits");
  check_i32(packed, "packed");
  MSG_CHECK(logits.scalar_type() == at::kFloat && logits.dim() == 2 && logits.stride(1) == 1,
            "logits must be float32 [B, V_shard]");
  const int64_t B = logits.size(0);
  MSG_CHECK(packed.dim() == 2 && packed.size(0) == B && packed.is_contiguous() &&
                packed.size(1) >= 2 * minisgl::sample_split_chunks(static_cast<int>(logits.size(1))),
            "packed partials must be int32 [B, >= 2 chunks]");
  minisgl::SampleArgs a{};
  a.logits = logits.data_ptr<float>();
  a.ld = static_cast<int>(logits.stride(0));
  a.B = static_cast<int>(B);
  a.V = static_cast<int>(logits.size(1));
  a.temperature = nullptr;
  if (temperature.has_value()) {
    MSG_CHECK(temperature->scalar_type() == at::kFloat && temperature->numel() >= B && temperature->is_contiguous(),
              "temperature must be float32 [B]");
    a.temperature = temperature->data_ptr<float>();
  }
  a.seed = static_cast<uint64_t>(seed);
  a.step = nullptr;
  if (step.has_value()) {
    MSG_CHECK(step->scalar_type() == at::kLong && step->is_cuda(), "step must be a CUDA int64 scalar");
    a.step = step->data_ptr<int64_t>();
  }
  a.index_offset = static_cast<int>(offset);
  const c10::cuda::CUDAGuard guard(logits.device());
  minisgl::launch_sample_shard_partials(a, packed.data_ptr<int32_t>(), static_cast<int>(packed.size(1)),
                                        stream_of(logits));
}

void sample_shard_reduce(at::Tensor out, const at::Tensor& gathered, int64_t chunks, int64_t ranks,
                         const c10::optional<at::Tensor>& temperature, const c10::optional<at::Tensor>& step) {
  check_i32(out, "out");
  check_i32(gathered, "gathered");
  const int64_t B = out.numel();
  MSG_CHECK(gathered.dim() == 2 && gathered.is_contiguous() && gathered.size(0) == ranks * B &&
                gathered.size(1) >= 2 * chunks,
            "gathered partials must be int32 [ranks * B, >= 2 chunks]");
  const float* t = nullptr;
  if (temperature.has_value()) {
    MSG_CHECK(temperature->scalar_type() == at::kFloat && temperature->numel() >= B, "temperature float32 [B]");
    t = temperature->data_ptr<float>();
  }
  int64_t* st = nullptr;
  if (step.has_value()) {
    MSG_CHECK(step->scalar_type() == at::kLong && step->is_cuda(), "step must be a CUDA int64 scalar");
    st = step->data_ptr<int64_t>();
  }
  const c10::cuda::CUDAGuard guard(gathered.device());
  minisgl::launch_sample_shard_reduce(out.data_ptr<int32_t>(), gathered.data_ptr<int32_t>(), static_cast<int>(chunks),
                                      static_cast<int>(gathered.size(1)), static_cast<int>(ranks),
                                      static_cast<int>(B), t, st, stream_of(gathered));
}

// -------------------------------------------------------------------- MoE
void moe_route(const at::Tensor& logits, const c10::optional<at::Tensor>& bias, at::Tensor topk_w,
               at::Tensor topk_ids, int64_t scoring, bool renormalize, int64_t n_group,
               int64_t topk_group, double routed_scale) {
  check_cuda(logits, "router logits");
  MSG_CHECK(logits.scalar_type() == at::kFloat && logits.is_contiguous() && logits.dim() == 2,
            "router logits must be contiguous float32 [T, E]");
  check_i32(topk_ids, "topk_ids");
  MSG_CHECK(topk_w.scalar_type() == at::kFloat && topk_w.is_contiguous() &&
                topk_w.sizes() == topk_ids.sizes() && topk_w.size(0) == logits.size(0),
            "topk output shape");
  minisgl::MoeRouteArgs a{};
  a.logits = logits.data_ptr<float>();
  a.bias = nullptr;
  if (bias.has_value()) {
    MSG_CHECK(bias->scalar_type() == at::kFloat && bias->numel() == logits.size(1), "router bias");
    a.bias = bias->data_ptr<float>();
  }
  a.topk_w = topk_w.data_ptr<float>();
  a.topk_ids = topk_ids.data_ptr<int32_t>();
  a.T = static_cast<int>(logits.size(0));
  a.E = static_cast<int>(logits.size(1));
  a.k = static_cast<int>(topk_ids.size(1));
  a.scoring = static_cast<int>(scoring);
  a.renormalize = renormalize;
  a.n_group = static_cast<int>(n_group);
  a.topk_group = static_cast<int>(topk_group);
  a.routed_scale = static_cast<float>(routed_scale);
  const c10::cuda::CUDAGuard guard(logits.device());
  minisgl::launch_moe_route(a, stream_of(logits));
}

// ------------------------------------------------------------ host helpers
int64_t fast_compare_key(const at::Tensor& a, const at::Tensor& b) {
  MSG_CHECK(a.is_cpu() && b.is_cpu() && a.dim() == 1 && b.dim() == 1, "keys must be 1-D CPU tensors");
  MSG_CHECK(a.is_contiguous() && b.is_contiguous(), "keys must be contiguous");
  const auto ea = a.element_size(), eb = b.element_size();
  MSG_CHECK((a.scalar_type() == at::kInt || a.scalar_type() == at::kLong) &&
                (b.scalar_type() == at::kInt || b.scalar_type() == at::kLong),
            "keys must be int32 or int64");
  return minisgl::compare_key_raw(a.data_ptr(), a.numel(), static_cast<int>(ea), b.data_ptr(),
                                  b.numel(), static_cast<int>(eb));
}

}  // namespace

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "minisgl native kernels for NVIDIA B200 (sm_100a)";
  m.def("gemm", &gemm, "tcgen05 bf16 GEMM: out = x @ w^T (+ bias)", py::arg("out"), py::arg("x"),
        py::arg("w"), py::arg("bias") = py::none(), py::arg("workspace") = py::none(),
        py::arg("force_splits") = 0, py::arg("force_mode") = 0, py::arg("err") = py::none(),
        py::arg("force_bn") = 0, py::arg("trace") = py::none(), py::arg("force_kps") = 0);
  m.def("gemm_plan", [](int64_t M, int64_t N, int64_t K) { return minisgl::gemm_plan_desc(M, N, K); });
  m.def("gemm_workspace_elems", &gemm_workspace_elems);
  m.def("rmsnorm", &rmsnorm);
  m.def("fused_add_rmsnorm", &fused_add_rmsnorm);
  m.def("act_and_mul", &act_and_mul, py::arg("out"), py::arg("x"), py::arg("act"), py::arg("interleaved") = false);
  m.def("embedding", &embedding);
  m.def("rope_store", &rope_store, py::arg("qkv"), py::arg("positions"), py::arg("cos_sin"), py::arg("q_norm_w"),
        py::arg("k_norm_w"), py::arg("k_cache"), py::arg("v_cache"), py::arg("out_loc"), py::arg("hq"),
        py::arg("hk"), py::arg("d"), py::arg("page_size"), py::arg("eps"), py::arg("err") = py::none());
  m.def("decode_attention", &decode_attention);
  m.def("gemm_fused", &gemm_fused);
  m.def("gemm_sample", &gemm_sample);
  m.def("moe_experts", &moe_experts, py::arg("out"), py::arg("x"), py::arg("w1"), py::arg("w2"), py::arg("topk_w"),
        py::arg("topk_ids"), py::arg("tile"), py::arg("xs"), py::arg("h"), py::arg("ys"), py::arg("sorted_pair"),
        py::arg("pair_pos"), py::arg("tile_expert"), py::arg("tile_row"), py::arg("num_tiles"), py::arg("err"),
        py::arg("combine") = true);
  m.def("ep_dispatch", &ep_dispatch);
  m.def("moe_combine", &moe_combine);
  m.def("ep_return", &ep_return);
  m.def("grouped_gemm", &grouped_gemm);
  m.def("mxfp4_quantize", &mxfp4_quantize);
  m.def("moe_experts_mxfp4", &moe_experts_mxfp4, py::arg("out"), py::arg("x"), py::arg("w1q"), py::arg("w1s"),
        py::arg("w2q"), py::arg("w2s"), py::arg("topk_w"), py::arg("topk_ids"), py::arg("tile"), py::arg("xs"),
        py::arg("h"), py::arg("ys"), py::arg("sorted_pair"), py::arg("pair_pos"), py::arg("tile_expert"),
        py::arg("tile_row"), py::arg("num_tiles"), py::arg("err"), py::arg("combine") = true);
  m.def("mx8_quantize", &mx8_quantize, py::arg("q"), py::arg("sf"), py::arg("x"), py::arg("idx"), py::arg("k"),
        py::arg("rows"), py::arg("tile"));
  m.def("moe_experts_mx", &moe_experts_mx, py::arg("out"), py::arg("x"), py::arg("w1q"), py::arg("w1sb"),
        py::arg("w2q"), py::arg("w2sb"), py::arg("topk_w"), py::arg("topk_ids"), py::arg("tile"), py::arg("xq"),
        py::arg("xsf"), py::arg("h"), py::arg("hq"), py::arg("hsf"), py::arg("ys"), py::arg("sorted_pair"),
        py::arg("pair_pos"), py::arg("tile_expert"), py::arg("tile_row"), py::arg("num_tiles"), py::arg("err"),
        py::arg("combine") = true);
  m.def("mla_prepare", &mla_prepare, py::arg("q_pe"), py::arg("xs"), py::arg("q"), py::arg("kv_a"),
        py::arg("norm_w"), py::arg("eps"), py::arg("positions"), py::arg("cos_sin"), py::arg("latent"),
        py::arg("out_loc"), py::arg("T_pad"), py::arg("err"), py::arg("cp_size") = 1, py::arg("cp_rank") = 0);
  m.def("mla_attention", &mla_attention, py::arg("out"), py::arg("q_lat"), py::arg("q_pe"), py::arg("latent"),
        py::arg("page_table"), py::arg("req_rows"), py::arg("seq_lens"), py::arg("cu_q"), py::arg("page_size"),
        py::arg("scale"), py::arg("splits"), py::arg("part_o"), py::arg("part_lse"), py::arg("err"),
        py::arg("trace") = py::none(), py::arg("cp_size") = 1, py::arg("cp_rank") = 0,
        py::arg("combine_only") = false, py::arg("own_only") = false);
  m.def("mla_prefill_attention", &mla_prefill_attention);
  m.def("mla_gather_keys", &mla_gather_keys);
  m.def("mla_scatter_kv", &mla_scatter_kv);
  m.def("mla_rope_q", &mla_rope_q);
  m.def("mla_store_latent", &mla_store_latent, py::arg("kv_a"), py::arg("norm_w"), py::arg("eps"),
        py::arg("positions"), py::arg("cos_sin"), py::arg("latent"), py::arg("out_loc"), py::arg("err"),
        py::arg("cp_size") = 1, py::arg("cp_rank") = 0);
  m.def("mla_prepare_q", &mla_prepare_q, py::arg("q_pe"), py::arg("xs"), py::arg("q"), py::arg("positions"),
        py::arg("cos_sin"), py::arg("T_pad"), py::arg("err"));
  m.def("mla_heads_to_rows", &mla_heads_to_rows, py::arg("out"), py::arg("in"), py::arg("T"),
        py::arg("row_map") = py::none(), py::arg("err") = py::none());
  m.def("mla_num_splits", [](int64_t T, int64_t H) { return minisgl::mla_num_splits(static_cast<int>(T), static_cast<int>(H)); });
  m.def("symm_create", &symm_create);
  m.def("symm_open", &symm_open);
  m.def("symm_close", &symm_close);
  m.def("symm_free", &symm_free);
  m.def("symm_collective", &symm_collective);
  m.def("symm_rsn", &symm_rsn);
  m.def("sample_shard_chunks", &sample_shard_chunks);
  m.def("sample_shard_partials", &sample_shard_partials);
  m.def("sample_shard_reduce", &sample_shard_reduce);
  m.def("gemm_allreduce", &gemm_allreduce);
  m.def("prefill_attention", &prefill_attention);
  m.def("argmax", &argmax);
  m.def("sample", &sample);
  m.def("moe_route", &moe_route);
  m.def("fast_compare_key", &fast_compare_key);
}
