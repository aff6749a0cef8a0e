// Plain-C++ launcher interface between the torch binding layer (binding.cpp)
// and the CUDA translation units. Nothing here includes torch headers, so the
// .cu files compile quickly and stay independent of the framework layer.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace minisgl {

enum class DType : int { kF32 = 0, kBF16 = 1, kF16 = 2 };

// ----------------------------------------------------------------- GEMM ----
// out[M, N] = x[M, K] @ w[N, K]^T (+ bias[N]); bf16 inputs, fp32 accumulate.
// Fused epilogues of the weight-major split-K GEMM (decode path). Flags:
//   kEpiNorm     out rows scaled by rstd_t = rsqrt(mean_k x[t, k]^2 + eps):
//                the RMSNorm of x whose weight was folded into w's columns
//                (w' = w * diag(norm_weight)), so x is the raw residual
//                stream; the sum of squares is taken from the x tiles the
//                GEMM streams anyway.
//   kEpiResidual out = acc + residual (out may alias residual).
//   kEpiSiluMul  w rows interleaved in blocks of 64 (64 gate rows, then the
//                64 matching up rows); out[t, j] = silu(gate) * up, N / 2
//                output columns.
//   kEpiRope     w is the fused qkv projection with head_dim 128: q/k heads
//                get their per-head RMSNorm (if weights are given) and NeoX
//                RoPE; q heads are written to out (the qkv row), k and v
//                heads to the paged KV cache at out_loc (not to out).
//   kEpiSample   the LM head (weight-major tiles): instead of logits, each
//                (token, 128-row vocabulary tile) writes its best score and
//                index, score = logit / T + Gumbel noise of the sampler's
//                counter-based stream (T <= 0: the plain logit, argmax);
//                launch_lm_sample_reduce turns the partials into tokens.
//   kEpiAllReduce tensor-parallel row-parallel GEMM: the CTA writes its
//                rounded partial tile into its symmetric heap (half epoch & 1),
//                flags it, waits for the same CTA's flag on every peer, and
//                stores sum over ranks (rank order) of the partials (+ residual
//                with kEpiResidual) into out. Needs every CTA of the grid
//                resident at once (checked; otherwise the host runs the GEMM
//                into the heap and the separate collective kernel).
enum : int { kEpiNorm = 1, kEpiResidual = 2, kEpiSiluMul = 4, kEpiRope = 8, kEpiSample = 16, kEpiAllReduce = 32 };
struct GemmEpilogue {
  int kind;
  float eps;                  // kEpiNorm
  const void* residual;       // kEpiResidual: bf16 [M, ld_res]
  int ld_res;
  const void* q_norm_w;       // kEpiRope: bf16 [128] or nullptr
  const void* k_norm_w;
  float head_eps;
  const float* cos_sin;       // [max_pos, 128]: 64 cos then 64 sin
  const int32_t* positions;   // [M]
  const int32_t* out_loc;     // [M] token slots
  void* k_cache;              // bf16 [pages, hk, page_size, 128] of this layer
  void* v_cache;
  int hq, hk, page_size;
  int64_t kv_slots;           // pages * page_size: slots outside [0, kv_slots) are reported, not written
  const float* temps;         // kEpiSample: [M] temperatures (nullptr: all greedy)
  uint64_t seed;
  const int64_t* step;        // device step counter (read only here)
  float* part_val;            // [M, ntiles]
  int32_t* part_idx;
  int ntiles;                 // ceil(N / 128)
  const int64_t* ar_bases;    // kEpiAllReduce: [world] heap bases (own included)
  const uint32_t* ar_epoch;   // this rank's call counter (the call uses epoch + 1)
  int ar_rank, ar_world;
  int64_t ar_half_bytes;      // bytes of one data half of the heap
};

struct GemmArgs {
  const void* x;      // bf16 [M, K], row stride ldx elements
  const void* w;      // bf16 [N, K], row stride ldw elements
  const void* bias;   // bf16 [N] or nullptr
  void* out;          // [M, N] (bf16 or fp32), row stride ldo elements
  float* workspace;   // fp32 scratch for split-K partial sums (may be nullptr)
  int64_t workspace_elems;
  int M, N, K;
  int ldx, ldw, ldo;
  bool out_f32;
  int force_splits;   // 0 = heuristic
  int force_mode;     // 0 = heuristic, 1 = token-major tiles, 2 = weight-major tiles (swap)
  int force_bn;       // 0 = heuristic, else the N tile (16..256)
  int force_kps;      // 0 = heuristic, else k-blocks per pipeline stage (1, 2 or 4)
  void* trace;        // optional uint64 [ctas * 8] phase timestamps (profiling)
  int* err;           // device error word (2 x int32) or nullptr
  GemmEpilogue epi;   // fused epilogue (kind 0: plain store)
  // grouped (MoE) GEMM: w = g_experts matrices of [N, K]; x rows are expert-
  // sorted and padded to the token tile (force_bn); see MoeAlignArgs
  const int32_t* g_tile_expert;
  const int32_t* g_tile_row;
  const int32_t* g_num_tiles;  // nullptr: plain GEMM
  int g_experts;
};
void launch_gemm(const GemmArgs& a, cudaStream_t stream);
// Stream-K weight-streaming GEMM for up to 256 tokens (gemm_streamk.cu):
// R = 1 or 2 weight sub-tiles of 128 rows per work tile; ws holds ws_slots
// fp32 partial tiles of ws_slot_floats each, flags ws_slots * 32 int32 (one
// flag per 128-byte line, all 0 between launches). grid <= ws_slots CTAs
// (one per SM).
struct GemmStreamKArgs {
  const void* x;
  const void* w;
  const void* bias;
  void* out;
  int M, N, K;
  int ldx, ldw, ldo;
  int out_f32;
  int R;
  int kps;  // 0 = from the shared-memory budget
  int grid;
  float* ws;
  int* flags;
  int ws_slots;
  int64_t ws_slot_floats;
  int* err;
  void* trace;  // optional uint64 [grid * 8] phase stamps
};
constexpr int64_t kStreamKSlotFloats = 2 * 256 * 128;  // R = 2, 256 tokens
constexpr int64_t kStreamKFlagWords = 32;               // per slot
int gemm_streamk_grid(int M, int N, int K, int R, int sms);
void launch_gemm_streamk(const GemmStreamKArgs& a, cudaStream_t stream);
// Persistent 128 x {128, 256} tiles with double-buffered TMEM accumulators
// (force_mode 3): plain GEMMs (no fused epilogue) with K % 64 == 0.
bool gemm_persistent_supported(const GemmArgs& a);
void launch_gemm_persistent(const GemmArgs& a, cudaStream_t stream);
bool gemm_pair_supported(const GemmArgs& a);
void launch_gemm_pair(const GemmArgs& a, cudaStream_t stream);
// Number of fp32 workspace elements launch_gemm may need for this shape.
int64_t gemm_workspace_elems(int M, int N, int K);

// ------------------------------------------------------ elementwise / norm ----
void launch_rmsnorm(void* out, const void* x, const void* w, int rows, int cols, int ld_x,
                    int ld_out, float eps, DType dt, cudaStream_t s);
// x <- rmsnorm(x + residual) * w ; residual <- x + residual  (in place)
void launch_fused_add_rmsnorm(void* x, void* residual, const void* w, int rows, int cols,
                              float eps, DType dt, cudaStream_t s);
// out[t, :d] = act(x[t, :d]) * x[t, d:2d]; act 0 = silu, 1 = gelu(tanh)
void launch_act_and_mul(void* out, const void* x, int rows, int d, int act, bool interleaved, DType dt,
                        cudaStream_t s);
// out[i, :] = (lo <= ids[i] < lo + n) ? w[ids[i] - lo, :] : 0
void launch_embedding(void* out, const void* w, const int32_t* ids, int num_tokens, int hidden,
                      int vocab_lo, int vocab_n, DType dt, cudaStream_t s);

// ----------------------------------- qk-norm + RoPE + paged KV-cache store ----
struct RopeStoreArgs {
  void* qkv;                 // [T, (hq + 2*hk) * d] in place: q and k get normed + rotated
  int ld_qkv;
  const int32_t* positions;  // [T]
  const float* cos_sin;      // [max_pos, rot_dim]: cos(rot_dim/2) | sin(rot_dim/2)
  const void* q_norm_w;      // [d] or nullptr
  const void* k_norm_w;      // [d] or nullptr
  void* k_cache;             // layer slice: [num_pages, hk, page, d]
  void* v_cache;
  const int32_t* out_loc;    // [T] token slot (page * page_size + offset)
  int T, hq, hk, d, rot_dim, page_size;
  float eps;
  DType dt;
  int64_t kv_slots;          // pages * page_size: slots outside [0, kv_slots) are reported, not written
  int* err;
};
void launch_rope_store(const RopeStoreArgs& a, cudaStream_t s);

// ------------------------------------------------------------- attention ----
// The KV pool is one tensor [2, layers, pages, hk, page_size, d]; kernels see
// it as a 2-D [pool_rows, d] matrix and address one layer's K (V) through the
// row offset k_row0 (v_row0). A (page, head) block of page_size rows is
// contiguous, so a tile of keys is a single TMA box.
struct AttnArgs {
  const void* q;             // [T, hq, d], token stride ld_q elements
  int ld_q;
  void* out;                 // [T, hq, d] contiguous
  const void* kv_pool;       // base of the whole pool (bf16)
  int64_t pool_rows;
  int64_t k_row0, v_row0;    // first row of this layer's K / V
  const int32_t* page_table; // [rows, ld_pt] token slots (page * page_size + offset)
  int ld_pt;
  const int32_t* req_rows;   // [B] row of page_table per request
  const int32_t* seq_lens;   // [B] total keys per request (cached + new)
  const int32_t* cu_q;       // [B + 1] query offsets (prefill only)
  int B, hq, hk, d, page_size;
  int max_q;                 // prefill: longest query segment (grid size)
  float scale;
  // split-KV scratch (decode): partial outputs and log-sum-exp values
  float* part_o;             // [B, hq, max_splits, d]
  float* part_lse;           // [B, hq, max_splits]
  int max_splits;
  int* err;
  int q_rows;                // prefill: rows of q (the TMA map extent); 0 selects the kernel without Q TMA
  int pt_rows;               // rows of page_table: a request row outside [0, pt_rows) is reported and skipped
  unsigned long long* trace; // optional [64 tiles x 8] %globaltimer stamps of one prefill CTA (profiling)
  // non-absorbed MLA prefill (launch_mla_prefill_attention): q heads are
  // q_head_stride elements apart in a q row (their first 128 are q_nope),
  // q_rope [q_rows, hq, 64] holds the rotated query rope parts and k_rope
  // [rope_rows, 64] the keys' shared rope rows at the page-table slots
  int q_head_stride;
  const void* q_rope;
  const void* k_rope;
  int64_t rope_rows;
};
void launch_decode_attention(const AttnArgs& a, cudaStream_t s);
void launch_prefill_attention(const AttnArgs& a, cudaStream_t s);
void launch_mla_prefill_attention(const AttnArgs& a, cudaStream_t s);

// ------------------------------------------------------------------ MLA ----
struct MlaPrepareArgs {
  // either half may be absent: q == nullptr stores key rows only, latent ==
  // nullptr prepares queries only
  const void* q;          // [T, H, nope + rope] (token stride ld_q)
  int ld_q;
  const void* kv_a;       // [T, kv_lora + rope] (token stride ld_kv_a)
  int ld_kv_a;
  const void* norm_w;     // [kv_lora] kv_a_layernorm weight
  float eps;
  const int32_t* positions;
  const float* cos_sin;   // [max_pos, rope]: rope / 2 cos then rope / 2 sin
  void* latent;           // [slots, kv_lora + rope] of this layer
  const int32_t* out_loc; // [T] cache slots
  void* q_pe;             // out: [T, H, rope]
  void* xs;               // out: [H, T_pad, nope] (grouped GEMM input)
  int T, T_pad, H, nope, kv_lora, rope;
  int cp_size, cp_rank;   // context parallelism: store only rows of owned 64-key tiles
  int page_size;          // (at local page = global page / cp_size)
  int64_t num_slots;      // latent rows of this layer's pool (0: unchecked)
  int* err;
};
struct MlaAttnArgs {
  const void* q_lat;      // [H, T_pad, kv_lora]
  const void* q_pe;       // [T, H, rope]
  const void* latent;     // [num_slots, kv_lora + rope] of this layer
  int64_t num_slots;
  const int32_t* page_table;  // [rows, ld_pt] token slots
  int ld_pt;
  const int32_t* req_rows;    // [B]
  const int32_t* seq_lens;    // [B] keys per request
  const int32_t* cu_q;        // [B + 1] query offsets
  void* out;                  // [H, T_pad, kv_lora]
  float* part_o;              // [splits, T, H, kv_lora] (splits > 1)
  float* part_lse;            // [splits, T, H]
  int B, T, T_pad, H, page_size, splits;
  float scale;
  int* err;
  // context parallelism: this rank attends over the 64-key tiles t with
  // t % cp_size == cp_rank and writes partials [cp_size * splits, T, H, ...]
  // at slots cp_rank * splits + split (merged by launch_mla_combine)
  int cp_size, cp_rank;
  // combine only: sum this rank's partial outputs under the normaliser of
  // every rank's log-sum-exps (token-sharded context parallelism)
  int own_only;
  // optional per-tile timestamps (%globaltimer ns) of CTA (0, 0, 0), 8 slots
  // per tile: 0 copy issued, 1 QK issued, 2 scores seen, 3 P written,
  // 4 PV issued, 5 PV seen complete
  unsigned long long* trace;
};
void launch_mla_prepare(const MlaPrepareArgs& a, cudaStream_t s);
void launch_mla_attention(const MlaAttnArgs& a, cudaStream_t s);
void launch_mla_combine(const MlaAttnArgs& a, cudaStream_t s);
void launch_mla_heads_to_rows(void* out, const void* in, int T, int T_pad, int H, int v, const int32_t* row_map,
                              int out_rows, int* err, cudaStream_t s);
int mla_num_splits(int T, int H);
void launch_mla_gather_keys(void* x, void* k_rope, const void* latent, int64_t num_slots, const int32_t* page_table,
                            int ld_pt, const int32_t* req_rows, const int32_t* row_req, const int32_t* row_pos, int R,
                            int* err, cudaStream_t s);
void launch_mla_scatter_kv(void* pool, const void* y, int R, int H, cudaStream_t s);

// -------------------------------------------------------------- sampling ----
// logits fp32 [B, V] (row stride ld); writes int32 token ids.
void launch_argmax(int32_t* out, const float* logits, int B, int V, int ld, cudaStream_t s);
struct SampleArgs {
  int32_t* out;
  const float* logits;       // [B, V] fp32
  int ld, B, V;
  const float* temperature;  // [B]
  const int32_t* top_k;      // [B] or nullptr (<= 0 or >= V means disabled)
  const float* top_p;        // [B] or nullptr
  uint64_t seed;
  const int64_t* step;       // device counter mixed into the random stream (may be nullptr)
  int index_offset;          // vocabulary index of column 0 (a tensor-parallel shard's first row)
};
void launch_sample(const SampleArgs& a, cudaStream_t s);
// Greedy (temperature == nullptr) or temperature sampling with each row
// split over vocabulary chunks: partials [B, sample_split_chunks(V)] then
// the per-row reduce; same tokens as launch_argmax / launch_sample.
int sample_split_chunks(int V);
void launch_sample_split(const SampleArgs& a, float* part_val, int32_t* part_idx, cudaStream_t s);
void launch_lm_sample_reduce(int32_t* out, const float* part_val, const int32_t* part_idx, int ntiles, int B,
                             const float* temps, int64_t* step, cudaStream_t s);
// Vocabulary-sharded sampling (tensor parallelism): partials of this rank's
// logits shard [B, V_shard] (global indices from a.index_offset), written as
// rows of `ld` int32 words: values (fp32 bits) in columns [0, chunks), indices
// in [chunks, 2 chunks); sample_split_chunks(V_shard) chunks per row.
void launch_sample_shard_partials(const SampleArgs& a, int32_t* packed, int ld, cudaStream_t s);
// Tokens from every rank's packed partials [ranks][B][ld] (same tie rule as
// the whole-vocabulary kernels); advances the step counter like them.
void launch_sample_shard_reduce(int32_t* out, const int32_t* packed, int chunks, int ld, int ranks, int B,
                                const float* temps, int64_t* step, cudaStream_t s);

// ------------------------------------------------------------------- MoE ----
struct MoeRouteArgs {
  const float* logits;       // [T, E] router logits (fp32)
  const float* bias;         // [E] correction bias (sigmoid routing) or nullptr
  float* topk_w;             // [T, k]
  int32_t* topk_ids;         // [T, k]
  int T, E, k;
  int scoring;               // 0 softmax, 1 sigmoid
  bool renormalize;
  int n_group, topk_group;   // grouped routing (sigmoid); 1/1 disables
  float routed_scale;
};
void launch_moe_route(const MoeRouteArgs& a, cudaStream_t s);

// Expert-sorted layout of the T * k (token, slot) pairs for the grouped
// expert GEMMs. Every expert's segment is padded to a multiple of `tile`
// rows; capacity P = T * k + E * (tile - 1) rows, P / tile tiles.
struct MoeAlignArgs {
  const int32_t* topk_ids;   // [T * k]
  int T, k, E, tile;
  int32_t* sorted_pair;      // [P]: pair index t * k + j, or -1 for padding rows
  int32_t* pair_pos;         // [T * k]: row of each pair in the sorted layout
  int32_t* tile_expert;      // [P / tile]: expert of each tile
  int32_t* tile_row;         // [P / tile]: first sorted row of each tile
  int32_t* num_tiles;        // [1]: tiles in use
};
void launch_moe_align(const MoeAlignArgs& a, cudaStream_t s);
// xs[r] = x[sorted_pair[r] / k] (zeros for padding rows); bf16 rows of H
void launch_moe_gather(void* xs, const void* x, const int32_t* sorted_pair, int P, int k, int H, cudaStream_t s);
// out[t] = sum_j topk_w[t, j] * ys[pair_pos[t * k + j]] (fixed j order), bf16 rows of H
void launch_moe_combine(void* out, const void* ys, const float* topk_w, const int32_t* pair_pos, int T, int k, int H,
                        cudaStream_t s);

// --------------------------------------------------- EP token dispatch ----
struct EpArgs {
  const int64_t* bases;   // [world] heap base of every rank
  uint32_t* epoch;        // this rank's call counter (identical on every rank)
  int rank, world;
  int cap;                // pair slots per rank and step
  int64_t ids_off, rows_off, back_off;  // byte offsets of the heap regions
  int H;
  // dispatch
  const void* x;          // [T, H] bf16 this rank's tokens
  const int32_t* topk_ids;  // [T * k] global expert ids
  int T, k, e_local;
  // return
  const void* ys;         // [P, H] bf16 expert outputs of the received rows
  const int32_t* pair_pos;  // [world * cap] row of ys per received slot (-1: none)
  int* err;
};
void launch_ep_dispatch(const EpArgs& a, cudaStream_t s);
void launch_ep_return(const EpArgs& a, cudaStream_t s);

// --------------------------------------------------------------- MXFP4 ----
// w [E, N, K] bf16 -> packed [E, N, K / 2] E2M1 + scales [E, K / 64, N, 2] E8M0
void launch_mxfp4_quantize(void* packed, void* scales, const void* w, int E, int N, int K, cudaStream_t s);
struct MoeMxfp4GemmArgs {
  const void* x;              // [P, K] bf16 expert-sorted token rows
  const void* packed;         // [E, N, K / 2]
  const void* scales;         // [E, K / 64, N, 2]
  void* out;                  // [P, ldo] bf16 (N / 2 features with silu, else N)
  int P, E, N, K, ldo, tile;
  bool silu;                  // interleaved gate|up rows -> silu(gate) * up
  const int32_t* tile_expert;
  const int32_t* tile_row;
  const int32_t* num_tiles;
  int* err;
};
void launch_moe_mxfp4_gemm(const MoeMxfp4GemmArgs& a, cudaStream_t s);

// Block-scaled MX grouped GEMM (mx_gemm.cu): MXFP4 weights x MXFP8 token rows
// on tcgen05 kind::mxf8f6f4 with E8M0 scales in the 512-byte scale-block layout.
struct MoeMxGemmArgs {
  const void* xq;             // [P, K] E4M3 expert-sorted token rows
  const void* sfx;            // [P / tile, K / 128, 512] their scale blocks
  const void* packed;         // [E, N, K / 2] E2M1 weights
  const void* sfw;            // [E, N / 128, K / 128, 512] weight scale blocks
  void* out;                  // [P, ldo] bf16 (N / 2 features with silu, else N)
  int P, E, N, K, ldo, tile;
  bool silu;                  // interleaved gate|up rows -> silu(gate) * up
  const int32_t* tile_expert;
  const int32_t* tile_row;
  const int32_t* num_tiles;
  int* err;
};
void launch_moe_mx_gemm(const MoeMxGemmArgs& a, cudaStream_t s);
// MXFP8 (E4M3 + E8M0 per 32) of `rows` bf16 rows of K into q [rows, K] and
// scale blocks [rows / tile, K / 128, 512]; row p comes from x[idx[p] / k]
// (zeros where idx[p] < 0) or, without idx, from x[p]. Rows of tiles at or
// beyond *num_tiles (when given) are skipped.
void launch_mx8_quantize_rows(void* q, void* sf, const void* x, const int32_t* idx, int k, int rows, int K, int tile,
                              const int32_t* num_tiles, cudaStream_t s);

// ------------------------------------------------------- NVLink collectives ----
// kind 0: all-reduce of every rank's partial (bf16, n_elems, at the data
// offset of each heap) into out (+ residual); kind 1: all-gather of
// rows_per_rank rows of row_elems from every heap into out. bases: device
// int64 [world] heap bases (own one included), epoch: this rank's uint32
// call counter. See symm.cu for the protocol.
void launch_symm_collective(int kind, const int64_t* bases, uint32_t* epoch, int rank, int world, int64_t n_elems,
                            void* out, const void* residual, int rows_per_rank, int row_elems, int* err,
                            cudaStream_t s);
// Reduce-scatter of every rank's partial [rows * world, hidden] (heap data
// region at data_off) into this rank's residual slice resid [rows, hidden]
// (+= when add_resid), RMSNorm of the new rows (times norm_w when given) and
// all-gather of the normalised rows into every heap's region at gather_off.
void launch_symm_rsn(const int64_t* bases, uint32_t* epoch, int rank, int world, int rows, int hidden,
                     int64_t data_off, int64_t gather_off, void* resid, bool add_resid, const void* norm_w, float eps,
                     int* err, cudaStream_t s);
constexpr int64_t kSymmSignalBytes = 4096;
// GEMM with the all-reduce fused (kEpiAllReduce) when the grid is resident,
// otherwise GEMM into the heap data region + launch_symm_collective. Heap
// layout for the fused kind: [signal 4 KB][flags 16 KB][half 0][half 1].
constexpr int64_t kSymmFlagBytes = 16384;
// advance a uint32 call counter after every CTA of the previous kernel read it
void launch_epoch_bump(uint32_t* epoch, cudaStream_t s);
void launch_gemm_allreduce(const GemmArgs& a, const int64_t* bases, uint32_t* epoch, int64_t own_base, int rank,
                           int world, int64_t half_bytes, void* residual_out, cudaStream_t s);

}  // namespace minisgl
