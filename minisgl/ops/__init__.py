"""Operator entry points used by the model layers.

CUDA tensors always run the hand-written sm_100a kernels of ``minisgl._C``;
if that library cannot be loaded on a GPU process the call raises instead of
falling back. CPU tensors run the fp32 PyTorch restatement in
``minisgl.ops.reference`` (the CPU oracle used by the CPU engine and tests).
"""

from __future__ import annotations

import functools
from typing import List, Optional, Tuple

import torch

from . import reference as ref

_NATIVE = None
_NATIVE_ERR: Optional[BaseException] = None

# Host-side count of native kernel launches issued through this module
# (CUDA-graph replays are added by the graph runner). Benchmarks report it.
LAUNCHES = [0]


def _count(n: int = 1) -> None:
    LAUNCHES[0] += n


def native():
    """The loaded ``minisgl._C`` module; raises if it is unavailable."""
    global _NATIVE, _NATIVE_ERR
    if _NATIVE is None:
        try:
            from minisgl import _C  # type: ignore[attr-defined]

            _NATIVE = _C
        except BaseException as e:  # pragma: no cover - depends on the build
            _NATIVE_ERR = e
            raise RuntimeError(
                "minisgl native library (minisgl/_C*.so) is not built or failed to load; "
                "run `python setup.py build_ext --inplace`"
            ) from e
    return _NATIVE


def native_available() -> bool:
    try:
        native()
        return True
    except RuntimeError:
        return False


# ------------------------------------------------------------------ scratch
_WORKSPACE: dict = {}
_ERR_WORDS: dict = {}
GEMM_WORKSPACE_ELEMS = 8 * 1024 * 1024  # 32 MiB fp32: bounds every split-K plan


def gemm_workspace(device: torch.device) -> torch.Tensor:
    key = (device.type, device.index)
    ws = _WORKSPACE.get(key)
    if ws is None:
        ws = torch.empty(GEMM_WORKSPACE_ELEMS, dtype=torch.float32, device=device)
        _WORKSPACE[key] = ws
    return ws


def _device_key(device) -> tuple:
    """(type, index) of a device; a CUDA device without an index is the
    current one, so torch.device("cuda") and the tensors' cuda:N agree."""
    device = torch.device(device)
    if device.type == "cuda" and device.index is None:
        return ("cuda", torch.cuda.current_device())
    return (device.type, device.index)


def error_word(device: torch.device) -> torch.Tensor:
    """Per-device int32[2]: (error code, site) written by kernels whose bounded
    waits ran out. Zero means no error."""
    key = _device_key(device)
    w = _ERR_WORDS.get(key)
    if w is None:
        w = torch.zeros(2, dtype=torch.int32, device=device)
        _ERR_WORDS[key] = w
    return w


class DeviceWaitTimeout(RuntimeError):
    """A kernel gave up on an mbarrier wait (its pipeline stalled) and returned."""


class DeviceIndexError(RuntimeError):
    """A kernel met an index outside the buffer it addresses (a KV slot past
    the cache, a request row past the page table), reported it and skipped
    the access instead of touching memory it does not own."""


class CommTimeoutError(RuntimeError):
    """A collective kernel gave up waiting for a peer rank's flag and returned:
    the peer is late, stalled or gone. The device context stays usable."""


ERR_MBAR_TIMEOUT = 1
ERR_PEER_TIMEOUT = 2
ERR_BAD_INDEX = 3


def check_device_errors(device: torch.device) -> None:
    """Raise if a kernel on ``device`` recorded an error (and clear it):
    CommTimeoutError for a peer wait that ran out, DeviceWaitTimeout for a
    pipeline wait, RuntimeError otherwise."""
    w = _ERR_WORDS.get(_device_key(device))
    if w is None:
        return
    code, site = w.tolist()
    if code != 0:
        w.zero_()
        if code == ERR_PEER_TIMEOUT:
            raise CommTimeoutError(f"minisgl collective kernel timed out waiting for a peer (site {site})")
        if code == ERR_MBAR_TIMEOUT:
            raise DeviceWaitTimeout(f"minisgl kernel pipeline wait timed out (site {site})")
        if code == ERR_BAD_INDEX:
            raise DeviceIndexError(f"minisgl kernel skipped an index outside its buffer (site {site}): a KV slot "
                                   "outside the cache or a request row outside the page table")
        raise RuntimeError(f"minisgl kernel reported error code {code} at site {site}")


# ------------------------------------------------------------------- GEMM
from .gemm_tune import lookup as _gemm_lookup  # noqa: E402  (autotuned plans by (M, N, K))

def gemm(
    x: torch.Tensor,
    w: torch.Tensor,
    bias: Optional[torch.Tensor] = None,
    out: Optional[torch.Tensor] = None,
    out_dtype: Optional[torch.dtype] = None,
) -> torch.Tensor:
    """out = x @ w^T (+ bias): the F.linear convention."""
    out_dtype = out_dtype or (out.dtype if out is not None else x.dtype)
    if not x.is_cuda:
        y = ref.gemm(x, w, bias, out_dtype)
        if out is not None:
            out.copy_(y)
            return out
        return y
    if out is None:
        out = torch.empty(x.shape[0], w.shape[0], dtype=out_dtype, device=x.device)
    plan = _gemm_lookup(x.shape[0], w.shape[0], x.shape[1])
    _count()
    if plan is None:
        native().gemm(out, x, w, bias, None, 0, 0, error_word(x.device))
    elif plan[0] == GEMM_STREAMK:
        _, r, kps = plan
        native().gemm(out, x, w, bias, streamk_workspace(x.device), 0, GEMM_STREAMK, error_word(x.device), r,
                      None, kps)
    else:
        mode, bn, splits = plan
        native().gemm(out, x, w, bias, None, splits, mode, error_word(x.device), bn)
    return out


# tile-plan mode of the stream-K weight-streaming GEMM (up to 256 tokens,
# K % 64 == 0); its plan is (GEMM_STREAMK, weight sub-tiles R, k-blocks per stage)
GEMM_STREAMK = 4
# persistent 256 x 256 tiles on CTA pairs (cta_group::2 MMAs, K % 64 == 0)
GEMM_PAIR = 5
_SK_WORKSPACE: dict = {}
_SK_SLOT_FLOATS = 2 * 256 * 128
_SK_FLAG_WORDS = 32


def streamk_workspace(device: torch.device) -> torch.Tensor:
    """Per (device, stream) scratch of the stream-K GEMM: one fp32 partial
    tile per SM, then one int32 ready flag per SM, each on its own 128-byte
    line (zero between launches). Kernels on one stream never overlap on it;
    each stream gets its own."""
    stream = torch.cuda.current_stream(device)
    key = (device.index, stream.cuda_stream)
    ws = _SK_WORKSPACE.get(key)
    if ws is None:
        sms = torch.cuda.get_device_properties(device).multi_processor_count
        ws = torch.zeros(sms * (_SK_SLOT_FLOATS + _SK_FLAG_WORDS), dtype=torch.float32, device=device)
        _SK_WORKSPACE[key] = ws
    return ws


# ------------------------------------------------------------ elementwise
EPI_NORM, EPI_RESIDUAL, EPI_SILU, EPI_ROPE, EPI_SAMPLE = 1, 2, 4, 8, 16
from .gemm_tune import FUSED_PLANS as _gemm_fused_plans  # noqa: E402  (best plans fused epilogues accept)


def gemm_fused(
    x: torch.Tensor,
    w: torch.Tensor,
    *,
    bias: Optional[torch.Tensor] = None,
    norm_eps: Optional[float] = None,
    residual: Optional[torch.Tensor] = None,
    silu: bool = False,
    rope: Optional[dict] = None,
    out: Optional[torch.Tensor] = None,
    plan: Optional[Tuple[int, int, int]] = None,
) -> torch.Tensor:
    """GEMM with a fused epilogue (``plan`` = (mode: 1 token-major / 2
    weight-major tiles, N tile, K splits) overrides the tuned / default
    plan; token-major tiles need an N tile of 128 or 256 for silu / rope):

    * ``norm_eps``: rows of x are RMS-normalised (x is the raw residual
      stream; the norm weight must already be folded into ``w``'s columns);
    * ``silu``: ``w`` holds gate|up rows interleaved in blocks of 64 and the
      result is silu(gate) * up, [M, N / 2];
    * ``residual``: out = x @ w^T + residual (``out`` may be ``residual``);
    * ``rope`` (dict: positions, cos_sin, q_norm_w, k_norm_w, head_eps,
      k_cache, v_cache, out_loc, hq, hk, page_size): q/k head norm + NeoX
      RoPE; q heads land in ``out`` (the qkv rows), k/v in the paged cache.
    """
    if not x.is_cuda:
        y = ref.gemm_fused(x, w, bias, norm_eps, residual, silu, rope)
        if out is not None:
            out.copy_(y[:, : out.shape[1]])  # rope: out may hold only the q heads
            return out
        return y
    M, N = x.shape[0], w.shape[0]
    if out is None:
        out = torch.empty(M, N // 2 if silu else N, dtype=x.dtype, device=x.device)
    kind = (EPI_NORM if norm_eps is not None else 0) | (EPI_RESIDUAL if residual is not None else 0)
    kind |= (EPI_SILU if silu else 0) | (EPI_ROPE if rope is not None else 0)
    if plan is None:
        plan = _gemm_fused_plans.get((M, N, x.shape[1]), (0, 0, 0))
    mode, bn, splits = plan
    r = rope or {}
    _count()
    native().gemm_fused(
        out, x, w, bias, mode, splits, bn, error_word(x.device), kind, norm_eps or 0.0, residual,
        r.get("q_norm_w"), r.get("k_norm_w"), r.get("head_eps", 0.0), r.get("cos_sin"), r.get("positions"),
        r.get("out_loc"), r.get("k_cache"), r.get("v_cache"), r.get("hq", 0), r.get("hk", 0), r.get("page_size", 0),
    )
    return out


def rmsnorm(x: torch.Tensor, w: Optional[torch.Tensor], eps: float, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """y = x / rms(x) * w (w None: no weight, e.g. folded into the next GEMM)."""
    if not x.is_cuda:
        y = ref.rmsnorm(x, w, eps)
        if out is not None:
            out.copy_(y)
            return out
        return y
    if out is None:
        out = torch.empty_like(x)
    _count()
    native().rmsnorm(out, x, w, eps)
    return out


def fused_add_rmsnorm(x: torch.Tensor, residual: torch.Tensor, w: Optional[torch.Tensor], eps: float) -> None:
    if not x.is_cuda:
        ref.fused_add_rmsnorm(x, residual, w, eps)
        return
    _count()
    native().fused_add_rmsnorm(x, residual, w, eps)


def silu_and_mul(x: torch.Tensor, out: Optional[torch.Tensor] = None, interleaved: bool = False) -> torch.Tensor:
    """silu(gate) * up; ``interleaved``: gate|up columns alternate in blocks of 64."""
    return _act_and_mul(x, "silu", out, interleaved)


def gelu_and_mul(x: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    return _act_and_mul(x, "gelu", out)


def _act_and_mul(x: torch.Tensor, act: str, out: Optional[torch.Tensor], interleaved: bool = False) -> torch.Tensor:
    if not x.is_cuda:
        if interleaved:
            assert act == "silu", "interleaved layout is used with SiLU only"
            y = ref.silu_mul_interleaved(x)
        else:
            y = ref.act_and_mul(x, act)
        if out is not None:
            out.copy_(y)
            return out
        return y
    if out is None:
        out = torch.empty(x.shape[0], x.shape[1] // 2, dtype=x.dtype, device=x.device)
    _count()
    native().act_and_mul(out, x, 0 if act == "silu" else 1, interleaved)
    return out


def embedding(ids: torch.Tensor, weight: torch.Tensor, vocab_range: Optional[Tuple[int, int]] = None,
              out: Optional[torch.Tensor] = None) -> torch.Tensor:
    lo, n = vocab_range if vocab_range is not None else (0, weight.shape[0])
    if not weight.is_cuda:
        y = ref.embedding(ids, weight, lo, n)
        if out is not None:
            out.copy_(y)
            return out
        return y
    if out is None:
        out = torch.empty(ids.numel(), weight.shape[1], dtype=weight.dtype, device=weight.device)
    _count()
    native().embedding(out, weight, ids.to(torch.int32), lo, n)
    return out


# ------------------------------------------------------- rope + KV store
def rope_store(
    qkv: torch.Tensor,
    positions: torch.Tensor,
    cos_sin: torch.Tensor,
    q_norm_w: Optional[torch.Tensor],
    k_norm_w: Optional[torch.Tensor],
    k_cache: torch.Tensor,
    v_cache: torch.Tensor,
    out_loc: torch.Tensor,
    hq: int,
    hk: int,
    d: int,
    page_size: int,
    eps: float,
) -> None:
    if not qkv.is_cuda:
        ref.rope_store(qkv, positions, cos_sin, q_norm_w, k_norm_w, k_cache, v_cache, out_loc, hq, hk, d, page_size, eps)
        return
    _count()
    native().rope_store(qkv, positions, cos_sin, q_norm_w, k_norm_w, k_cache, v_cache, out_loc, hq, hk, d, page_size, eps,
                        error_word(qkv.device))


# -------------------------------------------------------------- attention
def decode_attention(
    q: torch.Tensor,
    kv_pool: torch.Tensor,
    layer: int,
    page_table: torch.Tensor,
    req_rows: torch.Tensor,
    seq_lens: torch.Tensor,
    hq: int,
    hk: int,
    d: int,
    page_size: int,
    scale: float,
    part_o: Optional[torch.Tensor] = None,
    part_lse: Optional[torch.Tensor] = None,
    max_splits: int = 1,
    out: Optional[torch.Tensor] = None,
) -> torch.Tensor:
    """One query token per request; q is [B, >= hq*d] (row stride free)."""
    B = req_rows.numel()
    if not q.is_cuda:
        cu = torch.arange(B + 1, dtype=torch.int32)
        qv = q[:, : hq * d].reshape(B, hq, d)
        y = ref.attention(qv, kv_pool, layer, page_table, req_rows, seq_lens, cu, hq, hk, d, page_size, scale)
        y = y.view(B, hq * d)
        if out is not None:
            out.copy_(y)
            return out
        return y
    if out is None:
        out = torch.empty(B, hq * d, dtype=q.dtype, device=q.device)
    _count(2 if max_splits > 1 else 1)
    native().decode_attention(
        q, out, kv_pool, layer, page_table, req_rows, seq_lens, hq, hk, d, page_size, scale,
        part_o, part_lse, max_splits, error_word(q.device),
    )
    return out


def _group_tile(T: int) -> int:
    """Token tile of the head-grouped MLA GEMMs (rows of one head per tile)."""
    return 16 if T <= 16 else 32 if T <= 32 else 64 if T <= 64 else 128


_GROUP_TABLES: dict = {}


def _group_tables(groups: int, tiles_per_group: int, tile: int, device: torch.device):
    """Tile tables of a grouped GEMM whose G groups all have tiles_per_group
    tiles: tile i belongs to group i // tiles_per_group and starts at row
    i * tile (group g owns rows [g * T_pad, (g + 1) * T_pad))."""
    key = (groups, tiles_per_group, tile, device)
    t = _GROUP_TABLES.get(key)
    if t is None:
        n = groups * tiles_per_group
        idx = torch.arange(n, dtype=torch.int32)
        t = ((idx // tiles_per_group).to(device), (idx * tile).to(device),
             torch.tensor([n], dtype=torch.int32).to(device))
        _GROUP_TABLES[key] = t
    return t


def grouped_gemm(x: torch.Tensor, w: torch.Tensor, tile: int, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """out[g] = x[g] @ w[g]^T for G uniform groups: x [G, R, K] (R a multiple
    of ``tile``), w [G, N, K] -> [G, R, N]; one tcgen05 launch (weight-major
    tiles, heads or experts as groups)."""
    G, R, K = x.shape
    N = w.shape[1]
    if not x.is_cuda:
        y = torch.einsum("grk,gnk->grn", x.float(), w.float()).to(x.dtype)
        if out is not None:
            out.copy_(y)
            return out
        return y
    if out is None:
        out = torch.empty(G, R, N, dtype=x.dtype, device=x.device)
    te, tr, nt = _group_tables(G, R // tile, tile, x.device)
    _count()
    native().grouped_gemm(out.view(G * R, N), x.view(G * R, K), w, tile, te, tr, nt, error_word(x.device))
    return out


def mla_prepare(q: torch.Tensor, kv_a: torch.Tensor, w_uk_t: torch.Tensor, norm_w: torch.Tensor, eps: float,
                positions: torch.Tensor, cos_sin: torch.Tensor, latent: torch.Tensor, out_loc: torch.Tensor,
                page_size: int, cp_size: int = 1, cp_rank: int = 0) -> Tuple[torch.Tensor, torch.Tensor]:
    """MLA before attention: the normalised, rotated latent rows go into the
    cache; returns (q_lat [H, T_pad, kv_lora] head-major, q_pe [T, H, rope]).
    On the GPU one kernel writes the cache row, the rotated q_pe and q_nope
    head-major, then a grouped GEMM (heads as groups) absorbs q_nope through
    W_UK; rows past T of q_lat are padding."""
    if not q.is_cuda:
        return ref.mla_prepare(q, kv_a, w_uk_t, norm_w, eps, positions, cos_sin, latent, out_loc, page_size,
                               cp_size, cp_rank)
    T, H, qk = q.shape
    kv_lora, nope = w_uk_t.shape[1], w_uk_t.shape[2]
    rope = qk - nope
    tile = _group_tile(T)
    T_pad = (T + tile - 1) // tile * tile
    xs = torch.empty(H, T_pad, nope, dtype=q.dtype, device=q.device)
    q_pe = torch.empty(T, H, rope, dtype=q.dtype, device=q.device)
    _count()
    native().mla_prepare(q_pe, xs, q, kv_a, norm_w, eps, positions, cos_sin, latent, out_loc, T_pad,
                         error_word(q.device), cp_size, cp_rank)
    return grouped_gemm(xs, w_uk_t, tile), q_pe


def mla_store_latent(kv_a: torch.Tensor, norm_w: torch.Tensor, eps: float, positions: torch.Tensor,
                     cos_sin: torch.Tensor, latent: torch.Tensor, out_loc: torch.Tensor, page_size: int,
                     cp_size: int = 1, cp_rank: int = 0) -> None:
    """The cache half of ``mla_prepare`` alone: latent rows of the tokens of
    kv_a (under context parallelism only those of this rank's tiles)."""
    if not kv_a.is_cuda:
        return ref.mla_store_latent(kv_a, norm_w, eps, positions, cos_sin, latent, out_loc, page_size, cp_size,
                                    cp_rank)
    _count()
    native().mla_store_latent(kv_a, norm_w, eps, positions, cos_sin, latent, out_loc, error_word(kv_a.device),
                              cp_size, cp_rank)


def mla_prepare_q(q: torch.Tensor, w_uk_t: torch.Tensor, positions: torch.Tensor,
                  cos_sin: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
    """The query half of ``mla_prepare`` alone: (q_lat [H, T_pad, kv_lora],
    q_pe [T, H, rope])."""
    if not q.is_cuda:
        return ref.mla_prepare_q(q, w_uk_t, positions, cos_sin)
    T, H, qk = q.shape
    nope = w_uk_t.shape[2]
    tile = _group_tile(T)
    T_pad = (T + tile - 1) // tile * tile
    xs = torch.empty(H, T_pad, nope, dtype=q.dtype, device=q.device)
    q_pe = torch.empty(T, H, qk - nope, dtype=q.dtype, device=q.device)
    _count()
    native().mla_prepare_q(q_pe, xs, q, positions, cos_sin, T_pad, error_word(q.device))
    return grouped_gemm(xs, w_uk_t, tile), q_pe


def mla_output(o_lat: torch.Tensor, w_uv: torch.Tensor, T: int, row_map: Optional[torch.Tensor] = None,
               out_rows: Optional[int] = None) -> torch.Tensor:
    """[H, T_pad, kv_lora] latent attention output -> [T, H * v] through W_UV
    (a grouped GEMM with heads as groups, then a head-major -> row-major
    copy for o_proj). With ``row_map`` (int32 [T]) token t lands in row
    row_map[t] of an [out_rows, H * v] result; rows no token maps to are
    left unwritten on the GPU (zero on the CPU)."""
    if not o_lat.is_cuda:
        return ref.mla_output(o_lat, w_uv, T, row_map, out_rows)
    H, T_pad, _ = o_lat.shape
    ys = grouped_gemm(o_lat, w_uv, _group_tile(T))
    rows = T if row_map is None else out_rows
    out = torch.empty(rows, H * w_uv.shape[1], dtype=o_lat.dtype, device=o_lat.device)
    _count()
    native().mla_heads_to_rows(out, ys, T, row_map, error_word(o_lat.device))
    return out


class MlaPrefillPlan:
    """Host-built layout of a prefill batch's keys for the non-absorbed MLA
    path: every request's keys (cached and new) in a compact order padded to
    whole pages of 64, with the page table of that order and each compact
    row's (request, position) for the gather. Built once per batch; used by
    every layer."""

    PAGE = 64

    def __init__(self, lens: List[int], device: torch.device) -> None:
        import numpy as np

        P = self.PAGE
        pages = [(L + P - 1) // P for L in lens]
        base = np.concatenate([[0], np.cumsum(pages)]).astype(np.int64)
        self.rows = int(base[-1]) * P                       # R: compact key rows
        width = max(P, max(pages) * P)
        table = np.zeros((len(lens), width), dtype=np.int32)
        row_req = np.full(self.rows, -1, dtype=np.int32)
        row_pos = np.zeros(self.rows, dtype=np.int32)
        for b, L in enumerate(lens):
            start = int(base[b]) * P
            table[b, :pages[b] * P] = start + np.arange(pages[b] * P, dtype=np.int32)
            row_req[start:start + L] = b
            row_pos[start:start + L] = np.arange(L, dtype=np.int32)
        host = torch.from_numpy(np.concatenate([table.reshape(-1), row_req, row_pos]))
        if device.type == "cuda":
            host = host.pin_memory()
        dev = host.to(device, non_blocking=True)
        n = table.size
        self.page_table = dev[:n].view(len(lens), width)
        self.rows_in_order = torch.arange(len(lens), dtype=torch.int32, device=device)
        self.row_req = dev[n:n + self.rows]
        self.row_pos = dev[n + self.rows:]


def mla_rope_q(q: torch.Tensor, rope: int, positions: torch.Tensor, cos_sin: torch.Tensor) -> torch.Tensor:
    """Rotated rope parts [T, H, rope] of q [T, H, nope + rope] (no W_UK
    absorption): the non-absorbed prefill's queries keep q_nope as it is."""
    if not q.is_cuda:
        return ref.mla_rope_q(q, rope, positions, cos_sin)
    T, H, _ = q.shape
    q_pe = torch.empty(T, H, rope, dtype=q.dtype, device=q.device)
    _count()
    native().mla_rope_q(q_pe, q, positions, cos_sin, error_word(q.device))
    return q_pe


def mla_prefill_attention(q: torch.Tensor, q_rope: torch.Tensor, latent: torch.Tensor, page_table: torch.Tensor,
                          req_rows: torch.Tensor, seq_lens: torch.Tensor, cu_q: torch.Tensor, max_q: int,
                          w_kv_b: torch.Tensor, nope: int, v_dim: int, page_size: int, scale: float,
                          plan: Optional[MlaPrefillPlan] = None) -> torch.Tensor:
    """Non-absorbed causal MLA for prefill: q [T, H, nope + rope] (q_nope as
    projected), q_rope [T, H, rope] rotated -> [T, H * v_dim].

    On the GPU: gather every key's latent row of the batch (``plan`` order),
    expand c_kv through kv_b_proj with the tcgen05 GEMM into per-head
    k_nope / v, lay them out as a paged pool, and run the prefill attention
    kernel with the 64-dim rope part as a third Q chunk and a per-tile
    k_rope tile. Per query-key pair and head that is 2 * (192 + 128) FLOPs
    against 2 * (576 + 512) for the absorbed form, for an expansion of
    2 * 512 * H * 256 FLOPs per key once per layer."""
    T, H, qk = q.shape
    kv_lora = latent.shape[-1] - (qk - nope)
    if not q.is_cuda:
        return ref.mla_prefill_attention(q, q_rope, latent, page_table, req_rows, seq_lens, cu_q, w_kv_b, kv_lora,
                                         nope, v_dim, page_size, scale)
    if nope != 128 or v_dim != 128 or qk - nope != 64 or kv_lora != 512:
        raise ValueError("the sm_100a MLA prefill kernel takes nope 128, rope 64, v 128 and kv_lora 512")
    if plan is None:
        plan = MlaPrefillPlan(seq_lens.tolist(), q.device)
    nat = native()
    err = error_word(q.device)
    R = plan.rows
    x = torch.empty(R, kv_lora, dtype=q.dtype, device=q.device)
    k_rope = torch.empty(R, 64, dtype=q.dtype, device=q.device)
    _count()
    nat.mla_gather_keys(x, k_rope, latent, page_table, req_rows, plan.row_req, plan.row_pos, err)
    y = gemm(x, w_kv_b)                                           # [R, H * 256]
    pool = torch.empty(2, 1, R // MlaPrefillPlan.PAGE, H, MlaPrefillPlan.PAGE, 128, dtype=q.dtype, device=q.device)
    _count()
    nat.mla_scatter_kv(pool, y, H)
    out = torch.empty(T, H * v_dim, dtype=q.dtype, device=q.device)
    _count()
    nat.mla_prefill_attention(q.reshape(T, H * qk), out, pool, plan.page_table, plan.rows_in_order, seq_lens, cu_q,
                              max_q, H, qk, MlaPrefillPlan.PAGE, scale, q_rope, k_rope, err)
    return out


_MLA_SCRATCH: dict = {}


def mla_attention(
    q_lat: torch.Tensor,
    q_pe: torch.Tensor,
    latent: torch.Tensor,
    page_table: torch.Tensor,
    req_rows: torch.Tensor,
    seq_lens: torch.Tensor,
    cu_q: torch.Tensor,
    page_size: int,
    scale: float,
    splits: int = 0,
    trace: Optional[torch.Tensor] = None,
) -> torch.Tensor:
    """Causal absorbed MLA over the paged latent cache of one layer:
    q_lat [H, T_pad, kv_lora] + q_pe [T, H, rope] -> [H, T_pad, kv_lora]
    (one CTA per query token and 64 heads; split-KV when there are few
    tokens). ``trace``: optional int64 [512] device tensor that receives
    per-tile phase timestamps of the first CTA (copy issued, QK issued,
    scores seen, P written, PV issued, PV seen complete; 8 slots a tile)."""
    if not q_lat.is_cuda:
        return ref.mla_attention(q_lat, q_pe, latent, page_table, req_rows, seq_lens, cu_q, page_size, scale)
    H, T_pad, kv_lora = q_lat.shape
    T = q_pe.shape[0]
    nat = native()
    splits = splits or nat.mla_num_splits(T, H)
    out = torch.empty_like(q_lat)
    part_o = part_lse = None
    if splits > 1:
        part_o, part_lse = _mla_partials(splits, T, H, kv_lora, q_lat.device)
    _count(2 if splits > 1 else 1)
    nat.mla_attention(out, q_lat, q_pe, latent, page_table, req_rows, seq_lens, cu_q, page_size, scale, splits,
                      part_o, part_lse, error_word(q_lat.device), trace)
    return out


def _mla_partials(parts: int, T: int, H: int, kv_lora: int, device: torch.device):
    """fp32 partial outputs [parts, T, H, kv_lora] and log-sum-exps
    [parts, T, H] (one cached buffer per device)."""
    need = parts * T * H * (kv_lora + 1)
    buf = _MLA_SCRATCH.get(device)
    if buf is None or buf.numel() < need:
        buf = torch.empty(max(need, 148 * 64 * (kv_lora + 1)), dtype=torch.float32, device=device)
        _MLA_SCRATCH[device] = buf
    return buf[: parts * T * H * kv_lora], buf[parts * T * H * kv_lora: need]


def mla_attention_share(q_lat: torch.Tensor, q_pe: torch.Tensor, latent: torch.Tensor, page_table: torch.Tensor,
                        req_rows: torch.Tensor, seq_lens: torch.Tensor, cu_q: torch.Tensor, page_size: int,
                        scale: float, cp_size: int, cp_rank: int, cp_group, splits: int = 0) -> torch.Tensor:
    """Context-parallel MLA: this rank attends every query over the 64-key
    tiles it holds (tile t on rank t % cp) and returns its SHARE of the
    merged output, [H, T_pad, kv_lora]: its partial output weighted by
    exp(lse_rank - lse_all). Only the log-sum-exps cross the ranks (one
    in-place all-gather of [cp * splits, T, H] fp32); the shares add up to
    the attention output, so the caller reduces them after W_UV, where a
    token's row is 4x narrower than the latent output (128 vs 512 per head)."""
    import torch.distributed as dist

    H, T_pad, kv_lora = q_lat.shape
    T = q_pe.shape[0]
    if not q_lat.is_cuda:
        o, lse = ref.mla_attention_partial(q_lat, q_pe, latent, page_table, req_rows, seq_lens, cu_q, page_size,
                                           scale, cp_size, cp_rank)
        lses = [torch.empty_like(lse) for _ in range(cp_size)]
        dist.all_gather(lses, lse.contiguous(), group=cp_group)
        share = ref.mla_share(o, torch.stack(lses), cp_rank).to(q_lat.dtype)
        out = torch.zeros_like(q_lat)
        out[:, :T] = share
        return out
    nat = native()
    splits = splits or max(1, nat.mla_num_splits(T, H) // cp_size)
    part_o, part_lse = _mla_partials(splits * cp_size, T, H, kv_lora, q_lat.device)
    out = torch.empty_like(q_lat)
    _count(2)
    err = error_word(q_lat.device)
    nat.mla_attention(out, q_lat, q_pe, latent, page_table, req_rows, seq_lens, cu_q, page_size, scale, splits,
                      part_o, part_lse, err, None, cp_size, cp_rank, False)
    per_l = splits * T * H
    dist.all_gather_into_tensor(part_lse, part_lse[cp_rank * per_l:(cp_rank + 1) * per_l], group=cp_group)
    nat.mla_attention(out, q_lat, q_pe, latent, page_table, req_rows, seq_lens, cu_q, page_size, scale, splits,
                      part_o, part_lse, err, None, cp_size, cp_rank, True, True)
    return out


def prefill_attention(
    q: torch.Tensor,
    kv_pool: torch.Tensor,
    layer: int,
    page_table: torch.Tensor,
    req_rows: torch.Tensor,
    seq_lens: torch.Tensor,
    cu_q: torch.Tensor,
    max_q: int,
    hq: int,
    hk: int,
    d: int,
    page_size: int,
    scale: float,
    out: Optional[torch.Tensor] = None,
    trace: Optional[torch.Tensor] = None,
) -> torch.Tensor:
    """Causal prefill / extend attention over the paged pool. ``trace``:
    optional int64 [512] device tensor that receives %globaltimer stamps of
    the first 64 key tiles of one CTA (the one with the longest key range of
    request 0, head 0) — producer copy, QK issue, scores ready, exps done,
    previous PV done, P written, PV issue, scores read — for profiling."""
    T = q.shape[0]
    if not q.is_cuda:
        qv = q[:, : hq * d].reshape(T, hq, d)
        y = ref.attention(qv, kv_pool, layer, page_table, req_rows, seq_lens, cu_q, hq, hk, d, page_size, scale)
        y = y.view(T, hq * d)
        if out is not None:
            out.copy_(y)
            return out
        return y
    if out is None:
        out = torch.empty(T, hq * d, dtype=q.dtype, device=q.device)
    _count()
    native().prefill_attention(
        q, out, kv_pool, layer, page_table, req_rows, seq_lens, cu_q, max_q, hq, hk, d, page_size, scale,
        error_word(q.device), trace,
    )
    return out


# --------------------------------------------------------------- sampling
def argmax(logits: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    if not logits.is_cuda:
        y = ref.argmax(logits)
        if out is not None:
            out.copy_(y)
            return out
        return y
    if out is None:
        out = torch.empty(logits.shape[0], dtype=torch.int32, device=logits.device)
    _count(2)  # vocabulary-chunk partials + per-row reduce
    native().argmax(out, logits.float() if logits.dtype != torch.float32 else logits)
    return out


def sample(
    logits: torch.Tensor,
    temperature: torch.Tensor,
    top_k: Optional[torch.Tensor] = None,
    top_p: Optional[torch.Tensor] = None,
    seed: int = 0,
    step: Optional[torch.Tensor] = None,
    out: Optional[torch.Tensor] = None,
    generator: Optional[torch.Generator] = None,
) -> torch.Tensor:
    if not logits.is_cuda:
        y = ref.sample(logits, temperature, top_k, top_p, generator)
        if out is not None:
            out.copy_(y)
            return out
        return y
    if out is None:
        out = torch.empty(logits.shape[0], dtype=torch.int32, device=logits.device)
    lf = logits if logits.dtype == torch.float32 else logits.float()
    _count(2 if step is not None else 1)
    native().sample(out, lf, temperature, top_k, top_p, seed, step)
    return out


_SAMPLE_PARTS: dict = {}


def sample_sharded(logits: torch.Tensor, temperature: Optional[torch.Tensor], seed: int, step: torch.Tensor,
                   offset: int, comm) -> torch.Tensor:
    """Tokens from vocabulary-sharded logits under tensor parallelism: each
    rank reduces its shard [B, V_shard] (global indices from ``offset``) to
    per-chunk (best score, index) pairs, the pairs of every rank are gathered
    (``comm.all_gather``, a few KB instead of the [B, V] logits) and one small
    kernel picks each row's token. Scores are those of ``sample`` / ``argmax``
    over the whole vocabulary (same counter-based Gumbel stream, same tie
    rule), so every rank draws the same tokens as an unsharded sampler would.
    ``temperature`` None: greedy."""
    B = logits.shape[0]
    chunks = native().sample_shard_chunks(logits.shape[1])
    ld = (2 * chunks + 3) // 4 * 4  # rows of whole 16-byte vectors for the gather
    packed = torch.empty(B, ld, dtype=torch.int32, device=logits.device)
    out = torch.empty(B, dtype=torch.int32, device=logits.device)
    _count(2)
    native().sample_shard_partials(packed, logits, temperature, seed, step, offset)
    gathered = comm.all_gather(packed)
    native().sample_shard_reduce(out, gathered, chunks, gathered.shape[0] // max(B, 1), temperature, step)
    return out


def lm_head_sample(
    x: torch.Tensor,
    w: torch.Tensor,
    bias: Optional[torch.Tensor],
    temperature: Optional[torch.Tensor],
    seed: int,
    step: torch.Tensor,
    out: Optional[torch.Tensor] = None,
    plan: Optional[Tuple[int, int]] = None,
    generator: Optional[torch.Generator] = None,
) -> torch.Tensor:
    """Tokens sampled from x @ w^T (+ bias) without materialising the logits:
    the LM-head GEMM's epilogue keeps, per 128-row vocabulary tile, the best
    Gumbel-perturbed score (temperature None: the plain logit, i.e. greedy),
    and a small kernel reduces the tiles. Draws the same random numbers as
    ``sample`` for the same (seed, step), so both paths give the same tokens
    for the same logits. ``plan`` = (token tile, K splits) for tests."""
    M, N = x.shape[0], w.shape[0]
    if not x.is_cuda:
        logits = ref.gemm(x, w, bias, torch.float32)
        y = ref.argmax(logits) if temperature is None else ref.sample(logits, temperature, None, None, generator)
        if out is not None:
            out.copy_(y)
            return out
        return y
    if out is None:
        out = torch.empty(M, dtype=torch.int32, device=x.device)
    ntiles = (N + 127) // 128
    key = (x.device.index, N)
    buf = _SAMPLE_PARTS.get(key)
    if buf is None or buf[0].numel() < M * ntiles or torch.cuda.is_current_stream_capturing():
        buf = (torch.empty(M * ntiles, dtype=torch.float32, device=x.device),
               torch.empty(M * ntiles, dtype=torch.int32, device=x.device))
        if not torch.cuda.is_current_stream_capturing():
            _SAMPLE_PARTS[key] = buf
    if plan is None:
        tuned = _gemm_fused_plans.get((M, N, x.shape[1]))
        splits, bn = (tuned[2], tuned[1]) if tuned is not None and tuned[0] == 2 else (0, 0)
    else:
        bn, splits = plan
    _count(2)
    native().gemm_sample(out, x, w, bias, temperature, seed, step, buf[0], buf[1], splits, bn, error_word(x.device))
    return out


# -------------------------------------------------------------------- MoE
def moe_tile(tokens: int, k: int, experts: int) -> int:
    """Token tile of the grouped expert GEMMs: about the average number of
    rows an expert receives (padding per expert is below one tile)."""
    avg = tokens * k / max(1, experts)
    return 16 if avg <= 16 else 32 if avg <= 48 else 64 if avg <= 160 else 128


def moe_experts(x: torch.Tensor, w1: torch.Tensor, w2: torch.Tensor, topk_w: torch.Tensor,
                topk_ids: torch.Tensor, tile: int = 0) -> torch.Tensor:
    """sum_j topk_w[t, j] * w2_e (silu(gate) * up)(w1_e x_t) over the k routed
    experts e = topk_ids[t, j]; w1 [E, 2I, H] with gate|up rows interleaved in
    64-row blocks per expert, w2 [E, H, I]. Expert-sorted grouped tcgen05
    GEMMs (align, gather, gate_up with SiLU epilogue, down, combine)."""
    T, H = x.shape
    E, I, k = w1.shape[0], w2.shape[2], topk_ids.shape[1]
    out = torch.empty(T, H, dtype=x.dtype, device=x.device)
    if T == 0:
        return out
    tile = tile or moe_tile(T, k, E)
    P = T * k + E * (tile - 1)
    dev, i32 = x.device, torch.int32
    xs = torch.empty(P, H, dtype=x.dtype, device=dev)
    h = torch.empty(P, I, dtype=x.dtype, device=dev)
    ys = torch.empty(P, H, dtype=x.dtype, device=dev)
    sorted_pair = torch.empty(P, dtype=i32, device=dev)
    pair_pos = torch.empty(T * k, dtype=i32, device=dev)
    tile_expert = torch.empty(P // tile, dtype=i32, device=dev)
    tile_row = torch.empty(P // tile, dtype=i32, device=dev)
    num_tiles = torch.empty(1, dtype=i32, device=dev)
    _count(5)  # align, gather, two grouped GEMMs, combine
    native().moe_experts(out, x.contiguous(), w1, w2, topk_w.float().contiguous(), topk_ids.to(i32).contiguous(),
                         tile, xs, h, ys, sorted_pair, pair_pos, tile_expert, tile_row, num_tiles, error_word(dev))
    return out


def moe_tile_mxfp4(tokens: int, k: int, experts: int) -> int:
    """Token tile of the MXFP4 expert GEMMs: every tile expands its expert's
    weights to bf16 again, so tiles grow to 128 rows once an expert gets more
    than 64 (measured at Kimi-K2 expert dims: 0.51 vs 0.61 ms at 128 rows per
    expert)."""
    avg = tokens * k / max(1, experts)
    return 16 if avg <= 16 else 32 if avg <= 48 else 64 if avg <= 64 else 128


def moe_experts_mxfp4(x: torch.Tensor, w1q: torch.Tensor, w1s: torch.Tensor, w2q: torch.Tensor, w2s: torch.Tensor,
                      topk_w: torch.Tensor, topk_ids: torch.Tensor, tile: int = 0) -> torch.Tensor:
    """``moe_experts`` with MXFP4 expert weights (packed [E, N, K / 2] +
    scales [E, K / 64, N, 2], see minisgl.quant.mxfp4): the grouped GEMMs
    expand E2M1 to bf16 in shared memory, activations stay bf16."""
    T, H = x.shape
    E, I2 = w1q.shape[0], w1q.shape[1]
    I, k = I2 // 2, topk_ids.shape[1]
    out = torch.empty(T, H, dtype=x.dtype, device=x.device)
    if T == 0:
        return out
    tile = tile or moe_tile_mxfp4(T, k, E)
    P = T * k + E * (tile - 1)
    Pp = (P + tile - 1) // tile * tile
    dev, i32 = x.device, torch.int32
    xs = torch.empty(Pp, H, dtype=x.dtype, device=dev)
    h = torch.empty(Pp, I, dtype=x.dtype, device=dev)
    ys = torch.empty(Pp, H, dtype=x.dtype, device=dev)
    sorted_pair = torch.empty(P, dtype=i32, device=dev)
    pair_pos = torch.empty(T * k, dtype=i32, device=dev)
    tile_expert = torch.empty(P // tile, dtype=i32, device=dev)
    tile_row = torch.empty(P // tile, dtype=i32, device=dev)
    num_tiles = torch.empty(1, dtype=i32, device=dev)
    _count(5)  # align, gather, two grouped GEMMs, combine
    native().moe_experts_mxfp4(out, x.contiguous(), w1q, w1s, w2q, w2s, topk_w.float().contiguous(),
                               topk_ids.to(i32).contiguous(), tile, xs, h, ys, sorted_pair, pair_pos, tile_expert,
                               tile_row, num_tiles, error_word(dev))
    return out


def _moe_experts_mx_rows(x, mxfp4, blocked, topk_w, topk_ids, tile: int):
    """moe_experts_rows for block-scaled MX experts: (ys, pair_pos)."""
    T, H = x.shape
    k = topk_ids.shape[1]
    E, I = mxfp4[0].shape[0], mxfp4[0].shape[1] // 2
    P = T * k + E * (tile - 1)
    Pp = (P + tile - 1) // tile * tile
    dev, i32, u8 = x.device, torch.int32, torch.uint8
    ys = torch.empty(Pp, H, dtype=x.dtype, device=dev)
    pair_pos = torch.empty(T * k, dtype=i32, device=dev)
    _count(5)  # align, gather + quantise, gate_up GEMM, quantise, down GEMM
    native().moe_experts_mx(torch.empty(0, H, dtype=x.dtype, device=dev), x.contiguous(), mxfp4[0], blocked[0],
                            mxfp4[2], blocked[1], topk_w.float().contiguous(), topk_ids.to(i32).contiguous(), tile,
                            torch.empty(Pp, H, dtype=u8, device=dev),
                            torch.empty(Pp // tile, H // 128, 512, dtype=u8, device=dev),
                            torch.empty(Pp, I, dtype=x.dtype, device=dev), torch.empty(Pp, I, dtype=u8, device=dev),
                            torch.empty(Pp // tile, I // 128, 512, dtype=u8, device=dev), ys,
                            torch.empty(P, dtype=i32, device=dev), pair_pos,
                            torch.empty(P // tile, dtype=i32, device=dev), torch.empty(P // tile, dtype=i32, device=dev),
                            torch.empty(1, dtype=i32, device=dev), error_word(dev), False)
    return ys, pair_pos


def mx8_quantize(x: torch.Tensor, tile: int, idx: Optional[torch.Tensor] = None, k: int = 1,
                 rows: Optional[int] = None) -> Tuple[torch.Tensor, torch.Tensor]:
    """MXFP8 rows for the block-scaled expert GEMM (E4M3 + E8M0 per 32, as
    minisgl.quant.quantize_mx8_reference states it): returns (q uint8
    [rows, K], scale blocks uint8 [rows / tile, K / 128, 512]). Row p is
    x[idx[p] // k] (zeros where idx[p] < 0) or, without idx, x[p]."""
    K = x.shape[1]
    rows = rows if rows is not None else (idx.shape[0] if idx is not None else x.shape[0])
    q = torch.empty(rows, K, dtype=torch.uint8, device=x.device)
    sf = torch.empty(rows // tile, K // 128, 512, dtype=torch.uint8, device=x.device)
    _count()
    native().mx8_quantize(q, sf, x.contiguous(), None if idx is None else idx.to(torch.int32).contiguous(), k, rows,
                          tile)
    return q, sf


def moe_experts_mx(x: torch.Tensor, w1q: torch.Tensor, w1sb: torch.Tensor, w2q: torch.Tensor, w2sb: torch.Tensor,
                   topk_w: torch.Tensor, topk_ids: torch.Tensor, tile: int = 0) -> torch.Tensor:
    """``moe_experts`` on the block-scaled tensor cores: MXFP4 expert weights
    (packed [E, N, K / 2] with scale blocks [E, N / 128, K / 128, 512] from
    minisgl.quant.block_scales) times MXFP8 token rows (quantised on the
    fly, per 32 along K), tcgen05 .kind::mxf8f6f4 with E8M0 scales. Oracle:
    minisgl.quant.moe_experts_mx_reference. Takes the place of the
    reference's bf16 Triton expert kernel
    (python/minisgl/kernel/triton/fused_moe.py:50-193) for quantised experts."""
    T, H = x.shape
    E, I2 = w1q.shape[0], w1q.shape[1]
    I, k = I2 // 2, topk_ids.shape[1]
    out = torch.empty(T, H, dtype=x.dtype, device=x.device)
    if T == 0:
        return out
    tile = tile or moe_tile(T, k, E)
    P = T * k + E * (tile - 1)
    Pp = (P + tile - 1) // tile * tile
    dev, i32, u8 = x.device, torch.int32, torch.uint8
    xq = torch.empty(Pp, H, dtype=u8, device=dev)
    xsf = torch.empty(Pp // tile, H // 128, 512, dtype=u8, device=dev)
    h = torch.empty(Pp, I, dtype=x.dtype, device=dev)
    hq = torch.empty(Pp, I, dtype=u8, device=dev)
    hsf = torch.empty(Pp // tile, I // 128, 512, dtype=u8, device=dev)
    ys = torch.empty(Pp, H, dtype=x.dtype, device=dev)
    sorted_pair = torch.empty(P, dtype=i32, device=dev)
    pair_pos = torch.empty(T * k, dtype=i32, device=dev)
    tile_expert = torch.empty(P // tile, dtype=i32, device=dev)
    tile_row = torch.empty(P // tile, dtype=i32, device=dev)
    num_tiles = torch.empty(1, dtype=i32, device=dev)
    _count(6)  # align, gather + quantise, gate_up GEMM, quantise, down GEMM, combine
    native().moe_experts_mx(out, x.contiguous(), w1q, w1sb, w2q, w2sb, topk_w.float().contiguous(),
                            topk_ids.to(i32).contiguous(), tile, xq, xsf, h, hq, hsf, ys, sorted_pair, pair_pos,
                            tile_expert, tile_row, num_tiles, error_word(dev))
    return out


def moe_experts_quantised(x: torch.Tensor, mxfp4: tuple, topk_w: torch.Tensor, topk_ids: torch.Tensor) -> torch.Tensor:
    """MXFP4 routed experts: on the block-scaled tensor cores with MXFP8
    activations when the weights carry scale blocks (``--moe-quant
    mxfp4-a8``, minisgl.quant.MxfpExperts.blocked), else W4A16."""
    blocked = getattr(mxfp4, "blocked", None)
    if blocked is not None:
        return moe_experts_mx(x, mxfp4[0], blocked[0], mxfp4[2], blocked[1], topk_w, topk_ids)
    return moe_experts_mxfp4(x, *mxfp4, topk_w, topk_ids)


def moe_experts_rows(x: torch.Tensor, topk_w: torch.Tensor, topk_ids: torch.Tensor, w1=None, w2=None,
                     mxfp4: Optional[tuple] = None, tile: int = 0):
    """The expert pipeline without the combine: returns (ys [P, H] expert
    output rows, pair_pos [T * k] row of each (token, slot) pair, -1 for
    pairs whose expert is not here)."""
    T, H = x.shape
    k = topk_ids.shape[1]
    E = (mxfp4[0] if mxfp4 is not None else w1).shape[0]
    I = (mxfp4[2].shape[2] * 2) if mxfp4 is not None else w2.shape[2]
    blocked = getattr(mxfp4, "blocked", None)
    if blocked is not None:  # block-scaled MX experts (MXFP8 activations)
        return _moe_experts_mx_rows(x, mxfp4, blocked, topk_w, topk_ids, tile or moe_tile(T, k, E))
    tile = tile or (moe_tile_mxfp4(T, k, E) if mxfp4 is not None else moe_tile(T, k, E))
    P = T * k + E * (tile - 1)
    Pp = (P + tile - 1) // tile * tile
    dev, i32 = x.device, torch.int32
    xs = torch.empty(Pp, H, dtype=x.dtype, device=dev)
    h = torch.empty(Pp, I, dtype=x.dtype, device=dev)
    ys = torch.empty(Pp, H, dtype=x.dtype, device=dev)
    sorted_pair = torch.empty(P, dtype=i32, device=dev)
    pair_pos = torch.empty(T * k, dtype=i32, device=dev)
    tile_expert = torch.empty(P // tile, dtype=i32, device=dev)
    tile_row = torch.empty(P // tile, dtype=i32, device=dev)
    num_tiles = torch.empty(1, dtype=i32, device=dev)
    out = torch.empty(0, H, dtype=x.dtype, device=dev)
    _count(4)  # align, gather, two grouped GEMMs
    if mxfp4 is not None:
        native().moe_experts_mxfp4(out, x, *mxfp4, topk_w.float().contiguous(), topk_ids.to(i32).contiguous(), tile,
                                   xs, h, ys, sorted_pair, pair_pos, tile_expert, tile_row, num_tiles,
                                   error_word(dev), False)
    else:
        native().moe_experts(out, x, w1, w2, topk_w.float().contiguous(), topk_ids.to(i32).contiguous(), tile, xs, h,
                             ys, sorted_pair, pair_pos, tile_expert, tile_row, num_tiles, error_word(dev), False)
    return ys, pair_pos


def moe_combine(ys: torch.Tensor, topk_w: torch.Tensor, pair_pos: torch.Tensor, T: int, k: int) -> torch.Tensor:
    """out[t] = sum_j topk_w[t, j] * ys[pair_pos[t * k + j]] (slot order; -1 rows skipped)."""
    H = ys.shape[1]
    out = torch.empty(T, H, dtype=ys.dtype, device=ys.device)
    _count()
    native().moe_combine(out, ys, topk_w.float().contiguous(), pair_pos, T, k)
    return out


def moe_route(
    logits: torch.Tensor,
    k: int,
    scoring: str = "softmax",
    renormalize: bool = True,
    bias: Optional[torch.Tensor] = None,
    n_group: int = 1,
    topk_group: int = 1,
    routed_scale: float = 1.0,
) -> Tuple[torch.Tensor, torch.Tensor]:
    if not logits.is_cuda:
        return ref.moe_route(logits, k, scoring, renormalize, bias, n_group, topk_group, routed_scale)
    T = logits.shape[0]
    w = torch.empty(T, k, dtype=torch.float32, device=logits.device)
    ids = torch.empty(T, k, dtype=torch.int32, device=logits.device)
    _count()
    native().moe_route(
        logits.float().contiguous(), None if bias is None else bias.float(), w, ids,
        0 if scoring == "softmax" else 1, renormalize, n_group, topk_group, routed_scale,
    )
    return w, ids


# ------------------------------------------------------------ host helpers
@functools.lru_cache(maxsize=1)
def _host_compare():
    try:
        return native().fast_compare_key
    except RuntimeError:
        return None


def fast_compare_key(a: torch.Tensor, b: torch.Tensor) -> int:
    """Length of the common prefix of two 1-D CPU integer tensors."""
    fn = _host_compare()
    if fn is not None:
        return int(fn(a, b))
    return ref.fast_compare_key(a, b)
