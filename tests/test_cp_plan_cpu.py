"""Host-side decisions and layouts of the MLA paths, checked on their own
(no ranks, no kernels): the token-sharded context-parallel plan of a prefill
batch, the compact key layout of the non-absorbed MLA prefill and the FLOP
rule that picks the prefill form."""

import numpy as np
import torch

from minisgl.attention.mla import CPShardPlan
from minisgl.ops import MlaPrefillPlan


def _batch(starts, lens):
    """Positions and cu offsets of a prefill batch: request b extends from
    position starts[b] by lens[b] tokens."""
    pos = np.concatenate([np.arange(s, s + n) for s, n in zip(starts, lens)]).astype(np.int64)
    cu = np.concatenate([[0], np.cumsum(lens)]).astype(np.int64)
    return pos, cu


def test_cp_plan_shards_tokens_by_tile_owner():
    starts, lens = [0, 100, 5], [150, 70, 3]
    pos, cu = _batch(starts, lens)
    T = len(pos)
    out_loc = torch.arange(1000, 1000 + T, dtype=torch.int32)
    cp = 3
    owner = (pos // 64) % cp
    counts = np.bincount(owner, minlength=cp)
    plans = [CPShardPlan(pos, cu, cp, r, out_loc, torch.device("cpu"), None) for r in range(cp)]
    rm_rows = set()
    for r, p in enumerate(plans):
        assert p.T == T and p.T_max == counts.max() and p.T_own == counts[r]
        local = p.local.numpy()
        own = np.nonzero(owner == r)[0]
        assert (local[: len(own)] == own).all()
        # padding rows sit in another rank's tile: they store nothing here
        assert ((p.positions.numpy()[len(own):] // 64) % cp != r).all()
        assert (p.positions.numpy()[: len(own)] == pos[own]).all()
        assert torch.equal(p.out_loc[: len(own)], out_loc[torch.from_numpy(own)])
        # every rank agrees on the rank-major map; own tokens land in its block
        assert torch.equal(p.row_map, plans[0].row_map)
        rows = p.row_map.numpy()[own]
        assert (rows // p.T_max == r).all()
        assert sorted(rows % p.T_max) == list(range(len(own)))
        rm_rows.update(rows.tolist())
        # the last token of each request is found on exactly one rank
        last = cu[1:] - 1
        mine = np.nonzero(owner[last] == r)[0]
        assert (p.last_dst.numpy() == mine).all()
        assert (local[p.last_src.numpy()] == last[mine]).all()
    assert len(rm_rows) == T  # the map is one-to-one


def test_mla_prefill_plan_is_compact_and_page_aligned():
    lens = [1, 70, 128, 200]
    plan = MlaPrefillPlan(lens, torch.device("cpu"))
    pages = [(L + 63) // 64 for L in lens]
    assert plan.rows == 64 * sum(pages)
    base = 0
    req, pos = plan.row_req.numpy(), plan.row_pos.numpy()
    for b, L in enumerate(lens):
        start = base * 64
        # the request's keys fill its pages in order, the rest of the last page is padding
        assert (plan.page_table[b, :L].numpy() == start + np.arange(L)).all()
        assert (req[start:start + L] == b).all() and (pos[start:start + L] == np.arange(L)).all()
        assert (req[start + L:start + pages[b] * 64] == -1).all()
        base += pages[b]
    assert torch.equal(plan.rows_in_order, torch.arange(len(lens), dtype=torch.int32))


def test_mla_prefill_form_follows_flop_count(monkeypatch):
    """Kimi-K2 latent dims: the non-absorbed form (every key expanded through
    kv_b_proj) pays off once a request has a few hundred new tokens per key;
    a short extend over a long cached prefix stays absorbed; the switch
    forces either form."""
    from types import SimpleNamespace

    from minisgl.attention.mla import MLAAttnBackend

    dims = SimpleNamespace(kv_lora=512, nope=128, rope=64, v_dim=128)
    pick = lambda lens, qlens: MLAAttnBackend.expanded_prefill(dims, lens, qlens)  # noqa: E731
    monkeypatch.delenv("MINISGL_MLA_PREFILL", raising=False)
    assert pick([4096], [4096])             # a long prompt without cache
    assert not pick([64], [64])             # a short one
    assert not pick([8192], [16])           # a few new tokens after a long prefix
    monkeypatch.setenv("MINISGL_MLA_PREFILL", "expanded")
    assert pick([64], [64])
    monkeypatch.setenv("MINISGL_MLA_PREFILL", "absorbed")
    assert not pick([4096], [4096])
