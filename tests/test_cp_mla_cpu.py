"""Context parallelism for MLA on CPU ranks (gloo, world sizes 2 and 4):
each rank keeps the latent rows of the 64-key tiles it owns (tile t on rank
t % cp) in a pool of 1/cp of the pages (the allocator gives tile t a page of
id = t mod cp) and attends every query over them only. Prefill batches are
token-sharded (each rank runs the layers on the tokens of its own tiles);
the ranks' shares of the attention output meet after W_UV. The generated
tokens equal the single-rank engine's, also with the routed experts split
over the ranks (--ep). Prompts are longer than one tile so several ranks
hold keys, and chunks of 256 tokens put several requests and tiles of every
rank into one prefill batch."""

import socket

import pytest
import torch
import torch.multiprocessing as mp

PROMPTS = [[(13 * i + 7) % 1000 for i in range(150)], [(5 * i + 1) % 1000 for i in range(70)], [3, 4, 5]]


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _run(rank, world, port, cp, q, ep=1):
    from minisgl.core import SamplingParams
    from minisgl.llm import LLM
    from minisgl.parallel import DistributedInfo
    from minisgl.utils.synthetic import make_model_dir

    from minisgl.attention import mla as mla_backend

    plans = []  # (batch tokens, rows per rank) of every sharded prefill
    init = mla_backend.CPShardPlan.__init__

    def record(self, *args, **kwargs):
        init(self, *args, **kwargs)
        plans.append((self.T, self.T_max))

    mla_backend.CPShardPlan.__init__ = record
    llm = LLM(make_model_dir("tiny-kimi"), dtype=torch.float32, device="cpu", use_dummy_weight=True,
              tp_info=DistributedInfo(rank, world), page_size=64, num_page_override=64, max_running_req=4,
              max_seq_len_override=512, max_extend_tokens=256, distributed_port=port, cp_size=cp, ep_size=ep)
    if cp > 1:  # each rank holds one page in cp (plus spares)
        assert llm.engine.kv_cache.pool.shape[1] == llm.engine.num_pages // cp + 2
    outs = llm.generate(PROMPTS, SamplingParams(temperature=0.0, max_tokens=8, ignore_eos=True))
    q.put((rank, ([o["token_ids"] for o in outs], plans)))
    llm.shutdown()


def _generate(world, cp, ep=1):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_run, args=(r, world, port, cp, q, ep)) for r in range(world)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=300) for _ in range(world))
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    return results


@pytest.mark.parametrize("cp", [2, 4])
def test_cp_matches_single_rank(cp):
    single, plans = _generate(1, 1)[0]
    assert plans == []
    got = _generate(cp, cp)
    for r in range(cp):
        tokens, plans = got[r]
        assert tokens == single, (r, tokens, single)
        # the prefill really was split: some batch ran fewer rows per rank
        # than it has tokens
        assert plans and any(t_max < T for T, t_max in plans), plans


def test_cp_with_expert_parallelism_matches_single_rank():
    """cp 2 with the routed experts split over the two ranks: prefill rows
    travel to their experts' owners (all-to-all), decode rows run each
    rank's experts and are summed (all-reduce)."""
    single, _ = _generate(1, 1)[0]
    got = _generate(2, 2, ep=2)
    for r in range(2):
        tokens, plans = got[r]
        assert tokens == single, (r, tokens, single)
        assert plans and any(t_max < T for T, t_max in plans), plans
