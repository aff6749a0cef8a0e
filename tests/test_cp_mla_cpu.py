"""Context parallelism for MLA on CPU ranks (gloo, world size 2): each rank
keeps the latent rows of the 64-key tiles it owns (tile t on rank t % 2) in
a pool of half the pages (the allocator gives tile t a page of id = t mod 2),
attends over them only, and the partial outputs / log-sum-exps of the ranks
are gathered and merged; the generated tokens equal the single-rank
engine's. Prompts are longer than one tile so both ranks hold keys."""

import socket

import torch
import torch.multiprocessing as mp

PROMPTS = [[(13 * i + 7) % 1000 for i in range(150)], [(5 * i + 1) % 1000 for i in range(70)], [3, 4, 5]]


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _run(rank, world, port, cp, q):
    from minisgl.core import SamplingParams
    from minisgl.llm import LLM
    from minisgl.parallel import DistributedInfo
    from minisgl.utils.synthetic import make_model_dir

    llm = LLM(make_model_dir("tiny-kimi"), dtype=torch.float32, device="cpu", use_dummy_weight=True,
              tp_info=DistributedInfo(rank, world), page_size=64, num_page_override=64, max_running_req=4,
              max_seq_len_override=512, max_extend_tokens=64, distributed_port=port, cp_size=cp)
    if cp > 1:  # each rank holds one page in cp (plus spares)
        assert llm.engine.kv_cache.pool.shape[1] == llm.engine.num_pages // cp + 2
    outs = llm.generate(PROMPTS, SamplingParams(temperature=0.0, max_tokens=8, ignore_eos=True))
    q.put((rank, [o["token_ids"] for o in outs]))
    llm.shutdown()


def _generate(world, cp):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_run, args=(r, world, port, cp, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=300) for _ in range(world))
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    return results


def test_cp2_matches_single_rank():
    single = _generate(1, 1)[0]
    cp = _generate(2, 2)
    assert cp[0] == cp[1] == single
