"""Expert parallelism and MXFP4 experts on the CPU.

* EP=2 over gloo ranks (experts split in halves, attention replicated, the
  partial expert sums meet in the tensor-parallel all-reduce) generates what
  the single-rank engine generates from the same checkpoint.
* The PyTorch MXFP4 quantiser follows the OCP MX rules: E8M0 exponents of
  floor(log2 amax) - 2, round-to-nearest-even E2M1 codes, saturation; the
  expert layer with MXFP4 weights equals the fp32 experts on the
  dequantised weights.
"""

import shutil
import socket
import tempfile

import pytest
import torch
import torch.multiprocessing as mp

from minisgl.quant import dequantize_mxfp4, quantize_mxfp4_reference

PROMPTS = [[5, 6, 7, 8, 9, 10, 11, 12, 13], [100, 200, 300, 400, 500, 600, 700, 800, 900, 1000, 11, 12]]


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _run(rank, world, folder, port, ep, quant, out_q):
    from minisgl.core import SamplingParams
    from minisgl.llm import LLM
    from minisgl.parallel import DistributedInfo

    llm = LLM(folder, dtype=torch.float32, device="cpu", tp_info=DistributedInfo(rank, world), page_size=16,
              num_page_override=64, max_running_req=4, max_seq_len_override=256, max_extend_tokens=64,
              distributed_port=port, ep_size=ep, moe_quant=quant)
    outs = llm.generate(PROMPTS, SamplingParams(temperature=0.0, max_tokens=8, ignore_eos=True))
    out_q.put((rank, [o["token_ids"] for o in outs]))
    llm.shutdown()


@pytest.fixture(scope="module")
def checkpoint():
    from minisgl.utils.synthetic import make_model_dir, write_random_checkpoint

    folder = tempfile.mkdtemp(prefix="minisgl_ep_ckpt_")
    shutil.rmtree(folder)
    make_model_dir("tiny-qwen3-moe", folder=folder)
    write_random_checkpoint(folder, seed=5, std=0.05)
    yield folder
    shutil.rmtree(folder, ignore_errors=True)


def _generate(world, folder, ep=1, quant="none"):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_run, args=(r, world, folder, port, ep, quant, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=300) for _ in range(world))
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    return results


def test_ep2_matches_single_rank(checkpoint):
    single = _generate(1, checkpoint)[0]
    ep = _generate(2, checkpoint, ep=2)
    assert ep[0] == ep[1] == single


def test_ep2_mxfp4_matches_single_rank_mxfp4(checkpoint):
    single = _generate(1, checkpoint, quant="mxfp4")[0]
    ep = _generate(2, checkpoint, ep=2, quant="mxfp4")
    assert ep[0] == ep[1] == single


def test_mxfp4_scale_and_rounding_rules():
    # block 0: amax 6 -> e = 0; ties round to even codes; block 1: amax 0.75 -> e = -3
    b0 = [0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0, 6.0, -0.3, -7.0] + [0.0] * 22
    b1 = [0.75, 0.1, -0.0625, 0.03125] + [0.0] * 28
    w = torch.tensor(b0 + b1, dtype=torch.float32).view(1, 1, 64)
    packed, scales = quantize_mxfp4_reference(w)
    assert scales.flatten().tolist() == [127, 124]
    d = dequantize_mxfp4(packed, scales).flatten()
    assert d[:10].tolist() == [0.0, 1.0, 1.0, 2.0, 2.0, 4.0, 4.0, 6.0, -0.25 * 2, -6.0]  # -0.3 -> -0.5
    # scale 2^-3: 0.1 / 0.125 = 0.8 -> 1.0; 0.03125 / 0.125 = 0.25 is a tie -> 0
    assert d[32:36].tolist() == [0.75, 0.125, -0.0625, 0.0]
    assert torch.all(dequantize_mxfp4(*quantize_mxfp4_reference(torch.zeros(2, 4, 64))) == 0)


def test_mxfp4_error_and_layer():
    from minisgl.moe.fused import FusedMoe, moe_reference
    from minisgl.ops import reference as ref

    torch.manual_seed(0)
    E, H, I, T, k = 4, 128, 128, 9, 2
    w1 = torch.randn(E, 2 * I, H) * 0.02
    w2 = torch.randn(E, H, I) * 0.02
    q1, q2 = quantize_mxfp4_reference(w1), quantize_mxfp4_reference(w2)
    d1 = dequantize_mxfp4(*q1)
    rel = ((d1 - w1).norm() / w1.norm()).item()
    assert 0.05 < rel < 0.15  # E2M1 keeps ~1 mantissa bit
    x = torch.randn(T, H)
    logits = torch.randn(T, E)
    got = FusedMoe().forward(x, w1, w2, logits, k, True, mxfp4=(q1[0], q1[1], q2[0], q2[1]))
    tw, ti = ref.moe_route(logits, k, "softmax", True)
    want = moe_reference(x, d1, dequantize_mxfp4(*q2), tw, ti, "silu")
    assert torch.allclose(got, want, atol=1e-5)


def test_ep2_mx_a8_matches_single_rank(checkpoint):
    """Block-scaled MX experts (MXFP8 activations, ``--moe-quant mxfp4-a8``)
    through the expert-parallel dispatch generate what one rank generates."""
    single = _generate(1, checkpoint, quant="mxfp4-a8")[0]
    ep = _generate(2, checkpoint, ep=2, quant="mxfp4-a8")
    assert ep[0] == ep[1] == single
