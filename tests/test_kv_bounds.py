"""Host KV bounds check (MINISGL_DEBUG_BOUNDS=1): bad slots in a batch's
writes or in a request's page-table row raise KVBoundsError naming the
request; a normal run (chunked prefill, radix reuse, decode) passes with the
check on and produces the same tokens as without it. Also the keying of the
device error word that the in-kernel index checks report through."""

from types import SimpleNamespace

import pytest
import torch

from minisgl.engine.bounds import KVBoundsError, check_kv_bounds


def _batch(out_loc, reqs, phase="decode"):
    return SimpleNamespace(out_loc=torch.tensor(out_loc, dtype=torch.int32), reqs=reqs, phase=phase)


def _req(uid, row, n):
    return SimpleNamespace(uid=uid, table_idx=row, device_len=n)


def test_bounds_unit():
    pt = torch.arange(4 * 8, dtype=torch.int32).view(4, 8)  # 4 rows x 8 positions, slots 0..31
    check_kv_bounds(pt, _batch([3, 31], [_req(1, 0, 8), _req(2, 3, 8)]), num_slots=32)
    check_kv_bounds(pt, _batch([32, 35], []), num_slots=32, spare_slots=4)  # padding writes the spare page
    with pytest.raises(KVBoundsError, match="writes KV slots"):
        check_kv_bounds(pt, _batch([5, 32], [_req(1, 0, 2)]), num_slots=32)
    bad = pt.clone()
    bad[2, 5] = 99
    with pytest.raises(KVBoundsError, match="request 7: page-table row 2 maps position 5 to slot 99"):
        check_kv_bounds(bad, _batch([0], [_req(7, 2, 6)]), num_slots=32)
    check_kv_bounds(bad, _batch([0], [_req(7, 2, 5)]), num_slots=32)  # position 5 not read yet
    with pytest.raises(KVBoundsError, match="outside the page table"):
        check_kv_bounds(pt, _batch([0], [_req(8, 4, 1)]), num_slots=32)


def test_engine_run_with_bounds_check(monkeypatch):
    from minisgl.core import SamplingParams
    from minisgl.env import ENV
    from minisgl.llm import LLM
    from minisgl.utils.synthetic import make_model_dir

    d = make_model_dir("tiny-qwen3")
    llm = LLM(d, dtype=torch.float32, device="cpu", use_dummy_weight=True, page_size=16, max_extend_tokens=32,
              num_page_override=64, max_running_req=8, max_seq_len_override=256, cache_type="radix")
    try:
        prompts = [list(range(5, 45)), list(range(5, 30)) + [7, 8], [3, 4, 5]]
        sp = SamplingParams(temperature=0.0, max_tokens=6, ignore_eos=True)
        plain = [o["token_ids"] for o in llm.generate(prompts, sp)]
        import minisgl.engine.bounds as bounds

        calls = []
        real = bounds.check_kv_bounds
        monkeypatch.setattr(bounds, "check_kv_bounds", lambda *a, **k: (calls.append(1), real(*a, **k)))
        monkeypatch.setattr(ENV.DEBUG_BOUNDS, "value", True)
        checked = [o["token_ids"] for o in llm.generate(prompts, sp)]
        assert checked == plain
        assert len(calls) >= 6  # prefill chunks and every decode step were checked
    finally:
        llm.shutdown()


def test_error_word_key_names_the_current_device(monkeypatch):
    """The device error word is kept per (type, index); a CUDA device given
    without an index means the current one, so a check through
    torch.device("cuda") reads the word kernels on cuda:N write."""
    import torch

    from minisgl import ops

    monkeypatch.setattr(torch.cuda, "current_device", lambda: 3)
    assert ops._device_key(torch.device("cuda")) == ("cuda", 3)
    assert ops._device_key("cuda") == ("cuda", 3)
    assert ops._device_key(torch.device("cuda", 1)) == ("cuda", 1)
    assert ops._device_key(torch.device("cpu")) == ("cpu", None)
