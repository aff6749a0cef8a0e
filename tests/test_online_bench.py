"""Trace reading of the online benchmark client (no server needed): Qwen
traces carry seconds, Mooncake traces milliseconds; offsets start at zero,
scale with --trace-scale, and come back sorted; extra fields are ignored."""

import json

import pytest

from minisgl.benchmark.online import _stats, make_prompts, read_trace


def _write(path, rows):
    path.write_text("\n".join(json.dumps(r) for r in rows) + "\n")


def test_read_qwen_and_mooncake(tmp_path):
    q = tmp_path / "qwen.jsonl"
    _write(q, [{"chat_id": 1, "parent_chat_id": -1, "timestamp": 10.5, "input_length": 30, "output_length": 4,
                "type": "text", "turn": 1, "hash_ids": [1]},
               {"chat_id": 2, "parent_chat_id": -1, "timestamp": 10.0, "input_length": 20, "output_length": 6,
                "type": "text", "turn": 1, "hash_ids": [2]}])
    e = read_trace(str(q), "qwen")
    assert [(x.start_s, x.input_len, x.output_len) for x in e] == [(0.0, 20, 6), (0.5, 30, 4)]
    m = tmp_path / "mooncake.jsonl"
    _write(m, [{"timestamp": 0, "input_length": 8, "output_length": 2, "hash_ids": []},
               {"timestamp": 1500, "input_length": 9, "output_length": 3, "hash_ids": []},
               {"timestamp": 3000, "input_length": 10, "output_length": 4, "hash_ids": []}])
    e = read_trace(str(m), "mooncake", scale=2.0)
    assert [x.start_s for x in e] == [0.0, 3.0, 6.0]
    assert len(read_trace(str(m), "mooncake", n=2)) == 2
    with pytest.raises(ValueError):
        read_trace(str(m), "sharegpt")


def test_prompts_and_stats():
    p = make_prompts(3, 7, None, seed=1)
    assert len(p) == 3 and all(len(x.split()) == 7 for x in p) and p == make_prompts(3, 7, None, seed=1)
    st = _stats([0.001 * i for i in range(1, 101)])
    assert st["p50"] == pytest.approx(51.0) and st["max"] == pytest.approx(100.0) and st["avg"] == pytest.approx(50.5)
    assert _stats([]) == {}
