"""Benchmark helpers without a GPU or server: trace reading of the online
client (Qwen traces carry seconds, Mooncake traces milliseconds; offsets
start at zero, scale with --trace-scale, and come back sorted; extra fields
are ignored) and the kernel benchmarks' SM clock summary."""

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


def test_sm_clock_log_summary():
    """The kernel benchmarks' clock summary keeps only the chosen GPU's
    samples, takes the median clock of the samples under load and lists
    the throttle reasons seen active."""
    from minisgl.benchmark.perf import SmClockLog

    text = ("0, 1455, 1965, 950.3, Not Active, Not Active, Not Active, Active\n"
            "0, 1500, 1965, 980.0, Not Active, Not Active, Not Active, Not Active\n"
            "0, 1965, 1965, 120.0, Not Active, Not Active, Not Active, Not Active\n"
            "1, 900, 1965, 999.0, Active, Not Active, Not Active, Not Active\n"
            "garbage line\n")
    c = SmClockLog.summarize(text, 0)["clocks"]
    assert c["sm_mhz_median_under_load"] == 1477.5 and c["samples_under_load"] == 2
    assert c["sm_max_mhz"] == 1965.0 and c["reasons"] == ["sw_power_cap"]


def test_pool_prompts_and_rates():
    """A benchmark pool as text: lengths and output lengths follow the pool,
    shared id prefixes stay shared text prefixes (the radix cache's hits),
    and sweep rates must be positive."""
    from minisgl.benchmark.online import parse_rates, pool_prompts
    from minisgl.benchmark.workload import make_pool

    texts, outs, lens = pool_prompts("qwen3-32b", 60, None, seed=2)
    ids, want_outs = make_pool("qwen3-32b", 60, 2)
    assert outs == want_outs and lens == [len(p) for p in ids]
    assert [len(t.split()) for t in texts] == lens
    shared = [(i, j) for i in range(60) for j in range(i) if ids[i][:512] == ids[j][:512]]
    assert shared  # 30 % of the prompts start with one of 50 prefixes
    for i, j in shared:
        assert texts[i].split()[:512] == texts[j].split()[:512]
    assert parse_rates("0.5, 2,inf") == [0.5, 2.0, float("inf")]
    with pytest.raises(ValueError):
        parse_rates("1,0")
