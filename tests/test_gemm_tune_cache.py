"""The GEMM plan cache file (MINISGL_GEMM_TUNE_CACHE): plans written by one
run are read back unchanged by the next, per device name, so runs sharing the
file use the same kernels and produce bit-identical results. Fused-epilogue
entries use a negative M in their key."""

import json

from minisgl.ops import gemm_tune


def test_cache_roundtrip(tmp_path):
    path = str(tmp_path / "sub" / "plans.json")
    plans = {(64, 4096, 1024): (1, 128, 2), (-64, 3072, 1024): (2, 256, 1), (16384, 6144, 1024): (3, 256, 1)}
    gemm_tune._save(path, "NVIDIA B200", plans)
    gemm_tune._save(path, "other", {(1, 2, 3): (4, 5, 6)})
    assert gemm_tune._load(path, "NVIDIA B200") == plans
    assert gemm_tune._load(path, "other") == {(1, 2, 3): (4, 5, 6)}
    assert gemm_tune._load(path, "missing") == {}
    with open(path) as f:
        assert set(json.load(f)) == {"NVIDIA B200", "other"}


def test_cache_missing_or_corrupt(tmp_path):
    assert gemm_tune._load(None, "x") == {}
    assert gemm_tune._load(str(tmp_path / "none.json"), "x") == {}
    bad = tmp_path / "bad.json"
    bad.write_text("{not json")
    assert gemm_tune._load(str(bad), "x") == {}
    gemm_tune._save(None, "x", {(1, 1, 1): (1, 1, 1)})  # no path: nothing written, no error
