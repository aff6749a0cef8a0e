"""Command-line parsing (reference: python/minisgl/server/args.py:54-268):
defaults, the collective backend switch, context parallelism over all ranks
and the CPU dtype rule."""

import pytest
import torch

from minisgl.server.args import parse_args


def test_defaults_use_the_nvlink_collectives():
    args, shell = parse_args(["--model", "synthetic:tiny-qwen3", "--tp", "2"])
    assert not shell
    assert args.comm == "fused" and args.tp_info.size == 2 and args.tp_info.rank == 0
    assert args.use_dummy_weight  # a synthetic model has no checkpoint
    assert args.dtype == torch.bfloat16


def test_disable_pynccl_selects_the_nccl_baseline():
    args, _ = parse_args(["--model", "synthetic:tiny-qwen3", "--tp", "2", "--disable-pynccl"])
    assert args.comm == "nccl"
    args, _ = parse_args(["--model", "synthetic:tiny-qwen3", "--comm", "nccl"])
    assert args.comm == "nccl"


def test_context_parallel_spans_every_rank():
    args, _ = parse_args(["--model", "synthetic:tiny-kimi", "--cp", "4"])
    assert args.cp_size == 4 and args.tp_info.size == 4
    args, _ = parse_args(["--model", "synthetic:tiny-kimi", "--cp", "2", "--tp", "2", "--ep", "2"])
    assert args.tp_info.size == 2 and args.ep_size == 2
    with pytest.raises(SystemExit):
        parse_args(["--model", "synthetic:tiny-kimi", "--cp", "2", "--tp", "4"])


def test_cpu_device_runs_fp32_and_shell_mode_serves_one_request():
    args, shell = parse_args(["--model", "synthetic:tiny-qwen3", "--device", "cpu", "--shell-mode"])
    assert shell and args.dtype == torch.float32
    assert args.max_running_req == 1 and args.cuda_graph_max_bs == 1


def test_profile_steps_flag_sets_the_profiler_window(monkeypatch):
    from minisgl.env import ENV

    # recorded by monkeypatch, so the value parse_args sets is undone afterwards
    monkeypatch.setenv("MINISGL_CUDA_PROFILER_STEPS", "")
    monkeypatch.setattr(ENV.CUDA_PROFILER_STEPS, "value", "")
    parse_args(["--model", "synthetic:tiny-qwen3", "--profile-steps", "10:20"])
    import os

    assert os.environ["MINISGL_CUDA_PROFILER_STEPS"] == "10:20" and ENV.CUDA_PROFILER_STEPS.value == "10:20"
    with pytest.raises(SystemExit):
        parse_args(["--model", "synthetic:tiny-qwen3", "--profile-steps", "20:10"])
