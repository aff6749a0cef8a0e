"""Command-line flags -> ``ServerArgs``.

Every flag of the reference (python/minisgl/server/args.py:54-268) is kept
with the same names, aliases and defaults. Added: ``--ep-size/--ep``,
``--cp-size/--cp``, ``--enable-dp-attention``, ``--moe-quant``,
``--random-init`` (alias of ``--dummy-weight``: seeded N(0, 0.02) weights),
``--comm {fused,nccl}`` (default fused; ``--disable-pynccl`` selects nccl)
and ``--device``. ``--model synthetic:<shape>``
serves a synthetic model folder (see ``minisgl.utils.synthetic``).
"""

from __future__ import annotations

import argparse
import os
from dataclasses import dataclass
from typing import List, Tuple

import torch

from minisgl.parallel import DistributedInfo
from minisgl.scheduler import SchedulerConfig
from minisgl.utils import init_logger


@dataclass(frozen=True)
class ServerArgs(SchedulerConfig):
    server_host: str = "127.0.0.1"
    server_port: int = 1919
    num_tokenizer: int = 0
    silent_output: bool = False

    @property
    def share_tokenizer(self) -> bool:
        return self.num_tokenizer == 0

    @property
    def zmq_frontend_addr(self) -> str:
        return self.ipc_endpoint("frontend")

    @property
    def zmq_tokenizer_addr(self) -> str:
        if self.share_tokenizer:
            return self.zmq_detokenizer_addr
        return self.ipc_endpoint("tokenizer")

    @property
    def tokenizer_create_addr(self) -> bool:
        return self.share_tokenizer

    @property
    def backend_create_detokenizer_link(self) -> bool:
        return not self.share_tokenizer

    @property
    def frontend_create_tokenizer_link(self) -> bool:
        return not self.share_tokenizer

    @property
    def distributed_addr(self) -> str:
        return f"tcp://127.0.0.1:{self.server_port + 1}"


_DTYPES = {"float16": torch.float16, "bfloat16": torch.bfloat16, "float32": torch.float32}


def build_parser() -> argparse.ArgumentParser:
    from minisgl.attention import validate_attn_backend
    from minisgl.kvcache import SUPPORTED_CACHE_MANAGER
    from minisgl.moe import SUPPORTED_MOE_BACKENDS

    p = argparse.ArgumentParser(description="minisgl server (B200-native)")
    p.add_argument("--model-path", "--model", type=str, required=True,
                   help="HF folder or hub id, or synthetic:<shape> for a random-weight model of a named shape")
    p.add_argument("--dtype", type=str, default="auto", choices=["auto"] + list(_DTYPES))
    p.add_argument("--tensor-parallel-size", "--tp-size", type=int, default=1)
    p.add_argument("--expert-parallel-size", "--ep-size", dest="ep_size", type=int, default=1)
    p.add_argument("--context-parallel-size", "--cp-size", dest="cp_size", type=int, default=1)
    p.add_argument("--enable-dp-attention", action="store_true")
    p.add_argument("--moe-quant", choices=["none", "mxfp4", "mxfp4-a8"], default="none",
                   help="routed experts: bf16, MXFP4 weights with bf16 activations, or MXFP4 weights x MXFP8 "
                        "activations on the block-scaled tensor cores")
    p.add_argument("--comm", choices=["nccl", "fused"], default="fused",
                   help="TP collectives: in-kernel NVLink collectives (default) or NCCL (baseline); "
                        "ignored on --device cpu")
    p.add_argument("--device", default="cuda", help="cuda (one GPU per TP rank) or cpu (fp32 reference path)")
    p.add_argument("--max-running-requests", type=int, dest="max_running_req", default=ServerArgs.max_running_req)
    p.add_argument("--max-seq-len-override", type=int, default=ServerArgs.max_seq_len_override)
    p.add_argument("--memory-ratio", type=float, default=ServerArgs.memory_ratio)
    p.add_argument("--dummy-weight", "--random-init", action="store_true", dest="use_dummy_weight")
    p.add_argument("--disable-pynccl", action="store_false", dest="use_pynccl")
    p.add_argument("--host", type=str, dest="server_host", default=ServerArgs.server_host)
    p.add_argument("--port", type=int, dest="server_port", default=ServerArgs.server_port)
    p.add_argument("--cuda-graph-max-bs", "--graph", type=int, default=ServerArgs.cuda_graph_max_bs)
    p.add_argument("--num-tokenizer", "--tokenizer-count", type=int, default=ServerArgs.num_tokenizer)
    p.add_argument("--max-prefill-length", "--max-extend-length", type=int, dest="max_extend_tokens",
                   default=ServerArgs.max_extend_tokens)
    p.add_argument("--num-pages", type=int, dest="num_page_override", default=ServerArgs.num_page_override)
    p.add_argument("--page-size", type=int, default=ServerArgs.page_size)
    p.add_argument("--attention-backend", "--attn", type=validate_attn_backend, default=ServerArgs.attention_backend)
    p.add_argument("--model-source", type=str, default="huggingface", choices=["huggingface", "modelscope"])
    p.add_argument("--cache-type", type=str, default=ServerArgs.cache_type,
                   choices=SUPPORTED_CACHE_MANAGER.supported_names())
    p.add_argument("--moe-backend", default=ServerArgs.moe_backend,
                   choices=["auto"] + SUPPORTED_MOE_BACKENDS.supported_names())
    p.add_argument("--shell-mode", action="store_true")
    p.add_argument("--profile-steps", default=None, metavar="A:B",
                   help="bracket scheduler steps A..B-1 with cudaProfilerStart / Stop (for nsys "
                        "--capture-range=cudaProfilerApi or ncu --profile-from-start off); sets "
                        "MINISGL_CUDA_PROFILER_STEPS for the scheduler processes")
    return p


def parse_args(args: List[str], run_shell: bool = False) -> Tuple[ServerArgs, bool]:
    kw = vars(build_parser().parse_args(args)).copy()
    run_shell |= kw.pop("shell_mode")
    window = kw.pop("profile_steps")
    if window is not None:
        from minisgl.env import ENV
        from minisgl.scheduler.profile import parse_step_window

        try:
            parse_step_window(window)
        except ValueError as e:
            raise SystemExit(f"--profile-steps: {e}") from e
        # the scheduler processes read it when they start (spawned with this environment)
        os.environ["MINISGL_CUDA_PROFILER_STEPS"] = window
        ENV.CUDA_PROFILER_STEPS.value = window
    if run_shell:
        kw.update(cuda_graph_max_bs=1, max_running_req=1, silent_output=True)
    path: str = kw["model_path"]
    if path.startswith("synthetic:"):
        from minisgl.utils.synthetic import make_model_dir

        kw["model_path"] = make_model_dir(path.split(":", 1)[1])
        kw["use_dummy_weight"] = True
    elif path.startswith("~"):
        kw["model_path"] = os.path.expanduser(path)
    source = kw.pop("model_source")
    if source == "modelscope" and not os.path.isdir(kw["model_path"]):
        try:
            from modelscope import snapshot_download  # type: ignore
        except ImportError as e:
            raise SystemExit("--model-source modelscope needs the modelscope package") from e
        ignore = ["*.bin", "*.safetensors", "*.pt", "*.ckpt"] if kw["use_dummy_weight"] else []
        kw["model_path"] = snapshot_download(kw["model_path"], ignore_patterns=ignore)
    dtype = kw["dtype"]
    if dtype == "auto":
        from minisgl.utils import cached_load_hf_config

        cfg = cached_load_hf_config(kw["model_path"])
        dtype = getattr(cfg, "dtype", None) or getattr(cfg, "torch_dtype", None) or "bfloat16"
        if kw["device"] == "cpu":
            dtype = "float32"
    kw["dtype"] = _DTYPES[dtype] if isinstance(dtype, str) else dtype
    if kw["dtype"] == torch.float32 and kw["device"] != "cpu":
        kw["dtype"] = torch.bfloat16  # the GPU kernels run bf16
    if not kw["use_pynccl"]:
        # the reference's switch from its own NCCL kernels to torch.distributed:
        # here, from the in-kernel NVLink collectives to the NCCL baseline
        kw["comm"] = "nccl"
    ranks = kw.pop("tensor_parallel_size")
    if kw.get("cp_size", 1) > 1:
        # context parallelism spans every rank (KV split by 64-key tiles,
        # prefill tokens sharded, experts split with --ep cp)
        if ranks not in (1, kw["cp_size"]):
            raise SystemExit("--cp-size runs over all ranks: leave --tp at 1 or set it equal to --cp-size")
        ranks = kw["cp_size"]
    kw["tp_info"] = DistributedInfo(0, ranks)
    result = ServerArgs(**kw)
    init_logger(__name__).info(f"Parsed arguments:\n{result}")
    return result, run_shell


def default_args(model_path: str, **overrides) -> ServerArgs:
    """Build ServerArgs programmatically (tests, embedding in other apps)."""
    return ServerArgs(model_path=model_path, tp_info=overrides.pop("tp_info", DistributedInfo(0, 1)),
                      dtype=overrides.pop("dtype", torch.bfloat16), **overrides)


__all__ = ["ServerArgs", "parse_args", "build_parser", "default_args"]
