"""The per-rank engine: model, KV pool, page table, backends, sampler and
CUDA graphs on one device.

Construction order and memory budgeting follow the reference
(python/minisgl/engine/engine.py:29-189): the model is built on the meta
device and then receives real weights; the KV pool takes
``memory_ratio * free_before_load - model_bytes``; ranks agree on the
minimum free memory. B200 specifics: the KV layout is page-major per head
(TMA friendly), pages must be a power of two of at least 16 tokens, and the
default page is 64 tokens.
"""

from __future__ import annotations

import os
from datetime import timedelta
from typing import Dict, NamedTuple, Optional, Tuple

import torch

from minisgl.env import ENV

from minisgl import ops
from minisgl.attention import create_attention_backend
from minisgl.core import FusedSample, Batch, Context, Req, reset_global_ctx, set_global_ctx
from minisgl.kvcache import create_kvcache_pool
from minisgl.layers import set_rope_device
from minisgl.utils import fault
from minisgl.models import LazyRandomWeights, create_model, load_weight, random_weights
from minisgl.moe import create_moe_backend
from minisgl.parallel import (DistributedCommunicator, destroy_distributed, get_tp_info, reset_cp_info, reset_dp_info,
                              reset_tp_info, set_cp_info, set_dp_info, set_tp_info)
from minisgl.utils import align_ceil, init_logger, torch_dtype

from .config import EngineConfig
from .graph import GraphRunner, get_free_memory, mem_GB
from .sample import BatchSamplingArgs, Sampler

logger = init_logger(__name__)


class ForwardOutput(NamedTuple):
    next_tokens_gpu: torch.Tensor
    next_tokens_cpu: torch.Tensor
    copy_done_event: "torch.cuda.Event | _Done"


class _Done:
    """Stand-in for a CUDA event on the CPU path."""

    def synchronize(self) -> None:
        return None

    def query(self) -> bool:
        return True


def _resolve_device(config: EngineConfig) -> torch.device:
    if config.device == "cpu":
        return torch.device("cpu")
    if config.device.startswith("cuda:"):
        return torch.device(config.device)
    local = int(os.environ.get("MINISGL_DEVICE_OFFSET", "0"))
    return torch.device(f"cuda:{local + config.tp_info.rank}")


def _valid_page(p: int) -> bool:
    return p >= 16 and (p & (p - 1)) == 0


class Engine:
    def __init__(self, config: EngineConfig) -> None:
        if config.cp_size > 1:
            # context parallelism: every rank holds the model (the routed
            # experts split over the ranks with --ep cp) and the attention over
            # the KV tiles it owns; layers see one TP rank
            if config.tp_info.size != config.cp_size:
                raise ValueError("context parallelism runs over all ranks: tp_size must equal cp_size")
            if not config.model_config.is_mla:
                raise ValueError("context parallelism is implemented for MLA models (DeepSeek-V3 / Kimi-K2)")
            if config.ep_size not in (1, config.cp_size):
                raise ValueError("expert parallelism under context parallelism spans every rank: ep_size must be "
                                 "1 or cp_size")
            set_tp_info(0, 1)
            set_cp_info(config.tp_info.rank, config.cp_size)
        elif config.enable_dp_attention and config.tp_info.size > 1:
            # DP attention: replicated layers, experts split and tokens
            # dispatched to them (minisgl/moe/ep_a2a.py)
            if config.cp_size > 1:
                raise ValueError("DP attention and context parallelism are exclusive")
            set_tp_info(0, 1)
            set_dp_info(config.tp_info.rank, config.tp_info.size)
        else:
            if config.ep_size > 1 and config.ep_size != config.tp_info.size:
                raise ValueError("expert parallelism runs over the tensor-parallel ranks: ep_size must equal "
                                 "tp_size (or use --enable-dp-attention)")
            set_tp_info(config.tp_info.rank, config.tp_info.size)
        self.dp = config.enable_dp_attention and config.tp_info.size > 1
        self.config = config
        self.device = _resolve_device(config)
        self.is_cuda = self.device.type == "cuda"
        if self.is_cuda:
            torch.cuda.set_device(self.device)
            self.stream: Optional[torch.cuda.Stream] = torch.cuda.Stream(self.device)
            torch.cuda.set_stream(self.stream)
        else:
            self.stream = None
        torch.manual_seed(42)
        self.dtype = config.dtype
        page_size = config.page_size
        if self.is_cuda and not _valid_page(page_size):
            logger.warning_rank0(f"page size {page_size} is not supported by the sm_100a kernels; using 64")
            page_size = 64
        self.page_size = page_size
        self.ctx = Context(page_size)
        set_global_ctx(self.ctx)

        self.tp_cpu_group = self._init_communication(config)
        init_free = self._sync_get_memory()[1] if self.is_cuda else 0
        if self.is_cuda:
            logger.info_rank0(f"Free memory before loading model: {mem_GB(init_free)}")

        # ------------------------------------------------------------- model
        mcfg = config.model_config
        self.model_config = mcfg
        self.tp_rank = config.tp_info.rank
        self._step = 0  # forwards run so far (the fault-injection clock)
        self._faults = bool(fault.rules())
        set_rope_device(self.device)
        with torch.device("meta"), torch_dtype(config.dtype):
            self.model = create_model(mcfg)
        self.model.load_state_dict(self._load_weights(config))

        # ---------------------------------------------------------- KV cache
        self.num_pages = self._determine_num_pages(init_free, config)
        self.cp_size = config.cp_size if config.cp_size > 1 else 1
        if self.cp_size > 1:
            # context parallelism: page g lives on rank g % cp at local index
            # g // cp, so each rank allocates 1 / cp of the pages
            if page_size != 64:
                raise ValueError("context parallelism needs page size 64 (one page per 64-key tile)")
            self.num_pages -= self.num_pages % self.cp_size
        num_tokens = self.num_pages * page_size
        self.ctx.kv_cache = self.kv_cache = create_kvcache_pool(
            mcfg, self.num_pages + 1, page_size, self.dtype, self.device,
            cp_size=self.cp_size)  # +1: the dummy page
        self.max_seq_len = min(config.max_seq_len, num_tokens)
        width = align_ceil(self.max_seq_len + page_size, max(64, page_size))
        self.ctx.page_table = self.page_table = torch.zeros(
            (config.max_running_req + 1, width), dtype=torch.int32, device=self.device)

        # ---------------------------------------------------------- backends
        self.ctx.attn_backend = self.attn_backend = create_attention_backend(
            config.attention_backend, mcfg, config.max_running_req + 1)
        self._ep_heap = None
        if mcfg.is_moe:
            if self.dp and self.is_cuda and config.comm == "fused":
                from minisgl.parallel.ep_comm import EpHeap

                # pair capacity of one step: the longest forward times k
                cap = max(config.max_forward_len, config.max_running_req) * mcfg.num_experts_per_tok
                self._ep_heap = EpHeap(self.device, cap, mcfg.hidden_size)
            self.ctx.moe_backend = self.moe_backend = create_moe_backend(
                config.moe_backend, ep_dispatch=self.dp, ep_size=mcfg.ep_size, ep_rank=mcfg.ep_rank,
                group=self.tp_cpu_group if not self.is_cuda else None, heap=self._ep_heap,
                context_parallel=self.cp_size > 1 and mcfg.ep_size > 1)
        self.sampler = Sampler(self.device, mcfg.vocab_size, config.weight_seed)
        # tensor parallelism on GPUs: sample from each rank's vocabulary shard
        # of the logits instead of gathering [B, V] fp32 logits every step
        self._lm_head_local = None
        head = getattr(self.model, "lm_head", None)
        if (self.is_cuda and config.tp_info.size > 1 and not self.dp and config.cp_size <= 1
                and head is not None and hasattr(head, "local_logits")):
            head.local_logits = True
            self._lm_head_local = head
        if self.is_cuda:
            from minisgl import ops

            ops.gemm_workspace(self.device)
            ops.error_word(self.device)
            logger.info_rank0(f"Free memory after initialization: {mem_GB(self._sync_get_memory()[0])}")

        if self.is_cuda and config.gemm_autotune:
            self._tune_gemms(config)

        # ------------------------------------------------------ CUDA graphs
        self.dummy_req = Req(input_ids=torch.tensor([0], dtype=torch.int32), table_idx=config.max_running_req,
                             cached_len=0, output_len=1, uid=-1, sampling_params=None,  # type: ignore[arg-type]
                             cache_handle=None)  # type: ignore[arg-type]
        self.page_table[self.dummy_req.table_idx].fill_(num_tokens)  # -> the spare page
        self.graph_runner = GraphRunner(
            self.stream, self.device, self.model, self.attn_backend, config.cuda_graph_bs,
            self._graph_max_bs(config), init_free, width, mcfg.vocab_size, self.dummy_req,
            sampler=None if ENV.NO_FUSED_SAMPLING.value else self.sampler, cpu_group=self.tp_cpu_group)

    # ---------------------------------------------------------------- setup
    def _graph_max_bs(self, config: EngineConfig) -> Optional[int]:
        if not self.is_cuda or (self.dp and config.comm != "fused"):
            return 0  # DP attention over NCCL: the all-to-all needs host-side row counts
        # (the peer-store dispatch of --comm fused has fixed-capacity slots:
        # graphs of different batch sizes on different ranks still match)
        mx = config.cuda_graph_max_bs
        if mx is None:
            return min(config.max_running_req, 256)
        return min(mx, config.max_running_req)

    def _gemm_shapes(self):
        """(N, K) of every dense projection the decode graphs run."""
        from minisgl.layers import BaseOP, OPList, ParallelLMHead
        from minisgl.layers.linear import _Linear

        shapes, stack = set(), [self.model]
        while stack:
            op = stack.pop()
            if isinstance(op, OPList):
                stack.extend(op.op_list)
                continue
            if isinstance(op, _Linear):
                shapes.add(tuple(op.weight.shape))
            elif isinstance(op, ParallelLMHead):
                w = op._tied.weight if op._tied is not None else op.weight
                shapes.add(tuple(w.shape))
            for name, v in vars(op).items():
                if isinstance(v, BaseOP) and not name.startswith("_"):
                    stack.append(v)
        return sorted(shapes)

    def _tune_gemms(self, config: EngineConfig) -> None:
        import time

        from minisgl.ops import gemm_tune

        from .graph import determine_cuda_graph_bs

        bs = determine_cuda_graph_bs(config.cuda_graph_bs, self._graph_max_bs(config), 1 << 40)
        if not bs:
            # no graphs: eager decode batches still get tuned plans (the same
            # ones a graph engine would use, so both compute the same logits)
            bs = list(range(1, min(config.max_running_req, 256) + 1))
        t0 = time.perf_counter()
        cache = os.environ.get("MINISGL_GEMM_TUNE_CACHE") or None
        kinds = self.model.fused_gemm_kinds() if hasattr(self.model, "fused_gemm_kinds") else {}
        plans = gemm_tune.tune(self._gemm_shapes(), bs, self.device, cache, fused=kinds, prefill=True)
        if self.tp_cpu_group is not None:
            # every rank must run the same tile plans: the kernels with the
            # all-reduce fused pair CTA i of one rank with CTA i of the others
            import torch.distributed as dist

            tables = [dict(gemm_tune.PLANS), dict(gemm_tune.FUSED_PLANS)]
            dist.broadcast_object_list(tables, src=0, group=self.tp_cpu_group, device=torch.device("cpu"))
            gemm_tune.PLANS.clear()
            gemm_tune.PLANS.update(tables[0])
            gemm_tune.FUSED_PLANS.clear()
            gemm_tune.FUSED_PLANS.update(tables[1])
        logger.info_rank0(f"Tuned {len(plans)} GEMM plans in {time.perf_counter() - t0:.1f}s")

    def _init_communication(self, config: EngineConfig):
        import torch.distributed as dist

        size = config.tp_info.size
        if size == 1:
            return None
        if not dist.is_initialized():  # otherwise the launcher's group (e.g. torchrun's) is joined
            backend = "cpu:gloo,cuda:nccl" if self.is_cuda else "gloo"
            dist.init_process_group(backend=backend, rank=config.tp_info.rank, world_size=size,
                                    timeout=timedelta(seconds=config.distributed_timeout),
                                    init_method=config.distributed_addr,
                                    device_id=self.device if self.is_cuda else None)
            self._owns_pg = True
        if self.is_cuda and config.comm == "fused" and config.cp_size <= 1:
            from minisgl.parallel.symm import enable_symm_comm

            # one more row per rank: the sequence-parallel form pads token counts to a multiple of the ranks
            rows = config.max_forward_len + size
            enable_symm_comm(self.device, rows * config.model_config.hidden_size * self.dtype.itemsize)
        return dist.group.WORLD

    def _load_weights(self, config: EngineConfig) -> Dict[str, torch.Tensor]:
        if config.use_dummy_weight:
            mcfg = config.model_config
            first = mcfg.ep_rank * (mcfg.num_experts // mcfg.ep_size) if mcfg.ep_size > 1 else 0
            # quantised experts: draw each weight as the model takes it, so the
            # MoE layers quantise one layer's bf16 experts at a time
            draw = LazyRandomWeights if mcfg.moe_quant != "none" else random_weights
            return draw(self.model.state_dict(), self.device, seed=config.weight_seed,
                        gen_device=config.dummy_weight_device, first_expert=first)
        out: Dict[str, torch.Tensor] = {}
        mcfg = config.model_config
        for name, t in load_weight(config.model_path, self.device, ep_size=mcfg.ep_size, ep_rank=mcfg.ep_rank):
            keep_fp32 = t.dtype == torch.float32 and "correction_bias" in name
            out[name] = t if keep_fp32 else t.to(self.dtype)
        return out

    def _determine_num_pages(self, init_free: int, config: EngineConfig) -> int:
        mcfg = config.model_config
        per_page = self._bytes_per_page()
        if config.num_page_override is not None:
            pages = config.num_page_override
        elif self.is_cuda:
            model_bytes = init_free - self._sync_get_memory()[1]
            pages = int(config.memory_ratio * init_free - model_bytes) // per_page
        else:
            pages = (config.max_running_req * min(config.max_seq_len, 4096)) // self.page_size
        if pages <= 1:
            raise RuntimeError("not enough memory for the KV cache; lower --num-pages or the model size")
        logger.info_rank0(f"KV cache: {pages * self.page_size} tokens in {pages} pages of {self.page_size} "
                          f"({mem_GB(pages * per_page)}), model {mcfg.architectures[0]}")
        return pages

    def _bytes_per_page(self) -> int:
        m = self.model_config
        itemsize = self.dtype.itemsize
        if m.is_mla:  # under context parallelism a rank stores one page in cp
            cp = self.config.cp_size if self.config.cp_size > 1 else 1
            return max(1, m.num_layers * self.page_size * (m.kv_lora_rank + m.qk_rope_head_dim) * itemsize // cp)
        from minisgl.utils import div_even

        kv = div_even(m.num_kv_heads, get_tp_info().size, allow_replicate=True)
        return 2 * m.num_layers * kv * self.page_size * m.head_dim * itemsize

    def _sync_get_memory(self) -> Tuple[int, int]:
        """(min, max) free device memory over the TP ranks."""
        torch.cuda.synchronize(self.device)
        torch.cuda.empty_cache()
        free = get_free_memory(self.device)
        if self.tp_cpu_group is None:
            return free, free
        import torch.distributed as dist

        t = torch.tensor([free, -free], dtype=torch.int64)
        dist.all_reduce(t, op=dist.ReduceOp.MIN, group=self.tp_cpu_group)
        lo, hi = int(t[0]), -int(t[1])
        if hi - lo > (2 << 30):
            raise RuntimeError(f"free memory differs across TP ranks: {mem_GB(lo)} vs {mem_GB(hi)}")
        return lo, hi

    # -------------------------------------------------------------- forward
    def forward_batch(self, batch: Batch, args: BatchSamplingArgs) -> ForwardOutput:
        if self._faults:
            fault.at_step(self.tp_rank, self._step)
        self._step += 1
        if ENV.DEBUG_BOUNDS:
            from .bounds import check_kv_bounds

            check_kv_bounds(self.page_table, batch, self.num_pages * self.page_size, self.page_size)
        # greedy / temperature batches sample inside the LM-head GEMM (no
        # logits in memory); top-k / top-p batches sample from the logits
        fused = self.sampler.fusable(args, batch.size) and getattr(self.model, "samples_in_lm_head", False)
        tokens = None
        with self.ctx.forward_batch(batch):
            if self.graph_runner.can_use_cuda_graph(batch):
                if fused and self.graph_runner.can_sample(batch):
                    tokens = self.graph_runner.replay_sample(batch, args.temperatures)
                else:
                    logits = self.graph_runner.replay(batch)
            elif fused:
                self.ctx.fused_sample = FusedSample(args.temperatures, self.sampler.seed, self.sampler.step)
                try:
                    tokens = self.model.forward()
                finally:
                    self.ctx.fused_sample = None
            else:
                logits = self.model.forward()
        for r in batch.reqs:
            r.complete_one()
        if tokens is not None:
            next_gpu = tokens[: batch.size]
        elif self._lm_head_local is not None:
            next_gpu = self._sample_shards(logits[: batch.size], args)
        else:
            next_gpu = self.sampler.sample(logits[: batch.size], args)
        if not self.is_cuda:
            return ForwardOutput(next_gpu, next_gpu, _Done())
        next_cpu = torch.empty(next_gpu.shape, dtype=next_gpu.dtype, pin_memory=True)
        next_cpu.copy_(next_gpu, non_blocking=True)
        event = torch.cuda.Event()
        event.record(self.stream)
        return ForwardOutput(next_gpu, next_cpu, event)

    def _sample_shards(self, logits: torch.Tensor, args: BatchSamplingArgs) -> torch.Tensor:
        """Tokens from this rank's vocabulary shard of the logits: greedy and
        temperature batches sample from the shards (only per-chunk winners
        cross the ranks); top-k / top-p batches gather the whole rows first."""
        head = self._lm_head_local
        if args.top_k is None and args.top_p is None:
            lo, n = head.vocab_range
            return ops.sample_sharded(logits[:, :n], args.temperatures, self.sampler.seed, self.sampler.step, lo,
                                      DistributedCommunicator.plugins[-1])
        return self.sampler.sample(head.gather_logits(logits), args)

    def shutdown(self) -> None:
        self.graph_runner.destroy_cuda_graphs()
        import torch.distributed as dist

        if getattr(self, "_ep_heap", None) is not None:
            self._ep_heap.shutdown()
            self._ep_heap = None
        destroy_distributed()
        if getattr(self, "_owns_pg", False) and dist.is_initialized():
            dist.destroy_process_group()
        reset_global_ctx()
        reset_tp_info()
        reset_cp_info()
        reset_dp_info()
