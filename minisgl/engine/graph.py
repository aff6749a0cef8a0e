"""CUDA-graph capture and replay of decode steps.

One graph per padded batch size (1, 2, 4, then multiples of 8 up to the
maximum), captured largest first into a shared memory pool. A graph reads
its inputs from static buffers (token ids, positions, KV write slots and the
attention metadata) and writes fp32 logits to a static buffer; replay copies
the batch's tensors into those buffers on the engine stream. Batches are
padded with a dummy request whose page-table row points at a spare page.
The batch-size list and its memory-based default follow the reference
(python/minisgl/engine/graph.py:47-64, 152-166).
"""

from __future__ import annotations

import gc
from typing import TYPE_CHECKING, Dict, List, Optional

import torch

from minisgl import ops
from minisgl.core import Batch, FusedSample, Req, get_global_ctx
from minisgl.utils import init_logger

if TYPE_CHECKING:
    from minisgl.attention import BaseAttnBackend
    from minisgl.models import BaseLLMModel

    from .sample import Sampler

logger = init_logger(__name__)


def mem_GB(n: int) -> str:
    return f"{n / (1 << 30):.2f} GiB"


def get_free_memory(device: torch.device) -> int:
    return torch.cuda.mem_get_info(device)[0]


def determine_cuda_graph_bs(bs: Optional[List[int]], max_bs: Optional[int], free_memory: int) -> List[int]:
    if bs is not None:
        return sorted(set(bs))
    if max_bs is None:
        max_bs = 256 if free_memory > (80 << 30) else 160
    if max_bs < 1:
        return []
    return sorted({b for b in [1, 2, 4] + list(range(8, max_bs + 1, 8)) if b <= max_bs} | {max_bs})


class GraphRunner:
    def __init__(self, stream: Optional[torch.cuda.Stream], device: torch.device, model: "BaseLLMModel",
                 attn_backend: "BaseAttnBackend", cuda_graph_bs: Optional[List[int]],
                 cuda_graph_max_bs: Optional[int], free_memory: int, max_seq_len: int, vocab_size: int,
                 dummy_req: Req, sampler: Optional["Sampler"] = None, cpu_group=None) -> None:
        self.stream = stream
        self.sampler = sampler
        self.cpu_group = cpu_group  # tensor-parallel ranks agree on the measured layer forms
        # graphs that sample inside the LM head (greedy / temperature batches)
        self.sample_graph_map: Dict[int, torch.cuda.CUDAGraph] = {}
        self.logits_out: Dict[int, torch.Tensor] = {}
        self.tokens_out: Dict[int, torch.Tensor] = {}
        self.device = device
        self.attn_backend = attn_backend
        self.dummy_req = dummy_req
        self.graph_map: Dict[int, torch.cuda.CUDAGraph] = {}
        self.graph_launches: Dict[int, int] = {}  # native kernels inside each graph
        bs_list = determine_cuda_graph_bs(cuda_graph_bs, cuda_graph_max_bs, free_memory) if device.type == "cuda" else []
        self.graph_bs_list = bs_list
        self.max_graph_bs = max(bs_list) if bs_list else 0
        if self.max_graph_bs > 0:
            self._capture(model, max_seq_len, vocab_size)
        else:
            logger.info_rank0("CUDA graph is disabled.")

    def _capture(self, model: "BaseLLMModel", max_seq_len: int, vocab_size: int) -> None:
        n = self.max_graph_bs
        self.input_ids = torch.zeros(n, dtype=torch.int32, device=self.device)
        self.positions = torch.zeros(n, dtype=torch.int32, device=self.device)
        self.out_loc = torch.zeros(n, dtype=torch.int32, device=self.device)
        self.temps = torch.zeros(n, dtype=torch.float32, device=self.device)
        self.attn_backend.init_capture_graph(max_seq_len, self.graph_bs_list)
        torch.cuda.synchronize(self.device)
        logger.info_rank0(f"Capturing CUDA graphs for batch sizes {self.graph_bs_list}; "
                          f"free memory {mem_GB(get_free_memory(self.device))}")
        ctx = get_global_ctx()
        pool = None
        variants = model.forward_variants() if hasattr(model, "forward_variants") else (None,)
        chosen: Dict[int, object] = {}
        for bs in sorted(self.graph_bs_list, reverse=True):
            batch = Batch(reqs=[self.dummy_req] * bs, phase="decode")
            batch.padded_reqs = batch.reqs
            batch.input_ids = self.input_ids[:bs]
            batch.positions = self.positions[:bs]
            batch.out_loc = self.out_loc[:bs]
            self.attn_backend.prepare_for_capture(batch)
            # capture every layer form the model offers and keep the fastest
            # (every rank captures and replays the same forms the same number
            # of times, so the collectives inside them stay paired)
            captured = []
            for variant in variants:
                if variant is not None:
                    model.set_forward_variant(bs, variant)
                graph = torch.cuda.CUDAGraph()
                with ctx.forward_batch(batch):
                    model.forward()  # warm-up outside the capture
                    before = ops.LAUNCHES[0]
                    with torch.cuda.graph(graph, pool=pool, stream=self.stream):
                        # the graph's own output tensor is the static logits buffer
                        logits = model.forward()
                    launches = ops.LAUNCHES[0] - before
                    ops.LAUNCHES[0] = before
                if pool is None:
                    pool = graph.pool()
                ms = self._time_graph(graph) if len(variants) > 1 else 0.0
                captured.append((ms, variant, graph, logits, launches))
            times = self._slowest_rank([c[0] for c in captured])
            pick = min(range(len(captured)), key=lambda i: times[i])
            _, variant, graph, logits, launches = captured[pick]
            del captured
            if variant is not None:
                model.set_forward_variant(bs, variant)
                chosen[bs] = variant
            self.logits_out[bs] = logits
            self.graph_launches[bs] = launches
            self.graph_map[bs] = graph
            if (self.sampler is not None and getattr(model, "samples_in_lm_head", False)
                    and bs <= self.sampler.FUSED_MAX_ROWS):
                sgraph = torch.cuda.CUDAGraph()
                ctx.fused_sample = FusedSample(self.temps[:bs], self.sampler.seed, self.sampler.step)
                try:
                    with ctx.forward_batch(batch):
                        model.forward()  # warm-up (zero temperatures: greedy, the counter stays)
                        before = ops.LAUNCHES[0]
                        with torch.cuda.graph(sgraph, pool=pool, stream=self.stream):
                            self.tokens_out[bs] = model.forward()
                        self.graph_launches[-bs] = ops.LAUNCHES[0] - before
                        ops.LAUNCHES[0] = before
                finally:
                    ctx.fused_sample = None
                self.sample_graph_map[bs] = sgraph
        torch.cuda.synchronize(self.device)
        if chosen:
            fused = sorted(b for b, v in chosen.items() if v)
            logger.info_rank0(f"Fused-epilogue layers at batch sizes {fused}; plain GEMMs + row kernels at the rest")
        logger.info_rank0(f"CUDA graphs ready; free memory {mem_GB(get_free_memory(self.device))}")

    def _time_graph(self, graph: torch.cuda.CUDAGraph, reps: int = 3) -> float:
        """Device milliseconds of one replay (best of ``reps`` after one warm-up)."""
        graph.replay()
        best = float("inf")
        for _ in range(reps):
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record(self.stream)
            graph.replay()
            e.record(self.stream)
            e.synchronize()
            best = min(best, s.elapsed_time(e))
        return best

    def _slowest_rank(self, times: List[float]) -> List[float]:
        """Per layer form, the slowest tensor-parallel rank's time: every rank
        then picks the same form (graphs of different ranks must run the same
        collectives in the same order)."""
        if self.cpu_group is None or len(times) < 2:
            return times
        import torch.distributed as dist

        t = torch.tensor(times, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX, group=self.cpu_group)
        return t.tolist()

    def can_use_cuda_graph(self, batch: Batch) -> bool:
        return batch.is_decode and max(batch.size, 1) <= self.max_graph_bs

    def pad_batch(self, batch: Batch) -> None:
        size = max(batch.size, 1)  # an empty batch (a DP rank's filler step) runs the dummy request
        if self.can_use_cuda_graph(batch):
            size = next(b for b in self.graph_bs_list if b >= size)
        batch.padded_reqs = batch.reqs + [self.dummy_req] * (size - batch.size)

    def _load_inputs(self, batch: Batch) -> int:
        bs = batch.padded_size
        self.input_ids[:bs].copy_(batch.input_ids)
        self.positions[:bs].copy_(batch.positions)
        self.out_loc[:bs].copy_(batch.out_loc)
        self.attn_backend.prepare_for_replay(batch)
        return bs

    def replay(self, batch: Batch) -> torch.Tensor:
        bs = self._load_inputs(batch)
        self.graph_map[bs].replay()
        ops.LAUNCHES[0] += self.graph_launches[bs]
        return self.logits_out[bs][: batch.size]

    def can_sample(self, batch: Batch) -> bool:
        return batch.padded_size in self.sample_graph_map

    def replay_sample(self, batch: Batch, temperatures: Optional[torch.Tensor]) -> torch.Tensor:
        """Replay the graph that samples in the LM head; padded rows are greedy."""
        bs = self._load_inputs(batch)
        if temperatures is None:
            self.temps[:bs].zero_()
        else:
            self.temps[: batch.size].copy_(temperatures)
            if bs > batch.size:
                self.temps[batch.size : bs].zero_()
        self.sample_graph_map[bs].replay()
        ops.LAUNCHES[0] += self.graph_launches[-bs]
        return self.tokens_out[bs][: batch.size]

    def destroy_cuda_graphs(self) -> None:
        """Release graphs first: graphs holding collectives must go before
        the communicators they captured."""
        self.graph_map.clear()
        self.sample_graph_map.clear()
        self.logits_out.clear()
        self.tokens_out.clear()
        gc.collect()
