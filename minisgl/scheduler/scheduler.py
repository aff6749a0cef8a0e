"""The per-rank scheduler loop.

Overlap scheduling (after NanoFlow; python/minisgl/scheduler/scheduler.py:
83-131 in the reference): batch N+1 is prepared on a side stream and
launched on the engine stream before the host processes batch N's sampled
tokens, so host work hides behind GPU work. Token ids never round-trip
through the host between steps: every request's tokens live in the device
token pool, the next step's inputs are gathered from it, and the sampled
ids are scattered back into it.

Batch inputs (positions, request rows, write slots) are built with numpy and
shipped in ONE pinned host buffer / one asynchronous copy per step.
"""

from __future__ import annotations

import os
import time
from typing import TYPE_CHECKING, List, NamedTuple, Optional, Set, Tuple

import numpy as np
import torch

from minisgl.core import Batch, Req
from minisgl.env import ENV
from minisgl.message import AbortBackendMsg, BaseBackendMsg, BatchBackendMsg, DetokenizeMsg, ExitMsg, UserMsg
from minisgl.utils import init_logger

from .cache import CacheManager
from .config import SchedulerConfig
from .decode import DecodeManager
from .io import SchedulerIOMixin
from .prefill import ChunkedReq, PrefillManager
from .table import TableManager

if TYPE_CHECKING:
    from minisgl.engine import BatchSamplingArgs, ForwardOutput

logger = init_logger(__name__)


class ForwardInput(NamedTuple):
    """Everything a launched batch references; kept alive until its results
    are processed so no tensor is freed while the GPU may still read it."""

    batch: Batch
    sample_args: "BatchSamplingArgs"
    input_tuple: Tuple[torch.Tensor, torch.Tensor]   # (rows, positions) to gather token ids
    write_tuple: Tuple[torch.Tensor, torch.Tensor]   # (rows, positions) to store sampled ids


ForwardData = Tuple[ForwardInput, "ForwardOutput"]


class Scheduler(SchedulerIOMixin):
    def __init__(self, config: SchedulerConfig, tokenizer=None) -> None:
        from minisgl.engine import Engine

        self.config = config
        self.engine = Engine(config)
        self.device = self.engine.device
        self.is_cuda = self.engine.is_cuda
        if self.is_cuda:
            self.stream = torch.cuda.Stream(device=self.device)
            self.engine_stream_ctx = torch.cuda.stream(self.engine.stream)
            torch.cuda.set_stream(self.stream)
        page_size = self.engine.page_size
        self.table_manager = TableManager(config.max_running_req, self.engine.page_table)
        self.cache_manager = CacheManager(self.engine.num_pages, page_size, self.engine.page_table, config.cache_type,
                                          page_classes=self.engine.cp_size)
        self.decode_manager = DecodeManager(page_size)
        self.prefill_manager = PrefillManager(self.cache_manager, self.table_manager, self.decode_manager)
        self.finished_reqs: Set[Req] = set()
        if tokenizer is None:
            from minisgl.utils import load_tokenizer

            tokenizer = load_tokenizer(config.model_path)
        self.tokenizer = tokenizer
        self.eos_token_id = getattr(tokenizer, "eos_token_id", None)
        self.token_pool = self.table_manager.token_pool
        self.prefill_budget = config.max_extend_tokens
        self.step_count = 0
        self.h2d_bytes = 0
        self.d2h_bytes = 0
        self._stats_t = time.perf_counter()
        self.profiler = None
        if self.is_cuda and os.environ.get("MINISGL_PROFILE_STEPS", "0") == "1":
            from .profile import StepProfiler

            self.profiler = StepProfiler()
        self.cuda_profiler_window = None
        if self.is_cuda:
            from .profile import CudaProfilerWindow, parse_step_window

            window = parse_step_window(ENV.CUDA_PROFILER_STEPS.value)
            if window is not None:
                self.cuda_profiler_window = CudaProfilerWindow(window)
        super().__init__(config, self.engine.tp_cpu_group)
        # DP attention behind the server: rank 0 still pulls every message and
        # re-publishes it to the other ranks; each rank keeps the requests with
        # uid % ranks == rank, and the replies of each lockstep step (filler
        # steps included, so every rank takes part) are gathered to rank 0,
        # the only rank linked to the detokenizer
        self.dp_online = self.engine.dp and not config.offline_mode
        if self.dp_online:
            self.dp_rank, self.dp_size = config.tp_info.rank, config.tp_info.size
            self._dp_reply_rank0 = self.send_result
            self.send_result = self._dp_gather_reply

    # --------------------------------------------------------------- loops
    def run_when_idle(self) -> None:
        logger.info_rank0("Scheduler is idle, waiting for new requests...")
        self.cache_manager.check_integrity()

    def overlap_loop(self, last_data: Optional[ForwardData]) -> Optional[ForwardData]:
        blocking = last_data is None and not (self.prefill_manager.runnable or self.decode_manager.runnable)
        for msg in self.receive_msg(blocking=blocking):
            self._process_one_msg(msg)
        forward_input = self._schedule_next_batch()
        ongoing = None
        if forward_input is not None:
            with self.engine_stream_ctx:
                self.engine.stream.wait_stream(self.stream)
                ongoing = (forward_input, self._forward(forward_input))
        self._process_last_data(last_data)
        return ongoing

    def normal_loop(self) -> None:
        blocking = not (self.prefill_manager.runnable or self.decode_manager.runnable)
        for msg in self.receive_msg(blocking=blocking):
            self._process_one_msg(msg)
        forward_input = self._schedule_next_batch()
        data = None
        if forward_input is not None:
            data = (forward_input, self._forward(forward_input))
        self._process_last_data(data)

    # DP attention: every rank schedules its own requests, but the MoE
    # layers dispatch tokens between ranks, so all ranks run one forward per
    # step together; a rank with nothing to run does a one-token filler step
    def dp_loop(self) -> None:
        import torch.distributed as dist

        for msg in self.receive_msg(blocking=False):
            self._process_one_msg(msg)
        fin = self._schedule_next_batch()
        busy = fin is not None or self.dp_has_pending() or self.prefill_manager.runnable or \
            self.decode_manager.runnable
        flags = torch.tensor([int(busy), int(fin is not None)], dtype=torch.int64)
        dist.all_reduce(flags, op=dist.ReduceOp.MAX, group=self.tp_cpu_group)
        if int(flags[0]) == 0:
            self.dp_all_idle()
            return
        if fin is None and int(flags[1]) != 0:
            fin = self._prepare_batch(Batch(reqs=[], phase="decode"))
        data = (fin, self._forward(fin)) if fin is not None else None
        self._process_last_data(data)

    def _dp_gather_reply(self, reply: List[DetokenizeMsg]) -> None:
        import torch.distributed as dist

        parts = [None] * self.dp_size if self.dp_rank == 0 else None
        dist.gather_object(reply, parts, dst=0, group=self.tp_cpu_group)
        if self.dp_rank == 0:
            self._dp_reply_rank0([m for part in parts for m in part])

    def dp_has_pending(self) -> bool:
        """Requests this rank has accepted but not scheduled yet (offline mode)."""
        return False

    def dp_all_idle(self) -> None:
        """Every DP rank is idle this step."""
        time.sleep(0.001)

    @torch.inference_mode()
    def run_forever(self):
        if self.engine.dp:
            if self.is_cuda:
                with self.engine_stream_ctx:
                    self.engine.stream.wait_stream(self.stream)
                    while True:
                        self.dp_loop()
            while True:
                self.dp_loop()
        if not self.is_cuda:
            while True:
                self.normal_loop()
        if ENV.DISABLE_OVERLAP_SCHEDULING:
            with self.engine_stream_ctx:
                self.engine.stream.wait_stream(self.stream)
                while True:
                    self.normal_loop()
        data = None
        while True:
            data = self.overlap_loop(data)

    def shutdown(self) -> None:
        if self.is_cuda:
            torch.cuda.synchronize(self.device)
        self.sync_all_ranks()
        self.engine.shutdown()

    # ------------------------------------------------------------ results
    def _process_last_data(self, last: Optional[ForwardData]) -> None:
        if last is None:
            return
        fin, fout = last
        batch = fin.batch
        fout.copy_done_event.synchronize()
        tokens = fout.next_tokens_cpu.tolist()
        self.d2h_bytes += 4 * len(tokens)
        reply: List[DetokenizeMsg] = []
        newly_finished: Set[Req] = set()
        with self.cache_manager.lazy_free_region():
            for i, req in enumerate(batch.reqs):
                if isinstance(req, ChunkedReq):
                    continue
                tok = tokens[i]
                req.append_host(tok)
                done = not req.can_decode
                if not req.sampling_params.ignore_eos and tok == self.eos_token_id:
                    done = True
                reply.append(DetokenizeMsg(uid=req.uid, next_token=tok, finished=done))
                # with overlap a request can finish twice (its next step was already launched)
                if done and req not in self.finished_reqs:
                    self.decode_manager.remove_req(req)
                    self._free_req_resources(req)
                    newly_finished.add(req)
                elif batch.is_prefill and not done:
                    self.cache_manager.cache_req(req, finished=False)
        self.finished_reqs = newly_finished
        self.send_result(reply)

    def _process_one_msg(self, msg: BaseBackendMsg) -> None:
        if isinstance(msg, BatchBackendMsg):
            for m in msg.data:
                self._process_one_msg(m)
        elif isinstance(msg, ExitMsg):
            raise KeyboardInterrupt
        elif isinstance(msg, UserMsg):
            if self.dp_online and msg.uid % self.dp_size != self.dp_rank:
                return  # another DP rank serves this request
            n, cap = len(msg.input_ids), self.engine.max_seq_len
            room = cap - n
            warn = logger.warning if self.dp_online else logger.warning_rank0  # under DP the owner reports
            if room <= 0:
                warn(f"request {msg.uid} dropped: {n} prompt tokens exceed {cap}")
                return
            if msg.sampling_params.max_tokens > room:
                msg.sampling_params.max_tokens = room
                warn(f"request {msg.uid}: max_tokens clamped to {room}")
            self.prefill_manager.add_one_req(msg)
        elif isinstance(msg, AbortBackendMsg):
            req = self.prefill_manager.abort_req(msg.uid) or self.decode_manager.abort_req(msg.uid)
            if req is not None:
                self._free_req_resources(req)
        else:
            raise NotImplementedError(f"unknown message {type(msg)}")

    def _free_req_resources(self, req: Req) -> None:
        self.table_manager.free(req.table_idx)
        self.cache_manager.cache_req(req, finished=True)

    # ------------------------------------------------------------- batches
    def _schedule_next_batch(self) -> Optional[ForwardInput]:
        batch = self.prefill_manager.schedule_next_batch(self.prefill_budget) or \
            self.decode_manager.schedule_next_batch()
        return self._prepare_batch(batch) if batch is not None else None

    def _prepare_batch(self, batch: Batch) -> ForwardInput:
        self.engine.graph_runner.pad_batch(batch)
        self.cache_manager.allocate_paged(batch.reqs)
        padded = batch.padded_reqs
        rows = np.fromiter((r.table_idx for r in padded), np.int32, len(padded))
        if batch.is_decode:
            pos = np.fromiter((r.cached_len for r in padded), np.int32, len(padded))
            in_rows = rows
        else:
            lens = np.fromiter((r.extend_len for r in padded), np.int64, len(padded))
            starts = np.fromiter((r.cached_len for r in padded), np.int64, len(padded))
            offsets = np.cumsum(lens) - lens
            pos = (np.arange(int(lens.sum())) - np.repeat(offsets - starts, lens)).astype(np.int32)
            in_rows = np.repeat(rows, lens)
        reqs = batch.reqs
        w_rows = np.fromiter((r.table_idx for r in reqs), np.int32, len(reqs))
        w_pos = np.fromiter((r.device_len if r.can_decode else -1 for r in reqs), np.int32, len(reqs))
        host = np.concatenate([pos, in_rows, w_rows, w_pos])
        T, B = len(pos), len(reqs)
        buf = torch.from_numpy(host)
        if self.is_cuda:
            buf = buf.pin_memory()
        dev = buf.to(self.device, non_blocking=True)
        self.h2d_bytes += 4 * len(host)
        positions, in_rows_t = dev[:T], dev[T : 2 * T]
        w_rows_t, w_pos_t = dev[2 * T : 2 * T + B], dev[2 * T + B :]
        batch.positions = positions
        batch.out_loc = self.engine.page_table[in_rows_t, positions]
        self.engine.attn_backend.prepare_metadata(batch)
        return ForwardInput(batch, self.engine.sampler.prepare(batch), (in_rows_t, positions), (w_rows_t, w_pos_t))

    def _forward(self, fin: ForwardInput) -> "ForwardOutput":
        batch = fin.batch
        if self.cuda_profiler_window is not None:
            self.cuda_profiler_window.on_step(self.step_count)
        prof = self.profiler.begin() if self.profiler is not None else None
        batch.input_ids = self.token_pool[fin.input_tuple]
        out = self.engine.forward_batch(batch, fin.sample_args)
        if prof is not None:
            self.profiler.end(batch.phase, batch.size, prof)
        self.token_pool[fin.write_tuple] = out.next_tokens_gpu
        self.decode_manager.filter_reqs(batch.reqs)
        self.step_count += 1
        if ENV.DEBUG_CHECK_ERRORS and self.is_cuda:
            from minisgl import ops

            ops.check_device_errors(self.device)
        if ENV.STATS_INTERVAL.value and self.step_count % ENV.STATS_INTERVAL.value == 0:
            self._log_stats(batch)
        return out

    def _log_stats(self, batch: Batch) -> None:
        now = time.perf_counter()
        dt, self._stats_t = now - self._stats_t, now
        used = self.engine.num_pages * self.engine.page_size - self.cache_manager.available_size
        logger.info_rank0(f"step {self.step_count}: {batch.phase} bs={batch.size} "
                          f"running={len(self.decode_manager.running_reqs)} "
                          f"pending={len(self.prefill_manager.pending_list)} kv_used={used} "
                          f"{ENV.STATS_INTERVAL.value / dt:.1f} steps/s")
