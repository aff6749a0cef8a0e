"""Scheduler message I/O.

Rank 0 pulls requests from the tokenizer. With several TP ranks it
re-publishes the raw bytes to the other ranks over ZMQ PUB/SUB and
broadcasts the message count over the CPU process group, so every rank
consumes exactly the same messages in the same step; only rank 0 replies to
the detokenizer (protocol of python/minisgl/scheduler/io.py:15-133).
Offline mode (the ``LLM`` class) replaces both directions with in-process
hooks.
"""

from __future__ import annotations

from typing import TYPE_CHECKING, List

import torch

from minisgl.message import BaseBackendMsg, BaseTokenizerMsg, BatchTokenizerMsg, DetokenizeMsg
from minisgl.env import ENV
from minisgl.utils import ZmqPubQueue, ZmqPullQueue, ZmqPushQueue, ZmqSubQueue, fault, init_logger

if TYPE_CHECKING:
    from .config import SchedulerConfig

logger = init_logger(__name__)


class MessageLostError(RuntimeError):
    """A rank did not receive a request message that rank 0 counted for it."""


class SchedulerIOMixin:
    def __init__(self, config: "SchedulerConfig", tp_cpu_group) -> None:
        info = config.tp_info
        self.tp_cpu_group = tp_cpu_group
        if config.offline_mode:
            self.receive_msg = self.offline_receive_msg
            self.send_result = self.offline_send_result
            return
        if info.is_primary():
            self._recv_from_tokenizer = ZmqPullQueue(config.zmq_backend_addr, create=True,
                                                     decoder=BaseBackendMsg.decoder)
            self._send_into_tokenizer = ZmqPushQueue(config.zmq_detokenizer_addr,
                                                     create=config.backend_create_detokenizer_link,
                                                     encoder=BaseTokenizerMsg.encoder)
        recv, send = self._recv_single, self._reply_rank0
        self._published = 0  # request messages rank 0 re-published so far
        self._drop_faults = bool(fault.rules())
        if info.size > 1:
            if info.is_primary():
                self._send_into_ranks = ZmqPubQueue(config.zmq_scheduler_broadcast_addr, create=True,
                                                    encoder=BaseBackendMsg.encoder)
                recv = self._recv_multi_rank0
            else:
                self._recv_from_rank0 = ZmqSubQueue(config.zmq_scheduler_broadcast_addr, create=False,
                                                    decoder=BaseBackendMsg.decoder)
                recv, send = self._recv_multi_other, self._reply_other
        self.receive_msg = recv
        self.send_result = send

    # hooks provided by the scheduler / LLM
    def run_when_idle(self) -> None:
        raise NotImplementedError

    def offline_receive_msg(self, blocking: bool = False) -> List[BaseBackendMsg]:
        raise NotImplementedError

    def offline_send_result(self, reply: List[DetokenizeMsg]) -> None:
        raise NotImplementedError

    def sync_all_ranks(self) -> None:
        if self.tp_cpu_group is not None:
            import torch.distributed as dist

            dist.barrier(group=self.tp_cpu_group)

    # ------------------------------------------------------------- receive
    def _recv_single(self, blocking: bool = False) -> List[BaseBackendMsg]:
        msgs: List[BaseBackendMsg] = []
        if blocking:
            self.run_when_idle()
            msgs.append(self._recv_from_tokenizer.get())
        while not self._recv_from_tokenizer.empty():
            msgs.append(self._recv_from_tokenizer.get())
        return msgs

    def _recv_multi_rank0(self, blocking: bool = False) -> List[BaseBackendMsg]:
        import torch.distributed as dist

        msgs: List[BaseBackendMsg] = []
        if blocking:
            self.run_when_idle()
            raw = self._recv_from_tokenizer.get_raw()
            self._send_into_ranks.put_raw(raw)
            msgs.append(self._recv_from_tokenizer.decode(raw))
        raws: List[bytes] = []
        while not self._recv_from_tokenizer.empty():
            raws.append(self._recv_from_tokenizer.get_raw())
        count = torch.tensor(len(raws))
        dist.broadcast(count, src=0, group=self.tp_cpu_group)
        for raw in raws:
            if not (self._drop_faults and fault.drops_broadcast(0, self._published)):
                self._send_into_ranks.put_raw(raw)
            self._published += 1
            msgs.append(self._recv_from_tokenizer.decode(raw))
        return msgs

    def _recv_multi_other(self, blocking: bool = False) -> List[BaseBackendMsg]:
        import torch.distributed as dist

        msgs: List[BaseBackendMsg] = []
        if blocking:
            self.run_when_idle()
            msgs.append(self._recv_from_rank0.get())
        count = torch.tensor(-1)
        dist.broadcast(count, src=0, group=self.tp_cpu_group)
        # rank 0 publishes these right after the count broadcast; the poll budget
        # covers that delay, and a bounded wait turns a lost message into an
        # error instead of a rank that waits forever
        budget_ms = int(ENV.BROADCAST_TIMEOUT_S.value * 1000)
        for i in range(int(count)):
            if not self._recv_from_rank0.poll(budget_ms):
                raise MessageLostError(f"rank {dist.get_rank(self.tp_cpu_group)}: request message {i + 1} of "
                                       f"{int(count)} from rank 0 did not arrive within "
                                       f"{ENV.BROADCAST_TIMEOUT_S.value} s")
            msgs.append(self._recv_from_rank0.get())
        return msgs

    # --------------------------------------------------------------- reply
    def _reply_rank0(self, reply: List[DetokenizeMsg]) -> None:
        if len(reply) == 1:
            self._send_into_tokenizer.put(reply[0])
        elif reply:
            self._send_into_tokenizer.put(BatchTokenizerMsg(data=list(reply)))

    def _reply_other(self, reply: List[DetokenizeMsg]) -> None:
        return None
