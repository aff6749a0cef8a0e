"""Offline batch generation API: ``LLM(model).generate(prompts, params)``.

An in-process scheduler (offline mode): prompts are tokenized lazily, up to
one prefill budget per scheduler step, and generation runs until every
request finished (behaviour of python/minisgl/llm/llm.py).
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Dict, List, Sequence, Tuple, Union

import torch

from minisgl.core import SamplingParams
from minisgl.message import BaseBackendMsg, DetokenizeMsg, UserMsg
from minisgl.parallel import DistributedInfo
from minisgl.scheduler import Scheduler, SchedulerConfig

Prompt = Union[str, List[int]]


class RequestAllFinished(Exception):
    pass


@dataclass
class RequestStatus:
    uid: int
    input_ids: List[int]
    output_ids: List[int]


class LLM(Scheduler):
    def __init__(self, model_path: str, dtype: torch.dtype = torch.bfloat16, tokenizer=None, **kwargs) -> None:
        tp_info = kwargs.pop("tp_info", DistributedInfo(0, 1))
        config = SchedulerConfig(model_path=model_path, tp_info=tp_info, dtype=dtype, offline_mode=True, **kwargs)
        super().__init__(config, tokenizer=tokenizer)
        self.pending_requests: List[Tuple[Prompt, SamplingParams]] = []
        self.status_map: Dict[int, RequestStatus] = {}
        self.counter = 0

    def _tokenize(self, prompt: Prompt) -> torch.Tensor:
        if isinstance(prompt, str):
            return torch.tensor(self.tokenizer.encode(prompt), dtype=torch.int32)
        return torch.tensor(prompt, dtype=torch.int32)

    def offline_receive_msg(self, blocking: bool = False) -> List[BaseBackendMsg]:
        if blocking and not self.pending_requests:
            raise RequestAllFinished()
        out: List[BaseBackendMsg] = []
        taken, budget = 0, 0
        for prompt, params in self.pending_requests:
            if budget >= self.prefill_budget:
                break
            ids = self._tokenize(prompt)
            budget += len(ids)
            uid = self.counter + taken
            taken += 1
            out.append(UserMsg(uid=uid, input_ids=ids, sampling_params=params))
            self.status_map[uid] = RequestStatus(uid, ids.tolist(), [])
        self.counter += taken
        self.pending_requests = self.pending_requests[taken:]
        return out

    def offline_send_result(self, reply: List[DetokenizeMsg]) -> None:
        for msg in reply:
            st = self.status_map[msg.uid]
            if not (msg.finished and msg.next_token == self.eos_token_id):
                st.output_ids.append(msg.next_token)

    def run_when_idle(self) -> None:
        self.cache_manager.check_integrity()

    def dp_has_pending(self) -> bool:
        return bool(self.pending_requests)

    def dp_all_idle(self) -> None:
        raise RequestAllFinished()

    def generate(self, prompts: Sequence[Prompt],
                 sampling_params: Union[SamplingParams, Sequence[SamplingParams]]) -> List[Dict[str, object]]:
        self.pending_requests, self.status_map, self.counter = [], {}, 0
        if isinstance(sampling_params, SamplingParams):
            sampling_params = [sampling_params] * len(prompts)
        jobs = list(enumerate(zip(prompts, sampling_params)))
        dp = self.engine.dp
        if dp:  # DP attention: rank r serves prompts r, r + R, ...; results are gathered at the end
            rank, world = self.config.tp_info.rank, self.config.tp_info.size
            jobs = jobs[rank::world]
        self.pending_requests = [(p, SamplingParams(**vars(sp))) for _, (p, sp) in jobs]
        try:
            self.run_forever()
        except RequestAllFinished:
            pass
        mine = {}
        for local, (i, _) in enumerate(jobs):
            ids = self.status_map[local].output_ids
            text = self.tokenizer.decode(ids) if hasattr(self.tokenizer, "decode") else ""
            mine[i] = {"text": text, "token_ids": ids}
        if dp:
            import torch.distributed as dist

            parts = [None] * self.config.tp_info.size
            dist.all_gather_object(parts, mine, group=self.tp_cpu_group)
            for part in parts:
                mine.update(part)
        return [mine[i] for i in range(len(prompts))]
