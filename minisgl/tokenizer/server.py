"""Tokenizer / detokenizer worker process.

Pulls batches of messages, detokenises sampled tokens for the frontend,
tokenises new prompts for the scheduler and forwards aborts
(python/minisgl/tokenizer/server.py:30-110 in the reference).
"""

from __future__ import annotations

from typing import List, Optional

from minisgl.message import (
    AbortBackendMsg,
    AbortMsg,
    BaseBackendMsg,
    BaseFrontendMsg,
    BaseTokenizerMsg,
    BatchBackendMsg,
    BatchFrontendMsg,
    BatchTokenizerMsg,
    DetokenizeMsg,
    TokenizeMsg,
    UserMsg,
    UserReply,
)
from minisgl.utils import ZmqPullQueue, ZmqPushQueue, init_logger, load_tokenizer


def _flatten(msg: BaseTokenizerMsg) -> List[BaseTokenizerMsg]:
    return list(msg.data) if isinstance(msg, BatchTokenizerMsg) else [msg]


def _one_or_batch(items, batch_cls):
    return items[0] if len(items) == 1 else batch_cls(data=items)


def tokenize_worker(*, tokenizer_path: str, addr: str, create: bool, backend_addr: str, frontend_addr: str,
                    local_bs: int, tokenizer_id: int = -1, ack_queue=None, model_source: str = "huggingface",
                    max_iterations: Optional[int] = None) -> None:
    import torch

    torch.set_grad_enabled(False)
    from .detokenize import DetokenizeManager
    from .tokenize import TokenizeManager

    send_backend = ZmqPushQueue(backend_addr, create=False, encoder=BaseBackendMsg.encoder)
    send_frontend = ZmqPushQueue(frontend_addr, create=False, encoder=BaseFrontendMsg.encoder)
    recv = ZmqPullQueue(addr, create=create, decoder=BatchTokenizerMsg.decoder)
    tokenizer = load_tokenizer(tokenizer_path)
    logger = init_logger(__name__, f"tokenizer_{tokenizer_id}")
    tok_mgr, detok_mgr = TokenizeManager(tokenizer), DetokenizeManager(tokenizer)
    if ack_queue is not None:
        ack_queue.put(f"Tokenize server {tokenizer_id} is ready")
    it = 0
    try:
        while max_iterations is None or it < max_iterations:
            it += 1
            pending = _flatten(recv.get())
            while len(pending) < local_bs and not recv.empty():
                pending.extend(_flatten(recv.get()))
            detok = [m for m in pending if isinstance(m, DetokenizeMsg)]
            tok = [m for m in pending if isinstance(m, TokenizeMsg)]
            abort = [m for m in pending if isinstance(m, AbortMsg)]
            logger.debug(f"{len(detok)} detokenize, {len(tok)} tokenize, {len(abort)} abort")
            if detok:
                texts = detok_mgr.detokenize(detok)
                replies = [UserReply(uid=m.uid, incremental_output=t, finished=m.finished) for m, t in zip(detok, texts)]
                send_frontend.put(_one_or_batch(replies, BatchFrontendMsg))
            if tok:
                ids = tok_mgr.tokenize(tok)
                reqs = [UserMsg(uid=m.uid, input_ids=t, sampling_params=m.sampling_params) for m, t in zip(tok, ids)]
                send_backend.put(_one_or_batch(reqs, BatchBackendMsg))
            if abort:
                send_backend.put(_one_or_batch([AbortBackendMsg(uid=m.uid) for m in abort], BatchBackendMsg))
    except KeyboardInterrupt:
        pass
