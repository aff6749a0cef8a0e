"""Message serialisation round trips and the detokeniser."""

import msgpack
import torch

from minisgl.core import SamplingParams
from minisgl.message import (
    AbortBackendMsg, BaseBackendMsg, BaseFrontendMsg, BaseTokenizerMsg, BatchBackendMsg, BatchFrontendMsg,
    DetokenizeMsg, ExitMsg, TokenizeMsg, UserMsg, UserReply,
)


def _rt(msg, base):
    return base.decoder(msgpack.unpackb(msgpack.packb(base.encoder(msg), use_bin_type=True), raw=False))


def test_backend_roundtrip():
    m = BatchBackendMsg([UserMsg(3, torch.arange(7, dtype=torch.int32), SamplingParams(0.7, 5, 0.9, True, 33)),
                         AbortBackendMsg(4), ExitMsg()])
    back = _rt(m, BaseBackendMsg)
    assert isinstance(back, BatchBackendMsg)
    u = back.data[0]
    assert u.uid == 3 and torch.equal(u.input_ids, torch.arange(7, dtype=torch.int32))
    assert u.sampling_params == SamplingParams(0.7, 5, 0.9, True, 33)
    assert isinstance(back.data[1], AbortBackendMsg) and isinstance(back.data[2], ExitMsg)


def test_tokenizer_and_frontend_roundtrip():
    m = TokenizeMsg(1, [{"role": "user", "content": "hi"}], SamplingParams())
    assert _rt(m, BaseTokenizerMsg) == m
    d = DetokenizeMsg(2, 17, True)
    assert _rt(d, BaseTokenizerMsg) == d
    f = BatchFrontendMsg([UserReply(1, "abc", False), UserReply(2, "", True)])
    assert _rt(f, BaseFrontendMsg) == f


def test_detokenizer_streams_full_text():
    from minisgl.tokenizer.detokenize import DetokenizeManager
    from minisgl.utils import load_tokenizer
    from minisgl.utils.synthetic import make_model_dir

    tok = load_tokenizer(make_model_dir("tiny-qwen3"))
    mgr = DetokenizeManager(tok)
    ids = [10, 11, 12, 13]
    pieces = []
    for i, x in enumerate(ids):
        pieces += mgr.detokenize([DetokenizeMsg(uid=7, next_token=x, finished=i == len(ids) - 1)])
    assert "".join(pieces) == tok.decode(ids)
    assert 7 not in mgr.decode_map
