"""Incremental detokenisation for streaming.

Per request we keep the ids decoded so far and two offsets: ``surr`` (start
of a short context window re-decoded every step, so merges across token
boundaries come out right) and ``read`` (ids already folded into the output
string). Text is released only when it is stable: not ending in U+FFFD (a
partial UTF-8 sequence), and, while a word may still grow, only up to the
last space / newline / CJK character. This is the SGLang-style incremental
decoder the reference uses (python/minisgl/tokenizer/detokenize.py), with
the printable-text heuristic of Hugging Face's TextStreamer.
"""

from __future__ import annotations

from dataclasses import dataclass, field
from typing import Dict, List

from minisgl.message import DetokenizeMsg

_CJK = ((0x4E00, 0x9FFF), (0x3400, 0x4DBF), (0x20000, 0x2A6DF), (0x2A700, 0x2B73F), (0x2B740, 0x2B81F),
        (0x2B820, 0x2CEAF), (0xF900, 0xFAFF), (0x2F800, 0x2FA1F))


def _is_cjk(ch: str) -> bool:
    cp = ord(ch)
    return any(lo <= cp <= hi for lo, hi in _CJK)


def find_printable_text(text: str) -> str:
    if text.endswith("\n"):
        return text
    if text and _is_cjk(text[-1]):
        return text
    if len(text) > 1 and _is_cjk(text[-2]):
        return text[:-1]
    return text[: text.rfind(" ") + 1]


@dataclass
class DecodeStatus:
    decoded_ids: List[int] = field(default_factory=list)
    decoded_str: str = ""
    read_offset: int = 0
    surr_offset: int = 0
    sent_offset: int = 0


class DetokenizeManager:
    def __init__(self, tokenizer) -> None:
        self.tokenizer = tokenizer
        self.eos_token_id = getattr(tokenizer, "eos_token_id", None)
        self.decode_map: Dict[int, DecodeStatus] = {}

    def detokenize(self, msgs: List[DetokenizeMsg]) -> List[str]:
        windows, contexts = [], []
        for m in msgs:
            st = self.decode_map.setdefault(m.uid, DecodeStatus())
            if not (m.finished and m.next_token == self.eos_token_id):
                st.decoded_ids.append(m.next_token)
            windows.append(st.decoded_ids[st.surr_offset :])
            contexts.append(st.decoded_ids[st.surr_offset : st.read_offset])
        win_txt = self.tokenizer.batch_decode(windows)
        ctx_txt = self.tokenizer.batch_decode(contexts)
        out: List[str] = []
        for m, full, prefix in zip(msgs, win_txt, ctx_txt):
            st = self.decode_map[m.uid]
            new = full[len(prefix) :]
            if new and not new.endswith("�"):
                st.decoded_str += new
                text = st.decoded_str
                st.surr_offset, st.read_offset = st.read_offset, len(st.decoded_ids)
            else:
                text = st.decoded_str + find_printable_text(new)
            out.append(text[st.sent_offset :])
            st.sent_offset = len(text)
            if m.finished:
                del self.decode_map[m.uid]
        return out
