"""Prompt -> token ids (chat messages go through the tokenizer's template)."""

from __future__ import annotations

from typing import List

import torch

from minisgl.message import TokenizeMsg


class TokenizeManager:
    def __init__(self, tokenizer) -> None:
        self.tokenizer = tokenizer

    def tokenize(self, msgs: List[TokenizeMsg]) -> List[torch.Tensor]:
        out = []
        for m in msgs:
            text = m.text
            if isinstance(text, list):
                text = self.tokenizer.apply_chat_template(text, tokenize=False, add_generation_prompt=True)
            ids = self.tokenizer.encode(text)
            out.append(torch.tensor(ids, dtype=torch.int32))
        return out
