"""Hugging Face config / tokenizer / weight-folder helpers.

Local folders are used as they are. Hub ids are resolved through
``huggingface_hub`` (or ModelScope when selected); with no network access a
hub id fails with a clear message.
"""

from __future__ import annotations

import functools
import json
import os
from typing import Any


def load_tokenizer(model_path: str):
    from transformers import AutoTokenizer

    try:
        tok = AutoTokenizer.from_pretrained(model_path)
    except (ValueError, AttributeError, KeyError):
        # an unknown model type in config.json: the fast tokenizer file alone
        from transformers import PreTrainedTokenizerFast

        tok = PreTrainedTokenizerFast.from_pretrained(model_path)
    if not getattr(tok, "chat_template", None):
        # some checkpoints (e.g. Mistral) keep the template in its own file
        path = os.path.join(model_path, "chat_template.json")
        if not os.path.isfile(path):
            try:
                from huggingface_hub import hf_hub_download

                path = hf_hub_download(repo_id=model_path, filename="chat_template.json")
            except Exception:
                path = ""
        if path and os.path.isfile(path):
            with open(path, encoding="utf-8") as f:
                tok.chat_template = json.load(f)["chat_template"]
    return tok


@functools.lru_cache(maxsize=None)
def _load_config(model_path: str) -> Any:
    from transformers import AutoConfig

    try:
        return AutoConfig.from_pretrained(model_path)
    except ValueError:
        # model types transformers ships no class for (e.g. kimi_k2, whose
        # checkpoints rely on remote code): the fields of config.json as is
        path = os.path.join(model_path, "config.json")
        if not os.path.isfile(path):
            raise
        with open(path, encoding="utf-8") as f:
            return PlainConfig(**json.load(f))


class PlainConfig:
    """config.json fields as attributes (for model types without a
    transformers config class)."""

    def __init__(self, **fields: Any) -> None:
        self.__dict__.update(fields)

    def to_dict(self) -> dict:
        return dict(self.__dict__)


def cached_load_hf_config(model_path: str):
    """A fresh copy of the (cached) HF config, so callers may mutate it."""
    cfg = _load_config(model_path)
    return type(cfg)(**cfg.to_dict())


def download_hf_weight(model_path: str) -> str:
    if os.path.isdir(model_path):
        return model_path
    try:
        from huggingface_hub import snapshot_download

        return snapshot_download(model_path, allow_patterns=["*.safetensors"])
    except Exception as e:
        raise ValueError(f"model path {model_path!r} is neither a local folder nor a reachable hub id: {e}") from e
