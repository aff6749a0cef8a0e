"""Vocab-parallel embedding and LM head.

The vocabulary is split into ceil(V / tp) rows per rank. The embedding
gathers local rows (zero for ids owned by other ranks) and sums across
ranks; the LM head computes local logits for the last token of every
request (fp32 straight out of the GEMM epilogue) and gathers the vocab
shards (python/minisgl/layers/embedding.py:14-110).
"""

from __future__ import annotations

from typing import Dict, Optional

import torch

from minisgl import ops
from minisgl.core import get_global_ctx
from minisgl.parallel import DistributedCommunicator, get_tp_info
from minisgl.utils import div_ceil, nvtx_annotate

from .base import BaseOP


class VocabParallelEmbedding(BaseOP):
    def __init__(self, num_embeddings: int, embedding_dim: int) -> None:
        info = get_tp_info()
        self.tp_size = info.size
        self.num_embeddings = num_embeddings
        self.num_embeddings_tp = div_ceil(num_embeddings, info.size)
        start = self.num_embeddings_tp * info.rank
        stop = min(start + self.num_embeddings_tp, num_embeddings)
        self.vocab_range = (start, stop - start)
        self.weight = torch.empty(self.num_embeddings_tp, embedding_dim)
        self._comm = DistributedCommunicator()

    @nvtx_annotate("Embedding")
    def forward(self, ids: torch.Tensor) -> torch.Tensor:
        y = ops.embedding(ids, self.weight, self.vocab_range if self.tp_size > 1 else None)
        return self._comm.all_reduce(y) if self.tp_size > 1 else y


class ParallelLMHead(VocabParallelEmbedding):
    """``local_logits`` (set by the engine under tensor parallelism on GPUs):
    ``forward`` returns this rank's vocabulary shard of the logits; the
    engine samples from the shards (``ops.sample_sharded``) or, for top-k /
    top-p batches, gathers them with ``gather_logits``."""

    def __init__(self, num_embeddings: int, embedding_dim: int, bias: bool = False, tie_word_embeddings: bool = False,
                 tied_embedding: Optional[VocabParallelEmbedding] = None) -> None:
        super().__init__(num_embeddings, embedding_dim)
        assert (tied_embedding is not None) == tie_word_embeddings
        self.bias = torch.empty(self.num_embeddings_tp) if bias else None
        self._tied = tied_embedding
        self.local_logits = False
        if tied_embedding is not None:
            del self.weight  # the embedding table is the projection

    def named_tensors(self, prefix: str = ""):
        if self._tied is not None:
            return iter(())
        return super().named_tensors(prefix)

    def load_state_dict(self, state_dict: Dict[str, torch.Tensor], *, prefix: str = "", _internal: bool = False) -> None:
        if self._tied is None:
            return super().load_state_dict(state_dict, prefix=prefix, _internal=_internal)
        # tied checkpoints may still carry an lm_head copy: drop it
        state_dict.pop(f"{prefix}.weight", None)
        state_dict.pop(f"{prefix}.bias", None)

    @nvtx_annotate("LMHead")
    def forward(self, x: torch.Tensor) -> torch.Tensor:
        batch = get_global_ctx().batch
        bs = batch.size
        if batch.is_prefill:
            x = x.index_select(0, batch.attn_metadata.get_last_indices(bs))
        w = self._tied.weight if self._tied is not None else self.weight
        fs = get_global_ctx().fused_sample
        if fs is not None and self.tp_size == 1:
            # tokens straight from the GEMM epilogue (no logits in memory)
            return ops.lm_head_sample(x, w, self.bias.to(w.dtype) if self.bias is not None else None,
                                      fs.temperatures, fs.seed, fs.step, out=fs.out)
        logits = ops.gemm(x, w, self.bias.to(w.dtype) if self.bias is not None else None, out_dtype=torch.float32)
        if self.tp_size == 1 or self.local_logits:
            return logits
        return self.gather_logits(logits)

    def gather_logits(self, logits: torch.Tensor) -> torch.Tensor:
        """[rows, V] from every rank's [rows, V_tp] shard."""
        gathered = self._comm.all_gather(logits.contiguous())  # [tp * rows, V_tp]
        rows = logits.shape[0]
        full = gathered.view(self.tp_size, rows, -1).permute(1, 0, 2).reshape(rows, -1)
        return full[:, : self.num_embeddings]
