"""Host-side KV bounds check (MINISGL_DEBUG_BOUNDS=1).

Before a forward, every KV slot the batch will touch is checked against the
pool: the slots it writes (``out_loc``) and the page-table entries each
request's attention reads (positions below its ``device_len``). A bad entry
raises ``KVBoundsError`` on the host instead of letting a kernel read or
write outside the pool. The check reads device tensors back, so it
synchronizes; it is a debugging switch, off by default.
"""

from __future__ import annotations

import torch


class KVBoundsError(RuntimeError):
    """A batch would read or write a KV slot outside the pool."""


def check_kv_bounds(page_table: torch.Tensor, batch, num_slots: int, spare_slots: int = 0) -> None:
    """`num_slots`: slots of the pages requests may own. `spare_slots`: the
    spare page after them, which padding entries (CUDA-graph padding, a DP
    rank's filler step) write and nothing reads."""
    loc = getattr(batch, "out_loc", None)
    if loc is not None and loc.numel():
        lo, hi = int(loc.min()), int(loc.max())
        if lo < 0 or hi >= num_slots + spare_slots:
            raise KVBoundsError(f"{batch.phase} batch writes KV slots [{lo}, {hi}] outside the pool of "
                                f"{num_slots} + {spare_slots} spare")
    for req in batch.reqs:
        n = req.device_len
        if not 0 <= req.table_idx < page_table.shape[0] or n > page_table.shape[1]:
            raise KVBoundsError(f"request {req.uid}: table row {req.table_idx} / length {n} outside the page "
                                f"table {tuple(page_table.shape)}")
        if n == 0:
            continue
        row = page_table[req.table_idx, :n]
        lo, hi = int(row.min()), int(row.max())
        if lo < 0 or hi >= num_slots:
            bad = int(((row < 0) | (row >= num_slots)).nonzero()[0])
            raise KVBoundsError(f"request {req.uid}: page-table row {req.table_idx} maps position {bad} to slot "
                                f"{int(row[bad])}, outside the pool of {num_slots}")
