"""Request rows of the page table and of the on-device token pool."""

from __future__ import annotations

import torch


class TableManager:
    def __init__(self, max_running_reqs: int, page_table: torch.Tensor) -> None:
        self._free = list(range(max_running_reqs))
        self.page_table = page_table
        # every token a request has (prompt + sampled) lives here on the device;
        # zero-filled so padded dummy rows read a valid token id
        self.token_pool = torch.zeros_like(page_table, dtype=torch.int32)

    @property
    def available_size(self) -> int:
        return len(self._free)

    def allocate(self) -> int:
        return self._free.pop()

    def free(self, row: int) -> None:
        self._free.append(row)
