"""L2 eviction between timed launches.

``L2Flush()`` writes a buffer larger than L2 (126 MB on B200), then reads a
second one: the write evicts everything a previous launch left in L2, and the
read replaces the write's dirty lines with clean ones, so the dirty-line
write-back of the flush itself is not charged to the launch timed next.
Both run outside the timed events.
"""
from __future__ import annotations

import torch

FLUSH_BYTES = 256 << 20


class L2Flush:
    def __init__(self, device, nbytes: int = FLUSH_BYTES):
        n = nbytes // 4
        self.wbuf = torch.empty(n, dtype=torch.float32, device=device)
        self.rbuf = torch.ones(n, dtype=torch.float32, device=device)
        self.sink = torch.empty((), dtype=torch.float32, device=device)

    def __call__(self) -> None:
        self.wbuf.fill_(1.0)
        torch.sum(self.rbuf, dim=0, out=self.sink)
