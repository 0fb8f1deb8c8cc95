"""The running set of the generic ``LLM.generate`` path
(aios/scheduler/decode.py:1-36): every live request decodes one token per step."""

from __future__ import annotations

from dataclasses import dataclass, field
from typing import Iterable, Set

from ..core import Batch, Req


@dataclass
class DecodeManager:
    page_size: int
    running_reqs: Set[Req] = field(default_factory=set)

    def filter_reqs(self, reqs: Iterable[Req]) -> None:
        """Adds `reqs` to the running set and keeps only those that can decode."""
        self.running_reqs = {req for req in self.running_reqs.union(reqs) if req.can_decode}

    def remove_req(self, req: Req) -> None:
        self.running_reqs.discard(req)

    @property
    def inflight_tokens(self) -> int:
        """KV tokens the running set may still claim (pages rounded up)."""
        return sum(req.remain_len for req in self.running_reqs) + (self.page_size - 1) * len(self.running_reqs)

    def schedule_next_batch(self) -> Batch | None:
        return Batch(reqs=list(self.running_reqs), phase="decode") if self.running_reqs else None

    @property
    def runnable(self) -> bool:
        return bool(self.running_reqs)
