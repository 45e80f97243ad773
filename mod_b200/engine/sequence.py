"""Requests and sampling parameters.

Mirrors the reference's request lifecycle in ``BatchManager``
(``pio/common/managers/batch_manager.py:9-84``: add_request / step / status,
FAILED on exception) but for a continuous batcher.
"""
from __future__ import annotations

import enum
import itertools
import time
from dataclasses import dataclass, field
from typing import List, Optional, Tuple


class SeqStatus(enum.Enum):
    WAITING = "waiting"
    RUNNING = "running"
    FINISHED = "finished"
    FAILED = "failed"
    ABORTED = "aborted"


@dataclass
class SamplingParams:
    max_new_tokens: int = 16
    temperature: float = 0.0          # 0 -> greedy
    top_p: float = 1.0
    top_k: int = 0
    eos_token_id: Optional[int] = None
    ignore_eos: bool = False
    seed: Optional[int] = None
    stop_token_ids: Tuple[int, ...] = ()  # generation ends after emitting any of these (kept in the output)


_ids = itertools.count()


@dataclass
class Sequence:
    prompt: List[int]
    params: SamplingParams = field(default_factory=SamplingParams)
    req_id: int = field(default_factory=lambda: next(_ids))
    output: List[int] = field(default_factory=list)
    status: SeqStatus = SeqStatus.WAITING
    blocks: List[int] = field(default_factory=list)
    state_slot: int = -1
    num_cached: int = 0               # tokens whose KV is in the cache
    error: Optional[str] = None
    t_arrival: float = field(default_factory=time.perf_counter)
    t_first_token: Optional[float] = None
    t_finish: Optional[float] = None
    images: Optional[object] = None   # pixel tensor for vision-language prompts
    callback: Optional[object] = None  # streaming: callback(seq, token)
    swapped: bool = False             # preempted with its KV saved to host memory (resumes without recompute)

    @property
    def all_tokens(self) -> List[int]:
        return self.prompt + self.output

    @property
    def length(self) -> int:
        return len(self.prompt) + len(self.output)

    @property
    def last_token(self) -> int:
        return self.output[-1] if self.output else self.prompt[-1]

    def finished_by(self, token: int) -> bool:
        p = self.params
        if not p.ignore_eos and p.eos_token_id is not None and token == p.eos_token_id:
            return True
        if p.stop_token_ids and token in p.stop_token_ids:
            return True
        return len(self.output) >= p.max_new_tokens

    @property
    def ttft(self) -> Optional[float]:
        return None if self.t_first_token is None else self.t_first_token - self.t_arrival
