"""Per-step device metadata handed to the model.

One flat token dimension T covers every sequence in the step.  Decode steps
have one token per sequence (T == B); prefill steps carry each sequence's new
tokens back to back, with ``query_lens`` giving the split on the host.
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import List, Optional

import torch


@dataclass
class ForwardBatch:
    input_ids: torch.Tensor            # [T] int64
    positions: torch.Tensor            # [T] int32
    slot_mapping: torch.Tensor         # [T] int32, paged-KV slot of each token (-1: none)
    block_tables: torch.Tensor         # [B, max_blocks] int32
    ctx_lens: torch.Tensor             # [B] int32, tokens in cache after this step
    logits_idx: torch.Tensor           # [B] int64, rows of the hidden state that produce logits
    state_slots: torch.Tensor          # [B] int64, recurrent-state slot of each sequence
    is_decode: bool = True
    query_lens: List[int] = field(default_factory=list)   # prefill only (host)
    ctx_lens_host: List[int] = field(default_factory=list)
    attn_splits: int = 1
    inputs_embeds: Optional[torch.Tensor] = None          # [T, H] (vision tokens merged in)

    @property
    def num_seqs(self) -> int:
        return self.block_tables.shape[0]
