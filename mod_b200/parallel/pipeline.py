"""Pipeline parallelism: layer stages on different ranks, activations passed
point-to-point, micro-batched.

``PipelineStage`` owns a contiguous run of layers (any callables
``x -> x``); ``PipelineExecutor.forward`` splits the batch into
micro-batches, and for each one receives the activation from the previous
stage (``torch.distributed.recv``), runs its layers and sends the result on;
the last stage returns the outputs.  In a single process the stages simply
run in sequence.  The reference's pipeline is a sequential single-process
stage runner without micro-batching (``pio/core/parallelism/pipeline.py:12-61``).
"""
from __future__ import annotations

from typing import Callable, List, Optional, Sequence

import torch
import torch.distributed as dist


class PipelineStage:
    def __init__(self, layers: Sequence[Callable[[torch.Tensor], torch.Tensor]], rank: int):
        self.layers = list(layers)
        self.rank = rank

    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        for f in self.layers:
            x = f(x)
        return x


def split_layers(layers: Sequence, n_stages: int) -> List[List]:
    """Contiguous, as-even-as-possible split of ``layers`` into ``n_stages`` runs."""
    n = len(layers)
    out, start = [], 0
    for s in range(n_stages):
        k = n // n_stages + (1 if s < n % n_stages else 0)
        out.append(list(layers[start:start + k]))
        start += k
    return out


class PipelineExecutor:
    def __init__(self, stages: List[PipelineStage], micro_batches: int = 1, group=None):
        self.stages = stages
        self.micro = micro_batches
        self.group = group
        self.dist = dist.is_available() and dist.is_initialized() and dist.get_world_size(group) > 1

    def forward(self, x: Optional[torch.Tensor], shape=None, dtype=torch.float32) -> Optional[torch.Tensor]:
        if not self.dist:
            for st in self.stages:
                x = st(x)
            return x
        rank = dist.get_rank(self.group)
        world = dist.get_world_size(self.group)
        me = self.stages[rank]
        outs = []
        chunks = x.chunk(self.micro) if rank == 0 else [None] * self.micro
        for i in range(self.micro):
            if rank == 0:
                h = chunks[i].contiguous()
            else:
                mshape = list(shape)
                mshape[0] = shape[0] // self.micro
                h = torch.empty(mshape, dtype=dtype)
                dist.recv(h, src=rank - 1, group=self.group)
            h = me(h)
            if rank < world - 1:
                dist.send(h.contiguous(), dst=rank + 1, group=self.group)
            else:
                outs.append(h)
        return torch.cat(outs) if outs else None
