"""Token sampling: greedy, temperature, top-k, top-p (nucleus), per request.

Greedy rows use the argmax kernel; stochastic rows draw with the exponential
(Gumbel-max) trick over the filtered distribution, using a per-request
generator when the request has a seed.  The reference only has greedy
argmax (its CUDA argmax kernel is undefined, ``tensor_ops_cuda.cu:786``).
"""
from __future__ import annotations

from typing import Dict, List

import torch


def filter_logits(logits: torch.Tensor, temperature: torch.Tensor, top_k: torch.Tensor,
                  top_p: torch.Tensor) -> torch.Tensor:
    """logits [B, V] fp32 -> logits with filtered entries at -inf (temperature applied)."""
    x = logits / temperature.clamp(min=1e-5)[:, None]
    V = x.shape[-1]
    sorted_x, idx = torch.sort(x, dim=-1, descending=True)
    ranks = torch.arange(V, device=x.device)[None, :]
    k = torch.where(top_k > 0, top_k, torch.full_like(top_k, V))
    drop = ranks >= k[:, None]
    probs = torch.softmax(sorted_x, dim=-1)
    cum = probs.cumsum(-1) - probs          # mass strictly before each entry
    drop |= cum > top_p[:, None]
    sorted_x = sorted_x.masked_fill(drop, float("-inf"))
    return torch.empty_like(x).scatter_(-1, idx, sorted_x)


class Sampler:
    def __init__(self):
        self.gens: Dict[int, torch.Generator] = {}

    def __call__(self, logits: torch.Tensor, seqs: List) -> torch.Tensor:
        B = logits.shape[0]
        dev = logits.device
        lf = logits.float()
        out = lf.argmax(-1)
        temp = torch.tensor([max(s.params.temperature, 0.0) for s in seqs[:B]], device=dev)
        stoch = temp > 0
        if bool(stoch.any()):
            rows = stoch.nonzero().flatten()
            tk = torch.tensor([seqs[i].params.top_k for i in rows.tolist()], device=dev)
            tp = torch.tensor([seqs[i].params.top_p for i in rows.tolist()], device=dev, dtype=torch.float32)
            filt = filter_logits(lf[rows], temp[rows], tk, tp)
            probs = torch.softmax(filt, -1)
            noise = torch.empty_like(probs)
            for j, i in enumerate(rows.tolist()):
                s = seqs[i]
                g = None
                if s.params.seed is not None:
                    g = self.gens.get(s.req_id)
                    if g is None:
                        g = torch.Generator(device=dev)
                        g.manual_seed(s.params.seed)
                        self.gens[s.req_id] = g
                noise[j].exponential_(generator=g)
            out[rows] = (probs / noise).argmax(-1)
        return out
