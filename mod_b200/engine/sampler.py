"""Token sampling: greedy, temperature, top-k, top-p (nucleus), per request.

On CUDA with the native extension every row goes through one fused kernel
(``sample_tokens``: thresholds for top-k / top-p found without a sort, then a
Gumbel-max draw whose noise hashes (seed, step, token id), so a seeded request
replays exactly).  Elsewhere stochastic rows use the sort-based filter below
and exponential (Gumbel-max) noise from a per-request generator.  The reference only has greedy
argmax (its CUDA argmax kernel is undefined, ``tensor_ops_cuda.cu:786``).
"""
from __future__ import annotations

from typing import Dict, List, Optional

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
    def __init__(self, native: Optional[bool] = None):
        self.gens: Dict[int, torch.Generator] = {}
        self.native = native
        self._base_seed = int(torch.randint(0, 2**62, (1,)).item())

    def _use_native(self, logits) -> bool:
        if self.native is False or not logits.is_cuda:
            return False
        try:
            from ..ops import load_extension

            load_extension()
            return True
        except Exception:
            if self.native:
                raise
            return False

    def __call__(self, logits: torch.Tensor, seqs: List) -> torch.Tensor:
        B = logits.shape[0]
        dev = logits.device
        if self._use_native(logits):
            from ..ops import native as N

            ps = [s.params for s in seqs[:B]]
            temp = torch.tensor([max(p.temperature, 0.0) for p in ps], dtype=torch.float32)
            tk = torch.tensor([p.top_k for p in ps], dtype=torch.int32)
            tp = torch.tensor([p.top_p for p in ps], dtype=torch.float32)
            seeds = torch.tensor([p.seed if p.seed is not None else (self._base_seed + s.req_id) % 2**62
                                  for p, s in zip(ps, seqs)], dtype=torch.int64)
            steps = torch.tensor([len(s.output) for s in seqs[:B]], dtype=torch.int64)
            host = torch.stack([temp, tp]).pin_memory() if torch.cuda.is_available() else torch.stack([temp, tp])
            dev_f = host.to(dev, non_blocking=True)
            meta = torch.stack([seeds, steps, tk.long()]).to(dev, non_blocking=True)
            return N.sample_tokens(logits, dev_f[0], meta[2].int(), dev_f[1], meta[0], meta[1])
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
