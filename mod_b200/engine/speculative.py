"""Speculative decoding with n-gram (prompt-lookup) drafts, greedy verification.

The reference ships a prefix-match kernel and an ``ngram_speculate`` argument
that nothing calls (``src/inference_pio/plugins/cuda/c_src/tensor_ops_cuda.cu:496-505``,
``src/inference_pio/models/qwen3_coder_next/model.py:143``).  Here the pieces
are wired together:

1. draft: for each running sequence, find the most recent earlier occurrence
   of its last n tokens (n = ``ngram_max`` down to ``ngram_min``) and propose
   the (up to) ``k`` tokens that followed it;
2. verify: one forward pass over [last token, drafts...] per sequence on top
   of the cached context (the prefill path with a cached prefix), logits at
   every position, greedy target tokens;
3. accept: the longest prefix where draft == target (the verify-tokens
   kernel), plus the target token after it; KV entries written for rejected
   drafts are simply overwritten later (the sequence's cached length only
   advances over accepted positions).

The emitted tokens are exactly those of greedy decoding; a step emits between
1 and k + 1 tokens per sequence.  Models with recurrent (DeltaNet) layers are
rejected: their state cannot be rolled back past a rejected draft.
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import List, Optional, Sequence as Seq

import numpy as np
import torch

from .batch import ForwardBatch
from .sequence import SamplingParams, Sequence


def ngram_propose(tokens: List[int], k: int, ngram_max: int = 3, ngram_min: int = 1) -> List[int]:
    """Up to ``k`` tokens that followed the latest earlier match of the sequence's last n tokens."""
    L = len(tokens)
    for n in range(min(ngram_max, L - 1), ngram_min - 1, -1):
        tail = tokens[L - n:]
        for start in range(L - n - 1, -1, -1):  # most recent earlier occurrence first
            if tokens[start:start + n] == tail:
                nxt = tokens[start + n:start + n + k]
                if nxt:
                    return nxt
    return []


@dataclass
class SpecStats:
    steps: int = 0
    drafted: int = 0
    accepted: int = 0
    emitted: int = 0
    per_step: List[int] = field(default_factory=list)

    @property
    def acceptance(self) -> float:
        return self.accepted / self.drafted if self.drafted else 0.0


class NgramSpeculativeDecoder:
    """Greedy speculative generation on top of an ``LLMEngine`` (single process)."""

    def __init__(self, engine, k: int = 4, ngram_max: int = 3, ngram_min: int = 1):
        if engine.runner.states is not None:
            raise ValueError("speculative decoding needs attention-only models (recurrent state cannot roll back)")
        if getattr(engine, "expert_parallel", False) or getattr(engine, "tensor_parallel", False):
            raise ValueError("speculative decoding runs in a single process")
        self.eng, self.k, self.nmax, self.nmin = engine, k, ngram_max, ngram_min
        self.stats = SpecStats()

    # ------------------------------------------------------------------ verify forward
    def _verify(self, seqs: List[Sequence], drafts: List[List[int]]) -> List[List[int]]:
        r = self.eng.runner
        bs = r.blocks.block_size
        ids, pos, slots, ctx, qlens = [], [], [], [], []
        bt = np.zeros((len(seqs), r.max_blocks), dtype=np.int32)
        for i, (s, d) in enumerate(zip(seqs, drafts)):
            start = s.length - 1                     # the last emitted token is not cached yet
            toks = [s.last_token] + d
            p = np.arange(start, start + len(toks), dtype=np.int64)
            blk = np.asarray(s.blocks, dtype=np.int64)
            ids.append(np.asarray(toks, dtype=np.int64))
            pos.append(p)
            slots.append(blk[p // bs] * bs + p % bs)
            ctx.append(start + len(toks))
            qlens.append(len(toks))
            bt[i, :len(s.blocks)] = s.blocks
        dev = r.device
        T = int(sum(qlens))

        def up(x, dtype):
            return torch.as_tensor(np.concatenate(x) if isinstance(x, list) and isinstance(x[0], np.ndarray)
                                   else np.asarray(x)).to(dtype).to(dev)

        fb = ForwardBatch(input_ids=up(ids, torch.long), positions=up(pos, torch.int32),
                          slot_mapping=up(slots, torch.int32), block_tables=torch.from_numpy(bt).to(dev),
                          ctx_lens=up(ctx, torch.int32), logits_idx=torch.arange(T, device=dev),
                          state_slots=up([s.state_slot for s in seqs], torch.long), is_decode=False,
                          query_lens=qlens, ctx_lens_host=ctx)
        h = r.model.forward(fb, r.kv, r.states)
        tgt = r.model.sample_greedy(h).to("cpu").tolist()
        out, o = [], 0
        for ql in qlens:
            out.append(tgt[o:o + ql])
            o += ql
        return out

    def _accept_len(self, drafts: List[List[int]], targets: List[List[int]]) -> List[int]:
        """Matched-prefix length per sequence (verify-tokens kernel on the engine's device)."""
        K = max((len(d) for d in drafts), default=0)
        if K == 0:
            return [0] * len(drafts)
        dr = torch.full((len(drafts), K), -1, dtype=torch.long)   # the kernel takes int64 token ids
        tg = torch.full((len(drafts), K), -2, dtype=torch.long)
        for i, (d, t) in enumerate(zip(drafts, targets)):
            dr[i, :len(d)] = torch.tensor(d, dtype=torch.long)
            tg[i, :len(d)] = torch.tensor(t[:len(d)], dtype=torch.long)
        be = self.eng.backend
        if getattr(be, "N", None) is not None and self.eng.device.type == "cuda":
            n = be.N.verify_tokens(dr.to(self.eng.device), tg.to(self.eng.device))
        else:
            from ..ops import reference as R

            n = R.verify_tokens(dr, tg)
        return [min(int(x), len(d)) for x, d in zip(n.to("cpu").tolist(), drafts)]

    # ------------------------------------------------------------------ one speculative step
    def step(self, seqs: List[Sequence]) -> List[Sequence]:
        eng = self.eng
        drafts = []
        for s in seqs:
            room = min(self.k, s.params.max_new_tokens - len(s.output) - 1,
                       eng.runner.max_blocks * eng.blocks.block_size - s.length - 1)
            d = ngram_propose(s.all_tokens, max(0, room), self.nmax, self.nmin) if room > 0 else []
            if d and not eng.blocks.allocate(s, s.length + len(d)):
                d = []
            if not eng.blocks.allocate(s, s.length):
                raise RuntimeError("KV cache exhausted during speculative decoding")
            drafts.append(d)
        targets = self._verify(seqs, drafts)
        acc = self._accept_len(drafts, targets)
        done = []
        self.stats.steps += 1
        for s, d, t, a in zip(seqs, drafts, targets, acc):
            new = t[:a + 1]                          # accepted drafts (== targets) + the bonus target
            s.num_cached = s.length - 1 + a + 1      # KV valid for the last token and the accepted drafts
            self.stats.drafted += len(d)
            self.stats.accepted += a
            emitted = 0
            for tok in new:
                s.output.append(int(tok))
                emitted += 1
                if s.finished_by(int(tok)):
                    eng.scheduler.finish(s)
                    done.append(s)
                    break
            self.stats.emitted += emitted
            self.stats.per_step.append(emitted)
        return done

    def generate(self, prompts: Seq[Seq[int]], max_new_tokens: int = 64) -> List[List[int]]:
        eng = self.eng
        params = SamplingParams(max_new_tokens=max_new_tokens)
        ids = [eng.add_request(list(p), params) for p in prompts]
        # prefill (and any decode the scheduler interleaves) through the normal engine step
        while eng.scheduler.waiting or any(not s.output for s in eng.scheduler.running):
            eng.step()
        while eng.scheduler.running:
            self.step(list(eng.scheduler.running))
        return [eng.seqs.pop(i).output for i in ids]
