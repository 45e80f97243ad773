"""LLMEngine: the public serving API.

    eng = LLMEngine.from_preset("qwen3-30b-a3b", backend="native")
    outs = eng.generate([[1, 2, 3]], SamplingParams(max_new_tokens=32))

``add_request`` / ``step`` / ``has_unfinished`` give the incremental form a
serving loop or the streaming front-end uses; ``generate`` drives them to
completion.  The reference's per-plugin ``generate_text`` /
``BatchManager.add_request/step`` (``pio/models/qwen3_0_6b/plugin.py:139-152``,
``pio/common/managers/batch_manager.py:9-84``) map onto this.
"""
from __future__ import annotations

import logging
import os
import time
from typing import Dict, List, Optional, Sequence as Seq, Union

import torch

from ..config.models import ModelConfig
from ..config.presets import get_preset
from ..models.backend import make_backend
from ..models.decoder import DecoderLM
from ..models.weights import ModelWeights, random_weights
from .block_manager import BlockManager, PrefixCachingBlockManager
from .kv_cache import KVCache, StateCache
from .runner import ModelRunner
from .scheduler import Scheduler
from .sequence import SamplingParams, Sequence, SeqStatus
from ..utils import tracing

log = logging.getLogger("mod_b200.engine")


class LLMEngine:
    def __init__(self, cfg: ModelConfig, weights: Optional[ModelWeights] = None, backend: str = "native",
                 device: Union[str, torch.device] = "cuda", max_batch: int = 128, max_model_len: int = 4096,
                 num_blocks: Optional[int] = None, kv_mem_fraction: float = 0.85, use_graphs: Optional[bool] = None,
                 max_prefill_tokens: int = 16384, seed: int = 0, model=None, kv_heads: Optional[int] = None,
                 expert_parallel: Optional[bool] = None, tensor_parallel: bool = False,
                 quantization: Optional[str] = None, prefix_caching: bool = False,
                 prefill_chunk: Optional[int] = None, kv_swap: bool = True, kv_swap_bytes: int = 8 << 30,
                 offload_layers: Union[int, str, None] = None, model_path: Optional[str] = None,
                 tp_comm: Optional[str] = None):
        """``expert_parallel`` (default: on when a process group of >1 ranks
        exists and the model is MoE): every rank serves its own requests with a
        replicated attention stack and holds E/world experts; MoE layers
        exchange tokens with the fused NVLink dispatch/combine (native backend)
        or NCCL all-to-all (torch backend).  ``quantization="int8"`` stores the
        projection matrices as int8 with per-channel scales (int8 weight-only
        GEMMs); expert weights stay bf16 under expert parallelism.
        ``use_graphs`` (default: on for the native backend, off for the torch
        baseline): capture each padded decode batch size in a CUDA graph.
        ``kv_swap``: a sequence preempted for KV space keeps its KV in pinned
        host memory (up to ``kv_swap_bytes``) and resumes without recomputing.
        ``offload_layers`` (hybrid CPU/GPU execution): the last N decoder layers
        live in pinned host memory and are streamed to the device one layer
        ahead of use (``runtime.offload.LayerStreamer``); ``model_path``: an HF
        safetensors checkpoint (file or directory) read through the mmap
        reader, each rank taking only its part (its TP slices or its EP
        experts); ``"auto"`` takes N
        from the placement planner for this device's memory.  Streaming runs
        eagerly (no decode graphs).  ``tp_comm`` (tensor parallelism, native
        backend): the layer-boundary flavour, ``"p2p"`` (peer stores),
        ``"nvls"`` (NVSwitch multimem reduce + multicast stores) or ``"auto"``
        (the default: NVLS where every rank's device has NVLink multicast, else
        P2P); the ``MB_TP_COMM`` environment variable sets the default."""
        import torch.distributed as dist

        self.cfg = cfg
        self.device = torch.device(device)
        from ..runtime.memory import UnifiedMemoryManager

        # one owner of this rank's device memory: it records the free memory before any weight exists
        # and sizes the KV pool from what the weights, buffers and workspace leave
        self.memory = UnifiedMemoryManager(self.device)
        world = dist.get_world_size() if dist.is_available() and dist.is_initialized() else 1
        rank = dist.get_rank() if world > 1 else 0
        if expert_parallel is None:
            expert_parallel = world > 1 and cfg.is_moe
        self.expert_parallel = expert_parallel
        self.backend = make_backend(backend)
        # the C++ CPU backend computes in fp32; the GPU backends in bf16
        wdt = torch.float32 if backend == "cpu" else torch.bfloat16
        self.tensor_parallel = tensor_parallel and world > 1
        if self.tensor_parallel and model is None:
            if quantization not in (None, "none"):
                raise ValueError("tensor parallelism runs bf16 weights (int8 weight-only is single-GPU / EP)")
            from ..models.tp_decoder import TPDecoderLM, shard_weights
            from ..parallel.tp import make_tp_comm

            # hybrid (DeltaNet) or MoE models: heads split, experts expert-parallel over the same ranks
            hybrid = cfg.is_moe or any(cfg.layer_type(i) == "linear_attention"
                                       for i in range(cfg.num_hidden_layers))
            er = None  # MoE: only this rank's experts are read or made
            if cfg.is_moe:
                El = cfg.num_experts // world
                er = (rank * El, (rank + 1) * El)
            if model_path is not None and weights is None and not hybrid:
                from ..io.hf_loader import load_hf

                shard = load_hf(cfg, model_path, device=self.device, dtype=wdt, tp=(rank, world))
            else:
                if weights is None and model_path is not None:
                    # hybrid / MoE checkpoint: this rank's experts, then the dense parts sliced by heads
                    from ..io.hf_loader import load_hf

                    weights = load_hf(cfg, model_path, device=self.device, dtype=wdt, expert_range=er)
                elif weights is None:
                    weights = random_weights(cfg, device=self.device, dtype=wdt, seed=seed, expert_range=er)
                if hybrid:
                    from ..models.tp_hybrid import shard_hybrid_weights

                    shard = shard_hybrid_weights(cfg, weights, rank, world)
                else:
                    shard = shard_weights(cfg, weights, rank, world)
            weights = None
            mt = max(max_batch, max_prefill_tokens)
            # boundary flavour: P2P peer stores (default), NVLS multimem, or the NCCL baseline
            kind = tp_comm or os.environ.get("MB_TP_COMM", "auto")
            comm = make_tp_comm(kind if backend == "native" else "nccl", cfg.hidden_size, mt)
            if hybrid:
                from ..models.tp_hybrid import TPHybridLM
                from ..parallel.ep import FusedEPMoE, NcclEPMoE
                from ..parallel.tp import padded_tokens

                tp_moe = None
                if cfg.is_moe:  # the tokens a rank owns (its sequence-parallel rows) go through the exchange
                    rows = padded_tokens(max_batch, world) // world
                    tp_moe = (FusedEPMoE(cfg, self.backend, max_tokens=rows,
                                         prefill_tokens=max(rows, min(2048, padded_tokens(mt, world) // world)))
                              if backend == "native" else NcclEPMoE(cfg, self.backend, max_tokens=rows))
                model = TPHybridLM(cfg, shard, self.backend, comm, world, moe_impl=tp_moe)
            else:
                model = TPDecoderLM(cfg, shard, self.backend, comm, world)
            kv_heads = model.Hkv
            expert_parallel = False
            self.expert_parallel = False  # experts of a TP model are exchanged inside its MoE layers
        moe_impl = None
        if expert_parallel:
            El = cfg.num_experts // world
            if weights is None and model is None:
                if model_path is not None:
                    from ..io.hf_loader import load_hf

                    weights = load_hf(cfg, model_path, device=self.device, dtype=wdt,
                                      expert_range=(rank * El, (rank + 1) * El))
                else:
                    weights = random_weights(cfg, device=self.device, dtype=wdt, seed=seed,
                                             expert_range=(rank * El, (rank + 1) * El))
            from ..parallel.ep import FusedEPMoE, NcclEPMoE

            moe_impl = (FusedEPMoE(cfg, self.backend, max_tokens=max_batch,
                                   prefill_tokens=max(max_batch, min(2048, max_prefill_tokens)))
                        if backend == "native" else NcclEPMoE(cfg, self.backend, max_tokens=max_batch))
            if backend == "native" and os.environ.get("MB_EP_COMM", "p2p") == "agrs":
                # decode steps as NVLS all-gather -> local experts -> in-switch reduce (opt-in);
                # prefill and uncovered blocks keep the point-to-point exchange
                from ..parallel.ep_agrs import AgRsEPMoE
                from ..parallel.symm import nvls_supported

                if nvls_supported():
                    moe_impl = AgRsEPMoE(cfg, self.backend, max_tokens=max_batch, fallback=moe_impl)
        elif (backend == "native" and cfg.is_moe and world == 1 and model is None and self.device.type == "cuda"
              and quantization in (None, "none") and not cfg.shared_expert_intermediate_size
              and os.environ.get("MB_MOE_FUSED", "0") == "1"):
            # one GPU, opt-in (MB_MOE_FUSED=1): the same fused route + placement kernel and the combine
            # folded into the next add + RMSNorm (expert rows read in place), four launches per MoE layer
            # instead of nine.  Off by default: measured slower at Qwen3-30B-A3B decode on one B200
            # (7,451 vs 8,062 tok/s)
            from ..parallel.ep import FusedEPMoE

            moe_impl = FusedEPMoE(cfg, self.backend, max_tokens=max_batch,
                                  prefill_tokens=max(max_batch, min(2048, max_prefill_tokens)))
        if weights is None and model is None:
            if model_path is not None:
                from ..io.hf_loader import load_hf

                weights = load_hf(cfg, model_path, device=self.device, dtype=wdt)
            else:
                weights = random_weights(cfg, device=self.device, dtype=wdt, seed=seed)
        if quantization not in (None, "none", "int8"):
            raise ValueError(f"unknown quantization {quantization!r} (supported: int8)")
        if quantization == "int8" and weights is not None:
            from ..ops.quant import quantize_model

            quantize_model(weights, experts=not expert_parallel)
        self.quantization = quantization
        self.model = model if model is not None else DecoderLM(cfg, weights, self.backend, moe_impl=moe_impl)
        self.streamer = None
        if offload_layers == "auto":
            from ..parallel.planner import plan

            hbm = torch.cuda.get_device_properties(self.device).total_memory if self.device.type == "cuda" else 0
            offload_layers = plan(cfg, 1, hbm_bytes=hbm).offload_layers if hbm else 0
        if offload_layers and self.device.type == "cuda" and hasattr(self.model, "layer_source"):
            from ..runtime.offload import enable_streaming

            n = min(int(offload_layers), cfg.num_hidden_layers)
            self.streamer = enable_streaming(self.model, cfg.num_hidden_layers - n)
            use_graphs = False  # the streamer's copy schedule is decided per step on the host
        bs = 16
        if num_blocks is None:
            num_blocks = self._auto_blocks(kv_mem_fraction, max_batch, max_model_len, kv_heads)
        else:
            self.memory.define("kv", (num_blocks + 1) * KVCache.bytes_per_block(cfg, num_kv_heads=kv_heads or self.model.Hkv))
        # one block more than the allocator hands out: the last block is scratch that padded rows of a captured
        # decode step may write into (library-only path), so no live sequence's KV is touched
        self.kv = KVCache(cfg, num_blocks + 1, self.device, dtype=torch.float32 if backend == "cpu" else self.model.w.embed.dtype, block_size=bs, num_kv_heads=kv_heads or self.model.Hkv)
        has_delta = any(cfg.layer_type(i) == "linear_attention" for i in range(cfg.num_hidden_layers))
        if has_delta:  # a tensor-parallel model keeps only its heads' recurrent state
            sc = getattr(self.model, "state_cache", None)
            self.states = sc(max_batch + 1, self.device) if sc else StateCache(cfg, max_batch + 1, self.device)
        else:
            self.states = None
        # prefix caching shares KV blocks of common prompt prefixes; models with recurrent
        # (DeltaNet) state keep the plain manager, since their state is not in the KV blocks
        self.prefix_caching = bool(prefix_caching) and self.states is None
        mgr = PrefixCachingBlockManager if self.prefix_caching else BlockManager
        self.blocks = mgr(num_blocks, bs, max_seqs=max_batch)
        # chunked prefill (prefill_chunk tokens per step, alternating with decode steps); vision-language
        # models build a whole prompt's embeddings at once and keep whole-prompt prefill
        if prefill_chunk is not None and (prefill_chunk < 1 or getattr(self.model, "prefill_embeds", None)):
            prefill_chunk = None
        self.scheduler = Scheduler(self.blocks, max_batch=max_batch, max_prefill_tokens=max_prefill_tokens,
                                   prefill_chunk=prefill_chunk)
        # KV swap on preemption (attention-only models without prefix sharing): the preempted
        # sequence's blocks go to pinned host memory and come back into fresh blocks later
        self.swapper = None
        if kv_swap and self.states is None and not self.prefix_caching and self.kv.k:
            from ..runtime.memory import KVSwapper, PinnedPool

            self.swapper = KVSwapper(self.kv, PinnedPool(kv_swap_bytes))
            self.memory.define("host_swap", kv_swap_bytes)

            def on_preempt(seq):
                try:
                    self.swapper.swap_out(seq.req_id, list(seq.blocks))
                except Exception as e:  # pinned pool exhausted: fall back to recomputation
                    log.warning("KV swap-out failed (%s); request %d will be recomputed", e, seq.req_id)
                    return False
                return True

            self.scheduler.on_preempt = on_preempt
            self.scheduler.on_resume = lambda seq: self.swapper.swap_in(seq.req_id, list(seq.blocks))
        self.runner = ModelRunner(self.model, self.kv, self.states, self.blocks, max_batch, max_model_len,
                                  use_graphs=(backend == "native") if use_graphs is None else (use_graphs and backend != "cpu"),
                                  device=self.device)
        from .sampler import Sampler

        self.runner.sampler = Sampler()
        self.seqs: Dict[int, Sequence] = {}
        self.last_step: Dict[str, float] = {}
        # optional ``parallel.health.Heartbeat``: checked before every step so a lost
        # peer raises ``RankFailure`` here instead of stalling the next exchange
        self.health = None
        # expert parallelism with data-parallel attention: every rank takes part in every MoE
        # exchange, so the ranks step together (see ``_ep_step``)
        self._ep_lockstep = self.expert_parallel and world > 1 and moe_impl is not None
        self._ep_all_done = False
        self._ep_world = world
        self._ep_stop_requested = False
        self.ep_stopped = False   # every rank asked to stop: no further exchanges

    @classmethod
    def from_preset(cls, name: str, **kw) -> "LLMEngine":
        return cls(get_preset(name), **kw)

    def _auto_blocks(self, frac, max_batch, max_model_len, kv_heads) -> int:
        """KV blocks for ``max_batch`` sequences of ``max_model_len`` tokens, capped by what the
        memory manager has left after the weights and buffers already allocated on this device."""
        per_block = KVCache.bytes_per_block(self.cfg, num_kv_heads=kv_heads or self.model.Hkv)
        want = max_batch * ((max_model_len + 15) // 16) + max_batch
        if self.device.type != "cuda" or per_block == 0:
            self.memory.define("kv", max(want, 16) * per_block)
            return max(want, 16)
        free_now, _ = torch.cuda.mem_get_info(self.device)
        used = max(0, self.memory.free_at_start - free_now)   # weights, exchange buffers, caches so far
        cap = self.memory.plan_kv_blocks(per_block, used, workspace_bytes=1 << 30, fraction=frac) - 1
        n = max(16, min(want, cap))
        self.memory.define("kv", (n + 1) * per_block)
        return n

    # ------------------------------------------------------------------ API
    def add_request(self, prompt: Seq[int], params: Optional[SamplingParams] = None, images=None,
                    callback=None) -> int:
        seq = Sequence(prompt=list(int(t) for t in prompt), params=params or SamplingParams())
        seq.images, seq.callback = images, callback
        self.seqs[seq.req_id] = seq
        self.scheduler.add(seq)
        return seq.req_id

    def add_prefilled(self, prompt: Seq[int], first_token: int, k_layers: List[torch.Tensor],
                      v_layers: List[torch.Tensor], params: Optional[SamplingParams] = None) -> int:
        """Adds a request whose prompt was prefilled outside this engine (for example by a
        context-parallel prefill over several ranks): ``k_layers`` / ``v_layers`` hold the
        prompt's K (after QK-norm and RoPE) and V of every attention layer as [S, Hkv, D].
        The KV is handed to the swap path, so the scheduler copies it into fresh blocks
        and the request continues with decode steps; the prompt is never recomputed."""
        from ..parallel.cp_model import to_blocks

        if self.swapper is None:
            raise RuntimeError("add_prefilled needs the KV swap path (attention-only model, no prefix caching)")
        seq = Sequence(prompt=list(int(t) for t in prompt), params=params or SamplingParams())
        kb, vb = zip(*(to_blocks(k, v, self.kv.block_size) for k, v in zip(k_layers, v_layers)))
        self.swapper.stage(seq.req_id, [b.to(self.device) for b in kb + vb])
        seq.output.append(int(first_token))
        seq.num_cached = len(seq.prompt)
        seq.swapped = True
        seq.t_first_token = time.perf_counter()
        self.seqs[seq.req_id] = seq
        if seq.finished_by(int(first_token)):
            self.swapper.saved.pop(seq.req_id, None)
            self.swapper.external.discard(seq.req_id)
            seq.status, seq.t_finish = SeqStatus.FINISHED, seq.t_first_token
        else:
            self.scheduler.add(seq)
        return seq.req_id

    def generate_context_parallel(self, prompt: Seq[int], params: Optional[SamplingParams] = None,
                                  weights: Optional[ModelWeights] = None, group=None,
                                  mode: str = "ring") -> List[int]:
        """Collective: every rank of ``group`` passes the same long prompt.  The prompt is
        prefilled context-parallel (``parallel.cp_model.cp_prefill``: 1/N of the tokens per
        rank, ring or Ulysses attention across ranks), its KV lands in this engine's paged
        pool and the request decodes here.  ``weights`` defaults to the engine's own
        (unsharded) weights.  The first output token is the greedy choice."""
        from ..parallel.cp_model import cp_prefill

        w = weights if weights is not None else getattr(self.model, "w", None)
        if w is None:
            raise RuntimeError("generate_context_parallel needs the model's unsharded weights")
        logits, ks, vs = cp_prefill(self.cfg, w, prompt, group=group, mode=mode)
        rid = self.add_prefilled(prompt, int(logits.argmax()), ks, vs, params)
        seq = self.seqs[rid]
        while seq.status not in (SeqStatus.FINISHED, SeqStatus.FAILED, SeqStatus.ABORTED):
            self.step()
        if seq.error:
            raise RuntimeError(seq.error)
        return list(seq.output)

    def abort(self, req_id: int) -> bool:
        """Cancel a waiting or running request between steps; its KV blocks are freed.
        Returns False when the request is unknown or already finished."""
        seq = self.seqs.get(req_id)
        if seq is None or seq.status not in (SeqStatus.WAITING, SeqStatus.RUNNING):
            return False
        if seq in self.scheduler.waiting:
            self.scheduler.waiting.remove(seq)
            seq.status = SeqStatus.ABORTED
            if seq.blocks:
                self.blocks.release(seq)
        else:
            self.scheduler.finish(seq, SeqStatus.ABORTED)
        return True

    def has_unfinished(self) -> bool:
        return self.scheduler.has_work()

    def step(self) -> List[Sequence]:
        """Runs one prefill or decode step; returns sequences that finished in it.

        Under expert parallelism (several ranks) every rank must call ``step`` the same
        number of times: a rank with nothing to run takes part in its peers' MoE exchanges
        with a forward of one padding row."""
        sched = self.scheduler.schedule()
        if self._ep_lockstep:
            return self._ep_step(sched)
        if not sched.seqs:
            return []
        return self._run(sched)

    def keep_stepping(self) -> bool:
        """True while this rank must keep calling ``step``: it has work, or (expert
        parallelism) another rank may still have some."""
        return self.has_unfinished() or (self._ep_lockstep and not self._ep_all_done and not self.ep_stopped)

    def request_stop(self) -> None:
        """Expert parallelism: this rank will serve no more requests.  Stepping stops on every
        rank (``ep_stopped``) once all ranks have asked; until then this rank keeps taking
        part in its peers' steps."""
        self._ep_stop_requested = True

    def _ep_step(self, sched) -> List[Sequence]:
        """One lock-step of every expert-parallel rank.  One small all-reduce decides, for
        all ranks alike: whether any rank has work (if none, nothing runs); whether the step
        is eager (some rank prefills or samples, which takes the exchange's eager path with
        its own per-call agreement) or every rank replays a captured decode graph; and which
        decode graphs must be captured first (captures run collectively, since their warm-up
        forwards exchange too).  A rank without work runs a one-padding-row forward."""
        import torch.distributed as dist

        if self.ep_stopped:
            return []
        r = self.runner
        local_eager = bool(sched.seqs) and (not sched.is_decode or r.needs_sampling(sched.seqs))
        need = torch.zeros(3 + len(r.buckets), dtype=torch.int64)
        need[0] = int(local_eager)
        need[1] = int(bool(sched.seqs))
        need[2] = int(self._ep_stop_requested and not sched.seqs)
        if r.use_graphs:
            n = len(sched.seqs) if sched.seqs and sched.is_decode else 1
            need[3 + r.bucket_index(n)] = 1
        dev = self.device if dist.get_backend() == "nccl" else torch.device("cpu")
        need = need.to(dev)
        dist.all_reduce(need)
        need = need.cpu().tolist()
        if need[2] == self._ep_world:  # every rank is idle and asked to stop
            self.ep_stopped = True
            self._ep_all_done = True
            return []
        if not need[1]:
            self._ep_all_done = True
            return []
        self._ep_all_done = False
        eager = bool(need[0])
        if r.use_graphs and not eager:
            for i, b in enumerate(r.buckets):  # same buckets, same order, on every rank
                if need[3 + i] and b not in r.graphs:
                    r._copy_in(b)
                    r.capture(b)
        if not sched.seqs:
            r.idle_step(eager=eager)
            return []
        return self._run(sched, eager=eager)

    def _run(self, sched, eager: bool = False) -> List[Sequence]:
        if self.health is not None:
            self.health.check()
        t0 = time.perf_counter()
        try:
            with tracing.nvtx_range("decode" if sched.is_decode else "prefill"):
                if sched.is_decode:
                    toks = self.runner.decode(sched.seqs, eager=eager)
                else:
                    toks = self.runner.prefill(sched.seqs, sched.query_lens, self._embeds(sched))
        except Exception as e:  # fail the step's requests, keep serving others
            log.error("step failed: %s", e)
            for s in sched.seqs:
                s.error = repr(e)
                self.scheduler.finish(s, SeqStatus.FAILED)
            return list(sched.seqs)
        now = time.perf_counter()
        if self.prefix_caching:
            for s in sched.seqs:
                self.blocks.register(s)
        self.last_step = {"kind": 1.0 if sched.is_decode else 0.0, "seconds": now - t0, "batch": len(sched.seqs)}
        done = []
        for s, t in zip(sched.seqs, toks):
            if not sched.is_decode and s.num_cached < s.length:
                continue                      # a prefill chunk that did not reach the prompt's end
            if s.t_first_token is None:
                s.t_first_token = now
            s.output.append(int(t))
            if s.callback is not None:
                s.callback(s, int(t))
            if s.finished_by(int(t)):
                s.t_finish = now
                self.scheduler.finish(s)
                done.append(s)
        return done

    def _embeds(self, sched):
        hook = getattr(self.model, "prefill_embeds", None)
        return hook(sched) if hook is not None else None

    def generate(self, prompts: List[Seq[int]], params: Optional[SamplingParams] = None) -> List[List[int]]:
        ids = [self.add_request(p, params) for p in prompts]
        self._ep_all_done = False
        # expert parallelism: keep stepping (idle) until every rank is done
        while self.keep_stepping():
            self.step()
        out = []
        for i in ids:
            s = self.seqs.pop(i)
            if s.status == SeqStatus.FAILED:
                raise RuntimeError(f"request {i} failed: {s.error}")
            out.append(s.output)
        return out

    def stats(self) -> Dict[str, float]:
        return {"free_blocks": self.blocks.num_free, "running": len(self.scheduler.running),
                "waiting": len(self.scheduler.waiting), "preempted": self.scheduler.num_preempted,
                "swapped_out": self.scheduler.num_swapped_out, "resumed": self.scheduler.num_resumed,
                "h2d_bytes_last_step": self.runner.h2d_bytes, "d2h_bytes_last_step": self.runner.d2h_bytes}
