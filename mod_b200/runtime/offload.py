"""Hybrid CPU/GPU execution: stream layer weights from pinned host memory.

For models larger than device memory, :class:`LayerStreamer` keeps the first
``resident`` layers on the GPU and the rest in pinned host memory.  While layer
``i`` runs, layer ``i+1`` is copied host->device on a side stream into one of
two device slots; the compute stream waits on that copy's event before using
the slot.  This is the reference's "hybrid scheduler" policy (keep the current
layer on the device, prefetch the next ones on a transfer stream, evict the
old ones; ``pio/common/managers/hybrid_scheduler.py:40-94``), which in the
reference is never instantiated and calls non-existent backend hooks.
"""
from __future__ import annotations

import copy
from typing import List, Optional

import torch

from ..models.weights import LayerWeights, MLPWeights


def _tensors(obj, prefix=""):
    for k, v in vars(obj).items():
        if isinstance(v, torch.Tensor):
            yield prefix + k, obj, k, v
        elif isinstance(v, MLPWeights):
            yield from _tensors(v, prefix + k + ".")
        elif v is not None and hasattr(v, "__dict__") and not isinstance(v, (int, float, str)):
            yield from _tensors(v, prefix + k + ".")


def _layer_tensors(L: LayerWeights):
    for part in ("attn", "delta", "mlp", "moe"):
        o = getattr(L, part)
        if o is not None:
            yield from _tensors(o, part + ".")
    yield "in_norm", L, "in_norm", L.in_norm
    yield "post_norm", L, "post_norm", L.post_norm


class LayerStreamer:
    def __init__(self, layers: List[LayerWeights], device, resident: int):
        self.device = torch.device(device)
        self.resident = resident
        self.layers = layers
        self.copy_stream = torch.cuda.Stream(self.device)
        # move offloaded layers to pinned host memory
        for L in layers[resident:]:
            for _, obj, k, t in list(_layer_tensors(L)):
                if t.is_cuda:
                    setattr(obj, k, t.to("cpu").pin_memory())
        # two device slots shaped like an offloaded layer
        self.slots: List[Optional[LayerWeights]] = [None, None]
        self.slot_layer = [-1, -1]
        self.events = [torch.cuda.Event(), torch.cuda.Event()]
        if len(layers) > resident:
            for s in range(2):
                self.slots[s] = copy.deepcopy(_as_device_template(layers[resident], self.device))

    def _fill(self, slot: int, i: int) -> None:
        src, dst = self.layers[i], self.slots[slot]
        with torch.cuda.stream(self.copy_stream):
            for (name, _, _, t_src), (_, obj, k, t_dst) in zip(_layer_tensors(src), _layer_tensors(dst)):
                t_dst.copy_(t_src, non_blocking=True)
            self.events[slot].record(self.copy_stream)
        self.slot_layer[slot] = i

    def get(self, i: int) -> LayerWeights:
        if i < self.resident:
            if i + 1 == self.resident and i + 1 < len(self.layers):
                self._fill(0, i + 1)        # prefetch the first streamed layer
            return self.layers[i]
        slot = (i - self.resident) % 2
        if self.slot_layer[slot] != i:
            self._fill(slot, i)
        nxt = i + 1
        if nxt < len(self.layers):
            # the other slot is free once the compute stream has passed layer i-1
            self.copy_stream.wait_stream(torch.cuda.current_stream(self.device))
            self._fill(1 - slot, nxt)
        torch.cuda.current_stream(self.device).wait_event(self.events[slot])
        return self.slots[slot]


def _as_device_template(L: LayerWeights, device) -> LayerWeights:
    T = copy.copy(L)
    for part in ("attn", "delta", "mlp", "moe"):
        o = getattr(L, part)
        if o is not None:
            setattr(T, part, copy.deepcopy(o))
    for _, obj, k, t in list(_layer_tensors(T)):
        setattr(obj, k, torch.empty_like(t, device=device))
    return T


def enable_streaming(model, resident_layers: int) -> LayerStreamer:
    """Turns on weight streaming for a DecoderLM; returns the streamer."""
    st = LayerStreamer(model.w.layers, model.device, resident_layers)
    model.layer_source = st.get
    return st
