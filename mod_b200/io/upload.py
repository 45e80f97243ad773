"""Host -> device weight upload through two pinned staging buffers.

A tensor read from the checkpoint mapping is pageable memory, so a plain
``.to("cuda")`` copies it synchronously through the driver's own bounce
buffer, and the page-ins of the mapping, the host-side copy and the DMA all
run one after another.  :class:`StagedUploader` cuts each tensor's bytes into
chunks and alternates between two pinned buffers: while the DMA engine copies
chunk i from one buffer (on a side stream), the host copies chunk i+1 out of
the mapping into the other, so disk/page-cache reads overlap the PCIe / C2C
transfer.  A dtype change (e.g. an fp32 checkpoint served in bf16) runs on
the device after the raw bytes have landed.

The reference reads every tensor into host memory first and converts BF16 by
hand (``pio/common/custom_components/model_loader.py:77-123``).
"""
from __future__ import annotations

from typing import Optional

import torch


class StagedUploader:
    def __init__(self, device, chunk_bytes: int = 64 << 20):
        self.device = torch.device(device)
        self.chunk = int(chunk_bytes)
        self.bufs = [torch.empty(self.chunk, dtype=torch.uint8, pin_memory=True) for _ in range(2)]
        self.stream = torch.cuda.Stream(device=self.device)
        self.done = [torch.cuda.Event() for _ in range(2)]
        self.used = [False, False]
        self.nbytes = 0          # bytes uploaded so far
        self.nchunks = 0

    def upload(self, src: torch.Tensor, dtype: Optional[torch.dtype] = None) -> torch.Tensor:
        """``src`` (host tensor, any layout) -> a new contiguous device tensor of ``dtype``."""
        src = src.contiguous()
        raw = src.view(-1).view(torch.uint8) if src.numel() else src.new_empty(0, dtype=torch.uint8)
        dst = torch.empty(src.shape, dtype=src.dtype, device=self.device)
        draw = dst.view(-1).view(torch.uint8) if dst.numel() else None
        n = raw.numel()
        off = 0
        while off < n:
            i = self.nchunks & 1
            m = min(self.chunk, n - off)
            if self.used[i]:
                self.done[i].synchronize()          # the DMA that last read this buffer has finished
            self.bufs[i][:m].copy_(raw[off:off + m])  # host: mapping -> pinned (page-ins happen here)
            with torch.cuda.stream(self.stream):
                draw[off:off + m].copy_(self.bufs[i][:m], non_blocking=True)
                self.done[i].record(self.stream)
            self.used[i] = True
            self.nchunks += 1
            off += m
        self.nbytes += n
        # later work on the caller's stream (the dtype cast, the model) sees the finished copy, and the
        # allocator does not hand dst's memory to the caller's stream while the side stream still writes it
        torch.cuda.current_stream(self.device).wait_stream(self.stream)
        dst.record_stream(self.stream)
        if dtype is not None and dtype != dst.dtype:
            dst = dst.to(dtype)
        return dst

    def finish(self) -> None:
        self.stream.synchronize()
