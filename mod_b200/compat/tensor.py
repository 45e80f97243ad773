"""Reference-compatible ``Tensor`` method surface over ``torch.Tensor``.

The reference's tensor type (``src/inference_pio/core/engine/backend.py:201-654``)
wraps a C ``Tensor*`` (fp32 only) and exposes one method per C op.  Users of
that API can keep their code: this class holds a ``torch.Tensor`` (``.data``)
on the device named by the same strings (``"cpu"``, ``"cuda:N"``) and
implements every method with the same name, arguments and result shape.

Semantics follow the reference's CPU library where it is correct and fix it
where it is not: ``rope`` indexes its cos/sin table by sequence position for
every head (the reference folds the head into the index on CUDA);
``gather_by_value`` returns rows in ascending index order (the reference's
atomic counter makes the order arbitrary); GQA shapes never overrun.  Values
are fp32 like the reference; the engine's bf16 kernels are the fast path for
whole models, this class is for code written against the reference's op API.
Index results (``topk``, ``argmax``, ``gather_by_value``) are fp32 tensors as
in the reference, whose tensors are all fp32.
"""
from __future__ import annotations

from typing import List, Optional, Sequence, Tuple, Union

import torch
import torch.nn.functional as F


def _device(device: str) -> torch.device:
    if device.startswith("cuda"):
        if not torch.cuda.is_available():
            raise RuntimeError(f"device {device!r} requested but CUDA is not available")
        return torch.device(device if ":" in device else "cuda:0")
    if device != "cpu":
        raise ValueError(f"unsupported device {device!r} (cpu or cuda:N)")
    return torch.device("cpu")


class Tensor:
    __slots__ = ("data", "device")

    def __init__(self, shape: Sequence[int], data: Optional[Sequence[float]] = None, device: str = "cpu",
                 _t: Optional[torch.Tensor] = None):
        self.device = device
        if _t is not None:
            self.data = _t.to(device=_device(device), dtype=torch.float32)
        else:
            self.data = torch.zeros(*shape, dtype=torch.float32, device=_device(device))
            if data is not None:
                self.load(data)

    @classmethod
    def from_torch(cls, t: torch.Tensor, device: Optional[str] = None) -> "Tensor":
        dev = device or (f"cuda:{t.device.index or 0}" if t.is_cuda else "cpu")
        return cls(list(t.shape), device=dev, _t=t)

    def _new(self, t: torch.Tensor) -> "Tensor":
        return Tensor(list(t.shape), device=self.device, _t=t)

    # ------------------------------------------------------------------ storage
    def load(self, data: Sequence[float]) -> None:
        src = torch.as_tensor(list(data), dtype=torch.float32)
        if src.numel() != self.data.numel():
            raise ValueError(f"load: {src.numel()} values for a tensor of {self.data.numel()}")
        self.data.copy_(src.view(self.data.shape))

    def to_list(self) -> List[float]:
        return self.data.reshape(-1).tolist()

    def to(self, device: str, non_blocking: bool = False) -> "Tensor":
        return Tensor(list(self.shape), device=device, _t=self.data.to(_device(device), non_blocking=non_blocking))

    def synchronize(self) -> None:
        if self.data.is_cuda:
            torch.cuda.synchronize(self.data.device)

    @property
    def shape(self) -> Tuple[int, ...]:
        return tuple(self.data.shape)

    @property
    def ndim(self) -> int:
        return self.data.dim()

    @property
    def size(self) -> int:
        return self.data.numel()

    @property
    def dtype(self) -> str:
        return "float32"

    def fill(self, value: float) -> None:
        self.data.fill_(value)

    # ------------------------------------------------------------------ elementwise / linear algebra
    def matmul(self, other: "Tensor", transpose_b: bool = False) -> "Tensor":
        b = other.data.transpose(-1, -2) if transpose_b else other.data
        return self._new(torch.matmul(self.data, b))

    def add(self, other: "Tensor") -> "Tensor":
        return self._new(self.data + other.data)

    def mul(self, other: Union["Tensor", float]) -> "Tensor":
        return self._new(self.data * (other.data if isinstance(other, Tensor) else float(other)))

    def swiglu(self, up_proj_out: "Tensor") -> "Tensor":
        return self._new(F.silu(self.data) * up_proj_out.data)

    def fused_swiglu(self) -> "Tensor":
        g, u = self.data.chunk(2, dim=-1)
        return self._new(F.silu(g) * u)

    def permute(self, dims: Sequence[int]) -> "Tensor":
        if len(dims) != self.ndim:
            raise ValueError("Permute dims mismatch")
        return self._new(self.data.permute(*dims).contiguous())

    def reshape(self, new_shape: Sequence[int]) -> "Tensor":
        n = 1
        for s in new_shape:
            n *= s
        if n != self.size:
            raise ValueError("Reshape size mismatch")
        return self._new(self.data.reshape(*new_shape).clone())

    def gather(self, indices: "Tensor", axis: int = 0) -> "Tensor":
        return self._new(self.data.index_select(axis, indices.data.reshape(-1).long()))

    def scatter_add(self, indices: "Tensor", src: "Tensor", axis: int = 0) -> None:
        self.data.index_add_(axis, indices.data.reshape(-1).long(), src.data)

    def topk(self, k: int) -> Tuple["Tensor", "Tensor"]:
        v, i = torch.topk(self.data, k, dim=-1)
        return self._new(v), self._new(i.float())

    def linear(self, weight: "Tensor", bias: Optional["Tensor"] = None) -> "Tensor":
        w = weight.data if weight.ndim >= 2 else weight.data[None]
        if self.shape[-1] != w.shape[1]:
            raise ValueError("Linear shape mismatch")
        return self._new(F.linear(self.data, w, None if bias is None else bias.data))

    def conv2d(self, weight: "Tensor", bias: Optional["Tensor"] = None, stride: int = 1, padding: int = 0,
               groups: int = 1) -> "Tensor":
        if self.ndim != 4:
            raise ValueError("Conv2d requires 4D input")
        return self._new(F.conv2d(self.data, weight.data, None if bias is None else bias.data, stride, padding,
                                  groups=groups))

    def softmax(self, dim: int = -1) -> "Tensor":
        return self._new(torch.softmax(self.data, dim=dim))

    def silu(self) -> "Tensor":
        return self._new(F.silu(self.data))

    def gelu(self) -> "Tensor":
        return self._new(F.gelu(self.data, approximate="tanh"))

    def rms_norm(self, weight: "Tensor", eps: float = 1e-6) -> "Tensor":
        x = self.data
        return self._new(x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + eps) * weight.data)

    def fused_add_rms_norm(self, residual: "Tensor", weight: "Tensor", eps: float) -> "Tensor":
        """``self += residual`` (in place, as the reference's kernel), then RMSNorm(self) * weight."""
        self.data.add_(residual.data)
        return self.rms_norm(weight, eps)

    def dequantize(self, scale: "Tensor") -> "Tensor":
        return self._new(self.data * scale.data)

    # ------------------------------------------------------------------ positional encoding
    @staticmethod
    def _rotate(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
        # x [..., S, H, D]; cos/sin [S, D/2] indexed by sequence position for every head
        half = x.shape[-1] // 2
        c, s = cos[:, None, :], sin[:, None, :]
        x1, x2 = x[..., :half], x[..., half:]
        return torch.cat([x1 * c - x2 * s, x1 * s + x2 * c], dim=-1)

    def rope(self, k: "Tensor", cos: "Tensor", sin: "Tensor") -> Tuple["Tensor", "Tensor"]:
        """q = self [..., S, Hq, D], k [..., S, Hkv, D] (any head counts), cos/sin [S, D/2]."""
        return (self._new(self._rotate(self.data, cos.data, sin.data)),
                self._new(self._rotate(k.data, cos.data, sin.data)))

    def fused_split_rope(self, cos: "Tensor", sin: "Tensor", heads: int,
                         head_dim: int) -> Tuple["Tensor", "Tensor", "Tensor"]:
        """self [B, S, 3 * heads * head_dim] -> RoPE'd q, k and v, each [B, S, heads, head_dim]."""
        B, S = self.shape[0], self.shape[1]
        q, k, v = self.data.reshape(B, S, 3, heads, head_dim).unbind(2)
        return (self._new(self._rotate(q, cos.data, sin.data)), self._new(self._rotate(k, cos.data, sin.data)),
                self._new(v.contiguous()))

    # ------------------------------------------------------------------ selection
    def argmax(self, dim: int = -1) -> "Tensor":
        return self._new(self.data.argmax(dim=dim).float())

    def embed(self, indices: "Tensor") -> "Tensor":
        """self is the [vocab, hidden] table; indices of any shape."""
        ids = indices.data.long()
        if ids.numel() and (int(ids.min()) < 0 or int(ids.max()) >= self.shape[0]):
            raise IndexError("embed: token id out of range")
        return self._new(self.data[ids])

    def slice(self, start_indices: Union[Sequence[int], "Tensor"], slice_shapes: Sequence[int]) -> "Tensor":
        st = [int(x) for x in (start_indices.to_list() if isinstance(start_indices, Tensor) else start_indices)]
        if len(st) != self.ndim or len(slice_shapes) != self.ndim:
            raise ValueError("Slice args dim mismatch")
        idx = tuple(slice(a, a + n) for a, n in zip(st, slice_shapes))
        return self._new(self.data[idx].clone())

    def set_slice(self, src: "Tensor", start_indices: Union[Sequence[int], "Tensor"]) -> None:
        st = [int(x) for x in (start_indices.to_list() if isinstance(start_indices, Tensor) else start_indices)]
        if len(st) != self.ndim:
            raise ValueError("Set Slice args dim mismatch")
        idx = tuple(slice(a, a + n) for a, n in zip(st, src.shape))
        self.data[idx] = src.data

    def resize_image(self, target_h: int, target_w: int) -> "Tensor":
        """Bilinear resize of a [C, H, W] image (half-pixel centres, edge clamp)."""
        if self.ndim != 3:
            raise ValueError("Image resize expects 3D tensor")
        if not self.data.is_cuda:
            try:
                from .. import _cpu  # C++ backend

                out = torch.empty(self.shape[0], target_h, target_w)
                _cpu.resize_bilinear(self.data.contiguous(), out)
                return self._new(out)
            except ImportError:
                pass
        return self._new(F.interpolate(self.data[None], size=(target_h, target_w), mode="bilinear",
                                       align_corners=False)[0])

    # ------------------------------------------------------------------ MoE primitives
    def count_value(self, value: float) -> int:
        return int(((self.data - value).abs() < 1e-6).sum())

    def gather_by_value(self, indices: "Tensor", value: float) -> Tuple[Optional["Tensor"], Optional["Tensor"]]:
        """Rows i of self (one row per element of ``indices``) where indices[i] == value, in ascending i."""
        sel = ((indices.data.reshape(-1) - value).abs() < 1e-6).nonzero().reshape(-1)
        if sel.numel() == 0:
            return None, None
        rows = self.data.reshape(-1, self.shape[-1])
        return self._new(rows[sel]), self._new(sel.float())

    def scatter_add_by_index(self, src: "Tensor", indices: "Tensor") -> None:
        """self[indices[i]] += src[i]; out-of-range indices are skipped."""
        H = src.shape[-1]
        out = self.data.view(-1, H)
        idx = indices.data.reshape(-1).long()
        ok = (idx >= 0) & (idx < out.shape[0])
        out.index_add_(0, idx[ok], src.data.reshape(-1, H)[ok])

    def deltanet_recurrence(self, k: "Tensor", v: "Tensor", beta: "Tensor", state: "Tensor") -> "Tensor":
        """The reference's linear recurrence: S_t = beta_t * S_{t-1} + k_t v_t^T, o_t = q_t^T S_t.
        self = q [B, S, H, D], k/v [B, S, H, D], beta [B, S, H], state [B, H, D, D] (updated in place)."""
        q, kk, vv, bb = self.data, k.data, v.data, beta.data
        S = state.data
        out = torch.empty_like(q)
        for t in range(q.shape[1]):
            S.mul_(bb[:, t, :, None, None]).add_(kk[:, t, :, :, None] * vv[:, t, :, None, :])
            out[:, t] = torch.einsum("bhd,bhde->bhe", q[:, t], S)
        return self._new(out)

    def __repr__(self) -> str:
        return f"Tensor(shape={list(self.shape)}, device={self.device!r})"
