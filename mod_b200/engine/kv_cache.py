"""Paged KV cache and recurrent-state cache.

KV layout per full-attention layer: K ``[num_blocks, Hkv, block_size, D]`` and
V ``[num_blocks, Hkv, D, block_size]`` (transposed inside a block, so the
tensor-core P.V product reads it K-major, one 16-token block per MMA),
block_size 16.  A (block, head) tile is one contiguous 4 KiB run at D = 128,
which the decode kernel reads with 16-byte vector loads.  The reference keeps
a static ``[B, Smax, Hkv, D]`` cache per layer filled by ``set_slice``
(``pio/models/qwen3_0_6b/architecture.py:92-100, 188-201``).

Recurrent state (gated DeltaNet layers) is kept per sequence slot:
``conv [slots, C, K-1]`` and ``ssm [slots, Hv, dk, dv]`` in fp32.
"""
from __future__ import annotations

from typing import Dict, List

import torch

from ..config.models import ModelConfig


class KVCache:
    def __init__(self, cfg: ModelConfig, num_blocks: int, device, dtype=torch.bfloat16, block_size: int = 16,
                 num_kv_heads: int = None):
        self.block_size = block_size
        self.num_blocks = num_blocks
        hkv = num_kv_heads or cfg.num_key_value_heads
        self.layer_index: Dict[int, int] = {}
        self.k: List[torch.Tensor] = []
        self.v: List[torch.Tensor] = []
        for i in range(cfg.num_hidden_layers):
            if cfg.layer_type(i) == "full_attention":
                self.layer_index[i] = len(self.k)
                self.k.append(torch.zeros(num_blocks, hkv, block_size, cfg.head_dim, device=device, dtype=dtype))
                self.v.append(torch.zeros(num_blocks, hkv, cfg.head_dim, block_size, device=device, dtype=dtype))

    def layer(self, i: int):
        j = self.layer_index[i]
        return self.k[j], self.v[j]

    @staticmethod
    def bytes_per_block(cfg: ModelConfig, block_size: int = 16, dtype=torch.bfloat16, num_kv_heads: int = None) -> int:
        n_attn = sum(1 for i in range(cfg.num_hidden_layers) if cfg.layer_type(i) == "full_attention")
        hkv = num_kv_heads or cfg.num_key_value_heads
        return 2 * n_attn * hkv * block_size * cfg.head_dim * torch.tensor([], dtype=dtype).element_size()


class StateCache:
    def __init__(self, cfg: ModelConfig, max_seqs: int, device, num_v_heads: int = None, num_k_heads: int = None):
        self.layer_index: Dict[int, int] = {}
        self.conv: List[torch.Tensor] = []
        self.ssm: List[torch.Tensor] = []
        hv = num_v_heads or cfg.linear_num_value_heads
        hk = num_k_heads or cfg.linear_num_key_heads
        C = 2 * hk * cfg.linear_key_head_dim + hv * cfg.linear_value_head_dim
        for i in range(cfg.num_hidden_layers):
            if cfg.layer_type(i) == "linear_attention":
                self.layer_index[i] = len(self.conv)
                self.conv.append(torch.zeros(max_seqs, C, cfg.linear_conv_kernel_dim - 1, device=device,
                                             dtype=torch.float32))
                self.ssm.append(torch.zeros(max_seqs, hv, cfg.linear_key_head_dim, cfg.linear_value_head_dim,
                                            device=device, dtype=torch.float32))

    def layer(self, i: int):
        j = self.layer_index[i]
        return self.conv[j], self.ssm[j]

    def reset(self, slots) -> None:
        for c, s in zip(self.conv, self.ssm):
            c[slots] = 0
            s[slots] = 0
