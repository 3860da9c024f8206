"""Fixed sinusoidal positional encoding (drop-in for
triton_tagi/layers/positional_encoding.py): pe[t, d] = sin(t·f_d) for even d,
cos(t·f_d) for odd d, f_d = 10000^(−d/E); added to the means only, identity
backward. Runs as torch device ops (outside the fused moment path)."""

from __future__ import annotations

import torch
from torch import Tensor

from ..base import Layer


class PositionalEncoding(Layer):
    def __init__(self, embed_dim: int, max_seq_len: int = 2048, device="cuda") -> None:
        self.embed_dim, self.max_seq_len = embed_dim, max_seq_len
        self.device = torch.device(device)
        d = torch.arange(embed_dim, dtype=torch.float32, device=self.device)
        pos = torch.arange(max_seq_len, dtype=torch.float32, device=self.device)
        angle = pos.unsqueeze(1) * (1.0 / torch.pow(10000.0, d / embed_dim)).unsqueeze(0)
        even = (torch.arange(embed_dim, device=self.device) % 2 == 0).unsqueeze(0)
        self.pe_cache = torch.where(even, torch.sin(angle), torch.cos(angle))

    def forward(self, ma: Tensor, Sa: Tensor) -> tuple[Tensor, Tensor]:
        return ma + self.pe_cache[: ma.shape[-2]], Sa

    def backward(self, delta_ma: Tensor, delta_Sa: Tensor) -> tuple[Tensor, Tensor]:
        return delta_ma, delta_Sa

    def __repr__(self) -> str:
        return f"PositionalEncoding(embed_dim={self.embed_dim}, max_seq_len={self.max_seq_len})"
