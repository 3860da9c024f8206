"""Fixed sinusoidal positional encoding (drop-in for
triton_tagi/layers/positional_encoding.py): pe[t, d] = sin(t·f_d) for even d,
cos(t·f_d) for odd d, f_d = 10000^(−d/E); added to the means only
(tagi_positional_add), identity backward. The table is built once at
construction with the reference's torch operations on the host, in float32, and
copied to the device: CUDA's pow, sin and cos differ from the host's in the last
bit, and a one-bit difference of f_d becomes ~1e-5 in sin(t·f_d) at positions in
the hundreds, so a device-built table would not reproduce the reference's
host-built one."""

from __future__ import annotations

import torch
from torch import Tensor

from .._lib import check_cuda_f32, lib, stream
from ..base import Layer


class PositionalEncoding(Layer):
    def __init__(self, embed_dim: int, max_seq_len: int = 2048, device="cuda") -> None:
        self.embed_dim, self.max_seq_len = embed_dim, max_seq_len
        self.device = torch.device(device)
        d = torch.arange(embed_dim, dtype=torch.float32)
        pos = torch.arange(max_seq_len, dtype=torch.float32)
        angle = pos.unsqueeze(1) * (1.0 / torch.pow(10000.0, d / embed_dim)).unsqueeze(0)
        even = (torch.arange(embed_dim) % 2 == 0).unsqueeze(0)
        self.pe_cache = torch.where(even, torch.sin(angle), torch.cos(angle)).to(self.device)

    def forward(self, ma: Tensor, Sa: Tensor) -> tuple[Tensor, Tensor]:
        check_cuda_f32(ma)
        if ma.dim() < 2 or ma.shape[-1] != self.embed_dim or ma.shape[-2] > self.max_seq_len:
            raise ValueError(f"PositionalEncoding: input {tuple(ma.shape)} does not fit "
                             f"(S <= {self.max_seq_len}, E = {self.embed_dim})")
        ma = ma.contiguous()
        out = torch.empty_like(ma)
        S, E = ma.shape[-2], self.embed_dim
        lib()("tagi_positional_add", ma.data_ptr(), self.pe_cache.data_ptr(), out.data_ptr(),
              ma.numel() // E, S, E, stream(ma))
        return out, Sa

    def backward(self, delta_ma: Tensor, delta_Sa: Tensor) -> tuple[Tensor, Tensor]:
        return delta_ma, delta_Sa

    def __repr__(self) -> str:
        return f"PositionalEncoding(embed_dim={self.embed_dim}, max_seq_len={self.max_seq_len})"
