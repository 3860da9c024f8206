"""Gaussian embedding lookup (drop-in for triton_tagi/layers/embedding.py).

Forward gathers rows (μ_w[cat], S_w[cat]); backward accumulates
δμ·S_w[cat] and δS·S_w[cat]² into the rows with index_add (embedding.py:112-151).
This layer is outside the fused moment path and runs as torch device ops;
``padding_idx`` rows emit zeros and receive no update, as in the reference.
"""

from __future__ import annotations

import torch
from torch import Tensor

from ..base import LearnableLayer
from ..param_init import gaussian_param_init
from ..update.parameters import update_parameters


class Embedding(LearnableLayer):
    def __init__(self, num_embeddings: int, embedding_dim: int, input_size: int = 0,
                 scale: float = 1.0, padding_idx: int = -1, device="cuda") -> None:
        self.num_embeddings, self.embedding_dim = num_embeddings, embedding_dim
        self.input_size, self.scale, self.padding_idx = input_size, scale, padding_idx
        self.device = torch.device(device)
        self.has_bias = False
        self.mw, self.Sw = gaussian_param_init(scale, 1.0, (num_embeddings, embedding_dim),
                                               device=self.device)
        self.mb = self.Sb = None
        self.cat_idx = None
        self.delta_mw = self.delta_Sw = self.delta_mb = self.delta_Sb = None

    def forward(self, ma: Tensor, Sa: Tensor) -> tuple[Tensor, Tensor]:
        if ma.dim() == 3 and ma.shape[-1] == 1:
            ma = ma.squeeze(-1)
        cat = ma.long()
        self.cat_idx = cat
        mz, Sz = self.mw[cat], self.Sw[cat]
        if self.padding_idx >= 0:
            mask = (cat == self.padding_idx).unsqueeze(-1)
            mz, Sz = mz.masked_fill(mask, 0.0), Sz.masked_fill(mask, 0.0)
        return mz, Sz

    def _sums(self, delta_mz: Tensor, delta_Sz: Tensor):
        D = self.embedding_dim
        idx = self.cat_idx.reshape(-1)
        rows = self.Sw[idx]
        dm = delta_mz.reshape(-1, D)
        dS = delta_Sz.reshape(-1, D)
        if self.padding_idx >= 0:
            keep = (idx != self.padding_idx).unsqueeze(-1).to(dm.dtype)
            dm, dS = dm * keep, dS * keep
        return idx, dm, dS, rows

    def backward(self, delta_mz: Tensor, delta_Sz: Tensor) -> tuple[Tensor, Tensor]:
        idx, dm, dS, rows = self._sums(delta_mz, delta_Sz)
        if self._param_mode == "sums":
            buf = self._reducer.buffer(self, 2 * self.mw.numel(), torch.float32)
            g_m, g_S = buf.view(2, *self.mw.shape)
            g_m.zero_().index_add_(0, idx, dm)
            g_S.zero_().index_add_(0, idx, dS)
            self._reducer.ready(self)
        else:
            self.delta_mw = torch.zeros_like(self.mw).index_add_(0, idx, dm * rows)
            self.delta_Sw = torch.zeros_like(self.Sw).index_add_(0, idx, dS * rows * rows)
        z = torch.zeros(self.cat_idx.shape, dtype=delta_mz.dtype, device=delta_mz.device)
        return z, z.clone()

    def _sums_numel(self) -> int:
        return 2 * self.mw.numel()

    def _apply_sums(self, buf: Tensor, cap: float) -> None:
        g_m, g_S = buf.view(2, *self.mw.shape)
        update_parameters(self.mw, self.Sw, self.Sw * g_m, self.Sw * self.Sw * g_S, cap)

    def update(self, cap_factor: float) -> None:
        if self._param_mode == "sums":
            return
        update_parameters(self.mw, self.Sw, self.delta_mw, self.delta_Sw, cap_factor)

    @property
    def num_parameters(self) -> int:
        return 2 * self.mw.numel()

    def __repr__(self) -> str:
        return (f"Embedding(num_embeddings={self.num_embeddings}, "
                f"embedding_dim={self.embedding_dim}, padding_idx={self.padding_idx}, "
                f"scale={self.scale})")
