"""Gaussian embedding lookup (drop-in for triton_tagi/layers/embedding.py).

Forward gathers rows (μ_w[cat], S_w[cat]) (tagi_embedding_forward); backward
accumulates δμ·S_w[cat] and δS·S_w[cat]² per row in token order
(tagi_embedding_backward: deterministic, the same additions as the reference's
index_add on the CPU; embedding.py:112-151). ``padding_idx`` rows emit zeros and
receive no update, as in the reference; ids outside the table do the same
instead of aborting the device context.

Token ids travel to the kernels as float32, which holds every integer up to
2^24 exactly; larger vocabularies are refused at construction (an integer id
tensor would otherwise be rounded to a neighbouring row without error).
"""

from __future__ import annotations

import torch
from torch import Tensor

from .._lib import WGRAD_DELTAS, WGRAD_SUMS, check_cuda_f32, lib, stream
from ..base import LearnableLayer
from ..param_init import gaussian_param_init
from ..update.parameters import update_parameters


class Embedding(LearnableLayer):
    def __init__(self, num_embeddings: int, embedding_dim: int, input_size: int = 0,
                 scale: float = 1.0, padding_idx: int = -1, device="cuda") -> None:
        if num_embeddings > 2**24:
            raise ValueError(f"Embedding: num_embeddings={num_embeddings} exceeds 2^24, the "
                             "largest vocabulary whose ids float32 holds exactly")
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
        ids = ma.float().contiguous()
        check_cuda_f32(ids)
        self.mw, self.Sw = self.mw.contiguous(), self.Sw.contiguous()
        self._ids = ids
        self.cat_idx = ids.long()
        D = self.embedding_dim
        mz = torch.empty(*ids.shape, D, device=ids.device)
        Sz = torch.empty_like(mz)
        lib()("tagi_embedding_forward", ids.data_ptr(), self.mw.data_ptr(), self.Sw.data_ptr(),
              mz.data_ptr(), Sz.data_ptr(), ids.numel(), self.num_embeddings, D,
              self.padding_idx, stream(ids))
        return mz, Sz

    def backward(self, delta_mz: Tensor, delta_Sz: Tensor) -> tuple[Tensor, Tensor]:
        check_cuda_f32(delta_mz, delta_Sz)
        ids = self._ids
        dm, dS = delta_mz.contiguous(), delta_Sz.contiguous()
        if dm.numel() != ids.numel() * self.embedding_dim:
            raise ValueError("Embedding.backward: deltas do not match the last forward")
        V, D = self.num_embeddings, self.embedding_dim
        args = (ids.data_ptr(), dm.data_ptr(), dS.data_ptr(), self.Sw.data_ptr(), ids.numel(),
                V, D, self.padding_idx)
        if self._param_mode == "sums":
            buf = self._reducer.buffer(self, 2 * self.mw.numel(), torch.float32)
            g_m, g_S = buf.view(2, *self.mw.shape)
            lib()("tagi_embedding_backward", *args, WGRAD_SUMS, g_m.data_ptr(), g_S.data_ptr(),
                  stream(dm))
            self._reducer.ready(self)
        else:
            self.delta_mw = torch.empty_like(self.mw)
            self.delta_Sw = torch.empty_like(self.Sw)
            lib()("tagi_embedding_backward", *args, WGRAD_DELTAS, self.delta_mw.data_ptr(),
                  self.delta_Sw.data_ptr(), stream(dm))
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
