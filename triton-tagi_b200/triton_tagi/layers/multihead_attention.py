"""Bayesian multi-head self-attention, separate Q/K/V projections (drop-in for
triton_tagi/layers/multihead_attention.py; no RoPE, no causal mask, H_kv = H).

Forward (multihead_attention.py:154-207): Q, K, V Linear projections →
scores μ = s μ_q μ_kᵀ and var = s² Σ(S_q S_k + S_q μ_k² + S_k μ_q²) from one
fused batched kernel → Remax over each score row → μ_sv, var_sv from one fused
batched kernel over (score, V).
Backward (multihead_attention.py:212-268): δV = μ_scoreᵀ-shared product,
δscore = μ_v-shared product, Remax Jacobian (μ·J, var·J²), δQ and δK with
the scale s, then the three projection backwards summed.
"""

from __future__ import annotations

import math

import torch
from torch import Tensor

from ..base import LearnableLayer
from ..kernels.attention import bmm_shared_left, bmm_shared_right, bmm_tagi_moments
from .linear import Linear
from .relu import jacobian_backward
from .remax import triton_remax


class MultiheadAttentionV2(LearnableLayer):
    def __init__(self, embed_dim: int, num_heads: int, seq_len: int, num_kv_heads=None,
                 bias: bool = False, gain_weight: float = 1.0, gain_bias: float = 1.0,
                 init_method: str = "He", pos_emb: str = "", use_causal_mask: bool = False,
                 device="cuda") -> None:
        if pos_emb != "":
            raise NotImplementedError(
                f"MultiheadAttentionV2 only supports pos_emb='' (got {pos_emb!r})")
        if use_causal_mask:
            raise NotImplementedError("MultiheadAttentionV2 does not support causal masking")
        if num_kv_heads is None:
            num_kv_heads = num_heads
        if num_kv_heads != num_heads:
            raise NotImplementedError("Grouped-query attention (num_kv_heads != num_heads)")
        if embed_dim % num_heads != 0:
            raise ValueError(f"embed_dim ({embed_dim}) must be divisible by num_heads ({num_heads})")
        self.embed_dim, self.num_heads, self.num_kv_heads = embed_dim, num_heads, num_kv_heads
        self.seq_len, self.has_bias = seq_len, bias
        self.init_method, self.gain_weight, self.gain_bias = init_method, gain_weight, gain_bias
        self.device = torch.device(device)
        self.head_dim = embed_dim // num_heads
        kw = dict(device=device, init_method=init_method, gain_w=gain_weight, gain_b=gain_bias,
                  bias=bias)
        self.q_proj = Linear(embed_dim, num_heads * self.head_dim, **kw)
        self.k_proj = Linear(embed_dim, num_kv_heads * self.head_dim, **kw)
        self.v_proj = Linear(embed_dim, num_kv_heads * self.head_dim, **kw)
        self._scale = 1.0 / math.sqrt(self.head_dim)
        self._cache = None
        self._attn_mu = self._attn_var = None

    def _leaves(self):
        return [self.q_proj, self.k_proj, self.v_proj]

    def forward(self, ma: Tensor, Sa: Tensor) -> tuple[Tensor, Tensor]:
        B, S, E = ma.shape
        if E != self.embed_dim:
            raise ValueError(f"Expected last dim {self.embed_dim}, got {E}")
        H, D = self.num_heads, self.head_dim
        heads = lambda t: t.reshape(B, S, H, D).transpose(1, 2).contiguous()  # noqa: E731
        mq, Sq = map(heads, self.q_proj.forward(ma, Sa))
        mk, Sk = map(heads, self.k_proj.forward(ma, Sa))
        mv, Sv = map(heads, self.v_proj.forward(ma, Sa))
        s = self._scale
        mu_qk, var_qk = bmm_tagi_moments(mq, Sq, mk.transpose(-1, -2), Sk.transpose(-1, -2),
                                         s, s * s)
        mu_sc, var_sc, jcb = triton_remax(mu_qk.reshape(B * H * S, S), var_qk.reshape(B * H * S, S))
        mu_sc, var_sc, jcb = (t.reshape(B, H, S, S) for t in (mu_sc, var_sc, jcb))
        mu_sv, var_sv = bmm_tagi_moments(mu_sc, var_sc, mv, Sv, 1.0, 1.0)
        back = lambda t: t.transpose(1, 2).contiguous().reshape(B, S, H * D)  # noqa: E731
        self._cache = dict(B=B, S=S, H=H, D=D, mu_q=mq, mu_k=mk, mu_v=mv, mu_score=mu_sc, jcb=jcb)
        self._attn_mu, self._attn_var = mu_sc, var_sc
        return back(mu_sv), back(var_sv)

    def backward(self, delta_mz: Tensor, delta_Sz: Tensor) -> tuple[Tensor, Tensor]:
        c = self._cache
        B, S, H, D = c["B"], c["S"], c["H"], c["D"]
        heads = lambda t: t.reshape(B, S, H, D).transpose(1, 2).contiguous()  # noqa: E731
        d_mu, d_var = heads(delta_mz), heads(delta_Sz)
        dmv, dSv = bmm_shared_left(c["mu_score"].transpose(-1, -2), d_mu, d_var)
        dmsc, dSsc = bmm_shared_right(d_mu, d_var, c["mu_v"].transpose(-1, -2))
        sm, sv = jacobian_backward(dmsc, dSsc, c["jcb"])
        dmq, dSq = bmm_shared_right(sm, sv, c["mu_k"], scale=self._scale)
        dmk, dSk = bmm_shared_right(sm.transpose(-1, -2), sv.transpose(-1, -2), c["mu_q"],
                                    scale=self._scale)
        back = lambda t: t.transpose(1, 2).contiguous().reshape(B, S, H * D)  # noqa: E731
        a = self.q_proj.backward(back(dmq), back(dSq))
        b = self.k_proj.backward(back(dmk), back(dSk))
        v = self.v_proj.backward(back(dmv), back(dSv))
        return a[0] + b[0] + v[0], a[1] + b[1] + v[1]

    def update(self, cap_factor: float) -> None:
        for p in (self.q_proj, self.k_proj, self.v_proj):
            p.update(cap_factor)

    @property
    def num_parameters(self) -> int:
        return sum(p.num_parameters for p in (self.q_proj, self.k_proj, self.v_proj))

    def get_attention_scores(self) -> tuple[Tensor, Tensor]:
        if self._attn_mu is None:
            raise RuntimeError("No attention scores yet; call forward first.")
        return self._attn_mu, self._attn_var

    def __repr__(self) -> str:
        return (f"MultiheadAttentionV2(embed_dim={self.embed_dim}, num_heads={self.num_heads}, "
                f"seq_len={self.seq_len}, bias={self.has_bias})")
