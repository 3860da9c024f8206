"""CPU restatement of triton-tagi's layer classes and ``Sequential.step``
(test oracle and timed CPU baseline).

The classes hold the same public attributes as the reference layers
(``mw, Sw, mb, Sb``, ``delta_*``, ``running_mean/var``) so that parameters can be
copied between an oracle network and a CUDA network and compared after a step.
Each method cites the reference lines it follows.
"""

from __future__ import annotations

import math

import torch
from torch import Tensor

from . import moments as F


class Layer:
    learnable = False

    def forward(self, ma, Sa):  # pragma: no cover - interface
        raise NotImplementedError

    def backward(self, dm, dS):  # pragma: no cover - interface
        raise NotImplementedError


def _gauss(scale, gain, shape):
    """triton_tagi/param_init.py:57-84 (global torch RNG, as the reference)."""
    m = torch.randn(shape) * scale
    return m, torch.full(shape, (gain * scale) ** 2)


def _scale(init_method, fan_in, fan_out):
    """triton_tagi/param_init.py:22-54."""
    if init_method.lower() == "he":
        return F.he_scale(fan_in)
    if init_method.lower() == "xavier":
        return math.sqrt(2.0 / (fan_in + fan_out))
    raise ValueError(f"Unsupported init method: {init_method}")


class Linear(Layer):
    """triton_tagi/layers/linear.py:30-181."""

    learnable = True

    def __init__(self, in_features, out_features, device="cpu", init_method="He", gain_w=1.0,
                 gain_b=1.0, bias=True):
        in_f, out_f = in_features, out_features
        self.in_features, self.out_features, self.has_bias = in_f, out_f, bias
        s = _scale(init_method, in_f, out_f)
        self.mw, self.Sw = _gauss(s, gain_w, (in_f, out_f))
        if bias:
            self.mb, self.Sb = _gauss(s, gain_b, (1, out_f))
        else:
            self.mb, self.Sb = torch.zeros(1, out_f), torch.zeros(1, out_f)

    def forward(self, ma, Sa):
        self._shape = ma.shape
        a = ma.reshape(-1, self.in_features)
        s = Sa.reshape(-1, self.in_features)
        self.ma_in = a
        out = (*ma.shape[:-1], self.out_features)
        return (F.mean_forward(a, self.mw, self.mb).reshape(out),
                F.var_forward(a, s, self.mw, self.Sw, self.Sb).reshape(out))

    def backward(self, dmz, dSz):
        dm = dmz.reshape(-1, self.out_features)
        dS = dSz.reshape(-1, self.out_features)
        gmw, gSw = F.weight_grad(self.ma_in, dm, dS)
        self.delta_mw, self.delta_Sw = self.Sw * gmw, self.Sw * self.Sw * gSw
        if self.has_bias:
            self.delta_mb = self.Sb * dm.sum(0, keepdim=True)
            self.delta_Sb = self.Sb * self.Sb * dS.sum(0, keepdim=True)
        da, dSa = F.backward_delta(dm, dS, self.mw)
        shp = (*self._shape[:-1], self.in_features)
        return da.reshape(shp), dSa.reshape(shp)

    def update(self, cap):
        self.mw, self.Sw = F.capped_update(self.mw, self.Sw, self.delta_mw, self.delta_Sw, cap)
        if self.has_bias:
            self.mb, self.Sb = F.capped_update(self.mb, self.Sb, self.delta_mb, self.delta_Sb, cap)


class Conv2D(Layer):
    """triton_tagi/layers/conv2d.py:189-390."""

    learnable = True

    def __init__(self, C_in, C_out, kernel_size, stride=1, padding=0, padding_type=1,
                 device="cpu", init_method="He", gain_w=1.0, gain_b=1.0):
        k = kernel_size
        self.C_in, self.C_out, self.k = C_in, C_out, k
        self.stride, self.padding, self.padding_type = stride, padding, padding_type
        s = _scale(init_method, k * k * C_in, k * k * C_out)
        self.mw, self.Sw = _gauss(s, gain_w, (C_in * k * k, C_out))
        self.mb, self.Sb = _gauss(s, gain_b, (1, C_out))
        # True adjoint col2im instead of the reference's gather (differs only
        # for stride > 1; see oracle.moments.col2im).
        self.col2im_adjoint = False

    def forward(self, ma, Sa):
        self.input_shape = tuple(ma.shape)
        mz, Sz, self.patches_ma = F.conv_forward(ma, Sa, self.mw, self.Sw, self.mb, self.Sb,
                                                 self.k, self.stride, self.padding,
                                                 self.padding_type)
        return mz, Sz

    def backward(self, dmz, dSz):
        d_ma, d_Sa, gmw, gSw, gmb, gSb = F.conv_backward(
            dmz, dSz, self.patches_ma, self.mw, self.input_shape, self.k, self.stride,
            self.padding, self.padding_type, self.col2im_adjoint)
        self.delta_mw, self.delta_Sw = self.Sw * gmw, self.Sw * self.Sw * gSw
        self.delta_mb, self.delta_Sb = self.Sb * gmb, self.Sb * self.Sb * gSb
        return d_ma, d_Sa

    def update(self, cap):
        self.mw, self.Sw = F.capped_update(self.mw, self.Sw, self.delta_mw, self.delta_Sw, cap)
        self.mb, self.Sb = F.capped_update(self.mb, self.Sb, self.delta_mb, self.delta_Sb, cap)


class BatchNorm2D(Layer):
    """triton_tagi/layers/batchnorm2d.py:238-538 (training mode uses batch stats)."""

    learnable = True

    def __init__(self, num_features, momentum=0.1, eps=1e-5, device="cpu", gain_w=1.0,
                 gain_b=1.0, preserve_var=True):
        C = num_features
        self.num_features, self.momentum, self.eps = C, momentum, eps
        self.preserve_var, self.training, self._init = preserve_var, True, False
        scale = 2.0 / (C + C)
        self.mw, self.Sw = torch.ones(C), torch.full((C,), scale * gain_w**2)
        self.mb, self.Sb = torch.zeros(C), torch.full((C,), scale * gain_b**2)
        self.running_mean, self.running_var = torch.zeros(C), torch.ones(C)

    def forward(self, mz, Sz):
        if self.training:
            mean, var = F.bn_batch_stats(mz, Sz)
            if not self._init:  # batchnorm2d.py:346-351
                self.running_mean, self.running_var = mean.clone(), var.clone()
                if self.preserve_var:
                    self.mw = torch.sqrt(self.running_var + self.eps)
                self._init = True
            else:  # batchnorm2d.py:352-355
                a = self.momentum
                self.running_mean = (1 - a) * self.running_mean + a * mean
                self.running_var = (1 - a) * self.running_var + a * var
        else:
            mean, var = self.running_mean, self.running_var
        self._norm_var = var
        ma, Sa, self.m_hat, _ = F.bn_forward(mz, Sz, mean, var, self.mw, self.Sw, self.mb,
                                             self.Sb, self.eps)
        return ma, Sa

    def backward(self, dma, dSa):
        dmz, dSz, gmg, gSg, gmb, gSb = F.bn_backward(dma, dSa, self.m_hat, self._norm_var,
                                                     self.mw, self.eps)
        self.delta_mw, self.delta_Sw = self.Sw * gmg, self.Sw * self.Sw * gSg
        self.delta_mb, self.delta_Sb = self.Sb * gmb, self.Sb * self.Sb * gSb
        return dmz, dSz

    def update(self, cap):
        self.mw, self.Sw = F.capped_update(self.mw, self.Sw, self.delta_mw, self.delta_Sw, cap)
        self.mb, self.Sb = F.capped_update(self.mb, self.Sb, self.delta_mb, self.delta_Sb, cap)


class ReLU(Layer):
    """triton_tagi/layers/relu.py:125-169."""

    def forward(self, mz, Sz):
        ma, Sa, self.J = F.relu_moments(mz, Sz)
        return ma, Sa

    def backward(self, dm, dS):
        return dm * self.J, dS * self.J * self.J


class Remax(Layer):
    """triton_tagi/layers/remax.py:167-191."""

    def forward(self, mz, Sz):
        ma, Sa, self.J = F.remax(mz, Sz)
        return ma, Sa

    def backward(self, dm, dS):
        return dm * self.J, dS * self.J * self.J


class AvgPool2D(Layer):
    """triton_tagi/layers/avgpool2d.py:138-243."""

    def __init__(self, kernel_size, spatial_correlation=False):
        self.k, self.sc = kernel_size, spatial_correlation

    def forward(self, ma, Sa):
        self.input_shape = tuple(ma.shape)
        return F.avgpool_forward(ma, Sa, self.k, self.sc)

    def backward(self, dm, dS):
        return F.avgpool_backward(dm, dS, self.input_shape, self.k, self.sc)


class Flatten(Layer):
    """triton_tagi/layers/flatten.py:17-56."""

    def forward(self, ma, Sa):
        self.shape = ma.shape
        return ma.reshape(ma.shape[0], -1), Sa.reshape(Sa.shape[0], -1)

    def backward(self, dm, dS):
        return dm.reshape(self.shape), dS.reshape(self.shape)


class ResBlock(Layer):
    """triton_tagi/layers/resblock.py:221-472."""

    learnable = True

    def __init__(self, in_channels, out_channels, stride=1, device="cpu", gain_w=1.0,
                 gain_b=1.0):
        cin, cout = in_channels, out_channels
        kw = dict(gain_w=gain_w, gain_b=gain_b)
        self.conv1 = Conv2D(cin, cout, 3, stride, 1, 2 if stride > 1 else 1, **kw)
        self.relu1 = ReLU()
        self.bn1 = BatchNorm2D(cout, preserve_var=False, **kw)
        self.conv2 = Conv2D(cout, cout, 3, 1, 1, 1, **kw)
        self.relu2 = ReLU()
        self.bn2 = BatchNorm2D(cout, preserve_var=False, **kw)
        self.main = [self.conv1, self.relu1, self.bn1, self.conv2, self.relu2, self.bn2]
        self.use_projection = stride != 1 or cin != cout
        self.proj = []
        if self.use_projection:
            self.proj_conv = Conv2D(cin, cout, 2, stride, 0, 1, **kw)
            self.proj_relu, self.proj_bn = ReLU(), BatchNorm2D(cout, preserve_var=False, **kw)
            self.proj = [self.proj_conv, self.proj_relu, self.proj_bn]
        self._learnable = [self.conv1, self.bn1, self.conv2, self.bn2]
        if self.use_projection:
            self._learnable += [self.proj_conv, self.proj_bn]

    def forward(self, m, S):
        xm, xS = m, S
        for layer in self.main:
            m, S = layer.forward(m, S)
        for layer in self.proj:
            xm, xS = layer.forward(xm, xS)
        return m + xm, S + xS

    def backward(self, dm, dS):
        am, aS, bm, bS = dm, dS, dm, dS
        for layer in reversed(self.main):
            am, aS = layer.backward(am, aS)
        for layer in reversed(self.proj):
            bm, bS = layer.backward(bm, bS)
        return am + bm, aS + bS

    def update(self, cap):
        for layer in self._learnable:
            layer.update(cap)


class RMSNorm(Layer):
    """triton_tagi/layers/rms_norm.py:42-150."""

    learnable = True

    def __init__(self, normalized_shape, eps=1e-6, gain_w=1.0, device="cpu"):
        ni = normalized_shape if isinstance(normalized_shape, int) else normalized_shape[0]
        self.ni, self.eps = ni, eps
        self.mw = torch.ones(ni)
        self.Sw = torch.full((ni,), (2.0 / (ni + ni)) * gain_w**2)

    def forward(self, ma, Sa):
        self.ma_in = ma.reshape(-1, self.ni)
        mz, Sz, self.inv_rms = F.rmsnorm_forward(ma, Sa, self.mw, self.Sw, self.eps)
        return mz, Sz

    def backward(self, dmz, dSz):
        dma, dSa, s_mu, s_var = F.rmsnorm_backward(dmz, dSz, self.ma_in, self.inv_rms, self.mw)
        self.delta_mw, self.delta_Sw = s_mu * self.Sw, s_var * self.Sw * self.Sw
        return dma, dSa

    def update(self, cap):
        self.mw, self.Sw = F.capped_update(self.mw, self.Sw, self.delta_mw, self.delta_Sw, cap)


class Embedding(Layer):
    """triton_tagi/layers/embedding.py:39-168 (padding_idx disabled)."""

    learnable = True

    def __init__(self, num_embeddings, embedding_dim, input_size=0, scale=1.0, padding_idx=-1,
                 device="cpu"):
        V, D = num_embeddings, embedding_dim
        if padding_idx >= 0:
            raise NotImplementedError("oracle covers padding_idx=-1 only")
        self.V, self.D = V, D
        self.mw, self.Sw = _gauss(scale, 1.0, (V, D))

    def forward(self, ma, Sa):
        if ma.dim() == 3 and ma.shape[-1] == 1:
            ma = ma.squeeze(-1)
        self.cat = ma.long()
        return self.mw[self.cat], self.Sw[self.cat]

    def backward(self, dm, dS):
        idx = self.cat.reshape(-1)
        rows = self.Sw[idx]
        dmw = torch.zeros_like(self.mw).index_add_(0, idx, dm.reshape(-1, self.D) * rows)
        dSw = torch.zeros_like(self.Sw).index_add_(0, idx, dS.reshape(-1, self.D) * rows * rows)
        self.delta_mw, self.delta_Sw = dmw, dSw
        z = torch.zeros(self.cat.shape, dtype=dm.dtype)
        return z, z.clone()

    def update(self, cap):
        self.mw, self.Sw = F.capped_update(self.mw, self.Sw, self.delta_mw, self.delta_Sw, cap)


class PositionalEncoding(Layer):
    """triton_tagi/layers/positional_encoding.py:23-71."""

    def __init__(self, embed_dim, max_seq_len=2048, device="cpu"):
        self.pe = F.positional_encoding(max_seq_len, embed_dim)

    def forward(self, ma, Sa):
        return ma + self.pe[: ma.shape[-2]], Sa

    def backward(self, dm, dS):
        return dm, dS


class MultiheadAttentionV2(Layer):
    """triton_tagi/layers/multihead_attention.py:64-294 (no bias, no mask, H_kv = H)."""

    learnable = True

    def __init__(self, embed_dim, num_heads, seq_len, num_kv_heads=None, bias=False,
                 gain_weight=1.0, gain_bias=1.0, init_method="He", pos_emb="",
                 use_causal_mask=False, device="cpu"):
        E, H = embed_dim, num_heads
        self.E, self.H, self.D = E, H, E // H
        kw = dict(init_method=init_method, gain_w=gain_weight, gain_b=gain_bias, bias=bias)
        self.q_proj = Linear(E, E, **kw)
        self.k_proj = Linear(E, E, **kw)
        self.v_proj = Linear(E, E, **kw)
        self.scale = 1.0 / math.sqrt(self.D)

    def forward(self, ma, Sa):
        B, S, E = ma.shape
        H, D, s = self.H, self.D, self.scale
        heads = lambda t: t.reshape(B, S, H, D).transpose(1, 2)  # noqa: E731
        mq, Sq = map(heads, self.q_proj.forward(ma, Sa))
        mk, Sk = map(heads, self.k_proj.forward(ma, Sa))
        mv, Sv = map(heads, self.v_proj.forward(ma, Sa))
        mqk = s * (mq @ mk.transpose(-1, -2))
        Sqk = F.bmm_tagi_var(mq, Sq, mk.transpose(-1, -2), Sk.transpose(-1, -2), s * s)
        msc, Ssc, jcb = F.remax(mqk, Sqk)
        msv = msc @ mv
        Ssv = F.bmm_tagi_var(msc, Ssc, mv, Sv, 1.0)
        self.cache = (B, S, mq, mk, mv, msc, jcb)
        back = lambda t: t.transpose(1, 2).reshape(B, S, E)  # noqa: E731
        return back(msv), back(Ssv)

    def backward(self, dmz, dSz):
        B, S, mq, mk, mv, msc, jcb = self.cache
        H, D, s = self.H, self.D, self.scale
        heads = lambda t: t.reshape(B, S, H, D).transpose(1, 2)  # noqa: E731
        dm, dS = heads(dmz), heads(dSz)
        dmv, dSv = F.bmm_shared_left(msc.transpose(-1, -2), dm, dS)
        dmsc, dSsc = F.bmm_shared_right(dm, dS, mv.transpose(-1, -2))
        sm, sv = dmsc * jcb, dSsc * jcb * jcb
        dmq, dSq = F.bmm_shared_right(sm, sv, mk, s)
        dmk, dSk = F.bmm_shared_right(sm.transpose(-1, -2), sv.transpose(-1, -2), mq, s)
        back = lambda t: t.transpose(1, 2).reshape(B, S, H * D)  # noqa: E731
        a = self.q_proj.backward(back(dmq), back(dSq))
        b = self.k_proj.backward(back(dmk), back(dSk))
        c = self.v_proj.backward(back(dmv), back(dSv))
        return a[0] + b[0] + c[0], a[1] + b[1] + c[1]

    def update(self, cap):
        for p in (self.q_proj, self.k_proj, self.v_proj):
            p.update(cap)


class Sequential:
    """triton_tagi/network.py:40-152 (``forward`` and dense ``step``)."""

    def __init__(self, layers, device="cpu"):
        self.layers = layers

    def forward(self, x):
        m, S = x, torch.zeros_like(x)
        for layer in self.layers:
            m, S = layer.forward(m, S)
        return m, S

    def step(self, x, y, sigma_v):
        mu, var = self.forward(x)
        dm, dS = F.innovation(y, mu, var, sigma_v)
        for layer in reversed(self.layers):
            dm, dS = layer.backward(dm, dS)
        cap = F.get_cap_factor(x.shape[0])
        for layer in self.layers:
            if layer.learnable:
                layer.update(cap)
        return mu, var
