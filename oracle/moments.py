"""Functional CPU restatement of triton-tagi's moment equations (test oracle).

Every function states the reference lines it follows (paths are relative to the
triton-tagi project root). All arithmetic runs in the dtype of the inputs, so
the same code serves as an fp32 CPU baseline and, given float64 tensors, as a
high-precision checker.
"""

from __future__ import annotations

import math

import torch
from torch import Tensor

INV_SQRT_2PI = 0.3989422804014327
INV_SQRT_2 = 0.7071067811865476

# ----------------------------------------------------------------------------
#  Update rules
# ----------------------------------------------------------------------------


def get_cap_factor(batch_size: int) -> float:
    """Cap heuristic — triton_tagi/update/parameters.py:30-50."""
    if batch_size == 1:
        return 0.1
    return 2.0 if batch_size < 256 else 3.0


def capped_update(m: Tensor, S: Tensor, dm: Tensor, dS: Tensor, cap: float):
    """Capped closed-form update — triton_tagi/update/parameters.py:77-96.

    Returns new (m, S); inputs are not modified.
    """
    bound = torch.sqrt(torch.clamp(S, min=1e-10)) / cap
    m_new = m + torch.sign(dm) * torch.minimum(dm.abs(), bound)
    S_raw = S + torch.sign(dS) * torch.minimum(dS.abs(), bound)
    S_new = torch.where(S_raw <= 0, torch.full_like(S_raw, 1e-5), S_raw)
    return m_new, S_new


def innovation(y: Tensor, mu: Tensor, S: Tensor, sigma_v: float):
    """Dense output innovation — triton_tagi/update/observation.py:24-46 (kernel)
    and 119-163 (wrapper; dense branch only)."""
    Sy = S + sigma_v**2
    return (y - mu) / Sy, -1.0 / Sy


# ----------------------------------------------------------------------------
#  Dense moment contractions
# ----------------------------------------------------------------------------


def mean_forward(ma: Tensor, mw: Tensor, mb: Tensor | None) -> Tensor:
    """mz = ma @ mw + mb — triton_tagi/layers/linear.py:99."""
    mz = ma @ mw
    return mz + mb if mb is not None else mz


def var_forward(ma: Tensor, Sa: Tensor, mw: Tensor, Sw: Tensor, Sb: Tensor | None) -> Tensor:
    """Sz = ma²@Sw + Sa@(mw²+Sw) + Sb — triton_tagi/kernels/common.py:138-165."""
    Sz = (ma * ma) @ Sw + Sa @ (mw * mw + Sw)
    return Sz + Sb if Sb is not None else Sz


def backward_delta(dmz: Tensor, dSz: Tensor, mw: Tensor):
    """(dmz @ mwᵀ, dSz @ (mw²)ᵀ) — triton_tagi/kernels/common.py:257-284."""
    return dmz @ mw.T, dSz @ (mw * mw).T


def weight_grad(a: Tensor, dmz: Tensor, dSz: Tensor):
    """(aᵀ @ dmz, (a²)ᵀ @ dSz) — triton_tagi/kernels/common.py:374-407 and
    triton_tagi/layers/linear.py:138-141."""
    return a.T @ dmz, (a * a).T @ dSz


# ----------------------------------------------------------------------------
#  Activations
# ----------------------------------------------------------------------------


def relu_moments(mz: Tensor, Sz: Tensor):
    """Rectified-Gaussian moments and Jacobian — triton_tagi/layers/relu.py:63-86.

    Includes the reference's asymptotic branch Φ(α) ≈ φ(α)/|α| for α < −5.
    The reference's moments jump at α = −5 (by ~α²/2 in the variance), so in a
    float64 evaluation the branch is chosen where the reference's float32 α
    falls (the inputs rounded to float32, α = μ/√S in correctly rounded float32
    arithmetic, emulated in float64): elements within a rounding of the
    threshold then take the reference's branch. Float32 inputs are unaffected
    except that their branch test, too, uses the correctly rounded α.
    """
    Sz_safe = torch.clamp(Sz, min=1e-30)
    sd = torch.sqrt(Sz_safe)
    alpha = mz / sd
    pdf = torch.exp(-0.5 * alpha * alpha) * INV_SQRT_2PI
    sd32 = torch.sqrt(torch.clamp(Sz.float(), min=1e-30).double()).float()
    alpha32 = (mz.float().double() / sd32.double()).float()
    cdf = torch.where(alpha32 < -5.0, pdf / (-alpha), 0.5 * (1.0 + torch.erf(alpha * INV_SQRT_2)))
    mu = sd * pdf + mz * cdf
    var = -mu * mu + 2.0 * mu * mz - mz * sd * pdf + (Sz_safe - mz * mz) * cdf
    return mu, torch.clamp(var, min=0.0), cdf


def remax(mz: Tensor, Sz: Tensor):
    """Row-wise Remax moments and Jacobian — triton_tagi/layers/remax.py:33-114.

    Rows are the leading dims flattened; the class axis is the last one.
    """
    eps = 1e-6
    sd = torch.sqrt(Sz)
    alpha = mz / sd
    pdf = INV_SQRT_2PI * torch.exp(-0.5 * alpha * alpha)
    cdf = 0.5 + 0.5 * torch.erf(alpha * INV_SQRT_2)
    mu_m = torch.clamp(mz * cdf + sd * pdf, min=eps)
    var_m = -mu_m * mu_m + 2.0 * mu_m * mz - mz * sd * pdf + (Sz - mz * mz) * cdf
    var_m = torch.clamp(var_m, min=eps)
    mu_t = torch.clamp(mu_m.sum(-1, keepdim=True), min=eps)
    var_t = torch.clamp(var_m.sum(-1, keepdim=True), min=eps)
    vlog_m = torch.log(1.0 + var_m / (mu_m * mu_m))
    mlog_m = torch.log(mu_m) - 0.5 * vlog_m
    vlog_t = torch.log(1.0 + var_t / (mu_t * mu_t))
    mlog_t = torch.log(mu_t) - 0.5 * vlog_t
    cov_mt = torch.log(1.0 + var_m / (mu_m * mu_t))
    mlog_a = mlog_m - mlog_t
    vlog_a = torch.clamp(vlog_m + vlog_t - 2.0 * cov_mt, min=0.0)
    mu_raw = torch.clamp(torch.exp(mlog_a + 0.5 * vlog_a), min=eps)
    mu_a = mu_raw / torch.clamp(mu_raw.sum(-1, keepdim=True), min=eps)
    var_a = (torch.exp(vlog_a) - 1.0) * mu_a * mu_a
    cov_am = (torch.exp(vlog_m - cov_mt) - 1.0) * mu_a * mu_m
    cov_az = torch.minimum(torch.sqrt(var_a * Sz), cov_am / torch.clamp(cdf, min=eps))
    return mu_a, var_a, cov_az / Sz


# ----------------------------------------------------------------------------
#  Convolution via explicit patches
# ----------------------------------------------------------------------------


def conv_out_hw(H: int, W: int, k: int, stride: int, padding: int, padding_type: int):
    """Output size — triton_tagi/layers/conv2d.py:280-291."""
    if padding_type == 2 and padding > 0:
        return (H + padding - k) // stride + 1, (W + padding - k) // stride + 1
    return (H + 2 * padding - k) // stride + 1, (W + 2 * padding - k) // stride + 1


def _pad_for(x: Tensor, padding: int, padding_type: int) -> tuple[Tensor, int]:
    if padding_type == 2 and padding > 0:
        return torch.nn.functional.pad(x, (0, padding, 0, padding)), 0
    return x, padding


def im2col(x: Tensor, k: int, stride: int, padding: int, padding_type: int = 1) -> Tensor:
    """(N,C,H,W) → patches (N·L, C·k·k), row = (n, oh, ow), col = (c, kh, kw) —
    triton_tagi/layers/conv2d.py:40-77, 140-152, 280-297."""
    xp, p = _pad_for(x, padding, padding_type)
    cols = torch.nn.functional.unfold(xp, k, padding=p, stride=stride)  # (N, K, L)
    return cols.transpose(1, 2).reshape(-1, cols.shape[1])


def _ctrunc_div(a: Tensor, b: int) -> Tensor:
    return torch.div(a, b, rounding_mode="trunc")


def col2im(cols: Tensor, N: int, C: int, H: int, W: int, k: int, stride: int, padding: int,
           padding_type: int = 1, adjoint: bool = False) -> Tensor:
    """Sum patch rows back to (N,C,H,W) — triton_tagi/layers/conv2d.py:85-132,
    155-181, 361-370 (padding_type=2 folds onto the padded extent then crops).

    ``adjoint=False`` (default) restates the reference's gather exactly: for
    every input pixel and kernel tap it forms ``oh_num = h+p-kh`` and
    ``ow_num = w+p-kw``, divides both by the stride with C (truncating)
    semantics, and accepts the tap when ``oh_num % stride == 0`` and both
    quotients are in range (conv2d.py:119-130). The reference never tests
    ``ow_num % stride``, so for stride > 1 it also gathers taps whose column
    offset is not a multiple of the stride. For stride 1 this equals the true
    adjoint of ``im2col``. ``adjoint=True`` returns the true adjoint
    (``F.fold``), which the reference's own stride-1 tests use as ground truth
    (tests/validation/test_conv2d.py:162-185).
    """
    if padding_type == 2 and padding > 0:
        Hp, Wp, p = H + padding, W + padding, 0
    else:
        Hp, Wp, p = H, W, padding
    K = cols.shape[1]
    if adjoint or stride == 1:
        folded = torch.nn.functional.fold(cols.reshape(N, -1, K).transpose(1, 2), (Hp, Wp), k,
                                          padding=p, stride=stride)
        return folded[:, :, :H, :W].contiguous()
    Ho = (Hp + 2 * p - k) // stride + 1
    Wo = (Wp + 2 * p - k) // stride + 1
    c6 = cols.reshape(N, Ho, Wo, C, k, k)
    h = torch.arange(Hp)
    w = torch.arange(Wp)
    out = torch.zeros(N, C, Hp, Wp, dtype=cols.dtype)
    for kh in range(k):
        ohn = h + p - kh
        oh = _ctrunc_div(ohn, stride)
        vh = (torch.fmod(ohn, stride) == 0) & (oh >= 0) & (oh < Ho)
        for kw in range(k):
            ow = _ctrunc_div(w + p - kw, stride)
            vw = (ow >= 0) & (ow < Wo)
            g = c6[:, oh.clamp(0, Ho - 1)][:, :, ow.clamp(0, Wo - 1), :, kh, kw]  # (N,Hp,Wp,C)
            mask = (vh[:, None] & vw[None, :]).to(cols.dtype)
            out += (g * mask[None, :, :, None]).permute(0, 3, 1, 2)
    return out[:, :, :H, :W].contiguous()


def conv_forward(ma, Sa, mw, Sw, mb, Sb, k, stride, padding, padding_type=1):
    """Conv2D forward — triton_tagi/layers/conv2d.py:254-309. Returns
    (mz, Sz, patches_ma) with mz/Sz in NCHW."""
    N, C, H, W = ma.shape
    Ho, Wo = conv_out_hw(H, W, k, stride, padding, padding_type)
    pm = im2col(ma, k, stride, padding, padding_type)
    pS = im2col(Sa, k, stride, padding, padding_type)
    mz = mean_forward(pm, mw, mb)
    Sz = var_forward(pm, pS, mw, Sw, Sb)
    Co = mw.shape[1]
    to_nchw = lambda t: t.view(N, Ho, Wo, Co).permute(0, 3, 1, 2).contiguous()  # noqa: E731
    return to_nchw(mz), to_nchw(Sz), pm


def conv_backward(dmz, dSz, patches_ma, mw, in_shape, k, stride, padding, padding_type=1,
                  adjoint=False):
    """Conv2D backward — triton_tagi/layers/conv2d.py:314-371. Returns
    (d_ma, d_Sa, grad_mw, grad_Sw, grad_mb, grad_Sb) with raw (unscaled) sums.
    ``adjoint`` selects the col2im semantics (see ``col2im``)."""
    N, C, H, W = in_shape
    Co = mw.shape[1]
    dm = dmz.permute(0, 2, 3, 1).reshape(-1, Co)
    dS = dSz.permute(0, 2, 3, 1).reshape(-1, Co)
    gmw, gSw = weight_grad(patches_ma, dm, dS)
    dpm, dpS = backward_delta(dm, dS, mw)
    d_ma = col2im(dpm, N, C, H, W, k, stride, padding, padding_type, adjoint)
    d_Sa = col2im(dpS, N, C, H, W, k, stride, padding, padding_type, adjoint)
    return d_ma, d_Sa, gmw, gSw, dm.sum(0, keepdim=True), dS.sum(0, keepdim=True)


# ----------------------------------------------------------------------------
#  Normalisation, pooling, merges
# ----------------------------------------------------------------------------


def bn_batch_stats(mz: Tensor, Sz: Tensor):
    """Per-channel batch mean and Bessel-corrected variance —
    triton_tagi/layers/batchnorm2d.py:307-339."""
    N, C, H, W = mz.shape
    n = N * H * W
    mean = mz.mean(dim=(0, 2, 3))
    mean_S = Sz.mean(dim=(0, 2, 3))
    mean_sq = (mz * mz).mean(dim=(0, 2, 3))
    return mean, (mean_S + mean_sq - mean * mean) * (n / (n - 1))


def bn_forward(mz, Sz, mean, var, mg, Sg, mb, Sb, eps):
    """Normalise + Gaussian affine — triton_tagi/layers/batchnorm2d.py:59-126.
    Returns (ma, Sa, m_hat, S_hat)."""
    sh = (1, -1, 1, 1)
    inv_std = 1.0 / torch.sqrt(var.view(sh) + eps)
    m_hat = (mz - mean.view(sh)) * inv_std
    S_hat = Sz / (var.view(sh) + eps)
    g, Sgv, bb, Sbv = mg.view(sh), Sg.view(sh), mb.view(sh), Sb.view(sh)
    ma = g * m_hat + bb
    Sa = g * g * S_hat + Sgv * m_hat * m_hat + Sgv * S_hat + Sbv
    return ma, Sa, m_hat, S_hat


def bn_backward(dma, dSa, m_hat, var, mg, eps):
    """Delta propagation and raw γ/β sums — triton_tagi/layers/batchnorm2d.py:
    134-192 (kernel) and 465-482 (sums). Returns (dmz, dSz, g_mg, g_Sg, g_mb, g_Sb)."""
    sh = (1, -1, 1, 1)
    g = mg.view(sh)
    dmz = dma * g / torch.sqrt(var.view(sh) + eps)
    dSz = dSa * g * g / (var.view(sh) + eps)
    red = (0, 2, 3)
    return (dmz, dSz, (dma * m_hat).sum(red), (dSa * m_hat * m_hat).sum(red), dma.sum(red),
            dSa.sum(red))


def avgpool_forward(ma: Tensor, Sa: Tensor, k: int, spatial_correlation: bool = False):
    """triton_tagi/layers/avgpool2d.py:38-84, 170-198 (window k, stride k)."""
    inv_k2 = 1.0 / (k * k)
    var_scale = inv_k2 if spatial_correlation else inv_k2 * inv_k2
    N, C, H, W = ma.shape
    Ho, Wo = H // k, W // k
    win = lambda t: t[:, :, : Ho * k, : Wo * k].reshape(N, C, Ho, k, Wo, k).sum(dim=(3, 5))  # noqa: E731
    return win(ma) * inv_k2, win(Sa) * var_scale


def avgpool_backward(dm: Tensor, dS: Tensor, in_shape, k: int, spatial_correlation: bool = False):
    """triton_tagi/layers/avgpool2d.py:92-130, 200-239.

    Each input pixel receives its window's delta scaled by 1/k² (mean) and the
    forward's variance scale. When H or W is not a multiple of k, pixels past
    the last full window did not enter the forward and receive zero here (the
    reference's flat index would read a neighbouring row for them; every
    configuration this library targets has H, W divisible by k)."""
    inv_k2 = 1.0 / (k * k)
    var_scale = inv_k2 if spatial_correlation else inv_k2 * inv_k2
    N, C, H, W = in_shape
    Ho, Wo = H // k, W // k
    out_m = torch.zeros(N, C, H, W, dtype=dm.dtype)
    out_S = torch.zeros(N, C, H, W, dtype=dS.dtype)
    up = lambda t: t.repeat_interleave(k, dim=2).repeat_interleave(k, dim=3)  # noqa: E731
    out_m[:, :, : Ho * k, : Wo * k] = up(dm) * inv_k2
    out_S[:, :, : Ho * k, : Wo * k] = up(dS) * var_scale
    return out_m, out_S


def rmsnorm_forward(ma: Tensor, Sa: Tensor, mw: Tensor, Sw: Tensor, eps: float):
    """triton_tagi/layers/rms_norm.py:93-110. Rows = all leading dims."""
    ni = mw.shape[-1]
    m2 = ma.reshape(-1, ni)
    S2 = Sa.reshape(-1, ni)
    inv = 1.0 / torch.sqrt((m2 * m2 + S2).mean(dim=1, keepdim=True) + eps)
    mz = inv * m2 * mw
    Sz = inv * inv * (S2 * (mw * mw + Sw) + Sw * m2 * m2)
    return mz.reshape(ma.shape), Sz.reshape(ma.shape), inv


def rmsnorm_backward(dmz: Tensor, dSz: Tensor, ma: Tensor, inv: Tensor, mw: Tensor):
    """triton_tagi/layers/rms_norm.py:115-134. Returns (dma, dSa, sum_mu, sum_var)."""
    ni = mw.shape[-1]
    dm = dmz.reshape(-1, ni)
    dS = dSz.reshape(-1, ni)
    m2 = ma.reshape(-1, ni)
    t = inv * mw
    s_mu = (inv * m2 * dm).sum(0)
    s_var = (inv * inv * m2 * m2 * dS).sum(0)
    return (t * dm).reshape(dmz.shape), (t * t * dS).reshape(dSz.shape), s_mu, s_var


# ----------------------------------------------------------------------------
#  Attention products
# ----------------------------------------------------------------------------


def bmm_tagi_var(mu_a, var_a, mu_b, var_b, scale_sq: float = 1.0) -> Tensor:
    """triton_tagi/kernels/attention.py:66-131, 149-201."""
    return scale_sq * (var_a @ (mu_b * mu_b + var_b) + (mu_a * mu_a) @ var_b)


def bmm_shared_right(a_mean, a_var, b, scale: float = 1.0):
    """triton_tagi/kernels/attention.py:215-283, 286-336."""
    return scale * (a_mean @ b), (scale * scale) * (a_var @ (b * b))


def bmm_shared_left(a, b_mean, b_var, scale: float = 1.0):
    """triton_tagi/kernels/attention.py:339-374."""
    return scale * (a @ b_mean), (scale * scale) * ((a * a) @ b_var)


def positional_encoding(max_seq_len: int, embed_dim: int) -> Tensor:
    """Sinusoidal table — triton_tagi/layers/positional_encoding.py:40-52."""
    d = torch.arange(embed_dim, dtype=torch.float32)
    pos = torch.arange(max_seq_len, dtype=torch.float32)
    ang = pos[:, None] * (1.0 / torch.pow(10000.0, d / embed_dim))[None, :]
    even = (torch.arange(embed_dim) % 2 == 0)[None, :]
    return torch.where(even, torch.sin(ang), torch.cos(ang))


def he_scale(fan_in: float) -> float:
    """triton_tagi/param_init.py:22-37."""
    return math.sqrt(1.0 / fan_in)
