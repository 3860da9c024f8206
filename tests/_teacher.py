"""Teacher-forced per-layer parity of one ``Sequential.step``.

The device network runs its step as usual (fused update, the container
fusions, the same split plans as the benchmark). Every leaf layer's forward
and backward is wrapped: when the device layer returns, the oracle layer (in
float32, the reference's arithmetic, and in float64) is called on exactly the
inputs the device layer received, copied to the host, and the two outputs are
compared at once. After the step the oracle layers apply their updates from the
same pre-step parameters and the parameters are compared. So each row of the
report is one layer of one step with no error carried in from the layers
before it.

Leaves: every top-level layer, except that a ``ResBlock`` is entered (its main
and shortcut layers are leaves, and its merged input deltas are checked as a
row of their own). ``MultiheadAttentionV2`` is one leaf (its three projections
are checked through their parameters). A BatchNorm2D that applies the
preceding ReLU's Jacobian in its backward is compared with the oracle's
BatchNorm backward followed by that ReLU's backward.

Bars (``_tol``): means normwise ≤ ``mean_tol``; variances and variance deltas
element-wise ≤ ``var_tol`` relative (with the reference's own float32 error as
the allowance where that is larger, see ``elem_check``); updated variances
element-wise relative to the pre-update variance (``var_update_err``).
"""

from __future__ import annotations

import torch

from _nets import load, params, sync_bn_state
from _tol import elem_check, floor_flips, norm_check, var_update_err


def _branches(blk):
    """(main layers, shortcut layers) of a residual block (this library's
    ResBlock or the oracle's), or None for any other layer."""
    if hasattr(blk, "_main_layers"):
        return blk._main_layers, blk._proj_layers
    if hasattr(blk, "main") and hasattr(blk, "proj"):
        return blk.main, blk.proj
    return None


def _leaf_triples(dev, r32, r64, prefix=""):
    for i, (d, a, b) in enumerate(zip(dev, r32, r64)):
        name = f"{prefix}{i}.{type(d).__name__}"
        if _branches(d) is not None:
            (dm, dp), (am, ap), (bm, bp) = _branches(d), _branches(a), _branches(b)
            yield from _leaf_triples(dm, am, bm, name + ".main")
            yield from _leaf_triples(dp, ap, bp, name + ".proj")
        else:
            yield name, d, a, b


def _param_triples(name, d, a, b):
    if hasattr(d, "q_proj"):
        for p in ("q_proj", "k_proj", "v_proj"):
            yield f"{name}.{p}", getattr(d, p), getattr(a, p), getattr(b, p)
    elif getattr(d, "mw", None) is not None and _branches(d) is None:
        yield name, d, a, b


def _host(t, dtype):
    return t.detach().to("cpu", dtype)


class Report:
    def __init__(self, what):
        self.what, self.rows = what, []
        self.flips = self.nvar = 0  # updated variances that hit the floor on one side only

    def add(self, layer, qty, kind, worst, extra, plain):
        self.rows.append((layer, qty, kind, worst, extra, plain))

    def failures(self):
        return [r for r in self.rows if not r[3] <= 1.0]

    def text(self):
        lines = [f"teacher-forced parity, {self.what}: {len(self.rows)} checks",
                 f"{'layer':34s} {'quantity':12s} {'check':6s} {'worst/bar':>9s} "
                 f"{'rel err vs f32':>14s}  note"]
        for layer, qty, kind, worst, extra, plain in self.rows:
            lines.append(f"{layer:34s} {qty:12s} {kind:6s} {worst:9.3f} {plain:14.3e}  {extra}")
        return "\n".join(lines)


def teacher_forced_step(net, ref32, ref64, x, y, sigma_v, mean_tol=1e-5, var_tol=1e-4,
                        what="step"):
    """One ``net.step(x, y, sigma_v)`` with per-layer checks; returns a Report.

    ``ref32`` / ``ref64``: oracle layer lists of the same topology; their
    parameters (and BatchNorm state) are set from the device network first."""
    from oracle import moments as F

    dev_layers = net.layers
    load(ref32, [t.detach().cpu().numpy() for t in params(dev_layers)])
    load(ref64, [t.detach().cpu().numpy() for t in params(dev_layers)], dtype=torch.float64)
    sync_bn_state(dev_layers, ref32)
    sync_bn_state(dev_layers, ref64)
    rep = Report(what)
    triples = list(_leaf_triples(dev_layers, ref32, ref64))
    by_id = {id(d): (a, b) for _, d, a, b in triples}
    prev = {}
    for name, d, a, b in triples:
        for pname, pd, pa, pb in _param_triples(name, d, a, b):
            prev[pname] = {n: _host(getattr(pd, n), torch.float64)
                           for n in ("Sw", "Sb") if getattr(pd, n, None) is not None}

    def compare(layer, phase, got, r32, r64):
        if got is None or got[0] is None:
            return
        w, fb, plain = norm_check(got[0], r32[0], r64[0], mean_tol)
        rep.add(layer, f"{phase} mean", "norm", w, "f64 allowance" if fb else "", plain)
        w, nfb, plain = elem_check(got[1], r32[1], r64[1], var_tol)
        rep.add(layer, f"{phase} var", "elem", w,
                f"{nfb} elem on f64 allowance" if nfb else "", plain)

    originals = []

    def wrap(name, d, a, b):
        f0, b0 = d.forward, d.backward

        def fwd(ma, Sa, **kw):
            out = f0(ma, Sa, **kw)
            o32 = a.forward(_host(ma, torch.float32), _host(Sa, torch.float32))
            o64 = b.forward(_host(ma, torch.float64), _host(Sa, torch.float64))
            res = kw.get("residual")
            if res is not None:
                o32 = (o32[0] + _host(res[0], torch.float32), o32[1] + _host(res[1], torch.float32))
                o64 = (o64[0] + _host(res[0], torch.float64), o64[1] + _host(res[1], torch.float64))
            compare(name, "fwd", out, o32, o64)
            return out

        def bwd(dm, dS, **kw):
            out = b0(dm, dS, **kw)
            o32 = a.backward(_host(dm, torch.float32), _host(dS, torch.float32))
            o64 = b.backward(_host(dm, torch.float64), _host(dS, torch.float64))
            relu = kw.get("relu")
            if relu is not None:  # BatchNorm applying the preceding ReLU's Jacobian
                ra, rb = by_id[id(relu)]
                o32, o64 = ra.backward(*o32), rb.backward(*o64)
            compare(name + ("+ReLU" if relu is not None else ""), "bwd", out, o32, o64)
            d._tf_bwd = (o32, o64)
            return out

        d.forward, d.backward = fwd, bwd
        originals.append(d)

    def wrap_block(name, blk):
        b0 = blk.backward

        def bwd(dm, dS):
            out = b0(dm, dS)
            main, proj = _branches(blk)
            m32, m64 = main[0]._tf_bwd
            if proj:
                s32, s64 = proj[0]._tf_bwd
            else:
                s32 = (_host(dm, torch.float32), _host(dS, torch.float32))
                s64 = (_host(dm, torch.float64), _host(dS, torch.float64))
            compare(name + ".merge", "bwd", out, (m32[0] + s32[0], m32[1] + s32[1]),
                    (m64[0] + s64[0], m64[1] + s64[1]))
            return out

        blk.backward = bwd
        originals.append(blk)

    for name, d, a, b in triples:
        wrap(name, d, a, b)
    for i, layer in enumerate(dev_layers):
        if _branches(layer) is not None:
            wrap_block(f"{i}.{type(layer).__name__}", layer)
    try:
        net.step(x, y, sigma_v)
        if torch.cuda.is_available():
            torch.cuda.synchronize()
    finally:
        for o in originals:
            for attr in ("forward", "backward", "_tf_bwd"):
                o.__dict__.pop(attr, None)

    cap = F.get_cap_factor(x.shape[0])
    for ref in (ref32, ref64):
        for layer in ref:
            if getattr(layer, "learnable", False):
                layer.update(cap)
    for name, d, a, b in triples:
        for pname, pd, pa, pb in _param_triples(name, d, a, b):
            for n in ("mw", "mb", "running_mean"):
                if getattr(pd, n, None) is not None:
                    w, fb, plain = norm_check(getattr(pd, n), getattr(pa, n), getattr(pb, n),
                                              mean_tol)
                    rep.add(pname, n, "norm", w, "f64 allowance" if fb else "", plain)
            for n in ("Sw", "Sb"):
                if getattr(pd, n, None) is None:
                    continue
                got, r32 = getattr(pd, n), getattr(pa, n)
                e = var_update_err(got, r32, prev[pname][n])
                flips = floor_flips(got, r32)
                rep.flips += flips
                rep.nvar += got.numel()
                rep.add(pname, n, "upd", e / var_tol, f"{flips} floor flips" if flips else "", e)
            if getattr(pd, "running_var", None) is not None:
                w, nfb, plain = elem_check(pd.running_var, pa.running_var, pb.running_var,
                                           var_tol)
                rep.add(pname, "running_var", "elem", w, "", plain)
    return rep


def assert_report(rep, max_flip_frac=1e-4):
    """Print the report (pytest -s / -rP shows it) and fail on any row above its
    bar, or if more than ``max_flip_frac`` of the updated variances reached the
    1e-5 floor on one side only (those elements are excluded from the rows)."""
    print("\n" + rep.text())
    print(f"floor flips: {rep.flips} of {rep.nvar} updated variances")
    bad = rep.failures()
    assert not bad, "\n".join(f"{r[0]} {r[1]}: {r[3]:.3f} of the bar ({r[5]:.3e})" for r in bad)
    assert rep.flips <= max(3, max_flip_frac * rep.nvar), (rep.flips, rep.nvar)
    return max((r[3] for r in rep.rows), default=0.0)
