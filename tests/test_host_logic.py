"""Host-side behaviour of the drop-in API that needs no GPU."""

from __future__ import annotations

import pytest
import torch

import triton_tagi as tt
from triton_tagi.update.parameters import get_cap_factor


def test_cap_factor_matches_reference_rule():
    assert [get_cap_factor(b) for b in (1, 2, 255, 256, 1024)] == [0.1, 2.0, 2.0, 3.0, 3.0]


def test_layers_construct_on_cpu_with_reference_shapes():
    lin = tt.Linear(5, 3, device="cpu")
    assert lin.mw.shape == (5, 3) and lin.mb.shape == (1, 3)
    assert torch.allclose(lin.Sw, torch.full((5, 3), 1 / 5))
    conv = tt.Conv2D(3, 8, 5, padding=2, device="cpu")
    assert conv.mw.shape == (75, 8) and conv.mb.shape == (1, 8)
    bn = tt.BatchNorm2D(16, device="cpu")
    assert torch.equal(bn.mw, torch.ones(16)) and torch.allclose(bn.Sw, torch.full((16,), 1 / 16))
    rb = tt.ResBlock(8, 16, stride=2, device="cpu")
    assert rb.use_projection and rb.conv1.padding_type == 2 and rb.proj_conv.kH == 2
    assert rb.num_parameters == sum(l.num_parameters for l in rb._learnable)
    mha = tt.MultiheadAttentionV2(32, 4, 8, device="cpu")
    assert mha.head_dim == 8 and not mha.q_proj.has_bias


def test_cpu_tensors_are_rejected_not_computed():
    lin = tt.Linear(4, 3, device="cpu")
    with pytest.raises(ValueError, match="CUDA"):
        lin.forward(torch.zeros(2, 4), torch.zeros(2, 4))
    emb = tt.Embedding(8, 6, device="cpu")
    with pytest.raises(ValueError, match="CUDA"):
        emb.forward(torch.zeros(2, 5), torch.zeros(2, 5))
    pe = tt.PositionalEncoding(6, max_seq_len=16, device="cpu")
    with pytest.raises(ValueError, match="CUDA"):
        pe.forward(torch.zeros(2, 5, 6), torch.zeros(2, 5, 6))


def test_unported_options_raise_like_reference():
    with pytest.raises(NotImplementedError):
        tt.MultiheadAttentionV2(32, 4, 8, pos_emb="rope", device="cpu")
    with pytest.raises(NotImplementedError):
        tt.MultiheadAttentionV2(32, 4, 8, use_causal_mask=True, device="cpu")
    with pytest.raises(ValueError):
        tt.MultiheadAttentionV2(30, 4, 8, device="cpu")
    with pytest.raises(ValueError):
        tt.Conv2D(3, 8, 3, padding_type=3, device="cpu")


def test_param_modes_propagate_to_leaves():
    rb = tt.ResBlock(4, 8, stride=2, device="cpu")
    rb._set_param_mode("update", 2.0)
    assert all(l._param_mode == "update" and l._cap == 2.0 for l in rb._leaves())
    rb._set_param_mode("deltas")
    assert all(l._param_mode == "deltas" for l in rb._leaves())


def test_sequential_repr_and_count():
    net = tt.Sequential([tt.Linear(4, 3, device="cpu"), tt.ReLU(), tt.Linear(3, 2, device="cpu"),
                         tt.Remax()], device="cpu")
    assert net.num_parameters() == 2 * (12 + 3) + 2 * (6 + 2)
    assert "Remax" in repr(net)
