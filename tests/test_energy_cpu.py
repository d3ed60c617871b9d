"""The energy-network caller on CPU with the oracle attention: its second-order autograd chain matches plain softmax
attention (the reference's verify_second_order check, models/attention.py:89-173), and a training segment with graded
microsteps produces finite gradients."""

from __future__ import annotations

import torch

from ebr_b200.energy import EnergyConfig, EnergyReasoner, rms_norm, train_step_loss
from oracle.torch_attention import oracle_attention


def math_attention(q, k, v):
    """Plain softmax attention, differentiable to any order (the reference's math backend, attention.py:49-54)."""
    s = torch.matmul(q, k.transpose(-1, -2)) * q.shape[-1] ** -0.5
    return torch.matmul(s.softmax(-1), v)


def _model(attention, dtype=torch.float64):
    torch.manual_seed(3)
    cfg = EnergyConfig(board_height=3, board_width=4, vocab_size=6, hidden_size=32, num_heads=2, num_layers=2,
                       forward_dtype=dtype, layers="eager")  # fmt: skip
    return EnergyReasoner(cfg, attention=attention).to(dtype)


def _probe(model, z0, x, u):
    z = z0.clone().requires_grad_(True)
    params = [p for p in model.parameters()]
    with torch.enable_grad():
        e = model.energy(rms_norm(z), x, model.rope)
        (g,) = torch.autograd.grad(e.sum(), z, create_graph=True)
        hz, *ht = torch.autograd.grad((g * u).sum(), [z] + params, allow_unused=True)
    return g.detach(), hz, ht


def test_second_order_matches_math_attention():
    m_or, m_ma = _model(oracle_attention), _model(math_attention)
    m_ma.load_state_dict(m_or.state_dict())
    g = torch.Generator().manual_seed(5)
    tok = torch.randint(0, 6, (2, 12), generator=g)
    x = m_or.input_embeddings(tok).to(torch.float64)
    z0 = torch.randn(2, 12, 32, generator=g, dtype=torch.float64)
    u = torch.randn(2, 12, 32, generator=g, dtype=torch.float64)
    a, b = _probe(m_or, z0, x, u), _probe(m_ma, z0, x, u)
    rel = lambda p, r: float((p - r).abs().max() / r.abs().max().clamp_min(1e-12))
    assert rel(a[0], b[0]) < 1e-10
    assert rel(a[1], b[1]) < 1e-9
    for p, r in zip(a[2], b[2]):
        if r is not None:
            assert p is not None and rel(p, r) < 1e-9


def test_training_segment_gradients_are_finite():
    m = _model(oracle_attention, dtype=torch.float32)
    g = torch.Generator().manual_seed(6)
    tok = torch.randint(0, 6, (3, 12), generator=g)
    labels = torch.randint(0, 6, (3, 12), generator=g)
    x = m.input_embeddings(tok)
    z = m.fresh_states(3, "cpu")
    loss = train_step_loss(m, z, x, labels, prefix=1, graded=2)
    loss.backward()
    grads = [p.grad for p in m.parameters() if p.requires_grad]
    assert all(gr is not None and torch.isfinite(gr).all() for gr in grads)
    # the attention temperature is reached through the graded microsteps' double backward
    assert m.energy.blocks[0].attn.log_logit_scale.grad.abs().sum() > 0
