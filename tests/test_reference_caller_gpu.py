"""The reference's own callers, unmodified, driving this package's attention ops on a B200.

The reference is the package installed under ``baseline/_ref`` by ``baseline/install_reference.sh`` (the tests skip
when it is absent). Its ``fused`` attention backend is re-pointed at ``ebr_b200.fused_attn.fused_attention`` -- the
one import a maintainer changes (models/attention.py:61-65) -- before any network is built, so the reference's
``models.fused_attn`` package, which registers the same ``ebr_fused::`` op names, is never imported here. Then:

* ``verify_second_order`` (models/attention.py:89-173), the reference's own gate in front of graded microsteps, passes
  for the re-pointed backend: its float32 call as the network makes it (head_dim 16, CUDA-core kernels), and at
  head_dim 64 on the tensor-core kernels (N = 81 packed, N = 300 tiled) in float32 and bf16;
* ``EnergyDescent.forward`` (models/energy.py:285-319) of the reference's default architecture (config/arch/ebr.yaml:
  2 layers, hidden 256, 4 heads x 64) on a 9 x 9 board: one microstep without a graph and one graded microstep with
  the parameter gradients of a loss on z', against the same network with the ``math`` backend and the same weights;
* ``energy_compile: true`` (models/energy.py:345-384): the reference compiles dE/dz with ``torch.func.grad`` under
  inductor, checks it against eager to second order itself (``_verify_compiled_energy_grad``, raising on a mismatch),
  and the compiled dE/dz agrees with the eager one.
The yardstick is the reference's ``math`` backend (fp32 softmax) in the same bf16 network, with the reference's
norm-relative metric (models/energy.py:416-421); the bars sit at the bf16 network's own noise level.
"""

from __future__ import annotations

import sys
from pathlib import Path

import pytest
import torch

pytestmark = pytest.mark.gpu

REF = Path(__file__).resolve().parents[1] / "baseline" / "_ref"
DEV = "cuda"


@pytest.fixture(scope="module")
def ref():
    if not (REF / "models" / "energy.py").exists():
        pytest.skip("reference not installed (baseline/install_reference.sh)")
    if str(REF) not in sys.path:
        sys.path.insert(0, str(REF))
    import models.attention as ref_attention
    import models.energy as ref_energy

    from ebr_b200.fused_attn import fused_attention

    def ours(q, k, v):
        return fused_attention(q, k, v, scale=q.shape[-1] ** -0.5)

    saved = ref_attention.ATTENTION_BACKENDS["fused"]
    ref_attention.ATTENTION_BACKENDS["fused"] = ref_attention.AttentionBackend("fused", ours, True)
    yield ref_attention, ref_energy
    ref_attention.ATTENTION_BACKENDS["fused"] = saved
    assert "models.fused_attn" not in sys.modules  # the reference's own ops were never registered here


def _norm_rel(a: torch.Tensor, r: torch.Tensor) -> float:
    return float((a.float() - r.float()).norm() / r.float().norm().clamp_min(1e-12))


def _config(ref_energy, backend: str, compiled: bool):
    return ref_energy.EnergyConfig(
        seq_len=81, vocab_size=10, num_layers=2, hidden_size=256, expansion=4.0, num_heads=4, board_height=9,
        board_width=9, forward_dtype="bfloat16", attn_backend=backend, attn_nograd_backend=backend, cycles=16,
        grad_cycles=7, randomize_min_cycles=16, reset_cycles_low=7, reset_cycles_high=16, halt_max_steps=4,
        halt_exploration_prob=0.0, step_size=250.0, step_size_low=200.0, step_size_high=250.0, init_std=1.0,
        noise_scale=0.05, noise_cosine=False, noise_settle_hot=0.4, microstep_ce=0.5, microstep_ce_ramp=1.0,
        convergence_threshold=0.25, convergence_temperature=0.05, convergence_window=2, explore_k=1,
        energy_compile=compiled,
    )  # fmt: skip


def _networks(ref_energy, compiled: bool = False):
    """(math network, fused network) with the same weights."""
    torch.manual_seed(0)
    with torch.device(DEV):
        math_net = ref_energy.InnerNetwork(_config(ref_energy, "math", False))
        ours_net = ref_energy.InnerNetwork(_config(ref_energy, "fused", compiled))
    ours_net.load_state_dict(math_net.state_dict())
    return math_net, ours_net


def _inputs(net, rows: int = 6, seed: int = 5):
    g = torch.Generator().manual_seed(seed)
    tokens = torch.randint(0, 10, (rows, 81), generator=g).to(DEV)
    with torch.no_grad():
        x = net.input_embeddings(tokens)
        z = net.fresh_states((rows, 81, 256), x)
        noise = torch.randn(z.shape, generator=g).to(DEV, z.dtype) * 0.05
    return x, z, noise


@pytest.mark.parametrize("dtype,seq,head_dim", [
    (torch.float32, 32, 16),    # the call EnergyAttention._ensure_verified makes (models/attention.py:201-212)
    (torch.float32, 81, 64),
    (torch.float32, 300, 64),
    (torch.bfloat16, 81, 64),   # packed short-sequence tensor-core kernels
    (torch.bfloat16, 300, 64),  # tiled tensor-core kernels
], ids=str)  # fmt: skip
def test_reference_verify_second_order_passes(ref, dtype, seq, head_dim):
    ref_attention, _ = ref
    backend = ref_attention.get_backend("fused")
    assert backend.fn.__name__ == "ours"
    ref_attention.verify_second_order(backend, device=torch.device(DEV), dtype=dtype, heads=2, seq=seq,
                                      head_dim=head_dim)  # fmt: skip


def test_reference_energy_descent_with_our_ops(ref):
    """One microstep of the reference's EnergyDescent without a graph (dE/dz at v), and one graded microstep
    (train mode: dE/dz with create_graph, then the parameter gradients of a loss on z' through the double backward),
    each against the math backend."""
    _, ref_energy = ref
    math_net, ours_net = _networks(ref_energy)
    x, z, noise = _inputs(math_net)
    cs = math_net.cos_sin()
    for net in (math_net, ours_net):
        net.eval()
    z1 = {}
    with torch.no_grad():
        for name, net in (("math", math_net), ("ours", ours_net)):
            z1[name] = net.level(z, x, cs, noise=noise)
    err_step = _norm_rel(z1["ours"], z1["math"])
    v = math_net.level.normalize_descent_state(z) + noise
    g = {}
    for name, net in (("math", math_net), ("ours", ours_net)):
        with torch.enable_grad():
            g[name] = net.level._energy_gradient(v.detach().requires_grad_(True), x, cs, create_graph=False)
    err_grad = _norm_rel(g["ours"], g["math"])
    print(f"eager microstep: z' norm-rel {err_step:.2e}, dE/dz norm-rel {err_grad:.2e}")
    assert err_grad < 2e-2 and err_step < 2e-2

    grads = {}
    for name, net in (("math", math_net), ("ours", ours_net)):
        net.train()
        net.zero_grad(set_to_none=True)
        alpha = torch.full((z.shape[0], 1, 1), 220.0, device=DEV)
        with torch.enable_grad():
            zn = net.level(z, x, cs, noise=noise, alpha=alpha)
            assert zn.requires_grad
            zn.float().square().mul(torch.linspace(-1, 1, zn.shape[-1], device=DEV)).sum().backward()
        grads[name] = {n: p.grad.detach().clone() for n, p in net.level.energy.named_parameters() if p.grad is not None}
    assert grads["ours"].keys() == grads["math"].keys() and grads["math"]
    errs = {n: _norm_rel(grads["ours"][n], grads["math"][n]) for n in grads["math"]}
    worst = max(errs, key=errs.get)
    print(f"graded microstep: worst parameter-gradient norm-rel {errs[worst]:.2e} ({worst})")
    assert errs[worst] < 5e-2, errs


def test_reference_compiled_energy_grad_with_our_ops(ref):
    """The reference's inductor-compiled torch.func.grad of the energy (energy_compile: true) over our ops: its own
    eager-vs-compiled second-order check passes, and the compiled dE/dz (bf16, graded and not) matches eager."""
    _, ref_energy = ref
    torch._dynamo.reset()
    math_net, ours_net = _networks(ref_energy, compiled=True)
    x, z, noise = _inputs(math_net, rows=4, seed=9)
    cs = ours_net.cos_sin()
    v = (ours_net.level.normalize_descent_state(z) + noise).detach()
    ours_net.train()
    with torch.enable_grad():
        # graded first: runs verify_second_order and _verify_compiled_energy_grad (each raises on a mismatch)
        g_graded = ours_net.level._energy_gradient(v.clone().requires_grad_(True), x, cs, create_graph=True)
    assert ours_net.level._compiled_verified
    ours_net.eval()
    with torch.enable_grad():
        g_plain = ours_net.level._energy_gradient(v.clone().requires_grad_(True), x, cs, create_graph=False)
        g_math = math_net.level._energy_gradient(v.clone().requires_grad_(True), x, cs, create_graph=False)
    e_graded, e_plain = _norm_rel(g_graded, g_math), _norm_rel(g_plain, g_math)
    print(f"compiled dE/dz norm-rel vs math: graded {e_graded:.2e}, not graded {e_plain:.2e}")
    assert e_graded < 2e-2 and e_plain < 2e-2
