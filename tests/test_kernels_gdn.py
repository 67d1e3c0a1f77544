"""GDN chunk-recurrence kernels vs the float64 chunked/recurrent oracle (forward and gradients)."""

import pytest
import torch

from cq_pretrain_b200.ops import _ext
from cq_pretrain_b200.ops import reference as R
from cq_pretrain_b200.ops.gdn_cuda import gated_delta_cuda

pytestmark = pytest.mark.gpu


def _inputs(E, H, reads=0.3, seed=0):
    torch.manual_seed(seed)
    q = torch.randn(E, H, 128, device="cuda")
    k = torch.randn(E, H, 128, device="cuda")
    v = torch.randn(E, H, 128, device="cuda")
    g = -torch.rand(E, H, device="cuda") * 0.5
    beta = torch.rand(E, H, device="cuda")
    r = torch.rand(E, device="cuda") < reads
    k[r] = 0
    v[r] = 0
    g[r] = 0
    beta[r] = 0
    return q, k, v, g, beta


@pytest.mark.parametrize("bounds", [(0, 64), (0, 200), (0, 37, 300, 301, 520)])
def test_gdn_forward_backward(bounds):
    assert _ext.has("gdn_fwd")
    E, H = bounds[-1], 4
    q, k, v, g, beta = _inputs(E, H)
    args = [t.clone().requires_grad_() for t in (q, k, v, g, beta)]
    out = gated_delta_cuda(args[0].to(torch.bfloat16), args[1].to(torch.bfloat16), args[2].to(torch.bfloat16),
                           args[3], args[4], bounds)
    ref_args = [t.detach().double().requires_grad_() for t in (q, k, v, g, beta)]
    ref = R.chunk_gated_delta(*ref_args, bounds)
    scale = ref.abs().mean().item()
    err = (out.double() - ref).abs().max().item()
    assert err < 0.08 * max(scale, 1e-3) + 2e-2, (err, scale)
    grad = torch.randn_like(ref)
    out.double().backward(grad)
    ref.backward(grad)
    for name, a, b in zip("qkvgb", args, ref_args):
        rel = (a.grad.double() - b.grad).norm() / b.grad.norm().clamp_min(1e-12)
        assert rel < 5e-2, (name, rel.item())
    assert _ext.ops().gdn_status(True) == 0     # no bounded wait of the tcgen05 kernels expired


def test_gdn_prep_matches_factors():
    """Fused chunk-local factors (csrc/gdn_chunk.cu) vs the PyTorch chunk algebra."""
    from cq_pretrain_b200.ops.gdn_cuda import _factors
    assert _ext.has("gdn_prep")
    torch.manual_seed(3)
    Nc, H = 7, 3
    Q = torch.nn.functional.normalize(torch.randn(Nc, H, 64, 128, device="cuda"), dim=-1) * 128 ** -0.5
    K = torch.nn.functional.normalize(torch.randn(Nc, H, 64, 128, device="cuda"), dim=-1)
    V = torch.randn(Nc, H, 64, 128, device="cuda")
    G = -torch.rand(Nc, H, 64, device="cuda") * 0.3
    B = torch.rand(Nc, H, 64, device="cuda")
    K[:, :, 50:] = 0   # padded tail slots of a document's last chunk
    G[:, :, 50:] = 0
    B[:, :, 50:] = 0
    Q, K, V = (t.to(torch.bfloat16).contiguous() for t in (Q, K, V))
    W, U, P, Qd, Kt, gamma = _ext.ops().gdn_prep(Q, K, V, G.contiguous(), B.contiguous())
    f = _factors(Q, K, V, G, B, 64)
    for name, got in (("W", W), ("U", U), ("P", P), ("Qd", Qd), ("Kt", Kt), ("gamma", gamma)):
        want = f[name].float()
        rel = (got.float() - want).norm() / want.norm().clamp_min(1e-12)
        assert rel < 1.5e-2, (name, rel.item())
    assert _ext.ops().gdn_status(True) == 0     # no bounded wait of the tcgen05 kernel expired


@pytest.mark.parametrize("states", ["fp32", "bf16"])
def test_gdn_chunk_backward_matches_reference(states):
    """Fused chunk backward (csrc/gdn_chunk.cu) vs its PyTorch form on random states: fp32 states
    run the mma.sync kernel, bf16 states (with dgamma = <S, dS> given) the tcgen05 kernel."""
    from cq_pretrain_b200.ops.gdn_cuda import chunk_backward_reference
    assert _ext.has("gdn_chunk_bwd")
    torch.manual_seed(4)
    Nc, H = 5, 2
    Q = torch.nn.functional.normalize(torch.randn(Nc, H, 64, 128, device="cuda"), dim=-1) * 128 ** -0.5
    K = torch.nn.functional.normalize(torch.randn(Nc, H, 64, 128, device="cuda"), dim=-1)
    V = torch.randn(Nc, H, 64, 128, device="cuda")
    dO = torch.randn(Nc, H, 64, 128, device="cuda")
    G = -torch.rand(Nc, H, 64, device="cuda") * 0.3
    B = torch.rand(Nc, H, 64, device="cuda")
    K[-1, :, 40:] = 0
    V[-1, :, 40:] = 0
    G[-1, :, 40:] = 0
    B[-1, :, 40:] = 0
    S = torch.randn(Nc, H, 128, 128, device="cuda") * 0.5
    dS = torch.randn(Nc, H, 128, 128, device="cuda") * 0.5
    Q, K, V, dO = (t.to(torch.bfloat16).contiguous() for t in (Q, K, V, dO))
    if states == "bf16":
        S, dS = S.to(torch.bfloat16), dS.to(torch.bfloat16)
        dgamma = (S.float() * dS.float()).sum((-1, -2)).contiguous()
        got = _ext.ops().gdn_chunk_bwd(Q, K, V, dO, G.contiguous(), B.contiguous(), S, dS, dgamma)
        S, dS = S.float(), dS.float()
        assert _ext.ops().gdn_status(True) == 0
    else:
        got = _ext.ops().gdn_chunk_bwd(Q, K, V, dO, G.contiguous(), B.contiguous(), S, dS)
    want = chunk_backward_reference(Q, K, V, dO, G, B, S, dS)
    for name, a, b in zip(("dQ", "dK", "dV", "dG", "dBeta"), got, want):
        rel = (a.float() - b.float()).norm() / b.float().norm().clamp_min(1e-12)
        assert rel < 2e-2, (name, rel.item())


@pytest.mark.parametrize("bounds", [(0, 200), (0, 37, 37, 300, 520)])
def test_gdn_prefill_final_state_from_kernel(bounds):
    """Prefill (K8): outputs and the per-document final state come from the forward recurrence
    kernel; compared with the float64 chunked oracle (an empty document keeps the zero state)."""
    from cq_pretrain_b200.ops import gdn as GDN
    q, k, v, g, beta = _inputs(bounds[-1], 4, seed=3)
    y, state = GDN.prefill(q.to(torch.bfloat16), k.to(torch.bfloat16), v.to(torch.bfloat16), g, beta, bounds)
    ref_y, ref_state = R.chunk_gated_delta(q.double(), k.double(), v.double(), g.double(), beta.double(), bounds,
                                           final=True)
    assert state.dtype == torch.float32 and state.shape == ref_state.shape
    rel = (state.double() - ref_state).norm() / ref_state.norm()
    assert rel < 2e-2, rel.item()
    rel_y = (y.double() - ref_y).norm() / ref_y.norm()
    assert rel_y < 2e-2, rel_y.item()


def test_gdn_decode_step_matches_fp32_reference():
    """Fused recurrent decode step (K7) vs the float64 recurrence, three steps in a row."""
    from cq_pretrain_b200.ops import gdn as GDN
    torch.manual_seed(5)
    H, dk, dv = 16, 128, 128
    state = torch.randn(H, dk, dv, device="cuda") * 0.1
    ref = state.double().clone()
    for _ in range(3):
        q = torch.randn(2, H, dk, device="cuda")
        k = torch.randn(H, dk, device="cuda")
        v = torch.randn(H, dv, device="cuda")
        g = -torch.rand(H, device="cuda")
        beta = torch.rand(H, device="cuda")
        y = GDN.decode_step(state, q, k, v, g, beta)
        qn = R.l2norm(q.double()) * dk ** -0.5
        kn = R.l2norm(k.double())
        ref = ref * g.double().exp()[:, None, None]
        ref = ref + kn[:, :, None] * ((v.double() - torch.einsum("hkv,hk->hv", ref, kn)) * beta.double()[:, None])[:, None, :]
        ref_y = torch.einsum("hkv,bhk->bhv", ref, qn)
        assert (state.double() - ref).abs().max() < 1e-4
        assert (y.double() - ref_y).abs().max() < 1e-4 * max(1.0, ref_y.abs().max().item())
