"""Multi-tensor AdamW and squared-norm kernels (csrc/optim.cu) vs the fp32 PyTorch update."""

import pytest
import torch

from cq_pretrain_b200.ops import _ext

pytestmark = pytest.mark.gpu


def _reference(p, g, m, v, decay, gs, lr, b1, b2, eps, wd, bc1, bc2):
    g = g * gs
    m = m * b1 + (1 - b1) * g
    v = v * b2 + (1 - b2) * g * g
    update = (m / bc1) / ((v / bc2).sqrt() + eps)
    p = p * (1 - lr * wd * decay.float()) - lr * update
    return p, m, v


def test_adamw_multi_tensor_matches_reference():
    assert _ext.has("adamw_step")
    torch.manual_seed(0)
    sizes = [1, 3, 4096, 16384, 16385, 100_003]
    base = torch.randn(sum(sizes) + 1, device="cuda")
    masters, grads, ms, vs, decays, outs = [], [], [], [], [], []
    offset = 1  # the grads are views at an odd offset: exercises the unaligned (scalar) path
    for i, n in enumerate(sizes):
        masters.append(torch.randn(n, device="cuda"))
        grads.append(base[offset:offset + n] if i % 2 else torch.randn(n, device="cuda"))
        offset += n
        ms.append(torch.randn(n, device="cuda") * 0.1)
        vs.append(torch.rand(n, device="cuda") * 0.01)
        decays.append((torch.rand(n, device="cuda") < 0.5).to(torch.uint8))
        outs.append(torch.empty(n, device="cuda", dtype=torch.bfloat16 if i % 3 else torch.float32))
    args = dict(lr=1e-3, b1=0.9, b2=0.95, eps=1e-8, wd=0.1, bc1=1 - 0.9 ** 3, bc2=1 - 0.95 ** 3)
    gs = torch.tensor(0.7, device="cuda")
    expect = [_reference(p.clone(), g, m.clone(), v.clone(), d, 0.7, **args)
              for p, g, m, v, d in zip(masters, grads, ms, vs, decays)]
    for _ in range(2):  # second call hits the cached descriptor table
        ps_ = [p.clone() for p in masters]
        ms_ = [m.clone() for m in ms]
        vs_ = [v.clone() for v in vs]
        _ext.ops().adamw_step(ps_, grads, ms_, vs_, decays, outs, gs, *args.values())
        for (p, m, v), pk, mk, vk, out in zip(expect, ps_, ms_, vs_, outs):
            torch.testing.assert_close(pk, p, rtol=1e-5, atol=1e-6)
            torch.testing.assert_close(mk, m, rtol=1e-5, atol=1e-7)
            torch.testing.assert_close(vk, v, rtol=1e-5, atol=1e-8)
            assert torch.equal(out, pk.to(out.dtype))  # the published parameter is the new master


def test_sum_squares_multi_tensor():
    torch.manual_seed(1)
    xs = [torch.randn(n, device="cuda") for n in (5, 16384, 70_001)]
    base = torch.randn(1001, device="cuda")
    xs.append(base[1:])
    got = _ext.ops().sum_squares(xs)
    want = sum(x.double().square().sum() for x in xs)
    assert abs(got.item() - want.item()) < 1e-4 * want.item()
    again = _ext.ops().sum_squares(xs)
    assert got.item() == again.item()  # fixed reduction order


def test_adamw_fused_ema_matches_lerp():
    """EMA shadows lerped inside the AdamW pass equal a separate lerp toward the updated masters;
    tensors without a shadow (empty entry) are untouched, unaligned slices take the scalar path."""
    torch.manual_seed(2)
    sizes = [7, 4096, 10_001]
    masters = [torch.randn(n, device="cuda") for n in sizes]
    grads = [torch.randn(n, device="cuda") for n in sizes]
    ms = [torch.randn(n, device="cuda") * 0.1 for n in sizes]
    vs = [torch.rand(n, device="cuda") * 0.01 for n in sizes]
    decays = [torch.ones(n, device="cuda", dtype=torch.uint8) for n in sizes]
    outs = [torch.empty(n, device="cuda", dtype=torch.bfloat16) for n in sizes]
    store = torch.randn(sum(sizes) + 1, device="cuda")
    shadows = [store[1:8].clone(), torch.empty(0, device="cuda"), store[9:9 + 10_001]]   # unaligned view
    before = [s.clone() for s in shadows]
    args = dict(lr=1e-3, b1=0.9, b2=0.95, eps=1e-8, wd=0.1, bc1=0.1, bc2=0.05)
    expect = [_reference(p.clone(), g, m.clone(), v.clone(), d, 1.0, **args)[0]
              for p, g, m, v, d in zip(masters, grads, ms, vs, decays)]
    _ext.ops().adamw_step(masters, grads, ms, vs, decays, outs, torch.tensor(1.0, device="cuda"), *args.values(),
                          shadows, 0.25)
    for p_new, shadow, old in zip(expect, shadows, before):
        if shadow.numel():
            torch.testing.assert_close(shadow, old + 0.25 * (p_new - old), rtol=1e-5, atol=1e-6)
