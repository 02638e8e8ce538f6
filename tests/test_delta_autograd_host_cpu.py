"""Host logic of the delta rule's autograd path, on a machine without a GPU.

The C ABI is replaced by a fake that computes with the oracle: `fo_gdr_fwd`
writes the oracle's forward into the output tensors and `fo_gdr_bwd` writes
oracle.delta_rule_backward's gradients into the gradient tensors.  What is
checked is everything around the kernels: which tensors reach the entry points
(None for an unused final-state gradient or an initial state that needs none),
that autograd routes each gradient to its input (dtype casts of g and of the
initial state included), partial requires_grad, and that nothing is saved when
no gradient is needed.  The kernels themselves are checked on the GPU.
"""
import pytest
import torch

import oracle
from operators import _lib
import operators.chunk_gated_delta_rule as gdr

NAMES = ("q", "k", "v", "beta", "g")


@pytest.fixture()
def fake_abi(monkeypatch):
    calls = []

    def call(name, *args):
        calls.append((name, args))
        if name in ("fo_gdr_workspace_bytes", "fo_gdr_bwd_workspace_bytes"):
            args[-1]._obj.value = 0
        elif name == "fo_gdr_fwd":
            q, k, v, beta, g, h0, o, hT = args[:8]
            res = oracle.delta_rule_forward(q, k, v, beta, g, initial_state=h0,
                                            output_final_state=True)
            o.copy_(res[0])
            if hT is not None:
                hT.copy_(res[1])
        elif name == "fo_gdr_bwd":
            q, k, v, beta, g, h0, do, dhT, dq, dk, dv, dbeta, dg, dh0 = args[:14]
            res = oracle.delta_rule_backward(q, k, v, beta, g, do, h0, dhT)
            for out, key in ((dq, "q"), (dk, "k"), (dv, "v"), (dbeta, "beta"), (dg, "g")):
                out.copy_(res[key])
            if dh0 is not None:
                dh0.copy_(res["initial_state"])
        else:
            raise AssertionError(f"unexpected entry point {name}")

    monkeypatch.setattr(_lib, "call", call)
    monkeypatch.setattr(_lib, "ptr", lambda t: t)  # the fake receives the tensors themselves
    monkeypatch.setattr(_lib, "stream_of", lambda t: None)
    monkeypatch.setattr(_lib, "require_cuda", lambda t, op: None)
    return calls


def _inputs(B=1, H=2, L=9, D=16, dtype=torch.float32, gate_dtype=None, seed=0):
    gen = torch.Generator().manual_seed(seed)
    q, k, v = (torch.randn(B, H, L, D, generator=gen) for _ in range(3))
    k = k / k.norm(dim=-1, keepdim=True)
    beta = torch.sigmoid(torch.randn(B, H, L, generator=gen))
    g = torch.sigmoid(torch.randn(B, H, L, generator=gen))
    gd = gate_dtype or dtype
    return [q.to(dtype), k.to(dtype), v.to(dtype), beta.to(gd), g.to(gd)], gen


def _bwd(name, calls):
    return [a for n, a in calls if n == name]


def test_gradients_reach_every_input(fake_abi):
    ins, gen = _inputs()
    h0 = 0.1 * torch.randn(1, 2, 16, 16, generator=gen)
    leaves = [t.clone().requires_grad_() for t in ins]
    h0l = h0.clone().requires_grad_()
    o, hT = gdr.chunk_gated_delta_rule(*leaves, initial_state=h0l, output_final_state=True)
    do = torch.randn(o.shape, generator=gen)
    dhT = torch.randn(hT.shape, generator=gen)
    ((o * do).sum() + (hT * dhT).sum()).backward()
    ref = oracle.delta_rule_grads(*ins, do, h0, dhT)
    for name, leaf in zip(NAMES, leaves):
        torch.testing.assert_close(leaf.grad, ref[name], rtol=1e-4, atol=1e-5)
    torch.testing.assert_close(h0l.grad, ref["initial_state"], rtol=1e-4, atol=1e-5)
    (args,) = _bwd("fo_gdr_bwd", fake_abi)
    assert args[5] is not None and args[7] is not None and args[13] is not None


def test_unused_final_state_and_constant_initial_state(fake_abi):
    ins, gen = _inputs(seed=1)
    h0 = 0.1 * torch.randn(1, 2, 16, 16, generator=gen)  # no gradient wanted
    leaves = [t.clone().requires_grad_() for t in ins]
    o, hT = gdr.chunk_gated_delta_rule(*leaves, initial_state=h0, output_final_state=True)
    do = torch.randn(o.shape, generator=gen)
    (o * do).sum().backward()  # the final state is not used
    ref = oracle.delta_rule_grads(*ins, do, h0, None)
    for name, leaf in zip(NAMES, leaves):
        torch.testing.assert_close(leaf.grad, ref[name], rtol=1e-4, atol=1e-5)
    (args,) = _bwd("fo_gdr_bwd", fake_abi)
    assert args[5] is not None  # the forward's initial state is passed
    assert args[7] is None      # no final-state gradient
    assert args[13] is None     # no initial-state gradient computed


def test_only_final_state_used(fake_abi):
    ins, gen = _inputs(seed=2)
    leaves = [t.clone().requires_grad_() for t in ins]
    o, hT = gdr.chunk_gated_delta_rule(*leaves, output_final_state=True)
    dhT = torch.randn(hT.shape, generator=gen)
    (hT * dhT).sum().backward()  # o is not used: its gradient is zero
    ref = oracle.delta_rule_grads(*ins, torch.zeros_like(ins[0]), None, dhT)
    for name, leaf in zip(NAMES, leaves):
        torch.testing.assert_close(leaf.grad, ref[name], rtol=1e-4, atol=1e-5)


def test_gate_dtype_cast_routes_back(fake_abi):
    # g in float64 is cast to beta's float32 for the kernels; its gradient comes
    # back as float64
    ins, gen = _inputs(seed=3)
    ins[4] = ins[4].double()
    leaves = [t.clone().requires_grad_() for t in ins]
    o = gdr.chunk_gated_delta_rule(*leaves)
    do = torch.randn(o.shape, generator=gen)
    (o * do).sum().backward()
    assert leaves[4].grad.dtype == torch.float64 and leaves[3].grad.dtype == torch.float32
    ref = oracle.delta_rule_grads(*[t.float() for t in ins], do)
    torch.testing.assert_close(leaves[4].grad.float(), ref["g"], rtol=1e-4, atol=1e-5)


def test_partial_requires_grad(fake_abi):
    ins, gen = _inputs(seed=4)
    v = ins[2].clone().requires_grad_()
    o = gdr.chunk_gated_delta_rule(ins[0], ins[1], v, ins[3], ins[4])
    do = torch.randn(o.shape, generator=gen)
    (o * do).sum().backward()
    torch.testing.assert_close(v.grad, oracle.delta_rule_grads(*ins, do)["v"], rtol=1e-4,
                               atol=1e-5)


def test_no_gradient_needed_takes_the_plain_path(fake_abi):
    ins, _ = _inputs(seed=5)
    o = gdr.chunk_gated_delta_rule(*ins)
    assert o.grad_fn is None
    leaves = [t.clone().requires_grad_() for t in ins]
    with torch.no_grad():
        o = gdr.chunk_gated_delta_rule(*leaves)
    assert o.grad_fn is None
    assert not _bwd("fo_gdr_bwd", fake_abi)


def test_double_backward_raises(fake_abi):
    ins, gen = _inputs(seed=6)
    leaves = [t.clone().requires_grad_() for t in ins]
    o = gdr.chunk_gated_delta_rule(*leaves)
    (gq,) = torch.autograd.grad(o.sum(), leaves[0], create_graph=True)
    with pytest.raises(RuntimeError):
        gq.sum().backward()
