"""chunk_gated_delta_rule backward (fo_gdr_bwd) against the gradients the
reference defines: torch autograd through its CPU loop (_ref_forward,
chunk_gated_delta_rule.py:286-310), restated as oracle.delta_rule_grads; the
reference itself has no backward kernel.

Tolerance per element: |got - ref| <= rtol |ref| + rtol rms(ref), with
rtol = 2e-4 for fp32 inputs (fp32 arithmetic in another order) and 2e-2 for
bf16/fp16 inputs (gradients rounded to the input dtype; the forward's standard).
"""
import pytest
import torch

import oracle
from operators.chunk_gated_delta_rule import chunk_gated_delta_rule

pytestmark = pytest.mark.gpu
DEV = "cuda"
NAMES = ("q", "k", "v", "beta", "g")


def _make(B, H, L, D, dtype, seed, gate_dtype=None):
    gen = torch.Generator().manual_seed(seed)
    q = torch.randn(B, H, L, D, generator=gen)
    k = torch.randn(B, H, L, D, generator=gen)
    k = k / k.norm(dim=-1, keepdim=True).clamp(min=1e-6)
    v = torch.randn(B, H, L, D, generator=gen)
    beta = torch.sigmoid(torch.randn(B, H, L, generator=gen))
    g = torch.sigmoid(torch.randn(B, H, L, generator=gen))
    do = torch.randn(B, H, L, D, generator=gen)
    gd = gate_dtype or dtype
    return ([q.to(dtype), k.to(dtype), v.to(dtype), beta.to(gd), g.to(gd)], do.to(dtype),
            gen)


def _close(got, ref, rtol):
    got, ref = got.float().cpu(), ref.float().cpu()
    assert got.shape == ref.shape
    if ref.numel() == 0:
        return
    rms = ref.pow(2).mean().sqrt().item()
    err = (got - ref).abs()
    bound = rtol * ref.abs() + rtol * rms
    worst = (err / bound.clamp(min=1e-30)).max().item()
    assert bool((err <= bound).all()), f"max err {err.max().item():.3e} (rms {rms:.3e}, " \
                                       f"worst ratio {worst:.2f})"


def _grads(ins, do, h0=None, dhT=None, want=NAMES):
    leaves = [t.to(DEV).requires_grad_(n in want) for n, t in zip(NAMES, ins)]
    h0l = h0.to(DEV).requires_grad_(True) if h0 is not None else None
    out = chunk_gated_delta_rule(*leaves, initial_state=h0l, output_final_state=dhT is not None)
    if dhT is not None:
        o, hT = out
        loss = (o.float() * do.to(DEV).float()).sum() + (hT * dhT.to(DEV)).sum()
    else:
        loss = (out.float() * do.to(DEV).float()).sum()
    loss.backward()
    res = {n: x.grad for n, x in zip(NAMES, leaves) if n in want}
    if h0l is not None:
        res["initial_state"] = h0l.grad
    return res


@pytest.mark.parametrize("B,H,L,D", [(1, 2, 100, 16), (2, 1, 65, 32), (1, 1, 130, 64),
                                     (1, 2, 70, 128), (1, 1, 5, 128), (1, 1, 32, 64),
                                     (1, 1, 1, 16)])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("state", [False, True])
def test_backward_matches_autograd_of_reference(B, H, L, D, dtype, state):
    ins, do, gen = _make(B, H, L, D, dtype, seed=1000 * B + 10 * L + D)
    h0 = 0.1 * torch.randn(B, H, D, D, generator=gen) if state else None
    dhT = torch.randn(B, H, D, D, generator=gen) if state else None
    got = _grads(ins, do, h0, dhT)
    ref = oracle.delta_rule_grads(*ins, do, h0, dhT)
    rtol = 2e-4 if dtype == torch.float32 else 2e-2
    for name, gr in got.items():
        assert gr.dtype == (ins[NAMES.index(name)].dtype if name in NAMES else torch.float32)
        _close(gr, ref[name], rtol)


def test_backward_fp16_and_mixed_gate_dtypes():
    # fp16 inputs; then bf16 inputs with fp32 beta and bf16 g (g is cast to beta's
    # dtype for the kernels, and its gradient comes back in g's own dtype)
    ins, do, _ = _make(1, 2, 90, 64, torch.float16, seed=11)
    got = _grads(ins, do)
    ref = oracle.delta_rule_grads(*ins, do)
    for name in NAMES:
        _close(got[name], ref[name], 2e-2)
    ins, do, _ = _make(1, 2, 90, 64, torch.bfloat16, seed=12, gate_dtype=torch.float32)
    ins[4] = ins[4].bfloat16()
    got = _grads(ins, do)
    ref = oracle.delta_rule_grads(*ins, do)
    assert got["beta"].dtype == torch.float32 and got["g"].dtype == torch.bfloat16
    for name in NAMES:
        _close(got[name], ref[name], 2e-2)


def test_backward_some_inputs_only():
    ins, do, _ = _make(2, 1, 50, 32, torch.bfloat16, seed=13)
    got = _grads(ins, do, want=("v",))
    assert set(got) == {"v"}
    _close(got["v"], oracle.delta_rule_grads(*ins, do)["v"], 2e-2)


def test_backward_deterministic():
    ins, do, gen = _make(1, 2, 200, 128, torch.bfloat16, seed=14)
    dhT = torch.randn(1, 2, 128, 128, generator=gen)
    a = _grads(ins, do, dhT=dhT)
    b = _grads(ins, do, dhT=dhT)
    for name in NAMES:
        assert torch.equal(a[name], b[name]), name


def test_backward_zero_length():
    ins, do, gen = _make(1, 2, 0, 32, torch.bfloat16, seed=15)
    h0 = torch.randn(1, 2, 32, 32, generator=gen)
    dhT = torch.randn(1, 2, 32, 32, generator=gen)
    got = _grads(ins, do, h0, dhT)
    assert got["q"].shape == (1, 2, 0, 32) and got["beta"].shape == (1, 2, 0)
    torch.testing.assert_close(got["initial_state"].cpu(), dhT)


def test_backward_long_sequence_head_samples():
    # the benchmark's head shape over 1024 tokens, 3 heads: heads 0 and 2 checked
    # against autograd through the reference loop (heads are independent)
    ins, do, gen = _make(1, 3, 1024, 128, torch.bfloat16, seed=16)
    dhT = torch.randn(1, 3, 128, 128, generator=gen)
    got = _grads(ins, do, dhT=dhT)
    for h in (0, 2):
        sl = [t[:, h:h + 1] for t in ins]
        ref = oracle.delta_rule_grads(*sl, do[:, h:h + 1], None, dhT[:, h:h + 1])
        for name in NAMES:
            _close(got[name][:, h:h + 1], ref[name], 2e-2)


def test_backward_launches_the_cuda_kernel():
    from torch.profiler import ProfilerActivity, profile
    ins, do, _ = _make(1, 1, 64, 64, torch.bfloat16, seed=17)
    leaves = [t.to(DEV).requires_grad_() for t in ins]
    o = chunk_gated_delta_rule(*leaves)
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        o.backward(do.to(DEV))
        torch.cuda.synchronize()
    names = " ".join(e.name for e in prof.events())
    assert "gdr_bwd_kernel" in names, names[:400]


def test_no_grad_path_saves_nothing():
    ins, _, _ = _make(1, 1, 16, 16, torch.bfloat16, seed=18)
    leaves = [t.to(DEV).requires_grad_() for t in ins]
    with torch.no_grad():
        o = chunk_gated_delta_rule(*leaves)
    assert o.grad_fn is None
    o = chunk_gated_delta_rule(*[t.to(DEV) for t in ins])
    assert o.grad_fn is None
