"""fused_cross_entropy parity: sm_100a kernels (C ABI) vs the oracle.

Tolerances: fp32 rtol 1e-5; bf16 rtol 2e-2.  As the reference's own tests do
(tests/test_fused_cross_entropy.py:21-27 of Flag-Operators), half-precision
logits are checked against the oracle run on the same values upcast to fp32,
then rounded to the logits' dtype; torch's bf16 CPU path rounds log-probs to
bf16 before exponentiating, which alone moves small gradients by ~3%.
"""
import math

import pytest
import torch

import oracle
from conftest import load_golden
from operators.fused_cross_entropy import cross_entropy_loss, fused_cross_entropy

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _run(logits, target, **kw):
    x = logits.to(DEV).requires_grad_(True)
    loss = fused_cross_entropy(x, target.to(DEV), **kw)
    loss.backward(torch.ones_like(loss))
    return loss.detach().cpu(), x.grad.cpu()


def _ref(logits, target, **kw):
    loss, grad = oracle.fused_cross_entropy_grad(logits.float(), target, **kw)
    return loss.to(logits.dtype), grad.to(logits.dtype)


def _close(got, ref, dtype, what):
    if dtype == torch.float32:
        torch.testing.assert_close(got.float(), ref.float(), rtol=1e-5, atol=1e-6, msg=what)
    else:
        scale = ref.float().abs().max().item()
        torch.testing.assert_close(got.float(), ref.float(), rtol=2e-2, atol=2e-2 * scale * 1e-3,
                                   msg=what)


def test_golden_fixtures():
    z = load_golden("fused_cross_entropy")
    for red in ("none", "mean", "sum"):
        for ls in (0.0, 0.1):
            loss, grad = _run(z["lg"], z["tg"], reduction=red, label_smoothing=ls)
            torch.testing.assert_close(loss, z[f"loss_{red}_{ls}"], rtol=1e-5, atol=1e-5)
            torch.testing.assert_close(grad, z[f"grad_{red}_{ls}"], rtol=1e-5, atol=1e-7)
    loss, grad = _run(z["lgb"], z["tgb"])
    assert loss.dtype == torch.bfloat16 and grad.dtype == torch.bfloat16
    torch.testing.assert_close(loss.float(), z["lossb"].float(), rtol=2e-2, atol=0)
    lr, gr = _ref(z["lgb"], z["tgb"])
    _close(grad, gr, torch.bfloat16, "bf16 grad")


def test_baseline_config_forward_backward():
    """[8192, 128256] bf16, N(0, 2^2) logits, 5% ignore_index, mean."""
    g = torch.Generator().manual_seed(0)
    B, V = 8192, 128256
    logits = (2.0 * torch.randn(B, V, generator=g)).bfloat16()
    target = torch.randint(0, V, (B,), generator=g)
    target[torch.rand(B, generator=g) < 0.05] = -100
    loss, grad = _run(logits, target)
    # oracle on fp32-upcast rows, in blocks of rows to bound host memory
    valid = target != -100
    n_valid = int(valid.sum())
    row_loss = torch.cat([oracle.fused_cross_entropy(logits[i:i + 512].float(),
                                                     target[i:i + 512], reduction="none")
                          for i in range(0, B, 512)])
    ref_loss = row_loss[valid].double().sum() / n_valid
    torch.testing.assert_close(loss.double(), ref_loss, rtol=2e-2, atol=0)
    # gradient on a sample of rows: at most two bf16 rounding steps from the fp32 oracle
    rows = torch.arange(0, B, 97)
    _, g_rows = oracle.fused_cross_entropy_grad(logits[rows].float(), target[rows],
                                                reduction="sum")
    ref_grad = (g_rows / n_valid).bfloat16()
    diff = (grad[rows].view(torch.int16).int() - ref_grad.view(torch.int16).int()).abs()
    assert diff.max().item() <= 2
    assert torch.all(grad[~valid] == 0)


@pytest.mark.parametrize("reduction", ["none", "mean", "sum"])
@pytest.mark.parametrize("B,V", [(1, 10), (8, 100), (32, 1000), (128, 50257), (4, 131072)])
def test_correctness_fp32(B, V, reduction):
    logits = torch.randn(B, V)
    target = torch.randint(0, V, (B,))
    loss, grad = _run(logits, target, reduction=reduction)
    rl, rg = _ref(logits, target, reduction=reduction)
    _close(loss, rl, torch.float32, "loss")
    _close(grad, rg, torch.float32, "grad")


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("V", [1000, 32000, 50257])
def test_half_dtypes(dtype, V):
    logits = (torch.randn(16, V) * 2).to(dtype)
    target = torch.randint(0, V, (16,))
    target[2] = -100
    loss, grad = _run(logits, target)
    rl, rg = _ref(logits, target)
    torch.testing.assert_close(loss.float(), rl.float(), rtol=2e-2, atol=0)
    _close(grad, rg, dtype, "grad")


@pytest.mark.parametrize("ls", [0.1, 0.3])
@pytest.mark.parametrize("reduction", ["none", "mean", "sum"])
def test_label_smoothing_fused(ls, reduction):
    logits = torch.randn(32, 1000) * 3
    target = torch.randint(0, 1000, (32,))
    target[5] = -100
    loss, grad = _run(logits, target, reduction=reduction, label_smoothing=ls)
    rl, rg = _ref(logits, target, reduction=reduction, label_smoothing=ls)
    _close(loss, rl, torch.float32, "loss")
    _close(grad, rg, torch.float32, "grad")


def test_ignore_index_and_all_ignored():
    logits = torch.randn(16, 512)
    target = torch.randint(0, 512, (16,))
    target[0] = -100
    loss, grad = _run(logits, target)
    rl, rg = _ref(logits, target)
    _close(loss, rl, torch.float32, "loss")
    assert torch.all(grad[0] == 0)
    t_all = torch.full((8,), -100, dtype=torch.long)
    got = fused_cross_entropy(torch.randn(8, 100, device=DEV), t_all.to(DEV))
    assert math.isnan(got.item())  # torch semantics (the reference's GPU path returned 0)
    t7 = torch.randint(0, 100, (8,))
    t7[:] = 7
    got = fused_cross_entropy(torch.randn(8, 100, device=DEV), t7.to(DEV), ignore_index=7)
    assert math.isnan(got.item())


def test_known_answers():
    B, V = 4, 100
    logits = torch.full((B, V), -10.0)
    target = torch.randint(0, V, (B,))
    logits[torch.arange(B), target] = 100.0
    assert fused_cross_entropy(logits.to(DEV), target.to(DEV)).item() < 1e-3
    got = fused_cross_entropy(torch.zeros(8, 1000, device=DEV),
                              torch.randint(0, 1000, (8,), device=DEV))
    assert abs(got.item() - math.log(1000)) < 1e-5


def test_grad_output_scaling_and_vector():
    logits = torch.randn(8, 300)
    target = torch.randint(0, 300, (8,))
    x = logits.to(DEV).requires_grad_(True)
    (fused_cross_entropy(x, target.to(DEV), reduction="sum") * 3.5).backward()
    _, rg = _ref(logits, target, reduction="sum")
    torch.testing.assert_close(x.grad.cpu(), rg * 3.5, rtol=1e-5, atol=1e-7)
    x2 = logits.to(DEV).requires_grad_(True)
    go = torch.randn(8)
    fused_cross_entropy(x2, target.to(DEV), reduction="none").backward(go.to(DEV))
    _, rg2 = oracle.fused_cross_entropy_grad(logits, target, reduction="none", grad_output=go)
    torch.testing.assert_close(x2.grad.cpu(), rg2, rtol=1e-5, atol=1e-7)


def test_retain_graph_second_backward_recomputes():
    logits = torch.randn(8, 300)
    target = torch.randint(0, 300, (8,))
    x = logits.to(DEV).requires_grad_(True)
    loss = fused_cross_entropy(x, target.to(DEV))
    (loss * 2).backward(retain_graph=True)
    g1 = x.grad.clone()
    x.grad = None
    (loss * 2).backward()
    torch.testing.assert_close(x.grad, g1, rtol=1e-6, atol=1e-9)


def test_no_grad_forward_and_strided_rows():
    logits = torch.randn(16, 1024, device=DEV)
    target = torch.randint(0, 1000, (16,), device=DEV)
    with torch.no_grad():
        a = fused_cross_entropy(logits[:, :1000], target)
    b = oracle.fused_cross_entropy(logits[:, :1000].cpu(), target.cpu())
    torch.testing.assert_close(a.cpu(), b, rtol=1e-5, atol=1e-6)


def test_gradient_sum_vs_none():
    logits = torch.randn(8, 100)
    target = torch.randint(0, 100, (8,))
    xa = logits.to(DEV).requires_grad_(True)
    fused_cross_entropy(xa, target.to(DEV), reduction="sum").backward()
    xb = logits.to(DEV).requires_grad_(True)
    fused_cross_entropy(xb, target.to(DEV), reduction="none").sum().backward()
    torch.testing.assert_close(xa.grad, xb.grad, rtol=1e-6, atol=1e-8)


def test_cross_entropy_loss_dropin():
    logits = torch.randn(16, 500)
    target = torch.randint(0, 500, (16,))
    got = cross_entropy_loss(logits.to(DEV), target.to(DEV))
    torch.testing.assert_close(got.cpu(), oracle.fused_cross_entropy(logits, target),
                               rtol=1e-5, atol=1e-6)


def test_reference_assertions():
    with pytest.raises(AssertionError, match="2-D"):
        fused_cross_entropy(torch.randn(2, 3, 4, device=DEV), torch.zeros(2, dtype=torch.long,
                                                                          device=DEV))
    with pytest.raises(AssertionError, match="Unknown reduction"):
        fused_cross_entropy(torch.randn(2, 3, device=DEV), torch.zeros(2, dtype=torch.long,
                                                                       device=DEV), "avg")


def test_empty_batch():
    x = torch.empty(0, 10, device=DEV)
    t = torch.empty(0, dtype=torch.long, device=DEV)
    assert fused_cross_entropy(x, t, reduction="sum").item() == 0
    assert fused_cross_entropy(x, t, reduction="none").shape == (0,)


@pytest.mark.parametrize("dtype,V", [(torch.bfloat16, 16384), (torch.bfloat16, 128256),
                                     (torch.bfloat16, 262144), (torch.float16, 65536),
                                     (torch.float32, 8192), (torch.float32, 131072)])
@pytest.mark.parametrize("ls", [0.0, 0.1])
def test_long_rows_fused_grad(dtype, V, ls):
    """Rows long enough for the cluster kernel (the row split over 1-8 CTAs),
    with ignored rows, label smoothing and a target in the last column."""
    g = torch.Generator().manual_seed(V)
    B = 12
    logits = (torch.randn(B, V, generator=g) * 2).to(dtype)
    target = torch.randint(0, V, (B,), generator=g)
    target[3] = -100
    target[7] = V - 1
    target[8] = 0
    for red in ("mean", "sum"):
        loss, grad = _run(logits, target, reduction=red, label_smoothing=ls)
        rl, rg = _ref(logits, target, reduction=red, label_smoothing=ls)
        if dtype == torch.float32:
            _close(loss, rl, dtype, "loss")
        else:
            torch.testing.assert_close(loss.float(), rl.float(), rtol=2e-2, atol=0)
        _close(grad, rg, dtype, f"grad {red}")
        assert torch.all(grad[3] == 0)


def test_long_rows_strided_logits():
    """Rows of a wider buffer (row stride > V) through the fused gradient."""
    base = (torch.randn(6, 40000) * 2).bfloat16()
    logits = base[:, :32768]
    target = torch.randint(0, 32768, (6,))
    x = logits.to(DEV).requires_grad_(True)
    loss = fused_cross_entropy(x, target.to(DEV))
    loss.backward()
    rl, rg = _ref(logits.contiguous(), target)
    torch.testing.assert_close(loss.detach().cpu().float(), rl.float(), rtol=2e-2, atol=0)
    _close(x.grad.cpu(), rg, torch.bfloat16, "grad")
