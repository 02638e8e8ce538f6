"""rms_norm parity: sm_100a kernel (through the C ABI) vs the oracle.

Tolerances (stated by the target spec): fp32 rtol 1e-5 (atol 1e-5 for values
near zero); bf16 / fp16 rtol 2e-2.  The reference's own test matrix
(tests/test_rms_norm.py of Flag-Operators) is repeated on the GPU.
"""
import pytest
import torch

import oracle
from conftest import load_golden
from operators.rms_norm import rms_norm, rms_norm_forward, rms_norm_out

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _tol(dtype):
    return (1e-5, 1e-5) if dtype == torch.float32 else (2e-2, 2e-2)


def _check(x, w, eps=1e-5):
    y, inv = rms_norm_forward(x, (x.shape[-1],), w, eps=eps)
    y_ref, inv_ref = oracle.rms_norm_forward(x, (x.shape[-1],), w, eps=eps)
    rtol, atol = _tol(x.dtype)
    torch.testing.assert_close(y.cpu(), y_ref, rtol=rtol, atol=atol)
    torch.testing.assert_close(inv.cpu(), inv_ref, rtol=1e-5, atol=0)
    return y, inv


def test_golden_fixtures():
    z = load_golden("rms_norm")
    for i in range(z["n_cases"]):
        x, w, eps = z[f"x{i}"].to(DEV), z[f"w{i}"].to(DEV), z[f"eps{i}"]
        y, inv = rms_norm_forward(x, (x.shape[-1],), w, eps=eps)
        rtol, atol = _tol(x.dtype)
        torch.testing.assert_close(y.cpu(), z[f"y{i}"], rtol=rtol, atol=atol)
        torch.testing.assert_close(inv.cpu(), z[f"inv{i}"], rtol=1e-5, atol=0)
    y = rms_norm(z["ones_x"].to(DEV), (128,), torch.ones(128, device=DEV))
    assert torch.equal(y.cpu(), z["ones_y"])


@pytest.mark.parametrize("shape,dtype", [((4096, 4096), torch.float32),
                                         ((16384, 8192), torch.bfloat16)])
def test_baseline_configs(shape, dtype):
    g = torch.Generator().manual_seed(0)
    x = torch.randn(*shape, generator=g).to(dtype)
    w = (1 + 0.1 * torch.randn(shape[-1], generator=g)).to(dtype)
    y, inv = rms_norm_forward(x.to(DEV), (shape[-1],), w.to(DEV), eps=1e-6)
    y_ref, inv_ref = oracle.rms_norm_forward(x, (shape[-1],), w, eps=1e-6)
    rtol, atol = _tol(dtype)
    torch.testing.assert_close(y.cpu(), y_ref, rtol=rtol, atol=atol)
    torch.testing.assert_close(inv.cpu(), inv_ref, rtol=1e-5, atol=0)
    if dtype == torch.bfloat16:
        # at most one bf16 rounding step apart from the oracle
        diff = (y.cpu().view(torch.int16).int() - y_ref.view(torch.int16).int()).abs()
        assert diff.max().item() <= 1


@pytest.mark.parametrize("N", [64, 128, 256, 512, 1024, 2048, 4096])
@pytest.mark.parametrize("M", [1, 4, 16, 64])
def test_small_n_float32(M, N):
    _check(torch.randn(M, N, device=DEV), torch.ones(N, device=DEV))


@pytest.mark.parametrize("N", [5000, 8192, 16384, 32768, 65536])
def test_large_n_float32(N):
    _check(torch.randn(8, N, device=DEV), torch.randn(N, device=DEV))


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("N", [128, 1024, 4096, 8192, 20000])
def test_half_dtypes(dtype, N):
    _check(torch.randn(16, N, device=DEV, dtype=dtype), torch.ones(N, device=DEV, dtype=dtype))


@pytest.mark.parametrize("xd,wd", [(torch.bfloat16, torch.float32),
                                   (torch.float32, torch.bfloat16),
                                   (torch.float16, torch.float32)])
def test_mixed_weight_dtype(xd, wd):
    x = torch.randn(32, 1024, device=DEV).to(xd)
    w = (1 + 0.1 * torch.randn(1024, device=DEV)).to(wd)
    _check(x, w)


def test_non_unit_weight_and_3d():
    _check(torch.randn(16, 512, device=DEV), torch.rand(512, device=DEV) * 2.0)
    x = torch.randn(4, 128, 512, device=DEV)
    y = rms_norm(x, (512,), torch.ones(512, device=DEV))
    y_ref, _ = oracle.rms_norm_forward(x, (512,), torch.ones(512))
    assert y.shape == x.shape
    torch.testing.assert_close(y.cpu(), y_ref, rtol=1e-5, atol=1e-5)


def test_multi_dim_normalized_shape():
    x = torch.randn(6, 8, 32, device=DEV)
    w = torch.randn(8, 32, device=DEV)
    y, inv = rms_norm_forward(x, (8, 32), w)
    y_ref, inv_ref = oracle.rms_norm_forward(x, (8, 32), w)
    torch.testing.assert_close(y.cpu(), y_ref, rtol=1e-5, atol=1e-5)
    assert inv.shape == (6,)


@pytest.mark.parametrize("N", [100, 513, 1001, 3000, 7])
def test_non_power_of_two(N):
    _check(torch.randn(4, N, device=DEV), torch.ones(N, device=DEV))


def test_unaligned_rows_use_generic_path():
    base = torch.randn(4 * 257 + 1, device=DEV)
    x = base[1:].view(4, 257)      # 4-byte aligned only
    _check(x, torch.randn(257, device=DEV))


def test_eps_effect_and_inv_rms():
    x = torch.randn(4, 256, device=DEV) * 1e-3
    w = torch.ones(256, device=DEV)
    assert not torch.allclose(rms_norm(x, (256,), w, eps=1e-8), rms_norm(x, (256,), w, eps=1.0))
    x = torch.randn(8, 512, device=DEV)
    _, inv = rms_norm_forward(x, (512,), w.new_ones(512))
    manual = 1.0 / x.float().pow(2).mean(dim=-1).add(1e-5).sqrt()
    torch.testing.assert_close(inv, manual, rtol=1e-5, atol=1e-6)


def test_out_variant():
    x = torch.randn(8, 512, device=DEV)
    w = torch.ones(512, device=DEV)
    y_ref = rms_norm(x, (512,), w)
    out = torch.empty_like(x)
    assert rms_norm_out(out, x, (512,), w) is out
    assert torch.equal(out, y_ref)
    orig = x.clone()
    strided = torch.empty(512, 8, device=DEV).t()     # non-contiguous result
    rms_norm_out(strided, x, (512,), w)
    assert torch.equal(strided, y_ref) and torch.equal(x, orig)


def test_identical_rows_and_determinism():
    x = torch.randn(1, 256, device=DEV).expand(8, 256).contiguous()
    y = rms_norm(x, (256,), torch.ones(256, device=DEV))
    assert all(torch.equal(y[0], y[i]) for i in range(8))
    x = torch.randn(64, 4096, device=DEV)
    assert torch.equal(rms_norm(x, (4096,), torch.ones(4096, device=DEV)),
                       rms_norm(x, (4096,), torch.ones(4096, device=DEV)))


@pytest.mark.parametrize("N", [128, 4096, 8192])
def test_all_ones(N):
    # rms(ones) = sqrt(1 + eps) -> y = 1 within eps (reference test_rms_norm.py:191-200)
    x = torch.ones(4, N, device=DEV)
    y = rms_norm(x, (N,), torch.ones(N, device=DEV))
    torch.testing.assert_close(y, torch.ones_like(y), rtol=1e-5, atol=1e-5)
    y0 = rms_norm(x, (N,), torch.ones(N, device=DEV), eps=0.0)
    assert torch.all(y0 == 1)


def test_empty_rows():
    x = torch.empty(0, 64, device=DEV)
    y, inv = rms_norm_forward(x, (64,), torch.ones(64, device=DEV))
    assert y.shape == (0, 64) and inv.shape == (0,)


# ---------------------------------------------------------------------------
# backward (dx, dw) from inv_rms
# ---------------------------------------------------------------------------
def _bwd_case(M, N, dtype, wdtype=None, seed=0):
    g = torch.Generator().manual_seed(seed)
    x = (torch.randn(M, N, generator=g) * 1.5).to(dtype)
    w = (1 + 0.3 * torch.randn(N, generator=g)).to(wdtype or dtype)
    dy = torch.randn(M, N, generator=g).to(dtype)
    return x, w, dy


def _check_bwd(x, w, dy, eps=1e-6):
    from operators.rms_norm import rms_norm_backward
    N = x.shape[-1]
    xd, wd, dyd = x.to(DEV), w.to(DEV), dy.to(DEV)
    _, inv = rms_norm_forward(xd, (N,), wd, eps)
    dx, dw = rms_norm_backward(dyd, xd, inv, (N,), wd)
    assert dx.dtype == x.dtype and dw.dtype == w.dtype
    rdx, rdw = oracle.rms_norm_backward(dy, x, (N,), w, eps)
    if x.dtype == torch.float32:
        torch.testing.assert_close(dx.cpu(), rdx, rtol=1e-5, atol=1e-5)
    else:
        torch.testing.assert_close(dx.cpu().float(), rdx, rtol=2e-2, atol=2e-2)
    # dw sums M terms: its fp32 error is bounded by 1e-5 of the sum of their
    # magnitudes; a 16-bit dw adds one rounding (2^-8 relative for bf16)
    inv_c = inv.cpu()[:, None]
    scale = (dy.float() * x.float() * inv_c).abs().sum(0)
    tol = 1e-5 * scale + 1e-5
    if w.dtype != torch.float32:
        tol = tol + 8e-3 * rdw.abs()
    err = (dw.cpu().float() - rdw).abs()
    assert bool((err <= tol).all()), float(err.max())


@pytest.mark.parametrize("M,N", [(64, 1024), (33, 4096), (257, 2048), (16, 96), (8, 100),
                                 (5, 3000), (4, 16384)])
def test_backward_float32(M, N):
    _check_bwd(*_bwd_case(M, N, torch.float32))


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("N", [1024, 4096, 8192, 8200, 16384])
def test_backward_half(dtype, N):
    _check_bwd(*_bwd_case(48, N, dtype, seed=N))


def test_backward_mixed_weight_dtype():
    _check_bwd(*_bwd_case(40, 2048, torch.bfloat16, torch.float32))


def test_backward_benchmark_shape_bf16():
    """[16384, 8192] bf16, the forward benchmark's shape."""
    _check_bwd(*_bwd_case(16384, 8192, torch.bfloat16, seed=3))


def test_autograd_through_rms_norm():
    x, w, dy = _bwd_case(32, 512, torch.float32, seed=5)
    xd = x.to(DEV).requires_grad_(True)
    wd = w.to(DEV).requires_grad_(True)
    y = rms_norm(xd, (512,), wd, 1e-6)
    y.backward(dy.to(DEV))
    rdx, rdw = oracle.rms_norm_backward(dy, x, (512,), w, 1e-6)
    torch.testing.assert_close(xd.grad.cpu(), rdx, rtol=1e-5, atol=1e-5)
    torch.testing.assert_close(wd.grad.cpu(), rdw, rtol=1e-4, atol=1e-4)
    # only x requires grad
    xd2 = x.to(DEV).requires_grad_(True)
    rms_norm(xd2, 512, w.to(DEV), 1e-6).backward(dy.to(DEV))
    torch.testing.assert_close(xd2.grad.cpu(), rdx, rtol=1e-5, atol=1e-5)


def test_backward_empty_rows():
    from operators.rms_norm import rms_norm_backward
    x = torch.empty(0, 64, device=DEV)
    w = torch.randn(64, device=DEV)
    dx, dw = rms_norm_backward(torch.empty(0, 64, device=DEV), x,
                               torch.empty(0, device=DEV), (64,), w)
    assert dx.shape == (0, 64) and torch.all(dw == 0)
