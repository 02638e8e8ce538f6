"""Pins the oracle to the reference: oracle outputs vs golden fixtures (CPU only).

The fixtures were produced by the reference's own operators.* CPU branches
(tests/golden/make_golden.py).  Every oracle function must reproduce them
bit for bit (same torch arithmetic), and the independent numpy median rule
must reproduce torch's indices.
"""
import math

import numpy as np
import pytest
import torch

import oracle
from conftest import load_golden


def test_rms_norm_oracle_matches_reference():
    z = load_golden("rms_norm")
    for i in range(z["n_cases"]):
        x, w, eps = z[f"x{i}"], z[f"w{i}"], z[f"eps{i}"]
        y, inv = oracle.rms_norm_forward(x, (x.shape[-1],), w, eps=eps)
        assert torch.equal(y, z[f"y{i}"])
        assert torch.equal(inv, z[f"inv{i}"])
    y, _ = oracle.rms_norm_forward(z["ones_x"], (128,), torch.ones(128))
    assert torch.equal(y, z["ones_y"])
    torch.testing.assert_close(y, torch.ones_like(y), rtol=1e-5, atol=1e-5)  # sqrt(1 + eps)


@pytest.mark.parametrize("name", ["a", "b", "c", "s"])
def test_median_oracle_matches_reference(name):
    z = load_golden("median")
    x = z[f"x_{name}"]
    r = oracle.median(x, dim=-1)
    assert torch.equal(r.indices, z[f"i_{name}"])
    assert torch.equal(r.values, z[f"v_{name}"], ) or torch.allclose(
        r.values, z[f"v_{name}"], equal_nan=True, rtol=0, atol=0)
    # the independent numpy rule reproduces torch's index choice exactly
    v_np, i_np = oracle.median_dim_np(x.numpy())
    assert np.array_equal(i_np, z[f"i_{name}"].numpy())
    assert np.array_equal(v_np, z[f"v_{name}"].numpy(), equal_nan=True)


def test_median_oracle_known_answers_and_dims():
    z = load_golden("median")
    for i in range(z["n_known"]):
        assert torch.equal(oracle.median(z[f"kx{i}"]), z[f"kv{i}"])
    for d in (0, 1, 2):
        r = oracle.median(z["x3"], dim=d)
        assert torch.equal(r.values, z[f"v3_{d}"]) and torch.equal(r.indices, z[f"i3_{d}"])
    assert torch.equal(oracle.median(z["gx"]), z["gv"])


def test_median_tie_heavy_rule_is_stable_rank_not_first_or_last():
    z = load_golden("median")
    x = z["x_b"].numpy()
    _, i_np = oracle.median_dim_np(x)
    vals = x[np.arange(x.shape[0]), i_np]
    first = np.array([np.flatnonzero(row == v)[0] for row, v in zip(x, vals)])
    assert not np.array_equal(first, i_np)  # ties are resolved by stable rank


def test_scatter_oracle_matches_reference():
    z = load_golden("scatter_reduce")
    for dist in ("u", "z"):
        idx = z[f"idx_{dist}"]
        for red in ("sum", "prod", "amax", "amin", "mean"):
            for inc in (True, False):
                got = oracle.scatter_reduce(z["self1"], 0, idx, z["src1"], red,
                                            include_self=inc)
                assert torch.equal(got, z[f"o_{dist}_{red}_{int(inc)}"]), (dist, red, inc)
    for red in ("sum", "amax", "amin", "mean"):
        for inc in (True, False):
            got = oracle.scatter_reduce(z["self_i"], 0, z["idx_u"], z["src_i"], red,
                                        include_self=inc)
            assert torch.equal(got, z[f"oi_{red}_{int(inc)}"])
    for red in ("sum", "prod", "amax", "amin", "mean"):
        for inc in (True, False):
            assert torch.equal(oracle.scatter_reduce(z["self2"], 1, z["idx2"], z["src2"], red,
                                                     include_self=inc), z[f"o2_{red}_{int(inc)}"])
            assert torch.equal(oracle.scatter_reduce(z["self3"], 1, z["idx3"], z["src3"], red,
                                                     include_self=inc), z[f"o3_{red}_{int(inc)}"])
    assert torch.equal(oracle.scatter_reduce_(z["self1"], 0, z["idx_u"], z["src1"], "sum"),
                       z["o_inplace_sum"])
    assert torch.equal(oracle.scatter_reduce_out(z["self1"], z["self1"], 0, z["idx_u"], z["src1"],
                                                 "amax"), z["o_out_amax"])


def test_scatter_known_answers():
    z = load_golden("scatter_reduce")
    assert torch.equal(z["k_amax"], torch.tensor([5.0, 2.0, 7.0, 0.0]))
    assert torch.equal(z["k_prod"], torch.tensor([6.0, 4.0, 1.0]))
    assert torch.equal(z["k_mean"], torch.tensor([2.0, 2.0, 5.0]))
    assert math.isnan(z["k_nan_amax"][0].item())   # NaN propagates through amax


def test_scatter_int_mean_floors():
    inp = torch.tensor([0, 0], dtype=torch.int32)
    got = oracle.scatter_reduce(inp, 0, torch.tensor([0, 0]), torch.tensor([-6, -7],
                                dtype=torch.int32), "mean", include_self=False)
    assert got.tolist() == [-7, 0]    # floor(-13 / 2)


def test_cross_entropy_oracle_matches_reference():
    z = load_golden("fused_cross_entropy")
    for red in ("none", "mean", "sum"):
        for ls in (0.0, 0.1):
            loss, grad = oracle.fused_cross_entropy_grad(z["lg"], z["tg"], reduction=red,
                                                         label_smoothing=ls)
            assert torch.equal(loss, z[f"loss_{red}_{ls}"])
            assert torch.equal(grad, z[f"grad_{red}_{ls}"])
    loss, grad = oracle.fused_cross_entropy_grad(z["lgb"], z["tgb"])
    assert loss.dtype == torch.bfloat16 and grad.dtype == torch.bfloat16
    assert torch.equal(loss, z["lossb"]) and torch.equal(grad, z["gradb"])
    assert math.isnan(z["all_ignored"].item())   # torch: all-ignored mean is NaN


def test_delta_rule_oracle_matches_reference():
    z = load_golden("chunk_gated_delta_rule")
    for i in range(z["n_cases"]):
        o = oracle.delta_rule_forward(z[f"q{i}"], z[f"k{i}"], z[f"v{i}"], z[f"beta{i}"],
                                      z[f"g{i}"])
        assert torch.equal(o, z[f"o{i}"]), i
    o0 = oracle.delta_rule_forward(z["q1"], z["k1"], z["v1"], z["beta1"],
                                   torch.zeros_like(z["g1"]))
    assert torch.equal(o0, z["o_gate0"])
    q = torch.ones(1, 1, 1, 8)
    k = torch.zeros(1, 1, 1, 8); k[..., 0] = 1.0
    v = torch.zeros(1, 1, 1, 8); v[..., 0] = 2.0
    o = oracle.delta_rule_forward(q, k, v, torch.ones(1, 1, 1), torch.zeros(1, 1, 1))
    assert o[0, 0, 0, 0].item() == pytest.approx(2.0)
    assert torch.equal(o, z["known_o"])


def test_delta_rule_oracle_final_state_chains():
    """Running two halves with the carried state equals one full run."""
    torch.manual_seed(0)
    B, H, L, D = 1, 2, 48, 16
    q, k, v = (torch.randn(B, H, L, D) for _ in range(3))
    k = k / k.norm(dim=-1, keepdim=True)
    beta, g = torch.sigmoid(torch.randn(B, H, L)), torch.sigmoid(torch.randn(B, H, L))
    o, h = oracle.delta_rule_forward(q, k, v, beta, g, output_final_state=True)
    s = 20
    o1, h1 = oracle.delta_rule_forward(q[:, :, :s], k[:, :, :s], v[:, :, :s], beta[:, :, :s],
                                       g[:, :, :s], output_final_state=True)
    o2, h2 = oracle.delta_rule_forward(q[:, :, s:], k[:, :, s:], v[:, :, s:], beta[:, :, s:],
                                       g[:, :, s:], initial_state=h1, output_final_state=True)
    assert torch.allclose(torch.cat([o1, o2], 2), o, atol=1e-5)
    assert torch.allclose(h2, h, atol=1e-5)


def test_rms_norm_backward_oracle_matches_the_analytic_gradient():
    """The oracle's backward (autograd through the reference's CPU formula)
    against an independent float64 statement of the gradient."""
    g = torch.Generator().manual_seed(7)
    M, N, eps = 16, 96, 1e-5
    x = torch.randn(M, N, generator=g) * 1.5
    w = 1 + 0.3 * torch.randn(N, generator=g)
    dy = torch.randn(M, N, generator=g)
    dx, dw = oracle.rms_norm_backward(dy, x, (N,), w, eps)
    xd, wd, dyd = (t.double().numpy() for t in (x, w, dy))
    inv = 1.0 / np.sqrt((xd * xd).mean(axis=1, keepdims=True) + eps)
    gg = dyd * wd
    dx_ref = inv * gg - xd * inv ** 3 * (gg * xd).sum(axis=1, keepdims=True) / N
    dw_ref = (dyd * xd * inv).sum(axis=0)
    np.testing.assert_allclose(dx.numpy(), dx_ref, rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(dw.numpy(), dw_ref, rtol=1e-5, atol=1e-5)


@pytest.mark.parametrize("with_h0", [False, True])
@pytest.mark.parametrize("with_dhT", [False, True])
def test_delta_rule_backward_restatement_matches_autograd(with_h0, with_dhT):
    """The per-step reverse recurrence the CUDA backward implements equals torch
    autograd through the reference's loop (the gradients the reference defines)."""
    gen = torch.Generator().manual_seed(7)
    B, H, L, D = 2, 2, 37, 8
    q, k, v, do = (torch.randn(B, H, L, D, generator=gen, dtype=torch.float64)
                   for _ in range(4))
    k = k / k.norm(dim=-1, keepdim=True)
    beta = torch.sigmoid(torch.randn(B, H, L, generator=gen, dtype=torch.float64))
    g = torch.sigmoid(torch.randn(B, H, L, generator=gen, dtype=torch.float64))
    h0 = torch.randn(B, H, D, D, generator=gen, dtype=torch.float64) if with_h0 else None
    dhT = torch.randn(B, H, D, D, generator=gen, dtype=torch.float64) if with_dhT else None
    ref = oracle.delta_rule_grads(q, k, v, beta, g, do, h0, dhT)
    got = oracle.delta_rule_backward(q, k, v, beta, g, do, h0, dhT)
    for name, r in ref.items():
        r = r.double()
        scale = r.abs().max().item()
        assert (got[name] - r).abs().max().item() <= 1e-5 * scale + 1e-12, name


@pytest.mark.parametrize("C", [1, 5, 16, 64])
@pytest.mark.parametrize("with_state", [False, True])
def test_delta_rule_chunked_backward_algebra_matches_autograd(C, with_state):
    """The chunked backward (per chunk: transposes of T, U, P, Kt and the state
    products, gate gradients through the in-chunk products) equals autograd
    through the reference's loop for any chunk size, ragged last chunk included."""
    gen = torch.Generator().manual_seed(11)
    B, H, L, D = 2, 2, 37, 8
    q, k, v, do = (torch.randn(B, H, L, D, generator=gen, dtype=torch.float64)
                   for _ in range(4))
    k = k / k.norm(dim=-1, keepdim=True)
    beta = torch.sigmoid(torch.randn(B, H, L, generator=gen, dtype=torch.float64))
    g = 0.5 + 0.5 * torch.sigmoid(torch.randn(B, H, L, generator=gen, dtype=torch.float64))
    h0 = torch.randn(B, H, D, D, generator=gen, dtype=torch.float64) if with_state else None
    dhT = torch.randn(B, H, D, D, generator=gen, dtype=torch.float64) if with_state else None
    ref = oracle.delta_rule_grads(q, k, v, beta, g, do, h0, dhT)
    got = oracle.delta_rule_backward_chunked(q, k, v, beta, g, do, h0, dhT, C=C)
    for name, r in ref.items():
        r = r.double()
        assert (got[name] - r).abs().max().item() <= 1e-5 * r.abs().max().item(), name
