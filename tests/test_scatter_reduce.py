"""scatter_reduce parity vs the oracle (torch CPU scatter_reduce_, the reference's
CPU branch).

Standards (target spec): amax/amin and integer sum/mean bit-exact (amax/amin up
to the sign of a zero when +0.0 and -0.0 meet in one cell, where torch keeps
whichever came first); float sum/mean/prod within rtol 1e-5.  A float sum's
rounding error scales with the sum of |terms|, not with |result|, so sum/mean
use |got - ref| <= 1e-5 * sum(|terms|) per cell (plus 1e-6 absolute); prod uses
rtol 1e-5 + 4 * count * 2^-24 of |ref|.
"""
import math

import pytest
import torch

import oracle
from conftest import load_golden
from operators.scatter_reduce import scatter_reduce, scatter_reduce_, scatter_reduce_out

pytestmark = pytest.mark.gpu
DEV = "cuda"
REDUCES = ["sum", "prod", "amax", "amin", "mean"]


def _compare(got, ref, reduce, inp, dim, index, src, include_self):
    got = got.cpu()
    assert got.shape == ref.shape and got.dtype == ref.dtype
    if not got.dtype.is_floating_point:
        assert torch.equal(got, ref), f"{reduce}: integer result differs"
        return
    g, r = got.double(), ref.double()
    nan_ok = torch.equal(g.isnan(), r.isnan())
    assert nan_ok, f"{reduce}: NaN positions differ"
    m = ~r.isnan()
    g, r = g[m], r[m]
    if reduce in ("amax", "amin"):
        assert torch.equal(g, r), f"{reduce}: not bit-exact"
        return
    half = got.dtype in (torch.float16, torch.bfloat16)
    rtol = 2e-2 if half else 1e-5
    if reduce == "prod":
        _, cnt = oracle.scatter_reduce_scale(inp, dim, index, src, include_self)
        tol = (rtol + 4 * cnt[m] * 2.0 ** -24) * r.abs() + 1e-30
    else:
        scale, cnt = oracle.scatter_reduce_scale(inp, dim, index, src, include_self)
        scale, cnt = scale[m], cnt[m]
        if reduce == "mean":
            scale = scale / cnt.clamp(min=1)
        tol = rtol * scale + (1e-2 if half else 1e-6)
    bad = (g - r).abs() > tol
    assert not bool(bad.any()), (f"{reduce}: {int(bad.sum())} cells outside tolerance, "
                                 f"max err {float((g - r).abs().max()):.3e}")


def _check(inp, dim, index, src, reduce, include_self=True, variant="out"):
    ref = oracle.scatter_reduce(inp, dim, index, src, reduce, include_self=include_self)
    di, dx, ds = inp.to(DEV), index.to(DEV), src.to(DEV)
    if variant == "inplace":
        got = scatter_reduce_(di.clone(), dim, dx, ds, reduce, include_self=include_self)
    elif variant == "out=":
        o = torch.empty_like(di)
        got = scatter_reduce_out(o, di, dim, dx, ds, reduce, include_self=include_self)
        assert got is o
    else:
        got = scatter_reduce(di, dim, dx, ds, reduce, include_self=include_self)
        assert torch.equal(di.cpu().view(-1).view(torch.uint8),
                           inp.view(-1).view(torch.uint8)), "out-of-place modified its input"
    _compare(got, ref, reduce, inp, dim, index, src, include_self)


def test_golden_fixtures():
    z = load_golden("scatter_reduce")
    for dist in ("u", "z"):
        for red in REDUCES:
            for inc in (True, False):
                got = scatter_reduce(z["self1"].to(DEV), 0, z[f"idx_{dist}"].to(DEV),
                                     z["src1"].to(DEV), red, include_self=inc)
                _compare(got, z[f"o_{dist}_{red}_{int(inc)}"], red, z["self1"], 0,
                         z[f"idx_{dist}"], z["src1"], inc)
    for red in ("sum", "amax", "amin", "mean"):
        for inc in (True, False):
            got = scatter_reduce(z["self_i"].to(DEV), 0, z["idx_u"].to(DEV), z["src_i"].to(DEV),
                                 red, include_self=inc)
            assert torch.equal(got.cpu(), z[f"oi_{red}_{int(inc)}"]), (red, inc)
    for red in REDUCES:
        for inc in (True, False):
            for nm in ("2", "3"):
                got = scatter_reduce(z[f"self{nm}"].to(DEV), 1, z[f"idx{nm}"].to(DEV),
                                     z[f"src{nm}"].to(DEV), red, include_self=inc)
                _compare(got, z[f"o{nm}_{red}_{int(inc)}"], red, z[f"self{nm}"], 1,
                         z[f"idx{nm}"], z[f"src{nm}"], inc)
    ip = z["self1"].to(DEV)
    scatter_reduce_(ip, 0, z["idx_u"].to(DEV), z["src1"].to(DEV), "sum")
    _compare(ip, z["o_inplace_sum"], "sum", z["self1"], 0, z["idx_u"], z["src1"], True)
    o = torch.empty(1024, device=DEV)
    scatter_reduce_out(o, z["self1"].to(DEV), 0, z["idx_u"].to(DEV), z["src1"].to(DEV), "amax")
    assert torch.equal(o.cpu(), z["o_out_amax"])


def _zipf_index(n, m, g):
    r = torch.arange(1, m + 1, dtype=torch.float64)
    cdf = torch.cumsum(r.pow(-1.1) / r.pow(-1.1).sum(), 0)
    return torch.searchsorted(cdf, torch.rand(n, generator=g, dtype=torch.float64)).clamp(max=m - 1)


@pytest.fixture(scope="module")
def c3_inputs():
    g = torch.Generator().manual_seed(0)
    n_self, n_src = 1 << 20, 1 << 24
    self_ = torch.randn(n_self, generator=g)
    src = torch.randn(n_src, generator=g)
    idx_u = torch.randint(0, n_self, (n_src,), generator=g)
    idx_z = _zipf_index(n_src, n_self, g)
    return self_, src, idx_u, idx_z


@pytest.mark.parametrize("dist", ["uniform", "zipf"])
@pytest.mark.parametrize("reduce", REDUCES)
@pytest.mark.parametrize("include_self", [True, False])
def test_baseline_config(c3_inputs, dist, reduce, include_self):
    self_, src, idx_u, idx_z = c3_inputs
    idx = idx_u if dist == "uniform" else idx_z
    _check(self_, 0, idx, src, reduce, include_self)


@pytest.mark.parametrize("variant", ["inplace", "out="])
def test_baseline_config_variants(c3_inputs, variant):
    self_, src, idx_u, _ = c3_inputs
    _check(self_, 0, idx_u, src, "sum", True, variant)
    _check(self_, 0, idx_u, src, "amax", False, variant)


@pytest.mark.parametrize("reduce", ["sum", "mean", "amax", "amin"])
@pytest.mark.parametrize("include_self", [True, False])
def test_int32_bit_exact(c3_inputs, reduce, include_self):
    g = torch.Generator().manual_seed(1)
    _, _, idx_u, idx_z = c3_inputs
    n_self = 1 << 20
    self_i = torch.zeros(n_self, dtype=torch.int32)
    src_i = torch.randint(-100, 100, (idx_u.numel(),), generator=g, dtype=torch.int32)
    for idx in (idx_u, idx_z):
        _check(self_i, 0, idx, src_i, reduce, include_self)


def _make_inputs(shape, dim, dtype=torch.float32, index_frac=0.8):
    idx_shape = list(shape)
    idx_shape[dim] = max(1, int(shape[dim] * index_frac))
    inp = torch.rand(shape, dtype=torch.float32).to(dtype) + 0.1
    src = torch.rand(idx_shape, dtype=torch.float32).to(dtype) + 0.1
    index = torch.randint(0, shape[dim], idx_shape)
    return inp, index, src


@pytest.mark.parametrize("reduce", REDUCES)
@pytest.mark.parametrize("include_self", [True, False])
@pytest.mark.parametrize("shape,dim", [((16,), 0), ((32, 16), 0), ((32, 16), 1), ((8, 16, 8), 0),
                                       ((8, 16, 8), 1), ((8, 16, 8), 2), ((4, 8, 8, 4), 3),
                                       ((4, 8, 8, 4), -2)])
def test_reference_matrix(shape, dim, reduce, include_self):
    inp, index, src = _make_inputs(shape, dim if dim >= 0 else len(shape) + dim)
    _check(inp, dim, index, src, reduce, include_self)


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16, torch.int64, torch.int32])
@pytest.mark.parametrize("reduce", REDUCES)
def test_dtypes(dtype, reduce):
    if dtype.is_floating_point:
        inp, index, src = _make_inputs((64, 32), 1, dtype)
    else:
        inp = torch.randint(-20, 20, (64, 32)).to(dtype)
        index = torch.randint(0, 32, (64, 25))
        src = torch.randint(-20, 20, (64, 25)).to(dtype)
        if reduce == "prod":
            src = torch.randint(1, 3, (64, 25)).to(dtype)
    for inc in (True, False):
        _check(inp, 1, index, src, reduce, inc)


def test_src_larger_than_index_and_strided():
    inp = torch.randn(20, 30)
    src = torch.randn(25, 40)
    index = torch.randint(0, 30, (18, 12))
    for red in REDUCES:
        _check(inp, 1, index, src, red, True)
    base = torch.randn(30, 40)
    inp_t = base.t()                     # non-contiguous self [40, 30]
    idx = torch.randint(0, 40, (40, 30))
    s = torch.randn(40, 30)
    ref = oracle.scatter_reduce_(inp_t.contiguous(), 0, idx, s, "sum")
    d = inp_t.to(DEV)
    scatter_reduce_(d, 0, idx.to(DEV), s.to(DEV), "sum")
    _compare(d, ref, "sum", inp_t.contiguous(), 0, idx, s, True)


def test_known_answers():
    got = scatter_reduce_(torch.zeros(8, device=DEV), 0,
                          torch.tensor([0, 1, 2, 0, 1, 2, 3, 3], device=DEV),
                          torch.ones(8, device=DEV), "sum")
    assert got.tolist() == [2.0, 2.0, 2.0, 2.0, 0.0, 0.0, 0.0, 0.0]
    got = scatter_reduce_(torch.zeros(4, device=DEV), 0, torch.tensor([0, 0, 1, 2], device=DEV),
                          torch.tensor([3.0, 5.0, 2.0, 7.0], device=DEV), "amax",
                          include_self=False)
    assert got.tolist() == [5.0, 2.0, 7.0, 0.0]
    got = scatter_reduce_(torch.full((4,), 10.0, device=DEV), 0,
                          torch.tensor([0, 0, 1, 2], device=DEV),
                          torch.tensor([3.0, 5.0, 2.0, 7.0], device=DEV), "amin")
    assert got.tolist() == [3.0, 2.0, 7.0, 10.0]
    got = scatter_reduce_(torch.ones(3, device=DEV), 0, torch.tensor([0, 0, 1], device=DEV),
                          torch.tensor([2.0, 3.0, 4.0], device=DEV), "prod")
    assert got.tolist() == [6.0, 4.0, 1.0]
    got = scatter_reduce_(torch.zeros(3, device=DEV), 0, torch.tensor([0, 0, 1, 2], device=DEV),
                          torch.tensor([1.0, 3.0, 2.0, 5.0], device=DEV), "mean",
                          include_self=False)
    assert got.tolist() == [2.0, 2.0, 5.0]
    got = scatter_reduce(torch.tensor([0.0, 1.0, 2.0], device=DEV), 0,
                         torch.tensor([0, 1, 1], device=DEV),
                         torch.tensor([float("nan"), 3.0, -1.0], device=DEV), "amax")
    assert math.isnan(got[0].item()) and got[1:].tolist() == [3.0, 2.0]
    got = scatter_reduce(torch.tensor([0, 0], dtype=torch.int32, device=DEV), 0,
                         torch.tensor([0, 0], device=DEV),
                         torch.tensor([-6, -7], dtype=torch.int32, device=DEV), "mean",
                         include_self=False)
    assert got.tolist() == [-7, 0]     # floor(-13 / 2)


def test_nan_in_self_and_src():
    inp = torch.randn(64)
    inp[3] = float("nan")
    src = torch.randn(256)
    src[10] = float("nan")
    index = torch.randint(0, 64, (256,))
    for red in REDUCES:
        for inc in (True, False):
            _check(inp, 0, index, src, red, inc)


def test_empty_index_and_cpu_rejected():
    inp = torch.randn(8, device=DEV)
    got = scatter_reduce(inp, 0, torch.empty(0, dtype=torch.long, device=DEV),
                         torch.empty(0, device=DEV), "sum", include_self=False)
    assert torch.equal(got, inp)
    with pytest.raises(AssertionError, match="Unsupported reduce"):
        scatter_reduce(inp, 0, torch.zeros(1, dtype=torch.long, device=DEV),
                       torch.zeros(1, device=DEV), "median")


@pytest.mark.parametrize("reduce", REDUCES)
@pytest.mark.parametrize("include_self", [True, False])
def test_binned_path_edges(reduce, include_self):
    """The destination-binned pass (1-D contiguous updates, n >= 2^20): a length
    that is not a multiple of 4, slices left empty, a hot cell, signed values
    around 1 for products, NaN in amax/amin, a strided (span 2x) output, and
    int32 sums and means (bit-exact)."""
    g = torch.Generator().manual_seed(41)
    n = (1 << 20) + 3
    n_out = 50000
    idx = torch.randint(0, n_out, (n,), generator=g)
    idx[idx % 7 == 3] = 17                      # a hot cell
    idx[(idx >= 30000) & (idx < 38192)] = 5     # one slice never reached
    src = 1.0 + 0.01 * torch.randn(n, generator=g)
    src[::1001] *= -1.0
    if reduce in ("amax", "amin"):
        src[12345] = float("nan")
    inp = torch.randn(n_out, generator=g)
    _check(inp, 0, idx, src, reduce, include_self=include_self, variant="out")
    _check(inp, 0, idx, src, reduce, include_self=include_self, variant="inplace")
    # in place into a strided view (the output spans twice its cells)
    ref = oracle.scatter_reduce(inp, 0, idx, src, reduce, include_self=include_self)
    buf = torch.zeros(2 * n_out, device=DEV)
    view = buf[::2]
    view.copy_(inp.to(DEV))
    scatter_reduce_(view, 0, idx.to(DEV), src.to(DEV), reduce, include_self=include_self)
    _compare(view, ref, reduce, inp, 0, idx, src, include_self)
    assert bool((buf[1::2] == 0).all()), "cells between the view's elements were written"
    if reduce in ("sum", "mean"):
        inp_i = torch.randint(-50, 50, (n_out,), generator=g, dtype=torch.int32)
        src_i = torch.randint(-100, 100, (n,), generator=g, dtype=torch.int32)
        _check(inp_i, 0, idx, src_i, reduce, include_self=include_self)


def test_binned_path_out_of_range_indices_are_skipped():
    import operators.scatter_reduce as sr
    g = torch.Generator().manual_seed(42)
    n = 1 << 20
    idx = torch.randint(0, 1000, (n,), generator=g)
    bad = torch.rand(n, generator=g) < 0.01
    idx[bad] = 5000                              # outside [0, 1000)
    src = torch.randn(n, generator=g)
    inp = torch.zeros(1000)
    ref = oracle.scatter_reduce(inp, 0, idx[~bad], src[~bad], "sum")
    got = scatter_reduce(inp.to(DEV), 0, idx.to(DEV), src.to(DEV), "sum")
    _compare(got, ref, "sum", inp, 0, idx[~bad], src[~bad], True)
    if sr._CHECK:
        pytest.skip("index checking raises instead")
