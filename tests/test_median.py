"""median parity: values AND indices bit-exact against the oracle (torch CPU
median, the reference's CPU branch), on the golden fixtures, the three full-size
configurations and the edge cases torch defines (ties, -0/+0, NaN, inf)."""
import numpy as np
import pytest
import torch

import oracle
from conftest import load_golden
from operators.median import median

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _exact(x_cpu, dim=-1, keepdim=False, x_dev=None):
    got = median(x_cpu.to(DEV) if x_dev is None else x_dev, dim=dim, keepdim=keepdim)
    ref = oracle.median(x_cpu, dim=dim, keepdim=keepdim)
    assert got.values.shape == ref.values.shape and got.indices.shape == ref.indices.shape
    assert torch.equal(got.indices.cpu(), ref.indices), "indices differ"
    gv, rv = got.values.cpu(), ref.values
    if gv.dtype.is_floating_point:
        same = (gv.view(-1).float().isnan() & rv.view(-1).float().isnan()) | (
            gv.view(-1) == rv.view(-1))
        assert bool(same.all()), "values differ"
        # bit-exact where not NaN (x[idx] itself)
        nn = ~rv.view(-1).float().isnan()
        assert torch.equal(gv.view(-1)[nn].view(torch.int16 if gv.element_size() == 2
                                                else torch.int32),
                           rv.view(-1)[nn].view(torch.int16 if rv.element_size() == 2
                                                else torch.int32))
    else:
        assert torch.equal(gv, rv)


def test_golden_fixtures():
    z = load_golden("median")
    for name in ("a", "b", "c", "s"):
        got = median(z[f"x_{name}"].to(DEV), dim=-1)
        assert torch.equal(got.indices.cpu(), z[f"i_{name}"]), name
        assert np.array_equal(got.values.cpu().numpy(), z[f"v_{name}"].numpy(), equal_nan=True)
    for d in (0, 1, 2):
        got = median(z["x3"].to(DEV), dim=d)
        assert torch.equal(got.values.cpu(), z[f"v3_{d}"])
        assert torch.equal(got.indices.cpu(), z[f"i3_{d}"])
    for i in range(z["n_known"]):
        assert torch.equal(median(z[f"kx{i}"].to(DEV)).cpu(), z[f"kv{i}"])
    assert torch.equal(median(z["gx"].to(DEV)).cpu(), z["gv"])


@pytest.mark.parametrize("cfg", ["a", "b", "c"])
def test_baseline_configs(cfg):
    g = torch.Generator().manual_seed(0)
    if cfg == "a":
        x = torch.randn(8192, 2048, generator=g)
    elif cfg == "b":
        x = torch.randint(-64, 64, (8192, 2048), generator=g).float()
    else:
        x = torch.randn(65536, 257, generator=g)
    _exact(x)


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16, torch.int32, torch.int64,
                                   torch.int16, torch.uint8])
@pytest.mark.parametrize("N", [1, 2, 31, 257, 1024, 2048, 5000])
def test_dtypes(dtype, N):
    if dtype.is_floating_point:
        x = torch.randn(64, N).to(dtype)
    else:
        lo = 0 if dtype == torch.uint8 else -50
        x = torch.randint(lo, 50, (64, N)).to(dtype)
    _exact(x)


@pytest.mark.parametrize("N", [1, 2, 3, 32, 33, 127, 128, 129, 511, 512, 513, 2047, 2048, 2049,
                               4096, 10000, 70000])
def test_lengths_fp32(N):
    _exact(torch.randn(37, N))
    _exact(torch.randint(-3, 3, (37, N)).float())   # very tie-heavy


def test_special_values():
    x = torch.randn(64, 300)
    x[0] = 0.0
    x[1, ::2] = -0.0
    x[2, 5] = float("nan")
    x[3, 100:] = float("nan")
    x[4] = float("inf")
    x[5, :150] = float("-inf")
    x[6, 7] = float("nan"); x[6, 3] = float("nan")
    x[7] = torch.where(torch.rand(300) < 0.5, torch.tensor(-0.0), torch.tensor(0.0))
    _exact(x)
    xv = x.clone()[:, :256].contiguous()    # vector (16-byte) load path
    _exact(xv)


def test_dims_and_keepdim():
    x = torch.randn(4, 8, 16, 5)
    for d in range(-4, 4):
        for kd in (False, True):
            _exact(x, dim=d, keepdim=kd)
    _exact(torch.randn(7), dim=0)
    got = median(torch.tensor([5.0, 3.0, 1.0, 4.0, 2.0], device=DEV), dim=0)
    assert got.values.item() == 3.0 and got.indices.item() == 1


def test_global_median():
    for shape in [(1,), (7,), (16,), (4, 128, 128), (1000003,)]:
        x = torch.randn(*shape)
        assert torch.equal(median(x.to(DEV)).cpu(), oracle.median(x))
    xh = torch.randn(64).half()
    assert torch.equal(median(xh.to(DEV)).cpu(), oracle.median(xh))
    xn = torch.randn(100)
    xn[17] = float("nan")
    assert torch.isnan(median(xn.to(DEV))).item()
    with pytest.raises(RuntimeError, match="must not be empty"):
        median(torch.empty(0, device=DEV))


def test_non_contiguous_input():
    x = torch.randn(300, 64).t()     # [64, 300] view with stride (1, 64)
    _exact(x)


def test_empty_rows():
    got = median(torch.empty(0, 5, device=DEV), dim=1)
    assert got.values.shape == (0,) and got.indices.shape == (0,)


def test_deterministic():
    x = torch.randint(-5, 5, (512, 999)).float().to(DEV)
    a, b = median(x, dim=1), median(x, dim=1)
    assert torch.equal(a.indices, b.indices)


@pytest.mark.parametrize("dtype", [torch.float32, torch.float16, torch.bfloat16])
@pytest.mark.parametrize("N", [512, 1024, 2048])
def test_special_values_full_rows(dtype, N):
    """Rows that exactly fill a row group (the unpredicated kernel), with NaN,
    infinities, signed zeros, all-equal rows and wide buckets (uniform data)."""
    g = torch.Generator().manual_seed(N)
    x = torch.randn(48, N, generator=g)
    x[0] = 0.0
    x[1, ::2] = -0.0
    x[2, N - 1] = float("nan")
    x[3, 7:] = float("nan")
    x[4] = float("inf")
    x[5, : N // 2 + 3] = float("-inf")
    x[6, 9] = float("nan"); x[6, 4] = float("-nan")
    x[7] = torch.where(torch.rand(N, generator=g) < 0.5, torch.tensor(-0.0), torch.tensor(0.0))
    x[8] = 3.0
    x[9, ::3] = float("inf")
    x[10, 1::2] = float("-inf")
    x[11:20] = torch.rand(9, N, generator=g)                 # ~N/8 keys per top-digit bucket
    x[20:24] = torch.randint(-2, 3, (4, N), generator=g).float()
    x[24] = torch.arange(N).float()
    x[25] = -torch.arange(N).float()
    x[26, N // 2:] = 1e-40                                  # subnormals
    x[27] = torch.full((N,), -1e-40)
    _exact(x.to(dtype))


@pytest.mark.parametrize("N", [512, 2048])
def test_int32_full_rows(N):
    g = torch.Generator().manual_seed(1)
    x = torch.randint(-2**31, 2**31 - 1, (40, N), generator=g, dtype=torch.int64).to(torch.int32)
    x[0] = 7
    x[1, ::2] = -2**31
    x[2] = 2**31 - 1
    x[3:10] = torch.randint(-3, 3, (7, N), generator=g).to(torch.int32)
    _exact(x)


def _sweep_rows(N, g):
    """Rows that exercise the special paths of the row kernels."""
    x = torch.randn(24, N, generator=g)
    x[1] = torch.randint(-4, 4, (N,), generator=g).float()             # wide ties
    x[2] = torch.where(torch.rand(N, generator=g) < 0.5, torch.tensor(-0.0),
                       torch.tensor(0.0))                               # zeros of both signs
    x[3, ::3] = 0.0
    x[3, 1::3] = -0.0                                                    # zero median, mixed signs
    x[4] = 1.0 + torch.rand(N, generator=g) * 1e-4                       # one top-bit bin
    x[5] = torch.randn(N, generator=g) * 1e-39                           # subnormals around 0
    x[6, N // 3] = float("nan")
    x[7, : N // 2 + 1] = float("inf")
    x[8, ::2] = float("-inf")
    x[9] = torch.where(torch.rand(N, generator=g) < 0.5, torch.tensor(0.0),
                       torch.tensor(1e-42))                              # +0 beside subnormals
    x[10] = torch.where(torch.rand(N, generator=g) < 0.5, torch.tensor(-0.0),
                        torch.tensor(-1e-42))                            # -0 beside subnormals
    x[11] = -torch.arange(N).float()
    return x


@pytest.mark.parametrize("layout", ["vector", "scalar"])
def test_row_length_sweep(layout):
    """Row lengths 1..2048 in steps that cross every row-group size of the row
    kernels (full and partial groups), 16-byte and scalar loads (rows starting
    4 bytes past a 16-byte boundary), fp32 and int32, with ties, signed zeros,
    subnormals, NaN and infinities."""
    g = torch.Generator().manual_seed(77)
    if layout == "vector":
        lengths = sorted({4 * i for i in range(1, 513, 9)} | {128 * e for e in range(1, 17)})
    else:
        lengths = sorted(set(range(1, 2049, 23)) | {32 * e + 1 for e in range(0, 64)})
    for N in lengths:
        x = _sweep_rows(N, g)
        xi = torch.randint(-2**31, 2**31 - 1, (8, N), generator=g, dtype=torch.int64)
        xi[1] = torch.randint(-3, 3, (N,), generator=g)
        xi = xi.to(torch.int32)
        if layout == "scalar" and N % 4 == 0:
            # contiguous rows starting 4 bytes past a 16-byte boundary: scalar loads
            for t in (x, xi):
                buf = torch.zeros(t.numel() + 1, dtype=t.dtype, device=DEV)
                buf[1:] = t.reshape(-1).to(DEV)
                _exact(t, x_dev=buf[1:].view(t.shape))
        else:
            _exact(x)
            _exact(xi)


def test_no_handoff_timeouts():
    """Collected after the median tests above: none of their producer/consumer
    hand-offs ran out of polls."""
    from operators.median import timeouts
    median(torch.randn(300, 2048).to(DEV), dim=-1)
    torch.cuda.synchronize()
    assert timeouts() == 0


@pytest.mark.parametrize("case", ["randn", "ties", "const", "nan", "zeros", "int32", "int64",
                                  "bf16", "fp16", "odd", "offset", "zeros_bf16", "const_4m",
                                  "block_4m", "int64_4m"])
def test_global_median_grid_path(case):
    """n >= 2^20 elements: the grid-wide radix select (a CTA per chunk per pass)."""
    g = torch.Generator().manual_seed(11)
    n = 1 << 21
    if case == "randn":
        x = torch.randn(8192, 2048, generator=g)
    elif case == "ties":
        x = torch.randint(-5, 5, (n,), generator=g).float()
    elif case == "const":
        x = torch.full((n,), 2.5)
    elif case == "nan":
        x = torch.randn(n, generator=g)
        x[n - 7] = float("nan")
        x[123457] = float("nan")
    elif case == "zeros":
        x = torch.where(torch.rand(n, generator=g) < 0.5, torch.tensor(-0.0), torch.tensor(0.0))
        x[:1000] = 1.0
        x[-1000:] = -1.0
    elif case == "int32":
        x = torch.randint(-2**31, 2**31 - 1, (n,), generator=g, dtype=torch.int64).to(torch.int32)
    elif case == "int64":
        x = torch.randint(-2**62, 2**62, (n,), generator=g, dtype=torch.int64)
    elif case == "bf16":
        x = torch.randn(n, generator=g).bfloat16()
    elif case == "fp16":
        x = torch.randn(n, generator=g).half()
    elif case == "zeros_bf16":
        x = torch.where(torch.rand(n, generator=g) < 0.3, torch.tensor(-0.0), torch.tensor(0.0))
        x[:5000] = -2.0
        x = x.bfloat16()
    elif case == "offset":
        x = torch.randn(n + 3, generator=g)
    elif case == "const_4m":
        # the median's bin holds every element: too many candidates to keep
        x = torch.full((1 << 22,), -1.5)
    elif case == "block_4m":
        # the median's bin (values in [1, 1.25)) holds 20000 elements lying in one
        # or two chunks of sorted data: they fit the candidate regions as a whole
        # but overflow the CTAs that own them, so later passes read x again
        m = 1 << 22
        blk = 1.0 + 0.2 * torch.rand(20000, generator=g)
        lo = m // 2 - 10000
        x = torch.cat([torch.full((lo,), -2.0), blk.sort().values,
                       torch.full((m - lo - 20000,), 3.0)])
    elif case == "int64_4m":
        # six passes: later ones read the kept candidates
        x = torch.randint(-2**40, 2**40, (1 << 22,), generator=g, dtype=torch.int64)
    else:
        x = torch.randn((1 << 20) + 13, generator=g)
    if case == "offset":
        # a view starting 12 bytes into its storage: element loads instead of 16-byte loads
        got = median(x.to(DEV)[3:]).cpu()
        ref = oracle.median(x[3:])
    else:
        got = median(x.to(DEV)).cpu()
        ref = oracle.median(x)
    if case == "nan":
        assert torch.isnan(got).item()
    else:
        # torch's global median is the element std::nth_element leaves at rank k;
        # between +0.0 and -0.0 that choice is unspecified, so a zero median is
        # compared by value (the kernel returns an input zero, with its sign)
        assert torch.equal(got, ref), (got, ref)
    from operators.median import timeouts
    assert timeouts() == 0
