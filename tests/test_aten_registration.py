"""Dispatcher registration (operators/aten.py): flagops:: custom ops and the
use_flagops() aten overrides.

CPU: the overrides appear in (and leave) aten's CUDA dispatch table, nest, and
survive an exception; the custom ops' fake kernels give the right shapes.
GPU: inside use_flagops(), torch.median / Tensor.scatter_reduce(_) on CUDA
tensors run this library's kernels (seen in the profiler) and match the oracle
bit for bit (median values and indices, amax, int32 sum); after the block,
PyTorch's kernels serve them again.
"""
import pytest
import torch

import oracle
from operators import aten

OPS = ["aten::" + n for n in aten.OVERRIDDEN]


def _cuda_kernel_site(op: str) -> str:
    for line in torch._C._dispatch_dump_table(op).splitlines():
        if line.startswith("CUDA:"):
            return line
    return ""


def test_overrides_enter_and_leave_the_dispatch_table():
    before = {op: _cuda_kernel_site(op) for op in OPS}
    with aten.use_flagops():
        for op in OPS:
            assert "operators/aten.py" in _cuda_kernel_site(op), op
        with aten.use_flagops():  # nested: shares the registration
            assert "operators/aten.py" in _cuda_kernel_site(OPS[0])
        assert "operators/aten.py" in _cuda_kernel_site(OPS[0])
    assert {op: _cuda_kernel_site(op) for op in OPS} == before
    with pytest.raises(ValueError):
        with aten.use_flagops():
            raise ValueError("body failed")
    assert {op: _cuda_kernel_site(op) for op in OPS} == before


def test_custom_op_fake_shapes():
    from torch._subclasses.fake_tensor import FakeTensorMode
    with FakeTensorMode():
        x = torch.empty(8, 16, 5, device="cuda")
        v, i = torch.ops.flagops.median_dim(x, 1, False)
        assert v.shape == (8, 5) and i.shape == (8, 5) and i.dtype == torch.int64
        v, i = torch.ops.flagops.median_dim(x, -1, True)
        assert v.shape == (8, 16, 1) and v.dtype == x.dtype
        assert torch.ops.flagops.median(x).shape == ()
        idx = torch.empty(8, 16, 5, dtype=torch.int64, device="cuda")
        assert torch.ops.flagops.scatter_reduce(x, 0, idx, x, "sum", True).shape == x.shape


def _kernel_names(fn):
    from torch.profiler import ProfilerActivity, profile
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        fn()
        torch.cuda.synchronize()
    return [e.name for e in prof.events() if e.device_type == torch.autograd.DeviceType.CUDA]


@pytest.mark.gpu
def test_aten_median_runs_the_library_kernels():
    g = torch.Generator().manual_seed(5)
    x = torch.randint(-64, 64, (300, 2048), generator=g).float()  # ties: index rule matters
    xd = x.cuda()
    ref = oracle.median(x, dim=-1)
    with aten.use_flagops():
        res = {}
        names = _kernel_names(lambda: res.setdefault("r", torch.median(xd, dim=-1)))
        assert any("fo::" in n for n in names), names
        r = res["r"]
        assert torch.equal(r.values.cpu(), ref.values)
        assert torch.equal(r.indices.cpu(), ref.indices)
        v, i = xd.median(dim=0, keepdim=True)
        rk = oracle.median(x, dim=0, keepdim=True)
        assert torch.equal(v.cpu(), rk.values) and torch.equal(i.cpu(), rk.indices)
        assert torch.equal(torch.median(xd).cpu(), oracle.median(x))
        vo, io = torch.ops.flagops.median_dim(xd, -1, False)
        assert torch.equal(vo.cpu(), ref.values) and torch.equal(io.cpu(), ref.indices)
    names = _kernel_names(lambda: torch.median(xd, dim=-1))
    assert not any("fo::" in n for n in names), names


@pytest.mark.gpu
def test_aten_scatter_reduce_runs_the_library_kernels():
    g = torch.Generator().manual_seed(6)
    n_self, n_src = 4096, 1 << 16
    self_f = torch.randn(n_self, generator=g)
    src_f = torch.randn(n_src, generator=g)
    idx = torch.randint(0, n_self, (n_src,), generator=g)
    self_i = torch.randint(-100, 100, (n_self,), generator=g, dtype=torch.int32)
    src_i = torch.randint(-100, 100, (n_src,), generator=g, dtype=torch.int32)
    sd, srd, idd, sid, srid = (t.cuda() for t in (self_f, src_f, idx, self_i, src_i))
    with aten.use_flagops():
        res = {}
        names = _kernel_names(lambda: res.setdefault(
            "r", sd.scatter_reduce(0, idd, srd, "amax", include_self=False)))
        assert any("fo::" in n for n in names), names
        ref = oracle.scatter_reduce(self_f, 0, idx, src_f, "amax", include_self=False)
        assert torch.equal(res["r"].cpu(), ref)
        # in place and out=, exact int32 sums
        a = sid.clone()
        a.scatter_reduce_(0, idd, srid, "sum")
        assert torch.equal(a.cpu(), oracle.scatter_reduce(self_i, 0, idx, src_i, "sum"))
        out = torch.empty_like(sid)
        torch.scatter_reduce(sid, 0, idd, srid, "sum", include_self=False, out=out)
        assert torch.equal(out.cpu(), oracle.scatter_reduce(self_i, 0, idx, src_i, "sum",
                                                            include_self=False))
        r2 = torch.ops.flagops.scatter_reduce(sd, 0, idd, srd, "amin", True)
        assert torch.equal(r2.cpu(), oracle.scatter_reduce(self_f, 0, idx, src_f, "amin"))
    names = _kernel_names(lambda: sd.scatter_reduce(0, idd, srd, "amax"))
    assert not any("fo::" in n for n in names), names
