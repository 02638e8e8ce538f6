"""chunk_gated_delta_rule parity vs the oracle (the reference's fp32 sequential
recurrence, _ref_forward).

Tolerance (target spec): bf16 rtol 2e-2 against the fp32 recurrence; the check
is |got - ref| <= 2e-2 |ref| + 2e-2 rms(ref) per element (the absolute term
covers outputs near zero).  fp32 inputs on the per-step kernel: 1e-4.
"""
import pytest
import torch

import oracle
from conftest import load_golden
from operators import _lib
from operators.chunk_gated_delta_rule import chunk_gated_delta_rule, timeouts

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _make(B, H, L, D, dtype=torch.bfloat16, seed=0):
    gen = torch.Generator().manual_seed(seed)
    q = torch.randn(B, H, L, D, generator=gen)
    k = torch.randn(B, H, L, D, generator=gen)
    k = k / k.norm(dim=-1, keepdim=True).clamp(min=1e-6)
    v = torch.randn(B, H, L, D, generator=gen)
    beta = torch.sigmoid(torch.randn(B, H, L, generator=gen))
    g = torch.sigmoid(torch.randn(B, H, L, generator=gen))
    return [t.to(dtype) for t in (q, k, v, beta, g)]


def _close(got, ref, rtol=2e-2):
    got, ref = got.float().cpu(), ref.float().cpu()
    rms = ref.pow(2).mean().sqrt().item()
    err = (got - ref).abs()
    bound = rtol * ref.abs() + rtol * rms
    worst = (err / bound.clamp(min=1e-30)).max().item()
    assert bool((err <= bound).all()), f"max err {err.max().item():.3e} (rms {rms:.3e}, " \
                                       f"worst ratio {worst:.2f})"


def _run(inputs, **kw):
    return chunk_gated_delta_rule(*[t.to(DEV) for t in inputs], **kw)


@pytest.mark.parametrize("N,K", [(64, 64), (64, 128), (128, 64), (128, 128)])
@pytest.mark.parametrize("a_mn", [0, 1])
@pytest.mark.parametrize("b_mn", [0, 1])
def test_tcgen05_operand_layouts(N, K, a_mn, b_mn):
    """The K-major / MN-major 128B-swizzle descriptors used by the kernel."""
    A = torch.randn(128, K, device=DEV).bfloat16()
    Bm = torch.randn(N, K, device=DEV).bfloat16()
    d = torch.empty(128, N, device=DEV)
    a_in = A.t().contiguous() if a_mn else A
    b_in = Bm.t().contiguous() if b_mn else Bm
    _lib.call("fo_tc05_selftest", _lib.ptr(a_in), _lib.ptr(b_in), _lib.ptr(d), N, K, a_mn, b_mn,
              _lib.stream_of(d))
    ref = A.float() @ Bm.float().t()
    torch.testing.assert_close(d, ref, rtol=1e-4, atol=1e-3)


def test_golden_fixtures():
    z = load_golden("chunk_gated_delta_rule")
    for i in range(z["n_cases"]):
        ins = [z[f"{n}{i}"] for n in ("q", "k", "v", "beta", "g")]
        got = _run(ins)
        if ins[0].dtype == torch.float32:
            torch.testing.assert_close(got.cpu(), z[f"o{i}"], rtol=1e-4, atol=1e-4)
        else:
            _close(got, z[f"o{i}"])
    ins = [z[f"{n}1"] for n in ("q", "k", "v", "beta")] + [torch.zeros_like(z["g1"])]
    torch.testing.assert_close(_run(ins).cpu(), z["o_gate0"], rtol=1e-4, atol=1e-4)


@pytest.mark.parametrize("L", [1, 2, 63, 64, 65, 128, 200, 512])
def test_tensor_core_path_lengths(L):
    ins = _make(1, 3, L, 128)
    o, h = _run(ins, output_final_state=True)
    ref_o, ref_h = oracle.delta_rule_forward(*ins, output_final_state=True)
    _close(o, ref_o)
    _close(h, ref_h)
    assert timeouts() == 0


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_tensor_core_dtypes_and_fp32_gates(dtype):
    q, k, v, beta, g = _make(2, 2, 256, 128, dtype)
    _close(_run([q, k, v, beta, g]), oracle.delta_rule_forward(q, k, v, beta, g))
    b32, g32 = beta.float(), g.float()
    _close(_run([q, k, v, b32, g32]), oracle.delta_rule_forward(q, k, v, b32, g32))


def test_baseline_config():
    """B=8, H=16, L=8192, D=128 bf16: five heads spread over the batch against the
    oracle, all heads against the independent per-step CUDA kernel (fp32 state)."""
    B, H, L, D = 8, 16, 8192, 128
    ins = _make(B, H, L, D, seed=3)
    dins = [t.to(DEV) for t in ins]
    o, h = chunk_gated_delta_rule(*dins, output_final_state=True)
    sel = [(0, 0), (1, 5), (3, 9), (5, 2), (7, 15)]
    for b, hh in sel:
        sub = [t[b:b + 1, hh:hh + 1] for t in ins]
        ro, rh = oracle.delta_rule_forward(*sub, output_final_state=True)
        _close(o[b:b + 1, hh:hh + 1], ro)
        _close(h[b:b + 1, hh:hh + 1], rh)
    o2 = torch.empty_like(dins[0])
    h2 = torch.empty(B, H, D, D, device=DEV)
    _lib.call("fo_gdr_fwd_stepwise", *[_lib.ptr(t) for t in dins], None, _lib.ptr(o2),
              _lib.ptr(h2), B, H, L, D, _lib.dtype_code(torch.bfloat16),
              _lib.dtype_code(torch.bfloat16), _lib.stream_of(o2))
    _close(o, o2)
    _close(h, h2)
    assert timeouts() == 0


def test_initial_state_chaining():
    ins = _make(1, 2, 300, 128, seed=5)
    o, h = _run(ins, output_final_state=True)
    s = 130
    a = [t[:, :, :s] for t in ins]
    b = [t[:, :, s:] for t in ins]
    o1, h1 = _run(a, output_final_state=True)
    o2, h2 = _run(b, initial_state=h1, output_final_state=True)
    _close(torch.cat([o1, o2], 2), o)
    _close(h2, h)
    ref_o, _ = oracle.delta_rule_forward(*[t for t in b], initial_state=h1.cpu(),
                                         output_final_state=True)
    _close(o2, ref_o)


@pytest.mark.parametrize("case", ["g0", "beta0", "g_near_one", "beta_high", "neg_gates",
                                  "mixed_zero_gates"])
def test_gate_edge_cases(case):
    q, k, v, beta, g = _make(1, 2, 160, 128, torch.bfloat16, seed=7)
    if case == "g0":
        g = torch.zeros_like(g)
    elif case == "beta0":
        beta = torch.zeros_like(beta)
    elif case == "g_near_one":
        g = torch.full_like(g, 0.999)
    elif case == "beta_high":
        beta = torch.full_like(beta, 0.99)
    elif case == "neg_gates":
        g = (torch.rand(g.shape) * 1.8 - 0.9).to(g.dtype)
    else:
        g = g.clone()
        g[..., ::7] = 0
    got = _run([q, k, v, beta, g])
    if case == "beta0":
        assert got.abs().max().item() < 1e-5
    _close(got, oracle.delta_rule_forward(q, k, v, beta, g))


def _flags_of(ins):
    """Runs the C ABI directly and returns (o, hT, per-head range flags)."""
    import ctypes
    dins = [t.to(DEV) for t in ins]
    B, H, L, D = dins[0].shape
    o = torch.empty_like(dins[0])
    hT = torch.empty(B, H, D, D, device=DEV)
    n = ctypes.c_int64(0)
    _lib.call("fo_gdr_workspace_bytes", B, H, L, D, _lib.dtype_code(dins[0].dtype),
              ctypes.byref(n))
    ws = torch.full((n.value // 4,), -1, dtype=torch.int32, device=DEV)
    _lib.call("fo_gdr_fwd", *[_lib.ptr(t) for t in dins], None, _lib.ptr(o), _lib.ptr(hT),
              B, H, L, D, _lib.dtype_code(dins[0].dtype), _lib.dtype_code(dins[3].dtype),
              _lib.ptr(ws), n.value, _lib.stream_of(o))
    return o, hT, ws.cpu()[:B * H]   # the per-head range flags lead the workspace


@pytest.mark.parametrize("case", ["v_1e5", "q_1e5", "persistent_gates"])
def test_fp16_range_guard(case):
    """bf16 inputs whose values, or whose state, leave the fp16 range of the
    tensor-core operand tiles: the result still matches the fp32 recurrence and
    is finite.  Head 0 holds the large values; head 1 is ordinary and must stay
    on the tensor-core path (its range flag stays 0)."""
    L = 2048
    q, k, v, beta, g = [t.float() for t in _make(1, 2, L, 128, torch.bfloat16, seed=11)]
    if case == "v_1e5":
        v[:, 0] *= 1e5
    elif case == "q_1e5":
        q[:, 0] *= 1e5
    else:
        g[:, 0] = 0.9999
        beta[:, 0] = 1.0
        v[:, 0] *= 3e3
    ins = [t.bfloat16() for t in (q, k, v, beta, g)]
    o, hT, flags = _flags_of(ins)
    ref_o, ref_h = oracle.delta_rule_forward(*ins, output_final_state=True)
    assert bool(torch.isfinite(o).all()) and bool(torch.isfinite(hT).all())
    for hh in range(2):
        _close(o[:, hh], ref_o[:, hh])
        _close(hT[:, hh], ref_h[:, hh])
    assert flags[1].item() == 0, "an ordinary head left the tensor-core path"
    assert flags[0].item() in (0, 1)


def test_fp16_range_guard_flags_only_the_overflowing_head():
    q, k, v, beta, g = [t.float() for t in _make(1, 3, 256, 128, torch.bfloat16, seed=12)]
    v[:, 1] *= 1e5
    ins = [t.bfloat16() for t in (q, k, v, beta, g)]
    o, hT, flags = _flags_of(ins)
    assert flags.tolist() == [0, 1, 0]
    ref_o, ref_h = oracle.delta_rule_forward(*ins, output_final_state=True)
    _close(o, ref_o)
    _close(hT, ref_h)


@pytest.mark.parametrize("D", [16, 32, 64])
@pytest.mark.parametrize("L", [1, 63, 64, 65, 200, 512])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_tensor_core_path_small_head_dims(D, L, dtype):
    """D < 128 runs the tensor-core kernels with channels D..127 zero-filled by
    the tensor maps: outputs and the D x D state against the oracle, from a
    nonzero initial state."""
    ins = _make(2, 3, L, D, dtype, seed=7 * D + L)
    h0 = torch.randn(2, 3, D, D, generator=torch.Generator().manual_seed(L)) * 0.1
    o, hT = _run(ins, initial_state=h0.to(DEV), output_final_state=True)
    ref_o, ref_h = oracle.delta_rule_forward(*ins, initial_state=h0, output_final_state=True)
    assert o.shape == (2, 3, L, D) and hT.shape == (2, 3, D, D)
    _close(o, ref_o)
    _close(hT, ref_h)


def test_small_head_dims_launch_the_tensor_core_kernels():
    from torch.profiler import ProfilerActivity, profile
    ins = [t.to(DEV) for t in _make(1, 2, 256, 64, seed=3)]
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        chunk_gated_delta_rule(*ins)
        torch.cuda.synchronize()
    names = " ".join(e.name for e in prof.events())
    assert "gdr_tinv_kernel" in names and "gdr_tc_kernel" in names, names[:400]


@pytest.mark.parametrize("D", [16, 32, 64, 128])
@pytest.mark.parametrize("L", [8, 64, 256])
def test_stepwise_path_fp32(D, L):
    ins = _make(2, 2, L, D, torch.float32, seed=D + L)
    got = _run(ins)
    torch.testing.assert_close(got.cpu(), oracle.delta_rule_forward(*ins), rtol=1e-4, atol=1e-4)


def test_reference_matrix_small_d():
    for D in (16, 32, 64):
        for L in (8, 16, 32, 64):
            for B, H in ((1, 1), (2, 4)):
                ins = _make(B, H, L, D, torch.float32, seed=B * H + L)
                torch.testing.assert_close(_run(ins).cpu(), oracle.delta_rule_forward(*ins),
                                           rtol=1e-3, atol=1e-3)


def test_shapes_and_assertions():
    ins = _make(3, 4, 20, 64, torch.float32)
    assert _run(ins).shape == (3, 4, 20, 64)
    bad = _make(1, 1, 4, 48, torch.float32)
    with pytest.raises(AssertionError, match="not in supported set"):
        _run(bad)
