"""Generates tests/golden/*.npz from the reference implementation itself.

    python tests/golden/make_golden.py --ref <checkout of the reference>
    (or FLAGOPS_REFERENCE=<checkout> python tests/golden/make_golden.py)

Imports the reference's operators.* modules (iamsuperfly/Flag-Operators) and
runs their public functions on CPU tensors, i.e. the reference's CPU branch,
on seeded inputs plus the known-answer vectors of the reference's own tests.
Inputs and outputs are stored so the fixtures stand alone (the reference is not
needed to run the tests).  bf16 tensors are stored as their uint16 bit
patterns under a "<name>__bf16" key.

Run in its own process: the reference package is also called `operators`.
"""
from __future__ import annotations

import argparse
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))


def _np(t: torch.Tensor):
    t = t.detach().cpu()
    if t.dtype == torch.bfloat16:
        return t.view(torch.int16).numpy().view(np.uint16), "__bf16"
    return t.numpy(), ""


def _save(name: str, **tensors):
    out = {}
    for k, v in tensors.items():
        if isinstance(v, torch.Tensor):
            arr, suf = _np(v)
            out[k + suf] = arr
        else:
            out[k + "__s"] = np.asarray(v)   # plain scalar parameter
    path = os.path.join(HERE, name + ".npz")
    np.savez_compressed(path, **out)
    print(f"wrote {path} ({os.path.getsize(path)} bytes)")


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=os.environ.get("FLAGOPS_REFERENCE"),
                    help="checkout of iamsuperfly/Flag-Operators (or set FLAGOPS_REFERENCE)")
    args = ap.parse_args()
    if not args.ref:
        ap.error("give the reference checkout with --ref or FLAGOPS_REFERENCE")
    sys.path.insert(0, args.ref)
    from operators.rms_norm import rms_norm_forward            # reference module
    from operators.median import median
    from operators.scatter_reduce import scatter_reduce, scatter_reduce_, scatter_reduce_out
    from operators.fused_cross_entropy import fused_cross_entropy
    from operators.chunk_gated_delta_rule import chunk_gated_delta_rule

    g = torch.Generator().manual_seed(1234)

    # ---------------- rms_norm (reference CPU branch, rms_norm.py:209-216)
    cases = {}
    for i, (shape, dtype, eps) in enumerate([((16, 512), torch.float32, 1e-6),
                                             ((4, 1001), torch.float32, 1e-5),
                                             ((8, 1024), torch.bfloat16, 1e-6),
                                             ((3, 4, 256), torch.float32, 1e-5)]):
        x = torch.randn(*shape, generator=g).to(dtype)
        w = (1 + 0.1 * torch.randn(shape[-1], generator=g)).to(dtype)
        y, inv = rms_norm_forward(x, (shape[-1],), w, eps=eps)
        cases.update({f"x{i}": x, f"w{i}": w, f"y{i}": y, f"inv{i}": inv, f"eps{i}": eps})
    ones = torch.ones(4, 128)
    y1, _ = rms_norm_forward(ones, (128,), torch.ones(128))
    cases.update({"ones_x": ones, "ones_y": y1})
    _save("rms_norm", n_cases=4, **cases)

    # ---------------- median (median.py:348-352 -> torch.median on CPU)
    cases = {}
    xa = torch.randn(16, 2048, generator=g)
    xb = torch.randint(-64, 64, (16, 2048), generator=g).float()
    xc = torch.randn(64, 257, generator=g)
    specials = torch.tensor([[0.0, -0.0, 0.0, -0.0, 1.0],
                             [float("nan"), 1.0, float("nan"), 0.0, 2.0],
                             [3.0, 2.0, 1.0, float("nan"), 5.0],
                             [5.0, 5.0, 5.0, 5.0, 5.0],
                             [-1.0, float("-inf"), float("inf"), 0.5, -0.5]])
    for name, x in (("a", xa), ("b", xb), ("c", xc), ("s", specials)):
        r = median(x, dim=-1)
        cases.update({f"x_{name}": x, f"v_{name}": r.values, f"i_{name}": r.indices})
    x3 = torch.randn(4, 8, 16, generator=g)
    for d in (0, 1, 2):
        r = median(x3, dim=d)
        cases.update({f"v3_{d}": r.values, f"i3_{d}": r.indices})
    cases["x3"] = x3
    known = [[3.0, 1.0, 4.0, 1.0, 5.0], [1.0, 2.0, 3.0, 4.0], [42.0], [-5.0, -1.0, -3.0],
             [7.0] * 16, [2.0, 8.0]]
    for i, kv in enumerate(known):
        t = torch.tensor(kv)
        cases[f"kx{i}"] = t
        cases[f"kv{i}"] = median(t)
    gx = torch.randn(4, 128, 128, generator=g)
    cases.update({"gx": gx, "gv": median(gx)})
    _save("median", n_known=len(known), **cases)

    # ---------------- scatter_reduce (scatter_reduce.py:397-398, 427-429, 457-459)
    cases = {}
    n_self, n_src = 1024, 16384
    self1 = torch.randn(n_self, generator=g)
    src1 = torch.randn(n_src, generator=g)
    idx_u = torch.randint(0, n_self, (n_src,), generator=g)
    r = torch.arange(1, n_self + 1, dtype=torch.float64)
    p = r.pow(-1.1)
    cdf = torch.cumsum(p / p.sum(), 0)
    idx_z = torch.searchsorted(cdf, torch.rand(n_src, generator=g, dtype=torch.float64)).clamp(
        max=n_self - 1)
    cases.update({"self1": self1, "src1": src1, "idx_u": idx_u, "idx_z": idx_z})
    for dist, idx in (("u", idx_u), ("z", idx_z)):
        for red in ("sum", "prod", "amax", "amin", "mean"):
            for inc in (True, False):
                out = scatter_reduce(self1, 0, idx, src1, red, include_self=inc)
                cases[f"o_{dist}_{red}_{int(inc)}"] = out
    self_i = torch.randint(-100, 100, (n_self,), generator=g, dtype=torch.int32)
    src_i = torch.randint(-100, 100, (n_src,), generator=g, dtype=torch.int32)
    cases.update({"self_i": self_i, "src_i": src_i})
    for red in ("sum", "amax", "amin", "mean"):
        for inc in (True, False):
            cases[f"oi_{red}_{int(inc)}"] = scatter_reduce(self_i, 0, idx_u, src_i, red,
                                                           include_self=inc)
    # 2-D / 3-D along an inner dim, index smaller than src (as the reference tests)
    self2 = torch.rand(32, 16, generator=g) + 0.1
    src2 = torch.rand(32, 12, generator=g) + 0.1
    idx2 = torch.randint(0, 16, (32, 12), generator=g)
    self3 = torch.rand(8, 16, 8, generator=g) + 0.1
    src3 = torch.rand(8, 12, 8, generator=g) + 0.1
    idx3 = torch.randint(0, 16, (8, 12, 8), generator=g)
    cases.update({"self2": self2, "src2": src2, "idx2": idx2,
                  "self3": self3, "src3": src3, "idx3": idx3})
    for red in ("sum", "prod", "amax", "amin", "mean"):
        for inc in (True, False):
            cases[f"o2_{red}_{int(inc)}"] = scatter_reduce(self2, 1, idx2, src2, red,
                                                           include_self=inc)
            cases[f"o3_{red}_{int(inc)}"] = scatter_reduce(self3, 1, idx3, src3, red,
                                                           include_self=inc)
    # in-place and out= variants on the 1-D uniform case
    ip = self1.clone()
    scatter_reduce_(ip, 0, idx_u, src1, "sum")
    cases["o_inplace_sum"] = ip
    o = torch.empty_like(self1)
    scatter_reduce_out(o, self1, 0, idx_u, src1, "amax")
    cases["o_out_amax"] = o
    # known answers of tests/test_scatter_reduce.py:94-135
    ka = scatter_reduce(torch.zeros(4), 0, torch.tensor([0, 0, 1, 2]),
                        torch.tensor([3.0, 5.0, 2.0, 7.0]), "amax", include_self=False)
    kp = scatter_reduce(torch.ones(3), 0, torch.tensor([0, 0, 1]), torch.tensor([2.0, 3.0, 4.0]),
                        "prod")
    km = scatter_reduce(torch.zeros(3), 0, torch.tensor([0, 0, 1, 2]),
                        torch.tensor([1.0, 3.0, 2.0, 5.0]), "mean", include_self=False)
    kn = scatter_reduce(torch.tensor([0.0, 1.0, 2.0]), 0, torch.tensor([0, 1, 1]),
                        torch.tensor([float("nan"), 3.0, -1.0]), "amax")
    cases.update({"k_amax": ka, "k_prod": kp, "k_mean": km, "k_nan_amax": kn})
    _save("scatter_reduce", **cases)

    # ---------------- fused_cross_entropy (fused_cross_entropy.py:327-331)
    cases = {}
    B, V = 16, 1000
    lg = torch.randn(B, V, generator=g) * 2
    tg = torch.randint(0, V, (B,), generator=g)
    tg[3] = -100
    tg[7] = -100
    cases.update({"lg": lg, "tg": tg})
    for red in ("none", "mean", "sum"):
        for ls in (0.0, 0.1):
            x = lg.clone().requires_grad_(True)
            loss = fused_cross_entropy(x, tg, reduction=red, label_smoothing=ls)
            loss.backward(torch.ones_like(loss))
            cases[f"loss_{red}_{ls}"] = loss.detach()
            cases[f"grad_{red}_{ls}"] = x.grad
    lgb = (torch.randn(8, 4096, generator=g) * 2).bfloat16()
    tgb = torch.randint(0, 4096, (8,), generator=g)
    tgb[0] = -100
    x = lgb.clone().requires_grad_(True)
    loss = fused_cross_entropy(x, tgb)
    loss.backward()
    cases.update({"lgb": lgb, "tgb": tgb, "lossb": loss.detach(), "gradb": x.grad})
    allign = fused_cross_entropy(torch.randn(8, 100, generator=g),
                                 torch.full((8,), -100, dtype=torch.long))
    cases["all_ignored"] = allign
    _save("fused_cross_entropy", **cases)

    # ---------------- chunk_gated_delta_rule (CPU branch -> _ref_forward)
    cases = {}

    def make(Bn, Hn, L, D, dtype):
        q = torch.randn(Bn, Hn, L, D, generator=g)
        k = torch.randn(Bn, Hn, L, D, generator=g)
        k = k / k.norm(dim=-1, keepdim=True).clamp(min=1e-6)
        v = torch.randn(Bn, Hn, L, D, generator=g)
        beta = torch.sigmoid(torch.randn(Bn, Hn, L, generator=g))
        gg = torch.sigmoid(torch.randn(Bn, Hn, L, generator=g))
        return [t.to(dtype) for t in (q, k, v, beta, gg)]

    for i, (shape, dtype) in enumerate([((1, 2, 64, 16), torch.float32),
                                        ((2, 1, 100, 64), torch.float32),
                                        ((1, 1, 192, 128), torch.bfloat16)]):
        q, k, v, beta, gg = make(*shape, dtype)
        o = chunk_gated_delta_rule(q, k, v, beta, gg)
        cases.update({f"q{i}": q, f"k{i}": k, f"v{i}": v, f"beta{i}": beta, f"g{i}": gg,
                      f"o{i}": o})
        if i == 1:   # gate = 0 resets the state every step
            o0 = chunk_gated_delta_rule(q, k, v, beta, torch.zeros_like(gg))
            cases["o_gate0"] = o0
    # known answer, tests/test_chunk_gated_delta_rule.py:134-146
    q = torch.ones(1, 1, 1, 8)
    k = torch.zeros(1, 1, 1, 8); k[..., 0] = 1.0
    v = torch.zeros(1, 1, 1, 8); v[..., 0] = 2.0
    o = chunk_gated_delta_rule(q, k, v, torch.ones(1, 1, 1), torch.zeros(1, 1, 1))
    cases["known_o"] = o
    _save("chunk_gated_delta_rule", n_cases=3, **cases)


if __name__ == "__main__":
    main()
