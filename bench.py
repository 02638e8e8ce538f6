"""Benchmark of the five-operator kernel set on B200 (one JSON line on stdout).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--op NAME]
    torchrun --nproc-per-node N bench.py --gpus N ...       (N > 1)

Headline (`value`): the median workload of the target spec, x fp32 [8192, 2048]
~ N(0,1), values + indices along dim -1; metric = algorithmic HBM GB/s.  A step
is one median call; inputs stay resident in HBM and L2 is flushed before every
timed step (the input, 64 MiB, would otherwise sit in the 126 MB L2).
`e2e` is the same metric through the public API with pinned host buffers: the
host->device copy of x and the device->host copy of values and indices are inside
the timed region.  `per_op` holds every other configuration of the spec
(rms_norm fp32/bf16, median b/c, scatter_reduce variants, cross-entropy fwd+bwd,
the delta rule), each with its own roofline and CPU baseline.

--impl reference times the reference's CPU implementation of the path (the
oracle, i.e. the reference's torch CPU branch) on the host cores for the same
workload and metric.  Multi-GPU: one process per GPU; each rank runs the full
per-GPU workload (weak scaling, no collective on the data path); time = max over
ranks.  With N > 1, per_op also holds each workload split over the ranks
(strong scaling): rms_norm and median rows, cross-entropy rows (two one-float
all-reduces) and vocabulary columns (all-gather of row statistics), delta-rule
heads; each of those lines checks its rank's shard against the oracle and
reports `parity` ("ok" or "FAIL ..."); a failure makes the exit status 1.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

REPO = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(REPO, "flag-operators_b200")
for _p in (PKG, REPO):
    if _p not in sys.path:
        sys.path.insert(0, _p)

import torch  # noqa: E402

PEAKS_PATH = os.path.join(REPO, "MEASURED_PEAKS.json")
TRAFFIC_PATH = os.path.join(REPO, "profiles", "traffic.txt")
FALLBACK_HBM, FALLBACK_BF16 = 6650.0, 1590.0


def load_peaks():
    try:
        with open(PEAKS_PATH) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), float(p["bf16_tflops"]), "measured"
    except Exception:
        return FALLBACK_HBM, FALLBACK_BF16, "fallback"


def load_traffic():
    """profiles/traffic.txt: '<workload> <dram bytes per launch>' lines from ncu."""
    out = {}
    try:
        for line in open(TRAFFIC_PATH):
            line = line.split("#")[0].strip()
            if line:
                k, v = line.split()[:2]
                out[k] = float(v)
    except OSError:
        pass
    return out


# ---------------------------------------------------------------------------
# workloads (seeded synthetic inputs of the target spec's shapes/distributions)
# ---------------------------------------------------------------------------
def _gen(seed):
    return torch.Generator().manual_seed(seed)


def median_inputs(cfg):
    g = _gen(0)
    if cfg == "a":
        return torch.randn(8192, 2048, generator=g)
    if cfg == "b":
        return torch.randint(-64, 64, (8192, 2048), generator=g).float()
    return torch.randn(65536, 257, generator=g)


def median_bytes(x):
    M, N = x.shape
    return M * N * x.element_size() + M * (x.element_size() + 8)


def rms_inputs(cfg):
    g = _gen(0)
    shape, dt = ((4096, 4096), torch.float32) if cfg == "fp32" else ((16384, 8192), torch.bfloat16)
    x = torch.randn(*shape, generator=g).to(dt)
    w = (1 + 0.1 * torch.randn(shape[1], generator=g)).to(dt)
    return x, w


def rms_bytes(x):
    M, N = x.shape
    e = x.element_size()
    return 2 * M * N * e + N * e + M * 4


def rms_bwd_bytes(x):
    """read x, dy, inv_rms, weight; write dx, dw."""
    M, N = x.shape
    e = x.element_size()
    return 3 * M * N * e + 2 * N * e + M * 4


def scatter_inputs():
    g = _gen(0)
    n_self, n_src = 1 << 20, 1 << 24
    self_ = torch.randn(n_self, generator=g)
    src = torch.randn(n_src, generator=g)
    idx_u = torch.randint(0, n_self, (n_src,), generator=g)
    r = torch.arange(1, n_self + 1, dtype=torch.float64)
    cdf = torch.cumsum(r.pow(-1.1) / r.pow(-1.1).sum(), 0)
    idx_z = torch.searchsorted(cdf, torch.rand(n_src, generator=g, dtype=torch.float64)).clamp(
        max=n_self - 1)
    src_i = torch.randint(-100, 100, (n_src,), generator=g, dtype=torch.int32)
    return self_, src, idx_u, idx_z, src_i


SCATTER_BYTES = (1 << 24) * 4 + (1 << 24) * 8 + (1 << 20) * 4 * 2


CE_ROWS = 8192   # --ce-batch: a smaller batch of the same rows, for profiler captures


def ce_inputs():
    g = _gen(0)
    B, V = CE_ROWS, 128256
    logits = (2.0 * torch.randn(B, V, generator=g)).bfloat16()
    target = torch.randint(0, V, (B,), generator=g)
    target[torch.rand(B, generator=g) < 0.05] = -100
    return logits, target


def delta_inputs(B=8, H=16, L=8192, D=128):
    g = _gen(0)
    q = torch.randn(B, H, L, D, generator=g)
    k = torch.randn(B, H, L, D, generator=g)
    k = k / k.norm(dim=-1, keepdim=True).clamp(min=1e-6)
    v = torch.randn(B, H, L, D, generator=g)
    beta = torch.sigmoid(torch.randn(B, H, L, generator=g))
    gg = torch.sigmoid(torch.randn(B, H, L, generator=g))
    return [t.bfloat16() for t in (q, k, v, beta, gg)]


def delta_bytes(B=8, H=16, L=8192, D=128):
    return 4 * B * H * L * D * 2 + 2 * B * H * L * 2 + B * H * D * D * 4


def delta_flops(B=8, H=16, L=8192, D=128, C=64):
    return B * H * L * 2 * (4 * C * D + 3 * D * D)


# ---------------------------------------------------------------------------
# timing helpers
# ---------------------------------------------------------------------------
class Flusher:
    """Evicts the inputs from L2 (126 MB) between steps: writes a 256 MiB buffer,
    then reads a second 256 MiB buffer, so the dirty lines of the write are
    written back here, outside the timed region, and L2 ends full of clean lines
    of neither the inputs nor the outputs."""

    def __init__(self, dev):
        n = 256 * 1024 * 1024 // 4
        self.wbuf = torch.empty(n, dtype=torch.float32, device=dev)
        self.rbuf = torch.ones(n, dtype=torch.float32, device=dev)
        self.sink = torch.empty((), dtype=torch.float32, device=dev)

    def __call__(self):
        self.wbuf.fill_(1.0)
        torch.sum(self.rbuf, dim=0, out=self.sink)


# GPU-side spin enqueued before each timed step's start event, outside the timed
# region: while the GPU spins, the host enqueues the whole step, so the events
# never time a GPU waiting for the host's launches (which happened when several
# ranks' Python launch paths shared the host cores).  ~0.5 ms at 1.9 GHz.
_HOST_COVER_CYCLES = 1_000_000


def time_steps(fn, steps, warmup, flush=None, dist=None):
    """Sum of per-step CUDA-event times (ms) of `fn`, flush outside the events;
    barrier + synchronize on both sides; max over ranks."""
    for _ in range(warmup):
        if flush:
            flush()
        fn()
    torch.cuda.synchronize()
    if dist is not None:
        dist.barrier()
    torch.cuda.synchronize()
    evs = []
    for _ in range(steps):
        if flush:
            flush()
        torch.cuda._sleep(_HOST_COVER_CYCLES)
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        fn()
        e.record()
        evs.append((s, e))
    torch.cuda.synchronize()
    if dist is not None:
        dist.barrier()
    total = sum(s.elapsed_time(e) for s, e in evs)
    if dist is not None:
        t = torch.tensor([total], device="cuda", dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        total = float(t.item())
    return total


def cpu_time(fn, min_reps=3, min_seconds=1.0):
    fn()  # warm-up
    ts = []
    t_start = time.perf_counter()
    while len(ts) < min_reps or (time.perf_counter() - t_start) < min_seconds:
        t0 = time.perf_counter()
        fn()
        ts.append(time.perf_counter() - t0)
        if len(ts) >= 50:
            break
    return statistics.median(ts)


class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,utilization.gpu,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.proc = None
        self.idx = gpu_index
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={gpu_index}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
            out, _ = self.proc.communicate()
        rows = []
        for line in out.splitlines():
            p = [x.strip() for x in line.split(",")]
            if len(p) < 9:
                continue
            try:
                rows.append((float(p[1]), float(p[2]), float(p[4]), p[5:9]))
            except ValueError:
                continue
        if not rows:
            return None
        loaded = [r for r in rows if r[2] > 0] or rows
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in loaded for i, v in enumerate(r[3])
                          if v.lower().startswith("active")})
        return {"sm_mhz": statistics.median(r[0] for r in loaded),
                "sm_max_mhz": max(r[1] for r in rows), "reasons": reasons,
                "samples": len(loaded)}


# ---------------------------------------------------------------------------
# per-op measurements (our kernels)
# ---------------------------------------------------------------------------
def hbm_entry(name, nbytes, ms_total, steps, launches_per_step, peak_hbm, peak_src, traffic,
              cpu=None, extra=None):
    t = ms_total / steps / 1e3
    gbs = nbytes / t / 1e9
    e = {"metric": f"{name} HBM GB/s", "value": round(gbs, 1), "unit": "GB/s",
         "ms_per_step": round(ms_total / steps, 5),
         "roofline": {"bound": "hbm", "achieved": round(gbs, 1), "peak": peak_hbm,
                      "unit": "GB/s", "frac": round(gbs / peak_hbm, 4),
                      "traffic": traffic.get(name), "peak_source": peak_src,
                      "algorithmic_bytes": nbytes},
         "gpu_launches": launches_per_step * steps}
    if cpu:
        e["cpu_baseline"] = cpu
    if extra:
        e.update(extra)
    return e


def torch_threads():
    n = os.cpu_count() or 1
    torch.set_num_threads(n)
    return torch.get_num_threads()


def cpu_model():
    try:
        for line in open("/proc/cpuinfo"):
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def cpu_entry(fn, nbytes_or_units, unit, sample, kind="port", per="GB/s"):
    t = cpu_time(fn)
    val = nbytes_or_units / t / (1e9 if per == "GB/s" else 1.0)
    return {"value": round(val, 4), "unit": unit, "cores": torch.get_num_threads(), "kind": kind,
            "cpu": cpu_model(), "sample": sample}


def run_per_op(args, dev, peaks, traffic, do_cpu, dist=None):
    import oracle
    from operators.median import median
    from operators.rms_norm import rms_norm_backward, rms_norm_forward
    from operators.scatter_reduce import scatter_reduce
    from operators.fused_cross_entropy import fused_cross_entropy
    from operators.chunk_gated_delta_rule import chunk_gated_delta_rule
    hbm, tfl, src = peaks
    flush = Flusher(dev)
    K, W = args.steps, max(3, args.warmup)
    res = {}
    only = getattr(args, "only", None)

    def want(name):
        return only is None or name.startswith(only) or only.startswith(name)

    # rms_norm
    for cfg in ("fp32", "bf16"):
        if not want(f"rms_norm_{cfg}"):
            continue
        x, w = rms_inputs(cfg)
        xd, wd = x.to(dev), w.to(dev)
        ms = time_steps(lambda: rms_norm_forward(xd, (xd.shape[1],), wd, 1e-6), K, W, flush, dist)
        cpu = None
        if do_cpu:
            cpu = cpu_entry(lambda: oracle.rms_norm_forward(x, (x.shape[1],), w, 1e-6),
                            rms_bytes(x), "GB/s", f"full workload {tuple(x.shape)} {x.dtype}")
        res[f"rms_norm_{cfg}"] = hbm_entry(f"rms_norm_{cfg}", rms_bytes(x), ms, K, 1, hbm, src,
                                           traffic, cpu)
        del xd, wd

    # rms_norm backward (dx, dw) from inv_rms
    for cfg in ("fp32", "bf16"):
        if not want(f"rms_norm_bwd_{cfg}"):
            continue
        x, w = rms_inputs(cfg)
        dy = torch.randn(x.shape, generator=_gen(1)).to(x.dtype)
        xd, wd, dyd = x.to(dev), w.to(dev), dy.to(dev)
        _, invd = rms_norm_forward(xd, (xd.shape[1],), wd, 1e-6)
        ms = time_steps(lambda: rms_norm_backward(dyd, xd, invd, (xd.shape[1],), wd), K, W, flush,
                        dist)
        cpu = None
        if do_cpu:
            rows = 1024
            cpu = cpu_entry(lambda: oracle.rms_norm_backward(dy[:rows], x[:rows], (x.shape[1],), w,
                                                             1e-6),
                            rms_bwd_bytes(x[:rows]), "GB/s",
                            f"first {rows} of {x.shape[0]} rows (autograd through the CPU formula)")
        res[f"rms_norm_bwd_{cfg}"] = hbm_entry(f"rms_norm_bwd_{cfg}", rms_bwd_bytes(x), ms, K, 2, hbm,
                                               src, traffic, cpu)
        del xd, wd, dyd, invd

    # median a, b, c (a is also the headline)
    for cfg in (("a", "b", "c") if only else ("b", "c")):
        if not want(f"median_{cfg}"):
            continue
        x = median_inputs(cfg)
        xd = x.to(dev)
        ms = time_steps(lambda: median(xd, dim=-1), K, W, flush, dist)
        cpu = None
        if do_cpu:
            cpu = cpu_entry(lambda: oracle.median(x, dim=-1), median_bytes(x), "GB/s",
                            f"full workload {tuple(x.shape)}")
        res[f"median_{cfg}"] = hbm_entry(f"median_{cfg}", median_bytes(x), ms, K, 1, hbm, src,
                                         traffic, cpu)
        del xd

    # global median (dim=None) of the [8192, 2048] fp32 tensor: the grid-wide radix select
    if want("median_global"):
        x = median_inputs("a")
        xd = x.to(dev)
        ms = time_steps(lambda: median(xd), K, W, flush, dist)
        cpu = None
        if do_cpu:
            xs = x[:1024]
            cpu = cpu_entry(lambda: oracle.median(xs), xs.numel() * 4, "GB/s",
                            "first 1024 of 8192 rows, flattened")
        res["median_global"] = hbm_entry("median_global", x.numel() * 4 + 4, ms, K, 9, hbm, src,
                                         traffic, cpu)
        del xd

    # scatter_reduce
    if want("scatter"):
        self_, srcv, idx_u, idx_z, src_i = scatter_inputs()
        sd, srd, iud, izd, sid = (t.to(dev) for t in (self_, srcv, idx_u, idx_z, src_i))
        selfi_d = torch.zeros(1 << 20, dtype=torch.int32, device=dev)
        sub = 1 << 20   # CPU sample: first 1/16 of src/index, same self
        for dist_name, idx_d, idx_c in (("uniform", iud, idx_u), ("zipf", izd, idx_z)):
            for red in ("sum", "prod", "amax", "amin", "mean"):
                for inc in (True, False):
                    name = f"scatter_{dist_name}_{red}_{'self' if inc else 'noself'}"
                    if not want(name):
                        continue
                    ms = time_steps(lambda: scatter_reduce(sd, 0, idx_d, srd, red, include_self=inc),
                                    K, W, flush, dist)
                    cpu = None
                    if do_cpu:
                        sb = sub * 12 + (1 << 20) * 8
                        cpu = cpu_entry(lambda: oracle.scatter_reduce(self_, 0, idx_c[:sub],
                                                                      srcv[:sub], red,
                                                                      include_self=inc),
                                        sb, "GB/s", "first 2^20 of 2^24 index/src elements")
                    if red == "prod":
                        # destination binning: count, pairs, reduce (+ init and
                        # finalize of the cells without include_self)
                        launches = 3 if inc else 5
                    else:
                        launches = 1 if (red == "sum" and inc) else 3
                    res[name] = hbm_entry(name, SCATTER_BYTES, ms, K, launches, hbm, src, traffic,
                                          cpu)
        if want("scatter_uniform_int32_sum"):
            ms = time_steps(lambda: scatter_reduce(selfi_d, 0, iud, sid, "sum"), K, W, flush, dist)
            cpu = None
            if do_cpu:
                si = torch.zeros(1 << 20, dtype=torch.int32)
                cpu = cpu_entry(lambda: oracle.scatter_reduce(si, 0, idx_u[:sub], src_i[:sub], "sum"),
                                sub * 12 + (1 << 20) * 8, "GB/s", "first 2^20 of 2^24 elements")
            res["scatter_uniform_int32_sum"] = hbm_entry("scatter_uniform_int32_sum", SCATTER_BYTES,
                                                         ms, K, 1, hbm, src, traffic, cpu)
        del sd, srd, iud, izd, sid, selfi_d

    # fused cross-entropy forward + backward
    if want("ce_fwd_bwd"):
        logits, target = ce_inputs()
        ld, td = logits.to(dev), target.to(dev)
        B, V = logits.shape

        def ce_step():
            x = ld.detach().requires_grad_(True)
            loss = fused_cross_entropy(x, td)
            loss.backward()
            return x.grad

        ms = time_steps(ce_step, K, W, flush, dist)
        nbytes = 2 * B * V * 2 + B * 8 + B * 4 * 3
        cpu = None
        if do_cpu:
            rows = 512
            lsub, tsub = logits[:rows], target[:rows]
            cpu = cpu_entry(lambda: oracle.fused_cross_entropy_grad(lsub, tsub), 2 * rows * V * 2,
                            "GB/s", f"first {rows} of {B} rows, fwd+bwd")
        res["ce_fwd_bwd"] = hbm_entry(
            "ce_fwd_bwd", nbytes, ms, K, 4, hbm, src, traffic, cpu,
            {"note": "algorithmic bytes = one read of logits + one write of dlogits (fused fwd+bwd); "
                     "a recompute design needs 3 passes (6.30e9 B)",
             "effective_GBps_3pass": round(3 * B * V * 2 / (ms / K / 1e3) / 1e9, 1)})
        del ld, td, logits

    # delta rule
    if want("chunk_gated_delta_rule"):
        ins = delta_inputs()
        dins = [t.to(dev) for t in ins]
        ms = time_steps(lambda: chunk_gated_delta_rule(*dins, output_final_state=True), K, W, flush,
                        dist)
        t = ms / K / 1e3
        Bd, Hd, Ld, Dd = dins[0].shape
        toks = Bd * Ld / t
        nbytes, flops = delta_bytes(), delta_flops()
        # three kernels per call: chunk inverses, chunk scan, range-guard recompute
        e = hbm_entry("chunk_gated_delta_rule", nbytes, ms, K, 3, hbm, src, traffic)
        e.update({"metric": "chunk_gated_delta_rule tokens/s", "value": round(toks, 1),
                  "unit": "tokens/s (B*L per second)",
                  "tensor": {"achieved_tflops": round(flops / t / 1e12, 2), "peak_tflops": tfl,
                             "frac": round(flops / t / 1e12 / tfl, 4), "algorithmic_flops": flops}})
        if do_cpu:
            # the L=512 prefix of all B x H heads; the recurrence is linear in L
            Ls = 512
            sub_in = [(x[:, :, :Ls] if x.dim() == 3 else x[:, :, :Ls, :]).contiguous()
                      for x in ins]
            tc = cpu_time(lambda: oracle.delta_rule_forward(*sub_in, output_final_state=True),
                          min_reps=2, min_seconds=0.5)
            full_t = tc * (Ld / Ls)
            e["cpu_baseline"] = {"value": round(Bd * Ld / full_t, 3), "unit": "tokens/s",
                                 "cores": torch.get_num_threads(), "kind": "port",
                                 "cpu": cpu_model(),
                                 "sample": f"all {Bd}x{Hd} heads, L={Ls} prefix, scaled "
                                           f"linearly to L={Ld}"}
        res["chunk_gated_delta_rule"] = e
        del dins

    if want("chunk_gated_delta_rule_d64"):
        # head dimension 64 (the reference's own test matrix uses D <= 64): the
        # same tensor-core kernels with channels 64..127 zero-filled by TMA
        D64 = 64
        ins = delta_inputs(D=D64)
        dins = [t.to(dev) for t in ins]
        ms = time_steps(lambda: chunk_gated_delta_rule(*dins, output_final_state=True), K, W, flush,
                        dist)
        t = ms / K / 1e3
        Bd, Hd, Ld, Dd = dins[0].shape
        nbytes, flops = delta_bytes(D=D64), delta_flops(D=D64)
        e = hbm_entry("chunk_gated_delta_rule_d64", nbytes, ms, K, 3, hbm, src, traffic)
        e.update({"metric": "chunk_gated_delta_rule (D=64) tokens/s",
                  "value": round(Bd * Ld / t, 1), "unit": "tokens/s (B*L per second)",
                  "tensor": {"achieved_tflops": round(flops / t / 1e12, 2), "peak_tflops": tfl,
                             "frac": round(flops / t / 1e12 / tfl, 4), "algorithmic_flops": flops}})
        # the per-step CUDA-core kernel on the same inputs (the path D < 128 took
        # before), one call
        import ctypes
        from operators import _lib
        o2 = torch.empty_like(dins[0])
        s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s0.record()
        _lib.call("fo_gdr_fwd_stepwise", *[_lib.ptr(x) for x in dins], None, _lib.ptr(o2), None,
                  Bd, Hd, Ld, Dd, _lib.dtype_code(dins[0].dtype), _lib.dtype_code(dins[3].dtype),
                  _lib.stream_of(dins[0]))
        s1.record()
        torch.cuda.synchronize(dev)
        e["stepwise_kernel_ms"] = round(s0.elapsed_time(s1), 3)
        # parity: head 0 against the oracle's fp32 recurrence at the full length
        o, hT = chunk_gated_delta_rule(*dins, output_final_state=True)
        ro, rh = oracle.delta_rule_forward(*[x[:1, :1] for x in ins], output_final_state=True)
        ok1, d1 = _delta_close(o[:1, :1], ro)
        ok2, d2 = _delta_close(hT[:1, :1], rh)
        e["parity"] = "ok" if (ok1 and ok2) else f"FAIL head 0: o {d1}; state {d2}"
        res["chunk_gated_delta_rule_d64"] = e
        del dins, o2

    if want("chunk_gated_delta_rule_bwd"):
        # backward at the benchmark shape: one fo_gdr_bwd call (the kernel the
        # autograd Function runs) = dq, dk, dv, dbeta, dg from q, k, v, beta, g, do;
        # fp32 CUDA-core reverse scan with the states recomputed from 16-step
        # checkpoints
        from operators.chunk_gated_delta_rule import _backward
        ins = delta_inputs()
        dins = [t.to(dev) for t in ins]
        do_c = torch.randn(ins[0].shape, generator=_gen(1)).bfloat16()
        do_d = do_c.to(dev)
        ms = time_steps(lambda: _backward(*dins, None, do_d, None, False), K, W, flush, dist)
        t = ms / K / 1e3
        Bd, Hd, Ld, Dd = dins[0].shape
        n = Bd * Hd * Ld * Dd
        # read q, k, v, do and the gates; write dq, dk, dv and the gate gradients
        nbytes = 7 * n * 2 + 4 * Bd * Hd * Ld * 2
        e = hbm_entry("chunk_gated_delta_rule_bwd", nbytes, ms, K, 1, hbm, src, traffic)
        e.update({"metric": "chunk_gated_delta_rule backward tokens/s",
                  "value": round(Bd * Ld / t, 1), "unit": "tokens/s (B*L per second)",
                  "fp32_flops_per_call": 22 * Dd * Dd * Bd * Hd * Ld,
                  "note": "per-step fp32 CUDA-core kernel (no chunked tensor-core backward yet)"})
        if do_cpu:
            # autograd through the reference loop, L=64 prefix of all heads, scaled
            # linearly to L=8192
            Ls = 64
            sub = [(x[:, :, :Ls] if x.dim() == 3 else x[:, :, :Ls, :]).contiguous() for x in ins]
            tc = cpu_time(lambda: oracle.delta_rule_grads(*sub, do_c[:, :, :Ls]), min_reps=2,
                          min_seconds=0.5)
            e["cpu_baseline"] = {"value": round(Bd * Ld / (tc * Ld / Ls), 3), "unit": "tokens/s",
                                 "cores": torch.get_num_threads(), "kind": "port",
                                 "cpu": cpu_model(),
                                 "sample": f"autograd through the reference loop, all {Bd}x{Hd} "
                                           f"heads, L={Ls} prefix, scaled linearly to L={Ld}"}
        # parity: head 0, first 256 tokens, against autograd through the reference loop
        Lp = 256
        sl = [(x[:1, :1, :Lp] if x.dim() == 3 else x[:1, :1, :Lp, :]).contiguous() for x in ins]
        got = _backward(*[x.to(dev) for x in sl], None, do_c[:1, :1, :Lp].to(dev), None, False)
        ref = oracle.delta_rule_grads(*sl, do_c[:1, :1, :Lp])
        bad = []
        for name, gr in zip(("q", "k", "v", "beta", "g"), got[:5]):
            ok, d = _delta_close(gr, ref[name])
            if not ok:
                bad.append(f"d{name}: {d}")
        e["parity"] = "ok" if not bad else "FAIL head 0: " + "; ".join(bad)
        res["chunk_gated_delta_rule_bwd"] = e
        del dins, do_d
    return res


# ---------------------------------------------------------------------------
# strong-scaled splits over the ranks (N > 1), each with a parity check
# ---------------------------------------------------------------------------
def _bounds(n, rank, world):
    return rank * n // world, (rank + 1) * n // world


def _agree(dist, ok, detail):
    """'ok' when every rank passed, else 'FAIL <first failing rank's detail>'."""
    t = torch.tensor([0.0 if ok else 1.0], device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    if t.item() == 0.0:
        return "ok"
    return "FAIL " + (detail or "on another rank")


def _delta_close(got, ref, rtol=2e-2):
    got, ref = got.float().cpu(), ref.float().cpu()
    rms = ref.pow(2).mean().sqrt().item()
    err = (got - ref).abs()
    ok = bool((err <= rtol * ref.abs() + rtol * rms).all())
    return ok, f"max err {err.max().item():.3e} (rms {rms:.3e})"


SHARDED_LINES = ("rms_norm_bf16_rows", "median_a_rows", "ce_rows_sharded", "ce_vocab_sharded",
                 "delta_heads")


def run_sharded(args, dev, peaks, traffic, dist):
    """Each workload of the target spec split over the ranks (strong scaling):
    rms_norm and median rows, cross-entropy rows and vocabulary columns, delta
    rule heads.  value = bytes (tokens) of the whole workload / max-over-ranks
    time.  Every line checks its rank's shard against the oracle and reports
    `parity`; a failure makes bench.py exit non-zero."""
    import oracle
    from operators.median import median
    from operators.rms_norm import rms_norm_forward
    from operators.fused_cross_entropy import fused_cross_entropy
    from operators.chunk_gated_delta_rule import chunk_gated_delta_rule
    hbm, tfl, src = peaks
    P, rank = dist.get_world_size(), dist.get_rank()
    flush = Flusher(dev)
    K, W = args.steps, max(3, args.warmup)
    only = getattr(args, "only", None)
    res = {}

    def want(name):
        return only is None or name.startswith(only) or only.startswith(name)

    def line(name, nbytes, ms, launches, parity, extra=None):
        e = hbm_entry(name, nbytes, ms, K, launches, hbm * P, src, traffic)
        e.update({"scaling": "strong", "ranks": P, "parity": parity})
        if extra:
            e.update(extra)
        return e

    if want("rms_norm_bf16_rows"):
        x, w = rms_inputs("bf16")
        M, N = x.shape
        r0, r1 = _bounds(M, rank, P)
        xd, wd = x[r0:r1].contiguous().to(dev), w.to(dev)
        ms = time_steps(lambda: rms_norm_forward(xd, (N,), wd, 1e-6), K, W, flush, dist)
        y, _ = rms_norm_forward(xd, (N,), wd, 1e-6)
        rows = torch.arange(0, r1 - r0, 61)
        yr, _ = oracle.rms_norm_forward(x[r0:r1][rows], (N,), w, 1e-6)
        ok = bool(torch.allclose(y[rows.to(dev)].float().cpu(), yr.float(), rtol=2e-2, atol=2e-2))
        res["rms_norm_bf16_rows"] = line(
            "rms_norm_bf16_rows", rms_bytes(x), ms, 1,
            _agree(dist, ok, f"rank {rank} rms_norm rows"),
            {"shard": f"rows [{r0}, {r1}) of {M} on rank {rank} (each rank M/N rows)"})
        del xd, wd, y

    if want("median_a_rows"):
        x = median_inputs("a")
        M = x.shape[0]
        r0, r1 = _bounds(M, rank, P)
        xd = x[r0:r1].contiguous().to(dev)
        ms = time_steps(lambda: median(xd, dim=-1), K, W, flush, dist)
        got = median(xd, dim=-1)
        ref = oracle.median(x[r0:r1], dim=-1)
        ok = (torch.equal(got.values.cpu(), ref.values)
              and torch.equal(got.indices.cpu(), ref.indices))
        res["median_a_rows"] = line(
            "median_a_rows", median_bytes(x), ms, 1,
            _agree(dist, ok, f"rank {rank} median rows not bit-exact"),
            {"shard": f"rows [{r0}, {r1}) of {M} (each rank M/N rows)"})
        del xd

    if want("ce_rows_sharded") or want("ce_vocab_sharded"):
        lg, tg = ce_inputs()
        B, V = lg.shape
        tgd = tg.to(dev)
        nbytes = 2 * B * V * lg.element_size()       # one read + one write of B x V
        sample = torch.arange(0, B, 97)
        n_valid = int((tg != -100).sum())
        # oracle: full-batch loss on rank 0 (fp32 upcast), gradient rows sampled
        ref_loss = None
        if rank == 0:
            ref_loss = float(oracle.fused_cross_entropy(lg.float(), tg))
        _, gs = oracle.fused_cross_entropy_grad(lg[sample].float(), tg[sample], reduction="sum")
        gs = gs / n_valid

        def loss_ok(loss):
            t = torch.tensor([float(loss)], device=dev, dtype=torch.float64)
            lo, hi = t.clone(), t.clone()
            dist.all_reduce(lo, op=dist.ReduceOp.MIN)
            dist.all_reduce(hi, op=dist.ReduceOp.MAX)
            same = lo.item() == hi.item()
            if rank == 0:
                return same and abs(float(loss) - ref_loss) <= 2e-2 * abs(ref_loss), \
                    f"loss {float(loss):.6f} vs oracle {ref_loss:.6f}, ranks agree: {same}"
            return same, "ranks disagree on the loss"

        if want("ce_rows_sharded"):
            r0, r1 = _bounds(B, rank, P)
            lsh = lg[r0:r1].contiguous().to(dev)
            td = tgd[r0:r1].contiguous()

            def ce_rows():
                x = lsh.detach().requires_grad_(True)
                loss = fused_cross_entropy(x, td, process_group=dist.group.WORLD, shard="rows")
                loss.backward()
                return loss, x.grad

            ms = time_steps(lambda: ce_rows(), K, W, flush, dist)
            loss, grad = ce_rows()
            ok, det = loss_ok(loss.float().item())
            mine = sample[(sample >= r0) & (sample < r1)]
            if ok and mine.numel():
                ok = bool(torch.allclose(grad[(mine - r0).to(dev)].float().cpu(),
                                         gs[(sample >= r0) & (sample < r1)], rtol=2e-2,
                                         atol=2e-5 * float(gs.abs().max())))
                det = det if ok else f"rank {rank} gradient rows differ"
            res["ce_rows_sharded"] = line(
                "ce_rows_sharded", nbytes, ms, 4, _agree(dist, ok, det),
                {"shard": f"rows [{r0}, {r1}) of {B}, full vocabulary",
                 "collective": "all_reduce of the valid-row count, then of the loss sum (fp32)"})
            del lsh, grad

        if want("ce_vocab_sharded"):
            c0, c1 = _bounds(V, rank, P)
            lsh = lg[:, c0:c1].contiguous().to(dev)

            def ce_sh():
                x = lsh.detach().requires_grad_(True)
                loss = fused_cross_entropy(x, tgd, process_group=dist.group.WORLD,
                                           vocab_offset=c0, vocab_size=V)
                loss.backward()
                return loss, x.grad

            ms = time_steps(lambda: ce_sh(), K, W, flush, dist)
            loss, grad = ce_sh()
            ok, det = loss_ok(loss.float().item())
            if ok:
                ok = bool(torch.allclose(grad[sample.to(dev)].float().cpu(), gs[:, c0:c1],
                                         rtol=2e-2, atol=2e-5 * float(gs.abs().max())))
                det = det if ok else f"rank {rank} gradient block differs"
            from operators import fused_cross_entropy as fce
            fused = isinstance(fce._PEER.get((id(dist.group.WORLD), dev.index)),
                               fce._PeerRegions)
            res["ce_vocab_sharded"] = line(
                "ce_vocab_sharded", nbytes, ms, 3 if fused else 5, _agree(dist, ok, det),
                {"shard": f"columns [{c0}, {c1}) of {V}, all rows",
                 "collective": ("per-row (max, sum-exp, target logit, row sum) stored into every "
                                "rank's region over NVLink peer memory inside the fused kernel "
                                "(fo_ce_shard_p2p_fwd)") if fused else
                               "all_gather of per-row (max, sum-exp, target logit, row sum)",
                 "note": "algorithmic bytes = one read of the logits + one write of dlogits"})
            del lsh, grad
        del lg

    if want("delta_heads"):
        ins = delta_inputs()
        Bd, Hd, Ld, Dd = ins[0].shape
        nh = Bd * Hd
        h0, h1 = _bounds(nh, rank, P)

        def heads(t):
            return t.reshape(1, nh, *t.shape[2:])[:, h0:h1].contiguous()

        dins = [heads(t).to(dev) for t in ins]
        ms = time_steps(lambda: chunk_gated_delta_rule(*dins, output_final_state=True), K, W,
                        flush, dist)
        o, hT = chunk_gated_delta_rule(*dins, output_final_state=True)
        ro, rh = oracle.delta_rule_forward(*[heads(t)[:, :1] for t in ins],
                                           output_final_state=True)
        ok1, d1 = _delta_close(o[:, :1], ro)
        ok2, d2 = _delta_close(hT[:, :1], rh)
        t = ms / K / 1e3
        e = line("delta_heads", delta_bytes(), ms, 1,
                 _agree(dist, ok1 and ok2, f"rank {rank} head {h0}: o {d1}; state {d2}"),
                 {"shard": f"heads [{h0}, {h1}) of B*H = {nh} (each rank B*H/N heads)"})
        e.update({"metric": "chunk_gated_delta_rule tokens/s (heads split over ranks)",
                  "value": round(Bd * Ld / t, 1), "unit": "tokens/s (B*L per second)",
                  "tensor": {"achieved_tflops": round(delta_flops() / t / 1e12, 2),
                             "peak_tflops": tfl * P,
                             "frac": round(delta_flops() / t / 1e12 / (tfl * P), 4)}})
        res["delta_heads"] = e
        del dins
    return res


# ---------------------------------------------------------------------------
def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=30)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-per-op", action="store_true", help="headline only")
    ap.add_argument("--ce-batch", type=int, default=8192,
                    help="rows of the cross-entropy workload (default: the benchmark's 8192)")
    ap.add_argument("--only", default=None,
                    help="run one per-op workload (rms_norm_fp32, median_c, scatter, ce, "
                         "delta, ...) and print its entry; used for profiler captures")
    args = ap.parse_args()
    global CE_ROWS
    CE_ROWS = args.ce_batch
    if args.warmup < 3:
        args.warmup = 3

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    workload = {"workload": "median along dim=-1, x fp32 [8192, 2048] ~ N(0,1), values+indices",
                "global_batch": 8192 * world, "seq_len": 2048,
                "parallelism": f"rows replicated per rank x{world} (weak)",
                "l2": "flushed (256 MiB write) before every timed step"}

    if args.impl == "reference":
        if rank != 0:
            return
        import oracle
        n = torch_threads()
        x = median_inputs("a")
        nbytes = median_bytes(x)
        for _ in range(args.warmup):
            oracle.median(x, dim=-1)
        t0 = time.perf_counter()
        for _ in range(args.steps):
            oracle.median(x, dim=-1)
        dt = (time.perf_counter() - t0) / args.steps
        val = nbytes / dt / 1e9
        print(json.dumps({
            "impl": "reference", "metric": "median HBM GB/s", "value": round(val, 4),
            "unit": "GB/s", "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(dt * 1e3, 3), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded, spec shapes)",
            "config": workload,
            "cpu_baseline": {"value": round(val, 4), "unit": "GB/s", "cores": n, "kind": "port",
                             "cpu": cpu_model(),
                             "sample": "full workload per step (torch CPU median, the "
                                       "reference's CPU branch)"},
            "e2e": {"value": round(val, 4), "unit": "GB/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}))
        return

    dist = None
    sharded_only = bool(args.only) and args.only.startswith(SHARDED_LINES)
    if world > 1 or sharded_only:
        # --only <a sharded line> on one GPU runs that line with a single-rank
        # group (its kernels in one process, e.g. for a profiler capture)
        import torch.distributed as dist_mod
        torch.cuda.set_device(local)
        import datetime
        if world == 1:
            os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
            os.environ.setdefault("MASTER_PORT", "29561")
            os.environ.setdefault("RANK", "0")
            os.environ.setdefault("WORLD_SIZE", "1")
        dist_mod.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                    device_id=torch.device("cuda", local))
        dist = dist_mod
    dev = torch.device("cuda", local if world > 1 else 0)
    torch.cuda.set_device(dev)
    from operators import _lib
    from operators.median import median
    _lib.load()
    peaks = load_peaks()
    hbm, tfl, src = peaks
    traffic = load_traffic()
    sampler = ClockSampler(dev.index if world == 1 else local)

    if args.only:
        do_cpu = (rank == 0 and world == 1)
        per_op = {} if sharded_only else run_per_op(args, dev, peaks, traffic, do_cpu, dist)
        if dist is not None:
            per_op.update(run_sharded(args, dev, peaks, traffic, dist))
        clocks = sampler.stop()
        if rank == 0:
            print(json.dumps({"only": args.only, "per_op": per_op, "clocks": clocks}))
        if dist is not None:
            dist.barrier()
            dist.destroy_process_group()
        return 1 if _parity_failed(per_op) else 0

    # ---- headline: median (a), device-resident
    x = median_inputs("a")
    xd = x.to(dev)
    flush = Flusher(dev)
    nbytes = median_bytes(x)
    ms = time_steps(lambda: median(xd, dim=-1), args.steps, args.warmup, flush, dist)
    t = ms / args.steps / 1e3
    value = nbytes * world / t / 1e9

    # ---- e2e: pinned host input -> public API -> host outputs
    xh = x.pin_memory()
    vh = torch.empty(8192, dtype=torch.float32).pin_memory()
    ih = torch.empty(8192, dtype=torch.int64).pin_memory()
    xdev = torch.empty_like(xd)

    def e2e_step():
        xdev.copy_(xh, non_blocking=True)
        r = median(xdev, dim=-1)
        vh.copy_(r.values, non_blocking=True)
        ih.copy_(r.indices, non_blocking=True)

    ms_e2e = time_steps(e2e_step, args.steps, args.warmup, None, dist)
    t_e2e = ms_e2e / args.steps / 1e3
    e2e = {"value": round(nbytes * world / t_e2e / 1e9, 2), "unit": "GB/s",
           "h2d_bytes_per_step": x.numel() * 4, "d2h_bytes_per_step": 8192 * (4 + 8),
           "ms_per_step": round(ms_e2e / args.steps, 4)}

    do_cpu = (rank == 0 and world == 1)
    cpu = None
    if do_cpu:
        import oracle
        torch_threads()
        cpu = cpu_entry(lambda: oracle.median(x, dim=-1), nbytes, "GB/s",
                        "full workload (torch CPU median, the reference's CPU branch)")
    per_op = {} if args.no_per_op else run_per_op(args, dev, peaks, traffic, do_cpu, dist)
    if dist is not None and not args.no_per_op:
        per_op.update(run_sharded(args, dev, peaks, traffic, dist))
    clocks = sampler.stop()

    if rank == 0:
        gbs1 = nbytes / t / 1e9
        line = {
            "metric": "median HBM GB/s", "value": round(value, 1), "unit": "GB/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(ms / args.steps, 5), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded; shapes and distributions of the target spec)",
            "config": workload,
            "roofline": {"bound": "hbm", "achieved": round(gbs1, 1), "peak": hbm, "unit": "GB/s",
                         "frac": round(gbs1 / hbm, 4), "traffic": traffic.get("median_a"),
                         "peak_source": src, "algorithmic_bytes": nbytes},
            "cpu_baseline": cpu,
            "e2e": e2e,
            "gpu_launches": args.steps * (1 + 0),
            "clocks": clocks,
            "per_op": per_op,
        }
        line["gpu_launches"] = args.steps + sum(v.get("gpu_launches", 0) for v in per_op.values())
        print(json.dumps(line))
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()
    return 1 if _parity_failed(per_op) else 0


def _parity_failed(per_op):
    bad = {k: v["parity"] for k, v in per_op.items()
           if str(v.get("parity", "ok")).startswith("FAIL")}
    if bad:
        sys.stderr.write(f"parity failures: {bad}\n")
    return bool(bad)


if __name__ == "__main__":
    sys.exit(main())
