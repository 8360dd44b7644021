"""Benchmark of the fused FFT convolution (BASELINE.json metric):
"fused conv Gpoints/s + HBM GB/s (% of B200 peak) at N=4096 fp32 & int16-BFP".

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Workload (BASELINE.json configs[1] at N=4096): batch = 2^27/N transforms, so
the fp32 signal is 1 GiB (the int16-BFP run uses the same point count);
signal iid N(0,1) complex, filter taps iid U[-1,1) complex turned into a
spectrum (x 1/N) on the device by this library's own forward transform, one
filter per transform, mid-op multiply.  A step is one fused-convolution
launch over the whole batch.  Inputs are 3 GiB per step (1 GiB each for
signal, filter, result), far above the 126 MB L2, so no flush is needed.

value: device-resident Gpoints/s (points = batch * N), timed with CUDA events
on the launching stream, max over ranks.  e2e: the same metric through the
public host-data entry point (fufft_conv_c2c_f32_host) with pinned host
buffers: every step uploads signal and filter and downloads the result
(chunked, the two link directions overlapping), all inside the timed region.  roofline: algorithmic bytes (24 B/pt fp32, 12 B/pt BFP)
per launch over the measured launch time, against the measured HBM copy
bandwidth.  --gpus N > 1 (under torchrun): every rank runs its own full batch
(batch sharding, no collective on the data path): weak scaling.
--impl reference: the reference's own CPU transcription (oracle/_ref,
compiled from its sources; else the oracle restatement) on all host cores.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)
# the single-signal record maps peer memory with plain loads and stores; NCCL
# (barriers and one-element all-reduces only) runs with NVLS switched off
os.environ.setdefault("NCCL_NVLS_ENABLE", "0")

N = 4096
POINTS = 1 << 27
BYTES_F32 = 24      # read signal 8 + read filter 8 + write result 8 per point
BYTES_BFP = 12      # the same three streams at 4 B per point (+3 scales per transform)


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def profile_traffic(key):
    """dram bytes per launch from a committed ncu capture (profiles/traffic.json)"""
    try:
        with open(os.path.join(ROOT, "profiles", "traffic.json")) as f:
            return json.load(f).get(key)
    except Exception:
        return None


_SAMPLER = r"""
import sys, time
import pynvml as nv
nv.nvmlInit()
key = sys.argv[1]
h = nv.nvmlDeviceGetHandleByPciBusId(key) if ":" in key else nv.nvmlDeviceGetHandleByIndex(int(key))
mx = nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM)
rf = getattr(nv, "nvmlDeviceGetCurrentClocksEventReasons", None) or nv.nvmlDeviceGetCurrentClocksThrottleReasons
print("ready", flush=True)
while True:
    t = time.monotonic()
    print(t, nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM), mx, int(rf(h)), flush=True)
    time.sleep(0.001)
"""


class ClockSampler:
    """SM clock and throttle reasons of one GPU, sampled through NVML
    (read-only queries) every millisecond by a separate process, so that the
    samples do not wait for this process's interpreter lock.  Each sample
    carries a CLOCK_MONOTONIC time stamp; `mark()` / `mark(end=True)` bound the
    timed region and the summary keeps the samples inside it.  Falls back to
    `nvidia-smi -lms` when NVML is unavailable."""
    # NVML clocks-event-reason bits
    REASONS = {0x8: "hw_slowdown", 0x40: "hw_thermal_slowdown", 0x20: "sw_thermal_slowdown", 0x4: "sw_power_cap"}

    def __init__(self, device: int):
        self.device, self.rows, self.proc, self.t, self.source = device, [], None, None, None
        self.t0, self.t1 = None, None

    def _key(self):
        try:
            import torch
            p = torch.cuda.get_device_properties(self.device)
            return "%08x:%02x:%02x.0" % (p.pci_domain_id, p.pci_bus_id, p.pci_device_id)
        except Exception:
            return str(self.device)

    def __enter__(self):
        try:
            self.proc = subprocess.Popen([sys.executable, "-c", _SAMPLER, self._key()], stdout=subprocess.PIPE,
                                         stderr=subprocess.DEVNULL, text=True)
            if self.proc.stdout.readline().strip() != "ready":
                raise RuntimeError("sampler did not start")
            self.source = "nvml"
            self.t = threading.Thread(target=self._read, args=(False,), daemon=True)
            self.t.start()
        except Exception:
            self._stop()
            try:
                self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.device),
                                              "--query-gpu=clocks.sm,clocks.max.sm,clocks_event_reasons.active",
                                              "--format=csv,noheader,nounits", "-lms", "20"],
                                             stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
                self.source = "nvidia-smi"
                self.t = threading.Thread(target=self._read, args=(True,), daemon=True)
                self.t.start()
            except Exception:
                self.proc = None
        return self

    def _read(self, smi):
        for line in self.proc.stdout:
            try:
                if smi:
                    f = [x.strip() for x in line.split(",")]
                    self.rows.append((time.monotonic(), float(f[0]), float(f[1]), int(f[2], 16)))
                else:
                    f = line.split()
                    self.rows.append((float(f[0]), float(f[1]), float(f[2]), int(f[3])))
            except (ValueError, IndexError):
                pass

    def mark(self, end=False):
        if end:
            self.t1 = time.monotonic()
        else:
            self.t0 = time.monotonic()

    def _stop(self):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()
        if self.t:
            self.t.join(timeout=2)

    def __exit__(self, *exc):
        self._stop()

    def summary(self):
        rows = self.rows
        if self.t0 is not None and self.t1 is not None:
            inside = [r for r in rows if self.t0 <= r[0] <= self.t1]
            window = "timed region"
            if not inside:   # region shorter than one sample interval: the samples around it
                inside = [r for r in rows if self.t0 - 0.01 <= r[0] <= self.t1 + 0.01]
                window = "timed region +- 10 ms"
            rows = inside
        else:
            window = "whole block"
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0, "window": window}
        reasons = sorted({name for *_, bits in rows for bit, name in self.REASONS.items() if bits & bit})
        return {"sm_mhz": statistics.median(r[1] for r in rows), "sm_max_mhz": max(r[2] for r in rows),
                "reasons": reasons, "samples": len(rows), "source": self.source, "window": window}


# ------------------------------------------------------------------------------------------
def cpu_reference_rate(seconds: float, threads: int | None = None, n: int = N):
    """The reference's CPU path (kernel_pipeline_v16, verify_kernel.cpp:1051) on a
    bounded sample: `threads` host threads, each on its own slice of transforms.
    Returns (points/s, kind, threads, sample description)."""
    import ctypes as ct
    import numpy as np
    from oracle import oracle as orc
    threads = threads or os.cpu_count() or 1
    try:
        ref = orc.Reference()
        fn, kind = ref.L.ref_pipeline_v16, "reference"
        args_of = lambda a, b, o, bt: (n, 1, a.ctypes.data, b.ctypes.data, o.ctypes.data, bt)   # noqa: E731
    except Exception:
        o_ = orc.Oracle()
        fn, kind = o_.L.orc_conv, "port"
        args_of = lambda a, b, o, bt: (n, 16, 1, a.ctypes.data, b.ctypes.data, o.ctypes.data, bt, n)  # noqa: E731
    rng = np.random.default_rng(7)
    # calibrate one transform, then size each thread's slice to ~seconds of work
    a1 = (rng.standard_normal(n) + 1j * rng.standard_normal(n)).astype(np.complex64)
    b1 = (rng.uniform(-1, 1, n) + 1j * rng.uniform(-1, 1, n)).astype(np.complex64) / n
    o1 = np.empty_like(a1)
    t0 = time.perf_counter()
    fn(*args_of(a1, b1, o1, 1))
    per = max(time.perf_counter() - t0, 1e-5)
    per_thread = max(1, int(seconds / per))
    bufs = []
    for _ in range(threads):
        a = np.tile(a1, per_thread)
        b = np.tile(b1, per_thread)
        bufs.append((a, b, np.empty_like(a)))
    def work(i):
        a, b, o = bufs[i]
        fn(*args_of(a, b, o, per_thread))
    ths = [threading.Thread(target=work, args=(i,)) for i in range(threads)]
    t0 = time.perf_counter()
    for t in ths:
        t.start()
    for t in ths:
        t.join()
    dt = time.perf_counter() - t0
    pts = threads * per_thread * n
    return pts / dt, kind, threads, f"{threads} threads x {per_thread} transforms of N={n} ({pts} points, {dt:.1f} s)"


# ------------------------------------------------------------------------------------------
def make_inputs(ops, torch, n, batch, seed, device):
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    a = torch.randn(batch * n, dtype=torch.complex64, device=device, generator=g)
    taps = torch.complex(torch.rand(batch * n, device=device, generator=g) * 2 - 1,
                         torch.rand(batch * n, device=device, generator=g) * 2 - 1)
    spec = ops.fwd(taps, n, ops.LAYOUT_R16)           # chain order, radix-16
    spec.mul_(1.0 / n)
    del taps
    # chain order -> register-boundary layout: bperm[L + k*T] = chain[16 L + k]
    bperm = spec.view(batch, n // 16, 16).transpose(1, 2).contiguous().view(-1)
    return a, spec, bperm


# ------------------------------------------------------------------------------------------
# Parity of the buffers a timed loop just produced: float64 DFTs on the device
# (torch.fft in complex128) as an independent ground truth on the first, the
# last and 256 seeded-random transforms, outside the timed events.  (The oracle
# is test infrastructure; the tests compare the same launches with it.)
def sample_idx(batch, seed, k=256):
    import numpy as np
    rng = np.random.default_rng(seed)
    pick = rng.choice(batch, min(k, batch), replace=False).tolist()
    return sorted({0, batch - 1, *pick})


def rel_l2_t(torch, x, y):
    x = x.to(torch.complex128)
    y = y.to(torch.complex128)
    return float(torch.linalg.vector_norm(x - y) / torch.linalg.vector_norm(y))


def natural_rows(ops, torch, rows_chain, radices):
    """rows in the chain order of `radices` -> natural (frequency) order"""
    nat = torch.empty_like(rows_chain)
    nat[:, ops.chain_rev_table(radices, rows_chain.device)] = rows_chain
    return nat


def unbperm_rows(rows, n, v=16):
    """register-boundary order -> chain order: chain[v*L + k] = bperm[L + k*T]"""
    return rows.reshape(-1, v, n // v).transpose(1, 2).reshape(-1, n)


def conv_f64(torch, a, bnat):
    """unnormalised IDFT(DFT(a) * b), rows of complex128 (b carries the 1/n)"""
    return torch.fft.ifft(torch.fft.fft(a) * bnat, norm="forward")


def dequant_rows(torch, q, s):
    """int16 pairs [k, n, 2] and scales [k] -> complex128 [k, n]"""
    return torch.complex(q[..., 0].double(), q[..., 1].double()) * s.double()[:, None]


def parity_f32_1d(ops, torch, a, filt_chain_rows, out, n, batch, idx, radices=None):
    """fp32 output rows idx against float64; filt_chain_rows(idx) gives the
    filter rows in chain order"""
    ii = torch.tensor(idx, device=a.device)
    want = conv_f64(torch, a.view(batch, n)[ii].to(torch.complex128),
                    natural_rows(ops, torch, filt_chain_rows(ii), radices or ops.chain(n, 16)).to(torch.complex128))
    e = rel_l2_t(torch, out.view(batch, n)[ii], want)
    return {"rel_l2_vs_f64": float(f"{e:.3g}"), "tol": 3e-6, "ok": e < 3e-6, "checked": len(idx)}


def parity_bfp_1d(ops, torch, aq, as_, bq, bs, oq, os_, n, batch, idx, radices=None, bperm_v=0):
    """int16-BFP output rows idx against the exact (float64) convolution of the
    same quantised inputs; also the mantissas against the exactly rounded BFP
    result (scale from the exact abs-max, rint(x * 32767 / max))"""
    ii = torch.tensor(idx, device=aq.device)
    a64 = dequant_rows(torch, aq.view(batch, n, 2)[ii], as_[ii])
    b64 = dequant_rows(torch, bq.view(batch, n, 2)[ii], bs[ii])
    if bperm_v:
        b64 = unbperm_rows(b64, n, bperm_v)
    exact = conv_f64(torch, a64, natural_rows(ops, torch, b64, radices or ops.chain(n, 16)))
    q = oq.view(batch, n, 2)[ii]
    e = rel_l2_t(torch, dequant_rows(torch, q, os_[ii]), exact)
    mx = torch.maximum(exact.real.abs().amax(1), exact.imag.abs().amax(1)).clamp_min(1e-30)[:, None]
    qe = torch.stack([torch.round(exact.real * 32767 / mx), torch.round(exact.imag * 32767 / mx)], -1)
    dq = (q.double() - qe).abs()
    return {"rel_l2_vs_f64": float(f"{e:.3g}"), "tol": 6e-5, "ok": e < 6e-5,
            "max_dq_lsb_vs_exact": int(dq.max()), "mismatch_frac_vs_exact": float(f"{float((dq != 0).double().mean()):.4g}"),
            "checked": len(idx)}


def time_steps(torch, fn, steps, warmup, dist, clk=None):
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    st = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if clk:
        clk.mark()
    e0.record(st)
    for _ in range(steps):
        fn()
    e1.record(st)
    torch.cuda.synchronize()
    if clk:
        clk.mark(end=True)
    if dist:
        dist.barrier()
    ms = e0.elapsed_time(e1) / steps
    if dist:
        t = torch.tensor([ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    return ms


def headline_config(n, batch, world):
    """the `config` of the headline line (both arms print the same one)"""
    return {"workload": f"configs[1] fused fp32 cyclic conv N={n}, batch={batch} per GPU "
                        f"(1 GiB signal), one filter per transform, mid-op multiply, "
                        f"filter in the radix-16 register-boundary layout",
            "n": n, "batch_per_gpu": batch, "layout": "R16_BPERM", "parallelism": f"batch-sharded x{world}",
            "l2": "inputs 3 GiB per step > 126 MB L2 (no flush needed)"}


def run_ours(args, rank, world, dist):
    import torch
    from fufft_b200 import ops
    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", 0)))
    torch.cuda.set_device(dev)
    ops.init()
    n = args.n
    batch = POINTS // n
    hbm, peak_kind = peaks()
    a, spec, bperm = make_inputs(ops, torch, n, batch, 1000 * 2 + n + rank, dev)
    out = torch.empty_like(a)
    layout = ops.LAYOUT_R16_BPERM

    # ---- fp32 fused conv, device resident
    launches0 = ops.launch_count()
    with ClockSampler(torch.cuda.current_device()) as clk:
        ms = time_steps(torch, lambda: ops.conv(a, bperm, n, layout, ops.MID_MULTIPLY, out=out),
                        args.steps, args.warmup, dist, clk)
    launches = (ops.launch_count() - launches0) // (args.steps + args.warmup) * args.steps
    pts = batch * n
    gpts = pts / (ms * 1e-3) / 1e9
    achieved = BYTES_F32 * pts / (ms * 1e-3) / 1e9
    # the output of the timed launches, checked outside the events
    idx = sample_idx(batch, 17 + rank)
    parity = {"fp32": parity_f32_1d(ops, torch, a, lambda ii: unbperm_rows(bperm.view(batch, n)[ii], n),
                                    out, n, batch, idx)}

    # ---- int16 BFP fused conv (same points, the reference's linear filter layout)
    aq, as_ = ops.bfp_pack(a, n)
    bq, bs = ops.bfp_pack(spec, n)
    bout = (torch.empty_like(aq), torch.empty(batch, dtype=torch.float32, device=dev))
    ms_bfp = time_steps(torch, lambda: ops.conv_bfp(aq, as_, bq, bs, n, ops.LAYOUT_R16, ops.MID_MULTIPLY, out=bout),
                        args.steps, args.warmup, dist)
    gpts_bfp = pts / (ms_bfp * 1e-3) / 1e9
    ach_bfp = (BYTES_BFP * pts + 12 * batch) / (ms_bfp * 1e-3) / 1e9
    parity["bfp"] = parity_bfp_1d(ops, torch, aq, as_, bq, bs, bout[0], bout[1], n, batch, idx)
    del aq, bq, bout

    # ---- e2e through the public API with pinned host buffers: the host-data
    # entry point (fufft_conv_c2c_f32_host) moves signal and filter in and the
    # result out in chunks, uploads and downloads overlapping on the link
    e2e_steps = max(1, min(args.steps, 5))
    ha = a.cpu().pin_memory()
    hb = bperm.cpu().pin_memory()
    ho = torch.empty_like(ha).pin_memory()
    ws = ops.conv_host_workspace(n, batch, n, dev)

    def e2e_step():
        ops.conv_host(ha, hb, ho, n, layout, ops.MID_MULTIPLY, filter_stride=n, workspace=ws)

    ms_e2e = time_steps(torch, e2e_step, e2e_steps, 1, dist)
    # the host-data path runs the same kernel on the same data: bit-identical rows
    hrows = torch.tensor(idx)
    parity["e2e_equals_device"] = bool(torch.equal(ho.view(batch, n)[hrows], out.view(batch, n)[hrows.to(dev)].cpu()))
    world_pts = pts * world
    line = {
        "metric": "fused conv Gpoints/s + HBM GB/s (% of B200 peak) at N=4096 fp32 & int16-BFP",
        "value": round(world_pts / (ms * 1e-3) / 1e9, 3),
        "unit": "Gpoints/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(ms, 4),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "f32", "data": "synthetic (seeded: signal N(0,1), filter taps U[-1,1) -> spectrum/N)",
        "config": headline_config(n, batch, world),
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": hbm, "unit": "GB/s",
                     "frac": round(achieved / hbm, 4), "peak_kind": peak_kind,
                     "traffic": profile_traffic(f"conv_f32_r16_bperm_n{n}"),
                     "bytes_per_point": BYTES_F32, "kernel": f"conv_kernel<{n},16,...,MUL,BP_DIRECT> (1 launch/step)"},
        "bfp": {"value": round(gpts_bfp * world, 3), "unit": "Gpoints/s", "ms_per_step": round(ms_bfp, 4),
                "roofline": {"bound": "hbm", "achieved": round(ach_bfp, 1), "peak": hbm, "unit": "GB/s",
                             "frac": round(ach_bfp / hbm, 4), "bytes_per_point": BYTES_BFP,
                             "traffic": profile_traffic(f"conv_bfp_r16_n{n}")},
                "layout": "R16 (the reference's linear mixedrev16 order)"},
        "e2e": {"value": round(world_pts / (ms_e2e * 1e-3) / 1e9, 3), "unit": "Gpoints/s",
                "h2d_bytes_per_step": int(ha.numel() * 8 + hb.numel() * 8),
                "d2h_bytes_per_step": int(ho.numel() * 8), "steps": e2e_steps,
                "ms_per_step": round(ms_e2e, 3)},
        "gpu_launches": int(launches),
        "clocks": clk.summary(),
        "parity": parity,
    }
    del ha, hb, ho, a, spec, bperm, out, ws
    torch.cuda.empty_cache()
    if not args.no_configs:
        line["configs"] = run_configs(args, ops, torch, dist, hbm, rank, world, dev)
    if world > 1 and not args.no_dist:
        line["dist"] = run_dist_record(args, ops, torch, dist, rank, world, dev, hbm)
    if rank == 0 and not args.no_cpu_baseline:
        rate, kind, cores, sample = cpu_reference_rate(args.cpu_seconds)
        line["cpu_baseline"] = {"value": round(rate / 1e9, 6), "unit": "Gpoints/s", "cores": cores,
                                "kind": kind, "sample": sample}
    return line


def run_configs(args, ops, torch, dist, hbm, rank, world, dev):
    """Every BASELINE.json config besides the headline, compactly: per config
    the whole-job Gpoints/s (every rank runs its own copy: weak scaling, max
    over ranks), the fraction of the measured HBM peak under its byte model,
    and the float64 parity of sampled outputs of the timed buffers."""
    g = torch.Generator(device=dev)
    g.manual_seed(4321 + rank)
    steps, warm = args.steps, args.warmup
    C = torch.complex64

    def rec(ms, pts, bpp, extra=0, **kw):
        gbs = (bpp * pts + extra) / (ms * 1e-3) / 1e9
        return {"value": round(world * pts / (ms * 1e-3) / 1e9, 3), "unit": "Gpoints/s", "ms_per_step": round(ms, 4),
                "frac": round(gbs / hbm, 4), "bytes_per_point": bpp, **kw}

    res = {}
    # config 1: N=1024 x 4096 (32 MiB per array: inside L2).  Throughput of
    # back-to-back batches: four independent input/output sets (384 MiB in all,
    # > 3x L2) in turn, so every step's inputs were evicted by the three steps
    # before it.  Also the latency of one isolated launch with L2 flushed
    # before it (event-timed, so it carries the ~6 us launch-and-event floor of
    # any kernel timed alone: an empty kernel times at 6 us the same way)
    n, batch, nsets = 1024, 4096, 4
    sets = []
    for k in range(nsets):
        a, spec, bperm = make_inputs(ops, torch, n, batch, 1000 * 1 + 10 * k + n + rank, dev)
        del spec
        sets.append((a, bperm, torch.empty_like(a)))
    turn = [0]

    def c1_step():
        a, bperm, o = sets[turn[0] % nsets]
        turn[0] += 1
        ops.conv(a, bperm, n, ops.LAYOUT_R16_BPERM, out=o)
    ms = time_steps(torch, c1_step, steps * nsets, warm, dist)
    a, bperm, o = sets[0]
    ms1 = time_flushed(torch, lambda: ops.conv(a, bperm, n, ops.LAYOUT_R16_BPERM, out=o), steps, warm, dist=dist)
    res["c1_fp32_n1024_b4096"] = rec(ms, batch * n, 24, layout="R16_BPERM",
                                     l2=f"{nsets} input/output sets in turn ({nsets * 96} MiB > 3x L2)",
                                     single_launch_ms=round(ms1, 4),
                                     single_launch_l2="flushed before the launch",
                                     parity=parity_f32_1d(ops, torch, a, lambda ii: unbperm_rows(bperm.view(batch, n)[ii], n),
                                                          o, n, batch, sample_idx(batch, 1)))
    del sets, a, bperm, o

    # config 2: the other sizes of the sweep (1 GiB of signal), fp32 and int16-BFP;
    # at N=4096 also the reference's own linear filter orders (radix-16 and radix-8 chains)
    for n in (512, 1024, 2048, 4096):
        batch = POINTS // n
        a, spec, bperm = make_inputs(ops, torch, n, batch, 1000 * 2 + n + rank, dev)
        o = torch.empty_like(a)
        idx = sample_idx(batch, n)
        if n < 4096:
            ms = time_steps(torch, lambda: ops.conv(a, bperm, n, ops.LAYOUT_R16_BPERM, out=o), steps, warm, dist)
            res[f"c2_fp32_n{n}"] = rec(ms, batch * n, 24, layout="R16_BPERM", parity=parity_f32_1d(
                ops, torch, a, lambda ii: unbperm_rows(bperm.view(batch, n)[ii], n), o, n, batch, idx))
            aq, as_ = ops.bfp_pack(a, n)
            bq, bs = ops.bfp_pack(spec, n)
            bout = (torch.empty_like(aq), torch.empty(batch, dtype=torch.float32, device=dev))
            ms = time_steps(torch, lambda: ops.conv_bfp(aq, as_, bq, bs, n, ops.LAYOUT_R16, out=bout), steps, warm, dist)
            res[f"c2_bfp_n{n}"] = rec(ms, batch * n, 12, 12 * batch, layout="R16", parity=parity_bfp_1d(
                ops, torch, aq, as_, bq, bs, bout[0], bout[1], n, batch, idx))
            del aq, bq, bout
        else:
            del bperm
            ms = time_steps(torch, lambda: ops.conv(a, spec, n, ops.LAYOUT_R16, out=o), steps, warm, dist)
            res["c2_fp32_n4096_linear_r16"] = rec(ms, batch * n, 24, layout="R16 (mixedrev16 order)", parity=parity_f32_1d(
                ops, torch, a, lambda ii: spec.view(batch, n)[ii], o, n, batch, idx))
            # the radix-8 chain order of the same spectra
            r8 = ops.chain(n, 8)
            rev16, rev8 = ops.chain_rev_table(ops.chain(n, 16), dev), ops.chain_rev_table(r8, dev)
            nat_pos = torch.empty_like(rev16)
            nat_pos[rev16] = torch.arange(n, device=dev)          # natural bin -> radix-16 chain slot
            spec = spec.view(batch, n)[:, nat_pos[rev8]].reshape(-1)
            ms = time_steps(torch, lambda: ops.conv(a, spec, n, ops.LAYOUT_R8, out=o), steps, warm, dist)
            res["c2_fp32_n4096_linear_r8"] = rec(ms, batch * n, 24, layout="R8 (mixedrev order)", parity=parity_f32_1d(
                ops, torch, a, lambda ii: spec.view(batch, n)[ii], o, n, batch, idx, r8))
        del a, spec, o

    # config 3: 1024 real signals x 256 real filters, N=4096: packed pairs -> 512
    # spectra (once per step) -> every pair x every filter in one launch (4 GiB of
    # real outputs per mid-op).  Bytes: 4 per real output point + the spectra,
    # filters and signals read once (they stay in L2)
    n, nsig, nfilt = 4096, 1024, 256
    x = torch.randn(nsig * n, device=dev, generator=g)
    taps = torch.rand(nfilt, n, device=dev, generator=g) * 2 - 1
    b_nat = torch.fft.fft(taps.double(), dim=1) / n
    bp = ops.filter_permute(b_nat.to(C).reshape(-1), n, ops.LAYOUT_R16_BPERM)
    xs = x.view(nsig // 2, 2, n)
    xr, yr = xs[:, 0].contiguous().view(-1), xs[:, 1].contiguous().view(-1)
    o = torch.empty(nsig * nfilt * n, device=dev)
    pairs = [(int(i), int(f)) for i, f in zip(sample_idx(nsig, 3, 32)[:32], sample_idx(nfilt, 4, 32)[:32])]
    for mid, mname in [(ops.MID_MULTIPLY, "multiply"), (ops.MID_CONJ_MULTIPLY, "conj")]:
        def step():
            spec = ops.fwd_r2(xr, yr, n, ops.LAYOUT_R16_BPERM)
            ops.apply_grid_r2(spec, bp, n, ops.LAYOUT_R16_BPERM, mid, out=o)
        ms = time_steps(torch, step, steps, warm, dist)
        si = torch.tensor([p[0] for p in pairs], device=dev)
        fi = torch.tensor([p[1] for p in pairs], device=dev)
        bsel = b_nat[fi] if mid == ops.MID_MULTIPLY else b_nat[fi].conj()
        want = conv_f64(torch, x.view(nsig, n)[si].double().to(torch.complex128), bsel).real
        got = o.view(nsig, nfilt, n)[si, fi]
        e = rel_l2_t(torch, got, want)
        res[f"c3_grid_r2_{mname}"] = rec(ms, nsig * nfilt * n, 4, 8 * n * (nsig // 2 + nfilt) + 16 * n * (nsig // 2),
                                         unit_points="real output points",
                                         parity={"rel_l2_vs_f64": float(f"{e:.3g}"), "tol": 3e-6, "ok": e < 3e-6,
                                                 "checked": len(pairs)})
    del x, taps, b_nat, bp, xs, xr, yr, o

    # config 4: 2-D 256x256 x 512 images (re U[0,1), im 0), one shared filter:
    # Gaussian taps, sigma 8 px, centred at (0, 0) with cyclic wrap, plus N(0, 0.01)
    # noise (0.01 read as the variance)
    h = w = 256
    batch = 512
    a = torch.rand(batch * h * w, device=dev, generator=g).to(C)
    d = torch.minimum(torch.arange(h, device=dev), h - torch.arange(h, device=dev)).double()
    gauss = torch.exp(-(d[:, None] ** 2 + d[None, :] ** 2) / (2 * 8.0 ** 2))
    taps2 = gauss + 0.1 * torch.randn(h, w, device=dev, generator=g).double()
    b_nat = torch.fft.fft2(taps2) / (h * w)
    bk = ops.filter_permute2d(b_nat.to(C).reshape(-1), h, w, ops.LAYOUT_R16_BPERM)
    o = torch.empty_like(a)
    ms = time_steps(torch, lambda: ops.conv2d(a, bk, h, w, ops.LAYOUT_R16_BPERM, filter_stride=0, out=o), steps, warm,
                    dist)
    ii = torch.tensor(sample_idx(batch, 5, 16), device=dev)
    want = torch.fft.ifft2(torch.fft.fft2(a.view(batch, h, w)[ii].to(torch.complex128)) * b_nat, norm="forward")
    e = rel_l2_t(torch, o.view(batch, h, w)[ii], want)
    res["c4_conv2d_256x256_b512"] = rec(ms, batch * h * w, 16, 8 * h * w, layout="R16_BPERM", filter="shared",
                                        parity={"rel_l2_vs_f64": float(f"{e:.3g}"), "tol": 3e-6, "ok": e < 3e-6,
                                                "checked": int(ii.numel())})
    del a, b_nat, bk, o, taps2

    # config 5: four-step N=32768 x 2048, fp32 (cluster kernel, in place: the timed
    # steps re-convolve the previous result; parity from a fresh run) and int16-BFP
    n, batch = 32768, 2048
    r_out, mid = ops.large_plan(n, ops.LAYOUT_R16)
    lout, q = 0, n // mid
    while q > 1:
        q //= r_out
        lout += 1
    chain = [r_out] * lout + ops.chain(mid, 16)
    a = torch.randn(batch * n, dtype=C, device=dev, generator=g)
    taps = torch.complex(torch.rand(batch * n, device=dev, generator=g) * 2 - 1,
                         torch.rand(batch * n, device=dev, generator=g) * 2 - 1)
    b_chain = (torch.fft.fft(taps.view(batch, n)) / n)[:, ops.chain_rev_table(chain, dev)].reshape(-1).contiguous()
    del taps
    buf = a.clone()
    # the fp32 filter in the middle's register-boundary order, chunk by chunk
    b_bp = b_chain.view(-1, mid // 16, 16).transpose(1, 2).contiguous().view(-1)
    ms = time_steps(torch, lambda: ops.conv_large(buf, b_bp, n, ops.LAYOUT_R16_BPERM, r_out=r_out, mid_size=mid),
                    steps, warm, dist)
    buf.copy_(a)
    ops.conv_large(buf, b_bp, n, ops.LAYOUT_R16_BPERM, r_out=r_out, mid_size=mid)
    idx = sample_idx(batch, 6, 64)
    res["c5_fp32_n32768_b2048"] = rec(ms, batch * n, 24, layout="R16_BPERM", plan=[r_out, mid], parity=parity_f32_1d(
        ops, torch, a, lambda ii: b_bp.view(batch, n)[ii].reshape(-1, 16, mid // 16).transpose(1, 2).reshape(-1, n),
        buf, n, batch, idx, chain))
    del buf, b_bp
    aq, as_ = ops.bfp_pack(a, n)
    bq, bs = ops.bfp_pack(b_chain, n)
    del a, b_chain
    ws = torch.empty(int(ops.lib().fufft_conv_large_bfp_workspace(n, batch)), dtype=torch.uint8, device=dev)
    outq = []

    def bstep():
        outq[:] = ops.conv_large_bfp(aq, as_, bq, bs, n, ops.LAYOUT_R16, r_out=r_out, mid_size=mid, workspace=ws)
    ms = time_steps(torch, bstep, steps, warm, dist)
    res["c5_bfp_n32768_b2048"] = rec(ms, batch * n, 12, 12 * batch, layout="R16", plan=[r_out, mid],
                                     parity=parity_bfp_1d(ops, torch, aq, as_, bq, bs, outq[0], outq[1], n, batch, idx,
                                                          chain))
    del aq, bq, ws, outq
    torch.cuda.empty_cache()
    return res


def run_dist_record(args, ops, torch, dist, rank, world, dev, hbm):
    """config 5's single signal over the ranks (strong scaling): one N=2^26
    convolution with the all-to-alls fused into the outer passes as NVLink
    stores / loads; parity of the same scheme at N=2^20 against float64 on
    the gathered signal"""
    from fufft_b200.distributed import (GpuBackend, PeerBlocks, conv_distributed_p2p, filter_block,
                                        gather_signal, scatter_signal)
    be = GpuBackend()
    C = torch.complex64
    # parity: every rank builds the same global signal and filter
    ns = 1 << 20
    plan = be.plan(ns, world)
    g = torch.Generator(device=dev)
    g.manual_seed(777)
    xg = torch.randn(ns, dtype=C, device=dev, generator=g)
    taps = torch.complex(torch.rand(ns, device=dev, generator=g) * 2 - 1, torch.rand(ns, device=dev, generator=g) * 2 - 1)
    b_nat = torch.fft.fft(taps.to(torch.complex128)) / ns
    b_chain = b_nat[ops.chain_rev_table(plan.chain, dev)].to(C)
    x = scatter_signal(xg, ns, world, rank)
    peers = PeerBlocks(plan.n_blk)
    conv_distributed_p2p(x, filter_block(b_chain, ns, world, rank), ns, peers, backend=be, plan=plan)
    peers.close()
    parts = [torch.empty(2 * x.numel(), device=dev) for _ in range(world)]
    dist.all_gather(parts, torch.view_as_real(x).reshape(-1))
    yg = gather_signal([torch.view_as_complex(p.view(-1, 2)) for p in parts], ns)
    e = rel_l2_t(torch, yg[None], conv_f64(torch, xg[None].to(torch.complex128), b_nat[None]))
    del xg, taps, b_nat, b_chain, x, parts, yg
    # timing: N = 2^26
    n = 1 << 26
    plan = be.plan(n, world)
    g.manual_seed(5000 + rank)
    x0 = torch.randn(world * plan.cols, dtype=C, device=dev, generator=g)
    bb = torch.randn(plan.n_blk, dtype=C, device=dev, generator=g) / n
    peers = PeerBlocks(plan.n_blk)
    ms = time_steps(torch, lambda: conv_distributed_p2p(x0, bb, n, peers, backend=be, plan=plan), args.steps,
                    args.warmup, dist)
    peers.close()
    nvl = 2 * 8 * plan.n_blk * (world - 1) // world
    return {"value": round(n / (ms * 1e-3) / 1e9, 3), "unit": "Gpoints/s", "ms_per_step": round(ms, 4),
            "scaling": "strong", "n": n, "ranks": world,
            "plan": {"block": plan.n_blk, "r_out": plan.r_out, "mid": plan.mid, "chain": plan.chain},
            "exchange": "NVLink peer stores / loads fused into the outer passes (plain peer accesses)",
            "nvlink_bytes_per_gpu": nvl, "nvlink_gbs_per_gpu": round(nvl / (ms * 1e-3) / 1e9, 1),
            "hbm_frac_per_gpu_24B": round(24 * (n // world) / (ms * 1e-3) / 1e9 / hbm, 4),
            "parity": {"n": ns, "rel_l2_vs_f64": float(f"{e:.3g}"), "tol": 5e-6, "ok": e < 5e-6}}


def run_ncu_all():
    """one launch of every kernel family of the library (sizes > L2 where the
    kernel streams HBM), for a one-table ncu summary.  Prints a manifest:
    one line per library call, in launch order, with the points it covers and
    its algorithmic HBM bytes."""
    import torch
    from fufft_b200 import ops
    from fufft_b200._lib import check, lib
    ops.init()
    g = torch.Generator(device="cuda")
    g.manual_seed(7)
    C = torch.complex64
    n, batch = 4096, 16384                       # 0.5 GiB of fp32 signal
    pts = n * batch
    a = torch.randn(pts, dtype=C, device="cuda", generator=g)
    b = torch.randn(pts, dtype=C, device="cuda", generator=g) / n
    o = torch.empty_like(a)
    man = []

    def call(label, fn, points, nbytes, launches=1):
        fn()
        torch.cuda.synchronize()
        man.append((label, launches, points, nbytes))

    call("conv fp32 R16_BPERM (register-boundary filter, read directly)", lambda: ops.conv(a, b, n, ops.LAYOUT_R16_BPERM, out=o), pts, 24 * pts)
    call("conv fp32 R16 (linear mixedrev16 filter, staged per warp)", lambda: ops.conv(a, b, n, ops.LAYOUT_R16, out=o),
         pts, 24 * pts)
    call("conv fp32 R8_BPERM (radix-16 engine, filter read directly through the bit permutation)",
         lambda: ops.conv(a, b, n, ops.LAYOUT_R8_BPERM, out=o), pts, 24 * pts)
    call("conv fp32 R8 (linear mixedrev filter, radix-16 engine, bit-permutation staging)",
         lambda: ops.conv(a, b, n, ops.LAYOUT_R8, out=o), pts, 24 * pts)
    call("conv fp32 R16_BPERM conj-multiply", lambda: ops.conv(a, b, n, ops.LAYOUT_R16_BPERM, ops.MID_CONJ_MULTIPLY, out=o), pts, 24 * pts)
    aq, as_ = ops.bfp_pack(a, n)
    torch.cuda.synchronize()
    man.append(("bfp_pack (one pass: abs-max and quantise in one CTA per transform)", 1, pts, 12 * pts + 4 * batch))
    bq, bs = ops.bfp_pack(b, n)
    torch.cuda.synchronize()
    man.append(("bfp_pack (filter)", 1, pts, 12 * pts + 4 * batch))
    call("conv int16-BFP R16", lambda: ops.conv_bfp(aq, as_, bq, bs, n, ops.LAYOUT_R16), pts, 12 * pts + 12 * batch)
    call("conv int16-BFP R16_BPERM", lambda: ops.conv_bfp(aq, as_, bq, bs, n, ops.LAYOUT_R16_BPERM), pts, 12 * pts + 12 * batch)
    call("bfp_unpack", lambda: ops.bfp_unpack(aq, as_, n), pts, 12 * pts)
    del aq, bq
    call("fwd (split forward, R16_BPERM spectrum)", lambda: ops.fwd(a, n, ops.LAYOUT_R16_BPERM), pts, 16 * pts)
    spec = ops.fwd(a, n, ops.LAYOUT_R16_BPERM)
    torch.cuda.synchronize()
    man.append(("fwd (spectrum for apply)", 1, pts, 16 * pts))
    call("apply (split apply, R16_BPERM)", lambda: ops.apply(spec, b, n, ops.LAYOUT_R16_BPERM, out=o), pts, 24 * pts)
    # the reference's own split layout (radix-8 chain order) and the radix-16 chain order
    call("fwd (split forward, R8 spectrum: radix-16 engine, bit-permutation staging)",
         lambda: ops.fwd(a, n, ops.LAYOUT_R8), pts, 16 * pts)
    spec8 = ops.fwd(a, n, ops.LAYOUT_R8)
    torch.cuda.synchronize()
    man.append(("fwd (R8 spectrum for apply)", 1, pts, 16 * pts))
    call("apply (split apply, R8 spectrum and filter)", lambda: ops.apply(spec8, b, n, ops.LAYOUT_R8, out=o),
         pts, 24 * pts)
    del spec8
    call("fwd (split forward, R16 chain-order spectrum, staged per warp)", lambda: ops.fwd(a, n, ops.LAYOUT_R16),
         pts, 16 * pts)
    xr, yr = a.real.contiguous(), a.imag.contiguous()
    torch.cuda.synchronize()
    man.append(("(torch copies of re / im)", 2, 0, 0))
    call("conv_r2 two-for-one real", lambda: ops.conv_r2(xr, yr, b, n, ops.LAYOUT_R16_BPERM), 2 * pts, 12 * 2 * pts)
    call("conv_r2 two-for-one real, R8 filter (the reference's layout)",
         lambda: ops.conv_r2(xr, yr, b, n, ops.LAYOUT_R8), 2 * pts, 12 * 2 * pts)
    call("fwd_r2 (packed real pairs)", lambda: ops.fwd_r2(xr, yr, n, ops.LAYOUT_R16_BPERM), 2 * pts, 16 * pts)
    sp512 = spec[: 512 * n]
    fl = b[: 256 * n]
    og = torch.empty(2 * 512 * 256 * n, device="cuda")
    call("apply_grid_r2 (512 pairs x 256 filters)", lambda: ops.apply_grid_r2(sp512, fl, n, ops.LAYOUT_R16_BPERM, out=og),
         2 * 512 * 256 * n, 4 * 2 * 512 * 256 * n + 8 * n * (512 + 256))
    del og
    call("c2c forward (natural order)", lambda: ops.c2c(a, n, -1, out=o), pts, 16 * pts)
    call("filter_from_taps R16_BPERM", lambda: ops.filter_from_taps(a, n, ops.LAYOUT_R16_BPERM), pts, 16 * pts)
    call("filter_permute (device)", lambda: ops.filter_permute(a, n, ops.LAYOUT_R16_BPERM), pts, 16 * pts)
    h = w = 64
    call("conv2d 64x64 one CTA (shared filter, read directly)",
         lambda: ops.conv2d(a, b[: h * w], h, w, ops.LAYOUT_R16_BPERM, filter_stride=0, out=o), pts, 16 * pts)
    call("conv2d 64x64 per-image filter in the reference's radix-8 order (radix-16 engine, bit-permutation staging)",
         lambda: ops.conv2d(a, b, h, w, ops.LAYOUT_R8, out=o), pts, 24 * pts)
    call("conv2d 8x512 per-image filter in the reference's radix-8 order",
         lambda: ops.conv2d(a, b, 8, 512, ops.LAYOUT_R8, out=o), pts, 24 * pts)
    call("conv2d 256x256 cluster (shared filter)", lambda: ops.conv2d(a, b[: 65536], 256, 256, ops.LAYOUT_R16_BPERM, filter_stride=0, out=o),
         pts, 16 * pts)
    n2 = 32768
    call("conv N=32768 cluster C=8", lambda: ops.conv(a, b, n2, ops.LAYOUT_R16_BPERM, out=o), pts, 24 * pts)
    buf = a.clone()
    torch.cuda.synchronize()
    man.append(("(torch clone)", 1, 0, 0))
    call("four-step N=32768 cluster C=16", lambda: ops.conv_large(buf, b, n2, ops.LAYOUT_R16_BPERM, r_out=16, mid_size=2048), pts, 24 * pts)
    aq, as_ = ops.bfp_pack(a, n2)
    bq, bs = ops.bfp_pack(b, n2)
    torch.cuda.synchronize()
    man.append(("bfp_pack x2 (four-step inputs, n > 8192: abs-max pass + quantise pass)", 6, 0, 0))
    call("int16-BFP four-step N=32768 cluster C=16",
         lambda: ops.conv_large_bfp(aq, as_, bq, bs, n2, ops.LAYOUT_R16_BPERM, r_out=16, mid_size=2048),
         pts, 12 * pts + 12 * (pts // n2))
    del aq, bq
    n3 = 1 << 20
    r_out, mid = ops.large_plan(n3, ops.LAYOUT_R16)
    lout, q = 0, n3 // mid           # outer levels: n3 = r_out^lout * mid
    while q > 1:
        q //= r_out
        lout += 1
    call(f"four-step N=2^20 multi-kernel ({lout} outer r{r_out} levels each way, two per launch, + middle {mid})",
         lambda: ops.conv_large(buf, b, n3, ops.LAYOUT_R16, r_out=r_out, mid_size=mid), pts, 24 * pts,
         launches=2 * ((lout + 1) // 2) + 1)
    x = a[: 8 * (n3 // 64)].contiguous()
    torch.cuda.synchronize()
    man.append(("(torch copy)", 1, 0, 0))
    call("dist_pass (radix-8 outer pass of one rank, N=2^20)",
         lambda: check(lib().fufft_dist_pass(torch.view_as_real(x).data_ptr(), 8, n3 // 64, 0, n3, -1,
                                             torch.cuda.current_stream().cuda_stream), "fufft_dist_pass"),
         x.numel(), 16 * x.numel())
    assert ops.device_status() == 0
    for label, launches, points, nbytes in man:
        print(json.dumps({"call": label, "launches": launches, "points": points, "algorithmic_bytes": nbytes}))


def run_ncu_dist():
    """one process, two GPUs: one fused exchange launch of each kind per GPU
    (fufft_dist_pass_push: first DIF pass + NVLink stores into the peer's
    block; fufft_dist_pass_pull: NVLink loads + last DIT pass), n = 2^24, for
    an ncu capture of NVLink and DRAM bytes"""
    import ctypes as ct
    import torch
    from fufft_b200 import multi_gpu as mg
    from fufft_b200 import ops
    from fufft_b200._lib import check, lib
    world, n = 2, 1 << 24
    for d in range(world):
        torch.cuda.set_device(d)
        ops.init()
    cols = n // (world * world)
    slices, bb = [], []
    for r in range(world):
        g = torch.Generator(device=f"cuda:{r}")
        g.manual_seed(r)
        slices.append(torch.randn(world * cols, dtype=torch.complex64, device=f"cuda:{r}", generator=g))
        bb.append(torch.randn(n // world, dtype=torch.complex64, device=f"cuda:{r}", generator=g) / n)
    blocks = mg.conv_single_signal(slices, bb, n)       # enables peer access, allocates the blocks
    for r in range(world):
        torch.cuda.synchronize(r)
    addrs = (ct.c_uint64 * world)(*[b.data_ptr() for b in blocks])
    L = lib()
    for fn, name in ((L.fufft_dist_pass_push, "push"), (L.fufft_dist_pass_pull, "pull")):
        for r in range(world):
            with torch.cuda.device(r):
                check(fn(torch.view_as_real(slices[r]).data_ptr(), addrs, world, r, cols, n,
                         torch.cuda.current_stream().cuda_stream), name)
                torch.cuda.synchronize(r)


def run_ncu_case(which: str = "headline"):
    """one launch of each kernel of a group, on a batch of a few hundred MB
    (> L2), for ncu.  headline: fp32 (register-boundary filter), fp32 (linear
    chain filter, staged per warp), int16-BFP (linear chain filter) at N=4096; cluster: the
    cluster-fused N=32768 (radix-16 chain and the four-step recipe), 2-D
    256x256 and the int16-BFP four-step N=32768"""
    import torch
    from fufft_b200 import ops
    ops.init()
    if which == "cluster":
        g = torch.Generator(device="cuda")
        g.manual_seed(0)
        n, batch = 32768, 1024
        a = torch.randn(batch * n, dtype=torch.complex64, device="cuda", generator=g)
        b = torch.randn(batch * n, dtype=torch.complex64, device="cuda", generator=g) / n
        o = torch.empty_like(a)
        ops.conv(a, b, n, ops.LAYOUT_R16_BPERM, out=o)
        ops.conv_large(o, b, n, ops.LAYOUT_R16_BPERM, r_out=16, mid_size=2048)
        ops.conv2d(a, b[:65536], 256, 256, ops.LAYOUT_R16_BPERM, filter_stride=0, out=o)
        aq, as_ = ops.bfp_pack(a, n)
        bq, bs = ops.bfp_pack(b, n)
        ops.conv_large_bfp(aq, as_, bq, bs, n, ops.LAYOUT_R16_BPERM, r_out=16, mid_size=2048)
        torch.cuda.synchronize()
        assert ops.device_status() == 0
        return
    n, batch = N, POINTS // N // 2
    g = torch.Generator(device="cuda")
    g.manual_seed(0)
    a = torch.randn(batch * n, dtype=torch.complex64, device="cuda", generator=g)
    b = torch.randn(batch * n, dtype=torch.complex64, device="cuda", generator=g) / n
    out = torch.empty_like(a)
    aq = torch.randint(-32767, 32767, (batch * n, 2), dtype=torch.int16, device="cuda", generator=g)
    bq = torch.randint(-32767, 32767, (batch * n, 2), dtype=torch.int16, device="cuda", generator=g)
    sc = torch.full((batch,), 1e-4, device="cuda")
    ops.conv(a, b, n, ops.LAYOUT_R16_BPERM, ops.MID_MULTIPLY, out=out)
    ops.conv(a, b, n, ops.LAYOUT_R16, ops.MID_MULTIPLY, out=out)
    ops.conv_bfp(aq, sc, bq, sc, n, ops.LAYOUT_R16)
    torch.cuda.synchronize()
    assert ops.device_status() == 0


def run_dist(args, rank, world, dist):
    """one 2^26-point signal over `world` GPUs (config 5), two all-to-alls"""
    import torch
    from fufft_b200 import ops
    from fufft_b200.distributed import GpuBackend, PeerBlocks, conv_distributed, conv_distributed_p2p
    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", 0)))
    torch.cuda.set_device(dev)
    ops.init()
    n = 1 << 26
    be = GpuBackend()
    plan = be.plan(n, world)
    g = torch.Generator(device=dev)
    g.manual_seed(5000 + rank)
    x0 = torch.randn(world * plan.cols, dtype=torch.complex64, device=dev, generator=g)
    bb = torch.randn(plan.n_blk, dtype=torch.complex64, device=dev, generator=g) / n
    x = x0.clone()
    if args.dist_mode == "p2p":
        peers = PeerBlocks(plan.n_blk)
        ms = time_steps(torch, lambda: conv_distributed_p2p(x, bb, n, peers, backend=be, plan=plan), args.steps,
                        args.warmup, dist)
        peers.close()
    else:
        ms = time_steps(torch, lambda: conv_distributed(x, bb, n, backend=be, plan=plan), args.steps, args.warmup,
                        dist)
    hbm, _ = peaks()
    return {"metric": "distributed single-signal fused conv Gpoints/s, N=2^26", "value": round(n / (ms * 1e-3) / 1e9, 3),
            "unit": "Gpoints/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(ms, 4), "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "f32", "data": "synthetic", "config": {"workload": "configs[4] single N=2^26 signal",
            "plan": {"block": plan.n_blk, "r_out": plan.r_out, "mid": plan.mid, "chain": plan.chain},
            "nvlink_bytes_per_gpu": 2 * 8 * plan.n_blk * (world - 1) // world,
            "exchange": "NVLink stores / loads fused into the outer passes" if args.dist_mode == "p2p"
                        else "NCCL all_to_all"}}


def time_flushed(torch, fn, steps, warmup, flush_bytes=512 << 20, dist=None):
    """per-step device time of fn with L2 flushed before every step, outside
    the timed events; for workloads that fit in L2.  The flush writes a
    512 MiB buffer, then reads another 512 MiB one: the write evicts the
    step's data, the read turns L2 into clean lines, so the timed step pays
    neither for its own data in L2 nor for the write-back of the flush"""
    junk = torch.empty(flush_bytes, dtype=torch.uint8, device="cuda")
    clean = torch.ones(flush_bytes // 4, dtype=torch.float32, device="cuda")
    for _ in range(warmup):
        fn()
    tot = 0.0
    for _ in range(steps):
        junk.fill_(1)
        clean.sum()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        fn()
        e1.record()
        e1.synchronize()
        tot += e0.elapsed_time(e1)
    ms = tot / steps
    if dist:
        t = torch.tensor([ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    return ms


def run_sweep(args):
    """every BASELINE.json config on one GPU, one JSON line each (device time,
    Gpoints/s, algorithmic GB/s, fraction of the measured HBM peak)"""
    import torch
    from fufft_b200 import ops
    ops.init()
    hbm, _ = peaks()
    g = torch.Generator(device="cuda")
    g.manual_seed(1234)
    steps, warm = args.steps, args.warmup
    cfgs = {int(c) for c in args.configs.split(",")}

    def emit(cfg, ms, pts, bytes_per_pt, extra_bytes=0, **kw):
        gbs = (bytes_per_pt * pts + extra_bytes) / (ms * 1e-3) / 1e9
        print(json.dumps({"config": cfg, "ms": round(ms, 4), "Gpoints_s": round(pts / (ms * 1e-3) / 1e9, 2),
                          "GB_s": round(gbs, 1), "frac_hbm": round(gbs / hbm, 4), "bytes_per_point": bytes_per_pt,
                          **kw}), flush=True)

    # config 1: N=1024, batch 4096 (32 MiB per array: fits L2, so L2 is flushed per step)
    if 1 in cfgs:
        n, batch = 1024, 4096
        a = torch.randn(batch * n, dtype=torch.complex64, device="cuda", generator=g)
        b = torch.randn(batch * n, dtype=torch.complex64, device="cuda", generator=g) / n
        o = torch.empty_like(a)
        for lay, name in [(ops.LAYOUT_R16_BPERM, "R16_BPERM"), (ops.LAYOUT_R16, "R16")]:
            ms = time_flushed(torch, lambda: ops.conv(a, b, n, lay, out=o), steps, warm)
            emit(f"1: fp32 N={n} batch={batch} {name} (one launch, L2 flushed before it)", ms, batch * n, 24)
        # back-to-back batches over four input/output sets (384 MiB > 3x L2)
        sets = [(torch.randn_like(a), torch.randn_like(b), torch.empty_like(o)) for _ in range(4)]
        turn = [0]

        def step():
            x, f, y = sets[turn[0] % 4]
            turn[0] += 1
            ops.conv(x, f, n, ops.LAYOUT_R16_BPERM, out=y)
        ms = time_steps(torch, step, 4 * steps, warm, None)
        emit(f"1: fp32 N={n} batch={batch} R16_BPERM (back-to-back, 4 sets in turn)", ms, batch * n, 24)
        del a, b, o, sets
    # config 2: size sweep, 1 GiB of signal, fp32 and int16-BFP
    if 2 in cfgs:
        for n in (512, 1024, 2048, 4096):
            batch = POINTS // n
            a = torch.randn(batch * n, dtype=torch.complex64, device="cuda", generator=g)
            b = torch.randn(batch * n, dtype=torch.complex64, device="cuda", generator=g) / n
            o = torch.empty_like(a)
            for lay, name in [(ops.LAYOUT_R16_BPERM, "R16_BPERM"), (ops.LAYOUT_R16, "R16"), (ops.LAYOUT_R8, "R8")]:
                if n <= ops.max_n(lay):
                    ms = time_steps(torch, lambda: ops.conv(a, b, n, lay, out=o), steps, warm, None)
                    emit(f"2: fp32 N={n} {name}", ms, batch * n, 24)
            aq, as_ = ops.bfp_pack(a, n)
            bq, bs = ops.bfp_pack(b, n)
            for lay, name in [(ops.LAYOUT_R16, "R16"), (ops.LAYOUT_R16_BPERM, "R16_BPERM")]:
                ms = time_steps(torch, lambda: ops.conv_bfp(aq, as_, bq, bs, n, lay), steps, warm, None)
                emit(f"2: int16-BFP N={n} {name}", ms, batch * n, 12, 12 * batch)
            del a, b, o, aq, bq
    # config 3: 1024 real signals x 256 real filters at N=4096: packed pairs -> 512
    # spectra (fwd once per step) -> every pair against every filter in one launch,
    # 1024 x 256 x 4096 real outputs (4 GiB) per mid-op.  Bytes: 4 B per real output
    # point written; spectra, filters and the signals are read once (they stay in L2)
    if 3 in cfgs:
        n, nsig, nfilt = 4096, 1024, 256
        x = torch.randn(nsig * n, device="cuda", generator=g)
        taps = torch.rand(nfilt, n, device="cuda", generator=g) * 2 - 1
        b_nat = torch.fft.fft(taps.double(), dim=1) / n
        bp = ops.filter_permute(b_nat.to(torch.complex64).reshape(-1), n, ops.LAYOUT_R16_BPERM)
        xs = x.view(nsig // 2, 2, n)
        xr, yr = xs[:, 0].contiguous().view(-1), xs[:, 1].contiguous().view(-1)
        o = torch.empty(nsig * nfilt * n, device="cuda")
        for mid, mname in [(ops.MID_MULTIPLY, "multiply"), (ops.MID_CONJ_MULTIPLY, "conj-multiply")]:
            def step():
                spec = ops.fwd_r2(xr, yr, n, ops.LAYOUT_R16_BPERM)
                ops.apply_grid_r2(spec, bp, n, ops.LAYOUT_R16_BPERM, mid, out=o)
            ms = time_steps(torch, step, steps, warm, None)
            emit(f"3: real pairs N={n}: {nsig} signals x {nfilt} filters, fwd_r2 + apply_grid_r2 {mname} "
                 f"(4 GiB out)", ms, nsig * nfilt * n, 4, 8 * n * (nsig // 2 + nfilt) + 16 * n * (nsig // 2),
                 points="real output points")
        del x, taps, b_nat, bp, xs, xr, yr, o
    # 6: the rows beyond the configs -- natural-order c2c (16 B/pt: read + write)
    # and filter preparation from taps, N=4096 over 1 GiB of signal
    if 6 in cfgs:
        n = 4096
        batch = POINTS // n
        a = torch.randn(batch * n, dtype=torch.complex64, device="cuda", generator=g)
        o = torch.empty_like(a)
        for sign, name in [(-1, "forward"), (1, "inverse")]:
            ms = time_steps(torch, lambda: ops.c2c(a, n, sign, out=o), steps, warm, None)
            emit(f"6: natural-order c2c {name} N={n} batch={batch}", ms, batch * n, 16)
        ms = time_steps(torch, lambda: ops.filter_from_taps(a, n, ops.LAYOUT_R16_BPERM), steps, warm, None)
        emit(f"6: filter from taps N={n} batch={batch} (R16_BPERM)", ms, batch * n, 16)
        ms = time_steps(torch, lambda: ops.filter_permute(a, n, ops.LAYOUT_R16_BPERM), steps, warm, None)
        emit(f"6: filter permutation of natural spectra N={n} batch={batch} (R16_BPERM)", ms, batch * n, 16)
        # int16-BFP pack: one pass for n <= 8192 (8 read, 4 write per point, 4 per scale)
        ms = time_steps(torch, lambda: ops.bfp_pack(a, n), steps, warm, None)
        emit(f"6: int16-BFP pack N={n} batch={batch} (one pass)", ms, batch * n, 12, 4 * batch)
        # int16-BFP unpack: 4 read, 8 write per point, 4 per scale
        q, qs = ops.bfp_pack(a, n)
        ms = time_steps(torch, lambda: ops.bfp_unpack(q, qs, n), steps, warm, None)
        emit(f"6: int16-BFP unpack N={n} batch={batch}", ms, batch * n, 12, 4 * batch)
        del q, qs
        del o
        # fused two-for-one real convolution: 2 x 2^27 real points, one real filter
        # spectrum per pair (12 B per real point: 4+4 read, 8 filter per pair slot, 4+4 write)
        xr = a.real.contiguous()
        yr = a.imag.contiguous()
        taps = torch.rand(batch, n, device="cuda", generator=g) * 2 - 1
        bspec = ops.filter_from_taps(taps.to(torch.complex64).view(-1), n, ops.LAYOUT_R16_BPERM)
        del a, taps
        ms = time_steps(torch, lambda: ops.conv_r2(xr, yr, bspec, n, ops.LAYOUT_R16_BPERM), steps, warm, None)
        emit(f"6: two-for-one real conv N={n} x {2 * batch} real signals (R16_BPERM)", ms, 2 * batch * n, 12,
             points="real points")
        del xr, yr, bspec
    # 7: the reference's own yardstick (its published ratios are against a
    # cuFFT chain: README.md:12-13): cuFFT forward, pointwise multiply, cuFFT
    # inverse (torch.fft, three launches), against the fused kernel, same data
    if 7 in cfgs:
        for n in (512, 1024, 2048, 4096):
            batch = POINTS // n
            a = torch.randn(batch, n, dtype=torch.complex64, device="cuda", generator=g)
            b = torch.randn(batch, n, dtype=torch.complex64, device="cuda", generator=g) / n
            bp = ops.filter_permute(b.view(-1), n, ops.LAYOUT_R16_BPERM)
            o = torch.empty_like(a)
            ms_cufft = time_steps(torch, lambda: torch.fft.ifft(torch.fft.fft(a, dim=1) * b, dim=1, norm="forward"),
                                  steps, warm, None)
            ms_fused = time_steps(torch, lambda: ops.conv(a.view(-1), bp, n, ops.LAYOUT_R16_BPERM, out=o.view(-1)),
                                  steps, warm, None)
            emit(f"7: cuFFT chain fp32 N={n} (fft, multiply, ifft; comparison only)", ms_cufft, batch * n, 24,
                 fused_ms=round(ms_fused, 4), fused_speedup=round(ms_cufft / ms_fused, 2))
            del a, b, bp, o
    # config 4: 2-D 256x256 x 512 images, one shared filter
    if 4 in cfgs:
        h = w = 256
        batch = 512
        a = torch.rand(batch * h * w, device="cuda", generator=g).to(torch.complex64)
        b = torch.randn(h * w, dtype=torch.complex64, device="cuda", generator=g) / (h * w)
        o = torch.empty_like(a)
        for lay, name in [(ops.LAYOUT_R16, "R16"), (ops.LAYOUT_R16_BPERM, "R16_BPERM")]:
            ms = time_steps(torch, lambda: ops.conv2d(a, b, h, w, lay, filter_stride=0, out=o), steps, warm, None)
            emit(f"4: 2-D {h}x{w} batch={batch} shared filter {name} (cluster of 16 CTAs)", ms, batch * h * w, 16, 8 * h * w)
        del a, b, o
    # config 5: four-step N=32768, batch 2048, fp32 (cluster-fused) and int16-BFP (multi-kernel)
    if 5 in cfgs:
        n, batch = 32768, 2048
        r_out, mid = ops.large_plan(n, ops.LAYOUT_R16)
        a = torch.randn(batch * n, dtype=torch.complex64, device="cuda", generator=g)
        b = torch.randn(batch * n, dtype=torch.complex64, device="cuda", generator=g) / n
        buf = a.clone()
        for lay, name in [(ops.LAYOUT_R16, "R16"), (ops.LAYOUT_R16_BPERM, "R16_BPERM")]:
            ms = time_steps(torch, lambda: ops.conv_large(buf, b, n, lay, r_out=r_out, mid_size=mid),
                            steps, warm, None)
            emit(f"5: fp32 four-step N={n} batch={batch} {name} (r_out {r_out}, mid {mid}: one cluster kernel)",
                 ms, batch * n, 24)
            ms = time_steps(torch, lambda: ops.conv(a, b, n, lay, out=buf), steps, warm, None)
            emit(f"5: fp32 N={n} batch={batch} {name} radix-16 chain (cluster of 8 CTAs)", ms, batch * n, 24)
        aq, as_ = ops.bfp_pack(a, n)
        bq, bs = ops.bfp_pack(b, n)
        ws = torch.empty(batch * n * 8, dtype=torch.uint8, device="cuda")
        for lay, name in [(ops.LAYOUT_R16, "R16"), (ops.LAYOUT_R16_BPERM, "R16_BPERM")]:
            ms = time_steps(torch, lambda: ops.conv_large_bfp(aq, as_, bq, bs, n, lay, workspace=ws),
                            steps, warm, None)
            emit(f"5: int16-BFP four-step N={n} batch={batch} {name} (r_out {r_out}, mid {mid}: one cluster kernel)",
                 ms, batch * n, 12, 12 * batch)


def run_reference(args, rank, world):
    if rank != 0:
        return None
    # each step: a bounded sample of the workload on every host core, sized so
    # the whole run stays near 90 s whatever --steps / --warmup ask for
    rates = []
    kind = cores = sample = None
    per_step = min(args.ref_seconds, 90.0 / max(1, args.warmup + args.steps))
    for i in range(args.warmup + args.steps):
        rate, kind, cores, sample = cpu_reference_rate(per_step)
        if i >= args.warmup:
            rates.append(rate)
    v = statistics.median(rates) / 1e9
    return {
        "metric": "fused conv Gpoints/s + HBM GB/s (% of B200 peak) at N=4096 fp32 & int16-BFP",
        "impl": "reference", "value": round(v, 6), "unit": "Gpoints/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": headline_config(args.n, POINTS // args.n, world),
        "path": "host cores: the reference's own CPU transcription kernel_pipeline_v16 (verify_kernel.cpp:1051), "
                "one thread per batch slice",
        "cpu_baseline": {"value": round(v, 6), "unit": "Gpoints/s", "cores": cores, "kind": kind, "sample": sample},
        "e2e": {"value": round(v, 6), "unit": "Gpoints/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--n", type=int, default=N)
    ap.add_argument("--cpu-seconds", type=float, default=2.0, help="per-thread CPU baseline sample")
    ap.add_argument("--ref-seconds", type=float, default=1.0, help="per-thread sample per reference step")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-configs", action="store_true", help="headline only (no per-config records)")
    ap.add_argument("--no-dist", action="store_true", help="under torchrun: no single-signal record")
    ap.add_argument("--ncu-case", nargs="?", const="headline", default=None,
                    choices=["headline", "cluster", "all", "dist"],
                    help="one launch per kernel of a group, for ncu (dist: two GPUs, one process)")
    ap.add_argument("--dist-mode", choices=["p2p", "nccl"], default="p2p",
                    help="dist: all-to-alls fused into the outer passes over NVLink (p2p) or NCCL all_to_all")
    ap.add_argument("--configs", default="1,2,3,4,5,6,7",
                    help="sweep: which BASELINE.json configs (1-based); 6 = c2c and filter preparation, "
                         "7 = the cuFFT chain the reference compares against")
    ap.add_argument("--workload", choices=["batch", "dist", "sweep"], default="batch",
                    help="dist: one 2^26-point signal over all ranks (2, 4 or 8); sweep: every "
                         "BASELINE.json config on one GPU, one JSON line each")
    args = ap.parse_args()
    if args.ncu_case == "all":
        run_ncu_all()
        return
    if args.ncu_case == "dist":
        run_ncu_dist()
        return
    if args.ncu_case:
        run_ncu_case(args.ncu_case)
        return
    if args.workload == "sweep":
        run_sweep(args)
        return
    args.warmup = max(args.warmup, 3)

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    dist = None
    if world > 1 and args.impl == "ours":
        import datetime
        import torch
        import torch.distributed as td
        torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", 0)))
        td.init_process_group("nccl", timeout=datetime.timedelta(seconds=120))
        dist = td
    try:
        if args.impl == "reference":
            line = run_reference(args, rank, world)
        elif args.workload == "dist":
            line = run_dist(args, rank, world, dist)
        else:
            line = run_ours(args, rank, world, dist)
        if rank == 0 and line is not None:
            print(json.dumps(line), flush=True)
    finally:
        if dist is not None:
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
