"""Benchmark of the SSD prefill scan (one JSON line on rank 0).

Workload: S=1, L=8192, H=64, P=64, N=128, G=8, x/B/C
bf16, dt/A/s0 f32, y/s1 f32, multipass.  Under torchrun the 64 heads of that
one problem are split over the ranks in whole head groups (8 heads per rank
at N=8); heads never interact, so there is no collective on the data path
("scaling": "strong").  `value` = the problem's tokens over the max device
time of any rank.  --scaling weak gives every rank its own copy of the problem
instead (value counts every rank's tokens).

Timing: W warm-up steps, then K steps; before each step a 256 MiB buffer is
written (flushing the 126 MB L2; the flush is outside the timed events); each
step is bracketed by CUDA events on the launching stream; barrier +
synchronize on both sides of the loop; max over ranks.

Also reported: per-pass attribution (state, carry and output passes timed
alone, each with its algorithmic bytes, GB/s and fraction of measured HBM
bandwidth, and the state pass's contraction rate), the roofline of the
output kernel (the dominant one), e2e through the C ABI with pinned host
buffers (H2D of the step's inputs and D2H of y and s1 inside the timed region;
steps in flight on two buffer sets with the copies on their own streams, the
one-step-at-a-time figure beside it as serial_ms_per_step), the CPU baselines
(the reference's own fp64 oracles -- sequential scan and chunked scan --
compiled from its sources into oracle/_ref, run over (seq, head) slices on
all host cores over the whole workload), and SM clocks sampled during the
timed region.

--impl reference times the reference's CPU implementation alone (rank 0): one
step is one whole scan of the workload.
"""
from __future__ import annotations

import argparse
import ctypes as C
import json
import os
import statistics
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "SSD prefill tok/s and % of TC/HBM roofline, L=8192 H64 P64 N128, 1/2/4/8 B200"
UNIT = "tok/s"
BACKENDS = {"auto": 0, "sgmma": 1, "mpp": 2, "ref": 3}  # helix_backend
FAMILIES = {0: "exact fp32 cuda-core", 1: "tcgen05 bf16", 2: "tcgen05 fp32-class (bf16 hi+lo, three products)",
            3: "diagonal-A recurrence (cuda-core fp32)"}


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--config", default="c3")
    ap.add_argument("--compute", default="config", choices=["config", "bf16", "f32"],
                    help="operand precision (default: the config's: bf16 for c3/c5, f32 for c1/c2/c4)")
    ap.add_argument("--backend", default="auto", choices=["auto", "sgmma", "mpp", "ref"],
                    help="helix_backend of the descriptor (ref: the exact fp32 CUDA-core kernels)")
    ap.add_argument("--io", default="config", choices=["config", "bf16", "f32"],
                    help="storage of x, B, C (default: the config's)")
    ap.add_argument("--scaling", default="strong", choices=["strong", "weak"],
                    help="N>1: split one problem's heads over the ranks (strong) or give each rank its own")
    ap.add_argument("--cpu-sample-tokens", type=int, default=0,
                    help="tokens of the CPU baseline's sample (0: the whole sequence)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--lsplit", type=int, default=0,
                    help="token shards per head shard: run the L-split mesh on --config (default c5)")
    ap.add_argument("--seqs", type=int, default=0, help="override the config's sequence count (L-split mode)")
    ap.add_argument("--a-form", default="scalar", choices=["scalar", "diag"],
                    help="diag: one decay rate per (head, state) (Mamba-1), the recurrence kernels; "
                         "each head's rate times a seeded factor in [1/4, 4] per state")
    return ap.parse_args()


# ---------------------------------------------------------------------------
# CPU baseline: the reference's own oracle (or our restatement) on host cores.
# ---------------------------------------------------------------------------
def cpu_baseline(shape, sample_tokens: int, which: str = "scan"):
    """The reference's fp64 oracle (helix::ref::scan, or helix::ref::scan_chunked
    with which="chunked") over the workload's (seq, head) slices on all host
    cores; `sample_tokens` > 0 times only that many leading tokens."""
    import numpy as np

    from helix_b200.synth import make_inputs, to_numpy_f32
    from oracle.oracle import Oracle, Reference, available_reference

    kind = "reference" if available_reference() else "port"
    impl = Reference() if kind == "reference" else Oracle()
    T = min(sample_tokens, shape.L) if sample_tokens > 0 else shape.L
    sub = type(shape)(shape.S, T, shape.H, shape.P, shape.N, shape.G, shape.io)
    t = make_inputs(sub, seed=99)
    prob = {k: np.ascontiguousarray(to_numpy_f32(t[k])) for k in ("s0", "x", "dt", "A", "B", "C")}
    cores = len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else (os.cpu_count() or 1)
    base = Oracle().desc_init(T, sub.S, sub.H, sub.P, sub.N, sub.G)
    y = np.zeros((sub.S, T, sub.H, sub.P), np.float32)
    s1 = np.zeros((sub.S, sub.H, sub.P, sub.N), np.float32)
    F = C.POINTER(C.c_float)
    pre = "ref_" if kind == "reference" else "oracle_"
    fn = getattr(impl.lib, pre + ("scan_chunked" if which == "chunked" else "scan"))
    hpg = sub.H // sub.G

    # One call per (seq, head) slice: a descriptor with n_head = n_group = 1
    # and pointers offset to the slice, exactly the reference's own code per
    # slice; ctypes releases the GIL, so the slices run on all cores.
    def slice_call(seq, h):
        from helix_b200.abi import ScanDesc
        d = ScanDesc()
        C.memmove(C.byref(d), C.byref(base), C.sizeof(ScanDesc))
        d.n_head, d.n_group, d.n_seq = 1, 1, 1
        g = h // hpg
        off = lambda a, i: C.cast(a.ctypes.data + 4 * i, F)  # noqa: E731
        fn(C.byref(d), off(prob["s0"], seq * base.seq_s + h * base.s_s[0]),
           off(prob["x"], seq * base.seq_x + h * base.s_x[1]),
           off(prob["dt"], seq * base.seq_dt + h * base.s_dt[1]), off(prob["A"], h),
           off(prob["B"], seq * base.seq_b + g * base.s_b[1]),
           off(prob["C"], seq * base.seq_c + g * base.s_c[1]), None,
           off(y, seq * base.seq_y + h * base.s_y[1]), off(s1, seq * base.seq_s + h * base.s_s[0]))

    from concurrent.futures import ThreadPoolExecutor
    jobs = [(s, h) for s in range(sub.S) for h in range(sub.H)]
    t0 = time.perf_counter()
    with ThreadPoolExecutor(max_workers=cores) as ex:
        list(ex.map(lambda a: slice_call(*a), jobs))
    sec = time.perf_counter() - t0
    value = sub.S * T / sec  # tokens of the full H-head layer per second
    name = "helix::ref::scan_chunked" if which == "chunked" else "helix::ref::scan"
    return dict(value=value, unit=UNIT, cores=cores, kind=kind, seconds=sec,
                sample=f"{'all ' + str(T) if T == shape.L else str(T) + ' of ' + str(shape.L)} tokens, "
                       f"all {sub.H} heads, S={sub.S}; "
                       f"{name + ' (reference sources)' if kind == 'reference' else 'C port of ' + name}"
                       f" per (seq, head) slice on {cores} threads; {sec:.2f} s wall")


# ---------------------------------------------------------------------------
def _clock_sampler(bus_id, index, conn, stop):
    """Child process: polls NVML every ~0.2 ms from start-up until `stop`, then
    sends [(monotonic time, sm_mhz, event_reasons)] and the max SM clock."""
    rows, max_mhz = [], None
    try:
        import pynvml as nv
        nv.nvmlInit()
        try:
            h = nv.nvmlDeviceGetHandleByPciBusId(bus_id) if bus_id else nv.nvmlDeviceGetHandleByIndex(index)
        except Exception:
            h = nv.nvmlDeviceGetHandleByIndex(index)
        max_mhz = nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM)
        conn.send("ready")
        while not stop.is_set():
            try:
                rows.append((time.monotonic(), nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM),
                             nv.nvmlDeviceGetCurrentClocksEventReasons(h)))
            except Exception:
                pass
            time.sleep(0.0002)
    except Exception:
        try:
            conn.send("ready")
        except Exception:
            pass
    conn.send((rows, max_mhz))


class Clocks:
    """SM clock and throttle-reason sampler for the timed region: NVML polled
    every ~0.2 ms by a spawned child process (a thread of this process would
    wait for the GIL while the launching thread enqueues the steps, and
    nvidia-smi's cadence is too coarse for a region of a few milliseconds).
    The child polls from start-up; the samples kept are those taken between
    `__enter__` and `__exit__` (CLOCK_MONOTONIC is shared by the processes)."""

    REASONS = {"hw_slowdown": 0x8, "hw_thermal_slowdown": 0x40, "sw_thermal_slowdown": 0x20,
               "sw_power_cap": 0x4, "hw_power_brake_slowdown": 0x80}

    def __init__(self, index: int):
        self.index, self.rows, self.max_mhz, self.proc = index, [], None, None
        self.t0 = self.t1 = None
        self.polled, self.span_ms = 0, None  # all samples the child took; its first/last vs the window
        try:
            import multiprocessing as mp
            import torch
            bus = None
            try:  # same physical GPU as the CUDA ordinal, whatever the visibility mask
                pr = torch.cuda.get_device_properties(index)
                bus = f"{pr.pci_domain_id:08x}:{pr.pci_bus_id:02x}:{pr.pci_device_id:02x}.0"
            except Exception:
                pass
            ctx = mp.get_context("spawn")
            self.conn, child = ctx.Pipe()
            self.stop = ctx.Event()
            self.proc = ctx.Process(target=_clock_sampler, args=(bus, index, child, self.stop), daemon=True)
            self.proc.start()
            if not (self.conn.poll(60) and self.conn.recv() == "ready"):
                raise RuntimeError("sampler did not start")
        except Exception:
            self._end()

    def _end(self):
        if self.proc is not None:
            self.proc.kill()
            self.proc = None

    def __enter__(self):
        self.t0 = time.monotonic()
        return self

    def __exit__(self, *a):
        self.t1 = time.monotonic()
        if self.proc is None:
            return
        self.stop.set()
        try:
            if self.conn.poll(10):
                rows, self.max_mhz = self.conn.recv()
                self.rows = [(m, r) for t, m, r in rows if self.t0 <= t <= self.t1]
                self.polled = len(rows)
                if rows:
                    self.span_ms = (round(1e3 * (rows[0][0] - self.t0), 2), round(1e3 * (rows[-1][0] - self.t1), 2))
        except Exception:
            pass
        self.proc.join(timeout=5)
        self._end()

    def summary(self):
        if not self.rows:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": ["unsampled"], "samples": 0,
                    "polled": self.polled, "first_last_vs_window_ms": self.span_ms,
                    "window_ms": None if self.t1 is None else round(1e3 * (self.t1 - self.t0), 2)}
        mhz = [r[0] for r in self.rows]
        reasons = sorted({n for _, m in self.rows for n, bit in self.REASONS.items() if m & bit})
        return {"sm_mhz": statistics.median(mhz), "sm_max_mhz": self.max_mhz, "reasons": reasons,
                "samples": len(self.rows), "window_ms": round(1e3 * (self.t1 - self.t0), 2),
                "source": "nvml, polled every ~0.2 ms by a child process during the timed steps"}


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        j = json.loads(p.read_text())
        return float(j["hbm_gbs"]), float(j["bf16_tflops"]), "measured"
    return 6650.0, 1590.0, "fallback"


# ---------------------------------------------------------------------------
def bench_lsplit(a, rank: int, world: int, local: int) -> int:
    """L-split mesh: world = (world / K head shards) x (K token shards) over
    the global workload of --config.  A step is one scan_lsplit on every rank
    (shard state, two all-gathers over the token group, carry combine, shard
    scan); value = global tokens / max device time over ranks (strong
    scaling: the global problem is fixed)."""
    import torch
    import torch.distributed as dist
    from datetime import timedelta

    import helix_b200
    from helix_b200 import dist as hdist
    from helix_b200.synth import Shape, make_inputs

    cfg = a.config if a.config != "c3" else "c5"
    g = Shape.of(cfg)
    S = a.seqs or g.S
    K = a.lsplit
    if world % K or g.L % (K * 128):
        raise SystemExit(f"--lsplit {K} does not divide {world} ranks / L={g.L}")
    n_hs = world // K
    hs, ls = rank // K, rank % K
    h0, h1 = hdist.head_slice(g.H, g.G, hs, n_hs)
    Lk = g.L // K
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
    groups = [dist.new_group(list(range(q * K, (q + 1) * K))) for q in range(n_hs)] if world > 1 else [None]
    grp = groups[hs]
    local_shape = Shape(S, Lk, h1 - h0, g.P, g.N, (h1 - h0) // (g.H // g.G), g.io)
    t = make_inputs(local_shape, seed=7000 + rank, device=dev)
    gA = torch.Generator(device=dev)
    gA.manual_seed(9000 + hs)
    t["A"] = -torch.exp(torch.rand(h1 - h0, generator=gA, device=dev) * 2.772588722239781)
    ops = hdist.GpuOps(compute=a.compute)
    d_scan = helix_b200.desc_from_tensors(t["x"], t["dt"], t["B"], t["s0"], None, multipass=True,
                                          compute=a.compute)
    ctx = helix_b200._ctx_for(t["x"], None)
    n_sb = ctx.scratch_size(d_scan)
    has_runs = n_sb >= t["x"].shape[0] * t["x"].shape[2] * t["x"].shape[3] * t["s0"].shape[-1] * 4
    # per step: state kernel + fold, carry combine, then the shard scan from
    # the kept run states (carry kernel with several output spans, then the
    # output kernel + general-path kernel of the bf16 family, or the one
    # output kernel of the fp32-class family, which also casts first)
    if a.compute == "bf16":
        launches = 3 + (1 if has_runs else 0) + 2
    else:
        launches = 4 + (1 if has_runs else 0) + 1
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream(dev)

    def step():
        if world > 1:
            return hdist.scan_lsplit(t["x"], t["dt"], t["A"], t["B"], t["C"], t["s0"], group=grp, ops=ops)
        st, ld, keep = ops.shard_state_keep(t["x"], t["dt"], t["A"], t["B"], t["C"])
        carry = ops.carry_combine(t["s0"], st[None][:0], ld[None][:0], None)
        return ops.scan_shard(t["x"], t["dt"], t["A"], t["B"], t["C"], carry, keep)

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local])
        torch.cuda.synchronize(dev)

    for _ in range(a.warmup):
        flush.fill_(1)
        step()
    barrier()
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(a.steps)]
    with Clocks(local) as clk:
        barrier()
        for e0, e1 in evs:
            flush.fill_(1)
            e0.record(stream)
            step()
            e1.record(stream)
        barrier()
    ms = sum(e0.elapsed_time(e1) for e0, e1 in evs) / a.steps
    if world > 1:
        tt = torch.tensor([ms], device=dev, dtype=torch.float64)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        ms = float(tt.item())
    gshape = Shape(S, g.L, g.H, g.P, g.N, g.G, g.io)
    value = S * g.L / (ms * 1e-3)
    hbm, tc, peak_kind = peaks()
    if rank == 0:
        print(json.dumps({
            "metric": "SSD prefill tok/s, L-split mesh (head shards x token shards)", "value": value,
            "unit": UNIT, "n_gpus": world, "steps": a.steps, "warmup": a.warmup, "ms_per_step": ms,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "bf16" if a.compute == "bf16" else "f32",
            "data": "synthetic (seeded per rank, BASELINE distributions)",
            "config": {"workload": f"{cfg}: S={S} L={g.L} H={g.H} P={g.P} N={g.N} G={g.G} as {n_hs} head "
                                   f"shards x {K} token shards; per rank S={S} L={Lk} H={h1 - h0}",
                       "l2": "flushed before every timed step (256 MiB write, untimed)",
                       "step": "shard state + 2 all-gathers + carry combine + shard scan",
                       "tflops": gshape.flops() / (ms * 1e-3) / 1e12,
                       "path_gbs": gshape.alg_bytes() / (ms * 1e-3) / 1e9,
                       "path_hbm_frac_per_gpu": gshape.alg_bytes() / world / (ms * 1e-3) / 1e9 / hbm},
            "gpu_launches": launches * a.steps, "clocks": clk.summary()}), flush=True)
    if world > 1:
        dist.barrier(device_ids=[local])
        dist.destroy_process_group()
    return 0


def pass_figures(shape, info, ms, hbm, tc):
    """Algorithmic bytes (and flops) of each pass for one scan of `shape` under
    plan `info`, with the achieved rates of the measured times ms[pass]."""
    e = 2 if shape.io == "bf16" else 4
    S, L, H, P, N, G = shape.S, shape.L, shape.H, shape.P, shape.N, shape.G
    st = S * H * P * N * 4
    runs = info.state_runs
    tok_a = min(L, runs * info.run_tokens)
    # state pass: x, dt and B of the runs it reduces, one state + decay + span per run
    a_bytes = S * tok_a * (H * P * e + H * 4 + G * N * e) + runs * (st + 3 * S * H * 4)
    a_flops = 2.0 * S * H * tok_a * P * N
    # carry pass: run states read, span-entry states written back, s0 and decays read
    b_bytes = runs * st + max(info.n_spans - 1, 0) * st + st + runs * S * H * 4
    # output pass: x, B, C, dt read once, y written once, s0 (or span states) read, s1 written
    c_bytes = S * L * H * P * e + 2 * S * L * G * N * e + S * L * H * 4 + S * L * H * P * 4 + 2 * st
    # cast pass: B, C (and x, for the bf16 family) read as f32, written as
    # bf16 (hi, and lo for the fp32-class family, which reads the bench's
    # dense fp32 x in place)
    planes = 2 if info.family == 2 else 1
    x_bytes = S * L * ((H * P if info.family == 1 else 0) + 2 * G * N)
    x_bytes = x_bytes * 4 + x_bytes * 2 * planes
    out = {}
    for name, by, fl in (("state", a_bytes, a_flops), ("carry", b_bytes, 0.0), ("output", c_bytes, None),
                         ("cast", x_bytes, None)):
        t = ms.get(name, 0.0)
        if not t:
            continue
        gbs = by / (t * 1e-3) / 1e9
        d = {"ms": t, "alg_bytes": by, "gbs": gbs, "hbm_frac": gbs / hbm}
        if fl:
            d["tflops"] = fl / (t * 1e-3) / 1e12
            d["tensor_frac"] = d["tflops"] / tc
        out[name] = d
    return out, c_bytes


def reference_arm(a, shape, rank):
    if rank != 0:
        return 0
    steps = []
    cb = None
    for i in range(a.warmup + a.steps):
        cb = cpu_baseline(shape, a.cpu_sample_tokens)
        if i >= a.warmup:
            steps.append(cb["seconds"])
    sec = statistics.median(steps)
    v = shape.S * (min(a.cpu_sample_tokens, shape.L) if a.cpu_sample_tokens > 0 else shape.L) / sec
    cb["value"] = v
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": v, "unit": UNIT, "n_gpus": a.gpus,
        "steps": a.steps, "warmup": a.warmup, "ms_per_step": 1e3 * shape.S * shape.L / v,
        "higher_is_better": True, "scaling": a.scaling, "vs_baseline": None, "dtype": "f64",
        "data": "synthetic (seeded, BASELINE distributions)",
        "config": {"workload": f"{a.config}: S={shape.S} L={shape.L} H={shape.H} P={shape.P} "
                               f"N={shape.N} G={shape.G}; one whole scan per step on the host cores",
                   "sample": cb["sample"]},
        "cpu_baseline": cb, "e2e": {"value": v, "unit": UNIT, "h2d_bytes_per_step": 0,
                                    "d2h_bytes_per_step": 0}}), flush=True)
    return 0


def main():
    a = parse()
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))

    from helix_b200.synth import Shape
    if a.compute == "config":
        a.compute = "bf16" if Shape.of(a.config if not a.lsplit or a.config != "c3" else "c5").io == "bf16" else "f32"
    if a.lsplit and a.impl != "reference":
        return bench_lsplit(a, rank, world, local)
    gshape = Shape.of(a.config)
    if a.impl == "reference":
        return reference_arm(a, gshape, rank)

    import torch
    import torch.distributed as dist

    import helix_b200
    from helix_b200 import abi
    from helix_b200 import dist as hdist
    from helix_b200.synth import make_inputs

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)

    strong = a.scaling == "strong" and world > 1
    if strong:
        # this rank's whole head groups of the one global problem
        h0, h1 = hdist.head_slice(gshape.H, gshape.G, rank, world)
        hpg = gshape.H // gshape.G
        shape = Shape(gshape.S, gshape.L, h1 - h0, gshape.P, gshape.N, (h1 - h0) // hpg, gshape.io)
        t = make_inputs(gshape, seed=1000, device=dev, heads=(h0, h1))
    else:
        shape = gshape
        t = make_inputs(shape, seed=1000 + rank, device=dev)
    ctx = helix_b200.Context(local)
    x, dt, A, B, Cm, s0 = t["x"], t["dt"], t["A"], t["B"], t["C"], t["s0"]
    if a.compute == "bf16" and x.dtype != torch.bfloat16 and a.io == "bf16":
        x, B, Cm = x.to(torch.bfloat16), B.to(torch.bfloat16), Cm.to(torch.bfloat16)
    if a.io == "f32" and x.dtype != torch.float32:
        x, B, Cm = x.float(), B.float(), Cm.float()
    shape = Shape(shape.S, shape.L, shape.H, shape.P, shape.N, shape.G,
                  "bf16" if x.dtype == torch.bfloat16 else "f32")
    y = torch.empty(x.shape, dtype=torch.float32, device=dev)
    s1 = torch.empty_like(s0)
    if a.a_form == "diag":
        gen = torch.Generator(device=dev).manual_seed(4242)
        f = torch.exp((torch.rand(A.shape[0], shape.N, device=dev, generator=gen) * 2 - 1) * torch.log(
            torch.tensor(4.0, device=dev)))
        A = (A[:, None] * f).contiguous()
    d = helix_b200.desc_from_tensors(x, dt, B, s0, y, multipass=True, compute=a.compute,
                                     backend=BACKENDS[a.backend], A=A)
    if not ctx.supported(d):
        raise SystemExit(f"descriptor unsupported: {ctx.last_error()}")
    info = ctx.plan_info(d)
    nbytes = ctx.scratch_size(d)
    scratch = torch.empty(max(nbytes, 256), dtype=torch.uint8, device=dev)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream(dev)

    def step():
        st = ctx.encode(d, s0, x, dt, A, B, Cm, y, s1, scratch=scratch, stream=stream)
        if st != abi.HELIX_OK:
            raise SystemExit(f"encode failed: {ctx.last_error()}")

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local])
        torch.cuda.synchronize(dev)

    def timed(fn, k, pre=None):
        evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(k)]
        barrier()
        for e0, e1 in evs:
            flush.fill_(1)
            if pre:
                pre()
            e0.record(stream)
            fn()
            e1.record(stream)
        barrier()
        return [e0.elapsed_time(e1) for e0, e1 in evs]

    def max_over_ranks(v: float) -> float:
        if world == 1:
            return v
        tt = torch.tensor([v], device=dev, dtype=torch.float64)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        return float(tt.item())

    for _ in range(a.warmup):
        flush.fill_(1)
        step()
    barrier()
    with Clocks(local) as clk:
        ms = timed(step, a.steps)
    total_ms = max_over_ranks(sum(ms))
    ms_per_step = total_ms / a.steps
    # tcgen05 bf16 family: state + carry kernels when runs are carried, then
    # per 128 states the output kernels (fast path, general path); tcgen05
    # fp32-class family: state + carry, then one output kernel per 128
    # states; exact fp32 family: state kernel when runs are carried, then
    # the output kernel; plus the cast kernel where the plan has one
    has_runs = info.state_runs > 0
    n_half = (shape.N + 127) // 128
    if info.family == 1:
        launches = (2 if has_runs else 0) + 2 * n_half
    elif info.family == 2:
        launches = (2 if has_runs else 0) + n_half
    else:  # exact fp32 and diagonal-A families: state kernel when runs are carried, output kernel
        launches = (1 if has_runs else 0) + 1
    n_cast = cast_launches(ctx, d)
    launches += n_cast

    # ---- per-pass attribution (same steps, passes split) --------------
    def only(p):
        def f():
            os.environ["HELIX_ONLY_PASS"] = p
            try:
                step()
            finally:
                os.environ.pop("HELIX_ONLY_PASS", None)
        return f
    ms_pass = {"output": max_over_ranks(sum(timed(only("C"), a.steps))) / a.steps}
    if has_runs:
        ms_pass["state"] = max_over_ranks(sum(timed(only("A"), a.steps))) / a.steps
    if has_runs and info.family in (1, 2):
        ms_pass["carry"] = max_over_ranks(sum(timed(only("B"), a.steps))) / a.steps
    if n_cast:
        ms_pass["cast"] = max_over_ranks(sum(timed(only("X"), a.steps))) / a.steps

    hbm, tc, peak_kind = peaks()
    passes, out_bytes = pass_figures(shape, info, ms_pass, hbm, tc)
    if info.family in (1, 2):
        # MMA work the output kernels issue per scan (bf16 flops, every pass
        # of every GEMM at its full tile), against measured bf16 peak
        units = shape.S * shape.H * ((shape.P + 63) // 64) * ((shape.L + 127) // 128) * n_half
        per_unit = 2 * 128 * 128 * 128 * 3 + 9 * 2 * 128 * 64 * 128 if info.family == 2 else \
            (2 * 128 * 128 * 128 * 5) / 2  # bf16: five 128-cube GEMMs per pair of slabs
        mma = units * per_unit
        passes["output"]["mma_flops"] = mma
        passes["output"]["mma_tflops"] = mma / (ms_pass["output"] * 1e-3) / 1e12
        passes["output"]["mma_tensor_frac"] = passes["output"]["mma_tflops"] / tc
    if info.family == 3:
        # the recurrence: per (token, head, channel, state) one multiply and
        # two fused multiply-adds in the output pass (5 flops), one multiply
        # and one in the state pass (3), against the nominal CUDA-core fp32
        # rate (148 SMs x 128 lanes x 2 flops x the max SM clock)
        upd = shape.S * shape.L * shape.H * shape.P * shape.N
        fp32_peak = 148 * 128 * 2 * 1.965e9 / 1e12
        for name, fl, tok in (("output", 5.0, shape.L), ("state", 3.0, min(shape.L, info.state_runs * info.run_tokens))):
            if name in passes:
                tf = fl * upd * tok / shape.L / (ms_pass[name] * 1e-3) / 1e12
                passes[name].pop("tflops", None)
                passes[name].pop("tensor_frac", None)
                passes[name]["fp32_tflops"] = tf
                passes[name]["fp32_frac_of_nominal"] = tf / fp32_peak
    achieved = out_bytes / (ms_pass["output"] * 1e-3) / 1e9
    traffic = None  # DRAM bytes per launch of the output kernel, from the committed ncu capture
    tj = ROOT / "profiles" / "ncu_traffic.json"
    if tj.exists() and not strong:
        traffic = json.loads(tj.read_text()).get(f"{a.config}/{a.compute}", {}).get("dram_bytes_per_launch")
    # tokens the job processed: the problem's tokens (one GPU, or its heads
    # split over the ranks), or every rank's own copy of the problem (weak)
    job_tok = gshape.S * gshape.L * (world if a.scaling == "weak" and world > 1 else 1)
    path_gbs = shape.alg_bytes() / (ms_per_step * 1e-3) / 1e9
    tflops = (gshape.flops() if strong else world * shape.flops()) / (ms_per_step * 1e-3) / 1e12

    # ---- e2e through the C ABI with host buffers ------------------------
    e2e = None
    if not a.no_e2e:
        host = {k: v.to("cpu").pin_memory() for k, v in dict(x=x, dt=dt, A=A, B=B, C=Cm, s0=s0).items()}
        yh = torch.empty(y.shape, dtype=torch.float32, pin_memory=True)
        sh = torch.empty(s1.shape, dtype=torch.float32, pin_memory=True)
        h2d = sum(v.numel() * v.element_size() for v in host.values())
        d2h = yh.numel() * 4 + sh.numel() * 4

        def e2e_step():
            for k, v in host.items():
                dict(x=x, dt=dt, A=A, B=B, C=Cm, s0=s0)[k].copy_(v, non_blocking=True)
            step()
            yh.copy_(y, non_blocking=True)
            sh.copy_(s1, non_blocking=True)
        for _ in range(2):
            e2e_step()
        serial_ms = max_over_ranks(sum(timed(e2e_step, max(3, a.steps // 4)))) / max(3, a.steps // 4)

        # Steps in flight the way a serving loop runs them: two device buffer
        # sets, inputs uploaded on one copy stream and results read back on
        # another, so step k+1's upload and step k-1's read-back overlap step
        # k's scan.  Every step still moves its own inputs in and y, s1 out
        # inside the timed region; each step's working set (inputs + y) is
        # larger than L2, so no flush is needed between them.
        sets = [dict(x=x, dt=dt, A=A, B=B, C=Cm, s0=s0, y=y, s1=s1),
                {k: v.clone() for k, v in dict(x=x, dt=dt, A=A, B=B, C=Cm, s0=s0, y=y, s1=s1).items()}]
        yhs = [yh, torch.empty_like(yh, pin_memory=True)]
        shs = [sh, torch.empty_like(sh, pin_memory=True)]
        s_in, s_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev)

        def e2e_pipe(K: int) -> float:
            barrier()
            E = lambda: torch.cuda.Event(enable_timing=True)  # noqa: E731
            e0 = E()
            e0.record(stream)
            s_in.wait_event(e0)
            s_out.wait_event(e0)
            done_c, done_o = [None] * K, [None] * K
            for k in range(K):
                b = sets[k & 1]
                with torch.cuda.stream(s_in):
                    if k >= 2:
                        s_in.wait_event(done_c[k - 2])  # set b's inputs consumed
                    for n in ("x", "dt", "A", "B", "C", "s0"):
                        b[n].copy_(host[n], non_blocking=True)
                    ev_in = E()
                    ev_in.record(s_in)
                stream.wait_event(ev_in)
                if k >= 2:
                    stream.wait_event(done_o[k - 2])  # set b's y, s1 read back
                st = ctx.encode(d, b["s0"], b["x"], b["dt"], b["A"], b["B"], b["C"], b["y"], b["s1"],
                                scratch=scratch, stream=stream)
                if st != abi.HELIX_OK:
                    raise SystemExit(f"encode failed: {ctx.last_error()}")
                done_c[k] = E()
                done_c[k].record(stream)
                with torch.cuda.stream(s_out):
                    s_out.wait_event(done_c[k])
                    yhs[k & 1].copy_(b["y"], non_blocking=True)
                    shs[k & 1].copy_(b["s1"], non_blocking=True)
                    done_o[k] = E()
                    done_o[k].record(s_out)
            stream.wait_event(done_o[K - 1])
            e1 = E()
            e1.record(stream)
            barrier()
            return e0.elapsed_time(e1) / K

        e2e_pipe(3)
        kp = max(6, a.steps // 4)
        ems = max_over_ranks(e2e_pipe(kp))
        e2e = {"value": job_tok / (ems * 1e-3), "unit": UNIT, "ms_per_step": ems,
               "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
               "mode": f"{kp} steps in flight on two buffer sets (upload, scan, read-back on separate streams)"
                       + ("; per rank, its own heads" if world > 1 else ""),
               "serial_ms_per_step": serial_ms}

    value = job_tok / (ms_per_step * 1e-3)
    if strong:
        layout = (f"the problem's {gshape.H} heads split over {world} ranks in whole groups "
                  f"({shape.H} heads per rank)")
    elif world > 1:
        layout = "per rank its own copy of the problem (weak scaling)"
    else:
        layout = "one GPU"
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": a.steps,
        "warmup": a.warmup, "ms_per_step": ms_per_step, "higher_is_better": True,
        "scaling": "strong" if strong or world == 1 else "weak",
        "vs_baseline": None, "dtype": "bf16" if a.compute == "bf16" else "f32",
        "data": "synthetic (seeded, BASELINE distributions; random A, B, C, x, dt)",
        "config": {"workload": f"{a.config}: S={gshape.S} L={gshape.L} H={gshape.H} P={gshape.P} "
                               f"N={gshape.N} G={gshape.G}, x/B/C {shape.io}, dt/A/s0/y/s1 f32, multipass; "
                               f"{layout}" + ("; diagonal A (one rate per (head, state))" if a.a_form == "diag" else ""),
                   "l2": "flushed before every timed step (256 MiB write, untimed)",
                   "compute": a.compute, "runs_plan_scratch_bytes": nbytes,
                   "backend": a.backend,
                   "plan": {"family": FAMILIES.get(info.family, str(info.family)),
                            "chunk": info.chunk, "run_tokens": info.run_tokens, "n_runs": info.n_runs,
                            "runs_per_span": info.runs_per_span, "n_spans": info.n_spans,
                            "state_runs": info.state_runs},
                   "tflops": tflops, "path_alg_bytes_per_rank": shape.alg_bytes(),
                   "path_gbs_per_rank": path_gbs, "path_hbm_frac": path_gbs / hbm,
                   "passes": passes},
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": hbm, "unit": "GB/s",
                     "frac": achieved / hbm, "traffic": traffic, "kernel": "output kernel",
                     "alg_bytes_per_launch": out_bytes, "peak_kind": peak_kind},
        "gpu_launches": launches * a.steps,
        "clocks": clk.summary(),
    }
    if e2e:
        line["e2e"] = e2e
    if rank == 0 and world == 1 and not a.no_cpu_baseline and a.a_form == "scalar":
        line["cpu_baseline"] = cpu_baseline(gshape, a.cpu_sample_tokens)
        line["cpu_baseline_chunked"] = cpu_baseline(gshape, a.cpu_sample_tokens, "chunked")
    if rank == 0:
        print(json.dumps(line), flush=True)
    ctx.close()
    if world > 1:
        dist.barrier(device_ids=[local])
        dist.destroy_process_group()
    return 0


def cast_launches(ctx, d) -> int:
    """Kernels the scan adds to cast F32-stored x, B, C to bf16 (the bf16
    family with F32 storage, and the fp32-class family, which always reads
    bf16 hi | lo pairs; none for the exact fp32 family)."""
    info = ctx.plan_info(d)
    from helix_b200 import abi
    return 1 if (info.family == 1 and d.io_dtype == abi.HELIX_F32) or info.family == 2 else 0


if __name__ == "__main__":
    sys.exit(main())
