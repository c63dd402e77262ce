"""GPU: the token-split (L-split) entry points and their composition.

* helix_scan_shard_state against the oracle's state after the shard from a
  zero start (the oracle's s1) and the numpy log-decay, on both precision
  paths, with one run and with many runs;
* helix_scan_carry_combine against a numpy fold, with and without ids;
* the whole L-split emulated on one GPU (shards run one after another, the
  gathered pairs kept in device memory): the concatenated y and the last
  shard's s1 against the oracle's full-length scan;
* with two or more visible GPUs, the real thing: two ranks over NCCL.

Bounds: the same per-element and relative-L2 bounds as the single-GPU parity
tests of each path (gpu_harness), the state held to the state bounds."""
import os
import socket

import numpy as np
import pytest

from gpu_harness import (BF16_ABS, BF16_REL, BF16_RL2, F32_ABS, F32_REL, F32_RL2, X3_ABS, X3_REL, X3_RL2, record,
                         widen)
from helpers import compare
from helix_b200 import abi

pytestmark = pytest.mark.gpu

# "io" cases: F32-stored inputs on the fp32-class tensor-core family (the
# default for compute F32), on the exact CUDA-core family (backend REF), and
# bf16-stored inputs on the bf16 family.  State bounds: the fp32 parity
# suites'; the bf16 parity tests' carried-state bound (hi/lo split update).
ST_BOUNDS = {"f32": (X3_REL, X3_ABS, X3_RL2), "f32-exact": (F32_REL, F32_ABS, F32_RL2), "bf16": (2e-5, 2e-6, 1e-4)}
Y_BOUNDS = {"f32": (X3_REL, X3_ABS, X3_RL2), "f32-exact": (F32_REL, F32_ABS, F32_RL2),
            "bf16": (BF16_REL, BF16_ABS, BF16_RL2)}
BACKEND = {"f32": abi.HELIX_BACKEND_AUTO, "f32-exact": abi.HELIX_BACKEND_REF, "bf16": abi.HELIX_BACKEND_AUTO}
IOS = ["f32", "f32-exact", "bf16"]


def _torch(prob, io, dev="cuda:0"):
    import torch
    t = {k: torch.from_numpy(np.ascontiguousarray(prob[k])).to(dev) for k in ("s0", "x", "dt", "A", "B", "C")}
    if io == "bf16":
        for k in ("x", "B", "C"):
            t[k] = t[k].to(torch.bfloat16)
    return t


def _log_decay(prob, d):
    raw = prob["dt"].astype(np.float64)
    v = np.clip(np.where(raw > 20.0, raw, np.log1p(np.exp(raw))), d.dt_min, d.dt_max)
    return (v * prob["A"].astype(np.float64)[None, None, :]).sum(axis=1)


def _check(tag, got, want, bounds):
    rel, ab, rl2 = bounds
    c = compare(got, want, rel, ab)
    record(tag, ratio=c["ratio"], rel_l2=c["rel_l2"])
    assert c["ok"] and c["rel_l2"] <= rl2, (tag, c)


@pytest.fixture
def run_tokens():
    old = os.environ.get("HELIX_RUN_TOKENS")

    def set_(v):
        if v is None:
            os.environ.pop("HELIX_RUN_TOKENS", None)
        else:
            os.environ["HELIX_RUN_TOKENS"] = v
    yield set_
    set_(old)


SHAPES = [(300, 2, 4, 64, 128, 2), (1024, 1, 8, 64, 128, 8), (129, 3, 2, 72, 128, 1)]


@pytest.mark.parametrize("runs", [None, "128"], ids=["auto-runs", "runs128"])
@pytest.mark.parametrize("io", IOS)
@pytest.mark.parametrize("shape", SHAPES, ids=["L{}S{}H{}P{}N{}G{}".format(*s) for s in SHAPES])
@pytest.mark.parametrize("long_mem", [False, True], ids=["short", "long"])
def test_shard_state(ctx, oracle, run_tokens, shape, io, runs, long_mem):
    import helix_b200
    import torch
    L, S, H, P, N, G = shape
    prob = widen(oracle.harness_problem(*shape, 31, long_mem), io)
    d = oracle.desc_init(*shape)
    _, s_ref = oracle.scan(d, np.zeros_like(prob["s0"]), prob["x"], prob["dt"], prob["A"], prob["B"], prob["C"])
    t = _torch(prob, io)
    run_tokens(runs)
    state, ld = helix_b200.shard_state(t["x"], t["dt"], t["A"], t["B"], t["C"], ctx=ctx, backend=BACKEND[io])
    torch.cuda.synchronize()
    _check(f"shard_state {io} {shape}", state.cpu().numpy(), s_ref, ST_BOUNDS[io])
    np.testing.assert_allclose(ld.cpu().numpy(), _log_decay(prob, d), rtol=2e-5, atol=1e-4)


@pytest.mark.parametrize("n_prev", [0, 1, 3])
@pytest.mark.parametrize("with_ids", [False, True])
def test_carry_combine(ctx, n_prev, with_ids):
    import helix_b200
    import torch
    rng = np.random.default_rng(7 + n_prev)
    S, H, P, N = 3, 4, 72, 128
    s0 = rng.normal(0, 1, (S + 1, H, P, N)).astype(np.float32)
    states = rng.normal(0, 1, (n_prev, S, H, P, N)).astype(np.float32)
    lds = rng.uniform(-30, 0, (n_prev, S, H)).astype(np.float32)
    ids = np.array([3, 0, 2], np.int32) if with_ids else None
    rows = ids if with_ids else np.arange(S)
    want = s0[rows].astype(np.float64)
    for j in range(n_prev):
        want = np.exp(lds[j].astype(np.float64))[:, :, None, None] * want + states[j]
    dev = "cuda:0"
    s0_t = torch.from_numpy(s0 if with_ids else s0[:S].copy()).to(dev)
    got = helix_b200.carry_combine(s0_t, torch.from_numpy(states).to(dev), torch.from_numpy(lds).to(dev),
                                   None if ids is None else torch.from_numpy(ids).to(dev), ctx=ctx)
    torch.cuda.synchronize()
    np.testing.assert_allclose(got.cpu().numpy(), want, rtol=1e-5, atol=1e-5)


@pytest.mark.parametrize("via", ["scan", "scan_shard"])
@pytest.mark.parametrize("io", IOS)
@pytest.mark.parametrize("cuts", [(0, 512, 1024), (0, 100, 613, 640, 1024)], ids=["2shards", "4shards-ragged"])
def test_lsplit_emulated_on_one_gpu(ctx, oracle, run_tokens, io, cuts, via):
    """K token shards of one problem on one GPU: shard states, carry
    combine, shard scans -- through helix_scan_encode with the carry as s0,
    or through helix_scan_encode_shard on the shard-state scratch (no second
    state pass)."""
    import helix_b200
    import torch
    shape = (1024, 2, 4, 64, 128, 2)
    L, S, H, P, N, G = shape
    prob = widen(oracle.harness_problem(*shape, 17, True), io)
    prob["s0"] = np.random.default_rng(3).normal(0, 0.2, prob["s0"].shape).astype(np.float32)
    d = oracle.desc_init(*shape)
    y_ref, s_ref = oracle.scan(d, prob["s0"], prob["x"], prob["dt"], prob["A"], prob["B"], prob["C"])
    t = _torch(prob, io)
    shards = [(a, b) for a, b in zip(cuts[:-1], cuts[1:])]
    sl = lambda k, a, b: t[k][:, a:b].contiguous()
    run_tokens("128")  # several runs per shard: the run states carry
    be = BACKEND[io]
    pairs = [helix_b200.shard_state(sl("x", a, b), sl("dt", a, b), t["A"], sl("B", a, b), sl("C", a, b), ctx=ctx,
                                    keep_scratch=True, backend=be)
             for a, b in shards]
    states = torch.stack([p[0] for p in pairs]).contiguous()
    lds = torch.stack([p[1] for p in pairs]).contiguous()
    ys, s_last = [], None
    for k, (a, b) in enumerate(shards):
        carry = helix_b200.carry_combine(t["s0"], states[:k].contiguous(), lds[:k].contiguous(), ctx=ctx)
        if via == "scan":
            y, s_last = helix_b200.scan(sl("x", a, b), sl("dt", a, b), t["A"], sl("B", a, b), sl("C", a, b),
                                        carry, ctx=ctx, backend=be)
        else:
            y, s_last = helix_b200.scan_shard(sl("x", a, b), sl("dt", a, b), t["A"], sl("B", a, b),
                                              sl("C", a, b), carry, pairs[k][2], ctx=ctx, backend=be)
        ys.append(y)
    torch.cuda.synchronize()
    y = torch.cat(ys, dim=1).cpu().numpy()
    _check(f"lsplit y {io} {cuts} {via}", y, y_ref, Y_BOUNDS[io])
    _check(f"lsplit s1 {io} {cuts} {via}", s_last.cpu().numpy(), s_ref, ST_BOUNDS[io])


def _nccl_worker(rank, world, port, out_dir):
    import datetime
    import torch
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        from oracle.oracle import Oracle
        from helix_b200 import dist as hdist
        o = Oracle()
        shape = (1024, 2, 4, 64, 128, 2)
        prob = widen(o.harness_problem(*shape, 23, True), "bf16")
        prob["s0"] = np.random.default_rng(4).normal(0, 0.2, prob["s0"].shape).astype(np.float32)
        t = _torch(prob, "bf16", dev=f"cuda:{rank}")
        cut = [0, 384, 1024][: world + 1] if world == 2 else list(np.linspace(0, 1024, world + 1).astype(int))
        a, b = cut[rank], cut[rank + 1]
        sl = lambda k: t[k][:, a:b].contiguous()
        y, s1 = hdist.scan_lsplit(sl("x"), sl("dt"), t["A"], sl("B"), sl("C"), t["s0"])
        torch.cuda.synchronize()
        np.save(os.path.join(out_dir, f"y{rank}.npy"), y.cpu().numpy())
        np.save(os.path.join(out_dir, f"s{rank}.npy"), s1.cpu().numpy())
        np.save(os.path.join(out_dir, f"cut.npy"), np.array(cut))
    finally:
        dist.destroy_process_group()


def test_lsplit_two_ranks_nccl(oracle, tmp_path):
    import torch
    import torch.multiprocessing as mp
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    world = 2
    mp.start_processes(_nccl_worker, args=(world, port, str(tmp_path)), nprocs=world, join=True,
                       start_method="spawn")
    shape = (1024, 2, 4, 64, 128, 2)
    prob = widen(oracle.harness_problem(*shape, 23, True), "bf16")
    prob["s0"] = np.random.default_rng(4).normal(0, 0.2, prob["s0"].shape).astype(np.float32)
    d = oracle.desc_init(*shape)
    y_ref, s_ref = oracle.scan(d, prob["s0"], prob["x"], prob["dt"], prob["A"], prob["B"], prob["C"])
    y = np.concatenate([np.load(tmp_path / f"y{r}.npy") for r in range(world)], axis=1)
    _check("lsplit nccl y", y, y_ref, Y_BOUNDS["bf16"])
    _check("lsplit nccl s1", np.load(tmp_path / f"s{world - 1}.npy"), s_ref, ST_BOUNDS["bf16"])


def test_shard_state_rejects_small_scratch(ctx):
    """A scratch allocation smaller than helix_scan_shard_state_scratch_size()
    is rejected (the driver knows the allocation's size) and nothing runs."""
    import ctypes as C

    import helix_b200
    import torch
    dev = torch.device("cuda:0")
    S, L, H, P, N, G = 1, 1024, 4, 64, 128, 1
    x = torch.randn(S, L, H, P, device=dev)
    dt = torch.randn(S, L, H, device=dev) - 4
    A = -torch.rand(H, device=dev) - 1
    Bm = torch.randn(S, L, G, N, device=dev) / 11
    Cm = torch.randn(S, L, G, N, device=dev) / 11
    state = torch.full((S, H, P, N), float("nan"), device=dev)
    ld = torch.full((S, H), float("nan"), device=dev)
    d = helix_b200.desc_from_tensors(x, dt, Bm, state, multipass=True)
    need = ctx.shard_state_scratch_size(d)
    assert need > 4096
    rt = C.CDLL("libcudart.so.12")
    ptr = C.c_void_p()
    assert rt.cudaMalloc(C.byref(ptr), C.c_size_t(need - 4096)) == 0
    try:
        T = helix_b200._t
        st = ctx.lib.helix_scan_shard_state(ctx.handle, None, C.byref(d), T(x), T(dt), T(A), T(Bm), T(Cm),
                                            T(state), T(ld), abi.Tensor(ptr, 0))
        assert st == abi.HELIX_ERR_SCRATCH_TOO_SMALL
        assert "scratch" in ctx.last_error()
    finally:
        torch.cuda.synchronize()
        rt.cudaFree(ptr)
    assert bool(torch.isnan(state).all()) and bool(torch.isnan(ld).all())
