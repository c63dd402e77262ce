"""GPU: BASELINE config 5 (S=8, L=131072, H=128, P=64, N=128, G=8, bf16
x/B/C) at one rank's shape of its head x token mesh, on one GPU.

On 8 GPUs config 5 runs as (head shards) x (token shards); a rank of the
4 x 2 or 2 x 4 mesh holds 32 or 64 heads of half or a quarter of the tokens.
Here one GPU takes 16 heads (one head group) of all eight 131072-token
sequences and runs the token split's steps for four token shards exactly as
the ranks of one token group would (helix_b200.dist.scan_lsplit without the
all-gather): shard states, carry combine, shard scans from the kept run
states.  The fp64 oracle costs about 8 s per (sequence, head) at this length,
so it runs on a fixed, seeded subset of (sequence, head) pairs, each checked
in full:
  * y of all 131072 tokens and s1, against helix::ref::scan's restatement;
  * the carry entering every token shard, against the state snapshots of
    helix::ref::scan_with_snapshots (reference src/reference/scan_ref.cpp:80-143)
    at the shard boundaries.
Bounds are the bf16 parity suite's (y: the reference's calibrated bf16
per-element bound and 2e-2 relative L2; states: the carried-state bound)."""
import os
from concurrent.futures import ThreadPoolExecutor

import numpy as np
import pytest

from gpu_harness import BF16_ABS, BF16_REL, BF16_RL2, record
from helpers import compare

pytestmark = pytest.mark.gpu

S1_REL, S1_ABS, S1_RL2 = 2e-5, 2e-6, 1e-4
PAIRS = [(0, 0), (3, 7), (5, 12), (7, 15)]  # (sequence, head), fixed
K = 4  # token shards


def _check(tag, got, want, rel, abs_, rl2):
    c = compare(got, want, rel, abs_)
    record(tag, ratio=c["ratio"], rel_l2=c["rel_l2"])
    assert c["ok"] and c["rel_l2"] <= rl2, (tag, c)


def test_c5_rank_shape_token_split(ctx, oracle):
    import torch

    import helix_b200
    from helix_b200.synth import Shape, make_inputs

    g = Shape.of("c5")
    hpg = g.H // g.G
    sh = Shape(g.S, g.L, hpg, g.P, g.N, 1, g.io)  # one head group of the mesh
    dev = torch.device("cuda:0")
    t = make_inputs(sh, seed=5005, device=dev, s0_std=0.1)
    L, Ls = sh.L, sh.L // K
    sl = lambda k, a, b: t[k][:, a:b].contiguous()  # noqa: E731
    kept = [helix_b200.shard_state(sl("x", a, a + Ls), sl("dt", a, a + Ls), t["A"], sl("B", a, a + Ls),
                                   sl("C", a, a + Ls), ctx=ctx, keep_scratch=True) for a in range(0, L, Ls)]
    states = torch.stack([k[0] for k in kept]).contiguous()
    lds = torch.stack([k[1] for k in kept]).contiguous()
    carries, ys, s1 = [], [], None
    for k in range(K):
        carry = helix_b200.carry_combine(t["s0"], states[:k].contiguous(), lds[:k].contiguous(), ctx=ctx)
        a = k * Ls
        y, s1 = helix_b200.scan_shard(sl("x", a, a + Ls), sl("dt", a, a + Ls), t["A"], sl("B", a, a + Ls),
                                      sl("C", a, a + Ls), carry, kept[k][2], ctx=ctx)
        carries.append(carry)
        ys.append(y)
    torch.cuda.synchronize()
    assert bool(torch.isfinite(s1).all())

    # the oracle's one-(sequence, head) problems on the values the kernels saw
    def f32(v):
        return v.detach().float().cpu().numpy()

    jobs = []
    for seq, h in PAIRS:
        prob = dict(s0=f32(t["s0"][seq:seq + 1, h:h + 1]), x=f32(t["x"][seq:seq + 1, :, h:h + 1]),
                    dt=f32(t["dt"][seq:seq + 1, :, h:h + 1]), A=f32(t["A"][h:h + 1]),
                    B=f32(t["B"][seq:seq + 1]), C=f32(t["C"][seq:seq + 1]))
        got = dict(y=np.concatenate([f32(y[seq, :, h]) for y in ys]), s1=f32(s1[seq, h]),
                   carries=[f32(c[seq, h]) for c in carries])
        jobs.append((seq, h, prob, got))

    def oracle_run(job):
        seq, h, prob, _ = job
        d = oracle.desc_init(L, 1, 1, sh.P, sh.N, 1)
        y, s_1, snap = oracle.scan_with_snapshots(d, *[prob[k] for k in ("s0", "x", "dt", "A", "B", "C")], Ls)
        return y, s_1, snap

    with ThreadPoolExecutor(max_workers=min(len(jobs), os.cpu_count() or 1)) as ex:
        refs = list(ex.map(oracle_run, jobs))
    for (seq, h, prob, got), (y_ref, s_ref, snap) in zip(jobs, refs):
        tag = f"c5 seq {seq} head {h}"
        _check(tag + " y", got["y"], y_ref[0, :, 0], BF16_REL, BF16_ABS, BF16_RL2)
        _check(tag + " s1", got["s1"], s_ref[0, 0], S1_REL, S1_ABS, S1_RL2)
        for k in range(1, K):  # the carry entering shard k = the state after token k * Ls
            want = snap[k - 1].reshape(sh.P, sh.N)
            _check(tag + f" carry into shard {k}", got["carries"][k], want, S1_REL, S1_ABS, S1_RL2)
