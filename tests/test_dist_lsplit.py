"""CPU: the token-split (L-split) host logic of helix_b200.dist over gloo.

Each spawned rank holds a token shard of the reference harness problem and
runs scan_lsplit with compute steps done by the oracle (the CPU restatement),
so the test checks the collective part -- gather order, exclusive fold,
carry into the shard's scan -- against the oracle's own full-length scan.
Uneven shard lengths, world sizes 2 and 3, and ids-selected initial states
are covered."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from helix_b200 import dist as hdist

SHAPE = (301, 3, 4, 8, 16, 2)  # L, S, H, P, N, G


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


class OracleOps:
    """The three compute steps on CPU tensors, by the fp64 oracle."""

    def __init__(self, oracle, dims):
        self.o, self.dims = oracle, dims

    def _desc(self, L):
        _, S, H, P, N, G = self.dims
        return self.o.desc_init(L, S, H, P, N, G)

    def shard_state(self, x, dt, A, B, Cm):
        L = x.shape[1]
        _, S, H, P, N, G = self.dims
        d = self._desc(L)
        zero = np.zeros((S, H, P, N), np.float32)
        _, s1 = self.o.scan(d, zero, x.numpy(), dt.numpy(), A.numpy(), B.numpy(), Cm.numpy())
        raw = dt.numpy().astype(np.float64)
        v = np.where(raw > 20.0, raw, np.log1p(np.exp(raw)))
        v = np.clip(v, d.dt_min, d.dt_max)
        ld = (v * A.numpy().astype(np.float64)[None, None, :]).sum(axis=1)
        return torch.from_numpy(s1), torch.from_numpy(ld.astype(np.float32))

    def carry_combine(self, s0, states, log_decays, ids):
        S = states.shape[1] if states.shape[0] else (len(ids) if ids is not None else s0.shape[0])
        rows = ids.numpy() if ids is not None else np.arange(S)
        carry = s0.numpy()[rows].astype(np.float64)
        for j in range(states.shape[0]):
            carry = np.exp(log_decays[j].numpy().astype(np.float64))[:, :, None, None] * carry + \
                states[j].numpy()
        return torch.from_numpy(carry.astype(np.float32))

    def scan(self, x, dt, A, B, Cm, s0):
        d = self._desc(x.shape[1])
        y, s1 = self.o.scan(d, s0.numpy(), x.numpy(), dt.numpy(), A.numpy(), B.numpy(), Cm.numpy())
        return torch.from_numpy(y), torch.from_numpy(s1)


def _worker(rank, world, port, cuts, use_ids, out_dir):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import datetime
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        from oracle.oracle import Oracle
        o = Oracle()
        L, S, H, P, N, G = SHAPE
        prob = o.harness_problem(L, S, H, P, N, G, 99, True)
        s0 = np.ascontiguousarray(np.random.default_rng(5).normal(0, 0.3, prob["s0"].shape).astype(np.float32))
        ids = np.array([2, 0, 1], np.int32) if use_ids else None
        l0, l1 = cuts[rank], cuts[rank + 1]
        sl = lambda a: torch.from_numpy(np.ascontiguousarray(a[:, l0:l1]))
        y, s1 = hdist.scan_lsplit(sl(prob["x"]), sl(prob["dt"]), torch.from_numpy(prob["A"]), sl(prob["B"]),
                                  sl(prob["C"]), torch.from_numpy(s0),
                                  None if ids is None else torch.from_numpy(ids),
                                  ops=OracleOps(o, SHAPE))
        np.save(os.path.join(out_dir, f"y{rank}.npy"), y.numpy())
        np.save(os.path.join(out_dir, f"s{rank}.npy"), s1.numpy())
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("cuts,use_ids", [
    ((0, 150, 301), False),
    ((0, 1, 200, 301), False),
    ((0, 128, 129, 301), True),
], ids=["2ranks", "3ranks-tiny-first", "3ranks-ids"])
def test_lsplit_matches_full_scan(oracle, tmp_path, cuts, use_ids):
    world = len(cuts) - 1
    mp.start_processes(_worker, args=(world, _free_port(), cuts, use_ids, str(tmp_path)), nprocs=world,
                       join=True, start_method="spawn")
    L, S, H, P, N, G = SHAPE
    prob = oracle.harness_problem(L, S, H, P, N, G, 99, True)
    s0 = np.random.default_rng(5).normal(0, 0.3, prob["s0"].shape).astype(np.float32)
    ids = np.array([2, 0, 1], np.int32) if use_ids else None
    d = oracle.desc_init(L, S, H, P, N, G)
    y_ref, s_ref = oracle.scan(d, s0, prob["x"], prob["dt"], prob["A"], prob["B"], prob["C"], ids=ids)
    y = np.concatenate([np.load(tmp_path / f"y{r}.npy") for r in range(world)], axis=1)
    s_last = np.load(tmp_path / f"s{world - 1}.npy")
    np.testing.assert_allclose(y, y_ref, rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(s_last, s_ref, rtol=1e-5, atol=1e-6)
    # every rank's s1 is the state at the end of its own shard
    for r in range(world - 1):
        d_r = oracle.desc_init(cuts[r + 1], S, H, P, N, G)
        _, s_mid = oracle.scan(d_r, s0, prob["x"][:, :cuts[r + 1]].copy(), prob["dt"][:, :cuts[r + 1]].copy(),
                               prob["A"], prob["B"][:, :cuts[r + 1]].copy(), prob["C"][:, :cuts[r + 1]].copy(),
                               ids=ids)
        np.testing.assert_allclose(np.load(tmp_path / f"s{r}.npy"), s_mid, rtol=1e-5, atol=1e-6)


def test_head_slice_deals_whole_groups():
    assert hdist.head_slice(64, 8, 0, 8) == (0, 8)
    assert hdist.head_slice(64, 8, 3, 4) == (48, 64)
    assert hdist.head_slice(128, 8, 1, 2) == (64, 128)
    with pytest.raises(ValueError):
        hdist.head_slice(64, 8, 0, 3)
