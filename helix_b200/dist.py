"""helix_b200.dist -- the scan on several GPUs, one process per GPU.

Two layouts, combinable as a (head shards x token shards) mesh:

* Head sharding.  Each rank owns a contiguous range of whole head groups
  (x, dt, y and the states sliced on the head axis, B and C on the group
  axis).  Heads never interact, so every rank runs the ordinary scan on its
  slice and no collective is needed.  ``head_slice`` gives the range.

* Token sharding ("L-split").  The ranks of one ``group`` hold consecutive
  token ranges [l_k, l_{k+1}) of the same heads.  ``scan_lsplit`` runs, on
  every rank of the group:
    1. the shard's zero-start final state and log-decay
       (``helix_scan_shard_state``),
    2. an all-gather of those (state, log_decay) pairs over the group,
    3. the fold of ranks 0..k-1 onto the sequence's initial state, i.e. the
       exclusive scan of (a1, b1) o (a2, b2) = (a1 a2, a2 b1 + b2)
       (``helix_scan_carry_combine``),
    4. the scan of the shard with that carry as s0, reusing the run states
       of step 1 (``helix_scan_encode_shard``; no second state pass).
  The last rank's s1 is every sequence's final state.  The exchange is
  S * H * P * N * 4 bytes per rank (8.4 MB for 8 sequences of 32 heads of
  64 x 128) plus S * H log-decays, over NCCL; it lands in ordinary device
  memory (no peer-memory operands, no cluster-wide copies).

The compute steps go through ``ops`` (``GpuOps`` by default: the C ABI via
``helix_b200``); tests substitute CPU implementations to exercise the
collective logic with the gloo backend.
"""
from __future__ import annotations

from typing import Optional

__all__ = ["GpuOps", "head_slice", "scan_lsplit", "exclusive_carry"]


def head_slice(n_head: int, n_group: int, rank: int, world: int) -> tuple[int, int]:
    """Contiguous head range [h0, h1) of `rank` when heads are dealt out in
    whole groups (a group's heads share B and C).  Requires the group count to
    be a multiple of `world`."""
    if n_group % world:
        raise ValueError(f"{n_group} groups do not split over {world} ranks")
    hpg = n_head // n_group
    gpr = n_group // world
    return rank * gpr * hpg, (rank + 1) * gpr * hpg


class GpuOps:
    """The three compute steps through libhelix on the tensors' device."""

    def __init__(self, compute: str = "auto", multipass: bool = True, ctx=None, stream=None):
        self.compute, self.multipass, self.ctx, self.stream = compute, multipass, ctx, stream

    def shard_state(self, x, dt, A, B, Cm):
        import helix_b200
        return helix_b200.shard_state(x, dt, A, B, Cm, compute=self.compute, ctx=self.ctx, stream=self.stream)

    def shard_state_keep(self, x, dt, A, B, Cm):
        """shard_state plus the scratch holding its run states."""
        import helix_b200
        return helix_b200.shard_state(x, dt, A, B, Cm, compute=self.compute, ctx=self.ctx, stream=self.stream,
                                      keep_scratch=True)

    def scan_shard(self, x, dt, A, B, Cm, carry, keep):
        """The shard's scan from carry, without a second state pass."""
        import helix_b200
        return helix_b200.scan_shard(x, dt, A, B, Cm, carry, keep, compute=self.compute, ctx=self.ctx,
                                     stream=self.stream)

    def carry_combine(self, s0, states, log_decays, ids):
        import helix_b200
        return helix_b200.carry_combine(s0, states, log_decays, ids, ctx=self.ctx, stream=self.stream)

    def scan(self, x, dt, A, B, Cm, s0):
        import helix_b200
        return helix_b200.scan(x, dt, A, B, Cm, s0, multipass=self.multipass, compute=self.compute,
                               ctx=self.ctx, stream=self.stream)


def exclusive_carry(ops, s0, states: list, log_decays: list, rank: int, ids=None):
    """Carry entering shard `rank`, from the gathered per-shard pairs."""
    import torch
    if rank == 0:
        prev_s = states[0].new_empty((0,) + tuple(states[0].shape))
        prev_d = log_decays[0].new_empty((0,) + tuple(log_decays[0].shape))
    else:
        prev_s = torch.stack(states[:rank]).contiguous()
        prev_d = torch.stack(log_decays[:rank]).contiguous()
    return ops.carry_combine(s0, prev_s, prev_d, ids)


def scan_lsplit(x, dt, A, B, Cm, s0, ids=None, *, group=None, ops: Optional[object] = None):
    """Scan of this rank's token shard of every sequence, with the state
    carried in from the shards of lower-ranked members of `group`.

    x (S, L_k, H, P), dt (S, L_k, H), B and Cm (S, L_k, G, N) hold tokens
    [l_k, l_{k+1}); A (H,); s0 (S0, H, P, N) the sequences' initial state
    (rows picked by ids, if given).  Every rank of `group` must call this with
    the same S, H, P, N, G.  Returns (y of the shard, state after the shard);
    on the last rank the latter is the final state.  Collective: every rank
    takes the same two all-gathers in the same order."""
    import torch.distributed as dist
    ops = ops or GpuOps()
    rank = dist.get_rank(group)
    world = dist.get_world_size(group)
    # ops that can keep the shard's run states (GpuOps, multipass) scan the
    # shard from them afterwards, so the state pass runs once per shard
    keep = None
    if hasattr(ops, "shard_state_keep") and getattr(ops, "multipass", True):
        state, log_decay, keep = ops.shard_state_keep(x, dt, A, B, Cm)
    else:
        state, log_decay = ops.shard_state(x, dt, A, B, Cm)
    states = [state.new_empty(state.shape) for _ in range(world)]
    decays = [log_decay.new_empty(log_decay.shape) for _ in range(world)]
    dist.all_gather(states, state.contiguous(), group=group)
    dist.all_gather(decays, log_decay.contiguous(), group=group)
    carry = exclusive_carry(ops, s0, states, decays, rank, ids)
    if keep is not None:
        return ops.scan_shard(x, dt, A, B, Cm, carry, keep)
    return ops.scan(x, dt, A, B, Cm, carry)
