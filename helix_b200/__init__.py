"""helix_b200 -- B200-native (sm_100a) Mamba-2 SSD prefill scan behind the
HELIX C ABI.

The product is ``libhelix.so`` (C ABI in include/helix/helix.h).  This module
is a thin host-side convenience over it for PyTorch users: it maps torch
tensors (device memory) and the current CUDA stream onto the ABI's
``helix_tensor`` / ``cudaStream_t`` arguments.  There is no Python compute
path: every call goes through the library, and a missing library raises.
"""
from __future__ import annotations

import ctypes as C
from typing import Optional

from . import abi

__all__ = ["HelixError", "Context", "desc_from_tensors", "scan", "shard_state", "scan_shard", "carry_combine",
           "abi"]


class HelixError(RuntimeError):
    def __init__(self, status: int, msg: str):
        super().__init__(f"helix status {abi.STATUS_NAMES.get(status, status)}: {msg}")
        self.status = status


def _t(x) -> abi.Tensor:
    """torch tensor (or None) -> helix_tensor."""
    if x is None:
        return abi.NULL_TENSOR
    return abi.Tensor(C.c_void_p(x.data_ptr()), 0)


class Context:
    """Owns one helix_ctx bound to a CUDA device."""

    def __init__(self, device: Optional[int] = None):
        self.lib = abi.load()
        h = C.c_void_p()
        dev = C.c_int(device) if device is not None else None
        st = self.lib.helix_ctx_create(C.byref(h), C.byref(dev) if dev is not None else None, None)
        if st != abi.HELIX_OK:
            raise HelixError(st, self.lib.helix_ctx_last_error(None).decode())
        self.handle = h

    def close(self) -> None:
        if getattr(self, "handle", None):
            self.lib.helix_ctx_free(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def last_error(self) -> str:
        return self.lib.helix_ctx_last_error(self.handle).decode()

    def supported(self, d: abi.ScanDesc) -> bool:
        return bool(self.lib.helix_scan_supported(self.handle, C.byref(d)))

    def scratch_size(self, d: abi.ScanDesc) -> int:
        return int(self.lib.helix_scan_scratch_size(self.handle, C.byref(d)))

    def select_backend(self, d: abi.ScanDesc) -> int:
        return int(self.lib.helix_ctx_select_backend(self.handle, C.byref(d)))

    def backend_desc(self, d: abi.ScanDesc) -> str:
        return self.lib.helix_ctx_backend_desc(self.handle, C.byref(d)).decode()

    def _stream(self, stream, *tensors):
        if stream is None:
            import torch
            dev = next((t.device for t in tensors if t is not None), None)
            stream = torch.cuda.current_stream(dev)
        return C.c_void_p(getattr(stream, "cuda_stream", stream))

    def plan_info(self, d: abi.ScanDesc) -> abi.PlanInfo:
        out = abi.PlanInfo()
        st = int(self.lib.helix_scan_plan_info(self.handle, C.byref(d), C.byref(out)))
        if st != abi.HELIX_OK:
            raise HelixError(st, self.last_error())
        return out

    def shard_state_scratch_size(self, d: abi.ScanDesc) -> int:
        return int(self.lib.helix_scan_shard_state_scratch_size(self.handle, C.byref(d)))

    def encode_shard_state(self, d: abi.ScanDesc, x, dt, A, B, Cm, state, log_decay, scratch,
                           stream=None) -> int:
        return int(self.lib.helix_scan_shard_state(
            self.handle, self._stream(stream, x, state), C.byref(d), _t(x), _t(dt), _t(A), _t(B),
            _t(Cm), _t(state), _t(log_decay), _t(scratch)))

    def encode_shard(self, d: abi.ScanDesc, carry, x, dt, A, B, Cm, y, s1, scratch, stream=None) -> int:
        return int(self.lib.helix_scan_encode_shard(
            self.handle, self._stream(stream, x, y), C.byref(d), _t(carry), _t(x), _t(dt), _t(A), _t(B),
            _t(Cm), _t(y), _t(s1), _t(scratch)))

    def encode_carry_combine(self, d: abi.ScanDesc, s0, states, log_decays, n_prev: int, carry,
                             ids=None, stream=None) -> int:
        return int(self.lib.helix_scan_carry_combine(
            self.handle, self._stream(stream, s0, carry), C.byref(d), _t(s0), _t(ids), _t(states),
            _t(log_decays), C.c_uint32(n_prev), _t(carry)))

    def encode(self, d: abi.ScanDesc, s0, x, dt, A, B, Cm, y, s1, ids=None, scratch=None,
               stream=None, into: bool = False) -> int:
        """Enqueues one scan on `stream` (a torch.cuda.Stream, a raw handle, or
        None for torch's current stream).  Returns the helix_status."""
        if stream is None:
            import torch
            dev = next((t.device for t in (x, y, s0) if t is not None), None)
            stream = torch.cuda.current_stream(dev)
        handle = getattr(stream, "cuda_stream", stream)
        fn = self.lib.helix_scan_encode_into if into else self.lib.helix_scan_encode
        return int(fn(self.handle, C.c_void_p(handle), C.byref(d), _t(s0), _t(x), _t(dt), _t(A),
                      _t(B), _t(Cm), _t(ids), _t(y), _t(s1), _t(scratch)))


def desc_from_tensors(x, dt, B, s0, y=None, *, multipass: bool = True, compute: str = "auto",
                      backend: int = abi.HELIX_BACKEND_AUTO, A=None) -> abi.ScanDesc:
    """Descriptor for torch tensors laid out as in helix.h:
    x (S, L, H, P), dt (S, L, H), B and C (S, L, G, N), s0 (S, H, P, N),
    y (S, L, H, P).  Strides are taken from the tensors, so views work.
    A, if given, sets the decay form: (H,) scalar per head, (H, N) one rate
    per (head, state) (HELIX_A_DIAG_PER_CHANNEL, rows A.stride(0) apart)."""
    import torch
    S, L, H, P = x.shape
    G, N = B.shape[2], B.shape[3]
    d = abi.desc_init(L, S, H, P, N, G)
    d.s_x[:] = list(x.stride()[1:]); d.seq_x = x.stride(0)
    d.s_b[:] = list(B.stride()[1:]); d.seq_b = B.stride(0)
    d.s_c[:] = list(B.stride()[1:]); d.seq_c = B.stride(0)
    d.s_dt[:] = list(dt.stride()[1:]); d.seq_dt = dt.stride(0)
    d.s_s[:] = list(s0.stride()[1:]); d.seq_s = s0.stride(0)
    if y is not None:
        d.s_y[:] = list(y.stride()[1:]); d.seq_y = y.stride(0)
    d.io_dtype = abi.HELIX_BF16 if x.dtype == torch.bfloat16 else abi.HELIX_F32
    if compute == "auto":
        compute = "bf16" if x.dtype == torch.bfloat16 else "f32"
    d.compute_dtype = abi.HELIX_BF16 if compute == "bf16" else abi.HELIX_F32
    d.backend = backend
    d.multipass = multipass
    if A is not None:
        if A.dim() == 2:
            if A.stride(1) != 1:
                raise ValueError("a per-state A needs unit stride along d_state")
            d.a_form = abi.HELIX_A_DIAG_PER_CHANNEL
            d.s_a = A.stride(0)
        else:
            d.s_a = A.stride(0)
    return d


_default_ctx: dict[int, Context] = {}


def scan(x, dt, A, B, Cm, s0, ids=None, *, multipass: bool = True, compute: str = "auto",
         backend: int = abi.HELIX_BACKEND_AUTO, ctx: Optional[Context] = None, stream=None):
    """Runs the scan on torch CUDA tensors and returns (y, s1).

    Allocates y, s1 and the scratch with torch (this convenience wrapper is
    the only place that allocates; the library itself never does)."""
    import torch
    dev = x.device.index if x.device.index is not None else torch.cuda.current_device()
    if ctx is None:
        ctx = _default_ctx.get(dev) or _default_ctx.setdefault(dev, Context(dev))
    y = torch.empty(x.shape, dtype=torch.float32, device=x.device)
    s1 = torch.empty(s0.shape, dtype=torch.float32, device=x.device)
    d = desc_from_tensors(x, dt, B, s0, y, multipass=multipass, compute=compute, backend=backend, A=A)
    if Cm.stride() != B.stride():
        d.s_c[:] = list(Cm.stride()[1:]); d.seq_c = Cm.stride(0)
    nbytes = ctx.scratch_size(d)
    scratch = torch.empty(max(nbytes, 1), dtype=torch.uint8, device=x.device) if nbytes else None
    st = ctx.encode(d, s0, x, dt, A, B, Cm, y, s1, ids=ids, scratch=scratch, stream=stream)
    if scratch is not None and stream is not None and hasattr(stream, "cuda_stream"):
        scratch.record_stream(stream)
    if st != abi.HELIX_OK:
        raise HelixError(st, ctx.last_error())
    return y, s1


def _ctx_for(x, ctx):
    import torch
    dev = x.device.index if x.device.index is not None else torch.cuda.current_device()
    if ctx is None:
        ctx = _default_ctx.get(dev) or _default_ctx.setdefault(dev, Context(dev))
    return ctx


def shard_state(x, dt, A, B, Cm, *, compute: str = "auto", backend: int = abi.HELIX_BACKEND_AUTO,
                ctx: Optional[Context] = None, stream=None, keep_scratch: bool = False):
    """State this token shard leaves from a zero start, and its log-decay.

    x (S, L, H, P), dt (S, L, H), B and Cm (S, L, G, N) hold tokens
    [l0, l1) of every sequence.  Returns (state (S, H, P, N) f32,
    log_decay (S, H) f32 = sum_t A_h dt_t), plus the scratch holding the
    run states when keep_scratch (for scan_shard).  See helix_ext.h."""
    import torch
    ctx = _ctx_for(x, ctx)
    S, L, H, P = x.shape
    N = B.shape[3]
    state = torch.empty((S, H, P, N), dtype=torch.float32, device=x.device)
    log_decay = torch.empty((S, H), dtype=torch.float32, device=x.device)
    d = desc_from_tensors(x, dt, B, state, None, multipass=True, compute=compute, backend=backend, A=A)
    if Cm.stride() != B.stride():
        d.s_c[:] = list(Cm.stride()[1:]); d.seq_c = Cm.stride(0)
    nbytes = ctx.shard_state_scratch_size(d)
    scratch = torch.empty(max(nbytes, 1), dtype=torch.uint8, device=x.device)
    st = ctx.encode_shard_state(d, x, dt, A, B, Cm, state, log_decay, scratch, stream=stream)
    if stream is not None and hasattr(stream, "cuda_stream"):
        scratch.record_stream(stream)
    if st != abi.HELIX_OK:
        raise HelixError(st, ctx.last_error())
    return (state, log_decay, scratch) if keep_scratch else (state, log_decay)


def scan_shard(x, dt, A, B, Cm, carry, scratch, *, compute: str = "auto", backend: int = abi.HELIX_BACKEND_AUTO,
               ctx: Optional[Context] = None, stream=None):
    """The shard's scan from `carry`, reusing the run states that
    shard_state(..., keep_scratch=True) left in `scratch` (no second state
    pass).  Returns (y, s1)."""
    import torch
    ctx = _ctx_for(x, ctx)
    y = torch.empty(x.shape, dtype=torch.float32, device=x.device)
    s1 = torch.empty(carry.shape, dtype=torch.float32, device=x.device)
    d = desc_from_tensors(x, dt, B, carry, y, multipass=True, compute=compute, backend=backend, A=A)
    if Cm.stride() != B.stride():
        d.s_c[:] = list(Cm.stride()[1:]); d.seq_c = Cm.stride(0)
    st = ctx.encode_shard(d, carry, x, dt, A, B, Cm, y, s1, scratch, stream=stream)
    if stream is not None and hasattr(stream, "cuda_stream"):
        scratch.record_stream(stream)
    if st != abi.HELIX_OK:
        raise HelixError(st, ctx.last_error())
    return y, s1


def carry_combine(s0, states, log_decays, ids=None, *, ctx: Optional[Context] = None, stream=None):
    """State entering a shard: fold of S <- exp(log_decays[j]) S + states[j]
    over the earlier shards j = 0..n-1, from s0[ids[seq]].

    s0 (S0, H, P, N); states (n, S, H, P, N) and log_decays (n, S, H)
    contiguous f32.  Returns carry (S, H, P, N) f32."""
    import torch
    ctx = _ctx_for(s0, ctx)
    n = int(states.shape[0])
    S = int(ids.shape[0]) if ids is not None else int(s0.shape[0])
    H, P, N = s0.shape[1:]
    carry = torch.empty((S, H, P, N), dtype=torch.float32, device=s0.device)
    d = abi.desc_init(1, S, H, P, N, 1)
    d.s_s[:] = list(s0.stride()[1:]); d.seq_s = s0.stride(0)
    if tuple(carry.stride()) != tuple(s0.stride()):
        raise ValueError("s0 must be a dense (S, H, P, N) tensor")
    if n and (not states.is_contiguous() or not log_decays.is_contiguous()):
        raise ValueError("states and log_decays must be contiguous")
    st = ctx.encode_carry_combine(d, s0, states if n else None, log_decays if n else None, n, carry,
                                  ids=ids, stream=stream)
    if st != abi.HELIX_OK:
        raise HelixError(st, ctx.last_error())
    return carry
