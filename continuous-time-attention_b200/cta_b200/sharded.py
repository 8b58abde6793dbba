"""L-sharded diffusion stencil for sequences too long for one GPU.

The sequence axis of a [B, L, D] tensor is split into contiguous shards, one
per rank.  A fused forward (or adjoint) over `steps` steps needs, for every
output row, the input rows within `steps` of it (2*steps on one side for the
causal stencil and its adjoint), so each call:

  1. exchanges the halos -- the rows a neighbour needs are sent with NCCL
     point-to-point (``batch_isend_irecv``), a few tens of microseconds;
  2. runs the two small edge kernels, which read the received rows, on a side
     stream;
  3. meanwhile runs the interior kernel, which computes every output row whose
     stencil stays inside the local shard.

The exchange comes first because NCCL's kernel needs SMs of its own: queued
beside the interior kernel, whose one-warp CTAs occupy every SM in one wave, it
would start only at that kernel's tail (measured on 2 B200s: ~110 us of exposed
wait per call when the exchange was posted to run under the interior kernel).

Only the two global ends of the sequence use the copy boundary; shard edges
are interior rows.  The reference has no multi-device path (it runs the
stencil on one device); results are identical to the unsharded stencil.

The backward with d(alpha) (learnable per-step alphas) exchanges halos of both
the gradient and the forward input x, sums each rank's d(alpha) over its own
rows (interior + edge parts, in that order) and all-reduces the `steps` sums.

The compute step is injectable (``compute=``) so that the exchange protocol can
be exercised on CPU ranks (gloo) in the tests; the default is the sm_100a
kernels through :func:`cta_b200.ops.shard_part` / ``shard_part_dalpha``.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Callable, Optional

import torch
import torch.distributed as dist

from . import _lib

__all__ = ["ShardSpec", "halo_rows", "sharded_diffusion", "sharded_diffusion_backward_dalpha", "even_shards"]


@dataclass(frozen=True)
class ShardSpec:
    rank: int
    world: int
    pos_offset: int   # global row of local row 0
    local_len: int
    global_len: int


def even_shards(global_len: int, world: int, rank: int) -> ShardSpec:
    """Contiguous split, the first (global_len % world) shards one row longer."""
    base, rem = divmod(global_len, world)
    lens = [base + (1 if r < rem else 0) for r in range(world)]
    return ShardSpec(rank, world, sum(lens[:rank]), lens[rank], global_len)


def halo_rows(steps: int, causal: bool, backward: bool) -> tuple[int, int]:
    """(rows needed from the previous shard, rows needed from the next shard)."""
    if causal:
        return (0, 2 * steps) if backward else (2 * steps, 0)
    return steps, steps


def partition(spec: ShardSpec, steps: int, causal: bool, backward: bool) -> dict[int, tuple[int, int]]:
    """Local output rows of each launch part, {part: (begin, end)}.

    Interior rows are those whose stencil reach stays inside the shard (or
    runs off a global end); the edge parts are the rest.  The same rule is
    applied by cta_diffusion_shard_bld in the C ABI.
    """
    hl, hr = halo_rows(steps, causal, backward)
    L = spec.local_len
    has_lo = spec.pos_offset > 0
    has_hi = spec.pos_offset + L < spec.global_len
    ib = min(hl, L) if has_lo else 0
    ie = max(L - hr, ib) if has_hi else L
    return {_lib.SHARD_INTERIOR: (ib, ie), _lib.SHARD_LO_EDGE: (0, ib), _lib.SHARD_HI_EDGE: (ie, L)}


class _PartEvents:
    """Records (start, end) CUDA event pairs per part into a caller's dict."""

    def __init__(self, sink: Optional[dict]):
        self.sink = sink
        self.open: dict = {}

    def begin(self, name: str, stream) -> None:
        if self.sink is not None:
            e = torch.cuda.Event(enable_timing=True)
            e.record(stream)
            self.open[name] = e

    def end(self, name: str, stream) -> None:
        if self.sink is not None:
            e = torch.cuda.Event(enable_timing=True)
            e.record(stream)
            self.sink.setdefault(name, []).append((self.open.pop(name), e))


def _default_compute(part, x_local, out, *, lo_halo, hi_halo, spec, alpha, steps, causal, backward):
    from . import ops

    ops.shard_part(x_local, out, part, pos_offset=spec.pos_offset, global_len=spec.global_len, alpha=alpha,
                   steps=steps, causal=causal, backward=backward, lo_halo=lo_halo, hi_halo=hi_halo)


def sharded_diffusion(
    x_local: torch.Tensor,
    spec: ShardSpec,
    *,
    alpha: float,
    steps: int,
    causal: bool = False,
    backward: bool = False,
    group: Optional[dist.ProcessGroup] = None,
    comm_stream: Optional[torch.cuda.Stream] = None,
    compute: Optional[Callable] = None,
    timing: Optional[dict] = None,
    overlap: bool = True,
) -> torch.Tensor:
    """Fused `steps`-step stencil (or its adjoint) of this rank's shard.

    Every rank must call this with the same steps / causal / backward; ranks
    exchange halos with their neighbours only.  Returns the local output shard.

    `overlap` (CUDA): True posts the halo exchange and then the two edge kernels
    on the side stream `comm_stream` before the interior kernel is launched on
    the caller's stream, so the exchange runs beside the interior.  It needs
    NCCL on high-priority streams (ProcessGroupNCCL.Options with
    is_high_priority_stream, or TORCH_NCCL_HIGH_PRIORITY=1) and a high-priority
    `comm_stream` (the default one is): otherwise the interior's CTAs, which
    fill every SM, are scheduled ahead of NCCL's and the exchange waits for the
    interior to drain.  False exchanges first on the caller's stream (fully
    exposed, ~one NCCL round trip), then runs the edges beside the interior.

    `timing` (CUDA only): a dict that receives pairs of recorded CUDA events per
    part -- "interior" (the interior kernel), "exchange" (the halo send/recv),
    "exposed_wait" (caller stream idle after the interior kernel until the side
    stream's work is done) and "edges" (both edge kernels) -- for the caller to
    read after a synchronize.
    """
    if x_local.dim() != 3:
        raise ValueError("x_local must be (B, L_local, D)")
    if not 1 <= steps <= _lib.MAX_STEPS:
        raise ValueError(f"steps must be in 1..{_lib.MAX_STEPS}, got {steps}")
    B, Lloc, D = x_local.shape
    if Lloc != spec.local_len:
        raise ValueError(f"x_local has {Lloc} rows, spec says {spec.local_len}")
    hl, hr = halo_rows(steps, causal, backward)
    prev_rank = spec.rank - 1 if spec.rank > 0 else None
    next_rank = spec.rank + 1 if spec.rank + 1 < spec.world else None
    # a neighbour's request must be servable from one shard
    if (prev_rank is not None and hr and Lloc < hr) or (next_rank is not None and hl and Lloc < hl):
        raise ValueError("shard shorter than the halo it must provide")
    if compute is None:
        compute = _default_compute
    x_local = x_local.contiguous()
    out = torch.empty_like(x_local)
    if spec.global_len < 3:
        out.copy_(x_local)
        return out
    on_gpu = x_local.device.type == "cuda"
    cur = torch.cuda.current_stream(x_local.device) if on_gpu else None

    lo_halo = torch.empty((B, hl, D), dtype=x_local.dtype, device=x_local.device) if (prev_rank is not None and hl) else None
    hi_halo = torch.empty((B, hr, D), dtype=x_local.dtype, device=x_local.device) if (next_rank is not None and hr) else None

    def post_exchange():
        ops = []
        # my first hr rows are the next-shard halo of the previous rank; my last hl rows the lo halo of the next
        if prev_rank is not None and hr:
            ops.append(dist.P2POp(dist.isend, x_local[:, :hr].contiguous(), prev_rank, group))
        if next_rank is not None and hl:
            ops.append(dist.P2POp(dist.isend, x_local[:, Lloc - hl :].contiguous(), next_rank, group))
        if lo_halo is not None:
            ops.append(dist.P2POp(dist.irecv, lo_halo, prev_rank, group))
        if hi_halo is not None:
            ops.append(dist.P2POp(dist.irecv, hi_halo, next_rank, group))
        return dist.batch_isend_irecv(ops) if ops else []

    kw = dict(spec=spec, alpha=alpha, steps=steps, causal=causal, backward=backward)
    ev = _PartEvents(timing if on_gpu else None)
    if on_gpu:
        comm = comm_stream if comm_stream is not None else torch.cuda.Stream(device=x_local.device, priority=-1)
        comm.wait_stream(cur)
        if overlap:
            # exchange and edges on the side stream, queued ahead of the interior
            with torch.cuda.stream(comm):
                ev.begin("exchange", comm)
                for w in post_exchange():
                    w.wait()
                ev.end("exchange", comm)
        else:
            # the exchange first, on the caller's stream
            ev.begin("exchange", cur)
            for w in post_exchange():
                w.wait()
            ev.end("exchange", cur)
            comm.wait_stream(cur)
        # the edge parts read the halos; their few CTAs run beside the interior
        with torch.cuda.stream(comm):
            ev.begin("edges", comm)
            compute(_lib.SHARD_LO_EDGE, x_local, out, lo_halo=lo_halo, hi_halo=hi_halo, **kw)
            compute(_lib.SHARD_HI_EDGE, x_local, out, lo_halo=lo_halo, hi_halo=hi_halo, **kw)
            ev.end("edges", comm)
        ev.begin("interior", cur)
        compute(_lib.SHARD_INTERIOR, x_local, out, lo_halo=None, hi_halo=None, **kw)
        ev.end("interior", cur)
        ev.begin("exposed_wait", cur)
        cur.wait_stream(comm)
        ev.end("exposed_wait", cur)
        for h in (lo_halo, hi_halo):
            if h is not None:
                h.record_stream(comm)
        return out
    works = post_exchange()
    compute(_lib.SHARD_INTERIOR, x_local, out, lo_halo=None, hi_halo=None, **kw)
    for w in works:
        w.wait()
    compute(_lib.SHARD_LO_EDGE, x_local, out, lo_halo=lo_halo, hi_halo=hi_halo, **kw)
    compute(_lib.SHARD_HI_EDGE, x_local, out, lo_halo=lo_halo, hi_halo=hi_halo, **kw)
    return out


def halo_rows_dalpha(steps: int, causal: bool) -> dict[str, tuple[int, int]]:
    """Rows (before, after) the shard that the backward with d(alpha) needs, per
    stream: the gradient g and the forward input x."""
    if causal:
        return {"g": (0, 2 * steps), "x": (2 * steps, 0)}
    return {"g": (steps, steps), "x": (steps, steps)}


def partition_dalpha(spec: ShardSpec, steps: int, causal: bool) -> dict[int, tuple[int, int]]:
    """Local output rows of each launch part of the backward with d(alpha)
    (the rule of cta_diffusion_shard_bld_dalpha)."""
    h = halo_rows_dalpha(steps, causal)
    hl, hr = max(h["g"][0], h["x"][0]), max(h["g"][1], h["x"][1])
    L = spec.local_len
    has_lo = spec.pos_offset > 0
    has_hi = spec.pos_offset + L < spec.global_len
    ib = min(hl, L) if has_lo else 0
    ie = max(L - hr, ib) if has_hi else L
    return {_lib.SHARD_INTERIOR: (ib, ie), _lib.SHARD_LO_EDGE: (0, ib), _lib.SHARD_HI_EDGE: (ie, L)}


def _default_compute_dalpha(part, g_local, x_local, dx, dalpha, *, g_lo, g_hi, x_lo, x_hi, spec, alphas, steps,
                            causal):
    from . import ops

    ops.shard_part_dalpha(g_local, x_local, dx, dalpha, part, pos_offset=spec.pos_offset,
                          global_len=spec.global_len, alphas=alphas, steps=steps, causal=causal, g_lo=g_lo,
                          g_hi=g_hi, x_lo=x_lo, x_hi=x_hi)


def sharded_diffusion_backward_dalpha(
    g_local: torch.Tensor,
    x_local: torch.Tensor,
    spec: ShardSpec,
    *,
    alphas,
    steps: int,
    causal: bool = False,
    group: Optional[dist.ProcessGroup] = None,
    comm_stream: Optional[torch.cuda.Stream] = None,
    compute: Optional[Callable] = None,
    overlap: bool = True,
) -> tuple[torch.Tensor, torch.Tensor]:
    """Backward of `steps` fused steps with per-step `alphas` on this rank's
    shard: returns (dx_local, dalpha), dalpha (fp32 [steps]) summed over all
    ranks of `group`.  Every rank must call this with the same arguments.
    `overlap` as in `sharded_diffusion`: the exchange on the side stream beside
    the interior kernel (True) or first on the caller's stream (False); the
    edge parts run after the interior either way, because the three parts add
    their d(alpha) sums to one buffer in a fixed order."""
    if g_local.dim() != 3 or tuple(x_local.shape) != tuple(g_local.shape):
        raise ValueError("g_local and x_local must both be (B, L_local, D)")
    if not 1 <= steps <= _lib.MAX_STEPS:
        raise ValueError(f"steps must be in 1..{_lib.MAX_STEPS}, got {steps}")
    alphas = [float(a) for a in alphas]
    if len(alphas) != steps:
        raise ValueError("need one alpha per step")
    B, Lloc, D = g_local.shape
    if Lloc != spec.local_len:
        raise ValueError(f"g_local has {Lloc} rows, spec says {spec.local_len}")
    h = halo_rows_dalpha(steps, causal)
    need_lo = max(h["g"][0], h["x"][0])
    need_hi = max(h["g"][1], h["x"][1])
    prev_rank = spec.rank - 1 if spec.rank > 0 else None
    next_rank = spec.rank + 1 if spec.rank + 1 < spec.world else None
    if (prev_rank is not None and need_hi and Lloc < need_hi) or (next_rank is not None and need_lo and Lloc < need_lo):
        raise ValueError("shard shorter than the halo it must provide")
    if compute is None:
        compute = _default_compute_dalpha
    g_local = g_local.contiguous()
    x_local = x_local.contiguous()
    dev = g_local.device
    dx = torch.empty_like(g_local)
    dalpha = torch.zeros(steps, dtype=torch.float32, device=dev)
    if spec.global_len < 3:
        dx.copy_(g_local)
        return dx, dalpha
    on_gpu = dev.type == "cuda"
    cur = torch.cuda.current_stream(dev) if on_gpu else None

    def buf(rows, present):
        return torch.empty((B, rows, D), dtype=g_local.dtype, device=dev) if (present and rows) else None

    halos = {
        "g_lo": buf(h["g"][0], prev_rank is not None), "x_lo": buf(h["x"][0], prev_rank is not None),
        "g_hi": buf(h["g"][1], next_rank is not None), "x_hi": buf(h["x"][1], next_rank is not None),
    }

    def post_exchange():
        ops = []
        for name, t in (("g", g_local), ("x", x_local)):
            lo, hi = h[name]
            # my first `hi` rows are the previous rank's hi halo; my last `lo` rows the next rank's lo halo
            if prev_rank is not None and hi:
                ops.append(dist.P2POp(dist.isend, t[:, :hi].contiguous(), prev_rank, group))
            if next_rank is not None and lo:
                ops.append(dist.P2POp(dist.isend, t[:, Lloc - lo :].contiguous(), next_rank, group))
            if halos[name + "_lo"] is not None:
                ops.append(dist.P2POp(dist.irecv, halos[name + "_lo"], prev_rank, group))
            if halos[name + "_hi"] is not None:
                ops.append(dist.P2POp(dist.irecv, halos[name + "_hi"], next_rank, group))
        return dist.batch_isend_irecv(ops) if ops else []

    kw = dict(spec=spec, alphas=alphas, steps=steps, causal=causal)
    none = dict(g_lo=None, g_hi=None, x_lo=None, x_hi=None)
    if on_gpu and overlap:
        comm = comm_stream if comm_stream is not None else torch.cuda.Stream(device=dev, priority=-1)
        comm.wait_stream(cur)
        with torch.cuda.stream(comm):
            for w in post_exchange():
                w.wait()
        compute(_lib.SHARD_INTERIOR, g_local, x_local, dx, dalpha, **none, **kw)
        cur.wait_stream(comm)
        for t in halos.values():
            if t is not None:
                t.record_stream(comm)
    elif on_gpu:
        # exchange first on the caller's stream; the parts then add their
        # d(alpha) sums in a fixed order: interior, lo edge, hi edge
        for w in post_exchange():
            w.wait()
        compute(_lib.SHARD_INTERIOR, g_local, x_local, dx, dalpha, **none, **kw)
    else:
        works = post_exchange()
        compute(_lib.SHARD_INTERIOR, g_local, x_local, dx, dalpha, **none, **kw)
        for w in works:
            w.wait()
    compute(_lib.SHARD_LO_EDGE, g_local, x_local, dx, dalpha, **halos, **kw)
    compute(_lib.SHARD_HI_EDGE, g_local, x_local, dx, dalpha, **halos, **kw)
    if spec.world > 1:
        dist.all_reduce(dalpha, op=dist.ReduceOp.SUM, group=group)
    return dx, dalpha
