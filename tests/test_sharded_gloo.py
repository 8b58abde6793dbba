"""L-sharded halo exchange protocol on CPU ranks (gloo, world_size 2..3), and
host-side failure detection: a rank that dies before the exchange makes its
neighbour fail within the process-group timeout instead of hanging."""
from __future__ import annotations

import datetime
import os
import socket
import sys
import traceback

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import diffusion_oracle as O


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _cpu_compute(part, x_local, out, *, lo_halo, hi_halo, spec, alpha, steps, causal, backward):
    """Oracle stand-in for the shard kernels (non-causal forward): rows of `part`
    from [lo_halo | x_local | hi_halo]."""
    from cta_b200.sharded import partition

    ob, oe = partition(spec, steps, causal, backward)[part]
    if oe <= ob:
        return
    parts, start = [], spec.pos_offset
    if lo_halo is not None:
        parts.append(lo_halo)
        start -= lo_halo.shape[1]
    parts.append(x_local)
    if hi_halo is not None:
        parts.append(hi_halo)
    win = torch.cat(parts, dim=1)
    out[:, ob:oe] = O.window_bld(win, win_start=start, global_len=spec.global_len, out_start=spec.pos_offset + ob,
                                 out_stop=spec.pos_offset + oe, alpha=alpha, steps=steps)


def _worker(rank, world, port, L, steps, mode, q):
    sys.path[:0] = [os.environ["CTA_REPO"], os.path.join(os.environ["CTA_REPO"], "continuous-time-attention_b200")]
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    try:
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=6))
        from cta_b200.sharded import even_shards, sharded_diffusion

        torch.manual_seed(0)
        x = torch.randn(2, L, 8)
        spec = even_shards(L, world, rank)
        xl = x[:, spec.pos_offset : spec.pos_offset + spec.local_len]
        if mode == "die" and rank == world - 1:
            os._exit(3)  # leaves without joining the exchange
        y = sharded_diffusion(xl, spec, alpha=0.1, steps=steps, compute=_cpu_compute)
        ref = O.steps_bld(x, alpha=0.1, steps=steps)[:, spec.pos_offset : spec.pos_offset + spec.local_len]
        q.put((rank, "ok" if torch.equal(y, ref) else f"mismatch {(y - ref).abs().max().item()}"))
        dist.destroy_process_group()
    except Exception as e:  # noqa: BLE001
        q.put((rank, f"error {type(e).__name__}: {e}".splitlines()[0] + traceback.format_exc()[-200:]))


def _run(world, L, steps, mode, timeout=60):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    os.environ["CTA_REPO"] = str(__import__("pathlib").Path(__file__).resolve().parents[1])
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, L, steps, mode, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout)
    alive = [p for p in procs if p.is_alive()]
    for p in alive:
        p.kill()
    res = {}
    while not q.empty():
        r, v = q.get()
        res[r] = v
    return res, alive


@pytest.mark.parametrize("world,L,steps", [(2, 100, 8), (3, 61, 4), (2, 40, 1)])
def test_sharded_matches_unsharded(world, L, steps):
    res, alive = _run(world, L, steps, "ok")
    assert not alive, "a rank hung"
    assert res == {r: "ok" for r in range(world)}, res


def test_dead_rank_is_detected_not_hung():
    res, alive = _run(2, 100, 4, "die", timeout=90)
    assert not alive, "surviving rank hung instead of failing"
    assert 0 in res and res[0].startswith("error"), res
