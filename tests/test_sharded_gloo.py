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


def _cpu_compute_dalpha(part, g_local, x_local, dx, dalpha, *, g_lo, g_hi, x_lo, x_hi, spec, alphas, steps, causal):
    """Oracle stand-in for the d(alpha) shard kernels: dx rows of `part` and the
    part's d(alpha) sum from windows [lo halo | shard | hi halo] of g and x."""
    from cta_b200.sharded import halo_rows_dalpha, partition_dalpha

    ob, oe = partition_dalpha(spec, steps, causal)[part]
    if oe <= ob:
        return
    h = halo_rows_dalpha(steps, causal)
    B, Lloc, D = g_local.shape
    nlo = max(h["g"][0], h["x"][0]) if (g_lo is not None or x_lo is not None) else 0
    nhi = max(h["g"][1], h["x"][1]) if (g_hi is not None or x_hi is not None) else 0

    def window(t, lo, hi):
        z = torch.zeros(B, nlo + Lloc + nhi, D, dtype=t.dtype)
        z[:, nlo : nlo + Lloc] = t
        if lo is not None:
            z[:, nlo - lo.shape[1] : nlo] = lo
        if hi is not None:
            z[:, nlo + Lloc : nlo + Lloc + hi.shape[1]] = hi
        return z

    start = spec.pos_offset - nlo
    d, da = O.window_bld_grads(window(g_local, g_lo, g_hi), window(x_local, x_lo, x_hi), win_start=start,
                               global_len=spec.global_len, out_start=spec.pos_offset + ob,
                               out_stop=spec.pos_offset + oe, alphas=alphas, causal=causal)
    dx[:, ob:oe] = d
    dalpha += da.float()


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
        if mode.startswith("dalpha"):
            from cta_b200.sharded import sharded_diffusion_backward_dalpha

            causal = mode == "dalpha_causal"
            g = torch.randn(2, L, 8)
            al = [0.1, 0.05, 0.12, 0.02, 0.08, 0.03, 0.11, 0.07][:steps]
            gl = g[:, spec.pos_offset : spec.pos_offset + spec.local_len]
            dx, da = sharded_diffusion_backward_dalpha(gl, xl, spec, alphas=al, steps=steps, causal=causal,
                                                       compute=_cpu_compute_dalpha)
            dx_ref, da_ref = O.grads(lambda t, *a: O.fused_stack(t, list(a), layout="bld", causal=causal), x, g,
                                     [torch.tensor([v]) for v in al])
            dx_ref = dx_ref[:, spec.pos_offset : spec.pos_offset + spec.local_len]
            da_ref = torch.cat(da_ref)
            ok = (dx - dx_ref).abs().max().item() <= 1e-5 * dx_ref.abs().max().item() and \
                (da - da_ref).abs().max().item() <= 1e-4 * max(1.0, da_ref.abs().max().item())
            q.put((rank, "ok" if ok else f"mismatch dx {(dx - dx_ref).abs().max().item()} da {da} vs {da_ref}"))
            dist.destroy_process_group()
            return
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


@pytest.mark.parametrize("world,L,steps,mode", [(2, 100, 4, "dalpha"), (3, 61, 2, "dalpha"),
                                               (2, 100, 4, "dalpha_causal"), (3, 70, 3, "dalpha_causal")])
def test_sharded_backward_dalpha_matches_unsharded(world, L, steps, mode):
    """Halo exchange of g and x, per-part d(alpha) sums and the all-reduce
    reproduce the unsharded autograd gradients (dx and d(alpha))."""
    res, alive = _run(world, L, steps, mode)
    assert not alive, "a rank hung"
    assert res == {r: "ok" for r in range(world)}, res


def test_dead_rank_is_detected_not_hung():
    res, alive = _run(2, 100, 4, "die", timeout=90)
    assert not alive, "surviving rank hung instead of failing"
    assert 0 in res and res[0].startswith("error"), res
