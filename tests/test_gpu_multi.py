"""L-sharded stencil across real GPUs: NCCL halo exchange + interior/edge
kernels on 2 ranks reproduce the single-GPU fused kernels bit for bit.
Skipped when fewer than two GPUs are visible."""
from __future__ import annotations

import datetime
import os
import socket
import sys

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q):
    repo = os.environ["CTA_REPO"]
    sys.path[:0] = [repo, os.path.join(repo, "continuous-time-attention_b200")]
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    try:
        import torch.distributed as dist

        torch.cuda.set_device(rank)
        dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                                device_id=torch.device("cuda", rank))
        from cta_b200 import ops
        from cta_b200.sharded import even_shards, sharded_diffusion

        results = []
        for steps, causal, backward in [(8, False, False), (4, True, False), (8, False, True), (2, True, True)]:
            torch.manual_seed(0)
            x = torch.randn(2, 3001, 512, dtype=torch.bfloat16).cuda()
            spec = even_shards(3001, world, rank)
            xl = x[:, spec.pos_offset : spec.pos_offset + spec.local_len]
            y = sharded_diffusion(xl, spec, alpha=0.1, steps=steps, causal=causal, backward=backward)
            if backward:
                full, _ = ops.bld_backward(x, [0.1] * steps, steps, causal=causal)
            else:
                full = ops.bld_forward(x, [0.1] * steps, steps, causal=causal)
            ref = full[:, spec.pos_offset : spec.pos_offset + spec.local_len]
            torch.cuda.synchronize()
            results.append(bool(torch.equal(y, ref)))
        from cta_b200.sharded import sharded_diffusion_backward_dalpha

        for steps, causal in [(4, False), (3, True), (8, False), (7, True)]:
            torch.manual_seed(1)
            x = torch.randn(2, 3001, 512, dtype=torch.bfloat16).cuda()
            g = torch.randn(2, 3001, 512, dtype=torch.bfloat16).cuda()
            al = [0.1, 0.05, 0.12, 0.02, 0.08, 0.03, 0.11, 0.07][:steps]
            spec = even_shards(3001, world, rank)
            sl = slice(spec.pos_offset, spec.pos_offset + spec.local_len)
            dx, da = sharded_diffusion_backward_dalpha(g[:, sl], x[:, sl], spec, alphas=al, steps=steps,
                                                       causal=causal)
            full_dx, full_da = ops.bld_backward(g, al, steps, x=x, causal=causal, need_dalpha=True)
            torch.cuda.synchronize()
            scale = max(1.0, full_da.abs().max().item())
            results.append(bool(torch.equal(dx, full_dx[:, sl])) and
                           (da - full_da).abs().max().item() <= 1e-5 * scale)
        q.put((rank, results))
        dist.destroy_process_group()
    except Exception as e:  # noqa: BLE001
        q.put((rank, f"error {type(e).__name__}: {e}"))


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_two_gpu_sharded_matches_single_gpu():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    os.environ["CTA_REPO"] = str(__import__("pathlib").Path(__file__).resolve().parents[1])
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(240)
    for p in procs:
        if p.is_alive():
            p.kill()
    res = {}
    while not q.empty():
        r, v = q.get()
        res[r] = v
    assert res == {0: [True] * 8, 1: [True] * 8}, res
