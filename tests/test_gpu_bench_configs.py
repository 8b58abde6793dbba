"""Parity at the benchmarked configurations, against the oracle.

  * single-GPU fused forward, bf16 x[1, L, 512], L in {16384, 65536},
    steps in {2, 4, 8} (the headline workload and its sweep): the whole output
    bit for bit against the oracle in both arithmetics (src/cta/serving_vllm.py:
    29-46; the contracted update of kernels/diffusion_triton.py);
  * packed varlen prefill at full size: 64 sequences with lengths U[512, 8192]
    (generator seed 0), D = 4096 bf16, steps 4, both packing rules: the
    shortest, the longest and randomly chosen sequences, each against the
    oracle run on that sequence alone (src/cta/serving_vllm.py:72-111,
    :275-303; every sequence is independent given max_query_len);
  * the long-context stencil at full size on one GPU: bf16 x[1, 1048576, 4096],
    steps 8, cut into 8 shards whose interior and edge parts run as on 8 ranks
    (halos sliced from the full tensor); windows straddling all 7 shard edges
    and both global ends against the windowed oracle, forward bit for bit and
    adjoint to the bf16 bar, and the whole result against the unsharded kernel.
"""
from __future__ import annotations

import pytest
import torch

from oracle import diffusion_oracle as O

pytestmark = pytest.mark.gpu


def _ops():
    from cta_b200 import ops
    return ops


@pytest.mark.parametrize("L", [16384, 65536])
@pytest.mark.parametrize("steps", [2, 4, 8])
def test_headline_forward_full_size(L, steps):
    """Both arithmetics: the default contracted update against the contracted
    oracle, the exact one against the reference's op order, and the two within
    one bf16 rounding of each other (the 2e-2 bar)."""
    gen = torch.Generator().manual_seed(L + steps)
    x = torch.randn(1, L, 512, generator=gen).to(torch.bfloat16)
    xd = x.cuda()
    y = _ops().bld_forward(xd, [0.1] * steps, steps).cpu()
    ref = O.steps_bld(x, alpha=0.1, steps=steps, contracted=True)
    assert torch.equal(y, ref), (y.float() - ref.float()).abs().max()
    ye = _ops().bld_forward(xd, [0.1] * steps, steps, arith="exact").cpu()
    ref_e = O.steps_bld(x, alpha=0.1, steps=steps)
    assert torch.equal(ye, ref_e), (ye.float() - ref_e.float()).abs().max()
    assert (y.float() - ref_e.float()).abs().max().item() <= 2e-2


def _varlen_case():
    gen = torch.Generator().manual_seed(0)
    lens = torch.randint(512, 8193, (64,), generator=gen)
    qsl = torch.zeros(65, dtype=torch.int64)
    qsl[1:] = torch.cumsum(lens, 0)
    return lens, qsl


@pytest.mark.parametrize("pad_to_max", [True, False])
def test_varlen_mixer_full_size(pad_to_max):
    lens, qsl = _varlen_case()
    T, D, S = int(qsl[-1]), 4096, 4
    max_len = int(lens.max())
    dev_gen = torch.Generator(device="cuda").manual_seed(7)
    x = torch.randn(T, D, device="cuda", dtype=torch.bfloat16, generator=dev_gen)
    y = _ops().varlen_forward(x, qsl.to(torch.int32).cuda(), max_len, 0.1, S, pad_to_max=pad_to_max)
    pick = torch.randperm(64, generator=torch.Generator().manual_seed(1))[:3].tolist()
    pick += [int(lens.argmin()), int(lens.argmax()), 0, 63]
    for i in sorted(set(pick)):
        a, b = int(qsl[i]), int(qsl[i + 1])
        xs = x[a:b].cpu().unsqueeze(0)
        if pad_to_max:  # the reference rule: the sequence zero-padded to max_query_len
            xp = torch.zeros(1, max_len, D, dtype=xs.dtype)
            xp[:, : b - a] = xs
            ref = O.steps_bld(xp, alpha=0.1, steps=S, contracted=True)[:, : b - a]
        else:
            ref = O.steps_bld(xs, alpha=0.1, steps=S, contracted=True)
        assert torch.equal(y[a:b].cpu().unsqueeze(0), ref), (i, b - a)


def _run_parts(x, P, steps, backward):
    """Every shard's interior and edge launches, halos sliced from the full tensor."""
    from cta_b200 import _lib
    from cta_b200.sharded import even_shards, halo_rows

    B, L, D = x.shape
    hl, hr = halo_rows(steps, False, backward)
    out = torch.empty_like(x)
    edges = []
    for r in range(P):
        spec = even_shards(L, P, r)
        a, b = spec.pos_offset, spec.pos_offset + spec.local_len
        if a > 0:
            edges.append(a)
        xl = x[:, a:b].contiguous()
        lo = x[:, a - hl : a].contiguous() if a > 0 else None
        hi = x[:, b : b + hr].contiguous() if b < L else None
        ol = torch.empty_like(xl)
        for part in (_lib.SHARD_INTERIOR, _lib.SHARD_LO_EDGE, _lib.SHARD_HI_EDGE):
            _ops().shard_part(xl, ol, part, pos_offset=a, global_len=L, alpha=0.1, steps=steps,
                              backward=backward, lo_halo=lo, hi_halo=hi)
        out[:, a:b] = ol
        del xl, ol
    return out, edges


def test_long_context_sharded_full_size():
    L, D, S, P = 1 << 20, 4096, 8, 8
    gen = torch.Generator(device="cuda").manual_seed(1000)
    x = torch.randn(1, L, D, device="cuda", dtype=torch.bfloat16, generator=gen)
    y, edges = _run_parts(x, P, S, backward=False)
    assert len(edges) == P - 1
    assert torch.equal(y, _ops().bld_forward(x, [0.1] * S, S))
    w = 96  # output rows checked on each side of an edge / inside each end
    checks = [(0, w), (L - w, L)] + [(e - w, e + w) for e in edges]
    for a, b in checks:
        ws, we = max(0, a - S), min(L, b + S)
        ref = O.window_bld(x[:, ws:we].cpu(), win_start=ws, global_len=L, out_start=a, out_stop=b, alpha=0.1,
                           steps=S, contracted=True)
        assert torch.equal(y[:, a:b].cpu(), ref), (a, b)
    del y
    g = torch.randn(1, L, D, device="cuda", dtype=torch.bfloat16, generator=gen)
    dx, _ = _run_parts(g, P, S, backward=True)
    full_dx, _ = _ops().bld_backward(g, [0.1] * S, S)
    assert torch.equal(dx, full_dx)
    for a, b in checks:
        ws, we = max(0, a - S), min(L, b + S)
        ref_dx, _ = O.window_bld_grads(g[:, ws:we].cpu(), x[:, ws:we].cpu(), win_start=ws, global_len=L,
                                       out_start=a, out_stop=b, alphas=[0.1] * S)
        # the north-star bar for bf16: max-abs error <= 2e-2 relative to the largest |value|
        err = (dx[:, a:b].cpu().float() - ref_dx).abs().max().item()
        assert err <= 2e-2 * max(1.0, ref_dx.abs().max().item()), (a, b, err)
