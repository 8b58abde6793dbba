"""L-shard kernels on one GPU: every shard's interior and edge launches, fed
with halos sliced from the full tensor, reproduce the unsharded fused kernels
bit for bit (forward and adjoint, centred and causal stencils)."""
from __future__ import annotations

import pytest
import torch

from oracle import diffusion_oracle as O

pytestmark = pytest.mark.gpu


def _run_sharded(x, P, steps, causal, backward):
    from cta_b200 import _lib, ops
    from cta_b200.sharded import even_shards, halo_rows

    B, L, D = x.shape
    hl, hr = halo_rows(steps, causal, backward)
    outs = []
    for r in range(P):
        spec = even_shards(L, P, r)
        a, b = spec.pos_offset, spec.pos_offset + spec.local_len
        xl = x[:, a:b].contiguous()
        lo = x[:, a - hl : a].contiguous() if (a > 0 and hl) else None
        hi = x[:, b : b + hr].contiguous() if (b < L and hr) else None
        out = torch.empty_like(xl)
        for part in (_lib.SHARD_INTERIOR, _lib.SHARD_LO_EDGE, _lib.SHARD_HI_EDGE):
            ops.shard_part(xl, out, part, pos_offset=a, global_len=L, alpha=0.1, steps=steps, causal=causal,
                           backward=backward, lo_halo=lo, hi_halo=hi)
        outs.append(out)
    return torch.cat(outs, dim=1)


@pytest.mark.parametrize("P", [2, 3, 4])
@pytest.mark.parametrize("steps", [1, 2, 4, 8])
@pytest.mark.parametrize("D", [512, 6])
@pytest.mark.parametrize("causal", [False, True])
def test_sharded_forward_equals_unsharded(P, steps, D, causal):
    from cta_b200 import ops

    torch.manual_seed(P * 100 + steps)
    x = torch.randn(2, 1001, D, device="cuda", dtype=torch.bfloat16)
    full = ops.bld_forward(x, [0.1] * steps, steps, causal=causal)
    y = _run_sharded(x, P, steps, causal, backward=False)
    assert torch.equal(y, full)
    if not causal:
        assert torch.equal(y.cpu(), O.steps_bld(x.cpu(), alpha=0.1, steps=steps, contracted=True))


@pytest.mark.parametrize("P", [2, 4])
@pytest.mark.parametrize("steps", [1, 4, 8])
@pytest.mark.parametrize("causal", [False, True])
def test_sharded_adjoint_equals_unsharded(P, steps, causal):
    from cta_b200 import ops

    torch.manual_seed(P + steps)
    g = torch.randn(1, 777, 512, device="cuda", dtype=torch.float32)
    full, _ = ops.bld_backward(g, [0.1] * steps, steps, causal=causal)
    dx = _run_sharded(g, P, steps, causal, backward=True)
    assert torch.equal(dx, full)


def test_short_shards_need_both_halos():
    # shards shorter than the halo depth: edge tiles read both neighbours' rows
    from cta_b200 import ops

    torch.manual_seed(3)
    x = torch.randn(1, 40, 64, device="cuda")
    full = ops.bld_forward(x, [0.1] * 8, 8)
    y = _run_sharded(x, 4, 8, False, backward=False)
    assert torch.equal(y, full)


def _run_sharded_dalpha(g, x, P, steps, causal, alphas):
    from cta_b200 import _lib, ops
    from cta_b200.sharded import even_shards, halo_rows_dalpha

    B, L, D = g.shape
    h = halo_rows_dalpha(steps, causal)
    outs, das = [], []
    for r in range(P):
        spec = even_shards(L, P, r)
        a, b = spec.pos_offset, spec.pos_offset + spec.local_len

        def halos(t, name):
            lo, hi = h[name]
            return (t[:, a - lo : a].contiguous() if (a > 0 and lo) else None,
                    t[:, b : b + hi].contiguous() if (b < L and hi) else None)

        g_lo, g_hi = halos(g, "g")
        x_lo, x_hi = halos(x, "x")
        dx = torch.empty_like(g[:, a:b])
        da = torch.zeros(steps, dtype=torch.float32, device=g.device)
        for part in (_lib.SHARD_INTERIOR, _lib.SHARD_LO_EDGE, _lib.SHARD_HI_EDGE):
            ops.shard_part_dalpha(g[:, a:b].contiguous(), x[:, a:b].contiguous(), dx, da, part, pos_offset=a,
                                  global_len=L, alphas=alphas, steps=steps, causal=causal, g_lo=g_lo, g_hi=g_hi,
                                  x_lo=x_lo, x_hi=x_hi)
        outs.append(dx)
        das.append(da)
    return torch.cat(outs, dim=1), torch.stack(das).sum(0)


@pytest.mark.parametrize("P", [2, 3])
@pytest.mark.parametrize("steps", [1, 2, 3, 4])
@pytest.mark.parametrize("causal", [False, True])
@pytest.mark.parametrize("dtype,D", [(torch.float32, 512), (torch.bfloat16, 264), (torch.float32, 6)])
def test_sharded_backward_dalpha_equals_unsharded(P, steps, causal, dtype, D):
    """Interior + edge parts of every shard (halos of g and x sliced from the full
    tensors): dx bit-identical to the unsharded d(alpha) kernel, the summed
    d(alpha) equal up to the summation order, and both against the oracle."""
    from cta_b200 import _lib, ops

    torch.manual_seed(P * 10 + steps)
    al = [0.1, 0.05, 0.12, 0.02][:steps]
    x = torch.randn(2, 1001, D, device="cuda").to(dtype)
    g = torch.randn(2, 1001, D, device="cuda").to(dtype)
    full_dx, full_da = ops.bld_backward(g, al, steps, x=x, causal=causal, need_dalpha=True)
    dx, da = _run_sharded_dalpha(g, x, P, steps, causal, al)
    assert torch.equal(dx, full_dx)
    scale = max(1.0, full_da.abs().max().item())
    assert (da - full_da).abs().max().item() <= 1e-5 * scale, (da, full_da)
    if dtype == torch.float32 and D == 6:
        dx_ref, da_ref = O.grads(lambda t, *a: O.fused_stack(t, list(a), layout="bld", causal=causal), x.cpu(),
                                 g.cpu(), [torch.tensor([v]) for v in al])
        assert (dx.cpu() - dx_ref).abs().max().item() <= 1e-5 * dx_ref.abs().max().item()
        assert (da.cpu() - torch.cat(da_ref)).abs().max().item() <= 1e-4 * scale
    assert _lib.device_error() == 0


@pytest.mark.parametrize("P", [2, 3])
@pytest.mark.parametrize("steps", [5, 6, 7, 8])
@pytest.mark.parametrize("causal", [False, True])
@pytest.mark.parametrize("dtype,D", [(torch.bfloat16, 264), (torch.float32, 6)])
def test_sharded_backward_dalpha_deep_steps(P, steps, causal, dtype, D):
    """Steps 5..8 (the long-context configuration runs 8 learnable steps):
    dx bit-identical to the unsharded kernel, d(alpha) to the summation order,
    and the fp32 case against the oracle's autograd."""
    from cta_b200 import _lib, ops

    torch.manual_seed(P * 10 + steps + 100)
    al = [0.1, 0.05, 0.12, 0.02, 0.08, 0.03, 0.11, 0.07][:steps]
    x = torch.randn(2, 901, D, device="cuda").to(dtype)
    g = torch.randn(2, 901, D, device="cuda").to(dtype)
    full_dx, full_da = ops.bld_backward(g, al, steps, x=x, causal=causal, need_dalpha=True)
    dx, da = _run_sharded_dalpha(g, x, P, steps, causal, al)
    assert torch.equal(dx, full_dx)
    scale = max(1.0, full_da.abs().max().item())
    assert (da - full_da).abs().max().item() <= 1e-5 * scale, (da, full_da)
    if dtype == torch.float32:
        dx_ref, da_ref = O.grads(lambda t, *a: O.fused_stack(t, list(a), layout="bld", causal=causal), x.cpu(),
                                 g.cpu(), [torch.tensor([v]) for v in al])
        assert (dx.cpu() - dx_ref).abs().max().item() <= 1e-5 * dx_ref.abs().max().item()
        assert (da.cpu() - torch.cat(da_ref)).abs().max().item() <= 1e-4 * scale
    assert _lib.device_error() == 0
