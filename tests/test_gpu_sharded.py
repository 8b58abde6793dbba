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
        assert torch.equal(y.cpu(), O.steps_bld(x.cpu(), alpha=0.1, steps=steps))


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
