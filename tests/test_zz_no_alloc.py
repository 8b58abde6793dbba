"""The allocation-free backward entry point (cta_diffusion_bwd_bld_noalloc).

Some callers cannot give this library fresh device memory: an engine that has
already reserved almost the whole GPU for its own memory pool, or a hot path
that must not pay the implicit synchronisation of cudaMalloc.  For them the
d(alpha) reduction of the fused backward can use a scratch array built into the
library instead of a caller workspace.  These tests call that entry point
through the C ABI and check it against the regular entry point
(cta_diffusion_bwd_bld with a caller workspace), on two calls in a row, since
the built-in scratch is reused and keeps the previous call's contents.

The file is named so that pytest collects it last.
"""
from __future__ import annotations

import ctypes

import pytest
import torch

from conftest import assert_close

pytestmark = pytest.mark.gpu


def _noalloc(g, x, alphas, steps, causal=False, mask=None):
    from cta_b200 import _lib

    lib = _lib.load()
    B, L, D = g.shape
    dx = torch.empty_like(g)
    dalpha = torch.empty(steps, dtype=torch.float32, device=g.device)
    m = None if mask is None else mask.contiguous()
    rc = lib.cta_diffusion_bwd_bld_noalloc(
        g.data_ptr(), dx.data_ptr(), x.data_ptr(), dalpha.data_ptr(), B, L, D, g.stride(0), g.stride(1),
        x.stride(0), x.stride(1), dx.stride(0), dx.stride(1), _lib.dtype_code(g.dtype), steps, int(causal),
        _lib.float_array(alphas), None, 0, _lib.ptr(m), 2 if m is not None else 0,
        m.stride(0) if m is not None else 0, m.stride(1) if m is not None else 0, _lib.stream_ptr(g),
    )
    return rc, dx, dalpha


@pytest.mark.parametrize("dtype,causal,use_mask", [(torch.float32, False, True), (torch.float32, True, False),
                                                   (torch.bfloat16, False, False)])
def test_noalloc_matches_workspace_entry_twice(dtype, causal, use_mask):
    from cta_b200 import _lib, ops

    torch.manual_seed(11)
    B, L, D, steps = 2, 1500, 512, 4
    alphas = [0.1, 0.05, 0.12, 0.02]
    x = torch.randn(B, L, D, device="cuda").to(dtype)
    g = torch.randn(B, L, D, device="cuda").to(dtype)
    mask = None
    if use_mask:
        mask = torch.ones(B, L, dtype=torch.long, device="cuda")
        mask[1, 1300:] = 0
    dx_ref, da_ref = ops.bld_backward(g, alphas, steps, x=x, causal=causal, mask=mask, need_dalpha=True)
    torch.cuda.synchronize()
    rel = 1e-4 if dtype == torch.float32 else 2e-2
    for _ in range(2):  # the scratch keeps the previous call's contents
        rc, dx, da = _noalloc(g, x, alphas, steps, causal=causal, mask=mask)
        _lib.check(rc)
        torch.cuda.synchronize()
        assert_close(dx, dx_ref)
        scale = max(1.0, da_ref.abs().max().item())
        assert (da - da_ref).abs().max().item() <= rel * scale, (da, da_ref)
    assert _lib.device_error() == 0


def test_noalloc_rejects_shapes_beyond_its_scratch():
    from cta_b200 import _lib

    g = torch.empty(1, 1 << 20, 4096, dtype=torch.bfloat16, device="meta")
    lib = _lib.load()
    rc = lib.cta_diffusion_bwd_bld_noalloc(
        16, 16, 16, 16, 1, g.shape[1], g.shape[2], g.shape[1] * g.shape[2], g.shape[2], g.shape[1] * g.shape[2],
        g.shape[2], g.shape[1] * g.shape[2], g.shape[2], 1, 8, 0, _lib.float_array([0.1] * 8), None, 0, None, 0, 0,
        0, None,
    )
    assert rc == _lib.CTA_EINVAL
    msg = lib.cta_last_error().decode()
    assert "scratch" in msg and "caller-provided workspace" in msg
