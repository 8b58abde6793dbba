"""[B, D, L] kernel API (reference kernels/diffusion_triton.py entry points) vs the oracle."""
from __future__ import annotations

import pytest
import torch

from conftest import assert_close, contracted
from oracle import diffusion_oracle as O

pytestmark = pytest.mark.gpu

DTYPES = [torch.float32, torch.bfloat16, torch.float16]


def _api():
    from cta_b200 import diffusion as D
    return D


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("steps", [1, 2, 3, 4, 5, 6, 7, 8])
def test_fused_bitexact(dtype, steps):
    # reference test shape (tests/test_diffusion_triton_fused.py:27-41) plus every step count
    torch.manual_seed(0)
    x = torch.randn(2, 32, 1024, dtype=dtype)
    y = _api().diffusion_triton_fused(x.cuda(), alpha=0.1, steps=steps)
    ref = O.steps_bdl(x, alpha=0.1, steps=steps, contracted=contracted(dtype))
    assert y.dtype == dtype and y.shape == x.shape
    assert torch.equal(y.cpu(), ref), (y.cpu().float() - ref.float()).abs().max()
    # the exact arithmetic: bit for bit the reference's PyTorch path in every dtype
    from cta_b200 import ops
    ye = ops.bdl_simple(x.cuda(), 0.1, steps, arith="exact")
    assert torch.equal(ye.cpu(), O.steps_bdl(x, alpha=0.1, steps=steps))


@pytest.mark.parametrize("shape", [(1, 8, 257), (2, 3, 17), (1, 1, 3), (3, 5, 1000), (2, 4, 4096), (1, 2, 481),
                                   (2, 7, 241), (1, 3, 250)])
@pytest.mark.parametrize("steps", [1, 2, 4, 8])
def test_fused_shapes(shape, steps):
    torch.manual_seed(1)
    for dtype in (torch.float32, torch.bfloat16):
        x = torch.randn(*shape, dtype=dtype)
        y = _api().diffusion_triton_fused(x.cuda(), alpha=0.1, steps=steps)
        assert torch.equal(y.cpu(), O.steps_bdl(x, alpha=0.1, steps=steps, contracted=contracted(dtype)))


def test_noncontiguous_input():
    torch.manual_seed(2)
    base = torch.randn(2, 64, 300, device="cuda")
    x = base[:, ::2, :]  # non-contiguous view
    y = _api().diffusion_triton_fused(x, alpha=0.1, steps=4)
    assert torch.equal(y.cpu(), O.steps_bdl(x.cpu(), alpha=0.1, steps=4))


@pytest.mark.parametrize("L", [1, 2])
def test_short_sequence_identity(L):
    D = _api()
    x = torch.randn(2, 3, L, device="cuda")
    assert D.diffusion_triton_fused(x, steps=4) is x          # :846-847 returns x
    y = D.diffusion_step_triton(x)                            # :753-754 returns a clone
    assert y is not x and torch.equal(y, x)
    assert D.diffusion_step_triton_backward(x) is x           # :783-784 returns grad_out


def test_steps_zero_alias():
    x = torch.randn(1, 2, 10, device="cuda")
    assert _api().diffusion_triton_fused(x, steps=0) is x


def test_errors():
    D = _api()
    with pytest.raises(ValueError):
        D.diffusion_triton_fused(torch.randn(2, 3, 10), steps=2)       # CPU tensor
    with pytest.raises(ValueError):
        D.diffusion_triton_fused(torch.randn(3, 10, device="cuda"), steps=2)
    with pytest.raises(ValueError):
        D.diffusion_triton_fused(torch.randn(1, 3, 10, device="cuda"), steps=-1)
    with pytest.raises(ValueError):
        D.diffusion_triton_fused(torch.randn(1, 3, 10, device="cuda"), steps=9)
    with pytest.raises(ValueError):
        D.diffusion_step_triton_backward(torch.randn(2, 10, device="cuda"))


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_unfused_loop_rounds_each_step(dtype):
    torch.manual_seed(3)
    x = torch.randn(2, 16, 333, dtype=dtype)
    y = _api().diffusion_triton(x.cuda(), alpha=0.1, steps=4)
    ref = x
    for _ in range(4):
        ref = O.step_bdl(ref, alpha=0.1, contracted=contracted(dtype))
    assert torch.equal(y.cpu(), ref)


@pytest.mark.parametrize("L", [1, 2, 3, 4, 17, 1024])
def test_step_backward_matches_autograd(L):
    # tests/test_diffusion_triton_backward.py:20-43
    torch.manual_seed(0)
    x = torch.randn(2, 4, L, dtype=torch.float32)
    g = torch.randn_like(x)
    xg = x.cuda().requires_grad_(True)
    y = _api().diffusion_step_triton(xg, alpha=0.1)
    (y * g.cuda()).sum().backward()
    dx_ref, _ = O.grads(lambda t: O.steps_bdl(t, alpha=0.1, steps=1), x, g)
    torch.testing.assert_close(xg.grad.cpu(), dx_ref, rtol=1e-5, atol=1e-5)


@pytest.mark.parametrize("steps", [1, 2, 3, 4, 5, 6, 7, 8])
@pytest.mark.parametrize("shape", [(2, 8, 33), (1, 4, 1024), (2, 3, 250)])
def test_fused_backward_matches_autograd(steps, shape):
    # tests/test_diffusion_triton_backward.py:46-69, every step count, one fused launch
    torch.manual_seed(0)
    x = torch.randn(*shape, dtype=torch.float32)
    g = torch.randn_like(x)
    xg = x.cuda().requires_grad_(True)
    y = _api().diffusion_triton_fused(xg, alpha=0.1, steps=steps)
    (y * g.cuda()).sum().backward()
    dx_ref, _ = O.grads(lambda t: O.steps_bdl(t, alpha=0.1, steps=steps), x, g)
    assert_close(xg.grad, dx_ref)


def test_bf16_backward_tolerance():
    torch.manual_seed(5)
    x = torch.randn(1, 8, 2048, dtype=torch.bfloat16)
    g = torch.randn_like(x)
    xg = x.cuda().requires_grad_(True)
    y = _api().diffusion_triton_fused(xg, alpha=0.1, steps=8)
    (y.float() * g.cuda().float()).sum().backward()
    dx_ref, _ = O.grads(lambda t: O.steps_bdl(t, alpha=0.1, steps=8), x, g)
    assert_close(xg.grad, dx_ref)


@pytest.mark.parametrize("causal", [False, True])
@pytest.mark.parametrize("backward", [False, True])
@pytest.mark.parametrize("use_mask", [False, True])
@pytest.mark.parametrize("shape,dtype", [((1, 3, 4096), torch.bfloat16), ((2, 5, 2000), torch.float32),
                                         ((1, 1, 65536), torch.bfloat16), ((3, 2, 240), torch.float32)])
def test_tma_form_matches_oracle(causal, backward, use_mask, shape, dtype):
    """Row-aligned [B, D, L] tensors take the TMA pipeline form (two rows per CTA,
    consecutive 240-position windows): odd row counts, several windows per CTA,
    one-window rows, per-step alphas, causal stencils, masks, the adjoint."""
    from cta_b200 import _lib, ops

    torch.manual_seed(12)
    B, D, L = shape
    steps = 4
    al = [0.1, 0.05, 0.12, 0.02]
    x = torch.randn(B, D, L).to(dtype)
    mask = None
    if use_mask:
        mask = torch.ones(B, L, dtype=torch.long)
        mask[-1, L - L // 3 :] = 0
        mask[0, L // 5] = 0
    kw = dict(layout="bdl", causal=causal, attention_mask=mask)
    y = ops.bdl(x.cuda(), al, steps, causal=causal, backward=backward, mask=None if mask is None else mask.cuda())
    if not backward:
        assert torch.equal(y.cpu(), O.fused_stack(x, al, **kw, contracted=contracted(dtype)))
    else:
        # the adjoint is applied to x itself as the gradient; reference in fp32
        dx_ref, _ = O.grads(lambda t: O.fused_stack(t, al, **kw), torch.randn(B, D, L), x.float())
        assert_close(y, dx_ref)
    assert _lib.device_error() == 0
