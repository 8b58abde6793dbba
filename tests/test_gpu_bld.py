"""[B, L, D] kernels (layers, mixer, varlen) vs the oracle."""
from __future__ import annotations

import pytest
import torch

from conftest import assert_close, contracted
from oracle import diffusion_oracle as O

pytestmark = pytest.mark.gpu

DTYPES = [torch.float32, torch.bfloat16, torch.float16]
# D multiple of 8 -> TMA path; odd / small D -> generic loader path
SHAPES = [(1, 4096, 512), (2, 1000, 96), (2, 37, 6), (1, 3, 8), (3, 129, 264), (1, 77, 513), (2, 50, 1)]


def _ops():
    from cta_b200 import ops
    return ops


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("steps", [1, 2, 3, 4, 5, 6, 7, 8])
def test_forward_bitexact(dtype, steps):
    torch.manual_seed(0)
    x = torch.randn(2, 1024, 512, dtype=dtype)
    y = _ops().bld_forward(x.cuda(), [0.1] * steps, steps)
    ref = O.steps_bld(x, alpha=0.1, steps=steps, contracted=contracted(dtype))
    assert torch.equal(y.cpu(), ref), (y.cpu().float() - ref.float()).abs().max()
    ye = _ops().bld_forward(x.cuda(), [0.1] * steps, steps, arith="exact")
    assert torch.equal(ye.cpu(), O.steps_bld(x, alpha=0.1, steps=steps))
    # the contracted update stays within one rounding of the output dtype
    if contracted(dtype):
        ex = O.steps_bld(x, alpha=0.1, steps=steps)
        assert (y.cpu().float() - ex.float()).abs().max().item() <= 2e-2


@pytest.mark.parametrize("shape", SHAPES)
@pytest.mark.parametrize("steps", [1, 2, 4, 8])
def test_forward_shapes(shape, steps):
    torch.manual_seed(1)
    for dtype in (torch.float32, torch.bfloat16):
        x = torch.randn(*shape, dtype=dtype)
        y = _ops().bld_forward(x.cuda(), [0.1] * steps, steps)
        assert torch.equal(y.cpu(), O.steps_bld(x, alpha=0.1, steps=steps, contracted=contracted(dtype))), (shape, dtype)


def test_forward_strided_rows():
    torch.manual_seed(2)
    base = torch.randn(2, 600, 512, device="cuda")
    x = base[:, ::2, :]  # row stride 2*D (TMA with a non-dense row stride)
    y = _ops().bld_forward(x, [0.1] * 4, 4)
    assert torch.equal(y.cpu(), O.steps_bld(x.cpu(), alpha=0.1, steps=4))


def _mask(B, L, device="cpu"):
    m = torch.ones(B, L, dtype=torch.long)
    if L > 10:
        m[0, L - 7:] = 0
        m[-1, 3] = 0
        m[-1, L // 2 : L // 2 + 2] = 0
    return m.to(device)


@pytest.mark.parametrize("causal", [False, True])
@pytest.mark.parametrize("use_mask", [False, True])
@pytest.mark.parametrize("steps", [1, 2, 4, 8])
@pytest.mark.parametrize("shape", [(2, 300, 512), (2, 23, 6), (3, 1500, 264)])
def test_stack_forward_causal_mask(causal, use_mask, steps, shape):
    torch.manual_seed(3)
    B, L, D = shape
    x = torch.randn(B, L, D)
    alphas = [0.1, 0.03, 0.12, 0.05, 0.08, 0.02, 0.11, 0.07][:steps]
    m = _mask(B, L) if use_mask else None
    y = _ops().bld_forward(x.cuda(), alphas, steps, causal=causal, mask=None if m is None else m.cuda())
    ref = O.fused_stack(x, alphas, layout="bld", causal=causal, attention_mask=m)
    assert torch.equal(y.cpu(), ref)


@pytest.mark.parametrize("mask_dtype", [torch.bool, torch.int32, torch.int64, torch.float32, torch.uint8])
def test_mask_dtypes(mask_dtype):
    torch.manual_seed(4)
    x = torch.randn(2, 64, 16)
    m = _mask(2, 64)
    y = _ops().bld_forward(x.cuda(), [0.1, 0.05], 2, mask=m.to(mask_dtype).cuda())
    assert torch.equal(y.cpu(), O.fused_stack(x, [0.1, 0.05], layout="bld", attention_mask=m))


def test_device_alpha_scalars():
    torch.manual_seed(5)
    x = torch.randn(2, 200, 64)
    al = [torch.tensor([0.1]), torch.tensor([0.05], dtype=torch.bfloat16), torch.tensor([0.2])]
    y = _ops().bld_forward(x.cuda(), [a.cuda() for a in al], 3)
    ref = O.fused_stack(x, [a.float() for a in al], layout="bld")
    assert torch.equal(y.cpu(), ref)


@pytest.mark.parametrize("causal", [False, True])
@pytest.mark.parametrize("use_mask", [False, True])
@pytest.mark.parametrize("steps", [1, 2, 3, 4, 5, 6, 7, 8])
@pytest.mark.parametrize("shape", [(2, 300, 512), (2, 23, 6), (1, 700, 264)])
def test_backward_dx_dalpha(causal, use_mask, steps, shape):
    torch.manual_seed(6)
    B, L, D = shape
    x = torch.randn(B, L, D)
    g = torch.randn(B, L, D)
    alphas = [0.1, 0.03, 0.12, 0.05, 0.08, 0.02, 0.11, 0.07][:steps]
    m = _mask(B, L) if use_mask else None
    kw = dict(layout="bld", causal=causal, attention_mask=m)
    dx_ref, da_ref = O.grads(lambda t, *al: O.fused_stack(t, list(al), **kw), x, g,
                             [torch.tensor([a]) for a in alphas])
    ops = _ops()
    mc = None if m is None else m.cuda()
    dx, da = ops.bld_backward(g.cuda(), alphas, steps, x=x.cuda(), causal=causal, mask=mc, need_dalpha=True)
    assert_close(dx, dx_ref)
    da_ref = torch.cat(da_ref)
    scale = max(1.0, da_ref.abs().max().item())
    assert (da.cpu() - da_ref).abs().max().item() <= 1e-4 * scale, (da.cpu(), da_ref)
    dx2, none = ops.bld_backward(g.cuda(), alphas, steps, causal=causal, mask=mc)
    assert none is None
    assert torch.equal(dx2, dx)


def test_backward_dalpha_repeatable():
    torch.manual_seed(7)
    x = torch.randn(1, 4096, 512, device="cuda")
    g = torch.randn(1, 4096, 512, device="cuda")
    ops = _ops()
    r1 = ops.bld_backward(g, [0.1] * 4, 4, x=x, need_dalpha=True)[1].clone()
    r2 = ops.bld_backward(g, [0.1] * 4, 4, x=x, need_dalpha=True)[1].clone()
    assert torch.equal(r1, r2)  # deterministic reduction, workspace reusable


def test_out_buffers():
    """Caller-provided outputs: written in place and checked for shape and dtype."""
    torch.manual_seed(8)
    ops = _ops()
    x = torch.randn(2, 300, 264, device="cuda", dtype=torch.bfloat16)
    g = torch.randn_like(x)
    y = torch.full_like(x, 7.0)
    assert ops.bld_forward(x, [0.1] * 4, 4, out=y) is y
    assert torch.equal(y, ops.bld_forward(x, [0.1] * 4, 4))
    dx = torch.full_like(x, 7.0)
    r, _ = ops.bld_backward(g, [0.1] * 4, 4, out=dx)
    assert r is dx and torch.equal(dx, ops.bld_backward(g, [0.1] * 4, 4)[0])
    xt = x.transpose(1, 2).contiguous()
    yt = torch.empty_like(xt)
    assert ops.bdl_simple(xt, 0.1, 4, out=yt) is yt
    assert torch.equal(yt, ops.bdl_simple(xt, 0.1, 4))
    with pytest.raises(ValueError):
        ops.bld_forward(x, [0.1] * 4, 4, out=torch.empty(2, 300, 263, device="cuda", dtype=torch.bfloat16))
    with pytest.raises(ValueError):
        ops.bld_backward(g, [0.1] * 4, 4, out=torch.empty_like(x, dtype=torch.float32))
    with pytest.raises(ValueError):
        ops.bdl_simple(xt, 0.1, 4, out=torch.empty_like(x).transpose(1, 2))


@pytest.mark.parametrize("causal", [False, True])
def test_dalpha_tiling_invariance(causal):
    """d(alpha) through more CTAs than first-level reduction groups of 32 can
    hold (65536 CTAs, groups of 64), against the default tiling: dx bit-identical,
    d(alpha) equal up to the summation order (fp32 [32, 65536, 128])."""
    from cta_b200 import _lib
    torch.manual_seed(9)
    ops = _ops()
    B, L, D = 32, 65536, 128
    # coherent data (a periodic parabola along L, a positive gradient), so that
    # d(alpha) is not a cancelling sum and its rounding stays near fp32 epsilon
    rows = (torch.arange(L, device="cuda", dtype=torch.float32) % 64 - 32) ** 2 / 1024
    x = (rows[None, :, None] + 1e-3 * torch.randn(B, L, D, device="cuda")).contiguous()
    g = torch.rand_like(x)
    al = [0.1, 0.05, 0.12, 0.02]
    prev = _lib.set_tuning(1, 32)
    try:
        dx1, da1 = ops.bld_backward(g, al, 4, x=x, causal=causal, need_dalpha=True)
    finally:
        _lib.set_tuning(1, prev)
    dx2, da2 = ops.bld_backward(g, al, 4, x=x, causal=causal, need_dalpha=True)
    assert torch.equal(dx1, dx2)
    assert (da1 - da2).abs().max().item() <= 1e-5 * da2.abs().max().item(), (da1, da2)
    assert _lib.device_error() == 0


@pytest.mark.parametrize("steps", [1, 2, 3, 4, 8])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_varlen_reference_rule(steps, dtype):
    torch.manual_seed(8)
    lens = [5, 9, 3, 1, 2, 7, 40, 300, 33]
    qsl = [0]
    for n in lens:
        qsl.append(qsl[-1] + n)
    x = torch.randn(qsl[-1], 64).to(dtype)
    cu = torch.tensor(qsl, dtype=torch.int32, device="cuda")
    y = _ops().varlen_forward(x.cuda(), cu, max(lens), 0.1, steps, pad_to_max=True)
    assert torch.equal(y.cpu(), O.mixer_packed(x, qsl, max(lens), alpha=0.1, steps=steps,
                                               contracted=contracted(dtype)))


@pytest.mark.parametrize("steps", [1, 2, 4, 8])
def test_varlen_sequence_rule(steps):
    torch.manual_seed(9)
    lens = [5, 9, 3, 1, 2, 7, 40, 300, 33, 0, 17]
    qsl = [0]
    for n in lens:
        qsl.append(qsl[-1] + n)
    x = torch.randn(qsl[-1], 264)
    cu = torch.tensor(qsl, dtype=torch.int32, device="cuda")
    y = _ops().varlen_forward(x.cuda(), cu, max(lens), 0.1, steps, pad_to_max=False)
    assert torch.equal(y.cpu(), O.varlen_per_sequence(x, qsl, alpha=0.1, steps=steps))


def test_varlen_golden(golden):
    for c in golden["mixer_packed"]:
        cu = torch.tensor(c["qsl"], dtype=torch.int32, device="cuda")
        # the goldens are the reference's PyTorch path: the exact arithmetic
        y = _ops().varlen_forward(c["x"].cuda(), cu, c["max_len"], c["alpha"], c["steps"], pad_to_max=True,
                                  arith="exact")
        assert torch.equal(y.cpu(), c["y"])


# ---------------------------------------------------------------------------
# fused residual add (the decoder layer's `residual + mixer(attn_output)`)
# ---------------------------------------------------------------------------
@pytest.mark.parametrize("steps", [1, 2, 4, 5, 8])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32, torch.float16])
@pytest.mark.parametrize("pad", [True, False])
def test_varlen_residual_equals_two_pass(steps, dtype, pad):
    """One launch of residual + stencil equals the two-pass result bit for bit,
    and the reference rule equals the reference mixer + torch add."""
    torch.manual_seed(20 + steps)
    ops = _ops()
    lens = [700, 3, 1, 0, 257, 64, 1999]
    qsl = [0]
    for n in lens:
        qsl.append(qsl[-1] + n)
    T, D = qsl[-1], 264
    x = torch.randn(T, D).to(dtype)
    r = torch.randn(T, D).to(dtype)
    cu = torch.tensor(qsl, dtype=torch.int32, device="cuda")
    y1 = ops.varlen_forward(x.cuda(), cu, max(lens), 0.1, steps, pad_to_max=pad, residual=r.cuda())
    y2 = r.cuda() + ops.varlen_forward(x.cuda(), cu, max(lens), 0.1, steps, pad_to_max=pad)
    assert torch.equal(y1, y2)
    if pad:
        ref = r + O.mixer_packed(x, qsl, max(lens), alpha=0.1, steps=steps, contracted=contracted(dtype))
        assert torch.equal(y1.cpu(), ref)


@pytest.mark.parametrize("shape", [(2, 1000, 512), (1, 77, 513), (3, 129, 264), (2, 3, 8)])
@pytest.mark.parametrize("use_mask", [False, True])
def test_bld_residual_equals_two_pass(shape, use_mask):
    torch.manual_seed(21)
    ops = _ops()
    B, L, D = shape
    for dtype in (torch.bfloat16, torch.float32):
        x = torch.randn(B, L, D, device="cuda").to(dtype)
        base = torch.randn(B, L, D + 8, device="cuda").to(dtype)
        r = base[:, :, :D]  # rows with their own stride
        m = _mask(B, L, "cuda") if use_mask else None
        al = [0.1, 0.05, 0.12, 0.02]
        y1 = ops.bld_forward(x, al, 4, mask=m, residual=r)
        y2 = r + ops.bld_forward(x, al, 4, mask=m)
        assert torch.equal(y1, y2), (shape, dtype)


def test_bld_residual_rejects_causal_and_device_alphas():
    ops = _ops()
    x = torch.randn(1, 64, 32, device="cuda")
    with pytest.raises(ValueError):
        ops.bld_forward(x, [0.1] * 2, 2, causal=True, residual=x)
    with pytest.raises(ValueError):
        ops.bld_forward(x, [torch.tensor([0.1], device="cuda")], 1, residual=x)


@pytest.mark.parametrize("varlen_mode", ["reference", "sequence"])
def test_mixer_residual(varlen_mode):
    """CtaPostAttnMixer(..., residual=r) returns r + mixer(x): fused on the packed
    and [B, L, D] prefill paths, a plain add when the mixer is gated off."""
    from types import SimpleNamespace

    from cta_b200.serving_vllm import CtaConfig, CtaPostAttnMixer

    torch.manual_seed(22)
    mixer = CtaPostAttnMixer(CtaConfig(steps=4, alpha=0.1, varlen_mode=varlen_mode, trace=False))
    lens = [300, 41, 1200]
    qsl = torch.tensor([0, 300, 341, 1541], dtype=torch.int32, device="cuda")
    x = torch.randn(1541, 512, device="cuda", dtype=torch.bfloat16)
    r = torch.randn_like(x)
    md = SimpleNamespace(max_query_len=max(lens), query_start_loc=qsl, is_prefill=True)
    assert torch.equal(mixer(x, attn_metadata=md, residual=r), r + mixer(x, attn_metadata=md))
    decode = SimpleNamespace(max_query_len=1, query_start_loc=qsl, is_prefill=False)
    assert torch.equal(mixer(x, attn_metadata=decode, residual=r), r + x)
    x3 = torch.randn(2, 700, 512, device="cuda", dtype=torch.bfloat16)
    r3 = torch.randn_like(x3)
    assert torch.equal(mixer(x3, is_prefill=True, residual=r3), r3 + mixer(x3, is_prefill=True))
    long_mixer = CtaPostAttnMixer(CtaConfig(steps=11, alpha=0.1, max_steps=16, trace=False))
    assert torch.equal(long_mixer(x3, is_prefill=True, residual=r3), r3 + long_mixer(x3, is_prefill=True))


def test_bounded_wait_runs_out_reports_and_recovers():
    """The timeout path of the pipeline waits, on demand: with the test hook
    (tuning key 5) the first CTA waits 1 ms on an mbarrier phase that nothing
    completes, sets the device error word, drains the loads it issued and exits.
    The call returns, the error reads 1 and clears, the other tiles are right,
    and the next call is bit-exact."""
    from cta_b200 import _lib

    lib = _lib.load()
    torch.manual_seed(9)
    x = torch.randn(1, 4096, 512, dtype=torch.bfloat16)
    ref = O.steps_bld(x, alpha=0.1, steps=4, contracted=True)
    xd = x.cuda()
    torch.cuda.synchronize()
    assert lib.cta_device_error(1) == 0
    prev = lib.cta_set_tuning(5, 1000)
    try:
        y = _ops().bld_forward(xd, [0.1] * 4, 4)
        torch.cuda.synchronize()
    finally:
        lib.cta_set_tuning(5, prev)
    assert lib.cta_device_error(1) == 1
    assert lib.cta_device_error(0) == 0
    # the stalled CTA owns row tile 0 of column tile 0; every other column is written
    assert torch.equal(y[:, :, 128:].cpu(), ref[:, :, 128:])
    y2 = _ops().bld_forward(xd, [0.1] * 4, 4)
    assert torch.equal(y2.cpu(), ref)
    assert lib.cta_device_error(0) == 0


def test_arithmetic_modes_process_and_thread():
    """The process default (cta_b200.set_arithmetic) and the per-call override:
    bf16 follows them, fp32 is always exact, the layers always exact."""
    import threading

    import cta_b200
    from cta_b200.pde_layers import DiffusionPDELayer, diffusion_pde_stack

    torch.manual_seed(21)
    x = torch.randn(1, 1500, 264, dtype=torch.bfloat16)
    xd = x.cuda()
    exact = O.steps_bld(x, alpha=0.1, steps=4)
    contr = O.steps_bld(x, alpha=0.1, steps=4, contracted=True)
    assert not torch.equal(exact, contr)  # the inputs tell the two apart
    ops = _ops()
    assert cta_b200.set_arithmetic("exact") == "contracted"
    try:
        assert torch.equal(ops.bld_forward(xd, [0.1] * 4, 4).cpu(), exact)
        assert torch.equal(ops.bld_forward(xd, [0.1] * 4, 4, arith="contracted").cpu(), contr)
        # another thread sees the process default, not this thread's override
        seen = {}
        t = threading.Thread(target=lambda: seen.update(y=ops.bld_forward(xd, [0.1] * 4, 4).cpu()))
        t.start()
        t.join()
        assert torch.equal(seen["y"], exact)
    finally:
        assert cta_b200.set_arithmetic("contracted") == "exact"
    assert torch.equal(ops.bld_forward(xd, [0.1] * 4, 4).cpu(), contr)
    xf = x.float()
    assert torch.equal(ops.bld_forward(xf.cuda(), [0.1] * 4, 4).cpu(), O.steps_bld(xf, alpha=0.1, steps=4))
    layers = [DiffusionPDELayer(264, alpha_init=0.1, layout="bld").cuda() for _ in range(4)]
    with torch.no_grad():
        y = diffusion_pde_stack(xd, layers)
    assert torch.equal(y.cpu(), O.fused_stack(x, [0.1] * 4, layout="bld"))
    with pytest.raises(ValueError):
        ops.bld_forward(xd, [0.1] * 4, 4, arith="fast")


def _long_mask(B, L):
    """Masks whose long tiles hold every chunk form: a padded tail of 3000 rows
    and a 400-row hole (chunks with every tested row fixed), isolated one-row
    holes (per-row chunks) and long valid runs (branch-free chunks)."""
    m = torch.ones(B, L, dtype=torch.long)
    m[0, L - 3000 :] = 0
    m[0, 2000:2400] = 0
    m[-1, 517::700] = 0
    return m


@pytest.mark.parametrize("causal", [False, True])
@pytest.mark.parametrize("steps", [2, 4, 8])
@pytest.mark.parametrize("tile", [256, 1024])
def test_chunk_forms_in_masked_tiles(causal, steps, tile):
    """Tiles of 256 / 1024 rows (forced) with fixed rows: the forward bit for bit
    in both dtypes and the backward with d(alpha) against the oracle, so each
    of the three chunk forms runs next to the others in one tile."""
    from cta_b200 import _lib

    torch.manual_seed(30 + steps)
    B, L, D = 2, 8192, 64
    m = _long_mask(B, L)
    alphas = [0.1, 0.03, 0.12, 0.05, 0.08, 0.02, 0.11, 0.07][:steps]
    prev = _lib.set_tuning(1, tile)
    try:
        ops = _ops()
        for dtype in (torch.float32, torch.bfloat16):
            x = (2.0 * torch.randn(B, L, D)).to(dtype)
            y = ops.bld_forward(x.cuda(), alphas, steps, causal=causal, mask=m.cuda())
            ref = O.fused_stack(x, [torch.tensor([a]) for a in alphas], layout="bld", causal=causal,
                                attention_mask=m, contracted=contracted(dtype))
            assert torch.equal(y.cpu(), ref), dtype
        x = torch.randn(B, L, D)
        g = torch.randn(B, L, D)
        kw = dict(layout="bld", causal=causal, attention_mask=m)
        dx_ref, da_ref = O.grads(lambda t, *al: O.fused_stack(t, list(al), **kw), x, g,
                                 [torch.tensor([a]) for a in alphas])
        dx, da = ops.bld_backward(g.cuda(), alphas, steps, x=x.cuda(), causal=causal, mask=m.cuda(),
                                  need_dalpha=True)
        assert_close(dx, dx_ref)
        da_ref = torch.cat(da_ref)
        assert (da.cpu() - da_ref).abs().max().item() <= 1e-4 * max(1.0, da_ref.abs().max().item())
    finally:
        _lib.set_tuning(1, prev)
