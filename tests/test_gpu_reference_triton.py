"""Parity against the reference's own GPU kernels, run on the same GPU.

The reference's Triton kernels (kernels/diffusion_triton.py) and its vLLM
mixer (src/cta/serving_vllm.py) are imported unmodified from baseline/_ref
(placed there by baseline/install_reference.py) and JIT-compiled by Triton.
The default arithmetic for 16-bit tensors (the contracted update
c + alpha*lap as one fma, lap = (r - 2c) + l with the first two as one fma) is
meant to be the op order those kernels compile to, so bf16 / fp16 outputs must
be bit-identical to theirs:

  * diffusion_triton_fused, steps 2 / 4 / 8 (:829-868 and the s2/s4/s8 kernels);
  * diffusion_step_triton and the per-step-rounding loop diffusion_triton
    (:732-762, :812-826);
  * the post-attention mixer, dense [B, L, D] (transpose + Triton + transpose
    in the reference) and packed with mixed prefill / decode lengths.

fp32 stays in the exact arithmetic (the reference's PyTorch op order), so
fp32 outputs agree with the Triton kernels to fp32 rounding, and the adjoint
(the reference evaluates (1 - 2a) g + a (g[i-1] + g[i+1]), a different op
order) to the 16-bit bar.  Skipped when the reference install is absent.
"""
from __future__ import annotations

import sys
from pathlib import Path
from types import SimpleNamespace

import pytest
import torch

pytestmark = pytest.mark.gpu

REF_DIR = Path(__file__).resolve().parents[1] / "baseline" / "_ref"


@pytest.fixture(scope="module")
def ref():
    if not (REF_DIR / "kernels" / "diffusion_triton.py").is_file():
        pytest.skip("no reference install under baseline/_ref")
    if str(REF_DIR) not in sys.path:
        sys.path.append(str(REF_DIR))
    import cta.serving_vllm as sv
    import kernels.diffusion_triton as kt

    if getattr(kt, "triton", None) is None:
        pytest.skip("triton is not importable")
    return SimpleNamespace(kt=kt, sv=sv)


def _ours():
    from cta_b200 import diffusion, serving_vllm

    return diffusion, serving_vllm


SHAPES = [(2, 48, 1000), (1, 64, 4099), (3, 8, 5)]


@pytest.mark.parametrize("shape", SHAPES)
@pytest.mark.parametrize("steps", [2, 4, 8])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_fused_bit_identical_to_triton(ref, shape, steps, dtype):
    ours, _ = _ours()
    torch.manual_seed(steps + shape[2])
    x = (2.0 * torch.randn(*shape, device="cuda")).to(dtype)
    for alpha in (0.1, 0.23):
        want = ref.kt.diffusion_triton_fused(x, alpha=alpha, steps=steps)
        got = ours.diffusion_triton_fused(x, alpha=alpha, steps=steps)
        assert torch.equal(got, want), (alpha, (got.float() - want.float()).abs().max().item())


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_step_and_loop_bit_identical_to_triton(ref, dtype):
    ours, _ = _ours()
    torch.manual_seed(3)
    x = torch.randn(2, 40, 1537, device="cuda").to(dtype)
    assert torch.equal(ours.diffusion_step_triton(x, alpha=0.1), ref.kt.diffusion_step_triton(x, alpha=0.1))
    assert torch.equal(ours.diffusion_triton(x, alpha=0.1, steps=3), ref.kt.diffusion_triton(x, alpha=0.1, steps=3))


def test_fp32_within_rounding_of_triton(ref):
    """fp32 runs the reference's PyTorch op order; Triton contracts: the two
    differ by fp32 roundings only."""
    ours, _ = _ours()
    torch.manual_seed(4)
    x = torch.randn(2, 32, 2000, device="cuda")
    for steps in (2, 4, 8):
        want = ref.kt.diffusion_triton_fused(x, alpha=0.1, steps=steps)
        got = ours.diffusion_triton_fused(x, alpha=0.1, steps=steps)
        torch.testing.assert_close(got, want, rtol=1e-5, atol=1e-5)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_adjoint_matches_triton_backward(ref, dtype):
    ours, _ = _ours()
    torch.manual_seed(5)
    g = torch.randn(2, 24, 999, device="cuda").to(dtype)
    want = ref.kt.diffusion_step_triton_backward(g, alpha=0.1).float()
    got = ours.diffusion_step_triton_backward(g, alpha=0.1).float()
    tol = 1e-5 if dtype == torch.float32 else 2e-2
    assert (got - want).abs().max().item() <= tol * max(1.0, want.abs().max().item())


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_mixer_bit_identical_to_reference_mixer(ref, dtype):
    """The reference mixer (use_triton=True, the default) against ours, dense
    [B, L, D] and packed (prefills, decodes and a two-row speculative decode)."""
    _, ours_sv = _ours()
    torch.manual_seed(6)
    ref_m = ref.sv.CtaPostAttnMixer(ref.sv.CtaConfig(steps=4, alpha=0.1, trace=False))
    our_m = ours_sv.CtaPostAttnMixer(ours_sv.CtaConfig(steps=4, alpha=0.1, trace=False))
    x = torch.randn(2, 777, 96, device="cuda").to(dtype)
    assert torch.equal(our_m(x, is_prefill=True), ref_m(x, is_prefill=True))
    lens = [700, 1, 1, 300, 2, 41]
    qsl = torch.zeros(len(lens) + 1, dtype=torch.int32)
    qsl[1:] = torch.cumsum(torch.tensor(lens), 0)
    md = SimpleNamespace(query_start_loc=qsl.cuda(), max_query_len=max(lens))
    xp = torch.randn(int(qsl[-1]), 96, device="cuda").to(dtype)
    assert torch.equal(our_m(xp, attn_metadata=md, is_prefill=True), ref_m(xp, attn_metadata=md, is_prefill=True))
    for steps in (2, 8):
        ref_s = ref.sv.CtaPostAttnMixer(ref.sv.CtaConfig(steps=steps, alpha=0.1, trace=False))
        our_s = ours_sv.CtaPostAttnMixer(ours_sv.CtaConfig(steps=steps, alpha=0.1, trace=False))
        assert torch.equal(our_s(x, is_prefill=True), ref_s(x, is_prefill=True)), steps
