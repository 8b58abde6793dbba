"""The oracle reproduces the reference's own outputs (golden fixtures made by
tests/golden/make_golden.py from the reference source) -- CPU only."""
from __future__ import annotations

import hashlib

import pytest
import torch

from oracle import diffusion_oracle as O


def _sha(t: torch.Tensor) -> str:
    t = t.detach().contiguous()
    if t.dtype == torch.bfloat16:
        t = t.view(torch.int16)
    return hashlib.sha256(t.numpy().tobytes()).hexdigest()


def test_step_bdl_bitexact(golden):
    for c in golden["step_bdl"]:
        y = O.step_bdl(c["x"], alpha=c["alpha"])
        assert y.dtype == c["y"].dtype and torch.equal(y, c["y"])


def test_steps_bdl_bitexact(golden):
    for c in golden["steps_bdl"]:
        y = O.steps_bdl(c["x"], alpha=c["alpha"], steps=c["steps"])
        assert y.dtype == c["y"].dtype and torch.equal(y, c["y"]), (c["x"].dtype, c["steps"])


def test_steps_bld_bitexact(golden):
    for c in golden["steps_bld"]:
        y = O.steps_bld(c["x"], alpha=c["alpha"], steps=c["steps"])
        assert torch.equal(y, c["y"])


def test_layer_chain_bitexact_and_grads(golden):
    for c in golden["layer_chain"]:
        kw = dict(layout=c["layout"], causal=c["causal"], attention_mask=c["mask"])
        y = O.layer_chain(c["x"], c["alphas"], **kw)
        assert torch.equal(y, c["y"]), (c["layout"], c["causal"], c["mask"] is not None, c["x"].dtype)
        alphas = [torch.tensor([a]) for a in c["alphas"]]
        dx, das = O.grads(lambda x, *al: O.layer_chain(x, list(al), **kw), c["x"], c["g"], alphas)
        torch.testing.assert_close(dx.float(), c["dx"].float(), rtol=1e-6, atol=1e-6)
        torch.testing.assert_close(torch.cat(das), c["dalpha"], rtol=1e-5, atol=1e-5)


def test_mixer_packed_bitexact(golden):
    for c in golden["mixer_packed"]:
        y = O.mixer_packed(c["x"], c["qsl"], c["max_len"], alpha=c["alpha"], steps=c["steps"])
        assert torch.equal(y, c["y"])


def test_step_adjoint(golden):
    for c in golden["step_adjoint"]:
        dx = O.step_adjoint_bdl(c["g"], alpha=c["alpha"])
        torch.testing.assert_close(dx, c["dx"], rtol=1e-6, atol=1e-6)


def test_fused_stack_equals_reference_ops_in_fp32(golden):
    # fused stack keeps fp32 between layers: identical to the layer chain in fp32
    for c in golden["layer_chain"]:
        if c["x"].dtype != torch.float32:
            continue
        kw = dict(layout=c["layout"], causal=c["causal"], attention_mask=c["mask"])
        assert torch.equal(O.fused_stack(c["x"], c["alphas"], **kw), c["y"])


@pytest.mark.parametrize("idx", [0, 1, 2])
def test_c1_full_config(golden, idx):
    """Oracle configuration at full size: fp32 [2, 1024, 512], steps {1, 2, 4}."""
    meta = golden["c1_full"]
    c = meta["cases"][idx]
    torch.manual_seed(meta["seed_x"])
    x = torch.randn(*meta["shape"], dtype=torch.float32)
    torch.manual_seed(meta["seed_g"])
    g = torch.randn(*meta["shape"], dtype=torch.float32)
    y = O.steps_bld(x, alpha=meta["alpha"], steps=c["steps"])
    assert _sha(y) == c["y_sha256"]
    dx, _ = O.grads(lambda t: O.steps_bld(t, alpha=meta["alpha"], steps=c["steps"]), x, g)
    torch.testing.assert_close(dx[:, [0, 1, 2, 511, 1021, 1022, 1023], :], c["dx_rows"], rtol=1e-6, atol=1e-6)


def test_window_oracle_matches_full():
    torch.manual_seed(7)
    x = torch.randn(1, 300, 8)
    full = O.steps_bld(x, alpha=0.1, steps=8)
    for a, b in [(0, 40), (100, 180), (250, 300)]:
        lo, hi = max(0, a - 8), min(300, b + 8)
        w = O.window_bld(x[:, lo:hi], win_start=lo, global_len=300, out_start=a, out_stop=b, alpha=0.1, steps=8)
        assert torch.equal(w, full[:, a:b])


@pytest.mark.parametrize("causal", [False, True])
def test_window_grads_oracle_matches_full(causal):
    """Per-window dx rows and row-restricted d(alpha) sums add up to the full
    autograd gradients of the fused stack (the checker of the sharded backward)."""
    torch.manual_seed(8)
    B, L, D, al = 2, 90, 6, [0.1, 0.05, 0.12, 0.02]
    x, g = torch.randn(B, L, D), torch.randn(B, L, D)
    dx_ref, da_ref = O.grads(lambda t, *a: O.fused_stack(t, list(a), layout="bld", causal=causal), x, g,
                             [torch.tensor([v]) for v in al])
    da_ref = torch.cat(da_ref)
    h = 2 * len(al) if causal else len(al)
    dxs, das = [], torch.zeros(len(al), dtype=torch.float64)
    for a, b in [(0, 31), (31, 32), (32, 90)]:
        lo, hi = max(0, a - h), min(L, b + h)
        dx, da = O.window_bld_grads(g[:, lo:hi], x[:, lo:hi], win_start=lo, global_len=L, out_start=a, out_stop=b,
                                    alphas=al, causal=causal)
        dxs.append(dx)
        das += da
    torch.testing.assert_close(torch.cat(dxs, 1), dx_ref, rtol=1e-6, atol=1e-6)
    torch.testing.assert_close(das.float(), da_ref, rtol=1e-5, atol=1e-5)


def test_pde_layer_step_matches_reference(golden):
    """Advection- and reaction-diffusion layers: forward bit for bit, gradients
    (dx, d(alpha), d(beta)) to 1e-6, against the reference's own layers."""
    for c in golden["pde_step"]:
        kw = dict(layout=c["layout"], causal=c["causal"], attention_mask=c["mask"])
        y = O.pde_layer_step(c["x"], c["kind"], c["alpha"], c["beta"], **kw)
        assert torch.equal(y, c["y"]), (c["kind"], c["layout"], c["causal"], c["x"].dtype)
        dx, (da, db) = O.grads(lambda t, a, b: O.pde_layer_step(t, c["kind"], a, b, **kw), c["x"], c["g"],
                               [torch.tensor([c["alpha"]]), torch.tensor([c["beta"]])])
        tol = 1e-6 if c["x"].dtype == torch.float32 else 1e-2
        torch.testing.assert_close(dx.float(), c["dx"].float(), rtol=tol, atol=tol)
        torch.testing.assert_close(da, c["dalpha"], rtol=1e-5, atol=1e-5)
        torch.testing.assert_close(db, c["dbeta"], rtol=1e-5, atol=1e-5)
