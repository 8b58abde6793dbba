"""Generate the golden fixtures that pin the oracle to the reference.

Runs the reference project's own PyTorch code (imported read-only from its
source tree) on seeded CPU inputs and stores inputs and outputs in
``golden.pt`` next to this script.  Large configurations are stored as the
SHA-256 of the output bytes plus the seed that regenerates the input.

    python tests/golden/make_golden.py --ref <reference checkout>

(or set CTA_REFERENCE_ROOT instead of passing --ref).

Only this script reads the reference; the tests and the GPU box use the
committed ``golden.pt``.
"""
from __future__ import annotations

import argparse
import hashlib
import os
import sys
from pathlib import Path
from types import SimpleNamespace

import torch

HERE = Path(__file__).resolve().parent


def sha(t: torch.Tensor) -> str:
    t = t.detach().contiguous()
    if t.dtype == torch.bfloat16:
        t = t.view(torch.int16)
    return hashlib.sha256(t.numpy().tobytes()).hexdigest()


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=os.environ.get("CTA_REFERENCE_ROOT"),
                    help="root of the reference checkout (default: $CTA_REFERENCE_ROOT)")
    args = ap.parse_args()
    if not args.ref:
        ap.error("pass --ref <reference checkout> or set CTA_REFERENCE_ROOT")
    ref = Path(args.ref)
    sys.path.insert(0, str(ref / "src"))
    sys.path.insert(0, str(ref))
    from cta.ops.diffusion import diffusion_step_reference, diffusion_steps_reference
    from cta.serving_vllm import CtaConfig, CtaPostAttnMixer, _diffusion_steps_bld
    from models.pde_layers import AdvectionDiffusionPDELayer, DiffusionPDELayer, ReactionDiffusionPDELayer

    torch.set_num_threads(1)
    G: dict = {"meta": {"generator": "tests/golden/make_golden.py", "torch": torch.__version__}}

    # 1. single step, boundary copy, L in {1,2,3,4,5,17} (tests/test_diffusion_reference.py:53-70 shapes)
    cases = []
    for dtype in (torch.float32, torch.bfloat16):
        for L in (1, 2, 3, 4, 5, 17):
            torch.manual_seed(0)
            x = torch.randn(2, 3, L, dtype=dtype)
            cases.append({"x": x, "alpha": 0.1, "y": diffusion_step_reference(x, alpha=0.1)})
    G["step_bdl"] = cases

    # 2. multi-step, round once, every step count 0..8
    cases = []
    for dtype in (torch.float32, torch.bfloat16, torch.float16):
        for steps in range(0, 9):
            torch.manual_seed(1)
            x = torch.randn(2, 8, 37, dtype=dtype)
            cases.append({"x": x, "alpha": 0.1, "steps": steps,
                          "y": diffusion_steps_reference(x, alpha=0.1, steps=steps)})
    G["steps_bdl"] = cases

    # 3. [B, L, D] mixer form
    cases = []
    for dtype in (torch.float32, torch.bfloat16):
        for steps in (1, 2, 3, 4, 8):
            torch.manual_seed(2)
            x = torch.randn(2, 29, 16, dtype=dtype)
            cases.append({"x": x, "alpha": 0.07, "steps": steps,
                          "y": _diffusion_steps_bld(x, alpha=0.07, steps=steps)})
    G["steps_bld"] = cases

    # 4. DiffusionPDELayer chains: layout x causal x mask x dtype, with gradients
    cases = []
    for layout in ("bld", "bdl"):
        for causal in (False, True):
            for use_mask in (False, True):
                for dtype in (torch.float32, torch.bfloat16):
                    torch.manual_seed(3)
                    B, L, D = 2, 23, 6
                    x = torch.randn(B, L, D) if layout == "bld" else torch.randn(B, D, L)
                    x = x.to(dtype)
                    mask = None
                    if use_mask:
                        mask = torch.ones(B, L, dtype=torch.long)
                        mask[0, 17:] = 0
                        mask[1, 5] = 0
                        mask[1, 20:] = 0
                    alphas = [0.1, 0.03, 0.12, 0.05]
                    layers = [DiffusionPDELayer(D, alpha_init=a, layout=layout, causal=causal) for a in alphas]
                    xr = x.clone().requires_grad_(True)
                    y = xr
                    for layer in layers:
                        y = layer(y, attention_mask=mask)
                    torch.manual_seed(4)
                    g = torch.randn(y.shape).to(dtype)
                    (y.float() * g.float()).sum().backward()
                    cases.append({
                        "layout": layout, "causal": causal, "mask": mask, "x": x, "alphas": alphas, "g": g,
                        "y": y.detach(), "dx": xr.grad.detach(),
                        "dalpha": torch.cat([l.alpha.grad.detach() for l in layers]),
                    })
    G["layer_chain"] = cases

    # 4b. the advection- and reaction-diffusion layers: one layer, with gradients
    cases = []
    for kind, cls in (("advection", AdvectionDiffusionPDELayer), ("reaction", ReactionDiffusionPDELayer)):
        for layout in ("bld", "bdl"):
            for causal in (False, True):
                for use_mask in (False, True):
                    for dtype in (torch.float32, torch.bfloat16):
                        torch.manual_seed(5)
                        B, L, D = 2, 23, 6
                        x = torch.randn(B, L, D) if layout == "bld" else torch.randn(B, D, L)
                        x = (2.0 * x).to(dtype)
                        mask = None
                        if use_mask:
                            mask = torch.ones(B, L, dtype=torch.long)
                            mask[0, 17:] = 0
                            mask[1, 5] = 0
                        layer = cls(D, alpha_init=0.12, beta_init=0.07, layout=layout, causal=causal)
                        xr = x.clone().requires_grad_(True)
                        y = layer(xr, attention_mask=mask)
                        torch.manual_seed(6)
                        g = torch.randn(y.shape).to(dtype)
                        (y.float() * g.float()).sum().backward()
                        cases.append({
                            "kind": kind, "layout": layout, "causal": causal, "mask": mask, "x": x, "alpha": 0.12,
                            "beta": 0.07, "g": g, "y": y.detach(), "dx": xr.grad.detach(),
                            "dalpha": layer.alpha.grad.detach().clone(), "dbeta": layer.beta.grad.detach().clone(),
                        })
    G["pde_step"] = cases

    # 5. packed prefill through the reference mixer's torch path
    cases = []
    for steps in (1, 2, 3, 4, 8):
        torch.manual_seed(5)
        lens = [5, 9, 3, 1, 2, 7]
        qsl = [0]
        for n in lens:
            qsl.append(qsl[-1] + n)
        x = torch.randn(qsl[-1], 16)
        mixer = CtaPostAttnMixer(CtaConfig(use_triton=False, steps=steps, alpha=0.1))
        md = SimpleNamespace(max_query_len=max(lens), query_start_loc=torch.tensor(qsl, dtype=torch.int32),
                             is_prefill=True)
        y = mixer(x, attn_metadata=md)
        cases.append({"x": x, "qsl": qsl, "max_len": max(lens), "steps": steps, "alpha": 0.1, "y": y})
    G["mixer_packed"] = cases

    # 6. adjoint of one step by autograd of the single-step reference
    cases = []
    for L in (1, 2, 3, 4, 17):
        torch.manual_seed(6)
        x = torch.randn(2, 4, L, requires_grad=True)
        g = torch.randn(2, 4, L)
        y = diffusion_steps_reference(x, alpha=0.1, steps=1)
        (y * g).sum().backward()
        cases.append({"g": g, "alpha": 0.1, "dx": x.grad.detach()})
    G["step_adjoint"] = cases

    # 7. the full oracle configuration: fp32 [B=2, L=1024, D=512] ~ N(0,1) seed 0,
    #    alpha 0.1, steps {1,2,4}, forward + backward with grad_out ~ N(0,1) seed 1
    c1 = []
    torch.manual_seed(0)
    x_bld = torch.randn(2, 1024, 512, dtype=torch.float32)
    torch.manual_seed(1)
    g_bld = torch.randn(2, 1024, 512, dtype=torch.float32)
    for steps in (1, 2, 4):
        xr = x_bld.transpose(1, 2).detach().requires_grad_(True)
        y = diffusion_steps_reference(xr, alpha=0.1, steps=steps)
        (y * g_bld.transpose(1, 2)).sum().backward()
        y_bld = y.detach().transpose(1, 2).contiguous()
        dx_bld = xr.grad.detach().transpose(1, 2).contiguous()
        c1.append({"steps": steps, "y_sha256": sha(y_bld), "dx_sha256": sha(dx_bld),
                   "y_rows": y_bld[:, [0, 1, 2, 511, 1021, 1022, 1023], :].clone(),
                   "dx_rows": dx_bld[:, [0, 1, 2, 511, 1021, 1022, 1023], :].clone()})
    G["c1_full"] = {"shape": [2, 1024, 512], "seed_x": 0, "seed_g": 1, "alpha": 0.1, "cases": c1}

    out = HERE / "golden.pt"
    torch.save(G, out)
    print(f"wrote {out} ({out.stat().st_size} bytes)")


if __name__ == "__main__":
    main()
