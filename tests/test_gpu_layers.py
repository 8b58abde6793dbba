"""PDE layers, fused stacks, PDE Transformers and the vLLM mixer on the GPU."""
from __future__ import annotations

from types import SimpleNamespace

import pytest
import torch

from conftest import assert_close
from oracle import diffusion_oracle as O

pytestmark = pytest.mark.gpu


def test_layer_chain_matches_reference_golden(golden):
    """Each DiffusionPDELayer call is bit-identical to the reference layer (forward),
    so a chain of calls reproduces the reference chain; gradients within tolerance."""
    from cta_b200.pde_layers import DiffusionPDELayer

    for c in golden["layer_chain"]:
        x = c["x"].cuda().requires_grad_(True)
        D = x.shape[2] if c["layout"] == "bld" else x.shape[1]
        layers = [DiffusionPDELayer(D, alpha_init=a, layout=c["layout"], causal=c["causal"]).cuda()
                  for a in c["alphas"]]
        mask = None if c["mask"] is None else c["mask"].cuda()
        y = x
        for l in layers:
            y = l(y, attention_mask=mask)
        assert torch.equal(y.detach().cpu(), c["y"]), (c["layout"], c["causal"], c["mask"] is not None)
        (y.float() * c["g"].cuda().float()).sum().backward()
        assert_close(x.grad, c["dx"])
        da = torch.cat([l.alpha.grad for l in layers]).cpu()
        # d(alpha) is a reduction: relative bar; in bf16 every layer's input gradient is
        # rounded to bf16 (as in the reference), so earlier layers inherit 1-ulp differences
        rel = 1e-4 if c["x"].dtype == torch.float32 else 2e-2
        assert (da - c["dalpha"]).abs().max().item() <= rel * max(1.0, c["dalpha"].abs().max().item())


@pytest.mark.parametrize("layout", ["bld", "bdl"])
@pytest.mark.parametrize("causal", [False, True])
def test_fused_stack_forward_backward(layout, causal):
    from cta_b200.pde_layers import DiffusionPDELayer, diffusion_pde_stack

    torch.manual_seed(0)
    B, L, D = 2, 515, 64
    x = torch.randn(B, L, D) if layout == "bld" else torch.randn(B, D, L)
    g = torch.randn_like(x)
    m = torch.ones(B, L, dtype=torch.long)
    m[1, 400:] = 0
    alphas = [0.1, 0.05, 0.12, 0.02]
    layers = [DiffusionPDELayer(D, alpha_init=a, layout=layout, causal=causal).cuda() for a in alphas]
    xg = x.cuda().requires_grad_(True)
    y = diffusion_pde_stack(xg, layers, attention_mask=m.cuda())
    ref = O.fused_stack(x, alphas, layout=layout, causal=causal, attention_mask=m)
    assert torch.equal(y.detach().cpu(), ref)
    (y * g.cuda()).sum().backward()
    dx_ref, da_ref = O.grads(
        lambda t, *al: O.fused_stack(t, list(al), layout=layout, causal=causal, attention_mask=m), x, g,
        [torch.tensor([a]) for a in alphas])
    assert_close(xg.grad, dx_ref)
    da = torch.cat([l.alpha.grad for l in layers]).cpu()
    da_ref = torch.cat(da_ref)
    assert (da - da_ref).abs().max().item() <= 1e-4 * max(1.0, da_ref.abs().max().item())


def test_wave_layer_is_diffusion_with_alpha_squared():
    from cta_b200.pde_layers import create_pde_layer

    torch.manual_seed(1)
    x = torch.randn(2, 40, 8)
    layer = create_pde_layer("wave", 8, layout="bld").cuda()
    a = layer.alpha.detach().float().cpu() ** 2
    y = layer(x.cuda())
    assert torch.equal(y.cpu(), O.layer_step(x, a, layout="bld"))


@pytest.mark.parametrize("model", ["classifier", "lm"])
def test_pde_transformer_matches_layerwise_reference(model):
    """Same weights: fused-stack model vs. the same model refined layer by layer
    with the oracle's PDE math (fp32, Transformer parts identical)."""
    from cta_b200 import transformers as T

    torch.manual_seed(2)
    kw = dict(vocab_size=101, embed_dim=32, num_heads=4, hidden_dim=64, num_layers=2, pde_steps=3,
              max_length=64, dropout=0.0)
    if model == "classifier":
        net = T.PDETransformerClassifier(num_classes=3, **kw)
    else:
        net = T.PDETransformerLM(**kw)
    net = net.cuda().eval()
    ids = torch.randint(0, 101, (2, 50), device="cuda")
    mask = torch.ones(2, 50, dtype=torch.long, device="cuda")
    mask[1, 41:] = 0
    out = net(ids, mask)

    # reference forward with the oracle's layer chain in place of the fused stack
    causal = model == "lm"
    with torch.no_grad():
        x = net.embedding(ids) + net.pos_encoder[:, :50, :]
        if causal:
            pad = torch.zeros_like(mask, dtype=torch.float32).masked_fill(mask == 0, float("-inf"))
            cm = T.generate_causal_mask(50, x.device)
        for tl, plist in zip(net.transformer_layers, net.pde_layers):
            x = tl(x, src_mask=cm, src_key_padding_mask=pad) if causal else tl(x, src_key_padding_mask=mask == 0)
            xc = x.cpu()
            for p in plist:
                xc = O.layer_step(xc, p.alpha.detach().cpu(), layout="bld", causal=causal,
                                  attention_mask=mask.cpu())
            x = xc.cuda()
        if causal:
            ref = net.fc(x)
        else:
            em = mask.unsqueeze(-1).expand(x.size())
            ref = net.fc(torch.sum(x * em, 1) / torch.clamp(mask.sum(1, keepdim=True), min=1))
    torch.testing.assert_close(out.detach(), ref, rtol=1e-4, atol=1e-4)
    out.float().sum().backward()
    for plist in net.pde_layers:
        for p in plist:
            assert p.alpha.grad is not None and torch.isfinite(p.alpha.grad).all()


def test_state_dict_names_match_reference_layout():
    from cta_b200 import transformers as T

    net = T.PDETransformerLM(vocab_size=11, embed_dim=8, num_heads=2, hidden_dim=16, num_layers=2, pde_steps=4)
    names = [n for n in net.state_dict() if n.startswith("pde_layers")]
    assert names == [f"pde_layers.{i}.{k}.alpha" for i in range(2) for k in range(4)]


@pytest.mark.parametrize("layout", ["bld", "bdl"])
@pytest.mark.parametrize("steps", [1, 3, 4, 8])
def test_mixer_dense(layout, steps):
    from cta_b200.serving_vllm import CtaConfig, CtaPostAttnMixer

    torch.manual_seed(3)
    x = torch.randn(2, 257, 16) if layout == "bld" else torch.randn(2, 16, 257)
    x = x.to(torch.bfloat16)
    mixer = CtaPostAttnMixer(CtaConfig(steps=steps, alpha=0.1, layout=layout))
    y = mixer(x.cuda())
    # use_triton (default): the contracted update of the reference's Triton kernels
    ref = (O.steps_bld(x, alpha=0.1, steps=steps, contracted=True) if layout == "bld"
           else O.steps_bdl(x, alpha=0.1, steps=steps, contracted=True))
    assert torch.equal(y.cpu(), ref)
    # use_triton=False: the reference's PyTorch fallback, bit for bit
    ye = CtaPostAttnMixer(CtaConfig(steps=steps, alpha=0.1, layout=layout, use_triton=False))(x.cuda())
    ref = O.steps_bld(x, alpha=0.1, steps=steps) if layout == "bld" else O.steps_bdl(x, alpha=0.1, steps=steps)
    assert torch.equal(ye.cpu(), ref)
    # decode steps pass through untouched
    assert mixer(x.cuda(), is_prefill=False).data_ptr() != 0


def test_mixer_packed_reference_rule(golden):
    from cta_b200.serving_vllm import CtaConfig, CtaPostAttnMixer

    for c in golden["mixer_packed"]:
        # the goldens are the reference's PyTorch path (use_triton=False)
        mixer = CtaPostAttnMixer(CtaConfig(steps=c["steps"], alpha=c["alpha"], use_triton=False))
        md = SimpleNamespace(max_query_len=c["max_len"], is_prefill=True,
                             query_start_loc=torch.tensor(c["qsl"], dtype=torch.int32, device="cuda"))
        y = mixer(c["x"].cuda(), attn_metadata=md)
        assert torch.equal(y.cpu(), c["y"])


def test_mixer_packed_sequence_rule():
    from cta_b200.serving_vllm import CtaConfig, CtaPostAttnMixer

    torch.manual_seed(4)
    qsl = [0, 7, 9, 40, 41, 100]
    x = torch.randn(100, 32)
    mixer = CtaPostAttnMixer(CtaConfig(steps=4, alpha=0.1, varlen_mode="sequence"))
    md = SimpleNamespace(max_query_len=59, query_start_loc=qsl, num_prefill_tokens=100)
    y = mixer(x.cuda(), attn_metadata=md)
    assert torch.equal(y.cpu(), O.varlen_per_sequence(x, qsl, alpha=0.1, steps=4))


# ---------------------------------------------------------------------------
# advection- and reaction-diffusion layers (one kernel launch per step)
# ---------------------------------------------------------------------------
def _two_coef_layer(kind, D, layout, causal, alpha=0.12, beta=0.07):
    from cta_b200.pde_layers import AdvectionDiffusionPDELayer, ReactionDiffusionPDELayer

    cls = AdvectionDiffusionPDELayer if kind == "advection" else ReactionDiffusionPDELayer
    return cls(D, alpha_init=alpha, beta_init=beta, layout=layout, causal=causal).cuda()


def test_pde_step_layers_match_reference_golden(golden):
    """The reference's own layer outputs: advection bit for bit, reaction (its
    sigmoid uses the __expf and __fdividef intrinsics here) to the fp32 / bf16 bar; gradients within tolerance."""
    for c in golden["pde_step"]:
        D = c["x"].shape[2] if c["layout"] == "bld" else c["x"].shape[1]
        layer = _two_coef_layer(c["kind"], D, c["layout"], c["causal"], c["alpha"], c["beta"])
        x = c["x"].cuda().requires_grad_(True)
        mask = None if c["mask"] is None else c["mask"].cuda()
        y = layer(x, attention_mask=mask)
        tag = (c["kind"], c["layout"], c["causal"], c["mask"] is not None, c["x"].dtype)
        if c["kind"] == "advection":
            assert torch.equal(y.detach().cpu(), c["y"]), tag
        else:
            assert_close(y, c["y"])
        (y.float() * c["g"].cuda().float()).sum().backward()
        assert_close(x.grad, c["dx"])
        scale = max(1.0, c["dalpha"].abs().max().item(), c["dbeta"].abs().max().item())
        assert (layer.alpha.grad.cpu() - c["dalpha"]).abs().max().item() <= 1e-4 * scale, tag
        assert (layer.beta.grad.cpu() - c["dbeta"]).abs().max().item() <= 1e-4 * scale, tag


@pytest.mark.parametrize("kind", ["advection", "reaction"])
@pytest.mark.parametrize("layout", ["bld", "bdl"])
@pytest.mark.parametrize("causal", [False, True])
@pytest.mark.parametrize("shape", [(2, 1000, 512), (1, 77, 513), (3, 40, 6)])
def test_pde_step_layers_match_oracle(kind, layout, causal, shape):
    torch.manual_seed(13)
    B, L, D = shape
    for dtype in (torch.float32, torch.bfloat16):
        x = (2.0 * torch.randn(B, L, D)).to(dtype)
        if layout == "bdl":
            x = x.transpose(1, 2).contiguous()
        mask = torch.ones(B, L, dtype=torch.long)
        mask[-1, L - L // 4 :] = 0
        g = torch.randn(x.shape).to(dtype)
        layer = _two_coef_layer(kind, D, layout, causal)
        xg = x.cuda().requires_grad_(True)
        y = layer(xg, attention_mask=mask.cuda())
        kw = dict(layout=layout, causal=causal, attention_mask=mask)
        ref = O.pde_layer_step(x, kind, 0.12, 0.07, **kw)
        if kind == "advection":
            assert torch.equal(y.detach().cpu(), ref), (shape, dtype)
        else:
            assert_close(y, ref)
        (y.float() * g.cuda().float()).sum().backward()
        dx_ref, (da, db) = O.grads(lambda t, a, b: O.pde_layer_step(t, kind, a, b, **kw), x.float(), g.float(),
                                   [torch.tensor([0.12]), torch.tensor([0.07])])
        assert_close(xg.grad, dx_ref)
        scale = max(1.0, da.abs().max().item(), db.abs().max().item())
        rel = 1e-4 if dtype == torch.float32 else 2e-2
        assert (layer.alpha.grad.cpu() - da).abs().max().item() <= rel * scale, (shape, dtype, layer.alpha.grad, da)
        assert (layer.beta.grad.cpu() - db).abs().max().item() <= rel * scale, (shape, dtype, layer.beta.grad, db)


@pytest.mark.parametrize("pde_type", ["advection-diffusion", "reaction-diffusion"])
def test_pde_transformer_other_pde_types(pde_type):
    """PDETransformerLM / Classifier with the other two PDE types: the refinement
    runs layer by layer on the kernels and matches the oracle's layers."""
    from cta_b200 import transformers as T

    torch.manual_seed(3)
    kw = dict(vocab_size=101, embed_dim=32, num_heads=4, hidden_dim=64, num_layers=2, pde_steps=2,
              max_length=64, dropout=0.0, pde_type=pde_type)
    kind = pde_type.split("-")[0]
    for model in ("classifier", "lm"):
        net = (T.PDETransformerClassifier(num_classes=3, **kw) if model == "classifier" else T.PDETransformerLM(**kw))
        net = net.cuda().eval()
        ids = torch.randint(0, 101, (2, 50), device="cuda")
        mask = torch.ones(2, 50, dtype=torch.long, device="cuda")
        mask[1, 41:] = 0
        out = net(ids, mask)
        causal = model == "lm"
        with torch.no_grad():
            x = net.embedding(ids) + net.pos_encoder[:, :50, :]
            if causal:
                pad = torch.zeros_like(mask, dtype=torch.float32).masked_fill(mask == 0, float("-inf"))
                cm = T.generate_causal_mask(50, x.device)
            for tl, plist in zip(net.transformer_layers, net.pde_layers):
                x = tl(x, src_mask=cm, src_key_padding_mask=pad) if causal else tl(x, src_key_padding_mask=mask == 0)
                xc = x.cpu()
                for p in plist:
                    xc = O.pde_layer_step(xc, kind, p.alpha.detach().cpu(), p.beta.detach().cpu(), layout="bld",
                                          causal=causal, attention_mask=mask.cpu())
                x = xc.cuda()
            if causal:
                ref = net.fc(x)
            else:
                em = mask.unsqueeze(-1).expand(x.size())
                ref = net.fc(torch.sum(x * em, 1) / torch.clamp(mask.sum(1, keepdim=True), min=1))
        torch.testing.assert_close(out.detach(), ref, rtol=1e-4, atol=1e-4)
        out.float().sum().backward()
        for plist in net.pde_layers:
            for p in plist:
                assert torch.isfinite(p.alpha.grad).all() and torch.isfinite(p.beta.grad).all()


# ---------------------------------------------------------------------------
# the classifier's last refinement fused with its masked mean pool
# ---------------------------------------------------------------------------
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("steps", [1, 4, 8, 11])
@pytest.mark.parametrize("shape", [(3, 1000, 512), (2, 77, 264), (4, 40, 6)])
def test_stack_pool_matches_stack_then_pool(dtype, steps, shape):
    """pooled = masked mean of the stepped tensor (never written), against the
    stack followed by the reference's pooling; gradients through both paths."""
    from cta_b200 import ops
    from cta_b200.pde_layers import DiffusionPDELayer, diffusion_pde_stack, diffusion_stack_pool

    torch.manual_seed(30 + steps)
    B, L, D = shape
    x = torch.randn(B, L, D, device="cuda").to(dtype)
    mask = torch.ones(B, L, dtype=torch.long, device="cuda")
    mask[0, L - L // 3 :] = 0
    mask[-1, : L // 5] = 0
    if B == 4:
        mask[1] = 0  # a fully padded sequence: zero count, every tile skipped
    layers = [DiffusionPDELayer(D, alpha_init=0.1 - 0.005 * k, layout="bld").cuda() for k in range(steps)]

    def reference(t):
        y = diffusion_pde_stack(t, layers, attention_mask=mask)
        s = torch.sum(y * mask.unsqueeze(-1).expand(y.size()), dim=1)
        return s / torch.clamp(mask.sum(dim=1, keepdim=True), min=1)

    xa = x.clone().requires_grad_(True)
    xb = x.clone().requires_grad_(True)
    pa = diffusion_stack_pool(xa, layers, mask)
    pb = reference(xb)
    assert pa.dtype == pb.dtype and pa.shape == (B, D)
    assert_close(pa, pb)
    g = torch.randn(B, D, device="cuda").to(dtype)
    da = torch.autograd.grad((pa.float() * g.float()).sum(), [xa] + [l.alpha for l in layers])
    db = torch.autograd.grad((pb.float() * g.float()).sum(), [xb] + [l.alpha for l in layers])
    assert torch.equal(da[0], db[0])  # the same pooled gradient through the same backward kernels
    for u, v in zip(da[1:], db[1:]):
        assert torch.equal(u, v)
    with pytest.raises(ValueError):
        ops.bld_forward_pool(x, [0.1], 1, None)


@pytest.mark.parametrize("kind", ["advection", "reaction"])
@pytest.mark.parametrize("causal", [False, True])
@pytest.mark.parametrize("steps", [1, 2, 3, 4, 6])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_pde_stack_forward_matches_layer_chain(kind, causal, steps, dtype):
    """Consecutive advection / reaction layers fused into one launch (per 4
    layers), fp32 between the layers: against the oracle's layer chain run in
    fp32 and rounded once (advection bit for bit; reaction to the fp32 bar, its
    sigmoid uses __expf), and bit for bit against the per-layer kernels in fp32."""
    from cta_b200.pde_layers import pde_stack_forward

    torch.manual_seed(40 + steps)
    B, L, D = 2, 700, 264
    x = (2.0 * torch.randn(B, L, D)).to(dtype)
    mask = torch.ones(B, L, dtype=torch.long)
    mask[-1, L - L // 4 :] = 0
    layers = [_two_coef_layer(kind, D, "bld", causal, 0.1 - 0.01 * k, 0.05 + 0.01 * k) for k in range(steps)]
    y = pde_stack_forward(x.cuda(), layers, attention_mask=mask.cuda())
    ref = x.float()
    for k in range(steps):
        ref = O.pde_layer_step(ref, kind, 0.1 - 0.01 * k, 0.05 + 0.01 * k, layout="bld", causal=causal,
                               attention_mask=mask)
    ref = ref.to(dtype)
    if kind == "advection":
        assert torch.equal(y.cpu(), ref)
    else:
        assert_close(y, ref)
    if dtype == torch.float32:
        yl = x.cuda()
        with torch.no_grad():
            for l in layers:
                yl = l(yl, attention_mask=mask.cuda())
        assert torch.equal(y, yl)


@pytest.mark.parametrize("pde_type", ["advection-diffusion", "reaction-diffusion"])
def test_model_inference_fuses_two_coefficient_stacks(pde_type, monkeypatch):
    """The PDE-Transformer classifier in fp32 under no_grad takes the fused
    stack path and returns exactly what the per-layer path does.  Both runs are
    under no_grad, so the stock encoder layers take the same (inference fast)
    path; the per-layer run replaces the fused stack with the layer loop."""
    from cta_b200 import transformers as T

    torch.manual_seed(41)
    net = T.PDETransformerClassifier(vocab_size=100, embed_dim=32, num_heads=4, hidden_dim=64, num_layers=2,
                                     num_classes=2, pde_type=pde_type, pde_steps=3, max_length=128,
                                     dropout=0.0).cuda().eval()
    ids = torch.randint(0, 100, (2, 96), device="cuda")
    mask = torch.ones(2, 96, dtype=torch.long, device="cuda")
    mask[1, 80:] = 0
    calls = []
    real = T.pde_stack_forward

    def counting(*a, **k):
        calls.append(1)
        return real(*a, **k)

    monkeypatch.setattr(T, "pde_stack_forward", counting)
    with torch.no_grad():
        fused = net(ids, mask)
    assert len(calls) == 2  # one fused stack per encoder layer

    def layer_loop(x, layers, attention_mask=None, layout=None):
        for l in layers:
            x = l(x, attention_mask=attention_mask)
        return x

    monkeypatch.setattr(T, "pde_stack_forward", layer_loop)
    with torch.no_grad():
        per_layer = net(ids, mask)
    assert torch.equal(fused, per_layer)
