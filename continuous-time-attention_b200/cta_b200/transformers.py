"""PDE-refined Transformer models whose refinement runs on the fused kernels.

Drop-in for ``PDETransformerClassifier`` and ``PDETransformerLM`` of the
reference's src/models/transformers.py (:35-142 and :220-320): same
constructor arguments, same submodules and parameter names
(``pde_layers.{layer}.{step}.alpha``, so reference state_dicts load unchanged),
same forward.  The Transformer parts are stock PyTorch modules, exactly as in
the reference; the only change is that the ``pde_steps`` refinement layers
after each Transformer layer run as ONE fused launch forward and one backward
(:124-133, :309-317), with no layout transposes for ``pde_layout="bld"``.
"""
from __future__ import annotations

import torch
import torch.nn as nn

from .pde_layers import (
    _DiffusionFamilyLayer,
    _TwoCoefficientLayer,
    create_pde_layer,
    diffusion_pde_stack,
    diffusion_stack_pool,
    pde_stack_forward,
)

__all__ = ["generate_causal_mask", "PDETransformerClassifier", "PDETransformerLM"]


def generate_causal_mask(seq_len: int, device: torch.device) -> torch.Tensor:
    """Additive (seq_len, seq_len) mask, -inf above the diagonal (transformers.py:13-32)."""
    return torch.triu(torch.full((seq_len, seq_len), float("-inf"), device=device, dtype=torch.float32), diagonal=1)


def _refine(x: torch.Tensor, pde_list: nn.ModuleList, layout: str, attention_mask: torch.Tensor) -> torch.Tensor:
    if not all(isinstance(l, _DiffusionFamilyLayer) for l in pde_list):
        grad = torch.is_grad_enabled() and (x.requires_grad or any(p.requires_grad for p in pde_list.parameters()))
        kinds = {getattr(l, "KIND", None) for l in pde_list}
        if not grad and len(kinds) == 1 and all(isinstance(l, _TwoCoefficientLayer) for l in pde_list):
            # inference: the whole stack in one launch (per 4 layers); x is [B, L, D] here
            return pde_stack_forward(x, pde_list, attention_mask=attention_mask, layout="bld")
        # training (or mixed kinds): one step per layer, as the reference loops
        x_t = x.transpose(1, 2).contiguous() if layout == "bdl" else x
        for layer in pde_list:
            x_t = layer(x_t, attention_mask=attention_mask)
        return x_t.transpose(1, 2).contiguous() if layout == "bdl" else x_t
    if layout == "bdl":
        x_t = x.transpose(1, 2).contiguous()
        x_t = diffusion_pde_stack(x_t, pde_list, attention_mask=attention_mask)
        return x_t.transpose(1, 2).contiguous()
    return diffusion_pde_stack(x, pde_list, attention_mask=attention_mask)


class PDETransformerClassifier(nn.Module):
    """Sequence classifier with PDE refinement after every layer (transformers.py:35-142)."""

    def __init__(
        self,
        vocab_size,
        embed_dim,
        num_heads,
        hidden_dim,
        num_layers,
        num_classes,
        pde_type="diffusion",
        pde_steps=1,
        pde_layout: str = "bld",
        max_length=512,
        dropout=0.1,
        **pde_kwargs,
    ):
        super().__init__()
        self.embedding = nn.Embedding(vocab_size, embed_dim)
        self.pos_encoder = nn.Parameter(torch.randn(1, max_length, embed_dim))
        self.dropout = nn.Dropout(dropout)
        self.transformer_layers = nn.ModuleList(
            [
                nn.TransformerEncoderLayer(
                    d_model=embed_dim, nhead=num_heads, dim_feedforward=hidden_dim, dropout=dropout, batch_first=True
                )
                for _ in range(num_layers)
            ]
        )
        self.pde_layout = pde_layout
        self.pde_layers = nn.ModuleList(
            [
                nn.ModuleList(
                    [create_pde_layer(pde_type, embed_dim, layout=pde_layout, **pde_kwargs) for _ in range(pde_steps)]
                )
                for _ in range(num_layers)
            ]
        )
        self.fc = nn.Linear(embed_dim, num_classes)

    def forward(self, input_ids, attention_mask):
        x = self.embedding(input_ids)
        seq_len = x.size(1)
        x = x + self.pos_encoder[:, :seq_len, :]
        x = self.dropout(x)
        padding_mask = attention_mask == 0
        n = len(self.transformer_layers)
        for i, (transformer_layer, pde_list) in enumerate(zip(self.transformer_layers, self.pde_layers)):
            x = transformer_layer(x, src_key_padding_mask=padding_mask)
            if (i == n - 1 and self.pde_layout == "bld" and len(pde_list) > 0 and x.size(1) >= 3
                    and all(isinstance(l, _DiffusionFamilyLayer) and not l.causal for l in pde_list)):
                # the last refinement and the masked mean pool in one pass
                return self.fc(diffusion_stack_pool(x, pde_list, attention_mask))
            x = _refine(x, pde_list, self.pde_layout, attention_mask)
        expanded_mask = attention_mask.unsqueeze(-1).expand(x.size())
        sum_embeddings = torch.sum(x * expanded_mask, dim=1)
        sum_mask = torch.clamp(attention_mask.sum(dim=1, keepdim=True), min=1)
        return self.fc(sum_embeddings / sum_mask)


class PDETransformerLM(nn.Module):
    """Language model with causal PDE refinement after every layer (transformers.py:220-320)."""

    def __init__(
        self,
        vocab_size,
        embed_dim,
        num_heads,
        hidden_dim,
        num_layers,
        pde_type="diffusion",
        pde_steps=1,
        pde_layout: str = "bld",
        max_length=512,
        dropout=0.1,
        **pde_kwargs,
    ):
        super().__init__()
        self.embedding = nn.Embedding(vocab_size, embed_dim)
        self.pos_encoder = nn.Parameter(torch.randn(1, max_length, embed_dim))
        self.dropout = nn.Dropout(dropout)
        self.transformer_layers = nn.ModuleList(
            [
                nn.TransformerEncoderLayer(
                    d_model=embed_dim, nhead=num_heads, dim_feedforward=hidden_dim, dropout=dropout, batch_first=True
                )
                for _ in range(num_layers)
            ]
        )
        self.pde_layout = pde_layout
        self.pde_layers = nn.ModuleList(
            [
                nn.ModuleList(
                    [
                        create_pde_layer(pde_type, embed_dim, layout=pde_layout, causal=True, **pde_kwargs)
                        for _ in range(pde_steps)
                    ]
                )
                for _ in range(num_layers)
            ]
        )
        self.fc = nn.Linear(embed_dim, vocab_size)

    def forward(self, input_ids, attention_mask):
        x = self.embedding(input_ids)
        seq_len = x.size(1)
        x = x + self.pos_encoder[:, :seq_len, :]
        x = self.dropout(x)
        padding_mask = torch.zeros_like(attention_mask, dtype=torch.float32)
        padding_mask = padding_mask.masked_fill(attention_mask == 0, float("-inf"))
        causal_mask = generate_causal_mask(seq_len, device=x.device)
        for transformer_layer, pde_list in zip(self.transformer_layers, self.pde_layers):
            x = transformer_layer(x, src_mask=causal_mask, src_key_padding_mask=padding_mask)
            x = _refine(x, pde_list, self.pde_layout, attention_mask)
        return self.fc(x)
