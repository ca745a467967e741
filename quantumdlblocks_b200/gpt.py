"""Decoder-only GPT whose attention is flash-Born: the end-to-end data-parallel training workload.

The attention layer follows the flash-Born branch of the reference's Born attention layer
(``layers/attention.py:508-589`` and ``:691-715``): the block input is projected onto the unit
sphere, one fused projection gives Q, K, V in ``(B, H, T, hd)`` views, Q and K are rotated by the
unitary RoPE (``functional.py:104-121``: the two halves of each head turned by position-dependent
angles, base 10000) and normalised again, and ``flash_born_attention`` runs with the learnable
per-head scale clamped to [1, 100] (initialised to sqrt(hd), ``:390,429``) and eps 1e-12.  The
rest is a plain pre-norm GPT: RMSNorm, a 4x GELU MLP, token embeddings tied to the output head.
At d_model 1024, 6 layers, 16 heads and a 50,257-token vocabulary it has 127 M parameters.  The
embedding table is padded to a multiple of 64 rows (50,304, the reference GPT's own default
vocabulary size) so the output-head GEMMs have aligned leading dimensions (an odd width sends them
to unaligned kernels several times slower); the padded logits are held at -inf, so the loss and
every gradient equal the unpadded model's.

With the native attention op the layer's operand prologue is native too: ``l2_normalize`` of the
input and ``qkv_rope_l2norm`` (RoPE + L2 normalisation of Q and K, V copied to ``(B, H, T, hd)``)
each run as one kernel forward and one backward, where the reference runs a chain of PyTorch ops
(``:512-516, :573-589``).  With any other attention callable (the tests' eager restatement) the
layer runs those ops in PyTorch on strided views.  The native attention op stores O token-major,
so the head merge before the output projection is a view, and the loss is the native fused
cross-entropy over the bf16 logits (the reference's ``F.cross_entropy``, ``models/born_gpt.py:1291``,
runs over an fp32 copy of them).

Data parallelism (``make_ddp``): one process per GPU, ``torch.nn.parallel.DistributedDataParallel``
over NCCL, gradients all-reduced in buckets while the backward runs.
"""
from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Callable, Optional

import numpy as np
import torch
import torch.nn as nn
import torch.nn.functional as F

__all__ = ["GPTConfig", "BornGPT", "zipf_tokens", "make_ddp", "train_step", "param_count"]


@dataclass
class GPTConfig:
    vocab_size: int = 50257
    d_model: int = 1024
    n_layers: int = 6
    n_heads: int = 16
    seq_len: int = 1024
    mlp_ratio: int = 4
    eps: float = 1e-12
    pad_vocab_to: int = 64


def _l2n(x: torch.Tensor, eps: float) -> torch.Tensor:
    return x * torch.rsqrt(x.float().square().sum(-1, keepdim=True) + eps).to(x.dtype)


class BornAttention(nn.Module):
    def __init__(self, cfg: GPTConfig, attention: Callable, fused_prologue: bool):
        super().__init__()
        d, H = cfg.d_model, cfg.n_heads
        self.H, self.hd, self.eps = H, d // H, cfg.eps
        self.attention = attention
        self.fused_prologue = fused_prologue
        self.qkv = nn.Linear(d, 3 * d, bias=False)
        self.out = nn.Linear(d, d, bias=False)
        with torch.no_grad():
            for c in range(3):
                nn.init.orthogonal_(self.qkv.weight[c * d:(c + 1) * d])
            nn.init.orthogonal_(self.out.weight)
        self.head_scale = nn.Parameter(torch.full((1, H, 1, 1), math.sqrt(self.hd)))
        half = self.hd // 2
        inv = 1.0 / (10000.0 ** (torch.arange(half, dtype=torch.float32) / half))
        ang = torch.arange(cfg.seq_len, dtype=torch.float32)[:, None] * inv[None, :]
        self.register_buffer("cos", ang.cos(), persistent=False)
        self.register_buffer("sin", ang.sin(), persistent=False)

    def _rope(self, x: torch.Tensor) -> torch.Tensor:
        T, half = x.shape[-2], self.hd // 2
        c, s = self.cos[:T].to(x.dtype), self.sin[:T].to(x.dtype)
        x1, x2 = x[..., :half], x[..., half:]
        return torch.cat([x1 * c - x2 * s, x1 * s + x2 * c], dim=-1)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        B, T, D = x.shape
        if self.fused_prologue and x.is_cuda:
            from .kernels.prologue import l2_normalize, qkv_rope_l2norm

            q, k, v = qkv_rope_l2norm(self.qkv(l2_normalize(x, self.eps)), self.cos, self.sin, self.H, self.eps)
        else:
            psi = _l2n(x, self.eps)
            qkv = self.qkv(psi).view(B, T, 3, self.H, self.hd)
            q, k, v = (qkv[:, :, i].transpose(1, 2) for i in range(3))  # (B, H, T, hd) views
            q = _l2n(self._rope(q), self.eps)
            k = _l2n(self._rope(k), self.eps)
        scale = torch.clamp(self.head_scale, min=1.0, max=100.0)
        # the native op stores O token-major, so the head merge below is a view, not a copy
        kw = {"token_major": True} if self.fused_prologue else {}
        o = self.attention(q, k, v, scale=scale, is_causal=True, eps=self.eps, **kw)
        return self.out(o.transpose(1, 2).reshape(B, T, D))


class Block(nn.Module):
    def __init__(self, cfg: GPTConfig, attention: Callable, fused_prologue: bool):
        super().__init__()
        d = cfg.d_model
        self.attn = BornAttention(cfg, attention, fused_prologue)
        self.norm = nn.RMSNorm(d)
        self.fc = nn.Linear(d, cfg.mlp_ratio * d, bias=False)
        self.proj = nn.Linear(cfg.mlp_ratio * d, d, bias=False)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        x = x + self.attn(x)
        return x + self.proj(F.gelu(self.fc(self.norm(x)), approximate="tanh"))


class BornGPT(nn.Module):
    """``attention`` defaults to this package's ``flash_born_attention`` (CUDA only), which also
    switches the layers' operand prologue to the native kernels."""

    def __init__(self, cfg: GPTConfig, attention: Optional[Callable] = None):
        super().__init__()
        fused = attention is None
        self.native_loss = fused  # with the native attention, the loss runs on the native kernels too
        if attention is None:
            from .kernels.flash_born import flash_born_attention as attention
        self.cfg = cfg
        m = max(1, cfg.pad_vocab_to)
        rows = (cfg.vocab_size + m - 1) // m * m
        self.emb = nn.Embedding(rows, cfg.d_model)
        nn.init.normal_(self.emb.weight, std=0.02)
        mask = torch.zeros(rows)
        mask[cfg.vocab_size:] = float("-inf")
        self.register_buffer("logit_mask", mask, persistent=False)
        self.blocks = nn.ModuleList(Block(cfg, attention, fused) for _ in range(cfg.n_layers))
        self.norm = nn.RMSNorm(cfg.d_model)

    def forward(self, tokens: torch.Tensor, targets: torch.Tensor) -> torch.Tensor:
        x = self.emb(tokens)
        for blk in self.blocks:
            x = blk(x)
        h = self.norm(x)
        logits = F.linear(h, self.emb.weight, self.logit_mask.to(h.dtype))  # tied head, padded rows at -inf
        logits = logits.view(-1, logits.shape[-1])
        if self.native_loss and logits.is_cuda and logits.dtype == torch.bfloat16:
            from .kernels.xent import cross_entropy

            return cross_entropy(logits, targets.reshape(-1))
        return F.cross_entropy(logits.float(), targets.reshape(-1))


def param_count(model: nn.Module) -> int:
    """Parameters of the model as specified (the embedding rows that only pad the head excluded)."""
    n = sum(p.numel() for p in model.parameters())
    if isinstance(model, BornGPT):
        n -= (model.emb.num_embeddings - model.cfg.vocab_size) * model.cfg.d_model
    return n


def zipf_tokens(batch: int, seq_len: int, vocab: int, s: float = 1.1, seed: int = 0) -> np.ndarray:
    """``(batch, seq_len + 1)`` int64 token ids, Zipf(s) ranks over the vocabulary (rank 1 = id 0)."""
    rng = np.random.default_rng(seed)
    need = batch * (seq_len + 1)
    out = np.empty(0, dtype=np.int64)
    while out.size < need:
        draw = rng.zipf(s, size=2 * need)
        out = np.concatenate([out, draw[draw <= vocab] - 1])
    return out[:need].reshape(batch, seq_len + 1)


def make_ddp(model: nn.Module, device: torch.device, bucket_mb: float = 25.0):
    """Data-parallel wrapper: NCCL all-reduce of the gradients in ``bucket_mb`` buckets, launched
    as each bucket's gradients are produced in the backward (gradients are bucket views)."""
    from torch.nn.parallel import DistributedDataParallel

    dev_ids = [device.index] if device.type == "cuda" else None
    return DistributedDataParallel(model, device_ids=dev_ids, bucket_cap_mb=bucket_mb,
                                   gradient_as_bucket_view=True, static_graph=True)


def train_step(model: nn.Module, opt: torch.optim.Optimizer, tokens: torch.Tensor,
               autocast_dtype: Optional[torch.dtype] = torch.bfloat16) -> torch.Tensor:
    """One optimiser step on ``tokens`` ``(B, T + 1)``; returns the loss (a device tensor)."""
    inp, tgt = tokens[:, :-1], tokens[:, 1:]
    dev_type = tokens.device.type
    with torch.autocast(dev_type, dtype=autocast_dtype, enabled=autocast_dtype is not None):
        loss = model(inp, tgt)
    loss.backward()
    opt.step()
    opt.zero_grad(set_to_none=True)
    return loss.detach()
