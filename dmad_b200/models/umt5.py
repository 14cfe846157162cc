"""umT5 text encoder (the Wan conditioner): architecture, checkpoint keys and prompt encoding.

Parity: train/wan/rcm/utils/umt5.py (T5 encoder with per-layer relative position biases --
``shared_pos=False`` for umT5 --, RMS "T5LayerNorm", unscaled attention, gated GELU-tanh
feed-forward ``fc2(fc1(x) * gelu(gate(x)))``; umT5-XXL: vocab 256384, d 4096, 64 heads,
FFN 10240, 24 layers, 32 buckets, max distance 128) and the text-condition convention of the
Wan stack: 512 token rows per prompt, rows past the prompt's length zeroed.

The relative-position bucketing is T5's (Raffel et al., JMLR 2020, section 2.1): exact buckets for
distances below half the buckets, logarithmic buckets up to ``max_dist``, and for the bidirectional
encoder the sign in the top bucket half.  Attention runs through PyTorch SDPA with the bias as an
additive mask (scale 1).  Random-init weights unless a state dict is loaded; ``tokenize`` uses a
Hugging Face tokenizer directory when one is given, else a deterministic hash tokenizer (synthetic
runs: no network, no vocabulary files).
"""
from __future__ import annotations

import hashlib
import math
from dataclasses import dataclass

import torch
import torch.nn as nn
import torch.nn.functional as F


@dataclass
class UMT5Config:
    vocab: int = 256384
    dim: int = 4096
    dim_attn: int = 4096
    dim_ffn: int = 10240
    num_heads: int = 64
    num_layers: int = 24
    num_buckets: int = 32
    max_dist: int = 128
    text_len: int = 512


UMT5_XXL = UMT5Config()


def relative_bucket(rel: torch.Tensor, num_buckets: int, max_dist: int, bidirectional: bool = True) -> torch.Tensor:
    """T5 bucket index of key-minus-query offsets ``rel``."""
    if bidirectional:
        half = num_buckets // 2
        out = (rel > 0).long() * half
        dist = rel.abs()
    else:
        half = num_buckets
        out = torch.zeros_like(rel)
        dist = (-rel).clamp(min=0)
    exact = half // 2
    far = exact + (torch.log(dist.float().clamp(min=1) / exact) / math.log(max_dist / exact) * (half - exact)).long()
    far = far.clamp(max=half - 1)
    return out + torch.where(dist < exact, dist, far)


class RelPosBias(nn.Module):
    def __init__(self, num_buckets, num_heads, max_dist=128):
        super().__init__()
        self.num_buckets, self.max_dist = num_buckets, max_dist
        self.embedding = nn.Embedding(num_buckets, num_heads)

    def forward(self, lq, lk):
        dev = self.embedding.weight.device
        rel = torch.arange(lk, device=dev)[None] - torch.arange(lq, device=dev)[:, None]
        b = self.embedding(relative_bucket(rel, self.num_buckets, self.max_dist))  # [lq, lk, H]
        return b.permute(2, 0, 1)[None]


class T5Norm(nn.Module):
    def __init__(self, dim, eps=1e-6):
        super().__init__()
        self.eps = eps
        self.weight = nn.Parameter(torch.ones(dim))

    def forward(self, x):
        y = x * torch.rsqrt(x.float().pow(2).mean(-1, keepdim=True) + self.eps)
        return self.weight * y.to(self.weight.dtype if self.weight.dtype in (torch.float16, torch.bfloat16) else y.dtype)


class _Attn(nn.Module):
    def __init__(self, dim, dim_attn, num_heads):
        super().__init__()
        self.h = num_heads
        self.q = nn.Linear(dim, dim_attn, bias=False)
        self.k = nn.Linear(dim, dim_attn, bias=False)
        self.v = nn.Linear(dim, dim_attn, bias=False)
        self.o = nn.Linear(dim_attn, dim, bias=False)

    def forward(self, x, bias):
        B, L, _ = x.shape
        sh = lambda t: t.view(B, L, self.h, -1).transpose(1, 2)  # noqa: E731
        o = F.scaled_dot_product_attention(sh(self.q(x)), sh(self.k(x)), sh(self.v(x)), attn_mask=bias.to(x.dtype),
                                           scale=1.0)
        return self.o(o.transpose(1, 2).reshape(B, L, -1))


class _FFN(nn.Module):
    def __init__(self, dim, dim_ffn):
        super().__init__()
        self.gate = nn.Sequential(nn.Linear(dim, dim_ffn, bias=False), nn.GELU(approximate="tanh"))
        self.fc1 = nn.Linear(dim, dim_ffn, bias=False)
        self.fc2 = nn.Linear(dim_ffn, dim, bias=False)

    def forward(self, x):
        return self.fc2(self.fc1(x) * self.gate(x))


class _Block(nn.Module):
    def __init__(self, c: UMT5Config):
        super().__init__()
        self.norm1 = T5Norm(c.dim)
        self.attn = _Attn(c.dim, c.dim_attn, c.num_heads)
        self.norm2 = T5Norm(c.dim)
        self.ffn = _FFN(c.dim, c.dim_ffn)
        self.pos_embedding = RelPosBias(c.num_buckets, c.num_heads, c.max_dist)

    def forward(self, x, mask_bias):
        L = x.shape[1]
        bias = self.pos_embedding(L, L) + mask_bias
        x = x + self.attn(self.norm1(x), bias)
        return x + self.ffn(self.norm2(x))


class UMT5Encoder(nn.Module):
    def __init__(self, cfg: UMT5Config = UMT5_XXL):
        super().__init__()
        self.cfg = cfg
        self.token_embedding = nn.Embedding(cfg.vocab, cfg.dim)
        self.blocks = nn.ModuleList([_Block(cfg) for _ in range(cfg.num_layers)])
        self.norm = T5Norm(cfg.dim)

    def forward(self, ids, mask=None):
        """ids [B, L] int64, mask [B, L] (1 = token) -> hidden states [B, L, dim]."""
        x = self.token_embedding(ids)
        if mask is None:
            mask = torch.ones_like(ids)
        mask_bias = torch.zeros(mask.shape, dtype=torch.float32, device=ids.device)
        mask_bias = mask_bias.masked_fill(mask == 0, torch.finfo(torch.float32).min)[:, None, None, :]
        for blk in self.blocks:
            x = blk(x, mask_bias)
        return self.norm(x)


class HashTokenizer:
    """Deterministic whitespace / punctuation tokenizer into [2, vocab) with EOS id 1 (no vocabulary files)."""

    def __init__(self, vocab: int, text_len: int):
        self.vocab, self.text_len = vocab, text_len

    def __call__(self, texts):
        ids = torch.zeros(len(texts), self.text_len, dtype=torch.long)
        mask = torch.zeros_like(ids)
        for i, t in enumerate(texts):
            toks = [2 + int.from_bytes(hashlib.sha1(w.encode()).digest()[:4], "little") % (self.vocab - 2)
                    for w in t.lower().replace(",", " , ").replace(".", " . ").split()]
            toks = toks[: self.text_len - 1] + [1]
            ids[i, :len(toks)] = torch.tensor(toks)
            mask[i, :len(toks)] = 1
        return ids, mask


class TextEncoder:
    """Prompts -> ``[B, text_len, dim]`` context with rows past each prompt zeroed."""

    def __init__(self, cfg: UMT5Config = UMT5_XXL, device="cpu", dtype=torch.bfloat16, tokenizer_path: str | None = None,
                 model: UMT5Encoder | None = None):
        self.cfg = cfg
        self.model = (model or UMT5Encoder(cfg)).to(device=device, dtype=dtype).eval().requires_grad_(False)
        self.device = torch.device(device)
        if tokenizer_path:
            from transformers import AutoTokenizer
            tok = AutoTokenizer.from_pretrained(tokenizer_path)

            def hf(texts):
                enc = tok(texts, padding="max_length", truncation=True, max_length=cfg.text_len, return_tensors="pt",
                          add_special_tokens=True)
                return enc.input_ids, enc.attention_mask
            self.tokenize = hf
        else:
            self.tokenize = HashTokenizer(cfg.vocab, cfg.text_len)

    @torch.no_grad()
    def encode(self, texts: list[str]) -> torch.Tensor:
        ids, mask = self.tokenize(list(texts))
        ids, mask = ids.to(self.device), mask.to(self.device)
        h = self.model(ids, mask)
        return h * mask[..., None].to(h.dtype)
