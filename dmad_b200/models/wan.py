"""Wan2.1-shaped text-to-video DiT, written for the sm_100a kernels.

Architecture parity with the reference ``WanModel`` (train/wan/rcm/networks/wan2pt1.py:508-929):
patch embedding Linear(16*1*2*2 -> D); text embedding Linear(4096 -> D) -> GELU(tanh) -> Linear;
sinusoidal (fp64) timestep embedding -> Linear -> SiLU -> Linear, projection SiLU -> Linear(D -> 6D);
blocks = adaLN LayerNorm -> self-attention (q/k RMSNorm over D, 3D RoPE) -> gated residual
-> affine LayerNorm -> cross-attention to the text -> residual -> adaLN LayerNorm -> GELU FFN
-> gated residual; head = adaLN LayerNorm -> Linear.  Per-frame timesteps ``[B, T]`` are supported.
State-dict keys match the reference (``blocks.{i}.self_attn.q.weight`` ...), so reference
checkpoints load directly and exported weights load into the reference.

Execution differs from the reference: tokens are kept as ``[B*L, D]`` bf16 rows, every
norm / modulation / residual is one fused kernel, q/k/v and cross k/v are one GEMM each,
attention is the tcgen05 flash kernel, and the modulation MLP runs on the small-M kernel.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field

import torch
import torch.nn as nn
import torch.nn.functional as F

from .. import ops
from ..ops import norm as norm_ops
from .layers import SegLinear, cross_attention_core, install_segment_key_remap, self_attention_core
from .sac import checkpoint_block


@dataclass
class WanConfig:
    dim: int = 1536
    ffn_dim: int = 8960
    num_heads: int = 12
    num_layers: int = 30
    in_dim: int = 16
    out_dim: int = 16
    freq_dim: int = 256
    text_dim: int = 4096
    text_len: int = 512
    patch_size: tuple = (1, 2, 2)
    eps: float = 1e-6
    cross_attn_norm: bool = True
    # rope grid limits (VideoRopePosition3DEmb(len_h=128, len_w=128, len_t=32))
    rope_max_t: int = 32

    @property
    def head_dim(self):
        return self.dim // self.num_heads


# train/wan/rcm/configs/defaults/net.py:25-44
WAN_1P3B = WanConfig(dim=1536, ffn_dim=8960, num_heads=12, num_layers=30)
WAN_14B = WanConfig(dim=5120, ffn_dim=13824, num_heads=40, num_layers=40)


def wan_config(name: str, **overrides) -> WanConfig:
    base = {"wan2.1-1.3b": WAN_1P3B, "wan2.1-14b": WAN_14B}[name.lower()]
    cfg = WanConfig(**{**base.__dict__, **overrides})
    return cfg


def rope_3d_angles(T: int, H: int, W: int, head_dim: int, t_offset: int = 0, device=None) -> torch.Tensor:
    """[T*H*W, head_dim/2] fp32 rotation angles = cat(t * f_t, h * f_h, w * f_w).

    dim_h = dim_w = head_dim // 6 * 2, dim_t = head_dim - 2 * dim_h, theta 10000
    (VideoRopePosition3DEmb, train/wan/rcm/networks/wan2pt1.py:62-179).
    """
    dim_h = head_dim // 6 * 2
    dim_t = head_dim - 2 * dim_h
    sp = torch.arange(0, dim_h, 2, dtype=torch.float32, device=device)[: dim_h // 2] / dim_h
    tp = torch.arange(0, dim_t, 2, dtype=torch.float32, device=device)[: dim_t // 2] / dim_t
    f_h = 1.0 / (10000.0 ** sp)
    f_t = 1.0 / (10000.0 ** tp)
    t = torch.arange(t_offset, t_offset + T, dtype=torch.float32, device=device).repeat_interleave(H * W)
    h = torch.arange(H, dtype=torch.float32, device=device).repeat_interleave(W).repeat(T)
    w = torch.arange(W, dtype=torch.float32, device=device).repeat(H * T)
    return torch.cat([t[:, None] * f_t[None], h[:, None] * f_h[None], w[:, None] * f_h[None]], dim=-1)


class _Attn(nn.Module):
    """Holds the parameters of one attention layer under the reference names."""

    def __init__(self, dim, num_heads, cross: bool, eps):
        super().__init__()
        self.dim, self.num_heads, self.eps, self.cross = dim, num_heads, eps, cross
        if cross:
            self.q = SegLinear(dim, [("q", dim)], flat_name="")
            self.kv = SegLinear(dim, [("k", dim), ("v", dim)], flat_name="kv")
        else:
            self.qkv = SegLinear(dim, [("q", dim), ("k", dim), ("v", dim)], flat_name="qkv")
        self.o = SegLinear(dim, [("o", dim)], flat_name="")
        self.norm_q = nn.Module()
        self.norm_q.weight = nn.Parameter(torch.ones(dim))
        self.norm_k = nn.Module()
        self.norm_k.weight = nn.Parameter(torch.ones(dim))
        install_segment_key_remap(self)

    def init_weights(self):
        std = 1.0 / math.sqrt(self.dim)
        lins = [self.q, self.kv] if self.cross else [self.qkv]
        for lin in lins + [self.o]:
            nn.init.trunc_normal_(lin.weight, std=std)
            lin.bias.data.zero_()
        self.norm_q.weight.data.fill_(1.0)
        self.norm_k.weight.data.fill_(1.0)


class WanBlock(nn.Module):
    def __init__(self, cfg: WanConfig):
        super().__init__()
        D = cfg.dim
        self.cfg = cfg
        self.self_attn = _Attn(D, cfg.num_heads, False, cfg.eps)
        self.cross_attn = _Attn(D, cfg.num_heads, True, cfg.eps)
        self.norm3 = nn.LayerNorm(D, eps=cfg.eps, elementwise_affine=True) if cfg.cross_attn_norm else None
        self.ffn = nn.Module()
        self.ffn.add_module("0", SegLinear(D, [("0", cfg.ffn_dim)], flat_name=""))
        self.ffn.add_module("2", SegLinear(cfg.ffn_dim, [("2", D)], flat_name=""))
        self.modulation = nn.Parameter(torch.randn(1, 6, D) / D ** 0.5)

    def init_weights(self):
        self.self_attn.init_weights()
        self.cross_attn.init_weights()
        if self.norm3 is not None:
            self.norm3.reset_parameters()
        nn.init.trunc_normal_(self.modulation, std=1.0 / math.sqrt(self.cfg.dim))

    def linears(self):
        return [self.self_attn.qkv, self.self_attn.o, self.cross_attn.q, self.cross_attn.kv, self.cross_attn.o,
                getattr(self.ffn, "0"), getattr(self.ffn, "2")]

    def forward(self, x, e0, context, cos, sin, B, L, rpg, cp=None, attn_ctx=None):
        """x: [B*L, D] bf16 (L = this rank's tokens under context parallelism); e0: [G, 6, D] fp32;
        context: [B*Lc, D] bf16; rpg: rows per modulation group (int) or an int32 group index per row;
        attn_ctx: a block mask (``AttnMaskSpec``) or a KV-cache context (``AttnContext``) for the causal
        and teacher-forcing modes (None: full attention)."""
        cfg = self.cfg
        D, H = cfg.dim, cfg.num_heads
        Lc = context.shape[0] // B
        grp = {"gidx": rpg} if torch.is_tensor(rpg) else {"rows_per_group": rpg}
        e = self.modulation.float()[0] + e0  # [G, 6, D]
        h = ops.ln_mod(x, e[:, 1], e[:, 0], a_add=1.0, eps=cfg.eps, **grp)
        qkv = self.self_attn.qkv(h)
        if attn_ctx is not None:
            a = self._masked_self_attention(qkv, cos, sin, B, L, attn_ctx)
        elif cp is not None and cp.world > 1:
            from ..parallel.cp import hybrid_self_attention, ring_self_attention, self_attention_cp
            attn = {"ring": ring_self_attention, "hybrid": hybrid_self_attention}.get(cp.impl, self_attention_cp)
            a = attn(qkv, self.self_attn.norm_q.weight, self.self_attn.norm_k.weight, cos, sin, B, H, cfg.eps, cp)
        else:
            a = self_attention_core(qkv, self.self_attn.norm_q.weight, self.self_attn.norm_k.weight, cos, sin, B, L,
                                    H, cfg.eps)
        y = self.self_attn.o(a)
        x = ops.gate_residual(x, y, e[:, 2], **grp)
        h3 = ops.layer_norm_affine(x, self.norm3.weight, self.norm3.bias, cfg.eps) if self.norm3 is not None else x
        cq = self.cross_attn.q(h3)
        ckv = self.cross_attn.kv(context)
        c = cross_attention_core(cq, ckv, self.cross_attn.norm_q.weight, self.cross_attn.norm_k.weight, B, L, Lc, H,
                                 cfg.eps)
        x = x + self.cross_attn.o(c)
        h2 = ops.ln_mod(x, e[:, 4], e[:, 3], a_add=1.0, eps=cfg.eps, **grp)
        f = ops.gelu_tanh(getattr(self.ffn, "0")(h2))
        y2 = getattr(self.ffn, "2")(f)
        return ops.gate_residual(x, y2, e[:, 5], **grp)


    def _masked_self_attention(self, qkv, cos, sin, B, L, actx):
        """Self-attention under a block mask and / or against the KV cache (causal modes)."""
        from ..ops.block_attention import AttnMaskSpec, block_attention
        from .kv_cache import KVCacheMode

        cfg = self.cfg
        D, H = cfg.dim, cfg.num_heads
        hd = D // H
        q = norm_ops.rope(ops.rms_norm(qkv[:, :D], self.self_attn.norm_q.weight, cfg.eps), cos, sin, hd)
        k = norm_ops.rope(ops.rms_norm(qkv[:, D:2 * D], self.self_attn.norm_k.weight, cfg.eps), cos, sin, hd)
        q4, k4, v4 = q.reshape(B, L, H, hd), k.reshape(B, L, H, hd), qkv[:, 2 * D:].reshape(B, L, H, hd)
        if isinstance(actx, AttnMaskSpec):
            return block_attention(q4, k4, v4, actx).reshape(B * L, D)
        kk, vv = k4, v4
        cache = actx.kv_cache
        if actx.mode != KVCacheMode.DISABLED and cache is not None:
            at = cache.get_prefix_end(actx.block_range)
            if actx.mode == KVCacheMode.APPEND:
                if at != cache.current_len:
                    raise RuntimeError("an appended chunk must follow the whole committed prefix")
                _, end = cache.append(k4, v4)
                kk, vv = cache.k[:, :end], cache.v[:, :end]
            else:
                kk, vv = cache.write_transient(k4, v4, at)
        return block_attention(q4, kk, vv, actx.mask).reshape(B * L, D)


class _Head(nn.Module):
    def __init__(self, cfg: WanConfig):
        super().__init__()
        self.cfg = cfg
        self.head = nn.Linear(cfg.dim, math.prod(cfg.patch_size) * cfg.out_dim)
        self.modulation = nn.Parameter(torch.randn(1, 2, cfg.dim) / cfg.dim ** 0.5)

    def init_weights(self):
        nn.init.trunc_normal_(self.modulation, std=1.0 / math.sqrt(self.cfg.dim))
        nn.init.zeros_(self.head.weight)
        nn.init.zeros_(self.head.bias)

    def forward(self, x, e, rpg):
        m = self.modulation.float()[0]  # [2, D]
        shift = m[0][None] + e
        scale = m[1][None] + e
        grp = {"gidx": rpg} if torch.is_tensor(rpg) else {"rows_per_group": rpg}
        h = ops.ln_mod(x, scale, shift, a_add=1.0, eps=self.cfg.eps, **grp)
        # the reference runs the head under fp32 autocast
        return F.linear(h.float(), self.head.weight.float(), self.head.bias.float())


class WanModel(nn.Module):
    """Wan2.1 DiT.  ``forward(x [B,16,T,H,W], timesteps [B,1|T], context [B,Lc,4096]) -> [B,16,T,H,W]`` fp32."""

    def __init__(self, cfg: WanConfig = WAN_1P3B):
        super().__init__()
        self.cfg = cfg
        D = cfg.dim
        pin = cfg.in_dim * math.prod(cfg.patch_size)
        self.patch_embedding = nn.Linear(pin, D)
        self.text_embedding = nn.Sequential(nn.Linear(cfg.text_dim, D), nn.GELU(approximate="tanh"), nn.Linear(D, D))
        self.time_embedding = nn.Sequential(nn.Linear(cfg.freq_dim, D), nn.SiLU(), nn.Linear(D, D))
        self.time_projection = nn.Sequential(nn.SiLU(), nn.Linear(D, D * 6))
        self.blocks = nn.ModuleList([WanBlock(cfg) for _ in range(cfg.num_layers)])
        self.head = _Head(cfg)
        self.checkpoint_blocks = 0  # activation-checkpoint the first N blocks
        self.checkpoint_policy = "block_wise"  # or "mm_only" (keep matmul / attention outputs)
        self._rope_cache: dict = {}
        self.cp = None  # ContextParallel (sequence sharding) or None
        self.init_weights()

    # --------------------------------------------------------------- init (wan2pt1.py:839-880)
    def init_weights(self):
        for m in self.modules():
            if isinstance(m, nn.Linear):
                nn.init.xavier_uniform_(m.weight)
                if m.bias is not None:
                    nn.init.zeros_(m.bias)
            elif isinstance(m, SegLinear):
                nn.init.xavier_uniform_(m.weight)
                if m.bias is not None:
                    nn.init.zeros_(m.bias)
        for b in self.blocks:
            b.init_weights()
        self.head.init_weights()
        nn.init.xavier_uniform_(self.patch_embedding.weight)
        nn.init.zeros_(self.patch_embedding.bias)
        for seq in (self.text_embedding, self.time_embedding, self.time_projection):
            for m in seq.modules():
                if isinstance(m, nn.Linear):
                    nn.init.normal_(m.weight, std=0.02)
                    nn.init.zeros_(m.bias)
        nn.init.zeros_(self.head.head.weight)
        nn.init.zeros_(self.head.head.bias)

    # --------------------------------------------------------------- helpers
    def rope_tables(self, T, H, W, device, t_offset=0):
        key = (T, H, W, t_offset, str(device))
        tab = self._rope_cache.get(key)
        if tab is None:
            ang = rope_3d_angles(T, H, W, self.cfg.head_dim, t_offset, device=device)
            tab = (torch.cos(ang).contiguous(), torch.sin(ang).contiguous())
            self._rope_cache[key] = tab
        return tab

    def time_embed(self, t_flat):
        """[M] timesteps -> (e [M, D], e0 [M, 6, D]) fp32."""
        s = ops.sinusoidal_embedding(t_flat.float(), self.cfg.freq_dim)
        te0, te2 = self.time_embedding[0], self.time_embedding[2]
        h1 = ops.small_linear(s, te0.weight, te0.bias)
        e = ops.small_linear(h1, te2.weight, te2.bias, act_in="silu")
        tp = self.time_projection[1]
        e0 = ops.small_linear(e, tp.weight, tp.bias, act_in="silu")
        return e, e0.view(-1, 6, self.cfg.dim)

    def text_embed(self, ctx):
        l0, l2 = self.text_embedding[0], self.text_embedding[2]
        B, Lc, Dt = ctx.shape
        x = ctx.reshape(B * Lc, Dt).to(l0.weight.dtype)
        h = ops.gelu_tanh(F.linear(x, l0.weight, l0.bias))
        return F.linear(h, l2.weight, l2.bias)

    def patchify(self, x):
        kt, kh, kw = self.cfg.patch_size
        B, C, T, H, W = x.shape
        x = x.view(B, C, T // kt, kt, H // kh, kh, W // kw, kw)
        x = x.permute(0, 2, 4, 6, 1, 3, 5, 7).reshape(B * (T // kt) * (H // kh) * (W // kw), C * kt * kh * kw)
        return x.contiguous(), (T // kt, H // kh, W // kw)

    def unpatchify(self, x, B, grid):
        kt, kh, kw = self.cfg.patch_size
        T, H, W = grid
        C = self.cfg.out_dim
        x = x.view(B, T, H, W, kt, kh, kw, C).permute(0, 7, 1, 4, 2, 5, 3, 6)
        return x.reshape(B, C, T * kt, H * kh, W * kw)

    # --------------------------------------------------------------- forward
    def forward(self, x_B_C_T_H_W, timesteps_B_T, crossattn_emb, feature_hook_block: int | None = None,
                stop_after_block: int | None = None, attn_meta=None, inference_state=None, **unused):
        """Returns the denoiser output; with ``feature_hook_block`` returns (output, features [B, L, D])
        where features is the token output of that block (the critic's feature tap).  With
        ``stop_after_block`` the forward stops after that block and returns only its features.
        ``attn_meta`` (an ``AttnMaskSpec``) masks self-attention block-wise over the whole sequence;
        ``inference_state`` (a ``CausalInferenceState``) runs the input as the chunk at its current
        block against the per-layer KV caches, with RoPE at the chunk's frame offset."""
        cfg = self.cfg
        cp = self.cp if (self.cp is not None and self.cp.world > 1) else None
        if cp is not None and cp.broadcast_inputs:
            # every rank of the CP group works on rank 0's sample (wan2pt1.py:723-733)
            x_B_C_T_H_W = cp.broadcast(x_B_C_T_H_W)
            timesteps_B_T = cp.broadcast(timesteps_B_T)
            crossattn_emb = cp.broadcast(crossattn_emb)
        B = x_B_C_T_H_W.shape[0]
        wdt = self.patch_embedding.weight.dtype
        x, (T, H, W) = self.patchify(x_B_C_T_H_W.to(wdt))
        L = T * H * W
        if timesteps_B_T.ndim == 1:
            timesteps_B_T = timesteps_B_T[:, None]
        uniform = timesteps_B_T.shape[1] == 1
        assert uniform or timesteps_B_T.shape[1] == T, "timesteps must be [B, 1] or [B, T]"
        masked = inference_state is not None or (attn_meta is not None and attn_meta.mode != "none")
        if masked and cp is not None:
            raise NotImplementedError("block masks / KV caches run without context parallelism")
        t_off = inference_state.frame_offset() if inference_state is not None else 0
        cos, sin = self.rope_tables(T, H, W, x.device, t_off)
        Ll, r0 = L, 0
        if cp is not None:
            assert L % cp.world == 0, f"L = T*H*W = {L} must be divisible by cp = {cp.world}"
            Ll = L // cp.world
            r0 = cp.rank * Ll
            x = x.view(B, L, -1)[:, r0:r0 + Ll].reshape(B * Ll, -1)
            cos, sin = cos[r0:r0 + Ll].contiguous(), sin[r0:r0 + Ll].contiguous()
        if uniform:
            rpg = Ll
        elif cp is None:
            rpg = H * W
        else:  # per-frame modulation rows: group = b * T + global_row // (H*W)
            gr = torch.arange(r0, r0 + Ll, device=x.device) // (H * W)
            rpg = (torch.arange(B, device=x.device)[:, None] * T + gr[None]).reshape(-1).int()
        x = F.linear(x, self.patch_embedding.weight, self.patch_embedding.bias)
        e, e0 = self.time_embed(timesteps_B_T.reshape(-1))
        context = self.text_embed(crossattn_emb)
        feats = None
        nblocks = len(self.blocks) if stop_after_block is None else stop_after_block + 1
        for i in range(nblocks):
            blk = self.blocks[i]
            actx = None
            if inference_state is not None:
                actx = inference_state.context(i)
            elif masked:
                actx = attn_meta
            if self.training and torch.is_grad_enabled() and i < self.checkpoint_blocks:
                x = checkpoint_block(blk, x, e0, context, cos, sin, B, Ll, rpg, cp, actx, policy=self.checkpoint_policy)
            else:
                x = blk(x, e0, context, cos, sin, B, Ll, rpg, cp, actx)
            if feature_hook_block is not None and i == (feature_hook_block % len(self.blocks)):
                feats = x
        if stop_after_block is not None:
            return x.view(B, Ll, cfg.dim)
        out = self.head(x, e, rpg)
        if cp is not None:
            out = cp.gather(out.view(B, Ll, -1), dim=1).reshape(B * L, -1)
        out = self.unpatchify(out, B, (T, H, W))
        if feature_hook_block is not None:
            return out, feats.view(B, Ll, cfg.dim)
        return out

    def enable_context_parallel(self, cp):
        """Shard the token sequence over ``cp`` (a ``parallel.cp.ContextParallel``); None disables.
        Features returned for the critic are this rank's token slice (pool with ``cp.all_reduce_sum``)."""
        self.cp = cp

    # --------------------------------------------------------------- utilities
    def seg_linears(self):
        return [m for m in self.modules() if isinstance(m, SegLinear)]

    def enable_spectral_norm(self, block_range, power_iters=30) -> int:
        n = 0
        for i in block_range:
            for lin in self.blocks[i].linears():
                n += lin.enable_spectral_norm(power_iters)
        return n

    def enable_lora(self, rank=128, alpha=None, targets=("qkv", "o", "q", "kv", "ffn")):
        """Rank-r LoRA on the block Linears (the reference's to_q/to_k/to_v/to_out/ffn set)."""
        for b in self.blocks:
            b.self_attn.qkv.enable_lora(rank, alpha)
            b.self_attn.o.enable_lora(rank, alpha)
            b.cross_attn.q.enable_lora(rank, alpha)
            b.cross_attn.kv.enable_lora(rank, alpha)
            b.cross_attn.o.enable_lora(rank, alpha)
            getattr(b.ffn, "0").enable_lora(rank, alpha)
            getattr(b.ffn, "2").enable_lora(rank, alpha)
        for n, p in self.named_parameters():
            p.requires_grad_("lora_" in n)
