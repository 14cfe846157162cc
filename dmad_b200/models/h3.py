"""MiniMax-H3-shaped joint audio-video DiT over the packed ``[text | stereo audio | video]`` sequence.

The Diffusers ``MiniMaxH3Transformer3DModel`` is not available offline, so this is the H3-*shaped*
network reconstructed from what the reference relies on (dmad_h3/sampling.py:63-98 forward
signature; dmad_h3/lowmem.py:10-12, 416-461, 503-557 block structure and sizes;
tools/convert_lora_comfyui.py:4-16 SwiGLU layout; minimax_h3_dmad_trainer.py:172-175 frozen modules):

* inputs: video rows ``[1, Nv, 24*1*2*2]`` -> ``proj_in``; audio rows ``[1, Na, 32]`` -> ``audio_proj_in``;
  text ``[1, Nt, 5120]`` -> ``context_embedder`` -> ``token_refiner`` (2 blocks, text only);
* timestep: ``time_proj`` (sinusoid of the distinct row timesteps t = 1 - sigma) -> ``time_embedder``;
* 50 ``transformer_blocks``: LayerNorm ``norm1``/``norm2`` with adaLN modulation selected per row
  from a table ``adaln_proj(temb) -> 6 x [n_timesteps * 3 tags, D]`` by ``adaln_indices =
  timestep_index * 3 + token_tag``; attention ``to_q/to_k/to_v`` with per-head RMSNorm ``norm_q/norm_k``,
  3D RoPE over float ``position_ids [L, 3]``, ``to_out.0``; SwiGLU ``ff.net.0.proj`` (``[value; gate]``)
  and ``ff.net.2``;
* outputs: velocities for the video and audio rows (``proj_out``, ``audio_proj_out`` after an adaLN
  ``norm_out``).

Sizes of the 33B configuration (``H3_33B``): hidden 5120, 40 heads of 128, SwiGLU width 15360, 50 blocks,
adaLN projection 2816 -> 6*3*5120 (~0.26 B per block), ~0.345 B per block outside adaLN, which matches
the reference's 0.69 GB-per-block bf16 stream and 13 B of adaLN parameters.  Head count, SwiGLU width,
time-embedding width and the RoPE axis split are inferred, not read from a checkpoint.
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import torch
import torch.nn as nn
import torch.nn.functional as F

from .. import ops
from ..ops import attention as attn_ops
from .layers import SegLinear, install_segment_key_remap
from .sac import checkpoint_block


@dataclass
class H3Config:
    dim: int = 5120
    num_heads: int = 40
    ffn_dim: int = 15360
    num_layers: int = 50
    refiner_layers: int = 2
    in_channels: int = 24
    audio_in_channels: int = 32
    text_dim: int = 5120
    freq_dim: int = 256
    time_embed_dim: int = 2816
    patch_size: tuple = (1, 2, 2)
    num_tags: int = 3
    eps: float = 1e-6
    rope_theta: float = 10000.0

    @property
    def head_dim(self):
        return self.dim // self.num_heads


H3_33B = H3Config()


def rope_angles_from_positions(pos: torch.Tensor, head_dim: int, theta: float = 10000.0) -> torch.Tensor:
    """[L, 3] float positions (t, h, w) -> [L, head_dim/2] angles; axis split as the Wan 3D RoPE
    (dim_h = dim_w = head_dim // 6 * 2, dim_t = rest)."""
    dim_h = head_dim // 6 * 2
    dim_t = head_dim - 2 * dim_h
    dev = pos.device
    f_t = 1.0 / (theta ** (torch.arange(0, dim_t, 2, dtype=torch.float64, device=dev)[: dim_t // 2] / dim_t))
    f_s = 1.0 / (theta ** (torch.arange(0, dim_h, 2, dtype=torch.float64, device=dev)[: dim_h // 2] / dim_h))
    p = pos.to(torch.float64)
    return torch.cat([p[:, 0:1] * f_t, p[:, 1:2] * f_s, p[:, 2:3] * f_s], dim=-1).float()


class _H3Attention(nn.Module):
    def __init__(self, dim, heads, eps):
        super().__init__()
        self.heads, self.head_dim, self.eps = heads, dim // heads, eps
        self.qkv = SegLinear(dim, [("to_q", dim), ("to_k", dim), ("to_v", dim)], flat_name="qkv")
        self.to_out = nn.Module()
        self.to_out.add_module("0", SegLinear(dim, [("0", dim)], flat_name=""))
        self.norm_q = nn.Module()
        self.norm_q.weight = nn.Parameter(torch.ones(self.head_dim))
        self.norm_k = nn.Module()
        self.norm_k.weight = nn.Parameter(torch.ones(self.head_dim))
        install_segment_key_remap(self)

    def forward(self, x, cos, sin, L, cp=None, L_valid=None):
        """x [L, D] (batch 1; this rank's rows under context parallelism) -> [L, D].

        With ``cp`` the rows are one slice of a sequence padded at its end; ``L_valid`` is the
        true global length, so the padded keys are left out of every softmax."""
        H, hd = self.heads, self.head_dim
        D = H * hd
        qkv = self.qkv(x)
        q = ops.rms_norm(qkv[:, :D].reshape(L * H, hd), self.norm_q.weight, self.eps).reshape(L, D)
        k = ops.rms_norm(qkv[:, D:2 * D].reshape(L * H, hd), self.norm_k.weight, self.eps).reshape(L, D)
        if cos is not None:
            q = ops.rope(q, cos, sin, hd)
            k = ops.rope(k, cos, sin, hd)
        v = qkv[:, 2 * D:]
        if cp is not None and cp.world > 1 and torch.is_grad_enabled() and x.requires_grad:
            raise NotImplementedError("H3 context parallelism is inference-only (its exchanges carry no gradient)")
        if cp is not None and cp.world > 1 and cp.impl == "hybrid":
            from ..parallel.cp import hybrid_attention_fwd
            return getattr(self.to_out, "0")(hybrid_attention_fwd(q, k, v, 1, H, cp, L_valid))
        if cp is not None and cp.world > 1:
            # per-head q/k norms and RoPE are row-local, so they run before the head exchange
            g = cp.seq_to_head(torch.cat([q, k, v], dim=1), 1, 3, H, hd)       # [1, Lp, 3, H/cp, hd]
            lv = L_valid if L_valid is not None else g.shape[1]
            o = ops.flash_attention(g[:, :, 0], g[:, :lv, 1], g[:, :lv, 2])
            return getattr(self.to_out, "0")(cp.head_to_seq(o.unsqueeze(2), 1))
        o = ops.flash_attention(q.view(1, L, H, hd), k.view(1, L, H, hd), v.reshape(1, L, H, hd))
        return getattr(self.to_out, "0")(o.reshape(L, D))


class _SwiGLU(nn.Module):
    def __init__(self, dim, ffn_dim):
        super().__init__()
        self.net = nn.Module()
        p0 = nn.Module()
        p0.add_module("proj", SegLinear(dim, [("proj", 2 * ffn_dim)], flat_name=""))
        self.net.add_module("0", p0)
        self.net.add_module("2", SegLinear(ffn_dim, [("2", dim)], flat_name=""))
        self.ffn_dim = ffn_dim

    def forward(self, x):
        h = getattr(self.net, "0").proj(x)
        value, gate = h[:, : self.ffn_dim], h[:, self.ffn_dim:]
        return getattr(self.net, "2")(value * F.silu(gate))


class H3Block(nn.Module):
    def __init__(self, cfg: H3Config, modulated: bool = True):
        super().__init__()
        self.cfg = cfg
        self.modulated = modulated
        self.attn = _H3Attention(cfg.dim, cfg.num_heads, cfg.eps)
        self.ff = _SwiGLU(cfg.dim, cfg.ffn_dim)
        if modulated:
            self.adaln_proj = nn.Linear(cfg.time_embed_dim, 6 * cfg.num_tags * cfg.dim)
        else:
            self.norm1 = nn.LayerNorm(cfg.dim, eps=cfg.eps)
            self.norm2 = nn.LayerNorm(cfg.dim, eps=cfg.eps)

    def adaln_tables(self, temb):
        """temb [T, E] -> [6, T * num_tags, D] fp32 modulation tables."""
        T = temb.shape[0]
        m = F.linear(temb.float(), self.adaln_proj.weight.float(), self.adaln_proj.bias.float())
        return m.view(T, 6, self.cfg.num_tags, self.cfg.dim).permute(1, 0, 2, 3).reshape(6, T * self.cfg.num_tags,
                                                                                          self.cfg.dim)

    def forward(self, h, tables, adaln_idx, cos, sin, cp=None, L_valid=None, temb=None):
        """``tables``: the block's adaLN tables, or None to compute them here from ``temb`` (so that block
        weights bound only while the block runs, as when they are sharded, include the adaLN projection)."""
        L = h.shape[0]
        if self.modulated:
            if tables is None:
                tables = self.adaln_tables(temb)
            sh1, sc1, g1, sh2, sc2, g2 = tables
            x = ops.ln_mod(h, sc1, sh1, a_add=1.0, gidx=adaln_idx, eps=self.cfg.eps)
            h = ops.gate_residual(h, self.attn(x, cos, sin, L, cp, L_valid), g1, gidx=adaln_idx)
            x = ops.ln_mod(h, sc2, sh2, a_add=1.0, gidx=adaln_idx, eps=self.cfg.eps)
            return ops.gate_residual(h, self.ff(x), g2, gidx=adaln_idx)
        x = ops.layer_norm_affine(h, self.norm1.weight, self.norm1.bias, self.cfg.eps)
        h = h + self.attn(x, None, None, L)
        x = ops.layer_norm_affine(h, self.norm2.weight, self.norm2.bias, self.cfg.eps)
        return h + self.ff(x)


class H3Model(nn.Module):
    def __init__(self, cfg: H3Config = H3_33B):
        super().__init__()
        self.cfg = cfg
        D = cfg.dim
        self.patch_size = cfg.patch_size
        self.proj_in = nn.Linear(cfg.in_channels * math.prod(cfg.patch_size), D)
        self.audio_proj_in = nn.Linear(cfg.audio_in_channels, D)
        self.context_embedder = nn.Linear(cfg.text_dim, D)
        self.time_embedder = nn.Sequential(nn.Linear(cfg.freq_dim, cfg.time_embed_dim), nn.SiLU(),
                                           nn.Linear(cfg.time_embed_dim, cfg.time_embed_dim))
        self.token_refiner = nn.Module()
        self.token_refiner.refiner_blocks = nn.ModuleList([H3Block(cfg, modulated=False)
                                                           for _ in range(cfg.refiner_layers)])
        self.transformer_blocks = nn.ModuleList([H3Block(cfg) for _ in range(cfg.num_layers)])
        self.norm_out = nn.Module()
        self.norm_out.linear = nn.Linear(cfg.time_embed_dim, 2 * cfg.num_tags * D)
        self.proj_out = nn.Linear(D, cfg.in_channels * math.prod(cfg.patch_size))
        self.audio_proj_out = nn.Linear(D, cfg.audio_in_channels)
        self.checkpoint_blocks = 0
        self.checkpoint_policy = "block_wise"  # or "mm_only" (keep matmul / attention outputs)
        self._rope_cache = {}
        self.cp = None  # parallel.cp.ContextParallel: shard the packed sequence over a CP group
        self.init_weights()

    @torch.no_grad()
    def init_weights(self):
        for m in self.modules():
            if isinstance(m, (nn.Linear, SegLinear)):
                nn.init.normal_(m.weight, std=0.02)
                if m.bias is not None:
                    nn.init.zeros_(m.bias)
        for b in self.transformer_blocks:
            nn.init.normal_(b.adaln_proj.weight, std=0.002)
        nn.init.zeros_(self.proj_out.weight)
        nn.init.zeros_(self.audio_proj_out.weight)

    # ------------------------------------------------------------------ pieces
    def temb(self, timestep):
        s = ops.sinusoidal_embedding(timestep.float() * 1000.0, self.cfg.freq_dim)
        l0, l2 = self.time_embedder[0], self.time_embedder[2]
        h = ops.small_linear(s, l0.weight, l0.bias)
        return ops.small_linear(h, l2.weight, l2.bias, act_in="silu")

    def refine_text(self, prompt_embeds):
        x = F.linear(prompt_embeds.reshape(-1, prompt_embeds.shape[-1]).to(self.context_embedder.weight.dtype),
                     self.context_embedder.weight, self.context_embedder.bias)
        for blk in self.token_refiner.refiner_blocks:
            x = blk(x, None, None, None, None)
        return x

    def rope_tables(self, position_ids):
        key = (position_ids.data_ptr(), position_ids.shape[0], str(position_ids.device))
        tab = self._rope_cache.get(key)
        if tab is None:
            ang = rope_angles_from_positions(position_ids, self.cfg.head_dim, self.cfg.rope_theta)
            tab = (torch.cos(ang).contiguous(), torch.sin(ang).contiguous())
            self._rope_cache = {key: tab}
        return tab

    # ------------------------------------------------------------------ forward
    def forward(self, hidden_states, audio_hidden_states, encoder_hidden_states, timestep, timestep_indices, token_tags,
                position_ids, video_indices, audio_indices, text_indices, return_dict=False, stop_after_block=None,
                text_features=None, adaln_tables=None):
        """Velocities (video [1, Nv, 96], audio [1, Na, 32]); with ``stop_after_block`` the token
        output [1, L, D] of that block.  ``text_features``: precomputed refiner output (the text sees
        no timestep, so it is the same at every step); ``adaln_tables``: per-block precomputed tables."""
        cfg = self.cfg
        wdt = self.proj_in.weight.dtype
        txt = text_features if text_features is not None else self.refine_text(encoder_hidden_states)
        vid = F.linear(hidden_states[0].to(wdt), self.proj_in.weight, self.proj_in.bias)
        aud = F.linear(audio_hidden_states[0].to(wdt), self.audio_proj_in.weight, self.audio_proj_in.bias)
        # packed order is [text | audio | video] (contiguous index ranges)
        h = torch.cat([txt.to(wdt), aud, vid], dim=0)
        L = h.shape[0]
        adaln_idx = (timestep_indices.long() * cfg.num_tags + token_tags.long()).int()
        temb = self.temb(timestep) if adaln_tables is None else None
        cos, sin = self.rope_tables(position_ids)
        cp = self.cp if (getattr(self, "cp", None) is not None and self.cp.world > 1) else None
        full_idx = adaln_idx
        if cp is not None:
            # pad the packed [text | audio | video] sequence at its end to a multiple of cp and keep
            # this rank's contiguous slice; padded keys are excluded inside attention
            Lp = -(-L // cp.world) * cp.world
            pad = Lp - L
            if pad:
                h = torch.cat([h, h.new_zeros(pad, h.shape[1])])
                adaln_idx = torch.cat([adaln_idx, adaln_idx.new_zeros(pad)])
                cos = torch.cat([cos, cos.new_ones(pad, cos.shape[1])])
                sin = torch.cat([sin, sin.new_zeros(pad, sin.shape[1])])
            Ll = Lp // cp.world
            sl = slice(cp.rank * Ll, (cp.rank + 1) * Ll)
            h, adaln_idx, cos, sin = h[sl], adaln_idx[sl].contiguous(), cos[sl].contiguous(), sin[sl].contiguous()
        n = len(self.transformer_blocks) if stop_after_block is None else stop_after_block + 1
        for i in range(n):
            blk = self.transformer_blocks[i]
            tables = adaln_tables[i] if adaln_tables is not None else None
            if self.training and torch.is_grad_enabled() and i < self.checkpoint_blocks:
                h = checkpoint_block(blk, h, tables, adaln_idx, cos, sin, cp, L, temb, policy=self.checkpoint_policy)
            else:
                h = blk(h, tables, adaln_idx, cos, sin, cp, L, temb)
        if cp is not None:
            h = cp.gather(h[None], dim=1)[0, :L]
            adaln_idx = full_idx
        if stop_after_block is not None:
            return h.view(1, L, cfg.dim)
        if temb is None:
            temb = self.temb(timestep)
        T = temb.shape[0]
        mo = F.linear(temb.float(), self.norm_out.linear.weight.float(), self.norm_out.linear.bias.float())
        mo = mo.view(T, 2, cfg.num_tags, cfg.dim).permute(1, 0, 2, 3).reshape(2, T * cfg.num_tags, cfg.dim)
        ho = ops.ln_mod(h, mo[1], mo[0], a_add=1.0, gidx=adaln_idx, eps=cfg.eps)
        v_out = F.linear(ho[video_indices].float(), self.proj_out.weight.float(), self.proj_out.bias.float())
        a_out = F.linear(ho[audio_indices].float(), self.audio_proj_out.weight.float(),
                         self.audio_proj_out.bias.float())
        return v_out[None], a_out[None]

    # ------------------------------------------------------------------ adapters
    def enable_context_parallel(self, cp):
        """Shard the packed sequence over ``cp`` (a ``parallel.cp.ContextParallel``); None disables."""
        self.cp = cp

    def lora_linears(self, targets=("to_q", "to_k", "to_v", "to_out.0", "ff.net.0.proj", "ff.net.2")):
        out = []
        for b in self.transformer_blocks:
            segs = [s for s in ("to_q", "to_k", "to_v") if s in targets]
            if segs:
                out.append((b.attn.qkv, segs))
            if "to_out.0" in targets:
                out.append((getattr(b.attn.to_out, "0"), None))
            if "ff.net.0.proj" in targets:
                out.append((getattr(b.ff.net, "0").proj, None))
            if "ff.net.2" in targets:
                out.append((getattr(b.ff.net, "2"), None))
        return out

    def enable_lora(self, rank=128, alpha=None, targets=("to_q", "to_k", "to_v", "to_out.0", "ff.net.0.proj", "ff.net.2")):
        for lin, segs in self.lora_linears(targets):
            lin.enable_lora(rank, alpha, segments=segs)
        for n, p in self.named_parameters():
            p.requires_grad_("lora_" in n)
