"""Building blocks shared by the DiT models.

``SegLinear``
    One GEMM for several logical Linear layers that read the same input (q/k/v
    of self-attention, k/v of cross-attention).  The weight is stored fused
    ``[sum(out_i), in]`` but the state dict keeps one ``<name>.weight`` /
    ``<name>.bias`` pair per segment, so checkpoints use the reference's key
    layout (e.g. ``blocks.0.self_attn.q.weight``, train/wan/rcm/networks/wan2pt1.py:237-242).
    Each segment can carry
      * a frozen-gain spectral norm, ``W_eff = W * gain / sigma_max(W)`` with one
        power iteration per training forward and ``gain`` frozen at the initial
        ``sigma_max`` (train/wan/rcm/models/t2v_model_distill_dmad.py:488-517,
        train/image/main/edm/edm_guidance.py:54-80);
      * a rank-r LoRA adapter ``W x + (alpha/r) B A x`` in the Diffusers/PEFT
        layout (dmad_h3/lora.py:23-75).
``SelfAttnCore`` / ``CrossAttnCore``
    autograd functions that run q/k RMSNorm (+3D RoPE) and flash attention on
    the sm_100a kernels and produce the fused ``dqkv`` gradient directly.
"""
from __future__ import annotations

import math
from typing import Sequence

import torch
import torch.nn as nn
import torch.nn.functional as F

from .. import ops
from ..ops import attention as attn_ops
from ..ops import norm as norm_ops


# ----------------------------------------------------------------------------- spectral norm helpers


def _l2n(x, eps=1e-12):
    return x / x.norm().clamp_min(eps)


class _SNWeight(torch.autograd.Function):
    """W -> bf16(W * gain_s / sigma_s) on the fused CUDA kernels; ``u`` [O] and ``v`` [nseg, I] (fp32) are
    the power-iteration state, updated in place when ``train``."""

    @staticmethod
    def forward(ctx, w, u, v, gain, offsets, on, train):
        from ..ops import ext
        scale = torch.empty(w.shape[0], dtype=torch.float32, device=w.device)
        sigma = torch.empty(len(on), dtype=torch.float32, device=w.device)
        out = ext().sn_weight_fwd(w, u, v, gain, scale, sigma, offsets, on, bool(train))
        ctx.save_for_backward(w, u.clone(), v.clone(), gain, scale, sigma)
        ctx.meta = (offsets, on)
        return out

    @staticmethod
    def backward(ctx, g):
        from ..ops import ext
        w, u, v, gain, scale, sigma = ctx.saved_tensors
        if g.stride(-1) != 1 or g.stride(0) % 8 or g.data_ptr() % 16:
            g = g.contiguous()
        dw = ext().sn_weight_bwd(g, w, u, v, gain, scale, sigma, *ctx.meta)
        return dw, None, None, None, None, None, None


class SegLinear(nn.Module):
    def __init__(self, in_features: int, segments: Sequence[tuple[str, int]], bias: bool = True, flat_name: str = ""):
        super().__init__()
        self.in_features = in_features
        self.segments = [(n, int(o)) for n, o in segments]
        self.out_features = sum(o for _, o in self.segments)
        self.flat_name = flat_name
        self.weight = nn.Parameter(torch.empty(self.out_features, in_features))
        self.bias = nn.Parameter(torch.zeros(self.out_features)) if bias else None
        self.sn_enabled = False
        self.lora_rank = 0
        self.lora_scale = 0.0
        nn.init.xavier_uniform_(self.weight)

    # ------------------------------------------------------------------ segments
    def seg_slices(self):
        off = 0
        for name, o in self.segments:
            yield name, slice(off, off + o)
            off += o

    def seg_weight(self, name):
        for n, sl in self.seg_slices():
            if n == name:
                return self.weight[sl]
        raise KeyError(name)

    # ------------------------------------------------------------------ spectral norm
    @torch.no_grad()
    def enable_spectral_norm(self, power_iters: int = 30, segments: Sequence[str] | None = None) -> int:
        """Registers the frozen-gain spectral norm on every (or the named) segment.

        Returns the number of segments wrapped.  Zero-initialised segments are
        skipped (sigma would be 0), as the reference does.
        """
        n = 0
        dev = self.weight.device
        us, vs, gains, mask = [], [], [], []
        g = torch.Generator(device="cpu").manual_seed(0)
        for name, sl in self.seg_slices():
            w = self.weight[sl].float()
            u = _l2n(torch.randn(w.shape[0], generator=g).to(dev))
            v = _l2n(torch.randn(w.shape[1], generator=g).to(dev))
            on = False
            if segments is None or name in segments:
                # the power iteration's sigma decides (no SVD: a zero segment gives sigma = 0)
                ui, vi = u, v
                for _ in range(power_iters):
                    vi = _l2n(w.t() @ ui)
                    ui = _l2n(w @ vi)
                sigma = torch.dot(ui, w @ vi)
                on = float(sigma) >= 1e-8
                if on:
                    u, v = ui, vi
            if on:
                wn = w / sigma
                gain = (w.flatten() @ wn.flatten()) / (wn.flatten() @ wn.flatten())
                n += 1
            else:
                gain = torch.tensor(1.0, device=dev)
            us.append(u)
            vs.append(v)
            gains.append(gain.reshape(1))
            mask.append(on)
        self.register_buffer("sn_u", torch.cat(us), persistent=True)
        self.register_buffer("sn_v", torch.stack(vs), persistent=True)
        self.register_buffer("sn_gain", torch.cat(gains).float(), persistent=True)
        self.register_buffer("sn_mask", torch.tensor(mask, dtype=torch.bool, device=dev), persistent=True)
        self._sn_on = list(mask)  # host copy of sn_mask: reading the device tensor would wait for the GPU
        self.sn_enabled = n > 0
        return n

    def _sn_segments_on(self):
        """Which segments carry the spectral norm, from the host copy of ``sn_mask`` (refreshed when a
        state dict is loaded), so that the forward never reads a device tensor back."""
        if getattr(self, "_sn_on", None) is None:
            self._sn_on = [bool(b) for b in self.sn_mask.tolist()]
        return self._sn_on

    def _sn_row_scale(self):
        """Per-output-row scale gain/sigma (differentiable in W through sigma = u^T W v)."""
        w = self.weight
        scales = []
        on = self._sn_segments_on()
        for i, (name, sl) in enumerate(self.seg_slices()):
            o = sl.stop - sl.start
            if not on[i]:
                scales.append(torch.ones(o, device=w.device, dtype=torch.float32))
                continue
            ws = w[sl].float()
            u = self.sn_u[sl].float()
            v = self.sn_v[i].float()
            if self.training:
                with torch.no_grad():
                    v = _l2n(ws.t() @ u)
                    u = _l2n(ws @ v)
                    self.sn_u[sl].copy_(u)
                    self.sn_v[i].copy_(v)
            sigma = torch.dot(u, ws @ v)
            scales.append((self.sn_gain[i].float() / sigma).expand(o))
        return torch.cat(scales)

    def effective_weight(self):
        if not self.sn_enabled:
            return self.weight
        if (self.weight.is_cuda and self.weight.dtype == torch.bfloat16 and self.in_features % 8 == 0
                and len(self.segments) <= 8):
            return self._sn_weight_fused()  # fused kernels: power iteration, scaled weight and its gradient
        return (self.weight.float() * self._sn_row_scale()[:, None]).to(self.weight.dtype)

    def _sn_weight_fused(self):
        """``effective_weight`` through the fused spectral-norm kernels (the math of ``_sn_row_scale``:
        one power iteration per training forward, sigma differentiable in W with u, v held constant)."""
        on = [int(b) for b in self._sn_segments_on()]
        offs = [0]
        for _, sl in self.seg_slices():
            offs.append(sl.stop)
        u32 = self.sn_u if self.sn_u.dtype == torch.float32 else self.sn_u.float()
        v32 = self.sn_v if self.sn_v.dtype == torch.float32 else self.sn_v.float()
        if getattr(self, "_sn_gain32", None) is None:
            self._sn_gain32 = self.sn_gain.float().contiguous().clone()
        w = self.weight
        if w.stride(-1) != 1 or w.stride(0) % 8 or w.data_ptr() % 16:
            w = w.contiguous()
        w_eff = _SNWeight.apply(w, u32, v32, self._sn_gain32, offs, on, self.training)
        if self.training and u32 is not self.sn_u:
            with torch.no_grad():
                self.sn_u.copy_(u32)
                self.sn_v.copy_(v32)
        return w_eff

    @torch.no_grad()
    def folded_weight(self):
        """Weight with the frozen-gain spectral norm folded in: per segment one power iteration
        from the stored u (v = W^T u / |.|, u' = W v / |.|, sigma = u'^T W v), W * gain / sigma,
        as the release converter does (train/wan/scripts/dcp_to_pth_dmad.py:180-209)."""
        if not self.sn_enabled:
            return self.weight.detach().clone()
        w = self.weight.detach().float().clone()
        on = self._sn_segments_on()
        for i, (name, sl) in enumerate(self.seg_slices()):
            if not on[i]:
                continue
            ws = w[sl]
            v = _l2n(ws.t() @ self.sn_u[sl].float())
            u = _l2n(ws @ v)
            sigma = torch.dot(u, ws @ v)
            w[sl] = ws * (self.sn_gain[i].float() / sigma)
        return w.to(self.weight.dtype)

    # ------------------------------------------------------------------ LoRA
    def enable_lora(self, rank: int, alpha: float | None = None, segments: Sequence[str] | None = None):
        """Adds a LoRA adapter (A: [r, in] per segment, B: [out, r]) initialised so the output is unchanged."""
        self.lora_rank = int(rank)
        self.lora_alpha = float(alpha if alpha is not None else rank)
        self.lora_scale = self.lora_alpha / self.lora_rank
        self.lora_segments = [n for n, _ in self.segments] if segments is None else list(segments)
        # a weight left on the meta device (streamed from a checkpoint) gets host adapters
        dev = self.weight.device if self.weight.device.type != "meta" else torch.device("cpu")
        nseg = len(self.lora_segments)
        self.lora_A = nn.Parameter(torch.empty(nseg * rank, self.in_features, device=dev, dtype=self.weight.dtype))
        self.lora_B = nn.Parameter(torch.zeros(self.out_features, nseg * rank, device=dev, dtype=self.weight.dtype))
        for i in range(nseg):
            nn.init.kaiming_uniform_(self.lora_A.data[i * rank:(i + 1) * rank], a=math.sqrt(5))
        # block-diagonal structure: segment s only sees its own rank block
        mask = torch.zeros(self.out_features, nseg * rank, dtype=torch.bool, device=dev)
        for name, sl in self.seg_slices():
            if name in self.lora_segments:
                j = self.lora_segments.index(name)
                mask[sl, j * rank:(j + 1) * rank] = True
        self.register_buffer("lora_mask", mask, persistent=False)

    def lora_delta_weight(self):
        return self.lora_scale * (self.lora_B * self.lora_mask) @ self.lora_A

    # ------------------------------------------------------------------ forward
    def forward_rows(self, x, start: int, stop: int):
        """Output columns ``[start, stop)`` of ``forward(x)``, computed from those weight rows only
        (one segment of a fused projection, for instance)."""
        w = self.effective_weight()[start:stop]
        b = None if self.bias is None else self.bias[start:stop]
        if x.dtype != w.dtype:
            x = x.to(w.dtype)
        if self.lora_rank:
            bm = (self.lora_B * self.lora_mask)[start:stop]
            if x.is_cuda:
                from ..ops.linear import lora_linear
                return lora_linear(x, w, b, self.lora_A, bm, self.lora_scale)
            return F.linear(x, w, b) + self.lora_scale * F.linear(F.linear(x, self.lora_A), bm)
        return F.linear(x, w, b)

    def forward(self, x):
        w = self.effective_weight()
        b = self.bias
        if x.dtype != w.dtype:
            x = x.to(w.dtype)
        if self.lora_rank:
            if x.is_cuda:  # one tcgen05 GEMM over [x | s x A^T] [W | B o mask]^T
                from ..ops.linear import lora_linear
                return lora_linear(x, w, b, self.lora_A, self.lora_B * self.lora_mask, self.lora_scale)
            y = F.linear(x, w, b)
            return y + self.lora_scale * F.linear(F.linear(x, self.lora_A), self.lora_B * self.lora_mask)
        return F.linear(x, w, b)

    # ------------------------------------------------------------------ state dict (per-segment keys)
    def _split_prefix(self, prefix):
        if self.flat_name and prefix.endswith(self.flat_name + "."):
            return prefix[: -len(self.flat_name) - 1]
        return prefix

    def _save_to_state_dict(self, destination, prefix, keep_vars):
        base = self._split_prefix(prefix)
        w = self.weight if keep_vars else self.weight.detach()
        for i, (name, sl) in enumerate(self.seg_slices()):
            key = f"{base}{name}." if self.flat_name else f"{prefix}"
            destination[key + "weight"] = w[sl]
            if self.bias is not None:
                destination[key + "bias"] = (self.bias if keep_vars else self.bias.detach())[sl]
            if self.sn_enabled:
                destination[key + "sn_u"] = self.sn_u[sl]
                destination[key + "sn_v"] = self.sn_v[i]
                destination[key + "sn_gain"] = self.sn_gain[i:i + 1]
                destination[key + "sn_mask"] = self.sn_mask[i:i + 1]
        if self.lora_rank:
            r = self.lora_rank
            for name, sl in self.seg_slices():
                if name not in self.lora_segments:
                    continue
                j = self.lora_segments.index(name)
                key = f"{base}{name}." if self.flat_name else f"{prefix}"
                destination[key + "lora_A.weight"] = self.lora_A.detach()[j * r:(j + 1) * r]
                destination[key + "lora_B.weight"] = self.lora_B.detach()[sl, j * r:(j + 1) * r]

    def _load_from_state_dict(self, state_dict, prefix, local_metadata, strict, missing_keys, unexpected_keys, error_msgs):
        # keys arrive as <prefix><segment>.<name> (the parent's pre-hook maps the reference's
        # <parent>.<segment>.<name> layout under this module's prefix; see install_segment_key_remap)
        with torch.no_grad():
            consumed = set()
            for i, (name, sl) in enumerate(self.seg_slices()):
                key = f"{prefix}{name}." if self.flat_name else f"{prefix}"
                for pname, target in (("weight", self.weight), ("bias", self.bias)):
                    if target is None:
                        continue
                    k = key + pname
                    if k in state_dict:
                        target[sl].copy_(state_dict[k])
                        consumed.add(k)
                    elif strict:
                        missing_keys.append(k)
                if self.sn_enabled and key + "sn_u" in state_dict:
                    u = state_dict[key + "sn_u"]
                    self.sn_u[sl].copy_(u.reshape(-1))
                    if key + "sn_v" in state_dict:
                        self.sn_v[i].copy_(state_dict[key + "sn_v"])
                    else:  # a source that stores only u (the reference's parametrization export)
                        self.sn_v[i].copy_(_l2n(self.weight[sl].float().t() @ u.float().reshape(-1)))
                    self.sn_gain[i:i + 1].copy_(state_dict[key + "sn_gain"].reshape(1))
                    # a stored power-iteration state means the layer is spectrally normed
                    self.sn_mask[i:i + 1].copy_(state_dict.get(key + "sn_mask", torch.ones(1, dtype=torch.bool)))
                    self._sn_on = None  # re-read from the loaded mask on the next forward
                    self._sn_gain32 = None
                    consumed.update(key + n for n in ("sn_u", "sn_v", "sn_gain", "sn_mask"))
                if self.lora_rank and name in self.lora_segments:
                    r = self.lora_rank
                    j = self.lora_segments.index(name)
                    if key + "lora_A.weight" in state_dict:
                        self.lora_A[j * r:(j + 1) * r].copy_(state_dict[key + "lora_A.weight"])
                        self.lora_B[sl, j * r:(j + 1) * r].copy_(state_dict[key + "lora_B.weight"])
                        consumed.update((key + "lora_A.weight", key + "lora_B.weight"))
            for k in state_dict:
                if k.startswith(prefix) and k not in consumed and strict:
                    unexpected_keys.append(k)


def install_segment_key_remap(parent: nn.Module):
    """Maps the per-segment keys of the reference layout (``<parent>.q.weight``) onto the fused
    SegLinear children (``<parent>.qkv.q.weight``) when ``parent`` loads a state dict."""
    fused = {name: child for name, child in parent.named_children() if isinstance(child, SegLinear) and child.flat_name}

    def hook(state_dict, prefix, *args):
        for cname, child in fused.items():
            for seg, _ in child.segments:
                for k in list(state_dict.keys()):
                    head = f"{prefix}{seg}."
                    if k.startswith(head):
                        state_dict[f"{prefix}{cname}.{seg}." + k[len(head):]] = state_dict.pop(k)

    parent._register_load_state_dict_pre_hook(hook)


# ----------------------------------------------------------------------------- attention cores


class _SelfAttnCore(torch.autograd.Function):
    """qkv [R, 3D] (pre-norm) -> attention output [R, D].

    Forward: RMSNorm(q), RMSNorm(k) over D, interleaved RoPE, flash attention.
    Only qkv, the two rstd vectors, O and the LSE are kept; the normalised,
    rotated q/k are recomputed in backward (one elementwise pass) instead of
    being stored.
    """

    @staticmethod
    def forward(ctx, qkv, wq, wk, cos, sin, B, L, H, eps):
        R, D3 = qkv.shape
        D = D3 // 3
        hd = D // H
        qk, rq, rk = norm_ops.qk_norm_rope(qkv, wq, wk, cos, sin, D, hd, eps)
        q = qk[:, :D].view(B, L, H, hd)
        k = qk[:, D:].view(B, L, H, hd)
        v = qkv[:, 2 * D:].view(B, L, H, hd)
        scale = 1.0 / math.sqrt(hd)
        o, lse = attn_ops.flash_attn_fwd(q, k, v, scale)
        ctx.save_for_backward(qkv, wq, wk, cos, sin, rq, rk, o, lse)
        ctx.cfg = (B, L, H, hd, D, eps, scale)
        return o.view(R, D)

    @staticmethod
    def backward(ctx, do):
        qkv, wq, wk, cos, sin, rq, rk, o, lse = ctx.saved_tensors
        B, L, H, hd, D, eps, scale = ctx.cfg
        e = ops.ext()
        R = qkv.shape[0]
        qk, _, _ = norm_ops.qk_norm_rope(qkv, wq, wk, cos, sin, D, hd, eps)
        do = do.contiguous()
        dqkv = torch.empty_like(qkv)
        dqk = torch.empty((R, 2 * D), dtype=qkv.dtype, device=qkv.device)
        dd = torch.empty_like(lse)
        attn_ops.flash_bwd_into(qk[:, :D].view(B, L, H, hd), qk[:, D:].view(B, L, H, hd), qkv[:, 2 * D:].view(B, L, H, hd), o,
                    do.view(B, L, H, hd), lse, dqk[:, :D].view(B, L, H, hd), dqk[:, D:].view(B, L, H, hd),
                    dqkv[:, 2 * D:].view(B, L, H, hd), dd, scale)
        dwq = torch.zeros(D, dtype=torch.float32, device=qkv.device)
        dwk = torch.zeros(D, dtype=torch.float32, device=qkv.device)
        e.qk_norm_rope_bwd(dqk[:, :D], dqk[:, D:], qkv, dqkv, wq, wk, cos, sin, rq, rk, dwq, dwk, D, hd)
        return dqkv, dwq, dwk, None, None, None, None, None, None


def self_attention_core(qkv, wq, wk, cos, sin, B, L, H, eps=1e-6):
    """Self-attention of the Wan / H3 blocks on a fused [R, 3D] projection."""
    if not qkv.is_cuda:
        R, D3 = qkv.shape
        D = D3 // 3
        hd = D // H
        q = norm_ops.ln_mod_reference(qkv[:, :D], wq.reshape(1, -1), None, 0.0, None, None, eps, True)
        k = norm_ops.ln_mod_reference(qkv[:, D:2 * D], wk.reshape(1, -1), None, 0.0, None, None, eps, True)
        if cos is not None:
            q = norm_ops.rope_reference(q, cos, sin, hd)
            k = norm_ops.rope_reference(k, cos, sin, hd)
        v = qkv[:, 2 * D:]
        o = attn_ops.attention_reference(q.view(B, L, H, hd), k.view(B, L, H, hd), v.reshape(B, L, H, hd))
        return o.reshape(R, D)
    return _SelfAttnCore.apply(qkv, wq.float().contiguous(), wk.float().contiguous(), cos, sin, B, L, H, eps)


class _CrossAttnCore(torch.autograd.Function):
    """cq [R, D], ckv [Rc, 2D] (pre-norm) -> [R, D]; RMSNorm on q and k, no RoPE."""

    @staticmethod
    def forward(ctx, cq, ckv, wq, wk, B, L, Lc, H, eps):
        R, D = cq.shape
        hd = D // H
        qn, rq = _rms_fwd(cq, wq, eps)
        kn, rk = _rms_fwd(ckv[:, :D], wk, eps)
        scale = 1.0 / math.sqrt(hd)
        o, lse = attn_ops.flash_attn_fwd(qn.view(B, L, H, hd), kn.view(B, Lc, H, hd), ckv[:, D:].view(B, Lc, H, hd),
                                         scale)
        ctx.save_for_backward(cq, ckv, wq, wk, rq, rk, o, lse)
        ctx.cfg = (B, L, Lc, H, hd, D, eps, scale)
        return o.view(R, D)

    @staticmethod
    def backward(ctx, do):
        cq, ckv, wq, wk, rq, rk, o, lse = ctx.saved_tensors
        B, L, Lc, H, hd, D, eps, scale = ctx.cfg
        e = ops.ext()
        qn, _ = _rms_fwd(cq, wq, eps)
        kn, _ = _rms_fwd(ckv[:, :D], wk, eps)
        do = do.contiguous()
        dqn = torch.empty_like(qn)
        dkn = torch.empty_like(kn)
        dckv = torch.empty_like(ckv)
        dd = torch.empty_like(lse)
        attn_ops.flash_bwd_into(qn.view(B, L, H, hd), kn.view(B, Lc, H, hd), ckv[:, D:].view(B, Lc, H, hd), o,
                    do.view(B, L, H, hd), lse, dqn.view(B, L, H, hd), dkn.view(B, Lc, H, hd),
                    dckv[:, D:].view(B, Lc, H, hd), dd, scale)
        dcq = torch.empty_like(cq)
        dwq = torch.zeros((1, D), dtype=torch.float32, device=cq.device)
        dwk = torch.zeros((1, D), dtype=torch.float32, device=cq.device)
        e.ln_mod_bwd(dqn, cq, None, rq, wq.view(1, D), 0.0, max(cq.shape[0], 1), None, True, dcq, None, dwq, None,
                     None, None, None, None)
        dk_view = dckv[:, :D]
        e.ln_mod_bwd(dkn, ckv[:, :D], None, rk, wk.view(1, D), 0.0, max(ckv.shape[0], 1), None, True, dk_view, None,
                     dwk, None, None, None, None, None)
        return dcq, dckv, dwq.view(D), dwk.view(D), None, None, None, None, None


def _rms_fwd(x, w, eps):
    R, D = x.shape
    y = torch.empty((R, D), dtype=x.dtype, device=x.device)
    rstd = torch.empty(R, dtype=torch.float32, device=x.device)
    ops.ext().ln_mod_fwd(x, y, None, rstd, w.view(1, D), None, 0.0, max(R, 1), None, float(eps), True)
    return y, rstd


def cross_attention_core(cq, ckv, wq, wk, B, L, Lc, H, eps=1e-6):
    """Cross-attention of the Wan blocks: q from the video tokens, k/v from the text context."""
    if not cq.is_cuda:
        R, D = cq.shape
        hd = D // H
        q = norm_ops.ln_mod_reference(cq, wq.reshape(1, -1), None, 0.0, None, None, eps, True)
        k = norm_ops.ln_mod_reference(ckv[:, :D], wk.reshape(1, -1), None, 0.0, None, None, eps, True)
        v = ckv[:, D:]
        o = attn_ops.attention_reference(q.view(B, L, H, hd), k.view(B, Lc, H, hd), v.reshape(B, Lc, H, hd))
        return o.reshape(R, D)
    return _CrossAttnCore.apply(cq, ckv, wq.float().contiguous(), wk.float().contiguous(), B, L, Lc, H, eps)
