"""Block-by-block (causal) few-step generation with per-layer KV caches.

Parity: ``sample_causal`` of train/wan/evaluation/vbench_text2video/sample_videos.py:259-370 with the
KV cache and inference state of train/wan/rcm/utils/kv_cache.py.  The latent video is generated one
block of frames at a time (``BlockPattern``: a first chunk, then equal chunks).  Every block is denoised
on its RF grid with the re-noise rule ``x = (1 - t') (x - t v) + t' eps`` (``eps`` drawn once per step
for the whole video and sliced per block, so the result does not depend on the chunking) or the
Euler rule with ``ode``, attending read-only to the cached keys / values of the blocks already
generated; the finished block is then run once more at t = 0 in append mode to commit its keys /
values (or, with ``context_from_last_step``, the last denoising step itself commits them).  Classifier-
free guidance keeps a second set of caches for the unconditional branch.
"""
from __future__ import annotations

import torch

from ..models.kv_cache import CausalInferenceState, KVCacheMode
from ..ops.block_attention import BlockPattern


@torch.no_grad()
def sample_causal(net, noise, t_steps, ctx, first_chunk_frames: int = 1, chunk_frames: int = 1,
                  unctx=None, guidance: float = 1.0, t_steps_per_chunk=None, local_attn_blocks: int = 0,
                  sink_blocks: int = 0, generator=None, ode: bool = False, context_from_last_step: bool = False,
                  context_from_last_step_start_chunk: int = 0):
    """``noise`` [B, C, T, H, W] (latent frames), ``t_steps`` RF grid ending at 0 -> the sample (fp32)."""
    B, _, T, Hh, Ww = noise.shape
    kt, kh, kw = net.cfg.patch_size
    assert kt == 1, "causal generation works on single-frame temporal patches"
    assert (T - first_chunk_frames) % chunk_frames == 0, "frames must fill the chunk pattern"
    ft = (Hh // kh) * (Ww // kw)
    pat = BlockPattern(frame_tokens=ft, first_chunk_frames=first_chunk_frames, chunk_frames=chunk_frames)
    nblocks = 1 + (T - first_chunk_frames) // chunk_frames
    use_cfg = unctx is not None and guidance > 1.0

    def new_state():
        return CausalInferenceState(len(net.blocks), T * ft, pat, local_attn_blocks, sink_blocks)

    cond, uncond = new_state(), (new_state() if use_cfg else None)
    grids = [list(map(float, (t_steps_per_chunk[i] if t_steps_per_chunk else t_steps))) for i in range(nblocks)]
    step_noise = None
    if not ode:
        step_noise = [torch.randn(noise.shape, device=noise.device, generator=generator, dtype=torch.float32)
                      for _ in range(max(len(g) - 1 for g in grids))]
    dt = next(net.parameters()).dtype

    def run(state, c, x, ts):
        return net(x.to(dt), ts, c, inference_state=state)

    blocks = []
    for i in range(nblocks):
        f0 = pat.blocks_to_frames(i)
        f1 = f0 + pat.block_frames(i)
        grid = grids[i]
        last_ctx = context_from_last_step and i >= context_from_last_step_start_chunk
        x = noise[:, :, f0:f1].double() * grid[0]
        for s, (tc, tn) in enumerate(zip(grid[:-1], grid[1:])):
            mode = KVCacheMode.APPEND if (last_ctx and s == len(grid) - 2) else KVCacheMode.READONLY
            ts = torch.full((B, 1), tc * 1000.0, device=noise.device).to(dt).float()
            for st in (cond, uncond):
                if st is not None:
                    st.block_idx, st.mode = i, mode
            v = run(cond, ctx, x, ts).double()
            if use_cfg:
                vu = run(uncond, unctx, x, ts).double()
                v = vu + guidance * (v - vu)
            if ode:
                x = x - (tc - tn) * v
            else:
                x = (1 - tn) * (x - tc * v) + tn * step_noise[s][:, :, f0:f1].double()
        if not last_ctx:
            zero = torch.zeros((B, 1), device=noise.device)
            for st, c in ((cond, ctx), (uncond, unctx)):
                if st is not None:
                    st.block_idx, st.mode = i, KVCacheMode.APPEND
                    run(st, c, x, zero)
        blocks.append(x)
    return torch.cat(blocks, dim=2).float()
