"""MiniMax-H3 packed text-to-audio-video layout and few-step sampling.

Parity:
* packing: dmad_h3/packing.py:21-143 — padless ``[text | stereo audio | video]`` rows, tags
  (video 0, text 1, audio 2), float64 ``position_ids [L, 3]`` (text: t = index; audio: t = Nt + i,
  width position at the first / last spatial grid value for channel 0 / 1; video: temporal grid with the
  5/3 rescale and the (1, 4, 4, 4, 4) frames-per-latent pattern, centred spatial grid x32), latent
  frames (F - 5) / 17 * 5 + 2 with F = 17 n + 5, audio latents round(F / 24 * 40), row timesteps
  t = 1 - sigma in fp32 with ``torch.unique`` (distinct timesteps + inverse index);
* sampling: dmad_h3/sampling.py:19-98 — shifted sigma grid ``shift*s / (1 + (shift-1) s)``, initial
  noise from one CPU generator (video first, then audio rows) that also supplies the re-noise draws,
  re-noise rule ``x0 = x_t + sigma v; x' = (1 - sigma') x0 + sigma' eps`` and Euler rule
  ``x' = (sigma'/sigma) x_t + (1 - sigma'/sigma) x0``;
* decode / mux: dmad_h3/sampling.py:141-194 — unpatchify rows, latent de-normalisation, pixel
  de-normalisation with the ImageNet mean/std, H.264/AAC mp4 through an ffmpeg subprocess.
"""
from __future__ import annotations

import json
import math
import os
import shutil
import subprocess
import tempfile
from dataclasses import dataclass
from pathlib import Path

import numpy as np
import torch

VIDEO_TAG, TEXT_TAG, AUDIO_TAG = 0, 1, 2
FPS = 24
AUDIO_LATENTS_PER_SECOND = 40
AUDIO_CHANNELS = 2
FRAMES_PER_CHUNK = 17
LATENTS_PER_CHUNK = 5
ROPE_FRAME_RESCALE = 5.0 / 3.0
ROPE_FRAMES_PER_LATENT = (1, 4, 4, 4, 4)
ROPE_SPATIAL_SCALE = 32.0
AUDIO_SAMPLE_RATE = 32000
PIXEL_MEAN = (0.485, 0.456, 0.406)
PIXEL_STD = (0.229, 0.224, 0.225)


@dataclass(frozen=True)
class H3Geometry:
    patch_size: tuple = (1, 2, 2)
    video_latent_channels: int = 24
    audio_latent_channels: int = 32
    vae_spatial_scale_factor: int = 16

    @classmethod
    def from_model_dir(cls, model_dir):
        root = Path(model_dir).expanduser()
        t = json.load(open(root / "transformer" / "config.json"))
        v = json.load(open(root / "vae" / "config.json"))
        return cls(tuple(int(p) for p in t["patch_size"]), int(t["in_channels"]), int(t["audio_in_channels"]),
                   int(math.prod(v["spatial_downsample_factors"])))


def resolve_transformer_dir(path) -> Path:
    """The model root (with ``transformer/``) or the transformer directory itself."""
    path = Path(path).expanduser()
    if (path / "transformer" / "config.json").is_file():
        path = path / "transformer"
    elif not (path / "config.json").is_file():
        raise FileNotFoundError(f"no H3 transformer config below {path}")
    cfg = json.load(open(path / "config.json"))
    if cfg.get("_class_name") not in (None, "MiniMaxH3Transformer3DModel"):
        raise ValueError(f"{path} is not a MiniMaxH3Transformer3DModel checkpoint")
    return path


def config_from_transformer_dir(path):
    """``H3Config`` from a transformer ``config.json`` (keys the file does not name keep the 33B values)."""
    from ..models.h3 import H3Config

    c = json.load(open(resolve_transformer_dir(path) / "config.json"))
    base = H3Config()
    heads = int(c.get("num_attention_heads", base.num_heads))
    hd = int(c.get("attention_head_dim", base.dim // base.num_heads))
    return H3Config(dim=heads * hd, num_heads=heads, ffn_dim=int(c.get("ffn_dim", c.get("intermediate_size", base.ffn_dim))),
                    num_layers=int(c.get("num_layers", base.num_layers)),
                    refiner_layers=int(c.get("num_refiner_layers", base.refiner_layers)),
                    in_channels=int(c.get("in_channels", base.in_channels)),
                    audio_in_channels=int(c.get("audio_in_channels", base.audio_in_channels)),
                    text_dim=int(c.get("text_embed_dim", c.get("text_dim", base.text_dim))),
                    freq_dim=int(c.get("freq_dim", base.freq_dim)),
                    time_embed_dim=int(c.get("time_embed_dim", base.time_embed_dim)),
                    patch_size=tuple(int(p) for p in c.get("patch_size", base.patch_size)))


def load_transformer_weights(model, path, strict: bool = True):
    """Copies the ``*.safetensors`` shards of a transformer directory into ``model``, one shard at a
    time (peak host memory is one shard, tensors land on the parameters' device).  Returns
    ``(missing, unexpected)`` key lists; ``strict`` raises when either is non-empty."""
    from safetensors.torch import load_file

    root = resolve_transformer_dir(path)
    idx = root / "diffusion_pytorch_model.safetensors.index.json"
    if idx.is_file():
        files = sorted({root / f for f in json.load(open(idx))["weight_map"].values()})
    else:
        files = sorted(root.glob("*.safetensors"))
    if not files:
        raise FileNotFoundError(f"no safetensors weights in {root}")
    own = model.state_dict()
    seen, unexpected = set(), []
    with torch.no_grad():
        for f in files:
            for k, v in load_file(str(f)).items():
                if k not in own:
                    unexpected.append(k)
                    continue
                if own[k].shape != v.shape:
                    raise ValueError(f"{k}: checkpoint shape {tuple(v.shape)} != model {tuple(own[k].shape)}")
                own[k].copy_(v)
                seen.add(k)
    missing = [k for k in own if k not in seen]
    if strict and (missing or unexpected):
        raise KeyError(f"H3 weights do not match: {len(missing)} missing (e.g. {missing[:3]}), "
                       f"{len(unexpected)} unexpected (e.g. {unexpected[:3]})")
    return missing, unexpected


def load_transformer(path, dtype=torch.bfloat16, device="cpu", strict: bool = True):
    """This package's H3 network with the weights of a Diffusers-layout transformer directory
    (``config.json`` plus ``*.safetensors`` shards, with or without an index), built on ``device``.

    Parity: dmad_h3/model.py:33-54 (``resolve_transformer_dir`` / ``load_transformer``), which hands the
    folder to the Diffusers class.  Here the tensors are read with ``safetensors`` into ``H3Model``
    under this package's parameter names; a folder written with other names loads with ``strict=False``,
    which returns ``(model, (missing, unexpected))`` instead of raising."""
    from ..models.h3 import H3Model

    cfg = config_from_transformer_dir(path)
    prev = torch.get_default_dtype()
    torch.set_default_dtype(dtype)
    try:
        with torch.device(device):
            model = H3Model(cfg)
    finally:
        torch.set_default_dtype(prev)
    res = load_transformer_weights(model, path, strict)
    model.requires_grad_(False).eval()
    return model if strict else (model, res)


@dataclass(frozen=True)
class PackedSequence:
    sequence_length: int
    position_ids: torch.Tensor
    token_tags: torch.Tensor
    video_indices: torch.Tensor
    audio_indices: torch.Tensor
    text_indices: torch.Tensor

    def to(self, device):
        return PackedSequence(self.sequence_length, self.position_ids.to(device), self.token_tags.to(device),
                              self.video_indices.to(device), self.audio_indices.to(device),
                              self.text_indices.to(device))


def video_latent_num_frames(num_frames: int) -> int:
    if num_frames % FRAMES_PER_CHUNK != LATENTS_PER_CHUNK:
        raise ValueError(f"num_frames must be 17*n+5, got {num_frames}")
    return (num_frames - LATENTS_PER_CHUNK) // FRAMES_PER_CHUNK * LATENTS_PER_CHUNK + 2


def audio_latent_num_frames(num_frames: int) -> int:
    return int(round(num_frames / FPS * AUDIO_LATENTS_PER_SECOND))


def _spatial_grid(dim, patch, sqrt_area):
    ratio = dim / sqrt_area
    left = (1.0 - ratio) / 2.0
    n = dim // patch
    return torch.tensor([(left + ratio * i / n) * ROPE_SPATIAL_SCALE for i in range(n)], dtype=torch.float64)


def _temporal_grid(num_frames, origin):
    spans = torch.tensor([ROPE_FRAME_RESCALE * ROPE_FRAMES_PER_LATENT[i % 5] for i in range(num_frames)],
                         dtype=torch.float64)
    return origin + torch.cat([torch.zeros(1, dtype=torch.float64), spans[:-1].cumsum(0)])


def build_packed_sequence(text_token_tags, num_latent_frames, latent_height, latent_width, num_audio_latents,
                          patch_size=(1, 2, 2)) -> PackedSequence:
    pt, ph, pw = patch_size
    if pt != 1:
        raise ValueError("temporal patch size must be 1")
    if latent_height % ph or latent_width % pw:
        raise ValueError("latent canvas not divisible by the patch")
    tags = torch.as_tensor(text_token_tags, dtype=torch.long).flatten().cpu()
    nt = int(tags.numel())
    per_frame = (latent_height // ph) * (latent_width // pw)
    na = num_audio_latents * AUDIO_CHANNELS
    nv = num_latent_frames * per_frame
    a0, v0 = nt, nt + na
    L = v0 + nv
    pos = torch.zeros(L, 3, dtype=torch.float64)
    pos[:nt, 0] = torch.arange(nt, dtype=torch.float64)
    sqrt_area = math.sqrt(latent_height * latent_width)
    hg = _spatial_grid(latent_height, ph, sqrt_area)
    wg = _spatial_grid(latent_width, pw, sqrt_area)
    grid = torch.stack([a.reshape(-1) for a in torch.meshgrid(hg, wg, indexing="ij")], dim=-1)
    pos[a0:v0, 0] = (float(nt) + torch.arange(num_audio_latents, dtype=torch.float64)).repeat(AUDIO_CHANNELS)
    pos[a0:v0, 2] = torch.cat([torch.full((num_audio_latents,), float(wg[0]), dtype=torch.float64),
                               torch.full((num_audio_latents,), float(wg[-1]), dtype=torch.float64)])
    vp = torch.empty(num_latent_frames, per_frame, 3, dtype=torch.float64)
    vp[:, :, 0] = _temporal_grid(num_latent_frames, float(nt))[:, None]
    vp[:, :, 1:] = grid[None]
    pos[v0:] = vp.reshape(-1, 3)
    ti = torch.arange(nt)
    ai = torch.arange(a0, v0)
    vi = torch.arange(v0, L)
    token_tags = torch.empty(L, dtype=torch.long)
    token_tags[ti] = tags
    token_tags[ai] = AUDIO_TAG
    token_tags[vi] = VIDEO_TAG
    return PackedSequence(L, pos, token_tags, vi, ai, ti)


def build_row_timesteps(layout: PackedSequence, video_sigma, audio_sigma):
    """(distinct timesteps t = 1 - sigma, inverse index per row); the subtraction stays in fp32."""
    vt = float((1.0 - torch.as_tensor(video_sigma, dtype=torch.float32)).item())
    at = float((1.0 - torch.as_tensor(audio_sigma, dtype=torch.float32)).item())
    rows = torch.full((layout.sequence_length,), vt, dtype=torch.float32)
    rows[layout.audio_indices.cpu()] = at
    return torch.unique(rows, sorted=True, return_inverse=True)


def shift_sigma(sigma, shift):
    return shift * sigma / (1.0 + (shift - 1.0) * sigma)


def sigma_grid(steps, shift):
    return shift_sigma(torch.linspace(1.0, 0.0, steps + 1, dtype=torch.float32), shift)


def latent_shape_of(height, width, num_frames, geometry: H3Geometry):
    lf = video_latent_num_frames(num_frames)
    lh, lw = height // geometry.vae_spatial_scale_factor, width // geometry.vae_spatial_scale_factor
    pt, ph, pw = geometry.patch_size
    rows = lf * (lh // ph) * (lw // pw)
    na = audio_latent_num_frames(num_frames)
    return {"num_frames": num_frames, "latent_frames": lf, "latent_height": lh, "latent_width": lw,
            "audio_latents": na, "video_tokens": (1, rows, geometry.video_latent_channels * pt * ph * pw),
            "audio_tokens": (1, na * 2, geometry.audio_latent_channels)}


def patchify_video(z, patch_size):
    """[1, C, T, H, W] latent -> [T*(H/ph)*(W/pw), C*ph*pw] rows (channel-major inside a patch)."""
    _, ph, pw = patch_size
    _, C, T, H, W = z.shape
    x = z[0].reshape(C, T, H // ph, ph, W // pw, pw).permute(1, 2, 4, 0, 3, 5)
    return x.reshape(T * (H // ph) * (W // pw), C * ph * pw)


def unpatchify_video(rows, shape, geometry: H3Geometry):
    _, ph, pw = geometry.patch_size
    C = geometry.video_latent_channels
    t, hh, ww = shape["latent_frames"], shape["latent_height"] // ph, shape["latent_width"] // pw
    z = rows.reshape(t, hh, ww, C, ph, pw).permute(3, 0, 1, 4, 2, 5)
    return z.reshape(1, C, t, hh * ph, ww * pw)


def draw_init_noise(shape, geometry: H3Geometry, seed, device):
    g = torch.Generator(device="cpu").manual_seed(int(seed))
    nv = torch.randn((1, geometry.video_latent_channels, shape["latent_frames"], shape["latent_height"],
                      shape["latent_width"]), generator=g, dtype=torch.float32)
    na = torch.randn((shape["audio_latents"] * 2, geometry.audio_latent_channels), generator=g, dtype=torch.float32)
    return (patchify_video(nv, geometry.patch_size).to(device)[None], na.to(device)[None]), g


@torch.no_grad()
def rollout(transformer, prompt_embeds, layout: PackedSequence, shape, geometry, video_sigmas, audio_sigmas, seed,
            device, renoise=True, text_features=None, adaln_tables_per_step=None):
    """len(sigmas) - 1 student evaluations -> final (video rows, audio rows) x0 on CPU."""
    xt, g = draw_init_noise(shape, geometry, seed, device)
    x0 = None
    lay = layout.to(device)
    for step in range(len(video_sigmas) - 1):
        vs, as_ = video_sigmas[step].to(device), audio_sigmas[step].to(device)
        ts, ti = build_row_timesteps(layout, vs, as_)
        kw = {}
        if text_features is not None:
            kw["text_features"] = text_features
        if adaln_tables_per_step is not None:
            kw["adaln_tables"] = adaln_tables_per_step[step]
        vel = transformer(hidden_states=xt[0], audio_hidden_states=xt[1], encoder_hidden_states=prompt_embeds,
                          timestep=ts.to(device), timestep_indices=ti.to(device), token_tags=lay.token_tags,
                          position_ids=lay.position_ids, video_indices=lay.video_indices,
                          audio_indices=lay.audio_indices, text_indices=lay.text_indices, return_dict=False, **kw)
        x0 = (xt[0] + vs * vel[0].float(), xt[1] + as_ * vel[1].float())
        nv, na = video_sigmas[step + 1].to(device), audio_sigmas[step + 1].to(device)
        if renoise:
            ev = torch.randn(x0[0].shape, generator=g, dtype=torch.float32).to(device)
            ea = torch.randn(x0[1].shape, generator=g, dtype=torch.float32).to(device)
            xt = ((1.0 - nv) * x0[0] + nv * ev, (1.0 - na) * x0[1] + na * ea)
        else:
            rv, ra = nv / vs, na / as_
            xt = (rv * xt[0].float() + (1.0 - rv) * x0[0].float(), ra * xt[1].float() + (1.0 - ra) * x0[1].float())
    return x0[0].float().cpu(), x0[1].float().cpu()


@torch.no_grad()
def decode_rows(vae, audio_vae, video_rows, audio_rows, shape, geometry: H3Geometry, device=None):
    """Rows -> (uint8 frames [T, H, W, 3], float32 waveform [N, 2]).  ``vae`` / ``audio_vae`` are any
    modules with ``decode(z)`` returning pixels in ImageNet-normalised space / waveforms, and
    ``latents_mean`` / ``latents_std`` attributes (per channel)."""
    device = device or video_rows.device
    z = unpatchify_video(video_rows.float().to(device)[0] if video_rows.dim() == 3 else video_rows.float().to(device),
                         shape, geometry)
    vm = torch.as_tensor(vae.latents_mean, device=device).view(1, -1, 1, 1, 1)
    vsd = torch.as_tensor(vae.latents_std, device=device).view(1, -1, 1, 1, 1)
    px = vae.decode(z * vsd + vm)
    pm = torch.tensor(PIXEL_MEAN, device=device).view(3, 1, 1, 1)
    ps = torch.tensor(PIXEL_STD, device=device).view(3, 1, 1, 1)
    frames = ((px[0].float() * ps + pm).clamp(0, 1) * 255.0).round().byte().cpu().numpy().transpose(1, 2, 3, 0)
    za = audio_rows.float().to(device).reshape(1, 2, -1, geometry.audio_latent_channels)[0].permute(0, 2, 1)
    am = torch.as_tensor(audio_vae.latents_mean, device=device).view(1, -1, 1)
    asd = torch.as_tensor(audio_vae.latents_std, device=device).view(1, -1, 1)
    wav = audio_vae.decode(za * asd + am)[:, 0].float().clamp(-1, 1).cpu().numpy().T.astype(np.float32)
    return frames, wav


def write_mp4(frames, wav, out_path, sample_rate=AUDIO_SAMPLE_RATE):
    """Mux rgb24 frames (24 fps) and stereo float32 audio into an H.264/AAC mp4 (bt709).  Without an
    ffmpeg binary the frames and audio are written to ``<out>.npz`` instead (headless fallback)."""
    ffmpeg = shutil.which("ffmpeg")
    out_dir = os.path.dirname(os.path.abspath(out_path))
    os.makedirs(out_dir, exist_ok=True)
    if ffmpeg is None:
        np.savez_compressed(os.path.splitext(out_path)[0] + ".npz", frames=frames, audio=wav, fps=FPS,
                            sample_rate=sample_rate)
        return os.path.splitext(out_path)[0] + ".npz"
    h, w = frames.shape[1], frames.shape[2]
    with tempfile.TemporaryDirectory(dir=out_dir) as tmp:
        vraw, araw = os.path.join(tmp, "video.raw"), os.path.join(tmp, "audio.raw")
        with open(vraw, "wb") as f:
            f.write(np.ascontiguousarray(frames).tobytes())
        with open(araw, "wb") as f:
            f.write(np.ascontiguousarray(wav, dtype=np.float32).tobytes())
        subprocess.run([ffmpeg, "-y", "-hide_banner", "-loglevel", "error", "-f", "rawvideo", "-pix_fmt", "rgb24",
                        "-s", f"{w}x{h}", "-r", str(FPS), "-i", vraw, "-f", "f32le", "-ar", str(sample_rate),
                        "-ac", "2", "-i", araw, "-vf", "scale=in_range=full:out_color_matrix=bt709:out_range=tv",
                        "-colorspace", "bt709", "-color_primaries", "bt709", "-color_trc", "bt709",
                        "-c:v", "libx264", "-crf", "18", "-pix_fmt", "yuv420p", "-c:a", "aac", "-b:a", "160k",
                        "-shortest", out_path], check=True)
    return out_path
