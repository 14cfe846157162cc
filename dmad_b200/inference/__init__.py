"""Few-step sampling API (the ``dmad_h3`` public interface of the reference, dmad_h3/__init__.py:3-25).

H3: geometry, packed layouts, sigma grids, the re-noise / Euler rollout, decoding and muxing,
LoRA files and low-VRAM layer streaming.  Wan: ``cli.wan_sample.sample_bidirectional``.
"""
from .h3 import (H3Geometry, PackedSequence, audio_latent_num_frames, build_packed_sequence, build_row_timesteps,
                 decode_rows, draw_init_noise, latent_shape_of, patchify_video, rollout, shift_sigma, sigma_grid,
                 unpatchify_video, video_latent_num_frames, write_mp4, resolve_transformer_dir, load_transformer)
from .lowmem import LayerStreamer, LowMemH3, LowMemTextEncoder, SafetensorsCatalog, build_streamed_h3
from ..lora import attach_lora, lora_rank_alpha, merge_lora, read_lora_file, save_lora_file

__all__ = ["H3Geometry", "PackedSequence", "audio_latent_num_frames", "build_packed_sequence", "build_row_timesteps",
           "decode_rows", "draw_init_noise", "latent_shape_of", "patchify_video", "rollout", "shift_sigma",
           "sigma_grid", "unpatchify_video", "video_latent_num_frames", "write_mp4", "resolve_transformer_dir", "load_transformer", "LayerStreamer", "LowMemH3",
           "LowMemTextEncoder", "SafetensorsCatalog", "build_streamed_h3",
           "attach_lora", "lora_rank_alpha", "merge_lora", "read_lora_file", "save_lora_file"]
