"""Run a DMAD student the way the Diffusers MiniMax-H3 pipeline runs it, on this engine.

Counterpart of the reference's ``run_diffusers_pipeline.py`` (its flags, :32-48, and behaviour, :51-109):
the student LoRA is attached to the base transformer, the sampler takes ``--steps`` model evaluations on
the pipeline's grid of ``steps + 1`` shifted sigma points with the pipeline's Euler step rule (not the
re-noise rule the students were trained with), the video and audio shifts are the student's, and each
prompt is written to ``<output-dir>/<i:04d>.mp4`` (latents when no VAE is available) with its text and a
``settings.json``.  The reference hands these settings to Diffusers' ``ModularPipeline`` and moves idle
components to the CPU with its components manager; here the same settings drive this package's H3
pipeline, whose ``--offload`` is the native block streamer (the reference's block-level group offload).

    python -m dmad_b200.cli.diffusers_pipeline --model-dir /path/to/MiniMax-H3 \\
        --lora dmad_minimax_h3_4step_lora_critic.safetensors --prompt-file prompts.txt --output-dir outputs/diffusers
"""
from __future__ import annotations

import argparse

from . import h3_inference


def parse_args(argv=None):
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--model-dir", required=True, help="MiniMax-H3 model directory (Diffusers layout).")
    p.add_argument("--lora", required=True, help="DMAD student LoRA (.safetensors), attached to the base transformer.")
    p.add_argument("--lora-alpha", type=float)
    p.add_argument("--prompt", action="append", default=[])
    p.add_argument("--prompt-file")
    p.add_argument("--output-dir", required=True)
    p.add_argument("--seed", type=int, default=42)
    p.add_argument("--steps", type=int, default=4, help="Model evaluations (the scheduler gets steps + 1 grid points).")
    p.add_argument("--video-shift", type=float, default=12.0)
    p.add_argument("--audio-shift", type=float, default=2.0)
    p.add_argument("--height", type=int, default=768)
    p.add_argument("--width", type=int, default=1344)
    p.add_argument("--num-frames", type=int, default=124)
    p.add_argument("--offload", action="store_true",
                   help="Stream the transformer to the GPU one block at a time (the native streamer).")
    # not in the reference: runs without checkpoints (random weights of the --config shape)
    p.add_argument("--random-init", action="store_true", help=argparse.SUPPRESS)
    p.add_argument("--config", default="33b", choices=["33b", "tiny"], help=argparse.SUPPRESS)
    p.add_argument("--text-tokens", type=int, default=256, help=argparse.SUPPRESS)
    return p.parse_args(argv)


def to_h3_inference_args(a) -> list[str]:
    """The ``h3_inference`` command line with the same settings and the Euler step rule."""
    out = ["--model-dir", a.model_dir, "--lora", a.lora, "--output-dir", a.output_dir, "--seed", str(a.seed),
           "--steps", str(a.steps), "--video-shift", str(a.video_shift), "--audio-shift", str(a.audio_shift),
           "--height", str(a.height), "--width", str(a.width), "--num-frames", str(a.num_frames), "--euler",
           "--config", a.config, "--text-tokens", str(a.text_tokens)]
    if a.lora_alpha is not None:
        out += ["--lora-alpha", str(a.lora_alpha)]
    for pr in a.prompt:
        out += ["--prompt", pr]
    if a.prompt_file:
        out += ["--prompt-file", a.prompt_file]
    if a.offload:
        out += ["--low-vram", "auto"]
    if a.random_init:
        out += ["--random-init"]
    return out


def main(argv=None):
    a = parse_args(argv)
    if not a.prompt and not a.prompt_file:
        raise SystemExit("give --prompt and/or --prompt-file")
    return h3_inference.main(to_h3_inference_args(a))


if __name__ == "__main__":
    main()
