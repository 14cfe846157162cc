"""Prompt conditioning for the H3 model: a Qwen3-VL language model read at one hidden layer.

Parity: dmad_h3/text_encoder.py:12-66 -- the prompt is tokenised verbatim (no chat template, no special
tokens), run through the Qwen3-VL model as text only, and the hidden state after decoder layer 50
(``hidden_states[50]``, before the final norm) is the conditioning ``prompt_embeds [1, tokens, 5120]``
with ``text_token_tags`` = 1 for every token.

The decoder layers above the one read are never run: while a prompt is encoded the language model's
layer list is cut to ``layer`` entries and its final norm bypassed, so ``last_hidden_state`` *is*
``hidden_states[layer]`` and the 32B model's top 14 layers cost neither time nor (with ``drop_unused``)
memory.  The tokenizer is any callable with the Hugging Face signature
``tokenizer(text, add_special_tokens=False)["input_ids"]``.
"""
from __future__ import annotations

import contextlib
import json
from pathlib import Path

import torch
import torch.nn as nn

TEXT_ENCODER_LAYER = 50
TEXT_TAG = 1


def read_prompts(path) -> list[str]:
    """A UTF-8 ``.txt`` file (one prompt per line) or ``.jsonl`` (one ``{"prompt": ...}`` per line)."""
    with Path(path).expanduser().open("r", encoding="utf-8") as f:
        if str(path).endswith(".jsonl"):
            prompts = [json.loads(line)["prompt"] for line in f if line.strip()]
        else:
            prompts = [line.strip() for line in f if line.strip()]
    if not prompts:
        raise RuntimeError(f"no non-empty prompts in {path}")
    return prompts


def _language_model(model):
    """The text decoder (``embed_tokens``, ``layers``, ``norm``) of a Qwen3-VL model or its inner model."""
    inner = getattr(model, "model", model)
    lm = getattr(inner, "language_model", None)
    if lm is None or not hasattr(lm, "layers"):
        raise TypeError(f"{type(model).__name__} has no Qwen3-VL language model")
    return inner, lm


@contextlib.contextmanager
def _truncated(lm, layer: int):
    n = len(lm.layers)
    if not 0 <= layer <= n:
        raise ValueError(f"hidden layer {layer} outside 0..{n}")
    if layer == n:  # hidden_states[n] is the normed output: run everything
        yield
        return
    layers, norm = lm.layers, lm.norm
    lm.layers, lm.norm = nn.ModuleList(list(layers)[:layer]), nn.Identity()
    try:
        yield
    finally:
        lm.layers, lm.norm = layers, norm


class Qwen3VLConditioner:
    """``encode(prompt) -> {"prompt_embeds": [1, tokens, hidden] (CPU, output_dtype), "text_token_tags":
    [tokens] long}``."""

    def __init__(self, model, tokenizer, layer: int = TEXT_ENCODER_LAYER, processor=None, drop_unused: bool = False,
                 output_dtype=torch.bfloat16):
        self.model = model.requires_grad_(False).eval()
        self.inner, self.lm = _language_model(model)
        self.tokenizer = tokenizer
        self.processor = processor
        self.layer = int(layer)
        self.output_dtype = output_dtype
        if drop_unused and self.layer < len(self.lm.layers):
            # the layers above the one read are never used: free them for good
            self.lm.layers = nn.ModuleList(list(self.lm.layers)[:self.layer])
            self.lm.norm = nn.Identity()

    @classmethod
    def from_pretrained(cls, model_dir, device, dtype=torch.bfloat16, layer: int = TEXT_ENCODER_LAYER,
                        drop_unused: bool = True):
        """Loads ``<model_dir>/{text_encoder,tokenizer,processor}`` of an H3 release (local files only)."""
        from transformers import AutoTokenizer, Qwen3VLForConditionalGeneration

        root = Path(model_dir).expanduser().resolve()
        for sub in ("text_encoder", "tokenizer"):
            if not (root / sub).exists():
                raise FileNotFoundError(f"missing H3 component: {root / sub}")
        kw = {"dtype": dtype, "local_files_only": True}
        if str(device) != "cpu":
            kw["device_map"] = {"": str(device)}
        model = Qwen3VLForConditionalGeneration.from_pretrained(str(root / "text_encoder"), **kw)
        tok = AutoTokenizer.from_pretrained(str(root / "tokenizer"), local_files_only=True)
        proc = None
        if (root / "processor").exists():
            from transformers import AutoProcessor
            proc = AutoProcessor.from_pretrained(str(root / "processor"), local_files_only=True)
        return cls(model, tok, layer, proc, drop_unused)

    @property
    def device(self):
        return next(self.model.parameters()).device

    def inputs(self, prompt: str):
        ids = self.tokenizer(prompt, add_special_tokens=False)["input_ids"]
        if not ids:
            raise ValueError("the tokenizer produced no tokens for a non-empty prompt")
        input_ids = torch.tensor([list(ids)], dtype=torch.long, device=self.device)
        if self.processor is not None and hasattr(self.processor, "create_mm_token_type_ids"):
            mm = torch.tensor(self.processor.create_mm_token_type_ids([list(ids)]), dtype=torch.long,
                              device=self.device)
        else:  # a text-only prompt: every token is text (type 0)
            mm = torch.zeros_like(input_ids)
        return input_ids, mm

    @torch.inference_mode()
    def encode(self, prompt: str) -> dict:
        input_ids, mm = self.inputs(prompt)
        with _truncated(self.lm, self.layer):
            out = self.inner(input_ids=input_ids, attention_mask=torch.ones_like(input_ids), mm_token_type_ids=mm,
                             pixel_values=None, image_grid_thw=None, use_cache=False)
        emb = out.last_hidden_state.to(self.output_dtype).cpu()
        return {"prompt_embeds": emb, "text_token_tags": torch.full((input_ids.shape[1],), TEXT_TAG, dtype=torch.long)}

    def encode_all(self, prompts) -> list[dict]:
        return [self.encode(p) for p in prompts]
