"""Synthetic batches of the benchmark shapes (N(0,1) latents and text embeddings).

Every rank of a context-parallel group draws the same sample (seeded by the data-parallel rank),
so the group works on one sample as the reference's CP broadcast arranges.
"""
from __future__ import annotations

import torch


class SyntheticWanData:
    def __init__(self, latent_shape=(16, 21, 60, 104), text_shape=(512, 4096), batch_size: int = 1, dp_rank: int = 0,
                 seed: int = 1234, fixed: bool = True, with_negative: bool = False, start_iteration: int = 0):
        self.latent_shape, self.text_shape = tuple(latent_shape), tuple(text_shape)
        self.batch_size, self.with_negative = batch_size, with_negative
        self.seed, self.dp_rank = seed, dp_rank
        self.gen = torch.Generator()
        self.fixed = fixed
        self.iteration = start_iteration  # batch i is a function of (seed, dp rank, i): resumable
        self._cached = None

    def _draw(self):
        self.gen.manual_seed(self.seed + 1000 * self.dp_rank + 1_000_003 * (0 if self.fixed else self.iteration))
        self.iteration += 1
        B = self.batch_size
        b = {"latents": torch.randn((B,) + self.latent_shape, generator=self.gen),
             "real_latents": torch.randn((B,) + self.latent_shape, generator=self.gen),
             "context": torch.randn((B,) + self.text_shape, generator=self.gen).to(torch.bfloat16)}
        if self.with_negative:
            b["neg_context"] = torch.zeros((B,) + self.text_shape, dtype=torch.bfloat16)
        return b

    def __iter__(self):
        while True:
            if self.fixed:
                if self._cached is None:
                    self._cached = self._draw()
                yield self._cached
            else:
                yield self._draw()
