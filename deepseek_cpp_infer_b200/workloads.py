"""Seeded synthetic inputs with the shapes of the benchmark configurations.

No checkpoint or dataset is available offline, so every workload is drawn from
seeded generators with the configuration's shapes and value distributions.
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import numpy as np


@dataclass
class MlaCase:
    """Inputs of one absorbed-MLA decode call over a paged latent cache."""

    q_lat: object  # torch bf16 [B, H, R] on the device
    q_rope: object  # torch bf16 [B, H, P]
    cache: object  # torch bf16 [n_blocks, 64, R + P]
    block_table: object  # torch int32 [B, max_blocks] on the device
    block_table_host: np.ndarray
    seq_lens: np.ndarray  # int32 [B] (host)
    scale: float
    B: int
    H: int
    R: int
    P: int

    @property
    def kv_bytes(self) -> int:
        """Cache bytes one call must read: every token's [c | kr] row once."""
        return int(self.seq_lens.sum()) * (self.R + self.P) * 2

    @property
    def algorithmic_bytes(self) -> int:
        """KV rows + q (read) + latent output (written), bf16."""
        return self.kv_bytes + self.B * self.H * (self.R + self.P) * 2 + self.B * self.H * self.R * 2

    @property
    def flops(self) -> int:
        return int(sum(2 * self.H * int(L) * ((self.R + self.P) + self.R) for L in self.seq_lens))


def mla_case(B=64, H=128, R=512, P=64, lens=None, ctx_lo=1024, ctx_hi=8192, seed=1, device="cuda",
             nope=128, extra_blocks=0) -> MlaCase:
    """The isolated MLA decode workload: per-sequence lengths uniform in
    [ctx_lo, ctx_hi] (or `lens`), page size 64, block table a random
    permutation of all pages, q and cache N(0, 1) in bf16, scale 1/sqrt(nope+P)."""
    import torch

    rng = np.random.default_rng(seed)
    if lens is None:
        lens = rng.integers(ctx_lo, ctx_hi + 1, size=B)
    lens = np.asarray(lens, np.int32)
    B = len(lens)
    pages = (lens + 63) // 64
    max_blocks = int(pages.max())
    n_blocks = int(pages.sum()) + extra_blocks
    perm = rng.permutation(n_blocks).astype(np.int32)
    bt = np.zeros((B, max_blocks), np.int32)
    k = 0
    for b in range(B):
        bt[b, : pages[b]] = perm[k : k + pages[b]]
        k += pages[b]
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    q_lat = torch.randn(B, H, R, generator=g, device=device, dtype=torch.float32).to(torch.bfloat16)
    q_rope = torch.randn(B, H, P, generator=g, device=device, dtype=torch.float32).to(torch.bfloat16)
    cache = torch.randn(n_blocks, 64, R + P, generator=g, device=device, dtype=torch.float32).to(torch.bfloat16)
    return MlaCase(q_lat, q_rope, cache, torch.from_numpy(bt).to(device), bt, lens, 1.0 / math.sqrt(nope + P), B, H,
                   R, P)


def to_u16(t) -> np.ndarray:
    """A torch bf16 tensor as a host uint16 array (bit pattern preserved)."""
    import torch

    return t.detach().contiguous().view(torch.int16).cpu().numpy().view(np.uint16)
