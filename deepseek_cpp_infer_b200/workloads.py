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


# ------------------------------------------------------------------ models

TINY = dict(
    hidden_size=512, num_hidden_layers=4, num_attention_heads=8, vocab_size=4096, max_position_embeddings=256,
    intermediate_size=1024, moe_intermediate_size=256, n_routed_experts=16, n_shared_experts=2,
    num_experts_per_tok=4, first_k_dense_replace=1, q_lora_rank=0, kv_lora_rank=128, qk_nope_head_dim=64,
    qk_rope_head_dim=32, v_head_dim=64, scoring_func=0, n_group=1, topk_group=1, norm_topk_prob=0,
    routed_scaling_factor=1.0, rms_norm_eps=1e-6, rope_theta=10000.0,
)

V2_LITE = dict(
    hidden_size=2048, num_hidden_layers=27, num_attention_heads=16, vocab_size=102400, max_position_embeddings=4096,
    intermediate_size=10944, moe_intermediate_size=1408, n_routed_experts=64, n_shared_experts=2,
    num_experts_per_tok=6, first_k_dense_replace=1, q_lora_rank=0, kv_lora_rank=512, qk_nope_head_dim=128,
    qk_rope_head_dim=64, v_head_dim=128, scoring_func=0, n_group=1, topk_group=1, norm_topk_prob=0,
    routed_scaling_factor=1.0, rms_norm_eps=1e-6, rope_theta=10000.0,
)


# DeepSeek-V3 (671B) shape: FP8 block-scaled projections, FFN and experts.
V3 = dict(
    hidden_size=7168, num_hidden_layers=61, num_attention_heads=128, vocab_size=129280, max_position_embeddings=163840,
    intermediate_size=18432, moe_intermediate_size=2048, n_routed_experts=256, n_shared_experts=1,
    num_experts_per_tok=8, first_k_dense_replace=3, q_lora_rank=1536, kv_lora_rank=512, qk_nope_head_dim=128,
    qk_rope_head_dim=64, v_head_dim=128, scoring_func=1, n_group=8, topk_group=4, norm_topk_prob=1,
    routed_scaling_factor=2.5, rms_norm_eps=1e-6, rope_theta=10000.0, weights_fp8=1,
)


def bf16_round(a: np.ndarray) -> np.ndarray:
    """Round float32 values to the nearest bf16 value (ties to even), kept as float32."""
    u = np.ascontiguousarray(a, np.float32).view(np.uint32).astype(np.uint64)
    u = (u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000
    return u.astype(np.uint32).view(np.float32)


def model_tensors(cfg: dict, seed: int = 0, std: float = 0.02) -> dict:
    """HF-named weights of a random-init DeepSeek-V2-style model: N(0, std)
    matrices from numpy default_rng(seed), rounded to bf16 values, RMSNorm
    weights 1.  Layers < first_k_dense_replace are dense, the rest MoE."""
    rng = np.random.default_rng(seed)
    D, H, R = cfg["hidden_size"], cfg["num_attention_heads"], cfg["kv_lora_rank"]
    nope, P, v = cfg["qk_nope_head_dim"], cfg["qk_rope_head_dim"], cfg["v_head_dim"]
    E, I, Is = cfg["n_routed_experts"], cfg["moe_intermediate_size"], cfg["n_shared_experts"] * cfg["moe_intermediate_size"]

    def mat(*shape):
        return bf16_round(rng.standard_normal(shape, dtype=np.float32) * std)

    t = {"model.embed_tokens.weight": mat(cfg["vocab_size"], D)}
    for i in range(cfg["num_hidden_layers"]):
        p = f"model.layers.{i}."
        t[p + "input_layernorm.weight"] = np.ones(D, np.float32)
        t[p + "post_attention_layernorm.weight"] = np.ones(D, np.float32)
        t[p + "self_attn.q_proj.weight"] = mat(H * (nope + P), D)
        t[p + "self_attn.kv_a_proj_with_mqa.weight"] = mat(R + P, D)
        t[p + "self_attn.kv_a_layernorm.weight"] = np.ones(R, np.float32)
        t[p + "self_attn.kv_b_proj.weight"] = mat(H * (nope + v), R)
        t[p + "self_attn.o_proj.weight"] = mat(D, H * v)
        if i < cfg["first_k_dense_replace"]:
            Id = cfg["intermediate_size"]
            t[p + "mlp.gate_proj.weight"] = mat(Id, D)
            t[p + "mlp.up_proj.weight"] = mat(Id, D)
            t[p + "mlp.down_proj.weight"] = mat(D, Id)
        else:
            t[p + "mlp.gate.weight"] = mat(E, D)
            for e in range(E):
                q = p + f"mlp.experts.{e}."
                t[q + "gate_proj.weight"] = mat(I, D)
                t[q + "up_proj.weight"] = mat(I, D)
                t[q + "down_proj.weight"] = mat(D, I)
            t[p + "mlp.shared_experts.gate_proj.weight"] = mat(Is, D)
            t[p + "mlp.shared_experts.up_proj.weight"] = mat(Is, D)
            t[p + "mlp.shared_experts.down_proj.weight"] = mat(D, Is)
    t["model.norm.weight"] = np.ones(D, np.float32)
    t["lm_head.weight"] = mat(cfg["vocab_size"], D)
    return t


def tiny_prompt(seed: int = 0, n: int = 32, vocab: int = 4096) -> np.ndarray:
    """32 uniform token ids for the tiny-model generate workload."""
    return np.random.default_rng(seed + 7).integers(0, vocab, n).astype(np.int32)


# DeepSeek-V3 MoE layer (one layer of the 671B model): 256 routed experts top-8
# by sigmoid + bias over 8 groups (top-4 groups), 1 shared expert, FP8 weights.
V3_MOE = dict(hidden_size=7168, moe_intermediate_size=2048, n_routed_experts=256, n_shared_experts=1,
              num_experts_per_tok=8, n_group=8, topk_group=4, routed_scaling_factor=2.5, norm_topk_prob=1)


class MoeFp8Weights:
    """Random FP8 expert weights of one MoE layer in dsb_moe_ffn_fp8 layout.

    Each of the G = E + n_shared groups gets gate/up [I, D] and down [D, I]
    ~ N(0, std) (fp32, seeded torch generator on the device), quantised per
    128x128 block by dsb_quant_weight_128x128; gate and up rows are then
    interleaved and their scales arranged per 128-row tile (scale_rows 2).
    With keep_separate the per-matrix e4m3 codes and scales stay available
    for the oracle (small configurations only)."""

    def __init__(self, ctx, E, n_shared, D, I, seed=2, std=0.02, keep_separate=False):
        import torch

        G = E + n_shared
        self.E, self.n_shared, self.D, self.I = E, n_shared, D, I
        self.gate_up = torch.empty(G, 2 * I, D, dtype=torch.uint8, device="cuda")
        self.gate_up_scale = torch.empty(G, 2 * I // 128, 2, D // 128, dtype=torch.float32, device="cuda")
        self.down = torch.empty(G, D, I, dtype=torch.uint8, device="cuda")
        self.down_scale = torch.empty(G, D // 128, I // 128, dtype=torch.float32, device="cuda")
        gen = torch.Generator(device="cuda").manual_seed(seed)
        rows = torch.arange(2 * I // 128, device="cuda") * 64 // 128  # scale row of tile j's gate/up rows
        sep = [] if keep_separate else None
        qg = torch.empty(I, D, dtype=torch.uint8, device="cuda")
        qu = torch.empty_like(qg)
        sg = torch.empty(I // 128, D // 128, dtype=torch.float32, device="cuda")
        su = torch.empty_like(sg)
        for g in range(G):
            ctx.quant_weight(torch.randn(I, D, generator=gen, device="cuda") * std, qg, sg)
            ctx.quant_weight(torch.randn(I, D, generator=gen, device="cuda") * std, qu, su)
            ctx.quant_weight(torch.randn(D, I, generator=gen, device="cuda") * std, self.down[g], self.down_scale[g])
            self.gate_up[g] = torch.stack([qg, qu], 1).reshape(2 * I, D)
            self.gate_up_scale[g] = torch.stack([sg[rows], su[rows]], 1)
            if sep is not None:
                sep.append((qg.clone(), sg.clone(), qu.clone(), su.clone()))
        if sep is not None:
            cat = lambda i: np.ascontiguousarray(torch.stack([s[i] for s in sep]).cpu().numpy())  # noqa: E731
            self.gate_q, self.gate_s, self.up_q, self.up_s = cat(0), cat(1), cat(2), cat(3)
            self.down_q = np.ascontiguousarray(self.down.cpu().numpy())
            self.down_s = np.ascontiguousarray(self.down_scale.cpu().numpy())

    def bytes(self):
        return sum(t.numel() * t.element_size() for t in (self.gate_up, self.gate_up_scale, self.down, self.down_scale))
