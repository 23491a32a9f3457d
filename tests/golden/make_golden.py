"""Generate the golden fixtures of tests/golden/ from the reference itself.

Runs the reference's own CPU functions (oracle/_ref/libds_ref.so, compiled
from the deepseek_cpp_infer sources by oracle/Makefile) on seeded synthetic
inputs and stores inputs and outputs as .npz.  The reference ships no golden
vectors of its own, so these fixtures are what pins the C restatement in
oracle/oracle.c when the reference sources are not present.

    python tests/golden/make_golden.py
"""

from __future__ import annotations

import ctypes
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

import oracle as O  # noqa: E402


def f32(a):
    return np.ascontiguousarray(a, dtype=np.float32)


def primitives(rng):
    ref = O.ref()
    out = {}
    # rmsnorm over several lengths
    for n in (1, 7, 64, 512):
        x = f32(rng.standard_normal(n) * 3)
        w = f32(rng.standard_normal(n))
        y = np.zeros(n, np.float32)
        ref.ref_rmsnorm_f32(O.p(x, O.f32p), O.p(w, O.f32p), n, 1e-6, O.p(y, O.f32p))
        out[f"rms_x_{n}"], out[f"rms_w_{n}"], out[f"rms_y_{n}"] = x, w, y
    # rope at several positions and dims
    for dim in (2, 32, 64):
        for pos in (0, 1, 17, 4095, 100000):
            x = f32(rng.standard_normal(dim))
            y = x.copy()
            assert ref.ref_rope_inplace_f32(O.p(y, O.f32p), dim, pos, 10000.0) == 0
            out[f"rope_x_{dim}_{pos}"], out[f"rope_y_{dim}_{pos}"] = x, y
    # softmax, including a large dynamic range
    for n in (1, 5, 64, 1000):
        x = f32(rng.standard_normal(n) * (30 if n == 64 else 2))
        y = x.copy()
        assert ref.ref_softmax_f32(O.p(y, O.f32p), n) == 0
        out[f"smax_x_{n}"], out[f"smax_y_{n}"] = x, y
    # argmax with exact ties (lowest index wins)
    x = f32(rng.integers(0, 5, 257))
    out["argmax_x"] = x
    out["argmax_i"] = np.array([ref.ref_argmax_f32(O.p(x, O.f32p), x.size)], np.int64)
    return out


def mla_layer(rng):
    cfg = dict(D=64, H=4, nope=16, rope=8, v=16, R=32, T=12)
    D, H, nope, rope, v, R, T = (cfg[k] for k in ("D", "H", "nope", "rope", "v", "R", "T"))
    w_q = f32(rng.standard_normal((H * (nope + rope), D)) * 0.2)
    w_kva = f32(rng.standard_normal((R + rope, D)) * 0.2)
    w_kva_norm = f32(1.0 + 0.1 * rng.standard_normal(R))
    w_kvb = f32(rng.standard_normal((H * (nope + v), R)) * 0.2)
    w_o = f32(rng.standard_normal((D, H * v)) * 0.2)
    hidden = f32(rng.standard_normal((T, D)))
    c = O.RefConfig(hidden_size=D, num_attention_heads=H, qk_nope_head_dim=nope, qk_rope_head_dim=rope,
                    v_head_dim=v, kv_lora_rank=R, num_hidden_layers=1, vocab_size=8, max_position_embeddings=T,
                    rms_norm_eps=1e-6, rope_theta=10000.0, routed_scaling_factor=1.0)
    out = np.zeros((T, D), np.float32)
    assert O.ref().ref_mla_seq(ctypes.byref(c), O.p(w_q, O.f32p), O.p(w_kva, O.f32p), O.p(w_kva_norm, O.f32p),
                               O.p(w_kvb, O.f32p), O.p(w_o, O.f32p), O.p(hidden, O.f32p), T, O.p(out, O.f32p)) == 0
    return dict(cfg=np.array([D, H, nope, rope, v, R, T], np.int32), w_q=w_q, w_kva=w_kva, w_kva_norm=w_kva_norm,
                w_kvb=w_kvb, w_o=w_o, hidden=hidden, out=out)


def moe(rng):
    D, E, k, I, Is, T = 32, 8, 3, 16, 24, 6
    w_gate = f32(rng.standard_normal((E, D)) * 0.3)
    e_gate = f32(rng.standard_normal((E, I, D)) * 0.2)
    e_up = f32(rng.standard_normal((E, I, D)) * 0.2)
    e_down = f32(rng.standard_normal((E, D, I)) * 0.2)
    s_gate = f32(rng.standard_normal((Is, D)) * 0.2)
    s_up = f32(rng.standard_normal((Is, D)) * 0.2)
    s_down = f32(rng.standard_normal((D, Is)) * 0.2)
    x = f32(rng.standard_normal((T, D)))
    res = {}
    for norm in (0, 1):
        c = O.RefConfig(hidden_size=D, n_experts=E, moe_top_k=k, moe_intermediate_size=I, norm_topk_prob=norm,
                        routed_scaling_factor=2.5, num_hidden_layers=1, vocab_size=8)
        out = np.zeros((T, D), np.float32)
        assert O.ref().ref_moe_tokens(ctypes.byref(c), *(O.p(a, O.f32p) for a in (w_gate, e_gate, e_up, e_down,
                                                                                   s_gate, s_up, s_down)),
                                      Is, O.p(x, O.f32p), T, O.p(out, O.f32p)) == 0
        res[f"out_norm{norm}"] = out
    return dict(dims=np.array([D, E, k, I, Is, T], np.int32), w_gate=w_gate, e_gate=e_gate, e_up=e_up,
                e_down=e_down, s_gate=s_gate, s_up=s_up, s_down=s_down, x=x, **res)


def ref_model(cfg: dict, tensors: dict):
    """Build the reference DeepSeekModel over in-memory f32 tensors."""
    c = O.RefConfig(
        hidden_size=cfg["hidden_size"], intermediate_size=cfg["intermediate_size"],
        num_hidden_layers=cfg["num_hidden_layers"], num_attention_heads=cfg["num_attention_heads"],
        vocab_size=cfg["vocab_size"], max_position_embeddings=cfg["max_position_embeddings"],
        n_experts=cfg["n_routed_experts"], n_shared_experts=cfg["n_shared_experts"],
        moe_top_k=cfg["num_experts_per_tok"], moe_intermediate_size=cfg["moe_intermediate_size"],
        q_lora_rank=cfg["q_lora_rank"], kv_lora_rank=cfg["kv_lora_rank"], qk_nope_head_dim=cfg["qk_nope_head_dim"],
        qk_rope_head_dim=cfg["qk_rope_head_dim"], v_head_dim=cfg["v_head_dim"], norm_topk_prob=cfg["norm_topk_prob"],
        rms_norm_eps=cfg["rms_norm_eps"], rope_theta=cfg["rope_theta"],
        routed_scaling_factor=cfg["routed_scaling_factor"])
    names = list(tensors)
    arrs = [np.ascontiguousarray(tensors[n], np.float32) for n in names]
    c_names = (ctypes.c_char_p * len(names))(*[n.encode() for n in names])
    ndims = (ctypes.c_int * len(names))(*[a.ndim for a in arrs])
    shapes = (ctypes.c_int64 * sum(a.ndim for a in arrs))(*[d for a in arrs for d in a.shape])
    datas = (O.f32p * len(names))(*[O.p(a, O.f32p) for a in arrs])
    h = O.ref().ref_model_create(ctypes.byref(c), len(names), c_names, ndims, shapes, datas)
    assert h, "ref_model_create failed"
    return h, arrs


def tiny_model():
    """cfg1: the reference generates 64 greedy tokens after a 32-token prompt;
    teacher-forced logits on the same sequence are kept at a few steps."""
    from deepseek_cpp_infer_b200.workloads import TINY, model_tensors, tiny_prompt

    t = model_tensors(TINY, seed=0)
    prompt = tiny_prompt(0)
    h, keep = ref_model(TINY, t)
    gen = np.zeros(64, np.int32)
    assert O.ref().ref_model_generate(h, O.p(prompt, O.i32p), len(prompt), 64, O.p(gen, O.i32p)) == 0
    seq = np.concatenate([prompt, gen])
    O.ref().ref_model_reset(h)
    steps = [31, 32, 40, 63, 95]
    logits = np.zeros((len(steps), TINY["vocab_size"]), np.float32)
    greedy = np.zeros(len(seq), np.int32)
    row = np.zeros(TINY["vocab_size"], np.float32)
    g = ctypes.c_int32()
    for i, tok in enumerate(seq):
        assert O.ref().ref_model_step(h, int(tok), O.p(row, O.f32p), ctypes.byref(g)) == 0
        greedy[i] = g.value
        if i in steps:
            logits[steps.index(i)] = row
    O.ref().ref_model_destroy(h)
    assert np.array_equal(greedy[31:95], gen)  # teacher forcing reproduces the generation
    checksum = np.array([float(np.sum([np.float64(a).sum() for a in t.values()]))])
    return dict(prompt=prompt, generated=gen, greedy=greedy, steps=np.array(steps, np.int32), logits=logits,
                weight_checksum=checksum)


def main():
    O.build(with_ref=True)
    assert O.ref_available(), "reference build missing (oracle/_ref/libds_ref.so)"
    rng = np.random.default_rng(20251201)
    np.savez_compressed(os.path.join(HERE, "primitives.npz"), **primitives(rng))
    np.savez_compressed(os.path.join(HERE, "mla_layer.npz"), **mla_layer(rng))
    np.savez_compressed(os.path.join(HERE, "moe_softmax.npz"), **moe(rng))
    np.savez_compressed(os.path.join(HERE, "tiny_model.npz"), **tiny_model())
    for f in sorted(os.listdir(HERE)):
        if f.endswith(".npz"):
            print(f, os.path.getsize(os.path.join(HERE, f)), "bytes")


if __name__ == "__main__":
    main()
