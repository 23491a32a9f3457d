"""Parity at the benchmarked DeepSeek-V2-Lite layer shape, through the C ABI.

A two-layer model with V2-Lite's layer shapes - the dense layer 0 (FFN
10944) and one MoE layer (64 routed experts top-6 softmax, 2 shared,
moe_intermediate 1408), hidden 2048, 16 heads, kv_lora_rank 512, nope 128,
rope 64, v 128 - with the vocabulary cut to 4096 so the reference's CPU
forward stays fast.  Random N(0, 0.02) weights rounded to bf16 values
(seed 3), RMSNorm weights 1.  The GPU decodes 12 tokens one by one
(dsb_decode_step, bf16 weights and activations); the reference's own
DeepSeekModel (oracle/_ref: src/models/deepseek/model.cpp:112-221 on the CPU
backend, fp32) runs the same tokens on the same weights.

Bar: the stated layer-output tolerance on the logits, max-rel <= 2e-2 at
every step; the greedy id equal at every step whose reference top-1/top-2
gap exceeds twice that step's largest logit error (a smaller gap is a tie
at bf16 resolution).
"""

import ctypes
import os
import sys

import numpy as np
import pytest

import oracle as O
import deepseek_cpp_infer_b200 as dsb
from deepseek_cpp_infer_b200.workloads import V2_LITE, model_tensors

pytestmark = pytest.mark.gpu

sys.path.insert(0, os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden"))


def test_v2lite_layers_match_reference(gpu_ctx):
    if not O.ref_available():
        pytest.skip("oracle/_ref (the reference built from its sources) is not present")
    from make_golden import ref_model

    cfg = dict(V2_LITE, num_hidden_layers=2, vocab_size=4096, max_position_embeddings=64)
    t = model_tensors(cfg, seed=3)
    m = dsb.Model(gpu_ctx, dsb.ModelConfig(**cfg))
    for name, a in t.items():
        m.set_tensor(name, a)
    m.finalize()
    kv = dsb.KVCache(gpu_ctx, m, n_blocks=2, max_seqs=1, max_blocks_per_seq=1)
    s = kv.alloc_seq()
    toks = [int(x) for x in np.random.default_rng(5).integers(0, cfg["vocab_size"], 12)]
    got = []
    for tok in toks:
        _, lg = dsb.decode_step(gpu_ctx, m, kv, [s], [tok], want_logits=True)
        got.append(lg[0])
    kv.close()
    m.close()
    h, keep = ref_model(cfg, t)
    try:
        row = np.zeros(cfg["vocab_size"], np.float32)
        g = ctypes.c_int32()
        ref = []
        for tok in toks:
            assert O.ref().ref_model_step(h, tok, O.p(row, O.f32p), ctypes.byref(g)) == 0
            ref.append(row.copy())
    finally:
        O.ref().ref_model_destroy(h)
    got, ref = np.stack(got), np.stack(ref)
    abs_err = np.abs(got - ref).max(1)
    err = abs_err / np.abs(ref).max(1)
    srt = np.sort(ref, axis=1)
    gap = srt[:, -1] - srt[:, -2]
    decided = gap > 2 * abs_err
    same = got.argmax(1) == ref.argmax(1)
    print(f"V2-Lite layers vs reference: logits max-rel median {np.median(err):.3e} worst {err.max():.3e}; "
          f"greedy equal {int(same.sum())}/12 ({int(decided.sum())} steps decided beyond the error)")
    assert err.max() <= 2e-2, err
    assert same[decided].all(), (got.argmax(1), ref.argmax(1), gap, abs_err)
