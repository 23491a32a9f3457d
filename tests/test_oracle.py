"""Pin the CPU oracle (oracle/oracle.c) to the reference.

Two sources of truth: the golden fixtures in tests/golden/ (generated from the
reference's own CPU code by tests/golden/make_golden.py) and, when it was
built here, the live reference library oracle/_ref/libds_ref.so.
"""

import ctypes
import os

import numpy as np
import pytest

import oracle as O

GOLD = os.path.join(os.path.dirname(__file__), "golden")


def gold(name):
    return np.load(os.path.join(GOLD, name))


def f32(a):
    return np.ascontiguousarray(a, dtype=np.float32)


# ------------------------------------------------------------- primitives


def test_rmsnorm_matches_golden_bitwise():
    g = gold("primitives.npz")
    for n in (1, 7, 64, 512):
        x, w, y = f32(g[f"rms_x_{n}"]), f32(g[f"rms_w_{n}"]), g[f"rms_y_{n}"]
        out = np.zeros(n, np.float32)
        O.oracle().orc_rmsnorm_f32(O.p(x, O.f32p), O.p(w, O.f32p), n, 1e-6, O.p(out, O.f32p))
        assert np.array_equal(out.view(np.uint32), y.view(np.uint32)), n


def test_rope_matches_golden_bitwise():
    g = gold("primitives.npz")
    for dim in (2, 32, 64):
        for pos in (0, 1, 17, 4095, 100000):
            x = f32(g[f"rope_x_{dim}_{pos}"]).copy()
            assert O.oracle().orc_rope_inplace_f32(O.p(x, O.f32p), dim, pos, 10000.0) == 0
            assert np.array_equal(x.view(np.uint32), g[f"rope_y_{dim}_{pos}"].view(np.uint32)), (dim, pos)


def test_rope_odd_dim_rejected():
    x = np.zeros(3, np.float32)
    assert O.oracle().orc_rope_inplace_f32(O.p(x, O.f32p), 3, 0, 10000.0) == -1


def test_softmax_matches_golden_bitwise():
    g = gold("primitives.npz")
    for n in (1, 5, 64, 1000):
        x = f32(g[f"smax_x_{n}"]).copy()
        assert O.oracle().orc_softmax_f32(O.p(x, O.f32p), n) == 0
        assert np.array_equal(x.view(np.uint32), g[f"smax_y_{n}"].view(np.uint32)), n


def test_argmax_ties_lowest_index():
    g = gold("primitives.npz")
    x = f32(g["argmax_x"])
    assert O.oracle().orc_argmax_f32(O.p(x, O.f32p), x.size) == int(g["argmax_i"][0])
    y = np.array([1.0, 3.0, 3.0, 2.0], np.float32)
    assert O.oracle().orc_argmax_f32(O.p(y, O.f32p), 4) == 1


# ------------------------------------------------------------------- MLA


def run_orc_mla_layer(g):
    D, H, nope, rope, v, R, T = (int(x) for x in g["cfg"])
    out = np.zeros((T, D), np.float32)
    rc = O.oracle().orc_mla_layer_seq_f32(
        D, H, nope, rope, v, R, 1e-6, 10000.0, *(O.p(f32(g[k]), O.f32p) for k in
                                                 ("w_q", "w_kva", "w_kva_norm", "w_kvb", "w_o", "hidden")),
        T, O.p(out, O.f32p))
    assert rc == 0
    return out


def test_absorbed_mla_layer_matches_reference_golden():
    """The absorbed, latent-cache restatement equals the reference's
    non-absorbed mla_decode_step (per-head K/V cache) up to fp32 re-association."""
    g = gold("mla_layer.npz")
    out = run_orc_mla_layer(g)
    ref = g["out"]
    err = np.abs(out - ref).max() / np.abs(ref).max()
    assert err < 2e-5, err


@pytest.mark.skipif(not O.ref_available(), reason="reference build oracle/_ref absent")
def test_absorbed_mla_layer_matches_live_reference():
    g = gold("mla_layer.npz")
    D, H, nope, rope, v, R, T = (int(x) for x in g["cfg"])
    c = O.RefConfig(hidden_size=D, num_attention_heads=H, qk_nope_head_dim=nope, qk_rope_head_dim=rope,
                    v_head_dim=v, kv_lora_rank=R, num_hidden_layers=1, vocab_size=8, max_position_embeddings=T,
                    rms_norm_eps=1e-6, rope_theta=10000.0, routed_scaling_factor=1.0)
    ref = np.zeros((T, D), np.float32)
    args = [O.p(f32(g[k]), O.f32p) for k in ("w_q", "w_kva", "w_kva_norm", "w_kvb", "w_o", "hidden")]
    assert O.ref().ref_mla_seq(ctypes.byref(c), *args, T, O.p(ref, O.f32p)) == 0
    assert np.array_equal(ref, g["out"])  # the fixture is reproducible
    out = run_orc_mla_layer(g)
    assert np.abs(out - ref).max() / np.abs(ref).max() < 2e-5


def test_mla_paged_equals_contiguous_attention():
    """orc_mla_decode_paged reads pages through the block table: scattering the
    same rows over a shuffled page pool leaves the result bit-identical, and it
    matches a float64 softmax-attention computed with numpy."""
    rng = np.random.default_rng(5)
    B, H, R, P, bs = 3, 4, 32, 8, 64
    lens = np.array([1, 64, 130], np.int32)
    max_blocks = 3
    n_blocks = B * max_blocks
    rows = rng.standard_normal((B, max_blocks * bs, R + P)).astype(np.float32)
    q_lat = O.f32_to_bf16(rng.standard_normal((B, H, R)))
    q_rope = O.f32_to_bf16(rng.standard_normal((B, H, P)))
    perm = rng.permutation(n_blocks).astype(np.int32)
    bt = perm.reshape(B, max_blocks)
    cache = np.zeros((n_blocks, bs, R + P), np.uint16)
    for b in range(B):
        for j in range(max_blocks):
            cache[bt[b, j]] = O.f32_to_bf16(rows[b, j * bs:(j + 1) * bs])
    scale = 1 / np.sqrt(24.0)
    out = O.mla_decode_paged(q_lat, q_rope, cache, bt, lens, scale)
    # identity layout gives the same bits
    bt2 = np.arange(n_blocks, dtype=np.int32).reshape(B, max_blocks)
    cache2 = np.zeros_like(cache)
    for b in range(B):
        for j in range(max_blocks):
            cache2[bt2[b, j]] = cache[bt[b, j]]
    out2 = O.mla_decode_paged(q_lat, q_rope, cache2, bt2, lens, scale)
    assert np.array_equal(out, out2)
    # float64 check
    for b in range(B):
        kv = O.bf16_to_f32(np.concatenate([cache[bt[b, j]] for j in range(max_blocks)])[: lens[b]]).astype(np.float64)
        q = np.concatenate([O.bf16_to_f32(q_lat[b]), O.bf16_to_f32(q_rope[b])], axis=1).astype(np.float64)
        s = q @ kv.T * scale
        s = np.exp(s - s.max(1, keepdims=True))
        s /= s.sum(1, keepdims=True)
        ref = s @ kv[:, :R]
        assert np.abs(out[b] - ref).max() < 1e-5


# ------------------------------------------------------------------- MoE


def run_orc_moe(g, norm):
    D, E, k, I, Is, T = (int(x) for x in g["dims"])
    out = np.zeros((T, D), np.float32)
    w = [f32(g[n]) for n in ("w_gate", "e_gate", "e_up", "e_down", "s_gate", "s_up", "s_down")]
    x = f32(g["x"])
    for t in range(T):
        o = np.zeros(D, np.float32)
        xt = f32(x[t])
        assert O.oracle().orc_moe_softmax_f32(*(O.p(a, O.f32p) for a in w), Is, D, E, k, I, norm, 2.5,
                                              O.p(xt, O.f32p), O.p(o, O.f32p)) == 0
        out[t] = o
    return out


@pytest.mark.parametrize("norm", [0, 1])
def test_moe_softmax_greedy_matches_reference_golden_bitwise(norm):
    g = gold("moe_softmax.npz")
    out = run_orc_moe(g, norm)
    assert np.array_equal(out.view(np.uint32), g[f"out_norm{norm}"].view(np.uint32))


def test_router_softmax_topk_ties_lower_id():
    logits = np.array([[0.0, 1.0, 1.0, 0.5, 1.0]], np.float32)
    ids = np.zeros((1, 2), np.int32)
    w = np.zeros((1, 2), np.float32)
    assert O.oracle().orc_route_softmax_greedy(O.p(logits, O.f32p), 1, 5, 2, 1, 1.0, O.p(ids, O.i32p), O.p(w, O.f32p)) == 0
    assert ids.tolist() == [[1, 2]]
    assert np.allclose(w, 0.5)


def test_router_sigmoid_grouped_restatement():
    """Check the grouped sigmoid router against an independent numpy restatement."""
    rng = np.random.default_rng(11)
    T, E, G, TG, k = 64, 256, 8, 4, 8
    logits = f32(rng.standard_normal((T, E)) * 2)
    bias = f32(rng.standard_normal(E) * 0.01)
    ids = np.zeros((T, k), np.int32)
    w = np.zeros((T, k), np.float32)
    assert O.oracle().orc_route_sigmoid_grouped(O.p(logits, O.f32p), O.p(bias, O.f32p), T, E, G, TG, k, 1, 2.5,
                                                O.p(ids, O.i32p), O.p(w, O.f32p)) == 0
    s = 1 / (1 + np.exp(-logits.astype(np.float64)))
    sb = s + bias
    for t in range(T):
        grp = sb[t].reshape(G, -1)
        gs = np.sort(grp, axis=1)[:, -2:].sum(1)
        keep = np.argsort(-gs, kind="stable")[:TG]
        mask = np.full(E, -np.inf)
        for gidx in keep:
            mask[gidx * (E // G):(gidx + 1) * (E // G)] = sb[t, gidx * (E // G):(gidx + 1) * (E // G)]
        sel = np.argsort(-mask, kind="stable")[:k]
        assert ids[t].tolist() == sel.tolist()
        ww = s[t, sel] / s[t, sel].sum() * 2.5
        assert np.allclose(w[t], ww, rtol=1e-5)


def test_moe_permute_histogram_offsets():
    rng = np.random.default_rng(3)
    T, k, E = 37, 4, 16
    ids = np.stack([rng.choice(E, k, replace=False) for _ in range(T)]).astype(np.int32)
    counts = np.zeros(E, np.int32)
    offsets = np.zeros(E + 1, np.int32)
    dest = np.zeros(T * k, np.int32)
    src = np.zeros(T * k, np.int32)
    O.oracle().orc_moe_permute(O.p(ids, O.i32p), T, k, E, O.p(counts, O.i32p), O.p(offsets, O.i32p),
                               O.p(dest, O.i32p), O.p(src, O.i32p))
    assert counts.tolist() == np.bincount(ids.ravel(), minlength=E).tolist()
    assert offsets[-1] == T * k
    flat = ids.ravel()
    order = np.argsort(flat, kind="stable")
    assert src.tolist() == order.tolist()
    assert np.array_equal(dest[src], np.arange(T * k))


# ------------------------------------------------------------------- FP8


def test_e4m3_codec_exhaustive():
    o = O.oracle()
    vals = [o.orc_e4m3_to_f32(c) for c in range(256)]
    assert vals[0x7E] == 448.0 and vals[0xFE] == -448.0
    assert np.isnan(vals[0x7F]) and np.isnan(vals[0xFF])
    assert vals[0x01] == 2.0 ** -9  # smallest subnormal
    assert vals[0x08] == 2.0 ** -6  # smallest normal
    for c in range(256):
        if c in (0x7F, 0xFF):
            continue
        if c == 0x80:  # -0 encodes back to -0
            assert o.orc_f32_to_e4m3(-0.0) == 0x80
            continue
        assert o.orc_f32_to_e4m3(vals[c]) == c
    assert o.orc_f32_to_e4m3(1e6) == 0x7E and o.orc_f32_to_e4m3(-1e6) == 0xFE
    # round to nearest even between 1.0 (0x38) and 1.125 (0x39)
    assert o.orc_f32_to_e4m3(1.0625) == 0x38
    assert o.orc_f32_to_e4m3(1.0626) == 0x39


def test_fp8_linear_equals_reference_linear_on_dequantised():
    rng = np.random.default_rng(9)
    T, Od, K = 3, 256, 256
    w = f32(rng.standard_normal((Od, K)) * 0.02)
    x = f32(rng.standard_normal((T, K)))
    # weights: 128x128 block scales
    GK, GO = K // 128, Od // 128
    sw = np.zeros((GO, GK), np.float32)
    wq = np.zeros((Od, K), np.uint8)
    o = O.oracle()
    for bo in range(GO):
        for bk in range(GK):
            blk = w[bo * 128:(bo + 1) * 128, bk * 128:(bk + 1) * 128]
            sc = np.float32(np.abs(blk).max() / 448.0)
            sw[bo, bk] = sc
            for i in range(128):
                for j in range(128):
                    wq[bo * 128 + i, bk * 128 + j] = o.orc_f32_to_e4m3(float(blk[i, j] / sc))
    xq = np.zeros((T, K), np.uint8)
    sx = np.zeros((T, GK), np.float32)
    o.orc_quant_act_1x128(O.p(x, O.f32p), T, K, O.p(xq, O.u8p), O.p(sx, O.f32p))
    y = np.zeros((T, Od), np.float32)
    o.orc_fp8_linear(O.p(wq, O.u8p), O.p(sw, O.f32p), O.p(xq, O.u8p), O.p(sx, O.f32p), T, Od, K, O.p(y, O.f32p))
    lut = np.array([o.orc_e4m3_to_f32(c) for c in range(256)], np.float32)
    wd = f32(lut[wq] * np.repeat(np.repeat(sw, 128, 0), 128, 1))
    xd = f32(lut[xq] * np.repeat(sx, 128, 1))
    for t in range(T):
        ref = np.zeros(Od, np.float32)
        o.orc_linear_f32(O.p(wd, O.f32p), O.p(f32(xd[t]), O.f32p), K, O.p(ref, O.f32p), Od)
        assert np.abs(y[t] - ref).max() <= 1e-4 * np.abs(ref).max()
    # and the quantised product is close to the unquantised one
    full = x @ w.T
    assert np.abs(y - full).max() / np.abs(full).max() < 0.08


# ------------------------------------------------------------ whole model


def test_composed_model_oracle_matches_reference_golden():
    """oracle.model.forward (the layer restatements composed as decode_next)
    reproduces the reference's own teacher-forced logits on the tiny model
    up to fp32 re-association, and its greedy ids on the whole sequence."""
    import oracle.model as OM
    from deepseek_cpp_infer_b200.workloads import TINY, model_tensors

    g = gold("tiny_model.npz")
    seq = np.concatenate([g["prompt"], g["generated"]])
    logits, margins = OM.forward(TINY, model_tensors(TINY, seed=0), seq)
    for i, step in enumerate(g["steps"]):
        ref = g["logits"][i]
        assert np.abs(logits[step] - ref).max() <= 1e-5 * np.abs(ref).max()
    assert np.array_equal(np.argmax(logits, 1)[: len(g["greedy"])], g["greedy"])
    assert sorted(margins) == [1, 2, 3] and all(np.all(m >= 0) for m in margins.values())
