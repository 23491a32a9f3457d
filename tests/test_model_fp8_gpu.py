"""Whole-model decode with a block-scaled FP8 checkpoint (DeepSeek-V3 style:
e4m3 weights + "<name>_scale_inv" fp32 128x128 scales), through the C ABI.

The tiny configuration's projections, dense FFN, routed and shared experts
are quantised per 128x128 block by the oracle's restatement
(orc_quant_weight_128x128) and uploaded as FP8 (kv_b_proj too: the model
dequantises it at load).  A second model gets the same weights dequantised
(e4m3 * scale, rounded to bf16) and runs the bf16 path.  The two then differ
only in the FP8 path's 1x128 e4m3 quantisation of every GEMM's activations
(3 mantissa bits, about 2-4% per element), which compounds over the tiny
random model's ~25 GEMMs and flips greedy ids wherever its (small) logit
margins are below that.  The bar is therefore a consistency bar, stated
here: logits max-rel <= 0.15 over 24 teacher-forced steps and the same
greedy id at >= 75% of them (measured: 0.10 and 20/24).  The FP8 kernels
themselves are pinned tightly against the oracle in test_fp8_gpu.py and
test_moe_fp8_gpu.py.
"""

import numpy as np
import pytest

import oracle as O
import deepseek_cpp_infer_b200 as dsb
from deepseek_cpp_infer_b200.workloads import TINY, model_tensors
from fp8_tiny import build, quantise

pytestmark = pytest.mark.gpu


def test_fp8_checkpoint_model_tracks_dequantised_bf16_model(gpu_ctx):
    m8 = build(gpu_ctx, fp8=True)
    m16 = build(gpu_ctx, fp8=False)
    kvs = [dsb.KVCache(gpu_ctx, m, n_blocks=16, max_seqs=2, max_blocks_per_seq=4) for m in (m8, m16)]
    seqs = [kv.alloc_seq() for kv in kvs]
    toks = np.random.default_rng(7).integers(0, TINY["vocab_size"], 24)
    worst, same = 0.0, 0
    for t in toks:
        g8, l8 = dsb.decode_step(gpu_ctx, m8, kvs[0], [seqs[0]], [int(t)], want_logits=True)
        g16, l16 = dsb.decode_step(gpu_ctx, m16, kvs[1], [seqs[1]], [int(t)], want_logits=True)
        assert np.isfinite(l8).all()
        worst = max(worst, float(np.abs(l8 - l16).max() / np.abs(l16).max()))
        same += int(g8[0] == g16[0])
    print(f"FP8 vs dequantised-bf16 model: logits max-rel {worst:.3e}, greedy agreement {same}/{len(toks)}")
    assert worst <= 0.15
    assert same >= 0.75 * len(toks)
    for kv in kvs:
        kv.close()
    m8.close()
    m16.close()


def test_fp8_weight_without_scale_is_rejected(gpu_ctx):
    m = dsb.Model(gpu_ctx, dsb.ModelConfig(**TINY))
    tensors = model_tensors(TINY, seed=0)
    for name, a in tensors.items():
        if name == "model.layers.0.self_attn.o_proj.weight":
            q, _, _ = quantise(O.bf16_to_f32(a))
            m.set_tensor(name, q)  # no scale
        else:
            m.set_tensor(name, a)
    with pytest.raises(dsb.DsbError) as e:
        m.finalize()
    assert e.value.code == dsb.DSB_EINVAL
    m.close()


# A position this far from the oracle (logits max-rel) holds a discrete
# rounding difference to look for; after explaining what can be explained
# every position must be within FINAL of the oracle, half the stated 2e-2 bar.
STRICT = 5e-4
FINAL = 1e-2
# gate-logit gap (logit units) below which the last routed expert may swap
NEAR_TIE = 0.005


def test_fp8_model_matches_fp8_oracle(gpu_ctx):
    """The FP8 checkpoint model against oracle.model.forward_fp8, the
    composed restatement with the same activation quantisation points (bf16
    activation, e4m3 per token and 128 columns before every FP8 GEMM), the
    dequantised weights, and every activation stored where the batched
    decode stores it (bf16 cache rows, queries, probabilities, latent and
    per-head outputs; the split-KV plan of the decode), so that both feed
    the same bytes to every e4m3 quantiser.

    The GPU decodes a 16-token prompt and then generates 32 tokens greedily;
    the oracle is teacher-forced on the same 48 tokens.

    Rounding ambiguity.  The GPU sums its GEMMs and reductions in another
    order, so where a value's fp32 result lies within a few 1e-6 of a bf16
    rounding midpoint the two sides may store different bf16 neighbours,
    and where that changes an e4m3 code one element of the next GEMM's input
    differs by 6-12%.  On this random tiny model one such element moves the
    logits by up to 5%, so no implementation that sums in another order can
    hold the whole model to 2e-2 without accounting for it.  The oracle
    records every such ambiguous value (oracle.model.Fp8Quantiser: e4m3
    quantisation inputs within 3e-5, bf16 storage points - cache rows,
    query parts, probabilities, latent outputs - within 3e-6).  Position by
    position, the first position more than STRICT away is searched for the
    ambiguous value (at that position, or a cache row of an earlier one;
    nearest the midpoint first) or router near-tie whose other choice
    brings it closest; a choice that brings it at least 1.5x closer is
    taken and the oracle continues with it.  The search stops at the first
    position no single choice explains.  Bar: all 48 positions within FINAL
    (1e-2, half the stated 2e-2) of the oracle with the choices taken, and
    the oracle's greedy id equal to each of the 32 generated tokens."""
    import torch

    slots = torch.cuda.get_device_properties(0).multi_processor_count
    m8 = build(gpu_ctx, fp8=True)
    prompt = [int(x) for x in np.random.default_rng(7).integers(0, TINY["vocab_size"], 16)]
    kv = dsb.KVCache(gpu_ctx, m8, n_blocks=16, max_seqs=1, max_blocks_per_seq=4)
    s = kv.alloc_seq()
    seq, rows, gen = [], [], []
    nxt = None
    for i in range(16 + 32):
        tok = prompt[i] if i < 16 else nxt
        seq.append(tok)
        g, lg = dsb.decode_step(gpu_ctx, m8, kv, [s], [tok], want_logits=True)
        rows.append(lg[0])
        nxt = int(g[0])
        if i >= 15 and len(gen) < 32:
            gen.append(nxt)
    kv.close()
    m8.close()
    check_against_oracle(np.stack(rows), seq, gen, slots)


def check_against_oracle(got, seq, gen, slots):
    """The bar of test_fp8_model_matches_fp8_oracle on the GPU's logits `got`
    [48, V] for the token sequence `seq` (16 prompt + 32 generated `gen`)."""
    import oracle.model as OM
    from fp8_tiny import FP8_SUFFIXES

    t = model_tensors(TINY, seed=0)
    fp8 = {n: quantise(a)[2] for n, a in t.items()
           if n.startswith("model.layers.") and n.endswith(FP8_SUFFIXES) and "mlp.gate." not in n}

    def max_rel(ref):
        return np.abs(got - ref).max(1) / np.abs(ref).max(1)

    def run(flips, swaps, record=True):
        q = OM.Fp8Quantiser(flips, record=record)
        margins = {}
        ref = OM.forward_fp8(TINY, t, fp8, seq, slots=slots, swaps=swaps, margins=margins, quant=q)
        return ref, q.fragile, margins

    flips, swaps = set(), []
    ref, fragile, margins = run(flips, swaps)
    err = max_rel(ref)
    print(f"FP8 model vs FP8 oracle before explaining ambiguities: max-rel per position "
          f"{np.array2string(err, precision=1)}")
    unexplained = None
    for _ in range(24):
        bad = np.nonzero(err > STRICT)[0]
        if len(bad) == 0:
            break
        p0 = int(bad[0])
        cands = [("swap", (li, p0), float(m[p0])) for li, m in margins.items() if m[p0] < NEAR_TIE]
        cands += [("flip", f[:3], f[3]) for f in sorted(fragile, key=lambda f: f[3])
                  if f[1] == p0 or (f[1] < p0 and f[0][0] in ("c", "kr"))]
        best = None
        for kind, what, gap in cands[:32]:  # nearest first; stop at the first that explains the position
            r2, _, _ = run(flips | {what} if kind == "flip" else flips, swaps + [what] if kind == "swap" else swaps,
                           record=False)
            e2 = max_rel(r2)[p0]
            if best is None or e2 < best[0]:
                best = (e2, kind, what, gap)
            if e2 <= STRICT:
                break
        if best is None or best[0] > err[p0] / 1.5:
            unexplained = (p0, float(err[p0]))
            break
        if best[1] == "flip":
            flips.add(best[2])
        else:
            swaps.append(best[2])
        print(f"position {p0}: {best[1]} {best[2]} (distance {best[3]:.1e}) takes max-rel {err[p0]:.2e} "
              f"-> {best[0]:.2e}")
        ref, fragile, margins = run(flips, swaps)
        err = max_rel(ref)
    oracle_ids = ref.argmax(1)[15:47]
    same = int((oracle_ids == np.array(gen[:32])).sum())
    print(f"FP8 model vs FP8 oracle: logits max-rel median {np.median(err):.3e} worst {err.max():.3e}; "
          f"greedy {same}/32; rounding choices taken {len(flips)}, router swaps {len(swaps)}; "
          f"first position left unexplained {unexplained}")
    assert err.max() <= FINAL, err
    assert same == 32, (oracle_ids, gen)
