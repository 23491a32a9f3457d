"""The FP8 MoE expert FFN (dsb_moe_ffn_fp8) with the sigmoid + bias grouped
router, through the C ABI, against the oracle's FP8 restatement of moe_step
(oracle.model.moe_fp8: orc_quant_act_1x128, orc_fp8_linear, silu, in the
reference's summation order) on the same routed picks.

Tolerance: max-rel <= 2e-2 on the layer's expert output (the bf16/fp8 layer
bar).  Both sides round the SiLU product to the bf16 activation before its
1x128 quantisation; fp32 accumulation order (and CUDA's expf in the SiLU) can
still move a few products across an e4m3 rounding boundary.  Routing itself is checked bit-exact
against orc_route_sigmoid_grouped on the same logits (ids exact, weights to
the last place of expf).
"""

import numpy as np
import pytest

import oracle as O
import oracle.model as OM
import deepseek_cpp_infer_b200 as dsb
from deepseek_cpp_infer_b200.workloads import MoeFp8Weights

pytestmark = pytest.mark.gpu
TOL = 2e-2


def route(ctx, x, E, k, n_group, topk_group, seed):
    """Router logits (fp32) and sigmoid-grouped picks on the GPU; the picks
    are checked against the oracle router on the same logits."""
    import torch

    T, D = x.shape
    g = torch.Generator(device="cuda").manual_seed(seed)
    w_gate = torch.randn(E, D, generator=g, device="cuda") * 0.02
    bias = torch.randn(E, generator=g, device="cuda") * 0.01
    logits = torch.empty(T, E, device="cuda")
    ctx.router_logits(x.float().contiguous(), w_gate, logits)
    ids = torch.empty(T, k, dtype=torch.int32, device="cuda")
    wts = torch.empty(T, k, device="cuda")
    ctx.moe_route(logits, ids, wts, k, scoring=dsb.SCORE_SIGMOID, bias=bias, n_group=n_group,
                  topk_group=topk_group, norm_topk=1, routed_scale=2.5)
    ctx.sync()
    lg = np.ascontiguousarray(logits.cpu().numpy())
    rid = np.zeros((T, k), np.int32)
    rw = np.zeros((T, k), np.float32)
    b = np.ascontiguousarray(bias.cpu().numpy())
    assert O.oracle().orc_route_sigmoid_grouped(O.p(lg, O.f32p), O.p(b, O.f32p), T, E, n_group, topk_group, k, 1,
                                                2.5, O.p(rid, O.i32p), O.p(rw, O.f32p)) == 0
    assert np.array_equal(ids.cpu().numpy(), rid)
    # weights: CUDA's and the C library's expf may differ in the last place
    assert np.abs(wts.cpu().numpy() - rw).max() <= 2e-6 * 2.5
    return ids, wts


def expected(layer, x, ids, wts, rows):
    """Oracle expert sum for the given token rows (shared experts appended)."""
    E, ns = layer.E, layer.n_shared
    ids_n, w_n = ids.cpu().numpy()[rows], wts.cpu().numpy()[rows]
    ids_x = np.concatenate([ids_n, np.tile(E + np.arange(ns, dtype=np.int32), (len(rows), 1))], 1)
    w_x = np.concatenate([w_n, np.ones((len(rows), ns), np.float32)], 1)
    return OM.moe_fp8(x.float().cpu().numpy()[rows], ids_x, w_x, layer.gate_q, layer.gate_s, layer.up_q,
                      layer.up_s, layer.down_q, layer.down_s)


def run(ctx, layer, x, ids, wts, seed):
    import torch

    g = torch.Generator(device="cuda").manual_seed(seed)
    h0 = torch.randn(x.shape[0], x.shape[1], generator=g, device="cuda")
    h = h0.clone()
    ctx.moe_ffn_fp8(layer.gate_up, layer.gate_up_scale, layer.down, layer.down_scale, E=layer.E,
                    n_shared=layer.n_shared, x=x, ids=ids, weights=wts, h=h)
    ctx.sync()
    return (h - h0).double()


@pytest.mark.parametrize("T", [1, 24])
def test_moe_ffn_fp8_matches_oracle(gpu_ctx, T):
    import torch

    E, ns, D, I, k = 32, 1, 1024, 256, 4
    layer = MoeFp8Weights(gpu_ctx, E, ns, D, I, seed=31, keep_separate=True)
    x = torch.randn(T, D, generator=torch.Generator(device="cuda").manual_seed(32), device="cuda").to(torch.bfloat16)
    ids, wts = route(gpu_ctx, x, E, k, n_group=4, topk_group=2, seed=33)
    got = run(gpu_ctx, layer, x, ids, wts, seed=34)
    ref = torch.from_numpy(expected(layer, x, ids, wts, np.arange(T))).double().cuda()
    err = float((got - ref).abs().max() / ref.abs().max())
    print("moe fp8 max-rel", err)
    assert err <= TOL


def test_moe_ffn_fp8_large_batch_rows_and_determinism(gpu_ctx):
    """2048 tokens x (6 + 2) picks: the multi-block permute path; a sample of
    rows against the oracle, and two runs bitwise equal."""
    import torch

    E, ns, D, I, k, T = 64, 2, 512, 256, 6, 2048
    layer = MoeFp8Weights(gpu_ctx, E, ns, D, I, seed=41, keep_separate=True)
    x = torch.randn(T, D, generator=torch.Generator(device="cuda").manual_seed(42), device="cuda").to(torch.bfloat16)
    ids, wts = route(gpu_ctx, x, E, k, n_group=8, topk_group=4, seed=43)
    a = run(gpu_ctx, layer, x, ids, wts, seed=44)
    b = run(gpu_ctx, layer, x, ids, wts, seed=44)
    assert torch.equal(a, b)
    rows = np.array([0, 1, 777, 1024, 2047])
    ref = torch.from_numpy(expected(layer, x, ids, wts, rows)).double().cuda()
    got = a[torch.from_numpy(rows).cuda()]
    assert float((got - ref).abs().max() / ref.abs().max()) <= TOL


def expected_from_device(layer, x, ids, wts, rows):
    """expected() for a layer made without keep_separate: only the experts
    the sampled rows pick are copied back, their gate and up codes taken out
    of the interleaved [2I, D] matrix (row 2f gate f, 2f+1 up f) and their
    scales out of the per-128-row-tile layout."""
    E, ns = layer.E, layer.n_shared
    ids_n, w_n = ids.cpu().numpy()[rows], wts.cpu().numpy()[rows]
    ids_x = np.concatenate([ids_n, np.tile(E + np.arange(ns, dtype=np.int32), (len(rows), 1))], 1)
    w_x = np.concatenate([w_n, np.ones((len(rows), ns), np.float32)], 1)
    used = np.unique(ids_x)
    remap = {int(e): i for i, e in enumerate(used)}
    gu = layer.gate_up[used.tolist()].cpu().numpy()
    gs = layer.gate_up_scale[used.tolist()].cpu().numpy()
    gate_q, up_q = np.ascontiguousarray(gu[:, 0::2]), np.ascontiguousarray(gu[:, 1::2])
    gate_s, up_s = np.ascontiguousarray(gs[:, 0::2, 0]), np.ascontiguousarray(gs[:, 0::2, 1])
    down_q = np.ascontiguousarray(layer.down[used.tolist()].cpu().numpy())
    down_s = np.ascontiguousarray(layer.down_scale[used.tolist()].cpu().numpy())
    ids_l = np.vectorize(remap.get)(ids_x).astype(np.int32)
    return OM.moe_fp8(x.float().cpu().numpy()[rows], ids_l, w_x, gate_q, gate_s, up_q, up_s, down_q, down_s)


@pytest.mark.parametrize("T", [128, 4096])
def test_moe_fp8_cfg3_full_shape(gpu_ctx, T):
    """The isolated DeepSeek-V3 MoE layer of the benchmark at its own shape:
    D=7168, 256 routed experts + 1 shared, I=2048, sigmoid + bias router
    with 8 groups / top-4 groups / top-8, routed scale 2.5, T tokens N(0,1).
    Router ids bit-exact against the oracle (except at fp32 near-ties of
    expf, each checked to be one); the layer's expert output within 2e-2 of
    oracle.model.moe_fp8 on a sample of rows."""
    import torch

    from test_ops_gpu import sigmoid_route_boundary_ulps

    E, ns, D, I, k, G, TG = 256, 1, 7168, 2048, 8, 8, 4
    layer = MoeFp8Weights(gpu_ctx, E, ns, D, I, seed=2)
    x = torch.randn(T, D, generator=torch.Generator(device="cuda").manual_seed(52), device="cuda").to(torch.bfloat16)
    gen = torch.Generator(device="cuda").manual_seed(53)
    w_gate = torch.randn(E, D, generator=gen, device="cuda") * 0.02
    bias = torch.randn(E, generator=gen, device="cuda") * 0.01
    logits = torch.empty(T, E, device="cuda")
    gpu_ctx.router_logits(x.float().contiguous(), w_gate, logits)
    ids = torch.empty(T, k, dtype=torch.int32, device="cuda")
    wts = torch.empty(T, k, device="cuda")
    gpu_ctx.moe_route(logits, ids, wts, k, scoring=dsb.SCORE_SIGMOID, bias=bias, n_group=G, topk_group=TG,
                      norm_topk=1, routed_scale=2.5)
    gpu_ctx.sync()
    lg = np.ascontiguousarray(logits.cpu().numpy())
    b = np.ascontiguousarray(bias.cpu().numpy())
    rid = np.zeros((T, k), np.int32)
    rw = np.zeros((T, k), np.float32)
    assert O.oracle().orc_route_sigmoid_grouped(O.p(lg, O.f32p), O.p(b, O.f32p), T, E, G, TG, k, 1, 2.5,
                                                O.p(rid, O.i32p), O.p(rw, O.f32p)) == 0
    got_ids = ids.cpu().numpy()
    mism = np.nonzero(np.any(got_ids != rid, axis=1))[0]
    for t in mism:
        g_ulps, e_ulps = sigmoid_route_boundary_ulps(lg[t], b, G, TG, k)
        assert e_ulps <= 4.0 or g_ulps <= 8.0, (t, g_ulps, e_ulps)
    print(f"T={T}: router rows differing at near-ties: {len(mism)}")
    out = run(gpu_ctx, layer, x, ids, wts, seed=54)
    rows = np.array(sorted({0, 1, T // 2, T - 1}))
    ref = torch.from_numpy(expected_from_device(layer, x, ids, wts, rows)).double().cuda()
    got = out[torch.from_numpy(rows).cuda()]
    err = float((got - ref).abs().max() / ref.abs().max())
    print(f"T={T}: expert output max-rel {err:.3e} on rows {rows.tolist()}")
    assert err <= TOL


def test_moe_ffn_fp8_rejects_bad_sizes(gpu_ctx):
    import torch

    x = torch.zeros(4, 100, dtype=torch.bfloat16, device="cuda")
    ids = torch.zeros(4, 2, dtype=torch.int32, device="cuda")
    w = torch.zeros(4, 2, device="cuda")
    h = torch.zeros(4, 100, device="cuda")
    z8 = torch.zeros(1, dtype=torch.uint8, device="cuda")
    zf = torch.zeros(1, device="cuda")
    with pytest.raises(dsb.DsbError) as e:
        gpu_ctx.moe_ffn_fp8(z8, zf, z8.view(1, 1), zf, E=4, n_shared=0, x=x, ids=ids, weights=w, h=h)
    assert e.value.code == dsb.DSB_EINVAL
