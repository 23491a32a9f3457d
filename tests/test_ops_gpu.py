"""Row and routing kernels (through the C ABI) against the CPU oracle.

Integer results (router ids on identical logits, permutation, argmax) must be
bit-exact; floating-point results are compared with the tolerance written in
each test.
"""

import numpy as np
import pytest

import oracle as O
import deepseek_cpp_infer_b200 as dsb

pytestmark = pytest.mark.gpu


def cu(a):
    import torch

    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


@pytest.mark.parametrize("n", [512, 2048, 7168])
def test_rmsnorm(gpu_ctx, n):
    import torch

    rng = np.random.default_rng(n)
    rows = 5
    x = (rng.standard_normal((rows, n)) * 3).astype(np.float32)
    w = rng.standard_normal(n).astype(np.float32)
    yf = torch.empty(rows, n, device="cuda")
    yb = torch.empty(rows, n, dtype=torch.bfloat16, device="cuda")
    gpu_ctx.rmsnorm(cu(x), cu(w), 1e-6, y_bf16=yb, y_f32=yf)
    gpu_ctx.sync()
    for r in range(rows):
        ref = np.zeros(n, np.float32)
        O.oracle().orc_rmsnorm_f32(O.p(np.ascontiguousarray(x[r]), O.f32p), O.p(w, O.f32p), n, 1e-6, O.p(ref, O.f32p))
        # only the order of the sum of squares differs: a few ulp
        assert np.abs(yf[r].cpu().numpy() - ref).max() <= 1e-5 * np.abs(ref).max()
        assert np.abs(yb[r].float().cpu().numpy() - ref).max() <= 2 ** -7 * np.abs(ref).max()


@pytest.mark.parametrize("H,nope,R,P", [(16, 128, 512, 64), (8, 64, 128, 32)])
def test_kv_norm_rope_append(gpu_ctx, H, nope, R, P):
    import torch

    rng = np.random.default_rng(R + H)
    B, max_blocks, n_blocks = 6, 4, 30
    pos = np.array([0, 1, 63, 64, 200, 255], np.int32)
    bt = rng.permutation(n_blocks)[: B * max_blocks].reshape(B, max_blocks).astype(np.int32)
    kv = (rng.standard_normal((B, R + P)) * 2).astype(np.float32)
    w = (1 + 0.1 * rng.standard_normal(R)).astype(np.float32)
    q = O.f32_to_bf16(rng.standard_normal((B, H * (nope + P))))
    cache = torch.zeros(n_blocks, 64, R + P, dtype=torch.bfloat16, device="cuda")
    q_rope = torch.empty(B, H, P, dtype=torch.bfloat16, device="cuda")
    qd = torch.from_numpy(q.view(np.int16)).cuda().view(torch.bfloat16)
    gpu_ctx.kv_norm_rope_append(cu(kv), cu(w), qd, cu(pos), cu(bt), H, nope, R, P, 1e-6, 10000.0, cache, q_rope)
    gpu_ctx.sync()
    ref_cache = np.zeros((n_blocks, 64, R + P), np.uint16)
    ref_qr = np.zeros((B, H, P), np.float32)
    qf = O.bf16_to_f32(q).astype(np.float32)
    rc = O.oracle().orc_kv_norm_rope_append(
        O.p(kv, O.f32p), O.p(w, O.f32p), O.p(np.ascontiguousarray(qf), O.f32p), O.p(pos, O.i32p), O.p(bt, O.i32p),
        B, H, nope, R, P, 64, max_blocks, 1e-6, 10000.0, O.p(ref_cache, O.u16p), O.p(ref_qr, O.f32p))
    assert rc == 0
    got = O.bf16_to_f32(cache.view(torch.int16).cpu().numpy().view(np.uint16))
    exp = O.bf16_to_f32(ref_cache)
    # both sides round to bf16; fp32 differences of a few ulp may flip one bf16 rounding
    assert np.abs(got - exp).max() <= 2 ** -7 * np.abs(exp).max()
    assert np.count_nonzero(got) == np.count_nonzero(exp)
    qr = q_rope.float().cpu().numpy()
    assert np.abs(qr - ref_qr).max() <= 2 ** -7 * np.abs(ref_qr).max()


@pytest.mark.parametrize("T,D,E", [(33, 2048, 64), (300, 7168, 256), (65, 512, 16)])
def test_router_logits(gpu_ctx, T, D, E):
    """fp32 router logits (warp-per-dot kernel up to 64 tokens, tiled above)."""
    import torch

    rng = np.random.default_rng(4)
    x = rng.standard_normal((T, D)).astype(np.float32)
    w = (rng.standard_normal((E, D)) * 0.02).astype(np.float32)
    lg = torch.empty(T, E, device="cuda")
    gpu_ctx.router_logits(cu(x), cu(w), lg)
    gpu_ctx.sync()
    ref = x.astype(np.float64) @ w.astype(np.float64).T
    assert np.abs(lg.cpu().numpy() - ref).max() <= 1e-5 * np.abs(ref).max()


@pytest.mark.parametrize("E,k,norm", [(16, 4, 0), (64, 6, 0), (64, 6, 1), (256, 8, 1)])
def test_route_softmax_ids_bit_exact(gpu_ctx, E, k, norm):
    import torch

    rng = np.random.default_rng(E * 10 + k)
    T = 300
    logits = (rng.standard_normal((T, E)) * 2).astype(np.float32)
    ids = torch.empty(T, k, dtype=torch.int32, device="cuda")
    wts = torch.empty(T, k, device="cuda")
    gpu_ctx.moe_route(cu(logits), ids, wts, k, scoring=dsb.SCORE_SOFTMAX, norm_topk=norm, routed_scale=1.5)
    gpu_ctx.sync()
    rid = np.zeros((T, k), np.int32)
    rw = np.zeros((T, k), np.float32)
    O.oracle().orc_route_softmax_greedy(O.p(logits, O.f32p), T, E, k, norm, 1.5, O.p(rid, O.i32p), O.p(rw, O.f32p))
    assert np.array_equal(ids.cpu().numpy(), rid)
    assert np.abs(wts.cpu().numpy() - rw).max() <= 1e-6 * 1.5


def test_route_ties_go_to_lower_id(gpu_ctx):
    import torch

    logits = np.array([[0.0, 1.0, 1.0, 0.5, 1.0]], np.float32)
    ids = torch.empty(1, 2, dtype=torch.int32, device="cuda")
    wts = torch.empty(1, 2, device="cuda")
    gpu_ctx.moe_route(cu(logits), ids, wts, 2, norm_topk=1)
    gpu_ctx.sync()
    assert ids.cpu().tolist() == [[1, 2]]


@pytest.mark.parametrize("T", [1, 128, 4096])
def test_route_sigmoid_grouped_ids_bit_exact(gpu_ctx, T):
    import torch

    rng = np.random.default_rng(T)
    E, G, TG, k = 256, 8, 4, 8
    logits = (rng.standard_normal((T, E)) * 2).astype(np.float32)
    bias = (rng.standard_normal(E) * 0.01).astype(np.float32)
    ids = torch.empty(T, k, dtype=torch.int32, device="cuda")
    wts = torch.empty(T, k, device="cuda")
    gpu_ctx.moe_route(cu(logits), ids, wts, k, scoring=dsb.SCORE_SIGMOID, bias=cu(bias), n_group=G, topk_group=TG,
                      norm_topk=1, routed_scale=2.5)
    gpu_ctx.sync()
    rid = np.zeros((T, k), np.int32)
    rw = np.zeros((T, k), np.float32)
    O.oracle().orc_route_sigmoid_grouped(O.p(logits, O.f32p), O.p(bias, O.f32p), T, E, G, TG, k, 1, 2.5,
                                         O.p(rid, O.i32p), O.p(rw, O.f32p))
    got = ids.cpu().numpy()
    # Bit-exact except at exact fp32 ties: CUDA's expf and the C library's
    # differ by up to 2 ulp, so a row may differ only where a selection
    # boundary is within that error - the 4th/5th group scores (each a sum
    # of two biased sigmoids) or the 8th/9th biased sigmoid of the kept groups
    mism = np.nonzero(np.any(got != rid, axis=1))[0]
    for t in mism:
        g_ulps, e_ulps = sigmoid_route_boundary_ulps(logits[t], bias, G, TG, k)
        print(f"row {t}: group boundary {g_ulps:.1f} ulp, expert boundary {e_ulps:.1f} ulp")
        # a biased sigmoid carries up to ~4 ulp (expf 2, the add, the division,
        # the bias), a group score the sum of two of them
        assert e_ulps <= 4.0 or g_ulps <= 8.0, (t, g_ulps, e_ulps, got[t], rid[t])
    ok = np.ones(T, bool)
    ok[mism] = False
    assert np.abs(wts.cpu().numpy()[ok] - rw[ok]).max() <= 2e-6 * 2.5


def sigmoid_route_boundary_ulps(x, bias, G, TG, k):
    """Gaps, in fp32 ulps of the boundary value, at the two decisions of the
    sigmoid + bias grouped router for one row: the TG-th vs (TG+1)-th group
    score (sum of the group's two largest biased sigmoids) and the k-th vs
    (k+1)-th biased sigmoid among the kept groups' experts.  Scores are
    computed in float64 and rounded to fp32, as an exact sigmoid would give."""
    s = (1.0 / (1.0 + np.exp(-x.astype(np.float64)))).astype(np.float32)
    sb = (s + bias).astype(np.float32)
    E = len(x)
    grp = sb.reshape(G, E // G)
    gs = np.sort(np.sort(grp, axis=1)[:, -2:].astype(np.float64).sum(axis=1).astype(np.float32))[::-1]
    g_gap = float(gs[TG - 1]) - float(gs[TG]) if TG < G else np.inf
    g_ulps = g_gap / float(np.spacing(np.float32(abs(gs[TG - 1]))))
    kept = np.argsort(-np.sort(grp, axis=1)[:, -2:].astype(np.float64).sum(axis=1), kind="stable")[:TG]
    cand = np.sort(np.concatenate([grp[g] for g in kept]))[::-1]
    e_gap = float(cand[k - 1]) - float(cand[k])
    e_ulps = e_gap / float(np.spacing(np.float32(abs(cand[k - 1]))))
    return g_ulps, e_ulps


@pytest.mark.parametrize("T,k,E", [(1, 8, 256), (37, 4, 16), (32, 6, 64), (4096, 8, 256)])
def test_permute_bit_exact(gpu_ctx, T, k, E):
    import torch

    rng = np.random.default_rng(T + E)
    ids = np.stack([rng.choice(E, k, replace=False) for _ in range(T)]).astype(np.int32)
    counts = torch.empty(E, dtype=torch.int32, device="cuda")
    offsets = torch.empty(E + 1, dtype=torch.int32, device="cuda")
    dest = torch.empty(T * k, dtype=torch.int32, device="cuda")
    src = torch.empty(T * k, dtype=torch.int32, device="cuda")
    gpu_ctx.moe_permute(cu(ids), E, counts, offsets, dest, src)
    gpu_ctx.sync()
    rc, ro, rd, rs = (np.zeros(n, np.int32) for n in (E, E + 1, T * k, T * k))
    O.oracle().orc_moe_permute(O.p(ids, O.i32p), T, k, E, O.p(rc, O.i32p), O.p(ro, O.i32p), O.p(rd, O.i32p),
                               O.p(rs, O.i32p))
    for a, b in ((counts, rc), (offsets, ro), (dest, rd), (src, rs)):
        assert np.array_equal(a.cpu().numpy(), b)


def test_gather_combine_argmax_embed(gpu_ctx):
    import torch

    rng = np.random.default_rng(12)
    T, k, D, E, V = 9, 3, 256, 8, 1000
    ids = np.stack([rng.choice(E, k, replace=False) for _ in range(T)]).astype(np.int32)
    counts = torch.empty(E, dtype=torch.int32, device="cuda")
    offsets = torch.empty(E + 1, dtype=torch.int32, device="cuda")
    dest = torch.empty(T * k, dtype=torch.int32, device="cuda")
    src = torch.empty(T * k, dtype=torch.int32, device="cuda")
    gpu_ctx.moe_permute(cu(ids), E, counts, offsets, dest, src)
    x = torch.randn(T, D, device="cuda").to(torch.bfloat16)
    xp = torch.empty(T * k, D, dtype=torch.bfloat16, device="cuda")
    gpu_ctx.gather_rows(x, src, k, xp)
    y = torch.randn(T * k, D, device="cuda")
    sh = torch.randn(T, D, device="cuda")
    h = torch.randn(T, D, device="cuda")
    h0 = h.clone()
    gpu_ctx.moe_combine(y, dest, k, h, shared=sh)
    gpu_ctx.sync()
    s = src.cpu().numpy()
    assert torch.equal(xp.cpu(), x.cpu()[torch.from_numpy(s // k).long()])
    d = dest.cpu().numpy().reshape(T, k)
    ref = h0.cpu().clone()
    yc, shc = y.cpu(), sh.cpu()
    for t in range(T):
        acc = torch.zeros(D)
        for j in range(k):
            acc = acc + yc[d[t, j]]
        ref[t] = ref[t] + (acc + shc[t])
    assert torch.equal(h.cpu(), ref)
    # argmax: ties resolve to the first index
    logits = torch.randn(4, V, device="cuda")
    logits[1, 7] = 100.0
    logits[1, 900] = 100.0
    out = torch.empty(4, dtype=torch.int32, device="cuda")
    gpu_ctx.argmax(logits, out)
    gpu_ctx.sync()
    lc = np.ascontiguousarray(logits.cpu().numpy())
    for b in range(4):
        assert out[b].item() == O.oracle().orc_argmax_f32(O.p(np.ascontiguousarray(lc[b]), O.f32p), V)
    assert out[1].item() == 7
    # embedding gather
    table = torch.randn(50, D, device="cuda").to(torch.bfloat16)
    toks = torch.tensor([3, 0, 49], dtype=torch.int32, device="cuda")
    he = torch.empty(3, D, device="cuda")
    gpu_ctx.embed(table, toks, he)
    gpu_ctx.sync()
    assert torch.equal(he, table[toks.long()].float())
