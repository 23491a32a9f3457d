"""dsb_sample (on-device stochastic sampling) through the C ABI.

The reference's algorithm (ds::core::Sampler::sample, restated as
orc_sample and pinned to the reference by tests/test_sample.py) accumulates
probabilities in float, left to right; over 1e5 items that sum drifts by
~1e-5, the width of a typical token's interval, so a float oracle cannot
judge single draws at full vocabulary size.  The kernel's pick is therefore
checked against the exact distribution: probabilities in double, the cuts
and the scan order of the reference with its unspecified orders fixed as the
kernel fixes them (descending x, ties to the lower id), and the id must own
the draw u within TOL (where the top-p cut lies within CUT of top_p, under
the cut keeping one item more or less too).  Stratified draws u_j = (j + 0.5) / n over n
copies of one row must land in every id's exact interval to within two
counts (an edge may cross one point).  The float oracle still agrees except
near interval edges.  Ties at the top-k boundary keep the lower ids;
top_k = 1 is the argmax; results are deterministic; sampled generate
replays the reference Sampler's draw stream."""

import numpy as np
import pytest
import torch

import deepseek_cpp_infer_b200 as dsb
import oracle as O

pytestmark = pytest.mark.gpu
TOL = 2e-6    # exact-interval slack for the kernel (fixed-point masses, expf)
CUT = 1e-6    # a top-p cut this close to top_p may keep one item more or less
EDGE = 1e-4   # where the float oracle may disagree: its left-to-right float sums


def exact_intervals(logits, t, k, p):
    """Candidate (ids in scan order, cumulative upper edges) in double
    precision: one, or two or three when the top-p cut lies within CUT of
    top_p (then the kernel may keep one item more or less)."""
    t = 1.0 if t <= 0 else t
    x = (np.asarray(logits, np.float32) / np.float32(t)).astype(np.float64)
    V = x.size
    fk, fp = 0 < k < V, 0.0 < p < 1.0
    order = np.lexsort((np.arange(V), -x)) if (fk or fp) else np.arange(V)
    if fk:
        order = order[:k]
    e = np.exp(x[order] - x[order].max())
    pr = e / e.sum()
    if not fp:
        return [(order, np.cumsum(pr))]
    c = np.cumsum(pr)
    n0 = min(int(np.searchsorted(c, p, side="left")) + 1, len(pr))
    cuts = {n0}
    if n0 >= 2 and c[n0 - 2] >= p - CUT:
        cuts.add(n0 - 1)
    if c[n0 - 1] < p + CUT and n0 < len(pr):
        cuts.add(n0 + 1)
    return [(order[:n], np.cumsum(pr[:n] / pr[:n].sum())) for n in sorted(cuts)]


def owns(ivs, got, u):
    """The id's exact interval (under one of the candidate cuts) holds u, within TOL."""
    for order, c in ivs:
        j = np.flatnonzero(order == got)
        if j.size == 1:
            j = int(j[0])
            lo = c[j - 1] if j > 0 else 0.0
            if lo - TOL <= u <= c[j] + TOL:
                return True
    return False


CFGS = [(1.0, 0, 0.0), (0.7, 50, 0.0), (1.0, 0, 0.9), (0.8, 40, 0.95), (1.3, 2000, 0.5), (1.0, 1, 0.0),
        (0.0, 0, 1.0), (2.0, 0, 0.999), (0.5, 5000, 0.0)]


def run(ctx, logits, u, t, k, p):
    lg = torch.from_numpy(logits).cuda()
    uu = torch.from_numpy(u).cuda()
    out = torch.full((logits.shape[0],), -7, dtype=torch.int32, device="cuda")
    ctx.sample(lg, uu, out, temperature=t, top_k=k, top_p=p)
    ctx.sync()
    return out.cpu().numpy()


@pytest.mark.parametrize("V", [37, 1000, 4096, 102400, 129280])
@pytest.mark.parametrize("cfg", CFGS)
def test_sample_matches_oracle(gpu_ctx, V, cfg):
    t, k, p = cfg
    B = 64
    rng = np.random.default_rng(V + 17 * k)
    base = (rng.standard_normal(V) * 3).astype(np.float32)
    logits = np.stack([base if b % 2 == 0 else (rng.standard_normal(V) * 2).astype(np.float32) for b in range(B)])
    u = rng.random(B, dtype=np.float32)
    got = run(gpu_ctx, logits, u, t, k, p)
    assert ((got >= 0) & (got < V)).all()
    for b in range(B):
        assert owns(exact_intervals(logits[b], t, k, p), got[b], float(u[b])), (b, got[b])
        want, margin, cut = O.sample(logits[b], t, k, p, float(u[b]))
        assert got[b] == want or margin < EDGE or cut < EDGE, (b, got[b], want, margin, cut)


@pytest.mark.parametrize("cfg", [(1.0, 0, 0.0), (1.0, 30, 0.0), (0.9, 0, 0.7), (1.0, 100, 0.9)])
def test_stratified_draws_reproduce_the_distribution(gpu_ctx, cfg):
    V, n = 20000, 2048
    x = (np.random.default_rng(11).standard_normal(V) * 2.5).astype(np.float32)
    u = ((np.arange(n) + 0.5) / n).astype(np.float32)
    got = run(gpu_ctx, np.ascontiguousarray(np.broadcast_to(x, (n, V))), u, *cfg)
    order, c = exact_intervals(x, *cfg)[0]
    slot = np.minimum(np.searchsorted(c, u.astype(np.float64), side="left"), len(order) - 1)
    cg, cw = np.bincount(got, minlength=V), np.bincount(order[slot], minlength=V)
    # an interval edge may move across at most one stratum point: +-1 per edge
    assert np.abs(cg - cw).max() <= 2 and np.abs(cg - cw).sum() <= 8, (np.abs(cg - cw).max(), np.abs(cg - cw).sum())


def test_ties_keep_lower_ids_and_top1_is_argmax(gpu_ctx):
    V, B = 3000, 48
    rng = np.random.default_rng(4)
    logits = rng.integers(-4, 4, size=(B, V)).astype(np.float32)  # many equal values
    u = rng.random(B, dtype=np.float32)
    for k, p in [(1, 0.0), (10, 0.0), (700, 0.0), (10, 0.6), (0, 0.3), (0, 0.0)]:
        got = run(gpu_ctx, logits, u, 1.0, k, p)
        for b in range(B):
            assert owns(exact_intervals(logits[b], 1.0, k, p), got[b], float(u[b])), (k, p, b, got[b])
    got = run(gpu_ctx, logits, u, 1.0, 1, 0.0)
    assert np.array_equal(got, np.argmax(logits, axis=1).astype(np.int32))


def test_deterministic_and_rejects_bad_arguments(gpu_ctx):
    V, B = 129280, 32
    rng = np.random.default_rng(8)
    logits = (rng.standard_normal((B, V)) * 4).astype(np.float32)
    u = rng.random(B, dtype=np.float32)
    a = run(gpu_ctx, logits, u, 0.8, 0, 0.95)
    b = run(gpu_ctx, logits, u, 0.8, 0, 0.95)
    assert np.array_equal(a, b)
    lg = torch.zeros(2, 8, device="cuda")
    uu = torch.zeros(2, device="cuda")
    out = torch.zeros(2, dtype=torch.int32, device="cuda")
    for bad in [dict(logits=lg[:, :0]), dict(top_p=float("nan"))]:
        kw = dict(logits=lg, uniforms=uu, out=out)
        kw.update(bad)
        with pytest.raises(dsb.DsbError):
            gpu_ctx.sample(**kw)


# ------------------------------------------------------- whole-model sampling

@pytest.fixture(scope="module")
def tiny_model(gpu_ctx):
    from deepseek_cpp_infer_b200.workloads import TINY, model_tensors

    m = dsb.Model(gpu_ctx, dsb.ModelConfig(**TINY))
    for name, a in model_tensors(TINY, seed=0).items():
        m.set_tensor(name, a)
    m.finalize()
    yield m
    m.close()


PROMPTS = [[5, 99, 1024, 7, 3000], [42, 8], [1, 2, 3, 4, 5, 6, 7, 8, 9]]


def test_generate_sampled_replays_the_reference_draw_stream(gpu_ctx, tiny_model):
    """B = 1: dsb_generate_sampled's ids equal a replay through
    dsb_decode_step_sampled fed the reference Sampler's own uniforms
    (std::mt19937(seed)), and each owns its draw in the exact distribution of
    that step's logits."""
    cfg = dsb.Sampling(temperature=1.5, top_k=0, top_p=0.95, seed=1234)
    n_new = 24
    kv = dsb.KVCache(gpu_ctx, tiny_model, n_blocks=16, max_seqs=2, max_blocks_per_seq=4)
    s = kv.alloc_seq()
    gen = dsb.generate(gpu_ctx, tiny_model, kv, [s], [PROMPTS[0]], n_new, sampling=cfg)[0]
    kv.free_seq(s)
    assert len(gen) == n_new
    _, u = O.ref_sampler(np.zeros(8, np.float32), 1.0, 0, 0.0, 1234, n_new)  # the reference's draws
    s = kv.alloc_seq()
    for tok in PROMPTS[0][:-1]:
        dsb.decode_step(gpu_ctx, tiny_model, kv, [s], [tok])
    tok = PROMPTS[0][-1]
    for j in range(n_new):
        ids, lg = dsb.decode_step_sampled(gpu_ctx, tiny_model, kv, [s], [tok], cfg, [u[j]], want_logits=True)
        assert ids[0] == gen[j], (j, ids[0], gen[j])
        assert owns(exact_intervals(lg[0], cfg.temperature, cfg.top_k, cfg.top_p), ids[0], float(u[j])), j
        tok = int(ids[0])
    kv.close()


def test_generate_sampled_batches_and_degenerate_settings(gpu_ctx, tiny_model):
    kv = dsb.KVCache(gpu_ctx, tiny_model, n_blocks=32, max_seqs=4, max_blocks_per_seq=4)
    sids = [kv.alloc_seq() for _ in PROMPTS]
    greedy = dsb.generate(gpu_ctx, tiny_model, kv, sids, PROMPTS, 12)
    for s in sids:
        kv.free_seq(s)
    for cfg in (dsb.Sampling(0.0, 0, 0.0, 7), dsb.Sampling(1.0, 1, 0.0, 7), dsb.Sampling(0.9, 0, 1e-7, 7)):
        sids = [kv.alloc_seq() for _ in PROMPTS]
        got = dsb.generate(gpu_ctx, tiny_model, kv, sids, PROMPTS, 12, sampling=cfg)
        for s in sids:
            kv.free_seq(s)
        assert got == greedy, (cfg.temperature, cfg.top_k, cfg.top_p)
    # a real sampling setting: deterministic for a fixed seed, every sequence its own stream
    cfg = dsb.Sampling(1.2, 40, 0.9, 99)
    runs = []
    for _ in range(2):
        sids = [kv.alloc_seq() for _ in PROMPTS]
        runs.append(dsb.generate(gpu_ctx, tiny_model, kv, sids, PROMPTS, 12, sampling=cfg))
        for s in sids:
            kv.free_seq(s)
    assert runs[0] == runs[1] and runs[0] != greedy
    with pytest.raises(dsb.DsbError):
        s = kv.alloc_seq()
        dsb.decode_step_sampled(gpu_ctx, tiny_model, kv, [s], [1], cfg, [1.5])
    kv.close()
