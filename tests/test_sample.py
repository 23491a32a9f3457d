"""The sampling oracle (orc_sample, oracle/oracle.c) pinned against the
reference's own ds::core::Sampler (oracle/_ref), on the CPU.

The reference draws its uniform from std::mt19937(seed) inside sample();
oracle/_ref also exposes those draws, so the oracle is run on exactly the
reference's uniforms.  Where the reference's scan order is defined (no cut:
id order; a top-p cut: descending p, distinct here) the ids must be
identical draw for draw.  With a top-k cut alone the reference scans in
std::nth_element's unspecified arrangement, so there the ids must lie in
the same kept set and follow the same distribution (every id's frequency
over 20000 draws within 5 sigma of the oracle's probability)."""

import numpy as np
import pytest

import oracle as O

pytestmark = pytest.mark.skipif(not O.ref_available(), reason="reference build (oracle/_ref) not present")


def row(V=4096, scale=3.0, seed=0):
    return (np.random.default_rng(seed).standard_normal(V) * scale).astype(np.float32)


@pytest.mark.parametrize("cfg", [(0.7, 0, 0.0), (1.2, 0, 0.9), (1.0, 50, 0.8), (0.0, 0, 0.0), (-1.0, 0, 0.5),
                                 (1.0, 4096, 1.0), (2.0, 0, 0.999)])
def test_oracle_matches_reference_draw_for_draw(cfg):
    x = row()
    ids, u = O.ref_sampler(x, *cfg, seed=1234, n=3000)
    ours = np.array([O.sample(x, *cfg, float(r))[0] for r in u])
    assert np.array_equal(ours, ids), (cfg, int((ours != ids).sum()))


def oracle_probs(x, t, k, top_p):
    """The oracle's distribution: P(id) from its cumulative intervals over a fine grid of r."""
    n = 1 << 14
    r = (np.arange(n) + 0.5) / n
    ids = np.array([O.sample(x, t, k, top_p, float(v))[0] for v in r])
    return np.bincount(ids, minlength=x.size) / n


@pytest.mark.parametrize("cfg", [(1.0, 40, 0.0), (0.8, 200, 0.0)])
def test_top_k_distribution_matches_reference(cfg):
    x = row(V=2048, scale=2.0, seed=5)
    n = 20000
    ids, _ = O.ref_sampler(x, *cfg, seed=99, n=n)
    p = oracle_probs(x, *cfg)
    kept = set(np.argsort(-x, kind="stable")[: cfg[1]].tolist())  # the k largest (distinct values here)
    assert set(ids.tolist()) <= kept and set(np.flatnonzero(p > 0).tolist()) <= kept
    freq = np.bincount(ids, minlength=x.size) / n
    sigma = np.sqrt(p * (1 - p) / n) + 1.0 / n + 1.0 / (1 << 14)  # draws + the oracle grid's resolution
    assert np.all(np.abs(freq - p) <= 5 * sigma), float(np.max(np.abs(freq - p) / sigma))


def test_unfiltered_top_k_one_and_tiny_top_p_are_greedy():
    x = row(V=1000, seed=3)
    x[17] = x[901] = x.max() + 1.0  # a tie for the maximum: the lower id
    for r in (0.0, 0.3, 0.999999):
        assert O.sample(x, 1.0, 1, 0.0, r)[0] == 17
        assert O.sample(x, 1.0, 0, 1e-6, r)[0] == 17


from hypothesis import given, settings, strategies as st  # noqa: E402


@settings(max_examples=60, deadline=None, derandomize=True)
@given(seed=st.integers(0, 10**6), V=st.integers(2, 300), k=st.integers(0, 320), top_p=st.floats(0.0, 1.0),
       t=st.one_of(st.just(0.0), st.just(-1.0), st.floats(0.05, 3.0)), u1=st.floats(0.0, 0.999),
       u2=st.floats(0.0, 0.999))
def test_oracle_properties(seed, V, k, top_p, t, u1, u2):
    """orc_sample: the pick lies in the top-k set; with u growing the pick
    never moves earlier in the scan order (descending x, ties to the lower
    id, when a cut is active; id order otherwise); top_k = 1 is the argmax."""
    rng = np.random.default_rng(seed)
    x = (rng.standard_normal(V) * 2).astype(np.float32)
    if rng.random() < 0.3:
        x = np.round(x).astype(np.float32)  # ties
    lo, hi = sorted((u1, u2))
    a, b = O.sample(x, t, k, top_p, lo)[0], O.sample(x, t, k, top_p, hi)[0]
    p32 = np.float32(top_p)  # the arguments travel as float32
    filt = (0 < k < V) or (0.0 < p32 < 1.0)
    t32 = np.float32(t)
    xs = x / (np.float32(1.0) if t32 <= 0 else t32)
    order = list(np.lexsort((np.arange(V), -xs))) if filt else list(range(V))
    assert order.index(a) <= order.index(b)
    if 0 < k < V:
        assert a in order[:k] and b in order[:k]
    assert O.sample(x, t, 1, top_p, hi)[0] == int(np.argmax(xs))
