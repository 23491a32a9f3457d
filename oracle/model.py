"""Whole-model teacher-forced forward composed from the oracle's layer
functions (TEST INFRASTRUCTURE ONLY; see oracle/__init__.py for who may
import it).

It follows DeepSeekModel::decode_next (src/models/deepseek/model.cpp:117-184)
position by position: embedding row -> per layer RMSNorm -> MLA
(orc_mla_layer_seq_f32, the absorbed restatement of mla_decode_step) ->
residual -> RMSNorm -> dense MLP (dense_mlp_step, ops.cpp:96-108) or
softmax-greedy MoE (moe_step, ops.cpp:110-146) -> residual; final RMSNorm and
lm_head.  Every position of a layer is computed before the next layer, which
is the same arithmetic because position t only attends to positions <= t.

Besides the logits it reports, per position, the router margin of every MoE
layer: the k-th largest minus the (k+1)-th largest fp32 gate logit.  Where it
is small, a relative perturbation of the layer input far below bf16
resolution can swap the last routed expert; `swaps` forces such a swap (the
(k+1)-th expert takes the k-th slot with its own probability) at chosen
(layer, position) pairs, giving the output the reference would produce had
its router broken the near-tie the other way.

Covers the configurations with q_lora_rank 0 and softmax scoring (DeepSeek-V2
style); dimensions come from the same config dict as workloads.TINY.

forward_fp8 is the same forward for a block-scaled FP8 checkpoint (weights
e4m3 + 128x128 scales, as DeepSeek-V3 ships them; the reference has no FP8
path, so this is a restatement): every FP8 linear uses the dequantised
weight (e4m3 * scale) and sees its input as the FP8 GEMM does, rounded to
the bf16 activation and quantised per token and 128 columns
(orc_act_fp8_roundtrip).  The quantisation points are the projections' input
(the attention norm), o_proj's input, the dense FFN's input and its
SiLU(gate) * up activation, and every routed and shared expert's input and
activation; kv_b_proj is dequantised to bf16 once (absorbed attention keeps
it in bf16), the router and lm_head stay unquantised.

An e4m3 code is 6-12% wide, so a quantiser that sees an input one bf16 step
away rounds it to another code, and such flips compound over the layers.
forward_fp8 therefore also stores every activation at the precision a
batched B200 decode stores it, so that both feed the same bytes to every
quantiser: the latent cache rows [c | kr] in bf16, the query's nope part and
rotated rope part in bf16, the absorbed query q_lat = W_UK^T q_nope in bf16,
the attention probabilities in bf16 relative to a running maximum that is
only raised when a 64-token tile exceeds it by 2^8 (log2 domain), the
latent output and the per-head W_UV output in bf16, and the final norm in
bf16 before the lm_head.  A sequence longer than a work item (runs of whole
64-token pages planned from the lengths and the number of SMs, as
_mla_items restates) is attended per item and the items' partial sums are
merged by their maxima.  The arithmetic is the reference's absorbed MLA
(mla.cpp:41-119 re-associated); only where values are rounded follows the
batched kernels.
"""

from __future__ import annotations

import numpy as np

from . import f32p, i32p, oracle, p, u8p, u16p


def _f32(a):
    return np.ascontiguousarray(np.asarray(a, dtype=np.float32))


def _rmsnorm_rows(x, w, eps):
    out = np.zeros_like(x)
    for i in range(x.shape[0]):
        o = np.zeros(x.shape[1], np.float32)
        oracle().orc_rmsnorm_f32(p(_f32(x[i]), f32p), p(w, f32p), x.shape[1], eps, p(o, f32p))
        out[i] = o
    return out


def forward(cfg: dict, tensors: dict, seq, swaps=()):
    """Logits [T, V] for every position of `seq` and router margins
    {layer: [T] float64}.  `swaps`: iterable of (layer, position)."""
    if cfg.get("q_lora_rank", 0) or cfg.get("scoring_func", 0) != 0:
        raise NotImplementedError("oracle.model covers q_lora_rank 0 with softmax scoring")
    c = cfg
    W = {n: _f32(a) for n, a in tensors.items()}
    seq = np.asarray(seq, np.int64)
    T = len(seq)
    D, H, R = c["hidden_size"], c["num_attention_heads"], c["kv_lora_rank"]
    nope, rope, v = c["qk_nope_head_dim"], c["qk_rope_head_dim"], c["v_head_dim"]
    E, k, I = c["n_routed_experts"], c["num_experts_per_tok"], c["moe_intermediate_size"]
    eps = c["rms_norm_eps"]
    swaps = set(swaps)
    orc = oracle()
    h = _f32(W["model.embed_tokens.weight"][seq])
    margins = {}
    for li in range(c["num_hidden_layers"]):
        pre = f"model.layers.{li}."
        xn = _rmsnorm_rows(h, W[pre + "input_layernorm.weight"], eps)
        out = np.zeros((T, D), np.float32)
        rc = orc.orc_mla_layer_seq_f32(
            D, H, nope, rope, v, R, eps, c["rope_theta"],
            *(p(W[pre + "self_attn." + n + ".weight"], f32p)
              for n in ("q_proj", "kv_a_proj_with_mqa", "kv_a_layernorm", "kv_b_proj", "o_proj")),
            p(xn, f32p), T, p(out, f32p))
        assert rc == 0
        h = _f32(h + out)
        xn = _rmsnorm_rows(h, W[pre + "post_attention_layernorm.weight"], eps)
        out = np.zeros((T, D), np.float32)
        if pre + "mlp.gate.weight" not in W:
            wg, wu, wd = (W[pre + "mlp." + n + "_proj.weight"] for n in ("gate", "up", "down"))
            for t in range(T):
                o = np.zeros(D, np.float32)
                orc.orc_dense_mlp_f32(p(wg, f32p), p(wu, f32p), p(wd, f32p), p(_f32(xn[t]), f32p), D, wg.shape[0],
                                      p(o, f32p))
                out[t] = o
        else:
            eg, eu, ed = (_f32(np.stack([W[pre + f"mlp.experts.{e}.{n}_proj.weight"] for e in range(E)]))
                          for n in ("gate", "up", "down"))
            shared = pre + "mlp.shared_experts.gate_proj.weight" in W
            sg, su, sd = ((W[pre + f"mlp.shared_experts.{n}_proj.weight"] for n in ("gate", "up", "down"))
                          if shared else (None, None, None))
            Is = sg.shape[0] if shared else 0
            wgate = W[pre + "mlp.gate.weight"]
            margin = np.zeros(T)
            for t in range(T):
                x = _f32(xn[t])
                logits = np.zeros(E, np.float32)
                orc.orc_linear_f32(p(wgate, f32p), p(x, f32p), D, p(logits, f32p), E)
                srt = np.sort(logits.astype(np.float64))[::-1]
                margin[t] = srt[k - 1] - srt[k] if k < E else np.inf
                ids = np.zeros(k + 1 if k < E else k, np.int32)
                w = np.zeros(len(ids), np.float32)
                # top-(k+1) in the reference's order: the (k+1)-th is the swap candidate
                assert orc.orc_route_softmax_greedy(p(_f32(logits), f32p), 1, E, len(ids), 0, 1.0, p(ids, i32p),
                                                    p(w, f32p)) == 0
                if (li, t) in swaps:
                    ids[k - 1], w[k - 1] = ids[k], w[k]
                ids, w = np.ascontiguousarray(ids[:k]), _f32(w[:k])
                if c["norm_topk_prob"]:
                    s = np.float32(0)
                    for j in range(k):
                        s = np.float32(s + w[j])
                    if s > 0:
                        w = _f32(w / s)
                o = np.zeros(D, np.float32)
                orc.orc_moe_mix_f32(p(eg, f32p), p(eu, f32p), p(ed, f32p),
                                    *((p(a, f32p) for a in (sg, su, sd)) if shared else (None, None, None)),
                                    Is, D, I, k, p(ids, i32p), p(w, f32p), c["routed_scaling_factor"], p(x, f32p),
                                    p(o, f32p))
                out[t] = o
            margins[li] = margin
        h = _f32(h + out)
    hn = _rmsnorm_rows(h, W["model.norm.weight"], eps)
    logits = np.zeros((T, W["lm_head.weight"].shape[0]), np.float32)
    for t in range(T):
        orc.orc_linear_f32(p(W["lm_head.weight"], f32p), p(_f32(hn[t]), f32p), D, p(logits[t], f32p),
                           logits.shape[1])
    return logits, margins


def _bf16_round(a):
    """fp32 -> bf16 (round to nearest even) -> fp32."""
    a = _f32(a)
    u = np.zeros(a.shape, np.uint16)
    out = np.zeros(a.shape, np.float32)
    oracle().orc_f32_to_bf16_n(p(a, f32p), a.size, p(u, u16p))
    oracle().orc_bf16_to_f32_n(p(u, u16p), a.size, p(out, f32p))
    return out


def moe_fp8(x, ids, weights, gate_q, gate_s, up_q, up_s, down_q, down_s):
    """moe_step (src/models/deepseek/ops.cpp:133-145) with block-scaled FP8
    expert linears, per token: x quantised per 128 columns, gate/up through
    orc_fp8_linear, silu(gate) * up in fp32 rounded to the bf16 activation,
    that quantised again, the down projection, then out += w * expert(x) over
    the picks in order.

    x fp32 [T, D]; ids int32 / weights fp32 [T, kk] (shared experts included
    as picks of weight 1); gate_q/up_q uint8 [G, I, D] with scales
    [G, I/128, D/128]; down_q uint8 [G, D, I] with [G, D/128, I/128].
    Returns the fp32 [T, D] expert sum (without the residual)."""
    orc = oracle()
    T, D = x.shape
    I = gate_q.shape[1]
    out = np.zeros((T, D), np.float32)
    xq = np.zeros((1, D), np.uint8)
    xs = np.zeros((1, D // 128), np.float32)
    mq = np.zeros((1, I), np.uint8)
    ms = np.zeros((1, I // 128), np.float32)
    for t in range(T):
        orc.orc_quant_act_1x128(p(_f32(x[t : t + 1]), f32p), 1, D, p(xq, u8p), p(xs, f32p))
        acc = np.zeros(D, np.float32)
        for e, wt in zip(ids[t], weights[t]):
            g = np.zeros(I, np.float32)
            u = np.zeros(I, np.float32)
            orc.orc_fp8_linear(p(gate_q[e], u8p), p(gate_s[e], f32p), p(xq, u8p), p(xs, f32p), 1, I, D, p(g, f32p))
            orc.orc_fp8_linear(p(up_q[e], u8p), p(up_s[e], f32p), p(xq, u8p), p(xs, f32p), 1, I, D, p(u, f32p))
            # the activation between the two GEMMs is bf16 (then e4m3 per 1x128)
            mid = _bf16_round(_f32(g / (np.float32(1) + np.exp(-g)) * u))
            orc.orc_quant_act_1x128(p(mid.reshape(1, I), f32p), 1, I, p(mq, u8p), p(ms, f32p))
            y = np.zeros(D, np.float32)
            orc.orc_fp8_linear(p(down_q[e], u8p), p(down_s[e], f32p), p(mq, u8p), p(ms, f32p), 1, D, I, p(y, f32p))
            acc = _f32(acc + np.float32(wt) * y)
        out[t] = acc
    return out


def _act_fp8(x):
    """orc_act_fp8_roundtrip on a copy of x (rows = tokens)."""
    a = np.array(_f32(x), copy=True)
    a2 = a.reshape(-1, a.shape[-1])
    oracle().orc_act_fp8_roundtrip(p(a2, f32p), a2.shape[0], a2.shape[1])
    return a


class Fp8Quantiser:
    """The e4m3 activation quantisation points of forward_fp8, with rounding
    ambiguity made explicit.  An activation is rounded to bf16 and then
    quantised per 128 columns; the GPU computes the fp32 value before the
    bf16 rounding with another summation order, so where that value lies
    within `eps` (relative) of a bf16 rounding midpoint the GPU may hold the
    other bf16 neighbour, and where that neighbour quantises to another e4m3
    code the difference reaches the next GEMM.  Such elements are recorded
    in `fragile` as (tag, position, column, distance); `flips` holds
    (tag, position, column) triples for which the other neighbour is used."""

    def __init__(self, flips=(), eps=3e-5, eps_store=3e-6, record=True):
        self.flips = set(flips)
        self.eps = eps
        self.eps_store = eps_store
        self.record = record
        self.fragile = []

    def bf16(self, x, tag, positions):
        """A bf16 storage point (rows = positions): the value rounded to bf16,
        or to the other neighbour where flipped; every element within
        eps_store of a rounding midpoint is recorded (any flip changes the
        stored value)."""
        a = _f32(x).reshape(-1, np.shape(x)[-1])
        b, other, dist = self._neighbours(a)
        self._apply(b, other, tag, positions)
        if self.record:
            for r, c in zip(*np.nonzero(dist <= self.eps_store)):
                if (tag, positions[r], c) not in self.flips:
                    self.fragile.append((tag, positions[r], int(c), float(dist[r, c])))
        return b.reshape(np.shape(x))

    def _neighbours(self, a):
        b = _bf16(a)
        # the other bf16 neighbour (one bf16 step = 2^16 in the fp32 bit
        # pattern), on the side of the fp32 value
        u = b.view(np.uint32).astype(np.int64)
        step = np.where((a > b) == (b >= 0), 1, -1) * 65536
        other = (u + step).astype(np.uint32).view(np.float32).reshape(a.shape)
        mid = (b.astype(np.float64) + other.astype(np.float64)) / 2
        # distance to the midpoint relative to the value, or to a hundredth of
        # its 128-column block's largest value where the value is smaller
        # (a GEMM's fp32 error scales with its terms, not with a small sum)
        nb = (a.shape[1] + 127) // 128
        pad = np.zeros((a.shape[0], nb * 128))
        pad[:, : a.shape[1]] = np.abs(a)
        bmax = np.repeat(pad.reshape(a.shape[0], nb, 128).max(axis=2), 128, axis=1)[:, : a.shape[1]]
        dist = np.abs(a.astype(np.float64) - mid) / np.maximum(np.abs(a.astype(np.float64)), 0.01 * bmax + 1e-30)
        return b, other, dist

    def _apply(self, b, other, tag, positions):
        if self.flips:
            row_of = {pos: r for r, pos in enumerate(positions)}
            for (ftag, pos, c) in self.flips:
                if ftag == tag and pos in row_of:
                    b[row_of[pos], c] = other[row_of[pos], c]

    def __call__(self, x, tag, positions):
        a = _f32(x).reshape(-1, np.shape(x)[-1])
        b, other, dist = self._neighbours(a)
        self._apply(b, other, tag, positions)
        out = b.copy()
        oracle().orc_act_fp8_roundtrip(p(out, f32p), out.shape[0], out.shape[1])
        if self.record:
            for r, c in zip(*np.nonzero(dist <= self.eps)):
                if (tag, positions[r], c) in self.flips:
                    continue
                row = b[r:r + 1].copy()
                row[0, c] = other[r, c]
                oracle().orc_act_fp8_roundtrip(p(row, f32p), 1, row.shape[1])
                if not np.array_equal(row[0], out[r]):
                    self.fragile.append((tag, positions[r], int(c), float(dist[r, c])))
        return out.reshape(np.shape(x))


def _silu_mul(g, u):
    return _f32(g / (np.float32(1) + np.exp(-g)) * u)


def _bf16(a):
    """fp32 -> bf16 (round to nearest even) -> fp32, vectorised (finite inputs)."""
    u = np.ascontiguousarray(a, np.float32).view(np.uint32).astype(np.uint64)
    u = (u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000
    return u.astype(np.uint32).view(np.float32).reshape(np.shape(a))


def _mla_items(seq_lens, slots, H, R, P):
    """Work items of the split-KV MLA decode: runs of whole 64-token pages per
    sequence, (b, first page, pages, end token, split).  Candidate run
    lengths (the longest sequence in 1..16 equal runs, all pages spread over
    1..8 waves) are scored by a longest-first list schedule over `slots`:
    an item costs its pages + 2, and when its sequence is split, 1 + the
    bytes of its fp32 partial [H, R] written and read back in pages
    (64 x (R + P) bf16); the cheapest wins, at most 256 pages per item."""
    import heapq

    pages = [(int(L) + 63) // 64 for L in seq_lens]
    total, maxp = sum(pages), max([1] + pages)
    split_cost = 1.0 + float(H) * R * 4 * 2 / (64.0 * (R + P) * 2)
    caps = {min(maxp, 256)}
    for n in range(2, 17):
        caps.add(max(2, min((maxp + n - 1) // n, 256)))
    for k in range(1, 9):
        c = (total + k * slots - 1) // (k * slots)
        caps.add(max(2, min(c, 256)))
    caps = sorted(caps)
    best_cap, best = caps[-1], 1e300
    for cap in caps:
        costs = []
        for n_p in pages:
            n = (n_p + cap - 1) // cap
            for i in range(n):
                costs.append((i + 1) * n_p // n - i * n_p // n + 2.0 + (split_cost if n > 1 else 0.0))
        costs.sort(reverse=True)
        heap = [0.0] * slots
        span = 0.0
        for c in costs:
            t0 = heapq.heappop(heap)
            heapq.heappush(heap, t0 + c)
            span = max(span, t0 + c)
        if span < best - 1e-9:
            best, best_cap = span, cap
    items = []
    for b, n_p in enumerate(pages):
        n = (n_p + best_cap - 1) // best_cap
        for i in range(n):
            p0, p1 = i * n_p // n, (i + 1) * n_p // n
            items.append((b, p0, p1 - p0, min(int(seq_lens[b]), p1 * 64), n > 1))
    return items


def _attend_item(q_lat, q_rope, c, kr, tok0, tok_end, scale_log2, pstore=None):
    """One work item of the latent attention for all heads: tokens [tok0,
    tok_end) of the cache rows c [T, R], kr [T, P] (bf16 values); q_lat
    [H, R], q_rope [H, P] (bf16 values).  Scores in the log2 domain, a
    running maximum per head raised only when a 64-token tile exceeds it by
    8, probabilities rounded to bf16 and summed as rounded.  Returns the
    unnormalised output O [H, R] (fp32), the maximum m and the sum l [H]."""
    H = q_lat.shape[0]
    m = np.full(H, -np.inf, np.float32)
    l = np.zeros(H, np.float64)
    O = np.zeros((H, c.shape[1]), np.float64)
    for t0 in range(tok0, tok_end, 64):
        t1 = min(t0 + 64, tok_end)
        s = q_lat.astype(np.float64) @ c[t0:t1].T.astype(np.float64) + \
            q_rope.astype(np.float64) @ kr[t0:t1].T.astype(np.float64)
        s = s.astype(np.float32) * np.float32(scale_log2)
        mt = s.max(axis=1)
        up = mt > m + np.float32(8.0)
        factor = np.where(up, np.exp2((m - mt).astype(np.float64)).astype(np.float32), np.float32(1.0))
        m = np.where(up, mt, m)
        O *= factor[:, None].astype(np.float64)
        l *= factor.astype(np.float64)
        pr = np.exp2((s - m[:, None]).astype(np.float64)).astype(np.float32)
        pr = _bf16(pr) if pstore is None else pstore(pr, t0)
        l += pr.astype(np.float64).sum(axis=1)
        O += pr.astype(np.float64) @ c[t0:t1].astype(np.float64)
    return O.astype(np.float32), m, l.astype(np.float32)


def _attend_sequence(q_lat, q_rope, c, kr, items, scale_log2, pstore=None):
    """One sequence's latent attention output [H, R] over its work items
    (all items of `items` must belong to it), in fp32 before its bf16
    rounding: a whole-sequence item normalises its own sum; split items are
    merged as sum_i 2^(m_i - M) O_i / sum_i 2^(m_i - M) l_i."""
    parts = [(_attend_item(q_lat, q_rope, c, kr, p0 * 64, end, scale_log2, pstore), split)
             for (_, p0, n_p, end, split) in items]
    if len(parts) == 1 and not parts[0][1]:
        Ow, _, lw = parts[0][0]
        return _f32(Ow * (np.float32(1.0) / lw)[:, None])
    M = np.max(np.stack([m for (_, m, _), _ in parts]), axis=0)
    den = np.zeros(q_lat.shape[0], np.float32)
    acc = np.zeros((q_lat.shape[0], c.shape[1]), np.float32)
    for (Ow, m, lw), _ in parts:
        w = np.exp2((m - M).astype(np.float64)).astype(np.float32)
        den = _f32(den + w * lw)
        acc = _f32(acc + w[:, None] * Ow)
    return _f32(acc * (np.float32(1.0) / den)[:, None])


def mla_decode_storage_points(q_lat, q_rope, cache, block_table, seq_lens, scale, slots=148):
    """Absorbed MLA decode over a paged latent cache (kv_lora_rank 128, one
    CTA per work item) at the batched kernel's storage points: q_lat [B, H,
    R], q_rope [B, H, P], cache [n_blocks, 64, R + P] as fp32 arrays of bf16
    values; the batch is planned into work items as the kernel plans it
    (_mla_items over `slots`); returns [B, H, R] bf16 values as fp32."""
    B, H, R = q_lat.shape
    scale_log2 = np.float32(np.float32(scale) * np.float32(1.4426950408889634))
    items = _mla_items(seq_lens, slots, H, R, q_rope.shape[2])
    out = np.zeros((B, H, R), np.float32)
    for b in range(B):
        L = int(seq_lens[b])
        pages = block_table[b, : (L + 63) // 64]
        rows = cache[pages].reshape(-1, cache.shape[2])
        out[b] = _bf16(_attend_sequence(_f32(q_lat[b]), _f32(q_rope[b]), rows[:, :R], rows[:, R:],
                                        [it for it in items if it[0] == b], scale_log2))
    return out


def _mla_fp8_layer(c, Wq, Wkva, w_norm, Wkvb, Wo, xq, slots, quant=None, layer=0):
    """The attention block of one layer for a teacher-forced sequence, at the
    batched decode's storage points (see the module docstring).  xq [T, D]:
    the layer input as the FP8 GEMM sees it; returns the o_proj output [T, D]."""
    orc = oracle()
    T = xq.shape[0]
    H, R, nope, P, v = (c["num_attention_heads"], c["kv_lora_rank"], c["qk_nope_head_dim"], c["qk_rope_head_dim"],
                        c["v_head_dim"])
    eps, theta = c["rms_norm_eps"], c["rope_theta"]
    q = _f32(xq.astype(np.float64) @ Wq.T.astype(np.float64)).reshape(T, H, nope + P)
    kva = _f32(xq.astype(np.float64) @ Wkva.T.astype(np.float64))
    cache = np.zeros((T, R), np.float32)
    kr = np.zeros((T, P), np.float32)
    q_rope = np.zeros((T, H, P), np.float32)
    for t in range(T):
        row = np.zeros(R, np.float32)
        orc.orc_rmsnorm_f32(p(_f32(kva[t, :R]), f32p), p(w_norm, f32p), R, eps, p(row, f32p))
        cache[t] = row
        r = _f32(kva[t, R:]).copy()
        orc.orc_rope_inplace_f32(p(r, f32p), P, t, theta)
        kr[t] = r
        for h in range(H):
            r = _f32(q[t, h, nope:]).copy()
            orc.orc_rope_inplace_f32(p(r, f32p), P, t, theta)
            q_rope[t, h] = r
    store = (lambda x, tag: _bf16(x)) if quant is None else \
        (lambda x, tag: quant.bf16(x.reshape(T, -1), (tag, layer), list(range(T))).reshape(x.shape))
    cache, kr, q_rope = store(cache, "c"), store(kr, "kr"), store(q_rope, "q_rope")
    q_nope = store(_f32(q[:, :, :nope]), "q_nope")
    wkvb = Wkvb.reshape(H, nope + v, R)
    w_uk, w_uv = wkvb[:, :nope, :].astype(np.float64), wkvb[:, nope:, :].astype(np.float64)  # [H, nope, R], [H, v, R]
    q_lat = store(_f32(np.einsum("thn,hnr->thr", q_nope.astype(np.float64), w_uk)), "q_lat")
    scale = np.float32(1.0) / np.sqrt(np.float32(nope + P), dtype=np.float32)
    scale_log2 = np.float32(scale * np.float32(1.4426950408889634))
    o_lat = np.zeros((T, H, R), np.float32)
    for t in range(T):
        # position t decodes with t + 1 cached tokens, planned as a batch of one sequence
        # the probabilities of a 64-token tile starting at token t0 as one stored row (head-major)
        pstore = None if quant is None else (lambda x, t0, t=t: quant.bf16(x.reshape(1, -1), ("P", layer, t0),
                                                                            [t]).reshape(x.shape))
        o = _attend_sequence(q_lat[t], q_rope[t], cache, kr, _mla_items([t + 1], slots, H, R, P), scale_log2, pstore)
        o_lat[t] = _bf16(o) if quant is None else quant.bf16(o.reshape(1, -1), ("o_lat", layer), [t]).reshape(H, R)
    # the per-head W_UV output before its bf16 rounding (the quantiser rounds it)
    attn = _f32(np.einsum("thr,hvr->thv", o_lat.astype(np.float64), w_uv)).reshape(T, H * v)
    attn_q = _act_fp8(attn) if quant is None else quant(attn, ("o_proj", layer), list(range(T)))
    return _f32(attn_q.astype(np.float64) @ Wo.T.astype(np.float64))


def forward_fp8(cfg: dict, tensors: dict, fp8: dict, seq, slots: int = 148, swaps=(), margins=None, quant=None):
    """Logits [T, V] of `seq` for a block-scaled FP8 checkpoint: `tensors`
    holds every tensor (fp32 values), `fp8` maps the FP8 weights' names to
    their dequantised fp32 matrices (e4m3 * scale).  Softmax-greedy routing
    as forward(), with the same router margins (into the dict `margins`,
    {layer: [T]}, when given) and near-tie `swaps` ((layer, position) pairs
    whose (k+1)-th expert takes the k-th slot).  `slots`: the split-KV
    planner's parallel work slots (the GPU's SM count for kv_lora_rank 128).
    `quant`: an Fp8Quantiser (records the ambiguous roundings, applies
    chosen flips); None quantises plainly."""
    if cfg.get("q_lora_rank", 0) or cfg.get("scoring_func", 0) != 0:
        raise NotImplementedError("oracle.model covers q_lora_rank 0 with softmax scoring")
    c = cfg
    if quant is None:
        quant = Fp8Quantiser(record=False)
    W = {n: _f32(a) for n, a in tensors.items()}
    for n, a in fp8.items():
        W[n] = _bf16_round(a) if n.endswith("kv_b_proj.weight") else _f32(a)
    seq = np.asarray(seq, np.int64)
    T = len(seq)
    D = c["hidden_size"]
    E, k = c["n_routed_experts"], c["num_experts_per_tok"]
    eps = c["rms_norm_eps"]
    swaps = set(swaps)
    orc = oracle()
    h = _f32(W["model.embed_tokens.weight"][seq])
    for li in range(c["num_hidden_layers"]):
        pre = f"model.layers.{li}."
        allpos = list(range(T))
        xn = quant(_rmsnorm_rows(h, W[pre + "input_layernorm.weight"], eps), ("attn_in", li), allpos)
        a = pre + "self_attn."
        out = _mla_fp8_layer(c, W[a + "q_proj.weight"], W[a + "kv_a_proj_with_mqa.weight"],
                             W[a + "kv_a_layernorm.weight"], W[a + "kv_b_proj.weight"], W[a + "o_proj.weight"], xn,
                             slots, quant, li)
        h = _f32(h + out)
        xn = _rmsnorm_rows(h, W[pre + "post_attention_layernorm.weight"], eps)
        xq = quant(xn, ("ffn_in", li), allpos)

        def ffn(wg, wu, wd, x, tag, pos):
            g = _f32(x.astype(np.float64) @ wg.T.astype(np.float64))
            u = _f32(x.astype(np.float64) @ wu.T.astype(np.float64))
            mid = quant(_silu_mul(g, u), tag, pos)
            return _f32(mid.astype(np.float64) @ wd.T.astype(np.float64))

        if pre + "mlp.gate.weight" not in W:
            out = ffn(*(W[pre + "mlp." + n + "_proj.weight"] for n in ("gate", "up", "down")), xq, ("mid", li, -1),
                      allpos)
        else:
            wgate = W[pre + "mlp.gate.weight"]
            shared = pre + "mlp.shared_experts.gate_proj.weight" in W
            out = np.zeros((T, D), np.float32)
            margin = np.zeros(T)
            for t in range(T):
                logits = np.zeros(E, np.float32)
                orc.orc_linear_f32(p(wgate, f32p), p(_f32(xn[t]), f32p), D, p(logits, f32p), E)
                srt = np.sort(logits.astype(np.float64))[::-1]
                margin[t] = srt[k - 1] - srt[k] if k < E else np.inf
                kx = k + 1 if k < E else k
                ids = np.zeros(kx, np.int32)
                w = np.zeros(kx, np.float32)
                # top-(k+1) unnormalised, then the swap and the reference's renormalisation
                assert orc.orc_route_softmax_greedy(p(logits, f32p), 1, E, kx, 0, 1.0, p(ids, i32p),
                                                    p(w, f32p)) == 0
                if (li, t) in swaps:
                    ids[k - 1], w[k - 1] = ids[k], w[k]
                ids, w = np.ascontiguousarray(ids[:k]), _f32(w[:k])
                if c["norm_topk_prob"]:
                    s_ = np.float32(0)
                    for j in range(k):
                        s_ = np.float32(s_ + w[j])
                    if s_ > 0:
                        w = _f32(w / s_)
                w = _f32(w * np.float32(c["routed_scaling_factor"]))
                acc = np.zeros(D, np.float32)
                x = xq[t:t + 1]
                for e, wt in zip(ids, w):
                    y = ffn(*(W[pre + f"mlp.experts.{e}.{n}_proj.weight"] for n in ("gate", "up", "down")), x,
                            ("mid", li, int(e)), [t])
                    acc = _f32(acc + np.float32(wt) * y[0])
                if shared:
                    y = ffn(*(W[pre + f"mlp.shared_experts.{n}_proj.weight"] for n in ("gate", "up", "down")), x,
                            ("mid", li, E), [t])
                    acc = _f32(acc + y[0])
                out[t] = acc
            if margins is not None:
                margins[li] = margin
        h = _f32(h + out)
    hn = _bf16(_rmsnorm_rows(h, W["model.norm.weight"], eps))
    return _f32(hn.astype(np.float64) @ W["lm_head.weight"].T.astype(np.float64))
