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


def _silu_mul(g, u):
    return _f32(g / (np.float32(1) + np.exp(-g)) * u)


def forward_fp8(cfg: dict, tensors: dict, fp8: dict, seq):
    """Logits [T, V] of `seq` for a block-scaled FP8 checkpoint: `tensors`
    holds every tensor (fp32 values), `fp8` maps the FP8 weights' names to
    their dequantised fp32 matrices (e4m3 * scale).  Softmax-greedy routing
    as forward(); near-tie swaps are not modelled."""
    if cfg.get("q_lora_rank", 0) or cfg.get("scoring_func", 0) != 0:
        raise NotImplementedError("oracle.model covers q_lora_rank 0 with softmax scoring")
    c = cfg
    W = {n: _f32(a) for n, a in tensors.items()}
    for n, a in fp8.items():
        W[n] = _bf16_round(a) if n.endswith("kv_b_proj.weight") else _f32(a)
    seq = np.asarray(seq, np.int64)
    T = len(seq)
    D, H, R = c["hidden_size"], c["num_attention_heads"], c["kv_lora_rank"]
    nope, rope, v = c["qk_nope_head_dim"], c["qk_rope_head_dim"], c["v_head_dim"]
    E, k = c["n_routed_experts"], c["num_experts_per_tok"]
    eps = c["rms_norm_eps"]
    orc = oracle()
    h = _f32(W["model.embed_tokens.weight"][seq])
    for li in range(c["num_hidden_layers"]):
        pre = f"model.layers.{li}."
        xn = _act_fp8(_rmsnorm_rows(h, W[pre + "input_layernorm.weight"], eps))
        out = np.zeros((T, D), np.float32)
        rc = orc.orc_mla_layer_seq_fp8act_f32(
            D, H, nope, rope, v, R, eps, c["rope_theta"],
            *(p(W[pre + "self_attn." + n + ".weight"], f32p)
              for n in ("q_proj", "kv_a_proj_with_mqa", "kv_a_layernorm", "kv_b_proj", "o_proj")),
            p(xn, f32p), T, p(out, f32p))
        assert rc == 0
        h = _f32(h + out)
        xn = _rmsnorm_rows(h, W[pre + "post_attention_layernorm.weight"], eps)
        xq = _act_fp8(xn)

        def ffn(wg, wu, wd, x):
            mid = _act_fp8(_silu_mul(x @ wg.T, x @ wu.T))
            return _f32(mid @ wd.T)

        if pre + "mlp.gate.weight" not in W:
            out = ffn(*(W[pre + "mlp." + n + "_proj.weight"] for n in ("gate", "up", "down")), xq)
        else:
            wgate = W[pre + "mlp.gate.weight"]
            shared = pre + "mlp.shared_experts.gate_proj.weight" in W
            out = np.zeros((T, D), np.float32)
            for t in range(T):
                logits = np.zeros(E, np.float32)
                orc.orc_linear_f32(p(wgate, f32p), p(_f32(xn[t]), f32p), D, p(logits, f32p), E)
                ids = np.zeros(k, np.int32)
                w = np.zeros(k, np.float32)
                assert orc.orc_route_softmax_greedy(p(logits, f32p), 1, E, k, int(c["norm_topk_prob"]),
                                                    float(c["routed_scaling_factor"]), p(ids, i32p),
                                                    p(w, f32p)) == 0
                acc = np.zeros(D, np.float32)
                x = xq[t:t + 1]
                for e, wt in zip(ids, w):
                    y = ffn(*(W[pre + f"mlp.experts.{e}.{n}_proj.weight"] for n in ("gate", "up", "down")), x)
                    acc = _f32(acc + np.float32(wt) * y[0])
                if shared:
                    y = ffn(*(W[pre + f"mlp.shared_experts.{n}_proj.weight"] for n in ("gate", "up", "down")), x)
                    acc = _f32(acc + y[0])
                out[t] = acc
        h = _f32(h + out)
    hn = _rmsnorm_rows(h, W["model.norm.weight"], eps)
    return _f32(hn @ W["lm_head.weight"].T)
