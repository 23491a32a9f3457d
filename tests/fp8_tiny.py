"""Block-scaled FP8 versions of the tiny model's checkpoint tensors (test
helper): every projection, dense FFN, routed and shared expert matrix and
kv_b_proj quantised per 128x128 block by the oracle's restatement
(orc_quant_weight_128x128), uploaded as e4m3 bytes plus "<name>_scale_inv"
(scales before the weight for every other tensor, to cover both orders), or
as the dequantised values (e4m3 * scale) for a bf16 comparison model."""

import numpy as np

import oracle as O
import deepseek_cpp_infer_b200 as dsb
from deepseek_cpp_infer_b200.workloads import TINY, model_tensors

FP8_SUFFIXES = ("q_proj.weight", "kv_a_proj_with_mqa.weight", "kv_b_proj.weight", "o_proj.weight",
                "gate_proj.weight", "up_proj.weight", "down_proj.weight")


def quantise(w):
    """fp32 [M, K] -> (e4m3 uint8 [M, K], fp32 scales, dequantised fp32)."""
    w = np.ascontiguousarray(w, np.float32)
    M, K = w.shape
    q = np.zeros((M, K), np.uint8)
    s = np.zeros(((M + 127) // 128, (K + 127) // 128), np.float32)
    O.oracle().orc_quant_weight_128x128(O.p(w, O.f32p), M, K, O.p(q, O.u8p), O.p(s, O.f32p))
    lut = np.array([O.oracle().orc_e4m3_to_f32(c) for c in range(256)], np.float32)
    deq = lut[q] * np.repeat(np.repeat(s, 128, 0)[:M], 128, 1)[:, :K]
    return q, s, deq


def build(ctx, fp8, ep=None):
    tensors = model_tensors(TINY, seed=0)
    m = dsb.Model(ctx, dsb.ModelConfig(**TINY))
    if ep is not None:
        m.set_ep(ep)
    flip = False
    for name, a in tensors.items():
        if name.startswith("model.layers.") and name.endswith(FP8_SUFFIXES) and "mlp.gate." not in name:
            q, s, deq = quantise(O.bf16_to_f32(a) if a.dtype == np.uint16 else a)
            if fp8:
                pair = [(name, q), (name + "_scale_inv", s)]
                flip = not flip  # scales before the weight for every other tensor
                for n2, a2 in (reversed(pair) if flip else pair):
                    m.set_tensor(n2, a2)
            else:
                m.set_tensor(name, deq)
        else:
            m.set_tensor(name, a)
    m.finalize()
    return m


