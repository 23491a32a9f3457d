"""ctypes loader for the CPU oracle (TEST INFRASTRUCTURE ONLY).

liboracle.so is the C restatement in oracle.c; _ref/libds_ref.so is the
reference's own CPU code compiled in place (present only where the reference
sources were available at build time).  Only tests/, __graft_entry__.smoke()
and bench.py's cpu_baseline / reference legs may import this module; the
product library never does.
"""

from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_SO = os.path.join(HERE, "liboracle.so")
REF_SO = os.path.join(HERE, "_ref", "libds_ref.so")

f32p = ctypes.POINTER(ctypes.c_float)
u16p = ctypes.POINTER(ctypes.c_uint16)
u8p = ctypes.POINTER(ctypes.c_uint8)
i32p = ctypes.POINTER(ctypes.c_int32)
i64 = ctypes.c_int64

_oracle = None
_ref = None


def build(with_ref: bool = True) -> None:
    targets = ["oracle"] + (["ref"] if with_ref else [])
    subprocess.run(["make", "-s", "-C", HERE, "-j8", *targets], check=True)


def _proto(lib, name, res, args):
    fn = getattr(lib, name)
    fn.restype = res
    fn.argtypes = args


def oracle() -> ctypes.CDLL:
    global _oracle
    if _oracle is None:
        if not os.path.exists(ORACLE_SO):
            build(with_ref=False)
        l = ctypes.CDLL(ORACLE_SO)
        _proto(l, "orc_dot_f32", ctypes.c_float, [f32p, f32p, i64])
        _proto(l, "orc_rmsnorm_f32", None, [f32p, f32p, i64, ctypes.c_float, f32p])
        _proto(l, "orc_rope_inplace_f32", ctypes.c_int, [f32p, i64, i64, ctypes.c_float])
        _proto(l, "orc_softmax_f32", ctypes.c_int, [f32p, i64])
        _proto(l, "orc_argmax_f32", i64, [f32p, i64])
        _proto(l, "orc_sample", ctypes.c_int32,
               [f32p, i64, ctypes.c_float, ctypes.c_int32, ctypes.c_float, ctypes.c_float,
                ctypes.POINTER(ctypes.c_double), ctypes.POINTER(ctypes.c_double)])
        _proto(l, "orc_linear_f32", None, [f32p, f32p, i64, f32p, i64])
        _proto(l, "orc_bf16_to_f32_n", None, [u16p, i64, f32p])
        _proto(l, "orc_f32_to_bf16_n", None, [f32p, i64, u16p])
        _proto(
            l, "orc_mla_decode_paged", ctypes.c_int,
            [u16p, u16p, u16p, i32p, i32p, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
             ctypes.c_int, ctypes.c_float, f32p],
        )
        _proto(
            l, "orc_mla_layer_seq_f32", ctypes.c_int,
            [ctypes.c_int] * 6 + [ctypes.c_float, ctypes.c_float] + [f32p] * 6 + [ctypes.c_int, f32p],
        )
        _proto(
            l, "orc_mla_layer_seq_fp8act_f32", ctypes.c_int,
            [ctypes.c_int] * 6 + [ctypes.c_float, ctypes.c_float] + [f32p] * 6 + [ctypes.c_int, f32p],
        )
        _proto(l, "orc_act_fp8_roundtrip", None, [f32p, i64, i64])
        _proto(
            l, "orc_kv_norm_rope_append", ctypes.c_int,
            [f32p, f32p, f32p, i32p, i32p] + [ctypes.c_int] * 7 + [ctypes.c_float, ctypes.c_float, u16p, f32p],
        )
        _proto(l, "orc_route_softmax_greedy", ctypes.c_int,
               [f32p, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_float, i32p, f32p])
        _proto(l, "orc_route_sigmoid_grouped", ctypes.c_int,
               [f32p, f32p] + [ctypes.c_int] * 6 + [ctypes.c_float, i32p, f32p])
        _proto(l, "orc_moe_permute", None, [i32p, ctypes.c_int, ctypes.c_int, ctypes.c_int, i32p, i32p, i32p, i32p])
        _proto(l, "orc_e4m3_to_f32", ctypes.c_float, [ctypes.c_uint8])
        _proto(l, "orc_f32_to_e4m3", ctypes.c_uint8, [ctypes.c_float])
        _proto(l, "orc_quant_act_1x128", None, [f32p, i64, i64, u8p, f32p])
        _proto(l, "orc_fp8_linear", None, [u8p, f32p, u8p, f32p, i64, i64, i64, f32p])
        _proto(l, "orc_quant_weight_128x128", None, [f32p, i64, i64, u8p, f32p])
        _proto(l, "orc_dense_mlp_f32", None, [f32p, f32p, f32p, f32p, i64, i64, f32p])
        _proto(l, "orc_moe_softmax_f32", ctypes.c_int, [f32p] * 7 + [ctypes.c_int] * 6 + [ctypes.c_float, f32p, f32p])
        _proto(l, "orc_moe_mix_f32", None,
               [f32p] * 6 + [ctypes.c_int] * 4 + [i32p, f32p, ctypes.c_float, f32p, f32p])
        _oracle = l
    return _oracle


class RefConfig(ctypes.Structure):
    _fields_ = [
        (n, ctypes.c_int)
        for n in (
            "hidden_size", "intermediate_size", "num_hidden_layers", "num_attention_heads", "vocab_size",
            "max_position_embeddings", "n_experts", "n_shared_experts", "moe_top_k", "moe_intermediate_size",
            "q_lora_rank", "kv_lora_rank", "qk_nope_head_dim", "qk_rope_head_dim", "v_head_dim", "norm_topk_prob",
        )
    ] + [("rms_norm_eps", ctypes.c_float), ("rope_theta", ctypes.c_float), ("routed_scaling_factor", ctypes.c_float)]


def ref_available() -> bool:
    return os.path.exists(REF_SO)


def ref() -> ctypes.CDLL:
    """The reference's own CPU implementation (oracle/_ref/libds_ref.so)."""
    global _ref
    if _ref is None:
        l = ctypes.CDLL(REF_SO)
        _proto(l, "ref_dot_f32", ctypes.c_float, [f32p, f32p, ctypes.c_size_t])
        _proto(l, "ref_rmsnorm_f32", None, [f32p, f32p, ctypes.c_size_t, ctypes.c_float, f32p])
        _proto(l, "ref_rope_inplace_f32", ctypes.c_int, [f32p, ctypes.c_size_t, ctypes.c_size_t, ctypes.c_float])
        _proto(l, "ref_softmax_f32", ctypes.c_int, [f32p, ctypes.c_size_t])
        _proto(l, "ref_argmax_f32", i64, [f32p, ctypes.c_size_t])
        _proto(l, "ref_linear_f32", ctypes.c_int, [f32p, f32p, ctypes.c_size_t, f32p, ctypes.c_size_t])
        _proto(l, "ref_mla_seq", ctypes.c_int,
               [ctypes.POINTER(RefConfig), f32p, f32p, f32p, f32p, f32p, f32p, ctypes.c_int, f32p])
        _proto(l, "ref_moe_tokens", ctypes.c_int,
               [ctypes.POINTER(RefConfig)] + [f32p] * 7 + [ctypes.c_int, f32p, ctypes.c_int, f32p])
        _proto(l, "ref_model_create", ctypes.c_void_p,
               [ctypes.POINTER(RefConfig), ctypes.c_int, ctypes.POINTER(ctypes.c_char_p),
                ctypes.POINTER(ctypes.c_int), ctypes.POINTER(ctypes.c_int64), ctypes.POINTER(f32p)])
        _proto(l, "ref_model_destroy", None, [ctypes.c_void_p])
        _proto(l, "ref_model_reset", None, [ctypes.c_void_p])
        _proto(l, "ref_model_step", ctypes.c_int, [ctypes.c_void_p, ctypes.c_int32, f32p, i32p])
        _proto(l, "ref_model_generate", ctypes.c_int, [ctypes.c_void_p, i32p, ctypes.c_int, ctypes.c_int, i32p])
        _proto(l, "ref_checkpoint_summary", ctypes.c_int, [ctypes.c_char_p, ctypes.c_char_p, ctypes.c_int])
        _proto(l, "ref_sampler_draws", ctypes.c_int,
               [f32p, ctypes.c_int, ctypes.c_float, ctypes.c_int, ctypes.c_float, ctypes.c_uint32, ctypes.c_int, i32p])
        _proto(l, "ref_sampler_uniforms", ctypes.c_int, [ctypes.c_uint32, ctypes.c_int, f32p])
        _proto(l, "ref_tokenizer_encode", ctypes.c_int,
               [ctypes.c_char_p, ctypes.c_char_p, ctypes.c_int, i32p, ctypes.c_int, ctypes.c_char_p, ctypes.c_int])
        _proto(l, "ref_tokenizer_decode", ctypes.c_int,
               [ctypes.c_char_p, i32p, ctypes.c_int, ctypes.c_int, ctypes.c_char_p, ctypes.c_int])
        _ref = l
    return _ref


# ------------------------------------------------------------------ helpers


def p(a: np.ndarray, ctype):
    """Pointer to a C-contiguous numpy array."""
    assert a.flags["C_CONTIGUOUS"], "array must be C-contiguous"
    return a.ctypes.data_as(ctype)


def bf16_to_f32(a: np.ndarray) -> np.ndarray:
    return (a.astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16(a: np.ndarray) -> np.ndarray:
    a = np.ascontiguousarray(a, dtype=np.float32)
    out = np.empty(a.shape, dtype=np.uint16)
    oracle().orc_f32_to_bf16_n(p(a, f32p), a.size, p(out, u16p))
    return out


def mla_decode_paged(q_lat, q_rope, cache, block_table, seq_lens, scale):
    """orc_mla_decode_paged on uint16 (bf16) arrays; returns f32 [B, H, R]."""
    B, H, R = q_lat.shape
    P = q_rope.shape[2]
    out = np.zeros((B, H, R), np.float32)
    bt = np.ascontiguousarray(block_table, np.int32)
    lens = np.ascontiguousarray(seq_lens, np.int32)
    rc = oracle().orc_mla_decode_paged(
        p(np.ascontiguousarray(q_lat), u16p), p(np.ascontiguousarray(q_rope), u16p), p(np.ascontiguousarray(cache), u16p),
        p(bt, i32p), p(lens, i32p), B, H, R, P, cache.shape[1], bt.shape[1], float(scale), p(out, f32p),
    )
    assert rc == 0
    return out


def ref_checkpoint_summary(path: str) -> tuple[dict, list[tuple]]:
    """The reference's loader (parse_deepseek_config + load_model_dir) on a
    model directory: (config fields, [(name, dtype enum, nbytes, shape)] in
    name order).  Raises RuntimeError with the reference's message if it threw."""
    buf = ctypes.create_string_buffer(1 << 22)
    n = ref().ref_checkpoint_summary(os.fsencode(path), buf, len(buf))
    text = buf.value.decode()
    if n < 0:
        raise RuntimeError(text)
    cfg, tensors = {}, []
    for line in text.splitlines():
        f = line.split(" ")
        if f[0] == "cfg":
            cfg[f[1]] = f[2]
        elif f[0] == "t":
            tensors.append((f[1], int(f[2]), int(f[3]), tuple(int(x) for x in f[4:])))
    return cfg, tensors


def sample(logits, temperature, top_k, top_p, r) -> tuple[int, float, float]:
    """orc_sample on one fp32 row: (id, margin of r in the chosen interval, margin of the top-p cut)."""
    x = np.ascontiguousarray(logits, np.float32)
    m, c = ctypes.c_double(), ctypes.c_double()
    i = oracle().orc_sample(p(x, f32p), x.size, temperature, top_k, top_p, r, ctypes.byref(m), ctypes.byref(c))
    return int(i), m.value, c.value


def ref_sampler(logits, temperature, top_k, top_p, seed, n) -> tuple[np.ndarray, np.ndarray]:
    """The reference's Sampler with `seed`: (n sampled ids, the n uniform draws it made)."""
    x = np.ascontiguousarray(logits, np.float32)
    ids = np.zeros(n, np.int32)
    u = np.zeros(n, np.float32)
    assert ref().ref_sampler_draws(p(x, f32p), x.size, temperature, top_k, top_p, seed, n, p(ids, i32p)) == 0
    ref().ref_sampler_uniforms(seed, n, p(u, f32p))
    return ids, u


def ref_tokenize(path: str, data: bytes):
    """The reference's Tokenizer::encode on `data`: the id list, or the error message (str)."""
    cap = len(data) + 1
    ids = np.zeros(cap, np.int32)
    msg = ctypes.create_string_buffer(512)
    n = ref().ref_tokenizer_encode(os.fsencode(path), data, len(data), p(ids, i32p), cap, msg, len(msg))
    return msg.value.decode() if n < 0 else ids[:n].tolist()


def ref_detokenize(path: str, ids, skip_special: bool = True):
    """The reference's Tokenizer::decode: bytes, or None if it threw."""
    a = np.ascontiguousarray(np.asarray(ids, np.int32).reshape(-1))
    if a.size == 0:
        a = np.zeros(1, np.int32)
        n_ids = 0
    else:
        n_ids = a.size
    cap = 1 << 20
    out = ctypes.create_string_buffer(cap)
    n = ref().ref_tokenizer_decode(os.fsencode(path), p(a, i32p), n_ids, int(skip_special), out, cap)
    return None if n < 0 else out.raw[:n]
