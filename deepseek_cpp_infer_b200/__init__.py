"""Python view of libdsb.so, the B200 decode hot path of deepseek_cpp_infer.

The product is the C ABI declared in include/dsb/dsb.h; this module only binds
it with ctypes so that tests and bench.py can drive it with device buffers
(torch tensors are used for allocation; only raw pointers cross the ABI).
There is no CPU fallback: if libdsb.so is missing, importing the bindings
raises.
"""

from __future__ import annotations

import ctypes
import os
import re

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libdsb.so")
HEADER_PATH = os.path.join(os.path.dirname(_HERE), "include", "dsb", "dsb.h")

DSB_OK = 0
DSB_EINVAL = 1
DSB_ECUDA = 2
DSB_ENOMEM = 3
DSB_ETIMEOUT = 4
DSB_EUNSUPPORTED = 5
DSB_ELIMIT = 6

_c_i32p = ctypes.POINTER(ctypes.c_int32)
_vp, _i64, _ci, _cf = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, ctypes.c_float
SCORE_SOFTMAX, SCORE_SIGMOID = 0, 1


class DsbError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"dsb error {code}: {msg}")
        self.code = code


class Stats(ctypes.Structure):
    _fields_ = [
        ("kernel_launches", ctypes.c_uint64),
        ("mla_calls", ctypes.c_uint64),
        ("mla_work_items", ctypes.c_uint64),
        ("mla_partials", ctypes.c_uint64),
        ("workspace_bytes", ctypes.c_uint64),
        ("gemm_calls", ctypes.c_uint64),
        ("decode_steps", ctypes.c_uint64),
        ("prefill_tokens", ctypes.c_uint64),
    ]


EPI_STORE, EPI_ADD, EPI_SILU_GATE, EPI_ROWSCALE = 0, 1, 2, 3


class LinearArgs(ctypes.Structure):
    _fields_ = [
        ("w", ctypes.c_void_p), ("ldw", ctypes.c_int64), ("x", ctypes.c_void_p), ("ldx", ctypes.c_int64),
        ("x_group_col", ctypes.c_int64), ("tok_offsets", ctypes.c_void_p),
        ("T", ctypes.c_int), ("M", ctypes.c_int), ("K", ctypes.c_int), ("G", ctypes.c_int),
        ("max_tokens_per_group", ctypes.c_int), ("y", ctypes.c_void_p), ("ldy", ctypes.c_int64),
        ("y_group_col", ctypes.c_int64), ("y_f32", ctypes.c_int), ("epilogue", ctypes.c_int),
        ("row_scale", ctypes.c_void_p),
    ]


class LinearFp8Args(ctypes.Structure):
    _fields_ = [
        ("w", ctypes.c_void_p), ("ldw", ctypes.c_int64), ("w_scale", ctypes.c_void_p), ("scale_rows", ctypes.c_int),
        ("x", ctypes.c_void_p), ("ldx", ctypes.c_int64), ("x_scale", ctypes.c_void_p), ("ld_xs", ctypes.c_int64),
        ("x_group_col", ctypes.c_int64), ("tok_offsets", ctypes.c_void_p),
        ("T", ctypes.c_int), ("M", ctypes.c_int), ("K", ctypes.c_int), ("G", ctypes.c_int),
        ("max_tokens_per_group", ctypes.c_int), ("y", ctypes.c_void_p), ("ldy", ctypes.c_int64),
        ("y_group_col", ctypes.c_int64), ("y_f32", ctypes.c_int), ("epilogue", ctypes.c_int),
        ("row_scale", ctypes.c_void_p),
    ]


class MoeFp8Layer(ctypes.Structure):
    _fields_ = [
        ("gate_up", ctypes.c_void_p), ("gate_up_scale", ctypes.c_void_p), ("down", ctypes.c_void_p),
        ("down_scale", ctypes.c_void_p), ("E", ctypes.c_int), ("n_shared", ctypes.c_int), ("D", ctypes.c_int),
        ("I", ctypes.c_int),
    ]


DTYPE_F32, DTYPE_BF16, DTYPE_F16, DTYPE_F8E4M3 = 0, 1, 2, 3
STREAM_LEGACY = 1  # cudaStreamLegacy: the legacy default stream as a stream handle


class ModelConfig(ctypes.Structure):
    """dsb_model_config (the decode-path fields of ds::hf::DeepSeekConfig)."""

    _fields_ = [
        (n, ctypes.c_int)
        for n in (
            "hidden_size", "num_hidden_layers", "num_attention_heads", "vocab_size", "max_position_embeddings",
            "intermediate_size", "moe_intermediate_size", "n_routed_experts", "n_shared_experts",
            "num_experts_per_tok", "first_k_dense_replace", "q_lora_rank", "kv_lora_rank", "qk_nope_head_dim",
            "qk_rope_head_dim", "v_head_dim", "scoring_func", "n_group", "topk_group", "norm_topk_prob",
        )
    ] + [("routed_scaling_factor", ctypes.c_float), ("rms_norm_eps", ctypes.c_float), ("rope_theta", ctypes.c_float),
         ("weights_fp8", ctypes.c_int)]


class Sampling(ctypes.Structure):
    """dsb_sampling (ds::core::SamplerConfig)."""

    _fields_ = [("temperature", ctypes.c_float), ("top_k", ctypes.c_int), ("top_p", ctypes.c_float),
                ("seed", ctypes.c_uint32)]


DTYPE_OTHER = -1
CKPT_MAX_DIMS = 8


class TensorInfo(ctypes.Structure):
    """dsb_tensor_info: one tensor of an opened checkpoint."""

    _fields_ = [("name", ctypes.c_char_p), ("dtype_name", ctypes.c_char_p), ("dtype", ctypes.c_int),
                ("ndim", ctypes.c_int), ("shape", ctypes.c_int64 * CKPT_MAX_DIMS), ("data", ctypes.c_void_p),
                ("nbytes", ctypes.c_uint64)]


# (name, restype, argtypes) for every function of include/dsb/dsb.h
_PROTOS = [
    ("dsb_decode_step_sampled", ctypes.c_int,
     [_vp, _vp, _vp, _c_i32p, _c_i32p, _ci, ctypes.POINTER(Sampling), ctypes.POINTER(ctypes.c_float), _vp, _c_i32p]),
    ("dsb_generate_sampled", ctypes.c_int,
     [_vp, _vp, _vp, _vp, _ci, _vp, _vp, _ci, ctypes.c_int32, ctypes.POINTER(Sampling), _vp, _vp]),
    ("dsb_tokenizer_load", ctypes.c_int, [ctypes.c_char_p, ctypes.POINTER(ctypes.c_void_p)]),
    ("dsb_tokenizer_destroy", ctypes.c_int, [_vp]),
    ("dsb_tokenizer_error", ctypes.c_char_p, []),
    ("dsb_tokenizer_info", ctypes.c_int,
     [_vp, ctypes.POINTER(_ci), ctypes.POINTER(ctypes.c_int32), ctypes.POINTER(ctypes.c_int32),
      ctypes.POINTER(ctypes.c_int32)]),
    ("dsb_tokenizer_encode", ctypes.c_int,
     [_vp, ctypes.c_char_p, ctypes.c_size_t, _c_i32p, ctypes.c_size_t, ctypes.POINTER(ctypes.c_size_t)]),
    ("dsb_tokenizer_decode", ctypes.c_int,
     [_vp, _c_i32p, ctypes.c_size_t, _ci, ctypes.c_char_p, ctypes.c_size_t, ctypes.POINTER(ctypes.c_size_t)]),
    ("dsb_checkpoint_open", ctypes.c_int, [ctypes.c_char_p, ctypes.POINTER(ctypes.c_void_p)]),
    ("dsb_checkpoint_close", ctypes.c_int, [ctypes.c_void_p]),
    ("dsb_checkpoint_error", ctypes.c_char_p, []),
    ("dsb_checkpoint_config", ctypes.c_int, [ctypes.c_void_p, ctypes.POINTER(ModelConfig)]),
    ("dsb_checkpoint_num_tensors", ctypes.c_int, [ctypes.c_void_p, ctypes.POINTER(ctypes.c_int)]),
    ("dsb_checkpoint_tensor", ctypes.c_int, [ctypes.c_void_p, ctypes.c_int, ctypes.POINTER(TensorInfo)]),
    ("dsb_checkpoint_find", ctypes.c_int, [ctypes.c_void_p, ctypes.c_char_p, ctypes.POINTER(ctypes.c_int)]),
    ("dsb_model_upload_checkpoint", ctypes.c_int,
     [ctypes.c_void_p, ctypes.c_void_p, ctypes.POINTER(ctypes.c_int), ctypes.POINTER(ctypes.c_int)]),
    ("dsb_version", ctypes.c_int, []),
    ("dsb_ctx_create", ctypes.c_int, [ctypes.c_int, ctypes.POINTER(ctypes.c_void_p)]),
    ("dsb_ctx_destroy", ctypes.c_int, [ctypes.c_void_p]),
    ("dsb_ctx_set_stream", ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p]),
    ("dsb_ctx_stream", ctypes.c_void_p, [ctypes.c_void_p]),
    ("dsb_last_error", ctypes.c_char_p, [ctypes.c_void_p]),
    ("dsb_sync", ctypes.c_int, [ctypes.c_void_p]),
    ("dsb_get_stats", ctypes.c_int, [ctypes.c_void_p, ctypes.POINTER(Stats)]),
    ("dsb_reset_stats", ctypes.c_int, [ctypes.c_void_p]),
    ("dsb_mla_plan_create", ctypes.c_int,
     [ctypes.c_void_p, _c_i32p, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
      ctypes.POINTER(ctypes.c_void_p)]),
    ("dsb_mla_plan_destroy", ctypes.c_int, [ctypes.c_void_p]),
    ("dsb_mla_plan_info", ctypes.c_int, [ctypes.c_void_p, ctypes.POINTER(ctypes.c_int), ctypes.POINTER(ctypes.c_int)]),
    ("dsb_mla_decode_planned", ctypes.c_int,
     [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64,
      ctypes.c_void_p, ctypes.c_int, ctypes.c_float, ctypes.c_void_p]),
    ("dsb_linear", ctypes.c_int, [ctypes.c_void_p, ctypes.POINTER(LinearArgs)]),
    ("dsb_quant_act_1x128", ctypes.c_int, [_vp, _vp, _ci, _i64, _vp, _ci, _ci, _ci, _vp, _i64, _vp, _i64]),
    ("dsb_quant_weight_128x128", ctypes.c_int, [_vp, _vp, _ci, _i64, _i64, _vp, _vp]),
    ("dsb_linear_fp8", ctypes.c_int, [ctypes.c_void_p, ctypes.POINTER(LinearFp8Args)]),
    ("dsb_ep_create", ctypes.c_int, [_vp, _ci, _ci, _ci, _ci, _ci, _ci, ctypes.POINTER(ctypes.c_void_p)]),
    ("dsb_ep_window_handle", ctypes.c_int, [_vp, _vp]),
    ("dsb_ep_connect", ctypes.c_int, [_vp, _vp]),
    ("dsb_ep_info", ctypes.c_int, [_vp, ctypes.POINTER(_ci), ctypes.POINTER(_ci), ctypes.POINTER(ctypes.c_uint64)]),
    ("dsb_ep_dispatch", ctypes.c_int,
     [_vp, _vp, _i64, _ci, _vp, ctypes.POINTER(ctypes.c_void_p), ctypes.POINTER(ctypes.c_void_p)]),
    ("dsb_ep_combine", ctypes.c_int, [_vp, _vp, _i64, _ci, _vp, _vp, _ci, _vp]),
    ("dsb_ep_destroy", ctypes.c_int, [_vp]),
    ("dsb_model_set_ep", ctypes.c_int, [_vp, _vp]),
    ("dsb_kvcache_fill_random", ctypes.c_int, [_vp, _ci, _ci, ctypes.c_uint64, ctypes.c_float]),
    ("dsb_generate", ctypes.c_int, [_vp, _vp, _vp, _vp, _ci, _vp, _vp, _ci, ctypes.c_int32, _vp, _vp]),
    ("dsb_moe_ffn_fp8", ctypes.c_int,
     [ctypes.c_void_p, ctypes.POINTER(MoeFp8Layer), _vp, _i64, _ci, _ci, _vp, _vp, _vp]),
    ("dsb_rmsnorm", ctypes.c_int, [_vp, _vp, _i64, _vp, _ci, _ci, _cf, _vp, _i64, _vp, _i64]),
    ("dsb_kv_norm_rope_append", ctypes.c_int,
     [_vp, _vp, _vp, _vp, _vp, _vp, _ci, _ci, _ci, _ci, _ci, _ci, _cf, _cf, _vp, _vp]),
    ("dsb_router_logits", ctypes.c_int, [_vp, _vp, _vp, _ci, _ci, _ci, _vp]),
    ("dsb_moe_route", ctypes.c_int, [_vp, _vp, _vp, _ci, _ci, _ci, _ci, _ci, _ci, _ci, _cf, _vp, _vp]),
    ("dsb_moe_permute", ctypes.c_int, [_vp, _vp, _ci, _ci, _ci, _vp, _vp, _vp, _vp, _vp, _vp]),
    ("dsb_gather_rows", ctypes.c_int, [_vp, _vp, _i64, _vp, _ci, _ci, _ci, _vp]),
    ("dsb_moe_combine", ctypes.c_int, [_vp, _vp, _vp, _ci, _ci, _ci, _vp, _vp]),
    ("dsb_argmax", ctypes.c_int, [_vp, _vp, _i64, _ci, _ci, _vp]),
    ("dsb_sample", ctypes.c_int, [_vp, _vp, _i64, _ci, _ci, _cf, _ci, _cf, _vp, _vp]),
    ("dsb_embed", ctypes.c_int, [_vp, _vp, _ci, _vp, _ci, _ci, _vp]),
    ("dsb_model_create", ctypes.c_int, [_vp, ctypes.POINTER(ModelConfig), ctypes.POINTER(ctypes.c_void_p)]),
    ("dsb_model_destroy", ctypes.c_int, [_vp]),
    ("dsb_model_set_tensor", ctypes.c_int, [_vp, ctypes.c_char_p, _ci, ctypes.POINTER(ctypes.c_int64), _ci, _vp]),
    ("dsb_model_init_random", ctypes.c_int, [_vp, ctypes.c_uint64, _cf]),
    ("dsb_model_finalize", ctypes.c_int, [_vp]),
    ("dsb_model_weight_bytes", ctypes.c_int, [_vp, ctypes.POINTER(ctypes.c_uint64)]),
    ("dsb_kvcache_create", ctypes.c_int, [_vp, _vp, _i64, _ci, _ci, ctypes.POINTER(ctypes.c_void_p)]),
    ("dsb_kvcache_destroy", ctypes.c_int, [_vp]),
    ("dsb_kvcache_alloc_seq", ctypes.c_int, [_vp, ctypes.POINTER(ctypes.c_int)]),
    ("dsb_kvcache_free_seq", ctypes.c_int, [_vp, _ci]),
    ("dsb_kvcache_reset", ctypes.c_int, [_vp]),
    ("dsb_kvcache_seq_len", ctypes.c_int, [_vp, _ci, ctypes.POINTER(ctypes.c_int)]),
    ("dsb_kvcache_free_blocks", ctypes.c_int, [_vp, ctypes.POINTER(ctypes.c_int64)]),
    ("dsb_decode_step", ctypes.c_int, [_vp, _vp, _vp, _c_i32p, _c_i32p, _ci, _vp, _c_i32p]),
    ("dsb_prefill", ctypes.c_int, [_vp, _vp, _vp, _c_i32p, _c_i32p, _ci, _vp, _c_i32p, ctypes.POINTER(ctypes.c_int)]),
    ("dsb_mla_decode_noalloc", ctypes.c_int,
     [_vp, _vp, _vp, _vp, _i64, _ci, _vp, _ci, _c_i32p, _ci, _ci, _ci, _ci, _cf, _vp]),
    ("dsb_mla_noalloc_status", ctypes.c_int, [_vp]),
    ("dsb_ctx_set_wait_limit", ctypes.c_int, [_vp, ctypes.c_uint64]),
    ("dsb_ep_window_ptr", ctypes.c_int, [_vp, ctypes.POINTER(ctypes.c_void_p)]),
    ("dsb_ep_connect_local", ctypes.c_int, [_vp, ctypes.POINTER(ctypes.c_void_p)]),
    (
        "dsb_mla_decode",
        ctypes.c_int,
        [
            ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64, ctypes.c_int,
            ctypes.c_void_p, ctypes.c_int, _c_i32p, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
            ctypes.c_float, ctypes.c_void_p,
        ],
    ),
]

_lib = None


def lib() -> ctypes.CDLL:
    """Load libdsb.so (built in-tree by `make -C deepseek_cpp_infer_b200`)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(f"{LIB_PATH} is missing: build it with `make -C {_HERE}` (no CPU fallback exists)")
        l = ctypes.CDLL(LIB_PATH)
        for name, res, args in _PROTOS:
            fn = getattr(l, name)
            fn.restype = res
            fn.argtypes = args
        _lib = l
    return _lib


def header_functions() -> list[str]:
    """Names of the functions declared in include/dsb/dsb.h."""
    with open(HEADER_PATH) as f:
        text = f.read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(dsb_\w+)\s*\(", text)))


def _ptr(t) -> int:
    return 0 if t is None else int(t.data_ptr())


class Context:
    """One dsb_ctx: a device, a stream, a workspace and counters."""

    def __init__(self, device: int = 0):
        self._l = lib()
        h = ctypes.c_void_p()
        rc = self._l.dsb_ctx_create(device, ctypes.byref(h))
        if rc != DSB_OK:
            raise DsbError(rc, f"dsb_ctx_create({device}) failed")
        self.h = h
        self.device = device

    def close(self):
        if self.h:
            self._l.dsb_ctx_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def _check(self, rc: int):
        if rc != DSB_OK:
            raise DsbError(rc, self._l.dsb_last_error(self.h).decode())

    def set_stream(self, stream_handle: int | None):
        self._check(self._l.dsb_ctx_set_stream(self.h, stream_handle or None))

    def use_legacy_stream(self):
        """Run on CUDA's legacy default stream (torch's default stream), so
        the context's kernels are ordered after the torch operations that
        produced their inputs and before those that read their outputs."""
        self.set_stream(STREAM_LEGACY)

    @property
    def stream(self) -> int:
        return self._l.dsb_ctx_stream(self.h) or 0

    def sync(self):
        self._check(self._l.dsb_sync(self.h))

    def set_wait_limit(self, limit_ns: int):
        """Bound of the expert-parallel flag waits launched from now on (dsb_ctx_set_wait_limit)."""
        self._check(self._l.dsb_ctx_set_wait_limit(self.h, int(limit_ns)))

    def stats(self) -> dict:
        s = Stats()
        self._check(self._l.dsb_get_stats(self.h, ctypes.byref(s)))
        return {k: getattr(s, k) for k, _ in Stats._fields_}

    def reset_stats(self):
        self._check(self._l.dsb_reset_stats(self.h))

    def mla_plan(self, seq_lens, H, R, P, block_size=64):
        """dsb_mla_plan_create: a reusable split-KV plan for these lengths."""
        B = len(seq_lens)
        lens = (ctypes.c_int32 * B)(*[int(x) for x in seq_lens])
        h = ctypes.c_void_p()
        self._check(self._l.dsb_mla_plan_create(self.h, lens, B, H, R, P, block_size, ctypes.byref(h)))
        return MlaPlan(self, h, [int(x) for x in seq_lens])

    def mla_decode_planned(self, plan, q_lat, q_rope, kv_cache, block_table, softmax_scale, out):
        self._check(
            self._l.dsb_mla_decode_planned(
                self.h, plan.h, _ptr(q_lat), _ptr(q_rope), _ptr(kv_cache), kv_cache.shape[0], _ptr(block_table),
                block_table.shape[1], float(softmax_scale), _ptr(out),
            )
        )

    def linear(self, w, x, y, *, M, K, G=1, T=None, ldw=None, ldx=None, x_group_col=0, tok_offsets=None,
               max_tokens_per_group=0, ldy=None, y_group_col=0, epilogue=EPI_STORE, row_scale=None):
        """dsb_linear on torch device tensors (w, x bf16; y bf16 or fp32)."""
        import torch

        T = x.shape[0] if T is None else T
        a = LinearArgs(
            w=_ptr(w), ldw=ldw or w.shape[-1], x=_ptr(x), ldx=ldx or x.shape[-1], x_group_col=x_group_col,
            tok_offsets=_ptr(tok_offsets), T=T, M=M, K=K, G=G, max_tokens_per_group=max_tokens_per_group,
            y=_ptr(y), ldy=ldy or y.shape[-1], y_group_col=y_group_col, y_f32=int(y.dtype == torch.float32),
            epilogue=epilogue, row_scale=_ptr(row_scale),
        )
        self._check(self._l.dsb_linear(self.h, ctypes.byref(a)))

    def quant_act(self, x, q, scales, src_rows=None, k=1, T=None):
        """dsb_quant_act_1x128: x bf16/fp32 [.., K] -> q uint8 [T, K], scales fp32 [T, K/128]."""
        import torch

        T = (src_rows.shape[0] if src_rows is not None else x.shape[0]) if T is None else T
        dt = DTYPE_BF16 if x.dtype == torch.bfloat16 else DTYPE_F32
        self._check(self._l.dsb_quant_act_1x128(self.h, _ptr(x), dt, x.stride(0), _ptr(src_rows), k, T, q.shape[1],
                                                _ptr(q), q.stride(0), _ptr(scales), scales.stride(0)))

    def quant_weight(self, w, q, scales):
        """dsb_quant_weight_128x128: w bf16/fp32 [M, K] -> q uint8 [M, K], scales [ceil(M/128), ceil(K/128)]."""
        import torch

        dt = DTYPE_BF16 if w.dtype == torch.bfloat16 else DTYPE_F32
        self._check(self._l.dsb_quant_weight_128x128(self.h, _ptr(w), dt, w.shape[0], w.shape[1], _ptr(q),
                                                     _ptr(scales)))

    def linear_fp8(self, w, w_scale, x, x_scale, y, *, M, K, G=1, T=None, scale_rows=1, ldw=None, ldx=None,
                   x_group_col=0, tok_offsets=None, max_tokens_per_group=0, ldy=None, y_group_col=0,
                   epilogue=EPI_STORE, row_scale=None):
        """dsb_linear_fp8 on torch device tensors (w, x uint8 e4m3; scales fp32; y bf16 or fp32)."""
        import torch

        T = x.shape[0] if T is None else T
        a = LinearFp8Args(
            w=_ptr(w), ldw=ldw or w.shape[-1], w_scale=_ptr(w_scale), scale_rows=scale_rows, x=_ptr(x),
            ldx=ldx or x.shape[-1], x_scale=_ptr(x_scale), ld_xs=x_scale.stride(0), x_group_col=x_group_col,
            tok_offsets=_ptr(tok_offsets), T=T, M=M, K=K, G=G, max_tokens_per_group=max_tokens_per_group,
            y=_ptr(y), ldy=ldy or y.shape[-1], y_group_col=y_group_col, y_f32=int(y.dtype == torch.float32),
            epilogue=epilogue, row_scale=_ptr(row_scale),
        )
        self._check(self._l.dsb_linear_fp8(self.h, ctypes.byref(a)))

    def moe_ffn_fp8(self, gate_up, gate_up_scale, down, down_scale, *, E, n_shared, x, ids, weights, h):
        """dsb_moe_ffn_fp8: h[T, D] += experts(x[T, D] bf16) for picks ids/weights [T, k]."""
        T, D = x.shape
        I = down.shape[-1]
        layer = MoeFp8Layer(gate_up=_ptr(gate_up), gate_up_scale=_ptr(gate_up_scale), down=_ptr(down),
                            down_scale=_ptr(down_scale), E=E, n_shared=n_shared, D=D, I=I)
        self._check(self._l.dsb_moe_ffn_fp8(self.h, ctypes.byref(layer), _ptr(x), x.stride(0), T, ids.shape[1],
                                            _ptr(ids), _ptr(weights), _ptr(h)))

    # ---- row and routing ops (device tensors; shapes from the tensors)
    def rmsnorm(self, x, w, eps, y_bf16=None, y_f32=None):
        rows, n = x.shape
        self._check(self._l.dsb_rmsnorm(self.h, _ptr(x), x.stride(0), _ptr(w), rows, n, float(eps), _ptr(y_bf16),
                                        y_bf16.stride(0) if y_bf16 is not None else 0, _ptr(y_f32),
                                        y_f32.stride(0) if y_f32 is not None else 0))

    def kv_norm_rope_append(self, kv_a, w_norm, q, positions, block_table, H, nope, R, P, eps, theta, cache, q_rope):
        B = kv_a.shape[0]
        self._check(self._l.dsb_kv_norm_rope_append(
            self.h, _ptr(kv_a), _ptr(w_norm), _ptr(q), _ptr(positions), _ptr(block_table), block_table.shape[1], B,
            H, nope, R, P, float(eps), float(theta), _ptr(cache), _ptr(q_rope)))

    def router_logits(self, x, w_gate, logits):
        T, D = x.shape
        self._check(self._l.dsb_router_logits(self.h, _ptr(x), _ptr(w_gate), T, D, w_gate.shape[0], _ptr(logits)))

    def moe_route(self, logits, ids, weights, k, scoring=SCORE_SOFTMAX, bias=None, n_group=1, topk_group=1,
                  norm_topk=0, routed_scale=1.0):
        T, E = logits.shape
        self._check(self._l.dsb_moe_route(self.h, _ptr(logits), _ptr(bias), T, E, k, scoring, n_group, topk_group,
                                          int(norm_topk), float(routed_scale), _ptr(ids), _ptr(weights)))

    def moe_permute(self, ids, E, counts, offsets, dest, src_pair, weights=None, w_perm=None):
        T, k = ids.shape
        self._check(self._l.dsb_moe_permute(self.h, _ptr(ids), T, k, E, _ptr(counts), _ptr(offsets), _ptr(dest),
                                            _ptr(src_pair), _ptr(weights), _ptr(w_perm)))

    def gather_rows(self, x, src_pair, k, out):
        n, D = out.shape
        self._check(self._l.dsb_gather_rows(self.h, _ptr(x), x.stride(0), _ptr(src_pair), n, k, D, _ptr(out)))

    def moe_combine(self, y, dest, k, h, shared=None):
        T, D = h.shape
        self._check(self._l.dsb_moe_combine(self.h, _ptr(y), _ptr(dest), T, k, D, _ptr(shared), _ptr(h)))

    def argmax(self, logits, out):
        B, V = logits.shape
        self._check(self._l.dsb_argmax(self.h, _ptr(logits), logits.stride(0), B, V, _ptr(out)))

    def sample(self, logits, uniforms, out, temperature=1.0, top_k=0, top_p=0.0):
        """Sampled id per row of logits [B, V] (fp32) with one uniform draw per row."""
        B, V = logits.shape
        self._check(self._l.dsb_sample(self.h, _ptr(logits), logits.stride(0), B, V, temperature, top_k, top_p,
                                       _ptr(uniforms), _ptr(out)))

    def embed(self, table, tokens, h):
        import torch

        self._check(self._l.dsb_embed(self.h, _ptr(table), int(table.dtype == torch.bfloat16), _ptr(tokens),
                                      tokens.shape[0], table.shape[1], _ptr(h)))

    def mla_decode(self, q_lat, q_rope, kv_cache, block_table, seq_lens, softmax_scale, out, block_size=64):
        """Absorbed MLA decode (dsb_mla_decode).  q_lat [B,H,R], q_rope [B,H,P],
        kv_cache [n_blocks, 64, R+P] bf16 on the device; block_table int32
        device [B, max_blocks]; seq_lens a host sequence of ints; out [B,H,R] bf16."""
        B, H, R = q_lat.shape
        P = q_rope.shape[2]
        n_blocks = kv_cache.shape[0]
        lens = (ctypes.c_int32 * B)(*[int(x) for x in seq_lens])
        self._check(
            self._l.dsb_mla_decode(
                self.h, _ptr(q_lat), _ptr(q_rope), _ptr(kv_cache), n_blocks, block_size, _ptr(block_table),
                block_table.shape[1], lens, B, H, R, P, float(softmax_scale), _ptr(out),
            )
        )


def mla_decode_noalloc(stream_handle, q_lat, q_rope, kv_cache, block_table, seq_lens, softmax_scale, out,
                       block_size=64) -> int:
    """dsb_mla_decode_noalloc on torch device tensors; returns the status code."""
    B, H, R = q_lat.shape
    P = q_rope.shape[2]
    lens = (ctypes.c_int32 * B)(*[int(x) for x in seq_lens])
    return lib().dsb_mla_decode_noalloc(
        stream_handle or None, _ptr(q_lat), _ptr(q_rope), _ptr(kv_cache), kv_cache.shape[0], block_size,
        _ptr(block_table), block_table.shape[1], lens, B, H, R, P, float(softmax_scale), _ptr(out))


def mla_noalloc_status(stream_handle) -> int:
    """dsb_mla_noalloc_status: waits for the stream, returns the last allocation-free call's status code."""
    return lib().dsb_mla_noalloc_status(stream_handle or None)


class MlaPlan:
    """A dsb_mla_plan (released with close() or on garbage collection)."""

    def __init__(self, ctx: Context, h, seq_lens):
        self.ctx = ctx
        self.h = h
        self.seq_lens = seq_lens

    def info(self):
        n_items, n_part = ctypes.c_int(), ctypes.c_int()
        self.ctx._check(self.ctx._l.dsb_mla_plan_info(self.h, ctypes.byref(n_items), ctypes.byref(n_part)))
        return {"n_items": n_items.value, "n_partial": n_part.value}

    def close(self):
        if self.h:
            self.ctx._l.dsb_mla_plan_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class Model:
    """A dsb_model: device weights uploaded by checkpoint tensor name."""

    def __init__(self, ctx: Context, cfg: ModelConfig):
        self.ctx = ctx
        self.cfg = cfg
        h = ctypes.c_void_p()
        ctx._check(ctx._l.dsb_model_create(ctx.h, ctypes.byref(cfg), ctypes.byref(h)))
        self.h = h

    def set_tensor(self, name: str, array):
        """Upload a host numpy array (float32, uint16 holding bf16 bits, or uint8 holding e4m3 bytes)."""
        import numpy as np

        a = np.ascontiguousarray(array)
        dt = DTYPE_BF16 if a.dtype == np.uint16 else DTYPE_F8E4M3 if a.dtype == np.uint8 else DTYPE_F32
        if dt == DTYPE_F32:
            a = a.astype(np.float32, copy=False)
        shape = (ctypes.c_int64 * a.ndim)(*a.shape)
        self.ctx._check(self.ctx._l.dsb_model_set_tensor(self.h, name.encode(), dt, shape, a.ndim, a.ctypes.data))

    def upload_checkpoint(self, ck: "Checkpoint") -> tuple[int, int]:
        """Upload every decode-path tensor of an opened checkpoint; returns
        (tensors uploaded, tensors skipped)."""
        up, skip = ctypes.c_int(), ctypes.c_int()
        self.ctx._check(self.ctx._l.dsb_model_upload_checkpoint(self.h, ck.h, ctypes.byref(up), ctypes.byref(skip)))
        return up.value, skip.value

    def set_ep(self, ep: "EP"):
        """Keep only the routed experts of `ep`'s rank; MoE layers exchange through the group."""
        self.ctx._check(self.ctx._l.dsb_model_set_ep(self.h, ep.h))

    def init_random(self, seed: int, stddev: float = 0.02):
        self.ctx._check(self.ctx._l.dsb_model_init_random(self.h, seed, stddev))

    def finalize(self):
        self.ctx._check(self.ctx._l.dsb_model_finalize(self.h))

    def weight_bytes(self) -> int:
        n = ctypes.c_uint64()
        self.ctx._check(self.ctx._l.dsb_model_weight_bytes(self.h, ctypes.byref(n)))
        return n.value

    def close(self):
        if self.h:
            self.ctx._l.dsb_model_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class Checkpoint:
    """A Hugging Face model directory opened on the host (dsb_checkpoint):
    config.json plus safetensors shards, memory-mapped.  Needs no GPU."""

    def __init__(self, path: str):
        self._l = lib()
        h = ctypes.c_void_p()
        rc = self._l.dsb_checkpoint_open(os.fsencode(path), ctypes.byref(h))
        if rc != DSB_OK:
            raise DsbError(rc, self._l.dsb_checkpoint_error().decode())
        self.h = h

    def _check(self, rc: int):
        if rc != DSB_OK:
            raise DsbError(rc, self._l.dsb_checkpoint_error().decode())

    def config(self) -> ModelConfig:
        c = ModelConfig()
        self._check(self._l.dsb_checkpoint_config(self.h, ctypes.byref(c)))
        return c

    def __len__(self) -> int:
        n = ctypes.c_int()
        self._check(self._l.dsb_checkpoint_num_tensors(self.h, ctypes.byref(n)))
        return n.value

    def info(self, i: int) -> dict:
        t = TensorInfo()
        self._check(self._l.dsb_checkpoint_tensor(self.h, i, ctypes.byref(t)))
        return {"name": t.name.decode(), "dtype": t.dtype, "dtype_name": t.dtype_name.decode(),
                "shape": tuple(t.shape[: t.ndim]), "nbytes": int(t.nbytes), "data": t.data}

    def tensors(self) -> list[dict]:
        return [self.info(i) for i in range(len(self))]

    def find(self, name: str) -> int:
        i = ctypes.c_int()
        self._check(self._l.dsb_checkpoint_find(self.h, name.encode(), ctypes.byref(i)))
        return i.value

    def raw(self, name: str) -> bytes:
        """A tensor's bytes, copied out of the mapped shard."""
        i = self.find(name)
        if i < 0:
            raise KeyError(name)
        t = self.info(i)
        return ctypes.string_at(t["data"], t["nbytes"]) if t["nbytes"] else b""

    def close(self):
        if getattr(self, "h", None):
            self._l.dsb_checkpoint_close(self.h)
            self.h = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class Tokenizer:
    """dsb_tokenizer: the reference's greedy tokenizer over a tokenizer.json (host only)."""

    def __init__(self, path: str):
        self._l = lib()
        h = ctypes.c_void_p()
        rc = self._l.dsb_tokenizer_load(os.fsencode(path), ctypes.byref(h))
        if rc != DSB_OK:
            raise DsbError(rc, self._l.dsb_tokenizer_error().decode())
        self.h = h

    def _check(self, rc: int):
        if rc != DSB_OK:
            raise DsbError(rc, self._l.dsb_tokenizer_error().decode())

    def info(self) -> dict:
        n, b, e, u = ctypes.c_int(), ctypes.c_int32(), ctypes.c_int32(), ctypes.c_int32()
        self._check(self._l.dsb_tokenizer_info(self.h, ctypes.byref(n), ctypes.byref(b), ctypes.byref(e),
                                               ctypes.byref(u)))
        return {"n_ids": n.value, "bos": b.value, "eos": e.value, "unk": u.value}

    def encode(self, text: "str | bytes") -> list[int]:
        data = text.encode() if isinstance(text, str) else bytes(text)
        n = ctypes.c_size_t()
        cap = len(data) + 1  # at most one id per byte
        ids = (ctypes.c_int32 * cap)()
        self._check(self._l.dsb_tokenizer_encode(self.h, data, len(data), ids, cap, ctypes.byref(n)))
        return list(ids[: n.value])

    def decode(self, ids, skip_special: bool = True) -> bytes:
        arr = (ctypes.c_int32 * max(1, len(ids)))(*[int(i) for i in ids])
        n = ctypes.c_size_t()
        rc = self._l.dsb_tokenizer_decode(self.h, arr, len(ids), int(skip_special), None, 0, ctypes.byref(n))
        if rc != DSB_OK and n.value == 0:
            self._check(rc)
        buf = ctypes.create_string_buffer(n.value + 1)
        self._check(self._l.dsb_tokenizer_decode(self.h, arr, len(ids), int(skip_special), buf, n.value + 1,
                                                 ctypes.byref(n)))
        return buf.raw[: n.value]

    def close(self):
        if getattr(self, "h", None):
            self._l.dsb_tokenizer_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def load_model(ctx: "Context", path: str, ep: "EP | None" = None) -> "Model":
    """Create a model from a checkpoint directory, bind it to `ep` (expert
    parallel) when given, upload its decode-path tensors and finalize it."""
    with Checkpoint(path) as ck:
        m = Model(ctx, ck.config())
        try:
            if ep is not None:
                m.set_ep(ep)
            m.upload_checkpoint(ck)
            m.finalize()
        except Exception:
            m.close()
            raise
    return m


class EP:
    """An expert-parallel group member (dsb_ep): rank `rank` of `world`, owning
    experts [rank*E_local, (rank+1)*E_local).  Connect with every rank's
    window handle (bytes, rank order) before the first dispatch."""

    HANDLE_BYTES = 64

    def __init__(self, ctx: Context, rank: int, world: int, n_experts: int, hidden: int, top_k: int,
                 max_tokens: int):
        self.ctx, self._l = ctx, ctx._l
        h = ctypes.c_void_p()
        ctx._check(self._l.dsb_ep_create(ctx.h, rank, world, n_experts, hidden, top_k, max_tokens, ctypes.byref(h)))
        self.h = h
        self.rank, self.world, self.hidden, self.top_k = rank, world, hidden, top_k
        el, cap, nb = _ci(), _ci(), ctypes.c_uint64()
        ctx._check(self._l.dsb_ep_info(self.h, ctypes.byref(el), ctypes.byref(cap), ctypes.byref(nb)))
        self.E_local, self.capacity, self.window_bytes = el.value, cap.value, nb.value

    def window_handle(self) -> bytes:
        buf = ctypes.create_string_buffer(self.HANDLE_BYTES)
        self.ctx._check(self._l.dsb_ep_window_handle(self.h, buf))
        return buf.raw

    def connect(self, handles):
        blob = b"".join(handles)
        assert len(blob) == self.world * self.HANDLE_BYTES
        self.ctx._check(self._l.dsb_ep_connect(self.h, ctypes.create_string_buffer(blob, len(blob))))

    def window_ptr(self) -> int:
        p = ctypes.c_void_p()
        self.ctx._check(self._l.dsb_ep_window_ptr(self.h, ctypes.byref(p)))
        return p.value

    def connect_local(self, windows):
        """Connect with every rank's window device pointer (ranks driven from this process)."""
        arr = (ctypes.c_void_p * self.world)(*[int(w) if w else None for w in windows])
        self.ctx._check(self._l.dsb_ep_connect_local(self.h, arr))

    def dispatch(self, x, ids):
        """x bf16 [T, hidden], ids int32 [T, top_k] -> (recv_x, recv_offsets) torch views of the group's buffers."""
        import torch

        rx, ro = ctypes.c_void_p(), ctypes.c_void_p()
        self.ctx._check(self._l.dsb_ep_dispatch(self.h, _ptr(x), x.stride(0), x.shape[0], _ptr(ids), ctypes.byref(rx),
                                                ctypes.byref(ro)))
        recv = _device_view(rx.value, (self.capacity, self.hidden), torch.bfloat16, x.device)
        offs = _device_view(ro.value, (self.E_local + 1,), torch.int32, x.device)
        return recv, offs

    def combine(self, y, weights, h, shared=None):
        n_shared = 0 if shared is None else shared.shape[0]
        self.ctx._check(self._l.dsb_ep_combine(self.h, _ptr(y), y.stride(0), h.shape[0], _ptr(weights), _ptr(shared),
                                               n_shared, _ptr(h)))

    def close(self):
        if self.h:
            self._l.dsb_ep_destroy(self.h)
            self.h = None


def _device_view(ptr: int, shape, dtype, device):
    """A torch tensor over device memory owned by libdsb (no copy, no ownership)."""
    import torch

    class _Holder:
        pass

    hold = _Holder()
    n = 1
    for d in shape:
        n *= d
    itemsize = torch.empty((), dtype=dtype).element_size()
    hold.__cuda_array_interface__ = {
        "shape": tuple(shape), "typestr": {torch.bfloat16: "<V2", torch.int32: "<i4", torch.float32: "<f4"}[dtype],
        "data": (ptr, False), "version": 3, "strides": None,
    }
    if dtype == torch.bfloat16:
        hold.__cuda_array_interface__["typestr"] = "<i2"
        return torch.as_tensor(hold, device=device).view(torch.bfloat16)
    assert n * itemsize > 0
    return torch.as_tensor(hold, device=device)


class KVCache:
    """A dsb_kvcache: paged latent cache for every layer of a model."""

    def __init__(self, ctx: Context, model: Model, n_blocks: int, max_seqs: int, max_blocks_per_seq: int):
        self.ctx = ctx
        h = ctypes.c_void_p()
        ctx._check(ctx._l.dsb_kvcache_create(ctx.h, model.h, n_blocks, max_seqs, max_blocks_per_seq, ctypes.byref(h)))
        self.h = h

    def alloc_seq(self) -> int:
        s = ctypes.c_int()
        self.ctx._check(self.ctx._l.dsb_kvcache_alloc_seq(self.h, ctypes.byref(s)))
        return s.value

    def fill_random(self, seq: int, n_tokens: int, seed: int = 0, stddev: float = 1.0):
        """dsb_kvcache_fill_random: n_tokens synthetic cache positions for `seq`."""
        self.ctx._check(self.ctx._l.dsb_kvcache_fill_random(self.h, seq, n_tokens, seed, float(stddev)))

    def free_seq(self, seq: int):
        self.ctx._check(self.ctx._l.dsb_kvcache_free_seq(self.h, seq))

    def reset(self):
        self.ctx._check(self.ctx._l.dsb_kvcache_reset(self.h))

    def seq_len(self, seq: int) -> int:
        n = ctypes.c_int()
        self.ctx._check(self.ctx._l.dsb_kvcache_seq_len(self.h, seq, ctypes.byref(n)))
        return n.value

    def free_blocks(self) -> int:
        n = ctypes.c_int64()
        self.ctx._check(self.ctx._l.dsb_kvcache_free_blocks(self.h, ctypes.byref(n)))
        return n.value

    def close(self):
        if self.h:
            self.ctx._l.dsb_kvcache_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def decode_step(ctx: Context, model: Model, kv: KVCache, seq_ids, tokens, want_logits=False, logits_out=None):
    """dsb_decode_step: one token per sequence; returns (greedy ids, logits or None).

    logits_out: an optional C-contiguous float32 [B, vocab] host array that
    receives the logits (e.g. a view of pinned memory, so the copy back runs
    at full PCIe rate); otherwise a new array is allocated when want_logits.
    """
    import numpy as np

    B = len(seq_ids)
    sids = (ctypes.c_int32 * B)(*[int(x) for x in seq_ids])
    toks = (ctypes.c_int32 * B)(*[int(x) for x in tokens])
    greedy = (ctypes.c_int32 * B)()
    logits = logits_out
    if logits is not None:
        if (logits.dtype != np.float32 or logits.shape != (B, model.cfg.vocab_size)
                or not logits.flags["C_CONTIGUOUS"]):
            raise ValueError("logits_out must be a C-contiguous float32 [B, vocab] array")
    elif want_logits:
        logits = np.empty((B, model.cfg.vocab_size), np.float32)
    ctx._check(ctx._l.dsb_decode_step(ctx.h, model.h, kv.h, sids, toks, B,
                                      logits.ctypes.data if logits is not None else None, greedy))
    return np.array(greedy[:], np.int32), logits


PREFILL_MAX_TOKENS = 4096


def prefill(ctx: Context, model: Model, kv: KVCache, seq_ids, tokens, want_logits=False):
    """dsb_prefill: token rows (seq_ids[i], tokens[i]) in one pass, a sequence's
    tokens in order; returns (greedy ids, logits or None) for the last row of
    each distinct sequence, in order of first appearance."""
    import numpy as np

    n = len(seq_ids)
    if len(tokens) != n:
        raise ValueError("seq_ids and tokens differ in length")
    sids = (ctypes.c_int32 * n)(*[int(x) for x in seq_ids])
    toks = (ctypes.c_int32 * n)(*[int(x) for x in tokens])
    n_distinct = len(dict.fromkeys(int(x) for x in seq_ids))
    greedy = (ctypes.c_int32 * max(1, n_distinct))()
    logits = np.empty((n_distinct, model.cfg.vocab_size), np.float32) if want_logits else None
    n_seq = ctypes.c_int(0)
    ctx._check(ctx._l.dsb_prefill(ctx.h, model.h, kv.h, sids, toks, n,
                                  logits.ctypes.data if want_logits else None, greedy, ctypes.byref(n_seq)))
    return np.array(greedy[:n_seq.value], np.int32), logits


def prefill_prompts(ctx: Context, model: Model, kv: KVCache, seq_ids, prompts, chunk: int = PREFILL_MAX_TOKENS):
    """Prefill every sequence's prompt (lists of ids) through dsb_prefill in
    chunks of at most `chunk` rows (the prompts interleaved position by
    position); returns each sequence's greedy next id."""
    import numpy as np

    rows = []
    longest = max(len(p) for p in prompts)
    for i in range(longest):
        for s, p in zip(seq_ids, prompts):
            if i < len(p):
                rows.append((int(s), int(p[i])))
    nxt = {}
    for c0 in range(0, len(rows), chunk):
        part = rows[c0:c0 + chunk]
        g, _ = prefill(ctx, model, kv, [r[0] for r in part], [r[1] for r in part])
        for s, gid in zip(dict.fromkeys(r[0] for r in part), g):
            nxt[s] = int(gid)
    return np.array([nxt[int(s)] for s in seq_ids], np.int32)


def generate(ctx: Context, model: Model, kv: KVCache, seq_ids, prompts, max_new_tokens: int, eos_id: int = -1,
             sampling: "Sampling | None" = None):
    """dsb_generate (greedy), or dsb_generate_sampled when `sampling` is given:
    the continuation of every prompt (lists of ids); one id list per sequence."""
    import numpy as np

    B = len(prompts)
    toks = np.ascontiguousarray(np.concatenate([np.asarray(p, np.int32) for p in prompts]))
    offs = np.ascontiguousarray(np.concatenate([[0], np.cumsum([len(p) for p in prompts])]).astype(np.int32))
    sid = np.ascontiguousarray(np.asarray(seq_ids, np.int32))
    out = np.zeros((B, max(1, max_new_tokens)), np.int32)
    cnt = np.zeros(B, np.int32)
    if sampling is None:
        ctx._check(ctx._l.dsb_generate(ctx.h, model.h, kv.h, sid.ctypes.data, B, toks.ctypes.data,
                                       offs.ctypes.data, max_new_tokens, eos_id, out.ctypes.data, cnt.ctypes.data))
    else:
        ctx._check(ctx._l.dsb_generate_sampled(ctx.h, model.h, kv.h, sid.ctypes.data, B, toks.ctypes.data,
                                               offs.ctypes.data, max_new_tokens, eos_id, ctypes.byref(sampling),
                                               out.ctypes.data, cnt.ctypes.data))
    return [out[b, :cnt[b]].tolist() for b in range(B)]


def decode_step_sampled(ctx: Context, model: Model, kv: KVCache, seq_ids, tokens, sampling: "Sampling", uniforms,
                        want_logits=False):
    """dsb_decode_step_sampled: one token per sequence, next ids sampled with
    one uniform draw per row; returns (ids, logits or None)."""
    import numpy as np

    B = len(seq_ids)
    sids = (ctypes.c_int32 * B)(*[int(x) for x in seq_ids])
    toks = (ctypes.c_int32 * B)(*[int(x) for x in tokens])
    u = (ctypes.c_float * B)(*[float(x) for x in uniforms])
    out = (ctypes.c_int32 * B)()
    logits = np.empty((B, model.cfg.vocab_size), np.float32) if want_logits else None
    ctx._check(ctx._l.dsb_decode_step_sampled(ctx.h, model.h, kv.h, sids, toks, B, ctypes.byref(sampling), u,
                                              logits.ctypes.data if logits is not None else None, out))
    return np.array(out[:], np.int32), logits
