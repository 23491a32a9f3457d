"""Checkpoint ingest on the host (no GPU): dsb_checkpoint_* through the C ABI
on Hugging Face model directories written by tests/ckpt_files.py.

Pinned against the reference's own loader (oracle/_ref: load_model_dir and
parse_deepseek_config, src/hf/model_loader.cpp:17-94 and
src/models/deepseek/config.cpp:9-52) on the same directory: identical tensor
names, dtypes, byte counts and shapes, and identical config fields, except
the two fields where this reader deliberately differs (asserted below):
moe_intermediate_size, which the reference overwrites with
intermediate_size, and a JSON-boolean norm_topk_prob, which the reference's
get_int_or ignores.  The reference has no F8_E4M3 dtype (it reports UNKNOWN);
this reader maps it to DSB_DTYPE_F8E4M3.

Malformed files (truncated, out-of-range offsets, size mismatches, shard
names leaving the directory, bad JSON) must fail with a message, never
crash or read outside the mapping."""

import json
import os
import struct

import numpy as np
import pytest

import deepseek_cpp_infer_b200 as dsb
import oracle as O
from ckpt_files import MTP_LAYER, N_EXTRAS, hf_config, tiny_tensors, write_model_dir, write_safetensors
from deepseek_cpp_infer_b200.workloads import TINY, V2_LITE, V3

DT = {"F32": dsb.DTYPE_F32, "BF16": dsb.DTYPE_BF16, "F16": dsb.DTYPE_F16, "F8_E4M3": dsb.DTYPE_F8E4M3}
REF_DT = {"F16": 0, "BF16": 1, "F32": 2, "I32": 3, "I64": 4, "U8": 5}  # ds::hf::DType
REF_UNKNOWN = 6


def cfg_dict(c: dsb.ModelConfig) -> dict:
    return {n: getattr(c, n) for n, _ in c._fields_}


@pytest.fixture(scope="module")
def tiny_dir(tmp_path_factory):
    d = str(tmp_path_factory.mktemp("tiny"))
    tensors = tiny_tensors()
    write_model_dir(d, hf_config(TINY), tensors, n_shards=3)
    return d, tensors


def test_round_trip_names_dtypes_shapes_bytes(tiny_dir):
    d, tensors = tiny_dir
    with dsb.Checkpoint(d) as ck:
        got = cfg_dict(ck.config())
        for k, v in TINY.items():
            assert got[k] == pytest.approx(v), k
        assert got["weights_fp8"] == 0
        infos = ck.tensors()
        assert [t["name"] for t in infos] == [n for n, _, _ in tensors]
        for (name, dt, a), t in zip(tensors, infos):
            assert t["dtype"] == DT[dt] and t["dtype_name"] == dt and t["shape"] == a.shape, name
            assert t["nbytes"] == a.nbytes
            assert ck.raw(name) == np.ascontiguousarray(a).tobytes(), name
        assert ck.find("model.norm.weight") >= 0 and ck.find("no.such.tensor") == -1
        assert ck.find(f"model.layers.{MTP_LAYER}.enorm.weight") >= 0


def test_single_file_checkpoint(tmp_path):
    tensors = tiny_tensors(extras=False)[:20]
    write_model_dir(str(tmp_path), hf_config(TINY), tensors, n_shards=0)
    with dsb.Checkpoint(str(tmp_path)) as ck:
        assert [t["name"] for t in ck.tensors()] == [n for n, _, _ in tensors]
        assert ck.raw(tensors[5][0]) == tensors[5][2].tobytes()


def test_fp8_checkpoint_dtypes(tmp_path):
    tensors = tiny_tensors(fp8=True, extras=False)
    write_model_dir(str(tmp_path), hf_config(TINY, fp8=True), tensors, n_shards=2)
    with dsb.Checkpoint(str(tmp_path)) as ck:
        assert ck.config().weights_fp8 == 1
        w = ck.info(ck.find("model.layers.1.mlp.experts.3.down_proj.weight"))
        s = ck.info(ck.find("model.layers.1.mlp.experts.3.down_proj.weight_scale_inv"))
        assert w["dtype"] == dsb.DTYPE_F8E4M3 and w["dtype_name"] == "F8_E4M3"
        assert w["shape"] == (TINY["hidden_size"], TINY["moe_intermediate_size"]) and w["nbytes"] == 512 * 256
        assert s["dtype"] == dsb.DTYPE_F32 and s["shape"] == (4, 2)
        assert sum(t["dtype"] == dsb.DTYPE_F8E4M3 for t in ck.tensors()) == sum(dt == "F8_E4M3" for _, dt, _ in tensors)


def test_v3_config_fields(tmp_path):
    write_model_dir(str(tmp_path), hf_config(V3, fp8=True), [("x", "F32", np.zeros(4, np.float32))], n_shards=0)
    with dsb.Checkpoint(str(tmp_path)) as ck:
        c = cfg_dict(ck.config())
    for k, v in V3.items():
        assert c[k] == pytest.approx(v), k


def test_aliases_and_defaults(tmp_path):
    cfg = {"hidden_size": 64, "num_hidden_layers": 2, "vocab_size": 100, "num_experts": 8, "moe_top_k": 3,
           "intermediate_size": 96, "q_lora_rank": None, "norm_topk_prob": 1}
    write_model_dir(str(tmp_path), cfg, [("x", "F32", np.zeros(1, np.float32))], n_shards=0)
    with dsb.Checkpoint(str(tmp_path)) as ck:
        c = ck.config()
    assert (c.n_routed_experts, c.num_experts_per_tok, c.q_lora_rank, c.norm_topk_prob) == (8, 3, 0, 1)
    assert c.moe_intermediate_size == 96  # intermediate_size stands in when moe_intermediate_size is absent
    assert c.rms_norm_eps == pytest.approx(1e-5) and c.rope_theta == 10000.0 and c.routed_scaling_factor == 1.0
    assert (c.scoring_func, c.n_group, c.topk_group, c.weights_fp8) == (dsb.SCORE_SOFTMAX, 1, 1, 0)


@pytest.mark.skipif(not O.ref_available(), reason="reference build (oracle/_ref) not present")
@pytest.mark.parametrize("fp8", [False, True])
def test_matches_reference_loader(tmp_path, fp8):
    cfg = dict(V2_LITE, num_hidden_layers=TINY["num_hidden_layers"])
    tensors = tiny_tensors(fp8=fp8)
    write_model_dir(str(tmp_path), hf_config(cfg, fp8=fp8), tensors, n_shards=2)
    rcfg, rtensors = O.ref_checkpoint_summary(str(tmp_path))
    with dsb.Checkpoint(str(tmp_path)) as ck:
        ours = cfg_dict(ck.config())
        infos = ck.tensors()
    for k, v in rcfg.items():
        if k == "scoring_func":
            assert v == "softmax" and ours[k] == dsb.SCORE_SOFTMAX
        elif k == "moe_intermediate_size":
            # the reference lets intermediate_size override moe_intermediate_size
            assert int(v) == cfg["intermediate_size"] and ours[k] == cfg["moe_intermediate_size"]
        elif k in ("rms_norm_eps", "rope_theta", "routed_scaling_factor"):
            assert float(v) == pytest.approx(ours[k], rel=1e-6), k
        else:
            assert int(v) == ours[k], (k, v, ours[k])
    assert [t[0] for t in rtensors] == [t["name"] for t in infos]
    for (name, rdt, rbytes, rshape), t in zip(rtensors, infos):
        assert rbytes == t["nbytes"] and rshape == t["shape"], name
        assert rdt == (REF_UNKNOWN if t["dtype_name"] == "F8_E4M3" else REF_DT[t["dtype_name"]]), name


@pytest.mark.skipif(not O.ref_available(), reason="reference build (oracle/_ref) not present")
def test_norm_topk_prob_boolean_differs_from_reference(tmp_path):
    cfg = dict(hf_config(TINY), norm_topk_prob=True)
    write_model_dir(str(tmp_path), cfg, [("x", "F32", np.zeros(1, np.float32))], n_shards=1)  # the reference needs an index
    rcfg, _ = O.ref_checkpoint_summary(str(tmp_path))
    assert rcfg["norm_topk_prob"] == "0"  # the reference's get_int_or skips JSON booleans
    with dsb.Checkpoint(str(tmp_path)) as ck:
        assert ck.config().norm_topk_prob == 1


# ------------------------------------------------------------------ errors

def _header_file(path, header: bytes, data: bytes = b"", hlen: int | None = None):
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(header) if hlen is None else hlen) + header + data)


def _tensor_header(entries: dict) -> bytes:
    return json.dumps(entries).encode()


CFG = {"hidden_size": 8, "num_hidden_layers": 1, "vocab_size": 16}


def _case(tmp_path, name):
    d = str(tmp_path)
    cfg_text = json.dumps(CFG)
    st = os.path.join(d, "model.safetensors")
    good = _tensor_header({"a": {"dtype": "F32", "shape": [2, 3], "data_offsets": [0, 24]}})
    if name == "no_config":
        _header_file(st, good, bytes(24))
        return d, dsb.DSB_EINVAL, "config.json"
    if name == "config_bad_json":
        cfg_text = '{"hidden_size": 8,'
    elif name == "config_missing_fields":
        cfg_text = json.dumps({"hidden_size": 8})
    elif name == "config_scoring":
        cfg_text = json.dumps(dict(CFG, scoring_func="tanh"))
    elif name == "config_block":
        cfg_text = json.dumps(dict(CFG, quantization_config={"quant_method": "fp8", "weight_block_size": [64, 64]}))
    elif name == "config_quant":
        cfg_text = json.dumps(dict(CFG, quantization_config={"quant_method": "gptq"}))
    elif name == "config_int_range":
        cfg_text = json.dumps(dict(CFG, hidden_size=1 << 40))
    with open(os.path.join(d, "config.json"), "w") as f:
        f.write(cfg_text)
    expect = {"config_bad_json": (dsb.DSB_EINVAL, "config.json"),
              "config_missing_fields": (dsb.DSB_EINVAL, "missing required fields"),
              "config_scoring": (dsb.DSB_EUNSUPPORTED, "scoring_func"),
              "config_block": (dsb.DSB_EUNSUPPORTED, "weight_block_size"),
              "config_quant": (dsb.DSB_EUNSUPPORTED, "quant_method"),
              "config_int_range": (dsb.DSB_EINVAL, "out of range")}
    if name in expect:
        _header_file(st, good, bytes(24))
        return (d, *expect[name])
    if name == "no_weights":
        return d, dsb.DSB_EINVAL, "no model.safetensors"
    if name == "too_small":
        with open(st, "wb") as f:
            f.write(b"\x01\x00")
        return d, dsb.DSB_EINVAL, "too small"
    if name == "header_beyond_file":
        _header_file(st, good, bytes(24), hlen=1 << 40)
        return d, dsb.DSB_EINVAL, "header length"
    if name == "offsets_beyond_file":
        _header_file(st, good, bytes(20))
        return d, dsb.DSB_EINVAL, "beyond the file"
    if name == "size_mismatch":
        _header_file(st, _tensor_header({"a": {"dtype": "F32", "shape": [2, 3], "data_offsets": [0, 20]}}), bytes(24))
        return d, dsb.DSB_EINVAL, "does not match"
    if name == "offsets_reversed":
        _header_file(st, _tensor_header({"a": {"dtype": "F32", "shape": [0], "data_offsets": [8, 4]}}), bytes(24))
        return d, dsb.DSB_EINVAL, "data_offsets"
    if name == "unknown_dtype":
        _header_file(st, _tensor_header({"a": {"dtype": "F4", "shape": [2], "data_offsets": [0, 1]}}), bytes(4))
        return d, dsb.DSB_EINVAL, "unknown dtype"
    if name == "negative_dim":
        _header_file(st, _tensor_header({"a": {"dtype": "F32", "shape": [-1], "data_offsets": [0, 4]}}), bytes(4))
        return d, dsb.DSB_EINVAL, "bad shape"
    if name == "shape_overflow":
        _header_file(st, _tensor_header({"a": {"dtype": "F32", "shape": [1 << 31, 1 << 31, 1 << 31],
                                               "data_offsets": [0, 4]}}), bytes(4))
        return d, dsb.DSB_EINVAL, "does not match"
    if name == "missing_fields":
        _header_file(st, _tensor_header({"a": {"dtype": "F32", "shape": [1]}}), bytes(4))
        return d, dsb.DSB_EINVAL, "missing or malformed"
    if name == "too_deep":
        _header_file(st, b"[" * 100 + b"]" * 100)
        return d, dsb.DSB_EINVAL, "nested too deeply"
    if name == "repeated_key":
        _header_file(st, b'{"a": {"dtype": "F32", "shape": [1], "data_offsets": [0, 4]}, '
                         b'"a": {"dtype": "F32", "shape": [1], "data_offsets": [0, 4]}}', bytes(4))
        return d, dsb.DSB_EINVAL, "repeated key"
    if name == "trailing":
        _header_file(st, good + b" x", bytes(24))
        return d, dsb.DSB_EINVAL, "trailing"
    if name == "header_not_object":
        _header_file(st, b"[1, 2]")
        return d, dsb.DSB_EINVAL, "not an object"
    # indexed checkpoints
    idx = os.path.join(d, "model.safetensors.index.json")
    shard = os.path.join(d, "model-00001-of-00001.safetensors")
    _header_file(shard, good, bytes(24))
    if name == "missing_shard":
        wm = {"a": "model-00002-of-00002.safetensors"}
        err = "missing shard"
    elif name == "escaping_shard":
        wm = {"a": "../model-00001-of-00001.safetensors"}
        err = "bad shard name"
    elif name == "absolute_shard":
        wm = {"a": shard}
        err = "bad shard name"
    elif name == "tensor_not_in_shard":
        wm = {"a": "model-00001-of-00001.safetensors", "b": "model-00001-of-00001.safetensors"}
        err = "not found in shard header"
    elif name == "no_weight_map":
        with open(idx, "w") as f:
            json.dump({"metadata": {}}, f)
        return d, dsb.DSB_EINVAL, "weight_map"
    elif name == "empty_weight_map":
        wm = {}
        err = "no shards"
    else:
        raise AssertionError(name)
    with open(idx, "w") as f:
        json.dump({"weight_map": wm}, f)
    return d, dsb.DSB_EINVAL, err


ERROR_CASES = ["no_config", "config_bad_json", "config_missing_fields", "config_scoring", "config_block",
               "config_quant", "config_int_range", "no_weights", "too_small", "header_beyond_file",
               "offsets_beyond_file", "size_mismatch", "offsets_reversed", "unknown_dtype", "negative_dim",
               "shape_overflow", "missing_fields", "too_deep", "repeated_key", "trailing", "header_not_object",
               "missing_shard", "escaping_shard", "absolute_shard", "tensor_not_in_shard", "no_weight_map",
               "empty_weight_map"]


@pytest.mark.parametrize("name", ERROR_CASES)
def test_malformed_checkpoints_fail_with_a_message(tmp_path, name):
    d, code, text = _case(tmp_path, name)
    with pytest.raises(dsb.DsbError) as e:
        dsb.Checkpoint(d)
    assert e.value.code == code and text in str(e.value), (name, e.value.code, str(e.value))


def test_missing_directory(tmp_path):
    with pytest.raises(dsb.DsbError, match="config.json"):
        dsb.Checkpoint(str(tmp_path / "nope"))


def test_json_escapes_and_metadata(tmp_path):
    """Names with escapes (\\u00e9, a surrogate pair, \\/) decode to UTF-8; __metadata__ is not a tensor;
    a zero-element tensor is kept."""
    with open(tmp_path / "config.json", "w") as f:
        json.dump(CFG, f)
    hdr = ('{"__metadata__": {"format": "pt"}, "caf\\u00e9\\/x": {"dtype": "BF16", "shape": [2], '
           '"data_offsets": [0, 4]}, "z\\ud83d\\ude00": {"dtype": "I64", "shape": [1], "data_offsets": [4, 12]}, '
           '"empty": {"dtype": "F32", "shape": [0, 5], "data_offsets": [12, 12]}}').encode()
    _header_file(tmp_path / "model.safetensors", hdr, bytes(range(12)))
    with dsb.Checkpoint(str(tmp_path)) as ck:
        names = [t["name"] for t in ck.tensors()]
        assert names == sorted(["café/x", "z\U0001F600", "empty"], key=lambda s: s.encode())
        t = ck.info(ck.find("z\U0001F600"))
        assert t["dtype"] == dsb.DTYPE_OTHER and t["dtype_name"] == "I64" and ck.raw("z\U0001F600") == bytes(range(4, 12))
        assert ck.info(ck.find("empty"))["shape"] == (0, 5) and ck.raw("empty") == b""
        assert ck.raw("café/x") == bytes(range(4))


def test_abi_argument_checks():
    l = dsb.lib()
    import ctypes

    h = ctypes.c_void_p()
    assert l.dsb_checkpoint_open(None, ctypes.byref(h)) == dsb.DSB_EINVAL
    assert b"bad arguments" in l.dsb_checkpoint_error()
    assert l.dsb_checkpoint_close(None) == dsb.DSB_OK
    assert l.dsb_checkpoint_num_tensors(None, None) == dsb.DSB_EINVAL
    assert l.dsb_model_upload_checkpoint(None, None, None, None) == dsb.DSB_EINVAL


def test_out_of_range_tensor_index(tiny_dir):
    d, tensors = tiny_dir
    with dsb.Checkpoint(d) as ck:
        with pytest.raises(dsb.DsbError):
            ck.info(len(tensors))
        with pytest.raises(dsb.DsbError):
            ck.info(-1)
    assert N_EXTRAS == 3
