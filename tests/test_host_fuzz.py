"""Property tests of the host-side readers on untrusted input (no GPU): the
safetensors / config / index reader and the tokenizer.json reader must
return a status for any file, never crash or read outside the mapping, and
whatever they accept must be self-consistent (every tensor's bytes lie inside
its shard and match its dtype and shape; encode output decodes)."""

import json
import os
import struct

from hypothesis import HealthCheck, given, settings
from hypothesis import strategies as st

import deepseek_cpp_infer_b200 as dsb

CFG = {"hidden_size": 8, "num_hidden_layers": 1, "vocab_size": 16}
SETTINGS = settings(max_examples=150, deadline=None, derandomize=True, suppress_health_check=list(HealthCheck))

json_values = st.recursive(
    st.none() | st.booleans() | st.integers(-2**70, 2**70) | st.floats(allow_nan=False) | st.text(max_size=20),
    lambda children: st.lists(children, max_size=6) | st.dictionaries(st.text(max_size=8), children, max_size=6),
    max_leaves=30)


def _open(path):
    try:
        with dsb.Checkpoint(path) as ck:
            infos = ck.tensors()
            for t in infos:  # accepted tensors are self-consistent
                assert t["nbytes"] >= 0
                if t["nbytes"]:
                    assert len(ck.raw(t["name"])) == t["nbytes"]
            return infos
    except dsb.DsbError as e:
        assert e.code in (dsb.DSB_EINVAL, dsb.DSB_EUNSUPPORTED, dsb.DSB_ENOMEM)
        return None


@SETTINGS
@given(data=st.binary(max_size=300))
def test_random_bytes_as_a_shard(tmp_path_factory, data):
    d = tmp_path_factory.mktemp("fz")
    (d / "config.json").write_text(json.dumps(CFG))
    (d / "model.safetensors").write_bytes(data)
    _open(str(d))


@SETTINGS
@given(header=json_values, pad=st.integers(0, 64), hlen_delta=st.integers(-3, 3))
def test_random_json_headers(tmp_path_factory, header, pad, hlen_delta):
    d = tmp_path_factory.mktemp("fz")
    (d / "config.json").write_text(json.dumps(CFG))
    h = json.dumps(header).encode()
    (d / "model.safetensors").write_bytes(struct.pack("<Q", max(0, len(h) + hlen_delta)) + h + bytes(pad))
    _open(str(d))


@SETTINGS
@given(cut=st.integers(0, 400), flip=st.integers(0, 400), bit=st.integers(0, 7))
def test_truncated_and_flipped_valid_shards(tmp_path_factory, cut, flip, bit):
    d = tmp_path_factory.mktemp("fz")
    (d / "config.json").write_text(json.dumps(CFG))
    hdr = {"a": {"dtype": "F32", "shape": [2, 3], "data_offsets": [0, 24]},
           "b": {"dtype": "BF16", "shape": [5], "data_offsets": [24, 34]}, "__metadata__": {"format": "pt"}}
    h = json.dumps(hdr).encode()
    blob = bytearray(struct.pack("<Q", len(h)) + h + bytes(range(34)))
    if flip < len(blob):
        blob[flip] ^= 1 << bit
    (d / "model.safetensors").write_bytes(bytes(blob[: max(0, len(blob) - cut)] if cut < len(blob) else b""))
    _open(str(d))


@SETTINGS
@given(cfg=json_values)
def test_random_config_json(tmp_path_factory, cfg):
    d = tmp_path_factory.mktemp("fz")
    (d / "config.json").write_text(json.dumps(cfg))
    (d / "model.safetensors").write_bytes(struct.pack("<Q", 2) + b"{}")
    _open(str(d))


@SETTINGS
@given(doc=json_values, text=st.binary(max_size=60))
def test_random_tokenizer_json(tmp_path_factory, doc, text):
    d = tmp_path_factory.mktemp("fz")
    path = os.path.join(d, "tokenizer.json")
    with open(path, "w") as f:
        json.dump(doc, f)
    try:
        tok = dsb.Tokenizer(path)
    except dsb.DsbError:
        return
    try:
        ids = tok.encode(text)
    except dsb.DsbError:
        return
    tok.decode(ids, skip_special=False)


@SETTINGS
@given(vocab=st.dictionaries(st.text(min_size=1, max_size=6), st.integers(0, 300), min_size=1, max_size=40),
       text=st.text(max_size=40))
def test_random_vocabularies_encode_consistently(tmp_path_factory, vocab, text):
    """Whatever the vocabulary, every encoded id lies in the table and
    decoding the ids succeeds; a text made of single-character pieces always
    encodes (a longer greedy match ends on a character boundary, and every
    character after it is a piece)."""
    d = tmp_path_factory.mktemp("fz")
    path = os.path.join(d, "tokenizer.json")
    with open(path, "w") as f:
        json.dump({"model": {"vocab": vocab}}, f)
    tok = dsb.Tokenizer(path)
    n = tok.info()["n_ids"]
    assert n == max(vocab.values()) + 1
    pieces = [p for p in vocab if len(p) == 1 and not p.isspace()]
    joined = "".join(pieces[:5])
    for t in (text, joined):
        try:
            ids = tok.encode(t)
        except dsb.DsbError as e:
            assert "byte offset" in str(e) and t is text
            continue
        assert all(0 <= i < n for i in ids)
        tok.decode(ids, skip_special=False)
    tok.close()
