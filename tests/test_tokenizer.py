"""dsb_tokenizer (host C++, through the C ABI) against the reference's own
ds::rt::Tokenizer (oracle/_ref) on synthetic tokenizer.json files: the same
ids for every text (or the same failure at the same byte offset), the same
decoded bytes with and without special tokens.  The vocabularies mix the
conventions the reference handles: plain pieces, SentencePiece "▁" and
byte-level "Ġ" word starts, "</w>" word ends, "##" continuations, multi-byte
UTF-8, added tokens overriding ids, special tokens flagged 1 (both agree)
and true (only this library counts a JSON boolean; asserted as the one
difference).  Texts mix words, runs of the six C isspace bytes, punctuation
and UTF-8; a long text checks that encoding is not quadratic."""

import json
import time

import numpy as np
import pytest

import deepseek_cpp_infer_b200 as dsb
import oracle as O

from tok_files import BOOL_SPECIAL, GPT, SPM, make_tokenizer, random_text

def ours_encode(tok, data):
    try:
        return tok.encode(data)
    except dsb.DsbError as e:
        return str(e)


need_ref = pytest.mark.skipif(not O.ref_available(), reason="reference build (oracle/_ref) not present")


@need_ref
@pytest.mark.parametrize("seed", [0, 1, 2])
def test_encode_and_decode_match_reference(tmp_path, seed):
    path = str(tmp_path / "tokenizer.json")
    make_tokenizer(path, seed=seed, root_ids=seed == 2)
    tok = dsb.Tokenizer(path)
    rng = np.random.default_rng(100 + seed)
    for _ in range(150):
        data = random_text(rng, int(rng.integers(0, 40))).encode()
        want = O.ref_tokenize(path, data)
        got = ours_encode(tok, data)
        if isinstance(want, str):
            assert isinstance(got, str) and want in got, (data, want, got)
            continue
        assert got == want, data
        for skip in (False, True):
            ref = O.ref_detokenize(path, want, skip)
            mine = tok.decode(got, skip)
            if skip and BOOL_SPECIAL in want:
                assert mine == ref.replace(b"</s>", b""), data  # the boolean-special difference
            else:
                assert mine == ref, (data, skip)
    tok.close()


@need_ref
def test_decode_of_random_ids_matches_reference(tmp_path):
    """Every piece kind through the reference's trim (## / </w> / ▁ / Ġ, UTF-8, added tokens)."""
    path = str(tmp_path / "tokenizer.json")
    vocab = make_tokenizer(path, seed=3)
    tok = dsb.Tokenizer(path)
    rng = np.random.default_rng(9)
    n = max(vocab.values()) + 1
    kinds = {p[:1] for p in vocab}
    assert {SPM, GPT, "#"} <= kinds
    for _ in range(100):
        ids = rng.integers(0, n, size=int(rng.integers(0, 30))).tolist()
        assert tok.decode(ids, False) == O.ref_detokenize(path, ids, False), ids
        if BOOL_SPECIAL not in ids:
            assert tok.decode(ids, True) == O.ref_detokenize(path, ids, True), ids


@need_ref
def test_unencodable_bytes_fail_at_the_same_offset(tmp_path):
    path = str(tmp_path / "tokenizer.json")
    make_tokenizer(path)
    tok = dsb.Tokenizer(path)
    for data in (b"the quick \x01 fox", b"\x02", "café ☃".encode(), b"dog\xff"):
        want = O.ref_tokenize(path, data)
        assert isinstance(want, str) and "byte offset" in want
        with pytest.raises(dsb.DsbError) as e:
            tok.encode(data)
        assert want in str(e.value)


@need_ref
def test_whitespace_only_and_empty(tmp_path):
    path = str(tmp_path / "tokenizer.json")
    make_tokenizer(path)
    tok = dsb.Tokenizer(path)
    for data in (b"", b" ", b" \t\n\r\x0b\x0c ", b"   the"):
        assert tok.encode(data) == O.ref_tokenize(path, data)
    assert tok.decode([]) == b"" == O.ref_detokenize(path, [])


@need_ref
def test_boolean_special_is_the_one_difference(tmp_path):
    path = str(tmp_path / "tokenizer.json")
    make_tokenizer(path)
    tok = dsb.Tokenizer(path)
    assert tok.decode([7, BOOL_SPECIAL], skip_special=True) == b""
    assert O.ref_detokenize(path, [7, BOOL_SPECIAL], True) == b"</s>"
    assert tok.decode([7, BOOL_SPECIAL], skip_special=False) == b"<s></s>" == O.ref_detokenize(path, [7, 9], False)
    # decoding an out-of-range id fails in both
    assert O.ref_detokenize(path, [10 ** 6]) is None
    with pytest.raises(dsb.DsbError, match="out of range"):
        tok.decode([10 ** 6])
    assert tok.info()["n_ids"] == len(json.load(open(path))["model"]["vocab"])


def test_long_text_encodes_in_linear_time(tmp_path):
    path = str(tmp_path / "tokenizer.json")
    make_tokenizer(path)
    tok = dsb.Tokenizer(path)
    rng = np.random.default_rng(5)
    data = random_text(rng, 40000).encode()  # ~200 KB
    t0 = time.perf_counter()
    ids = tok.encode(data)
    dt = time.perf_counter() - t0
    assert len(ids) > 10000 and dt < 2.0, (len(ids), dt)
    if O.ref_available():  # the reference on a prefix that ends at a word boundary
        cut = data.index(b" ", 3000)
        assert tok.encode(data[:cut]) == O.ref_tokenize(path, data[:cut])


def test_buffer_protocol_and_errors(tmp_path):
    import ctypes

    path = str(tmp_path / "tokenizer.json")
    make_tokenizer(path)
    tok = dsb.Tokenizer(path)
    l = dsb.lib()
    n = ctypes.c_size_t()
    data = b"the quick brown fox"
    assert l.dsb_tokenizer_encode(tok.h, data, len(data), None, 0, ctypes.byref(n)) == dsb.DSB_EINVAL
    assert n.value == len(tok.encode(data)) > 0
    ids = (ctypes.c_int32 * n.value)(*tok.encode(data))
    m = ctypes.c_size_t()
    assert l.dsb_tokenizer_decode(tok.h, ids, n.value, 1, None, 0, ctypes.byref(m)) == dsb.DSB_EINVAL
    assert m.value == len(tok.decode(list(ids)))
    bad = tmp_path / "bad.json"
    for doc in ("{", "[]", '{"model": 3}', '{"model": {"vocab": []}}', '{"model": {"vocab": {"a": -3}}}',
                '{"model": {"vocab": {"a": 99999999999}}}', '{"model": {"vocab": {"a": 1, "a": 2}}}'):
        bad.write_text(doc)
        with pytest.raises(dsb.DsbError):
            dsb.Tokenizer(str(bad))
    with pytest.raises(dsb.DsbError):
        dsb.Tokenizer(str(tmp_path / "missing.json"))
    assert l.dsb_tokenizer_load(None, None) == dsb.DSB_EINVAL
    assert l.dsb_tokenizer_destroy(None) == dsb.DSB_OK
