"""ds_chat_b200, the command-line front end (the reference's ds_chat,
src/main.cpp:22-306, over the C ABI), on the host: the subcommands that need
no GPU (info, verify, strict) on a three-shard tiny checkpoint with a
tokenizer, and the failures (no CUDA device, bad options, missing files)
with the reference's "fatal: <message>" on stderr and exit status 1."""

import os
import subprocess

import pytest

import deepseek_cpp_infer_b200 as dsb
import oracle as O
from ckpt_files import hf_config, tiny_tensors, write_model_dir
from deepseek_cpp_infer_b200.workloads import TINY
from tok_files import make_tokenizer

CLI = os.path.join(os.path.dirname(dsb.LIB_PATH), "ds_chat_b200")


def cli(*args):
    if not os.path.exists(CLI):
        pytest.fail(f"{CLI} is missing: build it with `make -C deepseek_cpp_infer_b200`")
    return subprocess.run([CLI, *map(str, args)], capture_output=True, text=True, timeout=120)


@pytest.fixture(scope="module")
def model_dir(tmp_path_factory):
    d = str(tmp_path_factory.mktemp("tiny_cli"))
    tensors = list(tiny_tensors())
    write_model_dir(d, hf_config(TINY), tensors, n_shards=3)
    make_tokenizer(os.path.join(d, "tokenizer.json"), min_ids=TINY["vocab_size"])
    return d, len(tensors)


def test_info_verify_strict(model_dir):
    d, n = model_dir
    r = cli(d, "info")
    assert r.returncode == 0, r.stderr
    assert "layers: 4" in r.stdout and "Tokenizer: OK" in r.stdout and f"Tensors: {n}" in r.stdout
    r = cli(d)  # verify is the default
    assert r.returncode == 0 and f"OK (parsed headers). total_tensors={n}" in r.stdout, r.stderr
    assert "Index OK (required tensor keys present)" in r.stdout
    r = cli(d, "strict")
    assert r.returncode == 0, r.stderr
    assert "layer 0: dense" in r.stdout and "layer 3: MoE" in r.stdout and "MoE layers: 3/4" in r.stdout


def test_verify_names_a_missing_tensor(tmp_path):
    tensors = [t for t in tiny_tensors(extras=False) if t[0] != "model.layers.2.mlp.experts.15.down_proj.weight"]
    write_model_dir(str(tmp_path), hf_config(TINY), tensors, n_shards=1)
    r = cli(str(tmp_path), "verify")
    assert r.returncode == 1 and "missing tensor in index: model.layers.2.mlp.experts.15.down_proj.weight" in r.stderr


def test_help():
    r = cli("--help")
    assert r.returncode == 0 and r.stdout.startswith("usage: ds_chat_b200") and "generate" in r.stdout


def test_failures_are_fatal_with_a_message(model_dir, tmp_path):
    d, _ = model_dir
    cases = [
        ((), "usage: ds_chat_b200"),
        ((str(tmp_path / "none"), "info"), "missing config.json"),
        ((d, "generate", "--bogus", "1"), "unknown option: --bogus"),
        ((d, "generate", "--max-new-tokens"), "missing value for --max-new-tokens"),
        ((d, "generate", "--top-k", "x"), "bad value for --top-k"),
        ((d, "frobnicate", "--seed", "1"), "usage: ds_chat_b200"),
    ]
    if not __import__("torch").cuda.is_available():
        cases.append(((d, "run", "--prompt-ids", "1,2,3"), "no usable CUDA device"))
    for args, text in cases:
        r = cli(*args)
        assert r.returncode == 1 and "fatal: " in r.stderr and text in r.stderr, (args, r.stderr)


REF_CLI = os.path.join(os.path.dirname(O.REF_SO), "ds_chat")


@pytest.mark.skipif(not os.path.exists(REF_CLI), reason="reference command line (oracle/_ref/ds_chat) not built")
def test_strict_matches_the_reference_command_line(model_dir, tmp_path):
    """`strict` on the same checkpoint: the reference's ds_chat and this one
    report the same key count, layer map and tensor total; a missing expert
    tensor fails both with the same message."""
    d, n = model_dir

    def lines(out):
        keep = ("Index OK", "  layer ", "MoE layers", "total_tensors")
        return [ln.split(" bytes=")[0] for ln in out.splitlines() if ln.startswith(keep) or "total_tensors=" in ln]

    ref = subprocess.run([REF_CLI, d, "strict"], capture_output=True, text=True, timeout=120)
    ours = cli(d, "strict")
    assert ref.returncode == 0 == ours.returncode, ref.stderr
    ref_lines = [ln.split("OK (parsed headers). ")[-1] for ln in lines(ref.stdout)]
    our_lines = [ln.split("OK (parsed headers). ")[-1] for ln in lines(ours.stdout)]
    assert ref_lines == our_lines, (ref_lines, our_lines)
    tensors = [t for t in tiny_tensors(extras=False) if t[0] != "model.layers.2.mlp.experts.15.down_proj.weight"]
    write_model_dir(str(tmp_path), hf_config(TINY), tensors, n_shards=1)
    ref = subprocess.run([REF_CLI, str(tmp_path), "verify"], capture_output=True, text=True, timeout=120)
    ours = cli(str(tmp_path), "verify")
    assert ref.returncode == 1 == ours.returncode
    msg = "missing tensor in index: model.layers.2.mlp.experts.15.down_proj.weight"
    assert msg in ref.stderr and msg in ours.stderr


@pytest.mark.skipif(not os.path.exists(REF_CLI), reason="reference command line (oracle/_ref/ds_chat) not built")
def test_reference_command_line_reads_our_checkpoint_files(model_dir):
    """The reference's own ds_chat, on the checkpoint directory written by
    tests/ckpt_files.py, generates the golden continuation of the golden
    prompt (its CPU backend): the files are what its loader expects."""
    import numpy as np

    d, _ = model_dir
    g = np.load(os.path.join(os.path.dirname(__file__), "golden", "tiny_model.npz"))
    ids = ",".join(map(str, g["prompt"].tolist()))
    r = subprocess.run([REF_CLI, d, "generate", "--prompt-ids", ids, "--max-new-tokens", "16", "--backend", "cpu"],
                       capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr
    line = next(ln for ln in r.stdout.splitlines() if ln.startswith("Generated ids:"))
    assert [int(x) for x in line.split(":")[1].split()] == g["generated"][:16].tolist()


from hypothesis import given, settings, strategies as st  # noqa: E402

_words = st.sampled_from(["info", "verify", "strict", "run", "generate", "bench", "load", "--prompt", "--prompt-ids",
                          "--max-new-tokens", "--top-k", "--top-p", "--temperature", "--seed", "--max-seq", "1",
                          "-3", "x", "", "1,2,3", "0.5", "--device", "99"])


@settings(max_examples=40, deadline=None, derandomize=True)
@given(args=st.lists(_words, max_size=6))
def test_random_arguments_never_crash(model_dir, args):
    """Any argument list ends with status 0 or 1 (fatal message), never a signal."""
    d, _ = model_dir
    r = subprocess.run([CLI, d, *args], capture_output=True, text=True, timeout=120)
    assert r.returncode in (0, 1), (args, r.returncode, r.stderr[-200:])
    if r.returncode == 1:
        assert r.stderr.startswith("fatal: ")
