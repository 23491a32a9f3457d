"""ds_chat_b200, the command-line front end (the reference's ds_chat,
src/main.cpp:22-306, over the C ABI), on the host: the subcommands that need
no GPU (info, verify, strict) on a three-shard tiny checkpoint with a
tokenizer, and the failures (no CUDA device, bad options, missing files)
with the reference's "fatal: <message>" on stderr and exit status 1."""

import os
import subprocess

import pytest

import deepseek_cpp_infer_b200 as dsb
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
    r = cli(d, "strict")
    assert r.returncode == 0, r.stderr
    assert "layer 0: dense" in r.stdout and "layer 3: MoE" in r.stdout and "MoE layers: 3/4" in r.stdout


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
