"""ds_chat_b200 on the GPU against the Python API on the same checkpoint:
`run` prints the prefill's greedy id, `generate` the same ids as
dsb_generate (greedy) and dsb_generate_sampled (sampled, fixed seed), text
through the tokenizer, and `bench` a decode line."""

import os
import re
import subprocess

import pytest

import deepseek_cpp_infer_b200 as dsb
from ckpt_files import hf_config, tiny_tensors, write_model_dir
from deepseek_cpp_infer_b200.workloads import TINY
from tok_files import make_tokenizer

pytestmark = pytest.mark.gpu
CLI = os.path.join(os.path.dirname(dsb.LIB_PATH), "ds_chat_b200")
PROMPT = [5, 99, 1024, 7, 3000, 12, 700]


def cli(*args):
    r = subprocess.run([CLI, *map(str, args)], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr
    return r.stdout


@pytest.fixture(scope="module")
def model_dir(tmp_path_factory):
    d = str(tmp_path_factory.mktemp("tiny_cli_gpu"))
    write_model_dir(d, hf_config(TINY), list(tiny_tensors()), n_shards=2)
    make_tokenizer(os.path.join(d, "tokenizer.json"), min_ids=TINY["vocab_size"])
    return d


def python_generate(ctx, d, n, sampling=None):
    m = dsb.load_model(ctx, d)
    kv = dsb.KVCache(ctx, m, n_blocks=8, max_seqs=1, max_blocks_per_seq=4)
    s = kv.alloc_seq()
    ids = dsb.generate(ctx, m, kv, [s], [PROMPT], n, sampling=sampling)[0]
    kv.close()
    m.close()
    return ids


def test_run_and_generate_match_the_python_api(gpu_ctx, model_dir):
    d = model_dir
    ids_csv = ",".join(map(str, PROMPT))
    greedy = python_generate(gpu_ctx, d, 10)
    out = cli(d, "run", "--prompt-ids", ids_csv)
    assert f"Next token id: {greedy[0]}" in out and "Next token text:" in out
    out = cli(d, "generate", "--prompt-ids", ids_csv, "--max-new-tokens", 10)
    got = [int(x) for x in re.search(r"Generated ids:([ 0-9]*)", out).group(1).split()]
    assert got == greedy and "Generated text:" in out
    smp = dsb.Sampling(1.2, 40, 0.9, 5)
    sampled = python_generate(gpu_ctx, d, 10, sampling=smp)
    out = cli(d, "generate", "--prompt-ids", ids_csv, "--max-new-tokens", 10, "--temperature", 1.2, "--top-k", 40,
              "--top-p", 0.9, "--seed", 5)
    assert [int(x) for x in re.search(r"Generated ids:([ 0-9]*)", out).group(1).split()] == sampled


def test_text_prompt_load_and_bench(gpu_ctx, model_dir):
    d = model_dir
    out = cli(d, "generate", "--prompt", "the quick brown fox", "--max-new-tokens", 4)
    assert len(re.search(r"Generated ids:([ 0-9]*)", out).group(1).split()) == 4
    assert "OK" in cli(d, "load")
    out = cli(d, "bench", "--batch", 4, "--prompt-len", 64, "--steps", 4)
    assert re.search(r"Decode: 4 steps of 4 sequences .* tokens/s", out), out


def test_generate_prints_the_reference_continuation(gpu_ctx, model_dir):
    """The same command as the reference's ds_chat on the same checkpoint
    directory: the golden prompt's first 16 generated ids, which the
    reference's own CLI prints too (tests/test_cli.py)."""
    import numpy as np

    g = np.load(os.path.join(os.path.dirname(__file__), "golden", "tiny_model.npz"))
    out = cli(model_dir, "generate", "--prompt-ids", ",".join(map(str, g["prompt"].tolist())), "--max-new-tokens", 16)
    got = [int(x) for x in re.search(r"Generated ids:([ 0-9]*)", out).group(1).split()]
    assert got == g["generated"][:16].tolist(), got
