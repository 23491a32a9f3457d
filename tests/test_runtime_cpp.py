"""dsb/runtime.hpp, the reference's ds::rt C++ API (load_model, Model,
ModelSession, ModelExecutor, generate, Tokenizer, and BatchSession) over
the C ABI: a C++
program (tests/cpp/rt_demo.cpp) compiled against the header with warnings
as errors.  On the CPU: the tokenizer gives the C ABI's ids and text, and
load_model without a GPU throws dsb::rt::Error with its message.  On the GPU:
ModelExecutor::generate on the golden prompt prints the reference's
continuation, prefill / decode_next agree with it, sampled generation
prints the ids of the same calls replayed from Python with the reference
Sampler's draws for the seed, and a BatchSession
generates two prompts together as the Python batched generate does."""

import os
import subprocess

import numpy as np
import pytest

import deepseek_cpp_infer_b200 as dsb
from ckpt_files import hf_config, tiny_tensors, write_model_dir
from deepseek_cpp_infer_b200.workloads import TINY
from tok_files import make_tokenizer

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
GOLD = os.path.join(ROOT, "tests", "golden", "tiny_model.npz")


@pytest.fixture(scope="module")
def demo(tmp_path_factory):
    exe = str(tmp_path_factory.mktemp("rt") / "rt_demo")
    libdir = os.path.dirname(dsb.LIB_PATH)
    subprocess.run(["g++", "-std=c++17", "-O1", "-Wall", "-Wextra", "-Werror", "-pedantic",
                    f"-I{os.path.join(ROOT, 'include')}", os.path.join(ROOT, "tests", "cpp", "rt_demo.cpp"), "-o",
                    exe, f"-L{libdir}", "-ldsb", f"-Wl,-rpath,{libdir}"], check=True)
    return exe


@pytest.fixture(scope="module")
def model_dir(tmp_path_factory):
    d = str(tmp_path_factory.mktemp("rt_model"))
    write_model_dir(d, hf_config(TINY), list(tiny_tensors()), n_shards=2)
    make_tokenizer(os.path.join(d, "tokenizer.json"), min_ids=TINY["vocab_size"])
    return d


def run(*args):
    return subprocess.run([str(a) for a in args], capture_output=True, text=True, timeout=300)


def test_tokenizer_and_errors_on_the_host(demo, model_dir):
    path = os.path.join(model_dir, "tokenizer.json")
    text = "the quick brown fox jumps over the lazy dog"
    r = run(demo, "tok", path, text)
    assert r.returncode == 0, r.stderr
    tok = dsb.Tokenizer(path)
    ids = tok.encode(text)
    assert r.stdout.splitlines()[0] == "ids " + " ".join(map(str, ids))
    assert r.stdout.splitlines()[1] == "text " + tok.decode(ids, skip_special=False).decode()
    r = run(demo, "load", "/nonexistent-model-dir")
    assert r.returncode == 1 and r.stderr.startswith(f"error {dsb.DSB_EINVAL}:") and "config.json" in r.stderr
    if not __import__("torch").cuda.is_available():
        r = run(demo, "load", model_dir)
        assert r.returncode == 1 and "no usable CUDA device" in r.stderr


@pytest.mark.gpu
def test_executor_generates_the_reference_continuation(gpu_ctx, demo, model_dir):
    g = np.load(GOLD)
    prompt = g["prompt"].tolist()
    r = run(demo, "gen", model_dir, ",".join(map(str, prompt)), 16)
    assert r.returncode == 0, r.stderr
    lines = dict(ln.split(" ", 1) for ln in r.stdout.splitlines())
    assert [int(x) for x in lines["ids"].split()] == g["generated"][:16].tolist()
    assert int(lines["position"]) == len(prompt) + 15  # the last generated id is not fed back
    first, second, pos = (int(x) for x in lines["steps"].split())
    assert (first, second, pos) == (int(g["generated"][0]), int(g["generated"][1]), len(prompt) + 1)
    # sampled: the same calls replayed from Python (prefill of all but the last
    # prompt token, then sampled steps) with the reference Sampler's own
    # uniforms for seed 5 (std::mt19937(5)), as dsb::rt::generate draws them
    r = run(demo, "gen", model_dir, ",".join(map(str, prompt)), 12, 1.2, 40, 0.9, 5)
    assert r.returncode == 0, r.stderr
    got = [int(x) for x in r.stdout.splitlines()[0].split()[1:]]
    import oracle as O

    u = np.zeros(12, np.float32)
    O.ref().ref_sampler_uniforms(5, 12, O.p(u, O.f32p))
    cfg = dsb.Sampling(1.2, 40, 0.9, 5)
    m = dsb.load_model(gpu_ctx, model_dir)
    kv = dsb.KVCache(gpu_ctx, m, n_blocks=8, max_seqs=1, max_blocks_per_seq=4)
    s = kv.alloc_seq()
    dsb.prefill(gpu_ctx, m, kv, [s] * (len(prompt) - 1), prompt[:-1])
    tok, want = prompt[-1], []
    for j in range(12):
        ids, _ = dsb.decode_step_sampled(gpu_ctx, m, kv, [s], [tok], cfg, [float(u[j])])
        want.append(int(ids[0]))
        tok = want[-1]
    kv.close()
    m.close()
    assert got == want


@pytest.mark.gpu
def test_batch_session_matches_the_python_batched_generate(gpu_ctx, demo, model_dir):
    g = np.load(GOLD)
    p0, p1 = g["prompt"].tolist(), [5, 99, 1024, 7, 3000]
    r = run(demo, "batch", model_dir, ",".join(map(str, p0)), ",".join(map(str, p1)), 10)
    assert r.returncode == 0, r.stderr
    got = [[int(x) for x in ln.split()[1:]] for ln in r.stdout.splitlines()]
    assert got[0] == g["generated"][:10].tolist()
    m = dsb.load_model(gpu_ctx, model_dir)
    kv = dsb.KVCache(gpu_ctx, m, n_blocks=8, max_seqs=2, max_blocks_per_seq=4)
    seqs = [kv.alloc_seq(), kv.alloc_seq()]
    assert got == dsb.generate(gpu_ctx, m, kv, seqs, [p0, p1], 10)
    kv.close()
    m.close()
