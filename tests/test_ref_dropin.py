"""The drop-in at the reference's own plug-in API.

deepseek_cpp_infer_b200/refapi implements the reference's ds::rt::Model /
ModelSession (include/ds/runtime/model.h:37-51) over libdsb.so and a
ModelPackageDescriptor (include/ds/models/core/registry.h:23-30) whose load
returns it.  oracle/_ref/ds_dropin_demo links that package with the
reference's compiled sources and drives it with the reference's own
ds::rt::generate (src/runtime/model.cpp:14-49) and ModelExecutor
(src/runtime/model_executor.cpp:18-50), unchanged.

On the CPU: the descriptor keeps the DeepSeek package's host functions
(print_config prints the reference's lines), and loading without a GPU fails
with a message.  On the GPU: on the golden tiny checkpoint the reference's
generate and ModelExecutor produce the reference's own greedy continuation
(tests/golden/tiny_model.npz), prefill + decode_next give its first two ids
at the right position, a CPU-backend session and an empty forward fail as
documented.
"""

import os
import subprocess

import numpy as np
import pytest

from ckpt_files import hf_config, tiny_tensors, write_model_dir
from deepseek_cpp_infer_b200.workloads import TINY

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
DEMO = os.path.join(ROOT, "oracle", "_ref", "ds_dropin_demo")
GOLD = os.path.join(ROOT, "tests", "golden", "tiny_model.npz")

pytestmark = pytest.mark.skipif(not os.path.exists(DEMO), reason="oracle/_ref/ds_dropin_demo not built "
                                                                   "(the reference sources were absent)")


@pytest.fixture(scope="module")
def model_dir(tmp_path_factory):
    d = str(tmp_path_factory.mktemp("dropin_model"))
    write_model_dir(d, hf_config(TINY), list(tiny_tensors()), n_shards=2)
    return d


def run(*args):
    return subprocess.run([DEMO, *[str(a) for a in args]], capture_output=True, text=True, timeout=300)


def test_descriptor_host_functions(model_dir):
    r = run("info", model_dir)
    assert r.returncode == 0, r.stderr
    lines = r.stdout.splitlines()
    assert lines[0] == "package deepseek_b200"
    assert lines[1] == "Loaded config:" and "  family: deepseek" in lines
    assert f"  layers: {TINY['num_hidden_layers']}" in lines and f"  n_experts: {TINY['n_routed_experts']}" in lines


def test_load_without_gpu_fails_with_a_message(model_dir):
    import torch

    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    r = run("gen", model_dir, "1,2,3", 2)
    assert r.returncode == 1 and r.stderr.startswith("error: b200 package: no usable CUDA device")


@pytest.mark.gpu
def test_reference_generate_and_executor_run_the_b200_model(gpu_ctx, model_dir):
    g = np.load(GOLD)
    prompt = g["prompt"].tolist()
    r = run("gen", model_dir, ",".join(map(str, prompt)), 16)
    assert r.returncode == 0, r.stderr
    out = dict(ln.split(" ", 1) for ln in r.stdout.splitlines())
    want = g["generated"][:16].tolist()
    assert [int(x) for x in out["ids"].split()] == want
    assert [int(x) for x in out["exec"].split()] == want
    assert int(out["position"]) == len(prompt) + 15  # generate does not feed back its last id
    first, second, pos = (int(x) for x in out["steps"].split())
    assert (first, second, pos) == (want[0], want[1], len(prompt) + 1)
    assert out["backends"] == "1 0"
    assert out["empty"] == "error forward: token_ids must not be empty"
    r = run("cpu", model_dir)
    assert r.returncode == 1 and "runs on the CUDA backend only" in r.stderr
