"""Models loaded from Hugging Face checkpoint directories
(dsb_checkpoint_open + dsb_model_upload_checkpoint, through the C ABI) decode
exactly like the same weights uploaded tensor by tensor with
dsb_model_set_tensor: logits bit-identical at every step of the golden
sequence, for the bf16 tiny model (stored as BF16 / F32 in three shards)
and for its block-scaled FP8 version (F8_E4M3 codes plus F32
weight_scale_inv, as a DeepSeek-V3 checkpoint stores them).  The checkpoint
model also reproduces the reference's greedy continuation
(tests/golden/tiny_model.npz).  Tensors decoding does not run (a
multi-token-prediction layer past num_hidden_layers, rotary inv_freq) are
skipped and counted; unknown tensors and unsupported dtypes fail with the
tensor's name."""

import os

import numpy as np
import pytest

import deepseek_cpp_infer_b200 as dsb
from ckpt_files import N_EXTRAS, bf16_bits, hf_config, tiny_tensors, write_model_dir
from deepseek_cpp_infer_b200.workloads import TINY, model_tensors

pytestmark = pytest.mark.gpu
GOLD = os.path.join(os.path.dirname(__file__), "golden", "tiny_model.npz")


def decode(ctx, m, tokens):
    """Teacher-force `tokens` through one sequence: greedy id and logits after each."""
    kv = dsb.KVCache(ctx, m, n_blocks=16, max_seqs=1, max_blocks_per_seq=4)
    s = kv.alloc_seq()
    ids, logits = [], []
    for t in tokens:
        gid, lg = dsb.decode_step(ctx, m, kv, [s], [int(t)], want_logits=True)
        ids.append(int(gid[0]))
        logits.append(lg[0].copy())
    kv.close()
    return np.array(ids, np.int32), np.stack(logits)


def test_bf16_checkpoint_decodes_like_set_tensor(gpu_ctx, tmp_path):
    g = np.load(GOLD)
    n_gen = 16
    seq = np.concatenate([g["prompt"], g["generated"][:n_gen]])
    write_model_dir(str(tmp_path), hf_config(TINY), list(tiny_tensors()), n_shards=3)
    with dsb.Checkpoint(str(tmp_path)) as ck:
        m = dsb.Model(gpu_ctx, ck.config())
        up, skip = m.upload_checkpoint(ck)
        assert (up, skip) == (len(ck) - N_EXTRAS, N_EXTRAS)
    m.finalize()
    ref = dsb.Model(gpu_ctx, dsb.ModelConfig(**TINY))
    for name, a in model_tensors(TINY, seed=0).items():
        ref.set_tensor(name, a)
    ref.finalize()
    ids_c, lg_c = decode(gpu_ctx, m, seq)
    ids_r, lg_r = decode(gpu_ctx, ref, seq)
    m.close()
    ref.close()
    assert np.array_equal(lg_c.view(np.uint32), lg_r.view(np.uint32))
    assert np.array_equal(ids_c, ids_r)
    p = len(g["prompt"])
    assert ids_c[p - 1:p - 1 + n_gen].tolist() == g["generated"][:n_gen].tolist()


def test_fp8_checkpoint_decodes_like_set_tensor(gpu_ctx, tmp_path):
    from fp8_tiny import build

    g = np.load(GOLD)
    seq = g["prompt"][:24]
    write_model_dir(str(tmp_path), hf_config(TINY, fp8=True), list(tiny_tensors(fp8=True)), n_shards=2)
    m = dsb.load_model(gpu_ctx, str(tmp_path))
    ref = build(gpu_ctx, fp8=True)
    ids_c, lg_c = decode(gpu_ctx, m, seq)
    ids_r, lg_r = decode(gpu_ctx, ref, seq)
    m.close()
    ref.close()
    assert np.isfinite(lg_c).all()
    assert np.array_equal(lg_c.view(np.uint32), lg_r.view(np.uint32))
    assert np.array_equal(ids_c, ids_r)


@pytest.mark.parametrize("case", ["unknown_name", "unsupported_dtype", "wrong_shape"])
def test_upload_rejects_tensors_the_model_cannot_take(gpu_ctx, tmp_path, case):
    base = [t for t in tiny_tensors(extras=False)]
    if case == "unknown_name":
        extra = ("model.layers.0.mlp.foo.weight", "BF16", np.zeros((4, 4), np.uint16))
        code, text = dsb.DSB_EINVAL, "model.layers.0.mlp.foo.weight"
    elif case == "unsupported_dtype":
        extra = ("model.layers.1.mlp.gate.e_score_correction_bias", "I64", np.zeros(16, np.int64))
        code, text = dsb.DSB_EUNSUPPORTED, "I64"
    else:
        base = [t for t in base if t[0] != "model.norm.weight"]
        extra = ("model.norm.weight", "BF16", bf16_bits(np.ones(TINY["hidden_size"] + 1, np.float32)))
        code, text = dsb.DSB_EINVAL, "model.norm.weight"
    write_model_dir(str(tmp_path), hf_config(TINY), sorted(base + [extra], key=lambda t: t[0]), n_shards=1)
    with pytest.raises(dsb.DsbError) as e:
        dsb.load_model(gpu_ctx, str(tmp_path))
    assert e.value.code == code and text in str(e.value), str(e.value)
