"""Absorbed MLA decode on the GPU (dsb_mla_decode through the C ABI) against
the CPU oracle (orc_mla_decode_paged, pinned to the reference's
mla_decode_step by tests/test_oracle.py).

Tolerance: the layer-output bar of max-rel <= 2e-2, where
max-rel = max|gpu - oracle| / max|oracle|.  The kernel quantises the softmax
probabilities to bf16 before the P.V contraction and rounds the output to
bf16, which typically gives max-rel ~ 5e-3.
"""

import numpy as np
import pytest

import oracle as O
from deepseek_cpp_infer_b200 import DSB_EINVAL, DSB_EUNSUPPORTED, DsbError
from deepseek_cpp_infer_b200.workloads import mla_case, to_u16

pytestmark = pytest.mark.gpu
TOL = 2e-2


def run_gpu(ctx, case):
    import torch

    out = torch.empty(case.B, case.H, case.R, dtype=torch.bfloat16, device="cuda")
    ctx.mla_decode(case.q_lat, case.q_rope, case.cache, case.block_table, case.seq_lens, case.scale, out)
    ctx.sync()
    return out


def oracle_out(case, rows=None):
    rows = list(range(case.B)) if rows is None else rows
    return O.mla_decode_paged(
        to_u16(case.q_lat)[rows], to_u16(case.q_rope)[rows], to_u16(case.cache), case.block_table_host[rows],
        case.seq_lens[rows], case.scale)


def max_rel(gpu, ref):
    return float(np.abs(gpu - ref).max() / np.abs(ref).max())


def check(ctx, case, rows=None):
    import torch

    out = run_gpu(ctx, case).float().cpu().numpy()
    rows = list(range(case.B)) if rows is None else rows
    ref = oracle_out(case, rows)
    got = out[rows]
    assert np.isfinite(got).all()
    err = max_rel(got, ref)
    assert err <= TOL, err
    return out, err


@pytest.mark.parametrize("lens", [[1, 63, 64, 65, 777, 2048], [8192, 5, 130]])
def test_mla_v3_shape_ragged_lengths(gpu_ctx, lens):
    case = mla_case(H=128, R=512, P=64, lens=lens, seed=7)
    _, err = check(gpu_ctx, case)
    print("max-rel", err)


def test_mla_v2_lite_heads(gpu_ctx):
    case = mla_case(H=16, R=512, P=64, lens=[300, 1, 1024, 4097], seed=8)
    check(gpu_ctx, case)


def test_mla_small_rank(gpu_ctx):
    # tiny config: kv_lora_rank 128, rope 32, 8 heads, nope 64
    case = mla_case(H=8, R=128, P=32, lens=[1, 40, 64, 65, 500], seed=9, nope=64)
    check(gpu_ctx, case)


def test_mla_split_kv_long_sequences(gpu_ctx):
    # long sequences are split into several work items and merged
    case = mla_case(H=128, R=512, P=64, lens=[16384, 9000, 12], seed=10)
    gpu_ctx.reset_stats()
    check(gpu_ctx, case)
    assert gpu_ctx.stats()["mla_partials"] > 0


def test_mla_cfg2_full_size(gpu_ctx):
    """B=64, H=128, ctx U[1024, 8192], random block table: parity on the
    shortest and longest sequence; size-independent properties on all 64."""
    import torch

    case = mla_case(seed=1)
    out = run_gpu(gpu_ctx, case)
    o = out.float().cpu().numpy()
    assert np.isfinite(o).all()
    # convexity: every output is a convex combination of cache rows
    cmax = float(case.cache.float().abs().max())
    assert np.abs(o).max() <= cmax * 1.01
    rows = [int(np.argmin(case.seq_lens)), int(np.argmax(case.seq_lens))]
    err = max_rel(o[rows], oracle_out(case, rows))
    assert err <= TOL, err
    # moving every page to another physical block leaves the result bit-identical
    n_blocks = case.cache.shape[0]
    perm = torch.randperm(n_blocks, generator=torch.Generator().manual_seed(3))
    cache2 = torch.empty_like(case.cache)
    cache2[perm.cuda()] = case.cache
    bt2 = perm[case.block_table.long().cpu()].to(torch.int32)
    # unused table slots (beyond a sequence's pages) are never read
    case2 = type(case)(case.q_lat, case.q_rope, cache2, bt2.cuda(), bt2.numpy(), case.seq_lens, case.scale,
                       case.B, case.H, case.R, case.P)
    out2 = run_gpu(gpu_ctx, case2)
    assert torch.equal(out.view(torch.int16), out2.view(torch.int16))
    # repeat call gives the same bits (deterministic reduction order)
    out3 = run_gpu(gpu_ctx, case)
    assert torch.equal(out.view(torch.int16), out3.view(torch.int16))


def test_mla_rejects_unsupported(gpu_ctx):
    import torch

    case = mla_case(H=16, R=512, P=64, lens=[64], seed=2)
    out = torch.empty(1, 16, 512, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(DsbError) as e:
        gpu_ctx.mla_decode(case.q_lat, case.q_rope, case.cache, case.block_table, [0], case.scale, out)
    assert e.value.code == DSB_EINVAL
    with pytest.raises(DsbError) as e:
        gpu_ctx.mla_decode(case.q_lat, case.q_rope, case.cache, case.block_table, [64], case.scale, out,
                           block_size=32)
    assert e.value.code == DSB_EUNSUPPORTED


def _oracle_rows_worker(args):
    """Oracle attention of a few sequences (their pages gathered into a compact cache)."""
    import oracle as O

    q_lat, q_rope, cache, bt, lens, scale = args
    return O.mla_decode_paged(q_lat, q_rope, cache, bt, lens, scale)


def test_mla_cfg2_all_rows_against_oracle(gpu_ctx):
    """The benchmark configuration (B=64, H=128, R=512, P=64, ctx U[1024,
    8192], seed 1) with every one of its 64 rows against
    orc_mla_decode_paged, the sequences spread over a spawn pool of host
    processes (each gets only its sequences' pages)."""
    import multiprocessing as mp
    import os

    case = mla_case(seed=1)
    o = run_gpu(gpu_ctx, case).float().cpu().numpy()
    cache = to_u16(case.cache)
    ql, qr = to_u16(case.q_lat), to_u16(case.q_rope)
    workers = max(1, min(32, os.cpu_count() or 1))
    groups = [list(range(case.B))[i::workers] for i in range(workers)]
    jobs = []
    for rows in groups:
        if not rows:
            continue
        pages = [case.block_table_host[b, : (case.seq_lens[b] + 63) // 64] for b in rows]
        bt = np.zeros((len(rows), max(len(p) for p in pages)), np.int32)
        k = 0
        for i, p in enumerate(pages):
            bt[i, : len(p)] = np.arange(k, k + len(p))
            k += len(p)
        jobs.append((ql[rows], qr[rows], cache[np.concatenate(pages)], bt, case.seq_lens[rows], case.scale))
    with mp.get_context("spawn").Pool(len(jobs)) as pool:
        refs = pool.map(_oracle_rows_worker, jobs)
    ref = np.zeros_like(o)
    for rows, r in zip([g for g in groups if g], refs):
        ref[rows] = r
    errs = np.abs(o - ref).max(axis=(1, 2)) / np.abs(ref).max(axis=(1, 2))
    print("cfg2 per-row max-rel: median %.2e worst %.2e" % (np.median(errs), errs.max()))
    assert errs.max() <= TOL, errs


def test_mla_small_rank_storage_points(gpu_ctx):
    """kv_lora_rank 128 (one CTA per work item, fp32 scores): the kernel
    against oracle.model.mla_decode_storage_points, which rounds where the
    kernel stores (bf16 probabilities relative to the lazily raised running
    maximum, bf16 output, split items merged by their maxima) and plans the
    same work items.  Only fp32 summation order and the hardware exp2 differ,
    so nearly every output value is the same bf16 number."""
    import torch

    import oracle.model as OM

    slots = torch.cuda.get_device_properties(0).multi_processor_count
    case = mla_case(H=8, R=128, P=32, lens=[1, 40, 64, 65, 500, 3000, 130, 9000], seed=19, nope=64)
    plan = gpu_ctx.mla_plan(case.seq_lens, 8, 128, 32)
    try:
        info = plan.info()
    finally:
        plan.close()
    items = OM._mla_items(case.seq_lens, slots, 8, 128, 32)
    assert info["n_items"] == len(items)
    assert info["n_partial"] == sum(1 for it in items if it[4])
    out = run_gpu(gpu_ctx, case).float().cpu().numpy()
    ref = OM.mla_decode_storage_points(case.q_lat.float().cpu().numpy(), case.q_rope.float().cpu().numpy(),
                                       case.cache.float().cpu().numpy(), case.block_table_host, case.seq_lens,
                                       case.scale, slots)
    same = float((out == ref).mean())
    err = max_rel(out, ref)
    print(f"storage-point oracle: {same * 100:.3f}% identical bf16 values, max-rel {err:.2e}")
    assert same >= 0.995 and err <= 1e-2, (same, err)
