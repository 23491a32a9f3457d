"""dsb_mla_decode_noalloc through the C ABI.

The allocation-free entry point is for callers that cannot allocate device
memory on the call path: runtimes whose own allocator owns every byte of
device memory (a stray cudaMalloc/cudaFree breaks their accounting, and a
cudaFree synchronises the whole device) and plug-in hosts that hand over only
a stream and their buffers.  Its scratch is a fixed device array inside
libdsb.so.

Two calls in a row with different inputs must each match the context-based
entry point, dsb_mla_decode, and the CPU oracle within the MLA tolerance
(max-rel <= 2e-2), so the second call is not disturbed by what the first left
in the shared scratch; the status read-back reports a clean run.  The
fallback plan (one item per 16384 tokens) and the partial-count limit are
checked at their boundary.  This file is collected last; it also passes on
its own.
"""

import numpy as np
import pytest

import deepseek_cpp_infer_b200 as dsb
import oracle as O
from deepseek_cpp_infer_b200.workloads import mla_case, to_u16

pytestmark = pytest.mark.gpu
TOL = 2e-2


def max_rel(a, b):
    a, b = a.float(), b.float()
    return float((a - b).abs().max() / b.abs().max())


def oracle_rel(out, case, rows=None):
    rows = list(range(case.B)) if rows is None else rows
    ref = O.mla_decode_paged(to_u16(case.q_lat[rows]), to_u16(case.q_rope[rows]), to_u16(case.cache),
                             case.block_table_host[rows], case.seq_lens[rows], case.scale)
    got = out[rows].float().cpu().numpy()
    return float(np.abs(got - ref).max() / np.abs(ref).max())


def run_both(ctx, case):
    import torch

    ref = torch.empty(case.B, case.H, case.R, dtype=torch.bfloat16, device="cuda")
    ctx.mla_decode(case.q_lat, case.q_rope, case.cache, case.block_table, case.seq_lens, case.scale, ref)
    ctx.sync()
    stream = torch.cuda.Stream()
    out = torch.full_like(ref, float("nan"))
    stream.wait_stream(torch.cuda.current_stream())  # inputs and `out` were written on the default stream
    rc = dsb.mla_decode_noalloc(stream.cuda_stream, case.q_lat, case.q_rope, case.cache, case.block_table,
                                case.seq_lens, case.scale, out)
    assert rc == dsb.DSB_OK, rc
    assert dsb.mla_noalloc_status(stream.cuda_stream) == dsb.DSB_OK  # waits for the stream
    return out, ref


def test_noalloc_matches_mla_decode_and_oracle_twice(gpu_ctx):
    import torch

    # first call: long sequences that are split into partials
    c1 = mla_case(H=128, R=512, P=64, lens=[16384, 9000, 12, 3000], seed=21)
    out1, ref1 = run_both(gpu_ctx, c1)
    assert torch.isfinite(out1.float()).all()
    assert max_rel(out1, ref1) <= TOL
    assert oracle_rel(out1, c1) <= TOL
    # second call right after, different shapes and lengths, same scratch
    c2 = mla_case(H=16, R=512, P=64, lens=[1, 64, 65, 700, 2049], seed=22)
    out2, ref2 = run_both(gpu_ctx, c2)
    assert torch.isfinite(out2.float()).all()
    assert max_rel(out2, ref2) <= TOL
    assert oracle_rel(out2, c2) <= TOL


def test_noalloc_small_rank_and_fallback_plan(gpu_ctx):
    c = mla_case(H=8, R=128, P=32, lens=[40, 500, 1], seed=23, nope=64)
    out, ref = run_both(gpu_ctx, c)
    assert max_rel(out, ref) <= TOL
    assert oracle_rel(out, c) <= TOL
    # the usual plan splits these four 8192-token sequences into more partials
    # than the fixed scratch holds; the fallback (one item per sequence) fits
    lens = [8192] * 4
    plan = gpu_ctx.mla_plan(lens, H=8, R=128, P=32)
    try:
        n_partial = plan.info()["n_partial"]
    finally:
        plan.close()
    assert n_partial > 24, n_partial
    big = mla_case(H=8, R=128, P=32, lens=lens, seed=25, nope=64)
    out, ref = run_both(gpu_ctx, big)
    assert max_rel(out, ref) <= TOL
    assert oracle_rel(out, big) <= TOL


def test_noalloc_partial_limit_boundary(gpu_ctx):
    import torch

    # 17000 tokens = 266 pages -> 2 items, 2 partials each in the fallback plan:
    # 12 sequences need 24 partials (the limit), 13 need 26
    ok = mla_case(H=16, R=512, P=64, lens=[17000] * 12, seed=24)
    out, ref = run_both(gpu_ctx, ok)
    assert max_rel(out, ref) <= TOL
    assert oracle_rel(out, ok, rows=[0, 11]) <= TOL
    del ok, out, ref
    over = mla_case(H=16, R=512, P=64, lens=[17000] * 13, seed=26)
    o = torch.full((13, 16, 512), float("nan"), dtype=torch.bfloat16, device="cuda")
    rc = dsb.mla_decode_noalloc(0, over.q_lat, over.q_rope, over.cache, over.block_table, over.seq_lens,
                                over.scale, o)
    assert rc == dsb.DSB_ELIMIT
    torch.cuda.synchronize()
    assert torch.isnan(o.float()).all()  # nothing was enqueued
