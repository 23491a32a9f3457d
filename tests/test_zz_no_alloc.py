"""dsb_mla_decode_noalloc through the C ABI against dsb_mla_decode.

The allocation-free entry point is for callers that cannot allocate device
memory on the call path (graph capture, runtimes that own all device memory,
plug-in hosts handing over only a stream and buffers); its scratch is a fixed
device array inside libdsb.so.  Two calls in a row with different inputs must
each match the context-based entry point within the MLA tolerance (max-rel
<= 2e-2), so the second call is not disturbed by what the first left in the
shared scratch.  This file is collected last; it also passes on its own.
"""

import numpy as np
import pytest

import deepseek_cpp_infer_b200 as dsb
from deepseek_cpp_infer_b200.workloads import mla_case

pytestmark = pytest.mark.gpu
TOL = 2e-2


def max_rel(a, b):
    a, b = a.float(), b.float()
    return float((a - b).abs().max() / b.abs().max())


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
    stream.synchronize()
    return out, ref


def test_noalloc_matches_mla_decode_twice(gpu_ctx):
    import torch

    # first call: long sequences that are split into partials
    c1 = mla_case(H=128, R=512, P=64, lens=[16384, 9000, 12, 3000], seed=21)
    out1, ref1 = run_both(gpu_ctx, c1)
    assert torch.isfinite(out1.float()).all()
    assert max_rel(out1, ref1) <= TOL
    # second call right after, different shapes and lengths, same scratch
    c2 = mla_case(H=16, R=512, P=64, lens=[1, 64, 65, 700, 2049], seed=22)
    out2, ref2 = run_both(gpu_ctx, c2)
    assert torch.isfinite(out2.float()).all()
    assert max_rel(out2, ref2) <= TOL


def test_noalloc_small_rank_and_limit(gpu_ctx):
    import torch

    c = mla_case(H=8, R=128, P=32, lens=[40, 500, 1], seed=23, nope=64)
    out, ref = run_both(gpu_ctx, c)
    assert max_rel(out, ref) <= TOL
    # more long sequences than the fixed scratch holds partials for: rejected, nothing enqueued
    lens = [17000] * 25
    big = mla_case(B=25, H=16, R=512, P=64, lens=lens, seed=24)
    o = torch.empty(25, 16, 512, dtype=torch.bfloat16, device="cuda")
    rc = dsb.mla_decode_noalloc(0, big.q_lat, big.q_rope, big.cache, big.block_table, big.seq_lens, big.scale, o)
    assert rc == dsb.DSB_ELIMIT
