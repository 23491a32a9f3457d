"""Block-scaled FP8 (e4m3) quantisation and grouped linear through the C ABI.

Quantisation (dsb_quant_act_1x128, dsb_quant_weight_128x128) is byte work:
bit-exact against the oracle's restatement (orc_quant_act_1x128,
orc_quant_weight_128x128), codes and scales.

The linear (dsb_linear_fp8) is compared with the oracle's orc_fp8_linear
(double accumulation of the dequantised operands) on small shapes, and with a
float64 torch product of the same dequantised operands at larger ones.
Tolerance: max|y - ref| <= 2e-3 * max|ref| for fp32 outputs (each 128-deep K
block is summed by the tensor cores before the fp32 promotion), 1e-2 for bf16
outputs.
"""

import numpy as np
import pytest

import oracle as O
import deepseek_cpp_infer_b200 as dsb

pytestmark = pytest.mark.gpu
TOL32, TOL16 = 2e-3, 1e-2


def e4m3_lut():
    import torch

    return torch.tensor([O.oracle().orc_e4m3_to_f32(c) for c in range(256)], dtype=torch.float64, device="cuda")


def max_rel(a, ref):
    a, ref = a.double(), ref.double()
    return float((a - ref).abs().max() / ref.abs().max())


def quant_w(ctx, w):
    """bf16/fp32 [M, K] device -> (uint8 [M, K], fp32 [ceil(M/128), ceil(K/128)])."""
    import torch

    M, K = w.shape
    q = torch.empty(M, K, dtype=torch.uint8, device="cuda")
    s = torch.empty((M + 127) // 128, (K + 127) // 128, dtype=torch.float32, device="cuda")
    ctx.quant_weight(w, q, s)
    return q, s


def quant_x(ctx, x):
    import torch

    T, K = x.shape
    q = torch.empty(T, K, dtype=torch.uint8, device="cuda")
    s = torch.empty(T, K // 128, dtype=torch.float32, device="cuda")
    ctx.quant_act(x, q, s)
    return q, s


def deq_w(lut, q, s):
    M, K = q.shape
    sw = s.double().repeat_interleave(128, 0)[:M].repeat_interleave(128, 1)[:, :K]
    return lut[q.long()] * sw


def deq_x(lut, q, s):
    return lut[q.long()] * s.double().repeat_interleave(128, 1)


def normal(*shape, scale=1.0, seed=0, dtype=None):
    import torch

    g = torch.Generator(device="cuda").manual_seed(seed)
    x = torch.randn(*shape, generator=g, device="cuda") * scale
    return x if dtype is None else x.to(dtype)


@pytest.mark.parametrize("dtype", ["bf16", "f32"])
def test_quant_act_matches_oracle_bitwise(gpu_ctx, dtype):
    import torch

    T, K = 37, 512
    x = normal(T, K, scale=3.0, seed=1)
    x[3, 128:256] = 0.0           # all-zero group: scale 1
    x[5, 7] = 1e4                 # one large outlier in a group
    x[6, :128] = 1e-30            # tiny values (subnormal codes)
    x = x.to(torch.bfloat16 if dtype == "bf16" else torch.float32)
    q, s = quant_x(gpu_ctx, x)
    torch.cuda.synchronize()
    xf = np.ascontiguousarray(x.float().cpu().numpy())
    rq = np.zeros((T, K), np.uint8)
    rs = np.zeros((T, K // 128), np.float32)
    O.oracle().orc_quant_act_1x128(O.p(xf, O.f32p), T, K, O.p(rq, O.u8p), O.p(rs, O.f32p))
    assert np.array_equal(q.cpu().numpy(), rq)
    assert np.array_equal(s.cpu().numpy().view(np.uint32), rs.view(np.uint32))


def test_quant_act_gathers_permuted_rows(gpu_ctx):
    import torch

    T, K, k = 9, 256, 3
    x = normal(T, K, seed=2, dtype=torch.bfloat16)
    src = torch.tensor(np.random.default_rng(0).permutation(T * k), dtype=torch.int32, device="cuda")
    q = torch.empty(T * k, K, dtype=torch.uint8, device="cuda")
    s = torch.empty(T * k, K // 128, dtype=torch.float32, device="cuda")
    gpu_ctx.quant_act(x, q, s, src_rows=src, k=k)
    q0, s0 = quant_x(gpu_ctx, x)
    rows = (src // k).long()
    assert torch.equal(q, q0[rows]) and torch.equal(s, s0[rows])


def test_quant_weight_matches_oracle_bitwise(gpu_ctx):
    import torch

    M, K = 300, 384  # ragged last row block
    w = normal(M, K, scale=0.02, seed=3)
    w[128:256, 0:128] = 0.0
    q, s = quant_w(gpu_ctx, w)
    torch.cuda.synchronize()
    wf = np.ascontiguousarray(w.cpu().numpy())
    rq = np.zeros((M, K), np.uint8)
    rs = np.zeros(((M + 127) // 128, (K + 127) // 128), np.float32)
    O.oracle().orc_quant_weight_128x128(O.p(wf, O.f32p), M, K, O.p(rq, O.u8p), O.p(rs, O.f32p))
    assert np.array_equal(q.cpu().numpy(), rq)
    assert np.array_equal(s.cpu().numpy().view(np.uint32), rs.view(np.uint32))


def test_linear_fp8_matches_oracle(gpu_ctx):
    import torch

    M, K, T = 256, 512, 5
    wq, ws = quant_w(gpu_ctx, normal(M, K, scale=0.05, seed=4))
    xq, xs = quant_x(gpu_ctx, normal(T, K, seed=5))
    y = torch.empty(T, M, dtype=torch.float32, device="cuda")
    gpu_ctx.linear_fp8(wq, ws, xq, xs, y, M=M, K=K)
    gpu_ctx.sync()
    ref = np.zeros((T, M), np.float32)
    a = [np.ascontiguousarray(t.cpu().numpy()) for t in (wq, ws, xq, xs)]
    O.oracle().orc_fp8_linear(O.p(a[0], O.u8p), O.p(a[1], O.f32p), O.p(a[2], O.u8p), O.p(a[3], O.f32p), T, M, K,
                              O.p(ref, O.f32p))
    assert np.abs(y.cpu().numpy() - ref).max() <= TOL32 * np.abs(ref).max()


@pytest.mark.parametrize("T", [1, 16, 33, 100, 128, 200, 300])
@pytest.mark.parametrize("M,K", [(576, 7168), (2048, 1536)])
def test_linear_fp8_plain(gpu_ctx, T, M, K):
    import torch

    lut = e4m3_lut()
    wq, ws = quant_w(gpu_ctx, normal(M, K, scale=0.02, seed=6))
    xq, xs = quant_x(gpu_ctx, normal(T, K, seed=7, dtype=torch.bfloat16))
    ref = deq_x(lut, xq, xs) @ deq_w(lut, wq, ws).T
    y = torch.empty(T, M, dtype=torch.float32, device="cuda")
    gpu_ctx.linear_fp8(wq, ws, xq, xs, y, M=M, K=K)
    gpu_ctx.sync()
    assert max_rel(y, ref) <= TOL32, max_rel(y, ref)
    yb = torch.empty(T, M, dtype=torch.bfloat16, device="cuda")
    gpu_ctx.linear_fp8(wq, ws, xq, xs, yb, M=M, K=K)
    gpu_ctx.sync()
    assert max_rel(yb, ref) <= TOL16


@pytest.mark.parametrize("M", [200, 300])
@pytest.mark.parametrize("T", [7, 33, 90])
def test_linear_fp8_partial_tile_and_unaligned_output(gpu_ctx, T, M):
    """M = 200 ends inside a 128-row tile on a 16-byte boundary (vector
    output, clipped per warp); M = 300 leaves rows that are not a whole
    vector (element-wise output).  Store to f32 / bf16 and residual add."""
    import torch

    lut = e4m3_lut()
    K = 512
    wq, ws = quant_w(gpu_ctx, normal(M, K, scale=0.05, seed=41))
    xq, xs = quant_x(gpu_ctx, normal(T, K, seed=42, dtype=torch.bfloat16))
    ref = deq_x(lut, xq, xs) @ deq_w(lut, wq, ws).T
    y = torch.full((T, M), float("nan"), dtype=torch.float32, device="cuda")
    gpu_ctx.linear_fp8(wq, ws, xq, xs, y, M=M, K=K)
    yb = torch.full((T, M), float("nan"), dtype=torch.bfloat16, device="cuda")
    gpu_ctx.linear_fp8(wq, ws, xq, xs, yb, M=M, K=K)
    h = normal(T, M, seed=43)
    h0 = h.clone()
    gpu_ctx.linear_fp8(wq, ws, xq, xs, h, M=M, K=K, epilogue=dsb.EPI_ADD)
    gpu_ctx.sync()
    assert max_rel(y, ref) <= TOL32
    assert max_rel(yb, ref) <= TOL16
    assert max_rel(h, h0.double() + ref) <= TOL32


def test_linear_fp8_residual_add_split_k(gpu_ctx):
    import torch

    lut = e4m3_lut()
    M, K, T = 2048, 2048, 8
    wq, ws = quant_w(gpu_ctx, normal(M, K, scale=0.02, seed=8))
    xq, xs = quant_x(gpu_ctx, normal(T, K, seed=9))
    h = normal(T, M, seed=10)
    ref = h.double() + deq_x(lut, xq, xs) @ deq_w(lut, wq, ws).T
    gpu_ctx.linear_fp8(wq, ws, xq, xs, h, M=M, K=K, epilogue=dsb.EPI_ADD)
    gpu_ctx.sync()
    assert max_rel(h, ref) <= TOL32


def test_linear_fp8_grouped_experts_rowscale(gpu_ctx):
    import torch

    lut = e4m3_lut()
    E, M, K = 8, 256, 1024
    counts = [3, 0, 17, 1, 0, 140, 2, 300]
    offs = np.concatenate([[0], np.cumsum(counts)]).astype(np.int32)
    T = int(offs[-1])
    wq, ws = zip(*(quant_w(gpu_ctx, normal(M, K, scale=0.05, seed=20 + e)) for e in range(E)))
    wq, ws = torch.cat(wq), torch.cat(ws)  # [E*M, K], [E*M/128, K/128]
    xq, xs = quant_x(gpu_ctx, normal(T, K, seed=11, dtype=torch.bfloat16))
    scale = torch.rand(T, device="cuda")
    y = torch.full((T, M), float("nan"), dtype=torch.float32, device="cuda")
    gpu_ctx.linear_fp8(wq, ws, xq, xs, y, M=M, K=K, G=E, tok_offsets=torch.from_numpy(offs).cuda(),
                       max_tokens_per_group=max(counts), epilogue=dsb.EPI_ROWSCALE, row_scale=scale)
    gpu_ctx.sync()
    ref = torch.zeros(T, M, dtype=torch.float64, device="cuda")
    xd = deq_x(lut, xq, xs)
    for e in range(E):
        a, b = offs[e], offs[e + 1]
        if b > a:
            wd = deq_w(lut, wq[e * M:(e + 1) * M], ws[e * M // 128:(e + 1) * M // 128])
            ref[a:b] = (xd[a:b] @ wd.T) * scale[a:b, None].double()
    assert torch.isfinite(y).all()
    assert max_rel(y, ref) <= TOL32


@pytest.mark.parametrize("T", [4, 64, 200])
def test_linear_fp8_silu_gate_interleaved(gpu_ctx, T):
    """gate and up quantised as separate checkpoint matrices, rows interleaved
    (2f gate, 2f+1 up) with scale_rows 2."""
    import torch

    lut = e4m3_lut()
    I, K = 512, 1024
    gq, gs = quant_w(gpu_ctx, normal(I, K, scale=0.02, seed=12))
    uq, us = quant_w(gpu_ctx, normal(I, K, scale=0.03, seed=13))
    w = torch.stack([gq, uq], 1).reshape(2 * I, K).contiguous()
    tiles = 2 * I // 128
    # tile j holds gate/up rows 64j..64j+63, i.e. scale row (64j)//128 of each
    rows = torch.arange(tiles, device="cuda") * 64 // 128
    sc = torch.stack([gs[rows], us[rows]], 1).reshape(tiles * 2, K // 128).contiguous()
    xq, xs = quant_x(gpu_ctx, normal(T, K, seed=14, dtype=torch.bfloat16))
    y = torch.empty(T, I, dtype=torch.float32, device="cuda")
    gpu_ctx.linear_fp8(w, sc, xq, xs, y, M=2 * I, K=K, scale_rows=2, epilogue=dsb.EPI_SILU_GATE)
    gpu_ctx.sync()
    xd = deq_x(lut, xq, xs)
    g = xd @ deq_w(lut, gq, gs).T
    u = xd @ deq_w(lut, uq, us).T
    ref = g / (1 + torch.exp(-g)) * u
    assert max_rel(y, ref) <= TOL32


def test_linear_fp8_rejects_bad_shapes(gpu_ctx):
    import torch

    wq = torch.zeros(128, 192, dtype=torch.uint8, device="cuda")
    ws = torch.ones(1, 2, device="cuda")
    xq = torch.zeros(4, 192, dtype=torch.uint8, device="cuda")
    xs = torch.ones(4, 2, device="cuda")
    y = torch.empty(4, 128, device="cuda")
    with pytest.raises(dsb.DsbError) as e:
        gpu_ctx.linear_fp8(wq, ws, xq, xs, y, M=128, K=192)
    assert e.value.code == dsb.DSB_EINVAL
