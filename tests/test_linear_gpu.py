"""Grouped bf16 linear (dsb_linear through the C ABI) against a plain PyTorch
fp32 reference of the same op on the same bf16 inputs, plus one case against
the oracle's ds::rt::linear restatement (orc_linear_f32).

Tolerance: fp32 accumulation of bf16 products in a different order, then a
bf16 (or fp32) store: max-rel <= 1e-2 for bf16 outputs, 1e-4 for fp32.
"""

import numpy as np
import pytest

import oracle as O
import deepseek_cpp_infer_b200 as dsb

pytestmark = pytest.mark.gpu


def rand(*shape, scale=1.0, seed=0):
    import torch

    g = torch.Generator(device="cuda").manual_seed(seed)
    return (torch.randn(*shape, generator=g, device="cuda") * scale).to(torch.bfloat16)


def max_rel(a, b):
    a, b = a.float(), b.float()
    return float((a - b).abs().max() / b.abs().max())


@pytest.mark.parametrize("T", [1, 5, 32, 100, 256, 300])
@pytest.mark.parametrize("M,K", [(576, 2048), (2048, 1408)])
def test_linear_plain(gpu_ctx, T, M, K):
    import torch

    w = rand(M, K, scale=0.02, seed=1)
    x = rand(T, K, seed=2)
    y = torch.empty(T, M, dtype=torch.float32, device="cuda")
    gpu_ctx.linear(w, x, y, M=M, K=K)
    gpu_ctx.sync()
    ref = x.float() @ w.float().T
    assert max_rel(y, ref) <= 1e-4
    yb = torch.empty(T, M, dtype=torch.bfloat16, device="cuda")
    gpu_ctx.linear(w, x, yb, M=M, K=K)
    gpu_ctx.sync()
    assert max_rel(yb, ref) <= 1e-2


def test_linear_matches_oracle_linear(gpu_ctx):
    import torch

    M, K, T = 256, 512, 3
    w = rand(M, K, scale=0.05, seed=3)
    x = rand(T, K, seed=4)
    y = torch.empty(T, M, dtype=torch.float32, device="cuda")
    gpu_ctx.linear(w, x, y, M=M, K=K)
    gpu_ctx.sync()
    wf = np.ascontiguousarray(w.float().cpu().numpy())
    for t in range(T):
        ref = np.zeros(M, np.float32)
        xt = np.ascontiguousarray(x[t].float().cpu().numpy())
        O.oracle().orc_linear_f32(O.p(wf, O.f32p), O.p(xt, O.f32p), K, O.p(ref, O.f32p), M)
        assert np.abs(y[t].cpu().numpy() - ref).max() <= 1e-4 * np.abs(ref).max()


def test_linear_residual_add(gpu_ctx):
    import torch

    M, K, T = 2048, 2048, 32
    w = rand(M, K, scale=0.02, seed=5)
    x = rand(T, K, seed=6)
    h = torch.randn(T, M, device="cuda")
    h0 = h.clone()
    gpu_ctx.linear(w, x, h, M=M, K=K, epilogue=dsb.EPI_ADD)
    gpu_ctx.sync()
    ref = h0 + x.float() @ w.float().T
    assert max_rel(h, ref) <= 1e-4


@pytest.mark.parametrize("M", [200, 300])
@pytest.mark.parametrize("T", [7, 33])
def test_linear_partial_tile_and_unaligned_output(gpu_ctx, T, M):
    """M = 200 ends inside a 128-row tile on a 16-byte boundary (vector
    output, clipped per warp); M = 300 leaves rows that are not a whole
    vector (element-wise output).  Store to f32 / bf16 and residual add."""
    import torch

    K = 512
    w = rand(M, K, scale=0.05, seed=31)
    x = rand(T, K, seed=32)
    ref = x.float() @ w.float().T
    y = torch.full((T, M), float("nan"), dtype=torch.float32, device="cuda")
    gpu_ctx.linear(w, x, y, M=M, K=K)
    yb = torch.full((T, M), float("nan"), dtype=torch.bfloat16, device="cuda")
    gpu_ctx.linear(w, x, yb, M=M, K=K)
    h = torch.randn(T, M, device="cuda")
    h0 = h.clone()
    gpu_ctx.linear(w, x, h, M=M, K=K, epilogue=dsb.EPI_ADD)
    gpu_ctx.sync()
    assert max_rel(y, ref) <= 1e-4
    assert max_rel(yb, ref) <= 1e-2
    assert max_rel(h, h0 + ref) <= 1e-4


@pytest.mark.parametrize("T", [1, 32, 200])
def test_linear_silu_gate(gpu_ctx, T):
    import torch

    I, K = 1408, 2048
    wg = rand(I, K, scale=0.02, seed=7)
    wu = rand(I, K, scale=0.02, seed=8)
    # rows interleaved: row 2f = gate row f, row 2f+1 = up row f
    w = torch.stack([wg, wu], 1).reshape(2 * I, K).contiguous()
    x = rand(T, K, seed=9)
    y = torch.empty(T, I, dtype=torch.bfloat16, device="cuda")
    gpu_ctx.linear(w, x, y, M=2 * I, K=K, epilogue=dsb.EPI_SILU_GATE)
    gpu_ctx.sync()
    g = x.float() @ wg.float().T
    u = x.float() @ wu.float().T
    ref = g / (1 + torch.exp(-g)) * u
    assert max_rel(y, ref) <= 1e-2


def test_linear_grouped_experts_rowscale(gpu_ctx):
    import torch

    E, M, K = 8, 256, 512
    counts = [3, 0, 17, 1, 0, 40, 2, 9]
    offs = np.concatenate([[0], np.cumsum(counts)]).astype(np.int32)
    T = int(offs[-1])
    w = rand(E * M, K, scale=0.05, seed=10)
    x = rand(T, K, seed=11)
    scale = torch.rand(T, device="cuda")
    y = torch.full((T, M), float("nan"), dtype=torch.float32, device="cuda")
    gpu_ctx.linear(w, x, y, M=M, K=K, G=E, tok_offsets=torch.from_numpy(offs).cuda(),
                   max_tokens_per_group=max(counts), epilogue=dsb.EPI_ROWSCALE, row_scale=scale)
    gpu_ctx.sync()
    ref = torch.empty(T, M, device="cuda")
    for e in range(E):
        a, b = offs[e], offs[e + 1]
        if b > a:
            ref[a:b] = (x[a:b].float() @ w[e * M:(e + 1) * M].float().T) * scale[a:b, None]
    assert torch.isfinite(y).all()
    assert max_rel(y, ref) <= 1e-4


def test_linear_per_head_groups(gpu_ctx):
    """Absorbed q projection shape: per head h, q_lat[:, h] = W_UK[h]^T q_nope[:, h]."""
    import torch

    H, nope, rope, R, B = 16, 128, 64, 512, 32
    q = rand(B, H * (nope + rope), seed=12)
    wuk_t = rand(H * R, nope, scale=0.05, seed=13)  # stacked W_UK[h]^T, [R, nope] per head
    y = torch.empty(B, H * R, dtype=torch.bfloat16, device="cuda")
    gpu_ctx.linear(wuk_t, q, y, M=R, K=nope, G=H, x_group_col=nope + rope, y_group_col=R)
    gpu_ctx.sync()
    qv = q.float().view(B, H, nope + rope)[:, :, :nope]
    ref = torch.einsum("bhk,hrk->bhr", qv, wuk_t.float().view(H, R, nope)).reshape(B, H * R)
    assert max_rel(y, ref) <= 1e-2


def test_linear_rejects_bad_shapes(gpu_ctx):
    import torch

    w = rand(128, 100, seed=1)
    x = rand(4, 100, seed=2)
    y = torch.empty(4, 128, device="cuda")
    with pytest.raises(dsb.DsbError) as e:
        gpu_ctx.linear(w, x, y, M=128, K=100)
    assert e.value.code == dsb.DSB_EINVAL
