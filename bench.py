"""Benchmark of the B200 decode hot path (one JSON line on rank 0).

Workload "model" (default): DeepSeek-V2-Lite-shaped batched decode - 27
layers, hidden 2048, 16 heads, kv_lora_rank 512, 1 dense + 26 MoE layers (64
experts top-6, 2 shared), vocab 102400; random-init N(0, 0.02) bf16 weights
made on the device (seed 3); B=32 sequences per GPU with 512-token random
prompts, then timed decode steps.  A step is one dsb_decode_step: one new
token for each of the 32 sequences through every layer, greedy ids back to
the host.  On one GPU the prompts go through chunked dsb_prefill (untimed).
Under torchrun (N > 1) the routed experts are split over the ranks (expert
parallel, dispatch / combine kernels writing into the peers' memory) and
attention stays data parallel: every rank decodes its own B sequences
(weak scaling), prefilling in chunks of 512 rows in step; before that, the tiny model's
expert-parallel logits are checked against the unsplit model ("ep_parity").
The line also carries the isolated MLA (cfg2) and FP8 MoE layer (cfg3)
roofline fractions, and at 8 GPUs the DeepSeek-V3 target ("target").

Other workloads: "v3" (DeepSeek-V3 shape, FP8, 4096-token context), "mla"
(isolated absorbed-MLA decode, B=64, 128 heads, context U[1024, 8192]),
"expert-gemm" (the dominant kernel alone), "moe-fp8" (one V3 MoE layer),
"attn-linears" (the four attention-side linears of a V2-Lite layer alone).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload model|v3|mla|expert-gemm|moe-fp8|attn-linears]
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "decode tokens/s (box) at 1/2/4/8 B200; MLA/MoE HBM GB/s as % of peak"
L2_BYTES = 126 * 1024 * 1024
T_START = time.time()
# latest start of the DeepSeek-V3 target measurement, seconds into the run
TARGET_START_BUDGET_S = 420
# rows per expert-parallel prefill pass (bounds the exchange windows: world x rows x k)
EP_PREFILL_CHUNK = 512
# ncu summary of the expert gate|up GEMM launch the default roofline line times
EXPERT_GEMM_PROFILE = "profiles/gemm_bf16_expert_gateup_v2lite.md"


def profile_traffic(name):
    """DRAM traffic of one captured launch from an ncu summary in profiles/:
    (read + write bytes, the launch's algorithmic bytes), parsed from the rows
    `| dram__bytes_read.sum / write.sum | R MB / W MB |` and
    `| algorithmic bytes of the captured launch | N |`; None if absent."""
    import re

    try:
        with open(os.path.join(ROOT, name)) as f:
            text = f.read()
    except OSError:
        return None
    m = re.search(r"\|\s*dram__bytes_read\.sum / write\.sum\s*\|\s*([\d.]+) (MB|GB) / ([\d.]+) (MB|GB)", text)
    a = re.search(r"\|\s*algorithmic bytes of the captured launch\s*\|\s*([\d,]+)", text)
    if not m or not a:
        return None
    unit = {"MB": 1e6, "GB": 1e9}
    traffic = float(m.group(1)) * unit[m.group(2)] + float(m.group(3)) * unit[m.group(4)]
    return traffic, int(a.group(1).replace(",", ""))


def measured_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled every 200 ms."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device_index: int):
        self.dev = device_index
        self.proc = None
        self.f = None

    def start(self):
        try:
            self.f = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.dev}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=self.f, stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["clock sampling unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        self.f.flush()
        self.f.seek(0)
        rows = [r.split(",") for r in self.f.read().strip().splitlines() if r.strip()]
        os.unlink(self.f.name)
        sm, smax, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            try:
                sm.append(float(r[1]))
                smax = float(r[2])
                for i, n in enumerate(names):
                    if r[5 + i].strip().lower() == "active":
                        reasons.add(n)
            except (ValueError, IndexError):
                pass
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": smax, "reasons": sorted(reasons),
                "samples": len(sm)}


# --------------------------------------------------------------- CPU baselines


def _cpu_port_worker(args):
    """Time the oracle port of the reference's attention loop on sequences."""
    import numpy as np

    import oracle as O

    q_lat, q_rope, cache, bt, lens, scale = args
    t0 = time.perf_counter()
    O.mla_decode_paged(q_lat, q_rope, cache, bt, lens, scale)
    return time.perf_counter() - t0, int(np.asarray(lens).size)


def _cpu_sample(case, n_seq):
    """A bounded sample: the n_seq sequences nearest the mean length, with their
    pages gathered into a compact host cache."""
    import numpy as np

    from deepseek_cpp_infer_b200.workloads import to_u16

    mean = case.seq_lens.mean()
    idx = list(np.argsort(np.abs(case.seq_lens - mean))[:n_seq])
    q_lat = to_u16(case.q_lat)[idx]
    q_rope = to_u16(case.q_rope)[idx]
    pages = [case.block_table_host[b, : (case.seq_lens[b] + 63) // 64] for b in idx]
    allp = np.concatenate(pages)
    cache = to_u16(case.cache[torch_index(allp)])
    bt = np.zeros((len(idx), max(len(p) for p in pages)), np.int32)
    k = 0
    for i, p in enumerate(pages):
        bt[i, : len(p)] = np.arange(k, k + len(p))
        k += len(p)
    lens = case.seq_lens[idx]
    return q_lat, q_rope, cache, bt, lens, float(lens.mean() / mean)


def torch_index(a):
    import torch

    return torch.from_numpy(a.astype("int64")).to("cuda")


def cpu_baseline_port(case, budget_s=15.0):
    """1-thread oracle port on sequences near the mean length; tokens/s scaled
    to the workload's mean context."""
    q_lat, q_rope, cache, bt, lens, len_ratio = _cpu_sample(case, 2)
    dt, n = _cpu_port_worker((q_lat[:1], q_rope[:1], cache, bt[:1], lens[:1], case.scale))
    n_seq = 1
    if dt < budget_s / 2:
        dt2, _ = _cpu_port_worker((q_lat[1:], q_rope[1:], cache, bt[1:], lens[1:], case.scale))
        dt += dt2
        n_seq = 2
    tok_s = n_seq / dt * len_ratio
    return {"value": tok_s, "unit": "tokens/s", "cores": 1, "kind": "port",
            "sample": f"{n_seq} sequence(s) nearest the mean context ({', '.join(str(int(x)) for x in lens[:n_seq])} "
                      f"tokens) through orc_mla_decode_paged (the reference's attention loop, mla.cpp:86-116), "
                      f"scaled to the mean context"}


# ------------------------------------------------------------------ arms


def run_mla_reference(args):
    """The reference's CPU attention loop (oracle port) on the host cores."""
    import multiprocessing as mp

    import torch

    from deepseek_cpp_infer_b200.workloads import mla_case

    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    cores = os.cpu_count() or 1
    case = mla_case(seed=1, device="cuda" if torch.cuda.is_available() else "cpu")
    q_lat, q_rope, cache, bt, lens, len_ratio = _cpu_sample(case, cores)
    jobs = [(q_lat[i:i + 1], q_rope[i:i + 1], cache, bt[i:i + 1], lens[i:i + 1], case.scale) for i in range(len(lens))]
    ctxm = mp.get_context("spawn")
    with ctxm.Pool(cores) as pool:
        for _ in range(args.warmup):
            pool.map(_cpu_port_worker, jobs[:1])
        t0 = time.perf_counter()
        for _ in range(args.steps):
            pool.map(_cpu_port_worker, jobs)
        dt = time.perf_counter() - t0
    tok_s = len(jobs) * args.steps / dt * len_ratio
    line = {
        "metric": METRIC, "value": tok_s, "unit": "tokens/s", "n_gpus": args.gpus, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": dt / args.steps * 1e3, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic", "impl": "reference",
        "config": {"workload": "isolated MLA decode, DeepSeek-V3 shape (B=64, H=128, R=512, P=64, ctx U[1024,8192], "
                               "page 64, seed 1)", "sample": f"{len(jobs)} sequences per step"},
        "cpu_baseline": {"value": tok_s, "unit": "tokens/s", "cores": cores, "kind": "port",
                         "sample": f"{len(jobs)} sequences nearest the mean context per step, one per process "
                                   f"(spawn pool of {cores}), orc_mla_decode_paged"},
        "e2e": {"value": tok_s, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def run_mla_ours(args):
    import torch
    import torch.distributed as dist

    import deepseek_cpp_infer_b200 as dsb
    from deepseek_cpp_infer_b200.workloads import mla_case

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(x):
        t = torch.tensor([x], device=dev)
        if world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    ctx = dsb.Context(local)
    stream = torch.cuda.Stream(device=dev)  # owned by torch; the context only borrows it
    ctx.set_stream(stream.cuda_stream)
    case = mla_case(B=args.batch, seed=1 + 1000 * rank, device=f"cuda:{local}")
    out = torch.empty(case.B, case.H, case.R, dtype=torch.bfloat16, device=dev)
    plan = ctx.mla_plan(case.seq_lens, case.H, case.R, case.P)

    def step():
        ctx.mla_decode_planned(plan, case.q_lat, case.q_rope, case.cache, case.block_table, case.scale, out)

    def timed(fn, n):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(n):
            fn()
        e1.record(stream)
        e1.synchronize()
        ctx.sync()
        return e0.elapsed_time(e1) / n

    # ---------------- device-resident timing (KV cache 332 MB > L2, so no flush is needed)
    warm = max(3, args.warmup)
    for _ in range(warm):
        step()
    ctx.sync()
    sampler = ClockSampler(local)
    sampler.start()
    # keep the GPU busy ~1 s so the clock samples see the load, then time K steps
    t_probe = timed(step, 10)
    timed(step, max(1, int(1000.0 / max(t_probe, 1e-3))))
    barrier()
    torch.cuda.synchronize()
    ctx.reset_stats()
    ms = timed(step, args.steps)
    clocks = sampler.stop()
    launches = ctx.stats()["kernel_launches"]
    ms_max = max_over_ranks(ms)

    # ---------------- end to end through the C ABI with host buffers:
    # pinned q in, dsb_mla_decode (plans from host lengths, then decodes), latent out back
    q_lat_h = case.q_lat.cpu().pin_memory()
    q_rope_h = case.q_rope.cpu().pin_memory()
    out_h = torch.empty(out.shape, dtype=out.dtype).pin_memory()
    q_lat_d = torch.empty_like(case.q_lat)
    q_rope_d = torch.empty_like(case.q_rope)

    def e2e_step():
        with torch.cuda.stream(stream):
            q_lat_d.copy_(q_lat_h, non_blocking=True)
            q_rope_d.copy_(q_rope_h, non_blocking=True)
        ctx.mla_decode(q_lat_d, q_rope_d, case.cache, case.block_table, case.seq_lens, case.scale, out)
        with torch.cuda.stream(stream):
            out_h.copy_(out, non_blocking=True)

    for _ in range(3):
        e2e_step()
    ctx.sync()
    barrier()
    ms_e2e = max_over_ranks(timed(e2e_step, args.steps))
    h2d = case.q_lat.numel() * 2 + case.q_rope.numel() * 2 + case.B * 4
    d2h = out.numel() * 2

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline_port(case)

    if rank == 0:
        peak, peak_kind = measured_peaks()
        achieved = case.algorithmic_bytes / (ms_max * 1e-3) / 1e9
        tok_s = world * case.B / (ms_max * 1e-3)
        info = plan.info()
        line = {
            "metric": METRIC, "value": tok_s, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
            "warmup": warm, "ms_per_step": ms_max, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded N(0,1) q and cache, seed 1 + 1000*rank)",
            "config": {
                "workload": f"isolated MLA decode attention, DeepSeek-V3 shape: B={case.B} per GPU, H=128, kv_lora_rank 512, "
                            "rope 64, scale 1/sqrt(192), ctx U[1024,8192] (seed 1), 64-token pages, random block table",
                "kv_bytes_per_step": case.kv_bytes, "l2": "inputs larger than L2 (KV cache %.0f MB > 126 MB)"
                % (case.kv_bytes / 1e6), "parallelism": f"dp{world} (attention data-parallel over the batch)",
                "work_items": info["n_items"], "split_partials": info["n_partial"],
            },
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                         "traffic": None, "peak_kind": peak_kind,
                         "note": "algorithmic bytes (KV rows + q + latent out) per step / CUDA-event step time; a "
                                 "step is mla_decode_kernel + mla_combine_kernel"},
            "e2e": {"value": world * case.B / (ms_e2e * 1e-3), "unit": "tokens/s", "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h},
            "gpu_launches": launches, "clocks": clocks,
        }
        if cpu is not None:
            line["cpu_baseline"] = cpu
        print(json.dumps(line), flush=True)
    plan.close()
    ctx.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


# ============================================================ model workload


def model_cfg(args):
    from deepseek_cpp_infer_b200.workloads import V2_LITE, V3

    cfg = dict(V3 if args.workload == "v3" else V2_LITE)
    if args.layers:
        cfg["num_hidden_layers"] = args.layers
    if args.experts:
        # fewer routed experts: one GPU doing the per-rank expert work of a larger expert-parallel run
        cfg["n_routed_experts"] = args.experts
    return cfg


def step_bytes(cfg, B, ctx_len, world=1):
    """Algorithmic HBM bytes of one decode step on one GPU: every weight the
    step must read once (routed experts: the expected number touched by the
    world*B tokens under uniform routing, E * (1 - (1 - k/E)^(world*B)), split
    over the world ranks that own them), plus the KV rows of its B sequences."""
    D, H, R, P = cfg["hidden_size"], cfg["num_attention_heads"], cfg["kv_lora_rank"], cfg["qk_rope_head_dim"]
    nope, v, L = cfg["qk_nope_head_dim"], cfg["v_head_dim"], cfg["num_hidden_layers"]
    E, k, I = cfg["n_routed_experts"], cfg["num_experts_per_tok"], cfg["moe_intermediate_size"]
    Is, Id, V = cfg["n_shared_experts"] * I, cfg["intermediate_size"], cfg["vocab_size"]
    ql = cfg.get("q_lora_rank", 0)
    wb = 1 + 4 / (128 * 128) if cfg.get("weights_fp8") else 2  # bytes per projection / FFN weight (+ FP8 scales)
    q_proj = (ql * D + H * (nope + P) * ql) if ql else H * (nope + P) * D
    attn = (q_proj + (R + P) * D + D * H * v) * wb + (H * R * nope + H * v * R) * 2  # absorbed W_UK / W_UV in bf16
    dense_layers = min(cfg["first_k_dense_replace"], L)
    touched = E * (1 - (1 - k / E) ** (world * B)) / world
    moe = touched * 3 * I * D * wb + 3 * Is * D * wb + E * D * 4
    w = L * attn + dense_layers * 3 * Id * D * wb + (L - dense_layers) * moe + V * D * 2
    kv = L * B * ctx_len * (R + P) * 2
    return int(w + kv), int(w), int(kv), touched


def time_expert_gemm(ctx, stream, cfg, B, steps, world=1):
    """The dominant kernel in isolation: the expert gate|up GEMM of one MoE
    layer as this rank's decode step launches it, 2I x D bf16 weights per
    group, timed with CUDA events on the context stream.  One GPU: all E
    routed groups plus the n_shared shared groups in one launch, B*(k +
    n_shared) permuted rows of a random top-k routing.  Expert parallel: the
    rank's E/world routed groups receiving the world*B tokens' picks of them
    (the shared groups run in a launch of their own on the rank's tokens)."""
    import numpy as np
    import torch

    import deepseek_cpp_infer_b200 as dsb

    D, E, k, I = cfg["hidden_size"], cfg["n_routed_experts"], cfg["num_experts_per_tok"], cfg["moe_intermediate_size"]
    ns, EL = cfg.get("n_shared_experts", 0), E // world
    rng = np.random.default_rng(11)
    picks = np.stack([rng.choice(E, k, replace=False) for _ in range(world * B)])
    if world == 1:
        # the single-GPU step's permutation: every token's top-k plus each shared group
        ids = np.concatenate([picks, np.tile(E + np.arange(ns), (B, 1))], axis=1)
        counts = np.bincount(ids.ravel(), minlength=E + ns)
    else:
        counts = np.bincount(picks.ravel(), minlength=E)[:EL]
    G = len(counts)
    offs = torch.from_numpy(np.concatenate([[0], np.cumsum(counts)]).astype(np.int32)).cuda()
    rows = int(counts.sum())
    w = (torch.randn(G * 2 * I, D, device="cuda") * 0.02).to(torch.bfloat16)
    x = torch.randn(rows, D, device="cuda").to(torch.bfloat16)
    y = torch.empty(rows, I, dtype=torch.bfloat16, device="cuda")

    def launch():
        ctx.linear(w, x, y, M=2 * I, K=D, G=G, tok_offsets=offs, max_tokens_per_group=B,
                   epilogue=dsb.EPI_SILU_GATE)

    for _ in range(5):
        launch()
    ctx.sync()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    n = max(steps, 20)
    e0.record(stream)
    for _ in range(n):
        launch()
    e1.record(stream)
    e1.synchronize()
    ms = e0.elapsed_time(e1) / n
    touched = int((counts > 0).sum())
    nbytes = touched * 2 * I * D * 2 + rows * D * 2 + rows * I * 2
    del w
    return ms, nbytes, touched


def time_expert_gemm_fp8(ctx, stream, cfg, B, world, steps):
    """V3 shape: this rank's FP8 expert gate|up GEMM of one MoE layer in
    isolation -- E/world routed groups receiving the world*B tokens' picks of
    them under uniform routing, plus the shared group with this rank's B
    tokens -- timed with CUDA events on the context stream."""
    import numpy as np
    import torch

    import deepseek_cpp_infer_b200 as dsb
    from deepseek_cpp_infer_b200.workloads import MoeFp8Weights

    D, E, k, I = cfg["hidden_size"], cfg["n_routed_experts"], cfg["num_experts_per_tok"], cfg["moe_intermediate_size"]
    ns, EL = cfg["n_shared_experts"], E // world
    rng = np.random.default_rng(11)
    picks = np.stack([rng.choice(E, k, replace=False) for _ in range(world * B)]).ravel()
    counts = np.concatenate([np.bincount(picks, minlength=E)[:EL], [B] * ns])
    G = EL + ns
    offs = torch.from_numpy(np.concatenate([[0], np.cumsum(counts)]).astype(np.int32)).cuda()
    T = int(counts.sum())
    layer = MoeFp8Weights(ctx, EL, ns, D, I, seed=12)
    xq = torch.randint(0, 0x7E, (T, D), dtype=torch.uint8, device="cuda")
    sx = torch.full((T, D // 128), 1e-2, device="cuda")
    y = torch.empty(T, I, dtype=torch.bfloat16, device="cuda")

    def launch():
        ctx.linear_fp8(layer.gate_up.view(G * 2 * I, D), layer.gate_up_scale.view(-1, D // 128), xq, sx, y,
                       M=2 * I, K=D, G=G, scale_rows=2, tok_offsets=offs, max_tokens_per_group=B,
                       epilogue=dsb.EPI_SILU_GATE)

    for _ in range(5):
        launch()
    ctx.sync()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    n = max(steps, 20)
    e0.record(stream)
    for _ in range(n):
        launch()
    e1.record(stream)
    e1.synchronize()
    ms = e0.elapsed_time(e1) / n
    touched = int((counts > 0).sum())
    nbytes = touched * (2 * I * D + (2 * I // 128) * 2 * (D // 128) * 4) + T * D + T * I * 2
    del layer
    return ms, nbytes, touched


def isolated_mla_fraction(ctx, stream, dev, B=64, lens=None, seed=1, n=20):
    """The MLA decode kernel alone at DeepSeek-V3 shape (128 heads, rank 512,
    rope 64): B sequences with contexts U[1024, 8192] (or `lens`), random
    block table; dsb_mla_decode_planned timed with CUDA events.  Returns the
    HBM roofline record of one call (KV rows + q + latent out per call)."""
    import torch

    from deepseek_cpp_infer_b200.workloads import mla_case

    case = mla_case(B=B, lens=lens, seed=seed, device=str(dev))
    out = torch.empty(case.B, case.H, case.R, dtype=torch.bfloat16, device=dev)
    plan = ctx.mla_plan(case.seq_lens, case.H, case.R, case.P)

    def call():
        ctx.mla_decode_planned(plan, case.q_lat, case.q_rope, case.cache, case.block_table, case.scale, out)

    for _ in range(3):
        call()
    ctx.sync()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(n):
        call()
    e1.record(stream)
    e1.synchronize()
    ctx.sync()
    ms = e0.elapsed_time(e1) / n
    peak, peak_kind = measured_peaks()
    gbs = case.algorithmic_bytes / (ms * 1e-3) / 1e9
    plan.close()
    rec = {"bound": "hbm", "achieved": gbs, "peak": peak, "unit": "GB/s", "frac": gbs / peak, "peak_kind": peak_kind,
           "us_per_call": ms * 1e3, "bytes_per_call": case.algorithmic_bytes, "tflops": case.flops / (ms * 1e-3) / 1e12,
           "workload": f"B={case.B}, H=128, R=512, P=64, context mean {float(case.seq_lens.mean()):.0f}, 64-token "
                       f"pages, random block table (seed {seed})"}
    del case, out
    return rec


def isolated_moe_fp8_fraction(ctx, stream, T=128, seed=2, n=10):
    """One DeepSeek-V3 MoE layer alone (router + sigmoid/bias grouped top-8 +
    256 routed and 1 shared FP8 expert, D=7168, I=2048) for T tokens, timed
    with CUDA events; the HBM roofline record of one layer call (touched
    experts' e4m3 weights + scales, x, h, logits)."""
    import numpy as np
    import torch

    import deepseek_cpp_infer_b200 as dsb
    from deepseek_cpp_infer_b200.workloads import V3_MOE, MoeFp8Weights

    cfg = dict(V3_MOE)
    D, I, E, k, ns = (cfg["hidden_size"], cfg["moe_intermediate_size"], cfg["n_routed_experts"],
                      cfg["num_experts_per_tok"], cfg["n_shared_experts"])
    layer = MoeFp8Weights(ctx, E, ns, D, I, seed=seed)
    gen = torch.Generator(device="cuda").manual_seed(seed)
    w_gate = torch.randn(E, D, generator=gen, device="cuda") * 0.02
    bias = torch.randn(E, generator=gen, device="cuda") * 0.01
    x = torch.randn(T, D, generator=gen, device="cuda").to(torch.bfloat16)
    x32 = x.float()
    logits = torch.empty(T, E, device="cuda")
    ids = torch.empty(T, k, dtype=torch.int32, device="cuda")
    wts = torch.empty(T, k, device="cuda")
    h = torch.zeros(T, D, device="cuda")
    torch.cuda.synchronize()

    def call():
        ctx.router_logits(x32, w_gate, logits)
        ctx.moe_route(logits, ids, wts, k, scoring=dsb.SCORE_SIGMOID, bias=bias, n_group=cfg["n_group"],
                      topk_group=cfg["topk_group"], norm_topk=cfg["norm_topk_prob"],
                      routed_scale=cfg["routed_scaling_factor"])
        ctx.moe_ffn_fp8(layer.gate_up, layer.gate_up_scale, layer.down, layer.down_scale, E=E, n_shared=ns, x=x,
                        ids=ids, weights=wts, h=h)

    for _ in range(3):
        call()
    ctx.sync()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(n):
        call()
    e1.record(stream)
    e1.synchronize()
    ctx.sync()
    ms = e0.elapsed_time(e1) / n
    touched = len(np.unique(ids.cpu().numpy())) + ns
    wbytes = touched * 3 * I * D + touched * (3 * I * D // (128 * 128)) * 4
    nbytes = wbytes + T * D * 2 + 2 * T * D * 4 + T * E * 4
    peak, peak_kind = measured_peaks()
    gbs = nbytes / (ms * 1e-3) / 1e9
    del layer
    return {"bound": "hbm", "achieved": gbs, "peak": peak, "unit": "GB/s", "frac": gbs / peak, "peak_kind": peak_kind,
            "us_per_call": ms * 1e3, "bytes_per_call": nbytes, "experts_touched": int(touched),
            "workload": f"one V3 MoE layer, T={T} tokens, 256 routed (sigmoid + bias, 8 groups / top-4 / top-8) + "
                        f"1 shared FP8 expert, D=7168, I=2048 (seed {seed})"}


def ep_tiny_parity(ctx, rank, world, steps=6):
    """The tiny DeepSeek-V2-style model with its 16 experts split over the
    world ranks against the same model unsplit on this rank, for a few
    decode steps of this rank's own sequences: True when every step's logits
    are bit-identical (the exchange only moves rows and sums in moe_step's
    order).  Every rank takes the same collective steps."""
    import numpy as np
    import torch.distributed as dist

    import deepseek_cpp_infer_b200 as dsb
    from deepseek_cpp_infer_b200.workloads import TINY, model_tensors

    ep = dsb.EP(ctx, rank, world, TINY["n_routed_experts"], TINY["hidden_size"], TINY["num_experts_per_tok"],
                max_tokens=8)
    handles = [None] * world
    dist.all_gather_object(handles, ep.window_handle())
    ep.connect(handles)
    tensors = model_tensors(TINY, seed=0)
    models, kvs = [], []
    try:
        for use_ep in (True, False):
            m = dsb.Model(ctx, dsb.ModelConfig(**TINY))
            models.append(m)
            if use_ep:
                m.set_ep(ep)
            for name, a in tensors.items():
                m.set_tensor(name, a)
            m.finalize()
            kvs.append(dsb.KVCache(ctx, m, n_blocks=8, max_seqs=4, max_blocks_per_seq=1))
        B = 1 + rank % 3
        prompts = np.random.default_rng(50 + rank).integers(0, TINY["vocab_size"], (B, steps))
        seqs = [[kv.alloc_seq() for _ in range(B)] for kv in kvs]
        same = True
        for i in range(steps):
            toks = [int(t) for t in prompts[:, i]]
            g0, l0 = dsb.decode_step(ctx, models[0], kvs[0], seqs[0], toks, want_logits=True)
            g1, l1 = dsb.decode_step(ctx, models[1], kvs[1], seqs[1], toks, want_logits=True)
            same &= bool(np.array_equal(g0, g1) and np.array_equal(l0, l1))
        return same
    finally:
        for kv in kvs:
            kv.close()
        for m in models:
            m.close()
        ep.close()


def trace_steps(out_dir, rank, step, n, stream):
    """Per-kernel device times of decode steps from CUPTI activity records
    (torch.profiler; unlike an ncu replay it does not serialise the launches,
    so the expert-parallel kernels that wait on peer ranks run as they do
    untraced).  Runs n + 2 steps and keeps the last n (the first ones absorb
    the ranks' different profiler start-up).  Writes
    <out_dir>/kernels_rank<r>.md: per kernel name its launches, "advance"
    (end of the kernel minus end of the previous one: the stream's progress
    it accounts for, less what it overlapped with its predecessor through
    programmatic dependent launch; the advances sum to the traced time) and
    duration; then the kernels of one layer in order (the layers cut at each
    MLA launch), averaged over the layers of the same sequence."""
    import torch
    from torch.profiler import ProfilerActivity, profile

    os.makedirs(out_dir, exist_ok=True)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        for _ in range(2):
            step()
        e0.record(stream)
        for _ in range(n):
            step()
        e1.record(stream)
        e1.synchronize()
    evs = []
    for ev in prof.events():
        if str(getattr(ev, "device_type", "")).endswith("CUDA") and ev.time_range.end > ev.time_range.start:
            evs.append((ev.time_range.start, ev.time_range.end, ev.name))
    evs.sort()
    per_step = len(evs) // (n + 2)
    prev_end = evs[2 * per_step - 1][1] if per_step else None
    evs = evs[2 * per_step:]
    stats, seq = {}, []
    for t0, t1, name in evs:
        adv = t1 - t0 if prev_end is None else max(0.0, t1 - max(prev_end, t0))
        prev_end = t1 if prev_end is None else max(prev_end, t1)
        cnt, dur, a = stats.get(name, (0, 0.0, 0.0))
        stats[name] = (cnt + 1, dur + (t1 - t0), a + adv)
        seq.append((name, adv, t1 - t0))
    rows = sorted(stats.items(), key=lambda kv: -kv[1][2])
    total = sum(v[2] for _, v in rows) or 1.0
    short = lambda nm: nm.replace("dsb::(anonymous namespace)::", "").split("(")[0][:60]  # noqa: E731
    with open(os.path.join(out_dir, f"kernels_rank{rank}.md"), "w") as f:
        f.write(f"rank {rank}: {n} steps, {e0.elapsed_time(e1) / n * 1e3:.1f} us per step (CUDA events, traced)\n\n")
        f.write("| kernel | launches/step | advance us/step | share | duration us/step | mean duration us |\n"
                "|---|---|---|---|---|---|\n")
        for name, (cnt, dur, adv) in rows:
            f.write(f"| {short(name)} | {cnt / n:.1f} | {adv / n:.1f} | {100 * adv / total:.1f}% | {dur / n:.1f} | "
                    f"{dur / cnt:.2f} |\n")
        # one layer in order: segments between MLA launches of the last step, grouped by kernel sequence
        last = seq[-per_step:] if per_step else []
        cuts = [i for i, (nm, _, _) in enumerate(last) if "mla_decode_kernel" in nm]
        segs = [last[a:b] for a, b in zip(cuts, cuts[1:])]
        groups = {}
        for sg in segs:
            groups.setdefault(tuple(short(nm) for nm, _, _ in sg), []).append(sg)
        if groups:
            key, members = max(groups.items(), key=lambda kv: len(kv[1]))
            f.write(f"\nOne layer, MLA to MLA, mean over {len(members)} layers of the last step:\n\n"
                    "| # | kernel | advance us | duration us |\n|---|---|---|---|\n")
            for i, nm in enumerate(key):
                f.write(f"| {i} | {nm} | {sum(m[i][1] for m in members) / len(members):.1f} | "
                        f"{sum(m[i][2] for m in members) / len(members):.1f} |\n")


def measure_model(args, cfg, B, P, steps, env):
    """Build the random-init model (expert parallel over the world ranks when
    world > 1), fill every sequence's context, run warm-up steps, then time
    `steps` decode steps device-resident and `steps` more end to end (logits
    back to pinned host memory every step).  Returns the rank's figures with
    the times already maxed over ranks."""
    import numpy as np
    import torch
    import torch.distributed as dist

    import deepseek_cpp_infer_b200 as dsb

    ctx, stream, world, rank, local = env["ctx"], env["stream"], env["world"], env["rank"], env["local"]
    barrier, max_over_ranks = env["barrier"], env["max_over_ranks"]
    v3 = bool(cfg.get("weights_fp8"))
    model = dsb.Model(ctx, dsb.ModelConfig(**cfg))
    ep = kv = None
    try:
        if world > 1:
            # expert parallel: rank r owns routed experts [r*E/world, (r+1)*E/world); attention and
            # the shared experts stay data parallel (every rank decodes its own B sequences)
            # windows sized for the prefill chunks (rows of every rank's chunk may meet at one expert)
            ep = dsb.EP(ctx, rank, world, cfg["n_routed_experts"], cfg["hidden_size"], cfg["num_experts_per_tok"],
                        max_tokens=B if v3 else max(B, EP_PREFILL_CHUNK))
            handles = [None] * world
            dist.all_gather_object(handles, ep.window_handle())
            ep.connect(handles)
            model.set_ep(ep)
        model.init_random(seed=4 if v3 else 3, stddev=0.02)
        warm = max(3, args.warmup)
        total = P + warm + steps * 2 + 64
        max_blocks = (total + 63) // 64
        kv = dsb.KVCache(ctx, model, n_blocks=B * max_blocks, max_seqs=B, max_blocks_per_seq=max_blocks)
        seqs = [kv.alloc_seq() for _ in range(B)]
        prompts = np.random.default_rng((4 if v3 else 3) + 1000 * rank).integers(
            0, cfg["vocab_size"], (B, P)).astype(np.int32)
        t0 = time.time()
        if v3:
            # a P-token context per sequence: synthetic N(0,1) latents in every layer's cache rows
            # (decode reads the same bytes as after a real prefill), then one token each
            for j, sq in enumerate(seqs):
                kv.fill_random(sq, P - 1, seed=4 + 1000 * rank + j)
            greedy, _ = dsb.decode_step(ctx, model, kv, seqs, prompts[:, -1])
            prefill = "synthetic cache fill"
        elif world == 1:
            # chunked prefill: every prompt row of a chunk through the layers in one pass
            greedy = dsb.prefill_prompts(ctx, model, kv, seqs, [list(p) for p in prompts])
            prefill = "chunked dsb_prefill (<= 4096 rows per pass)"
        else:
            # expert parallel: every rank prefills its own prompts in chunks of the same row
            # count, in step (each chunk's MoE layers exchange all its rows' picks)
            greedy = dsb.prefill_prompts(ctx, model, kv, seqs, [list(p) for p in prompts], chunk=EP_PREFILL_CHUNK)
            prefill = f"chunked dsb_prefill, expert parallel (<= {EP_PREFILL_CHUNK} rows per pass)"
        prefill_s = time.time() - t0
        nxt = greedy
        logits_host = torch.empty((B, cfg["vocab_size"]), dtype=torch.float32, pin_memory=True).numpy()

        def step(want_logits=False):
            nonlocal nxt
            nxt, lg = dsb.decode_step(ctx, model, kv, seqs, nxt, logits_out=logits_host if want_logits else None)
            return lg

        def timed(n, want_logits=False):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            for _ in range(n):
                step(want_logits)
            e1.record(stream)
            e1.synchronize()
            return e0.elapsed_time(e1) / n

        for _ in range(warm):
            step()
        barrier()
        sampler = ClockSampler(local)
        sampler.start()
        time.sleep(0.4)  # the sampler's first sample lands inside the timed region
        ctx.reset_stats()
        torch.cuda.synchronize()
        ms = timed(steps)
        clocks = sampler.stop()
        launches = ctx.stats()["kernel_launches"]
        ms_max = max_over_ranks(ms)
        ctx_len = kv.seq_len(seqs[0])
        # end to end: the reference's ForwardOutput carries the logits, so e2e also
        # copies every step's [B, vocab] fp32 logits back to (pinned) host memory
        barrier()
        ms_e2e = max_over_ranks(timed(steps, want_logits=True))
        ctx.sync()
        if args.trace:
            barrier()
            try:
                trace_steps(args.trace, rank, lambda: step(), 3, stream)
            except Exception as e:  # noqa: BLE001  diagnostics only; the measured line stands
                print(f"trace failed: {type(e).__name__}: {e}", file=sys.stderr)
    finally:
        if kv is not None:
            kv.close()
        model.close()
        if ep is not None:
            ep.close()
    return {"ms": ms_max, "ms_e2e": ms_e2e, "launches": launches, "ctx_len": ctx_len, "clocks": clocks,
            "prefill_s": prefill_s, "prefill": prefill, "max_blocks": max_blocks, "warm": warm}


def run_model_ours(args):
    import torch
    import torch.distributed as dist

    import deepseek_cpp_infer_b200 as dsb

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev)

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(x):
        t = torch.tensor([x], device=dev)
        if world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    cfg = model_cfg(args)
    B, P = args.batch, args.prompt
    v3 = args.workload == "v3"
    ctx = dsb.Context(local)
    stream = torch.cuda.Stream(device=dev)
    ctx.set_stream(stream.cuda_stream)
    env = {"ctx": ctx, "stream": stream, "world": world, "rank": rank, "local": local, "barrier": barrier,
           "max_over_ranks": max_over_ranks}

    # expert-parallel correctness first: the tiny model split over the ranks must give the
    # unsplit model's logits bit for bit (every rank runs it; the flag is ANDed over ranks)
    ep_parity = None
    if world > 1:
        ok = ep_tiny_parity(ctx, rank, world)
        ep_parity = max_over_ranks(0.0 if ok else 1.0) == 0.0

    r = measure_model(args, cfg, B, P, args.steps, env)
    # the dominant kernel alone, for the roofline line
    if v3:
        g_ms, g_bytes, g_touched = time_expert_gemm_fp8(ctx, stream, cfg, B, world, args.steps)
    else:
        g_ms, g_bytes, g_touched = time_expert_gemm(ctx, stream, cfg, B, args.steps, world)
    # the two north-star kernels at their own benchmark shapes, each on this rank's GPU
    fractions = {}
    if not args.no_fractions:
        fractions["mla"] = isolated_mla_fraction(ctx, stream, dev)
        fractions["moe_fp8"] = isolated_moe_fp8_fraction(ctx, stream)
        torch.cuda.empty_cache()
    target = None
    if (world == 8 or args.target) and not v3 and not args.no_target:
        # the target builds a ~100 GB model per GPU: only when the run so far
        # leaves room for it (every rank takes the same decision)
        elapsed = max_over_ranks(time.time() - T_START)
        if elapsed <= TARGET_START_BUDGET_S:
            target = measure_target(args, env, dev)
        else:
            target = {"skipped": f"{elapsed:.0f} s into the run, above the {TARGET_START_BUDGET_S} s start budget"}

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline and not v3:
        cpu = model_cpu_baseline(cfg, r["ctx_len"], cores=1)

    if rank == 0:
        peak, peak_kind = measured_peaks()
        ms_max, ctx_len = r["ms"], r["ctx_len"]
        tot, wbytes, kvbytes, touched = step_bytes(cfg, B, ctx_len, world)
        g_gbs = g_bytes / (g_ms * 1e-3) / 1e9
        traffic = None
        if not v3:
            prof = profile_traffic(EXPERT_GEMM_PROFILE)
            if prof is not None:
                # the capture's DRAM traffic, scaled to this launch's algorithmic bytes
                # (the weight stream grows in proportion to the groups touched)
                traffic = prof[0] * g_bytes / prof[1]
        line = {
            "metric": METRIC, "value": world * B / (ms_max * 1e-3), "unit": "tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": r["warm"], "ms_per_step": ms_max, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "e4m3 weights, bf16 activations" if v3 else "bf16",
            "data": ("synthetic: random-init N(0,0.02) weights quantised to e4m3 with 128x128 scales (seed 4), "
                     "N(0,1) latent cache rows for the context" if v3 else
                     "synthetic: random-init N(0,0.02) bf16 weights (seed 3), uniform random prompt ids"),
            "config": {
                "workload": (f"DeepSeek-V3-shaped batched greedy decode: {cfg['num_hidden_layers']} layers, hidden 7168, "
                             f"128 heads, q_lora 1536, kv_lora_rank 512, 3 dense (FFN 18432) + "
                             f"{cfg['num_hidden_layers'] - 3} MoE layers ({cfg['n_routed_experts']} experts top-8 "
                             f"sigmoid grouped, 1 shared, moe_inter 2048), FP8 e4m3 block-scaled projections / FFN / "
                             f"experts, vocab 129280; B={B} per GPU, {P}-token context, step = one token for every "
                             f"sequence" if v3 else
                             f"DeepSeek-V2-Lite-shaped batched greedy decode: {cfg['num_hidden_layers']} layers, hidden "
                             f"2048, 16 heads, kv_lora_rank 512, 1 dense + {cfg['num_hidden_layers'] - 1} MoE layers "
                             f"(64 experts top-6 softmax, 2 shared, moe_inter 1408), vocab 102400; B={B} per GPU, "
                             f"{P}-token prompts, step = one token for every sequence"),
                "global_batch": world * B, "seq_len": ctx_len,
                "parallelism": "single GPU" if world == 1 else
                               f"ep{world} routed experts (peer-memory dispatch/combine) + dp{world} attention",
                "step_bytes": tot, "weight_bytes_per_step": wbytes, "kv_bytes_per_step": kvbytes,
                "experts_touched_per_layer": round(touched, 1), "prefill_s": round(r["prefill_s"], 2),
                "prefill": r["prefill"],
                "l2": f"every step streams {wbytes / 1e9:.1f} GB of weights per GPU, far above the 126 MB L2",
                "step_roofline_frac": tot / (ms_max * 1e-3) / 1e9 / peak,
            },
            "roofline": {"bound": "hbm", "achieved": g_gbs, "peak": peak, "unit": "GB/s", "frac": g_gbs / peak,
                         "traffic": traffic, "peak_kind": peak_kind,
                         "kernel": ("gemm_fp8_kernel (this rank's expert gate|up groups, SiLU epilogue)" if v3 else
                                    "gemm_bf16_kernel (expert gate|up, SiLU epilogue: " +
                                    ("routed + shared groups)" if world == 1 else
                                     f"this rank's {cfg['n_routed_experts'] // world} routed groups)")),
                         "note": f"{g_touched} expert groups' gate|up weights + activations per launch / "
                                 f"CUDA-event launch time ({g_ms * 1e3:.1f} us); traffic from "
                                 f"{EXPERT_GEMM_PROFILE if not v3 else 'none'}, scaled to this launch's "
                                 f"algorithmic bytes",
                         **fractions},
            "e2e": {"value": world * B / (r["ms_e2e"] * 1e-3), "unit": "tokens/s",
                    "h2d_bytes_per_step": B * 4 * (2 + r["max_blocks"]),
                    "d2h_bytes_per_step": B * 4 + B * cfg["vocab_size"] * 4},
            "gpu_launches": r["launches"], "clocks": r["clocks"],
        }
        if ep_parity is not None:
            line["ep_parity"] = ep_parity
        if target is not None:
            line["target"] = target
        if cpu is not None:
            line["cpu_baseline"] = cpu
        print(json.dumps(line), flush=True)
    ctx.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def measure_target(args, env, dev):
    """The north-star target: DeepSeek-V3 shape, FP8, B=32 sequences per GPU
    at a 4096-token context, experts over the world ranks (EP8 on 8 GPUs).
    Returns the box's tokens/s, the step's HBM roofline fraction, and the MLA
    and FP8 expert GEMM fractions at that shape; or {"error": ...} when any
    rank could not build it (every rank takes the same collective steps)."""
    import torch

    from deepseek_cpp_infer_b200.workloads import V3

    world, rank = env["world"], env["rank"]
    cfg = dict(V3)
    if args.target_experts:
        cfg["n_routed_experts"] = args.target_experts  # a smaller stand-in (one GPU exercising the path)
    B, P, steps = 32, 4096, 10
    torch.cuda.empty_cache()
    err = ""
    try:
        r = measure_model(args, cfg, B, P, steps, env)
    except Exception as e:  # noqa: BLE001  reported in the line; the ranks stay in step below
        err = f"rank {rank}: {type(e).__name__}: {e}"[:300]
        r = None
    failed = env["max_over_ranks"](1.0 if r is None else 0.0) > 0
    if failed:
        return {"error": err or "another rank failed"}
    g_ms, g_bytes, g_touched = time_expert_gemm_fp8(env["ctx"], env["stream"], cfg, B, world, 10)
    mla = isolated_mla_fraction(env["ctx"], env["stream"], dev, B=B, lens=[P + 16] * B, seed=5)
    peak, peak_kind = measured_peaks()
    tot, wbytes, kvbytes, touched = step_bytes(cfg, B, r["ctx_len"], world)
    fp8 = {"bound": "hbm", "achieved": g_bytes / (g_ms * 1e-3) / 1e9, "peak": peak, "unit": "GB/s",
           "frac": g_bytes / (g_ms * 1e-3) / 1e9 / peak, "peak_kind": peak_kind, "us_per_launch": g_ms * 1e3,
           "groups_touched": g_touched,
           "note": "this rank's FP8 expert gate|up launch at decode (HBM-bound: ~8 token rows per expert); the "
                   "tensor-peak point is the moe-fp8 workload at T=16384"}
    return {"workload": f"DeepSeek-V3 shape, FP8, {cfg['n_routed_experts']} experts over {world} ranks, B={B} per GPU, "
                        f"{P}-token context (synthetic cache fill)",
            "value": world * B / (r["ms"] * 1e-3), "unit": "tokens/s", "ms_per_step": r["ms"], "steps": steps,
            "e2e_value": world * B / (r["ms_e2e"] * 1e-3), "step_roofline_frac": tot / (r["ms"] * 1e-3) / 1e9 / peak,
            "step_bytes": tot, "gpu_launches": r["launches"], "clocks": r["clocks"], "mla": mla, "fp8_expert_gemm": fp8}


class RefModelSample:
    """The reference's CPU decode path at V2-Lite shape, as a bounded sample:
    one token through one layer of each kind plus a tenth of the lm_head, on
    one thread, through oracle/_ref (the reference's own code) when present,
    else the oracle's restatements.  sample() runs it once and returns
    (seconds the sample took, seconds of one whole-model token extrapolated
    from it): L attention layers (mla_decode_step at position 0 - its
    projections dominate - plus the per-head attention loop over ctx_len
    cached tokens, whose per-token cost is calibrated once from a 64-token
    run), the dense layers (three ds::rt::linear calls), the MoE layers
    (moe_step with 8 experts: the per-token cost of 6 routed + 2 shared
    experts does not depend on E) and the lm_head (a tenth, scaled by 10)."""

    def __init__(self, cfg, ctx_len):
        import numpy as np

        import oracle as O

        self.O, self.np, self.cfg, self.ctx_len = O, np, cfg, ctx_len
        D, H, R, P = cfg["hidden_size"], cfg["num_attention_heads"], cfg["kv_lora_rank"], cfg["qk_rope_head_dim"]
        nope, v, I, Id, V = (cfg["qk_nope_head_dim"], cfg["v_head_dim"], cfg["moe_intermediate_size"],
                             cfg["intermediate_size"], cfg["vocab_size"])
        Is = cfg["n_shared_experts"] * I
        self.use_ref = O.ref_available()
        self.kind = "reference" if self.use_ref else "port"
        f = lambda *shape: np.full(shape, 0.01, np.float32)  # noqa: E731  values do not change the cost
        self.c = O.RefConfig(hidden_size=D, num_attention_heads=H, qk_nope_head_dim=nope, qk_rope_head_dim=P,
                             v_head_dim=v, kv_lora_rank=R, num_hidden_layers=1, vocab_size=V,
                             max_position_embeddings=64, rms_norm_eps=1e-6, rope_theta=10000.0,
                             routed_scaling_factor=1.0, n_experts=8, moe_top_k=6, moe_intermediate_size=I)
        self.attn_w = (f(H * (nope + P), D), f(R + P, D), np.ones(R, np.float32), f(H * (nope + v), R), f(D, H * v),
                       f(64, D))
        self.attn_out = np.zeros((64, D), np.float32)
        self.wg, self.wd = f(Id, D), f(D, Id)
        self.x, self.y, self.z = f(D), np.zeros(Id, np.float32), np.zeros(D, np.float32)
        self.E = 8
        self.moe_w = (f(self.E, D), f(self.E, I, D), f(self.E, I, D), f(self.E, D, I), f(Is, D), f(Is, D), f(D, Is))
        self.Is, self.D, self.I = Is, D, I
        self.xo = np.zeros(D, np.float32)
        self.wl, self.yl = f(V // 10, D), np.zeros(V // 10, np.float32)
        self.per_tok = None

    def _attn(self, n_tok):
        import ctypes

        O, D, c = self.O, self.cfg["hidden_size"], self.cfg
        args = [O.p(a, O.f32p) for a in self.attn_w]
        t = time.perf_counter()
        if self.use_ref:
            O.ref().ref_mla_seq(ctypes.byref(self.c), *args, n_tok, O.p(self.attn_out, O.f32p))
        else:
            O.oracle().orc_mla_layer_seq_f32(D, c["num_attention_heads"], c["qk_nope_head_dim"], c["qk_rope_head_dim"],
                                             c["v_head_dim"], c["kv_lora_rank"], 1e-6, 10000.0, *args, n_tok,
                                             O.p(self.attn_out, O.f32p))
        return time.perf_counter() - t

    def _lin(self, w, xi, n_in, yo, n_out):
        O = self.O
        fn = O.ref().ref_linear_f32 if self.use_ref else O.oracle().orc_linear_f32
        fn(O.p(w, O.f32p), O.p(xi, O.f32p), n_in, O.p(yo, O.f32p), n_out)

    def calibrate(self):
        """Per-cached-token cost of the attention loop: positions 0..63 cost 64
        projections plus sum(pos) token visits."""
        t1 = self._attn(1)
        t64 = self._attn(64)
        self.per_tok = max(0.0, (t64 - 64 * t1) / (64 * 65 / 2))

    def sample(self):
        import ctypes

        O, cfg = self.O, self.cfg
        if self.per_tok is None:
            self.calibrate()
        t0 = time.perf_counter()
        t_attn = self._attn(1) + self.per_tok * self.ctx_len
        t = time.perf_counter()
        Id, D = cfg["intermediate_size"], self.D
        self._lin(self.wg, self.x, D, self.y, Id)
        self._lin(self.wg, self.x, D, self.y, Id)
        self._lin(self.wd, self.y, Id, self.z, D)
        t_dense = time.perf_counter() - t
        t = time.perf_counter()
        if self.use_ref:
            O.ref().ref_moe_tokens(ctypes.byref(self.c), *(O.p(a, O.f32p) for a in self.moe_w), self.Is,
                                   O.p(self.x, O.f32p), 1, O.p(self.xo, O.f32p))
        else:
            O.oracle().orc_moe_softmax_f32(*(O.p(a, O.f32p) for a in self.moe_w), self.Is, D, self.E, 6, self.I, 0,
                                           1.0, O.p(self.x, O.f32p), O.p(self.xo, O.f32p))
        t_moe = time.perf_counter() - t
        t = time.perf_counter()
        self._lin(self.wl, self.x, D, self.yl, cfg["vocab_size"] // 10)
        t_lm = (time.perf_counter() - t) * 10
        took = time.perf_counter() - t0
        L = cfg["num_hidden_layers"]
        nd = min(cfg["first_k_dense_replace"], L)
        return took, L * t_attn + nd * t_dense + (L - nd) * t_moe + t_lm


def model_cpu_baseline(cfg, ctx_len, cores=1):
    s = RefModelSample(cfg, ctx_len)
    took, sec = s.sample()
    src = "oracle/_ref (the reference's own CPU code)" if s.kind == "reference" else "the oracle restatement"
    return {"value": 1.0 / sec, "unit": "tokens/s", "cores": cores, "kind": s.kind,
            "sample": f"one token through one V2-Lite-shaped layer of each kind (attention at context {ctx_len}, "
                      f"dense MLP, MoE top-6 + 2 shared) and the lm_head on 1 thread via {src} ({took:.2f} s), "
                      f"extrapolated to {cfg['num_hidden_layers']} layers; the reference decodes one sequence at a "
                      f"time"}


def _model_ref_worker(a):
    """One host core: W untimed samples (the first also calibrates), then K
    timed ones; returns [(sample seconds, extrapolated token seconds)] and the kind."""
    cfg, ctx_len, warmup, steps = a
    s = RefModelSample(cfg, ctx_len)
    for _ in range(warmup):
        s.sample()
    return [s.sample() for _ in range(steps)], s.kind


def run_model_reference(args):
    """The reference's own CPU decode path on every host core: each core runs
    one sequence (the reference is single-sequence, single-threaded).  A step
    is a bounded sample per core (one token through one layer of each kind
    and a tenth of the lm_head); `steps` of them are run after `warmup`
    untimed ones, and each is extrapolated to a whole-model token (a full
    V2-Lite CPU token takes seconds per core)."""
    import multiprocessing as mp
    import statistics as st

    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    cfg = model_cfg(args)
    cores = os.cpu_count() or 1
    ctx_len = args.prompt + args.warmup + args.steps
    t0 = time.perf_counter()
    with mp.get_context("spawn").Pool(cores) as pool:
        res = pool.map(_model_ref_worker, [(cfg, ctx_len, args.warmup, args.steps)] * cores)
    wall = time.perf_counter() - t0
    kind = res[0][1]
    sample_s = st.mean(max(r[0][i][0] for r in res) for i in range(args.steps))  # slowest core per step
    per_tok = st.median(max(r[0][i][1] for r in res) for i in range(args.steps))
    tok_s = cores / per_tok
    line = {
        "metric": METRIC, "value": tok_s, "unit": "tokens/s", "n_gpus": args.gpus, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": sample_s * 1e3, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic (constant weights; the CPU cost does not depend on values)",
        "impl": "reference", "extrapolated": True,
        "config": {"workload": f"DeepSeek-V2-Lite-shaped greedy decode, {cfg['num_hidden_layers']} layers, one sequence "
                               f"per core at context {ctx_len}", "cores": cores,
                   "step": "per core: one token through one layer of each kind and a tenth of the lm_head (the "
                           "timed sample); value extrapolates each step to whole-model tokens",
                   "extrapolated_seconds_per_token_per_core": per_tok, "wall_s": round(wall, 1)},
        "cpu_baseline": {"value": tok_s, "unit": "tokens/s", "cores": cores, "kind": kind,
                         "sample": f"per core and step: one token through one layer of each kind and the lm_head "
                                   f"({sample_s:.2f} s), extrapolated to the full model ({per_tok:.2f} s per token)"},
        "e2e": {"value": tok_s, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def run_expert_gemm(args):
    """The dominant kernel of the model step alone (one MoE layer's expert
    gate|up GEMM at V2-Lite shape, B tokens top-6 of 64 routed experts plus the
    2 shared groups); one JSON line."""
    import torch

    import deepseek_cpp_infer_b200 as dsb

    torch.cuda.set_device(0)
    ctx = dsb.Context(0)
    stream = torch.cuda.Stream()
    ctx.set_stream(stream.cuda_stream)
    cfg = model_cfg(args)
    ms, nbytes, touched = time_expert_gemm(ctx, stream, cfg, args.batch, args.steps)
    peak, peak_kind = measured_peaks()
    print(json.dumps({"workload": "expert gate|up GEMM (routed + shared groups), V2-Lite shape", "tokens": args.batch,
                      "experts_touched": touched, "us_per_launch": ms * 1e3, "bytes_per_launch": nbytes,
                      "achieved_gbs": nbytes / (ms * 1e-3) / 1e9, "peak_gbs": peak, "peak_kind": peak_kind}),
          flush=True)
    ctx.close()


def run_attn_linears(args):
    """The attention-side linears of one V2-Lite decode layer, each alone at
    B tokens: fused q|kv_a (fp32 out), W_UK^T per head (16 groups), W_UV per
    head (16 groups), o_proj (+ residual).  Each launch reads a different
    copy of its weights (the copies together exceed L2 twice over), so every
    launch streams its weights from HBM as in the step; CUDA events on the
    context stream.  One JSON line."""
    import torch

    import deepseek_cpp_infer_b200 as dsb

    torch.cuda.set_device(0)
    ctx = dsb.Context(0)
    stream = torch.cuda.Stream()
    ctx.set_stream(stream.cuda_stream)
    B, D, H, nope, P, R, v = args.batch, 2048, 16, 128, 64, 512, 128
    QH = H * (nope + P)
    shapes = [  # name, G, M, K, x [T, ldx], x_group_col, y [T, ldy] dtype, y_group_col, epilogue
        ("q|kv_a", 1, QH + R + P, D, D, 0, QH + R + P, torch.float32, 0, dsb.EPI_STORE),
        ("W_UK^T per head", H, R, nope, QH, nope + P, H * R, torch.bfloat16, R, dsb.EPI_STORE),
        ("W_UV per head", H, v, R, H * R, R, H * v, torch.bfloat16, v, dsb.EPI_STORE),
        ("o_proj (+ residual)", 1, D, H * v, H * v, 0, D, torch.float32, 0, dsb.EPI_ADD),
    ]
    peak, peak_kind = measured_peaks()
    out = []
    for name, G, M, K, ldx, xgc, ldy, ydt, ygc, epi in shapes:
        wbytes = G * M * K * 2
        copies = max(2, -(-2 * L2_BYTES // wbytes))
        ws = [(torch.randn(G * M, K, device="cuda") * 0.02).to(torch.bfloat16) for _ in range(copies)]
        x = torch.randn(B, ldx, device="cuda").to(torch.bfloat16)
        y = torch.zeros(B, ldy, dtype=ydt, device="cuda")

        def launch(i):
            ctx.linear(ws[i % copies], x, y, M=M, K=K, G=G, x_group_col=xgc, y_group_col=ygc, epilogue=epi)

        for i in range(5):
            launch(i)
        ctx.sync()
        n = max(args.steps, 20)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for i in range(n):
            launch(i)
        e1.record(stream)
        e1.synchronize()
        us = e0.elapsed_time(e1) / n * 1e3
        nbytes = wbytes + B * G * K * 2 + B * G * M * (4 if ydt == torch.float32 else 2)
        out.append({"linear": name, "G": G, "M": M, "K": K, "us_per_launch": us, "bytes": nbytes,
                    "achieved_gbs": nbytes / (us * 1e-6) / 1e9, "frac": nbytes / (us * 1e-6) / 1e9 / peak})
        del ws
    print(json.dumps({"workload": f"V2-Lite attention-side linears, B={B} tokens, weights from HBM (rotated copies)",
                      "peak_gbs": peak, "peak_kind": peak_kind, "linears": out}), flush=True)
    ctx.close()


def fp8_peak_tflops():
    """Dense e4m3 GEMM throughput of this GPU (torch._scaled_mm, cuBLASLt,
    8192^3, 20 launches) as the tensor-roofline denominator for FP8 work."""
    import torch

    n = 8192
    a = torch.randn(n, n, device="cuda").to(torch.float8_e4m3fn)
    b = torch.randn(n, n, device="cuda").to(torch.float8_e4m3fn).t()
    one = torch.ones((), device="cuda")
    for _ in range(3):
        torch._scaled_mm(a, b, scale_a=one, scale_b=one, out_dtype=torch.bfloat16)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(20):
        torch._scaled_mm(a, b, scale_a=one, scale_b=one, out_dtype=torch.bfloat16)
    e1.record()
    e1.synchronize()
    return 2 * n ** 3 / (e0.elapsed_time(e1) / 20 * 1e-3) / 1e12


def moe_fp8_cpu_baseline(cfg, n_tokens=1):
    """The oracle's FP8 restatement of one token through k + n_shared experts
    (double accumulation, 1 core), as tokens/s of one MoE layer."""
    import numpy as np

    import oracle.model as OM

    D, I, k, ns = cfg["hidden_size"], cfg["moe_intermediate_size"], cfg["num_experts_per_tok"], cfg["n_shared_experts"]
    G = k + ns
    rng = np.random.default_rng(0)
    q = lambda *s: rng.integers(0, 0x7E, size=s, dtype=np.uint8)  # noqa: E731
    sc = lambda *s: np.full(s, 1e-3, np.float32)  # noqa: E731
    x = rng.standard_normal((n_tokens, D)).astype(np.float32)
    ids = np.tile(np.arange(G, dtype=np.int32), (n_tokens, 1))
    w = np.ones((n_tokens, G), np.float32)
    t0 = time.time()
    OM.moe_fp8(x, ids, w, q(G, I, D), sc(G, I // 128, D // 128), q(G, I, D), sc(G, I // 128, D // 128),
               q(G, D, I), sc(G, D // 128, I // 128))
    dt = time.time() - t0
    return {"value": n_tokens / dt, "unit": "tokens/s", "cores": 1, "kind": "port",
            "sample": f"{n_tokens} token(s) through {k} routed + {ns} shared FP8 experts (D={D}, I={I}) in the "
                      f"oracle's C restatement, double accumulation"}


def run_moe_fp8(args):
    """One DeepSeek-V3 MoE layer in FP8 on one GPU: fp32 router logits,
    sigmoid + bias grouped top-8, dsb_moe_ffn_fp8 (256 routed + 1 shared
    expert, D=7168, I=2048, e4m3 weights with 128x128 scales) for T tokens."""
    import numpy as np
    import torch

    import deepseek_cpp_infer_b200 as dsb
    from deepseek_cpp_infer_b200.workloads import V3_MOE, MoeFp8Weights

    cfg = dict(V3_MOE)
    if args.experts:
        cfg["n_routed_experts"] = args.experts
    torch.cuda.set_device(0)
    ctx = dsb.Context(0)
    stream = torch.cuda.Stream()
    ctx.set_stream(stream.cuda_stream)
    T, D, I = args.batch, cfg["hidden_size"], cfg["moe_intermediate_size"]
    E, k, ns = cfg["n_routed_experts"], cfg["num_experts_per_tok"], cfg["n_shared_experts"]
    layer = MoeFp8Weights(ctx, E, ns, D, I, seed=2)
    gen = torch.Generator(device="cuda").manual_seed(2)
    w_gate = torch.randn(E, D, generator=gen, device="cuda") * 0.02
    bias = torch.randn(E, generator=gen, device="cuda") * 0.01
    x = torch.randn(T, D, generator=gen, device="cuda").to(torch.bfloat16)
    x32 = x.float()
    logits = torch.empty(T, E, device="cuda")
    ids = torch.empty(T, k, dtype=torch.int32, device="cuda")
    wts = torch.empty(T, k, device="cuda")
    h = torch.zeros(T, D, device="cuda")
    torch.cuda.synchronize()

    def step():
        ctx.router_logits(x32, w_gate, logits)
        ctx.moe_route(logits, ids, wts, k, scoring=dsb.SCORE_SIGMOID, bias=bias, n_group=cfg["n_group"],
                      topk_group=cfg["topk_group"], norm_topk=cfg["norm_topk_prob"],
                      routed_scale=cfg["routed_scaling_factor"])
        ctx.moe_ffn_fp8(layer.gate_up, layer.gate_up_scale, layer.down, layer.down_scale, E=E, n_shared=ns, x=x,
                        ids=ids, weights=wts, h=h)

    def timed(fn, n):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(n):
            fn()
        e1.record(stream)
        e1.synchronize()
        ctx.sync()
        return e0.elapsed_time(e1) / n

    for _ in range(max(3, args.warmup)):
        step()
    ctx.sync()
    sampler = ClockSampler(0)
    sampler.start()
    t_probe = timed(step, 3)
    timed(step, max(1, int(1000.0 / max(t_probe, 1e-3))))
    ctx.reset_stats()
    ms = timed(step, args.steps)
    clocks = sampler.stop()
    launches = ctx.stats()["kernel_launches"] // args.steps

    picks = ids.cpu().numpy()
    touched = len(np.unique(picks)) + ns
    N = T * (k + ns)
    wbytes = touched * 3 * I * D + touched * (3 * I * D // (128 * 128)) * 4
    nbytes = wbytes + T * D * 2 + 2 * T * D * 4 + T * E * 4
    flops = 2 * N * 3 * I * D + 2 * T * E * D
    peak, peak_kind = measured_peaks()
    fp8_peak = fp8_peak_tflops()
    gbs, tfs = nbytes / (ms * 1e-3) / 1e9, flops / (ms * 1e-3) / 1e12
    bound = "hbm" if gbs / peak >= tfs / fp8_peak else "tensor"
    cpu = None if args.no_cpu_baseline else moe_fp8_cpu_baseline(cfg)
    line = {
        "metric": "DeepSeek-V3 MoE layer (FP8 experts) tokens/s", "value": T / (ms * 1e-3), "unit": "tokens/s",
        "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "e4m3 x e4m3 -> f32 (bf16 activations)",
        "data": "synthetic: N(0,0.02) weights quantised to e4m3 with 128x128 scales, N(0,1) bf16 tokens",
        "config": {"workload": f"one V3 MoE layer: router (fp32 logits, sigmoid + bias, 8 groups / top-4 / top-8, "
                               f"scale 2.5) + 256 routed and 1 shared FP8 expert, D=7168, I=2048; T={T} tokens",
                   "tokens": T, "experts_touched": int(touched), "weight_bytes": int(wbytes),
                   "l2": "every step streams the touched experts' weights (GBs), far above the 126 MB L2"},
        "roofline": {"bound": bound, "achieved": gbs if bound == "hbm" else tfs,
                     "peak": peak if bound == "hbm" else fp8_peak, "unit": "GB/s" if bound == "hbm" else "TFLOP/s",
                     "frac": gbs / peak if bound == "hbm" else tfs / fp8_peak, "traffic": None,
                     "peak_kind": peak_kind if bound == "hbm" else "measured on this GPU: torch._scaled_mm e4m3 8192^3",
                     "hbm_frac": gbs / peak, "tensor_frac": tfs / fp8_peak, "fp8_peak_tflops": fp8_peak,
                     "note": "whole layer: touched experts' e4m3 weights + scales + x, h, logits per step / step time"},
        "gpu_launches": launches, "clocks": clocks,
    }
    if cpu is not None:
        line["cpu_baseline"] = cpu
    print(json.dumps(line), flush=True)
    ctx.close()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=30)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="model",
                    choices=["model", "v3", "mla", "expert-gemm", "moe-fp8", "attn-linears"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--batch", type=int, default=0, help="sequences per GPU (0 = the workload's configuration)")
    ap.add_argument("--prompt", type=int, default=512, help="prompt tokens per sequence (model workload)")
    ap.add_argument("--layers", type=int, default=0, help="model layers (0 = the configuration's 27)")
    ap.add_argument("--trace", default="",
                    help="model workload: also write per-kernel device times of 3 traced steps per rank "
                         "(CUPTI via torch.profiler) into this directory")
    ap.add_argument("--no-fractions", action="store_true",
                    help="model workload: skip the isolated MLA (cfg2) and FP8 MoE layer (cfg3) fractions")
    ap.add_argument("--target", action="store_true",
                    help="model workload: also run the V3 target (default only at 8 GPUs)")
    ap.add_argument("--no-target", action="store_true", help="model workload: never run the V3 target")
    ap.add_argument("--target-experts", type=int, default=0,
                    help="routed experts of the V3 target (0 = 256; fewer lets one GPU exercise the path)")
    ap.add_argument("--experts", type=int, default=0,
                    help="moe-fp8 / v3: routed experts (0 = the configuration's; fewer for small profiling captures "
                         "or for one GPU standing in for one rank of an expert-parallel run)")
    args = ap.parse_args()
    if args.workload == "expert-gemm":
        args.batch = args.batch or 32
        run_expert_gemm(args)
    elif args.workload == "attn-linears":
        args.batch = args.batch or 32
        run_attn_linears(args)
    elif args.workload == "moe-fp8":
        args.batch = args.batch or 128
        run_moe_fp8(args)
    elif args.workload == "mla":
        args.batch = args.batch or 64
        run_mla_reference(args) if args.impl == "reference" else run_mla_ours(args)
    elif args.workload == "v3":
        args.batch = args.batch or 32
        args.prompt = 4096 if args.prompt == 512 else args.prompt
        if args.impl == "reference":
            print(json.dumps({"impl": "reference", "unavailable": "the reference has no FP8 dtype (safetensors parser: "
                              "F32/F16/BF16 only) and no multi-GPU path for the 671B-parameter V3 shape"}))
        else:
            run_model_ours(args)
    else:
        args.batch = args.batch or 32
        run_model_reference(args) if args.impl == "reference" else run_model_ours(args)


if __name__ == "__main__":
    main()
