"""Benchmark of the B200 decode hot path (one JSON line on rank 0).

Workload "model" (default): DeepSeek-V2-Lite-shaped batched decode - 27
layers, hidden 2048, 16 heads, kv_lora_rank 512, 1 dense + 26 MoE layers (64
experts top-6, 2 shared), vocab 102400; random-init N(0, 0.02) bf16 weights
made on the device (seed 3); B=32 sequences per GPU with 512-token random
prompts (prefilled token by token, untimed), then timed decode steps.  A step
is one dsb_decode_step: one new token for each of the 32 sequences through
every layer, greedy ids back to the host.  Under torchrun every rank runs its
own replica on its own batch (weak scaling, no collective).

Workload "mla": isolated absorbed-MLA decode attention at DeepSeek-V3 shape -
B=64, 128 heads, kv_lora_rank 512, rope 64, context U[1024, 8192] (seed 1),
64-token pages, random block table.  A step is one dsb_mla_decode call.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload model|mla]
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
# dram__bytes_read.sum + dram__bytes_write.sum of one routed-expert gate|up
# launch (B=32, V2-Lite shape) from an ncu --set full capture of
# `python bench.py --workload expert-gemm --steps 5` (716.0 MB + 4.0 MB)
EXPERT_GEMM_NCU_TRAFFIC = 719954176


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


def time_expert_gemm(ctx, stream, cfg, B, steps):
    """The dominant kernel in isolation: the expert gate|up GEMM of one MoE
    layer as the decode step runs it -- E routed groups plus n_shared shared
    groups of 2I x D bf16 weights, B*(k + n_shared) permuted token rows from a
    random top-k routing (every token also visits each shared group) -- timed
    with CUDA events on the context stream."""
    import numpy as np
    import torch

    import deepseek_cpp_infer_b200 as dsb

    D, E, k, I = cfg["hidden_size"], cfg["n_routed_experts"], cfg["num_experts_per_tok"], cfg["moe_intermediate_size"]
    ns = cfg.get("n_shared_experts", 0)
    G, kk = E + ns, k + ns
    rng = np.random.default_rng(11)
    ids = np.stack([np.concatenate([rng.choice(E, k, replace=False), E + np.arange(ns)]) for _ in range(B)])
    counts = np.bincount(ids.ravel(), minlength=G)
    offs = torch.from_numpy(np.concatenate([[0], np.cumsum(counts)]).astype(np.int32)).cuda()
    w = (torch.randn(G * 2 * I, D, device="cuda") * 0.02).to(torch.bfloat16)
    x = torch.randn(B * kk, D, device="cuda").to(torch.bfloat16)
    y = torch.empty(B * kk, I, dtype=torch.bfloat16, device="cuda")

    def launch():
        ctx.linear(w, x, y, M=2 * I, K=D, G=G, tok_offsets=offs, max_tokens_per_group=B, epilogue=dsb.EPI_SILU_GATE)

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
    nbytes = touched * 2 * I * D * 2 + B * kk * D * 2 + B * kk * I * 2
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


def run_model_ours(args):
    import numpy as np
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
    ctx = dsb.Context(local)
    stream = torch.cuda.Stream(device=dev)
    ctx.set_stream(stream.cuda_stream)
    model = dsb.Model(ctx, dsb.ModelConfig(**cfg))
    ep = None
    if world > 1:
        # expert parallel: rank r owns routed experts [r*E/world, (r+1)*E/world); attention and
        # the shared experts stay data parallel (every rank decodes its own B sequences)
        ep = dsb.EP(ctx, rank, world, cfg["n_routed_experts"], cfg["hidden_size"], cfg["num_experts_per_tok"],
                    max_tokens=B)
        handles = [None] * world
        dist.all_gather_object(handles, ep.window_handle())
        ep.connect(handles)
        model.set_ep(ep)
    model.init_random(seed=3, stddev=0.02)
    warm = max(3, args.warmup)
    total = P + warm + args.steps * 2 + 64
    max_blocks = (total + 63) // 64
    kv = dsb.KVCache(ctx, model, n_blocks=B * max_blocks, max_seqs=B, max_blocks_per_seq=max_blocks)
    seqs = [kv.alloc_seq() for _ in range(B)]
    prompts = np.random.default_rng(3 + 1000 * rank).integers(0, cfg["vocab_size"], (B, P)).astype(np.int32)
    t0 = time.time()
    v3 = args.workload == "v3"
    if v3:
        # a 4096-token context per sequence: synthetic N(0,1) latents in every layer's cache rows
        # (decode reads the same bytes as after a real prefill), then one token each
        for j, sq in enumerate(seqs):
            kv.fill_random(sq, P - 1, seed=4 + 1000 * rank + j)
        greedy, _ = dsb.decode_step(ctx, model, kv, seqs, prompts[:, -1])
    elif world == 1:
        # chunked prefill: every prompt row of a chunk through the layers in one pass
        greedy = dsb.prefill_prompts(ctx, model, kv, seqs, [list(p) for p in prompts])
    else:
        for i in range(P):  # token-serial prefill (expert-parallel ranks step together)
            greedy, _ = dsb.decode_step(ctx, model, kv, seqs, prompts[:, i])
    prefill_s = time.time() - t0
    nxt = greedy

    # the logits come back into pinned host memory (the copy runs at PCIe rate)
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
    ms = timed(args.steps)
    clocks = sampler.stop()
    st = ctx.stats()
    launches = st["kernel_launches"]
    ms_max = max_over_ranks(ms)
    ctx_len = kv.seq_len(seqs[0])
    # end to end: the reference's ForwardOutput carries the logits, so e2e also
    # copies every step's [B, vocab] fp32 logits back to (pinned) host memory
    barrier()
    ms_e2e = max_over_ranks(timed(args.steps, want_logits=True))
    # the dominant kernel alone, for the roofline line
    if v3:
        g_ms, g_bytes, g_touched = time_expert_gemm_fp8(ctx, stream, cfg, B, world, args.steps)
    else:
        g_ms, g_bytes, g_touched = time_expert_gemm(ctx, stream, cfg, B, args.steps)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline and not v3:
        cpu = model_cpu_baseline(cfg, ctx_len, cores=1)

    if rank == 0:
        peak, peak_kind = measured_peaks()
        tot, wbytes, kvbytes, touched = step_bytes(cfg, B, ctx_len, world)
        line = {
            "metric": METRIC, "value": world * B / (ms_max * 1e-3), "unit": "tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": warm, "ms_per_step": ms_max, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "e4m3 weights, bf16 activations" if v3 else "bf16",
            "data": ("synthetic: random-init N(0,0.02) weights quantised to e4m3 with 128x128 scales (seed 3), "
                     "N(0,1) latent cache rows for the context" if v3 else
                     "synthetic: random-init N(0,0.02) bf16 weights (seed 3), uniform random prompt ids"),
            "config": {
                "workload": (f"DeepSeek-V3-shaped batched greedy decode: {cfg['num_hidden_layers']} layers, hidden 7168, "
                             f"128 heads, q_lora 1536, kv_lora_rank 512, 3 dense (FFN 18432) + "
                             f"{cfg['num_hidden_layers'] - 3} MoE layers (256 experts top-8 sigmoid grouped, 1 shared, "
                             f"moe_inter 2048), FP8 e4m3 block-scaled projections / FFN / experts, vocab 129280; "
                             f"B={B} per GPU, {P}-token context, step = one token for every sequence" if v3 else
                             f"DeepSeek-V2-Lite-shaped batched greedy decode: {cfg['num_hidden_layers']} layers, hidden "
                             f"2048, 16 heads, kv_lora_rank 512, 1 dense + {cfg['num_hidden_layers'] - 1} MoE layers "
                             f"(64 experts top-6 softmax, 2 shared, moe_inter 1408), vocab 102400; B={B} per GPU, "
                             f"{P}-token prompts, step = one token for every sequence"),
                "global_batch": world * B, "seq_len": ctx_len,
                "parallelism": "single GPU" if world == 1 else
                               f"ep{world} routed experts (peer-memory dispatch/combine) + dp{world} attention",
                "step_bytes": tot, "weight_bytes_per_step": wbytes, "kv_bytes_per_step": kvbytes,
                "experts_touched_per_layer": round(touched, 1), "prefill_s": round(prefill_s, 2),
                "prefill": "chunked dsb_prefill (<= 4096 rows per pass)" if (world == 1 and not v3) else
                           ("synthetic cache fill" if v3 else "token by token"),
                "l2": f"every step streams {wbytes / 1e9:.1f} GB of weights per GPU, far above the 126 MB L2",
                "step_roofline_frac": tot / (ms_max * 1e-3) / 1e9 / peak,
            },
            "roofline": {"bound": "hbm", "achieved": g_bytes / (g_ms * 1e-3) / 1e9, "peak": peak, "unit": "GB/s",
                         "frac": g_bytes / (g_ms * 1e-3) / 1e9 / peak,
                         "traffic": None if v3 else EXPERT_GEMM_NCU_TRAFFIC,
                         "peak_kind": peak_kind,
                         "kernel": ("gemm_fp8_kernel (this rank's expert gate|up groups, SiLU epilogue)" if v3 else
                                    "gemm_bf16_kernel (expert gate|up: routed + shared groups, SiLU epilogue)"),
                         "note": f"{g_touched} expert groups' gate|up weights + activations per launch / "
                                 f"CUDA-event launch time ({g_ms * 1e3:.1f} us)"},
            "e2e": {"value": world * B / (ms_e2e * 1e-3), "unit": "tokens/s", "h2d_bytes_per_step": B * 4 * (2 + max_blocks),
                    "d2h_bytes_per_step": B * 4 + B * cfg["vocab_size"] * 4},
            "gpu_launches": launches, "clocks": clocks,
        }
        if cpu is not None:
            line["cpu_baseline"] = cpu
        print(json.dumps(line), flush=True)
    kv.close()
    model.close()
    if ep is not None:
        ep.close()
    ctx.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def _model_layer_times(cfg, ctx_len):
    """Seconds of the reference's CPU path for one token through one layer of
    each kind at V2-Lite shape, plus the lm_head: attention (mla_decode_step
    at position 0 - its projections dominate; the per-head attention loop over
    ctx_len cached tokens is added from a timed 64-token run), a dense MLP
    (three ds::rt::linear calls), an MoE block (moe_step with 8 experts - the
    per-token cost of 6 routed + 2 shared experts does not depend on E), and
    a 1/10 slice of the lm_head scaled by 10.  Uses oracle/_ref (the
    reference's own code) when present, else the oracle's restatements."""
    import ctypes

    import numpy as np

    import oracle as O

    D, H, R, P = cfg["hidden_size"], cfg["num_attention_heads"], cfg["kv_lora_rank"], cfg["qk_rope_head_dim"]
    nope, v, I, Id, V = cfg["qk_nope_head_dim"], cfg["v_head_dim"], cfg["moe_intermediate_size"], cfg["intermediate_size"], cfg["vocab_size"]
    Is = cfg["n_shared_experts"] * I
    use_ref = O.ref_available()
    f = lambda *shape: np.full(shape, 0.01, np.float32)  # noqa: E731  values do not change the cost
    c = O.RefConfig(hidden_size=D, num_attention_heads=H, qk_nope_head_dim=nope, qk_rope_head_dim=P, v_head_dim=v,
                    kv_lora_rank=R, num_hidden_layers=1, vocab_size=V, max_position_embeddings=64, rms_norm_eps=1e-6,
                    rope_theta=10000.0, routed_scaling_factor=1.0, n_experts=8, moe_top_k=6, moe_intermediate_size=I)
    wq, wkva, wn, wkvb, wo = f(H * (nope + P), D), f(R + P, D), np.ones(R, np.float32), f(H * (nope + v), R), f(D, H * v)
    hid = f(64, D)
    out = np.zeros((64, D), np.float32)
    args = [O.p(a, O.f32p) for a in (wq, wkva, wn, wkvb, wo, hid)]
    t = time.perf_counter()
    if use_ref:
        O.ref().ref_mla_seq(ctypes.byref(c), *args, 1, O.p(out, O.f32p))
    else:
        O.oracle().orc_mla_layer_seq_f32(D, H, nope, P, v, R, 1e-6, 10000.0, *args, 1, O.p(out, O.f32p))
    t_attn1 = time.perf_counter() - t
    # attention-loop cost per cached token: positions 0..63 cost 64 projections + sum(pos) token visits
    t = time.perf_counter()
    if use_ref:
        O.ref().ref_mla_seq(ctypes.byref(c), *args, 64, O.p(out, O.f32p))
    else:
        O.oracle().orc_mla_layer_seq_f32(D, H, nope, P, v, R, 1e-6, 10000.0, *args, 64, O.p(out, O.f32p))
    t64 = time.perf_counter() - t
    per_tok = max(0.0, (t64 - 64 * t_attn1) / (64 * 65 / 2))
    t_attn = t_attn1 + per_tok * ctx_len
    # dense MLP: gate, up [Id, D] and down [D, Id]
    wg, wd = f(Id, D), f(D, Id)
    x, y, z = f(D), np.zeros(Id, np.float32), np.zeros(D, np.float32)
    lin = (lambda w, xi, n_in, yo, n_out: O.ref().ref_linear_f32(O.p(w, O.f32p), O.p(xi, O.f32p), n_in, O.p(yo, O.f32p), n_out)) \
        if use_ref else (lambda w, xi, n_in, yo, n_out: O.oracle().orc_linear_f32(O.p(w, O.f32p), O.p(xi, O.f32p), n_in, O.p(yo, O.f32p), n_out))
    t = time.perf_counter()
    lin(wg, x, D, y, Id)
    lin(wg, x, D, y, Id)
    lin(wd, y, Id, z, D)
    t_dense = time.perf_counter() - t
    del wg, wd
    # MoE block, 8 experts top-6 plus 2 shared (moe_step)
    E = 8
    eg, eu, ed = f(E, I, D), f(E, I, D), f(E, D, I)
    sg, su, sd, gate = f(Is, D), f(Is, D), f(D, Is), f(E, D)
    xo = np.zeros(D, np.float32)
    t = time.perf_counter()
    if use_ref:
        O.ref().ref_moe_tokens(ctypes.byref(c), *(O.p(a, O.f32p) for a in (gate, eg, eu, ed, sg, su, sd)), Is,
                               O.p(x, O.f32p), 1, O.p(xo, O.f32p))
    else:
        O.oracle().orc_moe_softmax_f32(*(O.p(a, O.f32p) for a in (gate, eg, eu, ed, sg, su, sd)), Is, D, E, 6, I, 0,
                                       1.0, O.p(x, O.f32p), O.p(xo, O.f32p))
    t_moe = time.perf_counter() - t
    del eg, eu, ed
    # lm_head: a tenth of the vocabulary, scaled
    wl = f(V // 10, D)
    yl = np.zeros(V // 10, np.float32)
    t = time.perf_counter()
    lin(wl, x, D, yl, V // 10)
    t_lm = (time.perf_counter() - t) * 10
    return t_attn, t_dense, t_moe, t_lm, ("reference" if use_ref else "port")


def _model_cpu_token_seconds(cfg, ctx_len):
    t_attn, t_dense, t_moe, t_lm, kind = _model_layer_times(cfg, ctx_len)
    L = cfg["num_hidden_layers"]
    nd = min(cfg["first_k_dense_replace"], L)
    return L * t_attn + nd * t_dense + (L - nd) * t_moe + t_lm, kind


def model_cpu_baseline(cfg, ctx_len, cores=1):
    sec, kind = _model_cpu_token_seconds(cfg, ctx_len)
    src = "oracle/_ref (the reference's own CPU code)" if kind == "reference" else "the oracle restatement"
    return {"value": 1.0 / sec, "unit": "tokens/s", "cores": cores, "kind": kind,
            "sample": f"one token through one V2-Lite-shaped layer of each kind (attention at context {ctx_len}, "
                      f"dense MLP, MoE top-6 + 2 shared) and the lm_head on 1 thread via {src}, extrapolated to "
                      f"{cfg['num_hidden_layers']} layers; the reference decodes one sequence at a time"}


def _model_ref_worker(a):
    cfg, ctx_len = a
    return _model_cpu_token_seconds(cfg, ctx_len)


def run_model_reference(args):
    """The reference's own CPU decode path on every host core: each core runs
    one sequence (the reference is single-sequence, single-threaded); a step
    is one token per core, timed per layer kind and extrapolated to the whole
    model (a full V2-Lite CPU step does not fit a few minutes)."""
    import multiprocessing as mp

    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    cfg = model_cfg(args)
    cores = os.cpu_count() or 1
    ctx_len = args.prompt + args.warmup + args.steps
    with mp.get_context("spawn").Pool(cores) as pool:
        res = pool.map(_model_ref_worker, [(cfg, ctx_len)] * cores)
    per_tok = max(r[0] for r in res)  # the slowest core bounds the aggregate
    kind = res[0][1]
    tok_s = cores / per_tok
    line = {
        "metric": METRIC, "value": tok_s, "unit": "tokens/s", "n_gpus": args.gpus, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": per_tok * 1e3, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic (constant weights; the CPU cost does not depend on values)",
        "impl": "reference",
        "config": {"workload": f"DeepSeek-V2-Lite-shaped greedy decode, {cfg['num_hidden_layers']} layers, one sequence "
                               f"per core at context {ctx_len}", "cores": cores},
        "cpu_baseline": {"value": tok_s, "unit": "tokens/s", "cores": cores, "kind": kind,
                         "sample": "per core: one token through one layer of each kind and the lm_head, timed once "
                                   "and extrapolated to the full model"},
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
    ap.add_argument("--workload", default="model", choices=["model", "v3", "mla", "expert-gemm", "moe-fp8"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--batch", type=int, default=0, help="sequences per GPU (0 = the workload's configuration)")
    ap.add_argument("--prompt", type=int, default=512, help="prompt tokens per sequence (model workload)")
    ap.add_argument("--layers", type=int, default=0, help="model layers (0 = the configuration's 27)")
    ap.add_argument("--experts", type=int, default=0,
                    help="moe-fp8 / v3: routed experts (0 = the configuration's; fewer for small profiling captures "
                         "or for one GPU standing in for one rank of an expert-parallel run)")
    args = ap.parse_args()
    if args.workload == "expert-gemm":
        args.batch = args.batch or 32
        run_expert_gemm(args)
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
