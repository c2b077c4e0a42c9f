#!/usr/bin/env python
"""MoE-layer throughput on B200 (the headline metric: MoE-layer tokens/s).

Workload: one full-size MoE layer (hidden 2048, 512 routed
experts, top-10, one shared expert, intermediate 512, affine q4 with group
64), decode at batch 1 over 1000 seeded bf16 N(0,1) tokens, one token per
call. A step is those 1000 sequential calls. Synthetic weights and tokens
(the reference publishes no dataset for this path).

  value      tokens/s with the inputs already in HBM, timed with CUDA events
             over K steps (a CUDA graph of the 1000 qmoe_forward_dev calls
             per step), max over ranks, summed over ranks.
  e2e        tokens/s through qmoe_forward with host buffers (x read from and
             out written to pinned host memory on every call), one call per
             token from C (qmoe__forward_tokens); the Python loop beside it.
  roofline   the decode kernel's algorithmic bytes per launch / its mean
             duration in the timed region (the step's graph holds only that
             kernel, one launch per token), against MEASURED_PEAKS.json
             hbm_gbs; kernel_us_cold is the same kernel timed alone after an
             L2 flush.
  prefill    configs[2] beside it: one 4096-token call on a Zipf(1.1)-biased
             layer (graph replays, CUDA events), its per-kernel split, and
             the grouped GEMMs' algorithmic FLOP rate against bf16_tflops.
  hyper_connection  the config-1 layer inside its hyper connection (4
             residual streams, low-rank 64 q4 mixers): qmoe_forward_hc per
             token, graph replays, CUDA events.
  stack      configs[3]: the 76-layer MoE-only stack (RMSNorm + MoE +
             residual) at batch 64, one CUDA graph per step, expert-parallel
             over the torchrun ranks; HBM roofline of the step's bytes.
  stream     configs[4]: the same stack streamed from pinned host memory
             into an 8 GiB HBM pool per GPU (expert-parallel over the torchrun
             ranks); tokens/s, routed-expert hit rate and host->HBM GB/s for
             batch-1 decode and a 512-token prefill.
  cpu_baseline  the reference's own moe_forward (oracle/_ref, built from the
             reference sources) on the host cores, over a bounded sample.

--impl reference times only the reference CPU path (rank 0) on the same
metric. With --gpus N > 1 (torchrun), the ranks are independent replicas
(batch-1 decode does not shard): each rank runs its own token stream.
"""
import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(ROOT, "qwen3.8-flash-next_b200")
for p in (ROOT, PKG):
    if p not in sys.path:
        sys.path.insert(0, p)

import numpy as np  # noqa: E402

D, E, K_TOP, I_DIM, G = 2048, 512, 10, 512, 64
TOKENS = 1000
SEED = 20261201
METRIC = "MoE-layer decode tokens/s (batch 1)"
UNIT = "tokens/s"


# DRAM bytes per launch (dram__bytes_read.sum + dram__bytes_write.sum) from
# one ncu --set full capture of the kernel on this workload
# (`ncu --set full --clock-control none -k regex:k_decode_fused -s 8 -c 1
#  python bench.py --eager-tokens 20`)
NCU_TRAFFIC = {"decode_fused": 21658368}


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), float(p["bf16_tflops"]), "measured"
    except Exception:
        return 6650.0, 1590.0, "fallback"


def layer_bytes_per_token():
    slot = 1769472
    return E * D * 2 + (K_TOP + 1) * slot + D * 2 + D * 2 + D * 4


def kernel_bytes_per_token():
    """Algorithmic bytes one launch moves at T=1, per kernel."""
    gu_row, d_row = D + (D // G) * 8, I_DIM // 2 + (I_DIM // G) * 4
    return {
        "decode_fused": layer_bytes_per_token(),
        "router": E * D * 2 + D * 2 + D * 2 + (E + 1) * 4,
        "topk": (E + 1) * 4 + K_TOP * 8 + 4,
        "decode_gateup": (K_TOP + 1) * I_DIM * gu_row + D * 2 + (K_TOP + 1) * I_DIM * 4 + K_TOP * 4,
        "decode_down": (K_TOP + 1) * D * d_row + (K_TOP + 1) * I_DIM * 4 + D * 4 + K_TOP * 8,
    }


class Clocks:
    """nvidia-smi sampler for the timed region."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, dev):
        self.path = tempfile.mktemp(suffix=".csv")
        self.f = open(self.path, "w")
        try:
            self.p = subprocess.Popen(["nvidia-smi", f"--id={dev}", f"--query-gpu={self.Q}",
                                       "--format=csv,noheader,nounits", "-lms", "200"],
                                      stdout=self.f, stderr=subprocess.DEVNULL)
        except Exception:
            self.p = None

    def stop(self):
        if self.p is None:
            return None
        self.p.terminate()
        try:
            self.p.wait(5)
        except Exception:
            self.p.kill()
        self.f.close()
        sm, mx, reasons = [], 0.0, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in open(self.path):
            parts = [x.strip() for x in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = max(mx, float(parts[2]))
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        os.unlink(self.path)
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


def bench_config(world=1):
    """The `config` block of the headline line, shared by both arms."""
    return {"workload": "config1: one MoE layer, decode batch 1, 1000 tokens/step",
            "hidden": D, "experts": E, "top_k": K_TOP, "shared_experts": 1,
            "moe_inter": I_DIM, "quant": "affine q4 g64 (bf16 scale/bias)",
            "tokens_per_step": TOKENS, "parallelism": f"replicas x{world}",
            "l2": "inputs larger than L2: 906 MB of experts per layer vs 126 MB L2; "
                  "router and shared expert (3.9 MB) stay L2-resident across tokens",
            "activations": "decode: x as 16-bit and h as 24-bit block fixed point (one power-of-two "
                           "scale per 64 values) in integer dot products with the q4 weights; "
                           "multi-token calls: expert groups of at most 4 tokens the same way "
                           "(h scaled per 32 values), larger ones on fp16 tensor-core operands "
                           "(h as an fp16 hi/lo pair), fp32 accumulation; router fp64 in a fixed "
                           "order; outputs fp32"}


def _cpu_impl():
    """The timed CPU path: the reference's own moe_forward (oracle/_ref) with
    every host thread for its BLAS calls, or the C restatement (one thread)
    when the reference build is absent. Inputs come from the checkers' own
    generator (oracle.SynthLayer / oracle.synth_tokens): nothing of the
    product library is loaded on this path."""
    import oracle
    ref, kind = oracle.reference(), "reference"
    if ref is None:
        ref, kind = oracle.restatement(), "port"
    threads = os.cpu_count() or 1
    if kind == "reference":
        ref.lib.ref_set_threads(threads)
    return oracle, ref, kind, (threads if kind == "reference" else 1)


def _margin(out, ref, what):
    out = np.asarray(out, np.float64)
    ref = np.asarray(ref, np.float64)
    mab = float(np.abs(out - ref).max())
    rr = float(np.linalg.norm(out - ref) / np.linalg.norm(ref))
    return {"max_abs": mab, "rel_rms": rr, "bars": [2e-2, 1e-3], "ok": mab <= 2e-2 and rr <= 1e-3,
            "against": what}


def cpu_reference_rate(budget_s=12.0, max_tokens=1000, gpu_out=None):
    """configs[1] on the host cores: the reference's moe_forward per token,
    experts already dequantised in its cache (steady state). With gpu_out
    (the GPU arm's outputs for the same tokens), also the parity margin of
    the sampled tokens against the reference's outputs."""
    oracle, ref, kind, cores = _cpu_impl()
    s = oracle.SynthLayer(D, E, K_TOP, I_DIM, G, SEED)
    x = oracle.synth_tokens(SEED, 0, max_tokens, D)
    # size the sample from one warm token
    ref.forward(s, x[:1])
    t0 = time.perf_counter()
    ref.forward(s, x[:1])
    per = max(time.perf_counter() - t0, 1e-4)
    n = int(min(max_tokens, max(4, budget_s / per / 2)))
    sample = x[:n]
    for t in range(n):  # warm: fills the reference's expert cache for the sample
        ref.forward(s, sample[t:t + 1])
    outs = np.empty((n, D), np.float32)
    t0 = time.perf_counter()
    for t in range(n):
        outs[t] = ref.forward(s, sample[t:t + 1])[0][0]
    dt = time.perf_counter() - t0
    if kind == "reference":
        ref.lib.ref_reset_cache()
    r = {"value": n / dt, "unit": UNIT, "cores": cores, "kind": kind,
         "sample": f"{n} config-1 decode tokens, one moe_forward call each, experts "
                   f"pre-dequantised in the reference cache; {dt:.1f} s"}
    if gpu_out is not None:
        r["parity_margin"] = _margin(gpu_out[:n], outs, f"{kind} moe_forward, the {n} sampled tokens")
    return r


def cpu_prefill_rate(gpu_out=None):
    """configs[2] on the host cores: the whole 4096-token call, one
    moe_forward(n = 4096) on the Zipf(1.1)-biased layer the GPU leg runs,
    after a first call that dequantised the touched experts into the
    reference's cache (steady state). With gpu_out, the parity margin of all
    4096 GPU output rows against the reference's."""
    oracle, ref, kind, cores = _cpu_impl()
    s = oracle.SynthLayer(D, E, K_TOP, I_DIM, G, SEED, 1, zipf_s=1.1)
    x = oracle.synth_tokens(SEED, 3, PREFILL_T, D)
    t0 = time.perf_counter()
    ref.forward(s, x)
    fill = time.perf_counter() - t0
    t0 = time.perf_counter()
    out = ref.forward(s, x)[0]
    dt = time.perf_counter() - t0
    if kind == "reference":
        ref.lib.ref_reset_cache()
    r = {"value": PREFILL_T / dt, "unit": "tokens/s", "cores": cores, "kind": kind,
         "ms_per_call": 1e3 * dt,
         "sample": f"the full config-2 call: one moe_forward of {PREFILL_T} tokens, experts "
                   f"pre-dequantised (the first call, {fill:.1f} s, filled the cache); {dt:.1f} s"}
    if gpu_out is not None:
        r["parity_margin"] = _margin(gpu_out, out, f"{kind} moe_forward, all {PREFILL_T} rows")
    return r


def cpu_stack_rate(seed, stream, n_tokens, zipf, sample_layers, per_call, label):
    """configs[3]/[4] on the host cores: the stack h <- h + MoE_l(RMSNorm(h))
    over its first `sample_layers` layers (the reference's kernel_rmsnorm,
    c/src/kernel.c:10-20, and moe_forward), each layer timed after a warm
    pass that dequantised its touched experts into the reference's cache;
    the step time is the mean layer time x 76 (extrapolated). per_call
    tokens go through moe_forward at once (1: batch-1 decode, one token per
    call)."""
    oracle, ref, kind, cores = _cpu_impl()
    h = oracle.synth_tokens(seed, stream, n_tokens, D)
    times = []
    for l in range(sample_layers):
        s = oracle.SynthLayer(D, E, K_TOP, I_DIM, G, seed, l, zipf_s=zipf)

        def layer(h):
            out = np.empty_like(h)
            for a in range(0, n_tokens, per_call):
                y, _, _ = ref.forward(s, oracle.rmsnorm(h[a:a + per_call], 1e-6))
                out[a:a + per_call] = h[a:a + per_call] + y
            return out

        layer(h)  # warm: the touched experts into the cache
        t0 = time.perf_counter()
        h = layer(h)
        times.append(time.perf_counter() - t0)
        if kind == "reference":
            ref.lib.ref_reset_cache()
    step = statistics.mean(times) * STACK_L
    return {"value": n_tokens / step, "unit": "tokens/s", "cores": cores, "kind": kind,
            "ms_per_step": 1e3 * step, "extrapolated": True,
            "sample": f"{label}: layers 0-{sample_layers - 1} of the 76 timed ({n_tokens} tokens, "
                      f"{per_call} per moe_forward call, RMSNorm + moe_forward + residual, experts "
                      f"pre-dequantised), mean layer time x 76; {sum(times):.1f} s timed"}


def run_reference(args):
    """--impl reference: the reference's own CPU moe_forward on the host
    cores, on the GPU arm's metric and config, one bounded sample per step
    (8 decode tokens, one call each; the per-token rate is the metric).
    Rank 0 only; inputs from the checkers' generator, so the product library
    is never loaded here."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    oracle, ref, kind, cores = _cpu_impl()
    x = oracle.synth_tokens(SEED, 0, 64, D)
    s = oracle.SynthLayer(D, E, K_TOP, I_DIM, G, SEED)
    per_step = 8
    sample = x[:per_step]
    for _ in range(max(args.warmup, 1)):
        for t in range(per_step):
            ref.forward(s, sample[t:t + 1])
    t0 = time.perf_counter()
    for _ in range(args.steps):
        for t in range(per_step):
            ref.forward(s, sample[t:t + 1])
    dt = time.perf_counter() - t0
    v = args.steps * per_step / dt
    line = {
        "impl": "reference", "metric": METRIC, "value": v, "unit": UNIT, "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * dt / args.steps,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic",
        "config": bench_config(args.gpus),
        "sample_tokens_per_step": per_step,
        "cpu_baseline": {"value": v, "unit": UNIT, "cores": cores, "kind": kind,
                         "sample": f"{per_step} of the step's {TOKENS} config-1 tokens per timed "
                                   "step (a bounded sample: tokens/s is a per-token rate), one "
                                   "moe_forward call each, experts pre-dequantised (steady state)"},
        "e2e": {"value": v, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


PREFILL_T = 4096
PREFILL_FLOP = 283467841536  # 4096 tokens x 11 experts x 6 d I (gate, up, down)


def run_prefill_eager(n):
    """Small case for ncu captures of the prefill kernels: n eager calls of
    the config-2 layer (4096 tokens, Zipf(1.1) router bias)."""
    import torch

    import qmoe
    cfg = qmoe.make_config(D, E, K_TOP, I_DIM, G, max_tokens=PREFILL_T)
    layer = qmoe.SynthLayer(cfg, SEED, zipf_s=1.1)
    ctx = qmoe.Context(cfg)
    ctx.upload(0, layer)
    x = torch.from_numpy(qmoe.synth_tokens(SEED, 3, PREFILL_T, D)).cuda().to(torch.bfloat16)
    out = torch.empty((PREFILL_T, D), dtype=torch.float32, device="cuda")
    torch.cuda.synchronize()
    for _ in range(n):
        ctx.forward_dev(0, x.data_ptr(), qmoe.QMOE_BF16, PREFILL_T, out.data_ptr(), None)
    ctx.sync()
    ctx.close()
    print(f"prefill eager case: {n} calls ok")


def measure_prefill(ctx, layer_index, rank, reps=5, warmup=3):
    """configs[2] on this rank's GPU: whole-call time (graph replays, CUDA
    events on the launching stream) and the per-kernel split."""
    import torch

    import qmoe
    x = torch.from_numpy(qmoe.synth_tokens(SEED, 3 + rank, PREFILL_T, D)).cuda().to(torch.bfloat16)
    out = torch.empty((PREFILL_T, D), dtype=torch.float32, device="cuda")
    st = torch.cuda.Stream()
    cs = st.cuda_stream
    torch.cuda.synchronize()
    ctx.forward_dev(layer_index, x.data_ptr(), qmoe.QMOE_BF16, PREFILL_T, out.data_ptr(), cs)
    st.synchronize()
    ctx.sync()
    ctx.capture_begin(cs)
    ctx.forward_dev(layer_index, x.data_ptr(), qmoe.QMOE_BF16, PREFILL_T, out.data_ptr(), cs)
    g = ctx.capture_end(cs)
    for _ in range(warmup):
        g.launch(cs)
    st.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(st)
    for _ in range(reps):
        g.launch(cs)
    e1.record(st)
    st.synchronize()
    ctx.sync()
    ms = e0.elapsed_time(e1) / reps
    out_host = out.cpu().numpy()
    us = ctx.profile_forward(layer_index, x.data_ptr(), qmoe.QMOE_BF16, PREFILL_T, out.data_ptr(), reps)
    names = ["route_tc", "route_exact", "group_gather", "gemm_gateup", "gemm_down", "combine"]
    split = {n: float(u) for n, u in zip(names, us)}
    gemm_us = split.get("gemm_gateup", 0.0) + split.get("gemm_down", 0.0)
    _, bf16, src = peaks()
    tf = PREFILL_FLOP / (gemm_us * 1e-6) / 1e12 if gemm_us > 0 else None
    del g
    return {"workload": "config2: one MoE layer, prefill 4096 tokens, Zipf(1.1) router bias",
            "_out": out_host,
            "tokens_per_s": PREFILL_T / (ms / 1e3), "ms_per_call": ms, "kernel_us": split,
            "gpu_launches_per_call": 10,
            "gemm": {"bound": "tensor", "achieved": tf, "peak": bf16, "unit": "TFLOP/s",
                     "frac": (tf / bf16) if tf else None, "flop_per_call": PREFILL_FLOP,
                     "peak_source": src, "note": "algorithmic FLOPs of the two grouped GEMMs "
                     "over their event-timed durations; the down GEMM issues two fp16 MMAs "
                     "(h as a hi/lo pair) per algorithmic one"}}


HC_N, HC_LR, HC_SEED = 4, 64, 20261213


def measure_hc(ctx, rank, reps=5, warmup=3):
    """The config-1 layer inside its hyper connection (hc 4 residual streams,
    low-rank 64 q4 mixers), decode at batch 1: TOKENS sequential
    qmoe_forward_hc calls (gated_residual, the MoE block, the inject-add: one
    decode-kernel launch each) on
    h [TOKENS, hc*d] fp32, captured as one CUDA graph and replayed. The first
    replay's rows are the parity sample (each row depends only on its own
    input); later replays keep updating h in place."""
    import torch

    import qmoe
    H = qmoe.SynthHC(D, HC_N, HC_LR, HC_SEED)
    ctx.upload_hc(0, H)
    h0 = np.ascontiguousarray(np.concatenate(
        [qmoe.synth_tokens(SEED, 40 + rank * HC_N + j, TOKENS, D) for j in range(HC_N)], axis=1))
    h = torch.from_numpy(h0).cuda()
    st = torch.cuda.Stream()
    cs = st.cuda_stream
    row = HC_N * D * 4
    torch.cuda.synchronize()
    for t in range(4):  # eager warm-up on scratch rows (restored below)
        ctx.forward_hc(0, h.data_ptr() + t * row, 1, cs)
    st.synchronize()
    ctx.sync()
    h.copy_(torch.from_numpy(h0))
    torch.cuda.synchronize()
    ctx.capture_begin(cs)
    for t in range(TOKENS):
        ctx.forward_hc(0, h.data_ptr() + t * row, 1, cs)
    g = ctx.capture_end(cs)
    g.launch(cs)
    st.synchronize()
    first = h.cpu().numpy()
    for _ in range(warmup):
        g.launch(cs)
    st.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(st)
    for _ in range(reps):
        g.launch(cs)
    e1.record(st)
    st.synchronize()
    ctx.sync()
    ms = e0.elapsed_time(e1) / reps
    del g
    return {"workload": f"config1 layer inside a hyper connection (hc {HC_N}, lowrank {HC_LR}, "
                        f"q4 mixers), decode batch 1, {TOKENS} tokens/step",
            "_h0": h0, "_out": first,
            "tokens_per_s": TOKENS / (ms / 1e3), "us_per_token": 1e3 * ms / TOKENS,
            "gpu_launches_per_token": 1,
            "note": "per token one decode-kernel launch: its prologue computes gated_residual "
                    "(RMSNorm of the hc streams, the low-rank down mixer and the inject weights; "
                    "grid barrier; the up mixer and the stream mean, the block's input; grid "
                    "barrier), then the MoE block, whose combine also adds inject x output to "
                    "the hc streams; h fp32 in HBM"}


def cpu_hc_rate(h0, gpu_out, budget_s=10.0):
    """The hyper-connection leg on the host cores: the reference's own
    gated_residual + moe_forward + inject-add (ref_hc_moe_step, built from
    its sources) per token, experts pre-dequantised (steady state); the
    parity margin of the sampled rows' contribution h' - h0 against the GPU's."""
    oracle, ref, kind, cores = _cpu_impl()
    s = oracle.SynthLayer(D, E, K_TOP, I_DIM, G, SEED)
    H = oracle.SynthHC(D, HC_N, HC_LR, HC_SEED)
    ref.hc_moe_step(H, s, h0[:1])
    t0 = time.perf_counter()
    ref.hc_moe_step(H, s, h0[:1])
    per = max(time.perf_counter() - t0, 1e-4)
    n = int(min(len(h0), max(4, budget_s / per / 2)))
    for t in range(n):  # warm: the sample's experts into the reference cache
        ref.hc_moe_step(H, s, h0[t:t + 1])
    outs = np.empty((n, h0.shape[1]), np.float32)
    t0 = time.perf_counter()
    for t in range(n):
        outs[t] = ref.hc_moe_step(H, s, h0[t:t + 1])[0]
    dt = time.perf_counter() - t0
    if kind == "reference":
        ref.lib.ref_reset_cache()
    r = {"value": n / dt, "unit": "tokens/s", "cores": cores, "kind": kind,
         "sample": f"{n} tokens of the hyper-connection leg, one hc step each "
                   f"(gated_residual, moe_forward, inject-add), experts pre-dequantised; {dt:.1f} s"}
    r["parity_margin"] = _margin(gpu_out[:n] - h0[:n], outs - h0[:n],
                                 f"{kind} hc step, the {n} sampled tokens (h' - h)")
    return r


def exchange_label(ctx):
    """How a connected expert-parallel context moves its rows."""
    import ctypes

    import qmoe
    f = qmoe.lib().qmoe__ep_p2p
    f.restype, f.argtypes = ctypes.c_int, [ctypes.c_void_p]
    if f(ctx.h):
        return ("peer memory over NVLink: each rank writes its rows into the owners' receive rows and "
                "the partial rows into the token owners' return rows (CUDA IPC mappings), flags "
                "released and acquired at system scope")
    return "NCCL send/recv, fixed-size blocks of rows and fp32 partials"


def measure_prefill_ep(rank, world, local, local_ctx=None, local_layer=1, reps=5, warmup=2):
    """configs[2] expert-parallel over the torchrun ranks: the 4096 tokens
    split evenly, rank g owning experts [g E/W, (g+1) E/W), qmoe_forward_ep
    on each rank (NCCL through the library). Whole-call time = max over
    ranks of the CUDA-event time per call. ep_parity: every rank's output
    rows against the single-GPU path (local_ctx, the same layer with all
    experts, itself parity-tested against the reference) on the same tokens,
    worst margins over the ranks."""
    import torch
    import torch.distributed as dist

    import qmoe
    T_per = PREFILL_T // world
    cfg = qmoe.make_config(D, E, K_TOP, I_DIM, G, max_tokens=T_per, device=local,
                           ep_rank=rank, ep_world=world)
    ctx = qmoe.Context(cfg)
    ctx.upload(0, qmoe.SynthLayer(cfg, SEED, 1, zipf_s=1.1))
    uid = torch.zeros(128, dtype=torch.uint8, device="cuda")
    if rank == 0:
        uid.copy_(torch.frombuffer(bytearray(qmoe.ep_unique_id()), dtype=torch.uint8))
    dist.broadcast(uid, 0)
    ctx.ep_connect(bytes(uid.cpu().numpy().tobytes()))
    x_all = qmoe.synth_tokens(SEED, 3, PREFILL_T, D)
    x = torch.from_numpy(x_all[rank * T_per:(rank + 1) * T_per]).cuda().to(torch.bfloat16)
    out = torch.empty((T_per, D), dtype=torch.float32, device="cuda")
    st = torch.cuda.Stream()
    cs = st.cuda_stream
    torch.cuda.synchronize()
    for _ in range(warmup):
        ctx.forward_ep(0, x.data_ptr(), qmoe.QMOE_BF16, T_per, out.data_ptr(), cs)
    st.synchronize()
    ctx.sync()
    dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(st)
    for _ in range(reps):
        ctx.forward_ep(0, x.data_ptr(), qmoe.QMOE_BF16, T_per, out.data_ptr(), cs)
    e1.record(st)
    st.synchronize()
    ctx.sync()
    tt = torch.tensor([e0.elapsed_time(e1) / reps], device="cuda")
    dist.all_reduce(tt, op=dist.ReduceOp.MAX)
    ms = float(tt.item())
    xchg = exchange_label(ctx)
    ctx.close()
    ep_parity = None
    if local_ctx is not None:
        ref = torch.empty_like(out)
        local_ctx.forward_dev(local_layer, x.data_ptr(), qmoe.QMOE_BF16, T_per, ref.data_ptr(), cs)
        st.synchronize()
        local_ctx.sync()
        a, b = out.double(), ref.double()
        m = torch.tensor([float((a - b).abs().max()), float((a - b).norm() / b.norm())], device="cuda")
        dist.all_reduce(m, op=dist.ReduceOp.MAX)
        ep_parity = {"max_abs": float(m[0]), "rel_rms": float(m[1]), "bars": [2e-2, 1e-3],
                     "ok": float(m[0]) <= 2e-2 and float(m[1]) <= 1e-3,
                     "against": "the single-GPU path on the same tokens, every rank's rows, worst rank"}
    return {"workload": "config2 expert-parallel: 4096 tokens split over the ranks, Zipf(1.1)",
            "ranks": world, "tokens_per_s": PREFILL_T / (ms / 1e3), "ms_per_call": ms,
            "scaling": "strong", "timing": "CUDA events per rank, max over ranks",
            "exchange": xchg,
            "ep_parity": ep_parity}


STACK_L, STACK_T, STACK_SEED = 76, 64, 20261203
SLOT = 1769472


def measure_stack(rank, world, local, layers=STACK_L, reps=3, warmup=2):
    """the 76-layer MoE-only stack (h <- h + MoE_l(RMSNorm(h)),
    eps 1e-6), decode at batch 64, every layer with its own seeded router and
    experts (generated on the device: 68.9 GB of experts at one GPU). With
    world > 1 the ranks are expert-parallel (rank g owns experts
    [g E/W, (g+1) E/W) of every layer, 64/W tokens each, NCCL exchange inside
    the library). One step = the whole stack for the 64 tokens, captured as
    one CUDA graph per rank (inputs reset from a resident copy inside the
    graph); time = CUDA events per rank, max over ranks."""
    import torch
    import torch.distributed as dist

    import qmoe
    T_per = STACK_T // world
    cfg = qmoe.make_config(D, E, K_TOP, I_DIM, G, layers=layers, max_tokens=T_per, device=local,
                           ep_rank=rank if world > 1 else 0, ep_world=world if world > 1 else 0)
    ctx = qmoe.Context(cfg)
    t0 = time.perf_counter()
    for l in range(layers):
        ctx.synth_layer_dev(l, STACK_SEED)
    ctx.sync()
    synth_s = time.perf_counter() - t0
    if world > 1:
        uid = torch.zeros(128, dtype=torch.uint8, device="cuda")
        if rank == 0:
            uid.copy_(torch.frombuffer(bytearray(qmoe.ep_unique_id()), dtype=torch.uint8))
        dist.broadcast(uid, 0)
        ctx.ep_connect(bytes(uid.cpu().numpy().tobytes()))
    h0 = torch.from_numpy(qmoe.synth_tokens(STACK_SEED, 100 + rank, T_per, D)).cuda()
    h = h0.clone()
    st = torch.cuda.Stream()
    cs = st.cuda_stream
    torch.cuda.synchronize()
    ep_parity = None
    if world > 1:
        # layer 0 expert-parallel against the single-GPU path on this rank's
        # tokens (a local context holding all of layer 0's experts)
        hc = h0.clone()
        ctx.forward_stack(0, 1, hc.data_ptr(), T_per, 1e-6, cs)
        st.synchronize()
        ctx.sync()
        lc = qmoe.Context(qmoe.make_config(D, E, K_TOP, I_DIM, G, layers=1, max_tokens=T_per,
                                           device=local))
        lc.synth_layer_dev(0, STACK_SEED)
        hl = h0.clone()
        lc.forward_stack(0, 1, hl.data_ptr(), T_per, 1e-6, cs)
        st.synchronize()
        lc.sync()
        lc.close()
        a, b = (hc - h0).double(), (hl - h0).double()
        m = torch.tensor([float((a - b).abs().max()), float((a - b).norm() / b.norm())], device="cuda")
        dist.all_reduce(m, op=dist.ReduceOp.MAX)
        ep_parity = {"max_abs": float(m[0]), "rel_rms": float(m[1]), "bars": [2e-2, 1e-3],
                     "ok": float(m[0]) <= 2e-2 and float(m[1]) <= 1e-3,
                     "against": "layer 0 on the single-GPU path, same tokens, every rank, worst rank"}
    # census pass, layer by layer: the distinct experts each layer touches
    # (over all ranks' tokens), for the algorithmic bytes of a step
    lo, hi = rank * E // world, (rank + 1) * E // world
    touched = []
    for l in range(layers):
        ctx.forward_stack(l, l + 1, h.data_ptr(), T_per, 1e-6, cs)
        st.synchronize()
        idx = torch.from_numpy(ctx.routing(T_per)[0]).cuda()
        if world > 1:
            parts = [torch.empty_like(idx) for _ in range(world)]
            dist.all_gather(parts, idx)
            idx = torch.cat(parts)
        u = torch.unique(idx)
        touched.append(int(((u >= lo) & (u < hi)).sum()))
    h_eager = h.clone()
    # one graph per rank for the whole step
    ctx.capture_begin(cs)
    with torch.cuda.stream(st):
        h.copy_(h0)
    ctx.forward_stack(0, layers, h.data_ptr(), T_per, 1e-6, cs)
    g = ctx.capture_end(cs)
    for _ in range(warmup):
        g.launch(cs)
    st.synchronize()
    ctx.sync()
    same = bool(torch.equal(h, h_eager))
    if world > 1:
        dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(st)
    for _ in range(reps):
        g.launch(cs)
    e1.record(st)
    st.synchronize()
    ctx.sync()
    ms = e0.elapsed_time(e1) / reps
    stats = torch.tensor([ms, float(sum(touched)), 0.0 if same else 1.0], device="cuda")
    if world > 1:
        mx = stats.clone()
        dist.all_reduce(mx, op=dist.ReduceOp.MAX)
        sm = stats.clone()
        dist.all_reduce(sm, op=dist.ReduceOp.SUM)
        ms, all_touched, bad = float(mx[0]), float(sm[1]), float(mx[2])
    else:
        all_touched, bad = float(stats[1]), float(stats[2])
    g.close()
    xchg = exchange_label(ctx) if world > 1 else None
    ctx.close()
    # algorithmic bytes of one step, all ranks: every rank reads the router,
    # shared gate and shared expert of every layer, and its own touched experts
    per_layer_fixed = E * D * 2 + D * 2 + SLOT
    step_bytes = world * layers * per_layer_fixed + all_touched * SLOT
    hbm, _, src = peaks()
    gbs = step_bytes / (ms / 1e3) / 1e9
    return {"workload": f"config3: {layers}-layer MoE-only stack, decode batch {STACK_T}, "
                        "RMSNorm eps 1e-6 + residual",
            "ranks": world, "parallelism": f"ep{world}" if world > 1 else "single GPU",
            "tokens_per_s": STACK_T / (ms / 1e3), "ms_per_step": ms,
            "tokens_per_step": STACK_T, "layers": layers,
            "experts_touched_per_layer": all_touched / layers,
            "roofline": {"bound": "hbm", "achieved": gbs, "peak": hbm * world, "unit": "GB/s",
                         "frac": gbs / (hbm * world), "bytes_per_step": step_bytes,
                         "peak_source": f"{src}, x{world} GPUs",
                         "note": "router + shared expert + shared gate per layer per rank, "
                                 "plus the distinct routed experts the step touches"},
            "graph_equals_eager": bad == 0.0, "weights_generated_s": synth_s,
            "timing": "one CUDA graph per rank per step, CUDA events, max over ranks",
            "exchange": xchg,
            "ep_parity": ep_parity}


STREAM_LAYERS, STREAM_POOL_76, STREAM_DECODE, STREAM_PREFILL = 76, 8 * 2 ** 30, 16, 512


def mem_available():
    try:
        for line in open("/proc/meminfo"):
            if line.startswith("MemAvailable:"):
                return int(line.split()[1]) * 1024
    except OSError:
        pass
    return 0


def measure_stream(rank=0, world=1, local=0, layers=STREAM_LAYERS):
    """the MoE-only stack streamed from pinned host memory,
    Zipf(1.1) routing with a per-layer permutation, an adaptive HBM pool of
    8 GiB per GPU and route-predicted prefetches of depth 2 (the reference's
    prefetch_count). With world > 1 the ranks are expert-parallel (rank g
    streams experts [g E/W, (g+1) E/W) into its own pool; the batch-1 decode
    token lives on rank 0 and travels to the owners of its experts). The
    stack has `layers` of the 76 layers (the pinned stores of all ranks hold
    layers x 906 MB, 68.9 GB for all 76; fewer layers when that is more than
    half the host's available memory), and the pool is pro rata to 76
    layers. Decode: STREAM_DECODE seeded tokens, one at a time through the
    whole stack; prefill: one STREAM_PREFILL-token call through the stack,
    split over the ranks. CUDA events on the stream (the host's waits for
    fills show as the stream's idle time), max over ranks."""
    import torch
    import torch.distributed as dist

    import qmoe
    store_all = E * SLOT  # per layer, all ranks together
    avail = mem_available()
    if avail and layers * store_all * 2 > avail:
        layers = max(2, int(avail // (2 * store_all)))
    if world > 1:
        t = torch.tensor([layers], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MIN)
        layers = int(t.item())
    pool = int(STREAM_POOL_76 * layers / STACK_L)
    T_per = STREAM_PREFILL // world
    cfg = qmoe.make_config(D, E, K_TOP, I_DIM, G, layers=layers, max_tokens=T_per, pool_bytes=pool,
                           prefetch=2, device=local, ep_rank=rank if world > 1 else 0,
                           ep_world=world if world > 1 else 0)
    ctx = qmoe.Context(cfg)
    t0 = time.perf_counter()
    for l in range(layers):
        ctx.synth_layer_dev(l, STACK_SEED + 1, 1.1)
    ctx.sync()
    synth_s = time.perf_counter() - t0
    if world > 1:
        uid = torch.zeros(128, dtype=torch.uint8, device="cuda")
        if rank == 0:
            uid.copy_(torch.frombuffer(bytearray(qmoe.ep_unique_id()), dtype=torch.uint8))
        dist.broadcast(uid, 0)
        ctx.ep_connect(bytes(uid.cpu().numpy().tobytes()))
    h0 = torch.from_numpy(qmoe.synth_tokens(STACK_SEED + 1, 200, STREAM_PREFILL, D)).cuda()
    st = torch.cuda.Stream()
    cs = st.cuda_stream
    torch.cuda.synchronize()
    keys = ("expert_loads", "expert_bytes", "expert_wait_seconds", "prefetch_issued", "prefetch_hits",
            "routed_lookups", "routed_hits", "prefetch_wasted")

    def counters():
        a = ctx.stats()
        return [float(a[k]) for k in keys]

    def leg(run, n_tokens):
        c0 = counters()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(st)
        run()
        e1.record(st)
        st.synchronize()
        ctx.sync()
        ms = e0.elapsed_time(e1)
        dc = [b - a for a, b in zip(c0, counters())]
        if world > 1:
            mx = torch.tensor([ms], device="cuda")
            dist.all_reduce(mx, op=dist.ReduceOp.MAX)
            sm = torch.tensor(dc, device="cuda", dtype=torch.float64)
            dist.all_reduce(sm, op=dist.ReduceOp.SUM)
            ms, dc = float(mx.item()), [float(v) for v in sm]
        d = dict(zip(keys, dc))
        return {"tokens_per_s": n_tokens / (ms / 1e3), "ms": ms,
                "hit_rate": d["routed_hits"] / max(1.0, d["routed_lookups"]),
                "routed_experts": int(d["routed_lookups"]), "expert_fills": int(d["expert_loads"]),
                "h2d_bytes": int(d["expert_bytes"]),
                "h2d_gbs_over_leg": d["expert_bytes"] / (ms / 1e3) / 1e9,
                "host_blocked_s_in_fills": d["expert_wait_seconds"],
                "prefetch_issued": int(d["prefetch_issued"]), "prefetch_hits": int(d["prefetch_hits"]),
                "prefetch_wasted": int(d["prefetch_wasted"])}

    hd = torch.empty((1, D), dtype=torch.float32, device="cuda")
    n_dec = 1 if rank == 0 else 0  # one token per step, on rank 0

    def decode(tokens):
        def run():
            for t in tokens:
                with torch.cuda.stream(st):
                    hd.copy_(h0[t:t + 1])
                ctx.forward_stack(0, layers, hd.data_ptr(), n_dec, 1e-6, cs)
        return run

    decode(range(4))()  # warm-up: the pool and the route statistics start filling
    st.synchronize()
    dec = leg(decode(range(4, 4 + STREAM_DECODE)), STREAM_DECODE)
    hp = torch.empty((T_per, D), dtype=torch.float32, device="cuda")

    def prefill():
        with torch.cuda.stream(st):
            hp.copy_(h0[rank * T_per:(rank + 1) * T_per])
        ctx.forward_stack(0, layers, hp.data_ptr(), T_per, 1e-6, cs)

    pre = leg(prefill, STREAM_PREFILL)
    ctx.close()
    return {"workload": f"config4: {layers} of the 76 stack layers streamed from pinned host memory, "
                        f"HBM pool {pool / 2 ** 30:.2f} GiB per GPU (8 GiB x {layers}/76), Zipf(1.1) "
                        "with a per-layer permutation, prefetch depth 2",
            "ranks": world, "parallelism": f"ep{world}" if world > 1 else "single GPU",
            "layers": layers, "pool_bytes_per_gpu": pool, "host_store_bytes": layers * store_all,
            "host_mem_available": avail, "decode_batch1": dec,
            "prefill": {**pre, "tokens": STREAM_PREFILL}, "weights_generated_s": synth_s,
            "timing": "CUDA events on the stream, max over ranks; the host's wait for each layer's "
                      "routing is inside",
            "note": "fills and prefetches are queued on a copy stream behind the work they may "
                    "evict from; each layer's kernels wait for them on the device, the host only "
                    "for the layer's routing"}


def run_stack_eager(layers):
    """Small case for ncu captures: one eager pass of a `layers`-layer stack
    (configs[3] shapes, 64 tokens, weights generated on the device)."""
    import torch

    import qmoe
    cfg = qmoe.make_config(D, E, K_TOP, I_DIM, G, layers=layers, max_tokens=STACK_T)
    ctx = qmoe.Context(cfg)
    for l in range(layers):
        ctx.synth_layer_dev(l, STACK_SEED)
    h = torch.from_numpy(qmoe.synth_tokens(STACK_SEED, 100, STACK_T, D)).cuda()
    torch.cuda.synchronize()
    ctx.forward_stack(0, layers, h.data_ptr(), STACK_T, 1e-6, None)
    ctx.sync()
    ctx.close()
    print(f"stack case: {layers} layers x {STACK_T} tokens ok")


def run_stream_eager(n):
    """Small case for ncu captures of the per-token kernels: n single-token
    forwards of one streamed config-1 layer (Zipf(1.1) routing, a pool of 64
    expert slots): routing on the device (k_router, k_topk), misses filled
    from pinned host memory, then k_decode_gateup and k_decode_down."""
    import torch

    import qmoe
    cfg = qmoe.make_config(D, E, K_TOP, I_DIM, G, max_tokens=1, pool_bytes=64 * SLOT, prefetch=0)
    ctx = qmoe.Context(cfg)
    ctx.synth_layer_dev(0, STACK_SEED + 1, 1.1)
    x = torch.from_numpy(qmoe.synth_tokens(SEED, 0, n, D)).cuda()
    out = torch.empty((n, D), dtype=torch.float32, device="cuda")
    torch.cuda.synchronize()
    for t in range(n):
        ctx.forward_dev(0, x.data_ptr() + t * D * 4, qmoe.QMOE_F32, 1, out.data_ptr() + t * D * 4, None)
    ctx.sync()
    ctx.close()
    print(f"stream case: {n} tokens ok")


def run_hc_eager(n):
    """Small case for ncu captures of the hyper-connection kernels: n eager
    qmoe_forward_hc calls of one token (k_hc_pre1 and the decode kernel with
    the inject-add), then one call of 8 tokens (k_hc_down, k_hc_up, the
    grouped path, k_hc_inject), on the config-1 layer."""
    import torch

    import qmoe
    cfg = qmoe.make_config(D, E, K_TOP, I_DIM, G, max_tokens=8)
    ctx = qmoe.Context(cfg)
    ctx.upload(0, qmoe.SynthLayer(cfg, SEED))
    ctx.upload_hc(0, qmoe.SynthHC(D, HC_N, HC_LR, HC_SEED))
    h = torch.from_numpy(np.concatenate(
        [qmoe.synth_tokens(SEED, 40 + j, n + 8, D) for j in range(HC_N)], axis=1)).cuda()
    torch.cuda.synchronize()
    row = HC_N * D * 4
    for t in range(n):
        ctx.forward_hc(0, h.data_ptr() + t * row, 1, None)
    ctx.forward_hc(0, h.data_ptr() + n * row, 8, None)
    ctx.sync()
    ctx.close()
    print(f"hc case: {n} single-token calls and one 8-token call ok")


def run_eager(n):
    """Small case for ncu captures: n single-token forwards launched eagerly
    on the config-1 layer (906 MB of experts, larger than L2)."""
    import torch

    import qmoe
    cfg = qmoe.make_config(D, E, K_TOP, I_DIM, G, max_tokens=1)
    layer = qmoe.SynthLayer(cfg, SEED)
    ctx = qmoe.Context(cfg)
    ctx.upload(0, layer)
    x = torch.from_numpy(qmoe.synth_tokens(SEED, 0, n, D)).cuda().to(torch.bfloat16)
    out = torch.empty((n, D), dtype=torch.float32, device="cuda")
    torch.cuda.synchronize()
    for t in range(n):
        ctx.forward_dev(0, x.data_ptr() + t * D * 2, qmoe.QMOE_BF16, 1, out.data_ptr() + t * D * 4,
                        None)
    ctx.sync()
    ctx.close()
    print(f"eager case: {n} tokens ok")


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline leg")
    ap.add_argument("--eager-tokens", type=int, default=0,
                    help="profiling case: run N single-token forwards eagerly (no graph) and exit")
    ap.add_argument("--prefill-eager", type=int, default=0,
                    help="profiling case: run N eager 4096-token prefill calls and exit")
    ap.add_argument("--no-prefill", action="store_true", help="skip the configs[2] leg")
    ap.add_argument("--no-stack", action="store_true", help="skip the configs[3] leg")
    ap.add_argument("--no-stream", action="store_true", help="skip the configs[4] leg")
    ap.add_argument("--no-hc", action="store_true", help="skip the hyper-connection leg")
    ap.add_argument("--stream-only", type=int, default=0,
                    help="run only the configs[4] leg with this many layers and print it")
    ap.add_argument("--stack-eager", type=int, default=0,
                    help="profiling case: one eager pass of an N-layer configs[3] stack and exit")
    ap.add_argument("--stream-eager", type=int, default=0,
                    help="profiling case: N single-token forwards of one streamed layer and exit")
    ap.add_argument("--hc-eager", type=int, default=0,
                    help="profiling case: N single-token hyper-connection steps (and one of 8) and exit")
    ap.add_argument("--stack-only", type=int, default=0,
                    help="run only the configs[3] leg with this many layers and print it")
    args = ap.parse_args()
    if args.impl == "reference":
        run_reference(args)
        return
    if args.eager_tokens:
        run_eager(args.eager_tokens)
        return
    if args.prefill_eager:
        run_prefill_eager(args.prefill_eager)
        return
    if args.stack_eager:
        run_stack_eager(args.stack_eager)
        return
    if args.stream_eager:
        run_stream_eager(args.stream_eager)
        return
    if args.hc_eager:
        run_hc_eager(args.hc_eager)
        return
    if args.stream_only:
        import torch
        import torch.distributed as dist
        world = int(os.environ.get("WORLD_SIZE", "1"))
        rank = int(os.environ.get("RANK", "0"))
        local = int(os.environ.get("LOCAL_RANK", "0"))
        torch.cuda.set_device(local)
        if world > 1:
            import datetime
            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                    device_id=torch.device("cuda", local))
        r = measure_stream(rank, world, local, layers=args.stream_only)
        if rank == 0:
            print(json.dumps(r), flush=True)
        if world > 1:
            dist.destroy_process_group()
        return
    if args.stack_only:
        import torch
        import torch.distributed as dist
        world = int(os.environ.get("WORLD_SIZE", "1"))
        rank = int(os.environ.get("RANK", "0"))
        local = int(os.environ.get("LOCAL_RANK", "0"))
        torch.cuda.set_device(local)
        if world > 1:
            import datetime
            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                    device_id=torch.device("cuda", local))
        r = measure_stack(rank, world, local, layers=args.stack_only)
        if rank == 0:
            print(json.dumps(r), flush=True)
        if world > 1:
            dist.destroy_process_group()
        return

    import torch
    import torch.distributed as dist

    import qmoe

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))

    def barrier():
        if world > 1:
            dist.barrier()

    # layer 0: configs[1] (decode); layer 1: configs[2] (Zipf-biased router)
    nl = 1 if args.no_prefill else 2
    cfg = qmoe.make_config(D, E, K_TOP, I_DIM, G, layers=nl,
                           max_tokens=4 if args.no_prefill else PREFILL_T, device=local)
    layer = qmoe.SynthLayer(cfg, SEED)
    ctx = qmoe.Context(cfg)
    ctx.upload(0, layer)
    if not args.no_prefill:
        ctx.upload(1, qmoe.SynthLayer(cfg, SEED, 1, zipf_s=1.1))
    x_host = qmoe.synth_tokens(SEED, rank, TOKENS, D)
    x_dev = torch.from_numpy(x_host).cuda().to(torch.bfloat16).contiguous()
    out_dev = torch.empty((TOKENS, D), dtype=torch.float32, device="cuda")

    # one step = 1000 sequential single-token calls, captured once as a CUDA
    # graph by the library (qmoe_capture_begin/end) on a torch-owned stream
    stream = torch.cuda.Stream()
    cs = stream.cuda_stream
    xs, os_ = x_dev.data_ptr(), out_dev.data_ptr()
    torch.cuda.synchronize()
    for t in range(4):  # eager warm-up outside capture
        ctx.forward_dev(0, xs + t * D * 2, qmoe.QMOE_BF16, 1, os_ + t * D * 4, cs)
    stream.synchronize()
    ctx.sync()
    out_dev.zero_()
    torch.cuda.synchronize()
    ctx.capture_begin(cs)
    for t in range(TOKENS):
        ctx.forward_dev(0, xs + t * D * 2, qmoe.QMOE_BF16, 1, os_ + t * D * 4, cs)
    graph = ctx.capture_end(cs)
    for _ in range(args.warmup):
        graph.launch(cs)
    stream.synchronize()
    ctx.sync()

    clocks = Clocks(local) if rank == 0 else None
    barrier()
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record(stream)
    for _ in range(args.steps):
        graph.launch(cs)
    ev1.record(stream)
    torch.cuda.synchronize()
    barrier()
    clk = clocks.stop() if clocks else None
    ctx.sync()
    ms = ev0.elapsed_time(ev1)
    if world > 1:
        tt = torch.tensor([ms], device="cuda")
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        ms = float(tt.item())
    value = world * args.steps * TOKENS / (ms / 1e3)

    # parity spot check of the timed outputs (tokens 996..999 of the last
    # replay; out_dev was zeroed before capture, so these come from the graph)
    gpu_out = out_dev.cpu().numpy()  # every token of the last replay
    out_last = gpu_out[TOKENS - 4:]
    # (one eager single-token call each: the same kernel, so the same bits)
    ref4 = np.concatenate([ctx.forward(0, x_host[t:t + 1]) for t in range(TOKENS - 4, TOKENS)])
    parity_ok = bool(np.array_equal(out_last, ref4))

    # e2e through the host-pointer C ABI (qmoe_forward: x read from host
    # memory, out written to host memory, on every call), one call per token
    # made from C as the reference's C caller makes them (qmoe__forward_tokens
    # loops over qmoe_forward); the same loop from Python beside it
    import ctypes as C
    loop = qmoe.lib().qmoe__forward_tokens
    loop.restype = C.c_int
    loop.argtypes = [C.c_void_p, C.c_int, C.c_void_p, C.c_int, C.c_void_p, C.c_void_p]
    e2e_steps = max(1, min(args.steps, 3))
    out_all = np.empty((TOKENS, D), np.float32)
    xh = np.ascontiguousarray(x_host, np.float32)
    errb = qmoe.Err()
    if loop(ctx.h, 0, xh.ctypes.data, 16, out_all.ctypes.data, C.byref(errb)) != 0:
        raise RuntimeError(errb.text())
    barrier()
    t0 = time.perf_counter()
    for _ in range(e2e_steps):
        if loop(ctx.h, 0, xh.ctypes.data, TOKENS, out_all.ctypes.data, C.byref(errb)) != 0:
            raise RuntimeError(errb.text())
    e2e_s = time.perf_counter() - t0
    e2e_parity = bool(np.array_equal(out_all[TOKENS - 4:], out_last))
    out_h = np.empty((1, D), np.float32)
    for t in range(16):
        ctx.forward(0, x_host[t:t + 1])
    t0 = time.perf_counter()
    for t in range(TOKENS):
        out_h[:] = ctx.forward(0, x_host[t:t + 1])
    py_s = time.perf_counter() - t0
    if world > 1:
        tt = torch.tensor([e2e_s, py_s], device="cuda")
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        e2e_s, py_s = float(tt[0]), float(tt[1])
    e2e = world * e2e_steps * TOKENS / e2e_s
    e2e_py = world * TOKENS / py_s

    # per-kernel event timing (separate pass, one token replayed as a graph
    # with events between its kernels) -> roofline of the dominant kernel
    # distinct tokens, L2 flushed (256 MB write) before each, as in the timed loop
    acc = None
    nprof = 48
    flush = torch.empty(64 * 1024 * 1024, dtype=torch.float32, device="cuda")
    for t in range(nprof):
        flush.fill_(float(t))
        torch.cuda.synchronize()
        us = ctx.profile_forward(0, xs + t * D * 2, qmoe.QMOE_BF16, 1, os_ + t * D * 4, 1)
        acc = np.array(us) if acc is None else acc + np.array(us)
    del flush
    names = (["decode_fused"] if len(acc) == 1 else
             ["router", "topk", "decode_gateup", "decode_down"])
    per_launch_ms = {n: acc[i] / nprof / 1e3 for i, n in enumerate(names)}
    dom = max(per_launch_ms, key=per_launch_ms.get)
    kb = kernel_bytes_per_token()
    hbm, _, src = peaks()
    # the timed region holds only the decode kernel, one launch per token
    timed_launch_ms = ms / (args.steps * TOKENS)
    achieved = kb[dom] / (timed_launch_ms / 1e3) / 1e9
    traffic = NCU_TRAFFIC.get(dom)
    layer_gbs = layer_bytes_per_token() * (value / world) / 1e9

    prefill, prefill_out = None, None
    if not args.no_prefill:
        prefill = measure_prefill(ctx, 1, rank)
        prefill_out = prefill.pop("_out")
        if world > 1:
            prefill["expert_parallel"] = measure_prefill_ep(rank, world, local, ctx, 1)

    hc, hc_h0, hc_out = None, None, None
    if not args.no_hc:
        hc = measure_hc(ctx, rank)
        hc_h0, hc_out = hc.pop("_h0"), hc.pop("_out")

    stack = None
    if not args.no_stack:
        stack = measure_stack(rank, world, local)

    stream = None
    if not args.no_stream:
        stream = measure_stream(rank, world, local)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        try:
            cpu = cpu_reference_rate(gpu_out=gpu_out)
        except Exception as e:  # reported, never silently replaced
            cpu = {"value": None, "unit": UNIT, "cores": 0, "kind": "unavailable",
                   "sample": f"failed: {e}"}
        legs = []
        if prefill is not None:
            legs.append((prefill, lambda: cpu_prefill_rate(prefill_out)))
        if hc is not None:
            legs.append((hc, lambda: cpu_hc_rate(hc_h0, hc_out)))
        if stack is not None:
            legs.append((stack, lambda: cpu_stack_rate(STACK_SEED, 100, STACK_T, None, 3, STACK_T,
                                                       "config 3, decode batch 64")))
        if stream is not None:
            legs.append((stream["decode_batch1"],
                         lambda: cpu_stack_rate(STACK_SEED + 1, 200, 4, 1.1, 2, 1,
                                                "config 4 batch-1 decode, 4 tokens one at a time")))
            legs.append((stream["prefill"],
                         lambda: cpu_stack_rate(STACK_SEED + 1, 200, STREAM_PREFILL, 1.1, 2,
                                                STREAM_PREFILL, "config 4 prefill, 512 tokens")))
        for where, fn in legs:
            try:
                where["cpu_baseline"] = fn()
            except Exception as e:  # reported, never silently replaced
                where["cpu_baseline"] = {"value": None, "unit": "tokens/s", "cores": 0,
                                         "kind": "unavailable", "sample": f"failed: {e}"}

    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms / args.steps,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "f32", "data": "synthetic",
            "config": bench_config(world),
            "e2e": {"value": e2e, "unit": UNIT, "h2d_bytes_per_step": TOKENS * D * 4,
                    "d2h_bytes_per_step": TOKENS * (D * 4 + 8),
                    "caller": "C loop over qmoe_forward (host buffers), one call per token",
                    "python_loop_value": e2e_py, "outputs_equal_graph": e2e_parity},
            "gpu_launches": len(names) * TOKENS * args.steps,
            "roofline": {"bound": "hbm", "kernel": dom, "achieved": achieved, "peak": hbm,
                         "unit": "GB/s", "frac": achieved / hbm, "traffic": traffic,
                         "peak_source": src,
                         "bytes_per_launch": kb[dom],
                         "kernel_us": {dom: 1e3 * timed_launch_ms},
                         "kernel_us_cold": {n: 1e3 * v for n, v in per_launch_ms.items()},
                         "layer_gbs": layer_gbs, "layer_frac": layer_gbs / hbm},
            "cpu_baseline": cpu,
            "clocks": clk,
            "parity_spot_check": parity_ok,
            "parity_margin": (cpu or {}).get("parity_margin"),
            "prefill": prefill,
            "hyper_connection": hc,
            "stack": stack,
            "stream": stream,
        }
        print(json.dumps(line), flush=True)
    ctx.close()
    if world > 1:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
