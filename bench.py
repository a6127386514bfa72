"""Benchmark: Q8_0 decode tokens/s of the Qwen3 runner on B200 (liblq8.so), one JSON line.

Default workload (the configuration quoted at 1/2/4/8 B200): Qwen3-32B
architecture, seeded random-init Q8_0 weights, batch 8 of 1024-token seeded prompts prefilled
once, then greedy decode steps at context 1024+. On N GPUs (torchrun, one rank per GPU) the
model is tensor-parallel over all N ranks (--tp 0, the default): q/k/v and gate/up split by
output rows, o and down by K with the partial sums exchanged inside the persistent decode
kernel over NVLink (LQ_TP_NCCL=1: per-layer kernels with NCCL all-reduces), the LM head by
vocabulary rows; one batch for the whole group, so the scaling is strong. A step = one decode
step of every sequence (B tokens). The timed region replays the CUDA-graph decode step K times
with tokens and KV caches resident in HBM (device time, max over ranks); `e2e` times the same
steps through the public C-ABI call lq_qwen3_decode_step with host token buffers (host->device
copy of the input ids and device->host copy of the next ids inside the timed region). Every
step streams all Q8_0 weights of the rank (GBs, far above the 126 MB L2), so no L2 flush is
needed between steps.

Other workloads: --config qwen3-8b (config 3; batch 1, 2048-token prompt by default),
qwen3-0.6b (config 1), qwen3-30b-a3b (config 5, expert-parallel under N ranks); --tp 1 runs
independent replicas per rank ("scaling": "weak").

--impl reference: the reference's CPU path (the C restatement in oracle/, all host threads)
on the same model config at batch 1 (the reference decodes one sequence), bounded sample
(16-token prompt), rank 0 only.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

REPO = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(REPO, "qwen-omni-inference-rs_b200")
for _p in (REPO, PKG):
    if _p not in sys.path:
        sys.path.insert(0, _p)

CONFIGS = {
    "qwen3-8b": dict(hidden=4096, layers=36, n_heads=32, n_kv_heads=8, head_dim=128, inter=12288,
                     vocab=151936, max_pos=40960, tied=0, eps=1e-6, theta=1e6, init_std=0.02, norm_std=0.0),
    "qwen3-0.6b": dict(hidden=1024, layers=28, n_heads=16, n_kv_heads=8, head_dim=128, inter=3072,
                       vocab=151936, max_pos=40960, tied=1, eps=1e-6, theta=1e6, init_std=0.02, norm_std=0.0),
    "qwen3-32b": dict(hidden=5120, layers=64, n_heads=64, n_kv_heads=8, head_dim=128, inter=25600,
                      vocab=151936, max_pos=40960, tied=0, eps=1e-6, theta=1e6, init_std=0.02, norm_std=0.0),
    # Qwen3-30B-A3B: 48 MoE layers of 128 experts (moe_inter 768), top-8, renormalised
    "qwen3-30b-a3b": dict(hidden=2048, layers=48, n_heads=32, n_kv_heads=4, head_dim=128, inter=0,
                          vocab=151936, max_pos=40960, tied=0, eps=1e-6, theta=1e6, init_std=0.02,
                          norm_std=0.0, n_experts=128, top_k=8, moe_inter=768, norm_topk=1),
}
# (batch, prefill tokens) of each BASELINE configuration
DEFAULT_SHAPE = {"qwen3-32b": (8, 1024), "qwen3-8b": (1, 2048), "qwen3-0.6b": (1, 16), "qwen3-30b-a3b": (64, 512)}
SEED = 1234
METRIC = "Q8_0 decode tok/s"


def peaks():
    p = os.path.join(REPO, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


# ------------------------------------------------------------------------------ clocks
class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled every 200 ms during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.lines: list[str] = []
        self.thread = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
            return
        self.thread = threading.Thread(target=self._read, daemon=True)
        self.thread.start()

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        if self.thread:
            self.thread.join(timeout=2)
        sm, smax, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [x.strip() for x in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax = float(parts[2])
            except ValueError:
                continue
            for nm, val in zip(names, parts[5:9]):
                if val.lower() == "active":
                    reasons.add(nm)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": smax,
                "reasons": sorted(reasons), "samples": len(sm)}


# ------------------------------------------------------------------------------ helpers
def dist_env():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def gemv_bytes(n: int, k: int, m: int) -> int:
    """Algorithmic bytes of one Q8_0 GEMV launch: weights (qs + fp16 scales) read once, the
    quantized activations (qs + fp16 scales) and the f32 outputs."""
    return n * k + n * (k // 32) * 2 + m * k + m * (k // 32) * 2 + m * n * 4


def time_gemv_launches(lq8, ctx, model, cfg, B, reps=2):
    """CUDA-event duration of every decode GEMV launch shape (fused qkv, o, fused gate/up,
    down) of every layer, on the model's own weights and stream; layers are walked in order so
    each launch streams its weights from HBM (a layer's 205 MB exceed the L2)."""
    import ctypes as C

    import torch
    H, I = cfg["hidden"], cfg["inter"]
    kmax = max(H, I, cfg["n_heads"] * cfg["head_dim"])
    dev = torch.device("cuda", ctx.device)
    xq = torch.randint(-127, 128, (B, kmax), dtype=torch.int8, device=dev)
    xd = torch.full((B, kmax // 32), 0x2000, dtype=torch.int16, device=dev)  # fp16 ~0.0078
    nmax = max(2 * I, cfg["n_heads"] * cfg["head_dim"] + 2 * cfg["n_kv_heads"] * cfg["head_dim"], H)
    y = torch.empty((B, nmax), dtype=torch.float32, device=dev)
    stream = torch.cuda.ExternalStream(ctx.stream, device=dev)
    shapes = {}
    for rep in range(reps):
        evs = []
        for layer in range(cfg["layers"]):
            for kind in ("qkv", "o", "gate_up", "down"):
                w = model.linear(layer, kind)
                e0 = torch.cuda.Event(enable_timing=True)
                e1 = torch.cuda.Event(enable_timing=True)
                e0.record(stream)
                ctx.call("lq_q8_0_matmul", C.byref(w), xq.data_ptr(), xd.data_ptr(), B, y.data_ptr(), None, w.n)
                e1.record(stream)
                evs.append((kind, w.n, w.k, e0, e1))
        ctx.synchronize()
        if rep == 0:
            continue  # warm-up pass
        for kind, n, k, e0, e1 in evs:
            s = shapes.setdefault(kind, {"n": n, "k": k, "ms": []})
            s["ms"].append(e0.elapsed_time(e1))
    return shapes


def cpu_baseline_sample(O, cfgd, threads=1, samples=5, layer_counts=(2, 4)):
    """The oracle (reference CPU path restated in C) on a bounded sample of the decode step:
    models truncated to 2 and 4 layers (+ the LM head) each decode `samples` tokens one at a
    time after a 16-token prompt (one untimed token first); per-layer time = the difference of
    the two models' median token times / 2, extrapolated to the full layer count. A
    non-positive difference makes the sample invalid (None) instead of being clamped."""
    cfg = O.make_config(**cfgd)
    saved = O.get_threads()
    med, raw = {}, {}
    for nl in layer_counts:
        O.set_threads(saved)  # weight generation on every core; the timed tokens on `threads`
        m = O.Qwen3Model(cfg, SEED, layers_limit=nl, ctx_max=16 + samples + 2)
        prompt = O.gen_tokens(SEED, 0, 16 + samples + 1, cfg.vocab)
        O.set_threads(threads)
        m.forward(prompt[:16], 0)
        m.forward(prompt[16:17], 16)
        ts = []
        for i in range(samples):
            t0 = time.perf_counter()
            m.forward(prompt[17 + i:18 + i], 17 + i)
            ts.append(time.perf_counter() - t0)
        m.close()
        med[nl] = statistics.median(ts)
        raw[nl] = [round(t, 5) for t in ts]
    O.set_threads(saved)
    lo, hi = layer_counts
    per_layer = (med[hi] - med[lo]) / (hi - lo)
    det = {"samples_s": {f"{nl}_layers": raw[nl] for nl in layer_counts},
           "median_s": {f"{nl}_layers": med[nl] for nl in layer_counts}, "per_layer_s": per_layer}
    if per_layer <= 0:
        det["invalid"] = "the deeper model's median token time is not above the shallower one's"
        return None, det
    step = med[lo] + (cfgd["layers"] - lo) * per_layer
    det["step_s"] = step
    return 1.0 / step, det


# ------------------------------------------------------------------------------ arms
def run_reference(args, cfgd):
    """Reference arm: the oracle (C restatement of the reference's Rust CPU path, Q8_0 linears)
    with all host threads; each step is one greedy decode token of the full model after a
    16-token prompt (a bounded sample of the 2048-context workload)."""
    from oracle import oracle as O
    O.build()
    threads = os.cpu_count() or 1
    O.set_threads(threads)
    cfg = O.make_config(**cfgd)
    ctx_max = 16 + args.warmup + args.steps + 2
    m = O.Qwen3Model(cfg, SEED, ctx_max=ctx_max)
    prompt = O.gen_tokens(SEED, 0, 16, cfg.vocab)
    logits = m.forward(prompt, 0)
    tok = O.argmax(logits)
    pos = 16
    for _ in range(args.warmup):
        tok = O.argmax(m.forward(np.array([tok]), pos))
        pos += 1
    t0 = time.perf_counter()
    for _ in range(args.steps):
        tok = O.argmax(m.forward(np.array([tok]), pos))
        pos += 1
    dt = time.perf_counter() - t0
    value = args.steps / dt
    sample = (f"{args.steps} greedy decode steps of the full {args.config} model (batch 1) after a 16-token "
              f"prompt instead of 2048 (CPU prefill of 2048 tokens is out of reach), {threads} threads")
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1000 * dt / args.steps,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "int8/f32",
        "data": "synthetic (seeded random-init weights, seeded token ids)",
        "config": {"workload": f"{args.config} greedy decode, batch 1", "batch": 1, "prompt": 16},
        "cpu_baseline": {"value": value, "unit": "tok/s", "cores": threads, "kind": "port", "sample": sample},
        "e2e": {"value": value, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def run_ours(args, cfgd, world, rank, local):
    import torch

    import build
    import lq8
    build.build()
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    torch.cuda.set_device(local)
    B, L, K, W = args.batch, args.prompt, args.steps, args.warmup
    ctx_max = L + W + 2 * K + 8 + 2
    ctx = lq8.Context(local)
    cfg = lq8.make_config(**cfgd)
    comm = None
    tp = (args.tp or world) if world > 1 else 1
    if tp > 1:
        if tp != world:
            raise SystemExit(f"--tp {tp} needs exactly {tp} ranks (got {world})")
        comm = lq8.Comm.from_process_group(ctx)
    t_create = time.perf_counter()
    model = lq8.Qwen3ForCausalLM(ctx, cfg, SEED, max_batch=B, ctx_max=ctx_max, comm=comm)
    t_create = time.perf_counter() - t_create
    # replicas run their own prompts; a tensor-parallel group shares one batch
    rng_stream = 1000 * rank if tp == 1 else 0
    from oracle import oracle as O  # seeded token ids only (the generator is shared)
    prompts = np.stack([O.gen_tokens(SEED, rng_stream + b, L, cfgd["vocab"]) for b in range(B)])
    t_pre = time.perf_counter()
    nxt = model.prefill(prompts)
    t_pre = time.perf_counter() - t_pre
    model.set_batch(B)
    stream = torch.cuda.ExternalStream(ctx.stream, device=torch.device("cuda", local))
    if args.prefill_reps:
        # prefill timing: the same prompts again (the first call above was the warm-up), CUDA
        # events on the model's stream around each call; the median
        times = []
        for _ in range(args.prefill_reps):
            a = torch.cuda.Event(enable_timing=True)
            b = torch.cuda.Event(enable_timing=True)
            a.record(stream)
            model.prefill(prompts)
            b.record(stream)
            ctx.synchronize()
            times.append(a.elapsed_time(b))
        ms = statistics.median(times)
        if rank == 0:
            print(json.dumps({"metric": "prefill tok/s", "value": B * L / (ms / 1000.0), "unit": "tok/s",
                              "ms": ms, "samples_ms": times, "batch": B, "prompt": L, "config": args.config,
                              "kernel": "exact" if os.environ.get("LQ_PREFILL_EXACT") else "fp16 operands"}))
        model.close()
        ctx.close()
        return

    def barrier():
        ctx.synchronize()
        torch.cuda.synchronize()
        if dist is not None:
            dist.barrier()

    def max_over_ranks(v: float) -> float:
        if dist is None:
            return v
        t = torch.tensor([v], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    # ---- device-resident decode (value)
    model.decode_device(W)
    barrier()
    if args.trace:
        # timeline mode: K decode steps under torch.profiler (CUPTI sees the graph's kernels
        # with their real overlap); prints per-kernel time and the busy/idle split
        from torch.profiler import ProfilerActivity, profile
        with profile(activities=[ProfilerActivity.CUDA]) as prof:
            model.decode_device(args.trace)
            ctx.synchronize()
        ks = sorted((e.time_range.start, e.time_range.end, e.name.split("(")[0])
                    for e in prof.events() if e.device_type.name == "CUDA")
        span = ks[-1][1] - ks[0][0]
        busy, cs, ce = 0.0, ks[0][0], ks[0][1]
        for s, e, _ in ks[1:]:
            if s > ce:
                busy, cs, ce = busy + ce - cs, s, e
            else:
                ce = max(ce, e)
        busy += ce - cs
        agg = {}
        prev_end = ks[0][0]
        for s, e, n in ks:
            a = agg.setdefault(n, [0, 0.0, 0.0])
            a[0] += 1
            a[1] += e - s
            # with programmatic dependent launch a kernel starts before its predecessor ends but
            # cannot end before it: end-to-end deltas split the step among the kernels
            a[2] += max(0.0, e - prev_end)
            prev_end = max(prev_end, e)
        print(json.dumps({"trace_steps": args.trace, "us_per_step": span / args.trace,
                          "busy_us": busy, "idle_us": span - busy,
                          "kernels": {n: {"launches": c, "us_per_launch": t / c, "end_delta_us_per_step": d / args.trace}
                                      for n, (c, t, d) in sorted(agg.items(), key=lambda x: -x[1][2])},
                          "order": [[round(s - ks[0][0], 2), round(e - s, 2),
                                     round(e - (max(x[1] for x in ks[:i]) if i else s), 2), n]
                                    for i, (s, e, n) in enumerate(ks[:24])]}))
        model.close()
        ctx.close()
        return
    if args.ncu_steps:
        # profiling mode: only the decode steps between cudaProfilerStart/Stop, nothing timed
        torch.cuda.profiler.start()
        model.decode_device(args.ncu_steps)
        ctx.synchronize()
        torch.cuda.profiler.stop()
        if args.ncu_gemv:
            # the per-launch GEMV replay of the roofline measurement, also profiled
            torch.cuda.profiler.start()
            time_gemv_launches(lq8, ctx, model, cfgd, B, reps=1)
            torch.cuda.profiler.stop()
        model.close()
        ctx.close()
        return
    clocks = ClockSampler(local)
    clocks.start()
    time.sleep(0.3)
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    model.decode_device(K)
    e1.record(stream)
    barrier()
    clk = clocks.stop()
    ms = max_over_ranks(e0.elapsed_time(e1))
    groups = world // tp
    value = groups * B * K / (ms / 1000.0)
    launches = model.graph_kernels() * K

    # ---- end to end through the host-buffer C-ABI call (e2e)
    tok_buf = lq8.wrap_device(model.token_buffer_ptr(), (B,), "<i4")
    ids = tok_buf.cpu().numpy().astype(np.int32)
    for _ in range(2):
        ids = model.decode_step(ids)
    barrier()
    e2 = torch.cuda.Event(enable_timing=True)
    e3 = torch.cuda.Event(enable_timing=True)
    e2.record(stream)
    for _ in range(K):
        ids = model.decode_step(ids)
    e3.record(stream)
    barrier()
    ms_e2e = max_over_ranks(e2.elapsed_time(e3))
    e2e = groups * B * K / (ms_e2e / 1000.0)

    peak, peak_kind = peaks()
    if cfgd.get("n_experts", 0) > 0:
        roofline, step_gbs, wbytes = moe_step_roofline(cfgd, B, L + W + K, ms / K, peak, peak_kind)
        return finish(args, cfgd, world, rank, L, B, K, W, ms, value, e2e, ms_e2e, clk, launches, roofline,
                      step_gbs, wbytes, t_create, t_pre, model, ctx, dist, comm)
    # ---- roofline of the dominant kernel: the persistent decode step when the graph runs it
    # (embedding, decode_step_kernel, argmax finalisation), else the decode GEMV
    persistent = model.graph_kernels() == 3
    shapes = time_gemv_launches(lq8, ctx, model, cfgd, B)
    tot_b = tot_ms = 0.0
    per_shape = {}
    for kind, s in shapes.items():
        b = gemv_bytes(s["n"], s["k"], B)
        avg = sum(s["ms"]) / len(s["ms"])
        per_shape[kind] = {"n": s["n"], "k": s["k"], "bytes": b, "avg_us": 1000 * avg,
                           "gbs": b / (avg / 1000) / 1e9}
        tot_b += b * len(s["ms"])
        tot_ms += sum(s["ms"])
    dom = per_shape["gate_up"]
    traffic = None
    tf = os.path.join(REPO, "profiles", "q8_gemv_traffic.txt")
    if os.path.exists(tf):
        for ln in open(tf):
            if ln.startswith(f"traffic_bytes_per_launch gate_up B={B} "):
                traffic = float(ln.split()[-1])
    roofline = {
        "bound": "hbm", "kernel": f"q8_gemv (gate/up fused, M={B}, N={dom['n']}, K={dom['k']})",
        "achieved": dom["gbs"], "peak": peak, "unit": "GB/s", "frac": dom["gbs"] / peak,
        "peak_kind": f"{peak_kind} copy bandwidth", "traffic": traffic,
        "algorithmic_bytes_per_launch": dom["bytes"],
        "all_decode_gemv_gbs": tot_b / (tot_ms / 1000) / 1e9,
        "frac_of_8tbs_spec": dom["gbs"] / 8000.0,
        "per_shape": per_shape,
    }
    wbytes = model.weight_bytes()
    if persistent:
        # one launch per step streams every Q8_0 weight once and reads the KV cache rows of the
        # attended positions (K and V, f32); timed as the whole decode graph, of which the
        # persistent kernel is all but a few microseconds of device time (ncu launch list)
        hkv = cfgd["n_kv_heads"] // tp  # this rank's kv heads
        ctx_avg = L + W + (K + 1) / 2.0
        kv_bytes = cfgd["layers"] * B * hkv * ctx_avg * 128 * 4 * 2
        alg = wbytes + kv_bytes
        ach = alg / (ms / K / 1000) / 1e9
        ptraffic = None
        if os.path.exists(tf):
            for ln in open(tf):
                if ln.startswith(f"traffic_bytes_per_launch decode_step {args.config} B={B} "):
                    ptraffic = float(ln.split()[-1])
        roofline = {
            "bound": "hbm", "kernel": f"decode_step_kernel<{B}> (persistent: every layer + LM head per launch)",
            "achieved": ach, "peak": peak, "unit": "GB/s", "frac": ach / peak,
            "peak_kind": f"{peak_kind} copy bandwidth", "traffic": ptraffic,
            "algorithmic_bytes_per_launch": alg, "weight_bytes": wbytes, "kv_bytes": kv_bytes,
            "timed_as": "decode graph per step (memset, embedding, decode_step_kernel, argmax finalize)",
            "per_layer_gemv_kernels": per_shape,
        }
    step_gbs = wbytes / (ms / K / 1000) / 1e9
    return finish(args, cfgd, world, rank, L, B, K, W, ms, value, e2e, ms_e2e, clk, launches, roofline, step_gbs,
                  wbytes, t_create, t_pre, model, ctx, dist, comm)


def moe_step_roofline(cfgd, B, ctx_len, step_s_ms, peak, peak_kind):
    """MoE decode: the whole step against the HBM roofline. Bytes per step = attention
    weights + router + LM head + the experts a batch of B tokens touches (expected count
    E * (1 - (1 - k/E)^B) under uniform routing) + the f32 KV cache read at the mid context."""
    H, D, Hq, Hkv, E, k, I = (cfgd[x] for x in ("hidden", "head_dim", "n_heads", "n_kv_heads", "n_experts",
                                                "top_k", "moe_inter"))
    q8 = lambda n, kk: n * kk * 34 // 32
    layers = cfgd["layers"]
    attn = q8((Hq + 2 * Hkv) * D, H) + q8(H, Hq * D)
    router = q8(E, H)
    expert = q8(2 * I, H) + q8(H, I)
    touched = E * (1.0 - (1.0 - k / E) ** B)
    kv = 2 * Hkv * D * ctx_len * 4 * B
    lm = q8(cfgd["vocab"], H)
    step_bytes = layers * (attn + router + touched * expert + kv) + lm
    gbs = step_bytes / (step_s_ms / 1000) / 1e9
    roofline = {"bound": "hbm", "kernel": f"whole MoE decode step (B={B})", "achieved": gbs, "peak": peak,
                "unit": "GB/s", "frac": gbs / peak, "peak_kind": f"{peak_kind} copy bandwidth", "traffic": None,
                "algorithmic_bytes_per_step": step_bytes, "expected_experts_touched_per_layer": touched}
    return roofline, gbs, int(layers * (attn + router + touched * expert) + lm)


def finish(args, cfgd, world, rank, L, B, K, W, ms, value, e2e, ms_e2e, clk, launches, roofline, step_gbs, wbytes,
           t_create, t_pre, model, ctx, dist, comm=None):
    tp = comm.world if comm is not None else 1
    # ---- CPU baseline (rank 0, N = 1 only)
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        from oracle import oracle as O
        O.build()
        v, det = cpu_baseline_sample(O, cfgd, threads=1)
        cpu = {"value": v, "unit": "tok/s", "cores": 1, "kind": "port",
               "sample": (f"oracle (C restatement of the reference's single-threaded Rust CPU path with Q8_0 "
                          f"linears), 1 thread, batch 1 (the reference decodes one sequence): 5 decode tokens "
                          f"each through models of 2 and 4 of {cfgd['layers']} layers + LM head after a 16-token "
                          f"prompt; per-layer time from the difference of the median token times, extrapolated "
                          f"to the full model; context 16 instead of {L} (attention over the longer context is "
                          f"left out)"),
               "detail": det}

    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": world, "steps": K, "warmup": W,
            "ms_per_step": ms / K, "higher_is_better": True, "scaling": "strong" if tp > 1 else "weak",
            "vs_baseline": None,
            "dtype": "int8/f32",
            "data": "synthetic (seeded random-init N(0,0.02) weights, seeded uniform token ids)",
            "config": {"workload": f"{args.config} greedy decode after a {L}-token prefill, batch {B}",
                       "model": args.config, "global_batch": B * (world // tp), "seq_len": L,
                       "parallelism": ((f"ep{tp}" if cfgd.get("n_experts", 0) else f"tp{tp}") +
                                       (f" x dp{world // tp}" if world > tp else "")) if tp > 1
                       else (f"dp{world} replicas" if world > 1 else "single GPU"),
                       "l2": "no flush: each step streams the Q8_0 weights (GBs, far above the 126 MB L2)",
                       "context_range": [L + W, L + W + K]},
            "roofline": roofline,
            "step_weight_gbs": step_gbs,
            "weight_bytes_per_step": wbytes,
            "cpu_baseline": cpu,
            "e2e": {"value": e2e, "unit": "tok/s", "h2d_bytes_per_step": 4 * B, "d2h_bytes_per_step": 4 * B,
                    "ms_per_step": ms_e2e / K},
            "clocks": clk,
            "gpu_launches": launches,
            "setup_s": {"create": t_create, "prefill": t_pre},
        }
        print(json.dumps(line), flush=True)
    model.close()  # releases the decode graph (it holds NCCL calls) before the communicator
    if comm is not None:
        comm.close()
    ctx.close()
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


SWEEP_M = (1, 8, 16, 128, 512, 2048)
SWEEP_KN = ((1024, 3072), (3072, 1024), (4096, 12288), (12288, 4096), (5120, 25600), (5120, 51200),
            (25600, 5120))


def run_sweep(args):
    """Linear sweep: y = x . W^T through lq_q8_0_linear (activation quantization + Q8_0
    matmul), x = N(0,1) in f32 and bf16, W = N(0,0.02) packed to Q8_0. Rotates through
    >= 512 MB of distinct weight copies so every launch reads its weights from HBM; the
    median of per-launch CUDA-event times after warm-up. One JSON line per case."""
    import ctypes as C

    import torch

    import build
    import lq8
    build.build()
    ctx = lq8.Context(0)
    dev = torch.device("cuda", 0)
    stream = torch.cuda.ExternalStream(ctx.stream, device=dev)
    hbm, hbm_kind = peaks()
    cases = []
    if args.sweep_case:
        m, n, k = (int(v) for v in args.sweep_case.split(","))
        cases = [(m, k, n)]
    else:
        cases = [(m, k, n) for (k, n) in SWEEP_KN for m in SWEEP_M]
    reps = max(args.sweep_reps, 3)
    for (m, k, n) in cases:
        wbytes = n * k * 34 // 32
        copies = max(2, -(-512 * 2**20 // wbytes)) if not args.sweep_case else 2
        g = torch.Generator(device=dev).manual_seed(SEED)
        ws = []
        for _ in range(copies):
            wf = (torch.randn((n, k), generator=g, device=dev) * 0.02).to(torch.bfloat16)
            ws.append(lq8.QTensor.quantize(ctx, wf))
            del wf
        for src in ("f32", "bf16"):
            x = torch.randn((m, k), generator=g, device=dev)
            if src == "bf16":
                x = x.to(torch.bfloat16)
            dt = lq8.DTYPE_F32 if src == "f32" else lq8.DTYPE_BF16
            y = torch.empty((m, n), dtype=torch.float32, device=dev)
            structs = [w.struct() for w in ws]
            for i in range(3):
                ctx.call("lq_q8_0_linear", C.byref(structs[i % copies]), x.data_ptr(), dt, m, y.data_ptr())
            ctx.synchronize()
            ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(reps)]
            for i in range(reps):
                ev[i][0].record(stream)
                ctx.call("lq_q8_0_linear", C.byref(structs[i % copies]), x.data_ptr(), dt, m, y.data_ptr())
                ev[i][1].record(stream)
            ctx.synchronize()
            us = statistics.median(a.elapsed_time(b) for a, b in ev) * 1e3
            byts = wbytes + m * k * (4 if src == "f32" else 2) + m * n * 4
            flops = 2.0 * m * n * k
            print(json.dumps({"sweep": "q8_0_linear", "m": m, "k": k, "n": n, "x": src, "us": round(us, 2),
                              "GB/s": round(byts / us / 1e3, 1), "TOPS": round(flops / us / 1e6, 1),
                              "hbm_frac": round(byts / us / 1e3 / hbm, 3), "hbm_peak": hbm,
                              "peak_kind": hbm_kind, "weight_copies": copies}), flush=True)
        del ws
        torch.cuda.empty_cache()


def run_prefill_gemm(args):
    """Prefill GEMM: the exact tcgen05 kernel (lq_q8_0_matmul) against the fp16-operand kernel
    (lq_q8_0_matmul_prefill) at the config-2 prefill shapes, on the same pre-quantized operands
    (random Q8_0 weights and activation rows); median of per-launch CUDA-event times after
    warm-up, TOPS = 2 m n k / time. One JSON line per (case, kernel)."""
    import ctypes as C

    import torch

    import build
    import lq8
    build.build()
    ctx = lq8.Context(0)
    dev = torch.device("cuda", 0)
    stream = torch.cuda.ExternalStream(ctx.stream, device=dev)
    cases = ([tuple(int(v) for v in args.prefill_gemm_case.split(","))] if args.prefill_gemm_case else
             [(m, n, k) for m in (512, 2048) for (n, k) in ((6144, 4096), (4096, 4096), (24576, 4096), (4096, 12288),
                                                           (10240, 5120), (51200, 5120), (5120, 25600))])
    reps = max(args.sweep_reps, 3)
    g = torch.Generator(device=dev).manual_seed(SEED)
    for (m, n, k) in cases:
        w = lq8.QTensor.quantize(ctx, (torch.randn((n, k), generator=g, device=dev) * 0.02).to(torch.bfloat16))
        xq = torch.randint(-127, 128, (m, k), dtype=torch.int8, device=dev, generator=g)
        xd = torch.full((m, k // 32), 0x2000, dtype=torch.int16, device=dev)  # fp16 0.0078
        y = torch.empty((m, n), dtype=torch.float32, device=dev)
        ws = w.struct()
        for name in ("lq_q8_0_matmul", "lq_q8_0_matmul_prefill"):
            for _ in range(3):
                ctx.call(name, C.byref(ws), xq.data_ptr(), xd.data_ptr(), m, y.data_ptr(), None, n)
            ctx.synchronize()
            ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(reps)]
            for i in range(reps):
                ev[i][0].record(stream)
                ctx.call(name, C.byref(ws), xq.data_ptr(), xd.data_ptr(), m, y.data_ptr(), None, n)
                ev[i][1].record(stream)
            ctx.synchronize()
            us = statistics.median(a.elapsed_time(b) for a, b in ev) * 1e3
            print(json.dumps({"prefill_gemm": "exact" if name == "lq_q8_0_matmul" else "fp16 operands", "m": m,
                              "n": n, "k": k, "us": round(us, 2), "TOPS": round(2.0 * m * n * k / us / 1e6, 1)}),
                  flush=True)
        del w
        torch.cuda.empty_cache()


def run_moe(args):
    """MoE layer alone: lq_moe_forward (router, top-k, grouped expert GEMVs, combine) at the
    Qwen3-30B-A3B expert shape (128 experts, hidden 2048, moe_inter 768, top-8) with random
    Q8_0 weights, for rows in --moe-rows. Reports per call time, the touched expert bytes
    (experts actually selected) and their rate. One JSON line per row count."""
    import ctypes as C

    import torch

    import build
    import lq8
    build.build()
    ctx = lq8.Context(0)
    dev = torch.device("cuda", 0)
    stream = torch.cuda.ExternalStream(ctx.stream, device=dev)
    E, H, I, K = 128, 2048, 768, 8
    g = torch.Generator(device=dev).manual_seed(SEED)

    def q8(n, k):
        qs = torch.randint(-127, 128, (n, k), dtype=torch.int8, device=dev, generator=g)
        d = torch.randint(0x1400, 0x2000, (n, k // 32), dtype=torch.int16, device=dev, generator=g)
        return qs, d

    rq, rd = q8(E, H)
    gq, gd = q8(E * 2 * I, H)
    dq, dd = q8(E * H, I)
    router = lq8.Q8Tensor(E, H, rq.data_ptr(), rd.data_ptr())
    ex = lq8.MoeExperts(E, I, H, lq8.Q8Tensor(E * 2 * I, H, gq.data_ptr(), gd.data_ptr()),
                        lq8.Q8Tensor(E * H, I, dq.data_ptr(), dd.data_ptr()))
    expert_bytes = (2 * I * H + H * I) * 34 // 32
    for rows in (int(r) for r in args.moe_rows.split(",")):
        x = (torch.randn((rows, H), generator=g, device=dev)).to(torch.bfloat16)
        xq = torch.empty((rows, H), dtype=torch.int8, device=dev)
        xd = torch.empty((rows, H // 32), dtype=torch.int16, device=dev)
        ctx.call("lq_q8_0_quantize", x.data_ptr(), lq8.DTYPE_BF16, rows, H, xq.data_ptr(), xd.data_ptr())
        out = torch.zeros((rows, H), dtype=torch.float32, device=dev)
        ids = torch.empty((rows, K), dtype=torch.int32, device=dev)
        reps = max(args.sweep_reps, 3)
        for _ in range(3):
            ctx.call("lq_moe_forward", C.byref(router), C.byref(ex), xq.data_ptr(), xd.data_ptr(), rows, K, 1,
                     out.data_ptr(), None, ids.data_ptr(), None)
        ctx.synchronize()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(reps):
            ctx.call("lq_moe_forward", C.byref(router), C.byref(ex), xq.data_ptr(), xd.data_ptr(), rows, K, 1,
                     out.data_ptr(), None, ids.data_ptr(), None)
        e1.record(stream)
        ctx.synchronize()
        us = e0.elapsed_time(e1) * 1e3 / reps
        touched = int(torch.unique(ids).numel())
        byts = touched * expert_bytes + E * H * 34 // 32
        print(json.dumps({"moe": "lq_moe_forward", "rows": rows, "experts": E, "hidden": H, "moe_inter": I,
                          "top_k": K, "us": round(us, 2), "experts_touched": touched,
                          "weight_bytes": byts, "GB/s": round(byts / us / 1e3, 1),
                          "tokens_per_s": round(rows / us * 1e6, 1)}), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=64)
    ap.add_argument("--warmup", type=int, default=8)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--config", default="qwen3-32b", choices=sorted(CONFIGS))
    ap.add_argument("--batch", type=int, default=0, help="sequences per step (0: the config's batch)")
    ap.add_argument("--prompt", type=int, default=0, help="prompt tokens (0: the config's prefill length)")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline sample")
    ap.add_argument("--ncu-steps", type=int, default=0,
                    help="profiling: run this many decode steps between cudaProfilerStart/Stop and exit")
    ap.add_argument("--ncu-gemv", action="store_true",
                    help="profiling: also replay the decode GEMV launches inside the profiled range")
    ap.add_argument("--prefill-reps", type=int, default=0,
                    help="time this many prefills of the config's prompts (median, CUDA events) and exit")
    ap.add_argument("--trace", type=int, default=0,
                    help="timeline: run this many decode steps under torch.profiler and print a summary")
    ap.add_argument("--layers", type=int, default=0,
                    help="profiling: build only the first N layers (a smaller device footprint)")
    ap.add_argument("--sweep", action="store_true",
                    help="run the Linear sweep (M x (K, N) grid, f32 and bf16 inputs) and exit")
    ap.add_argument("--sweep-case", default="",
                    help="with --sweep: one case 'm,n,k' (two weight copies; for profiling)")
    ap.add_argument("--sweep-reps", type=int, default=20)
    ap.add_argument("--prefill-gemm", action="store_true",
                    help="time the exact and the fp16-operand prefill GEMMs at the config-2 prefill shapes and exit")
    ap.add_argument("--prefill-gemm-case", default="", help="with --prefill-gemm: one case 'm,n,k'")
    ap.add_argument("--tp", type=int, default=0,
                    help="model parallelism over the torchrun ranks: tensor-parallel for dense configs, "
                         "expert-parallel for MoE; 0 = all ranks, 1 = independent replicas")
    ap.add_argument("--moe", action="store_true",
                    help="time lq_moe_forward alone at the Qwen3-30B-A3B expert shape and exit")
    ap.add_argument("--moe-rows", default="1,8,64,512")
    args = ap.parse_args()
    if args.warmup < 3:
        ap.error("--warmup must be >= 3")
    if args.prefill_gemm:
        run_prefill_gemm(args)
        return
    if args.sweep:
        run_sweep(args)
        return
    if args.moe:
        run_moe(args)
        return
    world, rank, local = dist_env()
    cfgd = dict(CONFIGS[args.config])
    batch0, prompt0 = DEFAULT_SHAPE[args.config]
    args.batch = args.batch or batch0
    args.prompt = args.prompt or prompt0
    if args.layers:
        cfgd["layers"] = args.layers
    if args.impl == "reference":
        if rank == 0:
            run_reference(args, cfgd)
        return
    run_ours(args, cfgd, world, rank, local)


if __name__ == "__main__":
    main()
