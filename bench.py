"""Benchmark: DeepSeek-V3 MoE layer tokens/s on B200 (decode).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--tokens T] [--impl ours|reference]

A step is one MoE layer forward (router -> dispatch -> FP8 SwiGLU experts ->
weighted combine + shared expert) over a batch of T tokens (default 64, the
largest decode batch of config 2) with all 256 routed experts + the shared
expert resident in HBM (11.3 GB of e4m3 weights + fp32 block scales,
synthetic, seeded).  The weights streamed per step exceed the 126 MB L2, and
L2 is additionally flushed between timed steps (256 MiB written, then 256 MiB
of another buffer read, so no dirty line of the flush is written back inside
the timed step); each step is
timed with CUDA events on the launching stream.  The layer runs as one CUDA
graph replay (GraphedDsMoELayer: 7 kernels -- router logits, route + dispatch,
x staging, gate/up, activation staging, down, combine; 5 with --fused-decode);
the plain per-call path is timed too
(eager_ms_per_step), and the other decode-experts variant (one fused launch
or three) beside the one run (alt_ms_per_step).  The same measurement is repeated for
T = 1, 4, 16 ("sweep").

Printed (rank 0, one JSON line): tokens/s with inputs resident in HBM
(`value`), the same through the public API from pinned host buffers with the
copies inside the timed region (`e2e`), the HBM roofline of the dominant
kernel (the grouped GEMV gate/up stage), the reference's own CPU path timed
on this host (`cpu_baseline`, oracle/_ref), clocks sampled during the run.

Every run also checks what it timed (`parity`, after the timed regions):
each batch's expert ids against the oracle's router (ties within 1e-6
excused) and its outputs against the oracle's run_fp8_moe flow on the same
weights -- all tokens of the decode batches, a slice of the prefill ones --
with the north star's gate (rel-L2 <= 2e-2, cosine distance <= 1e-3).

--impl reference times the reference's CPU path alone (its own compiled
kernels, oracle/_ref, driven through run_fp8_moe's default flow) on the same
workload: the full 64-token batch, with every expert it selects.
With --gpus N > 1 (torchrun) the layer runs expert-parallel (pocketlm_b200/ep.py):
each rank holds 256/N routed experts plus the shared expert and router, routes
its own --tokens tokens and exchanges them with NCCL all-to-alls (weak
scaling); value is N * tokens / the slowest rank's step time.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))
os.environ.setdefault("OMP_NUM_THREADS", str(len(os.sched_getaffinity(0))))
os.environ.setdefault("PCKETLM_NATIVE_THREADS", os.environ["OMP_NUM_THREADS"])

import torch  # noqa: E402

METRIC = "DS-V3 MoE layer tokens/s @1/2/4/8 B200; % of HBM or FP8 TC roofline"
L2_FLUSH_BYTES = 256 << 20
# kernels per layer forward: router logits, route + dispatch + chunk list, then on the warp-MMA path
# x -> f16, gate/up, activations -> f16, down (else chunk list, gate/up, down), combine
KERNELS_PER_LAYER = {"auto": 7, "mma_regs": 7, "mma_tma": 7, "stream": 6, "direct": 6}
# with the fused decode experts: router logits, route + dispatch + chunk list, x -> f16, fused experts, combine
KERNELS_PER_LAYER_FUSED = 5
GEMV_IMPLS = {"auto": 0, "stream": 1, "direct": 2, "mma_regs": 3, "mma_tma": 4}
ROOFLINE_KERNEL = {
    "fused": "decode_fused_kernel<tiled>: gate/up+SwiGLU, activation staging and down (fp8_mma.cu)",
    "auto": "mma_gemv_async_kernel<2, swiglu> gate/up+SwiGLU (fp8_mma.cu)",
    "mma_regs": "mma_gemv_kernel<2, swiglu> gate/up+SwiGLU (fp8_mma.cu)",
    "mma_tma": "tma_mma_gemv_kernel<2, swiglu> gate/up+SwiGLU (fp8_mma.cu)",
    "stream": "stream_gemv_kernel gate/up+SwiGLU (fp8_stream.cu)",
    "direct": "grouped_gemv_kernel gate/up+SwiGLU (fp8_gemv.cu)",
}


def measured_peaks() -> dict:
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        return {**json.loads(path.read_text()), "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "source": "fallback"}


# ---------------------------------------------------------------------------
# clocks
# ---------------------------------------------------------------------------

class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.path = Path(os.environ.get("TMPDIR", "/tmp")) / f"moe_clocks_{os.getpid()}.csv"

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "50"], stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
            return self
        # the sampler is running (first line written) before the timed region starts
        deadline = time.monotonic() + 10.0
        while time.monotonic() < deadline and self.proc.poll() is None:
            if self.path.exists() and self.path.stat().st_size > 0:
                break
            time.sleep(0.02)
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self) -> dict:
        if self.proc is None or not self.path.exists():
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        rows = []
        for line in self.path.read_text().splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                rows.append((float(parts[1]), float(parts[2]), float(parts[3]), parts[5:9]))
            except ValueError:
                continue
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for _, _, _, flags in rows for i, f in enumerate(flags) if f == "Active"})
        loaded = [r for r in rows if r[2] > 200.0] or rows
        return {"sm_mhz": statistics.median(r[0] for r in loaded), "sm_max_mhz": max(r[1] for r in rows),
                "reasons": reasons, "samples": len(rows)}


# ---------------------------------------------------------------------------
# CPU baseline: the reference's own kernels (oracle/_ref) in run_fp8_moe's flow
# ---------------------------------------------------------------------------

def cpu_decode_sample_inputs(tokens: int, seed: int):
    """A bounded sample of the config-2 decode workload for the reference's
    CPU flow: `tokens` tokens and the layer's weights generated on the CPU for
    exactly the experts those tokens select (plus the shared one)."""
    import oracle
    from pocketlm_b200 import synth

    cfg = synth.C2_DSV3
    x = synth.make_hidden(tokens, cfg.hidden, seed=seed)
    probe = synth.make_fp8_layer(cfg, seed=seed, experts=[])
    route = oracle.route_deepseek(x, probe.router_weight, probe.bias, top_k=cfg.top_k, n_groups=cfg.n_group,
                                  topk_groups=cfg.topk_group, route_scale=cfg.route_scale)
    experts = sorted({int(v) for v in route.ids.reshape(-1).tolist()})
    layer = synth.make_fp8_layer(cfg, seed=seed, experts=experts + [cfg.n_routed],
                                 threads=len(os.sched_getaffinity(0)))
    return x, layer, experts


def cpu_reference_sample(tokens: int, seed: int, reps: int = 1, inputs=None) -> dict:
    """Time run_fp8_moe's default flow (fp8_source.py:1569-1884) on the host
    cores with the reference's compiled fp8_e4m3_block_mlp_f32 on a bounded
    sample of `tokens` tokens of the config-2 workload (cpu_decode_sample_inputs,
    or `inputs` made by it once for several timings)."""
    import oracle
    from oracle import ref

    if not ref.available():
        raise RuntimeError("reference build oracle/_ref missing")
    x, layer, experts = inputs if inputs is not None else cpu_decode_sample_inputs(tokens, seed)
    times = []
    for _ in range(max(1, reps)):
        t0 = time.perf_counter()
        oracle.ds_moe_layer(x, layer, route=None, mlp_fn=ref.fp8_mlp)
        times.append(time.perf_counter() - t0)
    per_step = statistics.median(times)
    return {"value": tokens / per_step, "unit": "tokens/s", "cores": len(os.sched_getaffinity(0)),
            "kind": "reference", "seconds_per_sample": per_step,
            "sample": (f"the whole {tokens}-token config-2 decode batch through run_fp8_moe's default flow "
                       f"(torch CPU router, per-expert fp8_e4m3_block_mlp_f32 from oracle/_ref, bf16 combine, "
                       f"shared expert); {len(experts)} routed experts; OMP threads {os.environ['OMP_NUM_THREADS']}; "
                       f"weights drawn on the host from the same seeded distributions")}


def cpu_fp8_layer_sample(layer, x: torch.Tensor, reps: int = 1) -> dict:
    """run_fp8_moe's default flow (fp8_source.py:1569-1884) on the host cores
    for the host tokens `x`, with `layer`'s own weights (any device) copied to
    the host for the experts those tokens select: torch CPU router, the
    reference's compiled fp8_e4m3_block_mlp_f32 per expert (oracle/_ref),
    bf16 combine, shared expert."""
    import oracle
    from oracle import ref
    from pocketlm_b200 import synth

    if not ref.available():
        raise RuntimeError("reference build oracle/_ref missing")
    cfg = layer.cfg
    rw = layer.router_weight.cpu()
    bias = None if layer.bias is None else layer.bias.cpu()
    route = oracle.route_deepseek(x, rw, bias, top_k=cfg.top_k, n_groups=cfg.n_group, topk_groups=cfg.topk_group,
                                  route_scale=cfg.route_scale)
    experts = sorted({int(v) for v in route.ids.reshape(-1).tolist()})
    if layer.w13.device.type == "cpu":
        host = layer  # already on the host (a full copy made once for the parity checks)
    else:
        ids = experts + [cfg.n_routed]
        idx = torch.tensor([e if layer.slots is None else layer.slots[e] for e in ids], device=layer.w13.device)
        host = synth.Fp8MoELayer(cfg, rw, bias, *(t.index_select(0, idx).cpu() for t in (layer.w13, layer.s13,
                                                                                         layer.w2, layer.s2)),
                                 {e: i for i, e in enumerate(ids)})
    times = []
    for _ in range(max(1, reps)):
        t0 = time.perf_counter()
        oracle.ds_moe_layer(x, host, route=None, mlp_fn=ref.fp8_mlp)
        times.append(time.perf_counter() - t0)
    per = statistics.median(times)
    return {"value": x.shape[0] / per, "unit": "tokens/s", "cores": len(os.sched_getaffinity(0)),
            "kind": "reference", "seconds_per_sample": per, "routed_experts": len(experts)}


def cpu_prefill_expert_sample(layer, x: torch.Tensor, ids: torch.Tensor, n_experts: int = 4) -> dict:
    """The reference's CPU cost of a prefill batch, from a bounded sample:
    run_fp8_moe's default flow calls the compiled fp8_e4m3_block_mlp_f32 once
    per selected expert on all of that expert's rows (fp8_source.py:1600-1660),
    and at prefill sizes those calls are the whole cost.  Time those calls
    (oracle/_ref) for the `n_experts` experts around the median load of this
    batch -- their full row sets, the layer's own weights copied to the host --
    and scale the per-row time to the batch's T * (k + 1) pairs."""
    from oracle import ref

    if not ref.available():
        raise RuntimeError("reference build oracle/_ref missing")
    cfg = layer.cfg
    T = int(ids.shape[0])
    counts = torch.bincount(ids.reshape(-1).cpu(), minlength=cfg.n_routed)
    order = [int(e) for e in torch.argsort(counts, stable=True).tolist() if int(counts[e]) > 0]
    mid = len(order) // 2
    chosen = order[max(0, mid - n_experts // 2):max(0, mid - n_experts // 2) + n_experts]
    flat = ids.reshape(-1)
    rows_total, seconds = 0, 0.0
    for e in chosen:
        rows = (flat == e).nonzero().reshape(-1) // cfg.top_k
        xe = x.index_select(0, rows.to(x.device)).cpu().float()
        i = e if layer.slots is None else layer.slots[e]
        w = [t.cpu() for t in (layer.w13[i, 0], layer.s13[i, 0], layer.w13[i, 1], layer.s13[i, 1], layer.w2[i],
                               layer.s2[i])]
        t0 = time.perf_counter()
        ref.fp8_mlp(*w, xe)
        seconds += time.perf_counter() - t0
        rows_total += int(rows.numel())
    per_row = seconds / max(1, rows_total)
    batch_seconds = per_row * T * (cfg.top_k + 1)
    return {"value": T / batch_seconds, "unit": "tokens/s", "cores": len(os.sched_getaffinity(0)),
            "kind": "reference", "seconds_per_sample": seconds, "sampled_rows": rows_total,
            "sampled_experts": chosen, "estimated_batch_seconds": batch_seconds}


def cpu_prefill_full_batch(host_layer, x: torch.Tensor) -> dict:
    """The reference's CPU flow timed on a whole prefill batch (one run):
    run_fp8_moe's default flow with the compiled fp8_e4m3_block_mlp_f32 on
    every selected expert's full row set, the layer's own weights on the host."""
    s = cpu_fp8_layer_sample(host_layer, x, reps=1)
    s["sample"] = (f"the whole {int(x.shape[0])}-token config-3 batch through run_fp8_moe's default flow "
                   f"(oracle/_ref kernels, {s['routed_experts']} routed experts, same weights and tokens), measured")
    return s


def cpu_q4_layer_sample(layer, x: torch.Tensor, reps: int = 1) -> dict:
    """The reference's Q4 token loop (layer_bridge.py:909-955: softmax top-k
    router in torch, then q4_moe_selected_forward_u16 per token,
    q4_dequant.cpp:357-476, compiled in oracle/_ref) on the host cores for the
    host tokens `x`, with `layer`'s own weights copied to the host."""
    import oracle
    from oracle import ref

    if not ref.available():
        raise RuntimeError("reference build oracle/_ref missing")
    cfg = layer.cfg
    rw = layer.router_weight.cpu()
    probe = oracle.route_softmax_topk(x, rw, top_k=cfg.top_k, normalize=True)
    host = {e: tuple(t.cpu() for t in layer.expert(e)) for e in sorted({int(v) for v in probe.ids.reshape(-1)})}
    times = []
    for _ in range(max(1, reps)):
        t0 = time.perf_counter()
        route = oracle.route_softmax_topk(x, rw, top_k=cfg.top_k, normalize=True)
        x16 = x.to(torch.float16)
        for t in range(x.shape[0]):
            ref.q4_moe_selected_forward(x16[t], [host[int(e)] for e in route.ids[t].tolist()],
                                        route.weights[t].float(), cfg.hidden, cfg.inter)
        times.append(time.perf_counter() - t0)
    per = statistics.median(times)
    return {"value": x.shape[0] / per, "unit": "tokens/s", "cores": len(os.sched_getaffinity(0)),
            "kind": "reference", "seconds_per_sample": per, "experts": len(host)}


# ---------------------------------------------------------------------------
# GPU measurement
# ---------------------------------------------------------------------------

class L2Flush:
    """Between timed steps: write 256 MiB (L2 is 126 MB), then read 256 MiB of
    another buffer.  The read evicts the dirty lines of the write, so their
    write-back happens here and not inside the next timed step (measured: a
    write alone adds ~6 us of write-back to a 1-token decode layer), and L2
    ends up holding only clean lines of the read buffer -- none of the
    step's weights or inputs."""

    def __init__(self, device: torch.device):
        self.write = torch.zeros((L2_FLUSH_BYTES // 4,), dtype=torch.float32, device=device)
        self.read = torch.ones((L2_FLUSH_BYTES // 4,), dtype=torch.float32, device=device)
        self.sink = torch.zeros((1,), dtype=torch.float32, device=device)

    def __call__(self) -> None:
        self.write.add_(1)
        self.sink.copy_(self.read.sum())


def flush_l2(flush) -> None:
    flush()


def time_steps(fn, steps: int, warmup: int, flush: torch.Tensor) -> list[float]:
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    stream = torch.cuda.current_stream()
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    for i in range(steps):
        flush_l2(flush)
        starts[i].record(stream)
        fn()
        ends[i].record(stream)
    torch.cuda.synchronize()
    return [s.elapsed_time(e) for s, e in zip(starts, ends)]


def layer_bytes(cfg, ids: torch.Tensor, tokens: int) -> dict:
    n_exp = len({int(v) for v in ids.reshape(-1).tolist()}) + 1  # + shared
    gs, ds = cfg.gate_scale_shape, cfg.down_scale_shape
    gateup = n_exp * (2 * cfg.inter * cfg.hidden + 2 * 4 * gs[0] * gs[1])
    down = n_exp * (cfg.hidden * cfg.inter + 4 * ds[0] * ds[1])
    router = cfg.n_routed * cfg.hidden * 2
    acts = tokens * cfg.hidden * 2 * 2
    return {"experts": n_exp, "gateup": gateup, "down": down, "router": router,
            "total": gateup + down + router + acts}


def stage_times(gpu_layer, x, steps: int, flush: torch.Tensor) -> list[float]:
    from pocketlm_b200 import native
    import ctypes

    lib = native.load_library()
    lib.moe_b200_stage_timing(1)
    acc = None
    buf = (ctypes.c_float * 8)()
    for _ in range(steps):
        # a long flush (~4 x 256 MiB of writes) keeps the GPU busy while the
        # host enqueues the layer, so the stage events time GPU work rather
        # than host launch latency
        for _ in range(4):
            flush_l2(flush)
        gpu_layer.forward(x)
        n = lib.moe_b200_stage_times(buf, 8)
        vals = [buf[i] for i in range(n)]
        acc = vals if acc is None else [a + v for a, v in zip(acc, vals)]
    lib.moe_b200_stage_timing(0)
    return [a / steps for a in acc]


def read_traffic(name: str):
    path = ROOT / "profiles" / name
    if not path.exists():
        return None
    for line in path.read_text().splitlines():
        if line.strip().startswith("traffic_bytes_per_launch:"):
            try:
                return int(line.split(":", 1)[1].strip().split()[0])
            except ValueError:
                return None
    return None


def parity_leg(fn, *a, **kw) -> dict:
    """The checker on a timed batch (oracle/parity.py), after its timing; a
    checker that cannot run is reported, never silently passed."""
    try:
        from oracle import parity

        return getattr(parity, fn)(*a, **kw)
    except Exception as exc:  # noqa: BLE001 -- reported in the JSON line
        return {"pass": False, "error": f"{type(exc).__name__}: {exc}"}


def run_ours(args, rank: int, world: int) -> dict | None:
    from pocketlm_b200 import native, synth
    from pocketlm_b200.runtime import DsMoELayerGPU

    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", 0)))
    torch.cuda.set_device(dev)
    native.load_library()
    cfg = synth.C2_DSV3
    layer = synth.make_fp8_layer(cfg, seed=args.seed, device=dev)
    gpu_layer = DsMoELayerGPU(layer)
    flush = L2Flush(dev)
    peaks = measured_peaks()
    lib = native.load_library()
    lib.moe_b200_fused_decode(1 if args.fused_decode else 0)
    fused = bool(lib.moe_b200_fused_decode_enabled()) and args.gemv == "auto"
    results = {}
    checked = {}  # T -> (x, out, ids) of the timed batch, for the parity leg
    sweep = [] if args.sweep == "none" else [int(v) for v in args.sweep.split(",") if v]
    token_list = [args.tokens] + [t for t in sweep if t != args.tokens]
    with ClockSampler(dev.index) as clocks:
        for T in token_list:
            x = synth.make_hidden(T, cfg.hidden, seed=args.seed + 100 * rank + T, device=dev)
            out = torch.empty((T, cfg.hidden), dtype=torch.bfloat16, device=dev)
            ids = torch.empty((T, cfg.top_k), dtype=torch.int64, device=dev)
            gpu_layer.forward(x, out=out, ids=ids)
            torch.cuda.synchronize()
            graphed = gpu_layer.capture(T)
            graphed.input.copy_(x)
            eager_ms = statistics.mean(time_steps(lambda: gpu_layer.forward(x, out=out), args.steps, args.warmup,
                                                  flush))
            if world > 1:
                torch.distributed.barrier()
            torch.cuda.synchronize()
            times = time_steps(graphed.replay, args.steps, args.warmup, flush)
            if world > 1:
                torch.distributed.barrier()
            torch.cuda.synchronize()
            ms = statistics.mean(times)
            if world > 1:
                t = torch.tensor([ms], device=dev)
                torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
                ms = float(t.item())
            stages = stage_times(gpu_layer, x, max(5, min(args.steps, 50)), flush)
            b = layer_bytes(cfg, ids, T)
            # stage intervals: [route + dispatch + chunk list + x to f16, then either the fused experts
            # or gate/up, (activations to f16 on the MMA path,) down; then combine]
            fused_ms = stages[1] if fused and len(stages) == 3 else None
            gateup_ms = stages[1] if not fused and len(stages) >= 2 else None
            down_ms = (stages[3] if len(stages) >= 5 else stages[2]) if not fused and len(stages) >= 3 else None
            # the other decode-experts variant on the same batch (fused vs three launches), for comparison
            alt_ms = None
            if args.gemv == "auto" and not args.no_alt_compare:
                lib.moe_b200_fused_decode(0 if fused else 1)
                g3 = gpu_layer.capture(T)
                g3.input.copy_(x)
                alt_ms = statistics.mean(time_steps(g3.replay, args.steps, args.warmup, flush))
                del g3
                lib.moe_b200_fused_decode(1 if fused else 0)
            # end to end through the public API: pinned host in, pinned host out
            x_host = x.cpu().pin_memory()
            out_host = torch.empty((T, cfg.hidden), dtype=torch.bfloat16).pin_memory()

            def e2e_step():
                graphed.input.copy_(x_host, non_blocking=True)
                graphed.replay()
                out_host.copy_(graphed.output, non_blocking=True)

            e2e_ms = statistics.mean(time_steps(e2e_step, args.steps, args.warmup, flush))
            if world > 1:
                t = torch.tensor([e2e_ms], device=dev)
                torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
                e2e_ms = float(t.item())
            torch.cuda.synchronize()
            # what the timed graph replays produced for this batch, for the parity leg
            checked[T] = (x.cpu(), graphed.output.cpu(), graphed.ids.cpu())
            results[T] = {
                "tokens": T, "ms_per_step": ms, "tokens_per_s": T * world / (ms / 1e3),
                "eager_ms_per_step": eager_ms,
                "e2e_tokens_per_s": T * world / (e2e_ms / 1e3), "e2e_ms": e2e_ms,
                "experts_streamed": b["experts"], "layer_bytes": b["total"],
                "layer_hbm_frac": (b["total"] / (ms / 1e3)) / (peaks["hbm_gbs"] * 1e9),
                "gateup_ms": gateup_ms, "down_ms": down_ms, "stage_ms": stages,
                "gateup_bytes": b["gateup"], "down_bytes": b["down"],
                "gateup_gbs": (b["gateup"] / (gateup_ms / 1e3) / 1e9) if gateup_ms else None,
                "down_gbs": (b["down"] / (down_ms / 1e3) / 1e9) if down_ms else None,
                "fused_experts_ms": fused_ms,
                "fused_experts_gbs": ((b["gateup"] + b["down"]) / (fused_ms / 1e3) / 1e9) if fused_ms else None,
                "alt_variant": None if alt_ms is None else ("three launches" if fused else "fused experts"),
                "alt_ms_per_step": alt_ms,
            }
        # the checker on every decode batch (all tokens), and the reference's CPU path on the headline batch,
        # both on one host copy of this layer's weights
        host_layer = layer.to("cpu") if not args.no_parity or not args.no_cpu_baseline else None
        parity = {}
        if not args.no_parity:
            for T, (xc, oc, ic) in sorted(checked.items()):
                parity[f"c2-dsv3-decode-T{T}"] = parity_leg("fp8_layer_parity", host_layer, xc, oc, ic)
        cpu = None
        if not args.no_cpu_baseline and rank == 0:
            try:
                cpu = cpu_fp8_layer_sample(host_layer, checked[args.tokens][0], reps=2)
                cpu["sample"] = (f"the whole {args.tokens}-token config-2 batch of the GPU run (same weights and "
                                 f"tokens) through run_fp8_moe's default flow: torch CPU router, the reference's "
                                 f"compiled fp8_e4m3_block_mlp_f32 (oracle/_ref) per selected expert "
                                 f"({cpu['routed_experts']}), bf16 combine, shared expert; OMP threads "
                                 f"{os.environ['OMP_NUM_THREADS']}")
            except Exception as exc:  # the baseline is reported, not required
                cpu = {"value": None, "unit": "tokens/s", "cores": len(os.sched_getaffinity(0)),
                       "kind": "reference", "sample": f"unavailable: {type(exc).__name__}: {exc}"}
        del host_layer
        prefill, q4, mla = {}, {}, {}
        if args.prefill_tokens != "none" or args.q4_tokens != "none" or args.mla_cache != "none":
            del gpu_layer, layer, graphed
            torch.cuda.empty_cache()
        if args.prefill_tokens != "none":
            prefill = run_prefill(args, dev, flush, peaks,
                                  [int(v) for v in args.prefill_tokens.split(",") if v])
        if args.q4_tokens != "none":
            q4 = run_q4(args, dev, flush, peaks, [int(v) for v in args.q4_tokens.split(",") if v])
        if args.mla_cache != "none" and rank == 0:  # no collectives inside: the other ranks go on
            mla = run_mla(args, dev, flush, peaks, int(args.mla_cache))
    clock_info = clocks.summary()
    if rank != 0:
        return None
    head = results[args.tokens]
    peak = peaks["hbm_gbs"]
    achieved = head["fused_experts_gbs"] if fused else head["gateup_gbs"]
    roofline_bytes = head["gateup_bytes"] + head["down_bytes"] if fused else head["gateup_bytes"]
    for block in (prefill, q4, mla):
        for key, rep in (block.pop("parity", None) or {}).items():
            parity[key] = rep
    parity_summary = {"gate": {"rel_l2": 2e-2, "cos_dist": 1e-3, "ids": "bit-exact, ties within 1e-6 excused"},
                      "all_pass": bool(parity) and all(r.get("pass") for r in parity.values()),
                      "cases": parity} if not args.no_parity else None
    t1 = results.get(1)
    return {
        "metric": METRIC, "value": head["tokens_per_s"], "unit": "tokens/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": head["ms_per_step"],
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "f32 (e4m3 weights decoded exactly, bf16 activations, fp32 accumulate)",
        "data": "synthetic (seeded random DS-V3-shape weights and activations; no checkpoint)",
        "config": {"workload": f"c2-dsv3-decode-T{args.tokens}", "tokens_per_gpu": args.tokens,
                   "hidden": cfg.hidden, "moe_intermediate": cfg.inter, "experts": f"{cfg.n_routed}+1",
                   "top_k": cfg.top_k, "n_group": cfg.n_group, "topk_group": cfg.topk_group,
                   "parallelism": "single GPU" if world == 1 else f"replicas x{world}",
                   "l2": "weights streamed per step exceed L2; between timed steps 256 MiB written, then 256 MiB of "
                         "another buffer read (the flush's dirty lines are written back before the step)"},
        "roofline": {"bound": "hbm", "kernel": ROOFLINE_KERNEL["fused" if fused else args.gemv],
                     "achieved": achieved, "peak": peak, "unit": "GB/s",
                     "frac": (achieved / peak) if achieved else None,
                     "peak_source": f"{peaks['source']} hbm_gbs",
                     "algorithmic_bytes_per_launch": roofline_bytes,
                     "traffic": read_traffic(f"decode_fused_c2_decode_T{args.tokens}.md" if fused else
                                             f"grouped_gemv_gateup_c2_decode_T{args.tokens}.md"),
                     "layer_frac": head["layer_hbm_frac"]},
        "e2e": {"value": head["e2e_tokens_per_s"], "unit": "tokens/s",
                "h2d_bytes_per_step": args.tokens * cfg.hidden * 2, "d2h_bytes_per_step": args.tokens * cfg.hidden * 2},
        "gpu_launches": (KERNELS_PER_LAYER_FUSED if fused else KERNELS_PER_LAYER[args.gemv]) * args.steps,
        "cpu_baseline": cpu,
        "clocks": clock_info,
        "parity": parity_summary,
        "decode_T1": None if t1 is None else {
            "ms_per_step": t1["ms_per_step"], "tokens_per_s": t1["tokens_per_s"],
            "layer_bytes": t1["layer_bytes"], "layer_hbm_frac": t1["layer_hbm_frac"],
            "stage_ms": t1["stage_ms"], "fused_experts_ms": t1["fused_experts_ms"],
            "fused_experts_gbs": t1["fused_experts_gbs"],
            "alt_variant": t1["alt_variant"], "alt_ms_per_step": t1["alt_ms_per_step"], "target_hbm_frac": 0.70},
        "sweep": {str(T): {k: v for k, v in r.items() if k != "stage_ms"} | {"stage_ms": r["stage_ms"]}
                  for T, r in sorted(results.items())},
        "prefill": prefill,
        "q4": q4,
        "mla": mla,
    }


def run_prefill(args, dev, flush, peaks, token_list) -> dict:
    """Config 3 on one GPU: the DS-V3 layer with the Zipf-skewed router bias,
    prefill batches on the tcgen05 grouped GEMM (prefill_gemm.cu).  Each step
    is one replay of the layer captured as a CUDA graph, as the decode steps
    are (the eager forward's time is reported beside it: its host launches
    leave gaps of 0.2-0.9 ms depending on the host), CUDA-event timed after
    warm-up with an L2 flush between steps.  FLOPs are the layer's
    algorithmic ones: T * (k + 1) * 3 * 2 * H * I for the experts + T * 2 * H
    * E for the router."""
    from pocketlm_b200 import synth
    from pocketlm_b200.runtime import DsMoELayerGPU

    cfg = synth.C2_DSV3
    layer = synth.make_fp8_layer(cfg, seed=args.seed + 1, device=dev, bias_kind="zipf")
    gpu_layer = DsMoELayerGPU(layer)
    bf16_peak = peaks.get("bf16_tflops", 1590.0)
    out = {}
    checked = {}
    for T in token_list:
        x = synth.make_hidden(T, cfg.hidden, seed=args.seed + T, device=dev)
        ids = torch.empty((T, cfg.top_k), dtype=torch.int64, device=dev)
        gpu_layer.forward(x, ids=ids)
        torch.cuda.synchronize()
        steps = max(3, min(args.steps, 10))
        y = torch.empty((T, cfg.hidden), dtype=torch.bfloat16, device=dev)
        eager_ms = statistics.mean(time_steps(lambda: gpu_layer.forward(x, out=y), steps, args.warmup, flush))
        graphed = gpu_layer.capture(T)
        graphed.input.copy_(x)
        ms = statistics.mean(time_steps(graphed.replay, steps, args.warmup, flush))
        torch.cuda.synchronize()
        checked[T] = (x.cpu(), graphed.output.cpu(), graphed.ids.cpu())  # the last timed replay's output
        del y, graphed
        stages = stage_times(gpu_layer, x, 3, flush)
        flops = T * (cfg.top_k + 1) * 3 * 2 * cfg.hidden * cfg.inter + T * 2 * cfg.hidden * cfg.n_routed
        pairs = T * (cfg.top_k + 1)
        gu_flops = pairs * 2 * 2 * cfg.hidden * cfg.inter
        gu_ms = stages[1] if len(stages) > 1 else None
        counts = torch.bincount(ids.reshape(-1), minlength=cfg.n_routed)
        out[str(T)] = {
            "tokens": T, "ms_per_step": ms, "tokens_per_s": T / (ms / 1e3), "eager_ms_per_step": eager_ms,
            "tflops": flops / (ms / 1e3) / 1e12,
            "frac_of_bf16_peak": flops / (ms / 1e3) / 1e12 / bf16_peak,
            "frac_of_fp8_nominal": flops / (ms / 1e3) / 1e12 / 4500.0,
            "gateup_tflops": (gu_flops / (gu_ms / 1e3) / 1e12) if gu_ms else None,
            "stage_ms": stages, "max_pairs_per_expert": int(counts.max()),
            "mma_kind": "tcgen05.mma kind::f16 (fp16 A/B, fp32 accumulate in TMEM)",
        }
        del x, ids
    host_layer = layer.to("cpu") if checked and (not args.no_parity or not args.no_cpu_baseline) else None
    parity = {}
    if not args.no_parity:
        from oracle.parity import slice_tokens

        for T, (xc, yc, ic) in sorted(checked.items()):
            parity[f"c3-dsv3-prefill-zipf-T{T}"] = parity_leg("fp8_layer_parity", host_layer, xc, yc, ic,
                                                              slice_tokens(ic))
    cpu = None
    if not args.no_cpu_baseline and token_list:
        # the reference's per-expert CPU calls on the 8192-token batch (or the largest), same weights
        T = 8192 if 8192 in checked else max(checked)
        xc, _y, ic = checked[T]
        try:
            cpu = cpu_prefill_expert_sample(host_layer, xc, ic, n_experts=max(1, args.cpu_prefill_experts))
            cpu["sample"] = (f"the reference's fp8_e4m3_block_mlp_f32 (oracle/_ref) on the full row sets of "
                             f"{len(cpu['sampled_experts'])} median-load experts of the {T}-token config-3 batch "
                             f"({cpu['sampled_rows']} rows, same weights); per-row time scaled to the batch's "
                             f"{T * (cfg.top_k + 1)} pairs; OMP threads {os.environ.get('OMP_NUM_THREADS')}")
        except Exception as exc:  # a baseline that cannot run must not cost the GPU numbers
            cpu = {"unavailable": f"{type(exc).__name__}: {exc}"}
        if args.cpu_prefill_full and args.cpu_prefill_full in checked:
            xf = checked[args.cpu_prefill_full][0]
            try:
                cpu["measured_full_batch"] = cpu_prefill_full_batch(host_layer, xf)
            except Exception as exc:  # noqa: BLE001
                cpu["measured_full_batch"] = {"unavailable": f"{type(exc).__name__}: {exc}"}
    del gpu_layer, layer, host_layer
    torch.cuda.empty_cache()
    return {"workload": "c3-dsv3-prefill-zipf", "peak_bf16_tflops": bf16_peak,
            "peak_source": f"{peaks['source']} bf16_tflops", "sweep": out, "cpu_baseline": cpu, "parity": parity}


def run_q4(args, dev, flush, peaks, token_list) -> dict:
    """Config 4 on one GPU: the Mixtral-8x7B-shape layer in the reference's Q4
    format (hidden 4096, ffn 14336, 8 experts, softmax top-2 renormalised),
    bf16 activations, through moe_q4_moe_layer_u16 (router, dispatch, Q4
    experts, combine): batches of 32+ pairs per expert on the tcgen05 grouped
    GEMM (int4 codes in the Q4 tiled layout, converted exactly to fp16), smaller
    ones on the warp-MMA GEMV.  Eager forwards, CUDA-event timed, L2 flushed
    between steps.  Bytes: the experts the batch selects (packed codes + fp16
    row scales) + router + activations; FLOPs: T * k * 3 * 2 * H * I."""
    from pocketlm_b200 import synth
    from pocketlm_b200.runtime import Q4MoELayerGPU

    cfg = synth.C4_MIXTRAL
    layer = Q4MoELayerGPU(synth.make_q4_layer(cfg, seed=args.seed, device=dev))
    out = {}
    parity = {}
    for T in token_list:
        x = synth.make_hidden(T, cfg.hidden, seed=args.seed + 7 * T, device=dev)
        ids = torch.empty((T, cfg.top_k), dtype=torch.int64, device=dev)
        layer.forward(x, ids=ids)
        torch.cuda.synchronize()
        steps = max(3, min(args.steps, 20))
        y = torch.empty_like(x)
        ms = statistics.mean(time_steps(lambda: layer.forward(x, out=y), steps, args.warmup, flush))
        torch.cuda.synchronize()
        if not args.no_parity:
            from oracle.parity import slice_tokens

            sel = None if T <= 64 else slice_tokens(ids, n_spread=32, n_heavy=8)
            parity[f"c4-mixtral-q4-T{T}"] = parity_leg("q4_layer_parity", layer.layer, x, y, ids, sel)
        del y
        n_exp = len({int(v) for v in ids.reshape(-1).tolist()})
        nbytes = n_exp * cfg.expert_bytes + cfg.n_experts * cfg.hidden * 2 + T * cfg.hidden * 4
        gemm = layer.tables_tiled is not None and T * cfg.top_k >= layer.prefill_pairs * cfg.n_experts
        flops = T * cfg.top_k * 3 * 2 * cfg.hidden * cfg.inter
        out[str(T)] = {"tokens": T, "ms_per_step": ms, "tokens_per_s": T / (ms / 1e3), "experts_streamed": n_exp,
                       "path": "tcgen05 GEMM" if gemm else "warp-MMA GEMV", "layer_bytes": nbytes,
                       "layer_hbm_frac": nbytes / (ms / 1e3) / (peaks["hbm_gbs"] * 1e9),
                       "tflops": flops / (ms / 1e3) / 1e12,
                       "frac_of_bf16_peak": flops / (ms / 1e3) / 1e12 / peaks.get("bf16_tflops", 1590.0)}
        del x, ids
    cpu = None
    if not args.no_cpu_baseline and token_list:
        n = max(1, args.cpu_q4_tokens)
        T = max(token_list)
        x = synth.make_hidden(T, cfg.hidden, seed=args.seed + 7 * T, device=dev)[:n].cpu()
        try:
            cpu = cpu_q4_layer_sample(layer.layer, x)
            cpu["sample"] = (f"first {n} tokens of the {T}-token config-4 batch, same weights, through the "
                             f"reference's token loop with oracle/_ref's q4_moe_selected_forward_u16")
        except Exception as exc:  # a baseline that cannot run must not cost the GPU numbers
            cpu = {"unavailable": f"{type(exc).__name__}: {exc}"}
    del layer
    torch.cuda.empty_cache()
    return {"workload": "c4-mixtral-q4", "kernel": "dense_mma_gemv_kernel<Q4> (dense_gemv.cu) / "
            "prefill_gemm_kernel<*, Q4> (prefill_gemm.cu)", "sweep": out, "cpu_baseline": cpu, "parity": parity}


def run_mla(args, dev, flush, peaks, cache_len: int) -> dict:
    """The DeepSeek-V3 MLA attention block for one decode token (ds_forward.cpp:647-782:
    hidden 7168, q_lora_rank 1536, kv_lora_rank 512, 128 heads, nope 128, rope 64, v 128),
    fp32 like the reference, over a cache of cache_len positions, through
    native.ds_attention_block_forward with weights and caches resident (the previous
    cache copied into the new one each call, as the reference's API returns it).  Bytes:
    the five fp32 projections, the cache read by the attention and the cache copy."""
    from pocketlm_b200 import native

    H, qr, R, heads, nope, rope, v = 7168, 1536, 512, 128, 128, 64, 128
    prev = cache_len - 1
    g = torch.Generator(device=dev).manual_seed(args.seed)

    def rnd(*shape, scale=1.0):
        return torch.randn(shape, generator=g, device=dev) * scale

    w = dict(q_a=rnd(qr, H, scale=H ** -0.5), q_b=rnd(heads * (nope + rope), qr, scale=qr ** -0.5),
             kv_a=rnd(R + rope, H, scale=H ** -0.5), kv_b=rnd(heads * (nope + v), R, scale=R ** -0.5),
             o_w=rnd(H, heads * v, scale=(heads * v) ** -0.5), q_norm=1 + 0.1 * rnd(qr), kv_norm=1 + 0.1 * rnd(R))
    prev_kv, prev_pe = rnd(prev, R), rnd(prev, rope)
    angles = torch.arange(rope // 2, device=dev, dtype=torch.float32) * cache_len * 1e-3
    cos, sin = angles.cos(), angles.sin()
    hidden = rnd(H)
    dims = dict(q_lora_rank=qr, kv_lora_rank=R, num_heads=heads, qk_nope_dim=nope, qk_rope_dim=rope, v_head_dim=v,
                rms_eps=1e-6, softmax_scale=(nope + rope) ** -0.5)
    order = ("q_a", "q_b", "kv_a", "kv_b", "o_w", "q_norm", "kv_norm")
    session = native.DeepSeekNativeSession(num_layers=1, hidden_dim=H, num_experts=0, top_k=0)

    def call(x):
        return native.ds_attention_block_forward(session, x, *(w[k] for k in order), previous_kv_cache=prev_kv,
                                                 previous_pe_cache=prev_pe, rope_cos=cos, rope_sin=sin, **dims)

    out, _ = call(hidden)
    torch.cuda.synchronize()
    steps = max(3, min(args.steps, 20))
    ms = statistics.mean(time_steps(lambda: call(hidden), steps, args.warmup, flush))
    host_x = hidden.cpu().pin_memory()
    e2e_ms = statistics.mean(time_steps(lambda: call(host_x)[0].cpu(), steps, args.warmup, flush))
    weight_elems = sum(w[k].numel() for k in order)
    cache_row = R + rope
    nbytes = 4 * (weight_elems + cache_len * cache_row + 2 * prev * cache_row)
    res = {"workload": f"dsv3-mla-attention-block-cache{cache_len}",
           "kernels": "mla_gemv_kernel x3, mla_norm_rope_kernel, mla_qabs_kernel, mla_attention_kernel, "
                      "mla_merge_kernel (mla.cu)",
           "ms_per_token": ms, "tokens_per_s": 1e3 / ms, "algorithmic_bytes": nbytes,
           "hbm_frac": nbytes / (ms / 1e3) / (peaks["hbm_gbs"] * 1e9), "peak_source": f"{peaks['source']} hbm_gbs",
           "e2e_ms_per_token": e2e_ms, "gpu_launches_per_token": 7,
           "invocations_counted": session.fused_attention_invocation_count()}
    parity = {}
    host = {k: t.cpu() for k, t in w.items()}
    if not args.no_parity:
        import oracle.mla as omla

        want, (wkv, wpe) = omla.attention_block(hidden.cpu(), *(host[k] for k in order), prev_kv.cpu(), prev_pe.cpu(),
                                                cos.cpu(), sin.cpu(), **dims)
        got, (kv, pe) = call(hidden)
        rel = float((got.cpu() - want).norm() / want.norm())
        rel_kv = float((kv[-1].cpu() - wkv[-1]).norm() / wkv[-1].norm())
        parity[f"mla-block-cache{cache_len}"] = {"rel_l2": rel, "new_cache_row_rel_l2": rel_kv, "gate": 1e-5,
                                                 "pass": rel <= 1e-5 and rel_kv <= 1e-5}
    cpu = None
    if not args.no_cpu_baseline:
        try:
            import oracle.ref as oref

            if not oref.available():
                raise FileNotFoundError("oracle/_ref not built")
            hx, pk, pp = hidden.cpu(), prev_kv.cpu(), prev_pe.cpu()
            args_ref = (hx, *(host[k] for k in order), pk, pp, cos.cpu(), sin.cpu())
            oref.attention_block(*args_ref, **dims)  # warm
            t0 = time.perf_counter()
            reps = 3
            for _ in range(reps):
                oref.attention_block(*args_ref, **dims)
            per = (time.perf_counter() - t0) / reps
            cpu = {"value": 1.0 / per, "unit": "tokens/s", "cores": int(os.environ.get("OMP_NUM_THREADS", "1")),
                   "kind": "reference", "sample": f"{reps} calls of the reference's ds_attention_block_forward_f32 "
                   f"(oracle/_ref, OpenMP) on the same weights and cache; {per * 1e3:.1f} ms per call"}
        except Exception as exc:  # the baseline is reported, not required
            cpu = {"unavailable": f"{type(exc).__name__}: {exc}"}
    res["cpu_baseline"] = cpu
    res["parity"] = parity
    session.close()
    del w, host, prev_kv, prev_pe
    torch.cuda.empty_cache()
    return res


def timed_max_over_ranks(fn, steps: int, warmup: int, flush: torch.Tensor, dev: torch.device) -> float:
    """Mean CUDA-event time of `steps` calls of fn on this rank (L2 flushed
    before each, warm-up first, barriers around), then the max over ranks."""
    import torch.distributed as dist

    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    dist.barrier()
    stream = torch.cuda.current_stream()
    times = []
    for _ in range(steps):
        flush_l2(flush)
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record(stream)
        fn()
        e.record(stream)
        e.synchronize()
        times.append(s.elapsed_time(e))
    dist.barrier()
    t = torch.tensor([statistics.mean(times)], device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def run_ours_ep(args, rank: int, world: int) -> dict | None:
    """N > 1: expert parallelism.  Rank r holds routed experts
    [r * 256 / N, (r + 1) * 256 / N) plus the shared expert and router, and
    routes its own --tokens tokens; a step is one layer forward on every rank
    (route, rows written straight into their experts' ranks over NVLink,
    local grouped experts, outputs written back, combine; ep.PeerExchange).  Timed per rank with CUDA events between barriers; the max over
    ranks is the step time; value = N * tokens / step time."""
    import torch.distributed as dist

    from pocketlm_b200 import synth
    from pocketlm_b200.ep import ExpertParallelLayer

    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", 0)))
    cfg = synth.C2_DSV3
    T = args.tokens
    ep = ExpertParallelLayer(cfg, rank, world, seed=args.seed, device=dev, peer_sync=args.ep_sync)
    flush = L2Flush(dev)
    x = synth.make_hidden(T, cfg.hidden, seed=args.seed + 100 * rank + T, device=dev)
    peaks = measured_peaks()

    def timed(fn, steps: int | None = None) -> float:
        return timed_max_over_ranks(fn, args.steps if steps is None else steps, args.warmup, flush, dev)

    # the peer exchange's step replays as one CUDA graph (kernels + NCCL), like the 1-GPU layer
    graphed = ep.capture(T) if ep.peer is not None else None
    step = (lambda: graphed(x)) if graphed is not None else (lambda: ep.forward(x))
    with ClockSampler(dev.index) as clocks:
        ms = timed(step)
        x_host = x.cpu().pin_memory()
        out_host = torch.empty((T, cfg.hidden), dtype=torch.bfloat16).pin_memory()

        def e2e():
            xd = x_host.to(dev, non_blocking=True)
            out = graphed(xd) if graphed is not None else ep.forward(xd)[0]
            out_host.copy_(out, non_blocking=True)

        e2e_ms = timed(e2e)
    del graphed  # a graph holding NCCL calls goes before the process group
    out_ep, ids, _w = ep.forward(x)
    gathered = [torch.empty_like(ids) for _ in range(world)]
    dist.all_gather(gathered, ids)
    clock_info = clocks.summary()
    parity = None
    if not args.no_parity:
        # the checker on this rank's batch: the experts its tokens selected, regenerated here from their own
        # seeded generators (identical to the copies on the ranks that own them), against the oracle's flow
        need = sorted({int(v) for v in ids.reshape(-1).tolist()}) + [cfg.n_routed]
        ref_layer = synth.make_fp8_layer(cfg, seed=args.seed, device=dev, experts=need)
        parity = parity_leg("fp8_layer_parity", ref_layer, x, out_ep, ids)
        del ref_layer
        torch.cuda.empty_cache()
    parity_by_rank = [None] * world
    dist.all_gather_object(parity_by_rank, parity)
    with ClockSampler(dev.index) as prefill_clocks:
        prefill = run_ep_prefill(args, rank, world, ep, timed, peaks)
    if prefill is not None:
        prefill["clocks"] = prefill_clocks.summary()
    if rank != 0:
        return None
    cases = {f"c2-dsv3-decode-T{T}-ep{world}-rank{r}": rep for r, rep in enumerate(parity_by_rank) if rep}
    for key, rep in ((prefill or {}).pop("parity", None) or {}).items():
        cases[key] = rep
    all_ids = torch.cat(gathered).cpu()
    per_rank = cfg.n_routed // world
    # bytes streamed by the busiest rank: its experts hit by any token (+ the shared expert)
    hit = sorted({int(v) for v in all_ids.reshape(-1).tolist()})
    busiest = max(sum(1 for e in hit if r * per_rank <= e < (r + 1) * per_rank) for r in range(world)) + 1
    gs, ds = cfg.gate_scale_shape, cfg.down_scale_shape
    expert_bytes = 3 * cfg.inter * cfg.hidden + 4 * (2 * gs[0] * gs[1] + ds[0] * ds[1])
    rank_bytes = busiest * expert_bytes + cfg.n_routed * cfg.hidden * 2
    achieved = rank_bytes / (ms / 1e3) / 1e9
    return {
        "metric": METRIC, "value": world * T / (ms / 1e3), "unit": "tokens/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None,
        "dtype": "f32 (e4m3 weights decoded exactly, bf16 activations, fp32 accumulate)",
        "data": "synthetic (seeded random DS-V3-shape weights and activations; no checkpoint)",
        "config": {"workload": f"c2-dsv3-decode-T{T}", "tokens_per_gpu": T, "hidden": cfg.hidden,
                   "moe_intermediate": cfg.inter, "experts": f"{cfg.n_routed}+1", "top_k": cfg.top_k,
                   "n_group": cfg.n_group, "topk_group": cfg.topk_group, "parallelism": f"ep{world}",
                   "ep_sync": args.ep_sync,
                   "l2": "between timed steps 256 MiB written, then 256 MiB of another buffer read"},
        "roofline": {"bound": "hbm", "kernel": "whole EP layer step on the busiest rank",
                     "achieved": achieved, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                     "frac": achieved / peaks["hbm_gbs"], "peak_source": f"{peaks['source']} hbm_gbs",
                     "algorithmic_bytes_per_launch": rank_bytes, "traffic": None,
                     "experts_on_busiest_rank": busiest},
        "e2e": {"value": world * T / (e2e_ms / 1e3), "unit": "tokens/s", "h2d_bytes_per_step": T * cfg.hidden * 2,
                "d2h_bytes_per_step": T * cfg.hidden * 2},
        # peer exchange: route (logits, select), rank counts, dispatch (rank keys, bucket, scatter to
        # peers), experts (bucket: 1 kernel, 3 above 2048 rows; home rows, chunk list, x staging, gate/up,
        # activation staging, down, rows home to their ranks), combine; all-to-all exchange: 13
        "gpu_launches": (15 + (2 if ep.peer is not None and ep.peer.capacity + T > 2048 else 0)
                         if ep.peer is not None else 13) * args.steps,
        "exchange": "peer-memory (symmetric memory, NVLink stores)" if ep.peer is not None else "NCCL all-to-all",
        "ep_prefill": prefill,
        "cpu_baseline": None,
        "clocks": clock_info,
        "parity": None if args.no_parity else {
            "gate": {"rel_l2": 2e-2, "cos_dist": 1e-3, "ids": "bit-exact, ties within 1e-6 excused"},
            "all_pass": bool(cases) and all(r.get("pass") for r in cases.values()), "cases": cases},
    }


def stack_share(batch: int, rank: int, world: int) -> int:
    """Tokens of a decode batch on `rank`: the batch spread over the ranks in
    order (data-parallel attention replicas), so a 1-token batch lives on
    rank 0 and the other ranks only serve experts."""
    return batch // world + (1 if rank < batch % world else 0)


def stack_critical_bytes(ids_by_rank: list, per_rank: int, expert_bytes: int, router_bytes: int) -> int:
    """Weight bytes on the stack's critical path: ids_by_rank[r][l] = rank
    r's expert ids [T_r, k] in layer l.  Layer l waits for its busiest rank:
    the routed experts in that rank's range hit by any token, plus, on a rank
    with tokens, its shared expert and the router.  Summed over the layers."""
    world = len(ids_by_rank)
    total = 0
    for li in range(len(ids_by_rank[0])):
        hit = {int(v) for r in range(world) for v in ids_by_rank[r][li].reshape(-1).tolist()}
        worst = 0
        for r in range(world):
            has_tokens = ids_by_rank[r][li].numel() > 0
            n = sum(1 for e in hit if r * per_rank <= e < (r + 1) * per_rank) + (1 if has_tokens else 0)
            worst = max(worst, n * expert_bytes + (router_bytes if has_tokens else 0))
        total += worst
    return total


def run_stack(args, rank: int, world: int) -> dict | None:
    """Config 5: the routed-expert stack of DS-V3 decode, --stack-layers
    layers (58 for the full model) of the config-2 shape with random weights,
    experts split expert-parallel over the N ranks (256 / N per rank per
    layer, tiled copy only: 84 GB per GPU at 58 layers and N = 8), attention
    replaced by the identity (h <- h + moe_l(h)).  For each batch of
    --stack-tokens (spread over the ranks, stack_share), one step = the whole
    stack for the batch, replayed as ONE CUDA graph per rank (every layer's
    route, peer exchange, experts, combine and residual add).  Step time =
    max over ranks = the end-to-end latency of every token of the batch.
    Roofline: per layer, the busiest rank's expert bytes (experts hit there +
    its shared expert + router) bound the layer; their sum over the layers ÷
    the step time, against measured HBM bandwidth."""
    import torch.distributed as dist

    from pocketlm_b200 import synth
    from pocketlm_b200.ep import ExpertParallelStack

    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", 0)))
    cfg = synth.C2_DSV3
    L = args.stack_layers
    batches = [int(v) for v in args.stack_tokens.split(",")]
    max_tokens = max(max(stack_share(b, 0, world), 1) for b in batches)
    stack = ExpertParallelStack(cfg, rank, world, L, seed=args.seed, device=dev, max_tokens=max_tokens,
                                peer_sync=args.ep_sync)
    flush = L2Flush(dev)
    peaks = measured_peaks()
    gs, ds = cfg.gate_scale_shape, cfg.down_scale_shape
    expert_bytes = 3 * cfg.inter * cfg.hidden + 4 * (2 * gs[0] * gs[1] + ds[0] * ds[1])
    router_bytes = cfg.n_routed * cfg.hidden * 2
    per_rank = cfg.n_routed // world
    steps = max(3, min(args.steps, 20))
    sweep = {}
    stack_parity: dict = {}
    with ClockSampler(dev.index) as clocks:
        for B in batches:
            T = stack_share(B, rank, world)
            x = synth.make_hidden(T, cfg.hidden, seed=args.seed + 100 * rank + B, device=dev)
            graphed = stack.capture(T) if stack.peer is not None else None
            step = (lambda: graphed(x)) if graphed is not None else (lambda: stack.forward(x))
            # the first replays of a fresh whole-stack graph run slower (measured: the first batch's graph-only
            # time 10 % above its own end-to-end time after 10 warm-up replays, about 90 ms of them); fifty
            # replays before timing -- a fixed count, since every rank replays in lockstep
            warm = max(args.warmup, 50)
            ms = timed_max_over_ranks(step, steps, warm, flush, dev)
            x_host = x.cpu().pin_memory()
            out_host = torch.empty((T, cfg.hidden), dtype=torch.bfloat16).pin_memory()

            def e2e():
                xd = x_host.to(dev, non_blocking=True)
                out = graphed(xd) if graphed is not None else stack.forward(xd)
                out_host.copy_(out, non_blocking=True)

            e2e_ms = timed_max_over_ranks(e2e, steps, warm, flush, dev)
            del graphed  # graphs holding NCCL calls go before the process group
            # routing of one eager step: per layer, the experts each rank serves
            ids_per_layer: list = []
            stack.forward(x, ids_out=ids_per_layer)
            gathered = [None] * world
            dist.all_gather_object(gathered, [i.cpu() for i in ids_per_layer])
            # the checker on layer 0 (every rank takes its collective steps; ranks with tokens check them):
            # the experts its tokens selected, regenerated from their own seeded generators, against the oracle
            out0, ids0, _w0 = stack.layers[0].forward(x)
            rep = None
            if not args.no_parity and T > 0:
                need = sorted({int(v) for v in ids0.reshape(-1).tolist()}) + [cfg.n_routed]
                ref_layer = synth.make_fp8_layer(cfg, seed=args.seed, device=dev, experts=need)
                rep = parity_leg("fp8_layer_parity", ref_layer, x, out0, ids0)
                del ref_layer
            reps = [None] * world
            dist.all_gather_object(reps, rep)
            for r, one in enumerate(reps):
                if one is not None:
                    stack_parity[f"c5-stack-layer0-B{B}-rank{r}"] = one
            crit = stack_critical_bytes(gathered, per_rank, expert_bytes, router_bytes)
            achieved = crit / (ms / 1e3) / 1e9
            sweep[str(B)] = {
                "batch": B, "tokens_per_rank": [stack_share(B, r, world) for r in range(world)],
                "ms_per_step": ms, "per_token_latency_ms": ms, "tokens_per_s": B / (ms / 1e3),
                "e2e_ms": e2e_ms, "e2e_tokens_per_s": B / (e2e_ms / 1e3),
                "critical_path_expert_bytes": crit, "achieved_gbs": achieved,
                "frac_of_hbm": achieved / peaks["hbm_gbs"],
            }
            del x, x_host, out_host
    clock_info = clocks.summary()
    if rank != 0:
        return None
    head = sweep[str(batches[0])]
    cpu = None
    if not args.no_cpu_baseline:
        # derived, as the reference runs one layer after another: its per-layer time x the layers
        try:
            s = cpu_reference_sample(max(1, batches[0]), seed=args.seed, reps=1)
            cpu = {"value": max(1, batches[0]) / (s["seconds_per_sample"] * L), "unit": "tokens/s",
                   "cores": s["cores"], "kind": "reference",
                   "sample": f"derived: the reference's time for one config-2 layer ({s['sample']}) x {L} layers"}
        except Exception as exc:  # a baseline that cannot run must not cost the GPU numbers
            cpu = {"unavailable": f"{type(exc).__name__}: {exc}"}
    return {
        "metric": METRIC, "value": head["tokens_per_s"], "unit": "tokens/s", "n_gpus": world, "steps": steps,
        "warmup": args.warmup, "ms_per_step": head["ms_per_step"], "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "f32 (e4m3 weights decoded exactly, bf16 activations, fp32 accumulate)",
        "data": "synthetic (seeded random DS-V3-shape weights and activations; no checkpoint)",
        "config": {"workload": f"c5-dsv3-stack{L}-decode-B{batches[0]}", "layers": L, "batches": batches,
                   "hidden": cfg.hidden, "moe_intermediate": cfg.inter, "experts": f"{cfg.n_routed}+1",
                   "top_k": cfg.top_k, "parallelism": f"ep{world}", "ep_sync": args.ep_sync,
                   "attention": "identity residual",
                   "l2": "between timed steps 256 MiB written, then 256 MiB of another buffer read"},
        "roofline": {"bound": "hbm", "kernel": "whole stack step, busiest rank per layer",
                     "achieved": head["achieved_gbs"], "peak": peaks["hbm_gbs"], "unit": "GB/s",
                     "frac": head["frac_of_hbm"], "peak_source": f"{peaks['source']} hbm_gbs",
                     "algorithmic_bytes_per_launch": head["critical_path_expert_bytes"], "traffic": None},
        "e2e": {"value": head["e2e_tokens_per_s"], "unit": "tokens/s",
                "h2d_bytes_per_step": stack_share(batches[0], 0, world) * cfg.hidden * 2,
                "d2h_bytes_per_step": stack_share(batches[0], 0, world) * cfg.hidden * 2},
        "exchange": "peer-memory (symmetric memory, NVLink stores), one buffer set for all layers",
        "sweep": sweep, "cpu_baseline": cpu, "clocks": clock_info,
        "parity": None if args.no_parity else {
            "gate": {"rel_l2": 2e-2, "cos_dist": 1e-3, "ids": "bit-exact, ties within 1e-6 excused"},
            "scope": "layer 0 of the stack on each rank's tokens (the whole stack is checked layer by layer "
                     "against the oracle in tests/test_gpu_stack.py)",
            "all_pass": bool(stack_parity) and all(r.get("pass") for r in stack_parity.values()),
            "cases": stack_parity},
    }


def run_ep_prefill(args, rank: int, world: int, ep, timed, peaks) -> dict | None:
    """Config 3 at N > 1: the Zipf-biased DS-V3 layer split expert-parallel
    (256 / N routed experts per rank), --ep-prefill-tokens tokens per rank,
    with either exchange: "nccl" = all-to-alls with host-read counts (the
    step's one host synchronisation); "p2p" = ep.PeerExchange (rows stored
    into the experts' ranks by our dispatch kernel, outputs stored home by the
    down GEMM's epilogue over NVLink).  Each rank's received rows run on the
    tcgen05 grouped GEMM.  Step time = max over ranks; value = N * tokens /
    step time.  The busiest rank's rows (routed pairs received + its own
    shared-expert rows) set the step, so its FLOP rate is reported against the
    bf16 peak."""
    import torch.distributed as dist

    from pocketlm_b200 import synth
    from pocketlm_b200.ep import ExpertParallelLayer

    if args.ep_prefill_tokens == "none":
        return None
    cfg, dev = ep.cfg, ep.device
    tokens = [int(v) for v in args.ep_prefill_tokens.split(",")]
    local = list(range(ep.first, ep.first + ep.n_local)) + [cfg.n_routed]
    zipf = synth.make_fp8_layer(cfg, seed=args.seed + 1, device=dev, bias_kind="zipf", experts=local)
    bf16_peak = peaks.get("bf16_tflops", 1590.0)
    sweeps = {}
    parity = {}
    for exchange in ("nccl", "p2p"):
        pre = ExpertParallelLayer(cfg, rank, world, layer=zipf, device=dev, exchange=exchange,
                                  max_tokens=max(tokens), peer_sync=args.ep_sync)
        sweep = {}
        for T in tokens:
            x = synth.make_hidden(T, cfg.hidden, seed=args.seed + 100 * rank + T, device=dev)
            ms = timed(lambda: pre.forward(x), steps=max(3, min(args.steps, 10)))
            _out, ids, _w = pre.forward(x)
            if exchange == "p2p" and not args.no_parity:
                from oracle.parity import slice_tokens

                sel = slice_tokens(ids, n_spread=32, n_heavy=8)
                need = sorted({int(v) for v in ids[sel].reshape(-1).tolist()}) + [cfg.n_routed]
                ref_layer = synth.make_fp8_layer(cfg, seed=args.seed + 1, device=dev, bias_kind="zipf",
                                                 experts=need)
                rep = parity_leg("fp8_layer_parity", ref_layer, x, _out, ids, sel)
                del ref_layer
                reps = [None] * world
                dist.all_gather_object(reps, rep)
                for r, one in enumerate(reps):
                    parity[f"c3-dsv3-prefill-zipf-T{T}-ep{world}-rank{r}"] = one
            per_rank = torch.bincount(ids.reshape(-1) // ep.n_local, minlength=world).to(torch.int64)
            dist.all_reduce(per_rank)
            rows = per_rank.cpu() + T  # each rank also runs its own tokens' shared expert
            flops = int(rows.max()) * 3 * 2 * cfg.hidden * cfg.inter
            sweep[str(T)] = {
                "tokens_per_gpu": T, "ms_per_step": ms, "tokens_per_s": world * T / (ms / 1e3),
                "rows_per_rank": [int(v) for v in rows], "busiest_rank_tflops": flops / (ms / 1e3) / 1e12,
                "busiest_rank_frac_of_bf16_peak": flops / (ms / 1e3) / 1e12 / bf16_peak,
            }
            del x, ids, _out, _w
        sweeps[exchange] = sweep
        del pre
        torch.cuda.empty_cache()
    del zipf
    torch.cuda.empty_cache()
    return {"workload": "c3-dsv3-prefill-zipf", "parallelism": f"ep{world}",
            "exchanges": {"nccl": "NCCL all-to-all (counts read on the host)",
                          "p2p": "peer memory: dispatch kernel stores rows, down-GEMM epilogue stores outputs home"},
            "expert_kernel": "tcgen05 grouped GEMM (prefill_gemm.cu) when a rank receives >= 16 rows per expert",
            "peak_bf16_tflops": bf16_peak, "peak_source": f"{peaks['source']} bf16_tflops", "sweep": sweeps,
            "parity": parity}


def run_profile_case(args) -> dict:
    """A small case for ncu: the config-2 layer with only the experts that
    `--tokens` tokens select materialised (the others are absent and skipped
    by the kernels), run eagerly warmup + steps times.  Holds about
    (experts selected + 1) x 44 MB of weights instead of 11.3 GB."""
    from pocketlm_b200 import native, synth
    from pocketlm_b200.runtime import DsMoELayerGPU, route_resident_layer

    dev = torch.device("cuda", 0)
    native.load_library()
    cfg = synth.C2_DSV3
    if args.profile_experts:
        # the config-2 expert shapes with fewer routed experts: a few GB on the device, for multi-metric captures
        cfg = synth.DsMoEConfig(f"c2-{args.profile_experts}e", hidden=cfg.hidden, inter=cfg.inter,
                                n_routed=args.profile_experts, top_k=cfg.top_k, n_group=cfg.n_group,
                                topk_group=cfg.topk_group, route_scale=cfg.route_scale)
    xd = synth.make_hidden(args.tokens, cfg.hidden, seed=args.seed).to(dev)
    # route on the GPU with the layer's own (device-generated) router, then
    # materialise exactly the experts that routing selects
    probe = synth.make_fp8_layer(cfg, seed=args.seed, device=dev, experts=[])
    ids = route_resident_layer(probe, xd).indices_tensor
    experts = sorted({int(v) for v in ids.reshape(-1).tolist()}) + [cfg.n_routed]
    if args.profile_no_experts:
        experts = []  # routing kernels only: every expert absent, the GEMVs skip them
    layer = DsMoELayerGPU(synth.make_fp8_layer(cfg, seed=args.seed, device=dev, experts=experts), allow_partial=True)
    for _ in range(args.warmup + args.steps):
        layer.forward(xd)
    torch.cuda.synchronize()
    gs = cfg.gate_scale_shape
    gateup_bytes = len(experts) * (2 * cfg.inter * cfg.hidden + 2 * 4 * gs[0] * gs[1])
    return {"profile_case": f"{cfg.name}-decode-T{args.tokens}", "experts_materialised": len(experts),
            "gateup_algorithmic_bytes": gateup_bytes, "launches": args.warmup + args.steps}


def run_profile_prefill(args) -> dict:
    """A prefill case for ncu: DS-V3 expert shapes (hidden 7168,
    intermediate 2048, top-8) with --profile-prefill-experts routed experts
    + shared (32: about 2.9 GB with the tiled copy, the small case for
    multi-pass captures; 256: the full config-3 layer, for single-pass launch
    lists), --tokens tokens on the tcgen05 GEMM."""
    from pocketlm_b200 import native, synth
    from pocketlm_b200.runtime import DsMoELayerGPU

    dev = torch.device("cuda", 0)
    native.load_library()
    E = args.profile_prefill_experts
    cfg = synth.DsMoEConfig("c3-profile", hidden=7168, inter=2048, n_routed=E, top_k=8, n_group=8, topk_group=4,
                            route_scale=2.5)
    layer = DsMoELayerGPU(synth.make_fp8_layer(cfg, seed=args.seed, device=dev, bias_kind="zipf"))
    x = synth.make_hidden(args.tokens, cfg.hidden, seed=args.seed + 1, device=dev)
    for _ in range(args.warmup + args.steps):
        layer.forward(x)
    torch.cuda.synchronize()
    return {"profile_case": f"c3-shape-{E}-experts-T{args.tokens}", "launches": args.warmup + args.steps}


def run_profile_q4(args) -> dict:
    """A Q4 case for ncu: the config-4 Mixtral layer (8 experts, 2.1 GB of
    packed codes + the tiled copy), --tokens tokens, eager forwards."""
    from pocketlm_b200 import native, synth
    from pocketlm_b200.runtime import Q4MoELayerGPU

    dev = torch.device("cuda", 0)
    native.load_library()
    layer = Q4MoELayerGPU(synth.make_q4_layer(synth.C4_MIXTRAL, seed=args.seed, device=dev))
    x = synth.make_hidden(args.tokens, synth.C4_MIXTRAL.hidden, seed=args.seed + 1, device=dev)
    for _ in range(args.warmup + args.steps):
        layer.forward(x)
    torch.cuda.synchronize()
    return {"profile_case": f"c4-mixtral-q4-T{args.tokens}", "launches": args.warmup + args.steps}


def run_profile_mla(args) -> dict:
    """An MLA case for ncu: the DS-V3 attention block over a cache of
    --mla-cache positions (777 MB of fp32 weights and cache), eager calls."""
    from pocketlm_b200 import native

    dev = torch.device("cuda", 0)
    native.load_library()
    H, qr, R, heads, nope, rope, v = 7168, 1536, 512, 128, 128, 64, 128
    L = int(args.mla_cache)
    g = torch.Generator(device=dev).manual_seed(args.seed)
    w = [torch.randn(s, generator=g, device=dev) * 0.01 for s in
         ((qr, H), (heads * (nope + rope), qr), (R + rope, H), (heads * (nope + v), R), (H, heads * v))]
    norms = [torch.ones(qr, device=dev), torch.ones(R, device=dev)]
    prev_kv, prev_pe = torch.randn((L - 1, R), device=dev), torch.randn((L - 1, rope), device=dev)
    cos, sin = torch.ones(rope // 2, device=dev), torch.zeros(rope // 2, device=dev)
    x = torch.randn(H, device=dev)
    with native.DeepSeekNativeSession(num_layers=1, hidden_dim=H, num_experts=0, top_k=0) as session:
        for _ in range(args.warmup + args.steps):
            native.ds_attention_block_forward(session, x, *w, *norms, previous_kv_cache=prev_kv,
                                              previous_pe_cache=prev_pe, rope_cos=cos, rope_sin=sin, q_lora_rank=qr,
                                              kv_lora_rank=R, num_heads=heads, qk_nope_dim=nope, qk_rope_dim=rope,
                                              v_head_dim=v, rms_eps=1e-6, softmax_scale=(nope + rope) ** -0.5)
    torch.cuda.synchronize()
    return {"profile_case": f"dsv3-mla-block-cache{L}", "launches": args.warmup + args.steps}


def run_reference(args, rank: int, world: int) -> dict | None:
    if rank != 0:
        return None
    from oracle import ref

    if not ref.available():
        return {"impl": "reference", "unavailable": "reference CPU build (oracle/_ref) missing"}
    samples = []
    inputs = cpu_decode_sample_inputs(args.tokens, args.seed)  # the whole batch, generated once, timed per step
    for i in range(args.warmup + args.steps):
        s = cpu_reference_sample(args.tokens, seed=args.seed, reps=1, inputs=inputs)
        if i >= args.warmup:
            samples.append(s["seconds_per_sample"])
    per = statistics.mean(samples)
    value = args.tokens / per
    return {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": per * 1e3, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32 (reference CPU: e4m3 LUT decode, fp32 accumulate)",
        "data": "synthetic (seeded random DS-V3-shape weights and activations; no checkpoint)",
        "config": {"workload": f"c2-dsv3-decode-T{args.tokens}", "tokens_per_gpu": args.tokens,
                   "hidden": 7168, "moe_intermediate": 2048, "experts": "256+1", "top_k": 8,
                   "parallelism": "host CPU", "routed_experts_in_batch": len(inputs[2])},
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": len(os.sched_getaffinity(0)),
                         "kind": "reference", "sample": s["sample"]},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


def main() -> None:
    parser = argparse.ArgumentParser()
    parser.add_argument("--gpus", type=int, default=1)
    parser.add_argument("--steps", type=int, default=50)
    parser.add_argument("--warmup", type=int, default=5)
    parser.add_argument("--tokens", type=int, default=64)
    parser.add_argument("--seed", type=int, default=20)
    parser.add_argument("--impl", choices=["ours", "reference"], default="ours")
    parser.add_argument("--no-cpu-baseline", action="store_true")
    parser.add_argument("--fused-decode", action="store_true",
                        help="run decode experts as one fused launch (decode_fused_kernel) instead of three")
    parser.add_argument("--no-alt-compare", action="store_true",
                        help="skip timing the other decode-experts variant (fused / three launches) beside the run one")
    parser.add_argument("--no-parity", action="store_true",
                        help="skip the parity leg (the oracle on each timed batch, after its timing)")
    parser.add_argument("--cpu-prefill-experts", type=int, default=4,
                        help="experts of the config-3 batch whose rows are timed through the reference's CPU kernel")
    parser.add_argument("--cpu-prefill-full", type=int, default=2048,
                        help="config-3 batch also timed whole through the reference's CPU flow (0: none)")
    parser.add_argument("--cpu-q4-tokens", type=int, default=4,
                        help="tokens of the config-4 batch timed through the reference's CPU token loop")
    parser.add_argument("--sweep", default="1,4,16,64",
                        help="comma-separated extra batch sizes measured after --tokens, or 'none'")
    parser.add_argument("--gemv", choices=list(GEMV_IMPLS), default="auto",
                        help="expert GEMV kernel (moe_b200_select_gemv); auto is the product default")
    parser.add_argument("--prefill-tokens", default="2048,8192,16384",
                        help="config-3 prefill batch sizes measured after the decode sweep, or 'none'")
    parser.add_argument("--mla-cache", default="4096",
                        help="cache positions of the MLA attention block leg ('none' to skip)")
    parser.add_argument("--q4-tokens", default="1,32,512,4096",
                        help="config-4 (Mixtral Q4) batch sizes measured after the prefill sweep, or 'none'")
    parser.add_argument("--ep-prefill-tokens", default="8192",
                        help="config-3 expert-parallel prefill tokens per rank measured after the decode step "
                             "at N > 1, or 'none'")
    parser.add_argument("--ep-sync", choices=["p2p", "nccl"], default="p2p",
                        help="N > 1, peer exchange: order its phases with the peer-memory barrier kernel (default) "
                             "or with NCCL collectives")
    parser.add_argument("--stack-layers", type=int, default=0,
                        help="config 5: time the expert-parallel stack of this many layers (58 = DS-V3) "
                             "instead of the one-layer bench; needs N GPUs with room for layers * 257 / N experts")
    parser.add_argument("--stack-tokens", default="1,2,32",
                        help="config-5 decode batches (spread over the ranks)")
    parser.add_argument("--profile", action="store_true",
                        help="run the small ncu case (selected experts only) instead of the benchmark")
    parser.add_argument("--profile-prefill", action="store_true",
                        help="run the small prefill ncu case (DS-V3 expert shapes, 32 experts) instead")
    parser.add_argument("--profile-prefill-experts", type=int, default=32,
                        help="routed experts of the --profile-prefill layer (32 small case, 256 full config 3)")
    parser.add_argument("--profile-mla", action="store_true",
                        help="eager MLA attention blocks (DS-V3 shape, --mla-cache positions) for ncu; no JSON bench line")
    parser.add_argument("--profile-q4", action="store_true",
                        help="run the config-4 Q4 layer for --tokens tokens (an ncu case)")
    parser.add_argument("--profile-experts", type=int, default=0,
                        help="with --profile: routed experts of the profiled layer (0: config 2's 256)")
    parser.add_argument("--profile-no-experts", action="store_true",
                        help="with --profile: materialise no expert (for captures of the routing kernels)")
    args = parser.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    # a process group for N > 1, and for the stack at N = 1 too (its exchange steps are collectives)
    use_pg = args.impl == "ours" and (world > 1 or args.stack_layers > 0)
    if use_pg:
        import datetime

        torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", 0)))
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        os.environ.setdefault("MASTER_PORT", "29571")
        torch.distributed.init_process_group("nccl", rank=rank, world_size=world,
                                             timeout=datetime.timedelta(seconds=120))
    if args.impl == "ours":
        from pocketlm_b200 import native

        native.load_library().moe_b200_select_gemv(GEMV_IMPLS[args.gemv])
        native.load_library().moe_b200_fused_decode(1 if args.fused_decode else 0)
    try:
        if args.profile_prefill:
            result = run_profile_prefill(args)
        elif args.profile_q4:
            result = run_profile_q4(args)
        elif args.profile_mla:
            result = run_profile_mla(args)
        elif args.profile:
            result = run_profile_case(args)
        else:
            if args.impl == "reference":
                result = run_reference(args, rank, world)
            elif args.stack_layers > 0:
                result = run_stack(args, rank, world)
            elif world > 1:
                result = run_ours_ep(args, rank, world)
            else:
                result = run_ours(args, rank, world)
        if result is not None:
            print(json.dumps(result), flush=True)
    finally:
        if use_pg:
            torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
