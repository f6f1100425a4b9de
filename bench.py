#!/usr/bin/env python3
"""Decode benchmark: Qwen3-30B-A3B-shape Q4_K_M model, batch 1, ctx 4096.

A step is one greedy decode token (the whole forward: 48 layers + vocab
projection + argmax) on the device.  Inputs: a random-init synthetic model
(N(0, 0.02) weights quantized by libqwen_tools, seed 0) and a 512-token random
prompt (seed 1) prefilled before timing; weights per step (~2 GB) exceed the
126 MB L2, so no flush is needed between steps.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                  [--config 2|3|4] [--replicas]

Prints one JSON line on rank 0.  `value` is device-resident decode tok/s over
all ranks; `e2e` is tok/s through qc_forward with the token copied in and the
logits copied out (pinned host memory) every step, and the host picking the
argmax, as the reference's chat loop does.  With N > 1 the N ranks run ONE
decode stream with the experts split over them (expert parallelism: each rank
holds experts/N, partial MoE vectors exchanged over NVLink inside the token
kernel; scaling "strong"); --replicas runs N independent streams instead.
At N = 1 the line also carries BASELINE config 2 (`matvec`: every isolated
matvec shape, event-timed GB/s with > 126 MB of distinct weights rotated past
L2) and config 3 (`moe_layer`: one MoE layer at 1-128 tokens, per-token kernels
against the tcgen05 grouped GEMMs), and the CPU baseline (the reference's CPU
path, 1 thread and all host threads).  `--impl reference` times the reference's
CPU path (the C++ restatement under oracle/, all host threads) on the same
model, at the same positions and step count.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))
from __graft_entry__ import load_package  # noqa: E402

load_package()

METRIC = "decode tok/s, Qwen3-30B-A3B-shape Q4_K_M ctx4096; matvec HBM GB/s vs peak"
PROMPT = 512
CTX = 4096


def log(*a):
    print(*a, file=sys.stderr, flush=True)


def peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": d["hbm_gbs"], "source": "measured"}
    return {"hbm_gbs": 6650.0, "source": "fallback"}


# DRAM bytes (dram__bytes_read.sum + dram__bytes_write.sum) of one k_token launch, from an ncu capture of
# `bench.py --layers 4` (4 layers of the same shapes): fixed part (vocab projection, logits) + per layer;
# a 48-layer token is scaled by the layer count (traffic grows in proportion to the layers).
TOKEN_TRAFFIC_FIXED, TOKEN_TRAFFIC_PER_LAYER = 255.9e6, 39.65e6


def model_bytes(spec, tools, pos_first: int, steps: int) -> dict:
    """Algorithmic bytes of one decode step (weights read once, KV read, KV row written)."""
    rb = tools.row_bytes
    H, L, D = spec.hidden, spec.layers, spec.head_dim
    Q, KV = spec.heads * D, spec.kvheads * D
    attn_w = Q * rb(spec.kind_attn, H) + 2 * KV * rb(spec.kind_attn, H)
    o_w = H * rb(spec.kind_attn_out, Q)
    router_w = spec.experts * rb(spec.kind_router, H)
    gate_up_w = spec.top * 2 * spec.intermediate * rb(spec.kind_gate_up, H)
    down_w = spec.top * H * rb(spec.kind_down, spec.intermediate)
    norms = (2 * H + 2 * D) * 4
    out_w = spec.vocab * rb(spec.kind_output, H)
    weights = L * (attn_w + o_w + router_w + gate_up_w + down_w + norms) + out_w + H * 4 + rb(spec.kind_embd, H)
    kv_row = 2 * KV * 4  # K and V of one position, one layer
    mean_time = pos_first + (steps + 1) / 2.0  # attended positions (pos + 1), averaged over the steps
    kv_read = L * kv_row * mean_time
    per_kernel = {  # per launch
        "attn_in": attn_w + 2 * H * 4 + (Q + 2 * KV) * 4,
        "attention": kv_row * mean_time + kv_row + (Q + 2 * KV) * 4 + Q * 4,
        "oproj": o_w + Q * 4 + 2 * H * 4,
        "router": router_w + 3 * H * 4,
        "gateup": gate_up_w + H * 4 + spec.top * spec.intermediate * 4,
        "down": down_w + spec.top * spec.intermediate * 4 + 2 * H * 4,
        "output": out_w + H * 8 + spec.vocab * 4,
        "embed": rb(spec.kind_embd, H) + H * 4,
    }
    return {"weights": weights, "kv_read": kv_read, "kv_write": L * kv_row, "per_token": weights + kv_read + L * kv_row,
            "per_kernel": per_kernel, "experts": L * (gate_up_w + down_w)}


class ClockSampler:
    """Samples SM clock and throttle reasons of one GPU (NVML) every 200 ms."""

    REASONS = {0x4: "sw_power_cap", 0x8: "hw_slowdown", 0x20: "sw_thermal_slowdown", 0x40: "hw_thermal_slowdown",
               0x80: "hw_power_brake_slowdown", 0x2: "applications_clocks_setting"}

    def __init__(self, device: int):
        self.samples, self.reasons, self.max_mhz, self._stop = [], set(), None, threading.Event()
        self.ok = False
        try:
            import pynvml
            import torch
            pynvml.nvmlInit()
            uuid = str(torch.cuda.get_device_properties(device).uuid)
            self.h = pynvml.nvmlDeviceGetHandleByUUID(uuid if uuid.startswith("GPU-") else "GPU-" + uuid)
            self.nv = pynvml
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
            self.ok = True
        except Exception as e:  # no NVML: report no clocks rather than fail the bench
            log("clock sampler unavailable:", e)

    def _run(self):
        while not self._stop.is_set():
            try:
                self.samples.append(self.nv.nvmlDeviceGetClockInfo(self.h, self.nv.NVML_CLOCK_SM))
                r = self.nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)
                for bit, name in self.REASONS.items():
                    if r & bit:
                        self.reasons.add(name)
            except Exception:
                pass
            self._stop.wait(0.2)

    def __enter__(self):
        if self.ok:
            self.t = threading.Thread(target=self._run, daemon=True)
            self.t.start()
        return self

    def __exit__(self, *a):
        self._stop.set()
        if self.ok:
            self.t.join()

    def summary(self) -> dict:
        return {"sm_mhz": statistics.median(self.samples) if self.samples else None, "sm_max_mhz": self.max_mhz,
                "reasons": sorted(self.reasons), "samples": len(self.samples)}


def cpu_cores() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except Exception:
        return os.cpu_count() or 1


def cpu_model() -> str:
    try:
        for line in open("/proc/cpuinfo"):
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except Exception:
        pass
    return "unknown"


def cpu_decode(img, tokens: list[int], threads: int) -> dict:
    """The reference's CPU path (oracle restatement, row-parallel over `threads`, every element
    decoded per use as backend.rs:28-52 does) on `tokens`; the first token is untimed (page-in)."""
    from oracle import oracle as O
    if not O.LIB_PATH.exists():
        O.build()
    m = O.Model(img, CTX, threads=threads)
    m.forward(tokens[0])
    t0 = time.perf_counter()
    for t in tokens[1:]:
        m.forward(t)
    dt = time.perf_counter() - t0
    m.close()
    return {"tok_s": (len(tokens) - 1) / dt, "seconds": dt, "tokens": len(tokens) - 1}


def cpu_baseline(img, prompt, ncores: int, tokens_all: int) -> dict:
    """CPU baseline of the main line: 1 thread (the reference's own CPU path is single-threaded,
    backend.rs:40-48) over 1 token and all host threads over `tokens_all` tokens, positions 1.."""
    toks = [int(x) for x in prompt[:tokens_all + 1]]
    one = cpu_decode(img, toks[:2], 1)
    allc = cpu_decode(img, toks, ncores)
    return {"value": allc["tok_s"], "unit": "tok/s", "cores": ncores, "kind": "port",
            "single_thread": {"value": one["tok_s"], "unit": "tok/s", "cores": 1, "seconds": one["seconds"],
                              "tokens": one["tokens"]},
            "sample": f"{allc['tokens']} decode tokens at positions 1..{allc['tokens']} of the same 30B-shape "
                      f"model over {ncores} threads ({allc['seconds']:.1f} s), and 1 token at position 1 on 1 "
                      f"thread ({one['seconds']:.1f} s): C++ restatement of backend.rs Cpu::matvec (per-element "
                      f"decode, sequential f32 folds) + ops.rs + model.rs, row-parallel, bit-identical for any "
                      f"thread count; {cpu_model()}"}


# (name, GGML kind, rows, cols) of every isolated matvec shape; each shape's Q8_0
# variant follows.
def matvec_shapes(T) -> list:
    base = [("q_proj", T.Q4_K, 4096, 2048), ("kv_proj", T.Q4_K, 512, 2048), ("o_proj", T.Q4_K, 2048, 4096),
            ("gate_up", T.Q4_K, 768, 2048), ("gate_up_q5k", T.Q5_K, 768, 2048), ("down", T.Q6_K, 2048, 768),
            ("router", T.F16, 128, 2048), ("vocab", T.Q6_K, 151936, 2048),
            # not a config-2 shape: the gate rows of all 128 experts of a layer as one Q4_K matrix
            # (113 MB), the Q4_K format streamed at a size where launch latency does not dominate
            ("gate_all_experts", T.Q4_K, 98304, 2048)]
    q8 = [(n + "_q8_0", T.Q8_0, r, c) for n, k, r, c in base if k != T.Q5_K and n != "gate_all_experts"]
    return base + q8


def matvec_study(T, E, torch, steps: int, warmup: int, only: str | None = None, rotate: int = 512 << 20) -> dict:
    """y = W x for every shape through qc_matrix_matvec, x ~ N(0,1), W ~ N(0,0.02)
    quantized from seed 0.  Each shape is uploaded as `copies` stacked matrices (>= 512 MB of distinct
    weights, so L2 serves no repeat) and one CUDA graph launches the kernel once per copy; the graph is
    replayed `steps` times between CUDA events.  GB/s = algorithmic bytes (packed W + 4 cols + 4 rows)
    per launch / the average launch time (inter-kernel gaps inside the graph included)."""
    pk = peaks()
    stream = torch.cuda.Stream()
    out = []
    for name, kind, rows, cols in matvec_shapes(T):
        if only and name != only:
            continue
        blocks = T.random_matrix(kind, rows, cols, seed=0, stream=T.stream_of(name))
        packed = blocks.size
        copies = int(min(1024, max(2, -(-rotate // packed))))
        m = E.Matrix(kind, rows, cols, np.tile(blocks, copies), experts=copies)
        del blocks
        g = torch.Generator(device="cuda").manual_seed(1)
        x = torch.randn(cols, device="cuda", dtype=torch.float32, generator=g)
        y = torch.empty(rows, device="cuda", dtype=torch.float32)
        with torch.cuda.stream(stream):
            m.matvec(x.data_ptr(), y.data_ptr(), stream.cuda_stream, expert=0)  # outside capture: first launch
        stream.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            for i in range(copies):
                m.matvec(x.data_ptr(), y.data_ptr(), stream.cuda_stream, expert=i)
        for _ in range(warmup):
            graph.replay()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        with torch.cuda.stream(stream):
            e0.record(stream)
            for _ in range(steps):
                graph.replay()
            e1.record(stream)
        torch.cuda.synchronize()
        us = e0.elapsed_time(e1) * 1e3 / (steps * copies)
        alg = packed + 4 * cols + 4 * rows
        gbs = alg / (us * 1e-6) / 1e9
        out.append({"shape": name, "kind": T.KIND_NAMES[kind], "rows": rows, "cols": cols, "packed_bytes": packed,
                    "bytes_per_launch": alg, "us_per_launch": us, "gbs": gbs, "frac": gbs / pk["hbm_gbs"],
                    "copies_rotated": copies})
        log(f"matvec {name:>14} {T.KIND_NAMES[kind]:>5} {rows}x{cols}: {us:8.2f} us  {gbs:7.1f} GB/s "
            f"({gbs / pk['hbm_gbs']:.3f} of peak)")
        del graph, m
    return {"results": out, "peak_gbs": pk["hbm_gbs"], "peak_source": pk["source"],
            "timing": f"CUDA events around {steps} replays of a graph of one launch per rotated copy; "
                      f"L2 defeated by >= {rotate >> 20} MB of distinct weights per shape"}


def moe_study(T, E, steps: int, warmup: int) -> dict:
    """one Qwen3-30B-A3B MoE layer for T in {1, 8, 32, 128} tokens, per-token
    decode kernels (path 1, matvecs) against tcgen05 grouped GEMMs (path 2); Zipf-skewed router."""
    spec = T.QWEN3_30B_A3B.with_(layers=1, vocab=512)
    img = T.synth_gguf(spec)
    T.skew_router(img, 0, 1.1)
    eng = E.Engine(img, 16)
    H, I, NE, top = spec.hidden, spec.intermediate, spec.experts, spec.top
    rv, _, _ = T.tensor_view(img, "blk.0.ffn_gate_inp.weight")
    router = np.frombuffer(rv.tobytes(), dtype=np.float16).reshape(NE, H).astype(np.float64)
    norm = np.frombuffer(T.tensor_view(img, "blk.0.ffn_norm.weight")[0].tobytes(), dtype=np.float32)
    gate_b, down_b = T.row_bytes(T.Q4_K, H) * I, T.row_bytes(T.Q6_K, I) * H
    expert_bytes = 2 * gate_b + down_b
    rng = np.random.default_rng(7)
    rows, load = [], np.zeros(NE, dtype=np.int64)
    for tokens in (1, 8, 32, 128):
        x = rng.normal(size=(tokens, H)).astype(np.float32)
        h = x / np.sqrt((x.astype(np.float64) ** 2).mean(axis=1, keepdims=True) + spec.eps) * norm
        sel = np.argsort(-(h @ router.T), axis=1, kind="stable")[:, :top]  # workload statistic only
        distinct = len(np.unique(sel))
        np.add.at(load, sel.ravel(), 1)
        res = {"tokens": tokens, "distinct_experts": distinct, "tokens_per_expert": tokens * top / distinct}
        byts = NE * H * 2 + distinct * expert_bytes
        flops = 2 * tokens * top * 3 * H * I
        for path in (1, 2):
            for _ in range(warmup):
                eng.moe_layer(0, x, path)
            ms = sorted(eng.moe_layer(0, x, path)[1] for _ in range(steps))
            med = ms[len(ms) // 2]
            res[f"path{path}"] = {"ms": med, "tok_s": tokens / (med / 1e3), "gbs": byts / (med / 1e3) / 1e9,
                                  "tflops": flops / (med / 1e3) / 1e12}
        res["bytes"], res["flops"] = byts, flops
        res["speedup_tc"] = res["path1"]["ms"] / res["path2"]["ms"]
        rows.append(res)
        log(f"moe T={tokens}: distinct {distinct}, per-token kernels {res['path1']['ms']:.3f} ms, "
            f"tensor cores {res['path2']['ms']:.3f} ms")
    eng.close()
    cross = next((r["tokens_per_expert"] for r in rows if r["speedup_tc"] > 1.0), None)
    ranked = np.sort(load)[::-1]
    return {"results": rows, "crossover_tokens_per_expert": cross,
            "load_share_top_8_experts": float(ranked[: max(1, NE // 16)].sum() / max(1, ranked.sum())),
            "timing": "device time of qc_moe_layer (CUDA events), median of steps",
            "data": "synthetic: N(0,0.02) weights (seed 0), router row e scaled by (e+1)^-1.1, hidden N(0,1) (seed 7)"}


def synth_image(tools, spec, rank: int, world: int):
    """The model image: in memory for one rank; shared through a file for several."""
    if world == 1:
        t = time.time()
        img = tools.synth_gguf(spec)
        log(f"synthetic model: {img.size / 1e9:.2f} GB in {time.time() - t:.1f} s on {cpu_cores()} cores")
        return img, None
    import torch.distributed as dist
    shm = Path("/dev/shm")
    n = tools.synth_size(spec)
    d = shm if shm.exists() and os.statvfs(shm).f_bavail * os.statvfs(shm).f_frsize > n * 1.1 else Path("/tmp")
    path = d / f"qwen30b_synth_seed{spec.seed}_{n}.gguf"
    if rank == 0 and not path.exists():
        img = tools.synth_gguf(spec)
        tmp = path.with_suffix(".tmp")
        img.tofile(tmp)
        os.replace(tmp, path)
        del img
    dist.barrier()
    return None, path


def run_ours(args) -> None:
    import torch
    from qwen30brust_b200 import engine as E, tools as T

    rank = int(os.environ.get("RANK", 0))
    world = int(os.environ.get("WORLD_SIZE", 1))
    local = int(os.environ.get("LOCAL_RANK", 0))
    torch.cuda.set_device(local)
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600), device_id=torch.device("cuda", local))
    spec = T.QWEN3_30B_A3B
    if args.layers:  # a shallower model of the same shapes: profiling runs only, not a bench line
        spec = spec.with_(layers=args.layers)
    img, path = synth_image(T, spec, rank, world)
    t = time.time()
    ep = world > 1 and not args.replicas
    if ep:  # one stream over all ranks: this rank's experts, peers' exchange buffers over NVLink
        src = img if img is not None else np.memmap(path, dtype=np.uint8, mode="r")
        eng = E.Engine.expert_parallel(src, CTX, local, rank, world)
        del src
        E.connect_group(eng)
    else:
        eng = E.Engine(path if path is not None else img, CTX, device=local)
    eng.set_decode_mode(args.decode_mode)
    decode_path = eng.decode_path
    log(f"rank {rank}: engine up in {time.time() - t:.1f} s; decode path {decode_path}")
    stream = torch.cuda.Stream()  # a real stream: NULL would mean the engine's own stream
    torch.cuda.set_stream(stream)
    eng.set_stream(stream.cuda_stream)
    prompt = np.random.default_rng(1).integers(0, spec.vocab, PROMPT).astype(np.uint32)
    eng.forward_tokens(prompt, want_logits=False)
    eng.decode_greedy(args.warmup)
    phases = eng.profile_step()
    pos0 = eng.position

    def barrier():
        if world > 1:
            import torch.distributed as dist
            dist.barrier()
        torch.cuda.synchronize()

    # ---- device-resident decode: K greedy steps chained on the device
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    sampler = ClockSampler(local)
    barrier()
    with sampler:
        ev0.record(stream)
        eng.decode_enqueue(args.steps)
        ev1.record(stream)
        torch.cuda.synchronize()
    eng.sync()
    barrier()
    ms = ev0.elapsed_time(ev1)

    # ---- end to end through qc_forward: token in, logits out, host argmax
    k2 = min(args.steps, CTX - eng.position - 1, 256)
    host_logits = torch.empty(spec.vocab, dtype=torch.float32, pin_memory=True).numpy()
    tok = int(eng.decode_greedy(1)[0][0])
    for _ in range(2):  # warm the host path
        eng.forward_into(tok, host_logits)
        tok = int(np.argmax(host_logits))
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    w0 = time.perf_counter()
    e0.record(stream)
    for _ in range(k2):
        eng.forward_into(tok, host_logits)
        tok = int(np.argmax(host_logits))
    e1.record(stream)
    torch.cuda.synchronize()
    wall_e2e = time.perf_counter() - w0
    ms_e2e = e0.elapsed_time(e1)
    barrier()

    times = torch.tensor([ms, ms_e2e], dtype=torch.float64, device="cuda")
    if world > 1:
        import torch.distributed as dist
        dist.all_reduce(times, op=dist.ReduceOp.MAX)
    ms, ms_e2e = times.tolist()
    studies = {}
    if world == 1 and not args.layers and not args.no_studies:  # BASELINE config 5, reduced, on the same engine
        try:
            studies["batch"] = dict(batch_study(T, E, eng, spec, 64, 128, 16),
                                    workload="BASELINE config 5 shape, reduced: 64 sequences x 128-token prompts, "
                                             "16 sampled steps (bench.py --config 5 runs 2048 x 512)")
        except Exception as exc:
            log(f"batch study failed: {exc!r}")
            studies["batch"] = {"error": repr(exc)}
    eng.close()
    if world == 1 and not args.layers and not args.no_studies:  # BASELINE configs 2 and 3 beside the decode line
        for key, fn in (("matvec", lambda: matvec_study(T, E, torch, steps=5, warmup=3)),
                        ("moe_layer", lambda: moe_study(T, E, steps=7, warmup=3))):
            try:
                studies[key] = fn()
            except Exception as exc:  # a failed study must not cost the decode line; it is reported instead
                log(f"{key} study failed: {exc!r}")
                studies[key] = {"error": repr(exc)}

    if rank == 0:
        pk = peaks()
        b = model_bytes(spec, T, pos0, args.steps)
        step_ms = ms / args.steps
        streams = 1 if ep else world  # decode streams the job runs
        if ep:  # per rank: replicated weights, KV and 1/world of the selected experts (uniform routing)
            b = dict(b, per_token=b["per_token"] - b["experts"] * (1 - 1 / world))
        value = args.steps * streams / (ms / 1e3)
        kinds = [k for k in E.PHASES]
        if phases["launches"] == 1:
            # the whole-token kernel is the step: its bytes are the token's, its duration the timed average
            dom, dom_ms, dom_bytes = "token", step_ms, b["per_token"]
            traffic = None if ep else TOKEN_TRAFFIC_FIXED + TOKEN_TRAFFIC_PER_LAYER * spec.layers  # 1-GPU capture
            phases_ms = {"token": phases["token"]}
        else:
            # dominant kernel of the step by device time (per-kernel CUDA events in a captured step graph)
            dom = max(kinds, key=lambda k: phases[k])
            launches = 1 if dom in ("embed", "output") else spec.layers
            dom_ms = phases[dom] / launches
            dom_bytes = b["per_kernel"][dom]
            phases_ms = {k: phases[k] for k in kinds}
            traffic = None
        achieved = dom_bytes / (dom_ms / 1e3) / 1e9
        step_gbs = b["per_token"] / (step_ms / 1e3) / 1e9
        cpu = None
        if not args.no_cpu_baseline and world == 1:
            src = img if img is not None else np.fromfile(path, dtype=np.uint8)
            cpu = cpu_baseline(src, prompt, cpu_cores(), args.cpu_tokens)
        out = {
            "metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": step_ms, "higher_is_better": True,
            "scaling": "strong" if ep else "weak",
            "vs_baseline": None, "dtype": "f32 (activations, accumulate); Q4_K/Q6_K/F16/Q8_0 weights",
            "data": "synthetic: random-init N(0,0.02) weights quantized from seed 0; 512-token random prompt (seed 1)",
            "config": {"workload": "BASELINE config 4: Qwen3-30B-A3B-shape decode, batch 1, greedy"
                       if not args.layers else f"profiling run: config 4 shapes with {args.layers} layers (not a bench line)",
                       "layers": spec.layers, "hidden": spec.hidden, "heads": f"{spec.heads}q/{spec.kvheads}kv x {spec.head_dim}",
                       "experts": f"{spec.experts} top-{spec.top}", "intermediate": spec.intermediate,
                       "vocab": spec.vocab, "ctx": CTX, "prompt": PROMPT, "positions": [pos0, pos0 + args.steps - 1],
                       "kv": "fp32",
                       "parallelism": (f"expert parallel x{world} (one stream)" if ep else f"replicas x{world}")
                       if world > 1 else "single GPU",
                       "l2": "no flush: each step reads ~2.07 GB of weights and KV, > 126 MB L2"},
            "hbm_roofline_decode": {"bytes_per_token": b["per_token"],
                                    "bytes_scope": "per rank (expert parallel)" if ep else "per stream", "achieved_gbs": step_gbs, "peak_gbs": pk["hbm_gbs"],
                                    "frac": step_gbs / pk["hbm_gbs"], "roofline_tok_s": pk["hbm_gbs"] * 1e9 / b["per_token"],
                                    "peak_source": pk["source"]},
            "roofline": {"kernel": f"k_{dom}", "bound": "hbm", "achieved": achieved, "peak": pk["hbm_gbs"], "unit": "GB/s",
                         "frac": achieved / pk["hbm_gbs"], "traffic": traffic,
                         "traffic_source": "ncu dram bytes of a 4-layer capture scaled by layers" if traffic else None,
                         "bytes_per_launch": dom_bytes, "ms_per_launch": dom_ms, "peak_source": pk["source"]},
            "phases_ms": phases_ms,
            "decode_path": "whole-token kernel (1 launch per token)" if decode_path[0] == 0
                           else f"per-phase kernels ({phases['launches']} launches per token)",
            "e2e": {"value": k2 * streams / (ms_e2e / 1e3), "unit": "tok/s", "steps": k2,
                    "h2d_bytes_per_step": 4, "d2h_bytes_per_step": spec.vocab * 4 + 8,
                    "wall_tok_s": k2 / wall_e2e,
                    "path": "qc_forward(token -> logits) per step + host argmax (reference chat loop, greedy)"},
            "cpu_baseline": cpu,
            "gpu_launches": phases["launches"] * args.steps,
            "clocks": sampler.summary(),
        }
        if ep:  # what crosses NVLink: every rank stores its partial MoE vector into every rank, per layer
            out["expert_parallel"] = {"ranks": world, "experts_per_rank": spec.experts // world,
                                      "weight_bytes_per_token_per_rank": b["per_token"],
                                      "exchange_bytes_per_token_per_rank": spec.layers * world * spec.hidden * 8,
                                      "exchange": "8-byte tagged f32 peer stores inside k_token, one per layer"}
        out.update(studies)
        print(json.dumps(out), flush=True)
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
        dist.destroy_process_group()
        if rank == 0 and path is not None:
            try:
                path.unlink()
            except OSError:
                pass


def run_reference(args) -> None:
    """The reference's own CPU path (its C++ restatement, all host threads), same metric, model and
    positions as the repo arm: the 512-token prompt and the repo arm's warm-up and profiled steps
    are prefilled (untimed, layer-major, bit-identical to token-by-token forwards), then `warmup`
    untimed and `steps` timed decode tokens at the repo arm's positions, each a full forward of
    the reference's per-element-decode path."""
    rank = int(os.environ.get("RANK", 0))
    if rank != 0:
        return
    from qwen30brust_b200 import tools as T
    from oracle import oracle as O
    if not O.LIB_PATH.exists():
        O.build()
    spec = T.QWEN3_30B_A3B
    img = T.synth_gguf(spec)
    ncores = cpu_cores()
    steps = max(1, min(args.steps, args.ref_max_steps))  # bounded: each step is ~1.5 s of CPU work
    prompt = np.random.default_rng(1).integers(0, spec.vocab, PROMPT).astype(np.uint32)
    # the repo arm times positions PROMPT + warmup + 1 ..: it runs the prompt, `warmup` greedy steps
    # and one profiled step first.  Here: the prompt and one more token prefilled (untimed), then
    # `warmup` untimed steps, so the timed steps run at the same positions.
    m = O.Model(img, CTX, threads=ncores, fast=True)
    t0 = time.perf_counter()
    m.prefill(np.concatenate([prompt, prompt[-1:]]))
    prefill_s = time.perf_counter() - t0
    m.set_fast(False)  # timed steps: every element decoded per use, as Cpu::matvec (backend.rs:28-52)
    tok = int(prompt[0])
    for _ in range(args.warmup):
        tok = O.sample_greedy(m.forward(tok))
    pos0 = m.position
    t0 = time.perf_counter()
    for _ in range(steps):
        tok = O.sample_greedy(m.forward(tok))
    dt = time.perf_counter() - t0
    value = steps / dt
    sample = (f"{steps} greedy decode tokens at positions {pos0}..{pos0 + steps - 1} of the 30B-shape model after a "
              f"{PROMPT}-token prompt (prefilled untimed in {prefill_s:.0f} s) and {args.warmup} untimed steps; C++ "
              f"restatement of the reference CPU path (per-element decode, sequential f32 folds), row-parallel over "
              f"{ncores} threads; {cpu_model()}")
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": 0, "steps": steps,
        "warmup": args.warmup, "ms_per_step": dt / steps * 1e3, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32",
        "data": "synthetic: random-init N(0,0.02) weights quantized from seed 0; 512-token random prompt (seed 1)",
        "config": {"workload": "BASELINE config 4: Qwen3-30B-A3B-shape decode, batch 1, greedy", "ctx": CTX,
                   "prompt": PROMPT, "positions": [pos0, pos0 + steps - 1]},
        "cpu_baseline": {"value": value, "unit": "tok/s", "cores": ncores, "kind": "port", "sample": sample},
        "e2e": {"value": value, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)


def batch_study(T, E, eng, spec, seqs: int, prompt: int, gen: int, log_every: int = 0, rank: int = 0,
                world: int = 1) -> dict:
    """`seqs` sequences, each a `prompt`-token random prompt (seed 3) prefilled in
    chunks of 128 tokens (one sequence per call), then `gen` decode steps of all sequences at once on
    the device (qc_batch_decode_sample: sample every sequence, run the step), temperature 0.7, top-p
    0.9, top-k off, one seeded sampler per sequence.  With world > 1 (an expert-parallel engine) this
    rank runs sequences [rank * seqs / world, (rank + 1) * seqs / world) and the counts returned are
    this rank's."""
    import torch
    n = seqs // world
    first = rank * n
    b = E.Batch(eng, n, CTX)
    if world > 1:
        E.connect_group(b)
    rng = np.random.default_rng(3)
    prompts = rng.integers(0, spec.vocab, (seqs, prompt)).astype(np.uint32)[first:first + n]
    seqs = n
    torch.cuda.synchronize()
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
    s0 = b.stats()
    w0 = time.perf_counter()
    for q in range(seqs):
        for c0 in range(0, prompt, 128):
            c1 = min(prompt, c0 + 128)
            b.forward(np.full(c1 - c0, q, dtype=np.uint32), prompts[q, c0:c1], want_logits=c1 == prompt)
        if log_every and (q + 1) % log_every == 0:
            log(f"batch: prefilled {q + 1}/{seqs} sequences")
    prefill_s = time.perf_counter() - w0
    s1 = b.stats()
    samplers = [E.Sampler(1000 + first + q, 0.7, 0, 0.9, device=torch.cuda.current_device()) for q in range(seqs)]
    if world > 1:
        dist.barrier()
    w1 = time.perf_counter()
    ids = b.decode_sample(samplers, np.arange(seqs, dtype=np.uint32), gen)
    decode_s = time.perf_counter() - w1
    s2 = b.stats()
    kv = s2["kv_bytes"]
    b.close()
    pre_tok, dec_tok = seqs * prompt, seqs * gen
    pre_ms, dec_ms = s1["matvec_ms"] - s0["matvec_ms"], s2["matvec_ms"] - s1["matvec_ms"]
    return {"sequences": seqs, "prompt": prompt, "generated": gen, "ctx": CTX, "kv_bytes": kv,
            "prefill": {"tok_s": pre_tok / prefill_s, "device_tok_s": pre_tok / (pre_ms / 1e3), "seconds": prefill_s,
                        "calls": seqs * ((prompt + 127) // 128)},
            "decode": {"tok_s": dec_tok / decode_s, "device_tok_s": dec_tok / (dec_ms / 1e3), "seconds": decode_s,
                       "ms_per_step": dec_ms / gen, "distinct_ids_seq0": int(len(set(ids[:, 0].tolist())))},
            "sampling": "T 0.7, top-p 0.9, top-k off, sampler seed 1000 + sequence (device, exact f32 folds)"}


def batch_job_rates(res: dict, seqs: int, prompt: int, gen: int, slowest) -> dict:
    """A batched run over several ranks as one job: `res` is this rank's batch_study result (its own
    sequences), `slowest(values)` the element-wise maximum of `values` over the ranks (a collective:
    every rank calls it).  Rates are all `seqs` sequences' tokens over the slowest rank's wall and
    device times; the result describes the whole job."""
    pre_dev = res["sequences"] * res["prompt"] / res["prefill"]["device_tok_s"]  # this rank's device seconds
    pre_s, dec_s, pre_dev_s, dec_ms = slowest(
        [res["prefill"]["seconds"], res["decode"]["seconds"], pre_dev, res["decode"]["ms_per_step"]])
    pre_tok, dec_tok = seqs * prompt, seqs * gen
    out = dict(res, sequences=seqs, prefill=dict(res["prefill"]), decode=dict(res["decode"]))
    out["prefill"].update(tok_s=pre_tok / pre_s, device_tok_s=pre_tok / pre_dev_s, seconds=pre_s)
    out["decode"].update(tok_s=dec_tok / dec_s, device_tok_s=dec_tok / (dec_ms * gen / 1e3), seconds=dec_s,
                         ms_per_step=dec_ms)
    return out


def run_batch(args) -> None:
    """BASELINE config 5 (`--config 5`): the batched line; under torchrun with N > 1 ranks the
    BASELINE split: sequences data-parallel, experts sharded, dispatch / combine per layer between
    the ranks (qc_batch_ep_*).  Times: the slowest rank's (device and wall)."""
    import torch
    from qwen30brust_b200 import engine as E, tools as T
    rank = int(os.environ.get("RANK", 0))
    world = int(os.environ.get("WORLD_SIZE", 1))
    local = int(os.environ.get("LOCAL_RANK", 0))
    torch.cuda.set_device(local)
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600), device_id=torch.device("cuda", local))
        if args.seqs % world:
            raise SystemExit("--seqs must be a multiple of the rank count")
    spec = T.QWEN3_30B_A3B
    if args.layers:  # a shallower model of the same shapes: profiling runs only
        spec = spec.with_(layers=args.layers)
    img, path = synth_image(T, spec, rank, world)
    if world > 1:
        src = np.memmap(path, dtype=np.uint8, mode="r")
        eng = E.Engine.expert_parallel(src, CTX, local, rank, world)
        del src
    else:
        eng = E.Engine(img, CTX)
    sampler = ClockSampler(local)
    with sampler:
        res = batch_study(T, E, eng, spec, args.seqs, args.prompt, args.gen, log_every=8 if rank == 0 else 0,
                          rank=rank, world=world)
    eng.close()
    if world > 1:  # whole-job rates: all ranks' tokens over the slowest rank's times
        def slowest(v: list[float]) -> list[float]:
            t = torch.tensor(v, dtype=torch.float64, device="cuda")
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            return t.tolist()
        res = batch_job_rates(res, args.seqs, args.prompt, args.gen, slowest)
        res["expert_parallel"] = {"ranks": world, "experts_per_rank": spec.experts // world,
                                  "sequences_per_rank": args.seqs // world,
                                  "exchange": "per layer: every rank's normalized inputs and selections gathered "
                                              "(hidden x 4 B per token), expert outputs pulled by each token's rank "
                                              "(top x hidden x 4 B per token), two flag barriers"}
        dist.destroy_process_group()
        if rank != 0:
            return
    print(json.dumps({"metric": "batched decode tok/s (BASELINE config 5)", "value": res["decode"]["tok_s"],
                      "unit": "tok/s", "higher_is_better": True, "n_gpus": world, "dtype": "f32 activations; Q4_K/Q6_K "
                      "weights; projections and MoE on tcgen05 (exact K-quant integers x fp16 hi/lo activations, fp32 accumulate)",
                      "data": "synthetic: random-init N(0,0.02) weights quantized from seed 0; random prompts (seed 3)",
                      "config": {"workload": "BASELINE config 5: 64 sequences x 2048-token prompts, 512 "
                                 "sampled steps" if (args.seqs, args.prompt, args.gen) == (64, 2048, 512)
                                 else f"BASELINE config 5 shape, reduced: {args.seqs} sequences x {args.prompt}-token "
                                      f"prompts, {args.gen} sampled steps" + (
                                          f", {args.layers} layers (profiling run, not a bench line)" if args.layers
                                          else ""),
                                 "parallelism": f"expert parallel x{world} (sequences data-parallel)" if world > 1
                                 else "single GPU"},
                      **res, "clocks": sampler.summary()}), flush=True)


def run_matvec(args) -> None:
    """BASELINE config 2 alone (`--config 2`, optionally one `--shape`): the matvec study's JSON line."""
    import torch
    from qwen30brust_b200 import engine as E, tools as T
    torch.cuda.set_device(0)
    sampler = ClockSampler(0)
    with sampler:
        res = matvec_study(T, E, torch, args.steps, args.warmup, only=args.shape)
    print(json.dumps({"metric": "matvec HBM GB/s (BASELINE config 2)", "unit": "GB/s", "higher_is_better": True,
                      "steps": args.steps, "warmup": args.warmup, "dtype": "f32 x and y; GGML weights",
                      "data": "synthetic: W ~ N(0,0.02) quantized from seed 0, x ~ N(0,1)",
                      "config": {"workload": "BASELINE config 2: isolated matvecs at Qwen3-30B-A3B shapes"},
                      **res, "clocks": sampler.summary()}), flush=True)


def run_moe_layer(args) -> None:
    """BASELINE config 3 alone (`--config 3`): the MoE-layer study's JSON line."""
    from qwen30brust_b200 import engine as E, tools as T
    sampler = ClockSampler(0)
    with sampler:
        res = moe_study(T, E, args.steps, args.warmup)
    print(json.dumps({
        "metric": "MoE layer tokens/s (BASELINE config 3), per-token decode kernels vs tcgen05 grouped GEMMs",
        "unit": "tok/s", "higher_is_better": True, "steps": args.steps, "warmup": args.warmup,
        "dtype": "f32 activations; Q4_K gate/up, Q6_K down, F16 router; tensor path: exact K-quant integers x fp16 hi/lo activations, fp32 accumulate",
        "config": {"workload": "BASELINE config 3: one Qwen3-30B-A3B MoE layer", "experts": 128, "top": 8},
        **res, "clocks": sampler.summary()}), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=256)
    ap.add_argument("--warmup", type=int, default=8)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--cpu-tokens", type=int, default=4, help="tokens timed on all host threads for the CPU baseline")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-studies", action="store_true", help="skip the config 2 / config 3 objects of the main line")
    ap.add_argument("--layers", type=int, default=0,
                    help="profiling only: the same model with this many layers (0 = all 48, the benchmark)")
    ap.add_argument("--decode-mode", type=int, default=0, choices=[0, 1],
                    help="0: whole-token kernel when the model fits it (default); 1: per-phase kernels")
    ap.add_argument("--ref-max-steps", type=int, default=32)
    ap.add_argument("--config", type=int, default=4, choices=[2, 3, 4, 5],
                    help="2: matvec study; 3: MoE-layer study; 4: the decode bench (default); 5: batched sequences")
    ap.add_argument("--seqs", type=int, default=64, help="--config 5: sequences")
    ap.add_argument("--prompt", type=int, default=2048, help="--config 5: prompt tokens per sequence")
    ap.add_argument("--gen", type=int, default=512, help="--config 5: sampled steps")
    ap.add_argument("--shape", default=None, help="--config 2: one shape only (e.g. q_proj, vocab)")
    ap.add_argument("--replicas", action="store_true",
                    help="N > 1: N independent decode streams instead of one expert-parallel stream")
    args = ap.parse_args()
    if args.warmup < 3:
        ap.error("--warmup must be >= 3")
    if args.config == 2:
        run_matvec(args)
    elif args.config == 5:
        run_batch(args)
    elif args.config == 3:
        run_moe_layer(args)
    elif args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
