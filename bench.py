#!/usr/bin/env python3
"""Decode benchmark: Qwen3-30B-A3B-shape Q4_K_M model, batch 1, ctx 4096.

A step is one greedy decode token (the whole forward: 48 layers + vocab
projection + argmax) on the device.  Inputs: a random-init synthetic model
(N(0, 0.02) weights quantized by libqwen_tools, seed 0) and a 512-token random
prompt (seed 1) prefilled before timing; weights per step (~2 GB) exceed the
126 MB L2, so no flush is needed between steps.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Prints one JSON line on rank 0.  `value` is device-resident decode tok/s over
all ranks; `e2e` is tok/s through qc_forward with the token copied in and the
logits copied out (pinned host memory) every step, and the host picking the
argmax, as the reference's chat loop does.  `--impl reference` times the
reference's CPU path (the C++ restatement under oracle/, all host threads) on
the same model.  With N > 1 each rank runs an independent replica by default
(scaling "weak"); with --ep the N ranks run ONE decode stream with the experts
split over them (expert parallelism: each rank holds experts/N, partial MoE
vectors exchanged over NVLink inside the token kernel), scaling "strong", and
`value` is that stream's tok/s.
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


# DRAM bytes of one k_token launch from the ncu capture in profiles/k_token_4layer.md (4 layers):
# 414.3 MB = 255.9 MB (vocab projection, logits) + 4 x 39.6 MB per layer; scaled by layer count.
TOKEN_TRAFFIC_FIXED, TOKEN_TRAFFIC_PER_LAYER = 255.9e6, 39.6e6


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
    """The reference's CPU path (oracle restatement, row-parallel over `threads`) on `tokens`."""
    from oracle import oracle as O
    if not O.LIB_PATH.exists():
        O.build()
    m = O.Model(img, CTX, threads=threads)
    m.forward(tokens[0])  # first token outside the timing (page-in of the 20 GB image)
    t0 = time.perf_counter()
    for t in tokens[1:]:
        m.forward(t)
    dt = time.perf_counter() - t0
    m.close()
    return {"tok_s": (len(tokens) - 1) / dt, "seconds": dt, "tokens": len(tokens) - 1}


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
    ep = world > 1 and args.ep
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
    eng.close()

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
        if not args.no_cpu_baseline:
            ncores = cpu_cores()
            toks = [int(x) for x in prompt[:args.cpu_tokens + 1]]
            src = img if img is not None else np.fromfile(path, dtype=np.uint8)
            c = cpu_decode(src, toks, ncores)
            cpu = {"value": c["tok_s"], "unit": "tok/s", "cores": ncores, "kind": "port",
                   "sample": f"{c['tokens']} decode tokens at positions 1..{c['tokens']} of the same 30B-shape model "
                             f"(C++ restatement of backend.rs Cpu::matvec + ops.rs + model.rs, row-parallel over "
                             f"{ncores} threads, bit-identical to 1 thread; {cpu_model()}); {c['seconds']:.1f} s"}
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
    """The reference's own CPU path (its C++ restatement, all host threads), same metric and config."""
    rank = int(os.environ.get("RANK", 0))
    if rank != 0:
        return
    from qwen30brust_b200 import tools as T
    spec = T.QWEN3_30B_A3B
    img = T.synth_gguf(spec)
    ncores = cpu_cores()
    # bounded: each step is one full token of the 30B model on the CPU; cap the timed steps
    steps = max(1, min(args.steps, args.ref_max_steps))
    prompt = np.random.default_rng(1).integers(0, spec.vocab, steps + args.warmup + 1).tolist()
    from oracle import oracle as O
    if not O.LIB_PATH.exists():
        O.build()
    m = O.Model(img, CTX, threads=ncores)
    for t in prompt[:args.warmup + 1]:
        m.forward(int(t))
    t0 = time.perf_counter()
    for t in prompt[args.warmup + 1:]:
        m.forward(int(t))
    dt = time.perf_counter() - t0
    value = steps / dt
    sample = (f"{steps} decode tokens (positions {args.warmup + 1}..{args.warmup + steps}) of the 30B-shape model; "
              f"C++ restatement of the reference CPU path, row-parallel over {ncores} threads; {cpu_model()}")
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": 0, "steps": steps,
        "warmup": args.warmup, "ms_per_step": dt / steps * 1e3, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32",
        "data": "synthetic: random-init N(0,0.02) weights quantized from seed 0",
        "config": {"workload": "BASELINE config 4: Qwen3-30B-A3B-shape decode, batch 1, greedy", "ctx": CTX},
        "cpu_baseline": {"value": value, "unit": "tok/s", "cores": ncores, "kind": "port", "sample": sample},
        "e2e": {"value": value, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)


def run_moe_layer(args) -> None:
    """one Qwen3-30B-A3B MoE layer for T in {1, 8, 32, 128} tokens, per-token
    decode kernels (path 1, matvecs) against tcgen05 grouped GEMMs (path 2); Zipf-skewed router."""
    import torch
    from qwen30brust_b200 import engine as E, tools as T
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
    sampler = ClockSampler(0)
    rows, load = [], np.zeros(NE, dtype=np.int64)
    with sampler:
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
                for _ in range(args.warmup):
                    eng.moe_layer(0, x, path)
                ms = sorted(eng.moe_layer(0, x, path)[1] for _ in range(args.steps))
                med = ms[len(ms) // 2]
                res[f"path{path}"] = {"ms": med, "tok_s": tokens / (med / 1e3), "gbs": byts / (med / 1e3) / 1e9,
                                      "tflops": flops / (med / 1e3) / 1e12}
            res["bytes"], res["flops"] = byts, flops
            res["speedup_tc"] = res["path1"]["ms"] / res["path2"]["ms"]
            rows.append(res)
            log(f"T={tokens}: distinct {distinct}, per-token kernels {res['path1']['ms']:.3f} ms, "
                f"tensor cores {res['path2']['ms']:.3f} ms")
    cross = next((r["tokens_per_expert"] for r in rows if r["speedup_tc"] > 1.0), None)
    ranked = np.sort(load)[::-1]
    top_share = ranked[: max(1, NE // 16)].sum() / max(1, ranked.sum())
    out = {
        "metric": "MoE layer tokens/s (BASELINE config 3), per-token decode kernels vs tcgen05 grouped GEMMs",
        "unit": "tok/s", "higher_is_better": True, "steps": args.steps, "warmup": args.warmup,
        "dtype": "f32 activations; Q4_K gate/up, Q6_K down, F16 router; tensor path fp16 hi/lo split, fp32 accumulate",
        "data": "synthetic: N(0,0.02) weights (seed 0), router row e scaled by (e+1)^-1.1, hidden N(0,1) (seed 7)",
        "config": {"workload": "BASELINE config 3: one Qwen3-30B-A3B MoE layer", "hidden": H, "experts": NE,
                   "top": top, "intermediate": I, "timing": "device time of qc_moe_layer, median of steps"},
        "results": rows,
        "crossover_tokens_per_expert": cross,
        "load_share_top_8_experts": float(top_share),
        "clocks": sampler.summary(),
    }
    print(json.dumps(out), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=256)
    ap.add_argument("--warmup", type=int, default=8)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--cpu-tokens", type=int, default=2, help="tokens timed for the CPU baseline line")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--layers", type=int, default=0,
                    help="profiling only: the same model with this many layers (0 = all 48, the benchmark)")
    ap.add_argument("--decode-mode", type=int, default=0, choices=[0, 1],
                    help="0: whole-token kernel when the model fits it (default); 1: per-phase kernels")
    ap.add_argument("--ref-max-steps", type=int, default=8)
    ap.add_argument("--config", type=int, default=4, choices=[3, 4],
                    help="3: the MoE-layer study (per-token kernels vs tensor cores); 4: the decode bench")
    ap.add_argument("--ep", action="store_true",
                    help="N > 1: one decode stream with the experts split over the ranks (expert parallelism)")
    args = ap.parse_args()
    if args.warmup < 3:
        ap.error("--warmup must be >= 3")
    if args.config == 3:
        run_moe_layer(args)
    elif args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
