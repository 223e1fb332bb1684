"""Benchmark: GPT-2 124M data-parallel training throughput on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Workload (configuration 3 of the spec): GPT-2 124M (L=12, NH=12, C=768,
V=50257 padded to 50304, maxT=1024), B=16 sequences of T=1024 tokens per GPU,
bf16 GEMMs and attention with fp32 master weights and AdamW (lr 3e-4,
betas 0.9/0.999, eps 1e-8, wd 0), seeded initialisation, synthetic uniform
tokens seeded per rank (1337 + rank). One step = forward + backward (with
the per-layer NCCL gradient all-reduce when N > 1) + AdamW, all on the native
trainer of libllmk.so (include/llmk_gpt2.h), replayed as one captured CUDA
graph per step (llmk_gpt2_use_graph).

value: tokens/s of the whole job with tokens already resident in HBM,
timed with CUDA events on the trainer's stream over exactly K steps between
barriers, max over ranks. e2e: the same through llmk_gpt2_train_step from
pinned host tokens to a host loss every step. roofline: the tcgen05 GEMM
kernel over every GEMM of the step, timed live in the step (K further steps
with CUDA events around each library call of the trainer); kernels: the same
per kernel class with its share of the step and its fraction of the measured
tensor or HBM peak; gemm_alone_*: each GEMM shape timed alone.
cpu_baseline: the reference's own CPU training step (oracle/_ref, the
llm.cpp sources built by oracle/Makefile) on a bounded sample, rank 0 only.
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
sys.path.insert(0, os.path.join(ROOT, "llm.cpp_b200"))
sys.path.insert(0, ROOT)

CFG = dict(max_seq_len=1024, vocab_size=50257, padded_vocab_size=50304, num_layers=12, num_heads=12, channels=768)
B_PER_GPU, T = 16, 1024
LR = 3e-4
METRIC = "GPT-2 124M train tokens/sec (B=16/GPU, T=1024)"
# Reference CPU sample: training steps of the same model at B=1, T=256. Its
# attention backward is O(T^3) per head (gpt2/attention.cpp:104-113), so one
# step at T=1024 would take tens of minutes; T=256 steps take a few seconds
# each and overstate, not understate, the reference's throughput at T=1024.
REF_SAMPLE = dict(B=1, T=256)
# DRAM bytes (read + write) per gemm_tc_kernel launch of one training step:
# an ncu capture of every GEMM shape of the step at BT = 8192 gave 56.8 MB per
# launch on average; all shapes scale with BT, so 113.5 MB at BT = 16384
# (profiles/gemm_step_shapes_bt8192_dram.md).
GEMM_TRAFFIC_PER_LAUNCH = 113.5e6


def seeded_init_params(seed: int):
    """GPT-2 init of the spec (N(0,0.02), projections / sqrt(2L), biases 0, LN 1/0,
    padded vocab rows 0), drawn on the device with torch's generator. The
    bench only needs a valid initialisation of the architecture; parity runs
    use the oracle's generator (tests/)."""
    import torch
    L, C, Vp, V, maxT = CFG["num_layers"], CFG["channels"], CFG["padded_vocab_size"], CFG["vocab_size"], CFG["max_seq_len"]
    sizes = [Vp * C, maxT * C, L * C, L * C, L * 3 * C * C, L * 3 * C, L * C * C, L * C, L * C, L * C, L * 4 * C * C,
             L * 4 * C, L * 4 * C * C, L * C, C, C]
    g = torch.Generator(device="cuda").manual_seed(seed)
    parts = []
    for i, n in enumerate(sizes):
        if i in (0, 1, 4, 6, 10, 12):
            sd = 0.02 / (2 * L) ** 0.5 if i in (6, 12) else 0.02
            t = torch.randn(n, generator=g, device="cuda") * sd
            if i == 0:
                t.view(Vp, C)[V:] = 0
        elif i in (2, 8, 14):
            t = torch.ones(n, device="cuda")
        else:
            t = torch.zeros(n, device="cuda")
        parts.append(t)
    return torch.cat(parts).cpu().numpy()


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled during the timed region."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.idx = gpu_index
        self.f = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        self.p = None

    def start(self):
        try:
            self.p = subprocess.Popen(["nvidia-smi", "-i", str(self.idx), f"--query-gpu={self.Q}",
                                       "--format=csv,noheader,nounits", "-lms", "200"], stdout=self.f,
                                      stderr=subprocess.DEVNULL)
        except Exception:
            self.p = None
            return
        # nvidia-smi takes a moment to start: begin timing once it is sampling
        t0 = time.time()
        while time.time() - t0 < 3.0 and self.p.poll() is None:
            if os.path.getsize(self.f.name) > 0:
                break
            time.sleep(0.02)

    def stop(self) -> dict:
        if self.p is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.p.terminate()
        try:
            self.p.wait(timeout=5)
        except Exception:
            self.p.kill()
        self.f.flush()
        self.f.seek(0)
        sm, smax, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.f.read().strip().splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                smax = float(f[2])
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        os.unlink(self.f.name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": smax, "reasons": sorted(reasons),
                "samples": len(sm)}


def measured_peaks() -> dict:
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return {"bf16_tflops": d["bf16_tflops"], "bf16_tflops_sustained": d.get("bf16_tflops_sustained"),
                "hbm_gbs": d["hbm_gbs"], "source": "measured"}
    return {"bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "hbm_gbs": 6650.0, "source": "fallback"}


def gemm_roofline(llmk, torch, BT: int, reps: int = 5) -> dict:
    """Times the tcgen05 GEMM alone on every GEMM shape of one training step
    (fwd / dinp / dweight of QKV, attproj, FC, FCproj and the tied lm_head at
    BT tokens) with CUDA events on the launching stream."""
    C, Vp = CFG["channels"], CFG["padded_vocab_size"]
    dev = "cuda"
    shapes = []  # (name, M, N, K, a_trans, b_trans, count per step)
    L = CFG["num_layers"]
    for name, IC, OC in [("qkv", C, 3 * C), ("attproj", C, C), ("fc", C, 4 * C), ("fcproj", 4 * C, C)]:
        shapes += [(f"{name}.fwd", BT, OC, IC, 0, 0, L), (f"{name}.dinp", BT, IC, OC, 0, 1, L),
                   (f"{name}.dweight", OC, IC, BT, 1, 1, L)]
    shapes += [("lm_head.fwd", BT, Vp, C, 0, 0, 1), ("lm_head.dinp", BT, C, Vp, 0, 1, 1),
               ("lm_head.dweight", Vp, C, BT, 1, 1, 1)]
    s = torch.cuda.current_stream()
    per = {}
    tot_flop = tot_ms = 0.0
    for name, M, N, K, at, bt, cnt in shapes:
        A = torch.randn((K, M) if at else (M, K), device=dev).bfloat16()
        B = torch.randn((K, N) if bt else (N, K), device=dev).bfloat16()
        D = torch.empty(M, N, device=dev, dtype=torch.float32 if "dweight" in name else torch.bfloat16)
        wsb = llmk.lib().llmk_gemm_workspace(M, N, K, llmk.MATH_BF16)
        ws = torch.empty(max(wsb // 4, 1), device=dev)
        for _ in range(2):
            llmk.gemm(D, A, B, a_trans=at, b_trans=bt, M=M, N=N, K=K, workspace=ws)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        e0.record(s)
        for _ in range(reps):
            llmk.gemm(D, A, B, a_trans=at, b_trans=bt, M=M, N=N, K=K, workspace=ws)
        e1.record(s)
        e1.synchronize()
        ms = e0.elapsed_time(e1) / reps
        flop = 2.0 * M * N * K
        per[name] = {"tflops": round(flop / ms / 1e9, 1), "ms": round(ms, 4)}
        tot_flop += flop * cnt
        tot_ms += ms * cnt
        del A, B, D, ws
    return {"per_gemm": per, "step_gemm_tflop": tot_flop / 1e12, "step_gemm_ms": tot_ms,
            "achieved_tflops": tot_flop / tot_ms / 1e9}


def reference_step_time(threads: int, steps: int = 3) -> dict:
    """The reference's own CPU training step (oracle/_ref/libref.so) on the
    REF_SAMPLE batch: `steps` steps of one model; median tokens/s."""
    import numpy as np
    import oracle as O
    if not O.ref_available():
        return {"unavailable": "oracle/_ref/libref.so not built (make -C oracle ref needs the reference tree)"}
    os.environ["OMP_NUM_THREADS"] = str(threads)
    cfg = O.config()
    params = O.init_params(cfg, 1337)
    Bs, Ts = REF_SAMPLE["B"], REF_SAMPLE["T"]
    toks = O.tokens(Bs * Ts + 1, cfg.vocab_size, 1337)
    with tempfile.TemporaryDirectory() as d:
        ck = os.path.join(d, "gpt2_124m.bin")
        O.write_checkpoint(ck, cfg, params)
        losses = np.zeros(steps, np.float32)
        ms = np.zeros(steps, np.float64)
        # the reference prints its model config on stdout: keep stdout for the JSON line
        sys.stdout.flush()
        saved = os.dup(1)
        os.dup2(2, 1)
        try:
            O.ref().ref_gpt2_train(ck.encode(), Bs, Ts, toks[:-1].copy(), toks[1:].copy(), steps, LR, losses, ms)
        finally:
            os.dup2(saved, 1)
            os.close(saved)
    per_step = [Bs * Ts / (x / 1e3) for x in ms]
    return {"value": statistics.median(per_step), "per_step": per_step, "step_s": statistics.median(ms) / 1e3,
            "sample": f"{steps} reference training steps of GPT-2 124M at B={Bs}, T={Ts} ({Bs * Ts} tokens each), "
                      f"median"}


def run_reference(args) -> None:
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    threads = os.cpu_count() or 1
    r = reference_step_time(threads, steps=args.warmup + args.steps)
    if "unavailable" in r:
        print(json.dumps({"impl": "reference", "unavailable": r["unavailable"]}))
        return
    v = statistics.median(r["per_step"][args.warmup:])
    line = {"metric": METRIC, "value": v, "unit": "tokens/s", "n_gpus": args.gpus, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": REF_SAMPLE["B"] * REF_SAMPLE["T"] / v * 1e3,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "impl": "reference",
            "config": {"workload": "gpt2-124M train step (config 3), reference CPU sample", "model": "gpt2-124M",
                       "global_batch": REF_SAMPLE["B"], "seq_len": REF_SAMPLE["T"], "parallelism": "cpu"},
            "cpu_baseline": {"value": v, "unit": "tokens/s", "cores": threads, "kind": "reference",
                             "sample": r["sample"]},
            "e2e": {"value": v, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line))


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=30)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    args = ap.parse_args()
    if args.impl == "reference":
        run_reference(args)
        return

    import numpy as np
    import torch
    import torch.distributed as dist
    import datetime
    import llmk

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", local))
    model = llmk.GPT2(B_PER_GPU, T, **CFG)
    params = seeded_init_params(1337)
    model.load_parameters(params)
    if world > 1:
        obj = [llmk.nccl_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(obj, src=0)
        model.enable_dp(obj[0], rank, world)
        model.broadcast_parameters(0)
    BT = B_PER_GPU * T
    rng = np.random.default_rng(1337 + rank)
    toks = rng.integers(0, CFG["vocab_size"], size=BT + 1, dtype=np.int32)
    inp_h, tgt_h = toks[:-1].copy(), toks[1:].copy()
    model.train_step(inp_h, tgt_h, 0.0, t=1, want_loss=False)  # tokens now resident in the model's buffers
    d_in, d_tg = model.buffers()
    # every later step replays one captured CUDA graph of forward + backward + AdamW
    model.use_graph(True)
    stream = torch.cuda.ExternalStream(model.stream)

    def barrier():
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()

    t = 1
    for _ in range(args.warmup):
        model.step_device(d_in, d_tg, LR, t)
        t += 1
    barrier()
    sampler = ClockSampler(local)
    sampler.start()
    n0 = llmk.lib().llmk_launch_count()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        model.step_device(d_in, d_tg, LR, t)
        t += 1
    e1.record(stream)
    model.synchronize(timeout_ms=600000)
    launches = llmk.lib().llmk_launch_count() - n0
    ms = e0.elapsed_time(e1) / args.steps
    clocks = sampler.stop()
    # per-kernel-class device time inside the training step: the same K steps
    # again, with CUDA events on the trainer stream around every library call
    # (kept out of the timed region above; the events add a little device time)
    model.set_timing(True)
    ei0, ei1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ei0.record(stream)
    for _ in range(args.steps):
        model.step_device(d_in, d_tg, LR, t)
        t += 1
    ei1.record(stream)
    ei1.synchronize()
    timed_ms = ei0.elapsed_time(ei1) / args.steps
    classes = model.timing_report()
    model.set_timing(False)
    # e2e: host tokens in, host loss out, every step
    barrier()
    w0 = time.perf_counter()
    e2e_steps = max(3, args.steps // 2)
    ee0, ee1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ee0.record(stream)
    last_loss = None
    for _ in range(e2e_steps):
        last_loss = model.train_step(inp_h, tgt_h, LR, t)
        t += 1
    ee1.record(stream)
    ee1.synchronize()
    e2e_ms = ee0.elapsed_time(ee1) / e2e_steps
    e2e_wall_ms = (time.perf_counter() - w0) * 1e3 / e2e_steps
    e2e_ms = max(e2e_ms, e2e_wall_ms)
    if world > 1:
        v = torch.tensor([ms, e2e_ms], device="cuda")
        dist.all_reduce(v, op=dist.ReduceOp.MAX)
        ms, e2e_ms = v.tolist()
    tokens_per_step = BT * world
    value = tokens_per_step / (ms / 1e3)
    e2e_value = tokens_per_step / (e2e_ms / 1e3)

    line = None
    if rank == 0:
        peaks = measured_peaks()
        # the burst GEMM peak while the step ran at the maximum SM clock, the
        # sustained one when the power cap held the clock down
        capped = "sw_power_cap" in (clocks.get("reasons") or []) or (
            clocks.get("sm_mhz") and clocks.get("sm_max_mhz") and clocks["sm_mhz"] < 0.97 * clocks["sm_max_mhz"])
        if capped and peaks.get("bf16_tflops_sustained"):
            tpeak, tsrc = peaks["bf16_tflops_sustained"], " bf16 sustained (the step ran under the power cap)"
        else:
            tpeak, tsrc = peaks["bf16_tflops"], " bf16 burst (the step ran at the maximum SM clock)"
        roof = gemm_roofline(llmk, torch, BT)
        kernels = {}
        for name, c in classes.items():
            if c["calls"] == 0:
                continue
            tensor = c["unit"] == "flop"
            rate = c["work"] / (c["ms"] * 1e-3) / (1e12 if tensor else 1e9) if c["ms"] > 0 else 0.0
            peak = tpeak if tensor else peaks["hbm_gbs"]
            kernels[name] = {"ms_per_step": round(c["ms"] / args.steps, 4),
                             "share": round(c["ms"] / args.steps / timed_ms, 4),
                             "launches_per_step": c["launches"] // args.steps,
                             "achieved": round(rate, 1), "unit": "TFLOP/s" if tensor else "GB/s",
                             "frac": round(rate / peak, 4)}
        gemm_cls = [c for n, c in classes.items() if n.startswith("gemm")]
        g = {k: sum(c[k] for c in gemm_cls) for k in ("ms", "work", "launches", "calls")}
        gemm_launches = max(g["launches"], 1)
        achieved = g["work"] / (g["ms"] * 1e-3) / 1e12
        line = {
            "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded uniform tokens, seeded init)",
            "config": {"workload": "gpt2-124M train step (config 3)", "model": "gpt2-124M",
                       "global_batch": B_PER_GPU * world, "seq_len": T, "parallelism": f"dp{world}",
                       "l2": "working set larger than L2 (about 7 GB of activations per step)"},
            "e2e": {"value": e2e_value, "unit": "tokens/s", "h2d_bytes_per_step": 2 * BT * 4,
                    "d2h_bytes_per_step": 4},
            "gpu_launches": int(launches),
            "loss": last_loss,
            "roofline": {"kernel": "gemm_tc_kernel (every GEMM of the step, timed live in the step)",
                         "bound": "tensor", "achieved": round(achieved, 1), "peak": tpeak,
                         "unit": "TFLOP/s", "frac": round(achieved / tpeak, 4),
                         "traffic": GEMM_TRAFFIC_PER_LAUNCH,
                         "flop_per_launch": g["work"] / gemm_launches,
                         "launch_ms": g["ms"] / gemm_launches,
                         "peak_source": peaks["source"] + tsrc},
            "kernels": kernels,
            "gemm_ms_per_step": round(g["ms"] / args.steps, 3),
            "instrumented_ms_per_step": round(timed_ms, 3),
            "gemm_alone_tflops": roof["per_gemm"],
            "gemm_alone_step_ms": round(roof["step_gemm_ms"], 3),
            "gemm_alone_tflops_avg": round(roof["achieved_tflops"], 1),
            "clocks": clocks,
        }
        if not args.no_cpu_baseline:
            cb = reference_step_time(os.cpu_count() or 1)
            if "unavailable" in cb:
                line["cpu_baseline"] = {"value": None, "unavailable": cb["unavailable"]}
            else:
                line["cpu_baseline"] = {"value": cb["value"], "unit": "tokens/s", "cores": os.cpu_count(),
                                        "kind": "reference", "sample": cb["sample"]}
        print(json.dumps(line), flush=True)
    model.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
