"""Throughput of the block-quantized decode path on B200.

Workload (the decode-bound Whisper-tiny configuration): 4 pre-LN decoder
blocks, d=384, 6 heads, FFN 1536, Q8_0 linears, tied Q4_0 readout 51865x384,
self-attention KV cache and cross-attention over seeded encoder states
[1,1500,384] ~ N(0,1); 4 prompt tokens per sequence, then greedy decode at
batch 32. One step = one greedy decode step of all 32 sequences through the
whole layer stack and readout (32 tokens). Weights are seeded synthetic
(N(0,0.02), fp16 pre-round, Q8_0/Q4_0); token ids uniform.

L2 policy: 8 independent weight replicas (8 x 20 MB > 126 MB L2) rotate
step by step, so every step streams its weights from HBM.

--impl reference times the reference's own CPU arithmetic for the same step
(the vendored ggml x86 quantizer + vec_dot kernels compiled from the
reference sources into oracle/_ref, driven row-parallel over every host core)
on a bounded number of steps.
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
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

BATCH = 32
PROMPT = 4
REPLICAS = 8
METRIC = "tokens/s per layer stack (Whisper-tiny decoder, Q8_0 body + Q4_0 readout, greedy decode)"
CONFIG = {"workload": "whisper-tiny decoder decode step: 4 layers d384 h6 ffn1536, Q8_0 linears, "
                      "Q4_0 tied readout 51865x384, cross-attention over [1,1500,384]",
          "batch": BATCH, "prompt_tokens": PROMPT, "l2": f"{REPLICAS} rotating weight replicas (> L2)"}


def env_rank():
    return int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1)), int(os.environ.get("LOCAL_RANK", 0))


# ----------------------------------------------------------------------------- clocks
class ClockSampler:
    """SM clock and clock-event reasons sampled while the timed region runs.

    NVML (nvidia-ml-py) is read in-process every ~0.5 ms from a thread and, while
    the host waits for the timed work to finish, from the waiting thread, so even
    a timed region of a few milliseconds gets samples; the GPU is matched by UUID
    (CUDA_VISIBLE_DEVICES-safe). Without NVML, nvidia-smi at its 200 ms period."""

    FIELDS = "index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active," \
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown," \
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap"
    REASONS = (("hw_slowdown", "nvmlClocksEventReasonHwSlowdown", 0x8),
               ("hw_thermal_slowdown", "nvmlClocksEventReasonHwThermalSlowdown", 0x40),
               ("sw_thermal_slowdown", "nvmlClocksEventReasonSwThermalSlowdown", 0x20),
               ("sw_power_cap", "nvmlClocksEventReasonSwPowerCap", 0x4))

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.lines = []
        self.samples = []          # (sm MHz, max sm MHz, reason bits) from NVML
        self.nvml = self.handle = None
        self.stop = threading.Event()
        self.thread = None
        try:
            import pynvml
            import torch
            pynvml.nvmlInit()
            try:
                uuid = str(torch.cuda.get_device_properties(gpu_index).uuid)
                self.handle = pynvml.nvmlDeviceGetHandleByUUID(uuid if uuid.startswith("GPU-") else "GPU-" + uuid)
            except Exception:
                self.handle = pynvml.nvmlDeviceGetHandleByIndex(gpu_index)
            self.nvml = pynvml
            self.max_sm = float(pynvml.nvmlDeviceGetMaxClockInfo(self.handle, pynvml.NVML_CLOCK_SM))
        except Exception:
            self.nvml = self.handle = None

    def _sample(self):
        n = self.nvml
        sm = float(n.nvmlDeviceGetClockInfo(self.handle, n.NVML_CLOCK_SM))
        self.samples.append((sm, self.max_sm, int(n.nvmlDeviceGetCurrentClocksEventReasons(self.handle))))

    def _poll(self):
        while not self.stop.is_set():
            try:
                self._sample()
            except Exception:
                return
            time.sleep(0.0005)

    def __enter__(self):
        if self.nvml is not None:
            self.thread = threading.Thread(target=self._poll, daemon=True)
            self.thread.start()
            return self
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            threading.Thread(target=self._read, daemon=True).start()
        except OSError:
            self.proc = None
        return self

    def wait(self, event) -> None:
        """Sample on the calling thread until the GPU reaches ``event`` (the end of the timed
        work): the launching thread would otherwise hold the interpreter lock for most of a
        short region, starving the polling thread."""
        if self.nvml is None:
            return
        while not event.query():
            try:
                self._sample()
            except Exception:
                return
            time.sleep(0.0002)

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        if self.thread is not None:
            self.stop.set()
            self.thread.join(timeout=5)
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        sm, mx, reasons = [], [], set()
        if self.samples:
            for clock, top, bits in self.samples:
                sm.append(clock)
                mx.append(top)
                for name, const, value in self.REASONS:
                    if bits & int(getattr(self.nvml, const, value)):
                        reasons.add(name)
            source = "nvml"
        else:
            source = "nvidia-smi"
        names = [r[0] for r in self.REASONS]
        for line in self.lines:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx.append(float(parts[2]))
            except ValueError:
                continue
            for name, flag in zip(names, parts[5:9]):
                if flag.lower() == "active":
                    reasons.add(name)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0, "source": None}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(mx), "reasons": sorted(reasons),
                "samples": len(sm), "source": source}


# ----------------------------------------------------------------------------- peaks
def measured_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return d.get("hbm_gbs", 6650.0), "measured"
    return 6650.0, "fallback"


def committed_traffic():
    """Per-launch DRAM bytes (read + write) of the readout kernel from the committed ncu summary."""
    p = ROOT / "profiles" / "readout_q4_vocab51865_b32.md"
    if not p.exists():
        return None
    for line in p.read_text().splitlines():
        if line.startswith("traffic_bytes_per_launch:"):
            try:
                return int(line.split(":")[1].strip())
            except ValueError:
                return None
    return None


# ----------------------------------------------------------------------------- cpu arm
def cpu_reference_step_rate(seconds: float = 10.0, max_steps: int = 200, warmup: int = 1):
    """The reference's CPU arithmetic for one decode step's linears at batch 32:
    vendored ggml x86 quantize_row_q8_0 + vec_dot (oracle/_ref), all host threads.
    Returns (steps/s, steps timed, cores)."""
    import numpy as np
    from oracle import oracle as O
    if O.ref_lib() is None:
        O.build()
    cores = O.cpu_cores()
    rng = np.random.default_rng(1)
    d, f, V = 384, 1536, 51865
    mats = []
    for _ in range(4):
        mats += [(O.pack_weights((rng.standard_normal((3 * d, d)) * 0.02).astype(np.float32)), "q8_0", d)]
        mats += [(O.pack_weights((rng.standard_normal((d, d)) * 0.02).astype(np.float32)), "q8_0", d)] * 3
        mats += [(O.pack_weights((rng.standard_normal((f, d)) * 0.02).astype(np.float32)), "q8_0", d)]
        mats += [(O.pack_weights((rng.standard_normal((d, f)) * 0.02).astype(np.float32)), "q8_0", f)]
    head = O.pack_weights((rng.standard_normal((V, d)) * 0.02).astype(np.float32), "q4_0")
    xs = {k: rng.standard_normal((BATCH, k)).astype(np.float32) for k in (d, f)}

    def step():
        for blocks, fmt, k in mats:
            O.ref_mul_mat(blocks, xs[k], fmt, threads=cores)
        O.ref_mul_mat(head, xs[d], "q4_0", threads=cores)

    for _ in range(max(1, warmup)):  # untimed warm-up steps
        step()
    t0 = time.perf_counter()
    n = 0
    while n < max_steps and time.perf_counter() - t0 < seconds:
        step()
        n += 1
    dt = time.perf_counter() - t0
    return n / dt, n, cores


def run_reference(args):
    rank, world, _ = env_rank()
    if rank != 0:
        return 0
    rate, n, cores = cpu_reference_step_rate(seconds=min(60.0, 2.0 + 0.5 * args.steps),
                                             max_steps=max(args.steps, 1), warmup=args.warmup)
    value = rate * BATCH
    line = {"metric": METRIC, "value": round(value, 2), "unit": "tokens/s", "n_gpus": args.gpus,
            "steps": n, "warmup": args.warmup, "ms_per_step": round(1e3 / rate, 3), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "q8_0/q4_0 x q8_0 -> f32", "data": "synthetic",
            "config": CONFIG, "impl": "reference",
            "cpu_baseline": {"value": round(value, 2), "unit": "tokens/s", "cores": cores, "kind": "reference",
                             "sample": f"{n} decode steps of the 33 block-quantized linears (batch 32) through "
                                       "the vendored ggml x86 kernels; attention/LayerNorm excluded"},
            "e2e": {"value": round(value, 2), "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)
    return 0


# ----------------------------------------------------------------------------- b200 arm
def run_b200(args):
    import torch
    import torch.distributed as dist
    from mstar_accelerators_b200 import native
    from mstar_accelerators_b200.linear import BlockLinear
    from mstar_accelerators_b200.whisper import GraphDecoder, WhisperConfig, WhisperDecoderB200, synthetic_weights

    rank, world, local = env_rank()
    torch.cuda.set_device(local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=torch.device("cuda", local))
    native.require_capability()
    cfg = WhisperConfig()
    weights = synthetic_weights(cfg, seed=1, device="cuda")
    g = torch.Generator().manual_seed(2)
    enc = torch.randn((1, cfg.source, cfg.d_model), generator=g).cuda()
    g3 = torch.Generator().manual_seed(3 + rank)
    prompt = torch.randint(0, cfg.vocab, (BATCH, PROMPT), generator=g3).cuda()

    decs, graphs = [], []
    for r in range(REPLICAS):
        dec = WhisperDecoderB200(weights, cfg, batch=BATCH)
        _, tok = dec.prefill(prompt, enc)
        gd = GraphDecoder(dec)
        gd.tokens.copy_(tok)
        gd.positions.fill_(PROMPT)
        gd.capture()
        decs.append(dec)
        graphs.append(gd)
    torch.cuda.synchronize()

    # positions must stay inside the 448-token self-attention capacity
    max_steps = cfg.target - PROMPT - 1

    def reset():
        for gd in graphs:
            gd.positions.fill_(PROMPT)

    def run_steps(k):
        for i in range(k):
            graphs[i % REPLICAS].graph.replay()

    per_replica = (args.warmup + args.steps + REPLICAS - 1) // REPLICAS + 1
    if per_replica > max_steps:
        raise SystemExit(f"--steps/--warmup exceed the {max_steps}-step context per replica")
    reset()
    run_steps(args.warmup)
    stream = torch.cuda.current_stream()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    with ClockSampler(local) as clocks:
        start.record(stream)
        run_steps(args.steps)
        end.record(stream)
        clocks.wait(end)
        torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    ms = start.elapsed_time(end)
    t = torch.tensor([ms], device="cuda")
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_max = float(t.item())
    value = BATCH * args.steps * world / (ms_max / 1e3)

    # e2e through the public step API with host buffers: H2D tokens, replay, D2H next tokens
    reset()
    host_in = torch.zeros(BATCH, dtype=torch.int64).pin_memory()
    host_out = torch.zeros(BATCH, dtype=torch.int64).pin_memory()
    for gd in graphs:
        host_in.copy_(gd.tokens.cpu())
    e2e_steps = args.steps
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    e_start, e_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e_start.record(stream)
    for i in range(e2e_steps):
        gd = graphs[i % REPLICAS]
        gd.tokens.copy_(host_in, non_blocking=True)
        gd.graph.replay()
        host_out.copy_(gd.tokens, non_blocking=True)
        stream.synchronize()
        host_in.copy_(host_out)
    e_end.record(stream)
    torch.cuda.synchronize()
    e2e_ms = torch.tensor([e_start.elapsed_time(e_end)], device="cuda")
    if world > 1:
        dist.all_reduce(e2e_ms, op=dist.ReduceOp.MAX)
    e2e_value = BATCH * e2e_steps * world / (float(e2e_ms.item()) / 1e3)

    # roofline of the dominant kernel: the Q4_0 vocab readout (one launch: query quantization,
    # tile GEMV, suppression, argmax), timed alone with events over rotating replicas
    # tile weights of 16 heads (180 MB) rotate through the 126 MB L2
    heads = [d.head for d in decs]
    heads += [BlockLinear(blocks=h.blocks, fmt=h.fmt, rows=h.rows, width=h.width) for h in heads]
    for h in heads:
        h.prepare_readout()
    x = torch.randn((BATCH, cfg.d_model), device="cuda")
    lg = torch.empty((BATCH, cfg.vocab), device="cuda")
    tk = torch.empty(BATCH, dtype=torch.int64, device="cuda")
    st = torch.zeros(1, dtype=torch.int32, device="cuda")
    cap_stream = torch.cuda.Stream()
    cap_stream.wait_stream(stream)
    with torch.cuda.stream(cap_stream):
        for h in heads:
            h.readout(x, logits=lg, token=tk, status=st)
    stream.wait_stream(cap_stream)
    rg = torch.cuda.CUDAGraph()
    with torch.cuda.graph(rg, stream=cap_stream):
        for i in range(2 * len(heads)):
            heads[i % len(heads)].readout(x, logits=lg, token=tk, status=st)
    for _ in range(3):
        rg.replay()
    r0, r1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    reps = max(5, args.steps // 4)
    r0.record(stream)
    for _ in range(reps):
        rg.replay()
    r1.record(stream)
    torch.cuda.synchronize()
    launch_s = r0.elapsed_time(r1) / 1e3 / (reps * 2 * len(heads))
    weight_bytes = cfg.vocab * (cfg.d_model // 32) * 18
    alg_bytes = weight_bytes + BATCH * cfg.d_model * 4 + BATCH * cfg.vocab * 4
    peak, peak_kind = measured_peaks()
    achieved = alg_bytes / launch_s / 1e9

    line = None
    if rank == 0:
        cpu = None
        if world == 1:
            rate, n, cores = cpu_reference_step_rate(seconds=10.0, max_steps=50, warmup=3)
            cpu = {"value": round(rate * BATCH, 2), "unit": "tokens/s", "cores": cores, "kind": "reference",
                   "sample": f"{n} decode steps of the 33 block-quantized linears (batch 32) through the "
                             "vendored ggml x86 kernels on the host cores; attention/LayerNorm excluded"}
        clk = clocks.summary()
        # embedding; per layer: qkv, cq (quantize + GEMV), fc1 (quantize + GEMV writing fc2's fragments),
        # out, cout, fc2 (GEMV on fragments written by their producer), self attention (1), cross attention
        # (one cluster launch); readout (one launch)
        launches_per_step = 1 + cfg.layers * (3 * 2 + 3 + 1 + 1) + 1
        line = {"metric": METRIC, "value": round(value, 2), "unit": "tokens/s", "n_gpus": world,
                "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_max / args.steps, 4),
                "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
                "dtype": "q8_0/q4_0 x q8_0 -> f32", "data": "synthetic",
                "config": dict(CONFIG, parallelism=f"replicas x{world}" if world > 1 else "single GPU"),
                "e2e": {"value": round(e2e_value, 2), "unit": "tokens/s", "h2d_bytes_per_step": BATCH * 8,
                        "d2h_bytes_per_step": BATCH * 8},
                "gpu_launches": launches_per_step * args.steps,
                "roofline": {"bound": "hbm", "kernel": "Q4_0 vocab readout (one launch: query quantization, tile GEMV, suppression, argmax)",
                             "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                             "frac": round(achieved / peak, 4), "peak_kind": peak_kind,
                             "algorithmic_bytes_per_launch": alg_bytes,
                             "launch_us": round(launch_s * 1e6, 3), "traffic": committed_traffic()},
                "cpu_baseline": cpu,
                "clocks": {k: clk[k] for k in ("sm_mhz", "sm_max_mhz", "reasons", "samples", "source")}}
    for gd in graphs:
        gd.graph = None
    rg = None
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if line is not None:
        print(json.dumps(line), flush=True)
    for d in decs:
        d.close()
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=64)
    ap.add_argument("--warmup", type=int, default=8)
    ap.add_argument("--impl", choices=["b200", "reference"], default="b200")
    args = ap.parse_args()
    if args.warmup < 3:
        raise SystemExit("--warmup must be at least 3")
    if args.impl == "reference":
        return run_reference(args)
    return run_b200(args)


if __name__ == "__main__":
    sys.exit(main())
