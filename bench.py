"""Throughput of the block-quantized Whisper encoder path on B200.

Workload (the Whisper-large-v3-shaped encoder): log-mel input [16, 128, 3000]
fp32 ~ U(-1.5, 1.0); two convolution stems (128 -> 1280 kernel 3, 1280 -> 1280
kernel 3 stride 2) with GELU, + positions; 32 pre-LN layers of width 1280,
20 heads of 64, FFN 5120 with GELU; final LayerNorm -> encoder states
[16, 1500, 1280] fp32. Every linear and both convolutions are Q8_0 (seeded
N(0, 0.02) weights, fp16 pre-round). One step = one forward of the whole
batch: 16 x 1500 = 24,000 tokens through the 32-layer stack.

--gpus 1 runs the encoder on one GPU (tensor parallelism 1). Under torchrun
with N ranks the same forward runs tensor-parallel over N GPUs (QKV and fc1
column-parallel by heads / FFN columns; out_proj and fc2 row-parallel with the
reduction over NVLink peer memory), so the total work per step is fixed:
``scaling: strong``, ``value`` = 24,000 tokens per step / step time (max over
ranks).

L2 policy: the inputs exceed L2 (the 24,000 x 1280 fp32 residual stream is
123 MB and each forward streams 668 MB of weights through the 126 MB L2).

--impl reference times the reference's own CPU arithmetic for the same encoder
on the host cores (oracle/encoder_cpu_baseline.py: the vendored ggml x86
quantizer + vec_dot kernels compiled from the reference sources into
oracle/_ref for every contraction), one utterance of the batch per step.
"""
from __future__ import annotations

import argparse
import hashlib
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

BATCH = 16
POSITIONS = 1500
LAYERS = 32
TOKENS = BATCH * POSITIONS
METRIC = "tokens/s per layer stack (Whisper-large-v3-shaped encoder, Q8_0)"
CONFIG = {"workload": "whisper-large-v3-shaped encoder: conv stems 128->1280->1280, 32 pre-LN layers d1280 h20 "
                      "ffn5120, Q8_0 linears and convolutions, log-mel [16,128,3000] -> states [16,1500,1280]",
          "batch": BATCH, "positions": POSITIONS, "layers": LAYERS,
          "l2": "inputs larger than L2 (123 MB fp32 residual stream, 668 MB of Q8_0 weights per forward)"}


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


# ----------------------------------------------------------------------------- peaks / traffic
def measured_peaks():
    """(peaks dict, "measured" | "fallback"): the measured copy bandwidth and bf16 GEMM rates in
    MEASURED_PEAKS.json beside this script when it exists, else fixed fallback figures."""
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": d.get("hbm_gbs", 6650.0), "bf16_tflops": d.get("bf16_tflops", 1590.0),
                "bf16_tflops_sustained": d.get("bf16_tflops_sustained", 1400.0)}, "measured"
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}, "fallback"


GEMM_SOURCE = ROOT / "mstar_accelerators_b200" / "csrc" / "gemm.cu"
GEMM_PROFILE = ROOT / "profiles" / "gemm_encoder_large_b16.md"


def gemm_traffic():
    """DRAM bytes (read + write) per GEMM launch of one encoder layer, from the ncu capture
    summarised in profiles/gemm_encoder_large_b16.md, or None when that capture was taken
    on another revision of the GEMM kernel (the summary records the source's SHA-256)."""
    if not GEMM_PROFILE.exists():
        return None, "no ncu capture committed"
    fields = {}
    for line in GEMM_PROFILE.read_text().splitlines():
        if ":" in line and line.split(":")[0].strip() in ("gemm_cu_sha256", "traffic_bytes_per_launch"):
            k, v = line.split(":", 1)
            fields[k.strip()] = v.strip().strip("`")
    sha = hashlib.sha256(GEMM_SOURCE.read_bytes()).hexdigest()
    if fields.get("gemm_cu_sha256") != sha:
        return None, "the committed ncu capture is of another revision of gemm.cu"
    try:
        return int(fields["traffic_bytes_per_launch"]), "ncu capture of this gemm.cu revision (" + GEMM_PROFILE.name + ")"
    except (KeyError, ValueError):
        return None, "capture summary unreadable"


# ----------------------------------------------------------------------------- cpu arm
def cpu_sample(sample_layers: int):
    from oracle.encoder_cpu_baseline import CpuEncoderSample
    return CpuEncoderSample(mels=128, width=1280, heads=20, layers=LAYERS, positions=POSITIONS,
                            sample_layers=sample_layers, seed=1)


def cpu_rate(sample, steps: int, warmup: int):
    """Tokens/s of the CPU encoder sample: `warmup` untimed, then `steps` timed forwards."""
    for _ in range(warmup):
        sample.forward_seconds()
    secs = [sample.forward_seconds() for _ in range(steps)]
    return POSITIONS * len(secs) / sum(secs), secs


def run_reference(args):
    rank, world, _ = env_rank()
    if rank != 0:
        return 0
    # each step is one utterance through the stems, a few layers and the final norm; fewer
    # sampled layers for long runs so the whole run stays within a few minutes
    sample = cpu_sample(2 if args.steps + args.warmup <= 40 else 1)
    value, secs = cpu_rate(sample, args.steps, args.warmup)
    line = {"metric": METRIC, "value": round(value, 2), "unit": "tokens/s", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(1e3 * sum(secs) / len(secs), 3),
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "q8_0 x q8_0 -> f32", "data": "synthetic", "config": CONFIG, "impl": "reference",
            "cpu_baseline": {"value": round(value, 2), "unit": "tokens/s", "cores": sample.threads,
                             "kind": "reference", "sample": sample.sample_text()},
            "e2e": {"value": round(value, 2), "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)
    return 0


# ----------------------------------------------------------------------------- b200 arm
def time_calls(calls, reps, stream):
    """Average device microseconds of each named call list: events around `reps` rounds."""
    import torch
    out = {}
    for name, fns in calls.items():
        for f in fns:   # warm
            f()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        for _ in range(reps):
            for f in fns:
                f()
        b.record(stream)
        b.synchronize()
        out[name] = a.elapsed_time(b) * 1e3 / (reps * len(fns))
    return out


def gemm_roofline(enc, tp: bool, stream):
    """Live CUDA-event timing of the encoder's GEMM launches (the dominant kernel), one
    layer's four shapes over 8 rotating layers (8 x 39 MB of fp16 weights > L2)."""
    import torch
    from mstar_accelerators_b200.linear import stage_rows
    cfg = enc.cfg
    M = BATCH * POSITIONS
    d = cfg.width
    st = enc.status
    layers = enc.layers[:8]
    x = torch.randn((M, d), device="cuda")
    a_d = stage_rows(x)
    if tp:
        dl, fl = enc.d_local, enc.f_local
        a_dl = stage_rows(torch.randn((M, dl), device="cuda"))
        h = torch.empty((M, fl), dtype=torch.float16, device="cuda")
        qkv = enc.qkv16
        part = enc.part[:M * d].view(M, d)
        calls = {
            "qkv": [lambda L=L: L["qkv"].gemm(a_d, out=qkv, out_format="f16", segments=(POSITIONS, cfg.padded_keys),
                                             status=st) for L in layers],
            "out_proj": [lambda L=L: L["out"].gemm(a_dl, out=part, bias=False, status=st) for L in layers],
            "fc1": [lambda L=L: L["fc1"].gemm(a_d, out=h, out_format="staged", gelu="tanh", status=st)
                    for L in layers],
            "fc2": [lambda L=L: L["fc2"].gemm(h, out=part, bias=False, status=st) for L in layers]}
        flops = {"qkv": 2 * M * 3 * dl * d, "out_proj": 2 * M * d * dl, "fc1": 2 * M * fl * d, "fc2": 2 * M * d * fl}
    else:
        f = cfg.ffn
        h = enc.hidden16[:M]
        qkv = enc.qkv16[:BATCH]
        xs = enc.x[:M]
        calls = {
            "qkv": [lambda L=L: L["qkv"].gemm(a_d, out=qkv, out_format="f16", segments=(POSITIONS, cfg.padded_keys),
                                             status=st) for L in layers],
            "out_proj": [lambda L=L: L["out"].gemm(a_d, out=xs, residual=xs, status=st) for L in layers],
            "fc1": [lambda L=L: L["fc1"].gemm(a_d, out=h, out_format="staged", gelu="tanh", status=st)
                    for L in layers],
            "fc2": [lambda L=L: L["fc2"].gemm(h, out=xs, residual=xs, status=st) for L in layers]}
        flops = {"qkv": 2 * M * 3 * d * d, "out_proj": 2 * M * d * d, "fc1": 2 * M * f * d, "fc2": 2 * M * d * f}
    us = time_calls(calls, 4, stream)
    per = {k: {"us": round(us[k], 2), "tflops": round(flops[k] / us[k] / 1e6, 1)} for k in us}
    tot_flops, tot_us = sum(flops.values()), sum(us.values())
    return tot_flops / len(us), tot_us / len(us), per


def decode_secondary(steps: int, warmup: int):
    """Whisper-tiny decode (Q8_0 body, tied Q4_0 readout 51865 x 384) at batch 32, one greedy
    step per CUDA-graph replay over 8 rotating weight replicas (> L2): the decode-bound line."""
    import torch
    from mstar_accelerators_b200.whisper import GraphDecoder, WhisperConfig, WhisperDecoderB200, synthetic_weights
    cfg, batch, prompt_len, replicas = WhisperConfig(), 32, 4, 8
    weights = synthetic_weights(cfg, seed=1, device="cuda")
    g = torch.Generator().manual_seed(2)
    enc = torch.randn((1, cfg.source, cfg.d_model), generator=g).cuda()
    prompt = torch.randint(0, cfg.vocab, (batch, prompt_len), generator=torch.Generator().manual_seed(3)).cuda()
    decs, graphs = [], []
    for _ in range(replicas):
        dec = WhisperDecoderB200(weights, cfg, batch=batch)
        _, tok = dec.prefill(prompt, enc)
        gd = GraphDecoder(dec)
        gd.tokens.copy_(tok)
        gd.positions.fill_(prompt_len)
        gd.capture()
        decs.append(dec)
        graphs.append(gd)
    steps = min(steps, (cfg.target - prompt_len - 2) * replicas - warmup)
    for i in range(warmup):
        graphs[i % replicas].graph.replay()
    stream = torch.cuda.current_stream()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    a.record(stream)
    for i in range(steps):
        graphs[(warmup + i) % replicas].graph.replay()
    b.record(stream)
    torch.cuda.synchronize()
    ms = a.elapsed_time(b) / steps
    weight_bytes = 8_767_488 + 11_202_840   # Q8_0 body + Q4_0 readout per step
    for gd in graphs:
        gd.graph = None
    for d in decs:
        d.close()
    return {"workload": "whisper-tiny decoder, batch 32, greedy decode step (4 layers d384, Q8_0 body, Q4_0 "
                        "readout 51865x384, cross-attention over 1500 positions), 8 rotating weight replicas",
            "value": round(batch / (ms / 1e3), 2), "unit": "tokens/s", "ms_per_step": round(ms, 4),
            "steps": steps, "weight_gbs": round(weight_bytes / (ms / 1e3) / 1e9, 1)}


def run_b200(args):
    import torch
    import torch.distributed as dist
    from mstar_accelerators_b200 import native
    from mstar_accelerators_b200.encoder import LARGE_V3, WhisperEncoderB200, synthetic_mel, synthetic_weights

    rank, world, local = env_rank()
    torch.cuda.set_device(local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=torch.device("cuda", local))
    native.require_capability()
    cfg = LARGE_V3
    weights = synthetic_weights(cfg, seed=1)
    mel_host = synthetic_mel(cfg, BATCH, seed=2).pin_memory()
    mel = mel_host.cuda()
    if world > 1:
        from mstar_accelerators_b200.encoder_tp import WhisperEncoderTP
        enc = WhisperEncoderTP(weights, cfg, max_batch=BATCH)
    else:
        enc = WhisperEncoderB200(weights, cfg, max_batch=BATCH)
    del weights
    states = torch.empty((BATCH, POSITIONS, cfg.width), dtype=torch.float32, device="cuda")

    def step():
        enc(mel, out=states)

    stream = torch.cuda.current_stream()
    for _ in range(args.warmup):
        step()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    with ClockSampler(local) as clocks:
        start.record(stream)
        for _ in range(args.steps):
            step()
        end.record(stream)
        clocks.wait(end)
        torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    t = torch.tensor([start.elapsed_time(end)], device="cuda")
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_max = float(t.item())
    value = TOKENS * args.steps / (ms_max / 1e3)
    status = int(enc.status.item())

    # e2e through the public forward with host buffers: pinned mel in, states back to pinned host memory
    states_host = torch.empty((BATCH, POSITIONS, cfg.width), dtype=torch.float32).pin_memory()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        mel.copy_(mel_host, non_blocking=True)
        enc(mel, out=states)
        states_host.copy_(states, non_blocking=True)
        stream.synchronize()
    e1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = torch.tensor([e0.elapsed_time(e1)], device="cuda")
    if world > 1:
        dist.all_reduce(e2e_ms, op=dist.ReduceOp.MAX)
    e2e_value = TOKENS * args.steps / (float(e2e_ms.item()) / 1e3)

    # roofline of the dominant kernel (the tcgen05 GEMM), timed live on this stream
    flops_per_launch, us_per_launch, per_shape = gemm_roofline(enc, world > 1, stream)
    peaks, peak_kind = measured_peaks()
    achieved = flops_per_launch / us_per_launch / 1e6   # TFLOP/s
    traffic, traffic_src = gemm_traffic()
    launches = enc.launches_per_forward() * args.steps

    line = None
    if rank == 0:
        cpu = None
        secondary = None
        if world == 1:
            sample = cpu_sample(2)
            cpu_value, secs = cpu_rate(sample, 2, 1)
            cpu = {"value": round(cpu_value, 2), "unit": "tokens/s", "cores": sample.threads, "kind": "reference",
                   "sample": sample.sample_text() + f"; {len(secs)} timed forwards"}
            if not args.no_decode:
                secondary = decode_secondary(64, 8)
        clk = clocks.summary()
        line = {"metric": METRIC, "value": round(value, 2), "unit": "tokens/s", "n_gpus": world,
                "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_max / args.steps, 4),
                "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
                "dtype": "q8_0 x q8_0 -> f32 (tensor cores on fp16(q*d) operands, fp32 accumulation)",
                "data": "synthetic", "config": dict(CONFIG, parallelism=f"tp{world}"),
                "e2e": {"value": round(e2e_value, 2), "unit": "tokens/s",
                        "h2d_bytes_per_step": mel_host.numel() * 4, "d2h_bytes_per_step": states_host.numel() * 4},
                "gpu_launches": launches,
                "roofline": {"bound": "tensor", "kernel": "k_gemm_pair (tcgen05 CTA-pair GEMM of the encoder "
                                                          "linears; average over one layer's four shapes)",
                             "achieved": round(achieved, 1), "peak": peaks["bf16_tflops"], "unit": "TFLOP/s",
                             "frac": round(achieved / peaks["bf16_tflops"], 4),
                             "peak_kind": peak_kind + " (burst bf16: the GEMMs are timed alone)",
                             "flops_per_launch": flops_per_launch, "launch_us": round(us_per_launch, 2),
                             "per_shape": per_shape, "traffic": traffic, "traffic_source": traffic_src},
                "cpu_baseline": cpu, "status": status,
                "clocks": {k: clk[k] for k in ("sm_mhz", "sm_max_mhz", "reasons", "samples", "source")}}
        if secondary is not None:
            line["secondary_decode"] = secondary
    if world > 1:
        dist.barrier()
    enc.close()
    if world > 1:
        dist.destroy_process_group()
    if line is not None:
        print(json.dumps(line), flush=True)
    return 0 if status == 0 else 1


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["b200", "reference"], default="b200")
    ap.add_argument("--no-decode", action="store_true", help="skip the secondary Whisper-tiny decode line")
    args = ap.parse_args()
    if args.warmup < 3:
        raise SystemExit("--warmup must be at least 3")
    if args.impl == "reference":
        return run_reference(args)
    return run_b200(args)


if __name__ == "__main__":
    sys.exit(main())
