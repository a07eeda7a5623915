"""Named small workloads for profiling one kernel or one step under ncu.

    python -m mstar_accelerators_b200.cases readout-q4-b32
    python -m mstar_accelerators_b200.cases decode-step-b32
    python -m mstar_accelerators_b200.cases encoder-large-b16
    python -m mstar_accelerators_b200.cases gemm-encoder-large-layer
    python -m mstar_accelerators_b200.cases moe-prefill-4096

Each case builds its inputs from fixed seeds, runs a few calls, synchronises
and prints "ok". The ncu summaries under profiles/ name the case they used.
"""
from __future__ import annotations

import sys

import torch


def readout_q4_b32():
    """Whisper-tiny tied Q4_0 readout (51865 x 384, tile layout), 32 query rows, three calls."""
    from .linear import BlockLinear
    g = torch.Generator(device="cuda").manual_seed(1)
    w = torch.randn(51865, 384, device="cuda", generator=g) * 0.02
    head = BlockLinear(w, fmt="q4_0")
    head.prepare_readout()
    x = torch.randn(32, 384, device="cuda", generator=g)
    for _ in range(3):
        head.readout(x)


def decode_step_b32():
    """One Whisper-tiny decoder at batch 32: prefill 4 tokens, capture the greedy
    decode step as a CUDA graph, replay it twice."""
    from .whisper import GraphDecoder, WhisperConfig, WhisperDecoderB200, synthetic_weights
    cfg = WhisperConfig()
    w = synthetic_weights(cfg, seed=1, device="cuda")
    g = torch.Generator(device="cuda").manual_seed(2)
    enc = torch.randn((1, cfg.source, cfg.d_model), device="cuda", generator=g)
    dec = WhisperDecoderB200(w, cfg, batch=32)
    prompt = torch.randint(0, cfg.vocab, (32, 4), device="cuda", generator=g)
    _, tok = dec.prefill(prompt, enc)
    gd = GraphDecoder(dec)
    gd.tokens.copy_(tok)
    gd.positions.fill_(4)
    gd.capture()
    gd.run(2)


def gemm_q8_8192x5120x1280():
    """Q8_0 prefill GEMM of a Whisper-large fc1 shape (N=5120, K=1280) over 8192 rows, three calls."""
    from .linear import BlockLinear
    g = torch.Generator(device="cuda").manual_seed(1)
    lin = BlockLinear(torch.randn(5120, 1280, device="cuda", generator=g) * 0.02)
    lin.prepare_gemm(8192)
    x = torch.randn(8192, 1280, device="cuda", generator=g)
    out = torch.empty(8192, 5120, device="cuda")
    for _ in range(3):
        lin(x, out=out)


def gemm_encoder_large_layer():
    """The four GEMMs of one Whisper-large-v3-shaped encoder layer at the bench's 24,000 rows, each
    in its encoder mode (QKV fp16 into padded planes; out_proj fp32 + residual; fc1 GELU + Q8_0-staged
    fp16; fc2 fp32 + residual), two rounds: 8 launches, the second four the ones to profile."""
    from .encoder import LARGE_V3
    from .linear import BlockLinear, stage_rows
    g = torch.Generator(device="cuda").manual_seed(1)
    d, f, M, T, P = LARGE_V3.width, LARGE_V3.ffn, 24000, 1500, LARGE_V3.padded_keys

    def lin(n, k):
        L = BlockLinear(torch.randn(n, k, device="cuda", generator=g) * 0.02,
                        bias=torch.randn(n, device="cuda", generator=g) * 0.02)
        L.prepare_gemm(M)
        return L
    qkv, out, fc1, fc2 = lin(3 * d, d), lin(d, d), lin(f, d), lin(d, f)
    a = stage_rows(torch.randn(M, d, device="cuda", generator=g))
    planes = torch.zeros((M // T, P, 3 * d), dtype=torch.float16, device="cuda")
    x = torch.randn(M, d, device="cuda", generator=g)
    h = torch.empty((M, f), dtype=torch.float16, device="cuda")
    for _ in range(2):
        qkv.gemm(a, out=planes, out_format="f16", segments=(T, P))
        out.gemm(a, out=x, residual=x)
        fc1.gemm(a, out=h, out_format="staged", gelu="tanh")
        fc2.gemm(h, out=x, residual=x)


def gemm_fc1_exact_and_f16():
    """The Whisper-large-v3 fc1 shape (N=5120, K=1280) at 24,000 rows, fp32 output, through the
    exact int8-tensor-pipe GEMM and through the fp16-staged GEMM, two calls each (launch order:
    exact activation quantization, exact GEMM, fp16 staging, fp16 GEMM, twice)."""
    from .linear import BlockLinear, stage_rows
    g = torch.Generator(device="cuda").manual_seed(1)
    lin = BlockLinear(torch.randn(5120, 1280, device="cuda", generator=g) * 0.02)
    lin.prepare_gemm(24000)
    lin.prepare_exact()
    x = torch.randn(24000, 1280, device="cuda", generator=g)
    out = torch.empty(24000, 5120, device="cuda")
    for _ in range(2):
        lin.exact(x, out=out)
        lin.gemm(stage_rows(x), out=out)


def thinker_stack_48():
    """The Qwen3-Omni thinker 48-layer stack (Q8_0 linears and experts) on one GPU: 32 sequences of
    1024 synthetic prompt tokens (a warm-up prefill, then the timed one), then 128 greedy decode
    steps, each one CUDA-graph replay of the 48 layers and the readout; prints the device times."""
    import json
    from .thinker_stack import ThinkerStackB200, ThinkerStackConfig
    cfg = ThinkerStackConfig()
    stack = ThinkerStackB200(cfg, max_seqs=32, max_len=1024 + 128 + 4)
    g = torch.Generator().manual_seed(3)
    prompt = torch.randint(0, cfg.vocab, (32, 1024), generator=g).cuda()
    stack.prefill(prompt)
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(4)]
    torch.cuda.synchronize()
    ev[0].record()
    _, tok = stack.prefill(prompt)
    ev[1].record()
    for _ in range(2):       # capture and a first replay
        _, tok = stack.decode(tok, graph=True)
    ev[2].record()
    for _ in range(128):
        _, tok = stack.decode(tok, graph=True)
    ev[3].record()
    torch.cuda.synchronize()
    pre, dec = ev[0].elapsed_time(ev[1]), ev[2].elapsed_time(ev[3])
    print(json.dumps({"prefill_ms": round(pre, 2), "prefill_tokens_per_s": round(32 * 1024 / (pre / 1e3), 1),
                      "decode_ms_per_step": round(dec / 128, 3), "decode_tokens_per_s": round(32 * 128 / (dec / 1e3), 1),
                      "status": int(stack.status.item())}))
    stack.close()


def thinker_stack_4_decode():
    """Four thinker layers (the 48-layer stack's geometry) decoding 32 sequences after a
    1024-token prompt: three warm-up steps, then one step inside the NVTX range "step"
    (not graph-captured, so a profiler sees each launch)."""
    from dataclasses import replace
    from .thinker_stack import ThinkerStackB200, ThinkerStackConfig
    cfg = replace(ThinkerStackConfig(), layers=4)
    stack = ThinkerStackB200(cfg, max_seqs=32, max_len=1024 + 8)
    g = torch.Generator().manual_seed(3)
    _, tok = stack.prefill(torch.randint(0, cfg.vocab, (32, 1024), generator=g).cuda())
    for _ in range(3):
        _, tok = stack.decode(tok)
    torch.cuda.synchronize()
    torch.cuda.nvtx.range_push("step")
    _, tok = stack.decode(tok)
    torch.cuda.nvtx.range_pop()
    torch.cuda.synchronize()
    stack.close()


def thinker_stack_4_prefill():
    """Four thinker layers (the 48-layer stack's geometry) prefilling 32 sequences of 1024
    tokens: a warm-up prefill, then one inside the NVTX range "prefill"."""
    from dataclasses import replace
    from .thinker_stack import ThinkerStackB200, ThinkerStackConfig
    cfg = replace(ThinkerStackConfig(), layers=4)
    stack = ThinkerStackB200(cfg, max_seqs=32, max_len=1024 + 8)
    prompt = torch.randint(0, cfg.vocab, (32, 1024), generator=torch.Generator().manual_seed(3)).cuda()
    stack.prefill(prompt)
    torch.cuda.synchronize()
    torch.cuda.nvtx.range_push("prefill")
    stack.prefill(prompt)
    torch.cuda.nvtx.range_pop()
    torch.cuda.synchronize()
    stack.close()


def thinker_stack_48_tp():
    """The 48-layer thinker stack with attention tensor-parallel and the experts expert-parallel over
    the ranks of a torchrun launch (one process per GPU, RANK / WORLD_SIZE / MASTER_* from the
    environment): the same workload as thinker-stack-48; device times are the maximum over ranks."""
    import json
    import os
    from datetime import timedelta
    import torch.distributed as dist
    from .thinker_stack import ThinkerStackConfig
    from .thinker_stack_tp import ThinkerStackTP
    rank = int(os.environ["RANK"])
    torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", rank)))
    dist.init_process_group("nccl", timeout=timedelta(seconds=300),
                            device_id=torch.device("cuda", torch.cuda.current_device()))
    try:
        cfg = ThinkerStackConfig()
        stack = ThinkerStackTP(cfg, max_seqs=32, max_len=1024 + 128 + 4, max_tokens=32 * 1024)
        g = torch.Generator().manual_seed(3)
        prompt = torch.randint(0, cfg.vocab, (32, 1024), generator=g).cuda()
        stack.prefill(prompt)
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(4)]
        torch.cuda.synchronize()
        dist.barrier()
        ev[0].record()
        _, tok = stack.prefill(prompt)
        ev[1].record()
        for _ in range(2):       # capture and a first replay
            _, tok = stack.decode(tok, graph=True)
        ev[2].record()
        for _ in range(128):
            _, tok = stack.decode(tok, graph=True)
        ev[3].record()
        torch.cuda.synchronize()
        t = torch.tensor([ev[0].elapsed_time(ev[1]), ev[2].elapsed_time(ev[3])], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        mine = torch.tensor([int(stack.status.item()) | stack.expert_status()], device="cuda")
        every = [torch.zeros_like(mine) for _ in range(dist.get_world_size())]
        dist.all_gather(every, mine)   # status bits of every rank (NCCL has no bitwise-or reduction)
        st = torch.tensor([0])
        for e in every:
            st |= e.cpu()
        pre, dec = t.tolist()
        if rank == 0:
            print(json.dumps({"ranks": dist.get_world_size(), "prefill_ms": round(pre, 2),
                              "prefill_tokens_per_s": round(32 * 1024 / (pre / 1e3), 1),
                              "decode_ms_per_step": round(dec / 128, 3),
                              "decode_tokens_per_s": round(32 * 128 / (dec / 1e3), 1), "status": int(st.item())}))
        stack.close()
    finally:
        dist.destroy_process_group()


def _encoder(cfg, batch, calls):
    from .encoder import WhisperEncoderB200, synthetic_mel, synthetic_weights
    w = {k: v.cuda() for k, v in synthetic_weights(cfg, seed=1).items()}
    mel = synthetic_mel(cfg, batch, seed=2).cuda()
    enc = WhisperEncoderB200(w, cfg, max_batch=batch)
    for i in range(calls):   # NVTX range per forward, so a profiler can keep one forward's launches only
        torch.cuda.nvtx.range_push(f"forward{i}")
        enc(mel)
        torch.cuda.nvtx.range_pop()


def encoder_tiny_b1():
    """Whisper-tiny encoder (4 layers, width 384) on one utterance, two calls."""
    from .encoder import TINY
    _encoder(TINY, 1, 2)


def encoder_large_b16():
    """Whisper-large-v3-shaped encoder (32 layers, width 1280) on 16 utterances, two calls."""
    from .encoder import LARGE_V3
    _encoder(LARGE_V3, 16, 2)


def moe_prefill_4096(fmt: str = "bf16"):
    """Qwen3-Omni thinker MoE layer (128 experts, I 768, H 2048, top-8) over 4096 tokens, three calls."""
    from .moe import ThinkerMoEB200, route
    g = torch.Generator(device="cuda").manual_seed(5)
    E, I, H, K, T = 128, 768, 2048, 8, 4096
    w1 = (torch.randn((E, 2 * I, H), device="cuda", generator=g) * 0.02).to(torch.bfloat16)
    w2 = (torch.randn((E, H, I), device="cuda", generator=g) * 0.02).to(torch.bfloat16)
    wr = (torch.randn((E, H), device="cuda", generator=g) * 0.02).to(torch.bfloat16)
    x = torch.randn((T, H), device="cuda", generator=g).to(torch.bfloat16)
    if fmt == "q8_0":  # canonical Q8_0 expert bytes
        from .linear import pack
        w1 = pack(w1.float().reshape(-1, H), "q8_0", preround=False).reshape(E, 2 * I, -1)
        w2 = pack(w2.float().reshape(-1, I), "q8_0", preround=False).reshape(E, H, -1)
        layer = ThinkerMoEB200(w1, w2, fmt=fmt, top_k=K, max_tokens=T, intermediate=I, hidden=H)
    else:
        layer = ThinkerMoEB200(w1, w2, fmt=fmt, top_k=K, max_tokens=T)
    w, ids = route(x, wr, top_k=K)
    for _ in range(3):
        layer(x, w, ids)


def moe_prefill_4096_q8():
    """The same layer with Q8_0 experts."""
    moe_prefill_4096("q8_0")


CASES = {"readout-q4-b32": readout_q4_b32, "decode-step-b32": decode_step_b32,
         "gemm-q8-8192x5120x1280": gemm_q8_8192x5120x1280, "gemm-encoder-large-layer": gemm_encoder_large_layer,
         "gemm-fc1-exact-and-f16": gemm_fc1_exact_and_f16, "thinker-stack-48": thinker_stack_48,
         "thinker-stack-48-tp": thinker_stack_48_tp, "thinker-stack-4-decode": thinker_stack_4_decode,
         "thinker-stack-4-prefill": thinker_stack_4_prefill,
         "encoder-tiny-b1": encoder_tiny_b1,
         "encoder-large-b16": encoder_large_b16, "moe-prefill-4096": moe_prefill_4096,
         "moe-prefill-4096-q8": moe_prefill_4096_q8}


def main(argv):
    if len(argv) != 1 or argv[0] not in CASES:
        print("cases:", ", ".join(CASES))
        return 2
    torch.cuda.set_device(0)
    CASES[argv[0]]()
    torch.cuda.synchronize()
    print("ok")
    return 0


if __name__ == "__main__":
    sys.exit(main(sys.argv[1:]))
