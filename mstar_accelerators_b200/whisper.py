"""Whisper decoder on B200: the reference decoder graph with every linear on
the block-quantized sm_100a kernels.

Mirrors backends/cpu_ggml/decoder.cpp:489-600 (Graph::build) and the token
entry cpu_decoder_token_run (decoder.cpp:857-921): per layer
  n = LN(x); q,k,v = Q8_0 linears(n); x += out_proj(attend(q, K, V))
  n = LN(x); q = Q8_0(n);            x += out_proj(attend(q, crossK, crossV))
  n = LN(x); x += fc2(gelu(fc1(n)))
then LN and the Q4_0 (or Q8_0) vocabulary readout with suppression and the
first-index / NaN-first argmax (decoder.cpp:583-588, 686-696). The cross K/V
planes are written once at prefill from one fused [3072 x 384] Q8_0
projection of the encoder states (decoder.cpp:247-250, 322-330).

B200 layout choices: q/k/v of a layer are one [1152 x 384] matrix (one
launch), every LayerNorm is fused into the quantize step of the linear that
consumes it, bias / GELU / residual run in the GEMV epilogue, K/V planes are
fp16 [seq][capacity][384], and a batch of sequences decodes together (each
row of the GEMV is one sequence). Host code only enqueues; the whole decode
step can be captured in one CUDA graph.
"""
from __future__ import annotations

import ctypes as C
import math
from dataclasses import dataclass

import torch

from . import native
from .linear import BlockLinear, _stream
from .native import check, error_buffer


@dataclass(frozen=True)
class WhisperConfig:
    d_model: int = 384
    layers: int = 4
    heads: int = 6
    ffn: int = 1536
    vocab: int = 51865
    source: int = 1500   # max_source_positions
    target: int = 448    # max_target_positions
    eps: float = 1e-5
    # whisper-tiny (decoder.cpp:194-195 admits exactly this geometry)


def weight_names(cfg: WhisperConfig) -> list[str]:
    names = ["decoder.embed_tokens.weight", "decoder.embed_positions.weight",
             "decoder.layer_norm.weight", "decoder.layer_norm.bias"]
    for i in range(cfg.layers):
        p = f"decoder.layers.{i}."
        for ln in ("self_attn_layer_norm", "encoder_attn_layer_norm", "final_layer_norm"):
            names += [p + ln + ".weight", p + ln + ".bias"]
        for att in ("self_attn", "encoder_attn"):
            for proj in ("q_proj", "k_proj", "v_proj", "out_proj"):
                names.append(p + f"{att}.{proj}.weight")
                if proj != "k_proj":
                    names.append(p + f"{att}.{proj}.bias")
        names += [p + "fc1.weight", p + "fc1.bias", p + "fc2.weight", p + "fc2.bias"]
    return names


def synthetic_weights(cfg: WhisperConfig, seed: int = 1, device="cpu") -> dict[str, torch.Tensor]:
    """Seeded random Whisper decoder weights: linears/embeddings N(0, 0.02),
    LayerNorm weight 1 + N(0, 0.02), biases N(0, 0.02)."""
    g = torch.Generator().manual_seed(seed)
    d, f = cfg.d_model, cfg.ffn
    out = {}
    for name in weight_names(cfg):
        if name.endswith("embed_tokens.weight"):
            shape = (cfg.vocab, d)
        elif name.endswith("embed_positions.weight"):
            shape = (cfg.target, d)
        elif "fc1.weight" in name:
            shape = (f, d)
        elif "fc1.bias" in name:
            shape = (f,)
        elif "fc2.weight" in name:
            shape = (d, f)
        elif name.endswith(".weight") and "norm" not in name:
            shape = (d, d)
        else:
            shape = (d,)
        t = torch.randn(shape, generator=g) * 0.02
        if "norm" in name and name.endswith(".weight"):
            t = t + 1.0
        out[name] = t.to(device)
    return out


class WhisperDecoderB200:
    """Prepared decoder for `batch` sequences on the current CUDA device."""

    def __init__(self, weights: dict[str, torch.Tensor], cfg: WhisperConfig = WhisperConfig(), *, batch: int = 1,
                 readout_format: str = "q4_0", rounding: str = "arm", shared_cross: bool = True,
                 suppressed: dict[str, list[int]] | None = None, device=None):
        if cfg.d_model // cfg.heads != 64:
            raise ValueError("the attention kernel is specialised for head_dim 64")
        self.lib = native.require_capability()
        self.cfg, self.batch, self.rounding = cfg, batch, rounding
        self.device = torch.device(device or "cuda")
        dev = self.device
        W = {k: v.detach().to(device=dev, dtype=torch.float32).contiguous() for k, v in weights.items()}
        d, L = cfg.d_model, cfg.layers
        zeros = torch.zeros(d, device=dev)

        def bias(name):
            return W.get(name, zeros)

        self.layers = []
        for i in range(L):
            p = f"decoder.layers.{i}."
            sa, ca = p + "self_attn.", p + "encoder_attn."
            qkv_w = torch.cat([W[sa + "q_proj.weight"], W[sa + "k_proj.weight"], W[sa + "v_proj.weight"]])
            qkv_b = torch.cat([bias(sa + "q_proj.bias"), bias(sa + "k_proj.bias"), bias(sa + "v_proj.bias")])
            self.layers.append(dict(
                ln1=(W[p + "self_attn_layer_norm.weight"], W[p + "self_attn_layer_norm.bias"], cfg.eps),
                qkv=BlockLinear(qkv_w, bias=qkv_b),
                out=BlockLinear(W[sa + "out_proj.weight"], bias=bias(sa + "out_proj.bias")),
                ln2=(W[p + "encoder_attn_layer_norm.weight"], W[p + "encoder_attn_layer_norm.bias"], cfg.eps),
                cq=BlockLinear(W[ca + "q_proj.weight"], bias=bias(ca + "q_proj.bias")),
                cout=BlockLinear(W[ca + "out_proj.weight"], bias=bias(ca + "out_proj.bias")),
                ln3=(W[p + "final_layer_norm.weight"], W[p + "final_layer_norm.bias"], cfg.eps),
                fc1=BlockLinear(W[p + "fc1.weight"], bias=W[p + "fc1.bias"]),
                fc2=BlockLinear(W[p + "fc2.weight"], bias=W[p + "fc2.bias"]),
                ck_b=bias(ca + "k_proj.bias"), cv_b=bias(ca + "v_proj.bias"),
            ))
        cross_w = torch.cat([torch.cat([W[f"decoder.layers.{i}.encoder_attn.k_proj.weight"],
                                        W[f"decoder.layers.{i}.encoder_attn.v_proj.weight"]]) for i in range(L)])
        self.cross = BlockLinear(cross_w)                       # [2*L*d, d], biases added at fill time
        self.lnf = (W["decoder.layer_norm.weight"], W["decoder.layer_norm.bias"], cfg.eps)
        self.tok = W["decoder.embed_tokens.weight"]
        self.pos = W["decoder.embed_positions.weight"]
        self.head = BlockLinear(self.tok, fmt=readout_format)   # tied readout (proj_out == embed_tokens)
        self.head.prepare_readout()
        self.suppressed = {k: torch.tensor(v, dtype=torch.int64, device=dev)
                           for k, v in (suppressed or {"prefill": [], "decode": []}).items()}
        self.shared_cross = shared_cross
        B = batch
        self.self_k = [torch.zeros((B, cfg.target, d), dtype=torch.float16, device=dev) for _ in range(L)]
        self.self_v = [torch.zeros_like(t) for t in self.self_k]
        nseq = 1 if shared_cross else B
        self.cross_k = [torch.zeros((nseq, cfg.source, d), dtype=torch.float16, device=dev) for _ in range(L)]
        self.cross_v = [torch.zeros_like(t) for t in self.cross_k]
        self.cross_len = torch.full((B,), cfg.source, dtype=torch.int64, device=dev)
        self.status = torch.zeros(1, dtype=torch.int32, device=dev)
        self._bufs = {}
        # split-attention workspaces per (queries, capacity, shared), zero-filled once
        self._ws = {}
        for nq in range(1, 5):
            for cap, sh in ((cfg.target, False), (cfg.source, self.shared_cross)):
                n = int(self.lib.mstar_b200_attend_workspace(cfg.heads, B, nq, cap, int(sh)))
                if n == 0:
                    raise ValueError("attention geometry outside the kernel's limits")
                self._ws[(nq, cap, sh)] = torch.zeros(n, dtype=torch.uint8, device=dev)

    # ------------------------------------------------------------------ buffers
    def _buf(self, name, shape, dtype=torch.float32):
        t = self._bufs.get(name)
        if t is None or tuple(t.shape) != tuple(shape):
            t = torch.empty(shape, dtype=dtype, device=self.device)
            self._bufs[name] = t
        return t

    # ------------------------------------------------------------------ pieces
    def _embed(self, ids: torch.Tensor, positions: torch.Tensor, x: torch.Tensor):
        e = error_buffer()
        check(self.lib.mstar_b200_embed(self.tok.data_ptr(), self.cfg.vocab, self.pos.data_ptr(), self.cfg.target,
                                        self.cfg.d_model, ids.data_ptr(), positions.data_ptr(), ids.numel(), 1.0,
                                        x.data_ptr(), self.status.data_ptr(), _stream(self.device), e, len(e)),
              e, "B200 embedding")

    def _attend(self, q, q_stride, k_new, v_new, kv_stride, kp, vp, capacity, nq, begin, kv_len, causal, shared, out,
                frags=None):
        """Attention into out; with frags (a linear's fragment descriptor) the rows are also
        quantized for that linear's run_frags."""
        ws = self._ws[(nq, capacity, bool(shared))]
        e = error_buffer()
        check(self.lib.mstar_b200_attend_q8(q.data_ptr(), q_stride, k_new.data_ptr() if k_new is not None else None,
                                            v_new.data_ptr() if v_new is not None else None, kv_stride,
                                            kp.data_ptr(), vp.data_ptr(), capacity, self.cfg.heads, 64, self.batch,
                                            nq, begin.data_ptr() if begin is not None else None,
                                            kv_len.data_ptr() if kv_len is not None else None, int(causal),
                                            int(shared), out.data_ptr(), out.stride(0), 1.0 / math.sqrt(64),
                                            self.status.data_ptr(), ws.data_ptr(), ws.numel(),
                                            C.byref(frags) if frags is not None else None, _stream(self.device),
                                            e, len(e)),
              e, "B200 attention")

    def _body(self, x: torch.Tensor, nq: int, begin: torch.Tensor):
        """All decoder layers over x [B*nq, d] (in place)."""
        cfg, B, r = self.cfg, self.batch, self.rounding
        d = cfg.d_model
        rows = B * nq
        qkv = self._buf(f"qkv{nq}", (rows, 3 * d))
        att = self._buf(f"att{nq}", (rows, d))
        cq = self._buf(f"cq{nq}", (rows, d))
        h = self._buf(f"h{nq}", (rows, cfg.ffn))
        fused = rows <= 32  # attention quantizes its rows straight into the out-projections' fragments
        for i, Lr in enumerate(self.layers):
            Lr["qkv"](x, out=qkv, norm=Lr["ln1"], rounding=r)
            self._attend(qkv, qkv.stride(0), qkv[:, d:], qkv[:, 2 * d:], qkv.stride(0), self.self_k[i],
                         self.self_v[i], cfg.target, nq, begin, None, True, False, att,
                         Lr["out"].frags(rows, r) if fused else None)
            if fused:
                Lr["out"].run_frags(rows, out=x, residual=x)
            else:
                Lr["out"](att, out=x, residual=x, rounding=r)
            Lr["cq"](x, out=cq, norm=Lr["ln2"], rounding=r)
            self._attend(cq, cq.stride(0), None, None, 0, self.cross_k[i], self.cross_v[i], cfg.source, nq, None,
                         self.cross_len, False, self.shared_cross, att, Lr["cout"].frags(rows, r) if fused else None)
            if fused:
                Lr["cout"].run_frags(rows, out=x, residual=x)
            else:
                Lr["cout"](att, out=x, residual=x, rounding=r)
            if fused:  # fc1's epilogue quantizes its GELU outputs straight into fc2's fragments
                Lr["fc1"](x, out=h, norm=Lr["ln3"], gelu="tanh", rounding=r, next_frags=Lr["fc2"].frags(rows, r))
                Lr["fc2"].run_frags(rows, out=x, residual=x)
            else:
                Lr["fc1"](x, out=h, norm=Lr["ln3"], gelu="tanh", rounding=r)
                Lr["fc2"](h, out=x, residual=x, rounding=r)

    def _readout(self, last: torch.Tensor, walk: str, logits, token):
        sup = self.suppressed.get(walk)
        return self.head.readout(last, sup if sup is not None and sup.numel() else None, rounding=self.rounding,
                                 norm=self.lnf, logits=logits, token=token, status=self.status)

    # ------------------------------------------------------------------ public
    def set_cross(self, encoder_states: torch.Tensor):
        """Write every layer's cross K/V planes from encoder states [S, source, d]
        (S = 1 shared, or the batch)."""
        cfg = self.cfg
        enc = encoder_states.to(device=self.device, dtype=torch.float32).reshape(-1, cfg.source, cfg.d_model)
        if enc.shape[0] != (1 if self.shared_cross else self.batch):
            raise ValueError("encoder states batch differs from the cross-plane layout")
        proj = self._buf("crossproj", (enc.shape[0] * cfg.source, 2 * cfg.layers * cfg.d_model))
        self.cross(enc.reshape(-1, cfg.d_model), out=proj, rounding=self.rounding)
        d = cfg.d_model
        for i, Lr in enumerate(self.layers):
            e = error_buffer()
            check(self.lib.mstar_b200_fill_kv(proj.data_ptr(), proj.stride(0), 2 * d * i, 2 * d * i + d,
                                              Lr["ck_b"].data_ptr(), Lr["cv_b"].data_ptr(),
                                              self.cross_k[i].data_ptr(), self.cross_v[i].data_ptr(), proj.shape[0],
                                              d, _stream(self.device), e, len(e)), e, "B200 cross KV")

    def prefill(self, tokens: torch.Tensor, encoder_states: torch.Tensor | None = None):
        """tokens [B, q] (q <= 4, positions 0..q-1) -> (logits [B, vocab], next token [B])."""
        cfg, B = self.cfg, self.batch
        tokens = tokens.to(self.device).reshape(B, -1)
        nq = tokens.shape[1]
        if encoder_states is not None:
            self.set_cross(encoder_states)
        positions = torch.arange(nq, device=self.device).repeat(B)
        x = self._buf(f"x{nq}", (B * nq, cfg.d_model))
        self.status.zero_()
        self._embed(tokens.reshape(-1).contiguous(), positions, x)
        begin = torch.zeros(B, dtype=torch.int64, device=self.device)
        self._body(x, nq, begin)
        last = x.view(B, nq, cfg.d_model)[:, -1]
        return self._readout(last, "prefill", None, None)[:2]

    def decode_into(self, tokens: torch.Tensor, positions: torch.Tensor, logits: torch.Tensor,
                    next_token: torch.Tensor):
        """One greedy step for every sequence: tokens [B] at positions [B] (device
        int64). Writes logits [B, vocab] and next_token [B]; graph-capturable."""
        x = self._buf("x1", (self.batch, self.cfg.d_model))
        self._embed(tokens, positions, x)
        self._body(x, 1, positions)
        self._readout(x, "decode", logits, next_token)

    def decode(self, tokens: torch.Tensor, positions: torch.Tensor):
        logits = torch.empty((self.batch, self.cfg.vocab), device=self.device)
        nxt = torch.empty(self.batch, dtype=torch.int64, device=self.device)
        self.decode_into(tokens.to(self.device), positions.to(self.device), logits, nxt)
        return logits, nxt

    def close(self):
        for Lr in self.layers:
            for k in ("qkv", "out", "cq", "cout", "fc1", "fc2"):
                Lr[k].close()
        self.cross.close()
        self.head.close()


class _StepConfig(C.Structure):
    """mstar_b200_decode_step_config (include/mstar_b200.h)."""
    _fields_ = [(n, C.c_int32) for n in ("batch", "layers", "width", "heads", "ffn", "target", "source",
                                         "shared_cross", "rounding")] + [
        ("eps", C.c_float), ("token_table", C.c_void_p), ("position_table", C.c_void_p), ("vocab", C.c_int64),
        ("positions_count", C.c_int64), ("linears", (C.c_void_p * 6) * 8), ("norms", (C.c_void_p * 6) * 8),
        ("self_k", C.c_void_p * 8), ("self_v", C.c_void_p * 8), ("cross_k", C.c_void_p * 8),
        ("cross_v", C.c_void_p * 8), ("head", C.c_void_p), ("final_norm_weight", C.c_void_p),
        ("final_norm_bias", C.c_void_p), ("suppressed", C.c_void_p), ("suppressed_count", C.c_uint64),
        ("tokens", C.c_void_p), ("positions", C.c_void_p), ("cross_length", C.c_void_p), ("logits", C.c_void_p),
        ("next_token", C.c_void_p), ("status", C.c_void_p)]


class PersistentStep:
    """The greedy decode step of a WhisperDecoderB200 as one persistent kernel
    (mstar_b200_decode_step_*): reads tokens / positions, writes logits and
    next tokens; identical results to WhisperDecoderB200.decode_into."""

    def __init__(self, dec: "WhisperDecoderB200", tokens: torch.Tensor, positions: torch.Tensor,
                 logits: torch.Tensor | None, next_token: torch.Tensor):
        cfg = dec.cfg
        if cfg.layers > 8:
            raise ValueError("the step kernel takes at most 8 layers")
        c = _StepConfig()
        c.batch, c.layers, c.width, c.heads, c.ffn = dec.batch, cfg.layers, cfg.d_model, cfg.heads, cfg.ffn
        c.target, c.source, c.shared_cross = cfg.target, cfg.source, int(dec.shared_cross)
        c.rounding, c.eps = native.ROUNDING[dec.rounding], cfg.eps
        c.token_table, c.position_table = dec.tok.data_ptr(), dec.pos.data_ptr()
        c.vocab, c.positions_count = cfg.vocab, cfg.target
        for i, Lr in enumerate(dec.layers):
            for k, name in enumerate(("qkv", "out", "cq", "cout", "fc1", "fc2")):
                c.linears[i][k] = Lr[name].handle
            for k, (ln, j) in enumerate((("ln1", 0), ("ln1", 1), ("ln2", 0), ("ln2", 1), ("ln3", 0), ("ln3", 1))):
                c.norms[i][k] = Lr[ln][j].data_ptr()
            c.self_k[i], c.self_v[i] = dec.self_k[i].data_ptr(), dec.self_v[i].data_ptr()
            c.cross_k[i], c.cross_v[i] = dec.cross_k[i].data_ptr(), dec.cross_v[i].data_ptr()
        c.head = dec.head.handle
        c.final_norm_weight, c.final_norm_bias = dec.lnf[0].data_ptr(), dec.lnf[1].data_ptr()
        sup = dec.suppressed.get("decode")
        self._sup = sup  # keep alive
        if sup is not None and sup.numel():
            c.suppressed, c.suppressed_count = sup.data_ptr(), sup.numel()
        c.tokens, c.positions, c.cross_length = tokens.data_ptr(), positions.data_ptr(), dec.cross_len.data_ptr()
        c.logits = logits.data_ptr() if logits is not None else None
        c.next_token, c.status = next_token.data_ptr(), dec.status.data_ptr()
        self.lib, self.dec = dec.lib, dec
        e = error_buffer()
        torch.cuda.synchronize(dec.device)
        h = self.lib.mstar_b200_decode_step_create(C.byref(c), e, len(e))
        if not h:
            raise native.NativeError("B200 decode step: " + e.value.decode(errors="replace"))
        self.handle = h

    def run(self):
        e = error_buffer()
        check(self.lib.mstar_b200_decode_step_run(self.handle, _stream(self.dec.device), e, len(e)), e,
              "B200 decode step")

    def close(self):
        if getattr(self, "handle", None):
            e = error_buffer()
            check(self.lib.mstar_b200_decode_step_close(self.handle, e, len(e)), e, "B200 decode step close")
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class GraphDecoder:
    """The whole greedy decode step captured once as a CUDA graph; replay feeds
    back its own next tokens (positions advance by one per step)."""

    def __init__(self, dec: WhisperDecoderB200, persistent: bool = False):
        self.dec = dec
        B, dev = dec.batch, dec.device
        self.tokens = torch.zeros(B, dtype=torch.int64, device=dev)
        self.positions = torch.zeros(B, dtype=torch.int64, device=dev)
        self.logits = torch.empty((B, dec.cfg.vocab), device=dev)
        self.next = torch.zeros(B, dtype=torch.int64, device=dev)
        self.graph = None
        # persistent: the step is one cooperative kernel instead of ~60 launches
        self.step = PersistentStep(dec, self.tokens, self.positions, self.logits, self.next) if persistent else None

    def _step(self):
        if self.step is not None:
            self.step.run()
        else:
            self.dec.decode_into(self.tokens, self.positions, self.logits, self.next)
        self.tokens.copy_(self.next)
        self.positions.add_(1)

    def capture(self):
        s = torch.cuda.Stream(self.dec.device)
        s.wait_stream(torch.cuda.current_stream(self.dec.device))
        saved = (self.tokens.clone(), self.positions.clone())
        with torch.cuda.stream(s):
            self._step()   # warm: first-call attribute setup happens outside capture
        torch.cuda.current_stream(self.dec.device).wait_stream(s)
        self.tokens.copy_(saved[0])
        self.positions.copy_(saved[1])
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph, stream=s):
            self._step()

    def run(self, steps: int):
        for _ in range(steps):
            self.graph.replay()
