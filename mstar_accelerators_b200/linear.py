"""Torch-facing wrappers of the block-quantized kernels.

``pack`` / ``quantize`` produce canonical ggml bytes on the device
(ggml-quants.c:113-147, :276-297; decoder.cpp:307-316, :816-842).
``BlockLinear`` is one prepared ``ggml_mul_mat(Q8_0|Q4_0 W, F32 x)`` node with
its fused epilogue (decoder.cpp:498-500, 563-588) and, on the same handle, the
greedy vocab readout (decoder.cpp:583-588, 686-696; cpu_q8/readout.c:30-54).
Every call is enqueued on the current torch CUDA stream; nothing here runs a
CPU computation in place of a kernel.
"""
from __future__ import annotations

import ctypes as C

import torch

from . import native
from .native import BIAS, GELU, GELU_ERF, RESIDUAL, check, error_buffer

Q8_BLOCK, Q4_BLOCK = 34, 18


def _stream(device=None) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def _nbytes(t: torch.Tensor) -> int:
    return t.numel() * t.element_size()


def _require_cuda(t: torch.Tensor, what: str, dtype=None) -> None:
    if t.device.type != "cuda":
        raise ValueError(f"{what} must be a CUDA tensor")
    if dtype is not None and t.dtype != dtype:
        raise ValueError(f"{what} must be {dtype}")


def block_bytes(fmt: str) -> int:
    return {"q8_0": Q8_BLOCK, "q4_0": Q4_BLOCK}[fmt]


def pack(weight: torch.Tensor, fmt: str = "q8_0", *, preround: bool = True, fused: bool = True) -> torch.Tensor:
    """Logical fp32 [rows, width] -> canonical ggml blocks (uint8 [rows, width/32*B]) on the device."""
    lib = native.require_capability()
    if weight.ndim != 2 or weight.shape[1] % 32:
        raise ValueError("packing needs a matrix with block-aligned width")
    w = weight.detach().to(device="cuda" if weight.device.type != "cuda" else weight.device,
                           dtype=torch.float32).contiguous()
    rows, width = w.shape
    out = torch.empty((rows, width // 32 * block_bytes(fmt)), dtype=torch.uint8, device=w.device)
    e = error_buffer()
    check(lib.mstar_b200_pack(native.FORMATS[fmt], w.data_ptr(), _nbytes(w), out.data_ptr(), _nbytes(out),
                              rows, width, int(preround), int(fused), _stream(w.device), e, len(e)),
          e, "B200 block packing")
    return out


def quantize(x: torch.Tensor, rounding: str = "arm") -> torch.Tensor:
    """fp32 [rows, k] -> Q8_0 activation blocks (q8cpu_quantize twin)."""
    lib = native.require_capability()
    _require_cuda(x, "activations", torch.float32)
    x = x.contiguous()
    rows, k = x.reshape(-1, x.shape[-1]).shape
    out = torch.empty((rows, k // 32 * Q8_BLOCK), dtype=torch.uint8, device=x.device)
    status = lib.mstar_b200_q8_quantize(x.data_ptr(), out.data_ptr(), _nbytes(out), rows, k,
                                        native.ROUNDING[rounding], _stream(x.device))
    if status:
        raise native.NativeError(f"B200 Q8_0 quantize failed with errno {status}")
    return out


def stage_rows(x: torch.Tensor, *, norm: tuple | None = None, rounding: str = "arm",
               out: torch.Tensor | None = None, status: torch.Tensor | None = None) -> torch.Tensor:
    """fp32 / fp16 rows [..., K] [-> LayerNorm] -> staged GEMM operand fp16(q * d) [rows, K]."""
    lib = native.require_capability()
    _require_cuda(x, "activations")
    if x.dtype not in (torch.float32, torch.float16):
        raise ValueError("staged rows are fp32 or fp16")
    k = x.shape[-1]
    x2 = x.reshape(-1, k)
    if x2.stride(-1) != 1:
        x2 = x2.contiguous()
    rows = x2.shape[0]
    if out is None:
        out = torch.empty((rows, k), dtype=torch.float16, device=x.device)
    if status is None:
        status = torch.zeros(1, dtype=torch.int32, device=x.device)
    lw, lb, eps = _norm(norm)
    e = error_buffer()
    check(lib.mstar_b200_stage_rows(x2.data_ptr(), native.ACT_F16 if x.dtype == torch.float16 else native.ACT_F32,
                                    x2.stride(0), rows, k, lw, lb, eps, out.data_ptr(), rows * k * 2,
                                    native.ROUNDING[rounding], status.data_ptr(), _stream(x.device), e, len(e)),
          e, "B200 row staging")
    return out


def stage_heads(attention: torch.Tensor, *, rounding: str = "arm", out: torch.Tensor | None = None,
                status: torch.Tensor | None = None) -> torch.Tensor:
    """Attention output bf16 [S, heads, n, D] (any strides over S, heads, n) -> the output
    projection's staged operand fp16(q * d) [S * n, heads * D] (row s * n + t: the heads of
    position t side by side), in one pass."""
    lib = native.require_capability()
    _require_cuda(attention, "attention output", torch.bfloat16)
    a = attention if attention.stride(-1) == 1 else attention.contiguous()
    S, H, n, D = a.shape
    if out is None:
        out = torch.empty((S * n, H * D), dtype=torch.float16, device=a.device)
    if status is None:
        status = torch.zeros(1, dtype=torch.int32, device=a.device)
    e = error_buffer()
    check(lib.mstar_b200_stage_heads(a.data_ptr(), S, H, n, D, a.stride(0), a.stride(1), a.stride(2),
                                     out.data_ptr(), out.numel() * 2, native.ROUNDING[rounding], status.data_ptr(),
                                     _stream(a.device), e, len(e)),
          e, "B200 attention staging")
    return out


def stage_conv(source: torch.Tensor, *, time_major: bool, stride: int, k_padded: int, rounding: str = "arm",
               out: torch.Tensor | None = None, status: torch.Tensor | None = None) -> torch.Tensor:
    """Convolution columns (kernel 3, padding 1) of fp32 [B, C, T] (or [B, T, C] when time_major),
    Q8_0-staged as fp16 [B * T_out, k_padded]."""
    lib = native.require_capability()
    _require_cuda(source, "convolution input", torch.float32)
    src = source.contiguous()
    if time_major:
        batch, time_in, channels = src.shape
    else:
        batch, channels, time_in = src.shape
    time_out = (time_in - 1) // stride + 1
    if out is None:
        out = torch.empty((batch * time_out, k_padded), dtype=torch.float16, device=src.device)
    if status is None:
        status = torch.zeros(1, dtype=torch.int32, device=src.device)
    e = error_buffer()
    check(lib.mstar_b200_stage_conv(src.data_ptr(), int(time_major), batch, channels, time_in, stride, k_padded,
                                    out.data_ptr(), batch * time_out * k_padded * 2, native.ROUNDING[rounding],
                                    status.data_ptr(), _stream(src.device), e, len(e)),
          e, "B200 convolution staging")
    return out


def layer_norm(x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor, eps: float = 1e-5,
               out: torch.Tensor | None = None) -> torch.Tensor:
    """ggml_norm(eps) * weight + bias over the last dimension of fp32 rows."""
    lib = native.require_capability()
    _require_cuda(x, "LayerNorm input", torch.float32)
    k = x.shape[-1]
    x2 = x.reshape(-1, k)
    if x2.stride(-1) != 1:
        x2 = x2.contiguous()
    if out is None:
        out = torch.empty(x.shape, dtype=torch.float32, device=x.device)
    o2 = out.reshape(-1, k)
    e = error_buffer()
    check(lib.mstar_b200_layer_norm(x2.data_ptr(), x2.stride(0), x2.shape[0], k, weight.data_ptr(), bias.data_ptr(),
                                    float(eps), o2.data_ptr(), o2.stride(0), _stream(x.device), e, len(e)),
          e, "B200 LayerNorm")
    return out


def categorical(logits: torch.Tensor, seeds: torch.Tensor, offsets: torch.Tensor, temperatures: torch.Tensor,
                out: torch.Tensor | None = None) -> torch.Tensor:
    """Positive-temperature categorical draws of fp32 logits [rows, vocab] (the reference's
    philox4x32-10-gumbel23-v1 operation): int64 seeds / offsets and fp32 temperatures per row;
    returns int64 tokens [rows], -1 for an invalid row (a NaN, nothing above -inf, or a
    temperature that is not positive and finite)."""
    lib = native.require_capability()
    _require_cuda(logits, "logits", torch.float32)
    if logits.ndim != 2 or logits.stride(1) != 1:
        raise ValueError("logits must be [rows, vocab] with unit column stride")
    rows, vocab = logits.shape
    for t, name, dt in ((seeds, "seeds", torch.int64), (offsets, "offsets", torch.int64),
                        (temperatures, "temperatures", torch.float32)):
        _require_cuda(t, name, dt)
        if t.shape != (rows,) or not t.is_contiguous():
            raise ValueError(f"{name} must be a contiguous [rows] tensor")
    if out is None:
        out = torch.empty(rows, dtype=torch.int64, device=logits.device)
    ws_bytes = int(lib.mstar_b200_categorical_workspace(rows))
    ws = torch.empty((ws_bytes + 15) // 16 * 4, dtype=torch.float32, device=logits.device)
    e = error_buffer()
    check(lib.mstar_b200_categorical(logits.data_ptr(), rows, vocab, logits.stride(0), seeds.data_ptr(),
                                     offsets.data_ptr(), temperatures.data_ptr(), out.data_ptr(), ws.data_ptr(),
                                     ws_bytes, _stream(logits.device), e, len(e)), e, "B200 categorical sampling")
    return out


def _rows(x: torch.Tensor, width: int) -> torch.Tensor:
    """[..., width] -> a 2-D view with unit inner stride and 16-byte aligned rows."""
    x2 = x.reshape(-1, width)
    if x2.stride(-1) != 1 or x2.stride(0) % 4 or x2.data_ptr() % 16:
        x2 = x2.contiguous()
    return x2


def _norm(norm):
    if norm is None:
        return None, None, 0.0
    weight, bias, eps = norm
    return weight.data_ptr(), bias.data_ptr(), float(eps)


class BlockLinear:
    """One prepared block-quantized linear on the current CUDA device."""

    def __init__(self, weight: torch.Tensor | None = None, *, blocks: torch.Tensor | None = None,
                 fmt: str = "q8_0", bias: torch.Tensor | None = None, rows: int | None = None,
                 width: int | None = None, preround: bool = True, fused: bool = True):
        self.lib = native.require_capability()
        if (weight is None) == (blocks is None):
            raise ValueError("give exactly one of a logical weight or canonical blocks")
        if weight is not None:
            rows, width = weight.shape
            blocks = pack(weight, fmt, preround=preround, fused=fused)
        elif rows is None or width is None:
            raise ValueError("canonical blocks need their logical rows and width")
        _require_cuda(blocks, "blocks", torch.uint8)
        blocks = blocks.contiguous()
        self.fmt, self.rows, self.width = fmt, int(rows), int(width)
        self.device = blocks.device
        bias_t = None
        if bias is not None:
            bias_t = bias.detach().to(device=self.device, dtype=torch.float32).contiguous()
            if bias_t.shape != (self.rows,):
                raise ValueError("bias shape differs from the weight rows")
        e = error_buffer()
        torch.cuda.current_stream(self.device).synchronize()
        handle = self.lib.mstar_b200_linear_create(native.FORMATS[fmt], blocks.data_ptr(), _nbytes(blocks),
                                                   self.rows, self.width,
                                                   bias_t.data_ptr() if bias_t is not None else None, e, len(e))
        if not handle:
            raise native.NativeError("B200 linear preparation: " + e.value.decode(errors="replace"))
        self.handle = handle
        self.has_bias = bias_t is not None
        self.bias_t = bias_t
        self.blocks = blocks  # canonical bytes stay available to callers (and tests)
        self.gemm_rows = 0
        self.readout_tiles = False

    # ggml_mul_mat + epilogue -------------------------------------------------
    def __call__(self, x: torch.Tensor, *, out: torch.Tensor | None = None, residual: torch.Tensor | None = None,
                 bias: bool = True, gelu: str | None = None, norm: tuple | None = None,
                 rounding: str = "arm", next_frags: "native.Q8Frags | None" = None) -> torch.Tensor:
        """ggml_mul_mat(W, [LayerNorm](x)) + epilogue; norm = (weight, bias, eps) fuses the LayerNorm.
        next_frags (another handle's frags(rows)) also quantizes the outputs for that handle's run_frags."""
        _require_cuda(x, "activations", torch.float32)
        lead = x.shape[:-1]
        x2 = _rows(x, self.width)
        m = x2.shape[0]
        if out is None:
            out = torch.empty((*lead, self.rows), dtype=torch.float32, device=x.device)
        o2 = out.reshape(-1, self.rows)
        flags = (BIAS if (bias and self.has_bias) else 0)
        flags |= {None: 0, "tanh": GELU, "erf": GELU_ERF}[gelu]
        r_ptr = None
        if residual is not None:
            r2 = residual.reshape(-1, self.rows)
            if r2.stride() != o2.stride():
                raise ValueError("residual layout differs from the output")
            flags |= RESIDUAL
            r_ptr = r2.data_ptr()
        lw, lb, eps = _norm(norm)
        e = error_buffer()
        if next_frags is not None:
            check(self.lib.mstar_b200_linear_run_q8out(self.handle, x2.data_ptr(), x2.stride(0), m, o2.data_ptr(),
                                                       o2.stride(0), r_ptr, flags, lw, lb, eps,
                                                       native.ROUNDING[rounding], C.byref(next_frags),
                                                       _stream(x.device), e, len(e)),
                  e, "B200 linear with fragment output")
            return out
        check(self.lib.mstar_b200_linear_run(self.handle, x2.data_ptr(), x2.stride(0), m, o2.data_ptr(), o2.stride(0),
                                             r_ptr, flags, lw, lb, eps, native.ROUNDING[rounding], _stream(x.device),
                                             e, len(e)),
              e, "B200 linear")
        return out

    def prepare_gemm(self, max_queries: int) -> None:
        """Enable the tcgen05 GEMM for calls of 64..max_queries rows (allocates and synchronises)."""
        e = error_buffer()
        check(self.lib.mstar_b200_linear_prepare_gemm(self.handle, self.blocks.data_ptr(), _nbytes(self.blocks),
                                                      int(max_queries), e, len(e)), e, "B200 GEMM preparation")
        self.gemm_rows = int(max_queries)

    def frags(self, queries: int, rounding: str = "arm") -> "native.Q8Frags":
        """Descriptor of this handle's Q8_0 activation fragments for `queries` (1..32) rows,
        for a producer that quantizes straight into them (attention with frags=)."""
        key = (int(queries), rounding)
        cache = self.__dict__.setdefault("_frags", {})
        if key not in cache:
            f = native.Q8Frags()
            e = error_buffer()
            check(self.lib.mstar_b200_linear_frags(self.handle, int(queries), native.ROUNDING[rounding],
                                                   C.byref(f), e, len(e)), e, "B200 fragment descriptor")
            cache[key] = f
        return cache[key]

    def run_frags(self, queries: int, *, out: torch.Tensor, residual: torch.Tensor | None = None, bias: bool = True,
                  gelu: str | None = None) -> torch.Tensor:
        """The decode GEMV + epilogue on fragments a producer wrote for `queries` rows."""
        o2 = out.reshape(-1, self.rows)
        flags = (BIAS if (bias and self.has_bias) else 0)
        flags |= {None: 0, "tanh": GELU, "erf": GELU_ERF}[gelu]
        r_ptr = None
        if residual is not None:
            r2 = residual.reshape(-1, self.rows)
            if r2.stride() != o2.stride():
                raise ValueError("residual layout differs from the output")
            flags |= RESIDUAL
            r_ptr = r2.data_ptr()
        e = error_buffer()
        check(self.lib.mstar_b200_linear_run_frags(self.handle, int(queries), o2.data_ptr(), o2.stride(0), r_ptr,
                                                   flags, _stream(out.device), e, len(e)), e, "B200 fragment GEMV")
        return out

    def prepare_readout(self) -> None:
        """Build the vocab-readout tile layout; later readout calls use the tile kernel (synchronises)."""
        if self.readout_tiles:
            return
        e = error_buffer()
        check(self.lib.mstar_b200_linear_prepare_readout(self.handle, self.blocks.data_ptr(), _nbytes(self.blocks),
                                                         e, len(e)), e, "B200 readout preparation")
        self.readout_tiles = True

    def gemm(self, staged: torch.Tensor, *, out: torch.Tensor | None = None, out_format: str = "f32",
             residual: torch.Tensor | None = None, residual_period: int = 0, segments: tuple[int, int] = (0, 0),
             bias: bool = True, gelu: str | None = None, rounding: str = "arm",
             status: torch.Tensor | None = None) -> torch.Tensor:
        """The prepared tcgen05 GEMM on a staged fp16 operand [rows, width].

        out_format: "f32", "f16" or "staged" (Q8_0-staged fp16, the next GEMM's operand).
        segments = (rows per segment, output rows per segment) places each segment's
        rows at the start of a padded output plane; residual_period repeats a residual
        table every that many rows."""
        if not self.gemm_rows:
            raise ValueError("prepare_gemm must run before gemm")
        _require_cuda(staged, "staged operand", torch.float16)
        if staged.ndim != 2 or staged.shape[1] != self.width or not staged.is_contiguous():
            raise ValueError("staged operand must be a contiguous [rows, width] fp16 matrix")
        rows = staged.shape[0]
        fmt = {"f32": native.OUT_F32, "f16": native.OUT_F16, "staged": native.OUT_STAGED}[out_format]
        seg, out_seg = segments
        out_rows = -(-rows // seg) * out_seg if seg else rows
        dtype = torch.float32 if out_format == "f32" else torch.float16
        if out is None:
            out = torch.empty((out_rows, self.rows), dtype=dtype, device=staged.device)
        o2 = out.reshape(-1, out.shape[-1])
        if o2.dtype != dtype or o2.stride(-1) != 1:
            raise ValueError("output dtype or layout differs from the output format")
        flags = (BIAS if (bias and self.has_bias) else 0)
        flags |= {None: 0, "tanh": GELU, "erf": GELU_ERF}[gelu]
        r_ptr, r_bytes, r_stride = None, 0, 0
        if residual is not None:
            r2 = residual.reshape(-1, residual.shape[-1])
            _require_cuda(r2, "residual", torch.float32)
            flags |= RESIDUAL
            r_rows = min(residual_period, rows) if residual_period else rows
            r_ptr, r_stride = r2.data_ptr(), r2.stride(0)
            r_bytes = ((r_rows - 1) * r_stride + self.rows) * 4
        if status is None:
            status = torch.zeros(1, dtype=torch.int32, device=staged.device)
        o_bytes = ((out_rows - 1) * o2.stride(0) + self.rows) * o2.element_size()
        e = error_buffer()
        check(self.lib.mstar_b200_linear_gemm(self.handle, staged.data_ptr(), rows * self.width * 2, rows,
                                              o2.data_ptr(), o_bytes, o2.stride(0), fmt, r_ptr, r_bytes, r_stride,
                                              int(residual_period), int(seg), int(out_seg), flags,
                                              native.ROUNDING[rounding], status.data_ptr(), _stream(staged.device),
                                              e, len(e)),
              e, "B200 GEMM")
        return out

    def gemm_push(self, staged: torch.Tensor, *, recv_ptrs: torch.Tensor, flag_ptrs: torch.Tensor, world: int,
                  rank: int, owner_rows: int, status: torch.Tensor) -> None:
        """Row-parallel partial product (fp32, no bias) of more than 128 staged rows, stored by
        the GEMM epilogue into the owning ranks' receive slots (row r -> owner r // owner_rows,
        slot ``rank``) with one arrival per 32 rows on the owner's counters.

        recv_ptrs / flag_ptrs: int64 device tensors of ``world`` device pointers (symmetric memory)."""
        if not self.gemm_rows:
            raise ValueError("prepare_gemm must run before gemm_push")
        _require_cuda(staged, "staged operand", torch.float16)
        if staged.ndim != 2 or staged.shape[1] != self.width or not staged.is_contiguous():
            raise ValueError("staged operand must be a contiguous [rows, width] fp16 matrix")
        rows = staged.shape[0]
        e = error_buffer()
        check(self.lib.mstar_b200_linear_gemm_push(self.handle, staged.data_ptr(), rows * self.width * 2, rows,
                                                   recv_ptrs.data_ptr(), flag_ptrs.data_ptr(), world, rank,
                                                   owner_rows, status.data_ptr(), _stream(staged.device), e, len(e)),
              e, "B200 pushed GEMM")

    def prepare_exact(self) -> None:
        """Lay the Q8_0 weights out for the exact int8-tensor-pipe GEMM (int8 quants + fp32 scales)."""
        if self.fmt != "q8_0":
            raise ValueError("the exact GEMM takes Q8_0 weights")
        if getattr(self, "_exact", None) is not None:
            return
        pad = int(self.lib.mstar_b200_q8_exact_pad(self.rows))
        wq = torch.empty((self.rows, self.width), dtype=torch.int8, device=self.device)
        ws = torch.zeros((self.width // 32, pad), dtype=torch.float32, device=self.device)
        e = error_buffer()
        check(self.lib.mstar_b200_q8_exact_weights(self.blocks.data_ptr(), _nbytes(self.blocks), self.rows, self.width,
                                                   wq.data_ptr(), ws.data_ptr(), _stream(self.device), e, len(e)),
              e, "B200 exact GEMM weights")
        self._exact = (wq, ws)

    def exact(self, x: torch.Tensor, *, out: torch.Tensor | None = None, bias: bool = True,
              rounding: str = "arm", status: torch.Tensor | None = None) -> torch.Tensor:
        """ggml_mul_mat(W, x) (+ bias) in ggml's generic block order for any row count: x's rows are
        Q8_0-quantized, every block's integer dot runs on the int8 tensor pipe and the blocks are
        rescaled and summed in order (bit-identical to the decode GEMV); slower than the fp16 GEMM."""
        self.prepare_exact()
        _require_cuda(x, "activations", torch.float32)
        x2 = _rows(x, self.width)
        m = x2.shape[0]
        if out is None:
            out = torch.empty((m, self.rows), dtype=torch.float32, device=x.device)
        if status is None:
            status = torch.zeros(1, dtype=torch.int32, device=x.device)
        xq = torch.empty((m, self.width), dtype=torch.int8, device=x.device)
        xs = torch.empty((m, self.width // 32), dtype=torch.float32, device=x.device)
        wq, ws = self._exact
        e = error_buffer()
        check(self.lib.mstar_b200_q8_exact_activations(x2.data_ptr(), x2.stride(0), m, self.width,
                                                       native.ROUNDING[rounding], xq.data_ptr(), xs.data_ptr(),
                                                       status.data_ptr(), _stream(x.device), e, len(e)),
              e, "B200 exact GEMM activations")
        check(self.lib.mstar_b200_gemm_q8_exact(xq.data_ptr(), xs.data_ptr(), m, wq.data_ptr(), ws.data_ptr(), self.rows,
                                                self.width, self.bias_t.data_ptr() if (bias and self.has_bias) else None,
                                                out.data_ptr(), out.stride(0), status.data_ptr(), _stream(x.device),
                                                e, len(e)),
              e, "B200 exact GEMM")
        return out

    def set_split(self, warps: int) -> None:
        """Force the K split (1, 2, 4, 8) or restore the automatic choice (0); results do not change."""
        e = error_buffer()
        check(self.lib.mstar_b200_linear_set_split(self.handle, warps, e, len(e)), e, "B200 split policy")

    def block_sums(self, x: torch.Tensor, rounding: str = "arm") -> torch.Tensor:
        """Exact int32 per-block dots [M, rows, width/32] of the same kernel path."""
        _require_cuda(x, "activations", torch.float32)
        x = _rows(x, self.width).contiguous()
        sums = torch.empty((x.shape[0], self.rows, self.width // 32), dtype=torch.int32, device=x.device)
        e = error_buffer()
        check(self.lib.mstar_b200_linear_block_sums(self.handle, x.data_ptr(), x.shape[0], sums.data_ptr(),
                                                    _nbytes(sums), native.ROUNDING[rounding], _stream(x.device),
                                                    e, len(e)), e, "B200 block sums")
        return sums

    def readout(self, x: torch.Tensor, suppressed: torch.Tensor | None = None, *, rounding: str = "arm",
                norm: tuple | None = None, logits: torch.Tensor | None = None, token: torch.Tensor | None = None,
                status: torch.Tensor | None = None):
        """Greedy readout of each row of x: (logits [M, rows], token int64 [M], status int32 [1])."""
        _require_cuda(x, "activations", torch.float32)
        x2 = _rows(x, self.width)
        m = x2.shape[0]
        dev = x.device
        logits = torch.empty((m, self.rows), dtype=torch.float32, device=dev) if logits is None else logits
        token = torch.empty((m,), dtype=torch.int64, device=dev) if token is None else token
        status = torch.empty((1,), dtype=torch.int32, device=dev) if status is None else status
        count, s_ptr = 0, None
        if suppressed is not None and suppressed.numel():
            _require_cuda(suppressed, "suppression list", torch.int64)
            suppressed = suppressed.contiguous()
            count, s_ptr = suppressed.numel(), suppressed.data_ptr()
        lw, lb, eps = _norm(norm)
        e = error_buffer()
        check(self.lib.mstar_b200_linear_readout(self.handle, x2.data_ptr(), x2.stride(0), m, logits.data_ptr(),
                                                 token.data_ptr(), status.data_ptr(), s_ptr, count, lw, lb, eps,
                                                 native.ROUNDING[rounding], _stream(dev), e, len(e)),
              e, "B200 readout")
        return logits, token, status

    def close(self) -> None:
        if getattr(self, "handle", None):
            e = error_buffer()
            check(self.lib.mstar_b200_linear_close(self.handle, e, len(e)), e, "B200 linear close")
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
