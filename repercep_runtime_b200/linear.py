"""FP8 GEMM and FP8 linears on the B200 tensor cores (librepercep_b200.so).

``fp8_gemm(A, B, a_scale, b_scale)`` is the reference's extension op
(kernels/hip/fp8_attn/binding.cpp:24-61, kernel fp8_gemm.hip:79-156): A (M, K)
and B (K, N) e4m3, C = bf16(A @ B * (a_scale * b_scale)) (M, N).  Same
argument checks, messages and meaning; the operands are torch.float8_e4m3fn,
the OCP encoding B200 computes in (the reference's gfx942 operands are
float8_e4m3fnuz).

``Fp8Linear`` is the FP8 DiT linear the reference plans for that GEMM
(docs/OPTIMIZATION.md:161-162): the weight quantized once per output channel,
the activations per token on every call, and one GEMM that applies both
scales and the bias in its epilogue.  Both quantizations use the attention
quantizer's steps with one scale group per row.

Torch allocates the outputs and supplies the current stream; the arithmetic
runs in the library, which has no fallback (a missing library raises).
"""

from __future__ import annotations

import torch

from . import _lib

FP8 = torch.float8_e4m3fn
_DTYPES = {torch.bfloat16: _lib.RP_DTYPE_BF16, torch.float16: _lib.RP_DTYPE_F16}


def _stream(t: torch.Tensor) -> int:
    return int(torch.cuda.current_stream(t.device).cuda_stream)


def _pitched(x: torch.Tensor, align: int) -> torch.Tensor:
    """``x`` (2-D, unit column stride) with rows starting on ``align``-element
    boundaries: ``x`` itself when it already has them, else a padded copy
    viewed back to x's shape."""
    rows, cols = x.shape
    if (
        x.stride(1) == 1
        and x.stride(0) >= cols
        and x.stride(0) % align == 0
        and x.data_ptr() % 16 == 0
    ):
        return x
    ld = max(align, (cols + align - 1) // align * align)
    buf = torch.empty(rows, ld, dtype=x.dtype, device=x.device)
    view = buf[:, :cols]
    view.copy_(x)
    return view


def fp8_gemm(A: torch.Tensor, B: torch.Tensor, a_scale: float, b_scale: float) -> torch.Tensor:
    """C (M, N) bf16 = bf16((A @ B) * (a_scale * b_scale)), A (M, K), B (K, N) e4m3."""
    if A.dim() != 2:
        raise RuntimeError("A must be 2-D")
    if B.dim() != 2:
        raise RuntimeError("B must be 2-D")
    if A.size(1) != B.size(0):
        raise RuntimeError("K mismatch")
    if not A.is_contiguous():
        raise RuntimeError("A must be contiguous")
    if not B.is_contiguous():
        raise RuntimeError("B must be contiguous")
    if A.dtype != FP8:
        raise RuntimeError("A must be float8_e4m3fn")
    if B.dtype != FP8:
        raise RuntimeError("B must be float8_e4m3fn")
    if not (A.is_cuda and B.is_cuda) or A.device != B.device:
        raise RuntimeError("A and B must be CUDA tensors on one device")
    M, K = (int(s) for s in A.shape)
    N = int(B.size(1))
    C = torch.empty(M, N, dtype=torch.bfloat16, device=A.device)
    if M == 0 or N == 0:
        return C
    a = _pitched(A, 16)
    b = _pitched(B, 16)
    lib = _lib.load()
    rc = lib.rp_fp8_gemm_ex(
        a.data_ptr(), a.stride(0), b.data_ptr(), b.stride(0), _lib.RP_B_KN,
        None, 0, float(a_scale), None, 0, float(b_scale), None,
        C.data_ptr(), C.stride(0), _lib.RP_DTYPE_BF16, M, N, K, _stream(C),
    )  # fmt: skip
    _lib.check("rp_fp8_gemm_ex", rc)
    return C


def gemm_ex(
    a8: torch.Tensor,
    b8: torch.Tensor,
    sa: torch.Tensor | float,
    sb: torch.Tensor | float,
    bias: torch.Tensor | None = None,
    out_dtype: torch.dtype = torch.bfloat16,
    b_layout: str = "nk",
    out: torch.Tensor | None = None,
) -> torch.Tensor:
    """C = out(acc * (sa[m] * sb[n]) + bias[n]) of e4m3 a8 (M, K) and b8.

    ``b_layout`` "nk": b8 is (N, K) (an nn.Linear weight); "kn": (K, N).
    ``sa`` / ``sb``: fp32 CUDA tensors of M / N per-row / per-column scales
    (or one element each), or Python floats.  ``bias``: (N,) in out_dtype."""
    if a8.dim() != 2 or b8.dim() != 2:
        raise ValueError("a8 and b8 must be 2-D")
    if a8.dtype != FP8 or b8.dtype != FP8:
        raise ValueError("a8 and b8 must be float8_e4m3fn")
    if out_dtype not in _DTYPES:
        raise ValueError(f"out_dtype must be bf16 or fp16, got {out_dtype}")
    if b_layout not in ("nk", "kn"):
        raise ValueError(f"unknown b_layout {b_layout!r}")
    M, K = (int(s) for s in a8.shape)
    N, Kb = (int(s) for s in b8.shape) if b_layout == "nk" else (int(b8.size(1)), int(b8.size(0)))
    if Kb != K:
        raise ValueError(f"K mismatch: a8 has {K}, b8 has {Kb}")
    dev = a8.device
    if out is None:
        out = torch.empty(M, N, dtype=out_dtype, device=dev)
    elif out.shape != (M, N) or out.dtype != out_dtype or out.stride(1) != 1:
        raise ValueError("out must be (M, N) of out_dtype with unit column stride")
    if M == 0 or N == 0:
        return out

    def scale_arg(s, n: int, name: str):  # type: ignore[no-untyped-def]
        if isinstance(s, torch.Tensor):
            if s.dtype != torch.float32 or s.device != dev:
                raise ValueError(f"{name} must be fp32 on {dev}")
            if s.numel() == 1:
                return s, 0, 1.0
            if s.numel() != n or s.dim() != 1:
                raise ValueError(f"{name} must hold 1 or {n} scales")
            return s, int(s.stride(0)), 1.0
        return None, 0, float(s)

    sa_t, sa_stride, a_scale = scale_arg(sa, M, "sa")
    sb_t, sb_stride, b_scale = scale_arg(sb, N, "sb")
    if bias is not None:
        if bias.dtype != out_dtype or bias.numel() != N or bias.device != dev:
            raise ValueError(f"bias must be ({N},) {out_dtype} on {dev}")
        bias = bias.contiguous()
    a = _pitched(a8, 16)
    b = _pitched(b8, 16)
    lib = _lib.load()
    rc = lib.rp_fp8_gemm_ex(
        a.data_ptr(), a.stride(0), b.data_ptr(), b.stride(0),
        _lib.RP_B_NK if b_layout == "nk" else _lib.RP_B_KN,
        sa_t.data_ptr() if sa_t is not None else None, sa_stride, a_scale,
        sb_t.data_ptr() if sb_t is not None else None, sb_stride, b_scale,
        bias.data_ptr() if bias is not None else None,
        out.data_ptr(), out.stride(0), _DTYPES[out_dtype], M, N, K, _stream(out),
    )  # fmt: skip
    _lib.check("rp_fp8_gemm_ex", rc)
    return out


def quantize_rows(x: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """Row-wise e4m3 quantization of a bf16/fp16 CUDA matrix (rows, cols).

    Returns (x8 (rows, cols) e4m3 with 16-byte row pitch, scales (rows,) fp32)."""
    if x.dim() != 2:
        raise ValueError("x must be 2-D")
    if x.dtype not in _DTYPES:
        raise ValueError(f"x must be bf16 or fp16, got {x.dtype}")
    if not x.is_cuda:
        raise ValueError("x must be a CUDA tensor")
    rows, cols = (int(s) for s in x.shape)
    xin = x
    if cols % 8 != 0:
        # zero columns change neither the row amax nor any dot product
        xin = torch.nn.functional.pad(x, (0, 8 - cols % 8))
    xin = _pitched(xin, 8)
    c8 = int(xin.size(1))
    ld = max(16, (c8 + 15) // 16 * 16)
    buf = torch.empty(rows, ld, dtype=FP8, device=x.device)
    scales = torch.empty(rows, dtype=torch.float32, device=x.device)
    if rows > 0:
        lib = _lib.load()
        rc = lib.rp_quant_fp8_rows(
            xin.data_ptr(), xin.stride(0), _DTYPES[x.dtype], rows, c8,
            buf.data_ptr(), ld, scales.data_ptr(), _stream(x),
        )  # fmt: skip
        _lib.check("rp_quant_fp8_rows", rc)
    return buf[:, :cols], scales


def fp8_linear(
    x: torch.Tensor, w8: torch.Tensor, w_scales: torch.Tensor, bias: torch.Tensor | None = None
) -> torch.Tensor:
    """y = x W^T + b with x quantized per token and W (N, K) per channel."""
    lead = x.shape[:-1]
    K = int(x.shape[-1])
    x8, xs = quantize_rows(x.reshape(-1, K))
    y = gemm_ex(x8, w8, xs, w_scales, bias, x.dtype, "nk")
    return y.reshape(*lead, int(w8.size(0)))


class Fp8Linear(torch.nn.Module):
    """Drop-in for an ``nn.Linear`` in a DiT block: e4m3 weight with one scale
    per output channel, per-token activation scales, bias fused in the GEMM."""

    def __init__(
        self, weight_fp8: torch.Tensor, weight_scales: torch.Tensor, bias: torch.Tensor | None
    ) -> None:
        super().__init__()
        self.out_features, self.in_features = (int(s) for s in weight_fp8.shape)
        self.register_buffer("weight_fp8", weight_fp8)
        self.register_buffer("weight_scales", weight_scales)
        self.register_buffer("bias", bias)

    @classmethod
    def from_linear(cls, linear: torch.nn.Linear) -> Fp8Linear:
        w = linear.weight.detach()
        if not w.is_cuda or w.dtype not in _DTYPES:
            raise ValueError("the linear's weight must be a bf16/fp16 CUDA tensor")
        w8, ws = quantize_rows(w)
        b = linear.bias.detach() if linear.bias is not None else None
        return cls(w8, ws, b)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        bias = self.bias.to(x.dtype) if self.bias is not None else None
        return fp8_linear(x, self.weight_fp8, self.weight_scales, bias)

    def extra_repr(self) -> str:
        return f"in_features={self.in_features}, out_features={self.out_features}, e4m3"


def gemm_qkv_quant(
    x8: torch.Tensor,
    w8: torch.Tensor,
    sa: torch.Tensor | float,
    sb: torch.Tensor | float,
    heads: int,
    seq_len: int,
    bias: torch.Tensor | None = None,
) -> list:
    """The QKV projection with the attention quantizer fused into its epilogue.

    ``x8`` (B*S, K) e4m3 activations, B batches of ``seq_len`` tokens;
    ``w8`` (3*heads*128, K) e4m3, the stacked Q, K, V projection weights
    (head-major inside each); ``sa`` / ``sb`` per-token / per-channel fp32
    scales (or floats); ``bias`` (3*heads*128,) bf16 or None.  Returns
    ``ops.Quantized`` q, k, v: (B, heads, S, 128) e4m3 with per-128-token-block
    scales, ready for ``ops.attention_fp8_quantized``.  Bit for bit the
    per-block ``ops.quantize_fp8`` of the bf16 ``gemm_ex`` output viewed as
    (B, S, 3, heads, 128) (the reference quantizes right before its kernel,
    kernels/triton_kernels/fp8_flash_attn_hopper.py:474-480); the bf16
    projection output is never written.
    """
    from . import ops

    if x8.dim() != 2 or w8.dim() != 2:
        raise ValueError("x8 and w8 must be 2-D")
    if x8.dtype != FP8 or w8.dtype != FP8:
        raise ValueError("x8 and w8 must be float8_e4m3fn")
    M, K = (int(s) for s in x8.shape)
    N = 3 * heads * 128
    if heads <= 0 or seq_len <= 0 or M % seq_len != 0:
        raise ValueError(f"{M} rows are not whole batches of seq_len={seq_len}")
    if tuple(w8.shape) != (N, K):
        raise ValueError(f"w8 must be ({N}, {K}) for {heads} heads of 128, got {tuple(w8.shape)}")
    B = M // seq_len
    dev = x8.device

    def scale_arg(s, n: int, name: str):  # type: ignore[no-untyped-def]
        if isinstance(s, torch.Tensor):
            if s.dtype != torch.float32 or s.device != dev:
                raise ValueError(f"{name} must be fp32 on {dev}")
            if s.numel() == 1:
                return s, 0, 1.0
            if s.numel() != n or s.dim() != 1:
                raise ValueError(f"{name} must hold 1 or {n} scales")
            return s, int(s.stride(0)), 1.0
        return None, 0, float(s)

    sa_t, sa_stride, a_scale = scale_arg(sa, M, "sa")
    sb_t, sb_stride, b_scale = scale_arg(sb, N, "sb")
    if bias is not None:
        if bias.dtype != torch.bfloat16 or bias.numel() != N or bias.device != dev:
            raise ValueError(f"bias must be ({N},) bf16 on {dev}")
        bias = bias.contiguous()
    nblk = (seq_len + ops.BLOCK - 1) // ops.BLOCK
    outs = [torch.empty((B, heads, seq_len, 128), dtype=FP8, device=dev) for _ in range(3)]
    scales = [torch.empty((B * heads, nblk), dtype=torch.float32, device=dev) for _ in range(3)]
    a = _pitched(x8, 16)
    w = _pitched(w8, 16)
    lib = _lib.load()
    rc = lib.rp_fp8_gemm_qkv_quant(
        a.data_ptr(), a.stride(0), w.data_ptr(), w.stride(0),
        sa_t.data_ptr() if sa_t is not None else None, sa_stride, a_scale,
        sb_t.data_ptr() if sb_t is not None else None, sb_stride, b_scale,
        bias.data_ptr() if bias is not None else None, B, seq_len, heads, K,
        outs[0].data_ptr(), outs[1].data_ptr(), outs[2].data_ptr(),
        scales[0].data_ptr(), scales[1].data_ptr(), scales[2].data_ptr(), _stream(outs[0]),
    )  # fmt: skip
    _lib.check("rp_fp8_gemm_qkv_quant", rc)
    return [ops.Quantized(o, s, ops.SCALE_PER_BLOCK128, 128) for o, s in zip(outs, scales)]


def qkv_projection_fp8(
    x: torch.Tensor, w8: torch.Tensor, ws: torch.Tensor, heads: int, bias: torch.Tensor | None = None
) -> list:
    """bf16 hidden states x (B, S, hidden) -> attention-ready e4m3 q, k, v:
    per-token activation quantize, then the QKV GEMM with the per-block
    quantizer in its epilogue (``gemm_qkv_quant``)."""
    if x.dim() != 3:
        raise ValueError("x must be (B, S, hidden)")
    B, S, K = (int(s) for s in x.shape)
    x8, xs = quantize_rows(x.reshape(B * S, K))
    return gemm_qkv_quant(x8, w8, xs, ws, heads, S, bias)
