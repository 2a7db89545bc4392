"""Torch-facing wrappers of the C ABI, plus the `repercep_b200::*` custom ops.

Torch only allocates buffers and provides the current stream here; all the
arithmetic runs in librepercep_b200.so.  Layout names follow the reference:
"bhsd" is (batch, heads, seq, head_dim) (``attention/types.py:22-40``),
"bshd" is the diffusers layout (``attention/diffusers_backend.py:264-267``).
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import torch

from . import _lib

FP8 = torch.float8_e4m3fn
BLOCK = 128

SCALE_PER_BH = _lib.RP_SCALE_PER_BH
SCALE_PER_BLOCK128 = _lib.RP_SCALE_PER_BLOCK128
P_E4M3 = _lib.RP_P_E4M3
P_E4M3_HILO = _lib.RP_P_E4M3_HILO


def _stream(t: torch.Tensor) -> int:
    return int(torch.cuda.current_stream(t.device).cuda_stream)


def _require_cuda(t: torch.Tensor, name: str, dtype: torch.dtype) -> None:
    if not t.is_cuda:
        raise ValueError(f"{name} must be a CUDA tensor")
    if t.dtype != dtype:
        raise ValueError(f"{name} must be {dtype}, got {t.dtype}")


def bhsd_strides(x: torch.Tensor, layout: str) -> tuple[int, int, int, int]:
    """Element strides of x indexed as (b, h, s, d)."""
    if layout == "bhsd":
        return (x.stride(0), x.stride(1), x.stride(2), x.stride(3))
    if layout == "bshd":
        return (x.stride(0), x.stride(2), x.stride(1), x.stride(3))
    raise ValueError(f"unknown layout {layout!r}")


def bhsd_shape(x: torch.Tensor, layout: str) -> tuple[int, int, int, int]:
    if layout == "bhsd":
        b, h, s, d = x.shape
    elif layout == "bshd":
        b, s, h, d = x.shape
    else:
        raise ValueError(f"unknown layout {layout!r}")
    return int(b), int(h), int(s), int(d)


@dataclass
class Quantized:
    """An e4m3 tensor (B*H, S, R) contiguous, viewed as (B, H, S, R), with scales.

    ``R`` is the row width in bytes: the head dim ``d``, or 128 for d = 32 / 64
    (rows zero-padded, the layout the attention kernel reads)."""

    data: torch.Tensor
    scales: torch.Tensor
    scale_mode: int
    d: int = 0

    def __post_init__(self) -> None:
        if self.d == 0:
            self.d = int(self.data.shape[-1])


_DTYPES = {torch.bfloat16: _lib.RP_DTYPE_BF16, torch.float16: _lib.RP_DTYPE_F16}


def _bh_phase(phase: int, xs, partials: torch.Tensor, layout: str, row_bytes: int | None):  # type: ignore[no-untyped-def]
    lib = _lib.load()
    B, H, S, D = bhsd_shape(xs[0], layout)
    row = D if row_bytes is None else int(row_bytes)
    dtype = xs[0].dtype
    if dtype not in _DTYPES:
        raise ValueError(f"inputs must be bf16 or fp16, got {dtype}")
    nblk = (S + BLOCK - 1) // BLOCK
    if partials.dtype != torch.int32 or partials.dim() != 3 or tuple(partials.shape[:2]) != (len(xs), B * H):
        raise ValueError(f"partials must be int32 ({len(xs)}, {B * H}, npart)")
    npart = int(partials.shape[2])
    if npart < nblk or not partials.is_contiguous():
        raise ValueError(f"partials need >= ceil(S/128) = {nblk} contiguous slots per row")
    outs, scales, strides = [], [], []
    for i, x in enumerate(xs):
        _require_cuda(x, f"x[{i}]", dtype)
        if bhsd_shape(x, layout) != (B, H, S, D):
            raise ValueError("all tensors must share one shape")
        if phase == _lib.RP_QUANT_PHASE_APPLY:
            outs.append(torch.empty((B, H, S, row), dtype=FP8, device=x.device))
            scales.append(torch.empty((B * H,), dtype=torch.float32, device=x.device))
        strides.extend(bhsd_strides(x, layout))
    apply = phase == _lib.RP_QUANT_PHASE_APPLY  # the amax phase takes no outputs
    rc = lib.rp_quant_fp8_e4m3_bh_phase(
        phase, len(xs), _lib.ptr_array(x.data_ptr() for x in xs), _lib.i64_array(strides),
        B, H, S, D, _DTYPES[dtype], partials.data_ptr(), npart,
        _lib.ptr_array(o.data_ptr() for o in outs) if apply else None, row,
        _lib.ptr_array(s.data_ptr() for s in scales) if apply else None, _stream(xs[0]),
    )  # fmt: skip
    _lib.check("rp_quant_fp8_e4m3_bh_phase", rc)
    return [Quantized(o, s, SCALE_PER_BH, D) for o, s in zip(outs, scales)]


def quantize_fp8_bh_partials(xs, npart: int | None = None, layout: str = "bhsd") -> torch.Tensor:  # type: ignore[no-untyped-def]
    """Phase 1 of the per-(b,h) quantizer for 1-3 tensors of one shape: the
    |x| max (bit patterns) of every 128-token chunk, as an int32 (n, B*H,
    npart) array with the slots past ceil(S/128) zero."""
    if not 1 <= len(xs) <= 3:
        raise ValueError("takes 1 to 3 tensors")
    B, H, S, _ = bhsd_shape(xs[0], layout)
    nblk = (S + BLOCK - 1) // BLOCK
    partials = torch.zeros((len(xs), B * H, nblk if npart is None else int(npart)), dtype=torch.int32,
                           device=xs[0].device)
    _bh_phase(_lib.RP_QUANT_PHASE_AMAX, xs, partials, layout, None)
    return partials


def quantize_fp8_bh_apply(xs, partials: torch.Tensor, layout: str = "bhsd",  # type: ignore[no-untyped-def]
                          row_bytes: int | None = None) -> list[Quantized]:
    """Phase 2: per-(b,h) scales from the max of each row of ``partials``
    (this tensor's chunks, or every rank's after an all-reduce MAX), then the
    quantize -- ``quantize_fp8``'s per-(b,h) bytes and scales."""
    return _bh_phase(_lib.RP_QUANT_PHASE_APPLY, xs, partials, layout, row_bytes)


def quantize_fp8_bh_phased(
    xs: list[torch.Tensor] | tuple[torch.Tensor, ...],
    combine,  # type: ignore[no-untyped-def]
    npart: int | None = None,
    layout: str = "bhsd",
    row_bytes: int | None = None,
) -> list[Quantized]:
    """Per-(b,h) quantize with ``combine(partials)`` between its two phases
    (``rp_quant_fp8_e4m3_bh_phase``): ``combine`` may fold other devices'
    partial maxima into the int32 array in place (an all-reduce MAX over the
    ranks a sequence is split across), so the scales are those of the whole
    sequence.  With a no-op ``combine`` this is ``quantize_fp8`` per-(b,h)."""
    partials = quantize_fp8_bh_partials(xs, npart, layout)
    combine(partials)
    return quantize_fp8_bh_apply(xs, partials, layout, row_bytes)


def per_block_view(q: Quantized) -> Quantized:
    """A per-(b,h) ``Quantized`` with its scale repeated for every 128-token
    block: the per-block kernels then compute exactly what the per-(b,h) ones
    do (every block of a (b,h) reads the same scale)."""
    if q.scale_mode == SCALE_PER_BLOCK128:
        return q
    S = int(q.data.shape[2])
    nblk = (S + BLOCK - 1) // BLOCK
    return Quantized(q.data, q.scales.reshape(-1, 1).expand(-1, nblk).contiguous(), SCALE_PER_BLOCK128, q.d)


def attention_row_bytes(head_dim: int) -> int:
    """e4m3 row width the attention kernel reads for ``head_dim``."""
    return 128 if head_dim <= 128 else head_dim


def quantize_fp8(
    xs: list[torch.Tensor] | tuple[torch.Tensor, ...],
    scale_mode: int = SCALE_PER_BH,
    layout: str = "bhsd",
    row_bytes: int | None = None,
) -> list[Quantized]:
    """Quantise 1-3 bf16 or fp16 tensors of one shape in a single native call.

    Per-(b,h) mode reproduces ``_per_bh_scale`` + ``_quantize`` of the
    reference (``kernels/triton_kernels/fp8_flash_attn_hopper.py:374-398``)
    bit for bit, for either input dtype; per-block mode applies the same
    formula to every 128-token block of each (b,h).  ``row_bytes`` (default D)
    widens the output rows with zero bytes.
    """
    if not 1 <= len(xs) <= 3:
        raise ValueError("quantize_fp8 takes 1 to 3 tensors")
    lib = _lib.load()
    B, H, S, D = bhsd_shape(xs[0], layout)
    row = D if row_bytes is None else int(row_bytes)
    dtype = xs[0].dtype
    if dtype not in _DTYPES:
        raise ValueError(f"inputs must be bf16 or fp16, got {dtype}")
    nblk = (S + BLOCK - 1) // BLOCK
    outs, scales, strides = [], [], []
    for i, x in enumerate(xs):
        _require_cuda(x, f"x[{i}]", dtype)
        if bhsd_shape(x, layout) != (B, H, S, D):
            raise ValueError("all tensors must share one shape")
        outs.append(torch.empty((B, H, S, row), dtype=FP8, device=x.device))
        shape = (B * H,) if scale_mode == SCALE_PER_BH else (B * H, nblk)
        scales.append(torch.empty(shape, dtype=torch.float32, device=x.device))
        strides.extend(bhsd_strides(x, layout))
    ws_bytes = _lib._c_size_t(0)
    _lib.check(
        "rp_quant_workspace_bytes",
        lib.rp_quant_workspace_bytes(len(xs), B, H, S, D, scale_mode, ws_bytes),
    )
    ws = None
    if ws_bytes.value:
        ws = torch.empty(ws_bytes.value, dtype=torch.uint8, device=xs[0].device)
    rc = lib.rp_quant_fp8_e4m3_ex(
        len(xs),
        _lib.ptr_array(x.data_ptr() for x in xs),
        _lib.i64_array(strides),
        B,
        H,
        S,
        D,
        _DTYPES[dtype],
        scale_mode,
        _lib.ptr_array(o.data_ptr() for o in outs),
        row,
        _lib.ptr_array(s.data_ptr() for s in scales),
        ws.data_ptr() if ws is not None else None,
        ws_bytes.value,
        _stream(xs[0]),
    )
    _lib.check("rp_quant_fp8_e4m3_ex", rc)
    return [Quantized(o, s, scale_mode, D) for o, s in zip(outs, scales)]


def attention_fp8_quantized(
    q: Quantized,
    k: Quantized,
    v: Quantized,
    *,
    causal: bool = False,
    scale: float | None = None,
    p_mode: int = P_E4M3,
    out: torch.Tensor | None = None,
    out_layout: str = "bhsd",
    out_dtype: torch.dtype = torch.bfloat16,
) -> torch.Tensor:
    """FP8 attention on already-quantised operands; bf16 (or fp16) output."""
    lib = _lib.load()
    B, H, Sq, row = q.data.shape
    D = q.d
    Skv = k.data.shape[2]
    if k.data.shape != v.data.shape or k.data.shape[:2] != (B, H) or k.data.shape[3] != row:
        raise ValueError("q, k, v shapes are inconsistent")
    if not (q.d == k.d == v.d):
        raise ValueError("q, k, v must share a head dim")
    if not (q.scale_mode == k.scale_mode == v.scale_mode):
        raise ValueError("q, k, v must share a scale mode")
    if out is None:
        shape = (B, H, Sq, D) if out_layout == "bhsd" else (B, Sq, H, D)
        out = torch.empty(shape, dtype=out_dtype, device=q.data.device)
    if out.dtype not in _DTYPES:
        raise ValueError(f"out must be bf16 or fp16, got {out.dtype}")
    _require_cuda(out, "out", out.dtype)
    rc = lib.rp_attn_fp8_fwd_ex(
        q.data.data_ptr(),
        k.data.data_ptr(),
        v.data.data_ptr(),
        q.scales.data_ptr(),
        k.scales.data_ptr(),
        v.scales.data_ptr(),
        q.scale_mode,
        B,
        H,
        Sq,
        Skv,
        D,
        row,
        float(scale) if scale is not None else 0.0,
        1 if causal else 0,
        p_mode,
        out.data_ptr(),
        _lib.i64_array(bhsd_strides(out, out_layout)),
        _DTYPES[out.dtype],
        _stream(q.data),
    )
    _lib.check("rp_attn_fp8_fwd_ex", rc)
    return out


def fp8_attention(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    *,
    causal: bool = False,
    scale: float | None = None,
    scale_mode: int = SCALE_PER_BH,
    p_mode: int = P_E4M3,
    layout: str = "bhsd",
    out: torch.Tensor | None = None,
) -> torch.Tensor:
    """Quantise Q/K/V (one native call) and run FP8 attention (one more).

    Same contract as the reference's ``fp8_flash_attention``
    (``fp8_flash_attn_hopper.py:432-586``): bf16 or fp16 in, D in
    {32, 64, 128, 256}, default scale 1/sqrt(D), output in the query's dtype
    and layout.
    """
    qshape, kshape = bhsd_shape(q, layout), bhsd_shape(k, layout)
    if k.shape != v.shape or qshape[:2] != kshape[:2] or qshape[3] != kshape[3]:
        raise ValueError("q, k, v must share batch, heads and head_dim; k and v one shape")
    if not (q.dtype == k.dtype == v.dtype):
        raise ValueError("q, k, v must share a dtype")
    row = attention_row_bytes(qshape[3])
    if q.shape == k.shape:
        qq, kq, vq = quantize_fp8((q, k, v), scale_mode=scale_mode, layout=layout, row_bytes=row)
    else:  # cross-length attention: one quantize call for Q, one for K and V
        (qq,) = quantize_fp8((q,), scale_mode=scale_mode, layout=layout, row_bytes=row)
        kq, vq = quantize_fp8((k, v), scale_mode=scale_mode, layout=layout, row_bytes=row)
    return attention_fp8_quantized(
        qq, kq, vq, causal=causal, scale=scale, p_mode=p_mode, out=out, out_layout=layout,
        out_dtype=q.dtype,
    )


def attention_fp8_chunked(
    q: Quantized,
    k_chunks: torch.Tensor,
    v_chunks: torch.Tensor,
    k_scales: torch.Tensor,
    v_scales: torch.Tensor,
    *,
    last_rows: int,
    scale: float | None = None,
    p_mode: int = P_E4M3,
    out: torch.Tensor | None = None,
    out_layout: str = "bhsd",
) -> torch.Tensor:
    """Attention of local queries over K/V gathered from several ranks.

    ``k_chunks``/``v_chunks``: e4m3 (n_chunks, B*H, chunk_rows, D); scales
    (n_chunks, B*H, chunk_rows/128).  Chunk i holds chunk_rows valid rows,
    except the last, which holds ``last_rows``.
    """
    lib = _lib.load()
    if q.scale_mode != SCALE_PER_BLOCK128:
        raise ValueError("chunked attention uses per-block scales")
    B, H, Sq, D = q.data.shape
    n_chunks, bh, chunk_rows, dk = k_chunks.shape
    if bh != B * H or dk != D or v_chunks.shape != k_chunks.shape:
        raise ValueError("chunk shapes are inconsistent with q")
    if out is None:
        shape = (B, H, Sq, D) if out_layout == "bhsd" else (B, Sq, H, D)
        out = torch.empty(shape, dtype=torch.bfloat16, device=q.data.device)
    rc = lib.rp_attn_fp8_fwd_chunked(
        q.data.data_ptr(),
        k_chunks.data_ptr(),
        v_chunks.data_ptr(),
        q.scales.data_ptr(),
        k_scales.data_ptr(),
        v_scales.data_ptr(),
        B,
        H,
        Sq,
        n_chunks,
        chunk_rows,
        int(last_rows),
        D,
        float(scale) if scale is not None else 0.0,
        p_mode,
        out.data_ptr(),
        _lib.i64_array(bhsd_strides(out, out_layout)),
        _stream(q.data),
    )
    _lib.check("rp_attn_fp8_fwd_chunked", rc)
    return out


def prefix_decode_fp8_quantized(
    q: Quantized,
    k_prefix: Quantized,
    v_prefix: Quantized,
    k_suffix: Quantized,
    v_suffix: Quantized,
    *,
    candidates: int,
    tokens: int,
    scale: float | None = None,
    p_mode: int = P_E4M3,
    out: torch.Tensor | None = None,
) -> torch.Tensor:
    """Shared-prefix candidate decode on quantised operands (per-block scales).

    q/k_suffix/v_suffix hold (1, H, C*T, D); k_prefix/v_prefix (1, H, P, D).
    Returns bf16 (C*T, H, D).
    """
    lib = _lib.load()
    _, H, rows, D = q.data.shape
    P = k_prefix.data.shape[2]
    if rows != candidates * tokens:
        raise ValueError("q rows must equal candidates * tokens")
    for t in (q, k_prefix, v_prefix, k_suffix, v_suffix):
        if t.scale_mode != SCALE_PER_BLOCK128:
            raise ValueError("prefix decode uses per-block scales")
    if out is None:
        out = torch.empty((rows, H, D), dtype=torch.bfloat16, device=q.data.device)
    rc = lib.rp_attn_fp8_prefix_decode(
        q.data.data_ptr(),
        k_prefix.data.data_ptr(),
        v_prefix.data.data_ptr(),
        k_suffix.data.data_ptr(),
        v_suffix.data.data_ptr(),
        q.scales.data_ptr(),
        k_prefix.scales.data_ptr(),
        v_prefix.scales.data_ptr(),
        k_suffix.scales.data_ptr(),
        v_suffix.scales.data_ptr(),
        candidates,
        tokens,
        P,
        H,
        D,
        float(scale) if scale is not None else 0.0,
        p_mode,
        out.data_ptr(),
        _lib.i64_array((out.stride(0), out.stride(1), out.stride(2))),
        _stream(q.data),
    )
    _lib.check("rp_attn_fp8_prefix_decode", rc)
    return out


def default_scale(head_dim: int) -> float:
    return 1.0 / math.sqrt(head_dim)


# ------------------------------------------------------------ custom ops
@torch.library.custom_op("repercep_b200::fp8_attention", mutates_args=())
def fp8_attention_op(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    causal: bool = False,
    scale: float = 0.0,
    scale_mode: int = SCALE_PER_BH,
    p_mode: int = P_E4M3,
) -> torch.Tensor:
    """``torch.ops.repercep_b200.fp8_attention`` — (B,H,S,D) bf16 or fp16 in/out."""
    return fp8_attention(
        q,
        k,
        v,
        causal=causal,
        scale=scale if scale > 0 else None,
        scale_mode=scale_mode,
        p_mode=p_mode,
    )


@fp8_attention_op.register_fake
def _fp8_attention_fake(q, k, v, causal=False, scale=0.0, scale_mode=0, p_mode=0):  # type: ignore[no-untyped-def]
    return torch.empty_like(q)


@torch.library.custom_op("repercep_b200::fp8_attention_bshd", mutates_args=())
def fp8_attention_bshd_op(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    causal: bool = False,
    scale: float = 0.0,
    scale_mode: int = SCALE_PER_BH,
    p_mode: int = P_E4M3,
) -> torch.Tensor:
    """``torch.ops.repercep_b200.fp8_attention_bshd`` — diffusers (B,S,H,D) bf16 or fp16 in/out."""
    return fp8_attention(
        q,
        k,
        v,
        causal=causal,
        scale=scale if scale > 0 else None,
        scale_mode=scale_mode,
        p_mode=p_mode,
        layout="bshd",
    )


@fp8_attention_bshd_op.register_fake
def _fp8_attention_bshd_fake(q, k, v, causal=False, scale=0.0, scale_mode=0, p_mode=0):  # type: ignore[no-untyped-def]
    return torch.empty_like(q)
