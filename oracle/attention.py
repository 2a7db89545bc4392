"""FP8 attention semantics, restated in numpy.  Test infrastructure only.

Three functions:

``attention_dequant``
    fp32 softmax attention over the *dequantised* e4m3 inputs — the oracle the
    accuracy tolerance (max-abs 2e-2, cosine >= 0.999) is stated against.
``reference_tile_loop``
    the reference kernel's algorithm, tile by tile
    (kernels/triton_kernels/fp8_flash_attn_hopper.py:240-338): qk = (q8 k8^T)
    * sm_scale * q_scale * k_scale (:275, :292-293), causal / tail masks
    (:296-302), online max/sum with natural exp (:305-311), P quantised as
    e4m3(p * 448) (:322) and accumulated with v_scale / 448 (:323-327),
    acc / l (:332).  Per-(b,h) scales only, as in the reference.
``prefix_decode_dequant``
    shared-prefix candidate decode: candidate c's token i attends to the whole
    prefix and to suffix tokens 0..i of candidate c (the semantics the
    reference obtains by expanding the prompt per candidate,
    scripts/run_vla_openvla_gpu.py:174-186).

e4m3 operands are (B*H, S, D) uint8 arrays; scales as produced by
``oracle.quantize`` ((B*H,) or (B*H, nblk)).
"""

from __future__ import annotations

import numpy as np

from .fp8 import e4m3_decode, e4m3_encode
from .quantize import expand_scales


def dequant(x8: np.ndarray, scales: np.ndarray) -> np.ndarray:
    """(BH, S, D) e4m3 bytes -> fp32 values."""
    BH, S, D = x8.shape
    return e4m3_decode(x8) * expand_scales(scales, S)[:, :, None]


def softmax_attention(
    q: np.ndarray,
    k: np.ndarray,
    v: np.ndarray,
    sm_scale: float,
    causal: bool = False,
    mask: np.ndarray | None = None,
) -> np.ndarray:
    """fp32 attention of (M, D) queries against (N, D) keys/values (float64 math)."""
    s = (q.astype(np.float64) @ k.astype(np.float64).T) * sm_scale
    if causal:
        rows = np.arange(q.shape[0])[:, None]
        cols = np.arange(k.shape[0])[None, :]
        s = np.where(cols <= rows, s, -np.inf)
    if mask is not None:
        s = np.where(mask, s, -np.inf)
    s = s - s.max(axis=1, keepdims=True)
    p = np.exp(s)
    return ((p @ v.astype(np.float64)) / p.sum(axis=1, keepdims=True)).astype(np.float32)


def attention_dequant(
    q8: np.ndarray,
    k8: np.ndarray,
    v8: np.ndarray,
    qs: np.ndarray,
    ks: np.ndarray,
    vs: np.ndarray,
    sm_scale: float,
    causal: bool = False,
    bh_index: list[int] | None = None,
    rows: np.ndarray | None = None,
) -> np.ndarray:
    """fp32 attention over dequantised inputs.

    Returns (len(bh_index), len(rows), D); all (b,h) and rows by default.
    Query rows are independent given the full K/V, so sampled rows are exact.
    """
    BH, Sq, D = q8.shape
    bh_index = list(range(BH)) if bh_index is None else list(bh_index)
    rows = np.arange(Sq) if rows is None else np.asarray(rows)
    out = np.empty((len(bh_index), len(rows), D), dtype=np.float32)
    for n, bh in enumerate(bh_index):
        qd = dequant(q8[bh : bh + 1], qs[bh : bh + 1])[0][rows]
        kd = dequant(k8[bh : bh + 1], ks[bh : bh + 1])[0]
        vd = dequant(v8[bh : bh + 1], vs[bh : bh + 1])[0]
        if causal:
            cols = np.arange(kd.shape[0])[None, :]
            mask = cols <= rows[:, None]
            out[n] = softmax_attention(qd, kd, vd, sm_scale, mask=mask)
        else:
            out[n] = softmax_attention(qd, kd, vd, sm_scale)
    return out


def reference_tile_loop(
    q8: np.ndarray,
    k8: np.ndarray,
    v8: np.ndarray,
    qs: np.ndarray,
    ks: np.ndarray,
    vs: np.ndarray,
    sm_scale: float,
    causal: bool = False,
    block_n: int = 128,
    fp8_max: float = 448.0,
    rescale_tau: float = 0.0,
    rescale_group: int = 32,
) -> np.ndarray:
    """The reference kernel's FA-2 loop in fp32; returns (BH, Sq, D) fp32.

    ``rescale_tau`` = 0 is the reference loop.  A positive value models the
    B200 kernel's rescale threshold (log2 units): within each group of
    ``rescale_group`` query rows (the rows one softmax warp holds) the running
    max is raised only when some row's max would grow by more than
    ``rescale_tau``; meanwhile p may reach 2^tau, so P is rounded as
    e4m3(p * fp8_max * 2^-tau) and the PV product is scaled back by 2^tau.
    """
    BH, Sq, D = q8.shape
    Skv = k8.shape[1]
    out = np.empty((BH, Sq, D), dtype=np.float32)
    qf, kf, vf = (e4m3_decode(x) for x in (q8, k8, v8))
    rows = np.arange(Sq)[:, None]
    for bh in range(BH):
        qk_scale = np.float32(sm_scale) * np.float32(qs[bh]) * np.float32(ks[bh])
        pv_scale = np.float32(vs[bh]) / np.float32(fp8_max)
        m = np.full((Sq,), -np.inf, dtype=np.float32)
        l = np.zeros((Sq,), dtype=np.float32)
        acc = np.zeros((Sq, D), dtype=np.float32)
        for n0 in range(0, Skv, block_n):
            cols = n0 + np.arange(block_n)[None, :]
            kt = np.zeros((block_n, D), np.float32)
            vt = np.zeros((block_n, D), np.float32)
            nv = min(block_n, Skv - n0)
            kt[:nv] = kf[bh, n0 : n0 + nv]
            vt[:nv] = vf[bh, n0 : n0 + nv]
            qk = (qf[bh] @ kt.T).astype(np.float32) * qk_scale
            if causal:
                qk = np.where(rows >= cols, qk, -np.inf)
            qk = np.where(cols < Skv, qk, -np.inf).astype(np.float32)
            m_cand = np.maximum(m, qk.max(axis=1))
            if rescale_tau > 0:
                with np.errstate(invalid="ignore"):
                    need = m_cand > m + np.float32(rescale_tau * np.log(2.0))
                g = int(rescale_group)
                need = np.concatenate([need, np.zeros((-Sq) % g, dtype=bool)])
                grp = np.repeat(need.reshape(-1, g).any(axis=1), g)[:Sq]
                m_new = np.where(grp, m_cand, m).astype(np.float32)
            else:
                m_new = m_cand
            m_use = np.where(m_new == -np.inf, np.float32(0), m_new).astype(np.float32)
            alpha = np.exp(m - m_use).astype(np.float32)
            p = np.exp(qk - m_use[:, None]).astype(np.float32)
            l = l * alpha + p.sum(axis=1, dtype=np.float32)
            acc = acc * alpha[:, None]
            shift = np.float32(2.0**-rescale_tau)
            p8 = e4m3_decode(e4m3_encode((p * np.float32(fp8_max) * shift).astype(np.float32)))
            acc = acc + (p8 @ vt).astype(np.float32) * (pv_scale / shift)
            m = m_new
        out[bh] = acc / l[:, None]
    return out


def prefix_decode_dequant(
    q8: np.ndarray,
    kp8: np.ndarray,
    vp8: np.ndarray,
    kx8: np.ndarray,
    vx8: np.ndarray,
    qs: np.ndarray,
    kps: np.ndarray,
    vps: np.ndarray,
    kxs: np.ndarray,
    vxs: np.ndarray,
    candidates: int,
    tokens: int,
    sm_scale: float,
    heads: list[int] | None = None,
) -> np.ndarray:
    """fp32 shared-prefix decode over dequantised inputs.

    q8/kx8/vx8: (H, C*T, D); kp8/vp8: (H, P, D).  Returns (len(heads), C*T, D).
    """
    H, rows, D = q8.shape
    P = kp8.shape[1]
    heads = list(range(H)) if heads is None else list(heads)
    r = np.arange(rows)
    cand = r // tokens
    suffix_mask = (cand[:, None] == cand[None, :]) & (r[None, :] <= r[:, None])
    mask = np.concatenate([np.ones((rows, P), dtype=bool), suffix_mask], axis=1)
    out = np.empty((len(heads), rows, D), dtype=np.float32)
    for n, h in enumerate(heads):
        qd = dequant(q8[h : h + 1], qs[h : h + 1])[0]
        kd = np.concatenate(
            [dequant(kp8[h : h + 1], kps[h : h + 1])[0], dequant(kx8[h : h + 1], kxs[h : h + 1])[0]]
        )
        vd = np.concatenate(
            [dequant(vp8[h : h + 1], vps[h : h + 1])[0], dequant(vx8[h : h + 1], vxs[h : h + 1])[0]]
        )
        out[n] = softmax_attention(qd, kd, vd, sm_scale, mask=mask)
    return out


def parity_metrics(out: np.ndarray, ref: np.ndarray) -> dict[str, float]:
    """max-abs error, cosine similarity and max |ref| of two arrays."""
    o = np.asarray(out, dtype=np.float64).ravel()
    r = np.asarray(ref, dtype=np.float64).ravel()
    cos = float(o @ r / (np.linalg.norm(o) * np.linalg.norm(r) + 1e-300))
    return {
        "max_abs": float(np.abs(o - r).max()),
        "cos": cos,
        "max_ref": float(np.abs(r).max()),
        "mean_abs": float(np.abs(o - r).mean()),
    }
