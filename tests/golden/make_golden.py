"""Generate the golden fixtures that pin the oracle to the reference.

Runs the reference's own code, imported from its source tree (``--reference``;
the tree exists only where the fixtures are generated):

  * ``_per_bh_scale`` + ``_quantize``
    (kernels/triton_kernels/fp8_flash_attn_hopper.py:374-398) on seeded bf16
    tensors covering N(0,1), N(0,0.5), x20 outliers, zeros, values under the
    1e-6 amax floor, huge values, NaN/inf and ragged sequence lengths;
  * ``fp8_flash_attention`` (:432-586) executed by Triton's interpreter
    (TRITON_INTERPRET=1, fixed 128x128 tile via REPERCEP_FP8_DISABLE_AUTOTUNE)
    on small non-causal, ragged and causal problems.

Triton 3.6's interpreter converts fp32 to e4m3 with a carry bug: when
rounding up overflows the 3-bit mantissa it drops the carry (0.1232 becomes
0.0625 instead of 0.125).  The reference kernel runs on GPUs, whose
conversion instruction rounds to nearest-even correctly, so for that one
cast (P -> e4m3, fp8_flash_attn_hopper.py:322) this script substitutes
PyTorch's e4m3 conversion -- the conversion the reference's own quantizer
uses (:398).  Every other interpreter operation is untouched.

Writes tests/golden/quantize_cases.npz and tests/golden/attention_cases.npz:
bf16 inputs as uint16 bit patterns, fp32 scales, e4m3 bytes, bf16 outputs;
and tests/golden/quantize_f16_cases.npz / attention_extra_cases.npz: the
quantizer on fp16 inputs, attention at head dims 32, 64, 256 and on fp16
(outputs in the input's dtype).

    python tests/golden/make_golden.py [--reference <reference source tree>]
"""

from __future__ import annotations

import argparse
import os
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
REPO = HERE.parent.parent
if str(REPO) not in sys.path:
    sys.path.insert(0, str(REPO))
sys.path.insert(0, str(HERE.parent))

QUANT_CASES = [
    # (name, shape (B,H,S,D), dist, seed)
    ("n1_1x2x300x64", (1, 2, 300, 64), "n1", 7),
    ("n05_1x1x256x128", (1, 1, 256, 128), "n05", 8),
    ("outlier_1x1x257x128", (1, 1, 257, 128), "n1_outlier", 9),
    ("qkdiv8_1x1x77x32", (1, 1, 77, 32), "qk_div8", 10),
    ("zeros_1x1x128x64", (1, 1, 128, 64), "zeros", 11),
    ("tiny_1x2x64x64", (1, 2, 64, 64), "tiny", 12),
    ("huge_1x1x64x128", (1, 1, 64, 128), "huge", 13),
    ("naninf_1x2x128x64", (1, 2, 128, 64), "naninf", 14),
]

ATTN_CASES = [
    # (name, (B,H,S,D), dist, seed, causal)
    ("qkdiv8_1x1x160x128", (1, 1, 160, 128), "qk_div8", 21, False),
    ("n1_1x1x200x128_ragged", (1, 1, 200, 128), "n1", 22, False),
    ("n1_1x1x192x128_causal", (1, 1, 192, 128), "n1", 23, True),
]

# The other head dims the reference's op advertises (fp8_hopper_triton.py:41)
# and fp16 inputs (its supports() takes BF16 and FP16), written to separate
# files so the fixtures above stay byte-identical.
QUANT_F16_CASES = [
    ("f16_n1_1x2x300x64", (1, 2, 300, 64), "n1", 31),
    ("f16_outlier_1x1x257x128", (1, 1, 257, 128), "n1_outlier", 32),
    ("f16_qkdiv8_1x1x77x32", (1, 1, 77, 32), "qk_div8", 33),
    ("f16_zeros_1x1x128x64", (1, 1, 128, 64), "zeros", 34),
    ("f16_tiny_1x2x64x64", (1, 2, 64, 64), "tiny", 35),
    ("f16_huge_1x1x64x128", (1, 1, 64, 128), "huge", 36),
    ("f16_naninf_1x2x128x256", (1, 2, 128, 256), "naninf", 37),
]

ATTN_EXTRA_CASES = [
    # (name, (B,H,S,D), dist, seed, causal, dtype)
    ("n05_1x1x192x64", (1, 1, 192, 64), "n05", 41, False, "bf16"),
    ("n05_1x1x160x32_causal", (1, 1, 160, 32), "n05", 42, True, "bf16"),
    ("n05_1x1x144x256", (1, 1, 144, 256), "n05", 43, False, "bf16"),
    ("f16_n05_1x1x200x128", (1, 1, 200, 128), "n05", 44, False, "f16"),
]


def gen(shape, dist, seed, dtype=None):  # type: ignore[no-untyped-def]
    import torch

    from helpers import gen_bf16

    dtype = torch.bfloat16 if dtype is None else dtype
    if dist != "naninf":
        return gen_bf16(shape, dist, seed, dtype)
    x = gen_bf16(shape, "n1", seed, dtype)
    x[0, 0, 3, 7] = float("nan")
    x[0, 1, 9, 1] = float("inf")
    x[0, 1, 10, 2] = float("-inf")
    return x.to(dtype)


def bits(t):  # type: ignore[no-untyped-def]
    import torch

    return t.contiguous().view(torch.int16).numpy().view(np.uint16)


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--reference", default=None,
                    help="reference source tree (default: $REPERCEP_REFERENCE_ROOT or ../reference)")
    args = ap.parse_args()
    from oracle.build_ref import reference_root

    ref = Path(args.reference) if args.reference else reference_root()
    if ref is None:
        raise SystemExit("reference source tree not found; pass --reference")
    os.environ["TRITON_INTERPRET"] = "1"
    os.environ["REPERCEP_FP8_DISABLE_AUTOTUNE"] = "1"
    sys.path.insert(0, str(ref / "kernels"))
    import torch
    import triton.language as tl
    from triton.runtime import interpreter

    convert = interpreter._convert_float

    def convert_fixed(data, src, dst, rounding_mode):  # type: ignore[no-untyped-def]
        if src == tl.float32 and dst == tl.float8e4nv:
            y = torch.from_numpy(np.ascontiguousarray(data, dtype=np.float32))
            return y.to(torch.float8_e4m3fn).view(torch.uint8).numpy()
        return convert(data, src, dst, rounding_mode)

    interpreter._convert_float = convert_fixed
    from triton_kernels.fp8_flash_attn_hopper import (  # type: ignore[import-not-found]
        _per_bh_scale,
        _quantize,
        fp8_flash_attention,
    )

    q_out: dict[str, np.ndarray] = {}
    for name, shape, dist, seed in QUANT_CASES:
        x = gen(shape, dist, seed)
        s = _per_bh_scale(x)
        q = _quantize(x, s)
        q_out[f"{name}/x"] = bits(x)
        q_out[f"{name}/scales"] = s.numpy().astype(np.float32)
        q_out[f"{name}/q"] = q.view(torch.uint8).numpy()
    np.savez_compressed(HERE / "quantize_cases.npz", **q_out)

    a_out: dict[str, np.ndarray] = {}
    for name, shape, dist, seed, causal in ATTN_CASES:
        q, k, v = (gen(shape, dist, seed + i) for i in range(3))
        o = fp8_flash_attention(q, k, v, causal=causal)
        a_out[f"{name}/q"] = bits(q)
        a_out[f"{name}/k"] = bits(k)
        a_out[f"{name}/v"] = bits(v)
        a_out[f"{name}/out"] = bits(o.to(torch.bfloat16))
        a_out[f"{name}/causal"] = np.array([int(causal)])
        print(f"{name}: out max {float(o.float().abs().max()):.4f}")
    np.savez_compressed(HERE / "attention_cases.npz", **a_out)

    f_out: dict[str, np.ndarray] = {}
    for name, shape, dist, seed in QUANT_F16_CASES:
        x = gen(shape, dist, seed, torch.float16)
        s = _per_bh_scale(x)
        q = _quantize(x, s)
        f_out[f"{name}/x"] = bits(x)
        f_out[f"{name}/scales"] = s.numpy().astype(np.float32)
        f_out[f"{name}/q"] = q.view(torch.uint8).numpy()
    np.savez_compressed(HERE / "quantize_f16_cases.npz", **f_out)

    e_out: dict[str, np.ndarray] = {}
    for name, shape, dist, seed, causal, fmt in ATTN_EXTRA_CASES:
        dt = torch.float16 if fmt == "f16" else torch.bfloat16
        q, k, v = (gen(shape, dist, seed + i, dt) for i in range(3))
        o = fp8_flash_attention(q, k, v, causal=causal)
        assert o.dtype == dt
        e_out[f"{name}/q"] = bits(q)
        e_out[f"{name}/k"] = bits(k)
        e_out[f"{name}/v"] = bits(v)
        e_out[f"{name}/out"] = bits(o)
        e_out[f"{name}/causal"] = np.array([int(causal)])
        e_out[f"{name}/f16"] = np.array([int(fmt == "f16")])
        print(f"{name}: out max {float(o.float().abs().max()):.4f}")
    np.savez_compressed(HERE / "attention_extra_cases.npz", **e_out)


if __name__ == "__main__":
    main()
