"""FP8 GEMM and FP8 linears on the B200 (librepercep_b200.so, rp_fp8_gemm_ex).

* The reference's known answers (tests/test_mfma_fragment_layout.py:262-318):
  all-ones operands give C == K, small integers in [-2, 2] give the bf16 of
  the exact integer product -- bit-exact, through the reference's own API.
* Random e4m3 operands, both B layouts, per-row / per-column / scalar scales,
  bias, bf16 and fp16 output, ragged M / N / K and more tiles than SMs:
  every element within one bf16 rounding of the float64 product plus an fp32
  accumulation bound (2^-20 of sum |a*b|), and almost every element
  bit-equal to the oracle (which sums in float64; the tensor cores sum in a
  different order).
* The row quantizer bit-exact against the oracle, NaN / inf / tiny rows too.
* Fp8Linear against the oracle linear and against torch's bf16 linear, and a
  DiT-sized GEMM against a torch fp32 matmul of the dequantized operands.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from helpers import bits, bytes_equal_nan_aware, fp8_bytes, gen_bf16, scales_equal
from oracle import gemm as og
from oracle.fp8 import bf16_bits_to_f32, e4m3_encode

pytestmark = pytest.mark.gpu

FP8 = torch.float8_e4m3fn


def _lin():  # type: ignore[no-untyped-def]
    from repercep_runtime_b200 import linear

    return linear


def _u8(a: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.uint8)).view(FP8).cuda()


def _rand_e4m3(rng: np.random.Generator, shape: tuple[int, int]) -> np.ndarray:
    """Finite e4m3 bytes: a normal sample scaled into e4m3's range and encoded."""
    y = rng.standard_normal(shape).astype(np.float32) * np.float32(rng.uniform(0.5, 64.0))
    return e4m3_encode(np.clip(y, -448, 448))


def _out_f32(t: torch.Tensor) -> np.ndarray:
    return t.float().cpu().numpy().astype(np.float64)


def _check_against_oracle(got: np.ndarray, a8, b8, sa, sb, bias_f32, layout, out_fmt):  # type: ignore[no-untyped-def]
    """|got - exact| <= one output rounding + 2^-20 of sum |a*b| * |sa*sb|.

    One output rounding is half an ulp: 2^-9 / 2^-12 of |x| for bf16 / fp16,
    and at least half the fp16 subnormal spacing (2^-25) near zero.  (On a
    B200 the accumulation error measured below 2^-25 of sum |a*b|.)"""
    ref = og.dequant_matmul(a8, b8, sa, sb, layout)
    mag = np.abs(og.dequant_matmul(a8 & 0x7F, b8 & 0x7F, np.abs(sa), np.abs(sb), layout))
    if bias_f32 is not None:
        ref = ref + bias_f32[None, :]
    rel, floor = (2.0**-8, 1e-30) if out_fmt == "bf16" else (2.0**-11, 2.0**-25)
    bound = rel * np.abs(ref) + 2.0**-20 * mag + floor
    err = np.abs(got - ref)
    assert (err <= bound).all(), f"max err/bound {np.max(err / bound):.3f}"


@pytest.mark.parametrize("M,N,K", [(16, 16, 32), (300, 520, 4096)])
def test_all_ones_sums_to_k(M, N, K):
    lin = _lin()
    a = torch.ones(M, K, device="cuda").to(FP8)
    b = torch.ones(K, N, device="cuda").to(FP8)
    c = lin.fp8_gemm(a, b, 1.0, 1.0).float()
    assert torch.equal(c, torch.full((M, N), float(K), device="cuda"))


@pytest.mark.parametrize("M,N,K", [(32, 32, 64), (257, 300, 320), (1, 16, 16)])
def test_small_integers_match_exactly(M, N, K):
    lin = _lin()
    g = torch.Generator(device="cuda").manual_seed(0)
    a_i = torch.randint(-2, 3, (M, K), device="cuda", generator=g, dtype=torch.float32)
    b_i = torch.randint(-2, 3, (K, N), device="cuda", generator=g, dtype=torch.float32)
    ref = (a_i.double() @ b_i.double()).float().to(torch.bfloat16).float()
    got = lin.fp8_gemm(a_i.to(FP8), b_i.to(FP8), 1.0, 1.0).float()
    assert torch.equal(got, ref), f"max abs diff {(got - ref).abs().max().item()}"
    # and the oracle agrees bit for bit
    o = og.fp8_gemm(fp8_bytes(a_i.to(FP8)), fp8_bytes(b_i.to(FP8)), 1.0, 1.0)
    assert (bits(got.to(torch.bfloat16)) == o).all()


def test_reference_api_argument_checks():
    lin = _lin()
    a = torch.ones(16, 32, device="cuda").to(FP8)
    with pytest.raises(RuntimeError, match="A must be 2-D"):
        lin.fp8_gemm(a[None], a.t(), 1.0, 1.0)
    with pytest.raises(RuntimeError, match="K mismatch"):
        lin.fp8_gemm(a, a, 1.0, 1.0)
    with pytest.raises(RuntimeError, match="A must be contiguous"):
        lin.fp8_gemm(a.t(), a, 1.0, 1.0)
    with pytest.raises(RuntimeError, match="float8_e4m3fn"):
        lin.fp8_gemm(a.float(), a.t().contiguous(), 1.0, 1.0)


def test_scalar_scales_follow_the_reference_write_back():
    lin = _lin()
    rng = np.random.default_rng(3)
    a8, b8 = _rand_e4m3(rng, (200, 96)), _rand_e4m3(rng, (96, 272))
    got = lin.fp8_gemm(_u8(a8), _u8(b8), 0.0123, 3.7)
    _check_against_oracle(_out_f32(got), a8, b8, 0.0123, 3.7, None, "kn", "bf16")
    o = og.fp8_gemm(a8, b8, 0.0123, 3.7)
    assert np.mean(bits(got) == o) > 0.99


CASES = [
    # M, N, K, layout, scales, bias, out
    (1, 8, 16, "nk", "row", True, torch.bfloat16),
    (127, 129, 48, "kn", "row", False, torch.bfloat16),
    (129, 300, 4100, "nk", "row", True, torch.float16),
    (300, 520, 1000, "kn", "scalar", True, torch.bfloat16),
    (1024, 2048, 512, "nk", "device_scalar", False, torch.bfloat16),
    (2048, 4096, 256, "nk", "row", True, torch.bfloat16),  # 256 tiles: two per CTA
    (4096, 4096, 128, "kn", "row", False, torch.float16),  # 512 tiles: parities wrap
    (333, 777, 2000, "nk", "row", True, torch.bfloat16),
]


@pytest.mark.parametrize("M,N,K,layout,scales,use_bias,out_dtype", CASES)
def test_random_operands_against_the_oracle(M, N, K, layout, scales, use_bias, out_dtype):
    lin = _lin()
    rng = np.random.default_rng(M * 7 + N * 3 + K)
    a8 = _rand_e4m3(rng, (M, K))
    b8 = _rand_e4m3(rng, (N, K) if layout == "nk" else (K, N))
    if scales == "row":
        sa = rng.uniform(1e-3, 1e-1, M).astype(np.float32)
        sb = rng.uniform(1e-3, 1e-1, N).astype(np.float32)
        sa_t, sb_t = torch.from_numpy(sa).cuda(), torch.from_numpy(sb).cuda()
    elif scales == "device_scalar":
        sa, sb = np.float32(0.02), np.float32(0.5)
        sa_t = torch.tensor([0.02], device="cuda")
        sb_t = torch.tensor([0.5], device="cuda")
    else:
        sa, sb = np.float32(0.01), np.float32(0.25)
        sa_t, sb_t = 0.01, 0.25
    fmt = "bf16" if out_dtype == torch.bfloat16 else "f16"
    bias_t = bias_bits = bias_f32 = None
    if use_bias:
        bias_t = gen_bf16((N,), "n1", seed=N, dtype=out_dtype).cuda()
        bias_bits = bits(bias_t)
        bias_f32 = bias_t.float().cpu().numpy().astype(np.float64)
    got = lin.gemm_ex(_u8(a8), _u8(b8), sa_t, sb_t, bias_t, out_dtype, layout)
    torch.cuda.synchronize()
    _check_against_oracle(_out_f32(got), a8, b8, sa, sb, bias_f32, layout, fmt)
    o = og.gemm_ex(a8, b8, sa, sb, bias_bits, fmt, layout)
    assert np.mean(bits(got) == o) > 0.99


def test_zero_k_writes_the_bias():
    lin = _lin()
    a8 = torch.zeros(130, 0, device="cuda", dtype=FP8)
    b8 = torch.zeros(40, 0, device="cuda", dtype=FP8)
    bias = gen_bf16((40,), "n1", seed=1).cuda()
    got = lin.gemm_ex(a8, b8, 1.0, 1.0, bias)
    assert torch.equal(got, bias[None, :].expand(130, 40))
    got = lin.gemm_ex(a8, b8, 1.0, 1.0)
    assert torch.equal(got, torch.zeros_like(got))


def test_output_into_a_strided_view():
    lin = _lin()
    rng = np.random.default_rng(9)
    a8, b8 = _rand_e4m3(rng, (100, 64)), _rand_e4m3(rng, (48, 64))
    big = torch.full((100, 80), 7.0, device="cuda", dtype=torch.bfloat16)
    out = big[:, 16:64]
    lin.gemm_ex(_u8(a8), _u8(b8), 0.5, 0.5, out=out)
    assert (big[:, :16] == 7).all() and (big[:, 64:] == 7).all()
    _check_against_oracle(_out_f32(out), a8, b8, 0.5, 0.5, None, "nk", "bf16")


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize(
    "rows,cols", [(1, 8), (5, 96), (300, 4096), (17, 13824), (9, 12), (6, 20000), (5, 40000), (7, 5120)]
)
def test_quantize_rows_bit_exact(rows, cols, dtype):
    lin = _lin()
    x = gen_bf16((rows, cols), "n1_outlier", seed=rows + cols, dtype=dtype)
    if rows >= 5:
        x[1] = 0
        x[2] = gen_bf16((cols,), "tiny", seed=2, dtype=dtype)
        x[3, 3] = float("inf")
        x[4, 1] = float("nan")
    q, s = lin.quantize_rows(x.cuda())
    fmt = "bf16" if dtype == torch.bfloat16 else "f16"
    oq8, os_ = og.quantize_rows(bits(x), fmt)
    assert q.shape == (rows, cols) and q.stride(0) % 16 == 0
    assert bytes_equal_nan_aware(fp8_bytes(q), oq8).all()
    assert scales_equal(s.cpu().numpy(), os_).all()


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_fp8_linear_against_the_oracle_and_torch(dtype):
    from repercep_runtime_b200.linear import Fp8Linear

    torch.manual_seed(0)
    lin = torch.nn.Linear(320, 200, bias=True).to(device="cuda", dtype=dtype)
    x = gen_bf16((2, 37, 320), "n1", seed=11, dtype=dtype).cuda()
    f8 = Fp8Linear.from_linear(lin)
    y = f8(x)
    assert y.shape == (2, 37, 200) and y.dtype == dtype
    fmt = "bf16" if dtype == torch.bfloat16 else "f16"
    o = og.linear(bits(x.reshape(-1, 320)), bits(lin.weight), bits(lin.bias), fmt)
    got = y.reshape(-1, 200).float().cpu().numpy()
    ref = (bf16_bits_to_f32(o) if fmt == "bf16" else o.view(np.float16).astype(np.float32))
    diff = np.abs(got - ref)
    assert np.mean(diff == 0) > 0.99
    assert (diff <= 2.0**-7 * np.abs(ref) + 1e-6).all()
    full = lin(x).float()
    cos = torch.nn.functional.cosine_similarity(y.float().flatten(), full.flatten(), dim=0)
    assert cos.item() > 0.998


def test_dit_sized_gemm_against_torch_fp32():
    lin = _lin()
    M, K, N = 4096, 4096, 3 * 4096  # a Cosmos-7B QKV projection over 4096 tokens
    g = torch.Generator(device="cuda").manual_seed(5)
    x = torch.randn(M, K, device="cuda", generator=g, dtype=torch.bfloat16)
    w = (torch.randn(N, K, device="cuda", generator=g) * 0.02).to(torch.bfloat16)
    x8, xs = lin.quantize_rows(x)
    w8, ws = lin.quantize_rows(w)
    y = lin.gemm_ex(x8, w8, xs, ws).float()
    ref = (x8.float() * xs[:, None]) @ (w8.float() * ws[:, None]).t()
    rel = ((y - ref).abs() / (ref.abs() + 1e-3)).max().item()
    cos = torch.nn.functional.cosine_similarity(y.flatten(), ref.flatten(), dim=0).item()
    assert cos > 0.99999 and rel < 2.0**-7, (cos, rel)


def test_single_cta_kernel_passes_the_same_suite():
    """REPERCEP_B200_GEMM_PAIR=0 selects the single-CTA kernel (128 x 256
    tiles, no cluster); the library reads the switch once per process."""
    import os
    import subprocess
    import sys
    from pathlib import Path

    if os.environ.get("REPERCEP_B200_GEMM_PAIR") == "0":
        pytest.skip("already running the single-CTA kernel")
    repo = Path(__file__).resolve().parent.parent
    env = dict(os.environ, REPERCEP_B200_GEMM_PAIR="0")
    proc = subprocess.run(
        [sys.executable, "-m", "pytest", "-q", "-x", "-p", "no:cacheprovider",
         "tests/test_gemm_gpu.py", "-k", "not single_cta"],
        cwd=repo, env=env, capture_output=True, text=True, timeout=900,
    )  # fmt: skip
    assert proc.returncode == 0, proc.stdout[-4000:] + proc.stderr[-2000:]
