"""silu_and_mul and rms_norm on the B200 against the oracle and vLLM's formulas.

Against the oracle (correctly rounded exp, fp64-accumulated mean) the bf16
outputs are bit-exact; against the reference's own fixtures they agree to
1 bf16 ulp on a small fraction of elements (the reference's fp32 summation
order and exp rounding).
"""

import json
import os

import numpy as np
import pytest
import torch

import configs as C
import oracle

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(os.path.dirname(__file__), "golden")
MANIFEST = json.load(open(os.path.join(GOLDEN, "manifest.json")))
DEV = "cuda:0"


def _m():
    import torch_mcpu_b200

    return torch_mcpu_b200


def bits(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.int16).cpu().numpy().view(np.uint16)


def ulp_diff(a, b):
    a = a.astype(np.int32)
    b = b.astype(np.int32)
    a = np.where(a & 0x8000, -(a & 0x7FFF), a)
    b = np.where(b & 0x8000, -(b & 0x7FFF), b)
    return np.abs(a - b)


def run_silu(x: torch.Tensor) -> torch.Tensor:
    xd = x.to(DEV)
    out = torch.empty(x.shape[0], x.shape[1] // 2, dtype=torch.bfloat16, device=DEV)
    _m().silu_and_mul(out, xd)
    torch.cuda.synchronize()
    return out


def run_rms(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    xd, wd = x.to(DEV), w.to(DEV)
    out = torch.empty_like(xd)
    _m().rms_norm(out, xd, wd, eps)
    torch.cuda.synchronize()
    return out


@pytest.mark.parametrize("T,d", [(64, 1024), (33, 1000), (4, 18432), (1, 8), (3, 1), (257, 24)])
def test_silu_and_mul_bit_exact_vs_oracle(T, d):
    x = C.silu_inputs(T, d)
    out = run_silu(x)
    ref = oracle.silu_and_mul_bf16(bits(x), exp_mode=oracle.EXP_CR)
    np.testing.assert_array_equal(bits(out), ref)


@pytest.mark.parametrize("name", [k for k in MANIFEST["bandwidth"] if k.startswith("silu")])
def test_silu_and_mul_vs_reference_fixture(name):
    e = MANIFEST["bandwidth"][name]
    x = C.silu_inputs(e["T"], e["d"])
    gold = np.load(os.path.join(GOLDEN, e["file"]))["out_bits"].view(np.uint16)
    d = ulp_diff(bits(run_silu(x)), gold)
    assert d.max() <= 1 and (d > 0).mean() < 2e-3


def test_silu_and_mul_special_values():
    vals = torch.tensor([0.0, -0.0, 1e-30, -1e-30, 1e-40, 59.9, 60.1, -60.1, 80.0, -80.0, -87.5,
                         -88.7, -100.0, -1e4, 1e4, 3e38, -3e38, float("inf"), float("-inf"),
                         float("nan"), 2.0 ** -126, -(2.0 ** -130)], dtype=torch.float32)
    n = vals.numel()
    a = vals.repeat(n).to(torch.bfloat16)
    b = vals.repeat_interleave(n).to(torch.bfloat16)
    x = torch.stack([a, b], 0).reshape(2, n * n).t().reshape(n * n, 2).contiguous()
    out = run_silu(x)
    ref = oracle.silu_and_mul_bf16(bits(x), exp_mode=oracle.EXP_CR)
    o = bits(out)
    nan_o = np.isnan(oracle.bf16_bits_to_f32(o))
    nan_r = np.isnan(oracle.bf16_bits_to_f32(ref))
    np.testing.assert_array_equal(nan_o, nan_r)
    np.testing.assert_array_equal(o[~nan_r], ref[~nan_r])


def test_silu_and_mul_dense_sweep_of_bf16_inputs():
    """Every finite bf16 value as `a` (b = 1.5), through the vectorised path:
    exercises both the fast evaluation and the near-midpoint re-evaluation."""
    a_bits = np.arange(0, 1 << 16, dtype=np.uint32).astype(np.uint16)
    a_bits = a_bits[np.isfinite(oracle.bf16_bits_to_f32(a_bits))]
    pad = (-a_bits.size) % 8
    a_bits = np.concatenate([a_bits, np.zeros(pad, np.uint16)]).reshape(-1, 8)
    x = np.concatenate([a_bits, np.full_like(a_bits, 0x3FC0)], 1)  # b = 1.5
    xt = torch.from_numpy(np.ascontiguousarray(x).view(np.int16)).view(torch.bfloat16)
    out = run_silu(xt)
    ref = oracle.silu_and_mul_bf16(x, exp_mode=oracle.EXP_CR)
    np.testing.assert_array_equal(bits(out), ref)


def test_silu_and_mul_full_size_bit_exact():
    T, d = C.SILU_FULL
    x = C.silu_inputs(T, d)
    out = run_silu(x)
    ref = oracle.silu_and_mul_bf16(bits(x), exp_mode=oracle.EXP_CR)
    np.testing.assert_array_equal(bits(out), ref)


def test_silu_and_mul_misaligned_and_empty():
    x = C.silu_inputs(16, 64)
    flat = torch.empty(1 + x.numel(), dtype=torch.bfloat16, device=DEV)
    xd = flat[1:].view(16, 128)
    xd.copy_(x.to(DEV))
    out = torch.empty(16, 64, dtype=torch.bfloat16, device=DEV)
    _m().silu_and_mul(out, xd)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(bits(out), oracle.silu_and_mul_bf16(bits(x), exp_mode=oracle.EXP_CR))
    e = torch.empty(0, 16, dtype=torch.bfloat16, device=DEV)
    _m().silu_and_mul(torch.empty(0, 8, dtype=torch.bfloat16, device=DEV), e)


def test_silu_and_mul_rejects_bad_arguments():
    x = torch.zeros(4, 16, dtype=torch.bfloat16, device=DEV)
    with pytest.raises(RuntimeError, match="out must be"):
        _m().silu_and_mul(torch.zeros(4, 16, dtype=torch.bfloat16, device=DEV), x)
    with pytest.raises(RuntimeError, match="bfloat16"):
        _m().silu_and_mul(torch.zeros(4, 8, device=DEV), x.float())
    with pytest.raises(RuntimeError, match="no CPU fallback"):
        _m().silu_and_mul(torch.zeros(4, 8, dtype=torch.bfloat16), x.cpu())


@pytest.mark.parametrize("T,H", [(16, 7168), (9, 4096), (8, 1000), (5, 20000), (1, 8), (300, 7168)])
def test_rms_norm_bit_exact_vs_oracle(T, H):
    x, w = C.rms_inputs(T, H)
    out = run_rms(x, w, C.RMS_EPS)
    np.testing.assert_array_equal(bits(out), oracle.rms_norm_bf16(bits(x), bits(w), C.RMS_EPS))


@pytest.mark.parametrize("name", [k for k in MANIFEST["bandwidth"] if k.startswith("rms")])
def test_rms_norm_vs_reference_fixture(name):
    e = MANIFEST["bandwidth"][name]
    x, w = C.rms_inputs(e["T"], e["H"])
    gold = np.load(os.path.join(GOLDEN, e["file"]))["out_bits"].view(np.uint16)
    d = ulp_diff(bits(run_rms(x, w, e["eps"])), gold)
    assert d.max() <= 1 and (d > 0).mean() < 2e-3


def test_rms_norm_full_size_bit_exact():
    T, H = C.RMS_FULL
    x, w = C.rms_inputs(T, H)
    out = run_rms(x, w, C.RMS_EPS)
    np.testing.assert_array_equal(bits(out), oracle.rms_norm_bf16(bits(x), bits(w), C.RMS_EPS))


def test_rms_norm_zero_rows_and_large_values():
    x, w = C.rms_inputs(4, 512)
    x[0] = 0
    x[1] = x[1] * 1e30
    out = run_rms(x, w, C.RMS_EPS)
    np.testing.assert_array_equal(bits(out), oracle.rms_norm_bf16(bits(x), bits(w), C.RMS_EPS))


def test_elementwise_sigmoid_silu_on_a_strided_sample_of_all_fp32():
    """The device's correctly rounded exp (fp32 arithmetic only) against the
    oracle's (float)exp((double)x) on every 97th fp32 bit pattern."""
    u = np.arange(0, 1 << 32, 97, dtype=np.uint64).astype(np.uint32)
    x = u.view(np.float32)
    x = x[np.isfinite(x)]
    xd = torch.from_numpy(x).to(DEV)
    s = _m().sigmoid(xd).cpu().numpy()
    t = _m().silu(xd).cpu().numpy()
    ref_s = oracle.sigmoid_f32(x, oracle.EXP_CR)
    np.testing.assert_array_equal(s.view(np.uint32), ref_s.view(np.uint32))
    ref_t = (x / (np.float32(1.0) + np.exp(-x.astype(np.float64)).astype(np.float32))).astype(np.float32)
    ok = ~(np.isnan(t) & np.isnan(ref_t))
    np.testing.assert_array_equal(t.view(np.uint32)[ok], ref_t.view(np.uint32)[ok])
