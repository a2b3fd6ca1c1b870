"""Prefill GEMM on the tcgen05 tensor cores (flock_op_gemm) against f64
references of the same matmul:

* exact math (dequantised weights, f32 activations): max relative error
  <= 1e-2, the tensor-core prefill bound, as absErrScaled (ops_ref.ts:206);
* the same product of the f16 operands the kernel forms (s * q rounded to
  f16; each x row scaled by the power of two that puts its largest magnitude
  in [2^13, 2^14), rounded to f16, scaled back): agreement to 1e-4, which
  leaves room only for f32 accumulation order and pins the operand layouts,
  swizzle, descriptors and row scaling.
"""
import numpy as np
import pytest

from flock_b200 import lib as flib
from flock_b200 import ops, synth
from flock_b200._abi import FlockError
from gpu_util import abs_err_scaled

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def dev():
    d = flib.get_device(0)
    yield d
    d.close()


def dequant(packed: np.ndarray, rows: int, cols: int, q8: bool) -> np.ndarray:
    """GGUF Q8_0 (34-byte) / Q4_0 (18-byte) blocks -> f64 [rows][cols]."""
    bs = 34 if q8 else 18
    b = packed.reshape(rows, cols // 32, bs)
    s = b[:, :, :2].copy().view(np.float16).astype(np.float64)[:, :, 0]
    if q8:
        q = b[:, :, 2:].view(np.int8).astype(np.float64)
    else:
        raw = b[:, :, 2:]
        q = np.concatenate([raw & 0x0F, raw >> 4], axis=2).astype(np.float64) - 8.0
    return (q * s[:, :, None]).reshape(rows, cols)


def f16w(w: np.ndarray) -> np.ndarray:
    """s * q (exact in f32) rounded to f16, as f64."""
    return np.asarray(w, np.float32).astype(np.float16).astype(np.float64)


def f16x(x: np.ndarray) -> np.ndarray:
    """Each row scaled by 2^-e (e = exponent of its largest magnitude - 13),
    rounded to f16, scaled back, as f64."""
    x = np.asarray(x, np.float32)
    mx = np.abs(x).max(axis=1)
    _, ex = np.frexp(mx)                   # mx = f * 2^ex, f in [0.5, 1)
    e = np.clip(np.where(mx > 0, ex - 1 - 13, 0), -120, 120)
    sc = np.ldexp(np.ones_like(mx, dtype=np.float64), -e)[:, None]
    return (x.astype(np.float64) * sc).astype(np.float16).astype(np.float64) / sc


CASES = [
    # (rows, cols, M)
    (1024, 1024, 16),
    (2048, 1024, 37),
    (1024, 2048, 128),
    (3072, 1024, 300),
    (1024, 3072, 512),
    (200, 1024, 20),     # rows not a multiple of 128
    (384, 4096, 64),
]


@pytest.mark.parametrize("q8", [True, False])
@pytest.mark.parametrize("rows,cols,m", CASES)
def test_gemm_matches_references(dev, q8, rows, cols, m):
    make = synth.q8_tensor if q8 else synth.q4_tensor
    packed = make(11, f"w{rows}x{cols}", rows, cols)
    t = flib.GpuTensor.from_packed(dev, packed, rows, cols, flib.FLOCK_Q8_0 if q8 else flib.FLOCK_Q4_0)
    x = synth.normal(12, f"x{m}x{cols}", m * cols).astype(np.float32)
    y = ops.gemm(dev, t, x, m).reshape(m, rows).astype(np.float64)
    w = dequant(packed, rows, cols, q8)
    exact = x.reshape(m, cols).astype(np.float64) @ w.T
    assert abs_err_scaled(y, exact) <= 1e-2
    rounded = f16x(x.reshape(m, cols)) @ f16w(w).T
    assert abs_err_scaled(y, rounded) <= 1e-4


def test_gemm_lm_head_rows(dev):
    """The 151936 x 1024 head (1187 row tiles) at M = 16."""
    rows, cols, m = 151936, 1024, 16
    packed = synth.q8_tensor(6, "head", rows, cols)
    t = flib.GpuTensor.from_packed(dev, packed, rows, cols)
    x = synth.normal(13, "xh", m * cols).astype(np.float32)
    y = ops.gemm(dev, t, x, m).reshape(m, rows).astype(np.float64)
    w = dequant(packed, rows, cols, True)
    rounded = f16x(x.reshape(m, cols)) @ f16w(w).T
    assert abs_err_scaled(y, rounded) <= 1e-4


def test_gemm_rejects_bad_cols(dev):
    packed = synth.q8_tensor(1, "bad", 128, 96)
    t = flib.GpuTensor.from_packed(dev, packed, 128, 96)
    with pytest.raises(FlockError, match="multiple of 64"):
        ops.gemm(dev, t, np.zeros(2 * 96, np.float32), 2)
