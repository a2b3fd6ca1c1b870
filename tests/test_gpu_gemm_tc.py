"""Prefill GEMM on the tcgen05 tensor cores (flock_op_gemm) against f64
references of the same matmul:

* exact math (dequantised weights, f32 activations): max relative error
  <= 1e-2, the bf16 prefill bound, as absErrScaled (ops_ref.ts:206);
* the same product of bf16-rounded operands (x and s * q rounded to nearest
  even): agreement to 1e-4, which leaves room only for f32 accumulation order
  and pins the operand layouts, swizzle and descriptors.
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


def bf16(a: np.ndarray) -> np.ndarray:
    """Round f32 values to bf16 (nearest even), returned as f64."""
    u = np.ascontiguousarray(a, np.float32).view(np.uint32).astype(np.uint64)
    u = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16) << 16
    return u.astype(np.uint32).view(np.float32).astype(np.float64)


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
    rounded = bf16(x.reshape(m, cols)) @ bf16(w.astype(np.float32)).T
    assert abs_err_scaled(y, rounded) <= 1e-4


def test_gemm_lm_head_rows(dev):
    """The 151936 x 1024 head (1187 row tiles) at M = 16."""
    rows, cols, m = 151936, 1024, 16
    packed = synth.q8_tensor(6, "head", rows, cols)
    t = flib.GpuTensor.from_packed(dev, packed, rows, cols)
    x = synth.normal(13, "xh", m * cols).astype(np.float32)
    y = ops.gemm(dev, t, x, m).reshape(m, rows).astype(np.float64)
    w = dequant(packed, rows, cols, True)
    rounded = bf16(x.reshape(m, cols)) @ bf16(w.astype(np.float32)).T
    assert abs_err_scaled(y, rounded) <= 1e-4


def test_gemm_rejects_bad_cols(dev):
    packed = synth.q8_tensor(1, "bad", 128, 96)
    t = flib.GpuTensor.from_packed(dev, packed, 128, 96)
    with pytest.raises(FlockError, match="multiple of 64"):
        ops.gemm(dev, t, np.zeros(2 * 96, np.float32), 2)
