"""FLOCK_MATVEC_FAST: the one-token matvec on the int8 tensor cores (x as
three int8 digits per 32-block, exact int32 block sums, f32 scaling) against
the oracle's cpuMatmulQ8F32(coop(64)) / cpuMatmulQ4F32 (kernels/lib.ts:213)
on the same seeded inputs.

Tolerance (north star, reassociated matvec): max relative error 1e-3 against
max(|ref|, 1e-3 * max|ref|) -- rows whose sum cancels to near zero have no
relative error of their own; absErrScaled (ops_ref.ts:206) is printed and
held to 1e-5.  The digit split is exact to ~6e-8 of each block's largest
|x|, so the measured errors sit near f32 rounding (~1e-6)."""
import numpy as np
import pytest

from flock_b200 import lib as flib
from flock_b200 import ops, synth
from gpu_util import abs_err_scaled, rel_err

pytestmark = pytest.mark.gpu

SHAPES = [(64, 32), (30, 1024), (128, 1024), (1024, 1024), (4096, 1024), (3072, 1024),
          (1024, 3072), (1024, 2048), (37, 96), (5, 4096), (17, 288), (4097, 2048),
          (151936, 1024)]


@pytest.fixture(scope="module")
def dev():
    d = flib.get_device(0)
    yield d
    d.close()


def _check(got, want, what):
    want = np.asarray(want, np.float64)
    rel = rel_err(got, want, floor=1e-3 * float(np.abs(want).max()))
    a = abs_err_scaled(got, want)
    print(f"{what}: rel {rel:.2e} (floor 1e-3*amax), maxRelErr {rel_err(got, want):.2e}, "
          f"absErrScaled {a:.2e}")
    assert rel <= 1e-3, rel
    assert a <= 1e-5, a


@pytest.mark.parametrize("q8", [True, False], ids=["q8_0", "q4_0"])
@pytest.mark.parametrize("rows,cols", SHAPES)
def test_matvec_fast_against_oracle(dev, oracle, rows, cols, q8):
    make = synth.q8_tensor if q8 else synth.q4_tensor
    packed = make(7, f"fw{rows}x{cols}", rows, cols)
    x = synth.normal(7, f"fx{cols}", cols)
    w = flib.GpuTensor.from_packed(dev, packed, rows, cols,
                                   flib.FLOCK_Q8_0 if q8 else flib.FLOCK_Q4_0)
    got = ops.matvec_fast(dev, w, x)
    want = (oracle.matmul_q8 if q8 else oracle.matmul_q4)(packed, x, rows, cols)
    _check(got, want, f"{'Q8_0' if q8 else 'Q4_0'} {rows}x{cols}")
    w.free()


@pytest.mark.parametrize("q8", [True, False], ids=["q8_0", "q4_0"])
def test_matvec_fast_block_ranges(dev, oracle, q8):
    """Zero blocks (no digits), blocks of one spike, and blocks 1e6 apart in
    scale: each block's digits follow its own maximum."""
    rows, cols = 300, 1024
    make = synth.q8_tensor if q8 else synth.q4_tensor
    packed = make(8, "frange", rows, cols)
    x = synth.normal(8, "frange_x", cols).astype(np.float32)
    x[0:64] = 0.0                      # two all-zero blocks
    x[64:96] = 0.0
    x[70] = 3.5                        # one spike in an otherwise zero block
    x[96:128] *= 1e3                   # blocks far apart in scale
    x[128:160] *= 1e-3
    x[160:192] = np.float32(2.0) ** -20
    w = flib.GpuTensor.from_packed(dev, packed, rows, cols,
                                   flib.FLOCK_Q8_0 if q8 else flib.FLOCK_Q4_0)
    got = ops.matvec_fast(dev, w, x)
    want = (oracle.matmul_q8 if q8 else oracle.matmul_q4)(packed, x, rows, cols)
    _check(got, want, f"{'Q8_0' if q8 else 'Q4_0'} block ranges")
    w.free()


def test_matvec_fast_extreme_weights(dev, oracle):
    """Q8_0 blocks of all -127 / +127 weights against all-positive x: the
    largest int32 block sums (|D| = 32 * 127 * 127)."""
    rows, cols = 64, 512
    packed = synth.q8_tensor(9, "fext", rows, cols).copy()
    blocks = packed.reshape(rows, cols // 32, 34)   # [f16 scale][32 x int8] per block
    blocks[0::2, :, 2:] = np.uint8(127)
    blocks[1::2, :, 2:] = np.int8(-127).view(np.uint8)
    x = np.abs(synth.normal(9, "fext_x", cols)).astype(np.float32) + 0.5
    w = flib.GpuTensor.from_packed(dev, packed, rows, cols)
    got = ops.matvec_fast(dev, w, x)
    want = oracle.matmul_q8(packed, x, rows, cols)
    _check(got, want, "Q8_0 extreme weights")
    w.free()
