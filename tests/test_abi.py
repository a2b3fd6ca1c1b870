"""The C-ABI library loads, exports every symbol include/flock_cuda.h declares,
and its host-only entry points behave.  CPU only (no kernel is launched)."""
import ctypes
import os
import re
import subprocess

import numpy as np
import pytest

from flock_b200 import _abi, synth
from flock_b200 import lib as flib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "flock_cuda.h")


def declared_symbols():
    src = open(HEADER).read()
    return sorted(set(re.findall(r"FLOCK_API\s+[\w\s\*]*?\b(flock_\w+)\s*\(", src)))


@pytest.fixture(scope="module")
def built():
    from flock_b200 import build
    return build.build()


def test_library_exports_every_declared_symbol(built):
    syms = declared_symbols()
    assert len(syms) >= 60
    out = subprocess.run(["nm", "-D", "--defined-only", built], capture_output=True, text=True,
                         check=True).stdout
    exported = set(re.findall(r"\bT (flock_\w+)", out))
    missing = [s for s in syms if s not in exported]
    assert not missing, missing
    # and nothing beyond the declared ABI leaks out
    extra = sorted(e for e in exported if e not in syms)
    assert not extra, extra


def test_python_binding_covers_the_abi(built):
    assert set(declared_symbols()) == set(_abi.SIGNATURES)
    lib = _abi.lib()
    for name in declared_symbols():
        assert hasattr(lib, name)


def test_config_struct_matches_the_header(tmp_path):
    """The ctypes mirror of flock_layer_config has the C compiler's layout."""
    fields = [f[0] for f in _abi.LayerConfigC._fields_]
    prog = tmp_path / "layout.c"
    prog.write_text('#include <stddef.h>\n#include <stdio.h>\n#include "flock_cuda.h"\n'
                    "int main(void) {\n"
                    '  printf("%zu", sizeof(flock_layer_config));\n'
                    + "".join(f'  printf(" %zu", offsetof(flock_layer_config, {f}));\n'
                              for f in fields)
                    + "  return 0;\n}\n")
    exe = tmp_path / "layout"
    subprocess.run(["gcc", "-std=c11", f"-I{os.path.dirname(HEADER)}", str(prog), "-o", str(exe)],
                   check=True)
    got = [int(v) for v in subprocess.run([str(exe)], capture_output=True, text=True,
                                          check=True).stdout.split()]
    want = [ctypes.sizeof(_abi.LayerConfigC)] + [getattr(_abi.LayerConfigC, f).offset
                                                 for f in fields]
    assert got == want


def test_version_and_error_strings(built):
    assert b"sm_100a" in _abi.lib().flock_version()
    assert isinstance(_abi.last_error(), str)


def test_repack_q8_is_bit_exact(built, oracle):
    # kernels/lib.ts:126 splitQ8 -- the C ABI's host repack vs the oracle's
    rows, cols = 37, 1024
    packed = synth.q8_tensor(11, "r", rows, cols)
    qs, sc = flib.split_q8(packed, rows, cols)
    oq, osc = oracle.split_q8(packed, rows, cols)
    assert np.array_equal(qs, oq) and np.array_equal(sc, osc)


def test_repack_q4_is_bit_exact(built, oracle):
    rows, cols = 9, 256
    packed = synth.q4_tensor(12, "r", rows, cols)
    qs, sc = flib.split_q4(packed, rows, cols)
    oq, osc = oracle.split_q4(packed, rows, cols)
    assert np.array_equal(qs, oq) and np.array_equal(sc, osc)


def test_repack_rejects_bad_cols(built):
    with pytest.raises(_abi.FlockError) as e:
        flib.split_q8(np.zeros(34, np.uint8), 1, 48)
    assert "multiple of 32" in str(e.value)


def test_device_open_without_gpu_is_an_error_not_a_crash(built):
    try:
        import torch
        if torch.cuda.is_available():
            pytest.skip("a GPU is present")
    except ImportError:
        pass
    h = ctypes.c_void_p()
    rc = _abi.lib().flock_dev_open(0, ctypes.byref(h))
    assert rc != 0 and not h.value


def test_one_token_step_reaches_the_abi(built):
    """Model.step([id]) passes its prebuilt one-id argument straight to
    flock_model_step: with no model behind the handle the library answers
    with its argument error (raised as FlockError, not a ctypes TypeError);
    ids outside int32 take the array path, as do longer id lists."""
    from flock_b200.layer import QWEN3_06B
    from flock_b200.model import Model
    M = Model(None, None, QWEN3_06B, 4096, 0, [])
    for ids in ([5], (7,), [np.int32(3)]):
        with pytest.raises(_abi.FlockError) as e:
            M.step(ids)
        assert e.value.code == _abi.FLOCK_E_ARG
    for ids in ([2**40], [1, 2]):
        with pytest.raises(_abi.FlockError):
            M.step(ids)
