"""The kernels/*.ts drop-in shim against the C ABI it binds (no TS runtime is
needed: the checks read the TypeScript as text).

* kernels/cuda_ffi.ts is exactly what kernels/gen_ffi.py renders from
  include/flock_cuda.h, and its symbol table agrees with the ctypes table
  (flock_b200/_abi.py) name for name, arity and type class;
* the flock_layer_config layout the TS packs equals the C/ctypes layout;
* every lib.ts / layer.ts / model.ts / shard.ts export the reference
  surface lists is there, every flock_* call in them names a symbol of the
  table with its arity, and every name imported between the shim modules is
  exported by the module it comes from;
* the host quantizers the shim's quantRowQ8/Q4 call are byte-identical to
  the oracle's (kernels/lib.ts:40, :64), half-way cases included.
"""
import ctypes
import os
import re
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, os.path.join(ROOT, "kernels"))

import gen_ffi  # noqa: E402

from flock_b200 import _abi  # noqa: E402

KDIR = os.path.join(ROOT, "kernels")


def read(name: str) -> str:
    with open(os.path.join(KDIR, name)) as f:
        return f.read()


def strip_ts_comments(s: str) -> str:
    s = re.sub(r"/\*.*?\*/", "", s, flags=re.S)
    return re.sub(r"//[^\n]*", "", s)


# ----------------------------------------------------------- symbol table
def ts_table() -> dict:
    src = read("cuda_ffi.ts")
    body = re.search(r"export const symbols = \{(.*?)\} as const;", src, re.S).group(1)
    out = {}
    for m in re.finditer(r"(flock_\w+): \{ parameters: \[([^\]]*)\], result: \"(\w+)\" \}", body):
        params = [p.strip().strip('"') for p in m.group(2).split(",") if p.strip()]
        out[m.group(1)] = (params, m.group(3))
    return out


def test_cuda_ffi_is_generated_from_the_header():
    assert read("cuda_ffi.ts") == gen_ffi.render(), "run python kernels/gen_ffi.py"


_CT = {"i32": {ctypes.c_int, ctypes.c_int32}, "i64": {ctypes.c_int64, ctypes.c_longlong},
       "u32": {ctypes.c_uint32, ctypes.c_uint}, "f32": {ctypes.c_float},
       "f64": {ctypes.c_double}}


def _is_pointer(ct) -> bool:
    return (ct in (ctypes.c_void_p, ctypes.c_char_p) or
            (isinstance(ct, type) and issubclass(ct, ctypes._Pointer)))


def test_table_agrees_with_ctypes_bindings():
    table = ts_table()
    protos, _, _, _ = gen_ffi.parse()
    assert set(table) == {p[0] for p in protos}
    assert set(table) == set(_abi.SIGNATURES), (
        sorted(set(table) ^ set(_abi.SIGNATURES)))
    for name, (params, res) in table.items():
        cts = _abi.SIGNATURES[name]
        assert len(params) == len(cts), name
        for i, (p, ct) in enumerate(zip(params, cts)):
            if p in ("pointer", "buffer"):
                assert _is_pointer(ct), f"{name} arg {i}: {p} vs {ct}"
            else:
                assert ct in _CT[p], f"{name} arg {i}: {p} vs {ct}"
        want = "pointer" if name in _abi._RESTYPE else "i32"
        assert res == want, name


def test_library_exports_the_table():
    lib = ctypes.CDLL(_abi.LIB_PATH)
    for name in ts_table():
        assert hasattr(lib, name), name


def test_layer_config_layout_matches_c():
    _, _, fields, size = gen_ffi.parse()
    assert size == ctypes.sizeof(_abi.LayerConfigC)
    c_fields = {n: getattr(_abi.LayerConfigC, n).offset for n, _ in _abi.LayerConfigC._fields_}
    assert {n: off for n, _, off in fields} == c_fields
    src = read("cuda_ffi.ts")
    assert f"export const LAYER_CONFIG_BYTES = {size};" in src
    for n, ty, off in fields:
        setter = {"int32_t": "Int32", "float": "Float32", "double": "Float64"}[ty]
        assert f"dv.set{setter}({off}, c.{n}, true);" in src


def test_enum_constants_match_ctypes_module():
    src = read("cuda_ffi.ts")
    for name in ["FLOCK_OK", "FLOCK_E_ARG", "FLOCK_E_CUDA", "FLOCK_E_STATE", "FLOCK_E_MISSING",
                 "FLOCK_E_LIMIT", "FLOCK_E_NCCL", "FLOCK_E_NOMEM", "FLOCK_E_UNSUPPORTED",
                 "FLOCK_Q8_0", "FLOCK_Q4_0", "FLOCK_F32", "FLOCK_DECODE_KERNELS",
                 "FLOCK_DECODE_STREAM", "FLOCK_KV_BF16", "FLOCK_ATTN_FAST"]:
        assert f"export const {name} = {getattr(_abi, name)};" in src, name


# ------------------------------------------------------------- surfaces
def exports(name: str) -> set:
    src = strip_ts_comments(read(name))
    out = set(re.findall(
        r"^export (?:async )?(?:function|class|const|let|interface|type) (\w+)", src, re.M))
    for m in re.finditer(r"^export \{([^}]*)\}", src, re.M):
        out |= {x.strip().split(" as ")[-1] for x in m.group(1).split(",") if x.strip()}
    return out


def class_members(name: str, cls: str) -> set:
    src = strip_ts_comments(read(name))
    start = src.index(f"export class {cls}")
    depth, i, body_start = 0, src.index("{", start), None
    body_start = i
    while True:
        if src[i] == "{":
            depth += 1
        elif src[i] == "}":
            depth -= 1
            if depth == 0:
                break
        i += 1
    body = src[body_start:i]
    # members at the class body's top level (two-space indent), plus the
    # constructor's parameter properties
    top = set(re.findall(
        r"^  (?:static |readonly |private |async |get |set )*(\w+)\s*[(:<]", body, re.M))
    return top | set(re.findall(r"^    (?:public |private )?readonly (\w+):", body, re.M))


SURFACE = {
    "lib.ts": ["getDevice", "splitQ8", "splitQ4", "quantRowQ8", "quantRowQ4", "quantMatrixQ8",
               "quantMatrixQ4", "cpuMatmulQ8F32", "cpuMatmulQ4F32", "coop", "SERIAL", "fma32",
               "halfToF32", "storageBuffer", "uniformBuffer", "readBack", "randVec", "maxRelErr",
               "ok", "summary", "Q8_BLOCK", "Q8_BYTES", "Q4_BLOCK", "Q4_BYTES", "SplitQ8",
               "Reduction"],
    "layer.ts": ["Layer", "QWEN3_06B", "LayerConfig", "LayerWeights", "GpuTensor", "LayerBuffers",
                 "wgslSource", "RopePairing"],
    "model.ts": ["Model", "ModelConfig"],
    "shard.ts": ["ShardedMatvec", "ShardedHead", "Direction", "ShardedMatvecOpts",
                 "ShardedHeadOpts"],
}
MEMBERS = {
    ("layer.ts", "Layer"): ["create", "fromBuffers", "encode", "encodePrefill", "forward",
                            "readOutput", "reset", "nKeys", "inputBuffer", "outputBuffer",
                            "cacheBuffers"],
    ("model.ts", "Model"): ["create", "step", "logits", "hiddenState", "encodePartial",
                            "projectHidden", "normedState", "embed", "generate", "stepsAmortized",
                            "rewind", "currentToken", "reset", "pos", "held"],
    ("shard.ts", "ShardedMatvec"): ["create", "setInput", "encode", "encodeShardsOnly",
                                    "encodeReduceOnly", "dispatchShards", "dispatchReduce",
                                    "output", "partials", "wireBytesPerCall", "destroy", "rows",
                                    "cols", "direction", "ranges", "uploadedBytes"],
    ("shard.ts", "ShardedHead"): ["create", "setInput", "encode", "logits", "argmaxBuffers",
                                  "shardBytes", "destroy", "vocab", "hidden", "nShards"],
}


@pytest.mark.parametrize("mod", sorted(SURFACE))
def test_module_exports_the_reference_surface(mod):
    missing = [n for n in SURFACE[mod] if n not in exports(mod)]
    assert not missing, f"{mod} lacks {missing}"


@pytest.mark.parametrize("key", sorted(MEMBERS))
def test_class_members(key):
    mod, cls = key
    have = class_members(mod, cls)
    missing = [n for n in MEMBERS[key] if n not in have]
    assert not missing, f"{cls} lacks {missing}"


def _calls(src: str):
    """(name, argument count) of every flock().flock_xxx(...) call."""
    for m in re.finditer(r"flock\(\)\.(flock_\w+)\(", src):
        i, depth, args, cur = m.end(), 1, 0, ""
        nonempty = False
        while depth:
            ch = src[i]
            if ch in "([{":
                depth += 1
            elif ch in ")]}":
                depth -= 1
            elif ch == "," and depth == 1:
                args += 1
            if depth and not ch.isspace():
                nonempty = True
            i += 1
        yield m.group(1), (args + 1 if nonempty else 0)


def test_every_call_names_a_symbol_with_its_arity():
    table = ts_table()
    seen = 0
    for mod in ["lib.ts", "layer.ts", "model.ts", "shard.ts"]:
        src = strip_ts_comments(read(mod))
        for name, n in _calls(src):
            assert name in table, f"{mod}: {name} is not in the symbol table"
            assert n == len(table[name][0]), f"{mod}: {name} called with {n} args"
            seen += 1
        # calls through an alias: const f = kind === ... ? flock().flock_a : flock().flock_b
        for name in re.findall(r"flock\(\)\.(flock_\w+)\b(?!\()", src):
            assert name in table, f"{mod}: {name}"
    assert seen > 40


def test_imports_between_shim_modules_resolve():
    reference_kept = {"shard_ref.ts", "real_weights.ts"}   # the reference's own CPU modules
    for mod in ["lib.ts", "layer.ts", "model.ts", "shard.ts"]:
        src = strip_ts_comments(read(mod))
        for m in re.finditer(r"import\s+(?:type\s+)?\{([^}]*)\}\s+from\s+\"\./([\w.]+)\"", src):
            target = m.group(2)
            if target in reference_kept:
                continue
            names = [x.strip().replace("type ", "").split(" as ")[0]
                     for x in m.group(1).split(",") if x.strip()]
            have = exports(target)
            missing = [n for n in names if n not in have]
            assert not missing, f"{mod} imports {missing} from {target}"


# ---------------------------------------------------------- quantizers
def _planted(rows, cols, seed):
    rng = np.random.default_rng(seed)
    w = (rng.standard_normal((rows, cols)) * rng.choice([1e-4, 1.0, 300.0], (rows, 1))).astype(np.float32)
    w[0, :32] = 0.0                                   # zero block: d = 0
    # a block whose values sit on half-way points of q = x/d (127 * k + 0.5)
    blk = np.arange(32, dtype=np.float32) - 16.0
    blk[0] = 127.0
    w[-1, :32] = blk + 0.5 * (blk != 127.0)
    if cols >= 64:
        w[-1, 40] = -np.abs(w[-1, 32:64]).max() * 1.5  # negative extreme (Q4 sign)
    return w


@pytest.mark.parametrize("rows,cols,seed", [(1, 32, 0), (5, 256, 1), (9, 1024, 2)])
def test_quantizers_match_the_oracle(rows, cols, seed):
    import oracle
    w = _planted(rows, cols, seed)
    for kind, bb, ref in (("q8", 34, oracle.quant_matrix_q8), ("q4", 18, oracle.quant_matrix_q4)):
        out = np.zeros(rows * cols // 32 * bb, np.uint8)
        _abi.call(f"flock_quant_{kind}", _abi.ptr(w, _abi._fp), rows, cols, _abi.ptr(out, _abi._u8p))
        assert np.array_equal(out, np.asarray(ref(w, rows, cols), np.uint8)), kind


def test_quantizers_reject_ragged_rows():
    w = np.zeros(40, np.float32)
    out = np.zeros(64, np.uint8)
    assert _abi.lib().flock_quant_q8(_abi.ptr(w, _abi._fp), 1, 40, _abi.ptr(out, _abi._u8p)) == \
        _abi.FLOCK_E_ARG
