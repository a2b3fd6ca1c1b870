"""The bf16 KV cache option on the CPU side: the oracle's rounding (fo_bf16_round,
RefLayer(kv="bf16")) pinned against torch's own f32 -> bf16 conversion and
against known answers, and the LayerConfig switch that selects it."""
import numpy as np
import pytest
import torch

from flock_b200 import _abi, synth
from flock_b200.layer import QWEN3_06B


def bf16_np(x):
    """f32 -> nearest bf16 (ties to even), as f32; finite inputs."""
    w = np.ascontiguousarray(x, np.float32).view(np.uint32).astype(np.uint64)
    w = ((w + 0x7FFF + ((w >> 16) & 1)) >> 16) << 16
    return w.astype(np.uint32).view(np.float32)


def _round(oracle, bits):
    x = np.array([bits], np.uint32).view(np.float32)[0]
    y = oracle.lib().fo_bf16_round(float(x))
    return int(np.array([y], np.float32).view(np.uint32)[0])


@pytest.mark.parametrize("bits,want", [
    (0x3F800000, 0x3F800000),  # 1.0
    (0x3F808000, 0x3F800000),  # 1 + 2^-8: a tie, to the even 1.0
    (0x3F818000, 0x3F820000),  # 1 + 3 * 2^-8: a tie, to the even 1 + 2^-6
    (0x3F80C000, 0x3F810000),  # above the tie: up
    (0x3F807FFF, 0x3F800000),  # below the tie: down
    (0xBF80C000, 0xBF810000),  # sign kept
    (0x7F7FFFFF, 0x7F800000),  # largest f32 rounds past bf16's largest: infinity
    (0x00008000, 0x00000000),  # a subnormal tie to the even zero
    (0x00018000, 0x00020000),  # a subnormal tie to the even 2
    (0x7F800000, 0x7F800000),  # infinity
])
def test_round_known_answers(oracle, bits, want):
    assert _round(oracle, bits) == want


def test_round_nan_stays_nan(oracle):
    got = _round(oracle, 0x7F800001)
    assert (got & 0x7F800000) == 0x7F800000 and (got & 0x007FFFFF) != 0


def test_round_matches_torch(oracle):
    rng = np.random.default_rng(5)
    x = np.concatenate([rng.standard_normal(4096).astype(np.float32),
                        rng.standard_normal(1024).astype(np.float32) * 1e-38,
                        (rng.standard_normal(1024) * 1e30).astype(np.float32)])
    want = torch.from_numpy(x).to(torch.bfloat16).to(torch.float32).numpy()
    assert np.array_equal(bf16_np(x).view(np.uint32), want.view(np.uint32))
    lib = oracle.lib()
    got = np.array([lib.fo_bf16_round(float(v)) for v in x[:512]], np.float32)
    assert np.array_equal(got.view(np.uint32), want[:512].view(np.uint32))


def _small():
    s = synth.Shape(hidden=256, n_heads=4, n_kv_heads=2, head_dim=128, ffn=512)
    cfg = dict(hidden=s.hidden, n_heads=s.n_heads, n_kv_heads=s.n_kv_heads, head_dim=s.head_dim,
               ffn=s.ffn)
    return s, synth.layer_weights(11, 0, s), cfg


def test_ref_layer_rounds_every_append(oracle):
    s, w, cfg = _small()
    kvw = s.n_kv_heads * s.head_dim
    x = synth.normal(12, "h", s.hidden) * 0.05
    f = oracle.RefLayer(w, cfg, 64)
    b = oracle.RefLayer(w, cfg, 64, kv="bf16")
    f.forward(x, 1)
    b.forward(x, 1)
    # one token: the same k/v before rounding, so the bf16 cache is the
    # rounded f32 cache
    fk, fv = f.cache()
    bk, bv = b.cache()
    assert np.array_equal(bk, bf16_np(fk)) and np.array_equal(bv, bf16_np(fv))
    # a preloaded cache is rounded too, and later appends stay bf16 values
    kc = synth.normal(12, "kc", 8 * kvw)
    vc = synth.normal(12, "vc", 8 * kvw)
    b.fill_cache(kc, vc)
    b.forward(x * 0.5, 1)
    bk, bv = b.cache()
    assert np.array_equal(bk[kvw:9 * kvw], bf16_np(kc))
    assert not np.any(bk.view(np.uint32) & 0xFFFF) and not np.any(bv.view(np.uint32) & 0xFFFF)


def test_ref_layer_bf16_prefill_equals_decode(oracle):
    # the prefill-equals-decode cache property holds with the rounding too
    s, w, cfg = _small()
    n = 5
    x = synth.normal(13, "h", n * s.hidden) * 0.05
    A = oracle.RefLayer(w, cfg, 64, kv="bf16")
    A.forward(x, n)
    B = oracle.RefLayer(w, cfg, 64, kv="bf16")
    for i in range(n):
        B.forward(x[i * s.hidden:(i + 1) * s.hidden], 1)
    ka, va = A.cache()
    kb, vb = B.cache()
    assert np.array_equal(ka, kb) and np.array_equal(va, vb)


def test_ref_layer_bf16_close_to_f32(oracle):
    s, w, cfg = _small()
    kvw = s.n_kv_heads * s.head_dim
    kc = synth.normal(14, "kc", 200 * kvw)
    vc = synth.normal(14, "vc", 200 * kvw)
    x = synth.normal(14, "x", s.hidden)
    outs = []
    for kv in ("f32", "bf16"):
        L = oracle.RefLayer(w, cfg, 256, kv=kv)
        L.fill_cache(kc, vc)
        outs.append(L.forward(x, 1))
    err = np.abs(outs[0] - outs[1]).max() / np.abs(outs[0]).max()
    assert 0 < err < 1e-2


def test_layer_config_kv_switch():
    assert QWEN3_06B.to_c().kv_dtype == _abi.FLOCK_KV_F32
    c = QWEN3_06B.with_(attention="fast", prefill="tensor", kv="bf16").to_c()
    assert c.kv_dtype == _abi.FLOCK_KV_BF16 and c.prefill == _abi.FLOCK_PREFILL_TENSOR
    with pytest.raises(ValueError):
        QWEN3_06B.with_(kv="fp16").to_c()
    with pytest.raises(ValueError):
        import oracle as o
        o.RefLayer({}, {}, 4, kv="fp16")
