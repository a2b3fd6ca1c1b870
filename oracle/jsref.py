"""Line-by-line transliteration of flock's CPU references in JS number semantics.

TEST INFRASTRUCTURE ONLY, and for small cases only (pure-Python loops).  It
exists to cross-check the C restatement in flock_oracle.c: a JS ``number`` is
an IEEE f64 exactly like a Python ``float``, ``Math.fround`` is a cast to f32,
and every function below follows the TypeScript statement by statement, so a
mistake in the C restatement (an int8 cast, an operator precedence, a missing
rounding) shows up as a disagreement between the two.

Citations are to the ethanhinson/flock sources the functions transliterate.
"""
from __future__ import annotations

import math
import struct

import numpy as np


def fr(x: float) -> float:
    """Math.fround."""
    return float(np.float32(x))


def fma32(a: float, b: float, c: float) -> float:
    """lib.ts:169 -- fround(a*b + c) in f64."""
    return fr(a * b + c)


def half_to_f32(h: int) -> float:
    """lib.ts:30"""
    s = -1.0 if (h & 0x8000) else 1.0
    e = (h >> 10) & 0x1F
    m = h & 0x3FF
    if e == 0:
        return s * m * math.pow(2, -24)
    if e == 31:
        return s * 3.4028235e38
    return s * (1 + m / 1024) * math.pow(2, e - 15)


def f32to16(v: float) -> int:
    """wire.mjs:309"""
    x = struct.unpack("<I", struct.pack("<f", np.float32(v)))[0]
    sign = (x >> 16) & 0x8000
    exp = (x >> 23) & 0xFF
    man = x & 0x7FFFFF
    if exp == 255:
        return sign | 0x7C00 | (0x200 if man else 0)
    exp = exp - 127 + 15
    if exp >= 31:
        return sign | 0x7C00
    if exp <= 0:
        if exp < -10:
            return sign
        man |= 0x800000
        shift = 14 - exp
        sub = man >> shift
        rem = man & ((1 << shift) - 1)
        half = 1 << (shift - 1)
        return sign | (sub + (1 if (rem > half or (rem == half and (sub & 1))) else 0))
    h = (exp << 10) | (man >> 13)
    rem = man & 0x1FFF
    if rem > 0x1000 or (rem == 0x1000 and (h & 1)):
        h += 1
    return sign | h


def js_round(x: float) -> float:
    """Math.round: halves go toward +infinity."""
    r = math.floor(x)
    return r + 1 if x - r >= 0.5 else r


def quant_row_q8(vals) -> bytes:
    """lib.ts:40"""
    nb = len(vals) // 32
    out = bytearray(nb * 34)
    for b in range(nb):
        amax = 0.0
        for i in range(32):
            amax = max(amax, abs(float(vals[b * 32 + i])))
        d = amax / 127
        struct.pack_into("<H", out, b * 34, f32to16(d))
        for i in range(32):
            q = 0 if d == 0 else js_round(float(vals[b * 32 + i]) / d)
            out[b * 34 + 2 + i] = int(max(-128, min(127, q))) & 0xFF
    return bytes(out)


def quant_row_q4(vals) -> bytes:
    """lib.ts:64"""
    nb = len(vals) // 32
    out = bytearray(nb * 18)
    for b in range(nb):
        amax = 0.0
        mx = 0.0
        for i in range(32):
            v = float(vals[b * 32 + i])
            if abs(v) > amax:
                amax = abs(v)
                mx = v
        d = mx / -8
        inv = 0 if d == 0 else 1 / d
        struct.pack_into("<H", out, b * 18, f32to16(d))
        for i in range(16):
            x0 = float(vals[b * 32 + i]) * inv + 8.5
            x1 = float(vals[b * 32 + i + 16]) * inv + 8.5
            q0 = min(15, max(0, math.floor(x0)))
            q1 = min(15, max(0, math.floor(x1)))
            out[b * 18 + 2 + i] = q0 | (q1 << 4)
    return bytes(out)


def _dot4(a, b) -> float:
    """lib.ts:196"""
    s = fr(a[0] * b[0])
    s = fma32(a[1], b[1], s)
    s = fma32(a[2], b[2], s)
    s = fma32(a[3], b[3], s)
    return s


def tree_sum(a) -> float:
    """lib.ts:312"""
    buf = [fr(v) for v in a]
    stride = len(buf) >> 1
    while stride > 0:
        for i in range(stride):
            buf[i] = fr(buf[i] + buf[i + stride])
        stride >>= 1
    return buf[0]


def _matmul(rows, cols, block_bytes, lanes, decode, x, pair):
    """lib.ts:213 matmulF32 (lanes == 0 is SERIAL)."""
    nb = cols // 32
    out = np.zeros(rows, np.float32)
    L = lanes if lanes else 1
    pairs = [pair(g) for g in range(4)]
    for r in range(rows):
        part = [0.0] * L
        for b in range(nb):
            scale, q = decode(r * nb * block_bytes + b * block_bytes)
            if lanes == 0:
                s = 0.0
                for i in range(32):
                    s = fma32(q[i], float(x[b * 32 + i]), s)
                part[0] = fma32(scale, s, part[0])
            else:
                lane = b % lanes
                for ia, ib in pairs:
                    d0 = _dot4([q[i] for i in ia], [float(x[b * 32 + i]) for i in ia])
                    d1 = _dot4([q[i] for i in ib], [float(x[b * 32 + i]) for i in ib])
                    part[lane] = fma32(scale, fr(d0 + d1), part[lane])
        out[r] = part[0] if lanes == 0 else tree_sum(part)
    return out


def cpu_matmul_q8(packed: bytes, x, rows, cols, lanes=64):
    """lib.ts:251"""
    def decode(base):
        q = [(packed[base + 2 + i] - 256) if packed[base + 2 + i] > 127 else packed[base + 2 + i]
             for i in range(32)]
        return fr(half_to_f32(struct.unpack_from("<H", packed, base)[0])), q
    return _matmul(rows, cols, 34, lanes, decode, x,
                   lambda g: ([g * 8 + k for k in range(4)], [g * 8 + 4 + k for k in range(4)]))


def cpu_matmul_q4(packed: bytes, x, rows, cols, lanes=64):
    """lib.ts:280"""
    def decode(base):
        q = [0] * 32
        for i in range(16):
            byte = packed[base + 2 + i]
            q[i] = (byte & 0xF) - 8
            q[i + 16] = (byte >> 4) - 8
        return fr(half_to_f32(struct.unpack_from("<H", packed, base)[0])), q
    return _matmul(rows, cols, 18, lanes, decode, x,
                   lambda g: ([g * 4 + k for k in range(4)], [g * 4 + 16 + k for k in range(4)]))


def rmsnorm(x, g, n, n_vecs, eps, wg=128):
    """ops_ref.ts:20"""
    out = np.zeros(n * n_vecs, np.float32)
    for v in range(n_vecs):
        base = v * n
        part = [0.0] * wg
        for t in range(wg):
            acc = 0.0
            for i in range(t, n, wg):
                acc = fma32(float(x[base + i]), float(x[base + i]), acc)
            part[t] = acc
        s = tree_sum(part)
        scale = fr(1 / math.sqrt(fr(fr(s / n) + eps)))
        for i in range(n):
            out[base + i] = fr(fr(float(x[base + i]) * scale) * float(g[i]))
    return out


def rope_inv_freq(head_dim, base):
    """ops_ref.ts:95"""
    return np.array([fr(1 / math.pow(base, (2 * j) / head_dim)) for j in range(head_dim // 2)],
                    np.float32)


def rope(x, n_tokens, n_heads, head_dim, pos0, inv_freq, neox=True):
    """ops_ref.ts:65"""
    out = [float(v) for v in x]
    half = head_dim // 2
    for t in range(n_tokens):
        for h in range(n_heads):
            for j in range(half):
                theta = fr((pos0 + t) * float(inv_freq[j]))
                c = fr(math.cos(theta))
                s = fr(math.sin(theta))
                base = (t * n_heads + h) * head_dim
                ia = base + (j if neox else j * 2)
                ib = base + (j + half if neox else j * 2 + 1)
                a, b = out[ia], out[ib]
                out[ia] = fr(-b * s + fr(a * c))
                out[ib] = fr(b * c + fr(a * s))
    return np.array(out, np.float32)


def swiglu(gate, up):
    """ops_ref.ts:103"""
    return np.array([fr(fr(fr(float(g) / fr(1 + fr(math.exp(-float(g))))) * float(u)))
                     for g, u in zip(gate, up)], np.float32)


def attn(q, k, v, n_heads, n_kv_heads, head_dim, n_keys):
    """ops_ref.ts:135"""
    out = np.zeros(n_heads * head_dim, np.float32)
    group = n_heads // n_kv_heads
    scale = fr(1 / math.sqrt(head_dim))
    for h in range(n_heads):
        kvh = h // group
        scores = [0.0] * n_keys
        for t in range(n_keys):
            acc = 0.0
            for i in range(head_dim):
                acc = fma32(float(q[h * head_dim + i]),
                            float(k[(t * n_kv_heads + kvh) * head_dim + i]), acc)
            scores[t] = fr(acc * scale)
        mx = -math.inf
        for t in range(n_keys):
            mx = max(mx, scores[t])
        s = 0.0
        for t in range(n_keys):
            scores[t] = fr(math.exp(fr(scores[t] - mx)))
            s = fr(s + scores[t])
        inv = fr(1 / s)
        for i in range(head_dim):
            acc = 0.0
            for t in range(n_keys):
                acc = fma32(scores[t], float(v[(t * n_kv_heads + kvh) * head_dim + i]), acc)
            out[h * head_dim + i] = fr(acc * inv)
    return out


def attn_prefill(q, k, v, n_heads, n_kv_heads, head_dim, n_queries, pos0, tile=64, wg=128):
    """head_ref.ts:99"""
    out = np.zeros(n_queries * n_heads * head_dim, np.float32)
    group = n_heads // n_kv_heads
    scale = fr(1 / math.sqrt(head_dim))

    def tree(a, f):
        buf = list(a)
        stride = len(buf) >> 1
        while stride > 0:
            for i in range(stride):
                buf[i] = fr(f(buf[i], buf[i + stride]))
            stride >>= 1
        return buf[0]

    for qi in range(n_queries):
        for h in range(n_heads):
            kvh = h // group
            qbase = (qi * n_heads + h) * head_dim
            n_keys = pos0 + qi + 1
            m, l = -math.inf, 0.0
            acc = [0.0] * head_dim
            for base in range(0, n_keys, tile):
                n_this = min(tile, n_keys - base)
                tile_s = [0.0] * tile
                for j in range(n_this):
                    kb = ((base + j) * n_kv_heads + kvh) * head_dim
                    s = 0.0
                    for i in range(head_dim):
                        s = fma32(float(q[qbase + i]), float(k[kb + i]), s)
                    tile_s[j] = fr(s * scale)
                part = [-math.inf] * wg
                for t in range(wg):
                    tm = -math.inf
                    for j in range(t, n_this, wg):
                        tm = max(tm, tile_s[j])
                    part[t] = fr(tm)
                tile_max = tree(part, max)
                m_new = max(m, tile_max)
                corr = fr(math.exp(fr(m - m_new)))
                part = [0.0] * wg
                for t in range(wg):
                    ts = 0.0
                    for j in range(t, n_this, wg):
                        e = fr(math.exp(fr(tile_s[j] - m_new)))
                        tile_s[j] = e
                        ts = fr(ts + e)
                    part[t] = ts
                tile_sum = tree(part, lambda a, b: fr(a + b))
                for i in range(head_dim):
                    a = fr(acc[i] * corr)
                    for j in range(n_this):
                        a = fma32(tile_s[j], float(v[((base + j) * n_kv_heads + kvh) * head_dim + i]),
                                  a)
                    acc[i] = a
                l = fma32(l, corr, tile_sum)
                m = m_new
            for i in range(head_dim):
                out[qbase + i] = fr(acc[i] / l)
    return out


def embed(packed: bytes, ids, cols):
    """head_ref.ts:34"""
    nb = cols // 32
    out = np.zeros(len(ids) * cols, np.float32)
    for t, row in enumerate(ids):
        for b in range(nb):
            base = row * nb * 34 + b * 34
            scale = fr(half_to_f32(struct.unpack_from("<H", packed, base)[0]))
            for i in range(32):
                q = packed[base + 2 + i]
                if q > 127:
                    q -= 256
                out[t * cols + b * 32 + i] = fr(q * scale)
    return out


def argmax(x) -> int:
    """head_ref.ts:65"""
    bi, bv = 0, float(x[0])
    for i in range(1, len(x)):
        if float(x[i]) > bv:
            bv = float(x[i])
            bi = i
    return bi


def shard_ranges(total, n, align=1):
    """shard_ref.ts:97"""
    if n < 1:
        raise ValueError(f"n shards must be >= 1, got {n}")
    if total < 0:
        raise ValueError(f"total must be >= 0, got {total}")
    if align < 1:
        raise ValueError(f"align must be >= 1, got {align}")
    if total % align != 0:
        raise ValueError(f"total {total} is not a multiple of align {align}")
    units = total // align
    if units < n:
        raise ValueError(f"cannot cut {total} into {n} shards aligned to {align}: only {units} units")
    base, extra = units // n, units % n
    out, at = [], 0
    for i in range(n):
        count = (base + (1 if i < extra else 0)) * align
        out.append((at, count))
        at += count
    return out
