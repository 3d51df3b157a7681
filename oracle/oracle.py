"""ctypes front-end of the CPU restatement (TEST INFRASTRUCTURE ONLY).

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline / reference
arm import this module, and only as the checker or as the timed CPU
baseline.  The product library never calls it.

PARITY UNPINNED: the reference (Rust) ships no tests or golden vectors and
cannot be built here; see qora_oracle.h for how the restatement is anchored.

All arrays are numpy, C-contiguous; shapes follow the reference layouts
(src/gemv.rs:133-168): DeltaNet state [num_v, hd, hd] with row = v-dim,
conv buffer [qkv_dim, ks-1], KV cache [seq, kv_heads, head_dim] f32.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "libqora_oracle.so")


class OrCfg(C.Structure):
    _fields_ = [
        ("num_qk_heads", C.c_int),
        ("num_v_heads", C.c_int),
        ("dn_head_dim", C.c_int),
        ("conv_kernel", C.c_int),
        ("num_attn_heads", C.c_int),
        ("num_kv_heads", C.c_int),
        ("attn_head_dim", C.c_int),
        ("rope_dim", C.c_int),
    ]


def build() -> str:
    """Compile the restatement with its Makefile (gcc only)."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


_lib = None


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            build()
        L = C.CDLL(_LIB_PATH)
        P = C.c_void_p
        L.or_cfg_default_4b.argtypes = [C.POINTER(OrCfg)]
        L.or_has_avx512.restype = C.c_int
        L.or_num_threads.restype = C.c_int
        L.or_set_num_threads.argtypes = [C.c_int]
        L.or_rope_table.argtypes = [C.c_float, C.c_int, C.c_int, P, P]
        L.or_dn_decode.argtypes = [C.POINTER(OrCfg)] + [P] * 9 + [C.c_int, P, P, P, P]
        L.or_dn_prefill.argtypes = [C.POINTER(OrCfg), C.c_int] + [P] * 10 + [C.c_int, C.c_int, P, P, P]
        L.or_gqa_decode.argtypes = [C.POINTER(OrCfg)] + [P] * 7 + [C.c_int] + [P] * 4
        L.or_gqa_decode.restype = C.c_int
        L.or_gqa_prefill_rows.argtypes = (
            [C.POINTER(OrCfg), C.c_int] + [P] * 10 + [C.c_int, P, C.c_int, P, P, P]
        )
        L.or_gqa_prefill_rows.restype = C.c_int
        L.or_quantize_q4.argtypes = [P, C.c_int, C.c_int, P, P]
        L.or_gemv_q4.argtypes = [P, P, P, C.c_int, C.c_int, P]
        L.or_gemv_f16.argtypes = [P, P, C.c_int, C.c_int, P]
        L.or_lm_head_f16.argtypes = [P, P, C.c_int, C.c_int, P]
        L.or_lm_head_q4.argtypes = [P, P, P, C.c_int, C.c_int, P]
        L.or_repetition_penalty.argtypes = [P, C.c_int, P, C.c_int, C.c_float]
        L.or_presence_penalty.argtypes = [P, C.c_int, P, C.c_int, C.c_float]
        L.or_sample_top_k.argtypes = [P, C.c_int, C.c_float, C.c_float, C.c_int, C.c_float,
                                      C.POINTER(C.c_double)]
        L.or_sample_top_k.restype = C.c_int
        L.or_rng_next_f32.argtypes = [C.POINTER(C.c_uint64)]
        L.or_rng_next_f32.restype = C.c_float
        _lib = L
    return _lib


def cfg_4b() -> OrCfg:
    c = OrCfg()
    lib().or_cfg_default_4b(C.byref(c))
    return c


def cfg(**kw) -> OrCfg:
    c = cfg_4b()
    for k, v in kw.items():
        setattr(c, k, v)
    return c


def _p(a):
    if a is None:
        return None
    assert a.flags["C_CONTIGUOUS"], "oracle arrays must be C-contiguous"
    return a.ctypes.data


def _f32(a):
    return np.ascontiguousarray(a, dtype=np.float32)


def has_avx512() -> bool:
    return bool(lib().or_has_avx512())


def num_threads() -> int:
    return lib().or_num_threads()


def set_num_threads(n: int) -> None:
    lib().or_set_num_threads(int(n))


def rope_table(theta: float = 1.0e7, rope_dim: int = 64, max_pos: int = 8192):
    """src/convert.rs:161-176 (extended to any max_pos)."""
    half = rope_dim // 2
    cos = np.empty((max_pos, half), np.float32)
    sin = np.empty((max_pos, half), np.float32)
    lib().or_rope_table(C.c_float(theta), rope_dim, max_pos, _p(cos), _p(sin))
    return cos, sin


class DnState:
    """Mirror of DeltaNetState (src/gemv.rs:133-157): zero-initialised."""

    def __init__(self, c: OrCfg):
        qkv = (2 * c.num_qk_heads + c.num_v_heads) * c.dn_head_dim
        self.s = np.zeros((c.num_v_heads, c.dn_head_dim, c.dn_head_dim), np.float32)
        self.conv_buf = np.zeros((qkv, c.conv_kernel - 1), np.float32)
        self.conv_pos = np.zeros(1, np.int64)

    def copy(self):
        o = DnState.__new__(DnState)
        o.s = self.s.copy()
        o.conv_buf = self.conv_buf.copy()
        o.conv_pos = self.conv_pos.copy()
        return o


def dn_decode(c, st: DnState, qkv, a, b, conv_w, a_log, dt_bias, use_avx512=True,
              z=None, norm_gamma=None):
    """src/gemv.rs:744-883 for one token.  Returns y [num_v, hd] (and gated)."""
    qkv, a, b = _f32(qkv), _f32(a), _f32(b)
    conv_w, a_log, dt_bias = _f32(conv_w), _f32(a_log), _f32(dt_bias)
    y = np.empty((c.num_v_heads, c.dn_head_dim), np.float32)
    gated = None
    if z is not None:
        z, norm_gamma = _f32(z), _f32(norm_gamma)
        gated = np.empty_like(y)
    lib().or_dn_decode(C.byref(c), _p(qkv), _p(a), _p(b), _p(conv_w), _p(a_log), _p(dt_bias),
                       _p(st.s), _p(st.conv_buf), _p(st.conv_pos), int(bool(use_avx512)),
                       _p(y), _p(z), _p(norm_gamma), _p(gated))
    return (y, gated) if z is not None else y


def dn_prefill(c, st: DnState, qkv, a, b, conv_w, a_log, dt_bias, vh_lo=0, vh_hi=None,
               z=None, norm_gamma=None):
    """src/gemv.rs:1119-1219 for T tokens (qkv f32, or uint16 bf16 bits)."""
    T = qkv.shape[0]
    qkv = np.ascontiguousarray(qkv)
    qf = qkv if qkv.dtype == np.float32 else None
    qb = qkv if qkv.dtype == np.uint16 else None
    assert qf is not None or qb is not None
    a, b = _f32(a), _f32(b)
    vh_hi = c.num_v_heads if vh_hi is None else vh_hi
    y = np.zeros((T, c.num_v_heads, c.dn_head_dim), np.float32)
    if z is not None:
        z, norm_gamma = _f32(z), _f32(norm_gamma)
    lib().or_dn_prefill(C.byref(c), T, _p(qf), _p(qb), _p(a), _p(b), _p(_f32(conv_w)),
                        _p(_f32(a_log)), _p(_f32(dt_bias)), _p(st.s), _p(st.conv_buf),
                        _p(st.conv_pos), int(vh_lo), int(vh_hi), _p(y), _p(z), _p(norm_gamma))
    return y


class KvCache:
    """Mirror of KvCacheEntry (src/gemv.rs:164-168) with preallocated rows."""

    def __init__(self, c: OrCfg, capacity: int, k=None, v=None):
        kvd = c.num_kv_heads * c.attn_head_dim
        self.k = np.zeros((capacity, c.num_kv_heads, c.attn_head_dim), np.float32)
        self.v = np.zeros_like(self.k)
        self.seq_len = np.zeros(1, np.int64)
        if k is not None:
            n = k.shape[0]
            self.k[:n] = k.reshape(n, c.num_kv_heads, c.attn_head_dim)
            self.v[:n] = v.reshape(n, c.num_kv_heads, c.attn_head_dim)
            self.seq_len[0] = n
        del kvd


def gqa_decode(c, kv: KvCache, q_gate, k_new, v_new, q_norm, k_norm, cos, sin):
    """src/gemv.rs:927-1011 for one token.  Returns out [H, D]."""
    out = np.empty((c.num_attn_heads, c.attn_head_dim), np.float32)
    if kv.seq_len[0] + 1 > kv.k.shape[0]:
        raise ValueError("oracle KV cache is full")
    rc = lib().or_gqa_decode(C.byref(c), _p(_f32(q_gate)), _p(_f32(k_new)), _p(_f32(v_new)),
                             _p(_f32(q_norm)), _p(_f32(k_norm)), _p(cos), _p(sin), cos.shape[0],
                             _p(kv.k), _p(kv.v), _p(kv.seq_len), _p(out))
    if rc != 0:
        raise ValueError("position beyond the RoPE table")
    return out


def gqa_prefill_rows(c, q_gate, k, v, q_norm, k_norm, cos, sin, rows, want_cache=False):
    """src/gemv.rs:1364-1444 for the query rows listed in `rows`.

    q_gate [S, H*2*D], k/v [S, KVH*D]; each f32 or uint16 (bf16 bits).
    Returns out [nrows, H, D] (and the f32 cache K/V [S, KVH, D]).
    """
    S = q_gate.shape[0]

    def split(x):
        x = np.ascontiguousarray(x)
        return (x, None) if x.dtype == np.float32 else (None, x)

    qf, qb = split(q_gate)
    kf, kb = split(k)
    vf, vb = split(v)
    rows = np.ascontiguousarray(rows, dtype=np.int32)
    out = np.empty((len(rows), c.num_attn_heads, c.attn_head_dim), np.float32)
    kc = vc = None
    if want_cache:
        kc = np.empty((S, c.num_kv_heads, c.attn_head_dim), np.float32)
        vc = np.empty_like(kc)
    rc = lib().or_gqa_prefill_rows(C.byref(c), S, _p(qf), _p(qb), _p(kf), _p(kb), _p(vf), _p(vb),
                                   _p(_f32(q_norm)), _p(_f32(k_norm)), _p(cos), _p(sin),
                                   cos.shape[0], _p(rows), len(rows), _p(out), _p(kc), _p(vc))
    if rc != 0:
        raise ValueError(f"or_gqa_prefill_rows failed ({rc})")
    return (out, kc, vc) if want_cache else out


def quantize_q4(w):
    """src/convert.rs:437-467: f32 [k, n] -> (packed uint8 [k, n/2], f16 scale bits uint16 [k, n/32])."""
    w = _f32(w)
    k, n = w.shape
    packed = np.empty((k, n // 2), np.uint8)
    scales = np.empty((k, n // 32), np.uint16)
    lib().or_quantize_q4(_p(w), k, n, _p(packed), _p(scales))
    return packed, scales


def dequantize_q4(packed, scales):
    """The weights a Q4 matrix stands for, f32 [k, n]: (q - 8) * f16 scale."""
    k = packed.shape[0]
    q = np.empty((k, packed.shape[1] * 2), np.float32)
    q[:, 0::2] = (packed & 0x0F).astype(np.float32) - 8.0
    q[:, 1::2] = (packed >> 4).astype(np.float32) - 8.0
    s = scales.view(np.float16).astype(np.float32)
    return q * np.repeat(s, 32, axis=1)


def gemv_q4(x, packed, scales):
    """src/gemv.rs:411-450 (scalar path): y[n] = x[k] . W_q4[k, n]."""
    x = _f32(x)
    k, n = packed.shape[0], packed.shape[1] * 2
    y = np.empty(n, np.float32)
    lib().or_gemv_q4(_p(x), _p(np.ascontiguousarray(packed)), _p(np.ascontiguousarray(scales)), k, n, _p(y))
    return y


def gemv_f16(x, w16):
    """src/gemv.rs:361-368 (scalar path): y[n] = x[k] . W_f16[k, n]; w16 = f16 bits uint16 [k, n]."""
    x = _f32(x)
    k, n = w16.shape
    y = np.empty(n, np.float32)
    lib().or_gemv_f16(_p(x), _p(np.ascontiguousarray(w16)), k, n, _p(y))
    return y


def lm_head_f16(x, e16):
    """src/gemv.rs:664-676: logits[v] = x . E[v] over f16 embedding rows (uint16 bits [vocab, hidden])."""
    x = _f32(x)
    vocab, hidden = e16.shape
    y = np.empty(vocab, np.float32)
    lib().or_lm_head_f16(_p(x), _p(np.ascontiguousarray(e16)), vocab, hidden, _p(y))
    return y


def lm_head_q4(x, packed, scales):
    """src/gemv.rs:677-707: the same over Q4 rows (packed uint8 [vocab, hidden/2], f16 bits [vocab, hidden/32])."""
    x = _f32(x)
    vocab, hidden = packed.shape[0], packed.shape[1] * 2
    y = np.empty(vocab, np.float32)
    lib().or_lm_head_q4(_p(x), _p(np.ascontiguousarray(packed)), _p(np.ascontiguousarray(scales)), vocab,
                        hidden, _p(y))
    return y


def penalize(logits, generated, repetition=1.0, presence=0.0, ban=-1):
    """src/generate.rs:58-83 in the order of the decode loop (185-196): repetition,
    then presence, then the banned token (-inf).  Returns a new array."""
    out = _f32(logits).copy()
    gen = np.ascontiguousarray(np.asarray(generated, np.int32))
    lib().or_repetition_penalty(_p(out), out.size, _p(gen), gen.size, repetition)
    lib().or_presence_penalty(_p(out), out.size, _p(gen), gen.size, presence)
    if ban >= 0:
        out[ban] = -np.inf
    return out


def sample_top_k(logits, temperature, top_p, top_k, r):
    """src/generate.rs:334-384 with the draw r given: (token, margin)."""
    lg = _f32(logits)
    m = C.c_double()
    tok = lib().or_sample_top_k(_p(lg), lg.size, temperature, top_p, top_k, r, C.byref(m))
    return int(tok), float(m.value)


class Rng:
    """The reference's xorshift64 (src/generate.rs:41-55) with a fixed seed."""

    def __init__(self, seed):
        self.state = C.c_uint64(seed | 1)

    def next_f32(self):
        return float(lib().or_rng_next_f32(C.byref(self.state)))
