"""Python front end of libqora_mixer.so (the B200 QORA-4B token-mixer library).

Mirrors the reference's mixer call surface (qora-protocol/QORA-LLM-4B):
  DnState        <-> DeltaNetState          (src/gemv.rs:133-157)
  KvCache        <-> KvCacheEntry           (src/gemv.rs:164-168)
  Mixer.dn_decode   <-> forward_deltanet_decode mixer region (gemv.rs:744-883)
  Mixer.gqa_decode  <-> forward_attn_decode attention region (gemv.rs:927-1011)
  Mixer.dn_prefill  <-> prefill_deltanet_layer loop (gemv.rs:1119-1219)
  Mixer.gqa_prefill <-> prefill_attn_layer attention (gemv.rs:1364-1444)
plus the multi-GPU pieces the reference does not have (shard_plan, Comm:
head-sharded states/caches and the all-gather of their outputs),
and raises QmError where the reference panics (layer/cache mismatch).

Everything runs through the C ABI declared in include/qora_mixer.h.  torch is
used only to own device memory and streams.  There is no CPU fallback: if
the shared library is missing, importing the bindings raises.
"""
from __future__ import annotations

import ctypes as C
import os
import weakref

_HERE = os.path.dirname(os.path.abspath(__file__))
PKG_DIR = os.path.dirname(_HERE)
# QORA_MIXER_LIB selects another build of the same ABI (the checked build,
# libqora_mixer_checked.so, for the device-side bounds self-check tests)
LIB_PATH = os.environ.get("QORA_MIXER_LIB") or os.path.join(PKG_DIR, "libqora_mixer.so")

QM_OK = 0
STATUS = {
    1: "QM_E_ARG", 2: "QM_E_SHAPE", 3: "QM_E_OOM", 4: "QM_E_CUDA", 5: "QM_E_NCCL",
    6: "QM_E_TIMEOUT", 7: "QM_E_RANGE", 8: "QM_E_MISMATCH", 9: "QM_E_UNSUPPORTED",
    10: "QM_E_CAPTURE",
}

# Every symbol include/qora_mixer.h declares (checked by the CPU test suite).
EXPORTS = [
    "qm_build_flags", "qm_shape_get", "qm_status_string", "qm_ctx_create", "qm_ctx_destroy", "qm_ctx_set_stream",
    "qm_ctx_get_stream", "qm_sync", "qm_last_error", "qm_ctx_reserve", "qm_ctx_set_host_parts",
    "qm_ctx_set_host_direct", "qm_ctx_host_calls", "qm_ctx_launch_count",
    "qm_ctx_set_timing", "qm_ctx_kernel_time",
    "qm_rope_table", "qm_dn_state_create", "qm_dn_state_wrap", "qm_dn_state_destroy",
    "qm_dn_state_reset", "qm_dn_state_snapshot", "qm_dn_state_restore", "qm_dn_state_read",
    "qm_dn_state_write", "qm_dn_state_conv_pos", "qm_dn_state_set_conv_pos",
    "qm_dn_state_batch", "qm_dn_state_data", "qm_dn_decode", "qm_dn_decode_host", "qm_dn_decode_seq",
    "qm_dn_prefill", "qm_dn_prefill_host", "qm_kv_create", "qm_kv_wrap", "qm_kv_destroy", "qm_kv_snapshot",
    "qm_kv_restore", "qm_kv_seq_len", "qm_kv_set_seq_len", "qm_kv_capacity", "qm_kv_batch",
    "qm_kv_data", "qm_gqa_decode", "qm_gqa_decode_host", "qm_gqa_prefill", "qm_gqa_prefill_host",
    "qm_gqa_decode_noalloc",
    "qm_dn_state_create_heads", "qm_dn_state_wrap_heads", "qm_dn_state_heads",
    "qm_kv_create_heads", "qm_kv_wrap_heads", "qm_kv_heads",
    "qm_gemv", "qm_gemv_multi", "qm_gemm", "qm_gemm_bf16", "qm_logits_penalize", "qm_sample", "qm_shard_plan", "qm_comm_unique_id", "qm_comm_create", "qm_comm_allgather",
    "qm_comm_enable_peer",
    "qm_comm_destroy",
]
COMM_ID_BYTES = 128


class QmError(RuntimeError):
    def __init__(self, code, msg=""):
        self.code = code
        super().__init__(f"{STATUS.get(code, code)}: {msg}")


class QmShape(C.Structure):
    _fields_ = [("num_qk_heads", C.c_int), ("num_v_heads", C.c_int), ("dn_head_dim", C.c_int),
                ("conv_kernel", C.c_int), ("num_attn_heads", C.c_int), ("num_kv_heads", C.c_int),
                ("attn_head_dim", C.c_int), ("rope_dim", C.c_int), ("rope_theta", C.c_float),
                ("rms_eps", C.c_float)]


class QmDnParams(C.Structure):
    _fields_ = [("conv_w", C.c_void_p), ("a_log", C.c_void_p), ("dt_bias", C.c_void_p),
                ("norm_gamma", C.c_void_p)]


class QmGqaParams(C.Structure):
    _fields_ = [("q_norm", C.c_void_p), ("k_norm", C.c_void_p), ("rope_cos", C.c_void_p),
                ("rope_sin", C.c_void_p), ("max_pos", C.c_int)]


class QmWeight(C.Structure):
    _fields_ = [("kind", C.c_int), ("k", C.c_int), ("n", C.c_int), ("data", C.c_void_p),
                ("scales", C.c_void_p)]


W_F16, W_Q4, W_F16_ROWS, W_Q4_ROWS = 0, 1, 2, 3


class QmShard(C.Structure):
    _fields_ = [("world", C.c_int), ("rank", C.c_int), ("vh_lo", C.c_int), ("nvh", C.c_int),
                ("kv_lo", C.c_int), ("nkv", C.c_int), ("seq_part", C.c_int),
                ("seq_parts", C.c_int)]


_lib = None


def lib():
    """Load the shared library (raises if it was not built)."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise ImportError(f"{LIB_PATH} is missing: build it with `make -C {PKG_DIR}` "
                          "(there is no CPU fallback)")
    L = C.CDLL(LIB_PATH)
    P, I, I64 = C.c_void_p, C.c_int, C.c_int64
    PP = C.POINTER(C.c_void_p)
    sig = {
        "qm_shape_get": ([C.POINTER(QmShape)], I),
        "qm_status_string": ([I], C.c_char_p),
        "qm_ctx_create": ([I, PP], I),
        "qm_ctx_destroy": ([P], I),
        "qm_ctx_set_stream": ([P, P], I),
        "qm_ctx_get_stream": ([P], P),
        "qm_sync": ([P], I),
        "qm_last_error": ([P], C.c_char_p),
        "qm_ctx_reserve": ([P, C.c_size_t], I),
        "qm_ctx_set_host_parts": ([P, I, I], I),
        "qm_ctx_set_host_direct": ([P, I], I),
        "qm_ctx_host_calls": ([P, C.POINTER(I64), C.POINTER(I64)], I),
        "qm_ctx_launch_count": ([P], I64),
        "qm_ctx_set_timing": ([P, I], I),
        "qm_ctx_kernel_time": ([P, C.c_char_p, C.POINTER(C.c_double), C.POINTER(C.c_int64)], I),
        "qm_rope_table": ([C.c_float, I, I, P, P], I),
        "qm_dn_state_create": ([P, I, PP], I),
        "qm_dn_state_wrap": ([P, I, P, P, PP], I),
        "qm_dn_state_destroy": ([P], I),
        "qm_dn_state_reset": ([P, P], I),
        "qm_dn_state_snapshot": ([P, P, PP], I),
        "qm_dn_state_restore": ([P, P, P], I),
        "qm_dn_state_read": ([P, P, I, P, P], I),
        "qm_dn_state_write": ([P, P, I, P, P], I),
        "qm_dn_state_conv_pos": ([P], I64),
        "qm_dn_state_set_conv_pos": ([P, I64], I),
        "qm_dn_state_batch": ([P], I),
        "qm_dn_state_data": ([P, PP, PP], I),
        "qm_dn_decode": ([P, C.POINTER(QmDnParams), P, P, P, P, P, P, P], I),
        "qm_dn_decode_host": ([P, C.POINTER(QmDnParams), P, P, P, P, P, P, P], I),
        "qm_dn_prefill": ([P, C.POINTER(QmDnParams), P, I, P, P, P, P, P, P], I),
        "qm_dn_decode_seq": ([P, C.POINTER(QmDnParams), P, I, P, P, P, P, P, P], I),
        "qm_build_flags": ([], I),
        "qm_dn_prefill_host": ([P, C.POINTER(QmDnParams), P, I, P, P, P, P, P, P], I),
        "qm_gqa_prefill_host": ([P, C.POINTER(QmGqaParams), P, I, P, P, P, P], I),
        "qm_kv_create": ([P, I, I, PP], I),
        "qm_kv_wrap": ([P, I, I, P, P, PP], I),
        "qm_kv_destroy": ([P], I),
        "qm_kv_snapshot": ([P, P, PP], I),
        "qm_kv_restore": ([P, P, P], I),
        "qm_kv_seq_len": ([P], I64),
        "qm_kv_set_seq_len": ([P, I64], I),
        "qm_kv_capacity": ([P], I),
        "qm_kv_batch": ([P], I),
        "qm_kv_data": ([P, PP, PP], I),
        "qm_gqa_decode": ([P, C.POINTER(QmGqaParams), P, P, P, P, P], I),
        "qm_gqa_decode_host": ([P, C.POINTER(QmGqaParams), P, P, P, P, P], I),
        "qm_gqa_prefill": ([P, C.POINTER(QmGqaParams), P, I, P, P, P, P], I),
        "qm_gqa_decode_noalloc": ([C.POINTER(QmGqaParams), P, P, I, I, I64, P, P, P, P, P], I),
        "qm_dn_state_create_heads": ([P, I, I, I, PP], I),
        "qm_dn_state_wrap_heads": ([P, I, I, I, P, P, PP], I),
        "qm_dn_state_heads": ([P, C.POINTER(I), C.POINTER(I)], I),
        "qm_kv_create_heads": ([P, I, I, I, I, PP], I),
        "qm_kv_wrap_heads": ([P, I, I, I, I, P, P, PP], I),
        "qm_kv_heads": ([P, C.POINTER(I), C.POINTER(I)], I),
        "qm_shard_plan": ([I, I, C.POINTER(QmShard)], I),
        "qm_gemv": ([P, C.POINTER(QmWeight), I, P, P], I),
        "qm_gemv_multi": ([P, C.POINTER(QmWeight), I, I, P, C.POINTER(C.c_void_p)], I),
        "qm_gemm": ([P, C.POINTER(QmWeight), I, P, P], I),
        "qm_gemm_bf16": ([P, C.POINTER(QmWeight), I, P, P], I),
        "qm_logits_penalize": ([P, P, I, I, P, P, I, C.c_float, C.c_float, I], I),
        "qm_sample": ([P, P, I, I, C.c_float, C.c_float, I, P, P], I),
        "qm_comm_unique_id": ([P], I),
        "qm_comm_create": ([P, P, I, I, I, PP], I),
        "qm_comm_allgather": ([P, P, P, C.c_size_t], I),
        "qm_comm_enable_peer": ([P, C.c_size_t, I], I),
        "qm_comm_destroy": ([P], I),
    }
    for name, (args, res) in sig.items():
        if hasattr(L, name):
            fn = getattr(L, name)
            fn.argtypes = args
            fn.restype = res
    _lib = L
    return L


def _ptr(t):
    """Device/host address of a torch tensor or numpy array (None -> NULL)."""
    if t is None:
        return None
    if hasattr(t, "data_ptr"):
        assert t.is_contiguous(), "tensors passed to the mixer must be contiguous"
        return t.data_ptr()
    assert t.flags["C_CONTIGUOUS"]
    return t.ctypes.data


def shape():
    s = QmShape()
    lib().qm_shape_get(C.byref(s))
    return s


def rope_table(theta=1.0e7, rope_dim=64, max_pos=8192):
    """Host tables from the reference formula (src/convert.rs:161-176), any max_pos."""
    import numpy as np

    half = rope_dim // 2
    cos = np.empty((max_pos, half), np.float32)
    sin = np.empty((max_pos, half), np.float32)
    rc = lib().qm_rope_table(C.c_float(theta), rope_dim, max_pos, cos.ctypes.data, sin.ctypes.data)
    if rc:
        raise QmError(rc, "qm_rope_table")
    return cos, sin


class Ctx:
    """One device + one stream (qm_ctx)."""

    def __init__(self, device: int = 0, stream=None):
        self._h = C.c_void_p()
        rc = lib().qm_ctx_create(device, C.byref(self._h))
        if rc:
            raise QmError(rc, "qm_ctx_create")
        self.device = device
        self._children = weakref.WeakSet()
        if stream is not None:
            self.set_stream(stream)

    @property
    def handle(self):
        return self._h

    def check(self, rc, what=""):
        if rc != QM_OK:
            msg = lib().qm_last_error(self._h)
            raise QmError(rc, f"{what}: {msg.decode() if msg else ''}")

    def set_stream(self, stream):
        """stream: a torch.cuda.Stream or a raw cudaStream_t int (0 = legacy default)."""
        raw = getattr(stream, "cuda_stream", stream)
        self.check(lib().qm_ctx_set_stream(self._h, raw or None), "set_stream")

    def adopt(self, child):
        self._children.add(child)

    def sync(self):
        self.check(lib().qm_sync(self._h), "qm_sync")

    def reserve(self, nbytes):
        self.check(lib().qm_ctx_reserve(self._h, int(nbytes)), "reserve")

    def set_host_parts(self, dn_parts=0, gqa_parts=0):
        """Overlapped parts of the _host variants (0: default)."""
        self.check(lib().qm_ctx_set_host_parts(self._h, int(dn_parts), int(gqa_parts)),
                   "set_host_parts")

    def set_host_direct(self, on=True):
        """_host calls on page-locked buffers run the kernels on them in place."""
        self.check(lib().qm_ctx_set_host_direct(self._h, int(bool(on))), "set_host_direct")

    def host_calls(self):
        """(in-place, staged) counts of the _host calls made on this context."""
        a, b = C.c_int64(), C.c_int64()
        self.check(lib().qm_ctx_host_calls(self._h, C.byref(a), C.byref(b)), "host_calls")
        return a.value, b.value

    def launch_count(self) -> int:
        return int(lib().qm_ctx_launch_count(self._h))

    def set_timing(self, on: bool):
        self.check(lib().qm_ctx_set_timing(self._h, int(bool(on))), "set_timing")

    def kernel_time(self, name: str):
        """(total device ms, launches) of kernel `name` since timing was turned on."""
        ms, n = C.c_double(), C.c_int64()
        self.check(lib().qm_ctx_kernel_time(self._h, name.encode(), C.byref(ms), C.byref(n)),
                   "kernel_time")
        return ms.value, n.value

    def close(self):
        if self._h:
            for ch in list(self._children):
                ch.close()
            lib().qm_ctx_destroy(self._h)
            self._h = C.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class DnState:
    """B DeltaNet recurrent states (DeltaNetState x B), owned or wrapping torch storage.

    heads=(vh_lo, nvh) makes a head-sharded state holding V heads
    [vh_lo, vh_lo+nvh) only (decode only; see shard_plan)."""

    def __init__(self, ctx: Ctx, batch: int, s=None, conv=None, heads=None):
        self.ctx = ctx
        self._h = C.c_void_p()
        self._keep = (s, conv)
        lo, n = heads if heads is not None else (0, 32)
        if s is None:
            rc = lib().qm_dn_state_create_heads(ctx.handle, batch, lo, n, C.byref(self._h))
        else:
            rc = lib().qm_dn_state_wrap_heads(ctx.handle, batch, lo, n, _ptr(s), _ptr(conv),
                                              C.byref(self._h))
        ctx.check(rc, "dn_state create")
        self.batch = batch
        self.heads = (lo, n)
        ctx.adopt(self)

    @property
    def handle(self):
        return self._h

    @property
    def conv_pos(self) -> int:
        return int(lib().qm_dn_state_conv_pos(self._h))

    @conv_pos.setter
    def conv_pos(self, v):
        self.ctx.check(lib().qm_dn_state_set_conv_pos(self._h, int(v)), "set_conv_pos")

    def reset(self):
        self.ctx.check(lib().qm_dn_state_reset(self.ctx.handle, self._h), "reset")

    def snapshot(self) -> "DnState":
        o = DnState.__new__(DnState)
        o.ctx, o.batch, o.heads, o._keep = self.ctx, self.batch, self.heads, (None, None)
        o._h = C.c_void_p()
        self.ctx.check(lib().qm_dn_state_snapshot(self.ctx.handle, self._h, C.byref(o._h)), "snapshot")
        self.ctx.adopt(o)
        return o

    def restore_from(self, src: "DnState"):
        self.ctx.check(lib().qm_dn_state_restore(self.ctx.handle, self._h, src._h), "restore")

    def read(self, b: int):
        """(S [nvh,128,128], conv_buf [8192,3]) of sequence b, reference layout."""
        import numpy as np

        s = np.empty((self.heads[1], 128, 128), np.float32)
        cb = np.empty((8192, 3), np.float32)
        self.ctx.check(lib().qm_dn_state_read(self.ctx.handle, self._h, b, s.ctypes.data,
                                              cb.ctypes.data), "read")
        return s, cb

    def write(self, b: int, s=None, conv_buf=None):
        import numpy as np

        sp = None if s is None else np.ascontiguousarray(s, np.float32)
        cp = None if conv_buf is None else np.ascontiguousarray(conv_buf, np.float32)
        self.ctx.check(lib().qm_dn_state_write(self.ctx.handle, self._h, b, _ptr(sp), _ptr(cp)),
                       "write")

    def close(self):
        if self._h:
            lib().qm_dn_state_destroy(self._h)
            self._h = C.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class KvCache:
    """B bf16 KV caches [B,nkv,capacity,256] (KvCacheEntry x B).

    heads=(kv_lo, nkv) makes a head-sharded cache of KV heads
    [kv_lo, kv_lo+nkv) (decode only; see shard_plan)."""

    def __init__(self, ctx: Ctx, batch: int, capacity: int, k=None, v=None, heads=None):
        self.ctx = ctx
        self._h = C.c_void_p()
        self._keep = (k, v)
        lo, n = heads if heads is not None else (0, 4)
        if k is None:
            rc = lib().qm_kv_create_heads(ctx.handle, batch, capacity, lo, n, C.byref(self._h))
        else:
            rc = lib().qm_kv_wrap_heads(ctx.handle, batch, capacity, lo, n, _ptr(k), _ptr(v),
                                        C.byref(self._h))
        ctx.check(rc, "kv create")
        self.batch, self.capacity, self.heads = batch, capacity, (lo, n)
        ctx.adopt(self)

    @property
    def handle(self):
        return self._h

    @property
    def seq_len(self) -> int:
        return int(lib().qm_kv_seq_len(self._h))

    @seq_len.setter
    def seq_len(self, n):
        rc = lib().qm_kv_set_seq_len(self._h, int(n))
        if rc:
            raise QmError(rc, "set_seq_len")

    def data_ptrs(self):
        k, v = C.c_void_p(), C.c_void_p()
        lib().qm_kv_data(self._h, C.byref(k), C.byref(v))
        return k.value, v.value

    def snapshot(self) -> "KvCache":
        o = KvCache.__new__(KvCache)
        o.ctx, o.batch, o.capacity, o.heads = self.ctx, self.batch, self.capacity, self.heads
        o._keep = (None, None)
        o._h = C.c_void_p()
        self.ctx.check(lib().qm_kv_snapshot(self.ctx.handle, self._h, C.byref(o._h)), "kv snapshot")
        self.ctx.adopt(o)
        return o

    def restore_from(self, src: "KvCache"):
        self.ctx.check(lib().qm_kv_restore(self.ctx.handle, self._h, src._h), "kv restore")

    def close(self):
        if self._h:
            lib().qm_kv_destroy(self._h)
            self._h = C.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def dn_params(conv_w, a_log, dt_bias, norm_gamma=None) -> QmDnParams:
    """Device tensors -> qm_dn_params (keep the tensors alive while in use)."""
    return QmDnParams(_ptr(conv_w), _ptr(a_log), _ptr(dt_bias), _ptr(norm_gamma))


def weight_q4(packed, scales) -> QmWeight:
    """Device Q4 weight (packed uint8 [k, n/2], f16 scale bits [k, n/32]) -> qm_weight."""
    k, n = int(packed.shape[0]), int(packed.shape[1]) * 2
    w = QmWeight(W_Q4, k, n, _ptr(packed), _ptr(scales))
    w._keep = (packed, scales)  # the descriptor holds raw pointers: keep the buffers alive with it
    return w


def weight_f16(w16) -> QmWeight:
    """Device f16 weight [k, n] (f16 or its bits) -> qm_weight."""
    w = QmWeight(W_F16, int(w16.shape[0]), int(w16.shape[1]), _ptr(w16), None)
    w._keep = (w16,)
    return w


def weight_q4_rows(packed, scales) -> QmWeight:
    """Device Q4 rows (packed uint8 [n, k/2], f16 scale bits [n, k/32]): the tied embedding as lm_head."""
    n, k = int(packed.shape[0]), int(packed.shape[1]) * 2
    w = QmWeight(W_Q4_ROWS, k, n, _ptr(packed), _ptr(scales))
    w._keep = (packed, scales)
    return w


def weight_f16_rows(e16) -> QmWeight:
    """Device f16 rows [n, k] (f16 or its bits)."""
    w = QmWeight(W_F16_ROWS, int(e16.shape[1]), int(e16.shape[0]), _ptr(e16), None)
    w._keep = (e16,)
    return w


def gqa_params(q_norm, k_norm, rope_cos, rope_sin) -> QmGqaParams:
    return QmGqaParams(_ptr(q_norm), _ptr(k_norm), _ptr(rope_cos), _ptr(rope_sin),
                       int(rope_cos.shape[0]))


class Mixer:
    """Per-layer mixer calls on one context (the reference's per-layer forward)."""

    def __init__(self, ctx: Ctx):
        self.ctx = ctx

    def gemv(self, w: QmWeight, x, y):
        """y[batch, n] = x[batch, k] . W (qm_gemv); x, y device f32."""
        batch = int(x.shape[0]) if len(x.shape) == 2 else 1
        self.ctx.check(lib().qm_gemv(self.ctx.handle, C.byref(w), batch, _ptr(x), _ptr(y)), "qm_gemv")

    def penalize(self, logits, tokens=None, lens=None, repetition=1.0, presence=0.0, ban=-1):
        """qm_logits_penalize on device logits [batch, vocab]; tokens int32 [batch, stride], lens int32 [batch]."""
        batch, vocab = int(logits.shape[0]), int(logits.shape[1])
        stride = int(tokens.shape[1]) if tokens is not None else 0
        self.ctx.check(lib().qm_logits_penalize(self.ctx.handle, _ptr(logits), batch, vocab,
                                                _ptr(tokens) if tokens is not None else None,
                                                _ptr(lens) if lens is not None else None, stride,
                                                repetition, presence, ban), "qm_logits_penalize")

    def sample(self, logits, temperature, top_p, top_k, r, ids):
        """qm_sample: ids[b] from device logits [batch, vocab] and draws r [batch] (device f32)."""
        batch, vocab = int(logits.shape[0]), int(logits.shape[1])
        self.ctx.check(lib().qm_sample(self.ctx.handle, _ptr(logits), batch, vocab, temperature, top_p,
                                       top_k, _ptr(r) if r is not None else None, _ptr(ids)), "qm_sample")

    def gemm(self, w: QmWeight, x, y):
        """qm_gemm: y [T, n] f32 = x [T, k] bf16 (bits as int16) . W (Q4 or F16, either layout) on the tensor cores."""
        self.ctx.check(lib().qm_gemm(self.ctx.handle, C.byref(w), int(x.shape[0]), _ptr(x), _ptr(y)), "qm_gemm")

    def gemm_bf16(self, w: QmWeight, x, y):
        """qm_gemm_bf16: y [T, n] bf16 (bits as int16), the f32 sum rounded to nearest."""
        self.ctx.check(lib().qm_gemm_bf16(self.ctx.handle, C.byref(w), int(x.shape[0]), _ptr(x), _ptr(y)),
                       "qm_gemm_bf16")

    def gemv_multi(self, ws, x, ys):
        """ys[i][batch, n_i] = x[batch, k] . W_i for up to 4 weights sharing x (qm_gemv_multi)."""
        batch = int(x.shape[0]) if len(x.shape) == 2 else 1
        arr = (QmWeight * len(ws))(*ws)
        yp = (C.c_void_p * len(ys))(*[_ptr(y) for y in ys])
        self.ctx.check(lib().qm_gemv_multi(self.ctx.handle, arr, len(ws), batch, _ptr(x), yp),
                       "qm_gemv_multi")

    def dn_decode(self, p: QmDnParams, st: DnState, qkv, a, b, y=None, z=None, out=None):
        rc = lib().qm_dn_decode(self.ctx.handle, C.byref(p), st.handle, _ptr(qkv), _ptr(a),
                                _ptr(b), _ptr(y), _ptr(z), _ptr(out))
        self.ctx.check(rc, "qm_dn_decode")

    def dn_decode_host(self, p: QmDnParams, st: DnState, qkv, a, b, y=None, z=None, out=None):
        rc = lib().qm_dn_decode_host(self.ctx.handle, C.byref(p), st.handle, _ptr(qkv), _ptr(a),
                                     _ptr(b), _ptr(y), _ptr(z), _ptr(out))
        self.ctx.check(rc, "qm_dn_decode_host")

    def dn_decode_seq(self, p: QmDnParams, st: DnState, T, qkv, a, b, y=None, z=None, out=None):
        """T decode steps per sequence in one launch (qkv [B,T,8192] f32)."""
        rc = lib().qm_dn_decode_seq(self.ctx.handle, C.byref(p), st.handle, int(T), _ptr(qkv),
                                    _ptr(a), _ptr(b), _ptr(y), _ptr(z), _ptr(out))
        self.ctx.check(rc, "qm_dn_decode_seq")

    def dn_prefill(self, p: QmDnParams, st: DnState, T, qkv_bf16, a, b, y=None, z=None, out=None):
        rc = lib().qm_dn_prefill(self.ctx.handle, C.byref(p), st.handle, int(T), _ptr(qkv_bf16),
                                 _ptr(a), _ptr(b), _ptr(y), _ptr(z), _ptr(out))
        self.ctx.check(rc, "qm_dn_prefill")

    def gqa_decode(self, p: QmGqaParams, kv: KvCache, q_gate, k_new, v_new, out):
        rc = lib().qm_gqa_decode(self.ctx.handle, C.byref(p), kv.handle, _ptr(q_gate),
                                 _ptr(k_new), _ptr(v_new), _ptr(out))
        self.ctx.check(rc, "qm_gqa_decode")

    def gqa_decode_host(self, p: QmGqaParams, kv: KvCache, q_gate, k_new, v_new, out):
        rc = lib().qm_gqa_decode_host(self.ctx.handle, C.byref(p), kv.handle, _ptr(q_gate),
                                      _ptr(k_new), _ptr(v_new), _ptr(out))
        self.ctx.check(rc, "qm_gqa_decode_host")

    def dn_prefill_host(self, p: QmDnParams, st: DnState, T, qkv_bf16, a, b, y, z=None, out=None):
        """qm_dn_prefill on host arrays (numpy / CPU tensors); returns after y (and out) are filled."""
        rc = lib().qm_dn_prefill_host(self.ctx.handle, C.byref(p), st.handle, int(T), _ptr(qkv_bf16),
                                      _ptr(a), _ptr(b), _ptr(y), _ptr(z), _ptr(out))
        self.ctx.check(rc, "qm_dn_prefill_host")

    def gqa_prefill_host(self, p: QmGqaParams, kv: KvCache, T, q_gate_bf16, k_bf16, v_bf16, out):
        """qm_gqa_prefill on host arrays; returns after out is filled."""
        rc = lib().qm_gqa_prefill_host(self.ctx.handle, C.byref(p), kv.handle, int(T), _ptr(q_gate_bf16),
                                       _ptr(k_bf16), _ptr(v_bf16), _ptr(out))
        self.ctx.check(rc, "qm_gqa_prefill_host")

    def gqa_prefill(self, p: QmGqaParams, kv: KvCache, T, q_gate_bf16, k_bf16, v_bf16, out):
        rc = lib().qm_gqa_prefill(self.ctx.handle, C.byref(p), kv.handle, int(T),
                                  _ptr(q_gate_bf16), _ptr(k_bf16), _ptr(v_bf16), _ptr(out))
        self.ctx.check(rc, "qm_gqa_prefill")


def gqa_decode_noalloc(p: QmGqaParams, k_cache, v_cache, batch, capacity, seq_len, q_gate, k_new,
                       v_new, out, stream=None):
    """qm_gqa_decode_noalloc: GQA decode for callers that cannot allocate device
    memory.  The caller owns the cache and its seq_len count.  Returns the status."""
    raw = getattr(stream, "cuda_stream", stream)
    return lib().qm_gqa_decode_noalloc(C.byref(p), _ptr(k_cache), _ptr(v_cache), int(batch),
                                       int(capacity), int(seq_len), _ptr(q_gate), _ptr(k_new),
                                       _ptr(v_new), _ptr(out), raw or None)


def shard_plan(world: int, rank: int) -> dict:
    """qm_shard_plan: the head-sharded layout of rank `rank` of `world`."""
    sh = QmShard()
    rc = lib().qm_shard_plan(int(world), int(rank), C.byref(sh))
    if rc:
        raise QmError(rc, f"qm_shard_plan({world}, {rank})")
    return {f: getattr(sh, f) for f, _ in QmShard._fields_}


def comm_unique_id() -> bytes:
    buf = (C.c_ubyte * COMM_ID_BYTES)()
    rc = lib().qm_comm_unique_id(buf)
    if rc:
        raise QmError(rc, "qm_comm_unique_id")
    return bytes(buf)


class Comm:
    """NCCL communicator of the head-sharded layout (qm_comm): all-gathers the
    per-layer mixer outputs on the context's stream."""

    def __init__(self, ctx: Ctx, uid: bytes, world: int, rank: int, timeout_ms: int = 60000):
        assert len(uid) == COMM_ID_BYTES
        self.ctx = ctx
        self._h = C.c_void_p()
        buf = (C.c_ubyte * COMM_ID_BYTES).from_buffer_copy(uid)
        ctx.check(lib().qm_comm_create(ctx.handle, buf, int(world), int(rank), int(timeout_ms),
                                       C.byref(self._h)), "qm_comm_create")
        self.world, self.rank = world, rank
        self.peer = False
        ctx.adopt(self)

    def allgather(self, send, recv):
        """recv (world x send.nbytes, contiguous) <- every rank's send, rank order."""
        nbytes = send.numel() * send.element_size() if hasattr(send, "numel") else send.nbytes
        self.ctx.check(lib().qm_comm_allgather(self._h, _ptr(send), _ptr(recv), nbytes),
                       "qm_comm_allgather")

    def enable_peer(self, max_bytes: int, wait_ms: int = 2000) -> bool:
        """Collective: gathers of at most max_bytes per rank go through the
        peer-memory kernel (qm_comm_enable_peer).  False when some rank cannot
        map the others' memory (NCCL stays in use)."""
        rc = lib().qm_comm_enable_peer(self._h, int(max_bytes), int(wait_ms))
        if rc == 9:  # QM_E_UNSUPPORTED
            return False
        self.ctx.check(rc, "qm_comm_enable_peer")
        self.peer = True
        return True

    def close(self):
        if self._h:
            lib().qm_comm_destroy(self._h)
            self._h = C.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
