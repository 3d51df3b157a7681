"""The .qor4b model file: read it, write it, and upload the mixer path.

The format is the reference's (src/save.rs): little-endian, a header (magic
"QOR4", version u32 1 or 2, format u8), the config (src/save.rs:263-281), the
layer types (one u8 each: 0 DeltaNet, 1 attention), then per layer its records
in a fixed order (src/save.rs:303-336), then the embedding, final norm and the
RoPE tables (342-345), then the optional vision encoder.  A weight record is
k u64, n u64, fmt u8 (0 F16, 1 Q4), then for F16 a vector of k*n f16, for Q4
a byte vector (k rows of n/2 bytes, the even column in the low nibble) and a
vector of k*n/32 f16 scales (src/save.rs:101-129); every vector is its length
u64 followed by the elements.

read_qor4b maps the file and returns zero-copy numpy views of every record.
write_qor4b writes the same layout (format version 2, no vision encoder); the
tests use it to build files.  upload_mixers copies what the mixer path uses
to the device: the projections as qm_weight descriptors, the DeltaNet and
GQA parameters (f16 norms widened to f32, the RoPE tables from the file), and
the embedding as row-layout lm_head weights.
"""
import struct
from dataclasses import dataclass, field

import numpy as np

MAGIC = b"QOR4"
VERSION = 2

# (name, kind): "u8" / "u32" / "f32" / "f64" scalars in file order (src/save.rs:263-281)
CONFIG_FIELDS = [
    ("vocab_size", "u32"), ("hidden_size", "u32"), ("num_layers", "u32"), ("num_attn_heads", "u32"),
    ("num_kv_heads", "u32"), ("attn_head_dim", "u32"), ("num_qk_heads", "u32"), ("num_v_heads", "u32"),
    ("deltanet_head_dim", "u32"), ("conv_kernel_size", "u32"), ("intermediate_size", "u32"),
    ("rope_theta", "f64"), ("partial_rotary_factor", "f32"), ("rms_norm_eps", "f64"),
    ("eos_token_id", "u32"), ("tie_word_embeddings", "u8"), ("has_vision", "u8"),
]
# per-layer records in file order: "w" a weight, "f32" / "f16" a vector (src/save.rs:303-336)
DELTANET_FIELDS = [
    ("in_proj_qkv", "w"), ("in_proj_a", "w"), ("in_proj_b", "w"), ("in_proj_z", "w"), ("out_proj", "w"),
    ("conv1d_weight", "f32"), ("a_log", "f32"), ("dt_bias", "f32"), ("attn_norm_weight", "f16"),
    ("gate_proj", "w"), ("up_proj", "w"), ("down_proj", "w"), ("input_norm", "f16"), ("post_attn_norm", "f16"),
]
ATTENTION_FIELDS = [
    ("q_proj", "w"), ("k_proj", "w"), ("v_proj", "w"), ("o_proj", "w"), ("q_norm", "f16"), ("k_norm", "f16"),
    ("gate_proj", "w"), ("up_proj", "w"), ("down_proj", "w"), ("input_norm", "f16"), ("post_attn_norm", "f16"),
]
GLOBAL_FIELDS = [("embed", "w"), ("final_norm", "f16"), ("rope_cos", "f32"), ("rope_sin", "f32")]

_SCALAR = {"u8": ("<B", 1), "u32": ("<I", 4), "u64": ("<Q", 8), "f32": ("<f", 4), "f64": ("<d", 8)}


class Qor4bError(ValueError):
    """A file the reference's loader would reject, or one whose records do not fit their shapes."""


@dataclass
class Weight:
    """One weight record: W [k rows][n cols] (src/gemv.rs:21-33)."""
    kind: str                  # "f16" or "q4"
    k: int
    n: int
    data: np.ndarray           # f16 bits uint16 [k, n], or packed uint8 [k, n/2]
    scales: np.ndarray = None  # q4: f16 bits uint16 [k, n/32]


@dataclass
class Model:
    version: int
    format_id: int
    config: dict
    layer_types: list          # 0 DeltaNet, 1 attention
    layers: list               # one dict of records per layer
    globals: dict
    vision_offset: int = -1    # byte offset of the vision encoder (not read), -1 without one
    extra: dict = field(default_factory=dict)


class _Cursor:
    def __init__(self, buf):
        self.buf = buf
        self.pos = 0

    def take(self, nbytes, what):
        if nbytes < 0 or self.pos + nbytes > len(self.buf):
            raise Qor4bError(f"truncated file: {what} needs {nbytes} bytes at offset {self.pos}")
        start = self.pos
        self.pos += nbytes
        return start

    def scalar(self, kind, what):
        fmt, size = _SCALAR[kind]
        start = self.take(size, what)
        return struct.unpack_from(fmt, self.buf, start)[0]

    def array(self, dtype, count, what):
        dtype = np.dtype(dtype)
        start = self.take(count * dtype.itemsize, what)
        return np.frombuffer(self.buf, dtype=dtype, count=count, offset=start)

    def vector(self, dtype, what):
        return self.array(dtype, self.scalar("u64", what + " length"), what)

    def weight(self, what):
        k = self.scalar("u64", what + " k")
        n = self.scalar("u64", what + " n")
        fmt = self.scalar("u8", what + " format")
        if fmt == 0:
            data = self.vector(np.uint16, what)
            if data.size != k * n:
                raise Qor4bError(f"{what}: {data.size} f16 values for a {k} x {n} weight")
            return Weight("f16", k, n, data.reshape(k, n))
        if fmt == 1:
            packed = self.vector(np.uint8, what)
            scales = self.vector(np.uint16, what + " scales")
            if n % 32 or packed.size != k * n // 2 or scales.size != k * n // 32:
                raise Qor4bError(f"{what}: {packed.size} bytes / {scales.size} scales for a Q4 {k} x {n} weight")
            return Weight("q4", k, n, packed.reshape(k, n // 2), scales.reshape(k, n // 32))
        raise Qor4bError(f"Unknown weight format {fmt} ({what})")  # src/save.rs:127

    def record(self, kind, what):
        if kind == "w":
            return self.weight(what)
        return self.vector(np.float32 if kind == "f32" else np.uint16, what)


def read_qor4b(path) -> Model:
    """Map a .qor4b file (src/save.rs:247-396) and return views of its records."""
    buf = np.memmap(path, dtype=np.uint8, mode="r")
    c = _Cursor(buf)
    magic = bytes(c.array(np.uint8, 4, "magic"))
    if magic != MAGIC:
        raise Qor4bError("Invalid magic (expected QOR4)")
    version = c.scalar("u32", "version")
    if version not in (1, VERSION):
        raise Qor4bError(f"Unsupported version {version} (expected 1 or {VERSION})")
    format_id = c.scalar("u8", "format")
    config = {name: c.scalar(kind, name) for name, kind in CONFIG_FIELDS}
    config["tie_word_embeddings"] = config["tie_word_embeddings"] != 0
    config["has_vision"] = config["has_vision"] != 0
    layer_types = [0 if c.scalar("u8", f"layer {i} type") == 0 else 1 for i in range(config["num_layers"])]
    layers = []
    for i, lt in enumerate(layer_types):
        fields = DELTANET_FIELDS if lt == 0 else ATTENTION_FIELDS
        layers.append({name: c.record(kind, f"layer {i} {name}") for name, kind in fields})
    globs = {name: c.record(kind, name) for name, kind in GLOBAL_FIELDS}
    vision_offset = c.pos if config["has_vision"] else -1
    return Model(version, format_id, config, layer_types, layers, globs, vision_offset)


def _put_scalar(out, kind, value):
    out.append(struct.pack(_SCALAR[kind][0], value))


def _put_vector(out, arr):
    arr = np.ascontiguousarray(arr)
    _put_scalar(out, "u64", arr.size)
    out.append(arr.tobytes())


def _put_weight(out, w: Weight):
    _put_scalar(out, "u64", w.k)
    _put_scalar(out, "u64", w.n)
    _put_scalar(out, "u8", 0 if w.kind == "f16" else 1)
    _put_vector(out, np.asarray(w.data, np.uint16 if w.kind == "f16" else np.uint8))
    if w.kind == "q4":
        _put_vector(out, np.asarray(w.scales, np.uint16))


def write_qor4b(path, model: Model):
    """Write `model` in the reference's layout (version 2, no vision encoder)."""
    if model.config.get("has_vision"):
        raise Qor4bError("writing a vision encoder is not supported")
    out = [MAGIC]
    _put_scalar(out, "u32", VERSION)
    _put_scalar(out, "u8", model.format_id)
    for name, kind in CONFIG_FIELDS:
        _put_scalar(out, kind, int(model.config[name]) if kind in ("u8", "u32") else model.config[name])
    for lt in model.layer_types:
        _put_scalar(out, "u8", lt)
    for lt, layer in zip(model.layer_types, model.layers):
        for name, kind in (DELTANET_FIELDS if lt == 0 else ATTENTION_FIELDS):
            (_put_weight if kind == "w" else _put_vector)(out, layer[name])
    for name, kind in GLOBAL_FIELDS:
        (_put_weight if kind == "w" else _put_vector)(out, model.globals[name])
    with open(path, "wb") as f:
        for chunk in out:
            f.write(chunk)


def _f16_to_f32(bits):
    return np.asarray(bits, np.uint16).view(np.float16).astype(np.float32)


def upload_mixers(model: Model):
    """Copy the mixer path of `model` to the current CUDA device.

    Returns a list with one dict per layer: DeltaNet {"type": 0, "in_proj": [qkv, a, b, z] (for
    Mixer.gemv_multi), "out_proj", "params" (qm_dn_params)}, attention {"type": 1, "in_proj": [q, k, v],
    "o_proj", "params" (qm_gqa_params)}, and a last dict {"lm_head": row-layout weight of the
    embedding, "final_norm": f32 tensor}.  Every descriptor keeps its device buffers alive."""
    import torch

    import qora_mixer as qm

    def dev(a):
        a = np.ascontiguousarray(a)
        if a.dtype == np.uint16:
            a = a.view(np.int16)
        return torch.from_numpy(a.copy()).cuda()

    def weight(w: Weight):
        if w.kind == "q4":
            return qm.weight_q4(dev(w.data), dev(w.scales))
        return qm.weight_f16(dev(w.data))

    out = []
    for lt, layer in zip(model.layer_types, model.layers):
        if lt == 0:
            keep = [dev(layer["conv1d_weight"]), dev(layer["a_log"]), dev(layer["dt_bias"]),
                    dev(_f16_to_f32(layer["attn_norm_weight"]))]
            params = qm.dn_params(*keep)
            params._keep = keep
            out.append({"type": 0, "params": params,
                        "in_proj": [weight(layer[n]) for n in ("in_proj_qkv", "in_proj_a", "in_proj_b", "in_proj_z")],
                        "out_proj": weight(layer["out_proj"])})
        else:
            half = int(model.config["attn_head_dim"] * model.config["partial_rotary_factor"]) // 2
            cos = np.asarray(model.globals["rope_cos"], np.float32).reshape(-1, half)
            sin = np.asarray(model.globals["rope_sin"], np.float32).reshape(-1, half)
            keep = [dev(_f16_to_f32(layer["q_norm"])), dev(_f16_to_f32(layer["k_norm"])), dev(cos), dev(sin)]
            params = qm.gqa_params(*keep)
            params._keep = keep
            out.append({"type": 1, "params": params,
                        "in_proj": [weight(layer[n]) for n in ("q_proj", "k_proj", "v_proj")],
                        "o_proj": weight(layer["o_proj"])})
    e = model.globals["embed"]  # [vocab rows][hidden]: the lm_head reads it row by row
    lm = qm.weight_q4_rows(dev(e.data), dev(e.scales)) if e.kind == "q4" else qm.weight_f16_rows(dev(e.data))
    out.append({"lm_head": lm, "final_norm": dev(_f16_to_f32(model.globals["final_norm"]))})
    return out
