"""Seeded synthetic inputs for the five mixer workloads.

Every config i draws from numpy's counter-based Philox generator seeded with
0x51A0 + i, so the same bytes reach the CUDA path and the CPU restatement.
bf16 tensors are kept as uint16 bit patterns (round-to-nearest-even from
f32); the checker widens exactly those values.  Value distributions follow
the five workload descriptions: conv weights N(0, 0.1), a/b N(0, 1),
A_log U(0, 2.7), dt_bias U(-1, 1), mixed qkv N(0, 1); GQA norm weights
N(1, 0.05) rounded to f16 and applied as (1 + gamma) like the reference's
per_head_rms_norm (src/gemv.rs:586-597); bf16 KV cache N(0, 1).

Large workloads (prefill, 32-layer decode) are generated on the device by
torch (its CUDA generator is Philox-4x32-10) and copied back where a check
needs them; see `device_normal_bf16`.
"""
from __future__ import annotations

import numpy as np

SEED_BASE = 0x51A0

# Qor4bConfig::default_4b mixer fields (src/config.rs:52-78)
NUM_QK = 16
NUM_V = 32
DN_HD = 128
CONV_K = 4
QKV_DIM = (2 * NUM_QK + NUM_V) * DN_HD  # 8192
V_DIM = NUM_V * DN_HD  # 4096
NUM_H = 16
NUM_KVH = 4
ATT_D = 256
ROPE_DIM = 64
ROPE_THETA = 1.0e7


def rng(config_index: int, stream: int = 0) -> np.random.Generator:
    return np.random.Generator(np.random.Philox(key=SEED_BASE + config_index, counter=stream))


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even f32 -> bf16, returned as uint16 bits."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    r = (u + 0x7FFF + ((u >> 16) & 1)) >> 16
    return r.astype(np.uint16)


def bf16_bits_to_f32(b: np.ndarray) -> np.ndarray:
    return (np.ascontiguousarray(b, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def round_f16(x: np.ndarray) -> np.ndarray:
    """Weights the reference stores as f16 (gemv.rs:71,86-87), widened back."""
    return np.asarray(x, np.float32).astype(np.float16).astype(np.float32)


def dn_layer_params(g: np.random.Generator, num_v=NUM_V, qkv_dim=QKV_DIM, hd=DN_HD):
    """conv1d weight [qkv_dim, 4] ~ N(0, 0.1), A_log ~ U(0, 2.7), dt_bias ~ U(-1, 1),
    per-head norm gamma ~ N(1, 0.05) rounded to f16 (plain gamma, gemv.rs:876)."""
    conv_w = (g.standard_normal((qkv_dim, CONV_K), dtype=np.float32) * np.float32(0.1))
    a_log = g.uniform(0.0, 2.7, num_v).astype(np.float32)
    dt_bias = g.uniform(-1.0, 1.0, num_v).astype(np.float32)
    norm_gamma = round_f16(1.0 + 0.05 * g.standard_normal(hd))
    return dict(conv_w=conv_w, a_log=a_log, dt_bias=dt_bias, norm_gamma=norm_gamma)


def dn_token_inputs(g: np.random.Generator, T: int, B: int = 1, num_v=NUM_V, qkv_dim=QKV_DIM):
    """Per-token mixed qkv [B, T, qkv_dim] ~ N(0,1), a, b [B, T, num_v] ~ N(0,1),
    z [B, T, num_v*128] ~ N(0,1) (only for the fused gate epilogue)."""
    qkv = g.standard_normal((B, T, qkv_dim), dtype=np.float32)
    a = g.standard_normal((B, T, num_v), dtype=np.float32)
    b = g.standard_normal((B, T, num_v), dtype=np.float32)
    z = g.standard_normal((B, T, num_v * DN_HD), dtype=np.float32)
    return dict(qkv=qkv, a=a, b=b, z=z)


def gqa_layer_params(g: np.random.Generator, max_pos: int):
    """q_norm/k_norm gamma ~ N(1, 0.05) rounded to f16 (used as 1+gamma), RoPE tables
    from the reference formula (src/convert.rs:161-176) extended to max_pos."""
    q_norm = round_f16(1.0 + 0.05 * g.standard_normal(ATT_D))
    k_norm = round_f16(1.0 + 0.05 * g.standard_normal(ATT_D))
    return dict(q_norm=q_norm, k_norm=k_norm)


def gqa_token_inputs(g: np.random.Generator, B: int = 1):
    """New-token q/gate [B, H, 2*D] (interleaved per head, gemv.rs:927), k, v [B, KVH, D]."""
    q_gate = g.standard_normal((B, NUM_H, 2 * ATT_D), dtype=np.float32)
    k_new = g.standard_normal((B, NUM_KVH, ATT_D), dtype=np.float32)
    v_new = g.standard_normal((B, NUM_KVH, ATT_D), dtype=np.float32)
    return dict(q_gate=q_gate, k_new=k_new, v_new=v_new)


def gqa_cache_bf16(g: np.random.Generator, B: int, L: int, std: float = 1.0):
    """bf16 KV cache contents in the device layout [B, KVH, L, D] (uint16 bits)."""
    k = g.standard_normal((B, NUM_KVH, L, ATT_D), dtype=np.float32)
    v = g.standard_normal((B, NUM_KVH, L, ATT_D), dtype=np.float32)
    if std != 1.0:
        k *= np.float32(std)
        v *= np.float32(std)
    return f32_to_bf16_bits(k), f32_to_bf16_bits(v)


def device_normal_bf16(shape, seed: int, std: float = 1.0, device="cuda"):
    """Large bf16 N(0, std) tensors drawn on the device by torch's Philox generator."""
    import torch

    gen = torch.Generator(device=device)
    gen.manual_seed(seed)
    t = torch.empty(shape, dtype=torch.bfloat16, device=device)
    t.normal_(0.0, std, generator=gen)
    return t


def device_normal_f32(shape, seed: int, std: float = 1.0, device="cuda"):
    import torch

    gen = torch.Generator(device=device)
    gen.manual_seed(seed)
    t = torch.empty(shape, dtype=torch.float32, device=device)
    t.normal_(0.0, std, generator=gen)
    return t
