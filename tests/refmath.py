"""Independent float64 numpy restatement of the mixer math (test helper).

Written from the equations, not from the C restatement, so that the two
can check each other: a slip in either shows up as a disagreement far above
f32 rounding.  Equation sources in the reference (qora-protocol/QORA-LLM-4B):
DeltaNet decode src/gemv.rs:744-883, GQA decode src/gemv.rs:927-1011,
GQA prefill src/gemv.rs:1364-1444, RoPE table src/convert.rs:161-176.
"""
import numpy as np


def silu(x):
    return x / (1.0 + np.exp(-x))


def softplus(x):
    return np.where(x > 20.0, x, np.log1p(np.exp(np.minimum(x, 20.0))))


def dn_decode_f64(qkv, a, b, conv_w, a_log, dt_bias, S, conv_buf, num_qk, num_v, hd,
                  z=None, norm_gamma=None):
    """One DeltaNet token.  S [num_v, hd, hd] (row = v-dim), conv_buf [C, ks-1].
    Returns (y [num_v, hd], S_new, conv_buf_new, gated or None)."""
    qkv = qkv.astype(np.float64)
    W = conv_w.astype(np.float64)
    buf = conv_buf.astype(np.float64)
    window = np.concatenate([buf, qkv[:, None]], axis=1)  # [C, ks]
    conv = (window * W).sum(axis=1)
    new_buf = window[:, 1:].copy()
    x = silu(conv)
    qd = num_qk * hd
    q = x[:qd].reshape(num_qk, hd)
    k = x[qd:2 * qd].reshape(num_qk, hd)
    v = x[2 * qd:].reshape(num_v, hd)
    qn = np.linalg.norm(q, axis=1, keepdims=True)
    kn = np.linalg.norm(k, axis=1, keepdims=True)
    q = np.where(qn > 1e-12, q / qn, q) / np.sqrt(hd)
    k = np.where(kn > 1e-12, k / kn, k)
    alpha = np.exp(-np.exp(a_log.astype(np.float64)) * softplus(a.astype(np.float64) + dt_bias))
    beta = 1.0 / (1.0 + np.exp(-b.astype(np.float64)))
    S = S.astype(np.float64).copy()
    y = np.empty((num_v, hd))
    rep = num_v // num_qk
    for h in range(num_v):
        kh, qh = k[h // rep], q[h // rep]
        Sd = alpha[h] * S[h]
        pred = Sd @ kh
        Sd = Sd + beta[h] * np.outer(v[h] - pred, kh)
        S[h] = Sd
        y[h] = Sd @ qh
    gated = None
    if z is not None:
        inv = 1.0 / np.sqrt((y * y).mean(axis=1, keepdims=True) + 1e-6)
        gated = y * inv * norm_gamma[None, :] * silu(z.astype(np.float64).reshape(num_v, hd))
    return y, S, new_buf, gated


def rope_f64(x, cos_row, sin_row, rot):
    half = rot // 2
    x = x.copy()
    x1 = x[..., :half].copy()
    x2 = x[..., half:rot].copy()
    x[..., :half] = x1 * cos_row - x2 * sin_row
    x[..., half:rot] = x2 * cos_row + x1 * sin_row
    return x


def qk_norm_f64(x, gamma):
    inv = 1.0 / np.sqrt((x * x).mean(axis=-1, keepdims=True) + 1e-6)
    return x * inv * (1.0 + gamma)


def gqa_decode_f64(q_gate, k_new, v_new, q_norm, k_norm, cos, sin, k_cache, v_cache, L,
                   H=16, KVH=4, D=256, rot=64):
    """k_cache/v_cache: [L, KVH, D] existing positions.  Returns out [H, D]."""
    qg = q_gate.astype(np.float64).reshape(H, 2 * D)
    q, gate = qg[:, :D], qg[:, D:]
    q = rope_f64(qk_norm_f64(q, q_norm), cos[L], sin[L], rot)
    kn = rope_f64(qk_norm_f64(k_new.astype(np.float64).reshape(KVH, D), k_norm), cos[L], sin[L], rot)
    K = np.concatenate([k_cache.astype(np.float64), kn[None]], axis=0)
    V = np.concatenate([v_cache.astype(np.float64), v_new.astype(np.float64).reshape(1, KVH, D)], axis=0)
    out = np.empty((H, D))
    g = H // KVH
    for h in range(H):
        s = K[:, h // g, :] @ q[h] / np.sqrt(D)
        p = np.exp(s - s.max())
        p /= p.sum()
        out[h] = p @ V[:, h // g, :]
    return out * (1.0 / (1.0 + np.exp(-gate)))


def gqa_prefill_rows_f64(q_gate, k, v, q_norm, k_norm, cos, sin, rows, H=16, KVH=4, D=256, rot=64):
    S = q_gate.shape[0]
    qg = q_gate.astype(np.float64).reshape(S, H, 2 * D)
    K = qk_norm_f64(k.astype(np.float64).reshape(S, KVH, D), k_norm)
    K = np.stack([rope_f64(K[t], cos[t], sin[t], rot) for t in range(S)])
    V = v.astype(np.float64).reshape(S, KVH, D)
    out = np.empty((len(rows), H, D))
    g = H // KVH
    for i, t in enumerate(rows):
        q = rope_f64(qk_norm_f64(qg[t, :, :D], q_norm), cos[t], sin[t], rot)
        gate = qg[t, :, D:]
        for h in range(H):
            s = K[: t + 1, h // g, :] @ q[h] / np.sqrt(D)
            p = np.exp(s - s.max())
            p /= p.sum()
            out[i, h] = (p @ V[: t + 1, h // g, :]) / (1.0 + np.exp(-gate[h]))
    return out, K


def rel_err(got, ref):
    """max |got - ref| / RMS(ref) — the north-star parity measure."""
    got = np.asarray(got, np.float64).reshape(-1)
    ref = np.asarray(ref, np.float64).reshape(-1)
    rms = np.sqrt(np.mean(ref * ref))
    return float(np.max(np.abs(got - ref)) / max(rms, 1e-30))
