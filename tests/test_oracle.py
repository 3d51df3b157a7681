"""CPU checks of the restatement (oracle/) — no GPU.

PARITY UNPINNED: the reference ships no golden vectors and cannot be built
here, so the restatement is pinned by (1) analytic known-answer cases,
(2) an independent float64 restatement (tests/refmath.py), (3) internal
consistency the reference guarantees (its prefill and decode loops share
arithmetic), and (4) the committed golden fixtures (tests/golden/).
"""
import numpy as np
import pytest

import refmath
from qora_mixer import inputs as I


def small_cfg(orc):
    return orc.cfg(num_qk_heads=2, num_v_heads=4, dn_head_dim=32, num_attn_heads=4,
                   num_kv_heads=1, attn_head_dim=64, rope_dim=16)


# ---------------------------------------------------------------- RoPE table
def test_rope_table_position0_identity_and_formula(orc):
    cos, sin = orc.rope_table(1.0e7, 64, 40000)
    assert cos.shape == (40000, 32)
    assert np.all(cos[0] == 1.0) and np.all(sin[0] == 0.0)
    i = np.arange(32, dtype=np.float64)
    freq = 1.0 / (1.0e7 ** (2.0 * i / 64.0))
    for pos in (1, 17, 8191, 8192, 32768):
        ang = pos * freq
        # f32 angle rounding dominates at large positions: |d angle| <= pos * 2^-24 * freq
        tol = 2e-6 + pos * 1.2e-7 * freq.max()
        assert np.max(np.abs(cos[pos] - np.cos(ang))) < tol
        assert np.max(np.abs(sin[pos] - np.sin(ang))) < tol


def test_rope_table_prefix_stable(orc):
    """Extending max_pos past the reference's 8192 keeps the first 8192 rows."""
    c1, s1 = orc.rope_table(1.0e7, 64, 8192)
    c2, s2 = orc.rope_table(1.0e7, 64, 32769)
    assert np.array_equal(c1, c2[:8192]) and np.array_equal(s1, s2[:8192])


# ---------------------------------------------------------------- DeltaNet
def _dn_params(c, g):
    qkv_dim = (2 * c.num_qk_heads + c.num_v_heads) * c.dn_head_dim
    return I.dn_layer_params(g, num_v=c.num_v_heads, qkv_dim=qkv_dim, hd=c.dn_head_dim)


def test_dn_kat_alpha1_beta1_zero_state(orc):
    """S0=0, alpha=1, beta=1  =>  S = v k^T and y = v (k.q)."""
    c = orc.cfg_4b()
    g = I.rng(100)
    p = _dn_params(c, g)
    qkv = g.standard_normal(I.QKV_DIM).astype(np.float32)
    a = np.full(32, -200.0, np.float32)   # softplus(-200 + dt) == 0 -> alpha == 1
    b = np.full(32, 100.0, np.float32)    # sigmoid(100) == 1 in f32
    st = orc.DnState(c)
    y = orc.dn_decode(c, st, qkv, a, b, p["conv_w"], p["a_log"], p["dt_bias"], use_avx512=False)
    # conv with zero buffer: out = x * w[:,3]
    x = refmath.silu((qkv * p["conv_w"][:, 3]).astype(np.float64))
    q = x[:2048].reshape(16, 128)
    k = x[2048:4096].reshape(16, 128)
    v = x[4096:].reshape(32, 128)
    q = q / np.linalg.norm(q, axis=1, keepdims=True) / np.sqrt(128)
    k = k / np.linalg.norm(k, axis=1, keepdims=True)
    for h in range(32):
        np.testing.assert_allclose(st.s[h], np.outer(v[h], k[h // 2]), rtol=0, atol=2e-6)
        np.testing.assert_allclose(y[h], v[h] * (k[h // 2] @ q[h // 2]), rtol=0, atol=2e-6)
    assert st.conv_pos[0] == 1
    np.testing.assert_array_equal(st.conv_buf[:, 2], qkv)
    np.testing.assert_array_equal(st.conv_buf[:, :2], 0)


def test_dn_kat_alpha0_forgets_history(orc):
    """alpha == 0 zeroes the history: y = beta v (k.q) whatever S was."""
    c = orc.cfg_4b()
    g = I.rng(101)
    p = _dn_params(c, g)
    p["a_log"][:] = 10.0
    qkv = g.standard_normal(I.QKV_DIM).astype(np.float32)
    a = np.full(32, 10.0, np.float32)
    b = g.standard_normal(32).astype(np.float32)
    p["dt_bias"][:] = 0.0
    st1 = orc.DnState(c)
    st1.s[:] = g.standard_normal(st1.s.shape).astype(np.float32)
    st2 = orc.DnState(c)
    y1 = orc.dn_decode(c, st1, qkv, a, b, p["conv_w"], p["a_log"], p["dt_bias"])
    y2 = orc.dn_decode(c, st2, qkv, a, b, p["conv_w"], p["a_log"], p["dt_bias"])
    np.testing.assert_array_equal(y1, y2)
    np.testing.assert_array_equal(st1.s, st2.s)


def test_dn_conv_identity_weights(orc):
    """conv weights (0,0,0,1) make the conv the identity, so a repeated token
    gives the same y whatever the buffer holds (alpha == 0 to drop S)."""
    c = orc.cfg_4b()
    g = I.rng(102)
    p = _dn_params(c, g)
    p["conv_w"][:] = 0.0
    p["conv_w"][:, 3] = 1.0
    p["a_log"][:] = 10.0
    p["dt_bias"][:] = 0.0
    a = np.full(32, 10.0, np.float32)
    b = g.standard_normal(32).astype(np.float32)
    st = orc.DnState(c)
    x1 = g.standard_normal(I.QKV_DIM).astype(np.float32)
    x2 = g.standard_normal(I.QKV_DIM).astype(np.float32)
    y_first = orc.dn_decode(c, orc.DnState(c), x2, a, b, p["conv_w"], p["a_log"], p["dt_bias"])
    orc.dn_decode(c, st, x1, a, b, p["conv_w"], p["a_log"], p["dt_bias"])
    y_second = orc.dn_decode(c, st, x2, a, b, p["conv_w"], p["a_log"], p["dt_bias"])
    np.testing.assert_array_equal(y_first, y_second)


@pytest.mark.parametrize("avx", [False, True])
def test_dn_decode_matches_float64(orc, avx):
    if avx and not orc.has_avx512():
        pytest.skip("no AVX-512 on this host")
    c = orc.cfg_4b()
    g = I.rng(0)
    p = _dn_params(c, g)
    st = orc.DnState(c)
    S64 = np.zeros((32, 128, 128))
    buf64 = np.zeros((I.QKV_DIM, 3))
    for t in range(6):
        qkv = g.standard_normal(I.QKV_DIM).astype(np.float32)
        a = g.standard_normal(32).astype(np.float32)
        b = g.standard_normal(32).astype(np.float32)
        z = g.standard_normal(4096).astype(np.float32)
        y, gated = orc.dn_decode(c, st, qkv, a, b, p["conv_w"], p["a_log"], p["dt_bias"],
                                 use_avx512=avx, z=z, norm_gamma=p["norm_gamma"])
        y64, S64, buf64, g64 = refmath.dn_decode_f64(qkv, a, b, p["conv_w"], p["a_log"],
                                                     p["dt_bias"], S64, buf64, 16, 32, 128,
                                                     z=z, norm_gamma=p["norm_gamma"])
        assert refmath.rel_err(y, y64) < 2e-5
        assert refmath.rel_err(gated, g64) < 2e-5
        assert refmath.rel_err(st.s, S64) < 2e-5
        np.testing.assert_array_equal(st.conv_buf, buf64.astype(np.float32))


def test_dn_scalar_vs_avx512(orc):
    """simd.rs:292-362 vs gemv.rs:836-861: same algorithm, different sum order."""
    if not orc.has_avx512():
        pytest.skip("no AVX-512 on this host")
    c = orc.cfg_4b()
    g = I.rng(103)
    p = _dn_params(c, g)
    s1, s2 = orc.DnState(c), orc.DnState(c)
    for t in range(8):
        qkv = g.standard_normal(I.QKV_DIM).astype(np.float32)
        a = g.standard_normal(32).astype(np.float32)
        b = g.standard_normal(32).astype(np.float32)
        y1 = orc.dn_decode(c, s1, qkv, a, b, p["conv_w"], p["a_log"], p["dt_bias"], use_avx512=False)
        y2 = orc.dn_decode(c, s2, qkv, a, b, p["conv_w"], p["a_log"], p["dt_bias"], use_avx512=True)
        assert refmath.rel_err(y2, y1) < 1e-5
    assert refmath.rel_err(s2.s, s1.s) < 1e-5


def test_dn_prefill_equals_scalar_decode_loop(orc):
    """prefill_deltanet_layer (gemv.rs:1119-1219) runs the same per-token
    arithmetic as the scalar decode path, so the two agree bit for bit."""
    c = small_cfg(orc)
    g = I.rng(104)
    p = _dn_params(c, g)
    T = 9
    qkv_dim = (2 * c.num_qk_heads + c.num_v_heads) * c.dn_head_dim
    qkv = g.standard_normal((T, qkv_dim)).astype(np.float32)
    a = g.standard_normal((T, c.num_v_heads)).astype(np.float32)
    b = g.standard_normal((T, c.num_v_heads)).astype(np.float32)
    sp = orc.DnState(c)
    y_pre = orc.dn_prefill(c, sp, qkv, a, b, p["conv_w"], p["a_log"], p["dt_bias"])
    sd = orc.DnState(c)
    for t in range(T):
        y = orc.dn_decode(c, sd, qkv[t], a[t], b[t], p["conv_w"], p["a_log"], p["dt_bias"],
                          use_avx512=False)
        np.testing.assert_array_equal(y, y_pre[t])
    np.testing.assert_array_equal(sp.s, sd.s)
    np.testing.assert_array_equal(sp.conv_buf, sd.conv_buf)
    assert sp.conv_pos[0] == sd.conv_pos[0] == T


def test_dn_prefill_head_subset_and_bf16(orc):
    c = orc.cfg_4b()
    g = I.rng(105)
    p = _dn_params(c, g)
    T = 5
    qkv_b = I.f32_to_bf16_bits(g.standard_normal((T, I.QKV_DIM)))
    a = g.standard_normal((T, 32)).astype(np.float32)
    b = g.standard_normal((T, 32)).astype(np.float32)
    s_full = orc.DnState(c)
    y_full = orc.dn_prefill(c, s_full, I.bf16_bits_to_f32(qkv_b), a, b, p["conv_w"], p["a_log"],
                            p["dt_bias"])
    s_sub = orc.DnState(c)
    y_sub = orc.dn_prefill(c, s_sub, qkv_b, a, b, p["conv_w"], p["a_log"], p["dt_bias"],
                           vh_lo=6, vh_hi=9)
    np.testing.assert_array_equal(y_sub[:, 6:9], y_full[:, 6:9])
    np.testing.assert_array_equal(s_sub.s[6:9], s_full.s[6:9])
    np.testing.assert_array_equal(s_sub.conv_buf, s_full.conv_buf)


# ---------------------------------------------------------------- GQA
def _gqa_setup(orc, seed, L, max_pos=None):
    g = I.rng(seed)
    c = orc.cfg_4b()
    max_pos = max_pos or (L + 8)
    cos, sin = orc.rope_table(1.0e7, 64, max_pos)
    pr = I.gqa_layer_params(g, max_pos)
    kb, vb = I.gqa_cache_bf16(g, 1, L)
    k = I.bf16_bits_to_f32(kb[0]).transpose(1, 0, 2).copy()  # [L, KVH, D]
    v = I.bf16_bits_to_f32(vb[0]).transpose(1, 0, 2).copy()
    tok = I.gqa_token_inputs(g, 1)
    return g, c, cos, sin, pr, k, v, tok


def test_gqa_kat_single_position(orc):
    """Empty cache: softmax over one position is 1, so out = v_new * sigmoid(gate)."""
    g, c, cos, sin, pr, k, v, tok = _gqa_setup(orc, 106, 0)
    kv = orc.KvCache(c, 4)
    out = orc.gqa_decode(c, kv, tok["q_gate"][0], tok["k_new"][0], tok["v_new"][0],
                         pr["q_norm"], pr["k_norm"], cos, sin)
    gate = tok["q_gate"][0][:, 256:]
    for h in range(16):
        ref = tok["v_new"][0][h // 4] * (1.0 / (1.0 + np.exp(-gate[h].astype(np.float64))))
        np.testing.assert_allclose(out[h], ref, rtol=1e-6, atol=1e-7)
    assert kv.seq_len[0] == 1


@pytest.mark.parametrize("L", [5, 63, 64, 300])
def test_gqa_decode_matches_float64(orc, L):
    g, c, cos, sin, pr, k, v, tok = _gqa_setup(orc, 107 + L, L)
    kv = orc.KvCache(c, L + 1, k.reshape(L, -1), v.reshape(L, -1))
    out = orc.gqa_decode(c, kv, tok["q_gate"][0], tok["k_new"][0], tok["v_new"][0],
                         pr["q_norm"], pr["k_norm"], cos, sin)
    ref = refmath.gqa_decode_f64(tok["q_gate"][0], tok["k_new"][0], tok["v_new"][0], pr["q_norm"],
                                 pr["k_norm"], cos, sin, k, v, L)
    assert refmath.rel_err(out, ref) < 2e-5
    assert kv.seq_len[0] == L + 1


def test_gqa_decode_rejects_position_past_table(orc):
    g, c, cos, sin, pr, k, v, tok = _gqa_setup(orc, 108, 8, max_pos=8)
    kv = orc.KvCache(c, 9, k.reshape(8, -1), v.reshape(8, -1))
    with pytest.raises(ValueError):
        orc.gqa_decode(c, kv, tok["q_gate"][0], tok["k_new"][0], tok["v_new"][0],
                       pr["q_norm"], pr["k_norm"], cos, sin)


def test_gqa_prefill_rows_equal_decode_loop_and_float64(orc):
    """Row t of the causal prefill (gemv.rs:1406-1429) uses the same arithmetic
    as a decode step at position t (gemv.rs:958-1011): bit-identical."""
    g = I.rng(109)
    c = orc.cfg_4b()
    S = 70
    cos, sin = orc.rope_table(1.0e7, 64, S + 1)
    pr = I.gqa_layer_params(g, S + 1)
    qg = g.standard_normal((S, 16 * 512)).astype(np.float32)
    kk = g.standard_normal((S, 1024)).astype(np.float32)
    vv = g.standard_normal((S, 1024)).astype(np.float32)
    rows = np.array([0, 1, 2, 33, 63, 64, 69])
    out, kc, vc = orc.gqa_prefill_rows(c, qg, kk, vv, pr["q_norm"], pr["k_norm"], cos, sin, rows,
                                       want_cache=True)
    kv = orc.KvCache(c, S)
    dec = []
    for t in range(S):
        dec.append(orc.gqa_decode(c, kv, qg[t], kk[t], vv[t], pr["q_norm"], pr["k_norm"], cos, sin))
    for i, t in enumerate(rows):
        np.testing.assert_array_equal(out[i], dec[t])
    np.testing.assert_array_equal(kc, kv.k)
    np.testing.assert_array_equal(vc, kv.v)
    ref, _ = refmath.gqa_prefill_rows_f64(qg, kk, vv, pr["q_norm"], pr["k_norm"], cos, sin, rows)
    assert refmath.rel_err(out, ref) < 2e-5


def test_q4_restatement_quantizes_and_multiplies(orc):
    """The Q4 restatement (src/convert.rs:437-467, src/gemv.rs:411-450): every
    weight is within half a quantisation step of its f32 value (steps of
    absmax/7 per group of 32), all-zero groups get scale 0, and the GEMV equals
    x . dequantised W up to f32 rounding; the F16 GEMV likewise."""
    g = np.random.default_rng(5)
    w = (g.standard_normal((48, 96)) * 0.03).astype(np.float32)
    w[3, 32:64] = 0.0
    packed, scales = orc.quantize_q4(w)
    sc = scales.view(np.float16).astype(np.float32)
    assert sc[3, 1] == 0.0
    step = np.repeat(np.abs(w).reshape(48, 3, 32).max(axis=2) / 7.0, 32, axis=1)
    wd = orc.dequantize_q4(packed, scales)
    # f16 rounding of the stored scale adds at most 2^-11 relative per step
    assert (np.abs(wd - w) <= 0.5 * step * (1 + 8 * 2.0 ** -11) + 1e-12).all()
    x = g.standard_normal(48).astype(np.float32)
    ref = x.astype(np.float64) @ wd.astype(np.float64)
    y = orc.gemv_q4(x, packed, scales)
    assert np.abs(y - ref).max() <= 1e-5 * np.sqrt((ref ** 2).mean())
    w16 = w.astype(np.float16).view(np.uint16)
    ref16 = x.astype(np.float64) @ w.astype(np.float16).astype(np.float64)
    assert np.abs(orc.gemv_f16(x, w16) - ref16).max() <= 1e-5 * np.sqrt((ref16 ** 2).mean())


def _py_sample(l, temp, top_p, top_k, r):
    """An independent pure-Python restatement of src/generate.rs:334-384 (f32 steps)."""
    f = np.float32
    l = l.astype(np.float32)
    if temp <= 0:
        best, bv = 0, -np.inf
        for i, v in enumerate(l):
            if v > bv:
                best, bv = i, v
        return best
    inv, mx = f(1) / f(temp), f(l.max())
    order = sorted(range(len(l)), key=lambda i: (-l[i], i))
    k = min(top_k, len(l)) if top_k > 0 else len(l)
    import math
    p = [f(math.exp(float(f(f(l[i] - mx) * inv)))) for i in order[:k]]
    s = f(0)
    for v in p:
        s = f(s + v)
    p = [f(v * (f(1) / s)) for v in p]
    cum, cut = f(0), k
    for i, v in enumerate(p):
        cum = f(cum + v)
        if cum >= f(top_p):
            cut = i + 1
            break
    tot = f(0)
    for v in p[:cut]:
        tot = f(tot + v)
    rv, acc = f(f(r) * tot), f(0)
    for i in range(cut):
        acc = f(acc + p[i])
        if acc >= rv:
            return order[i]
    return order[0]


def test_sampling_and_penalty_restatement(orc):
    """or_sample_top_k against a pure-Python restatement (the same token unless
    the oracle's decision margin is below 1e-5: Python's exp is a double exp),
    the reference's xorshift draws, and the penalties against their rules."""
    g = np.random.default_rng(3)
    rng = orc.Rng(4242)
    checked = 0
    for t in range(200):
        l = (g.standard_normal(700) * 3).astype(np.float32)
        if t % 5 == 0:
            l = (np.round(l * 2) / 2).astype(np.float32)  # ties
        temp, top_p, top_k = [(0.7, 0.95, 20), (1.0, 0.8, 0), (0.0, 0.9, 5), (1.2, 1.0, 700)][t % 4]
        r = rng.next_f32()
        tok, margin = orc.sample_top_k(l, temp, top_p, top_k, r)
        if margin > 1e-5:
            assert tok == _py_sample(l, temp, top_p, top_k, r), t
            checked += 1
    assert checked >= 190
    s = orc.Rng(1)
    st = 1
    for _ in range(5):  # xorshift64 with shifts 13, 7, 17; the top 24 bits / 2^24
        st ^= (st << 13) & 0xFFFFFFFFFFFFFFFF
        st ^= st >> 7
        st ^= (st << 17) & 0xFFFFFFFFFFFFFFFF
        assert s.next_f32() == np.float32((st >> 40) / 16777216.0)
    lg = g.standard_normal(40).astype(np.float32)
    gen = [3, 3, 7, 10, 3] + [20] * 70  # 20 repeats past the 64-token window
    out = orc.penalize(lg, gen, repetition=1.3, presence=1.5, ban=5)
    exp = lg.copy()
    for t in gen[-64:]:
        exp[t] = exp[t] / np.float32(1.3) if exp[t] > 0 else exp[t] * np.float32(1.3)
    for t in set(gen):
        exp[t] -= np.float32(1.5)
    exp[5] = -np.inf
    np.testing.assert_array_equal(out, exp)
