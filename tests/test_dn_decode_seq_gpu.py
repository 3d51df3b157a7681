"""qm_dn_decode_seq (T DeltaNet decode steps in one launch, state on chip) on
the GPU vs the CPU restatement of the reference's per-token update
(src/gemv.rs:744-883; the same loop as prefill_deltanet_layer,
src/gemv.rs:1129-1203).

Tolerance (north_star, fp32-state decode): max|gpu - cpu| / RMS(cpu) <= 1e-3
per token, and for the final state; the conv history holds raw inputs and
must match bit for bit.  The oracle runs the AVX-512 head update where the
host has it, as the reference does (src/simd.rs:18-27).
"""
import numpy as np
import pytest

import refmath
from gpu_util import dev, host, make_ctx
from qora_mixer import inputs as I

pytestmark = pytest.mark.gpu
TOL = 1e-3


@pytest.fixture(scope="module")
def ctx():
    c = make_ctx()
    yield c
    c.close()


def _setup(ctx, orc, B, seed, seed_state=False, heads=None):
    import qora_mixer as qm

    g = I.rng(seed)
    p = I.dn_layer_params(g)
    c = orc.cfg_4b()
    ost = [orc.DnState(c) for _ in range(B)]
    st = qm.DnState(ctx, B, heads=heads)
    if seed_state:
        for bi in range(B):
            ost[bi].s[:] = (g.standard_normal(ost[bi].s.shape) * 0.02).astype(np.float32)
            ost[bi].conv_buf[:] = (g.standard_normal(ost[bi].conv_buf.shape) * 0.02).astype(np.float32)
            if heads is None:
                st.write(bi, ost[bi].s, ost[bi].conv_buf)
            else:
                lo, n = heads
                st.write(bi, ost[bi].s[lo:lo + n], ost[bi].conv_buf)
    keep = [dev(p["conv_w"]), dev(p["a_log"]), dev(p["dt_bias"]), dev(p["norm_gamma"])]
    return g, p, c, ost, st, qm.dn_params(*keep), keep


def _oracle_tokens(orc, c, ost, p, toks, bi, t0, t1, fused):
    avx = orc.has_avx512()
    ys, gs = [], []
    for t in range(t0, t1):
        r = orc.dn_decode(c, ost[bi], toks["qkv"][bi, t], toks["a"][bi, t], toks["b"][bi, t],
                          p["conv_w"], p["a_log"], p["dt_bias"], use_avx512=avx,
                          z=toks["z"][bi, t] if fused else None,
                          norm_gamma=p["norm_gamma"] if fused else None)
        yo, go = (r if fused else (r, None))
        ys.append(yo)
        gs.append(go)
    return np.stack(ys), (np.stack(gs) if fused else None)


def _worst_per_token(got, ref):
    return max(refmath.rel_err(got[t], ref[t]) for t in range(ref.shape[0]))


def test_config0_256_tokens_one_launch(ctx, orc):
    """Config 0: one DeltaNet layer, batch 1, 256 sequential tokens from a zero
    state, in one launch; every token's y and the final state."""
    import torch

    import qora_mixer as qm

    B, T = 1, 256
    g, p, c, ost, st, prm, keep = _setup(ctx, orc, B, 0x51A0 + 0)
    toks = I.dn_token_inputs(g, T, B)
    y = torch.full((B, T, 32, 128), float("nan"), device="cuda")
    n0 = ctx.launch_count()
    qm.Mixer(ctx).dn_decode_seq(prm, st, T, dev(toks["qkv"]), dev(toks["a"]), dev(toks["b"]), y)
    ctx.sync()
    assert ctx.launch_count() - n0 == 1
    ref, _ = _oracle_tokens(orc, c, ost, p, toks, 0, 0, T, False)
    e = _worst_per_token(host(y)[0], ref)
    s_g, cb_g = st.read(0)
    es = refmath.rel_err(s_g, ost[0].s)
    assert e <= TOL and es <= TOL, (e, es)
    np.testing.assert_array_equal(cb_g, ost[0].conv_buf)
    assert st.conv_pos == T
    print(f"config 0 in one launch: worst per-token rel err {e:.2e}, final state {es:.2e}")


def test_matches_per_token_decode_calls(ctx, orc):
    """The same tokens through qm_dn_decode one at a time: same operation
    sequence per row, so the two agree far inside the tolerance."""
    import torch

    import qora_mixer as qm

    B, T = 4, 40
    g, p, c, ost, st, prm, keep = _setup(ctx, orc, B, 910, seed_state=True)
    st2 = qm.DnState(ctx, B)
    for bi in range(B):
        st2.write(bi, ost[bi].s, ost[bi].conv_buf)
    toks = I.dn_token_inputs(g, T, B)
    mx = qm.Mixer(ctx)
    y = torch.empty(B, T, 32, 128, device="cuda")
    mx.dn_decode_seq(prm, st, T, dev(toks["qkv"]), dev(toks["a"]), dev(toks["b"]), y)
    yd = torch.empty(B, 32, 128, device="cuda")
    worst = 0.0
    for t in range(T):
        mx.dn_decode(prm, st2, dev(toks["qkv"][:, t]), dev(toks["a"][:, t]), dev(toks["b"][:, t]), yd)
        ctx.sync()
        worst = max(worst, refmath.rel_err(host(y[:, t]), host(yd)))
    assert worst <= 1e-5, worst
    for bi in range(B):
        s1, c1 = st.read(bi)
        s2, c2 = st2.read(bi)
        assert refmath.rel_err(s1, s2) <= 1e-5
        np.testing.assert_array_equal(c1, c2)


@pytest.mark.parametrize("T", [1, 2, 3, 5, 67])
def test_short_runs_between_decode_steps(ctx, orc, T):
    """decode, decode, seq(T), decode: the conv history ring carries across
    the three entry points (runs shorter than the 3-token history included),
    gated output on, batch 3 from a seeded state."""
    import torch

    import qora_mixer as qm

    B = 3
    g, p, c, ost, st, prm, keep = _setup(ctx, orc, B, 920 + T, seed_state=True)
    n = T + 3
    toks = I.dn_token_inputs(g, n, B)
    mx = qm.Mixer(ctx)
    yd = torch.empty(B, 32, 128, device="cuda")
    od = torch.empty(B, 4096, device="cuda")
    worst = 0.0

    def dec(t):
        nonlocal worst
        mx.dn_decode(prm, st, dev(toks["qkv"][:, t]), dev(toks["a"][:, t]), dev(toks["b"][:, t]),
                     yd, dev(toks["z"][:, t]), od)
        ctx.sync()
        for bi in range(B):
            ref_y, ref_g = _oracle_tokens(orc, c, ost, p, toks, bi, t, t + 1, True)
            worst = max(worst, refmath.rel_err(host(yd)[bi], ref_y[0]),
                        refmath.rel_err(host(od)[bi], ref_g[0]))

    dec(0)
    dec(1)
    y = torch.empty(B, T, 32, 128, device="cuda")
    out = torch.empty(B, T, 32, 128, device="cuda")
    sl = slice(2, 2 + T)
    mx.dn_decode_seq(prm, st, T, dev(np.ascontiguousarray(toks["qkv"][:, sl])),
                     dev(np.ascontiguousarray(toks["a"][:, sl])), dev(np.ascontiguousarray(toks["b"][:, sl])),
                     y, dev(np.ascontiguousarray(toks["z"][:, sl])), out)
    ctx.sync()
    for bi in range(B):
        ref_y, ref_g = _oracle_tokens(orc, c, ost, p, toks, bi, 2, 2 + T, True)
        worst = max(worst, _worst_per_token(host(y)[bi], ref_y),
                    _worst_per_token(host(out)[bi].reshape(T, -1), ref_g))
    dec(2 + T)
    assert worst <= TOL, worst
    assert st.conv_pos == n
    for bi in range(B):
        s_g, cb_g = st.read(bi)
        assert refmath.rel_err(s_g, ost[bi].s) <= TOL
        np.testing.assert_array_equal(cb_g, ost[bi].conv_buf)


def test_head_sharded_state(ctx, orc):
    """A state holding V heads [8, 16): outputs [B,T,8,128] equal the full
    state's heads 8..15 bit for bit (the same kernel arithmetic per head)."""
    import torch

    import qora_mixer as qm

    B, T = 2, 9
    g, p, c, ost, st_full, prm, keep = _setup(ctx, orc, B, 930, seed_state=True)
    st_h = qm.DnState(ctx, B, heads=(8, 8))
    for bi in range(B):
        st_h.write(bi, ost[bi].s[8:16], ost[bi].conv_buf)
    toks = I.dn_token_inputs(g, T, B)
    mx = qm.Mixer(ctx)
    args = (dev(toks["qkv"]), dev(toks["a"]), dev(toks["b"]))
    y_full = torch.empty(B, T, 32, 128, device="cuda")
    y_h = torch.empty(B, T, 8, 128, device="cuda")
    mx.dn_decode_seq(prm, st_full, T, *args, y_full)
    mx.dn_decode_seq(prm, st_h, T, *args, y_h)
    ctx.sync()
    np.testing.assert_array_equal(host(y_h), host(y_full[:, :, 8:16]))
    for bi in range(B):
        sf, cf = st_full.read(bi)
        sh, ch = st_h.read(bi)
        np.testing.assert_array_equal(sh, sf[8:16])


def test_argument_errors(ctx, orc):
    import torch

    import qora_mixer as qm

    g, p, c, ost, st, prm, keep = _setup(ctx, orc, 1, 940)
    qkv = torch.zeros(1, 4, 8192 + 1, device="cuda")
    ab = torch.zeros(1, 4, 32, device="cuda")
    y = torch.empty(1, 4, 32, 128, device="cuda")
    mx = qm.Mixer(ctx)
    with pytest.raises(qm.QmError) as e:
        mx.dn_decode_seq(prm, st, 0, qkv, ab, ab, y)
    assert e.value.code == 1  # QM_E_ARG: T <= 0
    with pytest.raises(qm.QmError) as e:
        mx.dn_decode_seq(prm, st, 4, qkv.view(-1)[1:], ab, ab, y)
    assert e.value.code == 1  # QM_E_ARG: qkv not 16-byte aligned
    assert st.conv_pos == 0
