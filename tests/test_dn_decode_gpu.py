"""DeltaNet decode on the GPU vs the CPU restatement of src/gemv.rs:744-883.

Tolerance (north_star, fp32-state decode): max|gpu - cpu| / RMS(cpu) <= 1e-3.
The conv history holds raw inputs, so it must match bit for bit.
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


def _run(ctx, orc, B, T, seed, fused, seed_state=False):
    import torch

    import qora_mixer as qm

    g = I.rng(seed)
    p = I.dn_layer_params(g)
    toks = I.dn_token_inputs(g, T, B)
    c = orc.cfg_4b()
    avx = orc.has_avx512()
    ost = [orc.DnState(c) for _ in range(B)]
    st = qm.DnState(ctx, B)
    if seed_state:
        for bi in range(B):
            ost[bi].s[:] = (g.standard_normal(ost[bi].s.shape) * 0.02).astype(np.float32)
            ost[bi].conv_buf[:] = (g.standard_normal(ost[bi].conv_buf.shape) * 0.02).astype(np.float32)
            st.write(bi, ost[bi].s, ost[bi].conv_buf)
    keep = [dev(p["conv_w"]), dev(p["a_log"]), dev(p["dt_bias"]), dev(p["norm_gamma"])]
    prm = qm.dn_params(*keep)
    mx = qm.Mixer(ctx)
    y = torch.empty(B, 32, 128, device="cuda")
    out = torch.empty(B, 4096, device="cuda") if fused else None
    worst_y = worst_o = 0.0
    for t in range(T):
        z = dev(toks["z"][:, t]) if fused else None
        mx.dn_decode(prm, st, dev(toks["qkv"][:, t]), dev(toks["a"][:, t]), dev(toks["b"][:, t]),
                     y, z, out)
        ctx.sync()
        yg = host(y)
        og = host(out) if fused else None
        for bi in range(B):
            r = orc.dn_decode(c, ost[bi], toks["qkv"][bi, t], toks["a"][bi, t], toks["b"][bi, t],
                              p["conv_w"], p["a_log"], p["dt_bias"], use_avx512=avx,
                              z=toks["z"][bi, t] if fused else None,
                              norm_gamma=p["norm_gamma"] if fused else None)
            yo, go = (r if fused else (r, None))
            worst_y = max(worst_y, refmath.rel_err(yg[bi], yo))
            if fused:
                worst_o = max(worst_o, refmath.rel_err(og[bi], go))
    assert worst_y <= TOL, f"y rel err {worst_y:.3e}"
    assert worst_o <= TOL, f"gated rel err {worst_o:.3e}"
    assert st.conv_pos == T
    for bi in range(B):
        s_g, cb_g = st.read(bi)
        assert refmath.rel_err(s_g, ost[bi].s) <= TOL
        np.testing.assert_array_equal(cb_g, ost[bi].conv_buf)
    return st


def test_config0_decode_256_tokens(ctx, orc):
    """Config 0: one DeltaNet layer, batch 1, 256 sequential tokens."""
    _run(ctx, orc, B=1, T=256, seed=0x51A0 + 0, fused=False)


@pytest.mark.parametrize("B,fused", [(1, True), (3, True), (3, False), (8, True), (8, False)])
def test_decode_batch_and_split_variants(ctx, orc, B, fused):
    """B=1 -> 4 CTAs per head (cluster epilogue), B=3 -> 2, B=8 -> 1."""
    _run(ctx, orc, B=B, T=5, seed=200 + B, fused=fused)


def test_decode_config4_batch_seeded_state(ctx, orc):
    """Config-4 batch (64 sequences) from N(0, 0.02) states, two tokens."""
    _run(ctx, orc, B=64, T=2, seed=0x51A0 + 4, fused=True, seed_state=True)


def test_state_snapshot_restore_roundtrip(ctx, orc):
    import torch

    import qora_mixer as qm

    g = I.rng(300)
    p = I.dn_layer_params(g)
    toks = I.dn_token_inputs(g, 4, 2)
    keep = [dev(p["conv_w"]), dev(p["a_log"]), dev(p["dt_bias"])]
    prm = qm.dn_params(*keep)
    mx = qm.Mixer(ctx)
    st = qm.DnState(ctx, 2)
    y = torch.empty(2, 32, 128, device="cuda")
    for t in range(2):
        mx.dn_decode(prm, st, dev(toks["qkv"][:, t]), dev(toks["a"][:, t]), dev(toks["b"][:, t]), y)
    snap = st.snapshot()
    ys = []
    for t in range(2, 4):
        mx.dn_decode(prm, st, dev(toks["qkv"][:, t]), dev(toks["a"][:, t]), dev(toks["b"][:, t]), y)
        ys.append(host(y).copy())
    st.restore_from(snap)
    assert st.conv_pos == 2
    for i, t in enumerate(range(2, 4)):
        mx.dn_decode(prm, st, dev(toks["qkv"][:, t]), dev(toks["a"][:, t]), dev(toks["b"][:, t]), y)
        np.testing.assert_array_equal(host(y), ys[i])
    st.reset()
    s0, cb0 = st.read(1)
    assert not s0.any() and not cb0.any() and st.conv_pos == 0
    snap.close()


def test_host_variant_matches_device_variant(ctx):
    import torch

    import qora_mixer as qm

    g = I.rng(301)
    p = I.dn_layer_params(g)
    toks = I.dn_token_inputs(g, 1, 4)
    keep = [dev(p["conv_w"]), dev(p["a_log"]), dev(p["dt_bias"]), dev(p["norm_gamma"])]
    prm = qm.dn_params(*keep)
    mx = qm.Mixer(ctx)
    s1, s2 = qm.DnState(ctx, 4), qm.DnState(ctx, 4)
    y = torch.empty(4, 32, 128, device="cuda")
    out = torch.empty(4, 4096, device="cuda")
    mx.dn_decode(prm, s1, dev(toks["qkv"][:, 0]), dev(toks["a"][:, 0]), dev(toks["b"][:, 0]), y,
                 dev(toks["z"][:, 0]), out)
    yh = np.empty((4, 32, 128), np.float32)
    oh = np.empty((4, 4096), np.float32)
    mx.dn_decode_host(prm, s2, np.ascontiguousarray(toks["qkv"][:, 0]),
                      np.ascontiguousarray(toks["a"][:, 0]), np.ascontiguousarray(toks["b"][:, 0]),
                      yh, np.ascontiguousarray(toks["z"][:, 0]), oh)
    ctx.sync()
    # when the host variant runs the batch in overlapped parts, a head may
    # span more CTAs, so the gated output's sum of squares can be added in
    # another order
    np.testing.assert_array_equal(yh, host(y))
    assert refmath.rel_err(oh, host(out)) <= 1e-5


def test_decode_argument_errors(ctx):
    import torch

    import qora_mixer as qm

    g = I.rng(302)
    p = I.dn_layer_params(g)
    keep = [dev(p["conv_w"]), dev(p["a_log"]), dev(p["dt_bias"])]
    prm = qm.dn_params(*keep)
    mx = qm.Mixer(ctx)
    st = qm.DnState(ctx, 1)
    qkv = torch.zeros(1, 8192, device="cuda")
    ab = torch.zeros(1, 32, device="cuda")
    out = torch.empty(1, 4096, device="cuda")
    with pytest.raises(qm.QmError) as e:
        mx.dn_decode(prm, st, qkv, ab, ab, None, None, out)  # out without z
    assert e.value.code == 1
    other = qm.Ctx(0)
    with pytest.raises(qm.QmError) as e:
        qm.Mixer(other).dn_decode(prm, st, qkv, ab, ab, torch.empty(1, 32, 128, device="cuda"))
    assert e.value.code == 8  # QM_E_MISMATCH
    assert st.conv_pos == 0
    other.close()


def test_host_variant_pipelined_matches_device(ctx, orc):
    """qm_dn_decode_host cuts a batch of 16 into parts whose copies overlap
    the kernels; its y equals the device-buffer call's bit for bit (same
    per-row arithmetic) and the gated output agrees to a few f32 roundings (1e-5)."""
    import torch

    import qora_mixer as qm

    B = 16
    g = I.rng(830)
    p = I.dn_layer_params(g)
    toks = I.dn_token_inputs(g, 2, B)
    keep = [dev(p["conv_w"]), dev(p["a_log"]), dev(p["dt_bias"]), dev(p["norm_gamma"])]
    prm = qm.dn_params(*keep)
    mx = qm.Mixer(ctx)
    st_d, st_h = qm.DnState(ctx, B), qm.DnState(ctx, B)
    for t in range(2):
        qkv, a, b, z = (np.ascontiguousarray(toks[k][:, t]) for k in ("qkv", "a", "b", "z"))
        y = torch.empty(B, 32, 128, device="cuda")
        out = torch.empty(B, 4096, device="cuda")
        mx.dn_decode(prm, st_d, dev(qkv), dev(a), dev(b), y, dev(z), out)
        ctx.sync()
        yh = np.empty((B, 32, 128), np.float32)
        oh = np.empty((B, 4096), np.float32)
        mx.dn_decode_host(prm, st_h, qkv, a, b, yh, z, oh)
        np.testing.assert_array_equal(yh, host(y))
        assert refmath.rel_err(oh, host(out)) <= 1e-5
    assert st_h.conv_pos == 2
    for bi in (0, 7, 15):
        np.testing.assert_array_equal(st_h.read(bi)[0], st_d.read(bi)[0])


def _pinned(a):
    import torch

    return torch.from_numpy(np.ascontiguousarray(a)).pin_memory()


def test_host_variant_in_place_on_pinned_buffers(ctx, orc):
    """Page-locked host buffers: qm_dn_decode_host runs one kernel launch on
    them in place (inputs read and outputs written over PCIe) and matches the
    device-buffer call bit for bit and the oracle within 1e-3; with the
    in-place path switched off, or with one pageable buffer among pinned
    ones, the same call is staged through copies in two parts."""
    import torch

    import qora_mixer as qm

    B, T = 16, 3
    g = I.rng(850)
    p = I.dn_layer_params(g)
    toks = I.dn_token_inputs(g, T, B)
    keep = [dev(p["conv_w"]), dev(p["a_log"]), dev(p["dt_bias"]), dev(p["norm_gamma"])]
    prm = qm.dn_params(*keep)
    mx = qm.Mixer(ctx)
    st_d, st_h = qm.DnState(ctx, B), qm.DnState(ctx, B)
    c = orc.cfg_4b()
    ost = [orc.DnState(c) for _ in range(B)]
    try:
        for t in range(T):
            qkv, a, b, z = (np.ascontiguousarray(toks[k][:, t]) for k in ("qkv", "a", "b", "z"))
            y = torch.empty(B, 32, 128, device="cuda")
            out = torch.empty(B, 4096, device="cuda")
            mx.dn_decode(prm, st_d, dev(qkv), dev(a), dev(b), y, dev(z), out)
            ctx.sync()
            yh = torch.empty(B, 32, 128).pin_memory()
            oh = torch.empty(B, 4096).pin_memory()
            ins = [_pinned(x) for x in (qkv, a, b, z)]
            if t == 1:
                ctx.set_host_direct(False)
            if t == 2:
                ins[3] = z  # one pageable buffer: staged
            n0, c0 = ctx.launch_count(), ctx.host_calls()
            mx.dn_decode_host(prm, st_h, ins[0], ins[1], ins[2], yh, ins[3], oh)
            c1 = ctx.host_calls()
            assert ctx.launch_count() - n0 == (1 if t == 0 else 2)
            assert (c1[0] - c0[0], c1[1] - c0[1]) == ((1, 0) if t == 0 else (0, 1))
            ctx.set_host_direct(True)
            np.testing.assert_array_equal(yh.numpy(), host(y))
            if t == 0:
                np.testing.assert_array_equal(oh.numpy(), host(out))
            else:
                assert refmath.rel_err(oh.numpy(), host(out)) <= 1e-5
            for bi in range(B):
                yo, go = orc.dn_decode(c, ost[bi], qkv[bi], a[bi], b[bi], p["conv_w"], p["a_log"],
                                       p["dt_bias"], use_avx512=False, z=z[bi],
                                       norm_gamma=p["norm_gamma"])
                assert refmath.rel_err(yh.numpy()[bi], yo) <= TOL
                assert refmath.rel_err(oh.numpy()[bi], go) <= TOL
        assert st_h.conv_pos == T
        for bi in (0, 15):
            np.testing.assert_array_equal(st_h.read(bi)[0], st_d.read(bi)[0])
            np.testing.assert_array_equal(st_h.read(bi)[1], st_d.read(bi)[1])
    finally:
        ctx.set_host_direct(True)


def test_host_staged_in_parts(ctx, orc):
    """qm_ctx_set_host_parts: the staged qm_dn_decode_host cut into 1, 3 and 8
    parts (overlapped copies and launches on three streams) matches the
    device-buffer call within 1e-5 and the restatement within 1e-3, and
    advances the same conv history; part counts outside 0..8 are refused."""
    import torch

    import qora_mixer as qm

    B = 16
    g = I.rng(853)
    p = I.dn_layer_params(g)
    keep = [dev(p["conv_w"]), dev(p["a_log"]), dev(p["dt_bias"]), dev(p["norm_gamma"])]
    prm = qm.dn_params(*keep)
    mx = qm.Mixer(ctx)
    st_d, st_h = qm.DnState(ctx, B), qm.DnState(ctx, B)
    c = orc.cfg_4b()
    ost = [orc.DnState(c) for _ in range(B)]
    try:
        for parts in (1, 3, 8):
            toks = I.dn_token_inputs(g, 1, B)
            qkv, a, b, z = (np.ascontiguousarray(toks[k][:, 0]) for k in ("qkv", "a", "b", "z"))
            y = torch.empty(B, 32, 128, device="cuda")
            out = torch.empty(B, 4096, device="cuda")
            mx.dn_decode(prm, st_d, dev(qkv), dev(a), dev(b), y, dev(z), out)
            ctx.sync()
            yh = torch.empty(B, 32, 128).pin_memory()
            oh = torch.empty(B, 4096).pin_memory()
            ctx.set_host_direct(False)
            ctx.set_host_parts(parts, 0)
            n0, c0 = ctx.launch_count(), ctx.host_calls()
            mx.dn_decode_host(prm, st_h, _pinned(qkv), _pinned(a), _pinned(b), yh, _pinned(z), oh)
            assert ctx.launch_count() - n0 == parts  # one decode launch a part
            assert ctx.host_calls()[1] - c0[1] == 1  # staged
            assert refmath.rel_err(yh.numpy(), host(y)) <= 1e-5
            assert refmath.rel_err(oh.numpy(), host(out)) <= 1e-5
            for bi in range(B):
                yo, go = orc.dn_decode(c, ost[bi], qkv[bi], a[bi], b[bi], p["conv_w"], p["a_log"],
                                       p["dt_bias"], use_avx512=False, z=z[bi], norm_gamma=p["norm_gamma"])
                assert refmath.rel_err(yh.numpy()[bi], yo) <= TOL
                assert refmath.rel_err(oh.numpy()[bi], go) <= TOL
        for bi in (0, 7, 15):
            np.testing.assert_array_equal(st_h.read(bi)[1], st_d.read(bi)[1])  # conv history, raw inputs
        for bad in (9, -1):
            with pytest.raises(qm.QmError) as e:
                ctx.set_host_parts(bad, 0)
            assert e.value.code == 1  # QM_E_ARG
    finally:
        ctx.set_host_parts(0, 0)
        ctx.set_host_direct(True)
        st_d.close()
        st_h.close()
