"""DeltaNet chunked prefill on the GPU vs the sequential CPU restatement of
src/gemv.rs:1119-1219 (prefill_deltanet_layer).

Tolerance (north_star, tensor-core prefill): max|gpu - cpu| / RMS(cpu) <= 2e-2,
for every output token and for the final state; the conv history holds raw
inputs and must match bit for bit.
"""
import numpy as np
import pytest

import refmath
from gpu_util import dev, host, make_ctx
from qora_mixer import inputs as I

pytestmark = pytest.mark.gpu
TOL = 2e-2


@pytest.fixture(scope="module")
def ctx():
    c = make_ctx()
    yield c
    c.close()


def _case(ctx, orc, B, T, seed, decode_first=0, gate=False):
    import torch

    import qora_mixer as qm

    c = orc.cfg_4b()
    g = I.rng(seed)
    p = I.dn_layer_params(g)
    keep = [dev(p["conv_w"]), dev(p["a_log"]), dev(p["dt_bias"]), dev(p["norm_gamma"])]
    prm = qm.dn_params(*keep)
    mx = qm.Mixer(ctx)
    st = qm.DnState(ctx, B)
    ost = [orc.DnState(c) for _ in range(B)]
    # optional decode steps first: the prefill then continues a live state and conv history
    if decode_first:
        toks = I.dn_token_inputs(g, decode_first, B)
        y = torch.empty(B, 32, 128, device="cuda")
        for t in range(decode_first):
            mx.dn_decode(prm, st, dev(toks["qkv"][:, t]), dev(toks["a"][:, t]), dev(toks["b"][:, t]), y)
            for bi in range(B):
                orc.dn_decode(c, ost[bi], toks["qkv"][bi, t], toks["a"][bi, t], toks["b"][bi, t],
                              p["conv_w"], p["a_log"], p["dt_bias"], use_avx512=False)
    qkv = I.f32_to_bf16_bits(g.standard_normal((B, T, 8192), dtype=np.float32))
    a = g.standard_normal((B, T, 32), dtype=np.float32)
    b = g.standard_normal((B, T, 32), dtype=np.float32)
    z = g.standard_normal((B, T, 4096), dtype=np.float32) if gate else None
    y = torch.full((B, T, 32, 128), float("nan"), device="cuda")
    out = torch.full((B, T, 4096), float("nan"), device="cuda") if gate else None
    mx.dn_prefill(prm, st, T, dev(qkv), dev(a), dev(b), y, dev(z) if gate else None, out)
    ctx.sync()
    yg = host(y)
    og = host(out) if gate else None
    worst_y = worst_s = worst_o = 0.0
    for bi in range(B):
        yo = orc.dn_prefill(c, ost[bi], qkv[bi], a[bi], b[bi], p["conv_w"], p["a_log"], p["dt_bias"])
        worst_y = max(worst_y, refmath.rel_err(yg[bi], yo))
        if gate:
            # the reference applies the norm+gate in place on y (gemv.rs:1205-1219);
            # gated cases start from a fresh state
            assert not decode_first
            yo2 = orc.dn_prefill(c, orc.DnState(c), qkv[bi], a[bi], b[bi], p["conv_w"], p["a_log"],
                                 p["dt_bias"], z=z[bi], norm_gamma=p["norm_gamma"])
            worst_o = max(worst_o, refmath.rel_err(og[bi], yo2))
        s_g, cb_g = st.read(bi)
        worst_s = max(worst_s, refmath.rel_err(s_g, ost[bi].s))
        np.testing.assert_array_equal(cb_g, ost[bi].conv_buf)
    print(f"dn_prefill B={B} T={T}: y {worst_y:.2e} S {worst_s:.2e} gated {worst_o:.2e}")
    assert worst_y <= TOL and worst_s <= TOL and worst_o <= TOL, (worst_y, worst_s, worst_o)
    assert st.conv_pos == decode_first + T
    return st


@pytest.mark.parametrize("B,T", [(1, 64), (1, 100), (2, 200), (1, 3), (1, 1), (1, 65), (3, 128)])
def test_prefill_small_every_token(ctx, orc, B, T):
    """Full chunk, partial chunks, several chunks, a prompt shorter than the conv."""
    _case(ctx, orc, B, T, 900 + T + B)


def test_prefill_continues_decoded_state(ctx, orc):
    """5 decode steps, then a prefill: live state and conv history carried over."""
    _case(ctx, orc, 2, 130, 950, decode_first=5)


def test_prefill_fused_gate(ctx, orc):
    _case(ctx, orc, 1, 96, 960, gate=True)


def test_prefill_then_decode(ctx, orc):
    """Decode after a prefill continues from the chunked state."""
    import torch

    import qora_mixer as qm

    c = orc.cfg_4b()
    g = I.rng(970)
    p = I.dn_layer_params(g)
    keep = [dev(p["conv_w"]), dev(p["a_log"]), dev(p["dt_bias"])]
    prm = qm.dn_params(*keep)
    mx = qm.Mixer(ctx)
    st = qm.DnState(ctx, 1)
    ost = orc.DnState(c)
    T = 77
    qkv = I.f32_to_bf16_bits(g.standard_normal((1, T, 8192), dtype=np.float32))
    a = g.standard_normal((1, T, 32), dtype=np.float32)
    b = g.standard_normal((1, T, 32), dtype=np.float32)
    y = torch.empty(1, T, 32, 128, device="cuda")
    mx.dn_prefill(prm, st, T, dev(qkv), dev(a), dev(b), y)
    orc.dn_prefill(c, ost, qkv[0], a[0], b[0], p["conv_w"], p["a_log"], p["dt_bias"])
    toks = I.dn_token_inputs(g, 3, 1)
    yd = torch.empty(1, 32, 128, device="cuda")
    for t in range(3):
        mx.dn_decode(prm, st, dev(toks["qkv"][:, t]), dev(toks["a"][:, t]), dev(toks["b"][:, t]), yd)
        ctx.sync()
        yo = orc.dn_decode(c, ost, toks["qkv"][0, t], toks["a"][0, t], toks["b"][0, t], p["conv_w"],
                           p["a_log"], p["dt_bias"], use_avx512=False)
        assert refmath.rel_err(host(yd)[0], yo) <= TOL


def _oracle_prefill_heads(orc, c, qh, a, b, p, heads, groups=16):
    """The sequential recurrence (src/gemv.rs:1119-1219) for the V heads listed,
    split over a thread pool (the C restatement releases the GIL); each task
    runs on its own zero state and keeps only its heads' outputs."""
    from concurrent.futures import ThreadPoolExecutor

    heads = list(heads)
    per = max(1, -(-len(heads) // groups))
    parts = [heads[i:i + per] for i in range(0, len(heads), per)]

    def run(hs):
        st = orc.DnState(c)
        y = orc.dn_prefill(c, st, qh, a, b, p["conv_w"], p["a_log"], p["dt_bias"],
                           vh_lo=hs[0], vh_hi=hs[-1] + 1)
        return hs, y, st.s

    T = qh.shape[0]
    y = np.zeros((T, 32, 128), np.float32)
    s = np.zeros((32, 128, 128), np.float32)
    with ThreadPoolExecutor(max_workers=min(len(parts), 16)) as ex:
        for hs, yp, sp in ex.map(run, parts):
            y[:, hs] = yp[:, hs]
            s[hs] = sp[hs]
    return y, s


def test_config2_prefill(ctx, orc):
    """Config 2: batch 8 x 8192 tokens, chunk 64.  q/k/v raw inputs drawn on the
    device (bf16).  Checked in full against the sequential recurrence: every
    token of all 32 V heads and all 32 final states of all 8 sequences."""
    import torch

    import qora_mixer as qm

    c = orc.cfg_4b()
    B, T = 8, 8192
    g = I.rng(0x51A0 + 2)
    p = I.dn_layer_params(g)
    keep = [dev(p["conv_w"]), dev(p["a_log"]), dev(p["dt_bias"])]
    prm = qm.dn_params(*keep)
    qkv = I.device_normal_bf16((B, T, 8192), 0x51A2 * 10 + 1)
    a = g.standard_normal((B, T, 32), dtype=np.float32)
    b = g.standard_normal((B, T, 32), dtype=np.float32)
    st = qm.DnState(ctx, B)
    y = torch.empty(B, T, 32, 128, device="cuda")
    qm.Mixer(ctx).dn_prefill(prm, st, T, qkv.view(torch.int16), dev(a), dev(b), y)
    ctx.sync()
    worst = 0.0
    for bi in range(B):
        heads = range(32)
        qh = host(qkv[bi].view(torch.int16))
        yo, so = _oracle_prefill_heads(orc, c, qh, a[bi], b[bi], p, heads)
        s_g, _ = st.read(bi)
        yg = host(y[bi])
        for vh in heads:
            e = refmath.rel_err(yg[:, vh], yo[:, vh])
            es = refmath.rel_err(s_g[vh], so[vh])
            worst = max(worst, e, es)
            assert e <= TOL and es <= TOL, (bi, vh, e, es)
    print(f"config 2 prefill: worst rel err over y and S, all sequences and heads: {worst:.2e}")
