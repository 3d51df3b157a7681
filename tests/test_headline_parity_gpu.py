"""Parity at the shapes the headline benchmark runs (workload 4) on the GPU vs
the CPU restatement of the reference mixers.

* GQA decode at batch 64 x 32768 cached positions: the split-KV plan the
  benchmark uses (src/gemv.rs:927-1011), four seeded sequences, two steps.
* One whole 32-layer stack step at batch 64 through the same calls bench.py
  times (its `Stack`): every layer's output of two sampled sequences against
  the restatement of src/gemv.rs:744-883 (DeltaNet, fused norm * SiLU(z)
  epilogue) and src/gemv.rs:927-1011 (GQA), two steps so the updated states
  and appended cache rows are carried.

Tolerance (decode, fp32 state): max|gpu - cpu| / RMS(cpu) <= 1e-3.  The
bf16 row the GPU appends is copied into the oracle's cache after each step
(the oracle keeps f32), as the other decode tests do.
"""
import numpy as np
import pytest

import refmath
from gpu_util import dev, host, make_ctx
from qora_mixer import inputs as I

pytestmark = pytest.mark.gpu
TOL = 1e-3
CTX = 32768


@pytest.fixture(scope="module")
def ctx():
    c = make_ctx()
    yield c
    c.close()


def _oracle_cache(orc, c, K, V, b, L, cap):
    """The oracle's f32 cache of sequence b from the device bf16 cache [B,4,cap,256]."""
    kf = I.bf16_bits_to_f32(host(K[b, :, :L])).transpose(1, 0, 2).reshape(L, -1)
    vf = I.bf16_bits_to_f32(host(V[b, :, :L])).transpose(1, 0, 2).reshape(L, -1)
    return orc.KvCache(c, cap, kf, vf)


def _adopt_appended_row(okv, K, V, b, pos):
    """Replace the oracle's f32 row at `pos` by the bf16 row the GPU stored."""
    okv.k[pos] = I.bf16_bits_to_f32(host(K[b, :, pos]))
    okv.v[pos] = I.bf16_bits_to_f32(host(V[b, :, pos]))


def test_gqa_decode_batch64_ctx32768(ctx, orc):
    """Workload 4's GQA layer: 64 sequences, 32768 cached bf16 positions each
    (N(0,1), the harder of the two spec distributions for a softmax), new
    token at position 32768 then 32769.  Sequences 0, 21, 42, 63 are checked."""
    import torch

    import qora_mixer as qm

    c = orc.cfg_4b()
    B, L, cap = 64, CTX, CTX + 4
    g = I.rng(0x51A0 + 4, stream=11)
    pr = I.gqa_layer_params(g, cap + 1)
    cos, sin = qm.rope_table(1.0e7, 64, cap + 1)
    K = I.device_normal_bf16((B, 4, cap, 256), 0x51A4 * 10 + 1).view(torch.int16)
    V = I.device_normal_bf16((B, 4, cap, 256), 0x51A4 * 10 + 2).view(torch.int16)
    keep = [dev(pr["q_norm"]), dev(pr["k_norm"]), dev(cos), dev(sin)]
    prm = qm.gqa_params(*keep)
    kvh = qm.KvCache(ctx, B, cap, K, V)
    kvh.seq_len = L
    check = [0, 21, 42, 63]
    okv = {b: _oracle_cache(orc, c, K, V, b, L, cap + 1) for b in check}
    mx = qm.Mixer(ctx)
    out = torch.empty(B, 16, 256, device="cuda")
    worst = 0.0
    for step in range(2):
        tok = I.gqa_token_inputs(g, B)
        mx.gqa_decode(prm, kvh, dev(tok["q_gate"]), dev(tok["k_new"]), dev(tok["v_new"]), out)
        ctx.sync()
        og = host(out)
        assert np.isfinite(og).all()
        for b in check:
            ref = orc.gqa_decode(c, okv[b], tok["q_gate"][b], tok["k_new"][b], tok["v_new"][b],
                                 pr["q_norm"], pr["k_norm"], cos, sin)
            e = refmath.rel_err(og[b], ref)
            worst = max(worst, e)
            assert e <= TOL, (step, b, e)
            _adopt_appended_row(okv[b], K, V, b, L + step)
        assert kvh.seq_len == L + step + 1
    kvh.close()
    print(f"GQA decode B=64 L=32768: worst rel err {worst:.2e}")


def test_stack_step_batch64_every_layer(ctx, orc):
    """Two steps of bench.py's 32-layer stack at batch 64, context 32768: each
    of the 32 layers' outputs for sequences 0 and 63 against the restatement
    (DeltaNet with the fused RMSNorm(gamma) * SiLU(z) epilogue, GQA with the
    sigmoid gate)."""
    import bench

    c = orc.cfg_4b()
    B = 64
    cap = CTX + 8
    stack = bench.Stack(ctx, B, cap, seed=0, ctx_len=CTX)
    check = [0, 63]
    # the oracle's copy of every layer of the two sequences, as the GPU holds them now
    ost = {}
    cos, sin = (host(t) for t in stack.rope)
    for li, L in enumerate(stack.layers):
        for b in check:
            if L["kind"] == "dn":
                s, cb = L["st"].read(b)
                o = orc.DnState(c)
                o.s[:] = s
                o.conv_buf[:] = cb
                o.conv_pos[0] = CTX
                ost[li, b] = o
            else:
                K, V = L["store"]
                ost[li, b] = _oracle_cache(orc, c, K, V, b, CTX, cap + 1)
    params = []
    for L in stack.layers:
        params.append([host(t) for t in L["keep"]])
    inputs = [[host(t) for t in L["in"]] for L in stack.layers]
    worst = {"dn": 0.0, "attn": 0.0}
    for step in range(2):
        stack.step()
        ctx.sync()
        for li, L in enumerate(stack.layers):
            og = host(L["out"])
            for b in check:
                if L["kind"] == "dn":
                    conv_w, a_log, dt_bias, gamma = params[li]
                    qkv, a, bb, z = inputs[li]
                    _, ref = orc.dn_decode(c, ost[li, b], qkv[b], a[b], bb[b], conv_w, a_log, dt_bias,
                                           z=z[b], norm_gamma=gamma)
                    got = og[b]
                else:
                    qn, kn = params[li][0], params[li][1]
                    qg, kw, vw = inputs[li]
                    ref = orc.gqa_decode(c, ost[li, b], qg[b], kw[b], vw[b], qn, kn, cos, sin)
                    got = og[b].reshape(16, 256)
                    K, V = L["store"]
                    _adopt_appended_row(ost[li, b], K, V, b, CTX + step)
                e = refmath.rel_err(got, ref)
                worst[L["kind"]] = max(worst[L["kind"]], e)
                assert e <= TOL, (step, li, L["kind"], b, e)
    # the DeltaNet states after two steps, for the checked sequences
    for li, L in enumerate(stack.layers):
        if L["kind"] != "dn":
            continue
        for b in check:
            s, cb = L["st"].read(b)
            assert refmath.rel_err(s, ost[li, b].s) <= TOL
            np.testing.assert_array_equal(cb, ost[li, b].conv_buf)
    stack.close()
    print(f"stack B=64 ctx 32768, 2 steps, sequences {check}: worst rel err "
          f"DeltaNet {worst['dn']:.2e}, GQA {worst['attn']:.2e}")
