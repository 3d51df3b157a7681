"""qm_dn_prefill_host / qm_gqa_prefill_host (the reference's host-resident
prefill flow, src/gpu_inference.rs:464-476 and 591-604 for DeltaNet,
690-766 for GQA) against the device-buffer calls: the same kernels run on
the same bytes, so outputs, states and caches must agree bit for bit, and
the first call is also checked against the CPU restatement.
"""
import numpy as np
import pytest

import refmath
from gpu_util import dev, host, make_ctx
from qora_mixer import inputs as I

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ctx():
    c = make_ctx()
    yield c
    c.close()


@pytest.mark.parametrize("B,T,gate", [(2, 200, True), (1, 77, False)])
def test_dn_prefill_host_matches_device(ctx, orc, B, T, gate):
    import torch

    import qora_mixer as qm

    g = I.rng(1300 + T)
    p = I.dn_layer_params(g)
    keep = [dev(p["conv_w"]), dev(p["a_log"]), dev(p["dt_bias"]), dev(p["norm_gamma"])]
    prm = qm.dn_params(*keep)
    qkv = I.f32_to_bf16_bits(g.standard_normal((B, T, 8192), dtype=np.float32))
    a = g.standard_normal((B, T, 32), dtype=np.float32)
    b = g.standard_normal((B, T, 32), dtype=np.float32)
    z = g.standard_normal((B, T, 4096), dtype=np.float32) if gate else None
    mx = qm.Mixer(ctx)
    st_d, st_h = qm.DnState(ctx, B), qm.DnState(ctx, B)
    y_d = torch.empty(B, T, 32, 128, device="cuda")
    o_d = torch.empty(B, T, 4096, device="cuda") if gate else None
    mx.dn_prefill(prm, st_d, T, dev(qkv), dev(a), dev(b), y_d, dev(z) if gate else None, o_d)
    ctx.sync()
    y_h = np.full((B, T, 32, 128), np.nan, np.float32)
    o_h = np.full((B, T, 4096), np.nan, np.float32) if gate else None
    n0 = ctx.host_calls()
    mx.dn_prefill_host(prm, st_h, T, qkv, a, b, y_h, z, o_h)
    assert ctx.host_calls()[1] == n0[1] + 1  # a staged call
    np.testing.assert_array_equal(y_h, host(y_d))
    if gate:
        np.testing.assert_array_equal(o_h, host(o_d))
    assert st_h.conv_pos == st_d.conv_pos == T
    for bi in range(B):
        s1, c1 = st_h.read(bi)
        s2, c2 = st_d.read(bi)
        np.testing.assert_array_equal(s1, s2)
        np.testing.assert_array_equal(c1, c2)
    # and the first sequence against the sequential recurrence (src/gemv.rs:1119-1219)
    c = orc.cfg_4b()
    ost = orc.DnState(c)
    ref = orc.dn_prefill(c, ost, qkv[0], a[0], b[0], p["conv_w"], p["a_log"], p["dt_bias"])
    assert refmath.rel_err(y_h[0], ref) <= 2e-2
    st_d.close()
    st_h.close()


def test_gqa_prefill_host_matches_device(ctx, orc):
    import torch

    import qora_mixer as qm

    B, T, cap = 2, 300, 320
    g = I.rng(1400)
    pr = I.gqa_layer_params(g, cap + 1)
    cos, sin = qm.rope_table(1.0e7, 64, cap + 1)
    keep = [dev(pr["q_norm"]), dev(pr["k_norm"]), dev(cos), dev(sin)]
    prm = qm.gqa_params(*keep)
    qg = I.f32_to_bf16_bits(g.standard_normal((B, T, 16, 512), dtype=np.float32))
    kk = I.f32_to_bf16_bits(g.standard_normal((B, T, 4, 256), dtype=np.float32))
    vv = I.f32_to_bf16_bits(g.standard_normal((B, T, 4, 256), dtype=np.float32))
    mx = qm.Mixer(ctx)
    K1 = torch.zeros(B, 4, cap, 256, dtype=torch.int16, device="cuda")
    V1 = torch.zeros_like(K1)
    K2, V2 = K1.clone(), V1.clone()
    kv_d, kv_h = qm.KvCache(ctx, B, cap, K1, V1), qm.KvCache(ctx, B, cap, K2, V2)
    o_d = torch.empty(B, T, 16, 256, device="cuda")
    mx.gqa_prefill(prm, kv_d, T, dev(qg), dev(kk), dev(vv), o_d)
    ctx.sync()
    o_h = np.full((B, T, 16, 256), np.nan, np.float32)
    mx.gqa_prefill_host(prm, kv_h, T, qg, kk, vv, o_h)
    np.testing.assert_array_equal(o_h, host(o_d))
    np.testing.assert_array_equal(host(K2), host(K1))
    np.testing.assert_array_equal(host(V2), host(V1))
    assert kv_h.seq_len == kv_d.seq_len == T
    c = orc.cfg_4b()
    ref = orc.gqa_prefill_rows(c, qg[0].reshape(T, -1), kk[0].reshape(T, -1), vv[0].reshape(T, -1),
                               pr["q_norm"], pr["k_norm"], cos, sin, np.arange(T))
    assert refmath.rel_err(o_h[0], ref) <= 2e-2
    kv_d.close()
    kv_h.close()


def test_host_prefill_argument_errors(ctx):
    import qora_mixer as qm

    st = qm.DnState(ctx, 1)
    g = I.rng(1500)
    p = I.dn_layer_params(g)
    keep = [dev(p["conv_w"]), dev(p["a_log"]), dev(p["dt_bias"])]
    prm = qm.dn_params(*keep)
    qkv = np.zeros((1, 4, 8192), np.uint16)
    ab = np.zeros((1, 4, 32), np.float32)
    y = np.zeros((1, 4, 32, 128), np.float32)
    with pytest.raises(qm.QmError) as e:
        qm.Mixer(ctx).dn_prefill_host(prm, st, 0, qkv, ab, ab, y)
    assert e.value.code == 1  # QM_E_ARG: T <= 0
    with pytest.raises(qm.QmError) as e:
        qm.Mixer(ctx).dn_prefill_host(prm, st, 4, qkv, ab, ab, None)
    assert e.value.code == 1  # QM_E_ARG: y is required
    assert st.conv_pos == 0
    st.close()
