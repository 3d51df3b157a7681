"""The prefill projection GEMM (qm_gemm) on the tensor cores against the
reference's gemm over a prompt (src/gemv.rs:294-300): every row of y is the
reference's gemv_q4 of that row of x (the restatement, src/gemv.rs:411-450),
here checked against a float64 product with the same dequantised weights
(and, for a few rows, against the restatement itself).  F16 weights follow
gemm_f16 (src/gemv.rs:390) and are checked the same way against gemv_f16
(src/gemv.rs:361-368) and lm_head_f16 (664-676).  x arrives as bf16; W is
rounded to bf16 on the way to the tensor cores (8 bits of mantissa), so
max|gpu - ref| / RMS(ref) <= 2e-2, the prefill tolerance."""
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


@pytest.mark.parametrize("T,k,n", [(1, 64, 32), (200, 256, 288), (129, 2560, 8192), (300, 4096, 2560),
                                   (1000, 2560, 1024), (37, 2560, 32)])
def test_q4_gemm_matches_reference_rows(ctx, orc, T, k, n):
    import torch

    import qora_mixer as qm

    g = np.random.default_rng(T + k + n)
    w = (g.standard_normal((k, n)) * 0.02).astype(np.float32)
    w[0] = 0.0
    packed, scales = orc.quantize_q4(w)
    xb = I.f32_to_bf16_bits(g.standard_normal((T, k)).astype(np.float32))
    x = I.bf16_bits_to_f32(xb)
    y = torch.full((T, n), float("nan"), device="cuda")
    qm.Mixer(ctx).gemm(qm.weight_q4(dev(packed), dev(scales)), dev(xb), y)
    ctx.sync()
    yg = host(y)
    wd = orc.dequantize_q4(packed, scales).astype(np.float64)
    ref = x.astype(np.float64) @ wd
    assert np.isfinite(yg).all()
    err = refmath.rel_err(yg, ref)
    assert err <= TOL, err
    for t in sorted({0, T // 2, T - 1}):
        assert refmath.rel_err(yg[t], orc.gemv_q4(x[t], packed, scales)) <= TOL


def test_gemm_argument_errors(ctx):
    import torch

    import qora_mixer as qm

    mx = qm.Mixer(ctx)
    x = torch.zeros(4, 96, dtype=torch.int16, device="cuda")
    y = torch.zeros(4, 64, device="cuda")
    pk = torch.zeros(96, 32, dtype=torch.uint8, device="cuda")
    sc = torch.zeros(96, 2, dtype=torch.int16, device="cuda")
    with pytest.raises(qm.QmError) as e:
        mx.gemm(qm.weight_q4(pk, sc), x, y)  # k = 96: not a multiple of 64
    assert e.value.code == 2
    w16 = torch.zeros(64 * 64 + 1, dtype=torch.int16, device="cuda")
    bad = qm.QmWeight(7, 64, 64, w16.data_ptr(), None)  # no such weight kind
    with pytest.raises(qm.QmError) as e:
        mx.gemm(bad, torch.zeros(4, 64, dtype=torch.int16, device="cuda"), y)
    assert e.value.code == 9
    odd = qm.QmWeight(qm.W_F16, 64, 64, w16.data_ptr() + 2, None)  # F16 data 2 bytes off 16
    with pytest.raises(qm.QmError) as e:
        mx.gemm(odd, torch.zeros(4, 64, dtype=torch.int16, device="cuda"), y)
    assert e.value.code == 1


@pytest.mark.parametrize("T,vocab,hidden", [(1, 1024, 2560), (8, 4128, 2560), (64, 20032, 2560), (300, 96, 64)])
def test_q4_rows_gemm_is_batched_lm_head(ctx, orc, T, vocab, hidden):
    """The tied embedding (row layout, groups along hidden) through the same
    GEMM: logits for T sequences at once against the reference's
    lm_head_parallel (src/gemv.rs:677-707) on the bf16-rounded x."""
    import torch

    import qora_mixer as qm

    g = np.random.default_rng(T + vocab)
    e = (g.standard_normal((vocab, hidden)) * 0.02).astype(np.float32)
    e[3] = 0.0
    packed, scales = orc.quantize_q4(e)
    xb = I.f32_to_bf16_bits(g.standard_normal((T, hidden)).astype(np.float32))
    x = I.bf16_bits_to_f32(xb)
    y = torch.full((T, vocab), float("nan"), device="cuda")
    qm.Mixer(ctx).gemm(qm.weight_q4_rows(dev(packed), dev(scales)), dev(xb), y)
    ctx.sync()
    yg = host(y)
    assert np.isfinite(yg).all()
    for t in sorted({0, T // 2, T - 1}):
        assert refmath.rel_err(yg[t], orc.lm_head_q4(x[t], packed, scales)) <= TOL, t
    assert np.all(yg[:, 3] == 0.0)


@pytest.mark.parametrize("rows,f16", [(False, False), (True, False), (False, True)])
def test_bf16_output_is_the_f32_sum_rounded(ctx, orc, rows, f16):
    """qm_gemm_bf16 rounds the same accumulator qm_gemm stores: bit for bit
    the f32 result rounded to nearest bf16 (Q4 in both layouts, F16 [k][n])."""
    import torch

    import qora_mixer as qm

    g = np.random.default_rng(11 + rows + 2 * f16)
    T, k, n = 300, 2560, 1056
    w = (g.standard_normal((n, k) if rows else (k, n)) * 0.02).astype(np.float32)
    if f16:
        wt = qm.weight_f16(dev(w.astype(np.float16).view(np.uint16)))
    else:
        packed, scales = orc.quantize_q4(w)
        wt = qm.weight_q4_rows(dev(packed), dev(scales)) if rows else qm.weight_q4(dev(packed), dev(scales))
    xb = dev(I.f32_to_bf16_bits(g.standard_normal((T, k)).astype(np.float32)))
    y32 = torch.empty(T, n, device="cuda")
    y16 = torch.empty(T, n, dtype=torch.int16, device="cuda")
    mx = qm.Mixer(ctx)
    mx.gemm(wt, xb, y32)
    mx.gemm_bf16(wt, xb, y16)
    ctx.sync()
    np.testing.assert_array_equal(host(y16), I.f32_to_bf16_bits(host(y32)))


def test_prefill_projections_feed_the_prefill_mixer(ctx, orc):
    """A DeltaNet layer's prefill on the device end to end: x_norm (bf16) ->
    qm_gemm_bf16 (in_proj_qkv, src/gemv.rs:1114) and qm_gemm (in_proj_a / b,
    1115-1116) -> qm_dn_prefill, the mixer's output against the sequential
    restatement (src/gemv.rs:1119-1219) run on the projections the device
    produced, and those projections against the reference's gemv."""
    import torch

    import qora_mixer as qm

    T = 512
    g = np.random.default_rng(21)
    p = I.dn_layer_params(I.rng(22))
    keep = [dev(p["conv_w"]), dev(p["a_log"]), dev(p["dt_bias"]), dev(p["norm_gamma"])]
    prm = qm.dn_params(*keep)
    ws = {name: orc.quantize_q4((g.standard_normal((2560, n)) * 0.02).astype(np.float32))
          for name, n in (("qkv", 8192), ("a", 32), ("b", 32))}
    dws = {name: qm.weight_q4(dev(pk), dev(sc)) for name, (pk, sc) in ws.items()}
    xb = I.f32_to_bf16_bits(g.standard_normal((T, 2560)).astype(np.float32))
    xd = dev(xb)
    mx = qm.Mixer(ctx)
    qkv = torch.empty(1, T, 8192, dtype=torch.int16, device="cuda")
    a = torch.empty(1, T, 32, device="cuda")
    b = torch.empty(1, T, 32, device="cuda")
    mx.gemm_bf16(dws["qkv"], xd, qkv.view(T, 8192))
    mx.gemm(dws["a"], xd, a.view(T, 32))
    mx.gemm(dws["b"], xd, b.view(T, 32))
    st = qm.DnState(ctx, 1)
    y = torch.full((1, T, 32, 128), float("nan"), device="cuda")
    mx.dn_prefill(prm, st, T, qkv, a, b, y)
    ctx.sync()
    qkv_h, a_h, b_h = host(qkv)[0], host(a)[0], host(b)[0]
    x = I.bf16_bits_to_f32(xb)
    for t in (0, T - 1):
        assert refmath.rel_err(I.bf16_bits_to_f32(qkv_h[t]), orc.gemv_q4(x[t], *ws["qkv"])) <= TOL
        assert refmath.rel_err(a_h[t], orc.gemv_q4(x[t], *ws["a"])) <= TOL
    c = orc.cfg_4b()
    yo = orc.dn_prefill(c, orc.DnState(c), qkv_h, a_h, b_h, p["conv_w"], p["a_log"], p["dt_bias"])
    assert refmath.rel_err(host(y)[0], yo) <= TOL
    st.close()


def test_prefill_projections_feed_the_attention_prefill(ctx, orc):
    """An attention layer's prefill end to end on the device: x_norm (bf16) ->
    qm_gemm_bf16 for q_proj / k_proj / v_proj (src/gemv.rs:1366, 1384-1385;
    q_proj's [T, 16 x 512] is the per-head [Q, gate] layout the mixer takes) ->
    qm_gqa_prefill, against the restatement (src/gemv.rs:1364-1444) on the
    projections the device produced (sampled rows)."""
    import torch

    import qora_mixer as qm

    T = 400
    g = np.random.default_rng(31)
    pr = I.gqa_layer_params(I.rng(32), T + 1)
    cos, sin = qm.rope_table(1.0e7, 64, T + 1)
    keep = [dev(pr["q_norm"]), dev(pr["k_norm"]), dev(cos), dev(sin)]
    prm = qm.gqa_params(*keep)
    ws = {name: orc.quantize_q4((g.standard_normal((2560, n)) * 0.02).astype(np.float32))
          for name, n in (("q", 8192), ("k", 1024), ("v", 1024))}
    dws = {name: qm.weight_q4(dev(pk), dev(sc)) for name, (pk, sc) in ws.items()}
    xd = dev(I.f32_to_bf16_bits(g.standard_normal((T, 2560)).astype(np.float32)))
    mx = qm.Mixer(ctx)
    qg = torch.empty(1, T, 16, 512, dtype=torch.int16, device="cuda")
    kk = torch.empty(1, T, 4, 256, dtype=torch.int16, device="cuda")
    vv = torch.empty(1, T, 4, 256, dtype=torch.int16, device="cuda")
    mx.gemm_bf16(dws["q"], xd, qg.view(T, 8192))
    mx.gemm_bf16(dws["k"], xd, kk.view(T, 1024))
    mx.gemm_bf16(dws["v"], xd, vv.view(T, 1024))
    K = torch.zeros(1, 4, T, 256, dtype=torch.int16, device="cuda")
    V = torch.zeros_like(K)
    kv = qm.KvCache(ctx, 1, T, K, V)
    out = torch.full((1, T, 16, 256), float("nan"), device="cuda")
    mx.gqa_prefill(prm, kv, T, qg, kk, vv, out)
    ctx.sync()
    c = orc.cfg_4b()
    rows = np.array([0, 1, 127, 128, 255, 399])
    ref = orc.gqa_prefill_rows(c, host(qg)[0].reshape(T, -1), host(kk)[0].reshape(T, -1),
                               host(vv)[0].reshape(T, -1), pr["q_norm"], pr["k_norm"], cos, sin, rows)
    assert refmath.rel_err(host(out)[0][rows], ref) <= TOL
    kv.close()


@pytest.mark.parametrize("T,k,n", [(1, 64, 32), (200, 256, 288), (129, 2560, 8192), (300, 4096, 2560),
                                   (37, 2560, 32)])
def test_f16_gemm_matches_reference_rows(ctx, orc, T, k, n):
    """F16 weights [k][n] (gemm_f16, src/gemv.rs:390) against a float64
    product of the same f16 values and, for a few rows, gemv_f16."""
    import torch

    import qora_mixer as qm

    g = np.random.default_rng(T + k + n + 5)
    w16 = (g.standard_normal((k, n)) * 0.02).astype(np.float16)
    w16[0] = 0.0
    wb = w16.view(np.uint16)
    xb = I.f32_to_bf16_bits(g.standard_normal((T, k)).astype(np.float32))
    x = I.bf16_bits_to_f32(xb)
    y = torch.full((T, n), float("nan"), device="cuda")
    qm.Mixer(ctx).gemm(qm.weight_f16(dev(wb)), dev(xb), y)
    ctx.sync()
    yg = host(y)
    assert np.isfinite(yg).all()
    ref = x.astype(np.float64) @ w16.astype(np.float64)
    assert refmath.rel_err(yg, ref) <= TOL
    for t in sorted({0, T // 2, T - 1}):
        assert refmath.rel_err(yg[t], orc.gemv_f16(x[t], wb)) <= TOL


@pytest.mark.parametrize("T,vocab,hidden", [(1, 1024, 2560), (64, 20032, 2560), (300, 96, 64)])
def test_f16_rows_gemm_is_batched_lm_head(ctx, orc, T, vocab, hidden):
    """An f16 tied embedding (row layout) as a batched lm_head against
    lm_head_f16 (src/gemv.rs:664-676), bf16 output rounded from the same sum."""
    import torch

    import qora_mixer as qm

    g = np.random.default_rng(T + vocab + 9)
    e16 = (g.standard_normal((vocab, hidden)) * 0.02).astype(np.float16)
    e16[3] = 0.0
    eb = e16.view(np.uint16)
    xb = I.f32_to_bf16_bits(g.standard_normal((T, hidden)).astype(np.float32))
    x = I.bf16_bits_to_f32(xb)
    wt = qm.weight_f16_rows(dev(eb))
    y = torch.full((T, vocab), float("nan"), device="cuda")
    y16 = torch.empty(T, vocab, dtype=torch.int16, device="cuda")
    mx = qm.Mixer(ctx)
    mx.gemm(wt, dev(xb), y)
    mx.gemm_bf16(wt, dev(xb), y16)
    ctx.sync()
    yg = host(y)
    assert np.isfinite(yg).all()
    for t in sorted({0, T // 2, T - 1}):
        assert refmath.rel_err(yg[t], orc.lm_head_f16(x[t], eb)) <= TOL, t
    assert np.all(yg[:, 3] == 0.0)
    np.testing.assert_array_equal(host(y16), I.f32_to_bf16_bits(yg))


def test_split_k_repeats_and_shares_scratch_with_gemv(ctx, orc):
    """A short prompt splits K (32 tiles of 256 x 256 on 148 SMs): the same
    call repeated, with a split-K qm_gemv between them on the same scratch
    area and counters, gives the same bits, and both match the reference."""
    import torch

    import qora_mixer as qm

    g = np.random.default_rng(29)
    T, k, n = 100, 2560, 8192
    w = (g.standard_normal((k, n)) * 0.02).astype(np.float32)
    packed, scales = orc.quantize_q4(w)
    wt = qm.weight_q4(dev(packed), dev(scales))
    xb = I.f32_to_bf16_bits(g.standard_normal((T, k)).astype(np.float32))
    x = I.bf16_bits_to_f32(xb)
    mx = qm.Mixer(ctx)
    y1 = torch.empty(T, n, device="cuda")
    y2 = torch.empty(T, n, device="cuda")
    yv = torch.empty(2, n, device="cuda")
    mx.gemm(wt, dev(xb), y1)
    mx.gemv(wt, dev(x[:2]), yv)
    mx.gemm(wt, dev(xb), y2)
    ctx.sync()
    np.testing.assert_array_equal(host(y1), host(y2))
    ref = x.astype(np.float64) @ orc.dequantize_q4(packed, scales).astype(np.float64)
    assert refmath.rel_err(host(y1), ref) <= TOL
    for b in range(2):
        assert refmath.rel_err(host(yv)[b], orc.gemv_q4(x[b], packed, scales)) <= 5e-5
