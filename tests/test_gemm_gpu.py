"""The prefill projection GEMM (qm_gemm) on the tensor cores against the
reference's gemm over a prompt (src/gemv.rs:294-300): every row of y is the
reference's gemv_q4 of that row of x (the restatement, src/gemv.rs:411-450),
here checked against a float64 product with the same dequantised weights
(and, for a few rows, against the restatement itself).  x arrives as bf16;
W is dequantised to bf16 on the way to the tensor cores (8 bits of
mantissa), so max|gpu - ref| / RMS(ref) <= 2e-2, the prefill tolerance."""
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
    with pytest.raises(qm.QmError) as e:
        mx.gemm(qm.weight_f16(torch.zeros(64, 64, dtype=torch.int16, device="cuda")),
                torch.zeros(4, 64, dtype=torch.int16, device="cuda"), y)
    assert e.value.code == 9


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


@pytest.mark.parametrize("rows", [False, True])
def test_bf16_output_is_the_f32_sum_rounded(ctx, orc, rows):
    """qm_gemm_bf16 rounds the same accumulator qm_gemm stores: bit for bit
    the f32 result rounded to nearest bf16."""
    import torch

    import qora_mixer as qm

    g = np.random.default_rng(11 + rows)
    T, k, n = 300, 2560, 1056
    w = (g.standard_normal((n, k) if rows else (k, n)) * 0.02).astype(np.float32)
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
