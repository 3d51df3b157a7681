"""Projections around the mixers: the Q4 / F16 weight GEMV (qm_gemv) against the
CPU restatement of the reference's scalar paths (src/gemv.rs:361-368, 411-450;
Q4 format src/convert.rs:437-467).  The CPU restatement adds in row order, the
GPU in a fixed split order, so the two differ by f32 rounding only (up to
k = 4096 products of order one per output): max|gpu - cpu| / RMS(cpu) <= 5e-5.
A lost row or group moves the result by ~1/sqrt(k) >= 1.5e-2 of its RMS."""
import numpy as np
import pytest

import refmath
from gpu_util import dev, host, make_ctx

pytestmark = pytest.mark.gpu
TOL = 5e-5


@pytest.fixture(scope="module")
def ctx():
    c = make_ctx()
    yield c
    c.close()


def _q4(orc, g, k, n, zero_rows=(), zero_groups=()):
    w = (g.standard_normal((k, n)) * 0.02).astype(np.float32)
    for r in zero_rows:
        w[r] = 0.0
    for r, grp in zero_groups:
        w[r, grp * 32:(grp + 1) * 32] = 0.0
    return orc.quantize_q4(w)


# the mixer projections of one layer (hidden 2560): in_proj_qkv, in_proj_z,
# in_proj_a/b, out_proj, q_proj, k/v_proj, o_proj; plus ragged shapes
@pytest.mark.parametrize("k,n", [(2560, 8192), (2560, 4096), (2560, 32), (4096, 2560), (2560, 1024),
                                 (7, 96), (33, 288), (1000, 1056)])
@pytest.mark.parametrize("batch", [1, 3, 6])
def test_q4_gemv_matches_restatement(ctx, orc, k, n, batch):
    import torch

    import qora_mixer as qm

    g = np.random.default_rng(k * 31 + n + batch)
    packed, scales = _q4(orc, g, k, n, zero_rows=(0,), zero_groups=((min(1, k - 1), 0),))
    x = g.standard_normal((batch, k)).astype(np.float32)
    x[:, min(2, k - 1)] = 0.0
    p_d, s_d, x_d = dev(packed), dev(scales), dev(x)
    y = torch.full((batch, n), float("nan"), device="cuda")
    qm.Mixer(ctx).gemv(qm.weight_q4(p_d, s_d), x_d, y)
    ctx.sync()
    yg = host(y)
    for b in range(batch):
        ref = orc.gemv_q4(x[b], packed, scales)
        assert refmath.rel_err(yg[b], ref) <= TOL, (b, refmath.rel_err(yg[b], ref))


@pytest.mark.parametrize("k,n", [(2560, 4096), (4096, 2560), (9, 24)])
@pytest.mark.parametrize("batch", [1, 4, 5])
def test_f16_gemv_matches_restatement(ctx, orc, k, n, batch):
    import torch

    import qora_mixer as qm

    g = np.random.default_rng(k + 7 * n + batch)
    w16 = (g.standard_normal((k, n)) * 0.02).astype(np.float16).view(np.uint16)
    x = g.standard_normal((batch, k)).astype(np.float32)
    y = torch.full((batch, n), float("nan"), device="cuda")
    qm.Mixer(ctx).gemv(qm.weight_f16(dev(w16)), dev(x), y)
    ctx.sync()
    yg = host(y)
    for b in range(batch):
        assert refmath.rel_err(yg[b], orc.gemv_f16(x[b], w16)) <= TOL


def test_gemv_argument_errors(ctx):
    import torch

    import qora_mixer as qm

    mx = qm.Mixer(ctx)
    x = torch.zeros(1, 64, device="cuda")
    y = torch.zeros(1, 48, device="cuda")
    packed = torch.zeros(64, 24, dtype=torch.uint8, device="cuda")
    scales = torch.zeros(64, 2, dtype=torch.int16, device="cuda")
    with pytest.raises(qm.QmError) as e:
        mx.gemv(qm.weight_q4(packed, scales), x, y)  # n = 48: not a multiple of 32
    assert e.value.code == 2  # QM_E_SHAPE
    w = qm.QmWeight(7, 64, 64, packed.data_ptr(), scales.data_ptr())
    with pytest.raises(qm.QmError) as e:
        mx.gemv(w, x, torch.zeros(1, 64, device="cuda"))
    assert e.value.code == 1  # QM_E_ARG: unknown weight kind


@pytest.mark.parametrize("batch", [1, 5])
@pytest.mark.parametrize("layer", ["deltanet", "gqa"])
def test_multi_weight_launch_matches_restatement(ctx, orc, layer, batch):
    """qm_gemv_multi: the projections of one layer that share x_norm in one
    launch (in_proj_qkv / a / b / z, src/gemv.rs:742,788-789,865; q / k /
    v_proj, src/gemv.rs:928,941-942), each output checked alone."""
    import torch

    import qora_mixer as qm

    ns = [8192, 32, 32, 4096] if layer == "deltanet" else [8192, 1024, 1024]
    g = np.random.default_rng(len(ns) * 100 + batch)
    k = 2560
    qs = [_q4(orc, g, k, n) for n in ns]
    dq = [(dev(p), dev(s)) for p, s in qs]
    x = g.standard_normal((batch, k)).astype(np.float32)
    ys = [torch.full((batch, n), float("nan"), device="cuda") for n in ns]
    n0 = ctx.launch_count()
    qm.Mixer(ctx).gemv_multi([qm.weight_q4(p, s) for p, s in dq], dev(x), ys)
    ctx.sync()
    assert ctx.launch_count() - n0 == (batch + 3) // 4
    for (p, s), y in zip(qs, ys):
        yg = host(y)
        for b in range(batch):
            assert refmath.rel_err(yg[b], orc.gemv_q4(x[b], p, s)) <= TOL


def test_dependent_chain_and_graph_replay(ctx, orc):
    """Each launch reads its x only after the preceding kernel of the stream is
    done (its weight loads may start earlier): a chain x -> W1 -> W2 -> W3
    where every input is the previous output matches the restatement, issued
    directly and replayed from a CUDA graph."""
    import torch

    import qora_mixer as qm

    g = np.random.default_rng(77)
    shapes = [(2560, 4096), (4096, 2560), (2560, 8192)]
    qs = [_q4(orc, g, k, n) for k, n in shapes]
    dq = [(dev(p), dev(s)) for p, s in qs]
    ws = [qm.weight_q4(p, s) for p, s in dq]
    x = g.standard_normal((2, 2560)).astype(np.float32)
    ref = x
    for p, s in qs:
        ref = np.stack([orc.gemv_q4(r, p, s) for r in ref])
    mx = qm.Mixer(ctx)
    xd = dev(x)
    ys = [torch.empty(2, n, device="cuda") for _, n in shapes]

    def chain():
        inp = xd
        for w, y in zip(ws, ys):
            mx.gemv(w, inp, y)
            inp = y

    chain()
    ctx.sync()
    assert refmath.rel_err(host(ys[-1]), ref) <= 3 * TOL
    side = torch.cuda.Stream()
    graph = torch.cuda.CUDAGraph()
    for y in ys:
        y.fill_(float("nan"))
    torch.cuda.synchronize()
    ctx.set_stream(side)
    try:
        with torch.cuda.graph(graph, stream=side):
            chain()
    finally:
        ctx.set_stream(torch.cuda.current_stream())
    for y in ys:
        y.fill_(float("nan"))
    for _ in range(3):
        graph.replay()
    torch.cuda.synchronize()
    assert refmath.rel_err(host(ys[-1]), ref) <= 3 * TOL
    del graph


def test_multi_weight_mismatch(ctx):
    import torch

    import qora_mixer as qm

    p1 = torch.zeros(64, 16, dtype=torch.uint8, device="cuda")
    s1 = torch.zeros(64, 1, dtype=torch.int16, device="cuda")
    p2 = torch.zeros(32, 16, dtype=torch.uint8, device="cuda")
    s2 = torch.zeros(32, 1, dtype=torch.int16, device="cuda")
    x = torch.zeros(1, 64, device="cuda")
    ys = [torch.zeros(1, 32, device="cuda"), torch.zeros(1, 32, device="cuda")]
    with pytest.raises(qm.QmError) as e:
        qm.Mixer(ctx).gemv_multi([qm.weight_q4(p1, s1), qm.weight_q4(p2, s2)], x, ys)
    assert e.value.code == 8  # QM_E_MISMATCH: k differs
