"""Calls inside CUDA-graph capture that would have to allocate.

A workspace that must grow cannot be allocated while a stream is being
captured (cudaMalloc is not capturable), so the library refuses the call with
QM_E_CAPTURE before it issues anything: the capture stays valid, and the same
call made outside the capture (or after qm_ctx_reserve) then works.
"""
import numpy as np
import pytest

import refmath
from gpu_util import dev, host

pytestmark = pytest.mark.gpu

QM_E_CAPTURE = 10


def _prefill_case(seed, T):
    from qora_mixer import inputs as I

    g = I.rng(seed)
    p = I.dn_layer_params(g)
    qkv = I.f32_to_bf16_bits(g.standard_normal((1, T, 8192), dtype=np.float32))
    a = g.standard_normal((1, T, 32), dtype=np.float32)
    b = g.standard_normal((1, T, 32), dtype=np.float32)
    return p, qkv, a, b


@pytest.mark.filterwarnings("ignore:The CUDA Graph is empty")  # the refused call captured nothing
def test_workspace_growth_inside_capture_is_refused():
    import torch

    import qora_mixer as qm
    from oracle import oracle as orc

    T = 100
    p, qkv, a, b = _prefill_case(0xCA97, T)
    side = torch.cuda.Stream()
    ctx = qm.Ctx(0, stream=side)  # a fresh context: no workspace yet
    try:
        keep = [dev(p["conv_w"]), dev(p["a_log"]), dev(p["dt_bias"])]
        prm = qm.dn_params(*keep)
        st = qm.DnState(ctx, 1)
        y = torch.full((1, T, 32, 128), float("nan"), device="cuda")
        qd, ad, bd = dev(qkv), dev(a), dev(b)
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        code = None
        with torch.cuda.graph(graph, stream=side):
            try:
                qm.Mixer(ctx).dn_prefill(prm, st, T, qd, ad, bd, y)
            except qm.QmError as e:
                code = e.code
        assert code == QM_E_CAPTURE
        assert st.conv_pos == 0  # the refused call changed nothing
        del graph
        # outside the capture the same call grows the workspace and runs
        qm.Mixer(ctx).dn_prefill(prm, st, T, qd, ad, bd, y)
        ctx.sync()
        ost = orc.DnState(orc.cfg_4b())
        ref = orc.dn_prefill(orc.cfg_4b(), ost, qkv[0], a[0], b[0], p["conv_w"], p["a_log"], p["dt_bias"])
        assert refmath.rel_err(host(y)[0], ref) <= 2e-2
        st.close()
    finally:
        ctx.close()


def test_captured_call_replays_bit_exact():
    """Once a direct call has grown the workspace, the same call captured into
    a CUDA graph and replayed gives the direct call's output bit for bit."""
    import torch

    import qora_mixer as qm

    T = 100
    p, qkv, a, b = _prefill_case(0xCA98, T)
    side = torch.cuda.Stream()
    ctx = qm.Ctx(0, stream=side)
    try:
        keep = [dev(p["conv_w"]), dev(p["a_log"]), dev(p["dt_bias"])]
        prm = qm.dn_params(*keep)
        qd, ad, bd = dev(qkv), dev(a), dev(b)
        st_ref = qm.DnState(ctx, 1)
        y_ref = torch.empty(1, T, 32, 128, device="cuda")
        qm.Mixer(ctx).dn_prefill(prm, st_ref, T, qd, ad, bd, y_ref)
        ctx.sync()
        st = qm.DnState(ctx, 1)
        y = torch.full((1, T, 32, 128), float("nan"), device="cuda")
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=side):
            qm.Mixer(ctx).dn_prefill(prm, st, T, qd, ad, bd, y)
        graph.replay()
        torch.cuda.synchronize()
        ctx.sync()
        np.testing.assert_array_equal(host(y), host(y_ref))
        del graph
        st.close()
        st_ref.close()
    finally:
        ctx.close()
