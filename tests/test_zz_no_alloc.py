"""qm_gqa_decode_noalloc: GQA decode for callers that cannot allocate device
memory (an engine whose allocator owns all of HBM, or a plugin that only
borrows its host's buffers and stream).

Checks the entry point through the C ABI against the regular entry point
(qm_gqa_decode) on two calls in a row.  Both run the same three kernels with
the same split plan, so the outputs must agree bit for bit (a tolerance
could hide a wrong partial layout).  Also checks the documented size limit
from both sides: batch 16 at 32K context fits the fixed scratch on a
148-SM B200 and batch 64 at 32K is refused.  The
file sorts last so that a run stopping at the first failure has run every
other test; it also passes on its own in a fresh process.
"""
import numpy as np
import pytest

from gpu_util import dev, host, make_ctx
from qora_mixer import inputs as I

pytestmark = pytest.mark.gpu


def test_noalloc_matches_regular_entry_point_two_calls():
    import torch

    import qora_mixer as qm

    ctx = make_ctx()
    B, L, cap = 2, 1000, 1010
    g = I.rng(600)
    pr = I.gqa_layer_params(g, cap + 1)
    cos, sin = qm.rope_table(1.0e7, 64, cap + 1)
    kb, vb = I.gqa_cache_bf16(g, B, L)
    K1 = torch.zeros(B, 4, cap, 256, dtype=torch.int16, device="cuda")
    V1 = torch.zeros_like(K1)
    K1[:, :, :L] = dev(kb)
    V1[:, :, :L] = dev(vb)
    K2, V2 = K1.clone(), V1.clone()
    keep = [dev(pr["q_norm"]), dev(pr["k_norm"]), dev(cos), dev(sin)]
    prm = qm.gqa_params(*keep)
    kv = qm.KvCache(ctx, B, cap, K1, V1)
    kv.seq_len = L
    mx = qm.Mixer(ctx)
    stream = torch.cuda.current_stream()
    seq = L
    for step in range(2):
        tok = I.gqa_token_inputs(g, B)
        q, k, v = dev(tok["q_gate"]), dev(tok["k_new"]), dev(tok["v_new"])
        out_ref = torch.empty(B, 16, 256, device="cuda")
        out_na = torch.full((B, 16, 256), float("nan"), device="cuda")
        mx.gqa_decode(prm, kv, q, k, v, out_ref)
        rc = qm.gqa_decode_noalloc(prm, K2, V2, B, cap, seq, q, k, v, out_na, stream)
        assert rc == 0, qm.STATUS.get(rc, rc)
        seq += 1
        torch.cuda.synchronize()
        np.testing.assert_array_equal(host(out_na), host(out_ref))
        np.testing.assert_array_equal(host(K2[:, :, : seq]), host(K1[:, :, : seq]))
        np.testing.assert_array_equal(host(V2[:, :, : seq]), host(V1[:, :, : seq]))
    assert kv.seq_len == seq
    kv.close()
    ctx.close()


def test_noalloc_rejects_requests_beyond_its_scratch():
    import torch

    import qora_mixer as qm

    g = I.rng(601)
    pr = I.gqa_layer_params(g, 40000)
    cos, sin = qm.rope_table(1.0e7, 64, 40000)
    keep = [dev(pr["q_norm"]), dev(pr["k_norm"]), dev(cos), dev(sin)]
    prm = qm.gqa_params(*keep)
    small = torch.zeros(16, dtype=torch.int16, device="cuda")
    q = torch.zeros(64, 16, 512, device="cuda")
    kn = torch.zeros(64, 4, 256, device="cuda")
    out = torch.zeros(64, 16, 256, device="cuda")
    # 64 sequences at 32K context need ~70 MB of partials: refused before any launch
    rc = qm.gqa_decode_noalloc(prm, small, small, 64, 32800, 32768, q, kn, kn, out,
                               torch.cuda.current_stream())
    assert rc == 2  # QM_E_SHAPE
    rc = qm.gqa_decode_noalloc(prm, small, small, 1, 8, 8, q, kn, kn, out, None)
    assert rc == 7  # QM_E_RANGE: cache full


def test_noalloc_batch16_at_32k_context_fits():
    """The documented boundary: 16 sequences with 32767 cached positions run
    (QM_OK) and match qm_gqa_decode bit for bit."""
    import torch

    import qora_mixer as qm

    ctx = make_ctx()
    B, L, cap = 16, 32767, 32768
    g = I.rng(602)
    pr = I.gqa_layer_params(g, cap + 1)
    cos, sin = qm.rope_table(1.0e7, 64, cap + 1)
    K1 = I.device_normal_bf16((B, 4, cap, 256), 6021).view(torch.int16)
    V1 = I.device_normal_bf16((B, 4, cap, 256), 6022).view(torch.int16)
    K2, V2 = K1.clone(), V1.clone()
    keep = [dev(pr["q_norm"]), dev(pr["k_norm"]), dev(cos), dev(sin)]
    prm = qm.gqa_params(*keep)
    kv = qm.KvCache(ctx, B, cap, K1, V1)
    kv.seq_len = L
    tok = I.gqa_token_inputs(g, B)
    q, k, v = dev(tok["q_gate"]), dev(tok["k_new"]), dev(tok["v_new"])
    out_ref = torch.empty(B, 16, 256, device="cuda")
    out_na = torch.full((B, 16, 256), float("nan"), device="cuda")
    qm.Mixer(ctx).gqa_decode(prm, kv, q, k, v, out_ref)
    rc = qm.gqa_decode_noalloc(prm, K2, V2, B, cap, L, q, k, v, out_na, torch.cuda.current_stream())
    assert rc == 0, qm.STATUS.get(rc, rc)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(host(out_na), host(out_ref))
    np.testing.assert_array_equal(host(K2[:, :, L]), host(K1[:, :, L]))
    kv.close()
    ctx.close()
