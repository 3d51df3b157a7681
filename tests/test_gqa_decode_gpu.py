"""GQA decode on the GPU vs the CPU restatement of src/gemv.rs:927-1011.

The cache positions already present are bf16 (configs 1 and 4); the oracle
attends over exactly those values widened to f32 plus the new token in f32,
as the reference would after loading them.  After each step the oracle's
copy of the appended row is replaced by the widened bf16 row the GPU stored,
so multi-step runs compare like with like.
Tolerance: max|gpu - cpu| / RMS(cpu) <= 1e-3.
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


def _setup(ctx, orc, B, L, cap, seed, max_pos=None):
    import torch

    import qora_mixer as qm

    g = I.rng(seed)
    max_pos = max_pos or cap + 1
    pr = I.gqa_layer_params(g, max_pos)
    cos, sin = qm.rope_table(1.0e7, 64, max_pos)
    K = torch.zeros(B, 4, cap, 256, dtype=torch.int16, device="cuda")
    V = torch.zeros_like(K)
    c = orc.cfg_4b()
    okv = []
    if L > 0:
        kb, vb = I.gqa_cache_bf16(g, B, L)
        K[:, :, :L] = dev(kb)
        V[:, :, :L] = dev(vb)
    for bi in range(B):
        kv = orc.KvCache(c, cap + 1)
        if L > 0:
            kv.k[:L] = I.bf16_bits_to_f32(kb[bi]).transpose(1, 0, 2)
            kv.v[:L] = I.bf16_bits_to_f32(vb[bi]).transpose(1, 0, 2)
            kv.seq_len[0] = L
        okv.append(kv)
    kvh = qm.KvCache(ctx, B, cap, K, V)
    kvh.seq_len = L
    keep = [dev(pr["q_norm"]), dev(pr["k_norm"]), dev(cos), dev(sin)]
    prm = qm.gqa_params(*keep)
    return g, c, pr, cos, sin, K, V, okv, kvh, prm, keep


def _steps(ctx, orc, B, L, cap, steps, seed):
    import torch

    import qora_mixer as qm

    g, c, pr, cos, sin, K, V, okv, kvh, prm, keep = _setup(ctx, orc, B, L, cap, seed)
    mx = qm.Mixer(ctx)
    out = torch.empty(B, 16, 256, device="cuda")
    worst = 0.0
    for s in range(steps):
        tok = I.gqa_token_inputs(g, B)
        pos = L + s
        mx.gqa_decode(prm, kvh, dev(tok["q_gate"]), dev(tok["k_new"]), dev(tok["v_new"]), out)
        ctx.sync()
        og = host(out)
        kg = host(K[:, :, pos])  # [B,4,256] bf16 bits appended by the GPU
        vg = host(V[:, :, pos])
        for bi in range(B):
            ref = orc.gqa_decode(c, okv[bi], tok["q_gate"][bi], tok["k_new"][bi], tok["v_new"][bi],
                                 pr["q_norm"], pr["k_norm"], cos, sin)
            worst = max(worst, refmath.rel_err(og[bi], ref))
            # appended row = bf16(post-norm/RoPE k), bf16(raw v): within one bf16 ulp
            ko = okv[bi].k[pos]
            kgf = I.bf16_bits_to_f32(kg[bi])
            assert np.all(np.abs(kgf - ko) <= np.abs(ko) * 2.0 ** -8 + 1e-4)
            np.testing.assert_array_equal(vg[bi], I.f32_to_bf16_bits(tok["v_new"][bi]))
            okv[bi].k[pos] = kgf
            okv[bi].v[pos] = I.bf16_bits_to_f32(vg[bi])
        assert kvh.seq_len == pos + 1
    assert worst <= TOL, f"rel err {worst:.3e}"
    return worst


def test_config1_decode_L4096(ctx, orc):
    """Config 1: batch 1, 4096 cached bf16 positions, new token at position 4096."""
    _steps(ctx, orc, B=1, L=4096, cap=4100, steps=1, seed=0x51A0 + 1)


@pytest.mark.parametrize("B,L", [(1, 0), (1, 1), (2, 63), (2, 64), (3, 65), (1, 200), (2, 1000)])
def test_decode_edge_lengths(ctx, orc, B, L):
    """Empty cache, partial tiles, tile boundaries, odd batch sizes; 3 steps each."""
    _steps(ctx, orc, B=B, L=L, cap=L + 8, steps=3, seed=400 + L + B)


def test_decode_long_context_batch(ctx, orc):
    """Config-4 context length (32768 cached positions) at batch 2."""
    _steps(ctx, orc, B=2, L=32768, cap=32770, steps=1, seed=0x51A0 + 4)


def test_cache_full_and_rope_range_errors(ctx, orc):
    import torch

    import qora_mixer as qm

    g, c, pr, cos, sin, K, V, okv, kvh, prm, keep = _setup(ctx, orc, 1, 8, 8, 500)
    mx = qm.Mixer(ctx)
    tok = I.gqa_token_inputs(g, 1)
    out = torch.empty(1, 16, 256, device="cuda")
    with pytest.raises(qm.QmError) as e:
        mx.gqa_decode(prm, kvh, dev(tok["q_gate"]), dev(tok["k_new"]), dev(tok["v_new"]), out)
    assert e.value.code == 7  # QM_E_RANGE: cache full
    g, c, pr, cos, sin, K, V, okv, kvh, prm, keep = _setup(ctx, orc, 1, 8, 16, 501, max_pos=8)
    with pytest.raises(qm.QmError) as e:
        mx.gqa_decode(prm, kvh, dev(tok["q_gate"]), dev(tok["k_new"]), dev(tok["v_new"]), out)
    assert e.value.code == 7  # QM_E_RANGE: past the RoPE table (reference indexes past it)
    assert kvh.seq_len == 8


def test_snapshot_restore_and_host_variant(ctx, orc):
    import torch

    import qora_mixer as qm

    g, c, pr, cos, sin, K, V, okv, kvh, prm, keep = _setup(ctx, orc, 2, 100, 128, 502)
    mx = qm.Mixer(ctx)
    snap = kvh.snapshot()
    tok = I.gqa_token_inputs(g, 2)
    out = torch.empty(2, 16, 256, device="cuda")
    mx.gqa_decode(prm, kvh, dev(tok["q_gate"]), dev(tok["k_new"]), dev(tok["v_new"]), out)
    ctx.sync()
    first = host(out).copy()
    kvh.restore_from(snap)
    assert kvh.seq_len == 100
    oh = np.empty((2, 16, 256), np.float32)
    mx.gqa_decode_host(prm, kvh, np.ascontiguousarray(tok["q_gate"]), np.ascontiguousarray(tok["k_new"]),
                       np.ascontiguousarray(tok["v_new"]), oh)
    np.testing.assert_array_equal(oh, first)
    assert kvh.seq_len == 101
    snap.close()


def test_host_variant_pipelined_batch(ctx, orc):
    """qm_gqa_decode_host on a batch of 16 runs overlapped parts; every
    sequence still matches the oracle and the appended rows are in place."""
    import torch

    import qora_mixer as qm

    B, L = 16, 300
    g, c, pr, cos, sin, K, V, okv, kvh, prm, keep = _setup(ctx, orc, B, L, L + 8, 840)
    mx = qm.Mixer(ctx)
    tok = I.gqa_token_inputs(g, B)
    oh = np.empty((B, 16, 256), np.float32)
    mx.gqa_decode_host(prm, kvh, np.ascontiguousarray(tok["q_gate"]), np.ascontiguousarray(tok["k_new"]),
                       np.ascontiguousarray(tok["v_new"]), oh)
    assert kvh.seq_len == L + 1
    vg = host(V[:, :, L])
    worst = 0.0
    for bi in range(B):
        ref = orc.gqa_decode(c, okv[bi], tok["q_gate"][bi], tok["k_new"][bi], tok["v_new"][bi],
                             pr["q_norm"], pr["k_norm"], cos, sin)
        worst = max(worst, refmath.rel_err(oh[bi], ref))
        np.testing.assert_array_equal(vg[bi], I.f32_to_bf16_bits(tok["v_new"][bi]))
    assert worst <= TOL, worst


def test_host_variant_in_place_on_pinned_buffers(ctx, orc):
    """Page-locked host buffers: qm_gqa_decode_host runs the prep / attention
    / combine launches on them in place and matches the device-buffer call
    bit for bit; switched off, the same call is staged in two parts."""
    import torch

    import qora_mixer as qm

    B, L = 16, 200
    g, c, pr, cos, sin, K, V, okv, kvh, prm, keep = _setup(ctx, orc, B, L, L + 8, 860)
    K2, V2 = K.clone(), V.clone()
    kvd = qm.KvCache(ctx, B, L + 8, K2, V2)
    kvd.seq_len = L
    mx = qm.Mixer(ctx)
    try:
        for t, direct in enumerate((True, False)):
            tok = I.gqa_token_inputs(g, B)
            out = torch.empty(B, 16, 256, device="cuda")
            mx.gqa_decode(prm, kvd, dev(tok["q_gate"]), dev(tok["k_new"]), dev(tok["v_new"]), out)
            ctx.sync()
            ins = [torch.from_numpy(np.ascontiguousarray(tok[k])).pin_memory()
                   for k in ("q_gate", "k_new", "v_new")]
            oh = torch.empty(B, 16, 256).pin_memory()
            ctx.set_host_direct(direct)
            n0, c0 = ctx.launch_count(), ctx.host_calls()
            mx.gqa_decode_host(prm, kvh, *ins, oh)
            n, c1 = ctx.launch_count() - n0, ctx.host_calls()
            ctx.set_host_direct(True)
            assert (c1[0] - c0[0], c1[1] - c0[1]) == ((1, 0) if direct else (0, 1))
            n_dev = 3  # prep, attention, combine
            assert n == (n_dev if direct else 2 * n_dev), n
            if direct:
                np.testing.assert_array_equal(oh.numpy(), host(out))
            else:
                assert refmath.rel_err(oh.numpy(), host(out)) <= TOL
            assert kvh.seq_len == L + 1 + t
            np.testing.assert_array_equal(host(V[:, :, L + t]), host(V2[:, :, L + t]))
            np.testing.assert_array_equal(host(K[:, :, L + t]), host(K2[:, :, L + t]))
    finally:
        ctx.set_host_direct(True)
        kvd.close()


def test_cache_rows_past_seq_len_may_hold_nan(ctx, orc):
    """A caller's cache may hold anything at and past seq_len (the attention
    loads whole 64-position tiles): NaN bit patterns there must not reach the
    output.  L = 100 ends inside a tile."""
    import torch

    import qora_mixer as qm

    B, L, cap = 2, 100, 200
    g, c, pr, cos, sin, K, V, okv, kvh, prm, keep = _setup(ctx, orc, B, L, cap, 870)
    K[:, :, L:] = 0x7FC0  # bf16 quiet NaN
    V[:, :, L:] = 0x7FC0
    tok = I.gqa_token_inputs(g, B)
    out = torch.empty(B, 16, 256, device="cuda")
    qm.Mixer(ctx).gqa_decode(prm, kvh, dev(tok["q_gate"]), dev(tok["k_new"]), dev(tok["v_new"]), out)
    ctx.sync()
    o = host(out)
    assert np.isfinite(o).all()
    for bi in range(B):
        ref = orc.gqa_decode(c, okv[bi], tok["q_gate"][bi], tok["k_new"][bi], tok["v_new"][bi],
                             pr["q_norm"], pr["k_norm"], cos, sin)
        assert refmath.rel_err(o[bi], ref) <= TOL


def test_host_staged_in_parts(ctx, orc):
    """qm_ctx_set_host_parts: the staged qm_gqa_decode_host cut into 1, 3 and 8
    parts matches the device-buffer call within 1e-3 and appends the same V
    rows bit for bit and K rows within one bf16 rounding (a part of two
    sequences takes the one-launch kernel, the whole batch the split-KV one)."""
    import torch

    import qora_mixer as qm

    B, L = 16, 150
    g, c, pr, cos, sin, K, V, okv, kvh, prm, keep = _setup(ctx, orc, B, L, L + 8, 861)
    K2, V2 = K.clone(), V.clone()
    kvd = qm.KvCache(ctx, B, L + 8, K2, V2)
    kvd.seq_len = L
    mx = qm.Mixer(ctx)
    try:
        for t, parts in enumerate((1, 3, 8)):
            tok = I.gqa_token_inputs(g, B)
            out = torch.empty(B, 16, 256, device="cuda")
            mx.gqa_decode(prm, kvd, dev(tok["q_gate"]), dev(tok["k_new"]), dev(tok["v_new"]), out)
            ctx.sync()
            ins = [torch.from_numpy(np.ascontiguousarray(tok[k])).pin_memory()
                   for k in ("q_gate", "k_new", "v_new")]
            oh = torch.empty(B, 16, 256).pin_memory()
            ctx.set_host_direct(False)
            ctx.set_host_parts(0, parts)
            c0 = ctx.host_calls()
            mx.gqa_decode_host(prm, kvh, *ins, oh)
            assert ctx.host_calls()[1] - c0[1] == 1  # staged
            assert refmath.rel_err(oh.numpy(), host(out)) <= TOL
            assert kvh.seq_len == L + 1 + t
            np.testing.assert_array_equal(host(V[:, :, L + t]), host(V2[:, :, L + t]))
            kh = I.bf16_bits_to_f32(host(K[:, :, L + t]))
            kd = I.bf16_bits_to_f32(host(K2[:, :, L + t]))
            assert np.all(np.abs(kh - kd) <= np.abs(kd) * 2.0 ** -8 + 1e-4)
    finally:
        ctx.set_host_parts(0, 0)
        ctx.set_host_direct(True)
        kvd.close()
