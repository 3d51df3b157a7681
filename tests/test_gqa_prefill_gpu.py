"""GQA causal prefill on the GPU vs the CPU restatement of src/gemv.rs:1364-1444.

tensor-core prefill tolerance (north_star): max|gpu - cpu| / RMS(cpu) <= 2e-2
(the attention runs on fp16 operands; see gqa_prefill.cu).  The KV cache the prefill writes is checked position by position:
K (after QK-norm and RoPE) within one bf16 rounding of the oracle's f32 K,
V bit-exact (a copy of the bf16 input).
"""
import ctypes as C
import os

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


@pytest.mark.parametrize("fp16,a_tmem", [(0, 0), (1, 0), (1, 1), (0, 1)])
def test_tcgen05_descriptor_selftest(fp16, a_tmem):
    """Q.K^T (K-major operands via TMA, 128B swizzle; or Q copied to TMEM and
    read from there, as the prefill kernel does) and P.V (P written by
    threads, V MN-major) on one tile, against float64 products of the same
    bf16 (or fp16) values."""
    import torch

    import qora_mixer as qm

    qm.lib()  # the self-test library links against the product library
    L = C.CDLL(os.path.join(qm.PKG_DIR, "libqora_selftest.so"))
    fn = L.qm_selftest_umma
    fn.argtypes = [C.c_void_p] * 6 + [C.c_int]
    fn.restype = C.c_int
    dt = torch.float16 if fp16 else torch.bfloat16
    g = torch.Generator(device="cuda").manual_seed(7)
    a = torch.randn(128, 256, device="cuda", generator=g).to(dt)
    b = torch.randn(64, 256, device="cuda", generator=g).to(dt)
    v = torch.randn(64, 256, device="cuda", generator=g).to(dt)
    p = torch.rand(128, 64, device="cuda", generator=g).to(dt)
    d1 = torch.zeros(128, 64, device="cuda")
    d2 = torch.zeros(128, 256, device="cuda")
    torch.cuda.synchronize()
    rc = fn(a.data_ptr(), b.data_ptr(), v.data_ptr(), p.data_ptr(), d1.data_ptr(), d2.data_ptr(),
            fp16 | (a_tmem << 1))
    assert rc == 0
    r1 = a.double() @ b.double().T
    r2 = p.double() @ v.double()
    assert refmath.rel_err(d1.cpu().numpy(), r1.cpu().numpy()) < 1e-5
    assert refmath.rel_err(d2.cpu().numpy(), r2.cpu().numpy()) < 1e-5


def _run_prefill(ctx, B, T, seed, cap=None):
    import torch

    import qora_mixer as qm

    cap = cap or T
    g = I.rng(seed)
    pr = I.gqa_layer_params(g, cap + 1)
    cos, sin = qm.rope_table(1.0e7, 64, cap + 1)
    qg = I.f32_to_bf16_bits(g.standard_normal((B, T, 16, 512), dtype=np.float32))
    kk = I.f32_to_bf16_bits(g.standard_normal((B, T, 4, 256), dtype=np.float32))
    vv = I.f32_to_bf16_bits(g.standard_normal((B, T, 4, 256), dtype=np.float32))
    keep = [dev(pr["q_norm"]), dev(pr["k_norm"]), dev(cos), dev(sin)]
    prm = qm.gqa_params(*keep)
    K = torch.zeros(B, 4, cap, 256, dtype=torch.int16, device="cuda")
    V = torch.zeros_like(K)
    kv = qm.KvCache(ctx, B, cap, K, V)
    out = torch.full((B, T, 16, 256), float("nan"), device="cuda")
    qm.Mixer(ctx).gqa_prefill(prm, kv, T, dev(qg), dev(kk), dev(vv), out)
    ctx.sync()
    kv.K, kv.V = K, V
    return g, pr, cos, sin, qg, kk, vv, kv, out


@pytest.mark.parametrize("B,T", [(1, 1), (1, 64), (1, 128), (1, 129), (2, 200), (1, 391)])
def test_prefill_small_all_rows(ctx, orc, B, T):
    """Every row of short prompts: single tile, partial tiles, several query tiles."""
    c = orc.cfg_4b()
    g, pr, cos, sin, qg, kk, vv, kv, out = _run_prefill(ctx, B, T, 700 + T)
    og = host(out)
    for b in range(B):
        rows = np.arange(T)
        ref, kc, vc = orc.gqa_prefill_rows(c, qg[b].reshape(T, -1), kk[b].reshape(T, -1),
                                           vv[b].reshape(T, -1), pr["q_norm"], pr["k_norm"], cos, sin,
                                           rows, want_cache=True)
        e = refmath.rel_err(og[b], ref)
        assert e <= TOL, f"b={b} rel err {e:.3e}"
        print(f"prefill B={B} T={T} b={b}: rel err {e:.3e}")
    assert kv.seq_len == T


def test_prefill_writes_kv_cache(ctx, orc):
    import torch

    c = orc.cfg_4b()
    B, T, cap = 2, 300, 320
    g, pr, cos, sin, qg, kk, vv, kv, out = _run_prefill(ctx, B, T, 710, cap=cap)
    Kh = host(kv.K)
    Vh = host(kv.V)
    for b in range(B):
        _, kc, vc = orc.gqa_prefill_rows(c, qg[b].reshape(T, -1), kk[b].reshape(T, -1),
                                         vv[b].reshape(T, -1), pr["q_norm"], pr["k_norm"], cos, sin,
                                         np.array([0]), want_cache=True)
        kg = I.bf16_bits_to_f32(Kh[b, :, :T]).transpose(1, 0, 2)
        assert np.all(np.abs(kg - kc) <= np.abs(kc) * 2.0 ** -8 + 1e-4)
        np.testing.assert_array_equal(Vh[b, :, :T].transpose(1, 0, 2), vv[b])


def test_prefill_then_decode_continues(ctx, orc):
    """A decode step after a prefill attends over the prefilled cache."""
    import torch

    import qora_mixer as qm

    c = orc.cfg_4b()
    B, T, cap = 1, 150, 160
    g, pr, cos, sin, qg, kk, vv, kv, out = _run_prefill(ctx, B, T, 720, cap=cap)
    keep = [dev(pr["q_norm"]), dev(pr["k_norm"]), dev(cos), dev(sin)]
    prm = qm.gqa_params(*keep)
    tok = I.gqa_token_inputs(g, 1)
    o = torch.empty(1, 16, 256, device="cuda")
    qm.Mixer(ctx).gqa_decode(prm, kv, dev(tok["q_gate"]), dev(tok["k_new"]), dev(tok["v_new"]), o)
    ctx.sync()
    # oracle: cache = the GPU's bf16 cache contents widened (as decode tests do)
    Kh = I.bf16_bits_to_f32(host(kv.K)[0, :, :T]).transpose(1, 0, 2)
    Vh = I.bf16_bits_to_f32(host(kv.V)[0, :, :T]).transpose(1, 0, 2)
    okv = orc.KvCache(c, cap + 1, Kh.reshape(T, -1), Vh.reshape(T, -1))
    ref = orc.gqa_decode(c, okv, tok["q_gate"][0], tok["k_new"][0], tok["v_new"][0], pr["q_norm"],
                         pr["k_norm"], cos, sin)
    assert refmath.rel_err(host(o)[0], ref) <= 1e-3
    assert kv.seq_len == T + 1


def test_config3_prefill_sampled_rows(ctx, orc):
    """Config 3: batch 4 x 32768 tokens.  Inputs drawn on the device (torch's
    Philox generator); the oracle checks sampled query rows of every sequence
    (the first 64, the last 64 and 256 seeded random rows) over all 16 heads,
    plus the whole KV cache written for later decode."""
    import torch

    import qora_mixer as qm

    c = orc.cfg_4b()
    B, T = 4, 32768
    g = I.rng(0x51A0 + 3)
    pr = I.gqa_layer_params(g, T + 1)
    cos, sin = qm.rope_table(1.0e7, 64, T + 1)
    qg = I.device_normal_bf16((B, T, 16, 512), 0x51A3 * 10 + 1)
    kk = I.device_normal_bf16((B, T, 4, 256), 0x51A3 * 10 + 2)
    vv = I.device_normal_bf16((B, T, 4, 256), 0x51A3 * 10 + 3)
    keep = [dev(pr["q_norm"]), dev(pr["k_norm"]), dev(cos), dev(sin)]
    prm = qm.gqa_params(*keep)
    K = torch.zeros(B, 4, T, 256, dtype=torch.int16, device="cuda")
    V = torch.zeros_like(K)
    kv = qm.KvCache(ctx, B, T, K, V)
    out = torch.empty(B, T, 16, 256, device="cuda")
    qm.Mixer(ctx).gqa_prefill(prm, kv, T, qg.view(torch.int16), kk.view(torch.int16),
                              vv.view(torch.int16), out)
    ctx.sync()
    worst = 0.0
    for b in range(B):
        rows = np.concatenate([np.arange(64), np.arange(T - 64, T),
                               np.sort(g.choice(np.arange(64, T - 64), 256, replace=False))])
        qh = np.zeros((T, 16 * 512), np.uint16)
        qh[rows] = host(qg[b].view(torch.int16)[torch.from_numpy(rows).cuda()]).reshape(len(rows), -1)
        kh = host(kk[b].view(torch.int16)).reshape(T, -1)
        vh = host(vv[b].view(torch.int16)).reshape(T, -1)
        ref, kc, vc = orc.gqa_prefill_rows(c, qh, kh, vh, pr["q_norm"], pr["k_norm"], cos, sin, rows,
                                           want_cache=True)
        og = host(out[b][torch.from_numpy(rows).cuda()])
        e = refmath.rel_err(og, ref)
        worst = max(worst, e)
        assert e <= TOL, f"b={b} rel err {e:.3e}"
        # the cache written for later decode, all 32768 positions
        kg = I.bf16_bits_to_f32(host(K[b])).transpose(1, 0, 2)
        assert np.all(np.abs(kg - kc) <= np.abs(kc) * 2.0 ** -8 + 1e-4)
    assert kv.seq_len == T
    print(f"config 3 prefill: worst rel err over sampled rows {worst:.3e}")
