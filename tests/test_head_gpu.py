"""The decode loop's tail on the GPU against the CPU restatement: lm_head over
the tied embedding rows (src/gemv.rs:662-711), the logit penalties
(src/generate.rs:58-83 in the order of 185-196) and sample_token_top_k
(src/generate.rs:334-384) with the caller's draw r.

lm_head: max|gpu - cpu| / RMS(cpu) <= 5e-5 (f32 sums of 2560 products in
another order).  Penalties: bit-exact.  Sampling: the same token, except
where the oracle reports the draw or the top-p cut within 1e-5 (relative)
of a cumulative boundary: exp on the device and the host's expf differ by
one ulp for ~0.06 % of arguments."""
import numpy as np
import pytest

import refmath
from gpu_util import dev, host, make_ctx

pytestmark = pytest.mark.gpu
TOL = 5e-5
MARGIN = 1e-5


@pytest.fixture(scope="module")
def ctx():
    c = make_ctx()
    yield c
    c.close()


@pytest.mark.parametrize("vocab,hidden", [(20000, 2560), (999, 256), (5, 64), (4097, 32)])
@pytest.mark.parametrize("batch", [1, 3])
def test_lm_head_q4_rows(ctx, orc, vocab, hidden, batch):
    import torch

    import qora_mixer as qm

    g = np.random.default_rng(vocab + hidden + batch)
    e = (g.standard_normal((vocab, hidden)) * 0.02).astype(np.float32)
    e[0] = 0.0                                  # an all-zero row (every group skipped)
    e[min(1, vocab - 1), :32] = 0.0             # a zero group
    packed, scales = orc.quantize_q4(e)
    x = g.standard_normal((batch, hidden)).astype(np.float32)
    y = torch.full((batch, vocab), float("nan"), device="cuda")
    qm.Mixer(ctx).gemv(qm.weight_q4_rows(dev(packed), dev(scales)), dev(x), y)
    ctx.sync()
    yg = host(y)
    for b in range(batch):
        ref = orc.lm_head_q4(x[b], packed, scales)
        assert refmath.rel_err(yg[b], ref) <= TOL, (b, refmath.rel_err(yg[b], ref))
    assert np.all(yg[:, 0] == 0.0)


@pytest.mark.parametrize("vocab,hidden", [(7000, 2560), (33, 8)])
@pytest.mark.parametrize("batch", [1, 2, 3])
def test_lm_head_f16_rows(ctx, orc, vocab, hidden, batch):
    import torch

    import qora_mixer as qm

    g = np.random.default_rng(3 * vocab + hidden + batch)
    e16 = (g.standard_normal((vocab, hidden)) * 0.02).astype(np.float16).view(np.uint16)
    x = g.standard_normal((batch, hidden)).astype(np.float32)
    y = torch.full((batch, vocab), float("nan"), device="cuda")
    qm.Mixer(ctx).gemv(qm.weight_f16_rows(dev(e16)), dev(x), y)
    ctx.sync()
    yg = host(y)
    for b in range(batch):
        assert refmath.rel_err(yg[b], orc.lm_head_f16(x[b], e16)) <= TOL


def _histories(g, batch, vocab, lens, stride):
    toks = np.full((batch, stride), -1, np.int32)
    for b, n in enumerate(lens):
        h = g.integers(0, min(vocab, 50), n).astype(np.int32)  # a small id range: many repeats
        if n > 3:
            h[1] = vocab + 5  # out of range: ignored
            h[2] = -3
        toks[b, :n] = h
    return toks


@pytest.mark.parametrize("rep,pres,ban", [(1.3, 1.5, 7), (1.0, 1.5, -1), (2.0, 0.0, -1), (1.0, 0.0, 3)])
def test_penalties_bit_exact(ctx, orc, rep, pres, ban):
    import torch

    import qora_mixer as qm

    g = np.random.default_rng(int(rep * 10 + pres * 100 + ban + 50))
    vocab, lens, stride = 5000, [0, 5, 100, 64], 128
    batch = len(lens)
    logits = (g.standard_normal((batch, vocab)) * 2).astype(np.float32)
    toks = _histories(g, batch, vocab, lens, stride)
    ld = dev(logits)
    qm.Mixer(ctx).penalize(ld, dev(toks), dev(np.array(lens, np.int32)), rep, pres, ban)
    ctx.sync()
    got = host(ld)
    for b in range(batch):
        ref = orc.penalize(logits[b], toks[b, :lens[b]], rep, pres, ban)
        np.testing.assert_array_equal(got[b], ref)


def test_penalties_history_longer_than_stride_is_clamped(ctx, orc):
    """lens[b] > stride reads only the row (the first stride tokens)."""
    import torch

    import qora_mixer as qm

    g = np.random.default_rng(9)
    vocab, stride = 300, 16
    logits = (g.standard_normal((1, vocab))).astype(np.float32)
    toks = g.integers(0, vocab, (1, stride)).astype(np.int32)
    ld = dev(logits)
    qm.Mixer(ctx).penalize(ld, dev(toks), dev(np.array([1000], np.int32)), 1.5, 0.5, -1)
    ctx.sync()
    np.testing.assert_array_equal(host(ld)[0], orc.penalize(logits[0], toks[0], 1.5, 0.5, -1))


def _sample_check(ctx, orc, logits, temperature, top_p, top_k, seed):
    import torch

    import qora_mixer as qm

    batch = logits.shape[0]
    rng = orc.Rng(seed)
    r = np.array([rng.next_f32() for _ in range(batch)], np.float32)
    ids = torch.full((batch,), -1, dtype=torch.int32, device="cuda")
    qm.Mixer(ctx).sample(dev(logits), temperature, top_p, top_k, dev(r), ids)
    ctx.sync()
    got = host(ids)
    checked = 0
    for b in range(batch):
        tok, margin = orc.sample_top_k(logits[b], temperature, top_p, top_k, float(r[b]))
        if margin > MARGIN:
            assert got[b] == tok, (b, got[b], tok, margin)
            checked += 1
    return checked


def test_sample_greedy_first_max(ctx, orc):
    g = np.random.default_rng(1)
    logits = g.standard_normal((4, 248320)).astype(np.float32)
    logits[1, [5, 77777]] = 50.0   # a tie: the first index wins
    logits[2, :] = -np.inf         # nothing above -inf: token 0
    logits[3, 248319] = 60.0       # the last index
    assert _sample_check(ctx, orc, logits, 0.0, 0.95, 20, 3) == 4


@pytest.mark.parametrize("temperature,top_p,top_k", [(0.7, 0.95, 20), (1.0, 0.8, 40), (1.3, 1.0, 1),
                                                     (0.5, 0.5, 4096), (1.0, 0.95, 1000)])
def test_sample_top_k_top_p_full_vocab(ctx, orc, temperature, top_p, top_k):
    g = np.random.default_rng(int(temperature * 100) + top_k)
    logits = (g.standard_normal((8, 248320)) * 3).astype(np.float32)
    logits[0, 100:110] = -np.inf
    assert _sample_check(ctx, orc, logits, temperature, top_p, top_k, 77 + top_k) >= 7


def test_sample_ties_straddling_the_cut(ctx, orc):
    """Logits on a coarse grid: many equal values at the k-th place; the lowest
    indices among them are taken (the reference's stable sort)."""
    g = np.random.default_rng(5)
    logits = (np.round(g.standard_normal((6, 50000)) * 2) / 2).astype(np.float32)
    n = 0
    for top_k in (20, 300, 4096):
        n += _sample_check(ctx, orc, logits, 1.0, 1.0, top_k, 11 + top_k)
    assert n >= 16


def test_sample_whole_small_vocab_and_limits(ctx, orc):
    import torch

    import qora_mixer as qm

    g = np.random.default_rng(8)
    logits = (g.standard_normal((3, 3000)) * 2).astype(np.float32)
    assert _sample_check(ctx, orc, logits, 0.9, 0.9, 0, 21) >= 2  # top_k 0: the whole vocabulary
    tiny = (g.standard_normal((2, 5)) * 2).astype(np.float32)  # fewer tokens than CTAs per sequence
    assert _sample_check(ctx, orc, tiny, 0.0, 0.9, 3, 5) == 2
    assert _sample_check(ctx, orc, tiny, 1.0, 0.9, 3, 6) >= 1
    big = torch.zeros(1, 10000, device="cuda")
    ids = torch.zeros(1, dtype=torch.int32, device="cuda")
    r = torch.zeros(1, device="cuda")
    with pytest.raises(qm.QmError) as e:
        qm.Mixer(ctx).sample(big, 1.0, 0.9, 0, r, ids)  # 10000 candidates
    assert e.value.code == 9  # QM_E_UNSUPPORTED
    with pytest.raises(qm.QmError) as e:
        qm.Mixer(ctx).sample(big, 1.0, 0.9, 5000, r, ids)
    assert e.value.code == 9


def test_decode_tail_chain(ctx, orc):
    """final x -> lm_head (Q4 rows) -> penalties -> sampling on one stream,
    against the restatement's chain, for 4 sequences."""
    import torch

    import qora_mixer as qm

    g = np.random.default_rng(12)
    vocab, hidden, batch = 6000, 2560, 4
    e = (g.standard_normal((vocab, hidden)) * 0.05).astype(np.float32)
    packed, scales = orc.quantize_q4(e)
    x = g.standard_normal((batch, hidden)).astype(np.float32)
    lens = [0, 10, 70, 3]
    toks = _histories(g, batch, vocab, lens, 80)
    logits = torch.empty(batch, vocab, device="cuda")
    ids = torch.full((batch,), -1, dtype=torch.int32, device="cuda")
    rng = orc.Rng(99)
    r = np.array([rng.next_f32() for _ in range(batch)], np.float32)
    mx = qm.Mixer(ctx)
    mx.gemv(qm.weight_q4_rows(dev(packed), dev(scales)), dev(x), logits)
    mx.penalize(logits, dev(toks), dev(np.array(lens, np.int32)), 1.2, 1.5, -1)
    mx.sample(logits, 0.8, 0.95, 20, dev(r), ids)
    ctx.sync()
    got_logits, got_ids = host(logits), host(ids)
    for b in range(batch):
        ref = orc.penalize(orc.lm_head_q4(x[b], packed, scales), toks[b, :lens[b]], 1.2, 1.5, -1)
        assert refmath.rel_err(got_logits[b], ref) <= TOL
        # sample from the device's logits: the chain's token given its own logits
        tok, margin = orc.sample_top_k(got_logits[b], 0.8, 0.95, 20, float(r[b]))
        if margin > MARGIN:
            assert got_ids[b] == tok
