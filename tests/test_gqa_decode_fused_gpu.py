"""GQA decode, one-launch path for small batches (gqa_fused_kernel) against
the CPU restatement of src/gemv.rs:927-1011, and its hand-over with the
three-launch path.

Calls whose clusters (16 CTAs per sequence and KV head) fit in one wave and
whose context is at most 16384 positions take the fused kernel; the rest
take prep + split-KV attention + combine.  QORA_MIXER_GQA_FUSED=0 / =1 force
one path or the other (read once per process, so those cases run in a
child process).  Consecutive calls are issued without a host
synchronisation between them: each call lets the next one start early, and
the next call must still see the row its predecessor appended.
Tolerance: max|gpu - cpu| / RMS(cpu) <= 1e-3.
"""
import os
import subprocess
import sys

import numpy as np
import pytest

import refmath
from gpu_util import dev, host, make_ctx
from qora_mixer import inputs as I

pytestmark = pytest.mark.gpu
TOL = 1e-3
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.fixture(scope="module")
def ctx():
    c = make_ctx()
    yield c
    c.close()


def _setup(ctx, orc, B, L, cap, seed):
    import torch

    import qora_mixer as qm

    g = I.rng(seed)
    pr = I.gqa_layer_params(g, cap + 1)
    cos, sin = qm.rope_table(1.0e7, 64, cap + 1)
    K = torch.zeros(B, 4, cap, 256, dtype=torch.int16, device="cuda")
    V = torch.zeros_like(K)
    c = orc.cfg_4b()
    kb, vb = I.gqa_cache_bf16(g, B, L)
    K[:, :, :L] = dev(kb)
    V[:, :, :L] = dev(vb)
    okv = []
    for bi in range(B):
        kv = orc.KvCache(c, cap + 1)
        kv.k[:L] = I.bf16_bits_to_f32(kb[bi]).transpose(1, 0, 2)
        kv.v[:L] = I.bf16_bits_to_f32(vb[bi]).transpose(1, 0, 2)
        kv.seq_len[0] = L
        okv.append(kv)
    kvh = qm.KvCache(ctx, B, cap, K, V)
    kvh.seq_len = L
    keep = [dev(pr["q_norm"]), dev(pr["k_norm"]), dev(cos), dev(sin)]
    return g, c, pr, cos, sin, K, V, okv, kvh, qm.gqa_params(*keep), keep


def _back_to_back(ctx, orc, B, L, steps, seed, launches=None):
    """`steps` decode calls on one cache with no synchronisation between them,
    then every step against the restatement (fed the rows the GPU appended)."""
    import torch

    import qora_mixer as qm

    cap = L + steps + 8
    g, c, pr, cos, sin, K, V, okv, kvh, prm, keep = _setup(ctx, orc, B, L, cap, seed)
    mx = qm.Mixer(ctx)
    toks = [I.gqa_token_inputs(g, B) for _ in range(steps)]
    ins = [[dev(t[k]) for k in ("q_gate", "k_new", "v_new")] for t in toks]
    outs = [torch.empty(B, 16, 256, device="cuda") for _ in range(steps)]
    ctx.sync()
    n0 = ctx.launch_count()
    for s in range(steps):
        mx.gqa_decode(prm, kvh, *ins[s], outs[s])
    n = ctx.launch_count() - n0
    ctx.sync()
    assert kvh.seq_len == L + steps
    if launches is not None:
        assert n == launches, n
    worst = 0.0
    for s in range(steps):
        pos = L + s
        og = host(outs[s])
        kg, vg = host(K[:, :, pos]), host(V[:, :, pos])
        for bi in range(B):
            tk = toks[s]
            ref = orc.gqa_decode(c, okv[bi], tk["q_gate"][bi], tk["k_new"][bi], tk["v_new"][bi],
                                 pr["q_norm"], pr["k_norm"], cos, sin)
            worst = max(worst, refmath.rel_err(og[bi], ref))
            ko = okv[bi].k[pos]
            kgf = I.bf16_bits_to_f32(kg[bi])
            assert np.all(np.abs(kgf - ko) <= np.abs(ko) * 2.0 ** -8 + 1e-4)
            np.testing.assert_array_equal(vg[bi], I.f32_to_bf16_bits(tk["v_new"][bi]))
            okv[bi].k[pos] = kgf
            okv[bi].v[pos] = I.bf16_bits_to_f32(vg[bi])
    assert worst <= TOL, f"rel err {worst:.3e}"


def test_config1_one_launch_per_call(ctx, orc):
    """Workload 1's shape (batch 1, 4096 cached positions) takes the fused
    kernel: one launch per call, eight calls back to back."""
    _back_to_back(ctx, orc, B=1, L=4096, steps=8, seed=0x51A0 + 11, launches=8)


@pytest.mark.parametrize("B,L", [(1, 1), (2, 130), (1, 1000)])
def test_back_to_back_short(ctx, orc, B, L):
    """Position L-1 of each call is the previous call's append; L = 1 puts it
    in the first tile, 130 in a partial third tile."""
    _back_to_back(ctx, orc, B=B, L=L, steps=6, seed=900 + B + L)


def test_hand_over_between_paths(ctx, orc):
    """Contexts 16383 .. 16386: the first two calls are fused (256 tiles),
    the last two take the three-launch path (257 tiles), whose attention
    kernel must not load position L-1 before the fused call that wrote it
    has finished."""
    _back_to_back(ctx, orc, B=1, L=16383, steps=4, seed=950, launches=2 * 1 + 2 * 3)


SCRIPT = r'''
import sys
import numpy as np
import torch
sys.path[:0] = [ROOT, ROOT + "/qora-llm-4b_b200", ROOT + "/tests"]
import qora_mixer as qm
from qora_mixer import inputs as I
from oracle import oracle as orc
import refmath
from gpu_util import dev, host

ctx = qm.Ctx(0, stream=torch.cuda.current_stream())
mx = qm.Mixer(ctx)
c = orc.cfg_4b()
for B, L, per_call in CASES:
    g = I.rng(970 + B + L)
    cap = L + 4
    pr = I.gqa_layer_params(g, cap + 1)
    cos, sin = qm.rope_table(1.0e7, 64, cap + 1)
    kb, vb = I.gqa_cache_bf16(g, B, L)
    K = torch.zeros(B, 4, cap, 256, dtype=torch.int16, device="cuda")
    V = torch.zeros_like(K)
    K[:, :, :L] = dev(kb)
    V[:, :, :L] = dev(vb)
    kvh = qm.KvCache(ctx, B, cap, K, V)
    kvh.seq_len = L
    keep = [dev(pr["q_norm"]), dev(pr["k_norm"]), dev(cos), dev(sin)]
    tok = I.gqa_token_inputs(g, B)
    out = torch.empty(B, 16, 256, device="cuda")
    n0 = ctx.launch_count()
    mx.gqa_decode(qm.gqa_params(*keep), kvh, dev(tok["q_gate"]), dev(tok["k_new"]), dev(tok["v_new"]), out)
    assert ctx.launch_count() - n0 == per_call, (B, L, ctx.launch_count() - n0)
    ctx.sync()
    o = host(out)
    for bi in range(B):
        okv = orc.KvCache(c, cap + 1)
        okv.k[:L] = I.bf16_bits_to_f32(kb[bi]).transpose(1, 0, 2)
        okv.v[:L] = I.bf16_bits_to_f32(vb[bi]).transpose(1, 0, 2)
        okv.seq_len[0] = L
        ref = orc.gqa_decode(c, okv, tok["q_gate"][bi], tok["k_new"][bi], tok["v_new"][bi],
                             pr["q_norm"], pr["k_norm"], cos, sin)
        e = refmath.rel_err(o[bi], ref)
        assert e <= 1e-3, (B, L, e)
    kvh.close()
    del K, V
ctx.close()
print("forced path ok")
'''


@pytest.mark.parametrize("mode,cases", [
    ("1", [(1, 32768, 1), (2, 20000, 1)]),   # fused past the automatic context limit
    ("0", [(1, 4096, 3), (2, 64, 3)]),       # three launches at batch 1 and 2
])
def test_forced_path(mode, cases):
    env = dict(os.environ, QORA_MIXER_GQA_FUSED=mode)
    code = "ROOT = %r\nCASES = %r\n" % (ROOT, cases) + SCRIPT
    r = subprocess.run([sys.executable, "-c", code], env=env, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-4000:]
    assert "forced path ok" in r.stdout
