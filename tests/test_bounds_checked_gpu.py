"""The checked build (libqora_mixer_checked.so, -DQM_CHECK_BOUNDS): the
prefill and GEMM kernels compare every guarded buffer offset with the
buffer's extent and, instead of an out-of-range access, skip it and set the
error word.  This stands in for compute-sanitizer, which is closed on this
pool.  Small cases of each kernel run in a child process that loads the
checked library; they must match the CPU restatement and leave the error
word clean (qm_sync would return QM_E_RANGE otherwise).
"""
import os
import subprocess
import sys

import pytest

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
CHECKED = os.path.join(ROOT, "qora-llm-4b_b200", "libqora_mixer_checked.so")

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

assert qm.lib().qm_build_flags() & 1, "not the checked build"
ctx = qm.Ctx(0, stream=torch.cuda.current_stream())
mx = qm.Mixer(ctx)
c = orc.cfg_4b()

# GQA causal prefill: two query tiles, the second partial
B, T = 2, 200
g = I.rng(1600)
pr = I.gqa_layer_params(g, T + 1)
cos, sin = qm.rope_table(1.0e7, 64, T + 1)
qg = I.f32_to_bf16_bits(g.standard_normal((B, T, 16, 512), dtype=np.float32))
kk = I.f32_to_bf16_bits(g.standard_normal((B, T, 4, 256), dtype=np.float32))
vv = I.f32_to_bf16_bits(g.standard_normal((B, T, 4, 256), dtype=np.float32))
kv = qm.KvCache(ctx, B, T)
keep = [dev(pr["q_norm"]), dev(pr["k_norm"]), dev(cos), dev(sin)]
out = torch.empty(B, T, 16, 256, device="cuda")
mx.gqa_prefill(qm.gqa_params(*keep), kv, T, dev(qg), dev(kk), dev(vv), out)
ctx.sync()
for b in range(B):
    ref = orc.gqa_prefill_rows(c, qg[b].reshape(T, -1), kk[b].reshape(T, -1), vv[b].reshape(T, -1),
                               pr["q_norm"], pr["k_norm"], cos, sin, np.arange(T))
    assert refmath.rel_err(host(out)[b], ref) <= 2e-2
kv.close()

# DeltaNet chunked prefill with the gate: three chunks, the last partial
B, T = 2, 130
g = I.rng(1601)
p = I.dn_layer_params(g)
keep2 = [dev(p["conv_w"]), dev(p["a_log"]), dev(p["dt_bias"]), dev(p["norm_gamma"])]
qkv = I.f32_to_bf16_bits(g.standard_normal((B, T, 8192), dtype=np.float32))
a = g.standard_normal((B, T, 32), dtype=np.float32)
bb = g.standard_normal((B, T, 32), dtype=np.float32)
z = g.standard_normal((B, T, 4096), dtype=np.float32)
st = qm.DnState(ctx, B)
y = torch.empty(B, T, 32, 128, device="cuda")
o = torch.empty(B, T, 4096, device="cuda")
mx.dn_prefill(qm.dn_params(*keep2), st, T, dev(qkv), dev(a), dev(bb), y, dev(z), o)
ctx.sync()
for b in range(B):
    ost = orc.DnState(c)
    ref = orc.dn_prefill(c, ost, qkv[b], a[b], bb[b], p["conv_w"], p["a_log"], p["dt_bias"])
    assert refmath.rel_err(host(y)[b], ref) <= 2e-2
    s_g, _ = st.read(b)
    assert refmath.rel_err(s_g, ost.s) <= 2e-2
st.close()

# tensor-core GEMM: Q4 with split K (few tiles), and F16 rows
gg = np.random.default_rng(1602)
for kind, (k, n, T) in (("q4", (1024, 256, 100)), ("f16rows", (512, 320, 64))):
    x = I.f32_to_bf16_bits(gg.standard_normal((T, k)).astype(np.float32))
    if kind == "q4":
        w = (gg.standard_normal((k, n)) * 0.02).astype(np.float32)
        pk, sc = orc.quantize_q4(w)
        wk = (dev(pk), dev(sc))
        wt = qm.weight_q4(*wk)
        wref = orc.dequantize_q4(pk, sc).astype(np.float64)
    else:
        e16 = (gg.standard_normal((n, k)) * 0.02).astype(np.float16)
        wk = (dev(e16.view(np.int16)),)
        wt = qm.weight_f16_rows(*wk)
        wref = e16.astype(np.float64).T
    yg = torch.empty(T, n, device="cuda")
    mx.gemm(wt, dev(x), yg)
    ctx.sync()
    ref = I.bf16_bits_to_f32(x).astype(np.float64) @ wref
    assert refmath.rel_err(host(yg), ref) <= 2e-2, kind
ctx.close()
print("checked build ok")
'''


def test_normal_build_has_no_checks():
    import qora_mixer as qm

    if os.environ.get("QORA_MIXER_LIB"):
        pytest.skip("QORA_MIXER_LIB selects another build")
    assert qm.lib().qm_build_flags() == 0


def test_prefill_and_gemm_clean_under_bounds_checks():
    assert os.path.exists(CHECKED), "build libqora_mixer_checked.so first (make -C qora-llm-4b_b200)"
    env = dict(os.environ, QORA_MIXER_LIB=CHECKED)
    r = subprocess.run([sys.executable, "-c", "ROOT = %r\n" % ROOT + SCRIPT], env=env, capture_output=True,
                       text=True, timeout=600)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-4000:]
    assert "checked build ok" in r.stdout
