"""The .qor4b file (src/save.rs): the reader against files the writer makes
(every record byte for byte, the reference's rejections: bad magic, an
unsupported version, an unknown weight format; plus truncation and records
that do not fit their shapes), and on the GPU the path file -> device ->
projections -> mixers -> lm_head against the CPU restatement."""
import numpy as np
import pytest

from qora_mixer import qor4b as Q


def _q4(orc, g, k, n, scale=0.02):
    packed, scales = orc.quantize_q4((g.standard_normal((k, n)) * scale).astype(np.float32))
    return Q.Weight("q4", k, n, packed, scales)


def _f16(g, k, n):
    return Q.Weight("f16", k, n, (g.standard_normal((k, n)) * 0.02).astype(np.float16).view(np.uint16))


def _vec16(g, n, mean=0.0):
    return (mean + g.standard_normal(n) * 0.05).astype(np.float16).view(np.uint16)


def _model(orc, g, layer_types, hidden, qkv, vdim, nv, q_out, kv_out, head_dim, vocab, max_pos, kind="q4"):
    cfg = {"vocab_size": vocab, "hidden_size": hidden, "num_layers": len(layer_types), "num_attn_heads": 16,
           "num_kv_heads": 4, "attn_head_dim": head_dim, "num_qk_heads": 16, "num_v_heads": nv,
           "deltanet_head_dim": 128, "conv_kernel_size": 4, "intermediate_size": 64, "rope_theta": 1.0e7,
           "partial_rotary_factor": 0.25, "rms_norm_eps": 1e-6, "eos_token_id": 7,
           "tie_word_embeddings": True, "has_vision": False}
    W = (lambda k, n: _q4(orc, g, k, n)) if kind == "q4" else (lambda k, n: _f16(g, k, n))
    layers = []
    for lt in layer_types:
        mlp = {"gate_proj": W(32, 64), "up_proj": W(32, 64), "down_proj": W(64, 32),
               "input_norm": _vec16(g, hidden), "post_attn_norm": _vec16(g, hidden)}
        if lt == 0:
            layers.append({"in_proj_qkv": W(hidden, qkv), "in_proj_a": W(hidden, nv), "in_proj_b": W(hidden, nv),
                           "in_proj_z": W(hidden, vdim), "out_proj": W(vdim, hidden),
                           "conv1d_weight": (g.standard_normal(qkv * 4) * 0.3).astype(np.float32),
                           "a_log": g.uniform(0, 2.7, nv).astype(np.float32),
                           "dt_bias": g.uniform(-1, 1, nv).astype(np.float32),
                           "attn_norm_weight": _vec16(g, 128, 1.0), **mlp})
        else:
            layers.append({"q_proj": W(hidden, q_out), "k_proj": W(hidden, kv_out), "v_proj": W(hidden, kv_out),
                           "o_proj": W(q_out // 2, hidden), "q_norm": _vec16(g, head_dim, 1.0),
                           "k_norm": _vec16(g, head_dim, 1.0), **mlp})
    half = int(head_dim * 0.25) // 2
    ang = np.arange(max_pos)[:, None] * (1.0e7 ** (-2.0 * np.arange(half) / (2 * half)))[None, :]
    globs = {"embed": W(vocab, hidden), "final_norm": _vec16(g, hidden, 1.0),
             "rope_cos": np.cos(ang).astype(np.float32).reshape(-1),
             "rope_sin": np.sin(ang).astype(np.float32).reshape(-1)}
    return Q.Model(Q.VERSION, 1 if kind == "q4" else 0, cfg, list(layer_types), layers, globs)


def _same(a, b):
    if isinstance(a, Q.Weight):
        assert (a.kind, a.k, a.n) == (b.kind, b.k, b.n)
        np.testing.assert_array_equal(np.asarray(a.data).reshape(-1), np.asarray(b.data).reshape(-1))
        if a.kind == "q4":
            np.testing.assert_array_equal(np.asarray(a.scales).reshape(-1), np.asarray(b.scales).reshape(-1))
    else:
        np.testing.assert_array_equal(np.asarray(a), np.asarray(b))


@pytest.mark.parametrize("kind", ["q4", "f16"])
def test_round_trip_every_record(orc, tmp_path, kind):
    g = np.random.default_rng(1)
    m = _model(orc, g, [0, 0, 1, 0], hidden=64, qkv=96, vdim=64, nv=32, q_out=128, kv_out=32, head_dim=16,
               vocab=96, max_pos=10, kind=kind)
    p = tmp_path / "m.qor4b"
    Q.write_qor4b(p, m)
    r = Q.read_qor4b(p)
    assert (r.version, r.format_id, r.layer_types, r.vision_offset) == (2, m.format_id, [0, 0, 1, 0], -1)
    for key, v in m.config.items():
        assert r.config[key] == v, key
    for la, lb in zip(m.layers, r.layers):
        assert la.keys() == lb.keys()
        for name in la:
            _same(la[name], lb[name])
    for name in m.globals:
        _same(m.globals[name], r.globals[name])
    assert r.layers[0]["in_proj_qkv"].data.shape == ((64, 48) if kind == "q4" else (64, 96))


def test_rejections(orc, tmp_path):
    g = np.random.default_rng(2)
    m = _model(orc, g, [0, 1], hidden=64, qkv=96, vdim=64, nv=32, q_out=128, kv_out=32, head_dim=16,
               vocab=32, max_pos=4)
    p = tmp_path / "m.qor4b"
    Q.write_qor4b(p, m)
    raw = bytearray(p.read_bytes())

    def reject(data, msg):
        bad = tmp_path / "bad.qor4b"
        bad.write_bytes(bytes(data))
        with pytest.raises(Q.Qor4bError, match=msg):
            Q.read_qor4b(bad)

    reject(b"QOR5" + raw[4:], "magic")
    reject(raw[:4] + (3).to_bytes(4, "little") + raw[8:], "version 3")
    reject(raw[:-5], "truncated")
    # the first weight record starts after header (9), config (11 u32, f64, f32, f64, u32, u8, u8 = 70)
    # and the layer types (2); its format byte follows k and n
    off = 9 + 70 + 2 + 16
    assert raw[off] == 1
    reject(raw[:off] + bytes([7]) + raw[off + 1:], "Unknown weight format 7")
    wrong = bytearray(raw)
    wrong[off - 8:off] = (65).to_bytes(8, "little")  # n = 65: not a multiple of 32
    reject(wrong, "Q4")
    v1 = raw[:4] + (1).to_bytes(4, "little") + raw[8:]
    bad = tmp_path / "v1.qor4b"
    bad.write_bytes(bytes(v1))
    assert Q.read_qor4b(bad).version == 1  # version 1 reads the same (its vision section differs)


@pytest.mark.gpu
@pytest.mark.parametrize("kind", ["q4", "f16"])
def test_file_to_device_mixer_path(orc, tmp_path, kind):
    """A one-DeltaNet + one-attention model at the 4B's dimensions, Q4 or F16
    weights: every projection, both mixers and lm_head from the uploaded file
    against the restatement on the file's own records (gemv_q4 / gemv_f16 and
    lm_head_q4 / lm_head_f16 as the record's format says, src/gemv.rs:286-291,
    662-711)."""
    import torch

    import qora_mixer as qm
    import refmath
    from gpu_util import dev, host, make_ctx

    g = np.random.default_rng(3)
    m = _model(orc, g, [0, 1], hidden=2560, qkv=8192, vdim=4096, nv=32, q_out=8192, kv_out=1024, head_dim=256,
               vocab=1000, max_pos=64, kind=kind)
    p = tmp_path / "m.qor4b"
    Q.write_qor4b(p, m)
    r = Q.read_qor4b(p)
    ctx = make_ctx()
    try:
        up = Q.upload_mixers(r)
        mx = qm.Mixer(ctx)
        c = orc.cfg_4b()

        def ref_gemv(v, w):
            return orc.gemv_q4(v, w.data, w.scales) if w.kind == "q4" else orc.gemv_f16(v, w.data)

        x = g.standard_normal((1, 2560)).astype(np.float32)
        xd = dev(x)
        # DeltaNet layer: fused in_proj, the mixer with its fused gate, out_proj
        L0 = r.layers[0]
        outs = [torch.empty(1, n, device="cuda") for n in (8192, 32, 32, 4096)]
        mx.gemv_multi(up[0]["in_proj"], xd, outs)
        ctx.sync()
        got = [host(o)[0] for o in outs]
        for name, o in zip(("in_proj_qkv", "in_proj_a", "in_proj_b", "in_proj_z"), got):
            assert L0[name].kind == kind
            assert refmath.rel_err(o, ref_gemv(x[0], L0[name])) <= 5e-5, name
        st = qm.DnState(ctx, 1)
        y = torch.empty(1, 32, 128, device="cuda")
        gated = torch.empty(1, 4096, device="cuda")
        mx.dn_decode(up[0]["params"], st, outs[0], outs[1], outs[2], y, outs[3], gated)
        ctx.sync()
        ost = orc.DnState(c)
        gamma = np.asarray(L0["attn_norm_weight"]).view(np.float16).astype(np.float32)
        yo, go = orc.dn_decode(c, ost, got[0], got[1], got[2], np.asarray(L0["conv1d_weight"]),
                               np.asarray(L0["a_log"]), np.asarray(L0["dt_bias"]), z=got[3], norm_gamma=gamma)
        assert refmath.rel_err(host(y)[0], yo) <= 1e-3
        assert refmath.rel_err(host(gated)[0], go) <= 1e-3
        h = torch.empty(1, 2560, device="cuda")
        mx.gemv(up[0]["out_proj"], gated, h)
        ctx.sync()
        assert refmath.rel_err(host(h)[0], ref_gemv(host(gated)[0], L0["out_proj"])) <= 5e-5
        st.close()
        # attention layer at position 0 (empty cache)
        L1 = r.layers[1]
        qo = [torch.empty(1, n, device="cuda") for n in (8192, 1024, 1024)]
        mx.gemv_multi(up[1]["in_proj"], xd, qo)
        K = torch.zeros(1, 4, 8, 256, dtype=torch.int16, device="cuda")
        V = torch.zeros_like(K)
        kv = qm.KvCache(ctx, 1, 8, K, V)
        att = torch.empty(1, 16, 256, device="cuda")
        mx.gqa_decode(up[1]["params"], kv, qo[0].view(1, 16, 512), qo[1].view(1, 4, 256), qo[2].view(1, 4, 256),
                      att)
        ctx.sync()
        qg, kn, vn = (host(t)[0] for t in qo)
        okv = orc.KvCache(c, 9)
        f16 = lambda a: np.asarray(a).view(np.float16).astype(np.float32)  # noqa: E731
        cos = np.asarray(r.globals["rope_cos"]).reshape(-1, 32)
        sin = np.asarray(r.globals["rope_sin"]).reshape(-1, 32)
        ref = orc.gqa_decode(c, okv, qg.reshape(16, 512), kn.reshape(4, 256), vn.reshape(4, 256),
                             f16(L1["q_norm"]), f16(L1["k_norm"]), cos, sin)
        assert refmath.rel_err(host(att)[0], ref) <= 1e-3
        kv.close()
        # lm_head over the tied embedding rows
        logits = torch.empty(1, 1000, device="cuda")
        mx.gemv(up[-1]["lm_head"], xd, logits)
        ctx.sync()
        E = r.globals["embed"]
        ref_logits = orc.lm_head_q4(x[0], E.data, E.scales) if kind == "q4" else orc.lm_head_f16(x[0], E.data)
        assert refmath.rel_err(host(logits)[0], ref_logits) <= 5e-5
    finally:
        ctx.close()
