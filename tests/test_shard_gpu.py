"""Head-sharded decode on the GPU (the V/KV-head-sharded layout of workload 4).

Every rank of a world of 2, 4 or 8 is run in turn on one GPU: each holds its
head shard (qm_dn_state_create_heads / qm_kv_create_heads), reads the
full-width inputs and writes its slice of the outputs; the slices, stacked in
rank order as qm_comm_allgather would, must rebuild the oracle's outputs
(src/gemv.rs:744-883 and 927-1011) within the decode tolerance
max|gpu - cpu| / RMS(cpu) <= 1e-3.  The last test runs the real NCCL
all-gather between two GPUs and is skipped on a one-GPU box.
"""
import os
import socket

import numpy as np
import pytest

import refmath
from gpu_util import dev, host, make_ctx
from qora_mixer import inputs as I
from qora_mixer import layout

pytestmark = pytest.mark.gpu
TOL = 1e-3


@pytest.fixture(scope="module")
def ctx():
    c = make_ctx()
    yield c
    c.close()


def _dn_reference(orc, B, T, seed, fused):
    """Oracle outputs of T decode steps for B sequences from zero state."""
    c = orc.cfg_4b()
    g = I.rng(seed)
    p = I.dn_layer_params(g)
    toks = I.dn_token_inputs(g, T, B)
    ost = [orc.DnState(c) for _ in range(B)]
    ys, outs = [], []
    for t in range(T):
        yt, ot = [], []
        for b in range(B):
            r = orc.dn_decode(c, ost[b], toks["qkv"][b, t], toks["a"][b, t], toks["b"][b, t],
                              p["conv_w"], p["a_log"], p["dt_bias"], use_avx512=False,
                              z=toks["z"][b, t] if fused else None,
                              norm_gamma=p["norm_gamma"] if fused else None)
            y, o = r if fused else (r, None)
            yt.append(y)
            ot.append(o)
        ys.append(np.stack(yt))
        outs.append(np.stack(ot) if fused else None)
    return p, toks, ost, ys, outs


@pytest.mark.parametrize("world", [2, 4, 8])
def test_dn_head_shards_rebuild_decode(ctx, orc, world):
    import torch

    import qora_mixer as qm

    B, T = 3, 3
    p, toks, ost, ys, outs = _dn_reference(orc, B, T, 2000 + world, fused=True)
    keep = [dev(p["conv_w"]), dev(p["a_log"]), dev(p["dt_bias"]), dev(p["norm_gamma"])]
    prm = qm.dn_params(*keep)
    mx = qm.Mixer(ctx)
    plans = [qm.shard_plan(world, r) for r in range(world)]
    states = [qm.DnState(ctx, B, heads=(pl["vh_lo"], pl["nvh"])) for pl in plans]
    for t in range(T):
        gy, go = [], []
        for pl, st in zip(plans, states):
            y = torch.full((B, pl["nvh"] * 128), float("nan"), device="cuda")
            out = torch.full((B, pl["nvh"] * 128), float("nan"), device="cuda")
            mx.dn_decode(prm, st, dev(toks["qkv"][:, t]), dev(toks["a"][:, t]), dev(toks["b"][:, t]),
                         y, dev(toks["z"][:, t]), out)
            gy.append(y)
            go.append(out)
        ctx.sync()
        ry = host(layout.dn_from_gathered(torch.stack(gy), world, B))
        ro = host(layout.dn_from_gathered(torch.stack(go), world, B))
        assert refmath.rel_err(ry, ys[t]) <= TOL
        assert refmath.rel_err(ro, outs[t].reshape(B, 32, 128)) <= TOL
    for pl, st in zip(plans, states):
        assert st.conv_pos == T
        lo, n = pl["vh_lo"], pl["nvh"]
        for b in range(B):
            s_g, cb_g = st.read(b)
            assert refmath.rel_err(s_g, ost[b].s[lo:lo + n]) <= TOL
            # the shard advances the conv history of its own channels only
            qk = np.r_[lo // 2 * 128:(lo + n) // 2 * 128]
            ch = np.concatenate([qk, 2048 + qk, 4096 + np.r_[lo * 128:(lo + n) * 128]])
            np.testing.assert_array_equal(cb_g[ch], ost[b].conv_buf[ch])
        st.close()


@pytest.mark.parametrize("world,L", [(2, 200), (4, 64), (8, 1000)])
def test_gqa_head_shards_rebuild_decode(ctx, orc, world, L):
    import torch

    import qora_mixer as qm

    B, cap = 4, L + 8
    c = orc.cfg_4b()
    g = I.rng(2100 + world)
    pr = I.gqa_layer_params(g, cap + 1)
    cos, sin = qm.rope_table(1.0e7, 64, cap + 1)
    kb, vb = I.gqa_cache_bf16(g, B, L)  # [B,4,L,256] bf16 bits
    tok = I.gqa_token_inputs(g, B)
    ref = []
    for b in range(B):
        okv = orc.KvCache(c, cap + 1, I.bf16_bits_to_f32(kb[b]).transpose(1, 0, 2).reshape(L, -1),
                          I.bf16_bits_to_f32(vb[b]).transpose(1, 0, 2).reshape(L, -1))
        ref.append(orc.gqa_decode(c, okv, tok["q_gate"][b], tok["k_new"][b], tok["v_new"][b],
                                  pr["q_norm"], pr["k_norm"], cos, sin))
    ref = np.stack(ref)
    keep = [dev(pr["q_norm"]), dev(pr["k_norm"]), dev(cos), dev(sin)]
    prm = qm.gqa_params(*keep)
    mx = qm.Mixer(ctx)
    gathered = []
    for r in range(world):
        pl = qm.shard_plan(world, r)
        bp = B // pl["seq_parts"]
        s0 = pl["seq_part"] * bp
        lo, n = pl["kv_lo"], pl["nkv"]
        K = torch.zeros(bp, n, cap, 256, dtype=torch.int16, device="cuda")
        V = torch.zeros_like(K)
        K[:, :, :L] = dev(kb[s0:s0 + bp, lo:lo + n])
        V[:, :, :L] = dev(vb[s0:s0 + bp, lo:lo + n])
        kv = qm.KvCache(ctx, bp, cap, K, V, heads=(lo, n))
        kv.seq_len = L
        out = torch.full((bp, n * 4 * 256), float("nan"), device="cuda")
        mx.gqa_decode(prm, kv, dev(tok["q_gate"][s0:s0 + bp]), dev(tok["k_new"][s0:s0 + bp]),
                      dev(tok["v_new"][s0:s0 + bp]), out)
        ctx.sync()
        assert kv.seq_len == L + 1
        # the appended row went to this shard's heads: V is the bf16 of v_new
        np.testing.assert_array_equal(host(V[:, :, L]),
                                      I.f32_to_bf16_bits(tok["v_new"][s0:s0 + bp, lo:lo + n]))
        gathered.append(out)
        kv.close()
    rebuilt = host(layout.gqa_from_gathered(torch.stack(gathered), world, B))
    assert refmath.rel_err(rebuilt, ref) <= TOL


def test_prefill_rejects_head_shards(ctx):
    import torch

    import qora_mixer as qm

    st = qm.DnState(ctx, 1, heads=(0, 16))
    kv = qm.KvCache(ctx, 1, 64, heads=(1, 2))
    with pytest.raises(qm.QmError) as e:
        qm.Mixer(ctx).dn_prefill(qm.dn_params(*[torch.zeros(8192 * 4, device="cuda")] * 3), st, 8,
                                 torch.zeros(8, 8192, dtype=torch.int16, device="cuda"),
                                 torch.zeros(8, 32, device="cuda"), torch.zeros(8, 32, device="cuda"),
                                 torch.zeros(8, 32, 128, device="cuda"))
    assert e.value.code == 9  # QM_E_UNSUPPORTED
    z = torch.zeros(4096, device="cuda")
    prm = qm.gqa_params(z, z, torch.zeros(64, 32, device="cuda"), torch.zeros(64, 32, device="cuda"))
    with pytest.raises(qm.QmError) as e:
        qm.Mixer(ctx).gqa_prefill(prm, kv, 8, torch.zeros(8, 16, 512, dtype=torch.int16, device="cuda"),
                                  torch.zeros(8, 4, 256, dtype=torch.int16, device="cuda"),
                                  torch.zeros(8, 4, 256, dtype=torch.int16, device="cuda"),
                                  torch.zeros(8, 16, 256, device="cuda"))
    assert e.value.code == 9
    with pytest.raises(qm.QmError):
        qm.DnState(ctx, 1, heads=(1, 2))  # not QK-head aligned
    with pytest.raises(qm.QmError):
        qm.KvCache(ctx, 1, 64, heads=(3, 2))
    st.close()
    kv.close()


# ---------------------------------------------------------------------------
# two GPUs: head shards + the NCCL all-gather through qm_comm_allgather
# ---------------------------------------------------------------------------
def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _two_gpu_rank(rank, world, port, q):
    import sys

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    for p in (root, os.path.join(root, "qora-llm-4b_b200"), os.path.join(root, "tests")):
        if p not in sys.path:
            sys.path.insert(0, p)
    import datetime

    import torch
    import torch.distributed as dist

    import qora_mixer as qm
    from oracle import oracle as orc
    from qora_mixer import inputs as I
    from qora_mixer import layout

    import refmath

    torch.cuda.set_device(rank)
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    ctx = qm.Ctx(rank, stream=torch.cuda.current_stream())
    comm = None
    try:
        uid = [qm.comm_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(uid, src=0)
        comm = qm.Comm(ctx, uid[0], world, rank, timeout_ms=60000)
        pl = qm.shard_plan(world, rank)
        B = 4
        c = orc.cfg_4b()
        g = I.rng(2200)
        p = I.dn_layer_params(g)
        toks = I.dn_token_inputs(g, 1, B)
        keep = [torch.from_numpy(p[k]).cuda() for k in ("conv_w", "a_log", "dt_bias", "norm_gamma")]
        st = qm.DnState(ctx, B, heads=(pl["vh_lo"], pl["nvh"]))
        y = torch.empty(B, pl["nvh"] * 128, device="cuda")
        qm.Mixer(ctx).dn_decode(qm.dn_params(*keep), st, torch.from_numpy(toks["qkv"][:, 0]).cuda(),
                                torch.from_numpy(toks["a"][:, 0]).cuda(),
                                torch.from_numpy(toks["b"][:, 0]).cuda(), y)
        gy = torch.empty(world, B, pl["nvh"] * 128, device="cuda")
        comm.allgather(y, gy)
        ctx.sync()
        rebuilt = layout.dn_from_gathered(gy, world, B).cpu().numpy()
        ref = np.stack([orc.dn_decode(c, orc.DnState(c), toks["qkv"][b, 0], toks["a"][b, 0],
                                      toks["b"][b, 0], p["conv_w"], p["a_log"], p["dt_bias"],
                                      use_avx512=False) for b in range(B)])
        err = refmath.rel_err(rebuilt, ref)
        st.close()
        q.put((rank, float(err)))
    finally:
        if comm is not None:
            comm.close()
        ctx.close()
        dist.destroy_process_group()


def test_two_gpus_nccl_allgather_of_head_shards():
    import torch
    import torch.multiprocessing as mp

    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    world = 2
    mctx = mp.get_context("spawn")
    q = mctx.Queue()
    port = _free_port()
    procs = [mctx.Process(target=_two_gpu_rank, args=(r, world, port, q)) for r in range(world)]
    for pr in procs:
        pr.start()
    for pr in procs:
        pr.join(timeout=300)
    res = dict(q.get(timeout=5) for _ in range(world))
    for pr in procs:
        assert pr.exitcode == 0
    assert all(e <= TOL for e in res.values()), res


# ---------------------------------------------------------------------------
# peer-memory all-gather (qm_comm_enable_peer)
# ---------------------------------------------------------------------------
def _gather_cases(world, rank, torch, off_send=0, off_recv=0):
    """(send, recv) pairs of assorted sizes; offsets make unaligned views."""
    out = []
    for n in (16, 4112, 131072, 300003, 2 << 20):
        g = torch.Generator().manual_seed(n * 31 + rank)
        sb = torch.randint(0, 256, (n + off_send,), dtype=torch.uint8, generator=g).cuda()
        rb = torch.zeros(world * n + off_recv, dtype=torch.uint8, device="cuda")
        out.append((sb[off_send:off_send + n], rb[off_recv:off_recv + world * n]))
    return out


def test_peer_allgather_single_rank(ctx):
    """World of one: the gather kernel's own-row copy (16-byte and byte paths,
    one to sixteen chunks) and the NCCL path above the peer size limit."""
    import torch

    import qora_mixer as qm

    comm = qm.Comm(ctx, qm.comm_unique_id(), 1, 0, timeout_ms=30000)
    try:
        assert comm.enable_peer(1 << 20, wait_ms=1000)
        with pytest.raises(qm.QmError):
            comm.enable_peer(1 << 20)  # already on
        n0 = ctx.launch_count()
        for osend, orecv in ((0, 0), (1, 3)):
            for send, recv in _gather_cases(1, 0, torch, osend, orecv):
                comm.allgather(send, recv)
                ctx.sync()
                assert torch.equal(recv, send)
        assert ctx.launch_count() - n0 == 8  # the two 2 MiB gathers went to NCCL
    finally:
        comm.close()


def _two_gpu_peer_rank(rank, world, port, q):
    import sys

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    for p in (root, os.path.join(root, "qora-llm-4b_b200"), os.path.join(root, "tests")):
        if p not in sys.path:
            sys.path.insert(0, p)
    import datetime
    import time

    import torch
    import torch.distributed as dist

    import qora_mixer as qm

    torch.cuda.set_device(rank)
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    ctx = qm.Ctx(rank, stream=torch.cuda.current_stream())
    comm = None
    res = {"rank": rank}
    try:
        uid = [qm.comm_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(uid, src=0)
        comm = qm.Comm(ctx, uid[0], world, rank, timeout_ms=30000)
        # NCCL results first, then the same gathers through the peer kernel
        cases = {}
        for osend, orecv in ((0, 0), (1, 3)):
            for send, recv in _gather_cases(world, rank, torch, osend, orecv):
                comm.allgather(send, recv)
                ctx.sync()
                cases[(osend, orecv, send.numel())] = recv.clone()
        res["peer"] = comm.enable_peer(1 << 20, wait_ms=2000)
        same = True
        for rep in range(3):  # both slots, several epochs
            for osend, orecv in ((0, 0), (1, 3)):
                for send, recv in _gather_cases(world, rank, torch, osend, orecv):
                    recv.zero_()
                    comm.allgather(send, recv)
                    ctx.sync()
                    same &= bool(torch.equal(recv, cases[(osend, orecv, send.numel())]))
        res["same"] = same
        # a rank that skips one call: the other's bounded wait gives up
        send, recv = _gather_cases(world, rank, torch)[2]
        if rank == 0:
            t0 = time.time()
            comm.allgather(send, recv)
            try:
                ctx.sync()
                res["timeout_code"] = 0
            except qm.QmError as e:
                res["timeout_code"] = e.code
            res["waited_s"] = time.time() - t0
            try:
                comm.allgather(send, recv)
                res["after_code"] = 0
            except qm.QmError as e:
                res["after_code"] = e.code
        dist.barrier()
        comm.close()  # collective with the peer path on
        comm = None
        q.put(res)
    finally:
        if comm is not None:
            comm.close()
        ctx.close()
        dist.destroy_process_group()


def test_two_gpus_peer_allgather_matches_nccl():
    """Two GPUs: the peer-memory gather reproduces NCCL's bytes (aligned and
    unaligned buffers, sizes 16 B .. 300 KB, both slots), sizes above the
    limit still go to NCCL, and a rank that skips a call makes the other's
    device-side wait give up after its limit (QM_E_TIMEOUT from qm_sync and
    from every later call), with no GPU fault."""
    import torch
    import torch.multiprocessing as mp

    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    world = 2
    mctx = mp.get_context("spawn")
    q = mctx.Queue()
    port = _free_port()
    procs = [mctx.Process(target=_two_gpu_peer_rank, args=(r, world, port, q)) for r in range(world)]
    for pr in procs:
        pr.start()
    for pr in procs:
        pr.join(timeout=300)
    res = {r["rank"]: r for r in (q.get(timeout=5) for _ in range(world))}
    for pr in procs:
        assert pr.exitcode == 0
    for r in range(world):
        assert res[r]["peer"] and res[r]["same"], res
    assert res[0]["timeout_code"] == 6 and res[0]["after_code"] == 6, res
    assert 1.5 < res[0]["waited_s"] < 30, res
