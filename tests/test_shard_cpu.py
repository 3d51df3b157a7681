"""Head-sharded layout on the CPU: the plan (qm_shard_plan) covers every head
exactly once, the gather helpers invert the sharding, and two gloo ranks that
each hold one shard of the oracle's outputs rebuild the full outputs through a
real all-gather (the host-side half of the multi-GPU path; the device half is
in test_shard_gpu.py)."""
import os
import socket

import numpy as np
import pytest

from qora_mixer import inputs as I
from qora_mixer import layout


def test_plan_covers_every_head_once():
    import qora_mixer as qm

    for world in (1, 2, 4, 8, 16):
        plans = [qm.shard_plan(world, r) for r in range(world)]
        vh = np.zeros(32, int)
        cover = np.zeros((world, 4), int)  # (batch part, KV head)
        for p in plans:
            vh[p["vh_lo"]:p["vh_lo"] + p["nvh"]] += 1
            assert p["vh_lo"] % 2 == 0 and p["nvh"] % 2 == 0
            cover[p["seq_part"], p["kv_lo"]:p["kv_lo"] + p["nkv"]] += 1
            assert p["seq_parts"] * min(world, 4) == world
        assert (vh == 1).all(), world
        assert (cover[:plans[0]["seq_parts"]] == 1).all(), world
    for world, rank in ((3, 0), (32, 0), (2, 2), (0, 0)):
        with pytest.raises(qm.QmError):
            qm.shard_plan(world, rank)


@pytest.mark.parametrize("world", [1, 2, 4, 8, 16])
def test_gather_inverts_sharding(world):
    import qora_mixer as qm

    B = 16
    g = np.random.default_rng(world)
    y = g.standard_normal((B, 32, 128)).astype(np.float32)
    o = g.standard_normal((B, 16, 256)).astype(np.float32)
    plans = [qm.shard_plan(world, r) for r in range(world)]
    gy = np.stack([layout.dn_shard_of(y, p) for p in plans])
    go = np.stack([layout.gqa_shard_of(o, p) for p in plans])
    np.testing.assert_array_equal(layout.dn_from_gathered(gy, world, B), y)
    np.testing.assert_array_equal(layout.gqa_from_gathered(go, world, B), o)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, q):
    """One gloo rank: oracle outputs of a DeltaNet and a GQA decode step for
    B sequences, cut to this rank's shard, all-gathered, rebuilt."""
    import sys

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    for p in (root, os.path.join(root, "qora-llm-4b_b200")):
        if p not in sys.path:
            sys.path.insert(0, p)
    import torch
    import torch.distributed as dist

    import qora_mixer as qm
    from oracle import oracle as orc
    from qora_mixer import inputs as I
    from qora_mixer import layout

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        B, L = 4, 40
        c = orc.cfg_4b()
        g = I.rng(1234)
        p = I.dn_layer_params(g)
        toks = I.dn_token_inputs(g, 1, B)
        y = np.stack([orc.dn_decode(c, orc.DnState(c), toks["qkv"][b, 0], toks["a"][b, 0],
                                    toks["b"][b, 0], p["conv_w"], p["a_log"], p["dt_bias"],
                                    use_avx512=False) for b in range(B)])
        pr = I.gqa_layer_params(g, L + 2)
        cos, sin = orc.rope_table(1.0e7, 64, L + 2)
        kb, vb = I.gqa_cache_bf16(g, B, L)
        tok = I.gqa_token_inputs(g, B)
        o = []
        for b in range(B):
            kv = orc.KvCache(c, L + 1, I.bf16_bits_to_f32(kb[b]).transpose(1, 0, 2).reshape(L, -1),
                             I.bf16_bits_to_f32(vb[b]).transpose(1, 0, 2).reshape(L, -1))
            o.append(orc.gqa_decode(c, kv, tok["q_gate"][b], tok["k_new"][b], tok["v_new"][b],
                                    pr["q_norm"], pr["k_norm"], cos, sin))
        o = np.stack(o).reshape(B, 16, 256)
        plan = qm.shard_plan(world, rank)
        mine_y = torch.from_numpy(np.ascontiguousarray(layout.dn_shard_of(y.reshape(B, 32, 128), plan)))
        mine_o = torch.from_numpy(np.ascontiguousarray(layout.gqa_shard_of(o, plan)))
        gy = [torch.empty_like(mine_y) for _ in range(world)]
        go = [torch.empty_like(mine_o) for _ in range(world)]
        dist.all_gather(gy, mine_y)
        dist.all_gather(go, mine_o)
        ry = layout.dn_from_gathered(torch.stack(gy), world, B).numpy()
        ro = layout.gqa_from_gathered(torch.stack(go), world, B).numpy()
        ok = np.array_equal(ry, y.reshape(B, 32, 128)) and np.array_equal(ro, o)
        q.put((rank, bool(ok)))
    finally:
        dist.destroy_process_group()


def test_gloo_two_ranks_rebuild_outputs():
    import torch.multiprocessing as mp

    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, q)) for r in range(world)]
    for pr in procs:
        pr.start()
    for pr in procs:
        pr.join(timeout=180)
    res = dict(q.get(timeout=5) for _ in range(world))
    for pr in procs:
        assert pr.exitcode == 0
    assert res == {0: True, 1: True}
