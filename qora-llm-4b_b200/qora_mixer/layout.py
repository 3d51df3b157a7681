"""Head-sharded layout: which rank computes what, and how the all-gathered
mixer outputs map back to the reference's per-token layout.

The reference produces, per token, the DeltaNet output y [32,128] (V heads
in order, src/gemv.rs:814-862) and the GQA output [16,256] (query heads in
order, src/gemv.rs:1006-1011).  Under qm_shard_plan, rank r computes

  DeltaNet  y[:, vh_lo:vh_lo+nvh]          for all B sequences
  GQA       out[part, 4*kv_lo:4*(kv_lo+nkv)] for the batch part seq_part

and qm_comm_allgather stacks the ranks' buffers in rank order.  The two
functions below undo that stacking.  They work on numpy arrays and torch
tensors alike (reshape + axis swap, no copies of the data beyond one).
"""
from __future__ import annotations


def _swap01(x):
    return x.transpose(0, 1) if hasattr(x, "permute") else x.swapaxes(0, 1)


def groups_parts(world: int):
    """(KV-head groups, batch parts) of the head-sharded layout (qm_shard_plan)."""
    groups = min(world, 4)
    return groups, world // groups


def dn_from_gathered(g, world: int, batch: int):
    """[world, B, nvh*128] (rank order) -> [B, 32, 128]."""
    nvh = 32 // world
    x = g.reshape(world, batch, nvh, 128)
    x = _swap01(x)  # [B, world, nvh, 128]
    return x.reshape(batch, 32, 128)


def gqa_from_gathered(g, world: int, batch: int):
    """[world, B/parts, nkv*4*256] (rank order; rank = part*groups + group)
    -> [B, 16, 256]."""
    groups, parts = groups_parts(world)
    bp = batch // parts
    nh = 16 // groups
    x = g.reshape(parts, groups, bp, nh, 256)
    x = x.transpose(1, 2) if hasattr(x, "permute") else x.swapaxes(1, 2)  # [parts, bp, groups, nh, 256]
    return x.reshape(batch, 16, 256)


def dn_shard_of(y_full, plan: dict):
    """Rank `plan`'s DeltaNet output [B, nvh*128] cut from a full [B, 32, 128]."""
    lo, n = plan["vh_lo"], plan["nvh"]
    b = y_full.shape[0]
    return y_full[:, lo:lo + n].reshape(b, n * 128)


def gqa_shard_of(o_full, plan: dict):
    """Rank `plan`'s GQA output [B/parts, nkv*4*256] cut from a full [B, 16, 256]."""
    b = o_full.shape[0]
    bp = b // plan["seq_parts"]
    s0 = plan["seq_part"] * bp
    h0, nh = plan["kv_lo"] * 4, plan["nkv"] * 4
    return o_full[s0:s0 + bp, h0:h0 + nh].reshape(bp, nh * 256)
