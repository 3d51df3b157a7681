#!/usr/bin/env python
"""Benchmark: the QORA-4B 32-layer token-mixer stack in decode (workload 4).

One step = one new token for each of B=64 independent sequences per GPU
through all 32 mixer layers (3 x DeltaNet + 1 x GQA, 8 times), at context
32768: 24 fp32 DeltaNet states [32,128,128] and 8 bf16 KV caches
[4,32768,256] per sequence, seeded N(0, 0.02); per-layer inputs N(0, 1)
with the value distributions of workloads 0 and 1 (synthetic; random-init
layer parameters).  Sequences are sharded across GPUs with no collective,
so every rank carries its own 64 sequences (weak scaling; --strong keeps
64 sequences in total).

value  = tokens/s of the whole job with inputs resident in HBM.
e2e    = the same through the C ABI's _host entry points: every layer call
         copies its inputs from pinned host memory and its output back.
roofline = the dominant kernel (split-KV GQA attention) against the
         measured HBM copy bandwidth; its launch durations come from a further
         timed pass of the same steps with CUDA events around every launch
         (events between kernels serialise them, so `value`'s pass has none).
cpu_baseline = the CPU restatement of the reference mixer path on a bounded
         sample (rank 0, N=1 only).

--impl reference times that CPU restatement as the reference arm (the
reference is a Rust crate and no Rust toolchain exists on these machines).
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(ROOT, "qora-llm-4b_b200")
for _p in (ROOT, PKG):
    if _p not in sys.path:
        sys.path.insert(0, _p)

METRIC = json.load(open(os.path.join(ROOT, "BASELINE.json")))["metric"]
UNIT = "tok/s"
CTX = 32768
B_PER_GPU = 64
LAYERS = ["dn", "dn", "dn", "attn"] * 8
WORKLOAD = "mixer-stack decode: 32 layers (24 DeltaNet + 8 GQA), ctx 32768"

# algorithmic bytes (reference algorithm, minimal traffic)
DN_BYTES_TOKEN = 2 * 32 * 128 * 128 * 4 + 2 * 8192 * 3 * 4 + 8192 * 4 + 2 * 32 * 4 + 2 * 4096 * 4


def attn_bytes(B, L):
    """K and V of L cached positions, 4 KV heads x 256 dims bf16, per sequence."""
    return B * 2 * 4 * L * 256 * 2


def load_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return d["hbm_gbs"], "measured"
    return 6650.0, "fallback"


def load_tensor_peak():
    """Dense bf16 tensor peak (burst: the prefill kernels are timed alone)."""
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        return json.load(open(p))["bf16_tflops"], "measured"
    return 1590.0, "fallback"


def load_traffic():
    p = os.path.join(ROOT, "profiles", "traffic.json")
    if os.path.exists(p):
        return json.load(open(p))
    return {}


# ----------------------------------------------------------------------------
# clocks sampler (nvidia-smi during the timed region)
# ----------------------------------------------------------------------------
class Clocks:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device):
        self.device = device
        self.proc = None
        self.lines = []

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "20", "-i", str(self.device)],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except Exception:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if not self.proc:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        self.t.join(timeout=5)  # the reader has seen every line before the summary
        return self.summarize(list(self.lines))

    @staticmethod
    def summarize(lines):
        """Median SM clock, the max clock and the throttle reasons seen Active, from nvidia-smi CSV lines
        (malformed or not-available samples are skipped)."""
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm)}


# ----------------------------------------------------------------------------
# distributed plumbing
# ----------------------------------------------------------------------------
def dist_env():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return ws, rank, local


def init_dist(ws, local):
    import torch

    if ws > 1:
        import datetime

        import torch.distributed as dist

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600),
                                device_id=torch.device("cuda", local))


def barrier(ws):
    if ws > 1:
        import torch.distributed as dist

        dist.barrier()


def max_over_ranks(x, ws):
    if ws == 1:
        return x
    import torch
    import torch.distributed as dist

    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


# ----------------------------------------------------------------------------
# the stack
# ----------------------------------------------------------------------------
class Stack:
    """24 DeltaNet states + 8 KV caches for B sequences, with per-layer params and inputs."""

    def __init__(self, ctx, B, cap, seed, ctx_len=CTX):
        import numpy as np
        import torch

        import qora_mixer as qm
        from qora_mixer import inputs as I

        self.qm, self.B = qm, B
        self.ctx, self.mx = ctx, qm.Mixer(ctx)
        g = I.rng(4, stream=seed)
        cos, sin = qm.rope_table(1.0e7, 64, cap + 1)
        self.rope = (torch.from_numpy(cos).cuda(), torch.from_numpy(sin).cuda())
        self.layers = []
        dseed = 0x51A4 * 1000 + seed * 100
        for li, kind in enumerate(LAYERS):
            L = {}
            if kind == "dn":
                p = I.dn_layer_params(g)
                L["keep"] = [torch.from_numpy(p[k]).cuda() for k in ("conv_w", "a_log", "dt_bias", "norm_gamma")]
                L["prm"] = qm.dn_params(*L["keep"])
                s = I.device_normal_f32((B, 32, 128, 128), dseed + li, 0.02)
                cv = torch.zeros(B, 4, 8192, device="cuda")
                cv[:, 1:] = I.device_normal_f32((B, 3, 8192), dseed + 50 + li, 0.02)
                L["store"] = (s, cv)
                L["st"] = qm.DnState(ctx, B, s, cv)
                L["st"].conv_pos = ctx_len  # slots (ctx-3..ctx-1) % 4 = 1..3 hold the history
                tok = I.dn_token_inputs(g, 1, B)
                L["in"] = [torch.from_numpy(np.ascontiguousarray(tok[k][:, 0])).cuda()
                           for k in ("qkv", "a", "b", "z")]
                L["out"] = torch.empty(B, 4096, device="cuda")
            else:
                p = I.gqa_layer_params(g, cap + 1)
                L["keep"] = [torch.from_numpy(p["q_norm"]).cuda(), torch.from_numpy(p["k_norm"]).cuda(), *self.rope]
                L["prm"] = qm.gqa_params(*L["keep"])
                K = I.device_normal_bf16((B, 4, cap, 256), dseed + li, 0.02).view(torch.int16)
                V = I.device_normal_bf16((B, 4, cap, 256), dseed + 70 + li, 0.02).view(torch.int16)
                L["store"] = (K, V)
                L["kv"] = qm.KvCache(ctx, B, cap, K, V)
                L["kv"].seq_len = ctx_len
                tok = I.gqa_token_inputs(g, B)
                L["in"] = [torch.from_numpy(tok[k]).cuda() for k in ("q_gate", "k_new", "v_new")]
                L["out"] = torch.empty(B, 16, 256, device="cuda")
            L["kind"] = kind
            self.layers.append(L)
        torch.cuda.synchronize()

    def step(self):
        mx = self.mx
        for L in self.layers:
            if L["kind"] == "dn":
                qkv, a, b, z = L["in"]
                mx.dn_decode(L["prm"], L["st"], qkv, a, b, None, z, L["out"])
            else:
                mx.gqa_decode(L["prm"], L["kv"], *L["in"], L["out"])

    def make_host_io(self):
        """Pinned host copies of every layer's inputs and outputs (for e2e),
        and each layer's C-ABI call with its arguments bound once, as a
        compiled caller holds them (the per-call Python argument conversion of
        the ctypes mirror is not the library's cost)."""
        import ctypes as C

        import torch

        import qora_mixer as qm

        lib = qm.lib()
        for L in self.layers:
            L["hin"] = [t.cpu().pin_memory() for t in L["in"]]
            L["hout"] = torch.empty(L["out"].shape, dtype=torch.float32).pin_memory()
            hin = [t.data_ptr() for t in L["hin"]]
            out = L["hout"].data_ptr()
            if L["kind"] == "dn":
                qkv, a, b, z = hin
                L["host_call"] = (lib.qm_dn_decode_host,
                                  (self.ctx.handle, C.byref(L["prm"]), L["st"].handle, qkv, a, b, None, z, out))
            else:
                L["host_call"] = (lib.qm_gqa_decode_host,
                                  (self.ctx.handle, C.byref(L["prm"]), L["kv"].handle, *hin, out))
        h2d = sum(t.numel() * 4 for L in self.layers for t in L["hin"])
        d2h = sum(L["hout"].numel() * 4 for L in self.layers)
        return h2d, d2h

    def step_host(self):
        """One step through qm_dn_decode_host / qm_gqa_decode_host: each call
        returns once its output is in the pinned host buffer."""
        for L in self.layers:
            fn, args = L["host_call"]
            rc = fn(*args)
            if rc != 0:
                self.ctx.check(rc, "host-buffer layer call")

    def seq_len(self):
        return self.layers[3]["kv"].seq_len

    def close(self):
        for L in self.layers:
            for k in ("st", "kv"):
                if k in L:
                    L[k].close()
        self.layers = []


class ShardedStack:
    """Workload 4's head-sharded variant (qm_shard_plan): B sequences in total
    over all ranks.  This rank holds V heads [vh_lo, vh_lo+nvh) of the 24
    DeltaNet layers for all B sequences, and KV heads [kv_lo, kv_lo+nkv) of
    batch part seq_part for the 8 GQA layers.  Every layer's output slice is
    all-gathered (qm_comm_allgather: the peer-memory kernel once
    qm_comm_enable_peer is on, else NCCL) on the mixer's stream, as
    out_proj / o_proj would need it."""

    def __init__(self, ctx, comm, plan, B, cap, ctx_len=CTX):
        import numpy as np
        import torch

        import qora_mixer as qm
        from qora_mixer import inputs as I

        self.ctx, self.comm, self.mx, self.plan, self.B = ctx, comm, qm.Mixer(ctx), plan, B
        world = plan["world"]
        nvh, nkv = plan["nvh"], plan["nkv"]
        bp = B // plan["seq_parts"]
        g = I.rng(4, stream=77)
        cos, sin = qm.rope_table(1.0e7, 64, cap + 1)
        self.rope = (torch.from_numpy(cos).cuda(), torch.from_numpy(sin).cuda())
        self.layers = []
        dseed = 0x51A4 * 1000 + 7700 + plan["rank"] * 100
        for li, kind in enumerate(LAYERS):
            L = {"kind": kind}
            if kind == "dn":
                p = I.dn_layer_params(g)
                L["keep"] = [torch.from_numpy(p[k]).cuda() for k in ("conv_w", "a_log", "dt_bias", "norm_gamma")]
                L["prm"] = qm.dn_params(*L["keep"])
                s = I.device_normal_f32((B, nvh, 128, 128), dseed + li, 0.02)
                cv = torch.zeros(B, 4, 8192, device="cuda")
                cv[:, 1:] = I.device_normal_f32((B, 3, 8192), dseed + 50 + li, 0.02)
                L["store"] = (s, cv)
                L["st"] = qm.DnState(ctx, B, s, cv, heads=(plan["vh_lo"], nvh))
                L["st"].conv_pos = ctx_len
                tok = I.dn_token_inputs(g, 1, B)
                L["in"] = [torch.from_numpy(np.ascontiguousarray(tok[k][:, 0])).cuda()
                           for k in ("qkv", "a", "b", "z")]
                L["out"] = torch.empty(B, nvh * 128, device="cuda")
            else:
                p = I.gqa_layer_params(g, cap + 1)
                L["keep"] = [torch.from_numpy(p["q_norm"]).cuda(), torch.from_numpy(p["k_norm"]).cuda(), *self.rope]
                L["prm"] = qm.gqa_params(*L["keep"])
                K = I.device_normal_bf16((bp, nkv, cap, 256), dseed + li, 0.02).view(torch.int16)
                V = I.device_normal_bf16((bp, nkv, cap, 256), dseed + 70 + li, 0.02).view(torch.int16)
                L["store"] = (K, V)
                L["kv"] = qm.KvCache(ctx, bp, cap, K, V, heads=(plan["kv_lo"], nkv))
                L["kv"].seq_len = ctx_len
                tok = I.gqa_token_inputs(g, bp)
                L["in"] = [torch.from_numpy(tok[k]).cuda() for k in ("q_gate", "k_new", "v_new")]
                L["out"] = torch.empty(bp, nkv * 4 * 256, device="cuda")
            L["gathered"] = torch.empty((world,) + tuple(L["out"].shape), device="cuda")
            self.layers.append(L)
        torch.cuda.synchronize()

    def step(self):
        mx, comm = self.mx, self.comm
        for L in self.layers:
            if L["kind"] == "dn":
                qkv, a, b, z = L["in"]
                mx.dn_decode(L["prm"], L["st"], qkv, a, b, None, z, L["out"])
            else:
                mx.gqa_decode(L["prm"], L["kv"], *L["in"], L["out"])
            comm.allgather(L["out"], L["gathered"])

    def close(self):
        for L in self.layers:
            for k in ("st", "kv"):
                if k in L:
                    L[k].close()
        self.layers = []


def bench_head_sharded(ctx, ws, rank, args):
    """Time the head-sharded stack (B sequences in total across the ranks)."""
    import torch
    import torch.distributed as dist

    import qora_mixer as qm

    plan = qm.shard_plan(ws, rank)
    B = args.batch
    cap = args.context + 2 * (args.warmup + args.steps) + 16
    uid = [qm.comm_unique_id() if rank == 0 else None]
    if ws > 1:
        dist.broadcast_object_list(uid, src=0)
    comm = qm.Comm(ctx, uid[0], ws, rank, timeout_ms=120000)
    stack = ShardedStack(ctx, comm, plan, B, cap, ctx_len=args.context)
    peer = False
    if args.gather == "peer":
        peer = comm.enable_peer(max(L["out"].numel() * 4 for L in stack.layers), wait_ms=10000)
    stream = torch.cuda.current_stream()
    for _ in range(args.warmup):
        stack.step()
    ctx.sync()
    barrier(ws)
    n0 = ctx.launch_count()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        stack.step()
    e1.record(stream)
    torch.cuda.synchronize()
    barrier(ws)
    launches = ctx.launch_count() - n0
    ms = max_over_ranks(e0.elapsed_time(e1), ws)
    # The per-kernel split comes from a second pass of the same steps with an
    # event pair around every launch: an event between two kernels also keeps
    # the second from starting early behind the first (the all-gather behind a
    # DeltaNet decode), so the step time above is taken without them.
    ctx.set_timing(True)
    for _ in range(args.steps):
        stack.step()
    torch.cuda.synchronize()
    barrier(ws)
    kt = {k: ctx.kernel_time(k) for k in ("dn_decode", "gqa_prep", "gqa_attn", "gqa_combine", "allgather")}
    ctx.set_timing(False)
    stack.close()
    comm.close()
    torch.cuda.empty_cache()
    gather_bytes = len(LAYERS) * B * 4096 * 4  # every layer's [B, 4096] f32 output, gathered
    return {"workload": f"head-sharded mixer-stack decode, batch {B} in total, ctx {args.context}",
            "value": round(B * args.steps / (ms / 1e3), 2), "unit": UNIT,
            "ms_per_step": round(ms / args.steps, 4), "scaling": "strong",
            "parallelism": (f"DeltaNet V heads /{ws}, GQA KV heads /{min(ws, 4)}"
                            + (f" x batch /{ws // min(ws, 4)}" if ws > 4 else "")
                            + (", peer-memory all-gather (NVLink stores, one kernel)" if peer
                               else ", NCCL all-gather") + " of every layer's output"),
            "allgather_bytes_per_step": gather_bytes, "gpu_launches": launches,
            "kernels_ms_per_step": {k: round(v[0] / args.steps, 4) for k, v in kt.items()},
            "kernels_timing": "a second pass of the same steps with an event pair around every launch"}


def run_ours(args):
    import torch

    import qora_mixer as qm

    ws, rank, local = dist_env()
    init_dist(ws, local)
    torch.cuda.set_device(local)
    B = args.batch if not args.strong else max(1, args.batch // ws)
    ctx_len = args.context
    # tokens appended: warm-up, the timed steps, the per-kernel pass, the e2e pass
    cap = ctx_len + 3 * (args.warmup + args.steps) + 16
    ctx = qm.Ctx(local, stream=torch.cuda.current_stream())
    stack = Stack(ctx, B, cap, seed=rank, ctx_len=ctx_len)
    stream = torch.cuda.current_stream()

    # ---- device-resident run ----
    for _ in range(args.warmup):
        stack.step()
    ctx.sync()
    barrier(ws)
    clocks = Clocks(local)
    clocks.start()
    time.sleep(1.0)  # let nvidia-smi start sampling before the timed region
    n0 = ctx.launch_count()
    torch.cuda.synchronize()
    barrier(ws)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record(stream)
    for _ in range(args.steps):
        stack.step()
    ev1.record(stream)
    torch.cuda.synchronize()
    barrier(ws)
    launches = ctx.launch_count() - n0
    ms_local = ev0.elapsed_time(ev1)
    clk = clocks.stop()

    ms = max_over_ranks(ms_local, ws)
    ms_step = ms / args.steps
    tokens = B * ws * args.steps
    value = tokens / (ms / 1e3)

    # ---- e2e through the _host entry points ----
    e2e = None
    if not args.no_e2e:
        h2d, d2h = stack.make_host_io()
        for _ in range(min(2, args.warmup)):
            stack.step_host()
        torch.cuda.synchronize()
        barrier(ws)
        t0 = time.perf_counter()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(args.steps):
            stack.step_host()
        e1.record(stream)
        torch.cuda.synchronize()
        wall = (time.perf_counter() - t0) * 1e3
        e2e_ms = max_over_ranks(max(e0.elapsed_time(e1), wall), ws)
        e2e = {"value": round(tokens / (e2e_ms / 1e3), 2), "unit": UNIT,
               "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h}

    # ---- per-kernel durations: a further timed pass of the same K steps with
    # the library's event pair around every launch (on the launching stream),
    # after the e2e pass so that it runs where it always did.  An event between
    # two kernels also keeps the second from starting early behind the first,
    # so the step time above is taken without them. ----
    L0 = stack.seq_len()
    ctx.set_timing(True)
    torch.cuda.synchronize()
    barrier(ws)
    for _ in range(args.steps):
        stack.step()
    torch.cuda.synchronize()
    barrier(ws)
    ktimes = {k: ctx.kernel_time(k) for k in ("dn_decode", "gqa_prep", "gqa_attn", "gqa_combine")}
    ctx.set_timing(False)
    ctx.sync()
    # ---- roofline of the dominant kernel (split-KV attention) ----
    peak, peak_kind = load_peaks()
    att_ms, att_n = ktimes["gqa_attn"]
    L_avg = L0 + (args.steps - 1) / 2.0
    att_bytes = attn_bytes(B, L_avg)
    att_achieved = att_bytes / (att_ms / att_n / 1e3) / 1e9
    dn_ms, dn_n = ktimes["dn_decode"]
    dn_achieved = B * DN_BYTES_TOKEN / (dn_ms / dn_n / 1e3) / 1e9
    traffic = load_traffic().get("gqa_attn_bytes_per_seq_pos")
    att_traffic = traffic * B * L_avg if traffic else None
    step_kernel_ms = sum(v[0] for v in ktimes.values()) / args.steps

    line = {
        "metric": METRIC, "value": round(value, 2), "unit": UNIT, "n_gpus": ws,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_step, 4),
        "higher_is_better": True, "scaling": "strong" if args.strong else "weak",
        "vs_baseline": None, "dtype": "f32 state / bf16 KV (f32 math)",
        "data": "synthetic (seeded N(0,1) inputs, N(0,0.02) states/caches, random-init params)",
        "config": decode_config(ws, B, ctx_len),
        "e2e": e2e,
        "gpu_launches": launches,
        "roofline": {"bound": "hbm", "kernel": "gqa_attn (split-KV attention)",
                     "achieved": round(att_achieved, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(att_achieved / peak, 4), "peak_kind": peak_kind,
                     "traffic": att_traffic,
                     "traffic_source": ("not measured in this run: the DRAM bytes per (sequence, cached position) "
                                        "of an ncu capture of a smaller case (profiles/traffic.json) x batch x "
                                        "positions") if att_traffic else None,
                     "algorithmic_bytes_per_launch": att_bytes,
                     "avg_launch_us": round(att_ms / att_n * 1e3, 2),
                     "timing": ("CUDA events around every launch on the launching stream, over a further "
                                "timed pass of the same steps (the step time is taken without them: an "
                                "event between two kernels serialises them)")},
        "kernels": {
            k: {"launches_per_step": v[1] / args.steps, "ms_per_step": round(v[0] / args.steps, 4)}
            for k, v in ktimes.items()},
        "dn_decode_roofline": {"achieved": round(dn_achieved, 1), "peak": peak, "unit": "GB/s",
                               "frac": round(dn_achieved / peak, 4),
                               "algorithmic_bytes_per_launch": B * DN_BYTES_TOKEN},
        "kernel_ms_per_step": round(step_kernel_ms, 4),
        "clocks": clk,
    }
    stack.close()
    torch.cuda.empty_cache()
    if (ws > 1 and not args.no_head_sharded) or args.head_sharded:
        line["head_sharded"] = bench_head_sharded(ctx, ws, rank, args)
    if not args.no_prefill:
        line["prefill_dn"] = bench_dn_prefill(ctx, ws, args.prefill_reps)
        line["prefill_gqa"] = bench_gqa_prefill(ctx, ws, args.prefill_reps)
    if not args.no_small:
        cpu = rank == 0 and ws == 1 and not args.no_cpu_baseline
        line["decode_config0"] = bench_config0(ctx, args.prefill_reps * 3, cpu=cpu)
        line["decode_config1"] = bench_config1(ctx, args.prefill_reps * 3, cpu=cpu)
    if rank == 0 and ws == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_sample(args.cpu_tokens)
        line["cpu_baseline"]["batch_parallel"] = cpu_sample_batch(args.cpu_tokens)
    if rank == 0:
        print(json.dumps(line), flush=True)
    ctx.close()
    if ws > 1:
        import torch.distributed as dist

        dist.destroy_process_group()


# ----------------------------------------------------------------------------
# prefill (workload 3): GQA causal prefill, 4 x 32768 tokens
# ----------------------------------------------------------------------------
def bench_gqa_prefill(ctx, ws, reps, B=4, T=32768):
    import numpy as np
    import torch

    import qora_mixer as qm
    from qora_mixer import inputs as I

    g = I.rng(3)
    pr = I.gqa_layer_params(g, T + 1)
    cos, sin = qm.rope_table(1.0e7, 64, T + 1)
    keep = [torch.from_numpy(pr["q_norm"]).cuda(), torch.from_numpy(pr["k_norm"]).cuda(),
            torch.from_numpy(cos).cuda(), torch.from_numpy(sin).cuda()]
    prm = qm.gqa_params(*keep)
    qg = I.device_normal_bf16((B, T, 16, 512), 0x51A3 * 10 + 1).view(torch.int16)
    kk = I.device_normal_bf16((B, T, 4, 256), 0x51A3 * 10 + 2).view(torch.int16)
    vv = I.device_normal_bf16((B, T, 4, 256), 0x51A3 * 10 + 3).view(torch.int16)
    K = torch.zeros(B, 4, T, 256, dtype=torch.int16, device="cuda")
    V = torch.zeros_like(K)
    kv = qm.KvCache(ctx, B, T, K, V)
    out = torch.empty(B, T, 16, 256, device="cuda")
    mx = qm.Mixer(ctx)
    stream = torch.cuda.current_stream()
    for _ in range(2):
        mx.gqa_prefill(prm, kv, T, qg, kk, vv, out)
    ctx.sync()
    barrier(ws)
    ctx.set_timing(True)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(reps):
        mx.gqa_prefill(prm, kv, T, qg, kk, vv, out)
    e1.record(stream)
    torch.cuda.synchronize()
    ctx.sync()  # a device-side timeout in the timed calls fails the record instead of timing it
    call_ms = max_over_ranks(e0.elapsed_time(e1) / reps, ws)
    att_ms, att_n = ctx.kernel_time("gqa_prefill_attn")
    prep_ms, _ = ctx.kernel_time("gqa_prefill_prep")
    ctx.set_timing(False)
    kv.close()
    flops = B * 16 * 4 * 256 * T * (T + 1) / 2  # QK^T + PV, causal
    att = att_ms / att_n
    peak, peak_kind = load_tensor_peak()
    tflops = flops / (att / 1e3) / 1e12
    del qg, kk, vv, out, K, V
    torch.cuda.empty_cache()
    return {"workload": f"GQA causal prefill, batch {B} x {T} tokens (workload 3)",
            "value": round(B * T * ws / (call_ms / 1e3), 1), "unit": "tok/s",
            "ms_per_call": round(call_ms, 3), "attn_ms": round(att, 3), "prep_ms": round(prep_ms / reps, 3),
            "roofline": {"bound": "tensor", "kernel": "gqa_prefill_attn", "achieved": round(tflops, 1),
                         "peak": peak, "peak_kind": peak_kind, "unit": "TFLOP/s",
                         "frac": round(tflops / peak, 4),
                         "algorithmic_flops_per_launch": flops,
                         "operands": "fp16 x fp16 -> f32 (tcgen05 kind::f16)"}}


# ----------------------------------------------------------------------------
# projections around the mixers (the next row after the mixers): all 32 layers'
# in_proj_qkv/a/b/z + out_proj (DeltaNet) and q/k/v/o_proj (GQA) for one decode
# token at batch B, Q4 or F16 weights, each layer's weights distinct (734 MB in
# Q4: larger than L2, so every step streams them from HBM)
# ----------------------------------------------------------------------------
PROJ_DN = [(2560, 8192), (2560, 32), (2560, 32), (2560, 4096), (4096, 2560)]
PROJ_GQA = [(2560, 8192), (2560, 1024), (2560, 1024), (4096, 2560)]


def bench_gemv(ctx, reps, batch=1, kind="q4"):
    """Each form of the step is captured once in a CUDA graph and replayed
    `reps` times between two events: fused (qm_gemv_multi over the weights
    that share x, 2 launches per layer), one launch per weight (152), and the
    32 in_proj_qkv / q_proj launches alone (the per-kernel roofline)."""
    import torch

    import qora_mixer as qm

    gen = torch.Generator(device="cuda").manual_seed(0x51A5)
    layers = [PROJ_GQA if layer % 4 == 3 else PROJ_DN for layer in range(32)]
    weights, keep, nbytes = [], [], 0
    for shapes in layers:
        lw = []
        for k, n in shapes:
            if kind == "q4":
                pk = torch.randint(0, 256, (k, n // 2), dtype=torch.uint8, device="cuda", generator=gen)
                sc = (torch.rand(k, n // 32, device="cuda", generator=gen) * 0.01).half().view(torch.int16)
                lw.append(qm.weight_q4(pk, sc))
                nbytes += pk.numel() + sc.numel() * 2
            else:
                w16 = (torch.randn(k, n, device="cuda", generator=gen) * 0.02).half().view(torch.int16)
                lw.append(qm.weight_f16(w16))
                nbytes += w16.numel() * 2
        weights.append(lw)
    xs = {k: torch.randn(batch, k, device="cuda", generator=gen) for k in (2560, 4096)}
    ys = {n: torch.empty(batch, n, device="cuda") for n in (8192, 32, 4096, 2560, 1024)}
    ys_b = torch.empty(batch, 32, device="cuda")  # in_proj_b beside in_proj_a
    mx = qm.Mixer(ctx)

    def fused():
        for lw, shapes in zip(weights, layers):
            outs = [ys[n] for _, n in shapes[:-1]]
            if len(outs) == 4:
                outs[2] = ys_b
            mx.gemv_multi(lw[:-1], xs[2560], outs)
            mx.gemv(lw[-1], xs[4096], ys[2560])

    def unfused():
        for lw, shapes in zip(weights, layers):
            for w, (k, n) in zip(lw, shapes):
                mx.gemv(w, xs[k], ys[n])

    def big_only():
        for lw in weights:
            mx.gemv(lw[0], xs[2560], ys[8192])

    side = torch.cuda.Stream()

    def timed(fn):
        n0 = ctx.launch_count()
        fn()  # warm-up and the launch count
        launches = ctx.launch_count() - n0
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        ctx.set_stream(side)
        try:
            with torch.cuda.graph(g, stream=side):
                fn()
        finally:
            ctx.set_stream(torch.cuda.current_stream())
        for _ in range(3):
            g.replay()
        stream = torch.cuda.current_stream()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        e0.record(stream)
        for _ in range(reps):
            g.replay()
        e1.record(stream)
        torch.cuda.synchronize()
        del g
        return e0.elapsed_time(e1) / reps, launches

    f_ms, f_n = timed(fused)
    u_ms, u_n = timed(unfused)
    b_ms, b_n = timed(big_only)
    n0 = ctx.launch_count()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        fused()
    e1.record()
    torch.cuda.synchronize()
    d_ms = e0.elapsed_time(e1) / reps
    peak, peak_kind = load_peaks()
    per_w = 0.5625 if kind == "q4" else 2.0
    big_gbs = 2560 * 8192 * per_w / (b_ms / b_n / 1e3) / 1e9
    ach = nbytes / (f_ms / 1e3) / 1e9
    del keep, weights
    torch.cuda.empty_cache()
    return {"metric": "mixer projections, 32 layers, one decode token", "workload":
            f"in_proj_qkv/a/b/z + out_proj x 24 DeltaNet layers, q/k/v/o_proj x 8 GQA layers, batch {batch}, "
            f"{kind.upper()} weights ({nbytes / 1e6:.0f} MB, larger than L2)",
            "value": round(batch / (f_ms / 1e3), 1), "unit": "tok/s", "ms_per_step": round(f_ms, 4),
            "launches_per_step": f_n, "timing": "CUDA graph of the step, replayed; CUDA events",
            "one_launch_per_weight": {"ms_per_step": round(u_ms, 4), "launches_per_step": u_n},
            "fused_without_graph_ms_per_step": round(d_ms, 4),
            "roofline": {"bound": "hbm", "kernel": "qm_gemv_kernel", "achieved": round(ach, 1), "peak": peak,
                         "peak_kind": peak_kind, "unit": "GB/s", "frac": round(ach / peak, 4),
                         "algorithmic_bytes_per_step": nbytes,
                         "in_proj_qkv_alone_gbs": round(big_gbs, 1),
                         "in_proj_qkv_alone_frac": round(big_gbs / peak, 4)}}


# ----------------------------------------------------------------------------
# prefill projections: the Q4 / F16 GEMM over a whole prompt (tensor cores)
# ----------------------------------------------------------------------------
GEMM_SHAPES = [("in_proj_qkv / q_proj", 2560, 8192), ("in_proj_z", 2560, 4096), ("out_proj / o_proj", 4096, 2560),
               ("k_proj / v_proj", 2560, 1024)]


def bench_gemm(ctx, reps, T=8192, kind="q4"):
    import torch

    import qora_mixer as qm

    gen = torch.Generator(device="cuda").manual_seed(0x51A7)
    mx = qm.Mixer(ctx)
    stream = torch.cuda.current_stream()
    peak, peak_kind = load_tensor_peak()
    rows, tot_flops, tot_ms = [], 0.0, 0.0
    for name, k, n in GEMM_SHAPES:
        if kind == "q4":
            pk = torch.randint(0, 256, (k, n // 2), dtype=torch.uint8, device="cuda", generator=gen)
            sc = (torch.rand(k, n // 32, device="cuda", generator=gen) * 0.01).half().view(torch.int16)
            w = qm.weight_q4(pk, sc)
        else:
            pk = (torch.randn(k, n, device="cuda", generator=gen) * 0.02).half().view(torch.int16)
            sc = None
            w = qm.weight_f16(pk)
        x = torch.randn(T, k, device="cuda", generator=gen).bfloat16().view(torch.int16)
        y = torch.empty(T, n, device="cuda")
        for _ in range(3):
            mx.gemm(w, x, y)
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(reps):
            mx.gemm(w, x, y)
        e1.record(stream)
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / reps
        flops = 2.0 * T * k * n
        rows.append({"weight": name, "k": k, "n": n, "ms": round(ms, 4),
                     "tflops": round(flops / (ms / 1e3) / 1e12, 1)})
        tot_flops += flops
        tot_ms += ms
        del pk, sc, w, x, y
    torch.cuda.empty_cache()
    ach = tot_flops / (tot_ms / 1e3) / 1e12
    wdesc = "Q4 weights dequantised" if kind == "q4" else "F16 weights rounded"
    return {"metric": f"prefill projections ({kind.upper()} GEMM)", "workload": f"{T} tokens x the 4B's "
            f"projection shapes, bf16 x, {wdesc} to bf16 in the kernel, f32 y", "per_shape": rows,
            "value": round(T / (tot_ms / 1e3), 1), "unit": "tok/s (the 4 shapes once each)",
            "roofline": {"bound": "tensor", "kernel": "qm_gemm_kernel", "achieved": round(ach, 1),
                         "peak": peak, "peak_kind": peak_kind, "unit": "TFLOP/s", "frac": round(ach / peak, 4)}}


# ----------------------------------------------------------------------------
# the decode loop's tail: lm_head over the tied embedding (248,320 x 2,560),
# penalties over a 512-token history, top-k / top-p sampling
# ----------------------------------------------------------------------------
VOCAB, HIDDEN = 248320, 2560


def bench_head(ctx, reps, batch=1, kind="q4"):
    import torch

    import qora_mixer as qm

    gen = torch.Generator(device="cuda").manual_seed(0x51A6)
    if kind == "q4":
        pk = torch.randint(0, 256, (VOCAB, HIDDEN // 2), dtype=torch.uint8, device="cuda", generator=gen)
        sc = (torch.rand(VOCAB, HIDDEN // 32, device="cuda", generator=gen) * 0.01).half().view(torch.int16)
        w = qm.weight_q4_rows(pk, sc)
        nbytes = pk.numel() + sc.numel() * 2
    else:
        e16 = (torch.randn(VOCAB, HIDDEN, device="cuda", generator=gen) * 0.02).half().view(torch.int16)
        w = qm.weight_f16_rows(e16)
        nbytes = e16.numel() * 2
    x = torch.randn(batch, HIDDEN, device="cuda", generator=gen)
    logits = torch.empty(batch, VOCAB, device="cuda")
    hist = 512
    toks = torch.randint(0, VOCAB, (batch, hist), dtype=torch.int32, device="cuda", generator=gen)
    lens = torch.full((batch,), hist, dtype=torch.int32, device="cuda")
    r = torch.rand(batch, device="cuda", generator=gen)
    ids = torch.empty(batch, dtype=torch.int32, device="cuda")
    mx = qm.Mixer(ctx)
    stream = torch.cuda.current_stream()

    def head():
        mx.gemv(w, x, logits)

    def tail():
        mx.penalize(logits, toks, lens, 1.1, 1.5, -1)
        mx.sample(logits, 0.7, 0.95, 20, r, ids)

    def timed(fn):
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(reps):
            fn()
        e1.record(stream)
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / reps

    h_ms = timed(head)
    t_ms = timed(tail)
    ctx.set_timing(True)
    timed(tail)
    pen_ms, pen_n = ctx.kernel_time("penalize")
    smp_ms, smp_n = ctx.kernel_time("sample")
    ctx.set_timing(False)
    s_ms = timed(lambda: (head(), tail()))
    gemm_ms = None
    if kind == "q4" and batch > 1:  # the same logits for all sequences at once on the tensor cores (bf16 x)
        xb = x.bfloat16().view(torch.int16)
        gemm_ms = timed(lambda: mx.gemm(w, xb, logits))
    peak, peak_kind = load_peaks()
    launches_lm = (batch + (0 if kind == "q4" else 1)) // (1 if kind == "q4" else 2)
    ach = nbytes * launches_lm / (h_ms / 1e3) / 1e9
    del w, logits
    torch.cuda.empty_cache()
    return {"metric": "decode tail: lm_head + penalties + sampling", "workload":
            f"lm_head over the tied embedding {VOCAB} x {HIDDEN} ({kind.upper()}, {nbytes / 1e6:.0f} MB), "
            f"batch {batch}; repetition + presence penalties over {hist} tokens; top_k 20, top_p 0.95, T 0.7",
            "value": round(batch / (s_ms / 1e3), 1), "unit": "tok/s", "ms_per_step": round(s_ms, 4),
            "lm_head_ms": round(h_ms, 4), "penalize_ms": round(pen_ms / pen_n, 4),
            "sample_ms": round(smp_ms / smp_n, 4), "tail_ms": round(t_ms, 4),
            "lm_head_gemm_ms": round(gemm_ms, 4) if gemm_ms is not None else None,
            "roofline": {"bound": "hbm", "kernel": "qm_rows_kernel", "achieved": round(ach, 1), "peak": peak,
                         "peak_kind": peak_kind, "unit": "GB/s", "frac": round(ach / peak, 4),
                         "algorithmic_bytes_per_step": nbytes * launches_lm}}


# ----------------------------------------------------------------------------
# prefill (workload 2): DeltaNet chunked prefill, 8 x 8192 tokens, chunk 64
# ----------------------------------------------------------------------------
def bench_dn_prefill(ctx, ws, reps, B=8, T=8192):
    import torch

    import qora_mixer as qm
    from qora_mixer import inputs as I

    g = I.rng(2)
    p = I.dn_layer_params(g)
    keep = [torch.from_numpy(p[k]).cuda() for k in ("conv_w", "a_log", "dt_bias", "norm_gamma")]
    prm = qm.dn_params(*keep)
    qkv = I.device_normal_bf16((B, T, 8192), 0x51A2 * 10 + 1).view(torch.int16)
    a = I.device_normal_f32((B, T, 32), 0x51A2 * 10 + 2)
    bb = I.device_normal_f32((B, T, 32), 0x51A2 * 10 + 3)
    st = qm.DnState(ctx, B)
    y = torch.empty(B, T, 32, 128, device="cuda")
    mx = qm.Mixer(ctx)
    stream = torch.cuda.current_stream()
    for _ in range(2):
        st.reset()
        mx.dn_prefill(prm, st, T, qkv, a, bb, y)
    ctx.sync()
    barrier(ws)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    tot = 0.0
    for _ in range(reps):
        st.reset()  # each call is a fresh 8192-token prompt
        e0.record(stream)
        mx.dn_prefill(prm, st, T, qkv, a, bb, y)
        e1.record(stream)
        torch.cuda.synchronize()
        tot += e0.elapsed_time(e1)
    ctx.sync()  # a device-side timeout in the timed calls fails the record instead of timing it
    call_ms = max_over_ranks(tot / reps, ws)
    # the per-kernel split from the same calls again with an event pair around
    # every launch (events between the call's kernels would add gaps to call_ms)
    ctx.set_timing(True)
    for _ in range(reps):
        st.reset()
        mx.dn_prefill(prm, st, T, qkv, a, bb, y)
    torch.cuda.synchronize()
    ctx.sync()
    loc_ms, k_n = ctx.kernel_time("dn_chunk_local")
    sta_ms, _ = ctx.kernel_time("dn_chunk_state")
    prep_ms, _ = ctx.kernel_time("dn_prefill_prep")
    ctx.set_timing(False)
    st.close()
    flops = B * 32 * (T // 64) * (10 * 64 * 64 * 128 + 6 * 64 * 128 * 128 + 64 ** 3)
    executed = B * 32 * (T // 64) * 2 * (3 * 128 * 64 * 128 + 3 * 128 * 64 * 64 * 2 + 2 * 128 * 64 * 128
                                         + 3 * 128 * 64 * 64 + 3 * 128 * 128 * 64)
    bytes_alg = B * T * (8192 * 2 + 64 * 4 + 32 * 128 * 4)
    peak_t, peak_kind = load_tensor_peak()
    peak_b, _ = load_peaks()
    kk = (loc_ms + sta_ms) / k_n  # the two chunk kernels: the tensor-core part of the call
    del qkv, a, bb, y
    torch.cuda.empty_cache()
    return {"workload": f"DeltaNet chunked prefill, batch {B} x {T} tokens, chunk 64 (workload 2)",
            "value": round(B * T * ws / (call_ms / 1e3), 1), "unit": "tok/s",
            "ms_per_call": round(call_ms, 3), "chunk_kernels_ms": round(kk, 3),
            "chunk_local_ms": round(loc_ms / k_n, 3), "chunk_state_ms": round(sta_ms / k_n, 3),
            "prep_ms": round(prep_ms / reps, 3),
            "roofline": {"bound": "tensor (north-star target) / hbm",
                         "kernel": "dn_chunk_local + dn_chunk_state",
                         "achieved_tflops": round(flops / (kk / 1e3) / 1e12, 1), "peak_tflops": peak_t,
                         "peak_kind": peak_kind,
                         "frac_tensor": round(flops / (kk / 1e3) / 1e12 / peak_t, 4),
                         "executed_tflops": round(executed / (kk / 1e3) / 1e12, 1),
                         "achieved_gbs_call": round(bytes_alg / (call_ms / 1e3) / 1e9, 1), "peak_gbs": peak_b,
                         "frac_hbm_call": round(bytes_alg / (call_ms / 1e3) / 1e9 / peak_b, 4),
                         "algorithmic_flops": flops, "algorithmic_bytes": bytes_alg,
                         "operands": "fp16 hi/lo compensated (3 MMAs) intra-chunk, fp16 state products"}}


# ----------------------------------------------------------------------------
# workloads 0 and 1: single-layer decode at batch 1
# ----------------------------------------------------------------------------
CFG0_BYTES_TOKEN = 2 * 32 * 128 * 128 * 4 + 2 * 8192 * 3 * 4 + 8192 * 4 + 2 * 32 * 4 + 32 * 128 * 4
CFG1_L = 4096


def cfg1_bytes(L=CFG1_L):
    """K/V of L cached positions plus the new one read, the new row appended, q/gate, k, v in, out."""
    return 2 * 4 * (L + 1) * 256 * 2 + 2 * 4 * 256 * 2 + (16 * 512 + 2 * 4 * 256) * 4 + 16 * 256 * 4


def _graph_time(ctx, fn, reps):
    """fn captured once in a CUDA graph on a side stream, replayed reps times between two events."""
    import torch

    side = torch.cuda.Stream()
    fn()  # warm-up (grows any workspace outside the capture)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    ctx.set_stream(side)
    try:
        with torch.cuda.graph(g, stream=side):
            fn()
    finally:
        ctx.set_stream(torch.cuda.current_stream())
    for _ in range(3):
        g.replay()
    stream = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    e0.record(stream)
    for _ in range(reps):
        g.replay()
    e1.record(stream)
    torch.cuda.synchronize()
    del g
    return e0.elapsed_time(e1) / reps


def bench_config0(ctx, reps, cpu=True):
    """Workload 0: one DeltaNet layer, batch 1, 256 sequential tokens from a
    zero state.  Timed two ways: qm_dn_decode_seq (the 256 tokens in one
    launch, the 2 MiB state in registers throughout) and 256 qm_dn_decode
    calls (one per token, as a decode loop issues them) captured in a CUDA
    graph.  The algorithmic bytes are the per-token traffic of the reference
    algorithm with the state in memory (state read + write, conv history,
    inputs, output): with the state on chip, the GB/s figure is effective."""
    import numpy as np
    import torch

    import qora_mixer as qm
    from qora_mixer import inputs as I

    T = 256
    g = I.rng(0)
    p = I.dn_layer_params(g)
    toks = I.dn_token_inputs(g, T, 1)
    keep = [torch.from_numpy(p[k]).cuda() for k in ("conv_w", "a_log", "dt_bias", "norm_gamma")]
    prm = qm.dn_params(*keep)
    qkv, a, b = (torch.from_numpy(np.ascontiguousarray(toks[k])).cuda() for k in ("qkv", "a", "b"))
    st = qm.DnState(ctx, 1)
    y = torch.empty(1, T, 32, 128, device="cuda")
    yd = torch.empty(1, 32, 128, device="cuda")
    mx = qm.Mixer(ctx)
    stream = torch.cuda.current_stream()
    for _ in range(3):
        st.reset()
        mx.dn_decode_seq(prm, st, T, qkv, a, b, y)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    tot = 0.0
    for _ in range(reps):
        st.reset()
        e0.record(stream)
        mx.dn_decode_seq(prm, st, T, qkv, a, b, y)
        e1.record(stream)
        torch.cuda.synchronize()
        tot += e0.elapsed_time(e1)
    seq_ms = tot / reps
    tok_views = [(qkv[:, t], a[:, t], b[:, t]) for t in range(T)]

    def per_token():
        for q_t, a_t, b_t in tok_views:
            mx.dn_decode(prm, st, q_t, a_t, b_t, yd)

    st.reset()
    loop_ms = _graph_time(ctx, per_token, max(2, reps // 2))
    st.close()
    peak, peak_kind = load_peaks()
    alg = CFG0_BYTES_TOKEN * T
    ach = alg / (seq_ms / 1e3) / 1e9
    ach_loop = alg / (loop_ms / 1e3) / 1e9
    rec = {"workload": "DeltaNet layer decode, batch 1, 256 sequential tokens (workload 0)",
           "value": round(T / (seq_ms / 1e3), 1), "unit": "tok/s", "ms_per_256_tokens": round(seq_ms, 4),
           "path": "qm_dn_decode_seq: one launch, state on chip",
           "per_token_calls": {"path": "256 qm_dn_decode launches in a CUDA graph",
                               "value": round(T / (loop_ms / 1e3), 1), "unit": "tok/s",
                               "ms_per_256_tokens": round(loop_ms, 4),
                               "effective_gbs": round(ach_loop, 1), "frac": round(ach_loop / peak, 4)},
           "roofline": {"bound": "hbm (effective: the state stays on chip)", "kernel": "dn_decode_seq_kernel",
                        "achieved": round(ach, 1), "peak": peak, "peak_kind": peak_kind, "unit": "GB/s",
                        "frac": round(ach / peak, 4), "algorithmic_bytes_per_token": CFG0_BYTES_TOKEN}}
    if cpu:
        from oracle import oracle as orc

        c = orc.cfg_4b()
        ost = orc.DnState(c)
        avx = orc.has_avx512()
        t0 = time.perf_counter()
        for t in range(T):
            orc.dn_decode(c, ost, toks["qkv"][0, t], toks["a"][0, t], toks["b"][0, t], p["conv_w"],
                          p["a_log"], p["dt_bias"], use_avx512=avx)
        dt = time.perf_counter() - t0
        rec["cpu_baseline"] = {"value": round(T / dt, 2), "unit": "tok/s", "cores": 1, "kind": "port",
                               "sample": "the same 256 tokens through the CPU restatement, heads serial "
                                         "(gemv.rs:817) with the AVX-512 head update (simd.rs:292-362)"
                                         if avx else "the same 256 tokens, scalar head update (gemv.rs:836-861)"}
    return rec


def bench_config1(ctx, reps, cpu=True, ncache=24):
    """Workload 1: one GQA layer decode, batch 1, 4096 cached bf16 positions,
    new token at 4096.  One 16.8 MB cache fits in L2, so the timed calls
    rotate over `ncache` distinct caches (403 MB at 24): each call reads its
    K/V from HBM.  The calls, one per cache, are captured in a CUDA graph and
    replayed; every call appends at position 4096 of its cache."""
    import torch

    import qora_mixer as qm
    from qora_mixer import inputs as I

    L, cap = CFG1_L, CFG1_L + 8
    g = I.rng(1)
    pr = I.gqa_layer_params(g, cap + 1)
    cos, sin = qm.rope_table(1.0e7, 64, cap + 1)
    keep = [torch.from_numpy(pr["q_norm"]).cuda(), torch.from_numpy(pr["k_norm"]).cuda(),
            torch.from_numpy(cos).cuda(), torch.from_numpy(sin).cuda()]
    prm = qm.gqa_params(*keep)
    caches = []
    for i in range(ncache):
        K = I.device_normal_bf16((1, 4, cap, 256), 0x51A1 * 100 + 2 * i).view(torch.int16)
        V = I.device_normal_bf16((1, 4, cap, 256), 0x51A1 * 100 + 2 * i + 1).view(torch.int16)
        kv = qm.KvCache(ctx, 1, cap, K, V)
        kv.seq_len = L
        caches.append((kv, K, V))
    tok = I.gqa_token_inputs(g, 1)
    ins = [torch.from_numpy(tok[k]).cuda() for k in ("q_gate", "k_new", "v_new")]
    out = torch.empty(1, 16, 256, device="cuda")
    mx = qm.Mixer(ctx)

    def calls():
        for kv, _, _ in caches:
            kv.seq_len = L
            mx.gqa_decode(prm, kv, *ins, out)

    n0 = ctx.launch_count()
    calls()
    launches = (ctx.launch_count() - n0) // ncache
    ms = _graph_time(ctx, calls, max(10, reps * 5)) / ncache
    for kv, _, _ in caches:
        kv.close()
    del caches
    torch.cuda.empty_cache()
    peak, peak_kind = load_peaks()
    alg = cfg1_bytes(L)
    ach = alg / (ms / 1e3) / 1e9
    rec = {"workload": "GQA layer decode, batch 1, 4096 cached positions (workload 1)",
           "value": round(1 / (ms / 1e3), 1), "unit": "tok/s", "us_per_call": round(ms * 1e3, 3),
           "launches_per_call": launches,
           "l2": f"{ncache} distinct caches rotated ({ncache * alg / 1e6:.0f} MB > L2)",
           "timing": "one call per cache captured in a CUDA graph, replayed; CUDA events",
           "roofline": {"bound": "hbm",
                        "kernel": ("gqa_fused (q norm + RoPE, split-KV attention, cluster merge, gate: "
                                   "one launch)" if launches == 1 else
                                   "gqa_prep + gqa_attn + gqa_combine (whole call)"),
                        "achieved": round(ach, 1), "peak": peak, "peak_kind": peak_kind, "unit": "GB/s",
                        "frac": round(ach / peak, 4), "algorithmic_bytes_per_call": alg}}
    if cpu:
        import numpy as np

        from oracle import oracle as orc

        c = orc.cfg_4b()
        kb = I.f32_to_bf16_bits(g.standard_normal((L, 4 * 256), dtype=np.float32))
        vb = I.f32_to_bf16_bits(g.standard_normal((L, 4 * 256), dtype=np.float32))
        okv = orc.KvCache(c, cap + 1, I.bf16_bits_to_f32(kb), I.bf16_bits_to_f32(vb))
        orc.set_num_threads(host_threads())
        n = 20
        t0 = time.perf_counter()
        for _ in range(n):
            okv.seq_len[0] = L
            orc.gqa_decode(c, okv, tok["q_gate"][0], tok["k_new"][0], tok["v_new"][0], pr["q_norm"],
                           pr["k_norm"], cos, sin)
        dt = (time.perf_counter() - t0) / n
        rec["cpu_baseline"] = {"value": round(1 / dt, 2), "unit": "tok/s",
                               "cores": min(16, orc.num_threads()), "kind": "port",
                               "sample": f"{n} calls of the CPU restatement at L=4096, the 16 heads on an "
                                         "OpenMP pool as rayon runs them (gemv.rs:963)"}
    return rec


# ----------------------------------------------------------------------------
# CPU restatement on a bounded sample (reference arm and cpu_baseline)
# ----------------------------------------------------------------------------
class CpuStack:
    """One sequence of workload 4 on the CPU restatement: 24 DeltaNet states and
    8 GQA layers; the 8 layers' caches share one storage block (same shape and
    traffic per layer, 1/8 of the host memory)."""

    def __init__(self, ntok):
        import numpy as np

        from oracle import oracle as orc
        from qora_mixer import inputs as I

        self.orc, self.I = orc, I
        self.c = orc.cfg_4b()
        g = I.rng(4, stream=99)
        cap = CTX + ntok + 4
        self.cos, self.sin = orc.rope_table(1.0e7, 64, cap + 1)
        self.dn = []
        for li in range(24):
            p = I.dn_layer_params(g)
            st = orc.DnState(self.c)
            st.s[:] = (g.standard_normal(st.s.shape, dtype=np.float32) * np.float32(0.02))
            st.conv_buf[:] = (g.standard_normal(st.conv_buf.shape, dtype=np.float32) * np.float32(0.02))
            tok = I.dn_token_inputs(g, 1, 1)
            self.dn.append((p, st, tok))
        kb = I.f32_to_bf16_bits(g.standard_normal((CTX, 4, 256), dtype=np.float32) * np.float32(0.02))
        vb = I.f32_to_bf16_bits(g.standard_normal((CTX, 4, 256), dtype=np.float32) * np.float32(0.02))
        self.kv = orc.KvCache(self.c, cap, I.bf16_bits_to_f32(kb).reshape(CTX, -1),
                              I.bf16_bits_to_f32(vb).reshape(CTX, -1))
        self.att = []
        for li in range(8):
            pr = I.gqa_layer_params(g, cap + 1)
            tok = I.gqa_token_inputs(g, 1)
            self.att.append((pr, tok))
        self.avx = orc.has_avx512()

    def clone(self):
        """An independent copy (own states and cache) for another sequence."""
        import copy

        o = copy.copy(self)
        o.dn = [(p, st.copy(), tok) for (p, st, tok) in self.dn]
        kv = self.orc.KvCache.__new__(self.orc.KvCache)
        kv.k, kv.v, kv.seq_len = self.kv.k.copy(), self.kv.v.copy(), self.kv.seq_len.copy()
        o.kv = kv
        return o

    def token(self):
        """One decode token through all 32 layers (3 DeltaNet + 1 GQA, x8)."""
        orc = self.orc
        di = ai = 0
        for kind in LAYERS:
            if kind == "dn":
                p, st, tok = self.dn[di]
                di += 1
                orc.dn_decode(self.c, st, tok["qkv"][0, 0], tok["a"][0, 0], tok["b"][0, 0],
                              p["conv_w"], p["a_log"], p["dt_bias"], use_avx512=self.avx,
                              z=tok["z"][0, 0], norm_gamma=p["norm_gamma"])
            else:
                pr, tok = self.att[ai]
                ai += 1
                L = int(self.kv.seq_len[0])
                orc.gqa_decode(self.c, self.kv, tok["q_gate"][0], tok["k_new"][0], tok["v_new"][0],
                               pr["q_norm"], pr["k_norm"], self.cos, self.sin)
                self.kv.seq_len[0] = L  # all 8 layers attend over the same 32768+1 positions


def host_threads():
    """Every core this process may run on (torchrun sets OMP_NUM_THREADS=1 per rank)."""
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def cpu_sample(ntok):
    from oracle import oracle as orc

    orc.set_num_threads(host_threads())
    cs = CpuStack(ntok)
    cs.token()  # warm
    t0 = time.perf_counter()
    for _ in range(ntok):
        cs.token()
    dt = time.perf_counter() - t0
    return {"value": round(ntok / dt, 4), "unit": UNIT, "cores": min(16, orc.num_threads()),
            "kind": "port",
            "sample": (f"{ntok} decode tokens of one sequence through all 32 mixer layers at context "
                       f"{CTX}; GQA heads on an OpenMP pool (rayon over 16 heads, gemv.rs:963), "
                       "DeltaNet heads serial with the AVX-512 update (gemv.rs:817, simd.rs:292)"),
            "cpu": cpu_model()}


def cpu_sample_batch(ntok, nseq=None):
    """Independent sequences across the host cores, one per core, each run as
    the reference runs a sequence but with its own OpenMP team of one: the
    throughput a CPU host gets by batching sequences the way the GPU does."""
    from concurrent.futures import ThreadPoolExecutor

    from oracle import oracle as orc

    cores = host_threads()
    nseq = nseq or min(16, cores)
    orc.set_num_threads(1)
    base = CpuStack(ntok + 1)
    stacks = [base] + [base.clone() for _ in range(nseq - 1)]

    def run(cs, n=ntok):
        for _ in range(n):
            cs.token()

    with ThreadPoolExecutor(max_workers=nseq) as ex:
        list(ex.map(lambda cs: run(cs, 1), stacks))  # warm
        t0 = time.perf_counter()
        list(ex.map(run, stacks))
        dt = time.perf_counter() - t0
    orc.set_num_threads(cores)
    return {"value": round(nseq * ntok / dt, 4), "unit": UNIT, "cores": nseq, "kind": "port",
            "sample": (f"{nseq} independent sequences in parallel, one per core, {ntok} decode tokens each "
                       f"through all 32 mixer layers at context {CTX}; per sequence the reference's "
                       "arithmetic (DeltaNet heads serial with the AVX-512 update, GQA heads serial)"),
            "cpu": cpu_model()}


def cpu_model():
    try:
        for ln in open("/proc/cpuinfo"):
            if ln.startswith("model name"):
                return ln.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def decode_config(ws, B, ctx_len):
    """The decode workload's config, the same in both arms: the reference arm
    times a bounded sample of it (its cpu_baseline.sample says which)."""
    return {"workload": WORKLOAD if ctx_len == CTX and B == B_PER_GPU else
            f"mixer-stack decode: 32 layers, ctx {ctx_len}, batch {B} (reduced case)",
            "global_batch": B * ws, "batch_per_gpu": B,
            "context": ctx_len, "layers": "24 DeltaNet + 8 GQA",
            "parallelism": f"sequence-sharded x{ws}, no collective",
            "l2": f"inputs larger than L2 ({attn_bytes(B, ctx_len) * 8 / 1e9:.1f} GB of KV per GPU)"}


def run_reference(args):
    ws, rank, local = dist_env()
    if rank != 0:
        return
    from oracle import oracle as orc

    per_step = args.cpu_tokens_per_step
    orc.set_num_threads(host_threads())
    cs = CpuStack(per_step * (args.warmup + args.steps) + 1)
    for _ in range(args.warmup):
        for _ in range(per_step):
            cs.token()
    times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        for _ in range(per_step):
            cs.token()
        times.append(time.perf_counter() - t0)
    tot = sum(times)
    value = per_step * args.steps / tot
    sample = (f"{per_step} decode token(s) of one sequence per step through all 32 mixer layers at "
              f"context {CTX} (the reference processes sequences one at a time, so its rate over the "
              f"{B_PER_GPU * ws} sequences is this one's); GQA heads on an "
              "OpenMP pool as rayon does (gemv.rs:963), DeltaNet heads serial with the AVX-512 "
              "head update (gemv.rs:817, simd.rs:292-362)")
    line = {
        "impl": "reference", "metric": METRIC, "value": round(value, 4), "unit": UNIT,
        "n_gpus": ws, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(tot / args.steps * 1e3, 3), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded)",
        "config": decode_config(ws, B_PER_GPU, CTX),
        "cpu_baseline": {"value": round(value, 4), "unit": UNIT, "cores": min(16, orc.num_threads()),
                         "kind": "port", "sample": sample, "cpu": cpu_model()},
        "e2e": {"value": round(value, 4), "unit": UNIT, "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--strong", action="store_true", help="64 sequences in total instead of per GPU")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true", help="skip the host-buffer (e2e) pass")
    ap.add_argument("--no-prefill", action="store_true", help="skip the prefill measurements")
    ap.add_argument("--prefill-reps", type=int, default=3)
    ap.add_argument("--no-small", action="store_true", help="skip the workload 0 / 1 records")
    ap.add_argument("--small-only", action="store_true",
                    help="time workloads 0 and 1 alone (batch-1 single-layer decode); prints their records")
    ap.add_argument("--head-sharded", action="store_true",
                    help="also time the head-sharded variant at N=1 (always on for N>1)")
    ap.add_argument("--no-head-sharded", action="store_true")
    ap.add_argument("--gather", choices=["peer", "nccl"], default="peer",
                    help="head-sharded all-gather: peer-memory kernel (qm_comm_enable_peer) or NCCL")
    ap.add_argument("--batch", type=int, default=B_PER_GPU, help="sequences per GPU")
    ap.add_argument("--context", type=int, default=CTX, help="cached positions per sequence")
    ap.add_argument("--cpu-tokens", type=int, default=4)
    ap.add_argument("--cpu-tokens-per-step", type=int, default=1)
    ap.add_argument("--prefill-only", choices=["gqa", "dn"],
                    help="time one prefill alone (profiling small cases); prints its record")
    ap.add_argument("--prefill-batch", type=int, help="with --prefill-only: sequences")
    ap.add_argument("--prefill-len", type=int, help="with --prefill-only: tokens per sequence")
    ap.add_argument("--gemv-only", choices=["q4", "f16"],
                    help="time the 32 layers' mixer projections (Q4 / F16 weight GEMV) alone")
    ap.add_argument("--gemv-batch", type=int, default=1, help="with --gemv-only / --head-only: sequences per step")
    ap.add_argument("--gemm-only", nargs="?", const="q4", choices=["q4", "f16"],
                    help="time the prefill projection GEMM alone (Q4 weights unless f16 is given)")
    ap.add_argument("--head-only", choices=["q4", "f16"],
                    help="time the decode tail alone: lm_head, penalties and sampling")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.gemm_only:
        import torch

        import qora_mixer as qm

        torch.cuda.set_device(0)
        ctx = qm.Ctx(0, stream=torch.cuda.current_stream())
        print(json.dumps(bench_gemm(ctx, args.steps, args.prefill_len or 8192, args.gemm_only)), flush=True)
        ctx.close()
        return
    if args.head_only:
        import torch

        import qora_mixer as qm

        torch.cuda.set_device(0)
        ctx = qm.Ctx(0, stream=torch.cuda.current_stream())
        print(json.dumps(bench_head(ctx, args.steps, args.gemv_batch, args.head_only)), flush=True)
        ctx.close()
        return
    if args.gemv_only:
        import torch

        import qora_mixer as qm

        torch.cuda.set_device(0)
        ctx = qm.Ctx(0, stream=torch.cuda.current_stream())
        print(json.dumps(bench_gemv(ctx, args.steps, args.gemv_batch, args.gemv_only)), flush=True)
        ctx.close()
        return
    if args.small_only:
        import torch

        import qora_mixer as qm

        torch.cuda.set_device(0)
        ctx = qm.Ctx(0, stream=torch.cuda.current_stream())
        rec = {"decode_config0": bench_config0(ctx, args.steps, cpu=not args.no_cpu_baseline),
               "decode_config1": bench_config1(ctx, args.steps, cpu=not args.no_cpu_baseline)}
        print(json.dumps(rec), flush=True)
        ctx.close()
        return
    if args.prefill_only:
        import torch

        import qora_mixer as qm

        torch.cuda.set_device(0)
        ctx = qm.Ctx(0, stream=torch.cuda.current_stream())
        fn = bench_gqa_prefill if args.prefill_only == "gqa" else bench_dn_prefill
        kw = {}
        if args.prefill_batch:
            kw["B"] = args.prefill_batch
        if args.prefill_len:
            kw["T"] = args.prefill_len
        print(json.dumps(fn(ctx, 1, args.prefill_reps, **kw)), flush=True)
        ctx.close()
        return
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
