#!/usr/bin/env python
"""Benchmark of the weight-streaming decode path (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--workload NAME]

Headline workload: Nvfp4Gemv, R=1, K=8192, N=4096.  A step is one
replay of a CUDA graph holding `calls` back-to-back op calls that rotate over COPIES distinct
weight sets (>= 3x the 126 MB L2, so every call streams its weights from HBM).  `value` is the
achieved HBM throughput (algorithmic bytes / device time) summed over ranks; with N > 1 every
rank runs its own replica (the GEMV does not shard) and the time is the max over ranks.

Other configs of BASELINE.json are measured after the headline and reported under
"configs_measured" (µs/call, GB/s, fraction of the measured HBM peak).

--impl reference times the reference's CPU implementation of the same workload (the torch
restatement in oracle/, all host threads) on a bounded sample per step.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "µs/call and achieved HBM GB/s (% of B200 peak) for quant GEMV/MoE at R=1,8"
L2_BYTES = 126 * 1024 * 1024


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


# ------------------------------------------------------------------------------------------------
# workloads: name -> builder(device, copies) returning a dict
#   calls[i]()         one op call on weight copy i
#   bytes              algorithmic bytes per call (weights + scales + activations + outputs)
#   kernels            kernels launched per call
#   h2d / d2h          bytes of the per-call input / result for the end-to-end measurement
#   e2e(i, xh, yh)     one end-to-end call from pinned host buffers
#   cpu(sample)        oracle run on a bounded sample; returns bytes processed
# ------------------------------------------------------------------------------------------------
def _gemv_workload(kind, R, N, K, iq2=0):
    from nemotron_ops_b200 import ops
    from nemotron_ops_b200 import workloads as W

    def build(device, copies):
        sets = []
        for c in range(copies):
            if kind == "nvfp4":
                d = W.nvfp4_gemv(R=R, N=N, K=K, seed=c, device=device)
            elif kind == "q8":
                d = W.q8_gemv(R=R, N=N, K=K, seed=c, device=device)
            else:
                d = W.q4_gemv(R=R, N=N, K=K, iq2=iq2, seed=c, device=device)
            if c > 0:
                d["x"] = sets[0]["x"]
            sets.append(d)
        x = sets[0]["x"]

        def op(d, x):
            if kind == "nvfp4":
                return ops.Nvfp4Gemv(x, d["w"], d["w_scale"], d["g"])
            if kind == "q8":
                return ops.Q8Gemv(x, d["B"], d["scales"])
            return ops.Q4Gemv(x, d["B"], d["scales"], iq2=iq2)

        d0 = sets[0]
        if kind == "nvfp4":
            wbytes = d0["w"].numel() + d0["w_scale"].numel() + 4
        else:
            wbytes = d0["B"].numel() + d0["scales"].numel() * 2
        nbytes = wbytes + R * K * 2 + R * N * 2
        calls = [(lambda d=d: op(d, x)) for d in sets]
        pin = str(device) != "cpu"
        xh = x.cpu().pin_memory() if pin else x
        yh = torch.empty(R, N, dtype=torch.bfloat16).pin_memory() if pin else None
        xd = torch.empty_like(x)

        def e2e(i):
            ops.copy_async(xd, xh)
            y = op(sets[i], xd)
            ops.copy_async(yh, y)

        def cpu(sample_rows):
            import oracle as O
            c = {k: (v.cpu() if isinstance(v, torch.Tensor) else v) for k, v in d0.items()}
            n = min(N, sample_rows)
            if kind == "nvfp4":
                O.nvfp4_gemv(c["x"], c["w"][:n], c["w_scale"][:n], c["g"], fp32=True)
            elif kind == "q8":
                O.q8_gemv(c["x"], c["B"][:n], c["scales"][:n], fp32=True)
            else:
                O.q4_gemv(c["x"], c["B"][:n], c["scales"][:n], iq2=iq2, fp32=True)
            return nbytes * n / N

        dt = {"nvfp4": "f16", "q8": "f32" if R == 1 else "bf16", "q4": "f32" if (R == 1 and iq2 == 0) else "bf16"}[kind]
        return dict(calls=calls, bytes=nbytes, kernels=1, h2d=R * K * 2, d2h=R * N * 2, e2e=e2e, cpu=cpu,
                    cpu_sample=N, dtype=dt, kernel="gemv_q8_r1_kernel" if (kind == "q8" and R == 1) else
                    "gemv_nvfp4_r1_kernel" if (kind == "nvfp4" and R == 1) else
                    "gemv_q4_r1_kernel" if (kind == "q4" and R == 1 and iq2 == 0) else
                    "gemv_iq2n_r1_kernel" if (kind == "q4" and R == 1 and iq2 == 2) else "gemv_tc_kernel")
    return build


def _moe_workload(op_name, R, iq2=0, E=304, I=2304, topk=8, route=False):
    """One MoE layer per call; with route, MoeRoute and the layer run back to back in the same
    captured sequence (router gate weights, one distinct copy per expert set)."""
    from nemotron_ops_b200 import ops
    from nemotron_ops_b200 import workloads as W

    def build(device, copies):
        r = W.moe_route(R=R, E=E, K=4096, seed=0, device=device)
        if str(device) == "cpu":  # CPU reference arm: routing from the oracle
            import oracle as O
            idx, w, _ = O.moe_route(r["x"], r["gate_w"], r["bias"], topk, 5.0)
        else:
            idx, w, _ = ops.MoeRoute(r["x"], r["gate_w"], r["bias"], topk, 5.0)
        z = W.moe_latent(R=R, device=device)
        sets = [W.moe_experts(E=E, I=I, iq2=iq2, seed=10 + c, device=device) for c in range(copies)]
        uniq = len(set(idx.reshape(-1).tolist()))
        e0 = sets[0]
        per_expert = sum(e0[k][0].numel() * e0[k].element_size() for k in ("fc1_w", "fc1_s", "fc2_w", "fc2_s"))
        nbytes = uniq * per_expert + R * 1024 * 2 + R * topk * 8 + R * 1024 * 2
        if route:  # + gate weights, bias, x, scores, idx/w
            nbytes += E * 4096 * 2 + E * 4 + R * 4096 * 2 + R * E * 4 + R * topk * 8
            for d in sets:
                d["gate_w"] = r["gate_w"].clone()

        def op(d, zz):
            ii, ww = idx, w
            if route:
                ii, ww, _ = ops.MoeRoute(r["x"], d["gate_w"], r["bias"], topk, 5.0)
            a = [zz, ii, ww, d["fc1_w"], d["fc1_s"], d["fc2_w"], d["fc2_s"]]
            if op_name == "MoeDecode":
                return ops.MoeDecode(*a, topk=topk)[0]
            return ops.MoeVerify(*a, topk=topk, iq2=iq2)[0]

        calls = [(lambda d=d: op(d, z)) for d in sets]
        pin = str(device) != "cpu"
        zh = z.cpu().pin_memory() if pin else z
        yh = torch.empty(R, 1024, dtype=torch.bfloat16).pin_memory() if pin else None
        zd = torch.empty_like(z)

        def e2e(i):
            ops.copy_async(zd, zh)
            y = op(sets[i], zd)
            ops.copy_async(yh, y)

        def cpu(sample_pairs):
            import oracle as O
            n = max(1, min(R * topk, sample_pairs))
            c = [t.cpu() for t in (z, idx, w, e0["fc1_w"], e0["fc1_s"], e0["fc2_w"], e0["fc2_s"])]
            rows = max(1, n // topk)
            args = [c[0][:rows], c[1][:rows], c[2][:rows]] + c[3:]
            if route:
                O.moe_route(r["x"][:rows].cpu(), r["gate_w"].cpu(), r["bias"].cpu(), topk, 5.0)
            if op_name == "MoeDecode":
                O.moe_decode(*args, topk=topk, fp32=True)
            else:
                O.moe_verify(*args, topk=topk, iq2=iq2, fp32=True)
            return nbytes * rows / R

        # launches per call: MoeDecode fc1 + fc2 (finalize fused); MoeVerify fc1, fc2, finalize
        # (+ router logits, selection)
        kern = (2 if op_name == "MoeDecode" else 3) + (2 if route else 0)
        main_kernel = ("moe_stream_fc1_kernel + moe_stream_fc2_kernel" if op_name == "MoeDecode" else
                       "moe_vstream_kernel")
        return dict(calls=calls, bytes=nbytes, kernels=kern, h2d=R * 1024 * 2,
                    d2h=R * 1024 * 2, e2e=e2e, cpu=cpu, cpu_sample=R * topk, dtype="f32" if op_name == "MoeDecode"
                    else "bf16", unique_experts=uniq, kernel=main_kernel)
    return build


def _route_workload(R, E=304, K=4096, topk=8):
    """MoeRoute alone: the gate weights [E, K] bf16 are the stream (2.5 MB per call)."""
    from nemotron_ops_b200 import ops
    from nemotron_ops_b200 import workloads as W

    def build(device, copies):
        r = W.moe_route(R=R, E=E, K=K, seed=0, device=device)
        gates = [(torch.randn(E, K, generator=torch.Generator(device=device).manual_seed(20 + c), device=device)
                  * 0.02).to(torch.bfloat16) for c in range(copies)]
        nbytes = E * K * 2 + E * 4 + R * K * 2 + R * E * 4 + R * topk * 8
        calls = [(lambda gw=gw: ops.MoeRoute(r["x"], gw, r["bias"], topk, 5.0)) for gw in gates]
        pin = str(device) != "cpu"
        xh = r["x"].cpu().pin_memory() if pin else r["x"]
        ih = torch.empty(R, topk, dtype=torch.int32).pin_memory() if pin else None
        xd = torch.empty_like(r["x"])

        def e2e(i):
            ops.copy_async(xd, xh)
            idx, w, _ = ops.MoeRoute(xd, gates[i], r["bias"], topk, 5.0)
            ops.copy_async(ih, idx)

        def cpu(_sample):
            import oracle as O
            O.moe_route(r["x"].cpu(), gates[0].cpu(), r["bias"].cpu(), topk, 5.0)
            return nbytes

        return dict(calls=calls, bytes=nbytes, kernels=2, h2d=R * K * 2, d2h=R * topk * 4, e2e=e2e, cpu=cpu,
                    cpu_sample=1, dtype="f32", kernel="router_logits_kernel")
    return build


def _relu2_workload(R, C):
    """Relu2 over x bf16 [R, C]: 2 bytes read and 2 written per element (an HBM stream)."""
    from nemotron_ops_b200 import ops

    def build(device, copies):
        g = torch.Generator(device=device).manual_seed(0)
        xs = [(torch.randn(R, C, generator=g, device=device) * 3).to(torch.bfloat16) for _ in range(copies)]
        nbytes = 2 * R * C * 2
        calls = [(lambda x=x: ops.Relu2(x)) for x in xs]
        pin = str(device) != "cpu"
        xh = xs[0].cpu().pin_memory() if pin else xs[0]
        yh = torch.empty(R, C, dtype=torch.bfloat16).pin_memory() if pin else None
        xd = torch.empty_like(xs[0])

        def e2e(i):
            ops.copy_async(xd, xh)
            ops.copy_async(yh, ops.Relu2(xd))

        def cpu(sample_rows):
            import oracle as O
            rows = max(1, min(R, sample_rows))
            O.relu2(xs[0][:rows].cpu())
            return nbytes * rows / R

        return dict(calls=calls, bytes=nbytes, kernels=1, h2d=R * C * 2, d2h=R * C * 2, e2e=e2e, cpu=cpu,
                    cpu_sample=1, dtype="f32", kernel="relu2_kernel")
    return build


def _mamba_workload(R, verify, heads=128, ng=8):
    """MambaStep (verify: MambaVerify from row 3 of R-row state buffers) at the reference test's
    size (tests/test_bolt_ops.py:264): the fp32 SSM state dominates the bytes."""
    from nemotron_ops_b200 import ops

    def build(device, copies):
        g = torch.Generator(device=device).manual_seed(0)
        di, rows = heads * 64, (R if verify else 1)
        cd = di + 2 * ng * 128

        def rnd(*shape, scale=1.0):
            return torch.randn(*shape, generator=g, device=device) * scale

        shared = [(rnd(cd, 1, 4, scale=0.3)).bfloat16(), rnd(cd, scale=0.1).bfloat16(), rnd(heads, scale=0.3),
                  -torch.rand(heads, generator=g, device=device) * 4 - 0.1, rnd(heads),
                  torch.rand(di, generator=g, device=device) + 0.5]
        sets = [[rnd(R, di + cd + heads, scale=0.7).bfloat16(), rnd(rows, cd, 3, scale=0.5).bfloat16(),
                 rnd(rows, heads, 128, 64, scale=0.1)] for _ in range(copies)]
        sel = torch.tensor([3 % rows], dtype=torch.int32, device=device)
        attrs = dict(heads=heads, head_dim=64, d_state=128, n_groups=ng, epsilon=1e-5, time_step_min=0.001)

        def op(s3):
            if verify:
                return ops.MambaVerify(*s3, *shared, sel, **attrs)
            return ops.MambaStep(*s3, *shared, **attrs)

        state_rows_out = R if verify else 1
        nbytes = (R * (di + cd + heads) * 2 + cd * 3 * 2 + cd * 4 * 2 + cd * 2 + heads * 128 * 64 * 4 +
                  3 * heads * 4 + di * 4 + R * di * 2 + state_rows_out * (cd * 3 * 2 + heads * 128 * 64 * 4) +
                  R * cd * 2 + R * di * 4)
        calls = [(lambda s3=s3: op(s3)) for s3 in sets]
        pin = str(device) != "cpu"
        ph = sets[0][0].cpu().pin_memory() if pin else sets[0][0]
        yh = torch.empty(R, di, dtype=torch.bfloat16).pin_memory() if pin else None
        pd = torch.empty_like(sets[0][0])

        def e2e(i):
            ops.copy_async(pd, ph)
            ops.copy_async(yh, op([pd, sets[i][1], sets[i][2]])[0])

        def cpu(_sample):
            import oracle as O
            c = [t.cpu() for t in sets[0] + shared]
            O.mamba_step(*c, **attrs, sel=(3 % rows) if verify else None)
            return nbytes

        return dict(calls=calls, bytes=nbytes, kernels=3, h2d=R * (di + cd + heads) * 2, d2h=R * di * 2, e2e=e2e,
                    cpu=cpu, cpu_sample=1, dtype="f32", kernel="mamba_ssm_kernel")
    return build


WORKLOADS = {
    "nvfp4_r1": ("Nvfp4Gemv R=1 K=8192 N=4096 (configs[1])", _gemv_workload("nvfp4", 1, 4096, 8192)),
    "nvfp4_r8": ("Nvfp4Gemv R=8 K=8192 N=4096 (configs[1])", _gemv_workload("nvfp4", 8, 4096, 8192)),
    "q8_r1": ("Q8Gemv R=1 K=4096 N=4096 (configs[0])", _gemv_workload("q8", 1, 4096, 4096)),
    "q4_r1": ("Q4Gemv int4 R=1 K=4096 N=8192 (configs[2])", _gemv_workload("q4", 1, 8192, 4096)),
    "q4_r4": ("Q4Gemv int4 R=4 K=4096 N=8192 (configs[2])", _gemv_workload("q4", 4, 8192, 4096)),
    "q4_r8": ("Q4Gemv int4 R=8 K=4096 N=8192 (configs[2])", _gemv_workload("q4", 8, 8192, 4096)),
    "q4iq2n_r1": ("Q4Gemv iq2=2 R=1 K=4096 N=8192 (configs[2])", _gemv_workload("q4", 1, 8192, 4096, iq2=2)),
    "q4iq2n_r4": ("Q4Gemv iq2=2 R=4 K=4096 N=8192 (configs[2])", _gemv_workload("q4", 4, 8192, 4096, iq2=2)),
    "q4iq2n_r8": ("Q4Gemv iq2=2 R=8 K=4096 N=8192 (configs[2])", _gemv_workload("q4", 8, 8192, 4096, iq2=2)),
    "moe_decode_r1": ("MoeDecode R=1 E=304 k=8 I=2304 (configs[3])", _moe_workload("MoeDecode", 1)),
    "moe_verify_r8": ("MoeVerify int4 R=8 E=304 k=8 I=2304 (configs[4])", _moe_workload("MoeVerify", 8)),
    "moe_verify_iq2n_r8": ("MoeVerify iq2=2 R=8 E=304 k=8 I=2304 (configs[4])", _moe_workload("MoeVerify", 8, iq2=2)),
    "moe_route_r1": ("MoeRoute R=1 E=304 K=4096 topk=8 (configs[3] routing)", _route_workload(1)),
    "moe_route_r8": ("MoeRoute R=8 E=304 K=4096 topk=8 (configs[4] routing)", _route_workload(8)),
    "route_moe_decode_r1": ("MoeRoute + MoeDecode R=1 E=304 k=8 I=2304 in one captured sequence (configs[3])",
                            _moe_workload("MoeDecode", 1, route=True)),
    "route_moe_verify_r8": ("MoeRoute + MoeVerify int4 R=8 E=304 k=8 I=2304 in one captured sequence (configs[4])",
                            _moe_workload("MoeVerify", 8, route=True)),
    "relu2": ("Relu2 x bf16 [8, 4194304] (not a BASELINE config; HBM stream)", _relu2_workload(8, 4194304)),
    "mamba_step_r1": ("MambaStep R=1 heads=128 ng=8 (not a BASELINE config; reference test size)",
                      _mamba_workload(1, False)),
    "mamba_verify_r8": ("MambaVerify R=8 sel=3 heads=128 ng=8 (not a BASELINE config; reference test size)",
                        _mamba_workload(8, True)),
}


# ------------------------------------------------------------------------------------------------
class ClockSampler:
    """nvidia-smi clock / throttle-reason samples of one GPU during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.gpu = gpu_index
        self.proc = None

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                          "-lms", "100", "-i", str(self.gpu)], stdout=subprocess.PIPE,
                                         stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=5)
        except Exception:
            self.proc.kill()
            return None
        sms, mx, reasons = [], 0.0, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in out.strip().splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sms.append(float(f[1]))
                mx = max(mx, float(f[2]))
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        if not sms:
            return None
        return {"sm_mhz": statistics.median(sms), "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": len(sms)}


# ------------------------------------------------------------------------------------------------
def dist_setup():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime

        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    else:
        torch.cuda.set_device(0)
    return world, rank, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def max_over_ranks(v, world):
    if world == 1:
        return v
    import torch.distributed as dist
    t = torch.tensor([v], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def _gather_equal(t, world):
    """True when every rank holds the same bits in ``t``."""
    if world == 1:
        return True
    import torch.distributed as dist
    parts = [torch.empty_like(t) for _ in range(world)]
    dist.all_gather(parts, t.contiguous())
    return all(torch.equal(parts[0], q) for q in parts[1:])


def _all_ok(ok, world):
    if world == 1:
        return bool(ok)
    import torch.distributed as dist
    f = torch.tensor([1 if ok else 0], dtype=torch.int32, device="cuda")
    dist.all_reduce(f, op=dist.ReduceOp.MIN)
    return bool(f.item())


def sharded_measure(world, rank, device, op="MoeVerify", iq2=0, E=304, I=2304, R=8, topk=8, iters=30, warmup=5,
                    us_1gpu=None):
    """Expert-sharded MoeVerify / MoeDecode step: every rank routes the same seeded inputs, holds
    only its own experts' weights and computes its fp32 partial; the partials are summed either
    by an NCCL all-reduce followed by the bf16 cast (the default path) or, where that path is
    built and tested (MoeVerify at 2 GPUs), inside the op's last kernel through NVLink peer memory.

    Parity first: on one seeded full expert set, every rank compares its bf16 output of each path
    with the single-GPU op run on the full weights (within 1e-3 + 1e-2 * |ref|) and all ranks
    must hold identical bits.  Then timing: CUDA-graph replays over rotated local weight copies
    (larger than 3x L2), CUDA events on the compute stream, max over ranks."""
    import torch.distributed as dist

    from nemotron_ops_b200 import ops
    from nemotron_ops_b200 import workloads as W
    from nemotron_ops_b200.sharded import PeerReducer, expert_range

    verify = op == "MoeVerify"
    r = W.moe_route(R=R, E=E, K=4096, seed=0, device=device)
    idx, w, _ = ops.MoeRoute(r["x"], r["gate_w"], r["bias"], topk, 5.0)
    z = W.moe_latent(R=R, device=device)
    e0, e1 = expert_range(E, rank, world)
    keys = ("fc1_w", "fc1_s", "fc2_w", "fc2_s")
    P = R * topk
    out_p = torch.empty(R, 1024, dtype=torch.float32, device=device)
    out = torch.empty(R, 1024, dtype=torch.bfloat16, device=device)
    scratch = (torch.empty(P, I, dtype=torch.bfloat16, device=device),
               torch.empty(P, 1024, dtype=torch.float32, device=device),
               torch.empty(1 + P + 8 * P, dtype=torch.int32, device=device))
    # the fused peer-memory reduction (MoeVerify; its parity is checked below on these ranks)
    reducer = PeerReducer(max_rows=R, device=device) if verify else None

    def run(wts, mode):
        if mode == "peer":
            ops.moe_verify_shard_allreduce(z, idx, w, *wts, topk=topk, iq2=iq2, e_begin=e0, e_end=e1,
                                           reducer=reducer, num_experts=E, out=out, outputs=scratch)
            return
        if verify:
            ops.moe_verify_shard(z, idx, w, *wts, topk=topk, iq2=iq2, e_begin=e0, e_end=e1, num_experts=E,
                                 out_partial=out_p, outputs=scratch)
        else:
            ops.moe_decode_shard(z, idx, w, *wts, topk=topk, e_begin=e0, e_end=e1, num_experts=E,
                                 out_partial=out_p, outputs=scratch[:2])
        if mode == "nccl":
            dist.all_reduce(out_p, op=dist.ReduceOp.SUM)
        ops.f32_to_bf16(out_p, out=out)

    modes = ["nccl", "local"] + (["peer"] if reducer is not None else [])

    # ---- parity against the single-GPU op on the full weights
    full = W.moe_experts(E=E, I=I, iq2=iq2, seed=99, device=device)
    fa = [z, idx, w] + [full[k] for k in keys]
    ref = (ops.MoeVerify(*fa, topk=topk, iq2=iq2)[0] if verify else ops.MoeDecode(*fa, topk=topk)[0]).clone()
    loc = [full[k][e0:e1].contiguous() for k in keys]
    parity = {}
    for mode in ("nccl", "peer"):
        if mode not in modes:
            parity[mode] = None
            continue
        run(loc, mode)
        torch.cuda.synchronize()
        d = (out.float() - ref.float()).abs()
        # the op's tolerance plus 1% of the output's largest magnitude: a shard sums its pairs in its
        # own fp32 order and the exchange adds the shards, so a row that cancels to near zero keeps
        # the rounding of its large terms (the same bound as tests/test_gpu_sharded.py)
        tol = 1e-3 + 1e-2 * ref.float().abs() + 1e-2 * ref.float().abs().max()
        ok = bool((d <= tol).all()) and ops.device_status() == 0
        same = _gather_equal(out, world)
        ok = _all_ok(ok, world)
        parity[mode] = {"ok": bool(ok and same), "ranks_identical": bool(same),
                        "max_abs_err": round(max_over_ranks(float(d.max()), world), 6),
                        "bit_equal_1gpu": _all_ok(bool(torch.equal(out, ref)), world)}
    del full, fa, loc
    torch.cuda.empty_cache()

    # ---- timing over rotated local weight copies
    one = W.moe_experts(E=e1 - e0, I=I, iq2=iq2, seed=10 + rank, device=device)
    per_copy = sum(t.numel() * t.element_size() for t in one.values())
    copies = max(2, int((3 * L2_BYTES) // max(1, per_copy)) + 1)
    sets = [one] + [W.moe_experts(E=e1 - e0, I=I, iq2=iq2, seed=20 + rank + 8 * c, device=device)
                    for c in range(copies - 1)]
    weights = [[d[k] for k in keys] for d in sets]
    ids = idx.reshape(-1).tolist()
    local_uniq = len({e for e in ids if e0 <= e < e1})
    local_pairs = sum(1 for e in ids if e0 <= e < e1)
    per_expert = per_copy // (e1 - e0)

    def timed(mode):
        for i in range(warmup):
            run(weights[i % copies], mode)
        torch.cuda.synchronize()
        barrier(world)
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        g = torch.cuda.CUDAGraph()
        with torch.cuda.stream(side):
            with torch.cuda.graph(g):
                for i in range(iters):
                    run(weights[i % copies], mode)
        torch.cuda.current_stream().wait_stream(side)
        g.replay()
        torch.cuda.synchronize()
        barrier(world)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        g.replay()
        b.record()
        torch.cuda.synchronize()
        us = max_over_ranks(a.elapsed_time(b) * 1e3 / iters, world)
        del g  # graphs holding NCCL calls go before the process group does
        barrier(world)
        return us

    us = {m: timed(m) for m in modes}
    uniq_max = int(max_over_ranks(float(local_uniq), world))
    uniq_sum = float(local_uniq)
    if world > 1:
        t = torch.tensor([uniq_sum], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.SUM)
        uniq_sum = float(t.item())
    mean_u = uniq_sum / world
    res = {"us": round(us["nccl"], 2), "path": "shard kernels + NCCL fp32 all-reduce + cast",
           "us_compute": round(us["local"], 2), "us_exchange": round(us["nccl"] - us["local"], 2),
           "us_peer": round(us["peer"], 2) if "peer" in us else None,
           "us_exchange_peer": round(us["peer"] - us["local"], 2) if "peer" in us else None,
           "parity": parity, "U_max": uniq_max, "U_imbalance": round(uniq_max / max(mean_u, 1e-9), 2),
           "bytes_max_rank": int(uniq_max * per_expert), "experts_per_rank": e1 - e0,
           "local_pairs_rank0": local_pairs if rank == 0 else None}
    if us_1gpu:
        res["us_1gpu"] = round(us_1gpu, 2)
        res["speedup_vs_1gpu"] = round(us_1gpu / us["nccl"], 3)
    return res


def capture(calls, reps):
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        for c in calls:  # eager warm-up outside the capture
            c()
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for _ in range(reps):
            for c in calls:
                c()
    return g


def time_graph(g, steps, warmup, world, sampler=None):
    for _ in range(warmup):
        g.replay()
    torch.cuda.synchronize()
    barrier(world)
    torch.cuda.synchronize()
    if sampler:
        sampler.start()
        time.sleep(0.3)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        g.replay()
    e1.record()
    torch.cuda.synchronize()
    clocks = sampler.stop() if sampler else None
    barrier(world)
    ms = e0.elapsed_time(e1)
    return max_over_ranks(ms, world), clocks


def measure(name, device, steps, warmup, world, copies, calls_target_ms=20.0, sampler=None):
    desc, builder = WORKLOADS[name]
    wl = builder(device, copies)
    one = capture(wl["calls"], 1)
    ms1, _ = time_graph(one, 3, 2, 1)
    per_call_ms = ms1 / 3 / len(wl["calls"])
    reps = max(1, int(calls_target_ms / max(per_call_ms * len(wl["calls"]), 1e-3)))
    del one
    g = capture(wl["calls"], reps)
    ms, clocks = time_graph(g, steps, warmup, world, sampler)
    ncalls = steps * reps * len(wl["calls"])
    us_call = ms * 1e3 / ncalls
    return dict(desc=desc, wl=wl, ms=ms, reps=reps, ncalls=ncalls, us_call=us_call,
                gbs=wl["bytes"] / (us_call * 1e3), clocks=clocks, graph=g)


def e2e_measure(wl, steps, world):
    calls = len(wl["calls"])
    for i in range(calls):
        wl["e2e"](i)
    torch.cuda.synchronize()
    barrier(world)
    n = max(steps, 20)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    t0 = time.perf_counter()
    for i in range(n):
        wl["e2e"](i % calls)
    host_ms = (time.perf_counter() - t0) * 1e3  # enqueue time: H2D copy, op call, D2H copy
    e1.record()
    torch.cuda.synchronize()
    ms = max_over_ranks(e0.elapsed_time(e1), world)
    return ms / n, host_ms / n


def cpu_measure(wl, budget_s=10.0, max_samples=20):
    sample = wl["cpu_sample"]
    t0 = time.perf_counter()
    done, n = 0.0, 0
    while n < max_samples and (time.perf_counter() - t0) < budget_s:
        done += wl["cpu"](sample)
        n += 1
    dt = time.perf_counter() - t0
    return done / dt / 1e9, n, dt


def run_reference(args, world, rank):
    """CPU reference arm: the oracle's torch restatement of the reference's test references."""
    if rank != 0:
        return
    desc, builder = WORKLOADS[args.workload]
    torch.set_num_threads(os.cpu_count() or 1)
    wl = builder("cpu", 1)
    for _ in range(args.warmup):
        wl["cpu"](wl["cpu_sample"])
    t0 = time.perf_counter()
    done = 0.0
    for _ in range(args.steps):
        done += wl["cpu"](wl["cpu_sample"])
    dt = time.perf_counter() - t0
    gbs = done / dt / 1e9
    line = {"metric": METRIC, "value": round(gbs, 3), "unit": "GB/s", "n_gpus": args.gpus, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(dt * 1e3 / max(args.steps, 1), 3), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic", "impl": "reference",
            "config": {"workload": desc},
            "cpu_baseline": {"value": round(gbs, 3), "unit": "GB/s", "cores": torch.get_num_threads(),
                             "kind": "port", "sample": f"the full op on one weight set per step ({desc})"},
            "e2e": {"value": round(gbs, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def _ref_gpu_workload(name, device, copies):
    """The reference's own kernels (its src/bolt_ops.cu recompiled for sm_100a, oracle/_ref/libbolt_ref.so)
    on one of the configs, called through ONNX Runtime's custom-op interface (the stand-in session
    of oracle/ort_shim) with preallocated outputs: returns (calls, bytes per call, description)."""
    from nemotron_ops_b200 import workloads as W
    from oracle.ort_shim import build as shim_build
    from oracle.ort_shim.shim import OrtShim

    path = os.path.join(shim_build.OUT, "libbolt_ref.so")
    if not os.path.exists(path):
        raise RuntimeError("oracle/_ref/libbolt_ref.so is absent (built where the reference checkout exists)")
    shim = OrtShim(os.path.join(shim_build.OUT, "libort_shim_host.so"))
    lib = shim.load(path)
    bf, f32, i32 = torch.bfloat16, torch.float32, torch.int32
    desc, _ = WORKLOADS[name]
    gemv = {"nvfp4_r1": ("nvfp4", 1, 4096, 8192), "nvfp4_r8": ("nvfp4", 8, 4096, 8192), "q8_r1": ("q8", 1, 4096, 4096),
            "q4_r1": ("q4", 1, 8192, 4096), "q4_r8": ("q4", 8, 8192, 4096), "q4iq2n_r1": ("q4n", 1, 8192, 4096),
            "q4iq2n_r8": ("q4n", 8, 8192, 4096)}
    if name in gemv:
        kind, R, N, K = gemv[name]
        sets = []
        for c in range(copies):
            if kind == "nvfp4":
                d = W.nvfp4_gemv(R=R, N=N, K=K, seed=c, device=device)
                sets.append([d["x"], d["w"], d["w_scale"], d["g"]])
            elif kind == "q8":
                d = W.q8_gemv(R=R, N=N, K=K, seed=c, device=device)
                sets.append([d["x"], d["B"], d["scales"]])
            else:
                d = W.q4_gemv(R=R, N=N, K=K, iq2=2 if kind == "q4n" else 0, seed=c, device=device)
                sets.append([d["x"], d["B"], d["scales"]])
        op = {"nvfp4": "Nvfp4Gemv", "q8": "Q8Gemv"}.get(kind, "Q4Gemv")
        kern = shim.kernel(lib, op, **({"iq2": 2} if kind == "q4n" else {}))
        y = torch.empty(R, N, dtype=bf, device=device)
        nbytes = sum(t.numel() * t.element_size() for t in sets[0][1:]) + sets[0][0].numel() * 2 + R * N * 2
        calls = [(lambda s=s: kern.run(s, [y])) for s in sets]
        return calls, nbytes, desc, kern
    if name.startswith("moe_route"):
        R = 8 if name.endswith("r8") else 1
        r = W.moe_route(R=R, E=304, K=4096, seed=0, device=device)
        gates = [(torch.randn(304, 4096, generator=torch.Generator(device=device).manual_seed(20 + c), device=device)
                  * 0.02).to(bf) for c in range(copies)]
        kern = shim.kernel(lib, "MoeRoute", topk=8, scale=5.0)
        outs = [torch.empty(R, 8, dtype=i32, device=device), torch.empty(R, 8, dtype=f32, device=device),
                torch.empty(R, 304, dtype=f32, device=device)]
        nbytes = 304 * 4096 * 2 + 304 * 4 + R * 4096 * 2 + R * 304 * 4 + R * 8 * 8
        calls = [(lambda gw=gw: kern.run([r["x"], gw, r["bias"]], outs)) for gw in gates]
        return calls, nbytes, desc, kern
    moe = {"moe_decode_r1": ("MoeDecode", 1, 0), "moe_verify_r8": ("MoeVerify", 8, 0),
           "moe_verify_iq2n_r8": ("MoeVerify", 8, 2)}
    if name in moe:
        op, R, iq2 = moe[name]
        from nemotron_ops_b200 import ops
        r = W.moe_route(R=R, E=304, K=4096, seed=0, device=device)
        idx, w, _ = ops.MoeRoute(r["x"], r["gate_w"], r["bias"], 8, 5.0)  # the same routing as our arm
        z = W.moe_latent(R=R, device=device)
        sets = [W.moe_experts(E=304, I=2304, iq2=iq2, seed=10 + c, device=device) for c in range(copies)]
        kern = shim.kernel(lib, op, **({"topk": 8, "iq2": iq2} if iq2 else {"topk": 8}))
        P = R * 8
        outs = [torch.empty(R, 1024, dtype=bf, device=device), torch.empty(P, 2304, dtype=bf, device=device),
                torch.empty(P, 1024, dtype=f32, device=device)]
        if op == "MoeVerify":
            outs.append(torch.empty(1 + P + 8 * P, dtype=i32, device=device))
        uniq = len(set(idx.reshape(-1).tolist()))
        e0 = sets[0]
        per_expert = sum(e0[k][0].numel() * e0[k].element_size() for k in ("fc1_w", "fc1_s", "fc2_w", "fc2_s"))
        nbytes = uniq * per_expert + R * 1024 * 2 + R * 8 * 8 + R * 1024 * 2
        calls = [(lambda d=d: kern.run([z, idx, w, d["fc1_w"], d["fc1_s"], d["fc2_w"], d["fc2_s"]], outs)) for d in sets]
        return calls, nbytes, desc, kern
    raise RuntimeError(f"no reference-GPU form of workload {name}")


def run_reference_gpu(args, world, rank):
    """The reference's kernels on this B200 (rank 0 alone; other ranks exit without work)."""
    if rank != 0:
        return
    torch.cuda.set_device(0)
    device = "cuda:0"
    hbm, peak_kind = peaks()
    names = [args.workload] + ([] if args.no_extra else
                               [n for n in ("nvfp4_r8", "q8_r1", "q4_r1", "q4_r8", "q4iq2n_r1", "q4iq2n_r8",
                                            "moe_decode_r1", "moe_verify_r8", "moe_verify_iq2n_r8", "moe_route_r8")
                                if n != args.workload])
    res = {}
    for n in names:
        try:
            tmp = WORKLOADS[n][1](device, 1)
            copies = max(3, int((3 * L2_BYTES) // tmp["bytes"]) + 1)
            del tmp
            calls, nbytes, desc, _k = _ref_gpu_workload(n, device, copies)
            one = capture(calls, 1)
            ms1, _ = time_graph(one, 3, 2, 1)
            reps = max(1, int(20.0 / max(ms1 / 3, 1e-3)))
            del one
            g = capture(calls, reps)
            steps = args.steps if n == args.workload else 5
            ms, clocks = time_graph(g, steps, max(3, args.warmup), 1)
            us = ms * 1e3 / (steps * reps * len(calls))
            res[n] = {"us": round(us, 2), "frac": round(nbytes / (us * 1e3) / hbm, 3), "bytes": nbytes, "desc": desc,
                      "clocks": clocks}
            del g
        except Exception as e:  # report, never hide
            res[n] = {"error": str(e)[:200]}
        torch.cuda.empty_cache()
    head = res.get(args.workload, {})
    gbs = head["bytes"] / (head["us"] * 1e3) if "us" in head else None
    line = {"metric": METRIC, "value": round(gbs, 2) if gbs else None, "unit": "GB/s", "n_gpus": 1,
            "steps": args.steps, "warmup": args.warmup, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f16", "data": "synthetic", "impl": "reference-gpu",
            "us_per_call": head.get("us"),
            "config": {"workload": head.get("desc", args.workload),
                       "what": "the reference's own src/bolt_ops.cu kernels recompiled for sm_100a, called "
                               "through its RegisterCustomOps / ComputeV2 (ONNX Runtime stand-in session, "
                               "preallocated outputs) in CUDA graphs over rotated weight copies"},
            "roofline": {"bound": "hbm", "peak": hbm, "unit": "GB/s", "peak_source": peak_kind,
                         "frac": head.get("frac")},
            "configs_measured": {n: {k: v for k, v in r.items() if k not in ("desc", "bytes", "clocks")}
                                 for n, r in res.items() if n != args.workload}}
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=30)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference", "reference-gpu"],
                    help="reference: the reference's CPU path (torch restatement); reference-gpu: the "
                         "reference's own CUDA kernels recompiled for sm_100a, on this GPU")
    ap.add_argument("--workload", default="nvfp4_r1", choices=sorted(WORKLOADS))
    ap.add_argument("--no-extra", action="store_true", help="skip the other configs")
    ap.add_argument("--copies", type=int, default=0,
                    help="rotated weight copies (default: enough to exceed 3x L2); a small number is for "
                         "profiler captures, not for bench numbers")
    ap.add_argument("--no-cpu", action="store_true", help="skip the cpu_baseline leg")
    ap.add_argument("--extra", default="", help="comma-separated subset of the other configs to measure (default: all)")
    ap.add_argument("--pdl", type=int, default=1, choices=[0, 1, 2],
                    help="0: plain launches; 1: programmatic dependent launch (the library default); "
                         "2: PDL with early weight streaming")
    args = ap.parse_args()
    args.steps = max(1, args.steps)
    args.warmup = max(3, args.warmup)

    if args.impl == "reference":  # rank 0 alone runs the CPU reference; other ranks exit without work
        run_reference(args, int(os.environ.get("WORLD_SIZE", "1")), int(os.environ.get("RANK", "0")))
        return
    if args.impl == "reference-gpu":
        run_reference_gpu(args, int(os.environ.get("WORLD_SIZE", "1")), int(os.environ.get("RANK", "0")))
        return
    world, rank, local = dist_setup()

    from nemotron_ops_b200 import ops
    ops.set_launch_options(pdl=args.pdl >= 1, early_weights=args.pdl == 2)
    device = f"cuda:{local}"
    hbm, peak_kind = peaks()
    desc, builder = WORKLOADS[args.workload]
    # enough distinct weight copies to exceed 3x L2 (--copies: fewer, for profiler captures only;
    # the line then says so in config.cache)
    tmp = builder(device, 1)
    copies = args.copies or max(3, int((3 * L2_BYTES) // tmp["bytes"]) + 1)
    del tmp
    torch.cuda.empty_cache()
    vis = os.environ.get("CUDA_VISIBLE_DEVICES")
    sampler = ClockSampler(vis.split(",")[local] if vis else local)
    m = measure(args.workload, device, args.steps, args.warmup, world, copies, sampler=sampler)
    wl = m["wl"]
    copies_bytes = copies * wl["bytes"]
    value = wl["bytes"] * m["ncalls"] * world / (m["ms"] * 1e-3) / 1e9
    e2e_ms, e2e_host_ms = e2e_measure(wl, args.steps, world)
    e2e_gbs = wl["bytes"] * world / (e2e_ms * 1e-3) / 1e9
    del m["graph"]

    extra = {}
    if not args.no_extra:
        subset = [n for n in args.extra.split(",") if n] or list(WORKLOADS)
        for name in subset:
            if name == args.workload or name not in WORKLOADS:
                continue
            try:
                tmp = WORKLOADS[name][1](device, 1)
                cp = max(3, int((3 * L2_BYTES) // tmp["bytes"]) + 1)
                del tmp
                r = measure(name, device, 5, 3, world, cp)
                extra[name] = {"us": round(r["us_call"], 2), "frac": round(r["gbs"] / hbm, 3)}
                if "unique_experts" in r["wl"]:
                    extra[name]["U"] = r["wl"]["unique_experts"]
                del r
            except Exception as e:  # report, never hide
                extra[name] = {"error": str(e)[:200]}
            torch.cuda.empty_cache()

    if world > 1 and not args.no_extra:  # the one path with a real exchange step
        legs = (("moe_verify_sharded", "MoeVerify", 0, 8, "moe_verify_r8"),
                ("moe_verify_iq2n_sharded", "MoeVerify", 2, 8, "moe_verify_iq2n_r8"),
                ("moe_decode_sharded", "MoeDecode", 0, 1, "moe_decode_r1"))
        for name, op, q, rows, one_gpu in legs:
            try:
                extra[name] = sharded_measure(world, rank, device, op=op, iq2=q, R=rows,
                                              us_1gpu=(extra.get(one_gpu) or {}).get("us"))
            except Exception as e:  # report, never hide
                extra[name] = {"error": str(e)[:200]}
            torch.cuda.empty_cache()

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        torch.set_num_threads(os.cpu_count() or 1)
        gbs, n, dt = cpu_measure(wl)
        cpu = {"value": round(gbs, 4), "unit": "GB/s", "cores": torch.get_num_threads(), "kind": "port",
               "sample": f"{n} oracle runs of the full op on one weight set ({dt:.1f} s; torch CPU dequant + fp32 matmul)"}

    if rank == 0:
        traffic = None
        tpath = os.path.join(ROOT, "profiles", "traffic.json")
        if os.path.exists(tpath):
            try:
                traffic = json.load(open(tpath)).get(args.workload)
            except Exception:
                traffic = None
        line = {
            "metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(m["ms"] / args.steps, 4), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": wl["dtype"], "data": "synthetic",
            "us_per_call": round(m["us_call"], 3),
            "config": {"workload": desc, "calls_per_step": m["reps"] * len(wl["calls"]), "weight_copies": copies,
                       "bytes_per_call": wl["bytes"],
                       "cache": (f"inputs larger than L2: {copies} distinct weight copies ({copies_bytes / 1e6:.0f} MB) "
                                 f"rotated inside every step") if copies_bytes > L2_BYTES else
                                (f"profiler case: {copies} weight copies ({copies_bytes / 1e6:.0f} MB) fit in L2; not a "
                                 f"bench number"), "parallelism": "replicas" if world > 1 else "single",
                       "launch": ("plain", "pdl", "pdl+early_weights")[args.pdl]},
            "roofline": {"bound": "hbm", "achieved": round(wl["bytes"] / (m["us_call"] * 1e3), 1), "peak": hbm,
                         "unit": "GB/s", "frac": round(wl["bytes"] / (m["us_call"] * 1e3) / hbm, 4),
                         "traffic": traffic, "peak_source": peak_kind, "kernel": wl["kernel"]},
            "clocks": m["clocks"],
            "e2e": {"value": round(e2e_gbs, 2), "unit": "GB/s", "h2d_bytes_per_step": wl["h2d"],
                    "d2h_bytes_per_step": wl["d2h"], "us_per_call": round(e2e_ms * 1e3, 2),
                    "host_enqueue_us_per_call": round(e2e_host_ms * 1e3, 2),
                    "api": "nemotron_ops_b200.ops (ctypes -> C ABI): bolt_memcpy_async of pinned host inputs in, "
                           "the op, bolt_memcpy_async of the result out, every call"},
            "gpu_launches": m["ncalls"] * wl["kernels"],
            "cpu_baseline": cpu,
            "configs_measured": extra,
        }
        # the compact per-config numbers go right after the headline keys, the long strings last, so
        # a reader that keeps only the head of the line still sees every config
        order = ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
                 "scaling", "vs_baseline", "dtype", "data", "us_per_call", "configs_measured", "gpu_launches",
                 "roofline", "clocks", "cpu_baseline", "e2e", "config")
        line = {k: line[k] for k in order}
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
