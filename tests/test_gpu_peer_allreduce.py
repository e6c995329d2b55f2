"""bolt_moe_verify_shard_allreduce on 2 GPUs (one spawned process per GPU, NCCL on 127.0.0.1).

The fused op sums the ranks' fp32 partials through NVLink peer memory inside its last kernel.
With two ranks a + b is exact whatever the order, so its output must equal the NCCL path
(bolt_moe_verify_shard + all_reduce + cast) bit for bit, on consecutive calls (both buffer halves
and the call counters) and when replayed from a CUDA graph; and it must match the single-GPU
MoeVerify within the op's tolerance.  Skipped with fewer than 2 GPUs.
"""
import os
import socket
from datetime import timedelta

import pytest
import torch

pytestmark = pytest.mark.gpu

WORLD = 2


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, port, iq2, q):
    import torch.distributed as dist

    from nemotron_ops_b200 import ops
    from nemotron_ops_b200 import workloads as W
    from nemotron_ops_b200.sharded import PeerReducer, ShardedMoeVerify

    os.environ["MASTER_ADDR"], os.environ["MASTER_PORT"] = "127.0.0.1", str(port)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=WORLD, timeout=timedelta(seconds=60), device_id=dev)
    try:
        R, E, I, topk = 8, 40, 2304, 8
        ex = W.moe_experts(E=E, I=I, iq2=iq2, seed=31, device=dev)
        g = torch.Generator().manual_seed(5)
        idx = torch.stack([torch.randperm(E, generator=g)[:topk] for _ in range(R)]).int().to(dev)
        w = torch.rand(R, topk, generator=g).to(dev)
        z = W.moe_latent(R=R, seed=6, device=dev)
        full = [ex[k] for k in ("fc1_w", "fc1_s", "fc2_w", "fc2_s")]
        sh = ShardedMoeVerify(E, topk, iq2)
        local = [sh.local_slice(t) for t in full]
        red = PeerReducer(max_rows=R, device=dev)
        fused = [sh.fused(z, idx, w, local, red).clone() for _ in range(3)]
        nccl = sh(z, idx, w, local)
        single = ops.MoeVerify(z, idx, w, *full, topk=topk, iq2=iq2)[0]
        # graph replay: the call counters live in device memory, so replays stay in step
        out = torch.empty(R, 1024, dtype=torch.bfloat16, device=dev)
        scratch = (torch.empty(R * topk, I, dtype=torch.bfloat16, device=dev),
                   torch.empty(R * topk, 1024, dtype=torch.float32, device=dev),
                   torch.empty(1 + 9 * R * topk, dtype=torch.int32, device=dev))
        s = torch.cuda.Stream(dev)
        s.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(s):
            sh.fused(z, idx, w, local, red, out=out, outputs=scratch)
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph, stream=s):
                sh.fused(z, idx, w, local, red, out=out, outputs=scratch)
        torch.cuda.current_stream(dev).wait_stream(s)
        replays = []
        for _ in range(3):
            out.zero_()
            graph.replay()
            torch.cuda.synchronize(dev)
            replays.append(out.clone())
        del graph
        torch.cuda.synchronize(dev)
        err = []
        for i, o in enumerate(fused + replays):
            if not torch.equal(o, nccl):
                err.append(f"call {i}: differs from the NCCL path in {int((o != nccl).sum())} values")
        d = (nccl.float() - single.float()).abs()
        if not bool((d <= 1e-3 + 1e-2 * single.float().abs()).all()):
            err.append("the sharded result is outside the op's tolerance of the single-GPU MoeVerify")
        st = ops.device_status()
        if st:
            err.append(f"device status {st:#x}")
        q.put((rank, "; ".join(err)))
    except Exception as e:  # report, the parent asserts
        q.put((rank, f"{type(e).__name__}: {e}"))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < WORLD, reason="needs 2 GPUs")
@pytest.mark.parametrize("iq2", [0, 2])
def test_fused_sharded_verify_matches_nccl_path(iq2):
    ctx = torch.multiprocessing.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, port, iq2, q)) for r in range(WORLD)]
    for p in procs:
        p.start()
    results = {}
    try:
        for _ in range(WORLD):
            rank, msg = q.get(timeout=300)
            results[rank] = msg
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    assert all(msg == "" for msg in results.values()), results
