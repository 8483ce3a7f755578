"""Two-GPU parity of the fused TP2 o_proj GEMM + all-reduce (TP2OprojAllReduce).

Each rank runs in its own process on its own GPU (NCCL group on 127.0.0.1).  The fused
result must (1) be bit-identical on both ranks, (2) match the reference's composition
F.linear + NCCL all-reduce within one bf16 rounding step of each partial, and (3) match an
fp32 restatement of the whole projection within bf16 tolerance, over several calls (both
inbox halves) and token counts, eagerly and replayed from a CUDA graph.  Skipped unless two GPUs are
visible.
"""
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _rank_main(rank, port, result_dir):
    import datetime

    import torch.distributed as dist
    import torch.nn.functional as F

    from shardserve_b200.tp2 import TP2OprojAllReduce

    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("nccl", rank=rank, world_size=2,
                            timeout=datetime.timedelta(seconds=60), device_id=dev)
    report = []
    try:
        N, K = 2048, 1024
        op = TP2OprojAllReduce(dist.group.WORLD, dev, 256, N, K)
        for call, T in enumerate([64, 1, 200, 256, 33, 64]):
            g = torch.Generator(device="cpu").manual_seed(100 * call + rank)
            a = (torch.randn(T, K, generator=g) * 0.5).to(torch.bfloat16).to(dev)
            w = (torch.randn(N, K, generator=g) * K ** -0.5).to(torch.bfloat16).to(dev)
            got = op(a, w)
            ref = F.linear(a, w)
            dist.all_reduce(ref)
            parts = [torch.empty(T, K, dtype=torch.bfloat16, device=dev) for _ in range(2)]
            wts = [torch.empty(N, K, dtype=torch.bfloat16, device=dev) for _ in range(2)]
            dist.all_gather(parts, a)
            dist.all_gather(wts, w)
            exact = sum(p.float() @ q.float().t() for p, q in zip(parts, wts))
            other = [torch.empty_like(got) for _ in range(2)]
            dist.all_gather(other, got)
            torch.cuda.synchronize()
            report.append(dict(
                T=T, identical=bool(torch.equal(other[0], other[1])),
                vs_ref=float((got.float() - ref.float()).abs().max()),
                vs_exact=float((got.float() - exact).abs().max()),
                ref_vs_exact=float((ref.float() - exact).abs().max()),
                scale=float(exact.abs().max())))
        # Replays from a CUDA graph: the call number advances on the device.
        g = torch.Generator(device="cpu").manual_seed(999 + rank)
        a = torch.randn(64, K, generator=g).to(torch.bfloat16).to(dev)
        w = (torch.randn(N, K, generator=g) * K ** -0.5).to(torch.bfloat16).to(dev)
        eager = op(a, w).clone()
        out = torch.empty_like(eager)
        s = torch.cuda.Stream(dev)
        s.wait_stream(torch.cuda.current_stream(dev))
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.stream(s):
            with torch.cuda.graph(graph, stream=s):
                for _ in range(3):
                    op(a, w, out=out)
        torch.cuda.current_stream(dev).wait_stream(s)
        for _ in range(4):
            out.zero_()
            graph.replay()
            torch.cuda.synchronize()
            report.append(dict(T=64, identical=True, vs_ref=0.0, vs_exact=0.0, ref_vs_exact=0.0,
                               scale=1.0, graph_equal=bool(torch.equal(out, eager))))
        del graph
        report.append(dict(errors=op.device_errors()))
        op.close()
    finally:
        torch.save(report, os.path.join(result_dir, f"rank{rank}.pt"))
        dist.barrier()
        dist.destroy_process_group()


def test_fused_oproj_allreduce_two_gpus(tmp_path):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    mp.start_processes(_rank_main, args=(_free_port(), str(tmp_path)), nprocs=2,
                       start_method="spawn", join=True)
    for rank in range(2):
        rep = torch.load(tmp_path / f"rank{rank}.pt")
        assert rep[-1]["errors"] == 0
        for r in rep[:-1]:
            assert r.get("graph_equal", True), r
            assert r["identical"], r
            # Two bf16 roundings of partials plus one of the sum: within a few ulps of the
            # output's magnitude, as the reference's own composition is.
            tol = 4 * 2.0 ** -8 * max(r["scale"], 1e-3)
            assert r["vs_exact"] <= tol, r
            assert r["vs_ref"] <= tol, r
