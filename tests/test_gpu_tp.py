"""Row-parallel (K-sharded) exact linear on 2 GPUs over NCCL: every rank must get exactly the 1-GPU output bits.

Each rank holds a K slice of the activations and of the weight rows; whole-row scales come from a MAX all-reduce of
row maxima, the exact int64 partial totals are summed with an NCCL int64 all-reduce (exact in any ring order), then
the scaling epilogue runs on every rank (vllm_exact/parallel.py). Skipped on machines with fewer than 2 GPUs."""
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, root, q):
    import sys
    for p in (root, os.path.join(root, "vllm-exact_b200"), os.path.join(root, "tests", "golden")):
        sys.path.insert(0, p)
    import datetime
    import torch.distributed as dist
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            device_id=dev, timeout=datetime.timedelta(seconds=60))
    try:
        import recipes as R
        from vllm_exact import kernels as K, parallel as P
        res = {}
        for (M, N, Kd, F, tr) in [(24, 384, 4096, 14, True), (64, 4096, 12288, 14, True), (5, 200, 12288, 15, False),
                                  (256, 1024, 4096, 14, True)]:
            x, w = R.extreme_digits(M, N, Kd)
            x[1] *= 1e-3
            x[2, : Kd // 2] = 0.0
            xb, wb = x.bfloat16().to(dev), w.bfloat16().to(dev)
            ref = torch.empty(M, N, device=dev, dtype=torch.bfloat16)
            K.exact_linear(K.digitize(xb, F), K.digitize(wb, F), F, tr, out=ref)  # 1-GPU result
            ks = Kd // world
            a, b = rank * ks, (rank + 1) * ks
            wd = P.digitize_weight_row_sharded(wb[:, a:b].contiguous(), F)
            y = P.row_parallel_linear(xb[:, a:b], *wd, F, tr)
            res[(M, N, Kd, F)] = bool(torch.equal(y, ref))
        torch.cuda.synchronize()
        q.put((rank, res))
    finally:
        dist.destroy_process_group()


def test_row_parallel_two_gpus_bitexact():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, root, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=600) for _ in procs)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    for r in range(2):
        assert all(res[r].values()), res[r]


def _worker_config3(rank, world, port, root, q):
    """BASELINE config 3 K-sharded: the 16 fixed target rows (K=12288, N=4096) embedded at random positions in
    batches of M rows; every rank must return the 1-GPU bits for every target row."""
    import sys
    for p in (root, os.path.join(root, "vllm-exact_b200"), os.path.join(root, "tests", "golden")):
        sys.path.insert(0, p)
    import datetime
    import torch.distributed as dist
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            device_id=dev, timeout=datetime.timedelta(seconds=60))
    try:
        from vllm_exact import kernels as K, parallel as P
        Kd, N = 12288, 4096
        targets = torch.randn(16, Kd, generator=torch.Generator().manual_seed(0)).bfloat16().to(dev)
        w = (torch.randn(N, Kd, generator=torch.Generator().manual_seed(1)) * 0.02).bfloat16().to(dev)
        wd = K.digitize(w, 14)
        base = torch.empty(16, N, device=dev, dtype=torch.bfloat16)
        K.exact_linear(K.digitize(targets, 14), wd, 14, True, out=base)  # 1-GPU result of the targets
        ks = Kd // world
        a, b = rank * ks, (rank + 1) * ks
        wsd = P.digitize_weight_row_sharded(w[:, a:b].contiguous(), 14)
        res = {}
        for M in (1, 16, 100, 256):
            gm = torch.Generator().manual_seed(M)
            filler = torch.randn(M, Kd, generator=gm)
            filler[torch.rand(M, Kd, generator=gm) < 0.001] *= 50
            filler = filler.bfloat16().to(dev)
            nt = min(M, 16)
            pos = torch.randperm(M, generator=gm)[:nt].to(dev)
            filler[pos] = targets[:nt]
            y = P.row_parallel_linear(filler[:, a:b], *wsd, 14, True)
            res[M] = bool(torch.equal(y[pos], base[:nt]))
        torch.cuda.synchronize()
        q.put((rank, res))
    finally:
        dist.destroy_process_group()


def test_config3_k_sharded_on_2_4_8_gpus():
    """BASELINE config 3 across GPU counts: K-sharded over 2, 4 and 8 GPUs (as many as the machine has), int64 NCCL
    all-reduce of the partial totals; every target row is bitwise identical to the 1-GPU result."""
    n = torch.cuda.device_count()
    if n < 2:
        pytest.skip("needs 2 GPUs")
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    ctx = mp.get_context("spawn")
    for world in (w for w in (2, 4, 8) if w <= n):
        q = ctx.Queue()
        port = _port()
        procs = [ctx.Process(target=_worker_config3, args=(r, world, port, root, q)) for r in range(world)]
        for p in procs:
            p.start()
        res = dict(q.get(timeout=600) for _ in procs)
        for p in procs:
            p.join(timeout=120)
            assert p.exitcode == 0
        for r in range(world):
            assert all(res[r].values()), (world, r, res[r])
