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
