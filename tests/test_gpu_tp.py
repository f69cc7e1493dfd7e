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


def _worker_peer(rank, world, port, root, q):
    """Row-parallel layers with both exchanges over peer memory (PeerRowParallel) against the NCCL path and the 1-GPU
    result, over enough calls that every shared buffer is reused, eagerly and replayed from a CUDA graph."""
    import sys
    for p in (root, os.path.join(root, "vllm-exact_b200"), os.path.join(root, "tests", "golden")):
        sys.path.insert(0, p)
    import datetime
    import torch.distributed as dist
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            device_id=dev, timeout=datetime.timedelta(seconds=60))
    peer = None
    try:
        import recipes as R
        from vllm_exact import kernels as K, parallel as P
        peer = P.PeerRowParallel(256, 4096)
        res = {}
        for it, (M, N, Kd, F, tr) in enumerate([(1, 4096, 4096, 14, True), (16, 4096, 12288, 14, True),
                                                (64, 1024, 4096, 15, False), (5, 200, 12288, 15, True),
                                                (256, 4096, 4096, 14, True), (16, 4096, 12288, 14, True)]):
            x, w = R.extreme_digits(M, N, Kd, seed=it)
            x[1 % M] *= 1e-3
            xb, wb = x.bfloat16().to(dev), w.bfloat16().to(dev)
            ref = torch.empty(M, N, device=dev, dtype=torch.bfloat16)
            K.exact_linear(K.digitize(xb, F), K.digitize(wb, F), F, tr, out=ref)
            ks = Kd // world
            a, b = rank * ks, (rank + 1) * ks
            wd = P.digitize_weight_row_sharded(wb[:, a:b].contiguous(), F)
            y_nccl = P.row_parallel_linear(xb[:, a:b], *wd, F, tr)
            y_peer = peer.linear(xb[:, a:b], *wd, F, tr)
            res[it] = (bool(torch.equal(y_peer, ref)), bool(torch.equal(y_nccl, ref)))
        # CUDA graph: one call captured, replayed with new inputs; the epochs live on the device, so every replay runs
        # a fresh round of both peer protocols
        M, N, Kd = 16, 4096, 12288
        ks = Kd // world
        a, b = rank * ks, (rank + 1) * ks
        w = (torch.randn(N, Kd, generator=torch.Generator().manual_seed(7)) * 0.02).bfloat16().to(dev)
        wd_full = K.digitize(w, 14)
        wd = P.digitize_weight_row_sharded(w[:, a:b].contiguous(), 14)
        xin = torch.zeros(M, ks, dtype=torch.bfloat16, device=dev)
        st = torch.cuda.Stream(dev)
        K.reserve_workspace(K.lib().ex_linear_workspace_bytes(M, N, ks, 0, 0), dev, stream=st)
        st.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(st):
            peer.linear(xin, *wd, 14, True)
        torch.cuda.synchronize(dev)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=st):
            yg = peer.linear(xin, *wd, 14, True)
        for t in range(3):
            x = torch.randn(M, Kd, generator=torch.Generator().manual_seed(100 + t)).bfloat16().to(dev)
            ref = torch.empty(M, N, device=dev, dtype=torch.bfloat16)
            K.exact_linear(K.digitize(x, 14), wd_full, 14, True, out=ref)
            xin.copy_(x[:, a:b])
            torch.cuda.synchronize(dev)
            g.replay()
            torch.cuda.synchronize(dev)
            res[f"graph{t}"] = (bool(torch.equal(yg, ref)), True)
        del g
        # the maxima exchange alone, many calls back to back without a synchronization (ranks drift apart): every
        # call's digits equal the slice of the whole rows' digits
        M, Kd = 48, 8192
        ks = Kd // world
        a, b = rank * ks, (rank + 1) * ks
        x = torch.randn(M, Kd, generator=torch.Generator().manual_seed(11)).bfloat16().to(dev)
        ref = [t[:, a:b] if t.dim() == 2 else t for t in K.digitize(x, 14)]
        xs = x[:, a:b].contiguous()
        outs = [peer.digitize(xs, 14) for _ in range(20)]
        torch.cuda.synchronize()
        res["digitize_back_to_back"] = (all(torch.equal(o[0], ref[0]) and torch.equal(o[1], ref[1]) and
                                            torch.equal(o[3], ref[3]) for o in outs), True)
        # the same calls alternating between two streams with nothing ordering them: the object orders each call
        # after the previous one, so no two take the same epoch
        sts = [torch.cuda.Stream(dev), torch.cuda.Stream(dev)]
        outs = []
        for i in range(12):
            with torch.cuda.stream(sts[i % 2]):
                outs.append(peer.digitize(xs, 14))
        torch.cuda.synchronize()
        res["digitize_two_streams"] = (all(torch.equal(o[0], ref[0]) and torch.equal(o[1], ref[1]) and
                                           torch.equal(o[3], ref[3]) for o in outs), True)
        # the plugin's op: the group's peer object made once (as the plugin does at load time), then calls of up to
        # PEER_ROWS rows over peer memory and larger ones through NCCL, all equal to the 1-GPU layer
        from vllm_exact import ops  # noqa: F401  (registers exactmm::linear_row_parallel)
        auto = P.peer_for(dev, dist.group.WORLD, create=True)
        Kd, N = 4096, 1024
        ks = Kd // world
        a, b = rank * ks, (rank + 1) * ks
        w = (torch.randn(N, Kd, generator=torch.Generator().manual_seed(21)) * 0.02).bfloat16().to(dev)
        wd_full = K.digitize(w, 14)
        wd = P.digitize_weight_row_sharded(w[:, a:b].contiguous(), 14)
        for M in (3, P.PEER_ROWS, P.PEER_ROWS + 5):
            x = torch.randn(M, Kd, generator=torch.Generator().manual_seed(M)).bfloat16().to(dev)
            ref = torch.empty(M, N, device=dev, dtype=torch.bfloat16)
            K.exact_linear(K.digitize(x, 14), wd_full, 14, True, out=ref)
            y = torch.ops.exactmm.linear_row_parallel(x[:, a:b], *wd)
            res[f"op_M{M}"] = (auto is not None and bool(torch.equal(y, ref)), True)
        torch.cuda.synchronize()
        if auto is not None:
            auto.close()
        torch.cuda.synchronize()
        code = ctypes_code()
        q.put((rank, res, code))
    finally:
        torch.cuda.synchronize()
        dist.barrier()
        if peer is not None:
            peer.close()
        dist.destroy_process_group()


def ctypes_code():
    import ctypes
    from vllm_exact import _lib
    c = ctypes.c_int(0)
    _lib.lib().ex_device_error(ctypes.byref(c))
    return c.value


def test_peer_row_parallel_two_or_more_gpus_bitexact():
    """Row-parallel layers with both exchanges over peer memory give the 1-GPU bits (and the NCCL path's) on every
    rank, for 2 GPUs and, where present, 4 and 8."""
    n = torch.cuda.device_count()
    if n < 2:
        pytest.skip("needs 2 GPUs")
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    ctx = mp.get_context("spawn")
    for world in (w for w in (2, 4, 8) if w <= n):
        q = ctx.Queue()
        port = _port()
        procs = [ctx.Process(target=_worker_peer, args=(r, world, port, root, q)) for r in range(world)]
        for p in procs:
            p.start()
        res = {}
        for _ in procs:
            r, v, code = q.get(timeout=600)
            res[r] = (v, code)
        for p in procs:
            p.join(timeout=120)
            assert p.exitcode == 0
        for r in range(world):
            v, code = res[r]
            assert code == 0, (world, r, code)
            assert all(a and b for a, b in v.values()), (world, r, v)


def _one_gpu_peer_args(dev, M, N, world, out_dtype=torch.bfloat16):
    """Device arrays for a single-GPU call of ex_allreduce_epilogue_i64: every 'rank' is this process."""
    from vllm_exact import _lib
    parts = [torch.randint(-2**40, 2**40, (M, N), dtype=torch.int64, device=dev) for _ in range(world)]
    outs = [torch.zeros(M * N, dtype=torch.int64, device=dev) for _ in range(world)]  # (epoch, value) words
    flags = torch.zeros(_lib.tp_flag_words(world), dtype=torch.int32, device=dev)
    ctl = torch.zeros(2, dtype=torch.int32, device=dev)
    part_ptrs = torch.tensor([t.data_ptr() for t in parts], dtype=torch.int64, device=dev)
    out_ptrs = torch.tensor([t.data_ptr() for t in outs], dtype=torch.int64, device=dev)
    flag_ptrs = torch.tensor([flags.data_ptr()] * world, dtype=torch.int64, device=dev)
    return parts, outs, flags, ctl, part_ptrs, out_ptrs, flag_ptrs


def _lib_mod():
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path.insert(0, os.path.join(root, "vllm-exact_b200"))
    from vllm_exact import _lib, kernels as K
    return _lib, K


def test_peer_epilogue_one_rank_equals_epilogue():
    """world = 1: the reduce-scatter + epilogue + all-gather kernel is the plain exact epilogue (bitwise vs
    ex_epilogue_i64), over two calls (the device epoch advances; every exchange word of the second call carries the
    new epoch)."""
    if not torch.cuda.is_available():
        pytest.skip("needs a GPU")
    _lib, K = _lib_mod()
    dev = torch.device("cuda", 0)
    M, N = 33, 1000
    parts, outs, flags, ctl, part_ptrs, out_ptrs, flag_ptrs = _one_gpu_peer_args(dev, M, N, 1)
    sx = torch.randint(10, 20, (M,), dtype=torch.int32, device=dev)
    sw = torch.randint(15, 20, (N,), dtype=torch.int32, device=dev)
    ref = torch.empty(M, N, dtype=torch.bfloat16, device=dev)
    K.exact_epilogue(parts[0], sx, sw, ref)
    st = torch.cuda.current_stream().cuda_stream
    for call in (1, 2):
        y = torch.full((M, N), float("nan"), dtype=torch.bfloat16, device=dev)
        _lib.check("ex_allreduce_epilogue_i64",
                   _lib.lib().ex_allreduce_epilogue_i64(part_ptrs.data_ptr(), N, out_ptrs.data_ptr(),
                                                        flag_ptrs.data_ptr(), ctl.data_ptr(), 0, 1, sx.data_ptr(),
                                                        sw.data_ptr(), M, N, y.data_ptr(), _lib.EX_DTYPE_BF16, N, st))
        assert torch.equal(y, ref)
        assert ctypes_code() == 0
        assert ctl.tolist() == [call, 0] and flags.tolist() == [call]  # epoch advanced, ready flag of this call
        assert bool(((outs[0].view(-1)[: M * N // 2] >> 32) == call).all())  # every exchange word carries the epoch


def test_peer_epilogue_missing_peer_times_out_with_status():
    """Failure detection without a GPU fault: a 'peer' that never signals (a flag nothing sets) makes the bounded
    waits run out (about 2 s for the first; the others give up once the error is recorded); the kernel records
    EX_DEVERR_WAIT_PEER (6), writes no output and the context stays usable."""
    if not torch.cuda.is_available():
        pytest.skip("needs a GPU")
    _lib, K = _lib_mod()
    dev = torch.device("cuda", 0)
    M, N = 4, 256
    parts, outs, flags, ctl, part_ptrs, out_ptrs, flag_ptrs = _one_gpu_peer_args(dev, M, N, 2, torch.float32)
    sx = torch.full((M,), 12, dtype=torch.int32, device=dev)
    sw = torch.full((N,), 17, dtype=torch.int32, device=dev)
    y = torch.full((M, N), 7.0, dtype=torch.float32, device=dev)
    assert ctypes_code() == 0
    st = torch.cuda.current_stream().cuda_stream
    _lib.check("ex_allreduce_epilogue_i64",
               _lib.lib().ex_allreduce_epilogue_i64(part_ptrs.data_ptr(), N, out_ptrs.data_ptr(), flag_ptrs.data_ptr(),
                                                    ctl.data_ptr(), 0, 2, sx.data_ptr(), sw.data_ptr(), M, N,
                                                    y.data_ptr(), _lib.EX_DTYPE_F32, N, st))
    assert ctypes_code() == 6
    assert bool((y == 7.0).all())  # nothing written
    z = torch.ones(8, device=dev) * 3  # the context still works
    assert float(z.sum()) == 24.0


def test_tp_digitize_one_rank_equals_digitize():
    """world = 1: the row-maxima exchange + digitize kernel gives exactly ex_digitize's digits (F = 14 and 15, bf16 and
    fp32 rows with an all-zero row and a subnormal-maximum row), over three calls on one set of exchange slots."""
    if not torch.cuda.is_available():
        pytest.skip("needs a GPU")
    _lib, K = _lib_mod()
    dev = torch.device("cuda", 0)
    max_rows = 64
    xch = torch.zeros(2 * max_rows, dtype=torch.int64, device=dev)
    xch_ptrs = torch.tensor([xch.data_ptr()], dtype=torch.int64, device=dev)
    ctl = torch.zeros(2, dtype=torch.int32, device=dev)
    st = torch.cuda.current_stream().cuda_stream
    g = torch.Generator().manual_seed(3)
    for call, (M, Kd, F, dt) in enumerate([(7, 1000, 14, torch.bfloat16), (64, 1536, 15, torch.float32),
                                           (3, 4096, 14, torch.bfloat16)], start=1):
        x = torch.randn(M, Kd, generator=g)
        x[0] = 0.0
        if M > 2:
            x[2] = 0.0
            x[2, 5] = 1e-40  # subnormal row maximum
        x = x.to(dt).to(dev)
        h, l, cs, sh = K._alloc_digits(M, Kd, dev)
        _lib.check("ex_tp_digitize",
                   _lib.lib().ex_tp_digitize(x.data_ptr(), K._DT[dt], x.stride(0), M, Kd, F, xch_ptrs.data_ptr(),
                                             max_rows, ctl.data_ptr(), 0, 1, h.data_ptr(), l.data_ptr(), h.stride(0),
                                             cs.data_ptr(), sh.data_ptr(), st))
        ref = K.digitize(x, F)
        for a, b in zip((h, l, cs, sh), ref):
            assert torch.equal(a, b), (M, Kd, F, dt)
        assert ctl.tolist() == [call, 0]
    assert ctypes_code() == 0
