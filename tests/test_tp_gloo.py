"""Row-parallel (K-sharded) exact linear across 2 CPU ranks over gloo: the host logic of vllm_exact.parallel (global
row maxima by MAX all-reduce, slice digitization, int64 SUM all-reduce, epilogue) must reproduce the 1-GPU result bit
for bit. The compute steps are served by the CPU oracle here (the `ops` hook of parallel.py); on GPUs they are the
sm_100a kernels."""
import os
import socket

import numpy as np
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


class OracleOps:
    @staticmethod
    def row_absmax(x):
        return torch.from_numpy(np.abs(x.float().numpy()).max(axis=1).astype(np.float32))

    @staticmethod
    def digitize_given(x, F, amax):
        from oracle import exact_oracle as O
        return [torch.from_numpy(t) for t in O.digitize(x.float().numpy(), F, amax=amax.numpy())]

    @staticmethod
    def partial(xd, wd, F, trunc):
        from oracle import exact_oracle as O
        return torch.from_numpy(O.exact_linear_i64([t.numpy() for t in xd], [t.numpy() for t in wd], F, trunc))

    @staticmethod
    def epilogue(tot, sx, sw, dtype):
        from oracle import exact_oracle as O
        return torch.from_numpy(O.epilogue(tot.numpy(), sx.numpy(), sw.numpy())).to(dtype)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, root, result_q):
    import sys
    for p in (root, os.path.join(root, "vllm-exact_b200"), os.path.join(root, "tests", "golden")):
        sys.path.insert(0, p)
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    try:
        from oracle import exact_oracle as O
        from vllm_exact import parallel as Par
        import recipes as R
        out = {}
        for (M, N, Kd), F, tr, cuts in [((24, 384, 4096), 14, True, [0, 2048, 4096]),
                                        ((5, 200, 1000), 15, False, [0, 600, 1000]),
                                        ((7, 33, 512), 14, False, [0, 100, 512])]:
            x, w = R.extreme_digits(M, N, Kd)
            x[1] *= 1e-3            # a row whose maximum lives on one shard only
            x[2, : Kd // 2] = 0.0   # a row that is all zero on rank 0's shard
            a, b = cuts[rank], cuts[rank + 1]
            wd = Par.digitize_weight_row_sharded(w[:, a:b].contiguous(), F, ops=OracleOps)
            y = Par.row_parallel_linear(x[:, a:b].contiguous(), *wd, F, tr, ops=OracleOps, out_dtype=torch.float32)
            ref = O.exact_linear(O.digitize(x.numpy(), F), O.digitize(w.numpy(), F), F, tr)
            out[(M, N, Kd, F)] = bool(np.array_equal(y.numpy().view(np.uint32), ref.view(np.uint32)))
        result_q.put((rank, out))
    finally:
        dist.destroy_process_group()


def test_row_parallel_two_ranks_bitexact():
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, root, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=300) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for r in range(2):
        assert all(res[r].values()), res[r]


def _worker_peer_agreement(rank, world, port, root, result_q):
    """parallel.peer_for on 2 CPU ranks with the device steps of PeerRowParallel faked: a failure on one rank (no IPC
    handle, or a peer mapping that cannot be opened) gives None on every rank, success gives an object on every rank,
    and asking again takes no collective step."""
    import datetime
    import sys
    for p in (root, os.path.join(root, "vllm-exact_b200")):
        sys.path.insert(0, p)
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=30))
    try:
        from vllm_exact import _lib, parallel as Par
        torch.cuda.synchronize = lambda *a, **k: None  # no device here: the buffers are CPU tensors
        out = {}
        for case in ("handle_fails", "open_fails", "ok"):
            def handle(self, t, case=case):
                if case == "handle_fails" and rank == 1:
                    raise _lib.ExactError("ex_ipc_get_handle", 1, "faked")
                return (b"h%d" % rank, 0)

            def open_(self, h, case=case):
                if case == "open_fails" and rank == 1:
                    raise _lib.ExactError("ex_ipc_open_handle", 1, "faked")
                return 4096

            Par.PeerRowParallel._handle, Par.PeerRowParallel._open = handle, open_
            Par._PEERS.clear()
            g = dist.group.WORLD
            first = Par.peer_for("cpu", g, create=True)
            again = Par.peer_for("cpu", g, create=True)  # cached: no collective step (a lone one would time out)
            out[case] = (first is not None, again is first)
        # the path switched off: no object, no collective step
        Par._PEERS.clear()
        rows, Par.PEER_ROWS = Par.PEER_ROWS, 0
        out["off"] = (Par.peer_for("cpu", dist.group.WORLD, create=True) is not None, True)
        Par.PEER_ROWS = rows
        dist.barrier()
        result_q.put((rank, out))
    finally:
        dist.destroy_process_group()


def test_peer_path_made_on_every_rank_or_none():
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker_peer_agreement, args=(r, 2, port, root, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=300) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for r in range(2):
        assert res[r] == {"handle_fails": (False, True), "open_fails": (False, True), "ok": (True, True),
                          "off": (False, True)}, res[r]
