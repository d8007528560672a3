"""World-size-2 CPU tests (gloo) of the row-sharded path's host logic: the
product's row partition (shard_rows) and handle exchange (exchange_handles,
what Comm passes to qlm_comm_connect), and the assembly order of the gathered
output — checked against the unsharded product. The device data path is
covered by tests/test_gpu_multi.py on real GPUs."""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def test_shard_rows_partition():
    import quicklm_b200 as q
    for n in (1, 2, 7, 6144, 151936):
        for nr in (1, 2, 3, 4, 8):
            if nr > n:
                continue
            spans = [q.shard_rows(n, nr, r) for r in range(nr)]
            assert spans[0][0] == 0 and spans[-1][1] == n
            assert all(spans[i][1] == spans[i + 1][0] for i in range(nr - 1))
            sizes = [e - b for b, e in spans]
            assert max(sizes) - min(sizes) <= 1
    with pytest.raises(q.QlmError):
        q.shard_rows(10, 2, 2)


def _gloo_worker(rank, world, port, result_dir):
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        import quicklm_b200 as q
        from oracle.oracle import COracle, synth_case
        co = COracle()
        x, w = synth_case(1, 70, 96, 5)
        b, e = q.shard_rows(w.shape[0], world, rank)
        qs, ss = co.quantize(w[b:e])
        y_shard = co.matmul(x, qs, ss)[0]
        parts = [None] * world
        dist.all_gather_object(parts, (b, e, y_shard))

        def exchange(h):
            out = [None] * world
            dist.all_gather_object(out, h)
            return out

        # the product's handle exchange (what Comm passes to qlm_comm_connect)
        nb = 64
        allb = q.exchange_handles(bytes([rank]) * nb, world, exchange)
        ok_h = allb == b"".join(bytes([r]) * nb for r in range(world))
        try:  # a transport that loses a rank's handle is refused, not connected
            q.exchange_handles(bytes([rank]) * nb, world, lambda h: [h])
            ok_h = False
        except q.QlmError:
            pass
        y = np.empty(w.shape[0], np.float32)
        for (pb, pe, ys) in parts:
            y[pb:pe] = ys
        qf, sf = co.quantize(w)
        y_full = co.matmul(x, qf, sf)[0]
        ok = np.array_equal(y.view(np.uint32), y_full.view(np.uint32)) and ok_h
        with open(os.path.join(result_dir, f"r{rank}"), "w") as f:
            f.write("ok" if ok else "mismatch")
    finally:
        dist.destroy_process_group()


def test_sharded_gather_gloo(tmp_path, coracle):
    import torch.multiprocessing as mp
    world = 2
    mp.start_processes(_gloo_worker, args=(world, _free_port(), str(tmp_path)), nprocs=world, join=True,
                       start_method="spawn")
    for r in range(world):
        assert (tmp_path / f"r{r}").read_text() == "ok"
