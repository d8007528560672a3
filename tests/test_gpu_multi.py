"""Row-sharded GEMV with the fused NVLink all-gather, on 2 GPUs (one process
per GPU). Each rank quantizes only its rows; the gathered output must be
bit-identical to the unsharded product (row sharding preserves the
reference's bits), over several calls and across CUDA-graph replays (the
call epoch lives on the device). Skipped when fewer than 2 GPUs are visible."""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, result_dir):
    import datetime
    import torch
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    msg = "ok"
    try:
        import quicklm_b200 as q
        from oracle.oracle import synth_case
        x_np, w_np = synth_case(1, 6144, 2048, 0)
        wd = torch.from_numpy(w_np).cuda()
        b, e = q.shard_rows(6144, world, rank)
        shard = q.Int8Weight.quantize(wd, device=rank, row_begin=b, row_end=e)
        full = q.Int8Weight.quantize(wd, device=rank)

        def exchange(h):
            out = [None] * world
            dist.all_gather_object(out, h)
            return out

        comm = q.Comm(rank, rank, world, 6144, exchange)
        rng = np.random.default_rng(11)
        xs = [torch.from_numpy(rng.standard_normal((1, 2048)).astype(np.float32)).cuda() for _ in range(4)]
        for i, x in enumerate(xs):
            y = q.matmul_allgather(x, shard, comm, flags=q.SYNC)
            y_ref = q.matmul(x, full, flags=q.SYNC)
            if not torch.equal(y.view(torch.int32), y_ref.view(torch.int32)):
                msg = f"call {i}: gathered output differs from the unsharded product"
                break
        if msg == "ok":
            # graph replay: the same captured calls must keep gathering fresh results
            s = torch.cuda.Stream()
            xin = torch.empty((1, 2048), device="cuda")
            yout = torch.empty((1, 6144), device="cuda")
            xin.copy_(xs[0])
            with torch.cuda.stream(s):
                q.matmul_allgather(xin, shard, comm, yout, stream=s)
            torch.cuda.synchronize()
            dist.barrier()
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=s):
                q.matmul_allgather(xin, shard, comm, yout, stream=s)
            torch.cuda.synchronize()
            dist.barrier()
            for i, x in enumerate(xs):
                xin.copy_(x)
                torch.cuda.synchronize()
                dist.barrier()
                g.replay()
                torch.cuda.synchronize()
                y_ref = q.matmul(x, full, flags=q.SYNC)
                if not torch.equal(yout.view(torch.int32), y_ref.view(torch.int32)):
                    msg = f"replay {i}: gathered output differs"
                    break
            del g
        if q.load().qlm_device_status(rank, 1) != 0:
            msg = "device status reports a timeout"
        dist.barrier()
        comm.free()
    except Exception as exc:  # reported through the result file
        msg = f"{type(exc).__name__}: {exc}"
    finally:
        with open(os.path.join(result_dir, f"r{rank}"), "w") as f:
            f.write(msg)
        dist.destroy_process_group()


def test_fused_allgather_two_gpus(tmp_path, qlm_lib):
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp
    world = 2
    mp.start_processes(_worker, args=(world, _free_port(), str(tmp_path)), nprocs=world, join=True,
                       start_method="spawn")
    for r in range(world):
        assert (tmp_path / f"r{r}").read_text() == "ok"
