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
        if msg == "ok":
            # uneven shards of an odd gathered width with ragged K: the second
            # exchange half starts at a width that is not a multiple of 4
            xo, wo = synth_case(1, 1001, 300, 5)
            wod = torch.from_numpy(wo).cuda()
            b2, e2 = q.shard_rows(1001, world, rank)
            shard2 = q.Int8Weight.quantize(wod, device=rank, row_begin=b2, row_end=e2)
            full2 = q.Int8Weight.quantize(wod, device=rank)
            comm2 = q.Comm(rank, rank, world, 1001, exchange)
            xod = torch.from_numpy(xo).cuda()
            y_ref = q.matmul(xod, full2, flags=q.SYNC)
            for i in range(3):  # both exchange halves
                y = q.matmul_allgather(xod, shard2, comm2, flags=q.SYNC)
                if not torch.equal(y.view(torch.int32), y_ref.view(torch.int32)):
                    msg = f"odd width, call {i}: gathered output differs"
                    break
            # the same exchange serves int4 shards
            shard4 = q.Int8Weight.quantize(wod, device=rank, row_begin=b2, row_end=e2, bits=4)
            full4 = q.Int8Weight.quantize(wod, device=rank, bits=4)
            y4_ref = q.matmul(xod, full4, flags=q.SYNC)
            for i in range(2):
                y4 = q.matmul_allgather(xod, shard4, comm2, flags=q.SYNC)
                if msg == "ok" and not torch.equal(y4.view(torch.int32), y4_ref.view(torch.int32)):
                    msg = f"int4, call {i}: gathered output differs"
            # greedy choice over a row-sharded lm_head: each rank reduces its own
            # logits, one word per rank crosses NVLink (QuickLM's sample(), model.cpp:259-272)
            from oracle.oracle import greedy_argmax
            y_loc = q.matmul(xod, shard2, flags=q.SYNC)  # this rank's shard of the logits
            full_logits = y_ref.cpu().numpy()[0]
            got = q.argmax(y_loc, comm2, col0=b2)
            if msg == "ok" and got[0] != greedy_argmax(full_logits):
                msg = f"sharded argmax {got} != {greedy_argmax(full_logits)}"
            cases = []
            t = np.random.default_rng(3).standard_normal(1001).astype(np.float32)
            t[[10, 900]] = 7.0  # equal maxima in different shards: the lower index wins
            cases.append(t.copy())
            t[0] = np.nan       # NaN at global index 0: the answer is 0
            cases.append(t.copy())
            t[:] = -np.inf
            t[600] = np.nan
            cases.append(t.copy())
            for v in cases:
                loc = torch.from_numpy(v[b2:e2].copy()).cuda()
                got = q.argmax(loc, comm2, col0=b2)
                if msg == "ok" and got[0] != greedy_argmax(v):
                    msg = f"sharded argmax case: {got} != {greedy_argmax(v)}"
            # gathers of different grid sizes (126 and 13 CTAs) and the
            # one-CTA argmax interleaved on one communicator: every CTA index
            # must see the call's epoch
            _, ws_ = synth_case(1, 100, 300, 6)
            wsd = torch.from_numpy(ws_).cuda()
            b3, e3 = q.shard_rows(100, world, rank)
            shard3 = q.Int8Weight.quantize(wsd, device=rank, row_begin=b3, row_end=e3)
            full3 = q.Int8Weight.quantize(wsd, device=rank)
            y3_ref = q.matmul(xod, full3, flags=q.SYNC)
            for i, which in enumerate((3, 2, 3, 3, "a", 2, 3, 2)):
                if which == "a":
                    loc = torch.from_numpy(cases[0][b2:e2].copy()).cuda()
                    got = q.argmax(loc, comm2, col0=b2)
                    ok = got[0] == greedy_argmax(cases[0])
                elif which == 3:
                    ok = torch.equal(q.matmul_allgather(xod, shard3, comm2, flags=q.SYNC).view(torch.int32),
                                     y3_ref.view(torch.int32))
                else:
                    ok = torch.equal(q.matmul_allgather(xod, shard2, comm2, flags=q.SYNC).view(torch.int32),
                                     y_ref.view(torch.int32))
                if msg == "ok" and not ok:
                    msg = f"interleaved grid sizes, call {i} ({which}): result differs"
            torch.cuda.synchronize()
            dist.barrier()
            comm2.free()
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


def _timeout_worker(rank, world, port, result_dir):
    """Rank 1 skips one call; rank 0's bounded wait must give up within its
    short limit and report QLM_ERR_TIMEOUT; the failed communicator refuses
    further calls at once; new communicators on both ranks work again. The
    failure is made on the host (a rank that does not call): nothing faults
    or hangs a GPU, every device wait is bounded."""
    import datetime
    import time
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
        x_np, w_np = synth_case(1, 1024, 512, 9)
        wd = torch.from_numpy(w_np).cuda()
        b, e = q.shard_rows(1024, world, rank)
        shard = q.Int8Weight.quantize(wd, device=rank, row_begin=b, row_end=e)
        full = q.Int8Weight.quantize(wd, device=rank)
        x = torch.from_numpy(x_np).cuda()
        y_ref = q.matmul(x, full, flags=q.SYNC)

        def exchange(h):
            out = [None] * world
            dist.all_gather_object(out, h)
            return out

        comm = q.Comm(rank, rank, world, 1024, exchange)
        comm.set_timeout(0.2)
        y = q.matmul_allgather(x, shard, comm, flags=q.SYNC)
        if not torch.equal(y.view(torch.int32), y_ref.view(torch.int32)):
            msg = "first call: gathered output differs"
        dist.barrier()
        if rank == 0:
            t0 = time.perf_counter()
            try:
                q.matmul_allgather(x, shard, comm, flags=q.SYNC)
                msg = "the call without its peer did not report a timeout"
            except q.QlmError as exc:
                dt = time.perf_counter() - t0
                if exc.status != 5:
                    msg = f"expected QLM_ERR_TIMEOUT, got {exc}"
                elif dt > 10.0:
                    msg = f"the timeout took {dt:.1f} s against a 0.2 s limit"
            t0 = time.perf_counter()
            try:  # a failed communicator refuses further work at once
                q.matmul_allgather(x, shard, comm, flags=q.SYNC)
                if msg == "ok":
                    msg = "a failed communicator accepted a call"
            except q.QlmError as exc:
                if msg == "ok" and (exc.status != 5 or time.perf_counter() - t0 > 1.0):
                    msg = f"failed communicator: {exc}"
            try:
                comm.status()
                if msg == "ok":
                    msg = "comm.status() did not report the failure"
            except q.QlmError:
                pass
        torch.cuda.synchronize()
        dist.barrier()  # rank 1 skipped the call: nothing of it is in flight anywhere
        comm.free()
        comm = q.Comm(rank, rank, world, 1024, exchange)
        comm.set_timeout(2.0)
        for i in range(3):
            y = q.matmul_allgather(x, shard, comm, flags=q.SYNC)
            if msg == "ok" and not torch.equal(y.view(torch.int32), y_ref.view(torch.int32)):
                msg = f"recreated communicator, call {i}: gathered output differs"
        comm.status()
        torch.cuda.synchronize()
        dist.barrier()
        comm.free()
    except Exception as exc:  # reported through the result file
        msg = f"{type(exc).__name__}: {exc}"
    finally:
        with open(os.path.join(result_dir, f"r{rank}"), "w") as f:
            f.write(msg)
        dist.destroy_process_group()


def test_gather_timeout_recovery_two_gpus(tmp_path, qlm_lib):
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    world = 2
    mp.start_processes(_timeout_worker, args=(world, _free_port(), str(tmp_path)), nprocs=world, join=True,
                       start_method="spawn")
    for r in range(world):
        assert (tmp_path / f"r{r}").read_text() == "ok"
