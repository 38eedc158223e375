"""Tensor-parallel path on 2 GPUs: column- and row-parallel shards of real slots, run through the CUDA GEMV, gathered /
all-reduced (NCCL over NVLink, or the fused exchange of p8_tp_gemv_allreduce over peer memory), against the oracle's
full GEMV. Skips with fewer than 2 GPUs. NVLS stays off (NCCL_NVLS_ENABLE=0) and the fused exchange uses plain peer
stores only."""
import os
import socket

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

if not torch.cuda.is_available() or torch.cuda.device_count() < 2:
    pytest.skip("needs 2 CUDA GPUs", allow_module_level=True)

import torch.multiprocessing as mp  # noqa: E402


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _rank(rank, world, port, name, q):
    import datetime
    import sys

    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        sys.path.insert(0, os.path.dirname(__file__))
        from conftest import load_fixture

        from pingala8_llm_b200 import tp
        from pingala8_llm_b200.ops import device_error

        f = load_fixture(name)
        x = torch.from_numpy(f.x).cuda()
        col = tp.ColumnParallel(f.slot, f.K, f.rows, world, rank, unit=32)
        yc = col(x)
        n = torch.tensor([yc.numel()], device="cuda")
        ns = [torch.zeros_like(n) for _ in range(world)]
        dist.all_gather(ns, n)
        parts = [torch.zeros(int(v.item()), device="cuda") for v in ns]
        dist.all_gather(parts, yc)
        row = tp.RowParallel(f.slot, f.K, f.rows, world, rank)
        yr = row(x[row.lo:row.hi].contiguous())
        # batched (prefill) path: column shards gathered along the output columns, row shards all-reduced
        X = torch.from_numpy(f.X).cuda()
        Yc = col.mul_mat(X).contiguous()
        ws_ = [torch.zeros(X.shape[0], int(v.item()), device="cuda") for v in ns]
        dist.all_gather(ws_, Yc)
        Yr = row.mul_mat(X[:, row.lo:row.hi].contiguous())
        torch.cuda.synchronize()
        q.put((rank, torch.cat(parts).cpu().numpy(), yr.cpu().numpy(), device_error(), torch.cat(ws_, 1).cpu().numpy(),
               Yr.cpu().numpy()))
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("name", ["c1_1024x2560_c3", "cls3_64x512"])
def test_tp2_column_and_row_parallel(name):
    import sys

    sys.path.insert(0, os.path.dirname(__file__))
    from conftest import load_fixture

    f = load_fixture(name)
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_rank, args=(r, world, port, name, q)) for r in range(world)]
    for p in ps:
        p.start()
    res = [q.get(timeout=300) for _ in range(world)]
    for p in ps:
        p.join(timeout=120)
        assert p.exitcode == 0
    rel = lambda a: float(np.linalg.norm(a - f.y_ref) / np.linalg.norm(f.y_ref))
    relY = lambda a: float(np.linalg.norm(a - f.Y_ref) / np.linalg.norm(f.Y_ref))
    for rank, yc, yr, err, Yc, Yr in res:
        assert err == 0
        assert rel(yc) < 1e-5, (rank, rel(yc))
        assert rel(yr) < 1e-5, (rank, rel(yr))
        assert relY(Yc) < 1e-3 and relY(Yr) < 1e-3, (rank, relY(Yc), relY(Yr))  # the batched product's fp16 bar


def _rank_fused(rank, world, port, name, q):
    import datetime
    import sys

    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    graph = None
    try:
        sys.path.insert(0, os.path.dirname(__file__))
        from conftest import load_fixture

        from pingala8_llm_b200 import tp
        from pingala8_llm_b200.ops import device_error

        f = load_fixture(name)
        x = torch.from_numpy(f.x).cuda()
        comm = tp.TpComm.connect(max_rows=f.rows, timeout_ms=5000)
        row = tp.RowParallel(f.slot, f.K, f.rows, world, rank, comm=comm)
        assert row.comm is comm
        xl = x[row.lo:row.hi].contiguous()
        eager = [row(xl).clone() for _ in range(3)]
        # captured: replays advance the exchange parity through the device counter
        st = torch.cuda.Stream()
        out = torch.empty(f.rows, device="cuda")
        ws = row.t.workspace(1)
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.stream(st):
            with torch.cuda.graph(graph, stream=st):
                row(xl, out=out, workspace=ws, stream=st)
        replays = []
        for _ in range(5):
            graph.replay()
            replays.append(out.clone())
        torch.cuda.synchronize()
        err = device_error()
        epoch = comm.epoch()
        # a rank that skips a call: the other's bounded wait runs out (bit 3); both reset between steps and go on
        short = tp.TpComm.connect(max_rows=f.rows, timeout_ms=200)
        row_s = tp.RowParallel(f.slot, f.K, f.rows, world, rank, comm=short)
        if rank == 0:
            row_s(xl)
        torch.cuda.synchronize()
        err_skip = device_error()
        dist.barrier()
        short.reset()
        torch.cuda.synchronize()
        dist.barrier()
        after = row_s(xl).clone()
        torch.cuda.synchronize()
        err_after = device_error()
        ys = [y.cpu().numpy() for y in eager + replays + [after]]
        q.put((rank, ys, err, epoch, err_skip, err_after))
        dist.barrier()
    finally:
        graph = None
        dist.destroy_process_group()


@pytest.mark.parametrize("name,world", [("c1_1024x2560_c3", 2), ("cls3_64x512", 2), ("c1_1024x2560_c3", 4),
                                        ("c1_1024x2560_c3", 8)])
def test_tp_fused_row_parallel_exchange(name, world):
    """2, 4 or 8 ranks (skipped beyond the GPUs present): every rank gets the same bits on every call, eager and
    graph-replayed; a rank that skips a call makes rank 0's bounded wait run out, and a reset recovers."""
    import sys

    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} CUDA GPUs")
    sys.path.insert(0, os.path.dirname(__file__))
    from conftest import load_fixture

    f = load_fixture(name)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_rank_fused, args=(r, world, port, name, q)) for r in range(world)]
    for p in ps:
        p.start()
    res = sorted([q.get(timeout=300) for _ in range(world)], key=lambda r: r[0])
    for p in ps:
        p.join(timeout=120)
        assert p.exitcode == 0
    rel = lambda a: float(np.linalg.norm(a - f.y_ref) / np.linalg.norm(f.y_ref))
    y0 = res[0][1][0]
    for rank, ys, err, epoch, err_skip, err_after in res:
        assert err == 0 and err_after == 0
        assert epoch == 3 + 5
        assert err_skip == (8 if rank == 0 else 0)
        for y in ys:
            assert np.array_equal(y, y0)  # every call, every rank: the same bits
        assert rel(y0) < 1e-5, (rank, rel(y0))
