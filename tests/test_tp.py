"""Tensor-parallel host logic on CPU: the split plan, shard transforms and the all-reduce of row-parallel partials,
run as world_size-2 gloo ranks with the oracle standing in for the per-rank GEMV (the GPU path is tested in
test_gpu_tp.py)."""
import os
import socket

import numpy as np
import pytest

torch = pytest.importorskip("torch")
import torch.distributed as dist  # noqa: E402
import torch.multiprocessing as mp  # noqa: E402

from pingala8_llm_b200 import tp  # noqa: E402


DIMS = {"llama3.1-8b": tp.LLAMA3_8B, "qwen3-14b": tp.QWEN3_14B, "qwen3-4b": tp.QWEN3_4B}


@pytest.mark.parametrize("model", sorted(DIMS))
@pytest.mark.parametrize("world", [1, 2, 3, 4, 8])
def test_layer_plan_covers_and_pairs(model, world):
    d = DIMS[model]
    plans = [tp.layer_plan(d, world, r) for r in range(world)]
    for n in ("q", "k", "v", "o", "gate", "up", "down"):
        e0 = plans[0][n]
        total = e0.rows if e0.kind == "col" else e0.K
        got = [(p[n].lo, p[n].hi) for p in plans]
        assert got[0][0] == 0 and got[-1][1] == total
        assert all(a[1] == b[0] for a, b in zip(got, got[1:]))        # contiguous, no overlap
        assert all((hi - lo) % e0.unit == 0 for lo, hi in got)
        for p in plans:
            e = p[n]
            if e.kind == "col":
                assert e.lo % 32 == 0 and e.hi % 32 == 0              # whole 32-row tiles
            else:                                                     # the shard's blocks cover the rank's columns
                assert e.b0 == e.lo // 256 and e.b1 == (e.hi + 255) // 256 and e.shard_K == 256 * (e.b1 - e.b0)
                assert 256 * e.b0 <= e.lo <= e.hi <= 256 * e.b1
    for p in plans:  # each rank feeds its row-parallel projections from its own column-parallel outputs
        assert p["o"][2:4] == p["q"][2:4] and p["down"][2:4] == p["gate"][2:4] == p["up"][2:4]
        # GQA: the rank's query heads use exactly the rank's KV heads (group = heads / kv_heads), at every world size
        g = d.heads // d.kv_heads
        qh = (p["q"].lo // d.head_dim, p["q"].hi // d.head_dim)
        kh = (p["k"].lo // d.head_dim, p["k"].hi // d.head_dim)
        assert qh == (kh[0] * g, kh[1] * g) and p["v"][2:4] == p["k"][2:4]


def test_qwen3_14b_tp8_o_shards_share_boundary_blocks():
    """Qwen3-14B at TP8: 5 query heads = 640 o-input columns per rank, 2.5 Hadamard blocks: neighbours share a block"""
    plans = [tp.layer_plan(tp.QWEN3_14B, 8, r) for r in range(8)]
    assert [(p["o"].lo, p["o"].hi) for p in plans] == [(640 * r, 640 * (r + 1)) for r in range(8)]
    assert [(p["o"].b0, p["o"].b1) for p in plans] == [(0, 3), (2, 5), (5, 8), (7, 10), (10, 13), (12, 15), (15, 18), (17, 20)]
    assert sum(p["down"].b1 - p["down"].b0 for p in plans) == 17408 // 256   # down: whole blocks, 9/9/9/9/8/8/8/8


def test_unaligned_row_shards_sum_to_the_whole_product():
    """Row-parallel shards over an unaligned column split (a boundary block held by both ranks, each rank's input zero
    outside its columns) sum to the unsharded product: the Hadamard transform is linear. Oracle GEMVs on the CPU."""
    import sys

    sys.path.insert(0, os.path.dirname(__file__))
    from conftest import load_fixture
    from oracle.oracle import Oracle

    f = load_fixture("mix_256x1024_sal")  # K = 1024: 4 blocks; split at 640 (inside block 2)
    y_full = Oracle(f.slot, f.rows, f.K).mul_mat(f.x)[0]
    total = np.zeros(f.rows, np.float64)
    for rank, (lo, hi) in enumerate([(0, 640), (640, 1024)]):
        sh = tp.row_shard(f.slot, f.K, f.rows, 2, rank, cols=(lo, hi))
        b0 = lo // 256
        xs = np.zeros(sh.K, np.float32)
        xs[lo - 256 * b0:hi - 256 * b0] = f.x[lo:hi]
        total += Oracle(sh.slot, f.rows, sh.K).mul_mat(xs)[0]
    rel = np.linalg.norm(total - y_full) / np.linalg.norm(y_full)
    assert rel < 1e-3, rel  # each rank quantises its own masked block (x16), so the sum is within the x16 floor


def test_balanced_split_uneven():
    sizes = [tp.balanced(10, 4, r) for r in range(4)]
    assert sizes == [(0, 2), (2, 5), (5, 7), (7, 10)]
    assert tp.balanced(1, 2, 0) == (0, 0) and tp.balanced(1, 2, 1) == (0, 1)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _rank_main(rank, world, port, name, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        import sys

        sys.path.insert(0, os.path.join(os.path.dirname(__file__)))
        from conftest import load_fixture
        from oracle.oracle import Oracle

        f = load_fixture(name)
        o_full = Oracle(f.slot, f.rows, f.K)
        y_full = o_full.mul_mat(f.x)[0]
        # column-parallel: the rank's slice of y, gathered
        c = tp.column_shard(f.slot, f.K, f.rows, world, rank, unit=32)
        yc = torch.from_numpy(Oracle(c.slot, c.rows, f.K).mul_mat(f.x)[0].astype(np.float32))
        sizes = [torch.zeros(1, dtype=torch.int64) for _ in range(world)]
        dist.all_gather(sizes, torch.tensor([yc.numel()]))
        parts = [torch.zeros(int(s.item())) for s in sizes]
        dist.all_gather(parts, yc)
        col = torch.cat(parts).numpy()
        # row-parallel: partial y over the rank's 256-column blocks, summed by the same helper the GPU path uses
        r = tp.row_shard(f.slot, f.K, f.rows, world, rank)
        yp = torch.from_numpy(Oracle(r.slot, f.rows, r.K).mul_mat(f.x[r.lo:r.hi])[0].astype(np.float32))
        tp.reduce_partials(yp)
        rel = lambda a: float(np.linalg.norm(a - y_full) / np.linalg.norm(y_full))
        q.put((rank, rel(col), rel(yp.numpy()), (c.lo, c.hi), (r.lo, r.hi)))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("name", ["c1_1024x2560_c3", "cls4_64x512"])
def test_tp_world2_gloo_matches_full_gemv(name):
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_rank_main, args=(r, world, port, name, q)) for r in range(world)]
    for p in ps:
        p.start()
    res = [q.get(timeout=300) for _ in range(world)]
    for p in ps:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, rc, rr, cr, rrng in res:
        assert rc < 1e-6, (rank, rc)
        assert rr < 1e-5, (rank, rr)
