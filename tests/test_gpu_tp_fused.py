"""Fused row-parallel GEMV + all-reduce (p8_tp_gemv_allreduce) on one GPU.

One rank's launch is checked against the exchange protocol with the other ranks played by the test, never by a second
waiting kernel: their partial rows (plain GEMVs of their shards) are written into this rank's exchange buffer before
the call, and their exchange buffers are local stand-ins whose contents are checked after it. The bounded wait is made
to run out by leaving a peer's entries empty (nothing sets them); the launch must return with device error bit 3 and
the context stays usable. The real multi-GPU exchange runs in test_gpu_tp.py.
"""
import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():
    pytest.skip("needs a CUDA GPU", allow_module_level=True)

from pingala8_llm_b200 import fmt, synth, tp  # noqa: E402
from pingala8_llm_b200.ops import P8Tensor, device_error  # noqa: E402
from oracle.oracle import Oracle  # noqa: E402


PRM = {}


def _entries(y, rows):
    """exchange entries (output-row order, int64 bit patterns) of partial output y of the tensor set up last"""
    return tp.exchange_entries(y, rows)


def _setup(rows, K, world, seed=3, nd=11):
    slot = synth.make_slot(rows, K, seed=seed, nd=nd)
    PRM["prm"] = fmt.split_kernel_bytes(slot, K, rows)[2]  # shards keep the tensor's row order
    assert sorted(PRM["prm"].tolist()) == list(range(rows)) and PRM["prm"].tolist() != list(range(rows))
    x = np.random.default_rng(seed).normal(0, 1, K).astype(np.float32)
    shards = [tp.row_shard(slot, K, rows, world, q) for q in range(world)]
    ts = [P8Tensor(s.slot, s.K, rows) for s in shards]
    xs = [torch.from_numpy(x[s.lo:s.hi].copy()).cuda() for s in shards]
    parts = [t.mul_mat_vec(xq) for t, xq in zip(ts, xs)]
    torch.cuda.synchronize()
    ref = Oracle(slot, rows, K).mul_mat(x[None])[0]
    return ts, xs, parts, ref


def _rank_order_sum(parts):
    s = parts[0].clone()
    for p in parts[1:]:
        s = s + p
    return s


@pytest.mark.parametrize("rows,K,world,rank", [(4096, 4096, 2, 0), (4096, 14336, 4, 2), (512, 2048, 8, 7),
                                               (96, 1024, 3, 1)])
def test_fused_rank_against_played_peers(rows, K, world, rank):
    ts, xs, parts, ref = _setup(rows, K, world)
    comm = tp.TpComm(rank, world, max_rows=rows + 64, timeout_ms=2000)
    stand_in = {q: torch.zeros(2, world, rows + 64, dtype=torch.int64, device="cuda") for q in range(world) if q != rank}
    for q, b in stand_in.items():
        comm.set_peer(q, b.data_ptr())
    own = comm.buffer()
    want = _rank_order_sum(parts)
    for call in range(3):  # parities 1, 0, 1
        par = (comm.epoch() + 1) & 1
        for q in range(world):
            if q != rank:
                own[par, q, :rows] = _entries(parts[q], rows)
        y = ts[rank].mul_mat_vec_allreduce(xs[rank], comm)
        torch.cuda.synchronize()
        assert device_error() == 0
        assert comm.epoch() == call + 1
        assert torch.equal(y, want)  # the same fp32 adds in rank order: bit-exact
        assert float(np.linalg.norm(y.cpu().numpy() - ref) / np.linalg.norm(ref)) < 1e-5
        for q, b in stand_in.items():  # this rank's partial rows stored into every peer's buffer, nothing else
            assert torch.equal(b[par, rank, :rows], _entries(parts[rank], rows))
            b[par, rank, :rows] = 0
            assert torch.all(b == 0)
        assert torch.all(own == 0)  # consumed entries cleared
    comm.close()


def test_fused_world_one_is_the_plain_gemv():
    rows, K = 1024, 2048
    ts, xs, parts, _ = _setup(rows, K, 1)
    comm = tp.TpComm(0, 1, max_rows=rows)
    y = ts[0].mul_mat_vec_allreduce(xs[0], comm)
    torch.cuda.synchronize()
    assert device_error() == 0
    assert torch.equal(y, parts[0])


def test_fused_graph_capture_replays_advance_the_parity():
    rows, K, world, rank = 2048, 4096, 2, 1
    ts, xs, parts, _ = _setup(rows, K, world, seed=8)
    comm = tp.TpComm(rank, world, max_rows=rows)
    peer0 = torch.zeros(2, world, rows, dtype=torch.int64, device="cuda")
    comm.set_peer(0, peer0.data_ptr())
    own = comm.buffer()
    ws = ts[rank].workspace(1)
    out = torch.empty(rows, device="cuda")
    st = torch.cuda.Stream()
    st.wait_stream(torch.cuda.current_stream())
    g = torch.cuda.CUDAGraph()
    with torch.cuda.stream(st):
        own[1, 0, :rows] = _entries(parts[0], rows)
        ts[rank].mul_mat_vec_allreduce(xs[rank], comm, out=out, workspace=ws, stream=st)  # call 1 (parity 1), eager
        st.synchronize()
        with torch.cuda.graph(g, stream=st):
            ts[rank].mul_mat_vec_allreduce(xs[rank], comm, out=out, workspace=ws, stream=st)
    want = _rank_order_sum(parts)
    for i in range(4):  # replays are calls 2..5: parity from the device counter, not from captured arguments
        par = (2 + i) & 1
        out.zero_()
        own[par, 0, :rows] = _entries(parts[0], rows)
        g.replay()
        torch.cuda.synchronize()
        assert device_error() == 0
        assert torch.equal(out, want)
        assert torch.equal(peer0[par, rank, :rows], _entries(parts[rank], rows))
    assert comm.epoch() == 5


def test_fused_wait_runs_out_and_reset_recovers():
    """A peer whose partial rows never arrive: the bounded wait gives up (bit 3), the context stays usable, and after
    a reset the next call is correct."""
    rows, K, world = 1024, 2048, 2
    ts, xs, parts, _ = _setup(rows, K, world, seed=5)
    comm = tp.TpComm(0, world, max_rows=rows, timeout_ms=50)
    peer1 = torch.zeros(2, world, rows, dtype=torch.int64, device="cuda")
    comm.set_peer(1, peer1.data_ptr())
    ts[0].mul_mat_vec_allreduce(xs[0], comm)
    torch.cuda.synchronize()
    assert device_error() & 8
    comm.reset()
    own = comm.buffer()
    own[1, 1, :rows] = _entries(parts[1], rows)
    y = ts[0].mul_mat_vec_allreduce(xs[0], comm)
    torch.cuda.synchronize()
    assert device_error() == 0
    assert torch.equal(y, _rank_order_sum(parts))


def test_fused_foreign_tag_is_reported():
    rows, K, world = 512, 1024, 2
    ts, xs, parts, _ = _setup(rows, K, world, seed=6)
    comm = tp.TpComm(0, world, max_rows=rows + 32)
    peer1 = torch.zeros(2, world, rows + 32, dtype=torch.int64, device="cuda")
    comm.set_peer(1, peer1.data_ptr())
    comm.buffer()[1, 1, :rows] = _entries(parts[1], rows + 32)  # written for a tensor of another row count
    ts[0].mul_mat_vec_allreduce(xs[0], comm)
    torch.cuda.synchronize()
    assert device_error() & 16
    comm.reset()
    e = _entries(parts[1], rows)
    comm.buffer()[1, 1, :rows] = torch.roll(e, 1)  # a peer whose shard has another row order
    ts[0].mul_mat_vec_allreduce(xs[0], comm)
    torch.cuda.synchronize()
    assert device_error() & 16


def test_fused_call_arguments_are_checked():
    rows, K = 512, 1024
    ts, xs, _, _ = _setup(rows, K, 2, seed=7)
    small = tp.TpComm(0, 2, max_rows=rows - 32)
    dummy = torch.zeros(2, 2, rows, dtype=torch.int64, device="cuda")
    small.set_peer(1, dummy.data_ptr())
    with pytest.raises(Exception):
        ts[0].mul_mat_vec_allreduce(xs[0], small)  # more rows than the exchange buffer holds
    unattached = tp.TpComm(0, 2, max_rows=rows)
    with pytest.raises(Exception):
        ts[0].mul_mat_vec_allreduce(xs[0], unattached)  # peer 1's buffer not attached
    with pytest.raises(Exception):
        unattached.set_peer(0, dummy.data_ptr())  # a rank is not its own peer
