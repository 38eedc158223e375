"""C ABI of libpingala8_b200.so on the CPU: exports, host format helpers, loader checks, VR3, TP shards.

No GPU needed: these call only host entry points. Parity of the shard transforms is checked through the CPU oracle.
"""
import ctypes as C

import numpy as np
import pytest

import pingala8_llm_b200 as p8
from pingala8_llm_b200 import fmt, synth
from oracle.oracle import Oracle, RefOracle

from conftest import fixture_names, load_fixture


def test_library_exports_every_header_symbol():
    L = p8.lib()
    names = p8.header_functions()
    assert len(names) >= 20
    for n in names:
        assert hasattr(L, n), f"{n} declared in include/pingala8.h but not exported"


def test_status_strings():
    for s in p8.P8_STATUS:
        assert p8.lib().p8_status_str(s)


@pytest.mark.parametrize("name", fixture_names())
def test_golden_slots_pass_loader_checks(name):
    f = load_fixture(name)
    fmt.check_slot(f.slot, f.K, f.rows)


@pytest.mark.parametrize("name", fixture_names())
def test_assemble_reproduces_golden_slot(name):
    """p8_slot_assemble (vr_native_load CU:3527-3580) rebuilds the fixture slot byte for byte."""
    f = load_fixture(name)
    kb, c16, prm, (dr, dc, dv), signs = fmt.split_kernel_bytes(f.slot, f.K, f.rows)
    out = fmt.assemble_slot(kb, f.rows, f.K, c16, prm, dr, dc, dv if len(dv) else None, signs)
    assert out.size == f.meta["slot_nbytes"]
    assert np.array_equal(out, f.slot)


@pytest.mark.skipif(not RefOracle.available(), reason="reference CPU core not built")
def test_need_and_offsets_match_reference_contract():
    rng = np.random.default_rng(3)
    for _ in range(200):
        rows = 32 * int(rng.integers(1, 1000))
        K = 256 * int(rng.integers(1, 60))
        nd = int(rng.integers(0, 5000))
        kb = int(rng.integers(2064, 10**7))
        assert fmt.slot_need(kb, rows, K, nd) == RefOracle.need(kb, rows, K, nd)
        n = int(rng.integers(10**5, 10**8))
        o = fmt.slot_offsets(n, rows, K, nd)
        assert tuple(o[k] for k in ("E", "C", "P", "Q", "SG", "T")) == RefOracle.offsets(n, rows, K, nd)


def _corrupt(slot, K, rows, what):
    s = slot.copy()
    tr = s[-32:].view(np.uint32)
    nd = int(tr[3])
    o = fmt.slot_offsets(s.size, rows, K, nd)
    if what == "magic":
        s[-32] ^= 1
    elif what == "rows":
        s[-16:-12] = np.array([rows + 32], np.uint32).view(np.uint8)
    elif what == "ns":
        s[-8:-4] = np.array([104], np.uint32).view(np.uint8)
    elif what == "hdr_ns":
        s[2052:2056] = np.array([116], np.uint32).view(np.uint8)
    elif what == "class":  # change a tile's class: payload size no longer matches
        m = s[2064:2068].view(np.uint32).copy()
        m[0] = (m[0] & 0x1FFFFFFF) | (((int(m[0]) >> 29) % 7 + 1) << 29)
        s[2064:2068] = m.view(np.uint8)
    elif what == "prm":
        p = s[o["P"] : o["P"] + 2 * rows].view(np.int16)
        p[1] = p[0]
    elif what == "sign":
        s[o["SG"] + 3] = 0
    elif what == "kbytes":
        s[-24:-20] = np.array([int(tr[2]) + 16], np.uint32).view(np.uint8)
    return s


@pytest.mark.parametrize(
    "what,status",
    [("magic", -2), ("rows", -2), ("ns", -2), ("hdr_ns", -3), ("class", -4), ("prm", -5), ("sign", -7), ("kbytes", -4)],
)
def test_loader_checks_reject_corrupted_slots(what, status):
    """Host fault injection: each reference loader check (CU:3411-3580) rejects its corruption with a status."""
    f = load_fixture("mix_256x1024_sal")
    bad = _corrupt(f.slot, f.K, f.rows, what)
    assert fmt.slot_status(bad, f.K, f.rows) == status


def test_delta_out_of_range_rejected():
    s = synth.make_slot(64, 512, seed=4, nd=3)
    tr = s[-32:].view(np.uint32)
    o = fmt.slot_offsets(s.size, 64, 512, int(tr[3]))
    bad = s.copy()
    bad[o["E"] : o["E"] + 2] = np.array([64], np.uint16).view(np.uint8)  # row 64 of 64
    assert fmt.slot_status(bad, 512, 64) == -6
    assert fmt.slot_status(s, 512, 64) == 0


def test_shape_checks():
    s = synth.make_slot(64, 512, seed=1)
    assert fmt.slot_status(s, 512 + 1, 64) == -9
    assert fmt.slot_status(s, 512, 65) == -9
    with pytest.raises(p8.P8Error):
        synth.make_slot(32768, 256)


def _vr3_from_v2(kb, rows, K, c):
    """VR3 file bytes of a single-class v2 tensor (natural M order): header | tag | S | D (llama-vr3.h layout)."""
    nt = (rows // 32) * (K // 256)
    w515 = np.array([0x56523300 | c], np.uint32).view(np.uint8)
    S = kb[2064 + 4 * nt : 2064 + 68 * nt]
    D = kb[fmt.off_d(rows, K) :]
    return np.concatenate([kb[:2060], w515, S, D])


@pytest.mark.parametrize("name", ["c1_1024x2560_c3", "cls1_64x512", "cls7_256x1024"])
def test_vr3_expand_matches_reference(name):
    f = load_fixture(name)
    kb = fmt.split_kernel_bytes(f.slot, f.K, f.rows)[0]
    c = int(np.argmax(f.meta["class_hist"]))
    v3 = _vr3_from_v2(kb, f.rows, f.K, c)
    out, rows = fmt.vr3_expand(v3, f.K)
    assert rows == f.rows and np.array_equal(out, kb)
    if RefOracle.available():
        r, kbn = RefOracle.vr3_rows(v3.size, f.K, 0x56523300 | c)
        assert (r, kbn) == (f.rows, kb.size)
        assert np.array_equal(RefOracle.vr3_expand(v3, f.rows, f.K, kbn), out)
    # negative cases of the reference's own C test (research/detail/b3p_vr3_test.c): size, tag, class 0
    assert fmt.vr3_rows(v3.size - 4, f.K, 0x56523300 | c)[0] == 0
    assert fmt.vr3_rows(v3.size, f.K, (0x56523300 | c) ^ 0x100)[0] == 0
    assert fmt.vr3_rows(v3.size, f.K, 0x56523300)[0] == 0


@pytest.mark.parametrize("name", ["mix_256x1024_sal", "cls5_64x512", "c1_1024x2560_c3"])
def test_tp_shard_cols_exact(name):
    """Row-parallel shard on 256-column blocks: its dequant is the column slice of the full dequant, bit for bit,
    and the shard products sum to the full product."""
    f = load_fixture(name)
    W = Oracle(f.slot, f.rows, f.K).dequant()
    nb = f.K // 256
    cuts = [0, nb // 2, nb] if nb > 1 else [0, 1]
    y = np.zeros(f.rows)
    for b0, b1 in zip(cuts[:-1], cuts[1:]):
        sh = fmt.shard_cols(f.slot, f.K, f.rows, b0, b1)
        fmt.check_slot(sh, 256 * (b1 - b0), f.rows)
        o = Oracle(sh, f.rows, 256 * (b1 - b0))
        assert np.array_equal(o.dequant().view(np.uint32), W[:, 256 * b0 : 256 * b1].view(np.uint32))
        y += o.mul_mat(f.x[256 * b0 : 256 * b1])[0]
    assert np.linalg.norm(y - f.y_ref) / np.linalg.norm(f.y_ref) < 1e-5


@pytest.mark.parametrize("name,seed", [("c1_1024x2560_c3", 0), ("cls2_64x512", 1), ("cls7_256x1024", 2)])
def test_tp_shard_rows_exact(name, seed):
    """Column-parallel shard on ORIGINAL rows: re-tiled rows (lane rotation remapped) dequantise bit for bit."""
    f = load_fixture(name)
    W = Oracle(f.slot, f.rows, f.K).dequant()
    R = f.rows // 2 if f.rows >= 64 else 32
    for r0 in (0, f.rows - R):
        sh, orig = fmt.shard_rows(f.slot, f.K, f.rows, r0, r0 + R)
        fmt.check_slot(sh, f.K, R)
        assert sorted(orig.tolist()) == list(range(r0, r0 + R))
        Ws = Oracle(sh, R, f.K).dequant()
        assert np.array_equal(Ws.view(np.uint32), W[r0 : r0 + R].view(np.uint32))


def test_tp_shard_rows_rejects_mixed_classes():
    f = load_fixture("mix_256x1024_sal")
    with pytest.raises(p8.P8Error) as e:
        fmt.shard_rows(f.slot, f.K, f.rows, 0, 128)
    assert e.value.status == -13


def test_synthetic_slots_valid_and_decodable():
    for cls in range(1, 8):
        rows, K = (64, 512) if cls < 7 else (256, 1024)  # class 7 needs a larger tensor to fit a Q6_K slot
        s = synth.make_slot(rows, K, classes=cls, seed=cls, nd=5, c16="random")
        fmt.check_slot(s, K, rows)
        o = Oracle(s, rows, K)
        W = o.dequant()
        assert np.isfinite(W).all() and o.nd == 5


def test_tp_comm_create_checks_arguments_before_touching_the_device():
    """p8_tp_comm_create refuses bad rank / world / rows / timeout with P8_ERR_ARG (no CUDA call is made for them)."""
    from pingala8_llm_b200._lib import lib

    h = C.c_void_p()
    for rank, world, rows, tmo in [(0, 0, 64, 100), (0, 9, 64, 100), (2, 2, 64, 100), (-1, 2, 64, 100), (0, 2, 0, 100),
                                   (0, 2, 1 << 25, 100), (0, 2, 64, 0), (0, 2, 64, 600001)]:
        assert lib().p8_tp_comm_create(rank, world, rows, tmo, C.byref(h)) == -1, (rank, world, rows, tmo)
        assert not h.value
    assert lib().p8_tp_comm_create(0, 2, 64, 100, None) == -1
    assert lib().p8_tp_comm_destroy(None) == -1
    assert lib().p8_tp_gemv_allreduce(None, None, None, None, None, 0, None) == -12
