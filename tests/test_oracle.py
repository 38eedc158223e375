"""The CPU oracle (oracle/p8_oracle.c) pinned against the reference's own outputs.

Golden values come from tests/golden/gen_fixtures.py, which ran the reference's Python encoder/decoders
(research/detail/r48k.py, r51_transcode.py) and its CPU core (vr-native-cpu-core.h, compiled from the patch).
"""
import hashlib

import numpy as np
import pytest

from oracle.oracle import Oracle, RefOracle


def sha(a):
    a = np.ascontiguousarray(a)
    if a.dtype.kind == "f":
        a = a + a.dtype.type(0)  # by value: the reference decoders disagree on signed zeros
    return hashlib.sha256(a.tobytes()).hexdigest()


def rel(a, b):
    return float(np.linalg.norm(np.asarray(a, np.float64) - b) / np.linalg.norm(b))


def test_golden_kernel_byte_sizes(golden):
    """kernel-byte size implied by the M words == the size the reference transcoder wrote (CU:46-51)."""
    o = Oracle(golden.slot, golden.rows, golden.K)
    assert o.kbytes == golden.meta["kbytes"]
    if golden.name == "c1_1024x2560_c3":
        assert o.kbytes == 679184  # 1024x2560 class 3, logs/csq/check.log:2


def test_decode_matches_reference_port(golden):
    """exact ints * S (sorted rows) == r51_transcode.cpu_vr_port over the kernel bytes (r51_transcode.py:75-118)."""
    o = Oracle(golden.slot, golden.rows, golden.K)
    ints = o.decode_int().astype(np.float32)
    nt = (golden.rows // 32) * (golden.K // 256)
    S = np.frombuffer(golden.slot.tobytes(), np.float16, (golden.K // 256) * golden.rows, 2064 + 4 * nt)
    S = S.reshape(golden.K // 256, golden.rows).astype(np.float32)
    assert sha(ints * np.repeat(S.T, 256, axis=1)) == golden.meta["sha_port_vs"]


def test_dequant_matches_encoder_weights(golden):
    """vrc_dequant_f32 semantics == the encoder's clamp(ifw(Yq)/c) by value (r48k.py:237, r51_delta.py)."""
    W = Oracle(golden.slot, golden.rows, golden.K).dequant()
    assert sha(W) == golden.meta["sha_wq_clamped"]


@pytest.mark.skipif(not RefOracle.available(), reason="reference CPU core not built (oracle/build_ref.py)")
def test_oracle_bit_exact_vs_reference_core(golden):
    o = Oracle(golden.slot, golden.rows, golden.K)
    r = RefOracle(golden.slot, golden.rows, golden.K)
    W, Wr = o.dequant(), r.dequant()
    assert np.array_equal(W.view(np.uint32), Wr.view(np.uint32))  # bit for bit, zero signs included
    for g in range(0, golden.rows // 32, max(1, golden.rows // 32 // 4)):
        for b in range(golden.K // 256):
            assert np.array_equal(o.decode_tile_int(g, b), r.decode_tile_int(g, b))


def test_gemv_x16_vs_reference_outputs(golden):
    """x16 GEMV / batch restated (vrc_tg CP:1161-1199; batch CP:1201-1262) vs the reference core's stored outputs."""
    o = Oracle(golden.slot, golden.rows, golden.K)
    y = o.mul_mat(golden.x)[0]
    assert rel(y, golden.y_ref) < 1e-6
    Y = o.mul_mat(golden.X)
    assert rel(Y, golden.Y_ref) < 1e-6
    # the x16 activation quantisation floor vs an fp64 product (reference: 1.08e-4 on 1024x2560)
    y64 = o.mul_mat_f64(golden.x)[0]
    assert rel(y, y64) < 3e-4


def test_get_rows_equals_dequant_rows(golden):
    o = Oracle(golden.slot, golden.rows, golden.K)
    W = o.dequant()
    ids = np.array([0, golden.rows - 1, golden.rows // 3, 7 % golden.rows], np.int32)
    assert np.array_equal(o.get_rows(ids).view(np.uint32), W[ids].view(np.uint32))


def test_planted_mistake_is_caught():
    """A flipped payload bit in a copy of the slot must change the oracle's decode (the checker can fail)."""
    from conftest import load_fixture

    f = load_fixture("cls3_64x512")
    bad = f.slot.copy()
    nt = (f.rows // 32) * (f.K // 256)
    offD = (2064 + 68 * nt + 15) & ~15
    bad[offD + 5] ^= 0x10
    assert not np.array_equal(Oracle(bad, f.rows, f.K).dequant(), Oracle(f.slot, f.rows, f.K).dequant())


def test_zbit_gather_identity():
    """The GEMV gathers the 32 stage-1 MSBs of a class-3 lane (8 words) with one multiply per word pair:
    x = (w[2p+1] & 0x80808080) | ((w[2p] >> 4) & 0x08080808); bits 24-31 of x * 0x00204081 = steps 8p..8p+7.
    Checked here against the bit-by-bit definition."""
    rng = np.random.default_rng(0)
    for w in rng.integers(0, 2**32, (3000, 8), dtype=np.uint64):
        ref = 0
        for k in range(32):
            ref |= ((int(w[k // 4]) >> (8 * (k % 4) + 7)) & 1) << k
        pm = 0
        for p in range(4):
            x = (int(w[2 * p + 1]) & 0x80808080) | ((int(w[2 * p]) >> 4) & 0x08080808)
            pm |= (((x * 0x00204081) & 0xFFFFFFFF) >> 24) << (8 * p)
        assert pm == ref
