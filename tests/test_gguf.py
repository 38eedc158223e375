"""Model files: the native GGUF reader and Pingala-8 loader (p8_gguf_*) against files written by an independent writer
(gguf-py). Slots read back must equal the slots they were made from, byte for byte; every check of the reference
loader (vr_native_init / vr_native_load, CU:3411-3580) must refuse a file that breaks it."""
import numpy as np
import pytest

gguf = pytest.importorskip("gguf")

import pingala8_llm_b200 as p8  # noqa: E402
from pingala8_llm_b200 import fmt, synth  # noqa: E402
from pingala8_llm_b200.model_file import ModelFile  # noqa: E402

# one llama block at small width: (name, rows, K)
SHAPES = [("attn_q", 512, 512), ("attn_k", 256, 512), ("attn_v", 256, 512), ("attn_output", 512, 512),
          ("ffn_gate", 1024, 512), ("ffn_up", 1024, 512), ("ffn_down", 512, 1024)]


def _slots(permute=True, mixed=True):
    out = {}
    for i, (nm, rows, K) in enumerate(SHAPES):
        cls = 3
        if mixed and nm == "ffn_up":
            cls = np.random.default_rng(i).integers(1, 8, (rows // 32, K // 256))
        out[f"blk.0.{nm}.weight"] = (synth.make_slot(rows, K, classes=cls, seed=50 + i, nd=(5 if permute else 0),
                                                     permute=permute), rows, K)
    return out


def _vr3_file_bytes(kb, rows, K, c):
    """VR3 file tensor of a single-class slot with natural rows (llama-vr3.h): header | tag | S | D"""
    nt = (rows // 32) * (K // 256)
    w515 = np.array([0x56523300 | c], np.uint32).view(np.uint8)
    return np.concatenate([kb[:2060], w515, kb[2064 + 4 * nt : 2064 + 68 * nt], kb[fmt.off_d(rows, K) :]])


def _write(path, slots, layout=2, kv=None, drop=(), extra=None, block_count=1, n_linear=None, mutate=None):
    T = gguf.GGMLQuantizationType
    w = gguf.GGUFWriter(str(path), "llama")
    w.add_block_count(block_count)
    keys = {"vr.ns": 108, "vr.trl": 2, "vr.n_linear": len(slots) if n_linear is None else n_linear, "vr.layout": layout}
    keys.update(kv or {})
    w.add_string("vr.format", "pingala8")
    for k, v in keys.items():
        if v is not None:
            w.add_uint32(k, v)
    signs = None
    for name, (slot, rows, K) in slots.items():
        base = name[: -len(".weight")]
        kb, c16, prm, (drow, dcol, dval), signs = fmt.split_kernel_bytes(slot, K, rows)
        if layout == 3:
            c = int(slot[2064:2068].view(np.uint32)[0] >> 29)
            wb = _vr3_file_bytes(kb, rows, K, c)
        else:
            wb = kb
        if mutate:
            wb = mutate(name, wb)
        tensors = {f"{base}.weight": (wb.view(np.int8), T.I8), f"{base}.vr_c": (c16.copy(), T.F16)}
        if layout == 2:
            tensors[f"{base}.vr_prm"] = (prm.copy(), T.I16)
        if drow.size:
            tensors[f"{base}.vr_didx"] = (np.stack([drow, dcol]).view(np.int16), T.I16)
            tensors[f"{base}.vr_dval"] = (dval.copy(), T.F32)
        for tn, (arr, dt) in tensors.items():
            if tn not in drop:
                w.add_tensor(tn, arr, raw_dtype=dt)
    for tn, (arr, dt) in (extra or {}).items():
        w.add_tensor(tn, arr, raw_dtype=dt)
    if "vr.had_signs" not in drop:
        w.add_tensor("vr.had_signs", signs.copy(), raw_dtype=T.I8)
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()
    return path


def test_layout2_roundtrip(tmp_path):
    slots = _slots()
    with ModelFile(_write(tmp_path / "m.gguf", slots)) as mf:
        assert [li.name for li in mf.linears] == sorted(slots)
        for li in mf.linears:
            slot, rows, K = slots[li.name]
            assert (li.rows, li.K, li.layout, li.nbytes) == (rows, K, 2, slot.size)
            assert np.array_equal(mf.slot(li.name), slot)
            fmt.check_slot(mf.slot(li.index), K, rows)


def test_layout3_vr3_roundtrip(tmp_path):
    slots = _slots(permute=False, mixed=False)
    with ModelFile(_write(tmp_path / "m3.gguf", slots, layout=3)) as mf:
        for li in mf.linears:
            slot, rows, K = slots[li.name]
            assert (li.rows, li.K, li.layout) == (rows, K, 3)
            assert np.array_equal(mf.slot(li.name), slot)


def _status(path):
    with pytest.raises(p8.P8Error) as e:
        ModelFile(path)
    return e.value.status


def test_open_refuses_what_the_reference_loader_refuses(tmp_path):
    slots = _slots()
    one = dict(list(slots.items())[:1])
    assert _status(_write(tmp_path / "a.gguf", slots, kv={"vr.ns": 100})) == -17             # NS must be 108
    assert _status(_write(tmp_path / "b.gguf", slots, kv={"vr.ns": None})) == -17            # vr.ns missing
    assert _status(_write(tmp_path / "c.gguf", slots, kv={"vr.trl": 3})) == -17              # TRL must be 2
    assert _status(_write(tmp_path / "d.gguf", slots, kv={"vr.layout": 4})) == -17           # layout 2 or 3
    assert _status(_write(tmp_path / "e.gguf", slots, n_linear=6)) == -17                    # vr.n_linear count
    assert _status(_write(tmp_path / "f.gguf", one, n_linear=1, block_count=1)) == -17       # 7 per block
    name = next(iter(slots))[: -len(".weight")]
    assert _status(_write(tmp_path / "g.gguf", slots, drop=(f"{name}.vr_prm",))) == -17      # layout 2 needs vr_prm
    base_d = [n for n, (s, r, k) in slots.items() if int(s[-32:].view(np.uint32)[3])][0][: -len(".weight")]
    assert _status(_write(tmp_path / "h.gguf", slots, drop=(f"{base_d}.vr_dval",))) == -17   # didx without dval
    assert _status(_write(tmp_path / "i.gguf", slots, drop=("vr.had_signs",))) == -17
    s3 = _slots(permute=False, mixed=False)
    T = gguf.GGMLQuantizationType
    extra = {f"{next(iter(s3))[: -len('.weight')]}.vr_prm": (np.arange(512, dtype=np.int16), T.I16)}
    assert _status(_write(tmp_path / "j.gguf", s3, layout=3, extra=extra)) == -17             # no vr_prm in VR3
    p = _write(tmp_path / "k.gguf", slots)
    raw = bytearray(p.read_bytes())
    raw[0] ^= 0xFF
    (tmp_path / "k2.gguf").write_bytes(bytes(raw))
    assert _status(tmp_path / "k2.gguf") == -16                                              # not GGUF
    raw[0] ^= 0xFF
    (tmp_path / "k3.gguf").write_bytes(bytes(raw[: len(raw) - 100]))
    assert _status(tmp_path / "k3.gguf") == -16                                              # truncated
    assert _status(tmp_path / "missing.gguf") == -16


def test_load_refuses_bad_linears(tmp_path):
    slots = _slots()
    first = sorted(slots)[0]
    second = sorted(slots)[1]

    def other_codebook(name, wb):
        if name == second:
            wb = wb.copy()
            wb[4] ^= 1  # codebook word 1 of the second linear differs from the first's
        return wb

    with ModelFile(_write(tmp_path / "t.gguf", slots, mutate=other_codebook)) as mf:
        mf.slot(first)
        with pytest.raises(p8.P8Error) as e:
            mf.slot(second)
        assert e.value.status == -8  # P8_ERR_TABLES

    def short_payload(name, wb):
        return wb[:-64] if name == first else wb  # M words imply more payload than the tensor holds

    with ModelFile(_write(tmp_path / "u.gguf", slots, mutate=short_payload)) as mf:
        with pytest.raises(p8.P8Error):
            mf.slot(first)


@pytest.mark.gpu
def test_model_file_gemv_on_gpu(tmp_path):
    torch = pytest.importorskip("torch")
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA GPU")
    from oracle.oracle import Oracle

    slots = _slots()
    with ModelFile(_write(tmp_path / "g.gguf", slots)) as mf:
        for li in mf.linears:
            t = mf.tensor(li.name)
            x = np.random.default_rng(li.index).normal(0, 1, li.K).astype(np.float32)
            y = t.mul_mat_vec(torch.from_numpy(x).cuda()).cpu().numpy()
            ref = Oracle(slots[li.name][0], li.rows, li.K).mul_mat(x)[0]
            assert np.linalg.norm(y - ref) / np.linalg.norm(ref) < 1e-5
