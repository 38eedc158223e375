"""Offline trellis encoder (p8_encode_slice, pingala8_llm_b200.encoder) against the reference's own encoder.

Golden vectors: tests/golden/encoder_fixtures.npz, made by tests/golden/gen_encoder_fixtures.py with the reference's
research/detail/r48k.py encode (8 trellis states, production class shifts) on CPU: a mixed-class case (classes 0-7)
and a class-3 case with a random SPD Hessian (error feedback across the slice and across slices), and a mixed case
with H = I (no feedback).

CPU: the fixtures decode back to their own Q exactly through the format's trellis (the f1 MSBs drive the 8-state
recurrence, the coset offset of the state before each step is added) -- this pins the fixture and the code-to-value
rule the GPU test relies on. Values are compared, not bit patterns: the reference's float codebook holds some zero
entries as -0.0, so a zero value may carry the other sign. GPU: the encoder's codes decode to its Q bit for bit, and
its codes and values equal the reference's at every position. (The search is the reference's, operation for
operation where the reference fixes the order; its 4 x 4 products and the cuBLAS feedback GEMM between slices could
round differently in the last bit, which would flip a near-tie: on these fixtures none does.)
"""
import os

import numpy as np
import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
FIX = os.path.join(HERE, "golden", "encoder_fixtures.npz")
W1 = [0, 4, 6, 8, 8, 8, 8, 8]
W2 = [0, 0, 0, 0, 2, 4, 8, 8]
W3 = [0, 0, 0, 0, 0, 0, 0, 8]
S1 = [0, 0, 0, 0, 2, 3, 2, 4]
S2 = [0, 0, 0, 0, 0, 0, 0, 2]


def mc(k):
    return (1 << S1[k]) + ((1 << S2[k]) if W2[k] else 0) + (1 if W3[k] else 0)


def decode_idx(IDX, cls, Sb, A, c):
    """values of codes IDX [rows, n/4, 3] (natural rows): per 128-column slice the state starts at 0; at each step the
    coset offset of the current state (bit 1) is added, then the f1 MSB b moves the state to ((s << 1) | (b ^ s0 ^ s2)) & 7"""
    rows, nq, _ = IDX.shape
    n = 4 * nq
    A = A.astype(np.float32)
    c = c.astype(np.float32)
    Q = np.zeros((rows, n), np.float32)
    for r in range(rows):
        for b in range(n // 256):
            k = int(cls[r, b])
            if k == 0:
                continue
            S = np.float32(Sb[r, b])
            for sl in range(2):
                st = 0
                for t in range(32):
                    q = (b * 256 + sl * 128) // 4 + t
                    i1, i2, i3 = (int(v) for v in IDX[r, q])
                    v = A[i1] * np.float32(1 << S1[k])
                    if W2[k]:
                        v = v + A[i2] * np.float32(1 << S2[k])
                    if W3[k]:
                        v = v + A[i3]
                    v = v + np.float32((st >> 1) & 1) * (np.float32(mc(k)) * c)
                    Q[r, 4 * q:4 * q + 4] = (v * S).astype(np.float32)
                    bit = i1 >> (W1[k] - 1)
                    st = ((st << 1) | (bit ^ (st & 1) ^ ((st >> 2) & 1))) & 7
    return Q


def load(case):
    d = np.load(FIX)
    Uc = d["id_Uc"] if case == "id" else d["Uc"]
    return d[f"{case}_Y"], Uc, d[f"{case}_cls"], d[f"{case}_Sb"], d[f"{case}_Q"], d[f"{case}_IDX"], d["A"], d["c"]


@pytest.mark.parametrize("case", ["mix", "c3", "id"])
def test_reference_fixtures_decode_to_their_values(case):
    Y, Uc, cls, Sb, Q, IDX, A, c = load(case)
    assert np.array_equal(decode_idx(IDX, cls, Sb, A, c), Q)
    assert sorted(set(cls.ravel().tolist())) == ([3] if case == "c3" else list(range(8)))


def test_shipped_codebook_is_the_fixtures():
    from pingala8_llm_b200.synth import HEADER

    d = np.load(FIX)
    assert np.array_equal(HEADER[:1024].view(np.int8).reshape(256, 4), d["A"])
    assert np.array_equal(HEADER[2048:2052].view(np.int8), d["c"])


@pytest.mark.gpu
@pytest.mark.parametrize("case", ["mix", "c3", "id"])
def test_gpu_encoder_against_reference_encoder(case):
    torch = pytest.importorskip("torch")
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA GPU")
    from pingala8_llm_b200.encoder import encode
    from pingala8_llm_b200.ops import device_error

    Y, Uc, cls, Sb, Qr, IDXr, A, c = load(case)
    Q, IDX = encode(torch.from_numpy(Y).cuda(), torch.from_numpy(Uc).cuda(), torch.from_numpy(cls.astype(np.int64)),
                    torch.from_numpy(Sb))
    torch.cuda.synchronize()
    assert device_error() == 0
    Q, IDX = Q.cpu().numpy(), IDX.cpu().numpy()
    assert np.array_equal(decode_idx(IDX, cls, Sb, A, c).view(np.uint32), Q.view(np.uint32))
    live = np.repeat(cls > 0, 64, axis=1)  # (row, step) positions of quantised blocks
    same = np.all(IDX == IDXr, axis=2)[live].mean()
    assert np.all(IDX[~live] == 0) and np.all(Q[np.repeat(cls == 0, 256, axis=1)] == 0)
    err, err_ref = float(np.sum((Y - Q) ** 2)), float(np.sum((Y - Qr) ** 2))
    assert np.array_equal(IDX, IDXr), (same, err / err_ref)
    assert np.array_equal(Q, Qr)
    # deterministic
    Q2, IDX2 = encode(torch.from_numpy(Y).cuda(), torch.from_numpy(Uc).cuda(), torch.from_numpy(cls.astype(np.int64)),
                      torch.from_numpy(Sb))
    assert torch.equal(Q2.cpu(), torch.from_numpy(Q)) and torch.equal(IDX2.cpu(), torch.from_numpy(IDX))
    print(f"{case}: codes equal at {same:.4f} of steps, error ratio {err / err_ref:.5f}")


@pytest.mark.gpu
def test_gpu_encoder_model_size_tensor_runs_and_decodes():
    """a 4096 x 4096 class-3 tensor with a random Hessian: every row decodes to its Q; the time is printed"""
    torch = pytest.importorskip("torch")
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA GPU")
    import time

    from pingala8_llm_b200.encoder import encode
    from pingala8_llm_b200.ops import device_error

    n, rows = 4096, 4096
    g = torch.Generator(device="cuda").manual_seed(0)
    X = torch.randn(2 * n, n, device="cuda", generator=g, dtype=torch.float64)
    H = X.T @ X / (2 * n)
    H += 0.1 * H.diagonal().mean() * torch.eye(n, device="cuda", dtype=torch.float64)
    Uc = torch.linalg.cholesky(torch.cholesky_inverse(torch.linalg.cholesky(H)), upper=True).float()
    Y = torch.randn(rows, n, device="cuda", generator=g)
    cls = torch.full((rows, n // 256), 3, dtype=torch.int64)
    Sb = torch.full((rows, n // 256), 1 / 16.0)
    encode(Y[:64], Uc, cls[:64], Sb[:64])  # warm-up
    torch.cuda.synchronize()
    t0 = time.time()
    Q, IDX = encode(Y, Uc, cls, Sb)
    torch.cuda.synchronize()
    dt = time.time() - t0
    assert device_error() == 0
    d = np.load(FIX)
    sel = np.arange(0, rows, 257)
    Qd = decode_idx(IDX[sel].cpu().numpy(), cls[sel].numpy(), Sb[sel].numpy(), d["A"], d["c"])
    assert np.array_equal(Qd.view(np.uint32), Q[sel].cpu().numpy().view(np.uint32))
    print(f"4096 x 4096 class 3: {dt * 1e3:.1f} ms ({dt / (rows * n) * 1e9:.2f} ns per weight)")
