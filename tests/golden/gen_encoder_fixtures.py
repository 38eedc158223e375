"""Generate tests/golden/encoder_fixtures.npz with the REFERENCE's own trellis encoder (research/detail/r48k.py encode,
r48k.py:105, with vit_k r48k.py:57 and zero_ldlq r48k.py:97), run on CPU in the build container.

Run here only (it imports the reference checkout):  python tests/golden/gen_encoder_fixtures.py  REFERENCE_CHECKOUT
Settings are the production ones the golden slots use: R48K_NS=8 (Pingala-8 gana states) and
R48K_SHIFTS=0,0,0,0,2,3,2,4/0,0,0,0,0,0,0,2, tables research/work/r48k3/tables_vrc.pt (the codebook shipped in
pingala8_llm_b200/tables_pingala8.bin), trellis mode (tr = True).

Inputs are synthetic: Y ~ N(0, 1) (the FWHT-domain weights of one tensor), per-(row, 256-block) classes, scales
S = 1/20 .. 1/12 (int units of a few tens), and Uc = upper Cholesky factor of the inverse of a random SPD Hessian
(X^T X / m + 0.1 mean(diag) I), so the LDLQ error feedback is exercised; one case uses H = I (no feedback).
"""
import os
import sys
import time

import numpy as np


def main(ref_root):
    os.environ["R48K_NS"] = "8"
    os.environ["R48K_SHIFTS"] = "0,0,0,0,2,3,2,4/0,0,0,0,0,0,0,2"
    sys.path.insert(0, os.path.join(ref_root, "research", "detail"))
    import torch
    import r48k as K

    torch.set_num_threads(os.cpu_count() or 1)
    T = torch.load(os.path.join(ref_root, "research", "work", "r48k3", "tables_vrc.pt"))
    T = {k: v.float() for k, v in T.items()}
    n = 512
    rng = np.random.default_rng(2024)
    X = rng.normal(0, 1, (2 * n, n))
    H = X.T @ X / (2 * n)
    H += 0.1 * np.mean(np.diag(H)) * np.eye(n)
    Uc = np.linalg.cholesky(np.linalg.inv(H)).T.astype(np.float32)  # upper: Hi = Uc^T Uc
    out = {"Uc": Uc, "A": T["A"].numpy().astype(np.int8), "c": T["c"].numpy().astype(np.int8)}
    cases = [("mix", 64, None, Uc), ("c3", 96, 3, Uc), ("id", 64, None, (np.eye(n) / np.sqrt(1.1)).astype(np.float32))]
    for name, rows, cls_fixed, U in cases:
        r = np.random.default_rng(rows + len(name))
        Y = r.normal(0, 1, (rows, n)).astype(np.float32)
        cls = (np.full((rows, n // 256), cls_fixed) if cls_fixed is not None else r.integers(0, 8, (rows, n // 256))).astype(np.int64)
        Sb = r.uniform(1 / 20, 1 / 12, (rows, n // 256)).astype(np.float32)
        Sb[cls == 0] = 0
        t0 = time.time()
        Q, IDX = K.encode(torch.from_numpy(Y), torch.from_numpy(U), torch.from_numpy(cls), torch.from_numpy(Sb), T, True)
        print(name, rows, "x", n, "encoded in", round(time.time() - t0, 1), "s", flush=True)
        out.update({f"{name}_Y": Y, f"{name}_cls": cls.astype(np.uint8), f"{name}_Sb": Sb, f"{name}_Q": Q.numpy().astype(np.float32),
                    f"{name}_IDX": IDX.numpy().astype(np.uint8)})
        if name == "id":
            out["id_Uc"] = U
    np.savez_compressed(os.path.join(os.path.dirname(os.path.abspath(__file__)), "encoder_fixtures.npz"), **out)


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else "/root/reference")
