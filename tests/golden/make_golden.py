"""Generate the golden QR fixtures from the reference's own Python code.

Runs only where the reference tree is present (the build container); the
fixtures it writes (``golden_qr.npz`` beside this file) are committed and are
what the tests read everywhere else.

For every case it records, on CPU:

* ``A``        -- ``reference_repo/reference.py:23-87 generate_input`` (CPU generator),
* ``H_v1``/``tau_v1`` -- ``submissions/v1.py:66-79 _blocked_wy`` (the reference's
  pure-torch blocked WY, same Householder convention as its GPU kernels),
* ``H_geqrf``/``tau_geqrf`` -- ``reference.py:90-92 ref_kernel`` (``torch.geqrf``),
* ``chk_v1`` -- the scaled residuals printed by ``reference.py:127-192
  check_implementation`` for the v1 output
  (factor, reconstruction, triangular, orthogonality).

Usage: ``python tests/golden/make_golden.py /path/to/reference``
"""
from __future__ import annotations

import re
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent

# (name, batch, n, cond, seed, case)
CASES = [
    ("dense_b4_n1", 4, 1, 0, 101, "dense"),
    ("dense_b4_n2", 4, 2, 0, 102, "dense"),
    ("dense_b3_n3", 3, 3, 0, 103, "dense"),
    ("dense_b4_n5", 4, 5, 1, 105, "dense"),
    ("dense_b4_n8", 4, 8, 1, 108, "dense"),
    ("dense_b4_n16", 4, 16, 1, 116, "dense"),
    ("task_test0_b20_n32", 20, 32, 1, 53124, "dense"),   # task.yml:73
    ("dense_b4_n31", 4, 31, 1, 131, "dense"),
    ("dense_b4_n33", 4, 33, 1, 133, "dense"),
    ("dense_b3_n63", 3, 63, 1, 163, "dense"),
    ("dense_b4_n64", 4, 64, 0, 164, "dense"),
    ("dense_b2_n65", 2, 65, 1, 165, "dense"),
    ("dense_b2_n96", 2, 96, 2, 196, "dense"),
    ("dense_b1_n128", 1, 128, 2, 1128, "dense"),
    ("dense_cond4_b2_n64", 2, 64, 4, 264, "dense"),
]
for _n in (32, 64):
    for _i, _case in enumerate(("upper", "diagonal", "rankdef", "nearrank", "clustered",
                                "band", "nearcollinear", "rowscale")):
        CASES.append((f"{_case}_b2_n{_n}", 2, _n, 0, 7000 + 100 * _i + _n, _case))

_MSG_KEYS = ("scaled_factor_residual", "scaled_reconstruction_residual",
             "scaled_triangular_residual", "scaled_orthogonality_residual")


def main(ref_root: str) -> None:
    ref_root = Path(ref_root)
    sys.path.insert(0, str(ref_root / "reference_repo"))
    sys.path.insert(0, str(ref_root / "submissions"))
    import reference  # noqa: E402  (reference_repo/reference.py)
    import v1         # noqa: E402  (submissions/v1.py)

    torch.set_num_threads(4)
    out = {}
    names = []
    for name, batch, n, cond, seed, case in CASES:
        a = reference.generate_input(batch, n, cond, seed, case)
        assert a.device.type == "cpu"
        h1, t1 = v1._blocked_wy(a.clone())
        hg, tg = reference.ref_kernel(a.clone())
        ok, msg = reference.check_implementation(a, (h1, t1))
        assert ok, (name, msg)
        vals = [float(re.search(k + r"=([0-9.eE+-]+)", msg).group(1)) for k in _MSG_KEYS]
        out[f"{name}/A"] = a.numpy()
        out[f"{name}/H_v1"] = h1.numpy()
        out[f"{name}/tau_v1"] = t1.numpy()
        out[f"{name}/H_geqrf"] = hg.numpy()
        out[f"{name}/tau_geqrf"] = tg.numpy()
        out[f"{name}/chk_v1"] = np.array(vals, np.float64)
        out[f"{name}/spec"] = np.array([batch, n, cond, seed], np.int64)
        names.append(f"{name}:{case}")
    out["cases"] = np.array(names)
    np.savez_compressed(HERE / "golden_qr.npz", **out)
    print(f"wrote {len(names)} cases to {HERE / 'golden_qr.npz'}")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: make_golden.py REFERENCE_ROOT")
    main(sys.argv[1])
