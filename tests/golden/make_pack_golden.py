"""Golden vectors of the reference's CPU packing code (pack.py) for the GPU
packing kernels.

Usage (needs the reference checkout; writes tests/golden/reference_pack.npz):

    python tests/golden/make_pack_golden.py /path/to/maple-flash-dgx-spark

Inputs are regenerated from the seeds below with numpy's frozen RandomState
stream; the fixture holds the reference's outputs (and the inputs, which are
small).
"""

from __future__ import annotations

import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent

TERNARIZE = [(31, 6, 1408), (32, 3, 2048), (33, 2, 128), (34, 4, 384)]
RTN = [(41, 5, 256, 64), (42, 3, 2048, 128)]


def ternarize_input(seed, n, k):
    rs = np.random.RandomState(seed)
    w = (rs.standard_normal((n, k)) * 0.02).astype(np.float32)
    w[0, :16] = 0.0  # exact zeros stay code 1
    if n > 2:
        w[2] = 0.0  # all-zero row: alpha 0, every code 1
    return w


def rtn_input(seed, n, k):
    rs = np.random.RandomState(seed)
    w = (rs.standard_normal((n, k)) * 0.02).astype(np.float32)
    w[1, :64] = 0.5  # constant group: scale 0 -> code 0
    return w


def main(root: str) -> None:
    sys.path.insert(0, str(Path(root) / "src"))
    from maple_run.pack import pack_2bit, quantize_rtn, ternarize

    out = {}
    for seed, n, k in TERNARIZE:
        w = ternarize_input(seed, n, k)
        packed, alpha = ternarize(w)
        out[f"tern_{seed}_packed"] = packed
        out[f"tern_{seed}_alpha"] = alpha
    for seed, n, k, g in RTN:
        packed, scales, biases = quantize_rtn(rtn_input(seed, n, k), group_size=g)
        out[f"rtn_{seed}_packed"] = packed
        out[f"rtn_{seed}_scales"] = scales
        out[f"rtn_{seed}_biases"] = biases
    # codes above the 2-bit field carry into the next field (uint64 sum)
    codes = np.random.RandomState(51).randint(0, 6, size=(4, 64)).astype(np.uint32)
    out["pack_overflow_codes"] = codes
    out["pack_overflow_words"] = pack_2bit(codes)
    np.savez_compressed(HERE / "reference_pack.npz", **out)
    print(sorted(out))


if __name__ == "__main__":
    main(sys.argv[1])
