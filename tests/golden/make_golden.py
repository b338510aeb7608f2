"""Generate golden vectors by running the REFERENCE implementation on the CPU.

Usage (needs the reference checkout; writes tests/golden/*.npz):

    python tests/golden/make_golden.py /path/to/maple-flash-dgx-spark

The reference's Triton kernels are executed by Triton's interpreter
(``TRITON_INTERPRET=1``) on CPU tensors; their wrappers' ``is_cuda`` guard is
bypassed inside this process only.  fp32 activations are used because the
interpreter's bf16 dot paths are unreliable; where the reference rounds to
bf16 on the GPU the tests apply RNE themselves.  Inputs are regenerated in the
tests from the recorded seeds with numpy's frozen ``RandomState`` stream, so
the fixtures hold outputs only.
"""

from __future__ import annotations

import os
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent.parent))

from tests.golden.cases import CASES  # noqa: E402


def _setup_reference(root: str):
    os.environ["TRITON_INTERPRET"] = "1"
    sys.path.insert(0, str(Path(root) / "src"))
    import torch

    torch.Tensor.is_cuda = property(lambda self: True)  # interpreter only
    return torch


def main(root: str) -> None:
    torch = _setup_reference(root)
    out: dict[str, np.ndarray] = {}
    for name, case in CASES.items():
        res = case.run_reference(torch)
        for key, val in res.items():
            out[f"{name}/{key}"] = np.asarray(val)
        print(name, {k: np.asarray(v).shape for k, v in res.items()}, flush=True)
    np.savez_compressed(HERE / "reference_golden.npz", **out)
    print("wrote", HERE / "reference_golden.npz")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: python tests/golden/make_golden.py /path/to/maple-flash-dgx-spark")
    main(sys.argv[1])
