"""Regenerate the golden fixtures in this directory from the reference's own test data.

Reads the gsplat forward renders that the reference commits for its
``test_reference`` test (crates/brush-bench-test/test_cases/{tiny,basic}_case.safetensors,
produced by its generate_reference.py with gsplat) and stores the same
tensors as ``.npz``. Run where the reference tree is available:

    python tests/golden/make_golden.py /path/to/reference
"""
import sys
from pathlib import Path

import numpy as np
from safetensors.numpy import load_file

HERE = Path(__file__).resolve().parent


def main(ref_root: str) -> None:
    cases = Path(ref_root) / "crates" / "brush-bench-test" / "test_cases"
    for name in ("tiny_case", "basic_case"):
        d = load_file(str(cases / f"{name}.safetensors"))
        np.savez_compressed(HERE / f"{name}.npz", **{k: np.asarray(v) for k, v in d.items()})
        print(name, {k: v.shape for k, v in d.items()})


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: python tests/golden/make_golden.py /path/to/reference")
    main(sys.argv[1])
