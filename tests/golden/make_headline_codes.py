"""The 65,536 bposit16 codes of the determinism headline
(kernels/test_determinism_headline.cu:181-189: LCG log-uniform values on
[1e-3, 1e3], encoded by the headline's own float64 truncating encoder,
det:110-148), written to headline_codes.npy (uint16, 128 KiB).

bench.py loads the codes to run the headline on every GPU of a job; the
oracle's generator (oracle.bposit_oracle.det_headline_inputs) is pinned to
the same bits by tests/test_oracle_pins.py.

    python tests/golden/make_headline_codes.py
"""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent.parent))
from oracle import bposit_oracle as O  # noqa: E402


def main():
    _, _, codes = O.det_headline_inputs()
    np.save(HERE / "headline_codes.npy", codes.astype(np.uint16))
    print(f"wrote {codes.size} codes")


if __name__ == "__main__":
    main()
