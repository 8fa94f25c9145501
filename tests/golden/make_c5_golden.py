"""SHA-256 of the oracle's outputs for the C5 workload (16384 x 8192 x 28672
W8A8, per-token activation scales, per-channel weight scales), written to
c5_hashes.json.  The full output (470 M values per kind) is too large to
commit; its hashes pin the CUDA library's result bit for bit, in the
tests and in bench.py's multi-GPU runs.

    python tests/golden/make_c5_golden.py

Inputs: tests/golden/configs.py ``c5_inputs`` (numpy seed 0).  Outputs hashed
in the C ABI's column-major ``[M, N]`` layout (storage ``[N][M]``, each
output channel's M values contiguous):

* ``bp32``: bposit32 (truncating) of every exact INT32 dot product;
* ``y_f32``: ``(float)acc / (x_scale[m] * w_scale[n])`` in fp32.

Besides the full M = 16384, the same hashes over the first 256 and 2048 rows
(the reduced cases the tests run) are recorded.  About a minute on 8 cores.
"""
from __future__ import annotations

import hashlib
import json
import sys
import time
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent.parent))
sys.path.insert(0, str(HERE))
from oracle import bposit_oracle as O  # noqa: E402

import configs  # noqa: E402

ROW_CASES = (256, 2048, configs.C5[0])
BLOCK_N = 1024


def c5_outputs_hashes(rows=ROW_CASES, threads: int = 8, log=print) -> dict:
    """{rows: {"bp32": sha256, "y_f32": sha256}} for every row count in
    ``rows`` (each a prefix of the full activation)."""
    M = max(rows)
    _, K, N = configs.C5
    t0 = time.time()
    x, w = configs.c5_inputs(M)
    log(f"inputs {time.time() - t0:.1f} s")
    wq, ws = O.quant_per_channel(w.T)             # [K, N], [N]
    del w
    xq, xs = O.quant_per_token(x)                 # [M, K], [M]
    del x
    log(f"quantised {time.time() - t0:.1f} s")
    xf = xq.astype(np.float64)
    hashers = {r: {"bp32": hashlib.sha256(), "y_f32": hashlib.sha256()} for r in rows}
    with ThreadPoolExecutor(threads) as ex:
        for n0 in range(0, N, BLOCK_N):
            n1 = min(N, n0 + BLOCK_N)
            acc = (xf @ wq[:, n0:n1].astype(np.float64)).astype(np.int64)    # [M, nb], exact
            at = np.ascontiguousarray(acc.T)                                   # [nb, M]
            chunks = np.array_split(at.reshape(-1), 64)
            bp = np.concatenate(list(ex.map(lambda c: O.encode_int_array(c, 0, 32), chunks)))
            bp = bp.reshape(at.shape)
            y = O.dequant(acc, xs, ws[n0:n1]).T                               # [nb, M]
            for r in rows:
                hashers[r]["bp32"].update(np.ascontiguousarray(bp[:, :r]).tobytes())
                hashers[r]["y_f32"].update(np.ascontiguousarray(y[:, :r]).tobytes())
            if n0 % (8 * BLOCK_N) == 0:
                log(f"columns {n1}/{N} {time.time() - t0:.1f} s")
    return {r: {k: h.hexdigest() for k, h in hs.items()} for r, hs in hashers.items()}


def main() -> None:
    hashes = c5_outputs_hashes()
    out = {
        "workload": "C5 W8A8 16384x8192x28672, per-token x scales, per-channel w scales",
        "inputs": "tests/golden/configs.py c5_inputs (numpy default_rng(0): w [28672, 8192] "
                  "~N(0, 0.02) drawn first, then x [M, 8192] ~N(0, 1))",
        "layout": "column-major [M, N]: storage [N][M]",
        "bp32": "bposit32 truncating encode of the exact INT32 dot product",
        "y_f32": "(float)acc / (x_scale[m] * w_scale[n]) in fp32",
        "K": configs.C5[1], "N": configs.C5[2],
        "rows": {str(r): h for r, h in sorted(hashes.items())},
    }
    (HERE / "c5_hashes.json").write_text(json.dumps(out, indent=1) + "\n")
    print("wrote c5_hashes.json")


if __name__ == "__main__":
    main()
