"""Generates tests/golden/reference_digests.json: SHA-256 digests of what
LMCache-Ascend's own transfer tests (tests/v1/test_mem_kernels.py, all four
test functions at every parametrisation) draw and produce when they run,
unmodified, against the CPU oracle in this container
(tests/golden/reference_harness.py).

For each case the fixture records the seed, the digest of the paged caches
the test drew (torch.rand on the CPU generator, in creation order), the digest
of its slot mapping (random.sample), the digest of every LMCache object it
allocated, in order -- where the test fills its first objects with its own
torch expressions, those bytes come from the reference's code -- and the
digests of its caches and single-layer buffers after the test. The GPU parity
test (tests/test_reference_pinned_gpu.py) regenerates the same inputs, runs
the same calls through lmcache_b200.c_ops on the GPU and compares digests.

Run from the repository root (needs the reference checkout; about ten
minutes):  python tests/golden/make_reference_digests.py
"""

from __future__ import annotations

import json
import os
import sys
import time

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

import torch  # noqa: E402

from tests.golden import reference_harness as h  # noqa: E402

OUT = os.path.join(HERE, "reference_digests.json")


def main() -> None:
    if not h.available():
        raise SystemExit(f"reference tests not found under {h.REFERENCE_TESTS}")
    cases = []
    for test, n, tm in h.all_cases():
        t0 = time.perf_counter()
        cases.append(h.run_case(test, n, tm))
        print(f"{test} num_tokens={n} token_major={tm}: {time.perf_counter() - t0:.1f} s",
              flush=True)
    doc = {
        "source": "LMCache-Ascend tests/v1/test_mem_kernels.py and tests/v1/utils.py, run "
                  "unmodified against the CPU oracle by tests/golden/reference_harness.py",
        "torch": torch.__version__,
        "generators": "torch.manual_seed(seed) then the test's torch.rand calls on the CPU "
                      "generator; random.seed(seed) then random.sample for the slots",
        "cases": cases,
    }
    with open(OUT, "w") as f:
        json.dump(doc, f, indent=1)
    print("wrote", OUT)


if __name__ == "__main__":
    main()
