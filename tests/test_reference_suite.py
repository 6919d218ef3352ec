"""LMCache-Ascend's own transfer tests (tests/v1/test_mem_kernels.py), run
unmodified against the CPU oracle (tests/golden/reference_harness.py): the
reference's assertions must pass, and the digests of what the run drew and
produced must equal the committed fixture the GPU replay checks
(tests/golden/reference_digests.json), so the fixture is reproducible.

Needs the reference checkout ($LMCB_REFERENCE_ROOT, default /root/reference)
and skips without it. Two cases run here (about a minute); the fixture script
runs all twenty.
"""

import json
import os

import pytest

from tests.golden import reference_harness as h

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden",
                      "reference_digests.json")

pytestmark = pytest.mark.skipif(not h.available(), reason="reference checkout not present")


def _fixture(test, n, tm):
    with open(GOLDEN) as f:
        for c in json.load(f)["cases"]:
            if c["test"] == test and c["num_tokens"] == n and c.get("token_major") == tm:
                return c
    raise KeyError((test, n, tm))


@pytest.mark.parametrize("test,n,tm", [("test_extract_and_load_back", 256, None),
                                       ("test_single_layer_kernel", 500, False)])
def test_reference_test_passes_on_the_oracle_and_matches_the_fixture(test, n, tm):
    got = h.run_case(test, n, tm)  # raises if a reference assertion fails
    assert got == _fixture(test, n, tm)


def test_fixture_covers_every_reference_case():
    with open(GOLDEN) as f:
        cases = json.load(f)["cases"]
    want = {(t, n, tm) for t, n, tm in h.all_cases()}
    assert {(c["test"], c["num_tokens"], c.get("token_major")) for c in cases} == want
    for c in cases:
        if c["test"] in ("test_extract_and_load_back", "test_multi_layer_kernel",
                         "test_multi_layer_kernel_use_mla"):
            chunks = -(-c["num_tokens"] // 256)
            assert len(c["objects_sha256"]) == 2 * chunks
            # the reference's torch-made objects equal the op-made ones
            assert c["objects_sha256"][:chunks] == c["objects_sha256"][chunks:]
