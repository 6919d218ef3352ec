"""The shipped package never reaches the oracle: no source under the package
or the C ABI headers names it, and importing the package loads no oracle
module. The oracle is test infrastructure only (tests, the smoke check and the
benchmark's CPU baseline)."""

import pathlib
import subprocess
import sys

ROOT = pathlib.Path(__file__).resolve().parents[1]
PRODUCT_DIRS = [ROOT / "lmcache-ascend_b200", ROOT / "include"]
SUFFIXES = {".py", ".cu", ".cuh", ".cpp", ".h", ".hpp", ".c"}


def test_product_sources_do_not_name_the_oracle():
    offenders = []
    for d in PRODUCT_DIRS:
        for path in d.rglob("*"):
            if path.suffix in SUFFIXES and path.is_file():
                if "oracle" in path.read_text(errors="replace"):
                    offenders.append(str(path.relative_to(ROOT)))
    assert offenders == []


def test_importing_the_package_loads_no_oracle_module():
    code = (
        "import sys; sys.path.insert(0, %r)\n"
        "try:\n"
        "    import lmcache_b200  # noqa: F401\n"
        "except ImportError:\n"
        "    pass  # the extension is not built here; nothing may fall back\n"
        "bad = [m for m in sys.modules if m == 'oracle' or m.startswith('oracle.')]\n"
        "print(','.join(bad))\n" % str(ROOT / "lmcache-ascend_b200")
    )
    out = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True,
                         cwd=str(ROOT / "lmcache-ascend_b200"), timeout=300)
    assert out.returncode == 0, out.stderr
    assert out.stdout.strip() == ""
