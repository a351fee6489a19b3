"""Install the unmodified reference server into ``baseline/_ref`` (git-ignored; it travels
with the working tree to GPU boxes, where no reference checkout exists).

    python baseline/install_reference.py [--src DIR] [--force]

The reference checkout has no packaging metadata, so the package is copied to a
temporary directory, a minimal ``pyproject.toml`` naming the ``inference_server`` package
is written beside it, and pip installs it offline (``--no-index --no-build-isolation
--no-deps --target baseline/_ref``).  No reference source file is edited.  The reference's
own tests that pin the attention path (``tests/test_paged_attention.py``,
``tests/test_paged_attention_triton.py`` and their ``conftest.py``) are copied unchanged
to ``baseline/_ref/reference_tests/`` so GPU runs can execute them against the CUDA path.

Consumers: ``bench.py --impl reference`` (the reference's gather attention timed on host
cores) and the ``-m gpu`` tests that drive the reference's scheduler with the CUDA
executor.  Both fall back or skip with a stated reason when ``baseline/_ref`` is absent.
"""

from __future__ import annotations

import argparse
import shutil
import subprocess
import sys
import tempfile
from pathlib import Path

HERE = Path(__file__).resolve().parent
TARGET = HERE / "_ref"
DEFAULT_SRC = Path("/root/reference")
TESTS = ("conftest.py", "test_paged_attention.py", "test_paged_attention_triton.py")

PYPROJECT = """\
[build-system]
requires = ["setuptools"]
build-backend = "setuptools.build_meta"

[project]
name = "inference-server-reference"
version = "0.0.0"

[tool.setuptools.packages.find]
include = ["inference_server*"]
"""


def installed() -> bool:
    return (TARGET / "inference_server" / "core" / "attention.py").exists() and all(
        (TARGET / "reference_tests" / t).exists() for t in TESTS)


def install(src: Path = DEFAULT_SRC, force: bool = False, quiet: bool = True) -> bool:
    """Returns True when ``baseline/_ref`` holds the reference after the call."""
    if installed() and not force:
        return True
    if not (src / "inference_server").is_dir():
        return False
    if TARGET.exists():
        shutil.rmtree(TARGET)
    with tempfile.TemporaryDirectory(prefix="ref_install_") as tmp:
        stage = Path(tmp) / "src"
        stage.mkdir()
        shutil.copytree(src / "inference_server", stage / "inference_server",
                        ignore=shutil.ignore_patterns("__pycache__", "*.pyc"))
        (stage / "pyproject.toml").write_text(PYPROJECT)
        cmd = [sys.executable, "-m", "pip", "install", "--no-index", "--no-build-isolation", "--no-deps",
               "--target", str(TARGET), str(stage)]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"reference install failed:\n{r.stdout}\n{r.stderr}")
        if not quiet:
            print(r.stdout)
    tests = TARGET / "reference_tests"
    tests.mkdir(exist_ok=True)
    for t in TESTS:
        shutil.copy2(src / "tests" / t, tests / t)
    return installed()


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--src", type=Path, default=DEFAULT_SRC)
    ap.add_argument("--force", action="store_true")
    a = ap.parse_args()
    ok = install(a.src, a.force, quiet=False)
    print(f"baseline/_ref: {'installed' if ok else 'unavailable (no reference checkout at ' + str(a.src) + ')'}")
    sys.exit(0 if ok else 1)
