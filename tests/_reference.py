"""The unmodified reference server, as installed in ``baseline/_ref``, with the
dispatcher patch a maintainer applies — for the tests that
run the reference's own scheduler, executor and test-suite against ``ATTENTION=cuda``.

``baseline/_ref`` is written by ``baseline/install_reference.py`` (and by
``__graft_entry__.build()`` when a reference checkout is present).  Tests that need it skip
with that instruction when it is missing.  The patched copy is built in a temporary
directory; nothing under ``baseline/_ref`` is edited.
"""

from __future__ import annotations

import ast
import re
import shutil
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
REF = ROOT / "baseline" / "_ref"
REF_TESTS = REF / "reference_tests"
INTEGRATION = ROOT / "INTEGRATION.md"
MISSING = "reference not installed in baseline/_ref (run: python baseline/install_reference.py)"


def available() -> bool:
    return (REF / "inference_server" / "core" / "attention.py").exists()


def require() -> None:
    if not available():
        pytest.skip(MISSING)


def dispatcher_patch() -> str:
    """The ``paged_attention`` function of INTEGRATION.md section 1, verbatim."""
    text = INTEGRATION.read_text()
    sec = text.split("## 1.", 1)[1].split("\n## ", 1)[0]
    m = re.search(r"```python\n(.*?)```", sec, re.S)
    assert m, "INTEGRATION.md section 1 has no python block"
    return m.group(1)


def apply_dispatcher_patch(attention_py: Path) -> None:
    """Replace the reference's ``paged_attention`` function (found with ``ast``) by the
    INTEGRATION.md version; the rest of the file is untouched."""
    src = attention_py.read_text()
    tree = ast.parse(src)
    fn = next(n for n in tree.body if isinstance(n, ast.FunctionDef) and n.name == "paged_attention")
    lines = src.splitlines(keepends=True)
    new = lines[:fn.lineno - 1] + [dispatcher_patch()] + lines[fn.end_lineno:]
    attention_py.write_text("".join(new))


def make_patched_copy(dest: Path) -> Path:
    """Copy ``baseline/_ref/inference_server`` (and the reference tests) under ``dest``
    and apply the dispatcher patch.  Returns ``dest`` (the directory to put on
    ``sys.path``)."""
    require()
    dest.mkdir(parents=True, exist_ok=True)
    shutil.copytree(REF / "inference_server", dest / "inference_server",
                    ignore=shutil.ignore_patterns("__pycache__"))
    if REF_TESTS.exists():
        shutil.copytree(REF_TESTS, dest / "reference_tests", ignore=shutil.ignore_patterns("__pycache__"))
    apply_dispatcher_patch(dest / "inference_server" / "core" / "attention.py")
    return dest


def import_patched(dest: Path):
    """Import the patched reference package in this process (first on ``sys.path``).
    Returns the ``inference_server`` module."""
    for name in [m for m in sys.modules if m == "inference_server" or m.startswith("inference_server.")]:
        del sys.modules[name]
    sys.path.insert(0, str(dest))
    import inference_server  # noqa: F401
    import inference_server.core.attention as attention

    assert Path(attention.__file__).resolve().is_relative_to(dest.resolve()), attention.__file__
    return sys.modules["inference_server"]
