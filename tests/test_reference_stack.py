"""The drop-in claim, tested through relmo's own unchanged Python stack.

A temporary copy of the reference checkout's ``src/relmo`` package (read from
the checkout at test time; nothing of it is kept in this repository) receives
this repository's two libraries, ``relm_mp_ops.so`` and ``librelm_mp_b200.so``,
exactly where relmo's loader looks for them (``relmo/ops/mp_runtime.py:97-159``
globs ``relm_mp_ops*.so`` in the package directory). Then relmo's own op tests
(``tests/python/test_mp_ops.py``, ``test_mp_module_layout.py``,
``test_mp_runtime.py`` - the ones that need no torch_geometric) run against it
in a fresh process, with ``RELM_MP_FALLBACK=error`` so that a call relmo could
not send to the library raises instead of silently running relmo's Python
formulas. Runs on CPU (CPU tensors go to the library's CPU kernels); skipped
where the reference checkout is absent.
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
REFERENCE = Path(os.environ.get("RELMO_REFERENCE_ROOT", str(ROOT.parent / "reference")))
REF_TESTS = ("test_mp_ops.py", "test_mp_module_layout.py", "test_mp_runtime.py")
LIBS = ("relm_mp_ops.so", "librelm_mp_b200.so")

pytestmark = pytest.mark.skipif(
    not (REFERENCE / "src" / "relmo" / "ops" / "mp.py").is_file(), reason="reference checkout not present"
)


@pytest.fixture(scope="module")
def installed(tmp_path_factory) -> Path:
    """A copy of relmo with the B200 libraries dropped into its package directory."""

    base = tmp_path_factory.mktemp("relmo_dropin")
    shutil.copytree(REFERENCE / "src" / "relmo", base / "src" / "relmo",
                    ignore=shutil.ignore_patterns("*.so", "__pycache__"))
    for lib in LIBS:
        shutil.copy2(ROOT / "relmo_b200" / lib, base / "src" / "relmo" / lib)
    (base / "tests").mkdir()
    for name in REF_TESTS:
        shutil.copy2(REFERENCE / "tests" / "python" / name, base / "tests" / name)
    return base


def _run(installed: Path, args: list[str]) -> subprocess.CompletedProcess:
    env = dict(os.environ)
    env["PYTHONPATH"] = str(installed / "src")
    env["RELM_MP_FALLBACK"] = "error"
    env.pop("RELM_MP_ENABLE", None)
    return subprocess.run([sys.executable, *args], cwd=installed, env=env, capture_output=True, text=True,
                          timeout=600)


def test_relmo_loads_the_b200_library(installed: Path) -> None:
    probe = (
        "import torch\n"
        "from relmo.ops import mp, mp_runtime\n"
        "assert mp.available()\n"
        "print(mp_runtime.candidate_libraries()[0].name)\n"
        "print(torch.ops.relm_mp.build_info())\n"
        "x = torch.randn(5, 3); i = torch.tensor([0, 4, 2])\n"
        "print(mp.fanin_reduce(x, i, torch.tensor([1, 0, 1]), 2, 0).shape)\n"
    )
    proc = _run(installed, ["-c", probe])
    assert proc.returncode == 0, proc.stderr
    lines = proc.stdout.splitlines()
    assert lines[0] == "relm_mp_ops.so"
    assert "lib=relm_mp_b200" in lines[1] and "arch=sm_100a" in lines[1]
    assert lines[2] == "torch.Size([2, 3])"


def test_relmo_own_op_tests_pass(installed: Path) -> None:
    proc = _run(installed, ["-m", "pytest", "tests", "-q", "-p", "no:cacheprovider", "-rs"])
    tail = proc.stdout[-3000:] + proc.stderr[-2000:]
    assert proc.returncode == 0, tail
    assert " passed" in proc.stdout and "skipped" not in proc.stdout, tail
