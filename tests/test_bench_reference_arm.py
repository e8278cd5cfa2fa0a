"""The benchmark's reference arm never loads the reference's compiled attention extension (its sm_100 build faulted
on B200): with a stand-in package whose extension module records any import, the blocking step leaves the ops on
their PyTorch fallbacks and the extension module is never executed."""
import importlib
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]


@pytest.fixture
def fake_reference(tmp_path, monkeypatch):
    pkg = tmp_path / "flashattention_custom"
    pkg.mkdir()
    (pkg / "__init__.py").write_text("")
    (pkg / "_ext.py").write_text("import builtins\nbuiltins._HRM_EXT_IMPORTED = True\n")
    (pkg / "ops.py").write_text(
        "try:\n    from . import _ext as _ext\n    _HAS_EXT = True\nexcept (ImportError, OSError):\n"
        "    _ext = None\n    _HAS_EXT = False\n")
    monkeypatch.syspath_prepend(str(tmp_path))
    for k in [k for k in sys.modules if k.startswith("flashattention_custom")]:
        monkeypatch.delitem(sys.modules, k)
    yield
    for k in [k for k in sys.modules if k.startswith("flashattention_custom")]:
        sys.modules.pop(k, None)


def test_extension_present_but_never_imported(fake_reference, monkeypatch):
    import builtins
    monkeypatch.syspath_prepend(str(ROOT))
    bench = importlib.import_module("bench")
    monkeypatch.setattr(builtins, "_HRM_EXT_IMPORTED", False, raising=False)
    bench._block_reference_extension()
    ops = importlib.import_module("flashattention_custom.ops")
    assert ops._HAS_EXT is False and ops._ext is None
    assert builtins._HRM_EXT_IMPORTED is False


def test_without_blocking_the_stand_in_would_load(fake_reference):
    """Control: the stand-in package does import its extension when nothing blocks it."""
    ops = importlib.import_module("flashattention_custom.ops")
    assert ops._HAS_EXT is True
