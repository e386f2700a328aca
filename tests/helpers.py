"""Test helpers shared by the test modules (import as tests.helpers)."""
import importlib.util
import sys
from pathlib import Path

REPO = Path(__file__).resolve().parent.parent


def golden_module():
    """tests/golden/make_golden.py as a module (for its seeded input builders)."""
    path = REPO / "tests" / "golden" / "make_golden.py"
    spec = importlib.util.spec_from_file_location("make_golden", path)
    mod = importlib.util.module_from_spec(spec)
    sys.modules.setdefault("make_golden", mod)
    spec.loader.exec_module(mod)
    return mod
