"""Import helper: the package directory name is not a Python identifier, so put it on sys.path."""
import pathlib
import sys

PKG_DIR = pathlib.Path(__file__).resolve().parent.parent / "gemma4-e2b-laptop-cpu_b200"
if str(PKG_DIR) not in sys.path:
    sys.path.insert(0, str(PKG_DIR))

import g4  # noqa: E402,F401
