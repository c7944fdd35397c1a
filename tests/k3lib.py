"""Load the product package (its directory name is not a Python identifier)."""
import importlib.util
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG_DIR = os.path.join(ROOT, "kimi-k3-for-me_b200")


def load():
    if "k3b200" in sys.modules:
        return sys.modules["k3b200"]
    spec = importlib.util.spec_from_file_location("k3b200", os.path.join(PKG_DIR, "__init__.py"))
    mod = importlib.util.module_from_spec(spec)
    sys.modules["k3b200"] = mod
    spec.loader.exec_module(mod)
    return mod
