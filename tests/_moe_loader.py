"""Imports the product package (its directory name is not a Python identifier)."""
import importlib.util
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG_DIR = os.path.join(ROOT, "implementing-moe-architecture-operators-on-cann-platform_b200")


def load():
    if "moe_b200" in sys.modules:
        return sys.modules["moe_b200"]
    spec = importlib.util.spec_from_file_location(
        "moe_b200", os.path.join(PKG_DIR, "__init__.py"), submodule_search_locations=[PKG_DIR])
    m = importlib.util.module_from_spec(spec)
    sys.modules["moe_b200"] = m
    spec.loader.exec_module(m)
    return m
