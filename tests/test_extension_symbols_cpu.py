"""Every name the Python layer looks up on the compiled extension exists in the built module.

A binding added in csrc/bindings.cpp but left out of a commit makes a clean build lack a
function the Python code calls; training then fails at its first use. This runs on the CPU
(loading the module needs no GPU) and is skipped when the extension has not been built."""
import pathlib
import re

import pytest
import torch  # noqa: F401  (loads the libraries the extension links against)

ROOT = pathlib.Path(__file__).resolve().parents[1]


def test_every_referenced_binding_exists():
    try:
        from llmt import _C
    except ImportError:
        pytest.skip("llmt._C is not built")
    names = set()
    for p in (ROOT / "llmt").rglob("*.py"):
        src = p.read_text()
        names |= set(re.findall(r"ext\(\)\.(\w+)", src))
        names |= set(re.findall(r"\bC\.(\w+)\(", src))
    names.discard("_mod")  # attribute of the launch-counting wrapper, not a binding
    missing = sorted(n for n in names if not hasattr(_C, n))
    assert not missing, missing
