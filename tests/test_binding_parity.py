"""Binding parity: every attribute the Python layer reads from the native
extensions exists in the built modules (the role of the reference's FFI ABI
parity test, flodl-sys/src/ffi_parity.rs: a renamed or removed binding fails
here on the CPU instead of at first use on a GPU)."""
import ast
import os

import pytest

PKG = os.path.join(os.path.dirname(os.path.dirname(__file__)), "flodl_b200")
LOADERS = {"cuda_ext", "native", "ext", "_native", "C"}  # C() in ops returns the kernel module


def _uses(path):
    tree = ast.parse(open(path).read(), path)
    aliases = set()
    for node in ast.walk(tree):
        if isinstance(node, ast.Assign) and isinstance(node.value, ast.Call):
            f = node.value.func
            if isinstance(f, ast.Name) and f.id in LOADERS:
                aliases |= {t.id for t in node.targets if isinstance(t, ast.Name)}
    used = set()
    for node in ast.walk(tree):
        if isinstance(node, ast.Attribute):
            v = node.value
            if isinstance(v, ast.Call) and isinstance(v.func, ast.Name) and v.func.id in LOADERS:
                used.add(node.attr)
            elif isinstance(v, ast.Name) and v.id in aliases:
                used.add(node.attr)
    return used


def test_every_binding_used_from_python_exists():
    from flodl_b200 import _ext
    if _ext._C is None or _ext._native is None:
        pytest.skip(f"extensions not built: {_ext._C_ERR!r} {_ext._NATIVE_ERR!r}")
    have = set(dir(_ext._C)) | set(dir(_ext._native))
    missing = {}
    n_used = 0
    for root, _, files in os.walk(PKG):
        for f in files:
            if f.endswith(".py"):
                p = os.path.join(root, f)
                u = _uses(p)
                n_used += len(u)
                bad = sorted(a for a in u if a not in have)
                if bad:
                    missing[os.path.relpath(p, PKG)] = bad
    assert n_used > 40, "the scan found too few binding uses to be meaningful"
    assert not missing, f"bindings used but not exported: {missing}"
