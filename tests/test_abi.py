"""The C ABI: the library loads without a GPU and exports every declared entry point."""
import ctypes
import os
import re

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_functions():
    names = []
    for fn in sorted(os.listdir(os.path.join(ROOT, "include"))):
        if fn.endswith(".h"):
            src = open(os.path.join(ROOT, "include", fn)).read()
            src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
            names += re.findall(r"\b(dc_\w+)\s*\(", src)
    return sorted(set(names))


def test_every_declared_symbol_is_exported(P):
    lib = ctypes.CDLL(P._lib.LIB_PATH)
    names = declared_functions()
    assert len(names) >= 20
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, missing


def test_binding_covers_every_declared_symbol(P):
    bound = {n for n, _, _ in P._lib.SIGNATURES}
    assert set(declared_functions()) <= bound


def test_library_is_built_for_sm100a(P):
    """The build recipe targets sm_100a only, and ptxas compiled every kernel
    for it (its -v report, written beside the objects by the build)."""
    csrc = os.path.join(ROOT, "daisychain-infer_b200", "csrc")
    mk = open(os.path.join(csrc, "Makefile")).read()
    assert "-gencode arch=compute_100a,code=sm_100a" in mk
    assert not re.search(r"arch=compute_(?!100a)\d+", mk)
    logs = os.path.join(ROOT, "daisychain-infer_b200", "_build")
    reports = [os.path.join(logs, f) for f in os.listdir(logs) if f.endswith(".ptxas.log")] if os.path.isdir(logs) else []
    for r in reports:
        targets = set(re.findall(r"for '(sm_\w+)'", open(r).read()))
        assert targets <= {"sm_100a"}, (r, targets)
