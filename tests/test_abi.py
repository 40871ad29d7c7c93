"""The C-ABI library: it loads and exports every function include/*.h declares
(no compute calls; this runs without a GPU)."""
import re
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]


def declared_functions():
    names = set()
    for h in sorted((ROOT / "include").glob("*.h")):
        text = re.sub(r"/\*.*?\*/", "", h.read_text(), flags=re.S)
        text = re.sub(r"static\s+inline[^{]*\{[^}]*\}", "", text)
        for m in re.finditer(r"\b((?:mpk|mpemu)[A-Za-z0-9_]*)\s*\(", text):
            names.add(m.group(1))
    return sorted(names)


def test_headers_declare_the_reference_entry_points():
    names = set(declared_functions())
    for must in ("mpkMeansMixed", "mpkMeansFP32", "mpkParamsInit", "mpkEpsilon", "mpkShiftNonNegative",
                 "mpkMakeBlobs", "mpkInitRandomPoints", "mpkAssign", "mpkUpdate", "mpkMeansMixedMG"):
        assert must in names, must


def test_library_exports_every_declared_symbol():
    import mpkmeans_b200 as M
    lib = M.lib()
    missing = [n for n in declared_functions() if not hasattr(lib, n)]
    assert not missing, missing


def test_python_mirror_covers_the_headers():
    import mpkmeans_b200 as M
    missing = [n for n in declared_functions() if n not in M.SIGNATURES and not n.startswith("mpemuSplitPlane")]
    assert not missing, missing


def test_struct_layouts_match_the_reference():
    import ctypes
    import mpkmeans_b200 as M
    assert ctypes.sizeof(M.mpkParams) == 48
    # iters(4)+pad(4)+inertia(8)+9*8+n_hist(4)+pad(4)+256*8+2*8+8+stats_built(4)+pad(4)+8*8
    assert ctypes.sizeof(M.mpkStats) == 8 + 8 + 72 + 8 + 2048 + 16 + 8 + 8 + 64


def test_param_defaults_host_only():
    import mpkmeans_b200 as M
    p = M.params_init()
    assert (p.max_iter, p.tol, p.use_cond3, p.use_cond6, p.cascade, p.accum, p.mw_macs) == (100, 0.0, 1, 1, 0, 0, 3)
    assert M.epsilon(128) == pytest.approx(2 / 2048 + 128 / 2 ** 24 / (1 - 128 / 2 ** 24), rel=1e-15)
