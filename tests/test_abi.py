"""The C-ABI library loads on a machine without a GPU, exports every entry point declared in
include/*.h, and its public structs have the reference's layout (sizes checked against the
reference's own sizeof, oracle/_ref)."""
import ctypes
import os
import re

import pytest

from g2util import ROOT


def _declared_functions():
    names = set()
    pat = re.compile(r"^\s*(?:const\s+)?[A-Za-z_][\w\s\*]*?\b(ggemm_\w+)\s*\(", re.M)
    for fn in sorted(os.listdir(os.path.join(ROOT, "include"))):
        if not fn.endswith(".h"):
            continue
        text = open(os.path.join(ROOT, "include", fn)).read()
        text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
        for line in text.splitlines():
            if "static inline" in line or line.strip().startswith("#"):
                continue
            m = pat.match(line)
            if m:
                names.add(m.group(1))
    return names


def test_library_exports_every_declared_symbol(g2):
    names = _declared_functions()
    assert "ggemm_grouped_dgemm" in names and "ggemm_execute_plan" in names
    missing = [n for n in sorted(names) if not hasattr(g2.lib, n)]
    assert not missing, f"declared but not exported: {missing}"


def test_struct_layouts(g2):
    assert ctypes.sizeof(g2.Problem) == 80
    assert ctypes.sizeof(g2.Config) == 24
    assert ctypes.sizeof(g2.Stats) == 64
    assert ctypes.sizeof(g2.PrepDesc) == 56
    assert ctypes.sizeof(g2.GemmDesc) == 72
    assert ctypes.sizeof(g2.ReconDesc) == 120


def test_struct_sizes_match_reference(g2, ref):
    assert ref.L.ozr_sizeof_problem() == ctypes.sizeof(g2.Problem)


def test_enum_values(g2):
    assert [g2.PATH_NATIVE_LOOP, g2.PATH_NATIVE_GROUPED, g2.PATH_EMU_LOOP, g2.PATH_EMU_GROUPED,
            g2.PATH_AUTO, g2.PATH_EMU_GROUPED_REUSE, g2.PATH_EMU_LOOP_BATCHED] == list(range(7))
    assert (g2.REPAIR_DEFAULT, g2.REPAIR_OFF, g2.REPAIR_COUNT, g2.REPAIR_ON) == (0, 1, 2, 3)
    assert g2.MAX_MODULI == 20


def test_no_gpu_calls_fail_cleanly(g2):
    """Without a device: create fails with an error code instead of crashing."""
    if g2.lib.ggemm_device_count() > 0:
        pytest.skip("a GPU is present")
    h = ctypes.c_void_p()
    rc = g2.lib.ggemm_create(ctypes.byref(h), 4, 100, 100, 100, None)
    assert rc != 0


def test_version(g2):
    assert "sm_100a" in g2.version()
