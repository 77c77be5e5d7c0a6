"""The C-ABI library loads without a GPU and exports every entry point that
include/gofish_b200.h declares (no compute call is made here)."""

import re
import subprocess
from pathlib import Path

from gofish_b200 import _native
from gofish_b200.build import LIBRARY, build

HEADER = Path(__file__).resolve().parents[1] / "include" / "gofish_b200.h"


def declared_functions():
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(gf_[a-z0-9_]+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    build()
    out = subprocess.run(["nm", "-D", "--defined-only", str(LIBRARY)], capture_output=True, text=True, check=True)
    exported = {line.split()[-1] for line in out.stdout.splitlines() if line.strip()}
    declared = declared_functions()
    assert declared, "no declarations parsed"
    missing = [name for name in declared if name not in exported]
    assert not missing, missing


def test_ctypes_binding_covers_the_header():
    assert sorted(_native.EXPORTED_SYMBOLS) == declared_functions()


def test_library_loads_and_reports_abi_version():
    lib = _native.load()
    assert lib.gf_abi_version() == _native.ABI_VERSION == 7


def test_create_rejects_bad_configuration():
    import ctypes

    lib = _native.load()
    cfg = _native.GfTracerConfig()
    cfg.k_buffer_size = 7
    assert not lib.gf_tracer_create(ctypes.byref(cfg))
    assert b"k_buffer_size" in lib.gf_last_error()
    cfg.k_buffer_size = 16
    cfg.sort_key = 5
    assert not lib.gf_tracer_create(ctypes.byref(cfg))
    cfg.sort_key = 0
    handle = lib.gf_tracer_create(ctypes.byref(cfg))
    assert handle
    lib.gf_tracer_destroy(handle)


def test_ctypes_structures_match_the_header_layout(tmp_path):
    """Size and field offsets of every ctypes mirror equal those of the C
    struct in include/gofish_b200.h (compiled here with gcc)."""
    import ctypes
    import subprocess
    from pathlib import Path

    mirrors = {"gf_camera": _native.GfCamera, "gf_tracer_config": _native.GfTracerConfig,
               "gf_trace_inputs": _native.GfTraceInputs, "gf_trace_outputs": _native.GfTraceOutputs,
               "gf_trace_grads": _native.GfTraceGrads, "gf_trace_stats": _native.GfTraceStats,
               "gf_field_camera": _native.GfFieldCamera, "gf_field_stats": _native.GfFieldStats,
               "gf_shape_camera": _native.GfShapeCamera}
    header = Path(__file__).resolve().parents[1] / "include" / "gofish_b200.h"
    lines = ['#include <stddef.h>', '#include <stdio.h>', f'#include "{header}"', "int main(void) {"]
    for cname, mirror in mirrors.items():
        lines.append(f'    printf("{cname} size %zu\\n", sizeof({cname}));')
        for field, *_ in mirror._fields_:
            lines.append(f'    printf("{cname} {field} %zu\\n", offsetof({cname}, {field}));')
    lines += ["    return 0;", "}"]
    src = tmp_path / "layout.c"
    src.write_text("\n".join(lines) + "\n")
    exe = tmp_path / "layout"
    subprocess.run(["gcc", "-std=c11", str(src), "-o", str(exe)], check=True)
    out = subprocess.run([str(exe)], check=True, capture_output=True, text=True).stdout.split("\n")
    got = {tuple(line.split()[:2]): int(line.split()[2]) for line in out if line}
    for cname, mirror in mirrors.items():
        assert got[(cname, "size")] == ctypes.sizeof(mirror), cname
        for field, *_ in mirror._fields_:
            assert got[(cname, field)] == getattr(mirror, field).offset, (cname, field)
