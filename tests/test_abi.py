"""The C ABI boundary without a GPU: libgs3d.so loads, exports every symbol include/gs3d.h
declares, and the ctypes mirrors have the C struct layouts. No compute calls."""
import ctypes as C
import re
import subprocess
import textwrap
from pathlib import Path

import pytest

from gs3d import _abi

REPO = Path(__file__).resolve().parent.parent
HEADER = REPO / "include" / "gs3d.h"


def declared_symbols():
    text = HEADER.read_text()
    return sorted(set(re.findall(r"GS3D_API\s+[\w\s\*]+?\b(\w+)\s*\(", text)))


def test_header_declares_the_reference_sort_symbols():
    syms = declared_symbols()
    assert "sort_pairs" in syms and "determine_sort_pairs_temp_storage" in syms
    assert "gs3d_render_forward" in syms and "gs3d_backward" in syms and "gs3d_adam_step" in syms


def test_library_exports_every_declared_symbol():
    lib = _abi.lib()
    missing = [s for s in declared_symbols() if not hasattr(lib, s)]
    assert not missing, missing
    assert set(declared_symbols()) <= set(_abi.SIGNATURES)


def test_exports_are_visible_in_dynamic_symbol_table():
    out = subprocess.run(["nm", "-D", "--defined-only", str(_abi.LIB_PATH)], capture_output=True,
                         text=True, check=True).stdout
    exported = {line.split()[-1] for line in out.splitlines() if line.strip()}
    for s in declared_symbols():
        assert s in exported, s


STRUCTS = {
    "gs3d_camera": _abi.Camera, "gs3d_render_options": _abi.RenderOptionsC,
    "gs3d_tiling": _abi.TilingC, "gs3d_gaussians": _abi.GaussiansC,
    "gs3d_render_buffers": _abi.RenderBuffersC, "gs3d_render_outputs": _abi.RenderOutputsC,
    "gs3d_fgradients": _abi.FGradientsC, "gs3d_adam_moments": _abi.AdamMomentsC,
    "gs3d_adam_params": _abi.AdamParamsC, "gs3d_adc_buffers": _abi.AdcBuffersC,
    "gs3d_adc_params": _abi.AdcParamsC, "gs3d_render_only_gaussians": _abi.RenderOnlyGaussiansC,
}


def test_ctypes_struct_layouts_match_header(tmp_path):
    src = tmp_path / "sizes.c"
    lines = [f'printf("{n} %zu\\n", sizeof({n}));' for n in STRUCTS]
    src.write_text(textwrap.dedent(f"""
        #include <stdio.h>
        #include "gs3d.h"
        int main(void) {{ {' '.join(lines)} return 0; }}
    """))
    exe = tmp_path / "sizes"
    subprocess.run(["gcc", "-I", str(REPO / "include"), str(src), "-o", str(exe)], check=True)
    out = subprocess.run([str(exe)], capture_output=True, text=True, check=True).stdout
    sizes = dict(line.split() for line in out.splitlines())
    for name, cls in STRUCTS.items():
        assert int(sizes[name]) == C.sizeof(cls), name


def test_workspace_size_query_needs_no_gpu():
    out = C.c_size_t(0)
    _abi.check(_abi.lib().gs3d_render_forward_workspace_size(1000, 4000, 256, C.byref(out)))
    assert out.value > 4000 * 12
    n = _abi.lib().determine_sort_pairs_temp_storage(None, None, None, None, 10_000, 44)
    assert n >= 10_000 * 12


def test_invalid_arguments_are_reported_not_crashed():
    lib = _abi.lib()
    st = lib.gs3d_render_forward(None, None, None, None, None, None, None, 0, None)
    assert st == _abi.GS3D_ERR_INVALID_ARGUMENT
    assert b"invalid argument" in lib.gs3d_last_error_string()
    with pytest.raises(_abi.Gs3dError):
        _abi.check(st)


def test_render_only_entry_rejects_bad_arguments_without_a_gpu():
    """gs3d_render_forward_render_only validates its arguments before touching the device."""
    lib = _abi.lib()
    null = C.POINTER(_abi.RenderOnlyGaussiansC)()
    st = lib.gs3d_render_forward_render_only(None, null, None, None, None, None, None, 0, None)
    assert st == _abi.GS3D_ERR_INVALID_ARGUMENT
    ro = _abi.RenderOnlyGaussiansC()
    ro.n, ro.sh_degree = 10, 0
    st = lib.gs3d_render_forward_render_only(None, C.byref(ro), None, None, None, None, None, 0, None)
    assert st == _abi.GS3D_ERR_INVALID_ARGUMENT
    assert b"covariances" in lib.gs3d_last_error_string()
