"""The built C-ABI library loads and exports every entry point its header declares.

No compute call is made: this runs on hosts without a GPU.
"""

import ctypes
import re
from pathlib import Path

import pytest

from purin_b200 import _native

HEADER = Path(__file__).resolve().parents[1] / "include" / "purin_cp.h"


def declared_functions():
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"^\s*(?:int32_t|const char\*)\s+(purin_\w+)\s*\(", text,
                                 flags=re.M)))


def test_header_declares_the_entry_points():
    names = declared_functions()
    for required in ("purin_cp_plan_create", "purin_cp_forward", "purin_cp_adjoint",
                     "purin_cp_postprocess", "purin_cp_workspace_size", "purin_cp_last_error"):
        assert required in names


def test_library_loads_and_exports_every_declared_symbol():
    path = _native.library_path()
    if not path.exists():
        from purin_b200.csrc.build import build

        build()
    lib = ctypes.CDLL(str(path))
    missing = [name for name in declared_functions() if not hasattr(lib, name)]
    assert not missing, f"library does not export {missing}"
    lib.purin_cp_abi_version.restype = ctypes.c_int32
    assert lib.purin_cp_abi_version() == _native.ABI_VERSION


def test_plan_creation_reports_a_missing_device_or_bad_structure():
    """Without a GPU (or with bad input) plan creation fails with a message, not a crash."""
    lib = _native.load()
    row_ptr = (ctypes.c_int32 * 2)(0, 1)
    col = (ctypes.c_int32 * 1)(5)  # column out of range for n = 2
    s = _native.Structure(2, 1, 0, row_ptr, col, 0, 0)
    handle = ctypes.c_void_p()
    status = lib.purin_cp_plan_create(ctypes.byref(s), ctypes.byref(handle))
    assert status != 0
    assert lib.purin_cp_last_error()


def test_binding_constants_match_the_header_enums():
    """The ctypes binding's op and stage codes are the header's (a mismatch would
    size workspaces for the wrong computation)."""
    text = HEADER.read_text()
    enum = dict((name, int(value)) for name, value in
                re.findall(r"^\s*(PURIN_(?:CP|QP)_(?:OP|STAGE)_\w+)\s*=\s*(\d+)", text, flags=re.M))
    expected = {
        "PURIN_CP_OP_FORWARD": _native.OP_FORWARD,
        "PURIN_CP_OP_ADJOINT": _native.OP_ADJOINT,
        "PURIN_QP_OP_FORWARD": _native.QP_OP_FORWARD,
        "PURIN_QP_OP_ADJOINT": _native.QP_OP_ADJOINT,
        "PURIN_CP_OP_FORWARD_SAMPLE_VALUES": _native.OP_FORWARD_SAMPLE_VALUES,
        "PURIN_QP_OP_FORWARD_SAMPLE_VALUES": _native.QP_OP_FORWARD_SAMPLE_VALUES,
        "PURIN_CP_STAGE_PREPARE": _native.STAGE_PREPARE,
        "PURIN_CP_STAGE_CYCLE": _native.STAGE_CYCLE,
        "PURIN_CP_STAGE_FINISH": _native.STAGE_FINISH,
    }
    assert enum == expected
    for name in _native.EXPORTED:
        assert name in declared_functions()
