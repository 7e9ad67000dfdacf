"""The C-ABI library loads and exports every function include/boonta_b200.h declares
(CPU only: no compute call is made)."""
import ctypes
import re
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]


def declared_functions():
    text = (ROOT / "include" / "boonta_b200.h").read_text()
    return sorted(set(re.findall(r"BT_API [\w\s\*]+?\b(bt_\w+)\(", text)))


def test_header_declares_the_binding_list():
    from boonta_b200 import _lib

    assert declared_functions() == sorted(_lib.EXPORTS)


def test_library_exports_every_declared_symbol():
    from boonta_b200 import _lib

    lib = ctypes.CDLL(str(_lib.LIB_PATH))
    missing = [name for name in declared_functions() if not hasattr(lib, name)]
    assert not missing, missing


def test_version_and_error_strings_without_a_gpu():
    from boonta_b200 import _lib

    lib = _lib.lib()
    assert b"sm_100a" in lib.bt_version()
    # an invalid argument is rejected on the host, before any CUDA call
    rc = lib.bt_learner_create(None, None)
    assert rc == _lib.BT_ERR_INVALID
    assert b"null" in lib.bt_last_error()


def test_python_layout_is_aligned_and_disjoint():
    from boonta_b200 import configs
    from boonta_b200.spec import ALIGN, param_layout

    for name in configs.WORKLOADS:
        lay = param_layout(configs.make(name).network)
        end = 0
        for e in lay.entries:
            assert e.offset >= end
            end = e.offset + e.size
        assert lay.total % ALIGN == 0 and lay.total >= end
