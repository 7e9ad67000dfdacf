"""Static checks of the XLA FFI binding (boonta_b200/csrc/xla_ffi.cc, boonta_b200/jax_ffi.py).

Neither jax nor jaxlib's FFI headers are installed here, so the handler file cannot be compiled
or called in this image; these tests check, on the CPU, that the Python side registers exactly
the handler getters the C++ file exports and that every C-ABI function the handlers call is
declared in include/boonta_b200.h."""
import re
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]
CC = (ROOT / "boonta_b200" / "csrc" / "xla_ffi.cc").read_text()
HEADER = (ROOT / "include" / "boonta_b200.h").read_text()


def test_python_registers_exactly_the_exported_handler_getters():
    from boonta_b200 import jax_ffi

    exported = set(re.findall(r"BT_API void\* (bt_xla_\w+)\(\)", CC))
    assert exported == set(jax_ffi.TARGETS.values())
    assert set(jax_ffi.TARGETS) == {"boonta_gae", "boonta_ppo_update",
                                    "boonta_recurrent_ppo_update", "boonta_ppo_act"}


def test_handlers_call_only_declared_c_abi_functions():
    called = set(re.findall(r"\b(bt_[a-z_]+)\(", CC)) - {
        name for name in re.findall(r"\b(bt_xla_\w+)\(", CC)}
    declared = set(re.findall(r"BT_API [^(]*?\b(bt_\w+)\(", HEADER))
    assert called and called <= declared, called - declared


def test_the_build_compiles_the_handlers_only_against_jaxlib_headers():
    from boonta_b200 import build

    src = (ROOT / "boonta_b200" / "build.py").read_text()
    assert 'xla" / "ffi" / "api" / "ffi.h"' in src
    # no stand-in header ships with the repository
    assert not list(ROOT.rglob("ffi.h"))
    assert build.CSRC.joinpath("xla_ffi.cc").exists()
