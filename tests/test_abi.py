"""The C ABI library loads without a GPU and exports every symbol include/*.h declares."""
import glob
import os
import re
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared():
    names = set()
    for h in glob.glob(os.path.join(ROOT, "include", "*.h")):
        text = open(h).read()
        names |= set(re.findall(r"NMG_API\s+[\w\s\*]*?\b(nmg_\w+)\s*\(", text))
    return sorted(names)


def test_header_declares_the_boundary():
    names = declared()
    for must in ("nmg_kv_create", "nmg_kv_append", "nmg_kv_visible_rows", "nmg_attend", "nmg_append_attend",
                 "nmg_attend_batch", "nmg_delta_step", "nmg_delta_prefill", "nmg_gated_delta_step", "nmg_allgather"):
        assert must in names


def test_library_loads_and_exports_every_declared_symbol():
    from hero_b200 import _lib

    L = _lib.lib()  # loads with no GPU present: nothing runs at load time
    for name in declared():
        assert hasattr(L, name), name
    assert L.nmg_version().startswith(b"nmg")


def test_exports_are_exactly_the_abi():
    so = os.path.join(ROOT, "hero_b200", "libnmg.so")
    out = subprocess.run(["nm", "-D", "--defined-only", so], capture_output=True, text=True, check=True).stdout
    exported = {ln.split()[-1] for ln in out.splitlines() if " T " in ln and ln.split()[-1].startswith("nmg_")}
    assert exported == set(declared())


def test_python_binding_covers_the_abi():
    from hero_b200 import _lib

    assert set(_lib.SIGNATURES) | {"nmg_last_error", "nmg_version"} == set(declared())


def test_errors_map_to_reference_exception_types():
    from hero_b200 import _lib

    assert issubclass(_lib.InvalidArgument, ValueError)
    assert issubclass(_lib.OutOfRange, IndexError)
    assert issubclass(_lib.NoVisibleKeys, RuntimeError)
    with pytest.raises(_lib.InvalidArgument):
        # argument checking happens before any device work
        _lib.call("nmg_kv_create", 0, 128, 0, 0, 16, 0, None)


def test_layer_steps_check_arguments_before_device_work():
    # The steps either side of the reductions reject bad shapes with the
    # reference's exception types before touching a device.
    from hero_b200 import _lib

    p = 16  # any non-null address: nothing is dereferenced on these paths
    with pytest.raises(_lib.InvalidArgument):  # Hq not a multiple of Hkv
        _lib.call("nmg_attn_prepare", 3, 2, 128, 0, 4, p, 1, p, p, p, p, 0, 1e-6, 1e4, 1, 1, p, 0, p, None, None)
    with pytest.raises(_lib.InvalidArgument):  # rotary fraction above one
        _lib.call("nmg_attn_prepare", 4, 2, 128, 0, 4, p, 1, p, p, p, p, 0, 1e-6, 1e4, 5, 4, p, 0, p, None, None)
    with pytest.raises(_lib.InvalidArgument):  # a RoPE base must be positive
        _lib.call("nmg_attn_prepare", 4, 2, 128, 0, 4, p, 1, p, p, p, p, 0, 1e-6, 0.0, 1, 1, p, 0, p, None, None)
    with pytest.raises(_lib.Unsupported):  # head_dim not a multiple of 64
        _lib.call("nmg_attn_prepare", 4, 2, 96, 0, 4, p, 1, p, p, p, p, 0, 1e-6, 1e4, 1, 1, p, 0, p, None, None)
    with pytest.raises(_lib.InvalidArgument):  # V normed without a place to put it
        _lib.call("nmg_attn_prepare", 4, 2, 128, 0, 4, p, 0, p, p, p, p, 1, 1e-6, 1e4, 1, 1, p, 0, p, None, None)
    with pytest.raises(_lib.InvalidArgument):
        _lib.call("nmg_attn_prologue", None, 4, 0, 4, p, 1, p, p, p, p, 0, 1e-6, 1e4, 1, 1, p, 0, None)
    with pytest.raises(_lib.InvalidArgument):
        _lib.call("nmg_attn_gate", -1, 4, 128, p, p, 0, None)
    with pytest.raises(_lib.InvalidArgument):
        _lib.call("nmg_attn_gate", 4, 4, 128, p, p, 7, None)  # not a dtype
    _lib.call("nmg_attn_gate", 0, 4, 128, None, None, 0, None)  # zero rows: nothing to do
    import ctypes

    h = ctypes.c_void_p()
    with pytest.raises(_lib.InvalidArgument):
        _lib.call("nmg_conv_create", 0, 4, 0, ctypes.byref(h))  # CausalConv1dState needs channels
    with pytest.raises(_lib.Unsupported):
        _lib.call("nmg_conv_create", 8, 64, 0, ctypes.byref(h))  # a width no kernel is built for
    with pytest.raises(_lib.InvalidArgument):
        _lib.call("nmg_delta_prologue", None, p, 1, 2, 128, 128, 4, *([p] * 10), None)
    with pytest.raises(_lib.InvalidArgument):
        _lib.call("nmg_delta_epilogue", 0, 128, 4, p, p, p, 1e-6, p, None)
