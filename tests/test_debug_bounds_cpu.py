"""Host half of the bounds-checked comm kernels, without a GPU: the extent
registry both extension modules keep (tightest registered range containing a
pointer, unregistering), which build each module is, and the
``LRL_DEBUG_BOUNDS`` switch that routes the comm ops to the checked module."""

import importlib

import pytest


def _mods():
    import torch  # noqa: F401  (loads libc10 for the extensions)
    try:
        return importlib.import_module("lumenrl_b200._C"), importlib.import_module("lumenrl_b200._C_bounds")
    except ImportError as e:
        pytest.skip(f"extensions not built: {e}")


def test_builds_identify_themselves():
    C, B = _mods()
    assert C.debug_bounds_build() is False
    assert B.debug_bounds_build() is True
    assert C.bounds_status() == 0           # the ordinary build has no status word


@pytest.mark.parametrize("mod", [0, 1])
def test_registry_returns_tightest_containing_range(mod):
    M = _mods()[mod]
    base = 1 << 44                          # host-side bookkeeping only: never dereferenced
    M.bounds_register(base, 4096)
    M.bounds_register(base + 1024, 100)
    M.bounds_register(base + 8192, 64)
    try:
        assert M.bounds_lookup(base) == [base, base + 4096]
        assert M.bounds_lookup(base + 1030) == [base + 1024, base + 1124]   # nested: the inner range
        assert M.bounds_lookup(base + 1124) == [base, base + 4096]          # just past the inner one
        assert M.bounds_lookup(base + 8192 + 63) == [base + 8192, base + 8256]
        M.bounds_unregister(base + 1024)
        assert M.bounds_lookup(base + 1030) == [base, base + 4096]
    finally:
        for p in (base, base + 1024, base + 8192):
            M.bounds_unregister(p)


def test_registration_rejects_null_and_negative_sizes():
    C, _ = _mods()
    with pytest.raises(RuntimeError):
        C.bounds_register(0, 16)
    with pytest.raises(RuntimeError):
        C.bounds_register(1 << 44, -1)


def test_env_switch_routes_comm_ops(monkeypatch):
    _mods()
    ext_mod = importlib.import_module("lumenrl_b200.ops.ext")
    saved = (ext_mod._MOD, ext_mod._ERR)
    try:
        monkeypatch.setenv("LRL_DEBUG_BOUNDS", "0")
        ext_mod._MOD, ext_mod._ERR = None, None
        assert ext_mod.ext().debug_bounds_build() is False
        monkeypatch.setenv("LRL_DEBUG_BOUNDS", "1")
        ext_mod._MOD, ext_mod._ERR = None, None
        e = ext_mod.ext()
        assert e.debug_bounds_build() is True
        assert callable(e.rmsnorm_fwd) and callable(e.p2p_push)
    finally:
        ext_mod._MOD, ext_mod._ERR = saved
