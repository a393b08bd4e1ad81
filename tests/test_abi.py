"""The C ABI library: loads without a GPU, exports every symbol include/fkb200.h declares,
and rejects bad arguments before touching the device (no compute calls here)."""
import ctypes
import re
from pathlib import Path

import pytest

from fusedkernels_b200 import _lib

HEADER = Path(__file__).resolve().parents[1] / "include" / "fkb200.h"


def declared_symbols():
    text = HEADER.read_text()
    return sorted(set(re.findall(r"FK_API\s+[\w\s\*]+?\b(fk_\w+)\s*\(", text)))


def test_header_declares_entry_points():
    syms = declared_symbols()
    assert "fk_router_fwd" in syms and "fk_ce_fwd" in syms and len(syms) >= 12


def test_library_exports_every_declared_symbol():
    lib = ctypes.CDLL(str(_lib.LIB_PATH))
    missing = [s for s in declared_symbols() if not hasattr(lib, s)]
    assert not missing, f"missing exports: {missing}"


def test_binding_covers_header():
    assert set(declared_symbols()) <= set(_lib.SIGNATURES)


def test_status_strings():
    lib = _lib.load()
    assert lib.fk_version() >= 100
    assert lib.fk_status_string(0) == b"ok"
    assert lib.fk_status_string(1) == b"invalid argument"


@pytest.mark.parametrize("k,E", [(0, 8), (9, 8)])
def test_router_rejects_bad_k(k, E):
    lib = _lib.load()
    st = lib.fk_router_fwd(None, E, 0, 4, E, k, None, None, None)
    assert st == 1 and b"k" in lib.fk_last_error()


def test_router_rejects_too_many_experts():
    lib = _lib.load()
    assert lib.fk_router_fwd(None, 512, 0, 4, 512, 2, None, None, None) == 2


def test_negative_sizes_and_bad_dtype_rejected():
    lib = _lib.load()
    assert lib.fk_swiglu_fwd(None, None, None, -1, 0, None) == 1
    assert lib.fk_swiglu_fwd(None, None, None, 0, 0, None) == 0  # empty: no-op
    assert lib.fk_rmsnorm_fwd(None, 8, None, 0, None, 8, None, -1, 8, 1e-6, 0, None) == 1
    assert lib.fk_ce_fwd(None, 4, None, 4, None, 2, 0, -100, 0.0, 0, None, None, None, None,
                         None) == 1
    with pytest.raises(RuntimeError, match="invalid argument"):
        _lib.call("fk_router_bwd", None, None, None, None, 4, 8, 9, None)


def test_ce_rejects_bad_smoothing():
    lib = _lib.load()
    one = ctypes.c_int(0)
    f = ctypes.c_float(0)
    st = lib.fk_ce_fwd(None, 4, None, 4, None, 0, 4, -100, 1.5, 0, None, ctypes.byref(f),
                       ctypes.byref(one), ctypes.byref(one), None)
    assert st == 1


def test_ep_planning_workspace_and_peer_argument_checks():
    """The expert-parallel entry points validate their arguments on the host (no device
    work happens for a rejected call)."""
    lib = _lib.load()
    n = ctypes.c_size_t(0)
    assert lib.fk_ep_plan_workspace_size(1000, 8, ctypes.byref(n)) == 0
    assert n.value == 4 * 8 * 4  # ceil(1000 / 256) chunks x 8 ranks x int32
    assert lib.fk_ep_plan_workspace_size(10, 33, ctypes.byref(n)) == 1  # at most 32 ranks
    # n_ranks 0, my_rank out of range, phase out of range
    assert lib.fk_ep_peer_put_rows(None, 64, None, 4, 0, 0, None, None, 2, None, None, None,
                                   None, 0, None, 2, None) == 1
    assert lib.fk_ep_peer_put_rows(None, 64, None, 4, 2, 2, None, None, 2, None, None, None,
                                   None, 0, None, 2, None) == 1
    assert lib.fk_ep_peer_combine_put(None, 64, None, None, 4, 2, 0, 2, None, None, None, None,
                                      4, None, 2, None) == 1
    assert lib.fk_ep_peer_wait(None, 2, 0, None, 100, None, None) == 1
    assert lib.fk_ep_peer_wait(None, 0, 0, None, 100, None, None) == 1
    assert lib.fk_ipc_alloc(0, None, None) == 1
    assert lib.fk_ipc_open(None, None) == 1
