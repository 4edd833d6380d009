"""The C-ABI library loads without a GPU and exports every declared symbol."""
import ctypes as C

import pytest

from finchmoe_b200 import build as fbuild
from finchmoe_b200 import lib as L


@pytest.fixture(scope="module")
def so():
    fbuild.build()
    return L.load()


def test_header_symbols_all_exported(so):
    names = L.declared_symbols()
    assert len(names) >= 25
    for n in names:
        assert hasattr(so, n), f"{n} declared in include/finch_cuda.h but not exported"
    # and the binding table covers exactly the header
    assert sorted(L._PROTOS) == names


def test_status_strings(so):
    assert so.finch_status_str(L.OK) == b"ok"
    assert so.finch_status_str(L.E_TIMEOUT) == b"timeout"
    assert so.finch_status_str(L.E_UNSUPPORTED) == b"unsupported"


def test_ctx_create_rejects_bad_config_before_touching_cuda(so):
    h = C.c_void_p()
    bad = L.Config(0, 2000, 256, 8, 512, 512, 64, 40, 3, L.FP16, L.BF16, 8)  # hidden not a multiple of 128
    assert so.finch_ctx_create(C.byref(bad), C.byref(h)) == L.E_ARG
    bad = L.Config(0, 2048, 256, 9, 512, 512, 64, 40, 3, L.FP16, L.BF16, 8)  # top_k > 8
    assert so.finch_ctx_create(C.byref(bad), C.byref(h)) == L.E_ARG
    bad = L.Config(0, 2048, 256, 8, 512, 512, 64, 40, 4, L.FP16, L.BF16, 8)  # only the 3-bit expert tier
    assert so.finch_ctx_create(C.byref(bad), C.byref(h)) == L.E_ARG
    assert so.finch_ctx_create(None, C.byref(h)) == L.E_ARG


def test_null_handles_are_rejected(so):
    assert so.finch_sync(None) == L.E_ARG
    assert so.finch_matvec(None, None, None, None, 1) == L.E_ARG
    assert so.finch_pool_put(None, 0, 0, None) == L.E_ARG
    assert so.finch_event_wait(None, 1) == L.E_ARG
    assert so.finch_launch_count(None) == 0
