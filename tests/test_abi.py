"""libasap loads without a GPU and exports every function include/asap.h declares; argument checks that need
no device return the documented error codes."""

import ctypes
import os
import re

import pytest

from asap_b200 import _native as N

HEADER = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "include", "asap.h")


def header_functions():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(asap_[a-z0-9_]+)\s*\(", text)))


def test_header_lists_functions():
    fns = header_functions()
    assert "asap_dispatch" in fns and "asap_ffn_job" in fns and "asap_combine" in fns


def test_every_declared_symbol_is_exported():
    lib = ctypes.CDLL(N.LIB_PATH)
    missing = [f for f in header_functions() if not hasattr(lib, f)]
    assert not missing, missing


def test_binding_covers_header():
    assert sorted(N.exported_symbols()) == header_functions()


def test_version():
    assert b"sm_100a" in N.lib().asap_version()


def test_dispatch_rejects_bad_arguments_without_touching_a_gpu():
    g = N.Geometry_t(1, 1, 2, 64, 256, 2, 1)
    F = 1
    ep = (ctypes.c_int32 * F)(1)
    b = (ctypes.c_int32 * (F + 1))(0, 4)
    ptrs = (ctypes.c_uint64 * F)(0x1000)
    # n_tokens out of range
    rc = N.lib().asap_dispatch(ctypes.byref(g), 0, 0, 1, 0, ep, 0x1000, 0x1000, 0, 0x1000, 0, 65, b, ptrs, ptrs,
                               0x1000, 0x1000, 1, 0, 1, None)
    assert rc == N.ASAP_EINVAL
    assert "n_tokens 65" in N.lib().asap_last_error_string().decode()
    # bad epoch
    ep0 = (ctypes.c_int32 * F)(0)
    rc = N.lib().asap_dispatch(ctypes.byref(g), 0, 0, 1, 0, ep0, 0x1000, 0x1000, 0, 0x1000, 0, 4, b, ptrs, ptrs,
                               0x1000, 0x1000, 1, 0, 1, None)
    assert rc == N.ASAP_EINVAL
    assert "epoch=0" in N.lib().asap_last_error_string().decode()
    # layer out of range
    rc = N.lib().asap_dispatch(ctypes.byref(g), 0, 0, 1, 1024, ep, 0x1000, 0x1000, 0, 0x1000, 0, 4, b, ptrs, ptrs,
                               0x1000, 0x1000, 1, 0, 1, None)
    assert rc == N.ASAP_EINVAL


def test_ffn_entry_points_reject_unknown_handles():
    assert N.lib().asap_ffn_job(12345, 678, 16, 16, 16, 16, 0, ctypes.c_float(0), 0, 1, None) == N.ASAP_EINVAL
    assert N.lib().asap_experts_release(999) == N.ASAP_EINVAL
    assert N.lib().asap_ffn_ws_release(999) == N.ASAP_EINVAL


def test_experts_register_validates_shapes():
    e = N.Mxfp4Experts_t(0, 0, 7168, 2048, 32, 32, 32, 32)
    h = ctypes.c_uint64()
    assert N.lib().asap_experts_register(ctypes.byref(e), ctypes.byref(h)) == N.ASAP_EINVAL
    e = N.Mxfp4Experts_t(4, 0, 100, 2048, 32, 32, 32, 32)
    assert N.lib().asap_experts_register(ctypes.byref(e), ctypes.byref(h)) == N.ASAP_EINVAL


def test_ws_bytes_scale():
    small = N.lib().asap_ffn_ws_bytes(64, 2, 4, 256, 128)
    big = N.lib().asap_ffn_ws_bytes(16384, 8, 256, 7168, 2048)
    assert 0 < small < big
    assert N.lib().asap_ffn_ws_bytes(0, 2, 4, 256, 128) == 0


def test_route_ws_bytes():
    g = N.Geometry_t(4, 1, 2, 16384, 7168, 8, 4)
    assert N.lib().asap_route_ws_bytes(ctypes.byref(g)) == 512 + 8 * 16384 * 4  # row_of + tok_of per F rank


@pytest.mark.parametrize("status,expect", [(0, "ok"), (1 | (3 << 8) | (1 << 16) | (77 << 32), "backpressure timeout")])
def test_decode_status(status, expect):
    d = N.decode_status(status)
    assert d["what"] == expect
    if status:
        assert (d["f"], d["slot"], d["seq"]) == (3, 1, 77)


def test_host_pages_and_release_without_a_gpu(tmp_path):
    """asap_host_page_create/open and asap_release: every argument and file error is reported before any device
    call; with no GPU the registration fails and the page this call created is removed again."""
    lib = N.lib()
    host, dev = ctypes.c_uint64(), ctypes.c_uint64()
    assert lib.asap_release(0x1234) == N.ASAP_EINVAL
    assert "not handed out" in lib.asap_last_error_string().decode()
    assert lib.asap_host_page_create(None, 4096, ctypes.byref(host), ctypes.byref(dev)) == N.ASAP_EINVAL
    assert lib.asap_host_page_create(str(tmp_path / "p").encode(), 0, ctypes.byref(host), ctypes.byref(dev)) == \
        N.ASAP_EINVAL
    missing = str(tmp_path / "missing").encode()
    assert lib.asap_host_page_open(missing, 4096, ctypes.byref(host), ctypes.byref(dev)) == N.ASAP_EINVAL
    assert "cannot open" in lib.asap_last_error_string().decode()
    short = tmp_path / "short"
    short.write_bytes(b"\0" * 100)
    assert lib.asap_host_page_open(str(short).encode(), 4096, ctypes.byref(host), ctypes.byref(dev)) == N.ASAP_EINVAL
    assert "is not 4096 bytes" in lib.asap_last_error_string().decode()
    assert lib.asap_host_page_create(str(short).encode(), 4096, ctypes.byref(host), ctypes.byref(dev)) == \
        N.ASAP_EINVAL  # exists
    import torch

    if not torch.cuda.is_available():
        page = tmp_path / "page"
        rc = lib.asap_host_page_create(str(page).encode(), 4096, ctypes.byref(host), ctypes.byref(dev))
        assert rc == N.ASAP_ECUDA and not page.exists()
