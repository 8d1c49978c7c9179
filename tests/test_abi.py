"""The C-ABI library: it loads without a GPU, exports every entry point the header
declares, and its host-side checks reject bad arguments before touching the device."""

import ctypes
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "delrec_b200.h")


def _declared():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(delrec_[a-z0-9_]+)\s*\(", src)))


def test_library_exports_every_declared_symbol():
    from delrec import _lib
    handle = _lib.lib()
    names = _declared()
    assert len(names) >= 20
    for n in names:
        assert hasattr(handle, n), f"{n} declared in include/delrec_b200.h but not exported"
    # and the Python binding knows every one of them
    assert set(names) <= set(_lib.exported_symbols())


def test_version_string():
    from delrec import _lib
    assert _lib.lib().delrec_version().startswith(b"delrec_b200")


def _layer(kind=0, T=4, B=2, N=8, L=5, K=0, s_max=1.0):
    from delrec import _lib
    return _lib.Layer(kind, T, B, N, L, K, 0, 0, s_max)


def test_workspace_queries_are_host_only():
    from delrec import _lib
    lib = _lib.lib()
    for kind, fw, bw in ((0, "delrec_axonal_forward_workspace", "delrec_axonal_backward_workspace"),
                         (1, "delrec_synaptic_forward_workspace", "delrec_synaptic_backward_workspace"),
                         (2, "delrec_hybrid_forward_workspace", "delrec_hybrid_backward_workspace")):
        ly = _layer(kind=kind, T=250, B=256, N=512, L=37, K=8)
        f = getattr(lib, fw)(ctypes.byref(ly))
        b = getattr(lib, bw)(ctypes.byref(ly))
        assert f > 0 and b > 0
        assert b >= 250 * 256 * 512 * 4  # at least the gr buffer
        assert f % 256 == 0 and b % 256 == 0


def test_bad_arguments_are_rejected_without_device_work():
    from delrec import _lib
    lib = _lib.lib()
    lif = _lib.lif_struct(2.0, 1.0, 0.0, False, 1, 1.0, 2.0)
    ly = _layer()
    fake = ctypes.c_void_p(256)
    # null input pointer
    rc = lib.delrec_axonal_forward(ctypes.byref(ly), ctypes.byref(lif), None, fake, None, fake, fake,
                                   None, fake, fake, fake, 1 << 20, None)
    assert rc == 1
    # wrong kind for the entry point
    bad = _layer(kind=1)
    rc = lib.delrec_axonal_forward(ctypes.byref(bad), ctypes.byref(lif), fake, fake, None, fake, fake,
                                   None, fake, fake, fake, 1 << 20, None)
    assert rc == 1
    # misaligned / too small workspace
    rc = lib.delrec_axonal_forward(ctypes.byref(ly), ctypes.byref(lif), fake, fake, None, fake, fake,
                                   None, fake, fake, ctypes.c_void_p(257), 1 << 20, None)
    assert rc == 3
    rc = lib.delrec_axonal_forward(ctypes.byref(ly), ctypes.byref(lif), fake, fake, None, fake, fake,
                                   None, fake, fake, fake, 16, None)
    assert rc == 3
    # unsupported half-width
    wide = _layer(s_max=9.0)
    rc = lib.delrec_axonal_forward(ctypes.byref(wide), ctypes.byref(lif), fake, fake, None, fake, fake,
                                   None, fake, fake, fake, 1 << 20, None)
    assert rc == 4
    # DCLS shape checks
    rc = lib.delrec_dcls_forward(4, 2, 9, 128, 2, 5, 4, fake, fake, fake, fake, None, fake, fake, None)
    assert rc == 1


def test_cpu_tensors_raise():
    import torch
    from delrec import _lib
    with pytest.raises(RuntimeError, match="CUDA"):
        _lib.require_cuda(torch.zeros(3))
