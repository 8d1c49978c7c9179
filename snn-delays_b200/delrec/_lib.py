"""ctypes binding of ``libdelrec_b200.so`` (the C-ABI declared in include/delrec_b200.h).

The library is loaded from this directory; nothing here falls back to a CPU or
PyTorch implementation: a missing library, a non-CUDA tensor or a nonzero status
raises.  Scratch memory for the kernels comes from a per-(device, stream) workspace
tensor owned by this module and grown on demand through torch's caching allocator.
"""

from __future__ import annotations

import ctypes
import os

import torch

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libdelrec_b200.so")

OK = 0
ERRORS = {1: "invalid argument", 2: "CUDA error", 3: "workspace too small or misaligned",
          4: "unsupported shape"}
AXONAL, SYNAPTIC, HYBRID = 0, 1, 2
HARD_STE, HARD_APPROX = 1, 2     # delrec_axonal_backward_hard modes
SURR_TRIANGLE, SURR_ATAN = 0, 1


class LIF(ctypes.Structure):
    _fields_ = [("tau", ctypes.c_float), ("v_threshold", ctypes.c_float),
                ("v_reset", ctypes.c_float), ("soft_reset", ctypes.c_int32),
                ("detach_reset", ctypes.c_int32), ("surrogate", ctypes.c_int32),
                ("gamma", ctypes.c_float), ("alpha", ctypes.c_float)]


class Layer(ctypes.Structure):
    _fields_ = [("kind", ctypes.c_int32), ("T", ctypes.c_int32), ("B", ctypes.c_int32),
                ("N", ctypes.c_int32), ("L", ctypes.c_int32), ("K", ctypes.c_int32),
                ("has_bias", ctypes.c_int32), ("has_keep", ctypes.c_int32),
                ("s_max", ctypes.c_float), ("d_min", ctypes.c_float)]


class Grads(ctypes.Structure):
    _fields_ = [("dx", ctypes.c_void_p), ("dW", ctypes.c_void_p), ("dbias", ctypes.c_void_p),
                ("dd", ctypes.c_void_p), ("ds", ctypes.c_void_p)]


_P = ctypes.c_void_p
_I = ctypes.c_int
_F = ctypes.c_float
_S = ctypes.c_size_t
_SIGS = {
    "delrec_build_mask": (_I, [_I, _I, _P, _P, _I, _P, _P]),
    "delrec_axonal_forward_workspace": (_S, [_P]),
    "delrec_synaptic_forward_workspace": (_S, [_P]),
    "delrec_hybrid_forward_workspace": (_S, [_P]),
    "delrec_axonal_backward_workspace": (_S, [_P]),
    "delrec_synaptic_backward_workspace": (_S, [_P]),
    "delrec_hybrid_backward_workspace": (_S, [_P]),
    "delrec_axonal_forward": (_I, [_P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _S, _P]),
    "delrec_axonal_forward_noalloc": (_I, [_P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P]),
    "delrec_synaptic_forward": (_I, [_P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _S, _P]),
    "delrec_hybrid_forward": (_I, [_P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _S, _P]),
    "delrec_axonal_backward": (_I, [_P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _S, _P]),
    "delrec_axonal_backward_hard_workspace": (_S, [_P]),
    "delrec_axonal_backward_hard": (_I, [_P, _P, _I, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _S, _P]),
    "delrec_synaptic_backward": (_I, [_P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _S, _P]),
    "delrec_hybrid_backward": (_I, [_P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _S, _P]),
    "delrec_hybrid_delay_grad": (_I, [_I, _I, _P, _P, _P, _F, _P, _P]),
    "delrec_lif_forward": (_I, [_I, _I, _P, _P, _P, _P, _P]),
    "delrec_lif_backward": (_I, [_I, _I, _P, _P, _P, _P, _P]),
    "delrec_dcls_forward": (_I, [_I, _I, _I, _I, _I, _I, _I, _P, _P, _P, _P, _P, _P, _P, _P]),
    "delrec_dcls_backward_workspace": (_S, [_I, _I, _I, _I, _I, _I]),
    "delrec_dcls_backward": (_I, [_I, _I, _I, _I, _I, _I, _I, _P, _P, _P, _P, _P, _P, _P, _P,
                                  _P, _P, _P, _S, _P]),
    "delrec_linear_forward_workspace": (_S, [_I, _I, _I, _I]),
    "delrec_linear_forward": (_I, [_I, _I, _I, _P, _P, _P, _I, _P, _P, _S, _P]),
    "delrec_linear_backward_workspace": (_S, [_I, _I, _I, _I]),
    "delrec_linear_backward": (_I, [_I, _I, _I, _P, _P, _P, _I, _P, _P, _P, _P, _S, _P]),
    "delrec_count_nonbinary": (_I, [_P, _S, _P, _P]),
    "delrec_tc_gemm_workspace": (_S, [_I, _I, _I]),
    "delrec_tc_gemm": (_I, [_I, _I, _I, _I, _I, _P, ctypes.c_longlong, _I, _P, ctypes.c_longlong, _I, _P, _P, _I, _I,
                            _P, ctypes.c_longlong, _I, _P, _S, _P]),
    "delrec_get_status": (_I, [_P]),
    "delrec_clear_status": (_I, []),
    "delrec_version": (ctypes.c_char_p, []),
    "delrec_launch_count": (ctypes.c_ulonglong, []),
    "delrec_scan_timing": (_I, [_I]),
    "delrec_scan_time": (_I, [_P, _P]),
    "delrec_scan_time_part": (_I, [_I, _P, _P]),
    "delrec_set_reverse_scan": (_I, [_I]),
    "delrec_readout_sum_forward": (_I, [_I, _I, _I, _I, _P, _P, _P, _P, _P, _P]),
    "delrec_readout_sum_backward": (_I, [_I, _I, _I, _I, _P, _P, _P, _P, _P, _P, _P]),
    "delrec_exchange_floor_workspace": (_S, [_P]),
    "delrec_exchange_floor": (_I, [_P, _P, _S, _P]),
}

_lib = None


def lib():
    """The loaded library (raises if it was not built)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(
                f"delrec_b200: CUDA library not found at {LIB_PATH}; build it with "
                "`python -c 'import __graft_entry__ as g; g.build()'` (or `make` in csrc/)")
        handle = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in _SIGS.items():
            fn = getattr(handle, name)
            fn.restype = res
            fn.argtypes = args
        _lib = handle
    return _lib


def exported_symbols():
    return list(_SIGS)


def check(rc: int, what: str):
    if rc != OK:
        raise RuntimeError(f"delrec_b200: {what} failed: {ERRORS.get(rc, rc)} (code {rc})")


def ptr(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def require_cuda(*tensors):
    for t in tensors:
        if t is None:
            continue
        if not t.is_cuda:
            raise RuntimeError("delrec_b200 runs on CUDA tensors only (there is no CPU path)")
        if t.dtype != torch.float32:
            raise RuntimeError(f"delrec_b200 expects float32 tensors, got {t.dtype}")
        if not t.is_contiguous():
            raise RuntimeError("delrec_b200 expects contiguous tensors")


def stream_ptr(device=None):
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


_ws_cache: dict = {}


def workspace(nbytes: int, device) -> torch.Tensor:
    """A uint8 scratch tensor of at least ``nbytes`` (256-byte aligned) for ``device``,
    reused across calls on the current stream."""
    key = (torch.device(device).index, torch.cuda.current_stream(device).cuda_stream)
    buf = _ws_cache.get(key)
    need = max(int(nbytes), 256)
    if buf is None or buf.numel() < need:
        buf = torch.empty(need + 256, dtype=torch.uint8, device=device)
        _ws_cache[key] = buf
    off = (-buf.data_ptr()) % 256
    return buf[off:off + need]


def release_workspaces():
    _ws_cache.clear()


def lif_struct(tau, v_threshold, v_reset, detach_reset, surrogate_id, gamma, alpha) -> LIF:
    soft = v_reset is None
    return LIF(float(tau), float(v_threshold), 0.0 if soft else float(v_reset), int(soft),
               int(bool(detach_reset)), int(surrogate_id), float(gamma), float(alpha))


def launch_count() -> int:
    return int(lib().delrec_launch_count())


def scan_timing(enable: bool):
    check(lib().delrec_scan_timing(int(enable)), "delrec_scan_timing")


def scan_time(part=0):
    """(total milliseconds, launches) of the reverse-scan kernels timed since enabling:
    part 0 every scan, 1 the step launches of the chunked scans, 2 their chunk GEMMs."""
    ms = ctypes.c_double(0.0)
    n = ctypes.c_int(0)
    check(lib().delrec_scan_time_part(int(part), ctypes.byref(ms), ctypes.byref(n)), "delrec_scan_time_part")
    return ms.value, n.value


REVERSE_SCAN_CHUNKED, REVERSE_SCAN_STEPWISE, REVERSE_SCAN_CHUNKED_EXCHANGE = 0, 1, 2


def set_reverse_scan(variant: int):
    """Select the layer backwards' reverse scan for this process: REVERSE_SCAN_CHUNKED
    (default: hybrid layers contract their long-lag synapses once per 8-step chunk on the
    tensor cores) or REVERSE_SCAN_STEPWISE (the step-by-step scans only)."""
    check(lib().delrec_set_reverse_scan(int(variant)), "delrec_set_reverse_scan")


def exchange_floor_ms(T, B, N, K=0, repeats=3, device=None):
    """Milliseconds of the reverse scans' per-step exchange alone over T steps (the latency
    floor of one layer's scan) on the tiling used for a (T, B, N) layer; the median of
    ``repeats`` launches timed with CUDA events on the current stream."""
    import statistics
    layer = Layer(HYBRID, int(T), int(B), int(N), 2, int(K), 0, 0, 1.0, 0.0)
    nbytes = lib().delrec_exchange_floor_workspace(ctypes.byref(layer))
    if nbytes == 0:
        raise RuntimeError("delrec_b200: no exchange-floor tiling for this shape")
    ws = workspace(nbytes, device or torch.cuda.current_device())
    st = stream_ptr(device)
    times = []
    for _ in range(repeats + 1):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        check(lib().delrec_exchange_floor(ctypes.byref(layer), ptr(ws), nbytes, st), "delrec_exchange_floor")
        b.record()
        torch.cuda.synchronize()
        times.append(a.elapsed_time(b))
    return statistics.median(times[1:])


def status() -> int:
    out = ctypes.c_int(0)
    check(lib().delrec_get_status(ctypes.byref(out)), "delrec_get_status")
    return out.value
