"""ctypes binding of libictc_o2_b200.so, the C-ABI declared in include/ictc_o2_b200.h.

This is the only place Python touches the native library.  A missing library is a
hard error: the package has no CPU or PyTorch fallback for the kernels.
"""

from __future__ import annotations

import ctypes
import os
import threading
from pathlib import Path

import torch

LIBRARY = Path(__file__).resolve().parent / "_lib" / "libictc_o2_b200.so"

OK, ERR_INVALID, ERR_UNSUPPORTED, ERR_CUDA, ERR_WORKSPACE = range(5)
PARITY = {"canonical": 0, "full": 1}
NORMALIZATION = {"component": 0, "norm": 1}

_c_float_p = ctypes.POINTER(ctypes.c_float)
_i32, _i64, _size = ctypes.c_int32, ctypes.c_int64, ctypes.c_size_t
_vp = ctypes.c_void_p

# name -> (restype, argtypes); must mirror include/ictc_o2_b200.h
SIGNATURES = {
    "ictc_o2_last_error": (ctypes.c_char_p, []),
    "ictc_o2_abi_version": (_i32, []),
    "ictc_o2_device_error": (_i32, [ctypes.POINTER(_i32)]),
    "ictc_o2_test_wait_timeout": (_i32, [_i32, _vp, _vp]),
    "ictc_o2_tp_weight_numel": (_i32, [_i32, _i32, _i32, ctypes.POINTER(_i64)]),
    "ictc_o2_tp_path_table": (_i32, [_i32, _i32, ctypes.POINTER(_i32), _i32,
                                     ctypes.POINTER(_i32)]),
    "ictc_o2_tp_forward": (_i32, [_vp, _vp, _vp, _vp, _i64, _i32, _i32, _i32, _i32, _vp]),
    "ictc_o2_tp_backward_workspace": (_i32, [_i64, _i32, _i32, _i32, _i32,
                                             ctypes.POINTER(_size)]),
    "ictc_o2_tp_backward": (_i32, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _size, _i64, _i32,
                                   _i32, _i32, _i32, _vp]),
    "ictc_o2_tp_backward_noalloc": (_i32, [_vp] * 7 + [_i64, _i32, _i32, _i32, _i32, _vp]),
    "ictc_o2_tp_forward_layout": (_i32, [_vp, _vp, _vp, _vp, _i64, _i32, _i32, _i32, _i32, _i32,
                                         _vp]),
    "ictc_o2_tp_backward_layout": (_i32, [_vp] * 8 + [_size, _i64, _i32, _i32, _i32, _i32, _i32,
                                                      _vp]),
    "ictc_o2_uvu_table": (_i32, [_i32] * 8 + [ctypes.POINTER(_i32), _i64,
                                              ctypes.POINTER(_i64)]),
    "ictc_o2_uvu_workspace": (_i32, [_i32] * 8 + [_i32, _i64, _i32, ctypes.POINTER(_size),
                                                  ctypes.POINTER(_size)]),
    "ictc_o2_uvu_forward": (_i32, [_vp, _vp, _vp, _vp, _i64] + [_i32] * 8 +
                            [_i32, _vp, _vp, _size, _vp]),
    "ictc_o2_uvu_backward": (_i32, [_vp] * 7 + [_i64] + [_i32] * 8 +
                             [_i32, _i32, _vp, _vp, _size, _vp]),
    "ictc_o2_radial_workspace": (_i32, [_i32] * 8 + [_i64, _i32, ctypes.POINTER(_size),
                                                     ctypes.POINTER(_size)]),
    "ictc_o2_radial_forward": (_i32, [_vp] * 6 + [_i64] + [_i32] * 8 + [_vp, _vp, _size, _vp]),
    "ictc_o2_radial_backward": (_i32, [_vp] * 11 + [_i64] + [_i32] * 8 +
                                [_i32, _vp, _vp, _size, _vp]),
    "ictc_o2_radial_forward_gathered": (_i32, [_vp, _vp, _i64] + [_vp] * 5 + [_i64] +
                                        [_i32] * 8 + [_vp, _vp, _size, _vp]),
    "ictc_o2_radial_backward_gathered": (_i32, [_vp, _vp, _i64] + [_vp] * 10 + [_i64] +
                                         [_i32] * 8 + [_i32, _vp, _vp, _size, _vp]),
    "ictc_o2_gather_rows": (_i32, [_vp, _vp, _vp, _i64, _i64, _i64, _vp]),
    "ictc_o2_segment_sum": (_i32, [_vp, _vp, _vp, _vp, _i64, _i64, _i64, _vp]),
    "ictc_o2_graph_bad_index": (_i32, [ctypes.POINTER(_i32)]),
}

_lock = threading.Lock()
_handle = None


class NativeError(RuntimeError):
    """A CUDA or workspace failure reported by the native library."""


def load() -> ctypes.CDLL:
    """Loads the library once; raises if it has not been built."""
    global _handle
    if _handle is not None:
        return _handle
    with _lock:
        if _handle is None:
            path = Path(os.environ.get("ICTC_O2_B200_LIBRARY", LIBRARY))
            if not path.exists():
                raise RuntimeError(
                    f"{path} is missing: build it with `python -m ictc_o2_hp_b200.build` "
                    "(the kernels have no fallback)")
            lib = ctypes.CDLL(str(path))
            for name, (restype, argtypes) in SIGNATURES.items():
                fn = getattr(lib, name)
                fn.restype, fn.argtypes = restype, argtypes
            _handle = lib
    return _handle


def check(status: int, what: str) -> None:
    if status == OK:
        return
    message = load().ictc_o2_last_error().decode(errors="replace")
    text = f"{what}: {message}"
    if status == ERR_INVALID:
        raise ValueError(text)
    if status == ERR_UNSUPPORTED:
        raise NotImplementedError(text)
    raise NativeError(text)


def ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def stream_of(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def device_error() -> int:
    """Reads and clears the kernels' device-side error flag (0 = none)."""
    code = _i32()
    check(load().ictc_o2_device_error(ctypes.byref(code)), "device_error")
    return int(code.value)


def test_wait_timeout(limit_us: int, waited_ok) -> None:
    """Launches the bounded-wait probe (a wait that can never complete, limit
    `limit_us`); `waited_ok` is a one-element int32 CUDA tensor that receives 0."""
    check(load().ictc_o2_test_wait_timeout(int(limit_us), ptr(waited_ok),
                                           stream_of(waited_ok.device)), "test_wait_timeout")


def tp_weight_numel(channels: int, m_max: int, parity: str) -> int:
    out = _i64()
    check(load().ictc_o2_tp_weight_numel(channels, m_max, PARITY[parity], ctypes.byref(out)),
          "tp_weight_numel")
    return int(out.value)


def tp_path_table(m_max: int, parity: str) -> list[tuple]:
    lib = load()
    count = _i32()
    check(lib.ictc_o2_tp_path_table(m_max, PARITY[parity], None, 0, ctypes.byref(count)),
          "tp_path_table")
    buf = (_i32 * (23 * count.value))()
    check(lib.ictc_o2_tp_path_table(m_max, PARITY[parity], buf, count.value,
                                    ctypes.byref(count)), "tp_path_table")
    rows = []
    for p in range(count.value):
        r = buf[23 * p:23 * (p + 1)]
        terms = tuple(tuple(r[7 + 4 * k:11 + 4 * k]) for k in range(r[6]))
        rows.append((r[0], r[1], r[2], r[3], r[4], r[5], terms))
    return rows


def tp_forward(left, right, weight, out, channels, m_max, parity, normalization, layout=0):
    """layout: 0 channel-major, 1 component-major frequency blocks."""
    rows = left.shape[0]
    check(load().ictc_o2_tp_forward_layout(
        ptr(left), ptr(right), ptr(weight), ptr(out), rows, channels, m_max, PARITY[parity],
        NORMALIZATION[normalization], layout, stream_of(left.device)), "tp_forward")


def tp_backward_workspace(rows, channels, m_max, parity, device: torch.device) -> int:
    out = _size()
    check(load().ictc_o2_tp_backward_workspace(rows, channels, m_max, PARITY[parity],
                                               device.index or 0, ctypes.byref(out)),
          "tp_backward_workspace")
    return int(out.value)


def tp_backward(left, right, weight, grad_output, grad_left, grad_right, grad_weight,
                workspace, channels, m_max, parity, normalization, layout=0):
    rows = left.shape[0]
    check(load().ictc_o2_tp_backward_layout(
        ptr(left), ptr(right), ptr(weight), ptr(grad_output), ptr(grad_left), ptr(grad_right),
        ptr(grad_weight), ptr(workspace), workspace.numel() if workspace is not None else 0,
        rows, channels, m_max, PARITY[parity], NORMALIZATION[normalization], layout,
        stream_of(left.device)), "tp_backward")


# ------------------------------------------------------------------------ uvu
# config = (channels, channels_in2, m_max, parity, m_max_in2, parity_in2,
#           normalization, path_normalization) as ints


def uvu_table(config) -> "np.ndarray":
    import numpy as np
    lib = load()
    words = _i64()
    check(lib.ictc_o2_uvu_table(*config, None, 0, ctypes.byref(words)), "uvu_table")
    buf = np.zeros(words.value, dtype=np.int32)
    check(lib.ictc_o2_uvu_table(*config, buf.ctypes.data_as(ctypes.POINTER(_i32)), words.value,
                                ctypes.byref(words)), "uvu_table")
    return buf


def uvu_workspace(config, shared: bool, rows: int, device: torch.device) -> tuple[int, int]:
    fwd, bwd = _size(), _size()
    check(load().ictc_o2_uvu_workspace(*config, int(shared), rows, device.index or 0,
                                       ctypes.byref(fwd), ctypes.byref(bwd)), "uvu_workspace")
    return int(fwd.value), int(bwd.value)


def uvu_forward(left, right, weight, out, config, shared, table, workspace):
    check(load().ictc_o2_uvu_forward(
        ptr(left), ptr(right), ptr(weight), ptr(out), left.shape[0], *config, int(shared),
        ptr(table), ptr(workspace), workspace.numel() if workspace is not None else 0,
        stream_of(left.device)), "uvu_forward")


def uvu_backward(left, right, weight, grad_output, gx, gy, gw, config, shared, needed, table,
                 workspace):
    check(load().ictc_o2_uvu_backward(
        ptr(left), ptr(right), ptr(weight), ptr(grad_output), ptr(gx), ptr(gy), ptr(gw),
        left.shape[0], *config, int(shared), int(needed), ptr(table), ptr(workspace),
        workspace.numel() if workspace is not None else 0, stream_of(left.device)),
        "uvu_backward")


# --------------------------------------------------------------------- radial
# rconfig = (channels, m_max, parity, m_max_in2, parity_in2, normalization,
#            path_normalization, hidden) as ints


def radial_workspace(rconfig, rows: int, device: torch.device) -> tuple[int, int]:
    fwd, bwd = _size(), _size()
    check(load().ictc_o2_radial_workspace(*rconfig, rows, device.index or 0, ctypes.byref(fwd),
                                          ctypes.byref(bwd)), "radial_workspace")
    return int(fwd.value), int(bwd.value)


def radial_forward(left, angular, hidden, alpha, bias, out, rconfig, table, workspace):
    check(load().ictc_o2_radial_forward(
        ptr(left), ptr(angular), ptr(hidden), ptr(alpha), ptr(bias), ptr(out), left.shape[0],
        *rconfig, ptr(table), ptr(workspace), workspace.numel(), stream_of(left.device)),
        "radial_forward")


def radial_forward_gathered(nodes, index, angular, hidden, alpha, bias, out, rconfig, table,
                            workspace):
    """Raises NotImplementedError for a configuration the edge tile does not cover."""
    check(load().ictc_o2_radial_forward_gathered(
        ptr(nodes), ptr(index), nodes.shape[0], ptr(angular), ptr(hidden), ptr(alpha), ptr(bias),
        ptr(out), index.shape[0], *rconfig, ptr(table), ptr(workspace), workspace.numel(),
        stream_of(nodes.device)), "radial_forward_gathered")


def radial_backward_gathered(nodes, index, angular, hidden, alpha, bias, grad_output, gx, gy, gh,
                             ga, gb, rconfig, needed, table, workspace):
    """gx: per-edge gradient of the gathered rows.  Raises NotImplementedError for a
    request the edge tile does not cover."""
    check(load().ictc_o2_radial_backward_gathered(
        ptr(nodes), ptr(index), nodes.shape[0], ptr(angular), ptr(hidden), ptr(alpha), ptr(bias),
        ptr(grad_output), ptr(gx), ptr(gy), ptr(gh), ptr(ga), ptr(gb), index.shape[0], *rconfig,
        int(needed), ptr(table), ptr(workspace), workspace.numel(), stream_of(nodes.device)),
        "radial_backward_gathered")


def radial_backward(left, angular, hidden, alpha, bias, grad_output, gx, gy, gh, ga, gb, rconfig,
                    needed, table, workspace):
    check(load().ictc_o2_radial_backward(
        ptr(left), ptr(angular), ptr(hidden), ptr(alpha), ptr(bias), ptr(grad_output), ptr(gx),
        ptr(gy), ptr(gh), ptr(ga), ptr(gb), left.shape[0], *rconfig, int(needed), ptr(table),
        ptr(workspace), workspace.numel(), stream_of(left.device)), "radial_backward")


# ---------------------------------------------------------------------- graph


def gather_rows(source, index, out):
    check(load().ictc_o2_gather_rows(ptr(source), ptr(index), ptr(out), index.shape[0],
                                     source.shape[1] if source.dim() > 1 else 1,
                                     source.shape[0], stream_of(out.device)), "gather_rows")


def segment_sum(values, offsets, order, out):
    check(load().ictc_o2_segment_sum(ptr(values), ptr(offsets), ptr(order), ptr(out),
                                     out.shape[0], out.shape[1] if out.dim() > 1 else 1,
                                     values.shape[0], stream_of(out.device)), "segment_sum")


def graph_bad_index() -> int:
    """Reads and clears the out-of-range-index flag of the graph kernels."""
    flag = _i32()
    check(load().ictc_o2_graph_bad_index(ctypes.byref(flag)), "graph_bad_index")
    return int(flag.value)
