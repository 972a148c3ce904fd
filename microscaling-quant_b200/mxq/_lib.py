"""The boundary between the Python API and libmxq_b200.so (the C ABI declared in include/mxq_b200.h).

Every computing function of the package ends here: tensors are made contiguous float32 (or int64 / float64 where
the reference takes those) on a CUDA device, their pointers and the current stream go to one C entry point, and a
nonzero status becomes the exception the reference raises (ValueError / IndexError) or a RuntimeError.

There is no CPU path. A CPU tensor is copied to the current CUDA device, computed there, and the result copied
back, so a caller keeps the reference's device-in, device-out contract; without a CUDA device, or without the
built library, every call raises.
"""
import ctypes
import os
import threading

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "_lib", "libmxq_b200.so")

_lib = None
_lock = threading.Lock()

P = ctypes.c_void_p
I64 = ctypes.c_int64
I32 = ctypes.c_int32
F32 = ctypes.c_float

OK, ERR_VALUE, ERR_INDEX, ERR_UNSUPPORTED, ERR_CUDA = 0, 1, 2, 3, 4


class MxqArith(ctypes.Structure):
    _fields_ = [("kind", I32), ("prod_e", I32), ("prod_m", I32), ("has_floor", I32), ("floor_thr", F32),
                ("sat_limit", F32), ("sat_value", F32)]


class MxqQuantSpec(ctypes.Structure):
    _fields_ = [("family", I32), ("e", I32), ("m", I32), ("rounding", I32), ("scale_floor", F32),
                ("placement", I32), ("scale_emax", F32), ("via_e", I32), ("via_m", I32)]


class MxqAnchorSpec(ctypes.Structure):
    _fields_ = [("width", I32), ("nbits", I32), ("drop_rne", I32), ("headroom", I32), ("has_emin", I32),
                ("emin", I32)]


# entry point -> argument types (the return type of every entry point is int32 status)
_SIGS = {
    "mxq_round_bits": [P, P, I32, P, I64, I32, P],
    "mxq_round_pattern": [P, P, I64, P, I64, P, I64, P, I64, I32, P],
    "mxq_round_int_f32": [P, P, I64, I32, P],
    "mxq_round_int_f64": [P, P, I64, I32, P],
    "mxq_bf16": [P, P, I64, P],
    "mxq_float_em_f32": [P, P, I64, I32, I32, I32, I32, P],
    "mxq_float_em_f64": [P, P, I64, I32, I32, I32, I32, P],
    "mxq_microsoft": [P, P, I64, I32, I32, F32, I32, I32, P],
    "mxq_scale_mxquant": [P, P, I64, F32, P],
    "mxq_scale_ocp": [P, P, I64, I32, F32, P],
    "mxq_scale_ocp_no_clip": [P, P, I64, I32, I32, I32, F32, P],
    "mxq_exact_add": [P, P, P, I64, I32, I32, I32, I32, P],
    "mxq_truncate_significand": [P, P, I64, I32, P],
    "mxq_flush_product": [P, P, I64, F32, P],
    "mxq_saturate": [P, P, I64, F32, F32, P],
    "mxq_arith_product": [P, P, P, I64, ctypes.POINTER(MxqArith), P],
    "mxq_arith_acc_add": [P, P, P, I64, ctypes.POINTER(MxqArith), I32, I32, P],
    "mxq_arith_tile_add": [P, P, P, I64, ctypes.POINTER(MxqArith), P],
    "mxq_block_quantize": [P, P, P, I64, I64, I64, I64, ctypes.POINTER(MxqQuantSpec), P],
    "mxq_block_quantize_packed": [P, P, P, I64, I64, I64, I64, ctypes.POINTER(MxqQuantSpec), P, P],
    "mxq_block_quantize_multi": [P, P, P, I32, I64, I64, I64, I64, ctypes.POINTER(MxqQuantSpec), P],
    "mxq_unpack": [P, P, P, P, I64, I64, I32, I32, P],
    "mxq_dequantize_packed": [P, P, P, I64, I64, I64, I64, I32, I32, P],
    "mxq_block_amax": [P, P, I64, I64, I64, I64, P],
    "mxq_to_blocks": [P, P, P, I64, I64, I64, I64, P],
    "mxq_from_blocks": [P, P, I64, I64, I64, I64, P],
    "mxq_dequantize": [P, P, P, I64, I64, I64, I64, P],
    "mxq_systolic": [P, P, P, P, P, I64, I64, I64, I64, I64, ctypes.POINTER(MxqArith), P, P, P],
    "mxq_systolic_batched": [P, P, P, P, P, I64, I64, I64, I64, I64, I64, ctypes.POINTER(MxqArith), P, P, P],
    "mxq_adder_tree": [P, P, P, P, P, I64, I64, I64, I64, I64, ctypes.POINTER(MxqArith), P, P, P],
    "mxq_anchor_tree": [P, P, P, P, P, I64, I64, I64, I64, I64, ctypes.POINTER(MxqArith), P, P,
                        ctypes.POINTER(MxqAnchorSpec), P, P],
    "mxq_fp64_accum": [P, P, P, P, P, I64, I64, I64, I64, P],
    "mxq_lut_tables": [P, P, I64, I64, I64, I64, I32, I32, I32, I32, P, P],
    "mxq_lut_pick": [P, P, P, I64, I64, I64, I64, I32, I32, P],
    "mxq_lut_pick_lookup": [P, P, P, I64, I64, I64, I64, I32, I32, P],
    "mxq_block_lut_quantize": [P, P, P, I64, I64, I32, I64, ctypes.POINTER(MxqQuantSpec), I32, I32, P, I64, P, P],
    "mxq_block_lut_quantize_static": [P, P, P, I64, I64, I32, I64, ctypes.POINTER(MxqQuantSpec), I32, I32, P, P],
    "mxq_lut_lookup": [P, P, P, I64, I64, I32, I32, P],
    "mxq_lut_encode": [P, P, I64, I32, I32, P, P],
    "mxq_lut_decode": [P, P, I64, I32, I32, P, P],
    "mxq_lut_finder": [P, P, P, I64, I64, I32, I32, I32, P, P],
    "mxq_lut_format_tables": [I32, I32, P, P, P, P],
    "mxq_device_timeouts": [P],
    "mxq_wait_status_word": [P],
    "mxq_testing_wait_timeout": [P, P, P, I64, I64, ctypes.c_uint32, P],
}


def lib():
    """The loaded library; raises if it has not been built (python microscaling-quant_b200/build.py)."""
    global _lib
    if _lib is None:
        with _lock:
            if _lib is None:
                if not os.path.exists(LIB_PATH):
                    raise RuntimeError(f"mxq_b200: {LIB_PATH} is not built; run python microscaling-quant_b200/build.py "
                                       "(there is no CPU fallback)")
                L = ctypes.CDLL(LIB_PATH)
                for name, args in _SIGS.items():
                    f = getattr(L, name)
                    f.argtypes = args
                    f.restype = I32
                L.mxq_block_lut_workspace.argtypes = [I64, I64, I32, I32]
                L.mxq_block_lut_workspace.restype = I64
                L.mxq_last_error.restype = ctypes.c_char_p
                L.mxq_version.restype = ctypes.c_char_p
                _lib = L
    return _lib


def call(name, *args):
    """Call entry point `name`; a nonzero status raises the matching exception with the library's message."""
    rc = getattr(lib(), name)(*args)
    if rc != OK:
        msg = lib().mxq_last_error().decode()
        if rc == ERR_VALUE:
            raise ValueError(msg)
        if rc == ERR_INDEX:
            raise IndexError(msg)
        if rc == ERR_UNSUPPORTED:
            raise NotImplementedError(f"mxq_b200: {msg}")
        raise RuntimeError(f"mxq_b200: {msg}")


# ------------------------------------------------------------------------------------------------ devices
def device_for(*tensors):
    """The CUDA device the computation runs on: the first CUDA tensor's, else the current one."""
    for t in tensors:
        if isinstance(t, torch.Tensor) and t.is_cuda:
            return t.device
    if not torch.cuda.is_available():
        raise RuntimeError("mxq_b200 computes on CUDA devices only and none is available (there is no CPU path)")
    return torch.device("cuda", torch.cuda.current_device())


def on(t, device, dtype=torch.float32):
    """t as a contiguous tensor of `dtype` on `device` (a copy when it is elsewhere or strided)."""
    if not isinstance(t, torch.Tensor):
        t = torch.as_tensor(t)
    if t.dtype == dtype and t.device == device and t.is_contiguous():
        return t
    return t.detach().to(device=device, dtype=dtype).contiguous()


def ptr(t):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else ctypes.c_void_p(0)


def stream(device):
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


_raw_stream = getattr(torch._C, "_cuda_getCurrentRawStream", None)


def _stream_of(index):
    """The current stream of device `index` as a cudaStream_t (torch's raw getter when it has one)."""
    if _raw_stream is not None:
        return ctypes.c_void_p(_raw_stream(index))
    return ctypes.c_void_p(torch.cuda.current_stream(index).cuda_stream)


def back(t, like_device):
    """Return a result to the caller's device (the reference's tensors stay where they were)."""
    return t if like_device is None or t.device == like_device else t.to(like_device)


def home(*tensors):
    """The device results go back to: the first tensor argument's device."""
    for t in tensors:
        if isinstance(t, torch.Tensor):
            return t.device
    return None


class using:
    """Make `device` current for a library call (kernels launch on the current device's stream)."""

    def __init__(self, device):
        self.ctx = torch.cuda.device(device)

    def __enter__(self):
        self.ctx.__enter__()
        return self

    def __exit__(self, *exc):
        return self.ctx.__exit__(*exc)


def run(name, device, *args):
    """call() with `device` current; the last argument of every entry point is the stream, appended here. Raises
    RuntimeError if a bounded wait of an earlier kernel has given up (check_waits)."""
    cur = torch.cuda.current_device()
    idx = device.index if device.index is not None else cur
    if idx == cur:                                          # the usual case: no device switch
        call(name, *args, _stream_of(idx))
    else:
        with torch.cuda.device(device):
            call(name, *args, _stream_of(idx))
    check_waits()


# ------------------------------------------------------------------------------------------ wait status
_wait_word = None


def wait_word():
    """The library's wait-status word (pinned, mapped host memory) as a ctypes uint32 view: the number of bounded
    TMA waits that gave up in kernels that have finished. Read without synchronising."""
    global _wait_word
    if _wait_word is None:
        addr = ctypes.POINTER(ctypes.c_uint32)()
        call("mxq_wait_status_word", ctypes.byref(addr))
        _wait_word = ctypes.c_uint32.from_address(ctypes.addressof(addr.contents))
    return _wait_word


def check_waits():
    """Raise RuntimeError if any TMA-staged kernel that has finished gave up waiting for its tile. Such a tile is
    written as NaN codes and scales, so every result computed since is suspect; the error repeats on every call
    until clear_waits()."""
    w = _wait_word
    if w is not None and w.value:
        raise RuntimeError(f"mxq_b200: {w.value} bounded TMA wait(s) gave up in an earlier kernel (the tiles were "
                           "written as NaN): results since then are undefined; call mxq._lib.clear_waits() once "
                           "handled")


def clear_waits():
    """Reset the wait-status word to 0 (after a timeout has been handled)."""
    wait_word().value = 0


def cached(make):
    """`make` memoised on its (hashable) arguments, for building the small spec structs of a call: the structs are
    only read by the library (const pointers), so one object can serve every call with the same arguments.
    Unhashable arguments (a Format object, a list) build a fresh struct."""
    memo = {}

    def get(*args):
        try:
            return memo[args]
        except KeyError:
            if len(memo) >= 256:                            # e.g. NaN arguments, which never compare equal
                memo.clear()
            s = memo[args] = make(*args)
            return s
        except TypeError:
            return make(*args)
    return get
