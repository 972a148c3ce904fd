"""TEST INFRASTRUCTURE — numpy front end of the CPU oracle (oracle/mxq_oracle.c, oracle/lut_oracle.c).

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg may import this module, and only as the
checker or the timed CPU baseline; the product (the mxq package) never does. Every function takes and returns
numpy arrays and mirrors the reference call it restates (chloe-wong/microscaling-quant, paths mxq/...).

The reducers run one C call per slice of output rows on a thread pool (ctypes releases the GIL), so the oracle
uses every host core it is given.
"""
import ctypes
import math
import os
import subprocess
import threading
from concurrent.futures import ThreadPoolExecutor

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "_build", "libmxq_oracle.so")
_lib = None
_lock = threading.Lock()

MODES = {"ties_away": 0, "rne": 1, "truncate": 2}
GRIDS = {"qtorch": 0, "ieee": 1, "ocp": 2}
MS_ROUND = {"nearest": 0, "floor": 1, "even": 2}
# OCP element formats (mxq/element_quant/formats.py:23-29): name -> (e, m, emax, max_norm)
FORMATS = {
    "MXFP8_E4M3": (4, 3, 8, 448.0), "MXFP8_E5M2": (5, 2, 15, 57344.0), "MXFP6_E3M2": (3, 2, 4, 28.0),
    "MXFP6_E2M3": (2, 3, 2, 7.5), "MXFP4": (2, 1, 2, 6.0),
}

P_F32 = ctypes.POINTER(ctypes.c_float)
P_F64 = ctypes.POINTER(ctypes.c_double)
P_I64 = ctypes.POINTER(ctypes.c_int64)
P_I32 = ctypes.POINTER(ctypes.c_int32)
I64 = ctypes.c_int64
I32 = ctypes.c_int


class OSpec(ctypes.Structure):
    _fields_ = [("family", ctypes.c_int32), ("e", ctypes.c_int32), ("m", ctypes.c_int32),
                ("rounding", ctypes.c_int32), ("scale_floor", ctypes.c_float), ("placement", ctypes.c_int32),
                ("scale_emax", ctypes.c_float), ("via_e", ctypes.c_int32), ("via_m", ctypes.c_int32)]


class OArith(ctypes.Structure):
    _fields_ = [("kind", ctypes.c_int32), ("prod_e", ctypes.c_int32), ("prod_m", ctypes.c_int32),
                ("has_floor", ctypes.c_int32), ("floor_thr", ctypes.c_float), ("sat_limit", ctypes.c_float),
                ("sat_value", ctypes.c_float)]


class OAnchor(ctypes.Structure):
    _fields_ = [("width", ctypes.c_int32), ("nbits", ctypes.c_int32), ("drop_rne", ctypes.c_int32),
                ("headroom", ctypes.c_int32), ("has_emin", ctypes.c_int32), ("emin", ctypes.c_int32)]


def build() -> str:
    """Compile the oracle with oracle/Makefile (gcc); returns the library path."""
    subprocess.run(["make", "-s", "-C", HERE], check=True)
    return LIB_PATH


def lib():
    global _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                build()
            _lib = ctypes.CDLL(LIB_PATH)
    return _lib


def _f32(a):
    return np.ascontiguousarray(a, dtype=np.float32)


def _p(a, t):
    return a.ctypes.data_as(t)


# ----------------------------------------------------------------------------------------- elementwise
def round_bits(bits, keep, mode):
    bits = np.ascontiguousarray(bits, dtype=np.int64)
    keep = np.ascontiguousarray(np.broadcast_to(np.asarray(keep, dtype=np.int64), bits.shape))
    out = np.empty_like(bits)
    lib().o_round_bits(_p(bits, P_I64), _p(keep, P_I64), I64(bits.size), I32(MODES[mode]), _p(out, P_I64))
    return out


def round_int(k, mode):
    if np.asarray(k).dtype == np.float64:
        k = np.ascontiguousarray(k, dtype=np.float64)
        out = np.empty_like(k)
        lib().o_round_int_f64(_p(k, P_F64), I64(k.size), I32(MODES[mode]), _p(out, P_F64))
        return out
    k = _f32(k)
    out = np.empty_like(k)
    lib().o_round_int_f32(_p(k, P_F32), I64(k.size), I32(MODES[mode]), _p(out, P_F32))
    return out


def bf16(x):
    x = _f32(x)
    out = np.empty_like(x)
    lib().o_bf16(_p(x, P_F32), I64(x.size), _p(out, P_F32))
    return out


def float_em(z, e, m, rounding_mode="ties_away", grid="qtorch"):
    if np.asarray(z).dtype == np.float64:
        z = np.ascontiguousarray(z, dtype=np.float64)
        out = np.empty(z.shape, np.float32)
        lib().o_float_em_f64(_p(z, P_F64), I64(z.size), I32(e), I32(m), I32(MODES[rounding_mode]),
                             I32(GRIDS[grid]), _p(out, P_F32))
        return out
    z = _f32(z)
    out = np.empty_like(z)
    lib().o_float_em_f32(_p(z, P_F32), I64(z.size), I32(e), I32(m), I32(MODES[rounding_mode]), I32(GRIDS[grid]),
                         _p(out, P_F32))
    return out


def microsoft(A, fmt, rounding_mode="even", saturate_normals=True):
    e, m, _, mn = FORMATS[fmt]
    return microsoft_core(A, m + 2, e, mn, rounding_mode, saturate_normals)


def microsoft_core(A, bits, exp_bits, max_norm, rounding_mode, saturate_normals):
    A = _f32(A)
    out = np.empty_like(A)
    lib().o_microsoft(_p(A, P_F32), I64(A.size), I32(bits), I32(exp_bits), ctypes.c_float(max_norm),
                      I32(MS_ROUND[rounding_mode]), I32(int(saturate_normals)), _p(out, P_F32))
    return out


def scale_mxquant(amax, floor=1e-38):
    amax = _f32(amax)
    out = np.empty_like(amax)
    lib().o_scale_mxquant(_p(amax, P_F32), I64(amax.size), ctypes.c_float(floor), _p(out, P_F32))
    return out


def _scale_emax(scale_bits):
    return float(np.float32(2 ** (scale_bits - 1) - 1))


def scale_ocp(amax, emax, scale_bits=8):
    amax = _f32(amax)
    out = np.empty_like(amax)
    lib().o_scale_ocp(_p(amax, P_F32), I64(amax.size), I32(emax), ctypes.c_float(_scale_emax(scale_bits)),
                      _p(out, P_F32))
    return out


def scale_ocp_no_clip(amax, fmt, rounding_mode="even", scale_bits=8):
    e, m, _, _ = FORMATS[fmt]
    amax = _f32(amax)
    out = np.empty_like(amax)
    lib().o_scale_ocp_no_clip(_p(amax, P_F32), I64(amax.size), I32(e), I32(m), I32(MS_ROUND[rounding_mode]),
                              ctypes.c_float(_scale_emax(scale_bits)), _p(out, P_F32))
    return out


def exact_add(a, b, e, m, rounding_mode="rne", grid="ieee"):
    a, b = np.broadcast_arrays(_f32(a), _f32(b))
    a, b = _f32(a), _f32(b)
    out = np.empty_like(a)
    lib().o_exact_add(_p(a, P_F32), _p(b, P_F32), I64(a.size), I32(e), I32(m), I32(MODES[rounding_mode]),
                      I32(GRIDS[grid]), _p(out, P_F32))
    return out


def truncate_significand(x, m):
    x = _f32(x)
    out = np.empty_like(x)
    lib().o_truncate_significand(_p(x, P_F32), I64(x.size), I32(m), _p(out, P_F32))
    return out


def flush_product(x, floor_exp):
    x = _f32(x)
    out = np.empty_like(x)
    lib().o_flush_product(_p(x, P_F32), I64(x.size), ctypes.c_float(np.float32(2.0 ** floor_exp)), _p(out, P_F32))
    return out


def saturate(x, limit, value):
    x = _f32(x)
    out = np.empty_like(x)
    lib().o_saturate(_p(x, P_F32), I64(x.size), ctypes.c_float(limit), ctypes.c_float(value), _p(out, P_F32))
    return out


# --------------------------------------------------------------------------------------- block quantizers
FAMILIES = {"fp32": 0, "mxquant": 1, "mxgemmini": 2, "ocp": 3}
PLACEMENTS = {"top": 0, "below_top": 1, "no_clip": 2}


def block_quantize(V, family, fmt, axis=0, block_size=32, rounding_mode=None, scale_floor=1e-38, via=None,
                   scale_bits=8, placement="top", threads=None):
    """block.<family>.quantize(V, fmt, axis, block_size, ...) -> (P, X), as mxq/block/_driver.py:45-66 lays them out."""
    V = _f32(V)
    axis = axis % V.ndim
    outer = int(np.prod(V.shape[:axis], dtype=np.int64))
    inner = int(np.prod(V.shape[axis + 1:], dtype=np.int64))
    L = V.shape[axis]
    nb = (L + block_size - 1) // block_size
    fam = 0 if fmt in (None, "FP32") else FAMILIES[family]
    e, m = (FORMATS[fmt][:2] if fam else (0, 0))
    if family == "ocp":
        rnd = MS_ROUND[rounding_mode or "even"]
    else:
        rnd = MODES[rounding_mode or "ties_away"]
    spec = OSpec(fam, e, m, rnd, float(np.float32(scale_floor)), PLACEMENTS[placement], _scale_emax(scale_bits),
                 via[0] if via else 0, via[1] if via else 0)
    P = np.empty_like(V)
    xshape = list(V.shape)
    xshape[axis] = nb
    X = np.empty(xshape, np.float32)
    f = lib().o_block_quantize
    if outer > 1:
        # independent [len, inner] slabs: split them over threads
        def run(a, b):
            f(_p(V[a:b] if axis > 0 else V, P_F32), I64(b - a), I64(L), I64(inner), I64(block_size),
              ctypes.byref(spec), _p(P[a:b] if axis > 0 else P, P_F32), _p(X[a:b] if axis > 0 else X, P_F32))
        if axis > 0 and V.shape[0] == outer:
            _run_rows(run, outer, threads)
            return P, X
    elif inner > 1 and V.ndim == 2 and axis == 0:
        # blocks run down the columns: split the columns over threads (strided slabs, copied per thread)
        def run(a, b):
            v = np.ascontiguousarray(V[:, a:b])
            p = np.empty_like(v)
            x = np.empty((nb, b - a), np.float32)
            f(_p(v, P_F32), I64(1), I64(L), I64(b - a), I64(block_size), ctypes.byref(spec), _p(p, P_F32), _p(x, P_F32))
            P[:, a:b] = p
            X[:, a:b] = x
        _run_rows(run, inner, threads)
        return P, X
    f(_p(V, P_F32), I64(outer), I64(L), I64(inner), I64(block_size), ctypes.byref(spec), _p(P, P_F32), _p(X, P_F32))
    return P, X


# -------------------------------------------------------------------------------------------- arithmetic
def saturation(prod_e, prod_m):
    """_saturation (mxq/matmul/_arithmetic.py:88-102): (limit, value) of spike's product saturation."""
    b = (1 << (prod_e - 1)) - 1
    fp8 = (prod_e, prod_m) == (4, 3)
    limit = 2.0 ** (b + 1 if fp8 else b) * (1 + ((2 ** prod_m - 2) if fp8 else (2 ** prod_m - 1)) / 2 ** prod_m)
    value = 2.0 ** (b + 1) * (1 + (2 ** prod_m - 2) / 2 ** prod_m)
    if value > float(np.finfo(np.float32).max):
        value = float("inf")
    return limit, value


def arith_mxgemmini(prod_e=4, prod_m=3, prod_floor=-16):
    limit, value = saturation(prod_e, prod_m)
    thr = float(np.float32(2.0 ** prod_floor)) if prod_floor is not None else 0.0
    return OArith(1, prod_e, prod_m, int(prod_floor is not None), thr, float(np.float32(limit)),
                  float(np.float32(value)))


def arith_mxquant(prod_e, prod_m):
    return OArith(0, prod_e, prod_m, 0, 0.0, 0.0, 0.0)


def _threads():
    return int(os.environ.get("MXQ_ORACLE_THREADS", os.cpu_count() or 1))


def _run_rows(fn, M, threads=None):
    threads = threads or _threads()
    n = max(1, min(threads, M))
    cuts = [M * i // n for i in range(n + 1)]
    if n == 1:
        fn(0, M)
        return
    with ThreadPoolExecutor(n) as ex:
        list(ex.map(lambda i: fn(cuts[i], cuts[i + 1]), range(n)))


def _operands(P_A, X_A, P_B, X_B):
    P_A, X_A, P_B, X_B = (_f32(t) for t in (P_A, X_A, P_B, X_B))
    K, M = P_A.shape
    N = P_B.shape[1]
    return P_A, X_A, P_B, X_B, K, M, N


def systolic(P_A, X_A, P_B, X_B, arith, schedule, size=16, block_size=32, threads=None):
    P_A, X_A, P_B, X_B, K, M, N = _operands(P_A, X_A, P_B, X_B)
    se = np.array([e for e, _ in schedule], np.int32)
    sm = np.array([m for _, m in schedule], np.int32)
    Y = np.empty((M, N), np.float32)
    f = lib().o_systolic
    _run_rows(lambda a, b: f(_p(P_A, P_F32), _p(X_A, P_F32), _p(P_B, P_F32), _p(X_B, P_F32), I64(K), I64(M), I64(N),
                             I64(block_size), I64(size), ctypes.byref(arith), _p(se, P_I32), _p(sm, P_I32),
                             _p(Y, P_F32), I64(a), I64(b)), M, threads)
    return Y


def adder_tree(P_A, X_A, P_B, X_B, arith, schedule, size=16, block_size=32, threads=None):
    P_A, X_A, P_B, X_B, K, M, N = _operands(P_A, X_A, P_B, X_B)
    le = np.array([e for e, _ in schedule], np.int32)
    lm = np.array([m for _, m in schedule], np.int32)
    Y = np.empty((M, N), np.float32)
    f = lib().o_adder_tree
    _run_rows(lambda a, b: f(_p(P_A, P_F32), _p(X_A, P_F32), _p(P_B, P_F32), _p(X_B, P_F32), I64(K), I64(M), I64(N),
                             I64(block_size), I64(size), ctypes.byref(arith), _p(le, P_I32), _p(lm, P_I32),
                             _p(Y, P_F32), I64(a), I64(b)), M, threads)
    return Y


def anchor_tree(P_A, X_A, P_B, X_B, arith, schedule=None, size=16, block_size=32, *, width=None, bits=None,
                drop="truncate", headroom=None, emin=None, threads=None):
    """anchor_tree (mxq/matmul/_anchor.py:95-138): defaults and per-tree level bits resolved as the reference does."""
    P_A, X_A, P_B, X_B, K, M, N = _operands(P_A, X_A, P_B, X_B)
    width = size if width is None else width
    trees = size // width
    schedule = [(8, 7)] * trees if schedule is None else list(schedule)
    lg = math.ceil(math.log2(width + 1))
    head = max(4, lg + 1) if headroom is None else headroom
    per_tree = [([(m + 1) + head + lg + 1] * (lg + 1) if bits is None else list(bits)) for _, m in schedule]
    tb = np.array(per_tree, np.int32).reshape(-1)
    te = np.array([e for e, _ in schedule], np.int32)
    tm = np.array([m for _, m in schedule], np.int32)
    an = OAnchor(width, lg + 1, int(drop == "rne"), head, int(emin is not None), 0 if emin is None else emin)
    Y = np.empty((M, N), np.float32)
    f = lib().o_anchor_tree
    _run_rows(lambda a, b: f(_p(P_A, P_F32), _p(X_A, P_F32), _p(P_B, P_F32), _p(X_B, P_F32), I64(K), I64(M), I64(N),
                             I64(block_size), I64(size), ctypes.byref(arith), _p(te, P_I32), _p(tm, P_I32),
                             ctypes.byref(an), _p(tb, P_I32), _p(Y, P_F32), I64(a), I64(b)), M, threads)
    return Y


def fp64_accum(P_A, X_A, P_B, X_B, block_size=32, threads=None):
    P_A, X_A, P_B, X_B, K, M, N = _operands(P_A, X_A, P_B, X_B)
    Y = np.empty((M, N), np.float32)
    f = lib().o_fp64_accum
    _run_rows(lambda a, b: f(_p(P_A, P_F32), _p(X_A, P_F32), _p(P_B, P_F32), _p(X_B, P_F32), I64(K), I64(M), I64(N),
                             I64(block_size), _p(Y, P_F32), I64(a), I64(b)), M, threads)
    return Y


# ---------------------------------------------------------------------------------------------------- LUT
LUT_FORMATS = ("MXFP6_E3M2", "MXFP6_E2M3", "MXFP8_E5M2", "MXFP8_E4M3")


def lut_format_tables(fmt):
    e, m = FORMATS[fmt][:2]
    n = 1 << (1 + e + m)
    vals = np.empty(n, np.float32)
    fx = np.empty(n, np.int64)
    safe = np.empty(512, np.float32)
    ns = lib().o_lut_format_tables(I32(e), I32(m), _p(vals, P_F32), _p(fx, P_I64), _p(safe, P_F32))
    return vals, fx, safe[:ns].copy()


def lut_tables(P, fmt, group, max_iters):
    P = _f32(P)
    K, n = P.shape
    e, m = FORMATS[fmt][:2]
    ng = (n + (1 << group) - 1) >> group
    T = np.empty((ng, 16), np.float32)
    rc = lib().o_lut_tables(_p(P, P_F32), I64(K), I64(n), I32(group), I32(max_iters), I32(e), I32(m), _p(T, P_F32))
    if rc:
        raise ValueError(f"mxq.lut: P holds a value that is not a {fmt} code; quantize it first")
    return T


def lut_pick(P, T, group):
    P, T = _f32(P), _f32(T)
    K, n = P.shape
    I = np.empty((K, n), np.int64)
    lib().o_lut_pick(_p(P, P_F32), _p(T, P_F32), I64(K), I64(n), I32(group), I64(T.shape[1]), _p(I, P_I64))
    return I


def lut_lookup(I, T, group):
    I = np.ascontiguousarray(I, dtype=np.int64)
    T = _f32(T)
    K, n = I.shape
    out = np.empty((K, n), np.float32)
    lib().o_lut_lookup(_p(I, P_I64), _p(T, P_F32), I64(K), I64(n), I32(group), I64(T.shape[1]), _p(out, P_F32))
    return out


def lut_encode(T, fmt):
    T = _f32(T)
    e, m = FORMATS[fmt][:2]
    out = np.empty(T.shape, np.int64)
    if lib().o_lut_encode(_p(T, P_F32), I64(T.size), I32(e), I32(m), _p(out, P_I64)):
        raise ValueError(f"mxq.lut: a value is not an exact {fmt} value, so it cannot be a table entry")
    return out


def lut_finder(codes, T, fmt, group):
    codes = np.ascontiguousarray(codes, dtype=np.int64)
    T = _f32(T)
    K, n = codes.shape
    e, m = FORMATS[fmt][:2]
    out = np.empty((K, n), np.int64)
    rc = lib().o_lut_finder(_p(codes, P_I64), _p(T, P_F32), I64(K), I64(n), I32(group), I32(e), I32(m), _p(out, P_I64))
    if rc == -2:
        raise IndexError("mxq.lut.finder: a code is outside the format")
    if rc:
        raise ValueError(f"mxq.lut: a table value is not an exact {fmt} value")
    return out


def lut_decode(codes, fmt):
    """decode (mxq/lut/formats.py:114-117): torch indexing, negative codes from the end."""
    codes = np.ascontiguousarray(codes, dtype=np.int64)
    e, m = FORMATS[fmt][:2]
    out = np.empty(codes.shape, np.float32)
    if lib().o_lut_decode(_p(codes, P_I64), I64(codes.size), I32(e), I32(m), _p(out, P_F32)):
        raise IndexError("mxq.lut.decode: a code is outside the format")
    return out


def lut_block_quantize(V, fmt, axis, block_size, rounding_mode, scale_floor, group, max_iters):
    """block.lut.quantize (mxq/block/lut.py:23-34)."""
    P, X = block_quantize(V, "mxgemmini", fmt, axis, block_size, rounding_mode, scale_floor)
    Pk = P if axis % 2 == 0 else np.ascontiguousarray(P.T)
    T = lut_tables(Pk, fmt, group, max_iters)
    P_lut = lut_lookup(lut_pick(Pk, T, group), T, group)
    return (P_lut if axis % 2 == 0 else np.ascontiguousarray(P_lut.T)), X
