"""TEST INFRASTRUCTURE ONLY: Python bindings of the CPU oracle (pkm_oracle.c) and of the reference's own C row
loops (reference smlm/host_rows.c, compiled into oracle/_ref by oracle/Makefile). Only tests/, the smoke check
and the benchmark's CPU-baseline leg use this module, as the checker; the product never imports it.

All functions take and return numpy arrays (C-contiguous); bf16 data is carried as uint16 bit patterns.
"""
import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_SO = os.path.join(HERE, "build", "libpkm_oracle.so")
REF_SO = os.path.join(HERE, "_ref", "libhost_rows.so")

_p, _i64, _i32, _f32 = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, ctypes.c_float
_ORC = None
_REF = None


def build():
    subprocess.run(["make", "-s", "-C", HERE], check=True)


def lib():
    global _ORC
    if _ORC is None:
        if not os.path.exists(ORACLE_SO):
            build()
        L = ctypes.CDLL(ORACLE_SO)
        L.orc_subkey_scores_f32.argtypes = [_p, _p, _i64, _i64, _i64, _i64, _p, _p]
        L.orc_select.argtypes = [_p, _p, _i32, _i64, _i64, _i64, _i64, _p, _p, _p]
        L.orc_select.restype = _i32
        L.orc_select_backward.argtypes = [_p, _p, _p, _p, _i32, _i64, _i64, _i64, _i64, _p, _p]
        L.orc_bag_forward.argtypes = [_p, _p, _p, _i32, _i64, _i64, _i64, _i64, _p]
        L.orc_bag_forward.restype = _i64
        L.orc_bag_backward.argtypes = [_p, _p, _p, _p, _i32, _p, _p, _p, _i64, _i64, _i64, _i64, _i64]
        L.orc_bag_rows_subset.argtypes = [_p, _p, _p, _i64, _i64, _i64, _i64, _i64, _p, _p]
        L.orc_bag_rows_subset.restype = _i64
        L.orc_quantize_q4.argtypes = [_p, _i64, _i64, _p, _p]
        L.orc_bag_infer.argtypes = [_p, _p, _p, _i32, _p, _p, _i32, _i64, _i64, _i64, _i64, _p, _i32]
        L.orc_lazy_adam.argtypes = [_p, _p, _p, _p, _p, _i64, _i64, _f32, _f32, _f32, _f32, _f32, _f32, _f32]
        L.orc_lazy_adam_lowmem.argtypes = [_p, _p, _p, _p, _p, _p, _p, _i64, _i64, _i32] + [_f32] * 8
        L.orc_rowwise.argtypes = [_p, _p, _p, _p, _p, _i64, _i64, _f32, _i32, _f32, _f32, _f32]
        L.orc_touched_norm.argtypes = [_p, _p, _i64, _i64]
        L.orc_touched_norm.restype = ctypes.c_double
        _ORC = L
    return _ORC


def ref_lib():
    """The reference's host_rows.c (None if it was never built here)."""
    global _REF
    if _REF is None and os.path.exists(REF_SO):
        L = ctypes.CDLL(REF_SO)
        p, i64, f32, i32 = _p, _i64, _f32, _i32
        L.host_rows_adam.argtypes = [p, p, p, p, p, p, i64, i64, f32, f32, f32, f32, f32, f32, f32, i32]
        L.host_rows_rowwise.argtypes = [p, p, p, p, p, p, p, i64, i64, f32, f32, f32, f32, i32, i32]
        L.host_rows_adam.restype = L.host_rows_rowwise.restype = None
        _REF = L
    return _REF


def _c(a, dtype):
    return np.ascontiguousarray(a, dtype=dtype)


def _ptr(a):
    return None if a is None else a.ctypes.data_as(ctypes.c_void_p)


# ------------------------------------------------------------------------------------------- bf16 helpers
def f32_to_bf16_bits(x):
    """Round-to-nearest-even fp32 -> bf16 bit patterns (uint16), as c10::BFloat16."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    nan = np.isnan(np.asarray(x, dtype=np.float32))
    return np.where(nan, np.uint16(0x7FC0), r)


def bf16_bits_to_f32(b):
    return (np.ascontiguousarray(b, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


# ---------------------------------------------------------------------------------------------- wrappers
def subkey_scores_f32(q, keys):
    """q (n, h, 2 half), keys (h, 2, nk, half) fp32 -> s1, s2 (n, h, nk) (pkm.py:117-123, fmaf chains)."""
    q, keys = _c(q, np.float32), _c(keys, np.float32)
    n, h, kd = q.shape
    nk, half = keys.shape[2], keys.shape[3]
    s1 = np.empty((n, h, nk), np.float32)
    s2 = np.empty((n, h, nk), np.float32)
    lib().orc_subkey_scores_f32(_ptr(q), _ptr(keys), n, h, nk, half, _ptr(s1), _ptr(s2))
    return s1, s2


def select(s1, s2, knn, bf16):
    """Canonical product-key selection (pkm.py:125-136, kernels.py:146-177). s1, s2: fp32 arrays, or uint16
    bf16 bits with bf16=True. Returns scores (same encoding), indices int64, weights fp32."""
    dt = np.uint16 if bf16 else np.float32
    s1, s2 = _c(s1, dt), _c(s2, dt)
    n, h, nk = s1.shape
    sc = np.empty((n, h, knn), dt)
    idx = np.empty((n, h, knn), np.int64)
    w = np.empty((n, h, knn), np.float32)
    rc = lib().orc_select(_ptr(s1), _ptr(s2), int(bf16), n, h, nk, knn, _ptr(sc), _ptr(idx), _ptr(w))
    if rc:
        raise ValueError(f"orc_select failed ({rc})")
    return sc, idx, w


def select_backward(idx, w, gw, gs, nk, bf16):
    idx, w = _c(idx, np.int64), _c(w, np.float32)
    n, h, knn = idx.shape
    gw = None if gw is None else _c(gw, np.float32)
    gs = None if gs is None else _c(gs, np.uint16 if bf16 else np.float32)
    dt = np.uint16 if bf16 else np.float32
    ds1 = np.empty((n, h, nk), dt)
    ds2 = np.empty((n, h, nk), dt)
    lib().orc_select_backward(_ptr(idx), _ptr(w), _ptr(gw), _ptr(gs), int(bf16), n, h, nk, knn, _ptr(ds1), _ptr(ds2))
    return ds1, ds2


def bag_forward(idx, w, table, bf16=False):
    """out (n, d) fp32 = sum_j w * table[idx] (fmaf over j). table: fp32, or uint16 bf16 bits with bf16=True."""
    idx, w = _c(idx, np.int64), _c(w, np.float32)
    table = _c(table, np.uint16 if bf16 else np.float32)
    n, k = idx.shape
    rows, d = table.shape
    out = np.empty((n, d), np.float32)
    bad = lib().orc_bag_forward(_ptr(idx), _ptr(w), _ptr(table), int(bf16), n, k, rows, d, _ptr(out))
    return out, int(bad)


def bag_backward(g, idx, w, table, acc, touched, bf16=False, chunk=0):
    """In place on acc (fp32) / touched (uint8); returns gw (n, k). chunk > 0 reproduces a chunked summation
    schedule (see pkm_oracle.c)."""
    g, idx, w = _c(g, np.float32), _c(idx, np.int64), _c(w, np.float32)
    table = _c(table, np.uint16 if bf16 else np.float32)
    n, k = idx.shape
    rows, d = table.shape
    gw = np.empty((n, k), np.float32)
    assert acc is None or (acc.dtype == np.float32 and acc.flags.c_contiguous)
    assert touched is None or (touched.dtype == np.uint8 and touched.flags.c_contiguous)
    lib().orc_bag_backward(_ptr(g), _ptr(idx), _ptr(w), _ptr(table), int(bf16), _ptr(acc), _ptr(touched), _ptr(gw),
                           n, k, rows, d, chunk)
    return gw


def bag_rows_subset(g, idx, w, rows, sample, chunk=0):
    """The row sums bag_backward would add into a zeroed acc, for the rows in `sample` only (int64 array of
    distinct rows), in that order: (len(sample), d) fp32. Same sorted order and chunk pieces as bag_backward over
    all lookups; needs no table (for steps whose table does not fit host memory)."""
    g, idx, w = _c(g, np.float32), _c(idx, np.int64), _c(w, np.float32)
    n, k = idx.shape
    d = g.shape[1]
    sample = _c(sample, np.int64)
    slot = np.full(rows, -1, np.int32)
    slot[sample] = np.arange(sample.size, dtype=np.int32)
    out = np.zeros((sample.size, d), np.float32)
    lib().orc_bag_rows_subset(_ptr(g), _ptr(idx), _ptr(w), n, k, rows, d, chunk, _ptr(slot), _ptr(out))
    return out


def quantize_q4(table):
    table = _c(table, np.float32)
    rows, d = table.shape
    packed = np.empty((rows, d // 2), np.uint8)
    scales = np.empty(rows, np.uint16)
    lib().orc_quantize_q4(_ptr(table), rows, d, _ptr(packed), _ptr(scales))
    return packed, scales


def bag_infer(idx, w, table, table_type, scales=None, pre=None, pre_bf16=True, out_bf16=False):
    """table_type: 'f32', 'bf16' (uint16 bits) or 'q4' (packed uint8 + fp16-bit scales)."""
    idx, w = _c(idx, np.int64), _c(w, np.float32)
    tt = {"f32": 0, "bf16": 1, "q4": 3}[table_type]
    table = _c(table, {0: np.float32, 1: np.uint16, 3: np.uint8}[tt])
    n, k = idx.shape
    rows = table.shape[0]
    d = table.shape[1] * (2 if tt == 3 else 1)
    if pre is not None:
        pre = _c(pre, np.uint16 if pre_bf16 else np.float32)
    sc = None if scales is None else _c(scales, np.uint16)
    out = np.empty((n, d), np.float32)
    lib().orc_bag_infer(_ptr(idx), _ptr(w), _ptr(table), tt, _ptr(sc), _ptr(pre), int(pre_bf16), n, k, rows, d,
                        _ptr(out), int(out_bf16))
    return out


def adam_scalars(step, lr, beta1, beta2):
    """The float scalars of one lazy Adam step, computed in double as the reference does
    (host_optim.py:138-157)."""
    import math
    return dict(one_minus_b1=1 - beta1, b2=beta2, one_minus_b2=1 - beta2,
                bc2_sqrt=math.sqrt(1 - beta2 ** step), neg_step_size=-(lr / (1 - beta1 ** step)))


def lazy_adam(p, m, v, acc, touched, grad_scale, step, lr, beta1, beta2, eps):
    """In place (all fp32 arrays, touched uint8)."""
    s = adam_scalars(step, lr, beta1, beta2)
    rows, d = p.shape
    lib().orc_lazy_adam(_ptr(p), _ptr(m), _ptr(v), _ptr(acc), _ptr(touched), rows, d, grad_scale,
                        s["one_minus_b1"], s["b2"], s["one_minus_b2"], s["bc2_sqrt"], eps, s["neg_step_size"])


def lazy_adam_lowmem(p, m, v, m_scale, v_scale, acc, touched, grad_scale, step, lr, beta1, beta2, eps, int8):
    """In place. bf16: m, v uint16 bit arrays; int8: m int8, v uint8 codes with fp32 row scales."""
    import math
    rows, d = p.shape
    lib().orc_lazy_adam_lowmem(_ptr(p), _ptr(m), _ptr(v), _ptr(m_scale) if int8 else None,
                               _ptr(v_scale) if int8 else None, _ptr(acc), _ptr(touched), rows, d, int(int8),
                               grad_scale, beta1, beta2, 1 - beta1, 1 - beta2, eps, lr / (1 - beta1 ** step),
                               math.sqrt(1 - beta2 ** step))


def ref_lazy_adam(p, m, v, acc, touched, grad_scale, step, lr, beta1, beta2, eps, threads=1):
    """The reference's own host_rows_adam on the touched rows (host_optim.py:138-157)."""
    L = ref_lib()
    rows_list = np.ascontiguousarray(np.nonzero(touched)[0].astype(np.int64))
    s = adam_scalars(step, lr, beta1, beta2)
    L.host_rows_adam(_ptr(p), _ptr(acc), _ptr(m), _ptr(v), _ptr(touched), _ptr(rows_list), rows_list.size,
                     p.shape[1], grad_scale, s["one_minus_b1"], s["b2"], s["one_minus_b2"], s["bc2_sqrt"], eps,
                     s["neg_step_size"], threads)


def rowwise(p, acc, touched, v, count, grad_scale, kind, b2, eps, lr):
    rows, d = p.shape
    lib().orc_rowwise(_ptr(p), _ptr(acc), _ptr(touched), _ptr(v), _ptr(count), rows, d, grad_scale,
                      {"rowrms": 0, "rowadagrad": 1}[kind], b2, eps, lr)


def ref_rowwise(p, acc, touched, v, count, grad_scale, kind, b2, eps, lr, threads=1):
    L = ref_lib()
    rows_list = np.ascontiguousarray(np.nonzero(touched)[0].astype(np.int64))
    L.host_rows_rowwise(_ptr(p), _ptr(acc), None, _ptr(v), _ptr(count), _ptr(touched), _ptr(rows_list),
                        rows_list.size, p.shape[1], grad_scale, b2, eps, lr, {"rowrms": 0, "rowadagrad": 1}[kind],
                        threads)


def touched_norm(acc, touched):
    rows, d = acc.shape
    return lib().orc_touched_norm(_ptr(_c(acc, np.float32)), _ptr(_c(touched, np.uint8)), rows, d)


def ngram_rows(c, history, mult, orders, heads, rows):
    """Engram n-gram rows, restated in numpy int64 arithmetic from the reference's NgramHash.forward
    (smlm/engram.py:63-75): per order o, the XOR over i < n of c[:, history + t - i] * mult[o, h, i], then
    x ^= x >> 17 and row = x mod rows (floored) + (o * heads + h) * rows. c (B, history + T) int64 ->
    (B, T, len(orders) * heads) int64."""
    c = np.asarray(c, dtype=np.int64)
    mult = np.asarray(mult, dtype=np.int64)
    T = c.shape[1] - history
    out = []
    for o, n in enumerate(orders):
        x = np.zeros((c.shape[0], T, heads), dtype=np.int64)
        for i in range(n):
            x ^= c[:, history - i:history - i + T, None] * mult[o, :, i][None, None, :]
        x ^= x >> 17
        out.append(np.mod(x, rows) + (o * heads + np.arange(heads, dtype=np.int64)) * rows)
    return np.concatenate(out, -1)
