"""TEST INFRASTRUCTURE ONLY — NOT PART OF THE PRODUCT.

numpy/ctypes front end of the CPU oracle (``qmoe_oracle.c``): the restatement of the reference
engine's NVFP4 routed-expert and FP8/NVFP4 dense arithmetic (helgard-orlm/nemotron-super-8gb
``qmoe_ns.py``, ``dense_q.py``, ``nem_super.py``). Only ``tests/``, ``__graft_entry__.smoke()`` and
``bench.py``'s CPU-baseline leg import this module, and only as the checker or the timed CPU
baseline. The product package never imports it.

Pinned against golden vectors produced by the reference's own Python functions
(``tests/golden/make_golden.py``), checked by ``tests/test_oracle_golden.py``.
"""
import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "_lib", "libqmoe_oracle.so")

LAT, INTER = 1024, 2688
BLOCK = 3096576
O_UW, O_US, O_DW, O_DS = 0, 1376256, 1548288, 2924544
UPB = O_DW
G_DN = 168

_lib = None
_u8p = ctypes.POINTER(ctypes.c_uint8)
_f32p = ctypes.POINTER(ctypes.c_float)
_f64p = ctypes.POINTER(ctypes.c_double)
_i32p = ctypes.POINTER(ctypes.c_int32)
_u16p = ctypes.POINTER(ctypes.c_uint16)


def build():
    """Compile qmoe_oracle.c into _lib/ (make; gcc + OpenMP)."""
    subprocess.run(["make", "-s", "-C", HERE], check=True)


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build()
        L = ctypes.CDLL(LIB_PATH)
        L.orc_e4m3.restype = ctypes.c_float
        L.orc_e4m3.argtypes = [ctypes.c_uint8]
        L.orc_e2m1_table.argtypes = [_f32p]
        L.orc_deq.argtypes = [_u8p, _u8p, ctypes.c_float, ctypes.c_int64, ctypes.c_int64, ctypes.c_int, _f32p]
        L.orc_to_T.argtypes = [_u8p, _u8p]
        L.orc_from_T.argtypes = [_u8p, _u8p]
        L.orc_moe_decode.argtypes = [ctypes.POINTER(_u8p), ctypes.c_int, ctypes.c_int, _f32p, _f32p, _f32p,
                                     _f64p, _f64p, _f64p]
        L.orc_live_groups.argtypes = [_f32p, ctypes.c_int, _i32p, _i32p]
        L.orc_pairs.argtypes = [ctypes.POINTER(_u8p), ctypes.c_int, ctypes.c_int, _i32p, _i32p, _f32p, _f32p,
                                _f32p, _f64p]
        L.orc_dense.argtypes = [ctypes.c_int, _u8p, _u8p, ctypes.c_float, ctypes.c_int64, ctypes.c_int64, _f32p,
                                ctypes.c_int, _f64p]
        L.orc_dequant_rows_bf16.argtypes = [ctypes.c_int, _u8p, _u8p, ctypes.c_float, ctypes.c_int64,
                                            ctypes.c_int64, ctypes.c_int64, _u16p]
        L.orc_cpu_layer_fp32.argtypes = [ctypes.POINTER(_u8p), ctypes.c_int, ctypes.c_int, _f32p, _f32p, _f32p,
                                         ctypes.c_int, _f32p]
        L.orc_max_threads.restype = ctypes.c_int
        _lib = L
    return _lib


def _p(a, t):
    return a.ctypes.data_as(t)


def _c(a, dt):
    return np.ascontiguousarray(a, dtype=dt)


def bf16_bits_to_f32(bits):
    """uint16 bf16 bit patterns -> float32 (exact)."""
    return (np.asarray(bits, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16_bits(x):
    """float32 -> bf16 bits, round to nearest even (as torch's .to(torch.bfloat16))."""
    u = np.asarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    r = 0x7FFF + ((u >> 16) & 1)
    out = ((u + r) >> 16).astype(np.uint16)
    nan = (u & 0x7FFFFFFF) > 0x7F800000
    out[nan] = ((u[nan] >> 16) | 0x40).astype(np.uint16)
    return out


def e2m1_table():
    """qmoe_ns.py:391 (the table held by qmoe_oracle.c)."""
    out = np.empty(16, dtype=np.float32)
    lib().orc_e2m1_table(_p(out, _f32p))
    return out


def e4m3_table():
    """torch.float8_e4m3fn -> float32 for all 256 bytes."""
    L = lib()
    return np.array([L.orc_e4m3(i) for i in range(256)], dtype=np.float32)


def deq(w_u8, s_u8, ws2, swap=False):
    """qmoe_ns.py:395-404: w [N, K/2] u8, s [N, K/16] e4m3 bytes -> fp32 [N, K]."""
    w = _c(w_u8, np.uint8)
    s = _c(s_u8, np.uint8)
    N, K = w.shape[0], w.shape[1] * 2
    out = np.empty((N, K), dtype=np.float32)
    lib().orc_deq(_p(w, _u8p), _p(s, _u8p), float(ws2), N, K, int(swap), _p(out, _f32p))
    return out


def block_deq(blk, s2):
    """qmoe_ns.py:407-412: orig-layout block -> up [2688,1024], down [1024,2688] fp32."""
    b = _c(blk, np.uint8)
    u = deq(b[O_UW:O_US].reshape(INTER, LAT // 2), b[O_US:O_DW].reshape(INTER, LAT // 16), s2[0])
    d = deq(b[O_DW:O_DS].reshape(LAT, INTER // 2), b[O_DS:BLOCK].reshape(LAT, INTER // 16), s2[1])
    return u, d


def to_T(blk):
    """qmoe_ns.py:356-364."""
    b = _c(blk, np.uint8)
    out = np.empty(BLOCK, dtype=np.uint8)
    lib().orc_to_T(_p(b, _u8p), _p(out, _u8p))
    return out


def from_T(blk):
    """qmoe_ns.py:367-375."""
    b = _c(blk, np.uint8)
    out = np.empty(BLOCK, dtype=np.uint8)
    lib().orc_from_T(_p(b, _u8p), _p(out, _u8p))
    return out


def _blk_ptrs(blocks):
    arrs = [_c(b, np.uint8) for b in blocks]
    ptrs = (_u8p * len(arrs))(*[_p(a, _u8p) for a in arrs])
    return arrs, ptrs


def moe_decode(blocks, s2, coef, x, layoutT=False):
    """qmoe_ns.py:70-76 in fp64 (tests/kern_test.py:35-39): returns (y [1024], h [K,2688], yj [K,1024])."""
    K = len(blocks)
    keep, ptrs = _blk_ptrs(blocks)
    s2 = _c(s2, np.float32)
    coef = _c(coef, np.float32)
    x = _c(x, np.float32)
    h = np.empty((K, INTER), dtype=np.float64)
    yj = np.empty((K, LAT), dtype=np.float64)
    y = np.empty(LAT, dtype=np.float64)
    lib().orc_moe_decode(ptrs, int(layoutT), K, _p(s2, _f32p), _p(coef, _f32p), _p(x, _f32p), _p(h, _f64p),
                         _p(yj, _f64p), _p(y, _f64p))
    del keep
    return y, h, yj


def live_groups(h):
    """qmoe_ns.py:249-251: h [K,2688] -> gidx [K,168] int32, gcnt [K] int32."""
    h = _c(h, np.float32)
    K = h.shape[0]
    gidx = np.empty((K, G_DN), dtype=np.int32)
    gcnt = np.empty(K, dtype=np.int32)
    lib().orc_live_groups(_p(h, _f32p), K, _p(gidx, _i32p), _p(gcnt, _i32p))
    return gidx, gcnt


def pairs(blocks, pslot, ptok, s2p, coefp, X, layoutT=False):
    """qmoe_ns.py:127-133 in fp64: out [P, 1024]."""
    keep, ptrs = _blk_ptrs(blocks)
    pslot = _c(pslot, np.int32)
    ptok = _c(ptok, np.int32)
    s2p = _c(s2p, np.float32)
    coefp = _c(coefp, np.float32)
    X = _c(X, np.float32)
    P = pslot.shape[0]
    out = np.empty((P, LAT), dtype=np.float64)
    lib().orc_pairs(ptrs, int(layoutT), P, _p(pslot, _i32p), _p(ptok, _i32p), _p(s2p, _f32p), _p(coefp, _f32p),
                    _p(X, _f32p), _p(out, _f64p))
    del keep
    return out


def dense(fmt, w, sc, s, N, K, x):
    """dense_q.py:179-188 dequant + fp64 matvec: x [M,K] -> y [M,N]. fmt 'fp8' or 'nvfp4'."""
    w = _c(w, np.uint8)
    sc = _c(sc if sc is not None else np.zeros(1, np.uint8), np.uint8)
    x = _c(np.atleast_2d(x), np.float32)
    M = x.shape[0]
    y = np.empty((M, N), dtype=np.float64)
    lib().orc_dense(0 if fmt == "fp8" else 1, _p(w, _u8p), _p(sc, _u8p), float(s), N, K, _p(x, _f32p), M,
                    _p(y, _f64p))
    return y


def dequant_rows_bf16(fmt, w, sc, s, K, r0, r1):
    """dense_q.py:179-188 exactly (bf16 output bits [r1-r0, K])."""
    w = _c(w, np.uint8)
    sc = _c(sc if sc is not None else np.zeros(1, np.uint8), np.uint8)
    out = np.empty((r1 - r0, K), dtype=np.uint16)
    lib().orc_dequant_rows_bf16(0 if fmt == "fp8" else 1, _p(w, _u8p), _p(sc, _u8p), float(s), K, r0, r1,
                                _p(out, _u16p))
    return out


def cpu_layer_fp32(blocks, s2, coef, x, layoutT=False, nthreads=0):
    """The reference's fp32 CPU expert path (nem_super.py:342-346) for one decode token -> y [1024] fp32."""
    K = len(blocks)
    keep, ptrs = _blk_ptrs(blocks)
    s2 = _c(s2, np.float32)
    coef = _c(coef, np.float32)
    x = _c(x, np.float32)
    y = np.empty(LAT, dtype=np.float32)
    lib().orc_cpu_layer_fp32(ptrs, int(layoutT), K, _p(s2, _f32p), _p(coef, _f32p), _p(x, _f32p), int(nthreads),
                             _p(y, _f32p))
    del keep
    return y


def max_threads():
    return int(lib().orc_max_threads())


def prefill(blocks, s2, ids, w, X, layoutT=False):
    """Prompt-path layer in fp64: out[t] = sum over k (in k order) of w[t,k] * s2[e,1] * D_e relu(s2[e,0] U_e x_t)^2,
    e = ids[t,k]; ids of -1 are skipped (nem_super.py:336-348 with the pairs arithmetic of qmoe_ns.py:79-133)."""
    ids = np.asarray(ids)
    T, k = ids.shape
    valid = ids >= 0
    t_i, k_i = np.nonzero(valid)
    out = np.zeros((T, LAT), dtype=np.float64)
    if len(t_i) == 0:
        return out
    pslot = ids[t_i, k_i].astype(np.int32)
    y = pairs(blocks, pslot, t_i.astype(np.int32), np.asarray(s2, np.float32)[pslot],
              np.asarray(w, np.float32)[t_i, k_i], X, layoutT=layoutT)
    Yd = np.zeros((T, k, LAT), dtype=np.float64)
    Yd[t_i, k_i] = y
    for kk in range(k):          # fixed k order
        out += Yd[:, kk]
    return out


def ep_pack(x, ids, w, n_experts, world):
    """Expert-parallel dispatch pack (no reference counterpart): expert e on rank e // (n_experts // world);
    block d holds, in token order, the tokens with >= 1 expert on d: their x rows, block-local ids (-1 for
    experts elsewhere and for unused rows) and weights. Returns send_x [world, T, ...], ids [world, T, k],
    w [world, T, k], row_of [world, T] (-1: not in block d), cnt [world]."""
    ids = np.asarray(ids)
    T, k = ids.shape
    el = n_experts // world
    send_x = np.zeros((world,) + tuple(np.shape(x)), dtype=np.asarray(x).dtype)
    s_ids = np.full((world, T, k), -1, dtype=np.int32)
    s_w = np.zeros((world, T, k), dtype=np.float32)
    row_of = np.full((world, T), -1, dtype=np.int32)
    cnt = np.zeros(world, dtype=np.int32)
    for d in range(world):
        r = 0
        for t in range(T):
            loc = (ids[t] >= 0) & (ids[t] // el == d)
            if loc.any():
                send_x[d, r] = x[t]
                s_ids[d, r] = np.where(loc, ids[t] - d * el, -1)
                s_w[d, r] = w[t]
                row_of[d, t] = r
                r += 1
        cnt[d] = r
    return send_x, s_ids, s_w, row_of, cnt


def ep_combine(part, row_of):
    """out[t] = sum over ranks d in order of part[d, row_of[d, t]] (row_of -1 skipped)."""
    world, T = row_of.shape
    out = np.zeros((T,) + part.shape[2:], dtype=np.float64)
    for d in range(world):
        for t in range(T):
            if row_of[d, t] >= 0:
                out[t] += part[d, row_of[d, t]]
    return out
