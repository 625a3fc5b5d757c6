"""ctypes wrapper of liboracle.so, the CPU restatement of the reference's v2.4 neon-int8 and neon-fp16 paths and
the fp16 bodies of compiled models (TEST INFRASTRUCTURE).

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline legs use this module; the product library never
does. `make -C oracle` builds liboracle.so.
"""
import ctypes
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "liboracle.so")
_P, _I, _F, _L, _SZ, _S = ctypes.c_void_p, ctypes.c_int, ctypes.c_float, ctypes.c_long, ctypes.c_size_t, ctypes.c_char_p
_H = ctypes.c_uint16
SIGS = {
    "bnno_silu": (_F, [_F]), "bnno_sigmoid": (_F, [_F]), "bnno_frecpe": (_F, [_F]), "bnno_log2_acc": (_F, [_F]),
    "bnno_exp2_acc": (_F, [_F]), "bnno_expf": (_F, [_F]),
    "bnno_quant_rows": (None, [_P, _I, _I, _I, _I, _P, _P, _P, _P]),
    "bnno_s8_gemm": (None, [_P, _P, _P, _I, _I, _I, _I, _P, _P, _P, _P, _I, _P, _I, _I, _I, _P, _I, _I, _I]),
    "bnno_pw_s8": (None, [_P, _I, _I, _I, _I, _I, _I, _P, _P, _P, _P, _P, _I, _P, _I, _I, _I, _I, _P, _I, _I, _I,
                          _P, _P, _P]),
    "bnno_dw3": (None, [_P, _I, _I, _I, _I, _P, _P, _P, _I, _I, _P]),
    "bnno_se_gate": (None, [_I, _I, _P, _P, _P, _P, _P, _I, _P]),
    "bnno_c0pool": (None, [_P, _P, _P, _P]),
    "bnno_postpc": (None, [_P, _P, _P, _P, _P, _P]),
    "bnno_logmel_new": (_P, [_I, _I, _I, _I, _I, _I, _P, _P, _F, _F]),
    "bnno_logmel_frames": (_I, [_P]), "bnno_logmel_run": (None, [_P, _P, _P]), "bnno_logmel_free": (None, [_P]),
    "bnno_proto_quant_cells": (None, [_P, _I, _I, _I, _F, _P, _I, _P]),
    "bnno_proto_unpack": (None, [_P, _I, _I, _P]),
    "bnno_proto_quant_cells_f16": (None, [_P, _I, _I, _I, _F, _P, _P]),
    "bnno_proto_unpack12": (None, [_P, _I, _I, _P]),
    "bnno_proto_colmax": (None, [_P, _I, _P, _I, _P, _P, _I, _P]),
    "bnno_proto_colmax_rows": (None, [_P, _I, _P, _I, _P, _P, _I, _P]),
    "bnno_proto_logits": (_I, [_P, _P, _P, _I, _I, _P]),
    "bnno_proto_n4_check": (_I, [_P, _I, _P, _I]),
    "bnno_proto_s8_many": (_I, [_I, _I, _P, ctypes.c_longlong, _I, _I, _I, _F, _P, _P, _I, _I, _P, _P, _I, _I, _P]),
    "bnno_pkg_open": (_P, [_S, _S, _S, _SZ]), "bnno_pkg_close": (None, [_P]),
    "bnno_pkg_n_ops": (_I, [_P]), "bnno_pkg_n_bufs": (_I, [_P]), "bnno_pkg_op_code": (_I, [_P, _I]),
    "bnno_pkg_buf_elems": (_L, [_P, _I, _P]), "bnno_pkg_out_elems": (_I, [_P]), "bnno_pkg_emb_elems": (_I, [_P]),
    "bnno_pkg_run_range": (_I, [_P, _P, _I, _I]), "bnno_pkg_run": (_I, [_P, _P, _P, _P]),
    "bnno_pkg_get_buf": (_I, [_P, _I, _P, _SZ]), "bnno_pkg_set_buf": (_I, [_P, _I, _P, _SZ]),
    "bnno_pkg_run_many": (_I, [_S, _S, _I, _P, _P, _P, _I]),
    "bnno_h_fma": (_H, [_H, _H, _H]), "bnno_h_add": (_H, [_H, _H]), "bnno_h_mul": (_H, [_H, _H]),
    "bnno_h_silu": (_H, [_H]), "bnno_d2h": (_H, [ctypes.c_double]), "bnno_h2d": (ctypes.c_double, [_H]),
    "bnno_sigm_f16path": (_F, [_F]),
    "bnno_gemm_f16": (None, [_P, _I, _I, _P, _P, _P, _I, _I, _I, _P, _I, _I, _I, _P, _I]),
    "bnno_c0pool_f16": (None, [_P, _P, _P, _P]),
    "bnno_dw3_f16": (None, [_P, _I, _I, _I, _I, _I, _I, _P, _P, _P, _I, _I, _P]),
    "bnno_se_f16": (None, [_I, _I, _P, _P, _P, _P, _P, _I, _P]),
    "bnno_stem_f16": (None, [_P, _I, _I, _I, _I, _I, _I, _P, _P, _I, _I, _I, _P, _I, _I]),
    "bnno_dwk_f16": (None, [_P, _I, _I, _I, _I, _I, _I, _I, _P, _P, _I, _P, _I, _I, _P]),
    "bnno_pad_f16": (None, [_P, _I, _I, _I, _I, _I, _P]),
    "bnno_mean_f16": (None, [_P, _I, _I, _I, _P]),
    "bnno_postpc_f16": (_I, [_P, _P, _P, _P, _P, _P, _P]),
    "bnno_dense_f16": (None, [_P, _P, _I, _P, _P]), "bnno_dense_f32": (None, [_P, _P, _I, _P, _P]),
    "bnno_dbimg_new": (_P, [_P, _P, _P, _P, _P]), "bnno_dbimg_free": (None, [_P]),
    "bnno_dbimg_frames_count": (_I, [_P]), "bnno_dbimg_frames": (None, [_P, _P, _P, _I]),
    "bnno_dbimg_image": (None, [_P, _P, _P]), "bnno_dbimg_run": (None, [_P, _P, _P, _I]),
    "bnno_logf_cr": (_F, [_F]), "bnno_log_n": (None, [_P, _P, _L, _I]), "bnno_pkg_set_log_mode": (None, [_I]),
}
DTYPES = {0: np.float32, 1: np.float16, 2: np.int8, 3: np.int32}
_LIB = None


def lib():
    global _LIB  # pylint: disable=global-statement
    if _LIB is None:
        if not os.path.exists(LIB_PATH):
            raise OSError(f"{LIB_PATH} missing: run `make -C oracle`")
        h = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGS.items():
            getattr(h, name).restype = res
            getattr(h, name).argtypes = args
        _LIB = h
    return _LIB


def ptr(a):
    return None if a is None else a.ctypes.data


def fn(name, x):
    """An elementwise oracle function over an array."""
    f = getattr(lib(), name)
    x = np.asarray(x, np.float32).reshape(-1)
    return np.array([f(float(v)) for v in x], np.float32)


def logmel(pcm, frame, hop, pad, nfft, window, mel, floor, scale):
    """FE_LOGMEL on windows pcm [n][nsamp]: spec [n][nfr][nmel] (None if the geometry is refused)."""
    pcm = np.ascontiguousarray(pcm, np.float32)
    window = np.ascontiguousarray(window, np.float32)
    mel = np.ascontiguousarray(mel, np.float32)
    h = lib()
    f = h.bnno_logmel_new(pcm.shape[1], frame, hop, pad, nfft, mel.shape[0], ptr(window), ptr(mel), float(floor),
                          float(scale))
    if not f:
        return None
    try:
        nfr = h.bnno_logmel_frames(f)
        out = np.zeros((pcm.shape[0], max(nfr, 0), mel.shape[0]), np.float32)
        for w in range(pcm.shape[0]):
            h.bnno_logmel_run(f, ptr(pcm[w]), ptr(out[w]))
        return out
    finally:
        h.bnno_logmel_free(f)


def proto_unpack(qp):
    """The package's prototype panels [Np/4][Kp/16][4][16] as rows [Np][Kp]."""
    qp = np.ascontiguousarray(qp, np.int8)
    n_pad, k_pad = qp.shape[0] * 4, qp.shape[1] * 16
    rows = np.empty((n_pad, k_pad), np.int8)
    lib().bnno_proto_unpack(ptr(qp), n_pad, k_pad, ptr(rows))
    return rows


def proto_s8(x, rows, sw, cls_w, cls_b, eps, C, Kp):
    """PROTO_S8 on windows x [B][P][ld] with prototype rows [Np][Kp]: (qa [B][P][Kp], sx [B][P], colmax [B][Np],
    logits [B][nc], status [B]: 0 or -2), window by window."""
    x = np.ascontiguousarray(x, np.float32)
    B, P, ld = x.shape
    rows = np.ascontiguousarray(rows, np.int8)
    Np = rows.shape[0]
    sw = np.ascontiguousarray(sw, np.float32)
    cls_w = np.ascontiguousarray(cls_w, np.float32).reshape(-1)
    cls_b = np.ascontiguousarray(cls_b, np.float32)
    nc = cls_b.shape[0]
    ppc = cls_w.shape[0] // nc
    qa = np.zeros((B, P, Kp), np.int8)
    sx = np.zeros((B, P), np.float32)
    cm = np.zeros((B, Np), np.float32)
    lg = np.zeros((B, nc), np.float32)
    st = np.zeros(B, np.int32)
    h = lib()
    for w in range(B):
        h.bnno_proto_quant_cells(ptr(x[w]), P, C, ld, float(eps), ptr(qa[w]), Kp, ptr(sx[w]))
        h.bnno_proto_colmax_rows(ptr(qa[w]), Kp, ptr(sx[w]), P, ptr(rows), ptr(sw), Np, ptr(cm[w]))
        st[w] = h.bnno_proto_logits(ptr(cm[w]), ptr(cls_w), ptr(cls_b), nc, ppc, ptr(lg[w]))
    return qa, sx, cm, lg, st


def proto_s8h(x16, rows, sw, cls_w, cls_b, eps, C):
    """PROTO variant 2 on fp16 windows x16 [B][P][ld] (numpy float16) with prototype rows [Np][K]: (qa [B][P][K],
    sx [B][P], colmax [B][Np], logits [B][nc], status [B])."""
    x16 = np.ascontiguousarray(x16, np.float16)
    B, P, ld = x16.shape
    rows = np.ascontiguousarray(rows, np.int8)
    Np, K = rows.shape
    sw = np.ascontiguousarray(sw, np.float32)
    cls_w = np.ascontiguousarray(cls_w, np.float32).reshape(-1)
    cls_b = np.ascontiguousarray(cls_b, np.float32)
    nc = cls_b.shape[0]
    ppc = cls_w.shape[0] // nc
    qa = np.zeros((B, P, K), np.int8)
    sx = np.zeros((B, P), np.float32)
    cm = np.zeros((B, Np), np.float32)
    lg = np.zeros((B, nc), np.float32)
    st = np.zeros(B, np.int32)
    h = lib()
    for w in range(B):
        h.bnno_proto_quant_cells_f16(ptr(x16[w]), P, C, ld, float(eps), ptr(qa[w]), ptr(sx[w]))
        h.bnno_proto_colmax_rows(ptr(qa[w]), K, ptr(sx[w]), P, ptr(rows), ptr(sw), Np, ptr(cm[w]))
        st[w] = h.bnno_proto_logits(ptr(cm[w]), ptr(cls_w), ptr(cls_b), nc, ppc, ptr(lg[w]))
    return qa, sx, cm, lg, st


def h_op(name, *xs):
    """An elementwise fp16 oracle operation over uint16 (IEEE half bit) arrays of one shape."""
    f = getattr(lib(), name)
    xs = [np.asarray(x, np.uint16).reshape(-1) for x in xs]
    return np.array([f(*(int(x[i]) for x in xs)) for i in range(xs[0].size)], np.uint16)


def silu_table():
    """The oracle's fp16 SiLU coefficient table: {"c0": [16], "c1": [16], "c2": [16]} as 16-bit values."""
    return {k: list((_H * 16).in_dll(lib(), f"BNNO_SILU_{k.upper()}")) for k in ("c0", "c1", "c2")}


def gemm_f16(A, w, b32, b16, Kp, Np, act, M, ldo=None, ow=0, opad=0, res=None, ldr=0, out_rows=None):
    """src/gemm_f16.c on fp16 arrays (uint16 views): A [M][lda] -> out [out_rows][ldo]."""
    A = np.ascontiguousarray(A).view(np.uint16)
    ldo = ldo or Np
    rows = out_rows or (((M // ow) + 2 * opad) * (ow + 2 * opad) if opad else M)
    out = np.zeros((rows, ldo), np.uint16)
    r = None if res is None else np.ascontiguousarray(res).view(np.uint16)
    lib().bnno_gemm_f16(ptr(A), A.shape[1], M, ptr(np.ascontiguousarray(w).view(np.uint16)), ptr(b32),
                        ptr(np.ascontiguousarray(b16).view(np.uint16)), Kp, Np, act, ptr(out), ldo, ow, opad, ptr(r),
                        ldr)
    return out.view(np.float16)


class Package:
    """A package executed on the CPU, one window at a time."""

    def __init__(self, path, path_name="neon-int8"):
        err = ctypes.create_string_buffer(256)
        self.h = lib().bnno_pkg_open(path.encode(), path_name.encode(), err, 256)
        if not self.h:
            raise OSError(err.value.decode())
        self.path, self.path_name = path, path_name

    def close(self):
        if self.h:
            lib().bnno_pkg_close(self.h)
            self.h = None

    def __del__(self):
        self.close()

    @property
    def n_ops(self):
        return lib().bnno_pkg_n_ops(self.h)

    @property
    def n_bufs(self):
        return lib().bnno_pkg_n_bufs(self.h)

    def op_code(self, i):
        return lib().bnno_pkg_op_code(self.h, i)

    def buf_info(self, i):
        dt = ctypes.c_int()
        e = lib().bnno_pkg_buf_elems(self.h, i, ctypes.byref(dt))
        return e, DTYPES[dt.value]

    def run(self, pcm):
        nc, ne = lib().bnno_pkg_out_elems(self.h), lib().bnno_pkg_emb_elems(self.h)
        out, emb = np.empty(nc, np.float32), np.empty(ne, np.float32)
        x = np.ascontiguousarray(pcm, np.float32)
        if lib().bnno_pkg_run(self.h, ptr(x), ptr(out), ptr(emb)):
            raise RuntimeError("oracle run failed")
        return out, emb

    def run_range(self, pcm, op0, op1):
        self._pcm = np.ascontiguousarray(pcm, np.float32)  # keep alive: buffer 0 points at it
        if lib().bnno_pkg_run_range(self.h, ptr(self._pcm), op0, op1):
            raise RuntimeError("oracle run failed")

    def get(self, i):
        e, dt = self.buf_info(i)
        a = np.empty(e, dt)
        lib().bnno_pkg_get_buf(self.h, i, ptr(a), a.nbytes)
        return a

    def set(self, i, a):
        a = np.ascontiguousarray(a)
        lib().bnno_pkg_set_buf(self.h, i, ptr(a), a.nbytes)


def run_many(path, pcm, threads=1, path_name="neon-int8"):
    """n windows on `threads` CPU threads: (out [n][n_classes], emb [n][emb_dim])."""
    p = Package(path, path_name)
    nc, ne = lib().bnno_pkg_out_elems(p.h), lib().bnno_pkg_emb_elems(p.h)
    p.close()
    x = np.ascontiguousarray(pcm, np.float32)
    out = np.empty((x.shape[0], nc), np.float32)
    emb = np.empty((x.shape[0], ne), np.float32)
    if lib().bnno_pkg_run_many(path.encode(), path_name.encode(), x.shape[0], ptr(x), ptr(out), ptr(emb), threads):
        raise RuntimeError("oracle run failed")
    return out, emb


def set_log_mode(mode):
    """The logarithm of FE_DBIMG in packages the oracle runs: 0 this host's logf (the reference's call), 1 the
    correctly rounded logarithm (the B200 kernel's)."""
    lib().bnno_pkg_set_log_mode(int(mode))


def log_f32(x, log_mode):
    """the FE_DBIMG logarithm elementwise (bnno_log_n): log_mode 0 this host's logf, 1 the double-precision log
    rounded once to float"""
    x = np.ascontiguousarray(x, np.float32)
    y = np.empty_like(x)
    lib().bnno_log_n(ptr(x), ptr(y), x.size, int(log_mode))
    return y


class DbImg:
    """FE_DBIMG (oracle_dbimg.c) from the record's 21 ints and its four tensors."""

    def __init__(self, p, window, mel, rows, consts):
        self._keep = [np.ascontiguousarray(p, np.int32), np.ascontiguousarray(window, np.float32),
                      np.ascontiguousarray(mel, np.float32), np.ascontiguousarray(rows, np.int32),
                      np.ascontiguousarray(consts, np.float32)]
        self.p = self._keep[0]
        self.h = lib().bnno_dbimg_new(*[ptr(a) for a in self._keep])
        self.nfr = lib().bnno_dbimg_frames_count(self.h)

    def image_elems(self):
        p = self.p
        return (int(p[14]) + 2 * int(p[20])) * (int(p[15]) + 2 * int(p[20])) * int(p[19])

    def run(self, pcm, log_mode=0):
        """windows pcm [n][nsamp] -> images [n][image elems]"""
        x = np.ascontiguousarray(pcm, np.float32).reshape(-1, int(self.p[0]))
        out = np.empty((x.shape[0], self.image_elems()), np.float32)
        for w in range(x.shape[0]):
            lib().bnno_dbimg_run(self.h, ptr(x[w]), ptr(out[w]), log_mode)
        return out

    def db(self, pcm, log_mode=0):
        x = np.ascontiguousarray(pcm, np.float32).reshape(-1)
        out = np.empty((int(self.p[6]), self.nfr), np.float32)
        lib().bnno_dbimg_frames(self.h, ptr(x), ptr(out), log_mode)
        return out

    def close(self):
        if self.h:
            lib().bnno_dbimg_free(self.h)
            self.h = None

    def __del__(self):
        self.close()
