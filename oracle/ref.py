"""ctypes wrapper of oracle/_ref/libbnneon_ref.so (TEST INFRASTRUCTURE): the reference's own C runtime, compiled for
this x86 host from its unmodified sources by oracle/ref.mk (NEON intrinsics through the scalar stand-in
oracle/neon/arm_neon.h, the two assembly K-blocks through their scalar restatements).

It pins the oracle (oracle/liboracle.so, our C restatement) to the reference's code: tests/test_oracle_vs_ref.py
compares the two bit for bit. bench.py's reference arm times it. The product library never loads it.

The library is built where a checkout of the reference is present (BNN_REFERENCE, or a directory `reference` beside
this repository) and travels with the repository's other built files.
"""
import ctypes
import os
import subprocess
import tempfile
from concurrent.futures import ThreadPoolExecutor

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(HERE)
LIB_PATH = os.path.join(HERE, "_ref", "libbnneon_ref.so")
_LIB = None


def reference_checkout():
    """The reference checkout to build from, or None."""
    for d in (os.environ.get("BNN_REFERENCE"), os.path.join(os.path.dirname(REPO), "reference")):
        if d and os.path.exists(os.path.join(d, "src", "rt_pkg.c")):
            return d
    return None


def build(jobs=8):
    """make -f oracle/ref.mk when a reference checkout is present; returns the library path or None."""
    ref = reference_checkout()
    if ref is None:
        return LIB_PATH if os.path.exists(LIB_PATH) else None
    subprocess.run(["make", "-C", HERE, "-f", "ref.mk", f"REF={ref}", "-j", str(jobs)], check=True,
                   stdout=subprocess.DEVNULL)
    return LIB_PATH


def available():
    return os.path.exists(LIB_PATH)


class _Info(ctypes.Structure):
    """bnn_info (src/bnneon.h:36-55)"""
    _fields_ = [("struct_size", ctypes.c_uint32), ("model", ctypes.c_int), ("format_version", ctypes.c_int),
                ("sample_rate", ctypes.c_int), ("n_samples", ctypes.c_int), ("hop_samples", ctypes.c_int),
                ("n_classes", ctypes.c_int), ("output_kind", ctypes.c_int), ("post", ctypes.c_int),
                ("logit_scale", ctypes.c_float), ("emb_dim", ctypes.c_int), ("has_labels_sha", ctypes.c_int),
                ("labels_sha256", ctypes.c_ubyte * 32), ("model_id", ctypes.c_char * 64), ("path", ctypes.c_char * 32),
                ("precision", ctypes.c_char_p)]


def lib():
    global _LIB  # pylint: disable=global-statement
    if _LIB is None:
        if not os.path.exists(LIB_PATH):
            raise OSError(f"{LIB_PATH} missing: run `make -C oracle -f ref.mk REF=<reference checkout>`")
        h = ctypes.CDLL(LIB_PATH)
        P, I = ctypes.c_void_p, ctypes.c_int
        h.bnn_init.restype, h.bnn_init.argtypes = P, [ctypes.c_char_p, I]
        h.bnn_infer.restype, h.bnn_infer.argtypes = I, [P, P, P, P]
        h.bnn_free.restype, h.bnn_free.argtypes = None, [P]
        h.bnn_set_threads.restype, h.bnn_set_threads.argtypes = I, [P, I]
        h.bnn_get_info.restype, h.bnn_get_info.argtypes = I, [P, P]
        h.bnn_last_error.restype, h.bnn_last_error.argtypes = ctypes.c_char_p, []
        h.bnn_last_error_kind.restype, h.bnn_last_error_kind.argtypes = I, []
        _LIB = h
    return _LIB


class Context:
    """One reference context (bnn_init / bnn_infer / bnn_free, src/bnneon.h:59-99), single-threaded."""

    def __init__(self, path, mode, dump_dir=None):
        h = lib()
        old = os.environ.get("BNN_DUMP")
        if dump_dir:
            os.environ["BNN_DUMP"] = dump_dir  # read once by the context (src/rt_pkg.c:500)
        try:
            self.ctx = h.bnn_init(path.encode(), mode)
        finally:
            if dump_dir:
                if old is None:
                    del os.environ["BNN_DUMP"]
                else:
                    os.environ["BNN_DUMP"] = old
        if not self.ctx:
            raise RuntimeError(f"reference bnn_init: {h.bnn_last_error().decode()}")
        h.bnn_set_threads(self.ctx, 1)
        info = _Info()
        info.struct_size = ctypes.sizeof(_Info)
        h.bnn_get_info(self.ctx, ctypes.byref(info))
        self.n_classes, self.emb_dim, self.n_samples = info.n_classes, info.emb_dim, info.n_samples

    def infer(self, pcm, out=None, emb=None):
        """one window: returns (rc, out, emb); rc != 0 is a failed window (bnn_infer's return)"""
        x = np.ascontiguousarray(pcm, np.float32)
        out = np.empty(self.n_classes, np.float32) if out is None else out
        emb = (np.empty(self.emb_dim, np.float32) if self.emb_dim else None) if emb is None else emb
        rc = lib().bnn_infer(self.ctx, x.ctypes.data, out.ctypes.data, None if emb is None else emb.ctypes.data)
        return rc, out, emb

    def close(self):
        if self.ctx:
            lib().bnn_free(self.ctx)
            self.ctx = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()


def run_many(path, mode, pcm, threads=1):
    """n windows, one single-threaded context per worker thread (windows are independent): (out, emb, rc)"""
    x = np.ascontiguousarray(pcm, np.float32)
    n = x.shape[0]
    threads = max(1, min(threads, n))
    ctxs = [Context(path, mode) for _ in range(threads)]
    try:
        out = np.empty((n, ctxs[0].n_classes), np.float32)
        emb = np.empty((n, max(ctxs[0].emb_dim, 1)), np.float32)
        rc = np.zeros(n, np.int32)

        def work(t):
            for w in range(t, n, threads):
                rc[w] = ctxs[t].infer(x[w], out[w], emb[w] if ctxs[t].emb_dim else None)[0]
        with ThreadPoolExecutor(threads) as ex:
            list(ex.map(work, range(threads)))
        return out, emb[:, :ctxs[0].emb_dim], rc
    finally:
        for c in ctxs:
            c.close()


def dump_ops(path, mode, pcm):
    """One window through the reference with BNN_DUMP (src/rt_pkg.c:512-526): {(op, buffer argument): raw bytes} of
    every buffer each op writes, as it is right after that op, plus (rc, out, emb)."""
    with tempfile.TemporaryDirectory() as td:
        with Context(path, mode, dump_dir=td) as c:
            res = c.infer(pcm)
        dumps = {}
        for fn in os.listdir(td):
            if fn.startswith("op") and fn.endswith(".bin"):
                op, arg = fn[2:-4].split("_b")
                with open(os.path.join(td, fn), "rb") as f:
                    dumps[(int(op), int(arg))] = f.read()
    return dumps, res
