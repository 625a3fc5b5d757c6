"""Python binding for the B200 libbnneon (ctypes + numpy), the counterpart of the reference's binding.

    from bnneon_b200 import Model
    with Model("birdnet_v2.4-neon-int8.bnpk") as m:
        scores, emb = m.infer(pcm)                 # one window, m.info.n_samples float32 samples
        scores, emb = m.infer_batch(windows)       # [n][n_samples] -> [n][n_classes], [n][emb_dim]
        conf = m.confidences(scores)

The API follows python/bnneon/binding.py of the reference (Model, Info, BnnError, infer, confidences; the library
is loaded from `lib`, else the BNNEON_LIB environment variable, else the in-tree build), with the B200 additions of
include/bnneon_cuda.h: infer_batch, infer_device (device pointers), set_batch, and the op-level debug calls.
"""
import ctypes
import os

import numpy as np

API_VERSION = 2
MODE_DEFAULT, MODE_REFERENCE, MODE_FP32, MODE_FP16, MODE_INT8 = 0, 1, 2, 3, 4
POST_NONE, POST_SIGMOID, POST_SOFTMAX = 0, 1, 2
ERR_KINDS = {0: "NONE", 1: "PACKAGE", 2: "OOM", 3: "CPU", 4: "WINDOW", 5: "LABELS", 6: "USAGE"}

PKG_DIR = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
DEFAULT_LIB = os.path.join(PKG_DIR, "libbnneon.so")


class BnnError(RuntimeError):
    """A failed library call: str(e) is bnn_last_error(), e.kind the BNN_ERR_* name."""

    def __init__(self, message, kind):
        super().__init__(message)
        self.kind = kind


class Info(ctypes.Structure):
    """bnn_info (API 2; fields only ever appended)."""
    _fields_ = [("struct_size", ctypes.c_uint32), ("model", ctypes.c_int), ("format_version", ctypes.c_int),
                ("sample_rate", ctypes.c_int), ("n_samples", ctypes.c_int), ("hop_samples", ctypes.c_int),
                ("n_classes", ctypes.c_int), ("output_kind", ctypes.c_int), ("post", ctypes.c_int),
                ("logit_scale", ctypes.c_float), ("emb_dim", ctypes.c_int), ("has_labels_sha", ctypes.c_int),
                ("labels_sha256", ctypes.c_ubyte * 32), ("model_id", ctypes.c_char * 64),
                ("path", ctypes.c_char * 32), ("precision", ctypes.c_char_p)]


_P = ctypes.c_void_p
_FP = ctypes.POINTER(ctypes.c_float)
_I, _LL, _SZ, _S = ctypes.c_int, ctypes.c_longlong, ctypes.c_size_t, ctypes.c_char_p
SIGNATURES = {
    "bnn_api_version": (_I, []),
    "bnn_cpu_supported": (_I, [_I]),
    "bnn_probe": (_I, [_S, ctypes.POINTER(Info)]),
    "bnn_probe_meta": (_I, [_S, _S, _S, _SZ]),
    "bnn_meta": (_I, [_P, _S, _S, _SZ]),
    "bnn_init": (_P, [_S, _I]),
    "bnn_get_info": (_I, [_P, ctypes.POINTER(Info)]),
    "bnn_infer": (_I, [_P, _P, _P, _P]),
    "bnn_verify_labels": (_I, [_S, _S]),
    "bnn_last_error": (_S, []),
    "bnn_last_error_kind": (_I, []),
    "bnn_set_threads": (_I, [_P, _I]),
    "bnn_free": (None, [_P]),
    # bnneon_cuda.h
    "bnn_infer_batch": (_I, [_P, _I, _P, _P, _P]),
    "bnn_infer_device": (_I, [_P, _I, _P, _P, _P, _P]),
    "bnn_set_batch": (_I, [_P, _I]),
    "bnn_get_batch": (_I, [_P]),
    "bnn_launches_per_batch": (_I, [_P]),
    "bnn_profile_begin": (_I, [_P]),
    "bnn_profile_collect": (_I, [_P]),
    "bnn_profile_op_ms": (ctypes.c_double, [_P, _I]),
    "bnn_profile_end": (_I, [_P]),
    "bnn_cuda_peak_hfma2": (_I, [_I, _I, _P, _P]),
    "bnn_pw_f16_new": (_P, [_I, _I, _I, _I, _P, _P, _P]),
    "bnn_pw_f16_run": (_I, [_P, _I, _I, _P, _LL, _I, _I, _P, _LL, _I, _I, _I, _P, _LL, _I, _P]),
    "bnn_pw_f16_free": (None, [_P]),
    "bnn_cuda_dw3_f16": (_I, [_I, _P, _LL, _I, _I, _I, _I, _I, _I, _P, _P, _P, _LL, _I, _I, _P, _LL, _P]),
    "bnn_cuda_dwk_f16": (_I, [_I, _P, _LL, _I, _I, _I, _I, _I, _I, _I, _P, _P, _I, _P, _LL, _I, _I, _P, _LL, _P]),
    "bnn_cuda_stem_f16": (_I, [_I, _P, _LL, _I, _I, _I, _I, _I, _I, _P, _P, _I, _I, _I, _P, _LL, _I, _I, _P]),
    "bnn_debug_n_ops": (_I, [_P]),
    "bnn_debug_op_code": (_I, [_P, _I]),
    "bnn_debug_run_ops": (_I, [_P, _I, _P, _I, _I]),
    "bnn_debug_get_buffer": (_I, [_P, _I, _I, _P]),
    "bnn_debug_set_buffer": (_I, [_P, _I, _I, _P]),
    "bnn_cuda_device_init": (_I, []),
    "bnn_cuda_quant_rows": (_I, [_I, _I, _P, _LL, _I, _I, _I, _P, _LL, _P, _P, _P, _P]),
    "bnn_pw_s8_new": (_P, [_I, _I, _I, _I, _P, _P, _P, _P, _I]),
    "bnn_pw_s8_run": (_I, [_P, _I, _I, _P, _LL, _I, _P, _LL, _I, _P, _LL, _I, _I, _I, _P, _LL, _I, _I, _I, _P]),
    "bnn_pw_s8_run_static": (_I, [_P, _I, _I, _P, _LL, _I, _P, _LL, _I, _P, _LL, _I, _I, _I, _P, _LL, _I, _I, _I, _P]),
    "bnn_pw_s8_gemm": (_I, [_P, _I, _I, _P, _LL, _P, _P, _I, _P, _LL, _I, _I, _I, _P, _LL, _I, _I, _I, _P]),
    "bnn_pw_s8_error": (_I, [_P]),
    "bnn_pw_s8_free": (None, [_P]),
    "bnn_logmel_new": (_P, [_I, _I, _I, _I, _I, _I, _P, _P, ctypes.c_float, ctypes.c_float]),
    "bnn_logmel_frames": (_I, [_P]),
    "bnn_logmel_run": (_I, [_P, _I, _P, _LL, _P, _LL, _P]),
    "bnn_logmel_free": (None, [_P]),
    "bnn_dbimg_new": (_P, [_P, _I, _P, _P, _P, _P, _I]),
    "bnn_dbimg_image_elems": (_LL, [_P]),
    "bnn_dbimg_run": (_I, [_P, _I, _P, _LL, _P, _LL, _P]),
    "bnn_dbimg_free": (None, [_P]),
    "bnn_proto_s8_new": (_P, [_I, _I, _I, _I, _P, _P, _P, _P, _P, _I, _I, ctypes.c_float, _I, _I]),
    "bnn_proto_s8_run": (_I, [_P, _I, _P, _LL, _I, _P, _LL, _P, _LL, _P, _P]),
    "bnn_proto_s8h_new": (_P, [_I, _I, _I, _P, _P, _P, _P, _I, _I, ctypes.c_float, _I, _I]),
    "bnn_proto_s8h_run": (_I, [_P, _I, _P, _LL, _I, _P, _LL, _P, _LL, _P, _P]),
    "bnn_proto_s8_read_scratch": (_I, [_P, _I, _P, _P]),
    "bnn_proto_s8_error": (_I, [_P]),
    "bnn_proto_s8_free": (None, [_P]),
    "bnn_cuda_dw3": (_I, [_I, _P, _LL, _I, _I, _I, _I, _P, _P, _P, _LL, _I, _I, _P, _LL, _P]),
    "bnn_cuda_fn": (_I, [_I, _I, _P, _P, _P]),
    "bnn_debug_fail_alloc": (_I, [_I, _I]),
    "bnn_debug_stall_next_gemm": (None, []),
    "bnn_set_fp16_tensor": (_I, [_P, _I]),
    "bnn_get_fp16_tensor": (_I, [_P]),
    "bnn_cuda_op_error": (_I, []),
}

_LIB = None


def load_library(lib=None):
    """Loads libbnneon (lib, else BNNEON_LIB, else the in-tree build) and sets the signatures."""
    global _LIB  # pylint: disable=global-statement
    if _LIB is not None and lib is None:
        return _LIB
    path = lib or os.environ.get("BNNEON_LIB") or DEFAULT_LIB
    if not os.path.exists(path):
        raise OSError(f"{path} not found: build it first (make -C birdnet-neon-engine_b200, or "
                      f"__graft_entry__.build())")
    h = ctypes.CDLL(path)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(h, name)
        fn.restype = res
        fn.argtypes = args
    if h.bnn_api_version() != API_VERSION:
        raise BnnError(f"{path} speaks API {h.bnn_api_version()}, this binding {API_VERSION}", "USAGE")
    if lib is None:
        _LIB = h
    return h


def last_error(h=None):
    h = h or load_library()
    return BnnError(h.bnn_last_error().decode(errors="replace"), ERR_KINDS.get(h.bnn_last_error_kind(), "?"))


def _ptr(a):
    return None if a is None else a.ctypes.data


def probe(path, lib=None):
    h = load_library(lib)
    info = Info()
    info.struct_size = ctypes.sizeof(Info)
    if h.bnn_probe(path.encode(), ctypes.byref(info)):
        raise last_error(h)
    return info


def probe_meta(path, key, lib=None):
    h = load_library(lib)
    n = h.bnn_probe_meta(path.encode(), key.encode(), None, 0)
    if n < 0:
        return None
    buf = ctypes.create_string_buffer(n + 1)
    h.bnn_probe_meta(path.encode(), key.encode(), buf, n + 1)
    return buf.raw[:n]


class Model:
    """One context (one per thread). Results are bit-identical for any batch split and GPU count."""

    def __init__(self, path, mode=MODE_DEFAULT, lib=None, batch=None, devices=None, fp16_tensor=None):
        self.h = load_library(lib)
        self.ctx = self.h.bnn_init(path.encode(), mode)
        if not self.ctx:
            raise last_error(self.h)
        self.info = Info()
        self.info.struct_size = ctypes.sizeof(Info)
        self.h.bnn_get_info(self.ctx, ctypes.byref(self.info))
        if batch is not None:
            self.set_batch(batch)
        if devices is not None:
            self.set_threads(devices)
        if fp16_tensor is not None:
            self.set_fp16_tensor(fp16_tensor)

    def _check(self, rc):
        if rc:
            raise last_error(self.h)

    def close(self):
        if self.ctx:
            self.h.bnn_free(self.ctx)
            self.ctx = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:  # pylint: disable=broad-except
            pass

    def set_threads(self, n):
        self._check(self.h.bnn_set_threads(self.ctx, n))

    def set_batch(self, n):
        self._check(self.h.bnn_set_batch(self.ctx, n))

    def set_fp16_tensor(self, on):
        """the neon-fp16 path's 1x1 convs on the tensor cores (within a tolerance of the reference, not bit-exact)"""
        self._check(self.h.bnn_set_fp16_tensor(self.ctx, 1 if on else 0))

    @property
    def fp16_tensor(self):
        return bool(self.h.bnn_get_fp16_tensor(self.ctx))

    @property
    def batch(self):
        return self.h.bnn_get_batch(self.ctx)

    @property
    def launches_per_batch(self):
        return self.h.bnn_launches_per_batch(self.ctx)

    def meta(self, key):
        n = self.h.bnn_meta(self.ctx, key.encode(), None, 0)
        if n < 0:
            return None
        buf = ctypes.create_string_buffer(n + 1)
        self.h.bnn_meta(self.ctx, key.encode(), buf, n + 1)
        return buf.raw[:n]

    def infer(self, pcm):
        x = np.ascontiguousarray(pcm, np.float32).reshape(-1)
        if x.size != self.info.n_samples:
            raise BnnError(f"infer: {x.size} samples, the model takes {self.info.n_samples}", "USAGE")
        out = np.empty(self.info.n_classes, np.float32)
        emb = np.empty(self.info.emb_dim, np.float32) if self.info.emb_dim else None
        self._check(self.h.bnn_infer(self.ctx, _ptr(x), _ptr(out), _ptr(emb)))
        return out, emb

    def infer_batch(self, windows, out=None, emb=None):
        x = np.ascontiguousarray(windows, np.float32)
        n = x.shape[0]
        if x.ndim != 2 or x.shape[1] != self.info.n_samples:
            raise BnnError(f"infer_batch: shape {x.shape}, expected [n][{self.info.n_samples}]", "USAGE")
        if out is None:
            out = np.empty((n, self.info.n_classes), np.float32)
        if emb is None and self.info.emb_dim:
            emb = np.empty((n, self.info.emb_dim), np.float32)
        self._check(self.h.bnn_infer_batch(self.ctx, n, _ptr(x), _ptr(out), _ptr(emb)))
        return out, emb

    def infer_device(self, n, d_pcm, d_out, d_emb=None, stream=None):
        """Device pointers (ints); asynchronous on `stream` (a cudaStream_t as int) when given."""
        self._check(self.h.bnn_infer_device(self.ctx, n, d_pcm, d_out, d_emb, stream))

    def confidences(self, scores):
        z = np.asarray(scores, np.float64) * self.info.logit_scale
        if self.info.post == POST_SIGMOID:
            return (1.0 / (1.0 + np.exp(-z))).astype(np.float32)
        if self.info.post == POST_SOFTMAX:
            e = np.exp(z - z.max(-1, keepdims=True))
            return (e / e.sum(-1, keepdims=True)).astype(np.float32)
        return z.astype(np.float32)

    # op-level debugging (package buffer ids, n windows)
    @property
    def n_ops(self):
        return self.h.bnn_debug_n_ops(self.ctx)

    def op_code(self, i):
        return self.h.bnn_debug_op_code(self.ctx, i)

    def run_ops(self, pcm, op0, op1):
        x = None if pcm is None else np.ascontiguousarray(pcm, np.float32)
        n = 1 if x is None else x.shape[0]
        self._check(self.h.bnn_debug_run_ops(self.ctx, n, _ptr(x), op0, op1))

    def get_buffer(self, buf, n, dtype, elems):
        a = np.empty((n, elems), dtype)
        self._check(self.h.bnn_debug_get_buffer(self.ctx, buf, n, _ptr(a)))
        return a

    def set_buffer(self, buf, a):
        a = np.ascontiguousarray(a)
        self._check(self.h.bnn_debug_set_buffer(self.ctx, buf, a.shape[0], _ptr(a)))


def verify_labels(path, labels, lib=None):
    h = load_library(lib)
    if h.bnn_verify_labels(path.encode(), labels.encode()):
        raise last_error(h)
