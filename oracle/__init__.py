"""TEST INFRASTRUCTURE ONLY -- ctypes bindings for the CPU oracle.

Two CPU libraries live here, both built by ``oracle/Makefile``:

* ``liboracle.so`` -- this repository's plain-C restatement of pitorch's host
  decode/train arithmetic (``pt_oracle.c``), always built.
* ``_ref/libptref.so`` -- the reference's own host C sources compiled
  unchanged plus a thin shim (``ref_shim.c``); present only where the
  reference sources were available at build time.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline
leg may import this package, and only as the checker / CPU baseline. The
product library (``pitorch_b200``) never loads it.
"""
import ctypes
import os

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_SO = os.path.join(_HERE, "liboracle.so")
REF_SO = os.path.join(_HERE, "_ref", "libptref.so")

_f32p = ctypes.POINTER(ctypes.c_float)
_i32p = ctypes.POINTER(ctypes.c_int)


def _fp(a):
    return a.ctypes.data_as(_f32p)


def _ip(a):
    return a.ctypes.data_as(_i32p)


def build(with_ref=True):
    """Compile liboracle.so (and _ref/libptref.so when the sources exist)."""
    import subprocess
    target = "all" if with_ref else "oracle"
    subprocess.run(["make", "-s", "-C", _HERE, target], check=True)


_lib = None


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(ORACLE_SO):
            build(with_ref=False)
        L = ctypes.CDLL(ORACLE_SO)
        vp = ctypes.c_void_p
        for name in ("or_expf", "or_logf", "or_sinf", "or_cosf", "or_sqrtf"):
            getattr(L, name).restype = ctypes.c_float
            getattr(L, name).argtypes = [ctypes.c_float]
        L.or_open.restype = vp
        L.or_open.argtypes = [ctypes.c_char_p, ctypes.c_long, ctypes.c_int]
        L.or_close.argtypes = [vp]
        L.or_config.argtypes = [vp, _i32p]
        L.or_reset_kv.argtypes = [vp]
        L.or_forward.argtypes = [vp, ctypes.c_int, ctypes.c_int]
        L.or_logits.restype = _f32p
        L.or_logits.argtypes = [vp]
        L.or_x.restype = _f32p
        L.or_x.argtypes = [vp]
        L.or_set_x.argtypes = [vp, _f32p]
        L.or_forward_embed.argtypes = [vp, ctypes.c_int]
        L.or_forward_layers_range.argtypes = [vp, ctypes.c_int, ctypes.c_int, ctypes.c_int]
        L.or_forward_head.argtypes = [vp]
        L.or_decode_greedy.argtypes = [vp, _i32p, ctypes.c_int, ctypes.c_int, _i32p, _f32p]
        L.or_train_step.restype = ctypes.c_float
        L.or_train_step.argtypes = [vp, _i32p, ctypes.c_int, ctypes.c_float]
        L.or_forward_train.restype = ctypes.c_float
        L.or_forward_train.argtypes = [vp, _i32p, ctypes.c_int]
        L.or_blob.restype = vp
        L.or_blob.argtypes = [vp]
        L.or_blob_bytes.restype = ctypes.c_long
        L.or_blob_bytes.argtypes = [vp]
        L.or_grads.restype = _f32p
        L.or_grads.argtypes = [vp, ctypes.POINTER(ctypes.c_long)]
        L.or_matvec.argtypes = [_f32p, _f32p, _f32p, ctypes.c_int, ctypes.c_int]
        L.or_rmsnorm.argtypes = [_f32p, _f32p, _f32p, ctypes.c_int]
        L.or_softmax.argtypes = [_f32p, ctypes.c_int]
        L.or_silu.argtypes = [_f32p, ctypes.c_int]
        L.or_rope.argtypes = [_f32p, _f32p, ctypes.c_int, ctypes.c_int, ctypes.c_int]
        L.or_argmax.restype = ctypes.c_int
        L.or_argmax.argtypes = [_f32p, ctypes.c_int]
        L.or_rmsnorm_backward.argtypes = [_f32p, _f32p, _f32p, _f32p, _f32p, ctypes.c_int]
        L.or_rope_backward.argtypes = [_f32p, _f32p, _f32p, _f32p, ctypes.c_int, ctypes.c_int, ctypes.c_int]
        L.or_softmax_backward.argtypes = [_f32p, _f32p, _f32p, ctypes.c_int]
        _lib = L
    return _lib


_ref = None


def ref_available():
    return os.path.exists(REF_SO)


def ref_lib():
    """The reference's own host C (None when it was not built here)."""
    global _ref
    if _ref is None and ref_available():
        R = ctypes.CDLL(REF_SO)
        vp = ctypes.c_void_p
        R.ref_open.restype = vp
        R.ref_open.argtypes = [ctypes.c_char_p, ctypes.c_long, ctypes.c_int]
        R.ref_close.argtypes = [vp]
        R.ref_reset_kv.argtypes = [vp]
        R.ref_forward_step.restype = ctypes.c_int
        R.ref_forward_step.argtypes = [vp, ctypes.c_int]
        R.ref_logits.restype = _f32p
        R.ref_logits.argtypes = [vp]
        R.ref_train_step.restype = ctypes.c_float
        R.ref_train_step.argtypes = [vp, _i32p, ctypes.c_int, ctypes.c_float]
        R.ref_blob.restype = vp
        R.ref_blob.argtypes = [vp]
        R.ref_grads.restype = _f32p
        R.ref_grads.argtypes = [vp, ctypes.POINTER(ctypes.c_long)]
        R.ref_decode_greedy.argtypes = [vp, _i32p, ctypes.c_int, ctypes.c_int, _i32p, _f32p]
        R.ref_forward_embed.argtypes = [vp, ctypes.c_int]
        R.ref_forward_layers_range.argtypes = [vp, ctypes.c_int, ctypes.c_int, ctypes.c_int]
        R.ref_forward_head.argtypes = [vp]
        R.ref_x.restype = _f32p
        R.ref_x.argtypes = [vp]
        R.ref_matvec.argtypes = [_f32p, _f32p, _f32p, ctypes.c_int, ctypes.c_int]
        for name in ("pt_expf", "pt_logf", "pt_sinf", "pt_cosf", "pt_sqrtf"):
            getattr(R, name).restype = ctypes.c_float
            getattr(R, name).argtypes = [ctypes.c_float]
        _ref = R
    return _ref


class Model:
    """A model held by the oracle restatement (``impl='port'``) or by the
    reference's own host build (``impl='reference'``)."""

    def __init__(self, blob, max_T=0, impl="port"):
        self.impl = impl
        blob = bytes(blob)
        hdr = np.frombuffer(blob[:28], dtype=np.int32)
        self.dim, self.hidden, self.L, self.nh, self.nkv = (int(v) for v in hdr[:5])
        self.V = abs(int(hdr[5]))
        self.seq = int(hdr[6])
        self.nbytes = len(blob)
        if impl == "port":
            self._L = lib()
            self._h = self._L.or_open(blob, len(blob), max_T)
        elif impl == "reference":
            self._L = ref_lib()
            if self._L is None:
                raise RuntimeError("oracle/_ref/libptref.so was not built")
            self._h = self._L.ref_open(blob, len(blob), max_T)
        else:
            raise ValueError(impl)

    def close(self):
        if self._h:
            (self._L.or_close if self.impl == "port" else self._L.ref_close)(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def decode_greedy(self, prompt, n_pos, want_logits=False):
        prompt = np.ascontiguousarray(prompt, dtype=np.int32)
        toks = np.zeros(n_pos, dtype=np.int32)
        logits = np.zeros((n_pos, self.V), dtype=np.float32) if want_logits else None
        lp = _fp(logits) if want_logits else None
        f = self._L.or_decode_greedy if self.impl == "port" else self._L.ref_decode_greedy
        f(self._h, _ip(prompt), len(prompt), n_pos, _ip(toks), lp)
        return (toks, logits) if want_logits else toks

    def train_step(self, tokens, lr):
        tokens = np.ascontiguousarray(tokens, dtype=np.int32)
        f = self._L.or_train_step if self.impl == "port" else self._L.ref_train_step
        return float(f(self._h, _ip(tokens), len(tokens), ctypes.c_float(lr)))

    def blob(self):
        p = self._L.or_blob(self._h) if self.impl == "port" else self._L.ref_blob(self._h)
        return ctypes.string_at(p, self.nbytes)

    def grads(self):
        n = ctypes.c_long(0)
        f = self._L.or_grads if self.impl == "port" else self._L.ref_grads
        p = f(self._h, ctypes.byref(n))
        return np.ctypeslib.as_array(p, shape=(n.value,)).copy()

    # staged decode on the model's own state
    def forward_embed(self, token):
        (self._L.or_forward_embed if self.impl == "port" else self._L.ref_forward_embed)(self._h, token)

    def forward_layers_range(self, pos, l0, l1):
        f = self._L.or_forward_layers_range if self.impl == "port" else self._L.ref_forward_layers_range
        f(self._h, pos, l0, l1)

    def forward_head(self):
        (self._L.or_forward_head if self.impl == "port" else self._L.ref_forward_head)(self._h)

    def x(self):
        p = self._L.or_x(self._h) if self.impl == "port" else self._L.ref_x(self._h)
        return np.ctypeslib.as_array(p, shape=(self.dim,)).copy()

    def logits(self):
        p = self._L.or_logits(self._h) if self.impl == "port" else self._L.ref_logits(self._h)
        return np.ctypeslib.as_array(p, shape=(self.V,)).copy()

    def reset_kv(self):
        (self._L.or_reset_kv if self.impl == "port" else self._L.ref_reset_kv)(self._h)


def matvec(W, x, impl="port"):
    W = np.ascontiguousarray(W, dtype=np.float32)
    x = np.ascontiguousarray(x, dtype=np.float32)
    y = np.zeros(W.shape[0], dtype=np.float32)
    if impl == "port":
        lib().or_matvec(_fp(W), _fp(x), _fp(y), W.shape[0], W.shape[1])
    else:
        ref_lib().ref_matvec(_fp(W), _fp(x), _fp(y), W.shape[0], W.shape[1])
    return y
