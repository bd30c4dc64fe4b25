"""CPU oracle for the attention forward — TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg import
this module; the product (flash-attention-cuda_b200/) never does.

Two restatements of the reference's CPU path:
  * numpy (this file), following src/attention_cpu.py: stable_softmax
    (lines 13-27: subtract the row max, exp, divide by the row sum) and
    attention_cpu (lines 29-62: S = Q K^T * scale, P = softmax(S), O = P V),
    looped over (B, H), with the causal mask k <= q of csrc/prefill.cu:268 and
    the decode rules of csrc/decode.cu (seq_lens clamped to the cache length,
    line 69; no keys -> output 0, lines 164-172).
  * plain C (attention_oracle.c, double accumulation), loaded with ctypes
    from liboracle.so, built by `make -C oracle`.

Inputs are expected to hold fp16-representable values (the product's inputs
are fp16); both restatements compute in fp32/fp64 and return fp32.
"""

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
HEAD_DIM = 64


# ---------------------------------------------------------------------------
# numpy restatement
# ---------------------------------------------------------------------------
def stable_softmax(x):
    """Row-wise softmax with the row max subtracted (attention_cpu.py:13-27)."""
    x_max = np.max(x, axis=-1, keepdims=True)
    e = np.exp(x - x_max)
    return e / np.sum(e, axis=-1, keepdims=True)


def attention_cpu(q, k, v, scale=None, causal=False):
    """softmax(Q K^T * scale [+ causal mask]) V for one (N, d) head
    (attention_cpu.py:29-62, plus the causal mask of prefill.cu:268)."""
    n, d = q.shape
    if scale is None:
        scale = 1.0 / np.sqrt(d)
    s = (q @ k.T) * scale
    if causal:
        s = np.where(np.tril(np.ones((n, k.shape[0]), dtype=bool)), s, -np.inf)
    return stable_softmax(s) @ v


def prefill_ref(q, k, v, causal, scale, dtype=np.float64):
    """(B, H, N, 64) -> (B, H, N, 64), looping attention_cpu over (B, H)."""
    q = np.asarray(q, dtype=dtype)
    k = np.asarray(k, dtype=dtype)
    v = np.asarray(v, dtype=dtype)
    out = np.empty(q.shape, dtype=np.float32)
    for b in range(q.shape[0]):
        for h in range(q.shape[1]):
            out[b, h] = attention_cpu(q[b, h], k[b, h], v[b, h], scale, causal)
    return out


def decode_ref(q, k_cache, v_cache, seq_lens, scale, dtype=np.float64):
    """q (B, H, 1, 64), caches (B, H, S_max, 64), seq_lens (B,)."""
    q = np.asarray(q, dtype=dtype)
    out = np.zeros(q.shape, dtype=np.float32)
    s_max = k_cache.shape[2]
    for b in range(q.shape[0]):
        n = int(min(max(int(seq_lens[b]), 0), s_max))
        if n == 0:
            continue
        kb = np.asarray(k_cache[b, :, :n], dtype=dtype)
        vb = np.asarray(v_cache[b, :, :n], dtype=dtype)
        for h in range(q.shape[1]):
            out[b, h] = attention_cpu(q[b, h], kb[h], vb[h], scale, False)
    return out


# ---------------------------------------------------------------------------
# C restatement (ctypes)
# ---------------------------------------------------------------------------
_LIB = None


def lib_path():
    return os.path.join(HERE, "liboracle.so")


def build():
    """Compiles attention_oracle.c into liboracle.so (gcc, no GPU needed)."""
    subprocess.check_call(["make", "-s", "-C", HERE, "liboracle.so"])
    return lib_path()


def _lib():
    global _LIB
    if _LIB is None:
        if not os.path.exists(lib_path()):
            build()
        lib = ctypes.CDLL(lib_path())
        fp = ctypes.POINTER(ctypes.c_float)
        ip = ctypes.POINTER(ctypes.c_int)
        lib.oracle_prefill.argtypes = [fp, fp, fp, fp, ctypes.c_int,
                                       ctypes.c_int, ctypes.c_int,
                                       ctypes.c_int, ctypes.c_double]
        lib.oracle_prefill.restype = ctypes.c_int
        lib.oracle_decode.argtypes = [fp, fp, fp, ip, fp, ctypes.c_int,
                                      ctypes.c_int, ctypes.c_int,
                                      ctypes.c_double]
        lib.oracle_decode.restype = ctypes.c_int
        _LIB = lib
    return _LIB


def _f32(a):
    return np.ascontiguousarray(a, dtype=np.float32)


def _ptr(a, ctype=ctypes.c_float):
    return a.ctypes.data_as(ctypes.POINTER(ctype))


def prefill_c(q, k, v, causal, scale):
    q, k, v = _f32(q), _f32(k), _f32(v)
    b, h, n, d = q.shape
    assert d == HEAD_DIM and k.shape == q.shape and v.shape == q.shape
    o = np.empty_like(q)
    rc = _lib().oracle_prefill(_ptr(q), _ptr(k), _ptr(v), _ptr(o), b, h, n,
                               1 if causal else 0, float(scale))
    if rc != 0:
        raise MemoryError("oracle_prefill failed")
    return o


def decode_c(q, k_cache, v_cache, seq_lens, scale):
    q, k, v = _f32(q), _f32(k_cache), _f32(v_cache)
    lens = np.ascontiguousarray(seq_lens, dtype=np.int32)
    b, h, one, d = q.shape
    assert one == 1 and d == HEAD_DIM and k.shape[:2] == (b, h)
    o = np.empty_like(q)
    rc = _lib().oracle_decode(_ptr(q), _ptr(k), _ptr(v), _ptr(lens, ctypes.c_int),
                              _ptr(o), b, h, k.shape[2], float(scale))
    if rc != 0:
        raise MemoryError("oracle_decode failed")
    return o
