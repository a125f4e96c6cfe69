"""TEST INFRASTRUCTURE ONLY: ctypes binding of the C++ oracle (oracle/vdx_oracle.cpp).

The oracle is the CPU restatement of TVdxSampler (src/VindexLLM.Sampler.pas) used as
the parity checker by tests/, __graft_entry__.smoke() and bench.py's CPU legs. The
product library (vindexllm_b200) never imports this module.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

from vindexllm_b200.abi import VdxsConfig, DTYPE_F32, DTYPE_BF16, TIES_FAITHFUL

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "_build", "libvdxoracle.so")

_lib = None


def build(force: bool = False) -> str:
    """Compile the oracle with its Makefile (g++ only, no GPU needed)."""
    if force or not os.path.exists(LIB_PATH) or _stale():
        subprocess.run(["make", "-C", HERE, "-s"], check=True)
    return LIB_PATH


def _stale() -> bool:
    try:
        t = os.path.getmtime(LIB_PATH)
    except OSError:
        return True
    srcs = [os.path.join(HERE, f) for f in ("vdx_oracle.cpp", "vdx_oracle.h")]
    srcs.append(os.path.join(HERE, "..", "include", "vdx_sampler.h"))
    return any(os.path.exists(s) and os.path.getmtime(s) > t for s in srcs)


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build()
        L = C.CDLL(LIB_PATH)
        P = C.POINTER
        L.vdxo_create.restype = C.c_void_p
        L.vdxo_destroy.argtypes = [C.c_void_p]
        L.vdxo_default_config.argtypes = [P(VdxsConfig)]
        L.vdxo_set_config.argtypes = [C.c_void_p, P(VdxsConfig)]
        L.vdxo_get_config.argtypes = [C.c_void_p, P(VdxsConfig)]
        L.vdxo_add_to_history.argtypes = [C.c_void_p, C.c_int32]
        L.vdxo_reset_history.argtypes = [C.c_void_p]
        L.vdxo_get_history.argtypes = [C.c_void_p, P(C.c_int32), C.c_int32, P(C.c_int32), P(C.c_int32)]
        L.vdxo_get_history.restype = C.c_int32
        L.vdxo_process.argtypes = [C.c_void_p, P(C.c_float), C.c_int32]
        L.vdxo_process.restype = C.c_int32
        L.vdxo_next_uint64.argtypes = [C.c_void_p]
        L.vdxo_next_uint64.restype = C.c_uint64
        L.vdxo_next_float.argtypes = [C.c_void_p]
        L.vdxo_next_float.restype = C.c_float
        L.vdxo_get_state.argtypes = [C.c_void_p, P(C.c_uint64)]
        L.vdxo_set_state.argtypes = [C.c_void_p, P(C.c_uint64)]
        L.vdxo_splitmix64.argtypes = [P(C.c_uint64)]
        L.vdxo_splitmix64.restype = C.c_uint64
        L.vdxo_process_row.argtypes = [P(VdxsConfig), C.c_int32, P(C.c_float), C.c_int32,
                                       P(C.c_int32), C.c_int32, C.c_float, P(C.c_uint32),
                                       P(C.c_int32), P(C.c_float), C.c_int32]
        L.vdxo_process_row.restype = C.c_int32
        L.vdxo_sample_batch.argtypes = [P(VdxsConfig), C.c_int32, C.c_void_p, C.c_int32,
                                        C.c_int32, C.c_int32, C.c_int64, C.c_void_p, C.c_int64,
                                        C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p,
                                        C.c_void_p, C.c_void_p, C.c_int32, C.c_int32]
        L.vdxo_sample_batch.restype = C.c_int32
        L.vdxo_matvec_q4_0.argtypes = [C.c_void_p, C.c_void_p, C.c_int32, C.c_int32, C.c_int32, C.c_void_p,
                                       C.c_int32]
        L.vdxo_matvec_q4_0.restype = C.c_int32
        _lib = L
    return _lib


def _ptr(a):
    return None if a is None else a.ctypes.data_as(C.c_void_p)


class OracleSampler:
    """One TVdxSampler object (the reference's stateful API)."""

    def __init__(self):
        self._h = lib().vdxo_create()

    def close(self):
        if self._h:
            lib().vdxo_destroy(self._h)
            self._h = None

    def __del__(self):
        self.close()

    def set_config(self, cfg: VdxsConfig):
        lib().vdxo_set_config(self._h, C.byref(cfg))

    def get_config(self) -> VdxsConfig:
        c = VdxsConfig()
        lib().vdxo_get_config(self._h, C.byref(c))
        return c

    def add_to_history(self, tok: int):
        lib().vdxo_add_to_history(self._h, tok)

    def reset_history(self):
        lib().vdxo_reset_history(self._h)

    def history(self):
        cap = 1 << 16
        buf = (C.c_int32 * cap)()
        cnt, pos = C.c_int32(), C.c_int32()
        n = lib().vdxo_get_history(self._h, buf, cap, C.byref(cnt), C.byref(pos))
        return list(buf[:n]), cnt.value, pos.value

    def process(self, logits: np.ndarray) -> int:
        """Process(PSingle, V): mutates ``logits`` (float32, contiguous) like the reference."""
        assert logits.dtype == np.float32 and logits.flags.c_contiguous
        return lib().vdxo_process(self._h, logits.ctypes.data_as(C.POINTER(C.c_float)), logits.size)

    def next_uint64(self) -> int:
        return lib().vdxo_next_uint64(self._h)

    def next_float(self) -> float:
        return lib().vdxo_next_float(self._h)

    def get_state(self):
        st = (C.c_uint64 * 4)()
        lib().vdxo_get_state(self._h, st)
        return list(st)

    def set_state(self, st):
        lib().vdxo_set_state(self._h, (C.c_uint64 * 4)(*st))


def splitmix64(state: int):
    s = C.c_uint64(state)
    r = lib().vdxo_splitmix64(C.byref(s))
    return s.value, r


def process_row(cfg: VdxsConfig, logits: np.ndarray, history=None, uniform: float = 0.0,
                tie_mode: int = TIES_FAITHFUL, out_k: int = 0):
    """One row with an injected uniform. Returns (token, flags, idx[out_k], prob[out_k])."""
    x = np.ascontiguousarray(logits, dtype=np.float32).copy()
    h = None if history is None else np.ascontiguousarray(history, dtype=np.int32)
    flags = C.c_uint32()
    oi = np.full(max(out_k, 1), -1, np.int32)
    op = np.zeros(max(out_k, 1), np.float32)
    tok = lib().vdxo_process_row(
        C.byref(cfg), tie_mode, x.ctypes.data_as(C.POINTER(C.c_float)), x.size,
        None if h is None else h.ctypes.data_as(C.POINTER(C.c_int32)),
        0 if h is None else h.size, C.c_float(uniform), C.byref(flags),
        oi.ctypes.data_as(C.POINTER(C.c_int32)), op.ctypes.data_as(C.POINTER(C.c_float)), out_k)
    return tok, flags.value, oi[:out_k], op[:out_k]


def sample_batch(cfg: VdxsConfig, logits: np.ndarray, uniforms: np.ndarray, history=None,
                 history_count=None, tie_mode: int = TIES_FAITHFUL, out_k: int = 0,
                 nthreads: int = 1, diag: bool = True, vocab: int | None = None):
    """Batched oracle. ``logits`` is [B, stride] float32 or uint16 (bf16 bits)."""
    assert logits.ndim == 2 and logits.flags.c_contiguous
    if logits.dtype == np.float32:
        dt = DTYPE_F32
    elif logits.dtype in (np.uint16, np.int16):
        dt = DTYPE_BF16
    else:
        raise TypeError(f"unsupported logits dtype {logits.dtype}")
    B, stride = logits.shape
    V = stride if vocab is None else vocab
    u = np.ascontiguousarray(uniforms, dtype=np.float32)
    hist = hcnt = None
    hs = 0
    if history is not None:
        hist = np.ascontiguousarray(history, dtype=np.int32)
        hs = hist.shape[1]
        hcnt = np.ascontiguousarray(history_count, dtype=np.int32)
    tokens = np.zeros(B, np.int32)
    flags = np.zeros(B, np.uint32) if diag else None
    oi = np.full((B, out_k), -1, np.int32) if out_k else None
    op = np.zeros((B, out_k), np.float32) if out_k else None
    rc = lib().vdxo_sample_batch(C.byref(cfg), tie_mode, _ptr(logits), dt, B, V, stride,
                                 _ptr(hist), hs, _ptr(hcnt), _ptr(u), _ptr(tokens), _ptr(flags),
                                 _ptr(oi), _ptr(op), out_k, nthreads)
    if rc != 0:
        raise ValueError("vdxo_sample_batch rejected its arguments")
    return tokens, flags, oi, op


def matvec_q4_0(weights: np.ndarray, x: np.ndarray, nthreads: int = 1) -> np.ndarray:
    """Unembedding as shaders/matvec_q4_0.comp computes it: ``weights`` is [out_dim,
    in_dim / 32 * 18] uint8 (Q4_0 blocks, row-major), ``x`` is [batch, in_dim] float32;
    returns [batch, out_dim] float32."""
    w = np.ascontiguousarray(weights, np.uint8)
    xx = np.ascontiguousarray(np.atleast_2d(x), np.float32)
    batch, in_dim = xx.shape
    out_dim = w.shape[0]
    assert w.shape[1] == in_dim // 32 * 18 and in_dim % 32 == 0
    out = np.empty((batch, out_dim), np.float32)
    rc = lib().vdxo_matvec_q4_0(_ptr(w), _ptr(xx), batch, in_dim, out_dim, _ptr(out), nthreads)
    if rc != 0:
        raise ValueError("vdxo_matvec_q4_0: bad arguments")
    return out
