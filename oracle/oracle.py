"""TEST INFRASTRUCTURE ONLY — ctypes binding of the oracle library (oracle/gem_oracle.cpp), the CPU
restatement of the reference's scoring path. Used by tests/, __graft_entry__.smoke() and bench.py's
CPU-baseline leg as the checker or the timed CPU baseline; never by the product path."""
from __future__ import annotations

import ctypes as C
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB = HERE / "_build" / "libgem_oracle.so"

_f32p = C.POINTER(C.c_float)
_u32p = C.POINTER(C.c_uint32)
_i8p = C.POINTER(C.c_int8)
_u8p = C.POINTER(C.c_uint8)
_i64p = C.POINTER(C.c_int64)


def build() -> Path:
    subprocess.run(["make", "-s", "-C", str(HERE)], check=True)
    return LIB


_lib = None


def lib():
    global _lib
    if _lib is None:
        if not LIB.exists() or LIB.stat().st_mtime < (HERE / "gem_oracle.cpp").stat().st_mtime:
            build()
        L = C.CDLL(str(LIB))
        L.orc_last_error.restype = C.c_char_p
        L.orc_detect_isa.restype = C.c_char_p
        L.orc_open.restype = C.c_void_p
        L.orc_open.argtypes = [C.c_char_p, C.c_int, C.c_int, C.c_int, C.c_int, C.c_char_p]
        L.orc_close.argtypes = [C.c_void_p]
        L.orc_info.argtypes = [C.c_void_p, _i64p]
        L.orc_isa.restype = C.c_char_p
        L.orc_isa.argtypes = [C.c_void_p]
        L.orc_forward.argtypes = [C.c_void_p, C.c_uint32, C.c_uint32, _f32p]
        L.orc_full.argtypes = [C.c_void_p, _f32p, C.c_uint32, _f32p, _u32p, _f32p]
        L.orc_twolevel_load.argtypes = [C.c_void_p, C.c_char_p]
        L.orc_twolevel.argtypes = [C.c_void_p, _f32p, C.c_uint32, _f32p, _u32p, _f32p, _f32p]
        L.orc_greedy.argtypes = [C.c_void_p, _f32p, C.c_int, C.c_float, _u32p, C.c_int, _u32p, C.POINTER(C.c_int)]
        L.orc_twolevel_sample.argtypes = [C.c_void_p, _f32p, C.c_float, C.POINTER(C.c_uint64), _u32p]
        L.orc_score.argtypes = [C.c_void_p, _u32p, C.c_size_t, C.c_int, _f32p, _u32p,
                                C.POINTER(C.c_double), C.POINTER(C.c_double)]
        L.orc_mat_from_gguf.restype = C.c_void_p
        L.orc_mat_from_gguf.argtypes = [C.c_int, _u8p, C.c_size_t, C.c_size_t]
        L.orc_mat_free.argtypes = [C.c_void_p]
        L.orc_mat_requant.restype = C.c_void_p
        L.orc_mat_requant.argtypes = [C.c_void_p, C.c_int]
        L.orc_mat_info.argtypes = [C.c_void_p, _i64p]
        L.orc_mat_planes.argtypes = [C.c_void_p, _i8p, _f32p]
        L.orc_mat_dequant.argtypes = [C.c_void_p, _f32p]
        L.orc_matvec.argtypes = [C.c_void_p, _f32p, C.c_char_p, C.c_int, _f32p]
        L.orc_quantize.argtypes = [_f32p, C.c_size_t, C.c_char_p, _i8p, _f32p]
        L.orc_exp_fast.restype = C.c_float
        L.orc_exp_fast.argtypes = [C.c_float]
        L.orc_tanh_fast.restype = C.c_float
        L.orc_tanh_fast.argtypes = [C.c_float]
        L.orc_lse.restype = C.c_float
        L.orc_lse.argtypes = [_f32p, C.c_size_t]
        L.orc_f16.restype = C.c_float
        L.orc_f16.argtypes = [C.c_uint16]
        _lib = L
    return _lib


def _p(a: np.ndarray, t):
    return a.ctypes.data_as(t)


def _isa(isa):
    return None if isa is None else isa.encode()


def detect_isa() -> str:
    return lib().orc_detect_isa().decode()


class OracleError(RuntimeError):
    pass


def _check(rc):
    if rc != 0:
        raise OracleError(lib().orc_last_error().decode())


class Model:
    """Gemma::load + Full + TwoLevel of the reference, on the CPU."""

    def __init__(self, gguf: str | os.PathLike, ctx: int = 2048, body_bits: int = 8, head_bits: int = 0,
                 threads: int = 8, isa: str | None = None):
        L = lib()
        self.h = L.orc_open(str(gguf).encode(), ctx, body_bits, head_bits, threads, _isa(isa))
        if not self.h:
            raise OracleError(L.orc_last_error().decode())
        info = np.zeros(5, np.int64)
        L.orc_info(self.h, _p(info, _i64p))
        self.d, self.vocab, self.layers, self.ctx, self.bos = (int(v) for v in info)
        self.isa = L.orc_isa(self.h).decode()

    def close(self):
        if self.h:
            lib().orc_close(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def forward(self, tok: int, pos: int) -> np.ndarray:
        h = np.zeros(self.d, np.float32)
        _check(lib().orc_forward(self.h, tok, pos, _p(h, _f32p)))
        return h

    def full(self, h: np.ndarray, target: int, logits: bool = False):
        h = np.ascontiguousarray(h, np.float32)
        lp = np.zeros(1, np.float32)
        am = np.zeros(1, np.uint32)
        lg = np.zeros(self.vocab, np.float32) if logits else None
        _check(lib().orc_full(self.h, _p(h, _f32p), target, _p(lp, _f32p), _p(am, _u32p),
                              _p(lg, _f32p) if logits else None))
        return (float(lp[0]), int(am[0]), lg) if logits else (float(lp[0]), int(am[0]))

    def load_twolevel(self, prefix):
        _check(lib().orc_twolevel_load(self.h, str(prefix).encode()))

    def greedy(self, h: np.ndarray, top: int = 1, min_confidence: float = 0.0, always=()):
        """lean.rs Classes::next + next_token -> (token, fell_back)."""
        h = np.ascontiguousarray(h, np.float32)
        al = np.ascontiguousarray(np.asarray(always, np.uint32))
        tok, fb = C.c_uint32(), C.c_int()
        _check(lib().orc_greedy(self.h, _p(h, _f32p), top, min_confidence, _p(al, _u32p), len(al), C.byref(tok), C.byref(fb)))
        return tok.value, bool(fb.value)

    def sample(self, h: np.ndarray, temp: float, rng: int):
        """TwoLevel::sample -> (token, new rng state)."""
        h = np.ascontiguousarray(h, np.float32)
        st, tok = C.c_uint64(rng), C.c_uint32()
        _check(lib().orc_twolevel_sample(self.h, _p(h, _f32p), temp, C.byref(st), C.byref(tok)))
        return tok.value, st.value

    def twolevel(self, h: np.ndarray, target: int):
        h = np.ascontiguousarray(h, np.float32)
        lp = np.zeros(1, np.float32)
        am = np.zeros(1, np.uint32)
        _check(lib().orc_twolevel(self.h, _p(h, _f32p), target, _p(lp, _f32p), _p(am, _u32p), None, None))
        return float(lp[0]), int(am[0])

    def score(self, toks: np.ndarray, head: int):
        """gem bench's loop: len(toks) - 1 scored tokens. Returns (logprob, argmax, body_s, head_s)."""
        toks = np.ascontiguousarray(toks, np.uint32)
        n = len(toks) - 1
        lp = np.zeros(n, np.float32)
        am = np.zeros(n, np.uint32)
        tb, th = C.c_double(0), C.c_double(0)
        _check(lib().orc_score(self.h, _p(toks, _u32p), n, head, _p(lp, _f32p), _p(am, _u32p),
                               C.byref(tb), C.byref(th)))
        return lp, am, tb.value, th.value


class Mat:
    """q8.rs `Mat` built from GGUF tensor bytes (kind 8 Q8_0, 2 Q4_0, 1 F16)."""

    def __init__(self, kind: int, raw: np.ndarray, rows: int, cols: int, _h=None):
        L = lib()
        if _h is None:
            raw = np.ascontiguousarray(raw, np.uint8)
            _h = L.orc_mat_from_gguf(kind, _p(raw, _u8p), rows, cols)
            if not _h:
                raise OracleError(L.orc_last_error().decode())
        self.h = _h
        info = np.zeros(5, np.int64)
        L.orc_mat_info(self.h, _p(info, _i64p))
        self.bits, self.rows, self.cols, self.qbytes, self.nscales = (int(v) for v in info)

    def __del__(self):
        if getattr(self, "h", None):
            lib().orc_mat_free(self.h)
            self.h = None

    def requant(self, bits: int) -> "Mat":
        h = lib().orc_mat_requant(self.h, bits)
        if not h:
            raise OracleError(lib().orc_last_error().decode())
        return Mat(0, None, 0, 0, _h=h)

    def planes(self):
        q = np.zeros(self.qbytes, np.int8)
        s = np.zeros(self.nscales, np.float32)
        lib().orc_mat_planes(self.h, _p(q, _i8p), _p(s, _f32p))
        return q, s

    def dequant(self) -> np.ndarray:
        out = np.zeros((self.rows, self.cols), np.float32)
        lib().orc_mat_dequant(self.h, _p(out, _f32p))
        return out

    def matvec(self, x: np.ndarray, isa: str | None = None, threads: int = 1) -> np.ndarray:
        x = np.ascontiguousarray(x, np.float32)
        y = np.zeros(self.rows, np.float32)
        _check(lib().orc_matvec(self.h, _p(x, _f32p), _isa(isa), threads, _p(y, _f32p)))
        return y


def quantize(x: np.ndarray, isa: str | None = None):
    x = np.ascontiguousarray(x, np.float32)
    q = np.zeros(len(x), np.int8)
    s = np.zeros(len(x) // 32, np.float32)
    _check(lib().orc_quantize(_p(x, _f32p), len(x), _isa(isa), _p(q, _i8p), _p(s, _f32p)))
    return q, s


def exp_fast(x: float) -> float:
    return lib().orc_exp_fast(x)


def tanh_fast(x: float) -> float:
    return lib().orc_tanh_fast(x)


def lse(v: np.ndarray) -> float:
    v = np.ascontiguousarray(v, np.float32)
    return lib().orc_lse(_p(v, _f32p), len(v))


def f16(h: int) -> float:
    return lib().orc_f16(h)
