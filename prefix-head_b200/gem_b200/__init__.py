"""Python mirror of gem's model/head API over the C ABI of include/gem.h (libgem_b200.so).

Names follow crates/gem: `Gemma` (model.rs: load / forward), the full head and the two-level head
(main.rs: Full::run + logprob, TwoLevel::load + logprob) and the `bench`/`check` scoring loop. Every
call runs the sm_100a kernels of the shared library; there is no CPU path. If the library is missing
and cannot be built, importing a model raises.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess
from pathlib import Path

import numpy as np

PKG = Path(__file__).resolve().parents[1]          # prefix-head_b200/
LIB = PKG / "_build" / "libgem_b200.so"
SOURCES = [PKG / "csrc" / f for f in ("kernels.cu", "kernels_exact.cu", "pipeline.cu", "seq.cu", "decode.cu", "tc_gemm.cu",
                                      "noalloc.cu", "exact.cuh", "pipeline.cuh", "common.cuh", "kernels.cuh",
                                      "internal.hpp", "host.cpp", "host.hpp", "runtime.cpp")]

GEM_OK = 0
STATUS = {-1: "GEM_E_ARG", -2: "GEM_E_IO", -3: "GEM_E_FORMAT", -4: "GEM_E_CUDA", -5: "GEM_E_NOMEM",
          -6: "GEM_E_STATE", -7: "GEM_E_RANGE", -8: "GEM_E_NCCL", -9: "GEM_E_TIMEOUT"}


class GemError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"{STATUS.get(code, code)}: {msg}")
        self.code = code


class Info(C.Structure):
    _fields_ = [(n, C.c_int64) for n in ("d", "vocab", "layers", "n_heads", "n_kv_heads", "head_dim", "ffn", "ctx",
                                         "window", "bos", "body_bits", "head_bits", "classes", "per", "max_seqs",
                                         "body_bytes", "head_bytes", "device", "kernels_per_token_full",
                                         "kernels_per_token_twolevel")]


def build(force: bool = False) -> Path:
    """Compiles the CUDA kernels (sm_100a) and the host runtime into prefix-head_b200/_build."""
    if force or not LIB.exists() or any(s.stat().st_mtime > LIB.stat().st_mtime for s in SOURCES if s.exists()):
        subprocess.run(["make", "-s", "-C", str(PKG)], check=True)
    return LIB


_lib = None
_u32p = C.POINTER(C.c_uint32)
_f32p = C.POINTER(C.c_float)


def lib():
    global _lib
    if _lib is not None:
        return _lib
    if not LIB.exists():
        build()
    L = C.CDLL(str(LIB))
    vp = C.c_void_p
    L.gem_last_error.restype = C.c_char_p
    L.gem_version.restype = C.c_int
    L.gem_open.argtypes = [C.c_char_p, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, C.POINTER(vp)]
    L.gem_open_twolevel.argtypes = [vp, C.c_char_p]
    L.gem_close.argtypes = [vp]
    L.gem_close.restype = None
    L.gem_get_info.argtypes = [vp, C.POINTER(Info)]
    L.gem_reset.argtypes = [vp, C.c_int]
    L.gem_sync.argtypes = [vp]
    L.gem_get_stream.argtypes = [vp, C.POINTER(vp)]
    L.gem_set_schedule.argtypes = [vp, C.c_int]
    L.gem_set_tensor_cores.argtypes = [vp, C.c_int]
    L.gem_test_withhold_stage.argtypes = [vp, C.c_int, C.c_int]
    L.gem_set_profiling.argtypes = [vp, C.c_int]
    L.gem_get_phase_profile.argtypes = [vp, C.POINTER(C.c_double), C.c_int, C.POINTER(C.c_double), C.c_int]
    L.gem_get_schedule.argtypes = [vp, C.c_int, C.POINTER(C.c_int), C.POINTER(C.c_int)]
    L.gem_get_schedule_kind.argtypes = [vp, C.c_int, C.POINTER(C.c_int)]
    L.gem_get_parallel_profile.argtypes = [vp, C.POINTER(C.c_double), C.c_int]
    L.gem_get_last_launches.argtypes = [vp, C.POINTER(C.c_int64)]
    L.gem_set_numerics.argtypes = [vp, C.c_int, C.c_int]
    L.gem_forward.argtypes = [vp, C.c_uint32, C.c_uint32, _f32p]
    L.gem_full_logprob.argtypes = [vp, C.c_uint32, _f32p, _u32p]
    L.gem_twolevel_logprob.argtypes = [vp, C.c_uint32, _f32p, _u32p]
    L.gem_score.argtypes = [vp, _u32p, C.c_size_t, C.c_int, _f32p, _u32p]
    L.gem_score_dev.argtypes = [vp, vp, C.c_size_t, C.c_int, vp, vp]
    L.gem_score_batch.argtypes = [vp, _u32p, C.c_size_t, C.c_size_t, C.c_int, _f32p, _u32p]
    L.gem_nccl_unique_id.argtypes = [C.c_char_p]
    L.gem_greedy.argtypes = [vp, C.c_int, C.c_float, _u32p, C.c_int, _u32p, C.POINTER(C.c_int)]
    L.gem_twolevel_sample.argtypes = [vp, C.c_float, C.POINTER(C.c_uint64), _u32p]
    L.gem_greedy_dev.argtypes = [vp, vp, C.c_int, C.c_int, C.c_float, vp, C.c_int, vp, vp]
    L.gem_generate.argtypes = [vp, _u32p, C.c_size_t, C.c_size_t, C.POINTER(GenOpts), _u32p, C.POINTER(C.c_size_t)]
    L.gem_shard_init.argtypes = [vp, C.c_int, C.c_int, C.c_char_p]
    L.gem_score_batch_dev.argtypes = [vp, vp, C.c_size_t, C.c_size_t, C.c_int, vp, vp]
    L.gem_matvec_dev.argtypes = [vp, C.c_int, C.c_int, vp, vp]
    L.gem_head_full_dev.argtypes = [vp, vp, vp, C.c_int, vp, vp]
    L.gem_head_twolevel_dev.argtypes = [vp, vp, vp, C.c_int, vp, vp]
    L.gem_head_full_noalloc.argtypes = [vp, vp, vp, C.c_int, vp, vp]
    _lib = L
    return L


def _check(rc: int):
    if rc != GEM_OK:
        raise GemError(rc, lib().gem_last_error().decode())


def _p(a: np.ndarray, t):
    return a.ctypes.data_as(t)


class GenOpts(C.Structure):
    _fields_ = [("mode", C.c_int), ("top", C.c_int), ("min_confidence", C.c_float), ("always", C.POINTER(C.c_uint32)),
                ("n_always", C.c_int), ("temperature", C.c_float), ("seed", C.c_uint64), ("stops", C.POINTER(C.c_uint32)),
                ("n_stops", C.c_int)]


GREEDY_FULL, GREEDY_SCREEN, SAMPLE = 0, 1, 2
NCCL_UNIQUE_ID_BYTES = 128


def nccl_unique_id() -> bytes:
    """A fresh NCCL communicator id (one rank makes it; every rank passes it to Gemma.shard)."""
    buf = C.create_string_buffer(NCCL_UNIQUE_ID_BYTES)
    _check(lib().gem_nccl_unique_id(buf))
    return buf.raw


FULL, TWO_LEVEL = 0, 1
EXACT, FAST = 0, 1
AUTO, SEQUENTIAL, PIPELINED, PARALLEL = 0, 1, 2, 3
SCHEDULE_NAMES = {SEQUENTIAL: "sequential", PIPELINED: "pipelined", PARALLEL: "parallel"}


class Gemma:
    """Gemma::load + requantize + requantize_head (model.rs:154-279, main.rs:203-210) on one GPU."""

    def __init__(self, gguf: str | os.PathLike, ctx: int = 2048, body_bits: int = 8, head_bits: int = 0,
                 device: int = 0, max_seqs: int = 1):
        L = lib()
        h = C.c_void_p()
        _check(L.gem_open(str(gguf).encode(), ctx, body_bits, head_bits, device, max_seqs, C.byref(h)))
        self._h = h
        info = Info()
        _check(L.gem_get_info(self._h, C.byref(info)))
        self.info = {n: int(getattr(info, n)) for n, _ in Info._fields_}
        self.d, self.vocab, self.ctx, self.bos = (self.info[k] for k in ("d", "vocab", "ctx", "bos"))

    def close(self):
        if getattr(self, "_h", None):
            lib().gem_close(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def __enter__(self):
        return self

    def __exit__(self, *a):
        self.close()

    @property
    def handle(self):
        return self._h

    def load_twolevel(self, prefix: str | os.PathLike):
        """TwoLevel::load (main.rs:57-76)."""
        _check(lib().gem_open_twolevel(self._h, str(prefix).encode()))
        info = Info()
        _check(lib().gem_get_info(self._h, C.byref(info)))
        self.info = {n: int(getattr(info, n)) for n, _ in Info._fields_}

    def set_numerics(self, mode: int = EXACT, ref_threads: int = 8):
        """EXACT: bit-identical to the reference's AVX-512 path with a pool of ref_threads threads.
        FAST: tree reductions (within the reference's own cross-ISA spread)."""
        _check(lib().gem_set_numerics(self._h, mode, ref_threads))

    def set_tensor_cores(self, on: bool = True):
        """The parallel schedule's body products on the tensor cores (bit-identical to the CUDA cores)."""
        _check(lib().gem_set_tensor_cores(self._h, 1 if on else 0))

    def set_schedule(self, schedule: int = AUTO):
        """SEQUENTIAL: a CUDA graph per token. PIPELINED: two-level scoring as one layer-pipelined kernel.
        PARALLEL: every position of a chunk through each layer together. AUTO: the fastest supported."""
        _check(lib().gem_set_schedule(self._h, schedule))

    def schedule_kind(self, head: int = TWO_LEVEL):
        """(schedule that scoring with `head` runs, its name or why a faster one is not used)."""
        k = C.c_int()
        _check(lib().gem_get_schedule_kind(self._h, head, C.byref(k)))
        return k.value, lib().gem_last_error().decode()

    def schedule(self, head: int = TWO_LEVEL):
        """(pipelined, ctas per layer stage, head ctas, reason)."""
        p = C.c_int()
        sc = (C.c_int * 2)()
        _check(lib().gem_get_schedule(self._h, head, C.byref(p), sc))
        return bool(p.value), sc[0], sc[1], lib().gem_last_error().decode()

    def greedy(self, top: int = 1, min_confidence: float = 0.0, always=()):
        """lean.rs Classes::next + next_token on the last hidden state -> (token, fell_back)."""
        al = np.ascontiguousarray(np.asarray(always, np.uint32))
        tok, fb = C.c_uint32(), C.c_int()
        _check(lib().gem_greedy(self._h, top, min_confidence, _p(al, _u32p), len(al), C.byref(tok), C.byref(fb)))
        return tok.value, bool(fb.value)

    def sample(self, temperature: float, rng: int):
        """TwoLevel::sample on the last hidden state -> (token, new rng state)."""
        st, tok = C.c_uint64(rng), C.c_uint32()
        _check(lib().gem_twolevel_sample(self._h, temperature, C.byref(st), C.byref(tok)))
        return tok.value, st.value

    def greedy_dev(self, h_ptr: int, batch: int, top: int, min_confidence: float, always_ptr: int, n_always: int,
                   tok_ptr: int, fb_ptr: int | None):
        _check(lib().gem_greedy_dev(self._h, h_ptr, batch, top, min_confidence, always_ptr, n_always, tok_ptr, fb_ptr))

    def generate(self, prompt, max_new: int, mode: int = GREEDY_FULL, top: int = 1, min_confidence: float = 0.0,
                 always=(), temperature: float = 1.0, seed: int = 1, stops=()):
        """The completion loop: prompt, then up to max_new tokens (a stop token ends it, not emitted)."""
        prompt = np.ascontiguousarray(prompt, np.uint32)
        al = np.ascontiguousarray(np.asarray(always, np.uint32))
        sp = np.ascontiguousarray(np.asarray(stops, np.uint32))
        o = GenOpts(mode, top, min_confidence, _p(al, _u32p), len(al), temperature, seed, _p(sp, _u32p), len(sp))
        out = np.zeros(max(1, max_new), np.uint32)
        n = C.c_size_t()
        _check(lib().gem_generate(self._h, _p(prompt, _u32p), len(prompt), max_new, C.byref(o), _p(out, _u32p), C.byref(n)))
        return out[:n.value]

    def shard(self, nranks: int, rank: int, uid: bytes):
        """Vocab-shard the full head: this rank scores output rows [rank*ceil(V/n), ...) and the ranks
        merge their partial statistics over NCCL (the body stays replicated)."""
        if len(uid) != NCCL_UNIQUE_ID_BYTES:
            raise ValueError("uid must be the 128 bytes of nccl_unique_id()")
        _check(lib().gem_shard_init(self._h, nranks, rank, uid))

    def test_withhold_stage(self, stage: int, wait_ms: int = 2000):
        """Failure-detection hook: layer stage `stage` withholds its output (-1 restores normal runs)."""
        _check(lib().gem_test_withhold_stage(self._h, stage, wait_ms))

    LAYER_PHASES = ["wait", "attn_norm", "qkv", "bar1", "qknorm+scores", "bar2", "softmax+pv", "bar3", "combine+o",
                    "bar4", "norms", "gate_up", "bar5", "down", "bar6", "handoff"]
    HEAD_PHASES = ["wait", "norm+classes+block", "bar1", "select+top_block", "bar2", "argmax"]

    def set_profiling(self, on: bool = True):
        _check(lib().gem_set_profiling(self._h, 1 if on else 0))

    def phase_profile(self):
        """Mean us per token per phase of pipelined scoring: (layer stages, head stage)."""
        la = (C.c_double * 16)()
        ha = (C.c_double * 6)()
        _check(lib().gem_get_phase_profile(self._h, la, 16, ha, 6))
        return dict(zip(self.LAYER_PHASES, [round(v, 3) for v in la])), dict(zip(self.HEAD_PHASES, [round(v, 3) for v in ha]))

    PARALLEL_GROUPS = ["embed", "norm", "qkv", "attention", "o", "gate_up", "gate", "down", "head", "combine"]

    def parallel_profile(self):
        """Mean device us per scoring call in each launch group of parallel scoring (profiling on)."""
        n = len(self.PARALLEL_GROUPS)
        a = (C.c_double * n)()
        _check(lib().gem_get_parallel_profile(self._h, a, n))
        return dict(zip(self.PARALLEL_GROUPS, [round(v, 2) for v in a]))

    def last_launches(self) -> int:
        """Kernels launched by the last scoring call."""
        n = C.c_int64()
        _check(lib().gem_get_last_launches(self._h, C.byref(n)))
        return n.value

    def reset(self, seq: int = 0):
        _check(lib().gem_reset(self._h, seq))

    def forward(self, tok: int, pos: int) -> np.ndarray:
        """Gemma::forward (model.rs:286-430); returns the final-norm hidden state."""
        h = np.zeros(self.d, np.float32)
        _check(lib().gem_forward(self._h, tok, pos, _p(h, _f32p)))
        return h

    def full_logprob(self, target: int):
        """Full::run + Full::logprob (main.rs:30-37) on the last forward's hidden state."""
        lp, am = C.c_float(), C.c_uint32()
        _check(lib().gem_full_logprob(self._h, target, C.byref(lp), C.byref(am)))
        return lp.value, am.value

    def twolevel_logprob(self, target: int):
        """TwoLevel::logprob (main.rs:101-107) on the last forward's hidden state."""
        lp, am = C.c_float(), C.c_uint32()
        _check(lib().gem_twolevel_logprob(self._h, target, C.byref(lp), C.byref(am)))
        return lp.value, am.value

    def score(self, toks: np.ndarray, head: int = TWO_LEVEL):
        """The bench/check loop (main.rs:270-289): len(toks) - 1 scored tokens -> (logprob, argmax)."""
        toks = np.ascontiguousarray(toks, np.uint32)
        n = len(toks) - 1
        lp = np.zeros(n, np.float32)
        am = np.zeros(n, np.uint32)
        _check(lib().gem_score(self._h, _p(toks, _u32p), n, head, _p(lp, _f32p), _p(am, _u32p)))
        return lp, am

    def score_dev(self, toks_ptr: int, n: int, head: int, lp_ptr: int, am_ptr: int | None):
        """Same loop on device buffers (ints: device addresses); asynchronous on the model's stream."""
        _check(lib().gem_score_dev(self._h, toks_ptr, n, head, lp_ptr, am_ptr))

    def score_batch(self, toks: np.ndarray, head: int = TWO_LEVEL):
        """Batched scoring: toks [nseq][len + 1] -> (logprob, argmax), each [nseq][len]."""
        toks = np.ascontiguousarray(toks, np.uint32)
        nseq, n = toks.shape[0], toks.shape[1] - 1
        lp = np.zeros((nseq, n), np.float32)
        am = np.zeros((nseq, n), np.uint32)
        _check(lib().gem_score_batch(self._h, _p(toks, _u32p), nseq, n, head, _p(lp, _f32p), _p(am, _u32p)))
        return lp, am

    def score_batch_dev(self, toks_ptr: int, nseq: int, n: int, head: int, lp_ptr: int, am_ptr: int | None):
        """Batched scoring on device buffers (toks [nseq][n + 1], outputs [nseq][n]); asynchronous."""
        _check(lib().gem_score_batch_dev(self._h, toks_ptr, nseq, n, head, lp_ptr, am_ptr))

    def refresh_info(self):
        info = Info()
        _check(lib().gem_get_info(self._h, C.byref(info)))
        self.info = {n: int(getattr(info, n)) for n, _ in Info._fields_}
        return self.info

    @property
    def stream(self) -> int:
        """The model's cudaStream_t as an integer (for torch.cuda.ExternalStream)."""
        s = C.c_void_p()
        _check(lib().gem_get_stream(self._h, C.byref(s)))
        return int(s.value or 0)

    def sync(self):
        _check(lib().gem_sync(self._h))

    def matvec_dev(self, layer: int, which: int, x_ptr: int, y_ptr: int):
        _check(lib().gem_matvec_dev(self._h, layer, which, x_ptr, y_ptr))

    def head_full_dev(self, h_ptr: int, targets_ptr: int, batch: int, lp_ptr: int, am_ptr: int, sync: bool = True):
        """Full head on device buffers; the C call is stream-ordered, `sync` waits for the results."""
        _check(lib().gem_head_full_dev(self._h, h_ptr, targets_ptr, batch, lp_ptr, am_ptr))
        if sync:
            self.sync()

    def head_twolevel_dev(self, h_ptr: int, targets_ptr: int, batch: int, lp_ptr: int, am_ptr: int, sync: bool = True):
        """Two-level head on device buffers; stream-ordered like head_full_dev."""
        _check(lib().gem_head_twolevel_dev(self._h, h_ptr, targets_ptr, batch, lp_ptr, am_ptr))
        if sync:
            self.sync()

    def head_full_noalloc(self, h_ptr: int, targets_ptr: int, batch: int, lp_ptr: int, am_ptr: int):
        """gem_head_full_dev without any device allocation (static scratch; asynchronous)."""
        _check(lib().gem_head_full_noalloc(self._h, h_ptr, targets_ptr, batch, lp_ptr, am_ptr))
