"""GGUF container edge cases (crates/gem/src/gguf.rs:59-143) on CPU: the header is read in 4 MiB
chunks until it parses, so headers larger than one chunk load; a truncated header, a wrong magic, an
unsupported version or architecture are errors, not crashes; general.alignment moves the tensor data.
gem_open parses and validates before any CUDA call, so on a machine without a GPU a well-formed file
gets past parsing and fails only at device setup (GEM_E_CUDA), which separates the two outcomes."""
import shutil
import struct

import numpy as np
import pytest

from gem_b200 import Gemma, GemError, synth
from oracle import oracle as orc

GEM_E_IO, GEM_E_FORMAT, GEM_E_CUDA = -2, -3, -4


def _has_gpu():
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False


def _open_code(path):
    try:
        Gemma(path, ctx=64).close()
        return 0
    except GemError as e:
        return e.code


def _parses(path):
    return _open_code(path) in ((0,) if _has_gpu() else (GEM_E_CUDA,))


def test_truncated_header_is_an_io_error(small, tmp_path):
    p = tmp_path / "cut.gguf"
    p.write_bytes(small.gguf.read_bytes()[:300])
    assert _open_code(p) == GEM_E_IO


def test_bad_magic_and_version(small, tmp_path):
    b = bytearray(small.gguf.read_bytes())
    p = tmp_path / "magic.gguf"
    p.write_bytes(b"GGML" + bytes(b[4:]))
    assert _open_code(p) == GEM_E_FORMAT
    v = bytearray(b)
    v[4:8] = struct.pack("<I", 99)
    p2 = tmp_path / "version.gguf"
    p2.write_bytes(bytes(v))
    assert _open_code(p2) == GEM_E_FORMAT


def test_unsupported_architecture(tmp_path):
    cfg = dict(synth.CONFIGS["small"], arch="llama")
    p = synth.write_model(tmp_path / "llama.gguf", cfg, seed=3)
    assert _open_code(p) == GEM_E_FORMAT


def test_header_larger_than_one_read_chunk(tmp_path):
    """A 262144-entry token list makes a ~10 MiB header: three 4 MiB reads before it parses."""
    cfg = dict(synth.CONFIGS["small"], vocab=262144, layers=1)
    p = synth.write_model(tmp_path / "bigheader.gguf", cfg, seed=4, vocab_strings=True)
    assert p.stat().st_size > (8 << 20)
    assert _parses(p)
    o = orc.Model(p, ctx=32, threads=1)  # the oracle follows the same retry (gguf.rs:93-107)
    assert o.vocab == 262144


def test_alignment_moves_tensor_data_not_results(small, tmp_path):
    cfg = synth.CONFIGS["small"]
    p64 = synth.write_model(tmp_path / "a64.gguf", cfg, seed=1, alignment=64)
    assert _parses(p64)
    toks = synth.tokens(20, cfg["vocab"], seed=5)
    a = orc.Model(small.gguf, ctx=32, threads=2).score(toks, 0)[0]
    b = orc.Model(p64, ctx=32, threads=2).score(toks, 0)[0]
    assert np.array_equal(a, b)  # same seed, same weights: only the data offsets differ


@pytest.mark.gpu
def test_tensor_offset_that_wraps_is_an_io_error(small, tmp_path):
    """A crafted tensor offset chosen so that data start + offset wraps around 2^64 to the start of
    the file: the bounds check works in checked arithmetic and rejects it (GEM_E_IO) instead of
    reading the header's bytes as weights. Tensors are read after device setup, hence a GPU test."""
    if not _has_gpu():
        pytest.skip("no CUDA device")
    import gguf
    base = gguf.GGUFReader(str(small.gguf)).data_offset
    b = bytearray(small.gguf.read_bytes())
    name = b"token_embd.weight"
    i = b.index(name) + len(name)
    nd = struct.unpack_from("<I", b, i)[0]
    struct.pack_into("<Q", b, i + 4 + 8 * nd + 4, (1 << 64) - base)
    p = tmp_path / "wrap.gguf"
    p.write_bytes(bytes(b))
    assert _open_code(p) == GEM_E_IO
