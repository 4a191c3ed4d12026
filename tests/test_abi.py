"""The C-ABI library loads and exports every entry point include/gem.h declares; host-side validation
fails with the documented status codes before any device work (no GPU needed)."""
import ctypes as C
import re
from pathlib import Path

import numpy as np
import pytest

import gem_b200
from gem_b200 import synth

ROOT = Path(__file__).resolve().parents[1]


def declared():
    text = (ROOT / "include" / "gem.h").read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(gem_[a-z0-9_]+)\s*\(", text)))


def test_header_declares_entry_points():
    names = declared()
    for n in ("gem_open", "gem_open_twolevel", "gem_forward", "gem_full_logprob", "gem_twolevel_logprob",
              "gem_score", "gem_score_dev", "gem_matvec_dev", "gem_head_full_dev", "gem_head_twolevel_dev"):
        assert n in names


def test_library_exports_every_declared_symbol():
    gem_b200.build()
    lib = C.CDLL(str(gem_b200.LIB))
    missing = [n for n in declared() if not hasattr(lib, n)]
    assert not missing, missing


def test_library_targets_sm100a():
    out = gem_b200.LIB.read_bytes()
    assert b"sm_100a" in out


def _open_status(path, **kw):
    L = gem_b200.lib()
    h = C.c_void_p()
    args = dict(ctx=64, body_bits=8, head_bits=0, device=0, max_seqs=1)
    args.update(kw)
    rc = L.gem_open(str(path).encode(), args["ctx"], args["body_bits"], args["head_bits"], args["device"],
                    args["max_seqs"], C.byref(h))
    return rc, L.gem_last_error().decode()


def test_missing_file_is_io_error(tmp_path):
    rc, msg = _open_status(tmp_path / "nope.gguf")
    assert rc == -2 and "cannot open" in msg


def test_not_gguf_is_format_error(tmp_path):
    p = tmp_path / "x.gguf"
    p.write_bytes(b"NOTGGUF" * 100)
    rc, msg = _open_status(p)
    assert rc == -3 and "not a GGUF" in msg


def test_truncated_header_is_io_error(tmp_path, small):
    p = tmp_path / "t.gguf"
    p.write_bytes(small.gguf.read_bytes()[:200])
    rc, msg = _open_status(p)
    assert rc == -2 and "truncated" in msg


def test_bad_options_are_arg_errors(small):
    assert _open_status(small.gguf, body_bits=5)[0] == -1
    assert _open_status(small.gguf, head_bits=3)[0] == -1
    assert _open_status(small.gguf, max_seqs=0)[0] == -1
    assert _open_status(small.gguf, ctx=0)[0] == -1


def test_unsupported_architecture(tmp_path):
    gguf = pytest.importorskip("gguf")
    p = tmp_path / "llama.gguf"
    w = gguf.GGUFWriter(str(p), arch="llama")
    w.add_tensor("output_norm.weight", np.ones(32, np.float32))
    w.write_header_to_file(); w.write_kv_data_to_file(); w.write_tensors_to_file(); w.close()
    rc, msg = _open_status(p)
    assert rc == -3 and "architecture" in msg


def test_null_arguments():
    L = gem_b200.lib()
    assert L.gem_open(None, 64, 8, 0, 0, 1, None) == -1
    assert L.gem_forward(None, 0, 0, None) == -1
    assert L.gem_score(None, None, 0, 0, None, None) == -1


def test_rust_binding_declares_every_entry_point():
    """The reference-side binding a Rust host adds (the extern "C" blocks in INTEGRATION.md) names every
    function include/gem.h declares."""
    text = (ROOT / "INTEGRATION.md").read_text()
    missing = [n for n in declared() if f"fn {n}(" not in text]
    assert not missing, missing
