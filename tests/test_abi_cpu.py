"""CPU-only checks of the C ABI: the library builds for sm_100a, loads without a GPU,
and exports every entry point include/squirrel_cuda.h declares. No compute calls."""
import ctypes
import os
import re

from conftest import ROOT

HEADER = os.path.join(ROOT, "include", "squirrel_cuda.h")


def declared_symbols():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(sq_[a-z0-9_]+)\s*\(", text)))


def test_header_declares_entry_points():
    syms = declared_symbols()
    for s in ("sq_linear", "sq_linear_shared", "sq_embed", "sq_rms_norm", "sq_rope_rows", "sq_sdpa_cached",
              "sq_quantize_row_q8_0", "sq_argmax", "sq_model_load_gguf", "sq_forward", "sq_generate"):
        assert s in syms


def test_library_exports_every_declared_symbol():
    from sqb200 import lib
    L = lib.load()
    missing = [s for s in declared_symbols() if not hasattr(L, s)]
    assert not missing, missing
    assert b"sm_100a" in L.sq_version()


def test_python_binding_covers_header():
    from sqb200 import lib
    assert set(declared_symbols()) <= set(lib.SIGNATURES)


def test_last_error_empty_before_failures():
    from sqb200 import lib
    L = lib.load()
    assert isinstance(L.sq_last_error(), bytes)


def test_host_validation_without_gpu():
    """Shape checks run on the host before any launch, with KernelError kinds."""
    from sqb200 import lib
    L = lib.load()
    # in_dim not a multiple of 32 -> ShapeMismatch (matmul.rs:16-18); pointers are never touched
    st = L.sq_linear(None, ctypes.c_void_p(16), 1, 40, ctypes.c_void_p(16), lib.Q8_0, 2, ctypes.c_void_p(16), 0)
    assert st == 1
    st = L.sq_linear(None, ctypes.c_void_p(16), 1, 64, ctypes.c_void_p(16), 1, 2, ctypes.c_void_p(16), 0)
    assert st == 2  # F16 weights: InvalidType (linear.rs:35)
    st = L.sq_sdpa_cached(None, ctypes.c_void_p(16), ctypes.c_void_p(16), ctypes.c_void_p(16), ctypes.c_void_p(16),
                          1, 1, 3, 2, 32)
    assert st == 1  # attention.rs:22-24
    st = L.sq_argmax(None, ctypes.c_void_p(16), 0, ctypes.c_void_p(16))
    assert st == 3  # empty input
