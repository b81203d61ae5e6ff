"""The C-ABI library loads (without a GPU) and exports every declared symbol."""

import ctypes
import glob
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
DECL = re.compile(r"^\s*(?:const\s+)?[A-Za-z_][\w\s\*]*?\b(sb_\w+)\s*\(", re.M)


def declared_symbols():
    names = set()
    for header in glob.glob(os.path.join(ROOT, "include", "*.h")):
        text = open(header).read()
        text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
        names.update(m.group(1) for m in DECL.finditer(text))
    return names


@pytest.fixture(scope="module")
def library():
    from spark_b200 import _lib

    if not os.path.exists(_lib.LIB_PATH):
        import __graft_entry__

        __graft_entry__.build()
    return ctypes.CDLL(_lib.LIB_PATH)


def test_headers_declare_the_expected_entry_points():
    names = declared_symbols()
    for required in ("sb_affine_linear", "sb_w8a16_per_channel", "sb_w8a8_linear", "sb_int8_matmul_int32",
                     "sb_qkv_rope", "sb_int8_sdpa_decode", "sb_quantize_per_token", "sb_linear_ex"):
        assert required in names


def test_library_exports_every_declared_symbol(library):
    missing = [n for n in sorted(declared_symbols()) if not hasattr(library, n)]
    assert not missing, missing


def test_python_binding_covers_every_symbol():
    from spark_b200 import _lib

    assert declared_symbols() == set(_lib.SIGNATURES)


def test_host_side_calls_without_gpu(library):
    from spark_b200 import _lib

    lib = _lib.lib()
    assert lib.sb_version() >= 100
    # size queries and argument validation run on the host only
    assert lib.sb_int8_sdpa_workspace_size(1, 32, 8, 32768, 128) > 0
    assert lib.sb_int8_sdpa_workspace_size(1, 32, 8, 32768, 64) == 0
    assert lib.sb_affine_linear(None, 0, None, None, None, None, 0, 1, 1, 64, 4, None, 0, None) == _lib.SB_EINVAL
    assert b"nonempty" in lib.sb_last_error_message()
    assert lib.sb_w8a8_linear(None, 0, None, None, None, 0, None, 1, 8, 33, None, 0, None) == _lib.SB_EINVAL
    assert b"multiple of 32" in lib.sb_last_error_message()


def test_affine_sdpa_workspace_covers_the_decode_splits(library):
    """Single-query decode over affine KV tuples plans up to 64 token splits
    (one wave of two CTAs per SM over the (batch, KV head) pairs, at least 64
    tokens each); each split's partial is head_dim + 4 floats per query head,
    after the 128 KiB counter region."""
    from spark_b200 import _lib

    lib = _lib.lib()
    counters = 128 * 1024
    for batch, heads, n, dv in ((1, 16, 32768, 256), (1, 16, 4096, 256), (2, 32, 5000, 128), (1, 8, 700, 128)):
        rows = batch * heads
        splits = min(64, max(1, n // 64), -(-296 // max(1, -(-rows // 8))))
        need = counters + rows * splits * (dv + 4) * 4 if splits > 1 else 0
        assert lib.sb_affine_sdpa_workspace_size(batch, heads, 1, n, dv) >= need
    assert lib.sb_affine_sdpa_workspace_size(1, 16, 1, 40, 256) == 0  # one split: no workspace


def test_windowed_prefill_rejects_bad_arguments(library):
    from spark_b200 import _lib

    lib = _lib.lib()
    args = [None] * 6 + [1, 16, 4, 8, 8, 16, 256, 0.0625]
    assert lib.sb_int8_sdpa_prefill_window(*args, 12, 1, None) == _lib.SB_EINVAL
    assert b"null pointer" in lib.sb_last_error_message()
    fake = [16, 16, 16, 16, 16, 16]  # never dereferenced: the window check comes first
    assert lib.sb_int8_sdpa_prefill_window(*fake, *args[6:], -1, 1, None) == _lib.SB_EINVAL
    assert b"window" in lib.sb_last_error_message()
