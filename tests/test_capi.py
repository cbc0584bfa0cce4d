"""The C-ABI library loads and exports every entry point include/sabre_b200.h
declares; host-side validation rejects bad arguments without launching."""

import ctypes
import os
import re

import pytest

from sabrecoder_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def header_functions():
    src = open(os.path.join(ROOT, "include", "sabre_b200.h")).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(sabre_[a-z0-9_]+)\s*\(", src)))


def test_header_declares_the_bound_functions():
    assert set(header_functions()) == set(_lib.SIGNATURES)


def test_library_exports_every_declared_symbol():
    L = _lib.lib()
    for name in header_functions():
        assert hasattr(L, name), name


def test_status_strings_and_version():
    L = _lib.lib()
    assert L.sabre_version() >= 100
    assert L.sabre_status_string(0) == b"ok"
    assert b"workspace" in L.sabre_status_string(-5)


def test_prefill_rejects_bad_arguments_before_launch():
    L = _lib.lib()
    st = _lib.i64([1, 1, 1, 1])
    r = L.sabre_prefill_bsa(None, None, None, None, None, None, 1, 1, 1, 64, 128, 64, 1, st, st, st, st, st, st,
                            0.0, 0, None)
    assert r == -1 and b"null" in L.sabre_last_error()
    fake = 16
    r = L.sabre_prefill_bsa(fake, fake, fake, fake, fake, fake, 1, 1, 1, 64, 96, 64, 1, st, st, st, st, st, st,
                            0.0, 0, None)
    assert r == -2 and b"head_dim" in L.sabre_last_error()
    r = L.sabre_prefill_bsa(fake, fake, fake, fake, fake, fake, 1, 1, 1, 64, 128, 32, 1, st, st, st, st, st, st,
                            0.0, 0, None)
    assert r == -2 and b"block_size" in L.sabre_last_error()
    r = L.sabre_prefill_bsa(fake, fake, fake, fake, fake, fake, 1, 3, 2, 64, 128, 64, 1, st, st, st, st, st, st,
                            0.0, 0, None)
    assert r == -1 and b"multiple" in L.sabre_last_error()


def test_decode_and_mask_reject_bad_arguments():
    L = _lib.lib()
    st = _lib.i64([1, 1, 1, 1])
    r = L.sabre_decode_bsa(16, 16, 16, 16, 16, 16, 16, 1, 9, 1, 64, 128, 64, 1, st, st, st, st, st, st, 0.0, 0,
                           None, 0, None)
    assert r == -2
    assert L.sabre_decode_workspace_size(1, 4, 4, 128, 10) > 0
    r = L.sabre_build_block_mask(16, None, 16, 1, 16, None, 1000, 64, 64, 0, 0, 100, 0, 16, None, 16, 8, None)
    assert r == -1 and b"multiple of block_size" in L.sabre_last_error()
    r = L.sabre_build_block_mask(16, None, 16, 1, 16, None, 1000, 64, 64, 0, 0, 128, 0, 16, None, 16, 4, None)
    assert r == -5


def test_qkv_rope_decode_rejects_positions_outside_the_cache():
    L = _lib.lib()
    st = _lib.i64([1, 1, 1])
    args = lambda pos, t: (16, 16, 16, 16, 16, 16, 16, 16, 16, 1, 2048, 16, 16, 128, pos, t, 2048, 128, st, st, st,
                           0, None)
    assert L.sabre_qkv_rope_decode(*args(64, 64)) == -1 and b"outside" in L.sabre_last_error()
    assert L.sabre_qkv_rope_decode(*args(-1, 64)) == -1
    assert L.sabre_qkv_rope_decode(*args(0, 0)) == -1
    r = L.sabre_qkv_rope_decode(16, 16, 16, 16, 16, 16, 16, 16, 16, 9, 2048, 16, 16, 128, 0, 8, 2048, 128, st, st,
                                st, 0, None)
    assert r == -2 and b"batch" in L.sabre_last_error()


def test_rope_qkv_rejects_rows_past_the_cache():
    import torch
    from sabrecoder_b200 import kernels
    q = torch.zeros(1, 4, 2, 128, dtype=torch.bfloat16)
    kv = torch.zeros(1, 2, 8, 128, dtype=torch.bfloat16)
    cs = torch.zeros(1, 4, 128, dtype=torch.bfloat16)
    with pytest.raises(_lib.SabreError, match="do not fit"):
        kernels.rope_qkv(q, q, q, cs, cs, kv, kv, pos0=5)


def test_rope_qkv_c_entry_checks_rows_against_the_cache():
    """The C entry point itself rejects rows outside [0, max_seq) (callers
    from other languages do not pass through the Python checks)."""
    L = _lib.lib()
    st = _lib.i64([1024, 1024, 128])

    def call(pos0, seq_len, max_seq):
        return L.sabre_rope_qkv(16, 16, 16, 16, 16, 16, 16, 16, None, None, 1, seq_len, 2, 2, 128, 0, pos0,
                                max_seq, st, st, st, st, st, st, st, 0, None)

    assert call(5, 4, 8) == -1 and b"outside the cache" in L.sabre_last_error()
    assert call(0, 9, 8) == -1 and b"outside the cache" in L.sabre_last_error()
    assert call(-1, 4, 8) == -1
    assert call(2147483647, 4, 8) == -1  # pos0 + L overflows int32
    assert call(0, 4, 0) == -1


@pytest.mark.parametrize("what", ["cos_rows", "cos_batch", "kout_batch", "kout_heads", "k_len"])
def test_rope_qkv_rejects_mismatched_shapes(what):
    import torch
    from sabrecoder_b200 import kernels
    B, L, Hq, Hkv, D, T = 2, 4, 4, 2, 128, 8
    q = torch.zeros(B, L, Hq, D, dtype=torch.bfloat16)
    k = torch.zeros(B, L, Hkv, D, dtype=torch.bfloat16)
    cs = torch.zeros(B, L, D, dtype=torch.bfloat16)
    kv = torch.zeros(B, Hkv, T, D, dtype=torch.bfloat16)
    if what == "cos_rows":
        cs = torch.zeros(B, L - 1, D, dtype=torch.bfloat16)
    elif what == "cos_batch":
        cs = torch.zeros(B + 1, L, D, dtype=torch.bfloat16)  # neither B nor 1
    elif what == "kout_batch":
        kv = torch.zeros(B - 1, Hkv, T, D, dtype=torch.bfloat16)
    elif what == "kout_heads":
        kv = torch.zeros(B, Hkv + 1, T, D, dtype=torch.bfloat16)
    else:
        k = torch.zeros(B, L + 1, Hkv, D, dtype=torch.bfloat16)
    with pytest.raises(_lib.SabreError, match="rope_qkv"):
        kernels.rope_qkv(q, k, k, cs, cs, kv, kv)


def test_kernel_calls_fail_loudly_without_cuda_tensors():
    import torch
    from sabrecoder_b200 import kernels
    q = torch.zeros(1, 1, 64, 128, dtype=torch.bfloat16)
    with pytest.raises(_lib.SabreError, match="CUDA tensor"):
        kernels.prefill_bsa(q, q, q, torch.zeros(1, 1, 1, dtype=torch.int32), torch.ones(1, 1, dtype=torch.int32), 64)


def test_qkv_proj_rope_rejects_bad_arguments_before_launch():
    L = _lib.lib()
    st = _lib.i64([1024, 128, 128])

    def call(seq_len=256, pos0=0, max_seq=512, pool=None, pool_block=64, batch=1, hidden=2048, xs=2048):
        return L.sabre_qkv_proj_rope(16, 16, 16, 16, 16, 16, 16, pool, None, None, batch, seq_len, hidden, 2, 2,
                                     128, pool_block, pos0, max_seq, xs, st, st, st, st, 0, 0, None)

    assert call(seq_len=600) == -1 and b"outside the cache" in L.sabre_last_error()
    assert call(pos0=-1) == -1
    assert call(hidden=2044, xs=2044) == -3
    assert call(xs=1024) == -3
    assert call(pool=16, pool_block=32) == -2 and b"pooling" in L.sabre_last_error()
    assert call(pool=16, pos0=4) == -2
    assert call(pool=16, batch=2, seq_len=200) == -2
    assert L.sabre_qkv_proj_rope(None, 16, 16, 16, 16, 16, 16, None, None, None, 1, 4, 256, 2, 2, 128, 0, 0, 8, 256,
                                 st, st, st, st, 0, 0, None) == -1
