"""The allocation-free decode entry point against the workspace one and the
oracle.

sabre_decode_bsa_noalloc serves callers that cannot give this library any
device memory at decode time (a runtime that reserved all memory at start-up,
a binding with no allocator of its own). Its split partials live in a fixed
array inside the library, so this test calls it twice in a row with different
inputs through the C ABI and checks each result against sabre_decode_bsa and
the oracle's decode (same tolerance as the other attention tests): the second
call must not see the first call's leftovers. The file is named to be
collected last.
"""

import ctypes

import pytest
import torch

from oracle import attention_oracle as AO

pytestmark = pytest.mark.gpu

MAX_ABS = 2e-2
MEAN_ABS = 2e-3


def _case(seed, B, Hq, Hkv, Tmax, block, dev):
    gen = torch.Generator().manual_seed(seed)
    D = 128
    q = torch.randn(B, Hq, D, generator=gen).to(torch.bfloat16).to(dev)
    kc = torch.randn(B, Hkv, Tmax, D, generator=gen).to(torch.bfloat16).to(dev)
    vc = torch.randn(B, Hkv, Tmax, D, generator=gen).to(torch.bfloat16).to(dev)
    seq = torch.randint(1, Tmax + 1, (B,), generator=gen).to(torch.int32)
    nbk = (Tmax + block - 1) // block
    m = torch.rand(B, Hkv, nbk, generator=gen) < 0.5
    for b in range(B):
        m[b, :, (int(seq[b]) - 1) // block] = True
    cnt = m.sum(-1).to(torch.int32)
    mx = int(cnt.max())
    idx = torch.full((B, Hkv, mx), -1, dtype=torch.int32)
    for b in range(B):
        for h in range(Hkv):
            nz = torch.nonzero(m[b, h]).flatten().to(torch.int32)
            idx[b, h, : nz.numel()] = nz
    return q, kc, vc, idx.to(dev), cnt.to(dev), seq.to(dev)


def _noalloc(q, kc, vc, idx, cnt, seq, block):
    from sabrecoder_b200 import _lib
    L = _lib.lib()
    out = torch.empty_like(q)
    B, Hq, D = q.shape
    Hkv, Tmax = kc.shape[1], kc.shape[2]
    idx_strides = (idx.stride(0), idx.stride(1), idx.stride(2))
    cnt_strides = (cnt.stride(0), cnt.stride(1))
    rc = L.sabre_decode_bsa_noalloc(
        q.data_ptr(), kc.data_ptr(), vc.data_ptr(), out.data_ptr(), idx.data_ptr(), cnt.data_ptr(),
        seq.data_ptr(), B, Hq, Hkv, Tmax, D, block, int(idx.shape[-1]), _lib.i64(q.stride()),
        _lib.i64(kc.stride()), _lib.i64(vc.stride()), _lib.i64(out.stride()), _lib.i64(idx_strides),
        _lib.i64(cnt_strides), ctypes.c_float(0.0), 0, torch.cuda.current_stream().cuda_stream)
    assert rc == 0, L.sabre_last_error().decode()
    return out


def test_noalloc_decode_matches_workspace_decode_on_two_calls():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from sabrecoder_b200 import kernels as K
    dev = torch.device("cuda")
    # Groups of 4 and 7 query heads per KV head take the tensor-core decode,
    # one head per KV head the CUDA-core one.
    for seed, shape in ((1, (2, 8, 2, 3000, 64)), (2, (1, 7, 1, 2100, 128)), (3, (3, 4, 4, 1800, 64))):
        B, Hq, Hkv, Tmax, block = shape
        q, kc, vc, idx, cnt, seq = _case(seed, B, Hq, Hkv, Tmax, block, dev)
        ref = K.decode_bsa(q, kc, vc, idx, cnt, seq, block)
        out = _noalloc(q, kc, vc, idx, cnt, seq, block)
        torch.cuda.synchronize()
        d = (out.float() - ref.float()).abs()
        assert d.max().item() <= MAX_ABS, d.max().item()
        assert d.mean().item() <= MEAN_ABS, d.mean().item()
        # and against the oracle, so a fault shared by both entry points
        # (they run the same split and merge code) cannot hide
        want = AO.sparse_decode_fp32(q.cpu(), kc.cpu(), vc.cpu(), idx.cpu(), cnt.cpu(), seq.cpu(), block)
        d = (out.float().cpu() - want).abs()
        assert d.max().item() <= MAX_ABS, d.max().item()
        assert d.mean().item() <= MEAN_ABS, d.mean().item()


def test_noalloc_rejects_shapes_beyond_the_scratch():
    from sabrecoder_b200 import _lib
    L = _lib.lib()
    qs = _lib.i64([8, 8, 1])
    ks = _lib.i64([8, 8, 8, 1])
    # batch * heads_q * 130 floats > 2 MiB of scratch even with one split
    rc = L.sabre_decode_bsa_noalloc(16, 16, 16, 16, 16, 16, 16, 512, 64, 8, 64, 128, 64, 1, qs, ks, ks, qs, ks,
                                    qs, 0.0, 0, None)
    assert rc == -2
    assert b"scratch" in L.sabre_last_error()
