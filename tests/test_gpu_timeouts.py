"""The kernels' bounded waits on a B200: a wait that runs out ends the kernel
cleanly and the next call is correct.

With the wait limit lowered to 1 us (sabre_set_wait_limit_ns), the prefill
and the tensor-core decode kernels' waits for their copies and MMAs run out:
each CTA records SABRE_DEV_TIMEOUT, drains the copies and MMAs it issued (the
drains always allow 2 s), frees its tensor memory and exits without storing
its tile. The test checks that the launch completes, that the status word
reports the timeout, and that a call with the default limit afterwards
matches the oracle. Nothing here faults, traps or hangs the GPU: every wait
involved is bounded.
"""

import pytest
import torch

from oracle import attention_oracle as AO

pytestmark = pytest.mark.gpu

SABRE_DEV_TIMEOUT = 1


@pytest.fixture(scope="module")
def K():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from sabrecoder_b200 import kernels
    kernels.set_wait_limit_ns(0)
    kernels.device_status(clear=True)
    return kernels


def _close(out, ref):
    d = (out.float().cpu() - ref).abs()
    assert d.max().item() <= 2e-2 and d.mean().item() <= 2e-3, (d.max().item(), d.mean().item())


def test_wait_limit_rejects_values_out_of_range(K):
    from sabrecoder_b200._lib import SabreError
    with pytest.raises(SabreError, match="outside"):
        K.set_wait_limit_ns(10)
    with pytest.raises(SabreError, match="outside"):
        K.set_wait_limit_ns(61 * 10**9)


def test_prefill_wait_timeout_drains_and_next_call_is_correct(K):
    gen = torch.Generator().manual_seed(5)
    B, H, L, D, block = 1, 8, 4096, 128, 64
    q, k, v = (torch.randn(B, H, L, D, generator=gen).to(torch.bfloat16).cuda() for _ in range(3))
    nb = L // block
    # every causal block listed: each CTA walks a long key-tile list
    bi = torch.arange(nb, dtype=torch.int32).expand(B, nb, nb).contiguous().cuda()
    bc = torch.arange(1, nb + 1, dtype=torch.int32).expand(B, nb).contiguous().cuda()
    K.device_status(clear=True)
    K.set_wait_limit_ns(1000)
    try:
        K.prefill_bsa(q, k, v, bi, bc, block)
        torch.cuda.synchronize()
    finally:
        K.set_wait_limit_ns(0)
    assert K.device_status(clear=True) & SABRE_DEV_TIMEOUT
    out = K.prefill_bsa(q, k, v, bi, bc, block)
    torch.cuda.synchronize()
    assert K.device_status(clear=True) == 0
    _close(out[:, [0, H - 1]], AO.sparse_prefill_fp32(q.cpu(), k.cpu(), v.cpu(), bi.cpu(), bc.cpu(), block,
                                                      heads=[0, H - 1]))


def test_gqa_decode_wait_timeout_drains_and_next_call_is_correct(K):
    """Four query heads per KV head: the tcgen05 + TMA decode kernel (37
    splits per KV head, each walking ~14 key tiles)."""
    gen = torch.Generator().manual_seed(6)
    B, Hq, Hkv, T, D, block = 1, 32, 8, 32768, 128, 64
    q = torch.randn(B, Hq, D, generator=gen).to(torch.bfloat16).cuda()
    kc = torch.randn(B, Hkv, T, D, generator=gen).to(torch.bfloat16).cuda()
    vc = torch.randn(B, Hkv, T, D, generator=gen).to(torch.bfloat16).cuda()
    nbk = T // block
    lst = torch.arange(nbk, dtype=torch.int32).unsqueeze(0).cuda()
    cnt = torch.tensor([nbk], dtype=torch.int32).cuda()
    seq = torch.tensor([T], dtype=torch.int32).cuda()
    K.device_status(clear=True)
    K.set_wait_limit_ns(1000)
    try:
        K.decode_bsa(q, kc, vc, lst, cnt, seq, block)
        torch.cuda.synchronize()
    finally:
        K.set_wait_limit_ns(0)
    assert K.device_status(clear=True) & SABRE_DEV_TIMEOUT
    out = K.decode_bsa(q, kc, vc, lst, cnt, seq, block)
    torch.cuda.synchronize()
    assert K.device_status(clear=True) == 0
    _close(out, AO.sparse_decode_fp32(q.cpu(), kc.cpu(), vc.cpu(), lst.cpu(), cnt.cpu(), seq.cpu(), block))
