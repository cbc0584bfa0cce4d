"""GPU parity of the CUDA kernels against the oracle and the reference's
recorded outputs. Tolerances (bf16): max-abs 2e-2, mean-abs 2e-3 for
attention; bit-exact for masks, counts and index lists."""

import numpy as np
import pytest
import torch

import _golden as G
from oracle import attention_oracle as AO
from oracle import mask_oracle as MO

pytestmark = pytest.mark.gpu

MAX_ABS = 2e-2
MEAN_ABS = 2e-3


@pytest.fixture(scope="module")
def K():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from sabrecoder_b200 import kernels
    kernels.device_status(clear=True)
    return kernels


def _close(out, ref, max_abs=MAX_ABS, mean_abs=MEAN_ABS):
    d = (out.float().cpu() - ref.float().cpu()).abs()
    assert d.max().item() <= max_abs, f"max-abs {d.max().item():.3e}"
    assert d.mean().item() <= mean_abs, f"mean-abs {d.mean().item():.3e}"


def _random_lists(B, nb, gen, density=0.3, heads=None):
    shape = (B, nb, nb) if heads is None else (B, heads, nb, nb)
    m = torch.rand(shape, generator=gen) < density
    m = m | torch.eye(nb, dtype=torch.bool)
    m = m.tril()
    idx, cnt = MO.block_indices_from_mask(m.numpy())
    return torch.from_numpy(idx), torch.from_numpy(cnt)


@pytest.mark.parametrize("case", ["attn_b64.npz", "attn_b128.npz"])
def test_prefill_matches_reference_kernel_output(K, case):
    g = G.load(case)
    q, k, v = (G.bf16_bits_to_f32(g[n]).to(torch.bfloat16).cuda() for n in ("q_bf16", "k_bf16", "v_bf16"))
    bi = torch.from_numpy(g["block_indices"]).cuda()
    bc = torch.from_numpy(g["block_counts"]).cuda()
    out = K.prefill_bsa(q, k, v, bi, bc, int(g["block_size"]))
    torch.cuda.synchronize()
    _close(out, torch.from_numpy(g["out"]))


@pytest.mark.parametrize("B,Hq,Hkv,L,block,dtype,per_head,layout", [
    (1, 2, 2, 1000, 64, torch.bfloat16, False, "bhld"),
    (2, 4, 2, 512, 64, torch.bfloat16, False, "blhd"),
    (1, 4, 4, 700, 64, torch.bfloat16, True, "blhd"),
    (1, 2, 1, 900, 128, torch.bfloat16, False, "blhd"),
    (1, 2, 2, 640, 64, torch.float16, False, "bhld"),
    (1, 7, 1, 384, 128, torch.bfloat16, True, "blhd"),
    (1, 1, 1, 65, 64, torch.bfloat16, False, "bhld"),
    (1, 1, 1, 40, 64, torch.bfloat16, False, "bhld"),
])
def test_prefill_vs_oracle(K, B, Hq, Hkv, L, block, dtype, per_head, layout):
    gen = torch.Generator().manual_seed(L + Hq + block)
    D = 128

    def mk(H):
        if layout == "blhd":
            return torch.randn(B, L, H, D, generator=gen).to(dtype).transpose(1, 2)
        return torch.randn(B, H, L, D, generator=gen).to(dtype)

    q, k, v = mk(Hq), mk(Hkv), mk(Hkv)
    nb = (L + block - 1) // block
    bi, bc = _random_lists(B, nb, gen, heads=Hq if per_head else None)
    out = K.prefill_bsa(q.cuda(), k.cuda(), v.cuda(), bi.cuda(), bc.cuda(), block)
    torch.cuda.synchronize()
    ref = AO.sparse_prefill_fp32(q, k, v, bi, bc, block)
    _close(out, ref)


def test_prefill_ignores_invalid_entries(K):
    """Entries beyond the count, negative, past the query block, or repeated
    contribute nothing extra (the reference's causal mask drops the ones past
    the query block; valid lists never hold the others)."""
    gen = torch.Generator().manual_seed(3)
    B, H, L, D, block = 1, 2, 512, 128, 64
    q, k, v = (torch.randn(B, H, L, D, generator=gen).to(torch.bfloat16) for _ in range(3))
    nb = L // block
    bi, bc = _random_lists(B, nb, gen)
    ref = AO.sparse_prefill_fp32(q, k, v, bi, bc, block)
    cap = bi.shape[-1] + 3
    junk = torch.full((B, nb, cap), -1, dtype=torch.int32)
    for r in range(nb):
        c = int(bc[0, r])
        row = bi[0, r, :c].tolist()
        extra = [-5, nb + 3, min(r + 1, nb - 1) if r + 1 < nb else r] + row[:1]
        junk[0, r, : c + len(extra)] = torch.tensor((row + extra)[: cap], dtype=torch.int32)
        bc[0, r] = min(c + len(extra), cap)
    out = K.prefill_bsa(q.cuda(), k.cuda(), v.cuda(), junk.cuda(), bc.cuda(), block)
    torch.cuda.synchronize()
    _close(out, ref)


def test_prefill_empty_lists_give_zero_rows(K):
    """Query blocks with count 0 attend to nothing and output zeros (the
    reference divides by l = 1 when l == 0, :112); a whole 128-row tile with
    empty lists is covered too."""
    gen = torch.Generator().manual_seed(9)
    B, H, L, D, block = 1, 2, 640, 128, 64
    q, k, v = (torch.randn(B, H, L, D, generator=gen).to(torch.bfloat16) for _ in range(3))
    nb = L // block
    bi, bc = _random_lists(B, nb, gen)
    bc[0, 2] = 0
    bc[0, 3] = 0  # query blocks 2 and 3 form one 128-row tile
    bc[0, 7] = 0
    out = K.prefill_bsa(q.cuda(), k.cuda(), v.cuda(), bi.cuda(), bc.cuda(), block)
    torch.cuda.synchronize()
    ref = AO.sparse_prefill_fp32(q, k, v, bi, bc, block)
    _close(out, ref)
    assert out[:, :, 128:256].abs().max().item() == 0.0


@pytest.mark.parametrize("block", [64, 128])
def test_prefill_many_items_ragged(K, block):
    """Several 128-row tiles per CTA (more tiles than SMs) with ragged lists:
    empty tiles, tiles with one key block, odd and even counts, per head; the
    tiles of one CTA run back to back, so each must start its accumulators
    and running statistics afresh."""
    gen = torch.Generator().manual_seed(17 + block)
    B, H, L, D = 2, 12, 3000, 128
    q, k, v = (torch.randn(B, H, L, D, generator=gen).to(torch.bfloat16) for _ in range(3))
    nb = (L + block - 1) // block
    m = torch.rand(B, H, nb, nb, generator=gen) < 0.15
    kind = torch.randint(0, 5, (B, H, nb), generator=gen)
    m[kind == 0] = False                                   # empty row
    one = torch.zeros(B, H, nb, nb, dtype=torch.bool)
    one[..., 0] = True
    m = torch.where((kind == 1).unsqueeze(-1), one, m)     # only the first block
    m = m | (torch.eye(nb, dtype=torch.bool) & (kind != 0).unsqueeze(-1))
    idx, cnt = MO.block_indices_from_mask(m.tril().numpy())
    bi, bc = torch.from_numpy(idx), torch.from_numpy(cnt)
    out = K.prefill_bsa(q.cuda(), k.cuda(), v.cuda(), bi.cuda(), bc.cuda(), block)
    torch.cuda.synchronize()
    ref = AO.sparse_prefill_fp32(q, k, v, bi, bc, block)
    _close(out, ref)
    assert K.device_status() == 0


def test_prefill_small_union_counts(K):
    """128-row tiles whose union of key tiles is exactly 0, 1, 2, 3, 4 and 5
    (the counts where the kernel's first S commits and its per-tile commits
    meet), each tile on its own head; every wait completes (no timeout
    recorded) and the rows match the oracle."""
    gen = torch.Generator().manual_seed(41)
    B, H, L, D, block = 1, 6, 768, 128, 64
    q, k, v = (torch.randn(B, H, L, D, generator=gen).to(torch.bfloat16) for _ in range(3))
    nb = L // block                       # 12 query blocks, 6 tiles of 128 rows
    m = torch.zeros(B, H, nb, nb, dtype=torch.bool)
    for h, n_union in enumerate(range(6)):
        # tile 5 (query blocks 10 and 11): a union of exactly n_union key tiles
        keys = list(range(n_union))
        for qb in (10, 11):
            for kb in keys:
                m[0, h, qb, kb] = True
        # the other tiles of the head keep their diagonal block only
        for qb in range(10):
            m[0, h, qb, qb] = True
    idx, cnt = MO.block_indices_from_mask(m.numpy())
    bi, bc = torch.from_numpy(idx), torch.from_numpy(cnt)
    K.device_status(clear=True)
    out = K.prefill_bsa(q.cuda(), k.cuda(), v.cuda(), bi.cuda(), bc.cuda(), block)
    torch.cuda.synchronize()
    assert K.device_status() == 0
    ref = AO.sparse_prefill_fp32(q, k, v, bi, bc, block)
    _close(out, ref)
    assert out[0, 0, 640:768].abs().max().item() == 0.0   # union 0: nothing visible


def test_prefill_config0_shape(K):
    """B=1, H=16, L=4096, D=128, block 64 with a structure mask + top-8."""
    gen = torch.Generator().manual_seed(0)
    B, H, L, D, block = 1, 16, 4096, 128, 64
    q, k, v = (torch.randn(B, H, L, D, generator=gen).to(torch.bfloat16) for _ in range(3))
    g = G.load("mask_c0_4096.npz")
    base = g["block_mask"].astype(bool)
    qm = MO.pooled_block_means(q.float().numpy(), L, block)
    km = MO.pooled_block_means(k.float().numpy(), L, block)
    ext = MO.topk_extend_mask(base, MO.pooled_scores(qm, km), 8)
    idx, cnt = MO.block_indices_from_mask(ext)
    bi, bc = torch.from_numpy(idx), torch.from_numpy(cnt)
    out = K.prefill_bsa(q.cuda(), k.cuda(), v.cuda(), bi.cuda(), bc.cuda(), block)
    torch.cuda.synchronize()
    ref = AO.sparse_prefill_fp32(q, k, v, bi, bc, block)
    _close(out, ref)
    assert K.device_status(clear=True) == 0


@pytest.mark.parametrize("L,block", [(65536, 64), (65536 - 37, 64), (65536 - 37, 128)])
def test_prefill_at_the_maximum_length(K, L, block):
    """The longest prompt the kernel takes (L <= 65536: 1024 key tiles, the
    last bit of its key-tile bitmaps), also with a ragged last block and with
    128-token blocks; 8 query / 4 KV heads, so K/V (134 MB) exceed L2 and the
    CTAs run head-major. Lists shared by all heads (the reference's layout):
    the sink, a 4-block window, the block at half the row and 6 random
    earlier blocks."""
    Hq, Hkv, D = 8, 4, 128
    gen = torch.Generator().manual_seed(L + block)
    q, k, v = (torch.randn(1, H, L, D, generator=gen).to(torch.bfloat16) for H in (Hq, Hkv, Hkv))
    nb = (L + block - 1) // block
    rng = np.random.default_rng(L + block)
    m = np.zeros((1, nb, nb), dtype=bool)
    for qb in range(nb):
        m[0, qb, 0] = True
        m[0, qb, max(0, qb - 3):qb + 1] = True
        m[0, qb, qb // 2] = True
        m[0, qb, rng.integers(0, qb + 1, size=6)] = True
    idx, cnt = MO.block_indices_from_mask(m)
    bi, bc = torch.from_numpy(idx), torch.from_numpy(cnt)
    K.device_status(clear=True)
    out = K.prefill_bsa(q.cuda(), k.cuda(), v.cuda(), bi.cuda(), bc.cuda(), block)
    torch.cuda.synchronize()
    assert K.device_status(clear=True) == 0
    ref = AO.sparse_prefill_fp32_gathered(q, k, v, bi, bc, block)
    _close(out, ref)


def _kernel_mask(K, g):
    p = G.params(g)
    L = int(g["seq_len"])
    nchunks = g["chunk_type"].shape[0]
    flags = np.zeros(max(nchunks, 1), np.uint8)[:nchunks]
    for c in g["import_chunks"].tolist():
        if 0 <= c < nchunks:
            flags[c] |= 1
    deps = G.deps(g)
    ptr = np.zeros(nchunks + 1, np.int32)
    flat = []
    for c in range(nchunks):
        tg = sorted(deps.get(c, ()))
        flat.extend(tg)
        ptr[c + 1] = len(flat)
    dev = "cuda"
    bits, dense = K.build_block_mask(
        torch.from_numpy(g["token_to_chunk"].astype(np.int32)).to(dev), torch.from_numpy(flags).to(dev),
        torch.from_numpy(ptr).to(dev), torch.tensor(flat, dtype=torch.int32, device=dev),
        torch.from_numpy(g["global_token_mask"].astype(np.uint8)).to(dev), seq_len=L, **p)
    return bits, dense


@pytest.mark.parametrize("case", G.mask_cases())
def test_block_mask_kernel_bit_exact(K, case):
    g = G.load(case)
    bits, dense = _kernel_mask(K, g)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(dense.cpu().numpy(), g["block_mask"])
    nb = dense.shape[0]
    idx, cnt, mx = K.indices_from_bits(bits, nb)
    torch.cuda.synchronize()
    ma = int(mx.item())
    assert ma == g["indices_sorted"].shape[-1]
    np.testing.assert_array_equal(cnt.cpu().numpy(), g["block_counts"][0])
    np.testing.assert_array_equal(idx[:, :ma].cpu().numpy(), g["indices_sorted"][0])
    idx2, cnt2, mx2 = K.indices_from_dense(dense.unsqueeze(0))
    torch.cuda.synchronize()
    np.testing.assert_array_equal(idx2[..., :ma].cpu().numpy(), g["indices_sorted"])
    assert int(mx2.item()) == ma


def test_indices_from_dense_random(K):
    gen = torch.Generator().manual_seed(5)
    for nb in (1, 31, 32, 33, 200, 1100):
        m = (torch.rand(3, nb, nb, generator=gen) < 0.2).int()
        if nb == 33:
            m.zero_()
        idx, cnt, mx = K.indices_from_dense(m.cuda())
        torch.cuda.synchronize()
        ri, rc = MO.block_indices_from_mask(m.numpy())
        ma = int(mx.item())
        assert ma == ri.shape[-1]
        np.testing.assert_array_equal(cnt.cpu().numpy(), rc)
        np.testing.assert_array_equal(idx[..., :ma].cpu().numpy(), ri)


@pytest.mark.parametrize("B,Hq,Hkv,L,block,topk", [(1, 4, 4, 1000, 64, 8), (1, 4, 2, 640, 64, 3),
                                                    (2, 2, 2, 2000, 128, 8)])
def test_pooled_topk_bit_exact(K, B, Hq, Hkv, L, block, topk):
    gen = torch.Generator().manual_seed(L)
    D = 128
    q = torch.randn(B, L, Hq, D, generator=gen).to(torch.bfloat16).transpose(1, 2)
    k = torch.randn(B, L, Hkv, D, generator=gen).to(torch.bfloat16).transpose(1, 2)
    nb = (L + block - 1) // block
    base = np.tril(np.random.default_rng(L).random((nb, nb)) < 0.15) | np.eye(nb, dtype=bool)
    qm = K.pool_blocks(q.cuda(), block)
    km = K.pool_blocks(k.cuda(), block)
    torch.cuda.synchronize()
    qm_ref = MO.pooled_block_means(q.float().numpy(), L, block)
    km_ref = MO.pooled_block_means(k.float().numpy(), L, block)
    np.testing.assert_array_equal(qm.cpu().numpy(), qm_ref)
    np.testing.assert_array_equal(km.cpu().numpy(), km_ref)
    nwords = (nb + 31) // 32
    bits = np.zeros((nb, nwords), np.uint32)
    for i in range(nb):
        for j in np.nonzero(base[i])[0]:
            bits[i, j // 32] |= np.uint32(1) << np.uint32(j % 32)
    bits_t = torch.from_numpy(bits.view(np.int32)).cuda()
    idx, cnt, mx, _ = K.topk_extend(qm, km, bits_t, topk)
    torch.cuda.synchronize()
    g = Hq // Hkv
    sc = MO.pooled_scores(qm_ref, np.repeat(km_ref, g, axis=1))
    ext = MO.topk_extend_mask(base, sc, topk)
    ri, rc = MO.block_indices_from_mask(ext)
    ma = int(mx.item())
    assert ma == ri.shape[-1]
    np.testing.assert_array_equal(cnt.cpu().numpy(), rc)
    np.testing.assert_array_equal(idx[..., :ma].cpu().numpy(), ri)


@pytest.mark.parametrize("B,Hq,Hkv,Tmax,block,shared", [(1, 4, 4, 3000, 64, True), (2, 7, 1, 2048, 128, False),
                                                         (3, 8, 2, 1500, 64, False), (1, 2, 2, 64, 64, True),
                                                         (1, 16, 2, 5000, 64, False), (2, 4, 4, 700, 192, True),
                                                         # 9 or more (sequence, KV head) groups: the splits of a
                                                         # group merge inside one thread-block cluster
                                                         (1, 16, 16, 3000, 64, False), (2, 32, 8, 2000, 64, True),
                                                         (3, 24, 3, 1800, 128, False), (1, 32, 32, 4100, 64, True),
                                                         # a cache shorter than one 64-row tile
                                                         (2, 8, 2, 40, 64, False),
                                                         # blocks of three and four 64-row pieces: a split's
                                                         # share may start and end inside a block
                                                         (2, 14, 2, 2500, 192, False), (1, 8, 1, 4000, 256, True),
                                                         # long caches: lists of ~800 blocks over up to 296 splits
                                                         (1, 8, 1, 131072 + 33, 64, True), (1, 2, 2, 70000, 64, False)])
def test_decode_vs_oracle(K, B, Hq, Hkv, Tmax, block, shared):
    gen = torch.Generator().manual_seed(Tmax + Hq)
    D = 128
    q = torch.randn(B, Hq, D, generator=gen).to(torch.bfloat16)
    kc = torch.randn(B, Hkv, Tmax, D, generator=gen).to(torch.bfloat16)
    vc = torch.randn(B, Hkv, Tmax, D, generator=gen).to(torch.bfloat16)
    seq = torch.randint(1, Tmax + 1, (B,), generator=gen).to(torch.int32)
    nbk = (Tmax + block - 1) // block
    H = 1 if shared else Hkv
    m = torch.rand(B, H, nbk, generator=gen) < 0.4
    for b in range(B):
        m[b, :, (int(seq[b]) - 1) // block] = True
    idx, cnt = MO.block_indices_from_mask(m.numpy())
    bi, bc = torch.from_numpy(idx), torch.from_numpy(cnt)
    if shared:
        bi, bc = bi[:, 0], bc[:, 0]
    out = K.decode_bsa(q.cuda(), kc.cuda(), vc.cuda(), bi.cuda(), bc.cuda(), seq.cuda(), block)
    torch.cuda.synchronize()
    ref = AO.sparse_decode_fp32(q, kc, vc, bi, bc, seq, block)
    _close(out, ref)


@pytest.mark.parametrize("Hq,Hkv", [(4, 4), (8, 2)])
def test_decode_with_a_workspace_only_float_aligned(K, Hq, Hkv):
    """A workspace that is 4- but not 16-byte aligned (the split partials are
    then stored 4 bytes at a time) gives the oracle's result, for the
    CUDA-core and the tensor-core decode."""
    gen = torch.Generator().manual_seed(Hq + 100)
    B, T, D, block = 1, 3000, 128, 64
    q = torch.randn(B, Hq, D, generator=gen).to(torch.bfloat16)
    kc = torch.randn(B, Hkv, T, D, generator=gen).to(torch.bfloat16)
    vc = torch.randn(B, Hkv, T, D, generator=gen).to(torch.bfloat16)
    nbk = (T + block - 1) // block
    bi = torch.arange(nbk, dtype=torch.int32).unsqueeze(0)
    bc = torch.tensor([nbk], dtype=torch.int32)
    seq = torch.tensor([T], dtype=torch.int32)
    need = K.decode_workspace_bytes(B, Hq, Hkv, D, nbk)
    ws = torch.empty(need + 16, dtype=torch.uint8, device="cuda")[4:]
    assert ws.data_ptr() % 16 == 4
    out = K.decode_bsa(q.cuda(), kc.cuda(), vc.cuda(), bi.cuda(), bc.cuda(), seq.cuda(), block, workspace=ws)
    torch.cuda.synchronize()
    _close(out, AO.sparse_decode_fp32(q, kc, vc, bi, bc, seq, block))


@pytest.mark.parametrize("Hq,Hkv", [(4, 4), (8, 2)])
def test_decode_f16_vs_oracle(K, Hq, Hkv):
    """fp16 caches: one query head per KV head (CUDA-core kernel) and four
    (tensor-core kernel)."""
    gen = torch.Generator().manual_seed(99 + Hq)
    B, Tmax, block, D = 2, 1500, 64, 128
    q = torch.randn(B, Hq, D, generator=gen).to(torch.float16)
    kc = torch.randn(B, Hkv, Tmax, D, generator=gen).to(torch.float16)
    vc = torch.randn(B, Hkv, Tmax, D, generator=gen).to(torch.float16)
    seq = torch.tensor([Tmax, 901], dtype=torch.int32)
    nbk = (Tmax + block - 1) // block
    m = torch.rand(B, Hkv, nbk, generator=gen) < 0.4
    for b in range(B):
        m[b, :, (int(seq[b]) - 1) // block] = True
    idx, cnt = MO.block_indices_from_mask(m.numpy())
    bi, bc = torch.from_numpy(idx), torch.from_numpy(cnt)
    out = K.decode_bsa(q.cuda(), kc.cuda(), vc.cuda(), bi.cuda(), bc.cuda(), seq.cuda(), block)
    torch.cuda.synchronize()
    ref = AO.sparse_decode_fp32(q, kc, vc, bi, bc, seq, block)
    _close(out, ref)


@pytest.mark.parametrize("block,row_pad,Hq", [(32, 0, 4), (64, 128, 4), (64, 128, 14), (128, 64, 16),
                                               (192, 128, 4)])
def test_decode_strided_cache_vs_oracle(K, block, row_pad, Hq):
    """Caches whose rows are not contiguous per head (row stride > head_dim) or
    blocks that are not whole 64-row chunks take the register-streaming kernel;
    groups of 7 and 8 query heads per KV head read the same strided caches
    through TMA tensor maps on the tensor-core path."""
    gen = torch.Generator().manual_seed(block + row_pad + Hq)
    B, Hkv, Tmax, D = 2, 2, 1200, 128
    q = torch.randn(B, Hq, D, generator=gen).to(torch.bfloat16)
    kbig = torch.randn(B, Hkv, Tmax, D + row_pad, generator=gen).to(torch.bfloat16)
    vbig = torch.randn(B, Hkv, Tmax, D + row_pad, generator=gen).to(torch.bfloat16)
    seq = torch.tensor([Tmax, 777], dtype=torch.int32)
    nbk = (Tmax + block - 1) // block
    m = torch.rand(B, Hkv, nbk, generator=gen) < 0.5
    for b in range(B):
        m[b, :, (int(seq[b]) - 1) // block] = True
    idx, cnt = MO.block_indices_from_mask(m.numpy())
    bi, bc = torch.from_numpy(idx), torch.from_numpy(cnt)
    kc, vc = kbig.cuda()[..., :D], vbig.cuda()[..., :D]
    out = K.decode_bsa(q.cuda(), kc, vc, bi.cuda(), bc.cuda(), seq.cuda(), block)
    torch.cuda.synchronize()
    ref = AO.sparse_decode_fp32(q, kbig[..., :D], vbig[..., :D], bi, bc, seq, block)
    _close(out, ref)


@pytest.mark.parametrize("B,hidden,Hq,Hkv,dtype", [(1, 2048, 16, 16, torch.bfloat16), (3, 1024, 8, 2, torch.bfloat16),
                                                  (2, 1792, 14, 2, torch.float16),
                                                  # the 6.7B and 33B decode-step shapes
                                                  (1, 4096, 32, 32, torch.bfloat16), (1, 7168, 56, 8, torch.bfloat16)])
def test_qkv_rope_decode_vs_unfused(K, B, hidden, Hq, Hkv, dtype):
    """The fused decode projection + rotary + KV store against the unfused
    computation (cuBLAS projection rounded to the dtype, then transformers'
    apply_rotary_pos_emb); they differ only by the projection's summation
    order, so outputs agree within two ulps. Other cache rows stay untouched."""
    from transformers.models.llama.modeling_llama import apply_rotary_pos_emb
    gen = torch.Generator().manual_seed(hidden + Hq)
    D, T, pos = 128, 40, 29
    dev = torch.device("cuda")
    x = torch.randn(B, hidden, generator=gen).to(dtype).to(dev)
    w = [(torch.randn(h * D, hidden, generator=gen) / hidden ** 0.5).to(dtype).to(dev) for h in (Hq, Hkv, Hkv)]
    ang = torch.rand(B, D // 2, generator=gen) * 6.0
    emb = torch.cat([ang, ang], dim=-1)
    cos, sin = emb.cos().to(dtype).to(dev), emb.sin().to(dtype).to(dev)
    sentinel = torch.full((B, Hkv, T, D), 7.0, dtype=dtype, device=dev)
    kc, vc = sentinel.clone(), sentinel.clone()
    q = torch.empty(B, Hq, D, dtype=dtype, device=dev)
    K.qkv_rope_decode(x, w[0], w[1], w[2], cos, sin, q, kc, vc, pos)
    torch.cuda.synchronize()
    yq = torch.nn.functional.linear(x, w[0]).view(B, 1, Hq, D).transpose(1, 2)
    yk = torch.nn.functional.linear(x, w[1]).view(B, 1, Hkv, D).transpose(1, 2)
    yv = torch.nn.functional.linear(x, w[2]).view(B, Hkv, D)
    rq, rk = apply_rotary_pos_emb(yq, yk, cos.unsqueeze(1), sin.unsqueeze(1))
    tol = dict(rtol=2 ** -6, atol=2 ** -6)
    torch.testing.assert_close(q.float(), rq[:, :, 0].float(), **tol)
    torch.testing.assert_close(kc[:, :, pos].float(), rk[:, :, 0].float(), **tol)
    torch.testing.assert_close(vc[:, :, pos].float(), yv.float(), **tol)
    others = torch.ones(T, dtype=torch.bool)
    others[pos] = False
    assert torch.equal(kc[:, :, others], sentinel[:, :, others])
    assert torch.equal(vc[:, :, others], sentinel[:, :, others])


def test_no_device_timeouts_recorded(K):
    assert K.device_status(clear=True) == 0


def test_rope_qkv_batch_with_one_shared_table(K):
    """transformers hands every sequence the same [1, L, D] cos/sin when the
    position ids are shared; a batch of three must read that one table for
    each sequence (bit-exact with apply_rotary_pos_emb's broadcast)."""
    from transformers.models.llama.modeling_llama import apply_rotary_pos_emb
    gen = torch.Generator().manual_seed(11)
    B, L, Hq, Hkv, D = 3, 200, 4, 2, 128
    q = torch.randn(B, L, Hq, D, generator=gen).to(torch.bfloat16)
    k = torch.randn(B, L, Hkv, D, generator=gen).to(torch.bfloat16)
    v = torch.randn(B, L, Hkv, D, generator=gen).to(torch.bfloat16)
    ang = torch.rand(1, L, D // 2, generator=gen) * 50
    emb = torch.cat([ang, ang], -1)
    cos, sin = emb.cos().to(torch.bfloat16), emb.sin().to(torch.bfloat16)
    rq, rk = apply_rotary_pos_emb(q.transpose(1, 2), k.transpose(1, 2), cos, sin)
    qd = q.cuda().clone()
    kc = torch.zeros(B, Hkv, L, D, dtype=torch.bfloat16, device="cuda")
    vc = torch.zeros_like(kc)
    K.rope_qkv(qd, k.cuda(), v.cuda(), cos.cuda(), sin.cuda(), kc, vc)
    torch.cuda.synchronize()
    assert torch.equal(qd.transpose(1, 2).cpu(), rq)
    assert torch.equal(kc.cpu(), rk)
    assert torch.equal(vc.cpu(), v.transpose(1, 2))


@pytest.mark.parametrize("B,L,Hq,Hkv,pool,dtype", [(1, 1000, 4, 2, 64, torch.bfloat16), (2, 300, 2, 2, 128, torch.bfloat16),
                                                   (1, 1, 4, 4, 0, torch.bfloat16), (1, 257, 2, 1, 64, torch.float16),
                                                   # the c1 and c4 layer shapes of the benchmark
                                                   (1, 12288, 16, 16, 64, torch.bfloat16),
                                                   (1, 16384, 56, 8, 128, torch.bfloat16)])
def test_rope_qkv_bit_exact_with_hf(K, B, L, Hq, Hkv, pool, dtype):
    """Fused RoPE + KV store equals transformers' apply_rotary_pos_emb bit for
    bit; pools equal the oracle's block means of the rotated rows."""
    from transformers.models.llama.modeling_llama import apply_rotary_pos_emb
    gen = torch.Generator().manual_seed(L + Hq)
    D = 128
    qkv = torch.randn(B, L, (Hq + 2 * Hkv) * D, generator=gen).to(dtype)
    q = qkv[..., : Hq * D].view(B, L, Hq, D)
    k = qkv[..., Hq * D: (Hq + Hkv) * D].view(B, L, Hkv, D)
    v = qkv[..., (Hq + Hkv) * D:].view(B, L, Hkv, D)
    ang = torch.rand(B, L, D // 2, generator=gen) * 50
    emb = torch.cat([ang, ang], -1)
    cos, sin = emb.cos().to(dtype), emb.sin().to(dtype)
    rq, rk = apply_rotary_pos_emb(q.transpose(1, 2), k.transpose(1, 2), cos, sin)
    T, pos0 = L + 5, 3 if pool == 0 else 0
    qd = q.cuda().clone()
    kc = torch.zeros(B, Hkv, T + pos0, D, dtype=dtype, device="cuda")
    vc = torch.zeros_like(kc)
    _, qp, kp = K.rope_qkv(qd, k.cuda(), v.cuda(), cos.cuda(), sin.cuda(), kc, vc, pos0=pos0, pool_block=pool)
    torch.cuda.synchronize()
    assert torch.equal(qd.transpose(1, 2).cpu(), rq)
    assert torch.equal(kc[:, :, pos0: pos0 + L].cpu(), rk)
    assert torch.equal(vc[:, :, pos0: pos0 + L].cpu(), v.transpose(1, 2))
    if pool:
        np.testing.assert_array_equal(qp.cpu().numpy(), MO.pooled_block_means(rq.float().numpy(), L, pool))
        np.testing.assert_array_equal(kp.cpu().numpy(), MO.pooled_block_means(rk.float().numpy(), L, pool))


# (B, L, hidden, Hq, Hkv, pool_block, pos0, dtype): partial M and N tiles (7 + 2 heads = 4.5 tiles of
# 256 columns), sequences straddling 256-row tiles (B=2, L=200), pooling by 64 and 128, a cache offset.
@pytest.mark.parametrize("B,L,hidden,Hq,Hkv,pool,pos0,dtype", [
    (1, 1000, 512, 4, 2, 64, 0, torch.bfloat16),
    (2, 512, 256, 2, 2, 64, 0, torch.bfloat16),
    (1, 300, 1024, 7, 1, 128, 0, torch.bfloat16),
    (2, 200, 256, 2, 1, 0, 5, torch.bfloat16),
    (1, 257, 384, 2, 2, 64, 0, torch.float16),
])
def test_qkv_proj_rope_matches_projection_and_hf_rope(K, B, L, hidden, Hq, Hkv, pool, pos0, dtype):
    """Fused prefill projection: y = x W^T within bf16/fp16 rounding of an
    fp32 product; q/k rotated bit-exactly as apply_rotary_pos_emb rotates the
    kernel's own y; v stored as y; pools equal the oracle's block means of
    the rotated rows; cache rows outside pos0 .. pos0+L-1 untouched."""
    from transformers.models.llama.modeling_llama import apply_rotary_pos_emb
    gen = torch.Generator().manual_seed(L + hidden + Hq)
    D = 128
    N = (Hq + 2 * Hkv) * D
    x = (torch.randn(B, L, hidden, generator=gen) * 0.5).to(dtype)
    w = (torch.randn(N, hidden, generator=gen) / hidden ** 0.5).to(dtype)
    ang = torch.rand(B, L, D // 2, generator=gen) * 50
    emb = torch.cat([ang, ang], -1)
    cos, sin = emb.cos().to(dtype), emb.sin().to(dtype)
    T = pos0 + L + 3
    sentinel = torch.full((B, Hkv, T, D), 7.0, dtype=dtype)
    kc, vc = sentinel.clone().cuda(), sentinel.clone().cuda()
    q_out = torch.empty(B, L, Hq, D, dtype=dtype, device="cuda")
    y = torch.empty(B * L, N, dtype=dtype, device="cuda")
    qp, kp = K.qkv_proj_rope(x.cuda(), w.cuda(), cos.cuda(), sin.cuda(), q_out, kc, vc, pos0=pos0, pool_block=pool,
                             y_out=y)
    torch.cuda.synchronize()
    ref = (x.float().reshape(B * L, hidden) @ w.float().T)
    yc = y.float().cpu()
    assert (yc - ref).abs().max().item() <= 8e-3 * ref.abs().max().item()
    assert (yc - ref).abs().mean().item() <= 2e-3 * ref.abs().mean().item() + 1e-6
    yv = y.cpu().view(B, L, Hq + 2 * Hkv, D)
    q, k, v = yv[:, :, :Hq], yv[:, :, Hq:Hq + Hkv], yv[:, :, Hq + Hkv:]
    rq, rk = apply_rotary_pos_emb(q.transpose(1, 2), k.transpose(1, 2), cos, sin)
    assert torch.equal(q_out.cpu().transpose(1, 2), rq)
    assert torch.equal(kc[:, :, pos0:pos0 + L].cpu(), rk)
    assert torch.equal(vc[:, :, pos0:pos0 + L].cpu(), v.transpose(1, 2))
    outside = torch.ones(T, dtype=torch.bool)
    outside[pos0:pos0 + L] = False
    assert torch.equal(kc[:, :, outside].cpu(), sentinel[:, :, outside])
    assert torch.equal(vc[:, :, outside].cpu(), sentinel[:, :, outside])
    if pool:
        np.testing.assert_array_equal(qp.cpu().numpy(), MO.pooled_block_means(rq.float().numpy(), L, pool))
        np.testing.assert_array_equal(kp.cpu().numpy(), MO.pooled_block_means(rk.float().numpy(), L, pool))
    assert K.device_status(clear=True) == 0


@pytest.mark.parametrize("L,hidden,Hq,Hkv,pool", [
    (12288, 2048, 16, 16, 64),    # c1: deepseek-coder-1.3B layer
    (16384, 4096, 32, 32, 64),    # c3: 6.7B layer
    (16384, 7168, 56, 8, 128),    # c4: 33B layer (GQA 7:1), pooled by 128
])
def test_qkv_proj_rope_at_the_benched_layer_shapes(K, L, hidden, Hq, Hkv, pool):
    """One layer of each benched model: projection within bf16 rounding of
    cuBLAS, q/k bit-exact with apply_rotary_pos_emb of the kernel's own
    projection, v and the pooled means exact."""
    from transformers.models.llama.modeling_llama import apply_rotary_pos_emb
    gen = torch.Generator(device="cuda").manual_seed(3)
    B, D = 1, 128
    N = (Hq + 2 * Hkv) * D
    x = (torch.randn(B, L, hidden, generator=gen, device="cuda") * 0.5).to(torch.bfloat16)
    w = (torch.randn(N, hidden, generator=gen, device="cuda") / hidden ** 0.5).to(torch.bfloat16)
    ang = torch.rand(1, L, D // 2, generator=gen, device="cuda") * 50
    emb = torch.cat([ang, ang], -1)
    cos, sin = emb.cos().to(torch.bfloat16), emb.sin().to(torch.bfloat16)
    kc = torch.zeros(B, Hkv, L + 64, D, dtype=torch.bfloat16, device="cuda")
    vc = torch.zeros_like(kc)
    q_out = torch.empty(B, L, Hq, D, dtype=torch.bfloat16, device="cuda")
    y = torch.empty(B * L, N, dtype=torch.bfloat16, device="cuda")
    qp, kp = K.qkv_proj_rope(x, w, cos, sin, q_out, kc, vc, pool_block=pool, y_out=y)
    ref = torch.nn.functional.linear(x, w).view(B * L, N)  # cuBLAS, bf16 out
    torch.cuda.synchronize()
    d = (y.float() - ref.float()).abs()
    assert d.max().item() <= 8e-3 * ref.float().abs().max().item()
    yv = y.view(B, L, Hq + 2 * Hkv, D)
    rq, rk = apply_rotary_pos_emb(yv[:, :, :Hq].transpose(1, 2), yv[:, :, Hq:Hq + Hkv].transpose(1, 2), cos, sin)
    assert torch.equal(q_out.transpose(1, 2), rq)
    assert torch.equal(kc[:, :, :L], rk)
    assert torch.equal(vc[:, :, :L], yv[:, :, Hq + Hkv:].transpose(1, 2))
    for h in (0, Hq - 1):
        np.testing.assert_array_equal(qp[:, h:h + 1].cpu().numpy(),
                                      MO.pooled_block_means(rq[:, h:h + 1].float().cpu().numpy(), L, pool))
    np.testing.assert_array_equal(kp[:, Hkv - 1:].cpu().numpy(),
                                  MO.pooled_block_means(rk[:, Hkv - 1:].float().cpu().numpy(), L, pool))
    assert K.device_status(clear=True) == 0
