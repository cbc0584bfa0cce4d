"""GPU parity at the shapes the benchmark reports.

The prefill kernel (replacing ``_fwd_kernel_sabrecoder``,
methods/sabrecoder/sabrecoder_attention_triton.py:28-116, launched at
:2039-2053) runs on one layer's full shape of each workload with the lists
the benchmark builds for it, and a subset of heads (always including the
last KV-head group) is checked against the oracle over every query row:

* c1: deepseek-coder-1.3B attention, L=12288, 16 heads, block 64,
  structure lists + per-head pooled top-8;
* c2: the same at a ragged prompt length (14001 tokens);
* c3: 6.7B attention, L=16384, 32 heads, block 64, structure + top-8;
* c4: 33B attention, L=16384, 56 query / 8 KV heads, block 128, structure
  lists only.

Tolerance (bf16): max-abs 2e-2, mean-abs 2e-3. The per-head top-8 lists are
also compared with the oracle's (bit-exact) at the c1 and c3 shapes, and the
token-level variant runs on the c1 prompt against the oracle's dense token
mask (lists bit-exact, two heads over every row). Decode attention runs at
the decode-op benchmark's c1 / c3 / c4 shapes, dense and sparse lists, from a
CUDA graph as the benchmark times it.
"""

import numpy as np
import pytest
import torch

import bench
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


def _qkv(Hq, Hkv, L, seed):
    """Seeded bf16 q/k/v in the projection's [B, L, H, D] memory, viewed as
    [B, H, L, D] (the layout the patched model hands the kernel)."""
    dev = torch.device("cuda")
    g = torch.Generator(device=dev).manual_seed(seed)
    q = torch.randn(1, L, Hq, 128, device=dev, generator=g, dtype=torch.bfloat16).transpose(1, 2)
    k = torch.randn(1, L, Hkv, 128, device=dev, generator=g, dtype=torch.bfloat16).transpose(1, 2)
    v = torch.randn(1, L, Hkv, 128, device=dev, generator=g, dtype=torch.bfloat16).transpose(1, 2)
    return q, k, v


def _bench_lists(K, name, q, k, L):
    """The lists bench.py builds for the workload: structure spans with the
    workload's mix and mask parameters, then the pooled top-k per head."""
    from sabrecoder_b200.sabrecoder_attention import StructureAwareMaskBuilder
    from sabrecoder_b200.spans import BENCH_SPAN_MIX, make_spans
    mask, topk = bench.mask_cfg(name)
    mix = bench.C4_SPAN_MIX if name == "c4" else BENCH_SPAN_MIX
    seed = {"c1": 1000, "c2": 2000, "c3": 3000, "c4": 4000}[name]
    spans = make_spans(L, seed, **mix)
    mb = StructureAwareMaskBuilder(None, **mask)
    bi, bc, bm = mb.build_block_indices_from_spans(spans, torch.device("cuda"))
    blk = mask["block_size"]
    if topk:
        qm, km = K.pool_blocks(q, blk), K.pool_blocks(k, blk)
        idx, cnt, mx, _ = K.topk_extend(qm, km, mb.last_block_bits, topk)
        bi = idx[..., :int(mx.item())].contiguous()
        bc = cnt
    return bi, bc, bm, blk, topk


def _check(out, q, k, v, bi, bc, blk, heads):
    ref = AO.sparse_prefill_fp32(q.cpu(), k.cpu(), v.cpu(), bi.cpu(), bc.cpu(), blk, heads=heads)
    got = out[:, heads].float().cpu()
    d = (got - ref).abs()
    assert d.max().item() <= MAX_ABS, f"max-abs {d.max().item():.3e} over heads {heads}"
    assert d.mean().item() <= MEAN_ABS, f"mean-abs {d.mean().item():.3e} over heads {heads}"
    # every query row produced output (no tile skipped): rows with listed keys are non-zero
    assert torch.isfinite(got).all()


@pytest.mark.parametrize("name,Hq,Hkv,L,heads", [
    ("c1", 16, 16, 12288, [0, 7, 15]),
    # one of config 2's prompt lengths (12288-16384), not a multiple of 64 or 128
    ("c2", 16, 16, 14001, [0, 15]),
    ("c3", 32, 32, 16384, [0, 31]),
    ("c4", 56, 8, 16384, [0, 6, 49, 55]),
])
def test_prefill_at_benched_shape(K, name, Hq, Hkv, L, heads):
    q, k, v = _qkv(Hq, Hkv, L, seed=7)
    bi, bc, bm, blk, topk = _bench_lists(K, name, q, k, L)
    out = torch.empty(1, L, Hq, 128, device=q.device, dtype=q.dtype).transpose(1, 2)
    K.prefill_bsa(q, k, v, bi, bc, blk, out=out)
    torch.cuda.synchronize()
    assert K.device_status(clear=True) == 0
    _check(out, q, k, v, bi, bc, blk, heads)
    nb = (L + blk - 1) // blk
    dens = float(bc.sum().item()) / (bc.numel() // nb * nb * (nb + 1) / 2)
    print(f"{name}: L={L} Hq={Hq} Hkv={Hkv} block {blk} density {dens:.4f} max_active {bi.shape[-1]}")


@pytest.mark.parametrize("name,H,L", [("c1", 16, 12288), ("c3", 32, 16384)])
def test_topk_lists_match_oracle(K, name, H, L):
    """The per-head pooled top-8 lists of the c1 and c3 shapes equal the
    oracle's (pooled fp32 block means, fixed-order scores, ties to the lower
    block)."""
    q, k, v = _qkv(H, H, L, seed=7)
    bi, bc, bm, blk, topk = _bench_lists(K, name, q, k, L)
    qm = MO.pooled_block_means(q.float().cpu().numpy(), L, blk)
    km = MO.pooled_block_means(k.float().cpu().numpy(), L, blk)
    ext = MO.topk_extend_mask(bm.cpu().numpy().astype(bool), MO.pooled_scores(qm, km), topk)
    idx, cnt = MO.block_indices_from_mask(ext)
    np.testing.assert_array_equal(bc.cpu().numpy(), cnt)
    got = bi.cpu().numpy()
    for h in range(H):
        for r in range(ext.shape[-2]):
            c = int(cnt[0, h, r])
            np.testing.assert_array_equal(got[0, h, r, :c], idx[0, h, r, :c])


def test_token_mode_at_the_c1_prompt(K):
    """The token-level variant (use_token_level_sparsity; the reference's
    _fwd_kernel_sabrecoder_token_sparse, sabrecoder_attention_triton.py:119-215)
    on the c1 prompt: 12288 tokens with the benchmark's structure spans, the
    block lists and per-pair 64x64 masks built on the GPU from the token rule.
    The lists equal the blocks of the oracle's dense token mask, and two heads
    match the oracle's token-masked attention over every query row."""
    from sabrecoder_b200.spans import BENCH_SPAN_MIX, make_spans
    L, H, blk = 12288, 2, 64
    spans = make_spans(L, 1000, **BENCH_SPAN_MIX)
    t2c, grp, glob, dep, n = bench._token_rule_from_spans(spans, bench.MASK)
    dev = torch.device("cuda")

    def up(a, dt):
        return torch.as_tensor(np.ascontiguousarray(a), dtype=dt).to(dev)

    tc, tg, tgl = up(t2c, torch.int32), up(grp, torch.int32), up(glob, torch.uint8)
    db = up(dep.view(np.int32), torch.int32)
    w = bench.MASK["window_size"]
    bits = K.token_block_mask(tc, tg, tgl, db, n, w)
    nb = bits.shape[0]
    idx, cnt, mx = K.indices_from_bits(bits, nb)
    lists = idx[:, :max(int(mx.item()), 1)].contiguous()
    masks = K.token_tile_masks(tc, tg, tgl, db, n, w, lists, cnt)
    q, k, v = _qkv(H, H, L, seed=11)
    out = K.prefill_bsa(q, k, v, lists[None], cnt[None], blk, token_masks=masks)
    torch.cuda.synchronize()
    assert K.device_status(clear=True) == 0

    vis = MO.token_level_mask_tokens(spans.token_to_chunk(), len(spans.spans), spans.import_chunks, spans.deps,
                                     spans.signature_token_mask(), seq_len=L, **bench.MASK)
    ref_idx, ref_cnt = MO.block_indices_from_mask(MO.block_mask_from_token_mask(vis, blk))
    np.testing.assert_array_equal(cnt.cpu().numpy(), ref_cnt)
    got_lists = lists.cpu().numpy()
    for r in range(nb):
        c = int(ref_cnt[r])
        np.testing.assert_array_equal(got_lists[r, :c], ref_idx[r, :c])

    qc, kc, vc, got = q.cpu(), k.cpu(), v.cpu(), out.float().cpu()
    dmax, dsum = 0.0, 0.0
    for r0 in range(0, L, 2048):
        r1 = min(L, r0 + 2048)
        ref = AO.token_masked_prefill_fp32(qc[:, :, r0:r1], kc[:, :, :r1], vc[:, :, :r1],
                                           torch.from_numpy(vis[r0:r1, :r1]))
        d = (got[:, :, r0:r1] - ref).abs()
        dmax, dsum = max(dmax, d.max().item()), dsum + d.sum().item()
    assert dmax <= MAX_ABS, f"max-abs {dmax:.3e}"
    assert dsum / got.numel() <= MEAN_ABS, f"mean-abs {dsum / got.numel():.3e}"


@pytest.mark.parametrize("name", ["c1", "c3", "c4"])
@pytest.mark.parametrize("lists", ["dense", "sparse"])
def test_decode_at_benched_shape(K, name, lists):
    """Decode attention at the shapes the decode-op benchmark reports (c1:
    16 heads, 12288 + 64 cached tokens; c3: 32 heads, 16384 + 128; c4: 56
    query / 8 KV heads, block 128, 16384 + 64), dense lists (the reference
    decodes densely, sabrecoder_llama_triton.py:254-268) and the sparse lists
    the benchmark builds (the last prompt row's structure list plus every
    generated block). As the benchmark times it, the calls run from one CUDA
    graph over two layer caches (the split kernels are programmatic dependent
    launches); both outputs are checked against the oracle."""
    from sabrecoder_b200.sabrecoder_attention import StructureAwareMaskBuilder
    from sabrecoder_b200.spans import BENCH_SPAN_MIX, make_spans
    Hq, H, L, gen = bench.DECODE_SHAPES[name]
    mask, _ = bench.mask_cfg(name)
    blk = mask["block_size"]
    T = L + gen
    dev = torch.device("cuda")
    g = torch.Generator(device=dev).manual_seed(21)
    caches = [tuple(torch.randn(1, H, T, 128, device=dev, generator=g, dtype=torch.bfloat16) for _ in range(2))
              for _ in range(2)]
    q = torch.randn(1, Hq, 128, device=dev, generator=g, dtype=torch.bfloat16)
    nbk = (T + blk - 1) // blk
    if lists == "dense":
        lst = torch.arange(nbk, device=dev, dtype=torch.int32).unsqueeze(0)
    else:
        mb = StructureAwareMaskBuilder(None, **mask)
        mix = bench.C4_SPAN_MIX if name == "c4" else BENCH_SPAN_MIX
        bi, bc, _ = mb.build_block_indices_from_spans(make_spans(L, 1000, **mix), dev)
        nb_p = (L + blk - 1) // blk
        c_last = int(bc[0, nb_p - 1].item())
        lst = torch.cat([bi[0, nb_p - 1, :c_last].to(torch.int32),
                         torch.arange(nb_p, nbk, device=dev, dtype=torch.int32)]).unsqueeze(0).contiguous()
    cnt = torch.tensor([lst.shape[1]], dtype=torch.int32, device=dev)
    seq = torch.tensor([T], dtype=torch.int32, device=dev)
    ws = torch.empty(K.decode_workspace_bytes(1, Hq, H, 128, lst.shape[1]), dtype=torch.uint8, device=dev)
    outs = [torch.empty_like(q) for _ in caches]

    def step():
        for (kc, vc), o in zip(caches, outs):
            K.decode_bsa(q, kc, vc, lst, cnt, seq, blk, out=o, workspace=ws)

    step()
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        with torch.cuda.graph(graph, stream=side):
            step()
    torch.cuda.current_stream().wait_stream(side)
    for o in outs:
        o.zero_()
    graph.replay()
    torch.cuda.synchronize()
    assert K.device_status(clear=True) == 0
    for (kc, vc), o in zip(caches, outs):
        ref = AO.sparse_decode_fp32(q.cpu(), kc.cpu(), vc.cpu(), lst.cpu(), cnt.cpu(), seq.cpu(), blk)
        d = (o.float().cpu() - ref).abs()
        assert d.max().item() <= MAX_ABS and d.mean().item() <= MEAN_ABS, (d.max().item(), d.mean().item())
    del graph
