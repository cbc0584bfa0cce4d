"""The CPU oracle against golden vectors recorded from the reference."""

import json
import os

import numpy as np
import pytest
import torch

import _golden as G
from oracle import attention_oracle as AO
from oracle import mask_oracle as MO


@pytest.mark.parametrize("case", G.mask_cases())
def test_mask_from_chunks_matches_reference(case):
    g = G.load(case)
    lang = str(g["language"]) or None
    m = MO.build_block_mask_from_chunks(
        code=str(g["code"]), seq_len=int(g["seq_len"]), chunks=G.chunks(g), chunk_deps=G.deps(g),
        import_chunks=set(g["import_chunks"].tolist()), language=lang, tokenizer=G.tokenizer(g),
        **G.params(g))
    np.testing.assert_array_equal(m, g["block_mask"])


@pytest.mark.parametrize("case", G.mask_cases())
def test_token_level_inputs_match_reference(case):
    g = G.load(case)
    L = int(g["seq_len"])
    lang = str(g["language"]) or None
    ch = G.chunks(g)
    t2c = MO.map_tokens_to_chunks(str(g["code"]), ch, G.tokenizer(g), L)
    np.testing.assert_array_equal(t2c, g["token_to_chunk"])
    gtm = MO.global_token_mask_from_chunks(str(g["code"]), ch, G.tokenizer(g), L, lang)
    np.testing.assert_array_equal(gtm, g["global_token_mask"])


@pytest.mark.parametrize("case", G.mask_cases())
def test_mask_from_tokens_matches_reference(case):
    g = G.load(case)
    p = G.params(g)
    m = MO.build_block_mask_tokens(
        g["token_to_chunk"], g["chunk_type"].shape[0], g["import_chunks"].tolist(), G.deps(g),
        g["global_token_mask"], seq_len=int(g["seq_len"]), **p)
    np.testing.assert_array_equal(m, g["block_mask"])


@pytest.mark.parametrize("case", G.mask_cases() + ["builder_full.npz"])
def test_indices_canonical_form(case):
    g = G.load(case)
    bm = g["block_mask"]
    idx, cnt = MO.block_indices_from_mask(np.broadcast_to(bm, g["block_counts"].shape + bm.shape[-1:]))
    np.testing.assert_array_equal(cnt, g["block_counts"])
    np.testing.assert_array_equal(idx, g["indices_sorted"])
    # the reference's own (unsorted) rows hold the same sets
    raw = g["raw_indices"]
    for r in np.ndindex(*cnt.shape):
        c = int(cnt[r])
        assert sorted(raw[r][:c].tolist()) == idx[r][:c].tolist()
        assert (raw[r][c:] == -1).all()


def test_builder_full_matches_reference():
    g = G.load("builder_full.npz")
    from sabrecoder_b200.spans import LineTokenizer
    seg = G.chunks(g)
    filled = G.chunks(g, "filled_")
    deps = {}
    for s, t in zip(g["edge_src"].tolist(), g["edge_dst"].tolist()):
        deps.setdefault(s, set()).add(t)
        deps.setdefault(t, set()).add(s)
    imports = {i for i, c in enumerate(seg) if c.chunk_type.name == "IMPORT"}
    m = MO.build_block_mask_from_chunks(
        code=str(g["code"]), seq_len=int(g["seq_len"]), chunks=filled, chunk_deps=deps,
        import_chunks=imports, language=None, tokenizer=LineTokenizer(), **G.params(g))
    np.testing.assert_array_equal(m, g["block_mask"])


@pytest.mark.parametrize("case", ["attn_b64.npz", "attn_b128.npz"])
def test_prefill_oracle_matches_reference_kernel(case):
    g = G.load(case)
    q, k, v = (G.bf16_bits_to_f32(g[n]) for n in ("q_bf16", "k_bf16", "v_bf16"))
    out = AO.sparse_prefill_fp32(q, k, v, torch.from_numpy(g["block_indices"]),
                                 torch.from_numpy(g["block_counts"]), int(g["block_size"]))
    ref = torch.from_numpy(g["out"])
    assert (out - ref).abs().max().item() < 2e-5
    # the gathered form (listed blocks only, used for whole-model runs)
    out_g = AO.sparse_prefill_fp32_gathered(q, k, v, torch.from_numpy(g["block_indices"]),
                                            torch.from_numpy(g["block_counts"]), int(g["block_size"]))
    assert (out_g - ref).abs().max().item() < 2e-5
    # and a head subset of the row-chunked form
    H = q.shape[1]
    sub = AO.sparse_prefill_fp32(q, k, v, torch.from_numpy(g["block_indices"]),
                                 torch.from_numpy(g["block_counts"]), int(g["block_size"]), heads=[H - 1],
                                 row_chunk=100)
    assert (sub[:, 0] - ref[:, H - 1]).abs().max().item() < 2e-5


def test_sparsity_utils_values(golden_dir):
    from sabrecoder_b200 import sparsity_utils as SU
    with open(os.path.join(golden_dir, "sparsity_utils.json")) as f:
        vals = json.load(f)
    for m, n, want in vals["causal_total_blocks"]:
        assert SU.causal_total_blocks(m, n) == want
        assert MO.causal_total_blocks(m, n) == want
    for a, b, want in vals["ceil_div"]:
        assert SU.ceil_div(a, b) == want
    km = [0] * 1000
    for i in (3, 70, 71, 500, 999):
        km[i] = 1
    for L, w, bs, want in vals["window_plus_keys"]:
        got = SU.causal_active_blocks_window_plus_keys(L, w, key_token_mask=km[:L] if L == 1000 else None,
                                                         block_size=bs)
        assert list(got) == want
    for L, c, want in vals["attend_ratio_from_cap"]:
        assert abs(SU.causal_attend_ratio_from_cap(L, c) - want) < 1e-12


def test_topk_extension_properties():
    rng = np.random.default_rng(0)
    nb, D = 12, 16
    qm = rng.standard_normal((2, nb, D)).astype(np.float32)
    km = rng.standard_normal((2, nb, D)).astype(np.float32)
    sc = MO.pooled_scores(qm, km)
    base = np.tril(rng.random((nb, nb)) < 0.2) | np.eye(nb, dtype=bool)
    ext = MO.topk_extend_mask(base, sc, 3)
    for h in range(2):
        for qb in range(nb):
            added = ext[h, qb] & ~base[qb]
            assert added.sum() == min(3, int((~base[qb, : qb + 1]).sum()))
            assert not added[qb + 1:].any()
            cand = np.nonzero(~base[qb, : qb + 1])[0]
            if added.any():
                worst_in = sc[h, qb][added].min()
                out = [c for c in cand if not added[c]]
                assert all(sc[h, qb, c] <= worst_in for c in out)


@pytest.mark.parametrize("name", ["a", "b", "c"])
def test_similarity_edges_oracle_matches_reference(name):
    """The oracle's chunk-similarity edges equal the reference's
    _similarity_edges on seeded texts and a bf16 embedding table (fraction and
    percent top_percent, truncation to 5 tokens, source/target subsets, a
    blank chunk and a comment-marker-only chunk)."""
    from sabrecoder_b200.spans import HashTokenizer
    g = G.load("similarity.npz")
    texts, emb, p, src, tgt, want = G.sim_case(g, name)
    got = MO.similarity_edges(texts, HashTokenizer(128), emb, top_percent=p["chunk_similarity_top_percent"],
                              max_tokens=p["chunk_similarity_max_tokens_per_chunk"],
                              max_neighbors=p["chunk_similarity_max_neighbors"], src_indices=src, tgt_indices=tgt)
    assert got == want


def test_similarity_builder_end_to_end_oracle_matches_reference():
    from sabrecoder_b200.spans import HashTokenizer
    g = G.load("similarity.npz")
    chunks = G.chunks(g, "e2e_")
    texts = [str(t) for t in g["e2e_texts"]]
    for c, t in zip(chunks, texts):
        c.text = t
    emb = G.bf16_bits_to_np(g["e2e_emb_bf16"])
    deps = {4: {0}, 0: {4}}
    sim = MO.similarity_edges(texts, HashTokenizer(128), emb,
                              top_percent=g["e2e_p_chunk_similarity_top_percent"].item(),
                              max_tokens=int(g["e2e_p_chunk_similarity_max_tokens_per_chunk"]),
                              max_neighbors=int(g["e2e_p_chunk_similarity_max_neighbors"]))
    for s_, t_ in sim.items():
        deps.setdefault(s_, set()).update(t_)
    mp = {k: int(g[f"e2e_p_{k}"]) for k in ("window_size", "num_prefix_tokens", "num_suffix_tokens", "block_size",
                                          "global_last_k_chunks", "max_chunk_tokens")}
    m = MO.build_block_mask_from_chunks(code=str(g["e2e_code"]), seq_len=int(g["e2e_seq_len"]), chunks=chunks,
                                        chunk_deps=deps, import_chunks=set(), language=None,
                                        tokenizer=HashTokenizer(128), **mp)
    np.testing.assert_array_equal(m, g["e2e_block_mask"])


def test_similarity_reduction_orders_are_fixed():
    """chunk_vectors_f16 / similarity_scores follow their documented orders:
    a shuffled summation gives different low bits somewhere, the documented
    one is reproducible."""
    rng = np.random.default_rng(5)
    emb = rng.standard_normal((50, 300)).astype(np.float32)
    v1 = MO.chunk_vectors_f16(emb, [[1, 2, 3], [], [4]])
    v2 = MO.chunk_vectors_f16(emb, [[1, 2, 3], [], [4]])
    np.testing.assert_array_equal(v1, v2)
    assert not v1[1].any()  # an empty chunk is the zero vector
    n = np.linalg.norm(v1[0].astype(np.float64))
    assert abs(n - 1.0) < 2e-3
    sc = MO.similarity_scores(v1[0], v1)
    assert abs(sc[0] - 1.0) < 5e-3 and sc[1] == 0.0


@pytest.mark.parametrize("case", G.token_cases())
def test_token_level_mask_oracle_matches_reference(case):
    """The oracle's token-level visibility equals the reference's
    _build_mask_from_chunks (lower triangle; the reference's kernel applies
    causality), and its block mask lists exactly the blocks with a visible pair."""
    g = G.load(case)
    want = G.token_visible(g)
    got = MO.token_level_mask_from_chunks(
        code=str(g["code"]), seq_len=int(g["seq_len"]), chunks=G.chunks(g), chunk_deps=G.deps(g),
        import_chunks=set(g["import_chunks"].tolist()), language=str(g["language"]) or None,
        tokenizer=G.tokenizer(g), **G.params(g))
    np.testing.assert_array_equal(got, want)
    if "block_mask" in g:
        # recorded from the non-causal _build_mask_from_chunks; the forward path's
        # mask (build_token_level_mask) is causal, which only drops blocks above
        # the diagonal (a diagonal block is always listed: distance 0 is in the window)
        np.testing.assert_array_equal(MO.block_mask_from_token_mask(want, 64), np.tril(g["block_mask"]).astype(bool))


def test_token_level_attention_oracle_matches_reference_kernel():
    g = G.load("token_attn_256.npz")
    q, k, v = (G.bf16_bits_to_f32(g[n]) for n in ("q_bf16", "k_bf16", "v_bf16"))
    out = AO.token_masked_prefill_fp32(q, k, v, G.token_visible(g))
    assert (out - torch.from_numpy(g["out"])).abs().max().item() < 2e-5
