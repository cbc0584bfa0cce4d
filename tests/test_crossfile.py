"""Cross-file prompts: ``build_block_indices`` / ``build_token_level_mask``
with ``crossfile_code`` and ``current_code`` (reference
methods/sabrecoder/sabrecoder_attention_triton.py:1622-1772, :860-1081).

Fixtures: tests/golden/crossfile.npz, made by tests/golden/gen_golden.py
(``record_crossfile``) from the reference with a fixed segmenter/analyser.
CPU tests check the chunk assembly (segments, line and id shifts, imports,
global context chunk, similarity edges through the oracle) and pin the oracle
on the reference's block and token masks; GPU tests run the library's
builders end to end."""

import numpy as np
import pytest
import torch

import _golden as G
from oracle import mask_oracle as MO
from sabrecoder_b200.sabrecoder_attention import crossfile_segments
from sabrecoder_b200.spans import HashTokenizer

CASES = ["full", "seg", "segjava", "segtok"]
MASK_KEYS = ("block_size", "window_size", "num_prefix_tokens", "num_suffix_tokens", "max_chunk_tokens",
             "global_last_k_chunks")


@pytest.fixture(scope="module")
def fixture():
    return G.load("crossfile.npz")


def _oracle_similarity(c):
    """The builder's _similarity_edges computed by the oracle on the CPU."""
    def edges(chunks, code, *, src_indices=None, tgt_indices=None, top_percent=None):
        if not bool(c["p_use_chunk_similarity"]):
            return {}
        frac = c["p_chunk_similarity_top_percent"].item() if top_percent is None else top_percent
        return MO.similarity_edges([ch.text for ch in chunks], HashTokenizer(128),
                                   G.bf16_bits_to_np(c["emb_bf16"]), top_percent=frac,
                                   max_tokens=int(c["p_chunk_similarity_max_tokens_per_chunk"]),
                                   max_neighbors=int(c["p_chunk_similarity_max_neighbors"]),
                                   src_indices=src_indices, tgt_indices=tgt_indices)
    return edges


def _mask_params(c):
    return {k: int(c[f"p_{k}"]) for k in MASK_KEYS}


@pytest.mark.parametrize("name", CASES)
def test_crossfile_structure_matches_reference(fixture, name):
    """Chunks (types, lines, signature lines, texts), dependency edges
    (analyser + similarity) and import/global chunks equal what the reference
    hands to its mask builder."""
    c = G.crossfile_case(fixture, name)
    mb = G.crossfile_builder(c)
    mb._similarity_edges = _oracle_similarity(c)
    hit = mb._crossfile_structure(str(c["code"]), str(c["crossfile"]), str(c["current"]), None,
                                  bool(c["full_attention"]))
    got, want = hit["chunks"], c["ref_chunks"]
    assert len(got) == len(want)
    for i, (a, b) in enumerate(zip(got, want)):
        assert a.chunk_type.name == b.chunk_type.name, i
        assert (a.start_line, a.end_line) == (b.start_line, b.end_line), i
        assert (a.signature_start_line, a.signature_end_line) == (b.signature_start_line, b.signature_end_line), i
        assert a.text == str(c["ref_texts"][i]), i
    assert {k: v for k, v in hit["chunk_deps"].items() if v} == c["ref_deps"]
    assert hit["import_chunks"] == set(c["ref_imports"].tolist())


@pytest.mark.parametrize("name", CASES)
def test_crossfile_block_mask_oracle_matches_reference(fixture, name):
    """The oracle's block mask over the reference's cross-file structure
    equals the reference's block mask."""
    c = G.crossfile_case(fixture, name)
    code, L = str(c["code"]), int(c["seq_len"])
    tok = HashTokenizer(128)
    chunks = c["ref_chunks"]
    t2c = MO.map_tokens_to_chunks(code, chunks, tok, L)
    gtm = MO.global_token_mask_from_chunks(code, chunks, tok, L, None)
    bm = MO.build_block_mask_tokens(t2c, len(chunks), set(c["ref_imports"].tolist()), c["ref_deps"], gtm,
                                    seq_len=L, **_mask_params(c))
    np.testing.assert_array_equal(bm.astype(np.uint8), c["block_mask"])


def test_crossfile_token_mask_oracle_matches_reference(fixture):
    c = G.crossfile_case(fixture, "segtok")
    L = int(c["seq_len"])
    vis = MO.token_level_mask_from_chunks(code=str(c["code"]), seq_len=L, chunks=c["ref_chunks"],
                                          chunk_deps=c["ref_deps"], import_chunks=set(c["ref_imports"].tolist()),
                                          language=None, tokenizer=HashTokenizer(128), **_mask_params(c))
    np.testing.assert_array_equal(vis, G.token_visible(c))


def test_crossfile_segments_rules():
    """Header lines start segments; a span before the first header is its own
    segment; blank-only spans join the previous segment, else the next one;
    look-alike comment lines are not headers."""
    txt = "\n".join(["", "  ", "# a/b.py: 1 - 9", "# x = 1", "", "#c.py: 1 - 2", "# d.py: 3 - 4  ",
                     "# e: 1 - x", "// f.java: 10 - 20", ""])
    assert [(s, e) for s, e, _ in crossfile_segments(txt)] == [(1, 6), (7, 8), (9, 10)]
    assert crossfile_segments(txt)[0][2] == "\n".join(txt.split("\n")[:6])
    assert [(s, e) for s, e, _ in crossfile_segments("x\n\n# p: 1 - 2\ny")] == [(1, 2), (3, 4)]
    assert [(s, e) for s, e, _ in crossfile_segments("a\nb\n")] == [(1, 3)]
    assert crossfile_segments("\n \n") == []


def test_crossfile_requires_consistent_prompt(fixture):
    c = G.crossfile_case(fixture, "segjava")
    mb = G.crossfile_builder(c)
    with pytest.raises(ValueError, match="does not start with crossfile_code"):
        mb._crossfile_structure("other" + str(c["code"]), str(c["crossfile"]), str(c["current"]), None, False)


@pytest.fixture(scope="module")
def cuda():
    if not torch.cuda.is_available():
        pytest.skip("needs a GPU")
    return torch.device("cuda")


@pytest.mark.gpu
@pytest.mark.parametrize("name", CASES)
def test_crossfile_build_block_indices_matches_reference(fixture, cuda, name):
    """build_block_indices(crossfile_code=, current_code=) end to end on the
    GPU (similarity vectors, top-k and block mask kernels) equals the
    reference's block mask, counts and (sorted) index lists."""
    c = G.crossfile_case(fixture, name)
    mb = G.crossfile_builder(c, device=cuda)
    mb.embedding_weight = mb.embedding_weight.to(cuda)
    mb.clear_cache()
    bi, bc, bm = mb.build_block_indices(str(c["code"]), int(c["seq_len"]), cuda, crossfile_code=str(c["crossfile"]),
                                        current_code=str(c["current"]),
                                        crossfile_full_attention=bool(c["full_attention"]))
    np.testing.assert_array_equal(bm.cpu().numpy().astype(np.uint8), c["block_mask"])
    np.testing.assert_array_equal(bc.cpu().numpy(), c["block_counts"])
    want = c["indices_sorted"]
    np.testing.assert_array_equal(bi.cpu().numpy()[..., :want.shape[-1]], want)


@pytest.mark.gpu
def test_crossfile_token_level_mask_matches_reference(fixture, cuda):
    c = G.crossfile_case(fixture, "segtok")
    mb = G.crossfile_builder(c, device=cuda)
    mb.embedding_weight = mb.embedding_weight.to(cuda)
    mb.clear_cache()
    m = mb.build_token_level_mask(str(c["code"]), int(c["seq_len"]), cuda, torch.float32,
                                  crossfile_code=str(c["crossfile"]), current_code=str(c["current"]),
                                  crossfile_full_attention=bool(c["full_attention"]))
    np.testing.assert_array_equal((m == 0).cpu().numpy(), G.token_visible(c))
