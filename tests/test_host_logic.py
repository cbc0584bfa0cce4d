"""Host-side text processing of the mask builder against the reference's
recorded token-level inputs (CPU only)."""

import numpy as np
import pytest

import _golden as G
from sabrecoder_b200.chunks import ChunkType, CodeChunk
from sabrecoder_b200.sabrecoder_attention import StructureAwareMaskBuilder, deps_to_csr


def _builder(g, tok=None):
    return StructureAwareMaskBuilder(tok or G.tokenizer(g), **G.params(g))


@pytest.mark.parametrize("case", G.mask_cases())
def test_structure_to_tokens_matches_reference(case):
    g = G.load(case)
    mb = _builder(g)
    t2c, gtm, flags, ptr, idx = mb.structure_to_tokens(
        code=str(g["code"]), seq_len=int(g["seq_len"]), chunks=G.chunks(g), chunk_deps=G.deps(g),
        import_chunks=set(g["import_chunks"].tolist()), language=str(g["language"]) or None)
    np.testing.assert_array_equal(t2c, g["token_to_chunk"])
    np.testing.assert_array_equal(gtm, g["global_token_mask"])
    n = g["chunk_type"].shape[0]
    assert flags.shape == (n,)
    assert set(np.nonzero(flags & 1)[0].tolist()) == {c for c in g["import_chunks"].tolist() if 0 <= c < n}
    assert ptr[0] == 0 and ptr[-1] == idx.shape[0] and (np.diff(ptr) >= 0).all()
    assert ((idx >= 0) & (idx < n)).all()


def test_append_uncovered_line_chunks_matches_reference():
    g = G.load("builder_full.npz")
    from sabrecoder_b200.spans import LineTokenizer
    mb = StructureAwareMaskBuilder(LineTokenizer(), **G.params(g))
    seg = G.chunks(g)
    filled = mb._append_uncovered_line_chunks(str(g["code"]), seg)
    ref = G.chunks(g, "filled_")
    assert len(filled) == len(ref)
    for a, b in zip(filled, ref):
        assert (a.start_line, a.end_line) == (b.start_line, b.end_line)
        assert a.chunk_type.name == b.chunk_type.name


def test_validation_errors_match_reference():
    tok = object()
    with pytest.raises(ValueError, match="block_size"):
        StructureAwareMaskBuilder(tok, block_size=0)
    with pytest.raises(ValueError, match="global_last_k_chunks"):
        StructureAwareMaskBuilder(tok, global_last_k_chunks=-1)
    with pytest.raises(ValueError, match="max_chunk_tokens must be >= 0"):
        StructureAwareMaskBuilder(tok, max_chunk_tokens=-1)
    with pytest.raises(ValueError, match="multiple of block_size"):
        StructureAwareMaskBuilder(tok, max_chunk_tokens=100)
    with pytest.raises(ValueError, match="requires use_chunk_similarity"):
        StructureAwareMaskBuilder(tok, use_crossfile_chunk_similarity=True)
    with pytest.raises(ValueError, match="embedding_weight"):
        StructureAwareMaskBuilder(tok, use_chunk_similarity=True)


def test_deps_to_csr_drops_out_of_range():
    ptr, idx = deps_to_csr({0: {1, 5, -1}, 2: {0}, 9: {1}}, 3)
    assert ptr.tolist() == [0, 1, 1, 2]
    assert idx.tolist() == [1, 0]


def test_map_tokens_last_chunk_wins_and_negative_lines():
    from sabrecoder_b200.spans import LineTokenizer
    from oracle import mask_oracle as MO
    code = "\n".join(f"l{i}" for i in range(10))
    chunks = [CodeChunk(ChunkType.FUNCTION, 0, 0, "", start_line=1, end_line=6),
              CodeChunk(ChunkType.MODULE_CODE, 0, 0, "", start_line=4, end_line=12),
              CodeChunk(ChunkType.MODULE_CODE, 0, 0, "", start_line=-2, end_line=0)]
    mb = StructureAwareMaskBuilder(LineTokenizer())
    got = mb._map_tokens_to_chunks(code, chunks, 12)
    want = MO.map_tokens_to_chunks(code, chunks, LineTokenizer(), 12).tolist()
    assert got == want


def test_precomputed_blocks_round_trip_and_reference_format(tmp_path):
    """Files in the reference evaluator's format ({idx: (indices, counts)},
    torch.save) load, including its int64 unordered rows, and files written
    here load back unchanged."""
    import torch
    from sabrecoder_b200.precomputed import load_precomputed_blocks, precompute_blocks, save_precomputed_blocks
    g = G.load("builder_full.npz")
    raw = torch.from_numpy(g["raw_indices"]).long()      # reference rows: unordered, padded with -1
    cnt = torch.from_numpy(g["block_counts"]).long()
    ref_file = tmp_path / "ref.pt"
    torch.save({0: (raw[:1].clone(), cnt[:1].clone()), 3: (raw[1:].clone(), cnt[1:].clone())}, ref_file)
    got = load_precomputed_blocks(str(ref_file))
    assert sorted(got) == [0, 3]
    assert got[0][0].dtype == torch.int32 and got[0][1].dtype == torch.int32
    assert torch.equal(got[3][0], raw[1:].int()) and torch.equal(got[3][1], cnt[1:].int())
    ours = tmp_path / "ours.pt"
    save_precomputed_blocks(str(ours), got)
    back = torch.load(ours, weights_only=True)
    assert sorted(back) == [0, 3] and torch.equal(back[0][0], got[0][0])
    built = precompute_blocks(lambda i, s: (s[0], s[1], None), [(5, (raw[:1].int(), cnt[:1].int()))])
    assert list(built) == [5] and torch.equal(built[5][0], raw[:1].int())
    bad = tmp_path / "bad.pt"
    torch.save({1: (raw[0, 0], cnt)}, bad)
    with pytest.raises(ValueError):
        load_precomputed_blocks(str(bad))
    torch.save({1: (raw.float(), cnt)}, bad)
    with pytest.raises(TypeError):
        load_precomputed_blocks(str(bad))
