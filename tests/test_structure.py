"""The built-in Python segmenter and reference analyser against the
reference's TreeSitterSegmenter / CrossReferenceAnalyzer rules
(methods/sabrecoder/semantic_chunker.py, reference_graph.py), recorded in
tests/golden/structure.npz by tests/golden/gen_golden.py (``record_structure``,
which runs the reference's classes over the standard ast parse)."""

import numpy as np
import pytest

import _golden as G
from sabrecoder_b200.structure import PythonReferenceAnalyzer, PythonSegmenter, detect_language


@pytest.fixture(scope="module")
def fixture():
    return G.load("structure.npz")


def _case(g, name):
    return {k[len(name) + 1:]: v for k, v in g.items() if k.startswith(name + "_")}


@pytest.mark.parametrize("name", ["s0", "s1", "s2", "s3"])
def test_segmenter_matches_reference_rules(fixture, name):
    c = _case(fixture, name)
    code = str(c["code"])
    chunks = PythonSegmenter().segment_code(code, language="python")
    want = G.chunks(c)
    assert len(chunks) == len(want)
    for i, (a, b) in enumerate(zip(chunks, want)):
        assert a.chunk_type.name == b.chunk_type.name, i
        assert (a.start_line, a.end_line) == (b.start_line, b.end_line), i
        assert (a.signature_start_line, a.signature_end_line) == (b.signature_start_line, b.signature_end_line), i
        assert (a.start, a.end) == (int(c["start"][i]), int(c["end"][i])), i
        assert (a.name or "") == b.name and (a.parent_name or "") == str(c["parent"][i]), i
        assert a.text == str(c["text"][i]), i


@pytest.mark.parametrize("name", ["s0", "s1", "s2", "s3"])
def test_analyzer_matches_reference_rules(fixture, name):
    c = _case(fixture, name)
    code = str(c["code"])
    chunks = PythonSegmenter().segment_code(code, language="python")
    refs = PythonReferenceAnalyzer(chunks, code, language="python").analyze()
    got = sorted((r.source_chunk_idx, r.target_chunk_idx, r.line_number, r.name) for r in refs)
    want = list(zip(c["ref_src"].tolist(), c["ref_dst"].tolist(), c["ref_line"].tolist(),
                    [str(x) for x in c["ref_name"]]))
    assert got == want


def test_language_detection_and_non_python():
    assert detect_language("using System;\nclass A {}") == "c_sharp"
    assert detect_language("package a;\nimport java.util.List;") == "java"
    assert detect_language("package a;\npublic class B {}") == "c_sharp"  # C# markers are checked first
    assert detect_language("x = 1") == "python"
    with pytest.raises(ValueError, match="Python only"):
        PythonSegmenter().segment_code("package a;\npublic class B {}")
    assert PythonSegmenter().segment_code("   \n") == []


def test_truncated_source_keeps_the_parsed_prefix():
    """A prompt cut inside a statement: the line the error is on is
    neutralised, so the definitions around it keep their chunks and their
    references."""
    code = "import os\n\ndef f(x):\n    return g(x)\n\ndef g(y):\n    return (y +\n"
    chunks = PythonSegmenter().segment_code(code)
    kinds = [(c.chunk_type.name, c.start_line, c.end_line) for c in chunks]
    assert kinds == [("IMPORT", 1, 2), ("FUNCTION", 3, 5), ("FUNCTION", 6, 8)]
    refs = PythonReferenceAnalyzer(chunks, code).analyze()
    assert [(r.source_chunk_idx, r.target_chunk_idx, r.name) for r in refs] == [(1, 2, "g")]


def test_syntax_errors_cost_only_their_lines():
    """Python 2 print statements inside and between definitions: every
    definition still becomes a chunk, and calls elsewhere are still found."""
    code = ("import os\n\ndef f(x):\n    print 'hi'\n    return g(x)\n\nprint x\n\nclass K:\n"
            "    def m(self):\n        return f(1)\n\ndef g(y):\n    return y\n")
    chunks = PythonSegmenter().segment_code(code)
    got = [(c.chunk_type.name, c.name, c.start_line, c.end_line) for c in chunks]
    assert got == [("MODULE_CODE", "", 6, 8), ("IMPORT", "import", 1, 2), ("FUNCTION", "f", 3, 5),
                   ("CLASS", "K", 9, 12), ("METHOD", "m", 10, 11), ("FUNCTION", "g", 13, 15)]
    refs = PythonReferenceAnalyzer(chunks, code).analyze()
    assert sorted((r.source_chunk_idx, r.target_chunk_idx, r.name) for r in refs) == [(2, 5, "g"), (4, 2, "f")]


def test_builder_uses_builtin_structure_without_tree_sitter():
    """build_block_indices(code) on Python source needs no segmenter factory
    when tree-sitter is absent; the structure equals the built-in classes'."""
    from sabrecoder_b200.sabrecoder_attention import StructureAwareMaskBuilder
    from sabrecoder_b200.spans import HashTokenizer
    mb = StructureAwareMaskBuilder(HashTokenizer(128))
    code = "import os\n\ndef f(x):\n    return g(x)\n\ndef g(y):\n    return y\n"
    hit = mb._structure_for_code(code, "python")
    names = [(c.chunk_type.name, c.name) for c in hit["chunks"]]
    assert names[:3] == [("IMPORT", "import"), ("FUNCTION", "f"), ("FUNCTION", "g")]
    assert hit["import_chunks"] == {0}
    assert hit["chunk_deps"] == {1: {2}, 2: {1}}


@pytest.mark.gpu
@pytest.mark.parametrize("name", ["s0", "s1"])
def test_build_block_indices_on_python_source(fixture, name):
    """build_block_indices(code, ..., language="python") on raw Python source
    with the built-in structure: the block mask and counts equal the
    reference's (its segmenter and analyser rules, special lines on)."""
    import torch
    if not torch.cuda.is_available():
        pytest.skip("needs a GPU")
    from sabrecoder_b200.sabrecoder_attention import StructureAwareMaskBuilder
    from sabrecoder_b200.spans import HashTokenizer
    c = _case(fixture, name)
    p = {k[2:]: int(c[k]) for k in c if k.startswith("p_")}
    mb = StructureAwareMaskBuilder(HashTokenizer(128), **p)
    mb.clear_cache()
    dev = torch.device("cuda")
    _, bc, bm = mb.build_block_indices(str(c["code"]), int(c["seq_len"]), dev, language="python")
    np.testing.assert_array_equal(bm.cpu().numpy().astype(np.uint8), c["block_mask"])
    np.testing.assert_array_equal(bc.cpu().numpy(), c["block_counts"])


def test_block_mask_oracle_on_python_source(fixture):
    """The oracle's block mask over the built-in structure equals the
    reference's build_block_indices on the same source (CPU)."""
    from oracle import mask_oracle as MO
    from sabrecoder_b200.spans import HashTokenizer
    for name in ("s0", "s1"):
        c = _case(fixture, name)
        code, L = str(c["code"]), int(c["seq_len"])
        p = {k[2:]: int(c[k]) for k in c if k.startswith("p_")}
        chunks = PythonSegmenter().segment_code(code, language="python")
        deps = {}
        for r in PythonReferenceAnalyzer(chunks, code, language="python").analyze():
            deps.setdefault(r.source_chunk_idx, set()).add(r.target_chunk_idx)
            deps.setdefault(r.target_chunk_idx, set()).add(r.source_chunk_idx)
        imports = {i for i, ch in enumerate(chunks) if ch.chunk_type.name == "IMPORT"}
        tok = HashTokenizer(128)
        t2c = MO.map_tokens_to_chunks(code, chunks, tok, L)
        gtm = MO.global_token_mask_from_chunks(code, chunks, tok, L, "python")
        bm = MO.build_block_mask_tokens(t2c, len(chunks), imports, deps, gtm, seq_len=L, **p)
        np.testing.assert_array_equal(bm.astype(np.uint8), c["block_mask"])
