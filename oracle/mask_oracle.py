"""Oracle (test infrastructure only): CPU restatement of the reference's
block-mask and block-index construction.

Only tests, ``__graft_entry__.smoke()`` and the CPU-baseline leg of
``bench.py`` use this module, and only as a checker. The library's product
path never imports it.

Parity is pinned against golden fixtures produced by running the reference
itself (``tests/golden/gen_golden.py`` imports
methods/sabrecoder/sabrecoder_attention_triton.py with tree-sitter stubbed and
records its outputs).

Every function cites the reference code it restates. Arithmetic is plain
numpy; the mask is a dense ``bool[nb, nb]`` here, which is only practical for
the test sizes (nb <= a few thousand).
"""

from __future__ import annotations

import re
from typing import Dict, Iterable, List, Optional, Sequence, Set, Tuple

import numpy as np

_SIG_TYPES = {"FUNCTION", "CLASS", "METHOD"}


def _type_name(ct) -> str:
    return getattr(ct, "name", str(ct)).upper()


# --------------------------------------------------------------------------
# Token-level core: sabrecoder_attention_triton.py:1455-1604
# --------------------------------------------------------------------------

def chunk_block_sets(token_to_chunk: np.ndarray, nchunks: int, seq_len: int, block: int) -> np.ndarray:
    """``chunk_blocks`` as a bool matrix ``[nchunks, nb]``
    (sabrecoder_attention_triton.py:1479-1490): block ``b`` belongs to chunk
    ``c`` iff some token ``t`` in ``[b*B, (b+1)*B)`` has ``token_to_chunk[t] == c``."""
    nb = (seq_len + block - 1) // block
    cb = np.zeros((max(nchunks, 0), nb), dtype=bool)
    t2c = np.asarray(token_to_chunk[:seq_len], dtype=np.int64)
    tok = np.arange(t2c.shape[0])
    ok = (t2c >= 0) & (t2c < nchunks)
    cb[t2c[ok], tok[ok] // block] = True
    return cb


def build_block_mask_tokens(
    token_to_chunk: np.ndarray,
    nchunks: int,
    import_chunks: Iterable[int],
    chunk_deps: Dict[int, Iterable[int]],
    global_token_mask: Optional[np.ndarray],
    *,
    seq_len: int,
    block_size: int,
    window_size: int,
    num_prefix_tokens: int,
    num_suffix_tokens: int,
    max_chunk_tokens: int,
    global_last_k_chunks: int,
) -> np.ndarray:
    """Block mask ``int32[nb, nb]`` from token-level structure
    (sabrecoder_attention_triton.py:1455-1604, rules R0-R3 then ``tril``)."""
    B = int(block_size)
    L = int(seq_len)
    nb = (L + B - 1) // B
    mask = np.zeros((nb, nb), dtype=bool)
    cb = chunk_block_sets(token_to_chunk, nchunks, L, B)

    # R0 sliding window (:1492-1500)
    w = int(window_size)
    for qb in range(nb):
        j_min = max(0, qb * B - w) // B
        if j_min <= qb:
            mask[qb, j_min : qb + 1] = True

    # R1 within-chunk visibility (:1502-1525)
    if max_chunk_tokens > 0:
        bpg = max(1, int(max_chunk_tokens) // B)
        grp = np.arange(nb) // bpg
        same = grp[:, None] == grp[None, :]
        for c in range(nchunks):
            blk = cb[c]
            if blk.any():
                mask |= blk[:, None] & blk[None, :] & same
    else:
        for c in range(nchunks):
            blk = cb[c]
            if blk.any():
                mask |= blk[:, None] & blk[None, :]

    # R2 chunk dependencies (:1527-1544)
    for src, tgts in (chunk_deps or {}).items():
        src = int(src)
        if not (0 <= src < nchunks):
            continue
        sb = cb[src]
        if not sb.any():
            continue
        tb = np.zeros(nb, dtype=bool)
        for t in tgts:
            t = int(t)
            if 0 <= t < nchunks:
                tb |= cb[t]
        if tb.any():
            mask |= sb[:, None] & tb[None, :]

    # R3 globally visible key columns (:1546-1600)
    cols = np.zeros(nb, dtype=bool)
    for c in import_chunks or ():
        c = int(c)
        if 0 <= c < nchunks:
            cols |= cb[c]
    if global_token_mask is not None:
        g = np.nonzero(np.asarray(global_token_mask[:L]).astype(bool))[0]
        cols[g // B] = True
    p = min(int(num_prefix_tokens), L)
    if p > 0:
        cols[: (p - 1) // B + 1] = True
    s = min(int(num_suffix_tokens), L)
    if s > 0:
        cols[max(0, L - s) // B :] = True
    k = int(global_last_k_chunks)
    if k > 0 and nchunks > 0:
        for c in range(max(0, nchunks - k), nchunks):
            cols |= cb[c]
    mask[:, cols] = True

    # causal in block space (:1602-1604)
    return np.tril(mask).astype(np.int32)


# --------------------------------------------------------------------------
# Chunk/line front end: sabrecoder_attention_triton.py:407-456, 697-858
# --------------------------------------------------------------------------

def _char_to_line(code: str) -> List[int]:
    out: List[int] = []
    for i, ln in enumerate(code.split("\n")):
        out.extend([i + 1] * (len(ln) + 1))
    return out


def token_to_line(code: str, tokenizer, seq_len: int) -> List[int]:
    """sabrecoder_attention_triton.py:407-447 (uncached)."""
    c2l = _char_to_line(code)
    enc = tokenizer(code, add_special_tokens=True, truncation=True, max_length=seq_len,
                    return_offsets_mapping=True)
    offs, ids = enc.get("offset_mapping"), enc.get("input_ids")
    if offs is None or ids is None:
        raise RuntimeError("tokenizer must return offset_mapping and input_ids")
    out = [0] * seq_len
    for t in range(min(seq_len, len(ids))):
        sc, _ = offs[t]
        if sc is None or sc < 0:
            continue
        if not c2l:
            out[t] = 1
            continue
        out[t] = c2l[min(sc, len(c2l) - 1)]
    return out


def map_tokens_to_chunks(code: str, chunks: Sequence, tokenizer, seq_len: int) -> np.ndarray:
    """sabrecoder_attention_triton.py:807-858: token -> line -> chunk, the last
    chunk in list order wins for a line (:818-821)."""
    t2c = np.full(seq_len, -1, dtype=np.int32)
    if not chunks:
        return t2c
    lines = code.split("\n")
    nl = len(lines)
    l2c = [-1] * (nl + 1)
    for ci, ch in enumerate(chunks):
        for ln in range(ch.start_line, ch.end_line + 1):
            if ln <= nl:
                l2c[ln] = ci
    enc = tokenizer(code, add_special_tokens=True, truncation=True, max_length=seq_len,
                    return_offsets_mapping=True)
    offs, ids = enc.get("offset_mapping"), enc.get("input_ids")
    if offs is None or ids is None:
        raise RuntimeError("tokenizer must return offset_mapping and input_ids")
    if len(offs) < len(ids):
        raise RuntimeError("offset_mapping shorter than input_ids")
    if not ids:
        return t2c
    c2l = _char_to_line(code)
    for t in range(min(seq_len, len(ids))):
        sc, _ = offs[t]
        if sc is None or sc < 0:
            continue
        cp = min(sc, len(c2l) - 1) if c2l else 0
        ln = c2l[cp] if c2l else 1
        if ln < len(l2c):
            t2c[t] = l2c[ln]
    return t2c


def identify_special_lines(code: str, chunks: Sequence, language: Optional[str]) -> Set[int]:
    """Union of the four line sets of sabrecoder_attention_triton.py:697-752."""
    if language is None or str(language).lower() not in {"python", "py"}:
        return set()
    lines = code.split("\n")
    fc_lines: Set[int] = set()
    init_lines: Set[int] = set()
    for ch in chunks:
        tn = _type_name(ch.chunk_type)
        if tn in _SIG_TYPES:
            fc_lines.update(range(ch.start_line, ch.end_line + 1))
        if tn == "METHOD" and getattr(ch, "name", "") == "__init__":
            init_lines.update(range(ch.start_line, ch.end_line + 1))
    out: Set[int] = set()
    for i, line in enumerate(lines):
        n = i + 1
        st = line.strip()
        if not st or st.startswith("#"):
            continue
        if n not in fc_lines:
            if "=" in st and not any(kw in st for kw in ("==", "!=", "<=", ">=", "def ", "class ", "import ", "from ")):
                if re.match(r"^[A-Za-z_][A-Za-z0-9_]*\s*[:\[]?\s*=", st):
                    out.add(n)
        if "TypeAlias" in st or re.match(r"^[A-Z][A-Za-z0-9_]*\s*=\s*[A-Z][A-Za-z0-9_]*\[", st):
            out.add(n)
        if n in init_lines and re.match(r"^\s*self\.[A-Za-z_][A-Za-z0-9_]*\s*=", line):
            out.add(n)
        if n in fc_lines and re.match(r"^\s*return\b", st):
            out.add(n)
    return out


def global_token_mask_from_chunks(code: str, chunks: Sequence, tokenizer, seq_len: int,
                                  language: Optional[str]) -> np.ndarray:
    """Tokens on signature lines and special lines
    (sabrecoder_attention_triton.py:1557-1572 with :449-456)."""
    vis: Set[int] = set()
    for ch in chunks:
        if _type_name(ch.chunk_type) in _SIG_TYPES:
            s0 = getattr(ch, "signature_start_line", None)
            s1 = getattr(ch, "signature_end_line", None)
            if s0 and s1:
                vis.update(range(s0, s1 + 1))
    vis |= identify_special_lines(code, chunks, language)
    m = np.zeros(seq_len, dtype=np.uint8)
    if not vis:
        return m
    t2l = token_to_line(code, tokenizer, seq_len)
    for t, ln in enumerate(t2l):
        if ln in vis:
            m[t] = 1
    return m


def build_block_mask_from_chunks(*, code: str, seq_len: int, chunks: Sequence,
                                 chunk_deps: Dict[int, Set[int]], import_chunks: Set[int],
                                 language: Optional[str], tokenizer, block_size: int,
                                 window_size: int, num_prefix_tokens: int,
                                 num_suffix_tokens: int, max_chunk_tokens: int,
                                 global_last_k_chunks: int) -> np.ndarray:
    """Whole of ``_build_block_mask_from_chunks`` (sabrecoder_attention_triton.py:1455-1604)."""
    t2c = map_tokens_to_chunks(code, chunks, tokenizer, seq_len)
    gtm = global_token_mask_from_chunks(code, chunks, tokenizer, seq_len, language)
    return build_block_mask_tokens(
        t2c, len(chunks), import_chunks, chunk_deps, gtm, seq_len=seq_len,
        block_size=block_size, window_size=window_size, num_prefix_tokens=num_prefix_tokens,
        num_suffix_tokens=num_suffix_tokens, max_chunk_tokens=max_chunk_tokens,
        global_last_k_chunks=global_last_k_chunks)


# --------------------------------------------------------------------------
# Index lists: sabrecoder_attention_triton.py:1837-1859
# --------------------------------------------------------------------------

def block_indices_from_mask(mask: np.ndarray) -> Tuple[np.ndarray, np.ndarray]:
    """``compute_block_indices_from_mask`` in canonical form.

    ``mask`` has shape ``[..., nb, nb]``. Counts are the row sums;
    ``max_active = max(max(counts), 1)``; each row lists its active columns in
    ascending order, padded with -1. (The reference uses an unstable argsort,
    so its within-row order is arbitrary; the set per row is the same.)"""
    m = np.asarray(mask).astype(bool)
    counts = m.sum(-1).astype(np.int32)
    max_active = max(int(counts.max()) if counts.size else 0, 1)
    lead = m.shape[:-1]
    idx = np.full(lead + (max_active,), -1, dtype=np.int32)
    flat_m = m.reshape(-1, m.shape[-1])
    flat_i = idx.reshape(-1, max_active)
    for r in range(flat_m.shape[0]):
        nz = np.nonzero(flat_m[r])[0]
        flat_i[r, : nz.shape[0]] = nz
    return idx, counts


def mask_from_indices(idx: np.ndarray, counts: np.ndarray, nb: int) -> np.ndarray:
    """Inverse of :func:`block_indices_from_mask`: entries ``i < count`` that
    fall in ``[0, nb)`` set the column (duplicates collapse)."""
    idx = np.asarray(idx)
    counts = np.asarray(counts)
    lead = counts.shape
    m = np.zeros(lead + (nb,), dtype=bool)
    fi = idx.reshape(-1, idx.shape[-1])
    fc = counts.reshape(-1)
    fm = m.reshape(-1, nb)
    for r in range(fc.shape[0]):
        e = fi[r, : max(0, int(fc[r]))]
        e = e[(e >= 0) & (e < nb)]
        fm[r, e] = True
    return m


def causal_total_blocks(m: int, n: Optional[int] = None) -> int:
    """utils/sparsity_utils.py:29-46."""
    n = m if n is None else n
    if m <= 0 or n <= 0:
        return 0
    if m <= n:
        return m * (m + 1) // 2
    return n * (n + 1) // 2 + (m - n) * n


def density(mask2d: np.ndarray) -> float:
    """Active lower-triangle blocks over causal-eligible blocks
    (sabrecoder_llama_triton.py:140-160)."""
    m = np.asarray(mask2d)
    tot = causal_total_blocks(m.shape[0], m.shape[1])
    return float(np.tril(m).astype(bool).sum()) / tot if tot else 0.0


# --------------------------------------------------------------------------
# Pooled q.k top-k extension (no reference counterpart; its nearest analogue
# is the chunk-similarity top-k of sabrecoder_attention_triton.py:581-682:
# mean-pool, score, keep the top-k per source, self excluded).
# --------------------------------------------------------------------------

def pooled_block_means(x: np.ndarray, seq_len: int, block: int) -> np.ndarray:
    """Mean over the rows of each block, in fp32 with a fixed order: rows are
    summed first to last (one fp32 rounding per add), then divided by the row
    count (one rounding). ``x`` is ``[..., L, D]`` holding bf16 values."""
    x = np.asarray(x, dtype=np.float32)
    L = int(seq_len)
    nb = (L + block - 1) // block
    lead = x.shape[:-2]
    D = x.shape[-1]
    s = np.zeros(lead + (nb, D), dtype=np.float32)
    for r in range(block):
        rows = np.arange(nb) * block + r
        ok = rows < L
        if not ok.any():
            continue
        s[..., ok, :] = s[..., ok, :] + x[..., rows[ok], :]
    n = np.minimum(block, L - np.arange(nb) * block).astype(np.float32)
    return (s / n[:, None]).astype(np.float32)


def pooled_scores(qm: np.ndarray, km: np.ndarray) -> np.ndarray:
    """``score[..., i, j] = sum_d qm[..., i, d] * km[..., j, d]`` in fp32 with
    the products rounded to fp32 and added in order d = 0, 1, ... (no fused
    multiply-add)."""
    qm = np.asarray(qm, dtype=np.float32)
    km = np.asarray(km, dtype=np.float32)
    D = qm.shape[-1]
    acc = np.zeros(qm.shape[:-1] + (km.shape[-2],), dtype=np.float32)
    for d in range(D):
        acc = acc + (qm[..., :, d][..., :, None] * km[..., :, d][..., None, :]).astype(np.float32)
    return acc


def topk_extend_mask(mask: np.ndarray, scores: np.ndarray, topk: int) -> np.ndarray:
    """Add to each row ``qb`` the ``topk`` best causal blocks ``kb <= qb`` that
    the row does not already hold, best = higher score, ties to the lower kb.

    ``mask``: ``[..., nb, nb]`` (broadcast against ``scores``' leading dims);
    ``scores``: ``[..., nb, nb]``. Returns bool ``[..., nb, nb]``."""
    scores = np.asarray(scores, dtype=np.float32)
    m = np.broadcast_to(np.asarray(mask).astype(bool), scores.shape).copy()
    nb = scores.shape[-1]
    fm = m.reshape(-1, nb, nb)
    fs = scores.reshape(-1, nb, nb)
    for r in range(fm.shape[0]):
        for qb in range(nb):
            cand = np.nonzero(~fm[r, qb, : qb + 1])[0]
            if cand.size == 0 or topk <= 0:
                continue
            sc = fs[r, qb, cand]
            order = np.lexsort((cand, -sc))
            fm[r, qb, cand[order[:topk]]] = True
    return m


# ---------------------------------------------------------------------------
# Chunk-similarity edges (sabrecoder_attention_triton.py:458-682)
# ---------------------------------------------------------------------------

def clean_for_similarity(text: str) -> str:
    """Drop a leading "# " or "// " from every line (reference :458-472)."""
    out = []
    for ln in text.split("\n"):
        if ln.startswith("# "):
            out.append(ln[2:])
        elif ln.startswith("// "):
            out.append(ln[3:])
        else:
            out.append(ln)
    return "\n".join(out)


def tokenize_for_similarity(tokenizer, texts, max_tokens: int):
    """Token id lists as the reference obtains them (:526-554): one batched
    call with truncation and padding (ids where the attention mask is set),
    else ``encode`` per text cut to ``max_tokens``."""
    try:
        enc = tokenizer(texts, add_special_tokens=False, truncation=True, max_length=int(max_tokens),
                        padding=True, return_tensors="pt")
        ids, am = enc.get("input_ids", None), enc.get("attention_mask", None)
        if ids is None or am is None:
            raise RuntimeError("no input_ids/attention_mask")
        ids = np.asarray(ids)
        am = np.asarray(am)
        return [[int(t) for t, m in zip(ids[r], am[r]) if m] for r in range(ids.shape[0])]
    except Exception:  # noqa: BLE001 -- the reference falls back on any failure
        out = []
        for t in texts:
            e = tokenizer.encode(t, add_special_tokens=False) if t and t.strip() else []
            out.append([int(x) for x in e[: int(max_tokens)]])
        return out


def chunk_vectors_f16(embedding: np.ndarray, token_lists) -> np.ndarray:
    """fp16 unit vectors of the chunks' mean token embeddings, every fp32
    reduction in the order sabre_chunk_vectors uses: tokens added first to
    last; squares of d = t, t+256, ... added in order per t, then a halving
    tree over the 256 partials; v / max(sqrt(.), 1e-12)."""
    emb = np.asarray(embedding, dtype=np.float32)
    V, D = emb.shape
    T = 256
    P = (D + T - 1) // T
    out = np.zeros((len(token_lists), D), dtype=np.float16)
    for c, ids in enumerate(token_lists):
        s = np.zeros(D, dtype=np.float32)
        for i in ids:
            if 0 <= int(i) < V:
                s = (s + emb[int(i)]).astype(np.float32)
        m = (s / np.float32(max(len(ids), 1))).astype(np.float32)
        pad = np.zeros(P * T, dtype=np.float32)
        pad[:D] = m
        sq = (pad * pad).astype(np.float32).reshape(P, T)
        part = np.zeros(T, dtype=np.float32)
        for i in range(P):
            part = (part + sq[i]).astype(np.float32)
        h = T // 2
        while h > 0:
            part[:h] = (part[:h] + part[h:2 * h]).astype(np.float32)
            h //= 2
        denom = np.maximum(np.sqrt(part[0]).astype(np.float32), np.float32(1e-12))
        out[c] = (m / denom).astype(np.float32).astype(np.float16)
    return out


def similarity_scores(a16: np.ndarray, b16: np.ndarray) -> np.ndarray:
    """fp32 dot products of one fp16 vector with rows of ``b16`` in the order
    sabre_similarity_topk uses: lane l of 32 adds the products of
    d = l, l+32, ... in order, then an xor tree with strides 16, 8, 4, 2, 1."""
    W = 32
    D = a16.shape[0]
    P = (D + W - 1) // W
    pa = np.zeros(P * W, dtype=np.float32)
    pa[:D] = a16.astype(np.float32)
    pb = np.zeros((b16.shape[0], P * W), dtype=np.float32)
    pb[:, :D] = b16.astype(np.float32)
    prod = (pb * pa).astype(np.float32).reshape(b16.shape[0], P, W)
    lane = np.zeros((b16.shape[0], W), dtype=np.float32)
    for i in range(P):
        lane = (lane + prod[:, i, :]).astype(np.float32)
    idx = np.arange(W)
    for o in (16, 8, 4, 2, 1):
        lane = (lane + lane[:, idx ^ o]).astype(np.float32)
    return lane[:, 0]


def similarity_topk(vecs16: np.ndarray, src_rows, src_chunks, tgt_rows, tgt_chunks, k: int):
    """Per source, the target chunk ids of the min(k, ntgt) best scores
    (descending, ties to the lower target position), the chunk itself -1."""
    tr = np.asarray(tgt_rows, dtype=np.int64)
    tc = np.asarray(tgt_chunks, dtype=np.int64)
    out = []
    for r, c in zip(src_rows, src_chunks):
        sc = similarity_scores(vecs16[int(r)], vecs16[tr])
        sc = np.where(tc == int(c), np.float32(-np.inf), sc)
        order = sorted(range(len(tc)), key=lambda j: (-float(sc[j]), j))[: min(int(k), len(tc))]
        out.append([-1 if int(tc[j]) == int(c) else int(tc[j]) for j in order])
    return out


def similarity_edges(chunk_texts, tokenizer, embedding, *, top_percent: float, max_tokens: int,
                     max_neighbors: int, src_indices=None, tgt_indices=None):
    """Directed chunk-similarity edges {src: {tgt}} (reference :581-682)."""
    frac = float(top_percent)
    if frac > 1.0:
        frac /= 100.0
    frac = max(0.0, min(1.0, frac))
    if int(max_neighbors) <= 0 or frac <= 0.0:
        return {}
    n = len(chunk_texts)
    src = list(range(n)) if src_indices is None else list(src_indices)
    tgt = list(range(n)) if tgt_indices is None else list(tgt_indices)
    texts, idx_map = [], []
    for i, t in enumerate(chunk_texts):
        cl = clean_for_similarity(t or "")
        if cl and cl.strip():
            texts.append(cl)
            idx_map.append(i)
    if not idx_map:
        return {}
    vecs = chunk_vectors_f16(embedding, tokenize_for_similarity(tokenizer, texts, max_tokens))
    row_of = {c: r for r, c in enumerate(idx_map)}
    sr = [(c, row_of[c]) for c in src if c in row_of]
    tg = [(c, row_of[c]) for c in tgt if c in row_of]
    if not sr or not tg:
        return {}
    k = min(int(max_neighbors), int(np.floor(len(tg) * frac)))
    if k <= 0:
        return {}
    picks = similarity_topk(vecs, [r for _, r in sr], [c for c, _ in sr], [r for _, r in tg], [c for c, _ in tg], k)
    edges = {}
    for (c, _), row in zip(sr, picks):
        for t in row:
            if t >= 0:
                edges.setdefault(int(c), set()).add(int(t))
    return edges


# ---------------------------------------------------------------------------
# Token-level mask (sabrecoder_attention_triton.py:1171-1266) and its block
# mask (compute_block_mask_from_token_mask :1862-1885). Dense bool [L, L]:
# only for the small sizes the tests use.
# ---------------------------------------------------------------------------

def token_level_mask_tokens(token_to_chunk: np.ndarray, nchunks: int, import_chunks, chunk_deps,
                            global_token_mask: Optional[np.ndarray], *, seq_len: int, block_size: int,
                            window_size: int, num_prefix_tokens: int, num_suffix_tokens: int,
                            max_chunk_tokens: int, global_last_k_chunks: int) -> np.ndarray:
    """``visible[i, j]`` following the reference's steps in order: sliding
    window, same chunk (or same max_chunk_tokens group), chunk dependencies,
    import chunks, signature/special lines, prefix, suffix, last-k chunks,
    then causality."""
    L = int(seq_len)
    t2c = np.asarray(token_to_chunk, dtype=np.int64)[:L]
    pos = np.arange(L)
    dist = pos[:, None] - pos[None, :]
    m = (dist >= 0) & (dist <= int(window_size))
    ci, cj = t2c[:, None], t2c[None, :]
    if max_chunk_tokens > 0:
        bpg = max(1, int(max_chunk_tokens) // int(block_size))
        gidx = (pos // int(block_size)) // bpg
        ng = int(gidx.max()) + 2
        gid = t2c * ng + gidx
        m |= (gid[:, None] == gid[None, :]) & (ci != -1) & (cj != -1)
    else:
        m |= (ci == cj) & (ci != -1)
    for s, tg in (chunk_deps or {}).items():
        if not (0 <= int(s) < nchunks):
            continue
        src = t2c == int(s)
        if not src.any():
            continue
        tgt = np.zeros(L, dtype=bool)
        for t in tg:
            if 0 <= int(t) < nchunks:
                tgt |= t2c == int(t)
        m |= src[:, None] & tgt[None, :]
    for c in import_chunks or ():
        m[:, t2c == int(c)] = True
    if global_token_mask is not None:
        m[:, np.asarray(global_token_mask, dtype=bool)[:L]] = True
    npre = min(int(num_prefix_tokens), L)
    if npre > 0:
        m[:, :npre] = True
    nsuf = min(int(num_suffix_tokens), L)
    if nsuf > 0:
        m[:, max(0, L - nsuf):] = True
    k = int(global_last_k_chunks)
    if k > 0 and nchunks > 0:
        for c in range(max(0, nchunks - k), nchunks):
            m[:, t2c == c] = True
    return m & (dist >= 0)


def token_level_mask_from_chunks(*, code: str, seq_len: int, chunks: Sequence, chunk_deps, import_chunks,
                                 language: Optional[str], tokenizer, block_size: int, window_size: int,
                                 num_prefix_tokens: int, num_suffix_tokens: int, max_chunk_tokens: int,
                                 global_last_k_chunks: int) -> np.ndarray:
    """Whole of ``_build_mask_from_chunks`` as a bool visibility matrix."""
    t2c = map_tokens_to_chunks(code, chunks, tokenizer, seq_len)
    gtm = global_token_mask_from_chunks(code, chunks, tokenizer, seq_len, language)
    return token_level_mask_tokens(t2c, len(chunks), import_chunks, chunk_deps, gtm, seq_len=seq_len,
                                   block_size=block_size, window_size=window_size,
                                   num_prefix_tokens=num_prefix_tokens, num_suffix_tokens=num_suffix_tokens,
                                   max_chunk_tokens=max_chunk_tokens, global_last_k_chunks=global_last_k_chunks)


def block_mask_from_token_mask(visible: np.ndarray, block: int) -> np.ndarray:
    """Block (i, j) is listed iff any of its token pairs is visible."""
    L = visible.shape[0]
    nb = (L + block - 1) // block
    pad = np.zeros((nb * block, nb * block), dtype=bool)
    pad[:L, :L] = visible
    return pad.reshape(nb, block, nb, block).any(axis=(1, 3))
