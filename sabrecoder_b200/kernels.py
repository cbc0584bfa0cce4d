"""Torch-facing calls into libsabre_b200.so.

Every function launches the CUDA kernels through the C ABI on the current
stream of the tensors' device. Buffers (outputs and workspaces) are
allocated here through torch's caching allocator; the library itself never
allocates. There is no CPU path: non-CUDA tensors raise.
"""

from __future__ import annotations

import math
from typing import Optional, Tuple

import torch

from ._lib import SabreError, check, i64, lib

DTYPE_CODE = {torch.bfloat16: 0, torch.float16: 1}

# Number of CUDA kernels launched through this module (cumulative).
LAUNCHES = [0]
# When a list, prefill_bsa appends (start_event, end_event, block_counts,
# heads) per launch so callers can time the kernel on its own stream.
PREFILL_EVENTS = None


def set_prefill_timing(on: bool):
    global PREFILL_EVENTS
    PREFILL_EVENTS = [] if on else None
    return PREFILL_EVENTS


def _stream(t: torch.Tensor) -> int:
    return torch.cuda.current_stream(t.device).cuda_stream


def _need_cuda(**tensors) -> None:
    for name, t in tensors.items():
        if t is not None and not t.is_cuda:
            raise SabreError(f"{name} must be a CUDA tensor (got {t.device}); this library has no CPU path")


def _i32(t: torch.Tensor, name: str) -> torch.Tensor:
    if t.dtype != torch.int32:
        raise SabreError(f"{name} must be int32 (got {t.dtype})")
    return t


def _ptr(t: Optional[torch.Tensor]) -> Optional[int]:
    return None if t is None else t.data_ptr()


# ---------------------------------------------------------------------------
# (1) prefill
# ---------------------------------------------------------------------------

def prefill_bsa(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, block_indices: torch.Tensor,
                block_counts: torch.Tensor, block_size: int, softmax_scale: Optional[float] = None,
                out: Optional[torch.Tensor] = None, token_masks=None) -> torch.Tensor:
    """Block-sparse causal attention.

    q: ``[B, Hq, L, D]``; k, v: ``[B, Hkv, L, D]`` (any strides with unit
    head-dim stride, 16-byte aligned); block_indices ``[B, nb, max]`` (shared
    by heads, the reference layout) or ``[B, Hq, nb, max]``; block_counts
    ``[B, nb]`` or ``[B, Hq, nb]``. Returns ``[B, Hq, L, D]`` in q's dtype.

    ``token_masks=(tile_masks, row_ptr)`` (from :func:`token_tile_masks`,
    block size 64) also masks every element of a listed block: the
    token-level variant."""
    _need_cuda(q=q, k=k, v=v, block_indices=block_indices, block_counts=block_counts)
    if token_masks is not None and int(block_size) != 64:
        raise SabreError("the token-level variant needs block_size 64")
    if q.dtype not in DTYPE_CODE or k.dtype != q.dtype or v.dtype != q.dtype:
        raise SabreError(f"q/k/v must share dtype bf16 or f16 (got {q.dtype}, {k.dtype}, {v.dtype})")
    B, Hq, L, D = q.shape
    Hkv = k.shape[1]
    if k.shape != (B, Hkv, L, D) or v.shape != k.shape:
        raise SabreError(f"k/v shape {tuple(k.shape)}/{tuple(v.shape)} does not match q {tuple(q.shape)}")
    bi = _i32(block_indices, "block_indices")
    bc = _i32(block_counts, "block_counts")
    if bi.dim() == 3:
        idx_strides = (bi.stride(0), 0, bi.stride(1), bi.stride(2))
        cnt_strides = (bc.stride(0), 0, bc.stride(1))
    elif bi.dim() == 4:
        if bi.shape[1] not in (1, Hq):
            raise SabreError(f"block_indices head dim {bi.shape[1]} must be 1 or {Hq}")
        idx_strides = (bi.stride(0), bi.stride(1) if bi.shape[1] > 1 else 0, bi.stride(2), bi.stride(3))
        cnt_strides = (bc.stride(0), bc.stride(1) if bc.shape[1] > 1 else 0, bc.stride(2))
    else:
        raise SabreError(f"block_indices must be 3-D or 4-D (got {tuple(bi.shape)})")
    nb = (L + block_size - 1) // block_size
    if bi.shape[0] != B or bi.shape[-2] != nb or bc.shape[-1] != nb:
        raise SabreError(f"index lists {tuple(bi.shape)} / counts {tuple(bc.shape)} do not match B={B}, nb={nb}")
    if out is None:
        out = torch.empty_like(q)
    ev = None
    if PREFILL_EVENTS is not None:
        ev = (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
        ev[0].record(torch.cuda.current_stream(q.device))
    if token_masks is None:
        st = lib().sabre_prefill_bsa(
            q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(), bi.data_ptr(), bc.data_ptr(), B, Hq, Hkv, L,
            D, int(block_size), int(bi.shape[-1]), i64(q.stride()), i64(k.stride()), i64(v.stride()),
            i64(out.stride()), i64(idx_strides), i64(cnt_strides), float(softmax_scale or 0.0), DTYPE_CODE[q.dtype],
            _stream(q))
        check(st, "sabre_prefill_bsa")
    else:
        tm, rp = token_masks
        _need_cuda(tile_masks=tm, row_ptr=rp)
        _i32(rp, "row_ptr")
        st = lib().sabre_prefill_bsa_tokenmask(
            q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(), bi.data_ptr(), bc.data_ptr(), tm.data_ptr(),
            rp.data_ptr(), B, Hq, Hkv, L, D, int(bi.shape[-1]), i64(q.stride()), i64(k.stride()), i64(v.stride()),
            i64(out.stride()), i64(idx_strides), i64(cnt_strides), float(softmax_scale or 0.0), DTYPE_CODE[q.dtype],
            _stream(q))
        check(st, "sabre_prefill_bsa_tokenmask")
    LAUNCHES[0] += 1
    if ev is not None:
        ev[1].record(torch.cuda.current_stream(q.device))
        PREFILL_EVENTS.append((ev[0], ev[1], bc, Hq if bi.dim() == 3 or bi.shape[1] == 1 else 1, int(block_size)))
    return out


def rope_qkv(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor,
             k_out: torch.Tensor, v_out: torch.Tensor, *, q_out: Optional[torch.Tensor] = None, pos0: int = 0,
             pool_block: int = 0):
    """Rotary embedding of q and k plus the K/V store, in one pass.

    q, k, v: ``[B, L, H*, D]`` (unit head-dim stride); cos, sin: ``[B, L, D]``;
    k_out, v_out: ``[B, Hkv, T, D]`` receiving rows ``pos0 .. pos0+L-1``;
    q_out defaults to q (rotated in place). With ``pool_block > 0`` also
    returns fp32 per-block means of the rotated q and k
    (``[B, Hq, nb, D]``, ``[B, Hkv, nb, D]``). Returns ``(q_out, q_pool, k_pool)``."""
    if k_out.dim() != 4 or v_out.shape != k_out.shape or pos0 < 0 or pos0 + q.shape[1] > k_out.shape[2]:
        raise SabreError(f"rope_qkv: rows {pos0}..{pos0 + q.shape[1] - 1} do not fit k_out/v_out of shape "
                         f"{tuple(k_out.shape)} (need [B, Hkv, T, D] with pos0 + L <= T)")
    if q.dim() != 4 or k.dim() != 4 or v.shape != k.shape or k.shape[:2] != q.shape[:2]:
        raise SabreError(f"rope_qkv: q {tuple(q.shape)}, k {tuple(k.shape)}, v {tuple(v.shape)} must be "
                         f"[B, L, H*, D] with one B and L")
    B, L, Hq, D = q.shape
    Hkv = k.shape[2]
    if tuple(k_out.shape[:2]) != (B, Hkv) or k_out.shape[3] != D:
        raise SabreError(f"rope_qkv: k_out/v_out {tuple(k_out.shape)} do not match [B={B}, Hkv={Hkv}, T, D={D}]")
    if cos.dim() not in (2, 3) or sin.shape != cos.shape or cos.shape[-1] != D or cos.shape[-2] < L or (
            cos.dim() == 3 and cos.shape[0] not in (1, B)):
        raise SabreError(f"rope_qkv: cos/sin {tuple(cos.shape)} must be [B or 1, >= L, D] or [>= L, D] "
                         f"(B={B}, L={L}, D={D})")
    _need_cuda(q=q, k=k, v=v, cos=cos, sin=sin, k_out=k_out, v_out=v_out)
    if q.dtype not in DTYPE_CODE or any(t.dtype != q.dtype for t in (k, v, cos, sin, k_out, v_out)):
        raise SabreError("rope_qkv: q/k/v/cos/sin/k_out/v_out must share dtype bf16 or f16")
    if q_out is None:
        q_out = q
    if cos.dim() == 2:
        cos, sin = cos.unsqueeze(0), sin.unsqueeze(0)
    if cos.stride(-1) != 1 or sin.stride() != cos.stride():
        cos, sin = cos.contiguous(), sin.contiguous()
    # One table for every sequence (transformers builds [1, L, D] from shared
    # position ids): batch stride 0, so the kernel never reads past it.
    if cos.shape[0] != B:
        cos, sin = cos.expand(B, -1, -1), sin.expand(B, -1, -1)
    qp = kp = None
    if pool_block > 0:
        nb = (L + pool_block - 1) // pool_block
        qp = torch.empty(B, Hq, nb, D, dtype=torch.float32, device=q.device)
        kp = torch.empty(B, Hkv, nb, D, dtype=torch.float32, device=q.device)

    def s3(t):
        return i64((t.stride(0), t.stride(1), t.stride(2)))

    st = lib().sabre_rope_qkv(
        q.data_ptr(), k.data_ptr(), v.data_ptr(), cos.data_ptr(), sin.data_ptr(), q_out.data_ptr(),
        k_out.data_ptr(), v_out.data_ptr(), _ptr(qp), _ptr(kp), B, L, Hq, Hkv, D, int(pool_block), int(pos0),
        int(k_out.shape[2]), s3(q), s3(k), s3(v), i64((cos.stride(0), cos.stride(1))), s3(q_out), s3(k_out), s3(v_out),
        DTYPE_CODE[q.dtype], _stream(q))
    check(st, "sabre_rope_qkv")
    LAUNCHES[0] += 1
    return q_out, qp, kp


def qkv_proj_rope(x: torch.Tensor, w_qkv: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor,
                  q_out: torch.Tensor, k_out: torch.Tensor, v_out: torch.Tensor, *, pos0: int = 0,
                  pool_block: int = 0, y_out: Optional[torch.Tensor] = None):
    """Prefill q/k/v projection + rotary embedding + KV store (+ pooling) in
    one kernel: ``y = x @ w_qkv.T`` rounded to the storage dtype, then as
    :func:`rope_qkv` on y (same rounding and pooling).

    x: ``[B, L, hidden]`` (unit last stride); w_qkv: ``[(Hq + 2 Hkv) * 128,
    hidden]`` contiguous (``[Wq; Wk; Wv]``); cos, sin: ``[B or 1, >= L, 128]``;
    q_out: ``[B, L, Hq, 128]``; k_out, v_out: ``[B, Hkv, T, 128]`` receiving
    rows ``pos0 .. pos0+L-1``; y_out (optional): ``[B*L, N]`` gets y itself.
    Returns ``(q_pool, k_pool)`` (None unless ``pool_block > 0``)."""
    _need_cuda(x=x, w_qkv=w_qkv, cos=cos, sin=sin, q_out=q_out, k_out=k_out, v_out=v_out, y_out=y_out)
    ts = (x, w_qkv, cos, sin, q_out, k_out, v_out) + ((y_out,) if y_out is not None else ())
    if x.dtype not in DTYPE_CODE or any(t.dtype != x.dtype for t in ts):
        raise SabreError("qkv_proj_rope: all tensors must share dtype bf16 or f16")
    if x.dim() != 3 or x.stride(-1) != 1 or x.stride(0) != x.shape[1] * x.stride(1):
        raise SabreError("qkv_proj_rope: x must be [B, L, hidden] with rows at one stride")
    B, L, hidden = x.shape
    D = q_out.shape[-1]
    Hq = q_out.shape[2]
    Hkv = k_out.shape[1]
    if (q_out.dim() != 4 or tuple(q_out.shape[:2]) != (B, L) or k_out.dim() != 4 or v_out.shape != k_out.shape
            or k_out.shape[0] != B or not w_qkv.is_contiguous()
            or tuple(w_qkv.shape) != ((Hq + 2 * Hkv) * D, hidden)):
        raise SabreError("qkv_proj_rope: shapes do not match x [B, L, hidden], w_qkv [(Hq+2Hkv)*D, hidden], "
                         "q_out [B, L, Hq, D], k_out/v_out [B, Hkv, T, D]")
    if pos0 < 0 or pos0 + L > k_out.shape[2]:
        raise SabreError(f"qkv_proj_rope: rows {pos0}..{pos0 + L - 1} do not fit the cache of {k_out.shape[2]} rows")
    if cos.dim() == 2:
        cos, sin = cos.unsqueeze(0), sin.unsqueeze(0)
    if cos.dim() != 3 or sin.shape != cos.shape or cos.shape[-1] != D or cos.shape[1] < L or cos.shape[0] not in (1, B):
        raise SabreError(f"qkv_proj_rope: cos/sin {tuple(cos.shape)} must be [B or 1, >= L, D]")
    if cos.stride(-1) != 1 or sin.stride() != cos.stride():
        cos, sin = cos.contiguous(), sin.contiguous()
    if cos.shape[0] != B:
        cos, sin = cos.expand(B, -1, -1), sin.expand(B, -1, -1)
    qp = kp = None
    if pool_block > 0:
        nb = (L + pool_block - 1) // pool_block
        qp = torch.empty(B, Hq, nb, D, dtype=torch.float32, device=x.device)
        kp = torch.empty(B, Hkv, nb, D, dtype=torch.float32, device=x.device)

    def s3(t):
        return i64((t.stride(0), t.stride(1), t.stride(2)))

    st = lib().sabre_qkv_proj_rope(
        x.data_ptr(), w_qkv.data_ptr(), cos.data_ptr(), sin.data_ptr(), q_out.data_ptr(), k_out.data_ptr(),
        v_out.data_ptr(), _ptr(qp), _ptr(kp), _ptr(y_out), B, L, hidden, Hq, Hkv, D, int(pool_block), int(pos0),
        int(k_out.shape[2]), x.stride(1), i64((cos.stride(0), cos.stride(1))), s3(q_out), s3(k_out), s3(v_out),
        y_out.stride(0) if y_out is not None else 0, DTYPE_CODE[x.dtype], _stream(x))
    check(st, "sabre_qkv_proj_rope")
    LAUNCHES[0] += 1
    return qp, kp


def qkv_rope_decode(x: torch.Tensor, wq: torch.Tensor, wk: torch.Tensor, wv: torch.Tensor, cos: torch.Tensor,
                    sin: torch.Tensor, q_out: torch.Tensor, k_out: torch.Tensor, v_out: torch.Tensor,
                    pos0: int) -> torch.Tensor:
    """One decode token per sequence: ``q_out = rope(x @ wq.T)``, row ``pos0``
    of ``k_out`` / ``v_out`` = ``rope(x @ wk.T)`` / ``x @ wv.T`` (bias-free
    projections, each output rounded to the storage dtype, rope as in
    ``rope_qkv``).

    x: ``[B, hidden]``; w*: ``[H* * 128, hidden]`` contiguous; cos, sin:
    ``[B, 128]``; q_out: ``[B, Hq, 128]``; k_out, v_out: ``[B, Hkv, T, 128]``.
    Returns q_out."""
    _need_cuda(x=x, wq=wq, wk=wk, wv=wv, cos=cos, sin=sin, q_out=q_out, k_out=k_out, v_out=v_out)
    ts = (x, wq, wk, wv, cos, sin, q_out, k_out, v_out)
    if x.dtype not in DTYPE_CODE or any(t.dtype != x.dtype for t in ts):
        raise SabreError("qkv_rope_decode: all tensors must share dtype bf16 or f16")
    if not (wq.is_contiguous() and wk.is_contiguous() and wv.is_contiguous()):
        raise SabreError("qkv_rope_decode: weights must be contiguous")
    if x.stride(-1) != 1 or cos.stride(-1) != 1 or sin.stride() != cos.stride():
        raise SabreError("qkv_rope_decode: x, cos and sin need unit last stride (cos and sin alike)")
    B, hidden = x.shape
    D = q_out.shape[-1]
    Hq, Hkv = wq.shape[0] // D, wk.shape[0] // D
    T = k_out.shape[2] if k_out.dim() == 4 else 0
    if (wq.shape != (Hq * D, hidden) or wk.shape != (Hkv * D, hidden) or wv.shape != wk.shape
            or tuple(cos.shape) != (B, D) or tuple(q_out.shape) != (B, Hq, D)
            or k_out.dim() != 4 or tuple(k_out.shape) != (B, Hkv, T, D) or v_out.shape != k_out.shape):
        raise SabreError("qkv_rope_decode: shapes do not match x [B, hidden], w [H*D, hidden], cos [B, D], "
                         "q_out [B, Hq, D], k_out/v_out [B, Hkv, T, D]")
    st = lib().sabre_qkv_rope_decode(
        x.data_ptr(), wq.data_ptr(), wk.data_ptr(), wv.data_ptr(), cos.data_ptr(), sin.data_ptr(),
        q_out.data_ptr(), k_out.data_ptr(), v_out.data_ptr(), B, hidden, Hq, Hkv, D, int(pos0), T, x.stride(0),
        cos.stride(0), i64((q_out.stride(0), q_out.stride(1))), i64(k_out.stride()[:3]), i64(v_out.stride()[:3]),
        DTYPE_CODE[x.dtype], _stream(x))
    check(st, "sabre_qkv_rope_decode")
    LAUNCHES[0] += 1
    return q_out


# ---------------------------------------------------------------------------
# (2) decode
# ---------------------------------------------------------------------------

def decode_workspace_bytes(batch: int, heads_q: int, heads_kv: int, head_dim: int, max_active: int) -> int:
    return int(lib().sabre_decode_workspace_size(batch, heads_q, heads_kv, head_dim, max_active))


def decode_bsa(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor, block_indices: torch.Tensor,
               block_counts: torch.Tensor, seq_lens: torch.Tensor, block_size: int,
               softmax_scale: Optional[float] = None, out: Optional[torch.Tensor] = None,
               workspace: Optional[torch.Tensor] = None) -> torch.Tensor:
    """One query row per sequence over the KV cache.

    q: ``[B, Hq, D]``; k_cache, v_cache: ``[B, Hkv, Tmax, D]``;
    block_indices ``[B, max]`` (shared by heads) or ``[B, Hkv, max]``;
    block_counts ``[B]`` or ``[B, Hkv]``; seq_lens int32 ``[B]`` (device)."""
    _need_cuda(q=q, k_cache=k_cache, v_cache=v_cache, block_indices=block_indices, block_counts=block_counts,
               seq_lens=seq_lens)
    if q.dtype not in DTYPE_CODE or k_cache.dtype != q.dtype or v_cache.dtype != q.dtype:
        raise SabreError("q/k_cache/v_cache must share dtype bf16 or f16")
    B, Hq, D = q.shape
    Hkv, Tmax = k_cache.shape[1], k_cache.shape[2]
    bi = _i32(block_indices, "block_indices")
    bc = _i32(block_counts, "block_counts")
    _i32(seq_lens, "seq_lens")
    if bi.dim() == 2:
        idx_strides = (bi.stride(0), 0, bi.stride(1))
        cnt_strides = (bc.stride(0), 0)
    else:
        idx_strides = (bi.stride(0), bi.stride(1) if bi.shape[1] > 1 else 0, bi.stride(2))
        cnt_strides = (bc.stride(0), bc.stride(1) if bc.shape[1] > 1 else 0)
    max_active = int(bi.shape[-1])
    need = decode_workspace_bytes(B, Hq, Hkv, D, max_active)
    if workspace is None or workspace.numel() * workspace.element_size() < need:
        workspace = torch.empty(max(need, 16), dtype=torch.uint8, device=q.device)
    if out is None:
        out = torch.empty_like(q)
    st = lib().sabre_decode_bsa(
        q.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(), out.data_ptr(), bi.data_ptr(), bc.data_ptr(),
        seq_lens.data_ptr(), B, Hq, Hkv, Tmax, D, int(block_size), max_active, i64(q.stride()),
        i64(k_cache.stride()), i64(v_cache.stride()), i64(out.stride()), i64(idx_strides), i64(cnt_strides),
        float(softmax_scale or 0.0), DTYPE_CODE[q.dtype], workspace.data_ptr(),
        workspace.numel() * workspace.element_size(), _stream(q))
    check(st, "sabre_decode_bsa")
    LAUNCHES[0] += 2
    return out


# ---------------------------------------------------------------------------
# (3) mask + index lists
# ---------------------------------------------------------------------------

def build_block_mask(token_to_chunk: torch.Tensor, chunk_flags: torch.Tensor, dep_ptr: torch.Tensor,
                     dep_idx: torch.Tensor, global_token_mask: Optional[torch.Tensor], *, seq_len: int,
                     block_size: int, window_size: int, num_prefix_tokens: int, num_suffix_tokens: int,
                     max_chunk_tokens: int, global_last_k_chunks: int,
                     dense: bool = True) -> Tuple[torch.Tensor, Optional[torch.Tensor]]:
    """Block mask from token-level structure. Returns ``(bits, dense)``:
    bits int32 ``[nb, ceil(nb/32)]`` (uint32 words), dense int32 ``[nb, nb]``."""
    _need_cuda(token_to_chunk=token_to_chunk, chunk_flags=chunk_flags, dep_ptr=dep_ptr, dep_idx=dep_idx,
               global_token_mask=global_token_mask)
    dev = token_to_chunk.device
    nchunks = int(chunk_flags.numel())
    nb = (seq_len + block_size - 1) // block_size
    nwords = (nb + 31) // 32
    bits = torch.empty(nb, nwords, dtype=torch.int32, device=dev)
    dm = torch.empty(nb, nb, dtype=torch.int32, device=dev) if dense else None
    ws_bytes = int(lib().sabre_block_mask_workspace_size(nchunks, nb))
    ws = torch.empty(max(ws_bytes, 16), dtype=torch.uint8, device=dev)
    if global_token_mask is not None and global_token_mask.dtype != torch.uint8:
        global_token_mask = global_token_mask.to(torch.uint8)
    st = lib().sabre_build_block_mask(
        _i32(token_to_chunk, "token_to_chunk").data_ptr(), _ptr(global_token_mask),
        chunk_flags.data_ptr() if nchunks else None, nchunks, _i32(dep_ptr, "dep_ptr").data_ptr(),
        _i32(dep_idx, "dep_idx").data_ptr() if dep_idx.numel() else None, int(seq_len), int(block_size),
        int(window_size), int(num_prefix_tokens), int(num_suffix_tokens), int(max_chunk_tokens),
        int(global_last_k_chunks), bits.data_ptr(), _ptr(dm), ws.data_ptr(), ws.numel(), _stream(bits))
    check(st, "sabre_build_block_mask")
    LAUNCHES[0] += 2
    return bits, dm


def indices_from_bits(bits: torch.Tensor, ncols: int, cap: Optional[int] = None):
    """Ascending index lists from row bitsets ``[..., nwords]``. Returns
    ``(indices [..., cap], counts [...], max_active device int32[1])``."""
    _need_cuda(bits=bits)
    lead = bits.shape[:-1]
    rows = int(math.prod(lead)) if lead else 1
    cap = int(ncols if cap is None else cap)
    b = bits.reshape(rows, bits.shape[-1]).contiguous()
    idx = torch.empty(rows, cap, dtype=torch.int32, device=bits.device)
    cnt = torch.empty(rows, dtype=torch.int32, device=bits.device)
    mx = torch.empty(1, dtype=torch.int32, device=bits.device)
    check(lib().sabre_indices_from_bits(b.data_ptr(), rows, int(ncols), idx.data_ptr(), cap, cnt.data_ptr(),
                                        mx.data_ptr(), _stream(bits)), "sabre_indices_from_bits")
    LAUNCHES[0] += 1
    return idx.reshape(*lead, cap), cnt.reshape(lead), mx


def indices_from_dense(mask: torch.Tensor, cap: Optional[int] = None):
    """Ascending index lists from a dense mask ``[..., nb, ncols]`` (nonzero =
    active). Returns ``(indices [..., nb, cap], counts [..., nb], max_active)``."""
    _need_cuda(mask=mask)
    m = mask if mask.dtype == torch.int32 else mask.to(torch.int32)
    lead = m.shape[:-1]
    ncols = int(m.shape[-1])
    rows = int(math.prod(lead))
    m2 = m.reshape(rows, ncols)
    if m2.stride(-1) != 1:
        m2 = m2.contiguous()
    cap = int(ncols if cap is None else cap)
    idx = torch.empty(rows, cap, dtype=torch.int32, device=m.device)
    cnt = torch.empty(rows, dtype=torch.int32, device=m.device)
    mx = torch.empty(1, dtype=torch.int32, device=m.device)
    check(lib().sabre_indices_from_dense(m2.data_ptr(), rows, ncols, m2.stride(0), idx.data_ptr(), cap,
                                         cnt.data_ptr(), mx.data_ptr(), _stream(m)), "sabre_indices_from_dense")
    LAUNCHES[0] += 1
    return idx.reshape(*lead, cap), cnt.reshape(lead), mx


def pool_blocks(x: torch.Tensor, block_size: int) -> torch.Tensor:
    """Per-block mean of ``x [B, H, L, D]`` -> fp32 ``[B, H, nb, D]`` (rows
    summed first to last in fp32, then divided by the row count)."""
    _need_cuda(x=x)
    B, H, L, D = x.shape
    nb = (L + block_size - 1) // block_size
    out = torch.empty(B, H, nb, D, dtype=torch.float32, device=x.device)
    check(lib().sabre_pool_blocks(x.data_ptr(), B, H, L, D, int(block_size), i64(x.stride()), DTYPE_CODE[x.dtype],
                                  out.data_ptr(), _stream(x)), "sabre_pool_blocks")
    LAUNCHES[0] += 1
    return out


def topk_extend(q_pooled: torch.Tensor, k_pooled: torch.Tensor, base_bits: torch.Tensor, topk: int,
                cap: Optional[int] = None, want_bits: bool = False):
    """Per-(b, head) lists = base rows plus the top-k pooled-score blocks.
    Returns ``(indices [B, Hq, nb, cap], counts [B, Hq, nb], max_active, bits|None)``."""
    _need_cuda(q_pooled=q_pooled, k_pooled=k_pooled, base_bits=base_bits)
    B, Hq, nb, D = q_pooled.shape
    Hkv = k_pooled.shape[1]
    qp = q_pooled.contiguous()
    kp = k_pooled.contiguous()
    bb = base_bits.contiguous()
    cap = int(nb if cap is None else cap)
    idx = torch.empty(B, Hq, nb, cap, dtype=torch.int32, device=qp.device)
    cnt = torch.empty(B, Hq, nb, dtype=torch.int32, device=qp.device)
    mx = torch.empty(1, dtype=torch.int32, device=qp.device)
    ob = torch.empty(B, Hq, nb, bb.shape[-1], dtype=torch.int32, device=qp.device) if want_bits else None
    ws_bytes = int(lib().sabre_topk_workspace_size(B, Hq, nb))
    ws = torch.empty(max(ws_bytes, 16), dtype=torch.uint8, device=qp.device)
    check(lib().sabre_topk_extend(qp.data_ptr(), kp.data_ptr(), bb.data_ptr(), B, Hq, Hkv, nb, D, int(topk),
                                  idx.data_ptr(), cap, cnt.data_ptr(), mx.data_ptr(), _ptr(ob), ws.data_ptr(),
                                  ws.numel(), _stream(qp)),
          "sabre_topk_extend")
    LAUNCHES[0] += 2
    return idx, cnt, mx, ob


def device_status(clear: bool = True, stream: Optional[int] = None) -> int:
    import ctypes
    v = ctypes.c_uint(0)
    s = stream if stream is not None else (torch.cuda.current_stream().cuda_stream if torch.cuda.is_available()
                                           else None)
    check(lib().sabre_device_status(ctypes.byref(v), 1 if clear else 0, s), "sabre_device_status")
    return int(v.value)


def set_wait_limit_ns(ns: int) -> None:
    """Limit of the kernels' bounded waits on the current device, in ns
    (0 restores the default of 2 s). A wait that runs out records
    SABRE_DEV_TIMEOUT (read with device_status); the kernel drains what it
    issued and exits without writing its output tile."""
    check(lib().sabre_set_wait_limit_ns(int(ns)), "sabre_set_wait_limit_ns")


# ---------------------------------------------------------------------------
# (3d) chunk-similarity edges
# ---------------------------------------------------------------------------

_EMB_CODE = {torch.bfloat16: 0, torch.float16: 1, torch.float32: 2}


def chunk_vectors(embedding: torch.Tensor, tok_ptr: torch.Tensor, tok_ids: torch.Tensor) -> torch.Tensor:
    """fp16 ``[nchunks, dim]`` unit vectors: the fp32 mean of each chunk's
    embedding rows, L2-normalised (sabre_chunk_vectors). ``tok_ptr`` int32
    ``[nchunks + 1]`` and ``tok_ids`` int32 are CSR token lists on the
    embedding's device."""
    _need_cuda(embedding=embedding, tok_ptr=tok_ptr, tok_ids=tok_ids)
    if embedding.dtype not in _EMB_CODE or embedding.dim() != 2:
        raise SabreError("embedding must be a 2-D bf16, f16 or f32 tensor")
    emb = embedding.contiguous()
    _i32(tok_ptr, "tok_ptr")
    _i32(tok_ids, "tok_ids")
    n = tok_ptr.numel() - 1
    out = torch.empty(max(n, 0), emb.shape[1], dtype=torch.float16, device=emb.device)
    st = lib().sabre_chunk_vectors(emb.data_ptr(), _EMB_CODE[emb.dtype], emb.shape[0], emb.shape[1],
                                   tok_ptr.data_ptr(), tok_ids.data_ptr() if tok_ids.numel() else None, n,
                                   out.data_ptr(), _stream(emb))
    check(st, "sabre_chunk_vectors")
    LAUNCHES[0] += 1
    return out


def similarity_topk(vecs: torch.Tensor, src_rows: torch.Tensor, src_chunk: torch.Tensor, tgt_rows: torch.Tensor,
                    tgt_chunk: torch.Tensor, k: int) -> torch.Tensor:
    """int32 ``[nsrc, k]``: for each source the target chunk ids of its ``k``
    best-scoring targets (sabre_similarity_topk); -1 for the chunk itself and
    unused slots."""
    _need_cuda(vecs=vecs, src_rows=src_rows, tgt_rows=tgt_rows)
    if vecs.dtype != torch.float16 or not vecs.is_contiguous():
        raise SabreError("vecs must be contiguous fp16")
    for name, t in (("src_rows", src_rows), ("src_chunk", src_chunk), ("tgt_rows", tgt_rows),
                    ("tgt_chunk", tgt_chunk)):
        _i32(t, name)
    ns, nt = src_rows.numel(), tgt_rows.numel()
    out = torch.empty(ns, k, dtype=torch.int32, device=vecs.device)
    st = lib().sabre_similarity_topk(vecs.data_ptr(), vecs.shape[1], src_rows.data_ptr(), src_chunk.data_ptr(), ns,
                                     tgt_rows.data_ptr(), tgt_chunk.data_ptr(), nt, int(k), out.data_ptr(),
                                     _stream(vecs))
    check(st, "sabre_similarity_topk")
    LAUNCHES[0] += 1
    return out


# ---------------------------------------------------------------------------
# (3e) token-level sparsity
# ---------------------------------------------------------------------------

def token_block_mask(tok_chunk: torch.Tensor, tok_group: torch.Tensor, tok_global: torch.Tensor,
                     dep_bits: torch.Tensor, nchunks: int, window: int) -> torch.Tensor:
    """uint32-as-int32 ``[nb, ceil(nb/32)]`` row bitsets of the blocks (64)
    holding any visible token pair (sabre_token_block_mask)."""
    _need_cuda(tok_chunk=tok_chunk, tok_group=tok_group, tok_global=tok_global, dep_bits=dep_bits)
    L = tok_chunk.numel()
    nb = (L + 63) // 64
    bits = torch.empty(nb, (nb + 31) // 32, dtype=torch.int32, device=tok_chunk.device)
    st = lib().sabre_token_block_mask(tok_chunk.data_ptr(), tok_group.data_ptr(), tok_global.data_ptr(),
                                      dep_bits.data_ptr() if dep_bits.numel() else None, int(nchunks), L, int(window),
                                      bits.data_ptr(), _stream(tok_chunk))
    check(st, "sabre_token_block_mask")
    LAUNCHES[0] += 1
    return bits


def token_tile_masks(tok_chunk: torch.Tensor, tok_group: torch.Tensor, tok_global: torch.Tensor,
                     dep_bits: torch.Tensor, nchunks: int, window: int, indices: torch.Tensor,
                     counts: torch.Tensor):
    """``(tile_masks int64 [total, 64], row_ptr int32 [nb])``: the 64-bit key
    masks of the 64 query rows of every listed (query block, key block) pair,
    in list order (sabre_token_tile_masks). ``indices`` ``[nb, cap]``
    ascending, ``counts`` ``[nb]``."""
    _need_cuda(indices=indices, counts=counts)
    _i32(indices, "indices")
    _i32(counts, "counts")
    L = tok_chunk.numel()
    csum = torch.cumsum(counts.long(), 0)
    total = int(csum[-1].item()) if csum.numel() else 0
    row_ptr = (csum - counts.long()).to(torch.int32).contiguous()
    masks = torch.empty(max(total, 1), 64, dtype=torch.int64, device=indices.device)
    st = lib().sabre_token_tile_masks(tok_chunk.data_ptr(), tok_group.data_ptr(), tok_global.data_ptr(),
                                      dep_bits.data_ptr() if dep_bits.numel() else None, int(nchunks), L, int(window),
                                      indices.data_ptr(), int(indices.shape[-1]), counts.data_ptr(), row_ptr.data_ptr(),
                                      masks.data_ptr(), _stream(indices))
    check(st, "sabre_token_tile_masks")
    LAUNCHES[0] += 1
    return masks, row_ptr
