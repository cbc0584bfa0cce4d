/*
 * sabre_b200.h -- C ABI of libsabre_b200.so, the sm_100a (B200) kernels
 * behind SabreCoder's structure-aware block-sparse attention path.
 *
 * Conventions for every entry point:
 *  - Plain pointers and sizes; all tensors are device pointers unless stated
 *    otherwise; the caller allocates every buffer (no entry point allocates
 *    device memory).
 *  - Strides are in ELEMENTS, int64, in the order given by each function.
 *  - `stream` is a cudaStream_t passed as void* (NULL = legacy default).
 *  - Work is stream-ordered; entry points validate arguments on the host and
 *    return SABRE_OK (0) or a negative sabre_status_t WITHOUT launching on
 *    error. `sabre_last_error()` gives a message for the calling thread.
 *  - Kernels never trap. A bounded device-side wait that runs out records
 *    SABRE_DEV_TIMEOUT in a device status word (see sabre_device_status).
 *  - dtype: SABRE_BF16 or SABRE_F16 for Q/K/V/O; index lists are int32.
 */
#ifndef SABRE_B200_H_
#define SABRE_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum {
  SABRE_OK = 0,
  SABRE_ERR_INVALID_ARG = -1,  /* bad pointer, size or stride */
  SABRE_ERR_UNSUPPORTED = -2,  /* shape this build does not handle (e.g. head_dim != 128) */
  SABRE_ERR_ALIGNMENT = -3,    /* pointer or stride breaks the 16-byte TMA rule */
  SABRE_ERR_CUDA = -4,         /* a CUDA runtime/driver call failed */
  SABRE_ERR_WORKSPACE = -5     /* workspace missing or too small */
} sabre_status_t;

enum { SABRE_BF16 = 0, SABRE_F16 = 1, SABRE_F32 = 2 /* sabre_chunk_vectors embeddings only */ };

/* Device status flags (sabre_device_status). */
enum { SABRE_DEV_TIMEOUT = 1u, SABRE_DEV_BAD_SMEM_ALIGN = 2u };

int sabre_version(void);
const char* sabre_status_string(int status);
const char* sabre_last_error(void);

/* Read (and optionally clear) the device status word of the current device.
 * Synchronises `stream`. */
int sabre_device_status(unsigned int* flags_out, int clear, void* stream);

/* Limit, in nanoseconds, of every bounded wait in the kernels' main loops on
 * the current device (default 2 s; ns = 0 restores it; otherwise 1 us <= ns
 * <= 60 s). Applies to kernels launched after the call (synchronous). A wait
 * that runs out records SABRE_DEV_TIMEOUT, the CTA drains the copies and
 * MMAs it issued (those drains always allow 2 s), frees its tensor memory and
 * exits without writing its output tile. A limit shorter than a kernel's
 * normal waits makes correct calls fail this way: it is meant for tests of
 * the timeout path and for callers that want a tighter watchdog. No
 * counterpart in the reference (its Triton kernels have no bounded waits). */
int sabre_set_wait_limit_ns(unsigned long long ns);

/* ------------------------------------------------------------------------
 * (1) Block-sparse prefill attention.
 *
 * Replaces the launch of `_fwd_kernel_sabrecoder`
 * (methods/sabrecoder/sabrecoder_attention_triton.py:2039-2053; kernel
 * :28-116) from StructureAwareSparseAttentionTriton.forward (:1935-2066).
 *
 * q, o      : [B, Hq, L, D] strides q_strides/o_strides = {b, h, l, d}
 * k, v      : [B, Hkv, L, D] strides {b, h, l, d}; query head h reads kv head
 *             h / (Hq / Hkv) (the reference wrapper's repeat_interleave,
 *             sabrecoder_llama_triton.py:301-303, without the copy)
 * block_indices : int32 [B, Hidx, nb, max_active], strides idx_strides =
 *             {b, h, m, k}; h-stride 0 shares one list across heads (the
 *             reference's layout (B, nb, max_active))
 * block_counts  : int32 [B, Hidx, nb], strides cnt_strides = {b, h, m}
 * nb = ceil(L / block_size); block_size must be a multiple of 64;
 * head_dim must be 128; d-stride must be 1; other strides and base pointers
 * must be 16-byte multiples; L <= 65536.
 * Semantics: for each (b, h, query row r) softmax over keys n <= r inside
 * the listed blocks i < min(count, max_active); entries outside
 * [0, query block] contribute nothing (the reference's causal mask makes
 * them all -inf); duplicate entries count once. softmax_scale <= 0 selects
 * 1/sqrt(head_dim) (the reference's scale, :67).
 * ---------------------------------------------------------------------- */
int sabre_prefill_bsa(const void* q, const void* k, const void* v, void* o, const int32_t* block_indices,
                      const int32_t* block_counts, int batch, int heads_q, int heads_kv, int seq_len,
                      int head_dim, int block_size, int max_active, const int64_t* q_strides,
                      const int64_t* k_strides, const int64_t* v_strides, const int64_t* o_strides,
                      const int64_t* idx_strides, const int64_t* cnt_strides, float softmax_scale, int dtype,
                      void* stream);

/* ------------------------------------------------------------------------
 * (2) Split-K block-sparse decode attention over a KV cache.
 *
 * No reference counterpart for the sparse case: the reference decodes with
 * dense SDPA over the whole cache (sabrecoder_llama_triton.py:254-268,
 * :305-308). This entry replaces that SDPA call.
 *
 * q, o      : [B, Hq, D], strides {b, h, d}
 * k_cache, v_cache : [B, Hkv, Tmax, D], strides {b, h, t, d}
 * block_indices : int32 [B, Hidx, max_active] strides {b, h, k} (h-stride 0
 *             = shared), block_counts int32 [B, Hidx] strides {b, h}
 * seq_lens  : int32 [B] device: keys t >= seq_lens[b] are masked
 * workspace : >= sabre_decode_workspace_size(...) bytes of device memory,
 *             4-byte aligned (16-byte aligned lets the partials be stored 16
 *             bytes at a time)
 * ---------------------------------------------------------------------- */
size_t sabre_decode_workspace_size(int batch, int heads_q, int heads_kv, int head_dim, int max_active);
int sabre_decode_bsa(const void* q, const void* k_cache, const void* v_cache, void* o,
                     const int32_t* block_indices, const int32_t* block_counts, const int32_t* seq_lens,
                     int batch, int heads_q, int heads_kv, int max_seq, int head_dim, int block_size,
                     int max_active, const int64_t* q_strides, const int64_t* k_strides,
                     const int64_t* v_strides, const int64_t* o_strides, const int64_t* idx_strides,
                     const int64_t* cnt_strides, float softmax_scale, int dtype, void* workspace,
                     size_t workspace_bytes, void* stream);

/* ------------------------------------------------------------------------
 * (2b) Split-K decode that allocates nothing and takes no workspace.
 *
 * No counterpart in the reference. For callers that cannot provide device
 * memory at decode time (a runtime that reserves all device memory up front
 * and rejects later allocations, a foreign-language binding without access
 * to a caching allocator, a decode loop that must not synchronise on a
 * cudaMalloc). Same arguments and results as sabre_decode_bsa without the
 * workspace: the split partials live in a 2 MiB array compiled into the
 * library (held by every GPU that loads it until exit). Shapes whose
 * batch * heads_q * (head_dim + 2) floats exceed it are rejected with
 * SABRE_ERR_UNSUPPORTED. All calls share that array, so calls that overlap
 * on the GPU race. The first call on a device looks up the array's device
 * address (cudaGetSymbolAddress) with that device current; make it before
 * any stream capture. The address is kept for the life of the process: after
 * a cudaDeviceReset the module is loaded again and the array may move, so a
 * process that resets a device must reload this library before calling this
 * entry point again.
 * ---------------------------------------------------------------------- */
int sabre_decode_bsa_noalloc(const void* q, const void* k_cache, const void* v_cache, void* o,
                             const int32_t* block_indices, const int32_t* block_counts, const int32_t* seq_lens,
                             int batch, int heads_q, int heads_kv, int max_seq, int head_dim, int block_size,
                             int max_active, const int64_t* q_strides, const int64_t* k_strides,
                             const int64_t* v_strides, const int64_t* o_strides, const int64_t* idx_strides,
                             const int64_t* cnt_strides, float softmax_scale, int dtype, void* stream);

/* ------------------------------------------------------------------------
 * (1b) Fused rotary embedding + KV store + per-block pooling.
 *
 * Replaces apply_rotary_pos_emb and the KV-cache update of the reference
 * wrapper (methods/sabrecoder/sabrecoder_llama_triton.py:292-299) with one
 * pass: q_out = rope(q), k_out[pos0 + l] = rope(k), v_out[pos0 + l] = v, with
 * rope(x) = x*cos + rotate_half(x)*sin rounded per operation in the storage
 * dtype (bit-identical to transformers' apply_rotary_pos_emb).
 *
 * q, k, v  : [B, L, H*, D] strides {b, l, h} (d-stride 1)
 * cos, sin : [B, L, D] strides {b, l} (the model's position embeddings)
 * q_out    : [B, L, Hq, D] strides {b, l, h} (may alias q)
 * k_out, v_out : [B, Hkv, T, D] strides {b, h, t}, T = max_seq; rows
 *            pos0 .. pos0+L-1 are written (pos0 >= 0 and pos0 + L <= T, else
 *            SABRE_ERR_INVALID_ARG before launch)
 * q_pool, k_pool (optional, fp32, contiguous [B, Hq|Hkv, ceil(L/pool_block), D]):
 *            per-block means of the rotated rows (rows summed first to
 *            last, then divided by the row count); require pos0 == 0.
 * head_dim must be 128; strides multiples of 8 elements, pointers 16-byte aligned.
 * ---------------------------------------------------------------------- */
int sabre_rope_qkv(const void* q, const void* k, const void* v, const void* cos, const void* sin, void* q_out,
                   void* k_out, void* v_out, float* q_pool, float* k_pool, int batch, int seq_len, int heads_q,
                   int heads_kv, int head_dim, int pool_block, int pos0, int max_seq, const int64_t* q_strides,
                   const int64_t* k_strides, const int64_t* v_strides, const int64_t* cos_strides,
                   const int64_t* q_out_strides, const int64_t* k_out_strides, const int64_t* v_out_strides,
                   int dtype, void* stream);

/* ------------------------------------------------------------------------
 * (1b') Prefill q/k/v projection + rotary embedding + KV store + pooling.
 *
 * Replaces, for a prompt, the reference wrapper's q_proj/k_proj/v_proj,
 * apply_rotary_pos_emb and KV-cache update
 * (methods/sabrecoder/sabrecoder_llama_triton.py:288-299) with one kernel: a
 * tcgen05 GEMM Y = X W^T over the concatenated bias-free weights
 * W = [Wq; Wk; Wv] whose epilogue rounds Y to the storage dtype and then does
 * what sabre_rope_qkv (1b) does with Y (same rounding, same pooling), so Y
 * never goes to HBM.
 *
 * x        : [batch * seq_len, hidden] rows, row stride x_stride (>= hidden,
 *            multiple of 8), 16-byte aligned
 * w        : [(heads_q + 2 heads_kv) * 128, hidden], row-major, contiguous
 * cos, sin : [B, L, D] strides {b, l} (b-stride 0 for one shared table)
 * q_out    : [B, L, Hq, D] strides {b, l, h}
 * k_out, v_out : [B, Hkv, T, D] strides {b, h, t}, T = max_seq; rows
 *            pos0 .. pos0+L-1 are written (pos0 + L <= T)
 * q_pool, k_pool (optional fp32 [B, Hq|Hkv, ceil(L/pool_block), D]): as in
 *            (1b); need pool_block 64 or 128, pos0 == 0, and batch 1 or
 *            seq_len a multiple of 256
 * y_out    (optional): also store Y itself, [batch * seq_len, N] with row
 *            stride y_stride (for checking the projection)
 * head_dim must be 128; hidden a multiple of 8; strides multiples of 8
 * elements, pointers 16-byte aligned.
 * ---------------------------------------------------------------------- */
int sabre_qkv_proj_rope(const void* x, const void* w, const void* cos, const void* sin, void* q_out, void* k_out,
                        void* v_out, float* q_pool, float* k_pool, void* y_out, int batch, int seq_len, int hidden,
                        int heads_q, int heads_kv, int head_dim, int pool_block, int pos0, int max_seq,
                        int64_t x_stride, const int64_t* cos_strides, const int64_t* q_out_strides,
                        const int64_t* k_out_strides, const int64_t* v_out_strides, int64_t y_stride, int dtype,
                        void* stream);

/* ------------------------------------------------------------------------
 * (1c) Decode-step q/k/v projection + rotary embedding + KV store.
 *
 * Replaces, for one new token per sequence, the reference wrapper's
 * q_proj/k_proj/v_proj, apply_rotary_pos_emb and KV-cache update
 * (methods/sabrecoder/sabrecoder_llama_triton.py:288-299) with one kernel:
 * y = W x for the three bias-free projections (fp32 sums, each output
 * rounded to the storage dtype), then q_out = rope(y_q),
 * k_out[pos0] = rope(y_k), v_out[pos0] = y_v with rope as in (1b).
 *
 * x        : [B, hidden] row stride x_stride (16-byte aligned)
 * wq       : [heads_q*D, hidden], wk / wv: [heads_kv*D, hidden], row-major and
 *            contiguous (16-byte aligned)
 * cos, sin : [B, D] row stride cos_stride (the new token's position embeddings)
 * q_out    : [B, heads_q, D] strides {b, h}
 * k_out, v_out : [B, heads_kv, T, D] strides {b, h, t}, T = max_seq; row pos0 (< T) is written
 * batch <= 8, batch * hidden * 2 <= 160 KiB, hidden a multiple of 8,
 * head_dim 128, d-stride 1 everywhere.
 * ---------------------------------------------------------------------- */
int sabre_qkv_rope_decode(const void* x, const void* wq, const void* wk, const void* wv, const void* cos,
                          const void* sin, void* q_out, void* k_out, void* v_out, int batch, int hidden,
                          int heads_q, int heads_kv, int head_dim, int pos0, int max_seq, int64_t x_stride,
                          int64_t cos_stride, const int64_t* q_out_strides, const int64_t* k_out_strides,
                          const int64_t* v_out_strides, int dtype, void* stream);

/* ------------------------------------------------------------------------
 * (3) Block-mask construction from token-level structure.
 *
 * Replaces `StructureAwareMaskBuilder._build_block_mask_from_chunks`
 * (sabrecoder_attention_triton.py:1455-1604): rules R0 window (:1492-1500),
 * R1 within-chunk (:1502-1525), R2 dependencies (:1527-1544), R3 global key
 * columns (:1546-1600), then tril (:1603).
 *
 * token_to_chunk : int32 [L] chunk id per token, -1 = none
 * global_token_mask : uint8 [L] or NULL; 1 = token on a signature/special line
 * chunk_flags : uint8 [nchunks]; bit 0 = import chunk (global key columns)
 * dep_ptr, dep_idx : CSR of chunk dependencies, src -> targets (int32
 *             [nchunks+1], [dep_ptr[nchunks]]); out-of-range targets skipped
 * mask_bits (out): uint32 [nb, nwords], nwords = ceil(nb/32), bit j of row i
 *             = block (i, j) active
 * mask_dense (out, optional): int32 [nb, nb] (the reference's block_mask_2d)
 * workspace : >= sabre_block_mask_workspace_size(nchunks, nb) bytes
 * ---------------------------------------------------------------------- */
size_t sabre_block_mask_workspace_size(int nchunks, int num_blocks);
int sabre_build_block_mask(const int32_t* token_to_chunk, const uint8_t* global_token_mask,
                           const uint8_t* chunk_flags, int nchunks, const int32_t* dep_ptr,
                           const int32_t* dep_idx, int seq_len, int block_size, int window_size,
                           int num_prefix_tokens, int num_suffix_tokens, int max_chunk_tokens,
                           int global_last_k_chunks, uint32_t* mask_bits, int32_t* mask_dense, void* workspace,
                           size_t workspace_bytes, void* stream);

/* ------------------------------------------------------------------------
 * (3b) Index lists from a block mask.
 *
 * Replaces `compute_block_indices_from_mask`
 * (sabrecoder_attention_triton.py:1837-1859). Rows are emitted in ascending
 * column order (the reference's unstable argsort leaves the order arbitrary;
 * counts and per-row sets are identical), padded with -1 up to `cap`.
 * max_active_out (device int32[1]) receives max(max(counts), 1).
 *
 * From bits:  mask_bits uint32 [rows, nwords] -> indices int32 [rows, cap],
 *             counts int32 [rows]; rows = batch * heads * nb (any layout the
 *             caller flattens).
 * From dense: mask int32 [rows, ncols] with row stride `mask_row_stride`.
 * ---------------------------------------------------------------------- */
int sabre_indices_from_bits(const uint32_t* mask_bits, int rows, int ncols, int32_t* indices, int cap,
                            int32_t* counts, int32_t* max_active_out, void* stream);
int sabre_indices_from_dense(const int32_t* mask, int rows, int ncols, int64_t mask_row_stride,
                             int32_t* indices, int cap, int32_t* counts, int32_t* max_active_out,
                             void* stream);

/* ------------------------------------------------------------------------
 * (3c) Pooled q.k top-k extension (no reference counterpart; nearest
 * analogue is the chunk-similarity top-k, sabrecoder_attention_triton.py:
 * 581-682: mean-pool, score, per-source top-k).
 *
 * sabre_pool_blocks: x [B, H, L, D] strides {b,h,l,d} -> out fp32
 *   [B, H, nb, D] (contiguous): per block, rows summed first to last in
 *   fp32 then divided by the row count.
 * sabre_topk_extend: for each (b, h, query block qb) take the base row
 *   (base_bits [nb, nwords], shared by all heads), add the `topk` blocks
 *   kb <= qb not already active with the largest score
 *   sum_d qm[b,h,qb,d] * km[b,h/(Hq/Hkv),kb,d] (fp32, products rounded, added
 *   in order d = 0..D-1), ties to the lower kb; write the merged rows as
 *   ascending index lists int32 [B, Hq, nb, cap] + counts [B, Hq, nb] and
 *   max_active_out. Optional out_bits uint32 [B, Hq, nb, nwords].
 *   workspace: >= sabre_topk_workspace_size(B, Hq, nb) bytes (the fp32
 *   score matrix). nb <= 1024, topk <= 32, head_dim <= 256.
 * ---------------------------------------------------------------------- */
int sabre_pool_blocks(const void* x, int batch, int heads, int seq_len, int head_dim, int block_size,
                      const int64_t* x_strides, int dtype, float* out, void* stream);
size_t sabre_topk_workspace_size(int batch, int heads_q, int num_blocks);
int sabre_topk_extend(const float* q_pooled, const float* k_pooled, const uint32_t* base_bits, int batch,
                      int heads_q, int heads_kv, int num_blocks, int head_dim, int topk, int32_t* indices,
                      int cap, int32_t* counts, int32_t* max_active_out, uint32_t* out_bits, void* workspace,
                      size_t workspace_bytes, void* stream);

/* ----------------------------------------------------------------------
 * (3d) Chunk-similarity dependency edges.
 * Replaces StructureAwareMaskBuilder._get_or_build_similarity_vectors and
 * _similarity_edges (methods/sabrecoder/sabrecoder_attention_triton.py:490-682);
 * the caller keeps the text side (cleaning, tokenising, choosing k).
 *
 * sabre_chunk_vectors: embedding [vocab, dim] (SABRE_BF16, SABRE_F16 or
 *   SABRE_F32, contiguous); chunk c owns tok_ids[tok_ptr[c] .. tok_ptr[c+1]).
 *   out_f16 [nchunks, dim] = fp16(v / max(||v||, 1e-12)) with v the fp32 mean
 *   of the chunk's embedding rows (tokens added first to last; an empty chunk
 *   gives zeros). ||v||: thread t of 256 adds the squares of d = t, t+256, ...
 *   in order, then a halving tree over the 256 partials. dim <= 8192; token
 *   ids must lie in [0, vocab) (others are skipped).
 * sabre_similarity_topk: for source s (vector row src_rows[s], chunk
 *   src_chunk[s]) score every target t (row tgt_rows[t], chunk tgt_chunk[t]):
 *   fp32 dot product, lane l of 32 adding the rounded products of
 *   d = l, l+32, ... in order, then an xor tree (16, 8, 4, 2, 1); -inf when
 *   tgt_chunk[t] == src_chunk[s]. Keeps the min(k, ntgt) best (value
 *   descending, ties to the lower t) and writes their target chunk ids to
 *   out_tgt_chunk [nsrc, k], -1 for the chunk itself and for unused slots.
 *   k <= 64; ntgt <= 40960.
 * ---------------------------------------------------------------------- */
int sabre_chunk_vectors(const void* embedding, int emb_dtype, int vocab, int dim, const int32_t* tok_ptr,
                        const int32_t* tok_ids, int nchunks, void* out_f16, void* stream);
int sabre_similarity_topk(const void* vecs_f16, int dim, const int32_t* src_rows, const int32_t* src_chunk,
                          int nsrc, const int32_t* tgt_rows, const int32_t* tgt_chunk, int ntgt, int k,
                          int32_t* out_tgt_chunk, void* stream);

/* ----------------------------------------------------------------------
 * (3e) Token-level sparsity (the reference's use_token_level_sparsity=True:
 * build_token_level_mask / _build_mask_from_chunks,
 * sabrecoder_attention_triton.py:1171-1454, compute_block_mask_from_token_mask
 * :1862-1885 and _fwd_kernel_sabrecoder_token_sparse :119-215), block size 64,
 * without an L x L mask.
 *
 * Per token t < seq_len: tok_chunk[t] (chunk id, -1 if none), tok_group[t]
 * (chunk id, or chunk id combined with the max_chunk_tokens group), tok_global[t]
 * (1 = visible to every query: import chunk, signature / special line,
 * prefix, suffix, last-k chunk); dep_bits [nchunks][ceil(nchunks/32)]: bit t
 * of row s set when chunk t is a dependency of chunk s. Key j is visible to
 * query i when j <= i and (i - j <= window, tok_global[j], both chunks >= 0
 * with equal groups, or both chunks >= 0 with chunk(j) a dependency of chunk(i)).
 *
 * sabre_token_block_mask: row_bits uint32 [nb][ceil(nb/32)] (nb = ceil(L/64)):
 *   bit kb of row qb when any pair of query block qb and key block kb is
 *   visible (the reference's block mask from the token mask).
 * sabre_token_tile_masks: for every listed pair (indices [nb][cap] ascending,
 *   counts [nb], row_ptr [nb] = exclusive prefix sum of counts) the 64 query
 *   rows' 64-bit key masks at masks[(row_ptr[qb] + i) * 64 + row].
 * sabre_prefill_bsa_tokenmask: sabre_prefill_bsa (block_size 64) that also
 *   masks each element of a listed block by its tile mask. Lists must be
 *   the ascending lists the masks were written for, shared by all batch
 *   entries and heads (index/count strides as in sabre_prefill_bsa).
 * ---------------------------------------------------------------------- */
int sabre_token_block_mask(const int32_t* tok_chunk, const int32_t* tok_group, const uint8_t* tok_global,
                           const uint32_t* dep_bits, int nchunks, int seq_len, int window, uint32_t* row_bits,
                           void* stream);
int sabre_token_tile_masks(const int32_t* tok_chunk, const int32_t* tok_group, const uint8_t* tok_global,
                           const uint32_t* dep_bits, int nchunks, int seq_len, int window, const int32_t* indices,
                           int cap, const int32_t* counts, const int32_t* row_ptr, uint64_t* masks, void* stream);
int sabre_prefill_bsa_tokenmask(const void* q, const void* k, const void* v, void* o, const int32_t* block_indices,
                                const int32_t* block_counts, const uint64_t* tile_masks,
                                const int32_t* tile_row_ptr, int batch, int heads_q, int heads_kv, int seq_len,
                                int head_dim, int max_active, const int64_t* q_strides, const int64_t* k_strides,
                                const int64_t* v_strides, const int64_t* o_strides, const int64_t* idx_strides,
                                const int64_t* cnt_strides, float softmax_scale, int dtype, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* SABRE_B200_H_ */
