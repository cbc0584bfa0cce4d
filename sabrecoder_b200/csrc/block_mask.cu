// Block-mask construction, index lists and the pooled q.k top-k extension.
//
// Replaces the CPU builder `_build_block_mask_from_chunks`
// (methods/sabrecoder/sabrecoder_attention_triton.py:1455-1604) and
// `compute_block_indices_from_mask` (:1837-1859). Output is bit-exact with
// the reference: same mask, same counts, same per-row sets (rows emitted in
// ascending order; the reference's argsort leaves the order arbitrary).
//
// Representation: a block row is a bitset of nwords = ceil(nb/32) uint32
// words. Chunk block sets (the reference's `chunk_blocks`, :1479-1490) are
// bitsets too, built by one scatter pass over the tokens. Each row is then
// the OR of: its window range (R0), the block sets of the chunks that touch
// it -- restricted to its max_chunk_tokens group when that is set -- (R1),
// the block sets of those chunks' dependency targets (R2), and the global
// key columns (R3), clipped to j <= i (tril).
#include "common.cuh"

namespace sabre {
namespace mask {

constexpr int kMaxWordsPerLane = 4;  // nb <= 4096
constexpr int kMaxBlocks = 32 * 32 * kMaxWordsPerLane;

struct BuildParams {
  const int32_t* t2c;
  const uint8_t* gtm;
  const uint8_t* chunk_flags;
  const int32_t* dep_ptr;
  const int32_t* dep_idx;
  uint32_t* cb;      // [nchunks][nwords]
  uint32_t* gcols;   // [nwords]
  uint32_t* out_bits;
  int32_t* out_dense;
  int nchunks, L, B, nb, nwords, window, prefix, suffix, mct, last_k;
};

// Pass 1: chunk block sets and token-derived global columns.
__global__ void scatter_tokens_kernel(const BuildParams p) {
  const int t = blockIdx.x * blockDim.x + threadIdx.x;
  const unsigned full = 0xffffffffu;
  const bool in = t < p.L;
  const int c = in ? p.t2c[t] : -1;
  const int blk = in ? t / p.B : 0;
  const bool valid_c = in && c >= 0 && c < p.nchunks;
  // Warp-aggregate identical (chunk, block) pairs to one atomic.
  const long long key = valid_c ? static_cast<long long>(c) * p.nb + blk : -1ll;
  const unsigned grp = __match_any_sync(full, key);
  const bool leader = (__ffs(grp) - 1) == (threadIdx.x & 31);
  if (valid_c && leader) {
    atomicOr(&p.cb[static_cast<long long>(c) * p.nwords + (blk >> 5)], 1u << (blk & 31));
    // Import chunks (:1548-1555) and the last-k chunks (:1592-1600) are
    // global key columns: every block of theirs is visible to all rows.
    const bool glob = (p.chunk_flags[c] & 1u) || (p.last_k > 0 && c >= p.nchunks - p.last_k);
    if (glob) atomicOr(&p.gcols[blk >> 5], 1u << (blk & 31));
  }
  // Signature/special-line tokens (:1557-1576).
  const bool g = in && p.gtm != nullptr && p.gtm[t] != 0;
  const long long gkey = g ? blk : -1ll;
  const unsigned ggrp = __match_any_sync(full, gkey);
  if (g && (__ffs(ggrp) - 1) == (threadIdx.x & 31)) atomicOr(&p.gcols[blk >> 5], 1u << (blk & 31));
}

__device__ __forceinline__ uint32_t range_bits(int w, int lo, int hi) {
  // bits of word w inside [lo, hi) (block indices)
  const int a = max(lo - w * 32, 0);
  const int b = min(hi - w * 32, 32);
  if (a >= b) return 0u;
  const uint32_t upto = (b >= 32) ? 0xffffffffu : ((1u << b) - 1u);
  return upto & ~((1u << a) - 1u);
}

// Pass 2: one warp per block row.
__global__ void build_rows_kernel(const BuildParams p) {
  const int warp_global = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  const unsigned full = 0xffffffffu;
  const int i = warp_global;
  if (i >= p.nb) return;
  uint32_t r[kMaxWordsPerLane];
  // R0 window (:1492-1500)
  const int jmin = max(0, i * p.B - p.window) / p.B;
  // R3 prefix (:1579-1583) and suffix (:1585-1589) columns
  const int pre = min(p.prefix, p.L);
  const int pend = pre > 0 ? (pre - 1) / p.B + 1 : 0;
  const int suf = min(p.suffix, p.L);
  const int sstart = suf > 0 ? max(0, p.L - suf) / p.B : p.nb;
  // R1 group range of this row
  int glo = 0, ghi = p.nb;
  if (p.mct > 0) {
    const int bpg = max(1, p.mct / p.B);
    glo = (i / bpg) * bpg;
    ghi = glo + bpg;
  }
#pragma unroll
  for (int u = 0; u < kMaxWordsPerLane; ++u) {
    const int w = lane + 32 * u;
    uint32_t v = 0u;
    if (w < p.nwords) {
      v = range_bits(w, jmin, i + 1) | p.gcols[w] | range_bits(w, 0, pend) | range_bits(w, sstart, p.nb);
    }
    r[u] = v;
  }
  // R1 + R2 over the distinct chunks of the row's tokens.
  const int t0 = i * p.B;
  const int t1 = min(t0 + p.B, p.L);
  int last_done = -2;
  for (int tb = t0; tb < t1; tb += 32) {
    const int t = tb + lane;
    const int c = (t < t1) ? p.t2c[t] : -1;
    const bool valid_c = c >= 0 && c < p.nchunks;
    const unsigned grp = __match_any_sync(full, valid_c ? c : -1);
    unsigned leaders = __ballot_sync(full, valid_c && (__ffs(grp) - 1) == lane);
    while (leaders) {
      const int src = __ffs(leaders) - 1;
      leaders &= leaders - 1u;
      const int cc = __shfl_sync(full, c, src);
      if (cc == last_done) continue;
      last_done = cc;
      const uint32_t* cbc = p.cb + static_cast<long long>(cc) * p.nwords;
#pragma unroll
      for (int u = 0; u < kMaxWordsPerLane; ++u) {
        const int w = lane + 32 * u;
        if (w < p.nwords) r[u] |= cbc[w] & range_bits(w, glo, ghi);
      }
      const int e0 = p.dep_ptr[cc];
      const int e1 = p.dep_ptr[cc + 1];
      for (int e = e0; e < e1; ++e) {
        const int tg = p.dep_idx[e];
        if (tg < 0 || tg >= p.nchunks) continue;
        const uint32_t* cbt = p.cb + static_cast<long long>(tg) * p.nwords;
#pragma unroll
        for (int u = 0; u < kMaxWordsPerLane; ++u) {
          const int w = lane + 32 * u;
          if (w < p.nwords) r[u] |= cbt[w];
        }
      }
    }
  }
  // tril (:1602-1604) and store
#pragma unroll
  for (int u = 0; u < kMaxWordsPerLane; ++u) {
    const int w = lane + 32 * u;
    if (w < p.nwords) {
      r[u] &= range_bits(w, 0, i + 1);
      p.out_bits[static_cast<long long>(i) * p.nwords + w] = r[u];
    }
  }
  if (p.out_dense) {
    int32_t* drow = p.out_dense + static_cast<long long>(i) * p.nb;
    for (int j = lane; j < p.nb; j += 32) {
      const uint32_t word = p.out_bits[static_cast<long long>(i) * p.nwords + (j >> 5)];
      drow[j] = static_cast<int32_t>((word >> (j & 31)) & 1u);
    }
  }
}

// Write one row's ascending index list from the words held by the warp
// (lane owns words lane + 32u). Pads with -1 up to cap.
__device__ __forceinline__ void emit_row(const uint32_t (&r)[kMaxWordsPerLane], int nwords, int32_t* out, int cap,
                                         int32_t* count_out, int32_t* max_active_out) {
  const unsigned full = 0xffffffffu;
  const int lane = threadIdx.x & 31;
  int base = 0;
#pragma unroll
  for (int u = 0; u < kMaxWordsPerLane; ++u) {
    const int w = lane + 32 * u;
    const uint32_t word = (w < nwords) ? r[u] : 0u;
    const int pc = __popc(word);
    int incl = pc;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const int y = __shfl_up_sync(full, incl, off);
      if (lane >= off) incl += y;
    }
    const int total = __shfl_sync(full, incl, 31);
    int pos = base + incl - pc;
    uint32_t bitsleft = word;
    while (bitsleft) {
      const int bpos = __ffs(bitsleft) - 1;
      bitsleft &= bitsleft - 1u;
      if (pos < cap) out[pos] = w * 32 + bpos;
      ++pos;
    }
    base += total;
  }
  for (int k = base + lane; k < cap; k += 32) out[k] = -1;
  if (lane == 0) {
    *count_out = base;
    atomicMax(max_active_out, max(base, 1));
  }
}

__global__ void indices_from_bits_kernel(const uint32_t* bits, int rows, int nwords, int32_t* idx, int cap,
                                         int32_t* counts, int32_t* max_active) {
  const int row = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  uint32_t r[kMaxWordsPerLane];
#pragma unroll
  for (int u = 0; u < kMaxWordsPerLane; ++u) {
    const int w = lane + 32 * u;
    r[u] = (w < nwords) ? bits[static_cast<long long>(row) * nwords + w] : 0u;
  }
  emit_row(r, nwords, idx + static_cast<long long>(row) * cap, cap, counts + row, max_active);
}

__global__ void indices_from_dense_kernel(const int32_t* mask, int rows, int ncols, long long row_stride,
                                          int32_t* idx, int cap, int32_t* counts, int32_t* max_active) {
  const int row = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const unsigned full = 0xffffffffu;
  const int nwords = (ncols + 31) / 32;
  const int32_t* mr = mask + static_cast<long long>(row) * row_stride;
  uint32_t r[kMaxWordsPerLane];
#pragma unroll
  for (int u = 0; u < kMaxWordsPerLane; ++u) r[u] = 0u;
  for (int w = 0; w < nwords; ++w) {
    const int j = w * 32 + lane;
    const bool on = (j < ncols) && mr[j] != 0;
    const uint32_t word = __ballot_sync(full, on);
    const int owner = w & 31;
    const int slot = w >> 5;
#pragma unroll
    for (int u = 0; u < kMaxWordsPerLane; ++u)
      if (u == slot && lane == owner) r[u] = word;
  }
  emit_row(r, nwords, idx + static_cast<long long>(row) * cap, cap, counts + row, max_active);
}

// ---------------------------------------------------------------------------
// Pooled q.k top-k
// ---------------------------------------------------------------------------
template <typename T>
__global__ void pool_blocks_kernel(const T* x, int B, int H, int L, int D, int blk, long long sb, long long sh,
                                   long long sl, float* out) {
  const long long gid = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int nb = (L + blk - 1) / blk;
  const long long total = static_cast<long long>(B) * H * nb * D;
  if (gid >= total) return;
  const int d = static_cast<int>(gid % D);
  long long rest = gid / D;
  const int kb = static_cast<int>(rest % nb);
  rest /= nb;
  const int h = static_cast<int>(rest % H);
  const int b = static_cast<int>(rest / H);
  const T* base = x + b * sb + h * sh + d;
  const int r0 = kb * blk;
  const int n = min(blk, L - r0);
  float s = 0.f;
  for (int r = 0; r < n; ++r) s = __fadd_rn(s, DT<T>::to_f(base[static_cast<long long>(r0 + r) * sl]));
  out[gid] = __fdiv_rn(s, static_cast<float>(n));
}

}  // namespace mask
}  // namespace sabre

using namespace sabre;

extern "C" {

size_t sabre_block_mask_workspace_size(int nchunks, int num_blocks) {
  const size_t nwords = (static_cast<size_t>(num_blocks > 0 ? num_blocks : 0) + 31) / 32;
  return (static_cast<size_t>(nchunks > 0 ? nchunks : 0) + 1) * nwords * sizeof(uint32_t);
}

int sabre_build_block_mask(const int32_t* token_to_chunk, const uint8_t* global_token_mask,
                           const uint8_t* chunk_flags, int nchunks, const int32_t* dep_ptr,
                           const int32_t* dep_idx, int seq_len, int block_size, int window_size,
                           int num_prefix_tokens, int num_suffix_tokens, int max_chunk_tokens,
                           int global_last_k_chunks, uint32_t* mask_bits, int32_t* mask_dense, void* workspace,
                           size_t workspace_bytes, void* stream) {
  using namespace sabre::mask;
  if (seq_len <= 0 || block_size <= 0 || nchunks < 0 || !mask_bits)
    return sabre_fail(SABRE_ERR_INVALID_ARG, "sabre_build_block_mask: bad sizes or null output");
  if (!token_to_chunk)
    return sabre_fail(SABRE_ERR_INVALID_ARG, "sabre_build_block_mask: token_to_chunk is null");
  if (nchunks > 0 && (!chunk_flags || !dep_ptr))
    return sabre_fail(SABRE_ERR_INVALID_ARG, "sabre_build_block_mask: chunk_flags/dep_ptr null");
  if (global_last_k_chunks < 0 || max_chunk_tokens < 0)
    return sabre_fail(SABRE_ERR_INVALID_ARG, "sabre_build_block_mask: negative last_k or max_chunk_tokens");
  if (max_chunk_tokens > 0 && max_chunk_tokens % block_size != 0)
    return sabre_fail(SABRE_ERR_INVALID_ARG,
                      "sabre_build_block_mask: max_chunk_tokens must be a multiple of block_size");
  const int nb = (seq_len + block_size - 1) / block_size;
  if (nb > kMaxBlocks)
    return sabre_fail(SABRE_ERR_UNSUPPORTED, "sabre_build_block_mask: %d blocks > %d", nb, kMaxBlocks);
  const size_t need = sabre_block_mask_workspace_size(nchunks, nb);
  if (!workspace || workspace_bytes < need)
    return sabre_fail(SABRE_ERR_WORKSPACE, "sabre_build_block_mask: workspace %zu < %zu bytes", workspace_bytes,
                      need);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  BuildParams p;
  p.t2c = token_to_chunk;
  p.gtm = global_token_mask;
  p.chunk_flags = chunk_flags;
  p.dep_ptr = dep_ptr;
  p.dep_idx = dep_idx;
  p.nwords = (nb + 31) / 32;
  p.cb = static_cast<uint32_t*>(workspace);
  p.gcols = p.cb + static_cast<size_t>(nchunks) * p.nwords;
  p.out_bits = mask_bits;
  p.out_dense = mask_dense;
  p.nchunks = nchunks;
  p.L = seq_len;
  p.B = block_size;
  p.nb = nb;
  p.window = window_size;
  p.prefix = num_prefix_tokens;
  p.suffix = num_suffix_tokens;
  p.mct = max_chunk_tokens;
  p.last_k = global_last_k_chunks;
  cudaError_t e = cudaMemsetAsync(workspace, 0, need, s);
  if (e != cudaSuccess) return sabre_cuda_fail(e, "cudaMemsetAsync(workspace)");
  scatter_tokens_kernel<<<(seq_len + 255) / 256, 256, 0, s>>>(p);
  build_rows_kernel<<<(nb * 32 + 255) / 256, 256, 0, s>>>(p);
  e = cudaGetLastError();
  if (e != cudaSuccess) return sabre_cuda_fail(e, "sabre_build_block_mask launch");
  return SABRE_OK;
}

int sabre_indices_from_bits(const uint32_t* mask_bits, int rows, int ncols, int32_t* indices, int cap,
                            int32_t* counts, int32_t* max_active_out, void* stream) {
  using namespace sabre::mask;
  if (!mask_bits || !indices || !counts || !max_active_out || rows <= 0 || ncols <= 0 || cap <= 0)
    return sabre_fail(SABRE_ERR_INVALID_ARG, "sabre_indices_from_bits: bad arguments");
  if (ncols > kMaxBlocks)
    return sabre_fail(SABRE_ERR_UNSUPPORTED, "sabre_indices_from_bits: %d columns > %d", ncols, kMaxBlocks);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaError_t e = cudaMemsetAsync(max_active_out, 0, sizeof(int32_t), s);
  if (e != cudaSuccess) return sabre_cuda_fail(e, "cudaMemsetAsync(max_active)");
  const long long threads = static_cast<long long>(rows) * 32;
  indices_from_bits_kernel<<<static_cast<unsigned>((threads + 255) / 256), 256, 0, s>>>(
      mask_bits, rows, (ncols + 31) / 32, indices, cap, counts, max_active_out);
  e = cudaGetLastError();
  if (e != cudaSuccess) return sabre_cuda_fail(e, "sabre_indices_from_bits launch");
  return SABRE_OK;
}

int sabre_indices_from_dense(const int32_t* mask, int rows, int ncols, int64_t mask_row_stride, int32_t* indices,
                             int cap, int32_t* counts, int32_t* max_active_out, void* stream) {
  using namespace sabre::mask;
  if (!mask || !indices || !counts || !max_active_out || rows <= 0 || ncols <= 0 || cap <= 0 ||
      mask_row_stride < ncols)
    return sabre_fail(SABRE_ERR_INVALID_ARG, "sabre_indices_from_dense: bad arguments");
  if (ncols > kMaxBlocks)
    return sabre_fail(SABRE_ERR_UNSUPPORTED, "sabre_indices_from_dense: %d columns > %d", ncols, kMaxBlocks);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaError_t e = cudaMemsetAsync(max_active_out, 0, sizeof(int32_t), s);
  if (e != cudaSuccess) return sabre_cuda_fail(e, "cudaMemsetAsync(max_active)");
  const long long threads = static_cast<long long>(rows) * 32;
  indices_from_dense_kernel<<<static_cast<unsigned>((threads + 255) / 256), 256, 0, s>>>(
      mask, rows, ncols, mask_row_stride, indices, cap, counts, max_active_out);
  e = cudaGetLastError();
  if (e != cudaSuccess) return sabre_cuda_fail(e, "sabre_indices_from_dense launch");
  return SABRE_OK;
}

int sabre_pool_blocks(const void* x, int batch, int heads, int seq_len, int head_dim, int block_size,
                      const int64_t* x_strides, int dtype, float* out, void* stream) {
  using namespace sabre::mask;
  if (!x || !out || !x_strides || batch <= 0 || heads <= 0 || seq_len <= 0 || head_dim <= 0 || block_size <= 0)
    return sabre_fail(SABRE_ERR_INVALID_ARG, "sabre_pool_blocks: bad arguments");
  if (x_strides[3] != 1) return sabre_fail(SABRE_ERR_UNSUPPORTED, "sabre_pool_blocks: d-stride must be 1");
  const int nb = (seq_len + block_size - 1) / block_size;
  const long long total = static_cast<long long>(batch) * heads * nb * head_dim;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const unsigned grid = static_cast<unsigned>((total + 255) / 256);
  if (dtype == SABRE_BF16)
    pool_blocks_kernel<__nv_bfloat16><<<grid, 256, 0, s>>>(static_cast<const __nv_bfloat16*>(x), batch, heads,
                                                           seq_len, head_dim, block_size, x_strides[0],
                                                           x_strides[1], x_strides[2], out);
  else if (dtype == SABRE_F16)
    pool_blocks_kernel<__half><<<grid, 256, 0, s>>>(static_cast<const __half*>(x), batch, heads, seq_len, head_dim,
                                                    block_size, x_strides[0], x_strides[1], x_strides[2], out);
  else
    return sabre_fail(SABRE_ERR_INVALID_ARG, "sabre_pool_blocks: dtype %d", dtype);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return sabre_cuda_fail(e, "sabre_pool_blocks launch");
  return SABRE_OK;
}

}  // extern "C"
