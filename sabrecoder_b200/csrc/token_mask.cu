// Token-level sparsity without an L x L mask (block size 64).
//
// The reference's token-level variant (use_token_level_sparsity=True) builds a
// dense (L, L) float mask (build_token_level_mask / _build_mask_from_chunks,
// methods/sabrecoder/sabrecoder_attention_triton.py:1171-1266, :1269-1454),
// derives the block lists from it (compute_block_mask_from_token_mask :1862)
// and has its kernel (_fwd_kernel_sabrecoder_token_sparse :119-215) read the
// mask for every listed block. Here the same rule is evaluated on the GPU from
// per-token data, and only the listed blocks' 64x64 masks are kept, as one
// 64-bit word per query row (bit c = key c of the block):
//   key j is visible to query i  <=>  j <= i  and  ( i - j <= window
//       or global[j]                     (import chunk, signature / special
//                                         line, prefix, suffix, last-k chunk)
//       or chunk[i] >= 0, chunk[j] >= 0, group[i] == group[j]
//       or chunk[i] >= 0, chunk[j] >= 0, chunk[j] in deps[chunk[i]] )
// group[] is the chunk id, or the chunk id combined with the token's
// max_chunk_tokens group when grouping is on (computed by the caller).
#include "common.cuh"

namespace sabre {
namespace tokmask {

constexpr int kB = 64;  // block size of this variant

struct TokenRule {
  const int32_t* chunk;     // [L] chunk of each token, -1 if none
  const int32_t* group;     // [L] same-chunk group id
  const uint8_t* global;    // [L] 1 = visible to every query
  const uint32_t* deps;     // [nchunks][dwords] bit t of row s: chunk t is a dependency of chunk s
  int nchunks, dwords, L, window;
};

// 64-bit mask of query row i (absolute) against key block kb.
__device__ __forceinline__ unsigned long long row_word(const TokenRule& r, int i, int kb, const int32_t* s_chunk,
                                                       const int32_t* s_group, const uint8_t* s_global) {
  if (i >= r.L) return 0ull;
  const int ci = r.chunk[i];
  const int gi = r.group[i];
  const uint32_t* drow = (ci >= 0 && ci < r.nchunks) ? r.deps + static_cast<long long>(ci) * r.dwords : nullptr;
  unsigned long long w = 0ull;
  const int j0 = kb * kB;
  for (int c = 0; c < kB; ++c) {
    const int j = j0 + c;
    if (j > i || j >= r.L) break;
    bool ok = (i - j <= r.window) || s_global[c];
    const int cj = s_chunk[c];
    if (!ok && ci >= 0 && cj >= 0) {
      ok = (gi == s_group[c]);
      if (!ok && drow != nullptr && cj < r.nchunks) ok = (drow[cj >> 5] >> (cj & 31)) & 1u;
    }
    if (ok) w |= 1ull << c;
  }
  return w;
}

// Key block kb's per-token data into shared memory (thread t: token kb*64+t).
__device__ __forceinline__ void load_key_block(const TokenRule& r, int kb, int t, int32_t* s_chunk,
                                               int32_t* s_group, uint8_t* s_global) {
  const int j = kb * kB + t;
  s_chunk[t] = j < r.L ? r.chunk[j] : -1;
  s_group[t] = j < r.L ? r.group[j] : 0;
  s_global[t] = j < r.L ? r.global[j] : 0;
}

// One CTA (64 threads, thread = query row) per (key block, query block) pair
// with kb <= qb: bit kb of row_bits[qb] is set when any of its pairs is
// visible. row_bits starts zeroed. The pairs are independent, so the
// triangle of work spreads over the whole GPU.
__global__ void __launch_bounds__(kB) token_block_pairs_kernel(const TokenRule r, uint32_t* row_bits, int nwords) {
  __shared__ int32_t s_chunk[kB];
  __shared__ int32_t s_group[kB];
  __shared__ uint8_t s_global[kB];
  const int kb = blockIdx.x;
  const int qb = blockIdx.y;
  if (kb > qb) return;
  const int t = threadIdx.x;
  load_key_block(r, kb, t, s_chunk, s_group, s_global);
  __syncthreads();
  const unsigned long long wd = row_word(r, qb * kB + t, kb, s_chunk, s_group, s_global);
  if (__syncthreads_or(wd != 0ull) && t == 0)
    atomicOr(&row_bits[static_cast<long long>(qb) * nwords + (kb >> 5)], 1u << (kb & 31));
}

// One CTA per listed (query block, list entry): the 64 row words of that key
// block at masks[(row_ptr[qb] + e) * 64 + row].
__global__ void __launch_bounds__(kB) token_tile_masks_kernel(const TokenRule r, const int32_t* indices, int cap,
                                                             const int32_t* counts, const int32_t* row_ptr,
                                                             unsigned long long* masks) {
  __shared__ int32_t s_chunk[kB];
  __shared__ int32_t s_group[kB];
  __shared__ uint8_t s_global[kB];
  const int e = blockIdx.x;
  const int qb = blockIdx.y;
  if (e >= counts[qb]) return;
  const int t = threadIdx.x;
  const int kb = indices[static_cast<long long>(qb) * cap + e];
  load_key_block(r, kb, t, s_chunk, s_group, s_global);
  __syncthreads();
  masks[(row_ptr[qb] + static_cast<long long>(e)) * kB + t] = row_word(r, qb * kB + t, kb, s_chunk, s_group, s_global);
}

}  // namespace tokmask
}  // namespace sabre

using namespace sabre;

extern "C" {

static int token_rule(sabre::tokmask::TokenRule* r, const int32_t* tok_chunk, const int32_t* tok_group,
                      const uint8_t* tok_global, const uint32_t* dep_bits, int nchunks, int seq_len, int window,
                      const char* who) {
  if (!tok_chunk || !tok_group || !tok_global || (nchunks > 0 && !dep_bits))
    return sabre_fail(SABRE_ERR_INVALID_ARG, "%s: null pointer argument", who);
  if (seq_len <= 0 || nchunks < 0 || window < 0)
    return sabre_fail(SABRE_ERR_INVALID_ARG, "%s: bad sizes", who);
  if ((seq_len + 63) / 64 > 65535)
    return sabre_fail(SABRE_ERR_UNSUPPORTED, "%s: seq_len %d > %d", who, seq_len, 65535 * 64);
  r->chunk = tok_chunk;
  r->group = tok_group;
  r->global = tok_global;
  r->deps = dep_bits;
  r->nchunks = nchunks;
  r->dwords = (nchunks + 31) / 32;
  r->L = seq_len;
  r->window = window;
  return SABRE_OK;
}

int sabre_token_block_mask(const int32_t* tok_chunk, const int32_t* tok_group, const uint8_t* tok_global,
                           const uint32_t* dep_bits, int nchunks, int seq_len, int window, uint32_t* row_bits,
                           void* stream) {
  using namespace sabre::tokmask;
  TokenRule r;
  int st = token_rule(&r, tok_chunk, tok_group, tok_global, dep_bits, nchunks, seq_len, window,
                      "sabre_token_block_mask");
  if (st != SABRE_OK) return st;
  if (!row_bits) return sabre_fail(SABRE_ERR_INVALID_ARG, "sabre_token_block_mask: null row_bits");
  const int nb = (seq_len + kB - 1) / kB;
  const int nwords = (nb + 31) / 32;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaError_t e = cudaMemsetAsync(row_bits, 0, static_cast<size_t>(nb) * nwords * sizeof(uint32_t), s);
  if (e != cudaSuccess) return sabre_cuda_fail(e, "sabre_token_block_mask memset");
  token_block_pairs_kernel<<<dim3(nb, nb), kB, 0, s>>>(r, row_bits, nwords);
  e = cudaGetLastError();
  if (e != cudaSuccess) return sabre_cuda_fail(e, "sabre_token_block_mask launch");
  return SABRE_OK;
}

int sabre_token_tile_masks(const int32_t* tok_chunk, const int32_t* tok_group, const uint8_t* tok_global,
                           const uint32_t* dep_bits, int nchunks, int seq_len, int window, const int32_t* indices,
                           int cap, const int32_t* counts, const int32_t* row_ptr, uint64_t* masks, void* stream) {
  using namespace sabre::tokmask;
  TokenRule r;
  int st = token_rule(&r, tok_chunk, tok_group, tok_global, dep_bits, nchunks, seq_len, window,
                      "sabre_token_tile_masks");
  if (st != SABRE_OK) return st;
  if (!indices || !counts || !row_ptr || !masks || cap <= 0)
    return sabre_fail(SABRE_ERR_INVALID_ARG, "sabre_token_tile_masks: null list or output");
  const int nb = (seq_len + kB - 1) / kB;
  token_tile_masks_kernel<<<dim3(cap, nb), kB, 0, static_cast<cudaStream_t>(stream)>>>(
      r, indices, cap, counts, row_ptr, reinterpret_cast<unsigned long long*>(masks));
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return sabre_cuda_fail(e, "sabre_token_tile_masks launch");
  return SABRE_OK;
}

}  // extern "C"
