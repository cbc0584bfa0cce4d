// Chunk-similarity dependency edges on the GPU.
//
// Replaces StructureAwareMaskBuilder._get_or_build_similarity_vectors and
// _similarity_edges (methods/sabrecoder/sabrecoder_attention_triton.py:490-682):
//   vector(chunk) = fp16( normalize( mean of the chunk's token embeddings ) )
//   score(s, t)   = <vector(s), vector(t)> in fp32, -inf when s and t are the same chunk
//   edges(s)      = the k highest-scoring targets, the chunk itself dropped
// The host keeps the text side (cleaning, tokenising, choosing k) exactly as
// the reference does; these kernels do the gathers, reductions and selection.
//
// Every reduction runs in a fixed order so the results are reproducible:
//   mean     sum over the chunk's tokens first to last (fp32), one division
//   norm     thread t of 256 sums the squares of d = t, t+256, ... in order,
//            then a halving tree over the 256 partials; sqrt; max(norm, 1e-12)
//   score    lane l of a warp sums the products of d = l, l+32, ... in order
//            (products rounded, no fused multiply-add), then an xor tree over
//            the 32 lanes (strides 16, 8, 4, 2, 1)
//   top-k    value descending, ties to the lower target position (the
//            reference's torch.topk leaves the order of exact ties open)
#include <type_traits>

#include "common.cuh"

namespace sabre {
namespace sim {

constexpr int kVecThreads = 256;
constexpr int kMaxPerThread = 32;  // dim <= 8192
constexpr int kTopkThreads = 256;
constexpr int kMaxK = 64;

template <typename E>
__device__ __forceinline__ float emb_f(const E* p) {
  if constexpr (std::is_same<E, float>::value) return *p;
  else return DT<E>::to_f(*p);
}

template <typename E>
__global__ void __launch_bounds__(kVecThreads) chunk_vectors_kernel(const E* emb, int vocab, int dim,
                                                                    const int32_t* tok_ptr, const int32_t* tok_ids,
                                                                    __half* out) {
  __shared__ float red[kVecThreads];
  const int c = blockIdx.x;
  const int tid = threadIdx.x;
  const int t0 = tok_ptr[c], t1 = tok_ptr[c + 1];
  float acc[kMaxPerThread];
#pragma unroll
  for (int i = 0; i < kMaxPerThread; ++i) acc[i] = 0.f;
  for (int j = t0; j < t1; ++j) {
    const int id = tok_ids[j];
    if (id < 0 || id >= vocab) continue;  // rejected on the host; never read out of range
    const E* row = emb + static_cast<long long>(id) * dim;
#pragma unroll
    for (int i = 0; i < kMaxPerThread; ++i) {
      const int d = tid + i * kVecThreads;
      if (d < dim) acc[i] = __fadd_rn(acc[i], emb_f(row + d));
    }
  }
  const float n = static_cast<float>(max(t1 - t0, 1));
  float part = 0.f;
#pragma unroll
  for (int i = 0; i < kMaxPerThread; ++i) {
    const int d = tid + i * kVecThreads;
    if (d < dim) {
      acc[i] = __fdiv_rn(acc[i], n);
      part = __fadd_rn(part, __fmul_rn(acc[i], acc[i]));
    }
  }
  red[tid] = part;
  __syncthreads();
  for (int s = kVecThreads / 2; s > 0; s >>= 1) {
    if (tid < s) red[tid] = __fadd_rn(red[tid], red[tid + s]);
    __syncthreads();
  }
  const float denom = fmaxf(__fsqrt_rn(red[0]), 1e-12f);
  __half* o = out + static_cast<long long>(c) * dim;
#pragma unroll
  for (int i = 0; i < kMaxPerThread; ++i) {
    const int d = tid + i * kVecThreads;
    if (d < dim) o[d] = __float2half_rn(__fdiv_rn(acc[i], denom));
  }
}

// One CTA per source row: scores against every target into shared memory,
// then warp 0 picks the k best.
__global__ void __launch_bounds__(kTopkThreads) similarity_topk_kernel(const __half* vecs, int dim,
                                                                      const int32_t* src_rows, const int32_t* src_chunk,
                                                                      const int32_t* tgt_rows, const int32_t* tgt_chunk,
                                                                      int ntgt, int k, int32_t* out) {
  extern __shared__ float sims[];  // [ntgt] then taken flags as bytes
  unsigned char* taken = reinterpret_cast<unsigned char*>(sims + ntgt);
  const int s = blockIdx.x;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const __half* a = vecs + static_cast<long long>(src_rows[s]) * dim;
  const int schunk = src_chunk[s];
  for (int t = warp; t < ntgt; t += kTopkThreads / 32) {
    const __half* bv = vecs + static_cast<long long>(tgt_rows[t]) * dim;
    float p = 0.f;
    for (int d = lane; d < dim; d += 32) p = __fadd_rn(p, __fmul_rn(__half2float(a[d]), __half2float(bv[d])));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) p = __fadd_rn(p, __shfl_xor_sync(0xffffffffu, p, o));
    if (lane == 0) {
      sims[t] = (tgt_chunk[t] == schunk) ? -INFINITY : p;
      taken[t] = 0;
    }
  }
  __syncthreads();
  if (warp != 0) return;
  const int kk = min(k, ntgt);
  for (int r = 0; r < kk; ++r) {
    float best = 0.f;
    int bi = -1;
    for (int t = lane; t < ntgt; t += 32) {
      if (taken[t]) continue;
      const float v = sims[t];
      if (bi < 0 || v > best) {  // ascending t per lane: ties keep the lower position
        best = v;
        bi = t;
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, best, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      const bool take = (oi >= 0) && (bi < 0 || ov > best || (ov == best && oi < bi));
      if (take) {
        best = ov;
        bi = oi;
      }
    }
    if (lane == 0) {
      taken[bi] = 1;
      // The chunk itself is dropped from its own edges.
      out[static_cast<long long>(s) * k + r] = (tgt_chunk[bi] == schunk) ? -1 : tgt_chunk[bi];
    }
    __syncwarp();
  }
  for (int r = kk + lane; r < k; r += 32) out[static_cast<long long>(s) * k + r] = -1;
}

}  // namespace sim
}  // namespace sabre

using namespace sabre;

extern "C" {

int sabre_chunk_vectors(const void* embedding, int emb_dtype, int vocab, int dim, const int32_t* tok_ptr,
                        const int32_t* tok_ids, int nchunks, void* out_f16, void* stream) {
  using namespace sabre::sim;
  // tok_ids may be null only when no chunk has a token (it is never read then).
  if (!embedding || !tok_ptr || !out_f16)
    return sabre_fail(SABRE_ERR_INVALID_ARG, "sabre_chunk_vectors: null pointer argument");
  if (vocab <= 0 || dim <= 0 || nchunks < 0)
    return sabre_fail(SABRE_ERR_INVALID_ARG, "sabre_chunk_vectors: sizes must be positive");
  if (dim > kVecThreads * kMaxPerThread)
    return sabre_fail(SABRE_ERR_UNSUPPORTED, "sabre_chunk_vectors: dim %d > %d", dim, kVecThreads * kMaxPerThread);
  if (nchunks == 0) return SABRE_OK;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  __half* out = static_cast<__half*>(out_f16);
  if (emb_dtype == SABRE_BF16)
    chunk_vectors_kernel<__nv_bfloat16><<<nchunks, kVecThreads, 0, s>>>(
        static_cast<const __nv_bfloat16*>(embedding), vocab, dim, tok_ptr, tok_ids, out);
  else if (emb_dtype == SABRE_F16)
    chunk_vectors_kernel<__half><<<nchunks, kVecThreads, 0, s>>>(static_cast<const __half*>(embedding), vocab,
                                                                  dim, tok_ptr, tok_ids, out);
  else if (emb_dtype == SABRE_F32)
    chunk_vectors_kernel<float><<<nchunks, kVecThreads, 0, s>>>(static_cast<const float*>(embedding), vocab, dim,
                                                                 tok_ptr, tok_ids, out);
  else
    return sabre_fail(SABRE_ERR_INVALID_ARG, "sabre_chunk_vectors: dtype %d", emb_dtype);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return sabre_cuda_fail(e, "sabre_chunk_vectors launch");
  return SABRE_OK;
}

int sabre_similarity_topk(const void* vecs_f16, int dim, const int32_t* src_rows, const int32_t* src_chunk,
                          int nsrc, const int32_t* tgt_rows, const int32_t* tgt_chunk, int ntgt, int k,
                          int32_t* out_tgt_chunk, void* stream) {
  using namespace sabre::sim;
  if (!vecs_f16 || !src_rows || !src_chunk || !tgt_rows || !tgt_chunk || !out_tgt_chunk)
    return sabre_fail(SABRE_ERR_INVALID_ARG, "sabre_similarity_topk: null pointer argument");
  if (dim <= 0 || nsrc < 0 || ntgt < 0 || k <= 0)
    return sabre_fail(SABRE_ERR_INVALID_ARG, "sabre_similarity_topk: bad sizes");
  if (k > kMaxK) return sabre_fail(SABRE_ERR_UNSUPPORTED, "sabre_similarity_topk: k %d > %d", k, kMaxK);
  const size_t smem = static_cast<size_t>(ntgt) * (sizeof(float) + 1);
  if (smem > 200 * 1024)
    return sabre_fail(SABRE_ERR_UNSUPPORTED, "sabre_similarity_topk: %d targets exceed shared memory", ntgt);
  if (nsrc == 0) return SABRE_OK;
  if (ntgt == 0) {
    cudaError_t e = cudaMemsetAsync(out_tgt_chunk, 0xff, static_cast<size_t>(nsrc) * k * sizeof(int32_t),
                                    static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return sabre_cuda_fail(e, "sabre_similarity_topk memset");
    return SABRE_OK;
  }
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(similarity_topk_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem));
    if (e != cudaSuccess) return sabre_cuda_fail(e, "cudaFuncSetAttribute(similarity_topk_kernel)");
  }
  similarity_topk_kernel<<<nsrc, kTopkThreads, smem, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const __half*>(vecs_f16), dim, src_rows, src_chunk, tgt_rows, tgt_chunk, ntgt, k, out_tgt_chunk);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return sabre_cuda_fail(e, "sabre_similarity_topk launch");
  return SABRE_OK;
}

}  // extern "C"
