// Pooled q.k top-k block selection (extension; no reference counterpart).
//
// Nearest reference analogue: the chunk-similarity top-k of
// methods/sabrecoder/sabrecoder_attention_triton.py:581-682 (mean-pool,
// score, keep the top-k per source). Here, per (batch, head, query block qb):
// score(kb) = sum_d qm[qb][d] * km[kb][d] over the per-block means of the
// rotated Q and K, for causal kb <= qb not already in the structure row; the
// `topk` best are added (higher score first, ties to the lower kb).
//
// The score arithmetic is fixed so the selected blocks are reproducible bit
// for bit: each product is rounded to fp32 and added in order d = 0..D-1
// (no fused multiply-add).
//
// Kernel 1 (scores): 32x32 (qb, kb) tiles of the lower triangle; the 32 qm
// rows and 32 km rows of a tile are staged in shared memory (row pitch D+1
// floats, conflict-free) and each thread produces a 2x2 block of scores.
// Kernel 2 (select): one warp per (b, h, qb) reads its score row, runs
// `topk` warp arg-max rounds over the candidates and writes the merged row as
// an ascending index list.
#include "common.cuh"

namespace sabre {
namespace topk {

constexpr int kTile = 32;
constexpr int kMaxBlocks = 1024;
constexpr int kMaxWordsPerLane = 1;  // nb <= 1024 -> nwords <= 32: one word per lane
constexpr int kCandPerLane = kMaxBlocks / 32;
constexpr int kTopkMax = 32;

__global__ void __launch_bounds__(256) scores_kernel(const float* qm, const float* km, int Hq, int Hkv, int nb,
                                                     int D, float* scores) {
  extern __shared__ float sm[];
  const int kt = blockIdx.x;
  const int qt = blockIdx.y;
  if (kt > qt) return;  // strictly above the diagonal: never a candidate
  const int bh = blockIdx.z;
  const int b = bh / Hq;
  const int h = bh - b * Hq;
  const int hk = h / (Hq / Hkv);
  const int pitch = D + 1;
  float* Qs = sm;
  float* Ks = sm + kTile * pitch;
  const float* qsrc = qm + (static_cast<long long>(bh) * nb + qt * kTile) * D;
  const float* ksrc = km + ((static_cast<long long>(b) * Hkv + hk) * nb + kt * kTile) * D;
  for (int i = threadIdx.x; i < kTile * D; i += blockDim.x) {
    const int r = i / D, d = i - r * D;
    Qs[r * pitch + d] = (qt * kTile + r < nb) ? qsrc[i] : 0.f;
    Ks[r * pitch + d] = (kt * kTile + r < nb) ? ksrc[i] : 0.f;
  }
  __syncthreads();
  const int tx = threadIdx.x & 15;
  const int ty = threadIdx.x >> 4;
  const float* q0 = Qs + (2 * ty) * pitch;
  const float* q1 = q0 + pitch;
  const float* k0 = Ks + (2 * tx) * pitch;
  const float* k1 = k0 + pitch;
  float a00 = 0.f, a01 = 0.f, a10 = 0.f, a11 = 0.f;
  for (int d = 0; d < D; ++d) {
    const float x0 = q0[d], x1 = q1[d], y0 = k0[d], y1 = k1[d];
    a00 = __fadd_rn(a00, __fmul_rn(x0, y0));
    a01 = __fadd_rn(a01, __fmul_rn(x0, y1));
    a10 = __fadd_rn(a10, __fmul_rn(x1, y0));
    a11 = __fadd_rn(a11, __fmul_rn(x1, y1));
  }
  const int qb = qt * kTile + 2 * ty;
  const int kb = kt * kTile + 2 * tx;
  float* srow = scores + (static_cast<long long>(bh) * nb + qb) * nb;
  if (qb < nb) {
    if (kb < nb) srow[kb] = a00;
    if (kb + 1 < nb) srow[kb + 1] = a01;
  }
  if (qb + 1 < nb) {
    if (kb < nb) srow[nb + kb] = a10;
    if (kb + 1 < nb) srow[nb + kb + 1] = a11;
  }
}

__global__ void select_kernel(const float* scores, const uint32_t* base_bits, int B, int Hq, int nb, int topk,
                              int32_t* idx, int cap, int32_t* counts, int32_t* max_active, uint32_t* out_bits) {
  const int lane = threadIdx.x & 31;
  const long long row = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const long long rows = static_cast<long long>(B) * Hq * nb;
  if (row >= rows) return;
  const unsigned full = 0xffffffffu;
  const int qb = static_cast<int>(row % nb);
  const int nwords = (nb + 31) / 32;
  const uint32_t* brow = base_bits + static_cast<long long>(qb) * nwords;
  const float* srow = scores + row * nb;
  const uint32_t myword = (lane < nwords) ? brow[lane] : 0u;

  float sc[kCandPerLane];
  uint32_t live = 0u;  // bit i: candidate kb = lane + 32*i is live
#pragma unroll
  for (int i = 0; i < kCandPerLane; ++i) {
    // candidate kb = lane + 32*i sits in word i (held by lane i), bit `lane`
    const uint32_t w = __shfl_sync(full, myword, i);
    const int kb = lane + 32 * i;
    sc[i] = 0.f;
    if (kb <= qb && kb < nb && !((w >> lane) & 1u)) {
      sc[i] = srow[kb];
      live |= 1u << i;
    }
  }
  uint32_t chosen = 0u;  // lane owns word `lane`
  for (int round = 0; round < topk; ++round) {
    float best = 0.f;
    int bkb = -1;
#pragma unroll
    for (int i = 0; i < kCandPerLane; ++i) {
      if ((live >> i) & 1u) {
        if (bkb < 0 || sc[i] > best) {  // candidates of a lane ascend in kb: strict > keeps the lower kb
          best = sc[i];
          bkb = lane + 32 * i;
        }
      }
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
      const float ob = __shfl_xor_sync(full, best, off);
      const int okb = __shfl_xor_sync(full, bkb, off);
      if (okb >= 0 && (bkb < 0 || ob > best || (ob == best && okb < bkb))) {
        best = ob;
        bkb = okb;
      }
    }
    if (bkb < 0) break;
    if ((bkb & 31) == lane) live &= ~(1u << (bkb >> 5));
    if ((bkb >> 5) == lane) chosen |= 1u << (bkb & 31);
  }
  const uint32_t word = myword | chosen;
  if (out_bits && lane < nwords) out_bits[row * nwords + lane] = word;
  // ascending list from the words (one per lane)
  const int pc = __popc(word);
  int incl = pc;
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) {
    const int y = __shfl_up_sync(full, incl, off);
    if (lane >= off) incl += y;
  }
  const int total = __shfl_sync(full, incl, 31);
  int pos = incl - pc;
  int32_t* out = idx + row * cap;
  uint32_t left = word;
  while (left) {
    const int bpos = __ffs(left) - 1;
    left &= left - 1u;
    if (pos < cap) out[pos] = lane * 32 + bpos;
    ++pos;
  }
  for (int k = total + lane; k < cap; k += 32) out[k] = -1;
  if (lane == 0) {
    counts[row] = total;
    atomicMax(max_active, max(total, 1));
  }
}

}  // namespace topk
}  // namespace sabre

using namespace sabre;

extern "C" {

size_t sabre_topk_workspace_size(int batch, int heads_q, int num_blocks) {
  if (batch <= 0 || heads_q <= 0 || num_blocks <= 0) return 0;
  return static_cast<size_t>(batch) * heads_q * num_blocks * num_blocks * sizeof(float);
}

int sabre_topk_extend(const float* q_pooled, const float* k_pooled, const uint32_t* base_bits, int batch,
                      int heads_q, int heads_kv, int num_blocks, int head_dim, int topk, int32_t* indices, int cap,
                      int32_t* counts, int32_t* max_active_out, uint32_t* out_bits, void* workspace,
                      size_t workspace_bytes, void* stream) {
  using namespace sabre::topk;
  if (!q_pooled || !k_pooled || !base_bits || !indices || !counts || !max_active_out || batch <= 0 ||
      heads_q <= 0 || heads_kv <= 0 || num_blocks <= 0 || head_dim <= 0 || cap <= 0 || topk < 0)
    return sabre_fail(SABRE_ERR_INVALID_ARG, "sabre_topk_extend: bad arguments");
  if (heads_q % heads_kv != 0)
    return sabre_fail(SABRE_ERR_INVALID_ARG, "sabre_topk_extend: heads_q not a multiple of heads_kv");
  if (num_blocks > kMaxBlocks || topk > kTopkMax || head_dim > 256)
    return sabre_fail(SABRE_ERR_UNSUPPORTED,
                      "sabre_topk_extend: num_blocks %d (max %d), topk %d (max %d) or head_dim %d (max 256)",
                      num_blocks, kMaxBlocks, topk, kTopkMax, head_dim);
  const size_t need = sabre_topk_workspace_size(batch, heads_q, num_blocks);
  if (!workspace || workspace_bytes < need)
    return sabre_fail(SABRE_ERR_WORKSPACE, "sabre_topk_extend: workspace %zu < %zu bytes", workspace_bytes, need);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaError_t e = cudaMemsetAsync(max_active_out, 0, sizeof(int32_t), s);
  if (e != cudaSuccess) return sabre_cuda_fail(e, "cudaMemsetAsync(max_active)");
  float* scores = static_cast<float*>(workspace);
  const int tiles = (num_blocks + kTile - 1) / kTile;
  const size_t smem = 2u * kTile * (head_dim + 1) * sizeof(float);
  if (smem > 48u * 1024u) {
    e = cudaFuncSetAttribute(scores_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    if (e != cudaSuccess) return sabre_cuda_fail(e, "cudaFuncSetAttribute(scores_kernel)");
  }
  scores_kernel<<<dim3(tiles, tiles, batch * heads_q), 256, smem, s>>>(q_pooled, k_pooled, heads_q, heads_kv,
                                                                      num_blocks, head_dim, scores);
  const long long rows = static_cast<long long>(batch) * heads_q * num_blocks;
  select_kernel<<<static_cast<unsigned>((rows * 32 + 255) / 256), 256, 0, s>>>(
      scores, base_bits, batch, heads_q, num_blocks, topk, indices, cap, counts, max_active_out, out_bits);
  e = cudaGetLastError();
  if (e != cudaSuccess) return sabre_cuda_fail(e, "sabre_topk_extend launch");
  return SABRE_OK;
}

}  // extern "C"
