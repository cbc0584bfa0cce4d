// Block-sparse causal prefill attention for sm_100a (B200).
//
// Replaces `_fwd_kernel_sabrecoder` (methods/sabrecoder/sabrecoder_attention_triton.py:28-116,
// launched at :2039-2053). Same mathematics: for every query row, an online
// softmax over the keys of the listed key blocks with key <= query, scale
// 1/sqrt(D) (:67), P rounded to the input dtype before P.V (:107), fully
// masked rows output zeros (:112).
//
// Design (one CTA = 128 query rows of one head; 192 threads; 2 CTAs per SM):
//   warps 0-3  softmax + epilogue; thread t owns query row t = TMEM lane t
//   warp 4     TMA producer: Q tile once, then K/V key tiles (64 keys each)
//              into a 2-stage ring, only for the key tiles that the two
//              64-row halves of the query tile list
//   warp 5     TMEM allocator and single-thread tcgen05.mma issuer:
//              S = Q K^T (M=128, N=64, K=128) into a double-buffered TMEM
//              S tile, then O += P V (M=128, N=128, K=64) into TMEM O.
// TMEM: O at columns [0,128), S buffers at [128,192) and [192,256).
// Shared memory (bytes): Q 32768 | K 2x16384 | V 2x16384 | P 16384 |
// per-half key-tile bitmaps 256 | barriers | misc  (~112.4 KB).
// The key-tile list of a CTA is the union of the lists of the (one or two)
// query blocks its rows belong to, kept as two 1024-bit bitmaps (one per
// 64-row half) so any list order, duplicates and out-of-range entries are
// handled without sorting; a half masks the key tiles it does not list.
// Causal masking is per element: key < ks + nvalid where
// nvalid = clamp(row - ks + 1, 0, 64).
// The running max used to scale P is only raised when the row max grows by
// more than 2^8 (the result is exact: O and l share the same stale max);
// O in TMEM is then rescaled by the softmax threads between P.V MMAs.
#include "common.cuh"

namespace sabre {
namespace prefill {

constexpr int kD = 128;
constexpr int kTileM = 128;
constexpr int kTileN = 64;
constexpr int kStages = 2;
constexpr int kMaxKeyTiles = 1024;  // seq_len <= 65536
constexpr int kWords = kMaxKeyTiles / 32;
constexpr int kThreads = 192;

constexpr int kQBytes = kTileM * kD * 2;         // 32768
constexpr int kKVStageBytes = kTileN * kD * 2;   // 16384 (two 8 KB d-halves)
constexpr int kQOff = 0;
constexpr int kKOff = kQOff + kQBytes;
constexpr int kVOff = kKOff + kStages * kKVStageBytes;
constexpr int kPOff = kVOff + kStages * kKVStageBytes;
constexpr int kBitsOff = kPOff + kTileM * kTileN * 2;
constexpr int kBarOff = kBitsOff + 2 * kWords * 4;
enum Bar { Q_FULL = 0, KV_FULL = 1, KV_EMPTY = 3, S_FULL = 5, S_EMPTY = 7, P_FULL = 9, P_EMPTY = 10, MMA_DONE = 11,
           NUM_BARS = 12 };
constexpr int kMiscOff = kBarOff + NUM_BARS * 8;
constexpr int kSmemBytes = kMiscOff + 16;
constexpr uint32_t kTmemCols = 256;

struct Params {
  const int32_t* idx;
  const int32_t* cnt;
  void* o;
  long long idx_sb, idx_sh, idx_sm, idx_sk;
  long long cnt_sb, cnt_sh, cnt_sm;
  long long o_sb, o_sh, o_sl;
  int B, Hq, Hkv, L, block, max_active, ntiles, nkt;
  float scale_log2;
};

// Iterates the set bits of (a | b) over words [0, nw) in ascending order.
struct UnionIter {
  const uint32_t* a;
  const uint32_t* b;
  int w, nw;
  uint32_t cur;
  __device__ UnionIter(const uint32_t* a_, const uint32_t* b_, int nw_) : a(a_), b(b_), w(0), nw(nw_) {
    cur = nw_ > 0 ? (a_[0] | b_[0]) : 0u;
  }
  __device__ int next() {
    while (cur == 0u) {
      if (++w >= nw) return -1;
      cur = a[w] | b[w];
    }
    const int bit = __ffs(cur) - 1;
    cur &= cur - 1u;
    return w * 32 + bit;
  }
};

template <typename T>
__global__ void __launch_bounds__(kThreads, 2)
    prefill_bsa_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                       const __grid_constant__ CUtensorMap tmV, const Params p) {
  extern __shared__ __align__(1024) uint8_t smem[];
  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const uint32_t sbase = smem_u32(smem);
  uint32_t* bits = reinterpret_cast<uint32_t*>(smem + kBitsOff);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + kMiscOff);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + kMiscOff + 4);
  auto bar = [&](int i) -> uint32_t { return sbase + kBarOff + 8u * i; };

  const int bh = blockIdx.x;
  const int b = bh / p.Hq;
  const int h = bh - b * p.Hq;
  const int hk = h / (p.Hq / p.Hkv);
  // Heaviest (last) query tiles first: later rows list more key blocks.
  const int tile = p.ntiles - 1 - static_cast<int>(blockIdx.y);
  const int r0 = tile * kTileM;

  if (tid == 0) {
    const bool bad = (sbase & 1023u) != 0u;
    *abort_flag = bad ? 1 : 0;
    if (bad) record_status(SABRE_DEV_BAD_SMEM_ALIGN);
  }
  for (int i = tid; i < 2 * kWords; i += kThreads) bits[i] = 0u;
  if (warp == 4 && lane == 0) {
    mbar_init(bar(Q_FULL), 1);
    for (int s = 0; s < kStages; ++s) {
      mbar_init(bar(KV_FULL + s), 1);
      mbar_init(bar(KV_EMPTY + s), 1);
      mbar_init(bar(S_FULL + s), 1);
      mbar_init(bar(S_EMPTY + s), 128);
    }
    mbar_init(bar(P_FULL), 128);
    mbar_init(bar(P_EMPTY), 1);
    mbar_init(bar(MMA_DONE), 1);
    fence_mbar_init();
    tma_prefetch_desc(&tmQ);
    tma_prefetch_desc(&tmK);
    tma_prefetch_desc(&tmV);
  }
  if (warp == 5) {
    tmem_alloc(smem_u32(tmem_slot), kTmemCols);
    tmem_relinquish();
  }
  __syncthreads();

  // Key-tile bitmaps of the two 64-row halves from their query blocks' lists.
  if (tid < 128) {
    const int half = tid >> 6;
    const int rstart = r0 + half * 64;
    if (rstart < p.L) {
      const int qb = rstart / p.block;
      const int nb = (p.L + p.block - 1) / p.block;
      const int tpb = p.block / 64;
      const int32_t* ip = p.idx + b * p.idx_sb + h * p.idx_sh + qb * p.idx_sm;
      int c = p.cnt[b * p.cnt_sb + h * p.cnt_sh + qb * p.cnt_sm];
      c = min(c, p.max_active);
      for (int i = tid & 63; i < c; i += 64) {
        const int kb = ip[i * p.idx_sk];
        if (kb < 0 || kb > qb || kb >= nb) continue;
        for (int u = 0; u < tpb; ++u) {
          const int kt = kb * tpb + u;
          if (kt < p.nkt) atomicOr(&bits[half * kWords + (kt >> 5)], 1u << (kt & 31));
        }
      }
    }
  }
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const int last_kt = min(p.nkt - 1, (r0 + kTileM - 1) / 64);
  const int nw = last_kt / 32 + 1;
  int n = 0;
  for (int w = 0; w < nw; ++w) n += __popc(bits[w] | bits[kWords + w]);
  const bool start_ok = (*abort_flag == 0);

  constexpr uint32_t kIdescQK = idesc_f16(128, 64, DT<T>::kBf16, false);
  constexpr uint32_t kIdescPV = idesc_f16(128, 128, DT<T>::kBf16, true);

  if (warp == 4) {
    // ---------------- TMA producer ----------------
    if (lane == 0 && start_ok) {
      int issued[kStages] = {0, 0};
      mbar_arrive_expect_tx(bar(Q_FULL), kQBytes);
      tma_load_4d(sbase + kQOff, &tmQ, bar(Q_FULL), 0, r0, h, b);
      tma_load_4d(sbase + kQOff + kQBytes / 2, &tmQ, bar(Q_FULL), 64, r0, h, b);
      UnionIter it(bits, bits + kWords, nw);
      for (int j = 0;; ++j) {
        const int kt = it.next();
        if (kt < 0) break;
        const int s = j & 1;
        if (!mbar_wait(bar(KV_EMPTY + s), ((j >> 1) & 1) ^ 1, abort_flag)) break;
        mbar_arrive_expect_tx(bar(KV_FULL + s), 2 * kKVStageBytes);
        const uint32_t kd = sbase + kKOff + s * kKVStageBytes;
        const uint32_t vd = sbase + kVOff + s * kKVStageBytes;
        tma_load_4d(kd, &tmK, bar(KV_FULL + s), 0, kt * 64, hk, b);
        tma_load_4d(kd + kKVStageBytes / 2, &tmK, bar(KV_FULL + s), 64, kt * 64, hk, b);
        tma_load_4d(vd, &tmV, bar(KV_FULL + s), 0, kt * 64, hk, b);
        tma_load_4d(vd + kKVStageBytes / 2, &tmV, bar(KV_FULL + s), 64, kt * 64, hk, b);
        ++issued[s];
      }
      // Every issued copy must land before the CTA may exit.
      mbar_wait_drain(bar(Q_FULL), 0);
      for (int s = 0; s < kStages; ++s)
        if (issued[s] > 0) mbar_wait_drain(bar(KV_FULL + s), (issued[s] - 1) & 1);
    }
  } else if (warp == 5) {
    // ---------------- MMA issuer ----------------
    if (lane == 0 && start_ok) {
      const uint32_t qa = sbase + kQOff;
      const uint32_t pa = sbase + kPOff;
      bool ok = mbar_wait(bar(Q_FULL), 0, abort_flag);
      auto issue_pv = [&](int j1) -> bool {
        const int s1 = j1 & 1;
        if (!mbar_wait(bar(P_FULL), j1 & 1, abort_flag)) return false;
        tc_fence_after();
        const uint32_t va = sbase + kVOff + s1 * kKVStageBytes;
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
          const uint64_t ad = smem_desc_sw128(pa + kk * 32, 16, 1024);
          const uint64_t bd = smem_desc_sw128(va + kk * 2048, kKVStageBytes / 2, 1024);
          mma_f16_ss(tmem, ad, bd, kIdescPV, (j1 > 0 || kk > 0) ? 1u : 0u);
        }
        mma_commit(bar(KV_EMPTY + s1));
        mma_commit(bar(P_EMPTY));
        return true;
      };
      for (int j = 0; ok && j < n; ++j) {
        const int s = j & 1;
        const int ph = (j >> 1) & 1;
        if (!mbar_wait(bar(KV_FULL + s), ph, abort_flag)) { ok = false; break; }
        if (!mbar_wait(bar(S_EMPTY + s), ph ^ 1, abort_flag)) { ok = false; break; }
        tc_fence_after();
        const uint32_t ka = sbase + kKOff + s * kKVStageBytes;
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const uint64_t ad = smem_desc_sw128(qa + (kk >> 2) * (kQBytes / 2) + (kk & 3) * 32, 16, 1024);
          const uint64_t bd = smem_desc_sw128(ka + (kk >> 2) * (kKVStageBytes / 2) + (kk & 3) * 32, 16, 1024);
          mma_f16_ss(tmem + 128 + 64 * s, ad, bd, kIdescQK, kk > 0 ? 1u : 0u);
        }
        mma_commit(bar(S_FULL + s));
        if (j >= 1 && !issue_pv(j - 1)) { ok = false; break; }
      }
      if (ok && n >= 1) issue_pv(n - 1);
      // Whatever was issued must finish before TMEM is released.
      mma_commit(bar(MMA_DONE));
      mbar_wait_drain(bar(MMA_DONE), 0);
    }
  } else {
    // ---------------- softmax + epilogue (warps 0-3) ----------------
    const int row = tid;
    const int r_abs = r0 + row;
    const int half = row >> 6;
    const uint32_t tl = tmem + (static_cast<uint32_t>(warp * 32) << 16);
    const float sl2 = p.scale_log2;
    float m_run = -INFINITY;
    float l_run = 0.f;
    bool ok = start_ok;
    UnionIter it(bits, bits + kWords, nw);
    for (int j = 0; ok && j < n; ++j) {
      const int kt = it.next();
      const int s = j & 1;
      ok = mbar_wait(bar(S_FULL + s), (j >> 1) & 1, abort_flag);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) break;
      tc_fence_after();
      uint32_t sr0[32], sr1[32];
      tmem_ld32(tl + 128 + 64 * s, sr0);
      tmem_ld32(tl + 128 + 64 * s + 32, sr1);
      tmem_wait_ld();
      tc_fence_before();
      mbar_arrive(bar(S_EMPTY + s));

      const bool vis = (bits[half * kWords + (kt >> 5)] >> (kt & 31)) & 1u;
      const int nvalid = vis ? min(64, max(0, r_abs - kt * 64 + 1)) : 0;
      float x[64];
#pragma unroll
      for (int c = 0; c < 32; ++c) {
        x[c] = __uint_as_float(sr0[c]);
        x[c + 32] = __uint_as_float(sr1[c]);
      }
      if (nvalid < 64) {
#pragma unroll
        for (int c = 0; c < 64; ++c)
          if (c >= nvalid) x[c] = -INFINITY;
      }
      float mx = x[0];
#pragma unroll
      for (int c = 1; c < 64; ++c) mx = fmaxf(mx, x[c]);
      const float m_tile = mx * sl2;
      const bool rescale = m_tile > m_run + 8.0f;
      const float m_use = rescale ? m_tile : m_run;
      const float alpha = rescale ? ex2(m_run - m_use) : 1.0f;
      const float moff = (m_use == -INFINITY) ? 0.0f : m_use;
      float rs = 0.f;
      uint32_t pk[32];
#pragma unroll
      for (int c = 0; c < 64; c += 2) {
        const float p0 = ex2(fmaf(x[c], sl2, -moff));
        const float p1 = ex2(fmaf(x[c + 1], sl2, -moff));
        rs += p0 + p1;
        pk[c >> 1] = DT<T>::pack(p0, p1);
      }
      l_run = l_run * alpha + rs;
      m_run = m_use;

      // P.V of the previous key tile must be done before P is overwritten
      // and before O is rescaled.
      if (j >= 1) {
        ok = mbar_wait(bar(P_EMPTY), (j - 1) & 1, abort_flag);
        ok = __all_sync(0xffffffffu, ok);
        if (!ok) break;
        tc_fence_after();
        if (__any_sync(0xffffffffu, rescale)) {
#pragma unroll 1
          for (int ch = 0; ch < 4; ++ch) {
            uint32_t ov[32];
            tmem_ld32(tl + ch * 32, ov);
            tmem_wait_ld();
#pragma unroll
            for (int c = 0; c < 32; ++c) ov[c] = __float_as_uint(__uint_as_float(ov[c]) * alpha);
            tmem_st32(tl + ch * 32, ov);
          }
          tmem_wait_st();
        }
      }
      uint8_t* prow = smem + kPOff + row * 128;
#pragma unroll
      for (int c8 = 0; c8 < 8; ++c8) {
        *reinterpret_cast<uint4*>(prow + ((c8 ^ (row & 7)) << 4)) =
            make_uint4(pk[4 * c8], pk[4 * c8 + 1], pk[4 * c8 + 2], pk[4 * c8 + 3]);
      }
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(bar(P_FULL));
    }
    // Epilogue: O / l -> global, one row per thread.
    if (ok && n >= 1) {
      ok = mbar_wait(bar(P_EMPTY), (n - 1) & 1, abort_flag);
      ok = __all_sync(0xffffffffu, ok);
      tc_fence_after();
    }
    if (ok) {
      const float inv = (l_run > 0.f) ? 1.0f / l_run : 0.0f;
      T* orow = reinterpret_cast<T*>(p.o) + b * p.o_sb + h * p.o_sh + static_cast<long long>(r_abs) * p.o_sl;
#pragma unroll 1
      for (int ch = 0; ch < 4; ++ch) {
        uint32_t ov[32];
        if (n >= 1) {
          tmem_ld32(tl + ch * 32, ov);
          tmem_wait_ld();
        } else {
#pragma unroll
          for (int c = 0; c < 32; ++c) ov[c] = 0u;
        }
        if (r_abs < p.L) {
          uint32_t pkd[16];
#pragma unroll
          for (int c = 0; c < 32; c += 2)
            pkd[c >> 1] = DT<T>::pack(__uint_as_float(ov[c]) * inv, __uint_as_float(ov[c + 1]) * inv);
          uint4* dst = reinterpret_cast<uint4*>(orow + ch * 32);
#pragma unroll
          for (int q4 = 0; q4 < 4; ++q4)
            dst[q4] = make_uint4(pkd[4 * q4], pkd[4 * q4 + 1], pkd[4 * q4 + 2], pkd[4 * q4 + 3]);
        }
      }
    }
  }

  __syncthreads();
  if (warp == 5) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

}  // namespace prefill
}  // namespace sabre
