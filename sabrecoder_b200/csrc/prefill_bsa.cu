// Block-sparse causal prefill attention for sm_100a (B200).
//
// Replaces `_fwd_kernel_sabrecoder` (methods/sabrecoder/sabrecoder_attention_triton.py:28-116,
// launched at :2039-2053). Same mathematics: for every query row, an online
// softmax over the keys of the listed key blocks with key <= query, scale
// 1/sqrt(D) (:67), P rounded to the input dtype before P.V (:107), fully
// masked rows output zeros (:112).
//
// Design (one CTA = 128 query rows of one head; 224 threads; 2 CTAs per SM):
//   warps 0-3  softmax + epilogue; thread t owns query row t = TMEM lane t
//   warp 4     TMA producer for Q and K (2-stage ring: K stage j%2 is
//              released once S(j) has completed)
//   warp 5     TMEM allocator and single-thread tcgen05.mma issuer
//   warp 6     TMA producer for V (2-stage ring, released when P.V completes)
// Two S buffers, with P written over its own S: S(j+1) is issued right after
// P.V(j-1) (which read P(j-1) from the columns S(j+1) overwrites; the tensor
// pipe runs a thread's MMAs in issue order), so it is computed while the
// softmax works on S(j), and the softmax never waits for a P buffer.
// Each commit costs the tensor pipe about as much as a small MMA, so a key
// tile takes one: C(j), issued after P.V(j) and S(j+2), on DONE[j%2] (S(0)
// and S(1) commit to PRO[0], PRO[1]). C(j) is the softmax's "S(j+2) ready",
// the V producer's "stage j%2 free", the K producer's "stage j%2 free" for
// K(j+4), and the softmax's wait before it rescales O or reads it out.
// Every waiter takes each barrier's completions in order and a barrier's
// next completion needs its waiter's own next step, so a parity wait never
// confuses two phases (tests/test_prefill_protocol.py checks the protocol
// under random schedules).
// TMEM (256 columns): O [0,128), S0 [128,192), S1 [192,256); P(j) (bf16
// pairs) over the first 32 columns of S(j%2).
//   S = Q K^T      M=128 N=64  K=128, A and B from shared memory
//   O += P V       M=128 N=128 K=64,  A (P) from TMEM, B (V) from shared
//                  memory (MN-major)
// Shared memory (bytes): Q 32768 | K 2x16384 | V 2x16384 | key-tile bitmaps
// 256 | barriers (~96.5 KB).
// A CTA's fixed costs are kept off its critical path: the Q tile is
// requested right after the barriers are set up, while the block lists are
// still being read, and each softmax thread writes its finished output row
// straight to global memory with 16-byte stores (no staging, no wait for a
// bulk store to drain before the CTA can exit).
// Q is read once and O written once, so both go through L2 with an
// evict-first policy: the K/V rows that other CTAs of the head still read
// keep their place in L2.
//
// The key-tile list of a CTA is the union of the lists of the (one or two)
// query blocks its rows belong to, kept as two 1024-bit bitmaps (one per
// 64-row half) so any list order, duplicates and out-of-range entries are
// handled without sorting; a half masks the key tiles it does not list.
// Causal masking is per element: key < ks + nvalid where
// nvalid = clamp(row - ks + 1, 0, 64).
// The running max used to scale P is only raised when the row max grows by
// more than 2^8 (the result is exact: O and l share the same stale max);
// O in TMEM is then rescaled by the softmax threads between P.V MMAs.
// All waits are bounded (see common.cuh); on a timeout every role drains
// what it issued, TMEM is freed and the CTA exits.
#include "common.cuh"

namespace sabre {
namespace prefill {

constexpr int kD = 128;
constexpr int kTileM = 128;
constexpr int kTileN = 64;
constexpr int kKStages = 2;
constexpr int kVStages = 2;
constexpr int kMaxKeyTiles = 1024;  // seq_len <= 65536
constexpr int kWords = kMaxKeyTiles / 32;
constexpr int kThreads = 224;

constexpr int kQBytes = kTileM * kD * 2;        // 32768
constexpr int kKVStageBytes = kTileN * kD * 2;  // 16384 (two 8 KB d-halves)
constexpr int kQOff = 0;
constexpr int kKOff = kQOff + kQBytes;
constexpr int kVOff = kKOff + kKStages * kKVStageBytes;
constexpr int kBitsOff = kVOff + kVStages * kKVStageBytes;
constexpr int kBarOff = kBitsOff + 2 * kWords * 4;
static_assert(kKStages == 2 && kVStages == 2, "K and V stage j%2 go with S buffer j%2");
enum Bar {
  Q_FULL = 0,
  K_FULL = 1,                     // [kKStages]
  V_FULL = K_FULL + kKStages,     // [2]
  PRO = V_FULL + kVStages,        // [2] S(0), S(1) done (one completion each)
  DONE = PRO + 2,                 // [2] commit C(j) on DONE[j%2]: P.V(j) and S(j+2) done
  P_FULL = DONE + 2,              // [2] P(j) stored over S buffer j%2 (one arrival per softmax warp)
  MMA_DONE = P_FULL + 2,
  NUM_BARS = MMA_DONE + 1
};
constexpr int kMiscOff = kBarOff + NUM_BARS * 8;
constexpr int kSmemBytes = kMiscOff + 16;
constexpr uint32_t kTmemCols = 256;
constexpr uint32_t kTmemS = 128;  // + 64 * buffer: S(j) fp32, then P(j) (bf16 pairs) over its first 32 columns

struct Params {
  // Token-level variant only (block size 64): the 64-bit row masks of every
  // listed (query block, key block) pair, in list order from tmask_ptr[qb].
  const unsigned long long* tmask;
  const int32_t* tmask_ptr;
  void* o;                      // output rows, written with 16-byte stores
  long long o_sb, o_sh, o_sl;   // element strides (d stride 1)
  const int32_t* idx;
  const int32_t* cnt;
  long long idx_sb, idx_sh, idx_sm, idx_sk;
  long long cnt_sb, cnt_sh, cnt_sm;
  int B, Hq, Hkv, L, block, max_active, ntiles, nkt;
  int head_major;  // grid (tiles, B*Hq) instead of (B*Hq, tiles)
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

// Maximum of 64 scores: a tree of three-input maxima (32 instructions, depth 4).
__device__ __forceinline__ float row_max64(const float (&x)[64]) {
  float a[22];
#pragma unroll
  for (int i = 0; i < 21; ++i) a[i] = fmax3(x[3 * i], x[3 * i + 1], x[3 * i + 2]);
  a[21] = x[63];
  float b[8];
#pragma unroll
  for (int i = 0; i < 7; ++i) b[i] = fmax3(a[3 * i], a[3 * i + 1], a[3 * i + 2]);
  b[7] = a[21];
  return fmax3(fmax3(b[0], b[1], b[2]), fmax3(b[3], b[4], b[5]), fmaxf(b[6], b[7]));
}

// P = 2^(x * sl2 - moff) for one row of 64 scores (-inf gives 0), packed
// two per word in the storage type, and the row sum of the fp32 values (four
// packed partial sums, added in a fixed order). The scale/offset and the sums
// use the packed f32x2 forms: half the FMA-pipe instructions of scalar code.
template <typename T>
__device__ __forceinline__ float exp_tile(const float (&x)[64], float sl2, float moff, uint32_t (&pk)[32]) {
  const uint64_t sc = f2_pack(sl2, sl2);
  const uint64_t off = f2_pack(-moff, -moff);
  uint64_t acc[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) acc[i] = f2_pack(0.f, 0.f);
#pragma unroll
  for (int i = 0; i < 32; ++i) {
    float y0, y1;
    f2_unpack(f2_fma(f2_pack(x[2 * i], x[2 * i + 1]), sc, off), y0, y1);
    const float p0 = ex2(y0);
    const float p1 = ex2(y1);
    acc[i & 3] = f2_add(acc[i & 3], f2_pack(p0, p1));
    pk[i] = DT<T>::pack(p0, p1);
  }
  float s[8];
#pragma unroll
  for (int i = 0; i < 4; ++i) f2_unpack(acc[i], s[2 * i], s[2 * i + 1]);
  return ((s[0] + s[1]) + (s[2] + s[3])) + ((s[4] + s[5]) + (s[6] + s[7]));
}

// kTok: also apply the token-level masks of the listed blocks (Params::tmask).
template <typename T, bool kTok>
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

  // Heaviest (last) query tiles first: later rows list more key blocks.
  // Row-major (grid x = head): the heaviest tiles of all heads run first,
  // the best tail. Head-major (grid x = tile, for K/V larger than L2): the
  // tiles of one head run together, so the K/V rows of the few heads in
  // flight stay in L2 instead of being re-read from HBM.
  const int bh = p.head_major ? static_cast<int>(blockIdx.y) : static_cast<int>(blockIdx.x);
  const int b = bh / p.Hq;
  const int h = bh - b * p.Hq;
  const int hk = h / (p.Hq / p.Hkv);
  const int tile = p.ntiles - 1 - static_cast<int>(p.head_major ? blockIdx.x : blockIdx.y);
  const int r0 = tile * kTileM;

  if (tid == 0) {
    const bool bad = (sbase & 1023u) != 0u;
    *abort_flag = bad ? 1 : 0;
    if (bad) record_status(SABRE_DEV_BAD_SMEM_ALIGN);
  }
  for (int i = tid; i < 2 * kWords; i += kThreads) bits[i] = 0u;
  if (warp == 4 && lane == 0) {
    mbar_init(bar(Q_FULL), 1);
    for (int s = 0; s < kKStages; ++s) mbar_init(bar(K_FULL + s), 1);
    for (int s = 0; s < 2; ++s) {
      mbar_init(bar(V_FULL + s), 1);
      mbar_init(bar(PRO + s), 1);
      mbar_init(bar(DONE + s), 1);
      mbar_init(bar(P_FULL + s), 4);
    }
    mbar_init(bar(MMA_DONE), 1);
    fence_mbar_init();
    tma_prefetch_desc(&tmK);
    tma_prefetch_desc(&tmV);
    if ((sbase & 1023u) == 0u) {
      mbar_arrive_expect_tx(bar(Q_FULL), kQBytes);
      const uint64_t pol = l2_policy_evict_first();
      tma_load_4d_hint(sbase + kQOff, &tmQ, bar(Q_FULL), 0, r0, h, b, pol);
      tma_load_4d_hint(sbase + kQOff + kQBytes / 2, &tmQ, bar(Q_FULL), 64, r0, h, b, pol);
    }
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

  if (warp == 4 || warp == 6) {
    // ---------------- TMA producers (warp 4: Q and K, warp 6: V) ----------------
    if (lane == 0 && start_ok) {
      const bool is_k = (warp == 4);
      const int stages = is_k ? kKStages : kVStages;
      const int full0 = is_k ? K_FULL : V_FULL;
      // DONE[b]'s k-th completion is C(b + 2(k-1)): K(j) may overwrite stage
      // j%2 after S(j-2) (PRO[j-2] for j < 4, else in C(j-4)), V(j) after
      // P.V(j-2) (in C(j-2)). Every waiter takes a barrier's completions in
      // order, so no parity wait can mistake one for another.
      const uint32_t ring = sbase + (is_k ? kKOff : kVOff);
      const CUtensorMap* map = is_k ? &tmK : &tmV;
      int issued[kKStages > kVStages ? kKStages : kVStages] = {};
      UnionIter it(bits, bits + kWords, nw);
      for (int j = 0;; ++j) {
        const int kt = it.next();
        if (kt < 0) break;
        const int s = j % stages;
        if (j >= 2) {
          const int wb = is_k ? (j < 4 ? PRO + (j - 2) : DONE + s) : DONE + s;
          const int par = is_k ? (j < 4 ? 0 : (j >> 1) & 1) : ((j >> 1) - 1) & 1;
          if (!mbar_wait(bar(wb), par, abort_flag)) break;
        }
        mbar_arrive_expect_tx(bar(full0 + s), kKVStageBytes);
        const uint32_t dst = ring + s * kKVStageBytes;
        tma_load_4d(dst, map, bar(full0 + s), 0, kt * 64, hk, b);
        tma_load_4d(dst + kKVStageBytes / 2, map, bar(full0 + s), 64, kt * 64, hk, b);
        ++issued[s];
      }
      // Every issued copy must land before the CTA may exit.
      if (is_k) mbar_wait_drain(bar(Q_FULL), 0);
      for (int s = 0; s < stages; ++s)
        if (issued[s] > 0) mbar_wait_drain(bar(full0 + s), (issued[s] - 1) & 1);
    }
  } else if (warp == 5) {
    // ---------------- MMA issuer ----------------
    if (lane == 0 && start_ok) {
      // This thread shares its SM sub-partition with softmax warps that want
      // every issue slot, so its path is kept short: all shared-memory
      // descriptors are built once and stepped by adding constants to the
      // start-address field (units of 16 bytes; no carry out of the field).
      const uint64_t qd = smem_desc_sw128(sbase + kQOff, 16, 1024);
      const uint64_t kd0 = smem_desc_sw128(sbase + kKOff, 16, 1024);
      const uint64_t vd0 = smem_desc_sw128(sbase + kVOff, kKVStageBytes / 2, 1024);
      const uint32_t s_tmem = tmem + kTmemS;
      bool ok = mbar_wait(bar(Q_FULL), 0, abort_flag);
      // S(j) into S buffer j%2; it is issued after P.V(j-2), which read P(j-2)
      // from the same columns (the tensor pipe runs a thread's MMAs in order).
      // One commit per key tile: C(j) after P.V(j) and S(j+2), on DONE[j%2];
      // S(0) and S(1) commit to PRO[0], PRO[1].
      auto issue_s = [&](int j) -> bool {
        const int ks = j & 1;
        if (!mbar_wait(bar(K_FULL + ks), (j >> 1) & 1, abort_flag)) return false;
        tc_fence_after();
        const uint64_t kd = kd0 + static_cast<uint64_t>(ks * (kKVStageBytes >> 4));
        const uint32_t dst = s_tmem + 64 * (j & 1);
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const uint64_t qo = ((kk >> 2) * (kQBytes / 2) + (kk & 3) * 32) >> 4;
          const uint64_t ko = ((kk >> 2) * (kKVStageBytes / 2) + (kk & 3) * 32) >> 4;
          mma_f16_ss(dst, qd + qo, kd + ko, kIdescQK, kk > 0 ? 1u : 0u);
        }
        return true;
      };
      auto issue_pv = [&](int i) -> bool {
        const int pb = i & 1;
        if (!mbar_wait(bar(P_FULL + pb), (i >> 1) & 1, abort_flag)) return false;
        if (!mbar_wait(bar(V_FULL + pb), (i >> 1) & 1, abort_flag)) return false;
        tc_fence_after();
        const uint64_t vd = vd0 + static_cast<uint64_t>(pb * (kKVStageBytes >> 4));
        const uint32_t pa = s_tmem + 64 * pb;
        mma_f16_ts(tmem, pa, vd, kIdescPV, i > 0 ? 1u : 0u);
#pragma unroll
        for (int kk = 1; kk < 4; ++kk) mma_f16_ts(tmem, pa + 8 * kk, vd + kk * (2048 >> 4), kIdescPV, 1u);
        return true;
      };
      for (int j = 0; ok && j < 2 && j < n; ++j) {
        ok = issue_s(j);
        if (ok) mma_commit(bar(PRO + j));
      }
      for (int j = 0; ok && j < n; ++j) {
        if (!issue_pv(j)) { ok = false; break; }
        if (j + 2 < n && !issue_s(j + 2)) { ok = false; break; }
        mma_commit(bar(DONE + (j & 1)));
      }
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
    // Token-level variant: this half's listed tiles come in ascending order,
    // so a tile's position in its (ascending) list is a running count.
    int rank = 0;
    const bool trow = kTok && (r0 + half * 64) < p.L;
    const long long tbase = trow ? p.tmask_ptr[(r0 + half * 64) / 64] : 0;
    // Reads never pass this row's own masks, even for lists other than the
    // ones the masks were written for (a missing mask hides the whole tile).
    const int tcount = trow ? min(p.cnt[b * p.cnt_sb + h * p.cnt_sh + ((r0 + half * 64) / 64) * p.cnt_sm],
                                  p.max_active) : 0;
    UnionIter it(bits, bits + kWords, nw);
    // Token-level variant: a tile's mask word is loaded one tile ahead, so
    // the load has a whole softmax step to arrive (it decides whether the
    // warp skips the tile, before the S wait).
    auto tok_load = [&](int kt2) -> unsigned long long {
      const bool v2 = (bits[half * kWords + (kt2 >> 5)] >> (kt2 & 31)) & 1u;
      const unsigned long long w2 = (v2 && rank < tcount) ? p.tmask[(tbase + rank) * 64 + (row & 63)] : 0ull;
      rank += v2 ? 1 : 0;
      return w2;
    };
    int kt_ahead = -1;
    unsigned long long tw_ahead = 0ull;
    if constexpr (kTok) {
      if (n > 0) {
        kt_ahead = it.next();
        tw_ahead = tok_load(kt_ahead);
      }
    }
    for (int j = 0; ok && j < n; ++j) {
      int kt;
      unsigned long long tw = ~0ull;
      if constexpr (kTok) {
        kt = kt_ahead;
        tw = tw_ahead;
        if (j + 1 < n) {
          kt_ahead = it.next();
          tw_ahead = tok_load(kt_ahead);
        }
      } else {
        kt = it.next();
      }
      const bool vis = (bits[half * kWords + (kt >> 5)] >> (kt & 31)) & 1u;
      const int nvalid = vis ? min(64, max(0, r_abs - kt * 64 + 1)) : 0;
      // A warp whose 32 rows see no key of this tile (the tile is listed
      // only by the other half, lies wholly after the rows, or their token
      // masks hide it) stores P = 0 and leaves the exponential unit to the
      // other warps of its SM sub-partition.
      const bool dead = __all_sync(0xffffffffu, nvalid == 0 || (kTok && tw == 0ull));
      const int sb = j & 1;
      const uint32_t ts = tl + kTmemS + 64 * sb;
      // S(j): PRO[j] for j < 2, else in C(j-2)
      ok = j < 2 ? mbar_wait_warp(bar(PRO + j), 0, abort_flag)
                 : mbar_wait_warp(bar(DONE + sb), ((j >> 1) - 1) & 1, abort_flag);
      if (!ok) break;
      tc_fence_after();
      uint32_t pk[32];
      bool rescale = false;
      float alpha = 1.0f;
      if (dead) {
#pragma unroll
        for (int c = 0; c < 32; ++c) pk[c] = 0u;
      } else {
        uint32_t sr0[32], sr1[32];
        tmem_ld32(ts, sr0);
        tmem_ld32(ts + 32, sr1);
        tmem_wait_ld();
        float x[64];
#pragma unroll
        for (int c = 0; c < 32; ++c) {
          x[c] = __uint_as_float(sr0[c]);
          x[c + 32] = __uint_as_float(sr1[c]);
        }
        if (nvalid < 64 || (kTok && tw != ~0ull)) {
#pragma unroll
          for (int c = 0; c < 64; ++c)
            if (c >= nvalid || !((tw >> c) & 1ull)) x[c] = -INFINITY;
        }
        const float mx = row_max64(x);
        const float m_tile = mx * sl2;
        rescale = m_tile > m_run + 8.0f;
        const float m_use = rescale ? m_tile : m_run;
        alpha = rescale ? ex2(m_run - m_use) : 1.0f;
        const float moff = (m_use == -INFINITY) ? 0.0f : m_use;
        const float rs = exp_tile<T>(x, sl2, moff, pk);
        l_run = l_run * alpha + rs;
        m_run = m_use;
      }

      // O must not change under a running P.V: rescale only after P.V(j-1).
      if (j >= 1 && __any_sync(0xffffffffu, rescale)) {
        // P.V(j-1) is in C(j-1)
        ok = mbar_wait_warp(bar(DONE + ((j - 1) & 1)), ((j - 1) >> 1) & 1, abort_flag);
        if (!ok) break;
        tc_fence_after();
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
      // P(j) over S(j) (already read into registers).
      tmem_st32(ts, pk);
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar(P_FULL + sb));
    }
    // Epilogue: O / l, each thread stores its own row (256 bytes).
    if (ok && n >= 1) {
      ok = mbar_wait(bar(DONE + ((n - 1) & 1)), ((n - 1) >> 1) & 1, abort_flag);
      ok = __all_sync(0xffffffffu, ok);
      tc_fence_after();
    } else if (ok) {
      // No key tile: the Q load issued at the start must land before the CTA exits.
      ok = mbar_wait(bar(Q_FULL), 0, abort_flag);
      ok = __all_sync(0xffffffffu, ok);
    }
    ok = __all_sync(0xffffffffu, ok);
    // After a timeout anywhere in the CTA the tile is incomplete: store nothing.
    if (ok && *abort_flag == 0) {
      const float inv = (l_run > 0.f) ? 1.0f / l_run : 0.0f;
      T* orow = static_cast<T*>(p.o) + b * p.o_sb + h * p.o_sh + static_cast<long long>(r_abs) * p.o_sl;
      const bool row_ok = r_abs < p.L;
      const uint64_t opol = l2_policy_evict_first();
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
        uint32_t pkd[16];
#pragma unroll
        for (int c = 0; c < 32; c += 2)
          pkd[c >> 1] = DT<T>::pack(__uint_as_float(ov[c]) * inv, __uint_as_float(ov[c + 1]) * inv);
        if (row_ok) {
          uint4* dst = reinterpret_cast<uint4*>(orow + ch * 32);
#pragma unroll
          for (int q4 = 0; q4 < 4; ++q4)
            st_global_v4_hint(dst + q4, make_uint4(pkd[4 * q4], pkd[4 * q4 + 1], pkd[4 * q4 + 2], pkd[4 * q4 + 3]),
                              opol);
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
