// Split-K block-sparse decode attention over a KV cache (sm_100a).
//
// The reference decodes one token with dense SDPA over the whole cache
// (methods/sabrecoder/sabrecoder_llama_triton.py:254-268, :305-308); this
// kernel reads only the listed key blocks. It is HBM-bound: each CTA streams
// the K and V rows of its share of one KV head's block list with 16-byte
// coalesced loads (a warp covers 512 contiguous bytes per instruction: two
// 256-byte rows), scores all query heads of the GQA group against each row,
// and keeps an online softmax per (warp half, head). The CTA's partial
// (max, sum, acc[D]) goes to the workspace; a second kernel merges the
// splits in a fixed order, so results are deterministic.
#include "common.cuh"

namespace sabre {
namespace decode {

constexpr int kD = 128;
constexpr int kThreads = 128;       // 4 warps
constexpr int kRowsPerHalf = 4;     // rows per half-warp per step
constexpr int kRowsPerStep = 4 * 2 * kRowsPerHalf;  // 32 rows per CTA step
constexpr int kTargetCtas = 2 * 148;
constexpr int kMaxSplits = 256;
// Merge kernel: for more than kCombineWide splits per query head, four groups
// of kD threads each take every fourth split with 16 loads in flight per
// thread (one round of loads); fewer splits are merged by one group of kD
// threads, 8 loads at a time (measured faster there).
constexpr int kCombineWide = 16;
constexpr int kCombineGroups = 4;
static inline bool combine_wide(int splits) { return splits > kCombineWide; }
static inline int combine_threads(int splits) { return combine_wide(splits) ? kD * kCombineGroups : kD; }

struct Params {
  const void* q;
  const void* kc;
  const void* vc;
  void* o;
  const int32_t* idx;
  const int32_t* cnt;
  const int32_t* seq_lens;
  float* part_acc;  // [B][Hq][splits][D]
  float* part_ml;   // [B][Hq][splits][2]
  long long q_sb, q_sh;
  long long k_sb, k_sh, k_st;
  long long v_sb, v_sh, v_st;
  long long o_sb, o_sh;
  long long idx_sb, idx_sh, idx_sk;
  long long cnt_sb, cnt_sh;
  int B, Hq, Hkv, Tmax, block, max_active, splits, bps;
  float scale_log2;
};

// Splits per (sequence, KV head): enough CTAs for one wave of two per SM.
static inline int choose_splits(int batch, int heads_kv, int max_active) {
  long long groups = static_cast<long long>(batch) * heads_kv;
  int s = static_cast<int>(kTargetCtas / groups);
  s = s < 1 ? 1 : s;
  s = s > max_active ? max_active : s;
  return s > kMaxSplits ? kMaxSplits : s;
}

__device__ __forceinline__ void unpack8(const uint4& u, float (&f)[8], bool bf16) {
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    if (bf16) {
      f[2 * i] = __uint_as_float(w[i] << 16);
      f[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
    } else {
      const __half2 h = *reinterpret_cast<const __half2*>(&w[i]);
      const float2 ff = __half22float2(h);
      f[2 * i] = ff.x;
      f[2 * i + 1] = ff.y;
    }
  }
}

template <typename T, int G>
__global__ void __launch_bounds__(kThreads) decode_split_kernel(const Params p) {
  constexpr bool kBf16 = DT<T>::kBf16;
  // Let the combine kernel (a programmatic dependent launch) become resident
  // now: its griddepcontrol.wait still waits for this whole grid.
  if (threadIdx.x == 0) asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  // Launched as a programmatic dependent of the previous kernel: nothing
  // below may read before that kernel's writes are visible.
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int split = blockIdx.x;
  const int hk = blockIdx.y;
  const int b = blockIdx.z;
  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const int half = lane >> 4;
  const int c = lane & 15;  // 16-byte chunk of the 256-byte row
  const int g = p.Hq / p.Hkv;
  const unsigned full = 0xffffffffu;

  __shared__ float sm_m[8][G];
  __shared__ float sm_l[8][G];
  __shared__ float sm_acc[8][G][kD];

  // q chunk for each head of the group, pre-scaled into the log2 domain.
  float qv[G][8];
#pragma unroll
  for (int gi = 0; gi < G; ++gi) {
    if (gi < g) {
      const T* qp = static_cast<const T*>(p.q) + b * p.q_sb + (hk * g + gi) * p.q_sh + c * 8;
      const uint4 u = *reinterpret_cast<const uint4*>(qp);
      unpack8(u, qv[gi], kBf16);
#pragma unroll
      for (int e = 0; e < 8; ++e) qv[gi][e] *= p.scale_log2;
    } else {
#pragma unroll
      for (int e = 0; e < 8; ++e) qv[gi][e] = 0.f;
    }
  }
  float m[G], l[G], acc[G][8];
#pragma unroll
  for (int gi = 0; gi < G; ++gi) {
    m[gi] = -INFINITY;
    l[gi] = 0.f;
#pragma unroll
    for (int e = 0; e < 8; ++e) acc[gi][e] = 0.f;
  }

  const int T_valid = min(p.seq_lens[b], p.Tmax);
  int cnt = p.cnt[b * p.cnt_sb + hk * p.cnt_sh];
  cnt = min(cnt, p.max_active);
  const int j0 = split * p.bps;
  const int j1 = min(j0 + p.bps, cnt);
  const int32_t* ip = p.idx + b * p.idx_sb + hk * p.idx_sh;
  const T* kbase = static_cast<const T*>(p.kc) + b * p.k_sb + hk * p.k_sh + c * 8;
  const T* vbase = static_cast<const T*>(p.vc) + b * p.v_sb + hk * p.v_sh + c * 8;

  for (int jj = j0; jj < j1; ++jj) {
    const int kb = ip[jj * p.idx_sk];
    if (kb < 0) continue;
    const long long t_blk = static_cast<long long>(kb) * p.block;
    if (t_blk >= T_valid) continue;
    for (int rb = 0; rb < p.block; rb += kRowsPerStep) {
      uint4 kr[kRowsPerHalf], vr[kRowsPerHalf];
      bool valid[kRowsPerHalf];
#pragma unroll
      for (int u = 0; u < kRowsPerHalf; ++u) {
        const int row = rb + warp * (2 * kRowsPerHalf) + 2 * u + half;
        const long long t = t_blk + row;
        valid[u] = (row < p.block) && (t < T_valid);
        if (valid[u]) {
          kr[u] = __ldg(reinterpret_cast<const uint4*>(kbase + t * p.k_st));
          vr[u] = __ldg(reinterpret_cast<const uint4*>(vbase + t * p.v_st));
        } else {
          kr[u] = make_uint4(0u, 0u, 0u, 0u);
          vr[u] = make_uint4(0u, 0u, 0u, 0u);
        }
      }
      float s[kRowsPerHalf][G];
#pragma unroll
      for (int u = 0; u < kRowsPerHalf; ++u) {
        float kf[8];
        unpack8(kr[u], kf, kBf16);
#pragma unroll
        for (int gi = 0; gi < G; ++gi) {
          float d = 0.f;
#pragma unroll
          for (int e = 0; e < 8; ++e) d = fmaf(qv[gi][e], kf[e], d);
          d += __shfl_xor_sync(full, d, 8);
          d += __shfl_xor_sync(full, d, 4);
          d += __shfl_xor_sync(full, d, 2);
          d += __shfl_xor_sync(full, d, 1);
          s[u][gi] = valid[u] ? d : -INFINITY;
        }
      }
#pragma unroll
      for (int gi = 0; gi < G; ++gi) {
        float mt = s[0][gi];
#pragma unroll
        for (int u = 1; u < kRowsPerHalf; ++u) mt = fmaxf(mt, s[u][gi]);
        const float mn = fmaxf(m[gi], mt);
        if (mn == -INFINITY) continue;
        const float alpha = ex2(m[gi] - mn);
        float pr[kRowsPerHalf];
        float ps = 0.f;
#pragma unroll
        for (int u = 0; u < kRowsPerHalf; ++u) {
          pr[u] = ex2(s[u][gi] - mn);
          ps += pr[u];
        }
        l[gi] = l[gi] * alpha + ps;
        m[gi] = mn;
#pragma unroll
        for (int e = 0; e < 8; ++e) acc[gi][e] *= alpha;
#pragma unroll
        for (int u = 0; u < kRowsPerHalf; ++u) {
          float vf[8];
          unpack8(vr[u], vf, kBf16);
#pragma unroll
          for (int e = 0; e < 8; ++e) acc[gi][e] = fmaf(pr[u], vf[e], acc[gi][e]);
        }
      }
    }
  }

  // Merge the 8 (warp, half) partial states of the CTA.
  const int grp = warp * 2 + half;
#pragma unroll
  for (int gi = 0; gi < G; ++gi) {
    if (c == 0) {
      sm_m[grp][gi] = m[gi];
      sm_l[grp][gi] = l[gi];
    }
#pragma unroll
    for (int e = 0; e < 8; ++e) sm_acc[grp][gi][c * 8 + e] = acc[gi][e];
  }
  __syncthreads();
  const int d = tid;  // kThreads == kD
  for (int gi = 0; gi < g && gi < G; ++gi) {
    float M = -INFINITY;
#pragma unroll
    for (int r = 0; r < 8; ++r) M = fmaxf(M, sm_m[r][gi]);
    float L = 0.f, A = 0.f;
    if (M != -INFINITY) {
#pragma unroll
      for (int r = 0; r < 8; ++r) {
        const float w = ex2(sm_m[r][gi] - M);
        L += w * sm_l[r][gi];
        A += w * sm_acc[r][gi][d];
      }
    }
    const long long slot = (static_cast<long long>(b) * p.Hq + (hk * g + gi)) * p.splits + split;
    p.part_acc[slot * kD + d] = A;
    if (d == 0) {
      p.part_ml[slot * 2] = M;
      p.part_ml[slot * 2 + 1] = L;
    }
  }
}

// ---------------------------------------------------------------------------
// Streaming variant for caches whose rows are contiguous per head (row stride
// == head_dim, the layout of a [B, Hkv, T, D] cache): every 64-row chunk of a
// listed block is one 16 KB span of K and one of V, fetched by a single
// producer thread with bulk copies into a kBulkStages-deep shared-memory ring
// (mbarrier completion), while 4 consumer warps score and accumulate from
// shared memory with the same per-(warp half, head) online softmax as above.
// ~96 KB of copies in flight per CTA and 2 CTAs per SM cover HBM latency
// without holding the rows in registers.
// ---------------------------------------------------------------------------
constexpr int kBulkStages = 3;
constexpr int kChunkRows = 64;
constexpr int kChunkBytes = kChunkRows * kD * 2;  // 16384 per tensor
constexpr int kBulkConsumerWarps = 4;
constexpr int kBulkThreads = (kBulkConsumerWarps + 1) * 32;
constexpr int kBulkRingBytes = kBulkStages * 2 * kChunkBytes;
constexpr int kBulkBarOff = kBulkRingBytes;
constexpr int kBulkSmem = kBulkBarOff + 2 * kBulkStages * 8 + 16;
constexpr int kBulkTargetCtas = 2 * 148;

// Chunks of its share a split CTA asks L2 for before griddepcontrol.wait
// (two measured best of one to four).
constexpr int kPrefetchChunks = 2;

// Calls f(t, rows) for the first kPrefetchChunks 64-row chunks of a split's
// share (entries j0 .. j1-1 of the list at ip), for L2 prefetches issued
// before griddepcontrol.wait. The entries may still be written by the
// previous kernel, so a value read here is only a hint: chunks are clamped
// to the cache's Tmax rows and nothing else depends on them.
template <typename F>
__device__ __forceinline__ void prefetch_walk(const int32_t* ip, long long sk, int j0, int j1, int block, int Tmax,
                                              F&& f) {
  int kb[kPrefetchChunks];
#pragma unroll
  for (int i = 0; i < kPrefetchChunks; ++i) kb[i] = (j0 + i < j1) ? ip[(j0 + i) * sk] : -1;
  int left = kPrefetchChunks;
#pragma unroll
  for (int i = 0; i < kPrefetchChunks; ++i) {
    for (int sub = 0; sub < block / 64 && left > 0; ++sub, --left) {
      const long long t = static_cast<long long>(kb[i]) * block + sub * 64;
      if (kb[i] < 0 || t >= Tmax) break;
      f(static_cast<int>(t), static_cast<int>(min(64LL, Tmax - t)));
    }
  }
}

// Walks the 64-row chunks of a split's share of one list: the same sequence
// for the producer and the consumers.
struct ChunkWalk {
  const int32_t* ip;
  long long sk;
  int jj, j1, block, T_valid, kb, sub;
  __device__ ChunkWalk(const int32_t* ip_, long long sk_, int j0, int j1_, int block_, int T_valid_)
      : ip(ip_), sk(sk_), jj(j0 - 1), j1(j1_), block(block_), T_valid(T_valid_), kb(0), sub(0) {
    sub = block_ / kChunkRows;  // forces a fetch on the first next()
  }
  // Starts the walk at entry j0 with its value already read (j0 < j1).
  __device__ void seed(int kb0) {
    if (jj + 1 >= j1) return;
    jj += 1;
    kb = kb0;
    sub = (kb < 0) ? block / kChunkRows : 0;
  }
  // Next chunk: first row t0 and valid rows; false when the share is exhausted.
  __device__ bool next(long long& t0, int& rows) {
    for (;;) {
      if (sub < block / kChunkRows) {
        const long long t = static_cast<long long>(kb) * block + static_cast<long long>(sub) * kChunkRows;
        ++sub;
        if (t < T_valid) {
          t0 = t;
          rows = static_cast<int>(min(static_cast<long long>(kChunkRows), T_valid - t));
          return true;
        }
        sub = block / kChunkRows;
        continue;
      }
      if (++jj >= j1) return false;
      kb = ip[jj * sk];
      sub = (kb < 0) ? block / kChunkRows : 0;
    }
  }
};

template <typename T, int G>
__global__ void __launch_bounds__(kBulkThreads, 2) decode_bulk_kernel(const Params p) {
  constexpr bool kBf16 = DT<T>::kBf16;
  // Let the combine kernel (a programmatic dependent launch) become resident
  // now: its griddepcontrol.wait still waits for this whole grid.
  if (threadIdx.x == 0) asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  extern __shared__ __align__(128) uint8_t smem[];
  const uint32_t sbase = smem_u32(smem);
  const int split = blockIdx.x;
  const int hk = blockIdx.y;
  const int b = blockIdx.z;
  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const int g = p.Hq / p.Hkv;
  const unsigned full = 0xffffffffu;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + kBulkBarOff + 2 * kBulkStages * 8);
  auto full_bar = [&](int s) -> uint32_t { return sbase + kBulkBarOff + 8u * s; };
  auto empty_bar = [&](int s) -> uint32_t { return sbase + kBulkBarOff + 8u * (kBulkStages + s); };

  if (tid == 0) {
    *abort_flag = 0;
    for (int s = 0; s < kBulkStages; ++s) {
      mbar_init(full_bar(s), 1);
      mbar_init(empty_bar(s), kBulkConsumerWarps);
    }
    fence_mbar_init();
  }
  __syncthreads();
  if (warp == kBulkConsumerWarps && lane == 0 && kPrefetchChunks > 0) {
    const T* kb0 = static_cast<const T*>(p.kc) + b * p.k_sb + hk * p.k_sh;
    const T* vb0 = static_cast<const T*>(p.vc) + b * p.v_sb + hk * p.v_sh;
    const int j0p = split * p.bps;
    prefetch_walk(p.idx + b * p.idx_sb + hk * p.idx_sh, p.idx_sk, j0p, min(j0p + p.bps, p.max_active), p.block,
                  p.Tmax, [&](int t, int rows) {
                    bulk_prefetch_l2(kb0 + static_cast<long long>(t) * kD, static_cast<uint32_t>(rows) * kD * 2);
                    bulk_prefetch_l2(vb0 + static_cast<long long>(t) * kD, static_cast<uint32_t>(rows) * kD * 2);
                  });
  }
  // Launched as a programmatic dependent of the previous kernel: the set-up
  // above overlaps its tail; nothing below may read before its writes are
  // visible (the prefetches above are hints). The sequence length, the list
  // count and the split's first index are then independent loads, issued
  // together.
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int T_valid = min(p.seq_lens[b], p.Tmax);
  const unsigned long long wlim = wait_limit_ns();  // read once, not per wait (c1 dense 21.24 -> 21.04 us)
  int cnt = p.cnt[b * p.cnt_sb + hk * p.cnt_sh];
  const int j0 = split * p.bps;
  const int32_t* ip = p.idx + b * p.idx_sb + hk * p.idx_sh;
  const int first_kb = (warp == kBulkConsumerWarps && lane == 0 && j0 < p.max_active) ? ip[j0 * p.idx_sk] : -1;
  cnt = min(cnt, p.max_active);
  const int j1 = min(j0 + p.bps, cnt);
  const T* kbase = static_cast<const T*>(p.kc) + b * p.k_sb + hk * p.k_sh;
  const T* vbase = static_cast<const T*>(p.vc) + b * p.v_sb + hk * p.v_sh;

  float m[G], l[G], acc[G][8];
  if (warp == kBulkConsumerWarps) {
    // ---------------- producer ----------------
    if (lane == 0) {
      ChunkWalk walk(ip, p.idx_sk, j0, j1, p.block, T_valid);
      walk.seed(first_kb);
      long long t0;
      int rows;
      int issued[kBulkStages] = {0, 0, 0};
      for (int i = 0; walk.next(t0, rows); ++i) {
        const int s = i % kBulkStages;
        if (!mbar_wait_lim(empty_bar(s), ((i / kBulkStages) & 1) ^ 1, abort_flag, wlim)) break;
        const uint32_t bytes = static_cast<uint32_t>(rows) * kD * 2;
        mbar_arrive_expect_tx(full_bar(s), 2 * bytes);
        const uint32_t dst = sbase + s * 2 * kChunkBytes;
        bulk_load(dst, kbase + t0 * kD, bytes, full_bar(s));
        bulk_load(dst + kChunkBytes, vbase + t0 * kD, bytes, full_bar(s));
        ++issued[s];
      }
      // Every issued copy must land before the ring is reused or the CTA exits.
      for (int s = 0; s < kBulkStages; ++s)
        if (issued[s] > 0) mbar_wait_drain(full_bar(s), (issued[s] - 1) & 1);
    }
  } else {
    // ---------------- consumers: warp w owns rows [16w, 16w+16) of a chunk ----------------
    const int half = lane >> 4;
    const int c = lane & 15;
    float qv[G][8];
#pragma unroll
    for (int gi = 0; gi < G; ++gi) {
      if (gi < g) {
        const T* qp = static_cast<const T*>(p.q) + b * p.q_sb + (hk * g + gi) * p.q_sh + c * 8;
        const uint4 u = *reinterpret_cast<const uint4*>(qp);
        unpack8(u, qv[gi], kBf16);
#pragma unroll
        for (int e = 0; e < 8; ++e) qv[gi][e] *= p.scale_log2;
      } else {
#pragma unroll
        for (int e = 0; e < 8; ++e) qv[gi][e] = 0.f;
      }
      m[gi] = -INFINITY;
      l[gi] = 0.f;
#pragma unroll
      for (int e = 0; e < 8; ++e) acc[gi][e] = 0.f;
    }
    ChunkWalk walk(ip, p.idx_sk, j0, j1, p.block, T_valid);
    long long t0;
    int rows;
    for (int i = 0; walk.next(t0, rows); ++i) {
      const int s = i % kBulkStages;
      if (!mbar_wait_warp_lim(full_bar(s), (i / kBulkStages) & 1, abort_flag, wlim)) break;
      // The phase is complete; each lane's own probe gives it acquire order on the copied bytes.
      (void)mbar_test_wait(full_bar(s), (i / kBulkStages) & 1);
      const uint4* sk = reinterpret_cast<const uint4*>(smem + s * 2 * kChunkBytes);
      const uint4* sv = reinterpret_cast<const uint4*>(smem + s * 2 * kChunkBytes + kChunkBytes);
#pragma unroll
      for (int batch = 0; batch < 2; ++batch) {
        uint4 kr[kRowsPerHalf], vr[kRowsPerHalf];
        bool valid[kRowsPerHalf];
#pragma unroll
        for (int u = 0; u < kRowsPerHalf; ++u) {
          const int row = warp * 16 + half * 8 + batch * kRowsPerHalf + u;
          valid[u] = row < rows;
          kr[u] = valid[u] ? sk[row * 16 + c] : make_uint4(0u, 0u, 0u, 0u);
          vr[u] = valid[u] ? sv[row * 16 + c] : make_uint4(0u, 0u, 0u, 0u);
        }
        float sc[kRowsPerHalf][G];
#pragma unroll
        for (int u = 0; u < kRowsPerHalf; ++u) {
          float kf[8];
          unpack8(kr[u], kf, kBf16);
#pragma unroll
          for (int gi = 0; gi < G; ++gi) {
            float d = 0.f;
#pragma unroll
            for (int e = 0; e < 8; ++e) d = fmaf(qv[gi][e], kf[e], d);
            d += __shfl_xor_sync(full, d, 8);
            d += __shfl_xor_sync(full, d, 4);
            d += __shfl_xor_sync(full, d, 2);
            d += __shfl_xor_sync(full, d, 1);
            sc[u][gi] = valid[u] ? d : -INFINITY;
          }
        }
#pragma unroll
        for (int gi = 0; gi < G; ++gi) {
          float mt = sc[0][gi];
#pragma unroll
          for (int u = 1; u < kRowsPerHalf; ++u) mt = fmaxf(mt, sc[u][gi]);
          const float mn = fmaxf(m[gi], mt);
          if (mn == -INFINITY) continue;
          const float alpha = ex2(m[gi] - mn);
          float pr[kRowsPerHalf];
          float ps = 0.f;
#pragma unroll
          for (int u = 0; u < kRowsPerHalf; ++u) {
            pr[u] = ex2(sc[u][gi] - mn);
            ps += pr[u];
          }
          l[gi] = l[gi] * alpha + ps;
          m[gi] = mn;
#pragma unroll
          for (int e = 0; e < 8; ++e) acc[gi][e] *= alpha;
#pragma unroll
          for (int u = 0; u < kRowsPerHalf; ++u) {
            float vf[8];
            unpack8(vr[u], vf, kBf16);
#pragma unroll
            for (int e = 0; e < 8; ++e) acc[gi][e] = fmaf(pr[u], vf[e], acc[gi][e]);
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(empty_bar(s));
    }
  }
  __syncthreads();  // the ring is idle from here on: reuse it for the merge

  float* sm_m = reinterpret_cast<float*>(smem);            // [8][G]
  float* sm_l = sm_m + 8 * G;                              // [8][G]
  float* sm_acc = sm_l + 8 * G;                            // [8][G][kD]
  if (warp < kBulkConsumerWarps) {
    const int half = lane >> 4;
    const int c = lane & 15;
    const int grp = warp * 2 + half;
#pragma unroll
    for (int gi = 0; gi < G; ++gi) {
      if (c == 0) {
        sm_m[grp * G + gi] = m[gi];
        sm_l[grp * G + gi] = l[gi];
      }
#pragma unroll
      for (int e = 0; e < 8; ++e) sm_acc[(grp * G + gi) * kD + c * 8 + e] = acc[gi][e];
    }
  }
  __syncthreads();
  if (tid < kD) {
    const int d = tid;
    for (int gi = 0; gi < g && gi < G; ++gi) {
      float M = -INFINITY;
#pragma unroll
      for (int r = 0; r < 8; ++r) M = fmaxf(M, sm_m[r * G + gi]);
      float L = 0.f, A = 0.f;
      if (M != -INFINITY) {
#pragma unroll
        for (int r = 0; r < 8; ++r) {
          const float w = ex2(sm_m[r * G + gi] - M);
          L += w * sm_l[r * G + gi];
          A += w * sm_acc[(r * G + gi) * kD + d];
        }
      }
      const long long slot = (static_cast<long long>(b) * p.Hq + (hk * g + gi)) * p.splits + split;
      p.part_acc[slot * kD + d] = A;
      if (d == 0) {
        p.part_ml[slot * 2] = M;
        p.part_ml[slot * 2 + 1] = L;
      }
    }
  }
}

// One CTA per (b, query head): merge the splits. Launched as a programmatic
// dependent of the split kernel: it may start while the split kernel's last
// CTAs run, and waits here until that grid has finished and its partials are
// visible.
// The (m, l) of all splits are read in one parallel pass into shared memory;
// each of kGroups thread groups then sums every kGroups-th split's acc
// values with kBatch loads issued together (with 4 groups of 16, one round
// trip for up to 64 splits), and the group sums are added in group order, so
// the result is deterministic.
template <typename T, int kGroups, int kBatch>
__global__ void __launch_bounds__(kD * kGroups) decode_combine_kernel(const Params p) {
  // The next decode call's split kernel (a programmatic dependent too) may
  // start its set-up now; it waits for this grid before touching memory.
  if (threadIdx.x == 0) asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  asm volatile("griddepcontrol.wait;" ::: "memory");
  __shared__ float sm_m[kMaxSplits], sm_l[kMaxSplits];
  __shared__ float sm_L[kGroups][kD], sm_A[kGroups][kD];
  const int bh = blockIdx.x;
  const int b = bh / p.Hq;
  const int h = bh - b * p.Hq;
  const int d = threadIdx.x % kD;
  const int grp = threadIdx.x / kD;
  const long long base = static_cast<long long>(bh) * p.splits;
  // Thread group g takes splits g, g + G, g + 2G, ... with kBatch loads in
  // flight; the first batch is requested together with the (m, l) pass.
  float a[kBatch];
#pragma unroll
  for (int u = 0; u < kBatch; ++u) {
    const int s = grp + u * kGroups;
    a[u] = (s < p.splits) ? p.part_acc[(base + s) * kD + d] : 0.f;
  }
  for (int s = threadIdx.x; s < p.splits; s += kD * kGroups) {
    sm_m[s] = p.part_ml[(base + s) * 2];
    sm_l[s] = p.part_ml[(base + s) * 2 + 1];
  }
  __syncthreads();
  float M = -INFINITY;
  for (int s = 0; s < p.splits; ++s) M = fmaxf(M, sm_m[s]);
  float L = 0.f, A = 0.f;
  if (M != -INFINITY) {
    for (int s0 = grp; s0 < p.splits; s0 += kGroups * kBatch) {
      if (s0 != grp) {
#pragma unroll
        for (int u = 0; u < kBatch; ++u) {
          const int s = s0 + u * kGroups;
          a[u] = (s < p.splits) ? p.part_acc[(base + s) * kD + d] : 0.f;
        }
      }
#pragma unroll
      for (int u = 0; u < kBatch; ++u) {
        const int s = s0 + u * kGroups;
        if (s < p.splits) {
          const float w = ex2(sm_m[s] - M);
          L += w * sm_l[s];
          A += w * a[u];
        }
      }
    }
  }
  if constexpr (kGroups == 1) {
    const float out = (L > 0.f) ? A / L : 0.f;
    T* op = static_cast<T*>(p.o) + b * p.o_sb + h * p.o_sh;
    op[d] = DT<T>::from_f(out);
    return;
  }
  sm_L[grp][d] = L;
  sm_A[grp][d] = A;
  __syncthreads();
  if (grp == 0) {
    float Lt = 0.f, At = 0.f;
#pragma unroll
    for (int g = 0; g < kGroups; ++g) {  // fixed order: deterministic
      Lt += sm_L[g][d];
      At += sm_A[g][d];
    }
    const float out = (Lt > 0.f) ? At / Lt : 0.f;
    T* op = static_cast<T*>(p.o) + b * p.o_sb + h * p.o_sh;
    op[d] = DT<T>::from_f(out);
  }
}

template <typename T, int G>
static void launch_split(const Params& p, bool bulk, cudaStream_t s) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(p.splits, p.Hkv, p.B);
  cfg.blockDim = dim3(bulk ? kBulkThreads : kThreads);
  cfg.dynamicSmemBytes = bulk ? kBulkSmem : 0;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (bulk)
    cudaLaunchKernelEx(&cfg, decode_bulk_kernel<T, G>, p);
  else
    cudaLaunchKernelEx(&cfg, decode_split_kernel<T, G>, p);
}

// Groups of at least this many query heads per KV head decode on the tensor
// cores (decode_gqa.cu, defined later in this translation unit): scoring a
// row against that many heads costs the CUDA-core kernels more than reading
// it. The tiles there are 64 rows, so blocks must be multiples of 64.
constexpr int kGqaMinGroup = 3;
static int decode_gqa_launch(const Params& p, int dtype, cudaStream_t s);
static bool use_gqa(const Params& p) {
  return p.Hq / p.Hkv >= kGqaMinGroup && p.block % kChunkRows == 0;
}

// Bulk streaming needs rows contiguous per head and whole 64-row chunks per
// block; other layouts use the register-streaming kernel.
static bool bulk_layout(const Params& p) {
  return p.k_st == kD && p.v_st == kD && p.block % kChunkRows == 0;
}

template <typename T>
static cudaError_t launch_decode(const Params& p, int g, cudaStream_t s) {
  const bool bulk = bulk_layout(p);
  if (bulk) {
    cudaError_t e = cudaSuccess;
    if (g <= 1) e = cudaFuncSetAttribute(decode_bulk_kernel<T, 1>, cudaFuncAttributeMaxDynamicSharedMemorySize, kBulkSmem);
    else if (g <= 2) e = cudaFuncSetAttribute(decode_bulk_kernel<T, 2>, cudaFuncAttributeMaxDynamicSharedMemorySize, kBulkSmem);
    else if (g <= 4) e = cudaFuncSetAttribute(decode_bulk_kernel<T, 4>, cudaFuncAttributeMaxDynamicSharedMemorySize, kBulkSmem);
    else e = cudaFuncSetAttribute(decode_bulk_kernel<T, 8>, cudaFuncAttributeMaxDynamicSharedMemorySize, kBulkSmem);
    if (e != cudaSuccess) return e;
  }
  if (g <= 1)
    launch_split<T, 1>(p, bulk, s);
  else if (g <= 2)
    launch_split<T, 2>(p, bulk, s);
  else if (g <= 4)
    launch_split<T, 4>(p, bulk, s);
  else
    launch_split<T, 8>(p, bulk, s);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(p.B * p.Hq);
  cfg.blockDim = dim3(combine_threads(p.splits));
  cfg.dynamicSmemBytes = 0;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return combine_wide(p.splits) ? cudaLaunchKernelEx(&cfg, decode_combine_kernel<T, kCombineGroups, 16>, p)
                                : cudaLaunchKernelEx(&cfg, decode_combine_kernel<T, 1, 8>, p);
}

}  // namespace decode
}  // namespace sabre

using namespace sabre;

extern "C" {

size_t sabre_decode_workspace_size(int batch, int heads_q, int heads_kv, int head_dim, int max_active) {
  using namespace sabre::decode;
  if (batch <= 0 || heads_q <= 0 || heads_kv <= 0 || head_dim <= 0 || max_active <= 0) return 0;
  const size_t splits = static_cast<size_t>(choose_splits(batch, heads_kv, max_active));
  return static_cast<size_t>(batch) * heads_q * splits * (static_cast<size_t>(head_dim) + 2) * sizeof(float);
}

int sabre_decode_bsa(const void* q, const void* k_cache, const void* v_cache, void* o,
                     const int32_t* block_indices, const int32_t* block_counts, const int32_t* seq_lens,
                     int batch, int heads_q, int heads_kv, int max_seq, int head_dim, int block_size,
                     int max_active, const int64_t* q_strides, const int64_t* k_strides,
                     const int64_t* v_strides, const int64_t* o_strides, const int64_t* idx_strides,
                     const int64_t* cnt_strides, float softmax_scale, int dtype, void* workspace,
                     size_t workspace_bytes, void* stream) {
  using namespace sabre::decode;
  if (!q || !k_cache || !v_cache || !o || !block_indices || !block_counts || !seq_lens || !q_strides ||
      !k_strides || !v_strides || !o_strides || !idx_strides || !cnt_strides)
    return sabre_fail(SABRE_ERR_INVALID_ARG, "sabre_decode_bsa: null pointer argument");
  if (batch <= 0 || heads_q <= 0 || heads_kv <= 0 || max_seq <= 0 || max_active <= 0 || block_size <= 0)
    return sabre_fail(SABRE_ERR_INVALID_ARG, "sabre_decode_bsa: sizes must be positive");
  if (heads_q % heads_kv != 0 || heads_q / heads_kv > 8)
    return sabre_fail(SABRE_ERR_UNSUPPORTED, "sabre_decode_bsa: heads_q/heads_kv must be an integer <= 8");
  if (head_dim != kD) return sabre_fail(SABRE_ERR_UNSUPPORTED, "sabre_decode_bsa: head_dim %d (only 128)", head_dim);
  if (dtype != SABRE_BF16 && dtype != SABRE_F16)
    return sabre_fail(SABRE_ERR_INVALID_ARG, "sabre_decode_bsa: dtype %d", dtype);
  if (q_strides[2] != 1 || k_strides[3] != 1 || v_strides[3] != 1 || o_strides[2] != 1)
    return sabre_fail(SABRE_ERR_UNSUPPORTED, "sabre_decode_bsa: head_dim stride must be 1");
  auto al16 = [](const void* ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 15u) == 0; };
  if (!al16(q) || !al16(k_cache) || !al16(v_cache))
    return sabre_fail(SABRE_ERR_ALIGNMENT, "sabre_decode_bsa: q/k_cache/v_cache must be 16-byte aligned");
  const int64_t ss[6] = {q_strides[0], q_strides[1], k_strides[0], k_strides[1], k_strides[2], v_strides[2]};
  for (int i = 0; i < 6; ++i)
    if ((ss[i] * 2) % 16 != 0)
      return sabre_fail(SABRE_ERR_ALIGNMENT, "sabre_decode_bsa: q/k/v strides must be 16-byte multiples");
  if ((v_strides[0] * 2) % 16 != 0 || (v_strides[1] * 2) % 16 != 0)
    return sabre_fail(SABRE_ERR_ALIGNMENT, "sabre_decode_bsa: v strides must be 16-byte multiples");
  const size_t need = sabre_decode_workspace_size(batch, heads_q, heads_kv, head_dim, max_active);
  if (!workspace || workspace_bytes < need)
    return sabre_fail(SABRE_ERR_WORKSPACE, "sabre_decode_bsa: workspace %zu < %zu bytes", workspace_bytes, need);
  Params p;
  p.q = q;
  p.kc = k_cache;
  p.vc = v_cache;
  p.o = o;
  p.idx = block_indices;
  p.cnt = block_counts;
  p.seq_lens = seq_lens;
  p.q_sb = q_strides[0];
  p.q_sh = q_strides[1];
  p.k_sb = k_strides[0];
  p.k_sh = k_strides[1];
  p.k_st = k_strides[2];
  p.v_sb = v_strides[0];
  p.v_sh = v_strides[1];
  p.v_st = v_strides[2];
  p.o_sb = o_strides[0];
  p.o_sh = o_strides[1];
  p.idx_sb = idx_strides[0];
  p.idx_sh = idx_strides[1];
  p.idx_sk = idx_strides[2];
  p.cnt_sb = cnt_strides[0];
  p.cnt_sh = cnt_strides[1];
  p.B = batch;
  p.Hq = heads_q;
  p.Hkv = heads_kv;
  p.Tmax = max_seq;
  p.block = block_size;
  p.max_active = max_active;
  p.splits = choose_splits(batch, heads_kv, max_active);
  p.bps = (max_active + p.splits - 1) / p.splits;
  const size_t nslots = static_cast<size_t>(batch) * heads_q * p.splits;
  p.part_acc = static_cast<float*>(workspace);
  p.part_ml = p.part_acc + nslots * kD;
  const float scale = softmax_scale > 0.f ? softmax_scale : 1.0f / sqrtf(static_cast<float>(head_dim));
  p.scale_log2 = scale * 1.4426950408889634f;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int g = heads_q / heads_kv;
  if (use_gqa(p)) return decode_gqa_launch(p, dtype, s);
  cudaError_t e;
  if (dtype == SABRE_BF16)
    e = launch_decode<__nv_bfloat16>(p, g, s);
  else
    e = launch_decode<__half>(p, g, s);
  if (e != cudaSuccess) return sabre_cuda_fail(e, "sabre_decode_bsa launch");
  return SABRE_OK;
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Allocation-free decode.
//
// Some callers cannot hand this library a workspace: a serving runtime that
// reserves all device memory at start-up and rejects any later allocation,
// a foreign-language binding with no access to the framework's caching
// allocator, or a latency-critical decode loop where a cudaMalloc would
// synchronise the device. sabre_decode_bsa_noalloc keeps the split partials
// in a fixed array compiled into this library instead.
//
// The array is kNoAllocScratchFloats floats (2 MiB); every GPU that loads the
// library holds it until the process exits. One decode call needs
// batch * heads_q * splits * (head_dim + 2) floats. choose_splits picks
// either one split or a count with splits * batch * heads_kv <= kTargetCtas;
// with at most 8 query heads per KV head the latter needs at most
// kTargetCtas * 8 * (head_dim + 2) floats, which the array holds
// (static_assert below). So the only shapes turned away are those whose
// batch * heads_q * (head_dim + 2) floats do not fit even with one split.
// All calls share the array: calls whose kernels overlap on the GPU (on
// different streams, or on other host threads) race on it. Each call's split
// kernel writes every partial it later reads, so nothing needs clearing
// between calls.
//
// Host code cannot pass the array's name to a kernel (in host code it names a
// host-side stand-in, not device memory), so the device address is looked up
// with cudaGetSymbolAddress once per device, on the first call made while that
// device is current; make that first call before any stream capture.
// ---------------------------------------------------------------------------
#include <mutex>

namespace sabre {
namespace decode {

constexpr size_t kNoAllocScratchFloats = 512u * 1024u;  // 2 MiB
constexpr int kNoAllocMaxDevices = 64;

static_assert(static_cast<size_t>(kTargetCtas) * 8 * (kD + 2) <= kNoAllocScratchFloats,
              "the split partials of every accepted decode shape must fit the no-alloc scratch");

static __device__ __align__(256) float g_noalloc_scratch[kNoAllocScratchFloats];
static float* g_noalloc_scratch_ptr[kNoAllocMaxDevices] = {nullptr};
static std::mutex g_noalloc_mutex;

static int noalloc_scratch_address(float** out) {
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return sabre_cuda_fail(e, "cudaGetDevice");
  if (dev < 0 || dev >= kNoAllocMaxDevices)
    return sabre_fail(SABRE_ERR_UNSUPPORTED, "sabre_decode_bsa_noalloc: device ordinal %d >= %d", dev,
                      kNoAllocMaxDevices);
  std::lock_guard<std::mutex> lock(g_noalloc_mutex);
  if (g_noalloc_scratch_ptr[dev] == nullptr) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess) return sabre_cuda_fail(e, "cudaGetSymbolAddress(g_noalloc_scratch)");
    g_noalloc_scratch_ptr[dev] = static_cast<float*>(p);
  }
  *out = g_noalloc_scratch_ptr[dev];
  return SABRE_OK;
}

}  // namespace decode
}  // namespace sabre

extern "C" {

int sabre_decode_bsa_noalloc(const void* q, const void* k_cache, const void* v_cache, void* o,
                             const int32_t* block_indices, const int32_t* block_counts, const int32_t* seq_lens,
                             int batch, int heads_q, int heads_kv, int max_seq, int head_dim, int block_size,
                             int max_active, const int64_t* q_strides, const int64_t* k_strides,
                             const int64_t* v_strides, const int64_t* o_strides, const int64_t* idx_strides,
                             const int64_t* cnt_strides, float softmax_scale, int dtype, void* stream) {
  using namespace sabre::decode;
  if (!q || !k_cache || !v_cache || !o || !block_indices || !block_counts || !seq_lens || !q_strides ||
      !k_strides || !v_strides || !o_strides || !idx_strides || !cnt_strides)
    return sabre_fail(SABRE_ERR_INVALID_ARG, "sabre_decode_bsa_noalloc: null pointer argument");
  if (batch <= 0 || heads_q <= 0 || heads_kv <= 0 || max_seq <= 0 || max_active <= 0 || block_size <= 0)
    return sabre_fail(SABRE_ERR_INVALID_ARG, "sabre_decode_bsa_noalloc: sizes must be positive");
  if (heads_q % heads_kv != 0 || heads_q / heads_kv > 8)
    return sabre_fail(SABRE_ERR_UNSUPPORTED, "sabre_decode_bsa_noalloc: heads_q/heads_kv must be an integer <= 8");
  if (head_dim != kD)
    return sabre_fail(SABRE_ERR_UNSUPPORTED, "sabre_decode_bsa_noalloc: head_dim %d (only 128)", head_dim);
  if (dtype != SABRE_BF16 && dtype != SABRE_F16)
    return sabre_fail(SABRE_ERR_INVALID_ARG, "sabre_decode_bsa_noalloc: dtype %d", dtype);
  if (q_strides[2] != 1 || k_strides[3] != 1 || v_strides[3] != 1 || o_strides[2] != 1)
    return sabre_fail(SABRE_ERR_UNSUPPORTED, "sabre_decode_bsa_noalloc: head_dim stride must be 1");
  auto al16 = [](const void* ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 15u) == 0; };
  if (!al16(q) || !al16(k_cache) || !al16(v_cache))
    return sabre_fail(SABRE_ERR_ALIGNMENT, "sabre_decode_bsa_noalloc: q/k_cache/v_cache must be 16-byte aligned");
  const int64_t ss[8] = {q_strides[0], q_strides[1], k_strides[0], k_strides[1],
                         k_strides[2], v_strides[0], v_strides[1], v_strides[2]};
  for (int i = 0; i < 8; ++i)
    if ((ss[i] * 2) % 16 != 0)
      return sabre_fail(SABRE_ERR_ALIGNMENT, "sabre_decode_bsa_noalloc: q/k/v strides must be 16-byte multiples");

  // The split partials must fit the fixed array: a shape that fits with one
  // split fits with the count choose_splits picks (static_assert above).
  const size_t per_split = static_cast<size_t>(batch) * heads_q * (static_cast<size_t>(kD) + 2);
  if (per_split > kNoAllocScratchFloats)
    return sabre_fail(SABRE_ERR_UNSUPPORTED,
                      "sabre_decode_bsa_noalloc: batch*heads_q = %lld needs %zu floats of scratch per split; the "
                      "built-in scratch holds %zu floats (2 MiB); use sabre_decode_bsa with a workspace",
                      static_cast<long long>(batch) * heads_q, per_split, kNoAllocScratchFloats);
  float* scratch = nullptr;
  int st = noalloc_scratch_address(&scratch);
  if (st != SABRE_OK) return st;

  Params p;
  p.q = q;
  p.kc = k_cache;
  p.vc = v_cache;
  p.o = o;
  p.idx = block_indices;
  p.cnt = block_counts;
  p.seq_lens = seq_lens;
  p.q_sb = q_strides[0];
  p.q_sh = q_strides[1];
  p.k_sb = k_strides[0];
  p.k_sh = k_strides[1];
  p.k_st = k_strides[2];
  p.v_sb = v_strides[0];
  p.v_sh = v_strides[1];
  p.v_st = v_strides[2];
  p.o_sb = o_strides[0];
  p.o_sh = o_strides[1];
  p.idx_sb = idx_strides[0];
  p.idx_sh = idx_strides[1];
  p.idx_sk = idx_strides[2];
  p.cnt_sb = cnt_strides[0];
  p.cnt_sh = cnt_strides[1];
  p.B = batch;
  p.Hq = heads_q;
  p.Hkv = heads_kv;
  p.Tmax = max_seq;
  p.block = block_size;
  p.max_active = max_active;
  p.splits = choose_splits(batch, heads_kv, max_active);
  p.bps = (max_active + p.splits - 1) / p.splits;
  const size_t nslots = static_cast<size_t>(batch) * heads_q * p.splits;
  p.part_acc = scratch;
  p.part_ml = scratch + nslots * kD;
  const float scale = softmax_scale > 0.f ? softmax_scale : 1.0f / sqrtf(static_cast<float>(head_dim));
  p.scale_log2 = scale * 1.4426950408889634f;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int g = heads_q / heads_kv;
  if (use_gqa(p)) return decode_gqa_launch(p, dtype, s);
  cudaError_t e;
  if (dtype == SABRE_BF16)
    e = launch_decode<__nv_bfloat16>(p, g, s);
  else
    e = launch_decode<__half>(p, g, s);
  if (e != cudaSuccess) return sabre_cuda_fail(e, "sabre_decode_bsa_noalloc launch");
  return SABRE_OK;
}

}  // extern "C"
