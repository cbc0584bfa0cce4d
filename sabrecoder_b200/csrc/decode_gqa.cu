// Split-K block-sparse decode for grouped-query attention on the tensor cores
// (sm_100a). Included by sabre_capi.cu after the TMA descriptor helpers.
//
// Same contract and partials as the CUDA-core split kernels of decode_bsa.cu
// (the reference decodes with dense SDPA, methods/sabrecoder/
// sabrecoder_llama_triton.py:254-268): a CTA owns one split of the block list
// of one (sequence, KV head) and leaves (max, sum, acc[D]) per query head of
// the group for decode_combine_kernel. When one KV head serves many query
// heads, scoring each cache row against every head on the CUDA cores costs
// more than reading the row; here the g query rows of the group form the
// first g rows of a 128-row operand, so a 64-row tile of K and V costs one
// S = Q K^T (M=128 N=64 K=128, operands in shared memory) and one P V (M=128
// N=128 K=64, P from TMEM) whatever g is. Q is stored as 8 rows (rows g..7
// zero); its descriptor steps 0 bytes from one 8-row group to the next, so
// the MMA reads those 8 rows as rows 8..15, 16..23, ... as well. Only rows
// 0..g-1 of the results are read.
//   warp 0  online softmax of rows 0..31 (TMEM lanes 0..31; lane r = head r)
//           and the partials of rows 0..g-1
//   warp 1  TMA producer for K (3 stages)
//   warp 2  TMEM allocator and single-thread tcgen05.mma issuer
//   warp 3  TMA producer for V (3 stages)
// Barrier protocol as in the prefill kernel (S_FULL per K stage, one S
// buffer freed by S_EMPTY, P double-buffered and freed by P_EMPTY), plus
// V_EMPTY per V stage. Keys at or past the sequence length are masked; every
// wait is bounded. The roles walk the split's block list as they go, so the
// first copies are issued after one index load.
namespace sabre {
namespace decode {
namespace gqa {

constexpr int kKStages = 3;
constexpr int kVStages = 3;
constexpr int kThreads = 128;
// Hardware-suspended polls before a wait first reads the clock, at the
// default wait limit (c4 dense, per call in a layer sequence: 20.85 -> 20.35
// us; the bulk decode and prefill kernels measured no gain or a loss).
constexpr int kPolls = 4;
constexpr int kQBytes = 8 * kD * 2;            // 2048: [d-half][8 rows][128 B], 128-byte swizzle
constexpr int kStageBytes = 64 * kD * 2;       // 16384: [d-half][64 rows][128 B]
constexpr int kQOff = 0;
constexpr int kKOff = kQOff + kQBytes;
constexpr int kVOff = kKOff + kKStages * kStageBytes;
constexpr int kBarOff = kVOff + kVStages * kStageBytes;
enum Bar {
  K_FULL = 0,                  // [3]
  V_FULL = K_FULL + kKStages,  // [3]
  S_FULL = V_FULL + kVStages,  // [3] one per K stage; also "K stage free"
  S_EMPTY = S_FULL + kKStages,
  P_FULL = S_EMPTY + 1,        // [2]
  P_EMPTY = P_FULL + 2,        // [2]
  V_EMPTY = P_EMPTY + 2,       // [3] P.V of the stage's tile is done
  MMA_DONE = V_EMPTY + kVStages,
  NUM_BARS = MMA_DONE + 1
};
constexpr int kMiscOff = kBarOff + NUM_BARS * 8;
constexpr int kSmemBytes = kMiscOff + 16;
constexpr uint32_t kTmemCols = 256;
constexpr uint32_t kTmemS = 128;
constexpr uint32_t kTmemP = 192;  // + 32 * buffer

template <typename T>
__global__ void __launch_bounds__(kThreads, 2)
    decode_gqa_kernel(const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmV,
                      const Params p) {
  // Let the combine kernel (a programmatic dependent launch) become resident
  // now: its griddepcontrol.wait still waits for this whole grid.
  if (threadIdx.x == 0) asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  extern __shared__ __align__(1024) uint8_t smem[];
  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const uint32_t sbase = smem_u32(smem);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + kMiscOff);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + kMiscOff + 4);
  auto bar = [&](int i) -> uint32_t { return sbase + kBarOff + 8u * i; };
  const int split = blockIdx.x;
  const int hk = blockIdx.y;
  const int b = blockIdx.z;
  const int g = p.Hq / p.Hkv;

  if (tid == 0) {
    const bool bad = (sbase & 1023u) != 0u;
    *abort_flag = bad ? 1 : 0;
    if (bad) record_status(SABRE_DEV_BAD_SMEM_ALIGN);
    for (int s = 0; s < kKStages; ++s) {
      mbar_init(bar(K_FULL + s), 1);
      mbar_init(bar(S_FULL + s), 1);
    }
    for (int s = 0; s < kVStages; ++s) {
      mbar_init(bar(V_FULL + s), 1);
      mbar_init(bar(V_EMPTY + s), 1);
    }
    mbar_init(bar(S_EMPTY), 1);
    for (int s = 0; s < 2; ++s) {
      mbar_init(bar(P_FULL + s), 1);
      mbar_init(bar(P_EMPTY + s), 1);
    }
    mbar_init(bar(MMA_DONE), 1);
    fence_mbar_init();
    tma_prefetch_desc(&tmK);
    tma_prefetch_desc(&tmV);
  }
  if (warp == 2) {
    tmem_alloc(smem_u32(tmem_slot), kTmemCols);
    tmem_relinquish();
  }
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const bool start_ok = (*abort_flag == 0);
  if (tid == 32 && start_ok && kPrefetchChunks > 0) {
    const int j0p = split * p.bps;
    prefetch_walk(p.idx + b * p.idx_sb + hk * p.idx_sh, p.idx_sk, j0p, min(j0p + p.bps, p.max_active), p.block,
                  p.Tmax, [&](int t, int) {
                    tma_prefetch_l2_4d(&tmK, 0, t, hk, b);
                    tma_prefetch_l2_4d(&tmK, 64, t, hk, b);
                    tma_prefetch_l2_4d(&tmV, 0, t, hk, b);
                    tma_prefetch_l2_4d(&tmV, 64, t, hk, b);
                  });
  }
  // Launched as a programmatic dependent of the previous kernel: the set-up
  // above overlaps its tail; nothing below may read before its writes are
  // visible (the L2 prefetches above are hints).
  asm volatile("griddepcontrol.wait;" ::: "memory");
  // The start-up global loads are independent and issued together: the
  // sequence length, the list count, the split's first index (prefetched for
  // the producers' list walks) and this thread's 16 bytes of Q.
  const int T_valid = min(p.seq_lens[b], p.Tmax);
  const unsigned long long wlim = wait_limit_ns();  // read once, not per wait
  int cnt = p.cnt[b * p.cnt_sb + hk * p.cnt_sh];
  const int j0 = split * p.bps;
  const int32_t* ip = p.idx + b * p.idx_sb + hk * p.idx_sh;
  if (tid == 32 && j0 < p.max_active) asm volatile("prefetch.global.L1 [%0];" ::"l"(ip + j0 * p.idx_sk));
  // Q: row r < g is query head hk*g + r, stored as the 128-byte-swizzled
  // K-major layout a TMA load would produce (16-byte chunk c of row r of a
  // d-half at r*128 + ((c ^ (r & 7)) << 4)); rows g..7 are zero.
  static_assert(2 * 8 * 8 == kThreads, "one 16-byte chunk of Q per thread");
  {
    const int c = tid & 7;
    const int r = (tid >> 3) & 7;
    const int dh = tid >> 6;
    uint4 v = make_uint4(0u, 0u, 0u, 0u);
    if (r < g) {
      const T* qp = static_cast<const T*>(p.q) + b * p.q_sb + (hk * g + r) * p.q_sh + dh * 64 + c * 8;
      v = *reinterpret_cast<const uint4*>(qp);
    }
    *reinterpret_cast<uint4*>(smem + kQOff + dh * (kQBytes / 2) + r * 128 + ((c ^ (r & 7)) << 4)) = v;
  }
  fence_proxy_async_smem();  // the tensor cores read Q through the async proxy
  __syncthreads();

  cnt = min(cnt, p.max_active);
  const int j1 = min(j0 + p.bps, cnt);

  constexpr uint32_t kIdescQK = idesc_f16(128, 64, DT<T>::kBf16, false);
  constexpr uint32_t kIdescPV = idesc_f16(128, 128, DT<T>::kBf16, true);

  if (warp == 1 || warp == 3) {
    // ---------------- TMA producers (warp 1: K, warp 3: V) ----------------
    if (lane == 0 && start_ok) {
      const bool is_k = (warp == 1);
      const int stages = is_k ? kKStages : kVStages;
      const int full0 = is_k ? K_FULL : V_FULL;
      // K stage s is free when S_FULL[s] completes, V stage s when V_EMPTY[s] does.
      const int empty0 = is_k ? S_FULL : V_EMPTY;
      const uint32_t ring = sbase + (is_k ? kKOff : kVOff);
      const CUtensorMap* map = is_k ? &tmK : &tmV;
      int issued[kKStages] = {0, 0, 0};
      ChunkWalk w(ip, p.idx_sk, j0, j1, p.block, T_valid);
      long long t0;
      int rows;
      for (int j = 0; w.next(t0, rows); ++j) {
        const int s = j % stages;
        if (!mbar_wait_lim<kPolls>(bar(empty0 + s), ((j / stages) & 1) ^ 1, abort_flag, wlim)) break;
        mbar_arrive_expect_tx(bar(full0 + s), kStageBytes);
        const uint32_t dst = ring + s * kStageBytes;
        tma_load_4d(dst, map, bar(full0 + s), 0, static_cast<int>(t0), hk, b);
        tma_load_4d(dst + kStageBytes / 2, map, bar(full0 + s), 64, static_cast<int>(t0), hk, b);
        ++issued[s];
      }
      // Every issued copy must land before the CTA may exit.
      for (int s = 0; s < stages; ++s)
        if (issued[s] > 0) mbar_wait_drain(bar(full0 + s), (issued[s] - 1) & 1);
    }
  } else if (warp == 2) {
    // ---------------- MMA issuer ----------------
    if (lane == 0 && start_ok) {
      const uint64_t qd = smem_desc_sw128(sbase + kQOff, 16, 0);  // every 8-row group reads the same 8 rows
      const uint64_t kd0 = smem_desc_sw128(sbase + kKOff, 16, 1024);
      const uint64_t vd0 = smem_desc_sw128(sbase + kVOff, kStageBytes / 2, 1024);
      const uint32_t s_tmem = tmem + kTmemS;
      const uint32_t p_tmem = tmem + kTmemP;
      bool ok = true;
      auto issue_pv = [&](int i) -> bool {
        const int pb = i & 1;
        const int vs = i % kVStages;
        if (!mbar_wait_lim<kPolls>(bar(P_FULL + pb), (i >> 1) & 1, abort_flag, wlim)) return false;
        if (!mbar_wait_lim<kPolls>(bar(V_FULL + vs), (i / kVStages) & 1, abort_flag, wlim)) return false;
        tc_fence_after();
        const uint64_t vd = vd0 + static_cast<uint64_t>(vs * (kStageBytes >> 4));
        const uint32_t pa = p_tmem + 32 * pb;
        mma_f16_ts(tmem, pa, vd, kIdescPV, i > 0 ? 1u : 0u);
#pragma unroll
        for (int kk = 1; kk < 4; ++kk) mma_f16_ts(tmem, pa + 8 * kk, vd + kk * (2048 >> 4), kIdescPV, 1u);
        mma_commit(bar(P_EMPTY + pb));
        mma_commit(bar(V_EMPTY + vs));
        return true;
      };
      int n = 0;
      ChunkWalk w(ip, p.idx_sk, j0, j1, p.block, T_valid);
      long long t0;
      int rows;
      for (int j = 0; ok && w.next(t0, rows); ++j, n = j) {
        const int ks = j % kKStages;
        if (!mbar_wait_lim<kPolls>(bar(K_FULL + ks), (j / kKStages) & 1, abort_flag, wlim)) { ok = false; break; }
        if (!mbar_wait_lim<kPolls>(bar(S_EMPTY), (j & 1) ^ 1, abort_flag, wlim)) { ok = false; break; }
        tc_fence_after();
        const uint64_t kd = kd0 + static_cast<uint64_t>(ks * (kStageBytes >> 4));
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const uint64_t qo = ((kk >> 2) * (kQBytes / 2) + (kk & 3) * 32) >> 4;
          const uint64_t ko = ((kk >> 2) * (kStageBytes / 2) + (kk & 3) * 32) >> 4;
          mma_f16_ss(s_tmem, qd + qo, kd + ko, kIdescQK, kk > 0 ? 1u : 0u);
        }
        mma_commit(bar(S_FULL + ks));
        if (j >= 1 && !issue_pv(j - 1)) { ok = false; break; }
      }
      if (ok && n >= 1) issue_pv(n - 1);
      // Whatever was issued must finish before TMEM is released.
      mma_commit(bar(MMA_DONE));
      mbar_wait_drain(bar(MMA_DONE), 0);
    }
  } else {
    // ---------------- softmax + partials (warp 0) ----------------
    const int row = lane;  // query head hk*g + row when row < g
    const uint32_t tl = tmem;  // lanes 0..31
    const float sl2 = p.scale_log2;
    float m_run = -INFINITY;
    float l_run = 0.f;
    bool ok = start_ok;
    ChunkWalk w(ip, p.idx_sk, j0, j1, p.block, T_valid);
    int n = 0;  // tiles taken
    long long t0;
    int nvalid;  // keys t0 .. t0 + nvalid - 1 lie before the sequence end
    for (int j = 0; ok && w.next(t0, nvalid); ++j) {
      n = j + 1;
      ok = mbar_wait_warp_lim<kPolls>(bar(S_FULL + j % kKStages), (j / kKStages) & 1, abort_flag, wlim);
      if (!ok) break;
      tc_fence_after();
      uint32_t sr0[32], sr1[32];
      tmem_ld32(tl + kTmemS, sr0);
      tmem_ld32(tl + kTmemS + 32, sr1);
      tmem_wait_ld();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar(S_EMPTY));
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
      float m8[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) m8[i] = x[i];
#pragma unroll
      for (int c = 8; c < 64; ++c) m8[c & 7] = fmaxf(m8[c & 7], x[c]);
      const float mx = fmaxf(fmaxf(fmaxf(m8[0], m8[1]), fmaxf(m8[2], m8[3])),
                             fmaxf(fmaxf(m8[4], m8[5]), fmaxf(m8[6], m8[7])));
      const float m_tile = mx * sl2;
      const bool rescale = m_tile > m_run + 8.0f;
      const float m_use = rescale ? m_tile : m_run;
      const float alpha = rescale ? ex2(m_run - m_use) : 1.0f;
      const float moff = (m_use == -INFINITY) ? 0.0f : m_use;
      float s8[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
      uint32_t pk[32];
#pragma unroll
      for (int c = 0; c < 64; c += 2) {
        const float p0 = ex2(fmaf(x[c], sl2, -moff));
        const float p1 = ex2(fmaf(x[c + 1], sl2, -moff));
        s8[(c >> 1) & 7] += p0 + p1;
        pk[c >> 1] = DT<T>::pack(p0, p1);
      }
      const float rs = ((s8[0] + s8[1]) + (s8[2] + s8[3])) + ((s8[4] + s8[5]) + (s8[6] + s8[7]));
      l_run = l_run * alpha + rs;
      m_run = m_use;
      // O must not change under a running P.V: rescale only after P.V(j-1).
      if (j >= 1 && __any_sync(0xffffffffu, rescale)) {
        const int pb1 = (j - 1) & 1;
        ok = mbar_wait_warp_lim<kPolls>(bar(P_EMPTY + pb1), ((j - 1) >> 1) & 1, abort_flag, wlim);
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
      // P buffer j&1 was last read by P.V(j-2).
      const int pb = j & 1;
      ok = mbar_wait_warp_lim<kPolls>(bar(P_EMPTY + pb), ((j >> 1) & 1) ^ 1, abort_flag, wlim);
      if (!ok) break;
      tc_fence_after();
      tmem_st32(tl + kTmemP + 32 * pb, pk);
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar(P_FULL + pb));
    }
    if (ok && n >= 1) {
      ok = mbar_wait_warp_lim<kPolls>(bar(P_EMPTY + ((n - 1) & 1)), ((n - 1) >> 1) & 1, abort_flag, wlim);
      tc_fence_after();
    }
    // After a timeout anywhere in the CTA the partial is incomplete: write nothing.
    if (ok && *abort_flag == 0) {
      const bool real = row < g;
      const long long slot = (static_cast<long long>(b) * p.Hq + (hk * g + row)) * p.splits + split;
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
        if (real) {
          // 16-byte stores when the caller's workspace allows them (it need
          // only be float-aligned), else 4-byte stores.
          float* dst = p.part_acc + slot * kD + ch * 32;
          if ((reinterpret_cast<uintptr_t>(dst) & 15u) == 0u) {
#pragma unroll
            for (int c = 0; c < 32; c += 4)
              *reinterpret_cast<uint4*>(dst + c) = make_uint4(ov[c], ov[c + 1], ov[c + 2], ov[c + 3]);
          } else {
#pragma unroll
            for (int c = 0; c < 32; ++c) dst[c] = __uint_as_float(ov[c]);
          }
        }
      }
      if (real) {
        p.part_ml[slot * 2] = m_run;
        p.part_ml[slot * 2 + 1] = l_run;
      }
    }
  }

  __syncthreads();
  if (warp == 2) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

}  // namespace gqa

// Launches decode_gqa_kernel and the combine kernel; p carries the split
// count and partial buffers chosen by the entry point.
template <typename K, typename... A>
static cudaError_t launch_pdl(dim3 grid, int threads, int smem, cudaStream_t s, K kernel, A... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(threads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, args...);
}

static int decode_gqa_launch(const Params& p, int dtype, cudaStream_t s) {
  CUtensorMap mk, mv;
  int st;
  if ((st = make_map_bhld(&mk, p.kc, dtype, p.B, p.Hkv, p.Tmax, kD, p.k_sb, p.k_sh, p.k_st, 64, "k_cache")) !=
      SABRE_OK)
    return st;
  if ((st = make_map_bhld(&mv, p.vc, dtype, p.B, p.Hkv, p.Tmax, kD, p.v_sb, p.v_sh, p.v_st, 64, "v_cache")) !=
      SABRE_OK)
    return st;
  dim3 grid(p.splits, p.Hkv, p.B);
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
  if (dtype == SABRE_BF16) {
    if ((st = ensure_smem_attr(gqa::decode_gqa_kernel<__nv_bfloat16>, gqa::kSmemBytes)) != SABRE_OK) return st;
    SABRE_CUDA_TRY(launch_pdl(grid, gqa::kThreads, gqa::kSmemBytes, s, gqa::decode_gqa_kernel<__nv_bfloat16>, mk, mv, p));
    SABRE_CUDA_TRY(cudaGetLastError());
    SABRE_CUDA_TRY(combine_wide(p.splits)
                       ? cudaLaunchKernelEx(&cfg, decode_combine_kernel<__nv_bfloat16, kCombineGroups, 16>, p)
                       : cudaLaunchKernelEx(&cfg, decode_combine_kernel<__nv_bfloat16, 1, 8>, p));
  } else {
    if ((st = ensure_smem_attr(gqa::decode_gqa_kernel<__half>, gqa::kSmemBytes)) != SABRE_OK) return st;
    SABRE_CUDA_TRY(launch_pdl(grid, gqa::kThreads, gqa::kSmemBytes, s, gqa::decode_gqa_kernel<__half>, mk, mv, p));
    SABRE_CUDA_TRY(cudaGetLastError());
    SABRE_CUDA_TRY(combine_wide(p.splits)
                       ? cudaLaunchKernelEx(&cfg, decode_combine_kernel<__half, kCombineGroups, 16>, p)
                       : cudaLaunchKernelEx(&cfg, decode_combine_kernel<__half, 1, 8>, p));
  }
  return SABRE_OK;
}

}  // namespace decode
}  // namespace sabre
