// Fused prefill q/k/v projection + rotary embedding + KV store + pooling
// (sm_100a).
//
// Replaces, for a prompt of L tokens, the reference wrapper's three
// projections, apply_rotary_pos_emb and KV-cache update
// (methods/sabrecoder/sabrecoder_llama_triton.py:288-299) with one kernel:
// Y = X W^T for the concatenated bias-free weights W = [Wq; Wk; Wv]
// ([(Hq + 2 Hkv) * 128, hidden]), each output rounded to the storage dtype as
// the Linear layer's output is, then in the epilogue the rotation of the q and
// k heads with the per-operation rounding of rope_cache.cu (bit-identical to
// apply_rotary_pos_emb on Y), q written to [B, L, Hq, D], rotated k and v
// written straight into the [B, Hkv, T, D] cache at rows pos0.., and the
// per-block means of the rotated q and k for the pooled top-k (rows summed
// first to last in fp32, then divided by the row count). Y itself never
// touches HBM.
//
// GEMM: one CTA per 256 x 256 output tile (a tile's 256 columns are two
// heads), K in steps of 64. Warp 0 loads X (256 x 64) and W (256 x 64) tiles
// with TMA (128-byte swizzle, no multicast) into a 3-stage ring of 64 KB;
// warp 1 allocates all 512 TMEM columns and issues, per step, 4 x 2
// tcgen05.mma M=128 N=256 K=16 (rows 0-127 into columns 0-255, rows 128-255
// into 256-511; both read the same W tile), releasing the stage with a
// commit. Both operands are K-major in shared memory. Per byte of operand
// the tile does as much work as a 2-SM 256 x 256 tile.
// Epilogue: warps 2-9 (two per TMEM lane quadrant; thread = output row, one
// half of each head's columns) read a head's columns d and d + 64 as pairs of
// 32, round them to the storage type two per word and rotate with packed
// single-rounding 16-bit ops; 16-byte stores. For pooling each thread parks
// its rotated values in shared memory (the idle ring) and then sums one
// (head, column) down the rows of each pool block in order.
// All waits are bounded (common.cuh); a timeout drains what was issued, frees
// TMEM and stores nothing.
#include "common.cuh"

namespace sabre {
namespace qkvp {

constexpr int kD = 128;
constexpr int kBM = 256;
constexpr int kBN = 256;
constexpr int kBK = 64;
constexpr int kStages = 3;
constexpr int kABytes = kBM * kBK * 2;  // 32768
constexpr int kBBytes = kBN * kBK * 2;  // 32768
constexpr int kStageBytes = kABytes + kBBytes;
constexpr int kThreads = 320;  // warp 0 TMA, warp 1 MMA, warps 2-9 epilogue
constexpr int kEpiThreads = 256;
constexpr int kBarOff = kStages * kStageBytes;
enum Bar { FULL = 0, EMPTY = kStages, ACC_FULL = 2 * kStages, NUM_BARS = 2 * kStages + 1 };
constexpr int kMiscOff = kBarOff + NUM_BARS * 8;
constexpr int kSmemBytes = kMiscOff + 16;
constexpr uint32_t kTmemCols = 512;
constexpr int kPoolPitch = kD + 1;  // floats per parked row (conflict-free columns)
static_assert(2 * 128 * kPoolPitch * 4 <= kBarOff, "two heads of parked rows fit in the idle ring");

// Packed 16-bit pairs in a 32-bit word: each op rounds once to the type.
template <typename T>
__device__ __forceinline__ uint32_t v2_mul(uint32_t a, uint32_t b) {
  uint32_t d;
  if constexpr (DT<T>::kBf16)
    asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  else
    asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}
template <typename T>
__device__ __forceinline__ uint32_t v2_add(uint32_t a, uint32_t b) {
  uint32_t d;
  if constexpr (DT<T>::kBf16)
    asm("add.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  else
    asm("add.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}
template <typename T>
__device__ __forceinline__ uint32_t v2_neg(uint32_t a) {
  return a ^ 0x80008000u;  // flips both sign bits (exact)
}
template <typename T>
__device__ __forceinline__ float v2_lo(uint32_t w) {
  if constexpr (DT<T>::kBf16) return __uint_as_float(w << 16);
  else return __half2float(__ushort_as_half(static_cast<unsigned short>(w & 0xffffu)));
}
template <typename T>
__device__ __forceinline__ float v2_hi(uint32_t w) {
  if constexpr (DT<T>::kBf16) return __uint_as_float(w & 0xffff0000u);
  else return __half2float(__ushort_as_half(static_cast<unsigned short>(w >> 16)));
}

struct Params {
  const void* cos;
  const void* sin;
  long long c_sb, c_sl;
  void* q_out;
  long long qo_sb, qo_sl, qo_sh;
  void* k_out;
  long long ko_sb, ko_sh, ko_st;
  void* v_out;
  long long vo_sb, vo_sh, vo_st;
  float* q_pool;  // [B, Hq, nbp, D] or null
  float* k_pool;  // [B, Hkv, nbp, D] or null
  void* y_out;    // [M, N] projection (row stride y_sm) or null
  long long y_sm;
  int M, N, K, L, Hq, Hkv, pos0, pool_block, nbp;
};

template <typename T>
__global__ void __launch_bounds__(kThreads, 1)
    qkv_proj_rope_kernel(const __grid_constant__ CUtensorMap tmX, const __grid_constant__ CUtensorMap tmW,
                         const Params p) {
  extern __shared__ __align__(1024) uint8_t smem[];
  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const uint32_t sbase = smem_u32(smem);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + kMiscOff);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + kMiscOff + 4);
  auto bar = [&](int i) -> uint32_t { return sbase + kBarOff + 8u * i; };
  const int n0 = blockIdx.x * kBN;
  const int m0 = blockIdx.y * kBM;
  const int nk = (p.K + kBK - 1) / kBK;

  if (tid == 0) {
    const bool bad = (sbase & 1023u) != 0u;
    *abort_flag = bad ? 1 : 0;
    if (bad) record_status(SABRE_DEV_BAD_SMEM_ALIGN);
    for (int s = 0; s < kStages; ++s) {
      mbar_init(bar(FULL + s), 1);
      mbar_init(bar(EMPTY + s), 1);
    }
    mbar_init(bar(ACC_FULL), 1);
    fence_mbar_init();
    tma_prefetch_desc(&tmX);
    tma_prefetch_desc(&tmW);
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), kTmemCols);
    tmem_relinquish();
  }
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const bool start_ok = (*abort_flag == 0);

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0 && start_ok) {
      int issued[kStages] = {0, 0, 0};
      for (int ks = 0; ks < nk; ++ks) {
        const int s = ks % kStages;
        if (!mbar_wait(bar(EMPTY + s), ((ks / kStages) & 1) ^ 1, abort_flag)) break;
        mbar_arrive_expect_tx(bar(FULL + s), kStageBytes);
        const uint32_t dst = sbase + s * kStageBytes;
        tma_load_2d(dst, &tmX, bar(FULL + s), ks * kBK, m0);
        tma_load_2d(dst + kABytes, &tmW, bar(FULL + s), ks * kBK, n0);
        ++issued[s];
      }
      for (int s = 0; s < kStages; ++s)
        if (issued[s] > 0) mbar_wait_drain(bar(FULL + s), (issued[s] - 1) & 1);
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0 && start_ok) {
      constexpr uint32_t kIdesc = idesc_f16(128, 256, DT<T>::kBf16, false);
      for (int ks = 0; ks < nk; ++ks) {
        const int s = ks % kStages;
        if (!mbar_wait(bar(FULL + s), (ks / kStages) & 1, abort_flag)) break;
        tc_fence_after();
        const uint32_t st = sbase + s * kStageBytes;
        const uint64_t a0 = smem_desc_sw128(st, 16, 1024);
        const uint64_t a1 = smem_desc_sw128(st + kABytes / 2, 16, 1024);
        const uint64_t bd = smem_desc_sw128(st + kABytes, 16, 1024);
#pragma unroll
        for (int kk = 0; kk < kBK / 16; ++kk) {
          const uint32_t acc = (ks > 0 || kk > 0) ? 1u : 0u;
          const uint64_t ko = static_cast<uint64_t>((kk * 32) >> 4);
          mma_f16_ss(tmem, a0 + ko, bd + ko, kIdesc, acc);
          mma_f16_ss(tmem + 256, a1 + ko, bd + ko, kIdesc, acc);
        }
        mma_commit(bar(EMPTY + s));
      }
      // Also after a timeout: whatever was issued must finish before TMEM is freed.
      mma_commit(bar(ACC_FULL));
      mbar_wait_drain(bar(ACC_FULL), 0);
    }
  } else {
    // ---------------- epilogue (warps 2-9) ----------------
    // Warp w reads TMEM lane quadrant w % 4 (its 32 rows of each
    // accumulator); warps 2-5 take columns d in [0, 32) of every head and
    // their partners d + 64, warps 6-9 take [32, 64) and d + 64.
    const int quad = warp & 3;
    const int c2 = (warp - 2) >> 2;
    const int rloc = quad * 32 + lane;  // row within an accumulator
    const int et = (warp - 2) * 32 + lane;  // 0 .. 255
    const uint32_t tl = tmem + (static_cast<uint32_t>(quad * 32) << 16);
    const bool waited = start_ok && mbar_wait_warp(bar(ACC_FULL), 0, abort_flag);
    tc_fence_after();
    // One decision for all eight warps (the pooling below meets at named
    // barriers, so they must all take the same path): after every warp's
    // wait, one thread reads the abort flag and publishes what it saw.
    volatile int* go = reinterpret_cast<volatile int*>(smem + kMiscOff + 8);
    if (!waited && lane == 0) *abort_flag = 1;
    named_bar_sync(1, kEpiThreads);
    if (et == 0) *go = (*abort_flag == 0) ? 1 : 0;
    named_bar_sync(1, kEpiThreads);
    const bool ok = *go != 0;
    const int nheads = p.Hq + 2 * p.Hkv;
    float* park = reinterpret_cast<float*>(smem);  // [2 heads][128 rows][kPoolPitch]
    for (int a = 0; ok && a < 2; ++a) {
      const int m = m0 + a * 128 + rloc;
      const bool valid = m < p.M;
      const int b = valid ? m / p.L : 0;
      const int l = valid ? m - b * p.L : 0;
      const int d = 32 * c2;
      // cos/sin of this row, columns d .. d+31 and d+64 .. d+95, as pairs
      uint32_t cl[16], ch[16], sl[16], sh[16];
      if (valid) {
        const T* crow = static_cast<const T*>(p.cos) + b * p.c_sb + static_cast<long long>(l) * p.c_sl + d;
        const T* srow = static_cast<const T*>(p.sin) + b * p.c_sb + static_cast<long long>(l) * p.c_sl + d;
#pragma unroll
        for (int v4 = 0; v4 < 4; ++v4) {
          const uint4 c0 = *reinterpret_cast<const uint4*>(crow + 8 * v4);
          const uint4 c1 = *reinterpret_cast<const uint4*>(crow + 64 + 8 * v4);
          const uint4 s0 = *reinterpret_cast<const uint4*>(srow + 8 * v4);
          const uint4 s1 = *reinterpret_cast<const uint4*>(srow + 64 + 8 * v4);
          cl[4 * v4] = c0.x; cl[4 * v4 + 1] = c0.y; cl[4 * v4 + 2] = c0.z; cl[4 * v4 + 3] = c0.w;
          ch[4 * v4] = c1.x; ch[4 * v4 + 1] = c1.y; ch[4 * v4 + 2] = c1.z; ch[4 * v4 + 3] = c1.w;
          sl[4 * v4] = s0.x; sl[4 * v4 + 1] = s0.y; sl[4 * v4 + 2] = s0.z; sl[4 * v4 + 3] = s0.w;
          sh[4 * v4] = s1.x; sh[4 * v4 + 1] = s1.y; sh[4 * v4 + 2] = s1.z; sh[4 * v4 + 3] = s1.w;
        }
      }
      bool pooled_any = false;
#pragma unroll 1
      for (int hh = 0; hh < 2; ++hh) {
        const int hd = (n0 >> 7) + hh;  // uniform over the CTA
        if (hd >= nheads) continue;
        const int kind = hd < p.Hq ? 0 : (hd < p.Hq + p.Hkv ? 1 : 2);
        const int h = kind == 0 ? hd : (kind == 1 ? hd - p.Hq : hd - p.Hq - p.Hkv);
        const bool pool = (kind == 0 ? p.q_pool : (kind == 1 ? p.k_pool : nullptr)) != nullptr;
        pooled_any = pooled_any || pool;
        const uint32_t col = static_cast<uint32_t>(a * 256 + hh * 128 + d);
        uint32_t lo[32], hi[32];
        tmem_ld32(tl + col, lo);
        tmem_ld32(tl + col + 64, hi);
        tmem_wait_ld();
        if (!valid) continue;
        T* drow = nullptr;
        if (kind == 0)
          drow = static_cast<T*>(p.q_out) + b * p.qo_sb + static_cast<long long>(l) * p.qo_sl + h * p.qo_sh;
        else if (kind == 1)
          drow = static_cast<T*>(p.k_out) + b * p.ko_sb + h * p.ko_sh + static_cast<long long>(p.pos0 + l) * p.ko_st;
        else
          drow = static_cast<T*>(p.v_out) + b * p.vo_sb + h * p.vo_sh + static_cast<long long>(p.pos0 + l) * p.vo_st;
        // y rounded to the storage type, two columns per word
        uint32_t yl[16], yh[16], ol[16], oh[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          yl[j] = DT<T>::pack(__uint_as_float(lo[2 * j]), __uint_as_float(lo[2 * j + 1]));
          yh[j] = DT<T>::pack(__uint_as_float(hi[2 * j]), __uint_as_float(hi[2 * j + 1]));
        }
        if (p.y_out) {
          T* yr = static_cast<T*>(p.y_out) + static_cast<long long>(m) * p.y_sm + (n0 + hh * 128) + d;
#pragma unroll
          for (int v4 = 0; v4 < 4; ++v4) {
            *reinterpret_cast<uint4*>(yr + 8 * v4) = make_uint4(yl[4 * v4], yl[4 * v4 + 1], yl[4 * v4 + 2], yl[4 * v4 + 3]);
            *reinterpret_cast<uint4*>(yr + 64 + 8 * v4) =
                make_uint4(yh[4 * v4], yh[4 * v4 + 1], yh[4 * v4 + 2], yh[4 * v4 + 3]);
          }
        }
        if (kind == 2) {
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            ol[j] = yl[j];
            oh[j] = yh[j];
          }
        } else {
          // d < 64: y[d] cos[d] + (-y[d+64]) sin[d]; d >= 64: y[d] cos[d] + y[d-64] sin[d], every product
          // and sum rounded to the storage type (single-rounding packed ops; the same bits as rounding
          // each fp32 result, since products and sums of two 16-bit values are exact in fp32).
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            ol[j] = v2_add<T>(v2_mul<T>(yl[j], cl[j]), v2_mul<T>(v2_neg<T>(yh[j]), sl[j]));
            oh[j] = v2_add<T>(v2_mul<T>(yh[j], ch[j]), v2_mul<T>(yl[j], sh[j]));
          }
        }
#pragma unroll
        for (int v4 = 0; v4 < 4; ++v4) {
          *reinterpret_cast<uint4*>(drow + d + 8 * v4) = make_uint4(ol[4 * v4], ol[4 * v4 + 1], ol[4 * v4 + 2], ol[4 * v4 + 3]);
          *reinterpret_cast<uint4*>(drow + d + 64 + 8 * v4) =
              make_uint4(oh[4 * v4], oh[4 * v4 + 1], oh[4 * v4 + 2], oh[4 * v4 + 3]);
        }
        if (pool) {
          float* prow = park + (hh * 128 + rloc) * kPoolPitch + d;
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            prow[2 * j] = v2_lo<T>(ol[j]);
            prow[2 * j + 1] = v2_hi<T>(ol[j]);
            prow[64 + 2 * j] = v2_lo<T>(oh[j]);
            prow[64 + 2 * j + 1] = v2_hi<T>(oh[j]);
          }
        }
      }
      if (!pooled_any) continue;
      // Block means of the parked rows: thread et sums column et % 128 of
      // head et / 128 down the rows, first to last (two independent chains
      // for two blocks of 64). Accumulator a holds rows l0 .. l0+127 of one
      // sequence (pooling runs only where tiles do not straddle sequences).
      named_bar_sync(1, kEpiThreads);
      const int mrow0 = m0 + a * 128;
      const int hh = et >> 7;
      const int colx = et & 127;
      const int hd = (n0 >> 7) + hh;
      if (mrow0 < p.M && hd < p.Hq + p.Hkv) {
        const bool isq = hd < p.Hq;
        float* dstp = isq ? p.q_pool : p.k_pool;
        if (dstp) {
          const int bs = mrow0 / p.L;
          const int l0 = mrow0 - bs * p.L;
          const int h = isq ? hd : hd - p.Hq;
          const int H = isq ? p.Hq : p.Hkv;
          const float* cp = park + hh * 128 * kPoolPitch + colx;
          const int nrows = min(128, p.L - l0);
          const int pb = p.pool_block;
          const int n0b = min(pb, nrows);                   // rows of the first block
          const int n1b = pb == 64 ? max(0, nrows - 64) : 0;  // rows of the second (64-row blocks)
          float acc0 = 0.f, acc1 = 0.f;
          for (int r = 0; r < 64; r += 8) {
            float v0[8], v1[8];
#pragma unroll
            for (int u = 0; u < 8; ++u) {
              v0[u] = cp[(r + u) * kPoolPitch];
              v1[u] = cp[(64 + r + u) * kPoolPitch];
            }
#pragma unroll
            for (int u = 0; u < 8; ++u) {
              if (pb == 64) {
                if (r + u < n0b) acc0 = __fadd_rn(acc0, v0[u]);
                if (r + u < n1b) acc1 = __fadd_rn(acc1, v1[u]);
              } else {
                if (r + u < n0b) acc0 = __fadd_rn(acc0, v0[u]);
              }
            }
          }
          if (pb == 128) {  // rows 64 .. 127 continue the one chain, in order
            for (int r = 64; r < 128; r += 8) {
              float v0[8];
#pragma unroll
              for (int u = 0; u < 8; ++u) v0[u] = cp[(r + u) * kPoolPitch];
#pragma unroll
              for (int u = 0; u < 8; ++u)
                if (r + u < n0b) acc0 = __fadd_rn(acc0, v0[u]);
            }
          }
          float* base = dstp + (static_cast<long long>(bs) * H + h) * p.nbp * kD + colx;
          const int j0 = l0 / pb;
          base[static_cast<long long>(j0) * kD] = __fdiv_rn(acc0, static_cast<float>(n0b));
          if (n1b > 0) base[static_cast<long long>(j0 + 1) * kD] = __fdiv_rn(acc1, static_cast<float>(n1b));
        }
      }
      named_bar_sync(1, kEpiThreads);  // the parked rows are reused by the next accumulator
    }
  }

  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

}  // namespace qkvp
}  // namespace sabre

namespace sabre {
namespace qkvp {

// 2-D tiled map over a row-major [rows, cols] matrix (row stride in
// elements), box = (64 cols, box_rows rows), 128-byte swizzle; rows and
// columns past the end read as zero.
static int make_map_2d(CUtensorMap* m, const void* base, int dtype, long long rows, long long cols,
                       long long row_stride, int box_rows, const char* name) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return fail(SABRE_ERR_CUDA, "cuTensorMapEncodeTiled entry point unavailable");
  cuuint64_t gdim[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t gstr[1] = {(cuuint64_t)(row_stride * 2)};
  cuuint32_t box[2] = {64u, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1u, 1u};
  CUresult r = fn(m, dtype == SABRE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2,
                  const_cast<void*>(base), gdim, gstr, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(SABRE_ERR_CUDA, "%s: cuTensorMapEncodeTiled failed (%d)", name, (int)r);
  return SABRE_OK;
}

}  // namespace qkvp
}  // namespace sabre

extern "C" {

int sabre_qkv_proj_rope(const void* x, const void* w, const void* cos, const void* sin, void* q_out, void* k_out,
                        void* v_out, float* q_pool, float* k_pool, void* y_out, int batch, int seq_len, int hidden,
                        int heads_q, int heads_kv, int head_dim, int pool_block, int pos0, int max_seq,
                        int64_t x_stride, const int64_t* cos_strides, const int64_t* q_out_strides,
                        const int64_t* k_out_strides, const int64_t* v_out_strides, int64_t y_stride, int dtype,
                        void* stream) {
  using namespace sabre::qkvp;
  if (!x || !w || !cos || !sin || !q_out || !k_out || !v_out || !cos_strides || !q_out_strides || !k_out_strides ||
      !v_out_strides)
    return sabre::fail(SABRE_ERR_INVALID_ARG, "sabre_qkv_proj_rope: null pointer argument");
  if (batch <= 0 || seq_len <= 0 || hidden <= 0 || heads_q <= 0 || heads_kv <= 0 || pos0 < 0)
    return sabre::fail(SABRE_ERR_INVALID_ARG, "sabre_qkv_proj_rope: sizes must be positive");
  if (head_dim != kD) return sabre::fail(SABRE_ERR_UNSUPPORTED, "sabre_qkv_proj_rope: head_dim %d (only 128)", head_dim);
  if (dtype != SABRE_BF16 && dtype != SABRE_F16)
    return sabre::fail(SABRE_ERR_INVALID_ARG, "sabre_qkv_proj_rope: dtype %d", dtype);
  if (static_cast<long long>(pos0) + seq_len > static_cast<long long>(max_seq))
    return sabre::fail(SABRE_ERR_INVALID_ARG, "sabre_qkv_proj_rope: rows %d..%lld lie outside the cache of %d rows",
                       pos0, static_cast<long long>(pos0) + seq_len - 1, max_seq);
  if (hidden % 8 != 0 || x_stride < hidden || x_stride % 8 != 0)
    return sabre::fail(SABRE_ERR_ALIGNMENT, "sabre_qkv_proj_rope: hidden and x_stride must be multiples of 8 "
                                            "(16-byte TMA rows), x_stride >= hidden");
  const bool pooling = (q_pool != nullptr) || (k_pool != nullptr);
  if (pooling && ((pool_block != 64 && pool_block != 128) || pos0 != 0 || (batch > 1 && seq_len % kBM != 0)))
    return sabre::fail(SABRE_ERR_UNSUPPORTED,
                       "sabre_qkv_proj_rope: pooling needs pool_block 64 or 128, pos0 == 0 and one sequence or "
                       "seq_len a multiple of %d", kBM);
  const long long N = static_cast<long long>(heads_q + 2 * heads_kv) * kD;
  const long long M = static_cast<long long>(batch) * seq_len;
  if (y_out && (y_stride < N || y_stride % 8 != 0))
    return sabre::fail(SABRE_ERR_ALIGNMENT, "sabre_qkv_proj_rope: y_stride must be >= %lld and a multiple of 8", N);
  const int64_t* all[4] = {cos_strides, q_out_strides, k_out_strides, v_out_strides};
  const int nst[4] = {2, 3, 3, 3};
  for (int i = 0; i < 4; ++i)
    for (int j = 0; j < nst[i]; ++j)
      if (all[i][j] % 8 != 0)
        return sabre::fail(SABRE_ERR_ALIGNMENT, "sabre_qkv_proj_rope: strides must be multiples of 8 elements");
  const void* ptrs[8] = {x, w, cos, sin, q_out, k_out, v_out, y_out};
  for (int i = 0; i < 8; ++i)
    if ((reinterpret_cast<uintptr_t>(ptrs[i]) & 15u) != 0)
      return sabre::fail(SABRE_ERR_ALIGNMENT, "sabre_qkv_proj_rope: pointers must be 16-byte aligned");
  if ((M + kBM - 1) / kBM > 65535)
    return sabre::fail(SABRE_ERR_UNSUPPORTED, "sabre_qkv_proj_rope: batch * seq_len too large");

  CUtensorMap mx, mw;
  int st;
  if ((st = make_map_2d(&mx, x, dtype, M, hidden, x_stride, kBM, "x")) != SABRE_OK) return st;
  if ((st = make_map_2d(&mw, w, dtype, N, hidden, hidden, kBN, "w")) != SABRE_OK) return st;
  Params p;
  p.cos = cos;
  p.sin = sin;
  p.c_sb = cos_strides[0];
  p.c_sl = cos_strides[1];
  p.q_out = q_out;
  p.qo_sb = q_out_strides[0];
  p.qo_sl = q_out_strides[1];
  p.qo_sh = q_out_strides[2];
  p.k_out = k_out;
  p.ko_sb = k_out_strides[0];
  p.ko_sh = k_out_strides[1];
  p.ko_st = k_out_strides[2];
  p.v_out = v_out;
  p.vo_sb = v_out_strides[0];
  p.vo_sh = v_out_strides[1];
  p.vo_st = v_out_strides[2];
  p.q_pool = q_pool;
  p.k_pool = k_pool;
  p.y_out = y_out;
  p.y_sm = y_stride;
  p.M = static_cast<int>(M);
  p.N = static_cast<int>(N);
  p.K = hidden;
  p.L = seq_len;
  p.Hq = heads_q;
  p.Hkv = heads_kv;
  p.pos0 = pos0;
  p.pool_block = pooling ? pool_block : 64;
  p.nbp = (seq_len + p.pool_block - 1) / p.pool_block;
  dim3 grid(static_cast<unsigned>((N + kBN - 1) / kBN), static_cast<unsigned>((M + kBM - 1) / kBM));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (dtype == SABRE_BF16) {
    if ((st = sabre::ensure_smem_attr(qkv_proj_rope_kernel<__nv_bfloat16>, kSmemBytes)) != SABRE_OK) return st;
    qkv_proj_rope_kernel<__nv_bfloat16><<<grid, kThreads, kSmemBytes, s>>>(mx, mw, p);
  } else {
    if ((st = sabre::ensure_smem_attr(qkv_proj_rope_kernel<__half>, kSmemBytes)) != SABRE_OK) return st;
    qkv_proj_rope_kernel<__half><<<grid, kThreads, kSmemBytes, s>>>(mx, mw, p);
  }
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return sabre_cuda_fail(e, "sabre_qkv_proj_rope launch");
  return SABRE_OK;
}

}  // extern "C"
