// Fused rotary embedding + KV store + per-block pooling (sm_100a).
//
// Replaces the reference wrapper's apply_rotary_pos_emb
// (methods/sabrecoder/sabrecoder_llama_triton.py:292-293) and its KV-cache
// update (:295-299) with one HBM pass over the projection outputs:
//   q_out = q*cos + rotate_half(q)*sin,  k_out = k*cos + rotate_half(k)*sin,
//   v_out = v,
// where rotate_half(x) = [-x[D/2:], x[:D/2]]. Each product and the sum are
// rounded to the storage dtype exactly as the reference's elementwise torch
// ops round them, so the result is bit-identical to apply_rotary_pos_emb.
// K/V rows are written at positions pos0.. of a [B, Hkv, T, D] cache. When
// pool pointers are given, the rotated Q and K are also averaged per block of
// `pool_block` rows for the pooled q.k top-k (rows summed first to last in
// fp32, then divided by the row count -- the same order sabre_pool_blocks
// uses).
//
// Layout: a CTA owns a block of rows (the pool block, or 64 rows) for 16
// heads; its 4 warps take 4 heads each, 8 lanes per head. Lane c of a head
// group holds d = [8c, 8c+8) and the rotation partners [64+8c, 64+8c+8) as
// two 16-byte vectors, so the four heads of a warp read one contiguous 1 KB
// span of a [B, L, H, D] row. Each lane walks its rows in order (which keeps
// the pooled sums in row order) with kU rows of loads in flight. cos/sin rows
// are staged once per 64-row chunk in shared memory and shared by all heads.
#include "common.cuh"

namespace sabre {
namespace rope {

constexpr int kD = 128;
constexpr int kWarps = 4;
constexpr int kHeadsPerWarp = 4;
constexpr int kHeadsPerCta = kWarps * kHeadsPerWarp;
constexpr int kChunk = 64;  // rows of cos/sin staged at a time
constexpr int kU = 6;       // rows of q/k/v loads in flight per lane (6 rather than 4: c4 layer 156 -> 150 us; 8 spills)

struct Params {
  const void* q;
  const void* k;
  const void* v;
  const void* cos;
  const void* sin;
  void* q_out;
  void* k_out;
  void* v_out;
  float* q_pool;
  float* k_pool;
  long long q_sb, q_sl, q_sh;
  long long k_sb, k_sl, k_sh;
  long long v_sb, v_sl, v_sh;
  long long c_sb, c_sl;
  long long qo_sb, qo_sl, qo_sh;
  long long ko_sb, ko_sh, ko_st;
  long long vo_sb, vo_sh, vo_st;
  int B, L, Hq, Hkv, rows, pos0, nb;
};

template <typename T>
__device__ __forceinline__ float rnd(float x) {
  return DT<T>::to_f(DT<T>::from_f(x));
}

// 8 packed 16-bit values <-> 8 floats.
template <typename T>
__device__ __forceinline__ void unpack8(const uint4& u, float (&f)[8]) {
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    if constexpr (DT<T>::kBf16) {
      f[2 * i] = __uint_as_float(w[i] << 16);
      f[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
    } else {
      const float2 t = __half22float2(*reinterpret_cast<const __half2*>(&w[i]));
      f[2 * i] = t.x;
      f[2 * i + 1] = t.y;
    }
  }
}

template <typename T>
__device__ __forceinline__ uint4 pack8(const float (&f)[8]) {
  return make_uint4(DT<T>::pack(f[0], f[1]), DT<T>::pack(f[2], f[3]), DT<T>::pack(f[4], f[5]),
                    DT<T>::pack(f[6], f[7]));
}

template <typename T>
__global__ void __launch_bounds__(kWarps * 32, 4) rope_qkv_kernel(const Params p) {
  __shared__ uint4 s_cos[kChunk][kD / 8];
  __shared__ uint4 s_sin[kChunk][kD / 8];
  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const int c = lane & 7;
  const int head = blockIdx.y * kHeadsPerCta + warp * kHeadsPerWarp + (lane >> 3);
  const int b = blockIdx.z;
  const int r0 = blockIdx.x * p.rows;
  const int r1 = min(r0 + p.rows, p.L);
  const int nheads = p.Hq + 2 * p.Hkv;
  const bool active = head < nheads;
  const int kind = head < p.Hq ? 0 : (head < p.Hq + p.Hkv ? 1 : 2);
  const int h = kind == 0 ? head : (kind == 1 ? head - p.Hq : head - p.Hq - p.Hkv);

  const T* src = nullptr;
  long long s_l = 0, d_row = 0, d_base = 0;
  T* dst = nullptr;
  float* pool = nullptr;
  if (active) {
    if (kind == 0) {
      src = static_cast<const T*>(p.q) + b * p.q_sb + h * p.q_sh;
      s_l = p.q_sl;
      dst = static_cast<T*>(p.q_out);
      d_base = b * p.qo_sb + h * p.qo_sh;
      d_row = p.qo_sl;
      if (p.q_pool) pool = p.q_pool + ((static_cast<long long>(b) * p.Hq + h) * p.nb) * kD;
    } else if (kind == 1) {
      src = static_cast<const T*>(p.k) + b * p.k_sb + h * p.k_sh;
      s_l = p.k_sl;
      dst = static_cast<T*>(p.k_out);
      d_base = b * p.ko_sb + h * p.ko_sh + static_cast<long long>(p.pos0) * p.ko_st;
      d_row = p.ko_st;
      if (p.k_pool) pool = p.k_pool + ((static_cast<long long>(b) * p.Hkv + h) * p.nb) * kD;
    } else {
      src = static_cast<const T*>(p.v) + b * p.v_sb + h * p.v_sh;
      s_l = p.v_sl;
      dst = static_cast<T*>(p.v_out);
      d_base = b * p.vo_sb + h * p.vo_sh + static_cast<long long>(p.pos0) * p.vo_st;
      d_row = p.vo_st;
    }
  }
  const T* cbase = static_cast<const T*>(p.cos) + b * p.c_sb;
  const T* sbase = static_cast<const T*>(p.sin) + b * p.c_sb;

  float acc_lo[8], acc_hi[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) acc_lo[i] = acc_hi[i] = 0.f;

  for (int cr0 = r0; cr0 < r1; cr0 += kChunk) {
    const int cr1 = min(cr0 + kChunk, r1);
    __syncthreads();  // previous chunk's cos/sin no longer read
    for (int i = tid; i < (cr1 - cr0) * (kD / 8); i += kWarps * 32) {
      const int rr = i >> 4, cc = i & 15;
      const long long off = static_cast<long long>(cr0 + rr) * p.c_sl + cc * 8;
      s_cos[rr][cc] = *reinterpret_cast<const uint4*>(cbase + off);
      s_sin[rr][cc] = *reinterpret_cast<const uint4*>(sbase + off);
    }
    __syncthreads();
    if (!active) continue;
    for (int rb = cr0; rb < cr1; rb += kU) {
      uint4 xl[kU], xh[kU];
#pragma unroll
      for (int u = 0; u < kU; ++u) {
        if (rb + u < cr1) {
          const T* xr = src + static_cast<long long>(rb + u) * s_l + 8 * c;
          xl[u] = *reinterpret_cast<const uint4*>(xr);
          xh[u] = *reinterpret_cast<const uint4*>(xr + 64);
        }
      }
#pragma unroll
      for (int u = 0; u < kU; ++u) {
        const int r = rb + u;
        if (r >= cr1) break;
        float a[8], bh[8], ol[8], oh[8];
        unpack8<T>(xl[u], a);
        unpack8<T>(xh[u], bh);
        if (kind == 2) {
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            ol[i] = a[i];
            oh[i] = bh[i];
          }
        } else {
          float cl[8], ch[8], sl[8], sh[8];
          unpack8<T>(s_cos[r - cr0][c], cl);
          unpack8<T>(s_cos[r - cr0][8 + c], ch);
          unpack8<T>(s_sin[r - cr0][c], sl);
          unpack8<T>(s_sin[r - cr0][8 + c], sh);
          // d < 64: x[d]*cos[d] + (-x[d+64])*sin[d]; d >= 64: x[d]*cos[d] + x[d-64]*sin[d]
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            ol[i] = rnd<T>(rnd<T>(a[i] * cl[i]) + rnd<T>(-bh[i] * sl[i]));
            oh[i] = rnd<T>(rnd<T>(bh[i] * ch[i]) + rnd<T>(a[i] * sh[i]));
          }
        }
        T* dr = dst + d_base + static_cast<long long>(r) * d_row + 8 * c;
        *reinterpret_cast<uint4*>(dr) = pack8<T>(ol);
        *reinterpret_cast<uint4*>(dr + 64) = pack8<T>(oh);
        if (pool) {
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            acc_lo[i] = __fadd_rn(acc_lo[i], ol[i]);
            acc_hi[i] = __fadd_rn(acc_hi[i], oh[i]);
          }
        }
      }
    }
  }
  if (pool) {
    const float n = static_cast<float>(r1 - r0);
    float* pr = pool + static_cast<long long>(blockIdx.x) * kD + 8 * c;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      pr[i] = __fdiv_rn(acc_lo[i], n);
      pr[64 + i] = __fdiv_rn(acc_hi[i], n);
    }
  }
}

}  // namespace rope
}  // namespace sabre

using namespace sabre;

extern "C" {

int sabre_rope_qkv(const void* q, const void* k, const void* v, const void* cos, const void* sin, void* q_out,
                   void* k_out, void* v_out, float* q_pool, float* k_pool, int batch, int seq_len, int heads_q,
                   int heads_kv, int head_dim, int pool_block, int pos0, int max_seq, const int64_t* q_strides,
                   const int64_t* k_strides, const int64_t* v_strides, const int64_t* cos_strides,
                   const int64_t* q_out_strides, const int64_t* k_out_strides, const int64_t* v_out_strides,
                   int dtype, void* stream) {
  using namespace sabre::rope;
  if (!q || !k || !v || !cos || !sin || !q_out || !k_out || !v_out || !q_strides || !k_strides || !v_strides ||
      !cos_strides || !q_out_strides || !k_out_strides || !v_out_strides)
    return sabre_fail(SABRE_ERR_INVALID_ARG, "sabre_rope_qkv: null pointer argument");
  if (batch <= 0 || seq_len <= 0 || heads_q <= 0 || heads_kv <= 0 || pos0 < 0)
    return sabre_fail(SABRE_ERR_INVALID_ARG, "sabre_rope_qkv: sizes must be positive");
  if (static_cast<long long>(pos0) + seq_len > static_cast<long long>(max_seq))
    return sabre_fail(SABRE_ERR_INVALID_ARG,
                      "sabre_rope_qkv: rows %d..%lld lie outside the cache of %d rows (k_out/v_out)", pos0,
                      static_cast<long long>(pos0) + seq_len - 1, max_seq);
  if (head_dim != kD) return sabre_fail(SABRE_ERR_UNSUPPORTED, "sabre_rope_qkv: head_dim %d (only 128)", head_dim);
  if (dtype != SABRE_BF16 && dtype != SABRE_F16)
    return sabre_fail(SABRE_ERR_INVALID_ARG, "sabre_rope_qkv: dtype %d", dtype);
  if ((q_pool || k_pool) && (pool_block <= 0 || pos0 != 0))
    return sabre_fail(SABRE_ERR_INVALID_ARG, "sabre_rope_qkv: pooling needs pool_block > 0 and pos0 == 0");
  const int64_t* all[7] = {q_strides, k_strides, v_strides, cos_strides, q_out_strides, k_out_strides,
                           v_out_strides};
  const int nst[7] = {3, 3, 3, 2, 3, 3, 3};
  for (int i = 0; i < 7; ++i)
    for (int j = 0; j < nst[i]; ++j)
      if (all[i][j] % 8 != 0)
        return sabre_fail(SABRE_ERR_ALIGNMENT, "sabre_rope_qkv: strides must be multiples of 8 elements (16-byte access)");
  const void* ptrs[8] = {q, k, v, cos, sin, q_out, k_out, v_out};
  for (int i = 0; i < 8; ++i)
    if ((reinterpret_cast<uintptr_t>(ptrs[i]) & 15u) != 0)
      return sabre_fail(SABRE_ERR_ALIGNMENT, "sabre_rope_qkv: pointers must be 16-byte aligned");
  Params p;
  p.q = q;
  p.k = k;
  p.v = v;
  p.cos = cos;
  p.sin = sin;
  p.q_out = q_out;
  p.k_out = k_out;
  p.v_out = v_out;
  p.q_pool = q_pool;
  p.k_pool = k_pool;
  p.q_sb = q_strides[0];
  p.q_sl = q_strides[1];
  p.q_sh = q_strides[2];
  p.k_sb = k_strides[0];
  p.k_sl = k_strides[1];
  p.k_sh = k_strides[2];
  p.v_sb = v_strides[0];
  p.v_sl = v_strides[1];
  p.v_sh = v_strides[2];
  p.c_sb = cos_strides[0];
  p.c_sl = cos_strides[1];
  p.qo_sb = q_out_strides[0];
  p.qo_sl = q_out_strides[1];
  p.qo_sh = q_out_strides[2];
  p.ko_sb = k_out_strides[0];
  p.ko_sh = k_out_strides[1];
  p.ko_st = k_out_strides[2];
  p.vo_sb = v_out_strides[0];
  p.vo_sh = v_out_strides[1];
  p.vo_st = v_out_strides[2];
  p.B = batch;
  p.L = seq_len;
  p.Hq = heads_q;
  p.Hkv = heads_kv;
  p.pos0 = pos0;
  p.rows = (q_pool || k_pool) ? pool_block : 64;
  p.nb = (seq_len + p.rows - 1) / p.rows;
  const int nheads = heads_q + 2 * heads_kv;
  dim3 grid(p.nb, (nheads + kHeadsPerCta - 1) / kHeadsPerCta, batch);
  if (grid.y > 65535u || grid.z > 65535u)
    return sabre_fail(SABRE_ERR_UNSUPPORTED, "sabre_rope_qkv: grid too large");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (dtype == SABRE_BF16)
    rope_qkv_kernel<__nv_bfloat16><<<grid, kWarps * 32, 0, s>>>(p);
  else
    rope_qkv_kernel<__half><<<grid, kWarps * 32, 0, s>>>(p);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return sabre_cuda_fail(e, "sabre_rope_qkv launch");
  return SABRE_OK;
}

}  // extern "C"
