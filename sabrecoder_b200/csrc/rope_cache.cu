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
// Layout: one warp owns one head for a block of rows and walks the rows in
// order; lane l handles d = {2l, 2l+1} and their rotation partners
// {2l+64, 2l+65}, so a warp reads and writes each 256-byte row as two
// 128-byte segments.
#include "common.cuh"

namespace sabre {
namespace rope {

constexpr int kD = 128;
constexpr int kWarps = 4;
constexpr int kUnroll = 4;

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
__device__ __forceinline__ float2 ld2(const T* p) {
  const uint32_t u = *reinterpret_cast<const uint32_t*>(p);
  if constexpr (DT<T>::kBf16) {
    return make_float2(__uint_as_float(u << 16), __uint_as_float(u & 0xffff0000u));
  } else {
    return __half22float2(*reinterpret_cast<const __half2*>(&u));
  }
}

template <typename T>
__device__ __forceinline__ float rnd(float x) {
  return DT<T>::to_f(DT<T>::from_f(x));
}

template <typename T>
__device__ __forceinline__ void st2(T* p, float a, float b) {
  *reinterpret_cast<uint32_t*>(p) = DT<T>::pack(a, b);
}

template <typename T>
__global__ void __launch_bounds__(kWarps * 32) rope_qkv_kernel(const Params p) {
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int head = blockIdx.y * kWarps + warp;  // 0..Hq+2*Hkv-1
  const int b = blockIdx.z;
  const int r0 = blockIdx.x * p.rows;
  const int r1 = min(r0 + p.rows, p.L);
  const int nheads = p.Hq + 2 * p.Hkv;
  if (head >= nheads || r0 >= p.L) return;
  const int kind = head < p.Hq ? 0 : (head < p.Hq + p.Hkv ? 1 : 2);
  const int h = kind == 0 ? head : (kind == 1 ? head - p.Hq : head - p.Hq - p.Hkv);
  const int d0 = 2 * lane;

  const T* src;
  long long s_l;
  T* dst;
  long long d_row, d_base;
  float* pool = nullptr;
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
  const T* cbase = static_cast<const T*>(p.cos) + b * p.c_sb;
  const T* sbase = static_cast<const T*>(p.sin) + b * p.c_sb;

  float acc[4] = {0.f, 0.f, 0.f, 0.f};
  for (int rb = r0; rb < r1; rb += kUnroll) {
    float2 xl[kUnroll], xh[kUnroll], cl[kUnroll], ch[kUnroll], sl[kUnroll], sh[kUnroll];
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      const int r = rb + u;
      if (r < r1) {
        const T* xr = src + static_cast<long long>(r) * s_l;
        xl[u] = ld2(xr + d0);
        xh[u] = ld2(xr + d0 + 64);
        if (kind != 2) {
          const T* cr = cbase + static_cast<long long>(r) * p.c_sl;
          const T* sr = sbase + static_cast<long long>(r) * p.c_sl;
          cl[u] = ld2(cr + d0);
          ch[u] = ld2(cr + d0 + 64);
          sl[u] = ld2(sr + d0);
          sh[u] = ld2(sr + d0 + 64);
        }
      }
    }
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      const int r = rb + u;
      if (r >= r1) break;
      float ol0, ol1, oh0, oh1;
      if (kind == 2) {
        ol0 = xl[u].x;
        ol1 = xl[u].y;
        oh0 = xh[u].x;
        oh1 = xh[u].y;
      } else {
        // d < 64: x[d]*cos[d] + (-x[d+64])*sin[d]; d >= 64: x[d]*cos[d] + x[d-64]*sin[d]
        ol0 = rnd<T>(rnd<T>(xl[u].x * cl[u].x) + rnd<T>(-xh[u].x * sl[u].x));
        ol1 = rnd<T>(rnd<T>(xl[u].y * cl[u].y) + rnd<T>(-xh[u].y * sl[u].y));
        oh0 = rnd<T>(rnd<T>(xh[u].x * ch[u].x) + rnd<T>(xl[u].x * sh[u].x));
        oh1 = rnd<T>(rnd<T>(xh[u].y * ch[u].y) + rnd<T>(xl[u].y * sh[u].y));
      }
      T* dr = dst + d_base + static_cast<long long>(r) * d_row;
      st2(dr + d0, ol0, ol1);
      st2(dr + d0 + 64, oh0, oh1);
      if (pool) {
        acc[0] = __fadd_rn(acc[0], ol0);
        acc[1] = __fadd_rn(acc[1], ol1);
        acc[2] = __fadd_rn(acc[2], oh0);
        acc[3] = __fadd_rn(acc[3], oh1);
      }
    }
  }
  if (pool) {
    const float n = static_cast<float>(r1 - r0);
    float* pr = pool + static_cast<long long>(blockIdx.x) * kD;
    pr[d0] = __fdiv_rn(acc[0], n);
    pr[d0 + 1] = __fdiv_rn(acc[1], n);
    pr[d0 + 64] = __fdiv_rn(acc[2], n);
    pr[d0 + 65] = __fdiv_rn(acc[3], n);
  }
}

}  // namespace rope
}  // namespace sabre

using namespace sabre;

extern "C" {

int sabre_rope_qkv(const void* q, const void* k, const void* v, const void* cos, const void* sin, void* q_out,
                   void* k_out, void* v_out, float* q_pool, float* k_pool, int batch, int seq_len, int heads_q,
                   int heads_kv, int head_dim, int pool_block, int pos0, const int64_t* q_strides,
                   const int64_t* k_strides, const int64_t* v_strides, const int64_t* cos_strides,
                   const int64_t* q_out_strides, const int64_t* k_out_strides, const int64_t* v_out_strides,
                   int dtype, void* stream) {
  using namespace sabre::rope;
  if (!q || !k || !v || !cos || !sin || !q_out || !k_out || !v_out || !q_strides || !k_strides || !v_strides ||
      !cos_strides || !q_out_strides || !k_out_strides || !v_out_strides)
    return sabre_fail(SABRE_ERR_INVALID_ARG, "sabre_rope_qkv: null pointer argument");
  if (batch <= 0 || seq_len <= 0 || heads_q <= 0 || heads_kv <= 0 || pos0 < 0)
    return sabre_fail(SABRE_ERR_INVALID_ARG, "sabre_rope_qkv: sizes must be positive");
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
      if (all[i][j] % 2 != 0)
        return sabre_fail(SABRE_ERR_ALIGNMENT, "sabre_rope_qkv: strides must be even (4-byte pair access)");
  const void* ptrs[8] = {q, k, v, cos, sin, q_out, k_out, v_out};
  for (int i = 0; i < 8; ++i)
    if ((reinterpret_cast<uintptr_t>(ptrs[i]) & 3u) != 0)
      return sabre_fail(SABRE_ERR_ALIGNMENT, "sabre_rope_qkv: pointers must be 4-byte aligned");
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
  dim3 grid(p.nb, (nheads + kWarps - 1) / kWarps, batch);
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
