// Decode-step q/k/v projection + rotary embedding + KV store in one kernel
// (sm_100a). Included by sabre_capi.cu after rope_cache.cu.
//
// Replaces, for one new token per sequence, the reference wrapper's
// q_proj/k_proj/v_proj calls, apply_rotary_pos_emb and the KV-cache update
// (methods/sabrecoder/sabrecoder_llama_triton.py:288-299): three matrix-vector
// products whose weights (132 MB per layer, 8.2 GB per token at 33B) dominate,
// followed by a rotation and a cache write that separately cost a launch and
// a round trip each. Here every CTA streams 32 weight rows of one head with
// coalesced 16-byte loads (a warp covers 512 contiguous bytes of a row per
// instruction) against the token's hidden state staged in shared memory,
// reduces in fp32, rounds each output to the storage dtype (as the Linear
// layer's output is rounded) and, for q and k, applies
//   rope(x)[d]      = x[d]*cos[d] - x[d+64]*sin[d]        (d < 64)
//   rope(x)[d + 64] = x[d+64]*cos[d+64] + x[d]*sin[d+64]
// with every product and sum rounded in the storage dtype, as in
// rope_cache.cu. The 32 rows of a CTA are the 16 rotation pairs
// (d, d + 64) for d in [d0, d0 + 16), so the rotation needs no exchange
// between CTAs. Grid: 4 CTAs per head of q, k and v.
namespace sabre {
namespace qkvd {

constexpr int kD = 128;
constexpr int kPairs = 16;      // rotation pairs per CTA (32 weight rows)
constexpr int kThreads = 256;   // 8 warps x 2 pairs
constexpr int kMaxBatch = 8;
constexpr int kMaxStageBytes = 160 * 1024;  // hidden state of all sequences in shared memory

struct Params {
  const void* x;                  // [B, hidden], row stride x_sb
  const void* wq;                 // [Hq*D, hidden] row-major, contiguous
  const void* wk;                 // [Hkv*D, hidden]
  const void* wv;                 // [Hkv*D, hidden]
  const void* cos;                // [B, D], row stride c_sb
  const void* sin;
  void* q_out;                    // [B, Hq, D] strides {qo_sb, qo_sh, 1}
  void* k_out;                    // [B, Hkv, T, D] strides {ko_sb, ko_sh, ko_st, 1}; row pos0
  void* v_out;
  long long x_sb, c_sb, qo_sb, qo_sh, ko_sb, ko_sh, ko_st, vo_sb, vo_sh, vo_st;
  int B, hidden, Hq, Hkv, pos0;
};

template <typename T>
__device__ __forceinline__ float rnd_q(float x) {
  return DT<T>::to_f(DT<T>::from_f(x));
}

template <typename T>
__device__ __forceinline__ void unpack8q(const uint4& u, float (&f)[8]) {
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    if constexpr (DT<T>::kBf16) {
      f[2 * i] = __uint_as_float(w[i] << 16);
      f[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
    } else {
      const float2 ff = __half22float2(*reinterpret_cast<const __half2*>(&w[i]));
      f[2 * i] = ff.x;
      f[2 * i + 1] = ff.y;
    }
  }
}

template <typename T>
__global__ void __launch_bounds__(kThreads, 2) qkv_rope_decode_kernel(const Params p) {
  extern __shared__ uint4 sx[];  // [B][hidden / 8]
  __shared__ float sy[kMaxBatch][2 * kPairs];
  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const int slot = blockIdx.x >> 2;
  const int d0 = (blockIdx.x & 3) * kPairs;
  int kind, head;
  const T* W;
  if (slot < p.Hq) {
    kind = 0;
    head = slot;
    W = static_cast<const T*>(p.wq);
  } else if (slot < p.Hq + p.Hkv) {
    kind = 1;
    head = slot - p.Hq;
    W = static_cast<const T*>(p.wk);
  } else {
    kind = 2;
    head = slot - p.Hq - p.Hkv;
    W = static_cast<const T*>(p.wv);
  }
  const int nch = p.hidden / 8;  // 16-byte chunks per row
  for (int i = tid; i < p.B * nch; i += kThreads) {
    const int b = i / nch;
    const int c = i - b * nch;
    sx[i] = *reinterpret_cast<const uint4*>(static_cast<const T*>(p.x) + b * p.x_sb + c * 8);
  }
  __syncthreads();

  // This warp's rows: pairs 2w and 2w+1, low and high halves.
  const T* wrow[4];
#pragma unroll
  for (int u = 0; u < 4; ++u) {
    const int pr = 2 * warp + (u & 1);
    const int d = (u < 2) ? d0 + pr : d0 + 64 + pr;
    wrow[u] = W + static_cast<long long>(head * kD + d) * p.hidden;
  }
  float acc[4][kMaxBatch];
#pragma unroll
  for (int u = 0; u < 4; ++u)
#pragma unroll
    for (int b = 0; b < kMaxBatch; ++b) acc[u][b] = 0.f;
#pragma unroll 4
  for (int c = lane; c < nch; c += 32) {
    float wf[4][8];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const uint4 wv = __ldg(reinterpret_cast<const uint4*>(wrow[u]) + c);
      unpack8q<T>(wv, wf[u]);
    }
#pragma unroll
    for (int b = 0; b < kMaxBatch; ++b) {
      if (b < p.B) {
        float xf[8];
        unpack8q<T>(sx[b * nch + c], xf);
#pragma unroll
        for (int u = 0; u < 4; ++u)
#pragma unroll
          for (int e = 0; e < 8; ++e) acc[u][b] = fmaf(wf[u][e], xf[e], acc[u][b]);
      }
    }
  }
#pragma unroll
  for (int u = 0; u < 4; ++u) {
#pragma unroll
    for (int b = 0; b < kMaxBatch; ++b) {
      if (b < p.B) {
        float v = acc[u][b];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
        if (lane == 0) sy[b][(u < 2 ? 0 : kPairs) + 2 * warp + (u & 1)] = v;
      }
    }
  }
  __syncthreads();

  if (tid < p.B * kPairs) {
    const int b = tid / kPairs;
    const int pr = tid - b * kPairs;
    const int d = d0 + pr;
    const float a = rnd_q<T>(sy[b][pr]);           // x[d] as the Linear layer stores it
    const float bh = rnd_q<T>(sy[b][kPairs + pr]);  // x[d + 64]
    float lo = a, hi = bh;
    if (kind != 2) {
      const T* cr = static_cast<const T*>(p.cos) + b * p.c_sb;
      const T* sr = static_cast<const T*>(p.sin) + b * p.c_sb;
      const float cl = DT<T>::to_f(cr[d]), ch = DT<T>::to_f(cr[d + 64]);
      const float sl = DT<T>::to_f(sr[d]), sh = DT<T>::to_f(sr[d + 64]);
      lo = rnd_q<T>(rnd_q<T>(a * cl) + rnd_q<T>(-bh * sl));
      hi = rnd_q<T>(rnd_q<T>(bh * ch) + rnd_q<T>(a * sh));
    }
    T* dst;
    if (kind == 0)
      dst = static_cast<T*>(p.q_out) + b * p.qo_sb + head * p.qo_sh;
    else if (kind == 1)
      dst = static_cast<T*>(p.k_out) + b * p.ko_sb + head * p.ko_sh + static_cast<long long>(p.pos0) * p.ko_st;
    else
      dst = static_cast<T*>(p.v_out) + b * p.vo_sb + head * p.vo_sh + static_cast<long long>(p.pos0) * p.vo_st;
    dst[d] = DT<T>::from_f(lo);
    dst[d + 64] = DT<T>::from_f(hi);
  }
}

}  // namespace qkvd
}  // namespace sabre

extern "C" {

int sabre_qkv_rope_decode(const void* x, const void* wq, const void* wk, const void* wv, const void* cos,
                          const void* sin, void* q_out, void* k_out, void* v_out, int batch, int hidden,
                          int heads_q, int heads_kv, int head_dim, int pos0, int max_seq, int64_t x_stride,
                          int64_t cos_stride, const int64_t* q_out_strides, const int64_t* k_out_strides,
                          const int64_t* v_out_strides, int dtype, void* stream) {
  using namespace sabre::qkvd;
  if (!x || !wq || !wk || !wv || !cos || !sin || !q_out || !k_out || !v_out || !q_out_strides || !k_out_strides ||
      !v_out_strides)
    return sabre_fail(SABRE_ERR_INVALID_ARG, "sabre_qkv_rope_decode: null pointer argument");
  if (batch <= 0 || hidden <= 0 || heads_q <= 0 || heads_kv <= 0 || max_seq <= 0)
    return sabre_fail(SABRE_ERR_INVALID_ARG, "sabre_qkv_rope_decode: sizes must be positive");
  if (pos0 < 0 || pos0 >= max_seq)
    return sabre_fail(SABRE_ERR_INVALID_ARG, "sabre_qkv_rope_decode: position %d outside the cache's %d rows", pos0,
                      max_seq);
  if (head_dim != kD)
    return sabre_fail(SABRE_ERR_UNSUPPORTED, "sabre_qkv_rope_decode: head_dim %d (only 128)", head_dim);
  if (dtype != SABRE_BF16 && dtype != SABRE_F16)
    return sabre_fail(SABRE_ERR_INVALID_ARG, "sabre_qkv_rope_decode: dtype %d", dtype);
  if (batch > kMaxBatch)
    return sabre_fail(SABRE_ERR_UNSUPPORTED, "sabre_qkv_rope_decode: batch %d > %d", batch, kMaxBatch);
  if (hidden % 8 != 0 || x_stride % 8 != 0)
    return sabre_fail(SABRE_ERR_ALIGNMENT, "sabre_qkv_rope_decode: hidden and x stride must be multiples of 8");
  const size_t stage = static_cast<size_t>(batch) * hidden * 2;
  if (stage > static_cast<size_t>(kMaxStageBytes))
    return sabre_fail(SABRE_ERR_UNSUPPORTED, "sabre_qkv_rope_decode: batch x hidden = %zu bytes > %d", stage,
                      kMaxStageBytes);
  const void* ptrs[4] = {x, wq, wk, wv};
  for (int i = 0; i < 4; ++i)
    if ((reinterpret_cast<uintptr_t>(ptrs[i]) & 15u) != 0)
      return sabre_fail(SABRE_ERR_ALIGNMENT, "sabre_qkv_rope_decode: x and weights must be 16-byte aligned");
  sabre::qkvd::Params p;
  p.x = x;
  p.wq = wq;
  p.wk = wk;
  p.wv = wv;
  p.cos = cos;
  p.sin = sin;
  p.q_out = q_out;
  p.k_out = k_out;
  p.v_out = v_out;
  p.x_sb = x_stride;
  p.c_sb = cos_stride;
  p.qo_sb = q_out_strides[0];
  p.qo_sh = q_out_strides[1];
  p.ko_sb = k_out_strides[0];
  p.ko_sh = k_out_strides[1];
  p.ko_st = k_out_strides[2];
  p.vo_sb = v_out_strides[0];
  p.vo_sh = v_out_strides[1];
  p.vo_st = v_out_strides[2];
  p.B = batch;
  p.hidden = hidden;
  p.Hq = heads_q;
  p.Hkv = heads_kv;
  p.pos0 = pos0;
  const long long nctas = 4ll * (heads_q + 2ll * heads_kv);
  if (nctas > 2147483647ll) return sabre_fail(SABRE_ERR_UNSUPPORTED, "sabre_qkv_rope_decode: too many heads");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaError_t e;
  if (dtype == SABRE_BF16) {
    e = cudaFuncSetAttribute(qkv_rope_decode_kernel<__nv_bfloat16>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             kMaxStageBytes);
    if (e != cudaSuccess) return sabre_cuda_fail(e, "cudaFuncSetAttribute(qkv_rope_decode)");
    qkv_rope_decode_kernel<__nv_bfloat16><<<static_cast<unsigned>(nctas), kThreads, stage, s>>>(p);
  } else {
    e = cudaFuncSetAttribute(qkv_rope_decode_kernel<__half>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             kMaxStageBytes);
    if (e != cudaSuccess) return sabre_cuda_fail(e, "cudaFuncSetAttribute(qkv_rope_decode)");
    qkv_rope_decode_kernel<__half><<<static_cast<unsigned>(nctas), kThreads, stage, s>>>(p);
  }
  e = cudaGetLastError();
  if (e != cudaSuccess) return sabre_cuda_fail(e, "sabre_qkv_rope_decode launch");
  return SABRE_OK;
}

}  // extern "C"
