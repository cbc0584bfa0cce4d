// C-ABI of libsabre_b200.so (declared in include/sabre_b200.h).
//
// One translation unit: the kernel sources are included here so that the
// device status word and all kernels live in a single module.
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>

#include "common.cuh"
#include "prefill_bsa.cu"
#include "decode_bsa.cu"
#include "block_mask.cu"
#include "rope_cache.cu"
#include "qkv_decode.cu"
#include "topk.cu"
#include "similarity.cu"
#include "token_mask.cu"

#define SABRE_VERSION 100

namespace sabre {

static int fail(int status, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_sabre_last_error, sizeof(g_sabre_last_error), fmt, ap);
  va_end(ap);
  return status;
}

static int cuda_fail(cudaError_t e, const char* what) { return sabre_cuda_fail(e, what); }

#define SABRE_CUDA_TRY(expr)                      \
  do {                                            \
    cudaError_t _e = (expr);                      \
    if (_e != cudaSuccess) return cuda_fail(_e, #expr); \
  } while (0)

static bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// ---------------------------------------------------------------------------
// TMA descriptor encoding through the driver entry point (no -lcuda needed).
// ---------------------------------------------------------------------------
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(ptr);
  });
  return fn;
}

// 4-D tiled map over a [B, H, L, D] tensor with element strides
// {sb, sh, sl, 1}, dims ordered (d, l, h, b); box = (64 d, box_rows l, 1, 1);
// 128-byte swizzle; out-of-range rows read as zero.
static int make_map_bhld(CUtensorMap* m, const void* base, int dtype, int B, int H, int L, int D, long long sb,
                         long long sh, long long sl, int box_rows, const char* name) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return fail(SABRE_ERR_CUDA, "cuTensorMapEncodeTiled entry point unavailable");
  const long long es = 2;
  // Size-1 dimensions may carry any stride; give them a valid one.
  if (H == 1) sh = sl * L;
  if (B == 1) sb = sh * H;
  const long long strides[3] = {sl * es, sh * es, sb * es};
  for (int i = 0; i < 3; ++i) {
    if (strides[i] <= 0 || (strides[i] % 16) != 0 || strides[i] >= (1ll << 40))
      return fail(SABRE_ERR_ALIGNMENT, "%s: stride %lld bytes is not a positive multiple of 16", name, strides[i]);
  }
  cuuint64_t gdim[4] = {(cuuint64_t)D, (cuuint64_t)L, (cuuint64_t)H, (cuuint64_t)B};
  cuuint64_t gstr[3] = {(cuuint64_t)strides[0], (cuuint64_t)strides[1], (cuuint64_t)strides[2]};
  cuuint32_t box[4] = {64u, (cuuint32_t)box_rows, 1u, 1u};
  cuuint32_t estr[4] = {1u, 1u, 1u, 1u};
  CUresult r = fn(m, dtype == SABRE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4,
                  const_cast<void*>(base), gdim, gstr, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(SABRE_ERR_CUDA, "%s: cuTensorMapEncodeTiled failed (%d)", name, (int)r);
  return SABRE_OK;
}

template <typename Kern>
static int ensure_smem_attr(Kern kern, int bytes) {
  // Per-device attribute; cheap enough to set on every call.
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(MaxDynamicSharedMemorySize)");
  return SABRE_OK;
}

}  // namespace sabre

#include "decode_gqa.cu"
#include "qkv_prefill.cu"

using namespace sabre;

extern "C" {

int sabre_version(void) { return SABRE_VERSION; }

const char* sabre_status_string(int status) {
  switch (status) {
    case SABRE_OK: return "ok";
    case SABRE_ERR_INVALID_ARG: return "invalid argument";
    case SABRE_ERR_UNSUPPORTED: return "unsupported shape";
    case SABRE_ERR_ALIGNMENT: return "alignment (16-byte TMA rule)";
    case SABRE_ERR_CUDA: return "CUDA error";
    case SABRE_ERR_WORKSPACE: return "workspace too small";
    default: return "unknown status";
  }
}

const char* sabre_last_error(void) { return g_sabre_last_error; }

int sabre_device_status(unsigned int* flags_out, int clear, void* stream) {
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  SABRE_CUDA_TRY(cudaStreamSynchronize(st));
  unsigned int v = 0;
  SABRE_CUDA_TRY(cudaMemcpyFromSymbol(&v, g_device_status, sizeof(v)));
  if (flags_out) *flags_out = v;
  if (clear) {
    const unsigned int z = 0;
    SABRE_CUDA_TRY(cudaMemcpyToSymbol(g_device_status, &z, sizeof(z)));
  }
  return SABRE_OK;
}

int sabre_set_wait_limit_ns(unsigned long long ns) {
  if (ns != 0 && (ns < 1000ull || ns > 60000000000ull))
    return fail(SABRE_ERR_INVALID_ARG, "sabre_set_wait_limit_ns: %llu ns outside [1 us, 60 s] (0 = default)", ns);
  const unsigned long long v = ns == 0 ? kWaitNs : ns;
  SABRE_CUDA_TRY(cudaMemcpyToSymbol(g_wait_limit_ns, &v, sizeof(v)));
  return SABRE_OK;
}

}  // extern "C"

namespace sabre {
// Shared by sabre_prefill_bsa and sabre_prefill_bsa_tokenmask (tmask != null).
static int prefill_launch(const void* q, const void* k, const void* v, void* o, const int32_t* block_indices,
                          const int32_t* block_counts, int batch, int heads_q, int heads_kv, int seq_len,
                          int head_dim, int block_size, int max_active, const int64_t* q_strides,
                          const int64_t* k_strides, const int64_t* v_strides, const int64_t* o_strides,
                          const int64_t* idx_strides, const int64_t* cnt_strides, float softmax_scale, int dtype,
                          const uint64_t* tmask, const int32_t* tmask_ptr, void* stream) {
  using namespace sabre::prefill;
  if (!q || !k || !v || !o || !block_indices || !block_counts || !q_strides || !k_strides || !v_strides ||
      !o_strides || !idx_strides || !cnt_strides)
    return fail(SABRE_ERR_INVALID_ARG, "sabre_prefill_bsa: null pointer argument");
  if (batch <= 0 || heads_q <= 0 || heads_kv <= 0 || seq_len <= 0 || max_active <= 0)
    return fail(SABRE_ERR_INVALID_ARG, "sabre_prefill_bsa: sizes must be positive");
  if (heads_q % heads_kv != 0)
    return fail(SABRE_ERR_INVALID_ARG, "sabre_prefill_bsa: heads_q (%d) not a multiple of heads_kv (%d)",
                heads_q, heads_kv);
  if (head_dim != kD) return fail(SABRE_ERR_UNSUPPORTED, "sabre_prefill_bsa: head_dim %d (only 128)", head_dim);
  if (block_size <= 0 || block_size % 64 != 0)
    return fail(SABRE_ERR_UNSUPPORTED, "sabre_prefill_bsa: block_size %d (must be a multiple of 64)", block_size);
  if (seq_len > kMaxKeyTiles * 64)
    return fail(SABRE_ERR_UNSUPPORTED, "sabre_prefill_bsa: seq_len %d > %d", seq_len, kMaxKeyTiles * 64);
  if (dtype != SABRE_BF16 && dtype != SABRE_F16)
    return fail(SABRE_ERR_INVALID_ARG, "sabre_prefill_bsa: dtype %d", dtype);
  if (q_strides[3] != 1 || k_strides[3] != 1 || v_strides[3] != 1 || o_strides[3] != 1)
    return fail(SABRE_ERR_UNSUPPORTED, "sabre_prefill_bsa: head_dim stride must be 1");
  if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(o))
    return fail(SABRE_ERR_ALIGNMENT, "sabre_prefill_bsa: q/k/v/o must be 16-byte aligned");
  for (int i = 0; i < 3; ++i)
    if ((o_strides[i] * 2) % 16 != 0)
      return fail(SABRE_ERR_ALIGNMENT, "sabre_prefill_bsa: o stride %d not a 16-byte multiple", i);

  CUtensorMap mq, mk, mv;
  int st;
  if ((st = make_map_bhld(&mq, q, dtype, batch, heads_q, seq_len, head_dim, q_strides[0], q_strides[1],
                          q_strides[2], kTileM, "q")) != SABRE_OK)
    return st;
  if ((st = make_map_bhld(&mk, k, dtype, batch, heads_kv, seq_len, head_dim, k_strides[0], k_strides[1],
                          k_strides[2], kTileN, "k")) != SABRE_OK)
    return st;
  if ((st = make_map_bhld(&mv, v, dtype, batch, heads_kv, seq_len, head_dim, v_strides[0], v_strides[1],
                          v_strides[2], kTileN, "v")) != SABRE_OK)
    return st;

  Params p;
  p.tmask = reinterpret_cast<const unsigned long long*>(tmask);
  p.tmask_ptr = tmask_ptr;
  p.o = o;
  p.o_sb = o_strides[0];
  p.o_sh = o_strides[1];
  p.o_sl = o_strides[2];
  p.idx = block_indices;
  p.cnt = block_counts;
  p.idx_sb = idx_strides[0];
  p.idx_sh = idx_strides[1];
  p.idx_sm = idx_strides[2];
  p.idx_sk = idx_strides[3];
  p.cnt_sb = cnt_strides[0];
  p.cnt_sh = cnt_strides[1];
  p.cnt_sm = cnt_strides[2];
  p.B = batch;
  p.Hq = heads_q;
  p.Hkv = heads_kv;
  p.L = seq_len;
  p.block = block_size;
  p.max_active = max_active;
  p.ntiles = (seq_len + kTileM - 1) / kTileM;
  p.nkt = (seq_len + 63) / 64;
  const float scale = softmax_scale > 0.f ? softmax_scale : 1.0f / sqrtf(static_cast<float>(head_dim));
  p.scale_log2 = scale * 1.4426950408889634f;

  // K/V of every head larger than this -> head-major CTA order (measured on
  // B200, 126 MB L2: c1's 101 MB runs 3.6 % faster row-major, c3's 268 MB
  // 1.7 % faster head-major, with DRAM reads 3.6x -> 1.0x the algorithmic).
  const long long kv_bytes = 2ll * batch * heads_kv * seq_len * head_dim * 2;
  p.head_major = kv_bytes > (112ll << 20) ? 1 : 0;
  if ((long long)batch * heads_q > 2147483647ll || (p.head_major && (long long)batch * heads_q > 65535ll) ||
      p.ntiles > 65535)
    return fail(SABRE_ERR_UNSUPPORTED, "sabre_prefill_bsa: grid too large");
  dim3 grid = p.head_major ? dim3(p.ntiles, batch * heads_q) : dim3(batch * heads_q, p.ntiles);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const bool tok = (tmask != nullptr);
  if (dtype == SABRE_BF16 && !tok) {
    if ((st = ensure_smem_attr(prefill_bsa_kernel<__nv_bfloat16, false>, kSmemBytes)) != SABRE_OK) return st;
    prefill_bsa_kernel<__nv_bfloat16, false><<<grid, kThreads, kSmemBytes, s>>>(mq, mk, mv, p);
  } else if (dtype == SABRE_BF16) {
    if ((st = ensure_smem_attr(prefill_bsa_kernel<__nv_bfloat16, true>, kSmemBytes)) != SABRE_OK) return st;
    prefill_bsa_kernel<__nv_bfloat16, true><<<grid, kThreads, kSmemBytes, s>>>(mq, mk, mv, p);
  } else if (!tok) {
    if ((st = ensure_smem_attr(prefill_bsa_kernel<__half, false>, kSmemBytes)) != SABRE_OK) return st;
    prefill_bsa_kernel<__half, false><<<grid, kThreads, kSmemBytes, s>>>(mq, mk, mv, p);
  } else {
    if ((st = ensure_smem_attr(prefill_bsa_kernel<__half, true>, kSmemBytes)) != SABRE_OK) return st;
    prefill_bsa_kernel<__half, true><<<grid, kThreads, kSmemBytes, s>>>(mq, mk, mv, p);
  }
  SABRE_CUDA_TRY(cudaGetLastError());
  return SABRE_OK;
}

}  // namespace sabre

extern "C" {

int sabre_prefill_bsa(const void* q, const void* k, const void* v, void* o, const int32_t* block_indices,
                      const int32_t* block_counts, int batch, int heads_q, int heads_kv, int seq_len,
                      int head_dim, int block_size, int max_active, const int64_t* q_strides,
                      const int64_t* k_strides, const int64_t* v_strides, const int64_t* o_strides,
                      const int64_t* idx_strides, const int64_t* cnt_strides, float softmax_scale, int dtype,
                      void* stream) {
  return sabre::prefill_launch(q, k, v, o, block_indices, block_counts, batch, heads_q, heads_kv, seq_len, head_dim,
                               block_size, max_active, q_strides, k_strides, v_strides, o_strides, idx_strides,
                               cnt_strides, softmax_scale, dtype, nullptr, nullptr, stream);
}

int sabre_prefill_bsa_tokenmask(const void* q, const void* k, const void* v, void* o, const int32_t* block_indices,
                                const int32_t* block_counts, const uint64_t* tile_masks,
                                const int32_t* tile_row_ptr, int batch, int heads_q, int heads_kv, int seq_len,
                                int head_dim, int max_active, const int64_t* q_strides, const int64_t* k_strides,
                                const int64_t* v_strides, const int64_t* o_strides, const int64_t* idx_strides,
                                const int64_t* cnt_strides, float softmax_scale, int dtype, void* stream) {
  if (!tile_masks || !tile_row_ptr)
    return sabre::fail(SABRE_ERR_INVALID_ARG, "sabre_prefill_bsa_tokenmask: null tile masks");
  return sabre::prefill_launch(q, k, v, o, block_indices, block_counts, batch, heads_q, heads_kv, seq_len, head_dim,
                               64, max_active, q_strides, k_strides, v_strides, o_strides, idx_strides, cnt_strides,
                               softmax_scale, dtype, tile_masks, tile_row_ptr, stream);
}

}  // extern "C"
