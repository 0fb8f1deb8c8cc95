// Memory-bound row kernels: KV scatter, RMSNorm, fused add+RMSNorm, SwiGLU and
// the embedding gather. One warp per row, 128-bit vector accesses when the row
// base and length allow it, fp32 math, bf16 storage.
#include <algorithm>

#include "abi_util.h"
#include "common.cuh"

namespace aiosb {
namespace {

constexpr int kRowThreads = 256;  // 8 warps, one row per warp

// ---- KV scatter (aios/kernel/store.py:8-29) ------------------------------
// One warp per token; k and v rows are `width` bf16 values.
__global__ void kv_store_kernel(__nv_bfloat16* __restrict__ k_cache, __nv_bfloat16* __restrict__ v_cache,
                                int64_t cache_stride, int64_t num_slots, const int32_t* __restrict__ indices,
                                int64_t num_tokens, const __nv_bfloat16* __restrict__ k, int64_t k_stride,
                                const __nv_bfloat16* __restrict__ v, int64_t v_stride, int64_t width, bool vec,
                                int32_t* status) {
  pdl_enter();
  const int64_t t = (int64_t)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  const int lane = threadIdx.x & 31;
  if (t >= num_tokens) return;
  const int64_t slot = indices[t];
  if (slot < 0 || slot >= num_slots) {
    if (lane == 0) report(status, AIOSB_DEV_SLOT_RANGE);
    return;
  }
  __nv_bfloat16* kd = k_cache + slot * cache_stride;
  __nv_bfloat16* vd = v_cache + slot * cache_stride;
  const __nv_bfloat16* ks = k + t * k_stride;
  const __nv_bfloat16* vs = v + t * v_stride;
  if (vec) {
    const int64_t nv = width / 8;
    for (int64_t i = lane; i < nv; i += 32) {
      reinterpret_cast<uint4*>(kd)[i] = reinterpret_cast<const uint4*>(ks)[i];
      reinterpret_cast<uint4*>(vd)[i] = reinterpret_cast<const uint4*>(vs)[i];
    }
  } else {
    for (int64_t i = lane; i < width; i += 32) {
      kd[i] = ks[i];
      vd[i] = vs[i];
    }
  }
}

// ---- RMSNorm (FlashInfer rmsnorm semantics, aios/layers/norm.py:10-22) ---
// x and out may alias (in-place norm): each lane reads its vectors before writing them.
__global__ void rmsnorm_kernel(const __nv_bfloat16* x, int64_t rows, int hidden, int64_t hpt, int64_t token_stride,
                               const __nv_bfloat16* __restrict__ w, float eps, __nv_bfloat16* out,
                               int64_t out_token_stride, bool vec) {
  pdl_enter();
  const int64_t r = (int64_t)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  const int lane = threadIdx.x & 31;
  if (r >= rows) return;
  const __nv_bfloat16* xr = x + (r / hpt) * token_stride + (r % hpt) * hidden;
  __nv_bfloat16* orow = out + (r / hpt) * out_token_stride + (r % hpt) * hidden;
  float ss = 0.f;
  if (vec) {
    const int nv = hidden / 8;
    for (int i = lane; i < nv; i += 32) {
      uint4 u = reinterpret_cast<const uint4*>(xr)[i];
      const uint32_t p[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        float a = bf16_lo(p[j]), b = bf16_hi(p[j]);
        ss += a * a + b * b;
      }
    }
  } else {
    for (int i = lane; i < hidden; i += 32) {
      float a = bf16_to_f(xr[i]);
      ss += a * a;
    }
  }
  ss = warp_sum(ss);
  const float rcp = 1.0f / sqrtf(ss / (float)hidden + eps);
  if (vec) {
    const int nv = hidden / 8;
    for (int i = lane; i < nv; i += 32) {
      uint4 u = reinterpret_cast<const uint4*>(xr)[i];
      uint4 wu = reinterpret_cast<const uint4*>(w)[i];
      const uint32_t p[4] = {u.x, u.y, u.z, u.w};
      const uint32_t q[4] = {wu.x, wu.y, wu.z, wu.w};
      uint32_t o[4];
#pragma unroll
      for (int j = 0; j < 4; ++j)
        o[j] = pack_bf16x2(bf16_lo(p[j]) * rcp * bf16_lo(q[j]), bf16_hi(p[j]) * rcp * bf16_hi(q[j]));
      reinterpret_cast<uint4*>(orow)[i] = make_uint4(o[0], o[1], o[2], o[3]);
    }
  } else {
    for (int i = lane; i < hidden; i += 32)
      orow[i] = f_to_bf16(bf16_to_f(xr[i]) * rcp * bf16_to_f(w[i]));
  }
}

// ---- fused add + RMSNorm (FlashInfer fused_add_rmsnorm semantics) --------
// residual = bf16(x + residual); x = bf16((x + residual)_fp32 * rcp * w).
// Rows up to 4096 elements keep the fp32 sum in registers (16 vectors/lane).
constexpr int kMaxVecPerLane = 16;
template <int VPL>
__global__ void add_rmsnorm_kernel(__nv_bfloat16* __restrict__ x, __nv_bfloat16* __restrict__ res, int64_t rows,
                                   int hidden, const __nv_bfloat16* __restrict__ w, float eps) {
  pdl_enter();
  const int64_t r = (int64_t)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  const int lane = threadIdx.x & 31;
  if (r >= rows) return;
  __nv_bfloat16* xr = x + r * hidden;
  __nv_bfloat16* rr = res + r * hidden;
  const int nv = hidden / 8;
  float s[VPL][8];
  float ss = 0.f;
#pragma unroll
  for (int it = 0; it < VPL; ++it) {
    const int i = lane + it * 32;
    if (i < nv) {
      uint4 a = reinterpret_cast<const uint4*>(xr)[i];
      uint4 b = reinterpret_cast<const uint4*>(rr)[i];
      const uint32_t pa[4] = {a.x, a.y, a.z, a.w}, pb[4] = {b.x, b.y, b.z, b.w};
      uint32_t o[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        float lo = bf16_lo(pa[j]) + bf16_lo(pb[j]);
        float hi = bf16_hi(pa[j]) + bf16_hi(pb[j]);
        s[it][2 * j] = lo;
        s[it][2 * j + 1] = hi;
        ss += lo * lo + hi * hi;
        o[j] = pack_bf16x2(lo, hi);
      }
      reinterpret_cast<uint4*>(rr)[i] = make_uint4(o[0], o[1], o[2], o[3]);
    }
  }
  ss = warp_sum(ss);
  const float rcp = 1.0f / sqrtf(ss / (float)hidden + eps);
#pragma unroll
  for (int it = 0; it < VPL; ++it) {
    const int i = lane + it * 32;
    if (i < nv) {
      uint4 wu = reinterpret_cast<const uint4*>(w)[i];
      const uint32_t q[4] = {wu.x, wu.y, wu.z, wu.w};
      uint32_t o[4];
#pragma unroll
      for (int j = 0; j < 4; ++j)
        o[j] = pack_bf16x2(s[it][2 * j] * rcp * bf16_lo(q[j]), s[it][2 * j + 1] * rcp * bf16_hi(q[j]));
      reinterpret_cast<uint4*>(xr)[i] = make_uint4(o[0], o[1], o[2], o[3]);
    }
  }
}

// ---- SwiGLU (FlashInfer silu_and_mul semantics) ---------------------------
__device__ __forceinline__ float silu_f(float g) { return g / (1.0f + expf(-g)); }

__global__ void silu_mul_kernel(const __nv_bfloat16* __restrict__ x, int64_t rows, int64_t f,
                                __nv_bfloat16* __restrict__ out) {
  pdl_enter();
  const int64_t nvec = f / 8;
  const int64_t total = rows * nvec;
  for (int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; idx < total;
       idx += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = idx / nvec, c = idx % nvec;
    uint4 g = reinterpret_cast<const uint4*>(x + r * 2 * f)[c];
    uint4 u = reinterpret_cast<const uint4*>(x + r * 2 * f + f)[c];
    const uint32_t pg[4] = {g.x, g.y, g.z, g.w}, pu[4] = {u.x, u.y, u.z, u.w};
    uint32_t o[4];
#pragma unroll
    for (int j = 0; j < 4; ++j)
      o[j] = pack_bf16x2(silu_f(bf16_lo(pg[j])) * bf16_lo(pu[j]), silu_f(bf16_hi(pg[j])) * bf16_hi(pu[j]));
    reinterpret_cast<uint4*>(out + r * f)[c] = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

// ---- Embedding gather (aios/layers/embedding.py:17-18) --------------------
// One warp per token. With stat_x, also writes the row in fp32 and its sum of
// squares (stat_ss[t], a single part): the statistics a following
// aiosb_linear_stat_norm normalises from.
__global__ void embedding_kernel(const void* __restrict__ ids, bool ids64, int64_t n, const uint4* __restrict__ w,
                                 int64_t vocab, int64_t hidden, uint4* __restrict__ out, float* __restrict__ stat_x,
                                 float* __restrict__ stat_ss, int32_t* status) {
  pdl_enter();
  const int64_t t = (int64_t)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  const int lane = threadIdx.x & 31;
  if (t >= n) return;
  const int64_t id = ids64 ? reinterpret_cast<const int64_t*>(ids)[t] : reinterpret_cast<const int32_t*>(ids)[t];
  const int64_t nv = hidden / 8;
  const bool ok = id >= 0 && id < vocab;
  if (!ok && lane == 0) report(status, AIOSB_DEV_TOKEN_RANGE);
  float ss = 0.f;
  for (int64_t i = lane; i < nv; i += 32) {
    const uint4 v = ok ? w[id * nv + i] : make_uint4(0, 0, 0, 0);
    out[t * nv + i] = v;
    if (stat_x != nullptr) {
      const float f[8] = {bf16_lo(v.x), bf16_hi(v.x), bf16_lo(v.y), bf16_hi(v.y),
                          bf16_lo(v.z), bf16_hi(v.z), bf16_lo(v.w), bf16_hi(v.w)};
      float4* dst = reinterpret_cast<float4*>(stat_x + t * hidden + 8 * i);
      dst[0] = make_float4(f[0], f[1], f[2], f[3]);
      dst[1] = make_float4(f[4], f[5], f[6], f[7]);
#pragma unroll
      for (int j = 0; j < 8; ++j) ss += f[j] * f[j];
    }
  }
  if (stat_x != nullptr) {
    ss = warp_sum(ss);
    if (lane == 0) stat_ss[t] = ss;
  }
}

inline unsigned row_blocks(int64_t rows) { return (unsigned)((rows + kRowThreads / 32 - 1) / (kRowThreads / 32)); }

}  // namespace
}  // namespace aiosb

using namespace aiosb;

extern "C" int aiosb_kv_store(void* k_cache, void* v_cache, int64_t cache_token_stride, int64_t num_slots,
                              const int32_t* indices, int64_t num_tokens, const void* k, int64_t k_token_stride,
                              const void* v, int64_t v_token_stride, int64_t width, int32_t* status,
                              void* stream) {
  AIOSB_REQUIRE(num_tokens >= 0 && width > 0 && num_slots > 0, AIOSB_ERR_INVALID_ARG,
                "kv_store: bad sizes (tokens=%lld width=%lld slots=%lld)", (long long)num_tokens,
                (long long)width, (long long)num_slots);
  AIOSB_REQUIRE(cache_token_stride >= width && k_token_stride >= width && v_token_stride >= width,
                AIOSB_ERR_INVALID_ARG, "kv_store: token strides must cover the row width");
  if (num_tokens == 0) return AIOSB_OK;
  AIOSB_REQUIRE(k_cache && v_cache && indices && k && v, AIOSB_ERR_INVALID_ARG, "kv_store: null pointer");
  const bool vec = width % 8 == 0 && cache_token_stride % 8 == 0 && k_token_stride % 8 == 0 &&
                   v_token_stride % 8 == 0 && aligned16(k_cache) && aligned16(v_cache) && aligned16(k) &&
                   aligned16(v);
  cudaError_t e = launch_pdl(kv_store_kernel, dim3(row_blocks(num_tokens)), dim3(kRowThreads), 0, as_stream(stream),
                             (__nv_bfloat16*)k_cache, (__nv_bfloat16*)v_cache, cache_token_stride, num_slots, indices,
                             num_tokens, (const __nv_bfloat16*)k, k_token_stride, (const __nv_bfloat16*)v,
                             v_token_stride, width, vec, status);
  if (e != cudaSuccess) return set_error(AIOSB_ERR_LAUNCH, "kv_store: %s", cudaGetErrorString(e));
  return AIOSB_OK;
}

extern "C" int aiosb_rmsnorm(const void* x, int64_t rows, int64_t hidden, int64_t heads_per_token,
                             int64_t token_stride, const void* weight, float eps, void* out,
                             int64_t out_token_stride, void* stream) {
  AIOSB_REQUIRE(rows >= 0 && hidden > 0 && hidden <= 65536 && heads_per_token > 0, AIOSB_ERR_INVALID_ARG,
                "rmsnorm: bad sizes");
  AIOSB_REQUIRE(token_stride >= heads_per_token * hidden && out_token_stride >= heads_per_token * hidden,
                AIOSB_ERR_INVALID_ARG, "rmsnorm: token stride smaller than heads*hidden");
  if (rows == 0) return AIOSB_OK;
  AIOSB_REQUIRE(x && weight && out, AIOSB_ERR_INVALID_ARG, "rmsnorm: null pointer");
  const bool vec = hidden % 8 == 0 && token_stride % 8 == 0 && out_token_stride % 8 == 0 && aligned16(x) &&
                   aligned16(out) && aligned16(weight);
  cudaError_t e = launch_pdl(rmsnorm_kernel, dim3(row_blocks(rows)), dim3(kRowThreads), 0, as_stream(stream),
                             (const __nv_bfloat16*)x, rows, (int)hidden, heads_per_token, token_stride,
                             (const __nv_bfloat16*)weight, eps, (__nv_bfloat16*)out, out_token_stride, vec);
  if (e != cudaSuccess) return set_error(AIOSB_ERR_LAUNCH, "rmsnorm: %s", cudaGetErrorString(e));
  return AIOSB_OK;
}

extern "C" int aiosb_add_rmsnorm(void* x, void* residual, int64_t rows, int64_t hidden, const void* weight,
                                 float eps, void* stream) {
  AIOSB_REQUIRE(rows >= 0 && hidden > 0, AIOSB_ERR_INVALID_ARG, "add_rmsnorm: bad sizes");
  AIOSB_REQUIRE(hidden % 8 == 0 && hidden <= 8 * 32 * kMaxVecPerLane, AIOSB_ERR_UNSUPPORTED,
                "add_rmsnorm: hidden must be a multiple of 8 and <= %d", 8 * 32 * kMaxVecPerLane);
  if (rows == 0) return AIOSB_OK;
  AIOSB_REQUIRE(x && residual && weight, AIOSB_ERR_INVALID_ARG, "add_rmsnorm: null pointer");
  AIOSB_REQUIRE(aligned16(x) && aligned16(residual) && aligned16(weight), AIOSB_ERR_MISALIGNED,
                "add_rmsnorm: pointers must be 16-byte aligned");
  auto kern = hidden <= 1024 ? add_rmsnorm_kernel<4> : hidden <= 2048 ? add_rmsnorm_kernel<8> : add_rmsnorm_kernel<16>;
  cudaError_t e = launch_pdl(kern, dim3(row_blocks(rows)), dim3(kRowThreads), 0, as_stream(stream),
                             (__nv_bfloat16*)x, (__nv_bfloat16*)residual, rows, (int)hidden,
                             (const __nv_bfloat16*)weight, eps);
  if (e != cudaSuccess) return set_error(AIOSB_ERR_LAUNCH, "add_rmsnorm: %s", cudaGetErrorString(e));
  return AIOSB_OK;
}

extern "C" int aiosb_silu_mul(const void* x, int64_t rows, int64_t f, void* out, void* stream) {
  AIOSB_REQUIRE(rows >= 0 && f > 0, AIOSB_ERR_INVALID_ARG, "silu_mul: bad sizes");
  AIOSB_REQUIRE(f % 8 == 0, AIOSB_ERR_UNSUPPORTED, "silu_mul: width must be a multiple of 8");
  if (rows == 0) return AIOSB_OK;
  AIOSB_REQUIRE(x && out, AIOSB_ERR_INVALID_ARG, "silu_mul: null pointer");
  AIOSB_REQUIRE(aligned16(x) && aligned16(out), AIOSB_ERR_MISALIGNED, "silu_mul: pointers must be 16-byte aligned");
  const int64_t total = rows * (f / 8);
  const unsigned blocks = (unsigned)std::min<int64_t>((total + 255) / 256, (int64_t)sm_count() * 8);
  cudaError_t e = launch_pdl(silu_mul_kernel, dim3(blocks), dim3(256), 0, as_stream(stream), (const __nv_bfloat16*)x,
                             rows, f, (__nv_bfloat16*)out);
  if (e != cudaSuccess) return set_error(AIOSB_ERR_LAUNCH, "silu_mul: %s", cudaGetErrorString(e));
  return AIOSB_OK;
}

extern "C" int aiosb_embedding(const void* ids, int ids_is_int64, int64_t num_tokens, const void* weight,
                               int64_t vocab, int64_t hidden, void* out, int32_t* status, void* stream) {
  AIOSB_REQUIRE(num_tokens >= 0 && vocab > 0 && hidden > 0, AIOSB_ERR_INVALID_ARG, "embedding: bad sizes");
  AIOSB_REQUIRE(hidden % 8 == 0, AIOSB_ERR_UNSUPPORTED, "embedding: hidden must be a multiple of 8");
  if (num_tokens == 0) return AIOSB_OK;
  AIOSB_REQUIRE(ids && weight && out, AIOSB_ERR_INVALID_ARG, "embedding: null pointer");
  AIOSB_REQUIRE(aligned16(weight) && aligned16(out), AIOSB_ERR_MISALIGNED,
                "embedding: weight/out must be 16-byte aligned");
  cudaError_t e = launch_pdl(embedding_kernel, dim3(row_blocks(num_tokens)), dim3(kRowThreads), 0,
                             as_stream(stream), ids, ids_is_int64 != 0, num_tokens, (const uint4*)weight, vocab,
                             hidden, (uint4*)out, (float*)nullptr, (float*)nullptr, status);
  if (e != cudaSuccess) return set_error(AIOSB_ERR_LAUNCH, "embedding: %s", cudaGetErrorString(e));
  return AIOSB_OK;
}

extern "C" int aiosb_embedding_stat(const void* ids, int ids_is_int64, int64_t num_tokens, const void* weight,
                                    int64_t vocab, int64_t hidden, void* out, float* stat_x, float* stat_ss,
                                    int32_t* status, void* stream) {
  AIOSB_REQUIRE(num_tokens >= 0 && vocab > 0 && hidden > 0, AIOSB_ERR_INVALID_ARG, "embedding_stat: bad sizes");
  AIOSB_REQUIRE(hidden % 8 == 0, AIOSB_ERR_UNSUPPORTED, "embedding_stat: hidden must be a multiple of 8");
  if (num_tokens == 0) return AIOSB_OK;
  AIOSB_REQUIRE(ids && weight && out && stat_x && stat_ss, AIOSB_ERR_INVALID_ARG, "embedding_stat: null pointer");
  AIOSB_REQUIRE(aligned16(weight) && aligned16(out) && aligned16(stat_x), AIOSB_ERR_MISALIGNED,
                "embedding_stat: weight/out/stat_x must be 16-byte aligned");
  cudaError_t e = launch_pdl(embedding_kernel, dim3(row_blocks(num_tokens)), dim3(kRowThreads), 0,
                             as_stream(stream), ids, ids_is_int64 != 0, num_tokens, (const uint4*)weight, vocab,
                             hidden, (uint4*)out, stat_x, stat_ss, status);
  if (e != cudaSuccess) return set_error(AIOSB_ERR_LAUNCH, "embedding_stat: %s", cudaGetErrorString(e));
  return AIOSB_OK;
}
