// Block AttnRes depth mixer: one kernel for the RMS score, the depth softmax and
// the weighted value sum (replaces the two Triton kernels of
// aios/kernel/attnres.py:8-127).
//
// One warp owns one token row. Its lanes load every source row of that token
// once (bank sources, then the optional partial as the last source) with 128-bit
// loads, keep them in registers, reduce x.wq and x.x with warp shuffles, take
// the softmax over depth in fp32, round the weights to bf16 (the rounding point
// of aios/kernel/attnres.py:90-95) and write sum_s w_s x_s accumulated in fp32.
// The normalised bank and cat(bank, partial) never exist in memory: HBM traffic
// is exactly one read of each source row plus one write of the output row.
#include "abi_util.h"
#include "common.cuh"

namespace aiosb {
namespace {

constexpr int kMixWarps = 4;
constexpr int kMaxRegSources = 10;  // register-resident path: bank(<=9) + partial
constexpr int kMaxSources = 16;

// Score, depth softmax and weighted sum of one token whose NSRC source rows
// (bank sources, then the partial when present) are read through `rows`: lane l
// takes the 16-byte chunks l, l + 32, ... of every row, and wqr the same chunks
// of the weighted query. NSRC is known at compile time, so every loop is
// fixed-length and the 2 * NSRC warp reductions of the scores run interleaved
// instead of as NSRC dependent shuffle chains. rows(s, j) returns chunk
// lane + 32 j of source s; rows.between_phases() runs between the score pass and
// the weighted-sum pass.
template <int VPL, int NSRC, class Rows>
__device__ __forceinline__ void mix_token(const Rows& rows, const float (&wqr)[VPL][8], int nv, int hidden,
                                          float eps, int lane, uint4* __restrict__ out_row) {
  float score[NSRC];
  float mx = -INFINITY;
#pragma unroll
  for (int s = 0; s < NSRC; ++s) {
    float dot = 0.f, ss = 0.f;
#pragma unroll
    for (int j = 0; j < VPL; ++j) {
      const uint4 u = rows(s, j);
      const uint32_t p[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float a = bf16_lo(p[q]), b = bf16_hi(p[q]);
        dot += a * wqr[j][2 * q] + b * wqr[j][2 * q + 1];
        ss += a * a + b * b;
      }
    }
    dot = warp_sum(dot);
    ss = warp_sum(ss);
    score[s] = dot * (1.0f / sqrtf(ss / (float)hidden + eps));
    mx = fmaxf(mx, score[s]);
  }
  float denom = 0.f;
#pragma unroll
  for (int s = 0; s < NSRC; ++s) {
    score[s] = expf(score[s] - mx);
    denom += score[s];
  }
#pragma unroll
  for (int s = 0; s < NSRC; ++s) score[s] = round_bf16(score[s] / denom);
  rows.between_phases();
#pragma unroll
  for (int j = 0; j < VPL; ++j) {
    const int i = lane + j * 32;
    if (i < nv) {
      float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int s = 0; s < NSRC; ++s) {
        const uint4 u = rows(s, j);
        const uint32_t p[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          acc[2 * q] += score[s] * bf16_lo(p[q]);
          acc[2 * q + 1] += score[s] * bf16_hi(p[q]);
        }
      }
      out_row[i] = make_uint4(pack_bf16x2(acc[0], acc[1]), pack_bf16x2(acc[2], acc[3]),
                              pack_bf16x2(acc[4], acc[5]), pack_bf16x2(acc[6], acc[7]));
    }
  }
}

// Source rows already in registers. between_phases() marks them as rewritten,
// so the compiler converts them to fp32 again in the second pass instead of
// keeping 8 fp32 values per chunk live across the softmax (which spilled).
template <int VPL, int NSRC>
struct RegRows {
  uint4 (&x)[NSRC][VPL];
  __device__ __forceinline__ uint4 operator()(int s, int j) const { return x[s][j]; }
  __device__ __forceinline__ void between_phases() const {
#pragma unroll
    for (int s = 0; s < NSRC; ++s)
#pragma unroll
      for (int j = 0; j < VPL; ++j)
        asm volatile("" : "+r"(x[s][j].x), "+r"(x[s][j].y), "+r"(x[s][j].z), "+r"(x[s][j].w));
  }
};

// One warp per token, every source row loaded straight into registers. The
// weighted query, a model constant, is loaded before the wait on the producer.
template <int VPL, int NSRC>
__global__ void __launch_bounds__(kMixWarps * 32, 3)
    attnres_reg_kernel(const uint4* __restrict__ bank, int nsrc_bank, int64_t tokens, int hidden,
                       const uint4* __restrict__ partial, const float* __restrict__ wq, float eps,
                       uint4* __restrict__ out) {
  pdl_launch_dependents();
  const int64_t t = (int64_t)blockIdx.x * kMixWarps + threadIdx.x / 32;
  const int lane = threadIdx.x & 31;
  const int nv = hidden / 8;
  float wqr[VPL][8];
#pragma unroll
  for (int j = 0; j < VPL; ++j) {
    const int i = lane + j * 32;
#pragma unroll
    for (int e = 0; e < 8; ++e) wqr[j][e] = (i < nv) ? wq[i * 8 + e] : 0.f;
  }
  pdl_wait();
  if (t >= tokens) return;
  uint4 x[NSRC][VPL];
  // Issue every load first (maximum memory-level parallelism), then reduce.
#pragma unroll
  for (int s = 0; s < NSRC; ++s) {
    const uint4* src = (s < nsrc_bank) ? bank + ((int64_t)s * tokens + t) * nv : partial + t * nv;
#pragma unroll
    for (int j = 0; j < VPL; ++j) {
      const int i = lane + j * 32;
      x[s][j] = (i < nv) ? src[i] : make_uint4(0, 0, 0, 0);
    }
  }
  mix_token<VPL, NSRC>(RegRows<VPL, NSRC>{x}, wqr, nv, hidden, eps, lane, out + t * nv);
}

// Any hidden size / up to 16 sources: two passes over the sources (scores, then
// the weighted sum), still one warp per token.
__global__ void __launch_bounds__(kMixWarps * 32)
    attnres_generic_kernel(const uint4* __restrict__ bank, int nsrc_bank, int64_t tokens, int hidden,
                           const uint4* __restrict__ partial, const float* __restrict__ wq, float eps,
                           uint4* __restrict__ out) {
  pdl_enter();
  const int64_t t = (int64_t)blockIdx.x * kMixWarps + threadIdx.x / 32;
  const int lane = threadIdx.x & 31;
  if (t >= tokens) return;
  const int nv = hidden / 8;
  const int nsrc = nsrc_bank + (partial != nullptr ? 1 : 0);
  float score[kMaxSources];
  float mx = -INFINITY;
  for (int s = 0; s < nsrc; ++s) {
    const uint4* src = (s < nsrc_bank) ? bank + ((int64_t)s * tokens + t) * nv : partial + t * nv;
    float dot = 0.f, ss = 0.f;
    for (int i = lane; i < nv; i += 32) {
      const uint4 u = src[i];
      const uint32_t p[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float a = bf16_lo(p[q]), b = bf16_hi(p[q]);
        dot += a * wq[i * 8 + 2 * q] + b * wq[i * 8 + 2 * q + 1];
        ss += a * a + b * b;
      }
    }
    dot = warp_sum(dot);
    ss = warp_sum(ss);
    score[s] = dot * (1.0f / sqrtf(ss / (float)hidden + eps));
    mx = fmaxf(mx, score[s]);
  }
  float denom = 0.f;
  for (int s = 0; s < nsrc; ++s) {
    score[s] = expf(score[s] - mx);
    denom += score[s];
  }
  for (int s = 0; s < nsrc; ++s) score[s] = round_bf16(score[s] / denom);
  for (int i = lane; i < nv; i += 32) {
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    for (int s = 0; s < nsrc; ++s) {
      const uint4* src = (s < nsrc_bank) ? bank + ((int64_t)s * tokens + t) * nv : partial + t * nv;
      const uint4 u = src[i];
      const uint32_t p[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        acc[2 * q] += score[s] * bf16_lo(p[q]);
        acc[2 * q + 1] += score[s] * bf16_hi(p[q]);
      }
    }
    out[t * nv + i] = make_uint4(pack_bf16x2(acc[0], acc[1]), pack_bf16x2(acc[2], acc[3]),
                                 pack_bf16x2(acc[4], acc[5]), pack_bf16x2(acc[6], acc[7]));
  }
}

}  // namespace
}  // namespace aiosb

using namespace aiosb;

extern "C" int aiosb_attnres_mix(const void* bank, int64_t sources, int64_t tokens, int64_t hidden,
                                 const void* partial, const float* weighted_query, float eps, void* out,
                                 void* stream) {
  AIOSB_REQUIRE(sources >= 1 && tokens >= 1 && hidden >= 1, AIOSB_ERR_INVALID_ARG,
                "bank dimensions must be positive");
  const int64_t total = sources + (partial != nullptr ? 1 : 0);
  AIOSB_REQUIRE(total <= kMaxSources, AIOSB_ERR_UNSUPPORTED, "attnres_mix: at most %d sources", kMaxSources);
  AIOSB_REQUIRE(hidden % 8 == 0, AIOSB_ERR_UNSUPPORTED, "attnres_mix: hidden must be a multiple of 8");
  AIOSB_REQUIRE(bank && weighted_query && out, AIOSB_ERR_INVALID_ARG, "attnres_mix: null pointer");
  AIOSB_REQUIRE(aligned16(bank) && aligned16(out) && (partial == nullptr || aligned16(partial)),
                AIOSB_ERR_MISALIGNED, "attnres_mix: bank/partial/out must be 16-byte aligned");
  const dim3 grid((unsigned)((tokens + kMixWarps - 1) / kMixWarps));
  const int64_t nv = hidden / 8;
  cudaError_t e;
  if (total <= kMaxRegSources && nv <= 3 * 32) {
    auto kern = attnres_reg_kernel<3, 1>;
    switch (total) {
      case 1: kern = attnres_reg_kernel<3, 1>; break;
      case 2: kern = attnres_reg_kernel<3, 2>; break;
      case 3: kern = attnres_reg_kernel<3, 3>; break;
      case 4: kern = attnres_reg_kernel<3, 4>; break;
      case 5: kern = attnres_reg_kernel<3, 5>; break;
      case 6: kern = attnres_reg_kernel<3, 6>; break;
      case 7: kern = attnres_reg_kernel<3, 7>; break;
      case 8: kern = attnres_reg_kernel<3, 8>; break;
      case 9: kern = attnres_reg_kernel<3, 9>; break;
      default: kern = attnres_reg_kernel<3, 10>; break;
    }
    e = launch_pdl(kern, grid, dim3(kMixWarps * 32), 0, as_stream(stream), (const uint4*)bank, (int)sources, tokens,
                   (int)hidden, (const uint4*)partial, weighted_query, eps, (uint4*)out);
  } else {
    e = launch_pdl(attnres_generic_kernel, grid, dim3(kMixWarps * 32), 0, as_stream(stream), (const uint4*)bank,
                   (int)sources, tokens, (int)hidden, (const uint4*)partial, weighted_query, eps, (uint4*)out);
  }
  if (e != cudaSuccess) return set_error(AIOSB_ERR_LAUNCH, "attnres_mix: %s", cudaGetErrorString(e));
  return AIOSB_OK;
}
