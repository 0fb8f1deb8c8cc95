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
#include <algorithm>
#include <cstdlib>

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
// NORM: the output row is written RMS-normalised, bf16(h * rcp * nw) with h the
// bf16 mixer output and rcp = 1 / sqrt(mean(h^2) + norm_eps) (RMSNorm.forward,
// aios/layers/norm.py:10-22, applied to the mixer result); nwr holds this lane's
// chunks of the norm weight.
template <int VPL, int NSRC, bool NORM = false, class Rows>
__device__ __forceinline__ void mix_token(const Rows& rows, const float2 (&wqr)[VPL][4], int nv, int hidden,
                                          float eps, int lane, uint4* __restrict__ out_row,
                                          const uint4 (*nwr)[VPL] = nullptr, float norm_eps = 0.f) {
  float score[NSRC];
  float mx = -INFINITY;
#pragma unroll
  for (int s = 0; s < NSRC; ++s) {
    // even and odd elements accumulate in the two halves of packed fp32 FMAs
    float2 dot2 = make_float2(0.f, 0.f), ss2 = make_float2(0.f, 0.f);
#pragma unroll
    for (int j = 0; j < VPL; ++j) {
      const uint4 u = rows(s, j);
      const uint32_t p[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float2 v = make_float2(bf16_lo(p[q]), bf16_hi(p[q]));
        dot2 = __ffma2_rn(v, wqr[j][q], dot2);
        ss2 = __ffma2_rn(v, v, ss2);
      }
    }
    const float dot = warp_sum(dot2.x + dot2.y);
    const float ss = warp_sum(ss2.x + ss2.y);
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
  uint4 hbuf[VPL];  // NORM: the bf16 mixer output, normalised once the row is complete
#pragma unroll
  for (int j = 0; j < VPL; ++j) {
    const int i = lane + j * 32;
    hbuf[j] = make_uint4(0u, 0u, 0u, 0u);
    if (i < nv) {
      float2 acc[4] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
#pragma unroll
      for (int s = 0; s < NSRC; ++s) {
        const uint4 u = rows(s, j);
        const uint32_t p[4] = {u.x, u.y, u.z, u.w};
        const float2 w2 = make_float2(score[s], score[s]);
#pragma unroll
        for (int q = 0; q < 4; ++q) acc[q] = __ffma2_rn(w2, make_float2(bf16_lo(p[q]), bf16_hi(p[q])), acc[q]);
      }
      const uint4 packed = make_uint4(pack_bf16x2(acc[0].x, acc[0].y), pack_bf16x2(acc[1].x, acc[1].y),
                                      pack_bf16x2(acc[2].x, acc[2].y), pack_bf16x2(acc[3].x, acc[3].y));
      if (NORM) hbuf[j] = packed;
      else out_row[i] = packed;
    }
  }
  if (NORM) {
    float ss = 0.f;
#pragma unroll
    for (int j = 0; j < VPL; ++j) {
      if (lane + j * 32 < nv) {
        const uint32_t p[4] = {hbuf[j].x, hbuf[j].y, hbuf[j].z, hbuf[j].w};
#pragma unroll
        for (int q = 0; q < 4; ++q) ss += bf16_lo(p[q]) * bf16_lo(p[q]) + bf16_hi(p[q]) * bf16_hi(p[q]);
      }
    }
    ss = warp_sum(ss);
    const float rcp = 1.0f / sqrtf(ss / (float)hidden + norm_eps);
#pragma unroll
    for (int j = 0; j < VPL; ++j) {
      const int i = lane + j * 32;
      if (i < nv) {
        const uint32_t p[4] = {hbuf[j].x, hbuf[j].y, hbuf[j].z, hbuf[j].w};
        const uint4 wv = (*nwr)[j];
        const uint32_t w[4] = {wv.x, wv.y, wv.z, wv.w};
        uint32_t o[4];
#pragma unroll
        for (int q = 0; q < 4; ++q)
          o[q] = pack_bf16x2(bf16_lo(p[q]) * rcp * bf16_lo(w[q]), bf16_hi(p[q]) * rcp * bf16_hi(w[q]));
        out_row[i] = make_uint4(o[0], o[1], o[2], o[3]);
      }
    }
  }
}

// The weighted query chunks of this lane as (even, odd) element pairs.
template <int VPL>
__device__ __forceinline__ void load_wq(const float* __restrict__ wq, int nv, int lane, float2 (&wqr)[VPL][4]) {
#pragma unroll
  for (int j = 0; j < VPL; ++j) {
    const int i = lane + j * 32;
#pragma unroll
    for (int e = 0; e < 4; ++e)
      wqr[j][e] = (i < nv) ? make_float2(wq[i * 8 + 2 * e], wq[i * 8 + 2 * e + 1]) : make_float2(0.f, 0.f);
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
// weighted query, a model constant, is loaded before the wait on the producer,
// and so are the first `stable` bank sources: the caller guarantees that they
// were written before the previous kernel on the stream began (the Block AttnRes
// trunk: the outputs of finished blocks), so that only the newest source and the
// partial are read after the wait.
template <int VPL, int NSRC, bool NORM = false>
__global__ void __launch_bounds__(kMixWarps * 32, 3)
    attnres_reg_kernel(const uint4* __restrict__ bank, int nsrc_bank, int64_t tokens, int hidden,
                       const uint4* __restrict__ partial, const float* __restrict__ wq, float eps,
                       uint4* __restrict__ out, const uint4* __restrict__ norm_w = nullptr, float norm_eps = 0.f,
                       int stable = 0) {
  pdl_launch_dependents();
  const int64_t t = (int64_t)blockIdx.x * kMixWarps + threadIdx.x / 32;
  const int lane = threadIdx.x & 31;
  const int nv = hidden / 8;
  float2 wqr[VPL][4];
  load_wq<VPL>(wq, nv, lane, wqr);
  uint4 nwr[VPL];  // the norm weight, a model constant like wq
#pragma unroll
  for (int j = 0; j < VPL; ++j)
    nwr[j] = (NORM && lane + j * 32 < nv) ? norm_w[lane + j * 32] : make_uint4(0u, 0u, 0u, 0u);
  uint4 x[NSRC][VPL];
  // Issue every load of a phase first (maximum memory-level parallelism): the
  // stable sources before the wait, the others after it; then reduce.
  const bool row = t < tokens;
  auto load_source = [&](int s) {
    const uint4* src = (s < nsrc_bank) ? bank + ((int64_t)s * tokens + t) * nv : partial + t * nv;
#pragma unroll
    for (int j = 0; j < VPL; ++j) {
      const int i = lane + j * 32;
      x[s][j] = (i < nv) ? src[i] : make_uint4(0, 0, 0, 0);
    }
  };
#pragma unroll
  for (int s = 0; s < NSRC; ++s)
    if (row && s < stable) load_source(s);
  pdl_wait();
  if (!row) return;
#pragma unroll
  for (int s = 0; s < NSRC; ++s)
    if (s >= stable) load_source(s);
  mix_token<VPL, NSRC, NORM>(RegRows<VPL, NSRC>{x}, wqr, nv, hidden, eps, lane, out + t * nv, &nwr, norm_eps);
}

// Source rows of one token in a shared-memory stage, read once per pass: the
// compiler barrier between the passes makes the second pass load them again
// instead of keeping 8 fp32 values per loaded chunk live across the softmax.
struct SmemRows {
  const uint4* base;  // source 0's row of this token
  int src_stride;     // uint4 between two sources' rows
  int nv;
  int lane;
  __device__ __forceinline__ uint4 operator()(int s, int j) const {
    const int c = lane + j * 32;
    return c < nv ? base[s * src_stride + c] : make_uint4(0u, 0u, 0u, 0u);
  }
  __device__ __forceinline__ void between_phases() const { asm volatile("" ::: "memory"); }
};

// Large token counts: a persistent stream through shared memory. A tile is
// kStreamTok consecutive tokens; each source's rows of a tile are one
// contiguous run of HBM, fetched with one cp.async.bulk (plain, no multicast)
// into shared-memory stages guarded by full/empty mbarriers. Warp 0 (one lane)
// is the producer and issues the CTA's tiles in order; G groups of kStreamTok
// consumer warps take the tiles in turn, one warp per token, and release the
// stage once their token is mixed. Each group owns `spg` stages of its own and
// cycles through them, so the uses of a stage are consumed in order by one
// group: a consumer never waits on a phase two ahead of its barrier, whose
// parity would alias the previous one.
// The consumers are latency-bound (score reductions, softmax, two passes over
// the rows), so G is as large as shared memory allows: 16 consumer warps reached
// 79-85% of the measured HBM copy bandwidth where 8 reached 64%.
// Every wait is bounded: a wait that runs out stops the pipeline, the tokens it
// could not mix are written as NaN, and the CTA waits (bounded) for its copies in
// flight before it exits.
constexpr int kStreamTok = 4;
constexpr int kStreamMaxGroups = 4;
constexpr int kStreamMaxStages = 8;
constexpr int kStreamSmemBudget = 220 * 1024;

__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

template <int VPL, int NSRC, int G>
__global__ void __launch_bounds__((1 + kStreamTok * G) * 32, 1)
    attnres_stream_kernel(const uint4* __restrict__ bank, int nsrc_bank, int64_t tokens, int hidden,
                          const uint4* __restrict__ partial, const float* __restrict__ wq, float eps,
                          uint4* __restrict__ out, int spg, int32_t* status, int64_t stall_tile,
                          uint64_t wait_ns) {
  extern __shared__ __align__(128) uint8_t smem_raw[];
  __shared__ uint64_t full[kStreamMaxStages], empty[kStreamMaxStages];
  __shared__ int abort_flag;
  __shared__ int64_t issued_tiles;
  const int warp = threadIdx.x / 32, lane = threadIdx.x & 31;
  const int nv = hidden / 8;
  const int64_t row_bytes = (int64_t)hidden * 2;
  const int64_t src_tile_bytes = kStreamTok * row_bytes;  // one source's rows of one tile
  const int64_t stage_bytes = NSRC * src_tile_bytes;
  const int64_t ntiles = (tokens + kStreamTok - 1) / kStreamTok;
  const int64_t my_tiles = ntiles > (int64_t)blockIdx.x ? (ntiles - 1 - blockIdx.x) / gridDim.x + 1 : 0;
  const int stages = G * spg;  // <= kStreamMaxStages (host)
  // the CTA's tile i goes to group i % G, into that group's stage (i / G) % spg,
  // as use number (i / G) / spg
  auto stage_of = [&](int64_t i) { return (int)(i % G) * spg + (int)((i / G) % spg); };
  auto use_of = [&](int64_t i) { return (uint32_t)((i / G) / spg); };
  if (threadIdx.x == 0) {
    for (int s = 0; s < stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kStreamTok);
    }
    abort_flag = 0;
    issued_tiles = 0;
    fence_mbar_init();
  }
  pdl_launch_dependents();
  float2 wqr[VPL][4];
  if (warp > 0) load_wq<VPL>(wq, nv, lane, wqr);
  __syncthreads();
  pdl_wait();
  if (warp == 0) {
    if (lane == 0) {
      const uint8_t* bank_b = reinterpret_cast<const uint8_t*>(bank);
      const uint8_t* part_b = reinterpret_cast<const uint8_t*>(partial);
      int64_t i = 0;
      for (; i < my_tiles; ++i) {
        const int st = stage_of(i);
        const uint32_t use = use_of(i);
        if (use >= 1 && !mbar_wait_for(&empty[st], (use - 1) & 1, wait_ns)) {
          atomicExch(&abort_flag, 1);
          break;
        }
        if (*reinterpret_cast<volatile int*>(&abort_flag)) break;
        const int64_t t0 = ((int64_t)blockIdx.x + i * gridDim.x) * kStreamTok;
        const int64_t tt = tokens - t0 < kStreamTok ? tokens - t0 : kStreamTok;
        const uint32_t bytes = (uint32_t)(tt * row_bytes);
        mbar_arrive_expect_tx(&full[st], NSRC * bytes);
        // test hook: CTA 0 announces tile `stall_tile` but never copies it, so
        // its consumers' bounded wait runs out (no fault: nothing is in flight)
        if (blockIdx.x == 0 && i == stall_tile) continue;
        uint8_t* dst = smem_raw + st * stage_bytes;
#pragma unroll
        for (int s = 0; s < NSRC; ++s) {
          const uint8_t* src = s < nsrc_bank ? bank_b + ((int64_t)s * tokens + t0) * row_bytes : part_b + t0 * row_bytes;
          bulk_load(dst + s * src_tile_bytes, src, bytes, &full[st]);
        }
      }
      issued_tiles = i;
    }
  } else {
    const int cw = warp - 1;
    const int grp = cw / kStreamTok, tok = cw % kStreamTok;
    for (int64_t i = grp; i < my_tiles; i += G) {
      const int st = stage_of(i);
      const uint32_t use = use_of(i);
      const int64_t t = ((int64_t)blockIdx.x + i * gridDim.x) * kStreamTok + tok;
      const bool ready = mbar_wait_for(&full[st], use & 1, wait_ns) && !*reinterpret_cast<volatile int*>(&abort_flag);
      if (!ready) {
        atomicExch(&abort_flag, 1);
        for (int64_t k = i; k < my_tiles; k += G) {
          const int64_t tk = ((int64_t)blockIdx.x + k * gridDim.x) * kStreamTok + tok;
          if (tk < tokens)
            for (int c = lane; c < nv; c += 32)
              out[tk * nv + c] = make_uint4(0x7fc07fc0u, 0x7fc07fc0u, 0x7fc07fc0u, 0x7fc07fc0u);
        }
        break;
      }
      if (t < tokens) {
        const SmemRows rows{reinterpret_cast<const uint4*>(smem_raw + st * stage_bytes + tok * row_bytes),
                            (int)(src_tile_bytes / 16), nv, lane};
        mix_token<VPL, NSRC>(rows, wqr, nv, hidden, eps, lane, out + t * nv);
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[st]);
    }
  }
  __syncthreads();
  // after a wait ran out, the copies already issued still land in this CTA's
  // shared memory: wait for them (bounded) before exiting
  if (threadIdx.x == 0 && abort_flag) {
    report(status, AIOSB_DEV_WAIT_TIMEOUT);
    const int64_t n = issued_tiles;
    for (int64_t j = n > stages ? n - stages : 0; j < n; ++j)
      if (!(blockIdx.x == 0 && j == stall_tile)) mbar_wait_for(&full[stage_of(j)], use_of(j) & 1, wait_ns);
  }
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

// Test hook of the stream kernel (aiosb_test_attnres_stream_stall): a tile whose
// copies CTA 0 skips, and the bound of every wait.
struct StreamTest {
  int64_t stall_tile = -1;
  uint64_t wait_ns = kWaitLimitNs;
};
StreamTest g_stream_test;

template <int G>
cudaError_t launch_stream(int64_t total, const void* bank, int64_t sources, int64_t tokens, int64_t hidden,
                          const void* partial, const float* wq, float eps, void* out, int spg, int32_t* status,
                          void* stream) {
  auto kern = attnres_stream_kernel<3, 1, G>;
  switch (total) {
    case 1: kern = attnres_stream_kernel<3, 1, G>; break;
    case 2: kern = attnres_stream_kernel<3, 2, G>; break;
    case 3: kern = attnres_stream_kernel<3, 3, G>; break;
    case 4: kern = attnres_stream_kernel<3, 4, G>; break;
    case 5: kern = attnres_stream_kernel<3, 5, G>; break;
    case 6: kern = attnres_stream_kernel<3, 6, G>; break;
    case 7: kern = attnres_stream_kernel<3, 7, G>; break;
    case 8: kern = attnres_stream_kernel<3, 8, G>; break;
    case 9: kern = attnres_stream_kernel<3, 9, G>; break;
    default: kern = attnres_stream_kernel<3, 10, G>; break;
  }
  const size_t smem = (size_t)G * spg * total * kStreamTok * hidden * 2;
  cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  const int64_t tiles = (tokens + kStreamTok - 1) / kStreamTok;
  const dim3 grid((unsigned)std::min<int64_t>(tiles, sm_count()));
  return launch_pdl(kern, grid, dim3((1 + kStreamTok * G) * 32), smem, as_stream(stream), (const uint4*)bank,
                    (int)sources, tokens, (int)hidden, (const uint4*)partial, wq, eps, (uint4*)out, spg, status,
                    g_stream_test.stall_tile, g_stream_test.wait_ns);
}

// Token count from which the stream kernel replaces the register kernel
// (AIOSB_ATTNRES_STREAM_MIN_TOKENS overrides it, for measurements).
int64_t g_stream_min_tokens = [] {
  const char* env = getenv("AIOSB_ATTNRES_STREAM_MIN_TOKENS");
  return env != nullptr ? (int64_t)atoll(env) : (int64_t)2048;
}();

}  // namespace
}  // namespace aiosb

using namespace aiosb;

extern "C" int aiosb_attnres_mix(const void* bank, int64_t sources, int64_t tokens, int64_t hidden,
                                 const void* partial, const float* weighted_query, float eps, void* out,
                                 int32_t* status, void* stream) {
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
  const bool reg_shape = total <= kMaxRegSources && nv <= 3 * 32;
  // consumer groups (4 tokens of every source staged per group and stage) and
  // stages per group that fit the shared-memory budget
  const int64_t stage_bytes = total * kStreamTok * hidden * 2;
  const int groups = (int)std::min<int64_t>(kStreamMaxGroups, kStreamSmemBudget / stage_bytes);
  const int spg =
      groups >= 1 ? (int)std::min<int64_t>(kStreamMaxStages / groups, kStreamSmemBudget / (groups * stage_bytes)) : 0;
  if (reg_shape && tokens >= g_stream_min_tokens && groups >= 3) {
    e = groups == 4
            ? launch_stream<4>(total, bank, sources, tokens, hidden, partial, weighted_query, eps, out, spg, status,
                               stream)
            : launch_stream<3>(total, bank, sources, tokens, hidden, partial, weighted_query, eps, out, spg, status,
                               stream);
  } else if (reg_shape) {
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
                   (int)hidden, (const uint4*)partial, weighted_query, eps, (uint4*)out, (const uint4*)nullptr, 0.f,
                   0);
  } else {
    e = launch_pdl(attnres_generic_kernel, grid, dim3(kMixWarps * 32), 0, as_stream(stream), (const uint4*)bank,
                   (int)sources, tokens, (int)hidden, (const uint4*)partial, weighted_query, eps, (uint4*)out);
  }
  if (e != cudaSuccess) return set_error(AIOSB_ERR_LAUNCH, "attnres_mix: %s", cudaGetErrorString(e));
  return AIOSB_OK;
}

extern "C" int aiosb_attnres_mix_rmsnorm(const void* bank, int64_t sources, int64_t tokens, int64_t hidden,
                                         const void* partial, const float* weighted_query, float eps,
                                         const void* norm_w, float norm_eps, int64_t stable_sources, void* out,
                                         void* stream) {
  AIOSB_REQUIRE(sources >= 1 && tokens >= 1 && hidden >= 1, AIOSB_ERR_INVALID_ARG,
                "bank dimensions must be positive");
  const int64_t total = sources + (partial != nullptr ? 1 : 0);
  AIOSB_REQUIRE(total <= kMaxRegSources && hidden % 8 == 0 && hidden / 8 <= 3 * 32, AIOSB_ERR_UNSUPPORTED,
                "attnres_mix_rmsnorm: at most %d sources and hidden <= 768 (a multiple of 8)", kMaxRegSources);
  AIOSB_REQUIRE(bank && weighted_query && norm_w && out, AIOSB_ERR_INVALID_ARG, "attnres_mix_rmsnorm: null pointer");
  AIOSB_REQUIRE(aligned16(bank) && aligned16(out) && aligned16(norm_w) && (partial == nullptr || aligned16(partial)),
                AIOSB_ERR_MISALIGNED, "attnres_mix_rmsnorm: bank/partial/norm_w/out must be 16-byte aligned");
  const dim3 grid((unsigned)((tokens + kMixWarps - 1) / kMixWarps));
  auto kern = attnres_reg_kernel<3, 1, true>;
  switch (total) {
    case 1: kern = attnres_reg_kernel<3, 1, true>; break;
    case 2: kern = attnres_reg_kernel<3, 2, true>; break;
    case 3: kern = attnres_reg_kernel<3, 3, true>; break;
    case 4: kern = attnres_reg_kernel<3, 4, true>; break;
    case 5: kern = attnres_reg_kernel<3, 5, true>; break;
    case 6: kern = attnres_reg_kernel<3, 6, true>; break;
    case 7: kern = attnres_reg_kernel<3, 7, true>; break;
    case 8: kern = attnres_reg_kernel<3, 8, true>; break;
    case 9: kern = attnres_reg_kernel<3, 9, true>; break;
    default: kern = attnres_reg_kernel<3, 10, true>; break;
  }
  AIOSB_REQUIRE(stable_sources >= 0 && stable_sources <= sources, AIOSB_ERR_INVALID_ARG,
                "attnres_mix_rmsnorm: stable_sources must be in [0, sources]");
  cudaError_t e = launch_pdl(kern, grid, dim3(kMixWarps * 32), 0, as_stream(stream), (const uint4*)bank, (int)sources,
                             tokens, (int)hidden, (const uint4*)partial, weighted_query, eps, (uint4*)out,
                             (const uint4*)norm_w, norm_eps, (int)stable_sources);
  if (e != cudaSuccess) return set_error(AIOSB_ERR_LAUNCH, "attnres_mix_rmsnorm: %s", cudaGetErrorString(e));
  return AIOSB_OK;
}

extern "C" int aiosb_test_attnres_stream_stall(int64_t stall_tile, uint64_t wait_limit_ns) {
  g_stream_test.stall_tile = stall_tile;
  g_stream_test.wait_ns = wait_limit_ns > 0 ? wait_limit_ns : kWaitLimitNs;
  return AIOSB_OK;
}
