// Decode-width linears: y = x W^T for at most 16 token rows, on register-operand
// tensor-core MMAs (mma.sync m16n8k16, bf16 in, fp32 accumulate).
//
// At 8 candidate rows a decode linear is a weight stream with 8 dot products per
// weight element. It is bound by the dependency chain of the decode step (each
// kernel waits on its predecessor), not by math or bandwidth, so the work after
// the wait is kept short:
//   * the weights of the CTA's first tile (and the RMSNorm weight) are loaded
//     into registers before griddepcontrol.wait, while the previous kernel still
//     runs, already in the MMA A-fragment layout;
//   * after the wait each lane loads its B fragments (the activation rows, or
//     rows normalised from the fp32 residual statistics, RMSNormFused,
//     aios/layers/norm.py:34-40) straight from global memory, one 16-byte load
//     per fragment pair: there is no operand staging;
//   * 2 MMAs per 32-wide K block, a fixed-order sum of the 8 warps' partial
//     tiles through shared memory, then the epilogues of the tcgen05 GEMM (store,
//     SwiGLU on the 64-row interleaved gate/up layout, residual add with optional
//     fp32 statistics), written 16 bytes per token.
// Measured on the S10 decode step (57 linears of 8 rows): 4.56 us per launch for
// a CUDA-core GEMV that staged its operand in shared memory, 2.60 us here.
// tcgen05 is not used at this width: its MMA reads shared-memory descriptors,
// accumulates in TMEM and is read back with tcgen05.ld, and one-CTA probes timed
// about 150 cycles per instruction at N = 16, where a warp-level MMA on register
// operands completes in a few dozen cycles.
// Rounding points equal the tcgen05 path: fp32 accumulation, bf16 output, the
// gate/up values rounded to bf16 before SwiGLU, the delta rounded before the
// residual add. Summation order differs, so results agree to rounding.
#include <algorithm>

#include "abi_util.h"
#include "common.cuh"
#include "gemv.h"

namespace aiosb {
namespace {

constexpr int kGemvThreads = 256;  // 8 warps, splitting K
constexpr int kGemvFeat = kGemvThreads / 32;

// ---- register-operand tensor-core GEMV (mma.sync m16n8k16, bf16 -> fp32) ----
// A CTA computes one 16-row weight tile (16 output features; SwiGLU: 8 gate + 8
// up rows of 8 output features) for up to NT * 8 token rows. Its 8 warps split
// K; warp w owns the 32-wide K blocks [w * kb, (w + 1) * kb). Within a block the
// K order is permuted per lane so that every fragment is one 16-byte load: lane
// (g = lane / 4, t = lane % 4) takes physical elements [32 b + 8 t, 32 b + 8 t + 8)
// of weight rows g and g + 8 (A) and of token row g (B), and feeds them as the
// logical K positions {2t, 2t+1, 2t+8, 2t+9} of two consecutive k16 MMAs. A dot
// product is invariant under a permutation of K applied to both operands, so no
// shuffle or shared-memory staging is needed: the weights go to registers before
// griddepcontrol.wait, the activations straight from global memory after it.
// Partial tiles of the 8 warps are summed in warp order through shared memory.
__device__ __forceinline__ void mma_bf16_16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                               uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// GROUPS: more than one 16-row group along grid y (prefill widths). The decode
// instantiations (false) keep row 0 and streaming weight loads as constants, so
// their register use (and with it how many CTAs share an SM with the previous
// kernel's) is unchanged by the row-group addressing.
// ---- AttnRes mixer operand (MODE kGemvMix) ----------------------------------
// this lane's share of a source row's dot product with the routing query and of
// its sum of squares (8 elements, in order)
__device__ __forceinline__ void mix_sums(const uint4& v, const float (&wq)[8], float& dot, float& ss) {
  const uint32_t p[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const float lo = bf16_lo(p[q]), hi = bf16_hi(p[q]);
    dot += lo * wq[2 * q] + hi * wq[2 * q + 1];
    ss += lo * lo + hi * hi;
  }
}
// sums over the 4 lanes of a fragment row (lanes 4g .. 4g + 3)
__device__ __forceinline__ void quad_sum2(float& x, float& y) {
  x += __shfl_xor_sync(0xffffffffu, x, 1);
  y += __shfl_xor_sync(0xffffffffu, y, 1);
  x += __shfl_xor_sync(0xffffffffu, x, 2);
  y += __shfl_xor_sync(0xffffffffu, y, 2);
}

// MODE: 0 plain operand rows, 1 rows normalised from residual statistics,
// 2 the AttnRes mixer's rows, normalised (kGemvMix), 3 and 4 as 1 and 0 with
// the store epilogue also writing per-tile statistics (kGemvStatTiles,
// kGemvPlainTiles: the LM head).
// Launch bounds: the 8-row LM head with tile statistics is held to 80 registers
// so that three CTAs share an SM; the others carry an explicit one-CTA bound,
// under which ptxas gives the 768-wide decode linears 94 registers instead of
// 69, and the S10 keystroke is faster with it (2.715 against 2.750 ms p50,
// three runs each on one box).
template <int NT, int KB, int MODE, bool GROUPS>
__global__ void __launch_bounds__(kGemvThreads, ((MODE == kGemvStatTiles || MODE == kGemvPlainTiles) && NT == 1) ? 3 : 1)
    gemv_mma_kernel(const GemvArgs a) {
  constexpr bool TILES = MODE == kGemvStatTiles || MODE == kGemvPlainTiles;
  constexpr bool STAT = MODE == kGemvStat || MODE == kGemvStatTiles, MIX = MODE == kGemvMix;
  static_assert(!MIX || (NT == 1 && !GROUPS), "the mixer operand serves one 8-row group");
  static_assert(!TILES || !GROUPS, "tile statistics serve one row group");
  constexpr int TM = NT * 8;  // token rows covered
  __shared__ float red[kGemvFeat][NT][32][4];  // [warp][n tile][lane][fragment]
  __shared__ float tile[TM][17];               // reduced [token][row] (padded)
  __shared__ float ssw[kGemvFeat][TM];          // statistics mode: per-warp sums of squares
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, t4 = lane & 3;
  const int K = (int)a.k;
  const int kb = K / 256;  // 32-wide blocks per warp
  // grid row y covers token rows [row0, row0 + TM) (prefill widths: several row groups)
  const int row0 = GROUPS ? (int)blockIdx.y * TM : 0;
  const int T = min(TM, a.rows - row0);
  const bool silu = a.epilogue == AIOSB_EPI_SILU_MUL;
  const int feat_per_tile = silu ? 8 : 16;
  const int ntiles = (int)(a.n_out / feat_per_tile);
  const int64_t kbase = (int64_t)warp * kb * 32 + 8 * t4;  // this lane's first element, block 0

  // weight rows of tile `tl` held by this lane (rows g and g + 8 of the M tile)
  auto load_w = [&](int tl, uint4 (&wa)[KB], uint4 (&wb)[KB]) {
    int64_t r0, r1;
    if (silu) {  // packed [g0..63 | u0..63 | g64..]: gate and up rows of feature f
      const int64_t f = (int64_t)tl * 8 + g;
      r0 = (f / 64) * 128 + (f % 64);
      r1 = r0 + 64;
    } else {
      r0 = (int64_t)tl * 16 + g;
      r1 = r0 + 8;
    }
    // Weights are read once per forward and a decode step streams more of them
    // than L2 holds, so they are loaded cache-streaming (evict first): the
    // activations, the KV cache and the kernels' code stay in L2 across the step
    // instead of being refetched from DRAM (measured: 243.6 -> 220.5 us per S10
    // decode step; the sampler step kernel alone 35 -> 25 us). With several row
    // groups the other groups' CTAs read the same tile, so it stays cached.
#pragma unroll
    for (int b = 0; b < KB; ++b) {
      const bool ok = tl < ntiles && b < kb;
      const uint4* pa = reinterpret_cast<const uint4*>(a.w + r0 * K + kbase + b * 32);
      const uint4* pb = reinterpret_cast<const uint4*>(a.w + r1 * K + kbase + b * 32);
      wa[b] = ok ? (GROUPS ? __ldg(pa) : __ldcs(pa)) : make_uint4(0u, 0u, 0u, 0u);
      wb[b] = ok ? (GROUPS ? __ldg(pb) : __ldcs(pb)) : make_uint4(0u, 0u, 0u, 0u);
    }
  };
  uint4 wa[KB], wb[KB];
  load_w(blockIdx.x, wa, wb);
  uint4 nwv[KB];
  if (STAT || MIX) {
#pragma unroll
    for (int b = 0; b < KB; ++b)
      nwv[b] = b < kb ? *reinterpret_cast<const uint4*>(a.nw + kbase + b * 32) : make_uint4(0u, 0u, 0u, 0u);
  }
  // MIX, before the wait: the stable bank sources' rows of this CTA's tokens go
  // to shared memory, and this lane's partial dot products with the routing
  // query and sums of squares of them to mpart
  extern __shared__ __align__(16) uint8_t gemv_dyn[];
  const int RS = K + kMixRowPad;  // staged row stride (elements): bank-conflict free 16-byte reads
  __nv_bfloat16* mvals = reinterpret_cast<__nv_bfloat16*>(gemv_dyn);  // [stable][8][RS]
  // then [warp][row][source][dot, ss] partial sums and [row][source] weights
  float* mpart = reinterpret_cast<float*>(gemv_dyn + (size_t)(MIX ? a.mix_stable : 0) * 8 * RS * 2);
  float* malpha = mpart + kGemvFeat * 8 * kMixMaxSources * 2;
  auto mix_part = [&](int w, int row, int src) { return mpart + ((w * 8 + row) * kMixMaxSources + src) * 2; };
  float wqv[MIX ? KB : 1][8];
  if constexpr (MIX) {
    const int ST = a.mix_stable;
    const int nv8 = K / 8;
    for (int u = tid; u < ST * 8 * nv8; u += kGemvThreads) {
      const int sr = u / nv8, c = u % nv8, src = sr / 8, row = sr % 8;
      if (row < T)
        cp_async16(mvals + (int64_t)sr * RS + c * 8, a.mix_bank + ((int64_t)src * a.mix_tokens + row) * K + c * 8);
    }
#pragma unroll
    for (int b = 0; b < KB; ++b)
#pragma unroll
      for (int e = 0; e < 8; ++e) wqv[b][e] = b < kb ? a.mix_wq[kbase + b * 32 + e] : 0.f;
    cp_async_wait_all();
    __syncthreads();
    for (int src = 0; src < ST; ++src) {
      float dot = 0.f, ss = 0.f;
      if (g < T) {
#pragma unroll
        for (int b = 0; b < KB; ++b) {
          if (b < kb) {
            const uint4 v = *reinterpret_cast<const uint4*>(mvals + (int64_t)(src * 8 + g) * RS + kbase + b * 32);
            mix_sums(v, wqv[b], dot, ss);
          }
        }
      }
      quad_sum2(dot, ss);
      if (t4 == 0) {
        mix_part(warp, g, src)[0] = dot;
        mix_part(warp, g, src)[1] = ss;
      }
    }
  }
  // A residual-add linear (o, down) lets its successor launch at once: that
  // successor is a linear whose weights can stream in meanwhile (measured: 5.5 us
  // less per decode step). The others launch it only after their own wait, so a
  // kernel that follows them may read, before its own wait, anything written two
  // or more kernels back (the decode attention after the qkv linear does).
  // The caller may ask for the same early launch for other epilogues
  // (AIOSB_LINEAR_EARLY_DEPENDENTS) where the successor allows it. The LM head
  // with tile statistics always does: its successor, the CandidateGroup step,
  // reads only its state before its own wait.
  const bool early = a.epilogue == AIOSB_EPI_ADD || a.early_dependents || TILES;
  if (early) pdl_launch_dependents();
  pdl_wait();
  if (!early) pdl_launch_dependents();

  // ---- B fragments: token row n = nt * 8 + g, this lane's 8 elements per block
  uint4 xb[NT][KB];
  if constexpr (MIX) {
    // the sources read after the wait: the newest bank source if it is not
    // stable, and the partial (the block's running sum)
    const int S = a.mix_sources, ST = a.mix_stable;
    const int nlate = S - ST + (a.mix_partial != nullptr ? 1 : 0);  // <= 2 (host)
    const int ntot = S + (a.mix_partial != nullptr ? 1 : 0);
    uint4 late[2][KB];
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const bool live = i < nlate && g < T;
      const __nv_bfloat16* src = !live ? nullptr
                                 : i < S - ST ? a.mix_bank + ((int64_t)(ST + i) * a.mix_tokens + g) * K
                                              : a.mix_partial + (int64_t)g * K;
#pragma unroll
      for (int b = 0; b < KB; ++b)
        late[i][b] = (live && b < kb) ? *reinterpret_cast<const uint4*>(src + kbase + b * 32)
                                      : make_uint4(0u, 0u, 0u, 0u);
    }
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      if (i < nlate) {
        float dot = 0.f, ss = 0.f;
#pragma unroll
        for (int b = 0; b < KB; ++b)
          if (b < kb) mix_sums(late[i][b], wqv[b], dot, ss);
        quad_sum2(dot, ss);
        if (t4 == 0) {
          mix_part(warp, g, ST + i)[0] = dot;
          mix_part(warp, g, ST + i)[1] = ss;
        }
      }
    }
    __syncthreads();
    // depth softmax of token row `warp` (aios/kernel/attnres.py:8-127): every
    // lane sums the 8 warps' partials of every source in warp order and takes
    // score_s = dot_s / rms_s, the max, exp and their sum in source order, and
    // the weights rounded to bf16, as the mixer kernel does
    if (warp < T) {
      float score[kMixMaxSources];
      float mx = -INFINITY;
#pragma unroll
      for (int s2 = 0; s2 < kMixMaxSources; ++s2) {
        score[s2] = -INFINITY;
        if (s2 < ntot) {
          float dot = 0.f, ss = 0.f;
#pragma unroll
          for (int w = 0; w < kGemvFeat; ++w) {
            dot += mix_part(w, warp, s2)[0];
            ss += mix_part(w, warp, s2)[1];
          }
          score[s2] = dot * (1.0f / sqrtf(ss / (float)K + a.mix_eps));
          mx = fmaxf(mx, score[s2]);
        }
      }
      float denom = 0.f;
#pragma unroll
      for (int s2 = 0; s2 < kMixMaxSources; ++s2) {
        if (s2 < ntot) {
          score[s2] = expf(score[s2] - mx);
          denom += score[s2];
        }
      }
      if (lane < ntot) {
        float w8 = 0.f;
#pragma unroll
        for (int s2 = 0; s2 < kMixMaxSources; ++s2)
          if (s2 == lane) w8 = score[s2];
        malpha[warp * kMixMaxSources + lane] = round_bf16(w8 / denom);
      }
    }
    __syncthreads();
    // h = bf16(sum_s alpha_s x_s) (fp32 accumulation in source order), then the
    // RMSNorm that consumes it: bf16(h * rcp * nw)
    float ssh = 0.f;
    uint4 hx[KB];
#pragma unroll
    for (int b = 0; b < KB; ++b) {
      float acc[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) acc[e] = 0.f;
      if (g < T && b < kb) {
        for (int s2 = 0; s2 < ntot; ++s2) {
          const float al = malpha[g * kMixMaxSources + s2];
          uint4 v;
          if (s2 < ST) v = *reinterpret_cast<const uint4*>(mvals + (int64_t)(s2 * 8 + g) * RS + kbase + b * 32);
          else v = s2 - ST == 0 ? late[0][b] : late[1][b];
          const uint32_t p[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            acc[2 * q] = fmaf(al, bf16_lo(p[q]), acc[2 * q]);
            acc[2 * q + 1] = fmaf(al, bf16_hi(p[q]), acc[2 * q + 1]);
          }
        }
      }
      hx[b] = make_uint4(pack_bf16x2(acc[0], acc[1]), pack_bf16x2(acc[2], acc[3]), pack_bf16x2(acc[4], acc[5]),
                         pack_bf16x2(acc[6], acc[7]));
      const uint32_t hp[4] = {hx[b].x, hx[b].y, hx[b].z, hx[b].w};
#pragma unroll
      for (int q = 0; q < 4; ++q) ssh += bf16_lo(hp[q]) * bf16_lo(hp[q]) + bf16_hi(hp[q]) * bf16_hi(hp[q]);
    }
    ssh += __shfl_xor_sync(0xffffffffu, ssh, 1);
    ssh += __shfl_xor_sync(0xffffffffu, ssh, 2);
    if (t4 == 0) ssw[warp][g] = ssh;
    __syncthreads();
    float sst = 0.f;
#pragma unroll
    for (int w = 0; w < kGemvFeat; ++w) sst += ssw[w][g];
    const float rcp = 1.0f / sqrtf(sst / (float)K + a.eps);
#pragma unroll
    for (int b = 0; b < KB; ++b) {
      const uint32_t hp[4] = {hx[b].x, hx[b].y, hx[b].z, hx[b].w};
      const uint32_t w4[4] = {nwv[b].x, nwv[b].y, nwv[b].z, nwv[b].w};
      uint32_t o[4];
#pragma unroll
      for (int q = 0; q < 4; ++q)
        o[q] = pack_bf16x2(bf16_lo(hp[q]) * rcp * bf16_lo(w4[q]), bf16_hi(hp[q]) * rcp * bf16_hi(w4[q]));
      xb[0][b] = (g < T) ? make_uint4(o[0], o[1], o[2], o[3]) : make_uint4(0u, 0u, 0u, 0u);
    }
  } else if (!STAT) {
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      const int n = nt * 8 + g;
#pragma unroll
      for (int b = 0; b < KB; ++b)
        xb[nt][b] = (n < T && b < kb)
                        ? *reinterpret_cast<const uint4*>(a.x + (int64_t)(row0 + n) * a.x_stride + kbase + b * 32)
                        : make_uint4(0u, 0u, 0u, 0u);
    }
  } else {
    // rows normalised from the fp32 residual stream s (RMSNormFused,
    // aios/layers/norm.py:34-40): the sum of squares of a whole row is reduced
    // over the 4 lanes of a row and the 8 warps (in warp order)
    float4 sv[NT][KB][2];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      const int n = nt * 8 + g;
#pragma unroll
      for (int b = 0; b < KB; ++b) {
        const bool ok = n < T && b < kb;
        const float4* src = reinterpret_cast<const float4*>(a.stat_x + (int64_t)(row0 + n) * K + kbase + b * 32);
        sv[nt][b][0] = ok ? src[0] : make_float4(0.f, 0.f, 0.f, 0.f);
        sv[nt][b][1] = ok ? src[1] : make_float4(0.f, 0.f, 0.f, 0.f);
      }
    }
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      float ss = 0.f;
#pragma unroll
      for (int b = 0; b < KB; ++b)
#pragma unroll
        for (int h = 0; h < 2; ++h)
          ss += sv[nt][b][h].x * sv[nt][b][h].x + sv[nt][b][h].y * sv[nt][b][h].y +
                sv[nt][b][h].z * sv[nt][b][h].z + sv[nt][b][h].w * sv[nt][b][h].w;
      ss += __shfl_xor_sync(0xffffffffu, ss, 1);
      ss += __shfl_xor_sync(0xffffffffu, ss, 2);
      if (t4 == 0) ssw[warp][nt * 8 + g] = ss;
    }
    __syncthreads();
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      float ss = 0.f;
#pragma unroll
      for (int w = 0; w < kGemvFeat; ++w) ss += ssw[w][nt * 8 + g];
      const float rcp = 1.0f / sqrtf(ss / (float)K + a.eps);
#pragma unroll
      for (int b = 0; b < KB; ++b) {
        const uint32_t p[4] = {nwv[b].x, nwv[b].y, nwv[b].z, nwv[b].w};
        const float4 s0 = sv[nt][b][0], s1 = sv[nt][b][1];
        xb[nt][b] = make_uint4(
            pack_bf16x2(s0.x * rcp * bf16_lo(p[0]), s0.y * rcp * bf16_hi(p[0])),
            pack_bf16x2(s0.z * rcp * bf16_lo(p[1]), s0.w * rcp * bf16_hi(p[1])),
            pack_bf16x2(s1.x * rcp * bf16_lo(p[2]), s1.y * rcp * bf16_hi(p[2])),
            pack_bf16x2(s1.z * rcp * bf16_lo(p[3]), s1.w * rcp * bf16_hi(p[3])));
      }
    }
  }

  // epilogue thread (token, half) of the residual add: its 8 residual values are
  // requested now, so their round trip overlaps the activation loads and MMAs
  const bool epi_thread = tid < TM * 2 && (tid >> 1) < T && !silu;
  const int64_t epi_row = (int64_t)row0 + (tid >> 1);
  auto load_res = [&](int tl) {
    return (epi_thread && a.epilogue == AIOSB_EPI_ADD && tl < ntiles)
               ? *reinterpret_cast<const uint4*>(a.residual + epi_row * a.residual_stride + (int64_t)tl * 16 +
                                                 8 * (tid & 1))
               : make_uint4(0u, 0u, 0u, 0u);
  };
  uint4 rv = load_res(blockIdx.x);

  for (int tl = blockIdx.x; tl < ntiles; tl += gridDim.x) {
    uint4 na[KB], nb[KB];
    load_w(tl + gridDim.x, na, nb);  // next tile, in flight during this one
    float d[NT][4];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) d[nt][0] = d[nt][1] = d[nt][2] = d[nt][3] = 0.f;
#pragma unroll
    for (int b = 0; b < KB; ++b) {
      if (b < kb) {
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
          mma_bf16_16816(d[nt], wa[b].x, wb[b].x, wa[b].y, wb[b].y, xb[nt][b].x, xb[nt][b].y);
          mma_bf16_16816(d[nt], wa[b].z, wb[b].z, wa[b].w, wb[b].w, xb[nt][b].z, xb[nt][b].w);
        }
      }
    }
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
      *reinterpret_cast<float4*>(&red[warp][nt][lane][0]) = make_float4(d[nt][0], d[nt][1], d[nt][2], d[nt][3]);
    __syncthreads();
    // sum the 8 warps' partial tiles in warp order; element (row, token) of the
    // fragment layout: row = lane / 4 + 8 (j / 2), token = nt * 8 + 2 (lane % 4) + j % 2
    for (int i = tid; i < NT * 128; i += kGemvThreads) {
      const int nt = i / 128, l = (i / 4) % 32, j = i % 4;
      float sum = 0.f;
#pragma unroll
      for (int w = 0; w < kGemvFeat; ++w) sum += red[w][nt][l][j];
      tile[nt * 8 + 2 * (l & 3) + (j & 1)][(l >> 2) + 8 * (j >> 1)] = sum;
    }
    __syncthreads();
    // ---- epilogue: thread (token, half) writes 8 features (16 bytes)
    float ts_max = -INFINITY, ts_min = INFINITY, ts_sum = 0.f;  // tile statistics of the stored values
    bool ts_nan = false, ts_live = false;
    float ts_v[8];
    if (tid < TM * 2) {
      const int tk = tid >> 1, h = tid & 1;
      if (tk < T && (!silu || h == 0)) {
        float o[8];
        int64_t f0;
        if (silu) {
          f0 = (int64_t)tl * 8;
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            // gate_up output is bf16 before silu_and_mul (aios/models/qwen3.py:90-92)
            const float gt = round_bf16(tile[tk][j]), up = round_bf16(tile[tk][8 + j]);
            o[j] = gt / (1.0f + expf(-gt)) * up;
          }
        } else {
          f0 = (int64_t)tl * 16 + 8 * h;
          if (a.epilogue == AIOSB_EPI_ADD) {
            const uint32_t p[4] = {rv.x, rv.y, rv.z, rv.w};
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              const float res = (j & 1) ? bf16_hi(p[j >> 1]) : bf16_lo(p[j >> 1]);
              o[j] = res + round_bf16(tile[tk][8 * h + j]);
            }
            if (a.out_stat_x != nullptr) {
              float4* sx = reinterpret_cast<float4*>(a.out_stat_x + (int64_t)(row0 + tk) * a.n_out + f0);
              sx[0] = make_float4(o[0], o[1], o[2], o[3]);
              sx[1] = make_float4(o[4], o[5], o[6], o[7]);
              float ss = 0.f;
#pragma unroll
              for (int j = 0; j < 8; ++j) ss += o[j] * o[j];
              a.out_stat_ss[(f0 / kGemvStatGroup) * a.out_ss_stride + row0 + tk] = ss;
            }
          } else {
#pragma unroll
            for (int j = 0; j < 8; ++j) o[j] = tile[tk][8 * h + j];
          }
        }
        *reinterpret_cast<uint4*>(a.y + (int64_t)(row0 + tk) * a.y_stride + f0) =
            make_uint4(pack_bf16x2(o[0], o[1]), pack_bf16x2(o[2], o[3]), pack_bf16x2(o[4], o[5]),
                       pack_bf16x2(o[6], o[7]));
        if constexpr (TILES) {
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            ts_v[j] = round_bf16(o[j]);  // the stored logit
            ts_max = fmaxf(ts_max, ts_v[j]);
            ts_min = fminf(ts_min, ts_v[j]);
            ts_nan |= ts_v[j] != ts_v[j];
          }
          ts_live = true;
        }
      }
    }
    // Tile statistics for the sampler (the LM head, a store epilogue): per 16-id
    // tile and token row, the max, the sum of exp(v - max) and the min of the
    // stored bf16 logits (and whether any is NaN). Threads (tk, 0) and (tk, 1)
    // hold the two halves; warp 0 holds every epilogue thread.
    if (TILES && warp == 0) {
      const float pmax = __shfl_xor_sync(0xffffffffu, ts_max, 1);
      const float pmin = __shfl_xor_sync(0xffffffffu, ts_min, 1);
      const int pnan = __shfl_xor_sync(0xffffffffu, (int)ts_nan, 1);
      const float mx = fmaxf(ts_max, pmax);
      if (ts_live) {
#pragma unroll
        for (int j = 0; j < 8; ++j) ts_sum += expf(ts_v[j] - mx);
      }
      const float psum = __shfl_xor_sync(0xffffffffu, ts_sum, 1);
      if (ts_live && (tid & 1) == 0) {
        const int tk = tid >> 1;
        a.tile_stats[(int64_t)tl * a.rows + row0 + tk] =
            make_float4(mx, ts_sum + psum, fminf(ts_min, pmin), (ts_nan || pnan) ? 1.f : 0.f);
      }
    }
    if (tl + (int)gridDim.x < ntiles) rv = load_res(tl + gridDim.x);
#pragma unroll
    for (int b = 0; b < KB; ++b) {
      wa[b] = na[b];
      wb[b] = nb[b];
    }
  }
}

template <int NT, int KB, int MODE, bool GROUPS>
int launch_mma(const GemvArgs& a, cudaStream_t stream) {
  auto kern = gemv_mma_kernel<NT, KB, MODE, GROUPS>;
  const int64_t tiles = a.n_out / (a.epilogue == AIOSB_EPI_SILU_MUL ? 8 : 16);
  // as many CTAs as can be resident at once (each prefetches its first tile's
  // weights before the wait; a CTA with more tiles loads the rest one ahead)
  // the mixer operand stages its stable bank rows in dynamic shared memory
  const size_t dyn = MODE == kGemvMix ? mix_smem_bytes(a.mix_stable, a.k) : 0;
  static int per_sm = 0;  // one dynamic size per instantiation but the mixer's
  int resident_per_sm = per_sm;
  if (MODE == kGemvMix) {
    static bool attr_set = false;
    if (!attr_set) {
      cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           (int)mix_smem_bytes(kMixMaxSources - 1, kMixMaxK));
      attr_set = true;
    }
    int n = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kern, kGemvThreads, dyn) != cudaSuccess || n < 1) n = 1;
    resident_per_sm = n;
  } else if (per_sm == 0) {
    int n = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kern, kGemvThreads, 0) != cudaSuccess || n < 1) n = 2;
    per_sm = resident_per_sm = n;
  }
  const int groups = (a.rows + NT * 8 - 1) / (NT * 8);  // token row groups (grid y)
  // the LM head with tile statistics leaves one SM per row free, so that the
  // CandidateGroup step that follows (one CTA per row) starts while it runs
  constexpr bool TILES = MODE == kGemvStatTiles || MODE == kGemvPlainTiles;
  const int sms = TILES ? std::max(1, sm_count() - a.rows) : sm_count();
  const int64_t resident = std::max<int64_t>(1, (int64_t)resident_per_sm * sms / groups);
  const unsigned blocks = (unsigned)std::min<int64_t>(tiles, resident);
  cudaError_t e = launch_pdl(kern, dim3(blocks, (unsigned)groups), dim3(kGemvThreads), dyn, stream, a);
  if (e != cudaSuccess) return set_error(AIOSB_ERR_LAUNCH, "linear (gemv mma): %s", cudaGetErrorString(e));
  return AIOSB_OK;
}

template <int NT, int KB>
int launch_mma_rows(const GemvArgs& a, cudaStream_t stream) {
  if (a.tile_stats != nullptr) {  // tile_stats_eligible() holds
    if constexpr (KB == 3)
      return a.stat_x != nullptr ? launch_mma<NT, 3, kGemvStatTiles, false>(a, stream)
                                 : launch_mma<NT, 3, kGemvPlainTiles, false>(a, stream);
    return set_error(AIOSB_ERR_UNSUPPORTED, "linear: tile statistics need k <= 768");
  }
  if (a.rows > NT * 8)
    return a.stat_x != nullptr ? launch_mma<NT, KB, kGemvStat, true>(a, stream)
                               : launch_mma<NT, KB, kGemvPlain, true>(a, stream);
  return a.stat_x != nullptr ? launch_mma<NT, KB, kGemvStat, false>(a, stream)
                             : launch_mma<NT, KB, kGemvPlain, false>(a, stream);
}

bool g_gemv_enabled = [] {
  const char* env = getenv("AIOSB_DECODE_GEMV");
  return env == nullptr || atoi(env) != 0;
}();

}  // namespace

// Widest operand the register-operand path takes (more rows run as several
// 16-row groups, each re-reading the weight tile from L2); AIOSB_GEMV_MAX_ROWS
// lowers or raises it (1..kMaxGemvRows).
int g_gemv_max_rows = [] {
  const char* env = getenv("AIOSB_GEMV_MAX_ROWS");
  const int v = env ? atoi(env) : kGemvDefaultRows;
  return v >= 1 && v <= kMaxGemvRows ? v : kGemvDefaultRows;
}();

bool mix_eligible(int64_t rows, int64_t k, int64_t n_out, int64_t sources, int64_t stable, bool partial) {
  return g_gemv_enabled && rows >= 1 && rows <= 8 && k == kMixMaxK && n_out % 16 == 0 && sources >= 1 &&
         stable >= 0 && stable <= sources && sources - stable + (partial ? 1 : 0) <= 2 &&
         sources + (partial ? 1 : 0) <= kMixMaxSources;
}

bool tile_stats_eligible(int64_t rows, int64_t k, int64_t n_out) {
  return gemv_eligible(rows, k, n_out) && rows <= 16 && k <= 768;
}

bool gemv_eligible(int64_t rows, int64_t k, int64_t n_out) {
  return g_gemv_enabled && rows >= 1 && rows <= g_gemv_max_rows && k % 256 == 0 && k <= kMaxGemvK &&
         n_out % 16 == 0;
}

int gemv_launch(const GemvArgs& a, cudaStream_t stream) {
  if (a.mix_bank != nullptr) return launch_mma<1, 3, kGemvMix, false>(a, stream);  // mix_eligible() holds
  const bool k3 = a.k <= 768;  // the 768-wide model dimension: 3 blocks per warp, fewer registers
  if (a.rows <= 8) return k3 ? launch_mma_rows<1, 3>(a, stream) : launch_mma_rows<1, kMaxGemvK / 256>(a, stream);
  return k3 ? launch_mma_rows<2, 3>(a, stream) : launch_mma_rows<2, kMaxGemvK / 256>(a, stream);
}

}  // namespace aiosb
