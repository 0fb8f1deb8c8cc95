// Skinny GEMM on the 5th-generation tensor cores (tcgen05 + TMA), used for every
// linear layer of the model: the decode GEMVs (<= 8 candidate rows) and the
// prefix prefill GEMMs (13..512 rows).
//
// Operand roles are swapped ("swap AB"): the weight matrix W[n, k] is the UMMA A
// operand (M = 128 weight rows per tile) and the activations X[rows, k] are the
// B operand (N = 16..256 token columns), so D[m, t] = sum_k W[m, k] X[t, k] is
// Y^T for one 128-feature x BN-token tile. A decode step therefore streams each
// weight byte exactly once through TMA into shared memory while the token count
// only sets the (small) UMMA N.
//
// Per CTA: warp 0 lane 0 issues TMA loads into an S-stage mbarrier pipeline,
// warp 1 lane 0 issues tcgen05.mma (K = 16 per instruction, 4 per 64-wide
// stage) into a TMEM accumulator, then all four warps drain TMEM with
// tcgen05.ld. Split-K across a thread-block cluster (up to 16 CTAs along K)
// keeps ~all SMs streaming weights even for 768-row projections; the partial
// tiles are reduced deterministically through distributed shared memory.
// No TMA load uses cluster multicast: each CTA loads its own K slice.
#include <stdlib.h>
#include <string.h>

#include <algorithm>
#include <mutex>

#include "abi_util.h"
#include "gemv.h"
#include "common.cuh"

namespace aiosb {
namespace {

constexpr int kBM = 128;        // weight rows per tile (UMMA M)
constexpr int kBK = 64;         // K elements per stage (128 bytes: one swizzle atom)
constexpr int kMaxStages = 6;
constexpr int kThreads = 128;
constexpr int kMaxSplit = 16;
constexpr uint32_t kABytes = kBM * kBK * 2;  // 16 KiB

struct GemmArgs {
  int64_t rows;          // token rows of X
  int64_t n;             // weight rows
  int64_t y_row_stride;  // elements
  __nv_bfloat16* y;
  const __nv_bfloat16* residual;  // AIOSB_EPI_ADD: y = residual + bf16(x W^T)
  int64_t residual_stride;
  int32_t* status;
  int chunks_per_split;  // 64-wide K chunks handled by one CTA
  int stages;
  int split;
  int epilogue;
  // Fused RMSNorm prologue (norm != 0): the B operand is rmsnorm(nx [+ nres]) * nw,
  // computed by the CTA itself instead of loaded by TMA; nres_out <- nx + nres.
  int norm;
  int64_t k_total;
  const __nv_bfloat16* nx;
  const __nv_bfloat16* nres;
  __nv_bfloat16* nres_out;
  const __nv_bfloat16* nw;
  float neps;
  // Statistics mode (norm == 2): B = bf16(s * rcp * nw) with s = stat_x [rows, K]
  // fp32 and rcp from stat_parts partial sums of squares stat_ss[p * stat_ss_stride + row].
  const float* stat_x;
  const float* stat_ss;
  int64_t stat_ss_stride;
  int stat_parts;
  // AIOSB_EPI_ADD with out_stat_x: also store s = residual + bf16(acc) in fp32 into
  // out_stat_x [rows, n] and each 128-column tile's sum of squares of s into
  // out_stat_ss[m_tile * out_ss_stride + row].
  float* out_stat_x;
  float* out_stat_ss;
  int64_t out_ss_stride;
  // 1: launch the next kernel at entry (its weight prefetch overlaps this one);
  // 0: only once this CTA's accumulator is complete. A grid of more than one wave
  // uses 0, so that early-launched dependent CTAs (each holding an SM's shared
  // memory while it waits) do not take the SMs its later waves need.
  int early_dependents;
  // register-operand path, store epilogue: per 16-column tile statistics of the
  // output (see GemvArgs::tile_stats); the tcgen05 path does not write them
  float4* tile_stats;
  int user_early;  // AIOSB_LINEAR_EARLY_DEPENDENTS (register-operand path)
};

constexpr int kMaxNormRows = 64;
constexpr int kMaxStatParts = 256;  // sum-of-squares parts (8-column groups of n <= 2048)

template <int BN>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tm_w, const __grid_constant__ CUtensorMap tm_x,
                   const GemmArgs a) {
  constexpr uint32_t kBBytes = BN * kBK * 2;
  constexpr uint32_t kStageBytes = kABytes + kBBytes;
  constexpr uint32_t kTmemCols = BN < 32 ? 32 : BN;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const bool norm = a.norm != 0;
  const uint32_t stage_bytes = norm ? kABytes : kStageBytes;
  uint8_t* bnorm = smem + a.stages * stage_bytes;  // norm mode: every B chunk of this CTA
  const uint32_t pipe_bytes = (uint32_t)a.stages * stage_bytes + (norm ? (uint32_t)a.chunks_per_split * kBBytes : 0u);
  const uint32_t red_bytes = BN * kBM * 4;
  const uint32_t body = pipe_bytes > red_bytes ? pipe_bytes : red_bytes;
  __shared__ float rcp_s[256];  // per-token 1/rms (norm modes; BN <= 256)
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + body);
  uint64_t* empty = full + kMaxStages;
  uint64_t* accum = empty + kMaxStages;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(accum + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  float* red = reinterpret_cast<float*>(smem);  // [BN][128] fp32, reuses the pipeline buffers

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int m_tile = blockIdx.x;
  const int split_idx = blockIdx.y;
  const int n_tile = blockIdx.z;
  const int nch = a.chunks_per_split;
  const int k_chunk0 = split_idx * nch;

  if (a.early_dependents) pdl_launch_dependents();  // the next kernel may start its own weight prefetch now
  if (tid == 0) {
    for (int s = 0; s < a.stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(accum, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (tid == 32) {
    tma_prefetch_desc(&tm_w);
    tma_prefetch_desc(&tm_x);
  }
  if (warp == 0) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  // ---- weights do not depend on the previous kernel: request the first stages'
  // weight tiles before waiting on it (programmatic dependent launch).
  const int pre = nch < a.stages ? nch : a.stages;
  if (tid == 0) {
    for (int i = 0; i < pre; ++i) {
      mbar_arrive_expect_tx(&full[i], stage_bytes);
      tma_load_2d(smem + i * stage_bytes, &tm_w, &full[i], (k_chunk0 + i) * kBK, m_tile * kBM);
    }
  }
  pdl_wait();
  if (a.norm == 2) {
    // ---- RMSNorm from the producer's statistics: B = bf16(s * rcp * w), where s
    // is the fp32 residual stream the previous GEMM's ADD epilogue wrote and
    // rcp = 1 / sqrt(sum_p ss_p / K + eps) sums its per-tile partials in tile order.
    // Every load of a round is issued before any use (one L2 round trip per round);
    // with at most one unit per thread (decode) the partials ride in that round.
    const int64_t K = a.k_total;
    const int units = nch * BN * 8;
    const int P = a.stat_parts;
    const bool inline_rcp = units <= kThreads;
    if (!inline_rcp) {
      for (int t = tid; t < BN; t += kThreads) {
        const int64_t tg = (int64_t)n_tile * BN + t;
        float ss = 0.f;
        if (tg < a.rows) {
#pragma unroll 8
          for (int p = 0; p < P; ++p) ss += a.stat_ss[p * a.stat_ss_stride + tg];
        }
        rcp_s[t] = 1.0f / sqrtf(ss / (float)K + a.neps);
      }
      __syncthreads();
    }
    constexpr int kU = 4;
    for (int u0 = tid; u0 < units; u0 += kThreads * kU) {
      float4 s0[kU], s1[kU];
      uint4 wv[kU];
      float rc[kU];
#pragma unroll
      for (int j = 0; j < kU; ++j) {
        const int u = u0 + j * kThreads;
        s0[j] = make_float4(0.f, 0.f, 0.f, 0.f);
        s1[j] = s0[j];
        wv[j] = make_uint4(0u, 0u, 0u, 0u);
        rc[j] = 0.f;
        if (u < units) {
          const int i = u / (BN * 8), rem = u % (BN * 8), t = rem >> 3, c16 = rem & 7;
          const int64_t kk = (int64_t)(k_chunk0 + i) * kBK + c16 * 8;
          const int64_t tg = (int64_t)n_tile * BN + t;
          if (tg < a.rows) {
            const float4* sp = reinterpret_cast<const float4*>(a.stat_x + tg * K + kk);
            s0[j] = sp[0];
            s1[j] = sp[1];
            wv[j] = *reinterpret_cast<const uint4*>(a.nw + kk);
            if (inline_rcp) {
              float ss = 0.f;
#pragma unroll 8
              for (int p = 0; p < P; ++p) ss += a.stat_ss[p * a.stat_ss_stride + tg];
              rc[j] = 1.0f / sqrtf(ss / (float)K + a.neps);
            } else {
              rc[j] = rcp_s[t];
            }
          }
        }
      }
#pragma unroll
      for (int j = 0; j < kU; ++j) {
        const int u = u0 + j * kThreads;
        if (u < units) {
          const int i = u / (BN * 8), rem = u % (BN * 8), t = rem >> 3, c16 = rem & 7;
          const float sv[8] = {s0[j].x, s0[j].y, s0[j].z, s0[j].w, s1[j].x, s1[j].y, s1[j].z, s1[j].w};
          const uint32_t pw[4] = {wv[j].x, wv[j].y, wv[j].z, wv[j].w};
          uint32_t po[4];
#pragma unroll
          for (int q = 0; q < 4; ++q)
            po[q] = pack_bf16x2(sv[2 * q] * rc[j] * bf16_lo(pw[q]), sv[2 * q + 1] * rc[j] * bf16_hi(pw[q]));
          *reinterpret_cast<uint4*>(bnorm + (size_t)i * kBBytes + t * 128 + ((c16 ^ (t & 7)) << 4)) =
              make_uint4(po[0], po[1], po[2], po[3]);
        }
      }
    }
    // generic-proxy smem writes -> visible to the tensor core (async proxy)
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    __syncthreads();
  } else if (norm) {
    // ---- fused RMSNorm: per-row 1/rms over the full K, then this CTA's K chunks
    // of the normalised rows written straight into the UMMA B layout
    // (128-byte rows, 16-byte units swizzled by row % 8, as TMA SWIZZLE_128B).
    const int64_t K = a.k_total;
    const int nvec = (int)(K / 8);
    for (int t = warp; t < BN; t += kThreads / 32) {
      const int64_t tg = (int64_t)n_tile * BN + t;
      float ss = 0.f;
      if (tg < a.rows) {
        const uint4* xr = reinterpret_cast<const uint4*>(a.nx + tg * K);
        const uint4* rr = a.nres ? reinterpret_cast<const uint4*>(a.nres + tg * K) : nullptr;
        for (int i = lane; i < nvec; i += 32) {
          const uint4 xv = xr[i];
          const uint32_t px[4] = {xv.x, xv.y, xv.z, xv.w};
          uint32_t pr[4] = {0u, 0u, 0u, 0u};
          if (rr) {
            const uint4 rv = rr[i];
            pr[0] = rv.x; pr[1] = rv.y; pr[2] = rv.z; pr[3] = rv.w;
          }
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const float lo = bf16_lo(px[q]) + bf16_lo(pr[q]);
            const float hi = bf16_hi(px[q]) + bf16_hi(pr[q]);
            ss += lo * lo + hi * hi;
          }
        }
      }
      ss = warp_sum(ss);
      if (lane == 0) rcp_s[t] = 1.0f / sqrtf(ss / (float)K + a.neps);
    }
    __syncthreads();
    const int units = nch * BN * 8;
    for (int u = tid; u < units; u += kThreads) {
      const int i = u / (BN * 8), rem = u % (BN * 8), t = rem >> 3, c16 = rem & 7;
      const int64_t kk = (int64_t)(k_chunk0 + i) * kBK + c16 * 8;
      const int64_t tg = (int64_t)n_tile * BN + t;
      uint4 o = make_uint4(0u, 0u, 0u, 0u);
      if (tg < a.rows) {
        const uint4 xv = *reinterpret_cast<const uint4*>(a.nx + tg * K + kk);
        const uint4 wv = *reinterpret_cast<const uint4*>(a.nw + kk);
        const uint32_t px[4] = {xv.x, xv.y, xv.z, xv.w}, pw[4] = {wv.x, wv.y, wv.z, wv.w};
        uint32_t pr[4] = {0u, 0u, 0u, 0u};
        if (a.nres) {
          const uint4 rv = *reinterpret_cast<const uint4*>(a.nres + tg * K + kk);
          pr[0] = rv.x; pr[1] = rv.y; pr[2] = rv.z; pr[3] = rv.w;
        }
        const float rcp = rcp_s[t];
        uint32_t po[4], ps[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const float lo = bf16_lo(px[q]) + bf16_lo(pr[q]);
          const float hi = bf16_hi(px[q]) + bf16_hi(pr[q]);
          ps[q] = pack_bf16x2(lo, hi);
          po[q] = pack_bf16x2(lo * rcp * bf16_lo(pw[q]), hi * rcp * bf16_hi(pw[q]));
        }
        o = make_uint4(po[0], po[1], po[2], po[3]);
        if (a.nres_out != nullptr && m_tile == 0)
          *reinterpret_cast<uint4*>(a.nres_out + tg * K + kk) = make_uint4(ps[0], ps[1], ps[2], ps[3]);
      }
      *reinterpret_cast<uint4*>(bnorm + (size_t)i * kBBytes + t * 128 + ((c16 ^ (t & 7)) << 4)) = o;
    }
    // generic-proxy smem writes -> visible to the tensor core (async proxy)
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    __syncthreads();
  } else if (tid == 0) {
    for (int i = 0; i < pre; ++i)
      tma_load_2d(smem + i * stage_bytes + kABytes, &tm_x, &full[i], (k_chunk0 + i) * kBK, n_tile * BN);
  }

  if (tid == 0) {
    // ---- TMA producer for the remaining stages.
    for (int i = pre; i < nch; ++i) {
      const int s = i % a.stages;
      if (!mbar_wait(&empty[s], ((i / a.stages) & 1) ^ 1)) {
        report(a.status, AIOSB_DEV_WAIT_TIMEOUT);
        *abort_flag = 1;
        break;
      }
      mbar_arrive_expect_tx(&full[s], stage_bytes);
      tma_load_2d(smem + s * stage_bytes, &tm_w, &full[s], (k_chunk0 + i) * kBK, m_tile * kBM);
      if (!norm)
        tma_load_2d(smem + s * stage_bytes + kABytes, &tm_x, &full[s], (k_chunk0 + i) * kBK, n_tile * BN);
    }
  } else if (tid == 32) {
    // ---- MMA issuer.
    constexpr uint32_t idesc = umma_idesc_bf16(kBM, BN);
    bool ok = true;
    for (int i = 0; i < nch; ++i) {
      const int s = i % a.stages;
      if (!mbar_wait(&full[s], (i / a.stages) & 1)) {
        report(a.status, AIOSB_DEV_WAIT_TIMEOUT);
        *abort_flag = 1;
        ok = false;
        break;
      }
      tc_fence_after();
      const uint32_t a_base = smem_u32(smem + s * stage_bytes);
      const uint32_t b_base = norm ? smem_u32(bnorm + (size_t)i * kBBytes) : a_base + kABytes;
#pragma unroll
      for (int kk = 0; kk < kBK / 16; ++kk) {
        tc_mma_bf16(tmem, umma_desc_sw128(a_base + kk * 32), umma_desc_sw128(b_base + kk * 32), idesc,
                    (i | kk) != 0 ? 1u : 0u);
      }
      tc_commit(&empty[s]);
    }
    if (ok) tc_commit(accum);
  }

  // ---- Epilogue: TMEM -> registers -> shared [BN][128] fp32.
  bool have = mbar_wait(accum, 0);
  if (!have) {
    report(a.status, AIOSB_DEV_WAIT_TIMEOUT);
    *abort_flag = 1;
  }
  if (!a.early_dependents) pdl_launch_dependents();
  // tcgen05.ld is warp-collective (.sync.aligned): reconverge and agree first.
  __syncwarp();
  have = __all_sync(0xffffffffu, have);
  tc_fence_after();
  if (have) {
    // two 16-column loads in flight per wait
#pragma unroll
    for (int cb = 0; cb < BN / 16; cb += 2) {
      float v[2][16];
      tmem_ld16(tmem + ((uint32_t)(32 * warp) << 16) + (uint32_t)(cb * 16), v[0]);
      if (cb + 1 < BN / 16) tmem_ld16(tmem + ((uint32_t)(32 * warp) << 16) + (uint32_t)((cb + 1) * 16), v[1]);
      tc_wait_ld();
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        if (cb + h < BN / 16) {
#pragma unroll
          for (int j = 0; j < 16; ++j) red[((cb + h) * 16 + j) * kBM + 32 * warp + lane] = v[h][j];
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  const int split = a.split;
  if (split > 1) cluster_sync();

  // ---- Reduction over the cluster's K splits + fused epilogue. CTA rank r
  // owns token columns c with c % split == r; every column is summed over the
  // ranks in rank order, so results do not depend on scheduling.
  const bool ok_all = (*abort_flag == 0);
  if (ok_all) {
    const uint32_t rank = split > 1 ? cluster_ctarank() : 0u;
    const uint32_t red_addr = smem_u32(red);
    const int64_t t0 = (int64_t)n_tile * BN;
    // One unit per thread per iteration, four iterations unrolled so that their
    // partial-tile reads (local, or a peer's over distributed shared memory) are
    // in flight together; every unit sums the ranks in rank order. (An earlier
    // form that batched units through arrays and per-unit liveness flags ran
    // the split-1 epilogue of a 256-token tile in 8.2 us instead of 2.4 us.)
    auto part = [&](uint32_t off, int q) -> float4 {
      if (split > 1) return ld_dsmem_f4(map_shared_rank(red_addr + off, (uint32_t)q));
      return *reinterpret_cast<const float4*>(reinterpret_cast<const uint8_t*>(red) + off);
    };
    if (a.epilogue == AIOSB_EPI_STORE || a.epilogue == AIOSB_EPI_ADD) {
      // unit u: column c = (u / 32) * split + rank (a token; rank r owns the
      // columns c % split == r), tile rows m4 * 4 .. m4 * 4 + 3
      const int own = (BN + split - 1 - (int)rank) / split;
#pragma unroll 4
      for (int u = tid; u < own * 32; u += kThreads) {
        const int c = (u >> 5) * split + (int)rank, m4 = u & 31;
        const int64_t t = t0 + c;
        if (t < a.rows) {  // warp-uniform: a warp's 32 units share a column
          const uint32_t off = (uint32_t)((c * kBM + m4 * 4) * 4);
          float4 v = part(off, 0);
          for (int q = 1; q < split; ++q) {
            const float4 p = part(off, q);
            v.x += p.x; v.y += p.y; v.z += p.z; v.w += p.w;
          }
          __nv_bfloat16* dst = a.y + t * a.y_row_stride + (int64_t)m_tile * kBM + m4 * 4;
          if (a.epilogue == AIOSB_EPI_ADD) {
            // residual + delta with the delta rounded to bf16 first, as the
            // reference's bf16 `partial + delta` (aios/models/minimind_ime.py:237-252).
            const uint2 rv = *reinterpret_cast<const uint2*>(a.residual + t * a.residual_stride +
                                                            (int64_t)m_tile * kBM + m4 * 4);
            v.x = bf16_lo(rv.x) + round_bf16(v.x);
            v.y = bf16_hi(rv.x) + round_bf16(v.y);
            v.z = bf16_lo(rv.y) + round_bf16(v.z);
            v.w = bf16_hi(rv.y) + round_bf16(v.w);
            if (a.out_stat_x != nullptr) {
              // one warp owns column c: its 32 lanes cover the tile's 128 rows
              *reinterpret_cast<float4*>(a.out_stat_x + t * a.n + (int64_t)m_tile * kBM + m4 * 4) = v;
              float ss = v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
              ss = warp_sum(ss);
              if (lane == 0) a.out_stat_ss[(int64_t)m_tile * a.out_ss_stride + t] = ss;
            }
          }
          *reinterpret_cast<uint2*>(dst) = make_uint2(pack_bf16x2(v.x, v.y), pack_bf16x2(v.z, v.w));
        }
      }
    } else {
      // SILU_MUL: tile rows 0..63 are gate rows, 64..127 the matching up rows;
      // unit u: column c = (u / 16) * split + rank, 4 gate rows m4 * 4 .. and their up rows
      const int own = (BN + split - 1 - (int)rank) / split;
#pragma unroll 4
      for (int u = tid; u < own * 16; u += kThreads) {
        const int c = (u >> 4) * split + (int)rank, m4 = u & 15;
        const int64_t t = t0 + c;
        if (t < a.rows) {
          const uint32_t og = (uint32_t)((c * kBM + m4 * 4) * 4), ou = og + 64 * 4;
          float4 g = part(og, 0), up = part(ou, 0);
          for (int q = 1; q < split; ++q) {
            const float4 pg = part(og, q), pu = part(ou, q);
            g.x += pg.x; g.y += pg.y; g.z += pg.z; g.w += pg.w;
            up.x += pu.x; up.y += pu.y; up.z += pu.z; up.w += pu.w;
          }
          // gate_up output is bf16 before silu_and_mul (aios/models/qwen3.py:90-92).
          const float gv[4] = {round_bf16(g.x), round_bf16(g.y), round_bf16(g.z), round_bf16(g.w)};
          const float uv[4] = {round_bf16(up.x), round_bf16(up.y), round_bf16(up.z), round_bf16(up.w)};
          float r[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) r[e] = gv[e] / (1.0f + expf(-gv[e])) * uv[e];
          __nv_bfloat16* dst = a.y + t * a.y_row_stride + (int64_t)m_tile * (kBM / 2) + m4 * 4;
          *reinterpret_cast<uint2*>(dst) = make_uint2(pack_bf16x2(r[0], r[1]), pack_bf16x2(r[2], r[3]));
        }
      }
    }
  }
  if (split > 1) cluster_sync();  // peers may still read this CTA's partial tile
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

// ---- host side -------------------------------------------------------------
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

// 2-D bf16 tensor map over a row-major [rows, cols] matrix, box [box_rows, 64].
int make_map(CUtensorMap* m, const void* base, int64_t rows, int64_t cols, uint32_t box_rows) {
  EncodeTiledFn fn = encode_fn();
  if (fn == nullptr) return set_error(AIOSB_ERR_LAUNCH, "cuTensorMapEncodeTiled unavailable");
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)cols * 2};
  cuuint32_t box[2] = {(cuuint32_t)kBK, box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(AIOSB_ERR_LAUNCH, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return AIOSB_OK;
}

constexpr int max_stages_for(int bn) { return bn >= 256 ? 4 : bn >= 128 ? 5 : kMaxStages; }

template <int BN>
size_t smem_bytes(int stages, bool norm = false, int chunks = 0) {
  const size_t pipe = norm ? (size_t)stages * kABytes + (size_t)chunks * BN * kBK * 2
                           : (size_t)stages * (kABytes + BN * kBK * 2);
  const size_t red = (size_t)BN * kBM * 4;
  return std::max(pipe, red) + 1024 /*alignment*/ + 512 /*barriers*/;
}

constexpr int kMaxDynSmem = 227 * 1024 - 2048;  // opt-in limit minus the static rcp table

template <int BN>
int launch_gemm(const CUtensorMap& tw, const CUtensorMap& tx, GemmArgs a, int m_tiles, int n_tiles,
                cudaStream_t stream) {
  static bool configured[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  auto kern = gemm_tc_kernel<BN>;
  if (dev >= 0 && dev < 64 && !configured[dev]) {
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kMaxDynSmem);
    cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
    configured[dev] = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)m_tiles, (unsigned)a.split, (unsigned)n_tiles);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem_bytes<BN>(a.stages, a.norm != 0, a.chunks_per_split);
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  attr[1].id = cudaLaunchAttributeClusterDimension;
  attr[1].val.clusterDim.x = 1;
  attr[1].val.clusterDim.y = (unsigned)a.split;
  attr[1].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  cudaError_t e = cudaLaunchKernelEx(&cfg, kern, tw, tx, a);
  if (e != cudaSuccess) return set_error(AIOSB_ERR_LAUNCH, "linear: %s", cudaGetErrorString(e));
  return AIOSB_OK;
}

// Split-K factor: the largest divisor of the K chunk count (<= 16) that keeps
// the grid within one wave of CTAs.
// Largest split-K cluster; AIOSB_GEMM_MAX_SPLIT (1..16) lowers it, and it drops
// to 8 by itself if 16-CTA clusters cannot launch on the device.
int g_max_split = [] {
  const char* env = getenv("AIOSB_GEMM_MAX_SPLIT");
  const int v = env ? atoi(env) : kMaxSplit;
  return v >= 1 && v <= kMaxSplit ? v : kMaxSplit;
}();

int choose_split(int64_t tiles, int64_t chunks, int sms) {
  int best = 1;
  for (int d = 2; d <= g_max_split; ++d)
    if (chunks % d == 0 && tiles * d <= sms) best = d;
  return best;
}

}  // namespace
}  // namespace aiosb

using namespace aiosb;

namespace aiosb {
namespace {

int linear_impl(GemmArgs a, const void* x, int64_t rows, int64_t k, const void* w, int64_t n, void* stream) {
  int bn = rows <= 16 ? 16 : rows <= 32 ? 32 : rows <= 64 ? 64 : rows <= 128 ? 128 : 256;
  const int64_t m_tiles = n / kBM;
  int64_t n_tiles = (rows + bn - 1) / bn;
  const int64_t chunks = k / kBK;
  a.rows = rows;
  a.n = n;
  a.k_total = k;
  const int64_t n_out = a.epilogue == AIOSB_EPI_SILU_MUL ? n / 2 : n;
  if (a.norm != 1 && gemv_eligible(rows, k, n_out)) {
    // decode widths: register-operand MMA GEMV (weights requested before the dependency wait)
    GemvArgs g;
    memset(&g, 0, sizeof(g));
    g.x = (const __nv_bfloat16*)x;
    g.x_stride = k;
    g.stat_x = a.norm == 2 ? a.stat_x : nullptr;
    g.nw = a.nw;
    g.eps = a.neps;
    g.w = (const __nv_bfloat16*)w;
    g.n = n;
    g.n_out = n_out;
    g.k = k;
    g.rows = (int)rows;
    g.y = a.y;
    g.y_stride = a.y_row_stride;
    g.epilogue = a.epilogue;
    g.residual = a.residual;
    g.residual_stride = a.residual_stride;
    g.out_stat_x = a.out_stat_x;
    g.out_stat_ss = a.out_stat_ss;
    g.out_ss_stride = a.out_ss_stride;
    g.tile_stats = a.tile_stats;
    g.early_dependents = a.user_early;
    return gemv_launch(g, as_stream(stream));
  }
  auto plan = [&]() {
    a.split = choose_split(m_tiles * n_tiles, chunks, sm_count());
    a.chunks_per_split = (int)(chunks / a.split);
    a.stages = std::min(a.chunks_per_split, max_stages_for(bn));
    // keep the norm-mode B buffer + weight stages inside the shared-memory budget
    while (a.norm && a.stages > 1 &&
           (size_t)a.stages * kABytes + (size_t)a.chunks_per_split * bn * kBK * 2 + 2048 > (size_t)kMaxDynSmem)
      --a.stages;
  };
  // norm modes keep every B chunk of the CTA in shared memory: narrower token
  // tiles (more of them, so fewer K chunks per CTA) until one weight stage fits
  auto norm_fits = [&]() {
    return (size_t)a.stages * kABytes + (size_t)a.chunks_per_split * bn * kBK * 2 + 2048 <= (size_t)kMaxDynSmem;
  };
  auto plan_all = [&]() {
    plan();
    while (a.norm && !norm_fits() && bn > 16) {
      bn /= 2;
      n_tiles = (rows + bn - 1) / bn;
      plan();
    }
    a.early_dependents = m_tiles * n_tiles * a.split <= sm_count() ? 1 : 0;
  };
  plan_all();
  AIOSB_REQUIRE(!a.norm || norm_fits(), AIOSB_ERR_UNSUPPORTED, "linear: normalised operand of k=%lld too large",
                (long long)k);
  CUtensorMap tw, tx;
  int rc = make_map(&tw, w, n, k, kBM);
  if (rc) return rc;
  if (!a.norm) {
    rc = make_map(&tx, x, rows, k, (uint32_t)bn);
    if (rc) return rc;
  } else {
    tx = tw;  // unused in norm mode
  }
  cudaStream_t s = as_stream(stream);
  auto launch = [&]() {
    switch (bn) {
      case 16: return launch_gemm<16>(tw, tx, a, (int)m_tiles, (int)n_tiles, s);
      case 32: return launch_gemm<32>(tw, tx, a, (int)m_tiles, (int)n_tiles, s);
      case 64: return launch_gemm<64>(tw, tx, a, (int)m_tiles, (int)n_tiles, s);
      case 128: return launch_gemm<128>(tw, tx, a, (int)m_tiles, (int)n_tiles, s);
      default: return launch_gemm<256>(tw, tx, a, (int)m_tiles, (int)n_tiles, s);
    }
  };
  rc = launch();
  if (rc != AIOSB_OK && a.split > 8) {
    // Non-portable 16-CTA clusters are an opt-in; fall back to portable sizes.
    (void)cudaGetLastError();
    g_max_split = 8;
    plan_all();
    rc = launch();
  }
  return rc;
}

int check_common(const void* w, int64_t rows, int64_t k, int64_t n, void* y, int64_t y_row_stride, int epilogue,
                 const void* residual, int64_t residual_stride) {
  epilogue &= ~AIOSB_LINEAR_EARLY_DEPENDENTS;
  AIOSB_REQUIRE(rows >= 0 && k > 0 && n > 0, AIOSB_ERR_INVALID_ARG, "linear: bad sizes");
  AIOSB_REQUIRE(n % kBM == 0, AIOSB_ERR_UNSUPPORTED, "linear: n=%lld must be a multiple of 128", (long long)n);
  AIOSB_REQUIRE(k % kBK == 0, AIOSB_ERR_UNSUPPORTED, "linear: k=%lld must be a multiple of 64", (long long)k);
  AIOSB_REQUIRE(epilogue == AIOSB_EPI_STORE || epilogue == AIOSB_EPI_SILU_MUL || epilogue == AIOSB_EPI_ADD,
                AIOSB_ERR_INVALID_ARG, "linear: unknown epilogue %d", epilogue);
  AIOSB_REQUIRE(epilogue != AIOSB_EPI_ADD ||
                    (residual != nullptr && aligned16(residual) && residual_stride >= n && residual_stride % 8 == 0),
                AIOSB_ERR_INVALID_ARG, "linear: the add epilogue needs an aligned residual [rows, >= n]");
  const int64_t y_cols = epilogue == AIOSB_EPI_SILU_MUL ? n / 2 : n;
  AIOSB_REQUIRE(y_row_stride >= y_cols && y_row_stride % 8 == 0, AIOSB_ERR_INVALID_ARG,
                "linear: y row stride must cover the output and be a multiple of 8");
  if (rows == 0) return 1;
  AIOSB_REQUIRE(w && y, AIOSB_ERR_INVALID_ARG, "linear: null pointer");
  AIOSB_REQUIRE(aligned16(w) && aligned16(y), AIOSB_ERR_MISALIGNED, "linear: w and y must be 16-byte aligned");
  return AIOSB_OK;
}

GemmArgs base_args(void* y, int64_t y_row_stride, int epilogue, const void* residual, int64_t residual_stride,
                   int32_t* status) {
  GemmArgs a;
  memset(&a, 0, sizeof(a));
  a.user_early = (epilogue & AIOSB_LINEAR_EARLY_DEPENDENTS) ? 1 : 0;
  epilogue &= ~AIOSB_LINEAR_EARLY_DEPENDENTS;
  a.y_row_stride = y_row_stride;
  a.y = (__nv_bfloat16*)y;
  a.residual = (const __nv_bfloat16*)residual;
  a.residual_stride = residual_stride;
  a.status = status;
  a.epilogue = epilogue;
  return a;
}

}  // namespace
}  // namespace aiosb

extern "C" int aiosb_linear(const void* x, int64_t rows, int64_t k, const void* w, int64_t n, void* y,
                            int64_t y_row_stride, int epilogue, const void* residual, int64_t residual_stride,
                            int32_t* status, void* stream) {
  int rc = check_common(w, rows, k, n, y, y_row_stride, epilogue, residual, residual_stride);
  if (rc != AIOSB_OK) return rc == 1 ? AIOSB_OK : rc;
  AIOSB_REQUIRE(x && aligned16(x), AIOSB_ERR_MISALIGNED, "linear: x must be a 16-byte aligned pointer");
  return linear_impl(base_args(y, y_row_stride, epilogue, residual, residual_stride, status), x, rows, k, w, n,
                     stream);
}

extern "C" int aiosb_linear_rmsnorm(const void* x, const void* res, void* res_out, const void* norm_w, float eps,
                                    int64_t rows, int64_t k, const void* w, int64_t n, void* y, int64_t y_row_stride,
                                    int epilogue, const void* residual, int64_t residual_stride, int32_t* status,
                                    void* stream) {
  int rc = check_common(w, rows, k, n, y, y_row_stride, epilogue, residual, residual_stride);
  if (rc != AIOSB_OK) return rc == 1 ? AIOSB_OK : rc;
  AIOSB_REQUIRE(rows <= kMaxNormRows, AIOSB_ERR_UNSUPPORTED, "linear_rmsnorm: at most %d rows", kMaxNormRows);
  AIOSB_REQUIRE(x && norm_w && aligned16(x) && aligned16(norm_w) && (res == nullptr || aligned16(res)) &&
                    (res_out == nullptr || aligned16(res_out)),
                AIOSB_ERR_MISALIGNED, "linear_rmsnorm: x / res / res_out / norm_w must be 16-byte aligned");
  AIOSB_REQUIRE(res_out == nullptr || (res_out != res && res_out != x), AIOSB_ERR_INVALID_ARG,
                "linear_rmsnorm: res_out must not alias x or res (other CTAs still read them)");
  GemmArgs a = base_args(y, y_row_stride, epilogue, residual, residual_stride, status);
  a.norm = 1;
  a.nx = (const __nv_bfloat16*)x;
  a.nres = (const __nv_bfloat16*)res;
  a.nres_out = (__nv_bfloat16*)res_out;
  a.nw = (const __nv_bfloat16*)norm_w;
  a.neps = eps;
  return linear_impl(a, x, rows, k, w, n, stream);
}

extern "C" int aiosb_linear_add_stat(const void* x, int64_t rows, int64_t k, const void* w, int64_t n, void* y,
                                     int64_t y_row_stride, const void* residual, int64_t residual_stride,
                                     float* stat_x, float* stat_ss, int64_t stat_ss_stride, int64_t* stat_parts,
                                     int32_t* status, void* stream) {
  if (stat_parts != nullptr)
    *stat_parts = gemv_eligible(rows, k, n) ? n / kGemvStatGroup : n / kBM;
  int rc = check_common(w, rows, k, n, y, y_row_stride, AIOSB_EPI_ADD, residual, residual_stride);
  if (rc != AIOSB_OK) return rc == 1 ? AIOSB_OK : rc;
  AIOSB_REQUIRE(x && aligned16(x), AIOSB_ERR_MISALIGNED, "linear_add_stat: x must be a 16-byte aligned pointer");
  AIOSB_REQUIRE(stat_x && stat_ss && aligned16(stat_x), AIOSB_ERR_MISALIGNED,
                "linear_add_stat: stat_x must be a 16-byte aligned pointer and stat_ss non-null");
  AIOSB_REQUIRE(stat_ss_stride >= rows, AIOSB_ERR_INVALID_ARG, "linear_add_stat: stat_ss stride below rows");
  AIOSB_REQUIRE(n / kGemvStatGroup <= kMaxStatParts, AIOSB_ERR_UNSUPPORTED, "linear_add_stat: n above %d",
                kMaxStatParts * kGemvStatGroup);
  GemmArgs a = base_args(y, y_row_stride, AIOSB_EPI_ADD, residual, residual_stride, status);
  a.out_stat_x = stat_x;
  a.out_stat_ss = stat_ss;
  a.out_ss_stride = stat_ss_stride;
  return linear_impl(a, x, rows, k, w, n, stream);
}

extern "C" int aiosb_linear_stat_norm(const float* stat_x, const float* stat_ss, int64_t stat_ss_stride,
                                      int64_t parts, const void* norm_w, float eps, int64_t rows, int64_t k,
                                      const void* w, int64_t n, void* y, int64_t y_row_stride, int epilogue,
                                      const void* residual, int64_t residual_stride, int32_t* status,
                                      void* stream) {
  int rc = check_common(w, rows, k, n, y, y_row_stride, epilogue, residual, residual_stride);
  if (rc != AIOSB_OK) return rc == 1 ? AIOSB_OK : rc;
  AIOSB_REQUIRE(parts >= 1 && parts <= kMaxStatParts, AIOSB_ERR_INVALID_ARG,
                "linear_stat_norm: parts must be in [1, %d]", kMaxStatParts);
  AIOSB_REQUIRE(stat_ss_stride >= rows, AIOSB_ERR_INVALID_ARG, "linear_stat_norm: stat_ss stride below rows");
  AIOSB_REQUIRE(stat_x && stat_ss && norm_w && aligned16(stat_x) && aligned16(norm_w), AIOSB_ERR_MISALIGNED,
                "linear_stat_norm: stat_x and norm_w must be 16-byte aligned, stat_ss non-null");
  GemmArgs a = base_args(y, y_row_stride, epilogue, residual, residual_stride, status);
  a.norm = 2;
  a.stat_x = stat_x;
  a.stat_ss = stat_ss;
  a.stat_ss_stride = stat_ss_stride;
  a.stat_parts = (int)parts;
  a.nw = (const __nv_bfloat16*)norm_w;
  a.neps = eps;
  return linear_impl(a, nullptr, rows, k, w, n, stream);
}

extern "C" int aiosb_linear_tile_stats_eligible(int64_t rows, int64_t k, int64_t n) {
  return tile_stats_eligible(rows, k, n) ? 1 : 0;
}

extern "C" int aiosb_linear_tiles(const void* x, int64_t rows, int64_t k, const void* w, int64_t n, void* y,
                                  int64_t y_row_stride, float* tile_stats, int32_t* status, void* stream) {
  AIOSB_REQUIRE(tile_stats != nullptr && aligned16(tile_stats), AIOSB_ERR_MISALIGNED,
                "linear_tiles: tile_stats must be 16-byte aligned");
  AIOSB_REQUIRE(tile_stats_eligible(rows, k, n), AIOSB_ERR_UNSUPPORTED,
                "linear_tiles: only on the register-operand path with rows <= 16, k <= 768, k %% 256 == 0");
  int rc = check_common(w, rows, k, n, y, y_row_stride, AIOSB_EPI_STORE, nullptr, 0);
  if (rc != AIOSB_OK) return rc == 1 ? AIOSB_OK : rc;
  AIOSB_REQUIRE(x && aligned16(x), AIOSB_ERR_MISALIGNED, "linear_tiles: x must be a 16-byte aligned pointer");
  GemmArgs a = base_args(y, y_row_stride, AIOSB_EPI_STORE, nullptr, 0, status);
  a.tile_stats = reinterpret_cast<float4*>(tile_stats);
  return linear_impl(a, x, rows, k, w, n, stream);
}

extern "C" int aiosb_linear_stat_norm_tiles(const float* stat_x, const float* stat_ss, int64_t stat_ss_stride,
                                            int64_t parts, const void* norm_w, float eps, int64_t rows, int64_t k,
                                            const void* w, int64_t n, void* y, int64_t y_row_stride,
                                            float* tile_stats, int32_t* status, void* stream) {
  AIOSB_REQUIRE(tile_stats != nullptr && aligned16(tile_stats), AIOSB_ERR_MISALIGNED,
                "linear_stat_norm_tiles: tile_stats must be 16-byte aligned");
  AIOSB_REQUIRE(tile_stats_eligible(rows, k, n), AIOSB_ERR_UNSUPPORTED,
                "linear_stat_norm_tiles: only on the register-operand path with rows <= 16, k <= 768, k %% 256 == 0");
  int rc = check_common(w, rows, k, n, y, y_row_stride, AIOSB_EPI_STORE, nullptr, 0);
  if (rc != AIOSB_OK) return rc == 1 ? AIOSB_OK : rc;
  AIOSB_REQUIRE(parts >= 1 && parts <= kMaxStatParts, AIOSB_ERR_INVALID_ARG,
                "linear_stat_norm_tiles: parts must be in [1, %d]", kMaxStatParts);
  AIOSB_REQUIRE(stat_ss_stride >= rows, AIOSB_ERR_INVALID_ARG, "linear_stat_norm_tiles: stat_ss stride below rows");
  AIOSB_REQUIRE(stat_x && stat_ss && norm_w && aligned16(stat_x) && aligned16(norm_w), AIOSB_ERR_MISALIGNED,
                "linear_stat_norm_tiles: stat_x and norm_w must be 16-byte aligned, stat_ss non-null");
  GemmArgs a = base_args(y, y_row_stride, AIOSB_EPI_STORE, nullptr, 0, status);
  a.norm = 2;
  a.stat_x = stat_x;
  a.stat_ss = stat_ss;
  a.stat_ss_stride = stat_ss_stride;
  a.stat_parts = (int)parts;
  a.nw = (const __nv_bfloat16*)norm_w;
  a.neps = eps;
  a.tile_stats = reinterpret_cast<float4*>(tile_stats);
  return linear_impl(a, nullptr, rows, k, w, n, stream);
}

extern "C" int aiosb_linear_attnres_rmsnorm(const void* bank, int64_t sources, int64_t stable_sources,
                                            int64_t tokens, const void* partial, const float* weighted_query,
                                            float mix_eps, const void* norm_w, float norm_eps, const void* w,
                                            int64_t n, int64_t k, void* y, int64_t y_row_stride, int epilogue,
                                            int32_t* status, void* stream) {
  AIOSB_REQUIRE(epilogue == AIOSB_EPI_STORE || epilogue == AIOSB_EPI_SILU_MUL, AIOSB_ERR_INVALID_ARG,
                "linear_attnres_rmsnorm: store or SwiGLU epilogue");
  AIOSB_REQUIRE(n > 0 && n % 128 == 0, AIOSB_ERR_UNSUPPORTED, "linear_attnres_rmsnorm: n must be a multiple of 128");
  const int64_t n_out = epilogue == AIOSB_EPI_SILU_MUL ? n / 2 : n;
  AIOSB_REQUIRE(mix_eligible(tokens, k, n_out, sources, stable_sources, partial != nullptr), AIOSB_ERR_UNSUPPORTED,
                "linear_attnres_rmsnorm: 1..8 rows, k == %d, <= %d sources with at most two read after the wait",
                kMixMaxK, kMixMaxSources);
  AIOSB_REQUIRE(bank && weighted_query && norm_w && w && y, AIOSB_ERR_INVALID_ARG,
                "linear_attnres_rmsnorm: null pointer");
  AIOSB_REQUIRE(aligned16(bank) && aligned16(norm_w) && aligned16(w) && aligned16(y) &&
                    (partial == nullptr || aligned16(partial)) && y_row_stride >= n_out && y_row_stride % 8 == 0,
                AIOSB_ERR_MISALIGNED, "linear_attnres_rmsnorm: 16-byte aligned operands and output rows");
  GemvArgs g;
  memset(&g, 0, sizeof(g));
  g.nw = (const __nv_bfloat16*)norm_w;
  g.eps = norm_eps;
  g.w = (const __nv_bfloat16*)w;
  g.n = n;
  g.n_out = n_out;
  g.k = k;
  g.rows = (int)tokens;
  g.y = (__nv_bfloat16*)y;
  g.y_stride = y_row_stride;
  g.epilogue = epilogue;
  g.mix_bank = (const __nv_bfloat16*)bank;
  g.mix_partial = (const __nv_bfloat16*)partial;
  g.mix_wq = weighted_query;
  g.mix_eps = mix_eps;
  g.mix_sources = (int)sources;
  g.mix_stable = (int)stable_sources;
  g.mix_tokens = tokens;
  (void)status;
  return gemv_launch(g, as_stream(stream));
}
