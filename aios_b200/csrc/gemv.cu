// Decode-width linears: y = x W^T for at most 16 token rows on the CUDA cores.
//
// At 8 candidate rows a decode linear is a weight stream with 8 dot products per
// weight element: it is bound by HBM bandwidth and by the dependency chain of
// the step, not by math. This kernel family keeps that chain short:
//   * one warp owns one output feature (SwiGLU: its gate and up rows); its weight
//     slice (K/32 elements per lane, 16-byte loads) is requested into registers
//     before griddepcontrol.wait, i.e. while the previous kernel still runs;
//   * after the wait the CTA stages the activations in shared memory with one
//     round of loads: the bf16 rows themselves, or (statistics mode) rows
//     normalised from the fp32 residual stream s, each warp computing the sum of
//     squares of whole token rows itself (RMSNormFused, aios/layers/norm.py:34-40);
//   * fp32 dot products, a warp butterfly reduction, and the epilogues of the
//     tcgen05 GEMM (store, SwiGLU on the 64-row interleaved gate/up layout,
//     residual add with optional fp32 statistics), written 16 bytes per token.
// Rounding points equal the tcgen05 path: fp32 accumulation, bf16 output, the
// gate/up values rounded to bf16 before SwiGLU, the delta rounded before the
// residual add. Summation order differs (fp32), so results agree to rounding.
#include <algorithm>

#include "abi_util.h"
#include "common.cuh"
#include "gemv.h"

namespace aiosb {
namespace {

constexpr int kGemvThreads = 256;           // 8 warps = 8 output features per CTA
constexpr int kGemvFeat = kGemvThreads / 32;

// Reduce-scatter over the lane bits 4 and 3 (the 4 lanes l, l^8, l^16, l^24):
// afterwards lane l holds V/4 partial sums, of the value indices
// [q0, q0 + V/4) with q0 = ((l >> 4) & 1) * V/2 + ((l >> 3) & 1) * V/4.
template <int V>
__device__ __forceinline__ void reduce_scatter_34(float (&v)[V]) {
  const int lane = threadIdx.x & 31;
  {
    const bool upper = (lane & 16) != 0;
#pragma unroll
    for (int i = 0; i < V / 2; ++i) {
      const float send = upper ? v[i] : v[i + V / 2];
      const float keep = upper ? v[i + V / 2] : v[i];
      v[i] = keep + __shfl_xor_sync(0xffffffffu, send, 16);
    }
  }
  {
    const bool upper = (lane & 8) != 0;
#pragma unroll
    for (int i = 0; i < V / 4; ++i) {
      const float send = upper ? v[i] : v[i + V / 4];
      const float keep = upper ? v[i + V / 4] : v[i];
      v[i] = keep + __shfl_xor_sync(0xffffffffu, send, 8);
    }
  }
}

// NR weight rows per feature (2: SwiGLU gate + up), TMAX token rows (the operand
// is zero-padded to TMAX, so every loop over tokens is fixed-length), KC 16-byte
// weight vectors per lane and row (K / 256). STAT: the operand is normalised from
// the fp32 residual statistics instead of read as bf16 rows.
//
// A CTA computes 8 features; K is cut into 32 sub-slices of K/32: warp w takes
// sub-slices 4w..4w+3 and lane l the sub-slice 4w + l/8 of feature l % 8, so the
// 8 lanes of a sub-slice read the same operand address (a broadcast) and the
// per-lane work is K/32 elements x tokens. Partial sums: reduce-scatter over the
// 4 lanes of a feature, then over the 8 warps in warp order through shared memory.
// The operand rows are fp32 in shared memory (bf16 values, converted once), each
// K/32 sub-slice padded by 16 bytes so the 4 sub-slices a warp reads hit distinct
// banks. The CTA walks the 8-feature groups blockIdx.x, blockIdx.x + gridDim.x, ...;
// the next group's weights are in flight while the current one is computed.
template <int NR, int TMAX, int KC, bool STAT>
__global__ void __launch_bounds__(kGemvThreads) gemv_kernel(const GemvArgs a) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  float* xs = reinterpret_cast<float*>(smem_raw);  // [TMAX][32][K/32 + 4] fp32 operand rows
  constexpr int V = NR * TMAX;                      // partial sums per lane
  __shared__ float part[kGemvFeat][kGemvFeat][V];   // [warp][feature][value]
  __shared__ float accs[kGemvFeat][V];              // [feature][value]
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int K = (int)a.k;
  const int kc = K / 256;
  const int sub = K / 32;       // elements per sub-slice
  const int sstr = sub + 4;     // padded sub-slice stride (floats)
  const int rstr = 32 * sstr;   // padded row stride (floats)
  const int T = a.rows;
  const int ngroups = (int)(a.n_out / kGemvFeat);
  const int feat = lane & 7;                // feature within the group
  const int q = warp * 4 + (lane >> 3);     // K sub-slice of this lane

  // ---- weights (independent of the previous kernel) are requested before the wait
  auto load_w = [&](int grp, uint4 (&wv)[NR][KC]) {
    const int f = grp * kGemvFeat + feat;
    int64_t wrow[NR];
    if (NR == 2) {  // packed [g0..63 | u0..63 | g64..] rows of the SwiGLU epilogue
      wrow[0] = (int64_t)(f / 64) * 128 + (f % 64);
      wrow[NR - 1] = wrow[0] + 64;
    } else {
      wrow[0] = f;
    }
#pragma unroll
    for (int r = 0; r < NR; ++r)
#pragma unroll
      for (int c = 0; c < KC; ++c)
        wv[r][c] = (grp < ngroups && c < kc)
                       ? *reinterpret_cast<const uint4*>(a.w + wrow[r] * K + (int64_t)q * sub + c * 8)
                       : make_uint4(0u, 0u, 0u, 0u);
  };
  uint4 wv[NR][KC];
  load_w(blockIdx.x, wv);
  pdl_wait();
  // the next kernel launches once this one has its inputs: letting every kernel
  // launch its successor on entry ran the chain many kernels ahead, whose weight
  // prefetches then competed with this kernel's operand loads (measured:
  // 5.83 -> 5.70 ms per keystroke)
  pdl_launch_dependents();

  // ---- operand rows into shared memory (rows T..TMAX-1 zero)
  const int kv = K / 8;  // 8-element vectors per row; one never straddles a sub-slice
  auto xs_at = [&](int t, int k) { return xs + (int64_t)t * rstr + (k / sub) * sstr + (k % sub); };
  if (!STAT) {
    for (int v = tid; v < TMAX * kv; v += kGemvThreads) {
      const int t = v / kv, k = (v % kv) * 8;
      const uint4 x = t < T ? *reinterpret_cast<const uint4*>(a.x + (int64_t)t * a.x_stride + k)
                            : make_uint4(0u, 0u, 0u, 0u);
      float4* d = reinterpret_cast<float4*>(xs_at(t, k));
      d[0] = make_float4(bf16_lo(x.x), bf16_hi(x.x), bf16_lo(x.y), bf16_hi(x.y));
      d[1] = make_float4(bf16_lo(x.z), bf16_hi(x.z), bf16_lo(x.w), bf16_hi(x.w));
    }
  } else {
    // warp w normalises tokens w, w + 8: sum of squares of its fp32 row s, then
    // bf16(s * rcp * norm_w) as RMSNormFused does (stored as the fp32 value of the
    // bf16). All loads of a row are in flight before the first use.
    for (int t = warp; t < TMAX; t += kGemvFeat) {
      float4 s0[KC], s1[KC];
      uint4 nw[KC];
      const float* srow = a.stat_x + (int64_t)t * K;
#pragma unroll
      for (int j = 0; j < KC; ++j) {
        const int c8 = 32 * j + lane;
        const bool ok = t < T && j < kc;
        s0[j] = ok ? reinterpret_cast<const float4*>(srow)[2 * c8] : make_float4(0.f, 0.f, 0.f, 0.f);
        s1[j] = ok ? reinterpret_cast<const float4*>(srow)[2 * c8 + 1] : make_float4(0.f, 0.f, 0.f, 0.f);
        nw[j] = j < kc ? *reinterpret_cast<const uint4*>(a.nw + c8 * 8) : make_uint4(0u, 0u, 0u, 0u);
      }
      float ss = 0.f;
#pragma unroll
      for (int j = 0; j < KC; ++j)
        ss += s0[j].x * s0[j].x + s0[j].y * s0[j].y + s0[j].z * s0[j].z + s0[j].w * s0[j].w +
              s1[j].x * s1[j].x + s1[j].y * s1[j].y + s1[j].z * s1[j].z + s1[j].w * s1[j].w;
      ss = warp_sum(ss);
      const float rcp = 1.0f / sqrtf(ss / (float)K + a.eps);
#pragma unroll
      for (int j = 0; j < KC; ++j) {
        if (j < kc) {
          float4* d = reinterpret_cast<float4*>(xs_at(t, (32 * j + lane) * 8));
          d[0] = make_float4(round_bf16(s0[j].x * rcp * bf16_lo(nw[j].x)), round_bf16(s0[j].y * rcp * bf16_hi(nw[j].x)),
                             round_bf16(s0[j].z * rcp * bf16_lo(nw[j].y)), round_bf16(s0[j].w * rcp * bf16_hi(nw[j].y)));
          d[1] = make_float4(round_bf16(s1[j].x * rcp * bf16_lo(nw[j].z)), round_bf16(s1[j].y * rcp * bf16_hi(nw[j].z)),
                             round_bf16(s1[j].z * rcp * bf16_lo(nw[j].w)), round_bf16(s1[j].w * rcp * bf16_hi(nw[j].w)));
        }
      }
    }
  }
  __syncthreads();

  const float* xq = xs + q * sstr;  // this lane's sub-slice of token row 0
  for (int grp = blockIdx.x; grp < ngroups; grp += gridDim.x) {
    // residual of the ADD epilogue (thread t: token t's 8 features) goes out first
    const bool epi_thread = tid < T;
    const int64_t f0 = (int64_t)grp * kGemvFeat;
    uint4 rv = make_uint4(0u, 0u, 0u, 0u);
    if (a.epilogue == AIOSB_EPI_ADD && epi_thread)
      rv = *reinterpret_cast<const uint4*>(a.residual + (int64_t)tid * a.residual_stride + f0);
    uint4 wn[NR][KC];
    load_w(grp + gridDim.x, wn);  // next group, in flight during this one

    // ---- dot products over this lane's K/32 elements; one chain per token
    float acc[V];
#pragma unroll
    for (int i = 0; i < V; ++i) acc[i] = 0.f;
#pragma unroll
    for (int c = 0; c < KC; ++c) {
      if (c < kc) {
        float wf[NR][8];
#pragma unroll
        for (int r = 0; r < NR; ++r) {
          const uint32_t p[4] = {wv[r][c].x, wv[r][c].y, wv[r][c].z, wv[r][c].w};
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            wf[r][2 * e] = bf16_lo(p[e]);
            wf[r][2 * e + 1] = bf16_hi(p[e]);
          }
        }
#pragma unroll
        for (int t = 0; t < TMAX; ++t) {
          const float4 x0 = *reinterpret_cast<const float4*>(xq + (int64_t)t * rstr + c * 8);
          const float4 x1 = *reinterpret_cast<const float4*>(xq + (int64_t)t * rstr + c * 8 + 4);
          const float xv[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
#pragma unroll
          for (int r = 0; r < NR; ++r) {
            float s = acc[r * TMAX + t];
#pragma unroll
            for (int e = 0; e < 8; ++e) s = fmaf(wf[r][e], xv[e], s);
            acc[r * TMAX + t] = s;
          }
        }
      }
    }
    reduce_scatter_34<V>(acc);
    {
      const int q0 = ((lane >> 4) & 1) * (V / 2) + ((lane >> 3) & 1) * (V / 4);
#pragma unroll
      for (int i = 0; i < V / 4; ++i) part[warp][feat][q0 + i] = acc[i];
    }
    __syncthreads();
    if (tid < kGemvFeat * V) {
      const int j = tid / V, vi = tid % V;
      float sum = 0.f;
#pragma unroll
      for (int w = 0; w < kGemvFeat; ++w) sum += part[w][j][vi];
      accs[j][vi] = sum;
    }
    __syncthreads();

    // ---- epilogue: thread t writes token t's 8 features (16 bytes)
    if (epi_thread) {
      const int t = tid;
      float o[kGemvFeat];
      if (a.epilogue == AIOSB_EPI_SILU_MUL) {
#pragma unroll
        for (int j = 0; j < kGemvFeat; ++j) {
          // gate_up output is bf16 before silu_and_mul (aios/models/qwen3.py:90-92)
          const float g = round_bf16(accs[j][t]), u = round_bf16(accs[j][(NR - 1) * TMAX + t]);
          o[j] = g / (1.0f + expf(-g)) * u;
        }
      } else if (a.epilogue == AIOSB_EPI_ADD) {
        const uint32_t p[4] = {rv.x, rv.y, rv.z, rv.w};
#pragma unroll
        for (int j = 0; j < kGemvFeat; ++j) {
          const float res = (j & 1) ? bf16_hi(p[j >> 1]) : bf16_lo(p[j >> 1]);
          o[j] = res + round_bf16(accs[j][t]);
        }
        if (a.out_stat_x != nullptr) {
          float4* sx = reinterpret_cast<float4*>(a.out_stat_x + (int64_t)t * a.n_out + f0);
          sx[0] = make_float4(o[0], o[1], o[2], o[3]);
          sx[1] = make_float4(o[4], o[5], o[6], o[7]);
          float ss = 0.f;
#pragma unroll
          for (int j = 0; j < kGemvFeat; ++j) ss += o[j] * o[j];
          a.out_stat_ss[(int64_t)grp * a.out_ss_stride + t] = ss;
        }
      } else {
#pragma unroll
        for (int j = 0; j < kGemvFeat; ++j) o[j] = accs[j][t];
      }
      *reinterpret_cast<uint4*>(a.y + (int64_t)t * a.y_stride + f0) =
          make_uint4(pack_bf16x2(o[0], o[1]), pack_bf16x2(o[2], o[3]), pack_bf16x2(o[4], o[5]),
                     pack_bf16x2(o[6], o[7]));
    }
    __syncthreads();  // part / accs are rewritten by the next group
#pragma unroll
    for (int r = 0; r < NR; ++r)
#pragma unroll
      for (int c = 0; c < KC; ++c) wv[r][c] = wn[r][c];
  }
}

template <int NR, int TMAX, int KC, bool STAT>
int launch(const GemvArgs& a, cudaStream_t stream) {
  const size_t smem = (size_t)TMAX * 32 * (a.k / 32 + 4) * sizeof(float);
  auto kern = gemv_kernel<NR, TMAX, KC, STAT>;
  if (smem > 48 * 1024) cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  // at most two CTAs per SM; each walks several 8-feature groups
  const int64_t groups = a.n_out / kGemvFeat;
  const unsigned blocks = (unsigned)std::min<int64_t>(groups, 2 * (int64_t)sm_count());
  cudaError_t e = launch_pdl(kern, dim3(blocks), dim3(kGemvThreads), smem, stream, a);
  if (e != cudaSuccess) return set_error(AIOSB_ERR_LAUNCH, "linear (gemv): %s", cudaGetErrorString(e));
  return AIOSB_OK;
}

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

template <int NT, int KB, bool STAT>
__global__ void __launch_bounds__(kGemvThreads) gemv_mma_kernel(const GemvArgs a) {
  constexpr int TM = NT * 8;  // token rows covered
  __shared__ float red[kGemvFeat][NT][32][4];  // [warp][n tile][lane][fragment]
  __shared__ float tile[TM][17];               // reduced [token][row] (padded)
  __shared__ float ssw[kGemvFeat][TM];          // statistics mode: per-warp sums of squares
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, t4 = lane & 3;
  const int K = (int)a.k;
  const int kb = K / 256;  // 32-wide blocks per warp
  const int T = a.rows;
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
#pragma unroll
    for (int b = 0; b < KB; ++b) {
      const bool ok = tl < ntiles && b < kb;
      wa[b] = ok ? *reinterpret_cast<const uint4*>(a.w + r0 * K + kbase + b * 32) : make_uint4(0u, 0u, 0u, 0u);
      wb[b] = ok ? *reinterpret_cast<const uint4*>(a.w + r1 * K + kbase + b * 32) : make_uint4(0u, 0u, 0u, 0u);
    }
  };
  uint4 wa[KB], wb[KB];
  load_w(blockIdx.x, wa, wb);
  uint4 nwv[KB];
  if (STAT) {
#pragma unroll
    for (int b = 0; b < KB; ++b)
      nwv[b] = b < kb ? *reinterpret_cast<const uint4*>(a.nw + kbase + b * 32) : make_uint4(0u, 0u, 0u, 0u);
  }
  pdl_wait();
  pdl_launch_dependents();

  // ---- B fragments: token row n = nt * 8 + g, this lane's 8 elements per block
  uint4 xb[NT][KB];
  if (!STAT) {
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      const int n = nt * 8 + g;
#pragma unroll
      for (int b = 0; b < KB; ++b)
        xb[nt][b] = (n < T && b < kb) ? *reinterpret_cast<const uint4*>(a.x + (int64_t)n * a.x_stride + kbase + b * 32)
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
        const float4* src = reinterpret_cast<const float4*>(a.stat_x + (int64_t)n * K + kbase + b * 32);
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
            const uint4 rv = *reinterpret_cast<const uint4*>(a.residual + (int64_t)tk * a.residual_stride + f0);
            const uint32_t p[4] = {rv.x, rv.y, rv.z, rv.w};
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              const float res = (j & 1) ? bf16_hi(p[j >> 1]) : bf16_lo(p[j >> 1]);
              o[j] = res + round_bf16(tile[tk][8 * h + j]);
            }
            if (a.out_stat_x != nullptr) {
              float4* sx = reinterpret_cast<float4*>(a.out_stat_x + (int64_t)tk * a.n_out + f0);
              sx[0] = make_float4(o[0], o[1], o[2], o[3]);
              sx[1] = make_float4(o[4], o[5], o[6], o[7]);
              float ss = 0.f;
#pragma unroll
              for (int j = 0; j < 8; ++j) ss += o[j] * o[j];
              a.out_stat_ss[(f0 / kGemvStatGroup) * a.out_ss_stride + tk] = ss;
            }
          } else {
#pragma unroll
            for (int j = 0; j < 8; ++j) o[j] = tile[tk][8 * h + j];
          }
        }
        *reinterpret_cast<uint4*>(a.y + (int64_t)tk * a.y_stride + f0) =
            make_uint4(pack_bf16x2(o[0], o[1]), pack_bf16x2(o[2], o[3]), pack_bf16x2(o[4], o[5]),
                       pack_bf16x2(o[6], o[7]));
      }
    }
#pragma unroll
    for (int b = 0; b < KB; ++b) {
      wa[b] = na[b];
      wb[b] = nb[b];
    }
  }
}

template <int NT, int KB, bool STAT>
int launch_mma(const GemvArgs& a, cudaStream_t stream) {
  auto kern = gemv_mma_kernel<NT, KB, STAT>;
  const int64_t tiles = a.n_out / (a.epilogue == AIOSB_EPI_SILU_MUL ? 8 : 16);
  const unsigned blocks = (unsigned)std::min<int64_t>(tiles, 2 * (int64_t)sm_count());
  cudaError_t e = launch_pdl(kern, dim3(blocks), dim3(kGemvThreads), 0, stream, a);
  if (e != cudaSuccess) return set_error(AIOSB_ERR_LAUNCH, "linear (gemv mma): %s", cudaGetErrorString(e));
  return AIOSB_OK;
}

template <int NT, int KB>
int launch_mma_rows(const GemvArgs& a, cudaStream_t stream) {
  return a.stat_x != nullptr ? launch_mma<NT, KB, true>(a, stream) : launch_mma<NT, KB, false>(a, stream);
}

bool g_gemv_mma = [] {
  const char* env = getenv("AIOSB_GEMV_MMA");
  return env != nullptr && atoi(env) != 0;
}();

bool g_gemv_enabled = [] {
  const char* env = getenv("AIOSB_DECODE_GEMV");
  return env == nullptr || atoi(env) != 0;
}();

}  // namespace

bool gemv_eligible(int64_t rows, int64_t k, int64_t n_out) {
  return g_gemv_enabled && rows >= 1 && rows <= kMaxGemvRows && k % 256 == 0 && k <= kMaxGemvK &&
         n_out % kGemvFeat == 0;
}

template <int TMAX, int KC>
int launch_rows(const GemvArgs& a, cudaStream_t stream) {
  const bool silu = a.epilogue == AIOSB_EPI_SILU_MUL;
  if (a.stat_x != nullptr) return silu ? launch<2, TMAX, KC, true>(a, stream) : launch<1, TMAX, KC, true>(a, stream);
  return silu ? launch<2, TMAX, KC, false>(a, stream) : launch<1, TMAX, KC, false>(a, stream);
}

int gemv_launch(const GemvArgs& a, cudaStream_t stream) {
  const bool k3 = a.k <= 768;  // the 768-wide model dimension: 3 chunks, fewer registers
  if (g_gemv_mma && (a.epilogue == AIOSB_EPI_SILU_MUL || a.n_out % 16 == 0)) {
    if (a.rows <= 8) return k3 ? launch_mma_rows<1, 3>(a, stream) : launch_mma_rows<1, kMaxGemvK / 256>(a, stream);
    return k3 ? launch_mma_rows<2, 3>(a, stream) : launch_mma_rows<2, kMaxGemvK / 256>(a, stream);
  }
  if (a.rows <= 8) return k3 ? launch_rows<8, 3>(a, stream) : launch_rows<8, kMaxGemvK / 256>(a, stream);
  return k3 ? launch_rows<16, 3>(a, stream) : launch_rows<16, kMaxGemvK / 256>(a, stream);
}

}  // namespace aiosb
