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
#include <algorithm>
#include <mutex>

#include "abi_util.h"
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
};

template <int BN>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tm_w, const __grid_constant__ CUtensorMap tm_x,
                   const GemmArgs a) {
  constexpr uint32_t kBBytes = BN * kBK * 2;
  constexpr uint32_t kStageBytes = kABytes + kBBytes;
  constexpr uint32_t kTmemCols = BN < 32 ? 32 : BN;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t pipe_bytes = (uint32_t)a.stages * kStageBytes;
  const uint32_t red_bytes = BN * kBM * 4;
  const uint32_t body = pipe_bytes > red_bytes ? pipe_bytes : red_bytes;
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

  if (tid == 0) {
    // ---- TMA producer. Weights do not depend on the previous kernel, so the
    // first stages' weight tiles are requested before waiting on it (PDL).
    const int pre = nch < a.stages ? nch : a.stages;
    for (int i = 0; i < pre; ++i) {
      mbar_arrive_expect_tx(&full[i], kStageBytes);
      tma_load_2d(smem + i * kStageBytes, &tm_w, &full[i], (k_chunk0 + i) * kBK, m_tile * kBM);
    }
    pdl_wait();
    for (int i = 0; i < pre; ++i)
      tma_load_2d(smem + i * kStageBytes + kABytes, &tm_x, &full[i], (k_chunk0 + i) * kBK, n_tile * BN);
    for (int i = pre; i < nch; ++i) {
      const int s = i % a.stages;
      if (!mbar_wait(&empty[s], ((i / a.stages) & 1) ^ 1)) {
        report(a.status, AIOSB_DEV_WAIT_TIMEOUT);
        *abort_flag = 1;
        break;
      }
      mbar_arrive_expect_tx(&full[s], kStageBytes);
      tma_load_2d(smem + s * kStageBytes, &tm_w, &full[s], (k_chunk0 + i) * kBK, m_tile * kBM);
      tma_load_2d(smem + s * kStageBytes + kABytes, &tm_x, &full[s], (k_chunk0 + i) * kBK, n_tile * BN);
    }
  } else if (tid == 32) {
    // ---- MMA issuer.
    pdl_wait();
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
      const uint32_t a_base = smem_u32(smem + s * kStageBytes);
      const uint32_t b_base = a_base + kABytes;
#pragma unroll
      for (int kk = 0; kk < kBK / 16; ++kk) {
        tc_mma_bf16(tmem, umma_desc_sw128(a_base + kk * 32), umma_desc_sw128(b_base + kk * 32), idesc,
                    (i | kk) != 0 ? 1u : 0u);
      }
      tc_commit(&empty[s]);
    }
    if (ok) tc_commit(accum);
  } else {
    pdl_wait();
  }

  // ---- Epilogue: TMEM -> registers -> shared [BN][128] fp32.
  bool have = mbar_wait(accum, 0);
  if (!have) {
    report(a.status, AIOSB_DEV_WAIT_TIMEOUT);
    *abort_flag = 1;
  }
  // tcgen05.ld is warp-collective (.sync.aligned): reconverge and agree first.
  __syncwarp();
  have = __all_sync(0xffffffffu, have);
  tc_fence_after();
  if (have) {
    pdl_launch_dependents();
#pragma unroll
    for (int cb = 0; cb < BN / 16; ++cb) {
      float v[16];
      tmem_ld16(tmem + ((uint32_t)(32 * warp) << 16) + (uint32_t)(cb * 16), v);
      tc_wait_ld();
#pragma unroll
      for (int j = 0; j < 16; ++j) red[(cb * 16 + j) * kBM + 32 * warp + lane] = v[j];
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
    if (a.epilogue == AIOSB_EPI_STORE || a.epilogue == AIOSB_EPI_ADD) {
      // 32 float4 per column; 128 threads handle 4 columns per pass.
      for (int idx = tid; idx < BN * 32; idx += kThreads) {
        const int c = idx >> 5, m4 = idx & 31;
        if ((c % split) != (int)rank) continue;
        const int64_t t = t0 + c;
        if (t >= a.rows) continue;
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
        const uint32_t off = (uint32_t)((c * kBM + m4 * 4) * 4);
        for (int q = 0; q < split; ++q) {
          float4 p;
          if (split > 1) p = ld_dsmem_f4(map_shared_rank(red_addr + off, (uint32_t)q));
          else p = *reinterpret_cast<const float4*>(reinterpret_cast<const uint8_t*>(red) + off);
          acc.x += p.x; acc.y += p.y; acc.z += p.z; acc.w += p.w;
        }
        __nv_bfloat16* dst = a.y + t * a.y_row_stride + (int64_t)m_tile * kBM + m4 * 4;
        if (a.epilogue == AIOSB_EPI_ADD) {
          // residual + delta with the delta rounded to bf16 first, as the
          // reference's bf16 `partial + delta` (aios/models/minimind_ime.py:237-252).
          const uint2 rv = *reinterpret_cast<const uint2*>(a.residual + t * a.residual_stride +
                                                          (int64_t)m_tile * kBM + m4 * 4);
          acc.x = bf16_lo(rv.x) + round_bf16(acc.x);
          acc.y = bf16_hi(rv.x) + round_bf16(acc.y);
          acc.z = bf16_lo(rv.y) + round_bf16(acc.z);
          acc.w = bf16_hi(rv.y) + round_bf16(acc.w);
        }
        uint2 o = make_uint2(pack_bf16x2(acc.x, acc.y), pack_bf16x2(acc.z, acc.w));
        *reinterpret_cast<uint2*>(dst) = o;
      }
    } else {
      // SILU_MUL: tile rows 0..63 are gate rows, 64..127 the matching up rows.
      for (int idx = tid; idx < BN * 16; idx += kThreads) {
        const int c = idx >> 4, m4 = idx & 15;
        if ((c % split) != (int)rank) continue;
        const int64_t t = t0 + c;
        if (t >= a.rows) continue;
        float4 g = make_float4(0.f, 0.f, 0.f, 0.f), u = g;
        const uint32_t og = (uint32_t)((c * kBM + m4 * 4) * 4);
        const uint32_t ou = og + 64 * 4;
        for (int q = 0; q < split; ++q) {
          float4 pg, pu;
          if (split > 1) {
            pg = ld_dsmem_f4(map_shared_rank(red_addr + og, (uint32_t)q));
            pu = ld_dsmem_f4(map_shared_rank(red_addr + ou, (uint32_t)q));
          } else {
            pg = *reinterpret_cast<const float4*>(reinterpret_cast<const uint8_t*>(red) + og);
            pu = *reinterpret_cast<const float4*>(reinterpret_cast<const uint8_t*>(red) + ou);
          }
          g.x += pg.x; g.y += pg.y; g.z += pg.z; g.w += pg.w;
          u.x += pu.x; u.y += pu.y; u.z += pu.z; u.w += pu.w;
        }
        // gate_up output is bf16 before silu_and_mul (aios/models/qwen3.py:90-92).
        const float gv[4] = {round_bf16(g.x), round_bf16(g.y), round_bf16(g.z), round_bf16(g.w)};
        const float uv[4] = {round_bf16(u.x), round_bf16(u.y), round_bf16(u.z), round_bf16(u.w)};
        float r[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) r[j] = gv[j] / (1.0f + expf(-gv[j])) * uv[j];
        __nv_bfloat16* dst = a.y + t * a.y_row_stride + (int64_t)m_tile * (kBM / 2) + m4 * 4;
        *reinterpret_cast<uint2*>(dst) = make_uint2(pack_bf16x2(r[0], r[1]), pack_bf16x2(r[2], r[3]));
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
size_t smem_bytes(int stages) {
  const size_t pipe = (size_t)stages * (kABytes + BN * kBK * 2);
  const size_t red = (size_t)BN * kBM * 4;
  return std::max(pipe, red) + 1024 /*alignment*/ + 256 /*barriers*/;
}

template <int BN>
int launch_gemm(const CUtensorMap& tw, const CUtensorMap& tx, GemmArgs a, int m_tiles, int n_tiles,
                cudaStream_t stream) {
  static bool configured[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  auto kern = gemm_tc_kernel<BN>;
  if (dev >= 0 && dev < 64 && !configured[dev]) {
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem_bytes<BN>(max_stages_for(BN)));
    cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
    configured[dev] = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)m_tiles, (unsigned)a.split, (unsigned)n_tiles);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem_bytes<BN>(a.stages);
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
int g_max_split = kMaxSplit;  // lowered to 8 if 16-CTA clusters cannot launch

int choose_split(int64_t tiles, int64_t chunks, int sms) {
  int best = 1;
  for (int d = 2; d <= g_max_split; ++d)
    if (chunks % d == 0 && tiles * d <= sms) best = d;
  return best;
}

}  // namespace
}  // namespace aiosb

using namespace aiosb;

extern "C" int aiosb_linear(const void* x, int64_t rows, int64_t k, const void* w, int64_t n, void* y,
                            int64_t y_row_stride, int epilogue, const void* residual, int64_t residual_stride,
                            int32_t* status, void* stream) {
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
  if (rows == 0) return AIOSB_OK;
  AIOSB_REQUIRE(x && w && y, AIOSB_ERR_INVALID_ARG, "linear: null pointer");
  AIOSB_REQUIRE(aligned16(x) && aligned16(w) && aligned16(y), AIOSB_ERR_MISALIGNED,
                "linear: x, w and y must be 16-byte aligned");
  const int bn = rows <= 16 ? 16 : rows <= 32 ? 32 : rows <= 64 ? 64 : rows <= 128 ? 128 : 256;
  const int64_t m_tiles = n / kBM;
  const int64_t n_tiles = (rows + bn - 1) / bn;
  const int64_t chunks = k / kBK;
  GemmArgs a;
  a.rows = rows;
  a.n = n;
  a.y_row_stride = y_row_stride;
  a.y = (__nv_bfloat16*)y;
  a.residual = (const __nv_bfloat16*)residual;
  a.residual_stride = residual_stride;
  a.status = status;
  a.epilogue = epilogue;
  a.split = choose_split(m_tiles * n_tiles, chunks, sm_count());
  a.chunks_per_split = (int)(chunks / a.split);
  a.stages = std::min(a.chunks_per_split, max_stages_for(bn));
  CUtensorMap tw, tx;
  int rc = make_map(&tw, w, n, k, kBM);
  if (rc) return rc;
  rc = make_map(&tx, x, rows, k, (uint32_t)bn);
  if (rc) return rc;
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
    a.split = choose_split(m_tiles * n_tiles, chunks, sm_count());
    a.chunks_per_split = (int)(chunks / a.split);
    a.stages = std::min(a.chunks_per_split, max_stages_for(bn));
    rc = launch();
  }
  return rc;
}
