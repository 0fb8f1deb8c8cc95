// Persistent decode step: one launch runs a whole decode forward of the
// standard-residual MiniMind-IME decoder (aios/models/qwen3.py:101-155: the
// embedding, every layer's qkv linear, q/k RMSNorm + RoPE + KV store + paged
// attention, o linear + residual, gate/up linear + SwiGLU, down linear +
// residual, then the final RMSNorm and the LM head) for the <= 16 candidate rows
// of a CandidateGroup step.
//
// Why one launch: at 8 rows every decode linear is a weight stream with 8 dot
// products per weight, and a step is a chain of 71 dependent phases (5 per layer
// plus the LM head). As separate kernels each phase paid a kernel boundary.
// Here one CTA per SM runs the whole chain:
//   * a producer warp streams the CTA's share of every phase's weights, in the
//     order the CTA will use them, into a ring of shared-memory slots with
//     cp.async.bulk (evict-first in L2). Weights do not depend on activations, so
//     it runs up to a ring's worth of tiles ahead, across phase boundaries;
//   * 8 consumer warps run the phases. A phase's items (16-row weight tiles, or
//     (KV head, row) attention items) go round-robin over the CTAs, continuing
//     where the previous phase stopped, so consecutive phases land on different
//     CTAs and every CTA streams about the same bytes per step;
//   * phase p may start on a CTA once every CTA has arrived at phase p - 1: each
//     CTA adds 1 to a per-phase counter (release, after its own work of that
//     phase, or at once when it has none) and waits (acquire) on the previous
//     phase's counter only before a phase in which it has work. Arriving at p
//     implies having finished every phase <= p, so counter p - 1 complete means
//     all inputs of phase p exist.
// Every wait is bounded (a time limit; a global abort word stops the other CTAs'
// waits at once) and reports AIOSB_DEV_WAIT_TIMEOUT through the status word.
// The consumer warps' control flow never depends on the abort flag (which the
// producer warp may set at any time), so their named barriers always match up;
// an abort only skips waits and MMAs, and the launch's outputs are then void.
//
// Linears: register-operand mma.sync m16n8k16 (bf16 in, fp32 accumulate) with the
// K-permuted fragment layout of gemv.cu: lane (g, t) reads 16 contiguous bytes of
// weight rows g and g + 8 and of token row g per 32-wide K block, so every
// fragment is one 16-byte load; the 8 warps split K and their partial tiles are
// summed in warp order. The slot rows are padded to 1600 bytes (a 16-bank offset
// between consecutive rows), so the A-fragment reads are conflict-free. RMSNorm is
// folded into the operand load from the fp32 residual stream, as in the GEMV.
// Attention: one item per (KV head, row): the key history (prefix and older
// suffix, written by earlier launches) is staged in shared memory before the
// phase wait, then q/k RMSNorm + bf16 RoPE, the new K/V store and one online-
// softmax pass per 64 keys, as attn_decode_hist_kernel (attention.cu) does.
// Rounding points equal the per-kernel path: bf16 linear outputs, gate/up rounded
// before SwiGLU, the delta rounded before the residual add.
#include <algorithm>

#include "abi_util.h"
#include "attn_device.cuh"
#include "common.cuh"

namespace aiosb {
namespace {

constexpr int kCWarps = 8;                  // consumer warps
constexpr int kCThreads = kCWarps * 32;     // 256
constexpr int kStepThreads = kCThreads + 32;  // + the producer warp
constexpr int kHidden = 768;
constexpr int kFfn = 2048;
constexpr int kChunkK = 768;                 // K elements of one weight slot
constexpr int kRowPitch = kChunkK * 2 + 64;  // padded slot row (bytes)
constexpr int kSlotBytes = 16 * kRowPitch;   // 25600
constexpr int kMaxSlots = 8;
constexpr int kMaxChunks = (kFfn + kChunkK - 1) / kChunkK;  // 3 weight chunks per tile at K = 2048
constexpr int kOpBlocks = kMaxChunks * 3;    // operand fragment slots per lane: (chunk, 32-wide block)
constexpr int kSPrefix = 64;                 // staged prefix keys per attention item
constexpr int kSSuffix = 32;                 // staged suffix keys (incl. the new one)
constexpr int kSmemLimit = 232448;           // 227 KB opt-in per CTA

enum : int { kQKV = 0, kATT = 1, kO = 2, kGU = 3, kDN = 4, kLMH = 5 };

struct Phase {
  int kind, layer, items, chunks;
};

__device__ __forceinline__ Phase phase_of(int p, const aiosb_decode_step_args& a) {
  if (p == 5 * a.num_layers) return {kLMH, 0, (int)(a.vocab / 16), 1};
  const int l = p / 5, k = p % 5;
  const int nqkv = (a.num_qo_heads + 2 * a.num_kv_heads) * a.head_dim;
  switch (k) {
    case 0: return {kQKV, l, nqkv / 16, 1};
    case 1: return {kATT, l, a.num_kv_heads * a.rows, 0};
    case 2: return {kO, l, kHidden / 16, 1};
    case 3: return {kGU, l, kFfn / 8, 1};
    default: return {kDN, l, kHidden / 16, (kFfn + kChunkK - 1) / kChunkK};
  }
}

__device__ __forceinline__ int chunk_len(int kind, int c) {
  const int K = kind == kDN ? kFfn : kHidden;
  return min(kChunkK, K - c * kChunkK);
}

// First item of a phase on CTA `cta` when items start at CTA `offset`.
__device__ __forceinline__ int first_item(int cta, int offset, int grid) {
  return ((cta - offset) % grid + grid) % grid;
}

// ---- synchronisation primitives ----------------------------------------------
__device__ __forceinline__ uint32_t ld_acquire_u32(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ uint32_t ld_relaxed_u32(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
// Barrier of the 8 consumer warps (the producer warp never joins it). Lanes that
// diverged (one thread spinning on a counter) reconverge first.
__device__ __forceinline__ void consumer_sync() {
  __syncwarp();
  asm volatile("bar.sync 1, 256;" ::: "memory");
}

__device__ __forceinline__ uint64_t l2_evict_first() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}
__device__ __forceinline__ void bulk_row(void* dst, const void* src, uint32_t bytes, uint64_t* bar, uint64_t pol) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::
          "r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(smem_u32(bar)), "l"(pol)
      : "memory");
}

// mbarrier wait with a caller-given limit that also gives up when `abort_s` is set.
__device__ __forceinline__ bool bar_wait(uint64_t* bar, uint32_t parity, uint64_t limit,
                                         const volatile int* abort_s) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t start = global_ns();
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    if (*abort_s) return false;
    if (global_ns() - start > limit) return false;
  }
}

__device__ __forceinline__ void mma16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// Source of weight row `row` (0..15) of slot item `item` of a phase, and its K pitch.
__device__ __forceinline__ const __nv_bfloat16* weight_row(const aiosb_decode_step_args& a, const Phase& ph,
                                                           int item, int row) {
  const aiosb_decode_layer& L = a.layers[ph.layer];
  switch (ph.kind) {
    case kQKV: return static_cast<const __nv_bfloat16*>(L.w_qkv) + ((int64_t)item * 16 + row) * kHidden;
    case kO: return static_cast<const __nv_bfloat16*>(L.w_o) + ((int64_t)item * 16 + row) * kHidden;
    case kGU: {
      // [g0..63 | u0..63 | g64..]: slot rows 0-7 gate rows of features 8 item.., 8-15 their up rows
      const int64_t f = (int64_t)item * 8 + (row & 7);
      const int64_t r = (f / 64) * 128 + (f % 64) + (row >= 8 ? 64 : 0);
      return static_cast<const __nv_bfloat16*>(L.w_gate_up) + r * kHidden;
    }
    case kDN: return static_cast<const __nv_bfloat16*>(L.w_down) + ((int64_t)item * 16 + row) * kFfn;
    default: return static_cast<const __nv_bfloat16*>(a.lm_head) + ((int64_t)item * 16 + row) * kHidden;
  }
}

// Shared-memory layout (dynamic): [slots x kSlotBytes][scratch union][barriers]
template <int NT, int D>
struct StepSmem {
  static constexpr int TM = NT * 8;
  // linear scratch
  static constexpr int kRed = kCWarps * NT * 32 * 4 * 4;
  static constexpr int kTile = TM * 17 * 4;
  static constexpr int kSsw = kCWarps * TM * 4;
  static constexpr int kLinear = kRed + kTile + kSsw;
  // attention scratch
  static constexpr int KR = D + 2;
  static constexpr int kQ = 8 * D * 4;           // <= 8 query heads per KV head
  static constexpr int kTmp = kCWarps * D * 4;
  static constexpr int kKh = (kSPrefix + kSSuffix) * KR * 2;
  static constexpr int kVh = (kSPrefix + kSSuffix) * D * 2;
  static constexpr int kKw = kKeyChunk * KR * 2;
  static constexpr int kVw = kKeyChunk * D * 2;
  static constexpr int kRope = 4 * D * 2;
  static constexpr int kSlots = (kSPrefix + kSSuffix) * 4;
  static constexpr int kAttn = kQ + kTmp + kKh + kVh + kKw + kVw + kRope + kSlots;
  static constexpr int kScratch = ((kLinear > kAttn ? kLinear : kAttn) + 127) / 128 * 128;
  static constexpr int kBars = 2 * kMaxSlots * 8 + 64;
  static int slots() { return std::min(kMaxSlots, (kSmemLimit - kScratch - kBars) / kSlotBytes); }
  static size_t bytes(int nslots) { return (size_t)nslots * kSlotBytes + kScratch + kBars; }
};

template <int NT, int D>
__global__ void __launch_bounds__(kStepThreads, 1) decode_step_kernel(const aiosb_decode_step_args a, int nslots) {
  using SM = StepSmem<NT, D>;
  constexpr int TM = NT * 8;
  constexpr int DPL = D / 32;
  extern __shared__ __align__(128) uint8_t smem[];
  uint8_t* ring = smem;
  uint8_t* scratch = smem + (size_t)nslots * kSlotBytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(scratch + SM::kScratch);
  uint64_t* empty = full + kMaxSlots;
  __shared__ volatile int abort_s;
  __shared__ volatile int64_t issued_s;

  const int G = gridDim.x, cta = blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int NP = 5 * a.num_layers + 1;
  uint32_t* counters = a.sync;
  uint32_t* done_ctr = a.sync + NP;
  uint32_t* abort_g = a.sync + NP + 1;
  const uint64_t limit = a.wait_limit_ns != 0 ? a.wait_limit_ns : kWaitLimitNs;
  const uint32_t need = (uint32_t)G + a.test_extra_arrivals;
  const int R = a.rows;

  if (threadIdx.x == 0) {
    for (int s = 0; s < nslots; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kCWarps);
    }
    abort_s = 0;
    issued_s = 0;
    fence_mbar_init();
  }
  __syncthreads();

  auto fail = [&](int32_t code) {
    report(a.status, code);
    abort_s = 1;
    atomicExch(abort_g, 1u);
  };

  // =========================================================== producer warp
  if (warp == kCWarps) {
    if (lane == 0) {
      const uint64_t pol = l2_evict_first();
      int64_t seq = 0;
      int offset = 0;
      for (int p = 0; p < NP && !abort_s; ++p) {
        const Phase ph = phase_of(p, a);
        if (ph.chunks > 0) {
          for (int it = first_item(cta, offset, G); it < ph.items && !abort_s; it += G) {
            for (int c = 0; c < ph.chunks; ++c) {
              const int s = (int)(seq % nslots);
              const uint32_t use = (uint32_t)(seq / nslots);
              if (use >= 1 && !bar_wait(&empty[s], (use - 1) & 1, limit, &abort_s)) {
                if (!abort_s) fail(AIOSB_DEV_WAIT_TIMEOUT);
                break;
              }
              // after an abort, consumers release slots without waiting for their
              // copies, so a slot is never refilled once the abort is visible (it
              // is set before that release); the last copy per slot is drained at exit
              if (abort_s) break;
              const int klen = chunk_len(ph.kind, c);
              const uint32_t row_bytes = (uint32_t)klen * 2;
              mbar_arrive_expect_tx(&full[s], 16 * row_bytes);
              uint8_t* dst = ring + (size_t)s * kSlotBytes;
              for (int r = 0; r < 16; ++r)
                bulk_row(dst + r * kRowPitch, weight_row(a, ph, it, r) + c * kChunkK, row_bytes, &full[s], pol);
              ++seq;
              issued_s = seq;
            }
          }
        }
        offset = (offset + ph.items) % G;
      }
    }
    __syncwarp();
  } else {
    // ========================================================= consumer warps
    pdl_wait();  // the group step (previous kernel) wrote the rows' tokens and metadata
    const int tid = threadIdx.x;
    const int g = lane >> 2, t4 = lane & 3;
    float* red = reinterpret_cast<float*>(scratch);            // [warp][nt][lane][4]
    float* tile = reinterpret_cast<float*>(scratch + SM::kRed);  // [TM][17]
    float* ssw = reinterpret_cast<float*>(scratch + SM::kRed + SM::kTile);  // [warp][TM]
    const int nqkv = (a.num_qo_heads + 2 * a.num_kv_heads) * a.head_dim;
    const int gq = a.num_qo_heads / a.num_kv_heads;
    int64_t seq = 0;
    int offset = 0;

    // wait until every CTA arrived at phase p - 1
    auto wait_phase = [&](int p) {
      if (p == 0) return;
      if (tid == 0 && !abort_s) {
        const uint32_t* c = counters + (p - 1);
        if (ld_acquire_u32(c) < need) {
          const uint64_t start = global_ns();
          while (ld_acquire_u32(c) < need) {
            if (ld_relaxed_u32(abort_g) != 0) {
              abort_s = 1;
              break;
            }
            if (global_ns() - start > limit) {
              fail(AIOSB_DEV_WAIT_TIMEOUT);
              break;
            }
          }
        }
      }
      consumer_sync();
    };

    // ---- operand fragments of a linear phase (token rows in the B layout)
    uint4 xb[NT][kOpBlocks];  // [token tile][chunk * 3 + block]
    auto build_operand = [&](const Phase& ph) {
      if (ph.kind == kO || ph.kind == kDN) {  // plain bf16 rows: attention output / SwiGLU activation
        const __nv_bfloat16* src = static_cast<const __nv_bfloat16*>(ph.kind == kO ? a.attn : a.act);
        const int64_t ld = ph.kind == kO ? a.attn_stride : a.act_stride;
#pragma unroll
        for (int c = 0; c < kMaxChunks; ++c) {
          const int kb = c < ph.chunks ? chunk_len(ph.kind, c) / 256 : 0;
#pragma unroll
          for (int j = 0; j < 3; ++j) {
            if (j < kb) {
              const int k = c * kChunkK + (warp * kb + j) * 32 + 8 * t4;
#pragma unroll
              for (int nt = 0; nt < NT; ++nt) {
                const int n = nt * 8 + g;
                xb[nt][c * 3 + j] = n < R ? *reinterpret_cast<const uint4*>(src + (int64_t)n * ld + k)
                                          : make_uint4(0u, 0u, 0u, 0u);
              }
            }
          }
        }
        return;
      }
      // normalised from the fp32 residual stream (RMSNormFused, aios/layers/norm.py:34-40),
      // or for layer 0's qkv from the embedding rows (their fp32 values)
      const bool embed = ph.kind == kQKV && ph.layer == 0;
      const __nv_bfloat16* nw =
          static_cast<const __nv_bfloat16*>(ph.kind == kLMH ? a.final_norm
                                            : ph.kind == kQKV ? a.layers[ph.layer].in_norm
                                                              : a.layers[ph.layer].post_norm);
      float4 sv[NT][3][2];
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        const int n = nt * 8 + g;
        int64_t tok = 0;
        if (embed && n < R) {
          tok = a.tokens[n];
          if (tok < 0 || tok >= a.vocab) {
            if (t4 == 0 && warp == 0) report(a.status, AIOSB_DEV_TOKEN_RANGE);
            tok = 0;
          }
        }
#pragma unroll
        for (int j = 0; j < 3; ++j) {
          const int k = (warp * 3 + j) * 32 + 8 * t4;
          if (n >= R) {
            sv[nt][j][0] = sv[nt][j][1] = make_float4(0.f, 0.f, 0.f, 0.f);
          } else if (embed) {
            const uint4 e = *reinterpret_cast<const uint4*>(static_cast<const __nv_bfloat16*>(a.embed) +
                                                            tok * kHidden + k);
            sv[nt][j][0] = make_float4(bf16_lo(e.x), bf16_hi(e.x), bf16_lo(e.y), bf16_hi(e.y));
            sv[nt][j][1] = make_float4(bf16_lo(e.z), bf16_hi(e.z), bf16_lo(e.w), bf16_hi(e.w));
          } else {
            const float4* s4 = reinterpret_cast<const float4*>(a.resid_f32 + (int64_t)n * kHidden + k);
            sv[nt][j][0] = s4[0];
            sv[nt][j][1] = s4[1];
          }
        }
      }
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        float ss = 0.f;
#pragma unroll
        for (int j = 0; j < 3; ++j)
#pragma unroll
          for (int h = 0; h < 2; ++h)
            ss += sv[nt][j][h].x * sv[nt][j][h].x + sv[nt][j][h].y * sv[nt][j][h].y +
                  sv[nt][j][h].z * sv[nt][j][h].z + sv[nt][j][h].w * sv[nt][j][h].w;
        ss += __shfl_xor_sync(0xffffffffu, ss, 1);
        ss += __shfl_xor_sync(0xffffffffu, ss, 2);
        if (t4 == 0) ssw[warp * TM + nt * 8 + g] = ss;
      }
      consumer_sync();
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        float ss = 0.f;
#pragma unroll
        for (int w = 0; w < kCWarps; ++w) ss += ssw[w * TM + nt * 8 + g];
        const float rcp = 1.0f / sqrtf(ss / (float)kHidden + a.eps);
#pragma unroll
        for (int j = 0; j < 3; ++j) {
          const uint4 wv = *reinterpret_cast<const uint4*>(nw + (warp * 3 + j) * 32 + 8 * t4);
          const float4 s0 = sv[nt][j][0], s1 = sv[nt][j][1];
          xb[nt][j] = make_uint4(pack_bf16x2(s0.x * rcp * bf16_lo(wv.x), s0.y * rcp * bf16_hi(wv.x)),
                                 pack_bf16x2(s0.z * rcp * bf16_lo(wv.y), s0.w * rcp * bf16_hi(wv.y)),
                                 pack_bf16x2(s1.x * rcp * bf16_lo(wv.z), s1.y * rcp * bf16_hi(wv.z)),
                                 pack_bf16x2(s1.z * rcp * bf16_lo(wv.w), s1.w * rcp * bf16_hi(wv.w)));
        }
      }
      consumer_sync();  // ssw is rewritten by the next phase
    };

    // ---- one 16-row tile: MMAs over its chunks, warp-order reduction, epilogue
    auto run_tile = [&](const Phase& ph, int item) {
      float d[NT][4];
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) d[nt][0] = d[nt][1] = d[nt][2] = d[nt][3] = 0.f;
#pragma unroll
      for (int c = 0; c < kMaxChunks; ++c) {
        if (c < ph.chunks) {
          const int s = (int)(seq % nslots);
          const uint32_t use = (uint32_t)(seq / nslots);
          ++seq;
          const int kb = chunk_len(ph.kind, c) / 256;
          if (!abort_s && bar_wait(&full[s], use & 1, limit, &abort_s)) {
            const uint8_t* slot = ring + (size_t)s * kSlotBytes;
#pragma unroll
            for (int j = 0; j < 3; ++j) {
              if (j < kb) {
                const int koff = ((warp * kb + j) * 32 + 8 * t4) * 2;
                const uint4 wa = *reinterpret_cast<const uint4*>(slot + g * kRowPitch + koff);
                const uint4 wb = *reinterpret_cast<const uint4*>(slot + (g + 8) * kRowPitch + koff);
#pragma unroll
                for (int nt = 0; nt < NT; ++nt) {
                  const uint4 x = xb[nt][c * 3 + j];
                  mma16816(d[nt], wa.x, wb.x, wa.y, wb.y, x.x, x.y);
                  mma16816(d[nt], wa.z, wb.z, wa.w, wb.w, x.z, x.w);
                }
              }
            }
          } else if (!abort_s) {
            fail(AIOSB_DEV_WAIT_TIMEOUT);
          }
          __syncwarp();
          if (lane == 0) mbar_arrive(&empty[s]);
        }
      }
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
        *reinterpret_cast<float4*>(&red[((warp * NT + nt) * 32 + lane) * 4]) =
            make_float4(d[nt][0], d[nt][1], d[nt][2], d[nt][3]);
      consumer_sync();
      for (int i = tid; i < NT * 128; i += kCThreads) {
        const int nt = i / 128, l = (i / 4) % 32, j = i % 4;
        float sum = 0.f;
#pragma unroll
        for (int w = 0; w < kCWarps; ++w) sum += red[((w * NT + nt) * 32 + l) * 4 + j];
        tile[(nt * 8 + 2 * (l & 3) + (j & 1)) * 17 + (l >> 2) + 8 * (j >> 1)] = sum;
      }
      consumer_sync();
      if (tid < TM * 2) {
        const int tk = tid >> 1, h = tid & 1;
        const bool silu = ph.kind == kGU;
        if (tk < R && (!silu || h == 0)) {
          float o[8];
          if (silu) {
            const int64_t f0 = (int64_t)item * 8;
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              // gate_up output is bf16 before silu_and_mul (aios/models/qwen3.py:90-92)
              const float gt = round_bf16(tile[tk * 17 + j]), up = round_bf16(tile[tk * 17 + 8 + j]);
              o[j] = gt / (1.0f + expf(-gt)) * up;
            }
            *reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(a.act) + (int64_t)tk * a.act_stride + f0) =
                make_uint4(pack_bf16x2(o[0], o[1]), pack_bf16x2(o[2], o[3]), pack_bf16x2(o[4], o[5]),
                           pack_bf16x2(o[6], o[7]));
          } else {
            const int64_t f0 = (int64_t)item * 16 + 8 * h;
            if (ph.kind == kO || ph.kind == kDN) {
              // residual add: delta rounded to bf16, fp32 sum kept for the next norm,
              // the bf16 residual stored (aios/layers/norm.py:34-40)
              __nv_bfloat16* res = static_cast<__nv_bfloat16*>(a.resid) + (int64_t)tk * kHidden + f0;
              const uint4 rv = *reinterpret_cast<const uint4*>(res);
              const uint32_t p[4] = {rv.x, rv.y, rv.z, rv.w};
#pragma unroll
              for (int j = 0; j < 8; ++j) {
                const float rr = (j & 1) ? bf16_hi(p[j >> 1]) : bf16_lo(p[j >> 1]);
                o[j] = rr + round_bf16(tile[tk * 17 + 8 * h + j]);
              }
              float4* sx = reinterpret_cast<float4*>(a.resid_f32 + (int64_t)tk * kHidden + f0);
              sx[0] = make_float4(o[0], o[1], o[2], o[3]);
              sx[1] = make_float4(o[4], o[5], o[6], o[7]);
              *reinterpret_cast<uint4*>(res) = make_uint4(pack_bf16x2(o[0], o[1]), pack_bf16x2(o[2], o[3]),
                                                          pack_bf16x2(o[4], o[5]), pack_bf16x2(o[6], o[7]));
            } else {
#pragma unroll
              for (int j = 0; j < 8; ++j) o[j] = tile[tk * 17 + 8 * h + j];
              __nv_bfloat16* dst = ph.kind == kQKV
                                       ? static_cast<__nv_bfloat16*>(a.qkv) + (int64_t)tk * a.qkv_stride + f0
                                       : static_cast<__nv_bfloat16*>(a.logits) + (int64_t)tk * a.logits_stride + f0;
              *reinterpret_cast<uint4*>(dst) = make_uint4(pack_bf16x2(o[0], o[1]), pack_bf16x2(o[2], o[3]),
                                                          pack_bf16x2(o[4], o[5]), pack_bf16x2(o[6], o[7]));
            }
          }
        }
      }
      // the next tile's reduction rewrites `tile` only after its own consumer_sync
    };

    // ---- attention item (KV head h, row r) of layer l
    using SMA = StepSmem<NT, D>;
    constexpr int KR = SMA::KR;
    float* q_s = reinterpret_cast<float*>(scratch);
    float* tmp = reinterpret_cast<float*>(scratch + SMA::kQ);
    __nv_bfloat16* Kh = reinterpret_cast<__nv_bfloat16*>(scratch + SMA::kQ + SMA::kTmp);
    __nv_bfloat16* Vh = reinterpret_cast<__nv_bfloat16*>(scratch + SMA::kQ + SMA::kTmp + SMA::kKh);
    __nv_bfloat16* Kw = reinterpret_cast<__nv_bfloat16*>(scratch + SMA::kQ + SMA::kTmp + SMA::kKh + SMA::kVh);
    __nv_bfloat16* Vw = Kw + kKeyChunk * KR;
    __nv_bfloat16* cos_r = Vw + kKeyChunk * D;
    __nv_bfloat16* sin_r = cos_r + D;
    __nv_bfloat16* nq = sin_r + D;
    __nv_bfloat16* nk = nq + D;
    int32_t* slot_s = reinterpret_cast<int32_t*>(nk + D);
    const int64_t tok_stride = (int64_t)a.num_kv_heads * D;
    const int P = a.prefix_len != nullptr ? *a.prefix_len : 0;
    const int64_t prow = a.row_table[0];
    struct AttnItem {
      int h, r, np, ns, ns_old, nst, L, pos, pos_in, L_in;
      int64_t rrow, oslot;
      bool act, pos_ok, bad_slot;
    };
    // stage the key history of item `it` (everything but this step's key)
    auto attn_stage = [&](const Phase& ph, int it) -> AttnItem {
      AttnItem m;
      m.h = it % a.num_kv_heads;
      m.r = it / a.num_kv_heads;
      const aiosb_decode_layer& Ly = a.layers[ph.layer];
      m.rrow = a.row_table[m.r];
      m.act = a.active == nullptr || a.active[m.r] != 0;
      m.pos_in = a.positions[m.r];
      m.L_in = a.seq_lens[m.r];
      m.oslot = a.out_loc[m.r];
      const int L_lo = m.L_in > P + 1 ? m.L_in : P + 1;
      m.L = (int64_t)L_lo > a.table_stride ? (int)a.table_stride : L_lo;
      m.ns_old = max(0, m.L - 1 - P);
      m.np = min(P, kSPrefix);
      m.ns = min(m.ns_old, kSSuffix - 1);
      m.nst = m.act ? m.np + m.ns : 0;
      m.pos_ok = m.pos_in >= 0 && m.pos_in < a.max_pos;
      m.pos = m.pos_ok ? m.pos_in : 0;
      for (int i = tid; i < m.nst; i += kCThreads)
        slot_s[i] = a.page_table[i < m.np ? prow * a.table_stride + i : m.rrow * a.table_stride + P + (i - m.np)];
      const __nv_bfloat16* qn = static_cast<const __nv_bfloat16*>(Ly.q_norm);
      const __nv_bfloat16* kn = static_cast<const __nv_bfloat16*>(Ly.k_norm);
      const __nv_bfloat16* ct = static_cast<const __nv_bfloat16*>(a.cos_tab);
      const __nv_bfloat16* st = static_cast<const __nv_bfloat16*>(a.sin_tab);
      for (int i = tid; i < D; i += kCThreads) {
        nq[i] = qn[i];
        nk[i] = kn[i];
        cos_r[i] = ct[(int64_t)m.pos * D + i];
        sin_r[i] = st[(int64_t)m.pos * D + i];
      }
      consumer_sync();
      bool b = false;
      for (int j = lane; j < m.nst; j += 32) b |= slot_s[j] < 0 || slot_s[j] >= a.num_slots;
      m.bad_slot = __any_sync(0xffffffffu, b);
      const __nv_bfloat16* kc = static_cast<const __nv_bfloat16*>(Ly.k_cache);
      const __nv_bfloat16* vc = static_cast<const __nv_bfloat16*>(Ly.v_cache);
      for (int i = tid; i < m.nst * (D / 8); i += kCThreads) {
        const int j = i / (D / 8), c = i % (D / 8);
        int64_t slot = slot_s[j];
        if (slot < 0 || slot >= a.num_slots) slot = 0;  // reported after the wait
        const uint4 kv = reinterpret_cast<const uint4*>(kc + slot * tok_stride + (int64_t)m.h * D)[c];
        const uint4 vv = reinterpret_cast<const uint4*>(vc + slot * tok_stride + (int64_t)m.h * D)[c];
        uint32_t* kd = reinterpret_cast<uint32_t*>(Kh + j * KR) + c * 4;
        kd[0] = kv.x;
        kd[1] = kv.y;
        kd[2] = kv.z;
        kd[3] = kv.w;
        reinterpret_cast<uint4*>(Vh + j * D)[c] = vv;
      }
      consumer_sync();
      return m;
    };
    auto attn_run = [&](const Phase& ph, const AttnItem& m) {
      const aiosb_decode_layer& Ly = a.layers[ph.layer];
      __nv_bfloat16* kc = static_cast<__nv_bfloat16*>(Ly.k_cache);
      __nv_bfloat16* vc = static_cast<__nv_bfloat16*>(Ly.v_cache);
      const __nv_bfloat16* qkv = static_cast<const __nv_bfloat16*>(a.qkv);
      const int h = m.h, r = m.r;
      if (m.act) {
        if (tid == 0 && (!m.pos_ok || m.L_in < P + 1 || m.L_in > a.table_stride))
          report(a.status, AIOSB_DEV_POSITION_RANGE);
        if (warp <= gq) {
          float* tw = tmp + warp * D;
          float x[DPL];
          if (warp < gq) {
            const __nv_bfloat16* src = qkv + (int64_t)r * a.qkv_stride + (int64_t)(h * gq + warp) * D;
#pragma unroll
            for (int i = 0; i < DPL; ++i) x[i] = bf16_to_f(src[i * 32 + lane]);
            norm_rope<D>(x, nq, a.eps, cos_r, sin_r, true, true, lane, tw);
#pragma unroll
            for (int i = 0; i < DPL; ++i) q_s[warp * D + i * 32 + lane] = x[i];
          } else {
            const __nv_bfloat16* ksrc = qkv + (int64_t)r * a.qkv_stride + (int64_t)(a.num_qo_heads + h) * D;
            const __nv_bfloat16* vsrc =
                qkv + (int64_t)r * a.qkv_stride + (int64_t)(a.num_qo_heads + a.num_kv_heads + h) * D;
            __nv_bfloat16 vraw[DPL];
#pragma unroll
            for (int i = 0; i < DPL; ++i) {
              x[i] = bf16_to_f(ksrc[i * 32 + lane]);
              vraw[i] = vsrc[i * 32 + lane];
            }
            norm_rope<D>(x, nk, a.eps, cos_r, sin_r, true, true, lane, tw);
            const bool slot_ok = m.oslot >= 0 && m.oslot < a.num_slots;
            if (!slot_ok && lane == 0) report(a.status, AIOSB_DEV_SLOT_RANGE);
#pragma unroll
            for (int i = 0; i < DPL; ++i) {
              const __nv_bfloat16 kb = f_to_bf16(x[i]);
              Kh[m.nst * KR + i * 32 + lane] = kb;
              Vh[m.nst * D + i * 32 + lane] = vraw[i];
              if (slot_ok) {
                kc[m.oslot * tok_stride + (int64_t)h * D + i * 32 + lane] = kb;
                vc[m.oslot * tok_stride + (int64_t)h * D + i * 32 + lane] = vraw[i];
              }
            }
          }
        }
        if (tid == 0 && m.bad_slot) report(a.status, AIOSB_DEV_SLOT_RANGE);
      }
      consumer_sync();
      QState<D> st;
      qstate_init<D>(st);
      const bool mine = m.act && warp < gq;
      const int nfold = m.act ? m.nst + (m.ns_old == m.ns ? 1 : 0) : 0;
      for (int c0 = 0; c0 < nfold; c0 += kKeyChunk)
        if (mine) fold_chunk<D>(st, q_s + warp * D, Kh + c0 * KR, Vh + c0 * D, min(kKeyChunk, nfold - c0), a.scale, lane);
      // histories beyond the staged part stream from the cache: the rest of the
      // prefix, then the rest of the older suffix, then the new key
      auto stream_keys = [&](const int32_t* slots, int k0, int n) {
        for (int idx = tid; idx < n * (D / 2); idx += kCThreads) {
          const int j = idx / (D / 2), w = idx % (D / 2);
          int64_t slot = slots[k0 + j];
          if (slot < 0 || slot >= a.num_slots) {
            if (w == 0) report(a.status, AIOSB_DEV_SLOT_RANGE);
            slot = 0;
          }
          reinterpret_cast<uint32_t*>(Kw)[j * (D / 2 + 1) + w] =
              reinterpret_cast<const uint32_t*>(kc + slot * tok_stride + (int64_t)h * D)[w];
          reinterpret_cast<uint32_t*>(Vw)[j * (D / 2) + w] =
              reinterpret_cast<const uint32_t*>(vc + slot * tok_stride + (int64_t)h * D)[w];
        }
      };
      const int32_t* pslots = a.page_table + prow * a.table_stride;
      const int32_t* rslots = a.page_table + m.rrow * a.table_stride;
      if (m.act) {
        for (int k0 = m.np; k0 < P; k0 += kKeyChunk) {
          const int n = min(kKeyChunk, P - k0);
          stream_keys(pslots, k0, n);
          consumer_sync();
          if (mine) fold_chunk<D>(st, q_s + warp * D, Kw, Vw, n, a.scale, lane);
          consumer_sync();
        }
        if (m.ns_old > m.ns) {
          for (int k0 = P + m.ns; k0 < m.L - 1; k0 += kKeyChunk) {
            const int n = min(kKeyChunk, m.L - 1 - k0);
            stream_keys(rslots, k0, n);
            consumer_sync();
            if (mine) fold_chunk<D>(st, q_s + warp * D, Kw, Vw, n, a.scale, lane);
            consumer_sync();
          }
          if (mine) fold_chunk<D>(st, q_s + warp * D, Kh + m.nst * KR, Vh + m.nst * D, 1, a.scale, lane);
        }
      }
      if (warp < gq) {
        const float inv = m.act && st.l > 0.f ? 1.0f / st.l : 0.f;
        __nv_bfloat16* dst = static_cast<__nv_bfloat16*>(a.attn) + (int64_t)r * a.attn_stride + (int64_t)(h * gq + warp) * D;
#pragma unroll
        for (int i = 0; i < DPL; ++i) dst[i * 32 + lane] = f_to_bf16(st.acc[i] * inv);
      }
      consumer_sync();  // the staging area is reused by the next item
    };

    for (int p = 0; p < NP; ++p) {
      const Phase ph = phase_of(p, a);
      const int i0 = first_item(cta, offset, G);
      if (p == 0 && cta == G - 1) {
        // the residual stream starts as the embedding rows (read by the first o linear)
        for (int i = tid; i < R * (kHidden / 8); i += kCThreads) {
          const int n = i / (kHidden / 8), c = i % (kHidden / 8);
          int64_t tok = a.tokens[n];
          if (tok < 0 || tok >= a.vocab) tok = 0;  // reported by the qkv operand load
          const uint4 e = reinterpret_cast<const uint4*>(static_cast<const __nv_bfloat16*>(a.embed) + tok * kHidden)[c];
          reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(a.resid) + (int64_t)n * kHidden)[c] = e;
          float4* sx = reinterpret_cast<float4*>(a.resid_f32 + (int64_t)n * kHidden + c * 8);
          sx[0] = make_float4(bf16_lo(e.x), bf16_hi(e.x), bf16_lo(e.y), bf16_hi(e.y));
          sx[1] = make_float4(bf16_lo(e.z), bf16_hi(e.z), bf16_lo(e.w), bf16_hi(e.w));
        }
      }
      if (i0 < ph.items) {
        if (ph.kind == kATT) {
          AttnItem m = attn_stage(ph, i0);  // before the wait: the history is stable
          wait_phase(p);
          for (int it = i0; it < ph.items; it += G) {
            if (it != i0) m = attn_stage(ph, it);
            attn_run(ph, m);  // contains consumer barriers: runs on every path (after an abort its results are void)
          }
        } else {
          wait_phase(p);
          build_operand(ph);  // contains consumer barriers: runs on every path
          for (int it = i0; it < ph.items; it += G) run_tile(ph, it);
        }
      }
      consumer_sync();
      if (tid == 0) {
        __threadfence();
        atomicAdd(counters + p, 1u);
      }
      offset = (offset + ph.items) % G;
    }
    // after its last phase, the last CTA to finish resets the counters for the next launch
    if (tid == 0) {
      __threadfence();
      const uint32_t prev = atomicAdd(done_ctr, 1u);
      if (prev == (uint32_t)G - 1) {
        for (int p = 0; p <= NP + 1; ++p) atomicExch(counters + p, 0u);
        __threadfence();
      }
    }
    __syncwarp();
  }
  __syncthreads();
  // after an abort, copies the producer issued may still be landing in this CTA's
  // shared memory: wait for them (bounded) before the CTA exits
  if (threadIdx.x == 0 && abort_s) {
    const int64_t n = issued_s;
    for (int64_t j = n > nslots ? n - nslots : 0; j < n; ++j) {
      const uint64_t start = global_ns();
      while (!mbar_try_wait(&full[j % nslots], (uint32_t)(j / nslots) & 1)) {
        if (global_ns() - start > limit) break;
      }
    }
  }
}

template <int NT, int D>
int launch_step(const aiosb_decode_step_args& a, cudaStream_t stream) {
  using SM = StepSmem<NT, D>;
  auto kern = decode_step_kernel<NT, D>;
  const int nslots = SM::slots();
  const size_t smem = SM::bytes(nslots);
  static bool attr_set = false;
  if (!attr_set) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return set_error(AIOSB_ERR_LAUNCH, "decode_step: smem attribute: %s", cudaGetErrorString(e));
    attr_set = true;
  }
  const int grid = a.grid_ctas > 0 ? a.grid_ctas : sm_count();
  cudaError_t e = launch_pdl(kern, dim3((unsigned)grid), dim3(kStepThreads), smem, stream, a, nslots);
  if (e != cudaSuccess) return set_error(AIOSB_ERR_LAUNCH, "decode_step: %s", cudaGetErrorString(e));
  return AIOSB_OK;
}

}  // namespace
}  // namespace aiosb

using namespace aiosb;

extern "C" int64_t aiosb_decode_step_sync_words(int64_t num_layers) { return 5 * num_layers + 1 + 2; }

extern "C" int aiosb_decode_step(const aiosb_decode_step_args* a, void* stream) {
  AIOSB_REQUIRE(a != nullptr && a->layers != nullptr && a->sync != nullptr, AIOSB_ERR_INVALID_ARG,
                "decode_step: null pointer");
  AIOSB_REQUIRE(a->hidden == kHidden && a->intermediate == kFfn, AIOSB_ERR_UNSUPPORTED,
                "decode_step: hidden %d / intermediate %d (the kernel serves 768 / 2048)", (int)a->hidden,
                (int)a->intermediate);
  AIOSB_REQUIRE(a->head_dim == 64 || a->head_dim == 96, AIOSB_ERR_UNSUPPORTED, "decode_step: head_dim 64 or 96");
  AIOSB_REQUIRE(a->num_kv_heads >= 1 && a->num_qo_heads % a->num_kv_heads == 0 &&
                    a->num_qo_heads / a->num_kv_heads <= 7 && a->num_qo_heads * a->head_dim == kHidden,
                AIOSB_ERR_UNSUPPORTED, "decode_step: heads (q heads x head_dim = 768, at most 7 per KV head)");
  AIOSB_REQUIRE(((a->num_qo_heads + 2 * a->num_kv_heads) * a->head_dim) % 16 == 0 && a->vocab % 16 == 0 &&
                    a->vocab > 0,
                AIOSB_ERR_UNSUPPORTED, "decode_step: qkv width and vocab must be multiples of 16");
  AIOSB_REQUIRE(a->rows >= 1 && a->rows <= 16, AIOSB_ERR_UNSUPPORTED, "decode_step: 1..16 rows");
  AIOSB_REQUIRE(a->num_layers >= 1 && a->tokens && a->positions && a->out_loc && a->row_table && a->seq_lens &&
                    a->page_table && a->cos_tab && a->sin_tab && a->embed && a->final_norm && a->lm_head &&
                    a->resid_f32 && a->resid && a->qkv && a->attn && a->act && a->logits,
                AIOSB_ERR_INVALID_ARG, "decode_step: null pointer");
  AIOSB_REQUIRE(a->qkv_stride % 8 == 0 && a->attn_stride % 8 == 0 && a->act_stride % 8 == 0 &&
                    a->logits_stride % 8 == 0 && aligned16(a->qkv) && aligned16(a->attn) && aligned16(a->act) &&
                    aligned16(a->logits) && aligned16(a->resid) && aligned16(a->resid_f32) && aligned16(a->embed) &&
                    aligned16(a->lm_head),
                AIOSB_ERR_MISALIGNED, "decode_step: buffers and row strides must be 16-byte aligned");
  const cudaStream_t s = as_stream(stream);
  if (a->head_dim == 64) return a->rows <= 8 ? launch_step<1, 64>(*a, s) : launch_step<2, 64>(*a, s);
  return a->rows <= 8 ? launch_step<1, 96>(*a, s) : launch_step<2, 96>(*a, s);
}
