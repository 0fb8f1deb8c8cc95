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
//   * activations pass between phases as flagged lines (the low-latency protocol
//     of collective libraries): each 16-byte line holds two 32-bit data words and
//     two copies of a 32-bit flag, written by one 16-byte store, and the flag
//     names the launch and the phase that wrote the line. A consumer polls exactly
//     the lines it reads until both flags carry the expected value, so a phase
//     starts on a CTA as soon as its own inputs exist: one store-to-load hop, no
//     fence, no grid-wide barrier, and CTAs with nothing to do in a phase skip it.
//     A buffer is rewritten only by a phase that transitively consumed every
//     reader of its previous contents (qkv -> attention -> o -> gate/up -> down ->
//     next qkv each need ALL outputs of the phase before), and the phase field of
//     the flag tells a value of layer l from one of layer l - 1.
// Every wait is bounded (a time limit; a global abort word ends the other CTAs'
// waits at once) and reports AIOSB_DEV_WAIT_TIMEOUT through the status word.
// The consumer warps' control flow never depends on the abort flag, so their
// named barriers always match up; an abort only cuts waits short and MMAs out,
// and the launch's outputs are then void.
//
// Linears: register-operand mma.sync m16n8k16 (bf16 in, fp32 accumulate) with the
// K-permuted fragment layout of gemv.cu: lane (g, t) reads 16 contiguous bytes of
// weight rows g and g + 8 and of token row g per 32-wide K block, so every
// fragment is one 16-byte load; the 8 warps split K and their partial tiles are
// summed in warp order, for up to 4 of the CTA's tiles of a phase at once. The
// slot rows are padded to 1600 bytes (a 16-bank offset between consecutive rows),
// so the A-fragment reads are conflict-free. RMSNorm is folded into the operand
// load from the fp32 residual stream, as in the GEMV.
// Attention: one item per (KV head, row): the key history (prefix and older
// suffix, written by earlier launches) is staged in shared memory before the
// wait, then q/k RMSNorm + bf16 RoPE, the new K/V store and one online-softmax
// pass per 64 keys, as attn_decode_hist_kernel (attention.cu) does.
// Rounding points equal the per-kernel path: bf16 linear outputs, gate/up rounded
// before SwiGLU, the delta rounded before the residual add, the bf16 residual
// being the rounding of the fp32 residual stream.
#include <algorithm>

#include "abi_util.h"
#include "attn_device.cuh"
#include "common.cuh"

namespace aiosb {
namespace {

constexpr int kCWarps = 8;                    // consumer warps
constexpr int kCThreads = kCWarps * 32;       // 256
constexpr int kStepThreads = kCThreads + 32;  // + the producer warp
constexpr int kHidden = 768;
constexpr int kFfn = 2048;
constexpr int kChunkK = 768;                 // K elements of one weight slot
constexpr int kRowPitch = kChunkK * 2 + 64;  // padded slot row (bytes)
constexpr int kSlotBytes = 16 * kRowPitch;   // 25600
constexpr int kMaxSlots = 8;
constexpr int kMaxChunks = (kFfn + kChunkK - 1) / kChunkK;  // 3 weight chunks per tile at K = 2048
constexpr int kOpBlocks = kMaxChunks * 3;    // operand fragment slots per lane: (chunk, 32-wide block)
// tiles of a phase reduced together (fewer at 16 rows, whose accumulators are twice as many)
template <int NT>
constexpr int batch_of() { return NT == 1 ? 4 : 2; }
constexpr int kSPrefix = 64;                 // staged prefix keys per attention item
constexpr int kSSuffix = 32;                 // staged suffix keys (incl. the new one)
constexpr int kSmemLimit = 232448;           // 227 KB opt-in per CTA
constexpr int kWorkRows = 16;                // rows the work area is laid out for
constexpr int kMaxLayers = 48;               // phase index < 256 inside the flag
constexpr uint32_t kEpochWrap = 1u << 24;    // flag = (epoch << 8) + phase + 1

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
    default: return {kDN, l, kHidden / 16, kMaxChunks};
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

// ---- the work area: flagged 16-byte lines {d0, flag, d1, flag} -----------------
// residual stream s: fp32, 2 values per line  [kWorkRows][768 / 2]
// qkv projection:    bf16, 4 values per line  [kWorkRows][nqkv / 4]
// attention output:  bf16                     [kWorkRows][768 / 4]
// SwiGLU activation: bf16                     [kWorkRows][2048 / 4]
struct Work {
  uint4* s;
  uint4* qkv;
  uint4* attn;
  uint4* act;
  int qkv_lines;  // lines per qkv row
};
__host__ __device__ inline int64_t work_lines(int64_t nqkv) {
  return kWorkRows * (kHidden / 2 + nqkv / 4 + kHidden / 4 + kFfn / 4);
}
__device__ __forceinline__ Work work_of(void* base, int nqkv) {
  uint4* w = static_cast<uint4*>(base);
  Work k;
  k.s = w;
  k.qkv = k.s + kWorkRows * (kHidden / 2);
  k.qkv_lines = nqkv / 4;
  k.attn = k.qkv + kWorkRows * (nqkv / 4);
  k.act = k.attn + kWorkRows * (kHidden / 4);
  return k;
}

__device__ __forceinline__ void st_line(uint4* p, uint32_t d0, uint32_t d1, uint32_t flag) {
  asm volatile("st.volatile.global.v4.u32 [%0], {%1,%2,%3,%4};" ::"l"(p), "r"(d0), "r"(flag), "r"(d1), "r"(flag)
               : "memory");
}
__device__ __forceinline__ uint4 ld_line(const uint4* p) {
  uint4 v;
  asm volatile("ld.volatile.global.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p)
               : "memory");
  return v;
}
__device__ __forceinline__ bool line_ok(const uint4& v, uint32_t flag) { return v.y == flag && v.w == flag; }
// One polling pass over a thread's set of flagged lines: line `bit` of the set is
// loaded only while it is still missing from `have`; returns the line when it
// now carries `flag` (its data is then final), and records it in `have`.
__device__ __forceinline__ bool poll_line(const uint4* line, uint32_t flag, uint32_t bit, uint32_t& have, uint4& v) {
  if (have & bit) return false;
  v = ld_line(line);
  if (!line_ok(v, flag)) return false;
  have |= bit;
  return true;
}
__device__ __forceinline__ uint32_t ld_relaxed_u32(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Barrier of the 8 consumer warps (the producer warp never joins it). Lanes that
// diverged reconverge first.
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

// Source of weight row `row` (0..15) of tile `item` of a phase.
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
  static constexpr int kRed = batch_of<NT>() * kCWarps * NT * 32 * 4 * 4;
  static constexpr int kTile = batch_of<NT>() * TM * 17 * 4;
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
  static constexpr int kSlotIds = (kSPrefix + kSSuffix) * 4;
  static constexpr int kIn = 10 * D * 2;         // this step's q heads + k + v of the item (bf16)
  static constexpr int kAttn = kQ + kTmp + kKh + kVh + kKw + kVw + kRope + kSlotIds + kIn;
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
  constexpr int kBatch = batch_of<NT>();
  extern __shared__ __align__(128) uint8_t smem[];
  uint8_t* ring = smem;
  uint8_t* scratch = smem + (size_t)nslots * kSlotBytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(scratch + SM::kScratch);
  uint64_t* empty = full + kMaxSlots;
  __shared__ volatile int abort_s;
  __shared__ volatile int last_s;
  __shared__ volatile int64_t issued_s;

  const int G = gridDim.x, cta = blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int NP = 5 * a.num_layers + 1;
  uint32_t* done_ctr = a.sync;
  uint32_t* abort_g = a.sync + 1;
  uint32_t* epoch_g = a.sync + 2;
  const uint64_t limit = a.wait_limit_ns != 0 ? a.wait_limit_ns : kWaitLimitNs;
  const int R = a.rows;
  const int nqkv = (a.num_qo_heads + 2 * a.num_kv_heads) * a.head_dim;
  const Work wk = work_of(a.work, nqkv);

  if (threadIdx.x == 0) {
    for (int s = 0; s < nslots; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kCWarps);
    }
    abort_s = 0;
    last_s = 0;
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
    const uint32_t epoch = *epoch_g;  // advanced by the previous launch's last CTA
    // flag a phase writes, and the one a consumer of that phase's output expects
    auto wflag = [&](int p) { return (epoch << 8) + (uint32_t)p + 1u; };
    auto rflag = [&](int p) { return wflag(p) + a.test_flag_skew; };
    // Waits until every flagged line this thread reads is present. Each call of
    // `pass` loads, in parallel, the lines still missing (one L2 round trip) and
    // returns true once none is; a line is loaded again only while it is missing.
    // The wait is bounded; the global abort word is only looked at once a wait has
    // lasted 20 us (ordinary waits are a few microseconds), so the spinning
    // threads of all CTAs do not poll one shared address.
    auto wait_lines = [&](auto&& pass) {
      if (pass()) return;
      const uint64_t start = global_ns();
      uint32_t spins = 0;
      while (!pass()) {
        if (abort_s) return;
        const uint64_t waited = global_ns() - start;
        if (waited > 20000 && (++spins & 15) == 0 && ld_relaxed_u32(abort_g) != 0) {
          abort_s = 1;
          return;
        }
        if (waited > limit) {
          fail(AIOSB_DEV_WAIT_TIMEOUT);
          return;
        }
      }
    };
    float* red = reinterpret_cast<float*>(scratch);              // [batch][warp][nt][lane][4]
    float* tile = reinterpret_cast<float*>(scratch + SM::kRed);  // [batch][TM][17]
    float* ssw = reinterpret_cast<float*>(scratch + SM::kRed + SM::kTile);  // [warp][TM]
    const int gq = a.num_qo_heads / a.num_kv_heads;
    int64_t seq = 0;
    int offset = 0;

    // ---- operand fragments of a linear phase (token rows in the B layout)
    uint4 xb[NT][kOpBlocks];  // [token tile][chunk * 3 + block]
    auto build_operand = [&](const Phase& ph, int p) {
      if (ph.kind == kO || ph.kind == kDN) {
        // plain bf16 rows: attention output (o) or SwiGLU activation (down), both
        // written by the phase just before
        const uint4* src = ph.kind == kO ? wk.attn : wk.act;
        const int row_lines = ph.kind == kO ? kHidden / 4 : kFfn / 4;
        const uint32_t f = rflag(p - 1);
#pragma unroll
        for (int c = 0; c < kMaxChunks; ++c)
#pragma unroll
          for (int j = 0; j < 3; ++j)
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) xb[nt][c * 3 + j] = make_uint4(0u, 0u, 0u, 0u);
        uint32_t have = 0;  // bit (c * 3 + j) * NT * 2 + nt * 2 + q: line q of block (c, j), token tile nt
        wait_lines([&]() {
          bool all = true;
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
                  if (n < R) {
                    const uint4* ln = src + (int64_t)n * row_lines + k / 4;
                    const uint32_t bit = 1u << (((c * 3 + j) * NT + nt) * 2);
                    uint4 v;
                    if (poll_line(ln, f, bit, have, v)) {
                      xb[nt][c * 3 + j].x = v.x;
                      xb[nt][c * 3 + j].y = v.z;
                    }
                    if (poll_line(ln + 1, f, bit << 1, have, v)) {
                      xb[nt][c * 3 + j].z = v.x;
                      xb[nt][c * 3 + j].w = v.z;
                    }
                    all = all && (have & bit) && (have & (bit << 1));
                  }
                }
              }
            }
          }
          return all;
        });
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
      if (embed) {
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
          const int n = nt * 8 + g;
          int64_t tok = 0;
          if (n < R) {
            tok = a.tokens[n];
            if (tok < 0 || tok >= a.vocab) {
              if (t4 == 0 && warp == 0) report(a.status, AIOSB_DEV_TOKEN_RANGE);
              tok = 0;
            }
          }
#pragma unroll
          for (int j = 0; j < 3; ++j) {
            const int k = (warp * 3 + j) * 32 + 8 * t4;
            if (n < R) {
              const uint4 e = *reinterpret_cast<const uint4*>(static_cast<const __nv_bfloat16*>(a.embed) +
                                                              tok * kHidden + k);
              sv[nt][j][0] = make_float4(bf16_lo(e.x), bf16_hi(e.x), bf16_lo(e.y), bf16_hi(e.y));
              sv[nt][j][1] = make_float4(bf16_lo(e.z), bf16_hi(e.z), bf16_lo(e.w), bf16_hi(e.w));
            } else {
              sv[nt][j][0] = sv[nt][j][1] = make_float4(0.f, 0.f, 0.f, 0.f);
            }
          }
        }
      } else {
        // the residual stream after the previous residual add: this layer's o (for
        // gate/up, one phase back) or the previous layer's down (for qkv and the LM
        // head, one phase back as well)
        const uint32_t f = rflag(p - 1);
        uint32_t have = 0;  // bit ((nt * 3 + j) * 4 + q): line q of block j, token tile nt
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
          for (int j = 0; j < 3; ++j) sv[nt][j][0] = sv[nt][j][1] = make_float4(0.f, 0.f, 0.f, 0.f);
        wait_lines([&]() {
          bool all = true;
#pragma unroll
          for (int nt = 0; nt < NT; ++nt) {
            const int n = nt * 8 + g;
            if (n < R) {
#pragma unroll
              for (int j = 0; j < 3; ++j) {
                const int k = (warp * 3 + j) * 32 + 8 * t4;
                const uint4* ln = wk.s + (int64_t)n * (kHidden / 2) + k / 2;
                const uint32_t bit = 1u << ((nt * 3 + j) * 4);
                uint4 v;
                if (poll_line(ln, f, bit, have, v)) {
                  sv[nt][j][0].x = __uint_as_float(v.x);
                  sv[nt][j][0].y = __uint_as_float(v.z);
                }
                if (poll_line(ln + 1, f, bit << 1, have, v)) {
                  sv[nt][j][0].z = __uint_as_float(v.x);
                  sv[nt][j][0].w = __uint_as_float(v.z);
                }
                if (poll_line(ln + 2, f, bit << 2, have, v)) {
                  sv[nt][j][1].x = __uint_as_float(v.x);
                  sv[nt][j][1].y = __uint_as_float(v.z);
                }
                if (poll_line(ln + 3, f, bit << 3, have, v)) {
                  sv[nt][j][1].z = __uint_as_float(v.x);
                  sv[nt][j][1].w = __uint_as_float(v.z);
                }
                all = all && ((have >> ((nt * 3 + j) * 4)) & 15u) == 15u;
              }
            }
          }
          return all;
        });
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

    // ---- up to kBatch tiles of a phase: MMAs over their chunks, one warp-order
    // reduction for all of them, then their epilogues
    auto run_tiles = [&](const Phase& ph, int p, int first) {
      const int nb = min(kBatch, (ph.items - first + G - 1) / G);
      float d[kBatch][NT][4];
#pragma unroll
      for (int b = 0; b < kBatch; ++b)
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) d[b][nt][0] = d[b][nt][1] = d[b][nt][2] = d[b][nt][3] = 0.f;
#pragma unroll
      for (int b = 0; b < kBatch; ++b) {
        if (b < nb) {
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
                      mma16816(d[b][nt], wa.x, wb.x, wa.y, wb.y, x.x, x.y);
                      mma16816(d[b][nt], wa.z, wb.z, wa.w, wb.w, x.z, x.w);
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
            *reinterpret_cast<float4*>(&red[(((b * kCWarps + warp) * NT + nt) * 32 + lane) * 4]) =
                make_float4(d[b][nt][0], d[b][nt][1], d[b][nt][2], d[b][nt][3]);
        }
      }
      consumer_sync();
      for (int i = tid; i < nb * NT * 128; i += kCThreads) {
        const int b = i / (NT * 128), e = i % (NT * 128);
        const int nt = e / 128, l = (e / 4) % 32, j = e % 4;
        float sum = 0.f;
#pragma unroll
        for (int w = 0; w < kCWarps; ++w) sum += red[(((b * kCWarps + w) * NT + nt) * 32 + l) * 4 + j];
        tile[(b * TM + nt * 8 + 2 * (l & 3) + (j & 1)) * 17 + (l >> 2) + 8 * (j >> 1)] = sum;
      }
      consumer_sync();
      // ---- epilogues: thread (tile b, token, half) writes 8 output features
      if (tid < nb * TM * 2) {
        const int b = tid / (TM * 2), tk = (tid >> 1) % TM, h = tid & 1;
        const int item = first + b * G;
        const float* tr = tile + (b * TM + tk) * 17;
        const uint32_t f = wflag(p);
        if (tk < R) {
          if (ph.kind == kGU) {
            if (h == 0) {
              float o[8];
#pragma unroll
              for (int j = 0; j < 8; ++j) {
                // gate_up output is bf16 before silu_and_mul (aios/models/qwen3.py:90-92)
                const float gt = round_bf16(tr[j]), up = round_bf16(tr[8 + j]);
                o[j] = gt / (1.0f + expf(-gt)) * up;
              }
              uint4* dst = wk.act + (int64_t)tk * (kFfn / 4) + (item * 8) / 4;
              st_line(dst, pack_bf16x2(o[0], o[1]), pack_bf16x2(o[2], o[3]), f);
              st_line(dst + 1, pack_bf16x2(o[4], o[5]), pack_bf16x2(o[6], o[7]), f);
            }
          } else if (ph.kind == kO || ph.kind == kDN) {
            // residual add (aios/layers/norm.py:34-40): residual = bf16(s_old), the
            // delta rounded to bf16, s = residual + delta in fp32 kept for the next norm
            const int f0 = item * 16 + 8 * h;
            uint4* sl = wk.s + (int64_t)tk * (kHidden / 2) + f0 / 2;
            float s_old[8];
            if (ph.kind == kO && ph.layer == 0) {
              int64_t tok = a.tokens[tk];
              if (tok < 0 || tok >= a.vocab) tok = 0;  // reported by the qkv operand load
              const uint4 e = *reinterpret_cast<const uint4*>(static_cast<const __nv_bfloat16*>(a.embed) +
                                                              tok * kHidden + f0);
              const uint32_t q[4] = {e.x, e.y, e.z, e.w};
#pragma unroll
              for (int j = 0; j < 8; ++j) s_old[j] = (j & 1) ? bf16_hi(q[j >> 1]) : bf16_lo(q[j >> 1]);
            } else {
              // s of these columns: written by the previous layer's down (for o, three
              // phases back) or by this layer's o (for down, two phases back)
              const uint32_t fin = rflag(ph.kind == kO ? p - 3 : p - 2);
              uint4 v[4];
              uint32_t have = 0;
              wait_lines([&]() {
#pragma unroll
                for (int q = 0; q < 4; ++q) poll_line(sl + q, fin, 1u << q, have, v[q]);
                return have == 15u;
              });
#pragma unroll
              for (int q = 0; q < 4; ++q) {
                s_old[2 * q] = __uint_as_float(v[q].x);
                s_old[2 * q + 1] = __uint_as_float(v[q].z);
              }
            }
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              const float o0 = round_bf16(s_old[2 * q]) + round_bf16(tr[8 * h + 2 * q]);
              const float o1 = round_bf16(s_old[2 * q + 1]) + round_bf16(tr[8 * h + 2 * q + 1]);
              st_line(sl + q, __float_as_uint(o0), __float_as_uint(o1), f);
            }
          } else if (ph.kind == kQKV) {
            const int f0 = item * 16 + 8 * h;
            uint4* dst = wk.qkv + (int64_t)tk * wk.qkv_lines + f0 / 4;
            st_line(dst, pack_bf16x2(tr[8 * h + 0], tr[8 * h + 1]), pack_bf16x2(tr[8 * h + 2], tr[8 * h + 3]), f);
            st_line(dst + 1, pack_bf16x2(tr[8 * h + 4], tr[8 * h + 5]), pack_bf16x2(tr[8 * h + 6], tr[8 * h + 7]),
                    f);
          } else {  // LM head: plain bf16 logits for the next kernel
            const int64_t f0 = (int64_t)item * 16 + 8 * h;
            *reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(a.logits) + (int64_t)tk * a.logits_stride + f0) =
                make_uint4(pack_bf16x2(tr[8 * h + 0], tr[8 * h + 1]), pack_bf16x2(tr[8 * h + 2], tr[8 * h + 3]),
                           pack_bf16x2(tr[8 * h + 4], tr[8 * h + 5]), pack_bf16x2(tr[8 * h + 6], tr[8 * h + 7]));
          }
        }
      }
      consumer_sync();  // `tile` and `red` are rewritten by the next batch
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
    __nv_bfloat16* in_s = reinterpret_cast<__nv_bfloat16*>(slot_s + kSPrefix + kSSuffix);  // [gq + 2][D]
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
    auto attn_run = [&](const Phase& ph, int p, const AttnItem& m) {
      const aiosb_decode_layer& Ly = a.layers[ph.layer];
      __nv_bfloat16* kc = static_cast<__nv_bfloat16*>(Ly.k_cache);
      __nv_bfloat16* vc = static_cast<__nv_bfloat16*>(Ly.v_cache);
      const int h = m.h, r = m.r;
      // this step's projection row of the item: q heads h*gq.., k head h, v head h
      // (flagged lines of the qkv phase), D / 4 lines per head vector
      const int lines = (gq + 2) * (D / 4);
      if (tid < lines) {
        const int v = tid / (D / 4), c = tid % (D / 4);
        const int head = v < gq ? h * gq + v : (v == gq ? a.num_qo_heads + h : a.num_qo_heads + a.num_kv_heads + h);
        const uint4* ln = wk.qkv + (int64_t)r * wk.qkv_lines + (head * D) / 4 + c;
        const uint32_t f = rflag(p - 1);
        uint4 val = make_uint4(0u, 0u, 0u, 0u);
        uint32_t have = 0;
        wait_lines([&]() { return poll_line(ln, f, 1u, have, val) || have != 0u; });
        reinterpret_cast<uint2*>(in_s)[v * (D / 4) + c] = make_uint2(val.x, val.z);
      }
      consumer_sync();
      if (m.act) {
        if (tid == 0 && (!m.pos_ok || m.L_in < P + 1 || m.L_in > a.table_stride))
          report(a.status, AIOSB_DEV_POSITION_RANGE);
        if (warp <= gq) {
          float* tw = tmp + warp * D;
          float x[DPL];
          if (warp < gq) {
            const __nv_bfloat16* src = in_s + warp * D;
#pragma unroll
            for (int i = 0; i < DPL; ++i) x[i] = bf16_to_f(src[i * 32 + lane]);
            norm_rope<D>(x, nq, a.eps, cos_r, sin_r, true, true, lane, tw);
#pragma unroll
            for (int i = 0; i < DPL; ++i) q_s[warp * D + i * 32 + lane] = x[i];
          } else {
            const __nv_bfloat16* ksrc = in_s + gq * D;
            const __nv_bfloat16* vsrc = in_s + (gq + 1) * D;
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
      // normalise (zeros for an inactive row) and publish as flagged lines: the
      // warp's head vector goes through its tmp row, lanes 0 .. D/4-1 store a line each
      if (warp < gq) {
        const float inv = m.act && st.l > 0.f ? 1.0f / st.l : 0.f;
        __nv_bfloat16* ob = reinterpret_cast<__nv_bfloat16*>(tmp + warp * D);
#pragma unroll
        for (int i = 0; i < DPL; ++i) ob[i * 32 + lane] = f_to_bf16(st.acc[i] * inv);
        __syncwarp();
        if (lane < D / 4) {
          const uint2 v = reinterpret_cast<const uint2*>(ob)[lane];
          st_line(wk.attn + (int64_t)r * (kHidden / 4) + ((h * gq + warp) * D) / 4 + lane, v.x, v.y, wflag(p));
        }
      }
      consumer_sync();  // the staging area is reused by the next item
    };

    for (int p = 0; p < NP; ++p) {
      const Phase ph = phase_of(p, a);
      const int i0 = first_item(cta, offset, G);
      if (i0 < ph.items) {
        if (ph.kind == kATT) {
          for (int it = i0; it < ph.items; it += G) attn_run(ph, p, attn_stage(ph, it));
        } else {
          build_operand(ph, p);  // waits for this phase's inputs
          for (int b0 = i0; b0 < ph.items; b0 += kBatch * G) run_tiles(ph, p, b0);
        }
      }
      offset = (offset + ph.items) % G;
    }
    // after its last phase, the last CTA to finish advances the flag epoch for the
    // next launch (and, once every 2^24 launches, clears the work area so that no
    // line from the previous cycle can carry a flag of the next)
    if (tid == 0) {
      __threadfence();
      const uint32_t prev = atomicAdd(done_ctr, 1u);
      last_s = prev == (uint32_t)G - 1 ? 1 : 0;
    }
    consumer_sync();
    if (last_s) {
      const bool wrap = epoch + 1 >= kEpochWrap;
      if (wrap) {
        const int64_t n = work_lines(nqkv);
        for (int64_t i = tid; i < n; i += kCThreads) static_cast<uint4*>(a.work)[i] = make_uint4(0u, 0u, 0u, 0u);
      }
      consumer_sync();
      if (tid == 0) {
        __threadfence();
        atomicExch(epoch_g, wrap ? 0u : epoch + 1);
        atomicExch(abort_g, 0u);
        atomicExch(done_ctr, 0u);
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

extern "C" int64_t aiosb_decode_step_work_bytes(int64_t num_qo_heads, int64_t num_kv_heads, int64_t head_dim) {
  return work_lines((num_qo_heads + 2 * num_kv_heads) * head_dim) * 16;
}

extern "C" int64_t aiosb_decode_step_sync_words(void) { return 4; }

extern "C" int aiosb_decode_step(const aiosb_decode_step_args* a, void* stream) {
  AIOSB_REQUIRE(a != nullptr && a->layers != nullptr && a->sync != nullptr && a->work != nullptr,
                AIOSB_ERR_INVALID_ARG, "decode_step: null pointer");
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
  AIOSB_REQUIRE(a->rows >= 1 && a->rows <= kWorkRows, AIOSB_ERR_UNSUPPORTED, "decode_step: 1..16 rows");
  AIOSB_REQUIRE(a->num_layers >= 1 && a->num_layers <= kMaxLayers, AIOSB_ERR_UNSUPPORTED,
                "decode_step: 1..%d layers", kMaxLayers);
  AIOSB_REQUIRE(a->tokens && a->positions && a->out_loc && a->row_table && a->seq_lens && a->page_table &&
                    a->cos_tab && a->sin_tab && a->embed && a->final_norm && a->lm_head && a->logits,
                AIOSB_ERR_INVALID_ARG, "decode_step: null pointer");
  AIOSB_REQUIRE(a->logits_stride % 8 == 0 && aligned16(a->logits) && aligned16(a->work) && aligned16(a->embed) &&
                    aligned16(a->lm_head),
                AIOSB_ERR_MISALIGNED, "decode_step: buffers and row strides must be 16-byte aligned");
  const cudaStream_t s = as_stream(stream);
  if (a->head_dim == 64) return a->rows <= 8 ? launch_step<1, 64>(*a, s) : launch_step<2, 64>(*a, s);
  return a->rows <= 8 ? launch_step<1, 96>(*a, s) : launch_step<2, 96>(*a, s);
}
