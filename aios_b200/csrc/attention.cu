// Paged GQA attention for the CandidateGroup path (replaces the FlashInfer
// paged prefill/decode wrappers of aios/attention/flashinfer.py and the SDPA
// fallback _sdpa_prefill_attention, aios/attention/flashinfer.py:33-91).
//
// KV layout: the reference MHAKVCache buffer [2, L, pages, page_size, Hkv, d]
// (aios/kvcache/mha_pool.py:28-37). A token slot s (= page * page_size + offset)
// of one layer lives at k_cache + s * Hkv * d, so every kernel takes a per-token
// slot table ("page table", [rows, max_len] int32) and works for page_size 1
// and 16 alike.
//
// Decode is a cascade: one CTA per KV head stages each shared-prefix KV slot in
// shared memory ONCE and scores it against all rows x GQA-group query heads,
// then adds each row's own suffix slots; partial softmax states merge online.
// The decode kernel also owns the step's q/k RMSNorm, bf16 RoPE and the KV store
// of the new token (aios/models/qwen3.py:60-70 + aios/kernel/store.py), so the
// raw qkv projection output is its only input.
#include <algorithm>

#include "abi_util.h"
#include "attn_device.cuh"
#include "common.cuh"

namespace aiosb {
namespace {

constexpr int kAttnThreads = 256;
constexpr int kAttnWarps = kAttnThreads / 32;
constexpr int kMaxQPerWarp = 8;
constexpr int kMaxQueries = kAttnWarps * kMaxQPerWarp;  // 64 query vectors per CTA

struct DecodeArgs {
  // fused prologue inputs (qkv != nullptr) or pre-rotated q (q != nullptr)
  const __nv_bfloat16* qkv;  // [R, qkv_stride]: q heads | k heads | v heads (raw projection)
  int64_t qkv_stride;
  const __nv_bfloat16* q;  // [R, q_stride] already normalised/rotated (no prologue)
  int64_t q_stride;
  const __nv_bfloat16* q_norm_w;
  const __nv_bfloat16* k_norm_w;
  float eps;
  const __nv_bfloat16* cos_tab;  // [max_pos, D] bf16
  const __nv_bfloat16* sin_tab;
  int max_pos;
  const int32_t* positions;  // [R]
  const int32_t* out_loc;    // [R] slot of the new token
  // cache + slot table
  __nv_bfloat16* k_cache;
  __nv_bfloat16* v_cache;
  int64_t num_slots;
  const int32_t* page_table;
  int64_t table_stride;
  const int32_t* row_table;   // [R] page-table row of each local row
  const int32_t* seq_lens;    // [R] keys per row including the new token
  const int32_t* prefix_len;  // device scalar: shared prefix keys (0 = none)
  const int32_t* active;      // [R] nonzero = row runs; nullptr = all rows
  int stage_cap;              // history-staged kernel: prefix keys staged before the wait
  int rows, hq, hkv;
  float scale;
  __nv_bfloat16* out;  // [R, out_stride]
  int64_t out_stride;
  int32_t* status;
};

// ---- cascade decode -----------------------------------------------------------
// CTA (h, r) owns KV head h of candidate row r; the R CTAs of a head form one
// thread-block cluster. The shared prefix is split into 64-key chunks; chunk c
// is fetched from HBM once, by CTA c % R, into that CTA's shared memory, and the
// other rows of the head copy it over distributed shared memory. Each CTA then
// folds the prefix chunks and its own row's suffix keys into the online softmax
// of its g query heads (one warp per query head). Chunks beyond the cluster's
// staging capacity, and every key when the launch has no cluster, are read from
// the paged cache directly.
constexpr int kDecThreads = 128;
constexpr int kDecWarps = kDecThreads / 32;
constexpr int kStageChunks = 2;  // prefix chunks one CTA keeps for its cluster peers
constexpr int kMaxGroupQ = 2 * kDecWarps;

__device__ __forceinline__ uint4 ld_dsmem_u4(uint32_t addr) {
  uint4 v;
  asm volatile("ld.shared::cluster.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "r"(addr));
  return v;
}

template <int D>
__global__ void __launch_bounds__(kDecThreads) attn_decode_kernel(const DecodeArgs a, int cluster_rows) {
  constexpr int DPL = D / 32;
  constexpr int kKChunk = kKeyChunk * (D + 2);  // bf16 elements of one staged K chunk
  constexpr int kVChunk = kKeyChunk * D;
  extern __shared__ __align__(16) uint8_t smem_raw[];
  const int h = blockIdx.x;
  const int r = blockIdx.y;
  const int g = a.hq / a.hkv;
  float* q_s = reinterpret_cast<float*>(smem_raw);  // [g][D]
  float* tmp = q_s + g * D;                          // [warps][D]
  __nv_bfloat16* stK = reinterpret_cast<__nv_bfloat16*>(tmp + kDecWarps * D);
  __nv_bfloat16* stV = stK + kStageChunks * kKChunk;
  __nv_bfloat16* wK = stV + kStageChunks * kVChunk;
  __nv_bfloat16* wV = wK + kKChunk;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t tok_stride = (int64_t)a.hkv * D;
  const bool clustered = cluster_rows > 1;

  pdl_enter();
  const int P = a.prefix_len != nullptr ? *a.prefix_len : 0;
  const bool act = a.active == nullptr || a.active[r] != 0;

  // ---- prologue: q heads of this group + the new k/v of head h, for row r.
  if (act) {
    for (int it = warp; it < g + 1; it += kDecWarps) {
      float* tw = tmp + warp * D;
      float x[DPL];
      int pos = a.positions[r];
      if (pos < 0 || pos >= a.max_pos) {
        if (lane == 0 && a.qkv != nullptr) report(a.status, AIOSB_DEV_POSITION_RANGE);
        pos = 0;
      }
      if (it < g) {
        const int qh = h * g + it;
        if (a.qkv != nullptr) {
          const __nv_bfloat16* src = a.qkv + (int64_t)r * a.qkv_stride + (int64_t)qh * D;
#pragma unroll
          for (int i = 0; i < DPL; ++i) x[i] = bf16_to_f(src[i * 32 + lane]);
          norm_rope<D>(x, a.q_norm_w, a.eps, a.cos_tab + (int64_t)pos * D, a.sin_tab + (int64_t)pos * D, true,
                       true, lane, tw);
        } else {
          const __nv_bfloat16* src = a.q + (int64_t)r * a.q_stride + (int64_t)qh * D;
#pragma unroll
          for (int i = 0; i < DPL; ++i) x[i] = bf16_to_f(src[i * 32 + lane]);
        }
#pragma unroll
        for (int i = 0; i < DPL; ++i) q_s[it * D + i * 32 + lane] = x[i];
      } else if (a.qkv != nullptr) {
        const __nv_bfloat16* ksrc = a.qkv + (int64_t)r * a.qkv_stride + (int64_t)(a.hq + h) * D;
        const __nv_bfloat16* vsrc = a.qkv + (int64_t)r * a.qkv_stride + (int64_t)(a.hq + a.hkv + h) * D;
#pragma unroll
        for (int i = 0; i < DPL; ++i) x[i] = bf16_to_f(ksrc[i * 32 + lane]);
        norm_rope<D>(x, a.k_norm_w, a.eps, a.cos_tab + (int64_t)pos * D, a.sin_tab + (int64_t)pos * D, true, true,
                     lane, tw);
        const int64_t slot = a.out_loc[r];
        if (slot >= 0 && slot < a.num_slots) {
          __nv_bfloat16* kd = a.k_cache + slot * tok_stride + (int64_t)h * D;
          __nv_bfloat16* vd = a.v_cache + slot * tok_stride + (int64_t)h * D;
#pragma unroll
          for (int i = 0; i < DPL; ++i) {
            kd[i * 32 + lane] = f_to_bf16(x[i]);
            vd[i * 32 + lane] = vsrc[i * 32 + lane];
          }
        } else if (lane == 0) {
          report(a.status, AIOSB_DEV_SLOT_RANGE);
        }
      }
    }
  }

  // ---- stage this CTA's share of the prefix (chunks r, r + R, ...).
  const int nchunks = (P + kKeyChunk - 1) / kKeyChunk;
  const int32_t* pslots = a.page_table + (int64_t)a.row_table[0] * a.table_stride;
  if (clustered) {
    for (int s = 0; s < kStageChunks; ++s) {
      const int c = r + s * cluster_rows;
      if (c < nchunks)
        stage_chunk<D>(a.k_cache, a.v_cache, tok_stride, h, pslots, c * kKeyChunk, min(kKeyChunk, P - c * kKeyChunk),
                       a.num_slots, stK + s * kKChunk, stV + s * kVChunk, a.status);
    }
  }
  __syncthreads();  // q_s ready, staged chunks ready, new K/V visible to this CTA
  if (clustered) cluster_sync();

  QState<D> st[2];
  qstate_init<D>(st[0]);
  qstate_init<D>(st[1]);

  // ---- shared prefix
  for (int c = 0; c < nchunks; ++c) {
    const int nk = min(kKeyChunk, P - c * kKeyChunk);
    const __nv_bfloat16* K = wK;
    const __nv_bfloat16* V = wV;
    const int owner = clustered ? c % cluster_rows : 0;
    const int slot = clustered ? c / cluster_rows : kStageChunks;
    if (slot < kStageChunks && owner == r) {
      K = stK + slot * kKChunk;
      V = stV + slot * kVChunk;
    } else if (slot < kStageChunks) {
      const uint32_t rk = map_shared_rank(smem_u32(stK + slot * kKChunk), (uint32_t)owner);
      const uint32_t rv = map_shared_rank(smem_u32(stV + slot * kVChunk), (uint32_t)owner);
      for (int i = threadIdx.x; i < kKChunk / 8; i += kDecThreads)
        reinterpret_cast<uint4*>(wK)[i] = ld_dsmem_u4(rk + i * 16);
      for (int i = threadIdx.x; i < kVChunk / 8; i += kDecThreads)
        reinterpret_cast<uint4*>(wV)[i] = ld_dsmem_u4(rv + i * 16);
      __syncthreads();
    } else {
      stage_chunk<D>(a.k_cache, a.v_cache, tok_stride, h, pslots, c * kKeyChunk, nk, a.num_slots, wK, wV, a.status);
      __syncthreads();
    }
    if (act) {
#pragma unroll
      for (int t = 0; t < 2; ++t) {
        const int j = warp + t * kDecWarps;
        if (j < g) fold_chunk<D>(st[t], q_s + j * D, K, V, nk, a.scale, lane);
      }
    }
    __syncthreads();
  }

  // ---- this row's own keys [P, seq_len)
  if (act) {
    const int32_t* rslots = a.page_table + (int64_t)a.row_table[r] * a.table_stride;
    const int L = a.seq_lens[r];
    for (int k0 = P; k0 < L; k0 += kKeyChunk) {
      const int nk = min(kKeyChunk, L - k0);
      stage_chunk<D>(a.k_cache, a.v_cache, tok_stride, h, rslots, k0, nk, a.num_slots, wK, wV, a.status);
      __syncthreads();
#pragma unroll
      for (int t = 0; t < 2; ++t) {
        const int j = warp + t * kDecWarps;
        if (j < g) fold_chunk<D>(st[t], q_s + j * D, wK, wV, nk, a.scale, lane);
      }
      __syncthreads();
    }
  }

  // ---- normalise and store (zeros for inactive rows)
#pragma unroll
  for (int t = 0; t < 2; ++t) {
    const int j = warp + t * kDecWarps;
    if (j < g) {
      const float inv = act && st[t].l > 0.f ? 1.0f / st[t].l : 0.f;
      __nv_bfloat16* dst = a.out + (int64_t)r * a.out_stride + (int64_t)(h * g + j) * D;
#pragma unroll
      for (int i = 0; i < DPL; ++i) dst[i * 32 + lane] = f_to_bf16(st[t].acc[i] * inv);
    }
  }
  if (clustered) cluster_sync();  // peers may still be copying from this CTA's stage buffers
}

// ---- decode with the key history staged before the dependency wait -----------
// Used when the caller guarantees that everything but this step's projection row
// was written by launches at least two kernels back on the stream: the row table,
// the prefix length, each row's position, key count, output slot and active flag,
// the page-table entries before its current position and the K/V they point to
// (the CandidateGroup runtime: the prefix from the prefill, older suffix keys from
// earlier steps, the row metadata from this step's group step, which precedes the
// embedding and the qkv projection). CTA (h, r) then copies exactly the keys row r
// uses (the prefix up to a per-launch capacity: the caller's bound on the
// prefix length, at most hist_prefix_cap<D>() keys, the whole 512-position
// context at head_dim 64; and its older suffix up to kHistSuffix - 1 keys,
// contiguous; the shared-memory allocation follows the capacity),
// the RoPE rows of its position and the norm weights into shared memory BEFORE
// griddepcontrol.wait, i.e. while the qkv projection still runs, with cp.async
// (every copy in flight at once). After the wait it loads the projection row,
// applies q/k RMSNorm + bf16 RoPE, stores the new K/V (also as the staged row
// after the history) and folds all keys from shared memory in one pass per 64
// keys. Longer histories stream the rest from the cache after the wait.
//
// Prefix-once mode (cluster_rows > 1): the CTAs of one KV head's rows form a
// cluster; CTA c of the cluster reads only slice c of the prefix from the cache
// and pushes it into every peer's shared memory with cp.async.bulk
// (shared::cta -> shared::cluster, completing on the peer's mbarrier), so each
// shared-prefix KV row leaves HBM / L2 once per cluster of rows. All of it still
// happens before the dependency wait; the folds after it are the same.
constexpr int kHistSuffix = 32;
constexpr int kHistThreads = 256;  // 8 warps: one per query head of a KV group (g <= 8)
constexpr int kHistWarps = kHistThreads / 32;
constexpr int kHistDefaultPrefix = 128;  // staged prefix keys when the caller gives no bound
template <int D>
__host__ __device__ constexpr int hist_prefix_cap() {
  return D == 64 ? 512 : D == 96 ? 384 : 256;
}

// Staged K rows are dense (D bf16, 16-byte aligned, so cp.async and bulk copies
// can fill them) with their 16-byte chunks rotated: chunk c of key row j lives at
// chunk (c + rot(j)) mod (D / 8). A 16-byte shared-memory load is served in
// phases of 8 lanes; the fold's lanes read 8 consecutive rows at the same logical
// chunk, and these rotations put them in 8 distinct bank groups (checked
// exhaustively for D = 64, 96, 128: row strides of 128, 192 and 256 bytes).
template <int D>
__device__ __forceinline__ int k_chunk(int j, int c) {
  const int p = c + (D == 96 ? (j & 7) >> 1 : (j & 7));
  return p >= D / 8 ? p - D / 8 : p;
}

// q (fp32, shared, broadcast) . staged K row j, in the word order of dot_q_k.
template <int D>
__device__ __forceinline__ float dot_q_krow(const float* q, const __nv_bfloat16* K, int j) {
  float s = 0.f;
#pragma unroll
  for (int c = 0; c < D / 8; ++c) {
    const uint4 v = *reinterpret_cast<const uint4*>(K + (int64_t)j * D + k_chunk<D>(j, c) * 8);
    const uint32_t w4[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int t = 0; t < 4; ++t) {
      const float2 kv = bf16x2_to_f2(w4[t]);
      const int w = c * 4 + t;
      s += q[2 * w] * kv.x + q[2 * w + 1] * kv.y;
    }
  }
  return s;
}

// Folds staged rows [j0, j0 + nk) (nk <= 64) into `st`.
template <int D>
__device__ __forceinline__ void fold_staged(QState<D>& st, const float* qv, const __nv_bfloat16* K,
                                            const __nv_bfloat16* V, int j0, int nk, float scale, int lane) {
  const float s0 = lane < nk ? dot_q_krow<D>(qv, K, j0 + lane) * scale : -INFINITY;
  const float s1 = lane + 32 < nk ? dot_q_krow<D>(qv, K, j0 + lane + 32) * scale : -INFINITY;
  fold_scores<D>(st, s0, s1, nk, [&](int j, int i) { return bf16_to_f(V[(int64_t)(j0 + j) * D + i * 32 + lane]); });
}

template <int D>
size_t hist_decode_smem(int group, int cap) {
  const int rows = cap + kHistSuffix;
  return (size_t)group * D * 4 + (size_t)kHistWarps * D * 4 + (size_t)rows * D * 2 * 2 +
         (size_t)kKeyChunk * ((D + 2) * 2 + D * 2) + (size_t)4 * D * 2 +
         (size_t)kHistWarps * group * (D + 2) * 4;  // chunk-split partial states
}

template <int D>
__global__ void __launch_bounds__(kHistThreads) attn_decode_hist_kernel(const DecodeArgs a, int cluster_rows) {
  constexpr int DPL = D / 32;
  constexpr int KR = D + 2;  // padded K row of the streamed overflow chunks
  const int kCap = a.stage_cap;  // <= hist_prefix_cap<D>() (host)
  extern __shared__ __align__(16) uint8_t smem_raw[];
  __shared__ int32_t slot_s[hist_prefix_cap<D>() + kHistSuffix];
  __shared__ __align__(8) uint64_t pbar;  // prefix-once: the peers' slices have landed
  const int h = blockIdx.x, r = blockIdx.y;
  const int g = a.hq / a.hkv;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const bool clustered = cluster_rows > 1;
  float* q_s = reinterpret_cast<float*>(smem_raw);  // [g][D]
  float* tmp = q_s + g * D;                          // [warps][D]
  // staged keys, contiguous: [prefix | older suffix | the new key]
  __nv_bfloat16* Kh = reinterpret_cast<__nv_bfloat16*>(tmp + kHistWarps * D);  // [kCap + kHistSuffix][D], rotated
  __nv_bfloat16* Vh = Kh + (kCap + kHistSuffix) * D;                           // [kCap + kHistSuffix][D]
  __nv_bfloat16* Kw = Vh + (kCap + kHistSuffix) * D;                           // [kKeyChunk][KR]: streamed overflow
  __nv_bfloat16* Vw = Kw + kKeyChunk * KR;                                     // [kKeyChunk][D]
  __nv_bfloat16* cos_r = Vw + kKeyChunk * D;                                   // [D]: RoPE rows of this position
  __nv_bfloat16* sin_r = cos_r + D;
  __nv_bfloat16* nq = sin_r + D;  // [D]
  __nv_bfloat16* nk = nq + D;     // [D]
  float* part = reinterpret_cast<float*>(nk + D);  // [warps][g][D + 2]: chunk-split partial states
  const int64_t tok_stride = (int64_t)a.hkv * D;

  // ---- before the wait. Everything read here was written by launches at least
  // two kernels back on this stream (the prefill, earlier steps, and this step's
  // group step for the row's position, key count, slot and active flag). The
  // previous kernel launched this one only after its own griddepcontrol.wait, so
  // those launches have completed and their writes are visible. Grid rows past
  // `rows` (prefix-once padding to whole clusters) only stage their slice.
  const bool real = r < a.rows;
  const int P_in = a.prefix_len != nullptr ? *a.prefix_len : 0;
  const int P = (int64_t)P_in > a.table_stride ? (int)a.table_stride : (P_in < 0 ? 0 : P_in);
  const int64_t prow = a.row_table[0], rrow = real ? a.row_table[r] : prow;
  const bool act = real && (a.active == nullptr || a.active[r] != 0);
  const int pos_in = real ? a.positions[r] : 0;
  const int L_in = real ? a.seq_lens[r] : 0;
  const int64_t oslot = real ? a.out_loc[r] : -1;
  const int L_lo = L_in > P + 1 ? L_in : P + 1;
  const int L = (int64_t)L_lo > a.table_stride ? (int)a.table_stride : L_lo;
  const int ns_old = L - 1 - P;                // older suffix keys of this row (>= 0)
  const int np = min(P, kCap);                 // staged prefix keys
  const int ns = min(ns_old, kHistSuffix - 1);  // staged older suffix keys
  const int nst = act ? np + ns : 0;           // the new key goes to row np + ns
  const bool pos_ok = pos_in >= 0 && pos_in < a.max_pos;
  const int pos = pos_ok ? pos_in : 0;
  // the prefix rows this CTA reads from the cache: all of them, or its slice
  const uint32_t rank = clustered ? cluster_ctarank() : 0;
  const int lo = clustered ? (int)(rank * np / cluster_rows) : 0;
  const int hi = clustered ? (int)((rank + 1) * np / cluster_rows) : (act ? np : 0);
  if (clustered && threadIdx.x == 0) {
    mbar_init(&pbar, 1);
    fence_mbar_init();
  }
  for (int i = lo + threadIdx.x; i < hi; i += kHistThreads) slot_s[i] = a.page_table[prow * a.table_stride + i];
  for (int i = threadIdx.x; i < (act ? ns : 0); i += kHistThreads)
    slot_s[np + i] = a.page_table[rrow * a.table_stride + P + i];
  for (int i = threadIdx.x; i < D; i += kHistThreads) {
    nq[i] = a.q_norm_w[i];
    nk[i] = a.k_norm_w[i];
    cos_r[i] = a.cos_tab[(int64_t)pos * D + i];
    sin_r[i] = a.sin_tab[(int64_t)pos * D + i];
  }
  __syncthreads();
  // every incoming byte of the peers' prefix slices, announced before any peer
  // can push (the cluster barrier below)
  if (clustered && threadIdx.x == 0) mbar_arrive_expect_tx(&pbar, (uint32_t)(np - (hi - lo)) * D * 2 * 2);
  // the staged keys must be real slots (checked here, off the critical path;
  // reported after the wait)
  bool bad_slot = false;
  if (warp == 0) {
    bool b = false;
    for (int j = lo + lane; j < hi; j += 32) b |= slot_s[j] < 0 || slot_s[j] >= a.num_slots;
    for (int j = lane; j < (act ? ns : 0); j += 32) b |= slot_s[np + j] < 0 || slot_s[np + j] >= a.num_slots;
    bad_slot = __any_sync(0xffffffffu, b);
  }
  auto stage_rows = [&](int j0, int j1) {
    for (int i = threadIdx.x; i < (j1 - j0) * (D / 8); i += kHistThreads) {
      const int j = j0 + i / (D / 8), c = i % (D / 8);
      int64_t slot = slot_s[j];
      if (slot < 0 || slot >= a.num_slots) slot = 0;  // reported after the wait
      const int64_t off = slot * tok_stride + (int64_t)h * D + c * 8;
      cp_async16(Kh + (int64_t)j * D + k_chunk<D>(j, c) * 8, a.k_cache + off);
      cp_async16(Vh + (int64_t)j * D + c * 8, a.v_cache + off);
    }
  };
  stage_rows(lo, hi);
  if (act) stage_rows(np, np + ns);
  cp_async_wait_all();
  if (clustered) {
    // hand the own slice to the peers: the bulk copies read it through the async proxy
    fence_proxy_async_shared();
    __syncthreads();
    cluster_sync();  // every slice staged, every peer barrier armed
    if (threadIdx.x == 0 && hi > lo) {
      const uint32_t bytes = (uint32_t)(hi - lo) * D * 2;
      const uint32_t k_src = smem_u32(Kh + (int64_t)lo * D), v_src = smem_u32(Vh + (int64_t)lo * D);
      for (int p = 0; p < cluster_rows; ++p) {
        if (p == (int)rank) continue;
        const uint32_t bar = map_shared_rank(smem_u32(&pbar), (uint32_t)p);
        bulk_push_cluster(map_shared_rank(k_src, (uint32_t)p), k_src, bytes, bar);
        bulk_push_cluster(map_shared_rank(v_src, (uint32_t)p), v_src, bytes, bar);
      }
    }
    if (!mbar_wait(&pbar, 0) && threadIdx.x == 0) report(a.status, AIOSB_DEV_WAIT_TIMEOUT);
    cluster_sync();  // every push has landed: no CTA leaves while its slice is being read
  }
  // (no barrier needed here otherwise: after the wait only row np + ns, which
  // staging never writes, is stored before the barrier that precedes the folds)

  pdl_wait();
  // the next kernel (the o projection) launches once this one has its inputs,
  // which bounds how far ahead the chain prefetches (measured: 5.70 -> 5.54 ms)
  pdl_launch_dependents();
  if (threadIdx.x == 0 && bad_slot) report(a.status, AIOSB_DEV_SLOT_RANGE);
  // ---- after the wait: this step's projection row
  if (act) {
    if (threadIdx.x == 0 && (!pos_ok || L_in < P + 1 || L_in > a.table_stride))
      report(a.status, AIOSB_DEV_POSITION_RANGE);
    for (int it = warp; it < g + 1; it += kHistWarps) {
      float* tw = tmp + warp * D;
      float x[DPL];
      if (it < g) {
        const __nv_bfloat16* src = a.qkv + (int64_t)r * a.qkv_stride + (int64_t)(h * g + it) * D;
#pragma unroll
        for (int i = 0; i < DPL; ++i) x[i] = bf16_to_f(src[i * 32 + lane]);
        norm_rope<D>(x, nq, a.eps, cos_r, sin_r, true, true, lane, tw);
#pragma unroll
        for (int i = 0; i < DPL; ++i) q_s[it * D + i * 32 + lane] = x[i];
      } else {
        const __nv_bfloat16* ksrc = a.qkv + (int64_t)r * a.qkv_stride + (int64_t)(a.hq + h) * D;
        const __nv_bfloat16* vsrc = a.qkv + (int64_t)r * a.qkv_stride + (int64_t)(a.hq + a.hkv + h) * D;
        __nv_bfloat16 vraw[DPL];
#pragma unroll
        for (int i = 0; i < DPL; ++i) {
          x[i] = bf16_to_f(ksrc[i * 32 + lane]);
          vraw[i] = vsrc[i * 32 + lane];
        }
        norm_rope<D>(x, nk, a.eps, cos_r, sin_r, true, true, lane, tw);
        const bool slot_ok = oslot >= 0 && oslot < a.num_slots;
        if (!slot_ok && lane == 0) report(a.status, AIOSB_DEV_SLOT_RANGE);
#pragma unroll
        for (int i = 0; i < DPL; ++i) {
          const int e = i * 32 + lane;
          const __nv_bfloat16 kb = f_to_bf16(x[i]);
          Kh[(int64_t)nst * D + k_chunk<D>(nst, e / 8) * 8 + (e & 7)] = kb;
          Vh[(int64_t)nst * D + e] = vraw[i];
          if (slot_ok) {
            a.k_cache[oslot * tok_stride + (int64_t)h * D + e] = kb;
            a.v_cache[oslot * tok_stride + (int64_t)h * D + e] = vraw[i];
          }
        }
      }
    }
  }
  __syncthreads();

  // warp w owns query head w of the group (g <= kHistWarps) for the folds that
  // follow the staged ones and for the output
  QState<D> st;
  qstate_init<D>(st);
  const int32_t* pslots = a.page_table + prow * a.table_stride;
  const int32_t* rslots = a.page_table + rrow * a.table_stride;
  if (act) {
    auto fold_rows = [&](int j0, int n) {
      if (warp < g) fold_staged<D>(st, q_s + warp * D, Kh, Vh, j0, n, a.scale, lane);
    };
    auto fold_stream = [&](int n) {
      if (warp < g) fold_chunk<D>(st, q_s + warp * D, Kw, Vw, n, a.scale, lane);
    };
    // staged keys [prefix | older suffix] and, without a suffix overflow, the new
    // key right after them, 64 keys per chunk
    const int nfold = nst + (ns_old == ns ? 1 : 0);
    const int nchunks = (nfold + kKeyChunk - 1) / kKeyChunk;
    if (nchunks <= 1) {
      if (nfold > 0) fold_rows(0, nfold);
    } else {
      // several chunks: warp w folds chunks w, w + 8, ... for every head, then
      // head j's partial states are merged by warp j in warp order
      QState<D> sh[kMaxGroupQ];
#pragma unroll
      for (int j = 0; j < kMaxGroupQ; ++j) qstate_init<D>(sh[j]);
      for (int c = warp; c < nchunks; c += kHistWarps) {
        const int c0 = c * kKeyChunk, n = min(kKeyChunk, nfold - c0);
#pragma unroll
        for (int j = 0; j < kMaxGroupQ; ++j)
          if (j < g) fold_staged<D>(sh[j], q_s + j * D, Kh, Vh, c0, n, a.scale, lane);
      }
#pragma unroll
      for (int j = 0; j < kMaxGroupQ; ++j) {
        if (j < g) {
          float* ps = part + (warp * g + j) * (D + 2);
#pragma unroll
          for (int i = 0; i < DPL; ++i) ps[i * 32 + lane] = sh[j].acc[i];
          if (lane == 0) {
            ps[D] = sh[j].m;
            ps[D + 1] = sh[j].l;
          }
        }
      }
      __syncthreads();
      if (warp < g) {
        float m = -INFINITY;
        for (int w = 0; w < kHistWarps; ++w) m = fmaxf(m, part[(w * g + warp) * (D + 2) + D]);
        st.m = m;
        st.l = 0.f;
        for (int w = 0; w < kHistWarps; ++w) {
          const float* ps = part + (w * g + warp) * (D + 2);
          const float mw = ps[D];
          if (mw == -INFINITY) continue;  // a warp without a chunk
          const float e = expf(mw - m);
          st.l += ps[D + 1] * e;
#pragma unroll
          for (int i = 0; i < DPL; ++i) st.acc[i] += ps[i * 32 + lane] * e;
        }
      }
    }
    // longer histories: the prefix beyond the staged part, then the older suffix
    // beyond it, streamed from the cache, and the new key last
    for (int k0 = np; k0 < P; k0 += kKeyChunk) {
      const int n = min(kKeyChunk, P - k0);
      stage_chunk<D>(a.k_cache, a.v_cache, tok_stride, h, pslots, k0, n, a.num_slots, Kw, Vw, a.status);
      __syncthreads();
      fold_stream(n);
      __syncthreads();
    }
    if (ns_old > ns) {
      for (int k0 = P + ns; k0 < L - 1; k0 += kKeyChunk) {
        const int n = min(kKeyChunk, L - 1 - k0);
        stage_chunk<D>(a.k_cache, a.v_cache, tok_stride, h, rslots, k0, n, a.num_slots, Kw, Vw, a.status);
        __syncthreads();
        fold_stream(n);
        __syncthreads();
      }
      fold_rows(nst, 1);
    }
  }

  // ---- normalise and store (zeros for inactive rows)
  if (!real) return;
  if (warp < g) {
    const float inv = act && st.l > 0.f ? 1.0f / st.l : 0.f;
    __nv_bfloat16* dst = a.out + (int64_t)r * a.out_stride + (int64_t)(h * g + warp) * D;
#pragma unroll
    for (int i = 0; i < DPL; ++i) dst[i * 32 + lane] = f_to_bf16(st.acc[i] * inv);
  }
}

}  // namespace
}  // namespace aiosb

namespace aiosb {
namespace {

// ---- prefill prologue: q/k RMSNorm + RoPE, K/V store ----------------------
// One warp per (token, head) item; q heads write the rotated q buffer, KV heads
// write the paged cache at out_loc[t].
struct PrologueArgs {
  const __nv_bfloat16* qkv;
  int64_t qkv_stride;
  int64_t tokens;
  int hq, hkv;
  const __nv_bfloat16* q_norm_w;
  const __nv_bfloat16* k_norm_w;
  float eps;
  const __nv_bfloat16* cos_tab;
  const __nv_bfloat16* sin_tab;
  int max_pos;
  const int32_t* positions;
  const int32_t* out_loc;
  __nv_bfloat16* k_cache;
  __nv_bfloat16* v_cache;
  int64_t num_slots;
  __nv_bfloat16* q_out;
  int64_t q_out_stride;
  int32_t* status;
};

template <int D>
__global__ void __launch_bounds__(kAttnThreads) qk_norm_rope_store_kernel(const PrologueArgs a) {
  constexpr int DPL = D / 32;
  __shared__ float tmp_all[kAttnWarps][D];
  pdl_enter();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int heads = a.hq + a.hkv;
  const int64_t item = (int64_t)blockIdx.x * kAttnWarps + warp;
  if (item >= a.tokens * heads) return;
  const int64_t t = item / heads;
  const int hh = (int)(item % heads);
  int pos = a.positions[t];
  if (pos < 0 || pos >= a.max_pos) {
    if (lane == 0) report(a.status, AIOSB_DEV_POSITION_RANGE);
    pos = 0;
  }
  const __nv_bfloat16* row = a.qkv + t * a.qkv_stride;
  float x[DPL];
#pragma unroll
  for (int i = 0; i < DPL; ++i) x[i] = bf16_to_f(row[(int64_t)hh * D + i * 32 + lane]);
  const bool is_q = hh < a.hq;
  norm_rope<D>(x, is_q ? a.q_norm_w : a.k_norm_w, a.eps, a.cos_tab + (int64_t)pos * D, a.sin_tab + (int64_t)pos * D,
               true, true, lane, tmp_all[warp]);
  if (is_q) {
    __nv_bfloat16* dst = a.q_out + t * a.q_out_stride + (int64_t)hh * D;
#pragma unroll
    for (int i = 0; i < DPL; ++i) dst[i * 32 + lane] = f_to_bf16(x[i]);
    return;
  }
  const int kh = hh - a.hq;
  const int64_t slot = a.out_loc[t];
  if (slot < 0 || slot >= a.num_slots) {
    if (lane == 0) report(a.status, AIOSB_DEV_SLOT_RANGE);
    return;
  }
  const int64_t tok_stride = (int64_t)a.hkv * D;
  __nv_bfloat16* kd = a.k_cache + slot * tok_stride + (int64_t)kh * D;
  __nv_bfloat16* vd = a.v_cache + slot * tok_stride + (int64_t)kh * D;
  const __nv_bfloat16* vs = row + (int64_t)(a.hq + a.hkv + kh) * D;
#pragma unroll
  for (int i = 0; i < DPL; ++i) {
    kd[i * 32 + lane] = f_to_bf16(x[i]);
    vd[i * 32 + lane] = vs[i * 32 + lane];
  }
}

// ---- prefill attention: causal, cached-prefix offset, varlen requests ------
// CTA = (KV head, query tile of `tile_tokens` tokens of one request). Keys
// [0, cached_len + last query + 1) of the request's slot list are staged once
// per chunk and scored against all tile tokens x GQA heads with the causal mask
// key_pos <= cached_len + token index (aios/attention/flashinfer.py:33-91).
// ---- tensor-core prefill fold ------------------------------------------------
// Query rows of a prefill tile against a 64-key chunk on mma.sync m16n8k16 (bf16
// in, fp32 accumulate), FlashAttention-2 style: one warp owns 16 query rows,
// S = Q K^T for the chunk (8 key tiles of 8), masked (causal, chunk end) and
// scaled, an online softmax per row (the 4 lanes of a row reduce with shuffles),
// then O += P V with P as the A operand straight from the S accumulators. P is
// split into bf16 hi + lo halves (two MMAs) so that the PV product keeps about
// fp32 accuracy, where a single bf16 P would round every probability. Q, K and V
// are bf16 values already (q after its bf16 RoPE), so QK^T is exact up to fp32
// accumulation.
// Chunk rows in shared memory have a stride of D + 8 elements: the B-fragment
// word loads of K and the ldmatrix row reads of V are then bank-conflict free.
template <int D>
struct TcStride {
  static constexpr int kRow = D + 8;
};

__device__ __forceinline__ void mma_16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// Two 8x8 bf16 matrices, transposed: rows from lanes 0-7 (matrix 0) and 8-15
// (matrix 1), 16 bytes each.
__device__ __forceinline__ void ldsm_x2_trans(uint32_t& b0, uint32_t& b1, uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x2.trans.shared.b16 {%0,%1}, [%2];" : "=r"(b0), "=r"(b1) : "r"(addr));
}

// 16 query rows of one warp: Q A-fragments, O accumulators, and the running max
// and sum of rows lane / 4 and lane / 4 + 8.
template <int D>
struct TcRows {
  uint32_t qa[D / 16][4];
  float o[D / 8][4];
  float m[2], l[2];
  int qpos[2];  // absolute position of each row's query (-1: no query)
};

// q_s: [Q][D] fp32 query rows (bf16 values); rows row0 .. row0 + 15 of them.
template <int D, class PosFn>
__device__ __forceinline__ void tc_rows_init(TcRows<D>& t, const float* q_s, int row0, int Q, int lane,
                                             PosFn qpos_of) {
  const int g4 = lane >> 2, t4 = lane & 3;
  const int r[2] = {row0 + g4, row0 + g4 + 8};
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    t.m[h] = -INFINITY;
    t.l[h] = 0.f;
    t.qpos[h] = r[h] < Q ? qpos_of(r[h]) : -1;
  }
#pragma unroll
  for (int kk = 0; kk < D / 16; ++kk) {
    const int c0 = 16 * kk + 2 * t4, c1 = c0 + 8;
    t.qa[kk][0] = r[0] < Q ? pack_bf16x2(q_s[r[0] * D + c0], q_s[r[0] * D + c0 + 1]) : 0u;
    t.qa[kk][1] = r[1] < Q ? pack_bf16x2(q_s[r[1] * D + c0], q_s[r[1] * D + c0 + 1]) : 0u;
    t.qa[kk][2] = r[0] < Q ? pack_bf16x2(q_s[r[0] * D + c1], q_s[r[0] * D + c1 + 1]) : 0u;
    t.qa[kk][3] = r[1] < Q ? pack_bf16x2(q_s[r[1] * D + c1], q_s[r[1] * D + c1 + 1]) : 0u;
  }
#pragma unroll
  for (int jn = 0; jn < D / 8; ++jn) t.o[jn][0] = t.o[jn][1] = t.o[jn][2] = t.o[jn][3] = 0.f;
}

// Folds keys k0 .. k0 + nk - 1 (chunk rows 0 .. nk - 1 of Ks / Vs; the V rows
// nk .. 63 must hold finite values) into the warp's 16 rows.
template <int D>
__device__ __forceinline__ void tc_fold_chunk(TcRows<D>& t, const __nv_bfloat16* Ks, const __nv_bfloat16* Vs, int k0,
                                              int nk, float scale, int lane) {
  constexpr int R = TcStride<D>::kRow;
  const int g4 = lane >> 2, t4 = lane & 3;
  float s[8][4];
  const uint32_t* K32 = reinterpret_cast<const uint32_t*>(Ks);
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    s[j][0] = s[j][1] = s[j][2] = s[j][3] = 0.f;
    if (8 * j < nk) {
      const uint32_t* krow = K32 + (8 * j + g4) * (R / 2);
#pragma unroll
      for (int kk = 0; kk < D / 16; ++kk) mma_16816(s[j], t.qa[kk], krow[8 * kk + t4], krow[8 * kk + 4 + t4]);
    }
  }
  float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
  for (int j = 0; j < 8; ++j) {
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int key = 8 * j + 2 * t4 + (e & 1), h = e >> 1;
      const bool ok = key < nk && k0 + key <= t.qpos[h];
      s[j][e] = ok ? s[j][e] * scale : -INFINITY;
      mx[h] = fmaxf(mx[h], s[j][e]);
    }
  }
  float ref[2], corr[2], sum[2] = {0.f, 0.f};
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    mx[h] = fmaxf(mx[h], __shfl_xor_sync(0xffffffffu, mx[h], 1));
    mx[h] = fmaxf(mx[h], __shfl_xor_sync(0xffffffffu, mx[h], 2));
    const float m_new = fmaxf(t.m[h], mx[h]);
    ref[h] = m_new == -INFINITY ? 0.f : m_new;  // a row with no key yet keeps p = 0
    corr[h] = expf(t.m[h] - ref[h]);
    t.m[h] = m_new;
  }
#pragma unroll
  for (int j = 0; j < 8; ++j) {
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      s[j][e] = expf(s[j][e] - ref[e >> 1]);
      sum[e >> 1] += s[j][e];
    }
  }
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    sum[h] += __shfl_xor_sync(0xffffffffu, sum[h], 1);
    sum[h] += __shfl_xor_sync(0xffffffffu, sum[h], 2);
    t.l[h] = t.l[h] * corr[h] + sum[h];
  }
#pragma unroll
  for (int jn = 0; jn < D / 8; ++jn) {
    t.o[jn][0] *= corr[0];
    t.o[jn][1] *= corr[0];
    t.o[jn][2] *= corr[1];
    t.o[jn][3] *= corr[1];
  }
  const uint32_t vbase = smem_u32(Vs) + (uint32_t)((lane & 15) * R * 2);
#pragma unroll
  for (int kk = 0; kk < 4; ++kk) {
    if (16 * kk < nk) {
      uint32_t hi[4], lo[4];
      const float pv[4][2] = {{s[2 * kk][0], s[2 * kk][1]}, {s[2 * kk][2], s[2 * kk][3]},
                              {s[2 * kk + 1][0], s[2 * kk + 1][1]}, {s[2 * kk + 1][2], s[2 * kk + 1][3]}};
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        hi[q] = pack_bf16x2(pv[q][0], pv[q][1]);
        lo[q] = pack_bf16x2(pv[q][0] - bf16_lo(hi[q]), pv[q][1] - bf16_hi(hi[q]));
      }
#pragma unroll
      for (int jn = 0; jn < D / 8; ++jn) {
        uint32_t b0, b1;
        ldsm_x2_trans(b0, b1, vbase + (uint32_t)((16 * kk * R + 8 * jn) * 2));
        mma_16816(t.o[jn], hi, b0, b1);
        mma_16816(t.o[jn], lo, b0, b1);
      }
    }
  }
}

// Writes the warp's rows: out_of(row) gives the row's output vector (or nullptr).
template <int D, class OutFn>
__device__ __forceinline__ void tc_rows_store(const TcRows<D>& t, int row0, int Q, int lane, OutFn out_of) {
  const int g4 = lane >> 2, t4 = lane & 3;
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int r = row0 + g4 + 8 * h;
    if (r >= Q) continue;
    __nv_bfloat16* dst = out_of(r);
    const float inv = t.l[h] > 0.f ? 1.0f / t.l[h] : 0.f;
#pragma unroll
    for (int jn = 0; jn < D / 8; ++jn)
      *reinterpret_cast<uint32_t*>(dst + 8 * jn + 2 * t4) =
          pack_bf16x2(t.o[jn][2 * h] * inv, t.o[jn][2 * h + 1] * inv);
  }
}

// Stages chunk keys [k0, k0 + nc) from the paged cache and, after them, the new
// keys src_k / src_v rows [k0 + nc - cached, ...) up to nk rows (prefill-fused:
// keys of this request not yet in the cache), with the tensor-core row stride;
// V rows nk .. 63 are zeroed (their probabilities are 0; they must be finite).
template <int D>
__device__ __forceinline__ void tc_stage_chunk(const __nv_bfloat16* __restrict__ k_cache,
                                               const __nv_bfloat16* __restrict__ v_cache, int64_t tok_stride, int h,
                                               const int32_t* __restrict__ slots, int k0, int nc, int nk,
                                               const __nv_bfloat16* src_k, const __nv_bfloat16* src_v, int src0,
                                               int64_t num_slots, __nv_bfloat16* Ks, __nv_bfloat16* Vs,
                                               int32_t* status) {
  constexpr int R = TcStride<D>::kRow, kVec = D / 8;
  for (int idx = threadIdx.x; idx < kKeyChunk * kVec; idx += blockDim.x) {
    const int j = idx / kVec, c = idx % kVec;
    uint4 kv = make_uint4(0u, 0u, 0u, 0u), vv = kv;
    if (j < nc) {
      int64_t slot = slots[k0 + j];
      if (slot < 0 || slot >= num_slots) {
        if (c == 0) report(status, AIOSB_DEV_SLOT_RANGE);
        slot = 0;
      }
      kv = reinterpret_cast<const uint4*>(k_cache + slot * tok_stride + (int64_t)h * D)[c];
      vv = reinterpret_cast<const uint4*>(v_cache + slot * tok_stride + (int64_t)h * D)[c];
    } else if (j < nk) {
      kv = reinterpret_cast<const uint4*>(src_k + (int64_t)(src0 + j - nc) * D)[c];
      vv = reinterpret_cast<const uint4*>(src_v + (int64_t)(src0 + j - nc) * D)[c];
    }
    reinterpret_cast<uint4*>(Ks + j * R)[c] = kv;
    reinterpret_cast<uint4*>(Vs + j * R)[c] = vv;
  }
}

struct PrefillArgs {
  const __nv_bfloat16* q;
  int64_t q_stride;
  const __nv_bfloat16* k_cache;
  const __nv_bfloat16* v_cache;
  int64_t num_slots;
  const int32_t* page_table;
  int64_t table_stride;
  const int32_t* req_q_start;
  const int32_t* req_q_len;
  const int32_t* req_cached_len;
  const int32_t* req_table_row;
  const int32_t* tile_req;
  const int32_t* tile_q0;
  int tile_tokens;
  int hq, hkv;
  float scale;
  __nv_bfloat16* out;
  int64_t out_stride;
  int32_t* status;
};

template <int D>
__global__ void __launch_bounds__(kAttnThreads) attn_prefill_kernel(const PrefillArgs a) {
  extern __shared__ uint8_t smem_raw[];
  const int h = blockIdx.x;
  const int tile = blockIdx.y;
  const int g = a.hq / a.hkv;
  float* q_s = reinterpret_cast<float*>(smem_raw);
  const int Qmax = a.tile_tokens * g;
  __nv_bfloat16* Ks = reinterpret_cast<__nv_bfloat16*>(q_s + Qmax * D);  // [kKeyChunk][D + 8]
  __nv_bfloat16* Vs = Ks + kKeyChunk * TcStride<D>::kRow;                // [kKeyChunk][D + 8]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t tok_stride = (int64_t)a.hkv * D;

  pdl_enter();
  const int req = a.tile_req[tile];
  const int q0 = a.tile_q0[tile];
  const int qlen = a.req_q_len[req];
  const int nq = min(a.tile_tokens, qlen - q0);
  const int cached = a.req_cached_len[req];
  const int64_t qbase = a.req_q_start[req];
  const int32_t* slots = a.page_table + (int64_t)a.req_table_row[req] * a.table_stride;
  const int Q = nq * g;
  for (int idx = threadIdx.x; idx < Q * D; idx += blockDim.x) {
    const int qi = idx / D, e = idx % D;
    const int t = qi / g, j = qi % g;
    q_s[idx] = bf16_to_f(a.q[(qbase + q0 + t) * a.q_stride + (int64_t)(h * g + j) * D + e]);
  }
  __syncthreads();
  // query row qi = token (q0 + qi / g), head h * g + qi % g; warp w owns rows 16w..
  const int row0 = warp * 16;
  const bool folds = row0 < Q;
  TcRows<D> tr;
  tc_rows_init<D>(tr, q_s, row0, Q, lane, [&](int qi) { return cached + q0 + qi / g; });

  const int kv_end = cached + q0 + nq;
  for (int k0 = 0; k0 < kv_end; k0 += kKeyChunk) {
    const int nk = min(kKeyChunk, kv_end - k0);
    tc_stage_chunk<D>(a.k_cache, a.v_cache, tok_stride, h, slots, k0, nk, nk, nullptr, nullptr, 0, a.num_slots, Ks,
                      Vs, a.status);
    __syncthreads();
    if (folds) tc_fold_chunk<D>(tr, Ks, Vs, k0, nk, a.scale, lane);
    __syncthreads();
  }
  if (folds)
    tc_rows_store<D>(tr, row0, Q, lane, [&](int qi) {
      return a.out + (qbase + q0 + qi / g) * a.out_stride + (int64_t)(h * g + qi % g) * D;
    });
}

template <int D>
size_t decode_smem(int group) {
  const size_t chunk = (size_t)kKeyChunk * (D + 2) * 2 + (size_t)kKeyChunk * D * 2;
  return (size_t)group * D * 4 + (size_t)kDecWarps * D * 4 + (kStageChunks + 1) * chunk;
}

template <int D>
cudaError_t launch_decode(const DecodeArgs& a, int rows, int hkv, int group, cudaStream_t stream) {
  static bool configured[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  auto kern = attn_decode_kernel<D>;
  if (dev >= 0 && dev < 64 && !configured[dev]) {
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)decode_smem<D>(kMaxGroupQ));
    cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
    configured[dev] = true;
  }
  const int cluster_rows = rows <= 16 ? rows : 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)hkv, (unsigned)rows);
  cfg.blockDim = dim3(kDecThreads);
  cfg.dynamicSmemBytes = decode_smem<D>(group);
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  attr[1].id = cudaLaunchAttributeClusterDimension;
  attr[1].val.clusterDim.x = 1;
  attr[1].val.clusterDim.y = (unsigned)cluster_rows;
  attr[1].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  return cudaLaunchKernelEx(&cfg, kern, a, cluster_rows);
}
template <int D>
cudaError_t launch_decode_hist(const DecodeArgs& a, int rows, int hkv, int group, int cluster_rows,
                               cudaStream_t stream) {
  static bool configured[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  auto kern = attn_decode_hist_kernel<D>;
  if (dev >= 0 && dev < 64 && !configured[dev]) {
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         (int)hist_decode_smem<D>(kMaxGroupQ, hist_prefix_cap<D>()));
    configured[dev] = true;
  }
  // prefix-once: whole clusters of rows per KV head (padding rows only stage)
  const int grid_rows = (rows + cluster_rows - 1) / cluster_rows * cluster_rows;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)hkv, (unsigned)grid_rows);
  cfg.blockDim = dim3(kHistThreads);
  cfg.dynamicSmemBytes = hist_decode_smem<D>(group, a.stage_cap);
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  attr[1].id = cudaLaunchAttributeClusterDimension;
  attr[1].val.clusterDim.x = 1;
  attr[1].val.clusterDim.y = (unsigned)cluster_rows;
  attr[1].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = cluster_rows > 1 ? 2 : 1;
  return cudaLaunchKernelEx(&cfg, kern, a, cluster_rows);
}

template <int D>
size_t prefill_smem(int queries) {
  return (size_t)queries * D * 4 + (size_t)kKeyChunk * TcStride<D>::kRow * 2 * 2;
}

template <typename K>
void allow_smem(K kern, size_t bytes) {
  cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
}

}  // namespace
}  // namespace aiosb

using namespace aiosb;

extern "C" int aiosb_attention_decode(const void* qkv, int64_t qkv_stride, const void* q, int64_t q_stride,
                                      const void* q_norm_w, const void* k_norm_w, float eps, const void* cos_tab,
                                      const void* sin_tab, int64_t max_pos, const int32_t* positions,
                                      const int32_t* out_loc, void* k_cache, void* v_cache, int64_t num_slots,
                                      const int32_t* page_table, int64_t table_stride, const int32_t* row_table,
                                      const int32_t* seq_lens, const int32_t* prefix_len, const int32_t* active,
                                      int stable_history, int64_t staged_prefix, int64_t rows,
                                      int64_t num_qo_heads, int64_t num_kv_heads, int64_t head_dim, float scale,
                                      void* out, int64_t out_stride, int32_t* status, void* stream) {
  AIOSB_REQUIRE(rows >= 0 && num_kv_heads > 0 && num_qo_heads > 0 && num_qo_heads % num_kv_heads == 0,
                AIOSB_ERR_INVALID_ARG, "query head count must be divisible by KV head count");
  AIOSB_REQUIRE(head_dim == 64 || head_dim == 96 || head_dim == 128, AIOSB_ERR_UNSUPPORTED,
                "attention_decode: head_dim %lld unsupported (64, 96, 128)", (long long)head_dim);
  const int64_t g = num_qo_heads / num_kv_heads;
  AIOSB_REQUIRE(g <= kMaxGroupQ, AIOSB_ERR_UNSUPPORTED,
                "attention_decode: %lld query heads per KV head exceeds %d", (long long)g, kMaxGroupQ);
  if (rows == 0) return AIOSB_OK;
  AIOSB_REQUIRE((qkv != nullptr) != (q != nullptr), AIOSB_ERR_INVALID_ARG,
                "attention_decode: pass exactly one of qkv (fused prologue) or q (pre-rotated)");
  AIOSB_REQUIRE(k_cache && v_cache && page_table && row_table && seq_lens && out && positions,
                AIOSB_ERR_INVALID_ARG, "attention_decode: null pointer");
  AIOSB_REQUIRE(qkv == nullptr || (q_norm_w && k_norm_w && cos_tab && sin_tab && out_loc), AIOSB_ERR_INVALID_ARG,
                "attention_decode: fused prologue needs norm weights, rope tables and out_loc");
  DecodeArgs a;
  a.qkv = (const __nv_bfloat16*)qkv;
  a.qkv_stride = qkv_stride;
  a.q = (const __nv_bfloat16*)q;
  a.q_stride = q_stride;
  a.q_norm_w = (const __nv_bfloat16*)q_norm_w;
  a.k_norm_w = (const __nv_bfloat16*)k_norm_w;
  a.eps = eps;
  a.cos_tab = (const __nv_bfloat16*)cos_tab;
  a.sin_tab = (const __nv_bfloat16*)sin_tab;
  a.max_pos = (int)max_pos;
  a.positions = positions;
  a.out_loc = out_loc;
  a.k_cache = (__nv_bfloat16*)k_cache;
  a.v_cache = (__nv_bfloat16*)v_cache;
  a.num_slots = num_slots;
  a.page_table = page_table;
  a.table_stride = table_stride;
  a.row_table = row_table;
  a.seq_lens = seq_lens;
  a.prefix_len = prefix_len;
  a.active = active;
  a.stage_cap = kHistDefaultPrefix;
  a.rows = (int)rows;
  a.hq = (int)num_qo_heads;
  a.hkv = (int)num_kv_heads;
  a.scale = scale;
  a.out = (__nv_bfloat16*)out;
  a.out_stride = out_stride;
  a.status = status;
  cudaError_t e;
  cudaStream_t s = as_stream(stream);
  if (stable_history && qkv != nullptr) {
    AIOSB_REQUIRE(stable_history == AIOSB_HISTORY_STAGED || stable_history == AIOSB_HISTORY_PREFIX_ONCE,
                  AIOSB_ERR_INVALID_ARG, "attention_decode: unknown stable_history mode %d", stable_history);
    AIOSB_REQUIRE(aligned16(k_cache) && aligned16(v_cache), AIOSB_ERR_MISALIGNED,
                  "attention_decode: the KV cache must be 16-byte aligned");
    const int cr = stable_history == AIOSB_HISTORY_PREFIX_ONCE ? (int)std::min<int64_t>(rows, 8) : 1;
    // staged prefix keys: the caller's bound rounded up to 64, at most what fits
    const int64_t cap_max = head_dim == 64 ? hist_prefix_cap<64>() : head_dim == 96 ? hist_prefix_cap<96>()
                                                                                      : hist_prefix_cap<128>();
    const int64_t want = staged_prefix > 0 ? (staged_prefix + 63) / 64 * 64 : kHistDefaultPrefix;
    a.stage_cap = (int)std::min(want, cap_max);
    if (head_dim == 64) e = launch_decode_hist<64>(a, (int)rows, (int)num_kv_heads, (int)g, cr, s);
    else if (head_dim == 96) e = launch_decode_hist<96>(a, (int)rows, (int)num_kv_heads, (int)g, cr, s);
    else e = launch_decode_hist<128>(a, (int)rows, (int)num_kv_heads, (int)g, cr, s);
  } else if (head_dim == 64) {
    e = launch_decode<64>(a, (int)rows, (int)num_kv_heads, (int)g, s);
  } else if (head_dim == 96) {
    e = launch_decode<96>(a, (int)rows, (int)num_kv_heads, (int)g, s);
  } else {
    e = launch_decode<128>(a, (int)rows, (int)num_kv_heads, (int)g, s);
  }
  if (e != cudaSuccess) return set_error(AIOSB_ERR_LAUNCH, "attention_decode: %s", cudaGetErrorString(e));
  return AIOSB_OK;
}

extern "C" int aiosb_qk_norm_rope_store(const void* qkv, int64_t qkv_stride, int64_t tokens, int64_t num_qo_heads,
                                        int64_t num_kv_heads, int64_t head_dim, const void* q_norm_w,
                                        const void* k_norm_w, float eps, const void* cos_tab, const void* sin_tab,
                                        int64_t max_pos, const int32_t* positions, const int32_t* out_loc,
                                        void* k_cache, void* v_cache, int64_t num_slots, void* q_out,
                                        int64_t q_out_stride, int32_t* status, void* stream) {
  AIOSB_REQUIRE(tokens >= 0 && num_qo_heads > 0 && num_kv_heads > 0, AIOSB_ERR_INVALID_ARG,
                "qk_norm_rope_store: bad sizes");
  AIOSB_REQUIRE(head_dim == 64 || head_dim == 96 || head_dim == 128, AIOSB_ERR_UNSUPPORTED,
                "qk_norm_rope_store: head_dim %lld unsupported (64, 96, 128)", (long long)head_dim);
  if (tokens == 0) return AIOSB_OK;
  AIOSB_REQUIRE(qkv && q_norm_w && k_norm_w && cos_tab && sin_tab && positions && out_loc && k_cache && v_cache &&
                    q_out,
                AIOSB_ERR_INVALID_ARG, "qk_norm_rope_store: null pointer");
  PrologueArgs a;
  a.qkv = (const __nv_bfloat16*)qkv;
  a.qkv_stride = qkv_stride;
  a.tokens = tokens;
  a.hq = (int)num_qo_heads;
  a.hkv = (int)num_kv_heads;
  a.q_norm_w = (const __nv_bfloat16*)q_norm_w;
  a.k_norm_w = (const __nv_bfloat16*)k_norm_w;
  a.eps = eps;
  a.cos_tab = (const __nv_bfloat16*)cos_tab;
  a.sin_tab = (const __nv_bfloat16*)sin_tab;
  a.max_pos = (int)max_pos;
  a.positions = positions;
  a.out_loc = out_loc;
  a.k_cache = (__nv_bfloat16*)k_cache;
  a.v_cache = (__nv_bfloat16*)v_cache;
  a.num_slots = num_slots;
  a.q_out = (__nv_bfloat16*)q_out;
  a.q_out_stride = q_out_stride;
  a.status = status;
  const int64_t items = tokens * (num_qo_heads + num_kv_heads);
  const dim3 grid((unsigned)((items + kAttnWarps - 1) / kAttnWarps)), block(kAttnThreads);
  cudaStream_t s = as_stream(stream);
  cudaError_t e;
  if (head_dim == 64) e = launch_pdl(qk_norm_rope_store_kernel<64>, grid, block, 0, s, a);
  else if (head_dim == 96) e = launch_pdl(qk_norm_rope_store_kernel<96>, grid, block, 0, s, a);
  else e = launch_pdl(qk_norm_rope_store_kernel<128>, grid, block, 0, s, a);
  if (e != cudaSuccess) return set_error(AIOSB_ERR_LAUNCH, "qk_norm_rope_store: %s", cudaGetErrorString(e));
  return AIOSB_OK;
}

extern "C" int aiosb_prefill_tile_tokens(int64_t num_qo_heads, int64_t num_kv_heads) {
  if (num_kv_heads <= 0 || num_qo_heads <= 0 || num_qo_heads % num_kv_heads) return 0;
  const int64_t g = num_qo_heads / num_kv_heads;
  // one query vector per warp: a keystroke prefill has few tokens, and small
  // tiles spread them over more CTAs (each re-stages the short key list)
  if (g <= kAttnWarps) return (int)(kAttnWarps / g);
  return g > kMaxQueries ? 0 : (int)(kMaxQueries / g);
}

extern "C" int aiosb_attention_prefill(const void* q, int64_t q_stride, const void* k_cache, const void* v_cache,
                                       int64_t num_slots, const int32_t* page_table, int64_t table_stride,
                                       const int32_t* req_q_start, const int32_t* req_q_len,
                                       const int32_t* req_cached_len, const int32_t* req_table_row,
                                       const int32_t* tile_req, const int32_t* tile_q0, int64_t num_tiles,
                                       int64_t tile_tokens, int64_t num_qo_heads, int64_t num_kv_heads,
                                       int64_t head_dim, float scale, void* out, int64_t out_stride, int32_t* status,
                                       void* stream) {
  AIOSB_REQUIRE(num_tiles >= 0 && num_kv_heads > 0 && num_qo_heads % num_kv_heads == 0, AIOSB_ERR_INVALID_ARG,
                "query head count must be divisible by KV head count");
  AIOSB_REQUIRE(head_dim == 64 || head_dim == 96 || head_dim == 128, AIOSB_ERR_UNSUPPORTED,
                "attention_prefill: head_dim %lld unsupported (64, 96, 128)", (long long)head_dim);
  const int64_t g = num_qo_heads / num_kv_heads;
  AIOSB_REQUIRE(tile_tokens >= 1 && tile_tokens * g <= kMaxQueries, AIOSB_ERR_INVALID_ARG,
                "attention_prefill: tile_tokens * group must be in [1, %d]", kMaxQueries);
  if (num_tiles == 0) return AIOSB_OK;
  AIOSB_REQUIRE(q && k_cache && v_cache && page_table && req_q_start && req_q_len && req_cached_len &&
                    req_table_row && tile_req && tile_q0 && out,
                AIOSB_ERR_INVALID_ARG, "attention_prefill: null pointer");
  PrefillArgs a;
  a.q = (const __nv_bfloat16*)q;
  a.q_stride = q_stride;
  a.k_cache = (const __nv_bfloat16*)k_cache;
  a.v_cache = (const __nv_bfloat16*)v_cache;
  a.num_slots = num_slots;
  a.page_table = page_table;
  a.table_stride = table_stride;
  a.req_q_start = req_q_start;
  a.req_q_len = req_q_len;
  a.req_cached_len = req_cached_len;
  a.req_table_row = req_table_row;
  a.tile_req = tile_req;
  a.tile_q0 = tile_q0;
  a.tile_tokens = (int)tile_tokens;
  a.hq = (int)num_qo_heads;
  a.hkv = (int)num_kv_heads;
  a.scale = scale;
  a.out = (__nv_bfloat16*)out;
  a.out_stride = out_stride;
  a.status = status;
  const int Q = (int)(tile_tokens * g);
  const dim3 grid((unsigned)num_kv_heads, (unsigned)num_tiles), block(kAttnThreads);
  cudaStream_t s = as_stream(stream);
  cudaError_t e;
  if (head_dim == 64) {
    allow_smem(attn_prefill_kernel<64>, prefill_smem<64>(kMaxQueries));
    e = launch_pdl(attn_prefill_kernel<64>, grid, block, prefill_smem<64>(Q), s, a);
  } else if (head_dim == 96) {
    allow_smem(attn_prefill_kernel<96>, prefill_smem<96>(kMaxQueries));
    e = launch_pdl(attn_prefill_kernel<96>, grid, block, prefill_smem<96>(Q), s, a);
  } else {
    allow_smem(attn_prefill_kernel<128>, prefill_smem<128>(kMaxQueries));
    e = launch_pdl(attn_prefill_kernel<128>, grid, block, prefill_smem<128>(Q), s, a);
  }
  if (e != cudaSuccess) return set_error(AIOSB_ERR_LAUNCH, "attention_prefill: %s", cudaGetErrorString(e));
  return AIOSB_OK;
}

namespace aiosb {
namespace {

// ---- fused prefill: q/k RMSNorm + RoPE + K/V store + causal attention -------
// For requests of at most kKeyChunk new tokens (a keystroke's prefix prefill).
// CTA (KV head h, tile) normalises and rotates its own queries and the new keys
// of its causal window (the request's first q0 + nq new tokens; tiles of one
// request repeat that small work), and stores the K/V of its own tile's tokens.
// Keys are folded in the same 64-key chunks as attn_prefill_kernel, each taken
// from the cache (cached prefix) or from the new-key rows in shared memory, so
// the output equals qk_norm_rope_store_kernel followed by attn_prefill_kernel
// bit for bit, one launch and one kernel boundary fewer per layer.
struct FusedPrefillArgs {
  const __nv_bfloat16* qkv;  // [tokens, qkv_stride]: q heads | k heads | v heads (raw projection)
  int64_t qkv_stride;
  const __nv_bfloat16* q_norm_w;
  const __nv_bfloat16* k_norm_w;
  float eps;
  const __nv_bfloat16* cos_tab;  // [max_pos, D]
  const __nv_bfloat16* sin_tab;
  int max_pos;
  const int32_t* positions;  // [tokens]
  const int32_t* out_loc;    // [tokens]
  __nv_bfloat16* k_cache;
  __nv_bfloat16* v_cache;
  int64_t num_slots;
  const int32_t* page_table;
  int64_t table_stride;
  const int32_t* req_q_start;
  const int32_t* req_q_len;
  const int32_t* req_cached_len;
  const int32_t* req_table_row;
  const int32_t* tile_req;
  const int32_t* tile_q0;
  int tile_tokens;
  int hq, hkv;
  float scale;
  __nv_bfloat16* out;
  int64_t out_stride;
  int32_t* status;
};

template <int D>
size_t fused_prefill_smem(int queries) {
  // q_s | Ks | Vs | NK | NV | warp scratch | raw rows (queries + new keys) | cos | sin | norm weights | positions
  return (size_t)queries * D * 4 + (size_t)kKeyChunk * TcStride<D>::kRow * 2 * 2 + (size_t)kKeyChunk * D * 2 * 2 +
         (size_t)kAttnWarps * D * 4 + (size_t)(queries + kKeyChunk) * D * 2 + (size_t)kKeyChunk * D * 2 * 2 +
         (size_t)D * 2 * 2 + (size_t)kKeyChunk * 4;
}

template <int D>
__global__ void __launch_bounds__(kAttnThreads) attn_prefill_fused_kernel(const FusedPrefillArgs a) {
  constexpr int DPL = D / 32;
  extern __shared__ __align__(16) uint8_t smem_raw[];
  const int h = blockIdx.x;
  const int tile = blockIdx.y;
  const int g = a.hq / a.hkv;
  const int Qmax = a.tile_tokens * g;
  float* q_s = reinterpret_cast<float*>(smem_raw);                                // [Qmax][D]
  __nv_bfloat16* Ks = reinterpret_cast<__nv_bfloat16*>(q_s + Qmax * D);            // [kKeyChunk][D + 8]
  __nv_bfloat16* Vs = Ks + kKeyChunk * TcStride<D>::kRow;                           // [kKeyChunk][D + 8]
  __nv_bfloat16* NK = Vs + kKeyChunk * TcStride<D>::kRow;                           // new keys, rotated
  __nv_bfloat16* NV = NK + kKeyChunk * D;                                           // new values
  float* tmp = reinterpret_cast<float*>(NV + kKeyChunk * D);                        // [warps][D]
  __nv_bfloat16* RAW = reinterpret_cast<__nv_bfloat16*>(tmp + kAttnWarps * D);      // [Qmax + kKeyChunk][D]
  __nv_bfloat16* CS = RAW + (Qmax + kKeyChunk) * D;                                  // [kKeyChunk][D]
  __nv_bfloat16* SN = CS + kKeyChunk * D;                                            // [kKeyChunk][D]
  __nv_bfloat16* NQW = SN + kKeyChunk * D;                                           // [D]
  __nv_bfloat16* NKW = NQW + D;                                                      // [D]
  int* pos_s = reinterpret_cast<int*>(NKW + D);                                      // [kKeyChunk]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t tok_stride = (int64_t)a.hkv * D;

  // ---- before the wait: the request and tile arrays, the positions, the page
  // table, the norm weights and the RoPE rows were written before this forward
  // began (one host-to-device copy and the page-table reset precede the prefill
  // graph), so they are staged while the qkv projection still runs
  pdl_launch_dependents();
  const int req = a.tile_req[tile];
  const int q0 = a.tile_q0[tile];
  const int qlen = a.req_q_len[req];
  const int nq = min(a.tile_tokens, qlen - q0);
  const int cached = a.req_cached_len[req];
  const int64_t qbase = a.req_q_start[req];
  const int32_t* slots = a.page_table + (int64_t)a.req_table_row[req] * a.table_stride;
  const int nnew = q0 + nq;  // new keys in this tile's causal window
  if (nnew > kKeyChunk) {    // the host admits only requests of <= kKeyChunk new tokens
    if (threadIdx.x == 0) report(a.status, AIOSB_DEV_POSITION_RANGE);
    return;
  }
  const int Q = nq * g;
  constexpr int kVec = D / 8;  // 16-byte vectors per head row
  for (int j = threadIdx.x; j < nnew; j += blockDim.x) {
    int pos = a.positions[qbase + j];
    if (pos < 0 || pos >= a.max_pos) {
      report(a.status, AIOSB_DEV_POSITION_RANGE);
      pos = 0;
    }
    pos_s[j] = pos;
  }
  for (int i = threadIdx.x; i < D; i += blockDim.x) {
    NQW[i] = a.q_norm_w[i];
    NKW[i] = a.k_norm_w[i];
  }
  __syncthreads();
  for (int idx = threadIdx.x; idx < nnew * kVec; idx += blockDim.x) {
    const int j = idx / kVec, c = idx % kVec;
    const int64_t pr = (int64_t)pos_s[j] * kVec + c;
    reinterpret_cast<uint4*>(CS + j * D)[c] = reinterpret_cast<const uint4*>(a.cos_tab)[pr];
    reinterpret_cast<uint4*>(SN + j * D)[c] = reinterpret_cast<const uint4*>(a.sin_tab)[pr];
  }
  pdl_wait();
  // ---- after the wait: this layer's projection rows. Item it < Q is query
  // (token q0 + it / g, head h * g + it % g); the others are new key rows
  // 0 .. nnew - 1 of KV head h, staged so that the per-item work reads shared
  // memory only.
  const uint4* qkv4 = reinterpret_cast<const uint4*>(a.qkv);
  const int64_t row4 = a.qkv_stride / 8;
  for (int idx = threadIdx.x; idx < (Q + 2 * nnew) * kVec; idx += blockDim.x) {
    const int it = idx / kVec, c = idx % kVec;
    int j, hh;
    uint4* dst;
    if (it < Q) {
      j = q0 + it / g, hh = h * g + it % g, dst = reinterpret_cast<uint4*>(RAW + it * D);
    } else if (it < Q + nnew) {
      j = it - Q, hh = a.hq + h, dst = reinterpret_cast<uint4*>(RAW + it * D);
    } else {
      j = it - Q - nnew, hh = a.hq + a.hkv + h, dst = reinterpret_cast<uint4*>(NV + j * D);
    }
    dst[c] = qkv4[(qbase + j) * row4 + (int64_t)hh * kVec + c];
  }
  __syncthreads();
  for (int it = warp; it < Q + nnew; it += kAttnWarps) {
    const bool is_q = it < Q;
    const int j = is_q ? q0 + it / g : it - Q;  // token index within the request
    const int64_t t = qbase + j;
    float x[DPL];
#pragma unroll
    for (int i = 0; i < DPL; ++i) x[i] = bf16_to_f(RAW[it * D + i * 32 + lane]);
    norm_rope<D>(x, is_q ? NQW : NKW, a.eps, CS + j * D, SN + j * D, true, true, lane, tmp + warp * D);
    if (is_q) {
#pragma unroll
      for (int i = 0; i < DPL; ++i) q_s[it * D + i * 32 + lane] = x[i];
      continue;
    }
    // this tile's own tokens go to the cache (each token belongs to one tile)
    const bool own = j >= q0;
    const int64_t slot = own ? a.out_loc[t] : -1;
    const bool slot_ok = slot >= 0 && slot < a.num_slots;
    if (own && !slot_ok && lane == 0) report(a.status, AIOSB_DEV_SLOT_RANGE);
#pragma unroll
    for (int i = 0; i < DPL; ++i) {
      const __nv_bfloat16 kb = f_to_bf16(x[i]);
      const __nv_bfloat16 vb = NV[j * D + i * 32 + lane];
      NK[j * D + i * 32 + lane] = kb;
      if (slot_ok) {
        a.k_cache[slot * tok_stride + (int64_t)h * D + i * 32 + lane] = kb;
        a.v_cache[slot * tok_stride + (int64_t)h * D + i * 32 + lane] = vb;
      }
    }
  }
  __syncthreads();
  // query row qi = token (q0 + qi / g), head h * g + qi % g; warp w owns rows 16w..
  const int row0 = warp * 16;
  const bool folds = row0 < Q;
  TcRows<D> tr;
  tc_rows_init<D>(tr, q_s, row0, Q, lane, [&](int qi) { return cached + q0 + qi / g; });

  const int kv_end = cached + nnew;
  for (int k0 = 0; k0 < kv_end; k0 += kKeyChunk) {
    const int nk = min(kKeyChunk, kv_end - k0);
    const int nc = max(0, min(nk, cached - k0));  // keys of this chunk in the cache; the rest are new
    tc_stage_chunk<D>(a.k_cache, a.v_cache, tok_stride, h, slots, k0, nc, nk, NK, NV, k0 + nc - cached, a.num_slots,
                      Ks, Vs, a.status);
    __syncthreads();
    if (folds) tc_fold_chunk<D>(tr, Ks, Vs, k0, nk, a.scale, lane);
    __syncthreads();
  }
  if (folds)
    tc_rows_store<D>(tr, row0, Q, lane, [&](int qi) {
      return a.out + (qbase + q0 + qi / g) * a.out_stride + (int64_t)(h * g + qi % g) * D;
    });
}

}  // namespace
}  // namespace aiosb

extern "C" int aiosb_attention_prefill_fused(
    const void* qkv, int64_t qkv_stride, const void* q_norm_w, const void* k_norm_w, float eps, const void* cos_tab,
    const void* sin_tab, int64_t max_pos, const int32_t* positions, const int32_t* out_loc, void* k_cache,
    void* v_cache, int64_t num_slots, const int32_t* page_table, int64_t table_stride, const int32_t* req_q_start,
    const int32_t* req_q_len, const int32_t* req_cached_len, const int32_t* req_table_row, const int32_t* tile_req,
    const int32_t* tile_q0, int64_t num_tiles, int64_t tile_tokens, int64_t max_q_len, int64_t num_qo_heads,
    int64_t num_kv_heads, int64_t head_dim, float scale, void* out, int64_t out_stride, int32_t* status,
    void* stream) {
  AIOSB_REQUIRE(num_tiles >= 0 && num_kv_heads > 0 && num_qo_heads % num_kv_heads == 0, AIOSB_ERR_INVALID_ARG,
                "query head count must be divisible by KV head count");
  AIOSB_REQUIRE(head_dim == 64 || head_dim == 96 || head_dim == 128, AIOSB_ERR_UNSUPPORTED,
                "attention_prefill_fused: head_dim %lld unsupported (64, 96, 128)", (long long)head_dim);
  AIOSB_REQUIRE(max_q_len >= 0 && max_q_len <= kKeyChunk, AIOSB_ERR_UNSUPPORTED,
                "attention_prefill_fused: requests of at most %d new tokens (got %lld)", kKeyChunk,
                (long long)max_q_len);
  const int64_t g = num_qo_heads / num_kv_heads;
  AIOSB_REQUIRE(tile_tokens >= 1 && tile_tokens * g <= kMaxQueries, AIOSB_ERR_INVALID_ARG,
                "attention_prefill_fused: tile_tokens * group must be in [1, %d]", kMaxQueries);
  if (num_tiles == 0) return AIOSB_OK;
  AIOSB_REQUIRE(qkv && q_norm_w && k_norm_w && cos_tab && sin_tab && positions && out_loc && k_cache && v_cache &&
                    page_table && req_q_start && req_q_len && req_cached_len && req_table_row && tile_req &&
                    tile_q0 && out,
                AIOSB_ERR_INVALID_ARG, "attention_prefill_fused: null pointer");
  // the prologue stages projection and RoPE rows with 16-byte loads
  AIOSB_REQUIRE(qkv_stride % 8 == 0 && ((uintptr_t)qkv & 15u) == 0 && ((uintptr_t)cos_tab & 15u) == 0 &&
                    ((uintptr_t)sin_tab & 15u) == 0,
                AIOSB_ERR_MISALIGNED, "attention_prefill_fused: qkv rows and RoPE tables must be 16-byte aligned");
  FusedPrefillArgs a;
  a.qkv = (const __nv_bfloat16*)qkv;
  a.qkv_stride = qkv_stride;
  a.q_norm_w = (const __nv_bfloat16*)q_norm_w;
  a.k_norm_w = (const __nv_bfloat16*)k_norm_w;
  a.eps = eps;
  a.cos_tab = (const __nv_bfloat16*)cos_tab;
  a.sin_tab = (const __nv_bfloat16*)sin_tab;
  a.max_pos = (int)max_pos;
  a.positions = positions;
  a.out_loc = out_loc;
  a.k_cache = (__nv_bfloat16*)k_cache;
  a.v_cache = (__nv_bfloat16*)v_cache;
  a.num_slots = num_slots;
  a.page_table = page_table;
  a.table_stride = table_stride;
  a.req_q_start = req_q_start;
  a.req_q_len = req_q_len;
  a.req_cached_len = req_cached_len;
  a.req_table_row = req_table_row;
  a.tile_req = tile_req;
  a.tile_q0 = tile_q0;
  a.tile_tokens = (int)tile_tokens;
  a.hq = (int)num_qo_heads;
  a.hkv = (int)num_kv_heads;
  a.scale = scale;
  a.out = (__nv_bfloat16*)out;
  a.out_stride = out_stride;
  a.status = status;
  const int Q = (int)(tile_tokens * g);
  const dim3 grid((unsigned)num_kv_heads, (unsigned)num_tiles), block(kAttnThreads);
  cudaStream_t s = as_stream(stream);
  cudaError_t e;
  if (head_dim == 64) {
    allow_smem(attn_prefill_fused_kernel<64>, fused_prefill_smem<64>(kMaxQueries));
    e = launch_pdl(attn_prefill_fused_kernel<64>, grid, block, fused_prefill_smem<64>(Q), s, a);
  } else if (head_dim == 96) {
    allow_smem(attn_prefill_fused_kernel<96>, fused_prefill_smem<96>(kMaxQueries));
    e = launch_pdl(attn_prefill_fused_kernel<96>, grid, block, fused_prefill_smem<96>(Q), s, a);
  } else {
    allow_smem(attn_prefill_fused_kernel<128>, fused_prefill_smem<128>(kMaxQueries));
    e = launch_pdl(attn_prefill_fused_kernel<128>, grid, block, fused_prefill_smem<128>(Q), s, a);
  }
  if (e != cudaSuccess) return set_error(AIOSB_ERR_LAUNCH, "attention_prefill_fused: %s", cudaGetErrorString(e));
  return AIOSB_OK;
}
