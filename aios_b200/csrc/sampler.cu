// Raw-logprob sampler (replaces aios/engine/sample.py:54-163) and the
// CandidateGroup step bookkeeping of aios/ime.py:970-1054, on the device.
//
// One CTA samples one logits row; the row lives in registers (16-byte loads)
// and its sampling keys in shared memory:
//   raw log-softmax of the bf16 logits (fp32, aios/engine/sample.py:74);
//   forbidden ids -> -inf on the sampling copy only (sample.py:76-111), kept as
//   a bitmap;
//   greedy: first index of the maximum (torch argmax);
//   otherwise: scaled = logits / T (fp32) as order-preserving uint32 keys;
//   top-k <= 512: a lower bound of the k-th largest key from the 512 thread
//   maxima, then only the keys above it are compacted and sorted; larger k (or a
//   degenerate row) by an exact 4-pass radix select; candidates sorted by
//   (value desc, token id asc), softmax, top-p keep-mask with the one-position
//   shift of sample.py:140-146, re-softmax, index = #(cumsum < u) clamped
//   (sample.py:161-165).
// Cumulative sums accumulate in fp64 and round each prefix to fp32, the way
// torch's CPU cumsum does for float tensors. Equal logits are ordered by
// ascending token id; torch.topk leaves that order unspecified.
#include <algorithm>
#include <mutex>

#include "abi_util.h"
#include "common.cuh"

namespace aiosb {
namespace {

constexpr int kSampThreads = 512;
constexpr int kMaxVocab = 32768;
constexpr int kMaxSortK = 2048;  // candidates sorted in shared memory (top-k path)
constexpr int kVecPer = kMaxVocab / 8 / kSampThreads;  // 8-token groups a thread holds in registers
constexpr int kBanWords = kMaxVocab / 32;
constexpr int kFastTopK = 512;  // top-k bound of the thread-maximum threshold path
// Larger sorted candidate sets (any top-k above kMaxSortK, or top-p without top-k)
// sort the whole row in the dynamic shared memory as 8-byte keys: vocabularies
// of at most this many ids (padded to a power of two).
constexpr int kMaxLargeSort = 16384;

__host__ __device__ inline int large_sort_slots(int V) {
  int n = 1;
  while (n < V) n <<= 1;
  return n;
}

struct SampleParams {
  float temperature;
  int top_k;  // <= 0: no top-k
  float top_p;
  int greedy;
};

// Order-preserving uint32 key of an fp32 value (larger value -> larger key).
__device__ __forceinline__ uint32_t order_key(float v) {
  const uint32_t u = __float_as_uint(v);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
// Inverse of order_key.
__device__ __forceinline__ float key_value(uint32_t key) {
  return __uint_as_float((key & 0x80000000u) ? (key & 0x7fffffffu) : ~key);
}

// Fixed part of the per-CTA shared memory; the uint32 order keys of the
// sampling values (V entries) follow it in dynamic shared memory.
struct alignas(16) RowSmem {
  unsigned long long cand[kMaxSortK];   // (~key << 32 | id) sort keys
  float cval[kMaxSortK];                // candidate scaled logits in sorted order
  int cid[kMaxSortK];
  unsigned int hist[kSampThreads / 32][256];  // per-warp private radix histograms
  unsigned int hsum[256];
  unsigned int ban[kBanWords];          // forbidden-id bitmap of the sampling copy
  double dred[32];
  float red[32];
  int ired[32];
  int misc[8];
};

// The bf16 logits row in registers: thread t holds the 8-token groups
// t, t + 512, t + 1024, ... (16-byte loads).
struct RowRegs {
  uint4 v[kVecPer];
};

__device__ __forceinline__ float group_elem(const uint4& g, int e) {
  const uint32_t w = e < 4 ? (e < 2 ? g.x : g.y) : (e < 6 ? g.z : g.w);
  return (e & 1) ? bf16_hi(w) : bf16_lo(w);
}

// Block reduction of (value, index): max value, lowest index among ties.
__device__ __forceinline__ void block_argmax(float v, int i, RowSmem& s, float& out_v, int& out_i) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, v, o);
    const int oi = __shfl_xor_sync(0xffffffffu, i, o);
    if (ov > v || (ov == v && oi < i)) { v = ov; i = oi; }
  }
  __syncthreads();
  if (lane == 0) { s.red[warp] = v; s.ired[warp] = i; }
  __syncthreads();
  if (warp == 0) {
    v = lane < (int)(blockDim.x >> 5) ? s.red[lane] : -INFINITY;
    i = lane < (int)(blockDim.x >> 5) ? s.ired[lane] : 0x7fffffff;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, v, o);
      const int oi = __shfl_xor_sync(0xffffffffu, i, o);
      if (ov > v || (ov == v && oi < i)) { v = ov; i = oi; }
    }
    if (lane == 0) { s.red[0] = v; s.ired[0] = i; }
  }
  __syncthreads();
  out_v = s.red[0];
  out_i = s.ired[0];
  __syncthreads();
}

// Exclusive block scan of one int per thread (blockDim.x <= 1024).
__device__ __forceinline__ int block_exclusive_scan(int x, RowSmem& s, int& total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int incl = x;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += y;
  }
  __syncthreads();
  if (lane == 31) s.ired[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    const int nw = blockDim.x >> 5;
    int w = lane < nw ? s.ired[lane] : 0;
    int wi = w;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, wi, o);
      if (lane >= o) wi += y;
    }
    if (lane < nw) s.ired[lane] = wi - w;  // exclusive warp offsets
    if (lane == nw - 1) s.misc[7] = wi;
  }
  __syncthreads();
  const int res = s.ired[warp] + incl - x;
  total = s.misc[7];
  __syncthreads();
  return res;
}

// Exclusive block scan of one double per thread. Callers use it only when every
// partial sum is exactly representable, so the association order is irrelevant.
__device__ __forceinline__ double block_exclusive_scan_f64(double x, RowSmem& s) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  double incl = x;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const double y = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += y;
  }
  __syncthreads();
  if (lane == 31) s.dred[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    const int nw = blockDim.x >> 5;
    const double w = lane < nw ? s.dred[lane] : 0.0;
    double wi = w;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const double y = __shfl_up_sync(0xffffffffu, wi, o);
      if (lane >= o) wi += y;
    }
    if (lane < nw) s.dred[lane] = wi - w;
  }
  __syncthreads();
  const double res = s.dred[warp] + (incl - x);
  __syncthreads();
  return res;
}

// Loads a bf16 logits row into registers, clears the forbidden bitmap and returns
// the raw log-softmax pieces (max, log-sum-exp) of the unmasked row
// (aios/engine/sample.py:74). Ends with a barrier.
__device__ __forceinline__ void load_row(RowSmem& s, RowRegs& rr, const __nv_bfloat16* lrow, int V, float& mx,
                                         float& lse) {
  const int tid = threadIdx.x;
  const int ngroups = (V + 7) >> 3;
  const bool vec = (reinterpret_cast<uintptr_t>(lrow) & 15u) == 0;
  const uint16_t* h = reinterpret_cast<const uint16_t*>(lrow);
#pragma unroll
  for (int q = 0; q < kVecPer; ++q) {
    const int j = tid + q * kSampThreads;
    uint4 x = make_uint4(0u, 0u, 0u, 0u);
    if (j < ngroups) {
      if (vec && 8 * j + 8 <= V) {
        x = *reinterpret_cast<const uint4*>(lrow + 8 * j);
      } else {  // ragged tail or a row that is not 16-byte aligned
        uint32_t w[4] = {0u, 0u, 0u, 0u};
        for (int e = 0; e < 8; ++e)
          if (8 * j + e < V) w[e >> 1] |= (uint32_t)h[8 * j + e] << ((e & 1) * 16);
        x = make_uint4(w[0], w[1], w[2], w[3]);
      }
    }
    rr.v[q] = x;
  }
  for (int w = tid; w < (V + 31) / 32; w += kSampThreads) s.ban[w] = 0u;
  float m = -INFINITY;
#pragma unroll
  for (int q = 0; q < kVecPer; ++q) {
    const int j = tid + q * kSampThreads;
    if (j < ngroups) {
#pragma unroll
      for (int e = 0; e < 8; ++e)
        if (8 * j + e < V) m = fmaxf(m, group_elem(rr.v[q], e));
    }
  }
  m = block_max(m, s.red);
  float se = 0.f;
#pragma unroll
  for (int q = 0; q < kVecPer; ++q) {
    const int j = tid + q * kSampThreads;
    if (j < ngroups) {
#pragma unroll 1  // compact code: the step kernel runs cold each decode step
      for (int e = 0; e < 8; ++e)
        if (8 * j + e < V) se += expf(group_elem(rr.v[q], e) - m);
    }
  }
  se = block_sum(se, s.red);
  mx = m;
  lse = logf(se);
  __syncthreads();
}

// Forbids one id on the sampling copy (-inf, aios/engine/sample.py:76-111).
__device__ __forceinline__ void ban_id(RowSmem& s, int id) { atomicOr(&s.ban[id >> 5], 1u << (id & 31)); }

// Writes the order keys of the sampling values (forbidden -> -inf, then
// scaled = value / temperature, aios/engine/sample.py:120) into keys[] and
// returns the thread's largest key (0 when it holds no token).
__device__ __forceinline__ uint32_t make_keys(const RowSmem& s, const RowRegs& rr, uint32_t* keys, int V,
                                              float temperature) {
  const int ngroups = (V + 7) >> 3;
  uint32_t best = 0u;
#pragma unroll
  for (int q = 0; q < kVecPer; ++q) {
    const int j = threadIdx.x + q * kSampThreads;
    if (j < ngroups) {
      const uint32_t bits = s.ban[j >> 2] >> ((j & 3) * 8);  // 8 tokens of a group share a word
#pragma unroll 1  // compact code: the step kernel runs cold each decode step
      for (int e = 0; e < 8; ++e) {
        float v = group_elem(rr.v[q], e);
        if ((bits >> e) & 1u) v = -INFINITY;
        if (8 * j + e < V) {
          const uint32_t kk = order_key(v / temperature);
          keys[8 * j + e] = kk;
          best = kk > best ? kk : best;
        }
      }
    }
  }
  return best;
}

// Order keys of the unscaled values (forbidden -> -inf) for the sorted paths,
// whose candidates are divided by the temperature only after selection. For
// t > 0, v -> fl(v / t) is monotonic, and two distinct bf16 values differ by at
// least 2^-8 relatively, so their fp32 quotients stay distinct unless the
// quotient overflows, is subnormal (t >= 2^16) or the value is a NaN: ranking v
// then ranks fl(v / t), ties included. `hazard` is set when a value of the row
// is outside that range (|v| > big); the caller then uses make_keys.
__device__ __forceinline__ uint32_t make_raw_keys(const RowSmem& s, const RowRegs& rr, uint32_t* keys, int V,
                                                  float big, bool& hazard) {
  const int ngroups = (V + 7) >> 3;
  uint32_t best = 0u;
  bool hz = false;
#pragma unroll
  for (int q = 0; q < kVecPer; ++q) {
    const int j = threadIdx.x + q * kSampThreads;
    if (j < ngroups) {
      const uint32_t bits = s.ban[j >> 2] >> ((j & 3) * 8);
#pragma unroll 1  // compact code: the step kernel runs cold each decode step
      for (int e = 0; e < 8; ++e) {
        float v = group_elem(rr.v[q], e);
        if (8 * j + e < V) {
          hz |= !(fabsf(v) <= big);  // NaN included
          if ((bits >> e) & 1u) v = -INFINITY;
          const uint32_t kk = order_key(v);
          keys[8 * j + e] = kk;
          best = kk > best ? kk : best;
        }
      }
    }
  }
  hazard = hz;
  return best;
}

// Greedy: first index of the maximum of the masked (unscaled) row (torch argmax).
__device__ __forceinline__ int greedy_pick(RowSmem& s, const RowRegs& rr, int V) {
  const int ngroups = (V + 7) >> 3;
  float bv = -INFINITY;
  int bi = 0x7fffffff;
#pragma unroll
  for (int q = 0; q < kVecPer; ++q) {
    const int j = threadIdx.x + q * kSampThreads;
    if (j < ngroups) {
      const uint32_t bits = s.ban[j >> 2] >> ((j & 3) * 8);
#pragma unroll 1  // compact code: the step kernel runs cold each decode step
      for (int e = 0; e < 8; ++e) {
        const int i = 8 * j + e;
        float v = group_elem(rr.v[q], e);
        if ((bits >> e) & 1u) v = -INFINITY;
        if (i < V && (v > bv || (v == bv && i < bi))) { bv = v; bi = i; }
      }
    }
  }
  float mv;
  int mi;
  block_argmax(bv, bi, s, mv, mi);
  return mi == 0x7fffffff ? 0 : mi;
}

// Number of leading prefixes i of the probability sequence prob(0..k) with
// fl32(cumsum_i) < thr (strict) or <= thr. The cumulative sums accumulate in fp64
// and each prefix rounds to fp32, as torch's CPU cumsum does for float tensors.
// When every non-zero probability is >= 2^-29, every fp64 partial sum (< 2) is an
// exact multiple of 2^-52, so a parallel scan reproduces the sequential sums bit
// for bit; otherwise thread 0 runs the sequential loop.
template <class Prob>
__device__ int count_prefix(RowSmem& s, const Prob& prob, int k, int lo, int hi, float thr, bool strict) {
  bool ok = true;
  double tsum = 0.0;
  for (int i = lo; i < hi; ++i) {
    const float p = prob(i);
    ok &= (p == 0.f || p >= 0x1p-29f);
    tsum += (double)p;
  }
  if (__syncthreads_and(ok)) {
    double acc = block_exclusive_scan_f64(tsum, s);
    int cnt = 0;
    for (int i = lo; i < hi; ++i) {
      acc += (double)prob(i);
      const float f = __double2float_rn(acc);
      cnt += strict ? (f < thr) : (f <= thr);
    }
    int total;
    block_exclusive_scan(cnt, s, total);
    return total;
  }
  if (threadIdx.x == 0) {
    double acc = 0.0;
    int cnt = 0;
    for (int i = 0; i < k; ++i) {
      acc += (double)prob(i);
      const float f = __double2float_rn(acc);
      if (strict ? (f < thr) : (f <= thr)) cnt = i + 1;
      else break;
    }
    s.misc[4] = cnt;
  }
  __syncthreads();
  const int cnt = s.misc[4];
  __syncthreads();
  return cnt;
}

// pick_index for k <= 64 on warp 0 alone (lane l holds candidates l and l + 32),
// with the association of every sum and scan exactly as pick_index's block form
// has it for k <= 64 (one candidate per thread): the same results, no barriers.
template <class Val>
__device__ int pick_index_warp(const Val& val, int k, float top_p, float u) {
  const int lane = threadIdx.x & 31;
  const bool h0 = lane < k, h1 = lane + 32 < k;
  const float v0 = h0 ? val(lane) : -INFINITY, v1 = h1 ? val(lane + 32) : -INFINITY;
  const float mx = warp_max(fmaxf(v0, v1));
  const float e0 = h0 ? expf(v0 - mx) : 0.f, e1 = h1 ? expf(v1 - mx) : 0.f;
  // block_sum: each warp's tree sum, then the sum of the two warp totals
  const float inv = 1.0f / (warp_sum(e0) + warp_sum(e1));
  // #prefixes i with fl32(cumsum_i) compared to thr, cumsums in fp64 (exact when
  // every non-zero term is >= 2^-29, else the candidates are walked in order)
  const auto count = [&](float p0, float p1, float thr, bool strict) {
    const bool ok = __all_sync(0xffffffffu, (p0 == 0.f || p0 >= 0x1p-29f) && (p1 == 0.f || p1 >= 0x1p-29f));
    if (ok) {
      double a0 = p0, a1 = p1;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const double y0 = __shfl_up_sync(0xffffffffu, a0, o), y1 = __shfl_up_sync(0xffffffffu, a1, o);
        if (lane >= o) {
          a0 += y0;
          a1 += y1;
        }
      }
      a1 += __shfl_sync(0xffffffffu, a0, 31);
      const float f0 = __double2float_rn(a0), f1 = __double2float_rn(a1);
      const bool c0 = h0 && (strict ? f0 < thr : f0 <= thr), c1 = h1 && (strict ? f1 < thr : f1 <= thr);
      return __popc(__ballot_sync(0xffffffffu, c0)) + __popc(__ballot_sync(0xffffffffu, c1));
    }
    // sequential: every lane walks the candidates in order (each value fetched
    // from its lane by a shuffle, so the loop stays warp-uniform)
    int cnt = 0;
    double acc = 0.0;
    bool stop = false;
    for (int i = 0; i < k; ++i) {
      const float p = i < 32 ? __shfl_sync(0xffffffffu, p0, i) : __shfl_sync(0xffffffffu, p1, i - 32);
      acc += (double)p;
      const float f = __double2float_rn(acc);
      if (!stop && (strict ? (f < thr) : (f <= thr))) cnt = i + 1;
      else stop = true;
    }
    return cnt;
  };
  int keep = k;
  float inv2 = inv;
  if (top_p < 1.0f) {
    const int n_le = count(e0 * inv, e1 * inv, top_p, false);
    keep = n_le < k ? n_le + 1 : k;  // remove[i] = cumsum[i-1] > top_p, first kept
    const float s0 = lane < keep ? e0 : 0.f, s1 = lane + 32 < keep ? e1 : 0.f;
    inv2 = 1.0f / (warp_sum(s0) + warp_sum(s1));
  }
  const float q0 = lane < keep ? e0 * inv2 : 0.f, q1 = lane + 32 < keep ? e1 * inv2 : 0.f;
  const int idx = count(q0, q1, u, true);
  return idx > k - 1 ? k - 1 : idx;
}

// Softmax over the k candidate values val(0..k) (in candidate order), top-p with
// the one-position shifted mask (aios/engine/sample.py:134-146), re-softmax and
// the inverse CDF index = #(cumsum < u) clamped to k - 1 (sample.py:161-165).
template <class Val>
__device__ int pick_index(RowSmem& s, const Val& val, int k, float top_p, float u) {
  if (k <= 64) {
    if (threadIdx.x < 32) {
      const int idx = pick_index_warp(val, k, top_p, u);
      if (threadIdx.x == 0) s.misc[5] = idx;
    }
    __syncthreads();
    const int idx = s.misc[5];
    __syncthreads();
    return idx;
  }
  const int seg = (k + kSampThreads - 1) / kSampThreads;
  const int lo = min(k, (int)threadIdx.x * seg), hi = min(k, lo + seg);
  float mx = -INFINITY;
  for (int i = lo; i < hi; ++i) mx = fmaxf(mx, val(i));
  mx = block_max(mx, s.red);
  float sum = 0.f;
  for (int i = lo; i < hi; ++i) sum += expf(val(i) - mx);
  sum = block_sum(sum, s.red);
  const float inv = 1.0f / sum;  // torch's softmax scales by the reciprocal
  int keep = k;
  float inv2 = inv;
  if (top_p < 1.0f) {
    const auto p1 = [&](int i) { return expf(val(i) - mx) * inv; };
    const int n_le = count_prefix(s, p1, k, lo, hi, top_p, false);
    keep = n_le < k ? n_le + 1 : k;  // remove[i] = cumsum[i-1] > top_p, first kept
    float sum2 = 0.f;
    for (int i = lo; i < min(hi, keep); ++i) sum2 += expf(val(i) - mx);
    sum2 = block_sum(sum2, s.red);
    inv2 = 1.0f / sum2;
  }
  const auto p2 = [&](int i) { return i < keep ? expf(val(i) - mx) * inv2 : 0.f; };
  const int idx = count_prefix(s, p2, k, lo, hi, u, true);
  return idx > k - 1 ? k - 1 : idx;
}

// Bitonic sort (ascending) of np = 32 * E 64-bit keys held by one warp, E per lane
// in blocked order (lane l holds a[l*E .. l*E+E)).
template <int E>
__device__ __forceinline__ void warp_bitonic(unsigned long long* a) {
  const int lane = threadIdx.x & 31;
  unsigned long long x[E];
#pragma unroll
  for (int e = 0; e < E; ++e) x[e] = a[lane * E + e];
#pragma unroll
  for (int size = 2; size <= 32 * E; size <<= 1) {
#pragma unroll
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      if (stride >= E) {
        const int ls = stride / E;
        const bool lower = (lane & ls) == 0;
#pragma unroll
        for (int e = 0; e < E; ++e) {
          const unsigned long long y = __shfl_xor_sync(0xffffffffu, x[e], ls);
          const bool up = ((lane * E + e) & size) == 0;
          const unsigned long long lo = x[e] < y ? x[e] : y, hi = x[e] < y ? y : x[e];
          x[e] = (lower == up) ? lo : hi;
        }
      } else {
#pragma unroll
        for (int e = 0; e < E; ++e) {
          if ((e & stride) == 0) {
            const int f = e | stride;
            const bool up = ((lane * E + e) & size) == 0;
            const unsigned long long p = x[e], q = x[f];
            if ((p > q) == up) { x[e] = q; x[f] = p; }
          }
        }
      }
    }
  }
#pragma unroll
  for (int e = 0; e < E; ++e) a[lane * E + e] = x[e];
}

// Sorts s.cand[0..n) ascending (n <= kMaxSortK); pads to a power of two with ~0.
__device__ void sort_candidates(RowSmem& s, int n) {
  const int tid = threadIdx.x;
  int np = 32;
  while (np < n) np <<= 1;
  for (int i = n + tid; i < np; i += blockDim.x) s.cand[i] = ~0ull;
  __syncthreads();
  if (np <= 256) {
    if (tid < 32) {
      switch (np) {
        case 32: warp_bitonic<1>(s.cand); break;
        case 64: warp_bitonic<2>(s.cand); break;
        case 128: warp_bitonic<4>(s.cand); break;
        default: warp_bitonic<8>(s.cand); break;
      }
    }
    __syncthreads();
    return;
  }
  for (int size = 2; size <= np; size <<= 1) {
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      for (int i = tid; i < np; i += blockDim.x) {
        const int j = i ^ stride;
        if (j > i) {
          const bool up = (i & size) == 0;
          const unsigned long long a = s.cand[i], b = s.cand[j];
          if ((a > b) == up) { s.cand[i] = b; s.cand[j] = a; }
        }
      }
      __syncthreads();
    }
  }
}

// Exact top-k candidates by a four-pass radix select of the k-th largest key,
// collected in index order into s.cand[0..k) (ties at the threshold: lowest ids).
__device__ void radix_candidates(RowSmem& s, const uint32_t* keys, int V, int k) {
  const int tid = threadIdx.x;
  // four 8-bit passes, each a per-warp private histogram (no cross-warp atomic
  // contention) summed per bin, then a warp-parallel scan from the top bin down
  uint32_t prefix = 0, mask = 0;
  int remaining = k;
  const int warp = tid >> 5, lane = tid & 31;
  const int nwarps = blockDim.x >> 5;
  for (int shift = 24; shift >= 0; shift -= 8) {
    for (int b = tid; b < nwarps * 256; b += blockDim.x) (&s.hist[0][0])[b] = 0;
    __syncthreads();
    for (int i = tid; i < V; i += blockDim.x) {
      const uint32_t key = keys[i];
      const bool hit = (key & mask) == prefix;
      const unsigned bin = hit ? (key >> shift) & 0xFFu : 0x100u;
      // warp-aggregated: one atomic per distinct bin (logit keys share their top bytes)
      const unsigned peers = __match_any_sync(__activemask(), bin);
      if (hit && (__ffs(peers) - 1) == lane) atomicAdd(&s.hist[warp][bin], (unsigned)__popc(peers));
    }
    __syncthreads();
    for (int b = tid; b < 256; b += blockDim.x) {
      unsigned int t = 0;
      for (int w = 0; w < nwarps; ++w) t += s.hist[w][b];
      s.hsum[b] = t;
    }
    __syncthreads();
    if (warp == 0) {
      // lane l owns bins 255-8l .. 248-8l (descending); find the bin holding
      // the `remaining`-th largest key
      int local[8];
      int tot = 0;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        local[j] = (int)s.hsum[255 - 8 * lane - j];
        tot += local[j];
      }
      int incl = tot;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += y;
      }
      const int excl = incl - tot;
      if (excl < remaining && incl >= remaining) {
        int acc = excl, j = 0;
        for (; j < 7; ++j) {
          if (acc + local[j] >= remaining) break;
          acc += local[j];
        }
        s.misc[0] = 255 - 8 * lane - j;
        s.misc[1] = remaining - acc;
      }
    }
    __syncthreads();
    prefix |= (uint32_t)s.misc[0] << shift;
    mask |= 0xFFu << shift;
    remaining = s.misc[1];
    __syncthreads();
  }
  const uint32_t thr = prefix;    // key of the k-th largest value
  const int need_eq = remaining;  // how many keys == thr to take (lowest ids first)
  // each thread owns a contiguous id range; the counting walk starts at a
  // thread-dependent offset so that the 32 lanes of a warp hit 32 banks
  const int per = (V + blockDim.x - 1) / blockDim.x;
  const int lo = min(V, tid * per), hi = min(V, lo + per);
  const int cnt = hi - lo;
  int n_gt = 0, n_eq = 0;
  for (int t = 0; t < cnt; ++t) {
    const uint32_t key = keys[lo + (t + tid) % cnt];
    n_gt += key > thr;
    n_eq += key == thr;
  }
  int tot_gt, tot_eq;
  const int off_gt = block_exclusive_scan(n_gt, s, tot_gt);
  const int off_eq = block_exclusive_scan(n_eq, s, tot_eq);
  if (n_gt + n_eq > 0) {
    int wg = off_gt, we = off_eq;
    for (int i = lo; i < hi; ++i) {
      const uint32_t key = keys[i];
      int slot = -1;
      if (key > thr) slot = wg++;
      else if (key == thr) {
        if (we < need_eq) slot = tot_gt + we;
        ++we;
      }
      if (slot >= 0 && slot < kMaxSortK)
        s.cand[slot] = ((unsigned long long)(~key) << 32) | (unsigned long long)(uint32_t)i;
    }
  }
  __syncthreads();
}

// Sorts all V keys of a row in the dynamic shared memory: the uint32 keys[0..V)
// are widened in place into (~key << 32 | id) 8-byte sort keys over the first
// 8 * large_sort_slots(V) bytes, padded with ~0, and bitonic-sorted ascending, so
// entry i is the (i+1)-th largest value, equal values by ascending id: the first
// k entries are exactly the top-k set in the order the top-k path sorts it.
// The widening moves ids [hi / 2, hi) per round, from bytes [2 hi, 4 hi) to
// [4 hi, 8 hi): a round never writes where a later round (or itself) reads.
__device__ unsigned long long* sort_full_row(uint32_t* keys, int V) {
  const int tid = threadIdx.x;
  unsigned long long* big = reinterpret_cast<unsigned long long*>(keys);
  const int n = large_sort_slots(V);
  for (int i = V + tid; i < n; i += blockDim.x) big[i] = ~0ull;  // bytes >= 8 V: no key lives there
  for (int hi = n; hi > 1; hi >>= 1) {
    const int lo = hi >> 1;
    // sources [2 hi, 4 hi) and destinations [4 hi, 8 hi) of a round are disjoint,
    // and the destinations were read by the round before (one barrier back)
    for (int i = lo + tid; i < min(hi, V); i += blockDim.x)
      big[i] = ((unsigned long long)(~keys[i]) << 32) | (unsigned long long)(uint32_t)i;
    __syncthreads();
  }
  if (tid == 0 && V > 0) big[0] = ((unsigned long long)(~keys[0]) << 32);
  __syncthreads();
  for (int size = 2; size <= n; size <<= 1) {
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      for (int i = tid; i < n; i += blockDim.x) {
        const int j = i ^ stride;
        if (j > i) {
          const bool up = (i & size) == 0;
          const unsigned long long a = big[i], b = big[j];
          if ((a > b) == up) {
            big[i] = b;
            big[j] = a;
          }
        }
      }
      __syncthreads();
    }
  }
  return big;
}

// Samples one row. rr holds the bf16 logits, s.ban the forbidden ids; keys[] is
// V uint32 of scratch, or 8 * large_sort_slots(V) bytes when `large` (sorted
// candidate sets above kMaxSortK). Returns the token id (same value in every thread).
__device__ int sample_row(RowSmem& s, const RowRegs& rr, uint32_t* keys, int V, const SampleParams& p, float u,
                          bool large = false) {
  const int tid = threadIdx.x;
  if (p.greedy) return greedy_pick(s, rr, V);
  int k;
  bool sorted_path;
  if (p.top_k > 0) {
    k = min(p.top_k, V);
    sorted_path = true;
  } else if (p.top_p >= 1.0f) {
    k = V;
    sorted_path = false;  // candidates are all ids in index order (sample.py:126-130)
  } else {
    k = V;
    sorted_path = true;  // full descending sort (sample.py:131-132)
  }
  // sorted candidate sets above kMaxSortK need the full-row sort buffer; without
  // it (the host then rejects such a call) never index past the top-k buffer
  const bool full_sort = sorted_path && k > kMaxSortK && large;
  if (sorted_path && k > kMaxSortK && !large) k = kMaxSortK;
  // Sorted paths rank the unscaled values and divide only the selected
  // candidates (a block-wide check falls back to scaled keys, see make_raw_keys):
  // 16384 divisions fewer per row. The raw keys' low 16 bits are all zeros or
  // all ones (bf16 widened to fp32), so the bound below needs 16 bisection steps.
  uint32_t tmax;
  bool raw = false;
  if (sorted_path) {
    const float big = p.temperature < 65536.f ? 0x1.fffffep126f * p.temperature : -1.f;
    bool hz;
    tmax = make_raw_keys(s, rr, keys, V, big, hz);
    raw = __syncthreads_or(hz) == 0;
  }
  if (!raw) {
    tmax = make_keys(s, rr, keys, V, p.temperature);
    __syncthreads();
  }
  if (!sorted_path) {
    const auto val = [&](int i) { return key_value(keys[i]); };
    return pick_index(s, val, V, p.top_p, u);
  }
  if (full_sort) {
    const unsigned long long* big = sort_full_row(keys, V);
    const float t = p.temperature;
    // the same fp32 division of the selected candidates as the top-k path
    const auto val = [&](int i) {
      const float v = key_value(~(uint32_t)(big[i] >> 32));
      return raw ? v / t : v;
    };
    const int idx = pick_index(s, val, k, p.top_p, u);
    return (int)(uint32_t)(big[idx] & 0xffffffffull);
  }
  bool collected = false;
  if (k <= kFastTopK) {
    // The k-th largest of the 512 thread maxima is a lower bound L of the row's
    // k-th largest key (those k maxima are k keys >= L), so every top-k token is
    // in C = {key >= L}; |C| is close to k for non-degenerate rows. L by bisection
    // on the key bits with block-wide counts.
    uint32_t L = 0u;
    for (int b = 31; b >= (raw ? 16 : 0); --b) {
      const uint32_t c = L | (1u << b);
      if (__syncthreads_count(tmax >= c) >= k) L = c;
    }
    const int ngroups = (V + 7) >> 3;
    int n = 0;
#pragma unroll
    for (int q = 0; q < kVecPer; ++q) {
      const int j = tid + q * kSampThreads;
      if (j < ngroups && tmax >= L) {
#pragma unroll 1  // compact code: the step kernel runs cold each decode step
        for (int e = 0; e < 8; ++e) n += (8 * j + e < V && keys[8 * j + e] >= L) ? 1 : 0;
      }
    }
    int total;
    int off = block_exclusive_scan(n, s, total);
    if (total <= kMaxSortK) {
      if (n > 0) {
#pragma unroll
        for (int q = 0; q < kVecPer; ++q) {
          const int j = tid + q * kSampThreads;
          if (j < ngroups) {
#pragma unroll 1  // compact code: the step kernel runs cold each decode step
            for (int e = 0; e < 8; ++e) {
              const int i = 8 * j + e;
              if (i < V && keys[i] >= L)
                s.cand[off++] = ((unsigned long long)(~keys[i]) << 32) | (unsigned long long)(uint32_t)i;
            }
          }
        }
      }
      __syncthreads();
      sort_candidates(s, total);
      collected = true;
    }
  }
  if (!collected) {
    radix_candidates(s, keys, V, k);
    sort_candidates(s, k);
  }
  for (int i = tid; i < k; i += blockDim.x) {
    const unsigned long long c = s.cand[i];
    s.cid[i] = (int)(uint32_t)(c & 0xffffffffull);
    const float v = key_value(~(uint32_t)(c >> 32));
    s.cval[i] = raw ? v / p.temperature : v;  // the same fp32 division as make_keys
  }
  __syncthreads();
  const auto val = [&](int i) { return s.cval[i]; };
  const int idx = pick_index(s, val, k, p.top_p, u);
  return s.cid[idx];
}

}  // namespace
}  // namespace aiosb

namespace aiosb {
namespace {

// Forbids a shared list of ids on the sampling copy (ids outside the vocabulary
// are ignored, like the reference's index_fill on a filtered list).
__device__ __forceinline__ void apply_forbidden(RowSmem& s, int V, const int32_t* ids, int n) {
  for (int j = threadIdx.x; j < n; j += blockDim.x) {
    const int id = ids[j];
    if (id >= 0 && id < V) ban_id(s, id);
  }
}

// ---- generic sampler: Sampler.sample_with_logprobs ------------------------
__global__ void __launch_bounds__(kSampThreads, 1)
    sample_kernel(const __nv_bfloat16* __restrict__ logits, int64_t row_stride, int V, SampleParams p,
                  const float* __restrict__ uniforms, const int32_t* __restrict__ forbidden, int n_forbidden,
                  const int64_t* __restrict__ forbidden_rows, int n_forbidden_rows, int64_t* __restrict__ tok_out,
                  float* __restrict__ lp_out, int32_t* status, int large) {
  extern __shared__ uint8_t smem_raw[];
  RowSmem& s = *reinterpret_cast<RowSmem*>(smem_raw);
  uint32_t* keys = reinterpret_cast<uint32_t*>(smem_raw + sizeof(RowSmem));
  pdl_enter();
  const int r = blockIdx.x;
  const __nv_bfloat16* lrow = logits + (int64_t)r * row_stride;
  RowRegs rr;
  float mx, lse;
  load_row(s, rr, lrow, V, mx, lse);
  apply_forbidden(s, V, forbidden, n_forbidden);
  if (forbidden_rows != nullptr) {
    for (int j = threadIdx.x; j < n_forbidden_rows; j += blockDim.x) {
      const int64_t id = forbidden_rows[(int64_t)r * n_forbidden_rows + j];
      if (id >= 0 && id < V) ban_id(s, (int)id);
      else report(status, AIOSB_DEV_TOKEN_RANGE);
    }
  }
  __syncthreads();
  const float u = uniforms != nullptr ? uniforms[r] : 0.5f;
  const int tok = sample_row(s, rr, keys, V, p, u, large != 0);
  if (threadIdx.x == 0) {
    tok_out[r] = tok;
    lp_out[r] = (bf16_to_f(lrow[tok]) - mx) - lse;
  }
}

// ---- CandidateGroup step ----------------------------------------------------
// Row r of the group (aios/ime.py:998-1037) is sampled by one CTA, or by a
// cluster of C CTAs (AIOSB_GROUP_SPLIT). With C > 1 and a top-k sorted path (top_k <= 512, not
// greedy), CTA c of the cluster takes the c-th 1/C slice of the vocabulary: its
// max and sum of exponentials (the raw log-softmax pieces), the order keys of
// the unscaled values and its own k-th largest key L_c (exact, by bisection on
// the key bits). The slices exchange these over distributed
// shared memory; every key >= max_c L_c (at least k of them: CTA argmax_c L_c
// alone holds k; at most k per slice) goes to the leader (rank 0), which sorts the candidates and
// picks with the same arithmetic as the one-CTA path, and combines the log-sum-
// exp as M + log(sum_c s_c exp(m_c - M)). Greedy, top-p without top-k, larger
// k, more than 2048 candidates (rows of ties) and values where dividing by the
// temperature could overflow take the one-CTA path on the leader. Only leaders
// do the row bookkeeping; the last leader to finish runs the step's host-free
// epilogue: compaction of finished rows, FIFO slot allocation in active-row
// order (aios/scheduler/cache.py:46-51), page-table writes (aios/ime.py:1229)
// and the next forward's metadata.
constexpr int kMaxSplit = 8;
constexpr int kSplitVec = kVecPer / 2;  // 8-id groups per thread in a slice of at least 2
// Measured on the S10 keystroke (8 rows, one box, two runs each, ms p50):
// 1 CTA per row 3.018 / 3.017, 2 CTAs 3.016 / 3.041, 4 CTAs 3.030 / 3.042,
// 8 CTAs 3.040 / 3.055. The step is bound by its chain of block barriers and
// cold instruction fetches, not by the per-thread work a split divides, and a
// split adds two cluster barriers: one CTA per row stays the default.
constexpr int kDefaultSplit = 1;
struct SplitXchg {
  float m[kMaxSplit], se[kMaxSplit];
  uint32_t bound[kMaxSplit];
  int hazard[kMaxSplit];
  uint32_t count;  // leader: candidates reserved so far
  int base;
  int cnt[2][kSampThreads / 32];  // bisection counts per warp (two alternating buffers)
};

__device__ __forceinline__ void st_cluster_f32(uint32_t addr, float v) {
  asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(addr), "f"(v) : "memory");
}
__device__ __forceinline__ void st_cluster_u32(uint32_t addr, uint32_t v) {
  asm volatile("st.shared::cluster.u32 [%0], %1;" ::"r"(addr), "r"(v) : "memory");
}
__device__ __forceinline__ void st_cluster_u64(uint32_t addr, unsigned long long v) {
  asm volatile("st.shared::cluster.u64 [%0], %1;" ::"r"(addr), "l"(v) : "memory");
}
__device__ __forceinline__ uint32_t atom_add_cluster_u32(uint32_t addr, uint32_t v) {
  uint32_t old;
  asm volatile("atom.shared::cluster.add.u32 %0, [%1], %2;" : "=r"(old) : "r"(addr), "r"(v) : "memory");
  return old;
}

// SPLIT = false: the one-CTA kernel (C == 1), with no cluster code compiled in.
template <bool SPLIT>
__global__ void __launch_bounds__(kSampThreads, 1) group_step_kernel(aiosb_group_ptrs g, int large, int C, int Vl) {
  extern __shared__ uint8_t smem_raw[];
  RowSmem& s = *reinterpret_cast<RowSmem*>(smem_raw);
  uint32_t* keys = reinterpret_cast<uint32_t*>(smem_raw + sizeof(RowSmem));
  __shared__ SplitXchg xs;
  // After the decode forward (AIOSB_GROUP_AFTER_FORWARD) everything but the
  // logits and tile statistics was written before that forward began: the
  // state, the row arrays and the id lists are read while the LM head still
  // runs, and the wait comes just before the logits. Otherwise (after
  // group_begin, or any other caller) the step waits first.
  const bool early_reads = !SPLIT && (g.flags & AIOSB_GROUP_AFTER_FORWARD) != 0;
  pdl_launch_dependents();
  if (!early_reads) pdl_wait();
  aiosb_group_state* st = g.state;
  const int r = blockIdx.x / C;
  const int c = SPLIT ? (int)cluster_ctarank() : 0;
  const bool leader = c == 0;
  const int tid = threadIdx.x;
  const int lane = tid & 31;
  const bool warp0 = tid < 32 && leader;
  // The tile statistics (see the tile-statistics path below) are requested with
  // the state: their addresses need only the launch's vocabulary and rows, and
  // whether this step uses them is known once the state has arrived.
  constexpr int kTilesPer = kMaxVocab / 16 / kSampThreads;
  const int NTv = Vl >> 4;
  const bool tiles_in = !SPLIT && g.tile_stats != nullptr && (Vl & 15) == 0 && Vl <= kMaxVocab;
  float4 tv[kTilesPer];
  auto load_tiles = [&]() {
#pragma unroll
    for (int q = 0; q < kTilesPer; ++q) {
      const int t = tid + q * kSampThreads;
      tv[q] = make_float4(-INFINITY, 0.f, INFINITY, 0.f);
      if (tiles_in && t < NTv) tv[q] = reinterpret_cast<const float4*>(g.tile_stats)[(int64_t)t * gridDim.x + r];
    }
  };
  if (!early_reads) load_tiles();
  const int step = st->step;
  const int V = st->vocab;
  const int S = st->max_steps;
  const int st_done = st->done;
  const bool run = st_done == 0 && g.active[r] != 0;
  // The bookkeeping and the step epilogue run in warp 0 of leaders (of the last
  // one for the epilogue). Their inputs are requested now, so that the round
  // trips overlap the sampling instead of forming a chain after it: the state
  // fields that only the epilogue writes (no CTA of this launch writes them
  // before every leader has arrived). Measured: 2.5 us less per decode step.
  int R = 0, P = 1, prefix_len = 0, row_offset = 0, n_terminal = 0, eos_id = 0, pad_id = 0, amt = 0;
  int64_t head = 0, tail = 0, cap = 0, table_stride = 0;
  if (warp0) {
    R = st->rows;
    P = st->page_size;
    prefix_len = st->prefix_len;
    row_offset = st->row_offset;
    n_terminal = st->n_terminal;
    eos_id = st->eos_id;
    pad_id = st->pad_id;
    amt = st->active_model_tokens;
    head = st->head;
    tail = st->tail;
    cap = st->capacity;
    table_stride = st->table_stride;
  }
  SampleParams p;
  p.temperature = st->temperature;
  p.top_k = st->top_k;
  p.top_p = st->top_p;
  p.greedy = st->greedy;
  const __nv_bfloat16* lrow = reinterpret_cast<const __nv_bfloat16*>(g.logits) + (int64_t)r * V;
  // second round of epilogue inputs, addressed by the fields above: lane l holds
  // row l's active flag and suffix page, terminal id l, and the FIFO entry l
  // places past the head (the slot of the alive row of rank l)
  int e_active = 0, e_page = 0, e_term = -1, e_ring = 0, e_count = 0;
  float e_lpsum = 0.f;
  if (warp0) {
    if (lane < R) e_active = g.active[lane];
    if (lane < R && P > 1) e_page = g.row_page[lane];
    if (lane < n_terminal) e_term = g.terminal_ids[lane];
    if (cap > 0) e_ring = g.ring[(head + lane) % cap];
    if (lane == 0 && run) {
      e_count = g.counts[r];
      e_lpsum = g.logprob_sums[r];
    }
  }
  // the sampling copy's forbidden ids (aios/engine/sample.py:76-111): the
  // minimum-length list, and the refill exact-repeat bans (aios/ime.py:974-996):
  // for every banned sequence b, its token at `step` if this row's output so far
  // equals its prefix, otherwise the pad id (the reference fills non-matching
  // slots with pad)
  auto apply_bans = [&]() {
    if (step < st->min_new_tokens) apply_forbidden(s, V, g.minlen_ids, st->n_minlen);
    if (st->n_banned > 0 && step >= st->ban_min_prefix && step < st->banned_width) {
      for (int b = tid; b < st->n_banned; b += blockDim.x) {
        const int32_t* seq = g.banned + (int64_t)b * st->banned_width;
        bool match = g.banned_len[b] > step;
        for (int t = 0; t < step && match; ++t) match = g.output_ids[(int64_t)r * S + t] == seq[t];
        const int id = match ? seq[step] : st->pad_id;
        if (id >= 0 && id < V) ban_id(s, id);
      }
    }
  };
  const float u = run ? g.uniforms[(int64_t)r * S + step] : 0.f;
  if (early_reads) {
    pdl_wait();  // the LM head's logits and tile statistics
    load_tiles();
  }
  int tok = 0;
  float mx = 0.f, lse = 0.f;
  bool have = false;
  const bool split = SPLIT && run && !p.greedy && p.top_k >= 1 && p.top_k <= kFastTopK;
  if (split) {
    // ---- this CTA's slice: ids [lo, hi) as 8-id groups; thread t holds groups
    // t, t + 512, ... (at most kSplitVec: C >= 2 halves the widest row)
    const int W = (V + 8 * C - 1) / (8 * C) * 8;
    const int lo = c * W, hi = min(V, lo + W);
    const uint16_t* h16 = reinterpret_cast<const uint16_t*>(lrow);
    uint4 x[kSplitVec];
    int nvalid[kSplitVec];
#pragma unroll
    for (int q = 0; q < kSplitVec; ++q) {
      const int id0 = lo + 8 * (tid + q * kSampThreads);
      nvalid[q] = id0 < hi ? min(8, hi - id0) : 0;
      x[q] = make_uint4(0u, 0u, 0u, 0u);
      if (nvalid[q] == 8 && (reinterpret_cast<uintptr_t>(lrow + id0) & 15u) == 0) {
        x[q] = *reinterpret_cast<const uint4*>(lrow + id0);
      } else if (nvalid[q] > 0) {
        uint32_t w[4] = {0u, 0u, 0u, 0u};
        for (int e = 0; e < nvalid[q]; ++e) w[e >> 1] |= (uint32_t)h16[id0 + e] << ((e & 1) * 16);
        x[q] = make_uint4(w[0], w[1], w[2], w[3]);
      }
    }
    for (int w = lo / 32 + tid; w < (hi + 31) / 32; w += blockDim.x) s.ban[w] = 0u;
    if (leader && tid == 0) xs.count = 0u;
    __syncthreads();
    apply_bans();
    float m = -INFINITY;
#pragma unroll
    for (int q = 0; q < kSplitVec; ++q)
#pragma unroll
      for (int e = 0; e < 8; ++e)
        if (e < nvalid[q]) m = fmaxf(m, group_elem(x[q], e));
    m = block_max(m, s.red);
    float se = 0.f;
#pragma unroll
    for (int q = 0; q < kSplitVec; ++q)
#pragma unroll
      for (int e = 0; e < 8; ++e)
        if (e < nvalid[q]) se += expf(group_elem(x[q], e) - m);
    se = block_sum(se, s.red);  // ends with a barrier: the bans are complete
    const float big = p.temperature < 65536.f ? 0x1.fffffep126f * p.temperature : -1.f;
    uint32_t kv[kSplitVec][8];
    bool hz = false;
#pragma unroll
    for (int q = 0; q < kSplitVec; ++q) {
      const int id0 = lo + 8 * (tid + q * kSampThreads);
      const uint32_t bits = nvalid[q] > 0 ? s.ban[id0 >> 5] >> (id0 & 31) : 0u;  // id0 % 8 == 0: one word
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        kv[q][e] = 0u;
        if (e < nvalid[q]) {
          float v = group_elem(x[q], e);
          hz |= !(fabsf(v) <= big);  // NaN included
          if ((bits >> e) & 1u) v = -INFINITY;
          kv[q][e] = order_key(v);
        }
      }
    }
    const int k = min(p.top_k, V);
    // L_c: this slice's exact k-th largest key (0 when it holds fewer than k
    // ids), by bisection on the 16 significant bits of the raw keys with a block
    // count per step; the per-warp counts alternate between two buffers, so one
    // barrier per step suffices
    uint32_t L = 0u;
    const int warp = tid >> 5;
    for (int b = 31, buf = 0; b >= 16; --b, buf ^= 1) {
      const uint32_t cand = L | (1u << b);
      int n = 0;
#pragma unroll
      for (int q = 0; q < kSplitVec; ++q)
#pragma unroll
        for (int e = 0; e < 8; ++e) n += kv[q][e] >= cand ? 1 : 0;
      n = (int)__reduce_add_sync(0xffffffffu, (unsigned)n);
      if (lane == 0) xs.cnt[buf][warp] = n;
      __syncthreads();
      int tot = 0;
#pragma unroll
      for (int w = 0; w < kSampThreads / 32; ++w) tot += xs.cnt[buf][w];
      if (tot >= k) L = cand;
    }
    const int any_hz = __syncthreads_or(hz);
    // exchange 1: every CTA writes its slot c into every peer's exchange block
    if (tid < C) {
      const uint32_t q = (uint32_t)tid;
      st_cluster_f32(map_shared_rank(smem_u32(&xs.m[c]), q), m);
      st_cluster_f32(map_shared_rank(smem_u32(&xs.se[c]), q), se);
      st_cluster_u32(map_shared_rank(smem_u32(&xs.bound[c]), q), L);
      st_cluster_u32(map_shared_rank(smem_u32(&xs.hazard[c]), q), (uint32_t)any_hz);
    }
    cluster_sync();
    uint32_t Lg = 0u;
    bool hzg = false;
    float M = -INFINITY;
    for (int q = 0; q < C; ++q) {
      Lg = xs.bound[q] > Lg ? xs.bound[q] : Lg;
      hzg |= xs.hazard[q] != 0;
      M = fmaxf(M, xs.m[q]);
    }
    if (!hzg) {
      // exchange 2: candidates (key >= Lg) into the leader's buffer
      int n = 0;
#pragma unroll
      for (int q = 0; q < kSplitVec; ++q)
#pragma unroll
        for (int e = 0; e < 8; ++e) n += (e < nvalid[q] && kv[q][e] >= Lg) ? 1 : 0;
      int total;
      int off = block_exclusive_scan(n, s, total);
      if (tid == 0) xs.base = (int)atom_add_cluster_u32(map_shared_rank(smem_u32(&xs.count), 0u), (uint32_t)total);
      __syncthreads();
      off += xs.base;
      const uint32_t cand0 = map_shared_rank(smem_u32(&s.cand[0]), 0u);
#pragma unroll
      for (int q = 0; q < kSplitVec; ++q) {
        const int id0 = lo + 8 * (tid + q * kSampThreads);
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          if (e < nvalid[q] && kv[q][e] >= Lg) {
            if (off < kMaxSortK)
              st_cluster_u64(cand0 + (uint32_t)off * 8u,
                             ((unsigned long long)(~kv[q][e]) << 32) | (unsigned long long)(uint32_t)(id0 + e));
            ++off;
          }
        }
      }
      cluster_sync();
      if (!leader) return;  // nothing reads this CTA's shared memory after the barrier
      const int total_all = (int)xs.count;
      if (total_all <= kMaxSortK) {
        sort_candidates(s, total_all);
        for (int i = tid; i < k; i += blockDim.x) {
          const unsigned long long cv = s.cand[i];
          s.cid[i] = (int)(uint32_t)(cv & 0xffffffffull);
          s.cval[i] = key_value(~(uint32_t)(cv >> 32)) / p.temperature;  // the fp32 division of make_keys
        }
        __syncthreads();
        const auto val = [&](int i) { return s.cval[i]; };
        tok = s.cid[pick_index(s, val, k, p.top_p, u)];
        float sum = 0.f;
        for (int q = 0; q < C; ++q) sum += xs.se[q] * expf(xs.m[q] - M);
        mx = M;
        lse = logf(sum);
        have = true;
      }
    } else if (!leader) {
      return;
    }
  } else if (!leader) {
    return;
  }
  // ---- tile-statistics path (one CTA per row; steps whose logits the decode
  // forward's LM head wrote, with per-16-id tile statistics: max, sum of
  // exp(v - max), min, NaN flag of the stored logits). The row max is the max
  // of the tile maxima and the log-sum-exp M + log(sum_t s_t exp(m_t - M)); the
  // overflow check reads the tile max and min. With B forbidden ids at most
  // (the minimum-length list and the repeat bans), any L with k + B tiles whose
  // max is >= L bounds the k-th largest allowed value from below: those tiles'
  // maxima are distinct ids >= L, at most B of them forbidden. L is the
  // (k + B)-th largest of the threads' largest tile maxima. Only tiles whose
  // max is >= L can hold a candidate; their 16 logits are read, and the
  // keys >= L (forbidden -> -inf, as make_raw_keys) are sorted and picked
  // exactly as the thread-maximum path does, giving the same token. Rows that
  // could overflow, ask for more tiles than the row has, or hold more than
  // kMaxSortK candidates take the full path below.
  if (tiles_in && run && !have && V == Vl && NTv >= 16 && step > 0 && !p.greedy && p.top_k >= 1 &&
      p.top_k <= kFastTopK && (reinterpret_cast<uintptr_t>(g.logits) & 15u) == 0) {
    const int NT = NTv;
    const int warp = tid >> 5;
    const int k = min(p.top_k, V);
    int nb = step < st->min_new_tokens ? st->n_minlen : 0;
    if (st->n_banned > 0 && step >= st->ban_min_prefix && step < st->banned_width) nb += st->n_banned;
    const int need = k + nb;
    for (int w = tid; w < (V + 31) / 32; w += blockDim.x) s.ban[w] = 0u;
    __syncthreads();
    apply_bans();
    const float big = p.temperature < 65536.f ? 0x1.fffffep126f * p.temperature : -1.f;
    float m = -INFINITY;
    bool hz = false;
#pragma unroll
    for (int q = 0; q < kTilesPer; ++q) {
      const int t = tid + q * kSampThreads;
      if (t < NT) {
        m = fmaxf(m, tv[q].x);
        hz |= !(fabsf(tv[q].x) <= big) || !(fabsf(tv[q].z) <= big) || tv[q].w != 0.f;  // NaN included
      }
    }
    // per-warp max and sum of exponentials relative to it (combined after the
    // barrier), and this thread's largest tile key
    const float wm = warp_max(m);
    float ws = 0.f;
    uint32_t tmax = 0u;
#pragma unroll
    for (int q = 0; q < kTilesPer; ++q) {
      if (tid + q * kSampThreads < NT) {
        ws += tv[q].y * expf(tv[q].x - wm);
        tmax = max(tmax, order_key(tv[q].x));
      }
    }
    ws = warp_sum(ws);
    if (lane == 0) {
      s.red[warp] = wm;
      s.red[kSampThreads / 32 + warp] = ws;
      if (warp == 0) s.misc[0] = 0;
    }
    if (__syncthreads_or(hz) == 0 && need <= NT) {  // the barrier also completes the bans
      float M = -INFINITY;
#pragma unroll
      for (int w = 0; w < kSampThreads / 32; ++w) M = fmaxf(M, s.red[w]);
      float se = 0.f;
#pragma unroll
      for (int w = 0; w < kSampThreads / 32; ++w) se += s.red[kSampThreads / 32 + w] * expf(s.red[w] - M);
      // L: the need-th largest of the 512 thread maxima of the tile keys, a lower
      // bound of the need-th largest tile max (those need maxima are distinct
      // tiles), by bisection on the 16 significant bits (tile maxima are bf16
      // values) with one counting barrier per bit
      uint32_t L = 0u;
      for (int b = 31; b >= 16; --b) {
        const uint32_t cand = L | (1u << b);
        if (__syncthreads_count(tmax >= cand) >= need) L = cand;
      }
      // the tiles whose max is >= L into s.cid, one shared atomic per warp and
      // tile round (the list's order does not matter: the candidates are sorted)
#pragma unroll
      for (int q = 0; q < kTilesPer; ++q) {
        const int t = tid + q * kSampThreads;
        const bool pass = t < NT && order_key(tv[q].x) >= L;
        const unsigned bal = __ballot_sync(0xffffffffu, pass);
        int wbase = 0;
        if (lane == 0 && bal != 0u) wbase = atomicAdd(&s.misc[0], __popc(bal));
        wbase = __shfl_sync(0xffffffffu, wbase, 0);
        if (pass) s.cid[wbase + __popc(bal & ((1u << lane) - 1u))] = t;
      }
      if (tid == 0) s.misc[1] = 0;
      __syncthreads();
      const int npass = s.misc[0];
      // candidates: half a warp per listed tile, one id per lane; each warp
      // reserves its slots with one shared atomic (the sort fixes the order)
      for (int i0 = 0; i0 < npass; i0 += kSampThreads / 16) {
        const int i = i0 + 2 * warp + (lane >> 4);
        bool pass = false;
        uint32_t kk = 0u;
        int id = 0;
        if (i < npass) {
          id = 16 * s.cid[i] + (lane & 15);
          const float v = ((s.ban[id >> 5] >> (id & 31)) & 1u) ? -INFINITY : bf16_to_f(lrow[id]);
          kk = order_key(v);
          pass = kk >= L;
        }
        const unsigned bal = __ballot_sync(0xffffffffu, pass);
        int wbase = 0;
        if (lane == 0 && bal != 0u) wbase = atomicAdd(&s.misc[1], __popc(bal));
        wbase = __shfl_sync(0xffffffffu, wbase, 0);
        const int slot = wbase + __popc(bal & ((1u << lane) - 1u));
        if (pass && slot < kMaxSortK)
          s.cand[slot] = ((unsigned long long)(~kk) << 32) | (unsigned long long)(uint32_t)id;
      }
      __syncthreads();
      const int total = s.misc[1];
      if (total >= k && total <= kMaxSortK) {
        sort_candidates(s, total);
        for (int i = tid; i < k; i += blockDim.x) {
          const unsigned long long cv = s.cand[i];
          s.cid[i] = (int)(uint32_t)(cv & 0xffffffffull);
          s.cval[i] = key_value(~(uint32_t)(cv >> 32)) / p.temperature;  // the fp32 division of make_keys
        }
        __syncthreads();
        const auto val = [&](int i) { return s.cval[i]; };
        tok = s.cid[pick_index(s, val, k, p.top_p, u)];
        mx = M;
        lse = logf(se);
        have = true;
      }
    }
  }
  if (run && !have) {
    // the one-CTA path: the whole row in this CTA
    RowRegs rr;
    load_row(s, rr, lrow, V, mx, lse);
    apply_bans();
    __syncthreads();
    tok = sample_row(s, rr, keys, V, p, u, large != 0);
  }
  // the next forward's input row (aiosb_embedding_stat's warp-per-row form, so
  // the outputs are the same bit for bit): warp 1 of the row's leader CTA
  if (run && leader && g.embed_w != nullptr && (tid >> 5) == 1) {
    const int64_t nv = g.hidden / 8;
    const uint4* w = reinterpret_cast<const uint4*>(g.embed_w);
    uint4* out = reinterpret_cast<uint4*>(g.embed_out);
    const bool ok = tok >= 0 && tok < V;
    float ss = 0.f;
    for (int64_t i = lane; i < nv; i += 32) {
      const uint4 v = ok ? w[(int64_t)tok * nv + i] : make_uint4(0u, 0u, 0u, 0u);
      out[(int64_t)r * nv + i] = v;
      const float f[8] = {bf16_lo(v.x), bf16_hi(v.x), bf16_lo(v.y), bf16_hi(v.y),
                          bf16_lo(v.z), bf16_hi(v.z), bf16_lo(v.w), bf16_hi(v.w)};
      float4* dst = reinterpret_cast<float4*>(g.embed_stat_x + (int64_t)r * g.hidden + 8 * i);
      dst[0] = make_float4(f[0], f[1], f[2], f[3]);
      dst[1] = make_float4(f[4], f[5], f[6], f[7]);
#pragma unroll
      for (int j = 0; j < 8; ++j) ss += f[j] * f[j];
    }
    ss = warp_sum(ss);
    if (lane == 0) g.embed_stat_ss[r] = ss;
  }
  if (run && warp0) {
    const bool eos = tok == eos_id;
    const bool emitted = !eos;
    bool hit = false;
    for (int j = lane; j < n_terminal; j += 32) hit |= tok == (j == lane ? e_term : g.terminal_ids[j]);
    const bool terminal = emitted && __any_sync(0xffffffffu, hit);
    if (lane == 0) {
      const float lp = (bf16_to_f(lrow[tok]) - mx) - lse;
      g.output_ids[(int64_t)r * S + step] = emitted ? tok : pad_id;
      g.counts[r] = e_count + (emitted ? 1 : 0);
      g.logprob_sums[r] = e_lpsum + (emitted ? lp : 0.f);
      g.token_logprobs[(int64_t)r * S + step] = emitted ? lp : 0.f;
      if (eos) g.stop_codes[r] = 1;
      if (terminal) g.stop_codes[r] = 2;
      g.finished[r] = (eos || terminal) ? 1 : 0;
      g.tokens[r] = tok;
    }
  }
  // ---- last CTA: step epilogue, one lane of warp 0 per row: every flag and
  // state field is read in one round, the surviving rows' FIFO ranks come from a
  // ballot (row order, as the reference's allocate of active rows), and each lane
  // writes its own row's page-table entry and next-forward metadata.
  __syncthreads();
  __shared__ int is_last;
  if (threadIdx.x == 0) {
    __threadfence();
    const int prev = atomicAdd(&st->arrive, 1);
    is_last = prev == (int)(gridDim.x / C) - 1;  // one arrival per row (leaders)
  }
  __syncthreads();
  if (!is_last || threadIdx.x >= 32) return;
  __threadfence();  // the other CTAs' row results are visible to every lane
  if (lane == 0) st->arrive = 0;
  if (st_done) return;
  const int pos = prefix_len + step;  // position of the token sampled now
  const int64_t row_base = (int64_t)row_offset * table_stride;
  // the host-mapped cancel word is read here, not at entry: a read across the
  // host bus issued at entry delayed the row loads behind it (4 us per step)
  const bool cancel = g.cancel_flag != nullptr && *reinterpret_cast<volatile const int32_t*>(g.cancel_flag) != 0;
  const bool mine = lane < R;
  const bool alive = mine && e_active != 0 && g.finished[lane] == 0;
  const unsigned alive_mask = __ballot_sync(0xffffffffu, alive);
  const int n = __popc(alive_mask);
  const int rank = __popc(alive_mask & ((1u << lane) - 1u));
  bool done = step + 1 >= S || n == 0 || cancel;
  const bool new_page = P <= 1 || (step % P) == 0;
  const int64_t need = new_page ? n : 0;
  if (!done && head + need > tail) {
    if (lane == 0) report(g.status, AIOSB_DEV_POOL_EMPTY);
    done = true;
  }
  const int32_t fifo = __shfl_sync(0xffffffffu, e_ring, rank);  // ring[(head + rank) % cap]
  if (!done && alive) {
    int64_t slot;
    if (P <= 1) {
      slot = fifo;
    } else {
      int32_t page;
      if (new_page) {
        page = fifo;
        g.row_page[lane] = page;
      } else {
        page = e_page;
      }
      slot = (int64_t)page * P + (step % P);
    }
    g.page_table[row_base + (int64_t)lane * table_stride + pos] = (int32_t)slot;
    g.out_loc[lane] = (int32_t)slot;
    g.positions[lane] = pos;
    g.seq_lens[lane] = pos + 1;
  }
  if (mine) g.active[lane] = (!done && alive) ? 1 : 0;
  if (lane == 0) {
    if (!done) {
      st->head = head + need;
      st->active_model_tokens = amt + n;
      st->n_active = n;
      st->step = step + 1;
    } else {
      st->done = 1;
      st->cancelled = cancel ? 1 : 0;
      st->n_active = 0;
    }
    if (g.host_mirror != nullptr) {
      // [steps sampled so far, done, cancelled, active rows] in one 16-byte store
      // to the page-locked mirror: the host sees the four words together, so no
      // system-scope fence has to order them (the host only paces its launches
      // by them; results are read after an event wait)
      const int w0 = step + 1, w1 = done ? 1 : 0, w2 = (done && cancel) ? 1 : 0, w3 = done ? 0 : n;
      if ((reinterpret_cast<uintptr_t>(g.host_mirror) & 15u) == 0) {
        asm volatile("st.volatile.global.v4.s32 [%0], {%1, %2, %3, %4};" ::"l"(g.host_mirror), "r"(w0), "r"(w1),
                     "r"(w2), "r"(w3)
                     : "memory");
      } else {
        volatile int32_t* m = g.host_mirror;
        m[1] = w1;
        m[2] = w2;
        m[3] = w3;
        __threadfence_system();
        m[0] = w0;  // written last
      }
    }
  }
}

// ---- round start: reset per-row outputs, broadcast prefix logits, draw the
// stateless uniform streams (aios/engine/sample.py:12-45).
__device__ __forceinline__ float splitmix_uniform(uint64_t seed, uint64_t step) {
  uint64_t v = seed + (step + 1ull) * 0x9E3779B97F4A7C15ull;
  v = (v ^ (v >> 30)) * 0xBF58476D1CE4E5B9ull;
  v = (v ^ (v >> 27)) * 0x94D049BB133111EBull;
  v ^= v >> 31;
  const double d = ((double)((v >> 11) & ((1ull << 53) - 1ull)) + 0.5) / 9007199254740992.0;
  return __double2float_rn(d);
}

__global__ void group_begin_kernel(aiosb_group_ptrs g, const __nv_bfloat16* __restrict__ prefix_logits,
                                   uint64_t seed_base, int attempts) {
  pdl_enter();
  aiosb_group_state* st = g.state;
  const int R = st->rows, S = st->max_steps, V = st->vocab;
  const int64_t tid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t nthr = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = tid; i < (int64_t)R * V; i += nthr) reinterpret_cast<__nv_bfloat16*>(g.logits)[i] = prefix_logits[i % V];
  for (int64_t i = tid; i < (int64_t)R * S; i += nthr) {
    const int r = (int)(i / S), t = (int)(i % S);
    g.uniforms[i] = splitmix_uniform(seed_base + (uint64_t)r, (uint64_t)t);
    g.output_ids[i] = st->pad_id;
    g.token_logprobs[i] = 0.f;
  }
  for (int64_t i = tid; i < R; i += nthr) {
    g.counts[i] = 0;
    g.logprob_sums[i] = 0.f;
    g.stop_codes[i] = 0;
    // NULL for callers of aiosb_group_step_static, which keeps the flags itself
    if (g.finished != nullptr) g.finished[i] = 0;
    g.active[i] = i < attempts ? 1 : 0;
    g.row_page[i] = -1;
    g.out_loc[i] = -1;
    g.row_table[i] = st->row_offset + (int32_t)i;
  }
}

__global__ void uniforms_kernel(const int64_t* __restrict__ seeds, int64_t rows, int64_t steps,
                                float* __restrict__ out) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= rows * steps) return;
  out[i] = splitmix_uniform((uint64_t)seeds[i / steps], (uint64_t)(i % steps));
}

// ---- free-slot FIFO (aios/scheduler/cache.py:9-51) on a ring of `capacity`
// int32 entries; head/tail are monotonically increasing logical indices.
__global__ void slot_alloc_kernel(const int32_t* __restrict__ ring, int64_t capacity, int64_t head, int64_t n,
                                  int32_t* __restrict__ out) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    out[i] = ring[(head + i) % capacity];
}

__global__ void slot_free_kernel(int32_t* __restrict__ ring, int64_t capacity, int64_t tail,
                                 const int32_t* __restrict__ slots, int64_t n) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    ring[(tail + i) % capacity] = slots[i];
}

// Appends ring[begin .. begin+n) at the tail. Source and destination may
// overlap modulo the capacity; one CTA reads each 4096-entry chunk completely
// before writing it, and chunks run in increasing order, which never
// overwrites an entry that is still to be read.
constexpr int kFreeChunk = 4096;
__global__ void __launch_bounds__(1024) slot_free_range_kernel(int32_t* ring, int64_t capacity, int64_t begin,
                                                               int64_t n, int64_t tail) {
  for (int64_t c0 = 0; c0 < n; c0 += kFreeChunk) {
    int32_t v[kFreeChunk / 1024];
#pragma unroll
    for (int j = 0; j < kFreeChunk / 1024; ++j) {
      const int64_t i = c0 + j * 1024 + threadIdx.x;
      v[j] = i < n ? ring[(begin + i) % capacity] : 0;
    }
    __syncthreads();
#pragma unroll
    for (int j = 0; j < kFreeChunk / 1024; ++j) {
      const int64_t i = c0 + j * 1024 + threadIdx.x;
      if (i < n) ring[(tail + i) % capacity] = v[j];
    }
    __syncthreads();
  }
}

size_t sample_smem(int V) { return sizeof(RowSmem) + (size_t)V * sizeof(uint32_t); }
// With the full-row sort: 8 bytes per (padded) id.
size_t sample_smem_large(int V) { return sizeof(RowSmem) + (size_t)large_sort_slots(V) * 8; }
// The dynamic shared memory either launch needs at most (set once per kernel).
size_t sample_smem_max() { return std::max(sample_smem(kMaxVocab), sample_smem_large(kMaxLargeSort)); }

// Page-table reset for a keystroke: rows [0, rows) get the prefix slots in
// columns [0, n) and zeros in [n, width) (the reference builds a fresh zero table
// per keystroke and writes the prefix slots into every row, aios/ime.py:482-485,1155).
__global__ void page_table_fill_kernel(int32_t* __restrict__ table, int64_t stride, int rows, int width,
                                       const int32_t* __restrict__ prefix, int n) {
  pdl_enter();
  const int64_t total = (int64_t)rows * width;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int r = (int)(i / width), c = (int)(i % width);
    table[(int64_t)r * stride + c] = c < n ? prefix[c] : 0;
  }
}

// Raw log-probability of a given target per row (teacher-forced scoring).
__global__ void __launch_bounds__(kSampThreads)
    token_logprob_kernel(const __nv_bfloat16* __restrict__ logits, int64_t row_stride, int V,
                         const int64_t* __restrict__ targets, float* __restrict__ out, int32_t* status) {
  extern __shared__ uint8_t smem_raw[];
  RowSmem& s = *reinterpret_cast<RowSmem*>(smem_raw);
  pdl_enter();
  const int r = blockIdx.x;
  const __nv_bfloat16* lrow = logits + (int64_t)r * row_stride;
  RowRegs rr;
  float mx, lse;
  load_row(s, rr, lrow, V, mx, lse);
  if (threadIdx.x == 0) {
    const int64_t t = targets[r];
    if (t < 0 || t >= V) {
      report(status, AIOSB_DEV_TOKEN_RANGE);
      out[r] = -INFINITY;
    } else {
      out[r] = (bf16_to_f(lrow[t]) - mx) - lse;
    }
  }
}

}  // namespace
}  // namespace aiosb

using namespace aiosb;

namespace aiosb {
namespace {
// CTAs per row of the group step (AIOSB_GROUP_SPLIT: 1, 2, 4 or 8), at most
// 128 CTAs in all (one wave).
int g_group_split = [] {
  const char* env = getenv("AIOSB_GROUP_SPLIT");
  const int v = env ? atoi(env) : kDefaultSplit;
  return v == 1 || v == 2 || v == 4 || v == 8 ? v : kDefaultSplit;
}();

int launch_group_step(const aiosb_group_ptrs& g, int64_t rows, int64_t vocab, bool large, cudaStream_t stream) {
  int C = g_group_split;
  while (C > 1 && rows * C > 128) C >>= 1;
  auto kern = C > 1 ? group_step_kernel<true> : group_step_kernel<false>;
  cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sample_smem_max());
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(rows * C));
  cfg.blockDim = dim3(kSampThreads);
  cfg.dynamicSmemBytes = large ? sample_smem_large((int)vocab) : sample_smem((int)vocab);
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  attr[1].id = cudaLaunchAttributeClusterDimension;
  attr[1].val.clusterDim.x = (unsigned)C;
  attr[1].val.clusterDim.y = 1;
  attr[1].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = C > 1 ? 2 : 1;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, kern, g, (int)large, C, (int)vocab);
  return e == cudaSuccess ? AIOSB_OK : set_error(AIOSB_ERR_LAUNCH, "group_step: %s", cudaGetErrorString(e));
}
}  // namespace
}  // namespace aiosb

extern "C" int aiosb_sample(const void* logits, int64_t rows, int64_t vocab, int64_t row_stride, float temperature,
                            int64_t top_k, float top_p, int greedy, const float* uniforms, const int32_t* forbidden,
                            int64_t n_forbidden, const int64_t* forbidden_rows, int64_t n_forbidden_rows,
                            int64_t* token_out, float* logprob_out, int32_t* status, void* stream) {
  AIOSB_REQUIRE(rows >= 0 && vocab > 0 && vocab <= kMaxVocab && row_stride >= vocab, AIOSB_ERR_INVALID_ARG,
                "sample: bad sizes (vocab must be in [1, %d])", kMaxVocab);
  AIOSB_REQUIRE(greedy || temperature > 0.f, AIOSB_ERR_INVALID_ARG, "sample: temperature must be positive");
  bool large = false;
  if (!greedy) {
    const int64_t k = top_k > 0 ? std::min<int64_t>(top_k, vocab) : (top_p < 1.0f ? vocab : 0);
    large = k > kMaxSortK;
    AIOSB_REQUIRE(!large || vocab <= kMaxLargeSort, AIOSB_ERR_UNSUPPORTED,
                  "sample: a sorted candidate set of %lld needs a vocabulary of at most %d", (long long)k,
                  kMaxLargeSort);
  }
  if (rows == 0) return AIOSB_OK;
  AIOSB_REQUIRE(logits && token_out && logprob_out, AIOSB_ERR_INVALID_ARG, "sample: null pointer");
  SampleParams p;
  p.temperature = temperature;
  p.top_k = (int)top_k;
  p.top_p = top_p;
  p.greedy = greedy;
  const size_t smem = large ? sample_smem_large((int)vocab) : sample_smem((int)vocab);
  cudaFuncSetAttribute(sample_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sample_smem_max());
  cudaError_t e = launch_pdl(sample_kernel, dim3((unsigned)rows), dim3(kSampThreads), smem, as_stream(stream),
                             (const __nv_bfloat16*)logits, row_stride, (int)vocab, p, uniforms, forbidden,
                             (int)n_forbidden, forbidden_rows, (int)n_forbidden_rows, token_out, logprob_out, status,
                             (int)large);
  if (e != cudaSuccess) return set_error(AIOSB_ERR_LAUNCH, "sample: %s", cudaGetErrorString(e));
  return AIOSB_OK;
}

extern "C" int aiosb_group_begin(const aiosb_group_ptrs* g, const void* prefix_logits, uint64_t seed_base,
                                 int64_t attempts, int64_t rows, void* stream) {
  AIOSB_REQUIRE(g && g->state && prefix_logits, AIOSB_ERR_INVALID_ARG, "group_begin: null pointer");
  AIOSB_REQUIRE(attempts >= 1 && attempts <= rows, AIOSB_ERR_INVALID_ARG, "group_begin: attempts outside [1, rows]");
  cudaError_t e = launch_pdl(group_begin_kernel, dim3(64), dim3(256), 0, as_stream(stream), *g,
                             (const __nv_bfloat16*)prefix_logits, seed_base, (int)attempts);
  if (e != cudaSuccess) return set_error(AIOSB_ERR_LAUNCH, "group_begin: %s", cudaGetErrorString(e));
  return AIOSB_OK;
}

namespace aiosb {
namespace {
// The optional next-forward embedding of aiosb_group_ptrs: all of it or none.
int check_group_embed(const aiosb_group_ptrs* g) {
  if (g->embed_w == nullptr) return AIOSB_OK;
  AIOSB_REQUIRE(g->embed_out && g->embed_stat_x && g->embed_stat_ss && g->hidden > 0 && g->hidden % 8 == 0,
                AIOSB_ERR_INVALID_ARG, "group_step: embed_w needs embed_out, embed_stat_x, embed_stat_ss and "
                "a hidden size that is a positive multiple of 8");
  AIOSB_REQUIRE(aligned16(g->embed_w) && aligned16(g->embed_out) && aligned16(g->embed_stat_x), AIOSB_ERR_MISALIGNED,
                "group_step: embed_w, embed_out and embed_stat_x must be 16-byte aligned");
  return AIOSB_OK;
}
}  // namespace
}  // namespace aiosb

extern "C" int aiosb_group_step(const aiosb_group_ptrs* g, int64_t rows, int64_t vocab, int64_t top_k_max,
                                void* stream) {
  AIOSB_REQUIRE(g && g->state, AIOSB_ERR_INVALID_ARG, "group_step: null pointer");
  if (const int rc = check_group_embed(g); rc != AIOSB_OK) return rc;
  AIOSB_REQUIRE(rows >= 1 && vocab > 0 && vocab <= kMaxVocab, AIOSB_ERR_INVALID_ARG,
                "group_step: rows >= 1 and vocab in [1, %d]", kMaxVocab);
  // top_k_max: the largest sorted candidate set the group's rounds may ask for
  // (top-k, or the vocabulary for top-p without top-k); above kMaxSortK the step
  // sorts whole rows, for vocabularies of at most kMaxLargeSort ids
  const bool large = top_k_max > kMaxSortK;
  AIOSB_REQUIRE(!large || vocab <= kMaxLargeSort, AIOSB_ERR_UNSUPPORTED,
                "group_step: sorted candidate sets above %d need a vocabulary of at most %d", kMaxSortK,
                kMaxLargeSort);
  AIOSB_REQUIRE(rows <= 32, AIOSB_ERR_UNSUPPORTED, "group_step: at most 32 rows per group");
  return launch_group_step(*g, rows, vocab, large, as_stream(stream));
}

extern "C" int aiosb_token_logprobs(const void* logits, int64_t rows, int64_t vocab, int64_t row_stride,
                                    const int64_t* targets, float* out, int32_t* status, void* stream) {
  AIOSB_REQUIRE(rows >= 0 && vocab > 0 && vocab <= kMaxVocab && (row_stride >= vocab || row_stride == 0),
                AIOSB_ERR_INVALID_ARG,
                "token_logprobs: bad sizes (vocab must be in [1, %d], row stride >= vocab or 0)", kMaxVocab);
  if (rows == 0) return AIOSB_OK;
  AIOSB_REQUIRE(logits && targets && out, AIOSB_ERR_INVALID_ARG, "token_logprobs: null pointer");
  cudaFuncSetAttribute(token_logprob_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                       (int)sample_smem(kMaxVocab));
  cudaError_t e = launch_pdl(token_logprob_kernel, dim3((unsigned)rows), dim3(kSampThreads),
                             sample_smem((int)vocab), as_stream(stream), (const __nv_bfloat16*)logits, row_stride,
                             (int)vocab, targets, out, status);
  if (e != cudaSuccess) return set_error(AIOSB_ERR_LAUNCH, "token_logprobs: %s", cudaGetErrorString(e));
  return AIOSB_OK;
}

extern "C" int aiosb_page_table_fill(int32_t* table, int64_t stride, int64_t rows, int64_t width,
                                     const int32_t* prefix, int64_t n, void* stream) {
  AIOSB_REQUIRE(rows >= 0 && width >= 0 && n >= 0 && n <= width && stride >= width, AIOSB_ERR_INVALID_ARG,
                "page_table_fill: bad sizes");
  if (rows == 0 || width == 0) return AIOSB_OK;
  AIOSB_REQUIRE(table && (n == 0 || prefix), AIOSB_ERR_INVALID_ARG, "page_table_fill: null pointer");
  const int64_t total = rows * width;
  cudaError_t e = launch_pdl(page_table_fill_kernel, dim3((unsigned)std::min<int64_t>((total + 255) / 256, 148)),
                             dim3(256), 0, as_stream(stream), table, stride, (int)rows, (int)width, prefix, (int)n);
  if (e != cudaSuccess) return set_error(AIOSB_ERR_LAUNCH, "page_table_fill: %s", cudaGetErrorString(e));
  return AIOSB_OK;
}

extern "C" int aiosb_stateless_uniforms(const int64_t* seeds, int64_t rows, int64_t steps, float* out, void* stream) {
  AIOSB_REQUIRE(rows >= 0 && steps >= 1, AIOSB_ERR_INVALID_ARG, "steps must be positive");
  if (rows == 0) return AIOSB_OK;
  AIOSB_REQUIRE(seeds && out, AIOSB_ERR_INVALID_ARG, "stateless_uniforms: null pointer");
  const int64_t n = rows * steps;
  uniforms_kernel<<<(unsigned)((n + 255) / 256), 256, 0, as_stream(stream)>>>(seeds, rows, steps, out);
  return check_launch("stateless_uniforms");
}

extern "C" int aiosb_slot_alloc(const int32_t* ring, int64_t capacity, int64_t head, int64_t n, int32_t* out,
                                void* stream) {
  AIOSB_REQUIRE(capacity > 0 && n >= 0 && n <= capacity && head >= 0, AIOSB_ERR_INVALID_ARG, "slot_alloc: bad sizes");
  if (n == 0) return AIOSB_OK;
  AIOSB_REQUIRE(ring && out, AIOSB_ERR_INVALID_ARG, "slot_alloc: null pointer");
  slot_alloc_kernel<<<(unsigned)std::min<int64_t>((n + 255) / 256, 1024), 256, 0, as_stream(stream)>>>(
      ring, capacity, head, n, out);
  return check_launch("slot_alloc");
}

extern "C" int aiosb_slot_free(int32_t* ring, int64_t capacity, int64_t tail, const int32_t* slots, int64_t n,
                               void* stream) {
  AIOSB_REQUIRE(capacity > 0 && n >= 0 && n <= capacity && tail >= 0, AIOSB_ERR_INVALID_ARG, "slot_free: bad sizes");
  if (n == 0) return AIOSB_OK;
  AIOSB_REQUIRE(ring && slots, AIOSB_ERR_INVALID_ARG, "slot_free: null pointer");
  slot_free_kernel<<<(unsigned)std::min<int64_t>((n + 255) / 256, 1024), 256, 0, as_stream(stream)>>>(
      ring, capacity, tail, slots, n);
  return check_launch("slot_free");
}

extern "C" int aiosb_slot_free_range(int32_t* ring, int64_t capacity, int64_t begin, int64_t n, int64_t tail,
                                     void* stream) {
  AIOSB_REQUIRE(capacity > 0 && n >= 0 && n <= capacity && begin >= 0 && tail >= 0, AIOSB_ERR_INVALID_ARG,
                "slot_free_range: bad sizes");
  if (n == 0) return AIOSB_OK;
  AIOSB_REQUIRE(ring, AIOSB_ERR_INVALID_ARG, "slot_free_range: null pointer");
  slot_free_range_kernel<<<1, 1024, 0, as_stream(stream)>>>(ring, capacity, begin, n, tail);
  return check_launch("slot_free_range");
}

// ---- CandidateGroup step for callers that cannot allocate device memory -----
// aiosb_group_step hands each row's finish flag from the row's sampling CTA to
// the epilogue CTA through g->finished, a [rows] int32 array the caller
// allocates. This variant keeps those flags in a fixed array of the library
// instead. The array is part of the library image: every GPU that loads the
// library holds it until the process exits, and all calls share it.
constexpr int kStaticStepRows = 32;  // rows one call may step (the group limit)
static __device__ __align__(256) int32_t g_static_step_finished[kStaticStepRows];

namespace {
// The array's device address differs per CUDA context (one per device, and a new
// one after cudaDeviceReset), so the cache is keyed by the context's process-wide
// unique id (cuCtxGetId), fetched through the runtime's driver entry points so that
// the library needs no link to libcuda.
constexpr int kStaticMaxContexts = 64;
struct StaticScratchEntry {
  unsigned long long ctx_id;
  void* addr;
};
std::mutex g_static_step_mu;
StaticScratchEntry g_static_step_cache[kStaticMaxContexts];
int g_static_step_used = 0;

using CtxGetCurrentFn = int (*)(void**);
using CtxGetIdFn = int (*)(void*, unsigned long long*);

// Id of the calling thread's current context, or 0 when none is current yet.
unsigned long long current_context_id() {
  static CtxGetCurrentFn get_current = [] {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuCtxGetCurrent", &fn, 12000, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      fn = nullptr;
    return reinterpret_cast<CtxGetCurrentFn>(fn);
  }();
  static CtxGetIdFn get_id = [] {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuCtxGetId", &fn, 12000, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      fn = nullptr;
    return reinterpret_cast<CtxGetIdFn>(fn);
  }();
  void* ctx = nullptr;
  unsigned long long id = 0;
  if (get_current == nullptr || get_id == nullptr || get_current(&ctx) != 0 || ctx == nullptr) return 0;
  return get_id(ctx, &id) == 0 ? id : 0;
}

// Device address of g_static_step_finished in the current context. The host-side
// name of a __device__ array is only a stand-in, so the address is looked up with
// cudaGetSymbolAddress (with the caller's device current) the first time a context
// calls, and cached under the context's id.
int static_step_scratch(int32_t** out) {
  const unsigned long long id = current_context_id();
  std::lock_guard<std::mutex> lock(g_static_step_mu);
  for (int i = 0; id != 0 && i < g_static_step_used; ++i) {
    if (g_static_step_cache[i].ctx_id == id) {
      *out = static_cast<int32_t*>(g_static_step_cache[i].addr);
      return AIOSB_OK;
    }
  }
  void* p = nullptr;
  const cudaError_t e = cudaGetSymbolAddress(&p, g_static_step_finished);  // creates the context if needed
  if (e != cudaSuccess || p == nullptr)
    return set_error(AIOSB_ERR_LAUNCH, "group_step_static: cudaGetSymbolAddress: %s", cudaGetErrorString(e));
  const unsigned long long now = current_context_id();
  if (now != 0) {  // without a context id the address is looked up on every call
    StaticScratchEntry& slot = g_static_step_cache[g_static_step_used < kStaticMaxContexts
                                                       ? g_static_step_used++
                                                       : (int)(now % kStaticMaxContexts)];
    slot.ctx_id = now;
    slot.addr = p;
  }
  *out = static_cast<int32_t*>(p);
  return AIOSB_OK;
}
}  // namespace

extern "C" int aiosb_group_step_static(const aiosb_group_ptrs* g, int64_t rows, int64_t vocab, int64_t top_k_max,
                                       void* stream) {
  AIOSB_REQUIRE(g && g->state, AIOSB_ERR_INVALID_ARG, "group_step_static: null pointer");
  if (const int rc = check_group_embed(g); rc != AIOSB_OK) return rc;
  AIOSB_REQUIRE(rows >= 1 && vocab > 0 && vocab <= kMaxVocab, AIOSB_ERR_INVALID_ARG,
                "group_step_static: rows >= 1 and vocab in [1, %d]", kMaxVocab);
  const bool large = top_k_max > kMaxSortK;
  AIOSB_REQUIRE(!large || vocab <= kMaxLargeSort, AIOSB_ERR_UNSUPPORTED,
                "group_step_static: sorted candidate sets above %d need a vocabulary of at most %d", kMaxSortK,
                kMaxLargeSort);
  AIOSB_REQUIRE(rows <= kStaticStepRows, AIOSB_ERR_UNSUPPORTED,
                "group_step_static: %lld rows exceed the %d-row static scratch", (long long)rows, kStaticStepRows);
  int32_t* finished = nullptr;
  const int rc = static_step_scratch(&finished);
  if (rc != AIOSB_OK) return rc;
  // The array keeps the previous call's flags; start every call from zeros, as
  // aiosb_group_begin leaves a caller's g->finished.
  cudaError_t e = cudaMemsetAsync(finished, 0, kStaticStepRows * sizeof(int32_t), as_stream(stream));
  if (e != cudaSuccess) return set_error(AIOSB_ERR_LAUNCH, "group_step_static: memset: %s", cudaGetErrorString(e));
  aiosb_group_ptrs local = *g;
  local.finished = finished;
  return launch_group_step(local, rows, vocab, large, as_stream(stream));
}
