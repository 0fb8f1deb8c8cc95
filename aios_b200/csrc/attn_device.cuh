// Attention building blocks shared by the decode / prefill kernels (attention.cu)
// and the persistent decode-step kernel (decode_step.cu): the online-softmax
// state of one query vector (lane-distributed over head dims), key staging from
// the paged cache, the fold of a 64-key chunk, and the q/k RMSNorm + bf16 RoPE
// prologue.
#pragma once

#include "common.cuh"

namespace aiosb {

constexpr int kKeyChunk = 64;  // keys staged per shared-memory chunk

// Online-softmax state of one query vector, lane-distributed over head dims.
template <int D>
struct QState {
  float m, l;
  float acc[D / 32];
};

template <int D>
__device__ __forceinline__ void qstate_init(QState<D>& s) {
  s.m = -INFINITY;
  s.l = 0.f;
#pragma unroll
  for (int i = 0; i < D / 32; ++i) s.acc[i] = 0.f;
}

// Folds one block of up to 64 keys into `st`. s0/s1 are this lane's scores for
// keys lane and lane+32 (-inf when masked); v_at(j, i) returns V[j][i*32+lane].
template <int D, typename VFn>
__device__ __forceinline__ void fold_scores(QState<D>& st, float s0, float s1, int nk, VFn v_at) {
  const float cmax = warp_max(fmaxf(s0, s1));
  if (cmax == -INFINITY) return;
  const float m_new = fmaxf(st.m, cmax);
  const float corr = expf(st.m - m_new);
  const float p0 = expf(s0 - m_new), p1 = expf(s1 - m_new);
  st.l = st.l * corr + warp_sum(p0 + p1);
#pragma unroll
  for (int i = 0; i < D / 32; ++i) st.acc[i] *= corr;
  for (int j = 0; j < nk; ++j) {
    const float p = __shfl_sync(0xffffffffu, j < 32 ? p0 : p1, j & 31);
#pragma unroll
    for (int i = 0; i < D / 32; ++i) st.acc[i] += p * v_at(j, i);
  }
  st.m = m_new;
}

// q (fp32, shared, broadcast) . K row (bf16 pairs).
template <int D>
__device__ __forceinline__ float dot_q_k(const float* q, const __nv_bfloat162* k) {
  float s = 0.f;
#pragma unroll
  for (int w = 0; w < D / 2; ++w) {
    const float2 kv = __bfloat1622float2(k[w]);
    s += q[2 * w] * kv.x + q[2 * w + 1] * kv.y;
  }
  return s;
}

// Stage keys [k0, k0+nk) of one slot list for KV head h into shared memory.
// Ks rows are padded to D+2 elements (odd word stride: conflict-free per-lane
// row reads); Vs rows are dense.
template <int D>
__device__ __forceinline__ void stage_chunk(const __nv_bfloat16* __restrict__ k_cache,
                                            const __nv_bfloat16* __restrict__ v_cache, int64_t tok_stride, int h,
                                            const int32_t* __restrict__ slots, int k0, int nk, int64_t num_slots,
                                            __nv_bfloat16* Ks, __nv_bfloat16* Vs, int32_t* status) {
  constexpr int kWords = D / 2;  // 32-bit words per row
  for (int idx = threadIdx.x; idx < nk * kWords; idx += blockDim.x) {
    const int j = idx / kWords, w = idx % kWords;
    int64_t slot = slots[k0 + j];
    if (slot < 0 || slot >= num_slots) {
      if (w == 0) report(status, AIOSB_DEV_SLOT_RANGE);
      slot = 0;
    }
    const uint32_t* kr = reinterpret_cast<const uint32_t*>(k_cache + slot * tok_stride + (int64_t)h * D);
    const uint32_t* vr = reinterpret_cast<const uint32_t*>(v_cache + slot * tok_stride + (int64_t)h * D);
    reinterpret_cast<uint32_t*>(Ks)[j * (kWords + 1) + w] = kr[w];
    reinterpret_cast<uint32_t*>(Vs)[j * kWords + w] = vr[w];
  }
}

// RMSNorm of one head vector (lane-distributed: element i*32+lane), rounded to
// bf16, then bf16 RoPE exactly as aios/layers/attention.py:6-16 computes it:
// out = bf16(bf16(x*cos) + bf16(rotate_half(x)*sin)).
template <int D>
__device__ __forceinline__ void norm_rope(float (&x)[D / 32], const __nv_bfloat16* __restrict__ w, float eps,
                                          const __nv_bfloat16* cos_row, const __nv_bfloat16* sin_row,
                                          bool do_norm, bool do_rope, int lane, float* tmp /*shared D floats*/) {
  constexpr int DPL = D / 32;
  if (do_norm) {
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < DPL; ++i) ss += x[i] * x[i];
    ss = warp_sum(ss);
    const float rcp = 1.0f / sqrtf(ss / (float)D + eps);
#pragma unroll
    for (int i = 0; i < DPL; ++i) x[i] = round_bf16(x[i] * rcp * bf16_to_f(w[i * 32 + lane]));
  }
  if (do_rope) {
    // rotate_half needs element (e + D/2) mod D: exchange through shared memory.
#pragma unroll
    for (int i = 0; i < DPL; ++i) tmp[i * 32 + lane] = x[i];
    __syncwarp();
    float r[DPL];
#pragma unroll
    for (int i = 0; i < DPL; ++i) {
      const int e = i * 32 + lane;
      r[i] = e < D / 2 ? -tmp[e + D / 2] : tmp[e - D / 2];
    }
    __syncwarp();
#pragma unroll
    for (int i = 0; i < DPL; ++i) {
      const int e = i * 32 + lane;
      const float a = round_bf16(x[i] * bf16_to_f(cos_row[e]));
      const float b = round_bf16(r[i] * bf16_to_f(sin_row[e]));
      x[i] = round_bf16(a + b);
    }
  }
}

template <int D>
__device__ __forceinline__ void fold_chunk(QState<D>& st, const float* qv, const __nv_bfloat16* Ks,
                                           const __nv_bfloat16* Vs, int nk, float scale, int lane) {
  const __nv_bfloat162* K2 = reinterpret_cast<const __nv_bfloat162*>(Ks);
  const float s0 = lane < nk ? dot_q_k<D>(qv, K2 + lane * (D / 2 + 1)) * scale : -INFINITY;
  const float s1 = lane + 32 < nk ? dot_q_k<D>(qv, K2 + (lane + 32) * (D / 2 + 1)) * scale : -INFINITY;
  fold_scores<D>(st, s0, s1, nk, [&](int j, int i) { return bf16_to_f(Vs[j * D + i * 32 + lane]); });
}

}  // namespace aiosb
