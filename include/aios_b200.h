/*
 * aios_b200 — C ABI of the B200-native (sm_100a) CandidateGroup hot path.
 *
 * Every entry point takes plain device pointers, element counts and strides,
 * plus the caller's CUDA stream as `void*` (a cudaStream_t; NULL is the legacy
 * default stream). No torch type crosses this boundary.
 *
 * Ownership: all buffers are owned by the caller. The library never allocates or
 *   frees device memory; it launches kernels on the given stream and returns.
 * Errors: every call returns 0 (AIOSB_OK) or a negative AIOSB_ERR_* code before
 *   launching anything; aiosb_last_error() gives the message of the calling
 *   thread's last failure. Kernels never trap: faults that can only be seen on
 *   the device (a slot index outside the pool, an exhausted free list, a bounded
 *   wait that ran out) are written as an AIOSB_DEV_* code into the caller's int32
 *   status word (first error wins) and the kernel returns.
 * Threading: calls may come from any host thread as long as the caller orders
 *   them on its stream. The library holds no state of its own except the
 *   per-thread error message and, for aiosb_group_step_static only, a 32-entry
 *   device array in the library image plus a host cache of its address per CUDA
 *   context (guarded by a mutex). Calls of aiosb_group_step_static that overlap
 *   on the GPU share that array and race on it.
 *
 * Each entry point names the reference interface it replaces
 * (paths inside the 7155/aios repository).
 */
#ifndef AIOS_B200_H_
#define AIOS_B200_H_

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define AIOSB_API __attribute__((visibility("default")))
#else
#define AIOSB_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* ---- return codes ------------------------------------------------------- */
#define AIOSB_OK 0
#define AIOSB_ERR_INVALID_ARG -1 /* shape, size or pointer argument rejected      */
#define AIOSB_ERR_UNSUPPORTED -2 /* dims this build has no kernel for             */
#define AIOSB_ERR_MISALIGNED -3  /* pointer or stride breaks a 16-byte rule        */
#define AIOSB_ERR_LAUNCH -4      /* cudaLaunch* or driver call failed              */

/* ---- device status codes (written into the caller's status word) -------- */
#define AIOSB_DEV_WAIT_TIMEOUT 1  /* a bounded mbarrier / flag wait ran out        */
#define AIOSB_DEV_SLOT_RANGE 2    /* KV slot index outside [0, num_slots)          */
#define AIOSB_DEV_TOKEN_RANGE 3   /* token id outside [0, vocab)                    */
#define AIOSB_DEV_POOL_EMPTY 4    /* free-slot FIFO had fewer entries than asked    */
#define AIOSB_DEV_POSITION_RANGE 5 /* RoPE position outside the cos/sin table      */

/* GEMM epilogues for aiosb_linear. */
#define AIOSB_EPI_STORE 0    /* y = x W^T, bf16                                         */
#define AIOSB_EPI_SILU_MUL 1 /* W rows interleaved in 64-row gate/up blocks;
                                y[:, f] = silu(x Wg^T) * (x Wu^T), bf16              */
#define AIOSB_EPI_ADD 2      /* y = residual + bf16(x W^T), bf16 (residual may be y)  */
/* OR-ed into the epilogue of aiosb_linear / aiosb_linear_stat_norm: on the
 * register-operand path the next kernel on the stream may launch before this
 * one's dependency wait, as after an AIOSB_EPI_ADD linear. Only for a successor
 * whose reads before its own wait do not depend on this kernel's predecessor: a
 * linear (it reads only its weights there), or a decode attention whose history
 * and row metadata come from kernels that have completed whenever it can start. */
#define AIOSB_LINEAR_EARLY_DEPENDENTS 0x100

/* Library version (major*10000 + minor*100 + patch). */
AIOSB_API int aiosb_version(void);

/* Copies the calling thread's last error message (NUL-terminated, truncated to
 * len) and returns its AIOSB_ERR_* code (0 if none). */
AIOSB_API int aiosb_last_error(char* buf, size_t len);

/* Device address of page-locked host memory (for host-mapped flags the device
 * polls or writes, e.g. the CandidateGroup cancel flag and progress mirror). */
AIOSB_API int aiosb_host_device_pointer(void* host, void** device);

/* ---- KV cache scatter ----------------------------------------------------
 * Replaces aios/kernel/store.py:32-61 (store_cache) as called by
 * aios/kvcache/mha_pool.py:45-56 (MHAKVCache.store_kv).
 * k_cache[indices[t], :] = k[t, :]; v_cache[indices[t], :] = v[t, :] for
 * t < num_tokens, over `width` = num_kv_heads * head_dim bf16 elements.
 * Strides are in elements. Indices outside [0, num_slots) are skipped and
 * reported as AIOSB_DEV_SLOT_RANGE. */
AIOSB_API int aiosb_kv_store(void* k_cache, void* v_cache, int64_t cache_token_stride, int64_t num_slots,
                   const int32_t* indices, int64_t num_tokens, const void* k, int64_t k_token_stride,
                   const void* v, int64_t v_token_stride, int64_t width, int32_t* status, void* stream);

/* ---- Block AttnRes depth mixer -------------------------------------------
 * Replaces aios/kernel/attnres.py:130-223 (triton_attnres_mix: the two Triton
 * kernels _attnres_score_kernel 8-57 and _attnres_value_kernel 60-127) in one
 * kernel. bank: [sources, tokens, hidden] bf16 contiguous; partial: [tokens,
 * hidden] bf16 or NULL; weighted_query: [hidden] fp32; out: [tokens, hidden] bf16.
 * score = (x . wq) * rsqrt(mean(x^2) + eps) in fp32, softmax over depth in
 * fp32, weights rounded to bf16, out = sum_s w_s x_s accumulated in fp32.
 * hidden must be a multiple of 8; sources + (partial != NULL) <= 16.
 * status: the caller's int32 status word, or NULL. From 2048 tokens the mixer
 * streams its sources through bounded shared-memory waits; a wait that runs out
 * writes AIOSB_DEV_WAIT_TIMEOUT there (and NaN into the rows it did not mix). */
AIOSB_API int aiosb_attnres_mix(const void* bank, int64_t sources, int64_t tokens, int64_t hidden, const void* partial,
                      const float* weighted_query, float eps, void* out, int32_t* status, void* stream);

/* The mixer followed by the RMSNorm that consumes its output in the Block AttnRes
 * layers (aios/models/minimind_ime.py, the input / post-attention norms after
 * each mixer; aios/layers/norm.py:10-22): out = bf16(h * rcp * norm_w), h the
 * bf16 mixer output of aiosb_attnres_mix, rcp = 1 / sqrt(mean(h^2) + norm_eps).
 * The mixer result itself is not written. sources + (partial != NULL) <= 10,
 * hidden <= 768 (a multiple of 8); norm_w: [hidden] bf16. stable_sources (in
 * [0, sources]): the first bank sources that were written before the previous
 * kernel on the stream began; the kernel reads them before waiting on that
 * kernel (0: every read after the wait). */
AIOSB_API int aiosb_attnres_mix_rmsnorm(const void* bank, int64_t sources, int64_t tokens, int64_t hidden,
                                        const void* partial, const float* weighted_query, float eps,
                                        const void* norm_w, float norm_eps, int64_t stable_sources, void* out,
                                        void* stream);

/* Test hook, not for production callers: the next launches of the mixer's
 * stream kernel (aiosb_attnres_mix from 2048 tokens) have CTA 0 announce its
 * tile `stall_tile` without copying it, and bound every wait by wait_limit_ns
 * (0: the default 2 s), so that a bounded mbarrier wait runs out and the kernel
 * reports AIOSB_DEV_WAIT_TIMEOUT. stall_tile < 0 restores normal operation. */
AIOSB_API int aiosb_test_attnres_stream_stall(int64_t stall_tile, uint64_t wait_limit_ns);

/* ---- RMSNorm ---------------------------------------------------------------
 * Replaces aios/layers/norm.py:10-22 (RMSNorm.forward / forward_inplace, the
 * FlashInfer rmsnorm). Normalises rows of `hidden` elements:
 * out = x * rsqrt(mean(x^2) + eps) * weight, fp32 math, bf16 in/out.
 * Row r lives at x + (r / heads_per_token) * token_stride + (r % heads_per_token)
 * * hidden (the same for out with out_token_stride), so per-head q/k norms of a
 * packed qkv row are one call. out may equal x. */
AIOSB_API int aiosb_rmsnorm(const void* x, int64_t rows, int64_t hidden, int64_t heads_per_token, int64_t token_stride,
                  const void* weight, float eps, void* out, int64_t out_token_stride, void* stream);

/* Replaces aios/layers/norm.py:25-39 (RMSNormFused with a residual, the
 * FlashInfer fused_add_rmsnorm): residual = x + residual (bf16 store), then
 * x = rmsnorm(fp32 sum) * weight, in place on [rows, hidden] contiguous rows. */
AIOSB_API int aiosb_add_rmsnorm(void* x, void* residual, int64_t rows, int64_t hidden, const void* weight, float eps,
                      void* stream);

/* ---- SwiGLU ----------------------------------------------------------------
 * Replaces aios/layers/activation.py:9-12 (silu_and_mul): out[r, f] =
 * silu(x[r, f]) * x[r, F + f], fp32 math, bf16 in/out; x is [rows, 2F]. */
AIOSB_API int aiosb_silu_mul(const void* x, int64_t rows, int64_t f, void* out, void* stream);

/* ---- Embedding gather ------------------------------------------------------
 * Replaces aios/layers/embedding.py:17-18 (Embedding.forward). ids are int64
 * (ids_is_int64 != 0) or int32; out[t] = weight[ids[t]]. Out-of-range ids write
 * zeros and report AIOSB_DEV_TOKEN_RANGE. */
AIOSB_API int aiosb_embedding(const void* ids, int ids_is_int64, int64_t num_tokens, const void* weight, int64_t vocab,
                    int64_t hidden, void* out, int32_t* status, void* stream);

/* Embedding gather that also emits the RMSNorm statistics of its rows, for a
 * first layer whose input norm is a plain RMSNorm of the embeddings
 * (aios/models/qwen3.py:113 with residual None, aios/layers/norm.py:34-38):
 * stat_x [num_tokens, hidden] fp32 = the rows, stat_ss[t] = sum of squares of
 * row t (one part). aiosb_linear_stat_norm consumes them. */
AIOSB_API int aiosb_embedding_stat(const void* ids, int ids_is_int64, int64_t num_tokens, const void* weight,
                                   int64_t vocab, int64_t hidden, void* out, float* stat_x, float* stat_ss,
                                   int32_t* status, void* stream);

/* ---- Linear (tcgen05 tensor-core GEMM) -------------------------------------
 * Replaces the cuBLAS GEMMs behind aios/layers/linear.py:16-17 (Linear.forward)
 * and aios/layers/embedding.py:34-41 (LMHead.forward): y = x W^T.
 * x: [rows, k] bf16 row-major, row stride k; w: [n, k] bf16 row-major;
 * y: [rows, y_cols] bf16 with row stride y_row_stride, where y_cols = n
 * (AIOSB_EPI_STORE, AIOSB_EPI_ADD) or n/2 (AIOSB_EPI_SILU_MUL, w rows packed
 * as [gate 0..63 | up 0..63 | gate 64..127 | up 64..127 | ...]). For
 * AIOSB_EPI_ADD, residual is [rows, >= n] with row stride residual_stride and may
 * alias y (each element is read before it is written by the same thread).
 * Requires n % 128 == 0, k % 64 == 0, 16-byte aligned x/w/y. Up to 512 rows
 * (k % 256 == 0, k <= 2048; AIOSB_GEMV_MAX_ROWS changes the bound) run on a
 * register-operand MMA kernel that requests its weights before waiting on the
 * previous kernel (more than 16 rows as 16-row groups that share each weight tile
 * through L2); larger calls on tcgen05. Such an AIOSB_EPI_ADD call lets the next
 * kernel on the stream launch at once; the other epilogues let it launch only
 * after their own wait. */
AIOSB_API int aiosb_linear(const void* x, int64_t rows, int64_t k, const void* w, int64_t n, void* y,
                           int64_t y_row_stride, int epilogue, const void* residual, int64_t residual_stride,
                           int32_t* status, void* stream);

/* Linear with a fused RMSNorm on its input, for rows <= 64: y = (rmsnorm(x + res)
 * * norm_w) W^T, with the epilogues of aiosb_linear. Replaces the pair
 * RMSNormFused.forward (aios/layers/norm.py:25-39; res == NULL: plain RMSNorm,
 * aios/layers/norm.py:10-22) + Linear.forward: the normalised rows are built by
 * the GEMM's own CTAs straight into the tensor-core operand layout, and
 * res_out (when not NULL) receives the new residual bf16(x + res); res_out must
 * not alias x or res. x, res, res_out: [rows, k] contiguous bf16. */
AIOSB_API int aiosb_linear_rmsnorm(const void* x, const void* res, void* res_out, const void* norm_w, float eps,
                                   int64_t rows, int64_t k, const void* w, int64_t n, void* y, int64_t y_row_stride,
                                   int epilogue, const void* residual, int64_t residual_stride, int32_t* status,
                                   void* stream);

/* Residual GEMM that also emits RMSNorm statistics (producer half of a
 * residual add + RMSNorm split across two GEMMs). Replaces Linear.forward
 * followed by the add of RMSNormFused.forward (aios/layers/linear.py:21-22,
 * aios/layers/norm.py:34-40, as used at aios/models/qwen3.py:106-120):
 * y = bf16(s), s = residual + bf16(x W^T) in fp32 (residual may alias y),
 * stat_x [rows, n] fp32 = s, and the sums of squares of s over column groups:
 * stat_ss[p * stat_ss_stride + row] for parts p < *stat_parts. A part is 8
 * columns when the call runs on the register-operand MMA kernel (see
 * aiosb_linear), else 128; stat_ss must hold n / 8 parts. *stat_parts is written
 * before any check. n <= 2048. */
AIOSB_API int aiosb_linear_add_stat(const void* x, int64_t rows, int64_t k, const void* w, int64_t n, void* y,
                                    int64_t y_row_stride, const void* residual, int64_t residual_stride,
                                    float* stat_x, float* stat_ss, int64_t stat_ss_stride, int64_t* stat_parts,
                                    int32_t* status, void* stream);

/* GEMM on RMSNorm-ed rows given their statistics (consumer half): the
 * normalisation of RMSNormFused.forward (aios/layers/norm.py:34-40) followed by
 * Linear.forward / the SwiGLU or residual epilogues of aiosb_linear:
 * y = epilogue(bf16(s * rcp * norm_w) W^T), rcp = 1 / sqrt(sum_p stat_ss[p *
 * stat_ss_stride + row] / k + eps) with the parts summed in order, s = stat_x
 * [rows, k] fp32. The normalised rows are built by the GEMM's CTAs straight
 * into the tensor-core operand layout; no normalised tensor is written. */
AIOSB_API int aiosb_linear_stat_norm(const float* stat_x, const float* stat_ss, int64_t stat_ss_stride,
                                     int64_t parts, const void* norm_w, float eps, int64_t rows, int64_t k,
                                     const void* w, int64_t n, void* y, int64_t y_row_stride, int epilogue,
                                     const void* residual, int64_t residual_stride, int32_t* status,
                                     void* stream);

/* aiosb_linear_stat_norm with the store epilogue, that also writes, for every
 * 16-column tile t of the output and row r, tile_stats[(t * rows + r) * 4 + i] =
 * (max, sum of exp(v - max), min, 1 if any NaN else 0) of the tile's stored bf16
 * values (the LM head: what the CandidateGroup step needs to bound a row's top-k
 * and its log-sum-exp without scanning the row). Only on the register-operand
 * path with rows <= 16 and k <= 768 (else AIOSB_ERR_UNSUPPORTED); tile_stats:
 * [n / 16, rows, 4] fp32, 16-byte aligned. It lets the next kernel on the
 * stream launch at once, and leaves `rows` SMs free for it (the CandidateGroup
 * step, one CTA per row, with AIOSB_GROUP_AFTER_FORWARD). */
/* aiosb_linear with the store epilogue that also writes the tile statistics of
 * aiosb_linear_stat_norm_tiles (the LM head on already normalised rows). */
AIOSB_API int aiosb_linear_tiles(const void* x, int64_t rows, int64_t k, const void* w, int64_t n, void* y,
                                 int64_t y_row_stride, float* tile_stats, int32_t* status, void* stream);
/* 1 when aiosb_linear_tiles / aiosb_linear_stat_norm_tiles serve this shape, else 0. */
AIOSB_API int aiosb_linear_tile_stats_eligible(int64_t rows, int64_t k, int64_t n);
AIOSB_API int aiosb_linear_stat_norm_tiles(const float* stat_x, const float* stat_ss, int64_t stat_ss_stride,
                                           int64_t parts, const void* norm_w, float eps, int64_t rows, int64_t k,
                                           const void* w, int64_t n, void* y, int64_t y_row_stride,
                                           float* tile_stats, int32_t* status, void* stream);

/* Decode linear on the Block AttnRes mixer's normalised rows (replaces
 * BlockAttnResMixer.forward + RMSNorm.forward + Linear.forward,
 * aios/models/minimind_ime.py:162-190,237-252, aios/kernel/attnres.py:8-127):
 * y = epilogue(bf16(h * rcp * norm_w) W^T) with h = bf16(sum_s alpha_s x_s), the
 * sources x_s being bank [sources, tokens, k] and then partial [tokens, k] (when
 * not NULL), alpha = bf16(softmax_s(dot(x_s, weighted_query) / rms(x_s, mix_eps))),
 * rcp = 1 / sqrt(mean(h^2) + norm_eps). The mixer's rows exist only inside the
 * linear's CTAs: every CTA stages the first stable_sources bank sources (written
 * before the previous kernel on the stream began) before waiting on that kernel,
 * and reads the others after it. Decode widths only: 1..8 tokens, k == 768,
 * sources + (partial != NULL) <= 10, at most two of them read after the wait;
 * epilogue AIOSB_EPI_STORE or AIOSB_EPI_SILU_MUL (packed gate/up weights). */
AIOSB_API int aiosb_linear_attnres_rmsnorm(const void* bank, int64_t sources, int64_t stable_sources,
                                           int64_t tokens, const void* partial, const float* weighted_query,
                                           float mix_eps, const void* norm_w, float norm_eps, const void* w,
                                           int64_t n, int64_t k, void* y, int64_t y_row_stride, int epilogue,
                                           int32_t* status, void* stream);

/* ---- Attention ---------------------------------------------------------------
 * KV slots: token slot s of one layer lives at k_cache + s * num_kv_heads *
 * head_dim (the MHAKVCache layout [pages, page_size, Hkv, d] flattened); slot
 * lists come from the page table [rows, table_stride] int32. head_dim in
 * {64, 96, 128}.
 *
 * Decode replaces aios/attention/flashinfer.py:374-394 (FlashInferAttentionBackend
 * ._decode + plan) and, when qkv != NULL, also the q/k RMSNorm + bf16 RoPE of
 * aios/models/qwen3.py:60-70 and the KV store of the new token
 * (aios/kernel/store.py:32-61). Cascade: keys [0, *prefix_len) are read from
 * page_table row row_table[0] once per KV head for every row (the candidate rows
 * of a group share their prefix slots); keys [*prefix_len, seq_lens[r]) come from
 * row row_table[r]. Pass either qkv (raw projection [rows, qkv_stride]: q | k | v
 * heads) or q (already normalised and rotated [rows, q_stride]). Rows with
 * active[r] == 0 are skipped (output zeros, no store); active may be NULL.
 * rows * (num_qo_heads / num_kv_heads) <= 64. out: [rows, out_stride] bf16. *
 * stable_history != 0 (fused mode only) asserts that row_table, *prefix_len,
 * positions, seq_lens, out_loc, active, the page-table entries before each row's
 * current position and the K/V they point to were written by kernels that have
 * completed whenever this one can start: launches at least two kernels back when
 * the previous kernel launches this one only after its own wait, further back
 * when it launches it early (the CandidateGroup runtime: prefix from the
 * prefill, older suffix keys from earlier steps, row metadata from this step's
 * group step; the qkv linear just before launches it after its wait in the first
 * layer and early in the others, whose predecessors by then include a completed
 * attention of the previous layer). The kernel then copies the keys each row uses into shared memory
 * before waiting on the previous kernel, and after the wait only this step's
 * projection row stays on its critical path. stable_history selects how:
 * AIOSB_HISTORY_STAGED (1), every row's CTA reads the prefix itself;
 * AIOSB_HISTORY_PREFIX_ONCE (2), the rows of a KV head (up to 8 per cluster)
 * split the prefix, each reads its slice once and copies it to the others over
 * distributed shared memory. Both give identical results; k_cache and v_cache
 * must be 16-byte aligned. staged_prefix bounds the prefix keys staged before
 * the wait (rounded up to 64; 0 = 128; at most 512 / 384 / 256 keys for head_dim
 * 64 / 96 / 128): shared memory is sized by it, and longer prefixes are read
 * after the wait. */
#define AIOSB_HISTORY_STAGED 1
#define AIOSB_HISTORY_PREFIX_ONCE 2
AIOSB_API int aiosb_attention_decode(const void* qkv, int64_t qkv_stride, const void* q, int64_t q_stride,
                           const void* q_norm_w, const void* k_norm_w, float eps, const void* cos_tab,
                           const void* sin_tab, int64_t max_pos, const int32_t* positions, const int32_t* out_loc,
                           void* k_cache, void* v_cache, int64_t num_slots, const int32_t* page_table,
                           int64_t table_stride, const int32_t* row_table, const int32_t* seq_lens,
                           const int32_t* prefix_len, const int32_t* active, int stable_history,
                           int64_t staged_prefix, int64_t rows, int64_t num_qo_heads, int64_t num_kv_heads,
                           int64_t head_dim, float scale, void* out, int64_t out_stride, int32_t* status,
                           void* stream);

/* Prefill prologue: replaces the q/k RMSNorm (aios/models/qwen3.py:66-67),
 * apply_rotary_pos_emb (aios/layers/attention.py:11-16) and store_kv
 * (aios/attention/flashinfer.py:312) of a prefill batch. q heads are written,
 * normalised and rotated, to q_out; k (normalised, rotated) and v go to the
 * cache slots out_loc[t]. cos_tab/sin_tab: [max_pos, head_dim] bf16. */
AIOSB_API int aiosb_qk_norm_rope_store(const void* qkv, int64_t qkv_stride, int64_t tokens, int64_t num_qo_heads,
                             int64_t num_kv_heads, int64_t head_dim, const void* q_norm_w, const void* k_norm_w,
                             float eps, const void* cos_tab, const void* sin_tab, int64_t max_pos,
                             const int32_t* positions, const int32_t* out_loc, void* k_cache, void* v_cache,
                             int64_t num_slots, void* q_out, int64_t q_out_stride, int32_t* status, void* stream);

/* Tokens per prefill query tile for this head grouping (0 if unsupported). */
AIOSB_API int aiosb_prefill_tile_tokens(int64_t num_qo_heads, int64_t num_kv_heads);

/* Prefill attention: replaces the paged prefill of aios/attention/flashinfer.py:
 * 300-326 and _sdpa_prefill_attention (33-91): causal attention of each
 * request's new tokens over its slot list, query i at absolute position
 * cached_len + i. Requests: q rows [q_start, q_start + q_len) of q, keys from
 * page_table row table_row. The grid is a list of tiles (request, first query
 * token) of tile_tokens tokens each. */
AIOSB_API int aiosb_attention_prefill(const void* q, int64_t q_stride, const void* k_cache, const void* v_cache,
                            int64_t num_slots, const int32_t* page_table, int64_t table_stride,
                            const int32_t* req_q_start, const int32_t* req_q_len, const int32_t* req_cached_len,
                            const int32_t* req_table_row, const int32_t* tile_req, const int32_t* tile_q0,
                            int64_t num_tiles, int64_t tile_tokens, int64_t num_qo_heads, int64_t num_kv_heads,
                            int64_t head_dim, float scale, void* out, int64_t out_stride, int32_t* status,
                            void* stream);

/* Fused prefill: aiosb_qk_norm_rope_store followed by aiosb_attention_prefill in
 * one launch. It replaces the q/k RMSNorm and RoPE of aios/models/qwen3.py:66-70
 * (apply_rotary_pos_emb, aios/layers/attention.py:6-16) and the backend's store
 * and prefill (aios/attention/flashinfer.py:300-326), for batches whose requests have at most
 * max_q_len <= 64 new tokens (a keystroke's prefix prefill). qkv holds the raw
 * projection rows of the new tokens; each tile normalises and rotates its
 * queries and the new keys of its causal window, stores the K/V of its own
 * tokens at out_loc, and reads cached keys (positions below cached_len) from the
 * paged cache. Those cached keys must come from earlier launches. The output
 * and the stored K/V equal the two-call path bit for bit. The request and tile
 * arrays, positions, page table, norm weights and RoPE tables are read before
 * the kernel waits on the previous kernel of the stream: they must have been
 * written by copies, or by kernels that have completed whenever this one can
 * start (with a previous kernel that launches it after its own wait: two or
 * more kernels back). Only qkv is read after the wait. */
AIOSB_API int aiosb_attention_prefill_fused(
    const void* qkv, int64_t qkv_stride, const void* q_norm_w, const void* k_norm_w, float eps, const void* cos_tab,
    const void* sin_tab, int64_t max_pos, const int32_t* positions, const int32_t* out_loc, void* k_cache,
    void* v_cache, int64_t num_slots, const int32_t* page_table, int64_t table_stride, const int32_t* req_q_start,
    const int32_t* req_q_len, const int32_t* req_cached_len, const int32_t* req_table_row, const int32_t* tile_req,
    const int32_t* tile_q0, int64_t num_tiles, int64_t tile_tokens, int64_t max_q_len, int64_t num_qo_heads,
    int64_t num_kv_heads, int64_t head_dim, float scale, void* out, int64_t out_stride, int32_t* status,
    void* stream);

/* ---- Sampler -----------------------------------------------------------------
 * Replaces aios/engine/sample.py:54-163 (Sampler.sample_with_logprobs with
 * uniforms): per row, raw log-softmax of the bf16 logits, forbidden ids (the
 * shared list and row-specific int64 [rows, n_forbidden_rows]) set to -inf on the
 * sampling copy, then greedy argmax or temperature / top-k / top-p inverse-CDF
 * sampling with uniforms[r]. Ties between equal logits order by ascending token
 * id. Outputs token ids (int64) and raw log-probabilities (fp32).
 * vocab <= 32768; the sorted candidate set (top_k, or the whole vocabulary for a
 * top-p-only sampler) must not exceed 2048 entries. */
AIOSB_API int aiosb_sample(const void* logits, int64_t rows, int64_t vocab, int64_t row_stride, float temperature,
                 int64_t top_k, float top_p, int greedy, const float* uniforms, const int32_t* forbidden,
                 int64_t n_forbidden, const int64_t* forbidden_rows, int64_t n_forbidden_rows, int64_t* token_out,
                 float* logprob_out, int32_t* status, void* stream);

/* Teacher-forced scoring (aios/ime.py:731, 827-832, 858-860): out[r] =
 * log_softmax(float(logits[r]))[targets[r]] in fp32. Row r starts at
 * logits + r * row_stride; row_stride 0 scores every target against one shared
 * row (the prefix logits of the shared-decode scoring mode). */
AIOSB_API int aiosb_token_logprobs(const void* logits, int64_t rows, int64_t vocab, int64_t row_stride,
                                   const int64_t* targets, float* out, int32_t* status, void* stream);

/* Replaces stateless_uniforms (aios/engine/sample.py:12-45): out[r, t] is the
 * splitmix64 uniform of (seeds[r], t), computed in fp64 and rounded to fp32. */
AIOSB_API int aiosb_stateless_uniforms(const int64_t* seeds, int64_t rows, int64_t steps, float* out, void* stream);

/* ---- Free-slot FIFO ----------------------------------------------------------
 * Replaces CacheManager.allocate / _free (aios/scheduler/cache.py:16-18,46-51):
 * the free list is a device ring of `capacity` int32 slot (or page) ids with
 * logical head/tail counters kept by the caller; allocate takes the first n
 * entries, free appends at the tail, so the order is the reference's FIFO order.
 * slot_free copies from a separate array; slot_free_range appends ring entries
 * [begin, begin + n) (already allocated: begin + n <= head <= tail). */
AIOSB_API int aiosb_slot_alloc(const int32_t* ring, int64_t capacity, int64_t head, int64_t n, int32_t* out, void* stream);
AIOSB_API int aiosb_slot_free(int32_t* ring, int64_t capacity, int64_t tail, const int32_t* slots, int64_t n, void* stream);
AIOSB_API int aiosb_slot_free_range(int32_t* ring, int64_t capacity, int64_t begin, int64_t n, int64_t tail, void* stream);

/* Keystroke page-table reset (aios/ime.py:482-485, 1155): rows [0, rows) of the
 * table get prefix[0..n) in columns [0, n) and zeros in [n, width). */
AIOSB_API int aiosb_page_table_fill(int32_t* table, int64_t stride, int64_t rows, int64_t width,
                                   const int32_t* prefix, int64_t n, void* stream);

/* ---- CandidateGroup step -----------------------------------------------------
 * Device state of one branch batch (aios/ime.py:891-1054), written by the host
 * at round start and advanced by aiosb_group_step. */
typedef struct aiosb_group_state {
  int32_t step;            /* next step to sample                                   */
  int32_t max_steps;       /* max_new_tokens; row stride of the [rows, steps] arrays */
  int32_t min_new_tokens;  /* EOS/terminal ids banned while step < this             */
  int32_t prefix_len;      /* tokens of the shared prefix                           */
  int32_t row_offset;      /* first page-table row of this batch                    */
  int32_t rows;            /* local rows (attempts)                                 */
  int32_t vocab;
  int32_t eos_id;
  int32_t pad_id;
  int32_t greedy;
  int32_t top_k;
  float temperature;
  float top_p;
  int32_t page_size;       /* 1 or 16                                               */
  int32_t n_terminal;      /* terminal punctuation ids (stop code 2)                */
  int32_t n_minlen;        /* ids banned before min_new_tokens                      */
  int32_t n_banned;        /* refill exact-repeat sequences                         */
  int32_t banned_width;
  int32_t ban_min_prefix;  /* refill_ban_min_prefix_tokens                          */
  int32_t done;
  int32_t cancelled;
  int32_t n_active;
  int32_t active_model_tokens;
  int32_t arrive;          /* last-CTA counter, 0 between launches                  */
  int64_t head;            /* free-slot FIFO logical head / tail / ring capacity    */
  int64_t tail;
  int64_t capacity;
  int64_t table_stride;    /* page-table row stride (elements)                      */
} aiosb_group_state;

typedef struct aiosb_group_ptrs {
  aiosb_group_state* state;
  const int32_t* cancel_flag; /* host-mapped word set by the canceller, or NULL    */
  int32_t* host_mirror;       /* host-mapped [steps_done, done, cancelled, n_active]; 16-byte aligned: one store */
  void* logits;               /* [rows, vocab] bf16: next step's logits            */
  float* uniforms;            /* [rows, max_steps]                                  */
  int32_t* output_ids;        /* [rows, max_steps]                                  */
  float* token_logprobs;      /* [rows, max_steps]                                  */
  int32_t* counts;            /* [rows]                                             */
  float* logprob_sums;        /* [rows]                                             */
  int32_t* stop_codes;        /* [rows] 0 / 1 eos / 2 terminal                      */
  int32_t* active;            /* [rows]                                             */
  int32_t* finished;          /* [rows] scratch                                     */
  int32_t* tokens;            /* [rows] decode input ids                            */
  int32_t* positions;         /* [rows]                                             */
  int32_t* seq_lens;          /* [rows]                                             */
  int32_t* out_loc;           /* [rows] KV slot of the decode token                 */
  int32_t* row_page;          /* [rows] current suffix page (page_size > 1)         */
  int32_t* row_table;         /* [rows] page-table row of each local row            */
  const int32_t* terminal_ids;
  const int32_t* minlen_ids;
  const int32_t* banned;      /* [n_banned, banned_width]                           */
  const int32_t* banned_len;  /* [n_banned]                                         */
  int32_t* page_table;
  const int32_t* ring;        /* free-slot FIFO                                     */
  int32_t* status;
  /* Optional, or NULL: the LM head's per-16-id tile statistics of `logits`
   * (aiosb_linear_stat_norm_tiles, [vocab / 16, rows, 4] with `rows` the step's
   * rows). When set, steps after the first of a round (whose logits the decode
   * forward wrote, not aiosb_group_begin) bound a top-k row's candidates and its
   * log-sum-exp from the tiles instead of scanning the row; the tokens are the
   * same, the log-probabilities agree to fp32 rounding. */
  const float* tile_stats;
  /* AIOSB_GROUP_AFTER_FORWARD, or 0. */
  int64_t flags;
  /* Optional, or NULL: the next forward's input, written by the step for every
   * row it samples (the first kernel of the standard-residual forward, done here
   * instead of in a launch of its own). embed_out[r] = embed_w[token] (bf16
   * [rows, hidden]), embed_stat_x[r] its fp32 copy and embed_stat_ss[r] its sum
   * of squares: aiosb_embedding_stat's outputs, bit for bit. */
  const void* embed_w;   /* [vocab, hidden] bf16 embedding table */
  void* embed_out;       /* [rows, hidden] bf16 */
  float* embed_stat_x;   /* [rows, hidden] fp32 */
  float* embed_stat_ss;  /* [rows] fp32 */
  int64_t hidden;        /* multiple of 8 */
} aiosb_group_ptrs;

/* aiosb_group_ptrs.flags: the previous kernel on the stream is the decode
 * forward's last kernel (the LM head), which writes only `logits` and
 * `tile_stats`, and every other input of the step (the state, the row arrays,
 * uniforms, id lists, the FIFO) was written by work that had completed before
 * that forward began. The step then reads those inputs while the LM head still
 * runs, and waits on it only for the logits. */
#define AIOSB_GROUP_AFTER_FORWARD 1

/* Round start: resets the per-row outputs, copies the prefix logits [vocab] into
 * every row of `logits`, draws the uniform streams of seeds seed_base + r, sets
 * row_table[r] = row_offset + r and marks rows [0, attempts) active. */
AIOSB_API int aiosb_group_begin(const aiosb_group_ptrs* g, const void* prefix_logits, uint64_t seed_base, int64_t attempts,
                      int64_t rows, void* stream);

/* One sampling step of every active row plus the step epilogue (finished-row
 * compaction, FIFO slot allocation in row order, page-table write, next forward's
 * tokens/positions/seq_lens/out_loc). Reads everything it needs from device
 * memory, so one captured launch serves every step of every round. */
AIOSB_API int aiosb_group_step(const aiosb_group_ptrs* g, int64_t rows, int64_t vocab, int64_t top_k_max, void* stream);

/* ---- Persistent decode step ------------------------------------------------
 * Replaces one decode forward of the standard-residual decoder,
 * Qwen3ForCausalLM.forward (aios/models/qwen3.py:101-173) as driven by
 * ImeCompletionEngine._decode_step (aios/ime.py:1219-1251): the embedding, every
 * layer (RMSNormFused + qkv linear, q/k RMSNorm + RoPE + KV store + paged decode
 * attention, o linear + residual, RMSNormFused + gate/up linear + SwiGLU, down
 * linear + residual), the final norm and the LM head, in ONE kernel launch (one
 * CTA per SM; a producer warp streams each CTA's weight tiles into shared memory
 * while its consumer warps run the dependent phases). Activations pass between
 * CTAs through the caller's `work` area as flagged 16-byte lines, so each phase
 * waits (bounded) for exactly the values it reads. Serves hidden 768,
 * intermediate 2048, head_dim 64 or 96, at most 7 query heads per KV head, 1..16
 * rows, at most 48 layers. */
typedef struct aiosb_decode_layer {
  const void* w_qkv;      /* [(Hq + 2 Hkv) d, 768] bf16 (packed q | k | v)            */
  const void* w_o;        /* [768, Hq d] bf16                                         */
  const void* w_gate_up;  /* [4096, 768] bf16 in 64-row blocks [g0..63|u0..63|g64..] */
  const void* w_down;     /* [768, 2048] bf16                                         */
  const void* in_norm;    /* [768] bf16 input_layernorm weight                        */
  const void* post_norm;  /* [768] bf16 post_attention_layernorm weight               */
  const void* q_norm;     /* [d] bf16                                                 */
  const void* k_norm;     /* [d] bf16                                                 */
  void* k_cache;          /* [num_slots, Hkv, d] bf16: this layer's keys              */
  void* v_cache;          /* [num_slots, Hkv, d] bf16                                 */
} aiosb_decode_layer;

typedef struct aiosb_decode_step_args {
  const aiosb_decode_layer* layers; /* device array [num_layers]                       */
  int32_t num_layers, rows, hidden, intermediate, num_qo_heads, num_kv_heads, head_dim, vocab;
  float eps;                        /* RMSNorm epsilon                                  */
  float scale;                      /* attention scale (head_dim^-0.5)                  */
  const void* embed;                /* [vocab, 768] bf16                                */
  const void* final_norm;           /* [768] bf16                                       */
  const void* lm_head;              /* [vocab, 768] bf16 (the embedding when tied)      */
  /* decode metadata (written by aiosb_group_step before this launch) */
  const int32_t* tokens;            /* [rows] input ids                                 */
  const int32_t* positions;         /* [rows]                                           */
  const int32_t* out_loc;           /* [rows] KV slot of the new token                  */
  const int32_t* row_table;         /* [rows] page-table row of each local row          */
  const int32_t* seq_lens;          /* [rows] keys per row including the new one        */
  const int32_t* prefix_len;        /* device scalar: shared prefix keys                */
  const int32_t* active;            /* [rows] nonzero = row runs, or NULL               */
  const int32_t* page_table;
  int64_t table_stride;
  int64_t num_slots;
  const void* cos_tab;              /* [max_pos, d] bf16 RoPE tables                    */
  const void* sin_tab;
  int32_t max_pos;
  void* work;                       /* aiosb_decode_step_work_bytes() bytes, 16-byte
                                       aligned, zero before the first launch            */
  void* logits;                     /* [rows, vocab] bf16 output                        */
  int64_t logits_stride;
  uint32_t* sync;                   /* [aiosb_decode_step_sync_words()], zero before
                                       the first launch                                  */
  int32_t* status;
  uint64_t wait_limit_ns;           /* bound of every wait; 0 = 2 s                     */
  uint32_t test_flag_skew;          /* 0. Tests only: every wait then expects a flag no
                                       producer writes, so it runs out and reports
                                       AIOSB_DEV_WAIT_TIMEOUT                            */
  int32_t grid_ctas;                /* 0 = one CTA per SM                               */
} aiosb_decode_step_args;

/* Bytes of the `work` area for a model with these heads (any rows <= 16). */
AIOSB_API int64_t aiosb_decode_step_work_bytes(int64_t num_qo_heads, int64_t num_kv_heads, int64_t head_dim);

/* Words of the `sync` array (launch counter, abort word, flag epoch). */
AIOSB_API int64_t aiosb_decode_step_sync_words(void);

/* One decode forward (see above). Launches with programmatic dependent launch: the
 * weight streaming starts while the previous kernel (the group step) runs; the
 * phases wait for it. Launches that share `work` / `sync` must not overlap. */
AIOSB_API int aiosb_decode_step(const aiosb_decode_step_args* args, void* stream);

/* aiosb_group_step without the caller's scratch array. No counterpart in the
 * reference: it is an addition for callers that cannot call cudaMalloc, such as
 * a plugin inside a host process that owns all device memory through its own
 * allocator (a caching pool that has reserved the free HBM, or a fixed budget
 * handed out up front) and gives the plugin only the buffers it needs, so a
 * cudaMalloc of the plugin's own fails or escapes the host's accounting; and a
 * per-keystroke path where a cudaMalloc / cudaFree pair would synchronise the
 * device in the middle of a keystroke.
 * Same arguments, results and errors as aiosb_group_step, except that
 * g->finished is neither read nor written (it may be NULL here): the per-row
 * finish flags go through a 32-entry int32 array inside the library, so rows
 * above 32 are rejected with AIOSB_ERR_UNSUPPORTED. aiosb_group_begin zeroes
 * g->finished at round start when it is not NULL and skips it when it is, so a
 * caller without that array passes NULL to both calls.
 * The call allocates and frees nothing. Its first call in a CUDA context (one per
 * device, and a new one after cudaDeviceReset) looks up the array's device
 * address (cudaGetSymbolAddress, on the current device) and caches it under the
 * context's id; that first call should come before any stream capture. Each call
 * clears the array with an
 * asynchronous memset on `stream` before the step kernel. Every GPU that loads
 * the library holds the array until the process exits, and all calls on a device
 * share it: calls that overlap on the GPU (two groups stepping on different
 * streams at once) race on it. */
AIOSB_API int aiosb_group_step_static(const aiosb_group_ptrs* g, int64_t rows, int64_t vocab, int64_t top_k_max,
                                      void* stream);

#ifdef __cplusplus
}
#endif

#endif /* AIOS_B200_H_ */
