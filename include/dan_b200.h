/* dan_b200: C ABI of the B200 (sm_100a) kernels for dan's packed prefill read path.
 *
 * Conventions for every entry point:
 *   - pointers are device pointers unless named *_host; strides are in elements;
 *   - bf16 tensors are raw uint16 bf16 bit patterns; e4m3 tensors are bytes;
 *   - ``stream`` is a cudaStream_t (NULL = legacy default stream);
 *   - ``status`` is a device int32 word: kernels write the first error they detect
 *     (a bounded wait that ran out, an out-of-range index) instead of hanging or
 *     faulting; read it with dan_read_status once per batch;
 *   - the return value is 0, or a negative code with the text in dan_last_error();
 *   - callers own every buffer; the only allocation is the stream-K workspace of the GEMMs
 *     (dan_gemm_bf16 below), and dan_gemm_bf16_noalloc is the same GEMM without it.
 *
 * Each function names the reference (quangliz/dan) interface it replaces, except
 * dan_gemm_bf16_noalloc, which has no counterpart in the reference.
 *
 * The library caches per-device state (tensor-map encoder, SM counts, the stream-K workspace
 * and the static scratch's address) for the life of the process: it must not outlive the
 * device's primary context (no cudaDeviceReset between calls).
 */
#ifndef DAN_B200_H
#define DAN_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

const char* dan_version(void);
/* Text of the last error on the calling thread. */
const char* dan_last_error(void);
/* Copy *status_dev to *status_host, synchronise ``stream``, clear the device word if set. */
int dan_read_status(int32_t* status_dev, int32_t* status_host, void* stream);
/* Self-test of the kernels' bounded waits (dan's engine fails a batch whose forward raised,
 * dan/engine.py:102-107; this checks the device side of that path): one thread waits on an
 * mbarrier phase nothing completes (kind 0, reports 1 = kTimeoutFull) or on a device word
 * ``flag`` that stays 0 (kind 1, reports 6 = kTimeoutPartial), gives up after about a second
 * and returns, leaving the code in *status. */
int dan_selftest_wait(int kind, const void* flag, int32_t* status, void* stream);

/* Tree-masked attention over a packed batch, one launch for all segments and heads.
 * Replaces attend / _attend_varlen (dan/attention.py:200-241: three varlen flash calls,
 * row gathers, past concatenation and lse_merge, fused.py:94-101); semantics of
 * _attend_dense (attention.py:244-270).
 * q [n_rows, n_heads, head_dim], k/v [n_rows, n_kv_heads, head_dim] (row/head strides given,
 * unit stride in head_dim, 16-byte aligned); k_pool/v_pool [pool_rows, n_kv_heads, head_dim]
 * hold cached prefix pages of 128 tokens (may be NULL when no segment has a past).
 * tiles: int32 [n_tiles, 12] {row0, nrows, seg_start, past, ppad, split, nblk_a, blk_b0,
 * blk_b1, page0, q0v, 0}; row_own: int32 [n_rows] packed row where each row's run starts;
 * pages: int32 pool page per cached 128-token block. head_dim in {64, 128, 256}.
 * schedule (optional, paired-head kernel): int32 [sched_ctas + 1] CSR offsets then the work
 * items (tile * n_heads/2 + head pair) of each persistent CTA; NULL = round-robin. */
int dan_tree_attention(const void* q, int64_t q_row, int64_t q_head, const void* k, int64_t k_row, int64_t k_head,
                       const void* v, int64_t v_row, int64_t v_head, const void* k_pool, const void* v_pool,
                       int64_t pool_row, int64_t pool_head, int pool_rows, void* out, int64_t out_row,
                       int64_t out_head, int n_rows, int n_heads, int n_kv_heads, int head_dim, const int* tiles,
                       int n_tiles, const int* row_own, const int* pages, const int* schedule, int sched_ctas,
                       float scale, int32_t* status, void* stream);

/* C[m, n] = A[m, k] * W[n, k]^T in bf16 with fp32 accumulation on tcgen05 tensor cores.
 * Replaces nn.Linear in the decoder (dan/models/llama.py:78,87,102; qwen3_5.py:185,212,319,329,344)
 * and fuses: epilogue 0 store (+bias), 1 C = R + bf16(acc) (the residual adds, llama.py:116-117),
 * 2 SwiGLU over W rows interleaved in 128-row [gate | up] blocks, C has n/2 columns
 * (swiglu, dan/fused.py:59-61). C may alias R (in-place residual).
 * When m >= 256, k is at least 128 iterations of 128 bytes (8192 bf16 / 16384 e4m3) and the
 * last wave of 256 x 256 tiles is ragged, the first such call on a (device, stream) allocates
 * a stream-K workspace (cudaMalloc, ~19 MB on 148 SMs) kept for the life of the process;
 * calls sharing a stream use it in stream order. */
int dan_gemm_bf16(const void* a, int64_t lda, const void* w, int64_t ldw, void* c, int64_t ldc, const void* resid,
                  int64_t ldr, const void* bias, int m, int n, int k, int epilogue, int32_t* status, void* stream);

/* dan_gemm_bf16 for callers that cannot allocate device memory: processes whose device memory is
 * all handed out by their own allocator (a caching allocator or a memory plan made at start-up)
 * and servers that must not make the device-synchronising cudaMalloc in the middle of a request.
 * It has no counterpart in the reference. It allocates nothing: when a call takes the stream-K
 * path (m >= 256, k at least 8192 bf16, a ragged last wave of 256 x 256 tiles) the partial tiles
 * go to a static __device__ array of the library sized for at most 80 CTA pairs (about 21 MB,
 * held by every device that loads the library until the process exits). Such a call on a device
 * with more than 80 CTA pairs (160 SMs) returns -22; other shapes run on any device.
 * The first call on a device looks up the array's address (cudaGetSymbolAddress) with that
 * device current; make that first call before any stream capture. All calls share the array
 * and the kernel resets its per-tile counters itself, so each call starts from zeroed counters;
 * calls that overlap on the GPU (different streams without ordering) race on the array.
 * Same arguments and results as dan_gemm_bf16. */
int dan_gemm_bf16_noalloc(const void* a, int64_t lda, const void* w, int64_t ldw, void* c, int64_t ldc,
                          const void* resid, int64_t ldr, const void* bias, int m, int n, int k, int epilogue,
                          int32_t* status, void* stream);

/* e4m3 x e4m3 GEMM with per-row (token) and per-column (output channel) fp32 scales, bf16 out.
 * Replaces FP8Linear.forward (dan/quant.py:37-42, torch._scaled_mm row-wise); epilogues as above. */
int dan_gemm_e4m3(const void* a, int64_t lda, const float* a_scale, const void* w, int64_t ldw, const float* w_scale,
                  void* c, int64_t ldc, const void* resid, int64_t ldr, const void* bias, int m, int n, int k,
                  int epilogue, int32_t* status, void* stream);

/* out[r] = table[ids[r]] (nn.Embedding, dan/models/llama.py:157). */
int dan_embed(const int64_t* ids, const void* table, int64_t ldt, int64_t vocab, void* out, int64_t ldo, int rows,
              int cols, int32_t* status, void* stream);

/* RMSNorm over rows (r / inner, r % inner) of x; mode 0 Llama (dan/fused.py:35-40), 1 zero-centred
 * (fused.py:43-48). Optional fused per-row e4m3 quantisation of the result (fused.py:85-91). */
int dan_rms_norm(const void* x, int64_t x_outer, int64_t x_inner, int inner, const void* w, float eps, int mode,
                 void* y, int64_t y_outer, int64_t y_inner, void* q8, int64_t ldq, float* q8_scale, int rows,
                 int cols, void* stream);

/* Per-row e4m3 quantisation, scale = max(amax, 1e-12) / 448 (fp8_quantize, dan/fused.py:85-91;
 * weight quantisation, dan/quant.py:26-33). */
int dan_quantize_e4m3(const void* x, int64_t ldx, void* q, int64_t ldq, float* scale, int rows, int cols,
                      void* stream);

/* GEMMs with epilogue 3: RoPE on every rope_hd-column head of the first rope_cols output
 * columns, from cos/sin tables [m, rope_hd/2] (the q/k/v projection + rotary of
 * dan/models/llama.py:78-85 in one kernel). Other epilogues as dan_gemm_bf16 / dan_gemm_e4m3. */
int dan_gemm_bf16_rope(const void* a, int64_t lda, const void* w, int64_t ldw, void* c, int64_t ldc,
                       const void* resid, int64_t ldr, const void* bias, int m, int n, int k, int epilogue,
                       int rope_cols, int rope_hd, const float* cos_t, const float* sin_t, int32_t* status,
                       void* stream);
int dan_gemm_e4m3_rope(const void* a, int64_t lda, const float* a_scale, const void* w, int64_t ldw,
                       const float* w_scale, void* c, int64_t ldc, const void* resid, int64_t ldr, const void* bias,
                       int m, int n, int k, int epilogue, int rope_cols, int rope_hd, const float* cos_t,
                       const float* sin_t, int32_t* status, void* stream);

/* cos/sin tables [rows, half] of angle = float(pos) * inv_freq, rounded to bf16 as the reference
 * casts them (dan/models/llama.py:155-158; qwen3_5.py:411-414). Built once per forward. */
int dan_rope_table(const int64_t* pos, const float* inv_freq, int rows, int half, float* cos_t, float* sin_t,
                   void* stream);

/* In-place rotate-half RoPE on the first ``rot`` dims of each head from the tables
 * (dan/models/llama.py:43-45; rotate_partial, dan/fused.py:69-76). */
int dan_rope(void* x, int64_t ld_row, int64_t ld_head, int heads, int head_dim, int rot, const float* cos_t,
             const float* sin_t, int rows, void* stream);

/* o *= sigmoid(gate), gate read per head (sigmoid_gate, dan/fused.py:64-66; qwen3_5.py:328). */
int dan_sigmoid_gate(void* o, int64_t ldo, const void* g, int64_t ldg, int64_t g_head_stride, int head_dim, int rows,
                     int cols, void* stream);

/* Store packed k/v rows into prefix-pool rows (the prefix saves of dan/attention.py:202-204
 * and PrefixCache.put, dan/cache.py:30-39). */
int dan_kv_store(const void* k, const void* v, int64_t ld_row, int64_t ld_head, void* pool_k, void* pool_v,
                 int64_t pool_row, int64_t pool_head, const int* src_rows, const int* dst_rows, int count, int heads,
                 int head_dim, void* stream);

/* Per question q: final RMSNorm of h[read_rows[q]], logits = W_lm[label_ids[off[q]:off[q+1]]] @ h
 * in fp32, and their softmax. Replaces the read-row gather + per-branch label_logits loop
 * (dan/runner.py:73-74, dan/models/llama.py:161-165) and readout.softmax (dan/readout.py:13-17).
 * mode: 0 Llama norm, 1 zero-centred norm, 2 rows already normed (label_logits on a hidden
 * state). A question with more than max_labels labels sets kBadIndex and keeps its first
 * max_labels. */
int dan_label_readout(const void* h, int64_t ldh, const int* read_rows, const void* norm_w, float eps, int mode,
                      const void* w_lm, int64_t ldw, int64_t vocab, const int* label_ids, const int* offsets,
                      int n_questions, int hidden, int max_labels, float* logits, float* probs, int32_t* status,
                      void* stream);

/* Gated DeltaNet layers (Qwen3.5), dan/models/qwen3_5.py:161-298.
 * Row codes for conv sources: >= 0 packed row of src; -1 a zero row; <= -2 row (-code-2) of hist.
 * dan_causal_conv: out[r] = silu(sum_j w[:, j] * row(prev[r][2-j]) ... ) over the run's
 * [history; tokens] (F.conv1d + SiLU of _phase, qwen3_5.py:214-220); prev: int32 [rows, 3]
 * codes of the 1st/2nd/3rd previous rows; w: [channels, 4]. */
int dan_causal_conv(const void* src, int64_t ld_src, const void* hist, int64_t ld_hist, const void* weight,
                    const int* prev, void* out, int64_t ld_out, int rows, int channels, void* stream);
/* dst[i] = row(codes[i]): the conv tails stored with prefix-cache saves (qwen3_5.py:207-209). */
int dan_gather_rows(const void* src, int64_t ld_src, const void* hist, int64_t ld_hist, const int* codes, int count,
                    void* dst, int64_t ld_dst, int cols, void* stream);
/* Gated delta rule over the tree of runs of a packed batch (delta_rule, qwen3_5.py:136-158; the
 * trunk/branch phases of DeltaNet.forward, 196-210), with the gates (delta_gates, fused.py:79-82)
 * and the q/k l2 norms fused, in 64-token chunks (the WY form of chunk_gated_delta_rule).
 * segs: int32 [n_segs, 8] {trunk_start, trunk_len, cut, init_slot, save_slot, branch0,
 * n_branches, first chunk}; branches: int32 [.., 4] {start, len, first chunk, 0}; chunks: int32
 * [n_chunks, 2] {first row, rows <= 64}, each segment's runs (trunk to the cut, rest of the
 * trunk, each branch) cut into chunks listed contiguously in that order; state_pool: fp32
 * [slots, hv, 128, 128] of this layer (init / save slots, -1 = none). dk = dv = 128.
 * out: [rows, hv * 128] bf16, 16-byte aligned, ld_out a multiple of 8 (whole chunks of it are
 * written by TMA store). scratch: caller-owned device buffer of
 * dan_gated_delta_scratch_bytes(n_chunks, hk, hv) bytes (16-byte aligned) for the per-chunk
 * intermediates; it is fully rewritten by each call.
 * lead_chunk0 / lead_chunks: 0 / 0, or the chunk range [lead_chunk0, lead_chunk0 + lead_chunks)
 * of segment 0 (segs[0]), when the caller expects that segment's chain to outlast the pre-pass
 * of all the others: the call then runs that chain beside the other segments' pre-pass (a second
 * stream of the library's, forked from and joined back into ``stream`` by events); results are
 * identical either way. */
int dan_gated_delta_scan(const void* q, const void* k, const void* v, int64_t ld_qkv, const void* b, const void* a,
                         int64_t ld_ba, const float* a_log, const float* dt_bias, const int* segs, int n_segs,
                         const int* branches, const int* chunks, int n_chunks, float* state_pool,
                         int64_t slot_stride, void* out, int64_t ld_out, int hk, int hv, int dk, int dv,
                         float q_scale, void* scratch, int64_t scratch_bytes, int lead_chunk0, int lead_chunks,
                         int32_t* status, void* stream);
/* Bytes of scratch dan_gated_delta_scan needs for n_chunks chunks (59136 per chunk and value head
 * plus 16384 per chunk and key head). */
int64_t dan_gated_delta_scratch_bytes(int n_chunks, int hk, int hv);
/* dan_gated_delta_scan with the gates given instead of computed: beta [rows, hv] bf16 (row stride
 * ld_beta) and the log decay g [rows, hv] fp32 (row stride ld_g); q and k still l2-normalised
 * inside. Replaces delta_rule(q, k, v, g, beta, lengths, states) (dan/models/qwen3_5.py:136-158);
 * tables, scratch and state pool as dan_gated_delta_scan. */
int dan_delta_rule_scan(const void* q, const void* k, const void* v, int64_t ld_qkv, const void* beta, int64_t ld_beta,
                        const float* g, int64_t ld_g, const int* segs, int n_segs, const int* branches,
                        const int* chunks, int n_chunks, float* state_pool, int64_t slot_stride, void* out,
                        int64_t ld_out, int hk, int hv, int dk, int dv, float q_scale, void* scratch,
                        int64_t scratch_bytes, int32_t* status, void* stream);

/* Stand-alone element-wise steps that the model path fuses elsewhere (dan/fused.py):
 * out = bf16(bf16(silu(gate)) * up) (swiglu, fused.py:59-61); */
int dan_swiglu(const void* gate, int64_t ldg, const void* up, int64_t ldu, void* out, int64_t ldo, int rows, int cols,
               void* stream);
/* beta = bf16(sigmoid(b)), g = -exp(a_log) * softplus(a + dt_bias) fp32, per (row, head)
 * (delta_gates, fused.py:79-82); */
int dan_delta_gates(const void* b, int64_t ldb, const void* a, int64_t lda, const float* a_log, const float* dt_bias,
                    void* beta, int64_t ldbeta, float* g, int64_t ldg, int rows, int heads, void* stream);
/* exact merge of two attention results over disjoint key sets from their log-sum-exps;
 * o [t_rows, heads, head_dim] bf16 with row stride ld_row, lse [heads, t_rows] fp32
 * (lse_merge, fused.py:94-101); */
int dan_lse_merge(const void* o_a, const float* lse_a, const void* o_b, const float* lse_b, void* out, int64_t ld_row,
                  int t_rows, int heads, int head_dim, void* stream);
/* e4m3 codes with one scale for the tensor, *scale = max(amax, 1e-12) / 448 (fp8_quantize with
 * rowwise=False, fused.py:85-91; per-tensor FP8Linear, quant.py:26-33). */
int dan_quantize_e4m3_tensor(const void* x, int64_t ldx, void* q, int64_t ldq, float* scale, int rows, int cols,
                             void* stream);

/* y = bf16(w * bf16(x_hat)) * silu(z) per (row, head) (gated_rms_norm, dan/fused.py:51-56). */
int dan_gated_rms_norm(const void* x, int64_t ldx, const void* z, int64_t ldz, const void* w, float eps, void* y,
                       int64_t ldy, int rows, int heads, int dv, void* stream);

#ifdef __cplusplus
}
#endif

#endif
