/* specdec_b200.h -- C ABI of libspecdec_b200.so, the B200 (sm_100a) verify/accept hot path of
 * nano-vllm-speculative-decoding.
 *
 * Conventions
 *   - Every pointer argument is a device pointer unless stated; tensors are dense and row-major.
 *   - `stream` is a cudaStream_t (may be 0); every call is asynchronous on it and launches nothing elsewhere.
 *   - Every entry point returns 0 on success or a non-zero status; specdec_last_error() then returns a
 *     thread-local message.  Shapes, dtypes and sizes are validated on the host before any launch.
 *       1 invalid argument, 2 workspace too small, 3 unsupported by this build, 4 CUDA error, 5 device timeout
 *   - No entry point allocates device memory.  Scratch comes from a caller-owned workspace sized by the matching
 *     *_workspace_bytes query; it must be zero-filled once when allocated (its tickets and keys are left zeroed
 *     by every call), and one workspace must not be used by two streams at once.
 *   - dtype codes: 0 = fp32, 1 = bf16, 2 = fp16.
 *
 * Reference file:line citations are paths inside the nano-vllm-speculative-decoding repository.
 */
#ifndef SPECDEC_B200_H_
#define SPECDEC_B200_H_

#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ------------------------------------------------------------------------------------------ library */
/* Library plumbing, no counterpart in the reference (its Python raises): the calling thread's message for the
 * last non-zero status, the ABI version. */
const char* specdec_last_error(void);
int specdec_version(void);
/* 1 when the current CUDA device is compute capability 10.0 (the only target of this build). */
int specdec_device_supported(void);

/* ------------------------------------------------------------------------------------------ kernel 1: sampler */
/* Workspace bytes for the sampler entry points over `rows` rows of logits / probabilities (no counterpart in the
 * reference: torch allocates its temporaries). */
size_t specdec_sampler_workspace_bytes(long long rows);
/* Workspace bytes with which specdec_accept over T rows, B requests and vocabulary V races the tail over noise
 * codes: specdec_sampler_workspace_bytes(T) plus 2 bytes per element of the [B, V] noise.  A call whose E is NULL,
 * whose offset_E is a multiple of 4 (torch's always are) and whose rows do not truncate (max_top_k = 0) then
 * draws the noise once into 16-bit codes that bound each E from both sides, streams the tail rows against them
 * and regenerates exactly only the elements that can still win; the tokens are the ones the smaller workspace
 * gives.  Returns 0 for non-positive sizes. */
size_t specdec_accept_workspace_bytes(long long rows, long long B, long long V);

/* Philox offset increment torch's CUDA generator consumes for one torch.rand / exponential_ draw of `numel`
 * floats on the current device (ATen's calc_execution_policy); callers advance their generator by it, so it ends
 * where the reference's draws (nanovllm/layers/spec_sampler.py:141,149) leave it. */
unsigned long long specdec_philox_increment(long long numel);

/* probs_from_logits (nanovllm/layers/spec_sampler.py:65-69, truncate_logits :72-96).
 * logits [R, V] (dtype), parameter row of logits row r = r / rows_per_param; temperature [R/rows_per_param]
 * fp32 > 0; top_k int64 (required when max_top_k > 0, 0 = no truncation for that row); top_p fp32 (required
 * when has_top_p).  probs [R, V] fp32 = softmax(mask(logits / T)). */
int specdec_probs(const void* logits, int dtype, long long R, long long V, long long rows_per_param,
                  const float* temperature, const long long* top_k, const float* top_p, int max_top_k,
                  int has_top_p, float* probs, void* workspace, size_t workspace_bytes, void* stream);

/* accept_random / accept_random_varlen (spec_sampler.py:114-150), and with x_is_probs = 0 the round driver's
 * fused probs_from_logits + accept (nanovllm/engine/speculative.py:450-462).  Without top-k, logits rows are
 * reduced only up to each request's first rejected draft (its later rows cannot change the result): one
 * thread-block cluster per request walks its rows, when the requests fit one wave.
 * x [T, V]: fp32 probabilities (x_is_probs = 1) or logits of `dtype` with per-request temperature/top_k/top_p
 * [B].  q [B, k, V] fp32; drafts [B, k] int64; verified_lens [B] int64 in 1..k+1 summing to T, or NULL for
 * k + 1 each (T = B (k + 1)).  u [B, k] and E [B, V] (clamped Exp(1)) are the reference's two draws; when NULL
 * they are regenerated in-kernel exactly as torch's CUDA generator (seed, Philox offsets offset_u then
 * offset_E) would produce them.  Outputs n_accept [B], tail [B] int64.  Limits: B <= 1024, k <= 32,
 * T <= 16384, B * V < 2^31, top_k <= 1024. */
int specdec_accept(const void* x, int x_is_probs, int dtype, long long T, long long V, const float* q,
                   const long long* drafts, long long B, long long k, const long long* verified_lens,
                   const float* temperature, const long long* top_k, const float* top_p, int max_top_k,
                   int has_top_p, const float* u, const float* E, unsigned long long seed,
                   unsigned long long offset_u, unsigned long long offset_E, long long* n_accept,
                   long long* tail, void* workspace, size_t workspace_bytes, void* stream);

/* accept_greedy / accept_greedy_varlen (spec_sampler.py:153-169): logits [T, V] (dtype), drafts [B, k],
 * verified_lens as above.  One launch. */
int specdec_accept_greedy(const void* logits, int dtype, long long T, long long V, const long long* drafts,
                          long long B, long long k, const long long* verified_lens, long long* n_accept,
                          long long* tail, void* workspace, size_t workspace_bytes, void* stream);

/* race / sample (spec_sampler.py:104-111): out[r] = argmax_v weights[r, v] / E[r, v], first index on ties.
 * weights [R, V] fp32; E [R, V] fp32, or NULL to regenerate torch's exponential_ draw at (seed, offset_E). */
int specdec_race(const float* weights, long long R, long long V, const float* E, unsigned long long seed,
                 unsigned long long offset_E, long long* out, void* workspace, size_t workspace_bytes,
                 void* stream);

/* Plumbing for tests of the in-kernel draws (no counterpart in the reference): torch's exponential_ draw of numel
 * floats at (seed, offset), offset a multiple of 4, clamped at 1e-10 as nanovllm/layers/spec_sampler.py:101 does,
 * written either as the floats themselves (values [numel]) or as the 16-bit codes the accept's tail race reads
 * (codes [numel]; value i lies in [lo, hi), the floats whose bits are codes[i] << 16 and (codes[i] + 1) << 16).
 * Exactly one of codes and values is non-null. */
int specdec_exponential_codes(unsigned long long seed, unsigned long long offset, long long numel,
                              unsigned short* codes, float* values, void* stream);

/* specdec_accept without a workspace, for callers that cannot allocate device memory: a plugin whose host owns
 * the device memory budget and forbids cudaMalloc from extensions, or a latency-critical caller that may not
 * call cudaMalloc (which can synchronise the device).  No counterpart in the reference (it allocates through
 * torch).  Scratch is a fixed ~2.8 MB array in the library's device memory (held by every GPU that loads the
 * library until exit); T is limited to 1024 verified rows, larger calls fail with status 3.  The first call on
 * a device looks the array's address up (cudaGetSymbolAddress) and should come before any stream capture.
 * Every call clears the array's tickets and keys first; calls that overlap on the GPU race on the array.
 * Arguments and results as specdec_accept. */
int specdec_accept_noalloc(const void* x, int x_is_probs, int dtype, long long T, long long V, const float* q,
                           const long long* drafts, long long B, long long k, const long long* verified_lens,
                           const float* temperature, const long long* top_k, const float* top_p, int max_top_k,
                           int has_top_p, const float* u, const float* E, unsigned long long seed,
                           unsigned long long offset_u, unsigned long long offset_E, long long* n_accept,
                           long long* tail, void* stream);

/* ------------------------------------------------------------------------------------------ kernel 2: attention */
/* store_kvcache (nanovllm/layers/attention.py:10-40, the Triton store_kvcache_kernel): key/value rows [N, Hkv, D]
 * bf16 (row strides in elements) to flat slots slot_mapping[N] (int32) of k_cache / v_cache [num_slots, Hkv, D];
 * slot -1 is skipped, a slot >= num_slots is skipped and recorded in *err (device int, first error wins). */
int specdec_store_kvcache(const void* key, long long key_row_stride, const void* value, long long value_row_stride,
                          void* k_cache, void* v_cache, const int* slot_mapping, long long N, int num_kv_heads,
                          int head_dim, long long num_slots, int* err, void* stream);

/* Attention.forward's paged branches (nanovllm/layers/attention.py:59-77): flash_attn_varlen_func with
 * block_table (verify: cu_seqlens_q / cu_seqlens_k int32 [R + 1], causal bottom-right aligned) or
 * flash_attn_with_kvcache (decode: context_lens int32 [R], q_per_seq queries per row, causal or not).
 * q [T, H, 128] bf16 (row stride q_row_stride elements); caches [num_slots / block_size, block_size, Hkv, 128]
 * bf16; block_tables int32 [R, W]; out [T, H, 128] bf16 (row stride out_row_stride).  Limits: head_dim 128,
 * H / Hkv in {1, 2, 4, 8}, max_seqlen_q * H / Hkv <= 32, block_size a multiple of 128.  Rows whose metadata
 * is inconsistent are skipped and recorded in *err.  workspace: 256-byte aligned device bytes, zero-filled once
 * before first use (the kernel leaves it zeroed), at least specdec_attention_workspace_bytes(R, Hkv); calls that
 * share a workspace must not overlap on the GPU. */
long long specdec_attention_workspace_bytes(int R, int num_kv_heads);
int specdec_paged_attention(const void* q, long long T, long long q_row_stride, int num_heads, int num_kv_heads,
                            int head_dim, const void* k_cache, const void* v_cache, long long num_slots,
                            int block_size, const int* cu_seqlens_q, const int* cu_seqlens_k,
                            const int* context_lens, int q_per_seq, int R, const int* block_tables, int W,
                            int max_seqlen_q, float softmax_scale, int causal, void* out, long long out_row_stride,
                            void* workspace, long long workspace_bytes, int* err, void* stream);

/* specdec_paged_attention (Attention.forward, nanovllm/layers/attention.py:59-77) with launch flags.
 * SPECDEC_ATTN_EARLY_LAUNCH: launched as a programmatic dependent of
 * the preceding kernel in the stream, so its prologue (row metadata scan, barrier and tensor-memory setup) runs
 * while that kernel finishes; everything else waits for that kernel's completion.  The caller promises that the
 * preceding kernel does not write cu_seqlens_q / cu_seqlens_k / context_lens / block_tables (q and the caches it
 * may write).  specdec_paged_attention is this call with flags 0. */
#define SPECDEC_ATTN_EARLY_LAUNCH 1u
/* Bits 8..15 of flags: at most this many CTAs (persistent, one per SM; 0 = one per SM of the device), so the
 * kernel can share the GPU with work on another stream that runs on the remaining SMs.
 * SPECDEC_ATTN_MAX_CTAS(n) builds the field. */
#define SPECDEC_ATTN_CTAS_SHIFT 8u
#define SPECDEC_ATTN_MAX_CTAS(n) (((unsigned)(n) & 0xffu) << SPECDEC_ATTN_CTAS_SHIFT)
int specdec_paged_attention_ex(const void* q, long long T, long long q_row_stride, int num_heads, int num_kv_heads,
                               int head_dim, const void* k_cache, const void* v_cache, long long num_slots,
                               int block_size, const int* cu_seqlens_q, const int* cu_seqlens_k,
                               const int* context_lens, int q_per_seq, int R, const int* block_tables, int W,
                               int max_seqlen_q, float softmax_scale, int causal, void* out, long long out_row_stride,
                               void* workspace, long long workspace_bytes, int* err, unsigned flags, void* stream);

/* specdec_paged_attention_ex writing its output to num_outs (1 .. 8) destinations with the same offsets and row
 * stride: outs is a HOST array of device addresses, each a [T, H, 128] bf16 output (this GPU's memory, or a peer
 * GPU's memory mapped into this process).  For the KV-head tensor-parallel verify attention with peer stores:
 * under the reference's head split (nanovllm/models/qwen3.py:29-35, nanovllm/layers/linear.py:92) rank r attends
 * with its H/N heads and passes every rank's [T, H_total, 128] output at head offset r*H/N (out_row_stride =
 * H_total * 128), so each finished tile crosses NVLink as it is stored and no all-gather follows; the caller
 * orders the peers' reads after a cross-GPU barrier.  Replaces Attention.forward (attention.py:59-77) followed by
 * the gather of the heads. */
int specdec_paged_attention_multi(const void* q, long long T, long long q_row_stride, int num_heads,
                                  int num_kv_heads, int head_dim, const void* k_cache, const void* v_cache,
                                  long long num_slots, int block_size, const int* cu_seqlens_q,
                                  const int* cu_seqlens_k, const int* context_lens, int q_per_seq, int R,
                                  const int* block_tables, int W, int max_seqlen_q, float softmax_scale, int causal,
                                  void* const* outs, int num_outs, long long out_row_stride, void* workspace,
                                  long long workspace_bytes, int* err, unsigned flags, void* stream);

/* Cross-GPU barrier of the peer-store tensor-parallel verify attention (the step that replaces the all-gather of
 * the heads after Attention.forward, nanovllm/layers/attention.py:59-77, under the head split of
 * nanovllm/models/qwen3.py:29-35).  flags: HOST array of `world` device addresses, flags[t] = rank t's array of 8
 * uint32 arrival words (peer memory mapped into this process; all zero before the first barrier of a group);
 * epoch: this rank's uint32 counter in device memory (zero at first, advanced by the kernel, so a captured
 * launch replays correctly).  One block signals every rank (system-scope release after a system fence) and
 * waits for every rank's signal of the same epoch; a wait past timeout_ns sets *err = 21 and returns (this rank's
 * epoch has still advanced, so the group's epochs may now disagree: treat 21 as fatal for the group and zero
 * every flag array and epoch, with no barrier in flight, before using it again).  Every
 * rank must call it the same number of times, each on its own GPU: barriers of several ranks never share one
 * GPU (nothing makes separate launches run concurrently). */
int specdec_peer_barrier(void* const* flags, int world, int rank, unsigned* epoch, long long timeout_ns, int* err,
                         void* stream);

/* ------------------------------------------------------------------------------------------ kernel 3: Markov rows */
/* One row step of DFlashDrafter._markov_rows (nanovllm/engine/speculative.py:163-184) for every batch row: with
 * row_logits = logits[:, row] + bias (bias = markov_head(prev), [B, V]; rounded to bf16 when round_bf16):
 * greedy -> argmax; else the top `candidates` values (ties by ascending token id), probs_from_logits over them
 * with per-row temperature / top_k / top_p (spec_sampler.py:65-96), race against noise[b, row, :candidates]
 * (noise [B, k, noise_width]), q scattered into probs [B, k, V] (zeroed by the caller once per call).  Writes
 * drafts[b, row], prev_out[b] and, with w1 [V, rank] bf16, e_next[b] = w1[prev] (the next step's embedding).
 * logits [B, k, V] and bias of dtype codes as above.  Limits: candidates <= 1024.  Each row is split over several
 * CTAs; workspace: 256-byte aligned device bytes, zero-filled once before first use (the kernel leaves its
 * counters zeroed), at least specdec_markov_workspace_bytes(B, V, candidates, greedy); calls sharing it must not
 * overlap on the GPU.  last_ids (int32 [B, k, candidates], or null): with it, probs is a persistent buffer that
 * is zero except where this row scattered q on the previous call, listed in last_ids (-1 = none; all -1 and a
 * zeroed probs at first use); those entries are cleared and the new ids recorded, so the caller need not zero
 * the [B, k, V] probs (the reference's speculative.py:170-171 zero-fill) every call.  bias null: logits is this
 * step's already biased rows, [B, V] (as specdec_markov_bias writes them), and round_bf16 applies to nothing. */
long long specdec_markov_workspace_bytes(int B, int V, int candidates, int greedy);
int specdec_markov_step(const void* logits, int logits_dtype, const void* bias, int bias_dtype, int B, int k, int V,
                        int row, int candidates, int greedy, int round_bf16, const float* temperature,
                        const long long* top_k, const float* top_p, int max_top_k, int has_top_p, const float* noise,
                        int noise_width, long long* drafts, float* probs, long long* prev_out, const void* w1,
                        int rank, void* e_next, int* last_ids, void* workspace, long long workspace_bytes, int* err,
                        void* stream);

/* ------------------------------------------------------------------------------------------ kernel 4: ctx_store */
/* DFlashDraftModel.store_context_kv (nanovllm/models/dflash.py:88-96) for every draft layer in one launch, and
 * the target's q_norm / k_norm + RoPE + store_kvcache (nanovllm/models/qwen3.py:77-86, attention.py:62-63).
 * x [layers][T][(Hq + 2 Hkv) * 128] bf16 (layer / row strides in elements): Hq query heads, then Hkv K heads,
 * then Hkv V heads.  Query heads: RMSNorm(q_norm [128]) then RoPE -> q_out [T][Hq][128].  K heads:
 * RMSNorm(k_norm [layer][128]) then RoPE -> k_cache[layer][slot]; V heads copied to v_cache[layer][slot]; caches
 * [layers][num_slots][Hkv][128] (layer stride in elements).  cos_sin [max_position][128] fp32 (cos | sin);
 * positions [T] int64; slot_mapping [T] int32 (-1 skipped).  Out-of-range positions / slots are skipped and
 * recorded in *err. */
int specdec_norm_rope_store(const void* x, long long x_layer_stride, long long x_row_stride, int T, int layers,
                            int num_q_heads, int num_kv_heads, const void* q_norm, const void* k_norm,
                            long long k_norm_layer_stride, const float* cos_sin, long long max_position,
                            const long long* positions, const int* slot_mapping, void* k_cache, void* v_cache,
                            long long cache_layer_stride, long long num_slots, void* q_out, float eps, int* err,
                            void* stream);

/* ------------------------------------------------------------------------------------------ kernel 5: context GEMM */
/* The draft context path's projections (nanovllm/models/dflash.py:84-96: fc in context_features, the per-layer
 * W_kv of store_context_kv) on the tensor cores: out[T, O] = x[T, K] . w[O, K]^T, bf16 operands and output (one
 * rounding of the fp32 sum), row strides in elements (16-byte multiples).  1 <= T <= 288 tokens per call,
 * O a multiple of 128, K a multiple of 64.  workspace: 256-byte aligned device bytes, zero-filled once before
 * first use (the kernel leaves its counters zeroed), at least specdec_context_gemm_workspace_bytes(T, O); calls
 * that share a workspace must not overlap on the GPU.  Waits that run out record a code in *err. */
long long specdec_context_gemm_workspace_bytes(int T, int O);
int specdec_context_gemm(const void* x, long long x_row_stride, const void* w, long long w_row_stride, int T, int O,
                         int K, void* out, long long out_row_stride, void* workspace, long long workspace_bytes,
                         int* err, void* stream);
/* DSpark's biased row (nanovllm/engine/speculative.py:173 with MarkovHead, nanovllm/models/dflash.py:39-41):
 * out[b, v] = bf16(bf16(sum_r e[b, r] * w2[v, r]) + logits[b, v]) for b < B, the rank-`rank` Markov bias of the
 * previous tokens' embeddings e [B, rank] (markov_w1 rows) against markov_w2 [V, rank], added to this step's logits
 * rows in the same tensor-core GEMM's epilogue, so the bias never reaches memory; the biased rows go straight to
 * specdec_markov_step with a null bias.  bf16 throughout, row strides in elements (16-byte multiples for e and
 * w2); B <= 288, V a multiple of 128, rank a multiple of 64.  Workspace as for specdec_context_gemm with
 * T = B, O = V. */
int specdec_markov_bias(const void* w2, long long w2_row_stride, const void* e, long long e_row_stride, int B, int V,
                        int rank, const void* logits, long long logits_row_stride, void* out,
                        long long out_row_stride, void* workspace, long long workspace_bytes, int* err,
                        void* stream);
/* DFlashDraftModel.store_context_kv (dflash.py:88-96) fused: the same GEMM against the layers' stacked W_kv
 * ([layers * 2 * Hkv * 128, K]: per layer its K rows then its V rows) with the projection never leaving the chip:
 * each 128-row tile is one (layer, K|V, head); K rows get RMSNorm (k_norm [layers, 128], layer stride in
 * elements) and RoPE at positions[t] (cos_sin [max_position, 128]: cos | sin), and every row is stored at slot
 * slot_mapping[t] of k_cache / v_cache ([layers][num_slots][Hkv][128], layer stride in elements; slot -1
 * skipped).  A position or slot out of range is skipped and recorded in *err (4, 3).  Workspace as for
 * specdec_context_gemm with O = layers * 2 * Hkv * 128. */
int specdec_context_kv_store(const void* x, long long x_row_stride, const void* w_kv, long long w_row_stride, int T,
                             int layers, int num_kv_heads, int K, const void* k_norm, long long k_norm_layer_stride,
                             const float* cos_sin, long long max_position, const long long* positions,
                             const int* slot_mapping, void* k_cache, void* v_cache, long long cache_layer_stride,
                             long long num_slots, float eps, void* workspace, long long workspace_bytes, int* err,
                             void* stream);

/* ------------------------------------------------------------------------------------------ verify forward helpers */
/* RMSNorm.rms_forward / add_rms_forward (nanovllm/layers/layernorm.py:16-40): rows of `width` bf16 (a multiple of
 * 8, <= 8192).  With residual: s = x + residual, residual_out = s, out = norm(s) * weight; else out = norm(x). */
int specdec_rmsnorm(const void* x, const void* residual, const void* weight, void* out, void* residual_out,
                    long long T, int width, float eps, void* stream);

/* SiluAndMul (nanovllm/layers/activation.py:8-11): gate_up [T, 2 I] bf16 -> out [T, I] = silu(gate) * up. */
int specdec_silu_mul(const void* gate_up, void* out, long long T, int intermediate, void* stream);

#ifdef __cplusplus
}  /* extern "C" */
#endif

#endif  /* SPECDEC_B200_H_ */
