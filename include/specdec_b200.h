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
const char* specdec_last_error(void);
int specdec_version(void);
/* 1 when the current CUDA device is compute capability 10.0 (the only target of this build). */
int specdec_device_supported(void);

/* ------------------------------------------------------------------------------------------ kernel 1: sampler */
/* Workspace bytes for the sampler entry points over `rows` rows of logits / probabilities. */
size_t specdec_sampler_workspace_bytes(long long rows);

/* Philox offset increment torch's CUDA generator consumes for one torch.rand / exponential_ draw of `numel`
 * floats on the current device (ATen's calc_execution_policy); callers advance their generator by it. */
unsigned long long specdec_philox_increment(long long numel);

/* probs_from_logits (nanovllm/layers/spec_sampler.py:65-69, truncate_logits :72-96).
 * logits [R, V] (dtype), parameter row of logits row r = r / rows_per_param; temperature [R/rows_per_param]
 * fp32 > 0; top_k int64 (required when max_top_k > 0, 0 = no truncation for that row); top_p fp32 (required
 * when has_top_p).  probs [R, V] fp32 = softmax(mask(logits / T)). */
int specdec_probs(const void* logits, int dtype, long long R, long long V, long long rows_per_param,
                  const float* temperature, const long long* top_k, const float* top_p, int max_top_k,
                  int has_top_p, float* probs, void* workspace, size_t workspace_bytes, void* stream);

/* accept_random / accept_random_varlen (spec_sampler.py:114-150), and with x_is_probs = 0 the round driver's
 * fused probs_from_logits + accept (nanovllm/engine/speculative.py:450-462).
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

#ifdef __cplusplus
}  /* extern "C" */
#endif

#endif  /* SPECDEC_B200_H_ */
