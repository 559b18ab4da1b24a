// Kernel (1): the batched speculative sampler ("SpecSampler") for sm_100a.
//
// Reference behaviour restated here (nano-vllm-speculative-decoding, nanovllm/layers/spec_sampler.py):
//   probs_from_logits / truncate_logits   :65-96   softmax(mask(logits.float() / T)), HF top-k (ties kept) then
//                                                  top-p over the softmax of the top-k candidates
//   exponential_noise_ / race / sample    :99-111  argmax(w / clamp_min(Exp(1), 1e-10)), first index on ties
//   accept_random[_varlen]                :114-150 u * q_d < p_d & verified; prefix length; residual (p - q)+ at
//                                                  the first rejection or the bonus row; tail by the race
//   accept_greedy[_varlen]                :153-169 argmax match prefix; tail = argmax at start + n_accept
//   _verified_positions                   :172-180 starts = exclusive cumsum(lens); positions clamped to the
//                                                  bonus position; verified = j < len - 1
//
// Design (B200): the path is HBM-bound integer/float streaming, so it never touches the tensor cores.
//   pass 1  (stats)  early exit (stats_early_kernel, whenever the requests fit one wave): one thread-block
//                    cluster per request walks its verified rows in order, a chunk per CTA, meets each row's
//                    partial (max, sum) pairs in distributed shared memory and takes the accept test there, and
//                    stops at the first rejected draft - the later rows are never read.  Otherwise grid
//                    (chunks x rows): every verified row is read once with 16-byte loads and reduced to a
//                    partial per chunk; the last CTA of a request (an atomic ticket) merges the partials and
//                    decides the accepted prefix.  Rows that truncate (top_k > 0) are handled by one 512-thread
//                    CTA per row that radix-selects the k-th value over L2-resident re-reads.
//   pass 2  (tail)   the race over the request's tail row (bonus p or residual (p - q)+) against torch's
//                    exact Exp(1) draws, regenerated in-kernel (Philox4x32-10 at torch's counters and grid,
//                    torch's __logf transform, clamp at 1e-10), so the [B, V] noise is never read from HBM as
//                    floats: with room in the workspace the draws are first kept as 16-bit codes that bound each
//                    one (noise_codes_kernel, beside the early-exit pass) and the race streams the rows and codes,
//                    drawing exactly only the elements that can still win (tail_codes_kernel); without it every
//                    element is drawn in place (tail_accept_kernel).  The ratio w / E, an argmax key per request
//                    (first index on ties), one 64-bit atomicMax per request and warp run; the last CTA writes the
//                    tail tokens.
// Explicit u / E pointers replace the in-kernel draws (parity mode) without changing anything else.
#include "common.cuh"

#include <curand_kernel.h>
#include <math.h>

namespace specdec {
namespace sampler {

constexpr int kThreads = 256;        // stats / tail / greedy CTAs
constexpr int kTopkThreads = 512;    // one CTA per truncating row
constexpr int kStatsCtasPerSm = 4;   // stats_kernel residency its launch bounds guarantee (<= 64 registers)
constexpr int kGreedyCtasPerSm = 8;  // greedy_kernel residency its launch bounds guarantee (<= 32 registers)
constexpr int kMaxRequests = 1024;   // B cap (shared-memory tables are sized by it)
constexpr int kMaxRows = 16384;      // T cap (fixed-offset greedy key table)
constexpr int kMaxChunks = 64;       // chunks per row in pass 1
constexpr int kKeptCap = kTopkThreads; // ids of a truncated row's kept tokens recorded for the candidate tail race
constexpr int kMaxTopK = 1024;       // top_k cap of the in-kernel radix select
constexpr int kRngBlock = 256;       // torch's block_size_bound for distribution kernels

// Device-side input checks (the host cannot see verified_lens or drafts without a sync).  A failing check makes
// every kernel of the call return before touching memory it cannot bound, and leaves the code in the status word.
constexpr int kStatusBadLens = 1;     // a length outside 1..k+1, or lengths not summing to T
constexpr int kStatusBadDraft = 2;    // a draft id outside [0, V)
constexpr int kStatusBadTopK = 3;     // a row's top_k above the in-kernel cap

struct RowStat {   // per verified row: softmax max / sum over the kept entries, truncation threshold
  float m, s, thr, pad;
};
struct ReqDesc {   // per request: where its tail distribution lives
  long long x_row;   // flat row of x holding p_next
  long long q_row;   // flat row of q for the residual, or -1 for the bonus row / plain race
  float m, s, thr, temp;
};

// ---------------------------------------------------------------------------------------- workspace layout
// Self-cleaning tables (tickets, argmax keys) sit at fixed offsets at the front, so a workspace zeroed once at
// allocation stays valid across calls of any shape; per-call scratch follows.
struct Layout {
  size_t status, req_ticket, tail_key, tail_ticket, row_key, rows, partial, desc, kept_n, kept_ids, total;
};
static constexpr Layout layout(int64_t T) {
  Layout L{};
  size_t off = 0;
  auto take = [&off](size_t bytes) {
    size_t o = off;
    off += (bytes + 255) & ~size_t(255);
    return o;
  };
  L.status = take(256);
  L.req_ticket = take(sizeof(unsigned) * kMaxRequests);
  L.tail_key = take(sizeof(unsigned long long) * kMaxRequests);
  L.tail_ticket = take(256);
  L.row_key = take(sizeof(unsigned long long) * kMaxRows);
  L.rows = take(sizeof(RowStat) * (size_t)(T > 0 ? T : 1));
  L.partial = take(sizeof(float2) * (size_t)(T > 0 ? T : 1) * kMaxChunks);
  L.desc = take(sizeof(ReqDesc) * kMaxRequests);
  L.kept_n = take(sizeof(int) * (size_t)(T > 0 ? T : 1));
  L.kept_ids = take(sizeof(int) * (size_t)(T > 0 ? T : 1) * kKeptCap);
  L.total = off;
  return L;
}

struct Args {
  // inputs
  const void* x;            // [T, V] logits (dtype) or fp32 probabilities (probs_mode)
  long long T, V;
  int dtype, probs_mode;
  const float* q;           // [B, k, V] fp32 draft probabilities (may be null for greedy / race)
  const long long* drafts;  // [B, k]
  int B, k;
  const long long* lens;    // [B] verified lengths, or null = k + 1 each
  int rows_per_param;       // probs-only calls: parameter row of x row t is t / rows_per_param
  const float* temperature; // [B] (or [params]); null only in probs_mode / greedy
  const long long* top_k;   // [B] or null
  const float* top_p;       // [B] or null
  int has_top_p, truncate;  // host flags: some row has top_p < 1; max_top_k > 0
  const float* u;           // [B, k] uniforms or null (then drawn in-kernel)
  const float* E;           // [B, V] exponential noise or null (then drawn in-kernel)
  unsigned long long seed, offset_u, offset_E;
  // outputs
  long long* n_accept;      // [B]
  long long* tail;          // [B]
  float* probs_out;         // [T, V] for specdec_probs
  // layout
  int C, chunk, vec_ok;
  int u_grid;               // torch grid (blocks of 256) of the [B, k] uniform draw
  int e_grid, e_rounds;     // torch grid and grid-stride rounds of the [B, V] exponential draw
  long long e_numel;
  unsigned e_sq, e_sr;      // S / V and S % V for S = 256 * e_grid (incremental row tracking)
  // workspace
  int* status;              // [0] device-side input check: 0 ok, else a kStatus* code (first writer wins);
                            // [1] set when some request's tail row has no recorded kept set (full-row race)
  int tail_gate;            // tail_accept_kernel runs only if status[1] is set (truncating calls)
  unsigned* req_ticket;
  unsigned long long* tail_key;
  unsigned* tail_ticket;
  unsigned long long* row_key;
  RowStat* rows;
  float2* partial;
  ReqDesc* desc;
  int* kept_n;              // [T] tokens a truncated row keeps (ids in kept_ids), or -1: not recorded
  int* kept_ids;            // [T][kKeptCap]
  unsigned short* codes;    // [B, V] 16-bit codes of the tail noise (noise_codes_kernel), or null
  int codes_vec;            // tail rows, q rows and code rows are 16-byte aligned with V % 8 == 0
};

// ---------------------------------------------------------------------------------------- small helpers
__device__ __forceinline__ float scale_logit(float x, float temp) {
  // logits.float() / T, IEEE division (temperature 1 is the identity, as in fp32 division).
  return __fdiv_rn(x, temp);
}

// torch.rand's transform of a curand_uniform4 lane: (0, 1] with 1 mapped to 0.
__device__ __forceinline__ float torch_uniform(float r) { return r == 1.0f ? 0.0f : r; }

// torch's CUDA exponential_(lambda = 1) transform of a curand_uniform4 lane, then clamp_min(1e-10).  ATen takes the
// logarithm with the fast __logf intrinsic on the device (at::log in ATen/NumericUtils.h), so this does too: the
// accurate logf differs by up to ~5e-8 near r = 1, where the smallest draws (the likeliest race winners) sit.
__device__ __forceinline__ float torch_exponential_clamped(float r) {
  const float eps_half = 5.9604644775390625e-08f;  // numeric_limits<float>::epsilon() / 2
  float lg = (r >= 1.0f - eps_half) ? -eps_half : __logf(r);
  float e = -1.0f * lg;
  const float floor_v = 1e-10f;
  return e < floor_v ? floor_v : e;
}

// The four uniforms of call n of curand's Philox4x32-10 stream (seed, subsequence idx, offset 4 c0): the Philox
// block (Salmon et al., SC 2011) at counter (c0 + n, idx) under key seed, computed by curand's own block function
// and uniform transform, without the state bookkeeping of curand_uniform4.
__device__ __forceinline__ float4 philox_uniform4(unsigned long long seed, unsigned long long c0, unsigned idx,
                                                  int n) {
  const unsigned long long c = c0 + (unsigned long long)n;
  const uint4 ctr = make_uint4((unsigned)c, (unsigned)(c >> 32), idx, 0u);
  const uint2 key = make_uint2((unsigned)seed, (unsigned)(seed >> 32));
  return _curand_uniform4(curand_Philox4x32_10(ctr, key));
}

// Code of one uniform r in (0, 1] of the exponential draw: E = torch's transform of r lies in [lo, hi), lo = code
// << 16 and hi = (code + 1) << 16 read as floats.
__device__ __forceinline__ unsigned short noise_code(float r) {
  return static_cast<unsigned short>(__float_as_uint(torch_exponential_clamped(r)) >> 16);
}

// Uniform number li of a torch.rand draw of `numel` floats whose grid has `grid` blocks of 256 threads.
__device__ float torch_rand_at(unsigned long long seed, unsigned long long offset, long long li, int grid) {
  const long long S = (long long)kRngBlock * grid;
  const long long idx = li % S;
  const long long m = li / S;       // grid-stride step: round m / 4, lane m % 4 of curand_uniform4
  curandStatePhilox4_32_10_t st;
  curand_init(seed, (unsigned long long)idx, offset + 4ull * (unsigned long long)(m / 4), &st);
  float4 r = curand_uniform4(&st);
  const int lane = (int)(m & 3);
  float v = lane == 0 ? r.x : lane == 1 ? r.y : lane == 2 ? r.z : r.w;
  return torch_uniform(v);
}

// Exclusive prefix sums of the verified lengths into s_start[0..B] (s_start[B] = T).  Returns false (in every
// thread) when a length is outside 1..k1 or the lengths do not sum to T.
template <int NT>
__device__ bool starts_from_lens(const long long* lens, int B, int k1, long long T, int* s_start) {
  constexpr int PER = (kMaxRequests + NT - 1) / NT;
  __shared__ int warp_tot[NT / 32];
  __shared__ int s_bad;
  if (threadIdx.x == 0) s_bad = 0;
  __syncthreads();
  int vals[PER];
  int local = 0;
  const int base = threadIdx.x * PER;
#pragma unroll
  for (int i = 0; i < PER; ++i) {
    int idx = base + i;
    int v = 0;
    if (idx < B) {
      long long raw = lens ? lens[idx] : k1;
      if (raw < 1 || raw > k1) { s_bad = 1; raw = 1; }
      v = (int)raw;
    }
    vals[i] = v;
    local += v;
  }
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int incl = local;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    int n = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += n;
  }
  if (lane == 31) warp_tot[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    int w = lane < NT / 32 ? warp_tot[lane] : 0;
    int wi = w;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      int n = __shfl_up_sync(0xffffffffu, wi, o);
      if (lane >= o) wi += n;
    }
    if (lane < NT / 32) warp_tot[lane] = wi - w;
  }
  __syncthreads();
  int run = warp_tot[warp] + incl - local;
#pragma unroll
  for (int i = 0; i < PER; ++i) {
    int idx = base + i;
    if (idx < B) {
      s_start[idx] = run;
      run += vals[i];
      if (idx == B - 1) s_start[B] = run;
    }
  }
  __syncthreads();
  return s_bad == 0 && s_start[B] == T;
}

__device__ __forceinline__ void report(const Args& a, int code) { atomicCAS(a.status, 0, code); }

// Request holding flat row t: s_start[b] <= t < s_start[b + 1].
__device__ __forceinline__ int request_of_row(const int* s_start, int B, int t) {
  int lo = 0, hi = B - 1;
  while (lo < hi) {
    int mid = (lo + hi + 1) >> 1;
    if (s_start[mid] <= t) lo = mid; else hi = mid - 1;
  }
  return lo;
}

__device__ __forceinline__ void ms_combine(float& m, float& s, float m2, float s2) {
  if (m2 == -INFINITY) return;
  if (m == -INFINITY) { m = m2; s = s2; return; }
  if (m2 > m) { s = s * expf(m - m2) + s2; m = m2; }
  else { s = s + s2 * expf(m2 - m); }
}

// Block-wide (max, sum) combine; result valid in every thread.
template <int NT>
__device__ void block_ms(float& m, float& s) {
  __shared__ float sm_m[NT / 32], sm_s[NT / 32];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    float m2 = __shfl_xor_sync(0xffffffffu, m, o);
    float s2 = __shfl_xor_sync(0xffffffffu, s, o);
    ms_combine(m, s, m2, s2);
  }
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  __syncthreads();
  if (lane == 0) { sm_m[warp] = m; sm_s[warp] = s; }
  __syncthreads();
  m = sm_m[0];
  s = sm_s[0];
  for (int w = 1; w < NT / 32; ++w) ms_combine(m, s, sm_m[w], sm_s[w]);
  __syncthreads();
}

// exp(x) for the softmax normaliser sums: the hardware ex2 of x * log2(e).  The sum's order already differs
// from ATen's; this adds ~1e-7 relative error per term, far inside the 1e-5 probability tolerance and the 1e-6
// decision flags.  Per-element probabilities that decide tokens use the accurate expf.
__device__ __forceinline__ float exp_sum_term(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x * 1.4426950408889634f));
  return y;
}

// Online (max, sum of exp) over elements [lo, hi) of one row of scaled logits.
template <typename T, int NT>
__device__ void row_range_ms(const T* row, int lo, int hi, float temp, int vec_ok, float& m, float& s) {
  m = -INFINITY;
  s = 0.0f;
  constexpr int VE = 16 / sizeof(T);  // elements per 16-byte vector
  const bool unit_temp = temp == 1.0f;
  if (vec_ok) {
    // lo is a multiple of VE and the row base is 16-byte aligned.  Four 16-byte vectors per batch, the next
    // batch's loads in flight while this one is reduced: the batch maximum first (one rescale of the running
    // sum), then exp2(x * log2e - m * log2e) per element; vectors are unpacked where they are used.
    const int nvec = (hi - lo) / VE;
    const char* base = reinterpret_cast<const char*>(row + lo);
    const float kLog2e = 1.4426950408889634f;
    // -inf in every element of a vector past the range (f32 0xff800000, bf16 0xff80, f16 0xfc00)
    constexpr unsigned kNegInfWord = sizeof(T) == 4 ? 0xff800000u
                                   : std::is_same<T, __nv_bfloat16>::value ? 0xff80ff80u : 0xfc00fc00u;
    const uint4 kNegInf = make_uint4(kNegInfWord, kNegInfWord, kNegInfWord, kNegInfWord);
    auto load_batch = [&](int i, uint4 (&r)[4]) {
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int j = i + u * NT;
        r[u] = j < nvec ? ldg16(base + (size_t)j * 16) : kNegInf;
      }
    };
    auto unpack = [&](const uint4& r, float (&f)[VE]) {
      if constexpr (sizeof(T) == 4) {
        unpack16(r, f);
      } else if constexpr (std::is_same<T, __nv_bfloat16>::value) {
        unpack16_bf16(r, f);
      } else {
        unpack16_f16(r, f);
      }
#pragma unroll
      for (int e = 0; e < VE; ++e)
        if (!unit_temp) f[e] = scale_logit(f[e], temp);
    };
    uint4 cur[4];
    if ((int)threadIdx.x < nvec) load_batch(threadIdx.x, cur);
    for (int i = threadIdx.x; i < nvec; i += NT * 4) {
      uint4 nxt[4];
      const int inext = i + NT * 4;
      if (inext < nvec) load_batch(inext, nxt);
      float vm = -INFINITY;
      if constexpr (sizeof(T) == 2) {
        // the batch maximum on packed pairs (exact; NaN dropped as fmaxf does), then scaled once: x / T is
        // monotone in x, so max(x) / T is the maximum of the scaled values
        using H2 = typename std::conditional<std::is_same<T, __half>::value, __half2, __nv_bfloat162>::type;
        H2 mx2 = group_max_h2<H2>(cur[0]);
#pragma unroll
        for (int u = 1; u < 4; ++u) mx2 = __hmax2(mx2, group_max_h2<H2>(cur[u]));
        vm = fmaxf(__low2float(mx2), __high2float(mx2));
        if (!unit_temp) vm = scale_logit(vm, temp);
      } else {
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          float f[VE];
          unpack(cur[u], f);
#pragma unroll
          for (int e = 0; e < VE; ++e) vm = fmaxf(vm, f[e]);
        }
      }
      if (vm > m) {
        if (m != -INFINITY) s *= exp_sum_term(m - vm);
        m = vm;
      }
      if (m != -INFINITY) {
        const float mb = m * kLog2e;
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          float f[VE];
          unpack(cur[u], f);
#pragma unroll
          for (int e = 0; e < VE; ++e) {
            float y;
            asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(fmaf(f[e], kLog2e, -mb)));
            s += y;
          }
        }
      }
#pragma unroll
      for (int u = 0; u < 4; ++u) cur[u] = nxt[u];
    }
    // scalar tail of the range (fewer than VE elements)
    for (int v = lo + nvec * VE + threadIdx.x; v < hi; v += NT) {
      float f = to_f32(row[v]);
      if (!unit_temp) f = scale_logit(f, temp);
      if (f > m) {
        if (m != -INFINITY) s *= exp_sum_term(m - f);
        m = f;
      }
      if (m != -INFINITY) s += exp_sum_term(f - m);
    }
  } else {
    for (int v = lo + threadIdx.x; v < hi; v += NT) {
      float f = to_f32(row[v]);
      if (!unit_temp) f = scale_logit(f, temp);
      if (f > m) {
        if (m != -INFINITY) s *= exp_sum_term(m - f);
        m = f;
      }
      if (m != -INFINITY) s += exp_sum_term(f - m);
    }
  }
}

// p of one scaled logit f under row stats (masked entries give 0), exp(f - m) / s as ATen's softmax.
__device__ __forceinline__ float prob_of_scaled(float f, const RowStat& r) {
  return f >= r.thr ? __fdiv_rn(expf(f - r.m), r.s) : 0.0f;
}

template <typename T>
__device__ __forceinline__ float prob_at(const Args& a, long long row, long long col, const RowStat& rs, float temp) {
  float xv = to_f32(reinterpret_cast<const T*>(a.x)[row * a.V + col]);
  if (a.probs_mode) return xv;
  float f = temp == 1.0f ? xv : scale_logit(xv, temp);
  return prob_of_scaled(f, rs);
}

// Merges the chunk partials of row t (one warp); the result is valid in every lane.
__device__ RowStat merge_row_warp(const Args& a, int t) {
  const int lane = threadIdx.x & 31;
  float m = -INFINITY, s = 0.0f;
  for (int c = lane; c < a.C; c += 32) {
    float2 p = __ldcg(&a.partial[(size_t)t * kMaxChunks + c]);
    ms_combine(m, s, p.x, p.y);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    float m2 = __shfl_xor_sync(0xffffffffu, m, o);
    float s2 = __shfl_xor_sync(0xffffffffu, s, o);
    ms_combine(m, s, m2, s2);
  }
  RowStat r;
  r.m = m; r.s = s; r.thr = -INFINITY; r.pad = 0.0f;
  return r;
}

// Acceptance of request b once every one of its rows has final stats (run by a whole CTA).  need_merge: the
// rows' stats are still chunk partials, merged here into a.rows.  k <= 32 (one lane per draft).
template <typename T>
__device__ void decide_request(const Args& a, int b, int start, int len, bool need_merge) {
  __shared__ RowStat s_rows[33];
  const int warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5, lane = threadIdx.x & 31;
  if (!a.probs_mode) {
    for (int r = warp; r < len; r += nwarps) {
      RowStat rs;
      if (need_merge) {
        rs = merge_row_warp(a, start + r);
        if (lane == 0) a.rows[start + r] = rs;
      } else {
        float4 raw = __ldcg(reinterpret_cast<const float4*>(&a.rows[start + r]));
        rs.m = raw.x; rs.s = raw.y; rs.thr = raw.z; rs.pad = raw.w;
      }
      if (lane == 0) s_rows[r] = rs;
    }
  }
  __syncthreads();
  if (warp != 0) return;
  const float temp = a.probs_mode ? 1.0f : a.temperature[b];
  const RowStat identity{0.f, 1.f, -INFINITY, 0.f};
  bool accepted = false;
  const int j = lane;
  if (j < a.k) {
    const bool verified = j < len - 1;
    const int r = verified ? j : len - 1;
    const long long d = a.drafts[(long long)b * a.k + j];
    const long long li = (long long)b * a.k + j;
    const float u = a.u ? a.u[li] : torch_rand_at(a.seed, a.offset_u, li, a.u_grid);
    if (d < 0 || d >= a.V) {
      report(a, kStatusBadDraft);
    } else {
      const RowStat rs = a.probs_mode ? identity : s_rows[r];
      const float p_d = prob_at<T>(a, start + r, d, rs, temp);
      const float q_d = a.q[((long long)b * a.k + j) * a.V + d];
      accepted = (u * q_d < p_d) && verified;   // u < min(1, p/q) without dividing
    }
  }
  const unsigned acc_mask = __ballot_sync(0xffffffffu, accepted);
  // length of the accepted prefix: the trailing ones (lanes >= k never accept)
  const int n_acc = (~acc_mask) ? __ffs(~acc_mask) - 1 : 32;
  if (lane == 0) {
    a.n_accept[b] = n_acc;
    ReqDesc d;
    d.x_row = start + n_acc;
    d.q_row = (n_acc == len - 1) ? -1 : ((long long)b * a.k + (n_acc < a.k - 1 ? n_acc : a.k - 1));
    const RowStat rs = a.probs_mode ? identity : s_rows[n_acc];
    d.m = rs.m; d.s = rs.s; d.thr = rs.thr; d.temp = temp;
    a.desc[b] = d;
    // the tail row's kept set (written by its CTA before that CTA's ticket) decides which tail kernel races
    if (a.truncate && __ldcg(&a.kept_n[d.x_row]) < 0) atomicExch(a.status + 1, 1);
  }
}

// ---------------------------------------------------------------------------------------- pass 1: stats
// grid (C, T).  mode 0: acceptance (decide when the request's last chunk lands); mode 1: probabilities only.
template <typename T>
__global__ void __launch_bounds__(kThreads, kStatsCtasPerSm) stats_kernel(Args a, int mode) {
  __shared__ int s_start[kMaxRequests + 1];
  __shared__ int s_last;
  const int c = blockIdx.x, t = blockIdx.y;
  int b, start, len;
  float temp;
  if (mode == 0 && a.lens == nullptr) {        // every request verifies k + 1 rows (checked on the host)
    b = t / (a.k + 1);
    start = b * (a.k + 1);
    len = a.k + 1;
    temp = a.temperature[b];
  } else if (mode == 0) {
    if (!starts_from_lens<kThreads>(a.lens, a.B, a.k + 1, a.T, s_start)) {
      if (threadIdx.x == 0) report(a, kStatusBadLens);
      return;
    }
    b = request_of_row(s_start, a.B, t);
    start = s_start[b];
    len = s_start[b + 1] - start;
    temp = a.temperature[b];
  } else {
    b = t / a.rows_per_param;
    start = 0; len = 0;
    temp = a.temperature[b];
  }
  const int lo = c * a.chunk;
  const int hi = min((long long)lo + a.chunk, a.V);
  const T* row = reinterpret_cast<const T*>(a.x) + (long long)t * a.V;
  float m, s;
  row_range_ms<T, kThreads>(row, lo, hi, temp, a.vec_ok, m, s);
  block_ms<kThreads>(m, s);
  if (threadIdx.x == 0) a.partial[(size_t)t * kMaxChunks + c] = make_float2(m, s);
  if (mode != 0) return;
  // last CTA of request b decides its acceptance
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) {
    unsigned ticket = atomicAdd(&a.req_ticket[b], 1u);
    s_last = ticket == (unsigned)(len * a.C - 1);
  }
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  decide_request<T>(a, b, start, len, true);
  if (threadIdx.x == 0) atomicExch(&a.req_ticket[b], 0u);
}

// ---------------------------------------------------------------------------------------- pass 1, early exit
// The accept test walks a request's drafts in order and stops at the first rejection (spec_sampler.py:142-147),
// so the rows after it never matter.  Grid (C, B) in thread-block clusters of C: the C CTAs of request b stream
// its rows in order, chunk c of each; a row's C partial (max, sum) pairs meet in distributed shared memory at a
// cluster barrier, every CTA merges them in the same order and takes the draft's accept test itself (the same
// inputs and arithmetic, so the same outcome), and at the first rejection, or at the last verified row, chunk 0
// writes the request's result.  The cluster's CTAs are co-scheduled by the hardware; nothing waits on memory.
constexpr int kEarlyCtasPerSm = 3;   // the walk's decision code beside the streaming loop: up to 85 registers
constexpr int kEarlyMaxCluster = 8;  // portable cluster size
constexpr int kNoiseCtasPerSm = 4;   // the noise codes kernel beside the early-exit pass: CTAs per SM

// Barrier over every thread of the cluster; the release / acquire pair makes each CTA's shared-memory writes
// before it visible to the cluster's reads after it.
__device__ __forceinline__ void cluster_barrier() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// The float2 at `local`'s offset in the shared memory of the cluster's CTA `rank`.
__device__ __forceinline__ float2 ld_cluster_f2(const float2* local, unsigned rank) {
  const unsigned addr = static_cast<unsigned>(__cvta_generic_to_shared(local));
  unsigned remote;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(addr), "r"(rank));
  float2 v;
  asm volatile("ld.shared::cluster.v2.f32 {%0, %1}, [%2];" : "=f"(v.x), "=f"(v.y) : "r"(remote) : "memory");
  return v;
}

// Rows per step after the first: the largest divisor of the cluster size C not above the rows left (at least 1).
__device__ __forceinline__ int early_rows_per_step(int C, int left) {
  int k = 1;
  for (int d = 2; d <= C; ++d)
    if (C % d == 0 && d <= left) k = d;
  return k;
}

template <typename T>
__global__ void __launch_bounds__(kThreads, kEarlyCtasPerSm) stats_early_kernel(Args a) {
  __shared__ int s_start[kMaxRequests + 1];
  __shared__ int s_flag;      // 0 go on, 1 the request is decided, 2 a bad draft id
  __shared__ RowStat s_rs;
  __shared__ float2 s_part;   // this CTA's (max, sum) of the current row, read by the whole cluster
  // the walk's state lives in shared memory, so that no register holds it across the streaming loop
  __shared__ int s_j, s_row0, s_len, s_k;
  __shared__ float s_temp;
  __shared__ float s_u[32], s_q[32], s_x[32];   // per draft: its uniform, q and target logit (loaded up front)
  const int b = blockIdx.y;
  griddep_launch_dependents();   // the noise codes kernel may start beside the walk
  if (a.lens != nullptr && !starts_from_lens<kThreads>(a.lens, a.B, a.k + 1, a.T, s_start)) {
    if (threadIdx.x == 0) report(a, kStatusBadLens);
    return;                   // every CTA of every cluster leaves here
  }
  // every draft id is checked (the reference indexes them all): a bad one ends the request in all its CTAs.
  // Lane j loads draft j's uniform, q and target logit, so a row's decision waits on nothing but the row.
  if (threadIdx.x < 32) {
    const int row0 = a.lens == nullptr ? b * (a.k + 1) : s_start[b];
    const int len = a.lens == nullptr ? a.k + 1 : s_start[b + 1] - s_start[b];
    const int j = threadIdx.x;
    bool bad = false;
    if (j < a.k) {
      const long long li = (long long)b * a.k + j;
      const long long d = a.drafts[li];
      bad = d < 0 || d >= a.V;
      if (!bad && j < len - 1) {
        s_u[j] = a.u ? a.u[li] : torch_rand_at(a.seed, a.offset_u, li, a.u_grid);
        s_q[j] = a.q[li * a.V + d];
        s_x[j] = to_f32(reinterpret_cast<const T*>(a.x)[(row0 + j) * a.V + d]);
      }
    }
    bad = __any_sync(0xffffffffu, bad);
    if (j == 0) {
      s_flag = bad ? 2 : 0;
      s_j = 0;
      s_row0 = row0;
      s_len = len;
      s_k = (gridDim.x % 2 == 0 && len >= 2) ? 2 : 1;
      s_temp = a.temperature[b];
    }
  }
  __syncthreads();
  if (s_flag) {
    if (threadIdx.x == 0 && blockIdx.x == 0) report(a, kStatusBadDraft);
    return;                   // every CTA of this cluster leaves here
  }
  // each step reduces the next K rows at once, P = C / K CTAs (chunks) per row; the decisions then go row by row.
  // K is two at first (most walks end within two rows), then the most rows the cluster can give a CTA each of
  // (the walks that get that far tend to go on)
  while (true) {
    const int K = s_k, P = (int)gridDim.x / K;
    const int my_row = (int)blockIdx.x / P, my_chunk = (int)blockIdx.x % P;
    {
      constexpr int ve = sizeof(T) == 4 ? 4 : 8;
      const long long chunk = ((a.V + P - 1) / P + ve - 1) / ve * ve;
      const int jr = s_j + my_row;
      float m = -INFINITY, s = 0.0f;    // a row past the request's last, or an empty chunk, contributes nothing
      const long long lo = my_chunk * chunk;
      if (jr < s_len && lo < a.V) {
        const long long t = s_row0 + jr;
        const long long hi = min(lo + chunk, a.V);
        row_range_ms<T, kThreads>(reinterpret_cast<const T*>(a.x) + t * a.V, (int)lo, (int)hi, s_temp, a.vec_ok, m,
                                  s);
      }
      block_ms<kThreads>(m, s);
      if (threadIdx.x == 0) s_part = make_float2(m, s);
    }
    cluster_barrier();        // every chunk's partial of the step's rows is visible to the cluster
    if (threadIdx.x < 32) {
      const int lane = threadIdx.x;
      float pm = -INFINITY, ps = 0.0f;
      if (lane < (int)gridDim.x) {   // the cluster spans the grid's x dimension: rank = blockIdx.x
        const float2 p = ld_cluster_f2(&s_part, lane);
        pm = p.x;
        ps = p.y;
      }
      int decided = -1;
      RowStat rs_dec;
      rs_dec.m = 0.0f; rs_dec.s = 1.0f; rs_dec.thr = -INFINITY; rs_dec.pad = 0.0f;
      for (int r = 0; r < K; ++r) {   // warp-uniform; every lane (and CTA) merges in the same order
        float m = -INFINITY, s = 0.0f;
        for (int c = 0; c < P; ++c) {
          const float m2 = __shfl_sync(0xffffffffu, pm, r * P + c);
          const float s2 = __shfl_sync(0xffffffffu, ps, r * P + c);
          ms_combine(m, s, m2, s2);
        }
        const int j = s_j + r;
        if (decided >= 0 || j >= s_len) continue;
        RowStat rs;
        rs.m = m; rs.s = s; rs.thr = -INFINITY; rs.pad = 0.0f;
        bool stop = j == s_len - 1;
        if (!stop) {   // prob_at's arithmetic on the preloaded logit
          const float f = s_temp == 1.0f ? s_x[j] : scale_logit(s_x[j], s_temp);
          stop = !(s_u[j] * s_q[j] < prob_of_scaled(f, rs));   // u < min(1, p/q) without dividing
        }
        if (stop) {
          decided = j;
          rs_dec = rs;
        }
      }
      if (lane == 0) {
        s_flag = decided >= 0 ? 1 : 0;
        s_rs = rs_dec;
        s_j = decided >= 0 ? decided : s_j + K;
        s_k = early_rows_per_step((int)gridDim.x, s_len - s_j);
      }
    }
    cluster_barrier();        // the partials are read before any CTA overwrites (or leaves with) its own
    if (s_flag) {
      if (blockIdx.x == 0 && threadIdx.x == 0) {   // n_accept = j: drafts 0..j-1 accepted
        const int j = s_j;
        const long long t = s_row0 + j;
        const bool last_row = j == s_len - 1;
        a.n_accept[b] = j;
        ReqDesc d;
        d.x_row = t;
        d.q_row = last_row ? -1 : (long long)b * a.k + j;
        d.m = s_rs.m;
        d.s = s_rs.s;
        d.thr = s_rs.thr;
        d.temp = s_temp;
        a.desc[b] = d;
        a.rows[t] = s_rs;
      }
      return;
    }
  }
}

// ---------------------------------------------------------------------------------------- pass 1 (truncating)
// One CTA per row: radix select of the k-th largest scaled logit over L2-resident re-reads, sorted top-k,
// top-p over the top-k softmax, then (max, sum) over the kept entries.
template <int NT>
__device__ void select_digit(const unsigned* hist, int nbins, int rank, int* s_digit, int* s_above) {
  // rank: 1-based rank (from the top) of the wanted element among the elements counted in hist.
  __shared__ int warp_tot[NT / 32];
  const int per = nbins >= NT ? nbins / NT : 1;       // bins per owning thread
  const int owners = nbins / per;
  // thread i owns bins [i*per, (i+1)*per); suffix sums from the top
  int local = 0;
  if ((int)threadIdx.x < owners)
    for (int j = 0; j < per; ++j) local += hist[threadIdx.x * per + j];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  // inclusive scan from the top: reverse the thread order
  int incl = local;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    int n = __shfl_down_sync(0xffffffffu, incl, o);
    if (lane + o < 32) incl += n;
  }
  if (lane == 0) warp_tot[warp] = incl;
  __syncthreads();
  int above_warps = 0;
  for (int w = warp + 1; w < NT / 32; ++w) above_warps += warp_tot[w];
  int above = above_warps + incl - local;  // elements in bins above this thread's bins
  if ((int)threadIdx.x < owners) {
    for (int j = per - 1; j >= 0; --j) {
      int h = hist[threadIdx.x * per + j];
      if (above < rank && rank <= above + h) {
        *s_digit = threadIdx.x * per + j;
        *s_above = above;
      }
      above += h;
    }
  }
  __syncthreads();
}

template <typename T>
__device__ __forceinline__ float scaled_at(const T* row, int v, float temp) {
  float f = to_f32(row[v]);
  return temp == 1.0f ? f : scale_logit(f, temp);
}

// Scaled logits (x / T) of the 8 consecutive elements of group g of a row (16-byte loads when vec); returns how
// many exist; missing ones are -inf.
template <typename T>
__device__ __forceinline__ int load_group_scaled(const T* row, int g, int V, int vec, float temp, float (&f)[8]) {
  const int v0 = g * 8;
  const int n = min(8, V - v0);
  if (vec && n == 8) {
    if constexpr (sizeof(T) == 4) {
      float lo[4], hi[4];
      unpack16(ldg16(row + v0), lo);
      unpack16(ldg16(row + v0 + 4), hi);
#pragma unroll
      for (int e = 0; e < 4; ++e) { f[e] = lo[e]; f[e + 4] = hi[e]; }
    } else if constexpr (std::is_same<T, __nv_bfloat16>::value) {
      unpack16_bf16(ldg16(row + v0), f);
    } else {
      unpack16_f16(ldg16(row + v0), f);
    }
    if (temp != 1.0f) {
#pragma unroll
      for (int e = 0; e < 8; ++e) f[e] = scale_logit(f[e], temp);
    }
  } else {
#pragma unroll
    for (int e = 0; e < 8; ++e) f[e] = e < n ? scaled_at(row, v0 + e, temp) : -INFINITY;
  }
  return n;
}

template <typename T>
__global__ void __launch_bounds__(kTopkThreads, 2) topk_stats_kernel(Args a, int mode) {
  constexpr int NT = kTopkThreads;
  __shared__ int s_start[kMaxRequests + 1];
  __shared__ unsigned long long sel[4096];                // fast-path candidates; the radix fallback's histogram
  unsigned* hist = reinterpret_cast<unsigned*>(sel);      // (4096 bins) reuses the same bytes
  __shared__ int s_sel;
  __shared__ float cand[kMaxTopK];
  __shared__ int s_digit, s_above, s_cnt, s_last;
  __shared__ float s_thr;
  const int t = blockIdx.x;
  int b, start = 0, len = 0;
  if (mode == 0) {
    if (!starts_from_lens<NT>(a.lens, a.B, a.k + 1, a.T, s_start)) {
      if (threadIdx.x == 0) report(a, kStatusBadLens);
      return;
    }
    b = request_of_row(s_start, a.B, t);
    start = s_start[b];
    len = s_start[b + 1] - start;
  } else {
    b = t / a.rows_per_param;
  }
  const float temp = a.temperature[b];
  const long long tk = a.top_k ? a.top_k[b] : 0;
  const int V = (int)a.V;
  const T* row = reinterpret_cast<const T*>(a.x) + (long long)t * a.V;
  float m, s, thr = -INFINITY;
  if (tk <= 0) {
    row_range_ms<T, NT>(row, 0, V, temp, a.vec_ok, m, s);
    block_ms<NT>(m, s);
    if (threadIdx.x == 0) a.kept_n[t] = -1;
  } else {
    if (tk > kMaxTopK && V > kMaxTopK) {
      if (threadIdx.x == 0) report(a, kStatusBadTopK);
      return;
    }
    const int K = (int)(tk < V ? tk : V);
    // ---- fast path: thread-maxima bound and collection over the raw logits (x / T is monotone in x: the
    // collection margin of 2^-22 relative covers values whose quotient rounds onto the bound's), then the
    // collected candidates re-keyed by x / T and ranked: two passes over the row, no division in them
    int fast = -1;
    unsigned long long* top = nullptr;
    if (K <= NT) {
      const float slack = temp == 1.0f ? 0.0f : 2.384185791015625e-07f;
      if constexpr (sizeof(T) == 2) {
        using H2 = typename std::conditional<std::is_same<T, __half>::value, __half2, __nv_bfloat162>::type;
        if (a.vec_ok)   // 16-byte groups, no ragged end: packed maxima
          fast = select_by_thread_max_x16<NT, 4, H2>(
              V / 8, K, [&](int g) { return __ldg(reinterpret_cast<const uint4*>(row) + g); }, sel, 4096, &s_sel,
              &top, slack);
      }
      if (fast < 0 && (sizeof(T) == 4 || !a.vec_ok))
        fast = select_by_thread_max<NT, 2>(
            (V + 7) / 8, K, [&](int g, float (&x)[8]) { return load_group_scaled(row, g, V, a.vec_ok, 1.0f, x); },
            sel, 4096, &s_sel, &top, slack);
      if (fast >= 0 && temp != 1.0f) {
        const int n = top == sel ? fast : (fast + 31) / 32 * 32;
        for (int i = threadIdx.x; i < n; i += NT) {
          const unsigned long long key = sel[i];
          if (key) {
            const float f = scale_logit(key_to_float((unsigned)(key >> 32)), temp);
            sel[i] = (static_cast<unsigned long long>(ordered_key(f)) << 32) | (key & 0xffffffffull);
          }
        }
        __syncthreads();
        if (top == sel) {
          int P2 = 1;
          while (P2 < fast) P2 <<= 1;
          block_sort_desc_u64(sel, P2);
        } else {
          block_top_sorted<NT>(sel, fast, K, top);
        }
      }
      if (fast >= 0) {
        for (int i = threadIdx.x; i < K; i += NT) cand[i] = key_to_float((unsigned)(top[i] >> 32));
        __syncthreads();
      }
    }
    if (fast < 0) {
    // ---- radix select of the K-th largest key over three digits (12, 12, 8 bits)
    unsigned prefix = 0, pmask = 0;
    int rank = K;
    const int shifts[3] = {20, 8, 0};
    const int widths[3] = {12, 12, 8};
    const int lane = threadIdx.x & 31;
    for (int p = 0; p < 3; ++p) {
      const int nb = 1 << widths[p];
      for (int i = threadIdx.x; i < 4096; i += NT) hist[i] = 0;
      __syncthreads();
      const int ngroups = (V + 7) / 8;
      for (int gb = (threadIdx.x - lane) * 2; gb < ngroups; gb += NT * 2) {   // warp-uniform trip count
        float x0[8], x1[8];
        const int g0 = gb + lane, g1 = gb + 32 + lane;
        const int n0 = g0 < ngroups ? load_group_scaled(row, g0, V, a.vec_ok, temp, x0) : 0;
        const int n1 = g1 < ngroups ? load_group_scaled(row, g1, V, a.vec_ok, temp, x1) : 0;
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const unsigned k0 = ordered_key(x0[e]);
          warp_hist_add(hist, (k0 >> shifts[p]) & (nb - 1), e < n0 && (k0 & pmask) == prefix);
          const unsigned k1 = ordered_key(x1[e]);
          warp_hist_add(hist, (k1 >> shifts[p]) & (nb - 1), e < n1 && (k1 & pmask) == prefix);
        }
      }
      __syncthreads();
      select_digit<NT>(hist, nb, rank, &s_digit, &s_above);
      prefix |= (unsigned)s_digit << shifts[p];
      pmask |= (unsigned)(nb - 1) << shifts[p];
      rank -= s_above;
      __syncthreads();
    }
    const unsigned key_k = prefix;        // key of the K-th largest value
    const int n_gt = K - rank;            // elements strictly above it (< K)
    // ---- collect the values above the K-th, fill the rest with it, sort descending
    if (threadIdx.x == 0) s_cnt = 0;
    __syncthreads();
    {
      const int ngroups = (V + 7) / 8;
      for (int g = threadIdx.x; g < ngroups; g += NT) {
        float x[8];
        const int n = load_group_scaled(row, g, V, a.vec_ok, temp, x);
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          if (e < n && ordered_key(x[e]) > key_k) {
            int slot = atomicAdd(&s_cnt, 1);
            if (slot < kMaxTopK) cand[slot] = x[e];
          }
        }
      }
    }
    __syncthreads();
    int P = 1;
    while (P < K) P <<= 1;
    const float kth = key_to_float(key_k);
    for (int i = threadIdx.x; i < P; i += NT) {
      if (i >= n_gt) cand[i] = i < K ? kth : -INFINITY;
    }
    __syncthreads();
    // bitonic sort, descending
    for (int size = 2; size <= P; size <<= 1) {
      for (int stride = size >> 1; stride > 0; stride >>= 1) {
        for (int i = threadIdx.x; i < P; i += NT) {
          int j = i ^ stride;
          if (j > i) {
            bool desc = (i & size) == 0;
            float ci = cand[i], cj = cand[j];
            if (desc ? (ci < cj) : (ci > cj)) { cand[i] = cj; cand[j] = ci; }
          }
        }
        __syncthreads();
      }
    }
    }  // radix fallback
    // ---- thresholds (one thread; K is small)
    if (threadIdx.x == 0) {
      float th = cand[K - 1];
      if (a.has_top_p) {
        const float tp = a.top_p[b];
        const float c0 = cand[0];
        float z = 0.0f;
        for (int i = 0; i < K; ++i) z += expf(cand[i] - c0);
        float cum = 0.0f;
        int kept = 0;
        for (int i = 0; i < K; ++i) {
          float nu = __fdiv_rn(expf(cand[i] - c0), z);
          cum += nu;
          if (cum - nu < tp) ++kept;
        }
        if (kept >= 1 && kept <= K) th = fmaxf(th, cand[kept - 1]);
      }
      s_thr = th;
    }
    __syncthreads();
    thr = s_thr;
    m = cand[0];
    // ---- sum over the kept entries: every one of them (>= the K-th value) is among the collected candidates on
    // the fast path, whose ids are also recorded for the candidate tail race; the radix path re-reads the row
    float ls = 0.0f;
    if (fast >= 0) {
      if (threadIdx.x == 0) s_cnt = 0;
      __syncthreads();
      int* ids = a.kept_ids + (long long)t * kKeptCap;
      const int n = top == sel ? fast : (fast + 31) / 32 * 32;
      for (int i = threadIdx.x; i < n; i += NT) {
        const unsigned long long key = sel[i];
        if (key) {
          const float f = key_to_float((unsigned)(key >> 32));
          if (f >= thr) {
            ls += exp_sum_term(f - m);
            const int slot = atomicAdd(&s_cnt, 1);
            if (slot < kKeptCap) ids[slot] = (int)(0xffffffffu - (unsigned)(key & 0xffffffffull));
          }
        }
      }
      __syncthreads();
      if (threadIdx.x == 0) a.kept_n[t] = s_cnt <= kKeptCap ? s_cnt : -1;
    } else {
      if (threadIdx.x == 0) a.kept_n[t] = -1;
      const int ngroups = (V + 7) / 8;
      for (int g = threadIdx.x; g < ngroups; g += NT) {
        float x[8];
        const int n = load_group_scaled(row, g, V, a.vec_ok, temp, x);
#pragma unroll
        for (int e = 0; e < 8; ++e)
          if (e < n && x[e] >= thr) ls += exp_sum_term(x[e] - m);
      }
    }
    ls = warp_sum_f32(ls);
    __shared__ float sm_sum[NT / 32];
    if ((threadIdx.x & 31) == 0) sm_sum[threadIdx.x >> 5] = ls;
    __syncthreads();
    s = 0.0f;
    for (int w = 0; w < NT / 32; ++w) s += sm_sum[w];
  }
  if (threadIdx.x == 0) {
    RowStat r;
    r.m = m; r.s = s; r.thr = thr; r.pad = 0.0f;
    a.rows[t] = r;
  }
  if (mode != 0) return;
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) {
    unsigned ticket = atomicAdd(&a.req_ticket[b], 1u);
    s_last = ticket == (unsigned)(len - 1);
  }
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  decide_request<T>(a, b, start, len, false);
  if (threadIdx.x == 0) atomicExch(&a.req_ticket[b], 0u);
}

// ---------------------------------------------------------------------------------------- probs mode decide
// accept_random_varlen with p given: one CTA (one warp working) per request.
template <typename T>
__global__ void __launch_bounds__(64) decide_probs_kernel(Args a) {
  __shared__ int s_start[kMaxRequests + 1];
  if (!starts_from_lens<64>(a.lens, a.B, a.k + 1, a.T, s_start)) {
    if (threadIdx.x == 0) report(a, kStatusBadLens);
    return;
  }
  const int b = blockIdx.x;
  const int start = s_start[b], len = s_start[b + 1] - s_start[b];
  decide_request<T>(a, b, start, len, false);
}

// ---------------------------------------------------------------------------------------- write probabilities
template <typename T>
__global__ void __launch_bounds__(kThreads) write_probs_kernel(Args a, int merged) {
  __shared__ RowStat s_row;
  const int c = blockIdx.x, t = blockIdx.y;
  const int g = t / a.rows_per_param;
  const float temp = a.temperature[g];
  if (threadIdx.x < 32) {
    RowStat rs;
    if (merged) {
      float4 raw = __ldcg(reinterpret_cast<const float4*>(&a.rows[t]));
      rs.m = raw.x; rs.s = raw.y; rs.thr = raw.z; rs.pad = raw.w;
    } else {
      rs = merge_row_warp(a, t);
    }
    if (threadIdx.x == 0) s_row = rs;
  }
  __syncthreads();
  const RowStat rs = s_row;
  const int lo = c * a.chunk;
  const int hi = min((long long)lo + a.chunk, a.V);
  const T* row = reinterpret_cast<const T*>(a.x) + (long long)t * a.V;
  float* out = a.probs_out + (long long)t * a.V;
  for (int v = lo + threadIdx.x; v < hi; v += kThreads) {
    float f = scaled_at(row, v, temp);
    out[v] = prob_of_scaled(f, rs);
  }
}

// ---------------------------------------------------------------------------------------- pass 2: tail race
// Race keys of a warp's 32 elements, which may belong to two rows, folded into the rows' shared-memory maxima.
__device__ __forceinline__ void warp_segment_reduce(unsigned long long key, int b, bool active,
                                                    unsigned long long* s_best) {
  const int lane = threadIdx.x & 31;
  const int b0 = __shfl_sync(0xffffffffu, b, 0);
  const unsigned all = __ballot_sync(0xffffffffu, active);
  if (all == 0xffffffffu && __all_sync(0xffffffffu, b == b0)) {   // the common case: one row, every lane active
    const unsigned long long m = warp_max_u64_redux(key);
    if (lane == 0) atomicMax(&s_best[b0], m);
    return;
  }
  unsigned pending = all;
  while (pending) {
    const int leader = __ffs(pending) - 1;
    const int bb = __shfl_sync(0xffffffffu, b, leader);
    const bool mine = active && b == bb;
    const unsigned long long kk = warp_max_u64_redux(mine ? key : 0ull);
    if (lane == leader) atomicMax(&s_best[bb], kk);
    pending &= ~__ballot_sync(0xffffffffu, mine);
  }
}

// ---------------------------------------------------------------------------------------- pass 2: accept tail
// The tail race of the accept path: torch's exponential_ grid of the [B, V] noise with its draws regenerated
// in-kernel (exactly: Philox blocks, then torch's -log transform), the rest of the per-element arithmetic cut
// down.  p = e^(f - m) / s as exp_compensated(f - m) * (1/s)
// and w / E as a fast quotient: both within a few ulp (a few 1e-7 relative), inside the 1e-6 relative p
// uncertainty the parity rule allows for the race (a winner within that of another candidate is a near tie).
// One 32-bit max per warp and element round, the first lane among equals keeps torch's first-index rule.
struct alignas(16) TailDesc {    // per request, in shared memory (32 B: one float4 + two row pointers)
  float m, inv_s, thr, temp;
  const void* xrow;   // row of x holding p_next
  const float* qrow;  // row of q for the residual, or null (bonus row, plain p)
};
static_assert(sizeof(TailDesc) == 32, "TailDesc is read as float4 + two pointers");

// e^y to a few ulp: 2^(y log2 e) with the rounding error of the product y * log2(e) recovered by an FMA (the
// exact two-product of Dekker / Kahan, as in Muller et al., Handbook of Floating-Point Arithmetic) plus the low
// part of log2(e), applied as 2^t * (1 + err ln 2).  ex2.approx carries the remaining ~2 ulp.
__device__ __forceinline__ float exp_compensated(float y) {
  const float kL = 1.44269502162933349609375f;   // log2(e) rounded to float
  const float kLlo = 1.925963033500011e-08f;     // log2(e) - kL
  const float t = y * kL;
  const float err = fmaf(y, kL, -t) + y * kLlo;
  float p;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(p) : "f"(t));
  return p * fmaf(err, 0.6931471805599453f, 1.0f);
}

// The race weight of one element of a request's tail row: p (given, or e^(f - m) / s of the scaled logit with
// truncated entries at 0), minus q where the tail is a residual, floored at 0.  Both tail kernels call this one
// function so that their weights are the same floats.
__device__ __forceinline__ float tail_weight(float x, float q, const TailDesc& d, bool probs_mode, bool residual) {
  float p;
  if (probs_mode) {
    p = x;
  } else {
    const float f = d.temp == 1.0f ? x : scale_logit(x, d.temp);
    p = f >= d.thr ? exp_compensated(f - d.m) * d.inv_s : 0.0f;
  }
  return residual ? fmaxf(p - q, 0.0f) : p;
}

// One round's four elements (lane ii = grid-stride step ii of the round): loaded x and q values and where the
// round starts.  Element indices stay below 2^32 (B * V < 2^31 and S < 2^21), so they are 32-bit.
struct TailLoads {
  float x[4], q[4];
  unsigned b0, v0;
};

__device__ __forceinline__ void tail_step(const Args& a, unsigned& b, unsigned& v) {
  b += a.e_sq;
  v += a.e_sr;
  if (v >= (unsigned)a.V) { v -= (unsigned)a.V; ++b; }
}

template <typename T>
__device__ __forceinline__ void tail_issue_loads(const Args& a, const TailDesc* s_td, unsigned& b, unsigned& v,
                                                 unsigned li0, unsigned S, unsigned N, TailLoads& L) {
  L.b0 = b;
  L.v0 = v;
#pragma unroll
  for (int ii = 0; ii < 4; ++ii) {
    L.x[ii] = 0.0f;
    L.q[ii] = 0.0f;
    if (li0 + ii * S < N) {
      const TailDesc& d = s_td[b];
      L.x[ii] = to_f32(static_cast<const T*>(d.xrow)[v]);
      if (d.qrow) L.q[ii] = d.qrow[v];
    }
    tail_step(a, b, v);
  }
}


// Race-element filter.  After its first round every CTA holds, per request, a lower bound lb of the request's
// largest ratio (the best exact ratio any CTA had published by then).  An element with w < lb * E cannot win, and
// E = -__logf(u) is bounded below cheaply: -lg2.approx(u) ln 2 and __logf(u) are both within ~4e-7 absolute of
// ln(u), so for u < 0.999 (E > 1e-3) the value shrunk by 1e-3 relative stays below E.  Elements near u = 1 (tiny
// E, large ratios) and requests without a bound yet are never skipped.
__device__ __forceinline__ bool race_candidate(float w, float u, float lb) {
  if (!(lb > 0.0f) || u >= 0.999f) return true;
  float l2;
  asm("lg2.approx.ftz.f32 %0, %1;" : "=f"(l2) : "f"(u));
  const float e_lo = -l2 * (0.6931471805599453f * (1.0f - 1e-3f));
  return !(w < lb * e_lo);
}

// Accept-tail race.  Work per element: the Philox draw and torch's -log transform (exact), p = e^(f - m) / s as
// exp_compensated(f - m) * (1/s), the residual, w / E as a fast quotient (p and the quotient within a few 1e-7
// relative: inside the 1e-6 relative p uncertainty the parity rule allows for the race, where a winner within
// that of another candidate is a near tie), then one 32-bit max per warp; the first lane among equals keeps
// torch's first-index rule.  Round n + 1's loads are issued before round n is computed.
template <typename T>
__global__ void __launch_bounds__(kThreads, 4) tail_accept_kernel(Args a) {
  extern __shared__ __align__(16) unsigned char tail_smem[];
  TailDesc* s_td = reinterpret_cast<TailDesc*>(tail_smem);
  unsigned long long* s_best = reinterpret_cast<unsigned long long*>(tail_smem + sizeof(TailDesc) * a.B);
  float* s_lb = reinterpret_cast<float*>(tail_smem + (sizeof(TailDesc) + sizeof(unsigned long long)) * a.B);
  __shared__ int s_last;
  const volatile int* status = a.status;
  if (status[0] != 0) return;                   // pass 1 rejected its inputs
  if (a.tail_gate && status[1] == 0) return;    // every request raced among its kept tokens
  for (int i = threadIdx.x; i < a.B; i += kThreads) {
    s_best[i] = 0ull;
    s_lb[i] = 0.0f;                                           // no bound during the first round
    const ReqDesc d = a.desc[i];
    TailDesc t;
    t.m = d.m;
    t.inv_s = 1.0f / d.s;
    t.thr = d.thr;
    t.temp = d.temp;
    t.xrow = static_cast<const T*>(a.x) + d.x_row * a.V;
    t.qrow = d.q_row < 0 ? nullptr : a.q + d.q_row * a.V;
    s_td[i] = t;
  }
  __syncthreads();
  const int lane = threadIdx.x & 31;
  const unsigned S = kRngBlock * gridDim.x;
  const unsigned idx = blockIdx.x * kRngBlock + threadIdx.x;
  const unsigned N = (unsigned)a.e_numel;
  const unsigned V = (unsigned)a.V;
  const bool gen = a.E == nullptr;
  const bool direct = (a.offset_E & 3ull) == 0;     // torch's offsets are multiples of 4
  curandStatePhilox4_32_10_t st;
  if (gen && !direct) curand_init(a.seed, idx, a.offset_E, &st);
  const unsigned long long c0 = a.offset_E >> 2;
  unsigned b = idx / V, v = idx % V;
  unsigned li0 = idx;                      // element of lane ii = 0 in the current round
  unsigned warp0 = idx - lane;             // the warp's first element in the current round
  TailLoads cur{}, nxt{};
  if (a.e_rounds > 0 && warp0 < N) tail_issue_loads<T>(a, s_td, b, v, li0, S, N, cur);
  for (int n = 0; n < a.e_rounds; ++n) {
    if (n == 1) {
      // the bound exchange after the first round: this CTA's bests out, every CTA's published bests back (one
      // exchange measured best: later or repeated ones cost more than their tighter bounds save)
      __syncthreads();
      for (int i = threadIdx.x; i < a.B; i += kThreads)
        if (s_best[i]) atomicMax(&a.tail_key[i], s_best[i]);
      __syncthreads();
      for (int i = threadIdx.x; i < a.B; i += kThreads) {
        const unsigned long long kk = __ldcg(&a.tail_key[i]);
        s_lb[i] = kk ? __uint_as_float(static_cast<unsigned>(kk >> 32) & 0x7fffffffu) : 0.0f;
      }
      __syncthreads();
    }
    if (warp0 >= N) continue;                                  // warp-uniform (every warp reaches the exchange)
    if (n + 1 < a.e_rounds && warp0 + 4 * S < N) tail_issue_loads<T>(a, s_td, b, v, li0 + 4 * S, S, N, nxt);
    float uu[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    if (gen) {
      const float4 r4 = direct ? philox_uniform4(a.seed, c0, idx, n) : curand_uniform4(&st);
      uu[0] = r4.x;
      uu[1] = r4.y;
      uu[2] = r4.z;
      uu[3] = r4.w;
    }
    unsigned bb = cur.b0, vv = cur.v0;
    if (!a.probs_mode && warp0 + 3 * S + 32 <= N) {
      // full round: every element in range for the whole warp; selects instead of branches
#pragma unroll
      for (int ii = 0; ii < 4; ++ii) {
        const TailDesc& d = s_td[bb];
        const float w = tail_weight(cur.x[ii], cur.q[ii], d, false, d.qrow != nullptr);
        // the whole warp skips elements that provably cannot win (given draws have no u: never skipped)
        if (!__any_sync(0xffffffffu, !gen || race_candidate(w, uu[ii], s_lb[bb]))) {
          tail_step(a, bb, vv);
          continue;
        }
        const float e = gen ? torch_exponential_clamped(uu[ii]) : a.E[li0 + ii * S];
        const unsigned bits = __float_as_uint(__fdividef(w, e)) & 0x7fffffffu;
        if (__all_sync(0xffffffffu, vv >= (unsigned)lane)) {
          // 32 consecutive columns vv(lane 0) + lane of one row
          const unsigned mx = __reduce_max_sync(0xffffffffu, bits);
          const unsigned first = __ffs(__ballot_sync(0xffffffffu, bits == mx)) - 1;
          if (lane == 0)
            atomicMax(&s_best[bb],
                      (static_cast<unsigned long long>(mx | 0x80000000u) << 32) | (0xffffffffu - (vv + first)));
        } else {
          warp_segment_reduce((static_cast<unsigned long long>(bits | 0x80000000u) << 32) | (0xffffffffu - vv),
                              (int)bb, true, s_best);
        }
        tail_step(a, bb, vv);
      }
    } else {
#pragma unroll
      for (int ii = 0; ii < 4; ++ii) {
        if (warp0 + ii * S < N) {                                // warp-uniform
          const unsigned li = li0 + ii * S;
          const bool act = li < N;
          unsigned bits = 0u;
          if (act) {
            const TailDesc& d = s_td[bb];
            const float w = tail_weight(cur.x[ii], cur.q[ii], d, a.probs_mode, d.qrow != nullptr);
            const float e = gen ? torch_exponential_clamped(uu[ii]) : a.E[li];
            bits = __float_as_uint(__fdividef(w, e)) & 0x7fffffffu;   // w >= 0: clears a -0
          }
          const unsigned b0 = __shfl_sync(0xffffffffu, bb, 0);
          if (__all_sync(0xffffffffu, act && bb == b0)) {
            const unsigned mx = __reduce_max_sync(0xffffffffu, bits);
            const unsigned first = __ffs(__ballot_sync(0xffffffffu, bits == mx)) - 1;
            if (lane == 0)
              atomicMax(&s_best[bb],
                        (static_cast<unsigned long long>(mx | 0x80000000u) << 32) | (0xffffffffu - (vv + first)));
          } else {
            const unsigned long long key =
                act ? (static_cast<unsigned long long>(bits | 0x80000000u) << 32) | (0xffffffffu - vv) : 0ull;
            warp_segment_reduce(key, (int)bb, act, s_best);
          }
        }
        tail_step(a, bb, vv);
      }
    }
    cur = nxt;
    li0 += 4 * S;
    warp0 += 4 * S;
  }
  __syncthreads();
  for (int i = threadIdx.x; i < a.B; i += kThreads) {
    unsigned long long kk = s_best[i];
    if (kk) atomicMax(&a.tail_key[i], kk);
  }
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) {
    unsigned ticket = atomicAdd(a.tail_ticket, 1u);
    s_last = ticket == gridDim.x - 1;
  }
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  for (int i = threadIdx.x; i < a.B; i += kThreads) {
    unsigned long long kk = atomicExch(&a.tail_key[i], 0ull);
    a.tail[i] = (long long)argmax_key_index(kk);
  }
  if (threadIdx.x == 0) atomicExch(a.tail_ticket, 0u);
}

// ---------------------------------------------------------------------------------------- pass 2 over noise codes
// The accept tail race when the workspace holds 2 bytes per element of the [B, V] noise
// (specdec_accept_workspace_bytes).  noise_codes_kernel draws the noise on torch's exponential_ grid before
// pass 1 and keeps of each E only a 16-bit code, the upper half of its float bits, so that E lies in
// [lo(code), hi(code)) (truncation keeps the order of positive floats).  tail_codes_kernel then streams each
// request's tail row, its q row and its codes, bounds every element's ratio w / E from both sides, and draws
// exactly (the Philox block again, torch's transform, the quotient tail_accept_kernel takes) only the elements
// whose upper bound reaches the best lower bound: every other element provably loses, so the winner is the one
// tail_accept_kernel finds, bit for bit.
constexpr int kCodeVec = 8;           // elements per lane and group (16 bytes of codes)
constexpr int kCodeGroups = 2;        // groups per lane and item
constexpr int kCodeItem = 32 * kCodeVec * kCodeGroups;   // elements of one warp's item (512)
constexpr int kCodeCtasPerSm = 2;


// The [B, V] exponential draw at (seed, offset_E), as 16-bit codes (kFloats = false) or as the floats themselves
// (a test hook): launched with torch's grid (e_grid blocks of 256), each thread one Philox block per grid-stride
// round, element idx + (4 n + ii) S of round n taking lane ii.
template <bool kFloats>
__global__ void __launch_bounds__(kThreads) noise_codes_kernel(Args a, float* floats) {
  const unsigned S = kRngBlock * (unsigned)a.e_grid;   // torch's grid; this launch's grid strides over it
  const unsigned N = (unsigned)a.e_numel;
  const unsigned long long c0 = a.offset_E >> 2;
  for (unsigned idx = blockIdx.x * kRngBlock + threadIdx.x; idx < S; idx += gridDim.x * kRngBlock) {
    for (int n = 0; n < a.e_rounds; ++n) {
      const unsigned li0 = idx + 4u * (unsigned)n * S;
      if (li0 >= N) break;
      const float4 r4 = philox_uniform4(a.seed, c0, idx, n);
      const float r[4] = {r4.x, r4.y, r4.z, r4.w};
#pragma unroll
      for (int ii = 0; ii < 4; ++ii) {
        const unsigned li = li0 + (unsigned)ii * S;
        if (li < N) {
          if constexpr (kFloats) {
            floats[li] = torch_exponential_clamped(r[ii]);
          } else {
            a.codes[li] = noise_code(r[ii]);
          }
        }
      }
    }
  }
  // launched as a dependent of the accept's pass 1 (beside which it runs): its end then also implies pass 1's,
  // whose decisions the tail race reads with the codes (returns at once for an ordinary launch).  The race, a
  // dependent of this kernel, may start launching as its CTAs finish.
  griddep_launch_dependents();
  griddep_wait();
}

// Exact race key of element v of request b's tail row: torch's E regenerated from its Philox block, then the
// quotient and key exactly as tail_accept_kernel forms them.
// S = 256 * torch's grid, c0 = offset / 4.
__device__ __forceinline__ unsigned long long exact_race_key(unsigned long long seed, unsigned long long c0, unsigned S,
                                                          unsigned V, unsigned b, unsigned v, float w) {
  const unsigned li = b * V + v;
  const unsigned m = li / S;
  const float4 r4 = philox_uniform4(seed, c0, li - m * S, (int)(m >> 2));
  const unsigned lane = m & 3u;
  const float r = lane == 0 ? r4.x : lane == 1 ? r4.y : lane == 2 ? r4.z : r4.w;
  const float e = torch_exponential_clamped(r);
  const unsigned bits = __float_as_uint(__fdividef(w, e)) & 0x7fffffffu;
  return (static_cast<unsigned long long>(bits | 0x80000000u) << 32) | (0xffffffffu - v);
}

template <typename T>
__device__ __forceinline__ void load_x8(const T* row, unsigned v, float (&f)[8]) {
  if constexpr (sizeof(T) == 4) {
    float h[4];
    unpack16(ldg16(row + v), h);
#pragma unroll
    for (int j = 0; j < 4; ++j) f[j] = h[j];
    unpack16(ldg16(row + v + 4), h);
#pragma unroll
    for (int j = 0; j < 4; ++j) f[4 + j] = h[j];
  } else if constexpr (std::is_same<T, __nv_bfloat16>::value) {
    unpack16_bf16(ldg16(row + v), f);
  } else {
    unpack16_f16(ldg16(row + v), f);
  }
}

// Weights of 8 consecutive elements under one item's descriptor, with tail_weight's flags fixed per item (the same
// operations on the same inputs, so the same floats as tail_weight).
template <bool kProbs, bool kUnit, bool kResidual>
__device__ __forceinline__ void weights8(const float (&x)[8], const float (&q)[8], const TailDesc& d, float (&w)[8]) {
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    float p;
    if constexpr (kProbs) {
      p = x[j];
    } else {
      const float f = kUnit ? x[j] : scale_logit(x[j], d.temp);
      p = f >= d.thr ? exp_compensated(f - d.m) * d.inv_s : 0.0f;
    }
    w[j] = kResidual ? fmaxf(p - q[j], 0.0f) : p;
  }
}

template <bool kResidual>
__device__ __forceinline__ void weights8_any(int mode, const float (&x)[8], const float (&q)[8], const TailDesc& d,
                                             float (&w)[8]) {
  if (mode == 0) {
    weights8<true, true, kResidual>(x, q, d, w);
  } else if (mode == 1) {
    weights8<false, true, kResidual>(x, q, d, w);
  } else {
    weights8<false, false, kResidual>(x, q, d, w);
  }
}

// Float bits of the lower end of the code range of element j of a packed pair word (element 2i in the low half).
__device__ __forceinline__ unsigned code_lo_bits(unsigned word, int j) {
  return (j & 1) ? (word & 0xffff0000u) : (word << 16);
}

__device__ __forceinline__ float rcp_approx(float x) {
  float r;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(x));
  return r;
}

// The race of one warp's item once its values are in registers: x, q (0 where there is no residual) and the
// codes of the lane's kCodeGroups groups of 8 consecutive elements starting at `base` (+ 256 per group).  Per
// element only an upper bound of the ratio, ub = w / lo (a reciprocal), and per lane its maximum.  Since a code's
// range has hi / lo <= 129 / 128 (7 mantissa bits), ub * 128 / 129 bounds the same ratio from below, so the warp's
// largest ub, scaled so, or the best exact ratio any item of the request has published is a lower bound LB of
// the request's largest ratio, and so is `known`, the best key the warp knows for the request (published by other
// warps when its run of the row began, or found by itself since).  Only a lane whose largest ub reaches LB (past
// the quotients' error) can hold the winner: such lanes (one or two per item, none once `known` dominates) hand
// all their elements to the warp's candidate list, which is drawn exactly into `known`.  An item with no positive bound races its
// positive weights and its first element exactly (all-zero weights: the first index wins, as in torch).
__device__ __forceinline__ void race_item(const Args& a, float2* my_list, int lane, unsigned b, unsigned v0,
                                          unsigned base, unsigned V, const TailDesc& d, bool residual,
                                          unsigned long long& known, float (&x)[kCodeGroups][kCodeVec],
                                          float (&q)[kCodeGroups][kCodeVec],
                                          const unsigned (&cw)[kCodeGroups][kCodeVec / 2]) {
  const int mode = a.probs_mode ? 0 : (d.temp == 1.0f ? 1 : 2);
  float w[kCodeGroups][kCodeVec];
  float ub = 0.0f;
#pragma unroll
  for (int g = 0; g < kCodeGroups; ++g) {
    if (residual) {
      weights8_any<true>(mode, x[g], q[g], d, w[g]);
    } else {
      weights8_any<false>(mode, x[g], q[g], d, w[g]);
    }
    const bool in = base + (unsigned)g * (32 * kCodeVec) < V;
#pragma unroll
    for (int j = 0; j < kCodeVec; ++j) {
      if (!in || base + (unsigned)g * (32 * kCodeVec) + j >= V) w[g][j] = 0.0f;   // past the row
      ub = fmaxf(ub, w[g][j] * rcp_approx(__uint_as_float(code_lo_bits(cw[g][j / 2], j))));
    }
  }
  // ub_max * 128/129 bounds the best w / hi from below; shrunk past the reciprocal's and the exact quotients'
  // error, subnormal bounds dropped
  float lb = warp_max_f32(ub) * (128.0f / 129.0f) * (1.0f - 1e-5f);
  if (!(lb >= 1.17549435e-38f)) lb = 0.0f;
  const float pub = known ? __uint_as_float(static_cast<unsigned>(known >> 32) & 0x7fffffffu) : 0.0f;
  const float LB = fmaxf(lb, pub);
  unsigned n_cand = 0;
  if (LB > 0.0f) {
    const bool mine = ub * (1.0f + 1e-5f) >= LB;
    const unsigned ballot = __ballot_sync(0xffffffffu, mine);
    if (mine) {   // all the lane's elements, at its rank's slots (past the row: an empty weight at V)
      float2* slot = my_list + kCodeGroups * kCodeVec * __popc(ballot & ((1u << lane) - 1u));
#pragma unroll
      for (int g = 0; g < kCodeGroups; ++g) {
#pragma unroll
        for (int j = 0; j < kCodeVec; ++j) {
          const unsigned v = base + (unsigned)g * (32 * kCodeVec) + (unsigned)j;
          slot[g * kCodeVec + j] = make_float2(__uint_as_float(v < V ? v : V), w[g][j]);
        }
      }
    }
    n_cand = kCodeGroups * kCodeVec * __popc(ballot);
  } else {
#pragma unroll
    for (int g = 0; g < kCodeGroups; ++g) {
#pragma unroll
      for (int j = 0; j < kCodeVec; ++j) {
        const unsigned v = base + (unsigned)g * (32 * kCodeVec) + (unsigned)j;
        const bool cand = v < V && (w[g][j] > 0.0f || v == v0);
        const unsigned ballot = __ballot_sync(0xffffffffu, cand);
        if (cand) my_list[n_cand + __popc(ballot & ((1u << lane) - 1u))] = make_float2(__uint_as_float(v), w[g][j]);
        n_cand += __popc(ballot);
      }
    }
  }
  __syncwarp();
  unsigned long long best = 0ull;
  for (unsigned i = lane; i < n_cand; i += 32) {
    const float2 c = my_list[i];
    const unsigned v = __float_as_uint(c.x);
    if (v < V) {
      const unsigned long long key =
          exact_race_key(a.seed, a.offset_E >> 2, kRngBlock * (unsigned)a.e_grid, V, b, v, c.y);
      best = key > best ? key : best;
    }
  }
  __syncwarp();
  best = warp_max_u64_redux(best);
  known = best > known ? best : known;
}

// One item's 16-byte vectors for one lane (the fast path: V % 8 == 0 and 16-byte aligned rows, so a group of 8 is
// wholly in or out of the row).
template <typename T>
struct CodeLoads {
  uint4 x[kCodeGroups][sizeof(T) == 4 ? 2 : 1];
  uint4 q[kCodeGroups][2];
  uint4 c[kCodeGroups];
};

template <typename T>
__device__ __forceinline__ void issue_item(const Args& a, const TailDesc* s_td, unsigned item, unsigned per_row,
                                           unsigned V, int lane, CodeLoads<T>& L) {
  const unsigned b = item / per_row;
  const unsigned base = (item - b * per_row) * kCodeItem + (unsigned)lane * kCodeVec;
  const T* xrow = static_cast<const T*>(s_td[b].xrow);
  const float* qrow = s_td[b].qrow;
  const unsigned short* crow = a.codes + (size_t)b * V;
  const uint4 zero = make_uint4(0u, 0u, 0u, 0u);
#pragma unroll
  for (int g = 0; g < kCodeGroups; ++g) {
    const unsigned v = base + (unsigned)g * (32 * kCodeVec);
    const bool in = v < V;
#pragma unroll
    for (int h = 0; h < (sizeof(T) == 4 ? 2 : 1); ++h) L.x[g][h] = in ? ldg16(xrow + v + 4 * h) : zero;
    L.q[g][0] = in && qrow ? ldg16(qrow + v) : zero;
    L.q[g][1] = in && qrow ? ldg16(qrow + v + 4) : zero;
    L.c[g] = in ? ldg16(crow + v) : make_uint4(0x3f803f80u, 0x3f803f80u, 0x3f803f80u, 0x3f803f80u);   // 1.0
  }
}

// Items of kCodeItem elements of the requests' rows, a contiguous run of them per warp.  The requests'
// descriptors sit in shared memory; on the fast path (kVec) the next item's loads are issued before the current
// item is raced, so every warp keeps an item's bytes in flight while it computes.
template <typename T, bool kVec>
__global__ void __launch_bounds__(kThreads, kCodeCtasPerSm) tail_codes_kernel(Args a) {
  extern __shared__ __align__(16) unsigned char codes_smem[];
  TailDesc* s_td = reinterpret_cast<TailDesc*>(codes_smem);
  __shared__ int s_last;
  __shared__ float2 s_list[kThreads / 32][kCodeItem];   // per warp: (element, weight) of its item's candidates
  griddep_wait();                               // launched as a dependent of the pass that wrote its inputs
  const volatile int* status = a.status;
  if (status[0] != 0) return;                   // pass 1 rejected its inputs
  const unsigned V = (unsigned)a.V;
  for (int i = threadIdx.x; i < a.B; i += kThreads) {
    const ReqDesc rd = a.desc[i];
    TailDesc t;
    t.m = rd.m;
    t.inv_s = 1.0f / rd.s;
    t.thr = rd.thr;
    t.temp = rd.temp;
    t.xrow = static_cast<const T*>(a.x) + rd.x_row * (long long)V;
    t.qrow = rd.q_row < 0 ? nullptr : a.q + rd.q_row * (long long)V;
    s_td[i] = t;
  }
  __syncthreads();
  const int lane = threadIdx.x & 31;
  float2* my_list = s_list[threadIdx.x >> 5];
  const unsigned per_row = (V + kCodeItem - 1) / kCodeItem;
  const unsigned items = per_row * (unsigned)a.B;
  // each warp races a contiguous run of items (mostly of one request's row), keeping the best key it knows for
  // the request in registers and publishing it once per run of the row
  const unsigned long long nw = (unsigned long long)gridDim.x * (kThreads / 32);
  const unsigned long long wg = (unsigned long long)blockIdx.x * (kThreads / 32) + (threadIdx.x >> 5);
  unsigned item = (unsigned)(items * wg / nw);
  const unsigned item_end = (unsigned)(items * (wg + 1) / nw);
  unsigned row = 0xffffffffu;
  unsigned long long known = 0ull, published = 0ull;
  auto enter_row = [&](unsigned b) {
    if (b == row) return;
    if (row != 0xffffffffu && lane == 0 && known > published) atomicMax(&a.tail_key[row], known);
    row = b;
    published = __ldcg(&a.tail_key[b]);
    known = published;
  };
  if constexpr (kVec) {
    // two load sets, alternated (no register copies): an item's loads are issued one item ahead of its race
    auto race_loaded = [&](unsigned it, const CodeLoads<T>& L) {
      const unsigned b = it / per_row;
      const unsigned v0 = (it - b * per_row) * kCodeItem;
      enter_row(b);
      float x[kCodeGroups][kCodeVec], q[kCodeGroups][kCodeVec];
      unsigned cw[kCodeGroups][kCodeVec / 2];
#pragma unroll
      for (int g = 0; g < kCodeGroups; ++g) {
        if constexpr (sizeof(T) == 4) {
          float h[4];
          unpack16(L.x[g][0], h);
#pragma unroll
          for (int j = 0; j < 4; ++j) x[g][j] = h[j];
          unpack16(L.x[g][1], h);
#pragma unroll
          for (int j = 0; j < 4; ++j) x[g][4 + j] = h[j];
        } else if constexpr (std::is_same<T, __nv_bfloat16>::value) {
          unpack16_bf16(L.x[g][0], x[g]);
        } else {
          unpack16_f16(L.x[g][0], x[g]);
        }
        float h[4];
        unpack16(L.q[g][0], h);
#pragma unroll
        for (int j = 0; j < 4; ++j) q[g][j] = h[j];
        unpack16(L.q[g][1], h);
#pragma unroll
        for (int j = 0; j < 4; ++j) q[g][4 + j] = h[j];
        cw[g][0] = L.c[g].x;
        cw[g][1] = L.c[g].y;
        cw[g][2] = L.c[g].z;
        cw[g][3] = L.c[g].w;
      }
      const TailDesc& d = s_td[b];
      race_item(a, my_list, lane, b, v0, v0 + (unsigned)lane * kCodeVec, V, d, d.qrow != nullptr, known, x, q, cw);
    };
    CodeLoads<T> la, lb;
    if (item < item_end) issue_item<T>(a, s_td, item, per_row, V, lane, la);
    while (item < item_end) {
      if (item + 1 < item_end) issue_item<T>(a, s_td, item + 1, per_row, V, lane, lb);
      race_loaded(item, la);
      if (++item >= item_end) break;
      if (item + 1 < item_end) issue_item<T>(a, s_td, item + 1, per_row, V, lane, la);
      race_loaded(item, lb);
      ++item;
    }
  } else {
    for (; item < item_end; ++item) {
      const unsigned b = item / per_row;
      const unsigned v0 = (item - b * per_row) * kCodeItem;
      enter_row(b);
      const TailDesc& d = s_td[b];
      const T* xrow = static_cast<const T*>(d.xrow);
      const float* qrow = d.qrow;
      const unsigned short* crow = a.codes + (size_t)b * V;
      const unsigned base = v0 + (unsigned)lane * kCodeVec;
      float x[kCodeGroups][kCodeVec], q[kCodeGroups][kCodeVec];
      unsigned cw[kCodeGroups][kCodeVec / 2];
#pragma unroll
      for (int g = 0; g < kCodeGroups; ++g) {
        const unsigned v = base + (unsigned)g * (32 * kCodeVec);
#pragma unroll
        for (int j = 0; j < kCodeVec; ++j) {
          const bool in = v + j < V;
          x[g][j] = in ? to_f32(xrow[v + j]) : 0.0f;
          q[g][j] = in && qrow ? qrow[v + j] : 0.0f;
        }
#pragma unroll
        for (int j = 0; j < kCodeVec / 2; ++j) {   // 1.0 past the row
          const unsigned c0 = v + 2 * j < V ? crow[v + 2 * j] : 0x3f80u;
          const unsigned c1 = v + 2 * j + 1 < V ? crow[v + 2 * j + 1] : 0x3f80u;
          cw[g][j] = c0 | (c1 << 16);
        }
      }
      race_item(a, my_list, lane, b, v0, base, V, d, qrow != nullptr, known, x, q, cw);
    }
  }
  if (row != 0xffffffffu && lane == 0 && known > published) atomicMax(&a.tail_key[row], known);
  __threadfence();   // this warp's published keys before the CTA's ticket
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    const unsigned ticket = atomicAdd(a.tail_ticket, 1u);
    s_last = ticket == gridDim.x - 1;
  }
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  for (int i = threadIdx.x; i < a.B; i += kThreads) {
    const unsigned long long kk = atomicExch(&a.tail_key[i], 0ull);
    a.tail[i] = (long long)argmax_key_index(kk);
  }
  if (threadIdx.x == 0) atomicExch(a.tail_ticket, 0u);
}

// race() / sample(): w fp32 [B, V] (row b is request b), argmax over v of w / E with torch's exact quotient and
// its first-index rule; E drawn in-kernel (Philox blocks at torch's counters) on the exponential_ grid, or given.
__global__ void __launch_bounds__(kThreads) race_kernel(Args a) {
  __shared__ unsigned long long s_best[kMaxRequests];
  __shared__ int s_last;
  for (int i = threadIdx.x; i < a.B; i += kThreads) s_best[i] = 0ull;
  __syncthreads();
  const unsigned S = kRngBlock * gridDim.x;
  const unsigned idx = blockIdx.x * kRngBlock + threadIdx.x;
  const unsigned N = (unsigned)a.e_numel;
  const unsigned V = (unsigned)a.V;
  const float* w = reinterpret_cast<const float*>(a.x);
  const bool gen = a.E == nullptr;
  const bool direct = (a.offset_E & 3ull) == 0;     // torch's offsets are multiples of 4
  curandStatePhilox4_32_10_t st;
  if (gen && !direct) curand_init(a.seed, idx, a.offset_E, &st);
  unsigned b = idx / V, v = idx % V;
  unsigned li0 = idx, warp0 = idx - (threadIdx.x & 31);
  for (int n = 0; n < a.e_rounds; ++n) {
    if (warp0 >= N) break;                                     // warp-uniform
    float x[4], e[4];
    unsigned bb[4], vv[4];
#pragma unroll
    for (int ii = 0; ii < 4; ++ii) {                            // every load of the round first
      bb[ii] = b;
      vv[ii] = v;
      const bool act = li0 + ii * S < N;
      x[ii] = act ? w[(long long)b * V + v] : 0.0f;
      e[ii] = act && !gen ? a.E[li0 + ii * S] : 1.0f;
      tail_step(a, b, v);
    }
    if (gen) {
      const float4 r4 = direct ? philox_uniform4(a.seed, a.offset_E >> 2, idx, n) : curand_uniform4(&st);
      e[0] = torch_exponential_clamped(r4.x);
      e[1] = torch_exponential_clamped(r4.y);
      e[2] = torch_exponential_clamped(r4.z);
      e[3] = torch_exponential_clamped(r4.w);
    }
#pragma unroll
    for (int ii = 0; ii < 4; ++ii) {
      if (warp0 + ii * S < N) {                                // warp-uniform
        const bool act = li0 + ii * S < N;
        float ratio = __fdiv_rn(x[ii], e[ii]);
        if (ratio == 0.0f) ratio = 0.0f;                        // -0 and +0 compare equal in torch's argmax
        warp_segment_reduce(act ? argmax_key(ratio, vv[ii]) : 0ull, (int)bb[ii], act, s_best);
      }
    }
    li0 += 4 * S;
    warp0 += 4 * S;
  }
  __syncthreads();
  for (int i = threadIdx.x; i < a.B; i += kThreads) {
    unsigned long long kk = s_best[i];
    if (kk) atomicMax(&a.tail_key[i], kk);
  }
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) {
    unsigned ticket = atomicAdd(a.tail_ticket, 1u);
    s_last = ticket == gridDim.x - 1;
  }
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  for (int i = threadIdx.x; i < a.B; i += kThreads) {
    unsigned long long kk = atomicExch(&a.tail_key[i], 0ull);
    a.tail[i] = (long long)argmax_key_index(kk);
  }
  if (threadIdx.x == 0) atomicExch(a.tail_ticket, 0u);
}

// ---------------------------------------------------------------------------------------- pass 2: truncated tail
// Exp(1) draw li of torch's exponential_ over the [B, V] noise (S = 256 * e_grid threads): call li / S / 4 of
// thread li % S's Philox stream, lane (li / S) % 4.
__device__ __forceinline__ float torch_exponential_at(const Args& a, unsigned li) {
  const unsigned S = kRngBlock * (unsigned)a.e_grid;
  const unsigned idx = li % S, m = li / S;
  float4 r;
  if ((a.offset_E & 3ull) == 0) {
    r = philox_uniform4(a.seed, a.offset_E >> 2, idx, (int)(m >> 2));
  } else {
    curandStatePhilox4_32_10_t st;
    curand_init(a.seed, idx, a.offset_E + 4ull * (m >> 2), &st);
    r = curand_uniform4(&st);
  }
  const unsigned lane = m & 3u;
  return torch_exponential_clamped(lane == 0 ? r.x : lane == 1 ? r.y : lane == 2 ? r.z : r.w);
}

// The tail race of requests whose rows truncate (top-k / top-p): p is zero outside the row's kept tokens, so the
// residual max(p - q, 0) (or p itself on the bonus row) is too, and the race over the whole vocabulary is
// decided among the kept tokens (recorded by the stats pass) with their draws regenerated at their positions of
// the noise: the largest ratio wins (first index among equals); if every kept ratio is 0 the whole row ties at
// 0 and torch's first index, 0, wins.  Exact arithmetic (IEEE quotients, expf).  One CTA per request.  When some
// tail row has no recorded kept set (no top-k on its request, or a set above kKeptCap) the decision pass set
// status[1]: this kernel then does nothing and tail_accept_kernel races every request over its whole row.
template <typename T>
__global__ void __launch_bounds__(kThreads) tail_kept_kernel(Args a) {
  __shared__ unsigned long long s_red[kThreads / 32];
  const volatile int* status = a.status;
  if (status[0] != 0 || status[1] != 0) return;   // rejected inputs, or the full-row race runs instead
  const int b = blockIdx.x;
  const ReqDesc d = a.desc[b];
  const T* xrow = reinterpret_cast<const T*>(a.x) + d.x_row * a.V;
  const float* qrow = d.q_row < 0 ? nullptr : a.q + d.q_row * a.V;
  const int n = a.kept_n[d.x_row];
  const int* ids = a.kept_ids + d.x_row * kKeptCap;
  auto key_of = [&](int v) -> unsigned long long {
    const float xv = to_f32(xrow[v]);
    const float f = d.temp == 1.0f ? xv : scale_logit(xv, d.temp);
    const float p = f >= d.thr ? __fdiv_rn(expf(f - d.m), d.s) : 0.0f;
    const float w = qrow ? fmaxf(p - qrow[v], 0.0f) : p;
    const unsigned li = (unsigned)b * (unsigned)a.V + (unsigned)v;
    const float e = a.E ? a.E[li] : torch_exponential_at(a, li);
    float ratio = __fdiv_rn(w, e);
    if (ratio == 0.0f) ratio = 0.0f;                              // -0 and +0 compare equal in torch's argmax
    return argmax_key(ratio, (unsigned)v);
  };
  unsigned long long best = 0ull;
  for (int i = threadIdx.x; i < n; i += kThreads) {   // n >= 1 here (status[1] clear)
    const unsigned long long k = key_of(ids[i]);
    best = k > best ? k : best;
  }
  best = warp_max_u64(best);
  if ((threadIdx.x & 31) == 0) s_red[threadIdx.x >> 5] = best;
  __syncthreads();
  if (threadIdx.x == 0) {
    unsigned long long m = 0ull;
    for (int w = 0; w < kThreads / 32; ++w) m = s_red[w] > m ? s_red[w] : m;
    // a zero best ratio (or no kept token) leaves the whole row tied at 0: index 0 wins
    const bool zero = m == 0ull || key_to_float(static_cast<unsigned>(m >> 32)) == 0.0f;
    a.tail[b] = zero ? 0 : (long long)argmax_key_index(m);
  }
}

// ---------------------------------------------------------------------------------------- greedy
// grid (C, T): per-chunk argmax folded into a per-row 64-bit key; the request's last CTA decides.
template <typename T>
__global__ void __launch_bounds__(kThreads, kGreedyCtasPerSm) greedy_kernel(Args a) {
  __shared__ int s_start[kMaxRequests + 1];
  __shared__ unsigned long long s_red[kThreads / 32];
  __shared__ int s_last;
  const int c = blockIdx.x, t = blockIdx.y;
  if (!starts_from_lens<kThreads>(a.lens, a.B, a.k + 1, a.T, s_start)) {
    if (threadIdx.x == 0) report(a, kStatusBadLens);
    return;
  }
  const int b = request_of_row(s_start, a.B, t);
  const int start = s_start[b], len = s_start[b + 1] - start;
  const int lo = c * a.chunk;
  const int hi = min((long long)lo + a.chunk, a.V);
  const T* row = reinterpret_cast<const T*>(a.x) + (long long)t * a.V;
  unsigned long long best = 0ull;
  bool done = false;
  if constexpr (sizeof(T) == 2) {
    if (a.vec_ok) {
      // 16-byte groups of 8 (lo, hi multiples of 8): the largest 16-bit ordered key of each group by SIMD
      // halfword maxima (widening to fp32 is exact, so this is the order ordered_key gives the fp32 values), the
      // first group holding the thread's maximum kept, then the first element of that group with it
      const uint4* groups = reinterpret_cast<const uint4*>(row);
      unsigned best16 = 0u;
      int best_g = -1;
      auto okey2 = [](unsigned w) {      // two 16-bit ordered keys: negative values inverted, positive ones flagged
        return w ^ ((((w >> 15) & 0x00010001u) * 0x7fffu) | 0x80008000u);
      };
      constexpr int kU = 4;
      const int ng = hi / 8;
      for (int g0 = lo / 8 + threadIdx.x; g0 < ng; g0 += kU * kThreads) {
        uint4 w[kU];
#pragma unroll
        for (int u = 0; u < kU; ++u) {
          const int g = g0 + u * kThreads;
          w[u] = g < ng ? ldg16(groups + g) : make_uint4(0u, 0u, 0u, 0u);
        }
#pragma unroll
        for (int u = 0; u < kU; ++u) {   // ascending g: a later group replaces the kept one only when larger
          const int g = g0 + u * kThreads;
          const unsigned m2 = __vmaxu2(__vmaxu2(okey2(w[u].x), okey2(w[u].y)), __vmaxu2(okey2(w[u].z), okey2(w[u].w)));
          const unsigned gm = max(m2 & 0xffffu, m2 >> 16);
          if (g < ng && (gm > best16 || best_g < 0)) { best16 = gm; best_g = g; }
        }
      }
      if (best_g >= 0) {
        const uint4 w = ldg16(groups + best_g);
        const unsigned words[4] = {w.x, w.y, w.z, w.w};
        int e = 7;
#pragma unroll
        for (int i = 7; i >= 0; --i) {
          const unsigned k = (okey2(words[i >> 1]) >> ((i & 1) * 16)) & 0xffffu;
          if (k == best16) e = i;
        }
        const int v = best_g * 8 + e;
        best = argmax_key(to_f32(row[v]), (unsigned)v);
      }
      done = true;
    }
  }
  if (!done) {
    for (int v = lo + threadIdx.x; v < hi; v += kThreads) {
      unsigned long long kk = argmax_key(to_f32(row[v]), (unsigned)v);
      best = kk > best ? kk : best;
    }
  }
  best = warp_max_u64(best);
  if ((threadIdx.x & 31) == 0) s_red[threadIdx.x >> 5] = best;
  __syncthreads();
  if (threadIdx.x == 0) {
    unsigned long long m = 0ull;
    for (int w = 0; w < kThreads / 32; ++w) m = s_red[w] > m ? s_red[w] : m;
    atomicMax(&a.row_key[t], m);
  }
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) {
    unsigned ticket = atomicAdd(&a.req_ticket[b], 1u);
    s_last = ticket == (unsigned)(len * a.C - 1);
  }
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  if (threadIdx.x < 32) {
    const int lane = threadIdx.x;
    bool accepted = false;
    if (lane < a.k) {
      const int pos = start + (lane < len - 1 ? lane : len - 1);
      const unsigned long long kk = atomicAdd(&a.row_key[pos], 0ull);
      const long long target = argmax_key_index(kk);
      accepted = (target == a.drafts[(long long)b * a.k + lane]) && (lane < len - 1);
    }
    const unsigned acc_mask = __ballot_sync(0xffffffffu, accepted);
    const int n_acc = (~acc_mask) ? __ffs(~acc_mask) - 1 : 32;
    __syncwarp();
    if (lane == 0) {
      const unsigned long long kk = atomicAdd(&a.row_key[start + n_acc], 0ull);
      a.n_accept[b] = n_acc;
      a.tail[b] = argmax_key_index(kk);
    }
    __syncwarp();
    // reset this request's row keys for the next call
    for (int r = lane; r < len; r += 32) atomicExch(&a.row_key[start + r], 0ull);
    if (lane == 0) atomicExch(&a.req_ticket[b], 0u);
  }
}

// ---------------------------------------------------------------------------------------- host side
static int torch_rng_grid(long long numel, const DeviceInfo& info) {
  long long g = (numel + kRngBlock - 1) / kRngBlock;
  long long cap = (long long)info.sm_count * (info.max_threads_per_sm / kRngBlock);
  return (int)(g < cap ? g : cap);
}
static unsigned long long torch_rng_increment(long long numel, const DeviceInfo& info) {
  if (numel <= 0) return 0;
  const long long grid = torch_rng_grid(numel, info);
  return (unsigned long long)(((numel - 1) / (kRngBlock * grid * 4) + 1) * 4);
}

static void choose_chunks(Args& a, const DeviceInfo& info, int ctas_per_sm = kStatsCtasPerSm) {
  // (row, chunk) CTAs of 256 threads, ctas_per_sm resident per SM (the kernel's launch bounds): as many chunks
  // per row as fit one wave (a second, partial wave would run at a fraction of the occupancy), at least one
  const long long slots = (long long)info.sm_count * ctas_per_sm;
  long long C = slots / a.T;
  long long cmax = (a.V + 2047) / 2048;
  if (C > cmax) C = cmax;
  if (C > kMaxChunks) C = kMaxChunks;
  if (C < 1) C = 1;
  const int ve = a.dtype == kF32 ? 4 : 8;
  long long chunk = (a.V + C - 1) / C;
  chunk = (chunk + ve - 1) / ve * ve;
  a.chunk = (int)chunk;
  a.C = (int)((a.V + chunk - 1) / chunk);
}

static void bind_workspace(Args& a, void* ws) {
  Layout L = layout(a.T);
  char* base = static_cast<char*>(ws);
  a.status = reinterpret_cast<int*>(base + L.status);
  a.req_ticket = reinterpret_cast<unsigned*>(base + L.req_ticket);
  a.tail_key = reinterpret_cast<unsigned long long*>(base + L.tail_key);
  a.tail_ticket = reinterpret_cast<unsigned*>(base + L.tail_ticket);
  a.row_key = reinterpret_cast<unsigned long long*>(base + L.row_key);
  a.rows = reinterpret_cast<RowStat*>(base + L.rows);
  a.partial = reinterpret_cast<float2*>(base + L.partial);
  a.desc = reinterpret_cast<ReqDesc*>(base + L.desc);
  a.kept_n = reinterpret_cast<int*>(base + L.kept_n);
  a.kept_ids = reinterpret_cast<int*>(base + L.kept_ids);
}

// torch's grid and grid-stride rounds of the [B, V] exponential draw.
static void exponential_grid(Args& a, const DeviceInfo& info) {
  a.e_numel = (long long)a.B * a.V;
  a.e_grid = torch_rng_grid(a.e_numel, info);
  const long long S = (long long)kRngBlock * a.e_grid;
  a.e_rounds = (int)((a.e_numel - 1) / (S * 4) + 1);
  a.e_sq = (unsigned)(S / a.V);
  a.e_sr = (unsigned)(S % a.V);
}

template <typename T>
static int launch_tail(Args& a, const DeviceInfo& info, bool race, cudaStream_t stream) {
  exponential_grid(a, info);
  if (race) {
    race_kernel<<<a.e_grid, kThreads, 0, stream>>>(a);
  } else if (a.codes) {
    const long long warps = (long long)a.B * ((a.V + kCodeItem - 1) / kCodeItem);
    long long grid = (warps + kThreads / 32 - 1) / (kThreads / 32);
    const long long cap = (long long)info.sm_count * kCodeCtasPerSm;
    if (grid > cap) grid = cap;
    // the descriptors (up to 32 KB) beside the static candidate lists (32 KB) pass the 48 KB default
    const size_t smem = sizeof(TailDesc) * a.B;
    const int smem_max = (int)(sizeof(TailDesc) * kMaxRequests);
    auto kernel = a.codes_vec ? tail_codes_kernel<T, true> : tail_codes_kernel<T, false>;
    if (int st = a.codes_vec ? ensure_dynamic_smem<tail_codes_kernel<T, true>>(smem_max)
                             : ensure_dynamic_smem<tail_codes_kernel<T, false>>(smem_max))
      return st;
    SPECDEC_CUDA_TRY(launch_dependent_smem(kernel, dim3((unsigned)grid), dim3(kThreads), smem, stream, a));
  } else {
    const size_t smem = (sizeof(TailDesc) + sizeof(unsigned long long) + sizeof(float)) * a.B;
    tail_accept_kernel<T><<<a.e_grid, kThreads, smem, stream>>>(a);
  }
  SPECDEC_LAUNCH_CHECK();
  return kOk;
}

// The early-exit pass 1 (stats_early_kernel): clusters of C CTAs, one per request, C as large as one wave of the
// requests allows (at most the portable cluster size; each chunk at least 2048 elements).  kUnsupported when the
// requests alone do not fit one wave (the caller then runs stats_kernel over every row, which has no sequential
// walk to stretch over several waves).
template <typename T>
static int launch_early_stats(Args& a, const DeviceInfo& info, cudaStream_t stream) {
  int per_sm = 0;
  SPECDEC_CUDA_TRY(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, stats_early_kernel<T>, kThreads, 0));
  const long long resident = (long long)per_sm * info.sm_count;
  if (resident < a.B) return kUnsupported;
  long long C = resident / a.B;
  const long long cmax = (a.V + 2047) / 2048;
  if (C > cmax) C = cmax;
  if (C > kEarlyMaxCluster) C = kEarlyMaxCluster;
  a.C = (int)C;   // the kernel picks each step's rows and chunks
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)a.C, (unsigned)a.B);
  cfg.blockDim = dim3(kThreads);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = (unsigned)a.C;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  SPECDEC_CUDA_TRY(cudaLaunchKernelEx(&cfg, stats_early_kernel<T>, a));
  return kOk;
}

// Bytes of the noise codes tail_codes_kernel races over, placed after the fixed layout.
static size_t noise_code_bytes(long long B, long long V) {
  return (((size_t)B * (size_t)V * sizeof(unsigned short)) + 255) & ~size_t(255);
}

static bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

}  // namespace sampler
}  // namespace specdec

using namespace specdec;
using namespace specdec::sampler;

#define SPECDEC_DISPATCH_DTYPE(dtype, ...)                 \
  [&]() -> int {                                          \
    switch (dtype) {                                      \
      case kF32: { using Tx = float; return __VA_ARGS__(); }          \
      case kBF16: { using Tx = __nv_bfloat16; return __VA_ARGS__(); } \
      case kF16: { using Tx = __half; return __VA_ARGS__(); }         \
      default: return set_error(kInvalidArgument, "unknown dtype code %d", dtype); \
    }                                                     \
  }()

extern "C" {

size_t specdec_sampler_workspace_bytes(long long T) { return layout(T).total; }

size_t specdec_accept_workspace_bytes(long long T, long long B, long long V) {
  if (T < 1 || B < 1 || V < 1) return 0;
  return layout(T).total + noise_code_bytes(B, V);
}

unsigned long long specdec_philox_increment(long long numel) {
  DeviceInfo info;
  if (device_info(&info) != kOk) return 0;
  return torch_rng_increment(numel, info);
}

int specdec_probs(const void* logits, int dtype, long long R, long long V, long long rows_per_param,
                  const float* temperature, const long long* top_k, const float* top_p, int max_top_k,
                  int has_top_p, float* probs, void* workspace, size_t workspace_bytes, void* stream) {
  SPECDEC_CHECK_ARG(logits && probs && temperature, "logits, probs and temperature must be non-null");
  SPECDEC_CHECK_ARG(dtype_ok(dtype), "dtype code %d is not f32/bf16/f16", dtype);
  SPECDEC_CHECK_ARG(R >= 1 && R <= kMaxRows, "rows %lld out of range [1, %d]", R, kMaxRows);
  SPECDEC_CHECK_ARG(V >= 1 && V < (1ll << 31), "vocabulary %lld out of range", V);
  SPECDEC_CHECK_ARG(rows_per_param >= 1 && R % rows_per_param == 0, "rows_per_param must divide rows");
  SPECDEC_CHECK_ARG(max_top_k >= 0, "max_top_k must be >= 0");
  if (max_top_k > 0) {
    SPECDEC_CHECK_ARG(top_k != nullptr, "top_k required when max_top_k > 0");
    if (max_top_k > kMaxTopK && V > kMaxTopK)
      return set_error(kUnsupported, "top_k %d above this build's cap %d", max_top_k, kMaxTopK);
  }
  SPECDEC_CHECK_ARG(!has_top_p || top_p != nullptr, "top_p required when has_top_p");
  if (workspace_bytes < layout(R).total)
    return set_error(kWorkspaceTooSmall, "workspace %zu < %zu bytes", workspace_bytes, layout(R).total);
  DeviceInfo info;
  if (int st = device_info(&info)) return st;
  Args a{};
  a.x = logits; a.T = R; a.V = V; a.dtype = dtype; a.probs_mode = 0;
  a.B = (int)(R / rows_per_param); a.k = 0; a.rows_per_param = (int)rows_per_param;
  a.temperature = temperature; a.top_k = top_k; a.top_p = top_p; a.has_top_p = has_top_p;
  a.truncate = max_top_k > 0; a.probs_out = probs;
  choose_chunks(a, info);
  a.vec_ok = aligned16(logits) && ((V * (long long)dtype_bytes(dtype)) % 16 == 0);
  bind_workspace(a, workspace);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  SPECDEC_CUDA_TRY(cudaMemsetAsync(a.status, 0, sizeof(int), s));
  return SPECDEC_DISPATCH_DTYPE(dtype, [&] {
    if (a.truncate) {
      topk_stats_kernel<Tx><<<(unsigned)R, kTopkThreads, 0, s>>>(a, 1);
    } else {
      stats_kernel<Tx><<<dim3(a.C, (unsigned)R), kThreads, 0, s>>>(a, 1);
    }
    SPECDEC_LAUNCH_CHECK();
    write_probs_kernel<Tx><<<dim3(a.C, (unsigned)R), kThreads, 0, s>>>(a, a.truncate ? 1 : 0);
    SPECDEC_LAUNCH_CHECK();
    return (int)kOk;
  });
}

}  // extern "C"

namespace specdec {
namespace sampler {

// The host-side checks of specdec_accept's arguments (everything but the workspace), shared with the
// no-allocation entry point, which must reject a call before it touches its shared scratch.
static int check_accept_args(const void* x, int x_is_probs, int dtype, long long T, long long V, const float* q,
                             const long long* drafts, long long B, long long k, const long long* verified_lens,
                             const float* temperature, const long long* top_k, const float* top_p, int max_top_k,
                             int has_top_p, const long long* n_accept, const long long* tail) {
  SPECDEC_CHECK_ARG(x && q && drafts && n_accept && tail, "x, q, drafts, n_accept and tail must be non-null");
  SPECDEC_CHECK_ARG(dtype_ok(dtype), "dtype code %d is not f32/bf16/f16", dtype);
  SPECDEC_CHECK_ARG(!x_is_probs || dtype == kF32, "probabilities must be fp32");
  SPECDEC_CHECK_ARG(B >= 1 && B <= kMaxRequests, "batch %lld out of range [1, %d]", B, kMaxRequests);
  SPECDEC_CHECK_ARG(k >= 1 && k <= 32, "num_drafts %lld out of range [1, 32]", k);
  SPECDEC_CHECK_ARG(T >= B && T <= kMaxRows && T <= B * (k + 1), "rows %lld inconsistent with B=%lld, k=%lld",
                    T, B, k);
  SPECDEC_CHECK_ARG(verified_lens || T == B * (k + 1), "without verified_lens T must equal B * (k + 1)");
  SPECDEC_CHECK_ARG(V >= 1 && B * V < (1ll << 31), "B * V must stay below 2^31");
  SPECDEC_CHECK_ARG(x_is_probs || temperature, "temperature required for logits");
  SPECDEC_CHECK_ARG(max_top_k >= 0, "max_top_k must be >= 0");
  if (!x_is_probs && max_top_k > 0) {
    SPECDEC_CHECK_ARG(top_k != nullptr, "top_k required when max_top_k > 0");
    if (max_top_k > kMaxTopK && V > kMaxTopK)
      return set_error(kUnsupported, "top_k %d above this build's cap %d", max_top_k, kMaxTopK);
  }
  SPECDEC_CHECK_ARG(!has_top_p || top_p != nullptr, "top_p required when has_top_p");
  return kOk;
}

}  // namespace sampler
}  // namespace specdec

extern "C" {

int specdec_accept(const void* x, int x_is_probs, int dtype, long long T, long long V, const float* q,
                   const long long* drafts, long long B, long long k, const long long* verified_lens,
                   const float* temperature, const long long* top_k, const float* top_p, int max_top_k,
                   int has_top_p, const float* u, const float* E, unsigned long long seed,
                   unsigned long long offset_u, unsigned long long offset_E, long long* n_accept,
                   long long* tail, void* workspace, size_t workspace_bytes, void* stream) {
  if (int st = check_accept_args(x, x_is_probs, dtype, T, V, q, drafts, B, k, verified_lens, temperature, top_k,
                                 top_p, max_top_k, has_top_p, n_accept, tail))
    return st;
  if (workspace_bytes < layout(T).total)
    return set_error(kWorkspaceTooSmall, "workspace %zu < %zu bytes", workspace_bytes, layout(T).total);
  DeviceInfo info;
  if (int st = device_info(&info)) return st;
  Args a{};
  a.x = x; a.T = T; a.V = V; a.dtype = dtype; a.probs_mode = x_is_probs ? 1 : 0;
  a.q = q; a.drafts = drafts; a.B = (int)B; a.k = (int)k; a.lens = verified_lens; a.rows_per_param = 1;
  a.temperature = temperature; a.top_k = top_k; a.top_p = top_p; a.has_top_p = has_top_p;
  a.truncate = (!x_is_probs && max_top_k > 0);
  a.u = u; a.E = E; a.seed = seed; a.offset_u = offset_u; a.offset_E = offset_E;
  a.u_grid = torch_rng_grid(B * k, info);
  a.n_accept = n_accept; a.tail = tail;
  choose_chunks(a, info);
  a.vec_ok = aligned16(x) && ((V * (long long)dtype_bytes(dtype)) % 16 == 0);
  bind_workspace(a, workspace);
  // noise codes when the workspace holds them, the noise is drawn in-kernel at a block boundary (torch's offsets
  // are multiples of 4) and no row truncates (truncating calls race their kept sets, the whole row only rarely)
  const size_t codes_at = layout(T).total;
  if (E == nullptr && (offset_E & 3ull) == 0 && !a.truncate && workspace_bytes >= codes_at + noise_code_bytes(B, V)) {
    a.codes = reinterpret_cast<unsigned short*>(static_cast<char*>(workspace) + codes_at);
    a.codes_vec = a.vec_ok && V % 8 == 0 && aligned16(q) && aligned16(a.codes);
  }
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  SPECDEC_CUDA_TRY(cudaMemsetAsync(a.status, 0, 2 * sizeof(int), s));
  if (a.codes) exponential_grid(a, info);
  // the noise codes: before pass 1, or beside the early-exit pass as its programmatic dependent (the walk leaves
  // most issue slots idle; the codes kernel waits for the pass only at its end)
  auto draw_codes = [&](bool beside) -> int {
    if (!a.codes) return kOk;
    if (beside) {
      SPECDEC_CUDA_TRY(launch_dependent(noise_codes_kernel<false>, dim3((unsigned)(info.sm_count * kNoiseCtasPerSm)),
                                        dim3(kThreads), s, a, static_cast<float*>(nullptr)));
    } else {
      noise_codes_kernel<false><<<a.e_grid, kThreads, 0, s>>>(a, nullptr);
    }
    SPECDEC_LAUNCH_CHECK();
    return kOk;
  };
  return SPECDEC_DISPATCH_DTYPE(dtype, [&] {
    if (a.probs_mode) {
      if (int st = draw_codes(false)) return st;
      decide_probs_kernel<Tx><<<(unsigned)B, 64, 0, s>>>(a);
    } else if (a.truncate) {
      topk_stats_kernel<Tx><<<(unsigned)T, kTopkThreads, 0, s>>>(a, 0);
    } else if (int st = launch_early_stats<Tx>(a, info, s)) {
      if (st != kUnsupported) return st;
      if (int st2 = draw_codes(false)) return st2;
      stats_kernel<Tx><<<dim3(a.C, (unsigned)T), kThreads, 0, s>>>(a, 0);   // more requests than one wave holds
    } else if (int st2 = draw_codes(true)) {
      return st2;
    }
    SPECDEC_LAUNCH_CHECK();
    if (a.truncate) {   // truncating rows: the race over each request's kept tokens, or (gated) over whole rows
      a.e_numel = (long long)a.B * a.V;
      a.e_grid = torch_rng_grid(a.e_numel, info);
      tail_kept_kernel<Tx><<<(unsigned)B, kThreads, 0, s>>>(a);
      SPECDEC_LAUNCH_CHECK();
      a.tail_gate = 1;
    }
    return launch_tail<Tx>(a, info, false, s);
  });
}

int specdec_accept_greedy(const void* logits, int dtype, long long T, long long V, const long long* drafts,
                          long long B, long long k, const long long* verified_lens, long long* n_accept,
                          long long* tail, void* workspace, size_t workspace_bytes, void* stream) {
  SPECDEC_CHECK_ARG(logits && drafts && n_accept && tail, "logits, drafts, n_accept and tail must be non-null");
  SPECDEC_CHECK_ARG(dtype_ok(dtype), "dtype code %d is not f32/bf16/f16", dtype);
  SPECDEC_CHECK_ARG(B >= 1 && B <= kMaxRequests, "batch %lld out of range [1, %d]", B, kMaxRequests);
  SPECDEC_CHECK_ARG(k >= 1 && k <= 32, "num_drafts %lld out of range [1, 32]", k);
  SPECDEC_CHECK_ARG(T >= B && T <= kMaxRows && T <= B * (k + 1), "rows %lld inconsistent with B=%lld, k=%lld",
                    T, B, k);
  SPECDEC_CHECK_ARG(verified_lens || T == B * (k + 1), "without verified_lens T must equal B * (k + 1)");
  SPECDEC_CHECK_ARG(V >= 1 && V < (1ll << 31), "vocabulary %lld out of range", V);
  if (workspace_bytes < layout(T).total)
    return set_error(kWorkspaceTooSmall, "workspace %zu < %zu bytes", workspace_bytes, layout(T).total);
  DeviceInfo info;
  if (int st = device_info(&info)) return st;
  Args a{};
  a.x = logits; a.T = T; a.V = V; a.dtype = dtype; a.drafts = drafts; a.B = (int)B; a.k = (int)k;
  a.lens = verified_lens; a.n_accept = n_accept; a.tail = tail;
  a.vec_ok = aligned16(logits) && ((V * (long long)dtype_bytes(dtype)) % 16 == 0);
  choose_chunks(a, info, kGreedyCtasPerSm);
  bind_workspace(a, workspace);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  SPECDEC_CUDA_TRY(cudaMemsetAsync(a.status, 0, sizeof(int), s));
  return SPECDEC_DISPATCH_DTYPE(dtype, [&] {
    greedy_kernel<Tx><<<dim3(a.C, (unsigned)T), kThreads, 0, s>>>(a);
    SPECDEC_LAUNCH_CHECK();
    return (int)kOk;
  });
}

int specdec_race(const float* weights, long long R, long long V, const float* E, unsigned long long seed,
                 unsigned long long offset_E, long long* out, void* workspace, size_t workspace_bytes,
                 void* stream) {
  SPECDEC_CHECK_ARG(weights && out, "weights and out must be non-null");
  SPECDEC_CHECK_ARG(R >= 1 && R <= kMaxRequests, "rows %lld out of range [1, %d]", R, kMaxRequests);
  SPECDEC_CHECK_ARG(V >= 1 && R * V < (1ll << 31), "R * V must stay below 2^31");
  if (workspace_bytes < layout(R).total)
    return set_error(kWorkspaceTooSmall, "workspace %zu < %zu bytes", workspace_bytes, layout(R).total);
  DeviceInfo info;
  if (int st = device_info(&info)) return st;
  Args a{};
  a.x = weights; a.T = R; a.V = V; a.dtype = kF32; a.probs_mode = 1; a.B = (int)R; a.k = 0;
  a.E = E; a.seed = seed; a.offset_E = offset_E; a.tail = out;
  bind_workspace(a, workspace);
  return launch_tail<float>(a, info, true, static_cast<cudaStream_t>(stream));
}

int specdec_exponential_codes(unsigned long long seed, unsigned long long offset, long long numel,
                              unsigned short* codes, float* values, void* stream) {
  SPECDEC_CHECK_ARG((codes != nullptr) != (values != nullptr), "exactly one of codes and values must be non-null");
  SPECDEC_CHECK_ARG(numel >= 1 && numel < (1ll << 31), "numel %lld out of range", numel);
  SPECDEC_CHECK_ARG((offset & 3ull) == 0, "offset %llu is not a multiple of 4", offset);
  DeviceInfo info;
  if (int st = device_info(&info)) return st;
  Args a{};
  a.B = 1; a.V = numel; a.seed = seed; a.offset_E = offset; a.codes = codes;
  exponential_grid(a, info);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (codes) {
    noise_codes_kernel<false><<<a.e_grid, kThreads, 0, s>>>(a, nullptr);
  } else {
    noise_codes_kernel<true><<<a.e_grid, kThreads, 0, s>>>(a, values);
  }
  SPECDEC_LAUNCH_CHECK();
  return kOk;
}

}  // extern "C"

// ---------------------------------------------------------------------------------------- no-allocation entry
// specdec_accept for callers that cannot allocate device memory at all, not even the workspace the other entry
// points take: a plugin loaded into a host process that owns the whole device memory budget and forbids its
// extensions from calling cudaMalloc, or a caller on a latency-critical path where cudaMalloc (which may
// synchronise the device) is not allowed.  Its scratch is a fixed array in the library's own device memory,
// sized for at most kNoAllocMaxRows verified rows; every GPU that loads the library holds it until exit.
namespace specdec {
namespace sampler {

constexpr long long kNoAllocMaxRows = 1024;
constexpr size_t kNoAllocBytes = layout(kNoAllocMaxRows).total;            // about 2.8 MB
constexpr size_t kNoAllocHeaderBytes = layout(1).rows;                     // status, tickets and keys

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocBytes];

// The array's device address, looked up once per device with that device current (the first call on a device
// does this set-up, so it should come before any stream capture).  In host code the array's name is only a
// host-side stand-in, so kernels always receive this looked-up address.  Host threads calling at once serialise
// on the first lookup per device only.  A cudaDeviceReset ends the context that owns the array: the cached
// address is then stale, and this entry point must not be called again in that process.
static int noalloc_scratch(void** out) {
  static std::atomic<void*> addr[kMaxDevices];
  static std::mutex mu;
  int dev = 0;
  SPECDEC_CUDA_TRY(cudaGetDevice(&dev));
  if (dev < 0 || dev >= kMaxDevices) return set_error(kInvalidArgument, "device ordinal %d out of range", dev);
  void* p = addr[dev].load(std::memory_order_acquire);
  if (p == nullptr) {
    std::lock_guard<std::mutex> lock(mu);
    p = addr[dev].load(std::memory_order_relaxed);
    if (p == nullptr) {
      const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
      if (e != cudaSuccess)
        return set_error(kCudaError, "cudaGetSymbolAddress of the no-allocation scratch failed: %s",
                         cudaGetErrorString(e));
      addr[dev].store(p, std::memory_order_release);
    }
  }
  *out = p;
  return kOk;
}

}  // namespace sampler
}  // namespace specdec

extern "C" int specdec_accept_noalloc(const void* x, int x_is_probs, int dtype, long long T, long long V,
                                      const float* q, const long long* drafts, long long B, long long k,
                                      const long long* verified_lens, const float* temperature,
                                      const long long* top_k, const float* top_p, int max_top_k, int has_top_p,
                                      const float* u, const float* E, unsigned long long seed,
                                      unsigned long long offset_u, unsigned long long offset_E,
                                      long long* n_accept, long long* tail, void* stream) {
  using namespace specdec::sampler;
  if (T > kNoAllocMaxRows)
    return set_error(kUnsupported,
                     "specdec_accept_noalloc takes at most %lld verified rows (got %lld): its fixed scratch holds "
                     "%zu bytes; use specdec_accept with a caller workspace for more",
                     kNoAllocMaxRows, T, kNoAllocBytes);
  // A call the host rejects leaves the shared array alone (another call's work may be using it).
  if (int st = check_accept_args(x, x_is_probs, dtype, T, V, q, drafts, B, k, verified_lens, temperature, top_k,
                                 top_p, max_top_k, has_top_p, n_accept, tail))
    return st;
  void* scratch = nullptr;
  if (int st = noalloc_scratch(&scratch)) return st;
  // The array keeps the previous call's contents: clear the tickets and keys that must start at zero (a call
  // that stopped part-way could have left some behind).  Calls whose work overlaps on the GPU race on the array.
  SPECDEC_CUDA_TRY(cudaMemsetAsync(scratch, 0, kNoAllocHeaderBytes, static_cast<cudaStream_t>(stream)));
  return specdec_accept(x, x_is_probs, dtype, T, V, q, drafts, B, k, verified_lens, temperature, top_k, top_p,
                        max_top_k, has_top_p, u, E, seed, offset_u, offset_E, n_accept, tail, scratch,
                        kNoAllocBytes, stream);
}
