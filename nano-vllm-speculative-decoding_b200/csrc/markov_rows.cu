// Kernel (3): DSpark's in-block Markov row sampling, one row step at a time, for sm_100a.
//
// Reference (nano-vllm-speculative-decoding, nanovllm/engine/speculative.py:163-184, DFlashDrafter._markov_rows):
//   for row in range(k):
//       row_logits = logits[:, row] + markov_head(prev)                 (bf16 add, rounded)
//       greedy:      prev = argmax(row_logits)
//       candidates:  values, ids = row_logits.topk(C)                    (C = max_top_k + 64, every row truncates)
//                    probs = probs_from_logits(values, sampling)         (temperature, top-k with ties, top-p)
//                    prev = ids[race(probs, noise[:, row])]              (argmax probs / noise, first index)
//                    draft_probs[:, row].scatter_(-1, ids, probs)
//       drafts[:, row] = prev
// markov_head(prev) = W2 . W1[prev] is a plain GEMM [B, r] x [r, V] left to cuBLAS between steps; this kernel
// does everything else of a step for every row at once and writes the next step's W1[prev] rows.
//
// Design: one 512-thread CTA per batch row (the rows of a step are independent; the steps are not).  The biased
// row (V bf16 logits + V bias values) is re-read from L2 by every pass: a 12-bit and a 4-bit radix pass on the
// bf16 ordered key (warp-aggregated histogram atomics) find the C-th largest value, one pass collects the values above it, one warp-ordered pass takes
// the tied values by ascending token id (ballot ranks), then a bitonic sort of <= 1024 64-bit keys (value desc,
// id asc) orders the candidates.  The candidate softmax / truncation / race run in shared memory.  Candidate
// order among equal values is ascending token id (torch.topk leaves it unspecified).
#include "common.cuh"

#include <math.h>

namespace specdec {
namespace markov {

constexpr int kThreads = 512;
constexpr int kWarps = kThreads / 32;
constexpr int kMaxCand = 1024;
constexpr int kSelCap = 4096;          // elements the thread-maxima bound may admit before the radix fallback

struct Args {
  const void* logits;       // [B, k, V] (dtype ldt); with no bias, this step's biased rows [B, V]
  int ldt;
  const void* bias;         // [B, V] (dtype bdt) this step's Markov bias, or null (logits arrive biased)
  int bdt;
  int B, k, V, j, C, greedy, round_bf16;
  const float* temperature; // [B]
  const long long* top_k;   // [B]
  const float* top_p;       // [B] or null
  int max_top_k, has_top_p;
  const float* noise;       // [B, k, noise_width]
  int noise_width;
  long long* drafts;        // [B, k]
  float* probs;             // [B, k, V] or null (greedy)
  long long* prev_out;      // [B]
  const __nv_bfloat16* w1;  // [V, rank] or null
  int rank;
  __nv_bfloat16* e_next;    // [B, rank]
  int* err;
  int vec;                  // bf16 logits and bias, V % 8 == 0, 16-byte aligned rows: vector loads
  int P;                    // CTAs per row (grid.x); piece p covers groups [p * gchunk, (p + 1) * gchunk)
  int gchunk;               // groups of 8 elements per piece
  unsigned* tickets;        // [B] arrivals per row; the last CTA resets its entry
  unsigned long long* best; // [B] greedy argmax keys; reset by the last CTA
  unsigned long long* keys; // [B][P][C] each piece's top C keys (value << 32 | ~id), descending
  int* last_ids;            // [B][k][C] ids this row scattered q to last time (-1: none), or null: the caller
                            // zeroed probs; with it, probs stays zero elsewhere and only these are cleared
};

// Workspace: tickets [kMaxRowsWs] and greedy keys [kMaxRowsWs] (zeroed once, self-cleaning) at fixed offsets, so
// calls of any batch size share one workspace, then the pieces' candidate keys.
constexpr long long kMaxRowsWs = 65536;
constexpr long long kBestOffset = kMaxRowsWs * 4;
__host__ __device__ inline long long ws_head_bytes(int) { return kMaxRowsWs * (4 + 8); }

__device__ __forceinline__ float load_any(const void* p, int dt, long long i) {
  if (dt == kF32) return reinterpret_cast<const float*>(p)[i];
  if (dt == kBF16) return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p)[i]);
  return __half2float(reinterpret_cast<const __half*>(p)[i]);
}

__device__ __forceinline__ float row_value(const Args& a, long long lrow, long long brow, int v) {
  float x = load_any(a.logits, a.ldt, lrow + v);
  if (a.bias) x += load_any(a.bias, a.bdt, brow + v);
  if (a.round_bf16) x = __bfloat162float(__float2bfloat16_rn(x));
  return x;
}

// The biased values of the 8 consecutive elements of group g (16-byte loads on the vector path); returns how
// many of them exist.
__device__ __forceinline__ int load_group(const Args& a, long long lrow, long long brow, int g, float (&x)[8]) {
  const int v0 = g * 8;
  const int n = min(8, a.V - v0);
  if (a.vec && n == 8) {
    float l8[8], b8[8];
    unpack16_bf16(ldg16(reinterpret_cast<const __nv_bfloat16*>(a.logits) + lrow + v0), l8);
    if (a.bias) {
      unpack16_bf16(ldg16(reinterpret_cast<const __nv_bfloat16*>(a.bias) + brow + v0), b8);
#pragma unroll
      for (int e = 0; e < 8; ++e) x[e] = __bfloat162float(__float2bfloat16_rn(l8[e] + b8[e]));
    } else {
#pragma unroll
      for (int e = 0; e < 8; ++e) x[e] = l8[e];
    }
  } else {
#pragma unroll
    for (int e = 0; e < 8; ++e) x[e] = e < n ? row_value(a, lrow, brow, v0 + e) : -INFINITY;
  }
  return n;
}

// Eight bf16 sums, pairwise (one rounding each).
__device__ __forceinline__ uint4 bf16x8_add(const uint4& x, const uint4& y) {
  auto add = [](unsigned a, unsigned b) {
    const __nv_bfloat162 r = __hadd2(as_h2<__nv_bfloat162>(a), as_h2<__nv_bfloat162>(b));
    unsigned u;
    memcpy(&u, &r, sizeof(u));
    return u;
  };
  return make_uint4(add(x.x, y.x), add(x.y, y.y), add(x.z, y.z), add(x.w, y.w));
}

// 1-based rank `rank` among the counted elements: digit d with above(d) < rank <= above(d) + hist[d].
__device__ void pick_digit(const unsigned* hist, int nbins, int rank, int* s_digit, int* s_above) {
  __shared__ int warp_tot[kWarps];
  const int per = nbins / kThreads > 0 ? nbins / kThreads : 1;
  const int owners = nbins / per;
  int local = 0;
  if (threadIdx.x < owners)
    for (int i = 0; i < per; ++i) local += hist[threadIdx.x * per + i];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int incl = local;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    int n = __shfl_down_sync(0xffffffffu, incl, o);
    if (lane + o < 32) incl += n;
  }
  if (lane == 0) warp_tot[warp] = incl;
  __syncthreads();
  int above = incl - local;
  for (int w = warp + 1; w < kWarps; ++w) above += warp_tot[w];
  if (threadIdx.x < owners) {
    for (int i = per - 1; i >= 0; --i) {
      const int h = hist[threadIdx.x * per + i];
      if (above < rank && rank <= above + h) {
        *s_digit = threadIdx.x * per + i;
        *s_above = above;
      }
      above += h;
    }
  }
  __syncthreads();
}

__global__ void __launch_bounds__(kThreads, 2) markov_step_kernel(const Args a) {
  __shared__ unsigned long long sel[kSelCap];            // fast-path candidates, the pieces' keys when merging;
  unsigned* hist = reinterpret_cast<unsigned*>(sel);      // the radix fallback's histogram (4096 bins) reuses it
  __shared__ unsigned long long cand[kMaxCand];
  __shared__ int s_sel;
  __shared__ float cprob[kMaxCand];
  __shared__ int s_digit, s_above, s_cnt, s_prev, s_last;
  __shared__ int warp_ties[kWarps], warp_base[kWarps];
  __shared__ unsigned long long s_red[kWarps];
  __shared__ float s_thr, s_z;

  const int piece = blockIdx.x, b = blockIdx.y;
  const int V = a.V;
  const long long qrow = ((long long)b * a.k + a.j) * V;           // row (b, j) of q [B, k, V]
  const long long lrow = a.bias ? qrow : (long long)b * V;          // the logits' row: [B, k, V] or biased [B, V]
  const long long brow = (long long)b * V;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int C = a.C;

  // This CTA's piece of the row: groups [g_lo, g_lo + ngroups) of 8 elements.  Passes over it read 2 x 32
  // consecutive groups per warp per iteration (two 16-byte loads of logits and bias per group in flight per
  // thread); trip counts are warp-uniform.  Ids below are piece-local (group * 8 + e) until published.
  const int ngroups_row = (V + 7) / 8;
  const int g_lo = piece * a.gchunk;
  const int ngroups = min(ngroups_row - g_lo, a.gchunk);
  auto load = [&](int g, float (&x)[8]) { return load_group(a, lrow, brow, g_lo + g, x); };
  if (a.greedy) {
    unsigned long long best = 0ull;
    for (int gb = warp * 64; gb < ngroups; gb += kWarps * 64) {
      float x0[8], x1[8];
      const int g0 = gb + lane, g1 = gb + 32 + lane;
      const int n0 = g0 < ngroups ? load(g0, x0) : 0;
      const int n1 = g1 < ngroups ? load(g1, x1) : 0;
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        if (e < n0) { const unsigned long long k0 = argmax_key(x0[e], (unsigned)((g_lo + g0) * 8 + e)); best = k0 > best ? k0 : best; }
        if (e < n1) { const unsigned long long k1 = argmax_key(x1[e], (unsigned)((g_lo + g1) * 8 + e)); best = k1 > best ? k1 : best; }
      }
    }
    best = warp_max_u64(best);
    if (lane == 0) s_red[warp] = best;
    __syncthreads();
    if (threadIdx.x == 0) {
      unsigned long long m = 0ull;
      for (int w = 0; w < kWarps; ++w) m = s_red[w] > m ? s_red[w] : m;
      atomicMax(&a.best[b], m);
    }
  } else {
    // ---- the piece's top C, descending: thread-maxima bound + collect + sort, or an exact radix select
    int fast = -1;
    if (C <= kThreads) {
      unsigned long long* top = nullptr;
      if (a.vec) {
        // bf16 logits and bias: the biased row as packed pairs.  The bf16x2 add rounds the exact sum once, which
        // is what torch's bf16 add gives (its fp32 sum of two bf16 values is exact, or off only far below half
        // a bf16 ulp of the larger term).
        const uint4* lg = reinterpret_cast<const uint4*>(reinterpret_cast<const __nv_bfloat16*>(a.logits) + lrow) + g_lo;
        if (a.bias) {
          const uint4* bg =
              reinterpret_cast<const uint4*>(reinterpret_cast<const __nv_bfloat16*>(a.bias) + brow) + g_lo;
          fast = select_by_thread_max_x16<kThreads, 4, __nv_bfloat162>(
              ngroups, C, [&](int g) { return bf16x8_add(__ldg(lg + g), __ldg(bg + g)); }, sel, kSelCap, &s_sel,
              &top);
        } else {                      // the row arrives biased (specdec_markov_bias wrote it)
          fast = select_by_thread_max_x16<kThreads, 4, __nv_bfloat162>(
              ngroups, C, [&](int g) { return __ldg(lg + g); }, sel, kSelCap, &s_sel, &top);
        }
      } else {
        fast = select_by_thread_max<kThreads, 1>(ngroups, C, load, sel, kSelCap, &s_sel, &top);
      }
      if (fast >= 0)
        for (int i = threadIdx.x; i < C; i += kThreads) cand[i] = top[i];
    }
    if (fast < 0) {
    // ---- radix select of the C-th largest ordered key
    unsigned prefix = 0, pmask = 0;
    int rank = C;
    const int npass = a.round_bf16 ? 2 : 3;
    const int shifts_bf[2] = {20, 16}, widths_bf[2] = {12, 4};
    const int shifts_f[3] = {20, 8, 0}, widths_f[3] = {12, 12, 8};
    for (int p = 0; p < npass; ++p) {
      const int shift = a.round_bf16 ? shifts_bf[p] : shifts_f[p];
      const int width = a.round_bf16 ? widths_bf[p] : widths_f[p];
      const int nb = 1 << width;
      for (int i = threadIdx.x; i < nb; i += kThreads) hist[i] = 0;
      __syncthreads();
      for (int gb = warp * 64; gb < ngroups; gb += kWarps * 64) {
        float x0[8], x1[8];
        const int g0 = gb + lane, g1 = gb + 32 + lane;
        const int n0 = g0 < ngroups ? load(g0, x0) : 0;
        const int n1 = g1 < ngroups ? load(g1, x1) : 0;
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const unsigned k0 = ordered_key(x0[e]);
          warp_hist_add(hist, (k0 >> shift) & (nb - 1), e < n0 && (k0 & pmask) == prefix);
          const unsigned k1 = ordered_key(x1[e]);
          warp_hist_add(hist, (k1 >> shift) & (nb - 1), e < n1 && (k1 & pmask) == prefix);
        }
      }
      __syncthreads();
      pick_digit(hist, nb, rank, &s_digit, &s_above);
      prefix |= (unsigned)s_digit << shift;
      pmask |= (unsigned)(nb - 1) << shift;
      rank -= s_above;
      __syncthreads();
    }
    // bf16 values: the low 16 key bits follow from the sign (0 for positive, all ones for negative)
    const unsigned key_c = a.round_bf16 ? (prefix | ((prefix & 0x80000000u) ? 0u : 0xffffu)) : prefix;
    const int need_ties = rank;          // tied values to take, by ascending id
    const int n_gt = C - rank;
    // ---- values above the C-th (any order) and per-warp tie counts over contiguous group ranges
    if (threadIdx.x == 0) s_cnt = 0;
    __syncthreads();
    const int gspan = ((ngroups + kWarps - 1) / kWarps + 31) / 32 * 32;
    const int glo = warp * gspan, ghi = min(ngroups, glo + gspan);
    int ties = 0;
    for (int gb = glo; gb < ghi; gb += 32) {
      const int g = gb + lane;
      float x[8];
      const int n = g < ghi ? load(g, x) : 0;
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        if (e < n) {
          const unsigned key = ordered_key(x[e]);
          if (key > key_c) {
            const int slot = atomicAdd(&s_cnt, 1);
            if (slot < kMaxCand)
              cand[slot] = (static_cast<unsigned long long>(key) << 32) | (0xffffffffu - (unsigned)(g * 8 + e));
          }
          ties += key == key_c;
        }
      }
    }
    ties = __reduce_add_sync(0xffffffffu, ties);
    if (lane == 0) warp_ties[warp] = ties;
    __syncthreads();
    if (threadIdx.x == 0) {
      int run = 0;
      for (int w = 0; w < kWarps; ++w) {
        warp_base[w] = run;
        run += warp_ties[w];
      }
    }
    __syncthreads();
    // ---- the first need_ties tied values by ascending id (lane order = id order within a step)
    if (need_ties > 0 && warp_base[warp] < need_ties) {
      int seen = warp_base[warp];
      for (int gb = glo; gb < ghi && seen < need_ties; gb += 32) {
        const int g = gb + lane;
        float x[8];
        const int n = g < ghi ? load(g, x) : 0;
        unsigned mask = 0;
#pragma unroll
        for (int e = 0; e < 8; ++e)
          if (e < n && ordered_key(x[e]) == key_c) mask |= 1u << e;
        const int cnt = __popc(mask);
        int incl = cnt;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const int nb = __shfl_up_sync(0xffffffffu, incl, o);
          if (lane >= o) incl += nb;
        }
        int r = seen + incl - cnt;
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          if (mask & (1u << e)) {
            if (r < need_ties) cand[n_gt + r] = (static_cast<unsigned long long>(key_c) << 32) |
                                                (0xffffffffu - (unsigned)(g * 8 + e));
            ++r;
          }
        }
        seen += __shfl_sync(0xffffffffu, incl, 31);
      }
    }
    // ---- sort descending (value desc, id asc); pad with 0 keys
    int P2 = 1;
    while (P2 < C) P2 <<= 1;
    for (int i = C + threadIdx.x; i < P2; i += kThreads) cand[i] = 0ull;
    __syncthreads();
    block_sort_desc_u64(cand, P2);
    }  // radix fallback
    __syncthreads();
    // ---- publish the piece's top C with row-global ids (the low word holds ~id)
    unsigned long long* out = a.keys + ((long long)b * a.P + piece) * C;
    const unsigned shift_ids = (unsigned)g_lo * 8u;
    for (int i = threadIdx.x; i < C; i += kThreads) out[i] = cand[i] ? cand[i] - shift_ids : 0ull;
  }
  // ---- the last CTA of the row finishes it
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) {
    const unsigned ticket = atomicAdd(&a.tickets[b], 1u);
    s_last = ticket == (unsigned)(a.P - 1);
    if (s_last) a.tickets[b] = 0u;
  }
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  if (a.greedy) {
    if (threadIdx.x == 0) s_prev = (int)argmax_key_index(atomicExch(&a.best[b], 0ull));
    __syncthreads();
  } else {
    // ---- merge: the row's top C among the pieces' sorted top C lists.  Keys are distinct (value, then ~id), so
    // a key's rank in the union is its index in its own list plus, per other list, the count of larger keys
    // there (binary search); ties stay by ascending id because the keys say so.
    const int n = a.P * C;
    const unsigned long long* in = a.keys + (long long)b * a.P * C;
    for (int i = threadIdx.x; i < n; i += kThreads) sel[i] = __ldcg(in + i);
    __syncthreads();
    for (int t = threadIdx.x; t < n; t += kThreads) {
      const int p = t / C, i = t - p * C;
      const unsigned long long key = sel[t];
      int r = i;
      for (int q = 0; q < a.P; ++q) {
        if (q == p) continue;
        const unsigned long long* list = sel + q * C;
        int lo = 0, hi = C;
        while (lo < hi) {
          const int mid = (lo + hi) >> 1;
          if (list[mid] > key) lo = mid + 1; else hi = mid;
        }
        r += lo;
      }
      if (r < C) cand[r] = key;
    }
    __syncthreads();
    // ---- probs_from_logits over the C candidates (spec_sampler.py:65-96 on a [C] row)
    const float temp = a.temperature[b];
    if (threadIdx.x == 0) {
      const int nc = a.max_top_k < C ? a.max_top_k : C;
      const long long tk = a.top_k ? a.top_k[b] : 0;
      float thr = -INFINITY;
      if (a.max_top_k > 0 && tk > 0) {
        const int eff_k = (int)tk;
        const int kidx = (eff_k - 1) < (nc - 1) ? (eff_k - 1) : (nc - 1);
        auto scaled = [&](int i) { return __fdiv_rn(key_to_float((unsigned)(cand[i] >> 32)), temp); };
        thr = scaled(kidx);
        if (a.has_top_p) {
          const float tp = a.top_p[b];
          const int kk = eff_k < nc ? eff_k : nc;
          const float c0 = scaled(0);
          float z = 0.0f;
          for (int i = 0; i < kk; ++i) z += expf(scaled(i) - c0);
          float cum = 0.0f;
          int kept = 0;
          for (int i = 0; i < kk; ++i) {
            const float nu = __fdiv_rn(expf(scaled(i) - c0), z);
            cum += nu;
            if (cum - nu < tp) ++kept;
          }
          if (kept >= 1 && kept <= kk) thr = fmaxf(thr, scaled(kept - 1));
        }
      }
      s_thr = thr;
    }
    __syncthreads();
    const float thr = s_thr;
    const float m = __fdiv_rn(key_to_float((unsigned)(cand[0] >> 32)), temp);
    float zl = 0.0f;
    for (int i = threadIdx.x; i < C; i += kThreads) {
      const float f = __fdiv_rn(key_to_float((unsigned)(cand[i] >> 32)), temp);
      const float e = f >= thr ? expf(f - m) : 0.0f;
      cprob[i] = e;
      zl += e;
    }
    zl = warp_sum_f32(zl);
    __shared__ float zred[kWarps];
    if (lane == 0) zred[warp] = zl;
    __syncthreads();
    if (threadIdx.x == 0) {
      float z = 0.0f;
      for (int w = 0; w < kWarps; ++w) z += zred[w];
      s_z = z;
    }
    __syncthreads();
    const float z = s_z;
    // ---- race over the candidates with their noise; scatter q (after clearing the previous call's entries of
    // this row when probs is a persistent buffer)
    const float* noise = a.noise + ((long long)b * a.k + a.j) * a.noise_width;
    int* last = a.last_ids ? a.last_ids + ((long long)b * a.k + a.j) * C : nullptr;
    if (last) {
      for (int i = threadIdx.x; i < C; i += kThreads) {
        const int old = last[i];
        if (old >= 0 && old < V) a.probs[qrow + old] = 0.0f;
      }
      __syncthreads();
    }
    unsigned long long best = 0ull;
    for (int i = threadIdx.x; i < C; i += kThreads) {
      const float p = __fdiv_rn(cprob[i], z);
      const int id = (int)(0xffffffffu - (unsigned)(cand[i] & 0xffffffffull));
      a.probs[qrow + id] = p;
      if (last) last[i] = id;
      float ratio = __fdiv_rn(p, noise[i]);
      if (ratio == 0.0f) ratio = 0.0f;
      const unsigned long long key = argmax_key(ratio, (unsigned)i);
      best = key > best ? key : best;
    }
    best = warp_max_u64(best);
    if (lane == 0) s_red[warp] = best;
    __syncthreads();
    if (threadIdx.x == 0) {
      unsigned long long mk = 0ull;
      for (int w = 0; w < kWarps; ++w) mk = s_red[w] > mk ? s_red[w] : mk;
      const int winner = (int)argmax_key_index(mk);
      s_prev = (int)(0xffffffffu - (unsigned)(cand[winner] & 0xffffffffull));
    }
    __syncthreads();
  }
  const int prev = s_prev;
  if (threadIdx.x == 0) {
    a.drafts[(long long)b * a.k + a.j] = prev;
    a.prev_out[b] = prev;
  }
  if (a.w1)
    for (int i = threadIdx.x; i < a.rank; i += kThreads) a.e_next[(long long)b * a.rank + i] = a.w1[(long long)prev * a.rank + i];
}

// CTAs per row: enough to fill every SM twice over the batch, the pieces' keys fitting the merge buffer and
// each piece keeping at least 4096 elements (so the thread-maxima bound sees every thread, and every piece has
// C real keys, all distinct, for the merge's ranks).
static int pieces_per_row(int B, int V, int C, int greedy, int sm_count) {
  long long P = (2LL * sm_count) / B;
  const long long by_len = V / 4096;
  if (P > by_len) P = by_len;
  if (!greedy) {
    const long long by_merge = kSelCap / C;
    if (P > by_merge) P = by_merge;
  }
  if (P < 1) P = 1;
  return (int)P;
}

static long long workspace_bytes(int B, int V, int C, int greedy, int sm_count) {
  const int P = pieces_per_row(B, V, C, greedy, sm_count);
  return ws_head_bytes(B) + (greedy ? 0 : (long long)B * P * C * 8);
}

}  // namespace markov
}  // namespace specdec

using namespace specdec;

extern "C" {

int specdec_markov_step(const void* logits, int logits_dtype, const void* bias, int bias_dtype, int B, int k, int V,
                        int row, int candidates, int greedy, int round_bf16, const float* temperature,
                        const long long* top_k, const float* top_p, int max_top_k, int has_top_p, const float* noise,
                        int noise_width, long long* drafts, float* probs, long long* prev_out, const void* w1,
                        int rank, void* e_next, int* last_ids, void* workspace, long long workspace_bytes, int* err,
                        void* stream) {
  using namespace markov;
  SPECDEC_CHECK_ARG(logits && drafts && prev_out && err && workspace, "null pointer argument");
  SPECDEC_CHECK_ARG((reinterpret_cast<uintptr_t>(workspace) & 255) == 0, "workspace must be 256-byte aligned");
  SPECDEC_CHECK_ARG(dtype_ok(logits_dtype) && (!bias || dtype_ok(bias_dtype)), "unknown dtype code");
  SPECDEC_CHECK_ARG(B >= 1 && B <= 65535 && k >= 1 && V >= 1 && row >= 0 && row < k, "bad sizes");
  SPECDEC_CHECK_ARG(!w1 || (e_next && rank >= 1), "w1 needs e_next and rank");
  if (!greedy) {
    SPECDEC_CHECK_ARG(temperature && probs && noise, "random rows need temperature, probs and noise");
    SPECDEC_CHECK_ARG(candidates >= 1 && candidates <= V, "candidates %d out of range", candidates);
    if (candidates > kMaxCand)
      return set_error(kUnsupported, "%d candidates above this build's cap %d", candidates, kMaxCand);
    SPECDEC_CHECK_ARG(noise_width >= candidates, "noise width %d < candidates %d", noise_width, candidates);
    SPECDEC_CHECK_ARG(!has_top_p || top_p, "top_p required when has_top_p");
    SPECDEC_CHECK_ARG(max_top_k == 0 || top_k, "top_k required when max_top_k > 0");
  }
  Args a{};
  a.logits = logits; a.ldt = logits_dtype; a.bias = bias; a.bdt = bias_dtype;
  a.B = B; a.k = k; a.V = V; a.j = row; a.C = candidates; a.greedy = greedy; a.round_bf16 = round_bf16;
  a.temperature = temperature; a.top_k = top_k; a.top_p = top_p; a.max_top_k = max_top_k; a.has_top_p = has_top_p;
  a.noise = noise; a.noise_width = noise_width; a.drafts = drafts; a.probs = probs; a.prev_out = prev_out;
  a.w1 = static_cast<const __nv_bfloat16*>(w1); a.rank = rank; a.e_next = static_cast<__nv_bfloat16*>(e_next);
  a.err = err;
  a.last_ids = greedy ? nullptr : last_ids;
  a.vec = logits_dtype == kBF16 && (!bias || bias_dtype == kBF16) && V % 8 == 0 &&
          ((reinterpret_cast<uintptr_t>(logits) | reinterpret_cast<uintptr_t>(bias)) & 15) == 0;
  DeviceInfo info;
  if (int st = device_info(&info)) return st;
  const int C = greedy ? 1 : candidates;
  const long long need = markov::workspace_bytes(B, V, C, greedy, info.sm_count);
  if (workspace_bytes < need)
    return set_error(kWorkspaceTooSmall, "Markov workspace of %lld bytes, %lld needed", workspace_bytes, need);
  a.P = pieces_per_row(B, V, C, greedy, info.sm_count);
  a.gchunk = ((V + 7) / 8 + a.P - 1) / a.P;
  char* ws = static_cast<char*>(workspace);
  a.tickets = reinterpret_cast<unsigned*>(ws);
  a.best = reinterpret_cast<unsigned long long*>(ws + kBestOffset);
  a.keys = reinterpret_cast<unsigned long long*>(ws + ws_head_bytes(B));
  markov_step_kernel<<<dim3(a.P, B), kThreads, 0, static_cast<cudaStream_t>(stream)>>>(a);
  SPECDEC_LAUNCH_CHECK();
  return kOk;
}

long long specdec_markov_workspace_bytes(int B, int V, int candidates, int greedy) {
  DeviceInfo info;
  if (B < 1 || V < 1 || (!greedy && candidates < 1) || device_info(&info) != kOk) return -1;
  return markov::workspace_bytes(B, V, greedy ? 1 : candidates, greedy, info.sm_count);
}

}  // extern "C"
