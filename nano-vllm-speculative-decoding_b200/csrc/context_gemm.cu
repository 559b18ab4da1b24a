// Kernel (5): the draft context path's projections on tcgen05, for sm_100a.
//
// Reference behaviour (nano-vllm-speculative-decoding):
//   DFlashDraftModel.context_features   nanovllm/models/dflash.py:84-86   hidden_norm(fc(aux)): fc is a linear
//                                       map [T, 5 H] -> [T, H] (bf16 weights, no bias), output rounded to bf16
//   DFlashDraftModel.store_context_kv   nanovllm/models/dflash.py:88-96   per draft layer k, v = F.linear(c, W_kv)
//
// out[T, O] = x[T, K] . w[O, K]^T with bf16 operands, fp32 accumulation and one rounding to bf16, the shape
// of a projection of a few hundred tokens against a weight matrix of many rows.  Design (B200):
//   * swap-AB on the tensor core: D[128 weight rows x N tokens] = W_tile . X^T, A = the weight tile (K-major,
//     128-byte swizzle), B = the token rows (K-major), fp32 accumulators in tensor memory; every token of the call
//     in one accumulator (N = n_sub x tn <= 288 columns, one or two M128 UMMAs per 16-deep k step), so each
//     weight byte crosses HBM once;
//   * persistent stream-K: the (128-row tile, 64-deep k block) units form one sequence cut into equal shares, one
//     per SM, so every SM does the same work whatever the tile count; a tile cut between CTAs is published as
//     fp32 pieces and the last CTA to arrive (atomic counter, self-resetting) sums them in CTA order (the result
//     does not depend on arrival order);
//   * warp 0 streams the W and X tiles by TMA through a 4-stage ring, warp 1 owns the tensor memory and issues
//     the MMAs, warps 4-7 drain the accumulator (one TMEM lane quadrant each) and write bf16 rows.
// Every wait is bounded and reports through an error word.
#include "common.cuh"
#include "sm100.cuh"
#include "specdec_b200.h"

#include <cudaTypedefs.h>

namespace specdec {
namespace gemm {

using namespace sm100;

constexpr int kThreads = 256;                 // warps 0 TMA, 1 TMEM + MMA, 2-3 idle, 4-7 epilogue
constexpr int kBlockK = 64;                   // k elements per stage: 128-byte rows, 128-byte swizzle
constexpr int kStages = 4;
constexpr int kTileM = 128;
constexpr int kMaxCols = 288;                 // tokens per call (n_sub * tn)
constexpr int kABytes = kTileM * kBlockK * 2;                 // 16 KB
constexpr int kMaxBBytes = kMaxCols * kBlockK * 2;           // 36 KB
constexpr int kStageBytes = kABytes + kMaxBBytes;            // 52 KB
constexpr int kErrTimeout = 16;

struct Args {
  int mode;                    // 0: out = the product; 1: draft context K/V (tiles = (layer, K|V, head) of 128);
                               // 2: DSpark's biased row, out = bf16(bf16(product) + logits)
  int T, O, K;                 // tokens, output features, reduction length
  int n_sub, tn;               // UMMAs per k step and their width: n_sub * tn >= T, tn % 16 == 0, tn <= 256
  int kblocks;                 // K / 64
  int whole_tiles;             // 1: every CTA takes whole tiles (more tiles than CTAs), no split tiles
  int nbuf;                    // accumulators in tensor memory: 2 (MMAs of the next tile overlap this tile's
                               // epilogue) when whole tiles of <= 128 columns, else 1
  __nv_bfloat16* out;          // [T, O] (row stride out_stride)
  long long out_stride;
  int* counters;               // [O / 128] arrivals at split tiles (zero between launches)
  float* partial;              // [2 * gridDim.x][n_sub * tn][128] fp32 pieces: slot 2c = CTA c's first tile
  int* err;
  // mode 1 (store_context_kv): tile m is layer m / (2 Hkv), K heads then V heads of that layer
  int Hkv;
  const __nv_bfloat16* k_norm; // [layers][128] (layer stride k_norm_stride)
  long long k_norm_stride;
  const float* cos_sin;        // [max_position][128]: cos | sin
  long long max_position;
  const long long* positions;  // [T]
  const int* slots;            // [T], -1 = padding row (skipped)
  __nv_bfloat16* k_cache;      // [layers][num_slots][Hkv][128]
  __nv_bfloat16* v_cache;
  long long cache_layer_stride, num_slots;
  float eps;
  // mode 2 (the Markov bias): token t's logits row (token = batch row, output feature = vocabulary entry)
  const __nv_bfloat16* logits; // [T] rows of O values, row stride logits_stride
  long long logits_stride;
  int vec2;                    // mode 2 with T <= 64 and 16-byte aligned rows: the shared-memory epilogue
};

struct Smem {
  uint64_t full[kStages], empty[kStages];
  uint64_t acc_full[2], acc_empty[2];
  uint32_t tmem_base;
  int abort;
  int last;
  float ss[4][16];             // mode 1: per-warp sums of squares of 16 token columns
  float y[16][kTileM];         // mode 1: normalised K rows of 16 tokens (RoPE partners are 64 dims apart)
};

constexpr int kSmemBytes = kStages * kStageBytes + (int)sizeof(Smem) + 1024;
static_assert(kSmemBytes <= 232448, "shared memory above the sm_100 per-CTA limit");
// mode 2's transposed tile fits in stage 0 past the operands of a <= 64-column call
static_assert(kABytes + 64 * kBlockK * 2 + 64 * (kTileM + 8) * 2 <= kStageBytes, "mode 2 tile buffer");

__device__ __forceinline__ long long ceil_div_ll(long long x, long long y) { return (x + y - 1) / y; }
__device__ __forceinline__ float bf16_round(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

// Sum over the 32 lanes of 16 columns held by every lane; lane j ends with column (j & 15)'s sum; v is consumed.
__device__ __forceinline__ float lanes_sum16(float (&v)[16], int lane) {
#pragma unroll
  for (int c = 0; c < 16; ++c) v[c] += __shfl_xor_sync(0xffffffffu, v[c], 16);
#pragma unroll
  for (int w = 8; w >= 1; w >>= 1) {
    const bool upper = (lane & w) != 0;
#pragma unroll
    for (int c = 0; c < w; ++c) {
      const float send = upper ? v[c] : v[c + w];
      const float keep = upper ? v[c + w] : v[c];
      v[c] = keep + __shfl_xor_sync(0xffffffffu, send, w);
    }
  }
  return v[0];
}

// The final fp32 values of 16 token columns c0 .. c0 + 15 of tile m, weight row `row` of this thread (the 128
// epilogue threads call it together).  Mode 0: bf16 out.  Mode 1: dflash.py:88-96 for one (layer, K|V, head):
// the projection rounded to bf16, then for K the head's RMSNorm (k_norm) and RoPE at each token's position, the
// rows stored at the tokens' slots (slot -1 skipped) -- the arithmetic of norm_rope_store_kernel.
__device__ __forceinline__ void emit16(const Args& a, Smem& S, int m, int c0, int row, int w, int lane,
                                       float (&v)[16]) {
  if (a.mode == 0) {
    const int o = m * kTileM + row;
#pragma unroll
    for (int j = 0; j < 16; ++j)
      if (c0 + j < a.T) a.out[(long long)(c0 + j) * a.out_stride + o] = __float2bfloat16_rn(v[j]);
    return;
  }
  if (a.mode == 2) {
    // speculative.py:173: logits[:, row] + markov_head(prev), the head's F.linear output rounded to bf16, then
    // the bf16 sum (the exact fp32 sum of two bf16 values, rounded once)
    const int o = m * kTileM + row;
    float l[16];
#pragma unroll
    for (int j = 0; j < 16; ++j)
      l[j] = c0 + j < a.T ? __bfloat162float(a.logits[(long long)(c0 + j) * a.logits_stride + o]) : 0.0f;
#pragma unroll
    for (int j = 0; j < 16; ++j)
      if (c0 + j < a.T)
        a.out[(long long)(c0 + j) * a.out_stride + o] = __float2bfloat16_rn(bf16_round(v[j]) + l[j]);
    return;
  }
  const int layer = m / (2 * a.Hkv), kv = (m / a.Hkv) & 1, head = m % a.Hkv;
  float x[16];
#pragma unroll
  for (int j = 0; j < 16; ++j) x[j] = bf16_round(v[j]);          // F.linear's bf16 output
  __nv_bfloat16* cache = (kv ? a.v_cache : a.k_cache) + layer * a.cache_layer_stride;
  if (kv == 0) {
    float sq[16];
#pragma unroll
    for (int j = 0; j < 16; ++j) sq[j] = x[j] * x[j];
    const float part = lanes_sum16(sq, lane);
    if (lane < 16) S.ss[w][lane] = part;
    named_barrier(2, 128);
    const float wgt = __bfloat162float(a.k_norm[layer * a.k_norm_stride + row]);
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const float ss = (S.ss[0][j] + S.ss[1][j]) + (S.ss[2][j] + S.ss[3][j]);
      const float r = rsqrtf(ss / kTileM + a.eps);
      x[j] = bf16_round(bf16_round(x[j] * r) * wgt);                // x.to(bf16).mul_(weight)
      S.y[j][row] = x[j];
    }
    named_barrier(2, 128);
    const int d = row & 63;
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const int t = c0 + j;
      if (t < a.T) {
        const long long pos = a.positions[t];
        if (pos >= 0 && pos < a.max_position) {
          const float cs = a.cos_sin[pos * kTileM + d], sn = a.cos_sin[pos * kTileM + 64 + d];
          const float partner = S.y[j][row ^ 64];
          x[j] = row < 64 ? x[j] * cs - partner * sn : x[j] * cs + partner * sn;
        } else if (row == 0) {
          atomicCAS(a.err, 0, 4);
        }
      }
    }
    named_barrier(2, 128);                                         // S.y is rewritten by the next columns
  }
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    const int t = c0 + j;
    if (t < a.T) {
      const long long slot = a.slots[t];
      if (slot >= a.num_slots) {
        if (row == 0) atomicCAS(a.err, 0, 3);
      } else if (slot >= 0) {
        cache[(slot * a.Hkv + head) * kTileM + row] = __float2bfloat16_rn(x[j]);
      }
    }
  }
}

// Mode 2, a whole tile: this thread's vocabulary entry o of the tile for every batch row.  The logits of the first
// 64 rows were loaded (raw bf16) before the accumulator was ready, so the epilogue does not wait on them.
constexpr int kPrefetchCols = 64;
__device__ __forceinline__ void prefetch_logits(const Args& a, int m, int row, unsigned short (&pre)[kPrefetchCols]) {
  const unsigned short* lg = reinterpret_cast<const unsigned short*>(a.logits) + m * kTileM + row;
#pragma unroll
  for (int j = 0; j < kPrefetchCols; ++j) pre[j] = j < a.T ? __ldg(lg + (long long)j * a.logits_stride) : 0;
}

__device__ __forceinline__ void biased_tile(const Args& a, uint32_t acc, int m, int row, int ncols,
                                            const unsigned short (&pre)[kPrefetchCols]) {
  const int o = m * kTileM + row;
#pragma unroll
  for (int c0 = 0; c0 < kPrefetchCols; c0 += 16) {
    if (c0 < ncols) {
      float v[16];
      tmem_ld_32x32b_x16(acc + c0, v);
#pragma unroll
      for (int j = 0; j < 16; ++j)
        if (c0 + j < a.T)
          a.out[(long long)(c0 + j) * a.out_stride + o] =
              __float2bfloat16_rn(bf16_round(v[j]) + __uint_as_float((unsigned)pre[c0 + j] << 16));
    }
  }
  for (int c0 = kPrefetchCols; c0 < ncols; c0 += 16) {         // rows past the prefetched ones (B > 64)
    float v[16];
    tmem_ld_32x32b_x16(acc + c0, v);
#pragma unroll
    for (int j = 0; j < 16; ++j)
      if (c0 + j < a.T)
        a.out[(long long)(c0 + j) * a.out_stride + o] = __float2bfloat16_rn(
            bf16_round(v[j]) + __bfloat162float(a.logits[(long long)(c0 + j) * a.logits_stride + o]));
  }
}

// Mode 2, a whole tile of <= 64 batch rows through shared memory: the accumulator's columns (one vocabulary entry
// per thread, one batch row per column) rounded to bf16 and stored transposed into tb [row][128 entries], then
// every thread adds 16-byte vectors of the logits rows (loaded before the accumulator was ready) and writes 16-byte
// vectors of the biased rows.  tb lies in stage 0's bytes past the operands of a <= 64-column call, which TMA never
// writes.
constexpr int kTbStride = kTileM + 8;          // bf16 per transposed row (padding against bank conflicts)
constexpr int kVecPerThread = kPrefetchCols * (kTileM / 8) / 128;   // 8 vectors of 8 entries per epilogue thread
__device__ __forceinline__ void prefetch_logits_vec(const Args& a, int m, int tid, uint4 (&pre)[kVecPerThread]) {
#pragma unroll
  for (int i = 0; i < kVecPerThread; ++i) {
    const int id = tid + 128 * i, b = id >> 4, v0 = (id & 15) * 8;
    pre[i] = b < a.T ? ldg16(a.logits + (long long)b * a.logits_stride + m * kTileM + v0) : make_uint4(0, 0, 0, 0);
  }
}

__device__ __forceinline__ void biased_tile_vec(const Args& a, uint32_t acc, int m, int row, int tid, int ncols,
                                                __nv_bfloat16* tb, const uint4 (&pre)[kVecPerThread]) {
  for (int c0 = 0; c0 < ncols; c0 += 16) {
    float v[16];
    tmem_ld_32x32b_x16(acc + c0, v);
#pragma unroll
    for (int j = 0; j < 16; ++j) tb[(c0 + j) * kTbStride + row] = __float2bfloat16_rn(v[j]);   // the bf16 bias
  }
  named_barrier(3, 128);
#pragma unroll
  for (int i = 0; i < kVecPerThread; ++i) {
    const int id = tid + 128 * i, b = id >> 4, v0 = (id & 15) * 8;
    if (b < a.T) {
      const uint4 bias = *reinterpret_cast<const uint4*>(tb + b * kTbStride + v0);
      const uint4 l = pre[i];
      uint4 r;
      const unsigned* bp = reinterpret_cast<const unsigned*>(&bias);
      const unsigned* lp = reinterpret_cast<const unsigned*>(&l);
      unsigned* rp = reinterpret_cast<unsigned*>(&r);
#pragma unroll
      for (int e = 0; e < 4; ++e) {      // bf16 pairs: the exact sum of two bf16 values, rounded once
        __nv_bfloat162 x, y;
        memcpy(&x, &lp[e], 4);
        memcpy(&y, &bp[e], 4);
        const __nv_bfloat162 z = __hadd2(x, y);
        memcpy(&rp[e], &z, 4);
      }
      *reinterpret_cast<uint4*>(a.out + (long long)b * a.out_stride + m * kTileM + v0) = r;
    }
  }
  named_barrier(3, 128);                 // tb is rewritten by the next tile
}

__global__ void __launch_bounds__(kThreads, 1)
    context_gemm_kernel(const __grid_constant__ CUtensorMap wmap, const __grid_constant__ CUtensorMap xmap,
                        const Args a) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* base = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  Smem& S = *reinterpret_cast<Smem*>(base + kStages * kStageBytes);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int ncols = a.n_sub * a.tn;
  const int tmem_cols = ncols * a.nbuf > 256 ? 512 : 256;

  // ---- this CTA's share of the (tile, k block) units: stream-K over units, or (more tiles than CTAs) whole
  // tiles, tiles * c / G .. tiles * (c + 1) / G
  const long long tiles = a.O / kTileM;
  const long long U = tiles * a.kblocks;
  const long long c = blockIdx.x;
  long long Ge, xb, xe;
  if (a.whole_tiles) {
    Ge = tiles < (long long)gridDim.x ? tiles : (long long)gridDim.x;
    xb = c < Ge ? tiles * c / Ge * a.kblocks : 0;
    xe = c < Ge ? tiles * (c + 1) / Ge * a.kblocks : 0;
  } else {
    Ge = U < (long long)gridDim.x ? U : (long long)gridDim.x;
    xb = c < Ge ? U * c / Ge : 0;
    xe = c < Ge ? U * (c + 1) / Ge : 0;
  }

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&S.full[s], 1);
      mbar_init(&S.empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&S.acc_full[i], 1);
      mbar_init(&S.acc_empty[i], 4);     // one elected arrival per epilogue warp
    }
    S.abort = 0;
    fence_barrier_init();
    prefetch_tensormap(&wmap);
    prefetch_tensormap(&xmap);
  }
  if (warp == 1) {
    tmem_alloc(&S.tmem_base, tmem_cols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = S.tmem_base;
  volatile int* abort = &S.abort;

  if (xb < xe) {
    if (warp == 0 && lane == 0) {
      // ------------------------------------------------------------------ TMA producer
      const uint32_t bytes = kABytes + ncols * kBlockK * 2;
      int g = 0;
      for (long long x = xb; x < xe; ++x, ++g) {
        const int m = (int)(x / a.kblocks), kb = (int)(x % a.kblocks);
        const int stage = g % kStages;
        if (g >= kStages && !mbar_wait(&S.empty[stage], ((g / kStages) - 1) & 1, abort, a.err, kErrTimeout)) break;
        unsigned char* st = base + stage * kStageBytes;
        mbar_arrive_expect_tx(&S.full[stage], bytes);
        tma_load_2d(st, &wmap, kb * kBlockK, m * kTileM, &S.full[stage]);
        for (int h = 0; h < a.n_sub; ++h)
          tma_load_2d(st + kABytes + h * a.tn * 128, &xmap, kb * kBlockK, h * a.tn, &S.full[stage]);
      }
    } else if (warp == 1 && lane == 0) {
      // ------------------------------------------------------------------ MMA issuer
      const uint32_t idesc = idesc_bf16_f32(kTileM, a.tn, 0, 0);
      int g = 0, piece = 0;
      bool ok = true;
      long long x = xb;
      while (ok && x < xe) {
        const int m = (int)(x / a.kblocks);
        const long long end = (long long)(m + 1) * a.kblocks < xe ? (long long)(m + 1) * a.kblocks : xe;
        const int buf = piece % a.nbuf;
        if (piece >= a.nbuf && !mbar_wait(&S.acc_empty[buf], ((piece / a.nbuf) - 1) & 1, abort, a.err, kErrTimeout))
          break;
        tc_fence_after();
        const uint32_t acc = tmem + (uint32_t)(buf * ncols);
        for (bool first = true; x < end; ++x, ++g, first = false) {
          const int stage = g % kStages;
          if (!mbar_wait(&S.full[stage], (g / kStages) & 1, abort, a.err, kErrTimeout)) { ok = false; break; }
          tc_fence_after();
          const unsigned char* st = base + stage * kStageBytes;
#pragma unroll
          for (int kk = 0; kk < kBlockK / 16; ++kk) {
            const uint64_t adesc = smem_desc(st + kk * 32, 16, 1024, kSwizzle128B);
            for (int h = 0; h < a.n_sub; ++h) {
              const uint64_t bdesc = smem_desc(st + kABytes + h * a.tn * 128 + kk * 32, 16, 1024, kSwizzle128B);
              mma_bf16_ss(acc + h * a.tn, adesc, bdesc, idesc, (first && kk == 0) ? 0u : 1u);
            }
          }
          mma_commit(&S.empty[stage]);
        }
        if (!ok) break;
        mma_commit(&S.acc_full[buf]);
        ++piece;
      }
    } else if (warp >= 4) {
      // ------------------------------------------------------------------ epilogue
      const int w = warp & 3;
      const int row = w * 32 + lane;                       // the tile's weight row = output feature
      const uint32_t lane_off = static_cast<uint32_t>(w * 32) << 16;
      int piece = 0;
      long long x = xb;
      while (x < xe) {
        const int m = (int)(x / a.kblocks);
        const long long A = (long long)m * a.kblocks, B = A + a.kblocks;
        const long long end = B < xe ? B : xe;
        x = end;
        const long long c_lo = ceil_div_ll((A + 1) * Ge, U) - 1, c_hi = ceil_div_ll(B * Ge, U) - 1;
        const int buf = piece % a.nbuf;
        const bool biased = a.mode == 2 && a.whole_tiles;
        unsigned short pre[kPrefetchCols];
        uint4 prev[kVecPerThread];
        if (biased && a.vec2) prefetch_logits_vec(a, m, row, prev);   // independent of the MMAs: loaded meanwhile
        else if (biased) prefetch_logits(a, m, row, pre);
        if (!mbar_wait(&S.acc_full[buf], (piece / a.nbuf) & 1, abort, a.err, kErrTimeout)) break;
        tc_fence_after();
        const uint32_t acc = tmem + lane_off + (uint32_t)(buf * ncols);
        if (biased) {
          if (a.vec2)
            biased_tile_vec(a, acc, m, row, row, ncols,
                            reinterpret_cast<__nv_bfloat16*>(base + kABytes + kPrefetchCols * kBlockK * 2), prev);
          else
            biased_tile(a, acc, m, row, ncols, pre);
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&S.acc_empty[buf]);
        } else if (a.whole_tiles || c_lo == c_hi) {
          // the whole tile here: rows straight from the accumulator
          for (int c0 = 0; c0 < ncols; c0 += 16) {
            float v[16];
            tmem_ld_32x32b_x16(acc + c0, v);
            emit16(a, S, m, c0, row, w, lane, v);
          }
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&S.acc_empty[buf]);
        } else {
          // a piece: published (fp32), then the last CTA to arrive sums the pieces in CTA order
          float* mine = a.partial + (2LL * c + (xb < A ? 1 : 0)) * (long long)ncols * kTileM;
          for (int c0 = 0; c0 < ncols; c0 += 16) {
            float v[16];
            tmem_ld_32x32b_x16(acc + c0, v);
#pragma unroll
            for (int j = 0; j < 16; ++j) __stcg(mine + (long long)(c0 + j) * kTileM + row, v[j]);
          }
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&S.acc_empty[buf]);   // the MMAs may refill the accumulator now
          __threadfence();
          named_barrier(1, 128);
          if (threadIdx.x == 128) {
            int* counter = a.counters + m;
            const int last = atomicAdd(counter, 1) == (int)(c_hi - c_lo);
            if (last) atomicExch(counter, 0);
            S.last = last;
          }
          named_barrier(1, 128);
          const bool last = S.last != 0;
          named_barrier(1, 128);                           // S.last is rewritten by the next piece
          if (last) {
            __threadfence();
            for (int c0 = 0; c0 < ncols && c0 < a.T; c0 += 16) {
              float acc[16];
#pragma unroll
              for (int j = 0; j < 16; ++j) acc[j] = 0.0f;
              for (long long cc = c_lo; cc <= c_hi; ++cc) {
                const long long s_cc = U * cc / Ge;
                const float* pc = a.partial + (2 * cc + (s_cc < A ? 1 : 0)) * (long long)ncols * kTileM;
#pragma unroll
                for (int j = 0; j < 16; ++j) acc[j] += __ldcg(pc + (long long)(c0 + j) * kTileM + row);
              }
              emit16(a, S, m, c0, row, w, lane, acc);
            }
          }
        }
        ++piece;
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, tmem_cols);
  }
}

// ---------------------------------------------------------------------------------------- host side
// The driver's tensor-map encoder (one entry point for every device), looked up on first use; the initialisation
// of a function-local static is thread-safe.
static PFN_cuTensorMapEncodeTiled_v12000 encoder() {
  static const PFN_cuTensorMapEncodeTiled_v12000 fn = []() -> PFN_cuTensorMapEncodeTiled_v12000 {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      return reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    return nullptr;
  }();
  return fn;
}

// 2-D bf16 row-major matrix [rows, cols] (row stride in elements), 128-byte swizzle, box {64 cols, box_rows}.
static int make_map_2d(CUtensorMap* map, const void* base, uint64_t cols, uint64_t rows, uint64_t row_stride,
                       uint32_t box_rows) {
  auto fn = encoder();
  if (!fn) return set_error(kCudaError, "cuTensorMapEncodeTiled is unavailable from the driver");
  if ((reinterpret_cast<uintptr_t>(base) & 15) || ((row_stride * 2) & 15))
    return set_error(kInvalidArgument, "TMA needs a 16-byte aligned base and row stride");
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {row_stride * 2};
  cuuint32_t box[2] = {(cuuint32_t)kBlockK, box_rows};
  cuuint32_t elem[2] = {1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, elem,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(kCudaError, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return kOk;
}

static void columns(int T, int* n_sub, int* tn) {
  *n_sub = T > 256 ? 2 : 1;
  const int per = (T + *n_sub - 1) / *n_sub;
  *tn = (per + 15) / 16 * 16;
}

// Workspace: arrival counters for up to kMaxTiles tiles at a fixed offset (so calls of every shape share one
// workspace zeroed once: each call leaves its counters at zero and no call's pieces overlap them), then the pieces.
constexpr int kMaxTiles = 4096;
static long long counters_bytes(int) { return (long long)kMaxTiles * 4; }

static long long workspace_bytes(int T, int O, int grid) {
  int n_sub, tn;
  columns(T, &n_sub, &tn);
  return counters_bytes(O) + 2LL * grid * n_sub * tn * kTileM * 4;
}

// Shared host path of both entry points: checks, maps, workspace, launch; `a` carries the epilogue's fields.
static int launch(Args a, const void* x, long long x_row_stride, const void* w, long long w_row_stride,
                  void* workspace, long long workspace_bytes_given, int* err, void* stream) {
  SPECDEC_CHECK_ARG(x && w && workspace && err, "null pointer argument");
  SPECDEC_CHECK_ARG(a.T >= 1 && a.T <= kMaxCols, "T = %d: one call takes 1 .. %d tokens", a.T, kMaxCols);
  SPECDEC_CHECK_ARG(a.O >= kTileM && a.O % kTileM == 0 && a.O / kTileM <= kMaxTiles,
                    "O = %d must be a positive multiple of %d, at most %d", a.O, kTileM, kTileM * kMaxTiles);
  SPECDEC_CHECK_ARG(a.K >= kBlockK && a.K % kBlockK == 0, "K = %d must be a positive multiple of %d", a.K, kBlockK);
  SPECDEC_CHECK_ARG((reinterpret_cast<uintptr_t>(workspace) & 255) == 0, "workspace must be 256-byte aligned");
  SPECDEC_CHECK_ARG(x_row_stride >= a.K && w_row_stride >= a.K, "row strides below K");
  DeviceInfo info;
  if (int st = device_info(&info)) return st;
  const long long units = (long long)(a.O / kTileM) * (a.K / kBlockK);
  const int grid = (int)(units < info.sm_count ? units : info.sm_count);
  a.whole_tiles = a.O / kTileM >= grid ? 1 : 0;
  const long long need = workspace_bytes(a.T, a.O, info.sm_count);
  if (workspace_bytes_given < need)
    return set_error(kWorkspaceTooSmall, "context GEMM workspace of %lld bytes, %lld needed",
                     workspace_bytes_given, need);
  columns(a.T, &a.n_sub, &a.tn);
  a.kblocks = a.K / kBlockK;
  a.nbuf = a.whole_tiles && a.n_sub * a.tn <= 128 ? 2 : 1;
  a.counters = static_cast<int*>(workspace);
  a.partial = reinterpret_cast<float*>(static_cast<unsigned char*>(workspace) + counters_bytes(a.O));
  a.err = err;
  CUtensorMap wm, xm;
  if (int st = make_map_2d(&wm, w, a.K, a.O, w_row_stride, kTileM)) return st;
  if (int st = make_map_2d(&xm, x, a.K, a.T, x_row_stride, a.tn)) return st;
  if (int st = ensure_dynamic_smem<context_gemm_kernel>(kSmemBytes)) return st;
  context_gemm_kernel<<<grid, kThreads, kSmemBytes, static_cast<cudaStream_t>(stream)>>>(wm, xm, a);
  SPECDEC_LAUNCH_CHECK();
  return kOk;
}

}  // namespace gemm
}  // namespace specdec

using namespace specdec;

extern "C" {

long long specdec_context_gemm_workspace_bytes(int T, int O) {
  DeviceInfo info;
  if (T < 1 || T > gemm::kMaxCols || O < gemm::kTileM || device_info(&info) != kOk) return -1;
  return gemm::workspace_bytes(T, O, info.sm_count);
}

int specdec_context_gemm(const void* x, long long x_row_stride, const void* w, long long w_row_stride, int T, int O,
                         int K, void* out, long long out_row_stride, void* workspace, long long workspace_bytes,
                         int* err, void* stream) {
  SPECDEC_CHECK_ARG(out && out_row_stride >= O, "out missing, or its row stride below O");
  gemm::Args a{};
  a.mode = 0;
  a.T = T;
  a.O = O;
  a.K = K;
  a.out = static_cast<__nv_bfloat16*>(out);
  a.out_stride = out_row_stride;
  return gemm::launch(a, x, x_row_stride, w, w_row_stride, workspace, workspace_bytes, err, stream);
}

int specdec_markov_bias(const void* w2, long long w2_row_stride, const void* e, long long e_row_stride, int B, int V,
                        int rank, const void* logits, long long logits_row_stride, void* out,
                        long long out_row_stride, void* workspace, long long workspace_bytes, int* err,
                        void* stream) {
  SPECDEC_CHECK_ARG(logits && out, "null pointer argument");
  SPECDEC_CHECK_ARG(logits_row_stride >= V && out_row_stride >= V, "row strides below V");
  gemm::Args a{};
  a.mode = 2;
  a.T = B;
  a.O = V;
  a.K = rank;
  a.out = static_cast<__nv_bfloat16*>(out);
  a.out_stride = out_row_stride;
  a.logits = static_cast<const __nv_bfloat16*>(logits);
  a.logits_stride = logits_row_stride;
  a.vec2 = B <= gemm::kPrefetchCols && ((reinterpret_cast<uintptr_t>(logits) | reinterpret_cast<uintptr_t>(out)) & 15) == 0 &&
           logits_row_stride % 8 == 0 && out_row_stride % 8 == 0 && V % 8 == 0;
  return gemm::launch(a, e, e_row_stride, w2, w2_row_stride, workspace, workspace_bytes, err, stream);
}

int specdec_context_kv_store(const void* x, long long x_row_stride, const void* w_kv, long long w_row_stride, int T,
                             int layers, int num_kv_heads, int K, const void* k_norm, long long k_norm_layer_stride,
                             const float* cos_sin, long long max_position, const long long* positions,
                             const int* slot_mapping, void* k_cache, void* v_cache, long long cache_layer_stride,
                             long long num_slots, float eps, void* workspace, long long workspace_bytes, int* err,
                             void* stream) {
  SPECDEC_CHECK_ARG(k_norm && cos_sin && positions && slot_mapping && k_cache && v_cache, "null pointer argument");
  SPECDEC_CHECK_ARG(layers >= 1 && num_kv_heads >= 1, "bad sizes");
  SPECDEC_CHECK_ARG(((reinterpret_cast<uintptr_t>(k_cache) | reinterpret_cast<uintptr_t>(v_cache)) & 1) == 0,
                    "caches must be 2-byte aligned");
  gemm::Args a{};
  a.mode = 1;
  a.T = T;
  a.O = layers * 2 * num_kv_heads * gemm::kTileM;
  a.K = K;
  a.Hkv = num_kv_heads;
  a.k_norm = static_cast<const __nv_bfloat16*>(k_norm);
  a.k_norm_stride = k_norm_layer_stride;
  a.cos_sin = cos_sin;
  a.max_position = max_position;
  a.positions = positions;
  a.slots = slot_mapping;
  a.k_cache = static_cast<__nv_bfloat16*>(k_cache);
  a.v_cache = static_cast<__nv_bfloat16*>(v_cache);
  a.cache_layer_stride = cache_layer_stride;
  a.num_slots = num_slots;
  a.eps = eps;
  return gemm::launch(a, x, x_row_stride, w_kv, w_row_stride, workspace, workspace_bytes, err, stream);
}

}  // extern "C"
