// Kernel (2): paged verify attention for sm_100a (TMA + tcgen05 + TMEM), and the paged K/V store.
//
// Reference behaviour (nano-vllm-speculative-decoding):
//   store_kvcache / store_kvcache_kernel   nanovllm/layers/attention.py:10-40   K/V row of token t to slot
//                                          slot_mapping[t]; slot -1 skipped
//   Attention.forward, verify branch        nanovllm/layers/attention.py:62-70   flash_attn_varlen_func over the
//                                          paged cache (block_table), causal, bottom-right aligned: query j of a
//                                          row with L_q queries and L_k keys sees keys 0 .. L_k - L_q + j
//   Attention.forward, decode branch        nanovllm/layers/attention.py:71-76   flash_attn_with_kvcache with
//                                          query_len_per_seq queries per row, cache_seqlens, causal or not (the
//                                          DFlash draft block passes causal=False)
//   restated on CPU by tests/fake_paged_attention.py:14-41 (SDPA with the same mask rule).
//
// Design (B200).  A persistent kernel, one CTA per SM.  Work item = (row, KV head): the row's <= 8 query
// positions times the GQA group's 4 query heads are packed into N = 32 columns, so every K/V tile of that head is
// read from HBM exactly once.  The items' 128-key tiles form one sequence that is cut into equal contiguous
// shares, one per CTA (stream-K): no wave quantisation, and every SM streams the same number of tiles.  An item
// cut between CTAs is finished by whichever of its CTAs arrives last (an atomic counter per item): each piece is
// published as unnormalised O^T with its column maxima and sums, and the last one merges them in CTA order (the
// output does not depend on arrival order); nobody waits.
// The tensor core runs swap-AB: S^T[128 keys x 32] = K_tile[128 x 128] . Q^T and O^T[128 dims x 32] += V^T . P^T,
// both M = 128 UMMAs with fp32 accumulators in TMEM (S and O double-buffered, O by item).  K and V tiles of 128
// keys (half a 256-slot block) arrive by TMA through one tensor map over the whole paged cache (coordinates: dim,
// head, physical slot), so the block table is a coordinate, not a gather.  The pipelines run across items: the
// next item's Q (double-buffered) and first tiles load while the current item's epilogue runs.
//   warp 0      TMA producer: Q per item and the K tiles (3-stage ring)
//   warp 1      TMEM allocator + single-thread MMA issuer
//   warp 2      prologue: this CTA's share of the tile sequence from the row metadata
//   warp 3      TMA producer: the V tiles (3-stage ring)
//   warps 4-11  softmax over keys (one TMEM lane = one key; two warpgroups of 16 columns each), P^T to shared
//               memory, O rescale, epilogue
// The softmax is online per query column with lazy rescaling (O is rescaled only when a column's running max
// grows by more than 2^8), masked by key index (bottom-right causal or context length).  Keys past the row's
// context in its last tile are never read as values: their P is 0 and their V rows are zeroed in shared memory.
#include "common.cuh"
#include "sm100.cuh"
#include "specdec_b200.h"

#include <cudaTypedefs.h>
#include <math.h>
#include <stddef.h>

namespace specdec {
namespace attention {

using namespace sm100;

constexpr int kHeadDim = 128;
constexpr int kKeysPerTile = 128;
constexpr int kSubKeys = 32;                              // an item's last tile loads in 32-key sub-boxes
constexpr int kCols = 32;              // packed query columns (group x positions)
constexpr int kStages = 3;             // K ring and V ring depth
constexpr int kThreads = 384;            // warps 0-3: TMA (Q, K), MMA, prologue, TMA (V); 4-11: softmax
constexpr int kHalfTileBytes = kKeysPerTile * 128;     // 64 dims x 128 keys bf16 = 16 KB
constexpr int kTileBytes = 2 * kHalfTileBytes;          // 32 KB
constexpr int kQHalfBytes = kCols * 128;                // 32 rows x 64 dims bf16 = 4 KB
constexpr int kPBytes = kKeysPerTile * kCols * 2;       // 8 KB
constexpr uint32_t kTmemCols = 128;                     // S0 | S1 | O0 | O1

// error codes written to the global error word
constexpr int kErrTimeoutQ = 11, kErrTimeoutK = 12, kErrTimeoutV = 13, kErrTimeoutS = 14, kErrTimeoutP = 15,
              kErrTimeoutO = 16, kErrTimeoutEmpty = 17;

// One piece of a split item: O^T columns (unnormalised, relative to the piece's running maxima) then the maxima m
// and the sums l of the 32 columns.
constexpr int kPartialFloats = kCols * kHeadDim + 2 * kCols;
constexpr int kMaxOuts = 8;            // output destinations of one launch (one per rank of an 8-GPU node)

// Destinations beyond Args::out, written with the same offsets by the kPeers instantiation only (the peer-store
// tensor-parallel mode: every peer's [T, H, D] output, mapped into this process, this rank's head offset folded
// into the base).  A separate parameter, so the single-output kernel's code and Args are untouched.
struct PeerOuts {
  __nv_bfloat16* out[kMaxOuts - 1];
  int n;                     // 0 .. kMaxOuts - 1
};
constexpr float kNegBig = -1.0e30f;    // start value of the running maxima (finite: no -inf arithmetic)

struct Args {
  const int* cu_seqlens_q;   // [R + 1] or null (decode mode)
  const int* cu_seqlens_k;   // [R + 1] or null (decode mode)
  const int* context_lens;   // [R] (decode mode)
  int q_per_seq;             // decode mode: queries per row
  int R;
  const int* block_tables;   // [R, W]
  int W, block_size;
  int H, Hkv;
  float scale_log2;          // softmax_scale * log2(e)
  int causal;
  __nv_bfloat16* out;        // [T, H, D]
  long long out_row_stride;  // elements between tokens of out (and of every PeerOuts destination)
  int* counters;             // [R * Hkv] arrivals at split items; zero between launches (the last arrival resets)
  float* partial;            // [2 * gridDim.x][kPartialFloats]: slot 2c = CTA c's first item, 2c + 1 its last
  int* err;                  // global error word (0 = ok)
};

struct Smem {
  uint64_t q_full[2], q_empty[2];
  uint64_t k_full[kStages], k_empty[kStages], v_full[kStages], v_empty[kStages];
  uint64_t s_full[2], s_free[2], p_full[2], o_done[2], o_free[2];
  uint32_t tmem_base;
  int abort;
  long long total_tiles;     // tiles of all items
  long long x_begin, x_end;  // this CTA's share [x_begin, x_end) of the tile sequence
  long long row_tile0;       // sequence index of the first tile of row b_start
  int b_start;               // row holding tile x_begin
  int active;                // CTAs given tiles: min(gridDim.x, total_tiles)
  int r0[4];                 // row b_start's RowInfo (q_start, ql, L, nt)
  int slot0;                 // cache slot of the share's first tile
  int last_piece;            // the epilogue's broadcast: this CTA combines the split item
  alignas(16) float red_max[2][32][4];   // [tile parity][column][warp] maxima (read as float4)
  alignas(16) float red_sum[32][4];      // [column][warp] sums (epilogue)
};
static_assert(offsetof(Smem, red_max) % 16 == 0 && offsetof(Smem, red_sum) % 16 == 0, "float4 reads need 16 B");
static_assert(offsetof(Smem, total_tiles) % 8 == 0, "64-bit fields need 8 B");

constexpr int kQBytes = 2 * kQHalfBytes;                       // 8 KB, double-buffered by item
constexpr int kOffQ = 0;
constexpr int kOffK = kOffQ + 2 * kQBytes;                     // 16 KB
constexpr int kOffV = kOffK + kStages * kTileBytes;
constexpr int kOffP = kOffV + kStages * kTileBytes;
constexpr int kOffCtl = kOffP + 2 * kPBytes;
constexpr int kSmemBytes = kOffCtl + (int)sizeof(Smem) + 1024;   // + alignment slack
static_assert(kSmemBytes <= 232448, "shared memory above the sm_100 per-CTA limit");

// Max over the warp's 32 lanes in one instruction (sm_100a redux.sync on f32).
__device__ __forceinline__ float warp_max_redux(float v) {
  float r;
  asm volatile("redux.sync.max.f32 %0, %1, 0xffffffff;" : "=f"(r) : "f"(v));
  return r;
}

// Sum over the 32 lanes of 16 columns held by every lane; lane j ends with column (j & 15)'s sum; v is consumed.
__device__ __forceinline__ float column_reduce16(float (&v)[16], int lane) {
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

// A row's queries and keys; nt = 0 when the row has no work (no queries, or metadata that the kernel rejects).
struct RowInfo {
  int q_start, ql, L, nt;
};

template <int QMAX>
__device__ __forceinline__ RowInfo row_info(const Args& a, int b, bool report) {
  RowInfo r;
  if (a.cu_seqlens_q) {
    r.q_start = a.cu_seqlens_q[b];
    r.ql = a.cu_seqlens_q[b + 1] - r.q_start;
    r.L = a.cu_seqlens_k[b + 1] - a.cu_seqlens_k[b];
  } else {
    r.q_start = b * a.q_per_seq;
    r.ql = a.q_per_seq;
    r.L = a.context_lens[b];
  }
  r.nt = 0;
  if (r.ql > 0) {
    if (r.ql > QMAX || r.L <= 0 || r.L > a.W * a.block_size) {   // inconsistent metadata: report, never read
      if (report) atomicCAS(a.err, 0, 2);
    } else {
      r.nt = (r.L + kKeysPerTile - 1) / kKeysPerTile;
    }
  }
  return r;
}

// The item sequence: items (row b, KV head h) in row-major order, item (b, h) holding the sequence's tiles
// [A, A + r.nt).  Each role of a CTA walks it from the item holding x_begin to the one holding x_end - 1.
template <int QMAX>
struct Walk {
  int b, h;
  long long A;
  RowInfo r;
  __device__ __forceinline__ void start(const Args& a, const Smem& S) {
    b = S.b_start;
    r = RowInfo{S.r0[0], S.r0[1], S.r0[2], S.r0[3]};   // found by the prologue
    h = (int)((S.x_begin - S.row_tile0) / r.nt);
    A = S.row_tile0 + (long long)h * r.nt;
  }
  __device__ __forceinline__ void next(const Args& a) {
    A += r.nt;
    if (++h == a.Hkv) {
      h = 0;
      do {
        ++b;
        r = b < a.R ? row_info<QMAX>(a, b, false) : RowInfo{0, 0, 0, 1};
      } while (r.nt == 0);
    }
  }
  // this CTA's tiles of the item: item-local [t0, t1)
  __device__ __forceinline__ int t0(long long x_begin) const { return (int)(x_begin > A ? x_begin - A : 0); }
  __device__ __forceinline__ int t1(long long x_end) const {
    return (int)(x_end < A + r.nt ? x_end - A : (long long)r.nt);
  }
};

// Tile-by-tile cursor over the CTA's share: the segment (item piece) index n of the current tile and whether the
// tile is the segment's first / last.
template <int QMAX>
struct Cursor {
  Walk<QMAX> w;
  int n, left;
  bool first;
  __device__ __forceinline__ void start(const Args& a, const Smem& S) {
    w.start(a, S);
    n = 0;
    left = w.t1(S.x_end) - w.t0(S.x_begin);
    first = true;
  }
  __device__ __forceinline__ bool last() const { return left == 1; }
  __device__ __forceinline__ void advance(const Args& a, long long x_begin, long long x_end) {
    if (--left == 0) {
      w.next(a);
      ++n;
      left = w.t1(x_end) - w.t0(x_begin);
      first = true;
    } else {
      first = false;
    }
  }
};

__device__ __forceinline__ long long ceil_div(long long x, long long y) { return (x + y - 1) / y; }

template <int G, bool kPeers>
__global__ void __launch_bounds__(kThreads, 1)
    verify_attention_kernel(const __grid_constant__ CUtensorMap qmap, const __grid_constant__ CUtensorMap kmap,
                            const __grid_constant__ CUtensorMap vmap, const __grid_constant__ CUtensorMap kmap32,
                            const __grid_constant__ CUtensorMap vmap32, const Args a,
                            const __grid_constant__ PeerOuts peers) {
  constexpr int QMAX = kCols / G;     // query positions per row this build packs
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* base = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  unsigned char* sQ = base + kOffQ;
  unsigned char* sK = base + kOffK;
  unsigned char* sV = base + kOffV;
  unsigned char* sP = base + kOffP;
  Smem& S = *reinterpret_cast<Smem*>(base + kOffCtl);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(&S.q_full[i], 1);
      mbar_init(&S.q_empty[i], 1);
      mbar_init(&S.s_full[i], 1);
      mbar_init(&S.s_free[i], 8);     // one elected arrival per softmax warp
      mbar_init(&S.p_full[i], 8);
      mbar_init(&S.o_done[i], 1);
      mbar_init(&S.o_free[i], 8);
    }
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&S.k_full[s], 1);
      mbar_init(&S.k_empty[s], 1);
      mbar_init(&S.v_full[s], 1);
      mbar_init(&S.v_empty[s], 1);
    }
    S.abort = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(&S.tmem_base, kTmemCols);
    tmem_relinquish();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tensormap(&qmap);
    prefetch_tensormap(&kmap);
    prefetch_tensormap(&vmap);
    prefetch_tensormap(&kmap32);
    prefetch_tensormap(&vmap32);
  }
  if (warp == 2) {
    // ---- this CTA's share: the tile sequence split evenly over min(grid, tiles) CTAs, then the row holding
    // its first tile (two passes of 32 rows at a time over the row metadata)
    long long row_tiles = 0;
    for (int b0 = 0; b0 < a.R; b0 += 32) {
      const int b = b0 + lane;
      const int nt = b < a.R ? row_info<QMAX>(a, b, true).nt : 0;
      row_tiles += __reduce_add_sync(0xffffffffu, (unsigned)nt);
    }
    const long long T = row_tiles * a.Hkv;
    const long long Ge = T < (long long)gridDim.x ? T : (long long)gridDim.x;
    const long long c = blockIdx.x;
    long long xb = 0, xe = 0, row0 = 0;
    int bstart = 0, slot0 = 0;
    RowInfo r0{0, 0, 0, 1};
    if (c < Ge) {
      xb = T * c / Ge;
      xe = T * (c + 1) / Ge;
      long long pre = 0;
      for (int b0 = 0; b0 < a.R; b0 += 32) {
        const int b = b0 + lane;
        const RowInfo ri = b < a.R ? row_info<QMAX>(a, b, false) : RowInfo{0, 0, 0, 0};
        const long long v = (long long)ri.nt * a.Hkv;
        long long inc = v;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const long long y = __shfl_up_sync(0xffffffffu, inc, o);
          if (lane >= o) inc += y;
        }
        const long long first = pre + inc - v;
        const unsigned hit = __ballot_sync(0xffffffffu, v > 0 && xb >= first && xb < first + v);
        if (hit) {
          const int src = __ffs(hit) - 1;
          bstart = b0 + src;
          row0 = __shfl_sync(0xffffffffu, first, src);
          r0.q_start = __shfl_sync(0xffffffffu, ri.q_start, src);
          r0.ql = __shfl_sync(0xffffffffu, ri.ql, src);
          r0.L = __shfl_sync(0xffffffffu, ri.L, src);
          r0.nt = __shfl_sync(0xffffffffu, ri.nt, src);
          break;
        }
        pre += __shfl_sync(0xffffffffu, inc, 31);
      }
    }
    if (c < Ge && lane == 0) {       // the share's first tile: its key in the row and its cache slot
      const long long h = (xb - row0) / r0.nt;
      const int key0 = (int)(xb - row0 - h * r0.nt) * kKeysPerTile;
      slot0 = a.block_tables[(long long)bstart * a.W + key0 / a.block_size] * a.block_size + key0 % a.block_size;
      // the first item's Q and first K / V tile into L2 ahead of the loads (before an early launch's wait too)
      tma_prefetch_3d(&kmap, 0, (int)h, slot0);
      tma_prefetch_3d(&kmap, 64, (int)h, slot0);
      tma_prefetch_3d(&vmap, 0, (int)h, slot0);
      tma_prefetch_3d(&vmap, 64, (int)h, slot0);
      tma_prefetch_3d(&qmap, 0, (int)h * G, r0.q_start);
      tma_prefetch_3d(&qmap, 64, (int)h * G, r0.q_start);
    }
    if (lane == 0) {
      S.total_tiles = T;
      S.active = (int)Ge;
      S.x_begin = xb;
      S.x_end = xe;
      S.row_tile0 = row0;
      S.b_start = bstart;
      S.r0[0] = r0.q_start;
      S.r0[1] = r0.ql;
      S.r0[2] = r0.L;
      S.r0[3] = r0.nt;
      S.slot0 = slot0;
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  // An early (programmatic dependent) launch ran the prologue above while the preceding kernel finished; nothing
  // below reads or writes memory before that kernel's completion (a no-op for an ordinary launch).
  griddep_wait();
  const uint32_t tmem = S.tmem_base;
  volatile int* abort = &S.abort;
  const long long x_begin = S.x_begin, x_end = S.x_end;
  const int ntiles = (int)(x_end - x_begin);

  if (warp == 0 || warp == 3) {
    // ------------------------------------------------------------------ TMA producers
    // warp 0: Q per item and the K ring (a K slot frees as soon as its score MMA completes); warp 3: the V ring
    // (a V slot frees only after its PV MMA, so V waits never hold back the K loads)
    const bool kq = warp == 0;
    if (lane == 0 && ntiles > 0) {
      uint64_t* full = kq ? S.k_full : S.v_full;
      uint64_t* empty = kq ? S.k_empty : S.v_empty;
      unsigned char* ring = kq ? sK : sV;
      const CUtensorMap* map = kq ? &kmap : &vmap;
      const CUtensorMap* map32 = kq ? &kmap32 : &vmap32;
      Walk<QMAX> wk;
      wk.start(a, S);
      bool ok = true;
      int g = 0;
      for (int n = 0; ok && wk.A < x_end; wk.next(a), ++n) {
        if (kq) {
          const int qb = n & 1;
          if (n >= 2 && !mbar_wait(&S.q_empty[qb], ((n - 2) >> 1) & 1, abort, a.err, kErrTimeoutEmpty)) break;
          unsigned char* q = sQ + qb * kQBytes;
          mbar_arrive_expect_tx(&S.q_full[qb], kQBytes);
          tma_load_3d(q, &qmap, 0, wk.h * G, wk.r.q_start, &S.q_full[qb]);
          tma_load_3d(q + kQHalfBytes, &qmap, 64, wk.h * G, wk.r.q_start, &S.q_full[qb]);
        }
        const int* table = a.block_tables + (long long)wk.b * a.W;
        const int t1 = wk.t1(x_end);
        for (int t = wk.t0(x_begin); t < t1; ++t, ++g) {
          const int stage = g % kStages;
          const uint32_t use = g / kStages;
          const int key0 = t * kKeysPerTile;
          const int slot = g == 0 ? S.slot0 : table[key0 / a.block_size] * a.block_size + key0 % a.block_size;
          if (g >= kStages && !mbar_wait(&empty[stage], (use - 1) & 1, abort, a.err, kErrTimeoutEmpty)) {
            ok = false;
            break;
          }
          // the item's last tile: only the 32-key sub-boxes holding context keys (the rest of the stage keeps
          // stale rows, which the softmax masks in S and zeroes in V)
          const int subs = t == wk.r.nt - 1 ? (wk.r.L - key0 + kSubKeys - 1) / kSubKeys : kKeysPerTile / kSubKeys;
          unsigned char* dst = ring + stage * kTileBytes;
          if (subs == kKeysPerTile / kSubKeys) {
            mbar_arrive_expect_tx(&full[stage], kTileBytes);
            tma_load_3d(dst, map, 0, wk.h, slot, &full[stage]);
            tma_load_3d(dst + kHalfTileBytes, map, 64, wk.h, slot, &full[stage]);
          } else {
            mbar_arrive_expect_tx(&full[stage], subs * kSubKeys * 256);
            for (int j = 0; j < subs; ++j) {
              tma_load_3d(dst + j * kSubKeys * 128, map32, 0, wk.h, slot + j * kSubKeys, &full[stage]);
              tma_load_3d(dst + kHalfTileBytes + j * kSubKeys * 128, map32, 64, wk.h, slot + j * kSubKeys,
                          &full[stage]);
            }
          }
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    if (lane == 0 && ntiles > 0) {
      const uint32_t idesc_s = idesc_bf16_f32(128, kCols, 0, 0);
      const uint32_t idesc_o = idesc_bf16_f32(128, kCols, 1, 1);
      Cursor<QMAX> cs, cp;     // the score MMAs run two tiles ahead of the PV MMAs
      cs.start(a, S);
      cp.start(a, S);
      auto issue_s = [&](int g) -> bool {
        const int stage = g % kStages;
        const int qb = cs.n & 1;
        if (cs.first && !mbar_wait(&S.q_full[qb], (cs.n >> 1) & 1, abort, a.err, kErrTimeoutQ)) return false;
        if (!mbar_wait(&S.k_full[stage], (g / kStages) & 1, abort, a.err, kErrTimeoutK)) return false;
        if (g >= 2 && !mbar_wait(&S.s_free[g & 1], ((g - 2) >> 1) & 1, abort, a.err, kErrTimeoutS)) return false;
        tc_fence_after();
        const unsigned char* kt = sK + stage * kTileBytes;
        const unsigned char* qt = sQ + qb * kQBytes;
        const uint32_t tmem_s = tmem + (g & 1) * 32;
#pragma unroll
        for (int kk = 0; kk < kHeadDim / 16; ++kk) {
          const int half = kk >> 2, sub = (kk & 3) * 32;
          const uint64_t adesc = smem_desc(kt + half * kHalfTileBytes + sub, 16, 1024, kSwizzle128B);
          const uint64_t bdesc = smem_desc(qt + half * kQHalfBytes + sub, 16, 1024, kSwizzle128B);
          mma_bf16_ss(tmem_s, adesc, bdesc, idesc_s, kk > 0 ? 1u : 0u);
        }
        mma_commit(&S.s_full[g & 1]);
        mma_commit(&S.k_empty[stage]);
        if (cs.last()) mma_commit(&S.q_empty[qb]);
        cs.advance(a, x_begin, x_end);
        return true;
      };
      auto issue_pv = [&](int g) -> bool {
        const int stage = g % kStages;
        const int ob = cp.n & 1;
        if (cp.first && cp.n >= 2 && !mbar_wait(&S.o_free[ob], ((cp.n - 2) >> 1) & 1, abort, a.err, kErrTimeoutO))
          return false;
        if (!mbar_wait(&S.p_full[g & 1], (g >> 1) & 1, abort, a.err, kErrTimeoutP)) return false;
        if (!mbar_wait(&S.v_full[stage], (g / kStages) & 1, abort, a.err, kErrTimeoutV)) return false;
        tc_fence_after();
        const unsigned char* vt = sV + stage * kTileBytes;
        const unsigned char* pt = sP + (g & 1) * kPBytes;
        const uint32_t tmem_o = tmem + 64 + ob * 32;
        const bool fresh = cp.first;
#pragma unroll
        for (int kk = 0; kk < kKeysPerTile / 16; ++kk) {
          const uint64_t adesc = smem_desc(vt + kk * 2048, kHalfTileBytes, 1024, kSwizzle128B);
          const uint64_t bdesc = smem_desc(pt + kk * 1024, kPBytes, 512, kSwizzle64B);
          mma_bf16_ss(tmem_o, adesc, bdesc, idesc_o, (!fresh || kk > 0) ? 1u : 0u);
        }
        mma_commit(&S.o_done[g & 1]);
        mma_commit(&S.v_empty[stage]);
        cp.advance(a, x_begin, x_end);
        return true;
      };
      // S(g + 2) goes out as soon as the softmax has read S(g) (its buffer), before PV(g), which waits for the
      // softmax of tile g to finish: the score tiles stay two ahead of the softmax, across item boundaries too.
      bool ok = issue_s(0);
      if (ok && ntiles > 1) ok = issue_s(1);
      for (int g = 0; g < ntiles && ok; ++g) {
        if (g + 2 < ntiles) ok = issue_s(g + 2);
        if (ok) ok = issue_pv(g);
      }
    }
  } else if (warp >= 4 && ntiles > 0) {
    // ------------------------------------------------------------------ softmax / correction / epilogue
    // Two warpgroups split the 32 columns (16 each); warp w of either group reads TMEM lane quadrant w % 4.
    const int wg = (warp - 4) >> 2;          // column group: columns cb .. cb + 15
    const int cb = wg * 16;
    const int w = warp & 3;                  // TMEM lane quadrant
    const int row = (threadIdx.x - 128) & 127;   // key within the tile (S^T) / head dim (O^T)
    const int col = cb + (lane & 15);        // the column lane j (and lane j + 16) speaks for
    const uint32_t lane_off = static_cast<uint32_t>(w * 32) << 16;
    const int bar_wg = 1 + wg;               // named barrier of this group's 128 threads
    const long long T = S.total_tiles, Ge = S.active;
    const int c = blockIdx.x;
    Walk<QMAX> wk;
    wk.start(a, S);
    bool ok = true;
    int g = 0;
    for (int n = 0; ok && wk.A < x_end; wk.next(a), ++n) {
      const int L = wk.r.L, ql = wk.r.ql;
      const int t0 = wk.t0(x_begin), t1 = wk.t1(x_end);
      const uint32_t tmem_o = tmem + lane_off + 64 + (n & 1) * 32 + cb;
      const int min_limit = L - ql;            // smallest causal limit among the valid columns
      // The item's first piece, when this CTA holds it, reads the item's arrival counter now, while the tiles
      // stream: the other pieces (processed at the starts of later shares) have usually been published already,
      // and the epilogue then needs no counter round trip.
      const long long c_lo = ceil_div((wk.A + 1) * Ge, T) - 1, c_hi = ceil_div((wk.A + wk.r.nt) * Ge, T) - 1;
      int seen_early = -1;
      if (threadIdx.x == 128 && c_lo != c_hi && c == c_lo)
        seen_early = ld_acquire_gpu(a.counters + (long long)wk.b * a.Hkv + wk.h);
      // Running maxima (log2 domain): lane j owns column cb + (j & 15)'s (m_lane) and every thread keeps a copy
      // of its group's 16 (m_all), changed only when some column grows by more than 2^8 (lazy rescaling).  The
      // start value is a large negative finite number, so no -inf arithmetic is needed.  l_part: this thread's
      // share of the column sums over its own keys, reduced across the group once per item.
      float m_lane = kNegBig, m_all[16], l_part[16];
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        m_all[j] = kNegBig;
        l_part[j] = 0.0f;
      }
      for (int t = t0; t < t1; ++t, ++g) {
        const int buf = g & 1;               // partial buffers alternate by tile parity (no reuse hazard)
        if (!mbar_wait(&S.s_full[buf], (g >> 1) & 1, abort, a.err, kErrTimeoutS)) { ok = false; break; }
        tc_fence_after();
        float x[16];
        tmem_ld_32x32b_x16(tmem + lane_off + buf * 32 + cb, x);
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&S.s_free[buf]);
        const int key = t * kKeysPerTile + row;
        if ((t * kKeysPerTile + kKeysPerTile - 1) > min_limit || (t + 1) * kKeysPerTile > L) {
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const int p = (cb + j) / G;
            const int limit = (a.causal && p < ql) ? L - ql + p : L - 1;
            x[j] = key <= limit ? x[j] : -INFINITY;
          }
        }
        // ---- column maxima of the raw scores: this warp's (lane j keeps column cb + j's), then the four warps'
        float wmax = -INFINITY;
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          const float v = warp_max_redux(x[j]);
          wmax = lane == j ? v : wmax;
        }
        if (lane < 16) S.red_max[buf][col][w] = wmax;
        named_barrier(bar_wg, 128);
        const float4 r4 = *reinterpret_cast<const float4*>(S.red_max[buf][col]);
        const float tmax = fmaxf(fmaxf(r4.x, r4.y), fmaxf(r4.z, r4.w)) * a.scale_log2;
        const bool grow = tmax > m_lane + 8.0f;
        // every thread of the group reads the same maxima, so this branch is uniform over its 128 threads
        if (__any_sync(0xffffffffu, grow)) {
          const float m_new = grow ? tmax : m_lane;
          const float alpha_lane = ex2_approx(m_lane - m_new);   // 1 if unchanged, 0 from the start value
          m_lane = m_new;
          float alpha[16];
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            alpha[j] = __shfl_sync(0xffffffffu, alpha_lane, j);
            m_all[j] = __shfl_sync(0xffffffffu, m_new, j);
            l_part[j] *= alpha[j];
          }
          if (t > t0) {     // O holds this item's earlier tiles: rescale it once PV(g-1) has landed
            if (!mbar_wait(&S.o_done[(g - 1) & 1], ((g - 1) >> 1) & 1, abort, a.err, kErrTimeoutO)) { ok = false; break; }
            tc_fence_after();
            float o[16];
            tmem_ld_32x32b_x16(tmem_o, o);
#pragma unroll
            for (int j = 0; j < 16; ++j) o[j] *= alpha[j];
            tmem_st_32x32b_x16(tmem_o, o);
          }
        }
        // ---- probabilities relative to the running maxima (masked scores give ex2(-inf) = 0)
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          x[j] = ex2_approx(fmaf(x[j], a.scale_log2, -m_all[j]));
          l_part[j] += x[j];
        }
        // ---- this group's half of P^T row `row` (16 bf16, 32 bytes) into the SW64 buffer once PV(g-2) released it
        if (g >= 2 && !mbar_wait(&S.o_done[buf], ((g - 2) >> 1) & 1, abort, a.err, kErrTimeoutO)) { ok = false; break; }
        unsigned char* prow = sP + buf * kPBytes + row * 64;
#pragma unroll
        for (int h2 = 0; h2 < 2; ++h2) {
          uint4 chunk;
          uint32_t* wds = reinterpret_cast<uint32_t*>(&chunk);
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            __nv_bfloat162 pair = __floats2bfloat162_rn(x[h2 * 8 + 2 * e], x[h2 * 8 + 2 * e + 1]);
            wds[e] = *reinterpret_cast<uint32_t*>(&pair);
          }
          const int phys = (2 * wg + h2) ^ ((row >> 1) & 3);
          *reinterpret_cast<uint4*>(prow + phys * 16) = chunk;
        }
        // ---- the row's last tile: V rows past the context are zeroed (they may hold stale bits, even NaN);
        // each group zeroes one 64-dim half of the row
        if ((t + 1) * kKeysPerTile > L) {
          const int stage = g % kStages;
          if (!mbar_wait(&S.v_full[stage], (g / kStages) & 1, abort, a.err, kErrTimeoutV)) { ok = false; break; }
          if (key >= L) {
            uint4 zero = make_uint4(0, 0, 0, 0);
            unsigned char* v0 = sV + stage * kTileBytes + wg * kHalfTileBytes + row * 128;
#pragma unroll
            for (int cc = 0; cc < 8; ++cc) *reinterpret_cast<uint4*>(v0 + cc * 16) = zero;
          }
        }
        fence_proxy_async_smem();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&S.p_full[buf]);
      }
      if (!ok) break;
      // ---- item epilogue: column sums over the 128 key threads (lane j ends with column cb + (j & 15)'s), O^T
      // out of TMEM (the buffer is then free for the item after next)
      {
        const float s = column_reduce16(l_part, lane);
        if (lane < 16) S.red_sum[col][w] = s;
      }
      named_barrier(bar_wg, 128);
      const int gl = g - 1;
      if (!mbar_wait(&S.o_done[gl & 1], (gl >> 1) & 1, abort, a.err, kErrTimeoutO)) break;
      tc_fence_after();
      float o[16];
      tmem_ld_32x32b_x16(tmem_o, o);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&S.o_free[n & 1]);
      const float4 s4 = *reinterpret_cast<const float4*>(S.red_sum[col]);
      float l_lane = (s4.x + s4.y) + (s4.z + s4.w);
      // ---- an item split over CTAs c_lo..c_hi: every piece but the last to arrive is published; the last merges
      // them in CTA order (its own from registers when it holds the first piece and finds every other piece already
      // published; from its published copy otherwise), so the output does not depend on which CTA arrived last
      const long long A = wk.A;
      if (c_lo != c_hi) {
        int* counter = a.counters + (long long)wk.b * a.Hkv + wk.h;
        if (threadIdx.x == 128) {
          // the first piece arriving last (the usual case: it ends this CTA's share) skips its own publication
          const int need = (int)(c_hi - c_lo);
          S.last_piece = (c == c_lo && (seen_early == need || ld_acquire_gpu(counter) == need)) ? 2 : 0;
        }
        named_barrier(3, 256);
        const bool own_in_registers = S.last_piece == 2;
        if (!own_in_registers) {
          float* mine = a.partial + (2LL * c + (x_begin < A ? 1 : 0)) * kPartialFloats;
#pragma unroll
          for (int j = 0; j < 16; ++j) __stcg(mine + (cb + j) * kHeadDim + row, o[j]);
          if (w == 0 && lane < 16) {
            __stcg(mine + kCols * kHeadDim + col, m_lane);
            __stcg(mine + kCols * kHeadDim + kCols + col, l_lane);
          }
          __threadfence();
          named_barrier(3, 256);             // both groups published
          if (threadIdx.x == 128) {
            const int last = atomicAdd(counter, 1) == (int)(c_hi - c_lo);
            if (last) atomicExch(counter, 0);
            S.last_piece = last;
          }
          named_barrier(3, 256);
          // S.last_piece is next written at the next split item's epilogue, which thread 128 reaches only after
          // every softmax warp has handed over P for that item's tiles (so after every thread's read here)
          if (!S.last_piece) continue;
        } else if (threadIdx.x == 128) {
          atomicExch(counter, 0);            // every other piece has arrived: nobody else touches it
        }
        __threadfence();
        // lane j merges column cb + (j & 15)'s maximum and sum; one merge step per piece, the same arithmetic for
        // a piece from registers or from memory
        float m_acc = kNegBig, l_acc = 0.0f;
        const float m_own = m_lane, l_own = l_lane;
        auto merge = [&](float mp, float lp, const float* op) {
          const float mn = fmaxf(m_acc, mp);
          const float sa = ex2_approx(m_acc - mn), sb = ex2_approx(mp - mn);
          m_acc = mn;
          l_acc = __fmaf_rn(lp, sb, __fmul_rn(l_acc, sa));
#pragma unroll
          for (int j = 0; j < 16; ++j)
            o[j] = __fmaf_rn(op ? __ldcg(op + (cb + j) * kHeadDim + row) : o[j], __shfl_sync(0xffffffffu, sb, j),
                             __fmul_rn(op ? o[j] : 0.0f, __shfl_sync(0xffffffffu, sa, j)));
        };
        long long cc = c_lo;
        if (own_in_registers) {
          merge(m_own, l_own, nullptr);      // piece c_lo = this CTA's
          ++cc;
        } else {
#pragma unroll
          for (int j = 0; j < 16; ++j) o[j] = 0.0f;
        }
        for (; cc <= c_hi; ++cc) {
          const long long s_cc = T * cc / Ge;
          const float* piece = a.partial + (2 * cc + (s_cc < A ? 1 : 0)) * kPartialFloats;
          merge(__ldcg(piece + kCols * kHeadDim + col), __ldcg(piece + kCols * kHeadDim + kCols + col), piece);
        }
        l_lane = l_acc;
      }
      // ---- O^T / l, bf16, to out[token, head, dim]
      const float inv_lane = l_lane > 0.0f ? 1.0f / l_lane : 0.0f;
      const int d = row;
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const int p = (cb + j) / G, gq = (cb + j) % G;
        const float inv = __shfl_sync(0xffffffffu, inv_lane, j);
        if (p < ql) {
          const long long off =
              (long long)(wk.r.q_start + p) * a.out_row_stride + (long long)(wk.h * G + gq) * kHeadDim + d;
          const __nv_bfloat16 value = __float2bfloat16_rn(o[j] * inv);
          a.out[off] = value;
          if constexpr (kPeers) {
#pragma unroll
            for (int t = 0; t < kMaxOuts - 1; ++t)   // unrolled: static parameter reads
              if (t < peers.n) peers.out[t][off] = value;
          }
        }
      }
      // peer stores ordered (system scope) before anything this thread does later, the barrier's signal included
      if constexpr (kPeers) __threadfence_system();
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

// ---------------------------------------------------------------------------------------- K/V store
// One warp per token: the token's K and V rows (Hkv * D bf16 each) to its slot; slot < 0 is skipped.
__global__ void __launch_bounds__(256) store_kv_kernel(const __nv_bfloat16* key, long long key_stride,
                                                       const __nv_bfloat16* value, long long value_stride,
                                                       __nv_bfloat16* k_cache, __nv_bfloat16* v_cache,
                                                       const int* slot_mapping, long long N, int row_elems,
                                                       long long num_slots, int* err) {
  const long long t = (long long)blockIdx.x * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (t >= N) return;
  const long long slot = slot_mapping[t];
  if (slot < 0) return;
  if (slot >= num_slots) {
    if (lane == 0) atomicCAS(err, 0, 3);
    return;
  }
  const int nvec = row_elems / 8;    // 16-byte vectors
  const uint4* ks = reinterpret_cast<const uint4*>(key + t * key_stride);
  const uint4* vs = reinterpret_cast<const uint4*>(value + t * value_stride);
  uint4* kd = reinterpret_cast<uint4*>(k_cache + slot * row_elems);
  uint4* vd = reinterpret_cast<uint4*>(v_cache + slot * row_elems);
  for (int i = lane; i < nvec; i += 32) {
    kd[i] = ks[i];
    vd[i] = vs[i];
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

// 3-D bf16 tensor map (dim0 contiguous), 128-byte swizzle, box {64, box1, box2}.
static int make_map(CUtensorMap* map, const void* base, uint64_t d0, uint64_t d1, uint64_t d2, uint64_t stride1_bytes,
                    uint64_t stride2_bytes, uint32_t box1, uint32_t box2) {
  auto fn = encoder();
  if (!fn) return set_error(kCudaError, "cuTensorMapEncodeTiled is unavailable from the driver");
  if ((reinterpret_cast<uintptr_t>(base) & 15) || (stride1_bytes & 15) || (stride2_bytes & 15))
    return set_error(kInvalidArgument, "TMA needs 16-byte aligned base and strides (base %p, strides %llu, %llu)",
                     base, (unsigned long long)stride1_bytes, (unsigned long long)stride2_bytes);
  cuuint64_t dims[3] = {d0, d1, d2};
  cuuint64_t strides[2] = {stride1_bytes, stride2_bytes};
  cuuint32_t box[3] = {64, box1, box2};
  cuuint32_t elem[3] = {1, 1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box, elem,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(kCudaError, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return kOk;
}

template <int G, bool kPeers>
static int launch(const CUtensorMap& qm, const CUtensorMap& km, const CUtensorMap& vm, const CUtensorMap& km32,
                  const CUtensorMap& vm32, const Args& a, const PeerOuts& peers, int grid, bool early,
                  cudaStream_t stream) {
  if (int st = ensure_dynamic_smem<verify_attention_kernel<G, kPeers>>(kSmemBytes)) return st;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)grid);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = kSmemBytes;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = early ? 1 : 0;
  SPECDEC_CUDA_TRY(cudaLaunchKernelEx(&cfg, verify_attention_kernel<G, kPeers>, qm, km, vm, km32, vm32, a, peers));
  SPECDEC_LAUNCH_CHECK();
  return kOk;
}

// Workspace: two piece slots per SM (a size fixed per device), then R * Hkv arrival counters (256-byte padded).
// The counters sit at the same offset for calls of every shape, so a workspace zeroed once stays valid: every
// call leaves the counters it used at zero, and no call's pieces overlap another call's counters.
static long long partial_bytes(int sm_count) { return 2LL * sm_count * kPartialFloats * 4; }
static long long counters_bytes(long long R, int Hkv) { return (R * Hkv * 4 + 255) / 256 * 256; }
static long long workspace_bytes(long long R, int Hkv, int sm_count) {
  return partial_bytes(sm_count) + counters_bytes(R, Hkv);
}
static_assert((kPartialFloats * 4 * 2) % 256 == 0, "counters stay 256-byte aligned");

}  // namespace attention
}  // namespace specdec

using namespace specdec;

extern "C" {

int specdec_store_kvcache(const void* key, long long key_row_stride, const void* value, long long value_row_stride,
                          void* k_cache, void* v_cache, const int* slot_mapping, long long N, int num_kv_heads,
                          int head_dim, long long num_slots, int* err, void* stream) {
  SPECDEC_CHECK_ARG(key && value && k_cache && v_cache && slot_mapping && err, "null pointer argument");
  SPECDEC_CHECK_ARG(N >= 0 && num_kv_heads >= 1 && head_dim >= 1 && num_slots >= 1, "bad sizes");
  const int row = num_kv_heads * head_dim;
  SPECDEC_CHECK_ARG(row % 8 == 0 && key_row_stride % 8 == 0 && value_row_stride % 8 == 0,
                    "rows must be 16-byte multiples");
  SPECDEC_CHECK_ARG(((reinterpret_cast<uintptr_t>(key) | reinterpret_cast<uintptr_t>(value) |
                      reinterpret_cast<uintptr_t>(k_cache) | reinterpret_cast<uintptr_t>(v_cache)) & 15) == 0,
                    "pointers must be 16-byte aligned");
  if (N == 0) return kOk;
  const long long blocks = (N + 7) / 8;
  attention::store_kv_kernel<<<(unsigned)blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const __nv_bfloat16*>(key), key_row_stride, static_cast<const __nv_bfloat16*>(value),
      value_row_stride, static_cast<__nv_bfloat16*>(k_cache), static_cast<__nv_bfloat16*>(v_cache), slot_mapping, N,
      row, num_slots, err);
  SPECDEC_LAUNCH_CHECK();
  return kOk;
}

long long specdec_attention_workspace_bytes(int R, int num_kv_heads) {
  DeviceInfo info;
  if (R < 1 || num_kv_heads < 1 || device_info(&info) != kOk) return -1;
  return attention::workspace_bytes(R, num_kv_heads, info.sm_count);
}

int specdec_paged_attention_multi(const void* q, long long T, long long q_row_stride, int num_heads,
                                  int num_kv_heads, int head_dim, const void* k_cache, const void* v_cache,
                                  long long num_slots, int block_size, const int* cu_seqlens_q,
                                  const int* cu_seqlens_k, const int* context_lens, int q_per_seq, int R,
                                  const int* block_tables, int W, int max_seqlen_q, float softmax_scale, int causal,
                                  void* const* outs, int num_outs, long long out_row_stride, void* workspace,
                                  long long workspace_bytes, int* err, unsigned flags, void* stream) {
  using namespace attention;
  SPECDEC_CHECK_ARG((flags & ~((unsigned)SPECDEC_ATTN_EARLY_LAUNCH | SPECDEC_ATTN_MAX_CTAS(0xff))) == 0,
                    "unknown flags 0x%x", flags);
  SPECDEC_CHECK_ARG(outs && num_outs >= 1 && num_outs <= kMaxOuts, "num_outs %d: 1 .. %d destinations", num_outs,
                    kMaxOuts);
  for (int t = 0; t < num_outs; ++t)
    SPECDEC_CHECK_ARG(outs[t] && (reinterpret_cast<uintptr_t>(outs[t]) & 1) == 0,
                      "output destination %d null or not 2-byte aligned", t);
  SPECDEC_CHECK_ARG(q && k_cache && v_cache && block_tables && workspace && err, "null pointer argument");
  SPECDEC_CHECK_ARG((reinterpret_cast<uintptr_t>(workspace) & 255) == 0, "workspace must be 256-byte aligned");
  SPECDEC_CHECK_ARG(head_dim == kHeadDim, "head_dim %d: this build implements 128", head_dim);
  SPECDEC_CHECK_ARG(num_kv_heads >= 1 && num_heads % num_kv_heads == 0, "heads %d not a multiple of kv heads %d",
                    num_heads, num_kv_heads);
  const int G = num_heads / num_kv_heads;
  if (G != 1 && G != 2 && G != 4 && G != 8)
    return set_error(kUnsupported, "GQA group %d: this build packs groups of 1, 2, 4 or 8", G);
  SPECDEC_CHECK_ARG(max_seqlen_q >= 1, "max_seqlen_q must be >= 1");
  if (max_seqlen_q * G > kCols)
    return set_error(kUnsupported, "%d queries x group %d exceed the %d packed columns", max_seqlen_q, G, kCols);
  SPECDEC_CHECK_ARG(block_size % kKeysPerTile == 0, "block_size %d must be a multiple of %d", block_size,
                    kKeysPerTile);
  SPECDEC_CHECK_ARG(R >= 1 && R <= 65535 && W >= 1 && T >= 1, "bad row/table sizes");
  SPECDEC_CHECK_ARG((cu_seqlens_q && cu_seqlens_k) || (context_lens && q_per_seq >= 1),
                    "give cu_seqlens_q/k (varlen) or context_lens and q_per_seq (decode)");
  SPECDEC_CHECK_ARG(cu_seqlens_q || (q_per_seq <= max_seqlen_q && (long long)R * q_per_seq <= T),
                    "decode mode: q_per_seq must fit the batch");
  CUtensorMap qm, km, vm, km32, vm32;
  const uint64_t row_bytes = (uint64_t)num_kv_heads * head_dim * 2;
  if (int st = make_map(&qm, q, head_dim, num_heads, T, (uint64_t)head_dim * 2, (uint64_t)q_row_stride * 2, G,
                        kCols / G))
    return st;
  if (int st = make_map(&km, k_cache, head_dim, num_kv_heads, num_slots, (uint64_t)head_dim * 2, row_bytes, 1,
                        kKeysPerTile))
    return st;
  if (int st = make_map(&vm, v_cache, head_dim, num_kv_heads, num_slots, (uint64_t)head_dim * 2, row_bytes, 1,
                        kKeysPerTile))
    return st;
  if (int st = make_map(&km32, k_cache, head_dim, num_kv_heads, num_slots, (uint64_t)head_dim * 2, row_bytes, 1,
                        kSubKeys))
    return st;
  if (int st = make_map(&vm32, v_cache, head_dim, num_kv_heads, num_slots, (uint64_t)head_dim * 2, row_bytes, 1,
                        kSubKeys))
    return st;
  Args a{};
  a.cu_seqlens_q = cu_seqlens_q;
  a.cu_seqlens_k = cu_seqlens_k;
  a.context_lens = context_lens;
  a.q_per_seq = q_per_seq;
  a.block_tables = block_tables;
  a.W = W;
  a.block_size = block_size;
  a.H = num_heads;
  a.Hkv = num_kv_heads;
  a.scale_log2 = softmax_scale * 1.4426950408889634f;
  a.causal = causal;
  a.out = static_cast<__nv_bfloat16*>(outs[0]);
  a.out_row_stride = out_row_stride;
  PeerOuts peers{};
  for (int t = 1; t < num_outs; ++t) peers.out[t - 1] = static_cast<__nv_bfloat16*>(outs[t]);
  peers.n = num_outs - 1;
  a.err = err;
  a.R = R;
  // One CTA per SM, fewer when every row's table holds fewer tiles in total.
  DeviceInfo info;
  if (int st = device_info(&info)) return st;
  const long long max_tiles = (long long)R * num_kv_heads * ((long long)W * block_size / kKeysPerTile);
  const int cap = (int)((flags >> SPECDEC_ATTN_CTAS_SHIFT) & 0xffu);
  const int ctas = cap > 0 && cap < info.sm_count ? cap : info.sm_count;
  const int grid = (int)(max_tiles < ctas ? max_tiles : ctas);
  const long long need = attention::workspace_bytes(R, num_kv_heads, info.sm_count);
  if (workspace_bytes < need)
    return set_error(kWorkspaceTooSmall, "attention workspace of %lld bytes, %lld needed", workspace_bytes, need);
  a.partial = static_cast<float*>(workspace);
  a.counters = reinterpret_cast<int*>(static_cast<unsigned char*>(workspace) + partial_bytes(info.sm_count));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const bool early = (flags & SPECDEC_ATTN_EARLY_LAUNCH) != 0;
  if (peers.n > 0) {
    switch (G) {
      case 1: return launch<1, true>(qm, km, vm, km32, vm32, a, peers, grid, early, s);
      case 2: return launch<2, true>(qm, km, vm, km32, vm32, a, peers, grid, early, s);
      case 4: return launch<4, true>(qm, km, vm, km32, vm32, a, peers, grid, early, s);
      default: return launch<8, true>(qm, km, vm, km32, vm32, a, peers, grid, early, s);
    }
  }
  switch (G) {
    case 1: return launch<1, false>(qm, km, vm, km32, vm32, a, peers, grid, early, s);
    case 2: return launch<2, false>(qm, km, vm, km32, vm32, a, peers, grid, early, s);
    case 4: return launch<4, false>(qm, km, vm, km32, vm32, a, peers, grid, early, s);
    default: return launch<8, false>(qm, km, vm, km32, vm32, a, peers, grid, early, s);
  }
}

int specdec_paged_attention_ex(const void* q, long long T, long long q_row_stride, int num_heads, int num_kv_heads,
                               int head_dim, const void* k_cache, const void* v_cache, long long num_slots,
                               int block_size, const int* cu_seqlens_q, const int* cu_seqlens_k,
                               const int* context_lens, int q_per_seq, int R, const int* block_tables, int W,
                               int max_seqlen_q, float softmax_scale, int causal, void* out, long long out_row_stride,
                               void* workspace, long long workspace_bytes, int* err, unsigned flags, void* stream) {
  void* const outs[1] = {out};
  return specdec_paged_attention_multi(q, T, q_row_stride, num_heads, num_kv_heads, head_dim, k_cache, v_cache,
                                       num_slots, block_size, cu_seqlens_q, cu_seqlens_k, context_lens, q_per_seq, R,
                                       block_tables, W, max_seqlen_q, softmax_scale, causal,
                                       out ? outs : nullptr, 1, out_row_stride, workspace, workspace_bytes, err,
                                       flags, stream);
}

int specdec_paged_attention(const void* q, long long T, long long q_row_stride, int num_heads, int num_kv_heads,
                            int head_dim, const void* k_cache, const void* v_cache, long long num_slots,
                            int block_size, const int* cu_seqlens_q, const int* cu_seqlens_k,
                            const int* context_lens, int q_per_seq, int R, const int* block_tables, int W,
                            int max_seqlen_q, float softmax_scale, int causal, void* out, long long out_row_stride,
                            void* workspace, long long workspace_bytes, int* err, void* stream) {
  return specdec_paged_attention_ex(q, T, q_row_stride, num_heads, num_kv_heads, head_dim, k_cache, v_cache,
                                    num_slots, block_size, cu_seqlens_q, cu_seqlens_k, context_lens, q_per_seq, R,
                                    block_tables, W, max_seqlen_q, softmax_scale, causal, out, out_row_stride,
                                    workspace, workspace_bytes, err, 0u, stream);
}

}  // extern "C"
