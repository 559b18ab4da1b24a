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
// Design (B200).  One CTA per (row, KV head).  The row's <= 8 query positions times the GQA group's 4 query
// heads are packed into N = 32 columns, so every K/V tile of that head is read from HBM exactly once.  The
// tensor core runs swap-AB: S^T[128 keys x 32] = K_tile[128 x 128] . Q^T and O^T[128 dims x 32] += V^T . P^T,
// both M = 128 UMMAs with fp32 accumulators in TMEM (S double-buffered, O resident for the whole row).  K and V
// tiles of 128 keys (half a 256-slot block) arrive by TMA through one tensor map over the whole paged cache
// (coordinates: dim, head, physical slot), so the block table is a coordinate, not a gather.
//   warp 0      TMA producer (Q once, then K/V tiles into 3-stage rings)
//   warp 1      TMEM allocator + single-thread MMA issuer
//   warps 4-7   softmax over keys (one TMEM lane = one key), P^T to shared memory, O rescale, epilogue
// The softmax is online per query column with lazy rescaling (O is rescaled only when a column's running max
// grows by more than 2^8), masked by key index (bottom-right causal or context length).  Keys past the row's
// context in its last tile are never read as values: their P is 0 and their V rows are zeroed in shared memory.
#include "common.cuh"
#include "sm100.cuh"

#include <cudaTypedefs.h>
#include <math.h>

namespace specdec {
namespace attention {

using namespace sm100;

constexpr int kHeadDim = 128;
constexpr int kKeysPerTile = 128;
constexpr int kCols = 32;              // packed query columns (group x positions)
constexpr int kStages = 3;             // K ring and V ring depth
constexpr int kThreads = 256;
constexpr int kHalfTileBytes = kKeysPerTile * 128;     // 64 dims x 128 keys bf16 = 16 KB
constexpr int kTileBytes = 2 * kHalfTileBytes;          // 32 KB
constexpr int kQHalfBytes = kCols * 128;                // 32 rows x 64 dims bf16 = 4 KB
constexpr int kPBytes = kKeysPerTile * kCols * 2;       // 8 KB
constexpr uint32_t kTmemCols = 128;                     // S0 | S1 | O | spare

// error codes written to the global error word
constexpr int kErrTimeoutQ = 11, kErrTimeoutK = 12, kErrTimeoutV = 13, kErrTimeoutS = 14, kErrTimeoutP = 15,
              kErrTimeoutO = 16, kErrTimeoutEmpty = 17;

struct Args {
  const int* cu_seqlens_q;   // [R + 1] or null (decode mode)
  const int* cu_seqlens_k;   // [R + 1] or null (decode mode)
  const int* context_lens;   // [R] (decode mode)
  int q_per_seq;             // decode mode: queries per row
  const int* block_tables;   // [R, W]
  int W, block_size;
  int H, Hkv;
  float scale_log2;          // softmax_scale * log2(e)
  int causal;
  __nv_bfloat16* out;        // [T, H, D]
  long long out_row_stride;  // elements between tokens of out
  int* err;                  // global error word (0 = ok)
};

struct Smem {
  uint64_t q_full;
  uint64_t k_full[kStages], k_empty[kStages], v_full[kStages], v_empty[kStages];
  uint64_t s_full[2], s_free[2], p_full[2], o_done[2];
  uint32_t tmem_base;
  int abort;
  float red_max[2][4][32];   // per-warp column maxima, by tile parity
  float red_sum[1][4][32];   // per-warp column sums (epilogue)
};

constexpr int kOffQ = 0;
constexpr int kOffK = kOffQ + 2 * kQHalfBytes;                 // 8 KB
constexpr int kOffV = kOffK + kStages * kTileBytes;
constexpr int kOffP = kOffV + kStages * kTileBytes;
constexpr int kOffCtl = kOffP + 2 * kPBytes;
constexpr int kSmemBytes = kOffCtl + (int)sizeof(Smem) + 1024;   // + alignment slack

// Max over the warp's 32 lanes in one instruction (sm_100a redux.sync on f32).
__device__ __forceinline__ float warp_max_redux(float v) {
  float r;
  asm volatile("redux.sync.max.f32 %0, %1, 0xffffffff;" : "=f"(r) : "f"(v));
  return r;
}

// max (ADD=false) or sum (ADD=true) over the 32 lanes of column `lane`; v is consumed.
template <bool ADD>
__device__ __forceinline__ float column_reduce(float (&v)[32], int lane) {
#pragma unroll
  for (int w = 16; w >= 1; w >>= 1) {
    const bool upper = (lane & w) != 0;
#pragma unroll
    for (int c = 0; c < w; ++c) {
      const float send = upper ? v[c] : v[c + w];
      const float keep = upper ? v[c + w] : v[c];
      const float recv = __shfl_xor_sync(0xffffffffu, send, w);
      v[c] = ADD ? keep + recv : fmaxf(keep, recv);
    }
  }
  return v[0];
}

template <int G>
__global__ void __launch_bounds__(kThreads, 1)
    verify_attention_kernel(const __grid_constant__ CUtensorMap qmap, const __grid_constant__ CUtensorMap kmap,
                            const __grid_constant__ CUtensorMap vmap, const Args a) {
  constexpr int QMAX = kCols / G;     // query positions per row this build packs
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* base = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  unsigned char* sQ = base + kOffQ;
  unsigned char* sK = base + kOffK;
  unsigned char* sV = base + kOffV;
  unsigned char* sP = base + kOffP;
  Smem& S = *reinterpret_cast<Smem*>(base + kOffCtl);

  const int h = blockIdx.x;
  const int b = blockIdx.y;
  int q_start, ql, L;
  if (a.cu_seqlens_q) {
    q_start = a.cu_seqlens_q[b];
    ql = a.cu_seqlens_q[b + 1] - q_start;
    L = a.cu_seqlens_k[b + 1] - a.cu_seqlens_k[b];
  } else {
    q_start = b * a.q_per_seq;
    ql = a.q_per_seq;
    L = a.context_lens[b];
  }
  if (ql <= 0) return;
  if (ql > QMAX || L <= 0 || L > a.W * a.block_size) {   // inconsistent metadata: report, never read past it
    if (threadIdx.x == 0) atomicCAS(a.err, 0, 2);
    return;
  }
  const int nt = (L + kKeysPerTile - 1) / kKeysPerTile;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    mbar_init(&S.q_full, 1);
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&S.k_full[s], 1);
      mbar_init(&S.k_empty[s], 1);
      mbar_init(&S.v_full[s], 1);
      mbar_init(&S.v_empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&S.s_full[i], 1);
      mbar_init(&S.s_free[i], 4);     // one elected arrival per softmax warp
      mbar_init(&S.p_full[i], 4);
      mbar_init(&S.o_done[i], 1);
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
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = S.tmem_base;
  volatile int* abort = &S.abort;

  if (warp == 0) {
    // ------------------------------------------------------------------ TMA producer
    if (lane == 0) {
      mbar_arrive_expect_tx(&S.q_full, 2 * kQHalfBytes);
      tma_load_3d(sQ, &qmap, 0, h * G, q_start, &S.q_full);
      tma_load_3d(sQ + kQHalfBytes, &qmap, 64, h * G, q_start, &S.q_full);
      const int* table = a.block_tables + (long long)b * a.W;
      for (int t = 0; t < nt && !*abort; ++t) {
        const int stage = t % kStages;
        const uint32_t use = t / kStages;
        const int key0 = t * kKeysPerTile;
        const int slot = table[key0 / a.block_size] * a.block_size + key0 % a.block_size;
        if (t >= kStages && !mbar_wait(&S.k_empty[stage], (use - 1) & 1, abort, a.err, kErrTimeoutEmpty)) break;
        mbar_arrive_expect_tx(&S.k_full[stage], kTileBytes);
        tma_load_3d(sK + stage * kTileBytes, &kmap, 0, h, slot, &S.k_full[stage]);
        tma_load_3d(sK + stage * kTileBytes + kHalfTileBytes, &kmap, 64, h, slot, &S.k_full[stage]);
        if (t >= kStages && !mbar_wait(&S.v_empty[stage], (use - 1) & 1, abort, a.err, kErrTimeoutEmpty)) break;
        mbar_arrive_expect_tx(&S.v_full[stage], kTileBytes);
        tma_load_3d(sV + stage * kTileBytes, &vmap, 0, h, slot, &S.v_full[stage]);
        tma_load_3d(sV + stage * kTileBytes + kHalfTileBytes, &vmap, 64, h, slot, &S.v_full[stage]);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      const uint32_t idesc_s = idesc_bf16_f32(128, kCols, 0, 0);
      const uint32_t idesc_o = idesc_bf16_f32(128, kCols, 1, 1);
      const uint32_t tmem_o = tmem + 64;
      bool ok = mbar_wait(&S.q_full, 0, abort, a.err, kErrTimeoutQ);
      auto issue_s = [&](int t) -> bool {
        const int stage = t % kStages;
        if (!mbar_wait(&S.k_full[stage], (t / kStages) & 1, abort, a.err, kErrTimeoutK)) return false;
        if (t >= 2 && !mbar_wait(&S.s_free[t & 1], ((t - 2) >> 1) & 1, abort, a.err, kErrTimeoutS)) return false;
        tc_fence_after();
        const unsigned char* kt = sK + stage * kTileBytes;
        const uint32_t tmem_s = tmem + (t & 1) * 32;
#pragma unroll
        for (int kk = 0; kk < kHeadDim / 16; ++kk) {
          const int half = kk >> 2, sub = (kk & 3) * 32;
          const uint64_t adesc = smem_desc(kt + half * kHalfTileBytes + sub, 16, 1024, kSwizzle128B);
          const uint64_t bdesc = smem_desc(sQ + half * kQHalfBytes + sub, 16, 1024, kSwizzle128B);
          mma_bf16_ss(tmem_s, adesc, bdesc, idesc_s, kk > 0 ? 1u : 0u);
        }
        mma_commit(&S.s_full[t & 1]);
        mma_commit(&S.k_empty[stage]);
        return true;
      };
      auto issue_pv = [&](int t) -> bool {
        const int stage = t % kStages;
        if (!mbar_wait(&S.p_full[t & 1], (t >> 1) & 1, abort, a.err, kErrTimeoutP)) return false;
        if (!mbar_wait(&S.v_full[stage], (t / kStages) & 1, abort, a.err, kErrTimeoutV)) return false;
        tc_fence_after();
        const unsigned char* vt = sV + stage * kTileBytes;
        const unsigned char* pt = sP + (t & 1) * kPBytes;
#pragma unroll
        for (int kk = 0; kk < kKeysPerTile / 16; ++kk) {
          const uint64_t adesc = smem_desc(vt + kk * 2048, kHalfTileBytes, 1024, kSwizzle128B);
          const uint64_t bdesc = smem_desc(pt + kk * 1024, kPBytes, 512, kSwizzle64B);
          mma_bf16_ss(tmem_o, adesc, bdesc, idesc_o, (t > 0 || kk > 0) ? 1u : 0u);
        }
        mma_commit(&S.o_done[t & 1]);
        mma_commit(&S.v_empty[stage]);
        return true;
      };
      // Two score tiles run ahead of the softmax: S(t + 2) is issued as soon as PV(t) is, so the softmax of
      // tile t + 1 never waits for a score MMA issued after the softmax of tile t.
      if (ok) ok = issue_s(0);
      if (ok && nt > 1) ok = issue_s(1);
      for (int t = 0; t < nt && ok; ++t) {
        ok = issue_pv(t);
        if (ok && t + 2 < nt) ok = issue_s(t + 2);
      }
    }
  } else if (warp >= 4) {
    // ------------------------------------------------------------------ softmax / correction / epilogue
    const int w = warp - 4;                  // TMEM lane quadrant
    const int row = threadIdx.x - 128;       // key within the tile (S^T) / head dim (O^T)
    const uint32_t lane_off = static_cast<uint32_t>(w * 32) << 16;
    const int min_limit = L - ql;            // smallest causal limit among the valid columns
    // Running max per query column, kept identically by every softmax thread in registers (each thread reads
    // the four warps' partial maxima itself), and this thread's partial column sums over its own keys, reduced
    // across the 128 threads once in the epilogue: one named barrier per tile, no serial section.
    float m_run[32], l_part[32];
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      m_run[j] = -INFINITY;
      l_part[j] = 0.0f;
    }
    bool ok = true;
    for (int t = 0; t < nt && ok; ++t) {
      const int buf = t & 1;                 // partial buffers alternate by tile parity (no reuse hazard)
      if (!mbar_wait(&S.s_full[buf], (t >> 1) & 1, abort, a.err, kErrTimeoutS)) { ok = false; break; }
      tc_fence_after();
      float x[32];
      tmem_ld_32x32b_x32(tmem + lane_off + buf * 32, x);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&S.s_free[buf]);
      const int key = t * kKeysPerTile + row;
      const bool tile_masked = (t * kKeysPerTile + kKeysPerTile - 1) > min_limit || (t + 1) * kKeysPerTile > L;
      if (tile_masked) {
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          const int p = j / G;
          const int limit = (a.causal && p < ql) ? L - ql + p : L - 1;
          x[j] = key <= limit ? x[j] * a.scale_log2 : -INFINITY;
        }
      } else {
#pragma unroll
        for (int j = 0; j < 32; ++j) x[j] = x[j] * a.scale_log2;
      }
      // ---- column max over this warp's 32 keys (one warp reduction per column), then the four warps'
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        const float wm = warp_max_redux(x[j]);
        if (lane == j) S.red_max[buf][w][j] = wm;
      }
      named_barrier(1, 128);
      float alpha[32];
      bool any_rescale = false;
#pragma unroll
      for (int j4 = 0; j4 < 8; ++j4) {
        const float4 r0 = reinterpret_cast<const float4*>(S.red_max[buf][0])[j4];
        const float4 r1 = reinterpret_cast<const float4*>(S.red_max[buf][1])[j4];
        const float4 r2 = reinterpret_cast<const float4*>(S.red_max[buf][2])[j4];
        const float4 r3 = reinterpret_cast<const float4*>(S.red_max[buf][3])[j4];
        const float tm[4] = {fmaxf(fmaxf(r0.x, r1.x), fmaxf(r2.x, r3.x)), fmaxf(fmaxf(r0.y, r1.y), fmaxf(r2.y, r3.y)),
                             fmaxf(fmaxf(r0.z, r1.z), fmaxf(r2.z, r3.z)), fmaxf(fmaxf(r0.w, r1.w), fmaxf(r2.w, r3.w))};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int j = j4 * 4 + e;
          alpha[j] = 1.0f;
          if (tm[e] > m_run[j] + 8.0f) {       // lazy rescale: only when the max grows by 2^8
            if (m_run[j] != -INFINITY) {
              alpha[j] = ex2_approx(m_run[j] - tm[e]);
              any_rescale = true;
            } else {
              alpha[j] = 0.0f;
            }
            m_run[j] = tm[e];
          }
        }
      }
      // ---- probabilities relative to the running max; this thread's share of the column sums
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        x[j] = x[j] == -INFINITY ? 0.0f : ex2_approx(x[j] - m_run[j]);
        l_part[j] = l_part[j] * alpha[j] + x[j];
      }
      // ---- P^T row `row` (32 bf16, 64 bytes) into the SW64 buffer once PV(t-2) released it
      if (t >= 2 && !mbar_wait(&S.o_done[buf], ((t - 2) >> 1) & 1, abort, a.err, kErrTimeoutO)) { ok = false; break; }
      unsigned char* prow = sP + buf * kPBytes + row * 64;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        uint4 chunk;
        uint32_t* wds = reinterpret_cast<uint32_t*>(&chunk);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          __nv_bfloat162 pair = __floats2bfloat162_rn(x[c * 8 + 2 * e], x[c * 8 + 2 * e + 1]);
          wds[e] = *reinterpret_cast<uint32_t*>(&pair);
        }
        const int phys = c ^ ((row >> 1) & 3);
        *reinterpret_cast<uint4*>(prow + phys * 16) = chunk;
      }
      // ---- the last tile's V rows past the context are zeroed (they may hold stale bits, even NaN)
      if ((t + 1) * kKeysPerTile > L) {
        const int stage = t % kStages;
        if (!mbar_wait(&S.v_full[stage], (t / kStages) & 1, abort, a.err, kErrTimeoutV)) { ok = false; break; }
        if (key >= L) {
          uint4 zero = make_uint4(0, 0, 0, 0);
          unsigned char* v0 = sV + stage * kTileBytes + row * 128;
#pragma unroll
          for (int c = 0; c < 8; ++c) {
            *reinterpret_cast<uint4*>(v0 + c * 16) = zero;
            *reinterpret_cast<uint4*>(v0 + kHalfTileBytes + c * 16) = zero;
          }
        }
      }
      // ---- rescale O^T (lane = head dim) once PV(t-1) has landed (uniform: every thread decided alike)
      if (any_rescale && t >= 1) {
        if (!mbar_wait(&S.o_done[(t - 1) & 1], ((t - 1) >> 1) & 1, abort, a.err, kErrTimeoutO)) { ok = false; break; }
        tc_fence_after();
        float o[32];
        tmem_ld_32x32b_x32(tmem + lane_off + 64, o);
#pragma unroll
        for (int j = 0; j < 32; ++j) o[j] *= alpha[j];
        tmem_st_32x32b_x32(tmem + lane_off + 64, o);
      }
      fence_proxy_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&S.p_full[buf]);
    }
    // ---- epilogue: column sums over the 128 key threads, then O^T / l, bf16, to out[token, head, dim]
    if (ok) {
      S.red_sum[0][w][lane] = column_reduce<true>(l_part, lane);
      named_barrier(1, 128);
    }
    if (ok && mbar_wait(&S.o_done[(nt - 1) & 1], ((nt - 1) >> 1) & 1, abort, a.err, kErrTimeoutO)) {
      tc_fence_after();
      float o[32];
      tmem_ld_32x32b_x32(tmem + lane_off + 64, o);
      const int d = row;
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        const int p = j / G, g = j % G;
        if (p < ql) {
          const float l = (S.red_sum[0][0][j] + S.red_sum[0][1][j]) + (S.red_sum[0][2][j] + S.red_sum[0][3][j]);
          const float val = l > 0.0f ? o[j] / l : 0.0f;
          a.out[(long long)(q_start + p) * a.out_row_stride + (long long)(h * G + g) * kHeadDim + d] =
              __float2bfloat16_rn(val);
        }
      }
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
static PFN_cuTensorMapEncodeTiled_v12000 encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }
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

template <int G>
static int launch(const CUtensorMap& qm, const CUtensorMap& km, const CUtensorMap& vm, const Args& a, int R,
                  cudaStream_t stream) {
  static bool configured = false;
  if (!configured) {
    SPECDEC_CUDA_TRY(cudaFuncSetAttribute(verify_attention_kernel<G>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          kSmemBytes));
    configured = true;
  }
  dim3 grid(a.Hkv, R);
  verify_attention_kernel<G><<<grid, kThreads, kSmemBytes, stream>>>(qm, km, vm, a);
  SPECDEC_LAUNCH_CHECK();
  return kOk;
}

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

int specdec_paged_attention(const void* q, long long T, long long q_row_stride, int num_heads, int num_kv_heads,
                            int head_dim, const void* k_cache, const void* v_cache, long long num_slots,
                            int block_size, const int* cu_seqlens_q, const int* cu_seqlens_k,
                            const int* context_lens, int q_per_seq, int R, const int* block_tables, int W,
                            int max_seqlen_q, float softmax_scale, int causal, void* out, long long out_row_stride,
                            int* err, void* stream) {
  using namespace attention;
  SPECDEC_CHECK_ARG(q && k_cache && v_cache && block_tables && out && err, "null pointer argument");
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
  CUtensorMap qm, km, vm;
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
  a.out = static_cast<__nv_bfloat16*>(out);
  a.out_row_stride = out_row_stride;
  a.err = err;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  switch (G) {
    case 1: return launch<1>(qm, km, vm, a, R, s);
    case 2: return launch<2>(qm, km, vm, a, R, s);
    case 4: return launch<4>(qm, km, vm, a, R, s);
    default: return launch<8>(qm, km, vm, a, R, s);
  }
}

}  // extern "C"
