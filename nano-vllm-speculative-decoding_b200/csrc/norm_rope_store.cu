// Kernel (4) ctx_store, and the target-side siblings the verify forward needs around kernel (2).
//
// Reference behaviour (nano-vllm-speculative-decoding):
//   DFlashDraftModel.store_context_kv    nanovllm/models/dflash.py:88-96    per draft layer: k, v = split(W_kv c);
//                                        k = RoPE(k_norm(k)); store_kvcache(k, v, cache[layer], slot_mapping)
//   Qwen3Attention.forward (q/k part)    nanovllm/models/qwen3.py:77-86     q = q_norm(q), k = k_norm(k),
//                                        q, k = RoPE(positions, q, k), then Attention stores k, v
//   RMSNorm.rms_forward / add_rms_forward nanovllm/layers/layernorm.py:16-40  fp32 mean of squares, x * rsqrt(var
//                                        + eps), cast to the input dtype, times the weight
//   apply_rotary_emb                     nanovllm/layers/rotary_embedding.py:6-14  (x1, x2) halves in fp32:
//                                        (x1 cos - x2 sin, x2 cos + x1 sin), cast back
//   SiluAndMul                           nanovllm/layers/activation.py:8-11  silu(x) * y over the two halves
//
// ctx_store design: one launch covers every draft layer.  A warp owns one (token, layer, head) row of 128 dims
// (lane l holds dims 2l, 2l+1 and their RoPE partners 2l+64, 2l+65, as two bf16 pairs, so the row moves in
// 4-byte loads and stores and both partners of each rotation sit in the same lane): the K row is RMS-normalised
// with a warp reduction, rotated with the position's cos/sin, and written with the V row to the slot; slot -1
// rows are skipped before any load.  The kernel is HBM-bound (bytes: read kv, write cache).
#include "common.cuh"

#include <math.h>

namespace specdec {
namespace fused {

constexpr int kHeadDim = 128;

__device__ __forceinline__ float bf16_round(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

// A head row's 4 dims of lane l: x[0], x[1] = dims 2l, 2l+1; x[2], x[3] = dims 2l+64, 2l+65.
__device__ __forceinline__ void load_head(const __nv_bfloat16* row, int lane, float (&x)[4]) {
  const __nv_bfloat162 a = reinterpret_cast<const __nv_bfloat162*>(row)[lane];
  const __nv_bfloat162 b = reinterpret_cast<const __nv_bfloat162*>(row + 64)[lane];
  x[0] = __low2float(a);
  x[1] = __high2float(a);
  x[2] = __low2float(b);
  x[3] = __high2float(b);
}
__device__ __forceinline__ void store_head(__nv_bfloat16* row, int lane, const float (&x)[4]) {
  reinterpret_cast<__nv_bfloat162*>(row)[lane] = __floats2bfloat162_rn(x[0], x[1]);
  reinterpret_cast<__nv_bfloat162*>(row + 64)[lane] = __floats2bfloat162_rn(x[2], x[3]);
}

// RMSNorm of one 128-dim head row (lane layout of load_head), then the weight.
__device__ __forceinline__ void head_rmsnorm(float (&x)[4], const __nv_bfloat16* weight, int lane, float eps) {
  const __nv_bfloat162 wa = reinterpret_cast<const __nv_bfloat162*>(weight)[lane];
  const __nv_bfloat162 wb = reinterpret_cast<const __nv_bfloat162*>(weight + 64)[lane];
  const float w[4] = {__low2float(wa), __high2float(wa), __low2float(wb), __high2float(wb)};
  float ss = x[0] * x[0] + x[1] * x[1] + x[2] * x[2] + x[3] * x[3];
  ss = warp_sum_f32(ss);
  const float r = rsqrtf(ss / kHeadDim + eps);
#pragma unroll
  for (int i = 0; i < 4; ++i) x[i] = bf16_round(bf16_round(x[i] * r) * w[i]);   // x.to(bf16).mul_(weight)
}

// RoPE on the pairs (2l, 2l+64) and (2l+1, 2l+65): cos/sin index = dim % 64.
__device__ __forceinline__ void head_rope(float (&x)[4], const float* cos_sin, int lane) {
  const float2 c = reinterpret_cast<const float2*>(cos_sin)[lane];
  const float2 sn = reinterpret_cast<const float2*>(cos_sin + 64)[lane];
  const float x1a = x[0], x2a = x[2], x1b = x[1], x2b = x[3];
  x[0] = x1a * c.x - x2a * sn.x;
  x[2] = x2a * c.x + x1a * sn.x;
  x[1] = x1b * c.y - x2b * sn.y;
  x[3] = x2b * c.y + x1b * sn.y;
}

struct NormRopeArgs {
  const __nv_bfloat16* x;       // [layers][T][row] activations: (q heads,) k heads, v heads, 128 dims each
  long long x_layer_stride, x_row_stride;
  int T, layers, Hq, Hkv;
  const __nv_bfloat16* q_norm;  // [128] (Hq > 0)
  const __nv_bfloat16* k_norm;  // [layers][128]
  long long k_norm_layer_stride;
  const float* cos_sin;         // [max_position][128]: cos | sin
  const long long* positions;   // [T]
  const int* slot_mapping;      // [T]
  __nv_bfloat16* k_cache;       // [layers][num_slots][Hkv][128]
  __nv_bfloat16* v_cache;
  long long cache_layer_stride, num_slots;
  __nv_bfloat16* q_out;         // [T][Hq][128]
  long long max_position;
  float eps;
  int* err;
};

// grid: (ceil(T * (Hq + Hkv) / 8), layers); 8 warps per CTA, one (token, head) row per warp; V rows are copied by
// the warp that owns the K row of the same head.
__global__ void __launch_bounds__(256) norm_rope_store_kernel(const NormRopeArgs a) {
  griddep_launch_dependents();   // a dependent launched early (verify attention) may start its prologue
  griddep_wait();                // launched as a dependent of the projection that wrote its input
  const int lane = threadIdx.x & 31;
  const long long item = (long long)blockIdx.x * 8 + (threadIdx.x >> 5);
  const int heads = a.Hq + a.Hkv;
  if (item >= (long long)a.T * heads) return;
  const int layer = blockIdx.y;
  const int t = (int)(item / heads);
  const int hh = (int)(item % heads);
  const long long pos = a.positions[t];
  if (pos < 0 || pos >= a.max_position) {
    if (lane == 0) atomicCAS(a.err, 0, 4);
    return;
  }
  const float* cs = a.cos_sin + pos * kHeadDim;
  const __nv_bfloat16* row = a.x + layer * a.x_layer_stride + (long long)t * a.x_row_stride;
  if (hh < a.Hq) {
    float x[4];
    load_head(row + hh * kHeadDim, lane, x);
    head_rmsnorm(x, a.q_norm, lane, a.eps);
    head_rope(x, cs, lane);
    store_head(a.q_out + ((long long)t * a.Hq + hh) * kHeadDim, lane, x);
    return;
  }
  const int h = hh - a.Hq;
  const long long slot = a.slot_mapping[t];
  if (slot < 0) return;
  if (slot >= a.num_slots) {
    if (lane == 0) atomicCAS(a.err, 0, 3);
    return;
  }
  const __nv_bfloat16* ksrc = row + (a.Hq + h) * kHeadDim;
  const __nv_bfloat16* vsrc = row + (a.Hq + a.Hkv + h) * kHeadDim;
  const uint2 vv = reinterpret_cast<const uint2*>(vsrc)[lane];     // 8 bytes of the V row per lane
  float x[4];
  load_head(ksrc, lane, x);
  head_rmsnorm(x, a.k_norm + layer * a.k_norm_layer_stride, lane, a.eps);
  head_rope(x, cs, lane);
  const long long off = layer * a.cache_layer_stride + (slot * a.Hkv + h) * kHeadDim;
  store_head(a.k_cache + off, lane, x);
  reinterpret_cast<uint2*>(a.v_cache + off)[lane] = vv;
}

// ---------------------------------------------------------------------------------------- RMSNorm (+ residual)
// One CTA per token row of `width` bf16 (width % 8 == 0, <= 8192).  With residual: s = x + residual (fp32),
// residual_out = bf16(s), out = norm(s); without: out = norm(x).
__global__ void __launch_bounds__(256) rmsnorm_kernel(const __nv_bfloat16* __restrict__ x,
                                                      const __nv_bfloat16* __restrict__ residual,
                                                      const __nv_bfloat16* __restrict__ weight,
                                                      __nv_bfloat16* __restrict__ out,
                                                      __nv_bfloat16* __restrict__ residual_out, int width, float eps) {
  constexpr int kMaxVec = 4;   // 4 x 8 elements per thread: width <= 256 * 32 = 8192
  __shared__ float red[8];
  griddep_launch_dependents();
  griddep_wait();                // launched as a dependent of the kernel that wrote x
  const long long t = blockIdx.x;
  const uint4* xv = reinterpret_cast<const uint4*>(x + t * width);
  const uint4* rv = residual ? reinterpret_cast<const uint4*>(residual + t * width) : nullptr;
  const int nvec = width / 8;
  float v[kMaxVec][8];
  uint4 wraw[kMaxVec];
  const uint4* wv = reinterpret_cast<const uint4*>(weight);
#pragma unroll
  for (int u = 0; u < kMaxVec; ++u) {          // the weights load while the row is reduced
    const int i = threadIdx.x + u * 256;
    if (i < nvec) wraw[u] = wv[i];
  }
  // every load of the row is issued before the first residual store (the stores would otherwise order them)
  uint4 xraw[kMaxVec], rraw[kMaxVec];
#pragma unroll
  for (int u = 0; u < kMaxVec; ++u) {
    const int i = threadIdx.x + u * 256;
    if (i < nvec) {
      xraw[u] = xv[i];
      if (rv) rraw[u] = rv[i];
    }
  }
  float ss = 0.0f;
#pragma unroll
  for (int u = 0; u < kMaxVec; ++u) {
    const int i = threadIdx.x + u * 256;
    if (i < nvec) {
      float a[8];
      unpack16_bf16(xraw[u], a);
      if (rv) {
        float r[8];
        unpack16_bf16(rraw[u], r);
#pragma unroll
        for (int e = 0; e < 8; ++e) a[e] += r[e];
        uint4 packed;
        uint32_t* w = reinterpret_cast<uint32_t*>(&packed);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          __nv_bfloat162 p2 = __floats2bfloat162_rn(a[2 * e], a[2 * e + 1]);
          w[e] = *reinterpret_cast<uint32_t*>(&p2);
        }
        reinterpret_cast<uint4*>(residual_out + t * width)[i] = packed;
      }
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        v[u][e] = a[e];
        ss += a[e] * a[e];
      }
    }
  }
  ss = warp_sum_f32(ss);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  float total = 0.0f;
#pragma unroll
  for (int w = 0; w < 8; ++w) total += red[w];
  const float rs = rsqrtf(total / width + eps);
#pragma unroll
  for (int u = 0; u < kMaxVec; ++u) {
    const int i = threadIdx.x + u * 256;
    if (i < nvec) {
      float w8[8];
      unpack16_bf16(wraw[u], w8);
      uint4 packed;
      uint32_t* wd = reinterpret_cast<uint32_t*>(&packed);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float y0 = bf16_round(bf16_round(v[u][2 * e] * rs) * w8[2 * e]);
        const float y1 = bf16_round(bf16_round(v[u][2 * e + 1] * rs) * w8[2 * e + 1]);
        __nv_bfloat162 p2 = __floats2bfloat162_rn(y0, y1);
        wd[e] = *reinterpret_cast<uint32_t*>(&p2);
      }
      reinterpret_cast<uint4*>(out + t * width)[i] = packed;
    }
  }
}

// ---------------------------------------------------------------------------------------- SiLU * mul
// gate_up [T, 2I] -> out [T, I] = silu(gate) * up, computed in fp32 and rounded once to bf16.  silu(a) =
// a / (1 + e^-a) with the hardware exp2 and a fast quotient: a few fp32 ulp, far below the bf16 rounding.
__global__ void __launch_bounds__(256) silu_mul_kernel(const __nv_bfloat16* gate_up, __nv_bfloat16* out, long long T,
                                                       int I) {
  griddep_launch_dependents();
  griddep_wait();                // launched as a dependent of the projection that wrote gate_up
  const long long nvec_row = I / 8;
  const long long i = (long long)blockIdx.x * 256 + threadIdx.x;
  if (i >= T * nvec_row) return;
  const long long t = i / nvec_row, c = i % nvec_row;
  const uint4 g = reinterpret_cast<const uint4*>(gate_up + t * 2 * I)[c];
  const uint4 u = reinterpret_cast<const uint4*>(gate_up + t * 2 * I + I)[c];
  float gf[8], uf[8];
  unpack16_bf16(g, gf);
  unpack16_bf16(u, uf);
  uint4 packed;
  uint32_t* wd = reinterpret_cast<uint32_t*>(&packed);
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const float a0 = gf[2 * e], a1 = gf[2 * e + 1];
    const float y0 = __fdividef(a0, 1.0f + __expf(-a0)) * uf[2 * e];
    const float y1 = __fdividef(a1, 1.0f + __expf(-a1)) * uf[2 * e + 1];
    __nv_bfloat162 p2 = __floats2bfloat162_rn(y0, y1);
    wd[e] = *reinterpret_cast<uint32_t*>(&p2);
  }
  reinterpret_cast<uint4*>(out + t * I)[c] = packed;
}

}  // namespace fused
}  // namespace specdec

using namespace specdec;

extern "C" {

int specdec_norm_rope_store(const void* x, long long x_layer_stride, long long x_row_stride, int T, int layers,
                            int num_q_heads, int num_kv_heads, const void* q_norm, const void* k_norm,
                            long long k_norm_layer_stride, const float* cos_sin, long long max_position,
                            const long long* positions, const int* slot_mapping, void* k_cache, void* v_cache,
                            long long cache_layer_stride, long long num_slots, void* q_out, float eps, int* err,
                            void* stream) {
  SPECDEC_CHECK_ARG(x && k_norm && cos_sin && positions && slot_mapping && k_cache && v_cache && err,
                    "null pointer argument");
  SPECDEC_CHECK_ARG(T >= 0 && layers >= 1 && layers <= 65535 && num_kv_heads >= 1 && num_q_heads >= 0,
                    "bad sizes");
  SPECDEC_CHECK_ARG(num_q_heads == 0 || (q_norm && q_out), "q heads need q_norm and q_out");
  // rows move as 4-byte bf16 pairs (8-byte V chunks), cos/sin as float2: 8-byte aligned rows and tables
  auto a8 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 7) == 0; };
  SPECDEC_CHECK_ARG(a8(x) && a8(k_cache) && a8(v_cache) && a8(cos_sin) && (!q_out || a8(q_out)) &&
                        (reinterpret_cast<uintptr_t>(k_norm) & 3) == 0 && (!q_norm || (reinterpret_cast<uintptr_t>(q_norm) & 3) == 0),
                    "x, caches, q_out and cos_sin must be 8-byte aligned, the norm weights 4-byte aligned");
  SPECDEC_CHECK_ARG(x_layer_stride % 4 == 0 && x_row_stride % 4 == 0 && cache_layer_stride % 4 == 0 &&
                        k_norm_layer_stride % 2 == 0,
                    "row, layer and cache strides must keep 8-byte alignment");
  if (T == 0) return kOk;
  fused::NormRopeArgs a{};
  a.x = static_cast<const __nv_bfloat16*>(x);
  a.x_layer_stride = x_layer_stride;
  a.x_row_stride = x_row_stride;
  a.T = T;
  a.layers = layers;
  a.Hq = num_q_heads;
  a.Hkv = num_kv_heads;
  a.q_norm = static_cast<const __nv_bfloat16*>(q_norm);
  a.k_norm = static_cast<const __nv_bfloat16*>(k_norm);
  a.k_norm_layer_stride = k_norm_layer_stride;
  a.cos_sin = cos_sin;
  a.positions = positions;
  a.slot_mapping = slot_mapping;
  a.k_cache = static_cast<__nv_bfloat16*>(k_cache);
  a.v_cache = static_cast<__nv_bfloat16*>(v_cache);
  a.cache_layer_stride = cache_layer_stride;
  a.num_slots = num_slots;
  a.q_out = static_cast<__nv_bfloat16*>(q_out);
  a.max_position = max_position;
  a.eps = eps;
  a.err = err;
  const long long items = (long long)T * (num_q_heads + num_kv_heads);
  dim3 grid((unsigned)((items + 7) / 8), (unsigned)layers);
  SPECDEC_CUDA_TRY(launch_dependent(fused::norm_rope_store_kernel, grid, dim3(256), static_cast<cudaStream_t>(stream),
                                    a));
  SPECDEC_LAUNCH_CHECK();
  return kOk;
}

int specdec_rmsnorm(const void* x, const void* residual, const void* weight, void* out, void* residual_out,
                    long long T, int width, float eps, void* stream) {
  SPECDEC_CHECK_ARG(x && weight && out, "null pointer argument");
  SPECDEC_CHECK_ARG(!residual || residual_out, "residual needs residual_out");
  SPECDEC_CHECK_ARG(width % 8 == 0 && width <= 8192 && width > 0, "width %d must be a multiple of 8 up to 8192",
                    width);
  if (T <= 0) return kOk;
  SPECDEC_CUDA_TRY(launch_dependent(fused::rmsnorm_kernel, dim3((unsigned)T), dim3(256),
                                    static_cast<cudaStream_t>(stream), static_cast<const __nv_bfloat16*>(x),
                                    static_cast<const __nv_bfloat16*>(residual),
                                    static_cast<const __nv_bfloat16*>(weight), static_cast<__nv_bfloat16*>(out),
                                    static_cast<__nv_bfloat16*>(residual_out), width, eps));
  SPECDEC_LAUNCH_CHECK();
  return kOk;
}

int specdec_silu_mul(const void* gate_up, void* out, long long T, int intermediate, void* stream) {
  SPECDEC_CHECK_ARG(gate_up && out, "null pointer argument");
  SPECDEC_CHECK_ARG(intermediate % 8 == 0 && intermediate > 0, "intermediate must be a positive multiple of 8");
  if (T <= 0) return kOk;
  const long long n = T * (intermediate / 8);
  SPECDEC_CUDA_TRY(launch_dependent(fused::silu_mul_kernel, dim3((unsigned)((n + 255) / 256)), dim3(256),
                                    static_cast<cudaStream_t>(stream), static_cast<const __nv_bfloat16*>(gate_up),
                                    static_cast<__nv_bfloat16*>(out), T, intermediate));
  SPECDEC_LAUNCH_CHECK();
  return kOk;
}

}  // extern "C"
