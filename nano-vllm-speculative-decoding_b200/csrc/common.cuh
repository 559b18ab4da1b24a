// Shared device/host helpers of the B200 verify/accept library.
//
// Everything here is written for sm_100a (B200).  The library is a C-ABI shared object: every entry point
// returns an int status (0 = ok) and records a message for specdec_last_error() on failure.  No entry point
// allocates device memory; callers pass a workspace.
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>
#include <stdio.h>
#include <stdarg.h>

#include <atomic>
#include <mutex>

namespace specdec {

// ------------------------------------------------------------------------------------------- status codes
enum Status : int {
  kOk = 0,
  kInvalidArgument = 1,   // a shape, dtype, pointer or size the host rejected before any launch
  kWorkspaceTooSmall = 2, // the caller's workspace is smaller than the matching *_workspace_bytes query
  kUnsupported = 3,       // a valid request this build does not implement (e.g. top_k above the cap)
  kCudaError = 4,         // a CUDA runtime/driver call failed; the message carries cudaGetErrorString
  kDeviceTimeout = 5,     // a bounded device-side wait gave up (error flag set by a kernel)
};

// Records a printf-style message for specdec_last_error() (thread-local) and returns `code`.
int set_error(int code, const char* fmt, ...);

#define SPECDEC_CHECK_ARG(cond, ...)                                         \
  do {                                                                      \
    if (!(cond)) return ::specdec::set_error(::specdec::kInvalidArgument, __VA_ARGS__); \
  } while (0)

#define SPECDEC_CUDA_TRY(call)                                                         \
  do {                                                                                 \
    cudaError_t err__ = (call);                                                        \
    if (err__ != cudaSuccess)                                                          \
      return ::specdec::set_error(::specdec::kCudaError, "%s failed: %s (%s:%d)", #call, \
                                  cudaGetErrorString(err__), __FILE__, __LINE__);      \
  } while (0)

// Launch-error check right after a <<<>>> launch.
#define SPECDEC_LAUNCH_CHECK() SPECDEC_CUDA_TRY(cudaGetLastError())

// ------------------------------------------------------------------------------------------- dtypes
// Element type codes shared with the Python wrapper (nanovllm_b200/_lib.py).
enum DType : int { kF32 = 0, kBF16 = 1, kF16 = 2 };

inline size_t dtype_bytes(int dtype) { return dtype == kF32 ? 4 : 2; }
inline bool dtype_ok(int dtype) { return dtype == kF32 || dtype == kBF16 || dtype == kF16; }

template <int DT> struct Elem;
template <> struct Elem<kF32> { using T = float; };
template <> struct Elem<kBF16> { using T = __nv_bfloat16; };
template <> struct Elem<kF16> { using T = __half; };

__device__ __forceinline__ float to_f32(float x) { return x; }
__device__ __forceinline__ float to_f32(__nv_bfloat16 x) { return __bfloat162float(x); }
__device__ __forceinline__ float to_f32(__half x) { return __half2float(x); }

// Loads one element bypassing nothing special; used for scattered single reads (draft tokens).
template <typename T>
__device__ __forceinline__ float load_f32(const T* p) { return to_f32(*p); }

// 16-byte streaming load (read-once data: evict-first in L1/L2 is not wanted for rows re-read by the tail
// pass, so this is a plain non-coherent global load).
// Programmatic dependent launch: wait until the grid this one depends on has completed and its writes are
// visible (returns at once for a grid launched without the dependency), and let dependents start launching.
__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void griddep_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" :::); }

// Launches `kernel` as a programmatic dependent of the preceding work on `stream`: its CTAs may become resident
// while that work drains, so the kernel must call griddep_wait() before it reads anything the preceding work
// writes.  Saves the launch gap after each library GEMM in the layer loop.
template <typename... KArgs, typename... Args>
static cudaError_t launch_dependent_smem(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                                         cudaStream_t stream, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}
template <typename... KArgs, typename... Args>
static cudaError_t launch_dependent(void (*kernel)(KArgs...), dim3 grid, dim3 block, cudaStream_t stream,
                                    Args... args) {
  return launch_dependent_smem(kernel, grid, block, 0, stream, args...);
}

__device__ __forceinline__ uint4 ldg16(const void* p) { return __ldg(reinterpret_cast<const uint4*>(p)); }

// Unpacks a 16-byte vector of T into floats; returns the number of lanes (4 for f32, 8 for 16-bit types).
__device__ __forceinline__ void unpack16(const uint4& v, float (&out)[4]) {
  out[0] = __uint_as_float(v.x); out[1] = __uint_as_float(v.y);
  out[2] = __uint_as_float(v.z); out[3] = __uint_as_float(v.w);
}
__device__ __forceinline__ void unpack16_bf16(const uint4& v, float (&out)[8]) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    out[2 * i] = __uint_as_float(w[i] << 16);
    out[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
  }
}
__device__ __forceinline__ void unpack16_f16(const uint4& v, float (&out)[8]) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    __half2 h = *reinterpret_cast<const __half2*>(&w[i]);
    float2 f = __half22float2(h);
    out[2 * i] = f.x;
    out[2 * i + 1] = f.y;
  }
}

// ------------------------------------------------------------------------------------------- ordering keys
// Maps a float to a uint32 whose unsigned order is the float order (-inf < ... < +inf; +NaN above +inf).
__device__ __forceinline__ uint32_t ordered_key(float f) {
  uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float key_to_float(uint32_t k) {
  uint32_t u = (k & 0x80000000u) ? (k & 0x7fffffffu) : ~k;
  return __uint_as_float(u);
}
// argmax key: larger value wins; on equal values the smaller index wins (torch's first-index rule).
__device__ __forceinline__ unsigned long long argmax_key(float value, uint32_t index) {
  return (static_cast<unsigned long long>(ordered_key(value)) << 32) | (0xffffffffu - index);
}
__device__ __forceinline__ uint32_t argmax_key_index(unsigned long long key) {
  return 0xffffffffu - static_cast<uint32_t>(key & 0xffffffffull);
}

__device__ __forceinline__ unsigned long long warp_max_u64(unsigned long long v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    unsigned long long other = __shfl_xor_sync(0xffffffffu, v, o);
    v = other > v ? other : v;
  }
  return v;
}
// Max of a 64-bit key over the warp with two 32-bit warp reductions: the high words, then the low words of the
// lanes holding the winning high word.  All 32 lanes must call it.
__device__ __forceinline__ unsigned long long warp_max_u64_redux(unsigned long long v) {
  const unsigned hi = static_cast<unsigned>(v >> 32), lo = static_cast<unsigned>(v);
  const unsigned mhi = __reduce_max_sync(0xffffffffu, hi);
  const unsigned mlo = __reduce_max_sync(0xffffffffu, hi == mhi ? lo : 0u);
  return (static_cast<unsigned long long>(mhi) << 32) | mlo;
}

__device__ __forceinline__ float warp_max_f32(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
__device__ __forceinline__ float warp_sum_f32(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Histogram add aggregated over the warp: lanes whose (active, bin) agree add once with their count.  Random
// logits concentrate radix digits in a few bins, where per-lane shared atomics would serialise.  Must be called
// by all 32 lanes.
__device__ __forceinline__ void warp_hist_add(unsigned* hist, unsigned bin, bool active) {
  const unsigned tag = active ? bin : 0xffffffffu;
  const unsigned peers = __match_any_sync(0xffffffffu, tag);
  const int leader = __ffs(peers) - 1;
  if (active && (threadIdx.x & 31) == leader) atomicAdd(&hist[bin], (unsigned)__popc(peers));
}

// Descending bitonic sort of P (a power of two, <= 32 * blockDim) 64-bit keys in shared memory, whole block.
__device__ __forceinline__ void block_sort_desc_u64(unsigned long long* keys, int P) {
  for (int size = 2; size <= P; size <<= 1) {
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      for (int i = threadIdx.x; i < P; i += blockDim.x) {
        const int j = i ^ stride;
        if (j > i) {
          const bool desc = (i & size) == 0;
          const unsigned long long ki = keys[i], kj = keys[j];
          if (desc ? (ki < kj) : (ki > kj)) { keys[i] = kj; keys[j] = ki; }
        }
      }
      __syncthreads();
    }
  }
}
__device__ __forceinline__ void block_sort_desc_f32(float* keys, int P) {
  for (int size = 2; size <= P; size <<= 1) {
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      for (int i = threadIdx.x; i < P; i += blockDim.x) {
        const int j = i ^ stride;
        if (j > i) {
          const bool desc = (i & size) == 0;
          const float ki = keys[i], kj = keys[j];
          if (desc ? (ki < kj) : (ki > kj)) { keys[i] = kj; keys[j] = ki; }
        }
      }
      __syncthreads();
    }
  }
}

// Bitonic sort of one 64-bit key per lane across the warp, descending (lane 0 ends with the largest): shuffles
// only, no block barrier.
__device__ __forceinline__ unsigned long long warp_sort_desc_u64(unsigned long long key, int lane) {
#pragma unroll
  for (int size = 2; size <= 32; size <<= 1) {
#pragma unroll
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      const unsigned long long other = __shfl_xor_sync(0xffffffffu, key, stride);
      const bool up = (lane & size) == 0 || size == 32;
      const bool lower = (lane & stride) == 0;
      const unsigned long long hi = key > other ? key : other, lo = key > other ? other : key;
      key = (lower == up) ? hi : lo;
    }
  }
  return key;
}

// Number of keys in a descending list of 32 that are larger than key: branch-free binary lifting (five steps
// find min(count, 31), a sixth adds the 32nd), so independent counts can run interleaved.
__device__ __forceinline__ int count_larger32(const unsigned long long* list, unsigned long long key) {
  int pos = 0;
#pragma unroll
  for (int step = 16; step >= 1; step >>= 1) pos += list[pos + step - 1] > key ? step : 0;
  return pos + (list[pos] > key ? 1 : 0);
}


// The top C of n distinct nonzero keys keys[0..n), descending, into out[0..C) (C <= n): every 32-key chunk is
// sorted by one warp (shuffles), then each key's rank in the
// whole set is its position in its chunk plus, per other chunk, the count of larger keys there (binary search).
// keys is rewritten (chunks sorted, padded with 0 keys to whole chunks: keys needs room for that).  Two barriers.
template <int NT>
__device__ void block_top_sorted(unsigned long long* keys, int n, int C, unsigned long long* out) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int nchunks = (n + 31) / 32;
  for (int c = warp; c < nchunks; c += NT / 32) {
    const int i = c * 32 + lane;
    const unsigned long long k = i < n ? keys[i] : 0ull;
    keys[i] = warp_sort_desc_u64(k, lane);
  }
  __syncthreads();
  for (int t = threadIdx.x; t < nchunks * 32; t += NT) {
    const unsigned long long key = keys[t];
    if (key == 0ull) continue;                       // padding
    int r = 0;                                       // own chunk included: it counts t & 31 (keys are distinct)
    for (int q0 = 0; q0 < nchunks; q0 += 4) {
#pragma unroll
      for (int u = 0; u < 4; ++u)
        r += q0 + u < nchunks ? count_larger32(keys + (q0 + u) * 32, key) : 0;
    }
    if (r < C) out[r] = key;
  }
  __syncthreads();
}

// The C-th largest of the block's NT thread maxima (ties by thread index), returned to every thread.  buf holds
// NT keys of scratch; it is free again when this returns.
template <int NT>
__device__ float block_cth_thread_max(float mx, int C, unsigned long long* buf) {
  __shared__ float s_bound;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const unsigned long long mine = (static_cast<unsigned long long>(ordered_key(mx)) << 32) | (0xffffffffu - threadIdx.x);
  const unsigned long long sorted = warp_sort_desc_u64(mine, lane);
  buf[threadIdx.x] = sorted;
  __syncthreads();
  int r = 0;                         // own list included: it counts lane (keys are distinct)
#pragma unroll
  for (int q = 0; q < NT / 32; ++q) r += count_larger32(buf + q * 32, sorted);
  (void)warp;
  if (r == C - 1) s_bound = key_to_float(static_cast<unsigned>(sorted >> 32));
  __syncthreads();
  return s_bound;
}

// Collection bound: the C-th thread maximum, widened by slack_rel when that is positive.
__device__ __forceinline__ float widened_bound(float b, float slack_rel) {
  return slack_rel > 0.0f ? b - fabsf(b) * slack_rel - 1e-30f : b;
}

// Last phase of a thread-maxima selection: the top C of the *s_count collected keys in buf, in order.
template <int NT>
__device__ int finish_thread_max_selection(int C, unsigned long long* buf, int cap, int* s_count,
                                           unsigned long long** top) {
  __syncthreads();
  const int count = *s_count;
  if (count > cap) return -1;
  const int padded = (count + 31) / 32 * 32;
  if (count <= 1024 && padded + C <= cap) {
    *top = buf + cap - C;
    block_top_sorted<NT>(buf, count, C, *top);
    return count;
  }
  int P = 1;
  while (P < count) P <<= 1;
  for (int i = count + threadIdx.x; i < P; i += NT) buf[i] = 0ull;
  __syncthreads();
  block_sort_desc_u64(buf, P);
  *top = buf;
  return count;
}

// Top-C selection by a thread-maxima bound (whole block of NT threads; C <= NT).  load(g, x) fills the 8 values
// of element group g (missing ones -inf) and returns how many exist.  Every thread's maximum over its groups is
// an element; the C-th largest of those NT maxima is therefore <= the row's C-th largest value, so collecting
// every element at or above it keeps the top C and all of their ties.  slack_rel widens the collection to
// values >= bound - |bound| * slack_rel - 1e-30 (for callers that rank a monotone transform of the loaded values,
// where rounding may tie a slightly smaller value with the bound).  Collected entries are 64-bit keys (ordered value << 32 | ~id, all
// distinct) in buf (capacity cap); the count is returned, or -1 when more than cap elements reach the bound (the
// caller falls back to an exact radix select).  On return buf[0..count) still holds every collected key (in some
// order, padded with 0 keys to a multiple of 32) and *top points at the top C in descending order: inside buf
// past the collected keys, or at buf itself when the count exceeded 1024 (then all of buf[0..count) is sorted).
// Both orderings (the C-th thread maximum, the top C of up to 1024 collected keys) are warp sorts plus
// binary-search ranks: a few block barriers.
template <int NT, int UNROLL, typename Load>
__device__ int select_by_thread_max(int ngroups, int C, Load load, unsigned long long* buf, int cap, int* s_count,
                                    unsigned long long** top, float slack_rel = 0.0f) {
  float mx = -INFINITY;
  // UNROLL groups per thread in flight per iteration (their loads are independent)
  for (int g0 = threadIdx.x; g0 < ngroups; g0 += UNROLL * NT) {
    float x[UNROLL][8];
    int n[UNROLL];
#pragma unroll
    for (int u = 0; u < UNROLL; ++u) {
      const int g = g0 + u * NT;
      n[u] = g < ngroups ? load(g, x[u]) : 0;
    }
#pragma unroll
    for (int u = 0; u < UNROLL; ++u)
#pragma unroll
      for (int e = 0; e < 8; ++e)
        if (e < n[u]) mx = fmaxf(mx, x[u][e]);
  }
  if (threadIdx.x == 0) *s_count = 0;
  const float bound = widened_bound(block_cth_thread_max<NT>(mx, C, buf), slack_rel);
  for (int g0 = threadIdx.x; g0 < ngroups; g0 += UNROLL * NT) {
    float x[UNROLL][8];
    int n[UNROLL];
#pragma unroll
    for (int u = 0; u < UNROLL; ++u) {
      const int g = g0 + u * NT;
      n[u] = g < ngroups ? load(g, x[u]) : 0;
    }
#pragma unroll
    for (int u = 0; u < UNROLL; ++u) {
      const int g = g0 + u * NT;
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        if (e < n[u] && x[u][e] >= bound) {
          const int slot = atomicAdd(s_count, 1);
          if (slot < cap)
            buf[slot] = (static_cast<unsigned long long>(ordered_key(x[u][e])) << 32) | (0xffffffffu - (unsigned)(g * 8 + e));
        }
      }
    }
  }
  return finish_thread_max_selection<NT>(C, buf, cap, s_count, top);
}

// Packed 16-bit pairs (bf16 or f16) and their -inf.
template <typename H2> struct Packed16;
template <> struct Packed16<__nv_bfloat162> {
  static constexpr unsigned kNegInf = 0xff80ff80u;
  __device__ static __forceinline__ void unpack(const uint4& v, float (&out)[8]) { unpack16_bf16(v, out); }
};
template <> struct Packed16<__half2> {
  static constexpr unsigned kNegInf = 0xfc00fc00u;
  __device__ static __forceinline__ void unpack(const uint4& v, float (&out)[8]) { unpack16_f16(v, out); }
};
template <typename H2>
__device__ __forceinline__ H2 as_h2(unsigned u) {
  H2 h;
  memcpy(&h, &u, sizeof(h));
  return h;
}
template <typename H2>
__device__ __forceinline__ H2 group_max_h2(const uint4& w) {
  return __hmax2(__hmax2(as_h2<H2>(w.x), as_h2<H2>(w.y)), __hmax2(as_h2<H2>(w.z), as_h2<H2>(w.w)));
}

// select_by_thread_max over 16-bit values (bf16 or f16) delivered as packed 16-byte groups of 8: load(g) returns
// group g (0 <= g < ngroups, every group full).  Same result as select_by_thread_max on the unpacked values:
// thread maxima and the per-group test run on packed pairs (__hmax2 drops NaN as fmaxf does, and the maximum of
// 16-bit values is exact), so a group costs its loads and a few packed instructions; only a group whose maximum
// reaches the bound is unpacked and its elements collected.
template <int NT, int UNROLL, typename H2, typename LoadPacked>
__device__ int select_by_thread_max_x16(int ngroups, int C, LoadPacked load, unsigned long long* buf, int cap,
                                        int* s_count, unsigned long long** top, float slack_rel = 0.0f) {
  const unsigned neg = Packed16<H2>::kNegInf;
  H2 mx2 = as_h2<H2>(neg);
  for (int g0 = threadIdx.x; g0 < ngroups; g0 += UNROLL * NT) {
    uint4 w[UNROLL];
#pragma unroll
    for (int u = 0; u < UNROLL; ++u) {
      const int g = g0 + u * NT;
      w[u] = g < ngroups ? load(g) : make_uint4(neg, neg, neg, neg);
    }
#pragma unroll
    for (int u = 0; u < UNROLL; ++u) mx2 = __hmax2(mx2, group_max_h2<H2>(w[u]));
  }
  const float mx = fmaxf(__low2float(mx2), __high2float(mx2));
  if (threadIdx.x == 0) *s_count = 0;
  const float bound = widened_bound(block_cth_thread_max<NT>(mx, C, buf), slack_rel);
  for (int g0 = threadIdx.x; g0 < ngroups; g0 += UNROLL * NT) {
    uint4 w[UNROLL];
#pragma unroll
    for (int u = 0; u < UNROLL; ++u) {
      const int g = g0 + u * NT;
      w[u] = g < ngroups ? load(g) : make_uint4(neg, neg, neg, neg);
    }
#pragma unroll
    for (int u = 0; u < UNROLL; ++u) {
      const H2 m2 = group_max_h2<H2>(w[u]);
      const int g = g0 + u * NT;
      // rare: a candidate in this group (padding groups past the range hold -inf, which a -inf bound, fewer than
      // C finite thread maxima, would otherwise admit)
      if (g < ngroups && fmaxf(__low2float(m2), __high2float(m2)) >= bound) {
        float x[8];
        Packed16<H2>::unpack(w[u], x);
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          if (x[e] >= bound) {
            const int slot = atomicAdd(s_count, 1);
            if (slot < cap)
              buf[slot] = (static_cast<unsigned long long>(ordered_key(x[e])) << 32) | (0xffffffffu - (unsigned)(g * 8 + e));
          }
        }
      }
    }
  }
  return finish_thread_max_selection<NT>(C, buf, cap, s_count, top);
}

// Device properties the library needs (cached per device on first use; thread-safe).
struct DeviceInfo {
  int sm_count;
  int max_threads_per_sm;
  int cc_major, cc_minor;
};
int device_info(DeviceInfo* out);

constexpr int kMaxDevices = 64;

// Raises a kernel's dynamic shared-memory limit to `bytes` on the current device, once per device and kernel.
// The attribute belongs to the device that was current when it was set, so a process driving several GPUs needs
// it on each; host threads launching at once serialise on the first call per device only.
template <auto kKernel>
int ensure_dynamic_smem(int bytes) {
  static std::atomic<bool> done[kMaxDevices];
  static std::mutex mu;
  int dev = 0;
  SPECDEC_CUDA_TRY(cudaGetDevice(&dev));
  if (dev < 0 || dev >= kMaxDevices) return set_error(kInvalidArgument, "device ordinal %d out of range", dev);
  if (done[dev].load(std::memory_order_acquire)) return kOk;
  std::lock_guard<std::mutex> lock(mu);
  if (!done[dev].load(std::memory_order_relaxed)) {
    SPECDEC_CUDA_TRY(cudaFuncSetAttribute(kKernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes));
    done[dev].store(true, std::memory_order_release);
  }
  return kOk;
}

}  // namespace specdec
