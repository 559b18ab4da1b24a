// Cross-GPU barrier of the peer-store tensor-parallel verify attention.
//
// In that mode every rank's attention kernel stores its heads' output straight into every rank's [T, H, D]
// output buffer (peer memory mapped into each process, over NVLink / NVSwitch).  Before a rank reads its buffer
// it must know that every peer's kernel has finished storing into it; this barrier is that step.  It replaces
// the NCCL all-gather that would otherwise follow the attention (the head gather of a tensor-parallel forward
// whose other layers are replicated; the reference's head split is nanovllm/models/qwen3.py:29-35).
//
// Protocol (one block, one thread per rank): each rank keeps a per-rank arrival word in every rank's flag array
// (flags[r][s] = the last epoch rank s reached, as seen by rank r) and a local epoch counter that the kernel
// itself advances, so the same launch replays correctly inside a CUDA graph.  At epoch e thread t of rank r
// release-stores e into flags[t][r] (system scope, after a system fence that orders this GPU's earlier stores,
// including the attention kernel's peer stores, before the signal), then acquire-loads flags[r][t] until it
// reaches e.  Every wait is bounded: past timeout_ns it records kErrPeerTimeout in *err and returns, so the
// context stays usable and the host reads the status.
#include "common.cuh"
#include "sm100.cuh"

namespace specdec {
namespace peer {

constexpr int kMaxRanks = 8;
constexpr int kErrPeerTimeout = 21;

struct BarrierArgs {
  unsigned* flags[kMaxRanks];   // flags[t]: rank t's arrival words (kMaxRanks of them), mapped into this process
  unsigned* epoch;              // this rank's epoch counter (local memory)
  int rank, world;
  unsigned long long timeout_ns;
  int* err;                     // error word (0 = ok)
};

__device__ __forceinline__ void st_release_sys(unsigned* p, unsigned v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__global__ void __launch_bounds__(32) peer_barrier_kernel(const __grid_constant__ BarrierArgs a) {
  const int t = threadIdx.x;
  const unsigned e = *a.epoch + 1u;
  __syncwarp();
  if (t < a.world) {
    asm volatile("fence.acq_rel.sys;" ::: "memory");
    st_release_sys(a.flags[t] + a.rank, e);            // rank a.rank has arrived at epoch e
    const unsigned* mine = a.flags[a.rank] + t;
    const uint64_t start = sm100::global_timer_ns();
    while ((int)(ld_acquire_sys(mine) - e) < 0) {     // wrap-safe: rank t has not reached epoch e yet
      if (sm100::global_timer_ns() - start > a.timeout_ns) {
        atomicCAS(a.err, 0, kErrPeerTimeout);
        break;
      }
      __nanosleep(200);
    }
  }
  __syncwarp();
  if (t == 0) *a.epoch = e;
}

}  // namespace peer
}  // namespace specdec

extern "C" {

int specdec_peer_barrier(void* const* flags, int world, int rank, unsigned* epoch, long long timeout_ns, int* err,
                         void* stream) {
  using namespace specdec;
  using namespace specdec::peer;
  SPECDEC_CHECK_ARG(flags && epoch && err, "null pointer argument");
  SPECDEC_CHECK_ARG((reinterpret_cast<uintptr_t>(epoch) & 3) == 0 && (reinterpret_cast<uintptr_t>(err) & 3) == 0,
                    "epoch and err must be 4-byte aligned");
  SPECDEC_CHECK_ARG(world >= 1 && world <= kMaxRanks && rank >= 0 && rank < world, "rank %d of world %d (1 .. %d)",
                    rank, world, kMaxRanks);
  SPECDEC_CHECK_ARG(timeout_ns > 0, "timeout_ns must be positive");
  BarrierArgs a{};
  for (int t = 0; t < world; ++t) {
    SPECDEC_CHECK_ARG(flags[t] && (reinterpret_cast<uintptr_t>(flags[t]) & 3) == 0,
                      "flag array %d null or not 4-byte aligned", t);
    a.flags[t] = static_cast<unsigned*>(flags[t]);
  }
  a.epoch = epoch;
  a.rank = rank;
  a.world = world;
  a.timeout_ns = (unsigned long long)timeout_ns;
  a.err = err;
  peer_barrier_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(a);
  SPECDEC_LAUNCH_CHECK();
  return kOk;
}

}  // extern "C"
