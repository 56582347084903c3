// Cross-GPU arrival barrier over NVLink peer memory for the sequence-parallel attention.
//
// Every rank owns `world` 32-bit flags in memory the other ranks have mapped (CUDA IPC). To pass
// barrier number `epoch`, rank r stores epoch into flag r of every rank (a release store at
// system scope, after a system fence that publishes r's earlier stores, among them the q/k/v and
// attention rows it wrote into the other GPUs' buffers) and then waits until each of its own
// flags has reached epoch (acquire loads). A rank that is one barrier ahead may already have
// written epoch + 1, so the wait compares with wrap-around arithmetic. The wait is bounded: after
// KINO_WAIT_NS the kernel records KINO_ETIMEOUT in the device error word and returns.
#pragma once
#include "kino_common.cuh"

namespace kino {

constexpr int PEER_MAX_WORLD = 32;

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__global__ void peer_barrier_kernel(uint32_t* const* __restrict__ flags, int rank, int world,
                                    uint32_t epoch) {
  griddep_wait();
  const int i = threadIdx.x;
  if (i < world) {
    __threadfence_system();
    st_release_sys(flags[i] + rank, epoch);
    const uint32_t* mine = flags[rank] + i;
    const uint64_t start = global_ns();
    while (static_cast<int32_t>(ld_acquire_sys(mine) - epoch) < 0) {
      if (global_ns() - start > KINO_WAIT_NS) {
        atomicExch(&g_device_error, 4);
        break;
      }
    }
  }
  __syncthreads();
  griddep_launch();
}

}  // namespace kino
