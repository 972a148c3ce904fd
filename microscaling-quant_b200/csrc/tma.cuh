// Tensor Memory Accelerator (TMA) plumbing for sm_100a: tensor-map encoding on the host (through the driver entry
// point, no libcuda link) and the device-side mbarrier / cp.async.bulk.tensor wrappers the staged kernels use.
//
// Every wait on an mbarrier is bounded: after a limit of unsuccessful try_wait rounds (each round the hardware
// suspends the thread for a bounded time) the wait gives up, counts the event in the library's timeout counter
// (read with mxq_device_timeouts), raises the host-mapped wait-status word (read without a device synchronisation
// with mxq_wait_status_word) and the kernel returns instead of hanging. A TMA load always delivers its whole box
// (out-of-range elements zero-filled), so the expected byte counts are exact and the bound is a safety net.
#pragma once
#include <cuda.h>
#include <stdint.h>

#include "common.cuh"

namespace mxq {

// Encode a float32 tiled tensor map over `rank` dims (dims/strides innermost first; strides in bytes for dims 1..),
// box `box`; zero fill out of range, no swizzle. Returns MXQ_OK or an MXQ_ERR_* with the reason recorded.
int encode_tmap_f32(CUtensorMap* map, const void* base, int rank, const uint64_t* dims, const uint64_t* strides,
                    const uint32_t* box);

// The wait-status word: one 32-bit counter in pinned, mapped, portable host memory, allocated on first use (any
// device; the same address serves every device), which a kernel whose bounded wait gave up increments with a
// system-scope atomic. The host reads it with a plain load, so a caller can check it on every call without
// synchronising; it sees the kernels that have finished. nullptr (with the reason recorded) if the allocation
// failed.
unsigned* wait_status_word();

// per translation unit (no relocatable device code): each TU that stages through TMA owns a counter and reports it
static __device__ unsigned int g_wait_timeouts = 0;
constexpr unsigned kWaitLimit = 1u << 22;

// this TU's timeout count (synchronous read)
static inline unsigned read_wait_timeouts() {
  unsigned v = 0;
  cudaMemcpyFromSymbol(&v, g_wait_timeouts, sizeof(v));
  return v;
}

__device__ __forceinline__ unsigned smem_addr(const void* p) { return (unsigned)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void mbar_init(uint64_t* bar, unsigned count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;\n" ::"r"(smem_addr(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
}
__device__ __forceinline__ void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory"); }
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, unsigned bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n" ::"r"(smem_addr(bar)), "r"(bytes)
               : "memory");
}
// true when the phase with the given parity has completed; false after `rounds` unsuccessful rounds
__device__ __forceinline__ bool mbar_try_wait_rounds(uint64_t* bar, unsigned parity, unsigned rounds) {
  const unsigned addr = smem_addr(bar);
  for (unsigned it = 0; it < rounds; it++) {
    unsigned done;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(done)
        : "r"(addr), "r"(parity)
        : "memory");
    if (done) return true;
  }
  return false;
}
// count a wait that gave up: the device counter and the host-mapped status word (if any)
__device__ __forceinline__ void note_wait_timeout(unsigned* status_word) {
  atomicAdd(&g_wait_timeouts, 1u);
  if (status_word) {
    atomicAdd_system(status_word, 1u);
    __threadfence_system();
  }
}
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];\n" ::
          "r"(smem_addr(dst)),
      "l"(map), "r"(x), "r"(y), "r"(smem_addr(bar))
      : "memory");
}
__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, int x, int y, int z, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];\n" ::
          "r"(smem_addr(dst)),
      "l"(map), "r"(x), "r"(y), "r"(z), "r"(smem_addr(bar))
      : "memory");
}

}  // namespace mxq
