// Diagnostics of the tensor-core kernels' failure path.
//
// Every mbarrier wait in the tcgen05 kernels is bounded: on expiry the kernel
// sets bit 0 of a caller-provided status word, waits (bounded) for its own
// copies in flight, frees its tensor memory and returns, so the host learns of
// the failure and the context stays usable.  kadllm_diag_wait_timeout runs that
// same bounded wait on an mbarrier nothing ever completes, with a short limit.
#include "tcgen05.cuh"

namespace kb {
namespace {

__global__ void diag_wait_kernel(uint32_t* status, long long max_cycles) {
  __shared__ __align__(8) uint64_t bar;
  if (threadIdx.x == 0) {
    tc::mbar_init(&bar, 1);  // one arrival expected; none will come
    asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
  }
  __syncthreads();
  const bool ok = tc::mbar_wait(&bar, 0, max_cycles);
  if (!ok && threadIdx.x == 0) atomicOr(status, 1u);
}

}  // namespace
}  // namespace kb

extern "C" int kadllm_diag_wait_timeout(uint32_t* status, int64_t max_cycles, void* stream) {
  KB_REQUIRE(status != nullptr && max_cycles >= 1 && max_cycles <= (int64_t(1) << 32), KADLLM_EINVAL,
             "diag: status word and a wait limit of 1 .. 2^32 cycles required");
  kb::diag_wait_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(status, (long long)max_cycles);
  KB_CHECK_LAUNCH("diag wait launch");
  return KADLLM_OK;
}
