// Bounded device-side waits: the building block every spinning kernel here uses
// (peer flags in symm.cu, mbarriers in the GEMM / attention kernels), exposed as a
// standalone kernel so that the failure path can be exercised on a real GPU
// without faulting it.
//
// wait_flag_kernel spins on a device word until it reaches `target` or until
// `limit_ns` of globaltimer time has passed; on time-out it records `code` in the
// status word and returns normally, so the context stays usable and the host
// learns about the missing peer / producer by reading the status.
#include "common.cuh"

namespace mtorus {

__global__ void wait_flag_kernel(const uint32_t* flag, uint32_t target, uint64_t limit_ns, int* status,
                                 int code, uint64_t* waited_ns) {
  if (threadIdx.x != 0 || blockIdx.x != 0) return;
  const uint64_t t0 = globaltimer_ns();
  uint64_t now = t0;
  while (true) {
    uint32_t v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(flag) : "memory");
    if ((int32_t)(v - target) >= 0) break;
    now = globaltimer_ns();
    if (now - t0 > limit_ns) {
      atomicExch(status, code);
      break;
    }
    __nanosleep(256);
  }
  *waited_ns = now - t0;
}

// Waits on `flag` (int32 device tensor, 1 element) for at most limit_ms; returns
// nothing -- `status` (int32, 1 element) receives `code` on time-out and `waited`
// (int64, 1 element) the nanoseconds spent.
void wait_flag(const at::Tensor& flag, int64_t target, double limit_ms, at::Tensor status, int64_t code,
               at::Tensor waited) {
  MT_CHECK(flag.is_cuda() && flag.scalar_type() == at::kInt && flag.numel() >= 1, "wait_flag: int32 flag");
  MT_CHECK(status.is_cuda() && status.scalar_type() == at::kInt && status.numel() >= 1, "wait_flag: status");
  MT_CHECK(waited.is_cuda() && waited.scalar_type() == at::kLong && waited.numel() >= 1, "wait_flag: waited");
  MT_CHECK(limit_ms > 0 && limit_ms <= 10000, "wait_flag: limit must be in (0, 10 s]");
  wait_flag_kernel<<<1, 32, 0, cur_stream()>>>(reinterpret_cast<const uint32_t*>(flag.data_ptr()),
                                               (uint32_t)target, (uint64_t)(limit_ms * 1e6),
                                               status.data_ptr<int>(), (int)code,
                                               reinterpret_cast<uint64_t*>(waited.data_ptr()));
  MT_LAUNCH_CHECK();
}

}  // namespace mtorus
