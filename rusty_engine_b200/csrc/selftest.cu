// selftest.cu -- a check, on the GPU, of the wind-down the tensor-core kernels do when one of
// their bounded waits runs out.
//
// Every mbarrier wait in the tcgen05 kernels is bounded (tc::mbar_wait, about 1 s of
// globaltimer); when a wait runs out the kernel records DERR_TIMEOUT in its status word, stops
// issuing, releases its tensor memory and returns, so the context stays usable and the host
// call reports RMOE_ERR_DEVICE.  This kernel does the same steps on a barrier that nothing ever
// arrives at (the failure is made by construction, not by a fault): one CTA allocates tensor
// memory, one thread waits with the caller's (short) limit, the CTA records the timeout,
// frees the tensor memory and returns.
#include <cuda_runtime.h>

#include "layer_impl.h"
#include "tc_ptx.cuh"

namespace rmoe {

__global__ void __launch_bounds__(128) selftest_wait_kernel(unsigned* status, uint64_t limit_ns) {
    __shared__ __align__(8) uint64_t bar;
    __shared__ uint32_t tmem_holder;
    const int warp = threadIdx.x >> 5;
    const uint32_t b = smem_u32(&bar);
    if (threadIdx.x == 0) {
        tc::mbar_init(b, 1);  // one arrival expected; nothing arrives
        tc::fence_mbar_init();
    }
    if (warp == 1) tc::tmem_alloc(smem_u32(&tmem_holder), 32);
    __syncthreads();
    if (threadIdx.x == 0 && !tc::mbar_wait(b, 0, limit_ns)) atomicOr(status, (unsigned)DERR_TIMEOUT);
    __syncthreads();
    if (warp == 1) tc::tmem_dealloc(tmem_holder, 32);
}

}  // namespace rmoe

using namespace rmoe;

extern "C" {

rmoe_status rmoe_selftest_bounded_wait(int32_t device, uint32_t limit_us) {
    int ndev = 0;
    if (cudaGetDeviceCount(&ndev) != cudaSuccess || device < 0 || device >= ndev)
        return fail(RMOE_ERR_INVALID, "device %d out of range", device);
    if (limit_us == 0 || limit_us > 1000000) return fail(RMOE_ERR_INVALID, "limit %u us (1 .. 1000000)", limit_us);
    DeviceGuard g(device);
    unsigned* st = nullptr;
    cudaError_t e = cudaMalloc(&st, 4);
    if (e != cudaSuccess) return cuda_fail(e, "self-test status word");
    unsigned v = 0;
    e = cudaMemset(st, 0, 4);
    if (e == cudaSuccess) {
        selftest_wait_kernel<<<1, 128>>>(st, (uint64_t)limit_us * 1000ull);
        e = cudaGetLastError();
    }
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    if (e == cudaSuccess) e = cudaMemcpy(&v, st, 4, cudaMemcpyDeviceToHost);
    cudaFree(st);
    if (e != cudaSuccess) return cuda_fail(e, "self-test kernel");
    if (v & DERR_TIMEOUT)
        return fail(RMOE_ERR_DEVICE, "device status 0x%x: a bounded wait ran out after %u us (DERR_TIMEOUT)", v,
                    limit_us);
    return fail(RMOE_ERR_CUDA, "self-test: the wait did not run out (status 0x%x)", v);
}

}  // extern "C"
