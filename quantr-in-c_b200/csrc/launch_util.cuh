// launch_util.cuh -- host-side launch helper shared by the kernel files:
// cudaLaunchKernelEx with programmatic dependent launch, counted.
#pragma once
#include <atomic>
#include <utility>
#include <cuda_runtime.h>

#include "kernels.cuh"

namespace qr {

extern std::atomic<unsigned long long> g_launches;

template <typename... KArgs, typename... Args>
cudaError_t launch_ex(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, const LaunchCfg& c,
                      Args&&... args)
{
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = c.stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = c.pdl ? 1 : 0;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    g_launches.fetch_add(1, std::memory_order_relaxed);
    return cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
}

// Raises a kernel's dynamic shared-memory limit once per device.
template <typename K>
cudaError_t ensure_smem_attr(K kern, int bytes, int& configured_dev)
{
    int dev = 0;
    cudaGetDevice(&dev);
    if (configured_dev == dev) return cudaSuccess;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    if (e == cudaSuccess) configured_dev = dev;
    return e;
}

} // namespace qr
