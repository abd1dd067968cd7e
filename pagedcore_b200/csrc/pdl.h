// Launch of a kernel as a programmatic dependent of the previous kernel on
// its stream (cudaLaunchAttributeProgrammaticStreamSerialization): it may be
// scheduled once every CTA of that kernel has signalled (or exited), and its
// griddepcontrol.wait (pkv::pdl_wait) orders it after that kernel's
// completion.  Every kernel launched this way calls pdl_wait before it reads
// its inputs, writes its outputs or exits.
#pragma once

#include <cuda_runtime.h>

namespace pkv {

template <typename... KernelArgs, typename... Args>
cudaError_t launch_pdl(void (*kernel)(KernelArgs...), dim3 grid, dim3 block, cudaStream_t stream, Args... args) {
    cudaLaunchConfig_t config = {};
    config.gridDim = grid;
    config.blockDim = block;
    config.dynamicSmemBytes = 0;
    config.stream = stream;
    cudaLaunchAttribute attribute[1];
    attribute[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attribute[0].val.programmaticStreamSerializationAllowed = 1;
    config.attrs = attribute;
    config.numAttrs = 1;
    return cudaLaunchKernelEx(&config, kernel, static_cast<KernelArgs>(args)...);
}

}  // namespace pkv
