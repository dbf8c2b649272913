// gemv_launch.cuh — host-side dispatch of the GEMV template instances.
#pragma once
#include "gemv.cuh"

// Launch y = W . xn for up to 2 columns with the given epilogue.  Returns
// a cudaError_t.  `pdl` adds programmatic-dependent-launch serialisation so
// the launch overlaps the tail of the previous kernel in the stream.
cudaError_t gemv_launch(const GemvArgs &a, int epi, cudaStream_t st, bool pdl);

// Launch with any number of columns (groups of two per launch).
cudaError_t gemv_launch_cols(GemvArgs a, int ncol, int epi, cudaStream_t st, bool pdl);

// Repack GGUF rows (device memory) into the planes of `w` (already allocated).
cudaError_t repack_launch(const uint8_t *src, QWeight w, cudaStream_t st);

// Number of SMs of the current device (cached per device).
int device_sm_count();

// Launch helper with optional PDL attribute.
template <typename... KArgs, typename... Args>
cudaError_t launch_k(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem,
                     cudaStream_t st, bool pdl, Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    if (pdl) {
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
    }
    return cudaLaunchKernelEx(&cfg, kern, args...);
}
