// Tracing for the C entry points.
//  * NVTX ranges (NVTX 3, header-only: nothing to link; a push / pop is a
//    branch when no tool is attached) around each public call and the
//    refinement's stages, for ncu --nvtx and Nsight timelines.
//  * The reference's BROVISIONML_PROFILE marks (src/profile.cpp:9-29): when
//    the variable is set and not "0", profile_mark synchronises the stream
//    and prints the time since the calling thread's previous mark to stderr;
//    a null name only restarts the interval.
#pragma once

#include <cuda_runtime.h>
#include <nvtx3/nvToolsExt.h>

namespace bvml {

class NvtxRange {
public:
    explicit NvtxRange(const char* name) { nvtxRangePushA(name); }
    ~NvtxRange() { nvtxRangePop(); }
    NvtxRange(const NvtxRange&) = delete;
    NvtxRange& operator=(const NvtxRange&) = delete;
};

bool profile_enabled();
void profile_mark(cudaStream_t s, const char* name);

}  // namespace bvml
