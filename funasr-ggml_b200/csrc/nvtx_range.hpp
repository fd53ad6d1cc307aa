// Host-side NVTX ranges around the library's phases (step planning and uploads, graph
// capture, graph replay, the greedy loop, scheduler steps, encoder passes), so a
// profiler timeline shows where each call spends its host time. NVTX v3 is header-only:
// without a profiler attached, a range costs a couple of function-pointer checks.
#pragma once

#include <nvtx3/nvToolsExt.h>

namespace fa {

struct NvtxRange {
    explicit NvtxRange(const char* name) { nvtxRangePushA(name); }
    ~NvtxRange() { nvtxRangePop(); }
    NvtxRange(const NvtxRange&) = delete;
    NvtxRange& operator=(const NvtxRange&) = delete;
};

}  // namespace fa
