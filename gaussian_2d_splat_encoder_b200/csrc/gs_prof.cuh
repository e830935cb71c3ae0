// Optional CUDA-event timing of library stages (gs_profile_enable / gs_profile_collect).  Events are
// recorded on the launching stream around each stage, so durations are device time of exactly those
// kernels.  Slots: 0 binning, 1 fields fwd, 2 composite, 3 composite bwd + adjoint, 4 fields bwd,
// 5 finalize, 8 encoder input prep, 9..12 encoder convolutions 1..4, 13 heads, 14 GroupNorm/concat,
// 15 encoder coarse render (whole).
#pragma once
#include <cuda_runtime.h>

enum {
    PR_BIN = 0, PR_FIELDS_FWD = 1, PR_COMPOSITE = 2, PR_COMPOSITE_BWD = 3, PR_FIELDS_BWD = 4, PR_FINALIZE = 5,
    PR_ENC_PREP = 8, PR_CONV1 = 9, PR_CONV2 = 10, PR_CONV3 = 11, PR_CONV4 = 12, PR_HEADS = 13, PR_ENC_MISC = 14,
    PR_ENC_RENDER = 15, PR_N = 16
};

bool gs_prof_on();
void gs_prof_push(int region, cudaEvent_t a, cudaEvent_t b);
void gs_count_launch(unsigned long long n);

struct ProfScope {
    bool on;
    int region;
    cudaEvent_t a, b;
    cudaStream_t s;
    ProfScope(int r, cudaStream_t st) : on(gs_prof_on()), region(r), s(st) {
        if (!on) return;
        cudaEventCreate(&a);
        cudaEventCreate(&b);
        cudaEventRecord(a, s);
    }
    void stop() {
        if (!on) return;
        cudaEventRecord(b, s);
        gs_prof_push(region, a, b);
        on = false;
    }
    ~ProfScope() { stop(); }
};
