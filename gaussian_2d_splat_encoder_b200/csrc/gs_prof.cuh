// Optional CUDA-event timing of library stages (gs_profile_enable / gs_profile_collect).  Events are
// recorded on the launching stream around each stage, so durations are device time of exactly those
// kernels.  Slots: 0 binning, 1 fields fwd, 2 composite, 3 composite bwd + adjoint, 4 fields bwd,
// 5 finalize, 6 binning and 7 fields fwd of the encoder's internal coarse render, 8 encoder input prep,
// 9..12 encoder convolutions 1..4, 13 heads, 14 GroupNorm/concat, 15 encoder coarse render (whole).
#pragma once
#include <cuda_runtime.h>

enum {
    PR_BIN = 0, PR_FIELDS_FWD = 1, PR_COMPOSITE = 2, PR_COMPOSITE_BWD = 3, PR_FIELDS_BWD = 4, PR_FINALIZE = 5,
    PR_ENC_BIN = 6, PR_ENC_FIELDS_FWD = 7, PR_ENC_PREP = 8, PR_CONV1 = 9, PR_CONV2 = 10, PR_CONV3 = 11, PR_CONV4 = 12, PR_HEADS = 13, PR_ENC_MISC = 14,
    PR_ENC_RENDER = 15, PR_N = 16
};

bool gs_prof_on();
// While set (per host thread), a render's binning and field stages are timed in the encoder-render slots
// (6, 7) instead of 0, 1: the encoder sets it around its internal coarse render.
void gs_prof_set_internal(int on);
int gs_prof_internal();
// Takes an event pair from a pre-created pool (NULL events when the pool is exhausted).
void gs_prof_take(int region, cudaEvent_t *a, cudaEvent_t *b);
void gs_count_launch(unsigned long long n);

// Records on a capturing stream become external event-record nodes of the graph, so a graph replay
// re-records them and gs_profile_collect reads the last replay's durations.
inline void gs_prof_record(cudaEvent_t e, cudaStream_t s) {
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    cudaStreamIsCapturing(s, &cs);
    if (cs == cudaStreamCaptureStatusActive) cudaEventRecordWithFlags(e, s, cudaEventRecordExternal);
    else cudaEventRecord(e, s);
}

struct ProfScope {
    bool on;
    cudaEvent_t a, b;
    cudaStream_t s;
    ProfScope(int r, cudaStream_t st) : on(gs_prof_on()), a(nullptr), b(nullptr), s(st) {
        if (!on) return;
        gs_prof_take(r, &a, &b);
        if (!a) { on = false; return; }
        gs_prof_record(a, s);
    }
    void stop() {
        if (!on) return;
        gs_prof_record(b, s);
        on = false;
    }
    ~ProfScope() { stop(); }
};
