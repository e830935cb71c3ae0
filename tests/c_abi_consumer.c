/* A plain C99 consumer of include/gsplat_b200.h, linked against libgsplat_b200.so: the host-only
 * queries (architecture, pair bound, workspace sizes, argument checks) answer without a GPU.  Built and
 * run by tests/test_abi.py; prints one line of results. */
#include <stdio.h>
#include <string.h>

#include "gsplat_b200.h"

int main(void) {
    gs_render_desc d;
    memset(&d, 0, sizeof(d));
    d.mode = GS_MODE_OCTAVE;
    d.B = 1; d.N = 92160; d.C = 3; d.H = 768; d.W = 768; d.tile = 8; d.odds = 1; d.has_theta = 1;
    d.max_octaves = 6; d.cutoff = 3.0f; d.base_texels = 8.0f; d.max_pairs = 48000000; d.pair_capacity = 0;
    const long long bound = (long long)gs_render_pair_bound(&d);
    const unsigned long long ws_f = (unsigned long long)gs_render_workspace_size(&d, 0);
    const unsigned long long ws_b = (unsigned long long)gs_render_workspace_size(&d, 1);
    const int bad = gs_render_fwd(&d, NULL, NULL, NULL, NULL, NULL, NULL, NULL, NULL, 0, NULL);
    d.tile = 5;
    const unsigned long long ws_bad = (unsigned long long)gs_render_workspace_size(&d, 0);
    printf("arch=%d bound=%lld ws_fwd=%llu ws_bwd=%llu bad_args=%d ws_bad_tile=%llu\n", gs_build_arch(), bound,
           ws_f, ws_b, bad, ws_bad);
    return 0;
}
