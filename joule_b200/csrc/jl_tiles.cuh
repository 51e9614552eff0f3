// Token-tile table of the tensor-core path, built at the end of the dispatch
// step (device code shared by jl_router.cu and jl_tc.cu).
#pragma once

#include "jl_common.cuh"
#include "jl_internal.h"

namespace jl {

constexpr int kTcNT = 32;  // max tokens per tile: the MMA's N = 2 x tokens <= 64 TMEM columns

// rows of an expert with n tokens in the padded tile space: full 64-token
// tiles plus the last tile rounded up to a multiple of 16
__device__ __forceinline__ int tc_rows(int n) { return (n / kTcNT) * kTcNT + ((n % kTcNT + 15) & ~15); }

// Tile t = (expert id, tokens, first uidx position, padded row offset). Run by
// one warp once uh/sel are final; writes tc_tile[] and *tc_ntiles.
__device__ __forceinline__ void tc_build_tiles(const jl_ws& ws) {
    const int lane = threadIdx.x & 31;
    const int U = *ws.U;
    int tiles_before = 0, rows_before = 0;
    for (int u0 = 0; u0 < U; u0 += 32) {
        const int u = u0 + lane;
        const int n = (u < U) ? ws.uh[u + 1] - ws.uh[u] : 0;
        const int t = (n + kTcNT - 1) / kTcNT, r = tc_rows(n);
        int ti = t, ri = r;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int a = __shfl_up_sync(0xffffffffu, ti, o);
            const int b = __shfl_up_sync(0xffffffffu, ri, o);
            if (lane >= o) {
                ti += a;
                ri += b;
            }
        }
        if (u < U) {
            const int t_ex = tiles_before + ti - t, r_ex = rows_before + ri - r;
            const int e = ws.sel[u], p0 = ws.uh[u];
            for (int j = 0; j < t; j++) {
                int* tt = ws.tc_tile + (size_t)(t_ex + j) * 4;
                tt[0] = e;
                tt[1] = min(kTcNT, n - j * kTcNT);
                tt[2] = p0 + j * kTcNT;
                tt[3] = r_ex + j * kTcNT;
            }
        }
        tiles_before += __shfl_sync(0xffffffffu, ti, 31);
        rows_before += __shfl_sync(0xffffffffu, ri, 31);
    }
    if (lane == 0) *ws.tc_ntiles = tiles_before;
}

}  // namespace jl
