#pragma once
// Route selection for the B200 kernel (host only, no CUDA dependency).
//
// Reference counterpart: choose_tile (src/gemm.cpp:12-59) and splitk_S (src/dispatch.hpp:30-53),
// which pick among four gfx950 tiles from a 256-CU wave table. Here the choice is re-derived
// for B200: the kernel has 128-row tiles of width NT in {128, 256} and an optional split of K
// into S segments (FP32 partials in the caller's workspace plus one reduce pass). A small cost
// model estimates each candidate's time on `sms` SMs:
//
//   waves   = ceil(tiles * S / sms)                      persistent CTAs take tiles round-robin
//   mainloop= waves * ceil(slabs / S) * w * T_SLAB       one 128-deep K slab of a 128x256 tile
//   tile    = waves * T_TILE * w                         epilogue + pipeline fill per tile
//             (w = 1 for NT = 256, 0.6 for NT = 128)
//   splitk  = (2*S + 1) * M*N*4 / HBM                    partial write + reduce read + D write
//
// and takes the cheapest (ties: fewer splits, then the wider tile). gemm_workspace_size() and
// gemm() both call route_for(), so the workspace a caller sizes always matches what is used.
#include <cstddef>

namespace mxfp6 {

struct Route {
    int NT;      // tile width (columns of D per tile)
    int splits;  // K segments (1 = no split)
};

inline size_t splitk_bytes(int M, int N, int splits) {
    return (size_t)splits * (size_t)M * (size_t)N * sizeof(float);
}

inline double route_cost_us(int M, int N, int Kp, int NT, int S, int sms) {
    const double T_SLAB = 0.28;   // us: 4 x (128x256x32) MMAs at about 1.9 GHz
    const double T_TILE = 0.8;    // us: per-tile epilogue and ramp for a 256-wide tile
    const double HBM = 6.5e6;     // bytes per us
    const long long tiles = (long long)(M / 128) * ((N + NT - 1) / NT) * S;
    const long long waves = (tiles + sms - 1) / sms;
    const int slabs = Kp / 128;
    const int per = (slabs + S - 1) / S;
    // A 128-wide tile halves the MMA work per slab but not the A traffic: each slab streams
    // 32 KB through shared memory in 256 cycles, at the edge of its bandwidth; charge 0.6.
    const double w = NT == 256 ? 1.0 : 0.6;
    double t = (double)waves * (per * T_SLAB * w + T_TILE * w);
    if (S > 1) t += (2.0 * S + 1.0) * (double)M * N * 4.0 / HBM;
    return t;
}

inline Route route_for(int M, int N, int Kp, int sms) {
    Route best{N >= 256 ? 256 : 128, 1};
    if (M <= 0 || N <= 0 || Kp < 128 || sms <= 0) return best;
    const int slabs = Kp / 128;
    double best_t = route_cost_us(M, N, Kp, best.NT, 1, sms);
    const int widths[2] = {256, 128};
    for (int NT : widths) {
        if (NT == 256 && N < 256) continue;
        const int s_max = slabs / 4 < 32 ? slabs / 4 : 32;  // every segment keeps >= 4 slabs
        for (int S = 1; S <= (s_max > 1 ? s_max : 1); S++) {
            double t = route_cost_us(M, N, Kp, NT, S, sms);
            // a candidate must win by 3% to displace the simpler one found earlier
            if (t < best_t * 0.97) {
                best_t = t;
                best = Route{NT, S};
            }
        }
    }
    return best;
}

}  // namespace mxfp6
