#pragma once
// Route selection for the B200 kernels (host only, no CUDA dependency).
//
// Reference counterpart: choose_tile (src/gemm.cpp:12-59) and splitk_S (src/dispatch.hpp:30-53),
// which pick among four gfx950 tiles from a 256-CU wave table. Here the choice is re-derived
// for B200 over three tiles,
//   256 x 256  CTA pair (cluster of 2, tcgen05 cta_group::2), 74 pairs on 148 SMs
//   128 x 256  single CTA
//   128 x 128  single CTA
// and an optional split of K into S segments (FP32 partials in the caller's workspace plus one
// reduce pass). A cost model estimates each candidate's time on `sms` SMs:
//
//   units   = ceil(M/MT) * ceil(N/NT) * S              work items handed out round-robin
//   waves   = ceil(units / (sms / ctas_per_unit))      persistent CTAs (or pairs) take units
//   time    = waves * (ceil(slabs / S) * T_slab + T_tile)   one slab = 128-deep K step
//           + T_fixed                                      the kernel's start-up beyond the smallest
//           + T_reduce + (2S + 1) * M*N*4 / HBM  when S > 1   reduce launch, partial write + read, D
//
// With fewer 256 x 256 tiles than CTA pairs and a deep K, a banded split is a candidate
// (BandedSplit): each of the first L*T pairs takes one long K band of one tile, and the pairs
// left over take the short bands the rest of K is cut into, several tiles each. Every pair then
// walks K in step with the pairs that share its operands, and the split's partials are reduced
// in band order as for split-K.
// On the CTA pair, tiles that do not fill whole waves run with a stream-K tail (pair_stream_k):
// the slabs of the last waves are shared out evenly, so `waves` is fractional, plus the cost of
// handing accumulators between pairs (T_HANDOFF). It needs workspace: stream_k_bytes().
//
// T_slab is the time one SM (or pair) spends per slab: 256x256 and 128x256 tiles do the same
// MMA work per SM per slab; their constants reflect how well each keeps the tensor pipe fed
// (measured: the pair sustains a little more over several waves, the narrow tile streams A at
// half the work per byte).
// The cheapest candidate wins (a later candidate must win by 3%). gemm_workspace_size() and
// gemm() both call route_for(), so the workspace a caller sizes always matches what is used.
#include <cstddef>

namespace mxfp6 {

struct Route {
    int MT;      // tile rows: 256 = CTA pair, 128 = single CTA
    int NT;      // tile columns
    int splits;  // K segments (1 = no split); banded: long bands + short bands
    bool stream_k = false;  // CTA pair: stream-K tail (whole tiles do not fill whole waves)
    bool banded = false;    // CTA pair: banded split (BandedSplit below)
};

// Banded split of T tiles of k_slabs slabs over P CTA pairs (T < P). L = P / T long bands of
// `a` slabs each, one per pair, on the first L*T pairs; the rest of K (k_slabs - L*a slabs) cut
// into n short bands, whose n*T units go round-robin, band by band, to the R = P - L*T pairs
// left, at most q = ceil(n*T / R) each. `a` balances the two: a = q * (k_slabs - L*a) / n.
// Partial j is band j in K order: long bands 0..L-1, then the short bands.
struct BandedSplit {
    int L = 0, a = 0, n = 0;  // L == 0: none
    int splits() const { return L + n; }
};
// First slab and slab count of short band j of n over [L*a, k_slabs).
inline int band_short_begin(int k_slabs, int L, int a, int n, int j) {
    const int ks = k_slabs - L * a;
    return L * a + (int)((long long)ks * j / n);
}
inline BandedSplit banded_split(long long tiles, long long pairs, int k_slabs, int n) {
    BandedSplit b;
    if (tiles <= 0 || tiles >= pairs || n < 1 || k_slabs < 16) return b;
    const int L = (int)(pairs / tiles);
    const long long R = pairs - (long long)L * tiles;
    if (R <= 0) return b;
    const long long q = (n * tiles + R - 1) / R;
    // smallest a with q * ceil((k_slabs - L*a) / n) <= a
    const long long a = (q * k_slabs + (n + L * q) - 1) / (n + L * q);
    if (a < 4 || L * a >= k_slabs || (k_slabs - L * a) < n) return b;
    b.L = L;
    b.a = (int)a;
    b.n = n;
    return b;
}

inline size_t splitk_bytes(int M, int N, int splits) {
    return (size_t)splits * (size_t)M * (size_t)N * sizeof(float);
}

// Workspace of the pair kernel's stream-K tail on `pairs` CTA pairs: one 256 x 256 FP32
// accumulator per pair for hand-offs, then two 8-byte flags per pair.
inline size_t stream_k_bytes(int pairs) {
    return (size_t)pairs * (256 * 256 * sizeof(float) + 2 * sizeof(unsigned long long));
}

// Workspace a route uses: split-K partials, then the stream-K hand-off area.
inline size_t route_ws_bytes(const Route& r, int M, int N, int sms) {
    return (r.splits > 1 ? splitk_bytes(M, N, r.splits) : 0) + (r.stream_k ? stream_k_bytes(sms / 2) : 0);
}

// The pair kernel can run a stream-K tail when its tiles (no K split) leave the last wave of `slots`
// pairs partly empty and there is at least one whole wave, so that every pair's slab range covers
// at least one tile (a tile is then shared by at most two pairs, in one accumulator chain).
inline bool pair_stream_k(long long tiles, int splits, long long slots) {
    return splits == 1 && slots > 0 && tiles >= slots && tiles % slots != 0;
}

// The router takes the tail only where it pays. It costs about as much as 30-35 slabs of a tile
// wherever it runs (the hand-offs, and the skew it puts between the pairs that share operands),
// and saves the idle part of the last wave: (1 - last wave's fill) * slabs per tile. Measured on
// B200 against whole tiles (BF16, L2 flushed and back to back):
//   last wave 2/74:  16 slabs -18%, 32 +3%, 48 +10%, 64 +10%      (4096 x 3584)
//   last wave 4/74:  32 slabs -7%, 64 +6%                          (4096 x 7168)
//   last wave 34/74: 16 slabs -25%, 32 -9%, 48 -4%, 64 -1%, 96 +6% (4096 x 4096)
//   last wave 44/74: 32 slabs -12%, 64 -5%, 126 +1%                (2048 x 6144)
// so it runs where that idle part is at least STREAM_K_MIN_SLABS slabs.
constexpr int STREAM_K_MIN_SLABS = 35;
inline bool pair_stream_k_pays(long long tiles, int splits, long long slots, int k_slabs) {
    return pair_stream_k(tiles, splits, slots) &&
           (slots - tiles % slots) * (long long)k_slabs >= (long long)STREAM_K_MIN_SLABS * slots;
}

inline double route_cost_us(int M, int N, int Kp, int MT, int NT, int S, int sms) {
    const double HBM = 6.5e6;  // bytes per us
    // Fixed cost of a launch beyond the 128x128 kernel's, and of the split-K reduce's own launch,
    // in the model's units. Measured back to back on small shapes, where they dominate: 128x128
    // takes 6-8 us per call, 128x256 about 0.5 us more, the CTA pair about 4 us more, and a split
    // about 5 us more. On those shapes the slab terms read about 1.7x short, so the fixed terms
    // are scaled down by the same factor to keep the two comparable.
    const double T_REDUCE_LAUNCH = 3.0;
    double t_slab, t_tile, t_fixed;
    int per_unit;
    if (MT == 256) {
        t_slab = 0.30;  // us per 128-deep slab of a 256x256 pair tile (4 MMAs of 128x256 per SM)
        t_tile = 0.3;
        t_fixed = 2.5;
        per_unit = 2;
    } else if (NT == 256) {
        // measured against the pair (back to back, B200): 6% slower at 4096^3 (3.5 waves), level
        // or faster at one wave (2048x2048x4096: 21.0 against 22.9 us; 1024x4096x16384: 60.1
        // against 59.9 us)
        t_slab = 0.32;
        t_tile = 1.0;
        t_fixed = 0.3;
        per_unit = 1;
    } else {
        // about 0.9 of the pair's rate per slab at full occupancy (0.38-0.42 us a slab back to
        // back on 64-128 CTAs). At 0.24 the model kept deep-K shapes on one 128x128 wave that
        // run faster split: 2048x1024x12288 39.1 us against 31.9 us as a 2-way split on the pair,
        // 2048x256x4096 15.0 against 12.5 us split 3 ways (back to back, B200).
        t_slab = 0.27;
        t_tile = 0.6;
        t_fixed = 0.0;
        per_unit = 1;
    }
    const long long units = (long long)((M + MT - 1) / MT) * ((N + NT - 1) / NT) * S;
    const long long slots = sms / per_unit > 0 ? sms / per_unit : 1;
    const int slabs = Kp / 128;
    const int per = (slabs + S - 1) / S;
    double waves = (double)((units + slots - 1) / slots);
    double t_handoff = 0.0;
    if (MT == 256 && pair_stream_k_pays(units, S, slots, slabs)) {
        waves = (double)units / (double)slots;
        t_handoff = 30 * t_slab;  // hand-offs and skew: about 30 slabs' worth (measured, above)
    }
    double t = waves * (per * t_slab + t_tile) + t_fixed + t_handoff;
    if (S > 1) t += T_REDUCE_LAUNCH + (2.0 * S + 1.0) * (double)M * N * 4.0 / HBM;
    return t;
}

// The banded split's cost on the CTA pair: the critical path is one long band (a slabs) or a
// short-band pair's q units, plus the reduce over L + n partials.
inline double banded_cost_us(int M, int N, int Kp, int sms, const BandedSplit& b) {
    const double HBM = 6.5e6, T_REDUCE_LAUNCH = 3.0;
    const long long tiles = (long long)((M + 255) / 256) * ((N + 255) / 256);
    const int slabs = Kp / 128;
    const long long R = sms / 2 - (long long)b.L * tiles;
    const long long q = (b.n * tiles + R - 1) / R;
    const int c = (slabs - b.L * b.a + b.n - 1) / b.n;
    const double path = (double)(b.a > q * c ? b.a : q * c);
    const int S = b.splits();
    return path * 0.30 + 0.3 * (double)q + 2.5 + T_REDUCE_LAUNCH + (2.0 * S + 1.0) * (double)M * N * 4.0 / HBM;
}

// The tensor core's FP32 accumulation loses precision in proportion to the number of K blocks
// folded into one accumulator (measured: 3.5e-5 max-norm relative error against an exact sum at
// K = 105728, 1.8e-5 / 1.0e-5 / 0.5e-5 with 2 / 4 / 8 split segments). For FP32 output the route
// therefore keeps every split-K segment within FP32_SEGMENT_K, where the result stays within
// 1e-5 of a sequential FP32 sum; the segments are added by the FP32 reduce pass.
constexpr int FP32_SEGMENT_K = 12288;

inline int fp32_min_splits(int Kp) {
    const int s = (Kp + FP32_SEGMENT_K - 1) / FP32_SEGMENT_K;
    return s < 1 ? 1 : (s > 32 ? 32 : s);
}

inline Route route_for(int M, int N, int Kp, int sms, int min_splits = 1) {
    Route best{128, N >= 256 ? 256 : 128, 1};
    if (M <= 0 || N <= 0 || Kp < 128 || sms <= 0) return best;
    const int slabs = Kp / 128;
    if (min_splits > slabs) min_splits = slabs;
    if (min_splits < 1) min_splits = 1;
    best.splits = min_splits;
    double best_t = route_cost_us(M, N, Kp, best.MT, best.NT, min_splits, sms);
    const int shapes[3][2] = {{256, 256}, {128, 256}, {128, 128}};
    bool first = true;
    for (const auto& sh : shapes) {
        const int MT = sh[0], NT = sh[1];
        if (MT > 128 && sms < 2) continue;
        int s_max = slabs / 4 < 32 ? slabs / 4 : 32;  // every segment keeps >= 4 slabs
        if (s_max < min_splits) s_max = min_splits;
        for (int S = min_splits; S <= (s_max > 1 ? s_max : 1); S++) {
            const double t = route_cost_us(M, N, Kp, MT, NT, S, sms);
            if (first || t < best_t * 0.97) {
                best_t = t;
                best = Route{MT, NT, S};
                first = false;
            }
        }
    }
    const long long tiles = (long long)((M + 255) / 256) * ((N + 255) / 256);
    if (min_splits == 1 && sms >= 2) {
        for (int n = 1; n <= 3; n++) {
            const BandedSplit b = banded_split(tiles, sms / 2, slabs, n);
            if (b.L == 0) continue;
            const double t = banded_cost_us(M, N, Kp, sms, b);
            if (t < best_t * 0.97) {
                best_t = t;
                best = Route{256, 256, b.splits()};
                best.banded = true;
            }
        }
        if (best.banded) return best;
    }
    if (best.MT == 256) best.stream_k = pair_stream_k_pays(tiles, best.splits, sms / 2, slabs);
    return best;
}

}  // namespace mxfp6
