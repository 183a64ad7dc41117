#pragma once
// Host-side layout producers for the B200 MXFP6 GEMM. Same names, signatures and caller flow
// as the reference's helpers (reference: include/mxfp6/preprocess.hpp:12-233), so the caller
// sequence
//
//   Aq  = quantize_to_mxfp6(A, M, Kp);            Bq = preprocess_B(B, Kp, N);
//   Bsh = preshuffle_B(Bq);
//   tc  = choose_tile(M, N, Kp);
//   sA  = tile_scale(preprocess_scale(Aq.scales.data(), M, Kp), tc.MPW, K_TILE / 64);
//   sB  = tile_scale(preprocess_scale(Bq.scales.data(), N, Kp), tc.NPW, K_TILE / 64);
//   gemm(ot, M, N, Kp, dA, dBsh, dsA, dsB, dD, Aq.packed_row_bytes, Bq.packed_row_bytes, ws, wsb);
//
// compiles unchanged and produces the device layouts the B200 kernel reads:
//   * A and B^T stay row-major packed FP6 (the tensor-memory accelerator unpacks them);
//     preshuffle_B is therefore the identity on preprocess_B's output.
//   * Scales go into atoms of 128 rows x 4 K-blocks (512 bytes): within an atom, raw scale
//     (row r, block j) sits at byte (r%32)*16 + (r/32)*4 + j; atoms are ordered row-block major,
//     (row/128) * (Kp/128) + (block/4). One atom is exactly what tcgen05.cp copies into tensor
//     memory for one 128-element K slab, and the layout does not depend on the route, so the
//     group/subs arguments of tile_scale only keep the reference's call shape.
#include <algorithm>
#include <cassert>
#include <cmath>
#include <cstring>
#include <vector>

#include "mxfp6/gemm.hpp"  // K_TILE, kpad
#include "mxfp6/types.hpp"

namespace mxfp6 {

// ---- K padding: the "pad B only / compact A" recipe -----------------------------------------
// B (weights) is padded offline to kpad(K) with a zero K-tail; A may keep its compact layout
// (row stride A_row_bytes = fp6_packed_bytes(K)) provided A's scales are extended with a finite
// tail (pad_scales_k). The tensor-memory accelerator cannot address such a stride (it needs a
// multiple of 32 bytes), so gemm() loads compact A with the kernels' software producer, which
// zero-fills each row's K tail instead of reading into the next row: the end pad below is
// accepted but never read.
inline int a_compact_end_pad(int K) {
    return fp6_packed_bytes(kpad(K)) - fp6_packed_bytes(K);
}

// Extend raw scales [dim][K/32] to [dim][kpad(K)/32]; tail blocks get code 127 (2^0) so that a
// zero K-tail contributes 0 rather than NaN.
inline std::vector<uint8_t> pad_scales_k(const uint8_t* scales, int dim, int K) {
    const int sc = K / 32, scp = kpad(K) / 32;
    std::vector<uint8_t> out((size_t)dim * scp, 127);
    for (int r = 0; r < dim; r++)
        std::memcpy(out.data() + (size_t)r * scp, scales + (size_t)r * sc, (size_t)sc);
    return out;
}

// ---- quantisation ---------------------------------------------------------------------------

struct QuantizedMatrix {
    std::vector<uint8_t> packed_data;  // [rows * fp6_packed_bytes(cols)]
    std::vector<uint8_t> scales;       // [rows * (cols/32)]
    int rows, cols;
    int packed_row_bytes;  // fp6_packed_bytes(cols)
    int scale_cols;        // cols / 32
};

namespace detail {
// E8M0 code of the smallest power of two s with s >= max_abs / 7.5 (127 for an all-zero block).
inline uint8_t block_scale_code(float max_abs) {
    if (max_abs == 0.0f) return 127;
    float needed = max_abs / 7.5f;
    int e2;
    float m = std::frexp(needed, &e2);  // needed = m * 2^e2, m in [0.5, 1)
    // needed is a power of two exactly when m == 0.5; then 2^(e2-1) == needed is enough.
    int e = (m == 0.5f) ? e2 - 1 : e2;
    int code = e + 127;
    return (uint8_t)(code < 0 ? 0 : (code > 254 ? 254 : code));
}

// Quantise rows [r0, r1) of a [rows][cols] float matrix into q.
inline void quantize_rows(const float* mat, int cols, int r0, int r1, QuantizedMatrix& q) {
    uint8_t codes[32];
    for (int r = r0; r < r1; r++) {
        const float* row = mat + (size_t)r * cols;
        for (int b = 0; b < cols / 32; b++) {
            const float* x = row + 32 * b;
            float max_abs = 0.0f;
            for (int k = 0; k < 32; k++) {
                float a = std::fabs(x[k]);
                if (a > max_abs) max_abs = a;  // NaN never wins the comparison
            }
            uint8_t sc = block_scale_code(max_abs);
            q.scales[(size_t)r * q.scale_cols + b] = sc;
            float s = e8m0_to_float(sc);
            for (int k = 0; k < 32; k++) codes[k] = float_to_fp6_e2m3(x[k] / s);
            pack_fp6(codes, 32, q.packed_data.data() + (size_t)r * q.packed_row_bytes + 24 * b);
        }
    }
}
}  // namespace detail

// Float [rows][cols] -> MXFP6 (cols % 32 == 0): per 32-block, scale = smallest power of two
// >= max|x|/7.5, codes = nearest E2M3 of x/scale.
inline QuantizedMatrix quantize_to_mxfp6(const float* mat, int rows, int cols) {
    assert(cols % 32 == 0);
    QuantizedMatrix q;
    q.rows = rows;
    q.cols = cols;
    q.packed_row_bytes = fp6_packed_bytes(cols);
    q.scale_cols = cols / 32;
    q.packed_data.assign((size_t)rows * q.packed_row_bytes, 0);
    q.scales.assign((size_t)rows * q.scale_cols, 0);
    detail::quantize_rows(mat, cols, 0, rows, q);
    return q;
}

inline void dequantize_mxfp6(const QuantizedMatrix& q, float* out) {
    std::vector<uint8_t> codes(q.cols);
    for (int r = 0; r < q.rows; r++) {
        unpack_fp6(q.packed_data.data() + (size_t)r * q.packed_row_bytes, q.cols, codes.data());
        for (int c = 0; c < q.cols; c++)
            out[(size_t)r * q.cols + c] =
                fp6_e2m3_to_float(codes[c]) * e8m0_to_float(q.scales[(size_t)r * q.scale_cols + c / 32]);
    }
}

// B[K][N] -> B^T[N][K], quantised per 32-block along K (one scale per column of B).
inline QuantizedMatrix preprocess_B(const float* B, int K, int N) {
    assert(K % 32 == 0);
    std::vector<float> bt((size_t)N * K);
    for (int k = 0; k < K; k++)
        for (int n = 0; n < N; n++) bt[(size_t)n * K + k] = B[(size_t)k * N + n];
    return quantize_to_mxfp6(bt.data(), N, K);
}

// ---- scale layout -----------------------------------------------------------------------------

struct PreprocessedScale {
    std::vector<uint8_t> data;  // B200 atom layout (see the file comment)
    int dim, K;
    int num_tiles;  // dim / 32 (as in the reference)
    int k64_iters;  // K / 64 (as in the reference)
};

inline size_t tiled_scale_bytes(int dim, int K) {
    return (size_t)((dim + 127) / 128) * (size_t)(K / 128) * 512;
}

// Byte offset of raw scale (row r, block j) in the atom layout for a K-wide matrix.
inline size_t tiled_scale_offset(int r, int j, int K) {
    const size_t atom = (size_t)(r / 128) * (size_t)(K / 128) + (size_t)(j / 4);
    return atom * 512 + (size_t)((r % 32) * 16 + ((r % 128) / 32) * 4 + (j % 4));
}

// Raw scales [dim][K/32] (K % 128 == 0) -> atom layout; rows past dim in the last atom hold 127.
inline PreprocessedScale preprocess_scale(const uint8_t* scales, int dim, int K) {
    assert(K % K_TILE == 0);
    PreprocessedScale ps;
    ps.dim = dim;
    ps.K = K;
    ps.num_tiles = dim / 32;
    ps.k64_iters = K / 64;
    ps.data.assign(tiled_scale_bytes(dim, K), 127);
    const int sc = K / 32;
    for (int r = 0; r < dim; r++)
        for (int j = 0; j < sc; j++) ps.data[tiled_scale_offset(r, j, K)] = scales[(size_t)r * sc + j];
    return ps;
}

struct PreshuffledB {
    std::vector<uint8_t> data;  // B^T[N][K] packed rows (identity on preprocess_B's output)
    int N, K;
    int n_tiles;    // N / 32 (as in the reference)
    int k64_iters;  // K / 64 (as in the reference)
};

// On B200 the kernel reads B^T rows directly, so this is a copy of the packed data.
inline PreshuffledB preshuffle_B(const QuantizedMatrix& B_q) {
    PreshuffledB pb;
    pb.N = B_q.rows;
    pb.K = B_q.cols;
    pb.n_tiles = B_q.rows / 32;
    pb.k64_iters = B_q.cols / 64;
    pb.data = B_q.packed_data;
    return pb;
}

struct TiledScale {
    std::vector<uint8_t> data;
};

// The atom layout already is the device layout for every route; group and subs are accepted
// for source compatibility (reference call: tile_scale(ps, tc.MPW|NPW, K_TILE/64)).
inline TiledScale tile_scale(const PreprocessedScale& ps, int group, int subs) {
    (void)group;
    (void)subs;
    TiledScale ts;
    ts.data = ps.data;
    return ts;
}

}  // namespace mxfp6
