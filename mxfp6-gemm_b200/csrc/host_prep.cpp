// C face of the host preprocessing helpers in include/mxfp6/preprocess.hpp, for bindings that
// cannot instantiate the C++ header (ctypes, cgo, JNI). Quantisation fans rows out over threads;
// every row is quantised by the same code as quantize_to_mxfp6, so the result does not depend
// on the thread count.
#include <algorithm>
#include <thread>
#include <vector>

#include "mxfp6/preprocess.hpp"
#include "mxfp6_gemm.h"

using namespace mxfp6;

extern "C" {

void mxfp6_quantize(const float* mat, int rows, int cols, uint8_t* packed, uint8_t* scales,
                    int nthreads) {
    if (!mat || !packed || !scales || rows <= 0 || cols <= 0 || cols % 32) return;
    const int row_bytes = fp6_packed_bytes(cols), scale_cols = cols / 32;
    int nt = nthreads > 0 ? nthreads : (int)std::thread::hardware_concurrency();
    nt = std::max(1, std::min(nt, std::max(1, rows / 16)));
    // Each thread quantises a contiguous row range into its own QuantizedMatrix and copies it
    // out, so the bytes match a single quantize_to_mxfp6 call on the whole matrix.
    auto work = [&](int t) {
        const int r0 = (int)((long long)rows * t / nt), r1 = (int)((long long)rows * (t + 1) / nt);
        QuantizedMatrix part;
        part.rows = r1 - r0;
        part.cols = cols;
        part.packed_row_bytes = row_bytes;
        part.scale_cols = scale_cols;
        part.packed_data.assign((size_t)part.rows * row_bytes, 0);
        part.scales.assign((size_t)part.rows * scale_cols, 0);
        detail::quantize_rows(mat + (size_t)r0 * cols, cols, 0, part.rows, part);
        std::copy(part.packed_data.begin(), part.packed_data.end(), packed + (size_t)r0 * row_bytes);
        std::copy(part.scales.begin(), part.scales.end(), scales + (size_t)r0 * scale_cols);
    };
    std::vector<std::thread> pool;
    for (int t = 1; t < nt; t++) pool.emplace_back(work, t);
    work(0);
    for (auto& th : pool) th.join();
}

void mxfp6_dequantize(const uint8_t* packed, const uint8_t* scales, int rows, int cols, float* out) {
    if (!packed || !scales || !out || rows <= 0 || cols <= 0 || cols % 32) return;
    QuantizedMatrix q;
    q.rows = rows;
    q.cols = cols;
    q.packed_row_bytes = fp6_packed_bytes(cols);
    q.scale_cols = cols / 32;
    q.packed_data.assign(packed, packed + (size_t)rows * q.packed_row_bytes);
    q.scales.assign(scales, scales + (size_t)rows * q.scale_cols);
    dequantize_mxfp6(q, out);
}

size_t mxfp6_tiled_scale_bytes(int rows, int cols) {
    if (rows <= 0 || cols <= 0 || cols % K_TILE) return 0;
    return tiled_scale_bytes(rows, cols);
}

void mxfp6_tile_scales(const uint8_t* scales, int rows, int cols, uint8_t* tiled) {
    if (!scales || !tiled || rows <= 0 || cols <= 0 || cols % K_TILE) return;
    PreprocessedScale ps = preprocess_scale(scales, rows, cols);
    std::copy(ps.data.begin(), ps.data.end(), tiled);
}

void mxfp6_untile_scales(const uint8_t* tiled, int rows, int cols, uint8_t* scales) {
    if (!scales || !tiled || rows <= 0 || cols <= 0 || cols % K_TILE) return;
    const int sc = cols / 32;
    for (int r = 0; r < rows; r++)
        for (int j = 0; j < sc; j++) scales[(size_t)r * sc + j] = tiled[tiled_scale_offset(r, j, cols)];
}

}  // extern "C"
