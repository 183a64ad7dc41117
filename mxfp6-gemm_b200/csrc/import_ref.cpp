// Import of device buffers prepared for the reference library (eeezio/mxfp6-gemm, gfx950
// layouts) into this library's layouts, so callers holding preprocessed weights can switch
// without re-quantising. Host-side and one-time, like the reference's own preprocessing.
//
//   reference preshuffle_B (include/mxfp6/preprocess.hpp:182-207): per (32-column, 64-deep) tile,
//     1536 bytes; thread t of 64 covers column n = 32*tile_n + t%32 and K half t/32: its 24 packed
//     bytes are split 16 at t*16 and 8 at 1024 + t*8.
//   reference preprocess_scale + tile_scale (include/mxfp6/preprocess.hpp:136-162, 216-233): per
//     32-row tile and 64-deep step, 64 lane-ordered bytes (lane l: row l%16 + 16*((l/16)%2), block
//     2*k64 + l/32), regrouped as [(g*k_tiles + kt)*64 + lane][sub][group_pad].
// Both are inverted exactly here; the result is B^T packed rows and raw [rows][K/32] scales,
// which preprocess_scale / mxfp6_tile_scales turn into this library's scale atoms.
#include <cstdint>
#include <cstdio>
#include <cstring>

#include "mxfp6_gemm.h"

extern "C" {

int mxfp6_import_ref_B(const uint8_t* ref_bsh, int N, int Kp_ref, uint8_t* out, int out_row_bytes) {
    if (!ref_bsh || !out || N <= 0 || N % 32 || Kp_ref <= 0 || Kp_ref % 64 || out_row_bytes < Kp_ref / 4 * 3) {
        std::fprintf(stderr, "[mxfp6] import_ref_B: invalid arguments (N=%d Kp_ref=%d row_bytes=%d)\n", N, Kp_ref,
                     out_row_bytes);
        return MXFP6_ERR_INVALID_SHAPE;
    }
    const int k64 = Kp_ref / 64;
    for (int n = 0; n < N; n++)
        std::memset(out + (size_t)n * out_row_bytes + Kp_ref / 4 * 3, 0, out_row_bytes - Kp_ref / 4 * 3);
    for (int nt = 0; nt < N / 32; nt++)
        for (int ki = 0; ki < k64; ki++) {
            const uint8_t* tile = ref_bsh + ((size_t)nt * k64 + ki) * 1536;
            for (int t = 0; t < 64; t++) {
                uint8_t* dst = out + (size_t)(nt * 32 + t % 32) * out_row_bytes + ki * 48 + (t / 32) * 24;
                std::memcpy(dst, tile + t * 16, 16);
                std::memcpy(dst + 16, tile + 1024 + t * 8, 8);
            }
        }
    return MXFP6_OK;
}

int mxfp6_import_ref_scales(const uint8_t* ref_tiled, int dim, int Kp_ref, int group, int subs, uint8_t* raw_out) {
    if (!ref_tiled || !raw_out || dim <= 0 || dim % 32 || Kp_ref <= 0 || Kp_ref % 64 || group <= 0 || subs <= 0 ||
        (dim / 32) % group || (Kp_ref / 64) % subs) {
        std::fprintf(stderr, "[mxfp6] import_ref_scales: invalid arguments (dim=%d Kp_ref=%d group=%d subs=%d)\n",
                     dim, Kp_ref, group, subs);
        return MXFP6_ERR_INVALID_SHAPE;
    }
    const int group_pad = (group + 3) / 4 * 4, k_tiles = Kp_ref / 64 / subs, ng = dim / 32 / group;
    const int sc = Kp_ref / 32;
    for (int g = 0; g < ng; g++)
        for (int kt = 0; kt < k_tiles; kt++)
            for (int lane = 0; lane < 64; lane++)
                for (int sub = 0; sub < subs; sub++)
                    for (int j = 0; j < group; j++) {
                        const uint8_t v =
                            ref_tiled[(((size_t)(g * k_tiles + kt) * 64 + lane) * subs + sub) * group_pad + j];
                        const int tile = g * group + j, k64 = kt * subs + sub;
                        const int row = tile * 32 + lane % 16 + 16 * ((lane / 16) % 2);
                        const int block = 2 * k64 + lane / 32;
                        raw_out[(size_t)row * sc + block] = v;
                    }
    return MXFP6_OK;
}

int mxfp6_repad_rows(const uint8_t* src, int rows, int src_row_bytes, int src_bytes_used, uint8_t* dst,
                     int dst_row_bytes) {
    if (!src || !dst || rows <= 0 || src_bytes_used <= 0 || src_bytes_used > src_row_bytes ||
        src_bytes_used > dst_row_bytes) {
        std::fprintf(stderr, "[mxfp6] repad_rows: invalid arguments\n");
        return MXFP6_ERR_INVALID_STRIDE;
    }
    for (int r = 0; r < rows; r++) {
        std::memcpy(dst + (size_t)r * dst_row_bytes, src + (size_t)r * src_row_bytes, src_bytes_used);
        std::memset(dst + (size_t)r * dst_row_bytes + src_bytes_used, 0, dst_row_bytes - src_bytes_used);
    }
    return MXFP6_OK;
}

}  // extern "C"
