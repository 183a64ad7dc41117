// Device import of buffers prepared for the reference library (eeezio/mxfp6-gemm, gfx950
// layouts): the same permutations as the host import (import_ref.cpp), run as two gather kernels
// that write this library's layouts directly, so a caller holding preprocessed weights on the
// device converts them in one HBM pass instead of a host round trip.
//
//   import_b_kernel: the reference's preshuffle_B (include/mxfp6/preprocess.hpp:182-207) stores,
//     per (32-column, 64-deep) tile, 1536 bytes: for t in 0..63 (column 32*tile_n + t%32, K half
//     t/32), the 24 packed bytes of that column's 32 K values, split 16 at t*16 and 8 at
//     1024 + t*8. A block stages KI_PER_CTA consecutive tiles of one column tile (contiguous in
//     the reference buffer, read as 16-byte words) in shared memory and writes the 32 B^T rows
//     they cover as 16-byte words (8-byte for an output stride that is not a multiple of 16),
//     consecutive threads on consecutive words of a row.
//   import_scales_kernel: the reference's tile_scale(preprocess_scale(raw, dim, Kp_ref), group,
//     subs) (include/mxfp6/preprocess.hpp:136-162, 216-233) puts raw scale (row r, block j) at
//     byte ((((r/32/group)*k_tiles + k64/subs)*64 + lane)*subs + k64%subs)*group_pad +
//     (r/32)%group, with k64 = j/2 and lane = r%32 + 32*(j%2). Each thread builds one 32-bit word
//     of this library's 128 x 4 scale atoms (four blocks of one row) from four such bytes.
//
// Both kernels are HBM-bound byte moves; the B import reads 3/4 byte per K element and writes the
// same, plus a zero tail when this library's padded K exceeds the reference's.
#include <cuda_runtime.h>

#include <cstdint>
#include <cstdio>

#include "mxfp6_gemm.h"

namespace mxfp6 {
void note_launch();  // launch counter (gemm.cu)

namespace {

constexpr int REF_TILE_BYTES = 1536;  // one (32-column, 64-deep) tile of the reference's preshuffle_B
constexpr int REF_STEP_BYTES = 48;    // packed bytes of one column's 64 K values
constexpr int KI_PER_CTA = 16;        // tiles staged per block: 24 KB of shared memory
// Staged tiles sit 16 bytes further apart than in global memory: a warp's lanes read the same
// offset of different tiles, and 1536 bytes is a multiple of the 128-byte bank period.
constexpr int STAGE_STRIDE = REF_TILE_BYTES + 16;
constexpr int IMPORT_THREADS = 256;

// Grid: x = groups of KI_PER_CTA 64-deep steps, y = 32-column tiles. used_bytes = bytes of each
// B^T row taken from the reference (min of its 3*Kp_ref/4 and out_row_bytes); ref_row_bytes =
// 3*Kp_ref/4. Bytes [ref_row_bytes, out_row_bytes) of every row are zeroed by the last x block.
// UNIT = 16: 16-byte stores (out_row_bytes % 16 == 0, 16-byte aligned output); UNIT = 8 otherwise.
template <int UNIT>
__global__ void __launch_bounds__(IMPORT_THREADS)
    import_b_kernel(const uint8_t* __restrict__ ref, int k64, int used_bytes, int ref_row_bytes,
                    uint8_t* __restrict__ out, int out_row_bytes) {
    __shared__ __align__(16) uint8_t tiles[KI_PER_CTA * STAGE_STRIDE];
    const int nt = blockIdx.y;
    const int ki0 = blockIdx.x * KI_PER_CTA;
    const int nk = min(KI_PER_CTA, k64 - ki0);

    const uint4* src = reinterpret_cast<const uint4*>(ref + ((size_t)nt * k64 + ki0) * REF_TILE_BYTES);
    const int n16 = nk * (REF_TILE_BYTES / 16);
    for (int i = threadIdx.x; i < n16; i += IMPORT_THREADS) {
        const int kl = i / (REF_TILE_BYTES / 16), wi = i - kl * (REF_TILE_BYTES / 16);
        *reinterpret_cast<uint4*>(tiles + kl * STAGE_STRIDE + 16 * wi) = __ldg(src + i);
    }
    __syncthreads();

    // A column's 48-byte step is two 24-byte halves h (entries t = c and t = c + 32); byte b of
    // half h sits at t*16 + b (b < 16) or 1024 + t*8 + (b - 16) of the step's tile.
    auto src8 = [&](int kl, int c, int b48) -> uint2 {
        const int h = b48 >= 24 ? 1 : 0, b = b48 - 24 * h, t = c + 32 * h;
        return *reinterpret_cast<const uint2*>(tiles + kl * STAGE_STRIDE + (b < 16 ? t * 16 + b : 1024 + t * 8));
    };
    constexpr int PER_STEP = REF_STEP_BYTES / UNIT;
    const int units_per_row = nk * PER_STEP;
    uint8_t* rows = out + (size_t)nt * 32 * out_row_bytes;
    for (int u = threadIdx.x; u < 32 * units_per_row; u += IMPORT_THREADS) {
        const int c = u / units_per_row;
        const int w = u - c * units_per_row;
        const int kl = w / PER_STEP, q = w - kl * PER_STEP;
        const int col = (ki0 + kl) * REF_STEP_BYTES + UNIT * q;
        if (col >= used_bytes) continue;
        uint8_t* dst = rows + (size_t)c * out_row_bytes + col;
        if constexpr (UNIT == 16) {
            const uint2 lo = src8(kl, c, 16 * q), hi = src8(kl, c, 16 * q + 8);
            *reinterpret_cast<uint4*>(dst) = make_uint4(lo.x, lo.y, hi.x, hi.y);
        } else {
            *reinterpret_cast<uint2*>(dst) = src8(kl, c, 8 * q);
        }
    }
    if (blockIdx.x == gridDim.x - 1 && out_row_bytes > ref_row_bytes) {
        const int tail_words = (out_row_bytes - ref_row_bytes) / 8;
        for (int u = threadIdx.x; u < 32 * tail_words; u += IMPORT_THREADS) {
            const int c = u / tail_words, w = u - c * tail_words;
            *reinterpret_cast<uint2*>(rows + (size_t)c * out_row_bytes + ref_row_bytes + 8 * w) = make_uint2(0u, 0u);
        }
    }
}

// One thread per 32-bit word of the atom layout for (dim, Kp): word wi of atom a holds row
// (a / slabs)*128 + (wi%4)*32 + wi/4, blocks 4*(a % slabs) .. +3. Rows >= dim and blocks >=
// blocks_ref (this library's K padding past the reference's) get the finite code 127.
__global__ void __launch_bounds__(IMPORT_THREADS)
    import_scales_kernel(const uint8_t* __restrict__ ref, int dim, int blocks_ref, int group, int subs,
                         int group_pad, int k_tiles, uint32_t* __restrict__ out, int slabs, long long words) {
    for (long long w = (long long)blockIdx.x * IMPORT_THREADS + threadIdx.x; w < words;
         w += (long long)gridDim.x * IMPORT_THREADS) {
        const long long atom = w >> 7;
        const int wi = (int)(w & 127);
        const int r = (int)(atom / slabs) * 128 + (wi & 3) * 32 + (wi >> 2);
        const int j0 = (int)(atom % slabs) * 4;
        uint32_t v = 0;
#pragma unroll
        for (int b = 0; b < 4; b++) {
            const int j = j0 + b;
            uint32_t code = 127u;
            if (r < dim && j < blocks_ref) {
                const int tile = r >> 5;
                const int k64 = j >> 1;
                const int lane = (r & 31) + 32 * (j & 1);
                const size_t idx =
                    ((((size_t)(tile / group) * k_tiles + k64 / subs) * 64 + lane) * subs + k64 % subs) * group_pad +
                    tile % group;
                code = __ldg(ref + idx);
            }
            v |= code << (8 * b);
        }
        out[w] = v;
    }
}

int sm_count_here() {
    int dev = 0, n = 148;
    if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    return n > 0 ? n : 148;
}

}  // namespace
}  // namespace mxfp6

extern "C" int mxfp6_import_ref_B_device(const void* d_ref_bsh, int N, int Kp_ref, void* d_out, int out_row_bytes,
                                         void* stream) {
    using namespace mxfp6;
    if (!d_ref_bsh || !d_out || N <= 0 || N % 32 || N / 32 > 65535 || Kp_ref <= 0 || Kp_ref % 64 ||
        out_row_bytes <= 0 || out_row_bytes % 8) {
        std::fprintf(stderr, "[mxfp6] import_ref_B_device: invalid arguments (N=%d Kp_ref=%d row_bytes=%d)\n", N,
                     Kp_ref, out_row_bytes);
        return MXFP6_ERR_INVALID_SHAPE;
    }
    if ((reinterpret_cast<uintptr_t>(d_ref_bsh) & 15) || (reinterpret_cast<uintptr_t>(d_out) & 7)) {
        std::fprintf(stderr, "[mxfp6] import_ref_B_device: reference buffer must be 16-byte, output 8-byte aligned\n");
        return MXFP6_ERR_MISALIGNED;
    }
    const int k64 = Kp_ref / 64;
    const int ref_row_bytes = Kp_ref / 4 * 3;
    const int used = ref_row_bytes < out_row_bytes ? ref_row_bytes : out_row_bytes;
    dim3 grid((k64 + KI_PER_CTA - 1) / KI_PER_CTA, N / 32);
    const bool wide = out_row_bytes % 16 == 0 && (reinterpret_cast<uintptr_t>(d_out) & 15) == 0;
    if (wide)
        import_b_kernel<16><<<grid, IMPORT_THREADS, 0, static_cast<cudaStream_t>(stream)>>>(
            static_cast<const uint8_t*>(d_ref_bsh), k64, used, ref_row_bytes, static_cast<uint8_t*>(d_out),
            out_row_bytes);
    else
        import_b_kernel<8><<<grid, IMPORT_THREADS, 0, static_cast<cudaStream_t>(stream)>>>(
            static_cast<const uint8_t*>(d_ref_bsh), k64, used, ref_row_bytes, static_cast<uint8_t*>(d_out),
            out_row_bytes);
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) {
        std::fprintf(stderr, "[mxfp6] import_ref_B_device launch failed: %s\n", cudaGetErrorString(e));
        return MXFP6_ERR_CUDA;
    }
    note_launch();
    return MXFP6_OK;
}

extern "C" int mxfp6_import_ref_scales_device(const void* d_ref_tiled, int dim, int Kp_ref, int group, int subs,
                                              void* d_out_tiled, int Kp, void* stream) {
    using namespace mxfp6;
    if (!d_ref_tiled || !d_out_tiled || dim <= 0 || dim % 32 || Kp_ref <= 0 || Kp_ref % 64 || group <= 0 ||
        subs <= 0 || (dim / 32) % group || (Kp_ref / 64) % subs || Kp <= 0 || Kp % 128) {
        std::fprintf(stderr,
                     "[mxfp6] import_ref_scales_device: invalid arguments (dim=%d Kp_ref=%d group=%d subs=%d Kp=%d)\n",
                     dim, Kp_ref, group, subs, Kp);
        return MXFP6_ERR_INVALID_SHAPE;
    }
    if (reinterpret_cast<uintptr_t>(d_out_tiled) & 3) {
        std::fprintf(stderr, "[mxfp6] import_ref_scales_device: output must be 4-byte aligned\n");
        return MXFP6_ERR_MISALIGNED;
    }
    const int slabs = Kp / 128;
    const long long words = (long long)((dim + 127) / 128) * slabs * 128;
    long long blocks = (words + IMPORT_THREADS - 1) / IMPORT_THREADS;
    const long long cap = (long long)sm_count_here() * 8;
    if (blocks > cap) blocks = cap;
    import_scales_kernel<<<(int)blocks, IMPORT_THREADS, 0, static_cast<cudaStream_t>(stream)>>>(
        static_cast<const uint8_t*>(d_ref_tiled), dim, Kp_ref / 32, group, subs, (group + 3) / 4 * 4,
        Kp_ref / 64 / subs, static_cast<uint32_t*>(d_out_tiled), slabs, words);
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) {
        std::fprintf(stderr, "[mxfp6] import_ref_scales_device launch failed: %s\n", cudaGetErrorString(e));
        return MXFP6_ERR_CUDA;
    }
    note_launch();
    return MXFP6_OK;
}
