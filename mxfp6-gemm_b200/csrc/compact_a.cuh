#pragma once
// Producers for an A operand the 16U6 tensor load cannot address.
//
// The reference's "pad-B-only / compact-A" recipe (include/mxfp6/preprocess.hpp:12-38,
// tests/test_gemm.cpp:131-201) keeps activations in their natural layout: row stride
// S = A_row_bytes = 3K/4 with K % 128 != 0 (only K % 32 == 0 is required), while B and the scales
// are padded to Kp = kpad(K). The 16U6 unpack mode needs a row stride that is a multiple of 32
// bytes, so such an A is brought into the A stages another way, into exactly the shared-memory
// image the 16U6 load produces:
//
//   row r of the 128-row slab occupies bytes [128 r, 128 r + 128); its 128 codes form 8 groups of
//   16, group g = 12 packed bytes stored in the 16-byte slot (g XOR (r % 8)) (128-byte swizzle),
//   followed by 4 zero bytes.
//
// Bytes of a row at or past its valid length (K's packed length, or the stride if shorter) become
// zero codes: the K tail contributes 0 against B's zero tail, as in the reference, which reads the
// next row's codes there instead; no end pad (a_compact_end_pad) is ever read.
//
// Four loader warps copy the image directly with 4-byte cp.async: one warp instruction per row,
// lane l writing word l % 4 of slot (l / 4) XOR (r % 8) (all 32 banks; word 3 is the zero gap,
// a zero-fill copy) from the row's 96 contiguous packed bytes. Each thread signals a slab with
// cp.async.mbarrier.arrive.noinc right after issuing it and moves on to the next stage; the
// stage's full barrier completes when every copy has landed. Rows at or past M are skipped
// (their outputs are not stored).
//
// Measured on B200 (8192 x 8192 x 8160, FP16 out): 1.51 PFLOP/s, 0.57 of the same GEMM on a
// padded A through the tensor load (2.65 PFLOP/s). Alternatives that were built and measured
// slower: loader threads waiting for their own copies before a proxy fence and a barrier arrive
// (0.30); raw rows staged in shared memory by tensor loads from a row-pair tensor map and expanded
// there (0.33-0.39: two extra shared-memory passes, and every slab then waits on a store, a
// proxy fence and eight warp arrivals before the MMAs may read it); 8-byte global loads into a
// register ring written with 16-byte shared stores (0.34, same fence and arrival chain); eight
// loader warps instead of four (no change). An A that can be produced padded (quantize_device_padded,
// or a one-time repad_rows_device) runs at the full tensor-load speed.
#include <cstdint>

#include "sm100_ptx.cuh"

namespace mxfp6 {
namespace kern {

enum AMode : int { A_TMA = 0, A_CPASYNC = 1 };

constexpr int LOADER_WARPS = 4;
constexpr int LOADER_THREADS = 32 * LOADER_WARPS;
constexpr int LOADER_WARP0 = 6;  // after the producer, MMA and four epilogue warps

// Threads per CTA for an A mode (6 warps of the tensor-load kernel, plus the loader warps).
__host__ __device__ constexpr int threads_for(int amode) {
    return 192 + (amode == A_TMA ? 0 : LOADER_THREADS);
}

struct CompactA {
    const uint8_t* ptr;  // row-major packed FP6, row stride `stride` bytes
    int stride;          // bytes between rows (multiple of 4)
    int valid;           // bytes of real data per row (<= stride, multiple of 4)
};

// Issue this thread's copies of slab `kb` (K codes [128 kb, 128 kb + 128)) of rows
// [row0, row0 + 128) into the slab image at `dst`.
__device__ __forceinline__ void compact_issue_slab(uint32_t dst, const CompactA& a, int M, int row0, int kb, int lt) {
    const int lane = lt & 31, w = lt >> 5;
    const int g = lane >> 2, j = lane & 3;
    const int koff = kb * 96 + 12 * g + 4 * j;
    const bool in = j < 3 && koff + 4 <= a.valid;
    const uint32_t nbytes = in ? 4u : 0u;
    const uint8_t* src = a.ptr + (size_t)(row0 + w) * a.stride + koff;
    const size_t step = (size_t)4 * a.stride;
    const int rows = M - row0 < 128 ? M - row0 : 128;
#pragma unroll 8
    for (int r = w; r < rows; r += LOADER_WARPS) {
        const uint32_t d = dst + (uint32_t)r * 128u + ((uint32_t)(g ^ (r & 7)) << 4) + 4u * j;
        sm100::cp_async_4(d, in ? (const void*)src : (const void*)a.ptr, nbytes);
        src += step;
    }
}

}  // namespace kern
}  // namespace mxfp6
