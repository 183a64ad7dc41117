// Device-side MXFP6 quantiser: the reference's host quantize_to_mxfp6
// (include/mxfp6/preprocess.hpp:51-97 of eeezio/mxfp6-gemm) run on the GPU, bit for bit:
//   per row, per 32-element block: scale = smallest power of two >= max|x| / 7.5 (E8M0 code,
//   127 for an all-zero block, NaN inputs ignored by the max), codes = nearest E2M3 of x/scale
//   (ties to even, saturating at 7.5; NaN -> 0x18, as the reference's conversion gives on x86-64),
//   packed four codes per three bytes, least significant bits first.
// It is the step before the GEMM for activations (the FFN's A operand), so it writes the scales
// either raw [rows][cols/32] or directly in the GEMM's 128x4 atom layout.
//
// HBM bound: each element reads 4 bytes and writes 0.75 + 1/32. One warp quantises four blocks
// (128 elements, one float4 per lane) and writes its 96 packed bytes as 24 aligned words.
#include <cuda_runtime.h>

#include <atomic>
#include <cstdint>
#include <cstdio>

#include "mxfp6_gemm.h"

namespace mxfp6 {
void note_launch();  // launch counter (gemm.cu)

namespace {

// E8M0 code of the smallest power of two >= v (v > 0, finite or +Inf): from the float bits,
// the same result as frexp-based rounding up (a power of two maps to itself).
__device__ __forceinline__ uint32_t ceil_pow2_code(float v) {
    const uint32_t b = __float_as_uint(v);
    if (b >= 0x7F800000u) return 127;  // +Inf: the reference's frexp reports exponent 0
    int e;                              // v = m * 2^e with m in [1, 2)
    uint32_t man;
    if (b >= 0x00800000u) {
        e = (int)(b >> 23) - 127;
        man = b & 0x7FFFFFu;
    } else {  // subnormal: normalise the mantissa
        const int lz = __clz(b) - 8;    // leading zeros within the 24-bit significand field
        e = -126 - lz;
        man = (b << lz) & 0x7FFFFFu;
    }
    const int code = e + (man != 0 ? 1 : 0) + 127;
    return (uint32_t)(code < 0 ? 0 : (code > 254 ? 254 : code));
}

// Nearest integer of q >= 0 (exactly representable), ties to even.
__device__ __forceinline__ int rne(float q) {
    const float f = floorf(q);
    const float d = q - f;
    const int b = (int)f;
    return d > 0.5f ? b + 1 : (d < 0.5f ? b : b + (b & 1));
}

__device__ __forceinline__ uint32_t to_e2m3(float v) {
    uint32_t s = 0;
    if (v < 0.0f) {
        s = 0x20;
        v = -v;
    }
    if (v == 0.0f) return s;
    if (v != v) return 0x18;
    if (v > 7.5f) v = 7.5f;
    if (v < 1.0f) {
        const int m = rne(v * 8.0f);
        return m <= 0 ? s : (m >= 8 ? (s | 0x08) : (s | (uint32_t)m));
    }
    int e = v < 2.0f ? 1 : (v < 4.0f ? 2 : 3);
    const float frac = v / (float)(1 << (e - 1)) - 1.0f;
    int m = rne(frac * 8.0f);
    if (m >= 8) {
        m = 0;
        if (++e > 3) return s | 0x1F;
    }
    return s | ((uint32_t)e << 3) | (uint32_t)m;
}

// 2^(code - 127) from the bits (code 0 is the subnormal 2^-127; code 255 never occurs here).
__device__ __forceinline__ float e8m0_value(uint32_t code) {
    return code == 0 ? __int_as_float(0x00400000) : __int_as_float((int)(code << 23));
}

// grid: x = 128-element chunks of a row, y = rows (blockDim 32, one warp per chunk)
__global__ void __launch_bounds__(256) quantize_kernel(const float* __restrict__ in, int rows, int cols,
                                                       uint8_t* __restrict__ packed, uint8_t* __restrict__ scales,
                                                       int tiled) {
    const int lane = threadIdx.x & 31;
    const int chunk = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);  // 128 columns each
    const int row = blockIdx.y;
    if (chunk * 128 >= cols || row >= rows) return;
    const int col = chunk * 128 + 4 * lane;
    const bool live = col < cols;  // cols % 32 == 0, so whole 8-lane blocks are live or not
    float4 x = make_float4(0.f, 0.f, 0.f, 0.f);
    if (live) x = *reinterpret_cast<const float4*>(in + (size_t)row * cols + col);
    // block max over 8 lanes; NaN never wins a > comparison
    float m = 0.0f;
    for (float a : {fabsf(x.x), fabsf(x.y), fabsf(x.z), fabsf(x.w)})
        if (a > m) m = a;
#pragma unroll
    for (int off = 1; off < 8; off <<= 1) {
        const float o = __shfl_xor_sync(0xffffffffu, m, off);
        if (o > m) m = o;
    }
    const uint32_t code = m == 0.0f ? 127u : ceil_pow2_code(__fdiv_rn(m, 7.5f));
    const float sv = e8m0_value(code);
    const uint32_t q0 = to_e2m3(__fdiv_rn(x.x, sv)), q1 = to_e2m3(__fdiv_rn(x.y, sv)),
                   q2 = to_e2m3(__fdiv_rn(x.z, sv)), q3 = to_e2m3(__fdiv_rn(x.w, sv));
    const uint32_t g = q0 | (q1 << 6) | (q2 << 12) | (q3 << 18);  // this lane's 3 bytes
    // Bytes [3*lane, 3*lane + 3) of the warp's 96; lane w < 24 writes word w = bytes [4w, 4w + 4).
    const int lo = (4 * lane) / 3, hi = (4 * lane + 3) / 3;
    const uint32_t glo = __shfl_sync(0xffffffffu, g, lo & 31);
    const uint32_t ghi = __shfl_sync(0xffffffffu, g, hi & 31);
    const int sh = 4 * lane - 3 * lo;  // byte offset of word w inside lane lo's 3 bytes (0..2)
    const uint32_t word = (glo >> (8 * sh)) | (ghi << (8 * (3 - sh)));
    const int row_bytes = cols / 4 * 3;
    const int valid = min(96, row_bytes - chunk * 96);  // a multiple of 24 (cols % 32 == 0)
    if (lane < 24 && 4 * lane < valid)
        *reinterpret_cast<uint32_t*>(packed + (size_t)row * row_bytes + chunk * 96 + 4 * lane) = word;
    if (live && (lane & 7) == 0) {
        const int j = col / 32;  // block index in the row
        size_t off;
        if (tiled) {
            const size_t atom = (size_t)(row / 128) * (size_t)(cols / 128) + (size_t)(j / 4);
            off = atom * 512 + (size_t)((row % 32) * 16 + ((row % 128) / 32) * 4 + (j % 4));
        } else {
            off = (size_t)row * (cols / 32) + j;
        }
        scales[off] = (uint8_t)code;
    }
}

}  // namespace
}  // namespace mxfp6

extern "C" int mxfp6_quantize_device(const float* d_mat, int rows, int cols, uint8_t* d_packed, uint8_t* d_scales,
                                     int scale_layout, void* stream) {
    using namespace mxfp6;
    if (!d_mat || !d_packed || !d_scales || rows <= 0 || cols <= 0 || cols % 32 ||
        (scale_layout != 0 && scale_layout != 1) || (scale_layout == 1 && cols % 128)) {
        std::fprintf(stderr, "[mxfp6] quantize_device: invalid arguments (%d x %d, layout %d)\n", rows, cols,
                     scale_layout);
        return MXFP6_ERR_INVALID_SHAPE;
    }
    if ((reinterpret_cast<uintptr_t>(d_mat) & 15) || (reinterpret_cast<uintptr_t>(d_packed) & 3)) {
        std::fprintf(stderr, "[mxfp6] quantize_device: input must be 16-byte and output 4-byte aligned\n");
        return MXFP6_ERR_MISALIGNED;
    }
    if (rows > 65535) {
        std::fprintf(stderr, "[mxfp6] quantize_device: at most 65535 rows per call\n");
        return MXFP6_ERR_INVALID_SHAPE;
    }
    const int chunks = (cols + 127) / 128;
    dim3 grid((chunks + 7) / 8, rows);
    quantize_kernel<<<grid, 256, 0, static_cast<cudaStream_t>(stream)>>>(d_mat, rows, cols, d_packed, d_scales,
                                                                        scale_layout);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) {
        std::fprintf(stderr, "[mxfp6] quantize_device launch failed: %s\n", cudaGetErrorString(e));
        return MXFP6_ERR_CUDA;
    }
    note_launch();
    return MXFP6_OK;
}
