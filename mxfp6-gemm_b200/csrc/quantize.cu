// Device-side MXFP6 quantiser: the reference's host quantize_to_mxfp6
// (include/mxfp6/preprocess.hpp:51-97 of eeezio/mxfp6-gemm) run on the GPU, bit for bit:
//   per row, per 32-element block: scale = smallest power of two >= max|x| / 7.5 (E8M0 code,
//   127 for an all-zero block, NaN inputs ignored by the max), codes = nearest E2M3 of x/scale
//   (ties to even, saturating at 7.5; NaN -> 0x18, as the reference's conversion gives on x86-64),
//   packed four codes per three bytes, least significant bits first.
// It is the step before the GEMM for activations (the FFN's A operand), so it writes the scales
// either raw [rows][cols/32] or directly in the GEMM's 128x4 atom layout.
//
// Traffic: each element reads 4 bytes and writes 0.75 + 1/32. A warp quantises a 512-element
// chunk: 16 consecutive values per lane (four float4 loads), a 32-value block per lane pair, and
// each lane writes its own 12 packed bytes as three aligned words (quantize_kernel).
#include <cuda_runtime.h>

#include <atomic>
#include <cstdint>
#include <cstdio>

#include "mxfp6_gemm.h"
#include "sm100_ptx.cuh"

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

// E8M0 code of the reference's block scale for block max m >= 0: the smallest power of two
// >= RN(m / 7.5), 127 for m == 0. For P = 2^e >= 2^-125, RN(m / 7.5) <= P exactly when
// m <= 7.5 * P (the rounding boundary P + ulp(P)/2 lies below the next float above 7.5 * P), so
// with m = 1.f * 2^E the code is E - 2, plus 1 when the mantissa exceeds 1.875, plus the bias.
// Subnormal quotients, an infinite max and m == 0 take the division.
__device__ __forceinline__ uint32_t scale_code(float m) {
    const uint32_t mb = __float_as_uint(m);
    const int e = (int)(mb >> 23) - 129 + ((mb & 0x7FFFFFu) > 0x700000u ? 1 : 0);
    if (mb < 0x7F800000u && (mb >> 23) != 0u && e >= -125) return (uint32_t)(e + 127);
    return m == 0.0f ? 127u : ceil_pow2_code(__fdiv_rn(m, 7.5f));
}

// Nearest E2M3 codes of two values (round to nearest even, saturating at 7.5) with the
// hardware conversion cvt.rn.satfinite.e2m3x2.f32, which writes a's code to the upper byte and
// b's to the lower one. Two inputs are first replaced so that the codes equal the reference's
// conversion (include/mxfp6/types.hpp:26-72): NaN -> 4.0 (code 0x18, what the reference yields on
// x86-64) and -0.0 -> +0.0 (code 0; other negatives that round to zero keep the sign, 0x20).
// Returns code(b) | code(a) << 8.
__device__ __forceinline__ uint32_t to_e2m3x2(float a, float b) {
    a = a != a ? 4.0f : a + 0.0f;
    b = b != b ? 4.0f : b + 0.0f;
    uint16_t d;
    asm("cvt.rn.satfinite.e2m3x2.f32 %0, %1, %2;" : "=h"(d) : "f"(a), "f"(b));
    return d;
}

// 1 / 2^(code - 127) = 2^(127 - code), exact for every code the quantiser produces (0..254):
// multiplying by it rounds exactly like dividing by the scale.
__device__ __forceinline__ float e8m0_reciprocal(uint32_t code) {
    const int e = 254 - (int)code;  // biased exponent of 2^(127 - code)
    return e > 0 ? __int_as_float(e << 23) : __int_as_float(0x00400000 >> (-e));
}

// One warp quantises a 512-element chunk of a row: lane l owns the 16 consecutive values
// [16 l, 16 l + 16), so each 32-value block spans the lane pair (2b, 2b + 1) (one shuffle for its
// max) and each lane packs its own 16 codes into 12 bytes = 3 words (bytes [12 l, 12 l + 12) of
// the chunk's 384): no packing shuffles, and a warp's stores cover 384 contiguous bytes.
// Grid: x covers the chunks of a row (8 warps per block), y the rows.
__global__ void __launch_bounds__(256) quantize_kernel(const float* __restrict__ in, int rows, int cols,
                                                       uint8_t* __restrict__ packed, int out_row_bytes,
                                                       uint8_t* __restrict__ scales, int scale_cols, int tiled) {
    const int lane = threadIdx.x & 31;
    const int chunk = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int row = blockIdx.y;
    if (chunk * 512 >= cols || row >= rows) return;
    const int col = chunk * 512 + 16 * lane;  // first of this lane's 16 values
    const bool live = col < cols;             // cols % 32 == 0: a lane's 16 values are all in or all out
    float v[16];
    if (live) {
        const float4* src = reinterpret_cast<const float4*>(in + (size_t)row * cols + col);
#pragma unroll
        for (int i = 0; i < 4; i++) {
            const float4 q = __ldg(src + i);
            v[4 * i] = q.x;
            v[4 * i + 1] = q.y;
            v[4 * i + 2] = q.z;
            v[4 * i + 3] = q.w;
        }
    } else {
#pragma unroll
        for (int i = 0; i < 16; i++) v[i] = 0.0f;
    }
    float m = 0.0f;  // fmaxf returns the other operand for a NaN: NaN never wins the max
#pragma unroll
    for (int i = 0; i < 16; i++) m = fmaxf(m, fabsf(v[i]));
    m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 1));
    const uint32_t code = scale_code(m);
    const float inv = e8m0_reciprocal(code);
    uint32_t q[8];  // q[i] = code(v[2i]) | code(v[2i + 1]) << 8
#pragma unroll
    for (int i = 0; i < 8; i++) q[i] = to_e2m3x2(v[2 * i + 1] * inv, v[2 * i] * inv);
    // codes c0..c15 (6 bits each) -> bits 6k of three words
    uint32_t c[16];
#pragma unroll
    for (int i = 0; i < 8; i++) {
        c[2 * i] = q[i] & 0x3Fu;
        c[2 * i + 1] = (q[i] >> 8) & 0x3Fu;
    }
    const uint32_t w0 = c[0] | (c[1] << 6) | (c[2] << 12) | (c[3] << 18) | (c[4] << 24) | (c[5] << 30);
    const uint32_t w1 = (c[5] >> 2) | (c[6] << 4) | (c[7] << 10) | (c[8] << 16) | (c[9] << 22) | (c[10] << 28);
    const uint32_t w2 = (c[10] >> 4) | (c[11] << 2) | (c[12] << 8) | (c[13] << 14) | (c[14] << 20) | (c[15] << 26);
    if (live) {
        uint32_t* dst = reinterpret_cast<uint32_t*>(packed + (size_t)row * out_row_bytes + (size_t)col / 4 * 3);
        dst[0] = w0;
        dst[1] = w1;
        dst[2] = w2;
        if ((lane & 1) == 0) {
            const int j = col / 32;  // block index in the row
            size_t off;
            if (tiled) {
                const size_t atom = (size_t)(row / 128) * (size_t)(scale_cols / 4) + (size_t)(j / 4);
                off = atom * 512 + (size_t)((row % 32) * 16 + ((row % 128) / 32) * 4 + (j % 4));
            } else {
                off = (size_t)row * scale_cols + j;
            }
            scales[off] = (uint8_t)code;
        }
    }
}

// Padded rows: zero bytes [row_bytes, out_row_bytes) of each row, and give the scale blocks past
// the data the finite code 127 (a zero K-tail then contributes 0, never NaN).
__global__ void pad_tail_kernel(int rows, int row_bytes, uint8_t* __restrict__ packed, int out_row_bytes,
                                uint8_t* __restrict__ scales, int data_blocks, int scale_cols, int tiled) {
    const int row = blockIdx.x;
    if (row >= rows) return;
    uint8_t* dst = packed + (size_t)row * out_row_bytes;
    for (int i = row_bytes + threadIdx.x; i < out_row_bytes; i += blockDim.x) dst[i] = 0;
    for (int j = data_blocks + threadIdx.x; j < scale_cols; j += blockDim.x) {
        size_t off;
        if (tiled) {
            const size_t atom = (size_t)(row / 128) * (size_t)(scale_cols / 4) + (size_t)(j / 4);
            off = atom * 512 + (size_t)((row % 32) * 16 + ((row % 128) / 32) * 4 + (j % 4));
        } else {
            off = (size_t)row * scale_cols + j;
        }
        scales[off] = 127;
    }
}

// Copy rows between strides, zero-filling each destination row past bytes_used (re-padding
// compact operand rows for the tensor-memory accelerator). One block per row, in units of U
// bytes: the largest of 16, 8, 4, 1 that divides both bases, both strides and bytes_used, so
// that a compact stride of 3K/4 (a multiple of 8) still moves 8-byte words. HBM bound.
template <typename U>
__global__ void __launch_bounds__(256) repad_kernel(const uint8_t* __restrict__ src, int rows, int src_row_bytes,
                                                    int bytes_used, uint8_t* __restrict__ dst, int dst_row_bytes) {
    sm100::griddep_launch_dependents();
    sm100::griddep_wait();  // launched with programmatic stream serialization (launch_repad)
    const int row = blockIdx.x;
    if (row >= rows) return;
    const U* s = reinterpret_cast<const U*>(src + (size_t)row * src_row_bytes);
    U* d = reinterpret_cast<U*>(dst + (size_t)row * dst_row_bytes);
    const int used = bytes_used / (int)sizeof(U), total = dst_row_bytes / (int)sizeof(U);
    const int bd = blockDim.x;
    // four loads in flight per thread before their stores
    for (int base = threadIdx.x; base < used; base += 4 * bd) {
        U r[4];
#pragma unroll
        for (int k = 0; k < 4; k++)
            if (base + k * bd < used) r[k] = __ldcs(s + base + k * bd);
#pragma unroll
        for (int k = 0; k < 4; k++)
            if (base + k * bd < used) d[base + k * bd] = r[k];
    }
    U zero;
    memset(&zero, 0, sizeof(U));
    for (int i = used + threadIdx.x; i < total; i += bd) d[i] = zero;
}

}  // namespace

// Launch the re-pad copy with the widest unit the pointers and strides allow (used by
// mxfp6_repad_rows_device and by gemm() for compact A with a large enough workspace).
cudaError_t launch_repad(const uint8_t* src, int rows, int src_row_bytes, int bytes_used, uint8_t* dst,
                         int dst_row_bytes, cudaStream_t stream) {
    const uintptr_t a = reinterpret_cast<uintptr_t>(src) | reinterpret_cast<uintptr_t>(dst) |
                        (uintptr_t)src_row_bytes | (uintptr_t)dst_row_bytes | (uintptr_t)bytes_used;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(rows, 1, 1);
    cfg.blockDim = dim3(256, 1, 1);
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if ((a & 15) == 0)
        return cudaLaunchKernelEx(&cfg, repad_kernel<uint4>, src, rows, src_row_bytes, bytes_used, dst, dst_row_bytes);
    if ((a & 7) == 0)
        return cudaLaunchKernelEx(&cfg, repad_kernel<uint2>, src, rows, src_row_bytes, bytes_used, dst, dst_row_bytes);
    if ((a & 3) == 0)
        return cudaLaunchKernelEx(&cfg, repad_kernel<uint32_t>, src, rows, src_row_bytes, bytes_used, dst,
                                  dst_row_bytes);
    return cudaLaunchKernelEx(&cfg, repad_kernel<uint8_t>, src, rows, src_row_bytes, bytes_used, dst, dst_row_bytes);
}

}  // namespace mxfp6

extern "C" int mxfp6_quantize_device_padded(const float* d_mat, int rows, int cols, int padded_cols, uint8_t* d_packed,
                                            uint8_t* d_scales, int scale_layout, void* stream) {
    using namespace mxfp6;
    if (!d_mat || !d_packed || !d_scales || rows <= 0 || cols <= 0 || cols % 32 || padded_cols < cols ||
        padded_cols % 32 || (scale_layout != 0 && scale_layout != 1) || (scale_layout == 1 && padded_cols % 128)) {
        std::fprintf(stderr, "[mxfp6] quantize_device: invalid arguments (%d x %d padded to %d, layout %d)\n", rows,
                     cols, padded_cols, scale_layout);
        return MXFP6_ERR_INVALID_SHAPE;
    }
    const int out_row_bytes = padded_cols / 4 * 3;
    if ((reinterpret_cast<uintptr_t>(d_mat) & 15) || (reinterpret_cast<uintptr_t>(d_packed) & 3) || (cols % 4) ||
        (out_row_bytes % 4)) {
        std::fprintf(stderr, "[mxfp6] quantize_device: input must be 16-byte and output 4-byte aligned\n");
        return MXFP6_ERR_MISALIGNED;
    }
    if (rows > 65535) {
        std::fprintf(stderr, "[mxfp6] quantize_device: at most 65535 rows per call\n");
        return MXFP6_ERR_INVALID_SHAPE;
    }
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const int chunks = (cols + 511) / 512;
    dim3 grid((chunks + 7) / 8, rows);
    quantize_kernel<<<grid, 256, 0, st>>>(d_mat, rows, cols, d_packed, out_row_bytes, d_scales, padded_cols / 32,
                                          scale_layout);
    cudaError_t e = cudaGetLastError();
    if (e == cudaSuccess && padded_cols > cols) {
        pad_tail_kernel<<<rows, 128, 0, st>>>(rows, cols / 4 * 3, d_packed, out_row_bytes, d_scales, cols / 32,
                                             padded_cols / 32, scale_layout);
        e = cudaGetLastError();
        if (e == cudaSuccess) note_launch();
    }
    if (e != cudaSuccess) {
        std::fprintf(stderr, "[mxfp6] quantize_device launch failed: %s\n", cudaGetErrorString(e));
        return MXFP6_ERR_CUDA;
    }
    note_launch();
    return MXFP6_OK;
}

extern "C" int mxfp6_quantize_device(const float* d_mat, int rows, int cols, uint8_t* d_packed, uint8_t* d_scales,
                                     int scale_layout, void* stream) {
    return mxfp6_quantize_device_padded(d_mat, rows, cols, cols, d_packed, d_scales, scale_layout, stream);
}

extern "C" int mxfp6_repad_rows_device(const void* d_src, int rows, int src_row_bytes, int bytes_used, void* d_dst,
                                       int dst_row_bytes, void* stream) {
    using namespace mxfp6;
    if (!d_src || !d_dst || rows <= 0 || bytes_used <= 0 || bytes_used > src_row_bytes ||
        bytes_used > dst_row_bytes) {
        std::fprintf(stderr, "[mxfp6] repad_rows_device: invalid arguments\n");
        return MXFP6_ERR_INVALID_STRIDE;
    }
    const cudaError_t le = launch_repad(static_cast<const uint8_t*>(d_src), rows, src_row_bytes, bytes_used,
                                        static_cast<uint8_t*>(d_dst), dst_row_bytes,
                                        static_cast<cudaStream_t>(stream));
    cudaError_t e = le;
    if (e != cudaSuccess) {
        std::fprintf(stderr, "[mxfp6] repad_rows_device launch failed: %s\n", cudaGetErrorString(e));
        return MXFP6_ERR_CUDA;
    }
    note_launch();
    return MXFP6_OK;
}
