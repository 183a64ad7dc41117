// Test-only layout probe (built into tests/probe/libmxfp6probe.so, never into libmxfp6gemm.so):
// one tensor-memory-accelerator load of a packed FP6 box through the 16U6 unpack mode, dumped
// back to global memory. It pins, on the device, the two layout facts the GEMM kernels rely on:
// how 16 packed codes (12 bytes) land in a 16-byte shared-memory slot, and that the load reports
// 96 bytes per 128-code row to its mbarrier (the transaction count the kernels arm). The probe
// arms exactly that count; no other count can be requested.
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "sm100_ptx.cuh"

namespace {

using namespace mxfp6;

constexpr int kOk = 0;
constexpr int kBadArgs = 1;
constexpr int kCuda = 6;

__global__ void __launch_bounds__(32, 1)
    probe_tma_fp6_kernel(const __grid_constant__ CUtensorMap tm, uint32_t expect_bytes, int box_bytes,
                         uint8_t* out) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    const uint32_t raw = sm100::smem_u32(smem_raw);
    const uint32_t base = (raw + 1023u) & ~1023u;
    uint8_t* buf = smem_raw + (base - raw);
    const uint32_t bar = base + (uint32_t)box_bytes;
    __shared__ int s_ok;
    __shared__ int s_abort;
    // Pre-fill with a marker so untouched bytes are visible in the dump.
    for (int i = threadIdx.x; i < box_bytes; i += 32) buf[i] = 0xEE;
    __syncwarp();
    if (threadIdx.x == 0) {
        s_abort = 0;
        sm100::mbar_init(bar, 1);
        sm100::fence_mbar_init();
        sm100::fence_async_shared();
        sm100::mbar_arrive_expect_tx(bar, expect_bytes);
        sm100::tma_load_2d(base, &tm, bar, 0, 0);
        s_ok = sm100::wait_parity_bounded(bar, 0, &s_abort, 400000000LL) ? 1 : 0;
    }
    __syncwarp();
    for (int i = threadIdx.x; i < box_bytes; i += 32) out[i] = buf[i];
    if (threadIdx.x == 0) *reinterpret_cast<int*>(out + box_bytes) = s_ok;
}

}  // namespace

// dsrc: packed FP6 rows [rows][row_bytes] on the device (row_bytes % 32 == 0, >= 96); Kp % 128 == 0;
// rows in 1..256. dout receives rows*128 bytes of the shared-memory box and an int completion
// flag. The mbarrier expects rows*96 bytes. Returns 0, or 1 for bad arguments, 6 for a CUDA error.
extern "C" int mxfp6_probe_tma_fp6(const void* dsrc, int rows, int Kp, int row_bytes, int swizzle128, void* dout) {
    if (!dsrc || !dout || rows <= 0 || rows > 256 || Kp < 128 || Kp % 128 || row_bytes % 32 || row_bytes < 96)
        return kBadArgs;
    void* fnp = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fnp, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess || !fnp)
        return kCuda;
    using Fn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                            const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                            CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
    CUtensorMap tm;
    cuuint64_t dims[2] = {(cuuint64_t)Kp, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)row_bytes};
    cuuint32_t box[2] = {128u, (cuuint32_t)rows};
    cuuint32_t estr[2] = {1u, 1u};
    CUresult r = reinterpret_cast<Fn>(fnp)(&tm, CU_TENSOR_MAP_DATA_TYPE_16U6_ALIGN16B, 2, const_cast<void*>(dsrc),
                                           dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                                           swizzle128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                                           CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return kCuda;
    const int box_bytes = rows * 128;
    const int smem = 1024 + box_bytes + 64;
    if (cudaFuncSetAttribute(probe_tma_fp6_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
        return kCuda;
    probe_tma_fp6_kernel<<<1, 32, smem>>>(tm, (uint32_t)rows * 96u, box_bytes, static_cast<uint8_t*>(dout));
    if (cudaGetLastError() != cudaSuccess) return kCuda;
    return kOk;
}
