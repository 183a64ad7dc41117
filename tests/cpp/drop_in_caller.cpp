// A C++ caller written against the public headers only, the way a user of the reference library
// calls it (reference flow: tests/test_gemm.cpp:131-201 and :402-442 of eeezio/mxfp6-gemm):
// float matrices -> quantize_to_mxfp6 / preprocess_B -> preshuffle_B -> preprocess_scale +
// tile_scale -> gemm() with a caller-owned split-K workspace -> D read back and checked against
// a host double-precision product of the dequantised operands.
//
// Built with g++ (no CUDA compiler): the headers are device-free and the program links
// libmxfp6gemm.so plus the CUDA runtime for its own cudaMalloc / cudaMemcpy.
//
//   drop_in_caller host   checks the device-free part: kpad, choose_tile, workspace queries and
//                         argument validation (errors are recorded, nothing is launched)
//   drop_in_caller gpu    runs the GEMM flow on the current device for every output type, a
//                         split-K shape and a compact-A shape (K % 128 != 0)
//   drop_in_caller time   per-call time of the launch-bound BASELINE config 1 (256x256x512, FP32
//                         out) timed the reference's way: 8 warm-ups, then 20 back-to-back gemm()
//                         calls on the legacy default stream between two events, best of 4
//   drop_in_caller time M N K OUT   the same for one shape (OUT F32, F16 or BF16; K zero-padded
//                         to kpad(K) as the reference's harness pads it)
// Exit status 0 on success; each failure prints one line.
#include <cuda_runtime.h>

#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <random>
#include <string>
#include <vector>

#include "mxfp6/gemm.hpp"
#include "mxfp6/preprocess.hpp"
#include "mxfp6_gemm.h"

using namespace mxfp6;

namespace {

int g_failures = 0;

void fail(const std::string& what) {
    std::printf("FAIL %s\n", what.c_str());
    g_failures++;
}

#define CUDA_OK(call)                                                                     \
    do {                                                                                  \
        cudaError_t e_ = (call);                                                          \
        if (e_ != cudaSuccess) {                                                          \
            std::printf("FAIL cuda %s: %s\n", #call, cudaGetErrorString(e_));             \
            std::exit(1);                                                                 \
        }                                                                                 \
    } while (0)

float half_bits_to_float(uint16_t h) {
    const int s = h >> 15, e = (h >> 10) & 31, m = h & 1023;
    float v = e == 0 ? std::ldexp((float)m, -24)
                     : (e == 31 ? (m ? NAN : INFINITY) : std::ldexp((float)(1024 + m), e - 25));
    return s ? -v : v;
}

float bf16_bits_to_float(uint16_t b) {
    uint32_t u = (uint32_t)b << 16;
    float f;
    std::memcpy(&f, &u, 4);
    return f;
}

const char* name_of(OutType ot) {
    return ot == OutType::F32 ? "F32" : (ot == OutType::F16 ? "F16" : "BF16");
}

// ---- device-free checks ----------------------------------------------------------------------

void host_checks() {
    if (kpad(1952) != 2048 || kpad(4096) != 4096 || mxfp6_k_tile() != K_TILE) fail("kpad / K_TILE");

    for (int M : {128, 256, 1024, 8192})
        for (int N : {128, 384, 4096})
            for (int Kp : {128, 1024, 16384}) {
                TileChoice tc = choose_tile(M, N, Kp);
                if (tc.MT <= 0 || tc.NT <= 0 || tc.MPW != tc.MT / 32 || tc.NPW != tc.NT / 32)
                    fail("choose_tile " + std::to_string(M) + "x" + std::to_string(N));
                // The A-aware query never asks for less than the plain one.
                if (gemm_workspace_size(M, N, Kp, Kp * 3 / 4) != gemm_workspace_size(M, N, Kp))
                    fail("workspace query, padded A stride");
            }
    if (gemm_workspace_size(128, 256, 2048, 1952 * 3 / 4) < (size_t)128 * 2048 * 3 / 4)
        fail("A-aware workspace leaves no room for a padded copy of compact A");

    // Validation happens before any device work: bad arguments record an error, launch nothing.
    const uint64_t launches = mxfp6_launch_count();
    alignas(32) static uint8_t dummy[64];
    struct Case {
        int M, N, Kp, a_rb, b_rb;
        const void* A;
        int want;
    } cases[] = {
        {100, 256, 256, 192, 192, dummy, MXFP6_ERR_INVALID_SHAPE},
        {128, 256, 200, 150, 160, dummy, MXFP6_ERR_INVALID_SHAPE},
        {128, 256, 256, 192, 200, dummy, MXFP6_ERR_INVALID_STRIDE},
        {128, 256, 256, 192, 192, nullptr, MXFP6_ERR_NULL_POINTER},
        {128, 256, 256, 192, 192, dummy + 2, MXFP6_ERR_MISALIGNED},
    };
    for (const Case& c : cases) {
        gemm(OutType::F32, c.M, c.N, c.Kp, c.A, dummy, dummy, dummy, dummy, c.a_rb, c.b_rb, nullptr, 0);
        if (mxfp6_last_error() != c.want)
            fail("validation: want error " + std::to_string(c.want) + ", got " +
                 std::to_string(mxfp6_last_error()) + " (" + mxfp6_last_error_string() + ")");
    }
    if (mxfp6_launch_count() != launches) fail("a rejected call launched a kernel");
}

// ---- the reference's GEMM flow on the device -------------------------------------------------

struct Shape {
    int M, N, K;
    bool compact_a;  // keep A at the reference's compact stride 3K/4 (K % 128 != 0)
};

void run_case(const Shape& s, OutType ot, uint32_t seed) {
    const int M = s.M, N = s.N, K = s.K, Kp = kpad(K);
    std::mt19937 rng(seed);
    std::normal_distribution<float> nd(0.0f, 1.0f);
    // A is quantised at K (compact) or at Kp with a zero K-tail; B always at Kp with a zero tail.
    const int Ka = s.compact_a ? K : Kp;
    std::vector<float> A((size_t)M * Ka, 0.0f), B((size_t)Kp * N, 0.0f);
    for (int m = 0; m < M; m++)
        for (int k = 0; k < K; k++) A[(size_t)m * Ka + k] = nd(rng) * (1.0f + (m % 5));
    for (int k = 0; k < K; k++)
        for (int n = 0; n < N; n++) B[(size_t)k * N + n] = 0.05f * nd(rng);

    QuantizedMatrix Aq = quantize_to_mxfp6(A.data(), M, Ka);
    QuantizedMatrix Bq = preprocess_B(B.data(), Kp, N);
    PreshuffledB Bsh = preshuffle_B(Bq);
    TileChoice tc = choose_tile(M, N, Kp);
    std::vector<uint8_t> a_scales = s.compact_a ? pad_scales_k(Aq.scales.data(), M, K) : Aq.scales;
    TiledScale sA = tile_scale(preprocess_scale(a_scales.data(), M, Kp), tc.MPW, K_TILE / 64);
    TiledScale sB = tile_scale(preprocess_scale(Bq.scales.data(), N, Kp), tc.NPW, K_TILE / 64);

    // Compact A rows are 3K/4 bytes; the buffer carries the documented end pad.
    const int a_rb = Aq.packed_row_bytes;
    const size_t a_bytes = Aq.packed_data.size() + (s.compact_a ? (size_t)a_compact_end_pad(K) : 0);
    const size_t out_elt = ot == OutType::F32 ? 4 : 2;
    const size_t wsb = gemm_workspace_size(M, N, Kp, a_rb);

    void *dA, *dB, *dD, *ws = nullptr;
    uint8_t *dsA, *dsB;
    CUDA_OK(cudaMalloc(&dA, a_bytes));
    CUDA_OK(cudaMemset(dA, 0, a_bytes));
    CUDA_OK(cudaMalloc(&dB, Bsh.data.size()));
    CUDA_OK(cudaMalloc(&dsA, sA.data.size()));
    CUDA_OK(cudaMalloc(&dsB, sB.data.size()));
    CUDA_OK(cudaMalloc(&dD, (size_t)M * N * out_elt));
    if (wsb) CUDA_OK(cudaMalloc(&ws, wsb));
    CUDA_OK(cudaMemcpy(dA, Aq.packed_data.data(), Aq.packed_data.size(), cudaMemcpyHostToDevice));
    CUDA_OK(cudaMemcpy(dB, Bsh.data.data(), Bsh.data.size(), cudaMemcpyHostToDevice));
    CUDA_OK(cudaMemcpy(dsA, sA.data.data(), sA.data.size(), cudaMemcpyHostToDevice));
    CUDA_OK(cudaMemcpy(dsB, sB.data.data(), sB.data.size(), cudaMemcpyHostToDevice));

    gemm(ot, M, N, Kp, dA, dB, dsA, dsB, dD, a_rb, Bq.packed_row_bytes, ws, wsb);
    const int err = mxfp6_last_error();
    CUDA_OK(cudaDeviceSynchronize());
    const int dev_status = mxfp6_device_status();

    std::vector<uint8_t> Dh((size_t)M * N * out_elt);
    CUDA_OK(cudaMemcpy(Dh.data(), dD, Dh.size(), cudaMemcpyDeviceToHost));
    cudaFree(dA);
    cudaFree(dB);
    cudaFree(dsA);
    cudaFree(dsB);
    cudaFree(dD);
    if (ws) cudaFree(ws);

    char label[128];
    std::snprintf(label, sizeof label, "%dx%dx%d%s %s (ws %zu B)", M, N, K, s.compact_a ? " compact-A" : "",
                  name_of(ot), wsb);
    if (err != MXFP6_OK || dev_status != 0) {
        fail(std::string(label) + ": error " + std::to_string(err) + ", device status " + std::to_string(dev_status));
        return;
    }

    // Host product of the dequantised operands in double, on sampled rows (all columns, all K).
    // Products of FP6 codes and power-of-two scales are exact in FP32, so the kernel's only error
    // is FP32 accumulation: bounded by K * 2^-24 * sum|a*b| (with margin), plus the rounding of
    // the output type.
    std::vector<float> Ad((size_t)M * Ka), Bd((size_t)N * Kp);
    dequantize_mxfp6(Aq, Ad.data());
    dequantize_mxfp6(Bq, Bd.data());
    const double out_rel = ot == OutType::F32 ? 0.0 : (ot == OutType::F16 ? 1.0 / 2048 : 1.0 / 256);
    int bad = 0;
    double worst = 0.0;
    const int row_step = M > 512 ? 7 : 1;
    for (int m = 0; m < M; m += row_step)
        for (int n = 0; n < N; n++) {
            double acc = 0.0, mag = 0.0;
            for (int k = 0; k < K; k++) {
                const double p = (double)Ad[(size_t)m * Ka + k] * (double)Bd[(size_t)n * Kp + k];
                acc += p;
                mag += std::fabs(p);
            }
            const size_t i = (size_t)m * N + n;
            float got;
            if (ot == OutType::F32) std::memcpy(&got, &Dh[i * 4], 4);
            else {
                uint16_t h;
                std::memcpy(&h, &Dh[i * 2], 2);
                got = ot == OutType::F16 ? half_bits_to_float(h) : bf16_bits_to_float(h);
            }
            const double tol = 4.0 * K * std::ldexp(1.0, -24) * mag + out_rel * std::fabs(acc) + 1e-30;
            const double e = std::fabs((double)got - acc);
            if (!(e <= tol)) bad++;
            if (tol > 0 && e / tol > worst) worst = e / tol;
        }
    if (bad) fail(std::string(label) + ": " + std::to_string(bad) + " elements outside tolerance");
    else std::printf("ok   %s: worst error / tolerance %.3f\n", label, worst);
}

// BASELINE config 1 through the public C++ API, timed as the reference times its launch-bound
// floor (tests/test_gemm.cpp:32-52): host enqueue and device time of back-to-back calls.
// Per-call time of M x N x K (K zero-padded to kpad(K), as the reference's harness pads it) timed
// the reference's way: 8 warm-ups, then 20 back-to-back gemm() calls on the legacy default stream
// between two events, best of 4. Operands are N(0, 1) rows quantised with the public helpers.
void time_shape(int M, int N, int K, OutType ot, const std::string& label) {
    const int Kp = kpad(K);
    std::mt19937 rng(5);
    std::normal_distribution<float> nd(0.0f, 1.0f);
    std::vector<float> A((size_t)M * Kp, 0.0f), B((size_t)Kp * N, 0.0f);
    for (int r = 0; r < M; r++)
        for (int k = 0; k < K; k++) A[(size_t)r * Kp + k] = nd(rng);
    for (int k = 0; k < K; k++)
        for (int c = 0; c < N; c++) B[(size_t)k * N + c] = 0.05f * nd(rng);
    QuantizedMatrix Aq = quantize_to_mxfp6(A.data(), M, Kp);
    QuantizedMatrix Bq = preprocess_B(B.data(), Kp, N);
    PreshuffledB Bsh = preshuffle_B(Bq);
    TileChoice tc = choose_tile(M, N, Kp);
    TiledScale sA = tile_scale(preprocess_scale(Aq.scales.data(), M, Kp), tc.MPW, K_TILE / 64);
    TiledScale sB = tile_scale(preprocess_scale(Bq.scales.data(), N, Kp), tc.NPW, K_TILE / 64);
    const size_t wsb = gemm_workspace_size(M, N, Kp);
    const size_t esize = ot == OutType::F32 ? 4 : 2;
    void *dA, *dB, *dD, *ws = nullptr;
    uint8_t *dsA, *dsB;
    CUDA_OK(cudaMalloc(&dA, Aq.packed_data.size()));
    CUDA_OK(cudaMalloc(&dB, Bsh.data.size()));
    CUDA_OK(cudaMalloc(&dsA, sA.data.size()));
    CUDA_OK(cudaMalloc(&dsB, sB.data.size()));
    CUDA_OK(cudaMalloc(&dD, (size_t)M * N * esize));
    if (wsb) CUDA_OK(cudaMalloc(&ws, wsb));
    CUDA_OK(cudaMemcpy(dA, Aq.packed_data.data(), Aq.packed_data.size(), cudaMemcpyHostToDevice));
    CUDA_OK(cudaMemcpy(dB, Bsh.data.data(), Bsh.data.size(), cudaMemcpyHostToDevice));
    CUDA_OK(cudaMemcpy(dsA, sA.data.data(), sA.data.size(), cudaMemcpyHostToDevice));
    CUDA_OK(cudaMemcpy(dsB, sB.data.data(), sB.data.size(), cudaMemcpyHostToDevice));
    auto call = [&] {
        gemm(ot, M, N, Kp, dA, dB, dsA, dsB, dD, Aq.packed_row_bytes, Bq.packed_row_bytes, ws, wsb);
    };
    for (int i = 0; i < 8; i++) call();
    CUDA_OK(cudaDeviceSynchronize());
    cudaEvent_t e0, e1;
    CUDA_OK(cudaEventCreate(&e0));
    CUDA_OK(cudaEventCreate(&e1));
    float best = 1e30f;
    for (int rep = 0; rep < 4; rep++) {
        CUDA_OK(cudaEventRecord(e0, 0));
        for (int i = 0; i < 20; i++) call();
        CUDA_OK(cudaEventRecord(e1, 0));
        CUDA_OK(cudaEventSynchronize(e1));
        float ms = 0.0f;
        CUDA_OK(cudaEventElapsedTime(&ms, e0, e1));
        if (ms < best) best = ms;
    }
    if (mxfp6_last_error() != MXFP6_OK || mxfp6_device_status() != 0) fail(label + " timing calls reported an error");
    std::printf("%s back-to-back from C++: %.3f us per call (%dx%dx%d %s out, 20 calls, best of 4)\n", label.c_str(),
                best * 1000.0f / 20, M, N, K, ot == OutType::F32 ? "FP32" : ot == OutType::F16 ? "FP16" : "BF16");
    cudaEventDestroy(e0);
    cudaEventDestroy(e1);
    cudaFree(dA);
    cudaFree(dB);
    cudaFree(dsA);
    cudaFree(dsB);
    cudaFree(dD);
    if (ws) cudaFree(ws);
}

void gpu_checks() {
    int ndev = 0;
    if (cudaGetDeviceCount(&ndev) != cudaSuccess || ndev == 0) {
        fail("no CUDA device");
        return;
    }
    const Shape shapes[] = {
        {256, 512, 1024, false},
        {128, 256, 16384, false},  // skinny, deep K: takes the split-K route with the workspace
        {1024, 1024, 4096, false},
        {256, 384, 1952, true},    // reference compact A: row stride 3K/4 = 1464 bytes
    };
    uint32_t seed = 11;
    for (const Shape& s : shapes)
        for (OutType ot : {OutType::F32, OutType::F16, OutType::BF16}) run_case(s, ot, seed++);
}

}  // namespace

int main(int argc, char** argv) {
    const std::string mode = argc > 1 ? argv[1] : "host";
    if (mode == "host") host_checks();
    else if (mode == "gpu") {
        host_checks();
        gpu_checks();
    } else if (mode == "time") {
        if (argc == 2) {
            time_shape(256, 256, 512, OutType::F32, "cfg1");
        } else if (argc == 6) {
            const std::string o = argv[5];
            const OutType ot = o == "F32" ? OutType::F32 : o == "BF16" ? OutType::BF16 : OutType::F16;
            time_shape(std::atoi(argv[2]), std::atoi(argv[3]), std::atoi(argv[4]), ot, "shape");
        } else {
            std::printf("usage: %s time [M N K F32|F16|BF16]\n", argv[0]);
            return 2;
        }
    } else {
        std::printf("usage: %s host|gpu|time [M N K OUT]\n", argv[0]);
        return 2;
    }
    std::printf("%s: %d failure(s)\n", mode.c_str(), g_failures);
    return g_failures ? 1 : 0;
}
