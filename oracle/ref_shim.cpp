// C shim over the reference's own CPU path — TEST INFRASTRUCTURE ONLY.
//
// oracle/Makefile compiles this file against the reference's headers where they lie
// (REF_DIR/include/mxfp6/{types,preprocess}.hpp and REF_DIR/tests/reference.hpp of
// eeezio/mxfp6-gemm) into oracle/_ref/libmxfp6ref.so. Nothing of the reference is copied
// here: each function forwards to the reference's function of the same meaning, so tests can
// pin the C oracle (oracle/mxfp6_oracle.c) and generate golden vectors from the reference
// itself, and bench.py can time the reference's CPU GEMM as its CPU baseline.
//
//   ref_fp6_to_float / ref_float_to_fp6   mxfp6::fp6_e2m3_to_float / float_to_fp6_e2m3
//   ref_e8m0_to_float / ref_float_to_e8m0 mxfp6::e8m0_to_float / float_to_e8m0
//   ref_pack_fp6 / ref_unpack_fp6         mxfp6::pack_fp6 / unpack_fp6
//   ref_quantize                          mxfp6::quantize_to_mxfp6
//   ref_preshuffle_B / ref_tile_scales    mxfp6::preshuffle_B / tile_scale(preprocess_scale(..))
//   ref_gemm                              mxfp6::mxfp6_gemm_ref (single thread, as shipped)
//   ref_gemm_rows_mt                      mxfp6_gemm_ref on row slices of A over threads (each
//                                         output element keeps its summation order)
#include <cstring>
#include <thread>
#include <vector>

#include "reference.hpp"  // REF_DIR/tests; pulls in mxfp6/preprocess.hpp and mxfp6/types.hpp

using namespace mxfp6;

namespace {
QuantizedMatrix make_q(const uint8_t* packed, const uint8_t* scales, int rows, int cols) {
    QuantizedMatrix q;
    q.rows = rows;
    q.cols = cols;
    q.packed_row_bytes = fp6_packed_bytes(cols);
    q.scale_cols = cols / 32;
    q.packed_data.assign(packed, packed + (size_t)rows * q.packed_row_bytes);
    q.scales.assign(scales, scales + (size_t)rows * q.scale_cols);
    return q;
}
}  // namespace

extern "C" {

float ref_fp6_to_float(uint8_t c) { return fp6_e2m3_to_float(c); }
uint8_t ref_float_to_fp6(float v) { return float_to_fp6_e2m3(v); }
float ref_e8m0_to_float(uint8_t c) { return e8m0_to_float(c); }
uint8_t ref_float_to_e8m0(float v) { return float_to_e8m0(v); }
void ref_pack_fp6(const uint8_t* vals, int n, uint8_t* packed) { pack_fp6(vals, n, packed); }
void ref_unpack_fp6(const uint8_t* packed, int n, uint8_t* vals) { unpack_fp6(packed, n, vals); }

void ref_quantize(const float* mat, int rows, int cols, uint8_t* packed, uint8_t* scales) {
    QuantizedMatrix q = quantize_to_mxfp6(mat, rows, cols);
    std::memcpy(packed, q.packed_data.data(), q.packed_data.size());
    std::memcpy(scales, q.scales.data(), q.scales.size());
}

// preshuffle_B on B^T packed [N][3K/4] (N % 32 == 0, K % 64 == 0) -> (N/32)*(K/64)*1536 bytes.
void ref_preshuffle_B(const uint8_t* Bt, const uint8_t* sB, int N, int K, uint8_t* out) {
    QuantizedMatrix q = make_q(Bt, sB, N, K);
    PreshuffledB pb = preshuffle_B(q);
    std::memcpy(out, pb.data.data(), pb.data.size());
}

// tile_scale(preprocess_scale(raw, dim, K), group, subs) -> out (size returned by the query below).
size_t ref_tiled_scale_bytes(int dim, int K, int group, int subs) {
    int group_pad = (group + 3) / 4 * 4;
    return (size_t)(dim / 32 / group) * (size_t)(K / 64 / subs) * 64 * subs * group_pad;
}
void ref_tile_scales(const uint8_t* raw, int dim, int K, int group, int subs, uint8_t* out) {
    TiledScale ts = tile_scale(preprocess_scale(raw, dim, K), group, subs);
    std::memcpy(out, ts.data.data(), ts.data.size());
}

// A: packed [M][3K/4] + raw scales [M][K/32]; Bt: packed [N][3K/4] + scales [N][K/32].
void ref_gemm(const uint8_t* A, const uint8_t* sA, const uint8_t* Bt, const uint8_t* sB, int M, int N, int K,
              float* D) {
    QuantizedMatrix qa = make_q(A, sA, M, K), qb = make_q(Bt, sB, N, K);
    mxfp6_gemm_ref(qa, qb, D, M, K, N);
}

// Same result as ref_gemm, with the rows of A split over `nthreads` threads.
void ref_gemm_rows_mt(const uint8_t* A, const uint8_t* sA, const uint8_t* Bt, const uint8_t* sB, int M, int N,
                      int K, float* D, int nthreads) {
    if (nthreads < 1) nthreads = 1;
    if (nthreads > M) nthreads = M;
    const int rb = fp6_packed_bytes(K), sc = K / 32;
    QuantizedMatrix qb = make_q(Bt, sB, N, K);
    std::vector<std::thread> pool;
    for (int t = 0; t < nthreads; t++) {
        const int r0 = (int)((long long)M * t / nthreads), r1 = (int)((long long)M * (t + 1) / nthreads);
        pool.emplace_back([=, &qb] {
            if (r1 <= r0) return;
            QuantizedMatrix qa = make_q(A + (size_t)r0 * rb, sA + (size_t)r0 * sc, r1 - r0, K);
            mxfp6_gemm_ref(qa, qb, D + (size_t)r0 * N, r1 - r0, K, N);
        });
    }
    for (auto& th : pool) th.join();
}

}  // extern "C"
