#pragma once
// Public C++ API of the B200 MXFP6 GEMM library (libmxfp6gemm, sm_100a build).
//
//   D[M,N] = A[M,K] * B[K,N]
//
// A and B hold FP6 E2M3 codes with one E8M0 scale per 32-element block along K; D is FP32, FP16
// or BF16. The declarations below are the ones of the reference library's public header
// (reference: include/mxfp6/gemm.hpp:25-64) so that a caller recompiles unchanged; what changes
// is the meaning of the preprocessed device layouts, which come from this library's own
// mxfp6/preprocess.hpp helpers (same names as the reference's):
//   * dA   : row-major packed FP6 A, A_row_bytes per row (identical to the reference layout).
//   * dBsh : packed FP6 B^T[N][Kp], B_row_bytes per row (this library's preshuffle_B is the
//            identity on the preprocess_B output; the tensor-memory accelerator reads it as is).
//   * dsA / dsB : E8M0 scales in 128-row x 4-block atoms (preprocess_scale + tile_scale).
//
// This header is device-free: a host translation unit can include it and link the shared
// library without the CUDA compiler. Every call is asynchronous on the CUDA legacy default
// stream (the reference launches on the HIP null stream); mxfp6_gemm_stream() in
// mxfp6_gemm.h takes an explicit stream.
#include <cstddef>
#include <cstdint>

namespace mxfp6 {

enum class OutType { F32, F16, BF16 };

// K is consumed in tiles of K_TILE elements. On B200 the granule is 128 (the reference uses 192):
// a packed FP6 row of Kp elements is 0.75*Kp bytes, and the tensor-memory accelerator's 6-bit
// unpack mode needs 32-byte row strides, which 0.75*Kp meets exactly when Kp % 128 == 0.
// Callers pad K up to kpad(K); the padded K-tail must be zero on at least one operand.
constexpr int K_TILE = 128;
inline int kpad(int K) {
    return (K + K_TILE - 1) / K_TILE * K_TILE;
}

// Route chosen for (M,N,Kp): the output tile (MT x NT) of the B200 kernel that gemm() launches.
// MPW / NPW are kept for source compatibility with the reference (where they set the scale
// grouping); on B200 the scale layout does not depend on the route, and they report the number
// of 32-row blocks per tile on each side (MT/32, NT/32).
struct TileChoice {
    int MT, NT, MPW, NPW;
};
TileChoice choose_tile(int M, int N, int Kp);

// Bytes of split-K workspace gemm() uses for (M,N,Kp); 0 when the shape does not split.
// The caller owns this device buffer (allocate once, reuse across calls, one per stream).
size_t gemm_workspace_size(int M, int N, int Kp);

// The same for an A of row stride A_row_bytes (no counterpart in the reference): when that stride
// is not one the tensor load can address (the compact 3K/4 with K % 128 != 0), the size adds room
// for a padded copy of A, which gemm() then makes (one HBM pass) before running the tensor-load
// kernel. With a workspace sized by the three-argument query, gemm() makes the same copy in
// scratch from a stream-ordered memory pool of its own when M*N*Kp >= 2^31 (not while the
// stream captures a graph; mxfp6_set_repad_scratch in mxfp6_gemm.h switches it off), and
// otherwise the kernels' loader warps read A in place. The results are identical every way.
size_t gemm_workspace_size(int M, int N, int Kp, int A_row_bytes);

// D[M,N] = A[M,K] * B[K,N]; see the layout notes above. Requirements (checked; a violation
// prints "[mxfp6] ..." to stderr, records an error for mxfp6_last_error() and launches nothing):
//   M % 128 == 0, N % 128 == 0, Kp % 128 == 0, Kp > 0; B_row_bytes >= 0.75*Kp and a multiple of
//   32, dBsh 32-byte aligned; A_row_bytes a multiple of 4 holding the row's K codes
//   (> 0.75*Kp - 96: the reference's compact stride 3K/4 qualifies), dA 4-byte aligned (A strides
//   that are multiples of 32 on a 32-byte aligned base take the tensor load, others the kernels'
//   loader warps); dsA/dsB/dD 16-byte aligned.
// If the shape would split but ws is null or smaller than gemm_workspace_size(), gemm() runs
// unsplit (still correct) and warns on stderr, as the reference does.
void gemm(OutType ot, int M, int N, int Kp, const void* dA, const void* dBsh, const uint8_t* dsA,
          const uint8_t* dsB, void* dD, int A_row_bytes, int B_row_bytes, void* ws, size_t ws_bytes);

}  // namespace mxfp6
