/* C ABI of libmxfp6gemm (B200, sm_100a).
 *
 * Plain pointers and sizes only; no CUDA or torch types. Every entry point mirrors one of the
 * reference library's C++ entry points (eeezio/mxfp6-gemm, paths relative to that project) so a
 * foreign-function binding (ctypes, cgo, JNI, ...) can drive the same path:
 *
 *   mxfp6_gemm                  <- mxfp6::gemm                 include/mxfp6/gemm.hpp:63-64
 *   mxfp6_gemm_workspace_size   <- mxfp6::gemm_workspace_size  include/mxfp6/gemm.hpp:53
 *   mxfp6_choose_tile           <- mxfp6::choose_tile          include/mxfp6/gemm.hpp:46
 *   mxfp6_kpad / mxfp6_k_tile   <- mxfp6::kpad / K_TILE        include/mxfp6/gemm.hpp:30-33
 *   mxfp6_gemm_force_tile       <- mxfp6::gemm_force_tile      src/gemm.cpp:89-107 (test hook)
 *
 * Additions with no counterpart in the reference (it returns void and never checks errors):
 *   mxfp6_gemm_stream     the same call on an explicit cudaStream_t (passed as void*).
 *   mxfp6_last_error      status of the last call on this thread (0 = ok).
 *   mxfp6_device_status   synchronises the device and returns/clears the kernel status word
 *                         (bounded waits inside the kernel record timeouts there).
 *   mxfp6_gemm_gather     the GEMM with its output written to several (peer) destinations.
 *
 * Host preprocessing helpers (the C face of mxfp6/preprocess.hpp, used by bindings that cannot
 * instantiate the C++ header) are declared at the end.
 */
#ifndef MXFP6_GEMM_H_
#define MXFP6_GEMM_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Output element type; values match mxfp6::OutType. */
enum mxfp6_out_type { MXFP6_OUT_F32 = 0, MXFP6_OUT_F16 = 1, MXFP6_OUT_BF16 = 2 };

/* Error codes returned by mxfp6_last_error(). */
enum mxfp6_status {
    MXFP6_OK = 0,
    MXFP6_ERR_INVALID_SHAPE = 1,     /* M, N or Kp not a positive multiple of 128 */
    MXFP6_ERR_INVALID_STRIDE = 2,    /* B row bytes < 0.75*Kp or not a multiple of 32; A row bytes
                                        not a multiple of 4 or <= 0.75*Kp - 96 (shorter than any
                                        K with kpad(K) == Kp) */
    MXFP6_ERR_MISALIGNED = 3,        /* a pointer violates its alignment rule (A 4, B 32, scales and
                                        D 16 bytes) */
    MXFP6_ERR_NULL_POINTER = 4,      /* a required pointer is null */
    MXFP6_ERR_INVALID_OUT_TYPE = 5,  /* ot not one of mxfp6_out_type */
    MXFP6_ERR_CUDA = 6,              /* a CUDA runtime / driver call failed */
    MXFP6_ERR_DEVICE_TIMEOUT = 7,    /* a kernel wait hit its bound (see mxfp6_device_status) */
    MXFP6_ERR_WORKSPACE = 8,         /* workspace too small for a forced split */
    MXFP6_ERR_UNSUPPORTED = 9        /* route / option not available on this device */
};

/* Device status bits written by kernels (mxfp6_device_status). */
#define MXFP6_DEV_TIMEOUT_PRODUCER 0x1u /* TMA producer: an empty slot never came back */
#define MXFP6_DEV_TIMEOUT_MMA 0x2u      /* MMA issuer: a full slot or free accumulator never came */
#define MXFP6_DEV_TIMEOUT_EPILOGUE 0x4u /* epilogue: an accumulator was never committed */
#define MXFP6_DEV_TIMEOUT_DRAIN 0x8u    /* abort path: in-flight copies or MMAs did not settle */

/* D[M,N] = A[M,K]·B[K,N] on the legacy default stream. ot: mxfp6_out_type. See
 * include/mxfp6/gemm.hpp for layouts and requirements. On a validation error nothing is
 * launched, a message goes to stderr and mxfp6_last_error() returns the code.
 * A_row_bytes may be the reference's compact stride 3K/4 (K % 128 != 0, scales extended with
 * pad_scales_k): such an A, or any A whose stride is not a multiple of 32 bytes or whose base is
 * not 32-byte aligned, is loaded by the kernels' loader warps instead of the tensor load. */
void mxfp6_gemm(int ot, int M, int N, int Kp, const void* dA, const void* dBsh, const uint8_t* dsA,
                const uint8_t* dsB, void* dD, int A_row_bytes, int B_row_bytes, void* ws,
                size_t ws_bytes);

/* Same as mxfp6_gemm on an explicit stream (a cudaStream_t passed as void*; NULL = legacy). */
void mxfp6_gemm_stream(int ot, int M, int N, int Kp, const void* dA, const void* dBsh,
                       const uint8_t* dsA, const uint8_t* dsB, void* dD, int A_row_bytes,
                       int B_row_bytes, void* ws, size_t ws_bytes, void* stream);

/* Split-K workspace bytes gemm() wants for (M,N,Kp); 0 when the route does not split. The
 * query has no output type, so this is the largest need over the output types: FP32 output
 * splits long K into more segments to hold its tolerance. */
size_t mxfp6_gemm_workspace_size(int M, int N, int Kp);

/* The same for one output type (no counterpart in the reference): a caller that knows ot can
 * allocate exactly what that call uses. */
size_t mxfp6_gemm_workspace_size_out(int ot, int M, int N, int Kp);

/* Workspace for an A of row stride A_row_bytes (no counterpart in the reference): adds room for
 * a padded copy of A when the stride is one the tensor load cannot address (the compact 3K/4),
 * so that mxfp6_gemm re-pads A into the workspace and runs the tensor-load kernel. */
size_t mxfp6_gemm_workspace_size_a(int M, int N, int Kp, int A_row_bytes);

/* Column-parallel GEMM whose epilogue also performs the all-gather of the shards (no
 * counterpart in the reference, whose multi-GPU use is left to the caller): D = A·B (this
 * rank's N columns) is written into each of the n_dst (1..8) row-major [M][ldd] matrices dDs[i]
 * at column col0 — typically this rank's gathered output and its peers' (pointers from
 * mxfp6_ipc_import, reached over NVLink with plain peer stores). ldd and col0 must keep 16-byte
 * aligned rows. The kernel never waits on a peer: the caller orders the ranks (synchronise the
 * stream, then a barrier) before reading the gathered output. Same validation and workspace
 * contract as mxfp6_gemm_stream. */
void mxfp6_gemm_gather(int ot, int M, int N, int Kp, const void* dA, const void* dBsh, const uint8_t* dsA,
                       const uint8_t* dsB, void* const* dDs, int n_dst, long long ldd, int col0, int A_row_bytes,
                       int B_row_bytes, void* ws, size_t ws_bytes, void* stream);

/* CUDA IPC for mxfp6_gemm_gather's peer destinations. export: a 64-byte handle of the
 * allocation holding dptr, and dptr's offset in it. import (in another process, with its own
 * device current): maps the allocation, returns its base (for close) and the pointer. */
int mxfp6_ipc_export(const void* dptr, void* handle_out, size_t* offset_out);
int mxfp6_ipc_import(const void* handle, size_t offset, void** base_out, void** dptr_out);
int mxfp6_ipc_close(void* base);

/* Route for (M,N,Kp): writes MT, NT, MPW, NPW into out[0..3]. */
void mxfp6_choose_tile(int M, int N, int Kp, int* out4);

/* The route gemm() takes for output type ot (no counterpart in the reference): writes MT, NT
 * and the number of K splits into out[0..2]. FP32 output may split where FP16/BF16 does not. */
void mxfp6_route(int ot, int M, int N, int Kp, int* out3);

/* Whether the CTA-pair route runs a stream-K tail (no counterpart in the reference): 1 when its
 * 256 x 256 tiles do not fill whole waves of CTA pairs and the idle part of the last wave is deep
 * enough to repay the hand-offs (at least 35 slabs of 128 K), so the last waves' K slabs are
 * shared out evenly; 0 otherwise. A tile shared by two pairs is summed in one accumulator chain (the first
 * pair hands its FP32 accumulator to the second through the workspace), so results are identical
 * to the whole-tile schedule. The workspace then holds 256 KB + 16 bytes per CTA pair; it is in
 * gemm_workspace_size(). Without it the call runs whole tiles and warns, as for split-K. */
int mxfp6_route_stream_k(int ot, int M, int N, int Kp);

/* No counterpart in the reference (its split-K, src/dispatch.hpp:30-59, cuts K into S equal
 * segments per tile). 1 when the route is a banded split on the CTA pair. With fewer 256 x 256
 * tiles (T) than CTA pairs (P) and a deep K, each of the first L*T pairs (L = P / T) takes one
 * long K band of one tile, and the pairs left over take the short bands the rest of K is cut
 * into, several tiles each, so that no pair idles and the pairs sharing an operand walk K
 * together. mxfp6_route reports splits = L + the number of short bands; the workspace is
 * splits*M*N*4 bytes as for split-K, and the reduce adds each element's bands in K order. */
int mxfp6_route_banded(int ot, int M, int N, int Kp);

/* Workspace bytes of the stream-K tail on the current device (256 KB + 16 bytes per CTA pair). */
size_t mxfp6_stream_k_workspace_bytes(void);

/* K granule (128) and K padded to it. */
int mxfp6_k_tile(void);
int mxfp6_kpad(int K);

/* Test hook (reference: src/gemm.cpp:89-107 gemm_force_tile): run a specific tile and split
 * factor instead of the routed one. (MT, NT) in {(256,256) CTA pair, (128,256), (128,128)};
 * splits >= 1 (splits > 1 needs ws_bytes >= splits*M*N*4). Same validation as mxfp6_gemm;
 * stream may be NULL. */
void mxfp6_gemm_force_tile(int ot, int M, int N, int Kp, int MT, int NT, int splits, const void* dA,
                           const void* dBsh, const uint8_t* dsA, const uint8_t* dsB, void* dD,
                           int A_row_bytes, int B_row_bytes, void* ws, size_t ws_bytes,
                           void* stream);

/* Test hook (no counterpart in the reference): mxfp6_gemm_force_tile plus the CTA pair's stream-K
 * tail (stream_k 1 with MT = NT = 256 and splits = 1; it takes effect when the tiles do not fill
 * whole waves, and needs a 256-byte aligned workspace of 256 KB + 16 bytes per CTA pair; see
 * mxfp6_route_stream_k) or banded split (stream_k 2 with MT = NT = 256 and `splits` short bands,
 * fewer tiles than CTA pairs; the workspace holds (L + splits)*M*N*4 bytes; see
 * mxfp6_route_banded). mxfp6_gemm_force_tile runs whole tiles (stream_k = 0). */
void mxfp6_gemm_force_route(int ot, int M, int N, int Kp, int MT, int NT, int splits, int stream_k,
                            const void* dA, const void* dBsh, const uint8_t* dsA, const uint8_t* dsB, void* dD,
                            int A_row_bytes, int B_row_bytes, void* ws, size_t ws_bytes, void* stream);

/* No counterpart in the reference. The same computation as mxfp6_gemm_stream, for callers that
 * cannot call cudaMalloc: for example a plugin inside a host application that owns every device
 * allocation through its own pool, or a foreign-function binding that only forwards pointers it
 * was given and has no way to create a workspace. Nothing is allocated: when the route splits K,
 * the FP32 partial sums go to a fixed array inside this library (mxfp6_static_workspace_bytes(),
 * 32 MiB), which every GPU that loads the library reserves until the process exits. A shape whose
 * split needs more than that is rejected with MXFP6_ERR_WORKSPACE and nothing is launched.
 * The first call on a device looks up the array's device address (cudaGetSymbolAddress) with
 * that device current; make that first call before any stream capture. A lookup that fails is
 * not remembered: the next call on that device tries again. All calls share the one
 * array and it keeps the last call's contents (every partial is written before it is read, so
 * nothing needs clearing); calls that overlap on the GPU, on any streams, race on it. */
void mxfp6_gemm_static_workspace(int ot, int M, int N, int Kp, const void* dA, const void* dBsh,
                                 const uint8_t* dsA, const uint8_t* dsB, void* dD, int A_row_bytes,
                                 int B_row_bytes, void* stream);

/* Size in bytes of the static split-K array mxfp6_gemm_static_workspace uses. */
size_t mxfp6_static_workspace_bytes(void);

/* No counterpart in the reference. Re-pad scratch for a compact A (a row stride the tensor
 * load cannot address: the reference's compact stride 3K/4 with K % 128 != 0). mxfp6_gemm,
 * mxfp6_gemm_stream and mxfp6_gemm_gather re-pad such an A before the GEMM, which then runs at
 * about the speed of a padded A. The padded copy goes into the caller's workspace when
 * mxfp6_gemm_workspace_size_a sized it; otherwise, when M*N*Kp >= 2^31, into scratch that the
 * library takes, in stream order, from a memory pool of its own on the current device
 * (M * 0.75*Kp bytes per call, given back in stream order after the GEMM; the pool keeps what it
 * has mapped, in 32 MiB steps, for later calls). No scratch is taken for smaller GEMMs (there the
 * extra launch and pool calls cost more than they save), while the stream is capturing a graph,
 * when it is switched off, or when the allocation fails: the kernels then read A in place
 * (identical results; on large shapes about half the speed). mxfp6_gemm_static_workspace and the
 * force hooks never take it.
 *   mxfp6_set_repad_scratch       1 (default; MXFP6_REPAD_SCRATCH=0 in the environment at load
 *                                 makes it 0) lets calls take scratch, 0 forbids it; process-wide.
 *                                 Returns the previous setting.
 *   mxfp6_repad_scratch_bytes     bytes the pool holds on the current device.
 *   mxfp6_release_repad_scratch   synchronises the current device and returns the pool's memory
 *                                 to the driver; 0 or MXFP6_ERR_CUDA. */
int mxfp6_set_repad_scratch(int enable);
size_t mxfp6_repad_scratch_bytes(void);
int mxfp6_release_repad_scratch(void);

/* Status of the last mxfp6_* call on this thread, and a static message for it. */
int mxfp6_last_error(void);
const char* mxfp6_last_error_string(void);

/* Synchronises the current device, returns the sticky kernel status bits (MXFP6_DEV_*) and
 * clears them. Returns -1 if the synchronisation itself failed. */
int mxfp6_device_status(void);

/* No counterpart in the reference (whose kernels have no bounded waits). Sets the cycle budget
 * of the bounded barrier waits inside the GEMM kernels that this host thread launches from now
 * on; cycles <= 0 restores the default (4e9 cycles, about 2 s). Returns the previous setting
 * (0 = default). It exists to exercise the timeout path: with a budget far below the work, the
 * kernels give up, set MXFP6_DEV_* bits, wait out their copies and MMAs in flight, free tensor
 * memory and return; their outputs are then incomplete, and mxfp6_device_status() reports the
 * bits. Production callers leave it at the default. */
long long mxfp6_set_wait_budget(long long cycles);

/* Number of kernels this library has launched in this process (all devices). */
uint64_t mxfp6_launch_count(void);

/* ---- host preprocessing (C face of include/mxfp6/preprocess.hpp) --------------------------
 * All buffers are host memory, caller-allocated. Sizes: packed row = 3*cols/4 bytes,
 * raw scales = rows*(cols/32) bytes, tiled scales = mxfp6_tiled_scale_bytes(rows, cols). */

/* quantize_to_mxfp6 (reference: include/mxfp6/preprocess.hpp:51-97): float [rows][cols]
 * (cols % 32 == 0) -> packed FP6 [rows][3*cols/4] + raw E8M0 scales [rows][cols/32].
 * nthreads <= 0 uses all hardware threads; the result does not depend on it. */
void mxfp6_quantize(const float* mat, int rows, int cols, uint8_t* packed, uint8_t* scales,
                    int nthreads);

/* quantize_to_mxfp6 on the GPU (reference: include/mxfp6/preprocess.hpp:51-97), bit-identical to
 * the host version: device float [rows][cols] (cols % 32 == 0, 16-byte aligned) -> device packed
 * FP6 [rows][3*cols/4] (4-byte aligned) and scales, raw [rows][cols/32] (scale_layout 0) or
 * directly in the GEMM's tiled atom layout (scale_layout 1, cols % 128 == 0; rows past the
 * last full atom are not written). rows <= 65535. Asynchronous on `stream` (NULL = legacy).
 * Returns an mxfp6_status. */
int mxfp6_quantize_device(const float* d_mat, int rows, int cols, uint8_t* d_packed, uint8_t* d_scales,
                          int scale_layout, void* stream);

/* The same, writing rows of padded_cols codes (3*padded_cols/4 bytes, zero tail) and scales for
 * padded_cols/32 blocks (tail blocks get the finite code 127): activations quantised this way
 * meet the GEMM's 32-byte row-stride rule for any K with K % 32 == 0 (use padded_cols = kpad(K)).
 * No counterpart in the reference, whose "compact A" recipe reads rows of K codes in place. */
int mxfp6_quantize_device_padded(const float* d_mat, int rows, int cols, int padded_cols, uint8_t* d_packed,
                                 uint8_t* d_scales, int scale_layout, void* stream);

/* dequantize_mxfp6 (reference: include/mxfp6/preprocess.hpp:100-109). */
void mxfp6_dequantize(const uint8_t* packed, const uint8_t* scales, int rows, int cols,
                      float* out);

/* Bytes of the tiled scale layout for a [rows][cols/32] raw scale matrix (cols % 128 == 0):
 * ceil(rows/128) * (cols/128) * 512. */
size_t mxfp6_tiled_scale_bytes(int rows, int cols);

/* preprocess_scale + tile_scale (reference: include/mxfp6/preprocess.hpp:136-162,216-233):
 * raw scales [rows][cols/32] -> B200 atom layout. Rows past `rows` in the last atom get the
 * finite code 127. */
void mxfp6_tile_scales(const uint8_t* scales, int rows, int cols, uint8_t* tiled);

/* Inverse of mxfp6_tile_scales (for checks). */
void mxfp6_untile_scales(const uint8_t* tiled, int rows, int cols, uint8_t* scales);

/* ---- import of buffers prepared for the reference library (gfx950 layouts) -------------------
 * One-time host conversions, so weights preprocessed for the reference need no re-quantising. */

/* Inverse of the reference's preshuffle_B (include/mxfp6/preprocess.hpp:182-207): ref_bsh holds
 * (N/32)*(Kp_ref/64) tiles of 1536 bytes; out receives B^T packed rows [N][out_row_bytes], the
 * first 3*Kp_ref/4 bytes of each row filled and the rest zeroed (pad Kp up to a multiple of 128
 * and use out_row_bytes = 3*kpad(Kp_ref)/4). Returns an mxfp6_status. */
int mxfp6_import_ref_B(const uint8_t* ref_bsh, int N, int Kp_ref, uint8_t* out, int out_row_bytes);

/* Inverse of the reference's tile_scale(preprocess_scale(raw, dim, Kp_ref), group, subs)
 * (include/mxfp6/preprocess.hpp:136-162,216-233): writes raw scales [dim][Kp_ref/32]. group is
 * the reference's MPW/NPW for the route it tiled for, subs its K_TILE/64 (3). */
int mxfp6_import_ref_scales(const uint8_t* ref_tiled, int dim, int Kp_ref, int group, int subs, uint8_t* raw_out);

/* Device versions of the two imports (device pointers, asynchronous on `stream`, NULL = legacy),
 * writing this library's layouts directly in one pass.
 * mxfp6_import_ref_B_device: d_ref_bsh as for mxfp6_import_ref_B (16-byte aligned); d_out
 * receives B^T rows [N][out_row_bytes] (8-byte aligned, out_row_bytes % 8 == 0): the first
 * min(3*Kp_ref/4, out_row_bytes) bytes of each row from the reference buffer, the rest zeroed.
 * Use out_row_bytes = 3*kpad(K)/4; packed bytes dropped when that is below 3*Kp_ref/4 hold the
 * reference's zero K padding. */
int mxfp6_import_ref_B_device(const void* d_ref_bsh, int N, int Kp_ref, void* d_out, int out_row_bytes,
                              void* stream);

/* mxfp6_import_ref_scales_device: d_ref_tiled as for mxfp6_import_ref_scales; d_out_tiled (4-byte
 * aligned) receives mxfp6_tiled_scale_bytes(dim, Kp) bytes in this library's atom layout for
 * Kp (% 128 == 0): blocks past Kp_ref/32 and rows past dim get the finite code 127, blocks past
 * Kp/32 are dropped. */
int mxfp6_import_ref_scales_device(const void* d_ref_tiled, int dim, int Kp_ref, int group, int subs,
                                   void* d_out_tiled, int Kp, void* stream);

/* Device version of mxfp6_repad_rows (device pointers, asynchronous on `stream`): turns an A
 * operand in the reference's compact layout (row stride 3*K/4 with K % 128 != 0, which the
 * tensor-memory accelerator cannot address) into rows of 3*kpad(K)/4 bytes in a caller buffer;
 * pair it with pad_scales_k / mxfp6_tile_scales for the scales. */
int mxfp6_repad_rows_device(const void* d_src, int rows, int src_row_bytes, int bytes_used, void* d_dst,
                            int dst_row_bytes, void* stream);

/* Copy rows of src_bytes_used bytes from a src_row_bytes stride to a dst_row_bytes stride,
 * zero-filling each row's tail (re-padding A rows from the reference's Kp to this library's). */
int mxfp6_repad_rows(const uint8_t* src, int rows, int src_row_bytes, int src_bytes_used, uint8_t* dst,
                     int dst_row_bytes);

#ifdef __cplusplus
}
#endif

#endif /* MXFP6_GEMM_H_ */
