#pragma once
// C++ kernel ABI of the fixed BF16 GEMM, identical in signature and meaning to the
// reference's include/kernel_api.h:7-19 so that a runner written against the reference
// links against libmo_gemm.so unchanged.
//
//   C[m, n] = A[m, k] · B[k, n]
//
// All pointers are DEVICE pointers owned by the caller, holding row-major BF16 payloads
// stored as raw uint16_t bit patterns (lda = k, ldb = n, ldc = n).  Inputs are BF16, the
// product is accumulated in FP32 on the sm_100a tensor cores (tcgen05.mma, TMEM
// accumulators) and rounded once to BF16 (round-to-nearest-even).  The call is asynchronous
// on `stream`; the caller synchronises.
//
// Returns false, without launching anything, on a null pointer or a non-positive dimension
// (reference src/kernels/bf16_gemm_v1.cu:2106-2111), on an unsupported device, or when the
// launch itself reports an error (reference :2179, which also consumes the non-sticky
// launch error).  No exception crosses this boundary.
//
// Memory.  The reference's launch allocates nothing.  Here, shapes that run whole tiles
// allocate nothing either: the hero shape 6464x7776x7232, its 2- and 4-GPU column slabs, square
// 8192, the LLM projection 4096x28672x8192, and M = 1, 16, 129, 1000, 3333 at N = 7776,
// K = 7232.  Three kinds of call use a stream-ordered workspace from a pool the library keeps
// per device (cudaMallocFromPoolAsync, no device-wide synchronisation):
//   * shapes whose last wave of tiles is partial take the stream-K schedule (for example the
//     hero's 8-GPU column slab 6464x976, or the LLM projection's 2/4/8-GPU slabs):
//     (1 + K chunks) x 128 x tile width x 4 bytes per CTA of each split tile.  This workspace
//     stays with the stream (up to 16 streams per device) and later launches on that stream
//     reuse it; a launch allocates only when the stream has none as large yet;
//   * skinny shapes the cost model splits along K: K chunks x m x n x 4 bytes, handed back on
//     the same stream after the reduce;
//   * layouts TMA cannot describe (k or n not a multiple of 8, a pointer off a 16-byte
//     boundary): padded copies of A, B and C, handed back the same way.
// The library holds this memory until mo_release_workspace (include/mo_gemm.h).
// mo_launch_bf16_gemm_v1_noalloc allocates nothing at all.

#include <cstdint>

#include <cuda_runtime_api.h>

namespace matmul_optimizer {

bool launch_bf16_gemm_v1(
    const std::uint16_t* a_bf16,
    const std::uint16_t* b_bf16,
    std::uint16_t* c_bf16,
    int m,
    int n,
    int k,
    cudaStream_t stream);

}  // namespace matmul_optimizer
