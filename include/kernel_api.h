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
