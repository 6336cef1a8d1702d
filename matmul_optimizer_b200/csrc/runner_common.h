#pragma once
// The GEMM backend a runner executable drives.  runner_main.cpp implements the reference's
// runner contract (src/runner/main.cpp) once; it is linked either against libmo_gemm.so
// (custom_runner: backend = matmul_optimizer::launch_bf16_gemm_v1) or against cuBLASLt
// (cublas_runner: the same-box library baseline, cublas_runner.cpp).

#include <cstdint>

#include <cuda_runtime_api.h>

namespace mo_runner {

// C[m,n] = A[m,k] · B[k,n], row-major BF16 bits, device pointers on the current device,
// asynchronous on `stream`.  Returns false on any failure.
bool backend_gemm(const std::uint16_t* a, const std::uint16_t* b, std::uint16_t* c, int m,
                  int n, int k, cudaStream_t stream);

// Column slabs of one N-sharded GEMM, slab i on devices[i] and streams[i]:
// c[i][m, widths[i]] = a[i][m, k] · b[i][k, widths[i]]; slabs of width 0 are skipped.
// custom_runner issues them with the library's multi-device entry mo_gemm_nshard; cublas_runner
// issues one cuBLASLt call per slab.  Returns false on any failure.
bool backend_gemm_shards(int g, const int* devices, const std::uint16_t* const* a,
                         const std::uint16_t* const* b, std::uint16_t* const* c, int m, int k,
                         const int* widths, cudaStream_t const* streams);

// Short name written into the result JSON ("mo_sm100" or "cublaslt").
const char* backend_name();

}  // namespace mo_runner
