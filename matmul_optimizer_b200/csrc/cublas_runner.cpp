// cuBLASLt backend for the runner: BF16 inputs, FP32 compute, BF16 output, row-major
// operands through the transposed problem (C^T[n,m] = B^T[n,k] · A^T[k,m] in column-major
// terms, so no data is transposed).  This is the same-box library baseline that replaces
// the reference's CUTLASS Sm80 runner (src/runner/cutlass_main.cu:52-78, :515-539), whose
// CUTLASS 2.x kernels have no sm_100 path.

#include <cublasLt.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <map>
#include <mutex>
#include <tuple>

#include "runner_common.h"

namespace mo_runner {
namespace {

constexpr size_t kWorkspaceBytes = 64ull << 20;

struct DeviceLt {
  cublasLtHandle_t handle = nullptr;
  void* workspace = nullptr;
};

std::mutex g_mutex;
std::map<int, DeviceLt> g_devices;

struct PlanKey {
  int dev, m, n, k;
  bool operator<(const PlanKey& o) const {
    return std::tie(dev, m, n, k) < std::tie(o.dev, o.m, o.n, o.k);
  }
};

struct Plan {
  cublasLtMatmulDesc_t op = nullptr;
  cublasLtMatrixLayout_t a = nullptr, b = nullptr, c = nullptr;
  cublasLtMatmulAlgo_t algo{};
  bool ok = false;
};

std::map<PlanKey, Plan> g_plans;

DeviceLt* device_lt(int dev) {
  auto it = g_devices.find(dev);
  if (it != g_devices.end()) return &it->second;
  DeviceLt d;
  if (cublasLtCreate(&d.handle) != CUBLAS_STATUS_SUCCESS) return nullptr;
  if (cudaMalloc(&d.workspace, kWorkspaceBytes) != cudaSuccess) return nullptr;
  return &(g_devices[dev] = d);
}

Plan* get_plan(int dev, DeviceLt* lt, int m, int n, int k) {
  const PlanKey key{dev, m, n, k};
  auto it = g_plans.find(key);
  if (it != g_plans.end()) return it->second.ok ? &it->second : nullptr;
  Plan p;
  // Column-major view: D[n, m] = Bcm[n, k] · Acm[k, m].
  cublasLtMatmulDescCreate(&p.op, CUBLAS_COMPUTE_32F, CUDA_R_32F);
  cublasOperation_t t = CUBLAS_OP_N;
  cublasLtMatmulDescSetAttribute(p.op, CUBLASLT_MATMUL_DESC_TRANSA, &t, sizeof(t));
  cublasLtMatmulDescSetAttribute(p.op, CUBLASLT_MATMUL_DESC_TRANSB, &t, sizeof(t));
  cublasLtMatrixLayoutCreate(&p.a, CUDA_R_16BF, n, k, n);
  cublasLtMatrixLayoutCreate(&p.b, CUDA_R_16BF, k, m, k);
  cublasLtMatrixLayoutCreate(&p.c, CUDA_R_16BF, n, m, n);
  cublasLtMatmulPreference_t pref = nullptr;
  cublasLtMatmulPreferenceCreate(&pref);
  size_t ws = kWorkspaceBytes;
  cublasLtMatmulPreferenceSetAttribute(pref, CUBLASLT_MATMUL_PREF_MAX_WORKSPACE_BYTES, &ws,
                                       sizeof(ws));
  cublasLtMatmulHeuristicResult_t res{};
  int found = 0;
  if (cublasLtMatmulAlgoGetHeuristic(lt->handle, p.op, p.a, p.b, p.c, p.c, pref, 1, &res,
                                     &found) == CUBLAS_STATUS_SUCCESS &&
      found > 0) {
    p.algo = res.algo;
    p.ok = true;
  }
  cublasLtMatmulPreferenceDestroy(pref);
  auto& slot = (g_plans[key] = p);
  return slot.ok ? &slot : nullptr;
}

}  // namespace

bool backend_gemm(const std::uint16_t* a, const std::uint16_t* b, std::uint16_t* c, int m,
                  int n, int k, cudaStream_t stream) {
  if (a == nullptr || b == nullptr || c == nullptr || m <= 0 || n <= 0 || k <= 0) return false;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return false;
  std::lock_guard<std::mutex> lock(g_mutex);
  DeviceLt* lt = device_lt(dev);
  if (lt == nullptr) return false;
  Plan* p = get_plan(dev, lt, m, n, k);
  if (p == nullptr) return false;
  const float alpha = 1.0f, beta = 0.0f;
  const cublasStatus_t st =
      cublasLtMatmul(lt->handle, p->op, &alpha, b, p->a, a, p->b, &beta, c, p->c, c, p->c,
                     &p->algo, lt->workspace, kWorkspaceBytes, stream);
  return st == CUBLAS_STATUS_SUCCESS;
}

bool backend_gemm_shards(int g, const int* devices, const std::uint16_t* const* a,
                         const std::uint16_t* const* b, std::uint16_t* const* c, int m, int k,
                         const int* widths, cudaStream_t const* streams) {
  int prev = 0;
  if (cudaGetDevice(&prev) != cudaSuccess) return false;
  bool ok = true;
  for (int i = 0; i < g && ok; ++i) {
    if (widths[i] == 0) continue;
    ok = cudaSetDevice(devices[i]) == cudaSuccess &&
         backend_gemm(a[i], b[i], c[i], m, widths[i], k, streams[i]);
  }
  cudaSetDevice(prev);
  return ok;
}

const char* backend_name() { return "cublaslt"; }

}  // namespace mo_runner
