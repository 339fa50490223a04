// cuBLAS comparator used by bench.py and the GPU tests (not part of the GEMM product).
// Issues exactly the call the reference's harnesses time and check against
// (three_way.cu:75,88; check_all.cu:60): row-major C = alpha*A@B + beta*C computed as the
// column-major C^T = B^T A^T with cublasGemmEx(N, N, N, M, K, ..., CUBLAS_COMPUTE_32F,
// CUBLAS_GEMM_DEFAULT), fp16 operands and output.
#include <cublas_v2.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <mutex>

namespace {
std::mutex g_mu;
cublasHandle_t g_handle[64] = {};
}  // namespace

extern "C" int hgemm_cublas_ref(const __half *A, const __half *B, __half *C, int M, int N, int K,
                                float alpha, float beta, cudaStream_t stream) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 2;
  cublasHandle_t h;
  {
    std::lock_guard<std::mutex> lock(g_mu);
    if (!g_handle[dev] && cublasCreate(&g_handle[dev]) != CUBLAS_STATUS_SUCCESS) return 2;
    h = g_handle[dev];
  }
  if (cublasSetStream(h, stream) != CUBLAS_STATUS_SUCCESS) return 2;
  const cublasStatus_t s =
      cublasGemmEx(h, CUBLAS_OP_N, CUBLAS_OP_N, N, M, K, &alpha, B, CUDA_R_16F, N, A, CUDA_R_16F,
                   K, &beta, C, CUDA_R_16F, N, CUBLAS_COMPUTE_32F, CUBLAS_GEMM_DEFAULT);
  return s == CUBLAS_STATUS_SUCCESS ? 0 : 5;
}
