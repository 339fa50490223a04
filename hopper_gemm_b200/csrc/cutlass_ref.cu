// CUTLASS SM100 comparator: the third column of the shape grid and a second numerical
// cross-check in the GPU tests (not part of the GEMM product). The reference kept a CUTLASS
// build of the same contract beside its own kernel and cuBLAS (mma_half_cutlass.cu, the
// "3-way" table of three_way.cu); this is the B200 counterpart, instantiated from CUTLASS's
// SM100 CollectiveBuilder: row-major A (M x K), row-major B (K x N), row-major C updated in
// place as C = alpha * A @ B + beta * C, fp16 operands and output, fp32 accumulation.
//
// Kernel choice: 1-SM UMMA (tcgen05.mma cta_group::1), 128 x 256 x 64 tiles, cluster 1 x 1 x 1,
// so its operand loads are plain per-CTA TMA tile loads, like every load in this repository
// (whose multi-GPU jobs must not carry loads shared across a cluster). The library owns one grow-only
// workspace per device for CUTLASS's tile scheduler.
#include <cuda_runtime.h>

#include <mutex>

#include "cute/tensor.hpp"
#include "cutlass/cutlass.h"
#include "cutlass/epilogue/collective/collective_builder.hpp"
#include "cutlass/gemm/collective/collective_builder.hpp"
#include "cutlass/gemm/device/gemm_universal_adapter.h"
#include "cutlass/gemm/dispatch_policy.hpp"
#include "cutlass/gemm/kernel/gemm_universal.hpp"
#include "cutlass/util/packed_stride.hpp"

namespace {
using namespace cute;

using ElementAB = cutlass::half_t;
using ElementC = cutlass::half_t;
using ElementAcc = float;
using LayoutA = cutlass::layout::RowMajor;
using LayoutB = cutlass::layout::RowMajor;
using LayoutC = cutlass::layout::RowMajor;
constexpr int kAlign = 8;  // 16-byte aligned rows (the TMA path's requirement)

using TileShape = Shape<_128, _256, _64>;
using ClusterShape = Shape<_1, _1, _1>;

using CollectiveEpilogue = typename cutlass::epilogue::collective::CollectiveBuilder<
    cutlass::arch::Sm100, cutlass::arch::OpClassTensorOp, TileShape, ClusterShape,
    cutlass::epilogue::collective::EpilogueTileAuto, ElementAcc, ElementAcc, ElementC, LayoutC,
    kAlign, ElementC, LayoutC, kAlign,
    cutlass::epilogue::TmaWarpSpecialized1Sm>::CollectiveOp;

using CollectiveMainloop = typename cutlass::gemm::collective::CollectiveBuilder<
    cutlass::arch::Sm100, cutlass::arch::OpClassTensorOp, ElementAB, LayoutA, kAlign, ElementAB,
    LayoutB, kAlign, ElementAcc, TileShape, ClusterShape,
    cutlass::gemm::collective::StageCountAutoCarveout<static_cast<int>(
        sizeof(typename CollectiveEpilogue::SharedStorage))>,
    cutlass::gemm::KernelTmaWarpSpecialized1SmSm100>::CollectiveOp;

using GemmKernel = cutlass::gemm::kernel::GemmUniversal<Shape<int, int, int, int>,
                                                        CollectiveMainloop, CollectiveEpilogue>;
using Gemm = cutlass::gemm::device::GemmUniversalAdapter<GemmKernel>;

std::mutex g_mu;
void *g_ws[64] = {};
size_t g_ws_bytes[64] = {};
}  // namespace

// Returns 0 on success, 1 for unsupported arguments (pointers or row lengths not 16-byte
// aligned), 2 for CUDA errors, 5 for a CUTLASS launch failure.
extern "C" int hgemm_cutlass_ref(const __half *A, const __half *B, __half *C, int M, int N,
                                 int K, float alpha, float beta, cudaStream_t stream) {
  if (M <= 0 || N <= 0 || K <= 0) return 1;
  if (K % kAlign || N % kAlign) return 1;
  if ((reinterpret_cast<uintptr_t>(A) | reinterpret_cast<uintptr_t>(B) |
       reinterpret_cast<uintptr_t>(C)) % 16)
    return 1;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 2;

  using StrideA = typename Gemm::GemmKernel::StrideA;
  using StrideB = typename Gemm::GemmKernel::StrideB;
  using StrideC = typename Gemm::GemmKernel::StrideC;
  using StrideD = typename Gemm::GemmKernel::StrideD;
  const StrideA sa = cutlass::make_cute_packed_stride(StrideA{}, make_shape(M, K, 1));
  const StrideB sb = cutlass::make_cute_packed_stride(StrideB{}, make_shape(N, K, 1));
  const StrideC sc = cutlass::make_cute_packed_stride(StrideC{}, make_shape(M, N, 1));
  const StrideD sd = cutlass::make_cute_packed_stride(StrideD{}, make_shape(M, N, 1));

  typename Gemm::Arguments args{
      cutlass::gemm::GemmUniversalMode::kGemm,
      {M, N, K, 1},
      {reinterpret_cast<const ElementAB *>(A), sa, reinterpret_cast<const ElementAB *>(B), sb},
      {{alpha, beta},
       reinterpret_cast<const ElementC *>(C), sc, reinterpret_cast<ElementC *>(C), sd}};

  Gemm gemm;
  if (gemm.can_implement(args) != cutlass::Status::kSuccess) return 1;
  const size_t ws = Gemm::get_workspace_size(args);
  void *wsp = nullptr;
  {
    std::lock_guard<std::mutex> lock(g_mu);
    if (ws > g_ws_bytes[dev]) {
      if (g_ws[dev]) cudaFree(g_ws[dev]);
      g_ws[dev] = nullptr;
      g_ws_bytes[dev] = 0;
      if (cudaMalloc(&g_ws[dev], ws) != cudaSuccess) return 2;
      g_ws_bytes[dev] = ws;
    }
    wsp = g_ws[dev];
  }
  if (gemm.initialize(args, wsp, stream) != cutlass::Status::kSuccess) return 5;
  if (gemm.run(stream) != cutlass::Status::kSuccess) return 5;
  return 0;
}
