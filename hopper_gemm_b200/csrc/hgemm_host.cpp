// Host-buffer GEMM: the PCIe copies of a GEMM whose operands live in host memory, overlapped
// with the GEMM itself.
//
// A caller whose A, B and C are in (page-locked) host memory would otherwise copy A and B in,
// run the GEMM and copy C out, one after the other; on a B200 at 8192^3 the 384 MiB of copies
// take ~7 ms against ~0.7 ms of math. hgemm_launch_host splits the rows of A and C into
// blocks: B goes first (every row block needs all of it), then each block of A (and of C when
// beta != 0) on a copy-in stream; the GEMM of block i runs on the caller's stream as soon as
// block i has landed, and block i of C goes back on a copy-out stream as soon as its GEMM is
// done. Copies in both directions and the math then overlap, and a call costs about the
// host-to-device bytes at PCIe speed plus one block's GEMM and copy-out.
//
// Every block is the GEMM of its rows on row-offset pointers with split-K ruled out, so each
// element of C is summed in the same k order, and rounded the same way, as in one hgemm_launch
// of the whole GEMM: the result is bit-identical to it. Problems that hgemm_launch itself would
// split along K (a few tiles, long K) run as one block, and so do shapes whose B or C need the
// restride copy (N % 8 != 0), so that B is restrided once. Row blocks start on multiples of 256
// rows (the pair tile height), which keeps every block's A and C pointers 16-byte aligned.
//
// No counterpart in the reference (its solve() takes device pointers).

#include <cuda_runtime.h>

#include <algorithm>
#include <mutex>

#include "hgemm_b200.h"

// Defined in hgemm_sm100.cu, not part of the public header.
extern "C" __attribute__((visibility("hidden"))) int hgemm_internal_launch_unsplit(
    const hgemm_half_t *A, const hgemm_half_t *B, hgemm_half_t *C, int M, int N, int K,
    float alpha, float beta, hgemm_stream_t stream, int sm_limit);
extern "C" __attribute__((visibility("hidden"))) int hgemm_internal_plan_current(
    const hgemm_half_t *A, const hgemm_half_t *B, const hgemm_half_t *C, int M, int N, int K,
    float beta, hgemm_plan_t *out);

namespace {

constexpr int kMaxBlocks = 8;
constexpr int kBlockRowAlign = 256;
constexpr int kMinBlockRows = 1024;

struct HostPipe {
  bool init = false;
  cudaStream_t in = nullptr, out = nullptr;
  cudaEvent_t start = nullptr, b_in = nullptr, done = nullptr;
  cudaEvent_t blk_in[kMaxBlocks] = {}, blk_gemm[kMaxBlocks] = {};
};

std::mutex g_host_mu;
HostPipe g_pipe[64];

bool make_pipe(HostPipe &p) {
  if (p.init) return true;
  const unsigned fl = cudaEventDisableTiming;
  bool ok = cudaStreamCreateWithFlags(&p.in, cudaStreamNonBlocking) == cudaSuccess &&
            cudaStreamCreateWithFlags(&p.out, cudaStreamNonBlocking) == cudaSuccess &&
            cudaEventCreateWithFlags(&p.start, fl) == cudaSuccess &&
            cudaEventCreateWithFlags(&p.b_in, fl) == cudaSuccess &&
            cudaEventCreateWithFlags(&p.done, fl) == cudaSuccess;
  for (int i = 0; ok && i < kMaxBlocks; ++i)
    ok = cudaEventCreateWithFlags(&p.blk_in[i], fl) == cudaSuccess &&
         cudaEventCreateWithFlags(&p.blk_gemm[i], fl) == cudaSuccess;
  if (!ok) {
    cudaGetLastError();
    return false;
  }
  p.init = true;
  return true;
}

// Number of row blocks: about one per kMinBlockRows rows, at most kMaxBlocks.
int row_blocks(int M, int N) {
  if (N % 8 != 0) return 1;
  return std::max(1, std::min(kMaxBlocks, M / kMinBlockRows));
}

}  // namespace

extern "C" int hgemm_launch_host(const hgemm_half_t *A_h, const hgemm_half_t *B_h,
                                 hgemm_half_t *C_h, hgemm_half_t *dA, hgemm_half_t *dB,
                                 hgemm_half_t *dC, int M, int N, int K, float alpha, float beta,
                                 hgemm_stream_t stream) {
  if (M < 0 || N < 0 || K < 0) return HGEMM_ERR_INVALID_ARG;
  if (M == 0 || N == 0) return HGEMM_OK;
  if (!A_h || !B_h || !C_h || !dA || !dB || !dC) return HGEMM_ERR_INVALID_ARG;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return HGEMM_ERR_CUDA;
  std::lock_guard<std::mutex> lk(g_host_mu);
  HostPipe &p = g_pipe[dev];
  if (!make_pipe(p)) return HGEMM_ERR_CUDA;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);

  int nb = row_blocks(M, N);
  if (nb > 1) {
    // One block when the whole GEMM would be split along K: row blocks could then not
    // reproduce its summation order.
    hgemm_plan_t whole;
    if (hgemm_internal_plan_current(dA, dB, dC, M, N, K, beta, &whole) != HGEMM_OK ||
        whole.ksplit > 1)
      nb = 1;
  }
  int bounds[kMaxBlocks + 1];
  {
    // Equal blocks rounded up to kBlockRowAlign rows; the last one takes the rest.
    const int per = ((M + nb - 1) / nb + kBlockRowAlign - 1) / kBlockRowAlign * kBlockRowAlign;
    for (int i = 0; i <= nb; ++i) bounds[i] = std::min(M, i * per);
    bounds[nb] = M;
  }
  const size_t h = sizeof(hgemm_half_t);
  bool ok = true;
  auto chk = [&](cudaError_t e) {
    if (e != cudaSuccess) ok = false;
  };

  // Nothing starts before the work already queued on the caller's stream.
  chk(cudaEventRecord(p.start, s));
  chk(cudaStreamWaitEvent(p.in, p.start, 0));
  chk(cudaStreamWaitEvent(p.out, p.start, 0));
  if (ok && K > 0)
    chk(cudaMemcpyAsync(dB, B_h, static_cast<size_t>(K) * N * h, cudaMemcpyHostToDevice, p.in));
  if (ok) chk(cudaEventRecord(p.b_in, p.in));
  for (int i = 0; i < nb && ok; ++i) {
    const size_t r0 = static_cast<size_t>(bounds[i]);
    const size_t rows = static_cast<size_t>(bounds[i + 1]) - r0;
    if (rows > 0 && K > 0)
      chk(cudaMemcpyAsync(dA + r0 * K, A_h + r0 * K, rows * K * h, cudaMemcpyHostToDevice, p.in));
    if (rows > 0 && beta != 0.0f)
      chk(cudaMemcpyAsync(dC + r0 * N, C_h + r0 * N, rows * N * h, cudaMemcpyHostToDevice, p.in));
    chk(cudaEventRecord(p.blk_in[i], p.in));
  }

  int st = HGEMM_OK;
  if (ok) chk(cudaStreamWaitEvent(s, p.b_in, 0));
  for (int i = 0; i < nb && ok && st == HGEMM_OK; ++i) {
    const size_t r0 = static_cast<size_t>(bounds[i]);
    const int rows = bounds[i + 1] - bounds[i];
    chk(cudaStreamWaitEvent(s, p.blk_in[i], 0));
    if (rows > 0)
      st = nb == 1 ? hgemm_launch(dA, dB, dC, rows, N, K, alpha, beta, stream)
                   : hgemm_internal_launch_unsplit(dA + r0 * K, dB, dC + r0 * N, rows, N, K,
                                                   alpha, beta, stream, 0);
    chk(cudaEventRecord(p.blk_gemm[i], s));
    chk(cudaStreamWaitEvent(p.out, p.blk_gemm[i], 0));
    if (rows > 0)
      chk(cudaMemcpyAsync(C_h + r0 * N, dC + r0 * N, static_cast<size_t>(rows) * N * h,
                          cudaMemcpyDeviceToHost, p.out));
  }
  // The call is complete when the caller's stream passes this point, whatever happened
  // above: both copy streams are joined back into it.
  const bool joined = cudaEventRecord(p.done, p.out) == cudaSuccess &&
                      cudaStreamWaitEvent(s, p.done, 0) == cudaSuccess &&
                      cudaEventRecord(p.start, p.in) == cudaSuccess &&
                      cudaStreamWaitEvent(s, p.start, 0) == cudaSuccess;
  if (!ok || !joined) {
    cudaGetLastError();
    return HGEMM_ERR_CUDA;
  }
  return st;
}
