// Row-sharded multi-GPU GEMM over NCCL (one process per GPU).
//
// Rank r owns rows [row_begin(r), row_begin(r+1)) of A and C, with row_begin(r) =
// floor(M * r / nranks); B is replicated on every rank. Each rank computes its C row block
// with the single-GPU GEMM (hgemm_launch_ex) and the blocks are exchanged so that every
// rank ends with the full C, in place:
//   * equal blocks, one chunk: one in-place ncclAllGather (send = C + row_begin(r)*N);
//   * otherwise: per chunk, grouped ncclSend/ncclRecv of each rank's chunk to every peer.
// With chunks > 1 the exchange of chunk c runs on a communication stream while the GEMM of
// chunk c+1 runs on the caller's stream, so the NVLink transfer overlaps the math.
//
// The reference (yz-wqf/Hopper_GEMM) is single-GPU and has no counterpart for this layer.
// NCCL is resolved at run time from libnccl.so.2, so a process that already loaded NCCL
// (e.g. through torch.distributed) shares that copy instead of pulling in a second one.

#include <cuda_runtime.h>
#include <dlfcn.h>
#include <nccl.h>

#include <algorithm>
#include <cstdint>
#include <cstring>
#include <mutex>
#include <vector>

#include "hgemm_b200.h"

namespace {

struct NcclApi {
  bool ok = false;
  ncclResult_t (*GetUniqueId)(ncclUniqueId *) = nullptr;
  ncclResult_t (*CommInitRank)(ncclComm_t *, int, ncclUniqueId, int) = nullptr;
  ncclResult_t (*CommDestroy)(ncclComm_t) = nullptr;
  ncclResult_t (*CommAbort)(ncclComm_t) = nullptr;
  ncclResult_t (*CommGetAsyncError)(ncclComm_t, ncclResult_t *) = nullptr;
  ncclResult_t (*AllGather)(const void *, void *, size_t, ncclDataType_t, ncclComm_t,
                            cudaStream_t) = nullptr;
  ncclResult_t (*Send)(const void *, size_t, ncclDataType_t, int, ncclComm_t,
                       cudaStream_t) = nullptr;
  ncclResult_t (*Recv)(void *, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
  ncclResult_t (*GroupStart)() = nullptr;
  ncclResult_t (*GroupEnd)() = nullptr;
};

const NcclApi &nccl() {
  static NcclApi api = [] {
    NcclApi a;
    void *h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL | RTLD_NOLOAD);
    if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
    if (!h) return a;
#define HGEMM_SYM(field, name) a.field = reinterpret_cast<decltype(a.field)>(dlsym(h, name))
    HGEMM_SYM(GetUniqueId, "ncclGetUniqueId");
    HGEMM_SYM(CommInitRank, "ncclCommInitRank");
    HGEMM_SYM(CommDestroy, "ncclCommDestroy");
    HGEMM_SYM(CommAbort, "ncclCommAbort");
    HGEMM_SYM(CommGetAsyncError, "ncclCommGetAsyncError");
    HGEMM_SYM(AllGather, "ncclAllGather");
    HGEMM_SYM(Send, "ncclSend");
    HGEMM_SYM(Recv, "ncclRecv");
    HGEMM_SYM(GroupStart, "ncclGroupStart");
    HGEMM_SYM(GroupEnd, "ncclGroupEnd");
#undef HGEMM_SYM
    a.ok = a.GetUniqueId && a.CommInitRank && a.CommDestroy && a.CommAbort &&
           a.CommGetAsyncError && a.AllGather && a.Send && a.Recv && a.GroupStart && a.GroupEnd;
    return a;
  }();
  return api;
}

}  // namespace

struct hgemm_comm_s {
  ncclComm_t comm = nullptr;
  int nranks = 0;
  int rank = 0;
  int device = 0;
  cudaStream_t comm_stream = nullptr;
  std::vector<cudaEvent_t> chunk_done;  // GEMM of chunk c finished (caller stream)
  cudaEvent_t gather_done = nullptr;     // all exchanges finished (comm stream)
};

extern "C" {

int hgemm_shard_rows(int M, int nranks, int rank, int *row_begin, int *row_count) {
  if (M < 0 || nranks <= 0 || rank < 0 || rank >= nranks || !row_begin || !row_count)
    return HGEMM_ERR_INVALID_ARG;
  const long long b = static_cast<long long>(M) * rank / nranks;
  const long long e = static_cast<long long>(M) * (rank + 1) / nranks;
  *row_begin = static_cast<int>(b);
  *row_count = static_cast<int>(e - b);
  return HGEMM_OK;
}

int hgemm_comm_unique_id(void *id_out, size_t id_bytes) {
  if (!id_out || id_bytes < sizeof(ncclUniqueId)) return HGEMM_ERR_INVALID_ARG;
  const NcclApi &a = nccl();
  if (!a.ok) return HGEMM_ERR_NCCL;
  ncclUniqueId id;
  if (a.GetUniqueId(&id) != ncclSuccess) return HGEMM_ERR_NCCL;
  std::memcpy(id_out, &id, sizeof(id));
  return HGEMM_OK;
}

int hgemm_comm_init(hgemm_comm_t *out, int nranks, const void *id, size_t id_bytes, int rank) {
  if (!out || !id || id_bytes < sizeof(ncclUniqueId) || nranks <= 0 || rank < 0 ||
      rank >= nranks)
    return HGEMM_ERR_INVALID_ARG;
  const NcclApi &a = nccl();
  if (!a.ok) return HGEMM_ERR_NCCL;
  hgemm_comm_s *c = new hgemm_comm_s();
  c->nranks = nranks;
  c->rank = rank;
  if (cudaGetDevice(&c->device) != cudaSuccess) {
    delete c;
    return HGEMM_ERR_CUDA;
  }
  ncclUniqueId uid;
  std::memcpy(&uid, id, sizeof(uid));
  if (a.CommInitRank(&c->comm, nranks, uid, rank) != ncclSuccess) {
    delete c;
    return HGEMM_ERR_NCCL;
  }
  if (cudaStreamCreateWithFlags(&c->comm_stream, cudaStreamNonBlocking) != cudaSuccess ||
      cudaEventCreateWithFlags(&c->gather_done, cudaEventDisableTiming) != cudaSuccess) {
    a.CommDestroy(c->comm);
    delete c;
    return HGEMM_ERR_CUDA;
  }
  *out = c;
  return HGEMM_OK;
}

int hgemm_comm_destroy(hgemm_comm_t c) {
  if (!c) return HGEMM_ERR_INVALID_ARG;
  const NcclApi &a = nccl();
  int st = HGEMM_OK;
  if (c->comm_stream) cudaStreamSynchronize(c->comm_stream);
  if (c->comm && a.ok && a.CommDestroy(c->comm) != ncclSuccess) st = HGEMM_ERR_NCCL;
  for (cudaEvent_t e : c->chunk_done) cudaEventDestroy(e);
  if (c->gather_done) cudaEventDestroy(c->gather_done);
  if (c->comm_stream) cudaStreamDestroy(c->comm_stream);
  delete c;
  return st;
}

int hgemm_comm_check(hgemm_comm_t c) {
  if (!c) return HGEMM_ERR_INVALID_ARG;
  const NcclApi &a = nccl();
  if (!a.ok) return HGEMM_ERR_NCCL;
  ncclResult_t r = ncclSuccess;
  if (a.CommGetAsyncError(c->comm, &r) != ncclSuccess) return HGEMM_ERR_NCCL;
  return (r == ncclSuccess || r == ncclInProgress) ? HGEMM_OK : HGEMM_ERR_NCCL;
}

int hgemm_comm_abort(hgemm_comm_t c) {
  if (!c) return HGEMM_ERR_INVALID_ARG;
  const NcclApi &a = nccl();
  int st = HGEMM_OK;
  if (c->comm && a.ok && a.CommAbort(c->comm) != ncclSuccess) st = HGEMM_ERR_NCCL;
  c->comm = nullptr;
  for (cudaEvent_t e : c->chunk_done) cudaEventDestroy(e);
  if (c->gather_done) cudaEventDestroy(c->gather_done);
  if (c->comm_stream) cudaStreamDestroy(c->comm_stream);
  delete c;
  return st;
}

int hgemm_shard_chunk_rows(int rows, int chunks, int chunk, int *begin, int *count) {
  if (rows < 0 || chunks <= 0 || chunk < 0 || chunk >= chunks || !begin || !count)
    return HGEMM_ERR_INVALID_ARG;
  *begin = static_cast<int>(static_cast<long long>(rows) * chunk / chunks);
  *count = static_cast<int>(static_cast<long long>(rows) * (chunk + 1) / chunks) - *begin;
  return HGEMM_OK;
}

int hgemm_sharded_rank(hgemm_comm_t c, const hgemm_half_t *A_local, const hgemm_half_t *B,
                       hgemm_half_t *C, int M, int N, int K, float alpha, float beta, int chunks,
                       hgemm_stream_t stream) {
  if (!c || M < 0 || N < 0 || K < 0) return HGEMM_ERR_INVALID_ARG;
  const NcclApi &a = nccl();
  if (!a.ok) return HGEMM_ERR_NCCL;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const int P = c->nranks, me = c->rank;
  int rb = 0, rc = 0;
  hgemm_shard_rows(M, P, me, &rb, &rc);
  // Every rank must post the same sequence of collectives, so the chunk count may depend
  // only on (M, P, chunks): at most the smallest rank's row count.
  if (chunks < 1) chunks = 1;
  chunks = std::max(1, std::min(chunks, std::max(M / P, 1)));
  const size_t row_elems = static_cast<size_t>(N);

  // Rows [cb, cb + cn) of the rank-local block that make up chunk `ch`.
  auto chunk_rows = [&](int count, int ch, int *cb, int *cn) {
    hgemm_shard_chunk_rows(count, chunks, ch, cb, cn);
  };

  if (M % P == 0 && chunks == 1) {
    int st = HGEMM_OK;
    if (rc > 0)
      st = hgemm_launch_ex(A_local, B, C + static_cast<size_t>(rb) * row_elems, rc, N, K, alpha,
                           beta, stream, 0, 0, 0);
    if (st != HGEMM_OK) return st;
    if (P > 1 && a.AllGather(C + static_cast<size_t>(rb) * row_elems, C,
                             static_cast<size_t>(rc) * row_elems, ncclFloat16, c->comm,
                             s) != ncclSuccess)
      return HGEMM_ERR_NCCL;
    return HGEMM_OK;
  }

  while (static_cast<int>(c->chunk_done.size()) < chunks) {
    cudaEvent_t e;
    if (cudaEventCreateWithFlags(&e, cudaEventDisableTiming) != cudaSuccess) return HGEMM_ERR_CUDA;
    c->chunk_done.push_back(e);
  }
  for (int ch = 0; ch < chunks; ++ch) {
    int cb = 0, cn = 0;
    chunk_rows(rc, ch, &cb, &cn);
    if (cn > 0) {
      const int st = hgemm_launch_ex(A_local + static_cast<size_t>(cb) * K, B,
                                     C + static_cast<size_t>(rb + cb) * row_elems, cn, N, K,
                                     alpha, beta, stream, 0, 0, 0);
      if (st != HGEMM_OK) return st;
    }
    if (P == 1) continue;
    if (cudaEventRecord(c->chunk_done[ch], s) != cudaSuccess ||
        cudaStreamWaitEvent(c->comm_stream, c->chunk_done[ch], 0) != cudaSuccess)
      return HGEMM_ERR_CUDA;
    if (a.GroupStart() != ncclSuccess) return HGEMM_ERR_NCCL;
    bool ok = true;
    for (int peer = 0; peer < P && ok; ++peer) {
      if (peer == me) continue;
      int pb = 0, pc = 0, qb = 0, qn = 0;
      hgemm_shard_rows(M, P, peer, &pb, &pc);
      chunk_rows(pc, ch, &qb, &qn);
      if (cn > 0)
        ok = a.Send(C + static_cast<size_t>(rb + cb) * row_elems,
                    static_cast<size_t>(cn) * row_elems, ncclFloat16, peer, c->comm,
                    c->comm_stream) == ncclSuccess;
      if (ok && qn > 0)
        ok = a.Recv(C + static_cast<size_t>(pb + qb) * row_elems,
                    static_cast<size_t>(qn) * row_elems, ncclFloat16, peer, c->comm,
                    c->comm_stream) == ncclSuccess;
    }
    if (a.GroupEnd() != ncclSuccess || !ok) return HGEMM_ERR_NCCL;
  }
  if (P > 1) {
    if (cudaEventRecord(c->gather_done, c->comm_stream) != cudaSuccess ||
        cudaStreamWaitEvent(s, c->gather_done, 0) != cudaSuccess)
      return HGEMM_ERR_CUDA;
  }
  return HGEMM_OK;
}

}  // extern "C"
