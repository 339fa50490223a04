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
// Fused path: once every rank has registered its C buffer (hgemm_comm_register_output, which
// maps the peers' buffers into this process through CUDA IPC), hgemm_sharded_rank runs ONE
// kernel per rank whose epilogue TMA-stores every finished C tile into the local C and copies
// it into each peer's C over NVLink with 16-byte stores, tile by tile while the math goes on.
// Two epochs per step keep the ranks in order, both exchanged through flag arrays mapped the
// same way (release stores / acquire loads at system scope, bounded waits):
//   * entry: the kernel announces the step to every peer when it starts, and its epilogue
//     stores into a peer's C only once that peer has announced the step too, i.e. once the
//     peer's stream has passed everything queued before this step (its readers of C);
//   * exit: a one-warp barrier kernel after the GEMM, so every rank's C is complete before
//     anything queued after the call runs.
// No NCCL call is made on this path.
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

// GEMM that never uses split-K (hgemm_sm100.cu; internal to this library).
extern "C" __attribute__((visibility("hidden"))) int hgemm_internal_launch_unsplit(
    const hgemm_half_t *A, const hgemm_half_t *B, hgemm_half_t *C, int M, int N, int K,
    float alpha, float beta, hgemm_stream_t stream, int sm_limit);
// Cross-GPU flag barrier, step exit (entry = 0) or entry (entry = 1) (hgemm_sm100.cu;
// internal to this library).
extern "C" __attribute__((visibility("hidden"))) int hgemm_internal_peer_barrier(
    unsigned long long *const *flags, int rank, int nranks, unsigned long long epoch,
    int entry, hgemm_stream_t stream);
// Peer-store GEMM gated on the peers' step-entry epochs (hgemm_sm100.cu; internal).
extern "C" __attribute__((visibility("hidden"))) int hgemm_internal_launch_peers_gated(
    const hgemm_half_t *A, const hgemm_half_t *B, hgemm_half_t *C, int M, int N, int K,
    float alpha, float beta, hgemm_stream_t stream, hgemm_half_t *const *peer_C, int npeers,
    unsigned long long *const *post, const unsigned long long *const *wait,
    unsigned long long epoch);

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
  ncclResult_t (*AllReduce)(const void *, void *, size_t, ncclDataType_t, ncclRedOp_t,
                            ncclComm_t, cudaStream_t) = nullptr;
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
    HGEMM_SYM(AllReduce, "ncclAllReduce");
    HGEMM_SYM(GroupStart, "ncclGroupStart");
    HGEMM_SYM(GroupEnd, "ncclGroupEnd");
#undef HGEMM_SYM
    a.ok = a.GetUniqueId && a.CommInitRank && a.CommDestroy && a.CommAbort &&
           a.CommGetAsyncError && a.AllGather && a.Send && a.Recv && a.AllReduce &&
           a.GroupStart && a.GroupEnd;
    return a;
  }();
  return api;
}

constexpr int kDefaultReservedSms = 16;
constexpr int kMaxRanks = 8;  // the fused path stores to at most 7 peers
// Each rank's flag array: [0, kMaxRanks) the last step each rank finished (exit epochs),
// [kMaxRanks, 2 kMaxRanks) the last step each rank entered (entry epochs).
constexpr int kFlagWords = 2 * kMaxRanks;

// Start and size of the allocation that contains `p` (driver entry point, no -lcuda).
bool allocation_range(const void *p, char **base, size_t *size) {
  using Fn = int (*)(unsigned long long *, size_t *, unsigned long long);
  static Fn fn = [] {
    void *ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuMemGetAddressRange", &ptr, 12000, cudaEnableDefault,
                                         &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      ptr = nullptr;
    return reinterpret_cast<Fn>(ptr);
  }();
  unsigned long long b = 0;
  if (!fn || fn(&b, size, reinterpret_cast<unsigned long long>(p)) != 0) return false;
  *base = reinterpret_cast<char *>(b);
  return true;
}

// What each rank publishes about its registered C buffer and its barrier flags.
struct OutputRecord {
  cudaIpcMemHandle_t handle;
  cudaIpcMemHandle_t flags_handle;
  unsigned long long offset;  // C - allocation start
  unsigned long long bytes;
  int ok;
  int pad;
};

}  // namespace

struct hgemm_comm_s {
  ncclComm_t comm = nullptr;
  int nranks = 0;
  int rank = 0;
  int device = 0;
  int sm_count = 0;
  // SMs the chunk GEMMs leave free while chunks are exchanged, so that the collective's
  // kernels run next to the GEMM instead of waiting for its persistent CTAs to exit.
  int reserved_sms = kDefaultReservedSms;
  cudaStream_t comm_stream = nullptr;
  std::vector<cudaEvent_t> chunk_done;  // GEMM of chunk c finished (caller stream)
  cudaEvent_t gather_done = nullptr;     // all exchanges finished (comm stream)
  // Fused path state.
  int *barrier_word = nullptr;              // device int for the registration all-reduce
  unsigned long long *flags = nullptr;      // [kFlagWords] step epochs announced by each rank
  unsigned long long epoch = 0;             // fused steps issued by this rank
  std::vector<void *> peer_flags_base;      // [nranks] IPC mappings of the peers' flags
  std::vector<unsigned long long *> peer_flags;
  OutputRecord *records_dev = nullptr;      // [nranks] gathered OutputRecords
  hgemm_half_t *out_C = nullptr;            // this rank's registered C
  size_t out_bytes = 0;
  std::vector<void *> peer_base;            // [nranks] IPC mappings (nullptr for self)
  std::vector<hgemm_half_t *> peer_C;       // [nranks] peers' registered C in this process
};

namespace {
void unmap_outputs(hgemm_comm_s *c) {
  for (void *b : c->peer_base)
    if (b) cudaIpcCloseMemHandle(b);
  for (void *b : c->peer_flags_base)
    if (b) cudaIpcCloseMemHandle(b);
  c->peer_base.clear();
  c->peer_C.clear();
  c->peer_flags_base.clear();
  c->peer_flags.clear();
  c->out_C = nullptr;
  c->out_bytes = 0;
}
void free_fused_state(hgemm_comm_s *c) {
  unmap_outputs(c);
  if (c->barrier_word) cudaFree(c->barrier_word);
  if (c->records_dev) cudaFree(c->records_dev);
  if (c->flags) cudaFree(c->flags);
  c->flags = nullptr;
  c->barrier_word = nullptr;
  c->records_dev = nullptr;
}
}  // namespace

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
  if (cudaGetDevice(&c->device) != cudaSuccess ||
      cudaDeviceGetAttribute(&c->sm_count, cudaDevAttrMultiProcessorCount, c->device) !=
          cudaSuccess) {
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
      cudaEventCreateWithFlags(&c->gather_done, cudaEventDisableTiming) != cudaSuccess ||
      cudaMalloc(&c->barrier_word, sizeof(int)) != cudaSuccess ||
      cudaMalloc(&c->records_dev, sizeof(OutputRecord) * nranks) != cudaSuccess ||
      cudaMalloc(&c->flags, sizeof(unsigned long long) * kFlagWords) != cudaSuccess ||
      cudaMemset(c->flags, 0, sizeof(unsigned long long) * kFlagWords) != cudaSuccess ||
      cudaMemset(c->barrier_word, 0, sizeof(int)) != cudaSuccess) {
    free_fused_state(c);
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
  free_fused_state(c);
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
  free_fused_state(c);
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

int hgemm_comm_register_output(hgemm_comm_t c, hgemm_half_t *C, size_t bytes) {
  if (!c || (C == nullptr) != (bytes == 0)) return HGEMM_ERR_INVALID_ARG;
  const NcclApi &a = nccl();
  if (!a.ok || !c->comm) return HGEMM_ERR_NCCL;
  const int P = c->nranks, me = c->rank;
  if (cudaStreamSynchronize(c->comm_stream) != cudaSuccess) return HGEMM_ERR_CUDA;
  unmap_outputs(c);
  // Every rank takes part in both collectives below, whatever happened locally, so that the
  // ranks stay in step; the outcome is agreed on with a MIN all-reduce.
  OutputRecord mine;
  std::memset(&mine, 0, sizeof(mine));
  char *base = nullptr;
  size_t size = 0;
  if (C && P <= kMaxRanks && reinterpret_cast<uintptr_t>(C) % 16 == 0 &&
      allocation_range(C, &base, &size) && cudaIpcGetMemHandle(&mine.handle, base) == cudaSuccess &&
      cudaIpcGetMemHandle(&mine.flags_handle, c->flags) == cudaSuccess) {
    mine.offset = static_cast<unsigned long long>(reinterpret_cast<char *>(C) - base);
    mine.bytes = bytes;
    mine.ok = (mine.offset + bytes <= size) ? 1 : 0;
  }
  cudaGetLastError();
  std::vector<OutputRecord> all(P);
  bool ok = cudaMemcpy(c->records_dev + me, &mine, sizeof(mine), cudaMemcpyHostToDevice) ==
                cudaSuccess &&
            a.AllGather(c->records_dev + me, c->records_dev, sizeof(OutputRecord), ncclUint8,
                        c->comm, c->comm_stream) == ncclSuccess &&
            cudaStreamSynchronize(c->comm_stream) == cudaSuccess &&
            cudaMemcpy(all.data(), c->records_dev, sizeof(OutputRecord) * P,
                       cudaMemcpyDeviceToHost) == cudaSuccess;
  int local_ok = ok ? 1 : 0;
  c->peer_base.assign(P, nullptr);
  c->peer_C.assign(P, nullptr);
  c->peer_flags_base.assign(P, nullptr);
  c->peer_flags.assign(P, nullptr);
  c->peer_flags[me] = c->flags;
  for (int r = 0; r < P && local_ok; ++r) {
    if (!all[r].ok || all[r].bytes != bytes) local_ok = 0;
    if (r == me || !local_ok) continue;
    void *pb = nullptr;
    if (cudaIpcOpenMemHandle(&pb, all[r].handle, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
      cudaGetLastError();
      local_ok = 0;
      break;
    }
    c->peer_base[r] = pb;
    c->peer_C[r] = reinterpret_cast<hgemm_half_t *>(static_cast<char *>(pb) + all[r].offset);
    void *fb = nullptr;
    if (cudaIpcOpenMemHandle(&fb, all[r].flags_handle, cudaIpcMemLazyEnablePeerAccess) !=
        cudaSuccess) {
      cudaGetLastError();
      local_ok = 0;
      break;
    }
    c->peer_flags_base[r] = fb;
    c->peer_flags[r] = static_cast<unsigned long long *>(fb);
  }
  if (!C) local_ok = 0;
  int agreed = 0;
  ok = cudaMemcpy(c->barrier_word, &local_ok, sizeof(int), cudaMemcpyHostToDevice) ==
           cudaSuccess &&
       a.AllReduce(c->barrier_word, c->barrier_word, 1, ncclInt32, ncclMin, c->comm,
                   c->comm_stream) == ncclSuccess &&
       cudaStreamSynchronize(c->comm_stream) == cudaSuccess &&
       cudaMemcpy(&agreed, c->barrier_word, sizeof(int), cudaMemcpyDeviceToHost) == cudaSuccess;
  if (!ok || !agreed) {
    unmap_outputs(c);
    if (!ok) return HGEMM_ERR_NCCL;
    return C ? HGEMM_ERR_CUDA : HGEMM_OK;
  }
  c->out_C = C;
  c->out_bytes = bytes;
  return HGEMM_OK;
}

int hgemm_comm_output_ptr(hgemm_comm_t c, int r, hgemm_half_t **out) {
  if (!c || !out || r < 0 || r >= c->nranks) return HGEMM_ERR_INVALID_ARG;
  if (!c->out_C) return HGEMM_ERR_INVALID_ARG;
  *out = (r == c->rank) ? c->out_C : c->peer_C[r];
  return HGEMM_OK;
}

int hgemm_comm_set_reserved_sms(hgemm_comm_t c, int sms) {
  if (!c || sms < 0 || sms >= c->sm_count) return HGEMM_ERR_INVALID_ARG;
  c->reserved_sms = sms;
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

  if (c->out_C && C == c->out_C && M % P == 0 && P > 1 &&
      static_cast<size_t>(M) * N * sizeof(hgemm_half_t) <= c->out_bytes) {
    // Fused path: one kernel computes this rank's rows and stores each tile into every
    // peer's C as well, gated on the peers' entry epochs; the exit barrier follows whatever
    // happened locally, so that the ranks' flag sequences stay the same.
    const unsigned long long ep = ++c->epoch;
    hgemm_half_t *peers[kMaxRanks];
    unsigned long long *post[kMaxRanks];
    const unsigned long long *wait[kMaxRanks];
    int n = 0;
    for (int r = 0; r < P; ++r) {
      if (r == me) continue;
      peers[n] = c->peer_C[r] + static_cast<size_t>(rb) * row_elems;
      post[n] = c->peer_flags[r] + kMaxRanks + me;  // peer r's entry flag for this rank
      wait[n] = c->flags + kMaxRanks + r;            // this rank's entry flag for peer r
      ++n;
    }
    hgemm_half_t *Cl = C + static_cast<size_t>(rb) * row_elems;
    int st = HGEMM_OK;
    bool entered = false;
    if (rc > 0) {
      st = hgemm_internal_launch_peers_gated(A_local, B, Cl, rc, N, K, alpha, beta, stream,
                                             peers, n, post, wait, ep);
      entered = st == HGEMM_OK;  // the kernel itself announced and waited for the entry
      if (st == HGEMM_ERR_NOT_FUSABLE) {
        // Shapes without TMA stores: compute locally, then an entry barrier (no peer may
        // still be reading its C), then push the rows with copies.
        st = hgemm_internal_launch_unsplit(A_local, B, Cl, rc, N, K, alpha, beta, stream, 0);
        const int est = hgemm_internal_peer_barrier(c->peer_flags.data(), me, P, ep, 1, stream);
        entered = est == HGEMM_OK;
        if (st == HGEMM_OK) st = est;
        for (int i = 0; i < n && st == HGEMM_OK; ++i)
          if (cudaMemcpyAsync(peers[i], Cl, static_cast<size_t>(rc) * row_elems * 2,
                              cudaMemcpyDeviceToDevice, s) != cudaSuccess)
            st = HGEMM_ERR_CUDA;
      }
    }
    // A rank that launched no gated kernel still announces its entry, so that no peer's
    // gate waits in vain.
    if (!entered) hgemm_internal_peer_barrier(c->peer_flags.data(), me, P, ep, 1, stream);
    // Exit barrier: every rank announces the step in every peer's flag array and waits for
    // theirs (a 1-warp kernel with bounded waits; its failures land in the device status
    // word). Posted whatever happened locally, so that no peer waits in vain.
    const int bst = hgemm_internal_peer_barrier(c->peer_flags.data(), me, P, ep, 0, stream);
    return st != HGEMM_OK ? st : bst;
  }

  if (M % P == 0 && chunks == 1) {
    int st = HGEMM_OK;
    if (rc > 0)
      st = hgemm_internal_launch_unsplit(A_local, B, C + static_cast<size_t>(rb) * row_elems, rc,
                                         N, K, alpha, beta, stream, 0);
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
      const hgemm_half_t *Ac = A_local + static_cast<size_t>(cb) * K;
      hgemm_half_t *Cc = C + static_cast<size_t>(rb + cb) * row_elems;
      const int limit = c->sm_count - c->reserved_sms;
      const int st = hgemm_internal_launch_unsplit(
          Ac, B, Cc, cn, N, K, alpha, beta, stream,
          (P > 1 && c->reserved_sms > 0 && limit > 0) ? limit : 0);
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
