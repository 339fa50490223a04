/*
 * hgemm_b200.h -- C ABI of the B200 (sm_100a) FP16 GEMM library `libhgemm_b200.so`.
 *
 *     C[M,N] = alpha * (A[M,K] @ B[K,N]) + beta * C[M,N]
 *
 * All matrices are row-major, IEEE binary16 in and out, fp32 accumulation; A, B and C are
 * DEVICE pointers owned by the caller. C is both input (when beta != 0) and output, updated
 * in place. When beta == 0, C is never read, so NaN/Inf already in C do not propagate.
 * Each output element is alpha*acc (+ beta*C_in) computed in fp32 and rounded once to half
 * with round-to-nearest-even.
 *
 * Every entry point takes plain pointers and sizes; nothing here depends on PyTorch.
 * Reference interfaces replaced (yz-wqf/Hopper_GEMM):
 *   solve              <- extern "C" solve(...)            mma_half.cu:1636-1640
 *   hgemm_launch       <- h100_hgemm::launch(..., stream)  mma_half.cu:1530-1563
 *   hgemm_launch_ex    <- h100_hgemm::launch(..., force_bm, force_bn, group_m)
 *                                                         mma_half.cu:1530-1531
 *   hgemm_launch_tuned <- h100_hgemm::launch_tuned(...)    mma_half.cu:1624-1628
 *   hgemm_release      <- (the reference never frees g_pad, mma_half.cu:1308-1322)
 */
#ifndef HGEMM_B200_H_
#define HGEMM_B200_H_

#include <stddef.h>

#ifdef __cplusplus
#include <cuda_fp16.h>
typedef __half hgemm_half_t;
extern "C" {
#else
typedef unsigned short hgemm_half_t; /* IEEE binary16 bit pattern */
#endif

/* A CUDA stream handle (cudaStream_t / CUstream). 0 is the legacy default stream. */
typedef struct CUstream_st *hgemm_stream_t;

/* ---------------------------------------------------------------- status codes */
#define HGEMM_OK 0
#define HGEMM_ERR_INVALID_ARG 1      /* negative size, bad force_* tile, null pointer */
#define HGEMM_ERR_CUDA 2             /* a CUDA runtime call failed (see hgemm_status_string) */
#define HGEMM_ERR_TENSOR_MAP 3       /* cuTensorMapEncodeTiled rejected an operand */
#define HGEMM_ERR_ALLOC 4            /* scratch allocation for a restrided operand failed */
#define HGEMM_ERR_LAUNCH 5           /* kernel launch failed */
#define HGEMM_ERR_DEVICE_TIMEOUT 6   /* a bounded wait inside a kernel ran out (device status) */
#define HGEMM_ERR_UNSUPPORTED_DEVICE 7 /* not a compute capability 10.0 device */
#define HGEMM_ERR_NCCL 8             /* NCCL missing or an NCCL call failed */
#define HGEMM_ERR_TOO_LARGE 9        /* size beyond what this entry point supports */
#define HGEMM_ERR_NOT_FUSABLE 10     /* peer stores need the TMA-store tile path (N % 8 == 0,
                                        16-byte aligned C, K > 0); nothing was launched */

/* ---------------------------------------------------------------- GEMM entry points */

/* Drop-in for the reference's `solve`: launches on the legacy default stream, then
 * cudaDeviceSynchronize(). Returns nothing (like the reference); the outcome, including a
 * device-side wait timeout observed after the synchronize, is kept for hgemm_last_status(). */
void solve(const hgemm_half_t *A, const hgemm_half_t *B, hgemm_half_t *C, int M, int N, int K,
           float alpha, float beta);

/* Asynchronous launch on `stream` with the automatic tile / raster choice.
 * M == 0 or N == 0 is a no-op; K == 0 gives C = beta*C (alpha*0 added). Returns a status. */
int hgemm_launch(const hgemm_half_t *A, const hgemm_half_t *B, hgemm_half_t *C, int M, int N,
                 int K, float alpha, float beta, hgemm_stream_t stream);

/* Same, with the reference's override knobs. force_bm in {0, 128, 256} (256 = a 2-SM
 * UMMA pair of two 128-row CTAs), force_bn in {0, 64, 128, 256, 512}; 0 means automatic.
 * Valid explicit tiles: 256x512, 256x256, 256x128, 128x256, 128x128, 128x64.
 * group_m = raster band height in tile rows, M index fastest inside a band (0 = automatic);
 * a negative value -g selects bands of g tile columns with the N index fastest. */
int hgemm_launch_ex(const hgemm_half_t *A, const hgemm_half_t *B, hgemm_half_t *C, int M, int N,
                    int K, float alpha, float beta, hgemm_stream_t stream, int force_bm,
                    int force_bn, int group_m);

/* Opt-in autotuned launch: the first call per (device, M, N, K) times every tile x group_m
 * candidate (into a temporary output, so C is not disturbed) and caches the winner. */
int hgemm_launch_tuned(const hgemm_half_t *A, const hgemm_half_t *B, hgemm_half_t *C, int M,
                       int N, int K, float alpha, float beta, hgemm_stream_t stream);

/* No-allocation variant of hgemm_launch (no counterpart in the reference). For callers
 * that must not allocate device memory at call time -- a framework that owns a fixed
 * device-memory pool and forbids other cudaMalloc calls, or a latency-critical path that
 * cannot take the allocator's lock or its implicit device synchronisation. The only scratch
 * the GEMM can need (the restrided copy of A when K % 8 != 0, of B when N % 8 != 0, and the
 * 16-byte-strided copy of C when N % 8 != 0 and beta != 0) comes from a fixed array of
 * hgemm_noalloc_scratch_bytes() (64 MiB) that the library keeps on every device that loads
 * it, until the process exits; no cudaMalloc/cudaFree happens here. Shapes whose copies need
 * more in total (e.g. M x N above 32 Mi elements when only C needs the copy) return
 * HGEMM_ERR_TOO_LARGE before any work.
 * The first call on each device looks up the array's device address
 * (cudaGetSymbolAddress); make that first call outside any stream capture, and call
 * hgemm_release() after a device reset so that the address is looked up again. Each device has
 * its own copy of the array, and every call on a device shares that copy and leaves its
 * contents behind: two calls on one device that can overlap on the GPU (different streams)
 * race on it when both need restriding, so order them. Operands that do not start on a
 * 16-byte boundary, which hgemm_launch copies like ragged ones, run here on the scalar kernel,
 * which needs no scratch. Same arguments, semantics and status codes as hgemm_launch. */
int hgemm_launch_noalloc(const hgemm_half_t *A, const hgemm_half_t *B, hgemm_half_t *C, int M,
                         int N, int K, float alpha, float beta, hgemm_stream_t stream);
size_t hgemm_noalloc_scratch_bytes(void);

/* Host-buffer GEMM (no counterpart in the reference, whose solve() takes device pointers):
 * A_h, B_h and C_h are HOST pointers (page-locked, e.g. from cudaHostAlloc, for the copies to
 * run asynchronously), dA, dB, dC caller-owned device buffers of the full M x K, K x N and
 * M x N sizes. The call copies B in, then the rows of A (and of C when beta != 0) in blocks of
 * whole 256-row multiples; the GEMM of each block runs on `stream` as soon as its rows have
 * landed, and each finished block of C is copied back to C_h while later blocks are still
 * being copied in and computed, so the transfers in both directions overlap the math.
 * Asynchronous: C_h holds the result once `stream` passes the call (the library's own copy
 * streams are joined back into it). Same semantics and status codes as hgemm_launch, and the
 * same C bit for bit: the blocks never split K, and a problem that hgemm_launch would split
 * along K, or one with N % 8 != 0, runs as one block. Calls on one device are serialised on
 * the host. */
int hgemm_launch_host(const hgemm_half_t *A_h, const hgemm_half_t *B_h, hgemm_half_t *C_h,
                      hgemm_half_t *dA, hgemm_half_t *dB, hgemm_half_t *dC, int M, int N, int K,
                      float alpha, float beta, hgemm_stream_t stream);

/* ---------------------------------------------------------------- status, planning */

/* Status of the last call made by this host thread. */
int hgemm_last_status(void);
const char *hgemm_status_string(int status);

/* Device-side status word of the current device: HGEMM_OK, or HGEMM_ERR_DEVICE_TIMEOUT
 * when some kernel's bounded wait ran out since the last clear. Synchronizes the device.
 * `where` (may be NULL) receives the code of the wait that gave up. */
int hgemm_device_status(int clear, int *where);

/* Upper bound, in nanoseconds, on any single wait inside the GEMM kernels (default 2e9). */
void hgemm_set_wait_timeout_ns(unsigned long long ns);

/* Launches a kernel whose only wait is on an mbarrier that nothing arrives on, bounded by
 * `timeout_ns`, and returns the status that kernel reported (HGEMM_ERR_DEVICE_TIMEOUT when
 * the bound works). Leaves the CUDA context usable; clears the device status word. */
int hgemm_selftest_wait_timeout(unsigned long long timeout_ns);

/* Self-test of the multi-GPU barrier's bounded wait (one GPU, local memory only): runs the
 * barrier kernel as rank 0 of two with a partner that never announces. Returns
 * HGEMM_ERR_DEVICE_TIMEOUT when the wait gave up after ~timeout_ns and recorded its site
 * (the expected outcome), HGEMM_OK if it did not. Clears the device status word. */
int hgemm_selftest_peer_barrier(unsigned long long timeout_ns);

/* Multi-GPU step-entry gate self-test (one GPU, local memory only): runs the gated
 * peer-store kernel of hgemm_sharded_rank's fused path on a 256 x 256 x 64 GEMM whose one
 * "peer" C is a local buffer. satisfied != 0: the peer's entry flag is already set, and the
 * call returns HGEMM_OK when the peer copy was written and equals C. satisfied == 0: the
 * flag is never set; the call returns HGEMM_ERR_DEVICE_TIMEOUT when the gate gave up after
 * ~timeout_ns, recorded its site, left the peer copy untouched and still wrote the local C
 * (the expected outcome). Any other result means the gate misbehaved. Clears the device
 * status word. No counterpart in the reference. */
int hgemm_selftest_peer_entry(int satisfied, unsigned long long timeout_ns);

/* Frees the per-device scratch used to restride A (K % 8 != 0), B (N % 8 != 0) or C
 * (N % 8 != 0 with beta != 0), drops the autotuner's cache and forgets the cached device
 * addresses of hgemm_launch_noalloc's array. */
void hgemm_release(void);

/* Like hgemm_launch, but the GEMM runs on at most `sm_limit` SMs (persistent CTAs with a
 * static tile order), leaving the remaining SMs free for work that must run at the same time,
 * such as the collective kernels of hgemm_sharded_rank. No counterpart in the reference. */
int hgemm_launch_sm_limit(const hgemm_half_t *A, const hgemm_half_t *B, hgemm_half_t *C, int M,
                          int N, int K, float alpha, float beta, hgemm_stream_t stream,
                          int sm_limit);

/* Like hgemm_launch_sm_limit (sm_limit <= 0: every SM), and every C tile is also written
 * into `npeers` (<= 7) other M x N row-major buffers, such as the C buffers of peer GPUs
 * mapped into this process: after the local TMA store of each 32 x 64 chunk, the epilogue
 * copies the staged chunk to every destination with 16-byte stores. The peer buffers are
 * written asynchronously from the kernel and nothing here orders them against the
 * destinations' own work: the caller must make sure that no destination reads or writes its
 * buffer while this kernel may store into it, before and after. hgemm_sharded_rank's fused
 * path does that with step-entry and step-exit flags exchanged between the ranks. Returns
 * HGEMM_ERR_NOT_FUSABLE without launching when the shape takes a path without TMA stores.
 * No counterpart in the reference. */
int hgemm_launch_peers(const hgemm_half_t *A, const hgemm_half_t *B, hgemm_half_t *C, int M,
                       int N, int K, float alpha, float beta, hgemm_stream_t stream,
                       hgemm_half_t *const *peer_C, int npeers, int sm_limit);

/* Forces the one-CTA 128 x bn tile (bn = 64, 128 or 256) split over `ksplit` (1..8) CTAs
 * along K: each cluster of ksplit CTAs computes one tile, every CTA summing a contiguous
 * range of k-blocks, and the partial sums are reduced in a fixed order over distributed
 * shared memory (bit-stable). Shapes without the TMA-store epilogue (N % 8 != 0) run
 * unsplit. hgemm_launch picks split-K by itself for small problems. No counterpart in the
 * reference. */
int hgemm_launch_splitk(const hgemm_half_t *A, const hgemm_half_t *B, hgemm_half_t *C, int M,
                        int N, int K, float alpha, float beta, hgemm_stream_t stream, int bn,
                        int ksplit);

/* Host-only description of what hgemm_launch_ex would run; needs no GPU. */
typedef struct {
  int path;       /* 0 no-op, 1 tcgen05 tiles, 2 scalar kernel (K == 0) */
  int tile_m;     /* rows per tile: 128 (one CTA) or 256 (2-SM pair) */
  int tile_n;     /* columns per tile */
  int pair;       /* 1 or 2 CTAs per UMMA */
  int group_m;    /* raster band: > 0 tile rows (M fastest), < 0 tile columns (N fastest) */
  int stages;     /* smem pipeline depth */
  int tiles_m, tiles_n;
  int grid_ctas;  /* CTAs launched: with sched_static == 0 one cluster of `pair` CTAs per
                     tile, running clusters taking over not-yet-started ones (cluster launch
                     control); with sched_static == 1 one persistent cluster per slot */
  int pad_a, pad_b;      /* operand restrided into scratch (K % 8 or N % 8 != 0, or a base that
                            is not 16-byte aligned) */
  int lda, ldb;          /* leading dimensions the tensor maps use */
  int tma_store;         /* 1: TMA-store epilogue; 0: SIMT stores (N % 8 != 0 with beta == 0,
                            or C not 16-byte aligned) */
  size_t scratch_bytes;  /* scratch needed for restrided operands */
  int sched_static;      /* 1: cluster c takes tiles c, c + clusters, ... (short tiles, or all
                            tiles co-resident); 0: cluster launch control */
  int ksplit;            /* > 1: split-K, a cluster of ksplit one-CTA tiles shares each tile's
                            k-blocks (grid_ctas = tiles * ksplit) */
  int epi_warps;         /* epilogue warps per CTA: 4, or 8 where the epilogue sets the pace */
  int pad_c;             /* C computed in a 16-byte-strided copy (N % 8 != 0, beta != 0),
                            then compacted */
  int ldc;               /* row stride of the C the kernel writes */
} hgemm_plan_t;

/* `aligned16` says whether A, B and C all start on 16-byte boundaries (0: the plan for three
 * operands that do not, which restrides A and B and writes C with the SIMT-store epilogue);
 * `sm_count` and `pair_slots` (co-resident 2-CTA clusters) describe the device (<= 0: B200
 * defaults). */
int hgemm_plan(int M, int N, int K, float beta, int aligned16, int force_bm, int force_bn,
               int group_m, int sm_count, int pair_slots, hgemm_plan_t *out);

/* ---------------------------------------------------------------- multi-GPU (row shards)
 * One process per GPU. Rank r owns rows [row_begin(r), row_begin(r+1)) of A and C, with
 * row_begin(r) = (M * r) / nranks; B is replicated. hgemm_sharded_rank computes the local
 * C row block with the GEMM above and gathers C in place (NCCL, or the fused peer-store
 * path once the output is registered), so every rank ends with the full C. The reference
 * is single-GPU; this layer has no counterpart there (the survey's single-process
 * hgemm_sharded(ngpu, devs, ...) is served by one call of hgemm_sharded_rank per process).
 * NCCL is loaded at run time (libnccl.so.2); without it these return HGEMM_ERR_NCCL. */
typedef struct hgemm_comm_s *hgemm_comm_t;

int hgemm_comm_unique_id(void *id_out, size_t id_bytes); /* id_bytes >= 128 */
int hgemm_comm_init(hgemm_comm_t *comm, int nranks, const void *id, size_t id_bytes, int rank);
int hgemm_comm_destroy(hgemm_comm_t comm);

/* Collective (every rank calls it): registers this rank's full M x N output buffer C
 * (`bytes` long, 16-byte aligned, from cudaMalloc) and maps every peer's registered buffer
 * and step-flag array into this process through CUDA IPC. While registered,
 * hgemm_sharded_rank called with that buffer (on every rank) and M % nranks == 0 runs the
 * fused path: one kernel per rank that stores each finished tile into all ranks' C over
 * NVLink, then a one-warp barrier kernel; no NCCL kernel moves C and no NCCL call is made
 * per step. Ordering between steps uses two epochs in flag arrays (release stores /
 * acquire loads at system scope, every wait bounded by hgemm_set_wait_timeout_ns, a wait
 * that runs out recorded in the device status word): the kernel stores into a peer's C only
 * after that peer's stream has entered the same step (so the peer's readers of its C, queued
 * before the call on the stream passed to hgemm_sharded_rank, have finished), and the
 * barrier kernel returns only when every rank has finished the step (so readers queued
 * after the call see the whole C). C == NULL, bytes == 0 unregisters. Returns HGEMM_OK only
 * when every rank registered (the outcome is agreed on collectively). No counterpart in the
 * reference. */
int hgemm_comm_register_output(hgemm_comm_t comm, hgemm_half_t *C, size_t bytes);

/* Address, in this process, of rank r's registered output buffer (this rank's own C for
 * r == rank; a CUDA IPC mapping opened on this rank's device otherwise), or
 * HGEMM_ERR_INVALID_ARG when no output is registered. No counterpart in the reference. */
int hgemm_comm_output_ptr(hgemm_comm_t comm, int r, hgemm_half_t **out);

/* SMs that the chunk GEMMs of hgemm_sharded_rank (chunks > 1, nranks > 1) leave free for
 * the exchange kernels that run next to them (default 16; 0 = the GEMM takes every SM).
 * No counterpart in the reference. */
int hgemm_comm_set_reserved_sms(hgemm_comm_t comm, int sms);

/* A_local: this rank's rows of A (rows x K); B: full K x N on this device; C: full M x N on
 * this device (the local row block is read when beta != 0). Equal row blocks
 * (M % nranks == 0) gather in place with one ncclAllGather; otherwise grouped
 * ncclSend/ncclRecv of each rank's rows to every peer. `chunks` > 1 splits the local rows so
 * the gather of chunk c (grouped sends and receives) overlaps the GEMM of c+1. */
int hgemm_sharded_rank(hgemm_comm_t comm, const hgemm_half_t *A_local, const hgemm_half_t *B,
                       hgemm_half_t *C, int M, int N, int K, float alpha, float beta,
                       int chunks, hgemm_stream_t stream);

/* Row range helper, identical to the one hgemm_sharded_rank uses. */
int hgemm_shard_rows(int M, int nranks, int rank, int *row_begin, int *row_count);
/* Rows [begin, begin + count) of a `rows`-row block that form chunk `chunk` of `chunks`. */
int hgemm_shard_chunk_rows(int rows, int chunks, int chunk, int *begin, int *count);

/* HGEMM_OK while the communicator is healthy, HGEMM_ERR_NCCL once NCCL reports an
 * asynchronous error (e.g. a peer died); poll it between steps. */
int hgemm_comm_check(hgemm_comm_t comm);
/* Tears the communicator down without waiting for peers (after a failure); frees `comm`. */
int hgemm_comm_abort(hgemm_comm_t comm);

#ifdef __cplusplus
}
#endif

#endif /* HGEMM_B200_H_ */
