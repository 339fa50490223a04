// B200 (sm_100a) FP16 GEMM: C = alpha * A[M,K] @ B[K,N] + beta * C, row-major, half in/out,
// fp32 accumulate. Kernel, per-shape dispatcher and the C ABI declared in hgemm_b200.h.
//
// Design (B200-first, not a translation of the reference's sm_90a wgmma kernel):
//   * One CTA per SM (~226 KB of shared memory each), optionally launched
//     as 2-CTA clusters that act as one UMMA pair: `tcgen05.mma.cta_group::2` computes a
//     256 x BN tile, each CTA holding 128 rows of A and BN/2 columns of B in its own smem.
//     The pair shares B through the tensor core, which is what the reference bought by
//     broadcasting B across its cluster (mma_half.cu:331-367). Every TMA load here lands in
//     the issuing CTA's own shared memory.
//   * Warp roles: warp 0 = TMA producer (one lane), warp 1 = TMEM allocator + UMMA issuer
//     (one lane of the pair's leader CTA), warps 2..5 = epilogue (TMEM lane quarters).
//   * fp32 accumulators live in TMEM, double buffered (2 x BN columns), so the epilogue of
//     tile i overlaps the mainloop of tile i+1.
//   * A is consumed K-major and B N-major straight from the caller's row-major buffers;
//     both arrive through 128-byte-swizzled TMA boxes (64 halves wide). TMA zero-fills
//     out-of-range rows/columns, which handles every ragged M/N/K edge.
//   * Epilogue: tcgen05.ld -> alpha*acc (+ beta*C_in) in fp32 -> one RNE to half ->
//     128B-swizzled smem staging -> TMA store (N % 8 == 0), or coalesced predicated stores
//     when C's row stride is not 16-byte aligned (N % 8 != 0).
//   * Every wait is bounded (globaltimer); a wait that runs out records a device status
//     word, raises the CTA's abort flag and the kernel unwinds, freeing its TMEM.
//
// Reference correspondence (yz-wqf/Hopper_GEMM, mma_half.cu):
//   gemm_kernel 887-1222 -> hgemm_tc_kernel; store_c_tile(_tma) 724-872 -> epilogue below;
//   gemm_fallback 1225-1250 -> hgemm_simt_kernel; pad_copy_kernel 1254-1261 ->
//   restride_kernel; make_tensor_map/get_encode_tiled 1264-1297 -> encode_2d;
//   tma_compatible 1301-1306 / pad_workspace 1308-1322 / launch 1530-1563 -> launch_impl;
//   launch_mainloop 1441-1526 -> make_plan; autotune 1570-1628 -> hgemm_launch_tuned;
//   solve 1636-1640 -> solve.

#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <map>
#include <mutex>
#include <tuple>
#include <vector>

#include "hgemm_b200.h"
#include "ptx_sm100.cuh"

namespace hgemm {

// ============================================================================ constants
constexpr int BK = 64;          // k per pipeline stage: one 128-byte swizzle row of halves
constexpr int CTA_M = 128;      // accumulator rows per CTA (= TMEM lanes)
constexpr int UMMA_K = 16;      // k per tcgen05.mma.kind::f16
constexpr int EPI_ROWS = 32;    // rows per epilogue warp (its TMEM lane quarter)
constexpr int EPI_COLS = 64;    // columns per epilogue chunk (one 128-byte swizzle row)

constexpr int SMEM_LIMIT = 232448;  // sm_100 opt-in dynamic shared memory per block
constexpr int BAR_BYTES = 512;
// Peer-store launches keep the 256x512 tile only from this K on (longer main loop per tile).
constexpr int kPeerWideTileMinK = 12288;
// Largest split-K cluster (portable cluster size).
constexpr int kMaxSplit = 8;
// Tiles whose main loop is estimated shorter than this (cycles) use the static schedule.
constexpr double kStaticTileCycles = 8192.0;

// Device status word: 0, or kDevTimeout | where. Written once per failure (first wins).
constexpr unsigned kDevTimeout = 0x100u;
enum WaitSite : unsigned {
  kSiteProducerEmpty = 1,
  kSiteMmaTmemEmpty = 2,
  kSiteMmaFull = 3,
  kSiteEpiTmemFull = 4,
  kSiteDrain = 5,
  kSiteSelftest = 6,
  kSiteSchedEmpty = 7,
  kSiteSchedFull = 8,
  kSiteClc = 9,
  kSitePeerBarrier = 10,
  kSiteSplitReduce = 11,
  kSitePeerEntry = 12,
};
__device__ unsigned int g_dev_status = 0;

template <int PAIR, int BN, int EPIW = 4>
struct TileCfg {
  static constexpr int UMMA_N = BN < 256 ? BN : 256;        // N of one tcgen05.mma
  static constexpr int N_SUB = BN / UMMA_N;                  // UMMAs per k16 step
  static constexpr int ACC_BUFS = (2 * BN <= 512) ? 2 : 1;   // TMEM accumulator buffers
  static constexpr int SUB_COLS = UMMA_N / PAIR;             // B columns per CTA per UMMA
  static constexpr int SUB_BOXES = SUB_COLS / 64;            // 64-column TMA boxes each
  static constexpr int B_COLS = BN / PAIR;                   // B columns this CTA loads
  static constexpr int A_BYTES = CTA_M * BK * 2;             // 16 KB
  static constexpr int B_BYTES = B_COLS * BK * 2;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int TX_BYTES = STAGE_BYTES * PAIR;        // armed on the leader's barrier
  // Epilogue warps (EPIW): 4, one per TMEM lane quarter, or 8, two per quarter, each taking
  // half of the columns (for the one-accumulator 256x512 tile each group of four drains
  // one N half, so both halves drain at once). Each warp double-buffers a 4 KB staging
  // buffer, so 8 warps cost 32 KB of pipeline stages; the planner uses them where the
  // epilogue, not the main loop, sets the pace (see choose_epi_warps).
  static constexpr int EPI_WARPS = EPIW;
  // The one-accumulator tile (BN = 512) with 8 warps single-buffers its staging, so that it
  // keeps the 4-warp flavour's pipeline depth: its stores have a whole main loop to drain,
  // only the TMEM drain between tiles is on the critical path.
  static constexpr int EPI_BUFS = (ACC_BUFS == 1 && EPIW == 8) ? 1 : 2;
  static constexpr int THREADS = 64 + 32 * EPI_WARPS;
  static constexpr int EPI_COLS_PER_WARP = BN * 4 / EPI_WARPS;
  static constexpr int EPI_BYTES = EPI_WARPS * EPI_BUFS * EPI_ROWS * 128;
  static constexpr int STAGES_FIT = (SMEM_LIMIT - EPI_BYTES - 1024 - BAR_BYTES) / STAGE_BYTES;
  static constexpr int STAGES = STAGES_FIT > 8 ? 8 : STAGES_FIT;
  static constexpr int SMEM = 1024 + STAGES * STAGE_BYTES + EPI_BYTES + BAR_BYTES;
  static constexpr int TMEM_COLS = BN * ACC_BUFS;
  static constexpr int UMMA_M = CTA_M * PAIR;
  static constexpr int SCHED_SLOTS = 4;                      // tile-index ring depth
  static_assert(SUB_COLS % 64 == 0, "B slice must be whole 64-column swizzle blocks");
  static_assert(STAGES >= 3, "pipeline too shallow");
  static_assert(SMEM <= SMEM_LIMIT, "shared memory over budget");
  static_assert(TMEM_COLS >= 32 && TMEM_COLS <= 512 && (TMEM_COLS & (TMEM_COLS - 1)) == 0,
                "TMEM allocation must be a power of two in [32, 512]");
  static_assert(UMMA_N % 16 == 0 && UMMA_N <= 256, "UMMA N");
};

struct KParams {
  int M, N, K;
  int tiles_m, tiles_n, num_tiles, num_kb;
  int group_m;
  float alpha, beta;
  __half *C;
  unsigned long long timeout_ns;
  int sched_static;  // 1: cluster c takes tiles c, c + clusters, ...; 0: cluster launch control
  int c_evict_first;  // 1: C stores (local and peer) are marked evict-first in L2
  int ldc;            // row stride of C in halves (N, or N rounded up to 8 for the padded copy)
  int ksplit;         // > 1 (one-CTA tiles only): a cluster of ksplit CTAs shares each tile's
                      // k-blocks and reduces the partial sums over distributed shared memory
  int b4;             // 1: tmB is the 4-D view of B (every tile whole in N): one load per stage
};

// Other destinations of every C tile (e.g. the C buffers of peer GPUs mapped into this
// process): M x N row-major buffers with row stride N. The epilogue warps copy each staged
// 32 x 64 chunk to them with coalesced 16-byte stores after the local TMA store, so a
// row-sharded GEMM delivers its rows to every rank while it computes them (the SM's TMA
// unit only carries the local C and the operand loads; a TMA-store variant of the copy
// measured the same on 4 B200s).
//
// Step-entry gate (epoch != 0): a destination may still be reading its C from the previous
// step when this kernel starts. Every CTA therefore first announces `epoch` in each
// destination's entry flag for this rank (post[d], a system-scope release store: the
// kernel has started, so everything queued before it on this stream, including this
// rank's own readers of C, has finished), and each epilogue warp, before its first peer
// store, waits until every destination has announced the same epoch here (wait[d],
// acquire loads, bounded by the wait timeout). A wait that runs out records
// kSitePeerEntry in the device status word and the kernel keeps going without peer stores.
constexpr int kMaxPeers = 7;
struct PeerMaps {
  __half *ptr[kMaxPeers];
  unsigned long long *post[kMaxPeers];        // destination d's entry flag for this rank
  const unsigned long long *wait[kMaxPeers];  // this rank's entry flag for destination d
  unsigned long long epoch;                   // 0: no gate (the caller orders the readers)
  int n;
};
// C stores carry an L2 evict-first policy from this K on: with long main loops the A and B
// tiles are re-read from L2 many times and the streamed C should not displace them
// (8192^3: +1.4%); with short K the whole C fits in L2 and is written back after the
// kernel, which evict-first would pull into the kernel (4096x8192x128: -3%).
constexpr int kCEvictFirstMinK = 4096;

// ============================================================================ device helpers
struct WaitCtx {
  volatile int *abort_flag;     // this CTA's flag (generic pointer to smem)
  uint32_t peer_abort;          // shared::cluster address of the peer's flag (pair), or 0
  unsigned long long timeout_ns;
};

__device__ __forceinline__ void raise_abort(const WaitCtx &w, unsigned where) {
  atomicCAS(&g_dev_status, 0u, kDevTimeout | where);
  *w.abort_flag = 1;
  if (w.peer_abort)
    asm volatile("st.shared::cluster.u32 [%0], %1;" ::"r"(w.peer_abort), "r"(1) : "memory");
}

// Bounded mbarrier wait. Returns false if the CTA is aborting or the wait timed out.
template <bool CLUSTER_ACQ>
__device__ __forceinline__ bool wait_bar(uint32_t bar, uint32_t parity, const WaitCtx &w,
                                         unsigned where) {
  auto probe = [&]() {
    return CLUSTER_ACQ ? ptx::mbar_try_wait_cluster(bar, parity) : ptx::mbar_try_wait(bar, parity);
  };
  // Fast path first: a non-suspending test costs ~30 cycles less than try_wait when the
  // phase is already complete, which is the common case on the UMMA issuer's hot loop.
  if (ptx::mbar_test_wait_cluster(bar, parity)) return true;
  const uint64_t t0 = ptx::globaltimer();
  for (uint32_t n = 1;; ++n) {
    if (probe()) return true;
    if ((n & 15u) == 0) {
      if (*w.abort_flag) return false;
      if (ptx::globaltimer() - t0 > w.timeout_ns) {
        raise_abort(w, where);
        return false;
      }
    }
  }
}

__device__ __forceinline__ void decode_tile(int t, const KParams &p, int &tm, int &tn) {
  // Bands of |group_m| tile-rows (group_m > 0: M index fastest inside a band) or of
  // |group_m| tile-columns (group_m < 0: N index fastest), so the tiles in flight at the
  // same time share a few A row-blocks and B column-blocks in L2.
  if (p.group_m > 0) {
    const int band_tiles = p.group_m * p.tiles_n;
    const int band = t / band_tiles;
    const int idx = t - band * band_tiles;
    const int m0 = band * p.group_m;
    const int rows = min(p.group_m, p.tiles_m - m0);
    tm = m0 + idx % rows;
    tn = idx / rows;
  } else {
    const int g = -p.group_m;
    const int band_tiles = g * p.tiles_m;
    const int band = t / band_tiles;
    const int idx = t - band * band_tiles;
    const int n0 = band * g;
    const int cols = min(g, p.tiles_n - n0);
    tn = n0 + idx % cols;
    tm = idx / cols;
  }
}

__device__ __forceinline__ uint32_t pack_half2(float lo, float hi) {
  __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<uint32_t *>(&h);
}

// Offset of 16-byte chunk j of row r inside a 128B-swizzled 1024-byte-aligned buffer whose
// rows are 128 bytes: the chunk index is XORed with r mod 8 (TMA SWIZZLE_128B pattern).
__device__ __forceinline__ uint32_t sw128_off(int r, int j) {
  return static_cast<uint32_t>(r * 128 + ((j ^ (r & 7)) << 4));
}

// ============================================================================ the kernel
// Work distribution: the grid has one cluster (PAIR CTAs) per output tile. Each running
// cluster starts on its own tile and then takes over tiles of clusters that have not started
// yet through cluster launch control (clusterlaunchcontrol.try_cancel), so the tiles spread
// over the SMs by how fast each one actually goes (the two dies and their GPCs do not run at
// one clock under the power cap). The leader CTA's producer thread owns that sequence and
// publishes every tile index through a small shared-memory ring that the other roles of
// both CTAs read; -1 ends the sequence.
template <int PAIR, int BN, bool TMA_EPI, int EPIW, bool SPLITK, bool PEERS>
__global__ void __launch_bounds__(TileCfg<PAIR, BN, EPIW>::THREADS, 1)
    hgemm_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                    const __grid_constant__ CUtensorMap tmC, const KParams p,
                    const __grid_constant__ PeerMaps peers) {
#if defined(__CUDA_ARCH__) && (__CUDA_ARCH__ >= 1000)
  using Cfg = TileCfg<PAIR, BN, EPIW>;
  // Peer copies of every tile (fused multi-GPU path) exist only in the PEERS instances: the
  // code alone cost the plain GEMM 1-6% (register pressure in the epilogue).
  const int npeer = PEERS ? peers.n : 0;
  static_assert(!SPLITK || (PAIR == 1 && TMA_EPI), "split-K: one-CTA tiles with TMA stores");
  constexpr int S = Cfg::STAGES;
  constexpr int NSL = Cfg::SCHED_SLOTS;
  constexpr int ACC_BUFS = Cfg::ACC_BUFS;

  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = ptx::smem_u32(smem_raw);
  const uint32_t base = (raw_addr + 1023u) & ~1023u;
  uint8_t *smem = smem_raw + (base - raw_addr);
  const uint32_t sA0 = base;
  const uint32_t sB0 = base + S * Cfg::A_BYTES;
  uint8_t *epi = smem + S * Cfg::STAGE_BYTES;
  uint64_t *bars = reinterpret_cast<uint64_t *>(epi + Cfg::EPI_BYTES);
  uint64_t *full = bars;                    // [S]   TMA bytes landed (leader CTA's copy is used)
  uint64_t *empty = bars + S;               // [S]   UMMA finished reading the stage
  uint64_t *tfull = bars + 2 * S;           // [2]   accumulator buffer ready for the epilogue
  uint64_t *tempty = bars + 2 * S + 2;      // [2]   epilogue drained the accumulator buffer
  uint64_t *drain = bars + 2 * S + 4;       // [1]   teardown: all issued UMMAs retired
  uint64_t *sched_full = bars + 2 * S + 5;  // [NSL] tile index written
  uint64_t *sched_empty = bars + 2 * S + 5 + NSL;  // [NSL] every reader took it (leader's copy)
  uint64_t *clc_bar = bars + 2 * S + 5 + 2 * NSL;  // [1]  launch-control response landed
  uint64_t *red_ready = bars + 2 * S + 6 + 2 * NSL;  // [1] split-K: every partial is in smem
  uint64_t *red_done = bars + 2 * S + 7 + 2 * NSL;   // [1] split-K: nobody reads ours any more
  uint8_t *misc = reinterpret_cast<uint8_t *>(
      (reinterpret_cast<uintptr_t>(bars + 2 * S + 8 + 2 * NSL) + 15) & ~uintptr_t(15));
  uint8_t *clc_resp = misc;                                      // 16 bytes
  volatile int *sched_val = reinterpret_cast<volatile int *>(misc + 16);  // [NSL]
  uint32_t *tmem_holder = reinterpret_cast<uint32_t *>(misc + 16 + 4 * NSL);
  volatile int *abort_flag = reinterpret_cast<volatile int *>(misc + 20 + 4 * NSL);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = (PAIR == 2) ? ptx::cluster_ctarank() : 0u;
  // Split-K (SPLITK instances only): the cluster's CTAs share one tile, CTA `split` taking
  // k-blocks [kb_begin, kb_end).
  const int ksplit = SPLITK ? p.ksplit : 1;
  const int split = SPLITK ? static_cast<int>(ptx::cluster_ctarank()) : 0;
  const int kb_begin =
      SPLITK ? static_cast<int>(static_cast<long long>(p.num_kb) * split / ksplit) : 0;
  const int kb_end =
      SPLITK ? static_cast<int>(static_cast<long long>(p.num_kb) * (split + 1) / ksplit)
             : p.num_kb;
  constexpr bool clustered = PAIR == 2 || SPLITK;
  const int first_tile =
      clustered ? static_cast<int>(ptx::cluster_id_x()) : static_cast<int>(blockIdx.x);

  // One accumulator, 8 epilogue warps, TMA stores, beta == 0: warp group g (ew / 4) drains
  // columns [128 g, 128 g + 128) of each N half, so each half drains twice as fast as with one
  // group of 4 warps per half (the tensor core has only the deferred slice-1 work of the last
  // stages to do meanwhile).
  const bool wide_drain = ACC_BUFS == 1 && Cfg::EPI_WARPS == 8 && TMA_EPI && !SPLITK &&
                          p.beta == 0.0f;
  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      ptx::mbar_init(ptx::smem_u32(&full[s]), 1);
      ptx::mbar_init(ptx::smem_u32(&empty[s]), 1);
    }
    for (int a = 0; a < 2; ++a) {
      ptx::mbar_init(ptx::smem_u32(&tfull[a]), 1);
      // One accumulator (BN = 512): each N half is drained by 4 warps per CTA (all 4 warps
      // drain both halves, or with 8 warps each group of 4 drains one half).
      // With 8 warps and beta == 0 every warp drains a quarter of each half instead
      // (wide_drain below), so all 8 arrive on both halves.
      ptx::mbar_init(ptx::smem_u32(&tempty[a]),
                     (ACC_BUFS == 1 ? (wide_drain ? 8 : 4) : Cfg::EPI_WARPS) * PAIR);
    }
    ptx::mbar_init(ptx::smem_u32(drain), 1);
    // Readers of each tile index: leader MMA + the epilogue warps (+ the peer's producer and
    // epilogue warps for a pair).
    for (int i = 0; i < NSL; ++i) {
      ptx::mbar_init(ptx::smem_u32(&sched_full[i]), 1);
      ptx::mbar_init(ptx::smem_u32(&sched_empty[i]), (1 + Cfg::EPI_WARPS) * PAIR);
    }
    ptx::mbar_init(ptx::smem_u32(clc_bar), 1);
    // Split-K: each of the cluster's EPI_WARPS * ksplit epilogue warps arrives once on every
    // CTA.
    ptx::mbar_init(ptx::smem_u32(red_ready), Cfg::EPI_WARPS * ksplit);
    ptx::mbar_init(ptx::smem_u32(red_done), Cfg::EPI_WARPS * ksplit);
    *abort_flag = 0;
    ptx::fence_mbar_init_cluster();
  }
  if (warp == 0 && lane == 0) {
    ptx::prefetch_tmap(&tmA);
    ptx::prefetch_tmap(&tmB);
    if (TMA_EPI) {
      ptx::prefetch_tmap(&tmC);
    }
  }
  if (warp == 1) {
    ptx::tmem_alloc<PAIR>(ptx::smem_u32(tmem_holder), Cfg::TMEM_COLS);
    ptx::tmem_relinquish<PAIR>();
  }
  ptx::tc_fence_before();
  __syncthreads();
  if (clustered) ptx::cluster_sync();
  ptx::tc_fence_after();
  const uint32_t tmem_base = *reinterpret_cast<volatile uint32_t *>(tmem_holder);

  WaitCtx wctx;
  wctx.abort_flag = abort_flag;
  wctx.peer_abort =
      (PAIR == 2) ? ptx::mapa(ptx::smem_u32(const_cast<int *>(abort_flag)), rank ^ 1u) : 0u;
  wctx.timeout_ns = p.timeout_ns;

  // Readers take tile indices in ring order and release each slot to the leader's producer.
  const uint32_t sched_empty_leader0 =
      (PAIR == 2) ? ptx::mapa(ptx::smem_u32(&sched_empty[0]), 0u) : ptx::smem_u32(&sched_empty[0]);
  auto sched_take = [&](int &slot, uint32_t &sph, int &tile) {
    tile = sched_val[slot];
    const uint32_t eb = sched_empty_leader0 + static_cast<uint32_t>(slot) * 8u;
    if (PAIR == 2)
      ptx::mbar_arrive_remote(eb);
    else
      ptx::mbar_arrive(eb);
    if (++slot == NSL) {
      slot = 0;
      sph ^= 1u;
    }
  };
  auto sched_read = [&](int &slot, uint32_t &sph, int &tile) -> bool {
    if (!wait_bar<PAIR == 2>(ptx::smem_u32(&sched_full[slot]), sph, wctx, kSiteSchedFull))
      return false;
    sched_take(slot, sph, tile);
    return true;
  };
  // Non-blocking: takes the next index only if it is already there.
  auto sched_try_read = [&](int &slot, uint32_t &sph, int &tile) -> bool {
    if (!ptx::mbar_test_wait_cluster(ptx::smem_u32(&sched_full[slot]), sph)) return false;
    sched_take(slot, sph, tile);
    return true;
  };

  if (warp == 0) {
    // ------------------------------------------------------------------ TMA producer
    if (lane == 0) {
      int s = 0;
      uint32_t ph = 0;
      long long issued = 0;
      bool ok = true;
      int sslot = 0;
      uint32_t sph = 0;
      const uint32_t full_leader0 =
          (PAIR == 2) ? ptx::mapa(ptx::smem_u32(&full[0]), 0u) : ptx::smem_u32(&full[0]);

      // All k-blocks of one tile: this CTA's 128 rows of A and its share of B's columns
      // (for UMMA j, columns [j*UMMA_N + rank*SUB_COLS, +SUB_COLS) of the tile).
      auto load_tile = [&](int tile) -> bool {
        int tm, tn;
        decode_tile(tile, p, tm, tn);
        const int arow = tm * Cfg::UMMA_M + static_cast<int>(rank) * CTA_M;
        const int bcol = tn * BN + static_cast<int>(rank) * Cfg::SUB_COLS;
        for (int kb = kb_begin; kb < kb_end; ++kb) {
          if (!wait_bar<false>(ptx::smem_u32(&empty[s]), ph ^ 1u, wctx, kSiteProducerEmpty))
            return false;
          const uint32_t fbar = full_leader0 + static_cast<uint32_t>(s) * 8u;
          if (rank == 0) ptx::mbar_arrive_expect_tx(ptx::smem_u32(&full[s]), Cfg::TX_BYTES);
          const uint32_t dA = sA0 + static_cast<uint32_t>(s) * Cfg::A_BYTES;
          const uint32_t dB = sB0 + static_cast<uint32_t>(s) * Cfg::B_BYTES;
          if (PAIR == 2)
            ptx::tma_load_2d_pair(&tmA, dA, fbar, kb * BK, arow);
          else
            ptx::tma_load_2d(&tmA, dA, fbar, kb * BK, arow);
          if (p.b4) {
            // All N_SUB x SUB_BOXES blocks of 64 columns in one instruction: coordinates are
            // (column in block, k, first 64-column block of this CTA's slice 0, slice).
            if (PAIR == 2)
              ptx::tma_load_4d_pair(&tmB, dB, fbar, 0, kb * BK, bcol / 64, 0);
            else
              ptx::tma_load_4d(&tmB, dB, fbar, 0, kb * BK, bcol / 64, 0);
          } else {
#pragma unroll
            for (int j = 0; j < Cfg::N_SUB; ++j) {
#pragma unroll
              for (int b = 0; b < Cfg::SUB_BOXES; ++b) {
                const uint32_t dst = dB + static_cast<uint32_t>(j * Cfg::SUB_BOXES + b) * (BK * 128);
                const int col = bcol + j * Cfg::UMMA_N + 64 * b;
                if (PAIR == 2)
                  ptx::tma_load_2d_pair(&tmB, dst, fbar, col, kb * BK);
                else
                  ptx::tma_load_2d(&tmB, dst, fbar, col, kb * BK);
              }
            }
          }
          ++issued;
          if (++s == S) {
            s = 0;
            ph ^= 1u;
          }
        }
        return true;
      };

      if (rank == 0) {
        // Scheduler: publish each tile index to the ring (both CTAs' copies of the slot).
        auto publish = [&](int v) -> bool {
          if (!wait_bar<PAIR == 2>(ptx::smem_u32(&sched_empty[sslot]), sph ^ 1u, wctx,
                                   kSiteSchedEmpty))
            return false;
          sched_val[sslot] = v;
          const uint32_t fb = ptx::smem_u32(&sched_full[sslot]);
          if (PAIR == 2) {
            ptx::st_cluster_u32(ptx::mapa(ptx::smem_u32(const_cast<int *>(&sched_val[sslot])), 1u),
                                static_cast<uint32_t>(v));
            ptx::mbar_arrive_cluster(ptx::mapa(fb, 1u));
          }
          ptx::mbar_arrive(fb);
          if (++sslot == NSL) {
            sslot = 0;
            sph ^= 1u;
          }
          return true;
        };
        bool clc_live = p.sched_static == 0, clc_pending = false;
        const int stride =
            clustered ? static_cast<int>(ptx::nclusters_x()) : static_cast<int>(gridDim.x);
        uint32_t clc_ph = 0;
        int tile = first_tile;
        ok = publish(tile);
        while (ok && tile >= 0) {
          if (clc_live) {
            // Ask for the next tile now; the answer is needed only after this tile's loads.
            ptx::mbar_arrive_expect_tx(ptx::smem_u32(clc_bar), 16);
            ptx::clc_try_cancel(ptx::smem_u32(clc_resp), ptx::smem_u32(clc_bar));
            clc_pending = true;
          }
          if (!load_tile(tile)) {
            ok = false;
            break;
          }
          int next = -1;
          if (p.sched_static) {
            next = tile + stride < p.num_tiles ? tile + stride : -1;
          } else if (clc_live) {
            if (!wait_bar<false>(ptx::smem_u32(clc_bar), clc_ph, wctx, kSiteClc)) {
              ok = false;
              break;
            }
            clc_pending = false;
            clc_ph ^= 1u;
            uint32_t x = 0;
            if (ptx::clc_query(ptx::smem_u32(clc_resp), x))
              next = static_cast<int>(x) / PAIR;
            else
              clc_live = false;  // nothing left to take; never ask again
            ptx::fence_proxy_async_smem();
          }
          ok = publish(next);
          tile = next;
        }
        if (!ok && clc_pending) {
          // Unwinding: the launch-control response must land before the CTA exits.
          WaitCtx dctx = wctx;
          volatile int no_abort = 0;
          dctx.abort_flag = &no_abort;
          dctx.peer_abort = 0;
          dctx.timeout_ns = 50000000ull;
          wait_bar<false>(ptx::smem_u32(clc_bar), clc_ph, dctx, kSiteDrain);
        }
      } else {
        // The pair's second CTA follows the leader's tile sequence.
        int tile = -1;
        while (ok) {
          if (!sched_read(sslot, sph, tile)) {
            ok = false;
            break;
          }
          if (tile < 0) break;
          ok = load_tile(tile);
        }
      }
      if (!ok && rank == 0) {
        // Unwinding: let the loads this CTA armed land before the CTA can exit.
        const int armed = issued >= S ? S : static_cast<int>(issued);
        for (int j = 0; j < armed; ++j) {
          const uint32_t par = (j < s) ? ph : (ph ^ 1u);
          WaitCtx dctx = wctx;
          volatile int no_abort = 0;
          dctx.abort_flag = &no_abort;
          dctx.peer_abort = 0;
          dctx.timeout_ns = 50000000ull;
          if (!wait_bar<false>(ptx::smem_u32(&full[j]), par, dctx, kSiteDrain)) break;
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ UMMA issuer
    if (lane == 0 && rank == 0) {
      constexpr uint32_t idesc = ptx::umma_idesc_f16_f32(Cfg::UMMA_M, Cfg::UMMA_N);
      int s = 0;
      uint32_t ph = 0;
      int it = 0;
      int sslot = 0;
      uint32_t sph = 0;
      bool issued_any = false;
      bool ok = true;
      uint32_t dtm = tmem_base;
      // UMMA j (N-slice j) of one pipeline stage; A (K-major) advances 32 bytes per k16
      // inside the swizzle row, B (N-major) 16 rows of 128 bytes per k16, and UMMA j reads
      // the next SUB_BOXES blocks of 8 KB. Descriptor start addresses are in 16-byte units.
      auto issue_sub = [&](int stage, int kb, int j) {
        const uint64_t adesc = ptx::umma_desc_sw128(sA0 + stage * Cfg::A_BYTES, 16, 1024);
        const uint64_t bdesc = ptx::umma_desc_sw128(sB0 + stage * Cfg::B_BYTES, BK * 128, 1024);
#pragma unroll
        for (int k = 0; k < BK / UMMA_K; ++k)
          ptx::umma_f16<PAIR>(dtm + static_cast<uint32_t>(j * Cfg::UMMA_N),
                              adesc + static_cast<uint64_t>(2 * k),
                              bdesc + static_cast<uint64_t>(128 * k + j * Cfg::SUB_BOXES * (BK * 128 / 16)),
                              idesc, ((kb - kb_begin) | k) != 0 ? 1u : 0u);
        issued_any = true;
      };
      auto release_stage = [&](int stage) {
        const uint32_t eb = ptx::smem_u32(&empty[stage]);
        if (PAIR == 2)
          ptx::umma_commit_pair_mask(eb, 0x3);  // both CTAs' copies of empty[stage]
        else
          ptx::umma_commit<1>(eb);
      };
      // The issuer only needs to know whether another tile follows; it takes that index
      // without blocking during the current tile's last S k-blocks (the producer publishes it
      // once it has issued this tile's loads), so a tile start never waits on the ring.
      int tile = -1;
      if (!sched_read(sslot, sph, tile)) ok = false;
      while (ok && tile >= 0) {
        int next = -1;
        bool have_next = false;
        auto poll_next = [&](int kb) {
          if (!have_next && kb >= kb_end - S && sched_try_read(sslot, sph, next)) have_next = true;
        };
        const int acc = it % ACC_BUFS;
        const uint32_t aph = static_cast<uint32_t>(it / ACC_BUFS) & 1u;
        if constexpr (ACC_BUFS == 2) {
          if (!wait_bar<PAIR == 2>(ptx::smem_u32(&tempty[acc]), aph ^ 1u, wctx, kSiteMmaTmemEmpty)) {
            ok = false;
            break;
          }
          ptx::tc_fence_after();
          dtm = tmem_base + static_cast<uint32_t>(acc * BN);
          // One issuing thread has only ~4 UMMAs' time (BN=256) per k-block, so the hot loop
          // carries nothing but the wait, the UMMAs and the stage release; the look-ahead on
          // the tile ring happens in a separate tail loop over the last S k-blocks.
          const int main_kb = kb_end - S > kb_begin ? kb_end - S : kb_begin;
          auto kblock = [&](int kb) -> bool {
            if (!wait_bar<false>(ptx::smem_u32(&full[s]), ph, wctx, kSiteMmaFull)) return false;
            ptx::tc_fence_after();
#pragma unroll
            for (int j = 0; j < Cfg::N_SUB; ++j) issue_sub(s, kb, j);
            release_stage(s);
            if (++s == S) {
              s = 0;
              ph ^= 1u;
            }
            return true;
          };
          for (int kb = kb_begin; kb < main_kb && ok; ++kb) ok = kblock(kb);
          for (int kb = main_kb; kb < kb_end && ok; ++kb) {
            ok = kblock(kb);
            poll_next(kb);
          }
        } else {
          // One accumulator of two N halves, each handed back separately by the epilogue
          // (tempty[0], tempty[1]) and each announced separately to it (tfull[0], tfull[1]).
          //  * Tile start: as soon as half 0 is free, N-slice-0 UMMAs run ahead by up to S
          //    stages while half 1 still drains; the slice-1 UMMAs of those stages follow in
          //    k order once half 1 is free, and only then are the stages released.
          //  * Tile end: for the last S k-blocks the slice-0 UMMAs go first and tfull[0] is
          //    committed before the slice-1 UMMAs, so the epilogue drains half 0 while the
          //    tensor core still works on half 1 and the next tile can start on half 0
          //    without the pipe running dry.
          dtm = tmem_base;
          if (!wait_bar<PAIR == 2>(ptx::smem_u32(&tempty[0]), aph ^ 1u, wctx, kSiteMmaTmemEmpty)) {
            ok = false;
            break;
          }
          ptx::tc_fence_after();
          bool h1 = false;
          int pend_s = 0, pend_kb = 0, npend = 0;
          auto flush = [&]() {
            for (int q = 0; q < npend; ++q) {
              const int st = (pend_s + q) % S;
              issue_sub(st, pend_kb + q, 1);
              release_stage(st);
            }
            npend = 0;
          };
          auto wait_h1 = [&]() -> bool {
            if (h1) return true;
            if (!wait_bar<PAIR == 2>(ptx::smem_u32(&tempty[1]), aph ^ 1u, wctx, kSiteMmaTmemEmpty))
              return false;
            ptx::tc_fence_after();
            h1 = true;
            return true;
          };
          const int tail_from = p.num_kb - S;  // k-blocks at or past this one are skewed
          for (int kb = 0; kb < p.num_kb; ++kb) {
            if (!wait_bar<false>(ptx::smem_u32(&full[s]), ph, wctx, kSiteMmaFull)) {
              ok = false;
              break;
            }
            ptx::tc_fence_after();
            issue_sub(s, kb, 0);
            if (!h1 && ptx::mbar_test_wait_cluster(ptx::smem_u32(&tempty[1]), aph ^ 1u)) {
              ptx::tc_fence_after();
              h1 = true;
            }
            if (h1 && kb < tail_from) {
              flush();
              issue_sub(s, kb, 1);
              release_stage(s);
            } else {
              if (npend == 0) {
                pend_s = s;
                pend_kb = kb;
              }
              if (++npend == S) {
                // Every stage holds slice-0 work only; the producer needs one back.
                if (!wait_h1()) {
                  ok = false;
                  break;
                }
                flush();
              }
            }
            poll_next(kb);
            if (++s == S) {
              s = 0;
              ph ^= 1u;
            }
          }
          if (!ok) break;
          {
            const uint32_t fb0 = ptx::smem_u32(&tfull[0]);
            if (PAIR == 2)
              ptx::umma_commit_pair_mask(fb0, 0x3);
            else
              ptx::umma_commit<1>(fb0);
          }
          if (!wait_h1()) {
            ok = false;
            break;
          }
          flush();
          const uint32_t fb1 = ptx::smem_u32(&tfull[1]);
          if (PAIR == 2)
            ptx::umma_commit_pair_mask(fb1, 0x3);
          else
            ptx::umma_commit<1>(fb1);
        }
        if (!ok) break;
        if constexpr (ACC_BUFS == 2) {
          const uint32_t fb = ptx::smem_u32(&tfull[acc]);
          if (PAIR == 2)
            ptx::umma_commit_pair_mask(fb, 0x3);
          else
            ptx::umma_commit<1>(fb);
        }
        if (!have_next && !sched_read(sslot, sph, next)) {
          ok = false;
          break;
        }
        tile = next;
        ++it;
      }
      if (!ok && issued_any) {
        // Unwinding: every UMMA this thread issued must retire before TMEM is freed.
        ptx::umma_commit<PAIR>(ptx::smem_u32(drain));
        WaitCtx dctx = wctx;
        volatile int no_abort = 0;
        dctx.abort_flag = &no_abort;
        dctx.peer_abort = 0;
        dctx.timeout_ns = 50000000ull;
        wait_bar<false>(ptx::smem_u32(drain), 0u, dctx, kSiteDrain);
      }
    }
  } else {
    // ------------------------------------------------------------------ epilogue warps
    const int q = warp & 3;  // TMEM lanes [32q, 32q+32) are the ones this warp may read
    const int ew = warp - 2;  // epilogue warp index
    // Columns [ccol0, ccol0 + EPI_COLS_PER_WARP) of each tile are this warp's.
    const int ccol0 = (ew >> 2) * Cfg::EPI_COLS_PER_WARP;
    constexpr int EB = Cfg::EPI_BUFS;
    uint8_t *stg0 = epi + ew * (EB * EPI_ROWS * 128);
    const uint32_t tempty_leader =
        (PAIR == 2) ? ptx::mapa(ptx::smem_u32(&tempty[0]), 0u) : ptx::smem_u32(&tempty[0]);
    const float alpha = p.alpha, beta = p.beta;
    // Step-entry gate of the peer stores (see PeerMaps). Announced by one thread per CTA;
    // each warp waits once, here, while the first tile's main loop runs.
    int npeer_live = npeer;
    if (PEERS && npeer > 0 && peers.epoch != 0) {
      if (ew == 0 && lane == 0)
        for (int d = 0; d < npeer; ++d) ptx::st_release_sys_u64(peers.post[d], peers.epoch);
      int okp = 1;
      if (lane == 0) {
        const uint64_t t0 = ptx::globaltimer();
        for (int d = 0; d < npeer && okp; ++d) {
          for (uint32_t n = 0;; ++n) {
            if (ptx::ld_acquire_sys_u64(peers.wait[d]) >= peers.epoch) break;
            if ((n & 15u) == 15u &&
                (*abort_flag || ptx::globaltimer() - t0 > p.timeout_ns)) {
              atomicCAS(&g_dev_status, 0u, kDevTimeout | kSitePeerEntry);
              okp = 0;
              break;
            }
            ptx::nanosleep_ns(128);
          }
        }
      }
      okp = __shfl_sync(0xffffffffu, okp, 0);
      __syncwarp();
      if (!okp) npeer_live = 0;  // this rank's tiles stay local; the status word says why
    }
    int it = 0;
    int chunk_ctr = 0;
    int sslot = 0;
    uint32_t sph = 0;
    int c_prefetched = -1;
    // C tiles are written once and never re-read by the GEMM (see kCEvictFirstMinK).
    const uint64_t c_policy = ptx::l2_policy_evict_first();
    auto store_c = [&](const CUtensorMap *m, uint32_t src, int x, int y) {
      if (p.c_evict_first)
        ptx::tma_store_2d_hint(m, src, x, y, c_policy);
      else
        ptx::tma_store_2d(m, src, x, y);
    };
    // Peer copies of one staged 32 x 64 chunk (rows prow0.., columns pcol..) with 16-byte
    // stores: lane l moves row 4i + l/8, 16-byte group l%8, so every warp store writes four
    // whole 128-byte row segments.
    auto push_peers = [&](const uint8_t *stgp, int prow0, int pcol) {
      const int jj = lane & 7;
      const int gc = pcol + 8 * jj;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int rr = 4 * i + (lane >> 3);
        const int gr = prow0 + rr;
        const uint4 v = *reinterpret_cast<const uint4 *>(stgp + sw128_off(rr, jj));
        if (gr < p.M && gc < p.N) {
          const size_t off = static_cast<size_t>(gr) * p.N + gc;
          for (int d = 0; d < npeer_live; ++d) {
            if (p.c_evict_first)
              ptx::st_global_v4_hint(peers.ptr[d] + off, v, c_policy);
            else
              *reinterpret_cast<uint4 *>(peers.ptr[d] + off) = v;
          }
        }
      }
    };
    // L2 prefetch of the C_in rows this warp will read for `tile` (TMA, no smem).
    auto prefetch_c_rows = [&](int tile_idx) {
      int ptm, ptn;
      decode_tile(tile_idx, p, ptm, ptn);
      const int prow = ptm * Cfg::UMMA_M + static_cast<int>(rank) * CTA_M + EPI_ROWS * q;
      if (prow >= p.M) return;
#pragma unroll 1
      for (int c = ccol0 / EPI_COLS; c < (ccol0 + Cfg::EPI_COLS_PER_WARP) / EPI_COLS; ++c) {
        const int pcol = ptn * BN + c * EPI_COLS;
        if (pcol < p.N) ptx::tma_prefetch_l2_2d(&tmC, pcol, prow);
      }
    };
    for (;;) {
      // One lane takes the tile index and waits for the accumulator; the results are
      // broadcast so the warp stays converged for the .sync.aligned TMEM loads below.
      int ok = 1, tile = -1;
      const int acc = it % ACC_BUFS;
      const uint32_t aph = static_cast<uint32_t>(it / ACC_BUFS) & 1u;
      if (lane == 0) {
        ok = sched_read(sslot, sph, tile) ? 1 : 0;
        if (ok && tile >= 0)
          ok = wait_bar<PAIR == 2>(ptx::smem_u32(&tfull[acc]), aph, wctx, kSiteEpiTmemFull) ? 1 : 0;
      }
      ok = __shfl_sync(0xffffffffu, ok, 0);
      tile = __shfl_sync(0xffffffffu, tile, 0);
      if (!ok || tile < 0) break;
      ptx::tc_fence_after();
      int tm, tn;
      decode_tile(tile, p, tm, tn);
      const int row0 = tm * Cfg::UMMA_M + static_cast<int>(rank) * CTA_M + EPI_ROWS * q;
      const int col0 = tn * BN;
      if (TMA_EPI && beta != 0.0f && lane == 0) {
        // beta != 0: start bringing this warp's 32 rows of C_in into L2 now; for every tile
        // after the first this was already asked for one tile ahead (below).
        if (tile != c_prefetched) prefetch_c_rows(tile);
        // ... and the next tile's, if its index is already in the ring (read, not taken).
        if (ptx::mbar_test_wait_cluster(ptx::smem_u32(&sched_full[sslot]), sph)) {
          const int nt = sched_val[sslot];
          if (nt >= 0) {
            prefetch_c_rows(nt);
            c_prefetched = nt;
          }
        }
      }
      const uint32_t tbase =
          tmem_base + (static_cast<uint32_t>(EPI_ROWS * q) << 16) + static_cast<uint32_t>(acc * BN);
      // With one accumulator, half 1 is announced separately (tfull[1]) after half 0.
      auto wait_half1 = [&]() -> bool {
        int okk = 1;
        if (lane == 0)
          okk = wait_bar<PAIR == 2>(ptx::smem_u32(&tfull[1]), aph, wctx, kSiteEpiTmemFull) ? 1 : 0;
        okk = __shfl_sync(0xffffffffu, okk, 0);
        if (okk) ptx::tc_fence_after();
        return okk != 0;
      };
      if constexpr (SPLITK) {
        // ---- split-K: one tile per cluster, CTA `split` holds the sums of its k-blocks.
        // (1) partial sums -> this CTA's shared memory, fp32 (the pipeline stages are free:
        //     every UMMA of the cluster's only tile has retired). Row r (tile-local) starts
        //     at r * BN * 4 bytes; its 16-byte group g is stored at g ^ (r & 7).
        const uint32_t part = sA0;
        const int r_loc = EPI_ROWS * q + lane;
        const uint32_t prow = part + static_cast<uint32_t>(r_loc) * (BN * 4);
        const uint32_t rsw = static_cast<uint32_t>(r_loc & 7);
#pragma unroll 1
        for (int c = ccol0 / 32; c < (ccol0 + Cfg::EPI_COLS_PER_WARP) / 32; c += 2) {
          uint32_t v[64];
          ptx::tmem_ld_32x32b_x32(tbase + 32 * c, *reinterpret_cast<uint32_t(*)[32]>(&v[0]));
          ptx::tmem_ld_32x32b_x32(tbase + 32 * c + 32, *reinterpret_cast<uint32_t(*)[32]>(&v[32]));
          ptx::tmem_ld_wait();
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const uint32_t g = static_cast<uint32_t>(8 * c + j);
            ptx::st_shared_v4(prow + ((g ^ rsw) << 4), v[4 * j], v[4 * j + 1], v[4 * j + 2],
                              v[4 * j + 3]);
          }
        }
        // (2) announce this warp's rows to every CTA of the cluster, then wait for all of
        //     theirs (bounded).
        ptx::tc_fence_before();
        ptx::fence_acq_rel_cluster();
        __syncwarp();
        if (lane == 0)
          for (int t = 0; t < ksplit; ++t)
            ptx::mbar_arrive_cluster(ptx::mapa(ptx::smem_u32(red_ready), static_cast<uint32_t>(t)));
        int okr = 1;
        if (lane == 0)
          okr = wait_bar<true>(ptx::smem_u32(red_ready), 0u, wctx, kSiteSplitReduce) ? 1 : 0;
        okr = __shfl_sync(0xffffffffu, okr, 0);
        ptx::fence_acq_rel_cluster();
        // (3) reduce-scatter: the tile's (128/32) x (BN/64) chunks of 32 x 64 go round robin
        //     to the cluster's 4 * ksplit epilogue warps; each sums the ksplit partials of its
        //     chunk in split order (fixed, so results are bit-stable), applies alpha / beta,
        //     rounds once to half and TMA-stores the chunk. Reads are coalesced: lanes
        //     16h..16h+15 take one row's 64 columns (256 contiguous bytes), so a warp load
        //     covers two rows; lane l holds rows 2i + l/16 (i < 16), columns 4(l%16)..+3.
        const int workers = Cfg::EPI_WARPS * ksplit;
        const int lhalf = lane >> 4, lg = lane & 15;
#pragma unroll 1
        for (int ci = Cfg::EPI_WARPS * split + ew; okr && ci < 4 * (BN / 64); ci += workers) {
          const int rb = ci & 3, cb = ci >> 2;
          const int gcol = col0 + 64 * cb + 4 * lg;  // this lane's first column
          uint8_t *stg = stg0 + (chunk_ctr % EB) * (EPI_ROWS * 128);
          ++chunk_ctr;
          if (lane == 0) ptx::bulk_wait_group_read<EB - 1>();
          __syncwarp();
          // Two halves of 16 rows each, fully unrolled so the 32 sums stay in registers (a
          // 64-float array indexed from a partly unrolled loop lives in local memory and
          // made one chunk's reduction ~20 K cycles).
#pragma unroll 1
          for (int h = 0; h < 2; ++h) {
            float f[32];
#pragma unroll 1
            for (int t = 0; t < ksplit; ++t) {
              const uint32_t tb = (t == split) ? part : ptx::mapa(part, static_cast<uint32_t>(t));
              float4 x[8];
#pragma unroll
              for (int i = 0; i < 8; ++i) {
                const int rr = 32 * rb + 2 * (8 * h + i) + lhalf;
                const uint32_t g = static_cast<uint32_t>(16 * cb + lg);
                const uint32_t a = tb + static_cast<uint32_t>(rr) * (BN * 4) +
                                   ((g ^ static_cast<uint32_t>(rr & 7)) << 4);
                x[i] = (t == split) ? ptx::ld_shared_v4f(a) : ptx::ld_shared_cluster_v4f(a);
              }
#pragma unroll
              for (int i = 0; i < 8; ++i) {
                if (t == 0) {
                  f[4 * i] = x[i].x; f[4 * i + 1] = x[i].y; f[4 * i + 2] = x[i].z; f[4 * i + 3] = x[i].w;
                } else {
                  f[4 * i] += x[i].x; f[4 * i + 1] += x[i].y; f[4 * i + 2] += x[i].z; f[4 * i + 3] += x[i].w;
                }
              }
            }
#pragma unroll
            for (int e = 0; e < 32; ++e) f[e] *= alpha;
            if (beta != 0.0f) {
#pragma unroll
              for (int i = 0; i < 8; ++i) {
                const int grow = tm * CTA_M + 32 * rb + 2 * (8 * h + i) + lhalf;
                // ldc % 8 == 0: a group of 4 halves that starts inside a row ends inside its
                // stride (pad columns of a restrided C hold zeros and are never stored)
                if (grow < p.M && gcol < p.N) {
                  const uint2 u = __ldg(reinterpret_cast<const uint2 *>(
                      p.C + static_cast<long long>(grow) * p.ldc + gcol));
                  const float2 c0 = __half22float2(*reinterpret_cast<const __half2 *>(&u.x));
                  const float2 c1 = __half22float2(*reinterpret_cast<const __half2 *>(&u.y));
                  f[4 * i] = fmaf(beta, c0.x, f[4 * i]);
                  f[4 * i + 1] = fmaf(beta, c0.y, f[4 * i + 1]);
                  f[4 * i + 2] = fmaf(beta, c1.x, f[4 * i + 2]);
                  f[4 * i + 3] = fmaf(beta, c1.y, f[4 * i + 3]);
                }
              }
            }
            // staging layout of the TMA store: row r's 16-byte group j at r*128 + (j ^ (r&7))*16;
            // this lane's 4 halves are the (lg&1) half of group lg/2.
#pragma unroll
            for (int i = 0; i < 8; ++i) {
              const int r = 2 * (8 * h + i) + lhalf;
              uint2 w;
              w.x = pack_half2(f[4 * i], f[4 * i + 1]);
              w.y = pack_half2(f[4 * i + 2], f[4 * i + 3]);
              *reinterpret_cast<uint2 *>(stg + sw128_off(r, lg >> 1) + 8 * (lg & 1)) = w;
            }
          }
          ptx::fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            const int srow = tm * CTA_M + 32 * rb;
            const int scol = col0 + 64 * cb;
            if (srow < p.M && scol < p.N) store_c(&tmC, ptx::smem_u32(stg), scol, srow);
            ptx::bulk_commit_group();
          }
        }
        // (4) this warp no longer reads any CTA's partials: tell every CTA, and do not let
        //     this CTA exit (freeing its shared memory) before the whole cluster is done.
        ptx::fence_acq_rel_cluster();
        __syncwarp();
        if (lane == 0)
          for (int t = 0; t < ksplit; ++t)
            ptx::mbar_arrive_cluster(ptx::mapa(ptx::smem_u32(red_done), static_cast<uint32_t>(t)));
        int okd = 1;
        if (lane == 0)
          okd = wait_bar<true>(ptx::smem_u32(red_done), 0u, wctx, kSiteSplitReduce) ? 1 : 0;
        okd = __shfl_sync(0xffffffffu, okd, 0);
        if (!okr || !okd) break;
        ++it;
        continue;
      }
      if constexpr (ACC_BUFS == 1 && TMA_EPI && Cfg::EPI_WARPS == 8 && !SPLITK) {
        if (wide_drain) {
          // Each half: two batches of 64 TMEM columns into packed halves, the half handed
          // back right after the second wait, then two 32 x 64 chunks through this warp's
          // single staging buffer.
          const int g = ew >> 2;
          bool aborted = false;
#pragma unroll 1
          for (int h = 0; h < 2; ++h) {
            if (h == 1 && !wait_half1()) {
              aborted = true;
              break;
            }
            const uint32_t ta = tbase + static_cast<uint32_t>(h * (BN / 2) + g * 128);
            uint32_t P[64];
#pragma unroll
            for (int b = 0; b < 2; ++b) {
              uint32_t v[64];
              ptx::tmem_ld_32x32b_x32(ta + 64 * b, *reinterpret_cast<uint32_t(*)[32]>(&v[0]));
              ptx::tmem_ld_32x32b_x32(ta + 64 * b + 32, *reinterpret_cast<uint32_t(*)[32]>(&v[32]));
              ptx::tmem_ld_wait();
#pragma unroll
              for (int i = 0; i < 32; ++i)
                P[32 * b + i] = pack_half2(alpha * __uint_as_float(v[2 * i]),
                                           alpha * __uint_as_float(v[2 * i + 1]));
            }
            ptx::tc_fence_before();
            __syncwarp();
            if (lane == 0) {
              const uint32_t tb = tempty_leader + static_cast<uint32_t>(h) * 8u;
              if (PAIR == 2)
                ptx::mbar_arrive_remote(tb);
              else
                ptx::mbar_arrive(tb);
            }
            const uint32_t stg_base = ptx::smem_u32(stg0) + static_cast<uint32_t>(lane) * 128u;
            const uint32_t sw = static_cast<uint32_t>(lane & 7);
#pragma unroll
            for (int ch = 0; ch < 2; ++ch, ++chunk_ctr) {
              // The TMA store of the previous chunk must have read the staging buffer.
              if (lane == 0) ptx::bulk_wait_group_read<0>();
              __syncwarp();
#pragma unroll
              for (int j = 0; j < 8; ++j)
                ptx::st_shared_v4(stg_base + ((static_cast<uint32_t>(j) ^ sw) << 4),
                                  P[32 * ch + 4 * j + 0], P[32 * ch + 4 * j + 1],
                                  P[32 * ch + 4 * j + 2], P[32 * ch + 4 * j + 3]);
              ptx::fence_proxy_async_smem();
              __syncwarp();
              const int ccol = col0 + h * (BN / 2) + g * 128 + ch * EPI_COLS;
              if (lane == 0) {
                if (row0 < p.M && ccol < p.N) store_c(&tmC, ptx::smem_u32(stg0), ccol, row0);
                ptx::bulk_commit_group();
              }
              if (npeer_live > 0) push_peers(stg0, row0, ccol);
            }
          }
          if (aborted) break;
          ++it;
          continue;
        }
      }
      if constexpr (ACC_BUFS == 1 && TMA_EPI && Cfg::EPI_WARPS == 4) {
        if (beta == 0.0f) {
          // Single accumulator: drain each N half into registers as packed halves, give that
          // half of TMEM back at once, then store it through the swizzled staging buffers
          // with TMA stores.
          bool aborted = false;
#pragma unroll 1
          for (int h = 0; h < 2; ++h) {
            if (h == 1 && !wait_half1()) {
              aborted = true;
              break;
            }
            // Three batches of 32-column TMEM loads (128 + 64 + 64 columns), one wait each;
            // the half goes back to the UMMA issuer right after the last wait, before the
            // last conversion and any store.
            const uint32_t ta = tbase + static_cast<uint32_t>(h * (BN / 2));
            uint32_t P[128];
            {
              uint32_t v[128];
#pragma unroll
              for (int b = 0; b < 4; ++b)
                ptx::tmem_ld_32x32b_x32(ta + 32 * b, *reinterpret_cast<uint32_t(*)[32]>(&v[32 * b]));
              ptx::tmem_ld_wait();
#pragma unroll
              for (int i = 0; i < 64; ++i)
                P[i] = pack_half2(alpha * __uint_as_float(v[2 * i]),
                                  alpha * __uint_as_float(v[2 * i + 1]));
            }
            uint32_t v[64];
            ptx::tmem_ld_32x32b_x32(ta + 128, *reinterpret_cast<uint32_t(*)[32]>(&v[0]));
            ptx::tmem_ld_32x32b_x32(ta + 160, *reinterpret_cast<uint32_t(*)[32]>(&v[32]));
            ptx::tmem_ld_wait();
#pragma unroll
            for (int i = 0; i < 32; ++i)
              P[64 + i] = pack_half2(alpha * __uint_as_float(v[2 * i]),
                                     alpha * __uint_as_float(v[2 * i + 1]));
            ptx::tmem_ld_32x32b_x32(ta + 192, *reinterpret_cast<uint32_t(*)[32]>(&v[0]));
            ptx::tmem_ld_32x32b_x32(ta + 224, *reinterpret_cast<uint32_t(*)[32]>(&v[32]));
            ptx::tmem_ld_wait();
            ptx::tc_fence_before();
            __syncwarp();
            if (lane == 0) {
              const uint32_t tb = tempty_leader + static_cast<uint32_t>(h) * 8u;
              if (PAIR == 2)
                ptx::mbar_arrive_remote(tb);
              else
                ptx::mbar_arrive(tb);
            }
#pragma unroll
            for (int i = 0; i < 32; ++i)
              P[96 + i] = pack_half2(alpha * __uint_as_float(v[2 * i]),
                                     alpha * __uint_as_float(v[2 * i + 1]));
            const uint32_t stg_base = ptx::smem_u32(stg0) + static_cast<uint32_t>(lane) * 128u;
            const uint32_t sw = static_cast<uint32_t>(lane & 7);
#pragma unroll
            for (int ch = 0; ch < (BN / 2) / EPI_COLS; ++ch, ++chunk_ctr) {
              const uint32_t buf = static_cast<uint32_t>(chunk_ctr & 1) * (EPI_ROWS * 128);
              // The TMA store that used this staging buffer two chunks ago must have read it.
              if (lane == 0) ptx::bulk_wait_group_read<1>();
              __syncwarp();
#pragma unroll
              for (int j = 0; j < 8; ++j)
                ptx::st_shared_v4(stg_base + buf + ((static_cast<uint32_t>(j) ^ sw) << 4),
                                  P[32 * ch + 4 * j + 0], P[32 * ch + 4 * j + 1],
                                  P[32 * ch + 4 * j + 2], P[32 * ch + 4 * j + 3]);
              ptx::fence_proxy_async_smem();
              __syncwarp();
              const int ccol = col0 + h * (BN / 2) + ch * EPI_COLS;
              if (lane == 0) {
                if (row0 < p.M && ccol < p.N) {
                  store_c(&tmC, ptx::smem_u32(stg0) + buf, ccol, row0);
                }
                ptx::bulk_commit_group();
              }
              if (npeer_live > 0) push_peers(stg0 + buf, row0, ccol);
            }
          }
          if (aborted) break;
          ++it;
          continue;
        }
      }
      bool aborted_chunks = false;
      constexpr int NCH = BN / EPI_COLS;
      const bool unit_alpha = (alpha == 1.0f);
      const int cbeg = ccol0 / EPI_COLS, cend = (ccol0 + Cfg::EPI_COLS_PER_WARP) / EPI_COLS;
      // beta != 0 with TMA stores: C_in is read with coalesced 16-byte loads (lane l takes
      // row 4i + l/8, 16-byte group l%8), one chunk ahead, and transposed through the
      // staging buffer so that each lane gets its own row.
      const bool c_in = TMA_EPI && beta != 0.0f;
      uint4 cin[8];
      auto load_c = [&](int c) {
        const int gc = col0 + c * EPI_COLS + 8 * (lane & 7);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const int gr = row0 + 4 * i + (lane >> 3);
          if (gr < p.M && gc < p.N)
            cin[i] = __ldg(reinterpret_cast<const uint4 *>(p.C + static_cast<long long>(gr) * p.ldc + gc));
          else
            cin[i] = make_uint4(0u, 0u, 0u, 0u);
        }
      };
      if (c_in) load_c(cbeg);
      // With 4 warps (255 registers each) the TMEM loads run one chunk ahead of the
      // conversion and the stores; tcgen05.wait::ld waits for every load issued before it,
      // so the next chunk's loads go out only after this chunk's words were consumed. The
      // 8-warp flavours (168 registers) load each chunk when they reach it.
      constexpr bool kPipe = Cfg::EPI_WARPS == 4;
      uint32_t vn[kPipe ? 64 : 1];
      auto issue_ld = [&](int c) {
        if constexpr (kPipe) {
          ptx::tmem_ld_32x32b_x32(tbase + c * EPI_COLS, *reinterpret_cast<uint32_t(*)[32]>(&vn[0]));
          ptx::tmem_ld_32x32b_x32(tbase + c * EPI_COLS + 32,
                                  *reinterpret_cast<uint32_t(*)[32]>(&vn[32]));
        }
      };
      if (!(ACC_BUFS == 1 && cbeg == NCH / 2)) issue_ld(cbeg);
#pragma unroll 1
      for (int c = cbeg; c < cend; ++c, ++chunk_ctr) {
        if (ACC_BUFS == 1 && c == NCH / 2) {  // half 1 is announced separately
          if (!wait_half1()) {
            aborted_chunks = true;
            break;
          }
          issue_ld(c);  // (its first chunk could not be loaded ahead)
        }
        float f[64];
        if constexpr (kPipe) {
          ptx::tmem_ld_wait();
          if (unit_alpha) {
#pragma unroll
            for (int i = 0; i < 64; ++i) f[i] = __uint_as_float(vn[i]);
          } else {
#pragma unroll
            for (int i = 0; i < 64; ++i) f[i] = alpha * __uint_as_float(vn[i]);
          }
          if (c + 1 < cend && !(ACC_BUFS == 1 && c + 1 == NCH / 2)) issue_ld(c + 1);
        } else {
          uint32_t v[64];
          ptx::tmem_ld_32x32b_x32(tbase + c * EPI_COLS, *reinterpret_cast<uint32_t(*)[32]>(&v[0]));
          ptx::tmem_ld_32x32b_x32(tbase + c * EPI_COLS + 32,
                                  *reinterpret_cast<uint32_t(*)[32]>(&v[32]));
          ptx::tmem_ld_wait();
          if (unit_alpha) {
#pragma unroll
            for (int i = 0; i < 64; ++i) f[i] = __uint_as_float(v[i]);
          } else {
#pragma unroll
            for (int i = 0; i < 64; ++i) f[i] = alpha * __uint_as_float(v[i]);
          }
        }
        const bool last_of_half = (ACC_BUFS == 1) && (c == NCH / 2 - 1);
        if (c == cend - 1 || last_of_half) {
          // Accumulator (or, with one accumulator, one N half of it) fully read: hand it
          // back to the UMMA issuer.
          ptx::tc_fence_before();
          __syncwarp();
          if (lane == 0) {
            const int which = (ACC_BUFS == 1) ? (last_of_half ? 0 : 1) : acc;
            const uint32_t tb = tempty_leader + static_cast<uint32_t>(which) * 8u;
            if (PAIR == 2)
              ptx::mbar_arrive_remote(tb);
            else
              ptx::mbar_arrive(tb);
          }
        }
        const int ccol = col0 + c * EPI_COLS;
        uint8_t *stg = stg0 + (chunk_ctr % EB) * (EPI_ROWS * 128);

        if (TMA_EPI) {
          // The TMA store that used this staging buffer EB chunks ago must have read it.
          if (lane == 0) ptx::bulk_wait_group_read<EB - 1>();
          __syncwarp();
          if (c_in) {
#pragma unroll
            for (int i = 0; i < 8; ++i)
              *reinterpret_cast<uint4 *>(stg + sw128_off(4 * i + (lane >> 3), lane & 7)) = cin[i];
            __syncwarp();
            if (c + 1 < cend) load_c(c + 1);
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              // N % 8 == 0: a 16-byte group is wholly inside or outside C (zeros outside)
              const uint4 u = *reinterpret_cast<const uint4 *>(stg + sw128_off(lane, j));
              const __half2 *h = reinterpret_cast<const __half2 *>(&u);
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                const float2 cf = __half22float2(h[e]);
                f[8 * j + 2 * e] = fmaf(beta, cf.x, f[8 * j + 2 * e]);
                f[8 * j + 2 * e + 1] = fmaf(beta, cf.y, f[8 * j + 2 * e + 1]);
              }
            }
          }
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            uint4 w;
            w.x = pack_half2(f[8 * j + 0], f[8 * j + 1]);
            w.y = pack_half2(f[8 * j + 2], f[8 * j + 3]);
            w.z = pack_half2(f[8 * j + 4], f[8 * j + 5]);
            w.w = pack_half2(f[8 * j + 6], f[8 * j + 7]);
            *reinterpret_cast<uint4 *>(stg + sw128_off(lane, j)) = w;
          }
          ptx::fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            if (row0 < p.M && ccol < p.N) {
              store_c(&tmC, ptx::smem_u32(stg), ccol, row0);
            }
            ptx::bulk_commit_group();  // one group per chunk, empty when nothing was stored
          }
          if (npeer_live > 0) push_peers(stg, row0, ccol);
        } else {
          // C's rows are not 16-byte aligned: stage through smem, then coalesced 2-byte
          // accesses (lanes along a row), predicated on the M/N edges.
          __syncwarp();
          __half *sh = reinterpret_cast<__half *>(stg);
          if (beta != 0.0f) {
#pragma unroll 1
            for (int rr = 0; rr < EPI_ROWS; ++rr) {
              const int gr = row0 + rr;
#pragma unroll
              for (int h = 0; h < 2; ++h) {
                const int cc = lane + 32 * h;
                const int gc = ccol + cc;
                __half val = __float2half(0.0f);
                if (gr < p.M && gc < p.N) val = p.C[static_cast<long long>(gr) * p.N + gc];
                sh[(sw128_off(rr, cc >> 3) >> 1) + (cc & 7)] = val;
              }
            }
            __syncwarp();
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              const uint4 u = *reinterpret_cast<const uint4 *>(stg + sw128_off(lane, j));
              const __half2 *h = reinterpret_cast<const __half2 *>(&u);
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                const float2 cf = __half22float2(h[e]);
                f[8 * j + 2 * e] = fmaf(beta, cf.x, f[8 * j + 2 * e]);
                f[8 * j + 2 * e + 1] = fmaf(beta, cf.y, f[8 * j + 2 * e + 1]);
              }
            }
          }
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            uint4 w;
            w.x = pack_half2(f[8 * j + 0], f[8 * j + 1]);
            w.y = pack_half2(f[8 * j + 2], f[8 * j + 3]);
            w.z = pack_half2(f[8 * j + 4], f[8 * j + 5]);
            w.w = pack_half2(f[8 * j + 6], f[8 * j + 7]);
            *reinterpret_cast<uint4 *>(stg + sw128_off(lane, j)) = w;
          }
          __syncwarp();
#pragma unroll 1
          for (int rr = 0; rr < EPI_ROWS; ++rr) {
            const int gr = row0 + rr;
            if (gr >= p.M) break;
#pragma unroll
            for (int h = 0; h < 2; ++h) {
              const int cc = lane + 32 * h;
              const int gc = ccol + cc;
              if (gc < p.N)
                p.C[static_cast<long long>(gr) * p.N + gc] = sh[(sw128_off(rr, cc >> 3) >> 1) + (cc & 7)];
            }
          }
        }
      }
      if (aborted_chunks) break;
      ++it;
    }
    if (TMA_EPI && lane == 0) ptx::bulk_wait_group<0>();
    // Stores into peers' memory: complete and ordered system-wide before the CTA exits.
    if (npeer > 0) __threadfence_system();
    __syncwarp();
  }

  // ------------------------------------------------------------------ teardown
  if (*abort_flag) ptx::nanosleep_ns(20000);  // unwinding: let stray copies land
  ptx::tc_fence_before();
  __syncthreads();
  if (clustered) ptx::cluster_sync();
  if (warp == 1) {
    __syncwarp();
    ptx::tc_fence_after();
    ptx::tmem_dealloc<PAIR>(tmem_base, Cfg::TMEM_COLS);
  }
#endif
}

// ============================================================================ other kernels
// Scalar kernel (K == 0, and hgemm_launch_noalloc with a pointer off a 16-byte boundary):
// 64x64 output tile per block, 4x4 per thread, fp32 accumulation in increasing k, same
// alpha/beta/rounding rules as above.
__global__ void __launch_bounds__(256) hgemm_simt_kernel(const __half *__restrict__ A,
                                                         const __half *__restrict__ B,
                                                         __half *__restrict__ C, int M, int N,
                                                         int K, float alpha, float beta) {
  __shared__ float sa[16][64 + 4];
  __shared__ float sb[16][64 + 4];
  const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
  const int m0 = blockIdx.y * 64, n0 = blockIdx.x * 64;
  float acc[4][4] = {};
  for (int k0 = 0; k0 < K; k0 += 16) {
    for (int i = threadIdx.x; i < 16 * 64; i += 256) {
      const int kk = i / 64, mm = i % 64;
      const int gm = m0 + mm, gk = k0 + kk;
      sa[kk][mm] = (gm < M && gk < K) ? __half2float(A[static_cast<long long>(gm) * K + gk]) : 0.f;
      const int gn = n0 + mm;
      sb[kk][mm] = (gk < K && gn < N) ? __half2float(B[static_cast<long long>(gk) * N + gn]) : 0.f;
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < 16; ++kk) {
      float a[4], b[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) a[i] = sa[kk][ty + 16 * i];
#pragma unroll
      for (int j = 0; j < 4; ++j) b[j] = sb[kk][tx + 16 * j];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int gm = m0 + ty + 16 * i;
    if (gm >= M) continue;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int gn = n0 + tx + 16 * j;
      if (gn >= N) continue;
      const long long o = static_cast<long long>(gm) * N + gn;
      float v = alpha * acc[i][j];
      if (beta != 0.0f) v = fmaf(beta, __half2float(C[o]), v);
      C[o] = __float2half_rn(v);
    }
  }
}

// ---------------------------------------------------------------- restride / compact
// HBM-bound copies between a row-major matrix whose rows are not 16-byte aligned (row length
// `cols` halves, cols % 8 != 0) and a copy with a 16-byte row stride `ld` (ld % 8 == 0), the
// layout TMA needs. Every thread moves one 16-byte group of 8 halves with one 16-byte store;
// the 8 source halves, which start at an arbitrary even byte offset, come from the (at most
// two) aligned 16-byte blocks that contain the first and the last of them, merged with funnel
// shifts. Both blocks contain an element that is read, so no load reaches past the matrix.

// 16 bytes starting `shift` bytes (even, < 16) into the 32 bytes lo:hi. The shift depends on
// the row only (group starts are 16 bytes apart), so it is uniform across most warps.
__device__ __forceinline__ uint4 extract16(const uint4 lo, const uint4 hi, uint32_t shift) {
  const uint32_t b = (shift & 3u) * 8u;
  switch (shift >> 2) {
    case 0: return make_uint4(__funnelshift_r(lo.x, lo.y, b), __funnelshift_r(lo.y, lo.z, b),
                              __funnelshift_r(lo.z, lo.w, b), __funnelshift_r(lo.w, hi.x, b));
    case 1: return make_uint4(__funnelshift_r(lo.y, lo.z, b), __funnelshift_r(lo.z, lo.w, b),
                              __funnelshift_r(lo.w, hi.x, b), __funnelshift_r(hi.x, hi.y, b));
    case 2: return make_uint4(__funnelshift_r(lo.z, lo.w, b), __funnelshift_r(lo.w, hi.x, b),
                              __funnelshift_r(hi.x, hi.y, b), __funnelshift_r(hi.y, hi.z, b));
    default: return make_uint4(__funnelshift_r(lo.w, hi.x, b), __funnelshift_r(hi.x, hi.y, b),
                               __funnelshift_r(hi.y, hi.z, b), __funnelshift_r(hi.z, hi.w, b));
  }
}

// `n` (1..8) consecutive halves starting at p, in the low lanes of a 16-byte group; the rest
// of the group is zero.
__device__ __forceinline__ uint4 load_halves(const __half *p, int n) {
  const uintptr_t a0 = reinterpret_cast<uintptr_t>(p);
  const uintptr_t a1 = a0 + 2u * static_cast<uintptr_t>(n - 1);
  const uint4 lo = __ldg(reinterpret_cast<const uint4 *>(a0 & ~uintptr_t(15)));
  const uint4 hi = ((a1 & ~uintptr_t(15)) != (a0 & ~uintptr_t(15)))
                       ? __ldg(reinterpret_cast<const uint4 *>(a1 & ~uintptr_t(15)))
                       : lo;
  uint4 v = extract16(lo, hi, static_cast<uint32_t>(a0 & 15u));
  if (n < 8) {
    uint32_t *vw = reinterpret_cast<uint32_t *>(&v);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int e = 2 * j;  // halves e, e + 1 live in word j
      if (e >= n) vw[j] = 0u;
      else if (e + 1 >= n) vw[j] &= 0xffffu;
    }
  }
  return v;
}

// Up to three restrides in one launch (A, B and C of one GEMM): job j covers groups
// [first[j], first[j + 1]) of the grid-stride range.
struct RestrideJobs {
  const __half *src[3];
  __half *dst[3];
  int rows[3], cols[3], ld[3];
  long long first[4];
  long long total;  // first[n]
  int n;
};
__global__ void __launch_bounds__(256) restride_kernel(const RestrideJobs jb) {
  const long long total = jb.total;
  for (long long g = blockIdx.x * 256LL + threadIdx.x; g < total; g += 256LL * gridDim.x) {
    // The job's fields, selected with constant indices (an array of kernel parameters
    // indexed at run time would be copied to local memory).
    const __half *src = jb.src[0];
    __half *dst = jb.dst[0];
    int cols = jb.cols[0], ld = jb.ld[0];
    long long first = 0;
#pragma unroll
    for (int j = 1; j < 3; ++j) {
      if (j < jb.n && g >= jb.first[j]) {
        src = jb.src[j];
        dst = jb.dst[j];
        cols = jb.cols[j];
        ld = jb.ld[j];
        first = jb.first[j];
      }
    }
    const long long gj = g - first;
    const int gpr = ld / 8;
    const int r = static_cast<int>(gj / gpr);
    const int c = static_cast<int>(gj - static_cast<long long>(r) * gpr) * 8;
    const int n = min(8, cols - c);
    const uint4 v = n > 0 ? load_halves(src + static_cast<long long>(r) * cols + c, n)
                          : make_uint4(0u, 0u, 0u, 0u);
    *reinterpret_cast<uint4 *>(dst + static_cast<long long>(r) * ld + c) = v;
  }
}

// Inverse of restride_kernel: rows x cols out of a buffer with row stride `ld` into a
// row-major rows x cols matrix `dst` (16-byte aligned). Thread t writes elements
// [8t, 8t + 8) of dst with one 16-byte store; groups that cross a row end, and the last
// partial group, take their halves one by one.
__global__ void __launch_bounds__(256) compact_kernel(const __half *__restrict__ src,
                                                      __half *__restrict__ dst, int rows,
                                                      int cols, int ld) {
  const long long total = static_cast<long long>(rows) * cols;
  const long long groups = (total + 7) / 8;
  for (long long t = blockIdx.x * 256LL + threadIdx.x; t < groups; t += 256LL * gridDim.x) {
    const long long o = 8 * t;
    const long long r = o / cols;
    const int c = static_cast<int>(o - r * cols);
    if (c + 8 <= cols && o + 8 <= total) {
      *reinterpret_cast<uint4 *>(dst + o) = load_halves(src + r * ld + c, 8);
    } else {
      const int n = static_cast<int>(min(8LL, total - o));
      for (int e = 0; e < n; ++e) {
        const long long oe = o + e;
        const long long re = oe / cols;
        dst[oe] = src[re * ld + (oe - re * cols)];
      }
    }
  }
}

// The only wait is on a barrier nothing arrives on; it must give up after `timeout_ns`.
__global__ void wait_selftest_kernel(unsigned long long timeout_ns, int *out) {
  __shared__ __align__(8) uint64_t bar;
  __shared__ int flag;
  if (threadIdx.x == 0) {
    ptx::mbar_init(ptx::smem_u32(&bar), 1);
    flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    WaitCtx w;
    w.abort_flag = &flag;
    w.peer_abort = 0;
    w.timeout_ns = timeout_ns;
    const bool ok = wait_bar<false>(ptx::smem_u32(&bar), 0u, w, kSiteSelftest);
    *out = ok ? HGEMM_OK : HGEMM_ERR_DEVICE_TIMEOUT;
  }
}

// Cross-GPU barrier of a row-sharded step. Every rank owns an array of 2 x kMaxRanksBarrier
// 64-bit epochs: slot r is the last step that rank r has finished (its GEMM kernel, whose
// peer stores were completed and fenced system-wide, precedes this kernel in the stream),
// slot kMaxRanksBarrier + r the last step that rank r has entered (see PeerMaps). Lane i
// announces the epoch to rank i (release store, system scope, through the CUDA IPC mapping
// of rank i's array), then waits until rank i has announced it here (acquire load), at
// most timeout_ns; a wait that runs out records its site in the device status word and
// returns.
constexpr int kMaxRanksBarrier = 8;
static_assert(kMaxPeers + 1 == kMaxRanksBarrier, "one flag slot per rank");
struct BarrierArgs {
  unsigned long long *flags[kMaxRanksBarrier];  // rank i's flag array as mapped here
  int rank, nranks;
  int slot_base;  // 0: step-exit epochs; kMaxRanksBarrier: step-entry epochs
};
__global__ void peer_barrier_kernel(const BarrierArgs a, unsigned long long epoch,
                                    unsigned long long timeout_ns) {
  const int i = threadIdx.x;
  if (i >= a.nranks || i == a.rank) return;
  ptx::st_release_sys_u64(a.flags[i] + a.slot_base + a.rank, epoch);
  const unsigned long long *mine = a.flags[a.rank] + a.slot_base + i;
  const unsigned long long t0 = ptx::globaltimer();
  for (unsigned it = 0;; ++it) {
    if (ptx::ld_acquire_sys_u64(mine) >= epoch) return;
    if ((it & 15u) == 15u && ptx::globaltimer() - t0 > timeout_ns) {
      atomicCAS(&g_dev_status, 0u,
                kDevTimeout | (a.slot_base ? kSitePeerEntry : kSitePeerBarrier));
      return;
    }
    ptx::nanosleep_ns(64);
  }
}

// ============================================================================ host side
namespace {

thread_local int t_last_status = HGEMM_OK;
std::atomic<unsigned long long> g_timeout_ns{2000000000ull};

int set_status(int s) {
  t_last_status = s;
  return s;
}

using EncodeTiledFn = CUresult (*)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *,
                                   const cuuint64_t *, const cuuint64_t *, const cuuint32_t *,
                                   const cuuint32_t *, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = [] {
    void *ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &ptr, 12000, cudaEnableDefault,
                                         &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      ptr = nullptr;
    return reinterpret_cast<EncodeTiledFn>(ptr);
  }();
  return fn;
}

// Row-major rows x cols half matrix with row stride `ld` halves -> 2-D tensor map with a
// box of box_rows x box_cols, 128-byte swizzle, zero fill outside the matrix.
bool encode_2d(CUtensorMap *map, const void *ptr, int rows, int cols, long long ld, int box_rows,
               int box_cols) {
  EncodeTiledFn enc = encode_fn();
  if (!enc) return false;
  cuuint64_t gdim[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  cuuint64_t gstride[1] = {static_cast<cuuint64_t>(ld) * sizeof(__half)};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(box_cols), static_cast<cuuint32_t>(box_rows)};
  cuuint32_t estride[2] = {1, 1};
  return enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void *>(ptr), gdim, gstride, box,
             estride, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// B (K x N row-major, row stride ld halves) as a 4-D tensor for the producer's one-instruction
// stage load: dimensions (64 columns of a block, K, 64-column blocks of one UMMA slice, slices)
// with strides (2 bytes, ld * 2, 128 bytes, umma_n * 2 bytes). Dimensions 2 and 3 alias: block
// c2 of slice c3 is column block c2 + c3 * umma_n / 64, which the map cannot bounds-check, so
// it is only used when every tile is whole in N (N % tile_n == 0). The box of
// 64 x 64 x boxes x slices lands as consecutive 8 KB blocks, the layout of the 2-D loads.
bool encode_b4(CUtensorMap *map, const void *ptr, int K, int N, long long ld, int umma_n,
               int boxes, int slices) {
  EncodeTiledFn enc = encode_fn();
  if (!enc) return false;
  cuuint64_t gdim[4] = {64, static_cast<cuuint64_t>(K), static_cast<cuuint64_t>(N / 64),
                        static_cast<cuuint64_t>(N / umma_n)};
  cuuint64_t gstride[3] = {static_cast<cuuint64_t>(ld) * sizeof(__half), 128,
                           static_cast<cuuint64_t>(umma_n) * sizeof(__half)};
  cuuint32_t box[4] = {64, static_cast<cuuint32_t>(BK), static_cast<cuuint32_t>(boxes),
                       static_cast<cuuint32_t>(slices)};
  cuuint32_t estride[4] = {1, 1, 1, 1};
  return enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4, const_cast<void *>(ptr), gdim, gstride, box,
             estride, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// ---------------------------------------------------------------- kernel table
enum TileId {
  kT256x512 = 0,
  kT256x256 = 1,
  kT256x128 = 2,
  kT128x256 = 3,
  kT128x128 = 4,
  kT128x64 = 5,
  kNumTiles = 6
};
// Kernel flavours of one tile: TMA-store epilogue with 4 or 8 warps, the SIMT-store epilogue
// (N % 8 != 0, 4 warps), split-K (one-CTA tiles, TMA stores, 4 warps), and the peer-copy
// epilogues of the fused multi-GPU path (256x512 and 256x256 only). An 8-warp flavour that
// is not instantiated (128x64) maps to the 4-warp one; a missing split-K or peer flavour is
// reported by kernel_for returning nullptr.
enum Flavor {
  kFlavE4 = 0,
  kFlavE8 = 1,
  kFlavSimt = 2,
  kFlavSplit = 3,
  kFlavPeerE4 = 4,  // TMA-store epilogues that also copy every tile to peer buffers
  kFlavPeerE8 = 5,
  kNumFlavors = 6
};
struct FlavorInfo {
  int stages, smem, threads, epi_warps;
};
struct TileInfo {
  int pair, bn, acc_bufs;
  FlavorInfo flav[kNumFlavors];
};
#define HGEMM_FLAV(P, N, E)                                                                  \
  { TileCfg<P, N, E>::STAGES, TileCfg<P, N, E>::SMEM, TileCfg<P, N, E>::THREADS, E }
#define HGEMM_TILE(P, N, E4T, E8T)                                                           \
  {P, N, TileCfg<P, N>::ACC_BUFS,                                                            \
   {HGEMM_FLAV(P, N, E4T), HGEMM_FLAV(P, N, E8T), HGEMM_FLAV(P, N, 4), HGEMM_FLAV(P, N, 4),  \
    HGEMM_FLAV(P, N, E4T), HGEMM_FLAV(P, N, E8T)}}
constexpr TileInfo kTiles[kNumTiles] = {
    HGEMM_TILE(2, 512, 4, 8), HGEMM_TILE(2, 256, 4, 8), HGEMM_TILE(2, 128, 4, 8),
    HGEMM_TILE(1, 256, 4, 8), HGEMM_TILE(1, 128, 4, 8), HGEMM_TILE(1, 64, 4, 4),
};
#undef HGEMM_TILE
#undef HGEMM_FLAV

using KernelFn = void (*)(CUtensorMap, CUtensorMap, CUtensorMap, KParams, PeerMaps);

template <int P, int N, int E4T, int E8T, bool HAS_SPLIT, bool HAS_PEERS>
KernelFn flavor_kernel(int flavor) {
  switch (flavor) {
    case kFlavE8: return hgemm_tc_kernel<P, N, true, E8T, false, false>;
    case kFlavSimt: return hgemm_tc_kernel<P, N, false, 4, false, false>;
    case kFlavSplit:
      if constexpr (HAS_SPLIT) return hgemm_tc_kernel<P, N, true, 4, true, false>;
      return nullptr;
    case kFlavPeerE4:
      if constexpr (HAS_PEERS) return hgemm_tc_kernel<P, N, true, E4T, false, true>;
      return nullptr;
    case kFlavPeerE8:
      if constexpr (HAS_PEERS) return hgemm_tc_kernel<P, N, true, E8T, false, true>;
      return nullptr;
    default: return hgemm_tc_kernel<P, N, true, E4T, false, false>;
  }
}

KernelFn kernel_for(int tile, int flavor) {
  switch (tile) {
    case kT256x512: return flavor_kernel<2, 512, 4, 8, false, true>(flavor);
    case kT256x256: return flavor_kernel<2, 256, 4, 8, false, true>(flavor);
    case kT256x128: return flavor_kernel<2, 128, 4, 8, false, false>(flavor);
    case kT128x256: return flavor_kernel<1, 256, 4, 8, true, false>(flavor);
    case kT128x128: return flavor_kernel<1, 128, 4, 8, true, false>(flavor);
    default: return flavor_kernel<1, 64, 4, 4, true, false>(flavor);
  }
}

int tile_from_force(int force_bm, int force_bn) {
  for (int t = 0; t < kNumTiles; ++t)
    if (force_bm == CTA_M * kTiles[t].pair && force_bn == kTiles[t].bn) return t;
  return -1;
}

// ---------------------------------------------------------------- per-device state
struct DevState {
  bool init = false;
  int sm_count = 148;
  int cc_major = 0, cc_minor = 0;
  int pair_slots = 74;        // co-resident 2-CTA clusters at our shared-memory size
  bool attr_done[kNumTiles][kNumFlavors] = {};
  void *scratch = nullptr;
  size_t scratch_bytes = 0;
};
std::mutex g_mu;
DevState g_dev[64];

int current_device(int *dev) {
  if (cudaGetDevice(dev) != cudaSuccess || *dev < 0 || *dev >= 64) return HGEMM_ERR_CUDA;
  return HGEMM_OK;
}

// Caller holds g_mu.
int ensure_device(int dev, DevState **out) {
  DevState &d = g_dev[dev];
  if (!d.init) {
    cudaDeviceProp prop;
    if (cudaGetDeviceProperties(&prop, dev) != cudaSuccess) return HGEMM_ERR_CUDA;
    d.sm_count = prop.multiProcessorCount;
    d.cc_major = prop.major;
    d.cc_minor = prop.minor;
    d.pair_slots = d.sm_count / 2;
    d.init = true;
    if (d.cc_major == 10 && d.cc_minor == 0) {
      // Co-resident clusters of two at this shared-memory size (GPC pairing may leave SMs out).
      const FlavorInfo &fi = kTiles[kT256x256].flav[kFlavE4];
      KernelFn k = kernel_for(kT256x256, kFlavE4);
      if (cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, fi.smem) ==
          cudaSuccess) {
        d.attr_done[kT256x256][kFlavE4] = true;
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(2 * d.pair_slots, 1, 1);
        cfg.blockDim = dim3(fi.threads, 1, 1);
        cfg.dynamicSmemBytes = fi.smem;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeClusterDimension;
        attr[0].val.clusterDim.x = 2;
        attr[0].val.clusterDim.y = 1;
        attr[0].val.clusterDim.z = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        int n = 0;
        if (cudaOccupancyMaxActiveClusters(&n, k, &cfg) == cudaSuccess && n > 0)
          d.pair_slots = std::min(n, d.sm_count / 2);
        cudaGetLastError();
      }
    }
  }
  if (d.cc_major != 10 || d.cc_minor != 0) return HGEMM_ERR_UNSUPPORTED_DEVICE;
  *out = &d;
  return HGEMM_OK;
}

// ---------------------------------------------------------------- planning
int ceil_div(long long a, long long b) { return static_cast<int>((a + b - 1) / b); }

// Which of A, B, C start on a 16-byte boundary (bit 0, 1, 2), as make_plan takes it.
constexpr unsigned kAllAligned = 7u;
unsigned align_mask(const void *A, const void *B, const void *C) {
  return (reinterpret_cast<uintptr_t>(A) % 16 == 0 ? 1u : 0u) |
         (reinterpret_cast<uintptr_t>(B) % 16 == 0 ? 2u : 0u) |
         (reinterpret_cast<uintptr_t>(C) % 16 == 0 ? 4u : 0u);
}

// Tile choice: the tile whose persistent schedule has the least per-CTA work on the
// critical path (waves x columns per CTA), preferring the pair tiles, whose A+B traffic per
// flop is the lowest. group_m keeps the concurrently running tiles' A and B blocks small
// enough to stay in the 126 MB L2.
// Epilogue width of a tile's TMA-store flavour. 8 warps pay only where the epilogue sets the
// pace, tiles of at most 2 k-blocks (K <= 128: 4096x8192x128 0.78 -> 0.91 of cuBLAS,
// 16384x8192x128 0.89 -> 1.00 on B200); from K = 256 the 32 KB of pipeline stages they cost
// weigh more (4096x8192x256 on 256x256: 0.85 with 4 warps, 0.80 with 8).
// The one-accumulator 256x512 tile with beta == 0 takes 8 warps that each drain a quarter of
// every N half (wide_drain in the kernel), which shortens the hand-off between its tiles
// (B200, paired with cuBLAS, three runs each: 8192x8192x4096 0.961 -> 0.970,
// 16384x8192x4096 0.972 -> 0.979, 8192^3 0.982 -> 0.984).
int choose_epi_warps(int tile, int kbn, float beta) {
  if (tile == kT128x64) return 4;
  if (tile == kT256x512) return beta == 0.0f ? 8 : 4;
  return kbn <= 2 ? 8 : 4;
}

// aligned: bit 0 / 1 / 2 set when A / B / C start on a 16-byte boundary (kAllAligned: all).
int make_plan(int M, int N, int K, float beta, unsigned aligned, int force_bm, int force_bn,
              int group_m, int sm_count, int pair_slots, hgemm_plan_t *pl,
              bool persistent_only = false, int ksplit_req = 0) {
  std::memset(pl, 0, sizeof(*pl));
  if (M < 0 || N < 0 || K < 0) return HGEMM_ERR_INVALID_ARG;
  if ((force_bm != 0 || force_bn != 0) && tile_from_force(force_bm, force_bn) < 0)
    return HGEMM_ERR_INVALID_ARG;
  if (ksplit_req < 0 || ksplit_req > kMaxSplit ||
      (ksplit_req > 1 && (force_bm != CTA_M || force_bn == 0)))
    return HGEMM_ERR_INVALID_ARG;
  if (sm_count <= 0) sm_count = 148;
  if (pair_slots <= 0) pair_slots = sm_count / 2;
  if (M == 0 || N == 0) {
    pl->path = 0;
    return HGEMM_OK;
  }
  if (K == 0) {
    pl->path = 2;
    pl->tile_m = 64;
    pl->tile_n = 64;
    pl->pair = 1;
    pl->tiles_m = ceil_div(M, 64);
    pl->tiles_n = ceil_div(N, 64);
    pl->grid_ctas = pl->tiles_m * pl->tiles_n;
    return HGEMM_OK;
  }
  pl->path = 1;
  pl->lda = (K + 7) & ~7;
  pl->ldb = (N + 7) & ~7;
  // An operand whose base is not 16-byte aligned cannot be a TMA source either: it takes the
  // same restride copy as a ragged one (the copy's loads handle any 2-byte offset). The
  // reference sends such calls to its scalar fallback, which on B200 ran at 12-17 TFLOPS
  // (1024^3, 4096^3) where cuBLAS on the same misaligned buffers ran at 68-167.
  const bool a_al = (aligned & 1u) != 0, b_al = (aligned & 2u) != 0, c_al = (aligned & 4u) != 0;
  pl->pad_a = pl->lda != K || !a_al;
  pl->pad_b = pl->ldb != N || !b_al;
  // C with N % 8 != 0 has rows that TMA cannot address. With beta != 0 the GEMM runs on a
  // copy of C with a 16-byte row stride (restrided in, compacted back), two HBM-bound
  // passes instead of an epilogue of 2-byte loads and stores (B200: 4095^3 beta = 0.5
  // 374 -> 207 us, 8192x8191x8192 1634 -> 1032 us). With beta == 0 the compaction costs
  // more than the 2-byte stores save (4095^3: 162 us direct, 185 us padded), so those
  // shapes keep the SIMT-store epilogue. A C that does not start on a 16-byte boundary is
  // always written (and, with beta != 0, read) in place by the SIMT-store epilogue, whose
  // 2-byte accesses need no alignment; the compaction's 16-byte stores would.
  pl->pad_c = (N % 8 != 0) && beta != 0.0f && c_al;
  pl->ldc = pl->pad_c ? pl->ldb : N;
  pl->scratch_bytes = ((pl->pad_a ? static_cast<size_t>(M) * pl->lda : 0) +
                       (pl->pad_b ? static_cast<size_t>(K) * pl->ldb : 0) +
                       (pl->pad_c ? static_cast<size_t>(M) * pl->ldc : 0)) *
                      sizeof(__half);
  pl->tma_store = (c_al && (N % 8 == 0 || pl->pad_c)) ? 1 : 0;

  int tile = tile_from_force(force_bm, force_bn);
  if (tile < 0) {
    // Makespan model (cycles per CTA) for the dynamic cluster-launch-control schedule,
    // calibrated on B200:
    //   k-block time = max(UMMA time, issuer overhead). Every CTA owns 128 rows, so its UMMAs
    //     take BN/2 cycles per k16 (4 per 64-k block); one thread also waits for the stage,
    //     fences and commits, ~320 cycles per k-block whatever N is. An N=64 UMMA cannot be
    //     issued faster than ~48 cycles (it executes in 32), so narrow tiles are
    //     overhead-bound.
    //   tile time = k-blocks x k-block time + hand-off / epilogue cost (double-buffered
    //     accumulators hide most of it; the single 512-column accumulator does not).
    //   makespan = one tile when the tiles fit the co-resident slots, else
    //     tiles / slots + 1/2 tile of tail.
    // Per-flop factors: the 256x512 pair tile moves 25% fewer operand bytes per flop, which
    // keeps the clock higher under the 1 kW cap; one-CTA tiles read twice the B bytes.
    struct Cand {
      int tile;
      double factor, tile_cost;
    };
    const Cand cands[] = {{kT256x512, 0.95, 4000.0}, {kT256x256, 1.00, 1500.0},
                          {kT256x128, 1.00, 1500.0}, {kT128x256, 1.05, 1500.0},
                          {kT128x128, 1.05, 1500.0}};
    const double kb = std::ceil(static_cast<double>(K) / BK);
    // A pair tile also hands every tile index and stage across its two CTAs. With at most
    // four k-blocks per tile (K <= 256) that costs more than the pair saves (B200, one-CTA
    // 128x256 against the 256x256 pair: K = 128 4096x8192 0.77 -> 0.83 of cuBLAS,
    // 16384x8192 0.88 -> 0.98; K = 256 8192x8192 0.93 -> 0.96); from K = 512 the pair is
    // faster.
    // The same holds for a single wave of tiles with at most 8 k-blocks, where the pair's
    // start-up hand-offs are not amortised (2048x2048x512: 0.70 -> 0.85 on 128x256).
    double best = -1.0;
    for (const Cand &c : cands) {
      const TileInfo &ti = kTiles[c.tile];
      const double tiles =
          static_cast<double>(ceil_div(M, CTA_M * ti.pair)) * ceil_div(N, ti.bn);
      const double slots = ti.pair == 2 ? pair_slots : sm_count;
      const bool pair_slow = kb <= 4 || (kb <= 8 && tiles <= slots);
      const double pair_extra = pair_slow ? 3000.0 : 0.0;
      const double kb_time = std::max(4.0 * ti.bn / 2.0, 320.0);
      const double tile_time = kb * kb_time + c.tile_cost + (ti.pair == 2 ? pair_extra : 0.0);
      const double makespan = tiles <= slots ? 1.0 : tiles / slots + 0.5;
      const double cost = makespan * tile_time * c.factor;
      if (best < 0 || cost < best) {
        best = cost;
        tile = c.tile;
      }
    }
    // A single wave of pair tiles with K >= 1024 runs cold and TMA-latency bound; when the
    // 128x64 one-CTA tiles also fit in one wave they keep twice the SMs and more stages
    // busy (B200: 1024^3 0.62 -> 0.66 of cuBLAS, 384x2048x2048 0.55 -> 0.60).
    const double pair_tiles = static_cast<double>(ceil_div(M, 2 * CTA_M)) * ceil_div(N, kTiles[tile].bn);
    const double t64 = static_cast<double>(ceil_div(M, CTA_M)) * ceil_div(N, 64);
    if (kTiles[tile].pair == 2 && pair_tiles <= pair_slots && kb >= 16 && t64 <= sm_count)
      tile = kT128x64;
  }
  const TileInfo &ti = kTiles[tile];
  pl->pair = ti.pair;
  pl->tile_m = CTA_M * ti.pair;
  pl->tile_n = ti.bn;
  {
    const int kbn0 = ceil_div(K, BK);
    const int flav = !pl->tma_store ? kFlavSimt
                     : (choose_epi_warps(tile, kbn0, beta) == 8 ? kFlavE8 : kFlavE4);
    pl->stages = ti.flav[flav].stages;
    pl->epi_warps = ti.flav[flav].epi_warps;
  }
  pl->tiles_m = ceil_div(M, pl->tile_m);
  pl->tiles_n = ceil_div(N, pl->tile_n);
  const long long total = static_cast<long long>(pl->tiles_m) * pl->tiles_n;
  const int slots = ti.pair == 2 ? pair_slots : sm_count;
  const int units = static_cast<int>(std::min<long long>(total, slots));
  // Schedule. Cluster launch control (one cluster per tile; the running ones take over the
  // rest) balances long tiles across SMs that do not run at one clock, but one take-over
  // round trip costs ~3-4.5 K cycles, so tiles shorter than that (small K), and grids whose
  // tiles all fit at once, use a static persistent schedule instead.
  const double tile_cycles =
      std::ceil(static_cast<double>(K) / BK) * std::max(2.0 * ti.bn, 320.0);
  // persistent_only: the GEMM must stay on `sm_count` SMs (the others run concurrent work),
  // which only the static schedule guarantees.
  pl->sched_static =
      (persistent_only || total <= slots || tile_cycles < kStaticTileCycles) ? 1 : 0;
  pl->grid_ctas = static_cast<int>((pl->sched_static ? units : total) * ti.pair);
  pl->ksplit = 1;

  // Split-K. When the tiles occupy only a few SMs, each CTA walks all of K with only its
  // stages in flight (TMA-latency bound); a cluster of ksplit one-CTA tiles then shares each
  // tile's k-blocks and reduces over distributed shared memory. The reduction and its two
  // cluster-wide waits cost ~9 K cycles (B200, 1024^3 split 2: 19.8 us against 17.5 us
  // unsplit), so it is chosen only for grids that fill at most a quarter of the SMs. Needs the
  // TMA-store epilogue; at least 4 k-blocks per split.
  const int kbn = ceil_div(K, BK);
  int ks = 1, ks_tile = -1;
  if (ksplit_req > 1) {
    ks = std::min(ksplit_req, kbn);
    ks_tile = tile;
  } else if (ksplit_req == 0 && force_bm == 0 && !persistent_only && pl->tma_store) {
    const long long ctas_used = static_cast<long long>(units) * ti.pair;
    if (ctas_used * 4 <= static_cast<long long>(sm_count)) {
      long long best_ctas = ctas_used;
      for (int t : {kT128x256, kT128x128, kT128x64}) {
        const long long tt = static_cast<long long>(ceil_div(M, CTA_M)) * ceil_div(N, kTiles[t].bn);
        const int k = static_cast<int>(std::min<long long>(
            {static_cast<long long>(kMaxSplit), sm_count / std::max(tt, 1LL), kbn / 4}));
        if (k >= 2 && tt * k > best_ctas) {
          best_ctas = tt * k;
          ks = k;
          ks_tile = t;
        }
      }
    }
  }
  if (ks > 1 && pl->tma_store) {
    const TileInfo &st = kTiles[ks_tile];
    pl->pair = 1;
    pl->tile_m = CTA_M;
    pl->tile_n = st.bn;
    pl->stages = st.flav[kFlavSplit].stages;
    pl->epi_warps = st.flav[kFlavSplit].epi_warps;
    pl->tiles_m = ceil_div(M, CTA_M);
    pl->tiles_n = ceil_div(N, st.bn);
    pl->ksplit = ks;
    pl->sched_static = 1;
    pl->grid_ctas = pl->tiles_m * pl->tiles_n * ks;
    pl->group_m = 1;
    return HGEMM_OK;
  }
  if (group_m == 0) {
    // Working set of one wave ~ g tile-rows of A plus (units/g) tile-columns of B; choose g
    // near sqrt(units * tile_n / tile_m) (equal A and B footprints), at least 1.
    const double g = std::sqrt(static_cast<double>(units) * pl->tile_n / pl->tile_m);
    group_m = std::max(1, static_cast<int>(g + 0.5));
  }
  pl->group_m = group_m > 0 ? std::min(group_m, pl->tiles_m) : -std::min(-group_m, pl->tiles_n);
  return HGEMM_OK;
}

// ---------------------------------------------------------------- scratch
// Caller holds g_mu. Grow-only per-device buffer for restrided operands.
void *scratch_get(DevState &d, size_t bytes) {
  if (bytes <= d.scratch_bytes) return d.scratch;
  if (d.scratch) {
    cudaFree(d.scratch);
    d.scratch = nullptr;
    d.scratch_bytes = 0;
  }
  void *p = nullptr;
  if (cudaMalloc(&p, bytes) != cudaSuccess) {
    cudaGetLastError();
    return nullptr;
  }
  d.scratch = p;
  d.scratch_bytes = bytes;
  return p;
}

// One launch for every operand of a GEMM that needs a 16-byte row stride.
int launch_restrides(const RestrideJobs &jobs, int sm_count, cudaStream_t stream) {
  if (jobs.n == 0) return HGEMM_OK;
  const long long groups = jobs.total;
  const int blocks = static_cast<int>(std::min<long long>((groups + 255) / 256, sm_count * 8LL));
  restride_kernel<<<std::max(blocks, 1), 256, 0, stream>>>(jobs);
  return cudaGetLastError() == cudaSuccess ? HGEMM_OK : HGEMM_ERR_LAUNCH;
}

void add_restride(RestrideJobs &jobs, const __half *src, __half *dst, int rows, int cols, int ld) {
  const int j = jobs.n++;
  jobs.src[j] = src;
  jobs.dst[j] = dst;
  jobs.rows[j] = rows;
  jobs.cols[j] = cols;
  jobs.ld[j] = ld;
  jobs.first[j + 1] = jobs.first[j] + static_cast<long long>(rows) * (ld / 8);
  jobs.total = jobs.first[j + 1];
}

int launch_simt(const __half *A, const __half *B, __half *C, int M, int N, int K, float alpha,
                float beta, cudaStream_t stream) {
  dim3 grid(ceil_div(N, 64), ceil_div(M, 64));
  hgemm_simt_kernel<<<grid, 256, 0, stream>>>(A, B, C, M, N, K, alpha, beta);
  return cudaGetLastError() == cudaSuccess ? HGEMM_OK : HGEMM_ERR_LAUNCH;
}

// Step-entry gate of a peer-store launch (PeerMaps): per destination, where this rank posts
// its entry epoch and where that destination posts its own.
struct PeerGate {
  unsigned long long *const *post;
  const unsigned long long *const *wait;
  unsigned long long epoch;
};

// Launch the tcgen05 kernel for an already-made plan on operands with 16-byte strides.
int launch_tc(const hgemm_plan_t &pl, int tile, const __half *A, int lda, const __half *B,
              int ldb, __half *C, int M, int N, int K, float alpha, float beta,
              cudaStream_t stream, DevState &d, __half *const *peer_C = nullptr,
              int npeers = 0, const PeerGate *gate = nullptr) {
  const TileInfo &ti = kTiles[tile];
  const bool tma_epi = pl.tma_store != 0;
  CUtensorMap ta, tb, tc;
  const int umma_n = ti.bn < 256 ? ti.bn : 256;
  const int sub_boxes = umma_n / ti.pair / 64, n_sub = ti.bn / umma_n;
  // One 4-D load per stage for B when every tile is whole in N (see encode_b4).
  const bool b4 = (N % ti.bn == 0) && sub_boxes * n_sub > 1 &&
                  encode_b4(&tb, B, K, N, ldb, umma_n, sub_boxes, n_sub);
  if (!encode_2d(&ta, A, M, K, lda, CTA_M, BK) || (!b4 && !encode_2d(&tb, B, K, N, ldb, BK, 64)))
    return HGEMM_ERR_TENSOR_MAP;
  if (tma_epi) {
    if (!encode_2d(&tc, C, M, N, pl.ldc, EPI_ROWS, EPI_COLS)) return HGEMM_ERR_TENSOR_MAP;
  } else {
    tc = ta;
  }
  PeerMaps peers;
  std::memset(&peers, 0, sizeof(peers));
  if (npeers > 0) {
    if (!tma_epi || npeers > kMaxPeers || !peer_C) return HGEMM_ERR_NOT_FUSABLE;
    for (int i = 0; i < npeers; ++i) {
      if (!peer_C[i] || reinterpret_cast<uintptr_t>(peer_C[i]) % 16 != 0)
        return HGEMM_ERR_NOT_FUSABLE;
      peers.ptr[i] = peer_C[i];
      if (gate && gate->epoch != 0) {
        if (!gate->post || !gate->wait || !gate->post[i] || !gate->wait[i])
          return HGEMM_ERR_INVALID_ARG;
        peers.post[i] = gate->post[i];
        peers.wait[i] = gate->wait[i];
      }
    }
    peers.epoch = gate ? gate->epoch : 0ull;
    peers.n = npeers;
  }
  const int flav = !tma_epi ? kFlavSimt
                   : pl.ksplit > 1 ? kFlavSplit
                   : npeers > 0 ? (pl.epi_warps >= 8 ? kFlavPeerE8 : kFlavPeerE4)
                   : (pl.epi_warps >= 8 ? kFlavE8 : kFlavE4);
  const FlavorInfo &fi = ti.flav[flav];
  KernelFn k = kernel_for(tile, flav);
  if (!k) return npeers > 0 ? HGEMM_ERR_NOT_FUSABLE : HGEMM_ERR_INVALID_ARG;
  if (!d.attr_done[tile][flav]) {
    if (cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, fi.smem) !=
        cudaSuccess) {
      cudaGetLastError();
      return HGEMM_ERR_CUDA;
    }
    d.attr_done[tile][flav] = true;
  }
  KParams kp;
  kp.M = M;
  kp.N = N;
  kp.K = K;
  kp.tiles_m = pl.tiles_m;
  kp.tiles_n = pl.tiles_n;
  kp.num_tiles = pl.tiles_m * pl.tiles_n;
  kp.num_kb = ceil_div(K, BK);
  kp.group_m = pl.group_m;
  kp.alpha = alpha;
  kp.beta = beta;
  kp.C = C;
  kp.ldc = pl.ldc;
  kp.timeout_ns = g_timeout_ns.load();
  kp.sched_static = pl.sched_static;
  kp.ksplit = pl.ksplit > 1 ? pl.ksplit : 1;
  kp.b4 = b4 ? 1 : 0;
  // Peer copies are never read on the receiving GPU during the step either.
  kp.c_evict_first = (K >= kCEvictFirstMinK || npeers > 0) ? 1 : 0;

  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(pl.grid_ctas, 1, 1);
  cfg.blockDim = dim3(fi.threads, 1, 1);
  cfg.dynamicSmemBytes = fi.smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = ti.pair == 2 ? 2 : kp.ksplit;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = (ti.pair == 2 || kp.ksplit > 1) ? 1 : 0;
  if (cudaLaunchKernelEx(&cfg, k, ta, tb, tc, kp, peers) != cudaSuccess) {
    cudaGetLastError();
    return HGEMM_ERR_LAUNCH;
  }
  return HGEMM_OK;
}

int launch_compact(const __half *src, __half *dst, int rows, int cols, int ld, int sm_count,
                   cudaStream_t stream) {
  const long long groups = (static_cast<long long>(rows) * cols + 7) / 8;
  const int blocks = static_cast<int>(std::min<long long>((groups + 255) / 256, sm_count * 8LL));
  compact_kernel<<<std::max(blocks, 1), 256, 0, stream>>>(src, dst, rows, cols, ld);
  return cudaGetLastError() == cudaSuccess ? HGEMM_OK : HGEMM_ERR_LAUNCH;
}

// The tcgen05 path of a plan: restride A (K % 8 != 0) and B (N % 8 != 0) into scratch `w`,
// run the GEMM (into a 16-byte-strided copy of C when N % 8 != 0, read in first when
// beta != 0) and compact that copy back into C. `w` holds pl.scratch_bytes (A, then B, then
// C); every element the GEMM reads from it is written earlier on the same stream.
int launch_padded(const hgemm_plan_t &pl, const __half *A, const __half *B, __half *C, int M,
                  int N, int K, float alpha, float beta, cudaStream_t stream, DevState &d,
                  __half *w, __half *const *peer_C, int npeers,
                  const PeerGate *gate = nullptr) {
  int st = HGEMM_OK;
  const __half *Ause = A, *Buse = B;
  __half *Cuse = C;
  const size_t na = pl.pad_a ? static_cast<size_t>(M) * pl.lda : 0;
  const size_t nb = pl.pad_b ? static_cast<size_t>(K) * pl.ldb : 0;
  RestrideJobs jobs;
  std::memset(&jobs, 0, sizeof(jobs));
  if (pl.pad_a) {
    add_restride(jobs, A, w, M, K, pl.lda);
    Ause = w;
  }
  if (pl.pad_b) {
    add_restride(jobs, B, w + na, K, N, pl.ldb);
    Buse = w + na;
  }
  if (pl.pad_c) {
    Cuse = w + na + nb;
    if (beta != 0.0f) add_restride(jobs, C, Cuse, M, N, pl.ldc);
  }
  st = launch_restrides(jobs, d.sm_count, stream);
  if (st != HGEMM_OK) return st;
  int tile = -1;
  for (int t = 0; t < kNumTiles; ++t)
    if (kTiles[t].pair == pl.pair && kTiles[t].bn == pl.tile_n) tile = t;
  st = launch_tc(pl, tile, Ause, pl.lda, Buse, pl.ldb, Cuse, M, N, K, alpha, beta, stream, d,
                 peer_C, npeers, gate);
  if (st != HGEMM_OK || !pl.pad_c) return st;
  return launch_compact(Cuse, C, M, N, pl.ldc, d.sm_count, stream);
}

int launch_impl(const __half *A, const __half *B, __half *C, int M, int N, int K, float alpha,
                float beta, cudaStream_t stream, int force_bm, int force_bn, int group_m,
                int sm_limit = 0, __half *const *peer_C = nullptr, int npeers = 0,
                int ksplit_req = 0, const PeerGate *gate = nullptr) {
  if (M < 0 || N < 0 || K < 0) return HGEMM_ERR_INVALID_ARG;
  if (M == 0 || N == 0) return HGEMM_OK;
  if (!A || !B || !C) return HGEMM_ERR_INVALID_ARG;
  int dev;
  if (current_device(&dev) != HGEMM_OK) return HGEMM_ERR_CUDA;
  std::lock_guard<std::mutex> lock(g_mu);
  DevState *d = nullptr;
  int st = ensure_device(dev, &d);
  if (st != HGEMM_OK) return st;
  const unsigned aligned = align_mask(A, B, C);
  int sms = d->sm_count, pslots = d->pair_slots;
  if (sm_limit > 0 && sm_limit < sms) {
    sms = sm_limit;
    pslots = std::max(1, std::min(pslots, sm_limit / 2));
  }
  hgemm_plan_t pl;
  // Peer stores are issued by the tile's own epilogue, which split-K replaces.
  st = make_plan(M, N, K, beta, aligned, force_bm, force_bn, group_m, sms, pslots, &pl,
                 sm_limit > 0, npeers > 0 ? 1 : ksplit_req);
  if (st != HGEMM_OK) return st;
  if (pl.path == 0) return HGEMM_OK;
  if (npeers > 0 && (pl.path != 1 || !pl.tma_store || pl.pad_c)) return HGEMM_ERR_NOT_FUSABLE;
  if (npeers > 0 && force_bm == 0 &&
      !(pl.pair == 2 && (pl.tile_n == 256 || (pl.tile_n == 512 && K >= kPeerWideTileMinK)))) {
    // Every tile's epilogue also stores to the peers (peer flavours exist for 256x512 and
    // 256x256 only). With the single 512-column accumulator that longer epilogue sits
    // between tiles; the double-buffered 256x256 tile hides it behind the next tile's main
    // loop (measured on 2 B200s: faster at K = 8192, slower at K = 16384).
    st = make_plan(M, N, K, beta, aligned, 256, 256, group_m, sms, pslots, &pl, sm_limit > 0,
                   1);
    if (st != HGEMM_OK) return st;
  }
  if (pl.path == 2) return launch_simt(A, B, C, M, N, K, alpha, beta, stream);

  __half *w = nullptr;
  if (pl.pad_a || pl.pad_b || pl.pad_c) {
    w = static_cast<__half *>(scratch_get(*d, pl.scratch_bytes));
    if (!w) return HGEMM_ERR_ALLOC;
  }
  return launch_padded(pl, A, B, C, M, N, K, alpha, beta, stream, *d, w, peer_C, npeers, gate);
}

// ---------------------------------------------------------------- autotune cache
struct TuneCfg {
  int bm, bn, group_m;
};
std::map<std::tuple<int, int, int, int>, TuneCfg> g_tune;

// Forgets the cached device addresses of the no-allocation scratch array (defined with
// hgemm_launch_noalloc below), so that they are looked up again after a device reset.
void noalloc_forget_addresses();

}  // namespace
}  // namespace hgemm

// ============================================================================ C ABI
using namespace hgemm;

extern "C" {

int hgemm_launch_ex(const hgemm_half_t *A, const hgemm_half_t *B, hgemm_half_t *C, int M, int N,
                    int K, float alpha, float beta, hgemm_stream_t stream, int force_bm,
                    int force_bn, int group_m) {
  return set_status(launch_impl(A, B, C, M, N, K, alpha, beta,
                                reinterpret_cast<cudaStream_t>(stream), force_bm, force_bn,
                                group_m));
}

// GEMM without split-K for the multi-GPU layer (not part of the public header): its row
// chunks must sum every element in the order the unsplit full-size GEMM does.
__attribute__((visibility("hidden"))) int hgemm_internal_launch_unsplit(
    const hgemm_half_t *A, const hgemm_half_t *B, hgemm_half_t *C, int M, int N, int K,
    float alpha, float beta, hgemm_stream_t stream, int sm_limit) {
  return set_status(launch_impl(A, B, C, M, N, K, alpha, beta,
                                reinterpret_cast<cudaStream_t>(stream), 0, 0, 0,
                                sm_limit > 0 ? sm_limit : 0, nullptr, 0, 1));
}

// The plan hgemm_launch would run on the current device for these operands (not part of the
// public header; used by hgemm_launch_host to keep its row blocks on the one-launch
// arithmetic).
__attribute__((visibility("hidden"))) int hgemm_internal_plan_current(
    const hgemm_half_t *A, const hgemm_half_t *B, const hgemm_half_t *C, int M, int N, int K,
    float beta, hgemm_plan_t *out) {
  if (!out) return HGEMM_ERR_INVALID_ARG;
  int dev;
  if (current_device(&dev) != HGEMM_OK) return HGEMM_ERR_CUDA;
  std::lock_guard<std::mutex> lock(g_mu);
  DevState *d = nullptr;
  const int st = ensure_device(dev, &d);
  if (st != HGEMM_OK) return st;
  return make_plan(M, N, K, beta, align_mask(A, B, C), 0, 0, 0, d->sm_count, d->pair_slots,
                   out);
}

// Used by the multi-GPU layer only (not part of the public header). entry = 0: step-exit
// barrier; entry = 1: step-entry barrier (every rank has entered the step).
__attribute__((visibility("hidden"))) int hgemm_internal_peer_barrier(
    unsigned long long *const *flags, int rank, int nranks, unsigned long long epoch,
    int entry, hgemm_stream_t stream) {
  if (!flags || nranks < 1 || nranks > kMaxRanksBarrier || rank < 0 || rank >= nranks)
    return HGEMM_ERR_INVALID_ARG;
  BarrierArgs a;
  std::memset(&a, 0, sizeof(a));
  for (int r = 0; r < nranks; ++r) a.flags[r] = flags[r];
  a.rank = rank;
  a.nranks = nranks;
  a.slot_base = entry ? kMaxRanksBarrier : 0;
  peer_barrier_kernel<<<1, 32, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      a, epoch, g_timeout_ns.load());
  return cudaGetLastError() == cudaSuccess ? HGEMM_OK : HGEMM_ERR_LAUNCH;
}

// Peer-store GEMM with the step-entry gate (PeerMaps) for the multi-GPU layer (not part of
// the public header): post[d] / wait[d] are destination d's entry flag for this rank and this
// rank's entry flag for destination d; epoch > 0.
__attribute__((visibility("hidden"))) int hgemm_internal_launch_peers_gated(
    const hgemm_half_t *A, const hgemm_half_t *B, hgemm_half_t *C, int M, int N, int K,
    float alpha, float beta, hgemm_stream_t stream, hgemm_half_t *const *peer_C, int npeers,
    unsigned long long *const *post, const unsigned long long *const *wait,
    unsigned long long epoch) {
  if (npeers < 1 || npeers > kMaxPeers || !peer_C || !post || !wait || epoch == 0)
    return set_status(HGEMM_ERR_INVALID_ARG);
  const PeerGate gate{post, wait, epoch};
  return set_status(launch_impl(A, B, C, M, N, K, alpha, beta,
                                reinterpret_cast<cudaStream_t>(stream), 0, 0, 0, 0, peer_C,
                                npeers, 0, &gate));
}

int hgemm_launch_peers(const hgemm_half_t *A, const hgemm_half_t *B, hgemm_half_t *C, int M,
                       int N, int K, float alpha, float beta, hgemm_stream_t stream,
                       hgemm_half_t *const *peer_C, int npeers, int sm_limit) {
  if (npeers < 0 || npeers > kMaxPeers || (npeers > 0 && !peer_C))
    return set_status(HGEMM_ERR_INVALID_ARG);
  return set_status(launch_impl(A, B, C, M, N, K, alpha, beta,
                                reinterpret_cast<cudaStream_t>(stream), 0, 0, 0,
                                sm_limit > 0 ? sm_limit : 0, peer_C, npeers));
}

int hgemm_launch_splitk(const hgemm_half_t *A, const hgemm_half_t *B, hgemm_half_t *C, int M,
                        int N, int K, float alpha, float beta, hgemm_stream_t stream, int bn,
                        int ksplit) {
  if (ksplit < 1 || ksplit > kMaxSplit || (bn != 64 && bn != 128 && bn != 256))
    return set_status(HGEMM_ERR_INVALID_ARG);
  return set_status(launch_impl(A, B, C, M, N, K, alpha, beta,
                                reinterpret_cast<cudaStream_t>(stream), CTA_M, bn, 0, 0, nullptr,
                                0, ksplit));
}

int hgemm_launch_sm_limit(const hgemm_half_t *A, const hgemm_half_t *B, hgemm_half_t *C, int M,
                          int N, int K, float alpha, float beta, hgemm_stream_t stream,
                          int sm_limit) {
  if (sm_limit <= 0) return set_status(HGEMM_ERR_INVALID_ARG);
  return set_status(launch_impl(A, B, C, M, N, K, alpha, beta,
                                reinterpret_cast<cudaStream_t>(stream), 0, 0, 0, sm_limit));
}

int hgemm_launch(const hgemm_half_t *A, const hgemm_half_t *B, hgemm_half_t *C, int M, int N,
                 int K, float alpha, float beta, hgemm_stream_t stream) {
  return hgemm_launch_ex(A, B, C, M, N, K, alpha, beta, stream, 0, 0, 0);
}

void solve(const hgemm_half_t *A, const hgemm_half_t *B, hgemm_half_t *C, int M, int N, int K,
           float alpha, float beta) {
  int st = launch_impl(A, B, C, M, N, K, alpha, beta, 0, 0, 0, 0);
  const cudaError_t e = cudaDeviceSynchronize();
  if (st == HGEMM_OK && e != cudaSuccess) st = HGEMM_ERR_CUDA;
  if (st == HGEMM_OK) {
    unsigned v = 0;
    if (cudaMemcpyFromSymbol(&v, g_dev_status, sizeof(v)) == cudaSuccess && v != 0)
      st = HGEMM_ERR_DEVICE_TIMEOUT;
  }
  set_status(st);
}

int hgemm_launch_tuned(const hgemm_half_t *A, const hgemm_half_t *B, hgemm_half_t *C, int M,
                       int N, int K, float alpha, float beta, hgemm_stream_t stream) {
  int dev;
  if (current_device(&dev) != HGEMM_OK) return set_status(HGEMM_ERR_CUDA);
  const auto key = std::make_tuple(dev, M, N, K);
  TuneCfg best{0, 0, 0};
  bool have = false;
  {
    std::lock_guard<std::mutex> lock(g_mu);
    auto it = g_tune.find(key);
    if (it != g_tune.end()) {
      best = it->second;
      have = true;
    }
  }
  const bool aligned = (reinterpret_cast<uintptr_t>(A) % 16 == 0) &&
                       (reinterpret_cast<uintptr_t>(B) % 16 == 0) &&
                       (reinterpret_cast<uintptr_t>(C) % 16 == 0);
  if (!have && M > 0 && N > 0 && K > 0 && aligned) {
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    __half *scratchC = nullptr;
    if (cudaMalloc(&scratchC, static_cast<size_t>(M) * N * sizeof(__half)) != cudaSuccess) {
      cudaGetLastError();
      return set_status(HGEMM_ERR_ALLOC);
    }
    cudaEvent_t e0, e1;
    cudaEventCreate(&e0);
    cudaEventCreate(&e1);
    int bms[kNumTiles], bns[kNumTiles];
    for (int t = 0; t < kNumTiles; ++t) {
      bms[t] = CTA_M * kTiles[t].pair;
      bns[t] = kTiles[t].bn;
    }
    const int gms[5] = {0, 4, 8, 16, 32};
    float best_ms = 1e30f;
    for (int t = 0; t < kNumTiles; ++t) {
      for (int g : gms) {
        bool ok = true;
        for (int i = 0; i < 3 && ok; ++i)
          ok = launch_impl(A, B, scratchC, M, N, K, alpha, 0.0f, s, bms[t], bns[t], g) == HGEMM_OK;
        if (!ok || cudaStreamSynchronize(s) != cudaSuccess) continue;
        cudaEventRecord(e0, s);
        for (int i = 0; i < 5; ++i) launch_impl(A, B, scratchC, M, N, K, alpha, 0.0f, s, bms[t], bns[t], g);
        cudaEventRecord(e1, s);
        if (cudaEventSynchronize(e1) != cudaSuccess) continue;
        float ms = 0;
        cudaEventElapsedTime(&ms, e0, e1);
        if (ms > 0 && ms < best_ms) {
          best_ms = ms;
          best = TuneCfg{bms[t], bns[t], g};
        }
      }
    }
    cudaEventDestroy(e0);
    cudaEventDestroy(e1);
    cudaFree(scratchC);
    cudaGetLastError();
    std::lock_guard<std::mutex> lock(g_mu);
    g_tune[key] = best;
  }
  return set_status(launch_impl(A, B, C, M, N, K, alpha, beta,
                                reinterpret_cast<cudaStream_t>(stream), best.bm, best.bn,
                                best.group_m));
}

int hgemm_last_status(void) { return t_last_status; }

const char *hgemm_status_string(int s) {
  switch (s) {
    case HGEMM_OK: return "ok";
    case HGEMM_ERR_INVALID_ARG: return "invalid argument";
    case HGEMM_ERR_CUDA: return "CUDA runtime call failed";
    case HGEMM_ERR_TENSOR_MAP: return "tensor map encode failed";
    case HGEMM_ERR_ALLOC: return "scratch allocation failed";
    case HGEMM_ERR_LAUNCH: return "kernel launch failed";
    case HGEMM_ERR_DEVICE_TIMEOUT: return "bounded device wait ran out";
    case HGEMM_ERR_UNSUPPORTED_DEVICE: return "device is not sm_100 (B200)";
    case HGEMM_ERR_NCCL: return "NCCL unavailable or failed";
    case HGEMM_ERR_TOO_LARGE: return "size beyond this entry point's limit";
    case HGEMM_ERR_NOT_FUSABLE: return "shape or alignment takes a path without TMA stores";
    default: return "unknown status";
  }
}

int hgemm_device_status(int clear, int *where) {
  if (cudaDeviceSynchronize() != cudaSuccess) return set_status(HGEMM_ERR_CUDA);
  unsigned v = 0;
  if (cudaMemcpyFromSymbol(&v, g_dev_status, sizeof(v)) != cudaSuccess)
    return set_status(HGEMM_ERR_CUDA);
  if (where) *where = static_cast<int>(v & 0xffu);
  if (clear && v) {
    const unsigned z = 0;
    if (cudaMemcpyToSymbol(g_dev_status, &z, sizeof(z)) != cudaSuccess)
      return set_status(HGEMM_ERR_CUDA);
  }
  return v ? HGEMM_ERR_DEVICE_TIMEOUT : HGEMM_OK;
}

void hgemm_set_wait_timeout_ns(unsigned long long ns) { g_timeout_ns.store(ns ? ns : 1ull); }

int hgemm_selftest_wait_timeout(unsigned long long timeout_ns) {
  int *d_out = nullptr;
  if (cudaMalloc(&d_out, sizeof(int)) != cudaSuccess) return set_status(HGEMM_ERR_CUDA);
  int h = -1;
  wait_selftest_kernel<<<1, 32>>>(timeout_ns, d_out);
  int st = (cudaGetLastError() == cudaSuccess) ? HGEMM_OK : HGEMM_ERR_LAUNCH;
  if (st == HGEMM_OK && cudaMemcpy(&h, d_out, sizeof(int), cudaMemcpyDeviceToHost) != cudaSuccess)
    st = HGEMM_ERR_CUDA;
  cudaFree(d_out);
  int where = 0;
  hgemm_device_status(1, &where);  // the self-test recorded a timeout: clear it
  if (st != HGEMM_OK) return set_status(st);
  set_status(HGEMM_OK);
  return h;
}

int hgemm_selftest_peer_barrier(unsigned long long timeout_ns) {
  // Rank 0 of a two-rank barrier whose partner never announces: the bounded wait must run
  // out, record kSitePeerBarrier and return. Both flag arrays are local memory.
  unsigned long long *d = nullptr;
  if (cudaMalloc(&d, 4 * kMaxRanksBarrier * sizeof(unsigned long long)) != cudaSuccess)
    return set_status(HGEMM_ERR_CUDA);
  int st = cudaMemset(d, 0, 4 * kMaxRanksBarrier * sizeof(unsigned long long)) == cudaSuccess
               ? HGEMM_OK
               : HGEMM_ERR_CUDA;
  if (st == HGEMM_OK) {
    BarrierArgs a;
    std::memset(&a, 0, sizeof(a));
    a.flags[0] = d;
    a.flags[1] = d + 2 * kMaxRanksBarrier;
    a.rank = 0;
    a.nranks = 2;
    a.slot_base = 0;
    peer_barrier_kernel<<<1, 32>>>(a, 1ull, timeout_ns);
    st = cudaGetLastError() == cudaSuccess ? HGEMM_OK : HGEMM_ERR_LAUNCH;
    unsigned long long announced = 0;
    if (st == HGEMM_OK &&
        cudaMemcpy(&announced, d + 2 * kMaxRanksBarrier, sizeof(announced),
                   cudaMemcpyDeviceToHost) != cudaSuccess)
      st = HGEMM_ERR_CUDA;
    if (st == HGEMM_OK && announced != 1ull) st = HGEMM_ERR_CUDA;  // lane 1 must have announced
  }
  cudaFree(d);
  int where = 0;
  const int dev = hgemm_device_status(1, &where);  // read and clear what the test recorded
  if (st != HGEMM_OK) return set_status(st);
  set_status(HGEMM_OK);
  return (dev == HGEMM_ERR_DEVICE_TIMEOUT && where == static_cast<int>(kSitePeerBarrier))
             ? HGEMM_ERR_DEVICE_TIMEOUT
             : HGEMM_OK;
}

int hgemm_selftest_peer_entry(int satisfied, unsigned long long timeout_ns) {
  // A 256 x 256 x 64 GEMM of zeros through the gated peer-store kernel, on one GPU with local
  // memory only: its one "peer" C is a local buffer pre-filled with 0x5A bytes and its entry
  // flag is either already at the step's epoch (satisfied) or never set.
  constexpr int M = 256, N = 256, K = 64;
  const size_t nA = static_cast<size_t>(M) * K, nB = static_cast<size_t>(K) * N,
               nC = static_cast<size_t>(M) * N;
  const size_t bytes = (nA + nB + 2 * nC) * sizeof(__half) + 2 * sizeof(unsigned long long);
  char *buf = nullptr;
  if (cudaMalloc(&buf, bytes) != cudaSuccess) return set_status(HGEMM_ERR_CUDA);
  __half *A = reinterpret_cast<__half *>(buf), *B = A + nA, *C = B + nB, *P = C + nC;
  unsigned long long *flags = reinterpret_cast<unsigned long long *>(P + nC);
  const unsigned long long epoch = 1, want = satisfied ? epoch : 0;
  int st = (cudaMemset(A, 0, (nA + nB) * sizeof(__half)) == cudaSuccess &&
            cudaMemset(C, 0xFF, nC * sizeof(__half)) == cudaSuccess &&
            cudaMemset(P, 0x5A, nC * sizeof(__half)) == cudaSuccess &&
            cudaMemset(flags, 0, sizeof(unsigned long long)) == cudaSuccess &&
            cudaMemcpy(flags + 1, &want, sizeof(want), cudaMemcpyHostToDevice) == cudaSuccess)
               ? HGEMM_OK
               : HGEMM_ERR_CUDA;
  const unsigned long long saved = g_timeout_ns.load();
  if (st == HGEMM_OK) {
    g_timeout_ns.store(timeout_ns ? timeout_ns : 1ull);
    __half *peer[1] = {P};
    unsigned long long *post[1] = {flags};
    const unsigned long long *wait[1] = {flags + 1};
    const PeerGate gate{post, wait, epoch};
    st = launch_impl(A, B, C, M, N, K, 1.0f, 0.0f, 0, 0, 0, 0, 0, peer, 1, 0, &gate);
    if (cudaDeviceSynchronize() != cudaSuccess && st == HGEMM_OK) st = HGEMM_ERR_CUDA;
    g_timeout_ns.store(saved);
  }
  int where = 0;
  const int dev = hgemm_device_status(1, &where);  // read and clear what the kernel recorded
  std::vector<uint16_t> hc(nC), hp(nC);
  unsigned long long posted = 0;
  if (st == HGEMM_OK &&
      (cudaMemcpy(hc.data(), C, nC * sizeof(__half), cudaMemcpyDeviceToHost) != cudaSuccess ||
       cudaMemcpy(hp.data(), P, nC * sizeof(__half), cudaMemcpyDeviceToHost) != cudaSuccess ||
       cudaMemcpy(&posted, flags, sizeof(posted), cudaMemcpyDeviceToHost) != cudaSuccess))
    st = HGEMM_ERR_CUDA;
  cudaFree(buf);
  if (st != HGEMM_OK) return set_status(st);
  set_status(HGEMM_OK);
  // The local C is computed either way and the kernel announced its own entry.
  bool good = posted == epoch;
  for (size_t i = 0; i < nC && good; ++i) good = hc[i] == 0;
  if (satisfied) {
    for (size_t i = 0; i < nC && good; ++i) good = hp[i] == 0;
    if (!good) return HGEMM_ERR_CUDA;
    return dev;  // HGEMM_OK: no wait ran out
  }
  for (size_t i = 0; i < nC && good; ++i) good = hp[i] == 0x5A5Au;
  if (!good) return HGEMM_ERR_CUDA;
  return (dev == HGEMM_ERR_DEVICE_TIMEOUT && where == static_cast<int>(kSitePeerEntry))
             ? HGEMM_ERR_DEVICE_TIMEOUT
             : HGEMM_OK;
}

void hgemm_release(void) {
  std::lock_guard<std::mutex> lock(g_mu);
  int cur = 0;
  cudaGetDevice(&cur);
  for (int i = 0; i < 64; ++i) {
    if (g_dev[i].scratch) {
      cudaSetDevice(i);
      cudaFree(g_dev[i].scratch);
      g_dev[i].scratch = nullptr;
      g_dev[i].scratch_bytes = 0;
    }
  }
  cudaSetDevice(cur);
  g_tune.clear();
  noalloc_forget_addresses();
}

int hgemm_plan(int M, int N, int K, float beta, int aligned16, int force_bm, int force_bn,
               int group_m, int sm_count, int pair_slots, hgemm_plan_t *out) {
  if (!out) return HGEMM_ERR_INVALID_ARG;
  return make_plan(M, N, K, beta, aligned16 != 0 ? kAllAligned : 0u, force_bm, force_bn, group_m,
                   sm_count,
                   pair_slots, out);
}

}  // extern "C"

// ============================================================================ no-allocation entry
// Some callers cannot allocate device memory when they call the GEMM: a host that owns a
// fixed device-memory pool and forbids anything else to call cudaMalloc, a process whose
// caller-facing path must not take the allocator's lock or implicitly synchronise the
// device (cudaMalloc/cudaFree may do both), or code with a strict memory budget decided
// ahead of time. hgemm_launch_noalloc serves them: it is hgemm_launch, except that the one
// scratch buffer the path can need -- the restrided copy of A when K % 8 != 0, of B when
// N % 8 != 0, and the 16-byte-strided copy of C when N % 8 != 0 and beta != 0 -- lives in the
// fixed-size array below, which the library's module owns on every device that loads it
// (until the process exits), instead of coming from cudaMalloc. The array's device address
// is looked up once per device and cached; hgemm_release() forgets the cached addresses (call
// it after a device reset, which reloads the module).
namespace hgemm {
namespace {

constexpr size_t kNoallocScratchBytes = 64ull << 20;  // 64 MiB

// Device-side storage. Host code never uses this name as an address: the host-side symbol
// is only a stand-in, and a kernel handed it would fault (or quietly touch host memory).
// The real device address comes from cudaGetSymbolAddress, once per device.
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoallocScratchBytes];

std::mutex g_noalloc_mu;
void *g_noalloc_ptr[64] = {};

void noalloc_forget_addresses() {
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  for (void *&p : g_noalloc_ptr) p = nullptr;
}

// Caller holds g_noalloc_mu; `dev` is current.
int noalloc_scratch(int dev, __half **out) {
  if (!g_noalloc_ptr[dev]) {
    void *p = nullptr;
    if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess || !p) {
      cudaGetLastError();
      return HGEMM_ERR_CUDA;
    }
    g_noalloc_ptr[dev] = p;
  }
  *out = static_cast<__half *>(g_noalloc_ptr[dev]);
  return HGEMM_OK;
}

int launch_noalloc_impl(const __half *A, const __half *B, __half *C, int M, int N, int K,
                        float alpha, float beta, cudaStream_t stream) {
  if (M < 0 || N < 0 || K < 0) return HGEMM_ERR_INVALID_ARG;
  if (M == 0 || N == 0) return HGEMM_OK;
  if (!A || !B || !C) return HGEMM_ERR_INVALID_ARG;
  int dev;
  if (current_device(&dev) != HGEMM_OK) return HGEMM_ERR_CUDA;
  std::lock_guard<std::mutex> lock(g_mu);
  DevState *d = nullptr;
  int st = ensure_device(dev, &d);
  if (st != HGEMM_OK) return st;
  const unsigned aligned = align_mask(A, B, C);
  hgemm_plan_t pl;
  st = make_plan(M, N, K, beta, aligned, 0, 0, 0, d->sm_count, d->pair_slots, &pl);
  if (st != HGEMM_OK) return st;
  if (pl.path == 0) return HGEMM_OK;
  // Operands that do not start on a 16-byte boundary would need their copies in the fixed
  // array too; this entry point keeps them on the scalar kernel, which needs no scratch.
  if (pl.path == 2 || aligned != kAllAligned)
    return launch_simt(A, B, C, M, N, K, alpha, beta, stream);
  __half *w = nullptr;
  if (pl.pad_a || pl.pad_b || pl.pad_c) {
    if (pl.scratch_bytes > kNoallocScratchBytes) return HGEMM_ERR_TOO_LARGE;
    {
      std::lock_guard<std::mutex> lk(g_noalloc_mu);
      st = noalloc_scratch(dev, &w);
    }
    if (st != HGEMM_OK) return st;
    // Nothing here has to start at zero: each element the GEMM reads from the array is
    // written by the restride passes of this same call, earlier on the same stream (the C
    // copy is only read when beta != 0, after C was restrided into it).
  }
  return launch_padded(pl, A, B, C, M, N, K, alpha, beta, stream, *d, w, nullptr, 0);
}

}  // namespace
}  // namespace hgemm

extern "C" {

size_t hgemm_noalloc_scratch_bytes(void) { return hgemm::kNoallocScratchBytes; }

int hgemm_launch_noalloc(const hgemm_half_t *A, const hgemm_half_t *B, hgemm_half_t *C, int M,
                         int N, int K, float alpha, float beta, hgemm_stream_t stream) {
  return hgemm::set_status(hgemm::launch_noalloc_impl(
      A, B, C, M, N, K, alpha, beta, reinterpret_cast<cudaStream_t>(stream)));
}

}  // extern "C"
