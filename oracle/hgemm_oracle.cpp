// TEST INFRASTRUCTURE ONLY -- the CPU oracle for the FP16 GEMM path. Only tests/,
// __graft_entry__.smoke() and bench.py's CPU-baseline leg load this library, and only as a
// checker or as the timed CPU baseline; the GEMM product never calls it.
//
// What it restates from the reference (yz-wqf/Hopper_GEMM):
//   * oracle_gemm_f64*: the host fp64 reference GEMM of check_fp64.cu:39-44
//       acc = sum_k (double)A[i][k] * (double)B[k][j]   (k increasing, acc starting at 0)
//       r   = (double)alpha * acc + (double)beta * (double)C_in[i][j]
//     Products of two fp16 values are exact in fp64, and every (i, j) sum is accumulated in
//     the same k order as the reference's triple loop, so the results are bit-identical to
//     that loop; only the loop nest is reordered (blocks of rows and columns, k running
//     over all of K inside each block) for cache locality, and the blocks are spread over
//     std::thread workers.
//   * oracle_mt_*: the harnesses' seeded inputs -- std::mt19937(seed) with
//     std::uniform_real_distribution<float>(lo, hi) (check_all.cu:14, check_fp64.cu:16,
//     check_large.cu:15), each draw rounded to half by round-to-nearest-even
//     (__float2half, check_fp64.cu:28-30); normal(mean, std) for a C prefill.
//   * oracle_hash_fill_half: the counter-hash fill of three_way.cu:22-33 (every step exact
//     in fp32, so the host reproduces the device fill bit for bit).
//   * oracle_gemm_f64_ref_order: the reference's literal i-j-k loop (strided B reads),
//     single-threaded, kept to time the CPU baseline in the reference's own loop order.
#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <random>
#include <thread>
#include <vector>

namespace {

// IEEE binary16 <-> binary32, round-to-nearest-even (written from the format definition).
uint16_t f32_to_f16(float f) {
  uint32_t x;
  std::memcpy(&x, &f, 4);
  const uint32_t sign = (x >> 16) & 0x8000u;
  const uint32_t absx = x & 0x7fffffffu;
  if (absx >= 0x7f800000u) {  // Inf or NaN
    return static_cast<uint16_t>(sign | 0x7c00u | (absx > 0x7f800000u ? 0x200u : 0u));
  }
  if (absx >= 0x477ff000u) return static_cast<uint16_t>(sign | 0x7c00u);  // rounds to Inf
  const int exp = static_cast<int>(absx >> 23) - 127;
  if (exp < -14) {
    // Subnormal half (or zero): value = mant * 2^-24. Shift the 24-bit significand.
    if (exp < -25) return static_cast<uint16_t>(sign);  // below half of the smallest subnormal
    const uint32_t mant = (absx & 0x7fffffu) | 0x800000u;
    const int shift = -exp - 14 + 13;  // 14..24 -> bits dropped
    uint32_t q = mant >> shift;
    const uint32_t rem = mant & ((1u << shift) - 1u);
    const uint32_t half = 1u << (shift - 1);
    if (rem > half || (rem == half && (q & 1u))) ++q;
    return static_cast<uint16_t>(sign | q);
  }
  uint32_t h = ((static_cast<uint32_t>(exp + 15)) << 10) | ((absx >> 13) & 0x3ffu);
  const uint32_t rem = absx & 0x1fffu;
  if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) ++h;  // carry may bump the exponent
  return static_cast<uint16_t>(sign | h);
}

float f16_to_f32(uint16_t h) {
  const uint32_t sign = (static_cast<uint32_t>(h) & 0x8000u) << 16;
  const uint32_t exp = (h >> 10) & 0x1fu;
  const uint32_t mant = h & 0x3ffu;
  uint32_t x;
  if (exp == 0) {
    if (mant == 0) {
      x = sign;
    } else {  // subnormal: mant * 2^-24
      float v = std::ldexp(static_cast<float>(mant), -24);
      std::memcpy(&x, &v, 4);
      x |= sign;
    }
  } else if (exp == 31) {
    x = sign | 0x7f800000u | (mant << 13);
  } else {
    x = sign | ((exp - 15 + 127) << 23) | (mant << 13);
  }
  float f;
  std::memcpy(&f, &x, 4);
  return f;
}

// Every binary16 value as a double (512 KB, stays cache resident while B streams by).
const double *half_lut() {
  static const std::vector<double> lut = [] {
    std::vector<double> t(65536);
    for (uint32_t h = 0; h < 65536; ++h) t[h] = static_cast<double>(f16_to_f32(static_cast<uint16_t>(h)));
    return t;
  }();
  return lut.data();
}

void widen(const uint16_t *src, double *dst, size_t n) {
  const double *lut = half_lut();
  for (size_t i = 0; i < n; ++i) dst[i] = lut[src[i]];
}

int resolve_threads(int nthreads) {
  if (nthreads > 0) return nthreads;
  const unsigned hc = std::thread::hardware_concurrency();
  return hc ? static_cast<int>(hc) : 1;
}

// Runs body(worker, item) for item in [0, n) on `nthreads` workers, items handed out
// dynamically in blocks of `grain`.
template <class F>
void parallel_for(int n, int nthreads, int grain, F body) {
  nthreads = std::max(1, std::min(resolve_threads(nthreads), (n + grain - 1) / std::max(grain, 1)));
  std::atomic<int> next{0};
  auto work = [&](int w) {
    for (;;) {
      const int b = next.fetch_add(grain);
      if (b >= n) break;
      const int e = std::min(n, b + grain);
      for (int i = b; i < e; ++i) body(w, i);
    }
  };
  if (nthreads == 1) {
    work(0);
    return;
  }
  std::vector<std::thread> pool;
  for (int w = 0; w < nthreads; ++w) pool.emplace_back(work, w);
  for (auto &t : pool) t.join();
}

}  // namespace

extern "C" {

uint16_t oracle_f32_to_f16(float f) { return f32_to_f16(f); }
float oracle_f16_to_f32(uint16_t h) { return f16_to_f32(h); }

void oracle_f32_to_f16_array(const float *src, uint16_t *dst, size_t n) {
  for (size_t i = 0; i < n; ++i) dst[i] = f32_to_f16(src[i]);
}

// Inner update of one accumulator row over `n` columns: ac[j] += a * b[j], one product and
// one addition per element (no fused multiply-add: the library is built with
// -ffp-contract=off), so every element is summed exactly as the reference's loop sums it.
// Cloned for AVX2 and a baseline x86-64 target; the loader picks the one the CPU runs.
__attribute__((target_clones("avx2", "default"))) void axpy_row(double *ac, double a,
                                                               const float *b, int n) {
  for (int j = 0; j < n; ++j) ac[j] += a * static_cast<double>(b[j]);
}

// out[(r)*N + j] for the `nrows` rows listed in `rows` (any order, any subset).
// Cin may be null when beta == 0 (the reference never reads C then).
// B is widened to fp32 once (every binary16 value is exactly a float, and exactly the
// double it converts to); the work is split into tasks of up to kRowBlock rows x kColBlock
// columns whose accumulators stay in cache while k runs over all of K in increasing order.
void oracle_gemm_f64_rows(const uint16_t *A, const uint16_t *B, const uint16_t *Cin, double *out,
                          int M, int N, int K, double alpha, double beta, const int *rows,
                          int nrows, int nthreads) {
  (void)M;
  constexpr int kRowBlock = 8, kColBlock = 512;
  const double *lut = half_lut();
  std::vector<float> Bf(static_cast<size_t>(K) * N);
  parallel_for(K, nthreads, 16, [&](int, int k) {
    const uint16_t *b = B + static_cast<size_t>(k) * N;
    float *d = Bf.data() + static_cast<size_t>(k) * N;
    for (int j = 0; j < N; ++j) d[j] = static_cast<float>(lut[b[j]]);
  });
  const int nrb = (nrows + kRowBlock - 1) / kRowBlock;
  const int njt = (N + kColBlock - 1) / kColBlock;
  const int ntask = nrb * njt;
  const int nw = std::max(1, std::min(resolve_threads(nthreads), ntask));
  std::vector<std::vector<double>> acc_w(nw, std::vector<double>(kRowBlock * kColBlock));
  parallel_for(ntask, nw, 1, [&](int w, int task) {
    const int rbi = task / njt, jt = task % njt;
    const int t0 = rbi * kRowBlock, t1 = std::min(nrows, t0 + kRowBlock);
    const int j0 = jt * kColBlock, jw = std::min(N, j0 + kColBlock) - j0;
    double *acc = acc_w[w].data();
    std::fill(acc, acc + kRowBlock * kColBlock, 0.0);
    for (int k = 0; k < K; ++k) {
      const float *bk = Bf.data() + static_cast<size_t>(k) * N + j0;
      for (int t = t0; t < t1; ++t)
        axpy_row(acc + (t - t0) * kColBlock, lut[A[static_cast<size_t>(rows[t]) * K + k]], bk, jw);
    }
    for (int t = t0; t < t1; ++t) {
      const int i = rows[t];
      const double *ac = acc + (t - t0) * kColBlock;
      double *o = out + static_cast<size_t>(t) * N + j0;
      for (int j = 0; j < jw; ++j) {
        double r = alpha * ac[j];
        if (beta != 0.0)
          r += beta * static_cast<double>(f16_to_f32(Cin[static_cast<size_t>(i) * N + j0 + j]));
        o[j] = r;
      }
    }
  });
}

// Rows [row_begin, row_end) into out[(i - row_begin) * N + j].
void oracle_gemm_f64(const uint16_t *A, const uint16_t *B, const uint16_t *Cin, double *out,
                     int M, int N, int K, double alpha, double beta, int row_begin, int row_end,
                     int nthreads) {
  std::vector<int> rows;
  for (int i = row_begin; i < row_end; ++i) rows.push_back(i);
  oracle_gemm_f64_rows(A, B, Cin, out, M, N, K, alpha, beta, rows.data(),
                       static_cast<int>(rows.size()), nthreads);
}

// out[i * ncols + t] for the `ncols` columns listed in `cols`, all M rows.
void oracle_gemm_f64_cols(const uint16_t *A, const uint16_t *B, const uint16_t *Cin, double *out,
                          int M, int N, int K, double alpha, double beta, const int *cols,
                          int ncols, int nthreads) {
  std::vector<double> Bc(static_cast<size_t>(K) * ncols);  // Bc[t][k] = B[k][cols[t]]
  for (int t = 0; t < ncols; ++t)
    for (int k = 0; k < K; ++k)
      Bc[static_cast<size_t>(t) * K + k] =
          static_cast<double>(f16_to_f32(B[static_cast<size_t>(k) * N + cols[t]]));
  const int nw = std::max(1, std::min(resolve_threads(nthreads), M));
  std::vector<std::vector<double>> arow_w(nw, std::vector<double>(K));
  parallel_for(M, nw, 16, [&](int w, int i) {
    std::vector<double> &arow = arow_w[w];
    widen(A + static_cast<size_t>(i) * K, arow.data(), K);
    for (int t = 0; t < ncols; ++t) {
      const double *b = Bc.data() + static_cast<size_t>(t) * K;
      double acc = 0.0;
      for (int k = 0; k < K; ++k) acc += arow[k] * b[k];
      double r = alpha * acc;
      if (beta != 0.0)
        r += beta * static_cast<double>(f16_to_f32(Cin[static_cast<size_t>(i) * N + cols[t]]));
      out[static_cast<size_t>(i) * ncols + t] = r;
    }
  });
}

// The reference's literal loop nest (check_fp64.cu:39-44), single thread, rows
// [row_begin, row_end): for i, for j, for k with a stride-N walk down B's column.
void oracle_gemm_f64_ref_order(const uint16_t *A, const uint16_t *B, const uint16_t *Cin,
                               double *out, int M, int N, int K, double alpha, double beta,
                               int row_begin, int row_end) {
  (void)M;
  std::vector<float> fA(static_cast<size_t>(row_end - row_begin) * K), fB(static_cast<size_t>(K) * N);
  for (int i = row_begin; i < row_end; ++i)
    for (int k = 0; k < K; ++k)
      fA[static_cast<size_t>(i - row_begin) * K + k] = f16_to_f32(A[static_cast<size_t>(i) * K + k]);
  for (size_t x = 0; x < fB.size(); ++x) fB[x] = f16_to_f32(B[x]);
  for (int i = row_begin; i < row_end; ++i)
    for (int j = 0; j < N; ++j) {
      double acc = 0;
      for (int k = 0; k < K; ++k)
        acc += static_cast<double>(fA[static_cast<size_t>(i - row_begin) * K + k]) *
               fB[static_cast<size_t>(k) * N + j];
      double r = alpha * acc;
      if (beta != 0.0) r += beta * static_cast<double>(f16_to_f32(Cin[static_cast<size_t>(i) * N + j]));
      out[static_cast<size_t>(i - row_begin) * N + j] = r;
    }
}

// ------------------------------------------------------------------ seeded generators
void *oracle_mt_new(uint32_t seed) { return new std::mt19937(seed); }
void oracle_mt_free(void *g) { delete static_cast<std::mt19937 *>(g); }

// n draws of uniform_real_distribution<float>(lo, hi), each rounded to half.
void oracle_mt_uniform_half(void *g, uint16_t *out, size_t n, float lo, float hi) {
  std::mt19937 &rng = *static_cast<std::mt19937 *>(g);
  std::uniform_real_distribution<float> D(lo, hi);
  for (size_t i = 0; i < n; ++i) out[i] = f32_to_f16(D(rng));
}

// The raw float draws (before rounding), for cross-checking the generator itself.
void oracle_mt_uniform_f32(void *g, float *out, size_t n, float lo, float hi) {
  std::mt19937 &rng = *static_cast<std::mt19937 *>(g);
  std::uniform_real_distribution<float> D(lo, hi);
  for (size_t i = 0; i < n; ++i) out[i] = D(rng);
}

void oracle_mt_normal_half(void *g, uint16_t *out, size_t n, float mean, float stddev) {
  std::mt19937 &rng = *static_cast<std::mt19937 *>(g);
  std::normal_distribution<float> D(mean, stddev);
  for (size_t i = 0; i < n; ++i) out[i] = f32_to_f16(D(rng));
}

// three_way.cu:22-33: element i of a fill seeded `seed` (offset lets callers fill slices).
void oracle_hash_fill_half(uint16_t *out, size_t n, uint32_t seed, size_t offset) {
  for (size_t t = 0; t < n; ++t) {
    const size_t i = t + offset;
    uint32_t h = static_cast<uint32_t>(i * 2654435761u) ^ seed;
    h ^= h >> 15;
    h *= 2246822519u;
    h ^= h >> 13;
    h *= 3266489917u;
    h ^= h >> 16;
    out[t] = f32_to_f16((static_cast<float>(h & 0xffffu) / 32768.0f) - 1.0f);
  }
}

int oracle_max_threads(void) { return resolve_threads(0); }

}  // extern "C"
