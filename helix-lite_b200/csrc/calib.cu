// On-device calibration statistics: per group of samples, the outlier band
// and the nuq codebook.
//
// Follows xFuzzitx/helix-lite src/kvquant/calibration.py:106-188: for each
// group (K: one (head, channel) over the calibration tokens; V: one (head,
// position) over prompts x channels) the band is [quantile(x, p),
// quantile(x, 1 - p)] with numpy's default linear interpolation (numpy's
// float32 arithmetic for float32 samples), and the
// codebook is a 1-D k-means of the samples inside the band, centres sorted.
// The reference runs sklearn's KMeans (k-means++ seeding, n_init = 3, at most
// 20 iterations) on a random subsample of 5,000; here every in-band sample
// is used and the k-means is Lloyd's algorithm from equal-mass seeds, which in
// one dimension needs only the sorted samples and their prefix sums: a
// cluster is a contiguous run of the sorted samples, cut at the midpoints of
// adjacent centres (a sample exactly on a midpoint goes to the lower centre,
// the first of the equally near), so an iteration is 2 binary searches and 2
// prefix-sum reads per centre.
//
// One CTA per group; the samples come sorted ascending (the caller sorts
// them on the device).
#include <atomic>

#include "common.cuh"

namespace hx {

// numpy.quantile(x, q) for sorted float32 x with q a Python float (numpy 2,
// method "linear"; numpy/lib/_function_base_impl.py: quantile casts q to
// the array's float32, the virtual index is (n - 1) * q, _get_indexes clamps
// it to the ends, _lerp interpolates from the nearer end), in float32 with
// numpy's operation order, so the result is numpy's float32 value.
HX_DEVINL float np_quantile_sorted(const float* x, int64_t n, double q) {
  const float qf = (float)q;
  const float vi = __fmul_rn((float)(n - 1), qf);
  const float prev = floorf(vi);
  const float gamma = __fsub_rn(vi, prev);
  int64_t ip = (int64_t)prev, in = ip + 1;
  if (vi >= (float)(n - 1)) ip = in = n - 1;
  if (vi < 0.0f) ip = in = 0;
  const float a = x[ip], b = x[in];
  const float diff = __fsub_rn(b, a);
  if (gamma >= 0.5f) return __fsub_rn(b, __fmul_rn(diff, __fsub_rn(1.0f, gamma)));
  return __fadd_rn(a, __fmul_rn(diff, gamma));
}

// first index i in [lo, hi) with x[i] > t (x sorted), or hi
HX_DEVINL int64_t upper_bound(const float* x, int64_t lo, int64_t hi, double t) {
  while (lo < hi) {
    const int64_t mid = lo + ((hi - lo) >> 1);
    if ((double)x[mid] > t) hi = mid;
    else lo = mid + 1;
  }
  return lo;
}
// first index i in [lo, hi) with x[i] >= t, or hi
HX_DEVINL int64_t lower_bound(const float* x, int64_t lo, int64_t hi, double t) {
  while (lo < hi) {
    const int64_t mid = lo + ((hi - lo) >> 1);
    if ((double)x[mid] >= t) hi = mid;
    else lo = mid + 1;
  }
  return lo;
}

constexpr int kCalibThreads = 256;
constexpr int kMaxLevels = 16;
constexpr int kDpMax = 4096;  // points the exact k-means runs on (rank-stratified beyond)

// Per group: layer tables of the exact k-means (optimal SSE of the first i
// points in j clusters, the previous and the current layer) and the split
// points of every layer for the backtrack.
struct CalibSmem {
  double d[2][kDpMax + 1];
  uint16_t t[kMaxLevels][kDpMax + 1];
};

// scratch doubles per group: band prefix (n + 1), then the distinct points'
// count / sum / square-sum prefixes and their values (kDpMax + 1 each)
__host__ __device__ inline int64_t calib_row_doubles(int64_t n) { return n + 1 + 4 * (int64_t)(kDpMax + 1); }

// SSE of the distinct points [s, e) (weights W, sums S1, square sums S2)
HX_DEVINL double cluster_cost(const double* W, const double* S1, const double* S2, int s, int e) {
  const double n = __dsub_rn(W[e], W[s]), sum = __dsub_rn(S1[e], S1[s]), ss = __dsub_rn(S2[e], S2[s]);
  return __dsub_rn(ss, __ddiv_rn(__dmul_rn(sum, sum), n));
}

__global__ void __launch_bounds__(kCalibThreads, 1) calib_rows_kernel(const float* __restrict__ sorted, int64_t n,
                                                                     double q_lo, double q_hi, int k, int max_iter,
                                                                     float* lower, float* upper, float* centers,
                                                                     double* scratch, int32_t* iters_done) {
  extern __shared__ __align__(16) uint8_t calib_smem[];
  CalibSmem& sm = *reinterpret_cast<CalibSmem*>(calib_smem);
  __shared__ double s_c[kMaxLevels];
  __shared__ int64_t s_range[2];
  __shared__ double s_warp[kCalibThreads / 32];
  __shared__ int s_changed, s_U, s_kk;
  const int row = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const float* x = sorted + (int64_t)row * n;
  double* pre = scratch + (int64_t)row * calib_row_doubles(n);
  double* W = pre + (n + 1);
  double* S1 = W + (kDpMax + 1);
  double* S2 = S1 + (kDpMax + 1);
  double* U_val = S2 + (kDpMax + 1);
  if (tid == 0) {
    const float lo = np_quantile_sorted(x, n, q_lo), hi = np_quantile_sorted(x, n, q_hi);
    lower[row] = lo;
    upper[row] = hi;
    // the band's samples: lo <= x <= hi, compared in double as numpy does
    s_range[0] = lower_bound(x, 0, n, lo);
    s_range[1] = upper_bound(x, s_range[0], n, hi);
  }
  __syncthreads();
  const int64_t a = s_range[0], m = s_range[1] - s_range[0];
  // prefix sums of the band's samples in double: pre[i] = sum x[a .. a+i-1]
  double carry = 0.0;
  for (int64_t base = 0; base < m; base += kCalibThreads) {
    const int64_t i = base + tid;
    const double v = i < m ? (double)x[a + i] : 0.0;
    double incl = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const double y = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += y;
    }
    if (lane == 31) s_warp[warp] = incl;
    __syncthreads();
    double before = carry;
    for (int w = 0; w < warp; ++w) before += s_warp[w];
    if (i < m) pre[i + 1] = before + incl;
    double total = 0.0;
    for (int w = 0; w < kCalibThreads / 32; ++w) total += s_warp[w];
    __syncthreads();
    carry += total;
  }
  if (tid == 0) pre[0] = 0.0;
  __syncthreads();

  float* out = centers + (int64_t)row * k;
  if (m < k) {
    // the reference: zeros, the band's samples first, sorted (calibration.py:117-122)
    if (tid == 0) {
      float v[kMaxLevels];
      for (int j = 0; j < k; ++j) v[j] = j < m ? x[a + j] : 0.0f;
      for (int i = 1; i < k; ++i)  // insertion sort of at most 16 values
        for (int j = i; j > 0 && v[j - 1] > v[j]; --j) {
          const float t = v[j];
          v[j] = v[j - 1];
          v[j - 1] = t;
        }
      for (int j = 0; j < k; ++j) out[j] = v[j];
      if (iters_done) iters_done[row] = 0;
    }
    return;
  }

  // ---- the points of the exact k-means: every band sample, or kDpMax of
  // them stratified by rank; equal values merged into one weighted point.
  // One thread, in order, so the prefix sums are the sequential ones.
  if (tid == 0) {
    const int64_t N = m < kDpMax ? m : kDpMax;
    int U = 0;
    double w = 0.0, s1 = 0.0, s2 = 0.0;
    W[0] = S1[0] = S2[0] = 0.0;
    float cur = 0.0f;
    for (int64_t i = 0; i < N; ++i) {
      const int64_t r = m > kDpMax ? ((2 * i + 1) * m) / (2 * (int64_t)kDpMax) : i;
      const float v = x[a + r];
      if (U == 0 || v != cur) {
        if (U > 0) {
          W[U] = w;
          S1[U] = s1;
          S2[U] = s2;
        }
        U_val[U] = (double)v;
        cur = v;
        ++U;
      }
      const double dv = (double)v;
      w = __dadd_rn(w, 1.0);
      s1 = __dadd_rn(s1, dv);
      s2 = __dadd_rn(s2, __dmul_rn(dv, dv));
    }
    W[U] = w;
    S1[U] = s1;
    S2[U] = s2;
    s_U = U;
    s_kk = U < k ? U : k;
  }
  __syncthreads();
  const int U = s_U, kk = s_kk;
  if (kk == U) {
    // no more distinct points than levels: each is a centre (optimal)
    if (tid < k) s_c[tid] = U_val[tid < U ? tid : U - 1];
  } else {
    // layer 1: the first i points in one cluster
    for (int i = tid; i <= U; i += kCalibThreads) sm.d[0][i] = i >= 1 ? cluster_cost(W, S1, S2, 0, i) : 0.0;
    __syncthreads();
    // layers 2 .. kk: D_j(i) = min over s in [j-1, i-1] of D_{j-1}(s) + cost(s, i),
    // smallest s on ties; the smallest optimal s does not decrease with i, so
    // i's are solved middle first (a segment tree over [j, U], level by
    // level), each searching only between its solved neighbours' splits
    for (int j = 2; j <= kk; ++j) {
      const double* dp = sm.d[(j - 2) & 1];
      double* dc = sm.d[(j - 1) & 1];
      uint16_t* tj = sm.t[j - 1];
      const int R_lo = j, R_hi = U;
      for (int lvl = 0; lvl < 14; ++lvl) {
        const int nseg = 1 << lvl;
        for (int seg = warp; seg < nseg; seg += kCalibThreads / 32) {
          int lo = R_lo, hi = R_hi;
          for (int bit = lvl - 1; bit >= 0 && lo <= hi; --bit) {
            const int mid = (lo + hi) >> 1;
            if ((seg >> bit) & 1) lo = mid + 1;
            else hi = mid - 1;
          }
          if (lo > hi) continue;
          const int mid = (lo + hi) >> 1;
          const int s_lo = lo == R_lo ? j - 1 : (int)tj[lo - 1];
          const int s_hi = min(mid - 1, hi == R_hi ? R_hi - 1 : (int)tj[hi + 1]);
          double best = INFINITY;
          int bs = s_lo;
          for (int s = s_lo + lane; s <= s_hi; s += 32) {
            const double v = __dadd_rn(dp[s], cluster_cost(W, S1, S2, s, mid));
            if (v < best) {
              best = v;
              bs = s;
            }
          }
#pragma unroll
          for (int o = 16; o; o >>= 1) {
            const double ov = __shfl_xor_sync(0xffffffffu, best, o);
            const int os = __shfl_xor_sync(0xffffffffu, bs, o);
            if (ov < best || (ov == best && os < bs)) {
              best = ov;
              bs = os;
            }
          }
          if (lane == 0) {
            dc[mid] = best;
            tj[mid] = (uint16_t)bs;
          }
        }
        __syncthreads();
      }
    }
    // backtrack: the clusters' weighted means, ascending
    if (tid == 0) {
      int e = U;
      for (int j = kk; j >= 1; --j) {
        const int s = j == 1 ? 0 : (int)sm.t[j - 1][e];
        s_c[j - 1] = __ddiv_rn(__dsub_rn(S1[e], S1[s]), __dsub_rn(W[e], W[s]));
        e = s;
      }
    }
  }
  __syncthreads();
  // ---- Lloyd steps over every band sample from there (they never raise the SSE)
  int it = 0;
  for (; it < max_iter; ++it) {
    double nc = 0.0;
    bool moved = false;
    if (tid < k) {
      // cluster tid: samples above the midpoint with centre tid - 1, up to
      // and including the midpoint with centre tid + 1
      const int64_t b0 = tid == 0 ? 0 : upper_bound(x + a, 0, m, 0.5 * (s_c[tid - 1] + s_c[tid]));
      const int64_t b1 = tid == k - 1 ? m : upper_bound(x + a, 0, m, 0.5 * (s_c[tid] + s_c[tid + 1]));
      nc = s_c[tid];
      if (b1 > b0) nc = (pre[b1] - pre[b0]) / (double)(b1 - b0);
      moved = nc != s_c[tid];
    }
    if (tid == 0) s_changed = 0;
    __syncthreads();
    if (tid < k) {
      s_c[tid] = nc;
      if (moved) s_changed = 1;
    }
    __syncthreads();
    const int changed = s_changed;
    __syncthreads();  // every thread has read the flag before thread 0 clears it again
    if (!changed) break;
  }
  if (tid < k) out[tid] = (float)s_c[tid];
  if (tid == 0 && iters_done) iters_done[row] = it;
}

}  // namespace hx

using namespace hx;

extern "C" {

HX_API int64_t hx_calib_scratch_bytes(int32_t rows, int64_t n) {
  if (rows < 0 || n < 1) return -1;
  return (int64_t)rows * calib_row_doubles(n) * (int64_t)sizeof(double);
}

HX_API int hx_calib_rows(void* stream, const float* sorted, int32_t rows, int64_t n, double q_low, double q_high,
                         int32_t k, int32_t max_iter, float* lower, float* upper, float* centers, double* scratch,
                         int32_t* iters_done) {
  if (rows < 0 || n < 1 || k < 1 || k > kMaxLevels || max_iter < 0 || !(q_low >= 0.0) || !(q_high <= 1.0) ||
      q_low > q_high)
    return HX_ERR_ARG;
  if (rows == 0) return HX_OK;
  if (!sorted || !lower || !upper || !centers || !scratch) return HX_ERR_ARG;
  static std::atomic<bool> attr_set[64];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return HX_ERR_LAUNCH;
  if (!attr_set[dev].load(std::memory_order_acquire)) {
    if (cudaFuncSetAttribute(calib_rows_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)sizeof(CalibSmem)) != cudaSuccess)
      return HX_ERR_LAUNCH;
    attr_set[dev].store(true, std::memory_order_release);
  }
  calib_rows_kernel<<<rows, kCalibThreads, sizeof(CalibSmem), reinterpret_cast<cudaStream_t>(stream)>>>(
      sorted, n, q_low, q_high, k, max_iter, lower, upper, centers, scratch, iters_done);
  HX_LAUNCH_CHECK();
  return HX_OK;
}

}  // extern "C"
