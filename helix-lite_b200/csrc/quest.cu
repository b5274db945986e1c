// Kernel B: Quest page statistics, page scores and exact top-K selection.
//
// Follows xFuzzitx/helix-lite src/quest/reference.py:
//   compute_page_stats      :38-56  slot-axis min / max
//   page_upper_bound        :59-93  sum_d max(q,0)*kmax + min(q,0)*kmin
//   topk_pages_with_sinks   :96-133 sinks forced, best k of the rest, ascending
// and the GQA contraction of src/kvquant/compact_backend.py:225-231.
// The score arithmetic order is pinned (see hx_quest_scores in helix_kv.h) so
// the CPU oracle reproduces every bit and the selection is exact; ties in
// score go to the lower page index.
#include "common.cuh"

namespace hx {

constexpr int kBins = 4096;  // first-level histogram: top 12 bits of the key

// ---------------------------------------------------------------------------
// compute_page_stats

template <typename T>
HX_DEVINL float ldv(const T* p, int64_t i);
template <>
HX_DEVINL float ldv<float>(const float* p, int64_t i) { return p[i]; }
template <>
HX_DEVINL float ldv<uint16_t>(const uint16_t* p, int64_t i) { return h2f(p[i]); }

template <typename T>
HX_DEVINL void stv(T* p, int64_t i, float v);
template <>
HX_DEVINL void stv<float>(float* p, int64_t i, float v) { p[i] = v; }
template <>
HX_DEVINL void stv<uint16_t>(uint16_t* p, int64_t i, float v) { p[i] = f2h(v); }

template <typename T>
__global__ void page_stats_kernel(const T* k, int P, int S, int H, int D, T* kmin, T* kmax) {
  int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;  // over (P, H, D)
  int64_t n = (int64_t)P * H * D;
  if (i >= n) return;
  int64_t hd = i % ((int64_t)H * D);
  int64_t p = i / ((int64_t)H * D);
  float mn = ldv(k, (p * S) * H * D + hd), mx = mn;
  for (int s = 1; s < S; ++s) {
    float x = ldv(k, (p * S + s) * H * D + hd);
    mn = x < mn ? x : mn;
    mx = x > mx ? x : mx;
  }
  stv(kmin, i, mn);
  stv(kmax, i, mx);
}

// ---------------------------------------------------------------------------
// page scores

// Group terms of KV head h (pinned, see the oracle quest.py).
HX_DEVINL void group_terms(const uint16_t* q, int64_t qbase, int G, int D, int mode, int d, float& qp,
                           float& qn) {
  if (mode == 0) {
    qp = 0.0f;
    qn = 0.0f;
    for (int g = 0; g < G; ++g) {
      float x = h2f(q[qbase + (int64_t)g * D + d]);
      qp = __fadd_rn(qp, x > 0.0f ? x : 0.0f);
      qn = __fadd_rn(qn, x < 0.0f ? x : 0.0f);
    }
  } else {
    float s = 0.0f;
    for (int g = 0; g < G; ++g) s = __fadd_rn(s, h2f(q[qbase + (int64_t)g * D + d]));
    float m = h2f(f2h(__fdiv_rn(s, (float)G)));
    qp = m > 0.0f ? m : 0.0f;
    qn = m < 0.0f ? m : 0.0f;
  }
}

// One warp per (page, KV head); 8 warps per block, blockIdx.y = b * H + h.
template <typename TS, int V>
__global__ void __launch_bounds__(256) quest_scores_kernel(const uint16_t* __restrict__ q, int H, int G, int D,
                                                           int mode, const TS* __restrict__ kmin,
                                                           const TS* __restrict__ kmax, int64_t page_stride,
                                                           int64_t head_stride, const int32_t* __restrict__ bt,
                                                           int bt_stride, const int32_t* __restrict__ seq_lens,
                                                           int S, int max_pages, int sinks_req, int pages_per_block,
                                                           float* __restrict__ scores, uint32_t* __restrict__ hist) {
  __shared__ float s_qp[32 * V], s_qn[32 * V];
  const int bh = blockIdx.y;
  const int b = bh / H, h = bh % H;
  for (int d = threadIdx.x; d < 32 * V; d += blockDim.x) {
    float qp = 0.0f, qn = 0.0f;
    if (d < D) group_terms(q, ((int64_t)b * H * G + (int64_t)h * G) * D, G, D, mode, d, qp, qn);
    s_qp[d] = qp;
    s_qn[d] = qn;
  }
  __syncthreads();
  const int n = (seq_lens[b] + S - 1) / S;
  const int sinks = min(max(sinks_req, 0), n);
  const int lane = lane_id(), warp = threadIdx.x >> 5;
  const int j0 = blockIdx.x * pages_per_block;
  const int j1 = min(j0 + pages_per_block, min(n, max_pages));
  float qp[V], qn[V];
#pragma unroll
  for (int v = 0; v < V; ++v) {
    qp[v] = s_qp[V * lane + v];
    qn[v] = s_qn[V * lane + v];
  }
  for (int j = j0 + warp; j < j1; j += 8) {
    const int64_t phys = bt ? (int64_t)bt[(int64_t)b * bt_stride + j] : (int64_t)j;
    const TS* pmin = kmin + phys * page_stride + (int64_t)h * head_stride;
    const TS* pmax = kmax + phys * page_stride + (int64_t)h * head_stride;
    float acc = 0.0f;
    if (sizeof(TS) == 2 && V == 4 && 32 * V == D) {
      // fast path: 4 fp16 per lane, one 8-byte load per stat
      uint2 a = *reinterpret_cast<const uint2*>(pmax + 4 * lane);
      uint2 c = *reinterpret_cast<const uint2*>(pmin + 4 * lane);
      uint16_t xa[4] = {(uint16_t)(a.x & 0xffff), (uint16_t)(a.x >> 16), (uint16_t)(a.y & 0xffff),
                        (uint16_t)(a.y >> 16)};
      uint16_t xc[4] = {(uint16_t)(c.x & 0xffff), (uint16_t)(c.x >> 16), (uint16_t)(c.y & 0xffff),
                        (uint16_t)(c.y >> 16)};
#pragma unroll
      for (int v = 0; v < 4; ++v) {
        acc = __fadd_rn(acc, __fmul_rn(qp[v], h2f(xa[v])));
        acc = __fadd_rn(acc, __fmul_rn(qn[v], h2f(xc[v])));
      }
    } else {
#pragma unroll
      for (int v = 0; v < V; ++v) {
        int d = V * lane + v;
        if (d < D) {
          acc = __fadd_rn(acc, __fmul_rn(qp[v], ldv(pmax, d)));
          acc = __fadd_rn(acc, __fmul_rn(qn[v], ldv(pmin, d)));
        }
      }
    }
#pragma unroll
    for (int m = 16; m >= 1; m >>= 1) acc = __fadd_rn(acc, __shfl_xor_sync(0xffffffffu, acc, m));
    if (lane == 0) {
      scores[(int64_t)bh * max_pages + j] = acc;
      if (hist && j >= sinks) atomicAdd(&hist[(int64_t)bh * kBins + (order_key(acc) >> 20)], 1u);
    }
  }
}

// Histogram of given scores (for the API path where scores come from outside).
__global__ void quest_hist_kernel(const float* scores, int H, const int32_t* seq_lens, int S, int max_pages,
                                  int sinks_req, uint32_t* hist) {
  const int bh = blockIdx.y;
  const int b = bh / H;
  const int n = min((seq_lens[b] + S - 1) / S, max_pages);
  const int sinks = min(max(sinks_req, 0), n);
  for (int j = blockIdx.x * blockDim.x + threadIdx.x; j < n; j += gridDim.x * blockDim.x)
    if (j >= sinks) atomicAdd(&hist[(int64_t)bh * kBins + (order_key(scores[(int64_t)bh * max_pages + j]) >> 20)], 1u);
}

// ---------------------------------------------------------------------------
// exact threshold (radix select), last-block finish: no inter-block waits

struct SelPlan {
  int n, sinks, k_eff;
};

HX_DEVINL SelPlan plan_for(int seq_len, int S, int max_pages, int sinks_req, int k_fixed, int fnum, int fden) {
  SelPlan p;
  p.n = min((seq_len + S - 1) / S, max_pages);
  p.sinks = min(max(sinks_req, 0), p.n);
  long long kb = fden > 0 ? (long long)p.n * fnum / fden : (long long)k_fixed;
  long long ke = kb < (long long)(p.n - p.sinks) ? kb : (long long)(p.n - p.sinks);
  p.k_eff = (int)(ke > 0 ? ke : 0);
  return p;
}

// Block-wide: find the highest bin b* whose suffix count reaches `need`.
// Returns b* and writes the count strictly above it. blockDim == 256.
HX_DEVINL int find_boundary(const uint32_t* s_hist, uint32_t need, uint32_t& above, int* s_tmp) {
  // thread t owns bins [16t, 16t+16); suffix sums over threads from the top
  const int t = threadIdx.x;
  uint32_t local = 0;
  for (int i = 0; i < 16; ++i) local += s_hist[16 * t + i];
  s_tmp[t] = (int)local;
  __syncthreads();
  if (t == 0) {
    uint32_t acc = 0;
    int found = -1;
    uint32_t above_v = 0;
    for (int u = 255; u >= 0 && found < 0; --u) {
      uint32_t c = (uint32_t)s_tmp[u];
      if (acc + c >= need) {
        for (int bin = 16 * u + 15; bin >= 16 * u; --bin) {
          uint32_t hb = s_hist[bin];
          if (acc + hb >= need) {
            found = bin;
            above_v = acc;
            break;
          }
          acc += hb;
        }
      } else {
        acc += c;
      }
    }
    s_tmp[256] = found;
    s_tmp[257] = (int)above_v;
  }
  __syncthreads();
  above = (uint32_t)s_tmp[257];
  int r = s_tmp[256];
  __syncthreads();
  return r;
}

// Select the r-th largest among `cnt` unique 64-bit keys sharing their top 12
// bits, by 8-bit digit passes from bit 51 down. Returns the threshold T with
// exactly r keys >= T (among the candidates). blockDim == 256.
HX_DEVINL uint64_t radix_select(const uint64_t* cand, uint32_t cnt, uint32_t r, uint64_t prefix, uint32_t* s_h,
                                int* s_tmp) {
  uint64_t mask = 0xFFF0000000000000ull;
  int shift = 52;
  while (shift > 0) {
    int width = shift >= 8 ? 8 : shift;
    shift -= width;
    const uint32_t nb = 1u << width;
    for (int i = threadIdx.x; i < 256; i += blockDim.x) s_h[i] = 0;
    __syncthreads();
    for (uint32_t i = threadIdx.x; i < cnt; i += blockDim.x) {
      uint64_t key = cand[i];
      if ((key & mask) == prefix) atomicAdd(&s_h[(key >> shift) & (nb - 1)], 1u);
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      uint32_t acc = 0;
      int dsel = 0;
      for (int dg = (int)nb - 1; dg >= 0; --dg) {
        if (acc + s_h[dg] >= r) {
          dsel = dg;
          break;
        }
        acc += s_h[dg];
      }
      s_tmp[0] = dsel;
      s_tmp[1] = (int)acc;
      s_tmp[2] = (int)s_h[dsel];
    }
    __syncthreads();
    const uint64_t dsel = (uint64_t)s_tmp[0];
    r -= (uint32_t)s_tmp[1];
    const uint32_t in_bin = (uint32_t)s_tmp[2];
    __syncthreads();
    prefix |= dsel << shift;
    mask |= (uint64_t)(nb - 1) << shift;
    if (in_bin == r) return prefix;  // every key with this prefix is selected
  }
  return prefix;
}

__global__ void __launch_bounds__(256) quest_threshold_kernel(const float* __restrict__ scores, int H,
                                                              const int32_t* __restrict__ seq_lens, int S,
                                                              int max_pages, int sinks_req, int k_fixed, int fnum,
                                                              int fden, uint32_t* hist, uint64_t* cand,
                                                              uint32_t* counters, uint64_t* thresh, uint32_t* err) {
  __shared__ uint32_t s_hist[kBins];
  __shared__ int s_tmp[260];
  __shared__ uint32_t s_h2[256];
  __shared__ int s_last;
  const int bh = blockIdx.y;
  const int b = bh / H;
  const int C = gridDim.x;
  const SelPlan pl = plan_for(seq_lens[b], S, max_pages, sinks_req, k_fixed, fnum, fden);
  uint32_t* hist_bh = hist + (int64_t)bh * kBins;
  uint32_t* ctr = counters + 2 * (int64_t)bh;
  uint64_t* cand_bh = cand + (int64_t)bh * max_pages;
  const int n_ns = pl.n - pl.sinks;

  int bstar = -1;
  uint32_t above = 0, r = 0;
  const bool trivial = (pl.k_eff == 0) || (pl.k_eff >= n_ns);
  if (!trivial) {
    for (int i = threadIdx.x; i < kBins; i += blockDim.x) s_hist[i] = hist_bh[i];
    __syncthreads();
    bstar = find_boundary(s_hist, (uint32_t)pl.k_eff, above, s_tmp);
    r = (uint32_t)pl.k_eff - above;
    const bool full_bin = bstar >= 0 && s_hist[bstar] == r;
    if (bstar >= 0 && !full_bin) {
      // collect this block's candidates of bin b*
      const int per = (n_ns + C - 1) / C;
      const int a = pl.sinks + blockIdx.x * per;
      const int e = min(a + per, pl.n);
      for (int base = a; base < e; base += blockDim.x) {
        int j = base + threadIdx.x;
        bool hit = false;
        uint64_t key = 0;
        if (j < e) {
          float s = scores[(int64_t)bh * max_pages + j];
          hit = (int)(order_key(s) >> 20) == bstar;
          key = order_key64(s, (uint32_t)j);
        }
        uint32_t m = __ballot_sync(0xffffffffu, hit);
        uint32_t pos = 0;
        if (lane_id() == 0 && m) pos = atomicAdd(&ctr[0], (uint32_t)__popc(m));
        pos = __shfl_sync(0xffffffffu, pos, 0);
        if (hit) cand_bh[pos + __popc(m & ((1u << lane_id()) - 1))] = key;
      }
    }
  }
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) s_last = (atomicAdd(&ctr[1], 1u) == (uint32_t)(C - 1));
  __syncthreads();
  if (!s_last) return;
  __threadfence();

  uint64_t T;
  if (pl.k_eff == 0) {
    T = ~0ull;
  } else if (pl.k_eff >= n_ns) {
    T = 0ull;
  } else if (bstar < 0) {
    T = 0ull;
    if (threadIdx.x == 0) set_err(err, HX_DEV_ERR_SELECT);
  } else if (s_hist[bstar] == r) {
    T = (uint64_t)bstar << 52;
  } else {
    const uint32_t cnt = *((volatile uint32_t*)&ctr[0]);
    if (cnt != s_hist[bstar] && threadIdx.x == 0) set_err(err, HX_DEV_ERR_SELECT);
    T = radix_select(cand_bh, cnt, r, (uint64_t)bstar << 52, s_h2, s_tmp);
  }
  if (threadIdx.x == 0) {
    thresh[bh] = T;
    ctr[0] = 0;
    ctr[1] = 0;
  }
  for (int i = threadIdx.x; i < kBins; i += blockDim.x) hist_bh[i] = 0;
}

// ---------------------------------------------------------------------------
// compaction to ascending page lists (API output; the decode reads thresholds)

HX_DEVINL bool page_selected(const float* scores_bh, uint64_t T, int j, int sinks) {
  if (j < sinks) return true;
  return order_key64(scores_bh[j], (uint32_t)j) >= T;
}

__global__ void __launch_bounds__(1024) quest_compact_kernel(const float* scores, const uint64_t* thresh, int H,
                                                             const int32_t* seq_lens, int S, int max_pages,
                                                             int sinks_req, int union_heads, int max_out,
                                                             int32_t* out, int32_t* counts) {
  __shared__ int s_warp[32];
  __shared__ int s_round;
  __shared__ int s_base;
  const int row = blockIdx.x;  // (b, h), or b for the union over heads
  const int b = union_heads ? row : row / H;
  const int n = min((seq_lens[b] + S - 1) / S, max_pages);
  const int sinks = min(max(sinks_req, 0), n);
  if (threadIdx.x == 0) s_base = 0;
  __syncthreads();
  const int lane = lane_id(), warp = threadIdx.x >> 5;
  for (int base = 0; base < n; base += blockDim.x) {
    int j = base + threadIdx.x;
    bool sel = false;
    if (j < n) {
      if (union_heads) {
        for (int h = 0; h < H && !sel; ++h)
          sel = page_selected(scores + ((int64_t)b * H + h) * max_pages, thresh[(int64_t)b * H + h], j, sinks);
      } else {
        sel = page_selected(scores + (int64_t)row * max_pages, thresh[row], j, sinks);
      }
    }
    uint32_t m = __ballot_sync(0xffffffffu, sel);
    if (lane == 0) s_warp[warp] = __popc(m);
    __syncthreads();
    if (threadIdx.x == 0) {
      int acc = 0;
      for (int w = 0; w < (int)(blockDim.x >> 5); ++w) {
        int c = s_warp[w];
        s_warp[w] = acc;
        acc += c;
      }
      s_round = acc;
    }
    __syncthreads();
    if (sel) {
      int pos = s_base + s_warp[warp] + __popc(m & ((1u << lane) - 1));
      if (pos < max_out) out[(int64_t)row * max_out + pos] = j;
    }
    __syncthreads();
    if (threadIdx.x == 0) s_base += s_round;
    __syncthreads();
  }
  if (threadIdx.x == 0) counts[row] = min(s_base, max_out);
}

}  // namespace hx

// ===========================================================================
// C ABI

using namespace hx;

static inline cudaStream_t S_(void* s) { return reinterpret_cast<cudaStream_t>(s); }

extern "C" {

HX_API int hx_page_stats(void* stream, int32_t dtype, const void* k_pages, int32_t P, int32_t S, int32_t H,
                         int32_t D, void* kmin, void* kmax) {
  if ((dtype != 0 && dtype != 1) || P < 0 || S <= 0 || H <= 0 || D <= 0) return HX_ERR_ARG;
  int64_t n = (int64_t)P * H * D;
  if (n == 0) return HX_OK;
  if (!k_pages || !kmin || !kmax) return HX_ERR_ARG;
  unsigned blocks = (unsigned)((n + 255) / 256);
  if (dtype == 0)
    page_stats_kernel<float><<<blocks, 256, 0, S_(stream)>>>((const float*)k_pages, P, S, H, D, (float*)kmin,
                                                             (float*)kmax);
  else
    page_stats_kernel<uint16_t><<<blocks, 256, 0, S_(stream)>>>((const uint16_t*)k_pages, P, S, H, D,
                                                                (uint16_t*)kmin, (uint16_t*)kmax);
  HX_LAUNCH_CHECK();
  return HX_OK;
}

HX_API int hx_quest_scores(void* stream, const uint16_t* q, int32_t B, int32_t H, int32_t group, int32_t D,
                           int32_t gqa_mode, int32_t stats_dtype, const void* kmin, const void* kmax,
                           int64_t page_stride, int64_t head_stride, const int32_t* block_table, int32_t bt_stride,
                           const int32_t* seq_lens, int32_t page_size, int32_t max_pages, int32_t sink_pages,
                           float* scores, uint32_t* hist) {
  if (B < 0 || H <= 0 || group <= 0 || D <= 0 || D > 256 || page_size <= 0 || max_pages < 0) return HX_ERR_ARG;
  if ((gqa_mode != 0 && gqa_mode != 1) || (stats_dtype != 0 && stats_dtype != 1)) return HX_ERR_ARG;
  if (B == 0 || max_pages == 0) return HX_OK;
  if (!q || !kmin || !kmax || !seq_lens || !scores) return HX_ERR_ARG;
  const int ppb = 64;
  dim3 grid((max_pages + ppb - 1) / ppb, B * H);
  cudaStream_t s = S_(stream);
  const int V = (D + 31) / 32;
#define HX_SC(TS_, V_)                                                                                      \
  quest_scores_kernel<TS_, V_><<<grid, 256, 0, s>>>(q, H, group, D, gqa_mode, (const TS_*)kmin, (const TS_*)kmax, \
                                                    page_stride, head_stride, block_table, bt_stride, seq_lens,    \
                                                    page_size, max_pages, sink_pages, ppb, scores, hist)
  bool aligned = (((uintptr_t)kmin | (uintptr_t)kmax) & 7) == 0 && page_stride % 4 == 0 && head_stride % 4 == 0;
  if (stats_dtype == 1) {
    if (V == 4 && D == 128 && !aligned) return HX_ERR_ARG;
    if (V == 1) HX_SC(uint16_t, 1);
    else if (V == 2) HX_SC(uint16_t, 2);
    else if (V <= 4) HX_SC(uint16_t, 4);
    else HX_SC(uint16_t, 8);
  } else {
    if (V == 1) HX_SC(float, 1);
    else if (V == 2) HX_SC(float, 2);
    else if (V <= 4) HX_SC(float, 4);
    else HX_SC(float, 8);
  }
#undef HX_SC
  HX_LAUNCH_CHECK();
  return HX_OK;
}

HX_API int hx_quest_threshold(void* stream, const float* scores, int32_t B, int32_t H, const int32_t* seq_lens,
                              int32_t page_size, int32_t max_pages, int32_t sink_pages, int32_t k_fixed,
                              int32_t frac_num, int32_t frac_den, int32_t hist_ready, uint32_t* hist,
                              uint64_t* cand, uint32_t* counters, uint64_t* thresh, uint32_t* dev_err) {
  if (B < 0 || H <= 0 || page_size <= 0 || max_pages < 0 || frac_den < 0) return HX_ERR_ARG;
  if (B == 0) return HX_OK;
  if (!scores || !seq_lens || !hist || !cand || !counters || !thresh) return HX_ERR_ARG;
  cudaStream_t st = S_(stream);
  if (!hist_ready) {
    dim3 hg((max_pages + 255) / 256 < 64 ? (max_pages + 255) / 256 : 64, B * H);
    if (hg.x == 0) hg.x = 1;
    quest_hist_kernel<<<hg, 256, 0, st>>>(scores, H, seq_lens, page_size, max_pages, sink_pages, hist);
  }
  int C = (max_pages + 4095) / 4096;
  C = C < 1 ? 1 : (C > 64 ? 64 : C);
  dim3 grid(C, B * H);
  quest_threshold_kernel<<<grid, 256, 0, st>>>(scores, H, seq_lens, page_size, max_pages, sink_pages,
                                                       k_fixed, frac_num, frac_den, hist, cand, counters, thresh,
                                                       dev_err);
  HX_LAUNCH_CHECK();
  return HX_OK;
}

HX_API int hx_quest_compact(void* stream, const float* scores, const uint64_t* thresh, int32_t B, int32_t H,
                            const int32_t* seq_lens, int32_t page_size, int32_t max_pages, int32_t sink_pages,
                            int32_t union_heads, int32_t max_out, int32_t* out, int32_t* counts) {
  if (B < 0 || H <= 0 || page_size <= 0 || max_pages < 0 || max_out < 0) return HX_ERR_ARG;
  if (B == 0) return HX_OK;
  if (!scores || !thresh || !seq_lens || !counts || (max_out > 0 && !out)) return HX_ERR_ARG;
  int rows = union_heads ? B : B * H;
  quest_compact_kernel<<<rows, 1024, 0, S_(stream)>>>(scores, thresh, H, seq_lens, page_size, max_pages, sink_pages,
                                                      union_heads, max_out, out, counts);
  HX_LAUNCH_CHECK();
  return HX_OK;
}

}  // extern "C"
