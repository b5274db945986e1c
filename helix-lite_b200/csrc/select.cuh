// Exact top-K threshold of one (sequence, KV head) row inside a CTA of NT
// threads, for the decode's fused selection (HX_SEL_FUSED). The algorithm
// and its results are those of the threshold kernels in quest.cu (level-1
// histogram from the scoring kernel, boundary bin, candidates with a level-2
// histogram, exact rank of the boundary keys; ties to the lower page), with
// every candidate held in shared memory: rows of at most kFusedMaxPages.
#pragma once

#include "common.cuh"

namespace hx {
namespace fsel {

constexpr int kBins = 4096;
constexpr int kMaxSlices = 128;
constexpr int kFusedMaxPages = 16384;

HX_DEVINL int64_t bin_rel(uint32_t key, uint32_t anchor) {
  return (int64_t)key - (int64_t)anchor + ((int64_t)(kBins / 2) << 16);
}
HX_DEVINL int bin1(uint32_t key, uint32_t anchor) {
  const int64_t e = bin_rel(key, anchor);
  return e < 0 ? 0 : (int)min(e >> 16, (int64_t)(kBins - 1));
}
HX_DEVINL int bin2(uint32_t key, uint32_t anchor) { return (int)((bin_rel(key, anchor) >> 4) & (kBins - 1)); }
HX_DEVINL bool edge_bin(int b) { return b == 0 || b == kBins - 1; }
HX_DEVINL uint64_t bin_floor(int b1, int b2, uint32_t anchor) {
  if (b1 == 0 && b2 < 0) return 0ull;
  int64_t lo = (int64_t)anchor + ((int64_t)(b1 - kBins / 2) << 16) + (b2 > 0 ? 16ll * b2 : 0ll);
  lo = lo < 0 ? 0 : (lo > 0xFFFFFFFFll ? 0xFFFFFFFFll : lo);
  return (uint64_t)lo << 32;
}

template <int NT>
struct RowSel {
  uint32_t hist[kBins];     // level 1, then level 2, then the level-2 bin's keys
  uint64_t cand[kFusedMaxPages];
  uint32_t add[kMaxSlices];  // selected non-sink pages per slice
  uint32_t warp[NT / 32];
  uint32_t h2[256];
  int res[4];
  uint32_t nc;
  uint64_t T;
};

// Block-wide locate over NT threads: thread t owns count c_t; with suffix
// sums S_t = sum_{u >= t} c_u, the t with S_{t+1} < need <= S_t (or -1), and
// S_{t+1} in `above`.
template <int NT>
HX_DEVINL int suffix_locate(uint32_t c, uint32_t need, uint32_t& above, RowSel<NT>& s) {
  constexpr int NW = NT / 32;
  const int t = threadIdx.x, lane = t & 31, w = t >> 5;
  uint32_t v = c;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const uint32_t x = __shfl_down_sync(0xffffffffu, v, o);
    if (lane + o < 32) v += x;
  }
  if (lane == 0) s.warp[w] = v;
  if (t == 0) s.res[0] = -1;
  __syncthreads();
  uint32_t later = 0;
  for (int u = w + 1; u < NW; ++u) later += s.warp[u];
  const uint32_t incl = v + later, excl = incl - c;
  if (excl < need && incl >= need) {
    s.res[0] = t;
    s.res[1] = (int)excl;
  }
  __syncthreads();
  const int r = s.res[0];
  above = r >= 0 ? (uint32_t)s.res[1] : 0u;
  __syncthreads();
  return r;
}

// highest bin of s.hist whose suffix count reaches `need`
template <int NT>
HX_DEVINL int find_boundary(uint32_t need, uint32_t& above, RowSel<NT>& s) {
  constexpr int PER = kBins / NT;
  const int t = threadIdx.x;
  uint32_t local = 0;
#pragma unroll
  for (int i = 0; i < PER; ++i) local += s.hist[PER * t + i];
  uint32_t above_t;
  const int owner = suffix_locate<NT>(local, need, above_t, s);
  if (owner < 0) return -1;
  if (t == owner) {
    uint32_t acc = above_t;
    int found = PER * t;
    for (int bin = PER * t + PER - 1; bin >= PER * t; --bin) {
      if (acc + s.hist[bin] >= need) {
        found = bin;
        break;
      }
      acc += s.hist[bin];
    }
    s.res[2] = found;
    s.res[3] = (int)acc;
  }
  __syncthreads();
  above = (uint32_t)s.res[3];
  const int r = s.res[2];
  __syncthreads();
  return r;
}

// the r-th largest of cnt keys (8-bit digits from the top)
template <int NT>
HX_DEVINL uint64_t radix_select(const uint64_t* cand, uint32_t cnt, uint32_t r, RowSel<NT>& s) {
  uint64_t prefix = 0ull, mask = 0ull;
  int shift = 64;
  while (shift > 0) {
    shift -= 8;
    if (threadIdx.x < 256) s.h2[threadIdx.x] = 0;
    __syncthreads();
    for (uint32_t i = threadIdx.x; i < cnt; i += NT)
      if ((cand[i] & mask) == prefix) atomicAdd(&s.h2[(cand[i] >> shift) & 255u], 1u);
    __syncthreads();
    uint32_t above;
    const int dsel = suffix_locate<NT>(threadIdx.x < 256 ? s.h2[threadIdx.x] : 0u, r, above, s);
    const uint32_t in_bin = dsel >= 0 ? s.h2[dsel] : 0u;
    __syncthreads();
    if (dsel < 0) return prefix;
    r -= above;
    prefix |= (uint64_t)dsel << shift;
    mask |= 255ull << shift;
    if (in_bin == r) return prefix;
  }
  return prefix;
}

// Threshold of the row (n pages, `sinks` forced, k_eff of the rest) and its
// slices' selected counts in s.add (C slices of ceil((n - sinks) / C) pages).
// All NT threads call it; returns T (the same in every thread).
template <int NT>
HX_DEVINL uint64_t row_select(const float* __restrict__ sc, const uint32_t* __restrict__ hist_g, int n, int sinks,
                              int k_eff, int C, RowSel<NT>& s, uint32_t* err) {
  const int tid = threadIdx.x;
  const int n_ns = n - sinks;
  const int per = n_ns > 0 ? (n_ns + C - 1) / C : 1;
  // slice of a non-sink offset x (0 <= x < kFusedMaxPages): x / per by a
  // multiply with per's rounded-up 32-bit reciprocal, exact for every x below
  // 2^18 and per >= 2 (checked for all x, per < 2^14 + 1); per = 1 is x itself.
  // The division it replaces cost two ~35-instruction sequences a thread and
  // round, 0.74 of the pass's 1.2 us a round at 8,192 pages on B200.
  const uint32_t per_m = per > 1 ? (uint32_t)((0x100000000ull + (uint64_t)per - 1ull) / (uint64_t)per) : 0u;
  auto slice_of = [&](int x) -> int { return per > 1 ? (int)__umulhi((uint32_t)x, per_m) : x; };
  const bool trivial = k_eff == 0 || k_eff >= n_ns;
  for (int i = tid; i < C; i += NT) s.add[i] = (trivial && k_eff > 0) ? (uint32_t)max(0, min(per, n_ns - i * per)) : 0u;
  if (tid == 0) {
    s.nc = 0;
    s.T = k_eff == 0 ? ~0ull : 0ull;
  }
  __syncthreads();
  if (trivial) return s.T;
  const bool aligned = ((reinterpret_cast<uintptr_t>(sc) | (uintptr_t)(sinks * 4)) & 15u) == 0;
  // every load of the row's scores first: they are in flight while the
  // histogram is read and its boundary found
  constexpr int R = kFusedMaxPages / (4 * NT);
  float vv[R][4];
#pragma unroll
  for (int rr = 0; rr < R; ++rr) {
    const int j0 = sinks + rr * 4 * NT + 4 * tid;
    if (aligned && j0 + 3 < n) {
      const float4 f = __ldg(reinterpret_cast<const float4*>(sc + j0));
      vv[rr][0] = f.x;
      vv[rr][1] = f.y;
      vv[rr][2] = f.z;
      vv[rr][3] = f.w;
    } else {
#pragma unroll
      for (int u = 0; u < 4; ++u) vv[rr][u] = j0 + u < n ? __ldg(sc + j0 + u) : 0.0f;
    }
  }
  const uint32_t anchor = order_key(sc[sinks]);
  for (int i = tid; i < kBins / 4; i += NT)
    reinterpret_cast<uint4*>(s.hist)[i] = __ldcg(reinterpret_cast<const uint4*>(hist_g) + i);
  __syncthreads();
  uint32_t above;
  const int bstar = find_boundary<NT>((uint32_t)k_eff, above, s);
  if (bstar < 0) {
    if (tid == 0) set_err(err, HX_DEV_ERR_SELECT);
    __syncthreads();
    return s.T;
  }
  const uint32_t r = (uint32_t)k_eff - above;
  const bool full_bin = s.hist[bstar] == r;
  const bool split2 = !full_bin && !edge_bin(bstar);
  __syncthreads();
  for (int i = tid; i < kBins; i += NT) s.hist[i] = 0;
  __syncthreads();
  // four consecutive pages a thread per round (one 16-byte load when the
  // row is aligned): a thread's pages share a slice unless a slice starts
  // inside them; a warp's 128 pages add to their slice with one shared add
  // per warp and slice
#pragma unroll
  for (int rr = 0; rr < R; ++rr) {
    const int base = sinks + rr * 4 * NT;
    if (base >= n) break;
    const int j0 = base + 4 * tid;
    const float* v = vv[rr];
    const int s_first = j0 < n ? slice_of(j0 - sinks) : -1;
    const int s_last = j0 + 3 < n ? slice_of(j0 + 3 - sinks) : (j0 < n ? slice_of(n - 1 - sinks) : -1);
    uint32_t cnt = 0;
    bool mixed = s_first != s_last;
    uint32_t cmask = 0;
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int j = j0 + u;
      const bool valid = j < n;
      const uint32_t k32 = order_key(v[u]);
      const int b1 = valid ? bin1(k32, anchor) : -1;
      const bool take = b1 > bstar || (full_bin && b1 == bstar);
      if (take) {
        if (mixed) atomicAdd(&s.add[slice_of(j - sinks)], 1u);
        else ++cnt;
      }
      if (b1 == bstar && !full_bin) cmask |= 1u << u;
    }
    // slice counts: the warp's threads in one slice reduce first
    const int w_first = __shfl_sync(0xffffffffu, s_first, 0);
    const bool uniform = __all_sync(0xffffffffu, !mixed && (s_first == w_first || s_first < 0));
    if (uniform) {
      const uint32_t tot = __reduce_add_sync(0xffffffffu, cnt);
      if ((tid & 31) == 0 && tot) atomicAdd(&s.add[w_first], tot);
    } else if (cnt) {
      atomicAdd(&s.add[s_first], cnt);
    }
    // candidates: one reservation for the warp
    const uint32_t nmine = (uint32_t)__popc(cmask);
    uint32_t incl = nmine;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const uint32_t x = __shfl_up_sync(0xffffffffu, incl, o);
      if ((tid & 31) >= o) incl += x;
    }
    const uint32_t wtot = __shfl_sync(0xffffffffu, incl, 31);
    if (wtot) {
      uint32_t base0 = 0;
      if ((tid & 31) == 31) base0 = atomicAdd(&s.nc, wtot);
      base0 = __shfl_sync(0xffffffffu, base0, 31);
      uint32_t at = base0 + incl - nmine;
#pragma unroll
      for (int u = 0; u < 4; ++u)
        if ((cmask >> u) & 1u) {
          const uint32_t k32 = order_key(v[u]);
          if (at < (uint32_t)kFusedMaxPages) s.cand[at] = ((uint64_t)k32 << 32) | (uint64_t)(~(uint32_t)(j0 + u));
          if (split2) atomicAdd(&s.hist[bin2(k32, anchor)], 1u);
          ++at;
        }
    }
  }
  __syncthreads();
  const uint32_t cnt = min(s.nc, (uint32_t)kFusedMaxPages);
  uint64_t T;
  if (full_bin) {
    T = bin_floor(bstar, -1, anchor);
  } else if (!split2) {
    T = radix_select<NT>(s.cand, cnt, r, s);
  } else {
    uint32_t above2;
    const int b2 = find_boundary<NT>(r, above2, s);
    if (b2 < 0) {
      T = bin_floor(bstar, -1, anchor);
      if (tid == 0) set_err(err, HX_DEV_ERR_SELECT);
    } else {
      const uint32_t r2 = r - above2;
      if (s.hist[b2] == r2) {
        T = bin_floor(bstar, b2, anchor);
      } else {
        uint64_t* hand = reinterpret_cast<uint64_t*>(s.hist);
        constexpr uint32_t kHand = kBins / 2;
        __syncthreads();
        if (tid == 0) s.nc = 0;
        __syncthreads();
        for (uint32_t i = tid; i < cnt; i += NT) {
          const uint64_t key = s.cand[i];
          if (bin2((uint32_t)(key >> 32), anchor) == b2) {
            const uint32_t at = atomicAdd(&s.nc, 1u);
            if (at < kHand) hand[at] = key;
          }
        }
        __syncthreads();
        const uint32_t nc = s.nc;
        if (nc <= (uint32_t)NT) {
          if (tid == 0) s.res[0] = -1;
          __syncthreads();
          if ((uint32_t)tid < nc) {
            const uint64_t mine = hand[tid];
            uint32_t beat = 0;
            for (uint32_t i = 0; i < nc; ++i) beat += hand[i] > mine;
            if (beat + 1 == r2) s.res[0] = tid;
          }
          __syncthreads();
          const int w = s.res[0];
          T = w >= 0 ? hand[w] : bin_floor(bstar, b2, anchor);
          if (w < 0 && tid == 0) set_err(err, HX_DEV_ERR_SELECT);
        } else if (nc <= kHand) {
          T = radix_select<NT>(hand, nc, r2, s);
        } else {
          T = radix_select<NT>(s.cand, cnt, r, s);
        }
      }
    }
  }
  __syncthreads();
  if (!full_bin)
    for (uint32_t i = tid; i < cnt; i += NT) {
      const uint64_t key = s.cand[i];
      if (key >= T) atomicAdd(&s.add[min(slice_of((int)(~(uint32_t)key) - sinks), C - 1)], 1u);
    }
  if (tid == 0) s.T = T;
  __syncthreads();
  return s.T;
}

}  // namespace fsel
}  // namespace hx
