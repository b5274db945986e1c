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

constexpr int kBins = 4096;  // histogram bins per level

// Histogram bins are taken relative to an anchor: the order key of the score
// of the (sequence, head)'s first page after its sinks. Level 1 bins are 2^16
// key units wide (1/128 of an octave of score) and centred on the anchor, so
// a row's scores spread over many bins whatever their magnitude; the two end
// bins take everything more than 16 octaves away. Level 2 splits a level-1
// bin into 4096 bins of 16 key units. Both are monotonic in the key.
HX_DEVINL int64_t bin_rel(uint32_t key, uint32_t anchor) {
  return (int64_t)key - (int64_t)anchor + ((int64_t)(kBins / 2) << 16);
}
HX_DEVINL int bin1(uint32_t key, uint32_t anchor) {
  const int64_t e = bin_rel(key, anchor);
  return e < 0 ? 0 : (int)min(e >> 16, (int64_t)(kBins - 1));
}
HX_DEVINL int bin2(uint32_t key, uint32_t anchor) { return (int)((bin_rel(key, anchor) >> 4) & (kBins - 1)); }
HX_DEVINL bool edge_bin(int b) { return b == 0 || b == kBins - 1; }
// Smallest 64-bit page key of level-1 bin b1 (level-2 bin b2 < 0: whole bin):
// a page is in bins >= there iff its key64 >= the returned value.
HX_DEVINL uint64_t bin_floor(int b1, int b2, uint32_t anchor) {
  if (b1 == 0 && b2 < 0) return 0ull;
  int64_t lo = (int64_t)anchor + ((int64_t)(b1 - kBins / 2) << 16) + (b2 > 0 ? 16ll * b2 : 0ll);
  lo = lo < 0 ? 0 : (lo > 0xFFFFFFFFll ? 0xFFFFFFFFll : lo);
  return (uint64_t)lo << 32;
}

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
                                                           float* __restrict__ scores) {
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
    if (lane == 0) scores[(int64_t)bh * max_pages + j] = acc;
  }
}

// Fast path for fp16 stats with D = 128 (4 channels per lane): a warp scores
// 32 consecutive pages at once. Lane partials follow the pinned order; the
// 32 per-page butterflies are done as one transposed butterfly (stage m adds
// the same lane pairs l, l ^ m as the per-page butterfly, so every page's sum
// is the same tree and bit-identical), after which lane l holds page base + l.
__global__ void __launch_bounds__(256) quest_scores_d128_kernel(const uint16_t* __restrict__ q, int H, int G,
                                                                int mode, const uint16_t* __restrict__ kmin,
                                                                const uint16_t* __restrict__ kmax,
                                                                int64_t page_stride, int64_t head_stride,
                                                                const int32_t* __restrict__ bt, int bt_stride,
                                                                const int32_t* __restrict__ seq_lens, int S,
                                                                int max_pages, int sinks_req,
                                                                float* __restrict__ scores) {
  __shared__ float s_qp[128], s_qn[128];
  const int bh = blockIdx.y;
  const int b = bh / H, h = bh % H;
  if (threadIdx.x < 128) {
    float qp, qn;
    group_terms(q, ((int64_t)b * H * G + (int64_t)h * G) * 128, G, 128, mode, threadIdx.x, qp, qn);
    s_qp[threadIdx.x] = qp;
    s_qn[threadIdx.x] = qn;
  }
  __syncthreads();
  const int n = min((seq_lens[b] + S - 1) / S, max_pages);
  const int lane = lane_id(), warp = threadIdx.x >> 5;
  const int base = blockIdx.x * 256 + warp * 32;
  if (base < n) {
    float qp[4], qn[4];
#pragma unroll
    for (int v = 0; v < 4; ++v) {
      qp[v] = s_qp[4 * lane + v];
      qn[v] = s_qn[4 * lane + v];
    }
    float part[32];
#pragma unroll
    for (int g8 = 0; g8 < 4; ++g8) {
      uint2 a[8], c[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int j = base + 8 * g8 + u;
        if (j < n) {
          const int64_t phys = bt ? (int64_t)bt[(int64_t)b * bt_stride + j] : (int64_t)j;
          const int64_t off = phys * page_stride + (int64_t)h * head_stride + 4 * lane;
          a[u] = __ldg(reinterpret_cast<const uint2*>(kmax + off));
          c[u] = __ldg(reinterpret_cast<const uint2*>(kmin + off));
        } else {
          a[u] = make_uint2(0u, 0u);
          c[u] = make_uint2(0u, 0u);
        }
      }
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const uint16_t xa[4] = {(uint16_t)(a[u].x & 0xffff), (uint16_t)(a[u].x >> 16),
                                (uint16_t)(a[u].y & 0xffff), (uint16_t)(a[u].y >> 16)};
        const uint16_t xc[4] = {(uint16_t)(c[u].x & 0xffff), (uint16_t)(c[u].x >> 16),
                                (uint16_t)(c[u].y & 0xffff), (uint16_t)(c[u].y >> 16)};
        float acc = 0.0f;
#pragma unroll
        for (int v = 0; v < 4; ++v) {
          acc = __fadd_rn(acc, __fmul_rn(qp[v], h2f(xa[v])));
          acc = __fadd_rn(acc, __fmul_rn(qn[v], h2f(xc[v])));
        }
        part[8 * g8 + u] = acc;
      }
    }
    // transposed butterfly: stage m adds the pair (l, l ^ m) exactly as the
    // per-page butterfly does; afterwards lane l holds page base + l
#pragma unroll
    for (int m = 16; m >= 1; m >>= 1) {
      const bool upper = (lane & m) != 0;
#pragma unroll
      for (int i = 0; i < m; ++i) {
        const float send = upper ? part[i] : part[i + m];
        const float keep = upper ? part[i + m] : part[i];
        part[i] = __fadd_rn(keep, __shfl_xor_sync(0xffffffffu, send, m));
      }
    }
    const int j = base + lane;
    if (j < n) scores[(int64_t)bh * max_pages + j] = part[0];
  }
}

// TMA-staged scores for fp16 stats with D = 128 whose min and max rows are
// adjacent (kmax == kmin + 128, the pool layout). Persistent, 16 warps per
// SM so the scoring arithmetic hides its latencies: each warp takes batches
// of 8 pages of one (b, h); a page's 512-byte {min, max} record lands in a
// 3-stage smem ring by bulk copy (one copy per run of adjacent records). The
// arithmetic is the pinned order of quest_scores_d128_kernel: lane l scores
// channels 4l .. 4l+3 of every page, then the pages are summed across lanes
// in the butterfly order (xor 16, 8, 4, 2, 1), the first three stages
// transposed so that lane l ends with page l / 4.
constexpr int kQW = 16;      // warps per block
constexpr int kQPB = 8;      // pages per batch
constexpr int kQStages = 3;  // batches in smem per warp (2 in flight while one is scored)
constexpr int kQHistRows = 2;  // (b, h) rows a block counts in smem
struct __align__(128) QuestSmem {
  uint16_t rec[kQW][kQStages][kQPB][256];  // [warp][stage][page][min 128 | max 128]
  uint32_t hist[kQHistRows][kBins];        // level-1 counts of the block's first two rows
  uint64_t bar[kQW][kQStages];
};

// Order key of page a's score (fp16 stats, D = 128, min row then max row),
// by the same arithmetic as the batched scoring; lane l holds channels
// 4l .. 4l+3 of the group terms.
HX_DEVINL uint32_t anchor_key_d128(const uint16_t* __restrict__ kmin, int64_t page_stride, int64_t head_stride,
                                   int64_t phys, int h, const float* qp, const float* qn, int lane) {
  const uint16_t* pm = kmin + phys * page_stride + (int64_t)h * head_stride;
  const uint2 c = *reinterpret_cast<const uint2*>(pm + 4 * lane);
  const uint2 x = *reinterpret_cast<const uint2*>(pm + 128 + 4 * lane);
  const uint16_t xa[4] = {(uint16_t)(x.x & 0xffff), (uint16_t)(x.x >> 16), (uint16_t)(x.y & 0xffff),
                          (uint16_t)(x.y >> 16)};
  const uint16_t xc[4] = {(uint16_t)(c.x & 0xffff), (uint16_t)(c.x >> 16), (uint16_t)(c.y & 0xffff),
                          (uint16_t)(c.y >> 16)};
  float acc = 0.0f;
#pragma unroll
  for (int v = 0; v < 4; ++v) {
    acc = __fadd_rn(acc, __fmul_rn(qp[v], h2f(xa[v])));
    acc = __fadd_rn(acc, __fmul_rn(qn[v], h2f(xc[v])));
  }
#pragma unroll
  for (int m = 16; m >= 1; m >>= 1) acc = __fadd_rn(acc, __shfl_xor_sync(0xffffffffu, acc, m));
  return order_key(acc);
}

// group_terms for channels 4 lane .. 4 lane + 3 (D = 128): one 8-byte load
// per query head, the same per-channel arithmetic.
HX_DEVINL void group_terms4(const uint16_t* __restrict__ q, int64_t qbase, int G, int mode, int lane, float* qp,
                            float* qn) {
  float s[4] = {0.0f, 0.0f, 0.0f, 0.0f}, t[4] = {0.0f, 0.0f, 0.0f, 0.0f};
  auto add = [&](uint2 w) {
    const float x[4] = {h2f((uint16_t)(w.x & 0xffff)), h2f((uint16_t)(w.x >> 16)), h2f((uint16_t)(w.y & 0xffff)),
                        h2f((uint16_t)(w.y >> 16))};
#pragma unroll
    for (int v = 0; v < 4; ++v) {
      if (mode == 0) {
        s[v] = __fadd_rn(s[v], x[v] > 0.0f ? x[v] : 0.0f);
        t[v] = __fadd_rn(t[v], x[v] < 0.0f ? x[v] : 0.0f);
      } else {
        s[v] = __fadd_rn(s[v], x[v]);
      }
    }
  };
  // the first kPre heads' rows are all loaded before the sums (one round trip),
  // then added in head order like any further ones
  constexpr int kPre = 8;
  uint2 wv[kPre];
#pragma unroll
  for (int g = 0; g < kPre; ++g)
    wv[g] = g < G ? *reinterpret_cast<const uint2*>(q + qbase + (int64_t)g * 128 + 4 * lane) : make_uint2(0u, 0u);
#pragma unroll
  for (int g = 0; g < kPre; ++g)
    if (g < G) add(wv[g]);
  for (int g = kPre; g < G; ++g) add(*reinterpret_cast<const uint2*>(q + qbase + (int64_t)g * 128 + 4 * lane));
#pragma unroll
  for (int v = 0; v < 4; ++v) {
    if (mode == 0) {
      qp[v] = s[v];
      qn[v] = t[v];
    } else {
      const float m = h2f(f2h(__fdiv_rn(s[v], (float)G)));
      qp[v] = m > 0.0f ? m : 0.0f;
      qn[v] = m < 0.0f ? m : 0.0f;
    }
  }
}

__global__ void __launch_bounds__(kQW * 32) quest_scores_tma_kernel(
    const uint16_t* __restrict__ q, int B, int H, int G, int mode, const uint16_t* __restrict__ kmin,
    int64_t page_stride, int64_t head_stride, const int32_t* __restrict__ bt, int bt_stride,
    const int32_t* __restrict__ seq_lens, int S, int max_pages, int sinks_req, float* __restrict__ scores,
    uint32_t* __restrict__ hist, uint32_t* err) {
  extern __shared__ __align__(128) uint8_t smem_raw[];
  QuestSmem& sm = *reinterpret_cast<QuestSmem*>(smem_raw);
  const int lane = lane_id(), warp = threadIdx.x >> 5;
  const int nb = (max_pages + kQPB - 1) / kQPB;  // batches per (b, h)
  const int64_t total = (int64_t)B * H * nb;
  const int64_t gw = (int64_t)blockIdx.x * kQW + warp, nw = (int64_t)gridDim.x * kQW;
  pdl_allow_next();
  if (lane == 0) {
    for (int st = 0; st < kQStages; ++st) mbar_init(&sm.bar[warp][st], 1);
    fence_mbar_init();
  }
  if (hist)
    for (int i = threadIdx.x; i < kQHistRows * kBins; i += blockDim.x) (&sm.hist[0][0])[i] = 0;
  __syncthreads();
  pdl_wait();  // inputs (q, stats, tables, the histogram) may come from the kernels before

  // A warp takes a contiguous run of batches (so it rarely changes (b, h)):
  // batch k of this warp is global batch g0 + k. For a batch: its pages count
  // (lanes < cnt hold a page), the sequence's sinks, lane's physical page.
  struct Bat {
    int bh, b, h, j0, cnt, sinks, n;
    int64_t phys;
  };
  // The planner walks the warp's batches in order, so (b, h) and the batch
  // index advance by counting, and a sequence's length is read once per (b, h):
  // no division and no dependent global load per batch.
  int pl_bh = -1, pl_b = 0, pl_h = 0, pl_jb = 0, pl_n = 0;
  auto plan_next = [&](bool first, int64_t it) -> Bat {
    if (first) {
      pl_bh = (int)(it / nb);
      pl_jb = (int)(it % nb);
      pl_b = pl_bh / H;
      pl_h = pl_bh % H;
    } else if (++pl_jb == nb) {
      pl_jb = 0;
      ++pl_bh;
      if (++pl_h == H) {
        pl_h = 0;
        ++pl_b;
      }
    }
    Bat r;
    r.bh = pl_bh;
    r.b = pl_b;
    r.h = pl_h;
    r.j0 = pl_jb * kQPB;
    const int b = pl_b;
    if (first || pl_jb == 0) pl_n = min((seq_lens[b] + S - 1) / S, max_pages);
    r.cnt = max(0, min(kQPB, pl_n - r.j0));
    r.sinks = min(max(sinks_req, 0), pl_n);
    r.n = pl_n;
    const int j = r.j0 + lane;
    r.phys = (lane < r.cnt) ? (bt ? (int64_t)bt[(int64_t)b * bt_stride + j] : (int64_t)j) : 0;
    return r;
  };
  // Pages whose records are adjacent in memory (consecutive physical pages,
  // records page_stride == 256 elements apart) go as one copy per run: the
  // copy engine's cost is per copy, not per byte.
  const bool adjacent = page_stride == 256;
  auto issue = [&](const Bat& bb, int st) {
    if (bb.cnt <= 0) return;
    if (lane == 0) {
      fence_proxy_async();
      mbar_arrive_expect_tx(&sm.bar[warp][st], (uint32_t)bb.cnt * 512u);
    }
    __syncwarp();
    const int64_t prev = __shfl_up_sync(0xffffffffu, bb.phys, 1);
    const bool start = lane < bb.cnt && (lane == 0 || !adjacent || bb.phys != prev + 1);
    const uint32_t starts = __ballot_sync(0xffffffffu, start);
    if (start) {
      const uint32_t later = starts & ~((2u << lane) - 1u);  // run starts after this lane
      const int end = later ? __ffs(later) - 1 : bb.cnt;
      bulk_g2s(sm.rec[warp][st][lane], kmin + bb.phys * page_stride + (int64_t)bb.h * head_stride,
               512u * (uint32_t)(end - lane), &sm.bar[warp][st]);
    }
  };

  const int64_t per = (total + nw - 1) / nw;
  const int64_t g0 = gw * per;
  // the block's batches are contiguous: its first rows are counted in smem
  const int bh0 = (int)min((int64_t)blockIdx.x * kQW * per, total) / nb;
  const int nk = (int)max((int64_t)0, min(per, total - g0));
  Bat p0 = {0, 0, 0, 0, 0, 0, 0, 0}, p1 = {0, 0, 0, 0, 0, 0, 0, 0}, p2 = {0, 0, 0, 0, 0, 0, 0, 0};
  if (nk > 0) p0 = plan_next(true, g0);
  if (nk > 1) p1 = plan_next(false, 0);
  if (nk > 2) p2 = plan_next(false, 0);
  issue(p0, 0);
  issue(p1, 1 % kQStages);
  int cur_bh = -1;
  uint32_t phase = 0, anchor = 0;
  bool dead = false;
  float qp[4], qn[4];
  for (int k = 0; k < nk; ++k) {
    const int st = k % kQStages;
    // keep two batches in flight: issue k + 2 now, plan k + 3 (its block-table
    // reads overlap this batch's work)
    if (k + 2 < nk) issue(p2, (k + 2) % kQStages);
    Bat p3 = {0, 0, 0, 0, 0, 0, 0, 0};
    if (k + 3 < nk) p3 = plan_next(false, 0);
    const Bat cb = p0;
    if (cb.cnt > 0) {
      if (cb.bh != cur_bh) {
        const int b = cb.b, h = cb.h;
        // the row's anchor (page `sinks`, when there is one): its block-table
        // entry is loaded together with the query rows, its stats after
        const bool has_anchor = hist && cb.sinks < cb.n;
        const int64_t aphys =
            has_anchor ? (bt ? (int64_t)bt[(int64_t)b * bt_stride + cb.sinks] : (int64_t)cb.sinks) : 0;
        group_terms4(q, ((int64_t)b * H * G + (int64_t)h * G) * 128, G, mode, lane, qp, qn);
        anchor = has_anchor ? anchor_key_d128(kmin, page_stride, head_stride, aphys, h, qp, qn, lane) : 0u;
        cur_bh = cb.bh;
      }
      if (!dead && !mbar_wait(&sm.bar[warp][st], (phase >> st) & 1u)) {
        dead = true;
        if (lane == 0) set_err(err, HX_DEV_ERR_TIMEOUT);
      }
      phase ^= 1u << st;
      float part[kQPB];
#pragma unroll
      for (int u = 0; u < kQPB; ++u) {
        const uint2 c = *reinterpret_cast<const uint2*>(&sm.rec[warp][st][u][4 * lane]);
        const uint2 a = *reinterpret_cast<const uint2*>(&sm.rec[warp][st][u][128 + 4 * lane]);
        const uint16_t xa[4] = {(uint16_t)(a.x & 0xffff), (uint16_t)(a.x >> 16), (uint16_t)(a.y & 0xffff),
                                (uint16_t)(a.y >> 16)};
        const uint16_t xc[4] = {(uint16_t)(c.x & 0xffff), (uint16_t)(c.x >> 16), (uint16_t)(c.y & 0xffff),
                                (uint16_t)(c.y >> 16)};
        float acc = 0.0f;
#pragma unroll
        for (int v = 0; v < 4; ++v) {
          acc = __fadd_rn(acc, __fmul_rn(qp[v], h2f(xa[v])));
          acc = __fadd_rn(acc, __fmul_rn(qn[v], h2f(xc[v])));
        }
        part[u] = acc;
      }
      // stages 16, 8, 4 transposed (8 -> 1 values a lane), then 2, 1 plain
#pragma unroll
      for (int m = 16, half = kQPB / 2; m >= 4; m >>= 1, half >>= 1) {
        const bool upper = (lane & m) != 0;
#pragma unroll
        for (int i = 0; i < half; ++i) {
          const float send = upper ? part[i] : part[i + half];
          const float keep = upper ? part[i + half] : part[i];
          part[i] = __fadd_rn(keep, __shfl_xor_sync(0xffffffffu, send, m));
        }
      }
      part[0] = __fadd_rn(part[0], __shfl_xor_sync(0xffffffffu, part[0], 2));
      part[0] = __fadd_rn(part[0], __shfl_xor_sync(0xffffffffu, part[0], 1));
      const int u = lane >> 2, j = cb.j0 + u;
      const bool own = (lane & 3) == 0 && u < cb.cnt;
      if (own) scores[(int64_t)cb.bh * max_pages + j] = part[0];
      if (hist) {
        // pages of the batch that share a bin go as one atomic; the block's
        // first rows count in smem (flushed once at the end), any later row
        // in global memory
        const bool counted = own && j >= cb.sinks;
        const uint32_t bin = (uint32_t)bin1(order_key(part[0]), anchor);
        const uint32_t act = __ballot_sync(0xffffffffu, counted);
        if (counted) {
          const uint32_t peers = __match_any_sync(act, bin);
          const int row = cb.bh - bh0;
          if (lane == __ffs(peers) - 1) {
            if (row < kQHistRows) atomicAdd(&sm.hist[row][bin], (uint32_t)__popc(peers));
            else atomicAdd(&hist[(int64_t)cb.bh * 2 * kBins + bin], (uint32_t)__popc(peers));
          }
        }
      }
    }
    __syncwarp();
    p0 = p1;
    p1 = p2;
    p2 = p3;
  }
  if (hist) {  // flush the smem counts: one atomic per nonzero bin
    __syncthreads();
    for (int i = threadIdx.x; i < kQHistRows * kBins; i += blockDim.x) {
      const int row = i / kBins, bh = bh0 + row;
      const uint32_t c = (&sm.hist[0][0])[i];
      if (c && bh < B * H) atomicAdd(&hist[(int64_t)bh * 2 * kBins + (i % kBins)], c);
    }
  }
}

// Level-1 histogram of given scores (scores from outside, or from the scoring
// kernels that do not count as they go).
__global__ void quest_hist_kernel(const float* scores, int H, const int32_t* seq_lens, int S, int max_pages,
                                  int sinks_req, uint32_t* hist) {
  const int bh = blockIdx.y;
  const int b = bh / H;
  const int n = min((seq_lens[b] + S - 1) / S, max_pages);
  const int sinks = min(max(sinks_req, 0), n);
  if (sinks >= n) return;
  const uint32_t anchor = order_key(scores[(int64_t)bh * max_pages + sinks]);
  for (int j = sinks + blockIdx.x * blockDim.x + threadIdx.x; j < n; j += gridDim.x * blockDim.x)
    atomicAdd(&hist[(int64_t)bh * 2 * kBins + bin1(order_key(scores[(int64_t)bh * max_pages + j]), anchor)], 1u);
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

// Block-wide (256 threads) locate: thread t owns count c_t; with suffix sums
// S_t = sum_{u >= t} c_u, find the t with S_{t+1} < need <= S_t. Returns t
// (or -1 if the total is below need) and S_{t+1} in `above`.
HX_DEVINL int suffix_locate(uint32_t c, uint32_t need, uint32_t& above, uint32_t* s_warp, int* s_res) {
  const int t = threadIdx.x, lane = t & 31, w = t >> 5;
  uint32_t v = c;  // inclusive suffix sum within the warp (lanes >= this lane)
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    uint32_t x = __shfl_down_sync(0xffffffffu, v, o);
    if (lane + o < 32) v += x;
  }
  if (lane == 0) s_warp[w] = v;  // warp total
  if (t == 0) s_res[0] = -1;
  __syncthreads();
  uint32_t later = 0;  // totals of the warps above this one
  for (int u = w + 1; u < 8; ++u) later += s_warp[u];
  const uint32_t incl = v + later, excl = incl - c;
  if (excl < need && incl >= need) {
    s_res[0] = t;
    s_res[1] = (int)excl;
  }
  __syncthreads();
  const int r = s_res[0];
  above = r >= 0 ? (uint32_t)s_res[1] : 0u;
  __syncthreads();
  return r;
}

// Highest histogram bin whose suffix count reaches `need` (4096 bins).
HX_DEVINL int find_boundary(const uint32_t* s_hist, uint32_t need, uint32_t& above, uint32_t* s_warp,
                            int* s_res) {
  const int t = threadIdx.x;
  uint32_t local = 0;
#pragma unroll
  for (int i = 0; i < 16; ++i) local += s_hist[16 * t + i];
  uint32_t above_t;
  const int owner = suffix_locate(local, need, above_t, s_warp, s_res);
  if (owner < 0) return -1;
  // the owner's 16 bins, scanned from the top by that thread
  if (t == owner) {
    uint32_t acc = above_t;
    int found = 16 * t;
    for (int bin = 16 * t + 15; bin >= 16 * t; --bin) {
      if (acc + s_hist[bin] >= need) {
        found = bin;
        break;
      }
      acc += s_hist[bin];
    }
    s_res[2] = found;
    s_res[3] = (int)acc;
  }
  __syncthreads();
  above = (uint32_t)s_res[3];
  const int r = s_res[2];
  __syncthreads();
  return r;
}

// Select the r-th largest among `cnt` unique 64-bit keys, counting only keys
// whose bits above `shift` equal `prefix`, by 8-bit digit passes from bit
// shift-1 down. Returns the threshold T with
// exactly r keys >= T (among the candidates). blockDim == 256. kGlobal: the
// keys are in global memory written by other blocks (read through L2).
template <bool kGlobal>
HX_DEVINL uint64_t radix_select(const uint64_t* cand, uint32_t cnt, uint32_t r, uint64_t prefix, int shift,
                                uint32_t* s_h, uint32_t* s_warp, int* s_res) {
  uint64_t mask = shift >= 64 ? 0ull : ~((1ull << shift) - 1ull);
  while (shift > 0) {
    const int width = shift >= 8 ? 8 : shift;
    shift -= width;
    const uint32_t nb = 1u << width;
    s_h[threadIdx.x] = 0;
    __syncthreads();
    for (uint32_t i0 = 0; i0 < cnt; i0 += 4 * blockDim.x) {
      uint64_t key[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {  // written by other blocks: read through L2
        const uint32_t i = i0 + u * blockDim.x + threadIdx.x;
        key[u] = i < cnt ? (kGlobal ? __ldcg(cand + i) : cand[i]) : ~prefix;
      }
#pragma unroll
      for (int u = 0; u < 4; ++u)
        if (i0 + u * blockDim.x + threadIdx.x < cnt && (key[u] & mask) == prefix)
          atomicAdd(&s_h[(key[u] >> shift) & (nb - 1)], 1u);
    }
    __syncthreads();
    uint32_t above;
    const int dsel = suffix_locate(threadIdx.x < nb ? s_h[threadIdx.x] : 0u, r, above, s_warp, s_res);
    const uint32_t in_bin = dsel >= 0 ? s_h[dsel] : 0u;
    __syncthreads();
    if (dsel < 0) return prefix;  // inconsistent counts; the caller flags it
    r -= above;
    prefix |= (uint64_t)dsel << shift;
    mask |= (uint64_t)(nb - 1) << shift;
    if (in_bin == r) return prefix;  // every key with this prefix is selected
  }
  return prefix;
}

// Copy a 4096-bin histogram to smem with all of a thread's loads in flight
// (blockDim == 256: four 16-byte loads each), through L2: other blocks wrote it.
HX_DEVINL void load_hist(uint32_t* s_hist, const uint32_t* g) {
  uint4 v[4];
#pragma unroll
  for (int u = 0; u < 4; ++u) v[u] = __ldcg(reinterpret_cast<const uint4*>(g) + u * 256 + threadIdx.x);
#pragma unroll
  for (int u = 0; u < 4; ++u) reinterpret_cast<uint4*>(s_hist)[u * 256 + threadIdx.x] = v[u];
}

// hist layout per (b, h): [level 1: 4096 anchored bins (bin1) of the non-sink
// pages | level 2: 4096 bins (bin2) of the level-1 boundary bin's pages]. Every
// block finds the level-1 boundary bin b*, then counts its slice's pages in
// b* into level 2 and hands them to the last block as candidates; the last
// block finds the level-2 boundary bin and ranks its keys (a handful). The
// clamped end bins are not split by level 2: a boundary there is settled by
// an exact radix select over all of the bin's keys.
//
// With slice_off != NULL the non-sink pages [sinks, n) of a row are also cut
// into C = gridDim.x slices of ceil((n - sinks) / C) pages (block s = slice
// s) and slice_off (B*H, C + 1) receives the exclusive prefix of each slice's
// selected count: every block counts its slice's pages above the boundary bin
// (and, when the boundary bin is taken whole, in it), and the last block adds
// the boundary candidates that pass the threshold.
constexpr int kCandSmem = 1024;
constexpr int kMaxSlices = 128;
// threshold blocks (= slices) per row: one per 1024 pages, 1 .. kMaxSlices
inline int quest_slices(int max_pages) {
  const int c = (max_pages + 1023) / 1024;
  return c < 1 ? 1 : (c > kMaxSlices ? kMaxSlices : c);
}
__global__ void __launch_bounds__(256) quest_threshold_kernel(const float* __restrict__ scores, int H,
                                                              const int32_t* __restrict__ seq_lens, int S,
                                                              int max_pages, int sinks_req, int k_fixed, int fnum,
                                                              int fden, uint32_t* hist, uint64_t* cand,
                                                              uint32_t* counters, uint64_t* thresh,
                                                              int32_t* slice_off, uint32_t* err) {
  __shared__ __align__(16) uint32_t s_hist[kBins];
  __shared__ uint32_t s_warp[8];
  __shared__ int s_res[4];
  __shared__ uint32_t s_h2[256];
  __shared__ uint64_t s_cand[kCandSmem];
  __shared__ uint32_t s_nc, s_above;
  __shared__ int s_last;
  pdl_allow_next();
  pdl_wait();  // the scores and the histogram come from the scoring kernel
  const int bh = blockIdx.y;
  const int b = bh / H;
  const int C = gridDim.x;
  const SelPlan pl = plan_for(seq_lens[b], S, max_pages, sinks_req, k_fixed, fnum, fden);
  uint32_t* hist_bh = hist + (int64_t)bh * 2 * kBins;
  uint32_t* hist2_bh = hist_bh + kBins;
  uint32_t* ctr = counters + 2 * (int64_t)bh;
  uint64_t* cand_bh = cand + (int64_t)bh * max_pages;
  const int n_ns = pl.n - pl.sinks;

  int bstar = -1;
  uint32_t above = 0, r = 0, anchor = 0;
  bool full_bin = false;
  const bool trivial = (pl.k_eff == 0) || (pl.k_eff >= n_ns);
  if (!trivial) {
    anchor = order_key(scores[(int64_t)bh * max_pages + pl.sinks]);
    load_hist(s_hist, hist_bh);
    __syncthreads();
    bstar = find_boundary(s_hist, (uint32_t)pl.k_eff, above, s_warp, s_res);
    r = (uint32_t)pl.k_eff - above;
    full_bin = bstar >= 0 && s_hist[bstar] == r;
    if (bstar >= 0 && (!full_bin || slice_off)) {
      // this block's candidates of bin b*, with their level-2 histogram:
      // staged in smem, then one global reservation for the block (with
      // slices: also the count of its pages above b*, or at / above it when
      // b* is taken whole, in which case nothing else is gathered)
      const bool split2 = !edge_bin(bstar);
      const int per = (n_ns + C - 1) / C;
      const int a = pl.sinks + blockIdx.x * per;
      const int e = min(a + per, pl.n);
      uint32_t my_above = 0;
      if (threadIdx.x == 0) {
        s_nc = 0;
        s_above = 0;
      }
      __syncthreads();
      for (int base = a; base < e; base += 4 * blockDim.x) {
        float v[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {  // loads first, so they are in flight together
          const int j = base + u * blockDim.x + threadIdx.x;
          v[u] = j < e ? scores[(int64_t)bh * max_pages + j] : 0.0f;
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int j = base + u * blockDim.x + threadIdx.x;
          if (j < e) {
            const uint32_t k32 = order_key(v[u]);
            const int b1 = bin1(k32, anchor);
            my_above += (b1 > bstar || (full_bin && b1 == bstar)) ? 1u : 0u;
            if (b1 == bstar && !full_bin) {
              const uint64_t key = ((uint64_t)k32 << 32) | (uint64_t)(~(uint32_t)j);
              const uint32_t at = atomicAdd(&s_nc, 1u);
              if (at < (uint32_t)kCandSmem) s_cand[at] = key;
              else cand_bh[atomicAdd(&ctr[0], 1u)] = key;  // a slice past kCandSmem hits (long sequences)
              if (split2) atomicAdd(&hist2_bh[bin2(k32, anchor)], 1u);
            }
          }
        }
      }
      if (slice_off) {
#pragma unroll
        for (int o = 16; o; o >>= 1) my_above += __shfl_xor_sync(0xffffffffu, my_above, o);
        if ((threadIdx.x & 31) == 0 && my_above) atomicAdd(&s_above, my_above);
      }
      __syncthreads();
      if (slice_off && threadIdx.x == 0) slice_off[(int64_t)bh * (C + 1) + blockIdx.x] = (int32_t)s_above;
      const uint32_t nloc = min(s_nc, (uint32_t)kCandSmem);
      if (nloc) {
        if (threadIdx.x == 0) s_res[0] = (int)atomicAdd(&ctr[0], nloc);
        __syncthreads();
        const uint32_t gbase = (uint32_t)s_res[0];
        for (uint32_t i = threadIdx.x; i < nloc; i += blockDim.x) cand_bh[gbase + i] = s_cand[i];
      }
      __syncthreads();
    }
  }
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) s_last = (atomicAdd(&ctr[1], 1u) == (uint32_t)(C - 1));
  __syncthreads();
  if (!s_last) return;
  __threadfence();

  // One round of loads feeds the whole finish: the candidate count, the
  // candidates themselves (up to kCandSmem; reading past the count is harmless),
  // the level-2 histogram and the slices' partial counts.
  const bool gather = !trivial && bstar >= 0 && !full_bin;
  const uint32_t ncap = (uint32_t)min(kCandSmem, max(max_pages, 1));
  uint32_t cnt = 0;
  int32_t part = 0;
  if (slice_off && threadIdx.x < C && !trivial && bstar >= 0)
    part = __ldcg(slice_off + (int64_t)bh * (C + 1) + threadIdx.x);
  if (gather) {
    cnt = *((volatile uint32_t*)&ctr[0]);
    uint64_t kk[kCandSmem / 256];
#pragma unroll
    for (int u = 0; u < kCandSmem / 256; ++u) {
      const uint32_t i = threadIdx.x + 256u * u;
      kk[u] = i < ncap ? __ldcg(cand_bh + i) : 0ull;
    }
    if (!edge_bin(bstar)) load_hist(s_hist, hist2_bh);
#pragma unroll
    for (int u = 0; u < kCandSmem / 256; ++u) {
      const uint32_t i = threadIdx.x + 256u * u;
      if (i < ncap) s_cand[i] = kk[u];
    }
    __syncthreads();
  }
  const bool in_smem = cnt <= ncap;  // every candidate is in s_cand

  uint64_t T;
  if (pl.k_eff == 0) {
    T = ~0ull;
  } else if (pl.k_eff >= n_ns) {
    T = 0ull;
  } else if (bstar < 0) {
    T = 0ull;
    if (threadIdx.x == 0) set_err(err, HX_DEV_ERR_SELECT);
  } else if (full_bin) {
    T = bin_floor(bstar, -1, anchor);
  } else if (edge_bin(bstar)) {
    T = in_smem ? radix_select<false>(s_cand, cnt, r, 0ull, 64, s_h2, s_warp, s_res)
                : radix_select<true>(cand_bh, cnt, r, 0ull, 64, s_h2, s_warp, s_res);
  } else {
    uint32_t above2;
    const int b2 = find_boundary(s_hist, r, above2, s_warp, s_res);
    if (b2 < 0) {
      T = bin_floor(bstar, -1, anchor);
      if (threadIdx.x == 0) set_err(err, HX_DEV_ERR_SELECT);
    } else {
      const uint32_t r2 = r - above2;
      const uint32_t in_b2 = s_hist[b2];
      if (in_b2 == r2) {
        T = bin_floor(bstar, b2, anchor);
      } else {
        // gather the level-2 boundary bin's keys (the histogram's smem is free
        // now) and rank them
        uint64_t* hand = reinterpret_cast<uint64_t*>(s_hist);
        constexpr uint32_t kHand = kBins / 2;
        __syncthreads();
        if (threadIdx.x == 0) s_nc = 0;
        __syncthreads();
        for (uint32_t i = threadIdx.x; i < cnt; i += blockDim.x) {
          const uint64_t key = in_smem ? s_cand[i] : __ldcg(cand_bh + i);
          if (bin2((uint32_t)(key >> 32), anchor) == b2) {
            const uint32_t at = atomicAdd(&s_nc, 1u);
            if (at < kHand) hand[at] = key;
          }
        }
        __syncthreads();
        const uint32_t nc = s_nc;
        if (nc <= blockDim.x) {
          // a handful of keys: key i is T when exactly r2 - 1 keys beat it
          if (threadIdx.x == 0) s_res[0] = -1;
          __syncthreads();
          if (threadIdx.x < nc) {
            const uint64_t mine = hand[threadIdx.x];
            uint32_t beat = 0;
            for (uint32_t i = 0; i < nc; ++i) beat += hand[i] > mine;
            if (beat + 1 == r2) s_res[0] = (int)threadIdx.x;
          }
          __syncthreads();
          const int w = s_res[0];
          T = w >= 0 ? hand[w] : bin_floor(bstar, b2, anchor);
          if (w < 0 && threadIdx.x == 0) set_err(err, HX_DEV_ERR_SELECT);
        } else if (nc <= kHand) {
          T = radix_select<false>(hand, nc, r2, 0ull, 64, s_h2, s_warp, s_res);
        } else {
          // more keys within 16 units of key than fit: rank the whole bin
          T = in_smem ? radix_select<false>(s_cand, cnt, r, 0ull, 64, s_h2, s_warp, s_res)
                      : radix_select<true>(cand_bh, cnt, r, 0ull, 64, s_h2, s_warp, s_res);
        }
      }
    }
  }
  if (slice_off) {
    // final selected count of every slice, then the exclusive prefix (one warp)
    uint32_t* s_add = s_h2;  // C <= kMaxSlices <= 256 counters
    const int per = n_ns > 0 ? (n_ns + C - 1) / C : 1;
    __syncthreads();
    for (int i = threadIdx.x; i < C; i += blockDim.x) {
      uint32_t v;
      if (pl.k_eff == 0) v = 0;
      else if (pl.k_eff >= n_ns) v = (uint32_t)max(0, min(per, n_ns - i * per));  // every page
      else if (bstar < 0) v = 0;
      else v = (uint32_t)part;
      s_add[i] = v;
    }
    __syncthreads();
    if (gather) {
      for (uint32_t i = threadIdx.x; i < cnt; i += blockDim.x) {
        const uint64_t key = in_smem ? s_cand[i] : __ldcg(cand_bh + i);
        if (key >= T) {
          const int j = (int)(~(uint32_t)key);
          atomicAdd(&s_add[min((j - pl.sinks) / per, C - 1)], 1u);
        }
      }
      __syncthreads();
    }
    if (threadIdx.x < 32) {
      const int lane = threadIdx.x;
      uint32_t v[kMaxSlices / 32];
      uint32_t sum = 0;
#pragma unroll
      for (int q = 0; q < kMaxSlices / 32; ++q) {
        const int i = (kMaxSlices / 32) * lane + q;
        v[q] = i < C ? s_add[i] : 0u;
        sum += v[q];
      }
      uint32_t incl = sum;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const uint32_t x = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += x;
      }
      uint32_t acc = incl - sum;
#pragma unroll
      for (int q = 0; q < kMaxSlices / 32; ++q) {
        const int i = (kMaxSlices / 32) * lane + q;
        if (i < C) slice_off[(int64_t)bh * (C + 1) + i] = (int32_t)acc;
        acc += v[q];
      }
      if (lane == 31) slice_off[(int64_t)bh * (C + 1) + C] = (int32_t)incl;
    }
  }
  if (threadIdx.x == 0) {
    thresh[bh] = T;
    ctr[0] = 0;
    ctr[1] = 0;
  }
  for (int i = threadIdx.x; i < 2 * kBins; i += blockDim.x) hist_bh[i] = 0;
}

// ---------------------------------------------------------------------------
// exact threshold, one CTA per (b, h): for short rows (batched sequences)
// one block reads the whole row, so the boundary bin's candidates, the
// level-2 counts and the slice counts stay in shared memory and nothing waits
// on other blocks (no candidate reservation, fence or last-block counter).
// Same thresholds and slice counts as quest_threshold_kernel. Measured on
// B200 (with the histogram kernel): 8.7 us against 9.9 us for the sliced
// kernel at 2048 pages, but 16.6 against 11.7 us at 8192 pages, where one
// block's serial rounds over the row outweigh the saved round trips.

constexpr int kRowCand = 2048;      // boundary-bin candidates kept in smem
constexpr int kRowMaxPages = 2048;  // longer rows take the sliced kernel

// Count the warp's taken pages into their slices. Lanes hold consecutive
// pages (slice s >= 0; s < 0 and take false past the row's end), so when
// lanes 0 and 31 share a slice every lane does: one add for the warp.
// Otherwise (a slice edge or the row's tail) each taken lane adds its own.
HX_DEVINL void slice_add(uint32_t* s_add, int s, bool take) {
  const uint32_t taken = __ballot_sync(0xffffffffu, take);
  const int s0 = __shfl_sync(0xffffffffu, s, 0), s31 = __shfl_sync(0xffffffffu, s, 31);
  if (s0 == s31) {
    if (taken && lane_id() == 0) atomicAdd(&s_add[s0], (uint32_t)__popc(taken));
  } else if (take) {
    atomicAdd(&s_add[s], 1u);
  }
}

__global__ void __launch_bounds__(256) quest_threshold_row_kernel(
    const float* __restrict__ scores, int H, const int32_t* __restrict__ seq_lens, int S, int max_pages,
    int sinks_req, int k_fixed, int fnum, int fden, int C, uint32_t* hist, uint64_t* cand, uint64_t* thresh,
    int32_t* slice_off, uint32_t* err) {
  __shared__ __align__(16) uint32_t s_hist[kBins];  // level 1, then level 2, then the level-2 bin's keys
  __shared__ uint64_t s_cand[kRowCand];
  __shared__ uint32_t s_warp[8];
  __shared__ int s_res[4];
  __shared__ uint32_t s_h2[256];
  __shared__ uint32_t s_add[kMaxSlices];
  __shared__ uint32_t s_nc;
  pdl_allow_next();
  pdl_wait();  // the scores and the level-1 histogram come from the scoring kernel
  const int tid = threadIdx.x;
  const int bh = blockIdx.x;
  const SelPlan pl = plan_for(seq_lens[bh / H], S, max_pages, sinks_req, k_fixed, fnum, fden);
  uint32_t* hist_bh = hist + (int64_t)bh * 2 * kBins;
  uint64_t* cand_bh = cand + (int64_t)bh * max_pages;
  const float* sc = scores + (int64_t)bh * max_pages;
  const int n_ns = pl.n - pl.sinks;
  const int per = n_ns > 0 ? (n_ns + C - 1) / C : 1;
  const bool trivial = pl.k_eff == 0 || pl.k_eff >= n_ns;
  for (int i = tid; i < C; i += blockDim.x)
    s_add[i] = (trivial && pl.k_eff > 0) ? (uint32_t)max(0, min(per, n_ns - i * per)) : 0u;
  if (tid == 0) s_nc = 0;

  uint64_t T = pl.k_eff == 0 ? ~0ull : 0ull;
  if (!trivial) {
    const uint32_t anchor = order_key(sc[pl.sinks]);
    load_hist(s_hist, hist_bh);
    __syncthreads();
    uint32_t above;
    const int bstar = find_boundary(s_hist, (uint32_t)pl.k_eff, above, s_warp, s_res);
    if (bstar < 0) {
      if (tid == 0) set_err(err, HX_DEV_ERR_SELECT);
    } else {
      const uint32_t r = (uint32_t)pl.k_eff - above;
      const bool full_bin = s_hist[bstar] == r;
      const bool split2 = !full_bin && !edge_bin(bstar);
      __syncthreads();  // level 1 read: its smem becomes the level-2 counts
      for (int i = tid; i < kBins; i += blockDim.x) s_hist[i] = 0;
      __syncthreads();
      // the row: pages above the boundary bin go to their slice's count;
      // the bin's pages become candidates (every one in global memory, the
      // first kRowCand also in smem) with their level-2 counts
      constexpr int kRowU = 8;  // loads in flight per thread
      for (int base = pl.sinks; base < pl.n; base += kRowU * (int)blockDim.x) {
        float v[kRowU];
#pragma unroll
        for (int u = 0; u < kRowU; ++u) {  // loads first, so they are in flight together
          const int j = base + u * (int)blockDim.x + tid;
          v[u] = j < pl.n ? __ldg(sc + j) : 0.0f;
        }
#pragma unroll
        for (int u = 0; u < kRowU; ++u) {
          const int j = base + u * (int)blockDim.x + tid;
          const bool valid = j < pl.n;
          const uint32_t k32 = order_key(v[u]);
          const int b1 = valid ? bin1(k32, anchor) : -1;
          slice_add(s_add, valid ? (j - pl.sinks) / per : -1, b1 > bstar || (full_bin && b1 == bstar));
          if (b1 == bstar && !full_bin) {
            const uint64_t key = ((uint64_t)k32 << 32) | (uint64_t)(~(uint32_t)j);
            const uint32_t at = atomicAdd(&s_nc, 1u);
            cand_bh[at] = key;
            if (at < (uint32_t)kRowCand) s_cand[at] = key;
            if (split2) atomicAdd(&s_hist[bin2(k32, anchor)], 1u);
          }
        }
      }
      __syncthreads();
      const uint32_t cnt = s_nc;
      const bool in_smem = cnt <= (uint32_t)kRowCand;
      if (full_bin) {
        T = bin_floor(bstar, -1, anchor);
      } else if (!split2) {
        T = in_smem ? radix_select<false>(s_cand, cnt, r, 0ull, 64, s_h2, s_warp, s_res)
                    : radix_select<true>(cand_bh, cnt, r, 0ull, 64, s_h2, s_warp, s_res);
      } else {
        uint32_t above2;
        const int b2 = find_boundary(s_hist, r, above2, s_warp, s_res);
        if (b2 < 0) {
          T = bin_floor(bstar, -1, anchor);
          if (tid == 0) set_err(err, HX_DEV_ERR_SELECT);
        } else {
          const uint32_t r2 = r - above2;
          if (s_hist[b2] == r2) {
            T = bin_floor(bstar, b2, anchor);
          } else {
            // the level-2 bin's keys (the counts' smem is free now), ranked
            uint64_t* hand = reinterpret_cast<uint64_t*>(s_hist);
            constexpr uint32_t kHand = kBins / 2;
            __syncthreads();
            if (tid == 0) s_nc = 0;
            __syncthreads();
            for (uint32_t i = tid; i < cnt; i += blockDim.x) {
              const uint64_t key = in_smem ? s_cand[i] : __ldcg(cand_bh + i);
              if (bin2((uint32_t)(key >> 32), anchor) == b2) {
                const uint32_t at = atomicAdd(&s_nc, 1u);
                if (at < kHand) hand[at] = key;
              }
            }
            __syncthreads();
            const uint32_t nc = s_nc;
            if (nc <= blockDim.x) {
              // a handful of keys: key i is T when exactly r2 - 1 keys beat it
              if (tid == 0) s_res[0] = -1;
              __syncthreads();
              if ((uint32_t)tid < nc) {
                const uint64_t mine = hand[tid];
                uint32_t beat = 0;
                for (uint32_t i = 0; i < nc; ++i) beat += hand[i] > mine;
                if (beat + 1 == r2) s_res[0] = tid;
              }
              __syncthreads();
              const int w = s_res[0];
              T = w >= 0 ? hand[w] : bin_floor(bstar, b2, anchor);
              if (w < 0 && tid == 0) set_err(err, HX_DEV_ERR_SELECT);
            } else if (nc <= kHand) {
              T = radix_select<false>(hand, nc, r2, 0ull, 64, s_h2, s_warp, s_res);
            } else {
              T = in_smem ? radix_select<false>(s_cand, cnt, r, 0ull, 64, s_h2, s_warp, s_res)
                          : radix_select<true>(cand_bh, cnt, r, 0ull, 64, s_h2, s_warp, s_res);
            }
          }
        }
      }
      // the candidates that pass join their slices' counts
      __syncthreads();
      if (slice_off && !full_bin) {
        for (uint32_t i = tid; i < cnt; i += blockDim.x) {
          const uint64_t key = in_smem ? s_cand[i] : __ldcg(cand_bh + i);
          if (key >= T) atomicAdd(&s_add[min(((int)(~(uint32_t)key) - pl.sinks) / per, C - 1)], 1u);
        }
      }
    }
  }
  __syncthreads();
  if (slice_off && tid < 32) {  // exclusive prefix of the slice counts (one warp)
    const int lane = tid;
    uint32_t v[kMaxSlices / 32];
    uint32_t sum = 0;
#pragma unroll
    for (int q = 0; q < kMaxSlices / 32; ++q) {
      const int i = (kMaxSlices / 32) * lane + q;
      v[q] = i < C ? s_add[i] : 0u;
      sum += v[q];
    }
    uint32_t incl = sum;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const uint32_t x = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += x;
    }
    uint32_t acc = incl - sum;
#pragma unroll
    for (int q = 0; q < kMaxSlices / 32; ++q) {
      const int i = (kMaxSlices / 32) * lane + q;
      if (i < C) slice_off[(int64_t)bh * (C + 1) + i] = (int32_t)acc;
      acc += v[q];
    }
    if (lane == 31) slice_off[(int64_t)bh * (C + 1) + C] = (int32_t)incl;
  }
  if (tid == 0) thresh[bh] = T;
  // leave the level-1 counts zero for the next scoring (the scoring kernel
  // counts every row, trivial or not; level 2 lives in smem here)
  for (int i = tid; i < kBins; i += blockDim.x) hist_bh[i] = 0;
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

// Chunked list compaction for the decode: many CTAs per (b, h). Pass 1 counts
// the selected pages of each chunk of kListChunk pages; pass 2 sums the counts
// of the chunks before its own and writes its pages at that offset, so the
// list comes out ascending and identical run to run.
constexpr int kListChunk = 2048;
constexpr int kListThreads = 256;
constexpr int kListPer = kListChunk / kListThreads;  // consecutive pages per thread

HX_DEVINL int chunk_pages_n(const int32_t* seq_lens, int b, int S, int max_pages) {
  return min((seq_lens[b] + S - 1) / S, max_pages);
}

// selected-page bitmask of this thread's kListPer consecutive pages
HX_DEVINL uint32_t chunk_thread_mask(const float* sc, uint64_t T, int j0, int n, int sinks) {
  uint32_t m = 0;
#pragma unroll
  for (int i = 0; i < kListPer; ++i) {
    const int j = j0 + i;
    if (j < n && (j < sinks || order_key64(__ldg(sc + j), (uint32_t)j) >= T)) m |= 1u << i;
  }
  return m;
}

__global__ void __launch_bounds__(kListThreads) quest_list_count_kernel(const float* scores, const uint64_t* thresh,
                                                                       int H, const int32_t* seq_lens, int S,
                                                                       int max_pages, int sinks_req, int nch,
                                                                       int32_t* chunk_counts) {
  __shared__ int s_w[kListThreads / 32];
  const int row = blockIdx.y, c = blockIdx.x;
  const int n = chunk_pages_n(seq_lens, row / H, S, max_pages);
  const int sinks = min(max(sinks_req, 0), n);
  const int j0 = c * kListChunk + threadIdx.x * kListPer;
  const uint32_t m = chunk_thread_mask(scores + (int64_t)row * max_pages, thresh[row], j0, n, sinks);
  int cnt = __popc(m);
#pragma unroll
  for (int o = 16; o; o >>= 1) cnt += __shfl_xor_sync(0xffffffffu, cnt, o);
  if ((threadIdx.x & 31) == 0) s_w[threadIdx.x >> 5] = cnt;
  __syncthreads();
  if (threadIdx.x == 0) {
    int t = 0;
    for (int w = 0; w < kListThreads / 32; ++w) t += s_w[w];
    chunk_counts[(int64_t)row * nch + c] = t;
  }
}

__global__ void __launch_bounds__(kListThreads) quest_list_scatter_kernel(
    const float* scores, const uint64_t* thresh, int H, const int32_t* seq_lens, int S, int max_pages,
    int sinks_req, int nch, const int32_t* chunk_counts, int max_out, int32_t* out, int32_t* counts) {
  __shared__ int s_w[kListThreads / 32];
  __shared__ int s_base;
  const int row = blockIdx.y, c = blockIdx.x;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int n = chunk_pages_n(seq_lens, row / H, S, max_pages);
  const int sinks = min(max(sinks_req, 0), n);
  // offset of this chunk: the counts of the chunks before it
  int pre = 0;
  for (int i = threadIdx.x; i < c; i += kListThreads) pre += chunk_counts[(int64_t)row * nch + i];
#pragma unroll
  for (int o = 16; o; o >>= 1) pre += __shfl_xor_sync(0xffffffffu, pre, o);
  if (lane == 0) s_w[warp] = pre;
  __syncthreads();
  if (threadIdx.x == 0) {
    int t = 0;
    for (int w = 0; w < kListThreads / 32; ++w) t += s_w[w];
    s_base = t;
  }
  __syncthreads();
  const int base = s_base;
  const int j0 = c * kListChunk + threadIdx.x * kListPer;
  const uint32_t m = chunk_thread_mask(scores + (int64_t)row * max_pages, thresh[row], j0, n, sinks);
  const int cnt = __popc(m);
  // exclusive scan of the per-thread counts (threads hold consecutive pages)
  int inc = cnt;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int v = __shfl_up_sync(0xffffffffu, inc, o);
    if (lane >= o) inc += v;
  }
  __syncthreads();
  if (lane == 31) s_w[warp] = inc;
  __syncthreads();
  int woff = 0;
  for (int w = 0; w < warp; ++w) woff += s_w[w];
  int pos = base + woff + inc - cnt;
  int32_t* orow = out + (int64_t)row * max_out;
#pragma unroll
  for (int i = 0; i < kListPer; ++i) {
    if ((m >> i) & 1u) {
      if (pos < max_out) orow[pos] = j0 + i;
      ++pos;
    }
  }
  if (c == nch - 1 && threadIdx.x == kListThreads - 1) counts[row] = min(pos, max_out);
}

// ---------------------------------------------------------------------------
// global top-K over split-KV shards
//
// A threshold T over the whole sequence's pages (global page indices: the key
// of page g is order_key(score) << 32 | ~g) selects, among pages whose score
// key equals T's high word kT, those with g <= ~low(T). On a shard whose page
// 0 is global page `base`, the same pages are local pages j = g - base with
// key order_key(score) << 32 | ~j, so the shard's threshold keeps kT and
// moves the index bound down by `base`; when the bound lies before the shard
// none of its ties are taken (threshold kT + 1). 0 (every page) and ~0 (no
// page) need no change, and no score key reaches 0xFFFFFFFF, so a threshold
// with that high word selects nothing anywhere.
HX_DEVINL uint64_t shard_threshold(uint64_t Tg, uint32_t base) {
  if (Tg == 0ull || Tg == ~0ull) return Tg;
  const uint32_t kT = (uint32_t)(Tg >> 32);
  if (kT == 0xFFFFFFFFu) return Tg;
  const uint32_t gmax = ~(uint32_t)Tg;  // last global index of the ties taken
  if (gmax < base) return (uint64_t)(kT + 1u) << 32;
  return ((uint64_t)kT << 32) | (uint64_t)(~(gmax - base));
}

// One block per (b, h): this shard's threshold and the decode's slice counts
// of its local pages (the slices of hx_quest_threshold_slices: C slices of
// ceil((n - sinks) / C) non-sink pages, exclusive prefix of the selected
// counts, total in entry C).
__global__ void __launch_bounds__(1024) quest_localize_kernel(const uint64_t* __restrict__ thresh_g, int H,
                                                             const int32_t* __restrict__ seq_lens, int S,
                                                             int max_pages, int sinks_req, int page_begin,
                                                             const float* __restrict__ scores, int C,
                                                             uint64_t* __restrict__ thresh,
                                                             int32_t* __restrict__ slice_off) {
  __shared__ uint32_t s_cnt[kMaxSlices];
  const int bh = blockIdx.x;
  const int lane = lane_id();
  const int n = min((seq_lens[bh / H] + S - 1) / S, max_pages);
  const int sinks = min(max(sinks_req, 0), n);
  const uint64_t T = shard_threshold(thresh_g[bh], (uint32_t)page_begin);
  for (int i = threadIdx.x; i < C; i += blockDim.x) s_cnt[i] = 0;
  __syncthreads();
  const int n_ns = n - sinks;
  const int per = n_ns > 0 ? (n_ns + C - 1) / C : 1;
  const float* sc = scores + (int64_t)bh * max_pages;
  // a warp takes 32 consecutive pages per round (slice_add)
  for (int j0 = sinks + (threadIdx.x & ~31); j0 < n; j0 += blockDim.x) {
    const int j = j0 + lane;
    const bool sel = j < n && order_key64(__ldg(sc + j), (uint32_t)j) >= T;
    slice_add(s_cnt, j < n ? (j - sinks) / per : -1, sel);
  }
  __syncthreads();
  if (threadIdx.x < 32) {
    uint32_t v[kMaxSlices / 32];
    uint32_t sum = 0;
#pragma unroll
    for (int q = 0; q < kMaxSlices / 32; ++q) {
      const int i = (kMaxSlices / 32) * lane + q;
      v[q] = i < C ? s_cnt[i] : 0u;
      sum += v[q];
    }
    uint32_t incl = sum;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const uint32_t x = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += x;
    }
    uint32_t acc = incl - sum;
#pragma unroll
    for (int q = 0; q < kMaxSlices / 32; ++q) {
      const int i = (kMaxSlices / 32) * lane + q;
      if (i < C) slice_off[(int64_t)bh * (C + 1) + i] = (int32_t)acc;
      acc += v[q];
    }
    if (lane == 31) slice_off[(int64_t)bh * (C + 1) + C] = (int32_t)incl;
  }
  if (threadIdx.x == 0) thresh[bh] = T;
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
                                                    page_size, max_pages, sink_pages, ppb, scores)
  bool aligned = (((uintptr_t)kmin | (uintptr_t)kmax) & 7) == 0 && page_stride % 4 == 0 && head_stride % 4 == 0;
  if (stats_dtype == 1 && D == 128 && aligned && head_stride % 8 == 0 && page_stride % 8 == 0 &&
      ((uintptr_t)kmin & 15) == 0 && (const uint16_t*)kmax == (const uint16_t*)kmin + 128) {
    static bool attr[64] = {};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return HX_ERR_LAUNCH;
    if (!attr[dev]) {
      if (cudaFuncSetAttribute(quest_scores_tma_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               (int)sizeof(QuestSmem)) != cudaSuccess)
        return HX_ERR_LAUNCH;
      attr[dev] = true;
    }
    int64_t batches = (int64_t)B * H * ((max_pages + kQPB - 1) / kQPB);
    int64_t want = (batches + kQW - 1) / kQW;
    int grid = (int)(want < 148 ? want : 148);
    if (hx_launch_pdl(quest_scores_tma_kernel, dim3(grid), dim3(kQW * 32), sizeof(QuestSmem), s, q, B, H, group,
                      gqa_mode, (const uint16_t*)kmin, page_stride, head_stride, block_table, bt_stride, seq_lens,
                      page_size, max_pages, sink_pages, scores, hist, (uint32_t*)nullptr) != cudaSuccess) {
      (void)cudaGetLastError();
      return HX_ERR_LAUNCH;
    }
    return HX_OK;
  }
  if (stats_dtype == 1 && D == 128 && aligned) {
    dim3 g2((max_pages + 255) / 256, B * H);
    quest_scores_d128_kernel<<<g2, 256, 0, s>>>(q, H, group, gqa_mode, (const uint16_t*)kmin, (const uint16_t*)kmax,
                                                page_stride, head_stride, block_table, bt_stride, seq_lens, page_size,
                                                max_pages, sink_pages, scores);
  } else if (stats_dtype == 1) {
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
  if (hist) {  // these kernels do not count as they go
    dim3 hg((max_pages + 255) / 256 < 64 ? (max_pages + 255) / 256 : 64, B * H);
    if (hg.x == 0) hg.x = 1;
    quest_hist_kernel<<<hg, 256, 0, s>>>(scores, H, seq_lens, page_size, max_pages, sink_pages, hist);
    HX_LAUNCH_CHECK();
  }
  return HX_OK;
}

HX_API int32_t hx_quest_slices(int32_t max_pages) { return quest_slices(max_pages); }

HX_API int hx_quest_threshold(void* stream, const float* scores, int32_t B, int32_t H, const int32_t* seq_lens,
                              int32_t page_size, int32_t max_pages, int32_t sink_pages, int32_t k_fixed,
                              int32_t frac_num, int32_t frac_den, int32_t hist_ready, uint32_t* hist,
                              uint64_t* cand, uint32_t* counters, uint64_t* thresh, uint32_t* dev_err) {
  return hx_quest_threshold_slices(stream, scores, B, H, seq_lens, page_size, max_pages, sink_pages, k_fixed,
                                   frac_num, frac_den, hist_ready, hist, cand, counters, thresh, nullptr, dev_err);
}

HX_API int hx_quest_threshold_slices(void* stream, const float* scores, int32_t B, int32_t H,
                                     const int32_t* seq_lens, int32_t page_size, int32_t max_pages,
                                     int32_t sink_pages, int32_t k_fixed, int32_t frac_num, int32_t frac_den,
                                     int32_t hist_ready, uint32_t* hist, uint64_t* cand, uint32_t* counters,
                                     uint64_t* thresh, int32_t* slice_off, uint32_t* dev_err) {
  if (B < 0 || H <= 0 || page_size <= 0 || max_pages < 0 || frac_den < 0) return HX_ERR_ARG;
  if (B == 0) return HX_OK;
  if (!scores || !seq_lens || !hist || !cand || !counters || !thresh) return HX_ERR_ARG;
  cudaStream_t st = S_(stream);
  if (!hist_ready) {
    dim3 hg((max_pages + 255) / 256 < 64 ? (max_pages + 255) / 256 : 64, B * H);
    if (hg.x == 0) hg.x = 1;
    quest_hist_kernel<<<hg, 256, 0, st>>>(scores, H, seq_lens, page_size, max_pages, sink_pages, hist);
  }
  if (max_pages <= kRowMaxPages) {
    if (hx_launch_pdl(quest_threshold_row_kernel, dim3(B * H), dim3(256), 0, st, scores, (int)H, seq_lens,
                      (int)page_size, (int)max_pages, (int)sink_pages, (int)k_fixed, (int)frac_num, (int)frac_den,
                      quest_slices(max_pages), hist, cand, thresh, slice_off, dev_err) != cudaSuccess) {
      (void)cudaGetLastError();
      return HX_ERR_LAUNCH;
    }
    return HX_OK;
  }
  dim3 grid(quest_slices(max_pages), B * H);
  if (hx_launch_pdl(quest_threshold_kernel, grid, dim3(256), 0, st, scores, (int)H, seq_lens, (int)page_size,
                    (int)max_pages, (int)sink_pages, (int)k_fixed, (int)frac_num, (int)frac_den, hist, cand, counters,
                    thresh, slice_off, dev_err) != cudaSuccess) {
    (void)cudaGetLastError();
    return HX_ERR_LAUNCH;
  }
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

HX_API int hx_quest_lists(void* stream, const float* scores, const uint64_t* thresh, int32_t B, int32_t H,
                          const int32_t* seq_lens, int32_t page_size, int32_t max_pages, int32_t sink_pages,
                          int32_t max_out, int32_t* out, int32_t* counts, int32_t* chunk_counts) {
  if (B < 0 || H <= 0 || page_size <= 0 || max_pages < 0 || max_out < 0) return HX_ERR_ARG;
  if (B == 0) return HX_OK;
  if (!scores || !thresh || !seq_lens || !counts || (max_out > 0 && !out)) return HX_ERR_ARG;
  const int nch = max(1, (max_pages + kListChunk - 1) / kListChunk);
  if (nch > 1 && !chunk_counts) return HX_ERR_ARG;
  if ((int64_t)B * H > 65535) return HX_ERR_UNSUPPORTED;
  dim3 grid(nch, B * H);
  if (nch > 1) {
    quest_list_count_kernel<<<grid, kListThreads, 0, S_(stream)>>>(scores, thresh, H, seq_lens, page_size,
                                                                   max_pages, sink_pages, nch, chunk_counts);
    HX_LAUNCH_CHECK();
  }
  quest_list_scatter_kernel<<<grid, kListThreads, 0, S_(stream)>>>(scores, thresh, H, seq_lens, page_size,
                                                                   max_pages, sink_pages, nch, chunk_counts,
                                                                   max_out, out, counts);
  HX_LAUNCH_CHECK();
  return HX_OK;
}

HX_API int hx_quest_localize(void* stream, const uint64_t* thresh_global, const float* scores, int32_t B,
                             int32_t H, const int32_t* seq_lens, int32_t page_size, int32_t max_pages,
                             int32_t sink_pages, int32_t page_begin, uint64_t* thresh, int32_t* slice_off) {
  if (B < 0 || H <= 0 || page_size <= 0 || max_pages < 0 || page_begin < 0) return HX_ERR_ARG;
  if (B == 0) return HX_OK;
  if (!thresh_global || !scores || !seq_lens || !thresh || !slice_off) return HX_ERR_ARG;
  if ((int64_t)B * H > 2147483647ll) return HX_ERR_UNSUPPORTED;
  quest_localize_kernel<<<B * H, 1024, 0, S_(stream)>>>(thresh_global, H, seq_lens, page_size, max_pages,
                                                        sink_pages, page_begin, scores, quest_slices(max_pages),
                                                        thresh, slice_off);
  HX_LAUNCH_CHECK();
  return HX_OK;
}

}  // extern "C"
