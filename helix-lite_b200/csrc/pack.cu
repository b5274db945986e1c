// Kernel A and its companions: pack-on-write into the compact pool, staging
// unpack, dense (T, H, D) pack / unpack and the flat torch-spec quantiser.
//
// Semantics follow xFuzzitx/helix-lite src/kvquant:
//   code      argmin_l |fp32(x) - fp32(pole_l)|, strict <, first level wins
//             (triton_batched.py:65-72, compact_pool.py:258-268)
//   outlier   x < lower || x > upper (compact_pool.py:254-256)
//   K stats   running min / max of where(outlier, x, pole[code])
//             (compact_pool.py:270, 285-287)
//   V scales  row min(abs_pos, t_cal - 1) (compact_pool.py:190-201, 467)
#include "common.cuh"

namespace hx {

// ---------------------------------------------------------------------------
// pool maintenance

__global__ void pool_init_stats_kernel(uint16_t* stats, int64_t n_pairs, int D) {
  // stats (H*NB, 2, D): row 0 = +inf (min), row 1 = -inf (max)
  int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  int64_t total = n_pairs * 2 * D;
  for (; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    int64_t r = (i / D) & 1;
    stats[i] = r ? 0xFC00u : 0x7C00u;
  }
}

__global__ void pool_reset_pages_kernel(hx_pool_layer pool, const int32_t* pages, int n, uint32_t* err) {
  // one block per (listed page, head)
  int idx = blockIdx.x;
  int h = blockIdx.y;
  int pg = pages[idx];
  if (pg < 0 || pg >= pool.num_blocks) {
    if (threadIdx.x == 0) set_err(err, HX_DEV_ERR_BOUNDS);
    return;
  }
  const int D = pool.head_size;
  uint16_t* st = pool.stats + ((int64_t)h * pool.num_blocks + pg) * 2 * D;
  for (int i = threadIdx.x; i < 2 * D; i += blockDim.x) st[i] = (i < D) ? 0x7C00u : 0xFC00u;
  if (threadIdx.x < 2) {
    uint32_t* dr = pool.dir + (((int64_t)h * pool.num_blocks + pg) * 2 + threadIdx.x) * 4;
    dr[2] = 0;  // count
    dr[3] = 0;  // rows; offset and capacity are kept so the chunk is reused
  }
}

// ---------------------------------------------------------------------------
// code search

// Nearest level by the reference's scan. p[] holds fp32 poles; L <= LMAX.
template <int LMAX>
HX_DEVINL int nearest_level(float x, const float (&p)[LMAX], int L, float& pole) {
  float best = __int_as_float(0x7f800000);  // +inf
  int idx = 0;
  float bp = 0.0f;
#pragma unroll
  for (int l = 0; l < LMAX; ++l) {
    if (l < L) {
      float d = fabsf(__fsub_rn(x, p[l]));
      if (d < best) {
        best = d;
        idx = l;
        bp = p[l];
      }
    }
  }
  pole = bp;
  return idx;
}

// ---------------------------------------------------------------------------
// pack-on-write

struct OutList {  // directory record of one (head, page, K|V), held by lane 0
  uint32_t off, cap, cnt, rows;
};

HX_DEVINL uint32_t* dir_ptr(const hx_pool_layer& pool, int h, int pg, int kv) {
  return pool.dir + (((int64_t)h * pool.num_blocks + pg) * 2 + kv) * 4;
}

// Drop the entries of slots [t0, t1) from a page list (an overwrite), keeping
// the order of the others. Whole warp; returns the new count on every lane.
HX_DEVINL uint32_t filter_slots(uint32_t* arena, uint32_t off, uint32_t cnt, int t0, int t1) {
  const int lane = lane_id();
  uint32_t out = 0;
  for (uint32_t base = 0; base < cnt; base += 32) {
    uint32_t i = base + lane;
    uint32_t e = 0;
    bool keep = false;
    if (i < cnt) {
      e = __ldcg(arena + off + i);
      int t = (e >> 24) & 31;
      keep = (t < t0) || (t >= t1);
    }
    uint32_t m = __ballot_sync(0xffffffffu, keep);
    __syncwarp();
    if (keep) arena[off + out + __popc(m & ((1u << lane) - 1))] = e;
    out += __popc(m);
    __syncwarp();
  }
  return out;
}

// Make room for `need` entries; grows the chunk (doubling) from the arena.
// Returns false (and flags) when the arena is exhausted.
HX_DEVINL bool ensure_capacity(const hx_pool_layer& pool, OutList& L, uint32_t need, uint32_t* err) {
  const int lane = lane_id();
  uint32_t ok = 1;
  if (need > L.cap) {
    uint32_t new_cap = max(max((need + 7u) & ~7u, 2u * L.cap), 16u);
    uint32_t new_off = 0;
    if (lane == 0) {
      new_off = atomicAdd(pool.arena_top, new_cap);
      ok = ((int64_t)new_off + new_cap <= pool.arena_capacity) ? 1u : 0u;
      if (!ok) set_err(err, HX_DEV_ERR_ARENA_FULL);
    }
    ok = __shfl_sync(0xffffffffu, ok, 0);
    new_off = __shfl_sync(0xffffffffu, new_off, 0);
    if (!ok) return false;
    for (uint32_t i = lane; i < L.cnt; i += 32) pool.arena[new_off + i] = __ldcg(pool.arena + L.off + i);
    __syncwarp();
    L.off = new_off;
    L.cap = new_cap;
  }
  return true;
}

// Append one row's outliers (ballot masks m[k] over channels lane + 32k).
template <int KD>
HX_DEVINL void append_row(const hx_pool_layer& pool, OutList& L, const uint32_t (&m)[KD],
                          const uint16_t (&xb)[KD], int t, uint32_t* err) {
  const int lane = lane_id();
  uint32_t n = 0;
#pragma unroll
  for (int k = 0; k < KD; ++k) n += __popc(m[k]);
  if (n == 0) return;
  if (!ensure_capacity(pool, L, L.cnt + n, err)) return;
  uint32_t base = L.off + L.cnt;
  const uint32_t lt = (1u << lane) - 1;
#pragma unroll
  for (int k = 0; k < KD; ++k) {
    if ((m[k] >> lane) & 1u) {
      int d = lane + 32 * k;
      pool.arena[base + __popc(m[k] & lt)] = (uint32_t)xb[k] | ((uint32_t)d << 16) | ((uint32_t)t << 24);
    }
    base += __popc(m[k]);
  }
  L.cnt += n;
  __syncwarp();
}

HX_DEVINL void atomic_min_f16(uint16_t* addr, uint16_t v, uint32_t* err) {
  uint16_t old = __ldcg(addr);
  for (int it = 0; it < 256; ++it) {
    if (!(h2f(v) < h2f(old))) return;
    uint16_t prev = atomicCAS(reinterpret_cast<unsigned short*>(addr), old, v);
    if (prev == old) return;
    old = prev;
  }
  set_err(err, HX_DEV_ERR_TIMEOUT);
}

HX_DEVINL void atomic_max_f16(uint16_t* addr, uint16_t v, uint32_t* err) {
  uint16_t old = __ldcg(addr);
  for (int it = 0; it < 256; ++it) {
    if (!(h2f(v) > h2f(old))) return;
    uint16_t prev = atomicCAS(reinterpret_cast<unsigned short*>(addr), old, v);
    if (prev == old) return;
    old = prev;
  }
  set_err(err, HX_DEV_ERR_TIMEOUT);
}

// Write one packed code row from the warp's staged byte codes.
HX_DEVINL void store_row(uint8_t* dst, const uint8_t* codes, int D, int bits) {
  const int per = 8 / bits;
  const int nbytes = D / per;
  for (int b = lane_id(); b < nbytes; b += 32) {
    uint32_t v = 0;
    for (int j = 0; j < per; ++j) v |= (uint32_t)(codes[b * per + j] & ((1 << bits) - 1)) << (bits * j);
    dst[b] = (uint8_t)v;
  }
}

// One warp per (run leader token, head). A run is a maximal stretch of input
// tokens that fill consecutive slots of one page; the leader processes it in
// slot order. A page whose slots come as several runs in one launch (tokens in
// any order) is updated one run at a time: the warp holds the page lock (bit
// 31 of the K directory record's rows word) while it edits the page's lists.
constexpr uint32_t kGenericPageLock = 0x80000000u;

// Take / release a page lock (whole warp; bounded spin, false = gave up).
HX_DEVINL bool generic_page_lock(uint32_t* rows_word, uint32_t* err) {
  uint32_t got = 0;
  if (lane_id() == 0) {
    for (uint32_t it = 0; it < (1u << 20); ++it) {
      if ((atomicOr(rows_word, kGenericPageLock) & kGenericPageLock) == 0u) {
        got = 1;
        break;
      }
      __nanosleep(64);
    }
    if (!got) set_err(err, HX_DEV_ERR_TIMEOUT);
    __threadfence();
  }
  return __shfl_sync(0xffffffffu, got, 0) != 0;
}
template <int KD, int LK, int LV>
__global__ void __launch_bounds__(128) pack_append_kernel(hx_pool_layer pool, hx_layer_scales sc,
                                                          const uint16_t* __restrict__ key,
                                                          const uint16_t* __restrict__ value,
                                                          const int64_t* __restrict__ slots,
                                                          const int64_t* __restrict__ abspos, int T,
                                                          uint32_t* err) {
  __shared__ uint8_t s_codes[4][256];
  const int warp = threadIdx.x >> 5;
  const int lane = lane_id();
  const int H = pool.num_kv_heads, D = pool.head_size, S = pool.block_size;
  const int64_t w = (int64_t)blockIdx.x * 4 + warp;
  if (w >= (int64_t)T * H) return;
  const int i = (int)(w / H);
  const int h = (int)(w % H);
  const int64_t s0 = slots[i];
  if (s0 < 0) return;
  if (i > 0) {
    int64_t sp = slots[i - 1];
    if (sp >= 0 && sp + 1 == s0 && (s0 % S) != 0) return;  // not a run leader
  }
  const int64_t page64 = s0 / S;
  if (page64 >= pool.num_blocks) {
    if (lane == 0) set_err(err, HX_DEV_ERR_BOUNDS);
    return;
  }
  const int pg = (int)page64;
  const int t0 = (int)(s0 % S);
  int n = 1;
  while (i + n < T && t0 + n < S && slots[i + n] == s0 + n) ++n;

  const int rbk = D * pool.bits_k / 8, rbv = D * pool.bits_v / 8;
  uint8_t* seg = pool.codes + ((int64_t)h * pool.num_blocks + pg) * (int64_t)S * (rbk + rbv);
  uint8_t* sc8 = s_codes[warp];
  const int Tc = sc.t_cal;

  // K scales of this head: poles for channels lane + 32k
  float kp[KD][LK];
  float kup[KD], klo[KD];
#pragma unroll
  for (int k = 0; k < KD; ++k) {
    int d = lane + 32 * k;
    bool ok = d < D;
#pragma unroll
    for (int l = 0; l < LK; ++l)
      kp[k][l] = (ok && l < sc.levels_k) ? h2f(sc.k_poles[((int64_t)h * D + d) * sc.levels_k + l]) : 0.0f;
    kup[k] = ok ? h2f(sc.k_upper[(int64_t)h * D + d]) : 0.0f;
    klo[k] = ok ? h2f(sc.k_lower[(int64_t)h * D + d]) : 0.0f;
  }
  float rmin[KD], rmax[KD];
#pragma unroll
  for (int k = 0; k < KD; ++k) {
    rmin[k] = __int_as_float(0x7f800000);
    rmax[k] = __int_as_float(0xff800000);
  }

  if (!generic_page_lock(dir_ptr(pool, h, pg, 0) + 3, err)) return;
  OutList LKs, LVs;
  {
    uint32_t* dk = dir_ptr(pool, h, pg, 0);
    uint32_t* dv = dir_ptr(pool, h, pg, 1);
    // a record's last word: rows (bits 0-7, slots written) | the bandwidth
    // kernels' per-launch run count (bits 8-30, zero between launches) | lock (31)
    LKs = {__ldcg(dk), __ldcg(dk + 1), __ldcg(dk + 2), __ldcg(dk + 3) & 0xFFu};
    LVs = {__ldcg(dv), __ldcg(dv + 1), __ldcg(dv + 2), __ldcg(dv + 3) & 0xFFu};
    if ((int)LKs.rows > t0) LKs.cnt = filter_slots(pool.arena, LKs.off, LKs.cnt, t0, t0 + n);
    if ((int)LVs.rows > t0) LVs.cnt = filter_slots(pool.arena, LVs.off, LVs.cnt, t0, t0 + n);
  }

  // Count the run's outliers first and size the page lists once, so a
  // prefill run allocates exactly what it needs (no growth copies).
  {
    uint32_t needk = 0, needv = 0;
    for (int j = 0; j < n; ++j) {
      const int64_t row = ((int64_t)(i + j) * H + h) * D;
      int64_t p = abspos[i + j];
      p = p < 0 ? 0 : p;
      const int64_t prow = (int64_t)h * Tc + (p < Tc ? p : Tc - 1);
      const float vup = h2f(sc.v_upper[prow]), vlo = h2f(sc.v_lower[prow]);
#pragma unroll
      for (int k = 0; k < KD; ++k) {
        int d = lane + 32 * k;
        bool ok = d < D;
        float xk = ok ? h2f(key[row + d]) : 0.0f;
        float xv = ok ? h2f(value[row + d]) : 0.0f;
        needk += __popc(__ballot_sync(0xffffffffu, ok && ((xk > kup[k]) || (xk < klo[k]))));
        needv += __popc(__ballot_sync(0xffffffffu, ok && ((xv > vup) || (xv < vlo))));
      }
    }
    ensure_capacity(pool, LKs, LKs.cnt + needk, err);
    ensure_capacity(pool, LVs, LVs.cnt + needv, err);
  }

  for (int j = 0; j < n; ++j) {
    const int t = t0 + j;
    const int64_t row = ((int64_t)(i + j) * H + h) * D;
    // ---- K row
    uint32_t m[KD];
    uint16_t xb[KD];
#pragma unroll
    for (int k = 0; k < KD; ++k) {
      int d = lane + 32 * k;
      bool ok = d < D;
      xb[k] = ok ? key[row + d] : (uint16_t)0;
      float x = h2f(xb[k]);
      float pole;
      int c = nearest_level<LK>(x, kp[k], sc.levels_k, pole);
      bool out = ok && ((x > kup[k]) || (x < klo[k]));
      float rec = out ? x : pole;
      if (ok) {
        sc8[d] = (uint8_t)c;
        rmin[k] = (rec < rmin[k]) ? rec : rmin[k];
        rmax[k] = (rec > rmax[k]) ? rec : rmax[k];
      }
      m[k] = __ballot_sync(0xffffffffu, out);
    }
    __syncwarp();
    store_row(seg + (int64_t)t * rbk, sc8, D, pool.bits_k);
    append_row<KD>(pool, LKs, m, xb, t, err);
    __syncwarp();

    // ---- V row (per-token scales)
    int64_t p = abspos[i + j];
    if (p < 0) {
      if (lane == 0) set_err(err, HX_DEV_ERR_BOUNDS);
      p = 0;
    }
    const int64_t prow = (int64_t)h * Tc + (p < Tc ? p : Tc - 1);
    float vp[LV];
#pragma unroll
    for (int l = 0; l < LV; ++l) vp[l] = (l < sc.levels_v) ? h2f(sc.v_poles[prow * sc.levels_v + l]) : 0.0f;
    const float vup = h2f(sc.v_upper[prow]), vlo = h2f(sc.v_lower[prow]);
#pragma unroll
    for (int k = 0; k < KD; ++k) {
      int d = lane + 32 * k;
      bool ok = d < D;
      xb[k] = ok ? value[row + d] : (uint16_t)0;
      float x = h2f(xb[k]);
      float pole;
      int c = nearest_level<LV>(x, vp, sc.levels_v, pole);
      bool out = ok && ((x > vup) || (x < vlo));
      if (ok) sc8[d] = (uint8_t)c;
      m[k] = __ballot_sync(0xffffffffu, out);
    }
    __syncwarp();
    store_row(seg + (int64_t)S * rbk + (int64_t)t * rbv, sc8, D, pool.bits_v);
    append_row<KD>(pool, LVs, m, xb, t, err);
    __syncwarp();
  }

  // K page stats: fold the run's min / max into the page (fp16 is exact here)
  uint16_t* st = pool.stats + ((int64_t)h * pool.num_blocks + pg) * 2 * D;
#pragma unroll
  for (int k = 0; k < KD; ++k) {
    int d = lane + 32 * k;
    if (d < D) {
      atomic_min_f16(st + d, f2h(rmin[k]), err);
      atomic_max_f16(st + D + d, f2h(rmax[k]), err);
    }
  }
  __threadfence();  // entries and stats visible before the page is released
  __syncwarp();
  if (lane == 0) {
    uint32_t rows_new = (uint32_t)(t0 + n);
    uint32_t* dk = dir_ptr(pool, h, pg, 0);
    uint32_t* dv = dir_ptr(pool, h, pg, 1);
    dk[0] = LKs.off; dk[1] = LKs.cap; dk[2] = LKs.cnt;
    dv[0] = LVs.off; dv[1] = LVs.cap; dv[2] = LVs.cnt; dv[3] = max(LVs.rows, rows_new);
    __threadfence();
    atomicExch(dk + 3, max(LKs.rows, rows_new));  // rows, lock bit clear
  }
}

// ---------------------------------------------------------------------------
// staging unpack: one block per (selected page, head)

HX_DEVINL int code_at(const uint8_t* rowp, int d, int bits) {
  const int per = 8 / bits;
  return (rowp[d / per] >> ((d % per) * bits)) & ((1 << bits) - 1);
}

__global__ void __launch_bounds__(128) unpack_pages_kernel(hx_pool_layer pool, hx_layer_scales sc,
                                                           const int64_t* block_ids, const int64_t* first_pos,
                                                           uint16_t* sk, uint16_t* sv, uint32_t* err) {
  extern __shared__ uint16_t tile[];  // K (S, D) then V (S, D)
  const int k = blockIdx.x, h = blockIdx.y;
  const int H = pool.num_kv_heads, D = pool.head_size, S = pool.block_size;
  const int64_t pg = block_ids[k];
  if (pg < 0 || pg >= pool.num_blocks) {
    if (threadIdx.x == 0) set_err(err, HX_DEV_ERR_BOUNDS);
    return;
  }
  const int rbk = D * pool.bits_k / 8, rbv = D * pool.bits_v / 8;
  const uint8_t* seg = pool.codes + ((int64_t)h * pool.num_blocks + pg) * (int64_t)S * (rbk + rbv);
  const int64_t fp = first_pos[k];
  const int Tc = sc.t_cal;
  uint16_t* tk = tile;
  uint16_t* tv = tile + S * D;
  for (int e = threadIdx.x; e < S * D; e += blockDim.x) {
    int t = e / D, d = e % D;
    int ck = code_at(seg + t * rbk, d, pool.bits_k);
    int cv = code_at(seg + S * rbk + t * rbv, d, pool.bits_v);
    // a code >= levels can only come from an unwritten slot; it reads level 0
    ck = ck < sc.levels_k ? ck : 0;
    cv = cv < sc.levels_v ? cv : 0;
    int64_t p = fp + t;
    p = p < 0 ? 0 : (p < Tc ? p : Tc - 1);
    tk[e] = sc.k_poles[((int64_t)h * D + d) * sc.levels_k + ck];
    tv[e] = sc.v_poles[((int64_t)h * Tc + p) * sc.levels_v + cv];
  }
  __syncthreads();
  for (int kv = 0; kv < 2; ++kv) {
    const uint32_t* dr = dir_ptr(pool, h, (int)pg, kv);
    uint32_t off = dr[0], cnt = dr[2];
    uint16_t* tt = kv ? tv : tk;
    for (uint32_t i = threadIdx.x; i < cnt; i += blockDim.x) {
      uint32_t e = pool.arena[off + i];
      int t = (e >> 24) & 31, d = (e >> 16) & 255;
      if (t < S && d < D) tt[t * D + d] = (uint16_t)(e & 0xffffu);
      else set_err(err, HX_DEV_ERR_BOUNDS);
    }
  }
  __syncthreads();
  for (int e = threadIdx.x; e < S * D; e += blockDim.x) {
    int t = e / D, d = e % D;
    int64_t o = (((int64_t)k * S + t) * H + h) * D + d;
    sk[o] = tk[e];
    sv[o] = tv[e];
  }
}

// ---------------------------------------------------------------------------
// dense (T, H, D) pack / unpack, one thread per element

template <int LMAX>
__global__ void pack_dense_kernel(int mode, const uint16_t* __restrict__ values, const uint16_t* __restrict__ poles,
                                  const uint16_t* __restrict__ upper, const uint16_t* __restrict__ lower, int T,
                                  int H, int D, int L, uint8_t* codes, uint16_t* outv, uint8_t* outm) {
  int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  int64_t n = (int64_t)T * H * D;
  if (i >= n) return;
  int d = (int)(i % D);
  int64_t th = i / D;
  int h = (int)(th % H);
  int t = (int)(th / H);
  int64_t g = mode == 0 ? ((int64_t)h * D + d) : ((int64_t)h * T + t);  // scale group
  float p[LMAX];
#pragma unroll
  for (int l = 0; l < LMAX; ++l) p[l] = l < L ? h2f(poles[g * L + l]) : 0.0f;
  uint16_t xb = values[i];
  float x = h2f(xb);
  float pole;
  int c = nearest_level<LMAX>(x, p, L, pole);
  bool out = (x > h2f(upper[g])) || (x < h2f(lower[g]));
  codes[i] = (uint8_t)c;
  outv[i] = out ? xb : (uint16_t)0;
  outm[i] = out ? 1 : 0;
}

__global__ void unpack_dense_kernel(int mode, const uint8_t* __restrict__ codes, const uint16_t* __restrict__ outv,
                                    const uint8_t* __restrict__ outm, const uint16_t* __restrict__ poles, int T,
                                    int H, int D, int L, uint16_t* out) {
  int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  int64_t n = (int64_t)T * H * D;
  if (i >= n) return;
  int d = (int)(i % D);
  int64_t th = i / D;
  int h = (int)(th % H);
  int t = (int)(th / H);
  int64_t g = mode == 0 ? ((int64_t)h * D + d) : ((int64_t)h * T + t);
  int c = codes[i];
  // the reference selects level by level from 0 (triton_batched.py:113-118):
  // a code outside [0, L) reconstructs to 0
  uint16_t rec = c < L ? poles[g * L + c] : (uint16_t)0;
  out[i] = outm[i] ? outv[i] : rec;
}

// ---------------------------------------------------------------------------
// flat torch-spec quantiser (nuq.py), fp32 or fp16 elements

template <typename Tv>
HX_DEVINL float ld_f(const Tv* p, int64_t i);
template <>
HX_DEVINL float ld_f<float>(const float* p, int64_t i) { return p[i]; }
template <>
HX_DEVINL float ld_f<uint16_t>(const uint16_t* p, int64_t i) { return h2f(p[i]); }

// |x - p| rounded as torch rounds it for the element dtype: fp32 once; fp16
// through an fp32 op then a round to fp16 (torch's opmath for half).
template <typename Tv>
HX_DEVINL float tdiff(float x, float p);
template <>
HX_DEVINL float tdiff<float>(float x, float p) { return fabsf(__fsub_rn(x, p)); }
template <>
HX_DEVINL float tdiff<uint16_t>(float x, float p) { return fabsf(__half2float(__float2half_rn(__fsub_rn(x, p)))); }

template <typename Tv>
HX_DEVINL float tround(float v);
template <>
HX_DEVINL float tround<float>(float v) { return v; }
template <>
HX_DEVINL float tround<uint16_t>(float v) { return __half2float(__float2half_rn(v)); }

template <typename Tv>
__global__ void quant_mask_kernel(const Tv* values, const Tv* upper, const Tv* lower, int64_t n, int64_t seq_stride,
                                  int64_t seq_size, int first_few, uint8_t* mask) {
  int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  float x = ld_f(values, i);
  bool out = (x < ld_f(lower, i)) || (x > ld_f(upper, i));
  mask[i] = out ? 1 : 0;
}

// cap: one warp per row; an element stays when fewer than `cap` masked
// elements of its row have a larger magnitude (ties: lower index first).
template <typename Tv>
__global__ void cap_kernel(const Tv* values, const Tv* upper, const Tv* lower, int64_t rows, int row, int cap,
                           const uint8_t* mask_in, uint8_t* mask_out) {
  extern __shared__ float mag[];
  const int warp = threadIdx.x >> 5, lane = lane_id();
  const int64_t r = (int64_t)blockIdx.x * (blockDim.x / 32) + warp;
  if (r >= rows) return;
  float* m = mag + warp * row;
  const int64_t base = r * row;
  for (int j = lane; j < row; j += 32) {
    int64_t i = base + j;
    float x = ld_f(values, i), up = ld_f(upper, i), lo = ld_f(lower, i);
    // torch spec in the element dtype: zp = (u + l) / 2, hb = clamp((u - l) / 2, 1e-8)
    float zp = tround<Tv>(tround<Tv>(up + lo) / 2.0f);
    float hb = tround<Tv>(tround<Tv>(up - lo) / 2.0f);
    float eps = tround<Tv>(1e-8f);
    hb = hb < eps ? eps : hb;
    float nz = tround<Tv>(tround<Tv>(x - zp) / hb);
    m[j] = tround<Tv>(fabsf(nz) * (mask_in[i] ? 1.0f : 0.0f));
  }
  __syncwarp();
  for (int j = lane; j < row; j += 32) {
    float v = m[j];
    int rank = 0;
    for (int q = 0; q < row; ++q) {
      float u = m[q];
      rank += (u > v) || (u == v && q < j);
    }
    mask_out[base + j] = rank < cap ? 1 : 0;
  }
}

template <typename Tv, int LMAX>
__global__ void quant_recon_kernel(const Tv* values, const Tv* poles, int64_t n, int L, int64_t seq_stride,
                                   int64_t seq_size, int first_few, uint8_t* mask, Tv* recon) {
  int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  float x = ld_f(values, i);
  float best = __int_as_float(0x7f800000);
  int idx = 0;
#pragma unroll
  for (int l = 0; l < LMAX; ++l) {
    if (l < L) {
      float d = tdiff<Tv>(x, ld_f(poles, i * L + l));
      if (d < best) {
        best = d;
        idx = l;
      }
    }
  }
  bool out = mask[i] != 0;
  if (first_few > 0 && ((i / seq_stride) % seq_size) < first_few) out = true;
  mask[i] = out ? 1 : 0;
  recon[i] = out ? values[i] : poles[i * L + idx];
}

template <typename Tv>
__global__ void dequant_flat_kernel(const int64_t* codes, const Tv* outl, const uint8_t* mask, const Tv* poles,
                                    int64_t n, int L, Tv* out, uint32_t* err) {
  int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  if (mask[i]) {
    out[i] = outl[i];
    return;
  }
  int64_t c = codes[i];
  if (c < 0 || c >= L) {
    set_err(err, HX_DEV_ERR_BOUNDS);
    out[i] = Tv(0);
    return;
  }
  out[i] = poles[i * L + c];
}

}  // namespace hx

// ===========================================================================
// C ABI

using namespace hx;

static inline cudaStream_t S_(void* s) { return reinterpret_cast<cudaStream_t>(s); }

static bool pool_ok(const hx_pool_layer* p) {
  return p && p->codes && p->stats && p->dir && p->arena && p->arena_top && p->num_blocks > 0 &&
         p->block_size > 0 && p->block_size <= 32 && p->num_kv_heads > 0 && p->head_size > 0 &&
         p->head_size <= 256 && p->head_size % 8 == 0 && (p->bits_k == 2 || p->bits_k == 4) &&
         (p->bits_v == 2 || p->bits_v == 4);
}

static bool scales_ok(const hx_layer_scales* s, const hx_pool_layer* p) {
  return s && s->k_poles && s->k_upper && s->k_lower && s->v_poles && s->v_upper && s->v_lower &&
         s->levels_k >= 1 && s->levels_k <= (1 << p->bits_k) && s->levels_v >= 1 &&
         s->levels_v <= (1 << p->bits_v) && s->t_cal >= 1;
}

template <typename Tv>
static int quantize_flat_t(cudaStream_t s, const Tv* v, const Tv* p, const Tv* up, const Tv* lo, int64_t n, int L,
                           int cap, int64_t row, int64_t seq_stride, int64_t seq_size, int first_few, Tv* recon,
                           uint8_t* mask, uint8_t* scratch) {
  unsigned blocks = (unsigned)((n + 255) / 256);
  quant_mask_kernel<Tv><<<blocks, 256, 0, s>>>(v, up, lo, n, seq_stride, seq_size, first_few, mask);
  if (cap > 0) {
    if (!scratch || row <= 0 || n % row != 0 || row > 4096) return HX_ERR_ARG;
    int64_t rows = n / row;
    const int wpb = 4;
    size_t smem = (size_t)wpb * row * sizeof(float);
    if (smem > 48 * 1024) {
      if (cudaFuncSetAttribute(cap_kernel<Tv>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
        return HX_ERR_LAUNCH;
    }
    cudaMemcpyAsync(scratch, mask, (size_t)n, cudaMemcpyDeviceToDevice, s);
    cap_kernel<Tv><<<(unsigned)((rows + wpb - 1) / wpb), 32 * wpb, smem, s>>>(v, up, lo, rows, (int)row, cap, scratch,
                                                                           mask);
  }
  if (L <= 4)
    quant_recon_kernel<Tv, 4><<<blocks, 256, 0, s>>>(v, p, n, L, seq_stride, seq_size, first_few, mask, recon);
  else
    quant_recon_kernel<Tv, 16><<<blocks, 256, 0, s>>>(v, p, n, L, seq_stride, seq_size, first_few, mask, recon);
  HX_LAUNCH_CHECK();
  return HX_OK;
}

extern "C" {

HX_API const char* hx_version(void) { return "helix-kv 0.1 sm_100a"; }

HX_API int hx_pool_init(void* stream, const hx_pool_layer* pool) {
  if (!pool_ok(pool)) return HX_ERR_ARG;
  cudaStream_t s = S_(stream);
  const int64_t H = pool->num_kv_heads, NB = pool->num_blocks, S = pool->block_size, D = pool->head_size;
  const int64_t seg = S * D * (pool->bits_k + pool->bits_v) / 8;
  if (cudaMemsetAsync(pool->codes, 0, H * NB * seg, s) != cudaSuccess) return HX_ERR_LAUNCH;
  if (cudaMemsetAsync(pool->dir, 0, H * NB * 2 * 4 * sizeof(uint32_t), s) != cudaSuccess) return HX_ERR_LAUNCH;
  if (cudaMemsetAsync(pool->arena_top, 0, sizeof(uint32_t), s) != cudaSuccess) return HX_ERR_LAUNCH;
  pool_init_stats_kernel<<<1184, 256, 0, s>>>(pool->stats, H * NB, (int)D);
  HX_LAUNCH_CHECK();
  return HX_OK;
}

HX_API int hx_pool_reset_pages(void* stream, const hx_pool_layer* pool, const int32_t* pages, int32_t n,
                               uint32_t* dev_err) {
  if (!pool_ok(pool) || n < 0 || (n > 0 && !pages)) return HX_ERR_ARG;
  if (n == 0) return HX_OK;
  dim3 grid(n, pool->num_kv_heads);
  pool_reset_pages_kernel<<<grid, 128, 0, S_(stream)>>>(*pool, pages, n, dev_err);
  HX_LAUNCH_CHECK();
  return HX_OK;
}

HX_API int hx_pack_append(void* stream, const hx_pool_layer* pool, const hx_layer_scales* sc, const uint16_t* key,
                          const uint16_t* value, const int64_t* slot_mapping, const int64_t* abs_positions,
                          int32_t T, uint32_t* dev_err) {
  if (!pool_ok(pool) || !scales_ok(sc, pool) || T < 0) return HX_ERR_ARG;
  if (T == 0) return HX_OK;
  if (!key || !value || !slot_mapping || !abs_positions) return HX_ERR_ARG;
  const int D = pool->head_size;
  if (D > 128) return HX_ERR_UNSUPPORTED;
  {
    const int rc = hx_pack_fast_launch(S_(stream), pool, sc, key, value, slot_mapping, abs_positions, T, dev_err);
    if (rc != HX_ERR_UNSUPPORTED) return rc;
  }
  int64_t warps = (int64_t)T * pool->num_kv_heads;
  int64_t blocks = (warps + 3) / 4;
  if (blocks > 0x7fffffff) return HX_ERR_ARG;
  cudaStream_t s = S_(stream);
  const int KD = (D + 31) / 32;
  const int lk = sc->levels_k <= 4 ? 4 : 16, lv = sc->levels_v <= 4 ? 4 : 16;
#define HX_PACK_LAUNCH(KD_, LK_, LV_) \
  pack_append_kernel<KD_, LK_, LV_><<<(unsigned)blocks, 128, 0, s>>>(*pool, *sc, key, value, slot_mapping, abs_positions, T, dev_err)
#define HX_PACK_KD(KD_)                          \
  do {                                           \
    if (lk == 4 && lv == 4) HX_PACK_LAUNCH(KD_, 4, 4);   \
    else if (lk == 4) HX_PACK_LAUNCH(KD_, 4, 16);        \
    else if (lv == 4) HX_PACK_LAUNCH(KD_, 16, 4);        \
    else HX_PACK_LAUNCH(KD_, 16, 16);                    \
  } while (0)
  if (KD == 1) HX_PACK_KD(1);
  else if (KD == 2) HX_PACK_KD(2);
  else HX_PACK_KD(4);
#undef HX_PACK_KD
#undef HX_PACK_LAUNCH
  HX_LAUNCH_CHECK();
  return HX_OK;
}

HX_API int hx_unpack_pages(void* stream, const hx_pool_layer* pool, const hx_layer_scales* sc,
                           const int64_t* block_ids, const int64_t* first_pos, int32_t nk, uint16_t* staging_k,
                           uint16_t* staging_v, uint32_t* dev_err) {
  if (!pool_ok(pool) || !scales_ok(sc, pool) || nk < 0) return HX_ERR_ARG;
  if (nk == 0) return HX_OK;
  if (!block_ids || !first_pos || !staging_k || !staging_v) return HX_ERR_ARG;
  size_t smem = 2ull * pool->block_size * pool->head_size * sizeof(uint16_t);
  if (smem > 48 * 1024) {
    if (cudaFuncSetAttribute(unpack_pages_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) !=
        cudaSuccess)
      return HX_ERR_LAUNCH;
  }
  dim3 grid(nk, pool->num_kv_heads);
  unpack_pages_kernel<<<grid, 128, smem, S_(stream)>>>(*pool, *sc, block_ids, first_pos, staging_k, staging_v,
                                                       dev_err);
  HX_LAUNCH_CHECK();
  return HX_OK;
}

HX_API int hx_nuq_pack_dense(void* stream, int32_t mode, const uint16_t* values, const uint16_t* poles,
                             const uint16_t* upper, const uint16_t* lower, int32_t T, int32_t H, int32_t D,
                             int32_t L, uint8_t* codes, uint16_t* outv, uint8_t* outm) {
  if ((mode != 0 && mode != 1) || T < 0 || H <= 0 || D <= 0 || L < 1 || L > 16) return HX_ERR_ARG;
  int64_t n = (int64_t)T * H * D;
  if (n == 0) return HX_OK;
  if (!values || !poles || !upper || !lower || !codes || !outv || !outm) return HX_ERR_ARG;
  unsigned blocks = (unsigned)((n + 255) / 256);
  if (L <= 4)
    pack_dense_kernel<4><<<blocks, 256, 0, S_(stream)>>>(mode, values, poles, upper, lower, T, H, D, L, codes, outv, outm);
  else
    pack_dense_kernel<16><<<blocks, 256, 0, S_(stream)>>>(mode, values, poles, upper, lower, T, H, D, L, codes, outv, outm);
  HX_LAUNCH_CHECK();
  return HX_OK;
}

HX_API int hx_nuq_unpack_dense(void* stream, int32_t mode, const uint8_t* codes, const uint16_t* outv,
                               const uint8_t* outm, const uint16_t* poles, int32_t T, int32_t H, int32_t D,
                               int32_t L, uint16_t* out) {
  if ((mode != 0 && mode != 1) || T < 0 || H <= 0 || D <= 0 || L < 1) return HX_ERR_ARG;
  int64_t n = (int64_t)T * H * D;
  if (n == 0) return HX_OK;
  if (!codes || !outv || !outm || !poles || !out) return HX_ERR_ARG;
  unpack_dense_kernel<<<(unsigned)((n + 255) / 256), 256, 0, S_(stream)>>>(mode, codes, outv, outm, poles, T, H, D,
                                                                           L, out);
  HX_LAUNCH_CHECK();
  return HX_OK;
}

HX_API int hx_nuq_quantize_flat(void* stream, int32_t dtype, const void* values, const void* poles,
                                const void* upper, const void* lower, int64_t n, int32_t L, int32_t cap,
                                int64_t row, int64_t seq_stride, int64_t seq_size, int32_t first_few, void* recon,
                                uint8_t* mask, uint8_t* scratch_mask) {
  if (n < 0 || L < 1 || L > 16 || (dtype != 0 && dtype != 1)) return HX_ERR_ARG;
  if (n == 0) return HX_OK;
  if (!values || !poles || !upper || !lower || !recon || !mask) return HX_ERR_ARG;
  if (first_few > 0 && (seq_stride <= 0 || seq_size <= 0)) return HX_ERR_ARG;
  cudaStream_t s = S_(stream);
  if (dtype == 0)
    return quantize_flat_t<float>(s, (const float*)values, (const float*)poles, (const float*)upper,
                                  (const float*)lower, n, L, cap, row, seq_stride, seq_size, first_few,
                                  (float*)recon, mask, scratch_mask);
  return quantize_flat_t<uint16_t>(s, (const uint16_t*)values, (const uint16_t*)poles, (const uint16_t*)upper,
                                   (const uint16_t*)lower, n, L, cap, row, seq_stride, seq_size, first_few,
                                   (uint16_t*)recon, mask, scratch_mask);
}

HX_API int hx_nuq_dequantize_flat(void* stream, int32_t dtype, const int64_t* codes, const void* outliers,
                                  const uint8_t* mask, const void* poles, int64_t n, int32_t L, void* out,
                                  uint32_t* dev_err) {
  if (n < 0 || L < 1 || (dtype != 0 && dtype != 1)) return HX_ERR_ARG;
  if (n == 0) return HX_OK;
  if (!codes || !outliers || !mask || !poles || !out) return HX_ERR_ARG;
  unsigned blocks = (unsigned)((n + 255) / 256);
  if (dtype == 0)
    dequant_flat_kernel<float><<<blocks, 256, 0, S_(stream)>>>(codes, (const float*)outliers, mask,
                                                               (const float*)poles, n, L, (float*)out, dev_err);
  else
    dequant_flat_kernel<uint16_t><<<blocks, 256, 0, S_(stream)>>>(codes, (const uint16_t*)outliers, mask,
                                                                  (const uint16_t*)poles, n, L, (uint16_t*)out,
                                                                  dev_err);
  HX_LAUNCH_CHECK();
  return HX_OK;
}

}  // extern "C"
