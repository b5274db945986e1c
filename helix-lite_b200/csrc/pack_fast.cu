// Kernel A, bandwidth path: quantise + bit-pack + outlier lists + K page stats
// for 16-token pages of 128 channels, and the code-threshold tables it reads.
//
// Codes follow the reference's scan exactly: argmin_l |fp32(x) - fp32(p_l)|,
// strict <, the first level winning ties, starting from +inf with pole 0
// (xFuzzitx/helix-lite src/kvquant/compact_pool.py:258-268, the per-token V
// kernel :190-212, triton_batched.py:65-72). Instead of scanning L levels per
// element, the kernel compares the fp16 element with L - 1 decision
// thresholds of its codebook row by bisection on fp16 pairs:
//
//   P_l(x) = |x - p_{l+1}| < |x - p_l|   (fp32, exactly as the scan rounds)
//   t_l    = the largest fp16 x with P_l(x) false, found by bisection over
//            the fp16 values between p_l and p_{l+1}
//   code   = #{l : x > t_l}
//
// This equals the scan whenever the P_l hold for a prefix of l and each P_l
// is false below t_l and true above it. Both hold for a row whose poles are
// finite and strictly increasing, for every x below the row's bound X =
// p_0 + g * 2^22 (g = the smallest gap between poles): there |x - p_l| is
// rounded by less than g / 2, so two poles never round to equal distances.
// hx_scales_prepare writes t_0 .. t_14 and X (entry 15) per row; a row that
// is not strictly increasing and finite gets X = -inf. An element with
// !(x < X) (at or above the bound, +inf, NaN) takes the scan itself, in fp32
// from the poles, so every code is the reference's.
#include "common.cuh"

namespace hx {

constexpr uint16_t kH16PosInf = 0x7C00u, kH16NegInf = 0xFC00u;
constexpr uint32_t kPageLock = 0x80000000u;  // in the K directory record's `rows` word

// order-preserving key of an fp16 bit pattern (finite and inf; -0 < +0)
HX_DEVINL uint32_t h16_key(uint32_t b) { return (b & 0x8000u) ? (0x7FFFu - (b & 0x7FFFu)) : (0x8000u + b); }
HX_DEVINL uint32_t h16_from_key(uint32_t k) { return k >= 0x8000u ? (k - 0x8000u) : (0x8000u | (0x7FFFu - k)); }

// The reference's decision between adjacent levels: level l + 1 strictly closer.
HX_DEVINL bool prefers_next(float x, float pl, float pn) { return fabsf(__fsub_rn(x, pn)) < fabsf(__fsub_rn(x, pl)); }

// Thresholds of one codebook row (L poles, fp16) -> out[0..15] fp16 bit patterns.
HX_DEVINL void row_thresholds(const uint16_t* poles, int L, uint16_t (&out)[16]) {
  float p[16];
  bool ok = L >= 1 && L <= 16;
#pragma unroll
  for (int l = 0; l < 16; ++l) {
    p[l] = l < L ? h2f(poles[l]) : 0.0f;
    if (l < L) ok = ok && isfinite(p[l]);
  }
  float gap = __int_as_float(0x7f800000);
#pragma unroll
  for (int l = 0; l + 1 < 16; ++l)
    if (l + 1 < L) {
      ok = ok && p[l] < p[l + 1];
      gap = fminf(gap, __fsub_rd(p[l + 1], p[l]));  // rounded down: a lower bound of the gap
    }
#pragma unroll
  for (int l = 0; l < 15; ++l) out[l] = kH16PosInf;
  if (!ok) {
    out[15] = kH16NegInf;  // every element of this row takes the scan
    return;
  }
  // bound below which no two poles round to equal distances; rounded down
  const float X = L >= 2 ? __fadd_rd(p[0], __fmul_rd(gap, 4194304.0f)) : __int_as_float(0x7f800000);
  out[15] = X > 65504.0f ? kH16PosInf : __half_as_ushort(__float2half_rd(X));
#pragma unroll
  for (int l = 0; l + 1 < 16; ++l) {
    if (l + 1 >= L) break;
    // P_l is false at p_l and true at p_{l+1}; bisect the fp16 keys between
    uint32_t lo = h16_key(poles[l]), hi = h16_key(poles[l + 1]);
    for (int it = 0; it < 17 && hi - lo > 1; ++it) {
      const uint32_t mid = (lo + hi) >> 1;
      const float x = h2f((uint16_t)h16_from_key(mid));
      if (prefers_next(x, p[l], p[l + 1])) hi = mid;
      else lo = mid;
    }
    out[l] = (uint16_t)h16_from_key(lo);
  }
}

// mode 0: K rows (H*D rows, channel pairs packed as half2: out (H, D/2, 16) u32,
// half e of entry l of pair P is channel 2P + e); mode 1: V rows (H*Tc rows,
// out (rows, 16) u32 with the threshold in both halves).
__global__ void scales_prepare_kernel(int mode, const uint16_t* poles, int64_t rows, int L, uint32_t* out) {
  const int64_t r = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (r >= rows) return;
  uint16_t t[16];
  row_thresholds(poles + r * L, L, t);
  if (mode == 0) {
    uint16_t* o16 = reinterpret_cast<uint16_t*>(out);
    const int64_t pair = r >> 1, e = r & 1;
#pragma unroll
    for (int l = 0; l < 16; ++l) o16[(pair * 16 + l) * 2 + e] = t[l];
  } else {
#pragma unroll
    for (int l = 0; l < 16; ++l) out[r * 16 + l] = (uint32_t)t[l] * 0x00010001u;
  }
}

// ---- fp16-pair helpers ---------------------------------------------------------

HX_DEVINL uint32_t as_u32(__half2 v) { return *reinterpret_cast<uint32_t*>(&v); }
HX_DEVINL __half2 as_h2(uint32_t v) { return *reinterpret_cast<__half2*>(&v); }
HX_DEVINL uint32_t gt2(uint32_t a, uint32_t b) { return __hgt2_mask(as_h2(a), as_h2(b)); }
HX_DEVINL uint32_t geu2(uint32_t a, uint32_t b) { return __hgeu2_mask(as_h2(a), as_h2(b)); }
HX_DEVINL uint32_t lt2(uint32_t a, uint32_t b) { return __hlt2_mask(as_h2(a), as_h2(b)); }
// per-bit select: m ? a : b (m is 0xFFFF / 0 per half)
HX_DEVINL uint32_t sel2(uint32_t m, uint32_t a, uint32_t b) { return (a & m) | (b & ~m); }
HX_DEVINL uint32_t umin2(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("min.u16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}
HX_DEVINL uint32_t umax2(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("max.u16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}

// Codes of a pair of elements, one per half (0 .. 15 or 0 .. 3), from the
// thresholds t[0..14] of each half's row (bisection: 4 or 2 compares).
template <int BITS>
HX_DEVINL uint32_t codes2(uint32_t x, const uint32_t (&t)[16]) {
  if (BITS == 4) {
    const uint32_t m3 = gt2(x, t[7]);
    const uint32_t m2 = gt2(x, sel2(m3, t[11], t[3]));
    const uint32_t m1 = gt2(x, sel2(m3, sel2(m2, t[13], t[9]), sel2(m2, t[5], t[1])));
    const uint32_t q = sel2(m3, sel2(m2, sel2(m1, t[14], t[12]), sel2(m1, t[10], t[8])),
                            sel2(m2, sel2(m1, t[6], t[4]), sel2(m1, t[2], t[0])));
    const uint32_t m0 = gt2(x, q);
    return (m3 & 0x00080008u) | (m2 & 0x00040004u) | (m1 & 0x00020002u) | (m0 & 0x00010001u);
  } else {
    const uint32_t m1 = gt2(x, t[1]);
    const uint32_t m0 = gt2(x, sel2(m1, t[2], t[0]));
    return (m1 & 0x00020002u) | (m0 & 0x00010001u);
  }
}

// The reference's scan for one element (poles fp16 in global memory):
// returns the code and the winning pole (0 when no level is closer than +inf).
HX_DEVINL int scan_code(float x, const uint16_t* poles, int L, float& pole) {
  float best = __int_as_float(0x7f800000);
  int idx = 0;
  float bp = 0.0f;
  for (int l = 0; l < L; ++l) {
    const float p = h2f(poles[l]);
    const float d = fabsf(__fsub_rn(x, p));
    if (d < best) {
      best = d;
      idx = l;
      bp = p;
    }
  }
  pole = bp;
  return idx;
}

HX_DEVINL uint16_t half_of(uint32_t v, int e) { return (uint16_t)(e ? (v >> 16) : (v & 0xFFFFu)); }

// Set bits [sh, sh + width) of word wi of a small register array (the index
// is dynamic: a select per word keeps the array in registers).
template <int N>
HX_DEVINL void vw_set(uint32_t (&w)[N], int wi, int sh, uint32_t mask, uint32_t v) {
#pragma unroll
  for (int q = 0; q < N; ++q)
    if (q == wi) w[q] = (w[q] & ~(mask << sh)) | (v << sh);
}

struct ListRec {  // directory record of one (head, page, K|V)
  uint32_t off, cap, cnt, rows;
};

// Drop the entries of slots [s0, s1) from a list (an overwrite), keeping the rest.
HX_DEVINL uint32_t list_filter(uint32_t* arena, const ListRec& L, int s0, int s1) {
  const int lane = lane_id();
  uint32_t out = 0;
  for (uint32_t base = 0; base < L.cnt; base += 32) {
    const uint32_t i = base + lane;
    uint32_t e = 0;
    bool keep = false;
    if (i < L.cnt) {
      e = __ldcg(arena + L.off + i);
      const int s = (e >> 24) & 31;
      keep = s < s0 || s >= s1;
    }
    const uint32_t m = __ballot_sync(0xffffffffu, keep);
    __syncwarp();
    if (keep) arena[L.off + out + __popc(m & ((1u << lane) - 1))] = e;
    out += __popc(m);
    __syncwarp();
  }
  return out;
}

// Grow two lists at once (whole warp; one arena reservation for both). A list
// whose growth does not fit the arena keeps its old chunk and reports !ok
// (flagged); its new entries are dropped.
HX_DEVINL void lists_reserve(const hx_pool_layer& pool, ListRec& A, uint32_t need_a, ListRec& B, uint32_t need_b,
                             bool& ok_a, bool& ok_b, uint32_t* err) {
  const int lane = lane_id();
  const uint32_t ca = need_a > A.cap ? max(max((need_a + 7u) & ~7u, 2u * A.cap), 16u) : 0u;
  const uint32_t cb = need_b > B.cap ? max(max((need_b + 7u) & ~7u, 2u * B.cap), 16u) : 0u;
  ok_a = ok_b = true;
  if (ca + cb == 0u) return;
  uint32_t off = 0, ok = 0;
  if (lane == 0) {
    off = atomicAdd(pool.arena_top, ca + cb);
    ok = ((int64_t)off + ca + cb <= pool.arena_capacity) ? 1u : 0u;
    if (!ok) set_err(err, HX_DEV_ERR_ARENA_FULL);
  }
  ok = __shfl_sync(0xffffffffu, ok, 0);
  off = __shfl_sync(0xffffffffu, off, 0);
  if (!ok) {
    ok_a = ca == 0u;
    ok_b = cb == 0u;
    return;
  }
  if (ca) {
    for (uint32_t i = lane; i < A.cnt; i += 32) pool.arena[off + i] = __ldcg(pool.arena + A.off + i);
    A.off = off;
    A.cap = ca;
  }
  if (cb) {
    for (uint32_t i = lane; i < B.cnt; i += 32) pool.arena[off + ca + i] = __ldcg(pool.arena + B.off + i);
    B.off = off + ca;
    B.cap = cb;
  }
  __syncwarp();
}

// fp16 of channel 4 lane + k of batch token j from the K registers (static
// indexing: a select per token keeps the array in registers)
HX_DEVINL uint16_t kval8(const uint2 (&xk)[8], int j, int k) {
  uint32_t w = 0;
#pragma unroll
  for (int jj = 0; jj < 8; ++jj)
    if (jj == j) w = k < 2 ? xk[jj].x : xk[jj].y;
  return half_of(w, k & 1);
}

// fp16 of channel b of this lane's V half row
HX_DEVINL uint16_t vval(const uint4 (&xv)[8], int b) {
  const int u = b >> 3, comp = (b >> 1) & 3;
  uint32_t w = 0;
#pragma unroll
  for (int uu = 0; uu < 8; ++uu)
    if (uu == u) w = comp == 0 ? xv[uu].x : comp == 1 ? xv[uu].y : comp == 2 ? xv[uu].z : xv[uu].w;
  return half_of(w, b & 1);
}

HX_DEVINL int warp_excl_scan(int v, int& total) {
  const int lane = lane_id();
  int x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  total = __shfl_sync(0xffffffffu, x, 31);
  return x - v;
}

// Page lock: the K record's rows word carries kPageLock while one warp updates
// the page's lists and stats. Spins are bounded; false = gave up (flagged).
HX_DEVINL bool page_lock(uint32_t* rows_word, uint32_t* err) {
  uint32_t got = 0;
  if (lane_id() == 0) {
    for (uint32_t it = 0; it < (1u << 20); ++it) {
      if ((atomicOr(rows_word, kPageLock) & kPageLock) == 0u) {
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

// ---- the kernel -----------------------------------------------------------------
//
// One warp per (window of 16 input tokens, head). A run is a maximal stretch
// of input tokens filling consecutive slots of one page; each run starting in
// the window is processed whole (it may reach past the window's end). Tokens of
// a page may come in any order: a page that gets several runs in one launch is
// updated by one run at a time (page lock), so no list entry or stat is lost.
//
// K: lane l owns channels 4l .. 4l+3 over the run's tokens (thresholds per
// channel pair in registers; one 8-byte load per token row). V: lane l owns
// half a row (64 channels) of slot l >> 1 (the row's thresholds in registers;
// eight 16-byte loads, one or two 16-byte code stores).
constexpr int PF_D = 128, PF_S = 16;
constexpr int PF_STAGE = 512;  // outlier entries of one run staged in shared memory (more go direct)

template <int BK, int BV>
__global__ void __launch_bounds__(128, 4)
    pack_fast_kernel(const hx_pool_layer pool, const hx_layer_scales sc, const uint16_t* __restrict__ key,
                     const uint16_t* __restrict__ value, const int64_t* __restrict__ slots,
                     const int64_t* __restrict__ abspos, int T, uint32_t* err) {
  constexpr int RBK = PF_D * BK / 8, RBV = PF_D * BV / 8;  // code bytes per token row
  constexpr int SEG = PF_S * (RBK + RBV);
  __shared__ uint32_t s_ent[4][PF_STAGE];  // a run's outlier entries, K's then V's
  const int lane = lane_id();
  uint32_t* sent = s_ent[threadIdx.x >> 5];
  const int H = pool.num_kv_heads, NB = pool.num_blocks, Tc = sc.t_cal;
  const int64_t wg = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int64_t nwin = ((int64_t)T + 15) / 16;
  if (wg >= nwin * H) return;
  const int win = (int)(wg / H), h = (int)(wg % H);
  const int i0 = win * 16;

  // run leaders of the window
  bool lead = false;
  if (lane < 16 && i0 + lane < T) {
    const int64_t s = slots[i0 + lane];
    if (s >= 0) {
      lead = true;
      if (i0 + lane > 0) {
        const int64_t sp = slots[i0 + lane - 1];
        if (sp >= 0 && sp + 1 == s && (s % PF_S) != 0) lead = false;
      }
    }
  }
  uint32_t leaders = __ballot_sync(0xffffffffu, lead);
  if (!leaders) return;

  const int LK = sc.levels_k, LV = sc.levels_v;

  while (leaders) {
    const int r = __ffs(leaders) - 1;
    leaders &= leaders - 1;
    const int i = i0 + r;
    const int64_t s0 = slots[i];
    const int64_t pg64 = s0 / PF_S;
    if (pg64 >= NB) {
      if (lane == 0) set_err(err, HX_DEV_ERR_BOUNDS);
      continue;
    }
    const int pg = (int)pg64, t0 = (int)(s0 % PF_S);
    int n;
    {
      bool ok = false;
      if (lane >= 1 && lane < PF_S - t0 && i + lane < T) ok = slots[i + lane] == s0 + lane;
      const uint32_t m = __ballot_sync(0xffffffffu, ok) | 1u;
      n = __ffs(~m) - 1;
    }
    uint8_t* seg = pool.codes + ((int64_t)h * NB + pg) * SEG;
    uint32_t* dk = pool.dir + (((int64_t)h * NB + pg) * 2 + 0) * 4;
    uint32_t* dv = dk + 4;
    uint16_t* st = pool.stats + ((int64_t)h * NB + pg) * 2 * PF_D + 4 * lane;
    // A page that receives one run in this launch (the pre-pass counted the
    // page's runs into the last word of its V record) belongs to this warp
    // alone: its records and stats are read now, beside the data loads, and
    // written back without a lock. A page with several runs is read and
    // written under the page lock at the end.
    const bool excl = __ldcg(dv + 3) == 1u;
    uint4 rk = make_uint4(0u, 0u, 0u, 0u), rv = rk;
    uint2 smin = make_uint2(0u, 0u), smax = smin;
    if (excl) {
      rk = __ldcg(reinterpret_cast<const uint4*>(dk));
      rv = __ldcg(reinterpret_cast<const uint4*>(dv));
      smin = __ldcg(reinterpret_cast<const uint2*>(st));
      smax = __ldcg(reinterpret_cast<const uint2*>(st + PF_D));
    }

    // ---- K: issue the run's row loads, then code them token by token
    // K tables of this lane's channel pairs 2l, 2l+1 (channels 4l .. 4l+3)
    uint32_t ka[16], kb[16];
    {
      const uint4* ta = reinterpret_cast<const uint4*>(sc.k_thresh) + ((int64_t)h * (PF_D / 2) + 2 * lane) * 4;
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        if (BK == 2 && q > 0 && q < 3) continue;
        const uint4 a = __ldg(ta + q), b = __ldg(ta + 4 + q);
        ka[4 * q] = a.x; ka[4 * q + 1] = a.y; ka[4 * q + 2] = a.z; ka[4 * q + 3] = a.w;
        kb[4 * q] = b.x; kb[4 * q + 1] = b.y; kb[4 * q + 2] = b.z; kb[4 * q + 3] = b.w;
      }
    }
    const uint32_t kxa = ka[15], kxb = kb[15];  // bounds of the fast path
    uint32_t kupa, kupb, kloa, klob;
    {
      const uint2 u = *reinterpret_cast<const uint2*>(sc.k_upper + (int64_t)h * PF_D + 4 * lane);
      const uint2 lo = *reinterpret_cast<const uint2*>(sc.k_lower + (int64_t)h * PF_D + 4 * lane);
      kupa = u.x; kupb = u.y; kloa = lo.x; klob = lo.y;
    }
    uint32_t cmina = 0x001F001Fu, cminb = 0x001F001Fu, cmaxa = 0u, cmaxb = 0u;  // code range (+1 for max)
    float emin[4], emax[4];  // outliers and scanned elements, exact values
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      emin[k] = __int_as_float(0x7f800000);
      emax[k] = __int_as_float(0xff800000);
    }
    // two batches of 8 tokens: bit 4 jj + k of kout_b = channel 4 lane + k of
    // token 8 b + jj is an outlier; its entry is staged at kbase_b + rank
    uint32_t kout0 = 0, kout1 = 0;
    int kbase0 = 0, kbase1 = 0, totk = 0;
#pragma unroll 1
    for (int hb = 0; hb < 2; ++hb) {
      const int j0 = 8 * hb;
      if (j0 >= n) break;
      uint2 xk[8];
#pragma unroll
      for (int jj = 0; jj < 8; ++jj)
        xk[jj] = j0 + jj < n
                     ? *reinterpret_cast<const uint2*>(key + ((int64_t)(i + j0 + jj) * H + h) * PF_D + 4 * lane)
                     : make_uint2(0u, 0u);
      uint32_t kout = 0;
#pragma unroll
      for (int jj = 0; jj < 8; ++jj) {
        if (j0 + jj < n) {
          const uint32_t xa = xk[jj].x, xb = xk[jj].y;
          uint32_t ca = codes2<BK>(xa, ka), cb = codes2<BK>(xb, kb);
          const uint32_t oa = gt2(xa, kupa) | lt2(xa, kloa), ob = gt2(xb, kupb) | lt2(xb, klob);
          const uint32_t sa = geu2(xa, kxa), sb = geu2(xb, kxb);
          if (__any_sync(0xffffffffu, (sa | sb) != 0u)) {
            // elements outside the fast range: the reference's scan
#pragma unroll
            for (int k = 0; k < 4; ++k) {
              const uint32_t sm = k < 2 ? sa : sb;
              if (half_of(sm, k & 1)) {
                const uint32_t xw = k < 2 ? xa : xb;
                const float x = h2f(half_of(xw, k & 1));
                float pole;
                const int c = scan_code(x, sc.k_poles + ((int64_t)h * PF_D + 4 * lane + k) * LK, LK, pole);
                const uint32_t sh = (k & 1) ? 16u : 0u;
                if (k < 2) ca = (ca & ~(0xFu << sh)) | ((uint32_t)c << sh);
                else cb = (cb & ~(0xFu << sh)) | ((uint32_t)c << sh);
                const uint32_t om = k < 2 ? oa : ob;
                if (!half_of(om, k & 1)) {  // a scanned non-outlier reconstructs to its pole
                  emin[k] = fminf(emin[k], pole);
                  emax[k] = fmaxf(emax[k], pole);
                }
              }
            }
          }
          // code range of the fast non-outlier elements
          const uint32_t exa = oa | sa, exb = ob | sb;
          cmina = umin2(cmina, ca | (exa & 0x001F001Fu));
          cminb = umin2(cminb, cb | (exb & 0x001F001Fu));
          cmaxa = umax2(cmaxa, (ca + 0x00010001u) & ~exa);
          cmaxb = umax2(cmaxb, (cb + 0x00010001u) & ~exb);
          kout |= ((oa & 1u) | ((oa >> 15) & 2u) | ((ob & 1u) << 2) | ((ob >> 13) & 8u)) << (4 * jj);
          const int tt = t0 + j0 + jj;
          if (BK == 4) {
            const uint32_t w = (ca & 0xFu) | ((ca >> 12) & 0xF0u) | ((cb & 0xFu) << 8) | ((cb >> 4) & 0xF000u);
            *reinterpret_cast<uint16_t*>(seg + tt * RBK + 2 * lane) = (uint16_t)w;
          } else {
            const uint32_t w = (ca & 3u) | ((ca >> 14) & 0xCu) | ((cb & 3u) << 4) | ((cb >> 10) & 0xC0u);
            seg[tt * RBK + lane] = (uint8_t)w;
          }
        }
      }
      // the batch's K entries (lane-major, then token, then channel) staged
      // while the values are in registers; the outliers also enter the stats
      int tb;
      const int base = totk + warp_excl_scan(__popc(kout), tb);
      {
        uint32_t m = kout;
        int q = base;
        while (m) {
          const int b = __ffs(m) - 1;
          m &= m - 1;
          const int jj = b >> 2, k = b & 3;
          const uint16_t xb = kval8(xk, jj, k);
          if (q < PF_STAGE)
            sent[q] = (uint32_t)xb | ((uint32_t)(4 * lane + k) << 16) | ((uint32_t)(t0 + j0 + jj) << 24);
          ++q;
          const float x = h2f(xb);
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            if (kk == k) {
              emin[kk] = fminf(emin[kk], x);
              emax[kk] = fmaxf(emax[kk], x);
            }
        }
      }
      if (hb == 0) {
        kout0 = kout;
        kbase0 = base;
      } else {
        kout1 = kout;
        kbase1 = base;
      }
      totk += tb;
    }

    // ---- V: lane = (slot t, half row hf); the row's thresholds in registers
    const int t = lane >> 1, hf = lane & 1;
    const bool vact = t >= t0 && t < t0 + n;
    const int iv = i + (t - t0);
    uint64_t voutm = 0;
    uint4 xv[8];
    uint32_t tv[16], vup = 0, vlo = 0;
    int vrow = 0;
    if (vact) {
      const uint4* src = reinterpret_cast<const uint4*>(value + ((int64_t)iv * H + h) * PF_D + 64 * hf);
#pragma unroll
      for (int u = 0; u < 8; ++u) xv[u] = src[u];
      int64_t p = abspos[iv];
      if (p < 0) {
        set_err(err, HX_DEV_ERR_BOUNDS);
        p = 0;
      }
      vrow = (int)(p < Tc ? p : Tc - 1);
      const int64_t rr = (int64_t)h * Tc + vrow;
      const uint4* tr = reinterpret_cast<const uint4*>(sc.v_thresh) + rr * 4;
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        if (BV == 2 && q > 0 && q < 3) continue;
        const uint4 a = __ldg(tr + q);
        tv[4 * q] = a.x; tv[4 * q + 1] = a.y; tv[4 * q + 2] = a.z; tv[4 * q + 3] = a.w;
      }
      vup = (uint32_t)sc.v_upper[rr] * 0x00010001u;
      vlo = (uint32_t)sc.v_lower[rr] * 0x00010001u;
    } else {
#pragma unroll
      for (int u = 0; u < 8; ++u) xv[u] = make_uint4(0u, 0u, 0u, 0u);
#pragma unroll
      for (int q = 0; q < 16; ++q) tv[q] = 0u;
    }
    const uint32_t vx = tv[15];
    uint32_t vw[8];  // nuq4: 8 words (32 B); nuq2: words 0..3 (16 B)
    {
      uint64_t vslow = 0;
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const uint32_t xx[4] = {xv[u].x, xv[u].y, xv[u].z, xv[u].w};
        uint32_t w = 0;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const uint32_t c = codes2<BV>(xx[k], tv);
          if (BV == 4) w |= ((c & 0xFu) | ((c >> 12) & 0xF0u)) << (8 * k);
          else w |= ((c & 3u) | ((c >> 14) & 0xCu)) << (4 * k);
          const uint32_t o = gt2(xx[k], vup) | lt2(xx[k], vlo);
          const uint32_t sl = geu2(xx[k], vx);
          voutm |= (uint64_t)((o & 1u) | ((o >> 15) & 2u)) << (8 * u + 2 * k);
          vslow |= (uint64_t)((sl & 1u) | ((sl >> 15) & 2u)) << (8 * u + 2 * k);
        }
        if (BV == 4) vw[u] = w;
        else if (u & 1) vw[u >> 1] |= w << 16;
        else vw[u >> 1] = w;
      }
      if (!vact) voutm = vslow = 0;
      if (__any_sync(0xffffffffu, vslow != 0)) {
        // elements outside the fast range: the reference's scan, patched into the words
        const uint16_t* prow = sc.v_poles + ((int64_t)h * Tc + vrow) * LV;
        uint64_t m = vslow;
        while (m) {
          const int b = __ffsll((long long)m) - 1;  // channel 8u + 2k + e of the half row
          m &= m - 1;
          float pole;
          const int c = scan_code(h2f(value[((int64_t)iv * H + h) * PF_D + 64 * hf + b]), prow, LV, pole);
          if (BV == 4) {
            const int wi = b >> 3, sh = 4 * (b & 7);
            vw_set(vw, wi, sh, 0xFu, (uint32_t)c);
          } else {
            const int wi = b >> 4, sh = 2 * (b & 15);
            vw_set(vw, wi, sh, 0x3u, (uint32_t)c);
          }
        }
      }
    }
    if (vact) {
      uint4* dst = reinterpret_cast<uint4*>(seg + PF_S * RBK + t * RBV + hf * (RBV / 2));
      dst[0] = make_uint4(vw[0], vw[1], vw[2], vw[3]);
      if (BV == 4) dst[1] = make_uint4(vw[4], vw[5], vw[6], vw[7]);
    }

    // V entries (lane-major = slot, then channel), staged after K's
    int totv;
    const int basev = warp_excl_scan(__popcll(voutm), totv);
    {
      uint64_t m = voutm;
      int q = totk + basev;
      while (m) {
        const int b = __ffsll((long long)m) - 1;
        m &= m - 1;
        if (q < PF_STAGE) sent[q] = (uint32_t)vval(xv, b) | ((uint32_t)(64 * hf + b) << 16) | ((uint32_t)t << 24);
        ++q;
      }
    }

    // ---- page lists and stats
    if (!excl) {
      if (!page_lock(dk + 3, err)) continue;
      rk = __ldcg(reinterpret_cast<const uint4*>(dk));
      rv = __ldcg(reinterpret_cast<const uint4*>(dv));
      smin = __ldcg(reinterpret_cast<const uint2*>(st));
      smax = __ldcg(reinterpret_cast<const uint2*>(st + PF_D));
    }
    ListRec LKr = {rk.x, rk.y, rk.z, rk.w & ~kPageLock}, LVr = {rv.x, rv.y, rv.z, 0u};
    if ((int)LKr.rows > t0) {  // an overwrite: drop the old entries of these slots
      LKr.cnt = list_filter(pool.arena, LKr, t0, t0 + n);
      LVr.cnt = list_filter(pool.arena, LVr, t0, t0 + n);
    }
    bool okk, okv;
    lists_reserve(pool, LKr, LKr.cnt + totk, LVr, LVr.cnt + totv, okk, okv, err);
    __syncwarp();
    {
      // staged entries, coalesced
      const int ns = min(totk + totv, PF_STAGE);
      uint32_t* dk_e = pool.arena + LKr.off + LKr.cnt;
      uint32_t* dv_e = pool.arena + LVr.off + LVr.cnt - totk;
      for (int q = lane; q < ns; q += 32) {
        const uint32_t e = sent[q];
        if (q < totk) {
          if (okk) dk_e[q] = e;
        } else if (okv) {
          dv_e[q] = e;
        }
      }
      if (totk + totv > PF_STAGE) {  // entries past the staging buffer: rebuilt from the inputs
#pragma unroll
        for (int hb = 0; hb < 2; ++hb) {
          uint32_t m = hb ? kout1 : kout0;
          int q = hb ? kbase1 : kbase0;
          while (m) {
            const int b = __ffs(m) - 1;
            m &= m - 1;
            if (q >= PF_STAGE && okk) {
              const int j = 8 * hb + (b >> 2), c = 4 * lane + (b & 3);
              dk_e[q] = (uint32_t)key[((int64_t)(i + j) * H + h) * PF_D + c] | ((uint32_t)c << 16) |
                        ((uint32_t)(t0 + j) << 24);
            }
            ++q;
          }
        }
        uint64_t m = voutm;
        int q = totk + basev;
        while (m) {
          const int b = __ffsll((long long)m) - 1;
          m &= m - 1;
          if (q >= PF_STAGE && okv) {
            const int c = 64 * hf + b;
            dv_e[q] = (uint32_t)value[((int64_t)iv * H + h) * PF_D + c] | ((uint32_t)c << 16) | ((uint32_t)t << 24);
          }
          ++q;
        }
      }
      if (okk) LKr.cnt += totk;
      if (okv) LVr.cnt += totv;
    }
    // K page stats: the run's reconstructed min / max folded into the page's
    {
      uint32_t nmin[2], nmax[2];
      const uint16_t* kp = sc.k_poles + ((int64_t)h * PF_D + 4 * lane) * LK;
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const uint32_t cm = k < 2 ? cmina : cminb, cx = k < 2 ? cmaxa : cmaxb;
        const int lo = half_of(cm, k & 1), hi1 = half_of(cx, k & 1);
        float mn = emin[k], mx = emax[k];
        if (lo < 16) mn = fminf(mn, h2f(kp[k * LK + lo]));
        if (hi1 > 0) mx = fmaxf(mx, h2f(kp[k * LK + hi1 - 1]));
        const float om = h2f(half_of(k < 2 ? smin.x : smin.y, k & 1));
        const float oM = h2f(half_of(k < 2 ? smax.x : smax.y, k & 1));
        const uint16_t rm = mn < om ? f2h(mn) : f2h(om);
        const uint16_t rM = mx > oM ? f2h(mx) : f2h(oM);
        if (k & 1) {
          nmin[k >> 1] |= (uint32_t)rm << 16;
          nmax[k >> 1] |= (uint32_t)rM << 16;
        } else {
          nmin[k >> 1] = rm;
          nmax[k >> 1] = rM;
        }
      }
      *reinterpret_cast<uint2*>(st) = make_uint2(nmin[0], nmin[1]);
      *reinterpret_cast<uint2*>(st + PF_D) = make_uint2(nmax[0], nmax[1]);
    }
    const uint32_t rows_new = max(LKr.rows, (uint32_t)(t0 + n));
    if (excl) {
      if (lane == 0) {
        *reinterpret_cast<uint4*>(dk) = make_uint4(LKr.off, LKr.cap, LKr.cnt, rows_new);
        *reinterpret_cast<uint4*>(dv) = make_uint4(LVr.off, LVr.cap, LVr.cnt, 0u);  // run count back to 0
      }
    } else {
      __threadfence();  // this warp's entries and stats are visible before the page is released
      __syncwarp();
      if (lane == 0) {
        dk[0] = LKr.off; dk[1] = LKr.cap; dk[2] = LKr.cnt;
        dv[0] = LVr.off; dv[1] = LVr.cap; dv[2] = LVr.cnt;
        atomicSub(dv + 3, 1u);  // one run of this page done
        __threadfence();
        atomicExch(dk + 3, rows_new);  // rows, lock bit clear
      }
    }
    __syncwarp();
  }
}

// Pre-pass of hx_pack_append's bandwidth path: count the runs each (head,
// page) receives in this launch into the last word of the page's V record
// (the pack kernel resets it). Same run rule as pack_fast_kernel.
__global__ void pack_count_runs_kernel(const hx_pool_layer pool, const int64_t* __restrict__ slots, int T) {
  const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int H = pool.num_kv_heads;
  if (idx >= (int64_t)T * H) return;
  const int i = (int)(idx / H), h = (int)(idx % H);
  const int64_t s = slots[i];
  if (s < 0) return;
  if (i > 0) {
    const int64_t sp = slots[i - 1];
    if (sp >= 0 && sp + 1 == s && (s % PF_S) != 0) return;
  }
  const int64_t pg = s / PF_S;
  if (pg >= pool.num_blocks) return;
  atomicAdd(pool.dir + (((int64_t)h * pool.num_blocks + pg) * 2 + 1) * 4 + 3, 1u);
}

}  // namespace hx

using namespace hx;

// Launch the bandwidth path; HX_ERR_UNSUPPORTED when the request does not fit it.
int hx_pack_fast_launch(cudaStream_t s, const hx_pool_layer* pool, const hx_layer_scales* sc, const uint16_t* key,
                        const uint16_t* value, const int64_t* slots, const int64_t* abspos, int32_t T,
                        uint32_t* dev_err) {
  if (pool->head_size != PF_D || pool->block_size != PF_S || !sc->k_thresh || !sc->v_thresh) return HX_ERR_UNSUPPORTED;
  if ((reinterpret_cast<uintptr_t>(sc->k_thresh) | reinterpret_cast<uintptr_t>(sc->v_thresh) |
       reinterpret_cast<uintptr_t>(pool->codes) | reinterpret_cast<uintptr_t>(key) |
       reinterpret_cast<uintptr_t>(value) | reinterpret_cast<uintptr_t>(pool->stats) |
       reinterpret_cast<uintptr_t>(pool->dir) | reinterpret_cast<uintptr_t>(sc->k_upper) |
       reinterpret_cast<uintptr_t>(sc->k_lower)) & 15u)
    return HX_ERR_UNSUPPORTED;
  const int64_t warps = ((int64_t)T + 15) / 16 * pool->num_kv_heads;
  const int64_t blocks = (warps + 3) / 4;
  const int64_t cthreads = (int64_t)T * pool->num_kv_heads;
  if (blocks > 0x7fffffff || (cthreads + 255) / 256 > 0x7fffffff) return HX_ERR_ARG;
  pack_count_runs_kernel<<<(unsigned)((cthreads + 255) / 256), 256, 0, s>>>(*pool, slots, T);
  const dim3 grid((unsigned)blocks), block(128);
#define HX_PF(BK_, BV_) pack_fast_kernel<BK_, BV_><<<grid, block, 0, s>>>(*pool, *sc, key, value, slots, abspos, T, dev_err)
  if (pool->bits_k == 4 && pool->bits_v == 4) HX_PF(4, 4);
  else if (pool->bits_k == 4) HX_PF(4, 2);
  else if (pool->bits_v == 4) HX_PF(2, 4);
  else HX_PF(2, 2);
#undef HX_PF
  HX_LAUNCH_CHECK();
  return HX_OK;
}

extern "C" {

HX_API int hx_scales_prepare(void* stream, const hx_layer_scales* sc, int32_t H, int32_t D, uint32_t* k_thresh,
                             uint32_t* v_thresh) {
  if (!sc || !sc->k_poles || !sc->v_poles || H <= 0 || D <= 0 || (D & 1) || !k_thresh || !v_thresh) return HX_ERR_ARG;
  if (sc->levels_k < 1 || sc->levels_k > 16 || sc->levels_v < 1 || sc->levels_v > 16 || sc->t_cal < 1)
    return HX_ERR_ARG;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const int64_t rk = (int64_t)H * D, rv = (int64_t)H * sc->t_cal;
  scales_prepare_kernel<<<(unsigned)((rk + 127) / 128), 128, 0, s>>>(0, sc->k_poles, rk, sc->levels_k, k_thresh);
  scales_prepare_kernel<<<(unsigned)((rv + 127) / 128), 128, 0, s>>>(1, sc->v_poles, rv, sc->levels_v, v_thresh);
  HX_LAUNCH_CHECK();
  return HX_OK;
}

}  // extern "C"
