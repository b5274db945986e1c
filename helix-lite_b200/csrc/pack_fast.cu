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
#include <atomic>

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

// Asynchronous 16- / 8-byte copies global -> shared (no registers held).
HX_DEVINL void cp_async_16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
HX_DEVINL void cp_async_8(void* dst, const void* src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 8;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
HX_DEVINL void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
HX_DEVINL void cp_async_wait_all() { asm volatile("cp.async.wait_group 0;" ::: "memory"); }

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

// fp16 of channel 4 lane + k of batch token j from the registers (static
// indexing: a select per token keeps the array in registers)
template <int BT>
HX_DEVINL uint16_t kval_batch(const uint2 (&xk)[BT], int j, int k) {
  uint32_t w = 0;
#pragma unroll
  for (int jj = 0; jj < BT; ++jj)
    if (jj == j) w = k < 2 ? xk[jj].x : xk[jj].y;
  return half_of(w, k & 1);
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

// Elements of one token's 4 channels (pairs xa, xb) outside the fast range:
// the reference's scan. Returns the code pairs with the scanned codes patched
// in, and per channel the pole a scanned K non-outlier reconstructs to (NaN
// where there is none; it enters the K stats). Out of line: rarely taken.
struct ScanFix {
  uint32_t ca, cb;
  float p0, p1, p2, p3;
};

// Channel k's poles are at pbase + k * pstride (K: one row per channel; V: the
// token's row, pstride 0).
__device__ __noinline__ ScanFix scan_fix(const uint16_t* pbase, int pstride, int L, uint32_t xa, uint32_t xb,
                                         uint32_t sa, uint32_t sb, uint32_t oa, uint32_t ob, uint32_t ca,
                                         uint32_t cb) {
  float pl[4];
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    pl[k] = __int_as_float(0x7fc00000);
    const uint32_t sm = k < 2 ? sa : sb;
    if (half_of(sm, k & 1)) {
      const float xv = h2f(half_of(k < 2 ? xa : xb, k & 1));
      float pole;
      const int c = scan_code(xv, pbase + k * pstride, L, pole);
      const uint32_t sh = (k & 1) ? 16u : 0u;
      if (k < 2) ca = (ca & ~(0xFu << sh)) | ((uint32_t)c << sh);
      else cb = (cb & ~(0xFu << sh)) | ((uint32_t)c << sh);
      if (!half_of(k < 2 ? oa : ob, k & 1)) pl[k] = pole;
    }
  }
  return {ca, cb, pl[0], pl[1], pl[2], pl[3]};
}

// ---- the kernels ----------------------------------------------------------------
//
// Two launches per call, one per list kind (K, then V), after a pre-pass that
// counts the runs each (head, page) receives. One warp per (window of 16
// input tokens, head). A run is a maximal stretch of input tokens filling
// consecutive slots of one page; each run starting in the window is processed
// whole (it may reach past the window's end). One load of the window's slots
// (and positions) gives every run's leader, length and V rows. Per run, one
// round of asynchronous copies brings the run's rows (lane l: channels
// 4l .. 4l+3 of each token), V's threshold rows and, for a page with one run,
// its record and stats into shared memory; then the codes come by bisection
// (K: the thresholds of the lane's channel pairs in registers; V: each token's
// row from shared memory) and each token's packed row is stored (nuq4: two
// bytes per lane, nuq2: one).
//
// Each directory record's last word is rows (bits 0-7, slots written) |
// runs (bits 8-30, this launch's run count from the pre-pass) | lock (bit
// 31). A page with one run belongs to its warp and is written back plainly.
// A page with several runs (tokens of the page not contiguous in the input)
// is updated one run at a time under the record's lock, so no list entry or
// stat is lost; its run count, decremented as runs finish, goes from two to
// zero, so it never reads as a one-run page.
constexpr int PF_D = 128, PF_S = 16;
constexpr int PF_STAGE = PF_S * PF_D;  // one run's outlier entries, staged (every element at worst)
constexpr uint32_t kRunsOne = 1u << 8, kRunsMask = 0x7FFFFF00u, kRowsMask = 0xFFu;

struct __align__(16) PackWarpSmem {
  uint32_t rows[PF_S][PF_D / 2];  // the run's rows of this head (fp16 pairs), lane l at words 2l, 2l+1
  uint32_t vt[PF_S][20];          // V: per slot 16 thresholds + band (80-byte rows)
  uint32_t rec[4];                // an exclusive page's record
  uint32_t st[32][4];             // and its stats: lane l's min (2 words) then max (2 words)
  uint32_t ent[PF_STAGE];         // the run's outlier entries
};

// One (window, head) list kind per warp: `vblock` is the block's index
// among the blocks of its kind.
template <int BITS, bool IS_V>
__device__ __forceinline__ void pack_list_body(const hx_pool_layer& pool, const hx_layer_scales& sc,
                                               const uint16_t* __restrict__ x, const int64_t* __restrict__ slots,
                                               const int64_t* __restrict__ abspos, int T, uint32_t* err,
                                               int64_t vblock) {
  constexpr int RB = PF_D * BITS / 8;  // code bytes per slot
  extern __shared__ __align__(16) uint8_t pf_smem[];  // 4 warps' PackWarpSmem
  const int lane = lane_id(), warp = threadIdx.x >> 5;
  PackWarpSmem& ws = reinterpret_cast<PackWarpSmem*>(pf_smem)[warp];
  const int H = pool.num_kv_heads, NB = pool.num_blocks, Tc = sc.t_cal;
  const int64_t seg_bytes = (int64_t)PF_S * PF_D * (pool.bits_k + pool.bits_v) / 8;
  const int64_t blk_off = IS_V ? (int64_t)PF_S * PF_D * pool.bits_k / 8 : 0;
  const int64_t wg = vblock * (blockDim.x >> 5) + warp;
  const int64_t nwin = ((int64_t)T + 15) / 16;
  if (wg >= nwin * H) return;
  const int win = (int)(wg / H), h = (int)(wg % H);
  const int i0 = win * 16;

  // slots (and V positions) of tokens i0 - 1 .. i0 + 30: lane j holds token i0 - 1 + j
  const int tj = i0 - 1 + lane;
  const int64_t sj = (tj >= 0 && tj < T) ? slots[tj] : -1;
  int64_t pj = 0;
  if (IS_V && tj >= 0 && tj < T) {
    pj = abspos[tj];
    if (pj < 0 && sj >= 0) {
      set_err(err, HX_DEV_ERR_BOUNDS);
      pj = 0;
    }
  }
  const int64_t sprev = __shfl_up_sync(0xffffffffu, sj, 1);
  const bool lead = lane >= 1 && lane <= 16 && sj >= 0 &&
                    !(sprev >= 0 && sprev + 1 == sj && (sj % PF_S) != 0);
  uint32_t leaders = __ballot_sync(0xffffffffu, lead) >> 1;  // bit r: token i0 + r leads a run
  if (!leaders) return;
  const int L = IS_V ? sc.levels_v : sc.levels_k;

  // K: thresholds of channel pairs 2l, 2l+1 (channels 4l .. 4l+3) and the band
  uint32_t ka[16], kb[16], kupa = 0, kupb = 0, kloa = 0, klob = 0;
  if (!IS_V) {
    const uint4* ta = reinterpret_cast<const uint4*>(sc.k_thresh) + ((int64_t)h * (PF_D / 2) + 2 * lane) * 4;
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      if (BITS == 2 && q > 0 && q < 3) continue;
      const uint4 a = __ldg(ta + q), b = __ldg(ta + 4 + q);
      ka[4 * q] = a.x; ka[4 * q + 1] = a.y; ka[4 * q + 2] = a.z; ka[4 * q + 3] = a.w;
      kb[4 * q] = b.x; kb[4 * q + 1] = b.y; kb[4 * q + 2] = b.z; kb[4 * q + 3] = b.w;
    }
    const uint2 u = *reinterpret_cast<const uint2*>(sc.k_upper + (int64_t)h * PF_D + 4 * lane);
    const uint2 lo = *reinterpret_cast<const uint2*>(sc.k_lower + (int64_t)h * PF_D + 4 * lane);
    kupa = u.x; kupb = u.y; kloa = lo.x; klob = lo.y;
  }

  while (leaders) {
    const int r = __ffs(leaders) - 1;
    leaders &= leaders - 1;
    const int i = i0 + r;
    const int64_t s0 = __shfl_sync(0xffffffffu, sj, r + 1);
    const int64_t pg64 = s0 / PF_S;
    if (pg64 >= NB) {
      if (lane == 0) set_err(err, HX_DEV_ERR_BOUNDS);
      continue;
    }
    const int pg = (int)pg64, t0 = (int)(s0 % PF_S);
    int n;
    {  // lanes r + 1 + k, k >= 1, continue the run while their slots follow s0
      const int k = lane - (r + 1);
      const bool ok = k >= 1 && t0 + k < PF_S && sj == s0 + k;
      const uint32_t m = (__ballot_sync(0xffffffffu, ok) >> (r + 1)) | 1u;
      n = __ffs(~m) - 1;
      if (r + 1 + n > 31) n = 31 - r;  // tokens past the loaded ones: the next window's leaders are not affected
    }
    uint8_t* blk = pool.codes + ((int64_t)h * NB + pg) * seg_bytes + blk_off;
    uint32_t* rec = pool.dir + (((int64_t)h * NB + pg) * 2 + (IS_V ? 1 : 0)) * 4;
    uint16_t* st = pool.stats + ((int64_t)h * NB + pg) * 2 * PF_D + 4 * lane;

    // ---- one round of asynchronous copies: rows, V threshold rows, record, stats
    __syncwarp();  // the previous run's readers of the buffers are done
#pragma unroll
    for (int j = 0; j < PF_S; ++j)
      if (j < n) cp_async_8(&ws.rows[j][2 * lane], x + ((int64_t)(i + j) * H + h) * PF_D + 4 * lane);
    uint32_t vband = 0;  // V: lane j's slot band, staged after the copies are issued
    if (IS_V) {
      const int j = lane >> 1, e = lane & 1;
      const int64_t pos = __shfl_sync(0xffffffffu, pj, (r + 1 + j) & 31);
      if (j < n) {
        const int64_t rr = (int64_t)h * Tc + (pos < Tc ? pos : Tc - 1);
        const uint4* tr = reinterpret_cast<const uint4*>(sc.v_thresh) + rr * 4 + 2 * e;
        cp_async_16(&ws.vt[j][8 * e], tr);
        cp_async_16(&ws.vt[j][8 * e + 4], tr + 1);
        vband = e == 0 ? (uint32_t)sc.v_upper[rr] : (uint32_t)sc.v_lower[rr];
      }
    }
    // the record and stats come along whoever owns the page: for a page with
    // one run in this launch (the pre-pass's count) they are this warp's
    if (lane == 0) cp_async_16(ws.rec, rec);
    if (!IS_V) {
      cp_async_8(&ws.st[lane][0], st);
      cp_async_8(&ws.st[lane][2], st + PF_D);
    }
    cp_async_commit();
    if (IS_V) {
      const int j = lane >> 1, e = lane & 1;
      if (j < n) ws.vt[j][16 + e] = vband * 0x00010001u;
    }
    cp_async_wait_all();
    __syncwarp();
    const bool excl = (ws.rec[3] & kRunsMask) == kRunsOne;

    uint32_t cmina = 0x001F001Fu, cminb = 0x001F001Fu, cmaxa = 0u, cmaxb = 0u;  // K code range (+1 for max)
    float emin[4], emax[4];  // K outliers and scanned elements, exact values
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      emin[k] = __int_as_float(0x7f800000);
      emax[k] = __int_as_float(0xff800000);
    }
    int tot = 0;  // outlier entries staged so far (lane-major within each 8-token batch)
#pragma unroll 1
    for (int hb = 0; hb < 2; ++hb) {
      const int j0 = 8 * hb;
      if (j0 >= n) break;
      uint32_t outm = 0;
#pragma unroll
      for (int jj = 0; jj < 8; ++jj) {
        const int j = j0 + jj;
        if (j < n) {
          const uint2 xr = *reinterpret_cast<const uint2*>(&ws.rows[j][2 * lane]);
          const uint32_t xa = xr.x, xb = xr.y;
          uint32_t ca, cb, oa, ob, sa, sb;
          if (IS_V) {
            const uint32_t* vr = ws.vt[j];
            uint32_t tv[16];
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              if (BITS == 2 && q > 0 && q < 3) continue;
              const uint4 a = reinterpret_cast<const uint4*>(vr)[q];
              tv[4 * q] = a.x; tv[4 * q + 1] = a.y; tv[4 * q + 2] = a.z; tv[4 * q + 3] = a.w;
            }
            const uint32_t vup = vr[16], vlo = vr[17];
            ca = codes2<BITS>(xa, tv);
            cb = codes2<BITS>(xb, tv);
            oa = gt2(xa, vup) | lt2(xa, vlo);
            ob = gt2(xb, vup) | lt2(xb, vlo);
            sa = geu2(xa, tv[15]);
            sb = geu2(xb, tv[15]);
          } else {
            ca = codes2<BITS>(xa, ka);
            cb = codes2<BITS>(xb, kb);
            oa = gt2(xa, kupa) | lt2(xa, kloa);
            ob = gt2(xb, kupb) | lt2(xb, klob);
            sa = geu2(xa, ka[15]);
            sb = geu2(xb, kb[15]);
          }
          if (__any_sync(0xffffffffu, (sa | sb) != 0u)) {
            const uint16_t* pb;
            if (IS_V) {
              int64_t pos = abspos[i + j];
              pos = pos < 0 ? 0 : pos;
              pb = sc.v_poles + ((int64_t)h * Tc + (pos < Tc ? pos : Tc - 1)) * L;
            } else {
              pb = sc.k_poles + ((int64_t)h * PF_D + 4 * lane) * L;
            }
            const ScanFix f = scan_fix(pb, IS_V ? 0 : L, L, xa, xb, sa, sb, oa, ob, ca, cb);
            ca = f.ca;
            cb = f.cb;
            if (!IS_V) {  // fminf / fmaxf ignore the NaN of channels not scanned
              emin[0] = fminf(emin[0], f.p0); emax[0] = fmaxf(emax[0], f.p0);
              emin[1] = fminf(emin[1], f.p1); emax[1] = fmaxf(emax[1], f.p1);
              emin[2] = fminf(emin[2], f.p2); emax[2] = fmaxf(emax[2], f.p2);
              emin[3] = fminf(emin[3], f.p3); emax[3] = fmaxf(emax[3], f.p3);
            }
          }
          if (!IS_V) {  // code range of the fast non-outlier elements
            const uint32_t exa = oa | sa, exb = ob | sb;
            cmina = umin2(cmina, ca | (exa & 0x001F001Fu));
            cminb = umin2(cminb, cb | (exb & 0x001F001Fu));
            cmaxa = umax2(cmaxa, (ca + 0x00010001u) & ~exa);
            cmaxb = umax2(cmaxb, (cb + 0x00010001u) & ~exb);
          }
          outm |= ((oa & 1u) | ((oa >> 15) & 2u) | ((ob & 1u) << 2) | ((ob >> 13) & 8u)) << (4 * jj);
          // the token's packed row: nuq4 bytes 2l, 2l+1; nuq2 byte l
          uint8_t* row = blk + (t0 + j) * RB;
          if (BITS == 4) {
            const uint32_t w = (ca & 0xFu) | ((ca >> 12) & 0xF0u) | ((cb & 0xFu) << 8) | ((cb >> 4) & 0xF000u);
            *reinterpret_cast<uint16_t*>(row + 2 * lane) = (uint16_t)w;
          } else {
            row[lane] = (uint8_t)((ca & 3u) | ((ca >> 14) & 0xCu) | ((cb & 3u) << 4) | ((cb >> 10) & 0xC0u));
          }
        }
      }
      // the batch's entries (lane-major: channel group, then token, then
      // channel) staged; K's also enter the page stats
      int tb;
      const int base = tot + warp_excl_scan(__popc(outm), tb);
      {
        uint32_t m = outm;
        int q = base;
        while (m) {
          const int b = __ffs(m) - 1;
          m &= m - 1;
          const int j = j0 + (b >> 2), k = b & 3;
          const uint16_t xv = reinterpret_cast<const uint16_t*>(&ws.rows[j][2 * lane])[k];
          ws.ent[q++] = (uint32_t)xv | ((uint32_t)(4 * lane + k) << 16) | ((uint32_t)(t0 + j) << 24);
          if (!IS_V) {
            const float xf = h2f(xv);
#pragma unroll
            for (int kk = 0; kk < 4; ++kk)
              if (kk == k) {
                emin[kk] = fminf(emin[kk], xf);
                emax[kk] = fmaxf(emax[kk], xf);
              }
          }
        }
      }
      tot += tb;
    }

    // ---- the page's list (and K stats)
    uint4 rc;
    uint2 smin = make_uint2(0u, 0u), smax = smin;
    if (excl) {
      rc = *reinterpret_cast<const uint4*>(ws.rec);
      if (!IS_V) {
        smin = make_uint2(ws.st[lane][0], ws.st[lane][1]);
        smax = make_uint2(ws.st[lane][2], ws.st[lane][3]);
      }
    } else {
      if (!page_lock(rec + 3, err)) continue;
      rc = __ldcg(reinterpret_cast<const uint4*>(rec));
      if (!IS_V) {
        smin = __ldcg(reinterpret_cast<const uint2*>(st));
        smax = __ldcg(reinterpret_cast<const uint2*>(st + PF_D));
      }
    }
    ListRec LR = {rc.x, rc.y, rc.z, rc.w & kRowsMask};
    if ((int)LR.rows > t0) LR.cnt = list_filter(pool.arena, LR, t0, t0 + n);  // an overwrite
    bool ok;
    {
      ListRec none = {0u, 0u, 0u, 0u};
      bool ok2;
      lists_reserve(pool, LR, LR.cnt + tot, none, 0u, ok, ok2, err);
    }
    __syncwarp();
    if (ok) {
      uint32_t* de = pool.arena + LR.off + LR.cnt;
      for (int q = lane; q < tot; q += 32) de[q] = ws.ent[q];
      LR.cnt += tot;
    }
    if (!IS_V) {  // K page stats: the run's reconstructed min / max folded into the page's
      uint32_t nmin[2], nmax[2];
      const uint16_t* kp = sc.k_poles + ((int64_t)h * PF_D + 4 * lane) * L;
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const uint32_t cm = k < 2 ? cmina : cminb, cx = k < 2 ? cmaxa : cmaxb;
        const int lo = half_of(cm, k & 1), hi1 = half_of(cx, k & 1);
        float mn = emin[k], mx = emax[k];
        if (lo < 16) mn = fminf(mn, h2f(kp[k * L + lo]));
        if (hi1 > 0) mx = fmaxf(mx, h2f(kp[k * L + hi1 - 1]));
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
    const uint32_t rows_new = max(LR.rows, (uint32_t)(t0 + n));
    if (excl) {
      if (lane == 0) *reinterpret_cast<uint4*>(rec) = make_uint4(LR.off, LR.cap, LR.cnt, rows_new);  // runs, lock 0
    } else {
      __threadfence();  // this warp's entries and stats are visible before the page is released
      __syncwarp();
      if (lane == 0) {
        rec[0] = LR.off;
        rec[1] = LR.cap;
        rec[2] = LR.cnt;
        // A page with several runs never shows exactly one run while it is in
        // use: a run that reads one treats the page as its own and writes its
        // record and stats back from the copies it made without the lock, and
        // those copies may predate another run's release. So the count goes
        // from two straight to zero (and stays zero), and a run that reads zero
        // or two or more takes the lock.
        const uint32_t w = __ldcg(rec + 3);
        const uint32_t runs = (w & kRunsMask) > 2u * kRunsOne ? (w & kRunsMask) - kRunsOne : 0u;
        __threadfence();
        atomicExch(rec + 3, rows_new | runs);  // one run of this page done, lock clear
      }
    }
    __syncwarp();
  }
}

// Pre-pass of hx_pack_append's bandwidth path: count the runs each (head,
// page) receives in this launch into its K and V records (bits 8-30 of the
// last word; the pack kernels take them out again). Same run rule as the
// pack kernels.
// One list kind per launch (large appends: K, then V).
template <int BITS, bool IS_V>
__global__ void __launch_bounds__(128, 4)
    pack_list_kernel(const hx_pool_layer pool, const hx_layer_scales sc, const uint16_t* __restrict__ x,
                     const int64_t* __restrict__ slots, const int64_t* __restrict__ abspos, int T, uint32_t* err) {
  pack_list_body<BITS, IS_V>(pool, sc, x, slots, abspos, T, err, blockIdx.x);
}

// K and V lists in one launch for small appends: even blocks take K
// windows, odd blocks V windows (both kinds are held to 4 blocks an SM by
// their shared memory, so the K path's registers cost the V blocks nothing).
// One launch fewer and V beside K: config 1 (4,096 tokens) 29.7 -> 23.6 us
// on B200. Large appends keep the kinds apart: run side by side on 524,288
// tokens they took 1.36 ms against 1.06 ms one after the other.
template <int BK, int BV>
__global__ void __launch_bounds__(128, 4)
    pack_kv_kernel(const hx_pool_layer pool, const hx_layer_scales sc, const uint16_t* __restrict__ key,
                   const uint16_t* __restrict__ value, const int64_t* __restrict__ slots,
                   const int64_t* __restrict__ abspos, int T, uint32_t* err) {
  if (blockIdx.x & 1) pack_list_body<BV, true>(pool, sc, value, slots, abspos, T, err, blockIdx.x >> 1);
  else pack_list_body<BK, false>(pool, sc, key, slots, abspos, T, err, blockIdx.x >> 1);
}

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
  uint32_t* rec = pool.dir + ((int64_t)h * pool.num_blocks + pg) * 8;
  atomicAdd(rec + 3, kRunsOne);
  atomicAdd(rec + 7, kRunsOne);
}

}  // namespace hx

using namespace hx;

// Launch the bandwidth path; HX_ERR_UNSUPPORTED when the request does not fit it.
constexpr int kPackMergeMaxTokens = 32768;  // appends up to this size take the one-launch K + V kernel

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
  if (2 * blocks > 0x7fffffff || (cthreads + 255) / 256 > 0x7fffffff) return HX_ERR_ARG;
  const size_t smem = 4 * sizeof(PackWarpSmem);
  {
    // once per device: the kernels' dynamic shared memory above the default 48 KB
    static std::atomic<bool> attr_set[64];
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return HX_ERR_LAUNCH;
    if (!attr_set[dev].load(std::memory_order_acquire)) {
      if (cudaFuncSetAttribute(pack_list_kernel<4, false>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) ||
          cudaFuncSetAttribute(pack_list_kernel<2, false>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) ||
          cudaFuncSetAttribute(pack_list_kernel<4, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) ||
          cudaFuncSetAttribute(pack_list_kernel<2, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) ||
          cudaFuncSetAttribute(pack_kv_kernel<4, 4>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) ||
          cudaFuncSetAttribute(pack_kv_kernel<4, 2>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) ||
          cudaFuncSetAttribute(pack_kv_kernel<2, 4>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) ||
          cudaFuncSetAttribute(pack_kv_kernel<2, 2>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem))
        return HX_ERR_LAUNCH;
      attr_set[dev].store(true, std::memory_order_release);
    }
  }
  pack_count_runs_kernel<<<(unsigned)((cthreads + 255) / 256), 256, 0, s>>>(*pool, slots, T);
  const dim3 block(128);
  if (T > kPackMergeMaxTokens) {
    const dim3 grid((unsigned)blocks);
    if (pool->bits_k == 4) pack_list_kernel<4, false><<<grid, block, smem, s>>>(*pool, *sc, key, slots, abspos, T, dev_err);
    else pack_list_kernel<2, false><<<grid, block, smem, s>>>(*pool, *sc, key, slots, abspos, T, dev_err);
    if (pool->bits_v == 4) pack_list_kernel<4, true><<<grid, block, smem, s>>>(*pool, *sc, value, slots, abspos, T, dev_err);
    else pack_list_kernel<2, true><<<grid, block, smem, s>>>(*pool, *sc, value, slots, abspos, T, dev_err);
    HX_LAUNCH_CHECK();
    return HX_OK;
  }
  const dim3 grid((unsigned)(2 * blocks));
  if (pool->bits_k == 4 && pool->bits_v == 4)
    pack_kv_kernel<4, 4><<<grid, block, smem, s>>>(*pool, *sc, key, value, slots, abspos, T, dev_err);
  else if (pool->bits_k == 4)
    pack_kv_kernel<4, 2><<<grid, block, smem, s>>>(*pool, *sc, key, value, slots, abspos, T, dev_err);
  else if (pool->bits_v == 4)
    pack_kv_kernel<2, 4><<<grid, block, smem, s>>>(*pool, *sc, key, value, slots, abspos, T, dev_err);
  else
    pack_kv_kernel<2, 2><<<grid, block, smem, s>>>(*pool, *sc, key, value, slots, abspos, T, dev_err);
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
