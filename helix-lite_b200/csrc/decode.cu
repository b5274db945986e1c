// Kernel C: fused-dequant split-KV decode attention over the compact pool,
// the cross-shard (o, lse) merge, and the dense selected_attention API.
//
// Replaces KVQuantCompactImpl.forward's unpack_to_staging + FlashAttention
// (xFuzzitx/helix-lite src/kvquant/compact_backend.py:233-299, kernels
// compact_pool.py:293-395): the selected pages are dequantised on chip and
// never touch HBM as fp16. Attention math follows
// src/quest/reference.py:136-168 (softmax(q.K^T * scale) V, fp32 softmax),
// generalised to grouped-query heads (query head h*G+g reads KV head h).
//
// One CTA = (split, KV head, sequence), 16 warps, one CTA per SM; the CTA's
// pages (a balanced share of the selected list) are dealt to the warps. Each
// warp streams its pages: bulk copies (cp.async.bulk, no multicast) of the
// page's code segment, its outlier entries and, before t_cal, its per-token V
// level rows into a 2-stage buffer; LUT dequant of the 16 x 128 K tile into
// swizzled smem (one prmt-built table address per code), outlier patch,
// ldmatrix + mma.sync (tokens x heads), online softmax in fp32 (exp2 domain;
// the running max moves only when a score passes it by 2^8), P split into
// fp16 hi + lo parts so P.V keeps ~22 bits, V tile the same way, PV with two
// MMAs per m-tile. Warps merge in smem; the last CTA of each (b, h) merges
// the splits.
#include <atomic>

#include "common.cuh"
#include "select.cuh"

namespace hx {

constexpr int DD = 128;          // head_size
constexpr int DS = 16;           // page size (tokens)
constexpr int NW = 16;           // warps per CTA (one CTA per SM, 128 registers a thread)
constexpr int NT = NW * 32;
constexpr int NSTAGE = 2;        // pages in smem per warp (one in flight while one is used)
constexpr int LISTCAP = 512;     // pages gathered per round
constexpr int ENTCAP = 352;      // outlier entries staged per page, K's then V's (nuq2 pages: ~100 + ~150)
constexpr int SEGMAX = DS * DD;  // codes bytes per page segment at 4+4 bits
constexpr int PSZ = 8 * DD + 16; // floats per split partial: O[8][128], m[8], l[8]
constexpr int MAXSPLIT = 1024;   // splits the final merge stages weights for

struct DecodeParams {
  hx_pool_layer pool;
  hx_layer_scales sc;
  const uint16_t* q;
  int B, G;
  float scale_log2;
  const int32_t* bt;
  int bt_stride;
  const int32_t* seq_lens;
  int page_begin, max_pages, sel_mode;
  int vphys;  // V positions from the physical page (HX_VPOS_PHYSICAL)
  int cores;  // QK and PV on CUDA cores (HX_DECODE_CUDA_CORES)
  // fused selection (hx_decode_attn_select): each CTA finds its row's
  // threshold and slice counts from the scores and the level-1 histogram
  int fsel;
  uint32_t* fhist;
  int k_fixed, fnum, fden;
  uint64_t* thresh_out;
  int32_t* slice_out;
  const float* scores;
  const uint64_t* thresh;
  int sinks_req;
  const int32_t* lists;
  int list_stride;
  const int32_t* list_counts;
  int n_splits;
  float* part;
  uint32_t* ctr;
  float* o;
  float* lse;
  uint16_t* out16;
  uint32_t* err;
};

struct __align__(256) WarpSmem {
  uint8_t raw[NSTAGE][SEGMAX];          // code segments
  uint32_t ent[NSTAGE][ENTCAP];         // [stage] K entries, then V entries from a 16-byte boundary
  uint16_t tile[DS * DD];               // dequantised K, then V (swizzled rows)
  alignas(256) uint16_t vlut[DS * 16];  // per-token V levels of the current page (256-aligned)
  alignas(256) uint16_t vp[NSTAGE][DS * 16];  // per-token V levels copied with each page's codes
  uint64_t bar[NSTAGE];
};

struct __align__(256) CtaSmem {
  WarpSmem w[NW];
  alignas(256) uint16_t klut[16 * DD + 64];  // K tables (bank-spread, 256-aligned; layout at the fill)
  alignas(256) uint16_t vtail[16];           // V levels at positions >= t_cal (256-aligned)
  alignas(256) uint32_t vpair[16];           // nuq2: the same as level pairs (entry c0 | c1 << 2)
  alignas(16) uint32_t vplane[8];            // nuq4: the same as byte planes (low bytes, then high; lut8_reg)
  int32_t pages[LISTCAP];
  int32_t phys[LISTCAP];
  uint4 dir[LISTCAP][2];                // K and V directory records of each page
  float colM[8], colL[8];               // per-column max / sum for the merges
  int32_t count;
  int32_t wcount[NW];
  int32_t last;
  int32_t slice0, slice0_off;           // HX_SEL_SLICES: slice holding the CTA's first rank, its offset
};

// LUT dequant helpers. A table of 2-byte levels sits 256-aligned in smem; the
// element's byte (2 * code, with the lane's table-offset low bits OR-ed in)
// replaces the low byte of the table's base address in one prmt, and the
// load carries the per-channel offset as its immediate.
HX_DEVINL uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t r;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(sel));
  return r;
}
HX_DEVINL uint16_t lds16(uint32_t addr) {
  uint16_t v;
  asm volatile("ld.shared.u16 %0, [%1];" : "=h"(v) : "r"(addr));
  return v;
}
// four fp16 at a shared address (8-byte aligned) as floats
HX_DEVINL void lds_h4(uint32_t addr, float (&f)[4]) {
  uint32_t a, b;
  asm volatile("ld.shared.v2.u32 {%0, %1}, [%2];" : "=r"(a), "=r"(b) : "r"(addr));
  const float2 lo = __half22float2(*reinterpret_cast<const __half2*>(&a));
  const float2 hi = __half22float2(*reinterpret_cast<const __half2*>(&b));
  f[0] = lo.x;
  f[1] = lo.y;
  f[2] = hi.x;
  f[3] = hi.y;
}

// 8 levels for 8 consecutive 4-bit codes of word w (channels c0 .. c0+7):
// tab(c) = base + off + TSTRIDE * (c - c0). Only base's low byte is replaced,
// so off (a multiple of the table span, folded into the load's immediate once
// unrolled) must be added after the prmt.
template <int TSTRIDE>
HX_DEVINL uint4 lut8_nib(uint32_t w, uint32_t lowbits, uint32_t base, uint32_t off) {
  const uint32_t lo = ((w << 1) & 0x1E1E1E1Eu) | lowbits;  // 2 * code of nibbles 0, 2, 4, 6
  const uint32_t hi = ((w >> 3) & 0x1E1E1E1Eu) | lowbits;  // nibbles 1, 3, 5, 7
  uint16_t v[8];
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    v[2 * k] = lds16(prmt(lo, base, 0x7650u | k) + off + TSTRIDE * (2 * k));
    v[2 * k + 1] = lds16(prmt(hi, base, 0x7650u | k) + off + TSTRIDE * (2 * k + 1));
  }
  return make_uint4(pack_u16x2(v[0], v[1]), pack_u16x2(v[2], v[3]), pack_u16x2(v[4], v[5]),
                    pack_u16x2(v[6], v[7]));
}

// 8 levels for 8 consecutive 4-bit codes of word w from a 16-entry table held
// in registers as byte planes: lb[k] = the low bytes of levels 4k .. 4k+3, hb[k]
// the high bytes. prmt picks a byte out of 8 by a selector nibble's low three
// bits (bit 3, the sign-replicate flag, is cleared), so each plane half gives
// levels code & 7 and 8 + (code & 7); a second prmt takes byte i from the first
// or the second result by code bit 3, and a third interleaves low and high
// bytes into fp16 pairs. No shared-memory access.
HX_DEVINL uint4 lut8_reg(uint32_t w, const uint32_t (&lb)[4], const uint32_t (&hb)[4]) {
  const uint32_t s = w & 0x77777777u;                  // nibble i: code_i & 7
  const uint32_t t = ((w >> 1) & 0x44444444u) | 0x32103210u;  // nibble i: (i & 3) + 4 (code_i >> 3)
  const uint32_t sh = s >> 16, th = t >> 16;
  const uint32_t lo0 = prmt(prmt(lb[0], lb[1], s), prmt(lb[2], lb[3], s), t);    // low bytes, codes 0..3
  const uint32_t hi0 = prmt(prmt(hb[0], hb[1], s), prmt(hb[2], hb[3], s), t);    // high bytes, codes 0..3
  const uint32_t lo1 = prmt(prmt(lb[0], lb[1], sh), prmt(lb[2], lb[3], sh), th);  // codes 4..7
  const uint32_t hi1 = prmt(prmt(hb[0], hb[1], sh), prmt(hb[2], hb[3], sh), th);
  return make_uint4(prmt(lo0, hi0, 0x5140u), prmt(lo0, hi0, 0x7362u), prmt(lo1, hi1, 0x5140u),
                    prmt(lo1, hi1, 0x7362u));
}

HX_DEVINL void sts128(uint32_t addr, const uint4& v) {
  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w));
}
HX_DEVINL void ldsm_x4(uint32_t (&r)[4], uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
HX_DEVINL void ldsm_x4_trans(uint32_t (&r)[4], uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
HX_DEVINL uint32_t lds32(uint32_t addr) {
  uint32_t v;
  asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(addr));
  return v;
}

// 16 levels for 16 consecutive 2-bit codes of word w from level-pair tables:
// a nibble (two codes) picks one 4-byte entry holding both levels, so each
// load yields two channels. tab(pair n) = base + off + TSTRIDE * n, entry
// 4 * nibble; as in lut8_nib only base's low byte is replaced.
template <int TSTRIDE>
HX_DEVINL void lut8_pair(uint32_t w, uint32_t lowbits, uint32_t base, uint32_t off, uint4& o0, uint4& o1) {
  const uint32_t lo = ((w << 2) & 0x3C3C3C3Cu) | lowbits;  // 4 * low nibble: codes 4k, 4k+1
  const uint32_t hi = ((w >> 2) & 0x3C3C3C3Cu) | lowbits;  // 4 * high nibble: codes 4k+2, 4k+3
  uint32_t v[8];
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    v[2 * k] = lds32(prmt(lo, base, 0x7650u | k) + off + TSTRIDE * (2 * k));
    v[2 * k + 1] = lds32(prmt(hi, base, 0x7650u | k) + off + TSTRIDE * (2 * k + 1));
  }
  o0 = make_uint4(v[0], v[1], v[2], v[3]);
  o1 = make_uint4(v[4], v[5], v[6], v[7]);
}

// 16 levels for 16 consecutive 2-bit codes of word w, as two 8-wide chunks.
template <int TSTRIDE>
HX_DEVINL void lut16_crumb(uint32_t w, uint32_t lowbits, uint32_t base, uint32_t off, uint4& o0,
                           uint4& o1) {
  uint32_t g[4];
  g[0] = ((w << 1) & 0x06060606u) | lowbits;  // crumbs 0, 4, 8, 12
  g[1] = ((w >> 1) & 0x06060606u) | lowbits;  // crumbs 1, 5, 9, 13
  g[2] = ((w >> 3) & 0x06060606u) | lowbits;  // crumbs 2, 6, 10, 14
  g[3] = ((w >> 5) & 0x06060606u) | lowbits;  // crumbs 3, 7, 11, 15
  uint16_t v[16];
#pragma unroll
  for (int k = 0; k < 4; ++k)
#pragma unroll
    for (int sft = 0; sft < 4; ++sft)
      v[4 * k + sft] = lds16(prmt(g[sft], base, 0x7650u | k) + off + TSTRIDE * (4 * k + sft));
  o0 = make_uint4(pack_u16x2(v[0], v[1]), pack_u16x2(v[2], v[3]), pack_u16x2(v[4], v[5]), pack_u16x2(v[6], v[7]));
  o1 = make_uint4(pack_u16x2(v[8], v[9]), pack_u16x2(v[10], v[11]), pack_u16x2(v[12], v[13]),
                  pack_u16x2(v[14], v[15]));
}

// Tile layout: 16 tokens x 128 channels fp16, 256 bytes a token; 16-byte chunk
// c (channels 8c .. 8c+7) of token t sits at position c ^ (t & 7) ^ 4 (c >> 3)
// of its row. Eight consecutive rows at one chunk (an ldmatrix phase) land in
// 8 distinct bank groups, and so do the dequant stores, where a wavefront's 8
// lanes are tokens 4j .. 4j+3 x both row halves.

// Write a page's outlier values over its dequantised tile: the first nst
// entries from the staging buffer, any past them from the arena.
// An entry is fp16 | channel << 16 | token << 24, so x = en >> 16 holds
// token << 8 | channel and the tile byte offset 256 t + 16 (c ^ (t & 7) ^
// 4 (c >> 3)) + 2 (d & 7) is (x & 0xF00 | 2 x & 0xFE) ^ (x >> 4 & 0x70) ^
// (x & 0x40). The masks keep every offset inside the 4 KB tile; an entry with
// token >= 16 or channel >= 128 (bits 0xF080 of x) is flagged once per tile.
HX_DEVINL void patch_one(uint32_t tile0, uint32_t en, uint32_t& bad) {
  const uint32_t x = en >> 16;
  const uint32_t off = (((x & 0xF00u) | ((x << 1) & 0xFEu)) ^ ((x >> 4) & 0x70u)) ^ (x & 0x40u);
  asm volatile("st.shared.u16 [%0], %1;" ::"r"(tile0 + off), "h"((uint16_t)(en & 0xffffu)));
  bad |= x & 0xF080u;
}
HX_DEVINL void patch_tile(uint32_t tile0, const uint32_t* staged, const uint32_t* spill, uint32_t cnt, uint32_t nst,
                          int lane, uint32_t* err) {
  const uint32_t ns = min(cnt, nst);
  uint32_t bad = 0;
#pragma unroll 1
  for (uint32_t e = lane; e < ns; e += 32) patch_one(tile0, staged[e], bad);
  if (cnt > nst) {  // warp-uniform; entries past the staged ones
#pragma unroll 1
    for (uint32_t e = nst + lane; e < cnt; e += 32) patch_one(tile0, spill[e], bad);
  }
  if (bad) set_err(err, HX_DEV_ERR_BOUNDS);
}

// Entries staged for a page: K's (rounded up to whole 16-byte copies), then
// V's in what room is left; the arena serves the rest.
HX_DEVINL uint32_t stage_k(uint32_t cntk) { return min((cntk + 3u) & ~3u, (uint32_t)ENTCAP); }
HX_DEVINL uint32_t stage_v(uint32_t ek, uint32_t cntv) { return min((cntv + 3u) & ~3u, (uint32_t)ENTCAP - ek); }

// FMA: QK and PV in fp32 FFMA on the CUDA cores instead of mma.sync (the
// same pipeline, dequant, tile and softmax state; the comparison variant).
// FSEL: the fused selection (hx_decode_attn_select) compiled in; the other
// instances carry none of its code.
template <int BK, int BV, bool FMA, bool FSEL>
__global__ void __launch_bounds__(NT, 1) decode_kernel(const DecodeParams p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  CtaSmem& sm = *reinterpret_cast<CtaSmem*>(smem_raw);
  constexpr int NLK = 1 << BK, NLV = 1 << BV;
  if ((smem_u32(smem_raw) & 255u) != 0u) {  // the LUT address trick needs 256-aligned tables
    if (threadIdx.x == 0) set_err(p.err, HX_DEV_ERR_BOUNDS);
    return;
  }
  constexpr int RBK = DD * BK / 8, RBV = DD * BV / 8;
  constexpr int SEG = DS * (RBK + RBV);

  const int split = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int H = p.pool.num_kv_heads;
  const int bh = b * H + h;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int G = p.G;
  const int Tc = p.sc.t_cal;
  const int NB = p.pool.num_blocks;
  pdl_allow_next();

  // ---- per-CTA tables (all of a thread's loads in flight before its stores).
  // nuq4 K: channel d's 16 levels (32 B) at byte 32 d + 32 (d >> 5). nuq2 K:
  // channel pair P = (2P, 2P+1) as 16 level pairs (64 B; entry e holds the
  // levels of codes e & 3 and e >> 2) at byte 64 P + 64 (P >> 5). Either way the
  // tables a dequant load touches at once sit in disjoint bank windows.
  auto kpole = [&](int d, int c) -> uint16_t {
    return c < p.sc.levels_k ? p.sc.k_poles[((int64_t)h * DD + d) * p.sc.levels_k + c] : (uint16_t)0;
  };
  auto vtail_level = [&](int c) -> uint16_t {
    return c < p.sc.levels_v ? p.sc.v_poles[((int64_t)h * Tc + (Tc - 1)) * p.sc.levels_v + c] : (uint16_t)0;
  };
  if (BK == 4) {
    constexpr int PER = (16 * DD + NT - 1) / NT;
    uint16_t kv[PER];
#pragma unroll
    for (int u = 0; u < PER; ++u) {
      const int i = tid + u * NT;
      kv[u] = i < 16 * DD ? kpole(i >> 4, i & 15) : (uint16_t)0;
    }
#pragma unroll
    for (int u = 0; u < PER; ++u) {
      const int i = tid + u * NT, d = i >> 4;
      if (i < 16 * DD) sm.klut[16 * d + 16 * (d >> 5) + (i & 15)] = kv[u];
    }
  } else {
    constexpr int PER = (16 * (DD / 2) + NT - 1) / NT;
    uint32_t kv[PER];
#pragma unroll
    for (int u = 0; u < PER; ++u) {
      const int i = tid + u * NT, P = i >> 4, e = i & 15;
      kv[u] = i < 16 * (DD / 2) ? pack_u16x2(kpole(2 * P, e & 3), kpole(2 * P + 1, e >> 2)) : 0u;
    }
#pragma unroll
    for (int u = 0; u < PER; ++u) {
      const int i = tid + u * NT, P = i >> 4;
      if (i < 16 * (DD / 2)) reinterpret_cast<uint32_t*>(sm.klut)[16 * P + 16 * (P >> 5) + (i & 15)] = kv[u];
    }
  }
  if (tid < NLV) sm.vtail[tid] = vtail_level(tid);
  if (BV == 2 && tid >= 32 && tid < 48) sm.vpair[tid - 32] = pack_u16x2(vtail_level((tid - 32) & 3), vtail_level((tid - 32) >> 2));
  if (BV == 4 && tid >= 64 && tid < 72) {  // plane k: byte i = byte (k >> 2) of level 4 (k & 3) + i
    const int k = tid - 64, sh = 8 * (k >> 2);
    uint32_t v = 0u;
#pragma unroll
    for (int i = 0; i < 4; ++i) v |= (((uint32_t)vtail_level(4 * (k & 3) + i) >> sh) & 0xFFu) << (8 * i);
    sm.vplane[k] = v;
  }
  WarpSmem& ws = sm.w[warp];
  if (lane == 0 && !FSEL) {  // fused selection: after the selection, whose scratch they share
    for (int st = 0; st < NSTAGE; ++st) mbar_init(&ws.bar[st], 1);
    fence_mbar_init();
  }
  // everything above reads calibration tables only; from here on the inputs
  // may come from the kernels before this one
  pdl_wait();
  const int seq_len = p.seq_lens[b];
  const int n = min((seq_len + DS - 1) / DS, p.max_pages);
  // fused selection: the row's exact threshold and the exclusive prefix of
  // its slices' selected counts, computed here by every CTA of the row (the
  // warp buffers are its scratch; the mbarriers are set up afterwards)
  __shared__ int32_t s_soff[FSEL ? fsel::kMaxSlices + 1 : 1];
  uint64_t T_f = 0ull;
  if constexpr (FSEL) {
    fsel::RowSel<NT>& rs = *reinterpret_cast<fsel::RowSel<NT>*>(sm.w);
    const int fs = min(max(p.sinks_req, 0), n);
    const long long kb = p.fden > 0 ? (long long)n * p.fnum / p.fden : (long long)p.k_fixed;
    const long long ke = kb < (long long)(n - fs) ? kb : (long long)(n - fs);
    const int C = p.list_stride - 1;
    T_f = fsel::row_select<NT>(p.scores + (int64_t)bh * p.max_pages, p.fhist + (int64_t)bh * 2 * fsel::kBins, n, fs,
                               (int)(ke > 0 ? ke : 0), C, rs, p.err);
    if (tid < 32) {  // exclusive prefix of the C <= 128 slice counts (one warp)
      uint32_t v[fsel::kMaxSlices / 32];
      uint32_t sum = 0;
#pragma unroll
      for (int q = 0; q < fsel::kMaxSlices / 32; ++q) {
        const int i = (fsel::kMaxSlices / 32) * lane + q;
        v[q] = i < C ? rs.add[i] : 0u;
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
      for (int q = 0; q < fsel::kMaxSlices / 32; ++q) {
        const int i = (fsel::kMaxSlices / 32) * lane + q;
        if (i < C) s_soff[i] = (int32_t)acc;
        acc += v[q];
      }
      if (lane == 31) s_soff[C] = (int32_t)incl;
    }
    __syncthreads();
    if (split == 0) {
      if (tid == 0 && p.thresh_out) p.thresh_out[bh] = T_f;
      if (p.slice_out)
        for (int i = tid; i <= C; i += NT) p.slice_out[(int64_t)bh * (C + 1) + i] = s_soff[i];
    }
    __syncthreads();  // the scratch is free: the warps' mbarriers now
    if (lane == 0) {
      for (int st = 0; st < NSTAGE; ++st) mbar_init(&ws.bar[st], 1);
      fence_mbar_init();
    }
    __syncthreads();
  }
  // HX_SEL_SLICES: the row's slice offsets (exclusive selected counts of the
  // slices of the non-sink pages)
  const bool slices = p.sel_mode == HX_SEL_SLICES;
  const int nsl = slices ? p.list_stride - 1 : 1;
  const int32_t* soff = slices ? (FSEL ? s_soff : p.lists + (int64_t)bh * p.list_stride) : nullptr;
  const int32_t soff_lo = (slices && tid < nsl) ? soff[tid] : 0, soff_hi = (slices && tid < nsl) ? soff[tid + 1] : 0;
  const int32_t soff_all = slices ? soff[nsl] : 0;

  // dequant lanes: token t = lane >> 1, row half = lane & 1; x0 = which
  // 16-byte chunk of its half row (nuq4) the lane reads first is cx0
  const int t = lane >> 1, half = lane & 1, cx0 = (lane >> 2) & 1;
  // Tile byte addresses (the tile is 256-aligned): chunk c of token t is at
  // tile + 256 t + 16 (c ^ (t & 7) ^ 4 (c >> 3)). With c = 8 half + low, a
  // lane's dequant store is tw ^ 16 low, and each ldmatrix phase reads a lane
  // base ^ 16 k(step) with k(s) = 2 s ^ 4 (s >> 2).
  const uint32_t tile0 = smem_u32(ws.tile);
  const uint32_t tw = tile0 + 256u * t + 16u * ((8 * half) ^ (4 * half) ^ (t & 7));
  const uint32_t tw4 = tw ^ (64u * cx0);  // nuq4: chunk order cx0, cx0 ^ 1
  uint32_t tqk, tpv;
  {
    const int rk = (lane & 7) + ((lane >> 3) & 1) * 8, rv = (lane & 7) + ((lane >> 4) & 1) * 8;
    tqk = tile0 + 256u * rk + 16u * ((lane >> 4) ^ (rk & 7));
    tpv = tile0 + 256u * rv + 16u * (((lane >> 3) & 1) ^ (rv & 7));
  }
  // query fragments (B operand, k = channel, n = head column); for FMA the
  // lane's channels 4 lane .. 4 lane + 3 of every head column, as floats
  const int g = lane >> 2, qd = lane & 3;
  uint32_t bq[8][2];
  float qf[8][4];
  if constexpr (FMA) {
#pragma unroll
    for (int c = 0; c < 8; ++c) {
      const int64_t qrow = ((int64_t)b * H * G + (int64_t)h * G + c) * DD + 4 * lane;
#pragma unroll
      for (int i = 0; i < 4; ++i) qf[c][i] = c < G ? __half2float(__ushort_as_half(p.q[qrow + i])) : 0.0f;
    }
  } else {
    const int64_t qrow = ((int64_t)b * H * G + (int64_t)h * G + g) * DD;
#pragma unroll
    for (int ks = 0; ks < 8; ++ks) {
      if (g < G) {
        bq[ks][0] = *reinterpret_cast<const uint32_t*>(p.q + qrow + 16 * ks + 2 * qd);
        bq[ks][1] = *reinterpret_cast<const uint32_t*>(p.q + qrow + 16 * ks + 2 * qd + 8);
      } else {
        bq[ks][0] = 0u;
        bq[ks][1] = 0u;
      }
    }
  }

  float oacc[8][4];
#pragma unroll
  for (int mt = 0; mt < 8; ++mt) oacc[mt][0] = oacc[mt][1] = oacc[mt][2] = oacc[mt][3] = 0.0f;
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.0f, l1 = 0.0f;
  uint32_t phase = 0;     // bit s = parity to wait for on stage s
  uint32_t inflight = 0;  // bit s = a bulk copy into stage s not yet waited for
  bool timed_out = false;

  // ---- split range (over the selected pages' ranks: sinks first, then the
  // selected pages in ascending order)
  const int sinks = min(max(p.sinks_req, 0), n);
  const int sper = n > sinks ? (n - sinks + nsl - 1) / nsl : 1;
  int total;
  if (p.sel_mode == HX_SEL_LIST) total = min(p.list_counts[bh], p.list_stride);
  else if (slices) total = min(sinks + max(soff_all, 0), n);
  else total = n;
  // Split by cost, not by count: a page whose tokens start below t_cal reads
  // per-token V levels and costs about 11/8 of one past it (measured on B200:
  // 18.3 against 13.3 us for the split holding a 128K sequence's first
  // pages). Selected ranks are ascending in the page, so those pages are the
  // first m_tc ranks; m_tc is estimated from the share of the sequence's
  // pages below t_cal (any partition is correct; this one only balances).
  int ra, re;
  {
    const int p_tc = max(0, min(n, (Tc + DS - 1) / DS - p.page_begin));
    const long long m_tc = n > 0 ? min((long long)total, ((long long)total * p_tc + n - 1) / n) : 0ll;
    const long long cost_total = 8ll * total + 3ll * m_tc;
    auto rank_at = [&](long long c) -> int {  // first rank whose cumulative cost reaches c
      if (c <= 11ll * m_tc) return (int)((c + 10) / 11);
      return (int)(m_tc + (c - 11ll * m_tc + 7) / 8);
    };
    ra = min(rank_at(cost_total * split / p.n_splits), total);
    re = min(rank_at(cost_total * (split + 1) / p.n_splits), total);
  }
  const uint64_t T = FSEL ? T_f : ((p.sel_mode == HX_SEL_THRESHOLD || slices) ? p.thresh[bh] : 0ull);
  int j_cur = -1, r_cur = 0;  // HX_SEL_SLICES scan cursor: page, non-sink rank of the next selected page
  const float* sc_bh = p.scores ? p.scores + (int64_t)bh * p.max_pages : nullptr;
  // a page whose 16 tokens all lie before t_cal gets its per-token V levels by
  // bulk copy with its codes when the rows are contiguous and 16-byte aligned
  auto v_rows = [&](int pos0) -> const uint16_t* {
    return p.sc.v_poles + ((int64_t)h * Tc + pos0) * NLV;
  };
  auto v_bulk = [&](int pos0) -> bool {
    return pos0 + DS <= Tc && p.sc.levels_v == NLV && (reinterpret_cast<uintptr_t>(v_rows(pos0)) & 15u) == 0;
  };
  // absolute position of slot 0 of list entry li, clamped to t_cal (every use
  // only compares it with t_cal or reads rows below it): the logical page
  // (page_begin + j) * 16, or with HX_VPOS_PHYSICAL the physical page
  // (page_begin + block_table[j]) * 16, the reference pool's rule that a
  // token's V row is its slot
  auto vpos0 = [&](int li) -> int {
    const int64_t pg = (int64_t)p.page_begin + (p.vphys ? sm.phys[li] : sm.pages[li]);
    return (int)min(pg * DS, (int64_t)Tc);
  };
  __syncthreads();

  for (int rb = ra; rb < re; rb += LISTCAP) {
    const int rend = min(rb + LISTCAP, re);
    if (slices) {
      // the round's pages by rank: sinks are pages 0 .. sinks-1; the rest come
      // from scanning the slices (4 pages a thread per pass) from the cursor
      for (int r = rb + tid; r < rend; r += NT) sm.pages[r - rb] = r < sinks ? r : -1;
      const int nb = max(rb, sinks) - sinks, ne = rend - sinks, c0 = max(0, min(rend, sinks) - rb);
      if (nb < ne) {
        if (j_cur < 0) {  // the slice holding non-sink rank nb
          if (tid == 0) {
            sm.slice0 = 0;
            sm.slice0_off = 0;
          }
          __syncthreads();
          if (tid < nsl && soff_lo <= nb && nb < soff_hi) {
            sm.slice0 = tid;
            sm.slice0_off = soff_lo;
          }
          __syncthreads();
          j_cur = sinks + sm.slice0 * sper;
          r_cur = sm.slice0_off;
        }
        while (r_cur < ne && j_cur < n) {
          const int jt = j_cur + 4 * tid;
          bool f[4];
          int c = 0;
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            f[u] = jt + u < n && order_key64(sc_bh[jt + u], (uint32_t)(jt + u)) >= T;
            c += f[u] ? 1 : 0;
          }
          int incl = c;  // inclusive scan over the warp, then over the warps
#pragma unroll
          for (int o = 1; o < 32; o <<= 1) {
            const int x = __shfl_up_sync(0xffffffffu, incl, o);
            if (lane >= o) incl += x;
          }
          if (lane == 31) sm.wcount[warp] = incl;
          __syncthreads();
          int before = 0, tt = 0;
          for (int w = 0; w < NW; ++w) {
            const int v = sm.wcount[w];
            before += w < warp ? v : 0;
            tt += v;
          }
          int rank = r_cur + before + incl - c;
#pragma unroll
          for (int u = 0; u < 4; ++u)
            if (f[u]) {
              if (rank >= nb && rank < ne) sm.pages[c0 + rank - nb] = jt + u;
              ++rank;
            }
          __syncthreads();  // wcount is reused by the next pass
          if (r_cur + tt > ne) break;  // the next round starts inside this tile
          r_cur += tt;
          j_cur += 4 * NT;
        }
      }
      __syncthreads();
    }
    if (tid == 0) sm.count = 0;
    __syncthreads();
    // gather the round's selected pages (ascending) with their directory records
    for (int base = rb; base < rend; base += NT) {
      int idx = base + tid;
      int j = -1;
      bool sel = false;
      if (idx < rend) {
        j = p.sel_mode == HX_SEL_LIST ? p.lists[(int64_t)bh * p.list_stride + idx]
                                      : (slices ? sm.pages[idx - rb] : idx);
        if (j < 0 || j >= n) {
          if (p.sel_mode == HX_SEL_LIST || slices) set_err(p.err, HX_DEV_ERR_BOUNDS);
        } else if (p.sel_mode == HX_SEL_THRESHOLD) {
          sel = (j < sinks) || order_key64(sc_bh[j], (uint32_t)j) >= T;
        } else {
          sel = true;
        }
      }
      int32_t pp = 0;
      if (sel) {
        pp = p.bt ? p.bt[(int64_t)b * p.bt_stride + j] : j;
        if (pp < 0 || pp >= NB) {
          set_err(p.err, HX_DEV_ERR_BOUNDS);
          sel = false;
        }
      }
      uint4 d0 = make_uint4(0, 0, 0, 0), d1 = d0;
      if (sel) {
        const uint4* dr = reinterpret_cast<const uint4*>(p.pool.dir + ((int64_t)h * NB + pp) * 8);
        d0 = dr[0];
        d1 = dr[1];
      }
      uint32_t m = __ballot_sync(0xffffffffu, sel);
      if (lane == 0) sm.wcount[warp] = __popc(m);
      __syncthreads();
      int off = sm.count;
      for (int w = 0; w < warp; ++w) off += sm.wcount[w];
      if (sel) {
        int pos = off + __popc(m & ((1u << lane) - 1));
        sm.pages[pos] = j;
        sm.phys[pos] = pp;
        sm.dir[pos][0] = d0;
        sm.dir[pos][1] = d1;
      }
      __syncthreads();
      if (tid == 0) {
        int c = sm.count;
        for (int w = 0; w < NW; ++w) c += sm.wcount[w];
        sm.count = c;
      }
      __syncthreads();
    }
    const int cnt = sm.count;
    const int my_n = cnt > warp ? (cnt - warp + NW - 1) / NW : 0;

    // ---- warp pipeline over pages warp, warp + NW, ...
    auto issue = [&](int k) {
      if (timed_out) return;
      const int st = k % NSTAGE;
      inflight |= 1u << st;
      if (lane == 0) {
        const int li = warp + NW * k;
        const int pp = sm.phys[li];
        const uint4 dk = sm.dir[li][0], dv = sm.dir[li][1];
        const uint32_t ek = stage_k(dk.z), ev = stage_v(ek, dv.z);
        const int pos0 = vpos0(li);
        const bool vb = v_bulk(pos0);
        constexpr uint32_t VPB = 2u * DS * NLV;
        fence_proxy_async();
        mbar_arrive_expect_tx(&ws.bar[st], SEG + 4u * (ek + ev) + (vb ? VPB : 0u));
        bulk_g2s(ws.raw[st], p.pool.codes + ((int64_t)h * NB + pp) * SEG, SEG, &ws.bar[st]);
        if (ek) bulk_g2s(ws.ent[st], p.pool.arena + dk.x, 4u * ek, &ws.bar[st]);
        if (ev) bulk_g2s(ws.ent[st] + ek, p.pool.arena + dv.x, 4u * ev, &ws.bar[st]);
        if (vb) bulk_g2s(ws.vp[st], v_rows(pos0), VPB, &ws.bar[st]);
      }
    };

    for (int k = 0; k < NSTAGE - 1 && k < my_n; ++k) issue(k);
    for (int k = 0; k < my_n; ++k) {
      const int st = k % NSTAGE;
      if (k + NSTAGE - 1 < my_n) issue(k + NSTAGE - 1);  // its stage held page k - 1, done
      if (!timed_out) {
        if (mbar_wait(&ws.bar[st], (phase >> st) & 1u)) {
          phase ^= 1u << st;
          inflight &= ~(1u << st);
        } else {
          timed_out = true;
          if (lane == 0) set_err(p.err, HX_DEV_ERR_TIMEOUT);
        }
      }
      if (timed_out) continue;
      const int li = warp + NW * k;
      const uint4 dk = sm.dir[li][0], dv = sm.dir[li][1];
      const uint32_t offk = dk.x, cntk = dk.z, offv = dv.x, cntv = dv.z;
      const int j = sm.pages[li];
      const int pos0 = vpos0(li);
      const int valid = seq_len - j * DS;  // tokens of this page inside the sequence

      // ---- K tile: per-channel tables (lane = token t, half of the channels)
      {
        const uint8_t* rowp = ws.raw[st] + t * RBK + half * (RBK / 2);
        if (BK == 4) {
          // the half row's two 16-byte chunks in the lane's order cx0, cx0 ^ 1, so
          // the 8 lanes of a wavefront read 8 distinct bank groups
          const uint4 ca = *reinterpret_cast<const uint4*>(rowp + 16 * cx0);
          const uint4 cb = *reinterpret_cast<const uint4*>(rowp + 16 * (cx0 ^ 1));
          const uint32_t wv[8] = {ca.x, ca.y, ca.z, ca.w, cb.x, cb.y, cb.z, cb.w};
#pragma unroll
          for (int j = 0; j < 2; ++j) {
            // channels 64 half + 32 x .. +31: tables at klut + 2048 half + 1024 x
            // + 64 half + 32 x (+ 256 per 8 channels); the last term is the low byte
            const int x = cx0 ^ j;
            const uint32_t base = smem_u32(sm.klut) + 2048u * half + 1024u * x;
            const uint32_t low = (64u * half + 32u * x) * 0x01010101u;
#pragma unroll
            for (int i = 0; i < 4; ++i) sts128(tw4 ^ (64u * j + 16u * i), lut8_nib<32>(wv[4 * j + i], low, base, 256u * i));
          }
        } else {
          // pair P = 32 half + 8 w + n at klut + 2048 half + 64 half + 512 w + 64 n
          const uint4 c0 = *reinterpret_cast<const uint4*>(rowp);
          const uint32_t wv[4] = {c0.x, c0.y, c0.z, c0.w};
          const uint32_t base = smem_u32(sm.klut) + 2048u * half, low = 64u * half * 0x01010101u;
#pragma unroll
          for (int w4 = 0; w4 < 4; ++w4) {
            uint4 o0, o1;
            lut8_pair<64>(wv[w4], low, base, 512u * (uint32_t)w4, o0, o1);
            sts128(tw ^ (32u * w4), o0);
            sts128(tw ^ (32u * w4 + 16u), o1);
          }
        }
      }
      __syncwarp();
      const uint32_t ek = stage_k(cntk);  // K entries staged; V's follow them
      patch_tile(tile0, ws.ent[st], p.pool.arena + offk, cntk, ek, lane, p.err);
      __syncwarp();

      // ---- S^T = K . Q^T  (16 tokens x 8 head columns)
      float x0, x1, x2, x3;  // S[g][2qd], S[g][2qd + 1], S[g + 8][2qd], S[g + 8][2qd + 1]
      if constexpr (FMA) {
        // the lane's 4 channels of 2 tokens at a time against its q columns;
        // a halving butterfly sums each (token, column) over the warp and
        // leaves lanes l and l ^ 1 with S[2 grp + (l >> 4)][(l >> 1) & 7]
        float r[8];
#pragma unroll
        for (int grp = 0; grp < 8; ++grp) {
          float a[16];
#pragma unroll
          for (int tt = 0; tt < 2; ++tt) {
            const int tk = 2 * grp + tt;
            const uint32_t c = (uint32_t)lane >> 1;
            float kf[4];
            lds_h4(tile0 + 256u * tk + 16u * (c ^ (uint32_t)(tk & 7) ^ (4u * (c >> 3))) + 8u * (lane & 1), kf);
#pragma unroll
            for (int col = 0; col < 8; ++col)
              a[8 * tt + col] =
                  fmaf(kf[3], qf[col][3], fmaf(kf[2], qf[col][2], fmaf(kf[1], qf[col][1], kf[0] * qf[col][0])));
          }
#pragma unroll
          for (int m = 8; m >= 1; m >>= 1) {  // lane bits 4, 3, 2, 1 take index bits 3, 2, 1, 0
            const bool upper = (lane & (2 * m)) != 0;
#pragma unroll
            for (int i = 0; i < m; ++i) {
              const float send = upper ? a[i] : a[i + m];
              const float keep = upper ? a[i + m] : a[i];
              a[i] = keep + __shfl_xor_sync(0xffffffffu, send, 2 * m);
            }
          }
          r[grp] = a[0] + __shfl_xor_sync(0xffffffffu, a[0], 1);
        }
        // token g is in group g >> 1 (g + 8 in group 4 + (g >> 1)), at lane
        // (g & 1) << 4 | column << 1
        const int src = ((g & 1) << 4) | (qd << 2);
        const int gi = g >> 1;
        float y[4], z[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          y[u] = __shfl_sync(0xffffffffu, r[u], src);
          z[u] = __shfl_sync(0xffffffffu, r[u], src | 2);
        }
        x0 = (gi == 0 ? y[0] : gi == 1 ? y[1] : gi == 2 ? y[2] : y[3]) * p.scale_log2;
        x1 = (gi == 0 ? z[0] : gi == 1 ? z[1] : gi == 2 ? z[2] : z[3]) * p.scale_log2;
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          y[u] = __shfl_sync(0xffffffffu, r[4 + u], src);
          z[u] = __shfl_sync(0xffffffffu, r[4 + u], src | 2);
        }
        x2 = (gi == 0 ? y[0] : gi == 1 ? y[1] : gi == 2 ? y[2] : y[3]) * p.scale_log2;
        x3 = (gi == 0 ? z[0] : gi == 1 ? z[1] : gi == 2 ? z[2] : z[3]) * p.scale_log2;
      } else {
        // two accumulator chains
        float sa[4] = {0.0f, 0.0f, 0.0f, 0.0f}, sb[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
        for (int ks = 0; ks < 8; ++ks) {
          uint32_t a[4];
          ldsm_x4(a, tqk ^ (16u * ((2 * ks) ^ (4 * (ks >> 2)))));
          if (ks & 1) mma_16816(sb, a, bq[ks][0], bq[ks][1]);
          else mma_16816(sa, a, bq[ks][0], bq[ks][1]);
        }
        x0 = (sa[0] + sb[0]) * p.scale_log2;
        x1 = (sa[1] + sb[1]) * p.scale_log2;
        x2 = (sa[2] + sb[2]) * p.scale_log2;
        x3 = (sa[3] + sb[3]) * p.scale_log2;
      }
      // ---- online softmax (exp2 domain); rows = tokens g, g+8; cols = 2qd, 2qd+1
      if (g >= valid) x0 = x1 = -INFINITY;
      if (g + 8 >= valid) x2 = x3 = -INFINITY;
      // the running max moves only when a score passes it by more than 2^8
      const bool grow = fmaxf(x0, x2) > m0 + 8.0f || fmaxf(x1, x3) > m1 + 8.0f;
      if (__any_sync(0xffffffffu, grow)) {
        float mx0 = fmaxf(x0, x2), mx1 = fmaxf(x1, x3);
#pragma unroll
        for (int sft = 4; sft <= 16; sft <<= 1) {
          mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, sft));
          mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, sft));
        }
        const float mn0 = fmaxf(m0, mx0), mn1 = fmaxf(m1, mx1);
        const float al0 = m0 == -INFINITY ? 0.0f : exp2f(m0 - mn0);
        const float al1 = m1 == -INFINITY ? 0.0f : exp2f(m1 - mn1);
        l0 *= al0;
        l1 *= al1;
#pragma unroll
        for (int mt = 0; mt < 8; ++mt) {
          oacc[mt][0] *= al0;
          oacc[mt][1] *= al1;
          oacc[mt][2] *= al0;
          oacc[mt][3] *= al1;
        }
        m0 = mn0;
        m1 = mn1;
      }
      const float bs0 = m0 == -INFINITY ? 0.0f : m0, bs1 = m1 == -INFINITY ? 0.0f : m1;
      const float p0 = exp2f(x0 - bs0), p1 = exp2f(x1 - bs1), p2 = exp2f(x2 - bs0), p3 = exp2f(x3 - bs1);
      l0 += p0 + p2;
      l1 += p1 + p3;
      // P^T as the B operand (k = token, n = head column): hi and lo halves
      uint32_t bh0 = 0u, bh1 = 0u, bl0 = 0u, bl1 = 0u;
      if constexpr (!FMA) {
        const __half h0 = __float2half_rn(p0), h1 = __float2half_rn(p1);
        const __half h2 = __float2half_rn(p2), h3 = __float2half_rn(p3);
        const uint32_t phi_top = pack_u16x2(__half_as_ushort(h0), __half_as_ushort(h1));
        const uint32_t phi_bot = pack_u16x2(__half_as_ushort(h2), __half_as_ushort(h3));
        const uint32_t plo_top = pack_half2(p0 - __half2float(h0), p1 - __half2float(h1));
        const uint32_t plo_bot = pack_half2(p2 - __half2float(h2), p3 - __half2float(h3));
        bh0 = movmatrix_trans(phi_top);
        bh1 = movmatrix_trans(phi_bot);
        bl0 = movmatrix_trans(plo_top);
        bl1 = movmatrix_trans(plo_bot);
      }

      // ---- V tile: per-token LUT (row min(pos, t_cal - 1))
      const bool vshared = pos0 >= Tc;
      uint32_t vbase, vlow;
      if (vshared) {
        vbase = smem_u32(sm.vtail);  // one table for every token
        vlow = 0u;
      } else {
        if (v_bulk(pos0)) {
          vbase = smem_u32(ws.vp[st]);
        } else {
          uint16_t lv[DS * NLV / 32];
#pragma unroll
          for (int u = 0; u < DS * NLV / 32; ++u) {
            const int i = lane + 32 * u;
            const int r = i / NLV, c = i % NLV;
            const int pr = min(pos0 + r, Tc - 1);
            lv[u] = c < p.sc.levels_v ? p.sc.v_poles[((int64_t)h * Tc + pr) * p.sc.levels_v + c] : (uint16_t)0;
          }
#pragma unroll
          for (int u = 0; u < DS * NLV / 32; ++u) ws.vlut[lane + 32 * u] = lv[u];
          __syncwarp();
          vbase = smem_u32(ws.vlut);
        }
        vbase += 2u * NLV * (uint32_t)t;  // token t's table
        vlow = ((2u * NLV * (uint32_t)t) & 0xFFu) * 0x01010101u;
      }
      {
        const uint8_t* rowp = ws.raw[st] + DS * RBK + t * RBV + half * (RBV / 2);
        if (BV == 4) {
          const uint4 ca = *reinterpret_cast<const uint4*>(rowp + 16 * cx0);
          const uint4 cb = *reinterpret_cast<const uint4*>(rowp + 16 * (cx0 ^ 1));
          const uint32_t wv[8] = {ca.x, ca.y, ca.z, ca.w, cb.x, cb.y, cb.z, cb.w};
          if (vshared) {  // one table for every token: byte planes in registers
            const uint4 pl = *reinterpret_cast<const uint4*>(sm.vplane);
            const uint4 ph = *reinterpret_cast<const uint4*>(sm.vplane + 4);
            const uint32_t lb[4] = {pl.x, pl.y, pl.z, pl.w}, hb[4] = {ph.x, ph.y, ph.z, ph.w};
#pragma unroll
            for (int j = 0; j < 2; ++j)
#pragma unroll
              for (int i = 0; i < 4; ++i) sts128(tw4 ^ (64u * j + 16u * i), lut8_reg(wv[4 * j + i], lb, hb));
          } else {
#pragma unroll
            for (int j = 0; j < 2; ++j)
#pragma unroll
              for (int i = 0; i < 4; ++i)
                sts128(tw4 ^ (64u * j + 16u * i), lut8_nib<0>(wv[4 * j + i], vlow, vbase, 0u));
          }
        } else {
          const uint4 c0 = *reinterpret_cast<const uint4*>(rowp);
          const uint32_t wv[4] = {c0.x, c0.y, c0.z, c0.w};
          if (vshared) {  // one level-pair table for every token
            const uint32_t pb = smem_u32(sm.vpair);
#pragma unroll
            for (int w4 = 0; w4 < 4; ++w4) {
              uint4 o0, o1;
              lut8_pair<0>(wv[w4], 0u, pb, 0u, o0, o1);
              sts128(tw ^ (32u * w4), o0);
              sts128(tw ^ (32u * w4 + 16u), o1);
            }
          } else {
#pragma unroll
            for (int w4 = 0; w4 < 4; ++w4) {
              uint4 o0, o1;
              lut16_crumb<0>(wv[w4], vlow, vbase, 0u, o0, o1);
              sts128(tw ^ (32u * w4), o0);
              sts128(tw ^ (32u * w4 + 16u), o1);
            }
          }
        }
      }
      __syncwarp();
      patch_tile(tile0, ws.ent[st] + ek, p.pool.arena + offv, cntv, stage_v(ek, cntv), lane, p.err);
      __syncwarp();

      // ---- O^T += V^T . P^T  (128 channels x 8 head columns)
      if constexpr (FMA) {
        // lane (g, qd) keeps head columns 2qd, 2qd + 1 of channels 32k + 4g + i
        // (k, i < 4) in oacc[q >> 1][2 (q & 1) + column], q = 4k + i; token
        // tk's P comes from lane 4 (tk & 7) + qd (p0, p1 below token 8, else p2, p3)
#pragma unroll 1
        for (int tk = 0; tk < DS; ++tk) {
          const int srcl = 4 * (tk & 7) + qd;
          const float pc0 = __shfl_sync(0xffffffffu, tk < 8 ? p0 : p2, srcl);
          const float pc1 = __shfl_sync(0xffffffffu, tk < 8 ? p1 : p3, srcl);
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const uint32_t c = 4u * k + ((uint32_t)g >> 1);
            float vf[4];
            lds_h4(tile0 + 256u * tk + 16u * (c ^ (uint32_t)(tk & 7) ^ (4u * (c >> 3))) + 8u * (g & 1), vf);
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              const int q = 4 * k + i;
              oacc[q >> 1][2 * (q & 1)] = fmaf(pc0, vf[i], oacc[q >> 1][2 * (q & 1)]);
              oacc[q >> 1][2 * (q & 1) + 1] = fmaf(pc1, vf[i], oacc[q >> 1][2 * (q & 1) + 1]);
            }
          }
        }
      } else {
#pragma unroll
        for (int mt = 0; mt < 8; ++mt) {
          uint32_t a[4];
          ldsm_x4_trans(a, tpv ^ (16u * ((2 * mt) ^ (4 * (mt >> 2)))));
          mma_16816(oacc[mt], a, bh0, bh1);
          mma_16816(oacc[mt], a, bl0, bl1);
        }
      }
      __syncwarp();
    }
    if (timed_out) {
      // give copies still in flight one more bounded wait before the buffers
      // are reused, then stop this warp's work
      for (int st = 0; st < NSTAGE; ++st)
        if ((inflight >> st) & 1u && mbar_wait(&ws.bar[st], (phase >> st) & 1u)) {
          phase ^= 1u << st;
          inflight &= ~(1u << st);
        }
    }
    __syncthreads();
  }

  // ---- warp -> CTA merge (smem reuses the stage buffers)
  l0 += __shfl_xor_sync(0xffffffffu, l0, 4);
  l0 += __shfl_xor_sync(0xffffffffu, l0, 8);
  l0 += __shfl_xor_sync(0xffffffffu, l0, 16);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 4);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 8);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 16);
  float* wO = reinterpret_cast<float*>(ws.raw);     // [8][128] floats = 4 KB
  float* wml = reinterpret_cast<float*>(ws.vlut);   // m[8], l[8]
  if constexpr (FMA) {
#pragma unroll
    for (int q = 0; q < 16; ++q) {
      const int d = 32 * (q >> 2) + 4 * g + (q & 3);
      wO[(2 * qd) * DD + d] = oacc[q >> 1][2 * (q & 1)];
      wO[(2 * qd + 1) * DD + d] = oacc[q >> 1][2 * (q & 1) + 1];
    }
  } else {
#pragma unroll
    for (int mt = 0; mt < 8; ++mt) {
      const int d = 16 * mt + g;
      wO[(2 * qd) * DD + d] = oacc[mt][0];
      wO[(2 * qd + 1) * DD + d] = oacc[mt][1];
      wO[(2 * qd) * DD + d + 8] = oacc[mt][2];
      wO[(2 * qd + 1) * DD + d + 8] = oacc[mt][3];
    }
  }
  if (g == 0) {
    wml[2 * qd] = m0;
    wml[2 * qd + 1] = m1;
    wml[8 + 2 * qd] = l0;
    wml[8 + 2 * qd + 1] = l1;
  }
  __syncthreads();
  // per-column warp maxima and sums, then (column, channel) sums over the warps
  if (tid < G) {
    const int c = tid;
    float M = -INFINITY;
    for (int w = 0; w < NW; ++w) M = fmaxf(M, reinterpret_cast<float*>(sm.w[w].vlut)[c]);
    const float base = M == -INFINITY ? 0.0f : M;
    float L = 0.0f;
    for (int w = 0; w < NW; ++w) {
      const float* ml = reinterpret_cast<float*>(sm.w[w].vlut);
      L += exp2f(ml[c] - base) * ml[8 + c];
    }
    sm.colM[c] = M;
    sm.colL[c] = L;
  }
  __syncthreads();
  float* mypart = p.part + ((int64_t)bh * p.n_splits + split) * PSZ;
  for (int i = tid; i < G * DD; i += NT) {
    const int c = i / DD, d = i % DD;
    const float M = sm.colM[c];
    const float base = M == -INFINITY ? 0.0f : M;
    float O = 0.0f;
    for (int w = 0; w < NW; ++w) {
      const float sc = exp2f(reinterpret_cast<float*>(sm.w[w].vlut)[c] - base);
      O += sc * reinterpret_cast<float*>(sm.w[w].raw)[c * DD + d];
    }
    mypart[c * DD + d] = O;
  }
  if (tid < G) {
    mypart[8 * DD + tid] = sm.colM[tid];
    mypart[8 * DD + 8 + tid] = sm.colL[tid];
  }
  __threadfence();
  __syncthreads();
  if (tid == 0) sm.last = (atomicAdd(&p.ctr[bh], 1u) == (uint32_t)(p.n_splits - 1));
  __syncthreads();
  if (!sm.last) return;
  __threadfence();
  // every CTA of the row is past its selection: leave the row's level-1
  // histogram zero for the next scoring
  if constexpr (FSEL)
    for (int i = tid; i < fsel::kBins; i += NT) p.fhist[(int64_t)bh * 2 * fsel::kBins + i] = 0u;

  // ---- last CTA of (b, h): merge the splits
  __syncthreads();  // every thread is past its reads of the warp buffers
  const float* parts = p.part + (int64_t)bh * p.n_splits * PSZ;
  float* wts = reinterpret_cast<float*>(sm.w);  // [n_splits][8] weights (in the warp buffers)
  float* sMv = wts + MAXSPLIT * 8;               // [n_splits][8] split maxima
  float* sLv = sMv + MAXSPLIT * 8;               // [n_splits][8] split sums
  // two threads per (column, 4 channels): even and odd splits. A thread's
  // first kPreSplits partial rows are loaded before anything else, so they
  // are in flight together with the split maxima and sums below (one round
  // trip to L2 for a merge of up to 2 kPreSplits splits)
  constexpr int kPreSplits = 16;
  const int item = tid >> 1, mhalf = tid & 1;
  const bool mactive = item < G * (DD / 4);  // G * DD / 4 <= 256 groups: one pass covers them
  const int mc = mactive ? item / (DD / 4) : 0, md4 = item % (DD / 4);
  float4 pre[kPreSplits];
#pragma unroll
  for (int u = 0; u < kPreSplits; ++u) {
    const int s = mhalf + 2 * u;
    pre[u] = (mactive && s < p.n_splits)
                 ? __ldcg(reinterpret_cast<const float4*>(parts + (int64_t)s * PSZ + mc * DD) + md4)
                 : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
  }
  for (int i = tid; i < p.n_splits * 8; i += NT) {
    const int s = i >> 3, c = i & 7;
    sMv[i] = __ldcg(parts + (int64_t)s * PSZ + 8 * DD + c);
    sLv[i] = __ldcg(parts + (int64_t)s * PSZ + 8 * DD + 8 + c);
  }
  __syncthreads();
  if (warp < G) {
    const int c = warp;
    float M = -INFINITY;
    for (int s = lane; s < p.n_splits; s += 32) M = fmaxf(M, sMv[s * 8 + c]);
#pragma unroll
    for (int o = 16; o; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
    const float base = M == -INFINITY ? 0.0f : M;
    float L = 0.0f;
    for (int s = lane; s < p.n_splits; s += 32) {
      const float w = exp2f(sMv[s * 8 + c] - base);
      wts[s * 8 + c] = w;
      L += w * sLv[s * 8 + c];
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) L += __shfl_xor_sync(0xffffffffu, L, o);
    if (lane == 0) {
      sm.colM[c] = M;
      sm.colL[c] = L;
    }
  }
  __syncthreads();
  {
    // the preloaded partials, then any splits past them eight in flight per
    // pass; one shuffle adds the halves
    const int half = mhalf, c = mc, d4 = md4;
    const bool active = mactive;
    float4 acc[2];
    acc[0] = acc[1] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    if (active) {
#pragma unroll
      for (int u = 0; u < kPreSplits; ++u) {
        const int s = half + 2 * u;
        const float w = s < p.n_splits ? wts[s * 8 + c] : 0.0f;
        acc[u & 1].x += w * pre[u].x; acc[u & 1].y += w * pre[u].y;
        acc[u & 1].z += w * pre[u].z; acc[u & 1].w += w * pre[u].w;
      }
      int s = half + 2 * kPreSplits;
      for (; s + 14 < p.n_splits; s += 16) {
        float4 v[8];
#pragma unroll
        for (int u = 0; u < 8; ++u)
          v[u] = __ldcg(reinterpret_cast<const float4*>(parts + (int64_t)(s + 2 * u) * PSZ + c * DD) + d4);
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          const float w = wts[(s + 2 * u) * 8 + c];
          acc[u & 1].x += w * v[u].x; acc[u & 1].y += w * v[u].y;
          acc[u & 1].z += w * v[u].z; acc[u & 1].w += w * v[u].w;
        }
      }
      for (; s < p.n_splits; s += 8) {  // the last up to four, loaded together
        float4 v[4];
#pragma unroll
        for (int u = 0; u < 4; ++u)
          v[u] = s + 2 * u < p.n_splits
                     ? __ldcg(reinterpret_cast<const float4*>(parts + (int64_t)(s + 2 * u) * PSZ + c * DD) + d4)
                     : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const float w = s + 2 * u < p.n_splits ? wts[(s + 2 * u) * 8 + c] : 0.0f;
          acc[u & 1].x += w * v[u].x; acc[u & 1].y += w * v[u].y;
          acc[u & 1].z += w * v[u].z; acc[u & 1].w += w * v[u].w;
        }
      }
    }
    float4 A = make_float4(acc[0].x + acc[1].x, acc[0].y + acc[1].y, acc[0].z + acc[1].z, acc[0].w + acc[1].w);
    A.x += __shfl_xor_sync(0xffffffffu, A.x, 1);
    A.y += __shfl_xor_sync(0xffffffffu, A.y, 1);
    A.z += __shfl_xor_sync(0xffffffffu, A.z, 1);
    A.w += __shfl_xor_sync(0xffffffffu, A.w, 1);
    if (active && half == 0) {
      const float L = sm.colL[c];
      const float inv = L > 0.0f ? 1.0f / L : 0.0f;
      const float4 ov = make_float4(A.x * inv, A.y * inv, A.z * inv, A.w * inv);
      const int64_t row = (int64_t)b * H * G + (int64_t)h * G + c;
      float* orow = p.o + row * DD + 4 * d4;
      if ((reinterpret_cast<uintptr_t>(p.o) & 15u) == 0) {
        *reinterpret_cast<float4*>(orow) = ov;
      } else {
        orow[0] = ov.x; orow[1] = ov.y; orow[2] = ov.z; orow[3] = ov.w;
      }
      if (p.out16) {
        uint16_t* hrow = p.out16 + row * DD + 4 * d4;
        hrow[0] = f2h(ov.x); hrow[1] = f2h(ov.y); hrow[2] = f2h(ov.z); hrow[3] = f2h(ov.w);
      }
      if (d4 == 0) {
        const float M = sm.colM[c];
        p.lse[row] = L > 0.0f ? (M + log2f(L)) * 0.6931471805599453f : -INFINITY;
      }
    }
  }
  if (tid == 0) p.ctr[bh] = 0;
}

// ---------------------------------------------------------------------------
// cross-shard merge of normalised (o, lse)

// Rank r's partials: o at o_parts + r * o_stride (N x D), lse at
// lse_parts + r * lse_stride (N).
__global__ void merge_kernel(const float* o_parts, const float* lse_parts, int64_t o_stride, int64_t lse_stride, int R,
                             int N, int D, float* o, float* lse, uint16_t* out16) {
  const int i = blockIdx.x;
  float M = -INFINITY;
  for (int r = 0; r < R; ++r) M = fmaxf(M, lse_parts[(int64_t)r * lse_stride + i]);
  const float base = M == -INFINITY ? 0.0f : M;
  float W = 0.0f;
  for (int r = 0; r < R; ++r) W += expf(lse_parts[(int64_t)r * lse_stride + i] - base);
  for (int d = threadIdx.x; d < D; d += blockDim.x) {
    float acc = 0.0f;
    for (int r = 0; r < R; ++r) {
      float w = expf(lse_parts[(int64_t)r * lse_stride + i] - base);
      if (w > 0.0f) acc += w * o_parts[(int64_t)r * o_stride + (int64_t)i * D + d];
    }
    float v = W > 0.0f ? acc / W : 0.0f;
    o[(int64_t)i * D + d] = v;
    if (out16) out16[(int64_t)i * D + d] = f2h(v);
  }
  if (threadIdx.x == 0) lse[i] = W > 0.0f ? base + logf(W) : -INFINITY;
}

// ---------------------------------------------------------------------------
// dense selected_attention (fp32 CUDA cores): one block per query head

template <typename TD>
HX_DEVINL float ldx(const TD* p, int64_t i);
template <>
HX_DEVINL float ldx<float>(const float* p, int64_t i) { return p[i]; }
template <>
HX_DEVINL float ldx<uint16_t>(const uint16_t* p, int64_t i) { return h2f(p[i]); }

template <typename TD>
__global__ void selected_attention_kernel(const TD* q, const TD* K, const TD* V, const int64_t* idx, int k, int P,
                                          int S, int H, int Hq, int D, float scale, TD* out) {
  extern __shared__ float sh[];  // per warp: o[D]; then m, l per warp
  const int i = blockIdx.x;
  const int G = Hq / H;
  const int kv = i / G;
  const int warp = threadIdx.x >> 5, lane = lane_id(), nw = blockDim.x >> 5;
  float m = -INFINITY, l = 0.0f;
  float acc[8];  // D <= 256: 8 channels per lane
#pragma unroll
  for (int v = 0; v < 8; ++v) acc[v] = 0.0f;
  const int ntok = k * S;
  for (int tt = warp; tt < ntok; tt += nw) {
    const int64_t pg = idx[(int64_t)(tt / S) * H + kv];
    if (pg < 0 || pg >= P) continue;
    const int64_t row = ((pg * S + tt % S) * H + kv) * D;
    float s = 0.0f;
#pragma unroll
    for (int v = 0; v < 8; ++v) {
      int d = lane + 32 * v;
      if (d < D) s += ldx(q, (int64_t)i * D + d) * ldx(K, row + d);
    }
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    s *= scale;
    const float mn = fmaxf(m, s);
    const float al = expf(m - mn), pw = expf(s - mn);
    l = l * al + pw;
#pragma unroll
    for (int v = 0; v < 8; ++v) {
      int d = lane + 32 * v;
      acc[v] = acc[v] * al + (d < D ? pw * ldx(V, row + d) : 0.0f);
    }
    m = mn;
  }
  float* wo = sh + warp * D;
#pragma unroll
  for (int v = 0; v < 8; ++v) {
    int d = lane + 32 * v;
    if (d < D) wo[d] = acc[v];
  }
  float* wm = sh + nw * D;
  if (lane == 0) {
    wm[warp] = m;
    wm[nw + warp] = l;
  }
  __syncthreads();
  for (int d = threadIdx.x; d < D; d += blockDim.x) {
    float M = -INFINITY;
    for (int w = 0; w < nw; ++w) M = fmaxf(M, wm[w]);
    float L = 0.0f, O = 0.0f;
    for (int w = 0; w < nw; ++w) {
      float sc = wm[w] == -INFINITY ? 0.0f : expf(wm[w] - M);
      L += sc * wm[nw + w];
      O += sc * sh[w * D + d];
    }
    float v = L > 0.0f ? O / L : 0.0f;
    if (sizeof(TD) == 4) reinterpret_cast<float*>(out)[(int64_t)i * D + d] = v;
    else reinterpret_cast<uint16_t*>(out)[(int64_t)i * D + d] = f2h(v);
  }
}

}  // namespace hx

// ===========================================================================
// C ABI

using namespace hx;

static inline cudaStream_t S_(void* s) { return reinterpret_cast<cudaStream_t>(s); }

template <int BK, int BV, bool FMA, bool FSEL>
static int launch_decode(const DecodeParams& p, int H, cudaStream_t s) {
  const size_t smem = sizeof(CtaSmem);
  // per device, once: the attribute call is idempotent, so two threads that
  // race here both set it and both store true
  static std::atomic<bool> attr_set[64];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return HX_ERR_LAUNCH;
  if (!attr_set[dev].load(std::memory_order_acquire)) {
    if (cudaFuncSetAttribute(decode_kernel<BK, BV, FMA, FSEL>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) !=
        cudaSuccess)
      return HX_ERR_LAUNCH;
    attr_set[dev].store(true, std::memory_order_release);
  }
  dim3 grid(p.n_splits, H, p.B);
  if (hx_launch_pdl(decode_kernel<BK, BV, FMA, FSEL>, grid, dim3(NT), smem, s, p) != cudaSuccess) {
    (void)cudaGetLastError();
    return HX_ERR_LAUNCH;
  }
  return HX_OK;
}

extern "C" {

// Scratch layout: a fixed region of per-(b, h) split counters first (always
// at offset 0, so counters never land where an earlier call with another
// split count wrote partials), then the split partials.
constexpr int64_t kCtrBytes = 64 * 1024;
constexpr int64_t kMaxBH = kCtrBytes / 4;

HX_API int64_t hx_decode_scratch_bytes(int32_t B, int32_t H, int32_t n_splits) {
  if (B <= 0 || H <= 0 || n_splits <= 0 || (int64_t)B * H > kMaxBH) return 0;
  int64_t parts = (int64_t)B * H * n_splits * PSZ * (int64_t)sizeof(float);
  return kCtrBytes + parts;
}

// Validate a decode request and fill the kernel parameters (scratch aside).
// Shared by hx_decode_attn and hx_decode_attn_noalloc so that both reject the
// same requests before anything is queued on the stream.
static int prepare_decode(DecodeParams& p, const hx_pool_layer* pool, const hx_layer_scales* sc, const uint16_t* q,
                          int32_t B, int32_t group, float softmax_scale, const int32_t* block_table,
                          int32_t bt_stride, const int32_t* seq_lens, int32_t page_begin, int32_t max_pages,
                          int32_t sel_mode, const float* scores, const uint64_t* thresh, int32_t sink_pages,
                          const int32_t* lists, int32_t list_stride, const int32_t* list_counts, int32_t n_splits,
                          float* o, float* lse, uint16_t* out16, uint32_t* dev_err) {
  if (!pool || !sc || !q || !seq_lens || !o || !lse) return HX_ERR_ARG;
  if (B < 0 || group <= 0 || n_splits <= 0 || n_splits > MAXSPLIT || max_pages < 0 || page_begin < 0)
    return HX_ERR_ARG;
  if (pool->num_kv_heads <= 0 || pool->num_blocks <= 0 || !pool->codes || !pool->dir || !pool->arena)
    return HX_ERR_ARG;
  if (pool->head_size != DD || pool->block_size != DS || group > 8) return HX_ERR_UNSUPPORTED;
  if ((pool->bits_k != 2 && pool->bits_k != 4) || (pool->bits_v != 2 && pool->bits_v != 4)) return HX_ERR_ARG;
  if (!sc->k_poles || !sc->v_poles) return HX_ERR_ARG;
  if (sc->levels_k < 1 || sc->levels_v < 1 || sc->levels_k > (1 << pool->bits_k) ||
      sc->levels_v > (1 << pool->bits_v) || sc->t_cal < 1)
    return HX_ERR_ARG;
  if ((sel_mode & ~(HX_SEL_MODE_MASK | HX_VPOS_PHYSICAL | HX_DECODE_CUDA_CORES)) != 0) return HX_ERR_ARG;
  const int vphys = (sel_mode & HX_VPOS_PHYSICAL) ? 1 : 0;
  const int cores = (sel_mode & HX_DECODE_CUDA_CORES) ? 1 : 0;
  sel_mode &= HX_SEL_MODE_MASK;
  if (sel_mode < 0 || sel_mode > 3) return HX_ERR_ARG;
  if (sel_mode == HX_SEL_THRESHOLD && (!scores || !thresh)) return HX_ERR_ARG;
  if (sel_mode == HX_SEL_LIST && (!lists || !list_counts || list_stride <= 0)) return HX_ERR_ARG;
  if (sel_mode == HX_SEL_SLICES && (!scores || !thresh || !lists || list_stride < 2 || list_stride > NT + 1))
    return HX_ERR_ARG;
  if (block_table && bt_stride < max_pages) return HX_ERR_ARG;
  if ((int64_t)B * pool->num_kv_heads > kMaxBH) return HX_ERR_ARG;
  p.pool = *pool;
  p.sc = *sc;
  p.q = q;
  p.B = B;
  p.G = group;
  p.scale_log2 = softmax_scale * 1.4426950408889634f;
  p.bt = block_table;
  p.bt_stride = bt_stride;
  p.seq_lens = seq_lens;
  p.page_begin = page_begin;
  p.max_pages = max_pages;
  p.sel_mode = sel_mode;
  p.vphys = vphys;
  p.cores = cores;
  p.scores = scores;
  p.thresh = thresh;
  p.sinks_req = sink_pages;
  p.lists = lists;
  p.list_stride = list_stride;
  p.list_counts = list_counts;
  p.n_splits = n_splits;
  p.o = o;
  p.lse = lse;
  p.out16 = out16;
  p.err = dev_err;
  p.ctr = nullptr;
  p.part = nullptr;
  p.fsel = 0;
  p.fhist = nullptr;
  p.k_fixed = p.fnum = p.fden = 0;
  p.thresh_out = nullptr;
  p.slice_out = nullptr;
  return HX_OK;
}

static int launch_prepared(DecodeParams& p, void* scratch, cudaStream_t s) {
  p.ctr = reinterpret_cast<uint32_t*>(scratch);
  p.part = reinterpret_cast<float*>(reinterpret_cast<char*>(scratch) + kCtrBytes);
  const int H = p.pool.num_kv_heads;
  if (p.cores && p.fsel) return HX_ERR_UNSUPPORTED;  // the CUDA-core comparison runs with the threshold kernel
  if (p.cores) {
    if (p.pool.bits_k == 4 && p.pool.bits_v == 4) return launch_decode<4, 4, true, false>(p, H, s);
    if (p.pool.bits_k == 4 && p.pool.bits_v == 2) return launch_decode<4, 2, true, false>(p, H, s);
    if (p.pool.bits_k == 2 && p.pool.bits_v == 4) return launch_decode<2, 4, true, false>(p, H, s);
    return launch_decode<2, 2, true, false>(p, H, s);
  }
  if (p.fsel) {
    if (p.pool.bits_k == 4 && p.pool.bits_v == 4) return launch_decode<4, 4, false, true>(p, H, s);
    if (p.pool.bits_k == 4 && p.pool.bits_v == 2) return launch_decode<4, 2, false, true>(p, H, s);
    if (p.pool.bits_k == 2 && p.pool.bits_v == 4) return launch_decode<2, 4, false, true>(p, H, s);
    return launch_decode<2, 2, false, true>(p, H, s);
  }
  if (p.pool.bits_k == 4 && p.pool.bits_v == 4) return launch_decode<4, 4, false, false>(p, H, s);
  if (p.pool.bits_k == 4 && p.pool.bits_v == 2) return launch_decode<4, 2, false, false>(p, H, s);
  if (p.pool.bits_k == 2 && p.pool.bits_v == 4) return launch_decode<2, 4, false, false>(p, H, s);
  return launch_decode<2, 2, false, false>(p, H, s);
}

HX_API int hx_decode_attn_select(void* stream, const hx_pool_layer* pool, const hx_layer_scales* sc,
                                 const uint16_t* q, int32_t B, int32_t group, float softmax_scale,
                                 const int32_t* block_table, int32_t bt_stride, const int32_t* seq_lens,
                                 int32_t page_begin, int32_t max_pages, int32_t flags, const float* scores,
                                 uint32_t* hist, int32_t sink_pages, int32_t k_fixed, int32_t frac_num,
                                 int32_t frac_den, int32_t n_splits, void* scratch, float* o, float* lse,
                                 uint16_t* out16, uint64_t* thresh_out, int32_t* slice_out, uint32_t* dev_err) {
  if ((flags & ~(HX_VPOS_PHYSICAL | HX_DECODE_CUDA_CORES)) != 0) return HX_ERR_ARG;
  if (!scores || !hist || k_fixed < 0 || frac_num < 0 || frac_den < 0) return HX_ERR_ARG;
  if (max_pages > fsel::kFusedMaxPages) return HX_ERR_UNSUPPORTED;
  DecodeParams p;
  const int rc = prepare_decode(p, pool, sc, q, B, group, softmax_scale, block_table, bt_stride, seq_lens, page_begin,
                                max_pages, HX_SEL_DENSE | flags, scores, nullptr, sink_pages, nullptr, 0, nullptr,
                                n_splits, o, lse, out16, dev_err);
  if (rc != HX_OK) return rc;
  if (!scratch) return HX_ERR_ARG;
  if (B == 0) return HX_OK;
  const int C = hx_quest_slices(max_pages);
  if (C < 1 || C > fsel::kMaxSlices) return HX_ERR_UNSUPPORTED;
  p.sel_mode = HX_SEL_SLICES;
  p.fsel = 1;
  p.fhist = hist;
  p.k_fixed = k_fixed;
  p.fnum = frac_num;
  p.fden = frac_den;
  p.list_stride = C + 1;
  p.thresh_out = thresh_out;
  p.slice_out = slice_out;
  return launch_prepared(p, scratch, S_(stream));
}

HX_API int hx_decode_attn(void* stream, const hx_pool_layer* pool, const hx_layer_scales* sc, const uint16_t* q,
                          int32_t B, int32_t group, float softmax_scale, const int32_t* block_table,
                          int32_t bt_stride, const int32_t* seq_lens, int32_t page_begin, int32_t max_pages,
                          int32_t sel_mode, const float* scores, const uint64_t* thresh, int32_t sink_pages,
                          const int32_t* lists, int32_t list_stride, const int32_t* list_counts, int32_t n_splits,
                          void* scratch, float* o, float* lse, uint16_t* out16, uint32_t* dev_err) {
  DecodeParams p;
  const int rc = prepare_decode(p, pool, sc, q, B, group, softmax_scale, block_table, bt_stride, seq_lens, page_begin,
                                max_pages, sel_mode, scores, thresh, sink_pages, lists, list_stride, list_counts,
                                n_splits, o, lse, out16, dev_err);
  if (rc != HX_OK) return rc;
  if (!scratch) return HX_ERR_ARG;
  if (B == 0) return HX_OK;
  return launch_prepared(p, scratch, S_(stream));
}

// ---------------------------------------------------------------------------
// Allocation-free decode: the same kernel with its scratch in a fixed device
// array of this library. For callers that cannot call cudaMalloc: a serving
// engine that reserves nearly all HBM for its own KV pool at start-up and
// allows no allocation in its decode loop, or a foreign-language binding that
// holds only raw device pointers and has no allocator to hand us a buffer
// (cudaMalloc would also synchronise the device in the middle of a step).
// Every GPU that loads this library holds the array until the process exits.

constexpr int64_t kStaticMaxSplitRows = 1024;  // B * H * n_splits at most
constexpr int64_t kStaticScratchBytes = kCtrBytes + kStaticMaxSplitRows * PSZ * (int64_t)sizeof(float);
static __device__ __align__(256) unsigned char g_decode_scratch[kStaticScratchBytes];
static std::atomic<void*> g_decode_scratch_addr[64];

// The array's device address, looked up once per device with that device
// current (host code may not use the symbol itself as a pointer). Threads
// that race on the first call each look it up and store the same address.
static int static_decode_scratch(void** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return HX_ERR_LAUNCH;
  void* addr = g_decode_scratch_addr[dev].load(std::memory_order_acquire);
  if (!addr) {
    if (cudaGetSymbolAddress(&addr, g_decode_scratch) != cudaSuccess || !addr) {
      (void)cudaGetLastError();
      return HX_ERR_LAUNCH;
    }
    g_decode_scratch_addr[dev].store(addr, std::memory_order_release);
  }
  *out = addr;
  return HX_OK;
}

HX_API int hx_decode_attn_noalloc(void* stream, const hx_pool_layer* pool, const hx_layer_scales* sc,
                                  const uint16_t* q, int32_t B, int32_t group, float softmax_scale,
                                  const int32_t* block_table, int32_t bt_stride, const int32_t* seq_lens,
                                  int32_t page_begin, int32_t max_pages, int32_t sel_mode, const float* scores,
                                  const uint64_t* thresh, int32_t sink_pages, const int32_t* lists,
                                  int32_t list_stride, const int32_t* list_counts, int32_t n_splits, float* o,
                                  float* lse, uint16_t* out16, uint32_t* dev_err) {
  // every argument is checked before anything is queued (the memset below)
  DecodeParams p;
  const int rc = prepare_decode(p, pool, sc, q, B, group, softmax_scale, block_table, bt_stride, seq_lens, page_begin,
                                max_pages, sel_mode, scores, thresh, sink_pages, lists, list_stride, list_counts,
                                n_splits, o, lse, out16, dev_err);
  if (rc != HX_OK) return rc;
  if (B == 0) return HX_OK;
  if ((int64_t)B * pool->num_kv_heads * n_splits > kStaticMaxSplitRows) return HX_ERR_SCRATCH_LIMIT;
  void* scratch = nullptr;
  const int rs = static_decode_scratch(&scratch);
  if (rs != HX_OK) return rs;
  // the array keeps the previous call's contents: the split counters must start at zero
  if (cudaMemsetAsync(scratch, 0, (size_t)B * pool->num_kv_heads * sizeof(uint32_t), S_(stream)) != cudaSuccess)
    return HX_ERR_LAUNCH;
  return launch_prepared(p, scratch, S_(stream));
}

HX_API int hx_merge_partials(void* stream, const float* o_parts, const float* lse_parts, int32_t R, int32_t N,
                             int32_t D, float* o, float* lse, uint16_t* out16) {
  if (R <= 0 || N < 0 || D <= 0) return HX_ERR_ARG;
  if (N == 0) return HX_OK;
  if (!o_parts || !lse_parts || !o || !lse) return HX_ERR_ARG;
  merge_kernel<<<N, 128, 0, S_(stream)>>>(o_parts, lse_parts, (int64_t)N * D, (int64_t)N, R, N, D, o, lse, out16);
  HX_LAUNCH_CHECK();
  return HX_OK;
}

HX_API int hx_merge_gathered(void* stream, const float* gathered, int32_t R, int32_t N, int32_t D, float* o,
                             float* lse, uint16_t* out16) {
  if (R <= 0 || N < 0 || D <= 0) return HX_ERR_ARG;
  if (N == 0) return HX_OK;
  if (!gathered || !o || !lse) return HX_ERR_ARG;
  const int64_t row = (int64_t)N * (D + 1);
  merge_kernel<<<N, 128, 0, S_(stream)>>>(gathered, gathered + (int64_t)N * D, row, row, R, N, D, o, lse, out16);
  HX_LAUNCH_CHECK();
  return HX_OK;
}

HX_API int hx_selected_attention(void* stream, int32_t dtype, const void* q, const void* k_pages,
                                 const void* v_pages, const int64_t* page_idx, int32_t k, int32_t P, int32_t S,
                                 int32_t H, int32_t Hq, int32_t D, float softmax_scale, void* out) {
  if ((dtype != 0 && dtype != 1) || k < 0 || P < 0 || S <= 0 || H <= 0 || Hq <= 0 || Hq % H != 0 || D <= 0 ||
      D > 256)
    return HX_ERR_ARG;
  if (Hq == 0) return HX_OK;
  if (!q || !out || (k > 0 && (!k_pages || !v_pages || !page_idx))) return HX_ERR_ARG;
  const int threads = 256;
  size_t smem = (size_t)(threads / 32) * D * sizeof(float) + 2 * (threads / 32) * sizeof(float);
  if (dtype == 0)
    selected_attention_kernel<float><<<Hq, threads, smem, S_(stream)>>>(
        (const float*)q, (const float*)k_pages, (const float*)v_pages, page_idx, k, P, S, H, Hq, D, softmax_scale,
        (float*)out);
  else
    selected_attention_kernel<uint16_t><<<Hq, threads, smem, S_(stream)>>>(
        (const uint16_t*)q, (const uint16_t*)k_pages, (const uint16_t*)v_pages, page_idx, k, P, S, H, Hq, D,
        softmax_scale, (uint16_t*)out);
  HX_LAUNCH_CHECK();
  return HX_OK;
}

}  // extern "C"
