// Chunked-prefill attention over the compact pool.
//
// The reference's prefill reads vLLM's fp16 KV cache (it keeps that cache
// beside the compact pool: src/kvquant/compact_backend.py:12-15, :137-167),
// so the fp16 pool cannot go. Here a prefill chunk's queries attend every
// earlier token, and the chunk's own tokens causally, straight from the
// packed pages (the chunk is packed by hx_pack_append before the call):
// softmax(q . K^T * scale) V with K, V dequantised on chip exactly as
// hx_unpack_pages / dequantize_nuq do (src/kvquant/nuq.py:135-156,
// compact_pool.py:293-395), fp32 softmax (src/quest/reference.py:136-168),
// query head h*G+g on KV head h.
//
// One CTA = (tile of 64 query rows, KV head, sequence); a row is one (query
// token, head of the group) pair. Four warps: each dequantises one page of a
// group of four into swizzled smem tiles (K and V, outliers patched), then
// every warp runs its 16 rows over the 64 keys: S = Q K^T and O += P V with
// mma.sync m16n8k16 (ldmatrix from the tiles), online softmax in fp32 (exp2
// domain), P as fp16 hi + lo parts (two MMAs per PV tile).
#include "common.cuh"

namespace hx {

namespace pf {

constexpr int D = 128;      // head_size
constexpr int S = 16;       // page size
constexpr int NWP = 4;      // warps = pages per group
constexpr int ROWS = 16 * NWP;

struct Smem {
  alignas(256) uint16_t ktile[NWP][S * D];  // swizzled: chunk c of token t at 16 (c ^ (t & 7) ^ 4 (c >> 3))
  alignas(256) uint16_t vtile[NWP][S * D];
  uint16_t klut[D * 16];                    // K level c of channel d at 16 d + c (c >= levels: level 0)
  uint16_t vlev[NWP][S * 16];               // V levels of each token of the warp's page
};

HX_DEVINL uint32_t tile_off(int t, int c) { return 256u * t + 16u * (uint32_t)(c ^ (t & 7) ^ (4 * (c >> 3))); }

HX_DEVINL void ldsm4(uint32_t (&r)[4], uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
HX_DEVINL void ldsm4t(uint32_t (&r)[4], uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}

// code of channel d in a packed row (nuq4: nibble d of the row, low first;
// nuq2: crumb d)
template <int BITS>
HX_DEVINL uint32_t code_of(const uint32_t (&w)[BITS * 2], int i) {
  // w holds the lane's 64 channels: BITS * 2 words of 32 bits
  constexpr int PER = 32 / BITS;
  return (w[i / PER] >> (BITS * (i % PER))) & ((1u << BITS) - 1u);
}

// The warp's page into its tiles: token t = lane >> 1, channels 64 half ..
// 64 half + 63 (half = lane & 1). Then the page's outlier entries.
template <int BK, int BV>
HX_DEVINL void dequant_page(const hx_pool_layer& pool, const hx_layer_scales& sc, int h, int pp, int vpos0,
                            Smem& sm, int w, uint32_t* err) {
  const int lane = lane_id(), t = lane >> 1, half = lane & 1;
  const int NB = pool.num_blocks;
  constexpr int RBK = D * BK / 8, RBV = D * BV / 8;
  const uint8_t* seg = pool.codes + ((int64_t)h * NB + pp) * (int64_t)(S * (RBK + RBV));
  // V level rows of the page's tokens (row min(pos, t_cal - 1); levels >= L read level 0)
  {
    const int Tc = sc.t_cal, L = sc.levels_v;
    for (int i = lane; i < S * 16; i += 32) {
      const int tt = i >> 4, c = i & 15;
      const int64_t pos = (int64_t)vpos0 + tt;
      const int row = (int)(pos < Tc ? pos : Tc - 1);
      sm.vlev[w][i] = sc.v_poles[((int64_t)h * Tc + row) * L + (c < L ? c : 0)];
    }
  }
  uint32_t kw[BK * 2], vw[BV * 2];
  {
    const uint4* kr = reinterpret_cast<const uint4*>(seg + t * RBK + half * (RBK / 2));
    const uint4* vr = reinterpret_cast<const uint4*>(seg + S * RBK + t * RBV + half * (RBV / 2));
#pragma unroll
    for (int u = 0; u < BK / 2; ++u) {
      const uint4 x = __ldg(kr + u);
      kw[4 * u] = x.x;
      kw[4 * u + 1] = x.y;
      kw[4 * u + 2] = x.z;
      kw[4 * u + 3] = x.w;
    }
#pragma unroll
    for (int u = 0; u < BV / 2; ++u) {
      const uint4 x = __ldg(vr + u);
      vw[4 * u] = x.x;
      vw[4 * u + 1] = x.y;
      vw[4 * u + 2] = x.z;
      vw[4 * u + 3] = x.w;
    }
  }
  __syncwarp();
  const uint32_t kt = smem_u32(sm.ktile[w]), vt = smem_u32(sm.vtile[w]);
#pragma unroll
  for (int k = 0; k < 8; ++k) {  // chunk 8 half + k: channels 64 half + 8 k .. + 7
    uint32_t ko[4], vo[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int i0 = 8 * k + 2 * e, d0 = 64 * half + i0;
      const uint16_t k0 = sm.klut[16 * d0 + code_of<BK>(kw, i0)];
      const uint16_t k1 = sm.klut[16 * (d0 + 1) + code_of<BK>(kw, i0 + 1)];
      const uint16_t v0 = sm.vlev[w][16 * t + code_of<BV>(vw, i0)];
      const uint16_t v1 = sm.vlev[w][16 * t + code_of<BV>(vw, i0 + 1)];
      ko[e] = pack_u16x2(k0, k1);
      vo[e] = pack_u16x2(v0, v1);
    }
    const uint32_t off = tile_off(t, 8 * half + k);
    asm volatile("st.shared.v4.u32 [%0], {%1,%2,%3,%4};" ::"r"(kt + off), "r"(ko[0]), "r"(ko[1]), "r"(ko[2]),
                 "r"(ko[3])
                 : "memory");
    asm volatile("st.shared.v4.u32 [%0], {%1,%2,%3,%4};" ::"r"(vt + off), "r"(vo[0]), "r"(vo[1]), "r"(vo[2]),
                 "r"(vo[3])
                 : "memory");
  }
  __syncwarp();
  // outliers: entry = fp16 value | channel << 16 | slot << 24
  for (int kv = 0; kv < 2; ++kv) {
    const uint32_t* dr = pool.dir + (((int64_t)h * NB + pp) * 2 + kv) * 4;
    const uint32_t off = dr[0], cap = dr[1], cnt = dr[2];
    if (cnt > cap || (int64_t)off + cnt > pool.arena_capacity) {
      if (lane == 0) set_err(err, HX_DEV_ERR_BOUNDS);
      continue;
    }
    uint16_t* tile = kv ? sm.vtile[w] : sm.ktile[w];
    for (uint32_t i = lane; i < cnt; i += 32) {
      const uint32_t e = __ldg(pool.arena + off + i);
      const int tt = (e >> 24) & 31, d = (e >> 16) & 255;
      if (tt < S && d < D) tile[(tile_off(tt, d >> 3) >> 1) + (d & 7)] = (uint16_t)(e & 0xffffu);
      else set_err(err, HX_DEV_ERR_BOUNDS);
    }
  }
}

struct PrefillParams {
  hx_pool_layer pool;
  hx_layer_scales sc;
  const uint16_t* q;
  const int32_t* q_start;
  int G;
  float scale_log2;
  const int32_t* bt;
  int bt_stride;
  const int32_t* seq_lens;
  int vphys;
  float* lse;
  uint16_t* out16;
  float* out32;
  uint32_t* err;
};

template <int BK, int BV>
__global__ void __launch_bounds__(NWP * 32) prefill_kernel(const PrefillParams p) {
  __shared__ Smem sm;
  const int tile = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int H = p.pool.num_kv_heads, G = p.G, Hq = H * G;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, qd = lane & 3;
  const int q0 = p.q_start[b], qn = p.q_start[b + 1] - q0;
  const int seq = p.seq_lens[b];
  const int rows = qn * G;
  if (tile * ROWS >= rows || qn <= 0) return;
  if (qn > seq) {  // the chunk must be in the pool already
    if (threadIdx.x == 0) set_err(p.err, HX_DEV_ERR_BOUNDS);
    return;
  }
  const int first = seq - qn;  // absolute position of the chunk's first token

  // K level table of head h
  for (int i = threadIdx.x; i < D * 16; i += blockDim.x) {
    const int d = i >> 4, c = i & 15, L = p.sc.levels_k;
    sm.klut[i] = p.sc.k_poles[((int64_t)h * D + d) * L + (c < L ? c : 0)];
  }

  // this warp's rows: r = tile * 64 + 16 warp + {g, g + 8}
  const int ra = tile * ROWS + 16 * warp + g, rb = ra + 8;
  const int ta = ra / G, tb = rb / G;  // query tokens (chunk index)
  const int posa = first + ta, posb = first + tb;
  // Q fragments (A operand, rows x channels): a[ks] = {(g, 16ks + 2qd), (g + 8, ..), (g, +8), (g + 8, +8)}
  uint32_t qa[8][4];
  {
    const bool va = ra < rows, vb = rb < rows;
    const uint16_t* qra = p.q + ((int64_t)(q0 + (va ? ta : 0)) * Hq + h * G + ra % G) * D;
    const uint16_t* qrb = p.q + ((int64_t)(q0 + (vb ? tb : 0)) * Hq + h * G + rb % G) * D;
#pragma unroll
    for (int ks = 0; ks < 8; ++ks) {
      const int c = 16 * ks + 2 * qd;
      qa[ks][0] = va ? *reinterpret_cast<const uint32_t*>(qra + c) : 0u;
      qa[ks][1] = vb ? *reinterpret_cast<const uint32_t*>(qrb + c) : 0u;
      qa[ks][2] = va ? *reinterpret_cast<const uint32_t*>(qra + c + 8) : 0u;
      qa[ks][3] = vb ? *reinterpret_cast<const uint32_t*>(qrb + c + 8) : 0u;
    }
  }
  float o[16][4];
#pragma unroll
  for (int nt = 0; nt < 16; ++nt) o[nt][0] = o[nt][1] = o[nt][2] = o[nt][3] = 0.0f;
  float ma = -INFINITY, mb = -INFINITY, la = 0.0f, lb = 0.0f;

  // keys needed by the tile: up to the position of its last valid row
  const int last_row = min(rows, (tile + 1) * ROWS) - 1;
  const int pos_max = first + last_row / G;
  const int n_pages = pos_max / S + 1;
  const int NB = p.pool.num_blocks;

  for (int j0 = 0; j0 < n_pages; j0 += NWP) {
    __syncthreads();  // the tiles are free (and klut written, the first time)
    {
      const int j = j0 + warp;
      if (j < n_pages) {
        const int pp = j < p.bt_stride ? p.bt[(int64_t)b * p.bt_stride + j] : -1;
        if (pp < 0 || pp >= NB) {
          if (lane == 0) set_err(p.err, HX_DEV_ERR_BOUNDS);
        } else {
          const int vpos0 = (p.vphys ? pp : j) * S;
          dequant_page<BK, BV>(p.pool, p.sc, h, pp, vpos0, sm, warp, p.err);
        }
      }
    }
    __syncthreads();
    const int np = min(NWP, n_pages - j0);
    for (int u = 0; u < np; ++u) {
      const int kbase = (j0 + u) * S;  // position of the page's first key
      const uint32_t kt = smem_u32(sm.ktile[u]), vt = smem_u32(sm.vtile[u]);
      // ---- S = Q K^T (16 rows x 16 keys)
      float s[2][4] = {{0.0f, 0.0f, 0.0f, 0.0f}, {0.0f, 0.0f, 0.0f, 0.0f}};
#pragma unroll
      for (int ks = 0; ks < 8; ++ks) {
        uint32_t kb[4];  // (keys 0-7, ch lo), (keys 0-7, ch hi), (keys 8-15, ch lo), (keys 8-15, ch hi)
        const int mi = lane >> 3, key = (mi >> 1) * 8 + (lane & 7);
        ldsm4(kb, kt + tile_off(key, 2 * ks + (mi & 1)));
        mma_16816(s[0], qa[ks], kb[0], kb[1]);
        mma_16816(s[1], qa[ks], kb[2], kb[3]);
      }
      // ---- causal mask, online softmax (rows g: c0 c1, row g + 8: c2 c3)
      float x[2][4];
#pragma unroll
      for (int nt = 0; nt < 2; ++nt) {
        const int k0 = kbase + 8 * nt + 2 * qd;
        x[nt][0] = (k0 <= posa) ? s[nt][0] * p.scale_log2 : -INFINITY;
        x[nt][1] = (k0 + 1 <= posa) ? s[nt][1] * p.scale_log2 : -INFINITY;
        x[nt][2] = (k0 <= posb) ? s[nt][2] * p.scale_log2 : -INFINITY;
        x[nt][3] = (k0 + 1 <= posb) ? s[nt][3] * p.scale_log2 : -INFINITY;
      }
      float mxa = fmaxf(fmaxf(x[0][0], x[0][1]), fmaxf(x[1][0], x[1][1]));
      float mxb = fmaxf(fmaxf(x[0][2], x[0][3]), fmaxf(x[1][2], x[1][3]));
      mxa = fmaxf(mxa, __shfl_xor_sync(0xffffffffu, mxa, 1));
      mxa = fmaxf(mxa, __shfl_xor_sync(0xffffffffu, mxa, 2));
      mxb = fmaxf(mxb, __shfl_xor_sync(0xffffffffu, mxb, 1));
      mxb = fmaxf(mxb, __shfl_xor_sync(0xffffffffu, mxb, 2));
      const float mna = fmaxf(ma, mxa), mnb = fmaxf(mb, mxb);
      const float ala = mna == -INFINITY ? 1.0f : exp2f(ma - mna);
      const float alb = mnb == -INFINITY ? 1.0f : exp2f(mb - mnb);
      ma = mna;
      mb = mnb;
      const float bsa = ma == -INFINITY ? 0.0f : ma, bsb = mb == -INFINITY ? 0.0f : mb;
      float pr[2][4];
#pragma unroll
      for (int nt = 0; nt < 2; ++nt) {
        pr[nt][0] = exp2f(x[nt][0] - bsa);
        pr[nt][1] = exp2f(x[nt][1] - bsa);
        pr[nt][2] = exp2f(x[nt][2] - bsb);
        pr[nt][3] = exp2f(x[nt][3] - bsb);
      }
      la = la * ala + (pr[0][0] + pr[0][1] + pr[1][0] + pr[1][1]);
      lb = lb * alb + (pr[0][2] + pr[0][3] + pr[1][2] + pr[1][3]);
#pragma unroll
      for (int nt = 0; nt < 16; ++nt) {
        o[nt][0] *= ala;
        o[nt][1] *= ala;
        o[nt][2] *= alb;
        o[nt][3] *= alb;
      }
      // P as the A operand (rows x keys): {(g, 2qd), (g + 8, 2qd), (g, 8 + 2qd), (g + 8, 8 + 2qd)},
      // split into fp16 hi + lo parts so that P V keeps ~22 bits of P
      uint32_t pa[4], pl[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float u0 = pr[e >> 1][2 * (e & 1)], u1 = pr[e >> 1][2 * (e & 1) + 1];
        const __half2 hi = __floats2half2_rn(u0, u1);
        const float2 hf = __half22float2(hi);
        pa[e] = *reinterpret_cast<const uint32_t*>(&hi);
        pl[e] = pack_half2(u0 - hf.x, u1 - hf.y);
      }
      // ---- O += P V (16 rows x 128 channels): V^T fragments by transposed ldmatrix
#pragma unroll
      for (int np2 = 0; np2 < 8; ++np2) {
        uint32_t vb[4];  // (keys 0-7, chunk 2 np2), (keys 8-15, ..), (keys 0-7, chunk 2 np2 + 1), (keys 8-15, ..)
        const int mi = lane >> 3, key = (mi & 1) * 8 + (lane & 7);
        ldsm4t(vb, vt + tile_off(key, 2 * np2 + (mi >> 1)));
        mma_16816(o[2 * np2], pa, vb[0], vb[1]);
        mma_16816(o[2 * np2], pl, vb[0], vb[1]);
        mma_16816(o[2 * np2 + 1], pa, vb[2], vb[3]);
        mma_16816(o[2 * np2 + 1], pl, vb[2], vb[3]);
      }
    }
  }

  // ---- normalise and write: row sums over the quad, then channels 8 nt + 2 qd
  la += __shfl_xor_sync(0xffffffffu, la, 1);
  la += __shfl_xor_sync(0xffffffffu, la, 2);
  lb += __shfl_xor_sync(0xffffffffu, lb, 1);
  lb += __shfl_xor_sync(0xffffffffu, lb, 2);
  const float ia = la > 0.0f ? 1.0f / la : 0.0f, ib = lb > 0.0f ? 1.0f / lb : 0.0f;
  const bool va = ra < rows, vb = rb < rows;
  uint16_t* oa = p.out16 + ((int64_t)(q0 + ta) * Hq + h * G + ra % G) * D;
  uint16_t* ob = p.out16 + ((int64_t)(q0 + tb) * Hq + h * G + rb % G) * D;
#pragma unroll
  for (int nt = 0; nt < 16; ++nt) {
    const int c = 8 * nt + 2 * qd;
    if (va) *reinterpret_cast<uint32_t*>(oa + c) = pack_half2(o[nt][0] * ia, o[nt][1] * ia);
    if (vb) *reinterpret_cast<uint32_t*>(ob + c) = pack_half2(o[nt][2] * ib, o[nt][3] * ib);
  }
  if (p.out32) {
    float* fa = p.out32 + ((int64_t)(q0 + ta) * Hq + h * G + ra % G) * D;
    float* fb = p.out32 + ((int64_t)(q0 + tb) * Hq + h * G + rb % G) * D;
#pragma unroll
    for (int nt = 0; nt < 16; ++nt) {
      const int c = 8 * nt + 2 * qd;
      if (va) *reinterpret_cast<float2*>(fa + c) = make_float2(o[nt][0] * ia, o[nt][1] * ia);
      if (vb) *reinterpret_cast<float2*>(fb + c) = make_float2(o[nt][2] * ib, o[nt][3] * ib);
    }
  }
  if (p.lse && qd == 0) {
    constexpr float kLn2 = 0.6931471805599453f;
    if (va) p.lse[(int64_t)(q0 + ta) * Hq + h * G + ra % G] = la > 0.0f ? (ma + log2f(la)) * kLn2 : -INFINITY;
    if (vb) p.lse[(int64_t)(q0 + tb) * Hq + h * G + rb % G] = lb > 0.0f ? (mb + log2f(lb)) * kLn2 : -INFINITY;
  }
}

}  // namespace pf
}  // namespace hx

using namespace hx;

extern "C" {

HX_API int hx_prefill_attn(void* stream, const hx_pool_layer* pool, const hx_layer_scales* sc, const uint16_t* q,
                           const int32_t* q_start, int32_t B, int32_t group, float softmax_scale,
                           const int32_t* block_table, int32_t bt_stride, const int32_t* seq_lens,
                           int32_t max_q_len, int32_t flags, uint16_t* out16, float* out32, float* lse,
                           uint32_t* dev_err) {
  if (!pool || !sc || B < 0 || group < 1 || max_q_len < 0 || bt_stride < 1) return HX_ERR_ARG;
  if ((flags & ~HX_VPOS_PHYSICAL) != 0) return HX_ERR_ARG;
  if (B == 0 || max_q_len == 0) return HX_OK;
  if (!q || !q_start || !block_table || !seq_lens || !out16) return HX_ERR_ARG;
  if (pool->head_size != pf::D || pool->block_size != pf::S) return HX_ERR_UNSUPPORTED;
  if ((pool->bits_k != 2 && pool->bits_k != 4) || (pool->bits_v != 2 && pool->bits_v != 4)) return HX_ERR_UNSUPPORTED;
  if (sc->levels_k < 1 || sc->levels_k > 16 || sc->levels_v < 1 || sc->levels_v > 16 || sc->t_cal < 1)
    return HX_ERR_ARG;
  if (B > 65535 || pool->num_kv_heads > 65535) return HX_ERR_UNSUPPORTED;
  pf::PrefillParams p;
  p.pool = *pool;
  p.sc = *sc;
  p.q = q;
  p.q_start = q_start;
  p.G = group;
  p.scale_log2 = softmax_scale * 1.4426950408889634f;
  p.bt = block_table;
  p.bt_stride = bt_stride;
  p.seq_lens = seq_lens;
  p.vphys = (flags & HX_VPOS_PHYSICAL) ? 1 : 0;
  p.lse = lse;
  p.out16 = out16;
  p.out32 = out32;
  p.err = dev_err;
  const int64_t tiles = ((int64_t)max_q_len * group + pf::ROWS - 1) / pf::ROWS;
  if (tiles > 2147483647ll) return HX_ERR_UNSUPPORTED;
  dim3 grid((unsigned)tiles, pool->num_kv_heads, B);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (pool->bits_k == 4 && pool->bits_v == 4) pf::prefill_kernel<4, 4><<<grid, pf::NWP * 32, 0, s>>>(p);
  else if (pool->bits_k == 4) pf::prefill_kernel<4, 2><<<grid, pf::NWP * 32, 0, s>>>(p);
  else if (pool->bits_v == 4) pf::prefill_kernel<2, 4><<<grid, pf::NWP * 32, 0, s>>>(p);
  else pf::prefill_kernel<2, 2><<<grid, pf::NWP * 32, 0, s>>>(p);
  HX_LAUNCH_CHECK();
  return HX_OK;
}

}  // extern "C"
