// Split-KV exchange over peer memory: one kernel per layer that signals this
// rank's partials, waits for every rank's, and merges them read straight from
// the peers' buffers over NVLink (plain loads; no multicast, no library copy).
//
// Each rank owns a symmetric buffer of per-layer rows [o (N x D) | lse (N)]
// fp32 (its decode writes row `slot` of its own buffer) and a symmetric array
// of flags, R per layer slot: flag (slot, r) of rank q is set by rank r when
// its row `slot` is complete. The kernel of rank `rank` for slot `slot`:
//   1. sets flag (slot, rank) in every rank's array (release, system scope;
//      the decode that wrote the row finished earlier in the stream);
//   2. waits until all R flags (slot, *) of its own array are set (acquire,
//      system scope; bounded: after max_polls it flags HX_DEV_ERR_TIMEOUT and
//      returns without merging);
//   3. merges the R rows: o = sum_r exp(lse_r - M) o_r / sum_r exp(lse_r - M);
//   4. clears its own flags (slot, *).
// A flag is never set again before it is cleared: rank r sets (slot, r) for
// the next step only after it has seen every rank's flags of the last slot of
// this step, and each rank clears (slot, *) before it sets its own last-slot
// flags. No counter has to advance per step, so the kernels replay as a CUDA
// graph unchanged.
#include "common.cuh"

namespace hx {

HX_DEVINL void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
HX_DEVINL uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

constexpr int XM_THREADS = 1024;

__global__ void __launch_bounds__(XM_THREADS) exchange_merge_kernel(
    const uint64_t* __restrict__ peer_rows, const uint64_t* __restrict__ peer_flags, int R, int rank, int slot, int N,
    int D, float* o, float* lse, uint16_t* out16, uint32_t max_polls, uint32_t* err) {
  __shared__ float s_w[64][32];  // per query row and rank: merge weights (R <= 32, N <= 64)
  __shared__ float s_inv[64];
  __shared__ int s_ok;
  const int tid = threadIdx.x;
  const int64_t row = (int64_t)N * (D + 1);
  uint32_t* my_flags = reinterpret_cast<uint32_t*>(peer_flags[rank]) + (int64_t)slot * R;
  // 1. this rank's row is complete: tell every rank
  if (tid < R) {
    __threadfence_system();
    st_release_sys(reinterpret_cast<uint32_t*>(peer_flags[tid]) + (int64_t)slot * R + rank, 1u);
  }
  // 2. wait for every rank's (bounded)
  bool ok = true;
  if (tid < R) {
    uint32_t it = 0;
    while (ld_acquire_sys(my_flags + tid) == 0u) {
      if (++it >= max_polls) {
        ok = false;
        break;
      }
      __nanosleep(128);
    }
  }
  if (tid == 0) s_ok = 1;
  __syncthreads();
  if (!ok) atomicAnd(&s_ok, 0);
  __syncthreads();
  if (!s_ok) {
    if (tid == 0) set_err(err, HX_DEV_ERR_TIMEOUT);
    return;
  }
  // 3. merge weights per query row, then the rows
  for (int i = tid; i < N; i += XM_THREADS) {
    float M = -INFINITY;
    for (int r = 0; r < R; ++r) {
      const float* rr = reinterpret_cast<const float*>(peer_rows[r]) + (int64_t)slot * row + (int64_t)N * D;
      M = fmaxf(M, __ldcv(rr + i));
    }
    const float base = M == -INFINITY ? 0.0f : M;
    float W = 0.0f;
    for (int r = 0; r < R; ++r) {
      const float* rr = reinterpret_cast<const float*>(peer_rows[r]) + (int64_t)slot * row + (int64_t)N * D;
      const float l = __ldcv(rr + i);
      const float w = l == -INFINITY ? 0.0f : expf(l - base);
      s_w[i][r] = w;
      W += w;
    }
    s_inv[i] = W > 0.0f ? 1.0f / W : 0.0f;
    lse[i] = W > 0.0f ? base + logf(W) : -INFINITY;
  }
  __syncthreads();
  for (int e = tid; e < N * D; e += XM_THREADS) {
    const int i = e / D;
    float acc = 0.0f;
    for (int r = 0; r < R; ++r) {
      const float w = s_w[i][r];
      if (w > 0.0f) acc += w * __ldcv(reinterpret_cast<const float*>(peer_rows[r]) + (int64_t)slot * row + e);
    }
    const float v = acc * s_inv[i];
    o[e] = v;
    if (out16) out16[e] = f2h(v);
  }
  // 4. this slot's flags are consumed
  __syncthreads();
  if (tid < R) my_flags[tid] = 0u;
}

}  // namespace hx

using namespace hx;

extern "C" {

HX_API int hx_exchange_merge(void* stream, const uint64_t* peer_rows, const uint64_t* peer_flags, int32_t R,
                             int32_t rank, int32_t slot, int32_t N, int32_t D, float* o, float* lse,
                             uint16_t* out16, uint32_t max_polls, uint32_t* dev_err) {
  if (!peer_rows || !peer_flags || !o || !lse || R < 1 || R > 32 || rank < 0 || rank >= R || slot < 0 || N < 1 ||
      N > 64 || D < 1 || max_polls == 0)
    return HX_ERR_ARG;
  exchange_merge_kernel<<<1, XM_THREADS, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      peer_rows, peer_flags, R, rank, slot, N, D, o, lse, out16, max_polls, dev_err);
  HX_LAUNCH_CHECK();
  return HX_OK;
}

}  // extern "C"
