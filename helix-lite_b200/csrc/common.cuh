// Shared device helpers for the helix KV kernels (sm_100a).
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "helix_kv.h"

#define HX_DEVINL __device__ __forceinline__

namespace hx {

constexpr int WARP = 32;
// Upper bound on polls of one mbarrier phase before a wait gives up
// (try_wait itself suspends for a while per poll, so this is seconds).
constexpr uint32_t kMaxPolls = 1u << 22;

HX_DEVINL void set_err(uint32_t* err, uint32_t bits) {
  if (err) atomicOr(err, bits);
}

HX_DEVINL float h2f(uint16_t b) { return __half2float(__ushort_as_half(b)); }
HX_DEVINL uint16_t f2h(float f) { return __half_as_ushort(__float2half_rn(f)); }

// Order-preserving map of an fp32 score to uint32: larger key = larger score.
// -0 is folded onto +0 and NaN maps to 0, the lowest key.
HX_DEVINL uint32_t order_key(float s) {
  s = __fadd_rn(s, 0.0f);
  if (s != s) return 0u;
  uint32_t u = __float_as_uint(s);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

HX_DEVINL uint64_t order_key64(float s, uint32_t page) {
  return ((uint64_t)order_key(s) << 32) | (uint64_t)(~page);
}

HX_DEVINL uint32_t lane_id() { return threadIdx.x & 31; }

// ---- shared-memory address / async-proxy helpers --------------------------

HX_DEVINL uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

HX_DEVINL void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

HX_DEVINL void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

HX_DEVINL void fence_proxy_async() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

HX_DEVINL void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

// Bulk (non-tensor) TMA copy global -> shared, completing on an mbarrier.
// dst and src 16-byte aligned, bytes a multiple of 16. No multicast.
HX_DEVINL void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// Bounded wait for phase `parity` of an mbarrier. Returns false on timeout.
HX_DEVINL bool mbar_wait(uint64_t* bar, uint32_t parity) {
  uint32_t addr = smem_u32(bar);
  for (uint32_t i = 0; i < kMaxPolls; ++i) {
    uint32_t done;
    asm volatile(
        "{\n .reg .pred p;\n"
        " mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
        " selp.u32 %0, 1, 0, p;\n}"
        : "=r"(done)
        : "r"(addr), "r"(parity)
        : "memory");
    if (done) return true;
  }
  return false;
}

// ---- tensor-core fragments (mma.sync m16n8k16, f16 -> f32) ----------------

HX_DEVINL void ldmatrix_x4(uint32_t (&r)[4], const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(smem_u32(p)));
}

HX_DEVINL void ldmatrix_x4_trans(uint32_t (&r)[4], const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(smem_u32(p)));
}

HX_DEVINL void mma_16816(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// Transpose an 8x8 b16 fragment held one row pair per lane.
HX_DEVINL uint32_t movmatrix_trans(uint32_t x) {
  uint32_t y;
  asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(y) : "r"(x));
  return y;
}

HX_DEVINL uint32_t pack_half2(float lo, float hi) {
  __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}

HX_DEVINL uint32_t pack_u16x2(uint16_t lo, uint16_t hi) {
  return (uint32_t)lo | ((uint32_t)hi << 16);
}

// ---- programmatic dependent launch ------------------------------------------
// The step's kernels are launched so that the next one may start while this
// one runs: pdl_allow_next() lets the next grid launch once every CTA of this
// one has called it (or exited); pdl_wait() blocks until the previous grid in
// the stream has completed and its writes are visible. Work before pdl_wait()
// may touch only data no earlier kernel writes (this CTA's smem, calibration
// tables). Both are no-ops for a grid launched without the attribute.
HX_DEVINL void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
HX_DEVINL void pdl_allow_next() { asm volatile("griddepcontrol.launch_dependents;" :::); }

}  // namespace hx

// Launch with programmatic stream serialisation (see pdl_wait).
template <typename... KArgs, typename... Args>
static inline cudaError_t hx_launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                                        Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, args...);
}

// Bandwidth path of hx_pack_append (pack_fast.cu): HX_ERR_UNSUPPORTED when
// the request does not fit it (page size, head size, missing thresholds).
int hx_pack_fast_launch(cudaStream_t s, const hx_pool_layer* pool, const hx_layer_scales* sc, const uint16_t* key,
                        const uint16_t* value, const int64_t* slots, const int64_t* abspos, int32_t T,
                        uint32_t* dev_err);

// Host-side launch check shared by the C entry points.
#define HX_LAUNCH_CHECK()                                   \
  do {                                                      \
    if (cudaPeekAtLastError() != cudaSuccess) {             \
      (void)cudaGetLastError();                             \
      return HX_ERR_LAUNCH;                                 \
    }                                                       \
  } while (0)
